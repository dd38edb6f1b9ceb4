"""DSpark draft + verify attention benchmark on B200 (see BASELINE.json `metric`).

One step = one speculative round's attention on one GPU:
  * draft (config 2): 64 requests, context ~ U[128, 4096] (seed 1), one 7-row block
    each, non-causal attention for each of the 5 draft layers (B200DraftKernel);
  * verify (config 3): 128 requests, cached context ~ U[256, 8192] (seed 2), 7 new
    tokens each; for each of 28 layers the fused QK-norm + RoPE(1e6) + KV append +
    bottom-right attention (B200PersistentTargetKV.verify_layer), then one commit of
    the accepted prefixes (accept ~ U{0..6} + anchor) and rollback of the rest.
Metric: query-token-layers per second = (64*7*5 + 128*7*28) / step time, summed
over ranks (weak scaling: every rank runs its own full batch: the same context lengths,
K/V values seeded by rank).

    python bench.py [--gpus N --steps K --warmup W] [--impl reference]
                    [--case round|draft|verify] [--layers L]

``--case``/``--layers`` select a smaller workload (one path, fewer layers) for
profiler captures; the default is the full round the metric is quoted on.
``--case train`` measures config 4 (training-layout draft attention) alone;
``--case graph`` compares an eager and a CUDA-graph-replayed verify step at a small
serving batch; ``--case accept`` times the on-device greedy acceptance of one round;
``--case markov`` the fused greedy Markov proposal of one draft block; ``--case round5``
the full greedy speculative loop of config 5 on a Qwen3-0.6B-shaped model.

Multi-GPU: launched by torchrun, one rank per GPU; ranks share nothing on the data
path; one NCCL all_gather of per-rank stats after timing.
"""
import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, 'tests', 'golden'))

HQ, HKV, D, BLOCK = 16, 8, 128, 7
KV_ROW = 2 * HKV * D * 2             # bytes of one token's K+V for one layer (bf16)
Q_ROW = HQ * D * 2                   # bytes of one query row (bf16)
DRAFT = dict(requests=64, ctx_lo=128, ctx_hi=4096, seed=1, layers=5)
VERIFY = dict(requests=128, ctx_lo=256, ctx_hi=8192, seed=2, layers=28, q=7)
METRIC = 'draft+verify attn query-tok/s per GPU & at 1/2/4/8 B200; % of HBM roofline'
FALLBACK_HBM_GBS = 6650.0
FALLBACK_TFLOPS = 1590.0
TRAIN = dict(seqs=8, ctx=2048, anchors=32, seed=3)


def peaks():
    try:
        with open(os.path.join(ROOT, 'MEASURED_PEAKS.json')) as f:
            p = json.load(f)
        return float(p['hbm_gbs']), 'measured'
    except Exception:
        return FALLBACK_HBM_GBS, 'fallback'


def tensor_peak():
    """Dense bf16 TFLOP/s (burst: a kernel timed alone)."""
    try:
        with open(os.path.join(ROOT, 'MEASURED_PEAKS.json')) as f:
            return float(json.load(f)['bf16_tflops']), 'measured'
    except Exception:
        return FALLBACK_TFLOPS, 'fallback'


def _finite(obj):
    """JSON has no NaN/Inf: report unmeasured numbers as null."""
    if isinstance(obj, float):
        return obj if obj == obj and abs(obj) != float('inf') else None
    if isinstance(obj, dict):
        return {k: _finite(v) for k, v in obj.items()}
    if isinstance(obj, (list, tuple)):
        return [_finite(v) for v in obj]
    return obj


def captured_traffic(key):
    """DRAM bytes per launch from the committed ncu capture summary, or None."""
    try:
        with open(os.path.join(ROOT, 'profiles', 'ncu_traffic.json')) as f:
            return int(json.load(f)[key]['bytes'])
    except Exception:
        return None


def dist_env():
    return int(os.environ.get('RANK', 0)), int(os.environ.get('WORLD_SIZE', 1)), int(os.environ.get('LOCAL_RANK', 0))


def contexts(cfg):
    """The config's context lengths: ``requests`` draws of U{ctx_lo..ctx_hi} from numpy's
    PCG64 seeded with the config's seed. Every rank uses the same lengths (its K/V
    values differ), so each rank streams the same bytes and the 1 -> N curve measures
    the hardware, not the draw."""
    import numpy as np
    g = np.random.Generator(np.random.PCG64(cfg['seed']))
    return [int(x) for x in g.integers(cfg['ctx_lo'], cfg['ctx_hi'] + 1, cfg['requests'])]


def query_units(draft_layers=DRAFT['layers'], verify_layers=VERIFY['layers']):
    return DRAFT['requests'] * BLOCK * draft_layers + VERIFY['requests'] * VERIFY['q'] * verify_layers


# --------------------------------------------------------------------------- clocks
class ClockSampler:
    """nvidia-smi clock samples (every 50 ms) of the GPU this rank drives, kept when they
    fall inside the `with` block. nvidia-smi takes longer to start than a short timed
    region lasts, so entering waits (up to 10 s) for its first sample, and leaving waits
    (up to 1 s) for the first sample after the block, which is kept as well: a region
    shorter than the sampling period still gets the sample taken at its end."""
    FIELDS = ('index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,'
              'clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,'
              'clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap')

    def __init__(self, gpu):
        self.gpu, self.proc, self.samples, self.lines = gpu, None, [], []
        self.t0 = self.t1 = None

    def _read(self):
        for ln in self.proc.stdout:
            if ln.strip():
                self.samples.append((time.monotonic(), ln))

    def _wait_for_sample(self, after, limit):
        deadline = time.monotonic() + limit
        while time.monotonic() < deadline:
            if any(t > after for t, _ in list(self.samples)):
                return
            time.sleep(0.01)

    def __enter__(self):
        import threading
        try:
            self.proc = subprocess.Popen(['nvidia-smi', '-i', str(self.gpu), f'--query-gpu={self.FIELDS}',
                                          '--format=csv,noheader,nounits', '-lms', '50'],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        if self.proc is not None:
            self.reader = threading.Thread(target=self._read, daemon=True)
            self.reader.start()
            self._wait_for_sample(0.0, 10.0)
        self.t0 = time.monotonic()
        return self

    def __exit__(self, *exc):
        self.t1 = time.monotonic()
        if self.proc is None:
            return
        self._wait_for_sample(self.t1, 1.0)
        self.proc.terminate()
        try:
            self.proc.wait(timeout=5)
        except Exception:
            self.proc.kill()
        self.reader.join(timeout=5)
        inside = [ln for t, ln in self.samples if self.t0 <= t <= self.t1]
        after = [ln for t, ln in self.samples if t > self.t1][:1]
        self.lines = inside + after

    def summary(self):
        sm, mx, reasons = [], 0.0, set()
        names = ('hw_slowdown', 'hw_thermal_slowdown', 'sw_thermal_slowdown', 'sw_power_cap')
        for ln in self.lines:
            f = [x.strip() for x in ln.split(',')]
            try:
                sm.append(float(f[1]))
                mx = max(mx, float(f[2]))
            except (ValueError, IndexError):
                continue
            for name, val in zip(names, f[5:9]):
                if val.lower() == 'active':
                    reasons.add(name)
        return dict(sm_mhz=statistics.median(sm) if sm else None, sm_max_mhz=mx or None,
                    reasons=sorted(reasons), samples=len(sm))


# --------------------------------------------------------------------------- config 2 inputs
def build_draft_06b(pkg, device):
    """Random-init DSparkDraft at the Qwen3-0.6B draft geometry (hidden 1024, FFN 3072,
    16/8 heads, 5 layers fed by 5 target layers, theta 1e6, block 7), bf16, seeded; its
    q/k and context norm weights are N(1, 0.1) so that they are not the identity. A
    7-layer target with a 1024-token vocabulary supplies the shared embedding (config 2
    needs no vocabulary)."""
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM
    torch.manual_seed(1)
    cfg = Qwen3Config(vocab_size=1024, hidden_size=1024, intermediate_size=3072, num_hidden_layers=7,
                      num_attention_heads=16, num_key_value_heads=8, head_dim=128, max_position_embeddings=40960,
                      rms_norm_eps=1e-6, tie_word_embeddings=True,
                      rope_parameters={'rope_type': 'default', 'rope_theta': 1e6})
    with torch.device(device), torch.no_grad():
        target = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
        spec = pkg.DraftSpec(layer_ids=(0, 1, 2, 3, 4), num_layers=5, block_size=BLOCK, markov_rank=64,
                             mask_token_id=1000)
        draft = pkg.DSparkDraftModel(target, spec).to(torch.bfloat16).eval()
        for layer in draft.layers:
            for w in (layer.attention.k_norm.weight, layer.attention.q_norm.weight):
                w.copy_(1 + 0.1 * torch.randn_like(w))
        draft.context_norm.weight.copy_(1 + 0.1 * torch.randn_like(draft.context_norm.weight))
    return draft


def draft_cfg2_inputs(pkg, device, rank=0, layers=DRAFT['layers']):
    """Config 2's draft-layer inputs as its statement builds them: context K/V from the
    draft's own projection chain on N(0,1) target features [sum(c), 5 x 1024] (fc
    5x1024->1024, context RMSNorm, per-layer k_proj / k_norm / RoPE and v_proj: the fused
    append into the paged pool, packed_draft.py:129-168), block rows from the q/k/v
    projections of N(0,1) block states at positions c..c+6 (model.py:41-45). Returns the
    draft, its pool, the features and block states, and per layer the packed
    ``[sum(c + 7), 8, 128]`` K/V (each request's context rows, then its block rows), the
    ``[64 * 7, 16, 128]`` queries and the layout. Features are seeded 1 + 1000 * rank."""
    import torch
    ctx = contexts(DRAFT)
    R = DRAFT['requests']
    draft = build_draft_06b(pkg, device)
    pd = pkg.B200PackedDraft(draft, max_requests=R, context_capacity=max(ctx), slot_capacities=ctx)
    names = [f'd{i}' for i in range(R)]
    for r in names:
        pd.add_request(r)
    gen = torch.Generator(device=device)
    gen.manual_seed(1 + 1000 * rank)
    bf = torch.bfloat16
    feats = torch.randn((1, sum(ctx), 5 * 1024), generator=gen, device=device, dtype=bf)
    chunks, o = {}, 0
    for r, c in zip(names, ctx):
        chunks[r] = feats[:, o:o + c]
        o += c
    with torch.no_grad():
        pd.append_committed(chunks)
    block_states = torch.randn((1, R * BLOCK, 1024), generator=gen, device=device, dtype=bf)
    bpos = torch.cat([torch.arange(c, c + BLOCK, device=device) for c in ctx])
    # row index of every packed key into cat(pool rows, block rows)
    pool_rows = pd.pool_k[0].shape[0]
    index = []
    for i, (r, c) in enumerate(zip(names, ctx)):
        r0 = pd.slot_rows[pd._slots[r]]
        index += list(range(r0, r0 + c)) + list(range(pool_rows + i * BLOCK, pool_rows + (i + 1) * BLOCK))
    index = torch.tensor(index, dtype=torch.long, device=device)
    qs, ks, vs = [], [], []
    with torch.no_grad():
        cos, sin = draft.rotary(block_states, bpos[None])
        for li, layer in enumerate(draft.layers[:layers]):
            q, bk, bv = pd._project(layer.attention, block_states, cos, sin)
            qs.append(q.contiguous())
            ks.append(torch.cat((pd.pool_k[li], bk)).index_select(0, index))
            vs.append(torch.cat((pd.pool_v[li], bv)).index_select(0, index))
    layout = pkg.PackedLayout.from_lengths([BLOCK] * R, [c + BLOCK for c in ctx], device)
    return dict(draft=draft, pool=pd, names=names, contexts=ctx, features=feats, block_states=block_states,
                q=qs, k=ks, v=vs, layout=layout)


# --------------------------------------------------------------------------- workload
class Workload:
    """Device-resident synthetic inputs of one rank (inputs larger than L2: ~62 GB of KV)."""

    def __init__(self, pkg, device, rank, steps_total, draft_layers=DRAFT['layers'],
                 verify_layers=VERIFY['layers']):
        import torch
        self.pkg, self.device = pkg, device
        self.draft_layers, self.verify_layers = draft_layers, verify_layers
        gen = torch.Generator(device=device)
        gen.manual_seed(1234 + rank)
        bf = torch.bfloat16

        def randn(*shape):
            return torch.randn(*shape, device=device, dtype=bf, generator=gen)

        # draft: packed [sum(c+7), 8, 128] K/V per layer (context cache rows + block rows),
        # projected by the draft's own chain as config 2 states
        self.draft_ctx = contexts(DRAFT)
        self.draft_qlens = [BLOCK] * DRAFT['requests']
        self.draft_klens = [c + BLOCK for c in self.draft_ctx]
        if draft_layers:
            d2 = draft_cfg2_inputs(pkg, device, rank, draft_layers)
            self.draft_layout = d2['layout']
            self.draft_q, self.draft_k, self.draft_v = d2['q'], d2['k'], d2['v']
            del d2
        else:
            self.draft_layout = pkg.PackedLayout.from_lengths(self.draft_qlens, self.draft_klens, device)
            self.draft_q, self.draft_k, self.draft_v = [], [], []
        self.draft_kernel = pkg.B200DraftKernel(device)
        # verify: ragged persistent store, capacity = context + growth of every step
        self.verify_ctx = contexts(VERIFY)
        L, R, Q = max(verify_layers, 1), VERIFY['requests'], VERIFY['q']
        growth = Q * (steps_total + 2)
        caps = [c + growth for c in self.verify_ctx]
        self.store = pkg.B200PersistentTargetKV(layers=L, slots=R, context_capacity=max(caps),
                                                max_query_tokens=R * Q, device=device, slot_capacities=caps)
        self.handles = [self.store.add_request(f'r{i}') for i in range(R)]
        # fill resident prefixes layer by layer (random N(0,1) bf16; values do not affect speed)
        rows = self.store.rows_per_layer
        for buf in (self.store._keys, self.store._values):
            for layer in range(L):
                buf[layer * rows:(layer + 1) * rows].normal_(generator=gen)
        self.store.mirror_lengths(self.handles, self.verify_ctx)
        nqv = R * Q
        self.vq = [randn(nqv, HQ, D) for _ in range(L)]
        self.vk = [randn(nqv, HKV, D) for _ in range(L)]
        self.vv = [randn(nqv, HKV, D) for _ in range(L)]
        self.qw = torch.ones(D, dtype=bf, device=device)
        self.kw = torch.ones(D, dtype=bf, device=device)
        self.inv_freq = pkg.rope_inv_freq(1e6, device=device)
        import numpy as np
        self.accept_rng = np.random.Generator(np.random.PCG64(VERIFY['seed'] * 7919 + rank))
        torch.cuda.synchronize(device)

    # algorithmic bytes (K/V read once, Q read, O written) -------------------------
    def draft_layer_bytes(self):
        return sum(self.draft_klens) * KV_ROW + 2 * sum(self.draft_qlens) * Q_ROW

    def verify_layer_bytes(self, contexts_now):
        R, Q = VERIFY['requests'], VERIFY['q']
        attn = (sum(contexts_now) + R * Q) * KV_ROW + 2 * R * Q * Q_ROW
        prologue = R * Q * (Q_ROW + KV_ROW) * 2      # raw q/k/v read, roped q + k/v written
        return attn + prologue

    def step(self, events=None):
        """One round on device-resident inputs. ``events``: list to append (start, end, kind)
        CUDA event pairs per layer."""
        for layer in range(self.draft_layers):
            e0 = self._event(events)
            self.draft_kernel(self.draft_q[layer], self.draft_k[layer], self.draft_v[layer], self.draft_layout,
                              scale=D ** -0.5)
            self._close(events, e0, 'draft')
        if not self.verify_layers:
            return
        store = self.store
        tx = store.begin(self.handles, query_lengths=[VERIFY['q']] * VERIFY['requests'])
        ctx_now = tx.context_lengths
        for layer in range(self.verify_layers):
            e0 = self._event(events)
            store.verify_layer(tx, layer, self.vq[layer], self.vk[layer], self.vv[layer], self.qw, self.kw,
                               inv_freq=self.inv_freq)
            self._close(events, e0, 'verify', ctx_now)
        self._commit(tx)

    def _commit(self, tx):
        accept = self.accept_rng.integers(0, 7, VERIFY['requests'])
        self.store.commit(tx, {h: int(a) + 1 for h, a in zip(self.handles, accept)})

    def step_e2e(self, host):
        """One round from pinned host memory: every layer's inputs are copied in and every
        attention output copied out, each step.

        Copies run on their own streams so PCIe traffic overlaps the kernels: the inputs
        of layer i+2 upload while layer i computes (two device slots per layer kind, a
        slot is refilled once the layer that read it has finished), and each output is
        read back as soon as its layer ends. The step is complete on the compute stream
        only after its last read-back."""
        import torch
        cur = torch.cuda.current_stream(self.device)
        io = self._io
        tasks = [('draft', l) for l in range(self.draft_layers)] + [('verify', l) for l in range(self.verify_layers)]

        def upload(i):
            kind, layer = tasks[i]
            slot = io['slots'][kind][layer % 2]
            with torch.cuda.stream(io['h2d']):
                if slot['free'] is not None:
                    io['h2d'].wait_event(slot['free'])
                srcs = (host['dq'][layer],) if kind == 'draft' else (host['vq'][layer], host['vk'][layer],
                                                                     host['vv'][layer])
                for dst, src in zip(slot['inp'], srcs):
                    dst.copy_(src, non_blocking=True)
                slot['ready'].record(io['h2d'])
            return slot

        begin = torch.cuda.Event()
        begin.record(cur)
        io['h2d'].wait_event(begin)             # this step's copies start inside its own region
        pending = [upload(i) for i in range(min(2, len(tasks)))]
        tx = None
        for i, (kind, layer) in enumerate(tasks):
            slot = pending.pop(0)
            if kind == 'verify' and tx is None:
                tx = self.store.begin(self.handles, query_lengths=[VERIFY['q']] * VERIFY['requests'])
            cur.wait_event(slot['ready'])
            if kind == 'draft':
                out = self.draft_kernel(slot['inp'][0], self.draft_k[layer], self.draft_v[layer], self.draft_layout,
                                        scale=D ** -0.5)
                out.record_stream(io['d2h'])
                dst = host['do'][layer]
            else:
                q, k, v = slot['inp']
                out = self.store.verify_layer(tx, layer, q, k, v, self.qw, self.kw, inv_freq=self.inv_freq)
                out.record_stream(io['d2h'])
                dst = host['vo'][layer]
            done = torch.cuda.Event()
            done.record(cur)
            slot['free'] = done
            with torch.cuda.stream(io['d2h']):
                io['d2h'].wait_event(done)
                dst.copy_(out, non_blocking=True)
            if i + 2 < len(tasks):
                pending.append(upload(i + 2))
        if tx is not None:
            self._commit(tx)
        read = torch.cuda.Event()
        read.record(io['d2h'])
        cur.wait_event(read)

    def step_copies(self, host):
        """The host copies of ``step_e2e`` alone: the same bytes on the same two copy
        streams, no kernels. Timed with every rank copying at once, its time beside
        ``step_e2e``'s shows whether the host copy path bounds the end-to-end step."""
        import torch
        cur = torch.cuda.current_stream(self.device)
        io = self._io
        begin = torch.cuda.Event()
        begin.record(cur)
        for st in (io['h2d'], io['d2h']):
            st.wait_event(begin)
        with torch.cuda.stream(io['h2d']):
            for layer in range(self.draft_layers):
                io['slots']['draft'][layer % 2]['inp'][0].copy_(host['dq'][layer], non_blocking=True)
            for layer in range(self.verify_layers):
                srcs = (host['vq'][layer], host['vk'][layer], host['vv'][layer])
                for dst, src in zip(io['slots']['verify'][layer % 2]['inp'], srcs):
                    dst.copy_(src, non_blocking=True)
        with torch.cuda.stream(io['d2h']):
            for layer in range(self.draft_layers):
                host['do'][layer].copy_(self.draft_q[layer], non_blocking=True)
            for layer in range(self.verify_layers):
                host['vo'][layer].copy_(self.vq[layer], non_blocking=True)
        for st in (io['h2d'], io['d2h']):
            done = torch.cuda.Event()
            done.record(st)
            cur.wait_event(done)

    @staticmethod
    def _event(events):
        if events is None:
            return None
        import torch
        e = torch.cuda.Event(enable_timing=True)
        e.record()
        return e

    @staticmethod
    def _close(events, e0, kind, ctx=None):
        if events is None:
            return
        import torch
        e1 = torch.cuda.Event(enable_timing=True)
        e1.record()
        events.append((e0, e1, kind, ctx))

    def pinned_host(self):
        """Pinned host copies of every layer's inputs and room for every output, plus the
        copy streams and the two device input slots per layer kind that ``step_e2e`` uses."""
        import torch
        pin = lambda t: t.cpu().pin_memory()  # noqa: E731
        slot = lambda ts: dict(inp=[torch.empty_like(t) for t in ts], ready=torch.cuda.Event(), free=None)  # noqa
        slots = dict(draft=[slot(self.draft_q[:1]) for _ in range(2)] if self.draft_layers else [],
                     verify=[slot((self.vq[0], self.vk[0], self.vv[0])) for _ in range(2)]
                     if self.verify_layers else [])
        self._io = dict(h2d=torch.cuda.Stream(self.device), d2h=torch.cuda.Stream(self.device), slots=slots)
        return dict(dq=[pin(q) for q in self.draft_q], vq=[pin(x) for x in self.vq], vk=[pin(x) for x in self.vk],
                    vv=[pin(x) for x in self.vv],
                    do=[torch.empty(q.shape, dtype=q.dtype).pin_memory() for q in self.draft_q],
                    vo=[torch.empty(x.shape, dtype=x.dtype).pin_memory() for x in self.vq])

    def host_bytes(self, host):
        h2d = sum(t.numel() * t.element_size() for k in ('dq', 'vq', 'vk', 'vv') for t in host[k])
        d2h = sum(t.numel() * t.element_size() for k in ('do', 'vo') for t in host[k])
        return h2d, d2h


# --------------------------------------------------------------------------- config 4
def train_layout_leg(pkg, device, rank, warmup, iters=20):
    """Config 4: training-layout draft attention (8 sequences x 2048 context, 32 sorted
    anchors each from 0..2046, block 7), one launch per timed iteration with a 256 MiB
    write before each launch so every launch starts with K/V (89 MB, smaller than L2)
    out of L2. The per-block two-segment path is timed the same way beside it."""
    import numpy as np
    import torch
    g = np.random.Generator(np.random.PCG64(TRAIN['seed'] * 1000 + rank))
    S, C, N = TRAIN['seqs'], TRAIN['ctx'], TRAIN['anchors']
    anchors = [sorted(g.choice(C - 1, N, replace=False).tolist()) for _ in range(S)]
    layout = pkg.TrainingLayout.from_anchors([C] * S, anchors, BLOCK, device=device)
    gen = torch.Generator(device=device)
    gen.manual_seed(4321 + rank)
    nq, nk = layout.query_tokens, layout.key_tokens
    q = torch.randn(nq, HQ, D, device=device, dtype=torch.bfloat16, generator=gen)
    k = torch.randn(nk, HKV, D, device=device, dtype=torch.bfloat16, generator=gen)
    v = torch.randn(nk, HKV, D, device=device, dtype=torch.bfloat16, generator=gen)
    kernel = pkg.B200TrainingLayoutKernel(device)
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)

    def tc():
        return kernel(q, k, v, layout, scale=D ** -0.5)

    def seg():
        return pkg.segment_attention(q, layout.seg_cu_query, [BLOCK] * len(layout.seg_a_len), k, v,
                                     layout.seg_a_start, layout.seg_a_len, k, v, layout.seg_b_start,
                                     layout.seg_b_len, causal=False)

    def timed(fn):
        for _ in range(warmup):
            fn()
        pairs = []
        for _ in range(iters):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            pairs.append((a, b))
        torch.cuda.synchronize(device)
        return statistics.median(a.elapsed_time(b) for a, b in pairs)

    ms, seg_ms = timed(tc), timed(seg)
    alg_bytes = nk * KV_ROW + 2 * nq * Q_ROW       # K+V read once, Q read, O written
    flops = sum(4 * BLOCK * HQ * D * (min(max(a, 0), C) + BLOCK) for seq in anchors for a in seq)
    hbm, hbm_kind = peaks()
    tflops, t_kind = tensor_peak()
    bound_ms = max(alg_bytes / (hbm * 1e9), flops / (tflops * 1e12)) * 1e3
    return dict(
        workload='cfg4 training-layout draft attention: 8 seqs x 2048 ctx, 32 sorted anchors/seq, block 7, '
                 'tcgen05 kernel (B200TrainingLayoutKernel)',
        query_rows=nq, key_rows=nk, ms_per_launch=ms, query_tok_per_s=nq / (ms / 1e3),
        alg_bytes=alg_bytes, alg_flops=flops, achieved_gbs=alg_bytes / (ms / 1e3) / 1e9,
        achieved_tflops=flops / (ms / 1e3) / 1e12, roofline_ms=bound_ms, frac=bound_ms / ms,
        peaks=dict(hbm_gbs=hbm, bf16_tflops=tflops, source=f'{hbm_kind}/{t_kind}'),
        l2='256 MiB written before every launch', segment_path_ms=seg_ms)


# --------------------------------------------------------------------------- graph replay
GRAPH = dict(requests=8, ctx_lo=256, ctx_hi=2048, seed=5, layers=28, q=7)
# config 5's decode rounds: 32 requests, prompts 64/256/2048 cycling, 64 tokens into the
# 128-token generation, 1 + block 7 verified rows
GRAPH5 = dict(requests=32, prompts=(64, 256, 2048), generated=64, seed=5, layers=28, q=8)


def graph_leg(pkg, device, rank, warmup, steps, cfg=GRAPH):
    """Small serving batch (8 requests, context U[256,2048], 7 new rows, 28 layers):
    one verify step = begin + cos/sin table + 28 fused verify layers + commit, run
    eagerly (one host call per layer) and as a replay of the same 28 layers captured
    once into a CUDA graph over the store's bucket-bound metadata buffers. Device
    time per step, both ways, over the same rounds."""
    import numpy as np
    import torch
    g = np.random.Generator(np.random.PCG64(cfg['seed'] * 1000 + rank))
    if 'prompts' in cfg:
        ctx = [cfg['prompts'][i % len(cfg['prompts'])] + cfg['generated'] for i in range(cfg['requests'])]
    else:
        ctx = [int(x) for x in g.integers(cfg['ctx_lo'], cfg['ctx_hi'] + 1, cfg['requests'])]
    R, Q, L = cfg['requests'], cfg['q'], cfg['layers']
    growth = Q * 2 * (warmup + steps + 2)
    store = pkg.B200PersistentTargetKV(layers=L, slots=R, context_capacity=max(ctx) + growth,
                                       max_query_tokens=R * Q, device=device,
                                       slot_capacities=[c + growth for c in ctx])
    handles = [store.add_request(f'g{i}') for i in range(R)]
    gen = torch.Generator(device=device)
    gen.manual_seed(99 + rank)
    store._keys.normal_(generator=gen)
    store._values.normal_(generator=gen)
    store.mirror_lengths(handles, ctx)
    bf = torch.bfloat16
    vq = [torch.randn(R * Q, HQ, D, device=device, dtype=bf, generator=gen) for _ in range(L)]
    vk = [torch.randn(R * Q, HKV, D, device=device, dtype=bf, generator=gen) for _ in range(L)]
    vv = [torch.randn(R * Q, HKV, D, device=device, dtype=bf, generator=gen) for _ in range(L)]
    w = torch.ones(D, dtype=bf, device=device)
    inv = pkg.rope_inv_freq(1e6, device=device)
    outs = [torch.empty(R * Q, HQ, D, dtype=bf, device=device) for _ in range(L)]
    accept = np.random.Generator(np.random.PCG64(17 + rank))

    class Bucket:
        query_lengths = (Q,) * R

    bucket = Bucket()
    store.bind_bucket(bucket)

    def layers(tx):
        for layer in range(L):
            store.verify_layer(tx, layer, vq[layer], vk[layer], vv[layer], w, w, inv_freq=inv, out=outs[layer])

    def commit(tx):
        store.commit(tx, {h: int(a) + 1 for h, a in zip(handles, accept.integers(0, Q, R))})

    def eager_step():
        tx = store.begin(handles, query_lengths=[Q] * R)
        layers(tx)
        commit(tx)

    side = torch.cuda.Stream(device)
    side.wait_stream(torch.cuda.current_stream(device))
    with torch.cuda.stream(side):
        tx = store.capture_transaction(bucket)
        layers(tx)
        store.abort(tx)
    torch.cuda.current_stream(device).wait_stream(side)
    graph = torch.cuda.CUDAGraph()
    tx = store.capture_transaction(bucket)
    with torch.cuda.graph(graph, stream=side):
        layers(tx)
    store.abort(tx)

    def graph_step():
        tx = store.begin(handles, bucket)
        graph.replay()
        store.replayed(tx)
        commit(tx)

    def timed(step):
        for _ in range(warmup):
            step()
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0 = time.perf_counter()
        a.record()
        for _ in range(steps):
            step()
        b.record()
        host_ms = (time.perf_counter() - t0) * 1e3 / steps
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) / steps, host_ms

    eager_ms, eager_host = timed(eager_step)
    graph_ms, graph_host = timed(graph_step)
    units = R * Q * L
    # algorithmic bytes of one layer: resident + new K/V rows read once, q read, out written
    layer_bytes = sum(c + Q for c in ctx) * HKV * D * 2 * 2 + 2 * R * Q * HQ * D * 2
    span = (f'prompts {cfg["prompts"]} + {cfg["generated"]}' if 'prompts' in cfg
            else f'ctx U[{cfg["ctx_lo"]},{cfg["ctx_hi"]}]')
    hbm, kind = peaks()
    return dict(workload=f'{R} requests, {span}, q {Q}, {L} fused verify layers + cos/sin table + commit per step',
                layer_alg_bytes=layer_bytes, graph_gbs=layer_bytes * L / (graph_ms / 1e3) / 1e9,
                graph_frac=layer_bytes * L / (graph_ms / 1e3) / 1e9 / hbm, peak_gbs=hbm, peak_source=kind,
                eager_ms_per_step=eager_ms, graph_ms_per_step=graph_ms, eager_host_ms_per_step=eager_host,
                graph_host_ms_per_step=graph_host, eager_query_tok_per_s=units / (eager_ms / 1e3),
                graph_query_tok_per_s=units / (graph_ms / 1e3), speedup=eager_ms / graph_ms,
                graph_launches_per_step='1 graph (29 kernels) + commit')


# --------------------------------------------------------------------------- accept
def accept_leg(pkg, device, warmup, iters=20, vocab=151936):
    """On-device greedy acceptance for one config-3 verify round: argmax over the
    logits of 128 x 7 verified rows (Qwen3 vocab 151936, bf16: 272 MB, larger than
    L2, and L2 written over before each round) + the accept rule, with the EOS ids
    kept on the device as the round loops keep them. HBM roofline: the logits are
    read once."""
    import torch
    r, q = VERIFY['requests'], VERIFY['q']
    n = r * q
    gen = torch.Generator(device=device)
    gen.manual_seed(7)
    logits = torch.randn(n, vocab, device=device, dtype=torch.bfloat16, generator=gen)
    tokens = torch.randint(0, vocab, (n,), device=device, generator=gen)
    cu = torch.arange(0, n + 1, q, dtype=torch.int32, device=device)
    budget = torch.full((r,), 64, dtype=torch.int32, device=device)
    eos = torch.tensor([151645], dtype=torch.long, device=device)   # on the device once, as the round loops keep it
    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)
    for _ in range(warmup):
        pkg.greedy_accept(logits, tokens, cu, eos, budget)
    torch.cuda.synchronize(device)
    torch.cuda._sleep(4_000_000)            # every launch below is enqueued before it runs: device time only
    pairs = []
    for _ in range(iters):
        flush.zero_()                       # L2 written over: no logits carried over from the last round
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        pkg.greedy_accept(logits, tokens, cu, eos, budget)
        b.record()
        pairs.append((a, b))
    torch.cuda.synchronize(device)
    ms = statistics.median(a.elapsed_time(b) for a, b in pairs)
    nbytes = n * vocab * 2
    hbm, kind = peaks()
    return dict(workload=f'{r} requests x {q} verified rows, vocab {vocab}, bf16 logits', ms=ms,
                alg_bytes=nbytes, achieved_gbs=nbytes / (ms / 1e3) / 1e9,
                frac=nbytes / (ms / 1e3) / 1e9 / hbm, peak_gbs=hbm, peak_source=kind)


# --------------------------------------------------------------------------- markov
def markov_leg(pkg, device, warmup, iters=10, r=64, vocab=151936, rank=256, hdim=1024):
    """Greedy Markov proposal of one draft block (config 2's 64 requests, Qwen3 vocab,
    markov_rank 256 of the 0.6B draft config, block 7): the fused kernel (one launch
    per position, logits never written) vs the reference's torch loop on the same
    inputs. HBM roofline per block: 7 x (projection weight + one LM-head logits row
    per request)."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(11)
    bf = torch.bfloat16
    w = torch.randn(vocab, rank, device=device, dtype=bf, generator=gen) * 0.05
    e = torch.randn(vocab, rank, device=device, dtype=bf, generator=gen) * 0.5
    cw = torch.randn(hdim + rank, device=device, dtype=bf, generator=gen) * 0.05
    hidden = torch.randn(r * BLOCK, hdim, device=device, dtype=bf, generator=gen)
    base = torch.randn(r * BLOCK, vocab, device=device, dtype=bf, generator=gen)
    anchors = torch.randint(0, vocab, (r,), device=device, generator=gen)
    proj = torch.nn.Linear(rank, vocab, bias=False, device=device, dtype=bf)
    proj.weight.data.copy_(w)
    conf_lin = torch.nn.Linear(hdim + rank, 1, device=device, dtype=bf)
    conf_lin.weight.data.copy_(cw[None])
    conf_lin.bias.data.fill_(0.1)
    emb = torch.nn.Embedding(vocab, rank, device=device, dtype=bf)
    emb.weight.data.copy_(e)
    hv = hidden.view(r, BLOCK, hdim)
    bv = base.view(r, BLOCK, vocab)

    def fused():
        return pkg.markov_greedy(w, e, cw, 0.1, hidden, base, anchors, BLOCK)

    def torch_loop():                       # DSparkDraft._sample_greedy, batched over requests
        prev, toks, confs = anchors, [], []
        for k in range(BLOCK):
            em = emb(prev)
            confs.append(conf_lin(torch.cat((hv[:, k], em), -1)).sigmoid().flatten())
            prev = (bv[:, k] + proj(em)).argmax(-1)
            toks.append(prev)
        return torch.stack(toks, 1), torch.stack(confs, 1)

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)

    def timed(fn):
        for _ in range(warmup):
            fn()
        pairs = []
        for _ in range(iters):
            flush.zero_()                   # L2 written over: nothing carries over between blocks
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            pairs.append((a, b))
        torch.cuda.synchronize(device)
        return statistics.median(a.elapsed_time(b) for a, b in pairs)

    ms, torch_ms = timed(fused), timed(torch_loop)
    nbytes = BLOCK * (vocab * rank * 2 + r * vocab * 2)
    hbm, kind = peaks()
    return dict(workload=f'{r} requests x block {BLOCK}, vocab {vocab}, markov_rank {rank}, bf16',
                ms_per_block=ms, torch_loop_ms_per_block=torch_ms, speedup=torch_ms / ms, alg_bytes=nbytes,
                achieved_gbs=nbytes / (ms / 1e3) / 1e9, frac=nbytes / (ms / 1e3) / 1e9 / hbm, peak_gbs=hbm,
                peak_source=kind)


def propose_leg(pkg, device, warmup, iters=10, r=64, vocab=151936, rank=256, temperature=0.8):
    """Stochastic Markov proposal of one draft block (config 2's 64 requests, Qwen3 vocab,
    markov_rank 256, block 7, T = 0.8): per position the embedding gather and projection
    GEMM (torch), then one ``stochastic_propose`` launch (x = base + proj, the float64 law
    written out, the CDF draw) vs the reference's formula in torch on the same inputs
    (``float64_law`` + ``sample_rows``, DSparkDraft._sample_stochastic batched). Bytes
    per block: 7 x (projection weight + per request two bf16 rows read and a float64
    law row written)."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(13)
    bf = torch.bfloat16
    proj = torch.nn.Linear(rank, vocab, bias=False, device=device, dtype=bf)
    proj.weight.data.copy_(torch.randn(vocab, rank, device=device, dtype=bf, generator=gen) * 0.05)
    emb = torch.nn.Embedding(vocab, rank, device=device, dtype=bf)
    emb.weight.data.copy_(torch.randn(vocab, rank, device=device, dtype=bf, generator=gen) * 0.5)
    base = torch.randn(r, BLOCK, vocab, device=device, dtype=bf, generator=gen) * 2
    anchors = torch.randint(0, vocab, (r,), device=device, generator=gen)
    u = torch.rand(r, BLOCK, device=device, dtype=torch.float64, generator=gen)
    laws = torch.empty(r, BLOCK, vocab, device=device, dtype=torch.float64)
    idx = torch.arange(r, device=device, dtype=torch.int32)

    def fused():
        prev = anchors
        for k in range(BLOCK):
            pj = proj(emb(prev)).contiguous()
            prev, _ = pkg.stochastic_propose(base[:, k], idx, pj, temperature, u[:, k].contiguous(), laws[:, k])
        return prev

    def torch_formula():
        prev = anchors
        for k in range(BLOCK):
            law = pkg.float64_law(base[:, k] + proj(emb(prev)), temperature)
            prev = pkg.sample_rows(law, u[:, k])
            laws[:, k].copy_(law)
        return prev

    flush = torch.empty(256 << 20, dtype=torch.uint8, device=device)

    def timed(fn):
        for _ in range(warmup):
            fn()
        pairs = []
        for _ in range(iters):
            flush.zero_()
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            pairs.append((a, b))
        torch.cuda.synchronize(device)
        return statistics.median(a.elapsed_time(b) for a, b in pairs)

    assert torch.equal(fused(), torch_formula())          # same final tokens on these inputs
    ms, torch_ms = timed(fused), timed(torch_formula)
    nbytes = BLOCK * (vocab * rank * 2 + r * vocab * (2 + 2 + 8))
    hbm, kind = peaks()
    return dict(workload=f'{r} requests x block {BLOCK}, vocab {vocab}, markov_rank {rank}, T {temperature}, '
                         'float64 laws written out',
                ms_per_block=ms, torch_formula_ms_per_block=torch_ms, speedup=torch_ms / ms, alg_bytes=nbytes,
                achieved_gbs=nbytes / (ms / 1e3) / 1e9, frac=nbytes / (ms / 1e3) / 1e9 / hbm, peak_gbs=hbm,
                peak_source=kind)


def append_leg(pkg, device, warmup, iters=10):
    """Draft-context append at the 0.6B draft geometry (hidden 1024, five draft layers,
    five captured target layers of features; random weights, bf16): every layer's
    k = RoPE(k_norm(k_proj(c))) and v = v_proj(c) of the context rows c = context_norm(
    fc(features)) written into the paged pool. Two workloads of config 5: the prefill
    append (32 requests, prompts cycling 64/256/2048 = 24,000 rows) and one round's
    fixed-shape append (32 requests x 8 verified rows, random commit counts). Compared:
    the fused tcgen05 append (rope table + one GEMM-with-epilogue launch) and the
    reference's per-layer torch formula on the same pool. Tensor-core roofline of the
    fused kernel: 2 x rows x (layers x 2048) x hidden FLOPs."""
    import numpy as np
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM
    hidden, layers, nfeat = 1024, 5, 5
    torch.manual_seed(21)
    cfg = Qwen3Config(vocab_size=1024, hidden_size=hidden, intermediate_size=3072, num_hidden_layers=nfeat + 2,
                      num_attention_heads=16, num_key_value_heads=8, head_dim=128, max_position_embeddings=40960,
                      rms_norm_eps=1e-6, tie_word_embeddings=False,
                      rope_parameters={'rope_type': 'default', 'rope_theta': 1e6})
    with torch.device(device), torch.no_grad():
        model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
        spec = pkg.DraftSpec(layer_ids=tuple(range(1, nfeat + 1)), num_layers=layers, mask_token_id=1000)
        draft = pkg.DSparkDraftModel(model, spec).to(torch.bfloat16).eval()
    lens = [(64, 256, 2048)[i % 3] for i in range(32)]
    fused = pkg.B200PackedDraft(draft, max_requests=32, slot_capacities=[n + 64 for n in lens],
                                context_capacity=0)
    plain = pkg.B200PackedDraft(draft, max_requests=32, slot_capacities=[n + 64 for n in lens],
                                context_capacity=0)
    plain._fused_append_ready = lambda: False
    g = np.random.Generator(np.random.PCG64(22))

    def feats(n):
        return torch.from_numpy(g.standard_normal((1, n, nfeat * hidden)).astype(np.float32)).to(device, torch.bfloat16)

    def timed(fn, queued=False):
        # queued: the GPU first sleeps ~2 ms so that every launch below is enqueued
        # before it runs and the events time the device alone (a launch shorter than
        # its host-side call would otherwise time the call)
        for _ in range(warmup):
            fn()
        if queued:
            torch.cuda.synchronize(device)
            torch.cuda._sleep(4_000_000)
        pairs = []
        for _ in range(iters):
            a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            a.record()
            fn()
            b.record()
            pairs.append((a, b))
        torch.cuda.synchronize(device)
        return statistics.median(a.elapsed_time(b) for a, b in pairs)

    tflops_peak, kind = tensor_peak()
    out = {}
    cases = (('prefill', lens, lens), ('round', [8] * 32, [int(c) for c in g.integers(1, 9, 32)]))
    for name, widths, counts in cases:
        r, n = len(widths), sum(widths)
        cu = [0]
        for w in widths:
            cu.append(cu[-1] + w)
        meta = torch.tensor(cu + list(fused.slot_rows) + [0] * r + counts, dtype=torch.int32, device=device)
        x = feats(n)
        with torch.no_grad():
            ctx = draft.context_norm(draft.fc(x))[0].contiguous()
        kv_w, kn_w, rope = fused._append_operands()
        eps = draft.layers[0].attention.k_norm.variance_epsilon

        def kernel():
            pkg.kernels.draft_append(ctx, kv_w, kn_w, rope, meta, r, fused.pool_k, fused.pool_v,
                                     fused.trash_row, eps)

        with torch.no_grad():
            fused_ms = timed(lambda: fused._append_rows(x, meta, r, n))
            torch_ms = timed(lambda: plain._append_rows(x, meta, r, n))
        kernel_ms = timed(kernel, queued=True)
        flops = 2.0 * n * layers * 2048 * hidden
        out[name] = dict(rows=n, requests=r, fused_ms=fused_ms, torch_formula_ms=torch_ms,
                         speedup=torch_ms / fused_ms, append_kernel_ms=kernel_ms,
                         kernel_tflops=flops / (kernel_ms / 1e3) / 1e12,
                         kernel_frac=flops / (kernel_ms / 1e3) / 1e12 / tflops_peak)
    if hasattr(fused, 'capture_append'):
        reqs = tuple(f'g{i}' for i in range(32))
        for q in reqs:
            fused.add_request(q)
        fused.capture_append(32, 8)
        x = feats(256)
        counts = [0] * 32

        def replay():
            fused.append_verified_graph(x, reqs, counts)
        with torch.no_grad():
            out['round']['graph_replay_ms'] = timed(replay)
    out.update(workload='0.6B draft geometry: hidden 1024, 5 draft layers, 5 x 1024 features, bf16',
               peak_tflops=tflops_peak, peak_source=kind)
    return out


def stochastic_leg(pkg, device, warmup, iters=10, r=128, n=6, vocab=151936, temperature=0.8):
    """Stochastic acceptance of one verify round at config 3's shape (128 requests,
    6 proposals + 1 row each, Qwen3 vocabulary): target logits bf16 [R * 7, V], draft
    laws float64 [R * 6, V] (the reference's TensorProposal.draft_probs), float64
    uniforms. The on-device law statistics + acceptance (two launches) against the
    reference's verify_proposal formula run per request with torch float64 ops on the
    same GPU (logits_to_probabilities + the sequential accept loop)."""
    import torch
    gen = torch.Generator(device=device)
    gen.manual_seed(31)
    logits = (torch.randn(r * (n + 1), vocab, device=device, generator=gen) * 2).to(torch.bfloat16)
    draft_logits = logits[:0].float()
    rows = []
    for i in range(r):
        rows.append(logits[i * (n + 1):i * (n + 1) + n].float() + 0.3 * torch.randn(n, vocab, device=device,
                                                                                      generator=gen))
    q = torch.softmax(torch.cat(rows).double() / temperature, -1)
    q = q / q.sum(-1, keepdim=True)
    tokens = torch.multinomial(q.float(), 1, generator=gen).flatten()
    cu = torch.arange(0, r * n + 1, n, dtype=torch.int32, device=device)
    u = torch.rand(r, n + 1, dtype=torch.float64, device=device, generator=gen)
    budget = torch.full((r,), 1000, dtype=torch.int32, device=device)
    del draft_logits, rows

    def fused():
        return pkg.stochastic_accept(logits, tokens, q, cu, temperature, u, budget)

    def torch_formula():                     # the reference's per-request float64 loop (tensor_sampling.py)
        out = []
        for i in range(r):
            p = torch.softmax(logits[i * (n + 1):(i + 1) * (n + 1)].double() / temperature, -1)
            p = p / p.sum(-1, keepdim=True)
            qi, ti = q[i * n:(i + 1) * n], tokens[i * n:(i + 1) * n]
            alpha = torch.minimum(p[:n].gather(1, ti[:, None]).flatten() / qi.gather(1, ti[:, None]).flatten(),
                                  torch.ones(n, dtype=torch.float64, device=device))
            rej = (u[i, :n] >= alpha).nonzero()
            if rej.numel():
                j = int(rej[0, 0])
                res = (p[j] - qi[j]).relu()
                res = res / res.sum()
                out.append(torch.searchsorted(res.cumsum(-1), u[i, n:n + 1], right=True))
            else:
                out.append(torch.searchsorted(p[n].cumsum(-1), u[i, n:n + 1], right=True))
        return out

    def timed(fn, k):
        for _ in range(warmup):
            fn()
        torch.cuda.synchronize(device)
        a, b = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        a.record()
        for _ in range(k):
            fn()
        b.record()
        torch.cuda.synchronize(device)
        return a.elapsed_time(b) / k

    ms = timed(fused, iters)
    torch_ms = timed(torch_formula, 2)
    _, res = fused()
    res = res.cpu()
    nbytes = q.numel() * 8 + logits.numel() * 2
    hbm, kind = peaks()
    return dict(workload=f'{r} requests x {n} proposals, vocab {vocab}, bf16 target logits, float64 draft laws',
                ms=ms, torch_formula_ms=torch_ms, speedup=torch_ms / ms,
                mean_accepted=float(res[:, 1].float().mean()), status_ok=bool((res[:, 6] == 0).all()),
                alg_bytes=nbytes, achieved_gbs=nbytes / (ms / 1e3) / 1e9, frac=nbytes / (ms / 1e3) / 1e9 / hbm,
                peak_gbs=hbm, peak_source=kind)


# --------------------------------------------------------------------------- config 5
ROUND5 = dict(requests=32, prompts=(64, 256, 2048), new_tokens=128, seed=5)


def round5_leg(pkg, device, rank, warmup, pipelined_only=False):
    """Config 5: a full greedy speculative round loop on a Qwen3-0.6B-shaped target (28
    layers, hidden 1024, FFN 3072, vocab 151936, tied embeddings) and the 5-layer DSpark
    draft of the 0.6B config (layers 1/7/14/21/26, block 7, markov_rank 256), random
    weights (seeded), bf16, 32 requests with prompts cycling 64/256/2048 tokens, 128 new
    tokens each. Everything the round needs runs on this library: fused verify layers,
    commit/rollback, draft attention over the paged pool, the fused Markov proposal and
    on-device acceptance; the GEMMs are the library GEMMs of torch. ``pipelined_only``
    warms and times only the pipelined loop (the default bench line's config-5 leg)."""
    import numpy as np
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(vocab_size=151936, hidden_size=1024, intermediate_size=3072, num_hidden_layers=28,
                      num_attention_heads=16, num_key_value_heads=8, head_dim=128, max_position_embeddings=40960,
                      rms_norm_eps=1e-6, tie_word_embeddings=True,
                      rope_parameters={'rope_type': 'default', 'rope_theta': 1e6})
    cfg._attn_implementation = 'sdpa'
    torch.manual_seed(ROUND5['seed'] * 1000 + rank)
    with torch.device(device):
        model = Qwen3ForCausalLM(cfg).to(torch.bfloat16).eval()
        spec = pkg.DraftSpec()
        draft = pkg.DSparkDraftModel(model, spec).to(torch.bfloat16).eval()
    g = np.random.Generator(np.random.PCG64(ROUND5['seed'] * 1000 + rank))
    lens = [ROUND5['prompts'][i % len(ROUND5['prompts'])] for i in range(ROUND5['requests'])]
    cap = max(lens) + ROUND5['new_tokens'] + 16
    target = pkg.B200Qwen3Target(model, spec.layer_ids, slots=ROUND5['requests'], context_capacity=cap,
                                 max_query_tokens=sum(lens), slot_capacities=[n + ROUND5['new_tokens'] + 16 for n in lens])
    pdraft = pkg.B200PackedDraft(draft, max_requests=ROUND5['requests'], context_capacity=cap)

    def prompts(tag):
        return {f'{tag}{i}': torch.from_numpy(g.integers(0, 151643, (1, n))).to(device) for i, n in enumerate(lens)}

    def release(ps):
        for r in ps:
            target.remove_request(r)
            pdraft.remove_request(r)

    if not pipelined_only:
        for w in range(max(1, warmup // 3)):              # warm-up: library handles, allocator
            ps = prompts(f'w{w}_')
            pkg.speculative_greedy(target, pdraft, ps, 4)
            release(ps)

    def device_timer():
        """(start, stop): CUDA events on the current stream; stop() synchronises and returns s."""
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        torch.cuda.synchronize(device)
        e0.record()

        def stop():
            e1.record()
            torch.cuda.synchronize(device)
            return e0.elapsed_time(e1) / 1e3
        return stop

    def timed_loop(tag, graph):
        ps = prompts(tag)
        stop = device_timer()
        if graph == 'pipelined':
            out, rounds = pkg.speculative_greedy_pipelined(target, pdraft, ps, ROUND5['new_tokens'])
        else:
            out, rounds = pkg.speculative_greedy(target, pdraft, ps, ROUND5['new_tokens'], graph=graph)
        dt = stop()
        release(ps)
        return out, rounds, dt

    if pipelined_only:
        pkg.speculative_greedy_pipelined(target, pdraft, prompts('pw'), 4)   # capture and warm the loop
        release([f'pw{i}' for i in range(len(lens))])
        out_p, rounds_p, total_p = timed_loop('q', 'pipelined')
        generated = sum(len(v) for v in out_p.values())
        return dict(workload=f'Qwen3-0.6B-shaped target + 5-layer DSpark draft (random weights, bf16), '
                             f'{ROUND5["requests"]} requests, prompts {ROUND5["prompts"]} cycling, '
                             f'{ROUND5["new_tokens"]} new tokens each, speculative_greedy_pipelined',
                    generated_tokens=generated, rounds=len(rounds_p), total_s=total_p,
                    total_tok_per_s=generated / total_p)
    out, rounds, total_s = timed_loop('m', False)
    pkg.speculative_greedy(target, pdraft, prompts('gw'), 4, graph=True)   # capture + warm the replayed path
    release([f'gw{i}' for i in range(len(lens))])
    out_g, rounds_g, total_g = timed_loop('g', True)
    pkg.speculative_greedy_pipelined(target, pdraft, prompts('pw'), 4)   # warm the pipelined path
    release([f'pw{i}' for i in range(len(lens))])
    out_p, rounds_p, total_p = timed_loop('q', 'pipelined')
    # prefill alone (same prompts, fresh requests), to split the time
    ps = prompts('p')
    for r in ps:
        target.add_request(r)
        pdraft.add_request(r)
    stop = device_timer()
    feats = target.prefill(ps)
    pdraft.append_committed({r: feats.context_for(r) for r in ps})
    prefill_s = stop()
    release(ps)
    generated = sum(len(v) for v in out.values())
    accepted = [s['accepted'] for rd in rounds for s in rd.values()]
    decode_s = max(total_s - prefill_s, 1e-9)
    decode_g = max(total_g - prefill_s, 1e-9)
    return dict(workload=f'Qwen3-0.6B-shaped target + 5-layer DSpark draft (random weights, bf16), '
                         f'{ROUND5["requests"]} requests, prompts {ROUND5["prompts"]} cycling, '
                         f'{ROUND5["new_tokens"]} new tokens each',
                generated_tokens=generated, rounds=len(rounds), total_s=total_s, prefill_s=prefill_s,
                decode_tok_per_s=(generated - len(out)) / decode_s, total_tok_per_s=generated / total_s,
                graph_total_s=total_g, graph_decode_tok_per_s=(generated - len(out)) / decode_g,
                pipelined_total_s=total_p,
                pipelined_decode_tok_per_s=(generated - len(out)) / max(total_p - prefill_s, 1e-9),
                pipelined_total_tok_per_s=generated / total_p, graph_total_tok_per_s=generated / total_g,
                mean_accepted_per_round=float(np.mean(accepted)) if accepted else 0.0,
                note='random draft weights: acceptance is ~0, so every round emits one token per request; '
                     'eager and graph loops run different random prompts of the same lengths '
                     '(graph and eager tokens are compared on equal prompts in the GPU tests)')


# --------------------------------------------------------------------------- CPU legs
CPU_SAMPLE = dict(draft_requests=8, verify_requests=4)


def quantile_requests(ctx, n):
    """Indices of n requests at the (2i+1)/(2n) quantiles of the sorted context draw, so a
    small sample spans the whole distribution (shortest to longest)."""
    order = sorted(range(len(ctx)), key=ctx.__getitem__)
    return [order[(2 * i + 1) * len(ctx) // (2 * n)] for i in range(n)]


def set_host_threads():
    """Every host thread this process may use, set explicitly: torchrun exports
    OMP_NUM_THREADS=1, which an environment default would not override. Returns the
    thread count torch reports in effect."""
    import torch
    n = host_threads()
    os.environ['OMP_NUM_THREADS'] = str(n)
    os.environ['MKL_NUM_THREADS'] = str(n)
    torch.set_num_threads(n)
    return torch.get_num_threads()


class CPURound:
    """The reference's CPU round on a bounded sample of the bench's own workload: the
    torch operations of its draft and verify attention paths (``oracle/torch_cpu.py``,
    pinned to fixtures made by the reference's functions), float32 as the reference's
    CPU store defaults to, on all host threads.

    One sample step = one whole round for a subset of the requests: the draft attention
    of 8 config-2 requests for each of the 5 draft layers, then ``begin`` for 4 config-3
    requests, the 28 verify layers (q/k RMSNorm + RoPE, stage, gather, SDPA) and the
    commit of accept ~ U{0..6} + anchor. The requests sit at evenly spaced quantiles of
    their config's context draw, so the sample's mean context matches the full batch's."""

    def __init__(self, steps_total, seed=99):
        import torch
        from oracle.torch_cpu import VerifyRoundCPU
        from oracle.rope_norm import inv_freq
        import numpy as np
        self.threads = set_host_threads()
        gen = torch.Generator().manual_seed(seed)
        dall, vall = contexts(DRAFT), contexts(VERIFY)
        self.dctx = [dall[i] for i in quantile_requests(dall, CPU_SAMPLE['draft_requests'])]
        self.vctx = [vall[i] for i in quantile_requests(vall, CPU_SAMPLE['verify_requests'])]
        nd, nv, Q = len(self.dctx), len(self.vctx), VERIFY['q']
        self.dklens = [c + BLOCK for c in self.dctx]
        f32 = torch.float32
        self.dq = [torch.randn((nd * BLOCK, HQ, D), generator=gen) for _ in range(DRAFT['layers'])]
        self.dk = [torch.randn((sum(self.dklens), HKV, D), generator=gen) for _ in range(DRAFT['layers'])]
        self.dv = [torch.randn((sum(self.dklens), HKV, D), generator=gen) for _ in range(DRAFT['layers'])]
        growth = Q * (steps_total + 2)
        self.store = VerifyRoundCPU(VERIFY['layers'], self.vctx, nv * Q, HKV, D,
                                    slot_capacities=[c + growth for c in self.vctx], dtype=f32, generator=gen)
        self.vq = [torch.randn((nv * Q, HQ, D), generator=gen) for _ in range(VERIFY['layers'])]
        self.vk = [torch.randn((nv * Q, HKV, D), generator=gen) for _ in range(VERIFY['layers'])]
        self.vv = [torch.randn((nv * Q, HKV, D), generator=gen) for _ in range(VERIFY['layers'])]
        self.ones = torch.ones(D, dtype=f32)
        self.freqs = torch.from_numpy(inv_freq(1e6, D))
        self.accept = np.random.Generator(np.random.PCG64(seed))
        self.units = nd * BLOCK * DRAFT['layers'] + nv * Q * VERIFY['layers']
        self.fraction = self.units / query_units()

    def step(self):
        from oracle.torch_cpu import noncausal_varlen_sdpa
        for layer in range(DRAFT['layers']):
            noncausal_varlen_sdpa(self.dq[layer], self.dk[layer], self.dv[layer], [BLOCK] * len(self.dctx),
                                  self.dklens, D ** -0.5)
        store, Q = self.store, VERIFY['q']
        ws = store.begin([Q] * len(self.vctx))
        for layer in range(VERIFY['layers']):
            store.layer(ws, layer, self.vq[layer], self.vk[layer], self.vv[layer], self.ones, self.ones, self.freqs,
                        1e-6, D ** -0.5)
        store.commit(ws, [int(a) + 1 for a in self.accept.integers(0, Q, len(self.vctx))])

    def describe(self):
        return (f'torch CPU float32 restatement of the reference round (oracle/torch_cpu.py): per step one whole '
                f'round for {len(self.dctx)} cfg2 draft requests x{DRAFT["layers"]} layers (contexts '
                f'{self.dctx}) and {len(self.vctx)} cfg3 verify requests x{VERIFY["layers"]} layers with begin, '
                f'q/k norm + RoPE, stage, gather, SDPA and commit (contexts {self.vctx}); '
                f'{self.units} of the full step\'s {query_units()} query units ({self.fraction:.4f})')


def cpu_train_layout(seconds=3.0, threads=None):
    """Config 4 on the host as the reference's training forward runs it (oracle/torch_cpu.py:
    `block_mask` + dense-mask SDPA per sequence, float32), the whole workload per call:
    8 sequences x 2048 context, 32 sorted anchors each, block 7. Returns (query-tok/s, calls,
    seconds)."""
    import numpy as np
    import torch
    from oracle.torch_cpu import training_layout_sdpa
    if threads is None:
        set_host_threads()
    g = np.random.Generator(np.random.PCG64(TRAIN['seed'] * 1000))
    S, C, N = TRAIN['seqs'], TRAIN['ctx'], TRAIN['anchors']
    anchors = [sorted(g.choice(C - 1, N, replace=False).tolist()) for _ in range(S)]
    gen = torch.Generator().manual_seed(TRAIN['seed'])
    nq, nk = S * N * BLOCK, S * (C + N * BLOCK)
    q, k, v = (torch.randn((n, h, D), generator=gen) for n, h in ((nq, HQ), (nk, HKV), (nk, HKV)))
    training_layout_sdpa(q, k, v, [C] * S, anchors, BLOCK)
    calls, t0 = 0, time.perf_counter()
    while True:
        training_layout_sdpa(q, k, v, [C] * S, anchors, BLOCK)
        calls += 1
        el = time.perf_counter() - t0
        if el >= seconds:
            break
    return nq * calls / el, calls, el


def cpu_sample(seconds=12.0):
    """The GPU arm's ``cpu_baseline`` leg: CPURound steps after one warm-up step until
    ``seconds`` of host time. Returns (query-tok/s, steps, seconds, CPURound)."""
    rnd = CPURound(steps_total=64)
    rnd.step()
    steps, t0 = 0, time.perf_counter()
    while True:
        rnd.step()
        steps += 1
        el = time.perf_counter() - t0
        if el >= seconds or steps >= 60:
            break
    return rnd.units * steps / el, steps, el, rnd


def host_threads():
    try:
        return len(os.sched_getaffinity(0))
    except Exception:
        return os.cpu_count() or 1


def run_reference(args):
    """``--impl reference``: the reference's CPU round (CPURound) timed on the host
    threads, rank 0 only; other ranks exit without work. Each step is one measured
    sample step; ``ms_per_step`` is that measured time, not an extrapolation."""
    rank, world, _ = dist_env()
    if rank != 0:
        return
    rnd = CPURound(steps_total=args.warmup + args.steps)
    for _ in range(args.warmup):
        rnd.step()
    times = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        rnd.step()
        times.append(time.perf_counter() - t0)
    total = sum(times)
    value = rnd.units * args.steps / total
    ms = total / args.steps * 1e3
    print(json.dumps(dict(
        impl='reference', metric=METRIC, value=value, unit='query-tok/s', n_gpus=args.gpus, steps=args.steps,
        warmup=args.warmup, ms_per_step=ms, higher_is_better=True, scaling='weak', vs_baseline=None, dtype='f32',
        data='synthetic (seeded N(0,1); config 2 and 3 context draws)',
        config=dict(workload='cfg2 draft x5 layers + cfg3 verify x28 layers (+ begin/commit): the reference CPU '
                             'round on a quantile sample of the requests',
                    parallelism=f'{rnd.threads} host threads, rank 0 only'),
        sample=dict(query_units_per_step=rnd.units, full_step_query_units=query_units(), fraction=rnd.fraction,
                    measured_ms_per_sample_step=ms, draft_contexts=rnd.dctx, verify_contexts=rnd.vctx),
        cpu_baseline=dict(value=value, unit='query-tok/s', cores=rnd.threads, kind='port', sample=rnd.describe()),
        train_layout_cpu=dict(zip(('query_tok_per_s', 'calls', 'seconds'), cpu_train_layout(threads=rnd.threads)),
                              workload='config 4, whole workload per call: block_mask + dense SDPA per sequence, '
                                       'float32'),
        e2e=dict(value=value, unit='query-tok/s', h2d_bytes_per_step=0, d2h_bytes_per_step=0))), flush=True)


# --------------------------------------------------------------------------- ranks
def gather_stats(stats, world):
    """All ranks' stats rows [elapsed_ms, e2e_ms, device_status, launches, ...] -> [world, n]
    on the host (the main leg adds algorithmic bytes per step, copy-only ms and the
    verify context tokens as columns 4-6, config 5 tokens and seconds as 7-8).

    The only collective of the benchmark: one all_gather after timing (NCCL on GPUs)."""
    import torch
    import torch.distributed as dist
    if world == 1:
        return stats[None].cpu()
    gathered = [torch.zeros_like(stats) for _ in range(world)]
    dist.all_gather(gathered, stats)
    return torch.stack(gathered).cpu()


def aggregate_stats(allstats):
    """Whole-job numbers: the slowest rank's device times, OR of status bits, total launches."""
    status = 0
    for s in allstats[:, 2].tolist():
        status |= int(s)
    return dict(elapsed_ms=float(allstats[:, 0].max()), e2e_ms=float(allstats[:, 1].max()), status=status,
                launches=int(allstats[:, 3].sum()))


# --------------------------------------------------------------------------- GPU arm
def run_b200(args):
    import importlib
    import torch
    import torch.distributed as dist
    rank, world, local = dist_env()
    from datetime import timedelta
    device = torch.device('cuda', local)
    if world > 1:
        dist.init_process_group('nccl', timeout=timedelta(seconds=120), device_id=device)
    torch.cuda.set_device(device)
    pkg = importlib.import_module('qwen3-dspark_b200')
    pkg.read_device_status(clear=True)
    if args.case == 'round5':
        import torch
        res = round5_leg(pkg, device, rank, args.warmup)
        status = pkg.read_device_status(clear=True)
        # whole job: every rank's tokens over the slowest rank's device time, per loop kind
        row = torch.tensor([res['generated_tokens'], res['generated_tokens'] - ROUND5['requests'], res['total_s'],
                            res['graph_total_s'], res['pipelined_total_s'], res['prefill_s'], float(status),
                            res['rounds']], dtype=torch.float64, device=device)
        table = gather_stats(row, world)
        if rank == 0:
            gen_all, dec_all = float(table[:, 0].sum()), float(table[:, 1].sum())
            pre = float(table[:, 5].max())
            job = {}
            for name, col in (('eager', 2), ('graph', 3), ('pipelined', 4)):
                t_max = float(table[:, col].max())
                job[name] = dict(total_s=t_max, total_tok_per_s=gen_all / t_max,
                                 decode_tok_per_s=dec_all / max(t_max - pre, 1e-9))
            best = max(job.values(), key=lambda j: j['total_tok_per_s'])
            st = 0
            for x in table[:, 6].tolist():
                st |= int(x)
            print(json.dumps(_finite(dict(
                metric='config-5 greedy speculative decode: generated tokens/s (whole job)',
                value=best['total_tok_per_s'], unit='tok/s', n_gpus=world, steps=1, warmup=args.warmup,
                ms_per_step=best['total_s'] * 1e3 / max(res['rounds'], 1), higher_is_better=True, scaling='weak',
                dtype='bf16', data='synthetic (random weights, uniform-random prompt ids)',
                config=dict(workload=f'config 5: {ROUND5["requests"]} requests per GPU x {world} GPUs, prompts '
                                     f'{ROUND5["prompts"]} cycling, {ROUND5["new_tokens"]} new tokens each',
                            requests_total=ROUND5['requests'] * world, parallelism=f'dp{world}'),
                job=job, tok_per_s_per_gpu=best['total_tok_per_s'] / world,
                per_rank=dict(total_s=table[:, 2].tolist(), graph_total_s=table[:, 3].tolist(),
                              pipelined_total_s=table[:, 4].tolist(), prefill_s=table[:, 5].tolist(),
                              rounds=table[:, 7].tolist()),
                round5_rank0=res, device_status=st))), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.case == 'stochastic':
        res = stochastic_leg(pkg, device, args.warmup, iters=args.steps)
        status = pkg.read_device_status(clear=True)
        if rank == 0:
            print(json.dumps(_finite(dict(metric='on-device stochastic acceptance per verify round',
                                          value=res['achieved_gbs'], unit='GB/s', n_gpus=world, steps=args.steps,
                                          warmup=args.warmup, ms_per_step=res['ms'], higher_is_better=True,
                                          dtype='f64', data='synthetic', stochastic=res, device_status=status))),
                  flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.case == 'append':
        res = append_leg(pkg, device, args.warmup, iters=args.steps)
        status = pkg.read_device_status(clear=True)
        if rank == 0:
            print(json.dumps(_finite(dict(metric='fused draft-context append (prefill of config 5)',
                                          value=res['prefill']['kernel_tflops'], unit='TFLOP/s', n_gpus=world,
                                          steps=args.steps, warmup=args.warmup,
                                          ms_per_step=res['prefill']['fused_ms'], higher_is_better=True,
                                          dtype='bf16', data='synthetic', append=res, device_status=status))),
                  flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.case == 'markov':
        res = markov_leg(pkg, device, args.warmup, iters=args.steps)
        status = pkg.read_device_status(clear=True)
        if rank == 0:
            print(json.dumps(_finite(dict(metric='fused greedy Markov proposal per draft block',
                                          value=res['achieved_gbs'], unit='GB/s', n_gpus=world, steps=args.steps,
                                          warmup=args.warmup, ms_per_step=res['ms_per_block'], higher_is_better=True,
                                          dtype='bf16', data='synthetic', markov=res, device_status=status))),
                  flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.case == 'propose':
        res = propose_leg(pkg, device, args.warmup, iters=args.steps)
        status = pkg.read_device_status(clear=True)
        if rank == 0:
            print(json.dumps(_finite(dict(metric='stochastic Markov proposal per draft block',
                                          value=res['ms_per_block'], unit='ms', n_gpus=world, steps=args.steps,
                                          warmup=args.warmup, ms_per_step=res['ms_per_block'],
                                          higher_is_better=False, dtype='f64', data='synthetic', propose=res,
                                          device_status=status))), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.case == 'accept':
        res = accept_leg(pkg, device, args.warmup, iters=args.steps)
        status = pkg.read_device_status(clear=True)
        if rank == 0:
            print(json.dumps(_finite(dict(metric='on-device greedy accept (argmax + accept rule) per verify round',
                                          value=res['achieved_gbs'], unit='GB/s', n_gpus=world, steps=args.steps,
                                          warmup=args.warmup, ms_per_step=res['ms'], higher_is_better=True,
                                          dtype='bf16', data='synthetic', accept=res, device_status=status))),
                  flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.case in ('graph', 'graph5'):
        cfg = dict(GRAPH if args.case == 'graph' else GRAPH5)
        if args.layers:
            cfg['layers'] = min(cfg['layers'], args.layers)
        res = graph_leg(pkg, device, rank, args.warmup, args.steps, cfg)
        status = pkg.read_device_status(clear=True)
        if rank == 0:
            print(json.dumps(_finite(dict(metric='small-batch verify step, eager vs CUDA-graph replay',
                                          value=res['graph_query_tok_per_s'], unit='query-tok/s', n_gpus=world,
                                          steps=args.steps, warmup=args.warmup, ms_per_step=res['graph_ms_per_step'],
                                          higher_is_better=True, dtype='bf16', data='synthetic', graph=res,
                                          device_status=status))), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    if args.case == 'train':
        # config 4 alone (profiling and standalone measurement); rank 0 reports
        train = train_layout_leg(pkg, device, rank, args.warmup, iters=args.steps)
        status = pkg.read_device_status(clear=True)
        if rank == 0:
            print(json.dumps(_finite(dict(metric='cfg4 training-layout draft attention query-tok/s',
                                          value=train['query_tok_per_s'], unit='query-tok/s', n_gpus=world,
                                          steps=args.steps, warmup=args.warmup, ms_per_step=train['ms_per_launch'],
                                          higher_is_better=True, dtype='bf16', data='synthetic',
                                          train_layout=train, device_status=status))), flush=True)
        if world > 1:
            dist.barrier()
            dist.destroy_process_group()
        return
    dl = DRAFT['layers'] if args.case in ('round', 'draft') else 0
    vl = VERIFY['layers'] if args.case in ('round', 'verify') else 0
    if args.layers is not None:
        dl, vl = min(dl, args.layers), min(vl, args.layers)
    wl = Workload(pkg, device, rank, 2 * (args.warmup + args.steps) + 4, dl, vl)

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(device)

    for _ in range(args.warmup):
        wl.step()
    barrier()
    # ---- device-resident timed region (value) ----
    events = []
    start, end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with ClockSampler(local) as clocks:
        barrier()
        start.record()
        launches0 = pkg.launch_count()
        for _ in range(args.steps):
            wl.step(events)
        launches = pkg.launch_count() - launches0
        end.record()
        barrier()
    elapsed_ms = start.elapsed_time(end)
    # ---- end-to-end through the public API with pinned host buffers ----
    host = wl.pinned_host()
    for _ in range(args.warmup):
        wl.step_e2e(host)
    barrier()
    e_start, e_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e_start.record()
    for _ in range(args.steps):
        wl.step_e2e(host)
    e_end.record()
    barrier()
    e2e_ms = e_start.elapsed_time(e_end)
    # ---- the same host copies without kernels, every rank at once (the e2e limiter) ----
    for _ in range(2):
        wl.step_copies(host)
    barrier()
    c_start, c_end = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    c_start.record()
    for _ in range(args.steps):
        wl.step_copies(host)
    c_end.record()
    barrier()
    copy_ms = c_start.elapsed_time(c_end)
    # config 4 (training layout): its own roofline, reported beside the headline step
    train = train_layout_leg(pkg, device, rank, args.warmup) if args.case == 'round' else None
    # config 5 at its stated shape: 32 requests per GPU through the pipelined greedy loop
    r5 = round5_leg(pkg, device, rank, args.warmup, pipelined_only=True) if args.case == 'round' else None
    status = pkg.read_device_status(clear=True)
    # per-layer event durations inside the timed region
    per = {'draft': [], 'verify': []}
    vbytes = []
    for e0, e1, kind, ctx in events:
        per[kind].append(e0.elapsed_time(e1))
        if kind == 'verify':
            vbytes.append(wl.verify_layer_bytes(ctx))
    alg_bytes_step = (wl.draft_layer_bytes() * dl + sum(vbytes) / args.steps) if dl or vl else 0.0
    h2d_b, d2h_b = wl.host_bytes(host)
    stats = torch.tensor([elapsed_ms, e2e_ms, float(status), float(launches), alg_bytes_step, copy_ms,
                          float(sum(wl.verify_ctx)), float(r5['generated_tokens'] if r5 else 0),
                          float(r5['total_s'] if r5 else 0)], dtype=torch.float64, device=device)
    allstats = gather_stats(stats, world)
    if rank == 0:
        agg = aggregate_stats(allstats)
        max_ms, max_e2e = agg['elapsed_ms'], agg['e2e_ms']
        units = query_units(dl, vl) * args.steps * world
        value = units / (max_ms / 1e3)
        e2e_value = units / (max_e2e / 1e3)
        hbm, peak_kind = peaks()
        v_ms = statistics.mean(per['verify']) if per['verify'] else float('nan')
        v_bytes = statistics.mean(vbytes) if vbytes else float('nan')
        achieved = v_bytes / (v_ms / 1e3) / 1e9
        d_ms = statistics.mean(per['draft']) if per['draft'] else float('nan')
        d_achieved = wl.draft_layer_bytes() / (d_ms / 1e3) / 1e9
        h2d, d2h = wl.host_bytes(host)
        if args.no_cpu_baseline or world > 1:
            cpu_base = dict(value=None, unit='query-tok/s', cores=None, kind='port',
                            sample='not run: the CPU leg runs on rank 0 at N=1 only' if world > 1 else 'skipped')
        else:
            cpu_v, reps, el, rnd = cpu_sample(seconds=12.0)
            cpu_base = dict(value=cpu_v, unit='query-tok/s', cores=rnd.threads, kind='port',
                            sample=f'{reps} measured steps in {el:.1f} s; ' + rnd.describe())
            if train is not None:
                tv, tc, te = cpu_train_layout(threads=rnd.threads)
                train['cpu_query_tok_per_s'] = tv
                train['cpu_sample'] = (f'{tc} calls of the whole config-4 workload in {te:.1f} s on {rnd.threads} '
                                       'threads: block_mask + dense SDPA per sequence, float32')
        line = dict(
            metric=METRIC, value=value, unit='query-tok/s', n_gpus=world, steps=args.steps, warmup=args.warmup,
            ms_per_step=max_ms / args.steps, higher_is_better=True, scaling='weak', vs_baseline=None, dtype='bf16',
            data='synthetic: config-2 K/V projected by a random-init 0.6B draft from N(0,1) features; '
                 'config-3 seeded N(0,1) q/k/v and KV cache',
            config=dict(workload=f'cfg2 draft x{dl} layers + cfg3 verify x{vl} layers (+ commit/rollback) per step',
                        draft_requests=DRAFT['requests'], draft_ctx='U[128,4096] seed 1', verify_requests=VERIFY['requests'],
                        verify_ctx='U[256,8192] seed 2', verify_q=VERIFY['q'], heads='16/8', head_dim=D,
                        rope_theta=1e6, rms_eps=1e-6, parallelism=f'dp{world} (independent request batches)',
                        l2='inputs larger than L2 (~62 GB resident KV per GPU)'),
            roofline=dict(kernel='verify layer: qk-norm/rope/append + bottom-right attention + split merge',
                          bound='hbm', achieved=achieved, peak=hbm, unit='GB/s', frac=achieved / hbm,
                          peak_source=f'{peak_kind} hbm_gbs', traffic=captured_traffic('verify_layer_cfg3'),
                          traffic_source='ncu capture of one cfg3 verify layer (profiles/)',
                          alg_bytes_per_launch=v_bytes, avg_launch_ms=v_ms),
            draft_roofline=dict(kernel='draft layer: non-causal attention + split merge', achieved=d_achieved,
                                frac=d_achieved / hbm, alg_bytes_per_launch=wl.draft_layer_bytes(), avg_launch_ms=d_ms,
                                traffic=captured_traffic('draft_layer_cfg2')),
            cpu_baseline=cpu_base,
            e2e=dict(value=e2e_value, unit='query-tok/s', h2d_bytes_per_step=h2d, d2h_bytes_per_step=d2h,
                     path='B200DraftKernel / B200PersistentTargetKV.verify_layer with pinned host q/k/v in, '
                          'attention outputs out; copies on two copy streams overlapping the kernels'),
            gpu_launches=agg['launches'], clocks=clocks.summary(), device_status=agg['status'],
            per_rank=dict(ms_per_step=[x / args.steps for x in allstats[:, 0].tolist()],
                          e2e_ms_per_step=[x / args.steps for x in allstats[:, 1].tolist()],
                          copy_only_ms_per_step=[x / args.steps for x in allstats[:, 5].tolist()],
                          alg_gb_per_step=[x / 1e9 for x in allstats[:, 4].tolist()],
                          device_gbs=[b / (ms / args.steps) / 1e6 for b, ms in
                                      zip(allstats[:, 4].tolist(), allstats[:, 0].tolist())],
                          host_copy_gbs=[(h2d_b + d2h_b) / (ms / args.steps) / 1e6
                                         for ms in allstats[:, 5].tolist()],
                          verify_context_tokens=[int(x) for x in allstats[:, 6].tolist()]))
        if train is not None:
            line['train_layout'] = train
        if r5 is not None:
            gen_all, t_max = float(allstats[:, 7].sum()), float(allstats[:, 8].max())
            line['round5'] = dict(workload=r5['workload'] + f' per GPU x {world} GPUs',
                                  generated_tok_per_s=gen_all / t_max, tok_per_s_per_gpu=gen_all / t_max / world,
                                  total_s=t_max, rounds=r5['rounds'], timing='CUDA events, slowest rank')
        print(json.dumps(_finite(line)), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--gpus', type=int, default=1)
    ap.add_argument('--steps', type=int, default=30)
    ap.add_argument('--warmup', type=int, default=5)
    ap.add_argument('--impl', default='b200', choices=['b200', 'reference'])
    ap.add_argument('--case', default='round', choices=['round', 'draft', 'verify', 'train', 'graph', 'accept', 'markov', 'propose', 'append', 'round5', 'graph5', 'stochastic'])
    ap.add_argument('--layers', type=int, default=None, help='cap the layer count of each selected path')
    ap.add_argument('--no-cpu-baseline', action='store_true', help='skip the timed CPU oracle leg')
    args = ap.parse_args()
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == 'reference':
        run_reference(args)
    else:
        run_b200(args)


if __name__ == '__main__':
    main()
