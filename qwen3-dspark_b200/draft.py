"""B200 packed draft: DSpark block drafting over a paged projected-context pool.

Mirrors ``PackedDraft`` (dspark_qwen/packed_draft.py:63-252) for inference:
``add_request`` / ``append_committed`` / ``crop`` / ``remove_request`` /
``backbone`` / ``propose_greedy``. What changes is the cache layout and the
attention call:

* the projected context K/V of every draft layer live in a request-contiguous
  pool (slot ``s`` owns rows ``[slot_row[s], slot_row[s] + capacity[s])``);
  ``append_committed`` writes new rows in place and ``crop`` only moves a
  length, where the reference concatenates the whole cache on every append
  (packed_draft.py:146-158) and filters it on every crop (:170-179);
* ``backbone`` attends over the pool rows and the block rows through the
  two-source kernel (``segment_attention``), where the reference concatenates
  cache + block and gathers every request's rows into packed K/V for each
  layer (:215-226).

``DSparkDraftModel`` holds the draft weights with the same module and
parameter names as ``DSparkDraft`` (dspark_qwen/model.py:27-99), so its
state dict loads unchanged; ``embedding`` and ``lm_head`` are the target's.
"""
from dataclasses import dataclass, field

import math

import torch
from torch import nn
from transformers.models.qwen3.modeling_qwen3 import Qwen3MLP, Qwen3RMSNorm, Qwen3RotaryEmbedding

from .kernels import (HEAD_DIM, HKV, HQ, add_rms_norm, draft_append, rope_cache, float64_law, markov_greedy, merged_mlp_ready, qk_norm_rope,
                      rms_norm, sample_rows, segment_attention, silu_mul, stochastic_propose)
from .kv_store import _upload


def rotate_half_rope(x, cos, sin):
    """x * cos + rotate_half(x) * sin over the last dim; cos/sin broadcast over heads
    (the draft's ``rotate``, dspark_qwen/model.py:22-24)."""
    half = x.shape[-1] // 2
    rot = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos[:, None] + rot * sin[:, None]


@dataclass(frozen=True)
class DraftSpec:
    """The draft geometry fields of ``DraftConfig`` (dspark_qwen/config.py:5-14)."""
    layer_ids: tuple = (1, 7, 14, 21, 26)
    num_layers: int = 5
    block_size: int = 7
    markov_rank: int = 256
    mask_token_id: int = 151669


class _DraftAttention(nn.Module):
    def __init__(self, config):
        super().__init__()
        h = config.hidden_size
        self.heads, self.kv_heads, self.dim = config.num_attention_heads, config.num_key_value_heads, config.head_dim
        self.q_proj = nn.Linear(h, self.heads * self.dim, bias=config.attention_bias)
        self.k_proj = nn.Linear(h, self.kv_heads * self.dim, bias=config.attention_bias)
        self.v_proj = nn.Linear(h, self.kv_heads * self.dim, bias=config.attention_bias)
        self.o_proj = nn.Linear(self.heads * self.dim, h, bias=config.attention_bias)
        self.q_norm = Qwen3RMSNorm(self.dim, eps=config.rms_norm_eps)
        self.k_norm = Qwen3RMSNorm(self.dim, eps=config.rms_norm_eps)

    def project_kv(self, states, cos, sin):
        """[1, n, hidden] -> roped K [n, Hkv, D], V [n, Hkv, D] (model.py:41-45)."""
        n = states.shape[1]
        k = self.k_norm(self.k_proj(states).view(1, n, self.kv_heads, self.dim)).transpose(1, 2)
        v = self.v_proj(states).view(1, n, self.kv_heads, self.dim).transpose(1, 2)
        return rotate_half_rope(k, cos, sin)[0].transpose(0, 1), v[0].transpose(0, 1)

    def project_q(self, states, cos, sin):
        n = states.shape[1]
        q = self.q_norm(self.q_proj(states).view(1, n, self.heads, self.dim)).transpose(1, 2)
        return rotate_half_rope(q, cos, sin)[0].transpose(0, 1)


class _DraftBlock(nn.Module):
    def __init__(self, config):
        super().__init__()
        self.input_norm = Qwen3RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.attention = _DraftAttention(config)
        self.post_norm = Qwen3RMSNorm(config.hidden_size, eps=config.rms_norm_eps)
        self.mlp = Qwen3MLP(config)


class DSparkDraftModel(nn.Module):
    """Draft weights with ``DSparkDraft``'s module tree; ``target`` supplies embedding/lm_head."""

    def __init__(self, target, spec):
        super().__init__()
        c = target.config
        if not spec.layer_ids or any(not 0 <= i < c.num_hidden_layers - 1 for i in spec.layer_ids):
            raise ValueError('Draft layer_ids must be intermediate target layers')
        if not 0 <= spec.mask_token_id < c.vocab_size:
            raise ValueError('mask_token_id outside target vocabulary')
        self.spec = spec
        self.fc = nn.Linear(len(spec.layer_ids) * c.hidden_size, c.hidden_size, bias=False)
        self.context_norm = Qwen3RMSNorm(c.hidden_size, eps=c.rms_norm_eps)
        self.layers = nn.ModuleList([_DraftBlock(c) for _ in range(spec.num_layers)])
        self.norm = Qwen3RMSNorm(c.hidden_size, eps=c.rms_norm_eps)
        self.rotary = Qwen3RotaryEmbedding(c)
        self.markov_embedding = nn.Embedding(c.vocab_size, spec.markov_rank)
        self.markov_projection = nn.Linear(spec.markov_rank, c.vocab_size, bias=False)
        self.confidence = nn.Linear(c.hidden_size + spec.markov_rank, 1)
        self.embedding = target.get_input_embeddings().requires_grad_(False)
        self.lm_head = target.get_output_embeddings().requires_grad_(False)


@dataclass
class DraftFeatures:
    hidden: torch.Tensor          # [requests * block, hidden]
    requests: tuple
    block_size: int
    context_lengths: tuple
    work: dict = field(default_factory=dict)

    def for_request(self, request):
        i = self.requests.index(request)
        return self.hidden[i * self.block_size:(i + 1) * self.block_size]


class B200PackedDraft:
    """Inference-only packed draft with a paged context pool in ``kv_dtype``.

    ``kv_dtype`` is the attention dtype: float32 (exact path) or bfloat16, where
    the reference keeps the cache in the projection dtype and casts it at the
    attention boundary on every call (packed_draft.py:222-235); casting once at
    append time gives the same values.
    """

    def __init__(self, draft, *, max_requests, context_capacity, kv_dtype=None, slot_capacities=None):
        if draft.training:
            raise ValueError('Packed draft is inference-only; call eval first')
        self.draft = draft
        self.device = draft.fc.weight.device
        if self.device.type != 'cuda':
            raise RuntimeError('B200 packed draft requires a CUDA device; no CPU fallback')
        att = draft.layers[0].attention
        if (att.heads, att.kv_heads, att.dim) != (HQ, HKV, HEAD_DIM):
            raise ValueError('B200 draft attention supports Hq16/Hkv8/D128')
        self.kv_dtype = kv_dtype or draft.fc.weight.dtype
        if self.kv_dtype not in (torch.bfloat16, torch.float32):
            raise ValueError('Draft KV dtype must be bfloat16 or float32')
        caps = [context_capacity] * max_requests if slot_capacities is None else [int(c) for c in slot_capacities]
        if len(caps) != max_requests or any(c < 1 for c in caps):
            raise ValueError('One positive capacity per request slot required')
        rows = [0]
        for c in caps:
            rows.append(rows[-1] + c)
        if rows[-1] >= 2 ** 31:
            raise ValueError('Draft pool rows exceed the int32 row index')
        self.capacities, self.slot_rows = tuple(caps), tuple(rows[:-1])
        # one extra row no slot owns: the fixed-shape append writes its unused rows there
        self.trash_row = rows[-1]
        shape = (rows[-1] + 1, HKV, HEAD_DIM)
        self.pool_k = [torch.zeros(shape, dtype=self.kv_dtype, device=self.device) for _ in draft.layers]
        self.pool_v = [torch.zeros(shape, dtype=self.kv_dtype, device=self.device) for _ in draft.layers]
        self._slots = {}          # request -> slot index
        self._lengths = {}
        self._free = list(range(max_requests))
        self.last_projection_work = None

    # -- request lifecycle (packed_draft.py:89-101,170-184) -----------------------
    @property
    def lengths(self):
        return dict(self._lengths)

    def add_request(self, request):
        if not isinstance(request, str) or not request or request in self._slots:
            raise ValueError('Require a fresh nonempty request name')
        if not self._free:
            raise ValueError('Draft pool slots exhausted')
        self._slots[request] = self._free.pop(0)
        self._lengths[request] = 0

    def _request(self, request):
        if request not in self._slots:
            raise KeyError(request)

    def crop(self, request, length):
        self._request(request)
        if type(length) is not int or not 0 <= length <= self._lengths[request]:
            raise ValueError('Invalid committed draft crop length')
        self._lengths[request] = length          # rows past length are never read

    def remove_request(self, request):
        self._request(request)
        self._free.append(self._slots.pop(request))
        self._free.sort()
        del self._lengths[request]

    def request_kv(self, request):
        """Per draft layer (K, V) [n, Hkv, D] of the request's committed context."""
        self._request(request)
        r0, n = self.slot_rows[self._slots[request]], self._lengths[request]
        return tuple((k[r0:r0 + n].clone(), v[r0:r0 + n].clone()) for k, v in zip(self.pool_k, self.pool_v))

    # -- bf16 norms in one launch each ---------------------------------------------
    @staticmethod
    def _norm(module, x):
        """``module(x)`` for a Qwen3RMSNorm; bf16 activations and weights take the fused
        ``rms_norm`` launch (the same rounding steps) instead of transformers' eight
        kernels. The draft module itself is left as it is (its training forward keeps
        autograd through transformers' norm)."""
        if x.dtype == torch.bfloat16 and module.weight.dtype == torch.bfloat16:
            return rms_norm(x, module.weight, module.variance_epsilon)
        return module(x)

    def _mlp(self, mlp, x):
        """``mlp(x)``; a bf16 Qwen3MLP runs gate and up as one GEMM over a merged copy of
        the two weights and ``silu_mul``. The copy is rebuilt when either weight
        changes; replaced copies stay allocated, since a captured proposal keeps
        reading the copy it was captured with."""
        if x.dtype != torch.bfloat16 or not merged_mlp_ready(mlp):
            return mlp(x)
        cache = self.__dict__.setdefault('_merged_mlp', {})
        key = tuple((t.data_ptr(), t._version) for t in (mlp.gate_proj.weight, mlp.up_proj.weight))
        hit = cache.get(id(mlp))
        if hit is None or hit[0] != key:
            if hit is not None:
                self.__dict__.setdefault('_retired_mlp', []).append(hit[1])
            hit = (key, torch.cat((mlp.gate_proj.weight, mlp.up_proj.weight)).detach().contiguous())
            cache[id(mlp)] = hit
        return mlp.down_proj(silu_mul(torch.nn.functional.linear(x, hit[1]), mlp.gate_proj.out_features))

    @staticmethod
    def _add_norm(module, z, delta):
        """``(z + delta, module(z + delta))``; bf16 as one ``add_rms_norm`` launch."""
        if z.dtype == delta.dtype == module.weight.dtype == torch.bfloat16:
            return add_rms_norm(z, delta, module.weight, module.variance_epsilon)
        z = z + delta
        return z, module(z)

    def _project(self, att, x, cos, sin):
        """``att.project_q`` and ``att.project_kv`` (model.py:41-45): q [n, Hq, D], k and v
        [n, Hkv, D]. bf16 drafts run the q/k norms and RoPE as one ``qk_norm_rope``
        launch; other dtypes take transformers' norms and the torch rotation."""
        n = x.shape[1]
        if (x.dtype == cos.dtype == torch.bfloat16 and att.dim == HEAD_DIM
                and att.q_norm.weight.dtype == att.k_norm.weight.dtype == torch.bfloat16):
            q, k = qk_norm_rope(att.q_proj(x)[0], att.k_proj(x)[0], att.q_norm.weight, att.k_norm.weight,
                                att.q_norm.variance_epsilon, att.k_norm.variance_epsilon, cos[0], sin[0],
                                att.heads, att.kv_heads)
            return q, k, att.v_proj(x)[0].view(n, att.kv_heads, att.dim)
        q = self._norm(att.q_norm, att.q_proj(x).view(1, n, att.heads, att.dim)).transpose(1, 2)
        k = self._norm(att.k_norm, att.k_proj(x).view(1, n, att.kv_heads, att.dim)).transpose(1, 2)
        v = att.v_proj(x).view(1, n, att.kv_heads, att.dim).transpose(1, 2)
        return (rotate_half_rope(q, cos, sin)[0].transpose(0, 1), rotate_half_rope(k, cos, sin)[0].transpose(0, 1),
                v[0].transpose(0, 1))

    # -- context append (packed_draft.py:129-168) ---------------------------------
    def _fused_append_ready(self):
        d = self.draft
        att = d.layers[0].attention
        return (self.kv_dtype == torch.bfloat16 and d.fc.weight.dtype == torch.bfloat16
                and att.k_proj.bias is None and att.v_proj.bias is None and len(d.layers) <= 8
                and d.fc.out_features % 64 == 0 and float(getattr(d.rotary, 'attention_scaling', 1.0)) == 1.0)

    def _append_operands(self):
        """Stacked [k_proj; v_proj] weights of every layer, the stacked k_norm weights and
        the rotary cos/sin cache (``rope_cache``) for the fused append, rebuilt when one
        changes. A captured append reads the stacks made when it was captured. The cache
        covers every slot position plus a margin for the uncommitted rows of a
        fixed-shape chunk (they sit past the slot's length and land in the trash row)."""
        d = self.draft
        params = [t for layer in d.layers for t in (layer.attention.k_proj.weight, layer.attention.v_proj.weight,
                                                    layer.attention.k_norm.weight)] + [d.rotary.inv_freq]
        key = tuple((t.data_ptr(), t._version) for t in params)
        if getattr(self, '_append_key', None) != key:
            self._kv_weight = torch.cat([torch.cat((layer.attention.k_proj.weight, layer.attention.v_proj.weight))
                                         for layer in d.layers]).contiguous()
            self._k_norm_w = torch.stack([layer.attention.k_norm.weight for layer in d.layers]).contiguous()
            self._rope = rope_cache(d.rotary.inv_freq.float(), max(self.capacities) + 1024, self.device)
            self._append_key = key
        return self._kv_weight, self._k_norm_w, self._rope

    def _append_rows(self, feat, meta, r, n):
        """Project n feature rows [1, n, F] and write them into the pool. ``meta`` is an
        int32 device vector [4r + 1]: cu_rows (r + 1), slot_row, ctx_len, count (r each);
        row j of request i sits at position ctx_len[i] + j and is written to its slot
        when j < count[i], else to the trash row. No host reads: capturable."""
        d = self.draft
        context = self._norm(d.context_norm, d.fc(feat.to(d.fc.weight.dtype)))
        if self._fused_append_ready():
            kv_weight, k_norm_w, rope = self._append_operands()
            draft_append(context[0], kv_weight, k_norm_w, rope, meta, r, self.pool_k, self.pool_v,
                         self.trash_row, d.layers[0].attention.k_norm.variance_epsilon)
            return
        cu, slot, ctx, cnt = (meta[:r + 1].long(), meta[r + 1:2 * r + 1].long(), meta[2 * r + 1:3 * r + 1].long(),
                              meta[3 * r + 1:].long())
        g = torch.arange(n, device=self.device)
        i = torch.searchsorted(cu[1:].contiguous(), g, right=True)
        j = g - cu[i]
        pos = ctx[i] + j
        cos, sin = d.rotary(context, pos[None])
        idx = torch.where(j < cnt[i], slot[i] + pos, torch.full_like(pos, self.trash_row))
        for layer, pk, pv in zip(d.layers, self.pool_k, self.pool_v):
            k, v = layer.attention.project_kv(context, cos, sin)
            pk.index_copy_(0, idx, k.to(self.kv_dtype))
            pv.index_copy_(0, idx, v.to(self.kv_dtype))

    @torch.no_grad()
    def append_committed(self, chunks):
        """Project committed target features [1, n, F] once and write K/V rows in place."""
        if not chunks:
            raise ValueError('Require at least one committed feature chunk')
        d = self.draft
        features, cu, slots, starts, counts = [], [0], [], [], []
        for request, value in chunks.items():
            self._request(request)
            if (not isinstance(value, torch.Tensor) or value.ndim != 3 or value.shape[0] != 1 or value.shape[1] < 1
                    or value.shape[2] != d.fc.in_features or value.device != self.device
                    or not value.is_floating_point()):
                raise ValueError('Expected nonempty [1, tokens, target_features] on draft device')
            n, start = value.shape[1], self._lengths[request]
            slot = self._slots[request]
            if start + n > self.capacities[slot]:
                raise ValueError('Draft context exceeds the request slot capacity')
            features.append(value)
            cu.append(cu[-1] + n)
            slots.append(self.slot_rows[slot])
            starts.append(start)
            counts.append(n)
        r = len(chunks)
        meta = _upload(cu + slots + starts + counts, self.device)
        self._append_rows(torch.cat(features, dim=1), meta, r, cu[-1])
        for request, n in zip(chunks, counts):
            self._lengths[request] += n
        self.last_projection_work = dict(requests=r, new_context_tokens=cu[-1], context_projection_calls=1,
                                         kv_projection_calls=1 if self._fused_append_ready() else len(d.layers),
                                         cache_concatenation_kv_bytes=0)

    # -- fixed-shape append of whole verified chunks (capturable) -------------------
    def _verified_meta(self, requests, counts, q):
        for request in requests:
            self._request(request)
        n = [int(c) for c in counts]
        if len(n) != len(requests) or any(not 0 <= c <= q for c in n) or any(
                self._lengths[x] + c > self.capacities[self._slots[x]] for x, c in zip(requests, n)):
            raise ValueError('Committed counts must lie in [0, q] and fit the slot capacity')
        r = len(requests)
        host = ([q * i for i in range(r + 1)] + [self.slot_rows[self._slots[x]] for x in requests]
                + [self._lengths[x] for x in requests] + n)
        return host, n

    @torch.no_grad()
    def append_verified(self, features, requests, counts):
        """``append_committed`` of a round whose verified chunks all have q rows:
        ``features`` [1, len(requests) * q, F] in request order, of which the first
        ``counts[i]`` rows of request i are committed. Fixed shapes and no host-side
        slicing: every row is projected, uncommitted rows go to the trash row."""
        r = len(requests)
        if (features.ndim != 3 or r < 1 or features.shape[1] % r or features.shape[1] == 0
                or features.shape[2] != self.draft.fc.in_features or features.device != self.device):
            raise ValueError('Expected [1, requests * q, target_features] verified features')
        q = features.shape[1] // r
        host, n = self._verified_meta(requests, counts, q)
        self._append_rows(features, _upload(host, self.device), r, r * q)
        for request, c in zip(requests, n):
            self._lengths[request] += c

    @torch.no_grad()
    def capture_append(self, num_requests, width):
        """Capture ``append_verified`` for ``num_requests`` chunks of ``width`` rows
        into a CUDA graph reading fixed feature and metadata buffers."""
        graphs = self.__dict__.setdefault('_append_graphs', {})
        key = (num_requests, width)
        if key in graphs:
            raise ValueError('Append shape already captured')
        r, q = num_requests, width
        feat = torch.zeros((1, r * q, self.draft.fc.in_features), dtype=self.draft.fc.weight.dtype,
                           device=self.device)
        host = [q * i for i in range(r + 1)] + [self.trash_row] * r + [0] * r + [0] * r
        meta = torch.tensor(host, dtype=torch.int32, device=self.device)   # warm-up writes only the trash row
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):
            self._append_rows(feat, meta, r, r * q)
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            self._append_rows(feat, meta, r, r * q)
        graphs[key] = dict(graph=graph, feat=feat, meta=meta)
        return graph

    @torch.no_grad()
    def append_verified_graph(self, features, requests, counts):
        """``append_verified`` through the program captured for its shape."""
        r = len(requests)
        q = features.shape[1] // max(r, 1)
        ex = self.__dict__.get('_append_graphs', {}).get((r, q))
        if ex is None or features.shape != ex['feat'].shape:
            raise ValueError('Capture the append shape first')
        host, n = self._verified_meta(requests, counts, q)
        ex['feat'].copy_(features)
        ex['meta'].copy_(torch.tensor(host, dtype=torch.int32).pin_memory(), non_blocking=True)
        ex['graph'].replay()
        for request, c in zip(requests, n):
            self._lengths[request] += c

    # -- backbone (packed_draft.py:186-252) -----------------------------------------
    @torch.no_grad()
    def backbone(self, anchors):
        """One 7-row block per request: anchor + mask tokens at positions len..len+6."""
        if not anchors:
            raise ValueError('Require active anchor requests')
        d, size = self.draft, self.draft.spec.block_size
        requests = tuple(anchors)
        tokens, positions = [], []
        for request, anchor in anchors.items():
            self._request(request)
            if (not isinstance(anchor, torch.Tensor) or anchor.shape != (1, 1) or anchor.dtype != torch.long
                    or anchor.device != self.device):
                raise ValueError('Require one [1,1] long anchor per active request')
            block = anchor.new_full((1, size), d.spec.mask_token_id)
            block[:, :1] = anchor
            tokens.append(block)
            start = self._lengths[request]
            positions.extend(range(start, start + size))
        r = len(requests)
        cu = [size * i for i in range(r + 1)]
        meta = _upload(cu + [self.slot_rows[self._slots[q]] for q in requests]
                       + [self._lengths[q] for q in requests] + [size] * r, self.device)
        cu_q, a_start, a_len, b_len = meta[:r + 1], meta[r + 1:2 * r + 1], meta[2 * r + 1:3 * r + 1], meta[3 * r + 1:]
        b_start = cu_q[:r]
        z = d.embedding(torch.cat(tokens, dim=1)).to(d.fc.weight.dtype)
        pos = torch.tensor(positions, dtype=torch.long, device=self.device)
        cos, sin = d.rotary(z, pos[None])
        qlens = [size] * r
        pending = None                      # the last MLP output, added in the next norm's launch
        for layer, pk, pv in zip(d.layers, self.pool_k, self.pool_v):
            att = layer.attention
            if pending is None:
                x = self._norm(layer.input_norm, z)
            else:
                z, x = self._add_norm(layer.input_norm, z, pending)
            q, kb, vb = self._project(att, x, cos, sin)
            q = q.to(self.kv_dtype).contiguous()
            out = segment_attention(q, cu_q, qlens, pk, pv, a_start, a_len, kb.to(self.kv_dtype).contiguous(),
                                    vb.to(self.kv_dtype).contiguous(), b_start, b_len, causal=False)
            z, x = self._add_norm(layer.post_norm, z, att.o_proj(out.to(z.dtype).reshape(1, r * size, -1)))
            pending = self._mlp(layer.mlp, x)
        hidden = (self._norm(d.norm, z) if pending is None else self._add_norm(d.norm, z, pending)[1])[0]
        work = dict(requests=r, query_rows=r * size, attention_calls=len(d.layers),
                    context_block_concatenation_kv_bytes=0, gathered_kv_bytes=0)
        return DraftFeatures(hidden, requests, size, tuple(self._lengths[q] for q in requests), work)

    # -- captured proposal (fixed buffers, one CUDA graph per request count) ----------
    def _propose_body(self, anchor_buf, pos_buf, meta, r):
        """Backbone + LM head + greedy Markov loop over fixed-address inputs (bf16 drafts
        whose Markov head runs on the fused kernel)."""
        d, size = self.draft, self.draft.spec.block_size
        hidden, base = self._backbone_body(anchor_buf, pos_buf, meta, r)
        return markov_greedy(d.markov_projection.weight, d.markov_embedding.weight, d.confidence.weight.reshape(-1),
                             self._confidence_bias(), hidden, base, anchor_buf, size)

    def _stochastic_positions(self, base, prev, uniforms, temperature, steps):
        """Positions 0..steps-1 of the stochastic proposal for all r requests (bf16
        drafts): per position the embedding of the previous token, the Markov
        projection and one ``stochastic_propose`` launch writing the float64 law and
        drawing the token. Every position runs over all rows, whatever their limits, so
        the eager and the captured proposal compute the same things; the caller keeps
        each request's first limits[i] positions. Returns tokens [r, size] int64, laws
        [r, size, V] float64 and status [r, size] int32 (positions past ``steps`` are
        not written)."""
        d = self.draft
        r, size, vocab = base.shape
        laws = torch.empty((r, size, vocab), dtype=torch.float64, device=self.device)
        toks = torch.zeros((r, size), dtype=torch.long, device=self.device)
        status = torch.zeros((r, size), dtype=torch.int32, device=self.device)
        rows = torch.arange(r, dtype=torch.int32, device=self.device)
        for k in range(steps):
            proj = d.markov_projection(d.markov_embedding(prev)).contiguous()
            tok, st = stochastic_propose(base[:, k], rows, proj, temperature, uniforms[:, k].contiguous(), laws[:, k])
            toks[:, k] = tok
            status[:, k] = st
            prev = tok
        return toks, laws, status

    def _propose_stochastic_body(self, anchor_buf, pos_buf, meta, r, u_buf, temperature):
        """Backbone + LM head + every block position's law and draw over fixed-address
        inputs (the captured stochastic proposal)."""
        size = self.draft.spec.block_size
        hidden, base = self._backbone_body(anchor_buf, pos_buf, meta, r)
        return self._stochastic_positions(base.view(r, size, -1), anchor_buf, u_buf, temperature, size)

    def _backbone_body(self, anchor_buf, pos_buf, meta, r):
        """Backbone + final norm + LM head over fixed-address inputs: (hidden [r * block,
        H], base logits [r * block, V])."""
        d, size = self.draft, self.draft.spec.block_size
        cu_q, a_start, a_len, b_len = meta[:r + 1], meta[r + 1:2 * r + 1], meta[2 * r + 1:3 * r + 1], meta[3 * r + 1:]
        b_start = cu_q[:r]
        block = torch.full((r, size), d.spec.mask_token_id, dtype=torch.long, device=self.device)
        block[:, 0] = anchor_buf
        z = d.embedding(block.reshape(1, r * size)).to(d.fc.weight.dtype)
        cos, sin = d.rotary(z, pos_buf[None])
        qlens = [size] * r
        pending = None                      # the last MLP output, added in the next norm's launch
        for layer, pk, pv in zip(d.layers, self.pool_k, self.pool_v):
            att = layer.attention
            if pending is None:
                x = self._norm(layer.input_norm, z)
            else:
                z, x = self._add_norm(layer.input_norm, z, pending)
            q, kb, vb = self._project(att, x, cos, sin)
            q = q.to(self.kv_dtype).contiguous()
            out = segment_attention(q, cu_q, qlens, pk, pv, a_start, a_len, kb.to(self.kv_dtype).contiguous(),
                                    vb.to(self.kv_dtype).contiguous(), b_start, b_len, causal=False)
            z, x = self._add_norm(layer.post_norm, z, att.o_proj(out.to(z.dtype).reshape(1, r * size, -1)))
            pending = self._mlp(layer.mlp, x)
        hidden = (self._norm(d.norm, z) if pending is None
                  else self._add_norm(d.norm, z, pending)[1])[0].contiguous()
        return hidden, d.lm_head(hidden).contiguous()

    def _graph_ready(self):
        d = self.draft
        rank = d.markov_projection.weight.shape[1]
        return (d.markov_projection.weight.dtype == torch.bfloat16 and self.kv_dtype == torch.bfloat16
                and rank % 64 == 0 and rank <= 256 and d.markov_projection.weight.shape[0] % 8 == 0)

    @torch.no_grad()
    def capture_propose(self, num_requests):
        """Capture ``propose_greedy`` for ``num_requests`` requests into a CUDA graph:
        anchors, block positions and the attention metadata live in fixed buffers that
        ``propose_greedy_graph`` fills each round (bf16 drafts with the fused Markov
        head)."""
        if not self._graph_ready():
            raise ValueError('Graph proposal needs a bf16 draft whose Markov head runs on the fused kernel')
        graphs = self.__dict__.setdefault('_graphs', {})
        if num_requests in graphs:
            raise ValueError('Request count already captured')
        r, size = num_requests, self.draft.spec.block_size
        anchor_buf = torch.zeros(r, dtype=torch.long, device=self.device)
        pos_buf = torch.arange(r * size, dtype=torch.long, device=self.device) % size
        meta = torch.tensor([size * i for i in range(r + 1)] + [self.slot_rows[0]] * r + [0] * r + [size] * r,
                            dtype=torch.int32, device=self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):                       # warm-up: handles, allocator, workspace
            self._propose_body(anchor_buf, pos_buf, meta, r)
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            toks, conf = self._propose_body(anchor_buf, pos_buf, meta, r)
        graphs[r] = dict(graph=graph, anchors=anchor_buf, pos=pos_buf, meta=meta, tokens=toks, conf=conf)
        return graph

    def _fill_propose(self, ex, anchors):
        """Writes a round's anchors, block positions and attention metadata into a
        captured proposal's fixed buffers."""
        size = self.draft.spec.block_size
        requests = tuple(anchors)
        positions = []
        for request, anchor in anchors.items():
            self._request(request)
            if (not isinstance(anchor, torch.Tensor) or anchor.shape != (1, 1) or anchor.dtype != torch.long
                    or anchor.device != self.device):
                raise ValueError('Require one [1,1] long anchor per active request')
            start = self._lengths[request]
            positions.extend(range(start, start + size))
        r = len(requests)
        host = ([size * i for i in range(r + 1)] + [self.slot_rows[self._slots[q]] for q in requests]
                + [self._lengths[q] for q in requests] + [size] * r)
        ex['meta'].copy_(torch.tensor(host, dtype=torch.int32).pin_memory(), non_blocking=True)
        ex['pos'].copy_(torch.tensor(positions, dtype=torch.long).pin_memory(), non_blocking=True)
        ex['anchors'].copy_(torch.cat([anchors[q].view(1) for q in requests]))
        return requests

    @torch.no_grad()
    def propose_greedy_graph(self, anchors, on_device=False):
        """``propose_greedy`` through the program captured for ``len(anchors)`` requests.
        ``on_device`` returns the program's output buffers (tokens [R, block] int64,
        confidences [R, block] float32, valid until the next replay) without a host
        read."""
        ex = self.__dict__.get('_graphs', {}).get(len(anchors))
        if ex is None:
            raise ValueError('Capture the request count first')
        requests = self._fill_propose(ex, anchors)
        ex['graph'].replay()
        if on_device:
            return ex['tokens'], ex['conf']
        toks, confs = ex['tokens'].tolist(), ex['conf'].tolist()
        return {q: (toks[i], confs[i]) for i, q in enumerate(requests)}

    @torch.no_grad()
    def capture_propose_stochastic(self, num_requests, temperature):
        """Capture the stochastic proposal (``propose_stochastic``) of ``num_requests``
        requests at ``temperature`` into a CUDA graph (bf16 drafts with the fused Markov
        head): anchors, block positions, attention metadata and the round's proposal
        uniforms live in fixed buffers that ``propose_stochastic_graph`` fills; every
        block position runs for every request and each request keeps its first
        limits[i] positions, as the eager proposal does."""
        if not self._graph_ready():
            raise ValueError('Graph proposal needs a bf16 draft whose Markov head runs on the fused kernel')
        temperature = float(temperature)
        if not math.isfinite(temperature) or temperature <= 0:
            raise ValueError('temperature must be finite and strictly positive')
        graphs = self.__dict__.setdefault('_sgraphs', {})
        key = (num_requests, temperature)
        if key in graphs:
            raise ValueError('Request count and temperature already captured')
        r, size = num_requests, self.draft.spec.block_size
        anchor_buf = torch.zeros(r, dtype=torch.long, device=self.device)
        pos_buf = torch.arange(r * size, dtype=torch.long, device=self.device) % size
        meta = torch.tensor([size * i for i in range(r + 1)] + [self.slot_rows[0]] * r + [0] * r + [size] * r,
                            dtype=torch.int32, device=self.device)
        u_buf = torch.zeros((r, size), dtype=torch.float64, device=self.device)
        side = torch.cuda.Stream(self.device)
        side.wait_stream(torch.cuda.current_stream(self.device))
        with torch.cuda.stream(side):                       # warm-up: handles, allocator, workspace
            self._propose_stochastic_body(anchor_buf, pos_buf, meta, r, u_buf, temperature)
        torch.cuda.current_stream(self.device).wait_stream(side)
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(graph, stream=side):
            toks, laws, status = self._propose_stochastic_body(anchor_buf, pos_buf, meta, r, u_buf, temperature)
        graphs[key] = dict(graph=graph, anchors=anchor_buf, pos=pos_buf, meta=meta, u=u_buf, tokens=toks, laws=laws,
                           status=status)
        return graph

    @torch.no_grad()
    def propose_stochastic_graph(self, anchors, limits, uniforms, temperature):
        """``propose_stochastic`` through the program captured for ``len(anchors)``
        requests and ``temperature``: the same ({request: tokens [n] long}, {request:
        laws [n, V] float64}), as views of the program's buffers (valid until its next
        replay). A non-finite logit raises."""
        ex = self.__dict__.get('_sgraphs', {}).get((len(anchors), float(temperature)))
        if ex is None:
            raise ValueError('Capture the request count and temperature first')
        size = self.draft.spec.block_size
        requests = tuple(anchors)
        n = [int(limits[q]) for q in requests]
        if any(not 0 <= x <= size for x in n) or uniforms.shape != (len(requests), size):
            raise ValueError('limits in [0, block_size] and [R, block_size] uniforms required')
        self._fill_propose(ex, anchors)
        ex['u'].copy_(uniforms)
        ex['graph'].replay()
        return self._stochastic_result(requests, n, ex['tokens'], ex['laws'], ex['status'])

    def _stochastic_result(self, requests, n, toks, laws, status):
        """Per request its first n[i] proposed tokens and laws; a non-finite logit at one
        of those positions raises."""
        size = toks.shape[1]
        keep = torch.arange(size, device=self.device)[None, :] < _upload(n, self.device)[:, None]
        if bool(((status != 0) & keep).any()):
            raise ValueError('Non-finite draft logits in a stochastic proposal')
        return ({q: toks[i, :n[i]] for i, q in enumerate(requests)},
                {q: laws[i, :n[i]] for i, q in enumerate(requests)})

    @torch.no_grad()
    def propose_stochastic(self, anchors, limits, uniforms, temperature):
        """Stochastic block proposal (DSparkDraft._sample_stochastic, dspark_qwen/model.py:
        193-208, batched over requests as propose_packed, packed_sampling.py:73-94): one
        backbone + LM head for all requests, then per position k < limits[r] the float64
        law q = softmax((base_k + markov_projection(emb(prev))) / T) (normalised twice)
        and a token drawn by the strict CDF rule with ``uniforms[i, k]`` (request i of
        ``anchors``' order). A bf16 draft runs each position's law and draw as one
        ``stochastic_propose`` launch writing into one float64 [R, block, V] buffer;
        other dtypes take the torch formula. Returns ({request: tokens [n] long},
        {request: laws [n, V] float64}) on the device; the raw confidence logits are not
        part of acceptance and are not computed. A non-finite logit raises."""
        d = self.draft
        requests = tuple(anchors)
        n = [int(limits[r]) for r in requests]
        size = d.spec.block_size
        if any(not 0 <= x <= size for x in n) or uniforms.shape != (len(requests), size):
            raise ValueError('limits in [0, block_size] and [R, block_size] uniforms required')
        feats = self.backbone(anchors)
        r = len(requests)
        hidden = feats.hidden.reshape(r, size, -1)
        base = d.lm_head(hidden.to(d.lm_head.weight.dtype))
        prev = torch.cat([anchors[q].view(1) for q in requests])
        steps = max(n) if n else 0
        vocab = base.shape[-1]
        fused = base.dtype == torch.bfloat16 and d.markov_projection.weight.dtype == torch.bfloat16
        if fused:
            toks, laws_buf, status = self._stochastic_positions(base, prev, uniforms.to(torch.float64), temperature,
                                                                steps)
            return self._stochastic_result(requests, n, toks, laws_buf, status)
        tokens = [[] for _ in requests]
        laws = [[] for _ in requests]
        for k in range(steps):
            rows = [i for i in range(r) if k < n[i]]
            idx = torch.tensor(rows, dtype=torch.long, device=self.device)
            emb = d.markov_embedding(prev[idx])
            logits = base[idx, k] + d.markov_projection(emb)
            law = float64_law(logits, temperature)
            tok = sample_rows(law, uniforms[idx, k])
            prev = prev.index_copy(0, idx, tok)
            for j, i in enumerate(rows):
                tokens[i].append(tok[j:j + 1])
                laws[i].append(law[j])
        empty_t = torch.empty(0, dtype=torch.long, device=self.device)
        empty_l = torch.empty((0, base.shape[-1]), dtype=torch.float64, device=self.device)
        return ({q: torch.cat(tokens[i]) if tokens[i] else empty_t for i, q in enumerate(requests)},
                {q: torch.stack(laws[i]) if laws[i] else empty_l for i, q in enumerate(requests)})

    @torch.no_grad()
    def _confidence_bias(self):
        """confidence.bias as a host float, read once per parameter version."""
        b = self.draft.confidence.bias
        key = (b.data_ptr(), b._version)
        if getattr(self, '_bias_key', None) != key:
            self._bias_value, self._bias_key = float(b.float().item()), key
        return self._bias_value

    def propose_greedy(self, anchors):
        """Greedy block proposal per request: serial Markov argmax over the block rows
        (DSparkDraft._sample_greedy, dspark_qwen/model.py:210-221), batched over requests.
        Returns {request: (tokens, confidences)}."""
        feats = self.backbone(anchors)
        d, size = self.draft, feats.block_size
        r = len(feats.requests)
        prev = torch.cat([anchors[q].view(1) for q in feats.requests])
        rank = d.markov_projection.weight.shape[1]
        if (d.markov_projection.weight.dtype == torch.bfloat16 and feats.hidden.dtype == torch.bfloat16
                and rank % 64 == 0 and rank <= 256 and d.markov_projection.weight.shape[0] % 8 == 0):
            # fused on-device Markov loop: one tcgen05 launch per block position
            hidden = feats.hidden.reshape(r * size, -1).contiguous()
            base = d.lm_head(hidden).contiguous()
            bias = self._confidence_bias()
            toks, confs = markov_greedy(d.markov_projection.weight, d.markov_embedding.weight,
                                        d.confidence.weight.reshape(-1), bias, hidden, base, prev, size)
            toks, confs = toks.tolist(), confs.tolist()
            return {q: (toks[i], confs[i]) for i, q in enumerate(feats.requests)}
        hidden = feats.hidden.view(r, size, -1)
        base = d.lm_head(hidden.to(d.lm_head.weight.dtype))
        tokens, conf = [], []
        for k in range(size):
            emb = d.markov_embedding(prev)
            conf.append(d.confidence(torch.cat((hidden[:, k].to(emb.dtype), emb), -1)).sigmoid().flatten())
            prev = (base[:, k] + d.markov_projection(emb).to(base.dtype)).argmax(-1)
            tokens.append(prev)
        toks = torch.stack(tokens, 1).tolist()
        confs = torch.stack(conf, 1).tolist()
        return {q: (toks[i], confs[i]) for i, q in enumerate(feats.requests)}
