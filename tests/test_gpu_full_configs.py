"""Parity at the benchmark's own shapes: BASELINE configs 2 (draft) and 3 (verify).

The bench times these exact workloads (``bench.contexts`` gives the same context lengths
here and there), so every request of the headline step is compared with the oracle:

* config 3: 128 requests, cached contexts ~ U{256..8192} (seed 2), 7 new rows each.
  Resident K = RoPE(k_norm(N(0,1))) at positions 0..c-1 built with transformers' own
  modules on the GPU, V ~ N(0,1). One verify layer through
  ``B200PersistentTargetKV.verify_layer`` (fused kernel and prep path; k/q norm weights
  of ones and a seeded N(1, 0.1) variant; theta 1e6, eps 1e-6): the appended K equals the
  oracle's k_norm + RoPE bit for bit, V is the raw v, and the attention output meets
  the bf16 gate against the oracle's two-source bottom-right attention
  (persistent_qwen_target.py:30-42). Then commit accept ~ U{0..6} (+ anchor): lengths
  and the committed windows equal ``OracleKVStore.commit`` bit for bit, and no other
  resident byte changes (persistent_target_kv.py:463-491).
* config 2: 64 requests, contexts ~ U{128..4096} (seed 1). Context K/V come from the
  draft's own chain on N(0,1) target features: fc (5 x 1024 -> 1024), context RMSNorm,
  per-layer k_proj / k_norm / RoPE and v_proj (the fused tcgen05 append), the block rows
  from q/k/v projections of N(0,1) block states at positions c..c+6. Every draft layer's
  ``B200DraftKernel`` output meets the bf16 gate against ``noncausal_varlen``
  (packed_draft.py:35-47), and the pool K/V of a seeded sample of context rows match an
  oracle evaluation of the projection chain (float64 GEMM, then the reference's bf16
  rounding steps).
"""
import numpy as np
import pytest
import torch

import bench
import inputs as I
from gpu_util import assert_bf16_close, dev, status_clean
from oracle import (OracleKVStore, bf16_bits_to_f32, f32_to_bf16_bits, noncausal_varlen, qk_norm_rope_bf16,
                    two_segment_attention)
from oracle.rope_norm import rms_norm_bf16, rope_bf16, rope_cos_sin_bf16

pytestmark = pytest.mark.gpu

THETA, EPS = 1e6, 1e-6


def bits(t):
    return t.detach().contiguous().view(torch.int16).cpu().numpy().astype(np.uint16)


def from_bits(b):
    return torch.from_numpy(np.ascontiguousarray(b).astype(np.int16)).view(torch.bfloat16).to(dev())


def hf_rotary(theta):
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
    cfg = Qwen3Config(hidden_size=1024, num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                      rope_parameters={'rope_type': 'default', 'rope_theta': theta}, rms_norm_eps=EPS)
    return Qwen3RotaryEmbedding(cfg).to(dev())


def hf_norm_rope(raw, positions, rot, weight=None):
    """transformers' Qwen3RMSNorm + apply_rotary_pos_emb of raw [n, H, 128] bf16 on the GPU."""
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RMSNorm, apply_rotary_pos_emb
    norm = Qwen3RMSNorm(128, eps=EPS).to(dev(), torch.bfloat16)
    if weight is not None:
        norm.weight.data.copy_(weight)
    with torch.no_grad():
        x = norm(raw).transpose(0, 1)[None]                      # [1, H, n, 128]
        cos, sin = rot(x, positions[None])
        _, k = apply_rotary_pos_emb(x, x, cos, sin)
    return k[0].transpose(0, 1).contiguous()


@pytest.mark.parametrize('weights,path', [('ones', 'fused'), ('random', 'fused'), ('random', 'prep')])
def test_config3_verify_layer_and_commit_full_shape(pkg, weights, path):
    R, Q = bench.VERIFY['requests'], bench.VERIFY['q']
    ctx = bench.contexts(bench.VERIFY)
    assert (R, Q, len(ctx)) == (128, 7, 128) and min(ctx) >= 256 and max(ctx) <= 8192
    caps = [c + Q for c in ctx]
    store = pkg.B200PersistentTargetKV(layers=1, slots=R, context_capacity=max(caps), max_query_tokens=R * Q,
                                       device=dev(), slot_capacities=caps)
    handles = [store.add_request(f'r{i}') for i in range(R)]
    gen = torch.Generator(device=dev())
    gen.manual_seed(2)
    bf = torch.bfloat16
    rot = hf_rotary(THETA)
    # resident prefixes: K = RoPE(k_norm(N(0,1))) at 0..c-1 (transformers' modules), V ~ N(0,1)
    total = sum(ctx)
    raw = torch.randn((total, 8, 128), generator=gen, device=dev(), dtype=bf)
    pos = torch.cat([torch.arange(c, device=dev()) for c in ctx])
    res_k = hf_norm_rope(raw, pos, rot)
    res_v = torch.randn((total, 8, 128), generator=gen, device=dev(), dtype=bf)
    del raw
    o = 0
    for h, c in zip(handles, ctx):
        store.load_prefix(h, res_k[None, o:o + c], res_v[None, o:o + c])
        o += c
    # the new rows: raw projections, norm weights, one verify layer
    n = R * Q
    qr = torch.randn((n, 16, 128), generator=gen, device=dev(), dtype=bf)
    kr = torch.randn((n, 8, 128), generator=gen, device=dev(), dtype=bf)
    vr = torch.randn((n, 8, 128), generator=gen, device=dev(), dtype=bf)
    if weights == 'ones':
        qw = kw = torch.ones(128, device=dev(), dtype=bf)
    else:
        qw = (1 + 0.1 * torch.randn(128, generator=gen, device=dev())).to(bf)
        kw = (1 + 0.1 * torch.randn(128, generator=gen, device=dev())).to(bf)
    tx = store.begin(handles, query_lengths=[Q] * R)
    inv = pkg.rope_inv_freq(THETA, device=dev())
    out = store.verify_layer(tx, 0, qr, kr, vr, qw, kw, inv_freq=inv, eps=EPS, path=path)
    torch.cuda.synchronize()
    status_clean(pkg)
    positions = np.concatenate([np.arange(c, c + Q) for c in ctx])
    q_o, k_o = qk_norm_rope_bf16(bits(qr), bits(kr), bits(qw), bits(kw), positions, THETA, EPS)
    sk, sv = bits(store.scratch_keys[:n]), bits(store.scratch_values[:n])
    assert np.array_equal(sk, k_o)                     # appended K: the reference's CPU values
    assert np.array_equal(sv, bits(vr))
    # attention: every request against the oracle (resident rows read back per request)
    got = out.float().cpu().numpy()
    qf, skf, svf = bf16_bits_to_f32(q_o), bf16_bits_to_f32(sk), bf16_bits_to_f32(sv)
    o = 0
    for i, c in enumerate(ctx):
        rk = bf16_bits_to_f32(bits(res_k[o:o + c]))
        rv = bf16_bits_to_f32(bits(res_v[o:o + c]))
        ref = two_segment_attention(qf[i * Q:(i + 1) * Q], [Q], [((rk, rv, 0, c), (skf, svf, i * Q, Q))],
                                    I.SCALE, True)
        assert_bf16_close(torch.from_numpy(got[i * Q:(i + 1) * Q]), ref)
        o += c
    # commit the accepted prefixes (accept ~ U{0..6}, anchor included); roll back the rest
    accept = np.random.Generator(np.random.PCG64(2)).integers(0, 7, R)
    counts = [int(a) + 1 for a in accept]
    before_k, before_v = store._keys.clone(), store._values.clone()
    result = store.commit(tx, {h: m for h, m in zip(handles, counts)})
    torch.cuda.synchronize()
    oracle = OracleKVStore(1, R, Q, n, 8, 128, np.uint16)     # each slot's window [c, c + 7)
    oracle.stage_layer(0, sk, sv)
    oracle.commit(list(range(R)), [0] * R, [Q] * R, counts)
    assert result['committed_tokens'] == sum(counts)
    assert [store.length(h) for h in handles] == [c + m for c, m in zip(ctx, oracle.lengths)]
    want_k, want_v = before_k, before_v
    for i, (h, c) in enumerate(zip(handles, ctx)):
        r0 = store.slot_rows[h.index] + c
        want_k[r0:r0 + Q] = from_bits(oracle.keys[0, i])
        want_v[r0:r0 + Q] = from_bits(oracle.values[0, i])
    assert torch.equal(store._keys.view(torch.int16), want_k.view(torch.int16))
    assert torch.equal(store._values.view(torch.int16), want_v.view(torch.int16))
    status_clean(pkg)


def test_config2_draft_layers_full_shape(pkg):
    """The bench's own config-2 inputs (``bench.draft_cfg2_inputs``, rank 0) through
    ``B200DraftKernel`` for every draft layer, against the oracle."""
    R, B = bench.DRAFT['requests'], bench.BLOCK
    d2 = bench.draft_cfg2_inputs(pkg, dev())
    ctx = d2['contexts']
    assert (R, B, len(ctx)) == (64, 7, 64) and min(ctx) >= 128 and max(ctx) <= 4096
    pd, draft, names = d2['pool'], d2['draft'], d2['names']
    assert pd._fused_append_ready()
    torch.cuda.synchronize()
    status_clean(pkg)
    kernel = pkg.B200DraftKernel(dev())
    qlens, klens = [B] * R, [c + B for c in ctx]
    for li in range(len(draft.layers)):
        q, k, v = d2['q'][li], d2['k'][li], d2['v'][li]
        out = kernel(q, k, v, d2['layout'], scale=I.SCALE)
        torch.cuda.synchronize()
        ref = noncausal_varlen(bf16_bits_to_f32(bits(q)), bf16_bits_to_f32(bits(k)), bf16_bits_to_f32(bits(v)),
                               qlens, klens, I.SCALE)
        assert_bf16_close(out, ref)
        # the packed keys are each request's pool rows followed by its block rows
        o = 0
        for r, c in zip(names[:4], ctx[:4]):
            r0 = pd.slot_rows[pd._slots[r]]
            assert torch.equal(k[o:o + c].view(torch.int16), pd.pool_k[li][r0:r0 + c].view(torch.int16))
            o += c + B
    feats = d2['features']
    status_clean(pkg)
    # pool K/V of a seeded sample of context rows against the oracle's projection chain:
    # context = bf16(context_norm(bf16(fc(features)))) is the library's input, then per layer
    # k = RoPE(k_norm(bf16(context @ Wk^T))), v = bf16(context @ Wv^T) with a float64 GEMM
    sample = np.sort(np.random.Generator(np.random.PCG64(11)).choice(sum(ctx), 1024, replace=False))
    with torch.no_grad():     # the same fc + norm call (same shapes) the append made
        context = pd._norm(draft.context_norm, draft.fc(feats))[0]
    cb = bf16_bits_to_f32(bits(context[torch.from_numpy(sample).to(dev())])).astype(np.float64)
    cu = np.concatenate([[0], np.cumsum(ctx)])
    req = np.searchsorted(cu, sample, side='right') - 1
    spos = sample - cu[req]
    rows = np.array([pd.slot_rows[pd._slots[names[i]]] for i in req]) + spos
    # the draft's rotary buffer, in the dtype the module holds it (a bf16 draft rounds it)
    freqs = draft.rotary.inv_freq.float().cpu().numpy()
    cos_o, sin_o = rope_cos_sin_bf16(spos, freqs)
    for li, layer in enumerate(draft.layers):
        att = layer.attention
        wk = bf16_bits_to_f32(bits(att.k_proj.weight)).astype(np.float64)
        wv = bf16_bits_to_f32(bits(att.v_proj.weight)).astype(np.float64)
        kproj = f32_to_bf16_bits((cb @ wk.T).astype(np.float32)).reshape(-1, 8, 128)
        vproj = f32_to_bf16_bits((cb @ wv.T).astype(np.float32)).reshape(-1, 8, 128)
        k_want = rope_bf16(rms_norm_bf16(kproj, bits(att.k_norm.weight), EPS), cos_o, sin_o)
        ridx = torch.from_numpy(rows).to(dev())
        k_got, v_got = bits(pd.pool_k[li][ridx]), bits(pd.pool_v[li][ridx])
        # the tcgen05 GEMM accumulates in fp32 in its own order: a projection output can sit
        # one bf16 ulp from the float64 GEMM's rounding, which the norm and RoPE carry on
        assert_bf16_close(from_bits(k_got), bf16_bits_to_f32(k_want))
        assert_bf16_close(from_bits(v_got), bf16_bits_to_f32(vproj))
        assert np.mean(k_got == k_want) > 0.97 and np.mean(v_got == vproj) > 0.97
    status_clean(pkg)
