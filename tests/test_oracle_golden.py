"""Pin the CPU oracle: reference-generated fixtures and the reference tests' known answers."""
import numpy as np
import pytest

import inputs as I
from oracle import (OracleKVStore, begin_metadata, block_mask, bottom_right_varlen, f32_to_bf16_bits,
                    inv_freq, noncausal_varlen, packed_layout_from_metadata, qk_norm_rope_bf16,
                    rope_cos_sin_bf16, rms_norm_bf16, round_bf16, training_layout_attention)
from oracle.rope_norm import torch_order_sum128
from oracle.bf16 import bf16_bits_to_f32


def test_bf16_rounding_matches_torch():
    import torch
    g = I.rng(1)
    x = np.concatenate([g.standard_normal(4096, dtype=np.float32) * 10 ** g.uniform(-6, 6, 4096).astype(np.float32),
                        np.array([np.inf, -np.inf, 0.0, -0.0, 1.0 + 2 ** -8, 1.0 + 3 * 2 ** -8], np.float32)])
    expect = torch.from_numpy(x).to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint16)
    assert np.array_equal(f32_to_bf16_bits(x), expect)
    assert np.array_equal(bf16_bits_to_f32(expect), torch.from_numpy(expect.astype(np.int16)).view(torch.bfloat16).float().numpy())


@pytest.mark.parametrize('name,seed,contexts,bf16,tol', [
    ('draft_cfg1', 0, I.CFG1_CONTEXTS, False, 1e-5),
    ('draft_bf16_small', 11, I.DRAFT_BF16_CONTEXTS, True, 1e-5)])
def test_noncausal_draft_matches_reference(golden, name, seed, contexts, bf16, tol):
    g = golden(name)
    q, k, v, qlens, klens = I.draft_case(seed, contexts, bf16)
    assert I.digest(q, k, v) == str(g['digest'])
    out = noncausal_varlen(q, k, v, qlens, klens, I.SCALE)
    np.testing.assert_allclose(out, g['output'], atol=tol, rtol=tol)


def test_verify_probe_cases_match_reference(golden):
    for idx, (qlens, klens) in enumerate(I.PROBE_CASES):
        g = golden(f'verify_probe{idx}')
        q, k, v = I.varlen_case(I.PROBE_SEED + idx, qlens, klens, True)
        assert I.digest(q, k, v) == str(g['digest'])
        np.testing.assert_allclose(bottom_right_varlen(q, k, v, qlens, klens, I.SCALE), g['output'], atol=1e-5, rtol=1e-5)


def test_zero_q_ramp_is_bottom_right(golden):
    """reports/native-varlen-diagnostic-20261009: request 1 -> 0.25, request 2 -> (21..28)/64."""
    qlens, klens = I.PROBE_CASES[0]
    q = np.zeros((9, I.HQ, I.D), np.float32)
    ramp = np.concatenate([np.arange(n, dtype=np.float32) / 32 for n in klens])
    v = np.broadcast_to(ramp[:, None, None], (sum(klens), I.HKV, I.D)).copy()
    out = bottom_right_varlen(q, np.zeros_like(v), v, qlens, klens, I.SCALE)
    np.testing.assert_allclose(out, golden('zero_q_ramp')['output'], atol=1e-6)
    np.testing.assert_allclose(out[0], 0.25)
    np.testing.assert_allclose(out[1:, 0, 0], np.arange(21, 29) / 64)


def test_capacity_tail_nan_is_never_read(golden):
    qlens, klens, tail = I.CAPACITY_QLENS, I.CAPACITY_KLENS, I.CAPACITY_TAIL
    q, k, v = I.varlen_case(77, qlens, klens, True, tail=tail)
    k[sum(klens):] = np.nan
    v[sum(klens):] = np.nan
    out = bottom_right_varlen(q, k, v, qlens, klens, I.SCALE)
    assert np.isfinite(out).all()
    np.testing.assert_allclose(out, golden('verify_capacity')['output'], atol=1e-5, rtol=1e-5)


def test_known_answer_uniform_attention():
    """tests/test_varlen_target.py:65-80 (bottom-right [4,5,7/3]) and test_packed_draft.py:109-112 (all 2.0)."""
    lay = packed_layout_from_metadata([2, 2, 1], [2, 3, 2], [1, 1, 2, 2, 3, 3, 1, 2, 2], [0, 1, 0, 1, 0, 1, 2, 2, 3])
    assert lay.gather_indices == (2, 3, 7, 8, 0, 1, 6)
    physical = np.arange(9, dtype=np.float32)
    k = physical[list(lay.gather_indices)].reshape(7, 1, 1)
    out = bottom_right_varlen(np.zeros((3, 1, 1)), k, k, lay.query_lengths, lay.key_lengths, 1.0)
    np.testing.assert_allclose(out.reshape(-1), [4, 5, 7 / 3], atol=1e-12)
    lay = packed_layout_from_metadata([0, 0, 0], [2, 3, 4], [0] * 5, list(range(5)))
    v = np.broadcast_to(np.arange(5.0).reshape(5, 1, 1), (5, 2, 8))
    out = noncausal_varlen(np.zeros((3, 4, 8)), np.zeros((5, 2, 8)), v, lay.query_lengths, lay.key_lengths, 8 ** -.5)
    assert np.array_equal(out, np.full((3, 4, 8), 2.0))


def test_block_mask_truth_table(golden):
    """tests/test_core.py:39-45 plus the reference-generated mask."""
    m = block_mask([2, 4], 3, 7)
    assert np.array_equal(m, golden('block_mask_truth')['mask'])
    assert list(np.nonzero(m[0])[0]) == [0, 1, 7, 8, 9]
    assert list(np.nonzero(m[4])[0]) == [0, 1, 2, 3, 10, 11, 12]


def test_training_layout_matches_reference(golden):
    g = I.rng(3)
    anchors = [a for _, a in I.TRAIN_SEQS]
    ctxs = [c for c, _ in I.TRAIN_SEQS]
    nq = sum(len(a) * I.BLOCK for a in anchors)
    nk = sum(c + len(a) * I.BLOCK for c, a in I.TRAIN_SEQS)
    q, k, v = (I.normal(g, s, True) for s in ((nq, I.HQ, I.D), (nk, I.HKV, I.D), (nk, I.HKV, I.D)))
    ref = golden('train_layout')
    assert I.digest(q, k, v) == str(ref['digest'])
    out = training_layout_attention(q, k, v, ctxs, anchors, I.BLOCK, I.SCALE)
    np.testing.assert_allclose(out, ref['output'], atol=2e-5, rtol=1e-5)


@pytest.mark.parametrize('idx', [0, 1])
def test_layout_matches_reference(golden, idx):
    g = golden(f'layout{idx}')
    lay = packed_layout_from_metadata(g['qr'], g['qp'], g['kr'], g['kp'])
    assert lay.request_markers == tuple(g['markers'])
    assert lay.query_lengths == tuple(g['query_lengths'])
    assert lay.key_lengths == tuple(g['key_lengths'])
    assert lay.cu_query == tuple(g['cu_query'])
    assert lay.cu_key == tuple(g['cu_key'])
    assert lay.gather_indices == tuple(g['gather'])
    assert lay.pair_domain == int(g['pair_domain'])


def test_layout_refusals_match_reference():
    """tests/test_varlen_target.py:121-125."""
    for qreq, qpos, kreq, kpos in [([1, 2, 1], [0, 0, 1], [1, 1, 2], [0, 1, 0]), ([1], [0], [1, 1], [0, 1]),
                                   ([1], [1], [1, 1], [0, 2]), ([], [], [], [])]:
        with pytest.raises(ValueError):
            packed_layout_from_metadata(qreq, qpos, kreq, kpos)


def test_qk_norm_rope_matches_transformers(golden):
    """The oracle's q/k norm + RoPE equals transformers' CPU modules bit for bit: cos/sin
    tables, both RMSNorms and the roped outputs (positions up to 8197, theta 1e6)."""
    g = golden('qk_norm_rope')
    f = inv_freq(I.ROPE_THETA, I.D)
    np.testing.assert_array_equal(f, g['inv_freq'])
    cos, sin = rope_cos_sin_bf16(g['positions'], f)
    np.testing.assert_array_equal(f32_to_bf16_bits(cos), g['cos'])
    np.testing.assert_array_equal(f32_to_bf16_bits(sin), g['sin'])
    np.testing.assert_array_equal(rms_norm_bf16(g['q_raw'], g['q_weight'], I.RMS_EPS), g['q_norm'])
    np.testing.assert_array_equal(rms_norm_bf16(g['k_raw'], g['k_weight'], I.RMS_EPS), g['k_norm'])
    q, k = qk_norm_rope_bf16(g['q_raw'], g['k_raw'], g['q_weight'], g['k_weight'], g['positions'],
                             I.ROPE_THETA, I.RMS_EPS)
    np.testing.assert_array_equal(q, g['q_out'])
    np.testing.assert_array_equal(k, g['k_out'])


def test_torch_order_sum_matches_torch_cpu_sum():
    """The association order the oracle (and the verify kernels) use for the 128-wide sum
    of squares is the one this host's torch CPU reduction uses: equal on every row,
    including rows whose float64-exact sum differs from it."""
    import torch
    g = np.random.default_rng(5)
    x = f32_to_bf16_bits((g.standard_normal((20000, 128)) * np.exp(g.uniform(-4, 4, (20000, 1)))).astype(np.float32))
    sq = bf16_bits_to_f32(x) ** 2
    mine = torch_order_sum128(sq)[:, 0]
    ref = torch.from_numpy(bf16_bits_to_f32(x)).pow(2).sum(-1).numpy()
    np.testing.assert_array_equal(mine, ref)
    exact = sq.astype(np.float64).sum(-1).astype(np.float32)
    assert np.mean(exact != ref) > 0.1          # the order matters on these rows


def test_rotary_cache_matches_transformers_rotary_module(pkg):
    """``rope_cache`` (the table the verify kernels gather) holds exactly the bf16 cos/sin
    that transformers' Qwen3RotaryEmbedding computes on the CPU, at every position below
    16384, for theta 1e6 and 1e4."""
    import torch
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import Qwen3RotaryEmbedding
    for theta in (1e6, 1e4):
        cfg = Qwen3Config(hidden_size=2048, num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                          rope_parameters={'rope_type': 'default', 'rope_theta': theta})
        rot = Qwen3RotaryEmbedding(cfg)
        n = 16384
        x = torch.zeros((1, n, 8), dtype=torch.bfloat16)
        with torch.no_grad():
            cos, sin = rot(x, torch.arange(n)[None])
        cache = pkg.kernels.rope_cache(rot.inv_freq, n, 'cpu').numpy().view(np.uint32)
        ref_cos = cos[0, :, :64].contiguous().view(torch.int16).numpy().astype(np.uint16)
        ref_sin = sin[0, :, :64].contiguous().view(torch.int16).numpy().astype(np.uint16)
        np.testing.assert_array_equal((cache & 0xFFFF).astype(np.uint16), ref_cos)
        np.testing.assert_array_equal((cache >> 16).astype(np.uint16), ref_sin)


def test_kv_store_matches_reference(golden):
    g = golden('kv_store')
    store = OracleKVStore(layers=2, slots=3, context_capacity=24, max_query_tokens=8, heads=2, dim=4)
    for s, n, off in ((0, 3, 100), (1, 5, 500), (2, 9, 900)):
        x = np.arange(2 * n * 2 * 4, dtype=np.float32).reshape(2, n, 2, 4) + off
        store.load_prefix(s, x, x + 0.25)
    meta = begin_metadata([0, 1], [3, 5], [2, 3], int(g['key_capacity']), 24)
    for key in ('committed_indices', 'scratch_indices', 'from_scratch', 'valid', 'cu_query', 'cu_key', 'positions'):
        assert np.array_equal(meta[key], g[key]), key
    sk = np.arange(2 * 5 * 2 * 4, dtype=np.float32).reshape(2, 5, 2, 4) + 10000
    for layer in range(2):
        store.stage_layer(layer, sk[layer], sk[layer] + 0.5)
    k0, v0 = store.prepare_attention(meta, 0)
    assert np.array_equal(k0, g['prepared_k0']) and np.array_equal(v0, g['prepared_v0'])
    store.commit([0, 1], [3, 5], [2, 3], [1, 2])
    assert np.array_equal(store.keys, g['resident_keys']) and np.array_equal(store.values, g['resident_values'])
    assert store.lengths == list(g['lengths'])
    meta2 = begin_metadata([0, 1], store.lengths[:2], [2, 3], int(g['key_capacity']), 24)
    assert np.array_equal(meta2['cu_key'], g['cu_key2']) and np.array_equal(meta2['positions'], g['positions2'])
    with pytest.raises(ValueError):
        store.commit([0], [4], [2], [3])
