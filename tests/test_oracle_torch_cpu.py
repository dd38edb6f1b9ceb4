"""Pin the torch CPU restatement of the reference's round (the timed CPU baseline) to the
fixtures that the reference's own functions produced (tests/golden/make_golden.py)."""
import numpy as np
import torch

import inputs as I
from oracle.torch_cpu import (VerifyRoundCPU, apply_rope, block_mask, noncausal_varlen_sdpa, persistent_sdpa,
                              qwen3_rms_norm, rotary_cos_sin, training_layout_sdpa)


def t(x):
    return torch.from_numpy(np.ascontiguousarray(x))


def bf(bits):
    return torch.from_numpy(np.ascontiguousarray(bits).astype(np.int16)).view(torch.bfloat16)


def bits(x):
    return x.contiguous().view(torch.int16).numpy().astype(np.uint16)


def test_draft_sdpa_equals_reference_fixture(golden):
    for name, seed, contexts, is_bf16 in (('draft_cfg1', 0, I.CFG1_CONTEXTS, False),
                                          ('draft_bf16_small', 11, I.DRAFT_BF16_CONTEXTS, True)):
        g = golden(name)
        q, k, v, qlens, klens = I.draft_case(seed, contexts, is_bf16)
        out = noncausal_varlen_sdpa(t(q), t(k), t(v), qlens, klens, I.SCALE).numpy()
        np.testing.assert_allclose(out, g['output'], atol=1e-6, rtol=1e-6)


def test_persistent_sdpa_equals_reference_fixtures(golden):
    qlens, klens, tail = I.CAPACITY_QLENS, I.CAPACITY_KLENS, I.CAPACITY_TAIL
    q, k, v = I.varlen_case(77, qlens, klens, True, tail=tail)
    k[sum(klens):] = np.nan
    v[sum(klens):] = np.nan
    out = persistent_sdpa(t(q), t(k), t(v), qlens, klens, I.SCALE).numpy()
    np.testing.assert_allclose(out, golden('verify_capacity')['output'], atol=1e-6, rtol=1e-6)
    for idx, (ql, kl) in enumerate(I.PROBE_CASES):
        q, k, v = I.varlen_case(I.PROBE_SEED + idx, ql, kl, True)
        out = persistent_sdpa(t(q), t(k), t(v), ql, kl, I.SCALE).numpy()
        np.testing.assert_allclose(out, golden(f'verify_probe{idx}')['output'], atol=1e-6, rtol=1e-6)


def test_norm_and_rope_equal_transformers_bit_for_bit(golden):
    g = golden('qk_norm_rope')
    assert np.array_equal(bits(qwen3_rms_norm(bf(g['q_raw']), bf(g['q_weight']), I.RMS_EPS)), g['q_norm'])
    assert np.array_equal(bits(qwen3_rms_norm(bf(g['k_raw']), bf(g['k_weight']), I.RMS_EPS)), g['k_norm'])
    cos, sin = rotary_cos_sin(t(g['positions']), t(g['inv_freq']), torch.bfloat16)
    assert np.array_equal(bits(cos), g['cos']) and np.array_equal(bits(sin), g['sin'])
    assert np.array_equal(bits(apply_rope(bf(g['q_norm']), cos, sin)), g['q_out'])
    assert np.array_equal(bits(apply_rope(bf(g['k_norm']), cos, sin)), g['k_out'])


def test_verify_round_gathers_and_commits_like_the_reference_store(golden):
    """The reference store's growing-context scenario (kv_store fixture): same prepared
    layer-0 K/V rows over the logical keys, same resident bytes and lengths after commit."""
    g = golden('kv_store')
    store = VerifyRoundCPU(2, [3, 5, 9], 8, 2, 4, slot_capacities=[24, 24, 24])
    for i, (n, off) in enumerate(((3, 100), (5, 500), (9, 900))):
        x = torch.arange(2 * n * 2 * 4, dtype=torch.float32).reshape(2, n, 2, 4) + off
        store.keys[:, store.offsets[i]:store.offsets[i] + n] = x
        store.values[:, store.offsets[i]:store.offsets[i] + n] = x + 0.25
    store.lengths = [3, 5]                       # the bucket's two active requests
    ws = store.begin((2, 3))
    n = ws['rows']
    assert ws['cu_key'].tolist() == g['cu_key'][:3].tolist() and ws['positions'].tolist() == g['positions'].tolist()
    sk = torch.arange(2 * 5 * 2 * 4, dtype=torch.float32).reshape(2, 5, 2, 4) + 10000
    for layer in range(2):
        store.scratch_keys[layer, :5] = sk[layer]
        store.scratch_values[layer, :5] = sk[layer] + 0.5
    for resident, scratch, out in ((store.keys, store.scratch_keys, 'keys'),
                                   (store.values, store.scratch_values, 'values')):
        old = torch.index_select(resident[0], 0, ws['committed'])
        new = torch.index_select(scratch[0], 0, ws['scratch'])
        ws[out][:n] = torch.where(ws['from_scratch'], new, old)
    np.testing.assert_array_equal(ws['keys'][:n].numpy(), g['prepared_k0'][:n])
    np.testing.assert_array_equal(ws['values'][:n].numpy(), g['prepared_v0'][:n])
    store.commit(ws, [1, 2])
    assert store.lengths == g['lengths'][:2].tolist()
    for i in range(2):
        m = store.lengths[i]
        got = store.keys[:, store.offsets[i]:store.offsets[i] + m].numpy()
        np.testing.assert_array_equal(got, g['resident_keys'][:, i, :m])
        got = store.values[:, store.offsets[i]:store.offsets[i] + m].numpy()
        np.testing.assert_array_equal(got, g['resident_values'][:, i, :m])


def test_verify_layer_matches_the_numpy_oracle():
    """A whole layer (norm, RoPE, stage, gather, attention) against the float64 oracle."""
    from oracle import bottom_right_varlen
    from oracle.rope_norm import inv_freq
    gen = torch.Generator().manual_seed(5)
    ctx = [37, 5, 90]
    store = VerifyRoundCPU(1, ctx, 21, 8, 128, generator=gen)
    ws = store.begin((7, 7, 7))
    q = torch.randn((21, 16, 128), generator=gen)
    k = torch.randn((21, 8, 128), generator=gen)
    v = torch.randn((21, 8, 128), generator=gen)
    ones = torch.ones(128)
    freqs = torch.from_numpy(inv_freq(1e6, 128))
    out = store.layer(ws, 0, q, k, v, ones, ones, freqs, 1e-6, I.SCALE).numpy()
    # float32 throughout: the attention of the restatement's own normed, roped q against
    # the gathered K/V, evaluated by the float64 oracle
    cos, sin = rotary_cos_sin(ws['positions'], freqs, torch.float32)
    qr = apply_rope(qwen3_rms_norm(q, ones, 1e-6), cos, sin).numpy()
    keys, values = ws['keys'][:ws['rows']].numpy(), ws['values'][:ws['rows']].numpy()
    ref = bottom_right_varlen(qr, keys, values, [7] * 3, [c + 7 for c in ctx], I.SCALE)
    np.testing.assert_allclose(out, ref, atol=2e-5, rtol=1e-4)
    # the gathered keys are the resident prefixes followed by the staged (normed, roped) rows
    o = 0
    for i, c in enumerate(ctx):
        np.testing.assert_array_equal(keys[o:o + c], store.keys[0, store.offsets[i]:store.offsets[i] + c].numpy())
        o += c + 7


def test_training_layout_equals_reference_fixtures(golden):
    """block_mask's truth table and the packed training-layout attention, both made by the
    reference's own functions."""
    m = block_mask(torch.tensor([2, 4]), 3, 7)[0, 0].numpy()
    np.testing.assert_array_equal(m, golden('block_mask_truth')['mask'])
    g = I.rng(3)
    ctxs = [c for c, _ in I.TRAIN_SEQS]
    anchors = [a for _, a in I.TRAIN_SEQS]
    nq = sum(len(a) * I.BLOCK for a in anchors)
    nk = sum(c + len(a) * I.BLOCK for c, a in I.TRAIN_SEQS)
    q = I.normal(g, (nq, I.HQ, I.D), True)
    k = I.normal(g, (nk, I.HKV, I.D), True)
    v = I.normal(g, (nk, I.HKV, I.D), True)
    out = training_layout_sdpa(t(q), t(k), t(v), ctxs, anchors, I.BLOCK).numpy()
    np.testing.assert_allclose(out, golden('train_layout')['output'], atol=1e-6, rtol=1e-6)
