"""GPU parity of the draft (non-causal) and verify (bottom-right causal) kernels vs the oracle.

Every call goes through the drop-in kernel classes, i.e. through the C ABI of
lib/libdspark_b200.so. Tolerances: bf16 max-abs 2e-2 / rel 1e-2 and RMS <= 5e-3;
float32 1e-5.
"""
import numpy as np
import pytest
import torch

import inputs as I
from gpu_util import F32_TOL, assert_bf16_close, dev, i32, status_clean, to_dev
from oracle import bottom_right_varlen, noncausal_varlen, training_layout_attention, two_segment_attention

pytestmark = pytest.mark.gpu


@pytest.fixture(scope='module')
def kernels(pkg):
    torch.cuda.set_device(0)
    pkg.read_device_status(clear=True)
    return dict(draft=pkg.B200DraftKernel(dev()), causal=pkg.B200VarlenKernel(dev()),
                capacity=pkg.B200CapacityKernel(dev()))


def run(kernel, pkg, q, k, v, qlens, klens, dtype=torch.bfloat16):
    layout = pkg.PackedLayout.from_lengths(qlens, klens, dev())
    out = kernel(to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype), layout, scale=I.SCALE)
    torch.cuda.synchronize()
    return out


def test_draft_bf16_matches_reference_fixture(pkg, kernels, golden):
    q, k, v, qlens, klens = I.draft_case(11, I.DRAFT_BF16_CONTEXTS, True)
    out = run(kernels['draft'], pkg, q, k, v, qlens, klens)
    assert_bf16_close(out, golden('draft_bf16_small')['output'])
    assert_bf16_close(out, noncausal_varlen(q, k, v, qlens, klens, I.SCALE))
    status_clean(pkg)


def test_draft_fp32_config1_exact(pkg, kernels, golden):
    q, k, v, qlens, klens = I.draft_case(0, I.CFG1_CONTEXTS, False)
    out = run(kernels['draft'], pkg, q, k, v, qlens, klens, torch.float32).cpu().numpy()
    np.testing.assert_allclose(out, golden('draft_cfg1')['output'], atol=F32_TOL, rtol=F32_TOL)
    np.testing.assert_allclose(out, noncausal_varlen(q, k, v, qlens, klens, I.SCALE), atol=F32_TOL, rtol=F32_TOL)
    status_clean(pkg)


@pytest.mark.parametrize('idx', range(len(I.PROBE_CASES)))
def test_verify_probe_cases(pkg, kernels, golden, idx):
    qlens, klens = I.PROBE_CASES[idx]
    q, k, v = I.varlen_case(I.PROBE_SEED + idx, qlens, klens, True)
    out = run(kernels['causal'], pkg, q, k, v, qlens, klens)
    assert_bf16_close(out, golden(f'verify_probe{idx}')['output'])
    status_clean(pkg)


def test_zero_q_ramp_bottom_right_is_exact(pkg, kernels):
    """Zero Q, V = local key position / 32: request 1 -> 0.25, request 2 -> (21..28)/64 exactly."""
    qlens, klens = I.PROBE_CASES[0]
    q = np.zeros((9, I.HQ, I.D), np.float32)
    ramp = np.concatenate([np.arange(n, dtype=np.float32) / 32 for n in klens])
    v = np.broadcast_to(ramp[:, None, None], (sum(klens), I.HKV, I.D)).copy()
    out = run(kernels['causal'], pkg, q, np.zeros_like(v), v, qlens, klens).float().cpu().numpy()
    assert np.all(out[0] == 0.25)
    for r in range(8):
        assert np.all(out[1 + r] == np.float32((21 + r) / 64)), r


def test_capacity_tail_nan_never_read(pkg, kernels, golden):
    qlens, klens, tail = I.CAPACITY_QLENS, I.CAPACITY_KLENS, I.CAPACITY_TAIL
    q, k, v = I.varlen_case(77, qlens, klens, True, tail=tail)
    k[sum(klens):] = np.nan
    v[sum(klens):] = np.nan
    layout = pkg.PersistentAttentionLayout(qlens, klens, i32(np.cumsum((0,) + qlens)), i32(np.cumsum((0,) + klens)),
                                           sum(klens) + tail, max(klens), max(qlens))
    out = kernels['capacity'](to_dev(q), to_dev(k), to_dev(v), layout, scale=I.SCALE)
    assert_bf16_close(out, golden('verify_capacity')['output'])
    status_clean(pkg)


@pytest.mark.parametrize('causal', [False, True])
def test_random_ragged_batch(pkg, kernels, causal):
    """Config-2/3-like ragged contexts, q in {1,7,8} and >8 rows (several q-blocks)."""
    g = I.rng(101 + causal)
    ctx = g.integers(0, 3000, 24)
    qlens = tuple(int(x) for x in g.choice([1, 7, 7, 8, 13, 20], 24))
    klens = tuple(int(c) + q for c, q in zip(ctx, qlens))
    q = I.normal(g, (sum(qlens), I.HQ, I.D), True)
    k = I.normal(g, (sum(klens), I.HKV, I.D), True)
    v = I.normal(g, (sum(klens), I.HKV, I.D), True)
    kern = kernels['causal'] if causal else kernels['draft']
    out = run(kern, pkg, q, k, v, qlens, klens)
    ref = (bottom_right_varlen if causal else noncausal_varlen)(q, k, v, qlens, klens, I.SCALE)
    assert_bf16_close(out, ref)
    status_clean(pkg)


def test_long_single_request_split_across_all_ctas(pkg, kernels):
    """One request with 40k keys (2500 tiles): every CTA holds a slice, the merge kernel combines them."""
    g = I.rng(5)
    qlens, klens = (7,), (40000,)
    q = I.normal(g, (7, I.HQ, I.D), True)
    k = I.normal(g, (40000, I.HKV, I.D), True)
    v = I.normal(g, (40000, I.HKV, I.D), True)
    for causal in (False, True):
        kern = kernels['causal'] if causal else kernels['draft']
        out = run(kern, pkg, q, k, v, qlens, klens)
        ref = (bottom_right_varlen if causal else noncausal_varlen)(q, k, v, qlens, klens, I.SCALE)
        assert_bf16_close(out, ref)
    status_clean(pkg)


def test_poisoned_neighbours_do_not_change_output(pkg, kernels):
    """Overwriting other requests' K/V with +-1000 leaves request 0 bit-identical."""
    q, k, v, qlens, klens = I.draft_case(23, (300, 41, 900), True)
    for name in ('draft', 'causal'):
        before = run(kernels[name], pkg, q, k, v, qlens, klens)
        k2, v2 = k.copy(), v.copy()
        k2[klens[0]:] = 1000.0
        v2[klens[0]:] = -1000.0
        after = run(kernels[name], pkg, q, k2, v2, qlens, klens)
        assert torch.equal(before[:qlens[0]], after[:qlens[0]])


def test_segment_two_sources_matches_gather(pkg):
    """Context cache rows + block rows read in place == concat/gather then attention."""
    g = I.rng(31)
    contexts = [0, 5, 260, 1000, 77]
    cache_k = I.normal(g, (3000, I.HKV, I.D), True)
    cache_v = I.normal(g, (3000, I.HKV, I.D), True)
    starts = [0, 10, 400, 1200, 2900]
    blk_k = I.normal(g, (7 * len(contexts), I.HKV, I.D), True)
    blk_v = I.normal(g, (7 * len(contexts), I.HKV, I.D), True)
    q = I.normal(g, (7 * len(contexts), I.HQ, I.D), True)
    qlens = [7] * len(contexts)
    for causal in (False, True):
        out = pkg.segment_attention(to_dev(q), i32(np.cumsum([0] + qlens)), qlens, to_dev(cache_k), to_dev(cache_v),
                                    i32(starts), i32(contexts), to_dev(blk_k), to_dev(blk_v),
                                    i32([7 * i for i in range(5)]), i32(qlens), causal=causal)
        segs = [((cache_k, cache_v, s, c), (blk_k, blk_v, 7 * i, 7)) for i, (s, c) in enumerate(zip(starts, contexts))]
        assert_bf16_close(out, two_segment_attention(q, qlens, segs, I.SCALE, causal))
    status_clean(pkg)


def test_training_layout_blocks_as_segments(pkg, golden):
    """Training-layout mask (context < anchor + own block) through the two-source kernel."""
    g = I.rng(3)
    anchors = [a for _, a in I.TRAIN_SEQS]
    ctxs = [c for c, _ in I.TRAIN_SEQS]
    nq = sum(len(a) * I.BLOCK for a in anchors)
    nk = sum(c + len(a) * I.BLOCK for c, a in I.TRAIN_SEQS)
    q, k, v = (I.normal(g, s, True) for s in ((nq, I.HQ, I.D), (nk, I.HKV, I.D), (nk, I.HKV, I.D)))
    a_start, a_len, b_start, ko = [], [], [], 0
    for ctx, anc in I.TRAIN_SEQS:
        for b, a in enumerate(anc):
            a_start.append(ko)
            a_len.append(a)
            b_start.append(ko + ctx + 7 * b)
        ko += ctx + 7 * len(anc)
    nblk = len(a_start)
    kd, vd = to_dev(k), to_dev(v)
    out = pkg.segment_attention(to_dev(q), i32(np.arange(nblk + 1) * 7), [7] * nblk, kd, vd, i32(a_start), i32(a_len),
                                kd, vd, i32(b_start), i32([7] * nblk), causal=False)
    assert_bf16_close(out, golden('train_layout')['output'])
    assert_bf16_close(out, training_layout_attention(q, k, v, ctxs, anchors, I.BLOCK, I.SCALE))
    status_clean(pkg)


def test_host_refusals_before_launch(pkg, kernels):
    q, k, v, qlens, klens = I.draft_case(1, (10, 20), True)
    layout = pkg.PackedLayout.from_lengths(qlens, klens, dev())
    qd, kd, vd = to_dev(q), to_dev(k), to_dev(v)
    kern = kernels['causal']
    with pytest.raises(ValueError):
        kern(qd.half(), kd.half(), vd.half(), layout, scale=I.SCALE)
    with pytest.raises(ValueError):
        kern(qd, kd, vd, layout, scale=1.0)
    with pytest.raises(ValueError):
        kern(qd[:, :8].contiguous(), kd, vd, layout, scale=I.SCALE)
    with pytest.raises(ValueError):
        kern(qd[:-1], kd, vd, layout, scale=I.SCALE)
    bad = pkg.PackedLayout(layout.request_markers, qlens, klens, layout.cu_query.clone(), layout.cu_key.clone(),
                           layout.gather_indices, layout.physical_key_tokens)
    bad.cu_key[1] = 3
    with pytest.raises(ValueError):
        kern(qd, kd, vd, bad, scale=I.SCALE)
