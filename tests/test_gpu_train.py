"""GPU parity of the training-layout tensor-core kernel (tcgen05) vs the oracle.

Calls go through ``B200TrainingLayoutKernel`` -> ``dspark_train_attn`` (C ABI).
The layouts are the CPU plan-walk cases of test_train_plan.py (anchors at 0, at
and past the context, unsorted, block sizes 6..32, a sequence with no anchors),
the reference fixture, and the benchmark's config 4 (8 x 2048 context, 32
sorted anchors, block 7). bf16 tolerance: max-abs 2e-2 / rel 1e-2, RMS <= 5e-3;
float32 (two-segment CUDA-core path) 1e-5.
"""
import numpy as np
import pytest
import torch

import inputs as I
from gpu_util import F32_TOL, assert_bf16_close, dev, status_clean, to_dev
from oracle import training_layout_attention
from test_train_plan import CASES

pytestmark = pytest.mark.gpu


def run(pkg, ctx, anchors, bs, seed, dtype=torch.bfloat16):
    g = I.rng(seed)
    nq = sum(len(a) * bs for a in anchors)
    nk = sum(c + len(a) * bs for c, a in zip(ctx, anchors))
    q, k, v = (I.normal(g, s, True) for s in ((nq, I.HQ, I.D), (nk, I.HKV, I.D), (nk, I.HKV, I.D)))
    layout = pkg.TrainingLayout.from_anchors(ctx, anchors, bs, device=dev())
    kernel = pkg.B200TrainingLayoutKernel(dev())
    out = kernel(to_dev(q, dtype), to_dev(k, dtype), to_dev(v, dtype), layout, scale=I.SCALE)
    torch.cuda.synchronize()
    return out, training_layout_attention(q, k, v, ctx, anchors, bs, I.SCALE)


def test_reference_fixture(pkg, golden):
    ctx = [c for c, _ in I.TRAIN_SEQS]
    anchors = [list(a) for _, a in I.TRAIN_SEQS]
    g = I.rng(3)
    nq = sum(len(a) * I.BLOCK for a in anchors)
    nk = sum(c + len(a) * I.BLOCK for c, a in I.TRAIN_SEQS)
    q, k, v = (I.normal(g, s, True) for s in ((nq, I.HQ, I.D), (nk, I.HKV, I.D), (nk, I.HKV, I.D)))
    layout = pkg.TrainingLayout.from_anchors(ctx, anchors, I.BLOCK, device=dev())
    out = pkg.B200TrainingLayoutKernel(dev())(to_dev(q), to_dev(k), to_dev(v), layout, scale=I.SCALE)
    torch.cuda.synchronize()
    assert_bf16_close(out, golden('train_layout')['output'])
    status_clean(pkg)


@pytest.mark.parametrize('name,ctx,anchors,bs', CASES, ids=[c[0] for c in CASES])
def test_layouts_match_oracle(pkg, name, ctx, anchors, bs):
    out, ref = run(pkg, ctx, anchors, bs, seed=21)
    assert_bf16_close(out, ref)
    status_clean(pkg)


def test_config4_matches_oracle(pkg):
    g = I.rng(3)
    anchors = [sorted(g.choice(2047, 32, replace=False).tolist()) for _ in range(8)]
    out, ref = run(pkg, [2048] * 8, anchors, 7, seed=4)
    assert_bf16_close(out, ref)
    status_clean(pkg)


def test_float32_layout_is_exact(pkg):
    name, ctx, anchors, bs = CASES[1]
    out, ref = run(pkg, ctx, anchors, bs, seed=5, dtype=torch.float32)
    np.testing.assert_allclose(out.cpu().numpy(), ref, atol=F32_TOL, rtol=F32_TOL)
    status_clean(pkg)


def test_repeat_calls_identical(pkg):
    """Same inputs twice -> bit-identical outputs (no state leaks between launches)."""
    g = I.rng(8)
    ctx, anchors = [300, 700], [[0, 299, 150, 7], [650, 1, 699, 300, 20, 500]]
    nq = sum(len(a) * 7 for a in anchors)
    nk = sum(c + len(a) * 7 for c, a in zip(ctx, anchors))
    q, k, v = (to_dev(I.normal(g, s, True)) for s in ((nq, I.HQ, I.D), (nk, I.HKV, I.D), (nk, I.HKV, I.D)))
    layout = pkg.TrainingLayout.from_anchors(ctx, anchors, 7, device=dev())
    kernel = pkg.B200TrainingLayoutKernel(dev())
    a = kernel(q, k, v, layout, scale=I.SCALE)
    b = kernel(q, k, v, layout, scale=I.SCALE)
    torch.cuda.synchronize()
    assert torch.equal(a, b)
    status_clean(pkg)


def test_refusals_before_launch(pkg):
    layout = pkg.TrainingLayout.from_anchors([10], [[3]], 7, device=dev())
    kernel = pkg.B200TrainingLayoutKernel(dev())
    q = torch.zeros(7, 16, 128, dtype=torch.bfloat16, device=dev())
    kv = torch.zeros(17, 8, 128, dtype=torch.bfloat16, device=dev())
    with pytest.raises(ValueError):
        kernel(q, kv[:16], kv[:16], layout, scale=I.SCALE)          # key rows differ from the layout
    with pytest.raises(ValueError):
        kernel(q, kv, kv, layout, scale=0.1)
    with pytest.raises(ValueError):
        kernel(q.float(), kv, kv, layout, scale=I.SCALE)
    status_clean(pkg)
