"""Host logic of the training-layout tensor-core kernel, checked on CPU.

``dspark_train_plan`` (C-ABI, host only) splits the packed queries into 64-row
tiles per KV head and assigns them to CTAs. A numpy interpreter below walks each
plan item exactly as the kernel does (context key blocks of 128 rows up to the
tile's largest anchor, then one 128-row box starting at the tile's first block
row, with the same visibility ranges) and must reproduce the oracle's
block_mask attention (dspark_qwen/model.py:12-19,47-61). Every query row and
head must be produced exactly once, and the schedule must be balanced.
"""
import numpy as np
import pytest

import inputs as I
from oracle import training_layout_attention

TILE_Q, KEY_BLOCK, ITEM_WORDS, HEADER = 64, 128, 24, 8
MAGIC = 0x44535431


def plan_items(plan):
    plan = np.asarray(plan, dtype=np.int64)
    assert plan[0] == MAGIC
    n_items, grid = int(plan[1]), int(plan[2])
    offs = plan[HEADER:HEADER + grid + 1]
    at = ((HEADER + grid + 1) + 3) & ~3
    items = plan[at:at + n_items * ITEM_WORDS].reshape(n_items, ITEM_WORDS)
    return grid, offs, items, int(plan[3]), int(plan[4])


def interpret(plan, q, k, v, scale):
    """The kernel's walk over the plan, in float64 (zero rows past the key tensor)."""
    grid, offs, items, total_q, total_k = plan_items(plan)
    out = np.full(q.shape, np.nan)
    seen = np.zeros(q.shape[:2], dtype=np.int64)
    kpad = np.concatenate([k, np.zeros((2 * KEY_BLOCK,) + k.shape[1:], k.dtype)])
    vpad = np.concatenate([v, np.zeros((2 * KEY_BLOCK,) + v.shape[1:], v.dtype)])
    for c in range(grid):
        for it in items[offs[c]:offs[c + 1]]:
            q0, nq, g, kbase, ctx_keys, blk0, phase, nblocks, bs = (int(x) for x in it[:9])
            anchors = it[12:24]
            nctx = -(-ctx_keys // KEY_BLOCK)
            for qi in range(nq):
                rel = (phase + qi) // bs
                assert rel < nblocks
                anchor = min(max(int(anchors[rel]), 0), ctx_keys)
                keys, mask = [], []
                for n in range(nctx):
                    rows = kbase + n * KEY_BLOCK + np.arange(KEY_BLOCK)
                    keys.append(rows)
                    mask.append(n * KEY_BLOCK + np.arange(KEY_BLOCK) < anchor)
                rows = blk0 + np.arange(KEY_BLOCK)
                keys.append(rows)
                cols = np.arange(KEY_BLOCK)
                vis = (cols >= rel * bs) & (cols < rel * bs + bs)
                assert rows[vis].max() < total_k            # visible block rows are real rows
                mask.append(vis)
                keys, mask = np.concatenate(keys), np.concatenate(mask)
                for h in (2 * g, 2 * g + 1):
                    s = kpad[keys, g].astype(np.float64) @ q[q0 + qi, h].astype(np.float64) * scale
                    s = np.where(mask, s, -np.inf)
                    p = np.exp(s - s.max())
                    out[q0 + qi, h] = (p @ vpad[keys, g].astype(np.float64)) / p.sum()
                    seen[q0 + qi, h] += 1
    assert (seen == 1).all(), 'every query row and head exactly once'
    return out


def build(lib_pkg, ctx, anchors, bs, grid_limit=148):
    from importlib import import_module
    _lib = import_module('qwen3-dspark_b200._lib')
    return _lib.train_plan(list(ctx), [len(a) for a in anchors], [x for a in anchors for x in a], bs, grid_limit)


CASES = [
    ('fixture', [c for c, _ in I.TRAIN_SEQS], [list(a) for _, a in I.TRAIN_SEQS], 7),
    ('edges', [0, 1, 130, 300], [[0, 0], [1, 0, 1], [130, 0, 129, 128, 5, 64, 200, -3, 1], [299, 7]], 7),
    ('unsorted-bs13', [257, 40], [[250, 3, 100, 17, 256, 0], [39, 1, 20]], 13),
    ('bs6-bs32', [512], [[int(x) for x in np.linspace(0, 511, 23)]], 6),
    ('no-anchor-seq', [100, 80, 60], [[50, 99], [], [59, 0, 30]], 32),
]


@pytest.mark.parametrize('name,ctx,anchors,bs', CASES, ids=[c[0] for c in CASES])
def test_plan_walk_equals_oracle(pkg, name, ctx, anchors, bs):
    plan = build(pkg, ctx, anchors, bs)
    g = I.rng(11)
    nq = sum(len(a) * bs for a in anchors)
    nk = sum(c + len(a) * bs for c, a in zip(ctx, anchors))
    q = g.standard_normal((nq, I.HQ, I.D)).astype(np.float32)
    k = g.standard_normal((nk, I.HKV, I.D)).astype(np.float32)
    v = g.standard_normal((nk, I.HKV, I.D)).astype(np.float32)
    mine = interpret(plan, q, k, v, I.SCALE)
    # the oracle takes the anchors as given (out-of-range ones included)
    ref = training_layout_attention(q, k, v, ctx, anchors, bs, I.SCALE)
    np.testing.assert_allclose(mine, ref, atol=1e-9, rtol=1e-9)


def test_plan_balance_at_config4(pkg):
    """Config 4 (8 x 2048 context, 32 sorted anchors each): 256 items over 148 CTAs,
    the slowest CTA within one item of the mean load."""
    g = I.rng(3)
    anchors = [sorted(g.choice(2047, 32, replace=False).tolist()) for _ in range(8)]
    grid, offs, items, total_q, total_k = plan_items(build(pkg, [2048] * 8, anchors, 7))
    assert (grid, len(items), total_q, total_k) == (148, 256, 8 * 224, 8 * (2048 + 224))
    cost = -(-items[:, 4] // KEY_BLOCK) + 2
    loads = np.array([cost[offs[c]:offs[c + 1]].sum() for c in range(grid)])
    assert loads.max() <= loads.mean() + cost.max()
    assert sorted(offs.tolist()) == offs.tolist() and offs[-1] == len(items)


def test_plan_refusals(pkg):
    from importlib import import_module
    _lib = import_module('qwen3-dspark_b200._lib')
    for bs in (5, 33):
        with pytest.raises(ValueError):
            _lib.train_plan([10], [1], [3], bs, 148)
    with pytest.raises(ValueError):
        _lib.train_plan([-1], [1], [3], 7, 148)
    with pytest.raises(ValueError):
        pkg.TrainingLayout.from_anchors([10, 20], [[1], []], 40, device='cpu', grid_limit=4)
    with pytest.raises(ValueError):
        pkg.TrainingLayout.from_anchors([10], [[]], 7, device='cpu', grid_limit=4)
