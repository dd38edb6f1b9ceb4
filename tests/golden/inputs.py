"""Seeded synthetic inputs shared by the golden-fixture generator and the tests.

Only numpy's PCG64 generator is used, so the same seed produces the same bytes
on every machine; fixtures therefore store outputs plus an input digest, not
the (large, incompressible) random inputs themselves.
"""
import hashlib

import numpy as np

HQ, HKV, D = 16, 8, 128
SCALE = 128 ** -0.5
BLOCK = 7


def rng(seed):
    return np.random.Generator(np.random.PCG64(seed))


def normal(g, shape, bf16=False):
    x = g.standard_normal(shape, dtype=np.float32)
    if bf16:
        from oracle.bf16 import round_bf16
        x = round_bf16(x)
    return x


def digest(*arrays):
    h = hashlib.sha256()
    for a in arrays:
        h.update(np.ascontiguousarray(a).tobytes())
    return h.hexdigest()


def draft_case(seed, contexts, bf16, block=BLOCK):
    """Packed draft attention inputs: per request ``block`` queries, keys = context + block."""
    g = rng(seed)
    qlens = [block] * len(contexts)
    klens = [c + block for c in contexts]
    q = normal(g, (sum(qlens), HQ, D), bf16)
    k = normal(g, (sum(klens), HKV, D), bf16)
    v = normal(g, (sum(klens), HKV, D), bf16)
    return q, k, v, qlens, klens


def varlen_case(seed, qlens, klens, bf16, tail=0):
    """Bottom-right causal varlen inputs; ``tail`` extra capacity rows after the last key."""
    g = rng(seed)
    q = normal(g, (sum(qlens), HQ, D), bf16)
    k = normal(g, (sum(klens) + tail, HKV, D), bf16)
    v = normal(g, (sum(klens) + tail, HKV, D), bf16)
    return q, k, v


# Config 1 of the benchmark: 4 requests, contexts [64,128,200,256], one 7-row block each.
CFG1_CONTEXTS = (64, 128, 200, 256)
# Small bf16 draft case with an empty context and odd lengths.
DRAFT_BF16_CONTEXTS = (0, 1, 17, 130, 700)
# Tensor-gate cases of the reference's native varlen probe (scripts/probe_varlen.py:26-33).
PROBE_CASES = (((1, 8), (17, 29)), ((3, 2, 1), (11, 5, 1)), ((2,), (2,)))
PROBE_SEED = 20261009
# Capacity-tail verify case: 7-row verify chunks over cached prefixes, NaN tail.
CAPACITY_QLENS = (7, 7, 3, 8)
CAPACITY_KLENS = (300, 57, 10, 1031)
CAPACITY_TAIL = 37
# Training-layout draft case: per sequence (context length, anchors).
TRAIN_SEQS = ((40, (0, 2, 6, 39)), (64, (5, 17, 18, 63, 30)))
# QK-norm + RoPE positions: verify chunks at these committed context lengths.
ROPE_CONTEXTS = (0, 255, 4000, 8191)
ROPE_THETA = 1e6
RMS_EPS = 1e-6
