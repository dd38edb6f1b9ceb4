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


# Tiny Qwen3 target with the real attention geometry (16/8 heads, head dim 128)
# for the greedy-speculative parity case; the draft reads target layers 1 and 2.
TINY_TARGET = dict(vocab_size=1024, hidden_size=256, intermediate_size=512, num_hidden_layers=4,
                   num_attention_heads=16, num_key_value_heads=8, head_dim=128, max_position_embeddings=4096,
                   rms_norm_eps=1e-6, tie_word_embeddings=False, attention_dropout=0.0,
                   rope_parameters={'rope_type': 'default', 'rope_theta': 1e6})
TINY_DRAFT = dict(layer_ids=(1, 2), num_layers=2, block_size=7, markov_rank=16, mask_token_id=1023)
GREEDY_PROMPTS = (64, 256, 2048, 64, 256, 100)
GREEDY_NEW_TOKENS = 48
# stochastic speculative decode on the same model: one seeded generator per prompt
STOCH_ROUND_SEED = 4242
STOCH_ROUND_TEMPERATURE = 0.9


def deterministic_state(named_shapes, seed):
    """Weights by parameter name: every name gets its own PCG64 stream, so any module
    tree with the same names and shapes receives the same values on any machine."""
    import zlib
    out = {}
    for name, shape in named_shapes.items():
        g = rng(seed * 1_000_003 + zlib.crc32(name.encode()))
        if name.endswith('norm.weight'):
            x = 1.0 + 0.1 * g.standard_normal(shape)
        elif name.endswith('.bias'):
            x = 0.02 * g.standard_normal(shape)
        else:
            x = 0.05 * g.standard_normal(shape)
        out[name] = x.astype(np.float32)
    return out


def greedy_prompts(seed=55):
    g = rng(seed)
    return [g.integers(0, TINY_TARGET['vocab_size'] - 1, n).astype(np.int64) for n in GREEDY_PROMPTS]


# Stochastic acceptance (tensor_sampling.verify_proposal): seeded cases over a small
# vocabulary and, every fifth case, the Qwen3 vocabulary.
STOCH_SEED = 777
STOCH_CASES = 30
STOCH_SMALL_VOCAB = 1000
QWEN3_VOCAB = 151936


def softmax64(x):
    """float64 softmax normalised twice (a valid law within 1e-12 of sum one)."""
    x = np.asarray(x, dtype=np.float64)
    e = np.exp(x - x.max(axis=-1, keepdims=True))
    w = e / e.sum(axis=-1, keepdims=True)
    return w / w.sum(axis=-1, keepdims=True)


def stochastic_case(idx):
    """One verify_proposal case. Draft laws q [n, V] are float64 softmaxes of seeded
    logits at temperature T; proposals are sampled from q; target logits [n + 1, V]
    (float32 values exact in bf16) are the draft logits plus a case-dependent amount of
    noise; ``uniforms`` holds n + 1 draws (the most a round consumes); ``budget`` is the
    round's max_new_tokens and ``eos`` the stop tokens."""
    from oracle.bf16 import round_bf16
    g = rng(STOCH_SEED + idx)
    vocab = QWEN3_VOCAB if idx % 5 == 4 else STOCH_SMALL_VOCAB
    n = idx % 8
    temperature = (0.6, 1.0, 1.7)[idx % 3]
    draft_logits = g.standard_normal((n, vocab), dtype=np.float32) * 2
    q = softmax64(draft_logits.astype(np.float64) / temperature)
    tokens = np.array([int(min(np.searchsorted(np.cumsum(q[j]), g.random(), side='right'), vocab - 1))
                       for j in range(n)], dtype=np.int64)
    mix = (0.0, 0.05, 0.3, 1.0, 3.0)[idx % 5]
    base = np.concatenate([draft_logits, g.standard_normal((1, vocab), dtype=np.float32) * 2], axis=0)
    target_logits = round_bf16((base + mix * g.standard_normal(base.shape, dtype=np.float32)).astype(np.float32))
    uniforms = g.random(n + 1)
    budget = (100, 100, 3, 1, 0, 100, 2)[idx % 7]
    eos = (int(tokens[1]),) if idx % 6 == 1 and n > 1 else ((5,) if idx % 6 == 3 else ())
    return dict(tokens=tokens, q=q, target_logits=target_logits, temperature=temperature, uniforms=uniforms,
                budget=budget, eos=eos, vocab=vocab)
