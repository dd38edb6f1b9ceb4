"""Float64 stochastic acceptance law of the reference (TEST INFRASTRUCTURE ONLY).

numpy restatement of ``dspark_qwen/tensor_sampling.py`` for the checker side of the
tests: the temperature law, CDF sampling, the residual law and ``verify_proposal``.
Uniforms are taken from an explicit sequence in the order the reference draws them
(one per acceptance test, one for a residual or bonus sample), so a test can replay
the reference's draws exactly. Pinned against fixtures made by running the
reference's own functions with a scripted generator (``tests/golden/make_golden.py``).
"""
import numpy as np

ROUND_COMPLETE, EOS, BUDGET = 0, 1, 2          # stop reasons
EXTRA_NONE, EXTRA_RESIDUAL, EXTRA_BONUS = 0, 1, 2


def logits_to_probabilities(logits, temperature):
    """float64 softmax of logits / T, normalised once more (tensor_sampling.py:38-51)."""
    scaled = np.asarray(logits, dtype=np.float64) / float(temperature)
    m = scaled.max(axis=-1, keepdims=True)
    e = np.exp(scaled - m)
    weights = e / e.sum(axis=-1, keepdims=True)
    return weights / weights.sum(axis=-1, keepdims=True)


def sample_categorical(probs, u):
    """Strict CDF boundary (searchsorted right), past-the-end -> last positive index
    (tensor_sampling.py:77-84)."""
    probs = np.asarray(probs, dtype=np.float64)
    index = int(np.searchsorted(np.cumsum(probs), u, side='right'))
    if index >= probs.size:
        index = int(np.nonzero(probs > 0)[0][-1])
    return index


def residual_distribution(p, q):
    """relu(p - q) / mass (tensor_sampling.py:87-96); zero mass is an error."""
    positive = np.maximum(np.asarray(p, np.float64) - np.asarray(q, np.float64), 0.0)
    mass = positive.sum()
    if not mass > 0:
        raise ValueError('Zero residual mass')
    return positive / mass


def verify_proposal(tokens, q, p, uniforms, max_new_tokens, eos_ids=()):
    """tensor_sampling.py:114-162 with uniforms drawn from ``uniforms`` in order.

    tokens [n], q [n, V] (draft laws), p [n + 1, V] (target laws). Returns
    (emitted tokens, accepted, rejected index or -1, extra kind, stop reason, draws)."""
    it = iter(uniforms)
    draws = 0

    def draw():
        nonlocal draws
        draws += 1
        return float(next(it))

    stops = set(int(e) for e in eos_ids)
    emitted = []

    def reason(token):
        if token in stops:
            return EOS
        return BUDGET if len(emitted) == max_new_tokens else ROUND_COMPLETE

    if max_new_tokens == 0:
        return [], 0, -1, EXTRA_NONE, BUDGET, 0
    n = len(tokens)
    for j in range(n):
        t = int(tokens[j])
        alpha = min(p[j, t] / q[j, t], 1.0)
        if draw() >= alpha:
            replacement = sample_categorical(residual_distribution(p[j], q[j]), draw())
            emitted.append(replacement)
            return emitted, j, j, EXTRA_RESIDUAL, reason(replacement), draws
        emitted.append(t)
        stop = reason(t)
        if stop != ROUND_COMPLETE:
            return emitted, j + 1, -1, EXTRA_NONE, stop, draws
    bonus = sample_categorical(p[n], draw())
    emitted.append(bonus)
    return emitted, n, -1, EXTRA_BONUS, reason(bonus), draws
