"""The float64 stochastic-acceptance oracle (``oracle/sampling.py``) against fixtures
made by running the reference's own ``tensor_sampling.verify_proposal`` and
``logits_to_probabilities`` (tests/golden/make_golden.py: stochastic_fixtures) on the
seeded cases of ``inputs.stochastic_case``: target laws within 1e-14 and every decision
(emitted tokens, accepted count, rejected index, extra kind, stop reason, draws used)
identical."""
import numpy as np

import inputs as I
from oracle import sampling as S


def test_stochastic_oracle_matches_reference(golden):
    g = golden('stochastic_accept')
    kinds = set()
    for idx in range(I.STOCH_CASES):
        c = I.stochastic_case(idx)
        p = S.logits_to_probabilities(c['target_logits'], c['temperature'])
        probe = np.concatenate([np.arange(min(8, c['vocab'])), c['tokens']])
        np.testing.assert_allclose(p[:, probe], g[f'case{idx}_p_probe'], rtol=1e-13, atol=1e-300)
        np.testing.assert_allclose(p.sum(axis=1), g[f'case{idx}_p_rowsum'], rtol=0, atol=1e-13)
        emitted, accepted, rejected, extra, reason, draws = S.verify_proposal(
            c['tokens'], c['q'], p, c['uniforms'], c['budget'], c['eos'])
        assert emitted == g[f'case{idx}_tokens'].tolist(), idx
        assert [accepted, rejected, extra, reason, draws] == g[f'case{idx}_decision'].tolist(), idx
        kinds.add((extra, reason))
    # the cases cover residual and bonus tokens, budget and EOS stops
    assert {(S.EXTRA_RESIDUAL, S.ROUND_COMPLETE), (S.EXTRA_BONUS, S.ROUND_COMPLETE),
            (S.EXTRA_NONE, S.BUDGET), (S.EXTRA_NONE, S.EOS)} <= kinds


def test_sampling_edges():
    probs = np.array([0.25, 0.0, 0.75, 0.0])
    assert S.sample_categorical(probs, 0.0) == 0
    assert S.sample_categorical(probs, 0.25) == 2          # strict boundary: cdf 0.25 <= u -> next
    assert S.sample_categorical(probs, np.nextafter(1.0, 0)) == 2
    with np.testing.assert_raises(ValueError):
        S.residual_distribution(probs, probs)
    out = S.verify_proposal([], np.zeros((0, 4)), probs[None], [0.9], 0)
    assert out == ([], 0, -1, S.EXTRA_NONE, S.BUDGET, 0)
