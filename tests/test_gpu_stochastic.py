"""On-device stochastic acceptance (``dspark_stochastic_accept``) against the
reference's float64 law: the decisions of ``tensor_sampling.verify_proposal`` run by
the reference on the seeded cases of ``inputs.stochastic_case`` (fixture
``stochastic_accept``: emitted tokens, accepted count, rejected index, extra kind,
stop reason and uniforms used) must be reproduced exactly, per case and batched, from
f32 and bf16 target logits; the reference's refusals become status codes."""
import numpy as np
import pytest
import torch

import inputs as I
from gpu_util import dev, status_clean

pytestmark = pytest.mark.gpu


def pack(cases, dtype):
    rows, qs, toks, cu, us, budget = [], [], [], [0], [], []
    width = max(c['tokens'].size for c in cases) + 1
    for c in cases:
        rows.append(c['target_logits'])
        qs.append(c['q'])
        toks.append(c['tokens'])
        cu.append(cu[-1] + c['tokens'].size)
        u = np.zeros(width)
        u[:c['uniforms'].size] = c['uniforms']
        us.append(u)
        budget.append(c['budget'])
    vocab = cases[0]['vocab']
    logits = torch.from_numpy(np.concatenate(rows)).to(dev(), dtype)
    q = torch.from_numpy(np.concatenate(qs) if sum(x.shape[0] for x in qs) else np.zeros((0, vocab))).to(dev())
    tokens = torch.from_numpy(np.concatenate(toks).astype(np.int64)).to(dev())
    return (logits, tokens, q, torch.tensor(cu, dtype=torch.int32, device=dev()),
            torch.from_numpy(np.stack(us)).to(dev()), torch.tensor(budget, dtype=torch.int32, device=dev()))


def check(result, emitted, g, idx, i):
    res = result[i].tolist()
    want = g[f'case{idx}_decision'].tolist()
    tokens = g[f'case{idx}_tokens'].tolist()
    assert res[6] == 0, (idx, res)
    assert res[1:6] == want, (idx, res, want)
    assert res[0] == len(tokens)
    assert emitted[i, :res[0]].tolist() == tokens, idx
    assert (emitted[i, res[0]:] == -1).all()


@pytest.mark.parametrize('dtype', [torch.float32, torch.bfloat16])
def test_each_case_matches_reference(pkg, golden, dtype):
    g = golden('stochastic_accept')
    for idx in range(I.STOCH_CASES):
        c = I.stochastic_case(idx)
        emitted, result = pkg.stochastic_accept(*pack([c], dtype)[:4], c['temperature'], *pack([c], dtype)[4:],
                                                eos_ids=c['eos'])
        check(result.cpu(), emitted.cpu(), g, idx, 0)
    status_clean(pkg)


def test_batched_requests_match_reference(pkg, golden):
    g = golden('stochastic_accept')
    for temperature in (0.6, 1.0, 1.7):
        idxs = [i for i in range(I.STOCH_CASES) if I.stochastic_case(i)['temperature'] == temperature
                and not I.stochastic_case(i)['eos'] and I.stochastic_case(i)['vocab'] == I.STOCH_SMALL_VOCAB]
        cases = [I.stochastic_case(i) for i in idxs]
        logits, tokens, q, cu, u, budget = pack(cases, torch.float32)
        emitted, result = pkg.stochastic_accept(logits, tokens, q, cu, temperature, u, budget)
        emitted, result = emitted.cpu(), result.cpu()
        for i, idx in enumerate(idxs):
            check(result, emitted, g, idx, i)
    status_clean(pkg)


def test_refusals_become_status_codes(pkg):
    c = I.stochastic_case(5)                       # 5 proposals, vocab 1000
    base = pack([c], torch.float32)

    def run(**kw):
        logits, tokens, q, cu, u, budget = [kw.get(k, v) for k, v in
                                            zip(('logits', 'tokens', 'q', 'cu', 'u', 'budget'), base)]
        _, result = pkg.stochastic_accept(logits, tokens, q, cu, 1.0, u, budget)
        return result[0].tolist()

    assert run()[6] == 0
    q_bad = base[2].clone()
    q_bad[1] *= 1.001
    assert run(q=q_bad)[6] == 2
    t_bad = base[1].clone()
    t_bad[0] = c['vocab']
    assert run(tokens=t_bad)[6] == 3
    q_zero = base[2].clone()
    t0 = int(base[1][0])
    other = (t0 + 1) % c['vocab']
    q_zero[0, other] += q_zero[0, t0]
    q_zero[0, t0] = 0.0
    assert run(q=q_zero)[6] == 4
    l_nan = base[0].clone()
    l_nan[2, 7] = float('nan')
    assert run(logits=l_nan)[6] == 1
    u_bad = base[4].clone()
    u_bad[0, 0] = 1.0
    assert run(u=u_bad)[6] == 6
    res = run(budget=torch.zeros(1, dtype=torch.int32, device=dev()))
    assert res[:7] == [0, 0, -1, 0, 2, 0, 0]
    status_clean(pkg)
