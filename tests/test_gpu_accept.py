"""On-device greedy acceptance (row argmax + the accept rule of cached_decode.py:84-98)
vs torch.argmax and the host rule ``accept_greedy``, bit-exact on integers."""
import numpy as np
import pytest
import torch

from gpu_util import dev, status_clean

pytestmark = pytest.mark.gpu


def case(seed, qlens, vocab, dtype, eos_ids=(), budgets=None, ties=False, nan_row=None):
    from importlib import import_module
    spec = import_module('qwen3-dspark_b200.speculative')
    g = np.random.Generator(np.random.PCG64(seed))
    n = sum(qlens)
    logits = torch.from_numpy(g.standard_normal((n, vocab)).astype(np.float32)).to(dev(), dtype)
    if ties:                                   # duplicate each row's max at a later and an earlier index
        am = logits.float().argmax(-1)
        for row in range(0, n, 3):
            j = int(am[row])
            logits[row, (j + 7) % vocab] = logits[row, j]
            logits[row, max(j - 5, 0)] = logits[row, j]
    if nan_row is not None:
        logits[nan_row, vocab // 2] = float('nan')
        logits[nan_row, vocab // 3] = float('nan')
    pred = logits.float().argmax(-1).cpu().numpy()
    tokens = np.zeros(n, dtype=np.int64)
    off = 0
    for q in qlens:
        tokens[off] = g.integers(0, vocab)
        agree = g.integers(0, q)               # proposals matching the predictions before them
        for j in range(q - 1):
            tokens[off + 1 + j] = pred[off + j] if j < agree else (pred[off + j] + 1 + g.integers(0, 3)) % vocab
        off += q
    for e in eos_ids:                          # place some EOS tokens among accepted proposals / predictions
        tokens[min(2, n - 1)] = e
    return logits, tokens, pred, spec.accept_greedy


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
@pytest.mark.parametrize('vocab', [1024, 151936, 1001])
def test_argmax_and_accept_match_host(pkg, dtype, vocab):
    qlens = [8, 1, 5, 8, 3, 8]
    logits, tokens, pred, accept = case(vocab, qlens, vocab, dtype, ties=True, nan_row=4)
    cu = np.concatenate([[0], np.cumsum(qlens)]).astype(np.int32)
    budgets = np.array([8, 0, 2, 3, 8, 1], dtype=np.int32)
    eos = (int(tokens[2]),)
    got_pred, acc, ncommit, emitted = pkg.greedy_accept(
        logits, torch.from_numpy(tokens).to(dev()), torch.from_numpy(cu).to(dev()), eos,
        torch.from_numpy(budgets).to(dev()))
    torch.cuda.synchronize()
    ref_pred = logits.float().argmax(-1).cpu().numpy()
    assert (got_pred.cpu().numpy() == ref_pred).all()
    acc, ncommit, emitted = acc.cpu().numpy(), ncommit.cpu().numpy(), emitted.cpu().numpy()
    for i, q in enumerate(qlens):
        a, b = cu[i], cu[i + 1]
        accepted, committed = accept(tokens[a + 1:b].tolist(), ref_pred[a:b].tolist(), set(eos))
        committed = committed[:budgets[i]]
        assert acc[i] == accepted, i
        assert ncommit[i] == len(committed), i
        assert emitted[a:a + len(committed)].tolist() == committed, i
        assert (emitted[a + len(committed):b] == -1).all(), i
    status_clean(pkg)


def test_accept_without_budget_or_eos(pkg):
    qlens = [7] * 16
    logits, tokens, pred, accept = case(3, qlens, 4096, torch.bfloat16)
    cu = torch.tensor(np.concatenate([[0], np.cumsum(qlens)]), dtype=torch.int32, device=dev())
    _, acc, ncommit, emitted = pkg.greedy_accept(logits, torch.from_numpy(tokens).to(dev()), cu)
    ref_pred = logits.float().argmax(-1).cpu().numpy()
    for i in range(16):
        a = 7 * i
        accepted, committed = accept(tokens[a + 1:a + 7].tolist(), ref_pred[a:a + 7].tolist())
        assert int(acc[i]) == accepted and int(ncommit[i]) == len(committed)
        assert emitted[a:a + len(committed)].tolist() == committed
    status_clean(pkg)


def test_refusals(pkg):
    logits = torch.zeros(4, 16, dtype=torch.bfloat16, device=dev())
    tokens = torch.zeros(4, dtype=torch.long, device=dev())
    cu = torch.tensor([0, 4], dtype=torch.int32, device=dev())
    with pytest.raises(ValueError):
        pkg.greedy_accept(logits, tokens[:3], cu)
    with pytest.raises(ValueError):
        pkg.greedy_accept(logits, tokens, cu.long())
    with pytest.raises(ValueError):
        pkg.greedy_accept(logits, tokens, cu, budget=torch.zeros(2, dtype=torch.int32, device=dev()))


@pytest.mark.parametrize('dtype', [torch.bfloat16, torch.float32])
def test_argmax_edges_match_torch(pkg, dtype):
    """dspark_row_argmax vs torch.argmax: equal maxima at the two ends of a row (the
    lowest index wins), rows of -inf only (index 0), signed zeros (equal), NaN
    (the first one), rows all equal, tiny vocabularies, and rows that are not
    16-byte aligned (a padded leading dimension)."""
    from importlib import import_module
    _lib = import_module('qwen3-dspark_b200._lib')
    lib = _lib.load_library()
    code = _lib.DTYPE_BF16 if dtype == torch.bfloat16 else _lib.DTYPE_F32
    stream = torch.cuda.current_stream().cuda_stream
    for vocab, ld in ((151936, 151936), (1001, 1003), (7, 7), (3, 5), (1, 1), (4099, 4099)):
        g = torch.Generator(device='cpu').manual_seed(vocab)
        buf = torch.randn(12, ld, generator=g).to(dtype)
        x = buf[:, :vocab]
        x[0, vocab - 1] = 50.0
        x[0, 0] = 50.0                                   # first and last element tie
        x[1] = float('-inf')                             # nothing but -inf
        x[2] = -1.0
        x[2, vocab // 2] = -0.0
        x[2, vocab - 1] = 0.0                            # -0 == +0: the earlier one
        x[3, vocab // 3] = float('nan')                  # NaN beats numbers
        x[4, vocab - 1] = float('nan')
        x[4, vocab // 4] = float('nan')                  # the first NaN
        x[5] = 1.0                                       # all equal: index 0
        buf_d = buf.to(dev())
        pred = torch.empty(12, dtype=torch.int32, device=dev())
        _lib.check(lib.dspark_row_argmax(buf_d.data_ptr(), ld, 12, vocab, code, pred.data_ptr(), stream),
                   'dspark_row_argmax')
        torch.cuda.synchronize()
        ref = buf[:, :vocab].float().argmax(-1).to(torch.int32)
        assert torch.equal(pred.cpu(), ref), (vocab, ld, pred.cpu().tolist(), ref.tolist())
    status_clean(pkg)
