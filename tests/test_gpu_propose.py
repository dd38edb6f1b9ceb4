"""On-device stochastic draft proposal of one Markov position (``dspark_stochastic_propose``)
against the reference's formula run with torch on the same GPU: x = base + proj in bf16,
the float64 law softmax(x / T) normalised once more (tensor_sampling.py:38-51,
``float64_law``) and the strict CDF draw with the last positive index past the end
(tensor_sampling.py:77-84, ``sample_rows``). Tokens must be identical and laws equal to
within float64 rounding (the row sums are added in a different order); strided rows,
row indices, uniforms at the edges and a non-finite row are covered; the bf16 draft's
``propose_stochastic`` must equal the torch formula applied to the same backbone."""
import pytest
import torch

from gpu_util import dev, status_clean

pytestmark = pytest.mark.gpu


def torch_formula(pkg, base, proj, temperature, uniforms):
    law = pkg.float64_law(base + proj, temperature)
    return pkg.sample_rows(law, uniforms), law


# 24 rows run two CTAs per row (a cluster; with vocab 1000 / 997 the second CTA's half
# is empty), 100 rows one CTA per row (twice the rows would not fit the SMs at once).
@pytest.mark.parametrize('vocab,temperature,n', [(151936, 0.8, 24), (151936, 1.3, 24), (1000, 1.0, 24),
                                                 (997, 0.6, 24), (151936, 0.8, 100)])
def test_law_and_token_equal_the_torch_formula(pkg, vocab, temperature, n):
    g = torch.Generator(device=dev())
    g.manual_seed(vocab + int(temperature * 10) + n)
    # strided base / law rows (every other row of a larger buffer), row indices reversed
    base_buf = (torch.randn((2 * n, vocab), generator=g, device=dev()) * 3).to(torch.bfloat16)
    base = base_buf[::2]
    proj = (torch.randn((n, vocab), generator=g, device=dev()) * 2).to(torch.bfloat16)
    row_index = torch.arange(n - 1, -1, -1, dtype=torch.int32, device=dev())
    u = torch.rand(n, generator=g, device=dev(), dtype=torch.float64)
    u[0], u[1], u[2] = 0.0, 1.0 - 2.0 ** -53, 0.5
    law_buf = torch.full((2 * n, vocab), -1.0, dtype=torch.float64, device=dev())
    law = law_buf[::2]
    tok, status = pkg.stochastic_propose(base, row_index, proj, temperature, u, law)
    torch.cuda.synchronize()
    assert int(status.abs().sum()) == 0
    want_tok, want_law = torch_formula(pkg, base[row_index.long()], proj, temperature, u)
    assert torch.equal(tok, want_tok)
    got_law = law[row_index.long()]
    assert torch.allclose(got_law, want_law, rtol=1e-12, atol=1e-300)
    assert (law_buf[1::2] == -1.0).all()                  # the rows in between are untouched
    status_clean(pkg)


def test_crossing_at_the_last_index_and_peaked_laws(pkg):
    """A law whose mass sits in the last column (the crossing is the last index) and a
    law with one dominant column; the draw falls where the torch formula's falls."""
    vocab = 4096
    base = torch.full((3, vocab), -30.0, device=dev()).to(torch.bfloat16)
    base[0, -1] = 30.0
    base[1, 1234] = 30.0
    base[2, :] = 0.0
    proj = torch.zeros((3, vocab), device=dev(), dtype=torch.bfloat16)
    u = torch.tensor([0.999999, 0.3, 0.999999999], dtype=torch.float64, device=dev())
    law = torch.empty((3, vocab), dtype=torch.float64, device=dev())
    idx = torch.arange(3, dtype=torch.int32, device=dev())
    tok, status = pkg.stochastic_propose(base, idx, proj, 1.0, u, law)
    want_tok, want_law = torch_formula(pkg, base, proj, 1.0, u)
    assert torch.equal(tok, want_tok) and tok.tolist()[:2] == [vocab - 1, 1234]
    assert torch.allclose(law, want_law, rtol=1e-12, atol=1e-300)
    assert int(status.abs().sum()) == 0
    status_clean(pkg)


def test_non_finite_row_reports_and_stays_in_range(pkg):
    vocab = 2048
    base = torch.randn((2, vocab), device=dev()).to(torch.bfloat16)
    base[1, 7] = float('nan')
    proj = torch.zeros_like(base)
    law = torch.empty((2, vocab), dtype=torch.float64, device=dev())
    idx = torch.arange(2, dtype=torch.int32, device=dev())
    u = torch.tensor([0.25, 0.25], dtype=torch.float64, device=dev())
    tok, status = pkg.stochastic_propose(base, idx, proj, 1.0, u, law)
    assert status.tolist() == [0, 1]
    assert 0 <= int(tok[1]) < vocab
    status_clean(pkg)


def test_refusals_before_launch(pkg):
    base = torch.zeros((2, 64), device=dev(), dtype=torch.bfloat16)
    idx = torch.arange(2, dtype=torch.int32, device=dev())
    u = torch.zeros(2, dtype=torch.float64, device=dev())
    law = torch.empty((2, 64), dtype=torch.float64, device=dev())
    with pytest.raises(ValueError):
        pkg.stochastic_propose(base.float(), idx, base, 1.0, u, law)       # float32 logits
    with pytest.raises(ValueError):
        pkg.stochastic_propose(base, idx, base, 0.0, u, law)               # temperature
    with pytest.raises(ValueError):
        pkg.stochastic_propose(base, idx, base[:, :32], 1.0, u, law)       # vocab mismatch


def test_bf16_draft_proposal_equals_the_torch_formula(pkg):
    """``B200PackedDraft.propose_stochastic`` on a bf16 draft (fused per-position kernel)
    against the same positions evaluated with the torch formula from the same backbone
    and LM-head rows; requests of different limits."""
    import bench
    draft = bench.build_draft_06b(pkg, dev())
    pd = pkg.B200PackedDraft(draft, max_requests=4, context_capacity=512)
    g = torch.Generator(device=dev())
    g.manual_seed(5)
    names = [f'r{i}' for i in range(4)]
    for i, r in enumerate(names):
        pd.add_request(r)
        pd.append_committed({r: torch.randn((1, 64 + 40 * i, 5 * 1024), generator=g, device=dev(),
                                            dtype=torch.bfloat16)})
    anchors = {r: torch.tensor([[100 + 7 * i]], device=dev()) for i, r in enumerate(names)}
    limits = {r: lim for r, lim in zip(names, (7, 3, 0, 5))}
    u = torch.rand((4, 7), generator=g, device=dev(), dtype=torch.float64)
    with torch.no_grad():
        toks, laws = pd.propose_stochastic(anchors, limits, u, 0.9)
        feats = pd.backbone(anchors)
        d = draft
        hidden = feats.hidden.reshape(4, 7, -1)
        base = d.lm_head(hidden)
        for i, r in enumerate(names):
            prev = anchors[r].view(1)
            assert toks[r].shape == (limits[r],) and laws[r].shape == (limits[r], base.shape[-1])
            for k in range(limits[r]):
                logits = base[i, k:k + 1] + d.markov_projection(d.markov_embedding(prev))
                want_tok, want_law = torch_formula(pkg, logits, torch.zeros_like(logits), 0.9, u[i, k:k + 1])
                assert int(toks[r][k]) == int(want_tok[0]), (r, k)
                assert torch.allclose(laws[r][k], want_law[0], rtol=1e-12, atol=1e-300)
                prev = toks[r][k:k + 1]
    status_clean(pkg)
