"""Fused greedy Markov proposal (tcgen05 GEMM + in-TMEM argmax) vs the reference's
torch formula (DSparkDraft._sample_greedy, dspark_qwen/model.py:210-221) in bf16.

Each step is compared given the same previous token. The kernel's fp32 dot is
accumulated in a different order than a library GEMM, so after the reference's
bf16 rounding two logits can land one bf16 ulp apart the other way: a token may
differ only where the reference's own top logits are within one ulp, and at
least 98% of tokens must be identical.
"""
import numpy as np
import pytest
import torch

from gpu_util import dev, status_clean

pytestmark = pytest.mark.gpu


def make(seed, r, vocab, rank, hdim, block=7):
    g = torch.Generator(device='cpu').manual_seed(seed)
    bf = torch.bfloat16
    w = (torch.randn(vocab, rank, generator=g) * 0.05).to(bf)
    e = (torch.randn(vocab, rank, generator=g) * 0.5).to(bf)
    cw = (torch.randn(hdim + rank, generator=g) * 0.05).to(bf)
    cb = 0.1
    hidden = torch.randn(r * block, hdim, generator=g).to(bf)
    base = (torch.randn(r * block, vocab, generator=g) * 0.5).to(bf)
    anchors = torch.randint(0, vocab, (r,), generator=g)
    return [x.to(dev()) for x in (w, e, cw, hidden, base, anchors)] + [cb]


def ref_step(w, e, cw, cb, hidden_k, base_k, prev):
    emb = e[prev]                                                     # bf16 [R, rank]
    lin = torch.nn.functional.linear(torch.cat((hidden_k, emb), -1), cw[None], torch.tensor([cb], dtype=cw.dtype,
                                                                                             device=cw.device))
    conf = lin.sigmoid().flatten().float()
    logits = base_k + torch.nn.functional.linear(emb, w)             # bf16 projection, bf16 sum
    return logits, conf


@pytest.mark.parametrize('r,vocab,rank', [(64, 32768, 256), (5, 1024, 64), (128, 4096, 128), (130, 2048, 192)])
def test_markov_steps_match_reference(pkg, r, vocab, rank):
    hdim, block = 1024, 7
    w, e, cw, hidden, base, anchors, cb = make(r + vocab, r, vocab, rank, hdim, block)
    toks, conf = pkg.markov_greedy(w, e, cw, cb, hidden, base, anchors, block)
    torch.cuda.synchronize()
    toks_h = toks.cpu()
    same = total = 0
    for k in range(block):
        prev = anchors if k == 0 else toks[:, k - 1]
        rows = torch.arange(r, device=dev()) * block + k
        logits, rconf = ref_step(w, e, cw, cb, hidden[rows], base[rows], prev)
        ref = logits.float().argmax(-1).cpu()
        got = toks_h[:, k]
        lf = logits.float().cpu()
        for i in range(r):
            total += 1
            if got[i] == ref[i]:
                same += 1
                continue
            top, mine = lf[i, ref[i]].item(), lf[i, got[i]].item()
            ulp = 2.0 ** (np.floor(np.log2(max(abs(top), 1e-30))) - 7)
            assert top - mine <= ulp, (k, i, top, mine)
        np.testing.assert_allclose(conf[:, k].cpu().numpy(), rconf.cpu().numpy(), atol=1e-2)
    assert same / total >= 0.98, same / total
    status_clean(pkg)


def test_packed_draft_uses_fused_markov(pkg):
    """propose_greedy of a bf16 draft with rank 64 goes through markov_greedy and gives
    the tokens of the torch loop on the same backbone output (near-tie rule)."""
    import inputs as I
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(**I.TINY_TARGET)
    model = Qwen3ForCausalLM(cfg).eval()
    shapes = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    model.load_state_dict({k: torch.from_numpy(v) for k, v in I.deterministic_state(shapes, 1).items()})
    model = model.to(dev(), torch.bfloat16)
    spec = pkg.DraftSpec(**dict(I.TINY_DRAFT, markov_rank=64))
    draft = pkg.DSparkDraftModel(model, spec).eval()
    dshapes = {k: tuple(v.shape) for k, v in draft.state_dict().items() if not k.startswith(('embedding.', 'lm_head.'))}
    draft.load_state_dict({k: torch.from_numpy(v) for k, v in I.deterministic_state(dshapes, 2).items()}, strict=False)
    draft = draft.to(dev(), torch.bfloat16)
    pd = pkg.B200PackedDraft(draft, max_requests=4, context_capacity=300)
    g = np.random.Generator(np.random.PCG64(9))
    for i in range(4):
        pd.add_request(f'q{i}')
        ctx = torch.from_numpy(g.standard_normal((1, 20 + 30 * i, 256 * len(spec.layer_ids))).astype(np.float32))
        pd.append_committed({f'q{i}': ctx.to(dev(), torch.bfloat16)})
    anchors = {f'q{i}': torch.tensor([[int(g.integers(0, 1000))]], device=dev()) for i in range(4)}
    proposed = pd.propose_greedy(anchors)
    feats = pd.backbone(anchors)
    hidden = feats.hidden.reshape(4 * 7, -1)
    base = draft.lm_head(hidden)
    d = draft
    for i, q in enumerate(feats.requests):
        prev = anchors[q].view(1)
        toks = proposed[q][0]
        for k in range(7):
            emb = d.markov_embedding(prev)
            logits = (base[i * 7 + k] + d.markov_projection(emb)[0]).float()
            ref = int(logits.argmax())
            if toks[k] != ref:
                assert logits[ref] - logits[toks[k]] <= 2.0 ** (np.floor(np.log2(abs(float(logits[ref])))) - 7)
            prev = torch.tensor([toks[k]], device=dev())
    status_clean(pkg)


def test_markov_block_launch_equals_step_launches(pkg):
    """All positions of a block in one cooperative launch (dspark_markov_block) give
    the tokens and confidences of one launch per position (dspark_markov_step),
    bit for bit: 128 requests, a vocabulary whose last tile is partial, twice in a
    row (the scratch is left usable)."""
    from importlib import import_module
    _lib = import_module('qwen3-dspark_b200._lib')
    kern = import_module('qwen3-dspark_b200.kernels')
    r, vocab, rank, hdim, block = 128, 65544, 256, 1024, 7
    w, e, cw, hidden, base, anchors, cb = make(77, r, vocab, rank, hdim, block)
    lib = _lib.load_library()
    stream = torch.cuda.current_stream().cuda_stream
    for rep in range(2):
        fused_t, fused_c = pkg.markov_greedy(w, e, cw, cb, hidden, base, anchors, block)
        scratch = torch.zeros(int(lib.dspark_markov_scratch_bytes()), dtype=torch.uint8, device=dev())
        toks = torch.empty((r, block), dtype=torch.long, device=dev())
        conf = torch.empty((r, block), dtype=torch.float32, device=dev())
        for k in range(block):
            prev, stride = (anchors.data_ptr(), 1) if k == 0 else (toks[:, k - 1:].data_ptr(), block)
            _lib.check(lib.dspark_markov_step(w.data_ptr(), e.data_ptr(), vocab, rank, base.data_ptr(), block, k, prev,
                                              stride, hidden.data_ptr(), hdim, cw.data_ptr(), float(cb),
                                              toks.data_ptr(), conf.data_ptr(), block, r, scratch.data_ptr(), stream),
                       'dspark_markov_step')
        torch.cuda.synchronize()
        assert torch.equal(fused_t, toks), rep
        assert torch.equal(fused_c, conf), rep
        assert int(scratch[:3 * 128 * 8].count_nonzero()) == 0
        key = (dev().index, torch.cuda.current_stream().cuda_stream)
        assert int(kern._markov_scratch[key][:3 * 128 * 8 + 4].count_nonzero()) == 0   # best buffers, counter
    status_clean(pkg)


def test_markov_ties_zero_and_nan_follow_torch_argmax(pkg):
    """With a zero projection the logits are exactly the bf16 base rows, so the
    kernel must pick torch.argmax's index: planted equal maxima in different tiles
    (and CTAs) resolve to the lowest index, -0 and +0 compare equal, a NaN wins
    (the first NaN)."""
    r, vocab, rank, hdim, block = 6, 40960, 64, 256, 2
    w, e, cw, hidden, base, anchors, cb = make(5, r, vocab, rank, hdim, block)
    w.zero_()
    b = (-torch.rand(r * block, vocab, device=dev()) - 1.0).to(torch.bfloat16)   # all in [-2, -1)
    b[0, 300] = b[0, 39000] = 5.0                    # equal maxima in different tiles
    b[1, 17] = b[1, 18] = 3.0                        # adjacent equal maxima
    b[2, 5000] = -0.0
    b[2, 100] = 0.0                                  # +0 before -0: the lower index wins
    b[3, 7000] = float('nan')
    b[3, 20000] = float('nan')
    b[3, 10] = 9.0                                   # NaN beats 9
    b[4, vocab - 1] = 7.0                            # the last column of the vocabulary
    b[5:7, 123] = 1.0
    toks, _ = pkg.markov_greedy(w, e, cw, cb, hidden, b, anchors, block)
    torch.cuda.synchronize()
    for k in range(block):
        rows = torch.arange(r, device=dev()) * block + k
        ref = (b[rows].float() + 0.0).argmax(-1)
        assert torch.equal(toks[:, k], ref), (k, toks[:, k].tolist(), ref.tolist())
    status_clean(pkg)


@pytest.mark.parametrize('block', [1, 2, 65])
def test_markov_block_sizes_equal_step_launches(pkg, block):
    """Blocks of one and two positions (the fused launch's buffer rotation at its
    shortest) and of 65 positions (over the fused limit: one launch per position)
    give the per-position launches' tokens and confidences bit for bit, and leave
    the scratch ready for the next call."""
    from importlib import import_module
    _lib = import_module('qwen3-dspark_b200._lib')
    kern = import_module('qwen3-dspark_b200.kernels')
    r, vocab, rank, hdim = 64, 8192, 128, 256
    w, e, cw, hidden, base, anchors, cb = make(block + 3, r, vocab, rank, hdim, block)
    lib = _lib.load_library()
    stream = torch.cuda.current_stream().cuda_stream
    for rep in range(2):
        fused_t, fused_c = pkg.markov_greedy(w, e, cw, cb, hidden, base, anchors, block)
        scratch = torch.zeros(int(lib.dspark_markov_scratch_bytes()), dtype=torch.uint8, device=dev())
        toks = torch.empty((r, block), dtype=torch.long, device=dev())
        conf = torch.empty((r, block), dtype=torch.float32, device=dev())
        for k in range(block):
            prev, stride = (anchors.data_ptr(), 1) if k == 0 else (toks[:, k - 1:].data_ptr(), block)
            _lib.check(lib.dspark_markov_step(w.data_ptr(), e.data_ptr(), vocab, rank, base.data_ptr(), block, k, prev,
                                              stride, hidden.data_ptr(), hdim, cw.data_ptr(), float(cb),
                                              toks.data_ptr(), conf.data_ptr(), block, r, scratch.data_ptr(), stream),
                       'dspark_markov_step')
        torch.cuda.synchronize()
        assert torch.equal(fused_t, toks), (block, rep)
        assert torch.equal(fused_c, conf), (block, rep)
        key = (dev().index, torch.cuda.current_stream().cuda_stream)
        assert int(kern._markov_scratch[key][:3 * 128 * 8 + 4].count_nonzero()) == 0
    status_clean(pkg)


def test_grid_barrier_timeout_is_reported_and_the_next_call_is_correct(pkg):
    """Failure handling of the block kernel's grid barrier, made on purpose without a GPU
    fault: with the barrier's limit lowered to zero, CTAs that wait for the others give up
    at the first barrier, raise their abort flags and leave after draining their copies
    and MMAs (those waits keep the two-second limit). The call returns, the status word
    reports DSPARK_DEVICE_WAIT_TIMEOUT, and the next call on the same stream, with the
    limit restored, gives exactly the tokens and confidences of a clean call: the last CTA
    out of the failed call returned the shared scratch to zero."""
    r, vocab, rank, hdim, block = 64, 32768, 256, 1024, 7
    w, e, cw, hidden, base, anchors, cb = make(77, r, vocab, rank, hdim, block)
    pkg.read_device_status(clear=True)
    clean, clean_conf = pkg.markov_greedy(w, e, cw, cb, hidden, base, anchors, block)
    torch.cuda.synchronize()
    assert pkg.read_device_status(clear=True) == 0
    try:
        pkg._lib.set_grid_barrier_timeout(0)
        pkg.markov_greedy(w, e, cw, cb, hidden, base, anchors, block)
        torch.cuda.synchronize()
    finally:
        pkg._lib.set_grid_barrier_timeout()
    assert pkg.read_device_status(clear=True) & pkg._lib.DEVICE_WAIT_TIMEOUT
    for _ in range(2):
        again, conf = pkg.markov_greedy(w, e, cw, cb, hidden, base, anchors, block)
        torch.cuda.synchronize()
        assert torch.equal(again, clean)
        assert torch.equal(conf, clean_conf)
    status_clean(pkg)
