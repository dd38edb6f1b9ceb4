"""CUDA-graph capture and replay of the B200 verify forward (the counterpart of the
reference's fixed-buffer graph execution, persistent_qwen_graph.py:198-275).

One bucket (exact ordered query lengths) is captured once; every later verify
round of that bucket replays it after the host metadata is written into the
bucket's fixed buffers. The replayed logits must equal an eager verify of the
same round bit for bit, across rounds whose contexts and commits differ, and
commit/rollback after a replay must leave the same KV as after an eager verify.
"""
import numpy as np
import pytest
import torch

import inputs as I
from gpu_util import dev, status_clean

pytestmark = pytest.mark.gpu


def tiny_bf16_model():
    from transformers import Qwen3Config, Qwen3ForCausalLM
    cfg = Qwen3Config(**I.TINY_TARGET)
    cfg._attn_implementation = 'sdpa'
    model = Qwen3ForCausalLM(cfg).eval()
    shapes = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    model.load_state_dict({k: torch.from_numpy(v) for k, v in I.deterministic_state(shapes, 1).items()})
    return model.to(dev(), torch.bfloat16)


class _Bucket:
    """Minimal stand-in for the reference's frozen ``Bucket`` (hashable, exact Q)."""
    def __init__(self, query_lengths):
        self.query_lengths = tuple(query_lengths)

    def __hash__(self):
        return hash(self.query_lengths)

    def __eq__(self, other):
        return isinstance(other, _Bucket) and other.query_lengths == self.query_lengths


def test_graph_replay_equals_eager_verify(pkg):
    model = tiny_bf16_model()
    prompts = [torch.from_numpy(ids)[None].to(dev()) for ids in I.greedy_prompts()[:3]]
    eager = pkg.B200Qwen3Target(model, (1, 2), slots=3, context_capacity=2400, max_query_tokens=2500)
    for i in range(3):
        eager.add_request(f'r{i}')
    eager.prefill({f'r{i}': p for i, p in enumerate(prompts)})
    bucket = _Bucket((8, 8, 8))
    eager.capture(bucket)
    g = np.random.Generator(np.random.PCG64(77))
    for rnd in range(4):
        chunks = {f'r{i}': torch.from_numpy(g.integers(0, 1000, (1, 8))).to(dev()) for i in range(3)}
        ref = eager.verify(chunks)
        ref_logits = {r: v.clone() for r, v in eager.predict(ref).items()}
        ref_ctx = ref.context.clone()
        eager.abort(ref)
        got = eager.verify_graph(chunks, bucket)
        logits = eager.predict(got)
        for r in chunks:
            assert torch.equal(logits[r], ref_logits[r]), (rnd, r)
        assert torch.equal(got.context, ref_ctx)
        counts = {f'r{i}': int(x) for i, x in enumerate(g.integers(1, 9, 3))}
        before = eager.lengths
        eager.commit(got, counts)
        assert eager.lengths == {r: before[r] + counts[r] for r in before}
    status_clean(pkg)


def test_graph_commit_matches_eager_commit(pkg):
    """Two targets on the same weights: one verifies eagerly, one through the graph;
    after the same commits their resident KV and lengths are identical."""
    model = tiny_bf16_model()
    prompts = {f'r{i}': torch.from_numpy(ids)[None].to(dev()) for i, ids in enumerate(I.greedy_prompts()[3:6])}
    a = pkg.B200Qwen3Target(model, (1, 2), slots=3, context_capacity=600, max_query_tokens=600)
    for r in prompts:
        a.add_request(r)
    a.prefill(prompts)
    b_model = tiny_bf16_model()
    b = pkg.B200Qwen3Target(b_model, (1, 2), slots=3, context_capacity=600, max_query_tokens=600)
    for r in prompts:
        b.add_request(r)
    b.prefill(prompts)
    bucket = _Bucket((7, 7, 7))
    b.capture(bucket)
    g = np.random.Generator(np.random.PCG64(5))
    for rnd in range(3):
        chunks = {r: torch.from_numpy(g.integers(0, 1000, (1, 7))).to(dev()) for r in prompts}
        counts = {r: int(x) for r, x in zip(prompts, g.integers(0, 8, 3))}
        fa = a.verify(chunks)
        la = {r: v.clone() for r, v in a.predict(fa).items()}
        a.commit(fa, counts)
        fb = b.verify_graph(chunks, bucket)
        lb = b.predict(fb)
        for r in chunks:
            assert torch.equal(la[r], lb[r]), (rnd, r)
        b.commit(fb, counts)
    assert a.lengths == b.lengths
    for r in prompts:
        ka, va = a.pool.request_kv(a._handles[r])
        kb, vb = b.pool.request_kv(b._handles[r])
        assert torch.equal(ka, kb) and torch.equal(va, vb)
    status_clean(pkg)


def test_graph_refusals(pkg):
    model = tiny_bf16_model()
    t = pkg.B200Qwen3Target(model, (1, 2), slots=2, context_capacity=300, max_query_tokens=64)
    t.add_request('a')
    t.add_request('b')
    bucket = _Bucket((4, 4))
    with pytest.raises(ValueError):
        t.verify_graph({'a': torch.zeros(1, 4, dtype=torch.long, device=dev())}, bucket)   # not captured
    t.capture(bucket)
    with pytest.raises(ValueError):
        t.capture(bucket)
    with pytest.raises(ValueError):
        t.verify_graph({'a': torch.zeros(1, 4, dtype=torch.long, device=dev()),
                        'b': torch.zeros(1, 5, dtype=torch.long, device=dev())}, bucket)
    f = t.verify_graph({'a': torch.zeros(1, 4, dtype=torch.long, device=dev()),
                        'b': torch.ones(1, 4, dtype=torch.long, device=dev())}, bucket)
    t.abort(f)
    assert t.lengths == {'a': 0, 'b': 0}
    status_clean(pkg)


def test_speculative_loop_with_graph_replay_gives_the_same_tokens(pkg):
    """speculative_greedy(graph=True) (target verify, draft proposal and draft append
    replayed) and speculative_greedy_pipelined (the round state kept on the GPU, the
    host one round behind) emit the tokens of the eager loop on the same bf16 model and
    prompts."""
    model = tiny_bf16_model()
    spec = pkg.DraftSpec(**dict(I.TINY_DRAFT, markov_rank=64))
    outs = []
    for graph in (False, True, 'pipelined'):
        draft = pkg.DSparkDraftModel(model, spec).eval()
        dshapes = {k: tuple(v.shape) for k, v in draft.state_dict().items()
                   if not k.startswith(('embedding.', 'lm_head.'))}
        draft.load_state_dict({k: torch.from_numpy(v) for k, v in I.deterministic_state(dshapes, 2).items()},
                              strict=False)
        draft = draft.to(dev(), torch.bfloat16)
        target = pkg.B200Qwen3Target(model, spec.layer_ids, slots=4, context_capacity=400, max_query_tokens=700)
        pdraft = pkg.B200PackedDraft(draft, max_requests=4, context_capacity=400)
        prompts = {f'r{i}': torch.from_numpy(ids)[None].to(dev()) for i, ids in enumerate(I.greedy_prompts()[3:6])}
        if graph == 'pipelined':
            out, rounds = pkg.speculative_greedy_pipelined(target, pdraft, prompts, 24, eos_ids=(7,))
            # the host mirrors of the committed lengths follow the device state
            assert all(target.lengths[r] == prompts[r].shape[1] + len(out[r]) - 1 for r in prompts)
            assert all(pdraft.lengths[r] == target.lengths[r] for r in prompts)
        else:
            out, rounds = pkg.speculative_greedy(target, pdraft, prompts, 24, eos_ids=(7,), graph=graph)
        outs.append(out)
        target.close()
    assert outs[0] == outs[1] == outs[2]
    status_clean(pkg)


def test_stochastic_loop_with_graph_replay_gives_the_same_tokens(pkg):
    """speculative_sample(graph=True) (stochastic proposal, target verify and draft
    append replayed from CUDA graphs) emits the tokens, round statistics and generator
    states of the eager loop on the same bf16 model, prompts and seeds; requests whose
    budgets end mid-block exercise proposals with limits below the block size."""
    model = tiny_bf16_model()
    spec = pkg.DraftSpec(**dict(I.TINY_DRAFT, markov_rank=64))
    results = []
    for graph in (False, True):
        draft = pkg.DSparkDraftModel(model, spec).eval()
        dshapes = {k: tuple(v.shape) for k, v in draft.state_dict().items()
                   if not k.startswith(('embedding.', 'lm_head.'))}
        draft.load_state_dict({k: torch.from_numpy(v) for k, v in I.deterministic_state(dshapes, 2).items()},
                              strict=False)
        draft = draft.to(dev(), torch.bfloat16)
        target = pkg.B200Qwen3Target(model, spec.layer_ids, slots=4, context_capacity=400, max_query_tokens=700)
        pdraft = pkg.B200PackedDraft(draft, max_requests=4, context_capacity=400)
        prompts = {f'r{i}': torch.from_numpy(ids)[None].to(dev()) for i, ids in enumerate(I.greedy_prompts()[3:6])}
        gens = {}
        for i, r in enumerate(prompts):
            gens[r] = torch.Generator()
            gens[r].manual_seed(1000 + i)
        out, rounds = pkg.speculative_sample(target, pdraft, prompts, 23, gens, temperature=0.9, eos_ids=(7,),
                                             graph=graph)
        results.append((out, rounds, {r: g.get_state() for r, g in gens.items()}))
        if graph:
            assert pdraft.__dict__.get('_sgraphs'), 'the proposal ran from a captured graph'
        target.close()
    (o0, r0, g0), (o1, r1, g1) = results
    assert o0 == o1 and r0 == r1
    assert all(torch.equal(g0[r], g1[r]) for r in g0)
    status_clean(pkg)
