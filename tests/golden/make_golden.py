"""Generate golden fixtures by running the reference implementation's own functions.

Usage:  python tests/golden/make_golden.py --reference <qwen3-dspark checkout>

The reference (``dspark_qwen``) is imported from the given checkout; its CPU
oracles produce the outputs stored in ``tests/golden/*.npz``. Inputs come from
``tests/golden/inputs.py`` (numpy PCG64), so only outputs and an input digest are
stored. The GPU box never runs this script; the tests only read the fixtures.
"""
import argparse
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, HERE)

import inputs as I  # noqa: E402


def t(x):
    import torch
    return torch.from_numpy(np.ascontiguousarray(x))


def layout_for(qlens, klens):
    """Reference PackedLayout built from markers/positions (request-contiguous keys)."""
    import torch
    from dspark_qwen.varlen_target import PackedLayout
    qr, qp, kr, kp = [], [], [], []
    for m, (nq, nk) in enumerate(zip(qlens, klens)):
        qr += [m] * nq
        qp += list(range(nk - nq, nk))
        kr += [m] * nk
        kp += list(range(nk))
    L = lambda x: torch.tensor(x, dtype=torch.long)  # noqa: E731
    return PackedLayout.from_metadata(L(qr), L(qp), L(kr), L(kp))


def draft_fixtures(out):
    from dspark_qwen.packed_draft import test_only_noncausal_varlen
    for name, seed, contexts, bf16 in (('draft_cfg1', 0, I.CFG1_CONTEXTS, False),
                                       ('draft_bf16_small', 11, I.DRAFT_BF16_CONTEXTS, True)):
        q, k, v, qlens, klens = I.draft_case(seed, contexts, bf16)
        layout = layout_for(qlens, klens)
        o = test_only_noncausal_varlen(t(q), t(k), t(v), layout, scale=I.SCALE).numpy()
        out[name] = dict(output=o.astype(np.float32), digest=I.digest(q, k, v), seed=seed,
                         contexts=np.array(contexts), cu_query=layout.cu_query.numpy(),
                         cu_key=layout.cu_key.numpy())


def varlen_fixtures(out):
    from dspark_qwen.varlen_target import test_only_dense_varlen
    from dspark_qwen.persistent_qwen_target import PersistentAttentionLayout, test_only_persistent_sdpa
    import torch
    for idx, (qlens, klens) in enumerate(I.PROBE_CASES):
        q, k, v = I.varlen_case(I.PROBE_SEED + idx, qlens, klens, True)
        layout = layout_for(qlens, klens)
        o = test_only_dense_varlen(t(q), t(k), t(v), layout, scale=I.SCALE).numpy()
        out[f'verify_probe{idx}'] = dict(output=o, digest=I.digest(q, k, v), qlens=np.array(qlens), klens=np.array(klens))
    # Zero-Q ramp sentinel (reports/native-varlen-diagnostic-20261009: 0.25 and (21..28)/64).
    qlens, klens = I.PROBE_CASES[0]
    q = np.zeros((sum(qlens), I.HQ, I.D), np.float32)
    ramp = np.concatenate([np.arange(n, dtype=np.float32) / 32 for n in klens])
    v = np.broadcast_to(ramp[:, None, None], (sum(klens), I.HKV, I.D)).copy()
    k = np.zeros_like(v)
    o = test_only_dense_varlen(t(q), t(k), t(v), layout_for(qlens, klens), scale=I.SCALE).numpy()
    out['zero_q_ramp'] = dict(output=o)
    # Capacity-tail path: K/V carry NaN rows past cu_key[-1].
    qlens, klens, tail = I.CAPACITY_QLENS, I.CAPACITY_KLENS, I.CAPACITY_TAIL
    q, k, v = I.varlen_case(77, qlens, klens, True, tail=tail)
    k[sum(klens):] = np.nan
    v[sum(klens):] = np.nan
    cq = torch.tensor(np.cumsum((0,) + qlens), dtype=torch.int32)
    ck = torch.tensor(np.cumsum((0,) + klens), dtype=torch.int32)
    lay = PersistentAttentionLayout(qlens, klens, cq, ck, sum(klens) + tail, max(klens), max(qlens))
    o = test_only_persistent_sdpa(t(q), t(k), t(v), lay, scale=I.SCALE).numpy()
    out['verify_capacity'] = dict(output=o, digest=I.digest(q[:, :, :], np.nan_to_num(k), np.nan_to_num(v)))


def training_fixtures(out):
    import torch
    import torch.nn.functional as F
    from dspark_qwen.model import block_mask
    m = block_mask(torch.tensor([2, 4]), 3, 7)[0, 0]
    out['block_mask_truth'] = dict(mask=m.numpy())
    g = I.rng(3)
    ctxs = [c for c, _ in I.TRAIN_SEQS]
    anchors = [a for _, a in I.TRAIN_SEQS]
    nq = sum(len(a) * I.BLOCK for a in anchors)
    nk = sum(c + len(a) * I.BLOCK for c, a in I.TRAIN_SEQS)
    q = I.normal(g, (nq, I.HQ, I.D), True)
    k = I.normal(g, (nk, I.HKV, I.D), True)
    v = I.normal(g, (nk, I.HKV, I.D), True)
    rows, qo, ko = [], 0, 0
    for ctx, anc in I.TRAIN_SEQS:
        a = len(anc) * I.BLOCK
        mask = block_mask(torch.tensor(anc), I.BLOCK, ctx)
        qs = t(q[qo:qo + a]).transpose(0, 1)[None]
        ks = t(k[ko:ko + ctx + a]).transpose(0, 1)[None].repeat_interleave(2, dim=1)
        vs = t(v[ko:ko + ctx + a]).transpose(0, 1)[None].repeat_interleave(2, dim=1)
        rows.append(F.scaled_dot_product_attention(qs, ks, vs, attn_mask=mask, dropout_p=0.0,
                                                   is_causal=False)[0].transpose(0, 1).numpy())
        qo += a
        ko += ctx + a
    out['train_layout'] = dict(output=np.concatenate(rows), digest=I.digest(q, k, v))


def layout_fixtures(out):
    import torch
    from dspark_qwen.varlen_target import PackedLayout
    L = lambda x: torch.tensor(x, dtype=torch.long)  # noqa: E731
    g = I.rng(5)
    cases = [([2, 2, 1], [2, 3, 2], [1, 1, 2, 2, 3, 3, 1, 2, 2], [0, 1, 0, 1, 0, 1, 2, 2, 3])]
    # A random interleaved physical cache with an inactive request.
    lens = {7: 13, 3: 40, 9: 5, 4: 22}
    pairs = [(m, p) for p in range(64) for m, n in lens.items() if p < n]
    perm = g.permutation(len(pairs))
    # Keep each request's own keys in position order while interleaving requests.
    order = sorted(range(len(pairs)), key=lambda i: (perm[i] % 7, pairs[i][1]))
    seen = {m: 0 for m in lens}
    kr, kp = [], []
    for i in order:
        m = pairs[i][0]
        kr.append(m)
        kp.append(seen[m])
        seen[m] += 1
    qspec = [(3, 7), (9, 2), (7, 5)]   # (marker, query count); marker 4 is inactive
    qr = [m for m, c in qspec for _ in range(c)]
    qp = [p for m, c in qspec for p in range(lens[m] - c, lens[m])]
    cases.append((qr, qp, kr, kp))
    for idx, (qr, qp, kr, kp) in enumerate(cases):
        lay = PackedLayout.from_metadata(L(qr), L(qp), L(kr), L(kp))
        out[f'layout{idx}'] = dict(qr=np.array(qr), qp=np.array(qp), kr=np.array(kr), kp=np.array(kp),
                                   markers=np.array(lay.request_markers), query_lengths=np.array(lay.query_lengths),
                                   key_lengths=np.array(lay.key_lengths), cu_query=lay.cu_query.numpy(),
                                   cu_key=lay.cu_key.numpy(), gather=lay.gather_indices.numpy(),
                                   pair_domain=np.array(lay.pair_domain))


def rope_fixtures(out):
    import torch
    from transformers import Qwen3Config
    from transformers.models.qwen3.modeling_qwen3 import (Qwen3RMSNorm, Qwen3RotaryEmbedding,
                                                          apply_rotary_pos_emb)
    from oracle.bf16 import f32_to_bf16_bits
    cfg = Qwen3Config(hidden_size=1024, num_attention_heads=16, num_key_value_heads=8, head_dim=128,
                      rms_norm_eps=I.RMS_EPS, max_position_embeddings=40960,
                      rope_parameters={'rope_type': 'default', 'rope_theta': I.ROPE_THETA})
    g = I.rng(9)
    n = I.BLOCK * len(I.ROPE_CONTEXTS)
    q = I.normal(g, (n, I.HQ, I.D), True) * 3
    k = I.normal(g, (n, I.HKV, I.D), True) * 3
    qw = 1 + 0.1 * I.normal(g, (I.D,), True)
    kw = 1 + 0.1 * I.normal(g, (I.D,), True)
    qb = [f32_to_bf16_bits(x) for x in (q, k, qw, kw)]
    bf = lambda bits: torch.from_numpy(bits.astype(np.int16)).view(torch.bfloat16)  # noqa: E731
    qn, kn = Qwen3RMSNorm(I.D, I.RMS_EPS), Qwen3RMSNorm(I.D, I.RMS_EPS)
    qn.weight.data = bf(qb[2]).clone()
    kn.weight.data = bf(qb[3]).clone()
    positions = np.concatenate([np.arange(c, c + I.BLOCK) for c in I.ROPE_CONTEXTS])
    rot = Qwen3RotaryEmbedding(cfg)
    with torch.no_grad():
        qs = qn(bf(qb[0])).transpose(0, 1)[None]       # [1, Hq, n, D] as HF transposes
        ks = kn(bf(qb[1])).transpose(0, 1)[None]
        cos, sin = rot(qs, torch.from_numpy(positions)[None])
        qr, kr = apply_rotary_pos_emb(qs, ks, cos, sin)
    to_bits = lambda x: x.contiguous().view(torch.int16).numpy().astype(np.uint16)  # noqa: E731
    out['qk_norm_rope'] = dict(q_raw=qb[0], k_raw=qb[1], q_weight=qb[2], k_weight=qb[3],
                               positions=positions, inv_freq=rot.inv_freq.numpy(),
                               cos=to_bits(cos[0]), sin=to_bits(sin[0]),
                               q_norm=to_bits(qn(bf(qb[0]))), k_norm=to_bits(kn(bf(qb[1]))),
                               q_out=to_bits(qr[0].transpose(0, 1)), k_out=to_bits(kr[0].transpose(0, 1)))


def kv_store_fixtures(out):
    import torch
    from dspark_qwen.persistent_target_kv import Bucket, PersistentTargetKV
    # The reference's own growing-context scenario (tests/test_persistent_target_kv.py:37-64).
    pool = PersistentTargetKV(layers=2, slots=3, context_capacity=24, max_query_tokens=8, heads=2, dim=4)
    a, b, idle = (pool.add_request(r) for r in ('A', 'B', 'idle'))
    for h, n, off in ((a, 3, 100), (b, 5, 500), (idle, 9, 900)):
        x = torch.arange(pool.layers * n * 2 * 4, dtype=torch.float32).reshape(2, n, 2, 4) + off
        pool.load_prefix(h, x, x + 0.25)
    bucket = Bucket((2, 3), (12, 12), 'golden fixture')
    pool.register_bucket(bucket)
    tx = pool.begin([a, b], bucket)
    sk = torch.arange(2 * 5 * 2 * 4, dtype=torch.float32).reshape(2, 5, 2, 4) + 10000
    for layer in range(2):
        pool.stage_layer(tx, layer, sk[layer], sk[layer] + 0.5)
    ws = pool._workspaces[bucket]
    k0, v0, cq, ck, pos = pool.prepare_attention(tx, 0)
    # Workspace tensors are reused by the next begin(): copy every view now.
    rec = dict(committed_indices=ws.committed_indices.numpy().copy(), scratch_indices=ws.scratch_indices.numpy().copy(),
               from_scratch=ws.from_scratch.numpy().reshape(-1).copy(), valid=ws.valid.numpy().reshape(-1).copy(),
               cu_query=cq.numpy().copy(), cu_key=ck.numpy().copy(), positions=pos.numpy().copy(),
               prepared_k0=k0.numpy().copy(), prepared_v0=v0.numpy().copy(), key_capacity=np.array(bucket.key_capacity))
    pool.commit(tx, {a: 1, b: 2})
    rec.update(resident_keys=pool.keys.numpy().copy(), resident_values=pool.values.numpy().copy(),
               lengths=np.array([pool.length(h) for h in (a, b, idle)]))
    tx2 = pool.begin([a, b], bucket)
    ws = pool._workspaces[bucket]
    rec.update(cu_key2=ws.cu_key.numpy().copy(), positions2=ws.positions.numpy().copy())
    pool.abort(tx2)
    out['kv_store'] = rec


def greedy_fixtures(out):
    """Config-5 style parity: the reference's target greedy tokens and its own greedy
    speculative decode (cached_speculative_greedy) on a tiny fp32 model, plus the first
    draft proposal of request 0."""
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from dspark_qwen.cached_decode import DraftContextCache, cached_speculative_greedy
    from dspark_qwen.cached_target import CachedTarget
    from dspark_qwen.config import DraftConfig
    from dspark_qwen.model import DSparkDraft
    cfg = Qwen3Config(**I.TINY_TARGET)
    cfg._attn_implementation = 'sdpa'
    model = Qwen3ForCausalLM(cfg).eval()
    tshapes = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    model.load_state_dict({k: torch.from_numpy(v) for k, v in I.deterministic_state(tshapes, 1).items()})
    spec = DraftConfig(**I.TINY_DRAFT)
    draft = DSparkDraft(model, spec).eval()
    dshapes = {k: tuple(v.shape) for k, v in draft.state_dict().items()
               if not k.startswith(('embedding.', 'lm_head.'))}
    missing = draft.load_state_dict({k: torch.from_numpy(v) for k, v in I.deterministic_state(dshapes, 2).items()},
                                    strict=False)
    assert set(missing.missing_keys) <= {'embedding.weight', 'lm_head.weight'} and not missing.unexpected_keys
    target = CachedTarget(model, spec.layer_ids)
    tokens, spec_tokens, accepted = [], [], []
    with torch.no_grad():
        for ids in I.greedy_prompts():
            x = torch.from_numpy(ids)[None]
            greedy = target.greedy(x, I.GREEDY_NEW_TOKENS)
            sp, rounds = cached_speculative_greedy(target, draft, x, I.GREEDY_NEW_TOKENS)
            assert sp == greedy, 'reference speculative greedy must equal target greedy'
            tokens.append(greedy)
            spec_tokens.append(sp)
            accepted.append(sum(r['accepted'] for r in rounds))
        ids = torch.from_numpy(I.greedy_prompts()[0])[None]
        feats = target.prefill(ids)
        first = int(target.predict(feats, last_only=True).argmax(-1).item())
        cache = DraftContextCache(draft)
        cache.append(feats.context)
        anchor = torch.tensor([[first]])
        hidden = draft.backbone_cached(anchor, cache.layers, cache.length)
        proposals, _ = draft.propose_greedy_cached(anchor, cache.layers, cache.length)
    out['greedy_round'] = dict(tokens=np.array(tokens), accepted=np.array(accepted),
                               target_names=np.array(sorted(tshapes)), draft_names=np.array(sorted(dshapes)),
                               first_token=np.array(first), first_hidden=hidden.numpy(),
                               first_proposals=np.array(proposals))


def stochastic_fixtures(out):
    """Reference tensor_sampling.verify_proposal on the seeded cases of
    inputs.stochastic_case, its target laws from logits_to_probabilities, and a
    scripted generator that hands out the case's uniforms in order."""
    import torch
    from dspark_qwen.tensor_sampling import TensorProposal, logits_to_probabilities, verify_proposal

    class Scripted:
        def __init__(self, values):
            self.values, self.used = list(values), 0

        def uniform(self, reference):
            v = torch.tensor(self.values[self.used], dtype=torch.float64, device=reference.device)
            self.used += 1
            return v

    rec = {}
    for idx in range(I.STOCH_CASES):
        c = I.stochastic_case(idx)
        p = logits_to_probabilities(t(c['target_logits']), c['temperature'])
        n = c['tokens'].size
        proposal = TensorProposal(t(c['tokens']), t(c['q']), torch.zeros(n, dtype=torch.float32))
        rng = Scripted(c['uniforms'])
        r = verify_proposal(proposal, p, rng, max_new_tokens=c['budget'], eos_ids=c['eos'])
        extra = {None: 0, 'residual': 1, 'bonus': 2}[r.extra_token_kind]
        reason = {'round_complete': 0, 'eos': 1, 'budget': 2}[r.stop_reason]
        pn = p.numpy()
        probe = np.concatenate([np.arange(min(8, c['vocab'])), c['tokens']])
        rec[f'case{idx}_tokens'] = r.tokens.numpy()
        rec[f'case{idx}_decision'] = np.array([r.accepted_draft_tokens,
                                               -1 if r.rejected_index is None else r.rejected_index,
                                               extra, reason, rng.used])
        rec[f'case{idx}_p_probe'] = pn[:, probe]
        rec[f'case{idx}_p_rowsum'] = pn.sum(axis=1)
    out['stochastic_accept'] = rec


def stochastic_round_fixtures(out):
    """The reference's stochastic speculative decode (cached_speculative_sample) on the
    tiny fp32 model of the greedy case, one seeded CPU generator per prompt."""
    import torch
    from transformers import Qwen3Config, Qwen3ForCausalLM
    from dspark_qwen.cached_sampling import cached_speculative_sample
    from dspark_qwen.cached_target import CachedTarget
    from dspark_qwen.config import DraftConfig
    from dspark_qwen.model import DSparkDraft
    from dspark_qwen.tensor_sampling import TensorRandom
    cfg = Qwen3Config(**I.TINY_TARGET)
    cfg._attn_implementation = 'sdpa'
    model = Qwen3ForCausalLM(cfg).eval()
    tshapes = {k: tuple(v.shape) for k, v in model.state_dict().items()}
    model.load_state_dict({k: torch.from_numpy(v) for k, v in I.deterministic_state(tshapes, 1).items()})
    spec = DraftConfig(**I.TINY_DRAFT)
    draft = DSparkDraft(model, spec).eval()
    dshapes = {k: tuple(v.shape) for k, v in draft.state_dict().items()
               if not k.startswith(('embedding.', 'lm_head.'))}
    draft.load_state_dict({k: torch.from_numpy(v) for k, v in I.deterministic_state(dshapes, 2).items()}, strict=False)
    target = CachedTarget(model, spec.layer_ids)
    tokens, accepted, residual, bonus = [], [], [], []
    with torch.no_grad():
        for i, ids in enumerate(I.greedy_prompts()):
            rng = TensorRandom(torch.Generator().manual_seed(I.STOCH_ROUND_SEED + i))
            x = torch.from_numpy(ids)[None]
            o, rounds = cached_speculative_sample(target, draft, x, I.GREEDY_NEW_TOKENS,
                                                  temperature=I.STOCH_ROUND_TEMPERATURE, rng=rng)
            tokens.append(o + [-1] * (I.GREEDY_NEW_TOKENS - len(o)))
            accepted.append(sum(r['accepted'] for r in rounds))
            residual.append(sum(r['extra_token_kind'] == 'residual' for r in rounds))
            bonus.append(sum(r['extra_token_kind'] == 'bonus' for r in rounds))
    out['stochastic_round'] = dict(tokens=np.array(tokens), accepted=np.array(accepted),
                                   residual_rounds=np.array(residual), bonus_rounds=np.array(bonus))


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument('--reference', required=True, help='path of a qwen3-dspark checkout')
    ap.add_argument('--only', nargs='*', default=None, help='fixture functions to run (default: all)')
    args = ap.parse_args()
    os.environ.setdefault('PYTHONDONTWRITEBYTECODE', '1')
    sys.dont_write_bytecode = True
    sys.path.insert(0, os.path.abspath(args.reference))
    import torch
    torch.manual_seed(0)
    torch.set_num_threads(4)
    out = {}
    for fn in (draft_fixtures, varlen_fixtures, training_fixtures, layout_fixtures, rope_fixtures,
               kv_store_fixtures, greedy_fixtures, stochastic_fixtures,
               stochastic_round_fixtures):
        if args.only is None or fn.__name__ in args.only:
            fn(out)
    for name, rec in out.items():
        np.savez_compressed(os.path.join(HERE, f'{name}.npz'), **{k: np.asarray(v) for k, v in rec.items()})
        print(name, {k: np.asarray(v).shape for k, v in rec.items()})


if __name__ == '__main__':
    main()
