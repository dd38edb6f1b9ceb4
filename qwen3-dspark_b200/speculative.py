"""Batched greedy speculative decoding on the B200 target and draft.

Per request this is ``cached_speculative_greedy`` (dspark_qwen/cached_decode.py:45-122):
prefill the prompt, emit the target's argmax, then repeat: the draft proposes one
block from the latest token, the target verifies [anchor] + proposals in one pass,
the longest prefix of proposals matching the target's argmax is accepted plus the
target's correction (or the bonus token after a full accept), the target commits
the verified rows up to (excluding) the newest output token and rolls back the rest,
and the draft projects the committed features. Here all active requests share one
draft backbone call and one target verify forward per round.
Greedy acceptance makes the output equal to the target's own greedy decode.
"""
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class QueryBucket:
    """Exact ordered query lengths of a verify round: the key of a captured graph."""
    query_lengths: tuple


def accept_greedy(proposals, predictions, eos_ids=()):
    """Accept rule of cached_decode.py:84-98: returns (accepted, committed tokens)."""
    accepted, committed = 0, []
    for proposed, correct in zip(proposals, predictions):
        if proposed != correct:
            committed.append(correct)
            break
        committed.append(proposed)
        accepted += 1
        if proposed in eos_ids:
            break
    else:
        committed.append(predictions[-1])
    eos = next((i for i, t in enumerate(committed) if t in eos_ids), None)
    if eos is not None:
        committed = committed[:eos + 1]
    return accepted, committed


def _pinned(values, dtype, device):
    """Host list -> device tensor through pinned memory, without a host wait."""
    return torch.tensor(values, dtype=dtype).pin_memory().to(device, non_blocking=True)


def _accept_on_device(target, verified, ids, active, width, output, max_new_tokens, eos_ids):
    """One round's acceptance with the on-device argmax + accept kernels: the host
    reads back one small int64 vector (counts and committed tokens) per round.
    ``ids`` [R, width] are the verified chunks (anchor, proposals) in ``active`` order."""
    from .kernels import greedy_accept
    logits = target.model.get_output_embeddings()(verified.last)[0]
    tokens = ids.reshape(-1)
    cu = [width * i for i in range(len(active) + 1)]
    dev = logits.device
    cu_q = _pinned(cu, torch.int32, dev)
    budget = _pinned([max_new_tokens - len(output[r]) for r in active], torch.int32, dev)
    _pred, accepted, n_commit, emitted = greedy_accept(logits, tokens, cu_q, eos_ids, budget)
    host = torch.cat((accepted.long(), n_commit.long(), emitted)).cpu().tolist()
    n = len(active)
    result = {}
    for i, r in enumerate(active):
        k = host[n + i]
        result[r] = (host[i], host[2 * n + cu[i]:2 * n + cu[i] + k])
    return result


@torch.no_grad()
def speculative_greedy(target, draft, prompts, max_new_tokens, eos_ids=(), device_accept=True, graph=False):
    """prompts: {request: ids [1, P]} on the target device. Returns ({request: tokens}, rounds).

    ``device_accept`` runs the argmax and the accept rule on the GPU (one small
    read-back per round); otherwise each request's logits are read back and the rule
    runs on the host. Both give the same tokens. ``graph`` replays the target's verify
    forward from a CUDA graph captured once per set of chunk lengths (``QueryBucket``)
    and, for bf16 drafts with the fused Markov head, the draft proposal from a graph
    captured once per request count, instead of running them eagerly; the tokens are
    the same."""
    if type(max_new_tokens) is not int or max_new_tokens < 0:
        raise ValueError('max_new_tokens must be a nonnegative integer')
    eos_ids = set(eos_ids)
    for r in prompts:
        target.add_request(r)
        draft.add_request(r)
    if max_new_tokens == 0:
        return {r: [] for r in prompts}, []
    features = target.prefill(prompts)
    last = target.predict(features, last_only=True)
    output = {r: [int(last[r].argmax(-1).item())] for r in prompts}
    draft.append_committed({r: features.context_for(r) for r in prompts})
    active = [r for r in prompts if output[r][-1] not in eos_ids and max_new_tokens > 1]
    rounds = []
    width = draft.draft.spec.block_size + 1
    while active:
        # one upload of the anchors; the chunks are rows of one device tensor
        anchor_ids = _pinned([output[r][-1] for r in active], torch.long, target.device)
        anchors = {r: anchor_ids[i].view(1, 1) for i, r in enumerate(active)}
        if graph and getattr(draft, '_graph_ready', lambda: False)():
            if len(anchors) not in draft.__dict__.get('_graphs', {}):
                draft.capture_propose(len(anchors))
            proposed, _conf = draft.propose_greedy_graph(anchors, on_device=True)
            ids = torch.cat((anchor_ids[:, None], proposed), dim=1)        # no host read of the proposals
        else:
            proposed = draft.propose_greedy(anchors)
            ids = _pinned([[output[r][-1]] + proposed[r][0] for r in active], torch.long, target.device)
        chunks = {r: ids[i:i + 1] for i, r in enumerate(active)}
        if graph:
            bucket = QueryBucket((width,) * len(active))
            if bucket not in target._graphs:
                target.capture(bucket)
            verified = target.verify_graph(chunks, bucket)
        else:
            verified = target.verify(chunks)
        if device_accept:
            decided = _accept_on_device(target, verified, ids, active, width, output, max_new_tokens, eos_ids)
        else:
            logits = target.predict(verified)
            host_ids = ids.tolist()
            decided = {}
            for i, (r, v) in enumerate(logits.items()):
                accepted, committed = accept_greedy(host_ids[i][1:], v[0].argmax(-1).tolist(), eos_ids)
                decided[r] = (accepted, committed[:max_new_tokens - len(output[r])])
        commit, stats = {}, {}
        for r in active:
            accepted, committed = decided[r]
            output[r].extend(committed)
            commit[r] = len(committed)          # old anchor .. newest-1 are now committed KV
            stats[r] = dict(accepted=accepted, committed=len(committed))
        target.commit(verified, commit)
        counts = [commit[r] for r in active]
        if graph and hasattr(draft, 'capture_append'):
            # whole verified chunks through the captured fixed-shape append
            if (len(active), width) not in draft.__dict__.get('_append_graphs', {}):
                draft.capture_append(len(active), width)
            draft.append_verified_graph(verified.context, tuple(active), counts)
        else:
            draft.append_committed({r: verified.context_for(r)[:, :commit[r]] for r in active if commit[r]})
        rounds.append(stats)
        active = [r for r in active if len(output[r]) < max_new_tokens and output[r][-1] not in eos_ids]
    return output, rounds


@torch.no_grad()
def speculative_sample(target, draft, prompts, max_new_tokens, generators, temperature=1.0, eos_ids=()):
    """Batched stochastic speculative decoding; per request the rule of
    ``cached_speculative_sample`` (dspark_qwen/cached_sampling.py:80-175) under the
    reference's float64 law. ``generators``: {request: CPU torch.Generator}. Each
    request's uniforms come from its generator in the reference's draw order (the
    first token, then per round the proposal draws and the acceptance draws), and
    after each round the generator is left exactly where the reference's would be,
    so a request's tokens equal the reference's single-request run with the same
    seed. Acceptance runs on the GPU (``stochastic_accept``); the host reads back one
    small result per round. Returns ({request: tokens}, rounds)."""
    from .kernels import STOCHASTIC_STATUS, float64_law, sample_rows, stochastic_accept
    import math
    if type(max_new_tokens) is not int or max_new_tokens < 0:
        raise ValueError('max_new_tokens must be a nonnegative integer')
    temperature = float(temperature)
    if not math.isfinite(temperature) or temperature <= 0:
        raise ValueError('temperature must be finite and strictly positive')
    if set(generators) != set(prompts):
        raise ValueError('One generator per request required')
    eos_ids = set(int(e) for e in eos_ids)
    dev = target.device
    f64 = torch.float64
    for r in prompts:
        target.add_request(r)
        draft.add_request(r)
    if max_new_tokens == 0:
        return {r: [] for r in prompts}, []
    features = target.prefill(prompts)
    last = target.predict(features, last_only=True)
    requests = list(prompts)
    first_u = torch.stack([torch.rand((), dtype=f64, generator=generators[r]) for r in requests]).to(dev)
    law = float64_law(torch.cat([last[r].reshape(1, -1) for r in requests]), temperature)
    first = sample_rows(law, first_u).tolist()
    output = {r: [first[i]] for i, r in enumerate(requests)}
    draft.append_committed({r: features.context_for(r) for r in prompts})
    active = [r for r in requests if output[r][-1] not in eos_ids and max_new_tokens > 1]
    size = draft.draft.spec.block_size
    rounds = []
    while active:
        remaining = {r: max_new_tokens - len(output[r]) for r in active}
        n = {r: min(size, remaining[r]) for r in active}
        states = {r: generators[r].get_state() for r in active}
        drawn = {r: torch.rand(2 * n[r] + 1, dtype=f64, generator=generators[r]) for r in active}
        u_prop = torch.zeros((len(active), size), dtype=f64)
        u_acc = torch.zeros((len(active), size + 1), dtype=f64)
        for i, r in enumerate(active):
            u_prop[i, :n[r]] = drawn[r][:n[r]]
            u_acc[i, :n[r] + 1] = drawn[r][n[r]:]
        u_prop = u_prop.pin_memory().to(dev, non_blocking=True)
        u_acc = u_acc.pin_memory().to(dev, non_blocking=True)
        anchors = {r: torch.tensor([[output[r][-1]]], dtype=torch.long, device=dev) for r in active}
        tokens, laws = draft.propose_stochastic(anchors, n, u_prop, temperature)
        chunks = {r: torch.cat((anchors[r][0], tokens[r]))[None] for r in active}
        verified = target.verify(chunks)
        logits = target.model.get_output_embeddings()(verified.last)[0]
        cu = [0]
        for r in active:
            cu.append(cu[-1] + n[r])
        emitted, result = stochastic_accept(
            logits, torch.cat([tokens[r] for r in active]), torch.cat([laws[r] for r in active]),
            torch.tensor(cu, dtype=torch.int32).pin_memory().to(dev, non_blocking=True), temperature, u_acc,
            torch.tensor([remaining[r] for r in active], dtype=torch.int32).pin_memory().to(dev, non_blocking=True),
            eos_ids)
        res = result.cpu().tolist()
        em = emitted.cpu().tolist()
        bad = [(r, res[i][6]) for i, r in enumerate(active) if res[i][6]]
        if bad:
            # nothing of this round is kept: the caches roll back and the generators
            # return to where the round started
            target.abort(verified)
            for r in active:
                generators[r].set_state(states[r])
            r, status = bad[0]
            raise ValueError(f'stochastic acceptance refused request {r}: {STOCHASTIC_STATUS[status]}')
        commit, stats = {}, {}
        for i, r in enumerate(active):
            count, accepted, rejected, extra, reason, used, _status, _ = res[i]
            generators[r].set_state(states[r])
            torch.rand(n[r] + used, dtype=f64, generator=generators[r])   # consume exactly the used draws
            output[r].extend(em[i][:count])
            commit[r] = count
            stats[r] = dict(accepted=accepted, committed=count, rejected_index=None if rejected < 0 else rejected,
                            extra_token_kind={0: None, 1: 'residual', 2: 'bonus'}[extra],
                            stop_reason=('round_complete', 'eos', 'budget')[reason])
        target.commit(verified, commit)
        draft.append_committed({r: verified.context_for(r)[:, :commit[r]] for r in active if commit[r]})
        rounds.append(stats)
        active = [r for r in active if len(output[r]) < max_new_tokens and stats[r]['stop_reason'] != 'eos']
    return output, rounds
