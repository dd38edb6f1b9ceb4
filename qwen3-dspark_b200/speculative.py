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

from . import _lib


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


def _round_status(target=None, verified=None, where='decode round'):
    """Read and clear the library's device status word once per round, where the round's
    results are already synchronised. The kernels report a wait that ran out or an index
    they refused there instead of faulting, so a non-zero word means this round's logits or
    tokens may be partly written: the verify transaction is aborted (no KV is committed,
    the draft pool is untouched until the commit) and the loop raises."""
    status = _lib.read_device_status(clear=True)
    if status:
        if verified is not None:
            target.abort(verified)
        raise RuntimeError(f'device status {status:#x} after the {where} ({_lib.describe_status(status)}); '
                           'nothing of the round was kept')


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
    _round_status(where='prefill')
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
        _round_status(target, verified)
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
def speculative_sample(target, draft, prompts, max_new_tokens, generators, temperature=1.0, eos_ids=(),
                       graph=False):
    """Batched stochastic speculative decoding; per request the rule of
    ``cached_speculative_sample`` (dspark_qwen/cached_sampling.py:80-175) under the
    reference's float64 law. ``generators``: {request: CPU torch.Generator}. Each
    request's uniforms come from its generator in the reference's draw order (the
    first token, then per round the proposal draws and the acceptance draws), and
    after each round the generator is left exactly where the reference's would be,
    so a request's tokens equal the reference's single-request run with the same
    seed. Acceptance runs on the GPU (``stochastic_accept``); the host reads back one
    small result per round. ``graph`` replays the target's verify forward from a CUDA
    graph per set of chunk lengths and, for bf16 drafts with the fused Markov head, the
    stochastic proposal from a graph per (request count, temperature) and the draft
    append of whole chunks from a graph per shape; the tokens are those of the eager
    loop. Returns ({request: tokens}, rounds)."""
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
    _round_status(where='prefill')
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
        use_graph = graph and getattr(draft, '_graph_ready', lambda: False)()
        if use_graph:
            if (len(active), temperature) not in draft.__dict__.get('_sgraphs', {}):
                draft.capture_propose_stochastic(len(active), temperature)
            tokens, laws = draft.propose_stochastic_graph(anchors, n, u_prop, temperature)
        else:
            tokens, laws = draft.propose_stochastic(anchors, n, u_prop, temperature)
        chunks = {r: torch.cat((anchors[r][0], tokens[r]))[None] for r in active}
        if graph:
            bucket = QueryBucket(tuple(n[r] + 1 for r in active))
            if bucket not in target._graphs:
                target.capture(bucket)
            verified = target.verify_graph(chunks, bucket)
        else:
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
        try:
            _round_status(target, verified)
        except RuntimeError:
            for r in active:
                generators[r].set_state(states[r])
            raise
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
        width = size + 1
        if use_graph and hasattr(draft, 'capture_append') and all(n[r] + 1 == width for r in active):
            # whole verified chunks through the captured fixed-shape append
            if (len(active), width) not in draft.__dict__.get('_append_graphs', {}):
                draft.capture_append(len(active), width)
            draft.append_verified_graph(verified.context, tuple(active), [commit[r] for r in active])
        else:
            draft.append_committed({r: verified.context_for(r)[:, :commit[r]] for r in active if commit[r]})
        rounds.append(stats)
        active = [r for r in active if len(output[r]) < max_new_tokens and stats[r]['stop_reason'] != 'eos']
    return output, rounds


@torch.no_grad()
def speculative_greedy_pipelined(target, draft, prompts, max_new_tokens, eos_ids=()):
    """``speculative_greedy(graph=True)`` with the round state kept on the GPU, so the
    host never sits between two rounds (the device-side transaction metadata and
    accept-to-commit path of the reference's captured verify,
    persistent_qwen_graph.py:198-275 and persistent_target_kv.py:369-415).

    Every round runs the captured draft proposal, the captured target verify, the
    on-device greedy accept, the commit kernel and the captured fixed-shape draft
    append; between them, device ops derive the next round's inputs from this
    round's results: anchors (the last committed token), the target's context lengths
    and positions, the draft's lengths and positions, and each request's remaining
    budget (zeroed by an EOS). The host enqueues round k + 1 before it reads round k's
    small result vector, so the GPU never waits for it. A finished request stays in
    the fixed-shape batch and commits nothing. The same tokens as ``speculative_greedy``;
    needs a bf16 draft whose Markov head runs on the fused kernel. Returns
    ({request: tokens}, rounds)."""
    from .kernels import greedy_accept
    if type(max_new_tokens) is not int or max_new_tokens < 0:
        raise ValueError('max_new_tokens must be a nonnegative integer')
    if not draft._graph_ready():
        raise ValueError('The pipelined loop needs a bf16 draft whose Markov head runs on the fused kernel')
    eos_ids = sorted(set(int(e) for e in eos_ids))
    dev = target.device
    for r in prompts:
        target.add_request(r)
        draft.add_request(r)
    if max_new_tokens == 0:
        return {r: [] for r in prompts}, []
    features = target.prefill(prompts)
    last = target.predict(features, last_only=True)
    requests = list(prompts)
    output = {r: [int(last[r].argmax(-1).item())] for r in requests}
    _round_status(where='prefill')
    draft.append_committed({r: features.context_for(r) for r in requests})
    if max_new_tokens == 1 or all(output[r][-1] in eos_ids for r in requests):
        return output, []
    R, size = len(requests), draft.draft.spec.block_size
    width = size + 1
    store = target.pool
    handles = [target._handles[r] for r in requests]
    slots = [h.index for h in handles]
    # -- fixed buffers of the three captured programs -----------------------------------
    bucket = QueryBucket((width,) * R)
    if bucket not in target._graphs:
        target.capture(bucket)
    tg = target._graphs[bucket]
    tmeta = store.bind_bucket(bucket).meta
    if R not in draft.__dict__.get('_graphs', {}):
        draft.capture_propose(R)
    pg = draft._graphs[R]
    if (R, width) not in draft.__dict__.get('_append_graphs', {}):
        draft.capture_append(R, width)
    ag = draft._append_graphs[(R, width)]
    i32 = torch.int32
    cu_t = [width * i for i in range(R + 1)]
    ctx0 = [store.length(h) for h in handles]
    dlen0 = [draft._lengths[r] for r in requests]
    if any(c + max_new_tokens + width > store.capacities[s] for c, s in zip(ctx0, slots)):
        raise ValueError('Request slots cannot hold max_new_tokens plus one verify chunk')
    tmeta.copy_(torch.tensor(cu_t + [store.slot_rows[s] for s in slots] + ctx0
                             + [store.capacities[s] for s in slots], dtype=i32))
    pg['meta'].copy_(torch.tensor([size * i for i in range(R + 1)]
                                  + [draft.slot_rows[draft._slots[r]] for r in requests] + dlen0 + [size] * R,
                                  dtype=i32))
    ag['meta'].copy_(torch.tensor(cu_t + [draft.slot_rows[draft._slots[r]] for r in requests] + dlen0 + [0] * R,
                                  dtype=i32))
    ctx = tmeta[2 * R + 1:3 * R + 1]                  # target context lengths (device state)
    dlen = pg['meta'][2 * R + 1:3 * R + 1]            # draft context lengths (device state)
    anchors = torch.tensor([output[r][-1] for r in requests], dtype=torch.long, device=dev)
    budget = torch.tensor([max_new_tokens - 1 if output[r][-1] not in eos_ids else 0 for r in requests],
                          dtype=i32, device=dev)
    cu_dev = torch.tensor(cu_t, dtype=i32, device=dev)
    rep_t = torch.arange(R, device=dev).repeat_interleave(width)
    off_t = torch.arange(width, device=dev).repeat(R)
    rep_d = torch.arange(R, device=dev).repeat_interleave(size)
    off_d = torch.arange(size, device=dev).repeat(R)
    lm_head = target.model.get_output_embeddings()
    eos_dev = torch.tensor(eos_ids, dtype=torch.long, device=dev)
    lib = _lib.load_library()
    stream = torch.cuda.current_stream(dev)
    res_host = [torch.empty(2 * R + R * width, dtype=torch.long).pin_memory() for _ in range(2)]
    # the device status word after each round, copied with the round's results (a
    # synchronous read would wait for the round enqueued behind it)
    status_host = torch.zeros(2, dtype=torch.int32).pin_memory()
    events = [torch.cuda.Event() for _ in range(2)]

    def launch_round(k):
        pg['anchors'].copy_(anchors)
        pg['pos'].copy_((dlen.long()[rep_d] + off_d))
        pg['graph'].replay()
        tg['ids'][0].copy_(torch.cat((anchors[:, None], pg['tokens']), dim=1).reshape(-1))
        tg['pos'][0].copy_(ctx.long()[rep_t] + off_t)
        tg['graph'].replay()
        logits = lm_head(tg['last'])[0]
        _pred, accepted, n_commit, emitted = greedy_accept(logits, tg['ids'][0], cu_dev, eos_dev, budget)
        # commit the verified prefixes (rollback of the rest), all layers, one launch
        _lib.check(lib.dspark_commit_kv(
            store._keys.data_ptr(), store._values.data_ptr(), store.scratch_keys.data_ptr(),
            store.scratch_values.data_ptr(), tmeta.data_ptr(), tmeta[R + 1:].data_ptr(), ctx.data_ptr(),
            tmeta[3 * R + 1:].data_ptr(), n_commit.data_ptr(), R, store.layers, store.rows_per_layer,
            store.max_query_tokens, _lib.DTYPE_F32 if store.dtype == torch.float32 else _lib.DTYPE_BF16,
            stream.cuda_stream), 'dspark_commit_kv')
        ctx.add_(n_commit)
        # the draft projects the committed rows of every verified chunk
        ag['feat'].copy_(tg['context'])
        ag['meta'][2 * R + 1:3 * R + 1].copy_(dlen)
        ag['meta'][3 * R + 1:].copy_(n_commit)
        ag['graph'].replay()
        dlen.add_(n_commit)
        last_idx = cu_dev[:-1].long() + (n_commit.long() - 1).clamp(min=0)
        last_tok = emitted[last_idx]
        anchors.copy_(torch.where(n_commit > 0, last_tok, anchors))
        hit = (n_commit > 0) & torch.isin(last_tok, eos_dev) if eos_ids else torch.zeros_like(n_commit, dtype=torch.bool)
        budget.copy_(torch.where(hit, torch.zeros_like(budget), budget - n_commit))
        buf = res_host[k & 1]
        buf.copy_(torch.cat((accepted.long(), n_commit.long(), emitted)), non_blocking=True)
        _lib.check(lib.dspark_copy_device_status(status_host[k & 1:].data_ptr(), stream.cuda_stream),
                   'dspark_copy_device_status')
        events[k & 1].record(stream)

    rounds = []
    done = {r: output[r][-1] in eos_ids for r in requests}
    launch_round(0)
    k = 0
    while True:
        if not all(done.values()):
            launch_round(k + 1)                        # enqueued before round k is read
        events[k & 1].synchronize()
        status = int(status_host[k & 1])
        if status:
            # this round (and the one enqueued behind it) already committed on the
            # device, so nothing can be rolled back: the store refuses further use
            torch.cuda.synchronize(dev)
            _lib.read_device_status(clear=True)
            store.failed = True
            raise RuntimeError(f'device status {status:#x} in a pipelined decode round '
                               f'({_lib.describe_status(status)}); the KV store is invalidated')
        host = res_host[k & 1].tolist()
        stats = {}
        for i, r in enumerate(requests):
            if done[r]:
                continue
            n = host[R + i]
            committed = host[2 * R + width * i:2 * R + width * i + n]
            output[r].extend(committed)
            stats[r] = dict(accepted=host[i], committed=n)
            if len(output[r]) >= max_new_tokens or (committed and committed[-1] in eos_ids):
                done[r] = True
        rounds.append(stats)
        if all(done.values()):
            break
        k += 1
    torch.cuda.synchronize(dev)
    # the host mirrors of the committed lengths follow the device state
    store.mirror_lengths(handles, ctx.tolist())
    for r, d in zip(requests, dlen.tolist()):
        draft._lengths[r] = d
    return output, rounds
