"""Torch CPU restatement of the reference's own CPU attention round (test infrastructure).

TEST INFRASTRUCTURE ONLY: the timed CPU baseline of ``bench.py`` (``--impl reference``
and the GPU arm's ``cpu_baseline`` leg) and a checker in ``tests/``. Nothing in the
product package imports it.

The reference's CPU path for the two attention hot paths is plain torch on the host,
float32 by default, and this module issues the same torch operations in the same
order so that its time is the reference's time on the same host threads:

* draft: ``test_only_noncausal_varlen`` (dspark_qwen/packed_draft.py:35-47), one
  ``scaled_dot_product_attention`` per request, no mask, ``enable_gqa=True``;
* verify, per layer: the Qwen3 attention's q/k ``Qwen3RMSNorm`` and rotate-half RoPE
  (transformers ``modeling_qwen3.py``: ``Qwen3RMSNorm.forward`` 59-64,
  ``Qwen3RotaryEmbedding.forward`` 137-148, ``apply_rotary_pos_emb`` 151-181), then
  ``PersistentTargetKV.stage_layer`` (dspark_qwen/persistent_target_kv.py:427-439:
  scratch copy) and ``prepare_attention`` (441-461: two ``index_select`` gathers,
  ``where``, ``masked_fill`` over the bucket's key capacity, for K and for V), then
  ``test_only_persistent_sdpa`` (dspark_qwen/persistent_qwen_target.py:30-42: one SDPA
  per request with the bottom-right boolean mask);
* per round: ``begin`` (persistent_target_kv.py:369-415: host index lists for the
  bucket, uploaded with ``torch.tensor``) and ``commit`` (463-491: per-request copies of
  the accepted scratch prefix into every layer's resident rows);
* the training layout (config 4): ``block_mask`` and the dense-mask SDPA of
  ``DraftAttention.forward`` per sequence (dspark_qwen/model.py:12-19,47-61).

The one departure is storage: the reference's resident cache is one dense
``[layers, slots, context_capacity, heads, dim]`` tensor; this store gives each slot
its own capacity (the ``slot_capacities`` argument, default uniform as in the reference)
so that a sample of long and short requests fits host memory. Gathers read the same
rows either way. ``tests/test_oracle_torch_cpu.py`` checks every function against the
fixtures made by the reference's own functions (``tests/golden/make_golden.py``).
"""
import torch
import torch.nn.functional as F


def noncausal_varlen_sdpa(query, key, value, query_lengths, key_lengths, scale):
    """packed_draft.py:35-47: per request, every query row sees all of its keys."""
    rows, qo, ko = [], 0, 0
    for nq, nk in zip(query_lengths, key_lengths):
        out = F.scaled_dot_product_attention(
            query[qo:qo + nq].transpose(0, 1)[None], key[ko:ko + nk].transpose(0, 1)[None],
            value[ko:ko + nk].transpose(0, 1)[None], attn_mask=None, dropout_p=0., is_causal=False,
            scale=scale, enable_gqa=True)
        rows.append(out.squeeze(0).transpose(0, 1))
        qo += nq
        ko += nk
    return torch.cat(rows)


def persistent_sdpa(query, key, value, query_lengths, key_lengths, scale):
    """persistent_qwen_target.py:30-42: request-local bottom-right causal attention; key
    rows past sum(key_lengths) (a capacity tail) are never read."""
    rows, qo, ko = [], 0, 0
    for nq, nk in zip(query_lengths, key_lengths):
        visible = torch.arange(nk)[None, :] <= torch.arange(nk - nq, nk)[:, None]
        out = F.scaled_dot_product_attention(
            query[qo:qo + nq].transpose(0, 1)[None], key[ko:ko + nk].transpose(0, 1)[None],
            value[ko:ko + nk].transpose(0, 1)[None], attn_mask=visible[None, None], dropout_p=0.,
            is_causal=False, scale=scale, enable_gqa=True)
        rows.append(out[0].transpose(0, 1))
        qo += nq
        ko += nk
    return torch.cat(rows)


def qwen3_rms_norm(x, weight, eps):
    """Qwen3RMSNorm.forward: float32 variance, rsqrt, cast back, then the weight."""
    dtype = x.dtype
    h = x.to(torch.float32)
    variance = h.pow(2).mean(-1, keepdim=True)
    h = h * torch.rsqrt(variance + eps)
    return weight * h.to(dtype)


def rotary_cos_sin(positions, inv_freq, dtype):
    """Qwen3RotaryEmbedding.forward for one packed row list: float32 angles, cos/sin cast
    to the activation dtype (attention_scaling 1 for the default rope type)."""
    freqs = positions[:, None].to(torch.float32) * inv_freq[None, :].to(torch.float32)
    emb = torch.cat((freqs, freqs), dim=-1)
    return emb.cos().to(dtype), emb.sin().to(dtype)


def apply_rope(x, cos, sin):
    """apply_rotary_pos_emb on packed rows [n, heads, dim] with per-row cos/sin [n, dim]."""
    half = x.shape[-1] // 2
    rotated = torch.cat((-x[..., half:], x[..., :half]), dim=-1)
    return x * cos[:, None] + rotated * sin[:, None]


def block_mask(anchors, block_size, context_length):
    """model.py:12-19: context j < anchor of the query's block; the own block is
    bidirectional; [1, 1, n * bs, ctx + n * bs] booleans."""
    n = anchors.numel()
    q_block = torch.arange(n * block_size) // block_size
    ctx = torch.arange(context_length)
    visible_context = ctx[None, :] < anchors[q_block, None]
    visible_block = q_block[:, None] == q_block[None, :]
    return torch.cat((visible_context, visible_block), dim=-1)[None, None]


def training_layout_sdpa(query, key, value, context_lengths, anchors, block_size):
    """The training layout's attention as `DraftAttention.forward` runs it per sequence
    (model.py:47-61): K/V repeated per GQA group, one dense `block_mask` SDPA with the
    default 1/sqrt(d) scale; sequences packed back to back never see each other."""
    rows, qo, ko = [], 0, 0
    for ctx, anc in zip(context_lengths, anchors):
        nq = len(anc) * block_size
        nk = ctx + nq
        mask = block_mask(torch.as_tensor(anc, dtype=torch.long), block_size, ctx)
        groups = query.shape[1] // key.shape[1]
        q = query[qo:qo + nq].transpose(0, 1)[None]
        k = key[ko:ko + nk].transpose(0, 1)[None].repeat_interleave(groups, dim=1)
        v = value[ko:ko + nk].transpose(0, 1)[None].repeat_interleave(groups, dim=1)
        out = F.scaled_dot_product_attention(q, k, v, attn_mask=mask, dropout_p=0.0, is_causal=False)
        rows.append(out[0].transpose(0, 1))
        qo += nq
        ko += nk
    return torch.cat(rows)


class VerifyRoundCPU:
    """The reference's verify data path on the host: resident slots, a layer-indexed
    scratch, ``begin`` metadata, per-layer stage + gather + attention, and ``commit``.

    ``contexts`` are the slots' committed lengths; ``slot_capacities`` their capacities
    (default: one uniform capacity, the reference's layout). K/V are ``dtype`` (float32,
    the reference store's default)."""

    def __init__(self, layers, contexts, max_query_tokens, heads, dim, slot_capacities=None,
                 dtype=torch.float32, generator=None):
        caps = list(slot_capacities) if slot_capacities is not None else [max(contexts) + max_query_tokens] * len(
            contexts)
        if len(caps) != len(contexts) or any(c > cap for c, cap in zip(contexts, caps)):
            raise ValueError('every context must fit its slot capacity')
        self.layers, self.heads, self.dim, self.dtype = layers, heads, dim, dtype
        self.capacities = caps
        self.offsets = [0]
        for cap in caps:
            self.offsets.append(self.offsets[-1] + cap)
        rows = self.offsets[-1]
        # resident contents: N(0,1) rows of the first layer, repeated for the others (the
        # values do not change the work; drawing every layer would dominate set-up time)
        self.keys = torch.empty((layers, rows, heads, dim), dtype=dtype)
        self.values = torch.empty_like(self.keys)
        self.keys[0] = torch.randn((rows, heads, dim), dtype=dtype, generator=generator)
        self.values[0] = torch.randn((rows, heads, dim), dtype=dtype, generator=generator)
        self.keys[1:] = self.keys[:1]
        self.values[1:] = self.values[:1]
        self.scratch_keys = torch.zeros((layers, max_query_tokens, heads, dim), dtype=dtype)
        self.scratch_values = torch.zeros_like(self.scratch_keys)
        self.lengths = list(contexts)
        # the bucket workspace (persistent_target_kv.py:127-153), sized once for the
        # largest key count the slots can hold
        shape = (rows, heads, dim)
        self.ws = {name: torch.empty(shape, dtype=dtype) for name in ('old_k', 'old_v', 'new_k', 'new_v', 'keys',
                                                                      'values')}

    def begin(self, query_lengths):
        """persistent_target_kv.py:369-415: host index lists, one upload per list."""
        old, new, choose, positions, cq, ck = [], [], [], [], [0], [0]
        qo = 0
        for i, (c, q) in enumerate(zip(self.lengths, query_lengths)):
            base = self.offsets[i]
            old.extend(base + j for j in range(c))
            old.extend([0] * q)
            new.extend([0] * c)
            new.extend(range(qo, qo + q))
            choose.extend([False] * c + [True] * q)
            positions.extend(range(c, c + q))
            qo += q
            cq.append(qo)
            ck.append(ck[-1] + c + q)
        n = len(old)
        ws = self.ws
        ws.update(committed=torch.tensor(old, dtype=torch.long), scratch=torch.tensor(new, dtype=torch.long),
                  from_scratch=torch.tensor(choose, dtype=torch.bool).reshape(n, 1, 1),
                  valid=torch.ones((n, 1, 1), dtype=torch.bool),
                  positions=torch.tensor(positions, dtype=torch.long),
                  cu_query=torch.tensor(cq, dtype=torch.int32), cu_key=torch.tensor(ck, dtype=torch.int32),
                  rows=n, query_lengths=tuple(query_lengths),
                  key_lengths=tuple(c + q for c, q in zip(self.lengths, query_lengths)))
        return ws

    def layer(self, ws, layer, q_raw, k_raw, v, q_weight, k_weight, inv_freq, eps, scale):
        """One verify layer: q/k norm + RoPE, stage_layer, prepare_attention, SDPA."""
        cos, sin = rotary_cos_sin(ws['positions'], inv_freq, q_raw.dtype)
        q = apply_rope(qwen3_rms_norm(q_raw, q_weight, eps), cos, sin)
        k = apply_rope(qwen3_rms_norm(k_raw, k_weight, eps), cos, sin)
        nq = q.shape[0]
        self.scratch_keys[layer, :nq].copy_(k)
        self.scratch_values[layer, :nq].copy_(v)
        n = ws['rows']
        for resident, scratch, old, new, out in ((self.keys, self.scratch_keys, ws['old_k'], ws['new_k'], ws['keys']),
                                                 (self.values, self.scratch_values, ws['old_v'], ws['new_v'],
                                                  ws['values'])):
            old, new, out = old[:n], new[:n], out[:n]
            torch.index_select(resident[layer], 0, ws['committed'], out=old)
            torch.index_select(scratch[layer], 0, ws['scratch'], out=new)
            torch.where(ws['from_scratch'], new, old, out=out)
            out.masked_fill_(~ws['valid'], 0)
        return persistent_sdpa(q, ws['keys'][:n], ws['values'][:n], ws['query_lengths'], ws['key_lengths'], scale)

    def commit(self, ws, counts):
        """persistent_target_kv.py:463-491: copy each request's accepted scratch prefix
        into every layer's resident rows; lengths advance."""
        qo = 0
        for i, (c, q, m) in enumerate(zip(self.lengths, ws['query_lengths'], counts)):
            if not 0 <= m <= q or c + m > self.capacities[i]:
                raise ValueError('Commit must be a valid verified prefix')
            r0 = self.offsets[i] + c
            self.keys[:, r0:r0 + m].copy_(self.scratch_keys[:, qo:qo + m])
            self.values[:, r0:r0 + m].copy_(self.scratch_values[:, qo:qo + m])
            qo += q
        self.lengths = [c + m for c, m in zip(self.lengths, counts)]
