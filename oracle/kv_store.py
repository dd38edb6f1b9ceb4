"""Persistent target KV store oracle (numpy, test infrastructure only).

Restates the storage semantics of ``PersistentTargetKV``
(dspark_qwen/persistent_target_kv.py:163-530): resident KV
``[layers, slots, context_capacity, heads, dim]``, per-layer scratch
``[layers, max_query_tokens, heads, dim]``, transaction metadata built by
``begin`` (lines 392-411), the KV append ``stage_layer`` (427-438), the
resident+scratch gather ``prepare_attention`` (441-460), the accepted-prefix
copy ``commit`` (463-491) and ``abort`` (493-499), which drops scratch rows.
"""
import numpy as np


def begin_metadata(slot_indices, contexts, query_lengths, key_capacity, context_capacity):
    """Integer transaction metadata exactly as ``begin`` builds it (lines 392-411).

    Returns a dict with committed_indices, scratch_indices, from_scratch, valid
    (length ``key_capacity``), positions (length sum Q), cu_query and cu_key.
    """
    old, new, choose, positions, cq, ck = [], [], [], [], [0], [0]
    qo = 0
    for i, c, q in zip(slot_indices, contexts, query_lengths):
        old.extend(i * context_capacity + j for j in range(c))
        old.extend([0] * q)
        new.extend([0] * c)
        new.extend(range(qo, qo + q))
        choose.extend([False] * c + [True] * q)
        positions.extend(range(c, c + q))
        qo += q
        cq.append(qo)
        ck.append(ck[-1] + c + q)
    logical_k = len(old)
    tail = key_capacity - logical_k
    if tail < 0:
        raise ValueError('Actual context exceeds declared bucket applicability')
    old.extend([0] * tail)
    new.extend([0] * tail)
    choose.extend([False] * tail)
    return dict(committed_indices=np.array(old, np.int64), scratch_indices=np.array(new, np.int64),
                from_scratch=np.array(choose, bool), valid=np.array([True] * logical_k + [False] * tail, bool),
                positions=np.array(positions, np.int64), cu_query=np.array(cq, np.int32),
                cu_key=np.array(ck, np.int32))


class OracleKVStore:
    """Single-owner resident + scratch store; arrays may hold any numpy dtype."""

    def __init__(self, layers, slots, context_capacity, max_query_tokens, heads, dim, dtype=np.float32):
        self.layers, self.slots, self.context_capacity = layers, slots, context_capacity
        self.max_query_tokens, self.heads, self.dim = max_query_tokens, heads, dim
        self.keys = np.zeros((layers, slots, context_capacity, heads, dim), dtype)
        self.values = np.zeros_like(self.keys)
        self.scratch_keys = np.zeros((layers, max_query_tokens, heads, dim), dtype)
        self.scratch_values = np.zeros_like(self.scratch_keys)
        self.lengths = [0] * slots

    def load_prefix(self, slot, keys, values):
        n = keys.shape[1]
        if self.lengths[slot] or n > self.context_capacity:
            raise ValueError('Prefix bootstrap requires empty slot within capacity')
        self.keys[:, slot, :n] = keys
        self.values[:, slot, :n] = values
        self.lengths[slot] = n

    def stage_layer(self, layer, keys, values):
        q = keys.shape[0]
        self.scratch_keys[layer, :q] = keys
        self.scratch_values[layer, :q] = values

    def prepare_attention(self, meta, layer):
        """Gather resident prefix and scratch rows; tail rows zeroed (lines 452-459)."""
        out = []
        for resident, scratch in ((self.keys, self.scratch_keys), (self.values, self.scratch_values)):
            old = resident[layer].reshape(-1, self.heads, self.dim)[meta['committed_indices']]
            new = scratch[layer][meta['scratch_indices']]
            x = np.where(meta['from_scratch'][:, None, None], new, old)
            x = np.where(meta['valid'][:, None, None], x, 0)
            out.append(x)
        return out[0], out[1]

    def commit(self, slot_indices, contexts, query_lengths, committed):
        """Copy scratch rows [qo, qo+n) into resident [c, c+n) for every layer (lines 470-491)."""
        for s, c, q, n in zip(slot_indices, contexts, query_lengths, committed):
            if not 0 <= n <= q or c + n > self.context_capacity:
                raise ValueError('Commit must be a valid verified prefix')
        qo = 0
        for s, c, q, n in zip(slot_indices, contexts, query_lengths, committed):
            self.keys[:, s, c:c + n] = self.scratch_keys[:, qo:qo + n]
            self.values[:, s, c:c + n] = self.scratch_values[:, qo:qo + n]
            qo += q
        for s, n in zip(slot_indices, committed):
            self.lengths[s] += n
        return dict(committed_tokens=int(sum(committed)),
                    copied_kv_bytes=2 * self.layers * self.heads * self.dim * self.keys.itemsize * int(sum(committed)))
