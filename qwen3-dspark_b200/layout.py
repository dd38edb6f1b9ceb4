"""Packed varlen layouts consumed by the B200 kernels.

``PackedLayout`` mirrors the reference's layout type (dspark_qwen/varlen_target.py:17-82):
same fields, same ``from_metadata`` refusals, same int32 cumulative offsets.
The kernels read only ``query_lengths``/``key_lengths`` (host tuples) and
``cu_query``/``cu_key`` (int32 device tensors), so a reference ``PackedLayout``
or ``PersistentAttentionLayout`` instance works unchanged as well.
"""
from dataclasses import dataclass

import torch


@dataclass(frozen=True)
class PackedLayout:
    request_markers: tuple
    query_lengths: tuple
    key_lengths: tuple
    cu_query: torch.Tensor
    cu_key: torch.Tensor
    gather_indices: torch.Tensor
    physical_key_tokens: int

    @classmethod
    def from_metadata(cls, query_requests, query_positions, key_requests, key_positions):
        """Markers/positions -> lengths, cumulative offsets and gather order (varlen_target.py:28-60)."""
        arrays = (query_requests, query_positions, key_requests, key_positions)
        if any(not isinstance(x, torch.Tensor) or x.ndim != 1 or x.dtype != torch.long for x in arrays):
            raise ValueError('Expected flat long request/position metadata')
        if any(x.device != query_requests.device for x in arrays):
            raise ValueError('All layout metadata must share a device')
        if (query_requests.numel() == 0 or query_requests.shape != query_positions.shape
                or key_requests.shape != key_positions.shape):
            raise ValueError('Nonempty queries and matching marker/position lengths required')
        # One host copy of the metadata, then pure-Python checks (no per-request syncs).
        qr, qp, kr, kp = (x.tolist() for x in arrays)
        markers, counts = [], []
        for m in qr:
            if markers and markers[-1] == m:
                counts[-1] += 1
            else:
                markers.append(m)
                counts.append(1)
        if len(set(markers)) != len(markers):
            raise ValueError('Each request query must form one contiguous chunk')
        by_marker = {}
        for j, m in enumerate(kr):
            by_marker.setdefault(m, []).append(j)
        gathers, k_lengths, offset = [], [], 0
        for marker, count in zip(markers, counts):
            indices = by_marker.get(marker, [])
            length = len(indices)
            if length < count or any(kp[j] != p for p, j in enumerate(indices)):
                raise ValueError('Active keys must be a complete request-local prefix')
            if qp[offset:offset + count] != list(range(length - count, length)):
                raise ValueError('Queries must be the terminal suffix of their own key prefix')
            gathers.extend(indices)
            k_lengths.append(length)
            offset += count
        device = query_requests.device
        return cls(tuple(markers), tuple(counts), tuple(k_lengths), cumulative(counts, device),
                   cumulative(k_lengths, device), torch.tensor(gathers, dtype=torch.long, device=device),
                   key_requests.numel())

    @classmethod
    def from_lengths(cls, query_lengths, key_lengths, device):
        """Layout of request-contiguous packed K/V (gather order = identity)."""
        q, k = tuple(int(x) for x in query_lengths), tuple(int(x) for x in key_lengths)
        if not q or len(q) != len(k):
            raise ValueError('One query and key length per request required')
        return cls(tuple(range(len(q))), q, k, cumulative(q, device), cumulative(k, device),
                   torch.arange(sum(k), device=device), sum(k))

    @property
    def query_tokens(self):
        return sum(self.query_lengths)

    @property
    def gathered_key_tokens(self):
        return sum(self.key_lengths)

    @property
    def pair_domain(self):
        return sum(q * k for q, k in zip(self.query_lengths, self.key_lengths))

    def gather_kv(self, key, value):
        """[1,Hkv,physical_K,D] cache -> packed [sum K, Hkv, D] (varlen_target.py:74-82)."""
        if (key.ndim != 4 or key.shape[0] != 1 or value.shape != key.shape
                or key.shape[2] != self.physical_key_tokens or key.device != self.gather_indices.device
                or value.device != key.device or value.dtype != key.dtype):
            raise ValueError('Expected matching [1,Hkv,physical_K,D] cache tensors')
        return tuple(x.index_select(2, self.gather_indices).squeeze(0).transpose(0, 1).contiguous()
                     for x in (key, value))


@dataclass(frozen=True)
class PersistentAttentionLayout:
    """Capacity-tail verify layout (dspark_qwen/persistent_qwen_target.py:19-27)."""
    query_lengths: tuple
    key_lengths: tuple
    cu_query: torch.Tensor
    cu_key: torch.Tensor
    physical_key_capacity: int
    maximum_key_length: int = 0
    maximum_query_length: int = 0


def cumulative(lengths, device):
    ends = [0]
    for n in lengths:
        ends.append(ends[-1] + n)
    if ends[-1] >= 2 ** 31:
        raise ValueError('Varlen cumulative lengths exceed int32')
    return torch.tensor(ends, device=device, dtype=torch.int32)
