"""Packed varlen layout oracle (pure Python, test infrastructure only).

Restates ``PackedLayout.from_metadata`` (dspark_qwen/varlen_target.py:28-60):
request markers and positions become per-request query/key lengths, int32
cumulative offsets and the gather order of active key rows, with the same
refusals (non-contiguous request queries, incomplete key prefixes, queries that
are not the terminal suffix of their own key prefix, int32 overflow).
"""
from dataclasses import dataclass


@dataclass(frozen=True)
class OracleLayout:
    request_markers: tuple
    query_lengths: tuple
    key_lengths: tuple
    cu_query: tuple
    cu_key: tuple
    gather_indices: tuple
    physical_key_tokens: int

    @property
    def pair_domain(self):
        # varlen_target.py:71-72
        return sum(q * k for q, k in zip(self.query_lengths, self.key_lengths))


def _cumulative(lengths):
    ends = [0]
    for n in lengths:
        ends.append(ends[-1] + n)
    if ends[-1] >= 2 ** 31:
        raise ValueError('Varlen cumulative lengths exceed int32')
    return tuple(ends)


def packed_layout_from_metadata(query_requests, query_positions, key_requests, key_positions):
    qr, qp, kr, kp = (list(map(int, x)) for x in (query_requests, query_positions, key_requests, key_positions))
    if not qr or len(qr) != len(qp) or len(kr) != len(kp):
        raise ValueError('Nonempty queries and matching marker/position lengths required')
    markers, counts = [], []
    for m in qr:                       # unique_consecutive with counts
        if markers and markers[-1] == m:
            counts[-1] += 1
        else:
            markers.append(m)
            counts.append(1)
    if len(set(markers)) != len(markers):
        raise ValueError('Each request query must form one contiguous chunk')
    gathers, k_lengths, offset = [], [], 0
    for marker, count in zip(markers, counts):
        indices = [j for j, m in enumerate(kr) if m == marker]
        length = len(indices)
        if length < count or [kp[j] for j in indices] != list(range(length)):
            raise ValueError('Active keys must be a complete request-local prefix')
        if qp[offset:offset + count] != list(range(length - count, length)):
            raise ValueError('Queries must be the terminal suffix of their own key prefix')
        gathers.extend(indices)
        k_lengths.append(length)
        offset += count
    return OracleLayout(tuple(markers), tuple(counts), tuple(k_lengths), _cumulative(counts),
                        _cumulative(k_lengths), tuple(gathers), len(kr))
