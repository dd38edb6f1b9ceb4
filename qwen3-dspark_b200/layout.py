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

    # Sizes the reference's adapters read off a layout: packed query rows, packed key
    # rows, and the number of (query, key) pairs a dense per-request product covers.
    @property
    def query_tokens(self):
        return int(sum(self.query_lengths))

    @property
    def gathered_key_tokens(self):
        return int(sum(self.key_lengths))

    @property
    def pair_domain(self):
        return int(sum(nq * nk for nq, nk in zip(self.query_lengths, self.key_lengths)))

    def gather_kv(self, key, value):
        """Pack the layout's key rows out of a head-major cache pair.

        ``key``/``value``: [1, Hkv, physical_key_tokens, D] on the layout's device, one
        dtype. Returns two [sum K, Hkv, D] tensors holding, request after request, the
        rows ``gather_indices`` names: the request-contiguous THD operand the kernels read
        (the reference's ``PackedLayout.gather_kv``, varlen_target.py:74-82)."""
        want = (1, key.shape[1] if key.ndim == 4 else -1, self.physical_key_tokens,
                key.shape[-1] if key.ndim == 4 else -1)
        if (key.ndim != 4 or tuple(key.shape) != want or tuple(value.shape) != want or value.dtype != key.dtype
                or not key.device == value.device == self.gather_indices.device):
            raise ValueError(f'gather_kv needs a key/value pair of shape [1, Hkv, {self.physical_key_tokens}, D], '
                             'one dtype, on the layout device')
        rows = self.gather_indices
        return tuple(x[0].permute(1, 0, 2)[rows] for x in (key, value))


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


@dataclass(frozen=True)
class TrainingLayout:
    """Packed training layout of the draft attention over several sequences.

    Per sequence s (``DraftAttention.forward`` with ``block_mask``,
    dspark_qwen/model.py:12-19,47-61): ``context_lengths[s]`` context rows and one
    draft block of ``block_size`` rows per anchor in ``anchors[s]``. Queries are
    the block rows (block b = rows ``[block_size*b, +block_size)``), keys are
    ``[context rows ; block rows]`` (what ``project_kv(cat(context, z))`` builds).
    Block b sees context rows ``j < anchors[s][b]`` and its own rows; sequences
    never see each other (the packing rule of the vendored NeMo mask). Anchors
    outside ``[0, context]`` act as the nearest end, exactly as in the mask.

    ``plan`` is the tensor-core kernel's work plan (``dspark_train_plan``), built
    once on the host and kept on the device; the per-block ``seg_*`` tensors
    describe the same layout as two-segment requests for the float32 kernel.
    """
    context_lengths: tuple
    anchors: tuple
    block_size: int
    query_lengths: tuple
    key_lengths: tuple
    plan: torch.Tensor
    grid: int
    seg_cu_query: torch.Tensor
    seg_a_start: torch.Tensor
    seg_a_len: torch.Tensor
    seg_b_start: torch.Tensor
    seg_b_len: torch.Tensor

    @classmethod
    def from_anchors(cls, context_lengths, anchors, block_size=7, device='cuda', grid_limit=None):
        from . import _lib
        ctx = tuple(int(c) for c in context_lengths)
        anc = tuple(tuple(int(a) for a in seq) for seq in anchors)
        if not ctx or len(ctx) != len(anc) or any(c < 0 for c in ctx):
            raise ValueError('One nonnegative context length and one anchor list per sequence required')
        if type(block_size) is not int or not 6 <= block_size <= 32:
            raise ValueError('block_size must be an integer in [6, 32]')
        if not any(anc):
            raise ValueError('At least one anchor (draft block) is required')
        device = torch.device(device)
        if grid_limit is None:
            grid_limit = torch.cuda.get_device_properties(device).multi_processor_count
        plan = _lib.train_plan(ctx, [len(a) for a in anc], [a for seq in anc for a in seq], block_size,
                               int(grid_limit))
        qlens = tuple(len(a) * block_size for a in anc)
        klens = tuple(c + q for c, q in zip(ctx, qlens))
        a_start, a_len, b_start = [], [], []
        ko = 0
        for c, seq in zip(ctx, anc):
            for b, a in enumerate(seq):
                a_start.append(ko)
                a_len.append(min(max(a, 0), c))
                b_start.append(ko + c + block_size * b)
            ko += c + len(seq) * block_size
        nblk = len(a_start)

        def dev(x):
            t = torch.tensor(x, dtype=torch.int32)
            return t.pin_memory().to(device, non_blocking=True) if device.type == 'cuda' else t

        return cls(ctx, anc, block_size, qlens, klens, dev(plan), int(plan[2]),
                   dev([block_size * i for i in range(nblk + 1)]), dev(a_start), dev(a_len), dev(b_start),
                   dev([block_size] * nblk))

    @property
    def query_tokens(self):
        return sum(self.query_lengths)

    @property
    def key_tokens(self):
        return sum(self.key_lengths)


def cumulative(lengths, device):
    ends = [0]
    for n in lengths:
        ends.append(ends[-1] + n)
    if ends[-1] >= 2 ** 31:
        raise ValueError('Varlen cumulative lengths exceed int32')
    return torch.tensor(ends, device=device, dtype=torch.int32)
