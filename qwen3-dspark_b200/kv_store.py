"""Persistent target KV store with the fused B200 verify layer and one-launch commit.

Mirrors ``PersistentTargetKV`` (dspark_qwen/persistent_target_kv.py:163-530):
slot handles with incarnations, ``load_prefix``, ``begin`` / ``stage_layer`` /
``prepare_attention`` / ``commit`` / ``abort`` transactions, ``request_kv``,
``pointers`` and ``work``, with the same refusals. What changes is where the
bytes go:

* ``verify_layer`` runs one decoder layer's verify attention as one kernel:
  QK-RMSNorm + RoPE of the new tokens, their KV append into scratch, and
  bottom-right causal attention that reads the resident prefix in place. The
  reference's per-bucket gather workspace (6 capacity-sized tensors) and its
  index_select/where/masked_fill staging do not exist here.
* ``commit`` copies every request's accepted scratch prefix for all layers in
  one launch; rejected rows are simply not copied (rollback).

Resident memory is ``[layers * rows_per_layer, heads, dim]``; slot ``s`` owns
rows ``[slot_row[s], slot_row[s] + capacity[s])`` of every layer. With uniform
capacities this is byte-for-byte the reference's ``[layers, slots, C, H, D]``
layout (``keys`` returns that view); ragged ``slot_capacities`` let long and
short requests share HBM without padding every slot to the longest context.
"""
import heapq
from dataclasses import dataclass
from typing import Mapping

import torch

from . import _lib
from .kernels import HEAD_DIM, HKV, HQ, SCALE, rope_cache, rope_table, runtime_identity


@dataclass(frozen=True)
class Slot:
    """Handle of one admitted request: its id, its resident slot and the slot's
    generation when it was issued (the reference's ``Slot`` fields)."""
    request: str
    index: int
    incarnation: int


class _SlotTable:
    """Resident-slot ownership: which request holds which slot, and its committed length.

    A slot's generation advances every time a request is admitted into it, and the
    table keeps the one handle object it issued for the current generation. A handle
    is honoured only if it IS that object: a handle kept past ``release`` (the slot
    reused by a new request), a copy of a live handle, an equal-valued handle built by
    hand or one issued by another store all fail the same single identity check.
    Admission takes the lowest free index, so slot assignment is deterministic.
    """

    def __init__(self, count):
        self.count = count
        self.generation = [0] * count
        self.holder = [None] * count        # issued Slot of the live generation, or None
        self.length = [0] * count           # committed rows per slot (host mirror)
        self._free = list(range(count))     # min-heap of unoccupied indices
        self._requests = set()

    def admit(self, request):
        if not isinstance(request, str) or not request or request in self._requests:
            raise ValueError('request id must be a non-empty string that is not already resident')
        if not self._free:
            raise ValueError('no free resident slot: every slot holds a request')
        i = heapq.heappop(self._free)
        self.generation[i] += 1
        handle = Slot(request, i, self.generation[i])
        self.holder[i], self.length[i] = handle, 0
        self._requests.add(request)
        return handle

    def index_of(self, handle):
        i = handle.index if type(handle) is Slot else None
        if type(i) is not int or not 0 <= i < self.count or self.holder[i] is not handle:
            raise ValueError('request handle is stale, copied or issued by another store')
        return i

    def release(self, i):
        self._requests.discard(self.holder[i].request)
        self.holder[i], self.length[i] = None, 0
        heapq.heappush(self._free, i)

    def resident_tokens(self):
        return sum(self.length)


@dataclass(frozen=True)
class Transaction:
    sequence: int
    slots: tuple
    context_lengths: tuple
    query_lengths: tuple
    meta: torch.Tensor          # int32 [4R+1]: cu_q | slot_row | ctx_len | slot_cap
    rope: dict = None           # inv_freq tensor -> [sum Q, 64] cos/sin table, built once per transaction
    table: torch.Tensor = None  # fixed cos/sin buffer of a bound bucket (graph capture/replay)
    capture: bool = False       # the placeholder transaction a CUDA graph is captured under

    @property
    def query_tokens(self):
        return sum(self.query_lengths)


@dataclass
class _BucketBuffers:
    """Fixed-address per-bucket transaction state: what a captured verify program reads."""
    meta: torch.Tensor          # int32 [4R+1]
    table: torch.Tensor         # int32 [sum Q, 64] cos/sin of the new rows' positions


def _upload(values, device):
    """int32 host list -> device tensor through pinned memory, without blocking the host
    on the stream (a pageable copy could make the host wait for queued GPU work)."""
    host = torch.tensor(values, dtype=torch.int32).pin_memory()
    return host.to(device, non_blocking=True)


def rope_inv_freq(theta, dim=HEAD_DIM, device='cpu'):
    """float32 ``1 / theta ** (arange(0, dim, 2) / dim)`` computed like the transformers
    rotary module (modeling_qwen3.py:124-133), then moved to ``device``."""
    exponent = torch.arange(0, dim, 2, dtype=torch.int64).to(dtype=torch.float) / dim
    return (1.0 / (theta ** exponent)).to(device)


class B200PersistentTargetKV:
    def __init__(self, *, layers, slots, context_capacity, max_query_tokens, heads=HKV, dim=HEAD_DIM,
                 dtype=torch.bfloat16, device='cuda', slot_capacities=None):
        dims = (layers, slots, context_capacity, max_query_tokens, heads, dim)
        if any(type(n) is not int or n < 1 for n in dims):
            raise ValueError('All capacities and dimensions must be positive integers')
        if (heads, dim) != (HKV, HEAD_DIM) or dtype not in (torch.bfloat16, torch.float32):
            raise ValueError('B200 store holds bf16 (or exact-path fp32) Qwen3 KV: 8 heads x 128')
        caps = [context_capacity] * slots if slot_capacities is None else [int(c) for c in slot_capacities]
        if len(caps) != slots or any(c < 1 or c > context_capacity for c in caps):
            raise ValueError('One positive capacity <= context_capacity per slot required')
        self.device = torch.device(device)
        if self.device.index is None:
            self.device = torch.device('cuda', torch.cuda.current_device())
        self.runtime = runtime_identity(self.device)
        self.layers, self.slot_capacity, self.context_capacity = layers, slots, context_capacity
        self.max_query_tokens, self.heads, self.dim, self.dtype = max_query_tokens, heads, dim, dtype
        self.capacities = tuple(caps)
        rows = [0]
        for c in caps:
            rows.append(rows[-1] + c)
        self.slot_rows = tuple(rows[:-1])
        self.rows_per_layer = rows[-1]
        if layers * self.rows_per_layer >= 2 ** 31:
            raise ValueError('Resident rows exceed the int32 row index of the kernels')
        self._keys = torch.zeros((layers * self.rows_per_layer, heads, dim), dtype=dtype, device=self.device)
        self._values = torch.zeros_like(self._keys)
        self.scratch_keys = torch.zeros((layers * max_query_tokens, heads, dim), dtype=dtype, device=self.device)
        self.scratch_values = torch.zeros_like(self.scratch_keys)
        self._table = _SlotTable(slots)
        self._lengths = self._table.length   # committed rows per slot index (host mirror)
        self._sequence = 0
        self._pending = None
        self._staged = set()
        self._buckets = {}
        self._rotary = {}
        self.failed = False

    # -- views -----------------------------------------------------------------
    @property
    def keys(self):
        return self._layer_view(self._keys)

    @property
    def values(self):
        return self._layer_view(self._values)

    def _layer_view(self, x):
        if len(set(self.capacities)) == 1:
            return x.view(self.layers, self.slot_capacity, self.capacities[0], self.heads, self.dim)
        return x.view(self.layers, self.rows_per_layer, self.heads, self.dim)

    def _slot_rows_view(self, x, i, start, n):
        r0 = self.slot_rows[i] + start
        return x.view(self.layers, self.rows_per_layer, self.heads, self.dim)[:, r0:r0 + n]

    # -- slot lifecycle ----------------------------------------------------------
    # Observable contract of the reference store (persistent_target_kv.py:204-265):
    # a store poisoned by a failed copy refuses everything with RuntimeError;
    # admission, removal and prefix loads are refused with RuntimeError while a
    # transaction is open; a bad request id, a full store or a handle that is not
    # the live one for its slot are refused with ValueError.
    def _usable(self, *, idle=False):
        if self.failed:
            raise RuntimeError('store is poisoned by a failed device copy; build a new store')
        if idle and self._pending is not None:
            raise RuntimeError('a verify transaction is open; commit or abort it first')

    def _slot(self, handle):
        self._usable()
        return self._table.index_of(handle)

    def add_request(self, request):
        self._usable(idle=True)
        return self._table.admit(request)

    def remove_request(self, handle):
        """Free the request's slot; its rows stay in memory but no later handle reaches them."""
        self._usable(idle=True)
        self._table.release(self._table.index_of(handle))

    def length(self, handle):
        return self._lengths[self._slot(handle)]

    def handle_of(self, index):
        """The live handle of slot ``index`` (None when the slot is free)."""
        return self._table.holder[index]

    def mirror_lengths(self, handles, lengths):
        """Set the host's committed-length mirror of ``handles`` after the device changed
        the lengths itself (the pipelined decode loop commits from device-side counts)
        or after a caller filled resident rows directly (benchmarks)."""
        self._usable(idle=True)
        indices = [self._slot(h) for h in handles]
        lengths = [int(n) for n in lengths]
        if len(indices) != len(lengths) or any(not 0 <= n <= self.capacities[i] for i, n in zip(indices, lengths)):
            raise ValueError('one length within its slot capacity per handle required')
        for i, n in zip(indices, lengths):
            self._lengths[i] = n

    def _kv(self, keys, values, shape):
        for x in (keys, values):
            if (not isinstance(x, torch.Tensor) or tuple(x.shape) != shape or x.device != self.device
                    or x.dtype != self.dtype or x.requires_grad):
                raise ValueError(f'K/V must be {shape} {self.dtype} tensors on {self.device} without autograd')

    @torch.no_grad()
    def load_prefix(self, handle, keys, values):
        """Bootstrap committed KV [L, n, H, D] into an empty slot."""
        self._usable(idle=True)
        i = self._slot(handle)
        if self._lengths[i]:
            raise ValueError('prefix load needs an empty slot')
        if not isinstance(keys, torch.Tensor) or keys.ndim != 4 or not 0 <= keys.shape[1] <= self.capacities[i]:
            raise ValueError('prefix K/V must be [layers, n, heads, dim] with n within the slot capacity')
        n = keys.shape[1]
        self._kv(keys, values, (self.layers, n, self.heads, self.dim))
        try:
            self._slot_rows_view(self._keys, i, 0, n).copy_(keys)
            self._slot_rows_view(self._values, i, 0, n).copy_(values)
        except Exception:
            self.failed = True
            raise
        self._lengths[i] = n

    # -- fixed-buffer buckets (graph capture; persistent_qwen_graph.py:198-275) ---
    def bind_bucket(self, bucket):
        """Give ``bucket`` (exact ordered ``query_lengths``) fixed-address metadata and
        cos/sin buffers. ``begin(handles, bucket)`` then writes each transaction's
        metadata into those buffers, so a verify program captured once under
        ``capture_transaction(bucket)`` can be replayed for every transaction of the
        bucket. Metadata is still built on the host (as the reference's graph does)."""
        self._usable()
        qlens = tuple(bucket.query_lengths)
        if (not qlens or any(type(q) is not int or q < 1 for q in qlens) or sum(qlens) > self.max_query_tokens
                or len(qlens) > self.slot_capacity):
            raise ValueError('Bucket query lengths must be positive and fit the store')
        if bucket not in self._buckets:
            r, n = len(qlens), sum(qlens)
            self._buckets[bucket] = _BucketBuffers(
                torch.zeros(4 * r + 1, dtype=torch.int32, device=self.device),
                torch.zeros((n, HEAD_DIM // 2), dtype=torch.int32, device=self.device))
        return self._buckets[bucket]

    @torch.no_grad()
    def capture_transaction(self, bucket):
        """Placeholder transaction to capture a verify program under. Its metadata
        is a valid empty-context layout (every request reads only its new rows), so
        warm-up launches are well defined; a capture records launches without running
        them. End it with ``abort``."""
        self._usable(idle=True)
        buffers = self.bind_bucket(bucket)
        qlens = tuple(bucket.query_lengths)
        cu = [0]
        for q in qlens:
            cu.append(cu[-1] + q)
        host = cu + [0] * len(qlens) + [0] * len(qlens) + [min(self.capacities)] * len(qlens)
        buffers.meta.copy_(torch.tensor(host, dtype=torch.int32))
        self._sequence += 1
        tx = Transaction(self._sequence, (), (0,) * len(qlens), qlens, buffers.meta, {}, buffers.table, True)
        self._pending, self._staged = tx, set()
        return tx

    def replayed(self, tx):
        """Record that a captured program wrote every layer's scratch rows for ``tx``
        (a transaction of a bound bucket); ``commit`` then accepts it."""
        self._transaction(tx)
        if tx.table is None or tx.capture:
            raise ValueError('Only a bound-bucket transaction can be replayed')
        self._staged = set(range(self.layers))

    # -- transactions -----------------------------------------------------------
    @torch.no_grad()
    def begin(self, handles, bucket=None, *, query_lengths=None):
        """Metadata for one verify round (persistent_target_kv.py:369-415).

        ``query_lengths`` (or ``bucket.query_lengths``) gives each request's new rows.
        One host->device copy of [cu_q | slot_row | ctx_len | slot_cap] as int32.
        """
        self._usable(idle=True)
        handles = tuple(handles)
        if query_lengths is None:
            if bucket is None:
                raise ValueError('query_lengths or a bucket with query_lengths required')
            query_lengths = bucket.query_lengths
        query_lengths = tuple(query_lengths)
        if not handles or len(query_lengths) != len(handles):
            raise ValueError('One query length per active handle required')
        indices = [self._slot(h) for h in handles]
        if len(set(indices)) != len(indices):
            raise ValueError('Active request slots must be unique')
        contexts = tuple(self._lengths[i] for i in indices)
        if (any(type(q) is not int or q < 1 for q in query_lengths) or sum(query_lengths) > self.max_query_tokens
                or any(c + q > self.capacities[i] for i, c, q in zip(indices, contexts, query_lengths))):
            raise ValueError('Actual context exceeds declared bucket applicability')
        if bucket is not None and hasattr(bucket, 'accepts') and not bucket.accepts(query_lengths, contexts):
            raise ValueError('Actual context exceeds declared bucket applicability')
        cu = [0]
        for q in query_lengths:
            cu.append(cu[-1] + q)
        host = cu + [self.slot_rows[i] for i in indices] + list(contexts) + [self.capacities[i] for i in indices]
        buffers = self._buckets.get(bucket) if bucket is not None else None
        if buffers is not None and query_lengths == tuple(bucket.query_lengths):
            meta, table = buffers.meta, buffers.table
            meta.copy_(torch.tensor(host, dtype=torch.int32).pin_memory(), non_blocking=True)
        else:
            meta, table = _upload(host, self.device), None
        self._sequence += 1
        tx = Transaction(self._sequence, handles, contexts, query_lengths, meta, {}, table)
        self._pending, self._staged = tx, set()
        return tx

    def _transaction(self, tx):
        self._usable()
        if tx is not self._pending:
            raise ValueError('transaction is not the open one of this store (stale, copied or foreign)')
        for h, c in zip(tx.slots, tx.context_lengths):
            if self._lengths[self._slot(h)] != c:
                raise RuntimeError('a request\'s committed length changed while its transaction was open')

    @staticmethod
    def _meta(tx):
        r = len(tx.query_lengths)
        m = tx.meta
        return m[:r + 1], m[r + 1:2 * r + 1], m[2 * r + 1:3 * r + 1], m[3 * r + 1:4 * r + 1]

    def rotary_cache(self, inv_freq):
        """The [context_capacity, 64] cos/sin cache of ``inv_freq`` (``rope_cache``), built
        on the host the first time these frequencies are seen and kept for the store's
        life (every position a verify row can take is below ``context_capacity``)."""
        key = (inv_freq.data_ptr(), inv_freq._version)
        cache = self._rotary.get(key)
        if cache is None:
            cache = rope_cache(inv_freq, self.context_capacity, self.device)
            self._rotary[key] = cache
        return cache

    @torch.no_grad()
    def verify_layer(self, tx, layer, q_raw, k_raw, v_raw, q_norm_weight, k_norm_weight, *, inv_freq,
                     eps=1e-6, scale=SCALE, out=None, path='auto'):
        """Fused verify for one decoder layer; returns attention output [sum Q, 16, 128].

        ``q_raw``/``k_raw``/``v_raw`` are the layer's q/k/v projections of the new
        tokens before q_norm/k_norm/RoPE ([sum Q, 16|8, 128] bf16); norm weights [128]
        bf16; ``inv_freq`` [64] float32 on this device (see ``rope_inv_freq``).
        ``path``: 'fused' (norm/RoPE/append inside the attention kernel), 'prep' (a
        prep kernel per layer, then the attention kernel) or 'auto' (prep below 512
        new rows or for chunks longer than 16 rows); all give the same values.
        q/k/v may be row-strided views (heads and head dims packed, row stride a
        multiple of 8), e.g. column blocks of one merged q|k|v projection; strided
        rows take the prep path.
        """
        self._transaction(tx)
        if type(layer) is not int or not 0 <= layer < self.layers or layer in self._staged:
            raise ValueError('Each model layer must stage exactly once')
        n = tx.query_tokens
        if scale != SCALE:
            raise ValueError('B200 verify requires the 1/sqrt(128) scale')
        if self.dtype != torch.bfloat16:
            raise ValueError('The fused verify layer is bf16; use stage_layer + attend on a float32 store')
        for x, shape in ((q_raw, (n, HQ, HEAD_DIM)), (k_raw, (n, HKV, HEAD_DIM)), (v_raw, (n, HKV, HEAD_DIM)),
                         (q_norm_weight, (HEAD_DIM,)), (k_norm_weight, (HEAD_DIM,))):
            if (not isinstance(x, torch.Tensor) or tuple(x.shape) != shape or x.dtype != self.dtype
                    or x.device != self.device):
                raise ValueError('Verify inputs must be bf16 q/k/v projections and norm weights')
            if len(shape) == 1:
                ok = x.is_contiguous()
            else:                                   # rows may be strided, each row's heads packed
                ok = (x.stride(2) == 1 and x.stride(1) == HEAD_DIM
                      and (n == 1 or (x.stride(0) >= shape[1] * HEAD_DIM and x.stride(0) % 8 == 0)))
            if not ok:
                raise ValueError('Verify q/k/v rows must hold packed heads (row stride a multiple of 8)')
        lds = [x.stride(0) if n > 1 else x.shape[1] * HEAD_DIM for x in (q_raw, k_raw, v_raw)]
        if (not isinstance(inv_freq, torch.Tensor) or inv_freq.shape != (HEAD_DIM // 2,)
                or inv_freq.dtype != torch.float32 or inv_freq.device != self.device):
            raise ValueError('inv_freq must be float32 [64] on the store device')
        if out is None:
            out = torch.empty((n, HQ, HEAD_DIM), dtype=self.dtype, device=self.device)
        cu_q, slot_row, ctx, _cap = self._meta(tx)
        stream = torch.cuda.current_stream(self.device).cuda_stream
        lib = _lib.load_library()
        key = (inv_freq.data_ptr(), inv_freq._version)
        table = tx.rope.get(key)
        if table is None:
            # cos/sin of every new row's position, gathered once for all layers of this
            # transaction from the rotary cache of these frequencies
            table = rope_table(self.rotary_cache(inv_freq), cu_q, ctx, len(tx.query_lengths), n, out=tx.table)
            tx.rope.clear()
            tx.rope[key] = table
        ws = _lib.workspace(self.device, stream)
        _lib.check(lib.dspark_verify_strided(
            q_raw.data_ptr(), lds[0], k_raw.data_ptr(), lds[1], v_raw.data_ptr(), lds[2], q_norm_weight.data_ptr(),
            k_norm_weight.data_ptr(), table.data_ptr(), float(eps), cu_q.data_ptr(), slot_row.data_ptr(),
            ctx.data_ptr(), len(tx.query_lengths), n, max(tx.query_lengths), self._keys.data_ptr(),
            self._values.data_ptr(),
            self.rows_per_layer, self.scratch_keys.data_ptr(), self.scratch_values.data_ptr(),
            self.max_query_tokens, self.layers, layer, float(scale), _lib.VERIFY_PATHS[path], out.data_ptr(),
            ws.data_ptr(), ws.numel(), stream), 'dspark_verify_strided')
        self._staged.add(layer)
        return out

    @torch.no_grad()
    def stage_layer(self, tx, layer, keys, values):
        """Copy already-roped new K/V [sum Q, H, D] into scratch (persistent_target_kv.py:427-438)."""
        self._transaction(tx)
        if type(layer) is not int or not 0 <= layer < self.layers or layer in self._staged:
            raise ValueError('Each model layer must stage exactly once')
        q = tx.query_tokens
        self._kv(keys, values, (q, self.heads, self.dim))
        base = layer * self.max_query_tokens
        self.scratch_keys[base:base + q].copy_(keys)
        self.scratch_values[base:base + q].copy_(values)
        self._staged.add(layer)

    @torch.no_grad()
    def attend(self, tx, layer, query, *, scale=SCALE):
        """Bottom-right causal attention of already-roped ``query`` over resident prefix +
        staged scratch rows, read in place (the unfused counterpart of ``verify_layer``)."""
        from .kernels import segment_attention
        self._transaction(tx)
        if layer not in self._staged:
            raise ValueError('Layer scratch missing')
        cu_q, slot_row, ctx, _cap = self._meta(tx)
        rpl, sr = self.rows_per_layer, self.max_query_tokens
        return segment_attention(query, cu_q, tx.query_lengths,
                                 self._keys[layer * rpl:(layer + 1) * rpl], self._values[layer * rpl:(layer + 1) * rpl],
                                 slot_row, ctx, self.scratch_keys[layer * sr:(layer + 1) * sr],
                                 self.scratch_values[layer * sr:(layer + 1) * sr], causal=True, scale=scale)

    @torch.no_grad()
    def prepare_attention(self, tx, layer, key_capacity=None):
        """Audit path: gathered [capacity, H, D] K/V with a zero tail, cu_query, cu_key and
        positions, as the reference's workspace holds them (persistent_target_kv.py:441-460).
        The verify kernels never need this copy."""
        self._transaction(tx)
        if layer not in self._staged:
            raise ValueError('Layer scratch missing')
        q = tx.query_tokens
        logical = sum(tx.context_lengths) + q
        cap = logical if key_capacity is None else key_capacity
        if cap < logical:
            raise ValueError('Key capacity below active keys')
        keys = torch.zeros((cap, self.heads, self.dim), dtype=self.dtype, device=self.device)
        values = torch.zeros_like(keys)
        ck, positions, o, qo = [0], [], 0, 0
        base = layer * self.max_query_tokens
        for h, c, n in zip(tx.slots, tx.context_lengths, tx.query_lengths):
            i = h.index
            keys[o:o + c] = self._slot_rows_view(self._keys, i, 0, c)[layer]
            values[o:o + c] = self._slot_rows_view(self._values, i, 0, c)[layer]
            keys[o + c:o + c + n] = self.scratch_keys[base + qo:base + qo + n]
            values[o + c:o + c + n] = self.scratch_values[base + qo:base + qo + n]
            positions.extend(range(c, c + n))
            o += c + n
            qo += n
            ck.append(o)
        cu_q = self._meta(tx)[0]
        return (keys, values, cu_q, torch.tensor(ck, dtype=torch.int32, device=self.device),
                torch.tensor(positions, dtype=torch.long, device=self.device))

    @torch.no_grad()
    def commit(self, tx, committed_query_lengths: Mapping):
        """Commit caller-decided verified prefixes, anchor included (persistent_target_kv.py:463-491)."""
        self._transaction(tx)
        if tx.capture:
            raise ValueError('A capture placeholder transaction cannot commit')
        if set(committed_query_lengths) != set(tx.slots) or len(self._staged) != self.layers:
            raise ValueError('Complete layer scratch and one prefix count per active handle required')
        counts = []
        for h, c, q in zip(tx.slots, tx.context_lengths, tx.query_lengths):
            n = committed_query_lengths[h]
            if type(n) is not int or not 0 <= n <= q or c + n > self.capacities[h.index]:
                raise ValueError('Commit must be a valid verified prefix')
            counts.append(n)
        try:
            ncommit = _upload(counts, self.device)
            cu_q, slot_row, ctx, cap = self._meta(tx)
            stream = torch.cuda.current_stream(self.device).cuda_stream
            _lib.check(_lib.load_library().dspark_commit_kv(
                self._keys.data_ptr(), self._values.data_ptr(), self.scratch_keys.data_ptr(),
                self.scratch_values.data_ptr(), cu_q.data_ptr(), slot_row.data_ptr(), ctx.data_ptr(),
                cap.data_ptr(), ncommit.data_ptr(), len(tx.slots), self.layers, self.rows_per_layer,
                self.max_query_tokens, _lib.DTYPE_F32 if self.dtype == torch.float32 else _lib.DTYPE_BF16, stream),
                'dspark_commit_kv')
            for h, n in zip(tx.slots, counts):
                self._lengths[h.index] += n
        except Exception:
            self.failed = True
            raise
        self._pending, self._staged = None, set()
        return dict(committed_tokens=sum(counts),
                    copied_kv_bytes=2 * self.layers * self.heads * self.dim * self._keys.element_size() * sum(counts))

    def abort(self, tx):
        """Drop the transaction; scratch rows are simply never copied (persistent_target_kv.py:493-499)."""
        self._transaction(tx)
        self._pending, self._staged = None, set()

    def request_kv(self, handle):
        i = self._slot(handle)
        n = self._lengths[i]
        return (self._slot_rows_view(self._keys, i, 0, n).clone(), self._slot_rows_view(self._values, i, 0, n).clone())

    def pointers(self):
        return dict(committed_keys=self._keys.data_ptr(), committed_values=self._values.data_ptr(),
                    scratch_keys=self.scratch_keys.data_ptr(), scratch_values=self.scratch_values.data_ptr())

    def work(self, tx):
        self._transaction(tx)
        q = tx.query_tokens
        actual_k = sum(tx.context_lengths) + q
        kv_row = 2 * self.heads * self.dim * self._keys.element_size()
        return dict(active_requests=len(tx.slots), logical_query_tokens=q, physical_query_tokens=q,
                    logical_active_key_tokens=actual_k, physical_key_capacity=actual_k, padded_key_capacity=0,
                    inactive_resident_key_tokens=sum(self._lengths) - sum(tx.context_lengths),
                    gather_rows_per_kv_per_layer=0, staging_output_rows_per_layer=0,
                    attention_kv_bytes_per_layer=actual_k * kv_row,
                    allowed_causal_pairs=sum(c * n + n * (n + 1) // 2
                                             for c, n in zip(tx.context_lengths, tx.query_lengths)),
                    query_lengths=list(tx.query_lengths), queried_context_lengths=list(tx.context_lengths),
                    resident_allocated_kv_bytes=2 * self._keys.numel() * self._keys.element_size(),
                    scratch_allocated_kv_bytes=2 * self.scratch_keys.numel() * self._keys.element_size())
