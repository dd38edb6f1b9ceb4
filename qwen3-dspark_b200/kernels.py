"""Drop-in attention kernels with the reference's plugin signature.

Every class is callable as ``kernel(query, key, value, layout, *, scale) -> out``
(the boundary of dspark_qwen/packed_draft.py:23, rocm_varlen.py:108 and
persistent_qwen_target.py:223) and carries ``backend_name`` and
``native_varlen_calls_per_layer = 1``. Inputs are validated on the host before
any launch with the refusals of ``PinnedRocmVarlenKernel._validate_inputs``
(rocm_varlen.py:65-106); a launch error propagates as ``RuntimeError``; there is
no fallback, retry or split tuning.

* ``B200VarlenKernel``  - bottom-right causal, exact K (replaces PinnedRocmVarlenKernel)
* ``B200DraftKernel``   - non-causal (replaces PinnedRocmDraftKernel)
* ``B200CapacityKernel`` - bottom-right causal over a capacity-sized K whose tail
  past ``cu_key[-1]`` is never read (replaces PersistentQwenTarget._native_attention)
* ``B200TrainingLayoutKernel`` - the training-layout draft attention of
  ``DraftAttention.forward`` + ``block_mask`` (model.py:12-19,47-61) for packed
  sequences, on the tcgen05 tensor cores

bf16 runs on the tensor-core kernel; float32 inputs (the reference's exact CPU
configurations) run on the library's float32 CUDA-core kernel.
"""
import math

import numpy as np

import torch

from . import _lib

BACKEND = 'b200_sm100a_varlen_causal_v1'
DRAFT_BACKEND = 'b200_sm100a_noncausal_v1'
CAPACITY_BACKEND = 'b200_sm100a_capacity_causal_v1'
TRAIN_BACKEND = 'b200_sm100a_train_layout_tcgen05_v1'
HQ, HKV, HEAD_DIM = 16, 8, 128
SCALE = HEAD_DIM ** -0.5
_DTYPES = {torch.bfloat16: _lib.DTYPE_BF16, torch.float32: _lib.DTYPE_F32}


def runtime_identity(device):
    """The native runtime this kernel binds to; refuses anything but an sm_100 CUDA GPU."""
    if device.type != 'cuda' or not torch.cuda.is_available():
        raise RuntimeError('B200 attention requires an explicitly selected CUDA GPU; no CPU fallback')
    major, minor = torch.cuda.get_device_capability(device)
    if major != 10:
        raise RuntimeError(f'B200 attention is built for sm_100a only; device has sm_{major}{minor}')
    return dict(torch=torch.__version__, cuda=torch.version.cuda, device=torch.cuda.get_device_name(device),
                capability=(major, minor), library_abi=_lib.load_library().dspark_abi_version())


def _stream(device):
    return torch.cuda.current_stream(device).cuda_stream


class _NativeEntry:
    """Calls one C-ABI attention entry; replaceable by a test double on CPU."""

    def __init__(self, name):
        self.name = name

    def __call__(self, *args):
        _lib.check(getattr(_lib.load_library(), self.name)(*args), self.name)


class B200VarlenKernel:
    """Bottom-right causal packed varlen attention (exact-K contract of rocm_varlen.py:42-117)."""
    backend_name = BACKEND
    native_varlen_calls_per_layer = 1
    causal = True
    entry = 'dspark_varlen_attn'

    def __init__(self, device):
        self.device = torch.device(device)
        if self.device.type == 'cuda' and self.device.index is None:
            self.device = torch.device('cuda', torch.cuda.current_device())
        self.runtime = runtime_identity(self.device)
        self._operator = _NativeEntry(self.entry)
        self._validated_layout = None
        self._layout_versions = None

    # -- validation (mirrors rocm_varlen.py:65-106) -------------------------
    def _check_tensors(self, query, key, value, scale):
        tensors = (query, key, value)
        if any(not isinstance(t, torch.Tensor) or not t.is_cuda or t.device != self.device
               or t.dtype not in _DTYPES or t.dtype != query.dtype or t.requires_grad or t.ndim != 3
               or not t.is_contiguous() for t in tensors):
            raise ValueError('B200 varlen requires no-autograd contiguous BF16 (or FP32) THD tensors on its GPU')
        if (query.shape[1:] != (HQ, HEAD_DIM) or key.shape[1:] != (HKV, HEAD_DIM)
                or value.shape != key.shape or query.shape[0] == 0 or key.shape[0] == 0):
            raise ValueError('B200 varlen supports nonempty Hq16/Hkv8/D128 Qwen tensors only')
        if not isinstance(scale, (float, int)) or not math.isfinite(scale) or scale != SCALE:
            raise ValueError('B200 varlen requires the 1/sqrt(128) scale')

    def _check_layout(self, layout, key_rows_expected, key):
        for name in ('query_lengths', 'key_lengths', 'cu_query', 'cu_key'):
            if not hasattr(layout, name):
                raise ValueError('B200 varlen requires a packed layout')
        cu = (layout.cu_query, layout.cu_key)
        if any(not isinstance(t, torch.Tensor) or t.device != self.device or t.dtype != torch.int32
               or t.ndim != 1 or not t.is_contiguous() for t in cu):
            raise ValueError('B200 varlen requires contiguous int32 cumulative lengths on its GPU')
        if key.shape[0] != key_rows_expected:
            raise ValueError('Tensor token dimensions differ from packed layout')
        try:
            versions = tuple(t._version for t in cu)
        except RuntimeError:
            versions = None      # inference tensors: revalidate every call
        if versions is not None and layout is self._validated_layout and versions == self._layout_versions:
            return
        qs, ks = layout.query_lengths, layout.key_lengths
        markers = getattr(layout, 'request_markers', tuple(range(len(qs))))
        if (not qs or len(qs) != len(ks) or len(markers) != len(qs) or len(set(markers)) != len(qs)
                or any(type(q) is not int or type(k) is not int or not 0 < q <= k for q, k in zip(qs, ks))):
            raise ValueError('Invalid packed lengths/markers for bottom-right causal suffixes')
        if layout.cu_query.tolist() != _cumulative(qs) or layout.cu_key.tolist() != _cumulative(ks):
            raise ValueError('Cumulative lengths differ from packed metadata')
        self._validated_layout, self._layout_versions = layout, versions

    def _validate_inputs(self, query, key, value, layout, scale):
        self._check_tensors(query, key, value, scale)
        for name in ('query_lengths', 'key_lengths'):
            if not hasattr(layout, name):
                raise ValueError('B200 varlen requires a packed layout')
        if query.shape[0] != sum(layout.query_lengths):
            raise ValueError('Tensor token dimensions differ from packed layout')
        self._check_layout(layout, sum(layout.key_lengths), key)

    def __call__(self, query, key, value, layout, *, scale):
        self._validate_inputs(query, key, value, layout, scale)
        return self._launch(query, key, value, layout, scale)

    def _launch(self, query, key, value, layout, scale):
        out = torch.empty_like(query)
        ws = _lib.workspace(self.device, _stream(self.device))
        self._operator(query.data_ptr(), key.data_ptr(), value.data_ptr(), layout.cu_query.data_ptr(),
                       layout.cu_key.data_ptr(), len(layout.query_lengths), query.shape[0], key.shape[0],
                       max(layout.query_lengths), max(layout.key_lengths), float(scale), _DTYPES[query.dtype],
                       out.data_ptr(), ws.data_ptr(), ws.numel(), _stream(self.device))
        if out.shape != query.shape or out.dtype != query.dtype or out.device != query.device:
            raise RuntimeError('B200 varlen returned incompatible output')
        return out


class B200DraftKernel(B200VarlenKernel):
    """Non-causal packed varlen attention for the draft block (packed_draft.py:19-32)."""
    backend_name = DRAFT_BACKEND
    causal = False
    entry = 'dspark_draft_attn'


class B200CapacityKernel(B200VarlenKernel):
    """Capacity-tail verify attention (persistent_qwen_target.py:223-234).

    ``len(key) == layout.physical_key_capacity``; rows past ``cu_key[-1]`` are
    never read, so a NaN or stale tail cannot reach the output.
    """
    backend_name = CAPACITY_BACKEND

    def _validate_inputs(self, query, key, value, layout, scale):
        self._check_tensors(query, key, value, scale)
        cap = getattr(layout, 'physical_key_capacity', None)
        if (query.dtype != torch.bfloat16 or type(cap) is not int or len(key) != cap
                or len(query) != sum(layout.query_lengths) or sum(layout.key_lengths) > cap):
            raise ValueError('B200 capacity attention shape/dtype/scale differs')
        self._check_layout(layout, cap, key)


class B200TrainingLayoutKernel:
    """Training-layout draft attention for packed sequences (model.py:12-19,47-61).

    ``kernel(query, key, value, layout, *, scale)`` with a ``TrainingLayout``:
    query [sum blocks*block_size, 16, 128], key/value [sum(context + block rows),
    8, 128], contiguous, one dtype. bf16 runs the tcgen05 kernel
    (``dspark_train_attn``) over the layout's device plan; float32 (the exact
    configuration) runs each block as a two-segment request of the float32
    CUDA-core kernel.
    """
    backend_name = TRAIN_BACKEND
    native_varlen_calls_per_layer = 1

    def __init__(self, device):
        self.device = torch.device(device)
        if self.device.type == 'cuda' and self.device.index is None:
            self.device = torch.device('cuda', torch.cuda.current_device())
        self.runtime = runtime_identity(self.device)
        self._operator = _NativeEntry('dspark_train_attn')

    def __call__(self, query, key, value, layout, *, scale):
        tensors = (query, key, value)
        if any(not isinstance(t, torch.Tensor) or t.device != self.device or t.dtype not in _DTYPES
               or t.dtype != query.dtype or t.requires_grad or t.ndim != 3 or not t.is_contiguous()
               for t in tensors):
            raise ValueError('B200 training layout requires no-autograd contiguous BF16 (or FP32) THD tensors '
                             'on its GPU')
        if query.shape[1:] != (HQ, HEAD_DIM) or key.shape[1:] != (HKV, HEAD_DIM) or value.shape != key.shape:
            raise ValueError('B200 training layout supports Hq16/Hkv8/D128 Qwen tensors only')
        if not isinstance(scale, (float, int)) or not math.isfinite(scale) or scale != SCALE:
            raise ValueError('B200 training layout requires the 1/sqrt(128) scale')
        if (not hasattr(layout, 'plan') or len(query) != layout.query_tokens or len(key) != layout.key_tokens
                or layout.plan.device != self.device):
            raise ValueError('Query/key rows must match the training layout on this device')
        if query.dtype == torch.float32:
            return segment_attention(query, layout.seg_cu_query, [layout.block_size] * (len(layout.seg_a_len)),
                                     key, value, layout.seg_a_start, layout.seg_a_len, key, value,
                                     layout.seg_b_start, layout.seg_b_len, causal=False, scale=scale)
        out = torch.empty_like(query)
        self._operator(query.data_ptr(), key.data_ptr(), value.data_ptr(), query.shape[0], key.shape[0],
                       layout.plan.data_ptr(), layout.grid, float(scale), out.data_ptr(), _stream(self.device))
        return out


def _cumulative(lengths):
    out = [0]
    for n in lengths:
        out.append(out[-1] + n)
    if out[-1] >= 2 ** 31:
        raise ValueError('Packed cumulative length exceeds int32')
    return out


def segment_attention(query, cu_query, query_lengths, key_a, value_a, a_start, a_len, key_b=None, value_b=None,
                      b_start=None, b_len=None, *, causal, scale=SCALE, a_off=0, b_off=0, out=None):
    """Attention whose keys are two row ranges per request, read in place (no gather copy).

    Keys of request i: rows ``[a_off + a_start[i], + a_len[i])`` of ``key_a``/``value_a``
    then rows ``[b_off + b_start[i], + b_len[i])`` of ``key_b``/``value_b``. Used for the
    draft context cache + block rows (packed_draft.py:215-236), the resident prefix +
    verify scratch (persistent_target_kv.py:441-460) and the training layout, where each
    anchor block reads context rows [0, anchor) plus its own block (model.py:12-19).
    All index tensors are int32 on the query's device.
    """
    device = query.device
    if not query.is_cuda:
        raise RuntimeError('segment_attention requires CUDA tensors; no CPU fallback')
    tensors = [query, key_a, value_a] + ([key_b, value_b] if key_b is not None else [])
    if any(t.dtype != query.dtype or t.dtype not in _DTYPES or not t.is_contiguous() or t.device != device
           for t in tensors):
        raise ValueError('segment_attention requires contiguous same-dtype bf16/fp32 tensors on one device')
    if query.shape[1:] != (HQ, HEAD_DIM) or key_a.shape[1:] != (HKV, HEAD_DIM) or value_a.shape != key_a.shape:
        raise ValueError('segment_attention supports Hq16/Hkv8/D128 only')
    if key_b is not None and (key_b.shape[1:] != (HKV, HEAD_DIM) or value_b.shape != key_b.shape):
        raise ValueError('segment_attention supports Hq16/Hkv8/D128 only')
    ints = [cu_query, a_start, a_len] + [x for x in (b_start, b_len) if x is not None]
    if any(x.dtype != torch.int32 or x.device != device or not x.is_contiguous() for x in ints):
        raise ValueError('segment_attention index tensors must be contiguous int32 on the query device')
    if out is None:
        out = torch.empty_like(query)
    ws = _lib.workspace(device, _stream(device))
    nul = lambda t: t.data_ptr() if t is not None else None  # noqa: E731
    _lib.check(_lib.load_library().dspark_segment_attn(
        query.data_ptr(), key_a.data_ptr(), value_a.data_ptr(), key_a.shape[0], nul(key_b), nul(value_b),
        key_b.shape[0] if key_b is not None else 0, cu_query.data_ptr(), a_start.data_ptr(), a_len.data_ptr(),
        nul(b_start), nul(b_len), int(a_off), int(b_off), cu_query.numel() - 1, query.shape[0],
        max(query_lengths), int(bool(causal)), float(scale), _DTYPES[query.dtype], out.data_ptr(),
        ws.data_ptr(), ws.numel(), _stream(device)), 'dspark_segment_attn')
    return out


def rms_norm(x, weight, eps):
    """``Qwen3RMSNorm.forward`` of bf16 ``x`` [..., hidden] with bf16 ``weight`` [hidden]
    in one launch (transformers models/qwen3/modeling_qwen3.py:62-66; the reference
    runs it as eight torch kernels). Same shape and dtype as ``x``; each step rounds as
    the torch sequence does, only the float sum of squares is associated differently.
    """
    hidden = x.shape[-1]
    if (x.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16 or not x.is_cuda
            or weight.device != x.device or weight.shape != (hidden,) or hidden % 8 != 0):
        raise ValueError('bf16 x [..., hidden] and weight [hidden] on one CUDA device, hidden % 8 == 0 required')
    rows = x.reshape(-1, hidden)
    if rows.stride(-1) != 1 or rows.stride(0) % 8 != 0 or rows.data_ptr() % 16 != 0:
        rows = rows.contiguous()
    w = weight if weight.stride(0) == 1 and weight.data_ptr() % 16 == 0 else weight.contiguous()
    out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    _lib.check(_lib.load_library().dspark_rms_norm(rows.data_ptr(), max(rows.stride(0), hidden), w.data_ptr(),
                                                   float(eps), rows.shape[0], hidden, out.data_ptr(), hidden,
                                                   _stream(x.device)), 'dspark_rms_norm')
    return out


def add_rms_norm(x, delta, weight, eps):
    """Residual add + ``Qwen3RMSNorm`` in one launch: returns ``(s, rms_norm(s))`` with
    ``s = x + delta`` rounded to bf16 as torch's add rounds (same shapes as ``x``)."""
    hidden = x.shape[-1]
    if (x.dtype != torch.bfloat16 or delta.dtype != torch.bfloat16 or weight.dtype != torch.bfloat16
            or delta.shape != x.shape or not x.is_cuda or delta.device != x.device or weight.device != x.device
            or weight.shape != (hidden,) or hidden % 8 != 0):
        raise ValueError('bf16 x and delta [..., hidden] and weight [hidden] on one CUDA device, hidden % 8 == 0 '
                         'required')
    rows = [t.reshape(-1, hidden) for t in (x, delta)]
    rows = [r if r.stride(-1) == 1 and r.stride(0) % 8 == 0 and r.data_ptr() % 16 == 0 else r.contiguous()
            for r in rows]
    w = weight if weight.stride(0) == 1 and weight.data_ptr() % 16 == 0 else weight.contiguous()
    out = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    total = torch.empty(x.shape, dtype=torch.bfloat16, device=x.device)
    n = rows[0].shape[0]
    _lib.check(_lib.load_library().dspark_add_rms_norm(
        rows[0].data_ptr(), max(rows[0].stride(0), hidden), rows[1].data_ptr(), max(rows[1].stride(0), hidden),
        w.data_ptr(), float(eps), n, hidden, out.data_ptr(), hidden, total.data_ptr(), hidden,
        _stream(x.device)), 'dspark_add_rms_norm')
    return total, out


def qk_norm_rope(q, k, q_norm_weight, k_norm_weight, q_eps, k_eps, cos, sin, q_heads, kv_heads):
    """The draft block's q/k head RMSNorm + rotate-half RoPE (model.py:41-45, 22-24) in
    one launch: ``q`` [n, q_heads * 128] and ``k`` [n, kv_heads * 128] bf16 rows (unit
    column stride), ``cos`` / ``sin`` [n, 128] the rotary module's bf16 tables. Returns
    packed (q [n, q_heads, 128], k [n, kv_heads, 128]), rounded as torch's bf16 ops."""
    n = q.shape[0]
    ok = (q.ndim == k.ndim == cos.ndim == sin.ndim == 2 and k.shape[0] == cos.shape[0] == sin.shape[0] == n
          and q.shape[1] == q_heads * HEAD_DIM and k.shape[1] == kv_heads * HEAD_DIM
          and cos.shape[1] == sin.shape[1] == HEAD_DIM and cos.stride() == sin.stride()
          and all(t.dtype == torch.bfloat16 and t.is_cuda and t.device == q.device
                  for t in (q, k, cos, sin, q_norm_weight, k_norm_weight))
          and q_norm_weight.shape == k_norm_weight.shape == (HEAD_DIM,))
    if not ok:
        raise ValueError('bf16 q [n, Hq*128], k [n, Hkv*128], cos/sin [n, 128] and 128-wide norm weights on one '
                         'CUDA device required')
    q, k, cos, sin = (t if t.stride(-1) == 1 else t.contiguous() for t in (q, k, cos, sin))
    qw, kw = q_norm_weight.contiguous(), k_norm_weight.contiguous()
    q_out = torch.empty((n, q_heads, HEAD_DIM), dtype=torch.bfloat16, device=q.device)
    k_out = torch.empty((n, kv_heads, HEAD_DIM), dtype=torch.bfloat16, device=q.device)
    ld = lambda t: max(t.stride(0), t.shape[1])  # noqa: E731  (a single row may carry any stride)
    _lib.check(_lib.load_library().dspark_qk_norm_rope(
        q.data_ptr(), ld(q), k.data_ptr(), ld(k), qw.data_ptr(), kw.data_ptr(), float(q_eps), float(k_eps),
        cos.data_ptr(), sin.data_ptr(), ld(cos), n, q_heads, kv_heads, q_out.data_ptr(), k_out.data_ptr(),
        _stream(q.device)), 'dspark_qk_norm_rope')
    return q_out, k_out


def silu_mul(gate_up, inter):
    """``act_fn(gate) * up`` of a Qwen3MLP from one merged projection ``gate_up``
    [..., 2 * inter] bf16 (gate columns first); returns [..., inter] bf16, rounded as
    torch's silu kernel and bf16 product round."""
    if (gate_up.dtype != torch.bfloat16 or not gate_up.is_cuda or gate_up.shape[-1] != 2 * inter
            or inter % 8 != 0 or inter < 8):
        raise ValueError('bf16 gate_up [..., 2 * inter] on a CUDA device with inter % 8 == 0 required')
    rows = gate_up.reshape(-1, 2 * inter)
    if rows.stride(-1) != 1 or rows.stride(0) % 8 != 0 or rows.data_ptr() % 16 != 0:
        rows = rows.contiguous()
    out = torch.empty(gate_up.shape[:-1] + (inter,), dtype=torch.bfloat16, device=gate_up.device)
    _lib.check(_lib.load_library().dspark_silu_mul(rows.data_ptr(), max(rows.stride(0), 2 * inter), rows.shape[0],
                                                   inter, out.data_ptr(), inter, _stream(gate_up.device)),
               'dspark_silu_mul')
    return out


def merged_mlp_ready(mlp):
    """A bf16 Qwen3MLP whose gate/up projections can run as one GEMM + ``silu_mul``."""
    g, u = mlp.gate_proj, mlp.up_proj
    return (g.bias is None and u.bias is None and g.weight.dtype == u.weight.dtype == torch.bfloat16
            and g.weight.shape == u.weight.shape and g.out_features % 8 == 0
            and (type(mlp.act_fn).__name__ == 'SiLUActivation' or type(mlp.act_fn) is torch.nn.SiLU))


def greedy_accept(logits, tokens, cu_query, eos_ids=(), budget=None):
    """Greedy acceptance of one verify round on the GPU (cached_decode.py:84-98).

    ``logits`` [N, vocab] (bf16/fp32) are the target's logits of the N verified rows,
    ``tokens`` [N] int64 the verified chunk tokens (per request: anchor, proposals),
    ``eos_ids`` the stop tokens (an iterable, or an int64 device tensor, which avoids a
    host-to-device copy per call),
    ``cu_query`` int32 [R+1] the request boundaries. ``budget`` (optional, int32 [R])
    caps each request's committed tokens. Returns device tensors
    ``(pred [N] int32, accepted [R] int32, n_commit [R] int32, emitted [N] int64)``
    with ``emitted[cu_query[i] + k]`` the committed tokens of request i (-1 after).
    """
    device = logits.device
    if (logits.ndim != 2 or logits.dtype not in _DTYPES or logits.stride(1) != 1 or not logits.is_cuda
            or tokens.shape != (logits.shape[0],) or tokens.dtype != torch.long or tokens.device != device
            or cu_query.dtype != torch.int32 or cu_query.device != device or cu_query.ndim != 1
            or cu_query.numel() < 2):
        raise ValueError('logits [N,V] bf16/fp32 (unit column stride), tokens [N] int64 and int32 cu_query '
                         'on one CUDA device required')
    r = cu_query.numel() - 1
    if isinstance(eos_ids, torch.Tensor):
        if eos_ids.dtype != torch.long or eos_ids.device != device or eos_ids.ndim != 1:
            raise ValueError('eos_ids tensor must be int64 [n] on the logits device')
        eos = eos_ids.contiguous()
    else:
        eos = torch.tensor(sorted(set(int(e) for e in eos_ids)), dtype=torch.long, device=device)
    if budget is not None and (budget.shape != (r,) or budget.dtype != torch.int32 or budget.device != device):
        raise ValueError('budget must be int32 [R] on the logits device')
    n = logits.shape[0]
    pred = torch.empty(n, dtype=torch.int32, device=device)
    counts = torch.empty(2 * r, dtype=torch.int32, device=device)
    emitted = torch.empty(n, dtype=torch.long, device=device)
    lib, stream = _lib.load_library(), _stream(device)
    _lib.check(lib.dspark_row_argmax(logits.data_ptr(), logits.stride(0), n, logits.shape[1], _DTYPES[logits.dtype],
                                     pred.data_ptr(), stream), 'dspark_row_argmax')
    _lib.check(lib.dspark_greedy_accept(pred.data_ptr(), tokens.data_ptr(), cu_query.contiguous().data_ptr(), r, n,
                                        eos.data_ptr() if eos.numel() else None, eos.numel(),
                                        budget.data_ptr() if budget is not None else None, counts.data_ptr(),
                                        counts[r:].data_ptr(), emitted.data_ptr(), stream), 'dspark_greedy_accept')
    return pred, counts[:r], counts[r:], emitted


_markov_scratch = {}


def markov_greedy(proj_weight, emb_table, conf_weight, conf_bias, hidden, base, anchors, block_size):
    """Serial greedy Markov proposal of one draft block for every request on the
    GPU (DSparkDraft._sample_greedy, dspark_qwen/model.py:210-221), one fused
    tcgen05 kernel: all positions in one cooperative launch (``dspark_markov_block``),
    or one launch per position (``dspark_markov_step``) for blocks over 64.

    ``proj_weight``/``emb_table`` [V, rank] bf16 (markov_projection.weight /
    markov_embedding.weight), ``conf_weight`` [H + rank] bf16, ``conf_bias`` a float,
    ``hidden`` [R * block_size, H] bf16, ``base`` = lm_head(hidden) [R * block_size, V]
    bf16, ``anchors`` [R] int64. Returns device tensors ``tokens`` [R, block_size]
    int64 and ``conf`` [R, block_size] float32.
    """
    device = hidden.device
    v, rank = proj_weight.shape
    r = anchors.numel()
    h = hidden.shape[1]
    for x in (proj_weight, emb_table, conf_weight, hidden, base):
        if x.dtype != torch.bfloat16 or not x.is_contiguous() or x.device != device:
            raise ValueError('Markov proposal operands must be contiguous bf16 on one device')
    if (emb_table.shape != (v, rank) or conf_weight.shape != (h + rank,) or hidden.shape != (r * block_size, h)
            or base.shape != (r * block_size, v) or anchors.dtype != torch.long or anchors.device != device):
        raise ValueError('Markov proposal shapes do not match')
    # the packed maxima / arrival counter are shared by the calls on one stream (they
    # run in order); another stream gets its own, so concurrent calls cannot race
    key = (device.index, _stream(device))
    if key not in _markov_scratch:
        _markov_scratch[key] = torch.zeros(int(_lib.load_library().dspark_markov_scratch_bytes()),
                                           dtype=torch.uint8, device=device)
    scratch = _markov_scratch[key]
    tokens = torch.empty((r, block_size), dtype=torch.long, device=device)
    conf = torch.empty((r, block_size), dtype=torch.float32, device=device)
    anchors = anchors.contiguous()
    lib, stream = _lib.load_library(), _stream(device)
    for r0 in range(0, r, 128):
        n = min(128, r - r0)
        if block_size <= 64:
            # every position of the block in one cooperative launch
            _lib.check(lib.dspark_markov_block(
                proj_weight.data_ptr(), emb_table.data_ptr(), v, rank, base[r0 * block_size:].data_ptr(), block_size,
                anchors[r0:].data_ptr(), hidden[r0 * block_size:].data_ptr(), h, conf_weight.data_ptr(),
                float(conf_bias), tokens[r0:].data_ptr(), conf[r0:].data_ptr(), n, scratch.data_ptr(), stream),
                'dspark_markov_block')
            continue
        for k in range(block_size):
            prev, prev_stride = ((anchors[r0:].data_ptr(), 1) if k == 0
                                 else (tokens[r0:, k - 1:].data_ptr(), block_size))
            _lib.check(lib.dspark_markov_step(
                proj_weight.data_ptr(), emb_table.data_ptr(), v, rank, base[r0 * block_size:].data_ptr(), block_size,
                k, prev, prev_stride, hidden[r0 * block_size:].data_ptr(), h, conf_weight.data_ptr(),
                float(conf_bias), tokens[r0:].data_ptr(), conf[r0:].data_ptr(), block_size, n, scratch.data_ptr(),
                stream), 'dspark_markov_step')
    return tokens, conf


def rope_cache(inv_freq, rows, device):
    """Rotary cos/sin cache [rows, 64] int32 for positions 0..rows-1: per frequency f,
    bf16 cos of float32(p) * inv_freq[f] in the low 16 bits and bf16 sin in the high 16.

    Evaluated on the host with torch's float32 CPU ops, the ones transformers'
    ``Qwen3RotaryEmbedding.forward`` runs on the reference's CPU path (angle = one
    rounded float32 product, then ``cos``/``sin``, then the cast to bf16;
    modeling_qwen3.py:137-148), so a kernel that gathers rows of this cache applies
    the reference's RoPE values bit for bit. ``inv_freq`` may live on any device; it
    is copied to the host once, so build the cache outside CUDA-graph capture.
    """
    freqs = inv_freq.detach().to('cpu', torch.float32).reshape(-1)
    if freqs.numel() != HEAD_DIM // 2 or type(rows) is not int or rows < 1:
        raise ValueError('rope cache needs 64 float32 frequencies and a positive row count')
    angle = torch.arange(rows, dtype=torch.float32)[:, None] * freqs[None, :]
    bits = lambda t: t.to(torch.bfloat16).view(torch.int16).numpy().astype(np.uint32) & 0xFFFF  # noqa: E731
    packed = bits(angle.cos()) | (bits(angle.sin()) << 16)
    return torch.from_numpy(packed.view(np.int32)).to(device)


def rope_table(cache, cu_rows, ctx_len, num_requests, total_rows, out=None):
    """Per-row cos/sin table [total_rows, 64] int32 gathered from ``cache`` (``rope_cache``):
    row g of request i (cu_rows[i] <= g < cu_rows[i + 1]) takes the cache row of position
    ctx_len[i] + g - cu_rows[i] (``dspark_rope_table``)."""
    device = cache.device
    if (cache.dtype != torch.int32 or cache.ndim != 2 or cache.shape[1] != HEAD_DIM // 2
            or not cache.is_contiguous() or cu_rows.dtype != torch.int32 or ctx_len.dtype != torch.int32):
        raise ValueError('rope cache must be contiguous int32 [rows, 64] with int32 metadata')
    if out is None:
        out = torch.empty((total_rows, HEAD_DIM // 2), dtype=torch.int32, device=device)
    _lib.check(_lib.load_library().dspark_rope_table(cache.data_ptr(), cache.shape[0], cu_rows.data_ptr(),
                                                     ctx_len.data_ptr(), num_requests, total_rows, out.data_ptr(),
                                                     _stream(device)), 'dspark_rope_table')
    return out


def draft_append(context, kv_weight, k_norm_weight, rope, meta, num_requests, pool_k, pool_v, trash_row, eps):
    """Fused draft-context append (``dspark_rope_table`` + ``dspark_draft_append``):
    every layer's k = RoPE(k_norm(k_proj(context))) and v = v_proj(context) of the
    context rows, written into the layer's pool (PackedDraft.append_committed's
    project_kv + cache concatenation, dspark_qwen/packed_draft.py:146-158).

    ``context`` [n, hidden] bf16 (fc + context_norm output), ``kv_weight``
    [layers * 2048, hidden] bf16 (per layer k_proj then v_proj weight rows),
    ``k_norm_weight`` [layers, 128] bf16, ``rope`` the rotary cache (``rope_cache``) covering
    every position written, ``meta`` int32
    [4R + 1] on the device: cu_rows (R + 1), slot_row, ctx_len, count (R each).
    ``pool_k``/``pool_v``: per-layer [pool_rows, 8, 128] bf16 pools; row j of request
    i lands in slot_row[i] + ctx_len[i] + j when j < count[i], else in ``trash_row``.
    """
    import ctypes
    device = context.device
    n, hidden = context.shape
    layers = len(pool_k)
    for x in (context, kv_weight, k_norm_weight, *pool_k, *pool_v):
        if x.dtype != torch.bfloat16 or not x.is_contiguous() or x.device != device:
            raise ValueError('Draft append operands must be contiguous bf16 on one device')
    rows = pool_k[0].shape[0]
    if (kv_weight.shape != (layers * 2 * HKV * HEAD_DIM, hidden) or k_norm_weight.shape != (layers, HEAD_DIM)
            or len(pool_v) != layers or any(t.shape != (rows, HKV, HEAD_DIM) for t in (*pool_k, *pool_v))
            or meta.dtype != torch.int32 or meta.shape != (4 * num_requests + 1,) or meta.device != device
            or rope.device != device):
        raise ValueError('Draft append shapes do not match')
    r = num_requests
    table = rope_table(rope, meta, meta[2 * r + 1:], r, n)
    lib, stream = _lib.load_library(), _stream(device)
    pk = (ctypes.c_void_p * layers)(*[t.data_ptr() for t in pool_k])
    pv = (ctypes.c_void_p * layers)(*[t.data_ptr() for t in pool_v])
    _lib.check(lib.dspark_draft_append(context.data_ptr(), n, hidden, kv_weight.data_ptr(), layers,
                                       k_norm_weight.data_ptr(), table.data_ptr(), float(eps), meta.data_ptr(),
                                       meta[r + 1:].data_ptr(), meta[2 * r + 1:].data_ptr(),
                                       meta[3 * r + 1:].data_ptr(), r, pk, pv, rows, int(trash_row), stream),
               'dspark_draft_append')


STOCHASTIC_STATUS = {0: 'ok', 1: 'non-finite target logits', 2: 'draft row is not a float64 law',
                     3: 'proposal outside the vocabulary', 4: 'proposal with zero draft mass',
                     5: 'zero residual mass', 6: 'uniform outside [0, 1)', 7: 'inconsistent proposal offsets'}


def stochastic_accept(target_logits, tokens, draft_probs, cu_proposals, temperature, uniforms, budget, eos_ids=()):
    """Stochastic acceptance of one verify round on the GPU under the reference's
    float64 law (dspark_qwen/tensor_sampling.py:38-162, ``verify_proposal`` per request).

    ``target_logits`` [sum(n_i + 1), V] bf16/fp32 (request i's n_i + 1 verified rows,
    unit column stride), ``tokens`` [sum n_i] int64 proposals, ``draft_probs``
    [sum n_i, V] float64 (the draft laws they were sampled from), ``cu_proposals``
    int32 [R + 1], ``uniforms`` float64 [R, S] (S >= max n_i + 1; request i consumes
    them in the reference's draw order), ``budget`` int32 [R] (max new tokens).
    Returns device tensors ``emitted`` [R, S] int64 (-1 after the committed tokens)
    and ``result`` [R, 8] int32: count, accepted, rejected index (-1 none), extra
    (0 none, 1 residual, 2 bonus), stop reason (0 round complete, 1 EOS, 2 budget),
    uniforms used, status (0 ok, else the reference's refusal; see
    ``STOCHASTIC_STATUS``), 0.
    """
    device = target_logits.device
    r = cu_proposals.numel() - 1
    if (target_logits.ndim != 2 or target_logits.dtype not in _DTYPES or target_logits.stride(1) != 1
            or not target_logits.is_cuda or draft_probs.dtype != torch.float64 or draft_probs.ndim != 2
            or not draft_probs.is_contiguous() or draft_probs.shape[1] != target_logits.shape[1]
            or tokens.dtype != torch.long or tokens.shape != (draft_probs.shape[0],)
            or cu_proposals.dtype != torch.int32 or r < 1 or uniforms.dtype != torch.float64
            or uniforms.ndim != 2 or uniforms.shape[0] != r or not uniforms.is_contiguous()
            or budget.dtype != torch.int32 or budget.shape != (r,)
            or target_logits.shape[0] != draft_probs.shape[0] + r
            or any(t.device != device for t in (tokens, draft_probs, cu_proposals, uniforms, budget))):
        raise ValueError('stochastic_accept: [sum(n+1), V] logits, [sum n] int64 tokens, [sum n, V] float64 '
                         'draft laws, int32 [R+1] offsets, float64 [R, S] uniforms and int32 [R] budgets on '
                         'one CUDA device required')
    temperature = float(temperature)
    if not math.isfinite(temperature) or temperature <= 0:
        raise ValueError('temperature must be finite and strictly positive')
    eos = torch.tensor(sorted(set(int(e) for e in eos_ids)), dtype=torch.long, device=device)
    s = uniforms.shape[1]
    emitted = torch.empty((r, s), dtype=torch.long, device=device)
    result = torch.empty((r, 8), dtype=torch.int32, device=device)
    lib = _lib.load_library()
    rows = target_logits.shape[0] + draft_probs.shape[0]
    nbytes = int(lib.dspark_stochastic_scratch_bytes(rows))
    scratch = torch.empty(max(nbytes, 16), dtype=torch.uint8, device=device)
    _lib.check(lib.dspark_stochastic_accept(
        target_logits.data_ptr(), target_logits.stride(0), _DTYPES[target_logits.dtype], target_logits.shape[1],
        temperature, target_logits.shape[0], draft_probs.data_ptr() if draft_probs.numel() else None,
        draft_probs.shape[0], tokens.data_ptr() if tokens.numel() else None, cu_proposals.contiguous().data_ptr(),
        r, uniforms.data_ptr(), s, eos.data_ptr() if eos.numel() else None, eos.numel(), budget.data_ptr(),
        emitted.data_ptr(), result.data_ptr(), scratch.data_ptr(), scratch.numel(), _stream(device)),
        'dspark_stochastic_accept')
    return emitted, result


def stochastic_propose(base, row_index, proj, temperature, uniforms, law):
    """One Markov position of the stochastic draft proposal for several requests on the
    GPU (DSparkDraft._sample_stochastic, dspark_qwen/model.py:193-208): launch row r
    takes request row i = ``row_index[r]`` of ``base`` (bf16 [R, V] LM-head rows of the
    position, rows may be strided), adds ``proj[r]`` (bf16 [n, V] Markov projection) as
    torch adds bf16, writes the float64 law softmax(x / T) normalised once more into
    ``law[i]`` (float64 [R, V], rows may be strided) and draws a token with
    ``uniforms[r]`` by the strict CDF rule. Returns (tokens [n] int64, status [n] int32:
    0, or 1 for non-finite logits)."""
    device = base.device
    n = proj.shape[0]
    if (base.ndim != 2 or base.dtype != torch.bfloat16 or base.stride(1) != 1 or proj.ndim != 2
            or proj.dtype != torch.bfloat16 or proj.stride(1) != 1 or proj.shape[1] != base.shape[1]
            or law.ndim != 2 or law.dtype != torch.float64 or law.stride(1) != 1 or law.shape != base.shape
            or row_index.dtype != torch.int32 or row_index.shape != (n,) or not row_index.is_contiguous()
            or uniforms.dtype != torch.float64 or uniforms.shape != (n,) or not uniforms.is_contiguous()
            or any(t.device != device for t in (row_index, proj, uniforms, law)) or not base.is_cuda):
        raise ValueError('stochastic_propose: bf16 [R, V] base rows, int32 [n] row indices, bf16 [n, V] '
                         'projections, float64 [n] uniforms and a float64 [R, V] law on one CUDA device required')
    temperature = float(temperature)
    if not math.isfinite(temperature) or temperature <= 0:
        raise ValueError('temperature must be finite and strictly positive')
    tokens = torch.empty(n, dtype=torch.long, device=device)
    status = torch.empty(n, dtype=torch.int32, device=device)
    if n == 0:
        return tokens, status
    lib = _lib.load_library()
    nbytes = int(lib.dspark_propose_scratch_bytes())
    scratch = torch.empty(nbytes, dtype=torch.uint8, device=device)
    _lib.check(lib.dspark_stochastic_propose(
        base.data_ptr(), base.stride(0), row_index.data_ptr(), proj.data_ptr(), proj.stride(0), base.shape[1],
        temperature, uniforms.data_ptr(), n, law.data_ptr(), law.stride(0), tokens.data_ptr(), status.data_ptr(),
        scratch.data_ptr(), nbytes, _stream(device)), 'dspark_stochastic_propose')
    return tokens, status


def float64_law(logits, temperature):
    """The reference's sampling law of logits rows (tensor_sampling.py:38-51): float64
    softmax of logits / T, normalised once more. Torch ops on the logits' device."""
    scaled = logits.to(torch.float64) / float(temperature)
    weights = scaled.softmax(-1)
    return weights / weights.sum(-1, keepdim=True)


def sample_rows(laws, uniforms):
    """One token per law row by the strict CDF rule (tensor_sampling.py:77-84):
    searchsorted(cumsum(law), u, right=True), past the end -> last positive index."""
    vocab = laws.shape[-1]
    index = torch.searchsorted(laws.cumsum(-1), uniforms.reshape(-1, 1).to(torch.float64), right=True).flatten()
    last_positive = vocab - 1 - (laws.flip(-1) > 0).to(torch.int8).argmax(-1)
    return torch.where(index < vocab, index, last_positive)
