"""ctypes binding of the C ABI in include/dspark_b200.h.

The shared library is loaded from this package's ``lib/`` directory. There is
no fallback: if the library is missing or cannot load, every native entry
raises ``RuntimeError``.
"""
import ctypes
import os
import threading

from .build import LIB_PATH

OK, ERR_INVALID_ARGUMENT, ERR_UNSUPPORTED, ERR_CUDA = 0, 1, 2, 3
DTYPE_BF16, DTYPE_F32 = 0, 1
DEVICE_WAIT_TIMEOUT, DEVICE_BAD_SCHEDULE, DEVICE_BAD_ARGUMENT = 1, 2, 4
VERIFY_PATHS = {'auto': -1, 'fused': 0, 'prep': 1}

_vp, _i, _ll, _f, _sz = ctypes.c_void_p, ctypes.c_int, ctypes.c_longlong, ctypes.c_float, ctypes.c_size_t

# name -> (restype, argtypes); mirrors include/dspark_b200.h
SIGNATURES = {
    'dspark_abi_version': (_i, []),
    'dspark_launch_count': (ctypes.c_ulonglong, []),
    'dspark_status_string': (ctypes.c_char_p, [_i]),
    'dspark_attention_workspace_size': (_i, [_i, ctypes.POINTER(_sz)]),
    'dspark_read_device_status': (_i, [ctypes.POINTER(ctypes.c_uint), _i]),
    'dspark_copy_device_status': (_i, [_vp, _vp]),
    'dspark_draft_attn': (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _ll, _i, _i, _f, _i, _vp, _vp, _sz, _vp]),
    'dspark_varlen_attn': (_i, [_vp, _vp, _vp, _vp, _vp, _i, _i, _ll, _i, _i, _f, _i, _vp, _vp, _sz, _vp]),
    'dspark_segment_attn': (_i, [_vp, _vp, _vp, _ll, _vp, _vp, _ll, _vp, _vp, _vp, _vp, _vp, _i, _i, _i, _i, _i,
                                 _i, _f, _i, _vp, _vp, _sz, _vp]),
    'dspark_verify_fused': (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _f, _vp, _vp, _vp, _i, _i, _i, _vp, _vp, _ll, _vp,
                                 _vp, _i, _i, _i, _f, _i, _vp, _vp, _sz, _vp]),
    'dspark_verify_strided': (_i, [_vp, _ll, _vp, _ll, _vp, _ll, _vp, _vp, _vp, _f, _vp, _vp, _vp, _i, _i, _i, _vp,
                                   _vp, _ll, _vp, _vp, _i, _i, _i, _f, _i, _vp, _vp, _sz, _vp]),
    'dspark_rope_table': (_i, [_vp, _i, _vp, _vp, _i, _i, _vp, _vp]),
    'dspark_commit_kv': (_i, [_vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _vp, _i, _i, _ll, _i, _i, _vp]),
    'dspark_train_plan': (_i, [_i, _vp, _vp, _vp, _i, _i, _vp, _ll, ctypes.POINTER(_ll)]),
    'dspark_row_argmax': (_i, [_vp, _ll, _i, _i, _i, _vp, _vp]),
    'dspark_markov_scratch_bytes': (_sz, []),
    'dspark_propose_scratch_bytes': (_sz, []),
    'dspark_stochastic_propose': (_i, [_vp, _ll, _vp, _vp, _ll, _i, ctypes.c_double, _vp, _i, _vp, _ll, _vp, _vp,
                                       _vp, _sz, _vp]),
    'dspark_set_grid_barrier_timeout': (_i, [ctypes.c_ulonglong]),
    'dspark_markov_step': (_i, [_vp, _vp, _i, _i, _vp, _ll, _i, _vp, _ll, _vp, _i, _vp, _f, _vp, _vp, _ll, _i,
                                _vp, _vp]),
    'dspark_markov_block': (_i, [_vp, _vp, _i, _i, _vp, _i, _vp, _vp, _i, _vp, _f, _vp, _vp, _i, _vp, _vp]),
    'dspark_rms_norm': (_i, [_vp, _ll, _vp, _f, _i, _i, _vp, _ll, _vp]),
    'dspark_qk_norm_rope': (_i, [_vp, _ll, _vp, _ll, _vp, _vp, _f, _f, _vp, _vp, _ll, _i, _i, _i, _vp, _vp, _vp]),
    'dspark_silu_mul': (_i, [_vp, _ll, _i, _i, _vp, _ll, _vp]),
    'dspark_add_rms_norm': (_i, [_vp, _ll, _vp, _ll, _vp, _f, _i, _i, _vp, _ll, _vp, _ll, _vp]),
    'dspark_greedy_accept': (_i, [_vp, _vp, _vp, _i, _i, _vp, _i, _vp, _vp, _vp, _vp, _vp]),
    'dspark_train_attn': (_i, [_vp, _vp, _vp, _i, _ll, _vp, _i, _f, _vp, _vp]),
    'dspark_stochastic_scratch_bytes': (_sz, [_i]),
    'dspark_stochastic_accept': (_i, [_vp, _ll, _i, _i, ctypes.c_double, _i, _vp, _i, _vp, _vp, _i, _vp, _i, _vp, _i,
                                      _vp, _vp, _vp, _vp, _sz, _vp]),
    'dspark_draft_append': (_i, [_vp, _i, _i, _vp, _i, _vp, _vp, _f, _vp, _vp, _vp, _vp, _i, _vp, _vp, _ll, _ll,
                                 _vp]),
}

_lock = threading.Lock()
_lib = None


def load_library(path=LIB_PATH):
    """Load (once) and return the ctypes library with typed entry points."""
    global _lib
    with _lock:
        if _lib is not None:
            return _lib
        if not os.path.exists(path):
            raise RuntimeError(f'dspark B200 CUDA library not built ({path}); run build() first. '
                               'There is no CPU fallback.')
        lib = ctypes.CDLL(path)
        for name, (res, args) in SIGNATURES.items():
            fn = getattr(lib, name)
            fn.restype = res
            fn.argtypes = args
        if lib.dspark_abi_version() != 18:
            raise RuntimeError('dspark B200 library ABI version mismatch')
        _lib = lib
        return lib


def check(status, what):
    if status != OK:
        msg = load_library().dspark_status_string(status).decode()
        if status == ERR_INVALID_ARGUMENT:
            raise ValueError(f'{what}: {msg}')
        raise RuntimeError(f'{what}: {msg} (status {status})')


def launch_count():
    """Kernels launched by the library since load (host-side counter)."""
    return int(load_library().dspark_launch_count())


def read_device_status(clear=True):
    """Device status bits set by kernels since the last clear (synchronising)."""
    v = ctypes.c_uint(0)
    check(load_library().dspark_read_device_status(ctypes.byref(v), int(clear)), 'dspark_read_device_status')
    return v.value


STATUS_NAMES = {DEVICE_WAIT_TIMEOUT: 'a bounded wait ran out', DEVICE_BAD_SCHEDULE: 'tile schedules disagreed',
                DEVICE_BAD_ARGUMENT: 'a kernel refused an out-of-range index'}


def describe_status(status):
    return ', '.join(name for bit, name in STATUS_NAMES.items() if status & bit) or 'unknown bits'


def set_grid_barrier_timeout(ns=2_000_000_000):
    """Time limit of the Markov block kernel's grid barrier on the current device
    (nanoseconds; default two seconds). For failure-handling tests."""
    check(load_library().dspark_set_grid_barrier_timeout(int(ns)), 'dspark_set_grid_barrier_timeout')


_workspaces = {}


def workspace(device, stream):
    """Attention workspace for (device, stream); calls on one stream share it."""
    import torch
    key = (device.index, stream)
    ws = _workspaces.get(key)
    if ws is None:
        size = ctypes.c_size_t(0)
        check(load_library().dspark_attention_workspace_size(device.index, ctypes.byref(size)),
              'dspark_attention_workspace_size')
        ws = torch.empty(size.value, dtype=torch.uint8, device=device)
        _workspaces[key] = ws
    return ws


def train_plan(context_lengths, num_blocks, anchors, block_size, grid_limit):
    """Host-built work plan of the training-layout kernel (int32 list); no GPU needed."""
    lib = load_library()
    n = len(context_lengths)
    arr = lambda xs: (ctypes.c_int32 * max(len(xs), 1))(*xs)  # noqa: E731
    ctx, nb, anc = arr(context_lengths), arr(num_blocks), arr(anchors)
    words = ctypes.c_longlong(0)
    check(lib.dspark_train_plan(n, ctx, nb, anc, block_size, grid_limit, None, 0, ctypes.byref(words)),
          'dspark_train_plan')
    plan = (ctypes.c_int32 * words.value)()
    check(lib.dspark_train_plan(n, ctx, nb, anc, block_size, grid_limit, plan, words.value, ctypes.byref(words)),
          'dspark_train_plan')
    return list(plan)
