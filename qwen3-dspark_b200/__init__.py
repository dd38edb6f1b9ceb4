"""B200-native (sm_100a) DSpark draft/verify attention.

Drop-in replacements for the two attention hot paths of qwen3-dspark:

* packed varlen block-draft attention (non-causal): ``B200DraftKernel``;
* KV-cached GQA verify attention (bottom-right causal): ``B200VarlenKernel``,
  ``B200CapacityKernel``, and ``B200PersistentTargetKV`` with the fused
  QK-norm + RoPE + KV-append verify layer and one-launch commit/rollback.

The kernels live in ``lib/libdspark_b200.so`` (C ABI, include/dspark_b200.h),
built from ``csrc/`` by ``build.py``. Importing this package does not touch
the GPU; constructing a kernel object loads the library and fails loudly if it
is missing or the device is not an sm_100 GPU.
"""
from . import _lib
from .build import LIB_PATH, build
from .kernels import (add_rms_norm, BACKEND, CAPACITY_BACKEND, DRAFT_BACKEND, SCALE, TRAIN_BACKEND, B200CapacityKernel,
                      B200DraftKernel, B200TrainingLayoutKernel, B200VarlenKernel, draft_append, float64_law, greedy_accept, markov_greedy, qk_norm_rope, rms_norm, silu_mul,
                      sample_rows, stochastic_accept, stochastic_propose,
                      runtime_identity, segment_attention)
from .kv_store import B200PersistentTargetKV, Slot, Transaction, rope_inv_freq
from .layout import PackedLayout, PersistentAttentionLayout, TrainingLayout


def __getattr__(name):
    # model-level modules import transformers; load them on first use
    if name in ('B200PackedDraft', 'DSparkDraftModel', 'DraftSpec'):
        from . import draft
        return getattr(draft, name)
    if name == 'B200Qwen3Target':
        from .target import B200Qwen3Target
        return B200Qwen3Target
    if name in ('speculative_greedy', 'speculative_greedy_pipelined', 'speculative_sample', 'accept_greedy'):
        from . import speculative
        return getattr(speculative, name)
    raise AttributeError(name)


load_library = _lib.load_library
read_device_status = _lib.read_device_status
launch_count = _lib.launch_count

__all__ = ['add_rms_norm', 'BACKEND', 'CAPACITY_BACKEND', 'DRAFT_BACKEND', 'SCALE', 'TRAIN_BACKEND', 'B200CapacityKernel',
           'B200DraftKernel', 'B200TrainingLayoutKernel', 'B200VarlenKernel', 'B200PersistentTargetKV', 'LIB_PATH',
           'PackedLayout', 'PersistentAttentionLayout', 'TrainingLayout', 'Slot', 'Transaction', 'B200PackedDraft',
           'DSparkDraftModel', 'DraftSpec', 'B200Qwen3Target', 'speculative_greedy', 'speculative_greedy_pipelined', 'speculative_sample', 'accept_greedy', 'build',
           'draft_append', 'float64_law', 'greedy_accept', 'markov_greedy', 'qk_norm_rope', 'rms_norm', 'silu_mul', 'sample_rows', 'stochastic_accept', 'stochastic_propose', 'launch_count', 'load_library', 'read_device_status', 'rope_inv_freq', 'runtime_identity',
           'segment_attention']
