"""Qwen3 per-head QK-RMSNorm + rotate-half RoPE in bf16 (numpy, test infrastructure only).

Restates, rounding for rounding, the CPU evaluation of the transformers Qwen3
attention that the reference runs for every verify token (installed
``modeling_qwen3.py``: ``Qwen3RMSNorm.forward`` lines 59-64,
``compute_default_rope_parameters`` lines 124-133, ``Qwen3RotaryEmbedding.forward``
lines 137-148, ``rotate_half``/``apply_rotary_pos_emb`` lines 151-181, called from
``Qwen3Attention.forward`` lines 263-268; the draft's ``rotate`` in
dspark_qwen/model.py:22-24 is the same rotate-half form):

* RMSNorm: x -> float32; the sum of squares over the 128-wide head in the
  association order of torch's CPU float32 reduction (``torch_order_sum128``);
  mean = sum / 128; r = 1 / sqrt(mean + eps) with each step rounded to float32;
  x * r rounded to bf16, then ``weight * x`` rounded to bf16 (the cast happens
  before the weight multiply).
* RoPE: inv_freq = 1 / theta^(2i/d) in float32; angle = position * inv_freq in
  float32; cos/sin evaluated by torch's float32 CPU ``cos``/``sin`` (the op the
  rotary module runs; a correctly rounded cos differs from it in a few entries per
  million after the bf16 cast, e.g. sin at position 2954, frequency 8) and rounded
  to bf16; out = bf16(bf16(x*cos) + bf16(rotate_half(x)*sin)).

With these two choices the oracle equals transformers' CPU output bit for bit
(``tests/test_oracle_golden.py`` pins it to fixtures made by the reference's
modules), so the GPU kernels that follow the same order are checked for exact
equality, not within an ulp.
"""
import numpy as np

from .bf16 import bf16_bits_to_f32, f32_to_bf16_bits, round_bf16


def inv_freq(theta, dim):
    """float32 [dim/2]: 1 / theta ** (arange(0, dim, 2) / dim) (modeling_qwen3.py:130-132).

    The table is a host constant of the model's rotary module, computed by torch's
    float32 ``pow``; it is evaluated with the same torch expression here because
    numpy's float32/float64 ``pow`` differ from it in the last bit for some entries.
    """
    import torch
    exponent = torch.arange(0, dim, 2, dtype=torch.int64).to(dtype=torch.float) / dim
    return (1.0 / (theta ** exponent)).numpy().astype(np.float32)


def torch_order_sum128(sq):
    """float32 sum over the last axis (length 128) associated as torch's CPU float32
    reduction of a contiguous row associates it: 8-wide vectors v[m] = sq[8m:8m+8],
    four vector accumulators acc[k] = ((v[k] + v[k+4]) + v[k+8]) + v[k+12], then
    ((acc[0] + acc[1]) + acc[2]) + acc[3], then the 8 lanes added left to right.
    ``tests/test_oracle_golden.py`` checks this against ``torch.sum`` on the host."""
    sq = np.asarray(sq, np.float32)
    if sq.shape[-1] != 128:
        raise ValueError('torch_order_sum128 sums 128-element rows')
    v = sq.reshape(sq.shape[:-1] + (16, 8))
    acc = [((v[..., k, :] + v[..., k + 4, :]) + v[..., k + 8, :]) + v[..., k + 12, :] for k in range(4)]
    lanes = ((acc[0] + acc[1]) + acc[2]) + acc[3]
    total = lanes[..., 0]
    for j in range(1, 8):
        total = total + lanes[..., j]
    return total.astype(np.float32)[..., None]


def rope_cos_sin_bf16(positions, inv_freq_f32):
    """cos/sin tables [n, dim] as bf16 values (float32 storage), emb = cat(freqs, freqs).

    The angle is one rounded float32 product; cos/sin are torch's CPU float32 ops."""
    import torch
    pos = np.asarray(positions, dtype=np.float32)
    freqs = (pos[:, None] * inv_freq_f32[None, :]).astype(np.float32)
    emb = torch.from_numpy(np.concatenate((freqs, freqs), axis=-1))
    cos = round_bf16(emb.cos().numpy())
    sin = round_bf16(emb.sin().numpy())
    return cos, sin


def rms_norm_bf16(x_bits, w_bits, eps):
    """bf16 RMSNorm over a 128-wide last axis; inputs/outputs are bf16 bit patterns (uint16)."""
    x = bf16_bits_to_f32(x_bits)
    var = torch_order_sum128(x * x) / np.float32(x.shape[-1])
    r = np.float32(1) / np.sqrt((var + np.float32(eps)).astype(np.float32))
    y = round_bf16((x * r.astype(np.float32)).astype(np.float32))
    w = bf16_bits_to_f32(w_bits)
    return f32_to_bf16_bits((w * y).astype(np.float32))


def rope_bf16(x_bits, cos, sin):
    """Rotate-half RoPE of [n, heads, dim] bf16 bits with per-row cos/sin [n, dim]."""
    x = bf16_bits_to_f32(x_bits)
    half = x.shape[-1] // 2
    rot = np.concatenate((-x[..., half:], x[..., :half]), axis=-1)
    t1 = round_bf16((x * cos[:, None, :]).astype(np.float32))
    t2 = round_bf16((rot * sin[:, None, :]).astype(np.float32))
    return f32_to_bf16_bits((t1 + t2).astype(np.float32))


def qk_norm_rope_bf16(q_bits, k_bits, qw_bits, kw_bits, positions, theta, eps):
    """Qwen3 q/k path for new tokens: RMSNorm per head then RoPE at ``positions``.

    q_bits [n, Hq, D], k_bits [n, Hkv, D], weights [D]; returns (q, k) bf16 bits.
    """
    freqs = inv_freq(theta, q_bits.shape[-1])
    cos, sin = rope_cos_sin_bf16(positions, freqs)
    q = rope_bf16(rms_norm_bf16(q_bits, qw_bits, eps), cos, sin)
    k = rope_bf16(rms_norm_bf16(k_bits, kw_bits, eps), cos, sin)
    return q, k
