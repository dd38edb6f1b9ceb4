"""Qwen3 per-head QK-RMSNorm + rotate-half RoPE in bf16 (numpy, test infrastructure only).

Restates the bf16 arithmetic order of the transformers Qwen3 attention that the
reference runs for every verify token (installed ``modeling_qwen3.py``:
``Qwen3RMSNorm.forward`` lines 59-64, ``compute_default_rope_parameters``
lines 124-133, ``Qwen3RotaryEmbedding.forward`` lines 137-148,
``rotate_half``/``apply_rotary_pos_emb`` lines 151-181, called from
``Qwen3Attention.forward`` lines 263-268; the draft's ``rotate`` in
dspark_qwen/model.py:22-24 is the same rotate-half form):

* RMSNorm: x -> float32, x * rsqrt(mean(x^2) + eps), round to bf16, then
  ``weight * x`` rounded to bf16 (the cast happens before the weight multiply).
* RoPE: inv_freq = 1 / theta^(2i/d) in float32; angle = position * inv_freq in
  float32; cos/sin computed in float32 then rounded to bf16;
  out = bf16(bf16(x*cos) + bf16(rotate_half(x)*sin)).

Transcendentals are evaluated in float64 and rounded to float32, i.e. the
correctly rounded float32 value; library float32 cos/sin/rsqrt may differ from
it by an ulp, which can move a bf16 result by one bf16 ulp.
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


def rope_cos_sin_bf16(positions, inv_freq_f32):
    """cos/sin tables [n, dim] as bf16 values (float32 storage), emb = cat(freqs, freqs)."""
    pos = np.asarray(positions, dtype=np.float32)
    freqs = (pos[:, None] * inv_freq_f32[None, :]).astype(np.float32)
    emb = np.concatenate((freqs, freqs), axis=-1).astype(np.float64)
    cos = round_bf16(np.cos(emb).astype(np.float32))
    sin = round_bf16(np.sin(emb).astype(np.float32))
    return cos, sin


def rms_norm_bf16(x_bits, w_bits, eps):
    """bf16 RMSNorm over the last axis; inputs/outputs are bf16 bit patterns (uint16)."""
    x = bf16_bits_to_f32(x_bits)
    var = np.mean(x.astype(np.float64) ** 2, axis=-1, keepdims=True).astype(np.float32)
    r = (1.0 / np.sqrt(var.astype(np.float64) + np.float64(np.float32(eps)))).astype(np.float32)
    y = round_bf16((x * r).astype(np.float32))
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
