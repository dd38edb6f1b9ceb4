"""bfloat16 emulation in numpy (test infrastructure only).

bf16 is the upper 16 bits of an IEEE float32. Conversion float32 -> bf16 uses
round-to-nearest-even, which is what torch's ``Tensor.to(torch.bfloat16)`` and
CUDA's ``__float2bfloat16_rn`` do; NaN maps to the canonical quiet NaN 0x7FC0.
"""
import numpy as np


def f32_to_bf16_bits(x):
    x = np.ascontiguousarray(x, dtype=np.float32)
    u = x.view(np.uint32).astype(np.uint64)
    rounded = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    out = rounded.astype(np.uint16)
    out[np.isnan(x)] = 0x7FC0
    return out


def bf16_bits_to_f32(bits):
    bits = np.ascontiguousarray(bits, dtype=np.uint16)
    return (bits.astype(np.uint32) << 16).view(np.float32)


def round_bf16(x):
    """Round float32 values to the nearest bf16 value, returned as float32."""
    return bf16_bits_to_f32(f32_to_bf16_bits(x))
