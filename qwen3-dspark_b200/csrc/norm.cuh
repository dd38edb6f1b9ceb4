// Row RMSNorm of bf16 hidden states in one launch: the operation of
// transformers' Qwen3RMSNorm.forward (transformers 5.5,
// models/qwen3/modeling_qwen3.py:62-66), which the reference's target and draft
// layers run as eight separate elementwise and reduction kernels
// (to(float32), pow, mean, add, rsqrt, mul, to(bf16), weight mul).
//
//   h   = float(x)
//   var = sum(h * h) * fl(1 / hidden)            (torch's mean: sum times factor)
//   r   = rsqrtf(var + eps)
//   out = bf16(float(w) * float(bf16(h * r)))
//
// Each step rounds where the torch sequence rounds: h * h is exact in float for
// a bf16 h, the mean and the eps add are two roundings (no FMA contraction),
// h * r rounds to float and then to bf16, and the weight product is a bf16
// multiply. Only the association of the float sum differs from torch's
// reduction tree, which can move var by a few float ulps and so, rarely, one
// output by one bf16 ulp.
//
// One warp per row, 16-byte loads; the second pass re-reads the row from L1.
#pragma once
#include "ptx.cuh"

namespace dspark {

constexpr int kNormThreads = 256;
constexpr int kNormRowsPerCta = kNormThreads / 32;

__global__ void __launch_bounds__(kNormThreads)
    rms_norm_kernel(const __nv_bfloat16* __restrict__ x, long long ld_x, const __nv_bfloat16* __restrict__ weight,
                    float eps, float inv_hidden, int rows, int hidden, __nv_bfloat16* __restrict__ out,
                    long long ld_out) {
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * kNormRowsPerCta + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ld_x);
  const int nvec = hidden >> 3;
  float acc = 0.f;
  for (int v = lane; v < nvec; v += 32) {
    const uint4 u = __ldg(xr + v);
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(p[j]);
      acc = fmaf(f.x, f.x, acc);  // the product is exact, so this is h*h then the add
      acc = fmaf(f.y, f.y, acc);
    }
  }
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  const float r = rsqrtf(__fadd_rn(__fmul_rn(acc, inv_hidden), eps));
  const uint4* wr = reinterpret_cast<const uint4*>(weight);
  uint4* orow = reinterpret_cast<uint4*>(out + row * ld_out);
  for (int v = lane; v < nvec; v += 32) {
    const uint4 u = __ldg(xr + v), wu = __ldg(wr + v);
    const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
    const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&wu);
    uint4 o;
    __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&o);
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const float2 f = __bfloat1622float2(p[j]);
      const float2 w = __bfloat1622float2(wp[j]);
      const float2 n = __bfloat1622float2(__floats2bfloat162_rn(__fmul_rn(f.x, r), __fmul_rn(f.y, r)));
      op[j] = __floats2bfloat162_rn(__fmul_rn(w.x, n.x), __fmul_rn(w.y, n.y));
    }
    orow[v] = o;
  }
}

}  // namespace dspark
