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

// Residual form (kAdd): the rows normalised are s = bf16(x + delta), torch's bf16
// add of a decoder layer's residual and sublayer output; s is also written to
// sum_out (the new residual). Inputs must not overlap the outputs: the second
// pass recomputes s from x and delta.
template <bool kAdd>
__global__ void __launch_bounds__(kNormThreads)
    rms_norm_kernel(const __nv_bfloat16* __restrict__ x, long long ld_x, const __nv_bfloat16* __restrict__ delta,
                    long long ld_d, const __nv_bfloat16* __restrict__ weight, float eps, float inv_hidden, int rows,
                    int hidden, __nv_bfloat16* __restrict__ out, long long ld_out, __nv_bfloat16* __restrict__ sum_out,
                    long long ld_sum) {
  const int lane = threadIdx.x & 31;
  const long long row = static_cast<long long>(blockIdx.x) * kNormRowsPerCta + (threadIdx.x >> 5);
  if (row >= rows) return;
  const uint4* xr = reinterpret_cast<const uint4*>(x + row * ld_x);
  const uint4* dr = reinterpret_cast<const uint4*>(delta + (kAdd ? row * ld_d : 0));
  // the row's value vector v: x, or bf16(x + delta) in the residual form
  auto load = [&](int v) {
    uint4 u = __ldg(xr + v);
    if constexpr (kAdd) {
      const uint4 d = __ldg(dr + v);
      __nv_bfloat162* up = reinterpret_cast<__nv_bfloat162*>(&u);
      const __nv_bfloat162* dp = reinterpret_cast<const __nv_bfloat162*>(&d);
#pragma unroll
      for (int j = 0; j < 4; ++j) {
        const float2 a = __bfloat1622float2(up[j]), b = __bfloat1622float2(dp[j]);
        up[j] = __floats2bfloat162_rn(__fadd_rn(a.x, b.x), __fadd_rn(a.y, b.y));
      }
    }
    return u;
  };
  const int nvec = hidden >> 3;
  float acc = 0.f;
  for (int v = lane; v < nvec; v += 32) {
    const uint4 u = load(v);
    if constexpr (kAdd) reinterpret_cast<uint4*>(sum_out + row * ld_sum)[v] = u;
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
    const uint4 u = load(v), wu = __ldg(wr + v);
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

// Per-head RMSNorm and rotate-half RoPE of the draft block's projected q and k
// rows (head_dim 128): the draft's project_q / project_kv (dspark_qwen/model.py:
// 41-45, rotate at model.py:22-24) as one launch instead of eight norm kernels,
// neg, cat, two products, a sum and a copy per tensor. For head vector x with
// norm weight w and the rotary module's bf16 cos/sin of its row:
//   y = bf16(w * bf16(x * rsqrtf(sum(x*x) * (1/128) + eps)))     (Qwen3RMSNorm)
//   rot[d] = -y[d + 64] (d < 64), y[d - 64] (d >= 64)
//   out[d] = bf16(bf16(y[d] * cos[d]) + bf16(rot[d] * sin[d]))
// rounded where torch's bf16 ops round. One warp per (row, head); lane l holds
// dims 4l..4l+3 and its rotation partner is lane l ^ 16. Outputs are packed
// [rows, heads, 128].
constexpr int kRopeDim = 128;

__global__ void __launch_bounds__(kNormThreads)
    qk_norm_rope_kernel(const __nv_bfloat16* __restrict__ q, long long ld_q, const __nv_bfloat16* __restrict__ k,
                        long long ld_k, const __nv_bfloat16* __restrict__ q_w, const __nv_bfloat16* __restrict__ k_w,
                        float q_eps, float k_eps, const __nv_bfloat16* __restrict__ cos_t,
                        const __nv_bfloat16* __restrict__ sin_t, long long ld_cs, int rows, int q_heads, int kv_heads,
                        __nv_bfloat16* __restrict__ q_out, __nv_bfloat16* __restrict__ k_out) {
  const int lane = threadIdx.x & 31;
  const int heads = q_heads + kv_heads;
  const long long item = static_cast<long long>(blockIdx.x) * kNormRowsPerCta + (threadIdx.x >> 5);
  if (item >= static_cast<long long>(rows) * heads) return;
  const long long row = item / heads;
  const int h = static_cast<int>(item - row * heads);
  const bool is_q = h < q_heads;
  const int hh = is_q ? h : h - q_heads;
  const __nv_bfloat16* src = is_q ? q + row * ld_q + hh * kRopeDim : k + row * ld_k + hh * kRopeDim;
  const __nv_bfloat16* w = is_q ? q_w : k_w;
  __nv_bfloat16* dst = is_q ? q_out + (row * q_heads + hh) * kRopeDim : k_out + (row * kv_heads + hh) * kRopeDim;
  const float eps = is_q ? q_eps : k_eps;

  const uint2 u = *reinterpret_cast<const uint2*>(src + 4 * lane);
  const __nv_bfloat162* p = reinterpret_cast<const __nv_bfloat162*>(&u);
  const float2 x0 = __bfloat1622float2(p[0]), x1 = __bfloat1622float2(p[1]);
  float acc = 0.f;
  acc = fmaf(x0.x, x0.x, acc);
  acc = fmaf(x0.y, x0.y, acc);
  acc = fmaf(x1.x, x1.x, acc);
  acc = fmaf(x1.y, x1.y, acc);
#pragma unroll
  for (int o = 16; o; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  const float r = rsqrtf(__fadd_rn(__fmul_rn(acc, 1.0f / kRopeDim), eps));
  const uint2 wu = *reinterpret_cast<const uint2*>(w + 4 * lane);
  const __nv_bfloat162* wp = reinterpret_cast<const __nv_bfloat162*>(&wu);
  const float xs[4] = {x0.x, x0.y, x1.x, x1.y};
  const float2 w0 = __bfloat1622float2(wp[0]), w1 = __bfloat1622float2(wp[1]);
  const float ws[4] = {w0.x, w0.y, w1.x, w1.y};
  float y[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float n = __bfloat162float(__float2bfloat16_rn(__fmul_rn(xs[j], r)));
    y[j] = __bfloat162float(__float2bfloat16_rn(__fmul_rn(ws[j], n)));
  }
  const bool low = lane < 16;
  const uint2 cu = *reinterpret_cast<const uint2*>(cos_t + row * ld_cs + 4 * lane);
  const uint2 su = *reinterpret_cast<const uint2*>(sin_t + row * ld_cs + 4 * lane);
  const __nv_bfloat162* cp = reinterpret_cast<const __nv_bfloat162*>(&cu);
  const __nv_bfloat162* sp = reinterpret_cast<const __nv_bfloat162*>(&su);
  const float2 c0 = __bfloat1622float2(cp[0]), c1 = __bfloat1622float2(cp[1]);
  const float2 s0 = __bfloat1622float2(sp[0]), s1 = __bfloat1622float2(sp[1]);
  const float cs[4] = {c0.x, c0.y, c1.x, c1.y}, sn[4] = {s0.x, s0.y, s1.x, s1.y};
  float o[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float partner = __shfl_xor_sync(0xffffffffu, y[j], 16);
    const float rot = low ? -partner : partner;
    const float a = __bfloat162float(__float2bfloat16_rn(__fmul_rn(y[j], cs[j])));
    const float b = __bfloat162float(__float2bfloat16_rn(__fmul_rn(rot, sn[j])));
    o[j] = __fadd_rn(a, b);
  }
  uint2 out;
  __nv_bfloat162* op = reinterpret_cast<__nv_bfloat162*>(&out);
  op[0] = __floats2bfloat162_rn(o[0], o[1]);
  op[1] = __floats2bfloat162_rn(o[2], o[3]);
  *reinterpret_cast<uint2*>(dst + 4 * lane) = out;
}

// Gated activation of a Qwen3MLP (transformers models/qwen3/modeling_qwen3.py,
// Qwen3MLP.forward: down_proj(act_fn(gate_proj(x)) * up_proj(x))) from ONE
// merged [gate; up] projection: row i of gate_up (stride ld elements) holds the
// inter gate values, then the inter up values. For g, u of one column:
//   out = bf16(float(bf16(g / (1 + expf(-g)))) * float(u))
// which is torch's silu kernel on a bf16 tensor (float math, rounded to bf16)
// followed by the bf16 product. 8 columns per thread, 16-byte loads and stores.
constexpr int kSiluThreads = 256;

__global__ void __launch_bounds__(kSiluThreads)
    silu_mul_kernel(const __nv_bfloat16* __restrict__ gate_up, long long ld, int rows, int inter,
                    __nv_bfloat16* __restrict__ out, long long ld_out) {
  const int vecs = inter >> 3;
  const long long idx = static_cast<long long>(blockIdx.x) * kSiluThreads + threadIdx.x;
  if (idx >= static_cast<long long>(rows) * vecs) return;
  const long long row = idx / vecs;
  const int c = static_cast<int>(idx - row * vecs) * 8;
  const uint4 gv = *reinterpret_cast<const uint4*>(gate_up + row * ld + c);
  const uint4 uv = *reinterpret_cast<const uint4*>(gate_up + row * ld + inter + c);
  const __nv_bfloat162* g2 = reinterpret_cast<const __nv_bfloat162*>(&gv);
  const __nv_bfloat162* u2 = reinterpret_cast<const __nv_bfloat162*>(&uv);
  uint4 ov;
  __nv_bfloat162* o2 = reinterpret_cast<__nv_bfloat162*>(&ov);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    const float2 g = __bfloat1622float2(g2[j]);
    const float2 u = __bfloat1622float2(u2[j]);
    const float ax = __bfloat162float(__float2bfloat16_rn(g.x / (1.0f + expf(-g.x))));
    const float ay = __bfloat162float(__float2bfloat16_rn(g.y / (1.0f + expf(-g.y))));
    o2[j] = __floats2bfloat162_rn(__fmul_rn(ax, u.x), __fmul_rn(ay, u.y));
  }
  *reinterpret_cast<uint4*>(out + row * ld_out + c) = ov;
}

}  // namespace dspark
