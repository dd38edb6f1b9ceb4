// Verify-path companions of the attention kernel:
//  * qk_norm_rope_append_kernel: Qwen3 per-head RMSNorm + rotate-half RoPE of
//    the new tokens' q and k, with the KV append of roped k / raw v into the
//    layer's verify scratch rows (one launch instead of the ~10 eager ops of
//    the transformers attention plus the store's staging copies);
//  * commit_kernel: copies every request's accepted scratch prefix into its
//    resident rows for all layers in one launch (rollback = not copying).
#pragma once
#include "attention.cuh"

namespace dspark {

struct VerifyParams {
  const __nv_bfloat16* q_raw;   // [total_q, 16, 128]
  const __nv_bfloat16* k_raw;   // [total_q, 8, 128]
  const __nv_bfloat16* v_raw;   // [total_q, 8, 128]
  const __nv_bfloat16* q_w;     // [128]
  const __nv_bfloat16* k_w;     // [128]
  const float* inv_freq;        // [64]
  const int* cu_q;              // [R+1]
  const int* ctx_len;           // [R]: committed context = position of the first new token
  int num_requests;
  int total_q;
  float eps;
  __nv_bfloat16* q_out;         // [total_q, 16, 128] roped q
  __nv_bfloat16* scratch_k;     // rows of this layer's scratch: [max_q_rows, 8, 128]
  __nv_bfloat16* scratch_v;
  int scratch_rows;             // rows available in the layer's scratch
};

__device__ __forceinline__ int find_request(const int* cu, int n, int row) {
  int lo = 0, hi = n - 1;                 // largest i with cu[i] <= row
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= row) lo = mid; else hi = mid - 1;
  }
  return lo;
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// One block per new token row; warp w: 0-15 q heads, 16-23 k heads, 24-31 v heads.
// Lane l owns elements 4l..4l+3; the rotate-half partner lives in lane l^16.
__global__ void __launch_bounds__(1024) qk_norm_rope_append_kernel(const VerifyParams p) {
  const int row = blockIdx.x;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (row >= p.total_q || row >= p.scratch_rows) {
    if (threadIdx.x == 0) atomicOr(&g_device_status, kStatusBadArgument);
    return;
  }
  const int d0 = lane * 4;
  if (warp >= 24) {
    const int h = warp - 24;
    const uint2 v = *reinterpret_cast<const uint2*>(p.v_raw + (static_cast<size_t>(row) * kKVHeads + h) * 128 + d0);
    *reinterpret_cast<uint2*>(p.scratch_v + (static_cast<size_t>(row) * kKVHeads + h) * 128 + d0) = v;
    return;
  }
  const bool is_q = warp < 16;
  const int h = is_q ? warp : warp - 16;
  const __nv_bfloat16* src = is_q ? p.q_raw + (static_cast<size_t>(row) * 16 + h) * 128
                                  : p.k_raw + (static_cast<size_t>(row) * kKVHeads + h) * 128;
  const __nv_bfloat16* wgt = is_q ? p.q_w : p.k_w;
  const uint2 raw = *reinterpret_cast<const uint2*>(src + d0);
  const __nv_bfloat162* r2 = reinterpret_cast<const __nv_bfloat162*>(&raw);
  float x[4];
  x[0] = __low2float(r2[0]);
  x[1] = __high2float(r2[0]);
  x[2] = __low2float(r2[1]);
  x[3] = __high2float(r2[1]);
  // RMSNorm: float32 mean of squares, x * rsqrt(var + eps) -> bf16 -> * weight -> bf16.
  float ss = x[0] * x[0] + x[1] * x[1] + x[2] * x[2] + x[3] * x[3];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
  const float var = ss / 128.f;
  const float rs = 1.f / sqrtf(var + p.eps);
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) y[i] = bf16r(__bfloat162float(wgt[d0 + i]) * bf16r(x[i] * rs));
  // RoPE at this token's position: cos/sin in float32 rounded to bf16;
  // out = bf16(bf16(y*cos) + bf16(rotate_half(y)*sin)).
  const int req = min(find_request(p.cu_q, p.num_requests + 1, row), p.num_requests - 1);
  const int pos = p.ctx_len[req] + (row - p.cu_q[req]);
  float partner[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) partner[i] = __shfl_xor_sync(0xffffffffu, y[i], 16);
  float out[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int d = d0 + i;
    const float ang = static_cast<float>(pos) * p.inv_freq[d & 63];
    float sn, cs;
    sincosf(ang, &sn, &cs);
    const float rot = lane < 16 ? -partner[i] : partner[i];
    out[i] = bf16r(bf16r(y[i] * bf16r(cs)) + bf16r(rot * bf16r(sn)));
  }
  uint2 res;
  res.x = pack_bf16x2(out[0], out[1]);
  res.y = pack_bf16x2(out[2], out[3]);
  __nv_bfloat16* dst = is_q ? p.q_out + (static_cast<size_t>(row) * 16 + h) * 128
                            : p.scratch_k + (static_cast<size_t>(row) * kKVHeads + h) * 128;
  *reinterpret_cast<uint2*>(dst + d0) = res;
}

struct CommitParams {
  __nv_bfloat16* resident_k;     // [layers * rows_per_layer, 8, 128]
  __nv_bfloat16* resident_v;
  const __nv_bfloat16* scratch_k;  // [layers * scratch_rows, 8, 128]
  const __nv_bfloat16* scratch_v;
  const int* cu_q;               // [R+1] scratch row offsets
  const int* slot_row;           // [R] first resident row of each request's slot
  const int* ctx_len;            // [R] committed rows before this commit
  const int* slot_cap;           // [R] resident rows owned by each slot
  const int* n_commit;           // [R] accepted rows (anchor included)
  int num_requests;
  int num_layers;
  long long rows_per_layer;
  int scratch_rows;
};

// grid (R, layers); each block copies n_commit[i] rows of K and of V.
__global__ void __launch_bounds__(256) commit_kernel(const CommitParams p) {
  const int i = blockIdx.x, layer = blockIdx.y;
  const int n = p.n_commit[i];
  const int q0 = p.cu_q[i], q_len = p.cu_q[i + 1] - q0;
  const int c = p.ctx_len[i];
  if (n < 0 || n > q_len || c < 0 || c + n > p.slot_cap[i] || q0 + q_len > p.scratch_rows) {
    if (threadIdx.x == 0) atomicOr(&g_device_status, kStatusBadArgument);
    return;
  }
  constexpr int kVecPerRow = kKVHeads * 128 * 2 / 16;   // 128 x 16 B per row
  const size_t src_row = static_cast<size_t>(layer) * p.scratch_rows + q0;
  const size_t dst_row = static_cast<size_t>(layer) * p.rows_per_layer + p.slot_row[i] + c;
  const uint4* sk = reinterpret_cast<const uint4*>(p.scratch_k) + src_row * kVecPerRow;
  const uint4* sv = reinterpret_cast<const uint4*>(p.scratch_v) + src_row * kVecPerRow;
  uint4* dk = reinterpret_cast<uint4*>(p.resident_k) + dst_row * kVecPerRow;
  uint4* dv = reinterpret_cast<uint4*>(p.resident_v) + dst_row * kVecPerRow;
  for (int u = threadIdx.x; u < n * kVecPerRow; u += blockDim.x) {
    dk[u] = sk[u];
    dv[u] = sv[u];
  }
}

}  // namespace dspark
