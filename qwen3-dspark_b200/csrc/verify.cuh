// Verify-path commit: copies every request's accepted scratch prefix into its
// resident rows for all layers in one launch (rollback = not copying). The
// QK-norm + RoPE + KV append of the verify layer is fused into the attention
// kernel (attention.cuh, kFused).
#pragma once
#include "attention.cuh"

namespace dspark {

__device__ __forceinline__ int find_request(const int* cu, int n, int row) {
  int lo = 0, hi = n - 1;                 // largest i with cu[i] <= row
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (cu[mid] <= row) lo = mid; else hi = mid - 1;
  }
  return lo;
}

// cos/sin table of a transaction, shared by all layers: new row r of request i
// (global row cu_q[i] + r) is at position ctx_len[i] + r, and its table row is that
// position's row of the caller's rotary cache (bf16 cos | bf16 sin << 16 per
// frequency, evaluated once on the host by the same float32 ops as the model's
// rotary module, so the kernels use the reference's cos/sin values bit for bit).
// One thread per 16-byte quarter-chunk: 16 threads per row. A position outside the
// cache raises kStatusBadArgument and gives a zero row.
__global__ void __launch_bounds__(256) rope_table_kernel(const uint4* __restrict__ cache, int cache_rows,
                                                         const int* cu_q, const int* ctx_len, int num_requests,
                                                         int total_q, uint4* table) {
  const int row = blockIdx.x * 16 + (threadIdx.x >> 4);
  const int c = threadIdx.x & 15;
  if (row >= total_q) return;
  const int req = min(find_request(cu_q, num_requests + 1, row), num_requests - 1);
  const int pos = ctx_len[req] + (row - cu_q[req]);
  uint4 v = make_uint4(0u, 0u, 0u, 0u);
  if (pos >= 0 && pos < cache_rows) {
    v = cache[static_cast<size_t>(pos) * 16 + c];
  } else if (c == 0) {
    atomicOr(&g_device_status, kStatusBadArgument);
  }
  table[static_cast<size_t>(row) * 16 + c] = v;
}

// Verify-layer preparation of the new rows, shared by every tile that reads
// them: q_norm + RoPE of the raw q projections (written to q_out, which the
// attention kernel then reads), k_norm + RoPE of the raw k and a copy of the
// raw v into this layer's scratch rows (the KV append). transformers' order of
// bf16 roundings (modeling_qwen3.py:59-64,136-156): RMSNorm in fp32, cast to
// bf16, times the bf16 weight; each RoPE product and the sum rounded to bf16.
// One warp per (row, vector) with 32 vectors per row (16 q heads, 8 k, 8 v);
// lane l holds d = 4l..4l+3 and its rotate-half partner d +- 64 is lane l ^ 16.
struct VerifyPrepParams {
  const __nv_bfloat16* q_raw;   // [total_q, 16, 128]
  const __nv_bfloat16* k_raw;   // [total_q, 8, 128]
  const __nv_bfloat16* v_raw;
  const __nv_bfloat16* q_w;     // [128]
  const __nv_bfloat16* k_w;
  const uint32_t* rope;         // [total_q, 64] bf16 cos | bf16 sin << 16
  __nv_bfloat16* q_out;         // [total_q, 16, 128]
  __nv_bfloat16* scratch_k;     // this layer's scratch, row r = new row r
  __nv_bfloat16* scratch_v;
  int total_q;
  float eps;
  long long ld_q, ld_k, ld_v;   // row strides of q_raw / k_raw / v_raw in elements
};

__global__ void __launch_bounds__(256) verify_prep_kernel(const VerifyPrepParams p) {
  asm volatile("griddepcontrol.launch_dependents;");
  const int wid = static_cast<int>(blockIdx.x) * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
  const int row = wid >> 5, vec = wid & 31;
  if (row >= p.total_q) return;
  const int d0 = lane * 4;
  const __nv_bfloat16* src;
  __nv_bfloat16* dst;
  const __nv_bfloat16* w = nullptr;
  if (vec < kQHeads) {
    src = p.q_raw + static_cast<size_t>(row) * p.ld_q + static_cast<size_t>(vec) * kHeadDim;
    dst = p.q_out + (static_cast<size_t>(row) * kQHeads + vec) * kHeadDim;
    w = p.q_w;
  } else if (vec < kQHeads + kKVHeads) {
    src = p.k_raw + static_cast<size_t>(row) * p.ld_k + static_cast<size_t>(vec - kQHeads) * kHeadDim;
    dst = p.scratch_k + (static_cast<size_t>(row) * kKVHeads + vec - kQHeads) * kHeadDim;
    w = p.k_w;
  } else {
    src = p.v_raw + static_cast<size_t>(row) * p.ld_v +
          static_cast<size_t>(vec - kQHeads - kKVHeads) * kHeadDim;
    dst = p.scratch_v + (static_cast<size_t>(row) * kKVHeads + vec - kQHeads - kKVHeads) * kHeadDim;
  }
  const uint2 raw = *reinterpret_cast<const uint2*>(src + d0);
  if (w == nullptr) {                       // warp-uniform: v rows are copied as they are
    *reinterpret_cast<uint2*>(dst + d0) = raw;
    return;
  }
  const float2 a = unpack_bf16x2(raw.x), b = unpack_bf16x2(raw.y);
  float x[4] = {a.x, a.y, b.x, b.y};
  const float sq[4] = {__fmul_rn(x[0], x[0]), __fmul_rn(x[1], x[1]), __fmul_rn(x[2], x[2]), __fmul_rn(x[3], x[3])};
  const float rs = rms_reciprocal(torch_order_sumsq_lane4(sq), p.eps);
  const uint2 wr = *reinterpret_cast<const uint2*>(w + d0);
  const float2 wa = unpack_bf16x2(wr.x), wb = unpack_bf16x2(wr.y);
  const float wv[4] = {wa.x, wa.y, wb.x, wb.y};
#pragma unroll
  for (int i = 0; i < 4; ++i) x[i] = bf16r(wv[i] * bf16r(x[i] * rs));
  const uint4 cs = *reinterpret_cast<const uint4*>(p.rope + static_cast<size_t>(row) * 64 + (d0 & 63));
  const uint32_t cw[4] = {cs.x, cs.y, cs.z, cs.w};
  const bool lower = lane < 16;             // d < 64: partner d + 64 is lane + 16
  float y[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float partner = __shfl_xor_sync(0xffffffffu, x[i], 16);
    const float2 c = unpack_bf16x2(cw[i]);  // .x cos, .y sin
    y[i] = lower ? bf16r(bf16r(x[i] * c.x) + bf16r(-partner * c.y)) : bf16r(bf16r(x[i] * c.x) + bf16r(partner * c.y));
  }
  uint2 res;
  res.x = pack_bf16x2(y[0], y[1]);
  res.y = pack_bf16x2(y[2], y[3]);
  *reinterpret_cast<uint2*>(dst + d0) = res;
}

struct CommitParams {
  uint4* resident_k;             // [layers * rows_per_layer, 8, 128] of bf16 or fp32
  uint4* resident_v;
  const uint4* scratch_k;        // [layers * scratch_rows, 8, 128]
  const uint4* scratch_v;
  int vec_per_row;               // 16-byte vectors per row: 128 (bf16) or 256 (fp32)
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
  const size_t vpr = static_cast<size_t>(p.vec_per_row);
  const size_t src_row = static_cast<size_t>(layer) * p.scratch_rows + q0;
  const size_t dst_row = static_cast<size_t>(layer) * p.rows_per_layer + p.slot_row[i] + c;
  const uint4* sk = p.scratch_k + src_row * vpr;
  const uint4* sv = p.scratch_v + src_row * vpr;
  uint4* dk = p.resident_k + dst_row * vpr;
  uint4* dv = p.resident_v + dst_row * vpr;
  for (size_t u = threadIdx.x; u < n * vpr; u += blockDim.x) {
    dk[u] = sk[u];
    dv[u] = sv[u];
  }
}

}  // namespace dspark
