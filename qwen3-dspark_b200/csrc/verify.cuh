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

// cos/sin table of a verify transaction, shared by all layers: for new row r
// of request i (global row cu_q[i] + r, position ctx_len[i] + r) and frequency
// f: angle = float(position) * inv_freq[f] in float32, cos and sin rounded to
// bf16 and packed (cos low, sin high). Same values as the transformers rotary
// module computes once per forward (modeling_qwen3.py:137-148).
__global__ void __launch_bounds__(256) rope_table_kernel(const float* __restrict__ inv_freq, const int* cu_q,
                                                         const int* ctx_len, int num_requests, int total_q,
                                                         uint32_t* table) {
  const int row = blockIdx.x * 4 + (threadIdx.x >> 6);
  const int f = threadIdx.x & 63;
  if (row >= total_q) return;
  const int req = min(find_request(cu_q, num_requests + 1, row), num_requests - 1);
  const int pos = ctx_len[req] + (row - cu_q[req]);
  float sn, cs;
  sincosf(static_cast<float>(pos) * inv_freq[f], &sn, &cs);
  table[static_cast<size_t>(row) * 64 + f] = pack_bf16x2(cs, sn);
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
