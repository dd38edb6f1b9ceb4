// On-device greedy acceptance of one verify round.
//
// row_argmax_kernel: index of the maximum of every logits row (the target's
// greedy prediction for that verified position). Ties resolve to the lowest
// index and NaN counts as larger than any number, as torch.argmax does.
//
// greedy_accept_kernel: per request, the rule of cached_decode.py:84-98 /
// speculative.accept_greedy. The chunk of request i is [anchor, p_1 .. p_{Q-1}]
// at rows cu_q[i]..cu_q[i+1]-1 and pred[row] is the target's prediction after
// that row. Proposals are accepted while p_{j+1} == pred[j] (stopping after an
// accepted EOS); the first mismatch contributes the target's token instead, and
// a full accept contributes the bonus pred[Q-1]. The committed tokens are cut
// after their first EOS and to the request's remaining budget. n_commit is the
// number of verified rows whose KV is kept (anchor .. newest-1), i.e. the number
// of committed tokens, ready for dspark_commit_kv.
#pragma once
#include "ptx.cuh"

namespace dspark {

constexpr int kArgmaxThreads = 256;

struct ArgBest {
  float v;
  int i;
};

// a before b: larger value, NaN above numbers, lower index on ties.
__device__ __forceinline__ bool arg_better(const ArgBest& a, const ArgBest& b) {
  const bool an = a.v != a.v, bn = b.v != b.v;
  if (an != bn) return an;
  if (!an && a.v != b.v) return a.v > b.v;
  return a.i < b.i;
}

template <typename T>
__device__ __forceinline__ float to_f32(T x);
template <>
__device__ __forceinline__ float to_f32<float>(float x) { return x; }
template <>
__device__ __forceinline__ float to_f32<__nv_bfloat16>(__nv_bfloat16 x) { return __bfloat162float(x); }

// A thread visits its elements in increasing index order, so a strict '>'
// keeps the first maximum; a NaN replaces any number and is kept thereafter.
__device__ __forceinline__ void scan_one(ArgBest& best, float x, int idx) {
  if (x > best.v || (x != x && best.v == best.v)) best = ArgBest{x, idx};
}

// One CTA of 256 threads per row (eight per SM: a config-3 round's 896 rows are
// all resident at once; 512-thread CTAs left a half-occupied second wave and
// measured 7% slower); 4 independent 16-byte loads in flight per thread when the
// row start is 16-byte aligned (the element tail and unaligned rows go scalar).
template <typename T>
__global__ void __launch_bounds__(kArgmaxThreads) row_argmax_kernel(const T* __restrict__ logits, long long ld,
                                                                    int vocab, int* __restrict__ pred) {
  constexpr int kVec = 16 / sizeof(T), kUnroll = 4;
  const T* row = logits + static_cast<long long>(blockIdx.x) * ld;
  ArgBest best{-INFINITY, 0x7fffffff};
  const bool vec = (reinterpret_cast<uintptr_t>(row) & 15) == 0;
  int i0 = 0;
  if (vec) {
    const int nvec = vocab / kVec;
    const uint4* rv = reinterpret_cast<const uint4*>(row);
    // vector base + j*kArgmaxThreads + t: coalesced loads, increasing index per thread
    int base = 0;
    for (; base + kArgmaxThreads * kUnroll <= nvec; base += kArgmaxThreads * kUnroll) {
      uint4 raw[kUnroll];
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) raw[j] = __ldg(rv + base + j * kArgmaxThreads + threadIdx.x);
#pragma unroll
      for (int j = 0; j < kUnroll; ++j) {
        const T* x = reinterpret_cast<const T*>(&raw[j]);
        const int v0 = (base + j * kArgmaxThreads + threadIdx.x) * kVec;
#pragma unroll
        for (int e = 0; e < kVec; ++e) scan_one(best, to_f32(x[e]), v0 + e);
      }
    }
    for (int k = base + threadIdx.x; k < nvec; k += kArgmaxThreads) {
      const uint4 raw = __ldg(rv + k);
      const T* x = reinterpret_cast<const T*>(&raw);
#pragma unroll
      for (int e = 0; e < kVec; ++e) scan_one(best, to_f32(x[e]), k * kVec + e);
    }
    i0 = nvec * kVec;
  }
  for (int k = i0 + threadIdx.x; k < vocab; k += kArgmaxThreads) {
    const ArgBest c{to_f32(row[k]), k};
    if (arg_better(c, best)) best = c;
  }
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const ArgBest c{__shfl_xor_sync(0xffffffffu, best.v, o), __shfl_xor_sync(0xffffffffu, best.i, o)};
    if (arg_better(c, best)) best = c;
  }
  __shared__ ArgBest warp_best[kArgmaxThreads / 32];
  if ((threadIdx.x & 31) == 0) warp_best[threadIdx.x >> 5] = best;
  __syncthreads();
  if (threadIdx.x == 0) {
    ArgBest b = warp_best[0];
    for (int w = 1; w < kArgmaxThreads / 32; ++w)
      if (arg_better(warp_best[w], b)) b = warp_best[w];
    pred[blockIdx.x] = b.i == 0x7fffffff ? 0 : b.i;   // a row of -inf only: its first index, as torch.argmax
  }
}

struct AcceptParams {
  const int* pred;              // [N] argmax per verified row
  const long long* tokens;      // [N] chunk tokens (anchor first)
  const int32_t* cu_q;          // [R+1]
  const long long* eos;         // [n_eos]
  int n_eos;
  const int32_t* budget;        // [R] tokens each request may still emit, or null
  int num_requests;
  int total_rows;
  int32_t* accepted;            // [R] accepted proposals
  int32_t* n_commit;            // [R] committed tokens = verified rows kept
  long long* emitted;           // [N] committed tokens at the request's rows (rest -1)
};

__device__ __forceinline__ bool is_eos(const AcceptParams& p, long long t) {
  for (int e = 0; e < p.n_eos; ++e)
    if (p.eos[e] == t) return true;
  return false;
}

// One thread per request.
__global__ void greedy_accept_kernel(AcceptParams p) {
  const int r = blockIdx.x * blockDim.x + threadIdx.x;
  if (r >= p.num_requests) return;
  const int q0 = p.cu_q[r], q1 = p.cu_q[r + 1];
  if (q0 < 0 || q1 <= q0 || q1 > p.total_rows) {
    atomicOr(&g_device_status, kStatusBadArgument);
    p.accepted[r] = 0;
    p.n_commit[r] = 0;
    return;
  }
  const int q = q1 - q0;
  int acc = 0, n = 0;
  bool stop = false;
  for (int j = 0; j + 1 < q && !stop; ++j) {
    const long long proposed = p.tokens[q0 + 1 + j];
    const long long correct = static_cast<long long>(p.pred[q0 + j]);
    if (proposed != correct) {
      p.emitted[q0 + n++] = correct;
      stop = true;
      break;
    }
    p.emitted[q0 + n++] = proposed;
    ++acc;
    if (is_eos(p, proposed)) stop = true;
  }
  if (!stop) p.emitted[q0 + n++] = static_cast<long long>(p.pred[q1 - 1]);
  // cut after the first EOS, then to the budget
  for (int k = 0; k < n; ++k)
    if (is_eos(p, p.emitted[q0 + k])) {
      n = k + 1;
      break;
    }
  if (p.budget != nullptr) n = min(n, max(0, p.budget[r]));
  for (int k = n; k < q; ++k) p.emitted[q0 + k] = -1;
  p.accepted[r] = acc;
  p.n_commit[r] = n;
}

}  // namespace dspark
