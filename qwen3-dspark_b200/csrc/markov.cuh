// One step of the draft's serial Markov proposal (DSparkDraft._sample_greedy,
// dspark_qwen/model.py:210-221; batched as in packed_sampling.py:73-94):
//
//   emb      = markov_embedding[prev]                       [R, rank]
//   conf     = sigmoid(confidence(cat(hidden_k, emb)))     [R]   (before the token)
//   logits   = base_k + markov_projection(emb)             [R, V]
//   next     = argmax(logits)                               [R]
//
// with base_k = lm_head(hidden)[:, k] computed once per block by the caller. The
// [R, V] logits never reach HBM: a tcgen05 GEMM with M = requests (the gathered
// embeddings, padded to 128 rows), N = 128 vocabulary rows of the projection
// weight per tile and K = rank puts each logits tile in TMEM, where thread r
// (TMEM lane r) adds its base row, rounds like the reference's bf16 arithmetic
// (projection output to bf16, then the sum to bf16) and keeps a running
// first-maximum. Each CTA publishes one packed 64-bit atomicMax per request
// (order-preserving value bits high, inverted index low, so ties resolve to the
// lowest index); the last CTA to finish writes the tokens and clears the scratch.
//
// Roles (192 threads, persistent CTAs over the vocabulary tiles):
//   warps 0-3  gather emb rows into shared memory (A operand), confidence (one
//              warp per request, spread over the CTAs), epilogue (thread r =
//              request r = TMEM lane r);
//   warp 4     TMEM owner and MMA issuer (one thread);
//   warp 5     TMA producer of the projection-weight tiles (two stages).
#pragma once
#include "train.cuh"

namespace dspark {
namespace markov {

using train::instr_desc;
using train::smem_desc;
using train::tc_fence_after;
using train::tc_fence_before;
using train::tmem_alloc;
using train::tmem_dealloc;
using train::tmem_ld32;
using train::umma_bf16;
using train::umma_commit;
using train::wait_or_abort;

constexpr int kThreads = 192;
constexpr int kRows = 128;        // padded request rows (MMA M)
constexpr int kVocabTile = 128;   // vocabulary rows per tile (MMA N)
constexpr int kMaxRank = 256;
constexpr uint32_t kSmemA = 0;                           // 128 x rank bf16 (<= 64 KB)
constexpr uint32_t kSmemW = 65536;                       // 2 stages x 64 KB
constexpr uint32_t kSmemBar = kSmemW + 2 * 65536;
enum Barrier { kBarAReady = 0, kBarWFull0, kBarWFull1, kBarWEmpty0, kBarWEmpty1, kBarDFull0, kBarDFull1,
               kBarDFree0, kBarDFree1, kBarDrain, kNumBarriers };
constexpr uint32_t kSmemSlot = kSmemBar + kNumBarriers * 8;
constexpr uint32_t kSmemAbort = kSmemSlot + 4;
constexpr uint32_t kSmemLast = kSmemAbort + 4;
constexpr uint32_t kSmemBytes = 1024 + kSmemLast + 4;
constexpr uint32_t kTmemCols = 256;                      // two 128-column D buffers

struct Params {
  const __nv_bfloat16* emb_table;   // [V, rank] markov_embedding.weight
  const __nv_bfloat16* base;        // row (r * base_stride_r + k): lm_head logits of block row k, V wide
  long long base_stride_r;          // rows between requests in base (the block size)
  int k;                            // block position of this step
  const long long* prev;            // previous token of request r at prev[r * prev_stride]
  long long prev_stride;
  const __nv_bfloat16* hidden;      // [R * base_stride_r, H] backbone output (confidence input)
  int hidden_dim;
  const __nv_bfloat16* conf_w;      // [H + rank] confidence.weight
  float conf_b;
  long long* tokens;                // tokens[r * tok_stride + k] = next token
  long long tok_stride;
  float* conf;                      // conf[r * tok_stride + k] = sigmoid(confidence logit)
  unsigned long long* best;         // [kRows] packed maxima (zero between steps)
  unsigned int* arrivals;           // CTA arrival counter (zero between steps)
  int num_requests;                 // R <= 128
  int vocab;                        // V, multiple of 8
  int rank;                         // multiple of 64, <= 256
  int tiles;                        // ceil(V / 128)
};

// Unsigned key ordered like the float (for non-NaN values).
__device__ __forceinline__ unsigned int order_key(float f) {
  const unsigned int b = __float_as_uint(f);
  return (b & 0x80000000u) ? ~b : (b | 0x80000000u);
}

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__global__ void __launch_bounds__(kThreads, 1)
    markov_step_kernel(const __grid_constant__ CUtensorMap wmap, Params p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + kSmemBar;
  auto bar = [&](int i) { return bars + 8u * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmemAbort);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = p.rank / 64;                       // 64-wide K chunks (one 128-byte swizzle row each)
  const uint32_t tile_bytes = static_cast<uint32_t>(chunks) * 16384u;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBarriers; ++i) mbar_init(bar(i), (i == kBarAReady || i == kBarDFree0 || i == kBarDFree1) ? 128u : 1u);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5 && lane == 0) prefetch_tmap(&wmap);
  if (warp == 4) tmem_alloc(sbase + kSmemSlot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + kSmemSlot);
  const int n_mine = p.tiles > static_cast<int>(blockIdx.x)
                         ? (p.tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1 : 0;

  if (warp < 4) {
    // ---- gather emb rows (K-major, 128-byte swizzle) ---------------------------
    const int r = threadIdx.x;
    const bool live = r < p.num_requests;
    long long tok = 0;
    if (live) {
      tok = p.prev[r * p.prev_stride];
      if (tok < 0 || tok >= p.vocab) {
        atomicOr(&g_device_status, kStatusBadArgument);
        tok = 0;
      }
    }
    const uint4* src = reinterpret_cast<const uint4*>(p.emb_table + tok * p.rank);
    for (int c = 0; c < chunks; ++c)
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint4 v = live ? __ldg(src + c * 8 + j) : make_uint4(0, 0, 0, 0);
        *reinterpret_cast<uint4*>(smem + kSmemA + c * 16384 + r * 128 + ((j ^ (r & 7)) << 4)) = v;
      }
    fence_proxy_async_smem();
    mbar_arrive(bar(kBarAReady));
    // ---- confidence (before the token): request r on CTA r % grid, one warp ------
    for (int rr = static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) * warp; rr < p.num_requests;
         rr += 4 * static_cast<int>(gridDim.x)) {
      long long t = p.prev[rr * p.prev_stride];
      t = (t < 0 || t >= p.vocab) ? 0 : t;
      const __nv_bfloat16* h = p.hidden + (static_cast<long long>(rr) * p.base_stride_r + p.k) * p.hidden_dim;
      const __nv_bfloat16* em = p.emb_table + t * p.rank;
      float acc = 0.f;
      for (int i = lane; i < p.hidden_dim; i += 32)
        acc = fmaf(__bfloat162float(h[i]), __bfloat162float(p.conf_w[i]), acc);
      for (int i = lane; i < p.rank; i += 32)
        acc = fmaf(__bfloat162float(em[i]), __bfloat162float(p.conf_w[p.hidden_dim + i]), acc);
#pragma unroll
      for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
      if (lane == 0) {
        // bf16 Linear output (fp32 dot + bias, rounded once), then a bf16 sigmoid
        const float logit = bf16_round(acc + p.conf_b);
        p.conf[rr * p.tok_stride + p.k] = bf16_round(1.f / (1.f + expf(-logit)));
      }
    }
    // ---- epilogue: running first-maximum over this CTA's tiles --------------------
    float best_v = -INFINITY;
    int best_i = 0x7fffffff;
    const __nv_bfloat16* brow = p.base + (static_cast<long long>(r) * p.base_stride_r + p.k) * p.vocab;
    const uint32_t lane_addr = static_cast<uint32_t>(warp * 32) << 16;
    bool ok = true;
    for (int t = 0; t < n_mine; ++t) {
      const int b = t & 1;
      const int v0 = (static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x)) * kVocabTile;
      // this request's 128 base logits of the tile, loaded before the MMA result is
      // waited for so their latency overlaps it
      uint4 braw[16];
#pragma unroll
      for (int q = 0; q < 16; ++q)
        braw[q] = (live && v0 + q * 8 < p.vocab) ? __ldg(reinterpret_cast<const uint4*>(brow + v0 + q * 8))
                                                 : make_uint4(0, 0, 0, 0);
      ok = wait_or_abort(bar(kBarDFull0 + b), (t >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
#pragma unroll
      for (int c = 0; c < 4; ++c) {
        float d[32];
        tmem_ld32(tmem + lane_addr + b * 128 + c * 32, d);
        if (live) {
#pragma unroll
          for (int q = 0; q < 4; ++q) {
            const int v = v0 + c * 32 + q * 8;
            if (v >= p.vocab) break;
            const __nv_bfloat16* bv = reinterpret_cast<const __nv_bfloat16*>(&braw[c * 4 + q]);
#pragma unroll
            for (int e = 0; e < 8; ++e) {
              const float x = bf16_round(bf16_round(d[q * 8 + e]) + __bfloat162float(bv[e]));
              if (x > best_v || (x != x && best_v == best_v)) {
                best_v = x;
                best_i = v + e;
              }
            }
          }
        }
      }
      tc_fence_before();
      mbar_arrive(bar(kBarDFree0 + b));
    }
    if (!ok) *abort_flag = 1;
    if (live && best_i != 0x7fffffff)
      atomicMax(p.best + r, (static_cast<unsigned long long>(order_key(best_v)) << 32) |
                                static_cast<unsigned long long>(0xffffffffu - static_cast<unsigned int>(best_i)));
  } else if (warp == 4) {
    if (lane == 0) {
      constexpr uint32_t kIdesc = instr_desc(0);
      bool ok = wait_or_abort(bar(kBarAReady), 0, abort_flag);
      tc_fence_after();
      for (int t = 0; t < n_mine && ok; ++t) {
        const int st = t & 1, b = t & 1;
        if (!(ok = wait_or_abort(bar(kBarWFull0 + st), (t >> 1) & 1, abort_flag))) break;
        if (!(ok = wait_or_abort(bar(kBarDFree0 + b), ((t >> 1) & 1) ^ 1, abort_flag))) break;
        tc_fence_after();
        const uint32_t wbase = sbase + kSmemW + st * 65536;
        for (int kk = 0; kk < p.rank / 16; ++kk) {
          const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
          umma_bf16(tmem + b * 128, smem_desc(sbase + kSmemA + off, 16, 1024), smem_desc(wbase + off, 16, 1024),
                    kIdesc, kk > 0);
        }
        umma_commit(bar(kBarDFull0 + b));
        umma_commit(bar(kBarWEmpty0 + st));
      }
      if (!ok) *abort_flag = 1;
      umma_commit(bar(kBarDrain));
      volatile int never = 0;
      wait_or_abort(bar(kBarDrain), 0, &never);
    }
    __syncwarp();
  } else {
    if (lane == 0) {
      int armed[2] = {0, 0};
      bool ok = true;
      for (int t = 0; t < n_mine && ok; ++t) {
        const int st = t & 1;
        const int v0 = (static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x)) * kVocabTile;
        if (!(ok = wait_or_abort(bar(kBarWEmpty0 + st), ((t >> 1) & 1) ^ 1, abort_flag))) break;
        mbar_arrive_expect_tx(bar(kBarWFull0 + st), tile_bytes);
        for (int c = 0; c < chunks; ++c)
          tma_load_2d(sbase + kSmemW + st * 65536 + c * 16384, &wmap, c * 64, v0, bar(kBarWFull0 + st));
        ++armed[st];
      }
      if (!ok) *abort_flag = 1;
      volatile int never = 0;
      for (int st = 0; st < 2; ++st)
        if (armed[st]) wait_or_abort(bar(kBarWFull0 + st), (armed[st] - 1) & 1, &never);
    }
    __syncwarp();
  }

  // ---- the last CTA to arrive publishes the tokens and clears the scratch -------
  __threadfence();
  tc_fence_before();
  __syncthreads();
  volatile int* last = reinterpret_cast<volatile int*>(smem + kSmemLast);
  if (threadIdx.x == 0) *last = atomicAdd(p.arrivals, 1u) == gridDim.x - 1;
  __syncthreads();
  if (*last) {
    __threadfence();
    const int r = threadIdx.x;
    if (r < kRows) {
      const unsigned long long v = atomicExch(p.best + r, 0ull);
      if (r < p.num_requests)
        p.tokens[r * p.tok_stride + p.k] = static_cast<long long>(0xffffffffu - static_cast<unsigned int>(v));
    }
    if (threadIdx.x == 0) atomicExch(p.arrivals, 0u);
  }
  tc_fence_after();
  if (warp == 4) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace markov
}  // namespace dspark
