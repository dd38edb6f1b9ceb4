// Fused draft-context append: every draft layer's k/v projection of the
// committed context rows, Qwen3 k_norm and rotate-half RoPE of k, and the write
// of both into the request-contiguous K/V pool, in one launch.
//
// The reference appends committed target features with
//   context = context_norm(fc(features))                  (packed_draft.py:129-168)
//   k, v    = project_kv(context, cos, sin) per layer     (model.py:41-45)
//           = rope(k_norm(k_proj(context))), v_proj(context)
// and concatenates them onto the cache. Here fc and context_norm stay library
// GEMM + elementwise work; this kernel does the rest: a tcgen05 GEMM of the
// context [rows, hidden] against the stacked projection weights
// [layers * 2 * 8 * 128, hidden] (layer l: k_proj rows then v_proj rows), whose
// N tiles of 128 are exactly one head of one layer's K or V. The accumulator of
// a tile stays in TMEM; thread m of the epilogue owns row m of the tile (TMEM
// lane m) and the head's 128 values, so k_norm (a 128-wide RMSNorm) and the
// rotate-half partner d +- 64 are thread-local. Rounding follows the
// reference's bf16 arithmetic: projection output to bf16, RMSNorm in fp32 then
// bf16, times the bf16 weight then bf16, RoPE products and sum each to bf16.
//
// Input row g belongs to request i with cu_rows[i] <= g < cu_rows[i + 1]; its
// position is ctx_len[i] + (g - cu_rows[i]) and it lands in pool row
// slot_row[i] + position when g - cu_rows[i] < count[i], else in trash_row
// (a row no request owns): a fixed-shape append of whole verified chunks then
// writes only the committed rows, with no host-side slicing.
//
// Roles (320 threads, persistent CTAs over (row tile, head tile) pairs; a head
// tile is kHeads consecutive heads of one layer's K or V, N = 128 kHeads):
//   warps 0-7  epilogue: warp w reads TMEM lanes 32(w%4).. (tile rows); a thread
//              drains one head of its row, all 128 columns, with four TMEM loads
//              and one wait (each wait costs about a microsecond while the tensor
//              pipe is busy), so k_norm's sum and each RoPE pair are thread-local.
//              With two heads per tile warp half w/4 takes head w/4 of every tile;
//              with one, the tiles of accumulator w/4 (every other tile);
//   warp 8     TMEM owner and MMA issuer (one thread), two accumulators of
//              128 kHeads columns so one tile's epilogue overlaps the next one's
//              MMAs;
//   warp 9     TMA producer: context and weight 64-wide K chunks (six stages
//              with one head per tile, four with two).
// Two heads per tile (large appends: prefill) halve the context bytes streamed
// from L2 per MMA flop; one head per tile keeps small appends spread over the SMs.
// The largest appends run the 2-SM version below (tiles of 256 rows x 2 heads).
#pragma once
#include "pair.cuh"
#include "train.cuh"
#include "verify.cuh"

namespace dspark {
namespace append {

using train::instr_desc;
using train::smem_desc;
using train::tc_fence_after;
using train::tc_fence_before;
using train::tmem_alloc;
using train::tmem_dealloc;
using train::tmem_ld32_async;
using train::tmem_ld_landed;
using train::tmem_ld_wait;
using train::umma_bf16;
using train::umma_commit;
using train::wait_or_abort;

constexpr int kEpilogueWarps = 8;
constexpr int kMmaWarp = kEpilogueWarps, kTmaWarp = kEpilogueWarps + 1;
constexpr int kThreads = (kEpilogueWarps + 2) * 32;
constexpr int kTileRows = 128;        // context rows per tile (MMA M)
constexpr int kHeadCols = 128;        // one head
constexpr int kMaxLayers = 8;

// Layout of the kernel with kHeads heads per tile (MMA N = 128 kHeads).
template <int kHeads>
struct Cfg {
  static constexpr int kStages = kHeads == 1 ? 6 : 4;
  static constexpr uint32_t kStageBytes = 16384 * (1 + kHeads);   // context chunk + weight chunk
  static constexpr uint32_t kSmemBar = kStages * kStageBytes;
  enum Barrier { kBarFull0 = 0, kBarEmpty0 = kStages, kBarDFull0 = 2 * kStages, kBarDFull1, kBarDFree0, kBarDFree1,
                 kBarDrain, kNumBarriers };
  static constexpr uint32_t kSmemSlot = kSmemBar + kNumBarriers * 8;
  static constexpr uint32_t kSmemAbort = kSmemSlot + 4;
  static constexpr uint32_t kSmemBytes = 1024 + kSmemAbort + 16;
  static constexpr uint32_t kAccCols = kHeadCols * kHeads;
  static constexpr uint32_t kTmemCols = 2 * kAccCols;
  // fp32 D, bf16 A and B, both K-major, M = 128, N = 128 kHeads
  static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((kAccCols >> 3) << 17) | ((128u >> 4) << 24);
};
static_assert(Cfg<1>::kSmemBytes <= 232448 && Cfg<2>::kSmemBytes <= 232448, "dynamic shared memory above 227 KB");
static_assert(Cfg<1>::kIdesc == instr_desc(0), "one-head tiles use the plain M128 N128 descriptor");

struct Params {
  const __nv_bfloat16* k_norm_w;      // [layers, 128] k_norm.weight of each layer
  const uint32_t* rope;               // [rows, 64]: bf16 cos | bf16 sin << 16 of row g's position
  const int* cu_rows;                 // [R + 1]
  const int* slot_row;                // [R] first pool row of the request's slot
  const int* ctx_len;                 // [R] position of the request's first input row
  const int* count;                   // [R] rows of the request that are written
  __nv_bfloat16* pool_k[kMaxLayers];  // [pool rows, 8, 128] per layer
  __nv_bfloat16* pool_v[kMaxLayers];
  long long trash_row;
  long long pool_rows;                // rows of every pool tensor (destinations are checked)
  int num_requests;
  int rows;                           // input rows
  int k_chunks;                       // hidden / 64
  int head_tiles;                     // layers * 16 / kHeads
  int row_tiles;
  int layers;
  float eps;
};

// bf16 pair helpers: value 2j in the low half, 2j + 1 in the high half.
__device__ __forceinline__ float bf_lo(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf_hi(uint32_t v) { return __uint_as_float(v & 0xffff0000u); }
// round-to-nearest-even bf16 products of two bf16 pairs (the exact product of two
// bf16 values fits a float, so this equals the float product rounded to bf16)
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ uint32_t perm(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

// The epilogue of one head of a tile for this thread's row (TMEM lane), all 128
// columns: four TMEM loads and one wait. V stored as projected (bf16); K rounded to
// bf16, k_norm'ed (sum of squares of the row's 128 bf16 values in four partial
// sums) and rotated with the row's cos/sin, each step rounded as the reference's
// bf16 ops round: x * rsqrt in float then bf16, the weight and cos/sin products
// bf16 x bf16 (one rounding), the rotation's sums in float then bf16.
// w2: the layer's k_norm weight as bf16 pairs; cs: the row's 64 cos|sin words.
// dest < 0: nothing is written (a padding row, or a rejected destination).
__device__ __forceinline__ void drain_row(const Params& p, uint32_t acc, __nv_bfloat16* out, bool is_v,
                                          const uint32_t* w2, const uint4* cs, long long dest) {
  uint32_t r0[32], r1[32], r2[32], r3[32];
  if (!is_v) {  // the row's 256 bytes of cos|sin into L1 while TMEM is read
    asm volatile("prefetch.global.L1 [%0];" ::"l"(cs));
    asm volatile("prefetch.global.L1 [%0];" ::"l"(cs + 8));
  }
  tmem_ld32_async(acc, r0);
  tmem_ld32_async(acc + 32, r1);
  tmem_ld32_async(acc + 64, r2);
  tmem_ld32_async(acc + 96, r3);
  tmem_ld_wait();
  tmem_ld_landed(r0);
  tmem_ld_landed(r1);
  tmem_ld_landed(r2);
  tmem_ld_landed(r3);
  uint32_t pk[64];                             // bf16 pairs (x[2i], x[2i + 1])
#pragma unroll
  for (int i = 0; i < 16; ++i) {
    pk[i] = pack_bf16x2(__uint_as_float(r0[2 * i]), __uint_as_float(r0[2 * i + 1]));
    pk[16 + i] = pack_bf16x2(__uint_as_float(r1[2 * i]), __uint_as_float(r1[2 * i + 1]));
    pk[32 + i] = pack_bf16x2(__uint_as_float(r2[2 * i]), __uint_as_float(r2[2 * i + 1]));
    pk[48 + i] = pack_bf16x2(__uint_as_float(r3[2 * i]), __uint_as_float(r3[2 * i + 1]));
  }
  if (!is_v) {
    float s[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const float lo = bf_lo(pk[i]), hi = bf_hi(pk[i]);
      s[i & 3] = fmaf(lo, lo, s[i & 3]);
      s[i & 3] = fmaf(hi, hi, s[i & 3]);
    }
    const float rs = 1.f / sqrtf(((s[0] + s[1]) + (s[2] + s[3])) / 128.f + p.eps);
    // pairs (2j, 2j + 1) rotate with (2j + 64, 2j + 65); two halves of 16 pairs, each
    // with its own cos|sin words and weights (the pointers pass through an empty
    // statement so that the second half's loads are not hoisted over the first half)
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      const uint4* csh = cs + 8 * h;                 // words of columns [32 h, 32 h + 32)
      const uint32_t* wh = w2 + 16 * h;              // weight pairs 16 h.. and 32 + 16 h..
      asm volatile("" : "+l"(csh), "+l"(wh));
      uint4 c[8], wa[4], wb[4];
#pragma unroll
      for (int q = 0; q < 8; ++q) c[q] = __ldg(csh + q);
#pragma unroll
      for (int q = 0; q < 4; ++q) {
        wa[q] = __ldg(reinterpret_cast<const uint4*>(wh) + q);
        wb[q] = __ldg(reinterpret_cast<const uint4*>(wh + 32) + q);
      }
#pragma unroll
      for (int jj = 0; jj < 16; ++jj) {
        const int j = 16 * h + jj;
        const uint32_t xa = pk[j], xb = pk[32 + j];
        const uint32_t ya = pack_bf16x2(bf_lo(xa) * rs, bf_hi(xa) * rs);
        const uint32_t yb = pack_bf16x2(bf_lo(xb) * rs, bf_hi(xb) * rs);
        const uint4 ua = wa[jj / 4], ub = wb[jj / 4];
        const uint32_t wpa = (jj & 3) == 0 ? ua.x : (jj & 3) == 1 ? ua.y : (jj & 3) == 2 ? ua.z : ua.w;
        const uint32_t wpb = (jj & 3) == 0 ? ub.x : (jj & 3) == 1 ? ub.y : (jj & 3) == 2 ? ub.z : ub.w;
        const uint32_t a2 = mul_bf16x2(wpa, ya), b2 = mul_bf16x2(wpb, yb);
        const uint4 cq = c[jj / 2];
        const uint32_t w0 = (jj & 1) ? cq.z : cq.x, w1 = (jj & 1) ? cq.w : cq.y;   // columns 2j, 2j + 1
        const uint32_t cos2 = perm(w0, w1, 0x5410u), sin2 = perm(w0, w1, 0x7632u);
        const uint32_t ac = mul_bf16x2(a2, cos2), bs = mul_bf16x2(b2, sin2);
        const uint32_t bc = mul_bf16x2(b2, cos2), as = mul_bf16x2(a2, sin2);
        pk[j] = pack_bf16x2(bf_lo(ac) - bf_lo(bs), bf_hi(ac) - bf_hi(bs));
        pk[32 + j] = pack_bf16x2(bf_lo(bc) + bf_lo(as), bf_hi(bc) + bf_hi(as));
      }
    }
  }
  if (dest >= 0) {
    uint4* d = reinterpret_cast<uint4*>(out);
#pragma unroll
    for (int q = 0; q < 16; ++q) d[q] = make_uint4(pk[4 * q], pk[4 * q + 1], pk[4 * q + 2], pk[4 * q + 3]);
  }
}

template <int kHeads>
__global__ void __launch_bounds__(kThreads, 1)
    draft_append_kernel(const __grid_constant__ CUtensorMap cmap, const __grid_constant__ CUtensorMap wmap,
                        Params p) {
  using C = Cfg<kHeads>;
  constexpr int kStages = C::kStages;
  constexpr uint32_t kStageBytes = C::kStageBytes, kSmemBar = C::kSmemBar, kSmemSlot = C::kSmemSlot;
  constexpr uint32_t kSmemAbort = C::kSmemAbort, kTmemCols = C::kTmemCols;
  constexpr uint32_t kAccCols = C::kAccCols;
  constexpr int kBarFull0 = C::kBarFull0, kBarEmpty0 = C::kBarEmpty0, kBarDFull0 = C::kBarDFull0;
  constexpr int kBarDFree0 = C::kBarDFree0, kBarDFree1 = C::kBarDFree1, kBarDrain = C::kBarDrain;
  constexpr int kNumBarriers = C::kNumBarriers;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + kSmemBar;
  auto bar = [&](int i) { return bars + 8u * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmemAbort);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // threads that release an accumulator: all epilogue threads with two heads per
  // tile (warp half h drains head h), half of them with one (warp half h drains
  // the tiles of accumulator h)
  constexpr uint32_t kFreeThreads = kEpilogueWarps * 32 / (kHeads == 1 ? 2 : 1);
  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBarriers; ++i)
      mbar_init(bar(i), (i == kBarDFree0 || i == kBarDFree1) ? kFreeThreads : 1u);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kTmaWarp && lane == 0) {
    prefetch_tmap(&cmap);
    prefetch_tmap(&wmap);
  }
  if (warp == kMmaWarp) tmem_alloc(sbase + kSmemSlot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + kSmemSlot);
  const int tiles = p.row_tiles * p.head_tiles;
  const int n_mine = tiles > static_cast<int>(blockIdx.x)
                         ? (tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1 : 0;

  if (warp < kEpilogueWarps) {
    const int quarter = warp & 3, half = warp >> 2;
    const int m = quarter * 32 + lane;                  // tile row of this thread
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;
    int cur_rt = -1;
    long long dest = -1;
    int g = 0;
    for (int t = kHeads == 1 ? half : 0; t < n_mine; t += kHeads == 1 ? 2 : 1) {
      const int b = t & 1;
      const int tile = static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x);
      const int rt = tile / p.head_tiles, ht = (tile - rt * p.head_tiles) * kHeads;   // first head tile
      const int layer = ht >> 4, is_v = (ht >> 3) & 1, head0 = ht & 7;
      if (rt != cur_rt) {                       // destination row of this thread's input row
        cur_rt = rt;
        g = rt * kTileRows + m;
        dest = -1;
        if (g < p.rows) {
          const int i = min(find_request(p.cu_rows, p.num_requests + 1, g), p.num_requests - 1);
          const int j = g - p.cu_rows[i];
          dest = j < p.count[i] ? static_cast<long long>(p.slot_row[i]) + p.ctx_len[i] + j : p.trash_row;
          if (dest < 0 || dest >= p.pool_rows) {
            atomicOr(&g_device_status, kStatusBadArgument);
            dest = -1;
          }
        }
      }
      ok = wait_or_abort(bar(kBarDFull0 + b), (t >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      {
        const int hh = kHeads == 1 ? 0 : half;
        const uint32_t acc = tmem + lane_addr + b * kAccCols + hh * kHeadCols;
        __nv_bfloat16* out = (is_v ? p.pool_v[layer] : p.pool_k[layer]) +
                             (dest < 0 ? 0 : dest) * (kKVHeads * kHeadDim) + (head0 + hh) * kHeadDim;
        const uint4* cs = reinterpret_cast<const uint4*>(p.rope + static_cast<size_t>(g < p.rows ? g : 0) * 64);
        drain_row(p, acc, out, is_v, reinterpret_cast<const uint32_t*>(p.k_norm_w + layer * kHeadDim), cs, dest);
      }
      tc_fence_before();
      mbar_arrive(bar(kBarDFree0 + b));
    }
    if (!ok) *abort_flag = 1;
  } else if (warp == kMmaWarp) {
    if (lane == 0) {
      constexpr uint32_t kIdesc = C::kIdesc;
      bool ok = true;
      int st = 0;
      uint32_t ph = 0;
      for (int t = 0; t < n_mine && ok; ++t) {
        const int b = t & 1;
        if (!(ok = wait_or_abort(bar(kBarDFree0 + b), ((t >> 1) & 1) ^ 1, abort_flag))) break;
        tc_fence_after();
        for (int c = 0; c < p.k_chunks; ++c) {
          if (!(ok = wait_or_abort(bar(kBarFull0 + st), ph, abort_flag))) break;
          tc_fence_after();
          const uint32_t a = sbase + st * kStageBytes, w = a + 16384;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + b * kAccCols, smem_desc(a + kk * 32, 16, 1024), smem_desc(w + kk * 32, 16, 1024),
                      kIdesc, (c | kk) != 0);
          umma_commit(bar(kBarEmpty0 + st));
          if (++st == kStages) {
            st = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(bar(kBarDFull0 + b));
      }
      if (!ok) *abort_flag = 1;
      umma_commit(bar(kBarDrain));
      volatile int never = 0;
      wait_or_abort(bar(kBarDrain), 0, &never);
    }
    __syncwarp();
  } else {
    if (lane == 0) {
      int armed[kStages] = {};
      bool ok = true;
      int st = 0;
      uint32_t ph = 0;
      for (int t = 0; t < n_mine && ok; ++t) {
        const int tile = static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x);
        const int rt = tile / p.head_tiles, ht = tile - rt * p.head_tiles;
        for (int c = 0; c < p.k_chunks; ++c) {
          if (!(ok = wait_or_abort(bar(kBarEmpty0 + st), ph ^ 1, abort_flag))) break;
          mbar_arrive_expect_tx(bar(kBarFull0 + st), kStageBytes);
          const uint32_t dst = sbase + st * kStageBytes;
          tma_load_2d(dst, &cmap, c * 64, rt * kTileRows, bar(kBarFull0 + st));
#pragma unroll
          for (int hh = 0; hh < kHeads; ++hh)           // the heads' weight rows, one after the other
            tma_load_2d(dst + 16384 * (1 + hh), &wmap, c * 64, (ht * kHeads + hh) * kHeadCols, bar(kBarFull0 + st));
          ++armed[st];
          if (++st == kStages) {
            st = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok) *abort_flag = 1;
      volatile int never = 0;
      for (int s = 0; s < kStages; ++s)
        if (armed[s]) wait_or_abort(bar(kBarFull0 + s), (armed[s] - 1) & 1, &never);
    }
    __syncwarp();
  }

  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kMmaWarp) tmem_dealloc(tmem, kTmemCols);
}

// ---------------------------------------------------------------------------
// 2-SM version for large appends: a cluster of two CTAs computes one tile of
// 256 context rows x 2 heads with tcgen05.mma.cta_group::2 (M = 256, N = 256):
// each CTA loads its own 128 context rows (the A operand) and ONE head's weight
// chunk (its half of B, rank r: head 2 ht + r), so every 16 KB of context and
// 16 KB of weights a CTA streams from L2 feeds 4.2 MFLOP, twice the single-CTA
// one-head tile. Each CTA's TMEM holds its 128 rows x both heads; its epilogue
// writes them. Rank 0 issues the MMAs; both CTAs' copies of a stage count their
// bytes on rank 0's full barrier (`.cta_group::2` loads, no multicast); MMA
// completion reaches both CTAs through multicast commits; the epilogue warps of
// both CTAs release an accumulator on rank 0's barrier. Every wait is bounded
// and both CTAs meet at a cluster barrier before TMEM is released.
// ---------------------------------------------------------------------------
struct PairCfg {
  static constexpr int kStages = 7;
  static constexpr uint32_t kStageBytes = 32768;    // own 128-row context chunk + own head's weight chunk
  static constexpr uint32_t kSmemBar = kStages * kStageBytes;
  enum Barrier { kBarFull0 = 0, kBarEmpty0 = kStages, kBarDFull0 = 2 * kStages, kBarDFull1,
                 kBarDFree0, kBarDFree1, kBarDrain, kNumBarriers };
  static constexpr uint32_t kSmemSlot = kSmemBar + kNumBarriers * 8;
  static constexpr uint32_t kSmemAbort = kSmemSlot + 4;
  // (the k_norm weights are read from global memory: seven stages leave no room)
  static constexpr uint32_t kSmemBytes = 1024 + kSmemAbort + 16;
  static constexpr uint32_t kAccCols = 2 * kHeadCols;
  static constexpr uint32_t kTmemCols = 2 * kAccCols;
  // fp32 D, bf16 A and B, both K-major, M = 256 (the pair), N = 256
  static constexpr uint32_t kIdesc = (1u << 4) | (1u << 7) | (1u << 10) | ((256u >> 3) << 17) | ((256u >> 4) << 24);
};
static_assert(PairCfg::kSmemBytes <= 232448, "dynamic shared memory above 227 KB");

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads, 1)
    draft_append_pair_kernel(const __grid_constant__ CUtensorMap cmap, const __grid_constant__ CUtensorMap wmap,
                             Params p) {
  using C = PairCfg;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + C::kSmemBar;
  auto bar = [&](int i) { return bars + 8u * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + C::kSmemAbort);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = pair::cluster_rank();
  const int pair_id = static_cast<int>(pair::cluster_index()), n_pairs = static_cast<int>(gridDim.x) / 2;

  if (threadIdx.x == 0) {
    for (int i = 0; i < C::kNumBarriers; ++i)
      mbar_init(bar(i), (i == C::kBarDFree0 || i == C::kBarDFree1) ? 2u * kEpilogueWarps : 1u);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kTmaWarp && lane == 0) {
    prefetch_tmap(&cmap);
    prefetch_tmap(&wmap);
  }
  if (warp == kMmaWarp) pair::tmem_alloc_pair(sbase + C::kSmemSlot, C::kTmemCols);
  tc_fence_before();
  __syncthreads();
  pair::cluster_sync();                 // both CTAs' barriers initialised, TMEM allocated
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + C::kSmemSlot);
  // tiles: (256-row pair tile rt, head pair ht); p.row_tiles / p.head_tiles count them
  const int tiles = p.row_tiles * p.head_tiles;
  const int n_mine = tiles > pair_id ? (tiles - 1 - pair_id) / n_pairs + 1 : 0;

  if (warp < kEpilogueWarps) {
    const int quarter = warp & 3, half = warp >> 2;
    const int m = quarter * 32 + lane;                  // tile row of this thread in this CTA
    const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
    bool ok = true;
    int cur_rt = -1;
    long long dest = -1;
    int g = 0;
    for (int t = 0; t < n_mine; ++t) {
      const int b = t & 1;
      const int tile = pair_id + t * n_pairs;
      const int rt = tile / p.head_tiles, ht = (tile - rt * p.head_tiles) * 2;   // first head tile
      const int layer = ht >> 4, is_v = (ht >> 3) & 1, head0 = ht & 7;
      if (rt != cur_rt) {                       // destination row of this thread's input row
        cur_rt = rt;
        g = rt * 2 * kTileRows + static_cast<int>(rank) * kTileRows + m;
        dest = -1;
        if (g < p.rows) {
          const int i = min(find_request(p.cu_rows, p.num_requests + 1, g), p.num_requests - 1);
          const int j = g - p.cu_rows[i];
          dest = j < p.count[i] ? static_cast<long long>(p.slot_row[i]) + p.ctx_len[i] + j : p.trash_row;
          if (dest < 0 || dest >= p.pool_rows) {
            atomicOr(&g_device_status, kStatusBadArgument);
            dest = -1;
          }
        }
      }
      ok = pair::pair_wait(bar(C::kBarDFull0 + b), (t >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) break;
      tc_fence_after();
      {  // warp half h drains head 2 ht + h of the tile, whole rows
        const uint32_t acc = tmem + lane_addr + b * C::kAccCols + half * kHeadCols;
        __nv_bfloat16* out = (is_v ? p.pool_v[layer] : p.pool_k[layer]) +
                             (dest < 0 ? 0 : dest) * (kKVHeads * kHeadDim) + (head0 + half) * kHeadDim;
        const uint4* cs = reinterpret_cast<const uint4*>(p.rope + static_cast<size_t>(g < p.rows ? g : 0) * 64);
        drain_row(p, acc, out, is_v, reinterpret_cast<const uint32_t*>(p.k_norm_w + layer * kHeadDim), cs, dest);
      }
      // one arrival per warp on rank 0's barrier once the warp's TMEM reads are done
      tc_fence_before();
      __syncwarp();
      if (lane == 0) pair::arrive_rank0(bar(C::kBarDFree0 + b));
    }
    if (!ok) *abort_flag = 1;
  } else if (warp == kMmaWarp) {
    if (lane == 0 && rank == 0) {
      bool ok = true;
      int st = 0;
      uint32_t ph = 0;
      for (int t = 0; t < n_mine && ok; ++t) {
        const int b = t & 1;
        if (!(ok = pair::pair_wait(bar(C::kBarDFree0 + b), ((t >> 1) & 1) ^ 1, abort_flag))) break;
        tc_fence_after();
        for (int c = 0; c < p.k_chunks; ++c) {
          if (!(ok = pair::pair_wait(bar(C::kBarFull0 + st), ph, abort_flag))) break;
          tc_fence_after();
          const uint32_t a = sbase + st * C::kStageBytes, w = a + 16384;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            pair::umma_pair_ss(tmem + b * C::kAccCols, smem_desc(a + kk * 32, 16, 1024),
                               smem_desc(w + kk * 32, 16, 1024), C::kIdesc, (c | kk) != 0);
          pair::umma_commit_pair(bar(C::kBarEmpty0 + st));
          if (++st == C::kStages) {
            st = 0;
            ph ^= 1;
          }
        }
        if (!ok) break;
        pair::umma_commit_pair(bar(C::kBarDFull0 + b));
      }
      if (!ok) *abort_flag = 1;
      pair::umma_commit_pair_local(bar(C::kBarDrain));
      volatile int never = 0;
      wait_or_abort(bar(C::kBarDrain), 0, &never);
    }
    __syncwarp();
  } else {
    if (lane == 0) {
      int issued = 0;
      bool ok = true;
      int st = 0;
      uint32_t ph = 0;
      for (int t = 0; t < n_mine && ok; ++t) {
        const int tile = pair_id + t * n_pairs;
        const int rt = tile / p.head_tiles, ht = tile - rt * p.head_tiles;
        for (int c = 0; c < p.k_chunks; ++c) {
          if (!(ok = pair::pair_wait(bar(C::kBarEmpty0 + st), ph ^ 1, abort_flag))) break;
          if (rank == 0) mbar_arrive_expect_tx(bar(C::kBarFull0 + st), 2 * C::kStageBytes);
          const uint32_t dst = sbase + st * C::kStageBytes, full = pair::cluster_addr(bar(C::kBarFull0 + st), 0);
          pair::tma_load_2d_pair(dst, &cmap, c * 64, (rt * 2 + static_cast<int>(rank)) * kTileRows, full);
          pair::tma_load_2d_pair(dst + 16384, &wmap, c * 64, (ht * 2 + static_cast<int>(rank)) * kHeadCols, full);
          ++issued;
          if (++st == C::kStages) {
            st = 0;
            ph ^= 1;
          }
        }
      }
      if (!ok) *abort_flag = 1;
      // Wait until the MMAs have released every stage (or, after an abort, until the
      // copies in flight have landed), so no commit or copy outlives this CTA.
      volatile int never = 0;
#pragma unroll 1
      for (int s2 = 0; s2 < C::kStages; ++s2) {
        const int armed = issued > s2 ? (issued - 1 - s2) / C::kStages + 1 : 0;
        if (armed && !pair::pair_wait(bar(C::kBarEmpty0 + s2), (armed - 1) & 1, ok ? &never : abort_flag)) {
          if (rank == 0) {
            wait_or_abort(bar(C::kBarFull0 + s2), (armed - 1) & 1, &never);
          } else {
            // rank 1's copies count on rank 0's barrier: after an abort it cannot see
            // them land, so it waits 1 ms (copies land in microseconds), once
            const uint64_t t0 = globaltimer();
            while (globaltimer() - t0 < 1000000ull) __nanosleep(1000);
            break;
          }
        }
      }
    }
    __syncwarp();
  }
  tc_fence_before();
  pair::cluster_sync();
  tc_fence_after();
  if (warp == kMmaWarp) pair::tmem_dealloc_pair(tmem, C::kTmemCols);
}

}  // namespace append
}  // namespace dspark
