// The draft's serial Markov proposal (DSparkDraft._sample_greedy,
// dspark_qwen/model.py:210-221; batched as in packed_sampling.py:73-94). Step k:
//
//   emb      = markov_embedding[prev]                       [R, rank]
//   conf     = sigmoid(confidence(cat(hidden_k, emb)))     [R]   (before the token)
//   logits   = base_k + markov_projection(emb)             [R, V]
//   next     = argmax(logits)                               [R]   (prev of step k+1)
//
// with base_k = lm_head(hidden)[:, k] computed once per block by the caller. The
// [R, V] logits never reach HBM: a tcgen05 GEMM with M = requests (the gathered
// embeddings, padded to 128 rows), N = 128 vocabulary rows of the projection
// weight per tile and K = rank puts each logits tile in TMEM, where thread r
// (TMEM lane r) adds its base row, rounds like the reference's bf16 arithmetic
// (projection output to bf16, then the sum to bf16) and keeps a running
// first-maximum: each bf16 logit becomes an order-preserving 16-bit key (-0
// folded onto +0, NaN above everything, as torch.argmax orders them) packed
// above its inverted column, so one unsigned max per value keeps the largest
// value at its lowest index. Each CTA publishes one packed 64-bit atomicMax per
// request (key high, inverted index low).
//
// Two kernels share this body:
//   markov_step_kernel   one step per launch; the last CTA to finish writes the
//                        tokens and clears the scratch;
//   markov_block_kernel  all steps of a block in one cooperative launch (every
//                        CTA resident): the projection-weight stream runs on
//                        across steps (it does not depend on the tokens), and
//                        between steps the CTAs meet at a grid barrier (a
//                        generation counter with a bounded wait) after which
//                        every CTA reads the step's argmax for its next gather.
//                        Step s publishes into best buffer s % 3; CTA 0 writes
//                        the tokens and clears the buffer of step s - 2 during
//                        step s (all CTAs finished reading it before the
//                        barrier of step s - 1).
//
// Roles (192 threads, persistent CTAs over the vocabulary tiles):
//   warps 0-3  per step: gather emb rows into shared memory (A operand),
//              confidence (one warp per request, spread over the CTAs),
//              epilogue (thread m = TMEM lane m; the base row of the next tile
//              is loaded while the current tile is reduced). With at most 64
//              requests request r fills rows r and r + 64, and the threads of
//              the two rows reduce one half of the columns each, so all four
//              warps (TMEM lane quarters) do useful work;
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
using train::tmem_st32;
using train::umma_bf16_ts;
using train::umma_commit;
using train::wait_or_abort;

constexpr int kThreads = 192;
constexpr int kRows = 128;        // padded request rows (MMA M)
constexpr int kVocabTile = 128;   // vocabulary rows per tile (MMA N)
constexpr int kMaxRank = 256;
constexpr int kMaxSteps = 64;     // block positions per fused launch
constexpr int kWStages = 3;
constexpr uint32_t kSmemW = 0;                           // 3 stages x 64 KB (128 vocabulary rows x rank)
constexpr uint32_t kSmemBar = kSmemW + kWStages * 65536;
enum Barrier { kBarAReady = 0, kBarAFree, kBarWFull0, kBarWEmpty0 = kBarWFull0 + kWStages,
               kBarDFull0 = kBarWEmpty0 + kWStages, kBarDFull1, kBarDFree0, kBarDFree1, kBarDrain, kNumBarriers };
constexpr uint32_t kSmemSlot = kSmemBar + kNumBarriers * 8;
constexpr uint32_t kSmemAbort = kSmemSlot + 4;
constexpr uint32_t kSmemLast = kSmemAbort + 4;
constexpr uint32_t kSmemBytes = 1024 + kSmemLast + 4;
// TMEM: two 128-column D buffers, then the A operand (the gathered embedding
// rows, bf16 pairs: column j of lane m = elements 2j, 2j+1 of row m).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemA = 256;
// Scratch (zero between calls): three best buffers of kRows packed maxima, then four
// 32-bit words: the CTA arrival counter, the grid-barrier generation (the only word
// that is not returned to zero: it only ever advances), the CTA exit counter and the
// failed flag of the block kernel (a CTA gave up; the last CTA out resets the scratch).
constexpr size_t kScratchBytes = 3 * kRows * sizeof(unsigned long long) + 16;

struct Params {
  const __nv_bfloat16* emb_table;   // [V, rank] markov_embedding.weight
  const __nv_bfloat16* base;        // row (r * base_stride_r + k): lm_head logits of block row k, V wide
  long long base_stride_r;          // rows between requests in base (the block size)
  int k;                            // block position of this step (step kernel)
  int steps;                        // block positions 0 .. steps-1 (block kernel)
  const long long* prev;            // previous token of request r at prev[r * prev_stride] (step k / step 0)
  long long prev_stride;
  const __nv_bfloat16* hidden;      // [R * base_stride_r, H] backbone output (confidence input)
  int hidden_dim;
  int conf_vec;                     // hidden rows, conf_w and hidden_dim allow 16-byte loads
  const __nv_bfloat16* conf_w;      // [H + rank] confidence.weight
  float conf_b;
  long long* tokens;                // tokens[r * tok_stride + k] = next token
  long long tok_stride;
  float* conf;                      // conf[r * tok_stride + k] = sigmoid(confidence logit)
  unsigned long long* best;         // 3 x [kRows] packed maxima (zero between calls)
  unsigned int* arrivals;           // CTA arrival counter (zero between calls)
  unsigned int* generation;         // grid-barrier generation
  unsigned int* exits;              // CTAs that left the block kernel (zero between calls)
  unsigned int* failed;             // a CTA of the block kernel gave up (zero between calls)
  int num_requests;                 // R <= 128
  int dup;                          // R <= 64: request r also in row r + 64 (column halves split)
  int vocab;                        // V, multiple of 8
  int rank;                         // multiple of 64, <= 256
  int tiles;                        // ceil(V / 128)
};

__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// Two bf16 values (lo, hi halves) -> two 16-bit keys ordered like the values:
// -0 is first turned into +0 (they compare equal), then negative values map to
// ~b and others to b | 0x8000. A canonical NaN (0x7fff, what the conversions
// produce) gets the largest key; no value gets key 0.
__device__ __forceinline__ uint32_t bf16x2_order_keys(uint32_t b) {
  const uint32_t nonzero = ((b & 0x7fff7fffu) + 0x7fff7fffu) & 0x80008000u;   // bit 15: magnitude != 0
  b &= nonzero | 0x7fff7fffu;
  const uint32_t neg = (b >> 15) & 0x00010001u;
  return b ^ ((neg * 0x7fffu) | 0x80008000u);
}

// 32 lanes x 64 fp32 columns from TMEM (two loads, one wait).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  float (&a)[32] = *reinterpret_cast<float(*)[32]>(&v[0]);
  float (&b)[32] = *reinterpret_cast<float(*)[32]>(&v[32]);
  uint32_t ra[32], rb[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%64];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,"
      "%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%65];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(ra[0]), "=r"(ra[1]), "=r"(ra[2]), "=r"(ra[3]), "=r"(ra[4]), "=r"(ra[5]), "=r"(ra[6]), "=r"(ra[7]),
        "=r"(ra[8]), "=r"(ra[9]), "=r"(ra[10]), "=r"(ra[11]), "=r"(ra[12]), "=r"(ra[13]), "=r"(ra[14]), "=r"(ra[15]),
        "=r"(ra[16]), "=r"(ra[17]), "=r"(ra[18]), "=r"(ra[19]), "=r"(ra[20]), "=r"(ra[21]), "=r"(ra[22]), "=r"(ra[23]),
        "=r"(ra[24]), "=r"(ra[25]), "=r"(ra[26]), "=r"(ra[27]), "=r"(ra[28]), "=r"(ra[29]), "=r"(ra[30]), "=r"(ra[31]),
        "=r"(rb[0]), "=r"(rb[1]), "=r"(rb[2]), "=r"(rb[3]), "=r"(rb[4]), "=r"(rb[5]), "=r"(rb[6]), "=r"(rb[7]),
        "=r"(rb[8]), "=r"(rb[9]), "=r"(rb[10]), "=r"(rb[11]), "=r"(rb[12]), "=r"(rb[13]), "=r"(rb[14]), "=r"(rb[15]),
        "=r"(rb[16]), "=r"(rb[17]), "=r"(rb[18]), "=r"(rb[19]), "=r"(rb[20]), "=r"(rb[21]), "=r"(rb[22]), "=r"(rb[23]),
        "=r"(rb[24]), "=r"(rb[25]), "=r"(rb[26]), "=r"(rb[27]), "=r"(rb[28]), "=r"(rb[29]), "=r"(rb[30]), "=r"(rb[31])
      : "r"(taddr), "r"(taddr + 32)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) {
    a[i] = __uint_as_float(ra[i]);
    b[i] = __uint_as_float(rb[i]);
  }
}

// Token of a packed maximum.
__device__ __forceinline__ long long packed_token(unsigned long long v) {
  return static_cast<long long>(0xffffffffu - static_cast<unsigned int>(v));
}

__device__ __forceinline__ long long checked_token(const Params& p, long long t) {
  if (t < 0 || t >= p.vocab) {
    atomicOr(&g_device_status, kStatusBadArgument);
    return 0;
  }
  return t;
}

// TMEM lane m of the A operand (warp-collective: the warp writes its 32 lanes):
// the embedding of `tok`, or zeros for a padding row.
__device__ __forceinline__ void gather_row(const Params& p, uint32_t a_tmem, long long tok, bool live) {
  const uint4* src = reinterpret_cast<const uint4*>(p.emb_table + tok * p.rank);
  const int chunks = p.rank / 64;                  // 32 TMEM columns (64 elements) each
  uint4 v[kMaxRank / 8];                           // every load in flight before the first store
#pragma unroll
  for (int i = 0; i < kMaxRank / 8; ++i) v[i] = live && i < chunks * 8 ? __ldg(src + i) : make_uint4(0, 0, 0, 0);
#pragma unroll
  for (int c = 0; c < kMaxRank / 64; ++c)
    if (c < chunks) tmem_st32(a_tmem + 32 * c, *reinterpret_cast<const float(*)[32]>(&v[8 * c]));
}

// Confidence of block position k (before its token) for the requests of this
// CTA (request r on CTA grid - 1 - r % grid, one warp each: the last CTAs own
// the fewest vocabulary tiles); prev_of(rr) is request rr's previous token.
template <class PrevFn>
__device__ __forceinline__ void confidence_rows(const Params& p, int k, int warp, int lane, PrevFn prev_of) {
  const int from_end = static_cast<int>(gridDim.x) - 1 - static_cast<int>(blockIdx.x);
  for (int rr = from_end + static_cast<int>(gridDim.x) * warp; rr < p.num_requests;
       rr += 4 * static_cast<int>(gridDim.x)) {
    const long long t = prev_of(rr);
    const __nv_bfloat16* h = p.hidden + (static_cast<long long>(rr) * p.base_stride_r + k) * p.hidden_dim;
    const __nv_bfloat16* em = p.emb_table + t * p.rank;
    float acc = 0.f;
    if (p.conf_vec) {
      // 8 bf16 per 16-byte load, all of a lane's loads in flight together
      auto dot8 = [](uint4 a, uint4 b, float acc) {
        const __nv_bfloat16* x = reinterpret_cast<const __nv_bfloat16*>(&a);
        const __nv_bfloat16* y = reinterpret_cast<const __nv_bfloat16*>(&b);
#pragma unroll
        for (int e = 0; e < 8; ++e) acc = fmaf(__bfloat162float(x[e]), __bfloat162float(y[e]), acc);
        return acc;
      };
#pragma unroll 4
      for (int i = lane * 8; i < p.hidden_dim; i += 256)
        acc = dot8(__ldg(reinterpret_cast<const uint4*>(h + i)), __ldg(reinterpret_cast<const uint4*>(p.conf_w + i)),
                   acc);
#pragma unroll 2
      for (int i = lane * 8; i < p.rank; i += 256)
        acc = dot8(__ldg(reinterpret_cast<const uint4*>(em + i)),
                   __ldg(reinterpret_cast<const uint4*>(p.conf_w + p.hidden_dim + i)), acc);
    } else {
      for (int i = lane; i < p.hidden_dim; i += 32)
        acc = fmaf(__bfloat162float(h[i]), __bfloat162float(p.conf_w[i]), acc);
      for (int i = lane; i < p.rank; i += 32)
        acc = fmaf(__bfloat162float(em[i]), __bfloat162float(p.conf_w[p.hidden_dim + i]), acc);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if (lane == 0) {
      // bf16 Linear output (fp32 dot + bias, rounded once), then a bf16 sigmoid
      const float logit = bf16_round(acc + p.conf_b);
      p.conf[rr * p.tok_stride + k] = bf16_round(1.f / (1.f + expf(-logit)));
    }
  }
}

// Request r's base logits of tile t at block position k, columns c0 .. c0 +
// 64 nh - 1 of the tile (raw[q] = columns c0 + 8q ..; zeros past the vocabulary
// or for padding rows).
__device__ __forceinline__ void load_base(const Params& p, int k, int t, int n_mine, int r, bool live, int c0,
                                          int nh, uint4 (&raw)[16]) {
  const __nv_bfloat16* brow = p.base + (static_cast<long long>(r) * p.base_stride_r + k) * p.vocab;
  const int v0 = (static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x)) * kVocabTile + c0;
#pragma unroll
  for (int q = 0; q < 16; ++q)
    raw[q] = (live && t < n_mine && q < nh * 8 && v0 + q * 8 < p.vocab)
                 ? __ldg(reinterpret_cast<const uint4*>(brow + v0 + q * 8)) : make_uint4(0, 0, 0, 0);
}

// Epilogue of one step over this CTA's n_mine tiles (global tile counter g0 ..):
// the first maximum of request r's logits (best_key / best_idx, key 0 = none).
// bnext holds the base logits of the step's first tile on entry; each tile's are
// loaded one tile ahead of the MMA result they are added to, and the last tile
// loads the first tile of block position k_next (if >= 0), so their DRAM latency
// overlaps other work.
__device__ __forceinline__ bool epilogue_step(const Params& p, int k, int k_next, int g0, int n_mine, int r,
                                              bool live, int c0, int nh, uint32_t tmem, uint32_t bars,
                                              volatile int* abort_flag, uint4 (&bnext)[16], uint32_t& best_key,
                                              int& best_idx) {
  auto bar = [&](int i) { return bars + 8u * i; };
  const int warp = threadIdx.x >> 5;
  best_key = 0;
  best_idx = 0x7fffffff;
  const uint32_t lane_addr = static_cast<uint32_t>(warp * 32) << 16;
  for (int t = 0; t < n_mine; ++t) {
    const int g = g0 + t, b = g & 1;
    const int v0 = (static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x)) * kVocabTile;
    const int nvalid = min(kVocabTile, p.vocab - v0);   // the last tile may be partial
    uint4 braw[16];
#pragma unroll
    for (int q = 0; q < 16; ++q) braw[q] = bnext[q];
    if (t + 1 < n_mine)
      load_base(p, k, t + 1, n_mine, r, live, c0, nh, bnext);
    else if (k_next >= 0)
      load_base(p, k_next, 0, n_mine, r, live, c0, nh, bnext);
    const bool ok = wait_or_abort(bar(kBarDFull0 + b), (g >> 1) & 1, abort_flag);
    if (!__all_sync(0xffffffffu, ok)) return false;
    tc_fence_after();
    // running maxima of packed (key << 16 | 127 - column) over this thread's
    // columns c0 .. (two independent chains per 64 columns)
    uint32_t chain[4] = {0u, 0u, 0u, 0u};
#pragma unroll
    for (int h = 0; h < 2; ++h) {
      if (h >= nh) break;
      float d[64];
      tmem_ld64(tmem + lane_addr + b * 128 + c0 + h * 64, d);
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const int lc = h * 64 + 2 * i;             // column relative to c0 (static)
        const int col = c0 + lc;
        // projection output to bf16, plus the bf16 base logit, sum to bf16
        const uint32_t r1 = pack_bf16x2(d[2 * i], d[2 * i + 1]);
        const uint4& bq = braw[lc >> 3];
        const uint32_t bb = ((lc & 7) >> 1) == 0 ? bq.x : ((lc & 7) >> 1) == 1 ? bq.y
                          : ((lc & 7) >> 1) == 2 ? bq.z : bq.w;
        const float s0 = __uint_as_float(r1 << 16) + __uint_as_float(bb << 16);
        const float s1 = __uint_as_float(r1 & 0xffff0000u) + __uint_as_float(bb & 0xffff0000u);
        const uint32_t key = bf16x2_order_keys(pack_bf16x2(s0, s1));
        uint32_t p0 = (key << 16) | static_cast<uint32_t>(127 - col);
        uint32_t p1 = (key & 0xffff0000u) | static_cast<uint32_t>(126 - col);
        if (nvalid < kVocabTile) {
          p0 = col < nvalid ? p0 : 0u;
          p1 = col + 1 < nvalid ? p1 : 0u;
        }
        chain[lc >> 5] = max(chain[lc >> 5], max(p0, p1));
      }
    }
    tc_fence_before();
    mbar_arrive(bar(kBarDFree0 + b));
    const uint32_t tb = max(max(chain[0], chain[1]), max(chain[2], chain[3]));
    if (live && (tb >> 16) > best_key) {
      best_key = tb >> 16;
      best_idx = v0 + 127 - static_cast<int>(tb & 0xffffu);
    }
  }
  return true;
}

__device__ __forceinline__ void publish(const Params& p, unsigned long long* best, int r, bool live,
                                        uint32_t best_key, int best_idx) {
  if (live && best_idx != 0x7fffffff)
    atomicMax(best + r, (static_cast<unsigned long long>(best_key) << 32) |
                            static_cast<unsigned long long>(0xffffffffu - static_cast<unsigned int>(best_idx)));
}

// The four epilogue warps meet (a named barrier they all reach on every path).
__device__ __forceinline__ void epilogue_sync() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Grid barrier of the cooperative block kernel, run by thread 0 of each CTA:
// the last CTA to arrive resets the counter and advances the generation; the
// others wait (bounded) for the generation to change.
__device__ __forceinline__ void grid_barrier(const Params& p, volatile int* abort_flag) {
  if (*abort_flag) return;                         // the other CTAs' waits run out and report it
  volatile unsigned int* gen = p.generation;
  const unsigned int g = *gen;
  __threadfence();
  if (atomicAdd(p.arrivals, 1u) == gridDim.x - 1) {
    atomicExch(p.arrivals, 0u);
    __threadfence();
    atomicAdd(p.generation, 1u);
    return;
  }
  // A lowered limit (a failure-handling test) is checked on every poll, so that a wait
  // shorter than 64 polls gives up too; the default one every 64 polls.
  const unsigned long long limit = g_grid_barrier_limit_ns;
  const uint32_t every = limit < kWaitLimitNs ? 0u : 63u;
  const unsigned long long t0 = globaltimer();
  for (uint32_t it = 1; *gen == g; ++it) {
    if ((it & every) == 0 && globaltimer() - t0 >= limit) {
      atomicOr(&g_device_status, kStatusWaitTimeout);
      *abort_flag = 1;
      return;
    }
  }
  __threadfence();
}

template <bool kBlock>
__device__ __forceinline__ void markov_body(const CUtensorMap* wmap, const Params& p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + kSmemBar;
  auto bar = [&](int i) { return bars + 8u * i; };
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmemAbort);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int chunks = p.rank / 64;                       // 64-wide K chunks (one 128-byte swizzle row each)
  const uint32_t tile_bytes = static_cast<uint32_t>(chunks) * 16384u;
  const int steps = kBlock ? p.steps : 1;

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBarriers; ++i)
      mbar_init(bar(i), (i == kBarAReady || i == kBarDFree0 || i == kBarDFree1) ? 128u : 1u);
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == 5 && lane == 0) prefetch_tmap(wmap);
  if (warp == 4) tmem_alloc(sbase + kSmemSlot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + kSmemSlot);
  const int n_mine = p.tiles > static_cast<int>(blockIdx.x)
                         ? (p.tiles - 1 - static_cast<int>(blockIdx.x)) / static_cast<int>(gridDim.x) + 1 : 0;

  if (warp < 4) {
    const int m = threadIdx.x;                     // A row / TMEM lane
    const int r = p.dup ? (m & 63) : m;            // its request
    const bool live = r < p.num_requests;
    const int c0 = p.dup ? (m >> 6) * 64 : 0, nh = p.dup ? 1 : 2;   // its columns
    uint4 bnext[16];                               // base logits of the next tile to reduce
    load_base(p, kBlock ? 0 : p.k, 0, n_mine, r, live, c0, nh, bnext);
    for (int s = 0; s < steps; ++s) {
      const int k = kBlock ? s : p.k;
      unsigned long long* const best_now = p.best + (kBlock ? (s % 3) * kRows : 0);
      const unsigned long long* const best_prev = p.best + ((s + 2) % 3) * kRows;
      // previous token of request rr: the given one, or (block kernel, s > 0)
      // the argmax of step s - 1, read past L1 (other CTAs wrote it)
      auto prev_of = [&](int rr) -> long long {
        if (!kBlock || s == 0) return checked_token(p, p.prev[rr * p.prev_stride]);
        return checked_token(p, packed_token(__ldcg(best_prev + rr)));
      };
      const long long tok = live ? prev_of(r) : 0;
      // the A operand is free once the previous step's MMAs are done (decisions are
      // warp-uniform: the confidence and the TMEM loads are warp-collective)
      bool ok = __all_sync(0xffffffffu, !*abort_flag);
      if (ok && s > 0) ok = __all_sync(0xffffffffu, wait_or_abort(bar(kBarAFree), (s - 1) & 1, abort_flag));
      tc_fence_after();
      if (ok) gather_row(p, tmem + (static_cast<uint32_t>(warp * 32) << 16) + kTmemA, tok, live);
      tc_fence_before();
      mbar_arrive(bar(kBarAReady));
      if (kBlock && blockIdx.x == 0) {
        if (s > 0 && live && m == r) p.tokens[r * p.tok_stride + s - 1] = tok;
        // the buffer of step s - 2 (read by every CTA before the last barrier)
        // is cleared for step s + 1
        p.best[((s + 1) % 3) * kRows + m] = 0ull;
      }
      uint32_t best_key = 0;
      int best_idx = 0x7fffffff;
      if (ok)
        ok = epilogue_step(p, k, kBlock && s + 1 < steps ? s + 1 : -1, s * n_mine, n_mine, r, live, c0, nh, tmem,
                           bars, abort_flag, bnext, best_key, best_idx);
      if (!ok) *abort_flag = 1;
      publish(p, best_now, r, live, best_key, best_idx);
      // the confidence is off the MMA pipeline's path: after the tiles
      if (ok) confidence_rows(p, k, warp, lane, prev_of);
      if (kBlock) {
        __threadfence();
        epilogue_sync();
        if (threadIdx.x == 0) grid_barrier(p, abort_flag);
        epilogue_sync();
      }
    }
    if (kBlock && blockIdx.x == 0) {
      // after the last barrier: the last step's tokens, and the two buffers in use cleared
      const int last = steps - 1;
      const unsigned long long v = __ldcg(p.best + (last % 3) * kRows + m);
      if (m < p.num_requests) p.tokens[m * p.tok_stride + last] = v ? packed_token(v) : 0;
      p.best[(last % 3) * kRows + m] = 0ull;
      p.best[((last + 2) % 3) * kRows + m] = 0ull;
    }
  } else if (warp == 4) {
    if (lane == 0) {
      constexpr uint32_t kIdesc = instr_desc(0);
      bool ok = true;
      for (int s = 0; s < steps && ok; ++s) {
        if (!(ok = wait_or_abort(bar(kBarAReady), s & 1, abort_flag))) break;
        tc_fence_after();
        for (int t = 0; t < n_mine && ok; ++t) {
          const int g = s * n_mine + t, st = g % kWStages, b = g & 1;
          if (!(ok = wait_or_abort(bar(kBarWFull0 + st), (g / kWStages) & 1, abort_flag))) break;
          if (!(ok = wait_or_abort(bar(kBarDFree0 + b), ((g >> 1) & 1) ^ 1, abort_flag))) break;
          tc_fence_after();
          const uint32_t wbase = sbase + kSmemW + st * 65536;
          // D = A (TMEM, 8 columns per K=16 step) x W tile (shared memory)
          for (int kk = 0; kk < p.rank / 16; ++kk)
            umma_bf16_ts(tmem + b * 128, tmem + kTmemA + kk * 8,
                         smem_desc(wbase + (kk >> 2) * 16384 + (kk & 3) * 32, 16, 1024), kIdesc, kk > 0);
          umma_commit(bar(kBarDFull0 + b));
          umma_commit(bar(kBarWEmpty0 + st));
        }
        umma_commit(bar(kBarAFree));               // the A tile may be refilled for the next step
      }
      if (!ok) *abort_flag = 1;
      umma_commit(bar(kBarDrain));
      volatile int never = 0;
      wait_or_abort(bar(kBarDrain), 0, &never);
    }
    __syncwarp();
  } else {
    if (lane == 0) {
      // the projection-weight tiles of every step, streamed without waiting for the tokens
      int armed[kWStages] = {};
      bool ok = true;
      for (int g = 0; g < steps * n_mine && ok; ++g) {
        const int st = g % kWStages, t = g % n_mine;
        const int v0 = (static_cast<int>(blockIdx.x) + t * static_cast<int>(gridDim.x)) * kVocabTile;
        if (!(ok = wait_or_abort(bar(kBarWEmpty0 + st), ((g / kWStages) & 1) ^ 1, abort_flag))) break;
        mbar_arrive_expect_tx(bar(kBarWFull0 + st), tile_bytes);
        for (int c = 0; c < chunks; ++c)
          tma_load_2d(sbase + kSmemW + st * 65536 + c * 16384, wmap, c * 64, v0, bar(kBarWFull0 + st));
        ++armed[st];
      }
      if (!ok) *abort_flag = 1;
      volatile int never = 0;
      for (int st = 0; st < kWStages; ++st)
        if (armed[st]) wait_or_abort(bar(kBarWFull0 + st), (armed[st] - 1) & 1, &never);
    }
    __syncwarp();
  }

  if (!kBlock) {
    // ---- the last CTA to arrive publishes the tokens and clears the scratch -----
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
        if (r < p.num_requests) p.tokens[r * p.tok_stride + p.k] = packed_token(v);
      }
      if (threadIdx.x == 0) atomicExch(p.arrivals, 0u);
    }
    tc_fence_after();
  } else {
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    // Calls on a stream share the scratch. A call in which some CTA gave up leaves it
    // dirty: an arrival count short of the grid (the CTAs that aborted skip the later
    // barriers) and maxima published after CTA 0 cleared their buffer. Every CTA
    // counts itself out once all its roles are done; the last one out, when any CTA
    // failed, returns the maxima and the arrival counter to zero for the next call.
    volatile int* last = reinterpret_cast<volatile int*>(smem + kSmemLast);
    if (threadIdx.x == 0) {
      if (*abort_flag) atomicOr(p.failed, 1u);
      __threadfence();
      int verdict = 0;
      if (atomicAdd(p.exits, 1u) == gridDim.x - 1) {
        __threadfence();
        verdict = atomicExch(p.failed, 0u) != 0u ? 2 : 1;
        atomicExch(p.exits, 0u);
      }
      *last = verdict;
    }
    __syncthreads();
    if (*last == 2) {
      for (int i = threadIdx.x; i < 3 * kRows; i += blockDim.x) atomicExch(p.best + i, 0ull);
      if (threadIdx.x == 0) atomicExch(p.arrivals, 0u);
    }
  }
  if (warp == 4) tmem_dealloc(tmem, kTmemCols);
}

__global__ void __launch_bounds__(kThreads, 1)
    markov_step_kernel(const __grid_constant__ CUtensorMap wmap, Params p) {
  markov_body<false>(&wmap, p);
}

// Cooperative launch only (all CTAs resident: the grid barrier waits on them).
__global__ void __launch_bounds__(kThreads, 1)
    markov_block_kernel(const __grid_constant__ CUtensorMap wmap, Params p) {
  markov_body<true>(&wmap, p);
}

}  // namespace markov
}  // namespace dspark
