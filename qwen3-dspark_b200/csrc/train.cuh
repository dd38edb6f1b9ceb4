// Training-layout block-draft attention on the 5th-generation tensor cores.
//
// Semantics (dspark_qwen/model.py:12-19,47-61, one sequence at a time, several
// sequences packed back to back with no attention between them): sequence s has
// ctx_s context rows and n_s anchors; its keys are [context rows ; block rows],
// block b owns block rows [ctx_s + bs*b, +bs) and its queries are those same
// bs rows. Query row r of block b sees context rows j < anchor_b and the bs rows
// of its own block (bidirectional). GQA: q head h reads KV head h/2.
//
// Work unit ("tile"): 64 consecutive query rows of one sequence x the two q
// heads of one KV head = 128 rows of S (row m = 2*query + head), so one
// tcgen05.mma M=128 covers both heads sharing the K/V tile. Per tile the keys
// are the context prefix up to the tile's largest anchor, in 128-row blocks,
// then one 128-row block starting at the tile's first block row.
//
// Roles (384 threads, one CTA per SM):
//   warps 0-7  softmax: warps w and w + 4 share S/O rows 32w.. (TMEM lanes of
//              quarter w) and split each row's columns in halves; online
//              softmax with the running max raised only when it grows by more
//              than 2^8 (exact: the final O/l does not depend on the max used),
//              the row maximum of each block and the final row sum exchanged
//              between the two halves through TMEM and a bounded mbarrier
//              wait; P (bf16) written back over its own S buffer in TMEM,
//              where the PV MMA reads it as its A operand. Only a raised max
//              (rare after the first blocks) waits for the previous PV to
//              rescale O in TMEM, so the softmax of block n+1 overlaps the PV
//              MMA of block n;
//   warp 8     TMEM owner and QK issuer (one thread): S = Q K^T into one of
//              two S buffers;
//   warp 11    PV issuer (one thread): O += P V into the O accumulator;
//              completion is reported through tcgen05.commit on mbarriers;
//   warp 9     TMA producer of Q (per tile) and K (3-stage ring), one thread;
//   warp 10    TMA producer of V (3-stage ring), one thread. Separate K and V
//              producers let a K stage refill as soon as its QK is done.
// Every wait is bounded; a timed-out wait raises a CTA abort flag that ends all
// roles, the MMA thread drains its MMAs, the producer waits for its copies in
// flight, and TMEM is released before the CTA exits.
#pragma once
#include "ptx.cuh"

namespace dspark {
namespace train {

constexpr int kSoftmaxWarps = 8;     // two per TMEM lane quarter: column halves of each row
constexpr int kQkWarp = 8, kQkProducerWarp = 9, kVProducerWarp = 10, kPvWarp = 11;
constexpr int kThreads = 12 * 32;
constexpr int kTileQ = 64;          // query rows per tile (x2 heads = 128 MMA rows)
constexpr int kKeyBlock = 128;      // keys per S tile
constexpr int kMaxTileBlocks = 12;  // anchor slots per tile
constexpr int kMinBlock = 6, kMaxBlock = 32;

// Plan (int32 words, built on the host by dspark_train_plan):
//   [0] kPlanMagic [1] items [2] grid [3] total_q [4] total_k [5..7] 0
//   [8 .. 8+grid]   first item of each CTA (grid+1 offsets)
//   [items_at ..]   items of kItemWords words, in CTA order; items_at is a
//                   multiple of 4 words.
constexpr int kPlanMagic = 0x44535431;   // "DST1"
constexpr int kPlanHeader = 8;
constexpr int kItemWords = 24;
enum ItemField {
  kIQRow0 = 0,     // packed row of the tile's first query
  kINq = 1,        // query rows in the tile (1..64)
  kIHead = 2,      // KV head
  kIKBase = 3,     // packed key row of the sequence's first context row
  kICtxKeys = 4,   // context keys any row of the tile sees (= largest anchor)
  kIBlkKey0 = 5,   // packed key row of the tile's first block row
  kIPhase = 6,     // row of the first query inside its block
  kINBlocks = 7,   // blocks the tile's queries belong to (1..12)
  kIBlockSize = 8,
  kIAnchors = 12,  // anchors (clamped to [0, ctx]) of the tile's blocks
};

__host__ __device__ constexpr int plan_items_at(int grid) { return ((kPlanHeader + grid + 1) + 3) & ~3; }

// Shared memory (offsets from a 1024-byte aligned base). Every operand tile is
// two 16 KB halves of 128 rows x 64 bf16 in the 128-byte swizzle.
// Key block g uses K and V stage g%3 and TMEM S/P buffer g&1.
constexpr int kStages = 3;
constexpr uint32_t kSmemQ = 0;
constexpr uint32_t kSmemK = 32768;                       // 3 stages x 32 KB
constexpr uint32_t kSmemV = kSmemK + kStages * 32768;    // 3 stages x 32 KB
constexpr uint32_t kSmemBar = kSmemV + kStages * 32768;
// Per-block barriers of the S/P buffers come in pairs indexed by the block's
// parity and the stage barriers one per stage, so no waiter can ever be two
// phases behind its barrier.
enum Barrier {
  kBarQFull = 0, kBarQEmpty, kBarKFull0, kBarKEmpty0 = kBarKFull0 + kStages, kBarVFull0 = kBarKEmpty0 + kStages,
  kBarVEmpty0 = kBarVFull0 + kStages, kBarSFull0 = kBarVEmpty0 + kStages, kBarPFull0 = kBarSFull0 + 2,
  kBarODone0 = kBarPFull0 + 2, kBarOFree = kBarODone0 + 2, kBarDrain, kBarX0, kNumBarriers = kBarX0 + 4
};
constexpr uint32_t kSmemTmemSlot = kSmemBar + kNumBarriers * 8;
constexpr uint32_t kSmemAbort = kSmemTmemSlot + 4;
constexpr uint32_t kSmemBytes = 1024 + kSmemAbort + 4;

// TMEM columns: two S buffers and the O accumulator, 128 fp32 columns each. P
// (bf16, two per column) overwrites the first 64 columns of its own S buffer
// and is the A operand of the PV MMA straight from TMEM. Columns from kTmemX
// carry the row maxima and sums the two softmax warps of a lane quarter
// exchange (each warp owns half of every row's columns).
constexpr uint32_t kTmemCols = 512;
constexpr uint32_t kTmemS = 0, kTmemO = 256, kTmemX = 384;

// ---------------------------------------------------------------- tcgen05 PTX
__device__ __forceinline__ void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

__device__ __forceinline__ void tmem_alloc(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 in, fp32 accumulate, one thread.
__device__ __forceinline__ void umma_bf16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T: A is 128 rows (TMEM lanes) of K=16 bf16
// packed two per 32-bit column (the lower key in the low half), 8 columns.
__device__ __forceinline__ void umma_bf16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the mbarrier when every MMA this thread issued so far is done.
__device__ __forceinline__ void umma_commit(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

// Shared-memory matrix descriptor: 128-byte swizzle, sm_100 descriptor version.
// lbo/sbo in bytes (leading / stride dimension byte offsets).
__device__ __forceinline__ uint64_t smem_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(lbo >> 4) << 16) |
         (static_cast<uint64_t>(sbo >> 4) << 32) | (1ull << 46) | (2ull << 61);
}

// Instruction descriptor of kind::f16: fp32 D, bf16 A and B, A K-major,
// B K-major (b_mn = 0) or N-major (b_mn = 1), M = 128, N = 128.
__host__ __device__ constexpr uint32_t instr_desc(uint32_t b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn << 16) | ((128u >> 3) << 17) | ((128u >> 4) << 24);
}

// 32 lanes x 32 fp32 columns from TMEM, waited for inside the same statement so
// no use of the registers can be scheduled before the data has arrived.
// 32 columns of this warp's TMEM lanes into registers, without waiting for them.
__device__ __forceinline__ void tmem_ld32_async(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      :
        "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
}

// Waits for this thread's TMEM loads. The registers of each load pass through a
// statement ordered after the wait, so that no use of them is scheduled earlier.
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_ld_landed(uint32_t (&r)[32]) {
  asm volatile(""
               :
                 "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]),
                 "+r"(r[15]), "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]),
                 "+r"(r[22]), "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]),
                 "+r"(r[29]), "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// A full 128-column row block (4 x 32 columns) with a single wait.
__device__ __forceinline__ void tmem_ld128(uint32_t taddr, float (&v)[128]) {
  uint32_t r[128];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%128];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%32,%33,%34,%35,%36,%37,%38,%39,%40,%41,%42,%43,%44,%45,%46,%47,%48,%49,%50,%51,%52,%53,%54,%55,%56,%57,%58,%59,%60,%61,%62,%63}, [%129];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%64,%65,%66,%67,%68,%69,%70,%71,%72,%73,%74,%75,%76,%77,%78,%79,%80,%81,%82,%83,%84,%85,%86,%87,%88,%89,%90,%91,%92,%93,%94,%95}, [%130];\n\t"
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%96,%97,%98,%99,%100,%101,%102,%103,%104,%105,%106,%107,%108,%109,%110,%111,%112,%113,%114,%115,%116,%117,%118,%119,%120,%121,%122,%123,%124,%125,%126,%127}, [%131];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31]),
        "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]), "=r"(r[37]), "=r"(r[38]), "=r"(r[39]),
        "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]), "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]),
        "=r"(r[48]), "=r"(r[49]), "=r"(r[50]), "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]),
        "=r"(r[56]), "=r"(r[57]), "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63]),
        "=r"(r[64]), "=r"(r[65]), "=r"(r[66]), "=r"(r[67]), "=r"(r[68]), "=r"(r[69]), "=r"(r[70]), "=r"(r[71]),
        "=r"(r[72]), "=r"(r[73]), "=r"(r[74]), "=r"(r[75]), "=r"(r[76]), "=r"(r[77]), "=r"(r[78]), "=r"(r[79]),
        "=r"(r[80]), "=r"(r[81]), "=r"(r[82]), "=r"(r[83]), "=r"(r[84]), "=r"(r[85]), "=r"(r[86]), "=r"(r[87]),
        "=r"(r[88]), "=r"(r[89]), "=r"(r[90]), "=r"(r[91]), "=r"(r[92]), "=r"(r[93]), "=r"(r[94]), "=r"(r[95]),
        "=r"(r[96]), "=r"(r[97]), "=r"(r[98]), "=r"(r[99]), "=r"(r[100]), "=r"(r[101]), "=r"(r[102]), "=r"(r[103]),
        "=r"(r[104]), "=r"(r[105]), "=r"(r[106]), "=r"(r[107]), "=r"(r[108]), "=r"(r[109]), "=r"(r[110]), "=r"(r[111]),
        "=r"(r[112]), "=r"(r[113]), "=r"(r[114]), "=r"(r[115]), "=r"(r[116]), "=r"(r[117]), "=r"(r[118]), "=r"(r[119]),
        "=r"(r[120]), "=r"(r[121]), "=r"(r[122]), "=r"(r[123]), "=r"(r[124]), "=r"(r[125]), "=r"(r[126]), "=r"(r[127])
      : "r"(taddr), "r"(taddr + 32), "r"(taddr + 64), "r"(taddr + 96)
      : "memory");
#pragma unroll
  for (int i = 0; i < 128; ++i) v[i] = __uint_as_float(r[i]);
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float (&v)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
      "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
      "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
      "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
      "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
      "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
      "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
      "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
      "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
      "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
      "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

// One fp32 column per lane (32 lanes x 1 column), completed in the statement.
__device__ __forceinline__ void tmem_st1(uint32_t taddr, float v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x1.b32 [%0], {%1};\n\t"
      "tcgen05.wait::st.sync.aligned;" ::"r"(taddr),
      "r"(__float_as_uint(v))
      : "memory");
}

__device__ __forceinline__ float tmem_ld1(uint32_t taddr) {
  uint32_t r;
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x1.b32 {%0}, [%1];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r)
      : "r"(taddr)
      : "memory");
  return __uint_as_float(r);
}

// Bounded wait that also gives up as soon as another role has raised the CTA
// abort flag. A timeout raises the flag and the device status bit.
__device__ __forceinline__ bool wait_or_abort(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = globaltimer();
  for (uint32_t it = 1;; ++it) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((it & 63u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer() - t0 > kWaitLimitNs) {
        atomicOr(&g_device_status, kStatusWaitTimeout);
        *abort_flag = 1;
        return false;
      }
    }
  }
}

// Maximum of 64 values as a tree of three-input maxima (depth 4 instead of a
// 64-long dependent chain).
__device__ __forceinline__ float max3f(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}

__device__ __forceinline__ float max64(const float (&s)[64]) {
  float a[22], b[8];
#pragma unroll
  for (int j = 0; j < 21; ++j) a[j] = max3f(s[3 * j], s[3 * j + 1], s[3 * j + 2]);
  a[21] = s[63];
#pragma unroll
  for (int j = 0; j < 7; ++j) b[j] = max3f(a[3 * j], a[3 * j + 1], a[3 * j + 2]);
  b[7] = a[21];
  return max3f(max3f(b[0], b[1], b[2]), max3f(b[3], b[4], b[5]), fmaxf(b[6], b[7]));
}

// ---------------------------------------------------------------- item
struct Item {
  int q_row0, nq, head, k_base, ctx_keys, blk_key0, phase, nblocks, bs;
  __device__ int key_blocks() const { return (ctx_keys + kKeyBlock - 1) / kKeyBlock + 1; }
};

__device__ __forceinline__ bool load_item(const int* it, int total_q, int total_k, Item& x) {
  x.q_row0 = it[kIQRow0];
  x.nq = it[kINq];
  x.head = it[kIHead];
  x.k_base = it[kIKBase];
  x.ctx_keys = it[kICtxKeys];
  x.blk_key0 = it[kIBlkKey0];
  x.phase = it[kIPhase];
  x.nblocks = it[kINBlocks];
  x.bs = it[kIBlockSize];
  return x.nq >= 1 && x.nq <= kTileQ && x.head >= 0 && x.head < 8 && x.q_row0 >= 0 && x.q_row0 + x.nq <= total_q &&
         x.k_base >= 0 && x.ctx_keys >= 0 && x.k_base + x.ctx_keys <= total_k && x.blk_key0 >= 0 &&
         x.blk_key0 < total_k && x.bs >= kMinBlock && x.bs <= kMaxBlock && x.phase >= 0 && x.phase < x.bs &&
         x.nblocks >= 1 && x.nblocks <= kMaxTileBlocks && (x.phase + x.nq - 1) / x.bs < x.nblocks &&
         x.nblocks * x.bs <= kKeyBlock;
}

// ---------------------------------------------------------------- roles
// kKeys: Q per tile + K per key block; otherwise V per key block.
template <bool kKeys>
__device__ __forceinline__ void producer_role(const CUtensorMap* qmap, const CUtensorMap* kvmap, const int* items,
                                              int first, int last, int total_q, int total_k, uint32_t sbase,
                                              uint32_t bars, volatile int* abort_flag) {
  auto bar = [&](int i) { return bars + 8u * i; };
  constexpr int kFull = kKeys ? kBarKFull0 : kBarVFull0;
  constexpr int kEmpty = kKeys ? kBarKEmpty0 : kBarVEmpty0;
  constexpr uint32_t kRing = kKeys ? kSmemK : kSmemV;
  int gb = 0, it = 0, armed_q = 0;
  int armed[kStages] = {};
  bool ok = true;
  for (int idx = first; idx < last && ok; ++idx) {
    Item x;
    if (!load_item(items + static_cast<size_t>(idx) * kItemWords, total_q, total_k, x)) continue;
    const int nb = x.key_blocks(), nctx = nb - 1;
    if (kKeys) {
      if (!(ok = wait_or_abort(bar(kBarQEmpty), (it & 1) ^ 1, abort_flag))) break;
      mbar_arrive_expect_tx(bar(kBarQFull), 32768);
      tma_load_3d(sbase + kSmemQ, qmap, 0, 2 * x.head, x.q_row0, bar(kBarQFull));
      tma_load_3d(sbase + kSmemQ + 16384, qmap, 64, 2 * x.head, x.q_row0, bar(kBarQFull));
      ++armed_q;
    }
    for (int n = 0; n < nb; ++n) {
      const int g = gb + n, st = g % kStages;
      const int row = n < nctx ? x.k_base + n * kKeyBlock : x.blk_key0;
      if (!(ok = wait_or_abort(bar(kEmpty + st), ((g / kStages) & 1) ^ 1, abort_flag))) break;
      mbar_arrive_expect_tx(bar(kFull + st), 32768);
      tma_load_3d(sbase + kRing + st * 32768, kvmap, 0, x.head, row, bar(kFull + st));
      tma_load_3d(sbase + kRing + st * 32768 + 16384, kvmap, 64, x.head, row, bar(kFull + st));
      ++armed[st];
    }
    gb += nb;
    ++it;
  }
  if (!ok) *abort_flag = 1;
  // Copies in flight land before the CTA can exit (a no-op when all were consumed).
  volatile int never = 0;
  if (armed_q) wait_or_abort(bar(kBarQFull), (armed_q - 1) & 1, &never);
  for (int st = 0; st < kStages; ++st)
    if (armed[st]) wait_or_abort(bar(kFull + st), (armed[st] - 1) & 1, &never);
}

// Two MMA issuers, one thread each: an MMA instruction is accepted only about
// one ahead of the tensor pipe, so every mbarrier wait or commit on the issuing
// thread leaves the pipe idle; with S = Q K^T and O += P V issued from
// different warps, one issuer's waits overlap the other's MMAs. Their operands
// are disjoint (S buffers vs O in TMEM; Q, K vs P, V in shared memory).
//
// QK issuer: S(g) = Q K(g)^T into S buffer g&1, 8 MMAs of K=16 over the head
// dim.
__device__ __forceinline__ void qk_role(const int* items, int first, int last, int total_q, int total_k,
                                        uint32_t sbase, uint32_t bars, uint32_t tmem, volatile int* abort_flag) {
  auto bar = [&](int i) { return bars + 8u * i; };
  constexpr uint32_t kIdesc = instr_desc(0);
  int gb = 0, it = 0;
  bool ok = true;
  for (int idx = first; idx < last && ok; ++idx) {
    Item x;
    if (!load_item(items + static_cast<size_t>(idx) * kItemWords, total_q, total_k, x)) continue;
    const int nb = x.key_blocks();
    if (!(ok = wait_or_abort(bar(kBarQFull), it & 1, abort_flag))) break;
    for (int n = 0; n < nb; ++n) {
      const int g = gb + n, sb = g & 1, st = g % kStages;
      if (!(ok = wait_or_abort(bar(kBarKFull0 + st), (g / kStages) & 1, abort_flag))) break;
      // S buffer g&1 holds P(g-2) until PV(g-2) has read it.
      if (g >= 2 && !(ok = wait_or_abort(bar(kBarODone0 + sb), ((g - 2) >> 1) & 1, abort_flag))) break;
      tc_fence_after();
      const uint32_t kbase = sbase + kSmemK + st * 32768;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk) {
        const uint32_t off = (kk >> 2) * 16384 + (kk & 3) * 32;
        umma_bf16(tmem + kTmemS + sb * 128, smem_desc(sbase + kSmemQ + off, 16, 1024),
                  smem_desc(kbase + off, 16, 1024), kIdesc, kk > 0);
      }
      umma_commit(bar(kBarSFull0 + sb));
      umma_commit(bar(kBarKEmpty0 + st));
      if (n == nb - 1) umma_commit(bar(kBarQEmpty));
    }
    gb += nb;
    ++it;
  }
  if (!ok) *abort_flag = 1;
  // Every MMA issued above completes before TMEM is released.
  umma_commit(bar(kBarDrain));
  volatile int never = 0;
  wait_or_abort(bar(kBarDrain), 0, &never);
}

// PV issuer: O += P(g) V(g), A = P from TMEM (K-major over keys), B = V
// (N-major: d contiguous).
__device__ __forceinline__ void pv_role(const int* items, int first, int last, int total_q, int total_k,
                                        uint32_t sbase, uint32_t bars, uint32_t tmem, volatile int* abort_flag) {
  auto bar = [&](int i) { return bars + 8u * i; };
  constexpr uint32_t kIdesc = instr_desc(1);
  int gb = 0, it = 0;
  bool ok = true;
  for (int idx = first; idx < last && ok; ++idx) {
    Item x;
    if (!load_item(items + static_cast<size_t>(idx) * kItemWords, total_q, total_k, x)) continue;
    const int nb = x.key_blocks();
    for (int n = 0; n < nb; ++n) {
      const int g = gb + n, sb = g & 1, st = g % kStages;
      if (!(ok = wait_or_abort(bar(kBarPFull0 + sb), (g >> 1) & 1, abort_flag))) break;
      if (n == 0 && !(ok = wait_or_abort(bar(kBarOFree), (it & 1) ^ 1, abort_flag))) break;
      if (!(ok = wait_or_abort(bar(kBarVFull0 + st), (g / kStages) & 1, abort_flag))) break;
      tc_fence_after();
      const uint32_t vbase = sbase + kSmemV + st * 32768;
#pragma unroll
      for (int kk = 0; kk < 8; ++kk)
        umma_bf16_ts(tmem + kTmemO, tmem + kTmemS + sb * 128 + kk * 8, smem_desc(vbase + kk * 2048, 16384, 1024),
                     kIdesc, (n > 0 || kk > 0) ? 1u : 0u);
      umma_commit(bar(kBarODone0 + sb));
      umma_commit(bar(kBarVEmpty0 + st));
    }
    gb += nb;
    ++it;
  }
  if (!ok) *abort_flag = 1;
  umma_commit(bar(kBarDrain));
  volatile int never = 0;
  wait_or_abort(bar(kBarDrain), 0, &never);
}

__device__ __forceinline__ void softmax_role(const int* items, int first, int last, int total_q, int total_k,
                                             uint8_t* smem, uint32_t bars, uint32_t tmem, __nv_bfloat16* out,
                                             float scale_log2, volatile int* abort_flag) {
  auto bar = [&](int i) { return bars + 8u * i; };
  // warp w handles TMEM lanes 32 (w % 4) .. (rows) and column half w / 4 of every
  // row: keys [64 h, 64 h + 64) of S, their packed P columns [32 h, 32 h + 32) and
  // O columns (d) [64 h, 64 h + 64); the row maximum of each block and the final
  // row sum are exchanged with warp w ^ 4 through TMEM columns kTmemX.. and the
  // quarter's mbarrier (both warps arrive, each waits with a bound).
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int half = warp >> 2, quarter = warp & 3;
  const int m = quarter * 32 + lane;               // S/O row == TMEM lane
  const int qi = m >> 1;                           // query row inside the tile
  const uint32_t lane_addr = static_cast<uint32_t>(quarter * 32) << 16;
  const uint32_t xbar = bar(kBarX0 + quarter);
  uint32_t xcount = 0;                             // exchanges done (barrier phase)
  int gb = 0;
  bool ok = true;
  auto exchange = [&](uint32_t col0, float mine, float& theirs) {
    tmem_st1(tmem + lane_addr + col0 + half, mine);
    tc_fence_before();
    mbar_arrive(xbar);
    const bool w = wait_or_abort(xbar, xcount & 1, abort_flag);
    ++xcount;
    if (!__all_sync(0xffffffffu, w)) return false;
    tc_fence_after();
    theirs = tmem_ld1(tmem + lane_addr + col0 + (half ^ 1));
    return true;
  };
  for (int idx = first; idx < last && ok; ++idx) {
    const int* ip = items + static_cast<size_t>(idx) * kItemWords;
    Item x;
    if (!load_item(ip, total_q, total_k, x)) {
      if (threadIdx.x == 0) atomicOr(&g_device_status, kStatusBadArgument);
      continue;
    }
    const int nb = x.key_blocks(), nctx = nb - 1;
    const bool row_ok = qi < x.nq;
    const int rel = (x.phase + qi) / x.bs;         // block of this row inside the tile
    int anchor = row_ok ? ip[kIAnchors + min(rel, kMaxTileBlocks - 1)] : 0;
    anchor = max(0, min(anchor, x.ctx_keys));
    float m_run = -1e30f, l = 0.f;
    for (int n = 0; n < nb; ++n) {
      const int g = gb + n;
      ok = wait_or_abort(bar(kBarSFull0 + (g & 1)), (g >> 1) & 1, abort_flag);
      if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
      tc_fence_after();
      float s[64];
      tmem_ld32(tmem + lane_addr + kTmemS + (g & 1) * 128 + half * 64, *reinterpret_cast<float(*)[32]>(&s[0]));
      tmem_ld32(tmem + lane_addr + kTmemS + (g & 1) * 128 + half * 64 + 32, *reinterpret_cast<float(*)[32]>(&s[32]));
      int lo, hi;
      if (n < nctx) {
        lo = 0;
        hi = min(max(anchor - n * kKeyBlock, 0), kKeyBlock);
      } else {
        lo = rel * x.bs;
        hi = min(lo + x.bs, kKeyBlock);
      }
      if (!row_ok) hi = lo;
      lo = max(lo - half * 64, 0);                 // into this half's key index
      hi = min(hi - half * 64, 64);
      // Rows of a warp mostly share their visibility; a warp whose rows all see
      // the whole half skips the select. Otherwise the visible keys [lo, hi)
      // are a bit mask and every value is selected against its bit.
      if (!__all_sync(0xffffffffu, lo == 0 && hi == 64)) {
        const uint64_t bits = hi > lo ? ((hi >= 64 ? ~0ull : (1ull << hi) - 1) & ~((1ull << lo) - 1)) : 0ull;
        const uint32_t b0 = static_cast<uint32_t>(bits), b1 = static_cast<uint32_t>(bits >> 32);
#pragma unroll
        for (int i = 0; i < 64; ++i) s[i] = (((i < 32 ? b0 : b1) >> (i & 31)) & 1u) ? s[i] : -INFINITY;
      }
      float mb = max64(s);
      float mo;
      if (!(ok = exchange(kTmemX + (xcount & 1) * 2, mb, mo))) break;
      mb = fmaxf(mb, mo);
      const float m_new = fmaxf(m_run, mb * scale_log2);
      const bool resc = m_new > m_run + 8.f;
      float alpha = 1.f;
      if (resc) {
        alpha = ex2(m_run - m_new);
        m_run = m_new;
      }
      float sum = 0.f;
      uint32_t pk[32];
#pragma unroll
      for (int i = 0; i < 32; ++i) {
        const float p0 = ex2(fmaf(s[2 * i], scale_log2, -m_run));
        const float p1 = ex2(fmaf(s[2 * i + 1], scale_log2, -m_run));
        sum += p0 + p1;
        pk[i] = pack_bf16x2(p0, p1);
      }
      l = l * alpha + sum;
      if (n > 0 && __any_sync(0xffffffffu, resc)) {
        // A raised max rescales O once PV(g-1) has added into it.
        ok = wait_or_abort(bar(kBarODone0 + ((g - 1) & 1)), ((g - 1) >> 1) & 1, abort_flag);
        if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int c = 0; c < 2; ++c) {
          float o[32];
          tmem_ld32(tmem + lane_addr + kTmemO + half * 64 + c * 32, o);
#pragma unroll
          for (int i = 0; i < 32; ++i) o[i] *= alpha;
          tmem_st32(tmem + lane_addr + kTmemO + half * 64 + c * 32, o);
        }
      }
      // P of this half's 64 keys: packed columns [32 half, +32) of its own S buffer
      // (the other warp has read its S columns: it arrived at the exchange after)
      tmem_st32(tmem + lane_addr + kTmemS + (g & 1) * 128 + half * 32, *reinterpret_cast<const float(*)[32]>(pk));
      tc_fence_before();
      mbar_arrive(bar(kBarPFull0 + (g & 1)));
    }
    if (!ok) break;
    gb += nb;
    float lo_other;
    if (!(ok = exchange(kTmemX + 4, l, lo_other))) break;
    l += lo_other;
    ok = wait_or_abort(bar(kBarODone0 + ((gb - 1) & 1)), ((gb - 1) >> 1) & 1, abort_flag);
    if (!__all_sync(0xffffffffu, ok)) { ok = false; break; }
    tc_fence_after();
    const float inv_l = row_ok ? 1.f / l : 0.f;
    __nv_bfloat16* orow = out + (static_cast<size_t>(x.q_row0 + (row_ok ? qi : 0)) * 16 + 2 * x.head + (m & 1)) * 128 +
                          half * 64;
#pragma unroll
    for (int c = 0; c < 2; ++c) {
      float o[32];
      tmem_ld32(tmem + lane_addr + kTmemO + half * 64 + c * 32, o);
      if (row_ok) {
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          uint4 v;
          v.x = pack_bf16x2(o[8 * j] * inv_l, o[8 * j + 1] * inv_l);
          v.y = pack_bf16x2(o[8 * j + 2] * inv_l, o[8 * j + 3] * inv_l);
          v.z = pack_bf16x2(o[8 * j + 4] * inv_l, o[8 * j + 5] * inv_l);
          v.w = pack_bf16x2(o[8 * j + 6] * inv_l, o[8 * j + 7] * inv_l);
          *reinterpret_cast<uint4*>(orow + c * 32 + 8 * j) = v;
        }
      }
    }
    tc_fence_before();
    mbar_arrive(bar(kBarOFree));
  }
  if (!ok) *abort_flag = 1;
}

// ---------------------------------------------------------------- kernel
__global__ void __launch_bounds__(kThreads, 1)
    train_attn_kernel(const __grid_constant__ CUtensorMap qmap, const __grid_constant__ CUtensorMap kmap,
                      const __grid_constant__ CUtensorMap vmap, const int* __restrict__ plan,
                      __nv_bfloat16* __restrict__ out, int total_q, int total_k, float scale_log2) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  const uint32_t sbase = smem_u32(smem);
  const uint32_t bars = sbase + kSmemBar;
  volatile int* abort_flag = reinterpret_cast<volatile int*>(smem + kSmemAbort);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  // The plan must describe exactly the tensors this launch was given.
  const int grid = plan[2];
  const bool plan_ok = plan[0] == kPlanMagic && grid == static_cast<int>(gridDim.x) && plan[3] == total_q &&
                       plan[4] == total_k;
  int first = 0, last = 0;
  if (plan_ok) {
    first = plan[kPlanHeader + blockIdx.x];
    last = plan[kPlanHeader + blockIdx.x + 1];
    if (first < 0 || last < first || last > plan[1]) first = last = 0;
  } else if (threadIdx.x == 0) {
    atomicOr(&g_device_status, kStatusBadArgument);
  }
  const int* items = plan + plan_items_at(grid > 0 ? grid : 0);

  if (threadIdx.x == 0) {
    for (int i = 0; i < kNumBarriers; ++i)
      mbar_init(bars + 8u * i, (i == kBarPFull0 || i == kBarPFull0 + 1 || i == kBarOFree)
                                   ? 32u * kSoftmaxWarps
                                   : (i >= kBarX0 ? 64u : (i == kBarDrain ? 2u : 1u)));
    *abort_flag = 0;
    fence_barrier_init();
  }
  if (warp == kQkProducerWarp && lane == 0) {
    prefetch_tmap(&qmap);
    prefetch_tmap(&kmap);
  }
  if (warp == kVProducerWarp && lane == 0) prefetch_tmap(&vmap);
  if (warp == kQkWarp) tmem_alloc(sbase + kSmemTmemSlot, kTmemCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *reinterpret_cast<volatile uint32_t*>(smem + kSmemTmemSlot);

  if (warp < kSoftmaxWarps) {
    softmax_role(items, first, last, total_q, total_k, smem, bars, tmem, out, scale_log2, abort_flag);
  } else if (warp == kQkWarp) {
    if (lane == 0) qk_role(items, first, last, total_q, total_k, sbase, bars, tmem, abort_flag);
    __syncwarp();
  } else if (warp == kPvWarp) {
    if (lane == 0) pv_role(items, first, last, total_q, total_k, sbase, bars, tmem, abort_flag);
    __syncwarp();
  } else if (warp == kQkProducerWarp) {
    if (lane == 0)
      producer_role<true>(&qmap, &kmap, items, first, last, total_q, total_k, sbase, bars, abort_flag);
    __syncwarp();
  } else {
    if (lane == 0)
      producer_role<false>(&qmap, &vmap, items, first, last, total_q, total_k, sbase, bars, abort_flag);
    __syncwarp();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  if (warp == kQkWarp) tmem_dealloc(tmem, kTmemCols);
}

}  // namespace train
}  // namespace dspark
