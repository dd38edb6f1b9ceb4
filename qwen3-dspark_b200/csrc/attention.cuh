// Packed varlen GQA attention for DSpark draft (non-causal) and verify
// (bottom-right causal) on sm_100a.
//
// Geometry (Qwen3-0.6B attention): 16 query heads, 8 KV heads, head dim 128.
// A work item is one request's block of up to 8 query rows. For KV head h the
// item's 2 query heads (2h, 2h+1) x 8 rows form one 16-row MMA tile, so a
// single m16n8k16 row block covers the whole GQA group; query row r of head
// 2h+g sits in MMA row 8g + r, which gives both rows a thread holds the same
// causal limit.
//
// Keys of an item are the concatenation of two row ranges ("source A" then
// "source B") of [rows, 8, 128] bf16 tensors: the packed THD K/V of the
// reference kernel contract (B empty), or a resident prefix followed by the
// verify scratch rows, or a context cache followed by the draft block rows.
//
// Persistent schedule: the key tiles of all items (16 keys x 8 heads each,
// 64 KB of K+V) are numbered in request order and split into equal contiguous
// ranges, one per CTA (one CTA per SM). A CTA streams its range through a
// 3-stage TMA pipeline: warp 8 issues the loads, warps 0-7 (one per KV head)
// consume them. Items that lie wholly inside one range are normalised and
// written directly. An item cut by range boundaries leaves fp32 partials, and
// the CTA holding its first tile records it; split_merge_kernel, launched
// right after (programmatic dependent launch), combines the partials of every
// cut item with a log-sum-exp merge and writes the output. No CTA ever waits
// for another one, and the merges run in parallel on many SMs instead of
// trailing the contributor that arrives last.
//
// Fused verify mode (kFused): q holds the layer's raw q projections and source
// B is the raw k/v projections of the new tokens. Consumer warps apply Qwen3
// RMSNorm + RoPE to their Q fragments in registers and to the new k rows in
// shared memory after TMA delivers them, and append roped k / raw v to the
// layer's scratch rows (the KV append). cos/sin come from a per-transaction
// table (computed once for all layers, as the model's rotary module does); the
// producer bulk-copies a new-row tile's table rows next to its K/V box.
#pragma once
#include <cfloat>
#include <climits>
#include "ptx.cuh"

namespace dspark {

constexpr int kHeadDim = 128;
constexpr int kQHeads = 16;
constexpr int kKVHeads = 8;
constexpr int kQBlock = 8;                              // query rows per item
constexpr int kTileN = 16;                              // keys per pipeline tile
constexpr int kStages = 3;
constexpr int kConsumerWarps = kKVHeads;                // warp w computes KV head w
constexpr int kAttnThreads = (kConsumerWarps + 1) * 32;  // + one producer warp
constexpr int kHalfBoxBytes = kKVHeads * kTileN * 128;  // 64 bf16 x 16 rows x 8 heads
constexpr int kStageBytes = 4 * kHalfBoxBytes;          // K lo/hi + V lo/hi halves
constexpr int kRopeRowBytes = 64 * 4;                   // 64 (cos, sin) bf16 pairs per position
constexpr int kRopeStageBytes = kTileN * kRopeRowBytes;  // table rows of one source-B tile
// Dynamic shared memory: stages | rope rows per stage | q_norm, k_norm weights |
// full/empty barriers | schedule scratch (the base is rounded up to 1024 B).
constexpr int kSmemRopeOff = kStages * kStageBytes;
constexpr int kSmemWeightOff = kSmemRopeOff + kStages * kRopeStageBytes;
constexpr int kSmemBarOff = kSmemWeightOff + 2 * kHeadDim * 2;
constexpr int kPartFloatsPerSlot = kKVHeads * 16 * kHeadDim;
constexpr int kPartMlPerSlot = kKVHeads * 16 * 2;

enum KeyMode : int { kModeVarlen = 0, kModeSegmented = 1 };

struct AttnParams {
  const void* q;             // [total_q, 16, 128] (raw q projections in fused mode)
  void* out;                 // [total_q, 16, 128]
  const int* cu_q;           // [R+1]
  int num_requests;
  int total_q;
  int mode;                  // KeyMode
  int causal;                // bottom-right causal mask
  // kModeVarlen: keys of request i are rows [cu_k[i], cu_k[i+1]) of source A.
  const int* cu_k;
  // kModeSegmented: rows [a_off + a_start[i], + a_len[i]) of A, then rows
  // [b_off + (b_start ? b_start[i] : cu_q[i]), + (b_len ? b_len[i] : q_i)) of B.
  // A null b_start/b_len selects the verify-scratch convention; b_none drops B.
  const int* a_start;
  const int* a_len;
  const int* b_start;
  const int* b_len;
  int a_off;
  int b_off;
  int b_none;
  long long rows_a;          // extents, used by the fp32 path's bounds checks
  long long rows_b;
  float scale;
  float scale_log2;          // scale * log2(e)
  // fused verify: new token row r of request i is global row cu_q[i] + r of
  // k_new/v_new and of this layer's scratch; its position is a_len[i] + r.
  const __nv_bfloat16* k_new;   // [total_q, 8, 128] raw k projections
  const __nv_bfloat16* v_new;   // [total_q, 8, 128] raw v projections
  const __nv_bfloat16* q_w;     // [128] q_norm weight
  const __nv_bfloat16* k_w;     // [128] k_norm weight
  const uint32_t* rope;         // [total_q][64] bf16x2 (cos low, sin high) at each new row's position
  float eps;
  __nv_bfloat16* scratch_k;     // this layer's scratch rows (source B)
  __nv_bfloat16* scratch_v;
  int scratch_rows;
  // workspace (split items)
  float* part_o;             // [grid][2][8][16][128]
  float* part_ml;            // [grid][2][8][16][2]
  struct MergeEntry* merges; // [grid][8]: the cut item CTA c starts, per KV head
  long long* ranges;         // [grid][2]: tile range [start, end) of CTA c in this launch
  int grid;
};

// A cut item (one whose tiles span several CTAs) and KV head, recorded by the
// CTA holding its first tile for the merge kernel. Every launch rewrites the
// entries of all its CTAs, so stale entries are never read.
struct MergeEntry {
  long long item_start;      // global index of the item's first tile
  long long item_end;        // one past its last tile
  int first;                 // CTA holding the first tile (contributors: first, first + 1, ...)
  int slot_first;            // partial slot of the first contributor
  int q0, nrows;             // output rows of the item
  int valid;
  int pad[3];
};

// ---------------------------------------------------------------------------
// Item geometry and the tile walk shared by the scan, the producer and the
// consumers.
// ---------------------------------------------------------------------------
struct Item {
  int req, qb;
  int q0;        // first query row (global) of this block
  int nrows;     // valid query rows in this block (1..8)
  int q_len;     // request query rows
  int q_start;   // cu_q[req]
  int a_row, a_len, b_row, b_len;
  int k_len;     // a_len + b_len
  int vis;       // keys visible to the block's last row
  int tiles_a, tiles_b, tiles;
};

__device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }

__device__ __forceinline__ int request_q_len(const AttnParams& p, int req) {
  return p.cu_q[req + 1] - p.cu_q[req];
}

__device__ __forceinline__ void load_item(const AttnParams& p, int req, int qb, Item& it) {
  it.req = req;
  it.qb = qb;
  const int qs = p.cu_q[req];
  it.q_start = qs;
  it.q_len = p.cu_q[req + 1] - qs;
  it.q0 = qs + qb * kQBlock;
  it.nrows = min(kQBlock, it.q_len - qb * kQBlock);
  if (p.mode == kModeVarlen) {
    it.a_row = p.cu_k[req];
    it.a_len = p.cu_k[req + 1] - it.a_row;
    it.b_row = 0;
    it.b_len = 0;
  } else {
    it.a_row = p.a_off + p.a_start[req];
    it.a_len = p.a_len[req];
    if (p.b_none) {
      it.b_row = 0;
      it.b_len = 0;
    } else {
      it.b_row = p.b_off + (p.b_start ? p.b_start[req] : qs);
      it.b_len = p.b_len ? p.b_len[req] : it.q_len;
    }
  }
  if (it.a_len < 0 || it.b_len < 0 || it.nrows < 1) {
    atomicOr(&g_device_status, kStatusBadArgument);
    it.a_len = max(it.a_len, 0);
    it.b_len = max(it.b_len, 0);
    it.nrows = max(it.nrows, 1);
  }
  it.k_len = it.a_len + it.b_len;
  if (p.causal) {
    const int last_row = min(it.q_len, (qb + 1) * kQBlock);     // exclusive
    it.vis = min(it.k_len, it.k_len - it.q_len + last_row);
  } else {
    it.vis = it.k_len;
  }
  it.vis = max(it.vis, 0);
  const int va = min(it.vis, it.a_len);
  it.tiles_a = cdiv(va, kTileN);
  it.tiles_b = cdiv(it.vis - va, kTileN);
  // Every item owns at least one tile so the walk always advances; an item
  // with no visible key (rejected on the host) then reads nothing useful.
  it.tiles = max(it.tiles_a + it.tiles_b, 1);
}

__device__ __forceinline__ int request_qblocks(const AttnParams& p, int req) {
  return max(cdiv(request_q_len(p, req), kQBlock), 1);
}

__device__ long long request_tiles(const AttnParams& p, int req) {
  const int nqb = request_qblocks(p, req);
  long long t = 0;
  Item it;
  for (int qb = 0; qb < nqb; ++qb) {
    load_item(p, req, qb, it);
    t += it.tiles;
  }
  return t;
}

struct Tile {
  int src_b;      // 0: source A, 1: source B
  int row;        // first row of the tile in its source tensor
  int n_valid;    // keys of this tile inside the item's visible range
  int key_base;   // index of the tile's first key in the item's key order
  int b_first;    // source B: index of the tile's first row among the request's B rows
};

__device__ __forceinline__ Tile tile_of(const Item& it, int t) {
  Tile ti;
  if (t < it.tiles_a) {
    ti.src_b = 0;
    ti.row = it.a_row + t * kTileN;
    ti.n_valid = min(kTileN, min(it.vis, it.a_len) - t * kTileN);
    ti.key_base = t * kTileN;
    ti.b_first = 0;
  } else {
    const int tb = t - it.tiles_a;
    ti.src_b = 1;
    ti.row = it.b_row + tb * kTileN;
    ti.n_valid = min(kTileN, (it.vis - it.a_len) - tb * kTileN);
    ti.key_base = it.a_len + tb * kTileN;
    ti.b_first = tb * kTileN;
  }
  ti.n_valid = max(ti.n_valid, 0);
  return ti;
}

struct Walker {
  Item it;
  int t;          // tile index inside the item
  __device__ void begin(const AttnParams& p, int req, int qb, int t0) {
    load_item(p, req, qb, it);
    t = t0;
  }
  // Moves to the next tile; returns true when a new item was entered.
  __device__ bool advance(const AttnParams& p) {
    if (++t < it.tiles) return false;
    int req = it.req, qb = it.qb + 1;
    if (qb >= request_qblocks(p, req)) {
      ++req;
      qb = 0;
    }
    if (req < p.num_requests) load_item(p, req, qb, it);
    t = 0;
    return true;
  }
};

// CTA ranges are equal shares of *work*, not of tiles: an item costs its tiles
// plus kItemCost tiles' worth of switching (the q prologue, the partial write of
// a cut item and the pipeline refill). Per-CTA traces put an item switch at about
// four tiles of streaming time, but whole layers of configs 2 and 3 measure
// shortest with 8-16 (charging the switch more also steers the cuts of long
// items away from CTAs that already hold several starts); 12 is used. The tiles of all items are numbered in request
// order and each item is preceded by a kItemCost-unit overhead zone in work
// units; CTA c owns the tiles of work units [c W / G, (c + 1) W / G), a work
// position inside an overhead zone meaning the item's first tile. Ranges stay
// contiguous and ordered in tile space, so a CTA that would otherwise take on
// two or three item switches gets correspondingly fewer tiles.
constexpr long long kItemCost = 12;

// Ranges a launch of `total` tiles is split into: every CTA of the grid for large
// launches, and about one range per kMinTilesPerRange tiles for small ones, where
// the per-CTA fixed costs would otherwise dominate. Every range then holds more
// than kItemCost work units, so none is empty.
constexpr long long kMinTilesPerRange = 12;
__device__ __forceinline__ long long sched_grid(long long total, long long grid) {
  const long long g = total / kMinTilesPerRange;
  return g < 1 ? 1 : (g < grid ? g : grid);
}

// Inclusive block-wide scan of v over all threads of the CTA.
template <int kThreads>
__device__ long long block_scan(long long v, long long* tmp, long long& total) {
  constexpr int kWarps = kThreads / 32;
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const long long n = __shfl_up_sync(0xffffffffu, v, o);
    if (lane >= o) v += n;
  }
  if (lane == 31) tmp[warp] = v;
  __syncthreads();
  if (warp == 0) {
    long long w = lane < kWarps ? tmp[lane] : 0;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const long long n = __shfl_up_sync(0xffffffffu, w, o);
      if (lane >= o) w += n;
    }
    if (lane < kWarps) tmp[lane] = w;
  }
  __syncthreads();
  const long long prefix = warp > 0 ? tmp[warp - 1] : 0;
  total = tmp[kWarps - 1];
  __syncthreads();
  return v + prefix;
}

struct SchedShared {
  long long scan_tmp[32];
  long long total;
  long long start, end;
  long long req_prefix, last_prefix;
  int req0, qb0, t0;        // item and tile offset of this CTA's first tile
  int req_l, qb_l, t_l;     // item and tile offset of this CTA's last tile
  int issued[kStages];
};

// Tile offset inside request `req` of work offset `off` (its items laid out as
// [kItemCost overhead units][tiles] each; an offset inside an overhead zone maps
// to that item's first tile).
__device__ long long tile_in_request(const AttnParams& p, int req, long long off) {
  const int nqb = request_qblocks(p, req);
  long long before = 0;
  Item it;
  for (int qb = 0; qb < nqb; ++qb) {
    if (off < kItemCost) return before;
    off -= kItemCost;
    load_item(p, req, qb, it);
    if (off < it.tiles) return before + off;
    off -= it.tiles;
    before += it.tiles;
  }
  return before;
}

__device__ __forceinline__ long long request_work(const AttnParams& p, int req, long long tiles) {
  return tiles + kItemCost * request_qblocks(p, req);
}

// (q-block, tile offset) of the tile `off` tiles into request `req`.
__device__ __forceinline__ void locate_in_request(const AttnParams& p, int req, long long off, int& qb_out,
                                                  int& t_out, Item& it) {
  const int nqb = request_qblocks(p, req);
  int qb = 0;
  for (; qb < nqb; ++qb) {
    load_item(p, req, qb, it);
    if (off < it.tiles) break;
    off -= it.tiles;
  }
  qb_out = qb;
  t_out = static_cast<int>(off);
}

// Finds the total tile count and the items holding this CTA's first and last
// tiles. All threads of the CTA must call it. With at most one request per
// thread the tile counts are scanned once; otherwise twice (total, then place).
template <int kThreads>
__device__ void locate_range(const AttnParams& p, SchedShared& s) {
  const int tid = threadIdx.x;
  if (tid == 0) {
    s.req0 = -1;
    s.req_l = -1;
  }
  long long total, start, end, chunk_total, work;
  if (p.num_requests <= kThreads) {
    const long long t = tid < p.num_requests ? request_tiles(p, tid) : 0;
    const long long wk = tid < p.num_requests ? request_work(p, tid, t) : 0;
    const long long incl = block_scan<kThreads>(t, s.scan_tmp, total);
    const long long incl_w = block_scan<kThreads>(wk, s.scan_tmp, work);
    const long long g = sched_grid(total, p.grid);
    const long long ws = blockIdx.x < g ? (blockIdx.x * work) / g : work;
    const long long we = blockIdx.x < g ? ((blockIdx.x + 1) * work) / g : work;
    if (tid == 0) {
      s.start = total;
      s.end = total;
    }
    __syncthreads();
    if (tid < p.num_requests) {
      const long long ew = incl_w - wk, et = incl - t;
      if (ew <= ws && ws < incl_w) s.start = et + tile_in_request(p, tid, ws - ew);
      if (ew <= we && we < incl_w) s.end = et + tile_in_request(p, tid, we - ew);
    }
    __syncthreads();
    start = s.start;
    end = s.end;
    if (tid < p.num_requests && start < end) {
      const long long excl = incl - t;
      if (excl <= start && start < incl) {
        s.req0 = tid;
        s.req_prefix = excl;
      }
      if (excl <= end - 1 && end - 1 < incl) {
        s.req_l = tid;
        s.last_prefix = excl;
      }
    }
  } else {
    long long running = 0, running_w = 0, chunk_w;
    for (int base = 0; base < p.num_requests; base += kThreads) {
      const int i = base + tid;
      const long long t = i < p.num_requests ? request_tiles(p, i) : 0;
      const long long wk = i < p.num_requests ? request_work(p, i, t) : 0;
      block_scan<kThreads>(t, s.scan_tmp, chunk_total);
      block_scan<kThreads>(wk, s.scan_tmp, chunk_w);
      running += chunk_total;
      running_w += chunk_w;
    }
    total = running;
    work = running_w;
    const long long g = sched_grid(total, p.grid);
    const long long ws = blockIdx.x < g ? (blockIdx.x * work) / g : work;
    const long long we = blockIdx.x < g ? ((blockIdx.x + 1) * work) / g : work;
    if (tid == 0) {
      s.start = total;
      s.end = total;
    }
    __syncthreads();
    running = 0;
    running_w = 0;
    for (int base = 0; base < p.num_requests; base += kThreads) {
      const int i = base + tid;
      const long long t = i < p.num_requests ? request_tiles(p, i) : 0;
      const long long wk = i < p.num_requests ? request_work(p, i, t) : 0;
      const long long incl = running + block_scan<kThreads>(t, s.scan_tmp, chunk_total);
      const long long incl_w = running_w + block_scan<kThreads>(wk, s.scan_tmp, chunk_w);
      if (i < p.num_requests) {
        const long long ew = incl_w - wk, et = incl - t;
        if (ew <= ws && ws < incl_w) s.start = et + tile_in_request(p, i, ws - ew);
        if (ew <= we && we < incl_w) s.end = et + tile_in_request(p, i, we - ew);
      }
      running += chunk_total;
      running_w += chunk_w;
    }
    __syncthreads();
    start = s.start;
    end = s.end;
    if (start < end) {
      running = 0;
      for (int base = 0; base < p.num_requests; base += kThreads) {
        const int i = base + tid;
        const long long t = i < p.num_requests ? request_tiles(p, i) : 0;
        const long long incl = running + block_scan<kThreads>(t, s.scan_tmp, chunk_total);
        if (i < p.num_requests && incl - t <= start && start < incl) {
          s.req0 = i;
          s.req_prefix = incl - t;
        }
        if (i < p.num_requests && incl - t <= end - 1 && end - 1 < incl) {
          s.req_l = i;
          s.last_prefix = incl - t;
        }
        running += chunk_total;
      }
    }
  }
  __syncthreads();
  if (tid == 0) {
    s.total = total;
    s.start = start;
    s.end = end;
    p.ranges[2 * blockIdx.x] = start;                // read by the merge kernel
    p.ranges[2 * blockIdx.x + 1] = end;
    if (start < end) {
      if (s.req0 < 0 || s.req_l < 0) {
        atomicOr(&g_device_status, kStatusBadSchedule);
        s.end = s.start;   // nothing to do
      } else {
        Item it;
        locate_in_request(p, s.req0, start - s.req_prefix, s.qb0, s.t0, it);
        locate_in_request(p, s.req_l, end - 1 - s.last_prefix, s.qb_l, s.t_l, it);
      }
    }
  }
  __syncthreads();
}

__device__ __forceinline__ float quad_max(float v) {
  v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 1));
  return fmaxf(v, __shfl_xor_sync(0xffffffffu, v, 2));
}

__device__ __forceinline__ float quad_sum(float v) {
  v += __shfl_xor_sync(0xffffffffu, v, 1);
  return v + __shfl_xor_sync(0xffffffffu, v, 2);
}

__device__ __forceinline__ float bf16r(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

__device__ __forceinline__ float2 unpack_bf16x2(uint32_t v) {
  __nv_bfloat162 b = *reinterpret_cast<__nv_bfloat162*>(&v);
  return __bfloat1622float2(b);
}

// Sum of the 128 squares of one head vector, associated exactly as torch's CPU
// float32 reduction associates a contiguous 128-element row (8-wide vectors, four
// vector accumulators; transformers' Qwen3RMSNorm runs pow(2).mean(-1) through it).
// With d = 32 i + 8 k + j (i, k < 4, j < 8):
//   acc[k][j] = ((s[0,k,j] + s[1,k,j]) + s[2,k,j]) + s[3,k,j]
//   P[j]      = ((acc[0][j] + acc[1][j]) + acc[2][j]) + acc[3][j]
//   total     = (((((((P[0] + P[1]) + P[2]) + P[3]) + P[4]) + P[5]) + P[6]) + P[7])
// Each add rounds, so the association decides the last bit of the mean square and,
// through the rsqrt, which bf16 value a normalised element rounds to; with this order
// the normalised (and roped) head equals the reference's CPU result bit for bit.
// Explicit _rn intrinsics keep the compiler from contracting or reassociating.

// Warp layout: lane l holds s[r] = square of d = 4 l + r. Result broadcast to all lanes.
__device__ __forceinline__ float torch_order_sumsq_lane4(const float (&s)[4]) {
  constexpr unsigned kAll = 0xffffffffu;
  float t[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) {   // lanes 0..7 end with acc[lane >> 1][4 (lane & 1) + r]
    float a = __fadd_rn(s[r], __shfl_down_sync(kAll, s[r], 8));
    a = __fadd_rn(a, __shfl_down_sync(kAll, s[r], 16));
    t[r] = __fadd_rn(a, __shfl_down_sync(kAll, s[r], 24));
  }
#pragma unroll
  for (int r = 0; r < 4; ++r) {   // lanes 0, 1 end with P[4 lane + r]
    float a = __fadd_rn(t[r], __shfl_down_sync(kAll, t[r], 2));
    a = __fadd_rn(a, __shfl_down_sync(kAll, t[r], 4));
    t[r] = __fadd_rn(a, __shfl_down_sync(kAll, t[r], 6));
  }
  float upper[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) upper[r] = __shfl_down_sync(kAll, t[r], 1);
  float total = __fadd_rn(__fadd_rn(__fadd_rn(t[0], t[1]), t[2]), t[3]);
#pragma unroll
  for (int r = 0; r < 4; ++r) total = __fadd_rn(total, upper[r]);
  return __shfl_sync(kAll, total, 0);
}

// MMA A-fragment layout: the quad (t4 = lane & 3) holds one row; sq[ks][e] is the
// square of d = 16 ks + 2 t4 + (e & 1) + 8 (e >> 1), i.e. i = ks >> 1,
// k = 2 (ks & 1) + (e >> 1), j = 2 t4 + (e & 1). Result on all four lanes.
__device__ __forceinline__ float torch_order_sumsq_quad(const float (&sq)[8][4]) {
  float p[2];
#pragma unroll
  for (int jj = 0; jj < 2; ++jj) {
    float acc[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const int e = 2 * (k & 1) + jj, ks0 = k >> 1;
      float a = __fadd_rn(sq[ks0][e], sq[ks0 + 2][e]);
      a = __fadd_rn(a, sq[ks0 + 4][e]);
      acc[k] = __fadd_rn(a, sq[ks0 + 6][e]);
    }
    p[jj] = __fadd_rn(__fadd_rn(__fadd_rn(acc[0], acc[1]), acc[2]), acc[3]);
  }
  float total = 0.f;
#pragma unroll
  for (int q = 0; q < 4; ++q) {   // P[2q] and P[2q + 1] live on quad lane q
    const float pe = __shfl_sync(0xffffffffu, p[0], q, 4), po = __shfl_sync(0xffffffffu, p[1], q, 4);
    total = q == 0 ? __fadd_rn(pe, po) : __fadd_rn(__fadd_rn(total, pe), po);
  }
  return total;
}

// 1 / sqrt(sum / 128 + eps) with one rounding per step, as torch's CPU
// mean (sum then divide), add and rsqrt (a rounded sqrt, then a rounded divide).
__device__ __forceinline__ float rms_reciprocal(float sumsq, float eps) {
  return __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fmul_rn(sumsq, 0.0078125f), eps)));
}

// Qwen3 RMSNorm + rotate-half RoPE (bf16 arithmetic order of transformers) of
// one head of one MMA A-fragment row: regs lo[ks] hold d = 16ks+2t, +1 and
// hi[ks] hold d = 16ks+2t+8, +9 (t = lane & 3). The quad (4 lanes) holds the
// full 128-d row; the RoPE partner d+64 of d < 64 is the same thread's ks+4.
// cs/sn: bf16-rounded cos/sin of this thread's 16 frequencies (ks<4, e).
__device__ __forceinline__ void norm_rope_fragment(uint32_t (&lo)[8], uint32_t (&hi)[8], const AttnParams& p,
                                                   const __nv_bfloat16* w, const float (&cs)[4][4],
                                                   const float (&sn)[4][4], int t4) {
  float x[8][4], sq[8][4];
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const float2 a = unpack_bf16x2(lo[ks]), b = unpack_bf16x2(hi[ks]);
    x[ks][0] = a.x;
    x[ks][1] = a.y;
    x[ks][2] = b.x;
    x[ks][3] = b.y;
#pragma unroll
    for (int e = 0; e < 4; ++e) sq[ks][e] = __fmul_rn(x[ks][e], x[ks][e]);
  }
  const float rs = rms_reciprocal(torch_order_sumsq_quad(sq), p.eps);
#pragma unroll
  for (int ks = 0; ks < 8; ++ks)
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const int d = ks * 16 + 2 * t4 + (e & 1) + (e >> 1) * 8;
      x[ks][e] = bf16r(__bfloat162float(w[d]) * bf16r(x[ks][e] * rs));
    }
#pragma unroll
  for (int ks = 0; ks < 4; ++ks) {
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float c = cs[ks][e], s = sn[ks][e];
      const float a = x[ks][e], b = x[ks + 4][e];
      x[ks][e] = bf16r(bf16r(a * c) + bf16r(-b * s));
      x[ks + 4][e] = bf16r(bf16r(b * c) + bf16r(a * s));
    }
  }
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    lo[ks] = pack_bf16x2(x[ks][0], x[ks][1]);
    hi[ks] = pack_bf16x2(x[ks][2], x[ks][3]);
  }
}

// Fused verify: a source-B tile holds the raw k/v projections of a request's
// new rows (TMA-loaded from k_new/v_new like any other tile). The consumer
// warp of KV head h applies k_norm + RoPE to its head's rows in shared memory
// (row rr of the tile is request row b_first + rr, at position
// a_len + b_first + rr) and appends roped k and raw v to the layer's scratch.
// Lane l owns d = 4l..4l+3; the rotate-half partner of d lives in lane l ^ 16.
__device__ __forceinline__ void rope_new_rows_in_smem(const AttnParams& p, const Item& it, const Tile& ti, int h,
                                                      int lane, uint8_t* stage, const uint8_t* rope_rows,
                                                      const __nv_bfloat16* kw_smem) {
  const int d0 = lane * 4;
  float w[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) w[i] = __bfloat162float(kw_smem[d0 + i]);
  const int half = lane >> 4;                 // d < 64 -> low half box
  const int chunk = (lane & 15) >> 1;         // 16-byte chunk inside the 128-byte half row
  const int sub = (lane & 1) * 8;             // byte offset inside the chunk
  const int f0 = d0 & 63;                     // frequencies of d0..d0+3
  for (int rr = 0; rr < ti.n_valid; ++rr) {   // warp-uniform bound
    const int row = it.q_start + ti.b_first + rr;
    if (row < 0 || row >= p.total_q || row >= p.scratch_rows) continue;
    const int soff = (h * kTileN + rr) * 128 + ((chunk ^ (rr & 7)) << 4) + sub;
    uint2* ks = reinterpret_cast<uint2*>(stage + half * kHalfBoxBytes + soff);
    const uint2 raw = *ks;
    const uint2 vraw = *reinterpret_cast<const uint2*>(stage + (2 + half) * kHalfBoxBytes + soff);
    const uint4 cs4 = *reinterpret_cast<const uint4*>(rope_rows + rr * kRopeRowBytes + f0 * 4);
    const uint32_t csw[4] = {cs4.x, cs4.y, cs4.z, cs4.w};
    const float2 a = unpack_bf16x2(raw.x), b = unpack_bf16x2(raw.y);
    const float x[4] = {a.x, a.y, b.x, b.y};
    const float sq[4] = {__fmul_rn(x[0], x[0]), __fmul_rn(x[1], x[1]), __fmul_rn(x[2], x[2]), __fmul_rn(x[3], x[3])};
    const float rs = rms_reciprocal(torch_order_sumsq_lane4(sq), p.eps);
    float y[4], partner[4], out[4];
#pragma unroll
    for (int e = 0; e < 4; ++e) y[e] = bf16r(w[e] * bf16r(x[e] * rs));
#pragma unroll
    for (int e = 0; e < 4; ++e) partner[e] = __shfl_xor_sync(0xffffffffu, y[e], 16);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      const float2 c_s = unpack_bf16x2(csw[e]);
      const float rot = lane < 16 ? -partner[e] : partner[e];
      out[e] = bf16r(bf16r(y[e] * c_s.x) + bf16r(rot * c_s.y));
    }
    uint2 kv;
    kv.x = pack_bf16x2(out[0], out[1]);
    kv.y = pack_bf16x2(out[2], out[3]);
    *ks = kv;
    const size_t off = (static_cast<size_t>(row) * kKVHeads + h) * kHeadDim + d0;
    *reinterpret_cast<uint2*>(p.scratch_k + off) = kv;
    *reinterpret_cast<uint2*>(p.scratch_v + off) = vraw;
  }
}

// A cut item's contribution from this CTA (warp of KV head h): store the fp32
// partial O (unnormalised), row max m and row sum l. The CTA holding the
// item's first tile records the item for split_merge_kernel, which combines
// the partials after this kernel; no CTA waits on another one here.
__device__ __forceinline__ void finish_split_item(const AttnParams& p, const Item& it, long long item_start,
                                                  long long item_end, long long start, long long total, int h,
                                                  int lane, const float (&o)[16][4], float m_a, float m_b, float l_a,
                                                  float l_b) {
  const int g = lane >> 2, t4 = lane & 3;
  const int slot = item_start <= start ? 0 : 1;
  const size_t base = (static_cast<size_t>(blockIdx.x) * 2 + slot) * kKVHeads + h;
  float* po = p.part_o + base * 16 * kHeadDim;
#pragma unroll
  for (int j = 0; j < 16; ++j) {
    const int d = j * 8 + 2 * t4;
    __stcg(reinterpret_cast<float2*>(po + g * kHeadDim + d), make_float2(o[j][0], o[j][1]));
    __stcg(reinterpret_cast<float2*>(po + (g + 8) * kHeadDim + d), make_float2(o[j][2], o[j][3]));
  }
  if (t4 == 0) {
    float* pml = p.part_ml + base * 32;
    __stcg(reinterpret_cast<float2*>(pml + 2 * g), make_float2(m_a, l_a));
    __stcg(reinterpret_cast<float2*>(pml + 2 * (g + 8)), make_float2(m_b, l_b));
  }
  if (item_start >= start && lane == 0) {
    // Partial slot 1 holds an item that began after the range start (a CTA's
    // last item), slot 0 one that began at or before it (its first item); every
    // later contributor holds this item as its first one, in slot 0.
    MergeEntry e;
    e.item_start = item_start;
    e.item_end = item_end;
    e.first = static_cast<int>(blockIdx.x);
    e.slot_first = slot;
    e.q0 = it.q0;
    e.nrows = it.nrows;
    e.valid = 1;
    e.pad[0] = e.pad[1] = e.pad[2] = 0;
    p.merges[static_cast<size_t>(blockIdx.x) * kKVHeads + h] = e;
  }
}

// Merge of the cut items, launched right after the attention kernel (as a
// programmatic dependent launch where available, so its CTAs are resident
// before the attention kernel ends). CTA (c, h) merges the item CTA c
// recorded for KV head h, if any: warp w owns rows 4w..4w+3 of the head pair
// (row r: head 2h + r / 8, query row q0 + r % 8), lane l owns d = 4l..4l+3.
// Two passes over the contributors, four contributors' loads per round: the
// row maximum M and sum L = sum_c l_c 2^((m_c - M) s), then
// out = sum_c 2^((m_c - M) s) O_c / L. The contributors are the CTAs from the
// recorded first one whose ranges (written by every CTA of the launch) start
// before the item's end; ranges are never empty.
constexpr int kMergeThreads = 128;
__global__ void __launch_bounds__(kMergeThreads) split_merge_kernel(const AttnParams p) {
  asm volatile("griddepcontrol.wait;" ::: "memory");
  const int c0 = static_cast<int>(blockIdx.x) / kKVHeads, h = static_cast<int>(blockIdx.x) % kKVHeads;
  if (c0 >= p.grid) return;
  const MergeEntry e = p.merges[blockIdx.x];
  if (!e.valid) return;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // last contributor: ranges are ordered, so the contributors after the first are
  // the CTAs c > first with range start < item end (counted kMergeThreads at a time)
  int last = e.first;
  for (int base = e.first + 1; base < p.grid; base += kMergeThreads) {
    const int c = base + static_cast<int>(threadIdx.x);
    const int n = __syncthreads_count(c < p.grid && p.ranges[2 * c] < e.item_end);
    last += n;
    if (n < kMergeThreads) break;
  }
  const float sl2 = p.scale_log2;
  const int my_row = 4 * warp + (lane & 3);   // row whose statistics this lane tracks
  const int d = lane * 4;
  auto block = [&](int c) -> long long {
    if (c > last) return -1;
    const int sl = c == e.first ? e.slot_first : 0;
    return (static_cast<long long>(c) * 2 + sl) * kKVHeads + h;
  };
  float mrow = -INFINITY, lrow = 0.f;
#pragma unroll 1
  for (int c = e.first; c <= last; c += 4) {
    float2 ml[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long bi = block(c + u);
      ml[u] = bi >= 0 ? __ldcg(reinterpret_cast<const float2*>(p.part_ml + bi * 32 + 2 * my_row))
                      : make_float2(-INFINITY, 0.f);
    }
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const float mnew = fmaxf(mrow, ml[u].x);
      const float mu = mnew == -INFINITY ? 0.f : mnew;
      lrow = lrow * ex2((mrow - mu) * sl2) + ml[u].y * ex2((ml[u].x - mu) * sl2);
      mrow = mnew;
    }
  }
  const float mu = mrow == -INFINITY ? 0.f : mrow;
  const float inv = lrow > 0.f ? 1.f / lrow : 0.f;
  float4 acc[4];
#pragma unroll
  for (int r = 0; r < 4; ++r) acc[r] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
  for (int c = e.first; c <= last; c += 4) {
    float4 v[4][4];
    float wl[4];
#pragma unroll
    for (int u = 0; u < 4; ++u) {
      const long long bi = block(c + u);
      const float* po = p.part_o + (bi * 16 + 4 * warp) * kHeadDim + d;
      const float2 ml = bi >= 0 ? __ldcg(reinterpret_cast<const float2*>(p.part_ml + bi * 32 + 2 * my_row))
                                : make_float2(-INFINITY, 0.f);
#pragma unroll
      for (int r = 0; r < 4; ++r)
        v[u][r] = bi >= 0 ? __ldcg(reinterpret_cast<const float4*>(po + r * kHeadDim))
                          : make_float4(0.f, 0.f, 0.f, 0.f);
      wl[u] = ex2((ml.x - mu) * sl2) * inv;
    }
#pragma unroll
    for (int u = 0; u < 4; ++u)
#pragma unroll
      for (int r = 0; r < 4; ++r) {
        const float wr = __shfl_sync(0xffffffffu, wl[u], r);
        acc[r].x = fmaf(wr, v[u][r].x, acc[r].x);
        acc[r].y = fmaf(wr, v[u][r].y, acc[r].y);
        acc[r].z = fmaf(wr, v[u][r].z, acc[r].z);
        acc[r].w = fmaf(wr, v[u][r].w, acc[r].w);
      }
  }
  __nv_bfloat16* og = static_cast<__nv_bfloat16*>(p.out);
#pragma unroll
  for (int r = 0; r < 4; ++r) {
    const int rr = 4 * warp + r, qr = rr & 7, row = e.q0 + qr;
    if (qr >= e.nrows || row < 0 || row >= p.total_q) continue;
    __nv_bfloat16* dst = og + (static_cast<size_t>(row) * kQHeads + 2 * h + (rr >> 3)) * kHeadDim + d;
    uint2 res;
    res.x = pack_bf16x2(acc[r].x, acc[r].y);
    res.y = pack_bf16x2(acc[r].z, acc[r].w);
    *reinterpret_cast<uint2*>(dst) = res;
  }
}

// Q fragments of heads 2h (MMA rows 0-7) and 2h+1 (rows 8-15) for query row
// g of item `it`; in fused verify mode they are normalised and rotated here.
template <bool kFused>
__device__ __forceinline__ void load_q_fragments(const AttnParams& p, const Item& it, int h, int lane,
                                                 const __nv_bfloat16* qw_smem, uint32_t (&qf)[8][4]) {
  const int g = lane >> 2, t4 = lane & 3;
  const int row = it.q0 + g;
  const bool rv = g < it.nrows && row >= 0 && row < p.total_q;
  const __nv_bfloat16* qa =
      static_cast<const __nv_bfloat16*>(p.q) + (static_cast<size_t>(row) * kQHeads + 2 * h) * kHeadDim;
  const __nv_bfloat16* qb = qa + kHeadDim;
#pragma unroll
  for (int ks = 0; ks < 8; ++ks) {
    const int d = ks * 16 + 2 * t4;
    qf[ks][0] = rv ? ld_nc_u32(qa + d) : 0u;
    qf[ks][1] = rv ? ld_nc_u32(qb + d) : 0u;
    qf[ks][2] = rv ? ld_nc_u32(qa + d + 8) : 0u;
    qf[ks][3] = rv ? ld_nc_u32(qb + d + 8) : 0u;
  }
  if (kFused) {
    // q_norm + RoPE of the raw projections; row g sits at position a_len + qb*8 + g.
    // cos/sin of this row's position for d = 16ks+2t+{0,1} and +{8,9} (ks < 4).
    float cs[4][4], sn[4][4];
    const uint32_t* tr = p.rope + static_cast<size_t>(rv ? row : 0) * 64 + 2 * t4;
#pragma unroll
    for (int ks = 0; ks < 4; ++ks) {
      const uint2 lo2 = __ldg(reinterpret_cast<const uint2*>(tr + ks * 16));
      const uint2 hi2 = __ldg(reinterpret_cast<const uint2*>(tr + ks * 16 + 8));
      const uint32_t e4[4] = {lo2.x, lo2.y, hi2.x, hi2.y};
#pragma unroll
      for (int e = 0; e < 4; ++e) {
        const float2 cv = unpack_bf16x2(e4[e]);
        cs[ks][e] = cv.x;
        sn[ks][e] = cv.y;
      }
    }
    // One head at a time through the same code: this prologue runs once per item
    // and CTA, and an unrolled copy per head mostly costs instruction fetches.
    uint32_t lo[8], hi[8];
#pragma unroll 1
    for (int hh = 0; hh < 2; ++hh) {
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        lo[ks] = hh ? qf[ks][1] : qf[ks][0];
        hi[ks] = hh ? qf[ks][3] : qf[ks][2];
      }
      norm_rope_fragment(lo, hi, p, qw_smem, cs, sn, t4);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        if (hh) {
          qf[ks][1] = rv ? lo[ks] : 0u;
          qf[ks][3] = rv ? hi[ks] : 0u;
        } else {
          qf[ks][0] = rv ? lo[ks] : 0u;
          qf[ks][2] = rv ? hi[ks] : 0u;
        }
      }
    }
  }
}

// ---------------------------------------------------------------------------
// bf16 tensor-core kernel
// ---------------------------------------------------------------------------
template <bool kCausal, bool kFused>
__global__ void __launch_bounds__(kAttnThreads, 1)
    attn_bf16_kernel(const __grid_constant__ CUtensorMap tm_ka, const __grid_constant__ CUtensorMap tm_va,
                     const __grid_constant__ CUtensorMap tm_kb, const __grid_constant__ CUtensorMap tm_vb,
                     const AttnParams p) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + kSmemBarOff);
  uint64_t* empty = full + kStages;
  SchedShared& sched = *reinterpret_cast<SchedShared*>(empty + kStages);
  __nv_bfloat16* qw_smem = reinterpret_cast<__nv_bfloat16*>(smem + kSmemWeightOff);
  __nv_bfloat16* kw_smem = qw_smem + kHeadDim;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (kFused && threadIdx.x < kHeadDim) {
    qw_smem[threadIdx.x] = p.q_w[threadIdx.x];
    kw_smem[threadIdx.x] = p.k_w[threadIdx.x];
  }
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(smem_u32(&full[s]), 1);
      mbar_init(smem_u32(&empty[s]), kConsumerWarps);
      sched.issued[s] = 0;
    }
    fence_barrier_init();
  }
  asm volatile("griddepcontrol.launch_dependents;");
  // every CTA of the launch rewrites its merge entries (valid ones later)
  if (warp < kConsumerWarps && lane == 0) p.merges[static_cast<size_t>(blockIdx.x) * kKVHeads + warp].valid = 0;
  locate_range<kAttnThreads>(p, sched);   // contains __syncthreads
  const long long start = sched.start, end = sched.end, total = sched.total;
  if (start >= end) return;

  if (warp == kConsumerWarps) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      prefetch_tmap(&tm_ka);
      prefetch_tmap(&tm_va);
      prefetch_tmap(&tm_kb);
      prefetch_tmap(&tm_vb);
      int issued[kStages] = {};
      int kl = 0;
      bool prep_done = false;
      Walker w;
      w.begin(p, sched.req0, sched.qb0, sched.t0);
      {
        for (long long gk = start; gk < end; ++gk, ++kl) {
          const int stage = kl % kStages;
          const uint32_t parity = ((kl / kStages) & 1) ^ 1;
          if (!mbar_wait(smem_u32(&empty[stage]), parity)) break;
          const Tile ti = tile_of(w.it, w.t);
          if (ti.src_b && !prep_done) {
            // launched as a dependent of the verify prep kernel: the source-B
            // (scratch) rows are complete past this point; resident rows
            // before it stream while the prep runs (a no-op otherwise)
            asm volatile("griddepcontrol.wait;" ::: "memory");
            prep_done = true;
          }
          const uint32_t bar = smem_u32(&full[stage]);
          const CUtensorMap* mk = ti.src_b ? &tm_kb : &tm_ka;
          const CUtensorMap* mv = ti.src_b ? &tm_vb : &tm_va;
          const uint32_t dst = smem_u32(smem + stage * kStageBytes);
          // fused new-row tile: also its rows of the cos/sin table (clamped to the table)
          const int rope_rows = (kFused && ti.src_b) ? max(0, min(kTileN, p.total_q - ti.row)) : 0;
          mbar_arrive_expect_tx(bar, kStageBytes + rope_rows * kRopeRowBytes);
          if (rope_rows > 0)
            bulk_load(smem_u32(smem + kSmemRopeOff + stage * kRopeStageBytes),
                      p.rope + static_cast<size_t>(ti.row) * 64, rope_rows * kRopeRowBytes, bar);
          tma_load_3d(dst, mk, 0, ti.row, 0, bar);
          tma_load_3d(dst + kHalfBoxBytes, mk, 64, ti.row, 0, bar);
          tma_load_3d(dst + 2 * kHalfBoxBytes, mv, 0, ti.row, 0, bar);
          tma_load_3d(dst + 3 * kHalfBoxBytes, mv, 64, ti.row, 0, bar);
          ++issued[stage];
          w.advance(p);
        }
      }
      for (int s = 0; s < kStages; ++s) sched.issued[s] = issued[s];
    }
  } else {
    // ------------------------------ consumers -----------------------------
    const int h = warp;
    const int g = lane >> 2, t4 = lane & 3;
    const float sl2 = p.scale_log2;
    __nv_bfloat16* og = static_cast<__nv_bfloat16*>(p.out);

    uint32_t qf[8][4];
    float o[16][4];
    float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
    int kl = 0;
    Walker w;
    w.begin(p, sched.req0, sched.qb0, sched.t0);
    long long item_start = start - w.t;
    // launched as a dependent of the verify prep kernel: q is complete past this
    // point (a no-op for an ordinary launch)
    asm volatile("griddepcontrol.wait;" ::: "memory");
    load_q_fragments<kFused>(p, w.it, h, lane, qw_smem, qf);
#pragma unroll
    for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
    m_a = m_b = -INFINITY;
    l_a = l_b = 0.f;

    for (long long gk = start; gk < end; ++gk, ++kl) {
      const int stage = kl % kStages;
      const uint32_t parity = (kl / kStages) & 1;
      const Item& it = w.it;
      if (!mbar_wait(smem_u32(&full[stage]), parity)) break;
      const Tile ti = tile_of(it, w.t);
      const bool self_filled = kFused && ti.src_b;
      if (self_filled) {
        rope_new_rows_in_smem(p, it, ti, h, lane, smem + stage * kStageBytes,
                              smem + kSmemRopeOff + stage * kRopeStageBytes, kw_smem);
        __syncwarp();
      }
      const uint32_t sbase = smem_u32(smem + stage * kStageBytes);
      const uint32_t head_off = static_cast<uint32_t>(h * kTileN * 128);

      // S = Q K^T over 16 keys (two n8 tiles).
      float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
      {
        const int n = ((lane >> 4) << 3) + (lane & 7);
        const uint32_t rowaddr = sbase + head_off + n * 128;
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const int chunk = ((ks & 3) << 1) + ((lane >> 3) & 1);
          const uint32_t addr = rowaddr + (ks >> 2) * kHalfBoxBytes + ((chunk ^ (n & 7)) << 4);
          uint32_t b0, b1, b2, b3;
          ldsm_x4(addr, b0, b1, b2, b3);
          mma_bf16(s0, qf[ks], b0, b1);
          mma_bf16(s1, qf[ks], b2, b3);
        }
      }
      // Mask: keys past the tile's valid count, and (causal) past the row limit.
      const int j0 = 2 * t4, j2 = 8 + 2 * t4;
      int lim = ti.n_valid;
      if (kCausal) {
        const int row_lim = it.k_len - it.q_len + it.qb * kQBlock + g - ti.key_base + 1;
        lim = min(lim, row_lim);
      }
      const bool v0 = j0 < lim, v1 = j0 + 1 < lim, v2 = j2 < lim, v3 = j2 + 1 < lim;
      s0[0] = v0 ? s0[0] : -INFINITY;
      s0[1] = v1 ? s0[1] : -INFINITY;
      s0[2] = v0 ? s0[2] : -INFINITY;
      s0[3] = v1 ? s0[3] : -INFINITY;
      s1[0] = v2 ? s1[0] : -INFINITY;
      s1[1] = v3 ? s1[1] : -INFINITY;
      s1[2] = v2 ? s1[2] : -INFINITY;
      s1[3] = v3 ? s1[3] : -INFINITY;

      // Online softmax (fp32), rows A = head 2h, B = head 2h+1.
      const float mx_a = quad_max(fmaxf(fmaxf(s0[0], s0[1]), fmaxf(s1[0], s1[1])));
      const float mx_b = quad_max(fmaxf(fmaxf(s0[2], s0[3]), fmaxf(s1[2], s1[3])));
      const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
      const float mu_a = mn_a == -INFINITY ? 0.f : mn_a;
      const float mu_b = mn_b == -INFINITY ? 0.f : mn_b;
      const float alpha_a = ex2((m_a - mu_a) * sl2), alpha_b = ex2((m_b - mu_b) * sl2);
      m_a = mn_a;
      m_b = mn_b;
      const float nb_a = -mu_a * sl2, nb_b = -mu_b * sl2;
      float p0[4], p1[4];
      p0[0] = ex2(fmaf(s0[0], sl2, nb_a));
      p0[1] = ex2(fmaf(s0[1], sl2, nb_a));
      p1[0] = ex2(fmaf(s1[0], sl2, nb_a));
      p1[1] = ex2(fmaf(s1[1], sl2, nb_a));
      p0[2] = ex2(fmaf(s0[2], sl2, nb_b));
      p0[3] = ex2(fmaf(s0[3], sl2, nb_b));
      p1[2] = ex2(fmaf(s1[2], sl2, nb_b));
      p1[3] = ex2(fmaf(s1[3], sl2, nb_b));
      l_a = l_a * alpha_a + (p0[0] + p0[1] + p1[0] + p1[1]);
      l_b = l_b * alpha_b + (p0[2] + p0[3] + p1[2] + p1[3]);
#pragma unroll
      for (int j = 0; j < 16; ++j) {
        o[j][0] *= alpha_a;
        o[j][1] *= alpha_a;
        o[j][2] *= alpha_b;
        o[j][3] *= alpha_b;
      }
      uint32_t pa[4];
      pa[0] = pack_bf16x2(p0[0], p0[1]);
      pa[1] = pack_bf16x2(p0[2], p0[3]);
      pa[2] = pack_bf16x2(p1[0], p1[1]);
      pa[3] = pack_bf16x2(p1[2], p1[3]);

      // O += P V. Rows of V past the valid count may hold anything (next
      // request, capacity tail, NaN): zero them in the B fragments.
      const bool partial = ti.n_valid < kTileN;
      const uint32_t m_lo = (j0 < ti.n_valid ? 0x0000ffffu : 0u) | (j0 + 1 < ti.n_valid ? 0xffff0000u : 0u);
      const uint32_t m_hi = (j2 < ti.n_valid ? 0x0000ffffu : 0u) | (j2 + 1 < ti.n_valid ? 0xffff0000u : 0u);
      {
        const int n = (((lane >> 3) & 1) << 3) + (lane & 7);
        const uint32_t rowaddr = sbase + 2 * kHalfBoxBytes + head_off + n * 128;
#pragma unroll
        for (int j = 0; j < 16; j += 2) {
          const int chunk = (j & 7) + (lane >> 4);
          const uint32_t addr = rowaddr + (j >> 3) * kHalfBoxBytes + ((chunk ^ (n & 7)) << 4);
          uint32_t b0, b1, b2, b3;
          ldsm_x4_t(addr, b0, b1, b2, b3);
          if (partial) {
            b0 &= m_lo;
            b1 &= m_hi;
            b2 &= m_lo;
            b3 &= m_hi;
          }
          mma_bf16(o[j], pa, b0, b1);
          mma_bf16(o[j + 1], pa, b2, b3);
        }
      }
      // Generic-proxy writes into the stage must be ordered before the next TMA
      // write into it.
      if (self_filled) fence_proxy_async_smem();
      __syncwarp();
      if (lane == 0) mbar_arrive(smem_u32(&empty[stage]));

      const bool last_tile = w.t + 1 >= it.tiles;
      if (last_tile || gk + 1 == end) {
        const float la = quad_sum(l_a), lb = quad_sum(l_b);
        const long long item_end = item_start + it.tiles;
        if (item_start >= start && item_end <= end) {
          if (g < it.nrows && it.q0 + g < p.total_q && it.q0 + g >= 0) {
            const float ia = la > 0.f ? 1.f / la : 0.f, ib = lb > 0.f ? 1.f / lb : 0.f;
            __nv_bfloat16* oa = og + (static_cast<size_t>(it.q0 + g) * kQHeads + 2 * h) * kHeadDim;
            __nv_bfloat16* ob = oa + kHeadDim;
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int d = j * 8 + 2 * t4;
              *reinterpret_cast<uint32_t*>(oa + d) = pack_bf16x2(o[j][0] * ia, o[j][1] * ia);
              *reinterpret_cast<uint32_t*>(ob + d) = pack_bf16x2(o[j][2] * ib, o[j][3] * ib);
            }
          }
        } else {
          finish_split_item(p, it, item_start, item_end, start, total, h, lane, o, m_a, m_b, la, lb);
        }
        if (gk + 1 == end) break;                    // the range ends here
        // Next item: its Q replaces qf and its accumulators restart.
        w.advance(p);
        item_start = gk + 1;
        load_q_fragments<kFused>(p, w.it, h, lane, qw_smem, qf);
#pragma unroll
        for (int j = 0; j < 16; ++j) o[j][0] = o[j][1] = o[j][2] = o[j][3] = 0.f;
        m_a = m_b = -INFINITY;
        l_a = l_b = 0.f;
        continue;
      }
      w.advance(p);
    }
  }
  // Never leave the CTA with a TMA write still in flight (only possible after
  // a timed-out wait): wait, bounded, for the last load issued to each stage.
  __syncthreads();
  if (threadIdx.x == kConsumerWarps * 32) {
    for (int s = 0; s < kStages; ++s)
      if (sched.issued[s] > 0) mbar_wait(smem_u32(&full[s]), (sched.issued[s] - 1) & 1);
  }
}

// ---------------------------------------------------------------------------
// fp32 CUDA-core path: exact-precision companion for float32 inputs (the
// reference's CPU configurations). One CTA per (request, q-block, KV head).
// ---------------------------------------------------------------------------
constexpr int kF32Threads = 128;
constexpr int kF32Keys = 32;

__global__ void __launch_bounds__(kF32Threads)
    attn_f32_kernel(const float* __restrict__ ka, const float* __restrict__ va, const float* __restrict__ kb,
                    const float* __restrict__ vb, const AttnParams p) {
  __shared__ float sq[16][kHeadDim];
  __shared__ float sk[kF32Keys][kHeadDim + 1];
  __shared__ float sv[kF32Keys][kHeadDim];
  __shared__ float sp[16][kF32Keys];
  const int req = blockIdx.x, qb = blockIdx.y, h = blockIdx.z;
  if (qb >= request_qblocks(p, req)) return;
  Item it;
  load_item(p, req, qb, it);
  const float* qg = static_cast<const float*>(p.q);
  float* og = static_cast<float*>(p.out);
  const int tid = threadIdx.x;
  for (int u = tid; u < 16 * kHeadDim; u += kF32Threads) {
    const int m = u / kHeadDim, d = u % kHeadDim;
    const int r = m & 7, row = it.q0 + r;
    const bool ok = r < it.nrows && row < p.total_q;
    sq[m][d] = ok ? qg[(static_cast<size_t>(row) * kQHeads + 2 * h + (m >> 3)) * kHeadDim + d] : 0.f;
  }
  // thread -> (row m = tid/8, key group kq = tid%8): scores of keys 4kq..4kq+3
  const int m = tid >> 3, kq = tid & 7;
  float mrow = -INFINITY, lrow = 0.f;
  float acc[16];
#pragma unroll
  for (int i = 0; i < 16; ++i) acc[i] = 0.f;
  const int r = m & 7;
  const int row_lim = p.causal ? it.k_len - it.q_len + qb * kQBlock + r : INT_MAX;
  for (int kb0 = 0; kb0 < it.vis; kb0 += kF32Keys) {
    __syncthreads();
    for (int u = tid; u < kF32Keys * kHeadDim; u += kF32Threads) {
      const int n = u / kHeadDim, d = u % kHeadDim, j = kb0 + n;
      float kv = 0.f, vv = 0.f;
      if (j < it.vis) {
        long long row;
        const float *kp, *vp;
        long long rows;
        if (j < it.a_len) { row = static_cast<long long>(it.a_row) + j; kp = ka; vp = va; rows = p.rows_a; }
        else { row = static_cast<long long>(it.b_row) + (j - it.a_len); kp = kb; vp = vb; rows = p.rows_b; }
        if (row >= 0 && row < rows) {
          const size_t off = (static_cast<size_t>(row) * kKVHeads + h) * kHeadDim + d;
          kv = kp[off];
          vv = vp[off];
        } else {
          atomicOr(&g_device_status, kStatusBadArgument);
        }
      }
      sk[n][d] = kv;
      sv[n][d] = vv;
    }
    __syncthreads();
    float s[4];
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int n = kq * 4 + i, j = kb0 + n;
      float dot = 0.f;
      for (int d = 0; d < kHeadDim; ++d) dot = fmaf(sq[m][d], sk[n][d], dot);
      s[i] = (j < it.vis && j <= row_lim) ? dot * p.scale : -INFINITY;
    }
    float mx = fmaxf(fmaxf(s[0], s[1]), fmaxf(s[2], s[3]));
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    const float mn = fmaxf(mrow, mx);
    const float mu = mn == -INFINITY ? 0.f : mn;
    const float alpha = expf(mrow - mu);
    float ps = 0.f;
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const float e = expf(s[i] - mu);
      sp[m][kq * 4 + i] = e;
      ps += e;
    }
#pragma unroll
    for (int o = 1; o < 8; o <<= 1) ps += __shfl_xor_sync(0xffffffffu, ps, o);
    lrow = lrow * alpha + ps;
    mrow = mn;
    __syncwarp();
    // acc covers d = kq*16 .. kq*16+15 of row m
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] *= alpha;
    for (int n = 0; n < kF32Keys; ++n) {
      const float pn = sp[m][n];
#pragma unroll
      for (int i = 0; i < 16; ++i) acc[i] = fmaf(pn, sv[n][kq * 16 + i], acc[i]);
    }
  }
  const int row = it.q0 + r;
  if (r < it.nrows && row < p.total_q) {
    const float inv = lrow > 0.f ? 1.f / lrow : 0.f;
    float* dst = og + (static_cast<size_t>(row) * kQHeads + 2 * h + (m >> 3)) * kHeadDim + kq * 16;
#pragma unroll
    for (int i = 0; i < 16; ++i) dst[i] = acc[i] * inv;
  }
}

}  // namespace dspark
