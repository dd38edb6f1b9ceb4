// Stochastic acceptance of a verify round under the reference's float64 law
// (dspark_qwen/tensor_sampling.py): the target law p = softmax(logits / T)
// normalised once more (logits_to_probabilities, :38-51), the acceptance test
// u < min(p[t] / q[t], 1) per proposal, the residual law relu(p - q) / mass at the
// first rejection (residual_distribution, :87-96) or the bonus draw from the last
// target row, each sampled by the strict CDF rule with the last positive index
// past the end (sample_categorical, :77-84), and the stop rules of
// verify_proposal (:114-162).
//
// Three launches. scaled_table_kernel (bf16 logits only): x / T for all 65536
// bf16 bit patterns, the same IEEE division the reference does per element, so
// the later passes read it instead of dividing (the divisions were most of
// their float64 work). law_stats_kernel: one CTA per target row (max of x / T, the sum of
// exp(x / T - max) and the sum of the normalised weights) and one per draft row
// (a law: finite, in [0, 1], sum within 1e-12 of one). stochastic_accept_kernel:
// one CTA per request; thread 0 walks the proposals with the request's uniforms
// in the reference's draw order; a residual or bonus sample is a CTA-wide pass
// (mass, then a chunked CDF scan). All arithmetic is float64.
#pragma once
#include "pair.cuh"
#include "ptx.cuh"

namespace dspark {
namespace sampling {

constexpr int kThreads = 1024;   // one CTA per SM at 64 registers: twice the warps of 512 for the per-request kernel

enum Status {
  kOk = 0,
  kBadLogits = 1,        // non-finite logits or scaled logits
  kBadDraftLaw = 2,      // a draft row is not a float64 law
  kTokenRange = 3,       // proposal outside the vocabulary
  kZeroDraftMass = 4,    // proposal with zero mass under its own law
  kZeroResidual = 5,     // rejection with zero residual mass
  kBadUniform = 6,       // a uniform outside [0, 1)
  kBadLayout = 7,        // proposal offsets inconsistent with the buffers
};
enum Extra { kExtraNone = 0, kExtraResidual = 1, kExtraBonus = 2 };
enum Reason { kRoundComplete = 0, kEos = 1, kBudget = 2 };

struct RowStats {
  double m;    // max of x / T
  double s;    // sum of exp(x / T - m)
  double s2;   // sum of exp(x / T - m) / s
  int bad;     // status of the row (kOk, kBadLogits or kBadDraftLaw)
  int pad;
};

constexpr int kScaledTableSize = 65536;   // one float64 per bf16 bit pattern

struct Params {
  const void* logits;        // target rows, [rows, ld] bf16 or f32
  const double* scaled;      // bf16: x / T per bit pattern (kScaledTableSize); f32: null
  long long ld;
  int dtype;                 // 0 bf16, 1 f32
  int vocab;
  double temperature;
  int target_rows;
  const double* q;           // draft laws [draft_rows, vocab]
  int draft_rows;
  RowStats* stats;           // [target_rows + draft_rows]
  const long long* tokens;   // [draft_rows] proposals
  const int* cu_n;           // [R + 1] proposals of request i: rows cu_n[i] .. cu_n[i + 1]
  int num_requests;
  const double* uniforms;    // [R, u_stride]
  int u_stride;
  const long long* eos;
  int n_eos;
  const int* budget;         // [R] max new tokens of the round
  long long* emitted;        // [R, u_stride] committed tokens, -1 after
  int* result;               // [R, 8]: count, accepted, rejected, extra, reason, draws, status, 0
};

// x / T of the logit at (row, i): a table read for bf16 (x takes one of 65536
// values), the division for f32. Non-finite x gives non-finite x / T (T is
// finite and positive), so a finiteness check of x / T covers both.
__device__ __forceinline__ double load_scaled(const Params& p, long long row, int i) {
  if (p.dtype == 0)
    return p.scaled[static_cast<const unsigned short*>(p.logits)[row * p.ld + i]];
  return static_cast<double>(static_cast<const float*>(p.logits)[row * p.ld + i]) / p.temperature;
}

// Calls f(i, x_i / T) for this thread's share of row `row`: 8 consecutive bf16
// (one 16-byte load, their 8 table reads independent of each other, so they
// are in flight together) or 4 f32 per step when the row is 16-byte aligned,
// element by element otherwise and for the tail.
template <class F>
__device__ __forceinline__ void for_scaled(const Params& p, long long row, F f) {
  if (p.dtype == 0) {
    const unsigned short* r = static_cast<const unsigned short*>(p.logits) + row * p.ld;
    int i0 = 0;
    if ((reinterpret_cast<uintptr_t>(r) & 15) == 0) {
      const int nv = p.vocab / 8;
      for (int v = threadIdx.x; v < nv; v += kThreads) {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(r) + v);
        const unsigned short* h = reinterpret_cast<const unsigned short*>(&raw);
        double x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = __ldg(p.scaled + h[e]);
#pragma unroll
        for (int e = 0; e < 8; ++e) f(v * 8 + e, x[e]);
      }
      i0 = nv * 8;
    }
    for (int i = i0 + threadIdx.x; i < p.vocab; i += kThreads) f(i, p.scaled[r[i]]);
  } else {
    const float* r = static_cast<const float*>(p.logits) + row * p.ld;
    int i0 = 0;
    if ((reinterpret_cast<uintptr_t>(r) & 15) == 0) {
      const int nv = p.vocab / 4;
      for (int v = threadIdx.x; v < nv; v += kThreads) {
        const float4 raw = __ldg(reinterpret_cast<const float4*>(r) + v);
        f(v * 4, static_cast<double>(raw.x) / p.temperature);
        f(v * 4 + 1, static_cast<double>(raw.y) / p.temperature);
        f(v * 4 + 2, static_cast<double>(raw.z) / p.temperature);
        f(v * 4 + 3, static_cast<double>(raw.w) / p.temperature);
      }
      i0 = nv * 4;
    }
    for (int i = i0 + threadIdx.x; i < p.vocab; i += kThreads) f(i, static_cast<double>(r[i]) / p.temperature);
  }
}

__global__ void scaled_table_kernel(double* table, double temperature) {
  const int b = blockIdx.x * blockDim.x + threadIdx.x;
  if (b < kScaledTableSize)
    table[b] = static_cast<double>(__bfloat162float(__ushort_as_bfloat16(static_cast<unsigned short>(b)))) /
               temperature;
}

template <typename T, typename Op>
__device__ __forceinline__ T block_reduce(T v, T* scratch, Op op) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = op(v, __shfl_xor_sync(0xffffffffu, v, o));
  __syncthreads();                                   // scratch reuse across calls
  if (lane == 0) scratch[warp] = v;
  __syncthreads();
  v = scratch[0];
  for (int w = 1; w < kThreads / 32; ++w) v = op(v, scratch[w]);
  return v;
}

struct MaxOp {
  __device__ double operator()(double a, double b) const { return a > b || b != b ? a : b; }
};
struct SumOp {
  __device__ double operator()(double a, double b) const { return a + b; }
};
struct OrOp {
  __device__ int operator()(int a, int b) const { return a | b; }
};
struct MinIntOp {
  __device__ int operator()(int a, int b) const { return a < b ? a : b; }
};
struct MaxIntOp {
  __device__ int operator()(int a, int b) const { return a > b ? a : b; }
};

// Row statistics of the target laws and validation of the draft laws.
__global__ void __launch_bounds__(kThreads) law_stats_kernel(const Params p) {
  __shared__ double dscr[kThreads / 32];
  __shared__ int iscr[kThreads / 32];
  const int row = blockIdx.x;
  if (row < p.target_rows) {
    int bad = 0;
    double m = -INFINITY;
    for_scaled(p, row, [&](int, double s) {
      if (!isfinite(s)) bad = 1;
      m = s > m ? s : m;
    });
    bad = block_reduce(bad, iscr, OrOp());
    m = block_reduce(m, dscr, MaxOp());
    double sum = 0.0;
    for_scaled(p, row, [&](int, double s) { sum += exp(s - m); });
    sum = block_reduce(sum, dscr, SumOp());
    double sum2 = 0.0;
    for_scaled(p, row, [&](int, double s) { sum2 += exp(s - m) / sum; });
    sum2 = block_reduce(sum2, dscr, SumOp());
    if (threadIdx.x == 0) p.stats[row] = RowStats{m, sum, sum2, bad ? kBadLogits : kOk, 0};
  } else if (row < p.target_rows + p.draft_rows) {
    const int r = row - p.target_rows;
    const double* q = p.q + static_cast<long long>(r) * p.vocab;
    int bad = 0;
    double sum = 0.0;
    for (int i = threadIdx.x; i < p.vocab; i += kThreads) {
      const double v = q[i];
      if (!(v >= 0.0 && v <= 1.0)) bad = 1;            // NaN fails too
      sum += v;
    }
    bad = block_reduce(bad, iscr, OrOp());
    sum = block_reduce(sum, dscr, SumOp());
    if (threadIdx.x == 0) {
      const bool law = !bad && isfinite(sum) && fabs(sum - 1.0) <= 1e-12;
      p.stats[row] = RowStats{0.0, sum, 0.0, law ? kOk : kBadDraftLaw, 0};
    }
  }
}

// Target law value at (row, i).
__device__ __forceinline__ double law_at(const Params& p, const RowStats& st, long long row, int i) {
  return exp(load_scaled(p, row, i) - st.m) / st.s / st.s2;
}

__global__ void __launch_bounds__(kThreads) stochastic_accept_kernel(const Params p) {
  __shared__ double dscr[kThreads / 32];
  __shared__ int iscr[kThreads / 32];
  __shared__ double sh_u;
  __shared__ int sh_action, sh_row, sh_qrow;
  const int r = blockIdx.x;
  if (r >= p.num_requests) return;
  const int q0 = p.cu_n[r], n = p.cu_n[r + 1] - q0;
  const long long t0 = static_cast<long long>(q0) + r;     // target rows of request r: t0 .. t0 + n
  long long* out = p.emitted + static_cast<long long>(r) * p.u_stride;
  const double* u = p.uniforms + static_cast<long long>(r) * p.u_stride;
  int count = 0, accepted = 0, rejected = -1, extra = kExtraNone, reason = kRoundComplete, draws = 0,
      status = kOk;
  const bool layout_ok = n >= 0 && n + 1 <= p.u_stride && q0 >= 0 && q0 + n <= p.draft_rows &&
                         t0 + n < p.target_rows;
  if (threadIdx.x == 0) {
    sh_action = 0;
    if (!layout_ok) status = kBadLayout;
    for (int j = 0; j <= n && status == kOk; ++j)
      if (p.stats[t0 + j].bad) status = p.stats[t0 + j].bad;
    for (int j = 0; j < n && status == kOk; ++j) {
      const long long t = p.tokens[q0 + j];
      if (p.stats[p.target_rows + q0 + j].bad) status = kBadDraftLaw;
      else if (t < 0 || t >= p.vocab) status = kTokenRange;
      else if (!(p.q[static_cast<long long>(q0 + j) * p.vocab + t] > 0.0)) status = kZeroDraftMass;
    }
    const int budget = p.budget[r];
    auto is_eos = [&](long long t) {
      for (int e = 0; e < p.n_eos; ++e)
        if (p.eos[e] == t) return true;
      return false;
    };
    auto next_uniform = [&](double& v) {
      v = u[draws++];
      if (!(v >= 0.0 && v < 1.0)) status = kBadUniform;
      return status == kOk;
    };
    if (status == kOk) {
      if (budget <= 0) {
        reason = kBudget;
      } else {
        bool stopped = false;
        for (int j = 0; j < n; ++j) {
          const long long t = p.tokens[q0 + j];
          const double pj = law_at(p, p.stats[t0 + j], t0 + j, static_cast<int>(t));
          const double qj = p.q[static_cast<long long>(q0 + j) * p.vocab + t];
          const double alpha = fmin(pj / qj, 1.0);
          double v;
          if (!next_uniform(v)) break;
          if (v >= alpha) {
            double v2;
            if (!next_uniform(v2)) break;
            accepted = j;
            rejected = j;
            extra = kExtraResidual;
            sh_action = 1;
            sh_row = j;
            sh_qrow = q0 + j;
            sh_u = v2;
            stopped = true;
            break;
          }
          out[count++] = t;
          accepted = j + 1;
          if (is_eos(t) || count == budget) {
            reason = is_eos(t) ? kEos : kBudget;
            stopped = true;
            break;
          }
        }
        if (!stopped && status == kOk) {
          double v2;
          if (next_uniform(v2)) {
            accepted = n;
            extra = kExtraBonus;
            sh_action = 2;
            sh_row = n;
            sh_qrow = -1;
            sh_u = v2;
          }
        }
      }
    }
  }
  __syncthreads();
  const int action = sh_action;
  if (action != 0) {
    // the sampled law: relu(p - q) / mass (residual) or p (bonus); chunked CDF scan
    const long long trow = t0 + sh_row;
    const RowStats st = p.stats[trow];
    const double* q = sh_qrow >= 0 ? p.q + static_cast<long long>(sh_qrow) * p.vocab : nullptr;
    auto value = [&](int i) {
      const double pv = law_at(p, st, trow, i);
      return q ? fmax(pv - q[i], 0.0) : pv;
    };
    double mass = 1.0;
    if (q) {
      double sum = 0.0;
      for_scaled(p, trow, [&](int i, double s) { sum += fmax(exp(s - st.m) / st.s / st.s2 - q[i], 0.0); });
      mass = block_reduce(sum, dscr, SumOp());
    }
    // contiguous chunks of a multiple of 8 elements, read 8 at a time (one
    // 16-byte load of bf16 logits, independent table reads) when aligned
    const int chunk = ((p.vocab + kThreads - 1) / kThreads + 7) & ~7;
    const int lo = min(p.vocab, static_cast<int>(threadIdx.x) * chunk), hi = min(p.vocab, lo + chunk);
    double local = 0.0;
    int last_pos = -1;
    auto visit = [&](int i, double x) {
      const double pv = exp(x - st.m) / st.s / st.s2;
      const double e = q ? fmax(pv - q[i], 0.0) / mass : pv;
      local += e;
      if (e > 0.0) last_pos = i;
    };
    const unsigned short* lrow = static_cast<const unsigned short*>(p.logits) + trow * p.ld;
    int i = lo;
    if (p.dtype == 0 && (reinterpret_cast<uintptr_t>(lrow) & 15) == 0)
      for (; i + 8 <= hi; i += 8) {
        const uint4 raw = __ldg(reinterpret_cast<const uint4*>(lrow + i));
        const unsigned short* h = reinterpret_cast<const unsigned short*>(&raw);
        double x[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) x[e] = __ldg(p.scaled + h[e]);
#pragma unroll
        for (int e = 0; e < 8; ++e) visit(i + e, x[e]);
      }
    for (; i < hi; ++i) visit(i, load_scaled(p, trow, i));
    // exclusive prefix of the chunk sums (ordered by thread, i.e. by index)
    __shared__ double chunk_sum[kThreads];
    chunk_sum[threadIdx.x] = local;
    __syncthreads();
    double prefix = 0.0;
    for (int k = 0; k < static_cast<int>(threadIdx.x); ++k) prefix += chunk_sum[k];
    int found = p.vocab;
    const double uu = sh_u;
    double cdf = prefix;
    // A chunk whose end (prefix + local) lies more than 1e-12 below u cannot hold
    // the crossing: the sequential sum below differs from prefix + local by at
    // most a few hundred ulps of 1 (< 1e-13). Only the one or two chunks at the
    // crossing scan element by element (the strict CDF rule of the reference).
    if (prefix + local > uu - 1e-12)
      for (int i = lo; i < hi; ++i) {
        cdf += q ? value(i) / mass : value(i);
        if (cdf > uu) {
          found = i;
          break;
        }
      }
    found = block_reduce(found, iscr, MinIntOp());
    last_pos = block_reduce(last_pos, iscr, MaxIntOp());
    if (threadIdx.x == 0) {
      if (q && !(mass > 0.0)) {
        status = kZeroResidual;
      } else {
        const long long tok = found < p.vocab ? found : last_pos;
        out[count++] = tok;
        const int budget = p.budget[r];
        bool eos = false;
        for (int e = 0; e < p.n_eos; ++e) eos = eos || p.eos[e] == tok;
        reason = eos ? kEos : (count == budget ? kBudget : kRoundComplete);
      }
    }
  }
  if (threadIdx.x == 0) {
    if (status != kOk) count = 0;
    for (int k = count; k < p.u_stride; ++k) out[k] = -1;
    int* res = p.result + static_cast<long long>(r) * 8;
    res[0] = count;
    res[1] = accepted;
    res[2] = rejected;
    res[3] = extra;
    res[4] = reason;
    res[5] = draws;
    res[6] = status;
    res[7] = 0;
  }
}

// ---------------------------------------------------------------------------
// Draft proposal of one Markov position (DSparkDraft._sample_stochastic,
// dspark_qwen/model.py:193-208): per request the bf16 logits x = base + proj (the
// LM-head row of the position plus the Markov projection of the previous token's
// embedding, rounded to bf16 as torch adds them), the float64 law
// q = softmax(x / T) normalised once more (logits_to_probabilities,
// tensor_sampling.py:38-51) written out for the later acceptance test, and one
// token drawn by the strict CDF rule with the last positive index past the end
// (sample_categorical, tensor_sampling.py:77-84). One CTA per request row, each
// thread owning one contiguous chunk of the row: the max of x / T, the sum of
// exp(x / T - max) (the exponentials stored in the law row), the sum of the
// normalised weights, then the law itself with each chunk's sum; the chunk
// holding the crossing of u scans its values in order.
struct ProposeParams {
  const unsigned short* base;   // bf16 rows: request r's at base + row_index[r] * ld_base
  long long ld_base;
  const int* row_index;         // [rows]: the request row each launch row reads and writes
  const unsigned short* proj;   // bf16 [rows, ld_proj]: Markov projection of launch row r
  long long ld_proj;
  int vocab;
  const double* scaled;         // x / T for the 65536 bf16 bit patterns
  const double* uniforms;       // [rows]
  double* law;                  // request r's law at law + row_index[r] * ld_law
  long long ld_law;
  long long* tokens;            // [rows]
  int* status;                  // [rows]: kOk or kBadLogits (non-finite x / T)
  int rows;
};

// bf16 bits of x = bf16(float(a) + float(b)), the rounding of torch's bf16 add.
__device__ __forceinline__ unsigned short add_bf16_bits(unsigned short a, unsigned short b) {
  const float f = __bfloat162float(__ushort_as_bfloat16(a)) + __bfloat162float(__ushort_as_bfloat16(b));
  return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}

__global__ void __launch_bounds__(kThreads) propose_law_kernel(const ProposeParams p) {
  __shared__ double dscr[kThreads / 32];
  __shared__ int iscr[kThreads / 32];
  __shared__ double chunk_sum[kThreads];
  const int r = blockIdx.x;
  if (r >= p.rows) return;
  const long long row = p.row_index ? p.row_index[r] : r;
  const unsigned short* br = p.base + row * p.ld_base;
  const unsigned short* pr = p.proj + static_cast<long long>(r) * p.ld_proj;
  double* law = p.law + row * p.ld_law;
  // Every pass walks the row coalesced, 8 consecutive elements per thread per step
  // (one 16-byte load of each bf16 row, their 8 table reads in flight together); the
  // exponentials are formed again in each pass rather than stored and re-read.
  const bool vec = ((reinterpret_cast<uintptr_t>(br) | reinterpret_cast<uintptr_t>(pr)) & 15) == 0;
  auto scaled8 = [&](int i0, double (&x)[8]) {      // x / T of elements i0 .. i0 + 7 (0 past the row)
    if (vec && i0 + 8 <= p.vocab) {
      const uint4 ra = __ldg(reinterpret_cast<const uint4*>(br + i0));
      const uint4 rb = __ldg(reinterpret_cast<const uint4*>(pr + i0));
      const unsigned short* ha = reinterpret_cast<const unsigned short*>(&ra);
      const unsigned short* hb = reinterpret_cast<const unsigned short*>(&rb);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = __ldg(p.scaled + add_bf16_bits(ha[e], hb[e]));
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = i0 + e < p.vocab ? p.scaled[add_bf16_bits(br[i0 + e], pr[i0 + e])] : 0.0;
    }
  };
  constexpr int kTile = kThreads * 8;
  int bad = 0;
  double m = -INFINITY;
  for (int i0 = threadIdx.x * 8; i0 < p.vocab; i0 += kTile) {
    double x[8];
    scaled8(i0, x);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (i0 + e < p.vocab) {
        if (!isfinite(x[e])) bad = 1;
        m = x[e] > m ? x[e] : m;
      }
  }
  bad = block_reduce(bad, iscr, OrOp());
  m = block_reduce(m, dscr, MaxOp());
  double sum = 0.0;
  for (int i0 = threadIdx.x * 8; i0 < p.vocab; i0 += kTile) {
    double x[8];
    scaled8(i0, x);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (i0 + e < p.vocab) sum += exp(x[e] - m);
  }
  sum = block_reduce(sum, dscr, SumOp());
  double sum2 = 0.0;
  for (int i0 = threadIdx.x * 8; i0 < p.vocab; i0 += kTile) {
    double x[8];
    scaled8(i0, x);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (i0 + e < p.vocab) sum2 += exp(x[e] - m) / sum;
  }
  sum2 = block_reduce(sum2, dscr, SumOp());
  // The law, tile by tile in index order: each thread's 8 values, a block-wide scan
  // of their sums (thread order = index order inside a tile) and the CDF carried
  // across tiles; the first element whose CDF exceeds u is the draw.
  const double u = p.uniforms[r];
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool law16 = (reinterpret_cast<uintptr_t>(law) & 15) == 0;   // 16-byte stores only when aligned
  double carry = 0.0;
  int found = p.vocab, last_pos = -1;
  for (int t0 = 0; t0 < p.vocab; t0 += kTile) {
    const int i0 = t0 + threadIdx.x * 8;
    double v[8], seg = 0.0;
    if (i0 < p.vocab) {
      double x[8];
      scaled8(i0, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[e] = i0 + e < p.vocab ? exp(x[e] - m) / sum / sum2 : 0.0;
        seg += v[e];
        if (v[e] > 0.0) last_pos = i0 + e;
      }
      if (law16 && i0 + 8 <= p.vocab) {
#pragma unroll
        for (int e = 0; e < 8; e += 2) *reinterpret_cast<double2*>(law + i0 + e) = make_double2(v[e], v[e + 1]);
      } else {
        for (int e = 0; i0 + e < p.vocab; ++e) law[i0 + e] = v[e];
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.0;
    }
    // inclusive scan of seg over the CTA's threads
    double incl = seg;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) chunk_sum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      double w = lane < kThreads / 32 ? chunk_sum[lane] : 0.0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double n = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += n;
      }
      chunk_sum[32 + lane] = w;                       // inclusive warp prefixes
    }
    __syncthreads();
    const double excl = (warp > 0 ? chunk_sum[32 + warp - 1] : 0.0) + incl - seg;
    double cdf = carry + excl;
    if (found == p.vocab && cdf + seg > u - 1e-12) {
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        cdf += v[e];
        if (cdf > u && i0 + e < p.vocab) {
          found = i0 + e;
          break;
        }
      }
    }
    carry += chunk_sum[32 + kThreads / 32 - 1];
    __syncthreads();                                  // chunk_sum is rewritten by the next tile
  }
  found = block_reduce(found, iscr, MinIntOp());
  last_pos = block_reduce(last_pos, iscr, MaxIntOp());
  if (threadIdx.x == 0) {
    // a row without positive mass (non-finite logits) gets token 0 and a bad status,
    // so that no out-of-range index reaches the next position's embedding gather
    p.tokens[r] = found < p.vocab ? found : (last_pos >= 0 ? last_pos : 0);
    p.status[r] = bad || last_pos < 0 ? kBadLogits : kOk;
  }
}


// The same proposal with each request row split between a cluster of two CTAs, so
// that a launch of few rows (64 requests) fills twice the SMs. Rank 0 takes the
// row's first ceil(tiles / 2) tiles of kThreads * 8 values, rank 1 the rest; after
// each pass the two partial results (max and bad flag, sum, sum of normalised
// weights) cross through shared memory and both CTAs combine them in rank order,
// so both hold the same statistics. The law pass records each tile's total; rank 1
// starts its CDF from rank 0's total, which is the running CDF the one-CTA kernel
// carries at that tile, and each CTA scans again only the tile holding the crossing
// of u (values formed as in the law pass, the same scan), so the draw follows the
// same CDF association as the one-CTA kernel.
constexpr int kPairMaxTiles = 64;     // tiles per CTA (vocabularies up to 128 tiles)

__device__ __forceinline__ double ld_cluster_f64(const double* local, uint32_t rank) {
  double v;
  asm volatile("ld.shared::cluster.f64 %0, [%1];" : "=d"(v) : "r"(pair::cluster_addr(smem_u32(local), rank))
               : "memory");
  return v;
}

__device__ __forceinline__ int ld_cluster_s32(const int* local, uint32_t rank) {
  int v;
  asm volatile("ld.shared::cluster.s32 %0, [%1];" : "=r"(v) : "r"(pair::cluster_addr(smem_u32(local), rank))
               : "memory");
  return v;
}

__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(kThreads) propose_law_pair_kernel(const ProposeParams p) {
  __shared__ double dscr[kThreads / 32];
  __shared__ int iscr[kThreads / 32];
  __shared__ double chunk_sum[kThreads];
  __shared__ double tile_total[kPairMaxTiles];
  __shared__ double xd[4];    // crossing the cluster: max, sum, sum of normalised weights, CDF total
  __shared__ int xi[3];       // crossing the cluster: bad flag, last positive index, draw
  const uint32_t rank = pair::cluster_rank();
  const int r = static_cast<int>(blockIdx.x >> 1);   // the grid is exactly two CTAs per row
  const long long row = p.row_index ? p.row_index[r] : r;
  const unsigned short* br = p.base + row * p.ld_base;
  const unsigned short* pr = p.proj + static_cast<long long>(r) * p.ld_proj;
  double* law = p.law + row * p.ld_law;
  constexpr int kTile = kThreads * 8;
  const int ntiles = (p.vocab + kTile - 1) / kTile;
  const int split = min(p.vocab, ((ntiles + 1) / 2) * kTile);
  const int lo = rank == 0 ? 0 : split, hi = rank == 0 ? split : p.vocab;
  const bool vec = ((reinterpret_cast<uintptr_t>(br) | reinterpret_cast<uintptr_t>(pr)) & 15) == 0;
  auto scaled8 = [&](int i0, double (&x)[8]) {      // x / T of elements i0 .. i0 + 7 (0 past the row)
    if (vec && i0 + 8 <= p.vocab) {
      const uint4 ra = __ldg(reinterpret_cast<const uint4*>(br + i0));
      const uint4 rb = __ldg(reinterpret_cast<const uint4*>(pr + i0));
      const unsigned short* ha = reinterpret_cast<const unsigned short*>(&ra);
      const unsigned short* hb = reinterpret_cast<const unsigned short*>(&rb);
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = __ldg(p.scaled + add_bf16_bits(ha[e], hb[e]));
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) x[e] = i0 + e < p.vocab ? p.scaled[add_bf16_bits(br[i0 + e], pr[i0 + e])] : 0.0;
    }
  };
  // pass 1: max of x / T and non-finite values
  int bad = 0;
  double m = -INFINITY;
  for (int i0 = lo + threadIdx.x * 8; i0 < hi; i0 += kTile) {
    double x[8];
    scaled8(i0, x);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (i0 + e < p.vocab) {
        if (!isfinite(x[e])) bad = 1;
        m = x[e] > m ? x[e] : m;
      }
  }
  bad = block_reduce(bad, iscr, OrOp());
  m = block_reduce(m, dscr, MaxOp());
  if (threadIdx.x == 0) {
    xd[0] = m;
    xi[0] = bad;
  }
  pair::cluster_sync();
  m = MaxOp()(ld_cluster_f64(&xd[0], 0), ld_cluster_f64(&xd[0], 1));
  bad = ld_cluster_s32(&xi[0], 0) | ld_cluster_s32(&xi[0], 1);
  // pass 2: sum of exp(x / T - max)
  double sum = 0.0;
  for (int i0 = lo + threadIdx.x * 8; i0 < hi; i0 += kTile) {
    double x[8];
    scaled8(i0, x);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (i0 + e < p.vocab) sum += exp(x[e] - m);
  }
  sum = block_reduce(sum, dscr, SumOp());
  if (threadIdx.x == 0) xd[1] = sum;
  pair::cluster_sync();
  sum = ld_cluster_f64(&xd[1], 0) + ld_cluster_f64(&xd[1], 1);
  // pass 3: sum of the normalised weights
  double sum2 = 0.0;
  for (int i0 = lo + threadIdx.x * 8; i0 < hi; i0 += kTile) {
    double x[8];
    scaled8(i0, x);
#pragma unroll
    for (int e = 0; e < 8; ++e)
      if (i0 + e < p.vocab) sum2 += exp(x[e] - m) / sum;
  }
  sum2 = block_reduce(sum2, dscr, SumOp());
  if (threadIdx.x == 0) xd[2] = sum2;
  pair::cluster_sync();
  sum2 = ld_cluster_f64(&xd[2], 0) + ld_cluster_f64(&xd[2], 1);
  // One tile's values (written to the law when `store`), this thread's 8-value sum and
  // the CTA-wide exclusive prefix of those sums; returns the tile's total.
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const bool law16 = (reinterpret_cast<uintptr_t>(law) & 15) == 0;
  int last_pos = -1;
  auto tile = [&](int t0, bool store, double (&v)[8], double& seg, double& excl) {
    const int i0 = t0 + threadIdx.x * 8;
    seg = 0.0;
    if (i0 < hi) {
      double x[8];
      scaled8(i0, x);
#pragma unroll
      for (int e = 0; e < 8; ++e) {
        v[e] = i0 + e < p.vocab ? exp(x[e] - m) / sum / sum2 : 0.0;
        seg += v[e];
        if (v[e] > 0.0) last_pos = i0 + e;
      }
      if (store) {
        if (law16 && i0 + 8 <= p.vocab) {
#pragma unroll
          for (int e = 0; e < 8; e += 2) *reinterpret_cast<double2*>(law + i0 + e) = make_double2(v[e], v[e + 1]);
        } else {
          for (int e = 0; i0 + e < p.vocab; ++e) law[i0 + e] = v[e];
        }
      }
    } else {
#pragma unroll
      for (int e = 0; e < 8; ++e) v[e] = 0.0;
    }
    double incl = seg;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const double n = __shfl_up_sync(0xffffffffu, incl, o);
      if (lane >= o) incl += n;
    }
    if (lane == 31) chunk_sum[warp] = incl;
    __syncthreads();
    if (warp == 0) {
      double w = lane < kThreads / 32 ? chunk_sum[lane] : 0.0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const double n = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += n;
      }
      chunk_sum[32 + lane] = w;                       // inclusive warp prefixes
    }
    __syncthreads();
    excl = (warp > 0 ? chunk_sum[32 + warp - 1] : 0.0) + incl - seg;
    const double total = chunk_sum[32 + kThreads / 32 - 1];
    __syncthreads();                                  // chunk_sum is rewritten by the next tile
    return total;
  };
  // pass 4: the law of this CTA's tiles, each tile's total recorded
  int my_tiles = 0;
  double carry = 0.0;
  for (int t0 = lo; t0 < hi; t0 += kTile, ++my_tiles) {
    double v[8], seg, excl;
    const double total = tile(t0, true, v, seg, excl);
    if (threadIdx.x == 0) tile_total[my_tiles] = total;
    carry += total;
  }
  last_pos = block_reduce(last_pos, iscr, MaxIntOp());
  if (threadIdx.x == 0) {
    xd[3] = carry;
    xi[1] = last_pos;
  }
  pair::cluster_sync();
  // (kept apart from last_pos, which the rescans below update per thread)
  const int last_all = max(ld_cluster_s32(&xi[1], 0), ld_cluster_s32(&xi[1], 1));
  // the draw: the first element whose CDF exceeds u, searched in the tiles whose
  // running total can reach it (the CDF of rank 1 starts at rank 0's total)
  const double u = p.uniforms[r];
  int found = p.vocab;
  carry = rank == 0 ? 0.0 : ld_cluster_f64(&xd[3], 0);
  for (int k = 0; k < my_tiles; ++k) {
    if (carry + tile_total[k] > u - 1e-12) {
      double v[8], seg, excl;
      tile(lo + k * kTile, false, v, seg, excl);
      const int i0 = lo + k * kTile + threadIdx.x * 8;
      int f = p.vocab;
      double cdf = carry + excl;
      if (cdf + seg > u - 1e-12) {
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          cdf += v[e];
          if (cdf > u && i0 + e < p.vocab) {
            f = i0 + e;
            break;
          }
        }
      }
      f = block_reduce(f, iscr, MinIntOp());
      if (f < p.vocab) {
        found = f;
        break;
      }
    }
    carry += tile_total[k];
  }
  if (threadIdx.x == 0) xi[2] = found;
  pair::cluster_sync();
  if (rank == 0 && threadIdx.x == 0) {
    found = min(ld_cluster_s32(&xi[2], 0), ld_cluster_s32(&xi[2], 1));
    p.tokens[r] = found < p.vocab ? found : (last_all >= 0 ? last_all : 0);
    p.status[r] = bad || last_all < 0 ? kBadLogits : kOk;
  }
  pair::cluster_sync();                               // rank 1's shared memory is read until here
}

}  // namespace sampling
}  // namespace dspark
