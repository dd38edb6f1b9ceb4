// C-ABI of the DSpark B200 attention library (declared in include/dspark_b200.h).
// Host side: argument checks that need no device reads, TMA descriptor
// encoding and kernel launches on the caller's stream. No allocation happens
// here: scratch for split items is the caller's workspace.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>
#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdint>
#include <cstdio>
#include <mutex>
#include <numeric>
#include <queue>
#include <utility>
#include <vector>

#include "accept.cuh"
#include "append.cuh"
#include "attention.cuh"
#include "markov.cuh"
#include "norm.cuh"
#include "sampling.cuh"
#include "train.cuh"
#include "verify.cuh"
#include "../../include/dspark_b200.h"

using namespace dspark;

namespace {

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  bool ready = false;
  int sms = 0;
  int append_pairs = 0;   // CTA pairs of the 2-SM append kernel resident at once (0: not used)
  int max_smem_optin = 0;
  int cc_major = 0, cc_minor = 0;
};

std::mutex g_mu;
DeviceInfo g_dev[kMaxDevices];
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
// Verify launches with fewer new rows take the prep-kernel path (measured on
// B200: 28-layer decode steps of 8 and 32 requests 30-40% faster; at 128
// requests x 7 rows over 0.5 M resident rows the fused kernel is ~1.5% faster,
// its in-register q prologue being amortised over long CTA ranges).
constexpr int kVerifyPrepMaxRows = 512;
// Chunks longer than this (prefill) also take the prep path: the fused kernel
// normalises and rotates a new-row tile in every item that reads it, which for a
// 2048-row prompt is 256 q-blocks redoing the same tiles.
constexpr int kVerifyFusedMaxQ = 16;
// Kernels launched by this library since load (all devices, all streams).
std::atomic<unsigned long long> g_launches{0};

constexpr size_t kAttnSmemBytes = 1024 + static_cast<size_t>(kSmemBarOff) + 2 * kStages * sizeof(uint64_t) +
                                  sizeof(SchedShared);

int device_info(int dev, DeviceInfo* out) {
  if (dev < 0 || dev >= kMaxDevices) return DSPARK_ERR_INVALID_ARGUMENT;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    if (cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.max_smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&d.cc_minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess)
      return DSPARK_ERR_CUDA;
    if (d.cc_major != 10) return DSPARK_ERR_UNSUPPORTED;   // built for sm_100a only
    if (static_cast<size_t>(d.max_smem_optin) < kAttnSmemBytes ||
        static_cast<size_t>(d.max_smem_optin) < train::kSmemBytes)
      return DSPARK_ERR_UNSUPPORTED;
    int cur = -1;
    cudaGetDevice(&cur);
    if (cur != dev) return DSPARK_ERR_INVALID_ARGUMENT;     // attributes are per current device
    if (cudaFuncSetAttribute(attn_bf16_kernel<false, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kAttnSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(attn_bf16_kernel<true, false>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kAttnSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(attn_bf16_kernel<true, true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(kAttnSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(train::train_attn_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(train::kSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(markov::markov_step_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(markov::kSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(markov::markov_block_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(markov::kSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(append::draft_append_kernel<1>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(append::Cfg<1>::kSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(append::draft_append_kernel<2>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(append::Cfg<2>::kSmemBytes)) != cudaSuccess ||
        cudaFuncSetAttribute(append::draft_append_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                             static_cast<int>(append::PairCfg::kSmemBytes)) != cudaSuccess)
      return DSPARK_ERR_CUDA;
    {
      // CTA pairs of the 2-SM append the GPU holds at once (a pair needs two SMs of
      // one GPC); a refused query leaves the single-CTA kernels in use.
      cudaLaunchConfig_t cfg = {};
      cfg.gridDim = dim3(static_cast<unsigned>(d.sms & ~1));
      cfg.blockDim = dim3(append::kThreads);
      cfg.dynamicSmemBytes = append::PairCfg::kSmemBytes;
      int clusters = 0;
      if (cudaOccupancyMaxActiveClusters(&clusters, append::draft_append_pair_kernel, &cfg) != cudaSuccess) {
        cudaGetLastError();
        clusters = 0;
      }
      d.append_pairs = clusters < d.sms / 2 ? clusters : d.sms / 2;
    }
    if (!g_encode) {
      cudaDriverEntryPointQueryResult q;
      void* fn = nullptr;
      if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
          q != cudaDriverEntryPointSuccess || fn == nullptr)
        return DSPARK_ERR_CUDA;
      g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    }
    d.ready = true;
  }
  *out = d;
  return DSPARK_OK;
}

int current_device_info(DeviceInfo* out) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return DSPARK_ERR_CUDA;
  return device_info(dev, out);
}

// Workspace: fp32 partials of up to two cut items per CTA, one merge entry per
// (CTA, KV head) and each CTA's tile range. Every launch rewrites what it reads.
constexpr size_t workspace_for_grid(int grid) {
  return static_cast<size_t>(grid) * (2 * (kPartFloatsPerSlot + kPartMlPerSlot) * sizeof(float) +
                                      kKVHeads * sizeof(MergeEntry) + 2 * sizeof(long long));
}

void bind_workspace(AttnParams& p, void* workspace, int grid) {
  uint8_t* ws = static_cast<uint8_t*>(workspace);
  p.part_o = reinterpret_cast<float*>(ws);
  p.part_ml = reinterpret_cast<float*>(ws + static_cast<size_t>(grid) * 2 * kPartFloatsPerSlot * sizeof(float));
  p.merges = reinterpret_cast<MergeEntry*>(
      ws + static_cast<size_t>(grid) * 2 * (kPartFloatsPerSlot + kPartMlPerSlot) * sizeof(float));
  p.ranges = reinterpret_cast<long long*>(p.merges + static_cast<size_t>(grid) * kKVHeads);
  p.grid = grid;
}


bool aligned(const void* p, size_t a) { return (reinterpret_cast<uintptr_t>(p) % a) == 0; }

// K/V rows tensor [rows, 8, 128] bf16 viewed as dims (d, row, head) so one box
// (64 d, 16 rows, 8 heads) lands in shared memory as [head][row][64 d] with
// the 128-byte swizzle keyed on the row, conflict-free for ldmatrix.
int encode_kv_map(CUtensorMap* m, const void* base, long long rows) {
  if (!aligned(base, 16) || rows < 1 || rows >= (1ll << 31)) return DSPARK_ERR_INVALID_ARGUMENT;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(rows),
                        static_cast<cuuint64_t>(kKVHeads)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kKVHeads * kHeadDim * 2), static_cast<cuuint64_t>(kHeadDim * 2)};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(kTileN), static_cast<cuuint32_t>(kKVHeads)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSPARK_OK : DSPARK_ERR_CUDA;
}

int launch_status() {
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return DSPARK_ERR_CUDA;
  g_launches.fetch_add(1, std::memory_order_relaxed);
  return DSPARK_OK;
}

// The cut-item merge after an attention launch on the same stream, as a
// programmatic dependent launch (its CTAs wait in griddepcontrol.wait for the
// attention kernel's completion and memory); a plain launch where the
// attribute is refused.
int launch_merge(const AttnParams& p, cudaStream_t stream) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(p.grid * kKVHeads));
  cfg.blockDim = dim3(kMergeThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, split_merge_kernel, p) != cudaSuccess) {
    cudaGetLastError();
    cfg.numAttrs = 0;
    if (cudaLaunchKernelEx(&cfg, split_merge_kernel, p) != cudaSuccess) return DSPARK_ERR_CUDA;
  }
  return launch_status();
}

struct KeySources {
  const void* ka;
  const void* va;
  long long rows_a;
  const void* kb;
  const void* vb;
  long long rows_b;
};

// Shared launch path of every attention entry point; `fused` selects the
// verify kernel that normalises/rotates q and produces the source-B rows.
int run_attention(AttnParams p, const KeySources& src, int dtype, int max_q, void* workspace,
                  size_t workspace_bytes, cudaStream_t stream, bool fused = false, bool dependent = false) {
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != DSPARK_OK) return st;
  if (dtype == DSPARK_DTYPE_F32) {
    if (max_q < 1) return DSPARK_ERR_INVALID_ARGUMENT;
    p.rows_a = src.rows_a;
    p.rows_b = src.rows_b;
    dim3 grid(p.num_requests, (max_q + kQBlock - 1) / kQBlock, kKVHeads);
    if (grid.y > 65535) return DSPARK_ERR_UNSUPPORTED;
    attn_f32_kernel<<<grid, kF32Threads, 0, stream>>>(static_cast<const float*>(src.ka),
                                                      static_cast<const float*>(src.va),
                                                      static_cast<const float*>(src.kb),
                                                      static_cast<const float*>(src.vb), p);
    return launch_status();
  }
  if (dtype != DSPARK_DTYPE_BF16) return DSPARK_ERR_INVALID_ARGUMENT;
  const int grid = dev.sms;
  if (workspace == nullptr || workspace_bytes < workspace_for_grid(grid) || !aligned(workspace, 16))
    return DSPARK_ERR_INVALID_ARGUMENT;
  bind_workspace(p, workspace, grid);
  p.rows_a = src.rows_a;
  p.rows_b = src.rows_b;
  CUtensorMap ka, va, kb, vb;
  if ((st = encode_kv_map(&ka, src.ka, src.rows_a)) != DSPARK_OK) return st;
  if ((st = encode_kv_map(&va, src.va, src.rows_a)) != DSPARK_OK) return st;
  if (src.kb != nullptr) {
    if ((st = encode_kv_map(&kb, src.kb, src.rows_b)) != DSPARK_OK) return st;
    if ((st = encode_kv_map(&vb, src.vb, src.rows_b)) != DSPARK_OK) return st;
  } else {
    kb = ka;
    vb = va;
  }
  if (dependent && p.causal && !fused) {
    // programmatic dependent launch after the verify prep kernel: the schedule
    // and the first loads of resident rows overlap the prep's tail
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(grid));
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = kAttnSmemBytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if (cudaLaunchKernelEx(&cfg, attn_bf16_kernel<true, false>, ka, va, kb, vb, p) != cudaSuccess) {
      cudaGetLastError();
      cfg.numAttrs = 0;
      if (cudaLaunchKernelEx(&cfg, attn_bf16_kernel<true, false>, ka, va, kb, vb, p) != cudaSuccess)
        return DSPARK_ERR_CUDA;
    }
  } else if (fused)
    attn_bf16_kernel<true, true><<<grid, kAttnThreads, kAttnSmemBytes, stream>>>(ka, va, kb, vb, p);
  else if (p.causal)
    attn_bf16_kernel<true, false><<<grid, kAttnThreads, kAttnSmemBytes, stream>>>(ka, va, kb, vb, p);
  else
    attn_bf16_kernel<false, false><<<grid, kAttnThreads, kAttnSmemBytes, stream>>>(ka, va, kb, vb, p);
  if ((st = launch_status()) != DSPARK_OK) return st;
  return launch_merge(p, stream);
}

bool common_ok(const void* q, const void* out, const int32_t* cu_q, int num_requests, int total_q, float scale,
               int dtype) {
  const size_t align = dtype == DSPARK_DTYPE_F32 ? 4 : 16;
  return q && out && cu_q && num_requests >= 1 && total_q >= 1 && scale > 0.f && aligned(q, align) &&
         aligned(out, align) && aligned(cu_q, 4);
}

AttnParams base_params(const void* q, void* out, const int32_t* cu_q, int num_requests, int total_q, float scale,
                       int causal) {
  AttnParams p{};
  p.q = q;
  p.out = out;
  p.cu_q = cu_q;
  p.num_requests = num_requests;
  p.total_q = total_q;
  p.causal = causal;
  p.scale = scale;
  p.scale_log2 = scale * 1.4426950408889634f;
  return p;
}

int varlen_common(const void* q, const void* k, const void* v, const int32_t* cu_q, const int32_t* cu_k,
                  int num_requests, int total_q, long long key_rows, int max_q, float scale, int dtype, int causal,
                  void* out, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!common_ok(q, out, cu_q, num_requests, total_q, scale, dtype) || !k || !v || !cu_k || key_rows < 1)
    return DSPARK_ERR_INVALID_ARGUMENT;
  AttnParams p = base_params(q, out, cu_q, num_requests, total_q, scale, causal);
  p.mode = kModeVarlen;
  p.cu_k = cu_k;
  KeySources src{k, v, key_rows, nullptr, nullptr, 0};
  return run_attention(p, src, dtype, max_q, workspace, workspace_bytes, stream);
}

// Packed q or K/V [rows, heads, 128] bf16 as dims (d, head, row): one box of
// (64 d, box_heads, box_rows) lands in shared memory as [row][head][64 d] rows of
// 128 bytes in the 128-byte swizzle, the K-major operand layout of tcgen05.mma.
int encode_rows_map(CUtensorMap* m, const void* base, long long rows, int heads, int box_heads, int box_rows) {
  if (!aligned(base, 16) || rows < 1 || rows >= (1ll << 31)) return DSPARK_ERR_INVALID_ARGUMENT;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(kHeadDim), static_cast<cuuint64_t>(heads),
                        static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(kHeadDim * 2), static_cast<cuuint64_t>(heads * kHeadDim * 2)};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_heads), static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[3] = {1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 3, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? DSPARK_OK : DSPARK_ERR_CUDA;
}

}  // namespace

extern "C" {

int dspark_abi_version(void) { return DSPARK_ABI_VERSION; }

unsigned long long dspark_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

const char* dspark_status_string(int status) {
  switch (status) {
    case DSPARK_OK: return "ok";
    case DSPARK_ERR_INVALID_ARGUMENT: return "invalid argument";
    case DSPARK_ERR_UNSUPPORTED: return "unsupported device or shape";
    case DSPARK_ERR_CUDA: return "CUDA runtime error";
    default: return "unknown status";
  }
}

int dspark_attention_workspace_size(int device, size_t* bytes) {
  if (bytes == nullptr) return DSPARK_ERR_INVALID_ARGUMENT;
  int sms = 0;
  if (cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, device) != cudaSuccess) return DSPARK_ERR_CUDA;
  *bytes = workspace_for_grid(sms);
  return DSPARK_OK;
}

int dspark_read_device_status(unsigned int* status, int clear) {
  if (status == nullptr) return DSPARK_ERR_INVALID_ARGUMENT;
  if (cudaMemcpyFromSymbol(status, g_device_status, sizeof(unsigned int)) != cudaSuccess) return DSPARK_ERR_CUDA;
  if (clear) {
    const unsigned int zero = 0;
    if (cudaMemcpyToSymbol(g_device_status, &zero, sizeof(unsigned int)) != cudaSuccess) return DSPARK_ERR_CUDA;
  }
  return DSPARK_OK;
}

int dspark_copy_device_status(unsigned int* dst, cudaStream_t stream) {
  if (dst == nullptr) return DSPARK_ERR_INVALID_ARGUMENT;
  void* src = nullptr;
  if (cudaGetSymbolAddress(&src, g_device_status) != cudaSuccess || src == nullptr) return DSPARK_ERR_CUDA;
  return cudaMemcpyAsync(dst, src, sizeof(unsigned int), cudaMemcpyDefault, stream) == cudaSuccess ? DSPARK_OK
                                                                                                  : DSPARK_ERR_CUDA;
}

int dspark_draft_attn(const void* q, const void* k, const void* v, const int32_t* cu_q, const int32_t* cu_k,
                      int num_requests, int total_q, long long key_rows, int max_q, int max_k, float scale,
                      int dtype, void* out, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  (void)max_k;
  return varlen_common(q, k, v, cu_q, cu_k, num_requests, total_q, key_rows, max_q, scale, dtype, 0, out, workspace,
                       workspace_bytes, stream);
}

int dspark_varlen_attn(const void* q, const void* k, const void* v, const int32_t* cu_q, const int32_t* cu_k,
                       int num_requests, int total_q, long long key_rows, int max_q, int max_k, float scale,
                       int dtype, void* out, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  (void)max_k;
  return varlen_common(q, k, v, cu_q, cu_k, num_requests, total_q, key_rows, max_q, scale, dtype, 1, out, workspace,
                       workspace_bytes, stream);
}

int dspark_segment_attn(const void* q, const void* ka, const void* va, long long rows_a, const void* kb,
                        const void* vb, long long rows_b, const int32_t* cu_q, const int32_t* a_start,
                        const int32_t* a_len, const int32_t* b_start, const int32_t* b_len, int a_off, int b_off,
                        int num_requests, int total_q, int max_q, int causal, float scale, int dtype, void* out,
                        void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (!common_ok(q, out, cu_q, num_requests, total_q, scale, dtype) || !ka || !va || !a_start || !a_len ||
      rows_a < 1 || (causal != 0 && causal != 1))
    return DSPARK_ERR_INVALID_ARGUMENT;
  const bool has_b = kb != nullptr;
  if (has_b && (!vb || rows_b < 1)) return DSPARK_ERR_INVALID_ARGUMENT;
  if (!has_b && (b_start || b_len)) return DSPARK_ERR_INVALID_ARGUMENT;
  AttnParams p = base_params(q, out, cu_q, num_requests, total_q, scale, causal);
  p.mode = kModeSegmented;
  p.a_start = a_start;
  p.a_len = a_len;
  p.b_start = b_start;
  p.b_len = b_len;
  p.a_off = a_off;
  p.b_off = b_off;
  p.b_none = has_b ? 0 : 1;
  KeySources src{ka, va, rows_a, kb, vb, has_b ? rows_b : 0};
  return run_attention(p, src, dtype, max_q, workspace, workspace_bytes, stream);
}

int dspark_rope_table(const void* rope_cache, int cache_rows, const int32_t* cu_q, const int32_t* ctx_len,
                      int num_requests, int total_q, void* table, cudaStream_t stream) {
  if (!rope_cache || cache_rows < 1 || !cu_q || !ctx_len || !table || num_requests < 1 || total_q < 1 ||
      !aligned(table, 16) || !aligned(rope_cache, 16))
    return DSPARK_ERR_INVALID_ARGUMENT;
  rope_table_kernel<<<(total_q + 15) / 16, 256, 0, stream>>>(static_cast<const uint4*>(rope_cache), cache_rows,
                                                            cu_q, ctx_len, num_requests, total_q,
                                                            static_cast<uint4*>(table));
  return launch_status();
}

namespace {

// Body of dspark_verify_fused / dspark_verify_strided. Row strides other than the
// packed ones are read by the prep kernel only: the fused kernel's new-row
// sources are packed, so strided projections always take the prep path.
int verify_impl(const void* q_raw, long long ld_q, const void* k_raw, long long ld_k, const void* v_raw,
                long long ld_v, const void* q_norm_weight, const void* k_norm_weight, const void* rope_table,
                float eps, const int32_t* cu_q, const int32_t* slot_row, const int32_t* ctx_len, int num_requests,
                int total_q, int max_q, void* resident_k, void* resident_v, long long rows_per_layer,
                void* scratch_k, void* scratch_v, int scratch_rows, int num_layers, int layer, float scale,
                int path, void* out, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  if (path != DSPARK_VERIFY_AUTO && path != DSPARK_VERIFY_FUSED && path != DSPARK_VERIFY_PREP)
    return DSPARK_ERR_INVALID_ARGUMENT;
  const long long q_row = static_cast<long long>(kQHeads) * kHeadDim, kv_row = static_cast<long long>(kKVHeads) * kHeadDim;
  if (ld_q < q_row || ld_k < kv_row || ld_v < kv_row || ld_q % 8 != 0 || ld_k % 8 != 0 || ld_v % 8 != 0)
    return DSPARK_ERR_INVALID_ARGUMENT;
  const bool packed = ld_q == q_row && ld_k == kv_row && ld_v == kv_row;
  if (!packed && path == DSPARK_VERIFY_FUSED) return DSPARK_ERR_INVALID_ARGUMENT;
  if (!common_ok(q_raw, out, cu_q, num_requests, total_q, scale, DSPARK_DTYPE_BF16) || !k_raw || !v_raw ||
      !q_norm_weight || !k_norm_weight || !rope_table || !aligned(rope_table, 16) || !slot_row || !ctx_len ||
      !resident_k || !resident_v ||
      !scratch_k || !scratch_v || !aligned(k_raw, 16) || !aligned(v_raw, 16) || !aligned(scratch_k, 16) ||
      !aligned(scratch_v, 16) || rows_per_layer < 1 || scratch_rows < total_q || num_layers < 1 || layer < 0 ||
      layer >= num_layers || !(eps > 0.f))
    return DSPARK_ERR_INVALID_ARGUMENT;
  const size_t row_bytes = static_cast<size_t>(kKVHeads) * kHeadDim * 2;
  const long long res_row0 = static_cast<long long>(layer) * rows_per_layer;
  if (res_row0 + rows_per_layer >= (1ll << 31)) return DSPARK_ERR_UNSUPPORTED;
  uint8_t* sk = static_cast<uint8_t*>(scratch_k) + static_cast<size_t>(layer) * scratch_rows * row_bytes;
  uint8_t* sv = static_cast<uint8_t*>(scratch_v) + static_cast<size_t>(layer) * scratch_rows * row_bytes;
  // One launch: q_norm/k_norm + RoPE + KV append of the new rows into this
  // layer's scratch, and bottom-right attention over the resident prefix rows
  // followed by the new rows.
  AttnParams p = base_params(q_raw, out, cu_q, num_requests, total_q, scale, 1);
  p.mode = kModeSegmented;
  p.a_start = slot_row;
  p.a_len = ctx_len;
  p.b_start = nullptr;     // new rows follow cu_q
  p.b_len = nullptr;       // and number q_i per request
  p.a_off = 0;
  p.b_off = 0;
  p.b_none = 0;
  p.k_new = static_cast<const __nv_bfloat16*>(k_raw);
  p.v_new = static_cast<const __nv_bfloat16*>(v_raw);
  p.q_w = static_cast<const __nv_bfloat16*>(q_norm_weight);
  p.k_w = static_cast<const __nv_bfloat16*>(k_norm_weight);
  p.rope = static_cast<const uint32_t*>(rope_table);
  p.eps = eps;
  p.scratch_k = reinterpret_cast<__nv_bfloat16*>(sk);
  p.scratch_v = reinterpret_cast<__nv_bfloat16*>(sv);
  p.scratch_rows = scratch_rows;
  const uint8_t* rk = static_cast<const uint8_t*>(resident_k) + res_row0 * row_bytes;
  const uint8_t* rv = static_cast<const uint8_t*>(resident_v) + res_row0 * row_bytes;
  const bool prep = path == DSPARK_VERIFY_PREP || !packed ||
                    (path == DSPARK_VERIFY_AUTO && (total_q < kVerifyPrepMaxRows || max_q > kVerifyFusedMaxQ));
  if (prep) {
    // q_norm/k_norm + RoPE + KV append once per new row, then the plain causal
    // kernel over [resident prefix ; scratch rows] with q read from `out` in
    // place (an item's q rows are read only by its own contributors, and its
    // output rows are written by its single CTA or by the merge kernel after
    // every contributor has finished).
    VerifyPrepParams vp{static_cast<const __nv_bfloat16*>(q_raw), static_cast<const __nv_bfloat16*>(k_raw),
                        static_cast<const __nv_bfloat16*>(v_raw), static_cast<const __nv_bfloat16*>(q_norm_weight),
                        static_cast<const __nv_bfloat16*>(k_norm_weight), static_cast<const uint32_t*>(rope_table),
                        static_cast<__nv_bfloat16*>(out), reinterpret_cast<__nv_bfloat16*>(sk),
                        reinterpret_cast<__nv_bfloat16*>(sv), total_q, eps, ld_q, ld_k, ld_v};
    const long long warps = static_cast<long long>(total_q) * 32;
    verify_prep_kernel<<<static_cast<unsigned>((warps + 7) / 8), 256, 0, stream>>>(vp);
    int st = launch_status();
    if (st != DSPARK_OK) return st;
    p.q = out;
    KeySources src{rk, rv, rows_per_layer, sk, sv, scratch_rows};
    return run_attention(p, src, DSPARK_DTYPE_BF16, max_q, workspace, workspace_bytes, stream, false, true);
  }
  // Source B = the raw new-row projections; the kernel normalises/rotates them
  // in shared memory and writes the scratch rows itself.
  KeySources src{rk, rv, rows_per_layer, k_raw, v_raw, total_q};
  return run_attention(p, src, DSPARK_DTYPE_BF16, max_q, workspace, workspace_bytes, stream, true);
}

}  // namespace

int dspark_verify_fused(const void* q_raw, const void* k_raw, const void* v_raw, const void* q_norm_weight,
                        const void* k_norm_weight, const void* rope_table, float eps, const int32_t* cu_q,
                        const int32_t* slot_row, const int32_t* ctx_len, int num_requests, int total_q, int max_q,
                        void* resident_k, void* resident_v, long long rows_per_layer, void* scratch_k,
                        void* scratch_v, int scratch_rows, int num_layers, int layer, float scale, int path,
                        void* out, void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return verify_impl(q_raw, kQHeads * kHeadDim, k_raw, kKVHeads * kHeadDim, v_raw, kKVHeads * kHeadDim,
                     q_norm_weight, k_norm_weight, rope_table, eps, cu_q, slot_row, ctx_len, num_requests, total_q,
                     max_q, resident_k, resident_v, rows_per_layer, scratch_k, scratch_v, scratch_rows, num_layers,
                     layer, scale, path, out, workspace, workspace_bytes, stream);
}

int dspark_verify_strided(const void* q_raw, long long ld_q, const void* k_raw, long long ld_k, const void* v_raw,
                          long long ld_v, const void* q_norm_weight, const void* k_norm_weight,
                          const void* rope_table, float eps, const int32_t* cu_q, const int32_t* slot_row,
                          const int32_t* ctx_len, int num_requests, int total_q, int max_q, void* resident_k,
                          void* resident_v, long long rows_per_layer, void* scratch_k, void* scratch_v,
                          int scratch_rows, int num_layers, int layer, float scale, int path, void* out,
                          void* workspace, size_t workspace_bytes, cudaStream_t stream) {
  return verify_impl(q_raw, ld_q, k_raw, ld_k, v_raw, ld_v, q_norm_weight, k_norm_weight, rope_table, eps, cu_q,
                     slot_row, ctx_len, num_requests, total_q, max_q, resident_k, resident_v, rows_per_layer,
                     scratch_k, scratch_v, scratch_rows, num_layers, layer, scale, path, out, workspace,
                     workspace_bytes, stream);
}

int dspark_commit_kv(void* resident_k, void* resident_v, const void* scratch_k, const void* scratch_v,
                     const int32_t* cu_q, const int32_t* slot_row, const int32_t* ctx_len, const int32_t* slot_cap,
                     const int32_t* n_commit, int num_requests, int num_layers, long long rows_per_layer,
                     int scratch_rows, int dtype, cudaStream_t stream) {
  if (!resident_k || !resident_v || !scratch_k || !scratch_v || !cu_q || !slot_row || !ctx_len || !slot_cap ||
      !n_commit || num_requests < 1 || num_layers < 1 || num_layers > 65535 || rows_per_layer < 1 ||
      scratch_rows < 1 || !aligned(resident_k, 16) || !aligned(resident_v, 16) || !aligned(scratch_k, 16) ||
      !aligned(scratch_v, 16) || (dtype != DSPARK_DTYPE_BF16 && dtype != DSPARK_DTYPE_F32))
    return DSPARK_ERR_INVALID_ARGUMENT;
  CommitParams cp;
  cp.resident_k = static_cast<uint4*>(resident_k);
  cp.resident_v = static_cast<uint4*>(resident_v);
  cp.scratch_k = static_cast<const uint4*>(scratch_k);
  cp.scratch_v = static_cast<const uint4*>(scratch_v);
  cp.vec_per_row = kKVHeads * kHeadDim * (dtype == DSPARK_DTYPE_F32 ? 4 : 2) / 16;
  cp.cu_q = cu_q;
  cp.slot_row = slot_row;
  cp.ctx_len = ctx_len;
  cp.slot_cap = slot_cap;
  cp.n_commit = n_commit;
  cp.num_requests = num_requests;
  cp.num_layers = num_layers;
  cp.rows_per_layer = rows_per_layer;
  cp.scratch_rows = scratch_rows;
  commit_kernel<<<dim3(num_requests, num_layers), 256, 0, stream>>>(cp);
  return launch_status();
}

int dspark_row_argmax(const void* logits, long long ld, int rows, int vocab, int dtype, int32_t* pred,
                      cudaStream_t stream) {
  if (!logits || !pred || rows < 1 || vocab < 1 || ld < vocab || (dtype != DSPARK_DTYPE_BF16 && dtype != DSPARK_DTYPE_F32))
    return DSPARK_ERR_INVALID_ARGUMENT;
  if (dtype == DSPARK_DTYPE_BF16)
    row_argmax_kernel<__nv_bfloat16><<<rows, kArgmaxThreads, 0, stream>>>(static_cast<const __nv_bfloat16*>(logits),
                                                                            ld, vocab, pred);
  else
    row_argmax_kernel<float><<<rows, kArgmaxThreads, 0, stream>>>(static_cast<const float*>(logits), ld, vocab, pred);
  return launch_status();
}

int dspark_rms_norm(const void* x, long long ld_x, const void* weight, float eps, int rows, int hidden, void* out,
                    long long ld_out, cudaStream_t stream) {
  if (rows < 0 || rows > (1 << 30) || hidden < 8 || hidden % 8 != 0 || ld_x < hidden || ld_out < hidden ||
      ld_x % 8 != 0 || ld_out % 8 != 0 || !(eps >= 0.f))
    return DSPARK_ERR_INVALID_ARGUMENT;
  if (rows == 0) return DSPARK_OK;  // empty tensors may carry null pointers
  if (!x || !weight || !out || !aligned(x, 16) || !aligned(weight, 16) || !aligned(out, 16))
    return DSPARK_ERR_INVALID_ARGUMENT;
  const float inv_hidden = 1.0f / static_cast<float>(hidden);
  rms_norm_kernel<false><<<(rows + kNormRowsPerCta - 1) / kNormRowsPerCta, kNormThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), ld_x, nullptr, 0, static_cast<const __nv_bfloat16*>(weight), eps,
      inv_hidden, rows, hidden, static_cast<__nv_bfloat16*>(out), ld_out, nullptr, 0);
  return launch_status();
}

int dspark_add_rms_norm(const void* x, long long ld_x, const void* delta, long long ld_d, const void* weight,
                        float eps, int rows, int hidden, void* out, long long ld_out, void* sum_out,
                        long long ld_sum, cudaStream_t stream) {
  if (rows < 0 || rows > (1 << 30) || hidden < 8 || hidden % 8 != 0 || ld_x < hidden || ld_d < hidden ||
      ld_out < hidden || ld_sum < hidden || ld_x % 8 != 0 || ld_d % 8 != 0 || ld_out % 8 != 0 || ld_sum % 8 != 0 ||
      !(eps >= 0.f))
    return DSPARK_ERR_INVALID_ARGUMENT;
  if (rows == 0) return DSPARK_OK;  // empty tensors may carry null pointers
  if (!x || !delta || !weight || !out || !sum_out || !aligned(x, 16) || !aligned(delta, 16) ||
      !aligned(weight, 16) || !aligned(out, 16) || !aligned(sum_out, 16))
    return DSPARK_ERR_INVALID_ARGUMENT;
  // the second pass re-reads x and delta after the first pass's stores: an output that
  // shares bytes with an input (an in-place residual update) would change it mid-row
  auto span = [&](const void* p, long long ld) {
    const uintptr_t a = reinterpret_cast<uintptr_t>(p);
    return std::make_pair(a, a + static_cast<uintptr_t>(((rows - 1) * ld + hidden) * 2));
  };
  auto overlap = [](std::pair<uintptr_t, uintptr_t> u, std::pair<uintptr_t, uintptr_t> v) {
    return u.first < v.second && v.first < u.second;
  };
  const auto sx = span(x, ld_x), sd = span(delta, ld_d), so = span(out, ld_out), ss = span(sum_out, ld_sum);
  if (overlap(sx, so) || overlap(sx, ss) || overlap(sd, so) || overlap(sd, ss) || overlap(so, ss))
    return DSPARK_ERR_INVALID_ARGUMENT;
  const float inv_hidden = 1.0f / static_cast<float>(hidden);
  rms_norm_kernel<true><<<(rows + kNormRowsPerCta - 1) / kNormRowsPerCta, kNormThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(x), ld_x, static_cast<const __nv_bfloat16*>(delta), ld_d,
      static_cast<const __nv_bfloat16*>(weight), eps, inv_hidden, rows, hidden, static_cast<__nv_bfloat16*>(out),
      ld_out, static_cast<__nv_bfloat16*>(sum_out), ld_sum);
  return launch_status();
}

int dspark_qk_norm_rope(const void* q, long long ld_q, const void* k, long long ld_k, const void* q_norm_weight,
                        const void* k_norm_weight, float q_eps, float k_eps, const void* cos_table,
                        const void* sin_table, long long ld_cs, int rows, int q_heads, int kv_heads, void* q_out,
                        void* k_out, cudaStream_t stream) {
  if (rows < 0 || rows > (1 << 24) || q_heads < 1 || kv_heads < 1 || q_heads > 256 || kv_heads > 256 ||
      ld_q < static_cast<long long>(q_heads) * kRopeDim || ld_k < static_cast<long long>(kv_heads) * kRopeDim ||
      ld_cs < kRopeDim || ld_q % 4 != 0 || ld_k % 4 != 0 || ld_cs % 4 != 0 || !(q_eps >= 0.f) || !(k_eps >= 0.f))
    return DSPARK_ERR_INVALID_ARGUMENT;
  if (rows == 0) return DSPARK_OK;  // empty tensors may carry null pointers
  if (!q || !k || !q_norm_weight || !k_norm_weight || !cos_table || !sin_table || !q_out || !k_out ||
      !aligned(q, 8) || !aligned(k, 8) || !aligned(q_norm_weight, 8) || !aligned(k_norm_weight, 8) ||
      !aligned(cos_table, 8) || !aligned(sin_table, 8) || !aligned(q_out, 8) || !aligned(k_out, 8))
    return DSPARK_ERR_INVALID_ARGUMENT;
  const long long items = static_cast<long long>(rows) * (q_heads + kv_heads);
  qk_norm_rope_kernel<<<static_cast<unsigned>((items + kNormRowsPerCta - 1) / kNormRowsPerCta), kNormThreads, 0,
                        stream>>>(
      static_cast<const __nv_bfloat16*>(q), ld_q, static_cast<const __nv_bfloat16*>(k), ld_k,
      static_cast<const __nv_bfloat16*>(q_norm_weight), static_cast<const __nv_bfloat16*>(k_norm_weight), q_eps,
      k_eps, static_cast<const __nv_bfloat16*>(cos_table), static_cast<const __nv_bfloat16*>(sin_table), ld_cs, rows,
      q_heads, kv_heads, static_cast<__nv_bfloat16*>(q_out), static_cast<__nv_bfloat16*>(k_out));
  return launch_status();
}

int dspark_silu_mul(const void* gate_up, long long ld, int rows, int inter, void* out, long long ld_out,
                    cudaStream_t stream) {
  if (rows < 0 || rows > (1 << 24) || inter < 8 || inter % 8 != 0 || inter > (1 << 24) ||
      ld < 2ll * inter || ld % 8 != 0 || ld_out < inter || ld_out % 8 != 0)
    return DSPARK_ERR_INVALID_ARGUMENT;
  if (rows == 0) return DSPARK_OK;  // empty tensors may carry null pointers
  if (!gate_up || !out || !aligned(gate_up, 16) || !aligned(out, 16)) return DSPARK_ERR_INVALID_ARGUMENT;
  const long long threads = static_cast<long long>(rows) * (inter / 8);
  silu_mul_kernel<<<static_cast<unsigned>((threads + kSiluThreads - 1) / kSiluThreads), kSiluThreads, 0, stream>>>(
      static_cast<const __nv_bfloat16*>(gate_up), ld, rows, inter, static_cast<__nv_bfloat16*>(out), ld_out);
  return launch_status();
}

int dspark_greedy_accept(const int32_t* pred, const long long* tokens, const int32_t* cu_q, int num_requests,
                         int total_rows, const long long* eos, int n_eos, const int32_t* budget, int32_t* accepted,
                         int32_t* n_commit, long long* emitted, cudaStream_t stream) {
  if (!pred || !tokens || !cu_q || num_requests < 1 || total_rows < num_requests || n_eos < 0 ||
      (n_eos > 0 && !eos) || !accepted || !n_commit || !emitted)
    return DSPARK_ERR_INVALID_ARGUMENT;
  AcceptParams p{pred, tokens, cu_q, eos, n_eos, budget, num_requests, total_rows, accepted, n_commit, emitted};
  greedy_accept_kernel<<<(num_requests + 127) / 128, 128, 0, stream>>>(p);
  return launch_status();
}

size_t dspark_markov_scratch_bytes(void) { return markov::kScratchBytes; }

int dspark_set_grid_barrier_timeout(unsigned long long ns) {
  return cudaMemcpyToSymbol(g_grid_barrier_limit_ns, &ns, sizeof(ns)) == cudaSuccess ? DSPARK_OK : DSPARK_ERR_CUDA;
}

namespace {

// Shared argument checks and parameter block of the Markov entries.
int markov_setup(const void* proj_weight, const void* emb_table, int vocab, int rank, const void* base,
                 long long base_stride_r, const void* hidden, int hidden_dim, const void* conf_w, float conf_b,
                 long long* tokens, float* conf, long long tok_stride, int num_requests, void* scratch,
                 CUtensorMap* wm, markov::Params* pp, int* grid) {
  if (!proj_weight || !emb_table || !base || !hidden || !conf_w || !tokens || !conf || !scratch || vocab < 8 ||
      vocab % 8 != 0 || rank < 64 || rank > markov::kMaxRank || rank % 64 != 0 || hidden_dim < 1 ||
      num_requests < 1 || num_requests > markov::kRows || base_stride_r < 1 || !aligned(proj_weight, 16) ||
      !aligned(emb_table, 16) || !aligned(base, 16) || !aligned(scratch, 16))
    return DSPARK_ERR_INVALID_ARGUMENT;
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != DSPARK_OK) return st;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(rank), static_cast<cuuint64_t>(vocab)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(rank) * 2};
  cuuint32_t box[2] = {64, static_cast<cuuint32_t>(markov::kVocabTile)};
  cuuint32_t estr[2] = {1, 1};
  if (g_encode(wm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(proj_weight), dims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return DSPARK_ERR_CUDA;
  markov::Params& p = *pp;
  p = markov::Params{};
  p.emb_table = static_cast<const __nv_bfloat16*>(emb_table);
  p.base = static_cast<const __nv_bfloat16*>(base);
  p.base_stride_r = base_stride_r;
  p.hidden = static_cast<const __nv_bfloat16*>(hidden);
  p.hidden_dim = hidden_dim;
  p.conf_vec = hidden_dim % 8 == 0 && aligned(hidden, 16) && aligned(conf_w, 16);
  p.conf_w = static_cast<const __nv_bfloat16*>(conf_w);
  p.conf_b = conf_b;
  p.tokens = tokens;
  p.tok_stride = tok_stride;
  p.conf = conf;
  p.best = static_cast<unsigned long long*>(scratch);
  p.arrivals = reinterpret_cast<unsigned int*>(static_cast<uint8_t*>(scratch) + 3 * markov::kRows * 8);
  p.generation = p.arrivals + 1;
  p.exits = p.arrivals + 2;
  p.failed = p.arrivals + 3;
  p.num_requests = num_requests;
  p.dup = num_requests <= 64;
  p.vocab = vocab;
  p.rank = rank;
  p.tiles = (vocab + markov::kVocabTile - 1) / markov::kVocabTile;
  *grid = p.tiles < dev.sms ? p.tiles : dev.sms;
  return DSPARK_OK;
}

}  // namespace

int dspark_markov_step(const void* proj_weight, const void* emb_table, int vocab, int rank, const void* base,
                       long long base_stride_r, int k, const long long* prev, long long prev_stride,
                       const void* hidden, int hidden_dim, const void* conf_w, float conf_b, long long* tokens,
                       float* conf, long long tok_stride, int num_requests, void* scratch, cudaStream_t stream) {
  if (!prev || k < 0 || k >= base_stride_r || prev_stride < 0 || tok_stride <= k) return DSPARK_ERR_INVALID_ARGUMENT;
  CUtensorMap wm;
  markov::Params p;
  int grid = 0;
  int st = markov_setup(proj_weight, emb_table, vocab, rank, base, base_stride_r, hidden, hidden_dim, conf_w, conf_b,
                        tokens, conf, tok_stride, num_requests, scratch, &wm, &p, &grid);
  if (st != DSPARK_OK) return st;
  p.k = k;
  p.steps = 1;
  p.prev = prev;
  p.prev_stride = prev_stride;
  markov::markov_step_kernel<<<grid, markov::kThreads, markov::kSmemBytes, stream>>>(wm, p);
  return launch_status();
}

int dspark_markov_block(const void* proj_weight, const void* emb_table, int vocab, int rank, const void* base,
                        int block_size, const long long* anchors, const void* hidden, int hidden_dim,
                        const void* conf_w, float conf_b, long long* tokens, float* conf, int num_requests,
                        void* scratch, cudaStream_t stream) {
  if (!anchors || block_size < 1 || block_size > markov::kMaxSteps) return DSPARK_ERR_INVALID_ARGUMENT;
  CUtensorMap wm;
  markov::Params p;
  int grid = 0;
  int st = markov_setup(proj_weight, emb_table, vocab, rank, base, block_size, hidden, hidden_dim, conf_w, conf_b,
                        tokens, conf, block_size, num_requests, scratch, &wm, &p, &grid);
  if (st != DSPARK_OK) return st;
  p.steps = block_size;
  p.prev = anchors;
  p.prev_stride = 1;
  // Cooperative: the runtime refuses the launch unless every CTA can be
  // resident at once, which the grid barrier between steps relies on.
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid);
  cfg.blockDim = dim3(markov::kThreads);
  cfg.dynamicSmemBytes = markov::kSmemBytes;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeCooperative;
  attr[0].val.cooperative = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (cudaLaunchKernelEx(&cfg, markov::markov_block_kernel, wm, p) == cudaSuccess) return launch_status();
  (void)cudaGetLastError();
  // Refused (other work holds SMs): one launch per position, same results.
  for (int k = 0; k < block_size; ++k) {
    p.k = k;
    p.steps = 1;
    p.prev = k == 0 ? anchors : tokens + (k - 1);
    p.prev_stride = k == 0 ? 1 : block_size;
    markov::markov_step_kernel<<<grid, markov::kThreads, markov::kSmemBytes, stream>>>(wm, p);
    if ((st = launch_status()) != DSPARK_OK) return st;
  }
  return DSPARK_OK;
}

int dspark_draft_append(const void* context, int rows, int hidden, const void* kv_weight, int num_layers,
                        const void* k_norm_weight, const void* rope_table, float eps, const int32_t* cu_rows,
                        const int32_t* slot_row, const int32_t* ctx_len, const int32_t* count, int num_requests,
                        void* const* pool_k, void* const* pool_v, long long pool_rows, long long trash_row,
                        cudaStream_t stream) {
  if (!context || !kv_weight || !k_norm_weight || !rope_table || !cu_rows || !slot_row || !ctx_len || !count ||
      !pool_k || !pool_v || rows < 1 || hidden < 64 || hidden % 64 != 0 || num_layers < 1 ||
      num_layers > append::kMaxLayers || num_requests < 1 || !(eps > 0.f) || pool_rows < 1 ||
      pool_rows >= (1ll << 40) || trash_row < 0 || trash_row >= pool_rows || !aligned(context, 16) ||
      !aligned(kv_weight, 16) || !aligned(k_norm_weight, 16) || !aligned(rope_table, 16))
    return DSPARK_ERR_INVALID_ARGUMENT;
  for (int l = 0; l < num_layers; ++l)
    if (!pool_k[l] || !pool_v[l] || !aligned(pool_k[l], 16) || !aligned(pool_v[l], 16))
      return DSPARK_ERR_INVALID_ARGUMENT;
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != DSPARK_OK) return st;
  CUtensorMap cm, wm;
  cuuint32_t box[2] = {64, 128};
  cuuint32_t estr[2] = {1, 1};
  cuuint64_t cdims[2] = {static_cast<cuuint64_t>(hidden), static_cast<cuuint64_t>(rows)};
  cuuint64_t wdims[2] = {static_cast<cuuint64_t>(hidden), static_cast<cuuint64_t>(num_layers) * 2 * 1024};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(hidden) * 2};
  if (g_encode(&cm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(context), cdims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS ||
      g_encode(&wm, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(kv_weight), wdims, strides, box, estr,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return DSPARK_ERR_CUDA;
  append::Params p{};
  p.k_norm_w = static_cast<const __nv_bfloat16*>(k_norm_weight);
  p.rope = static_cast<const uint32_t*>(rope_table);
  p.cu_rows = cu_rows;
  p.slot_row = slot_row;
  p.ctx_len = ctx_len;
  p.count = count;
  for (int l = 0; l < num_layers; ++l) {
    p.pool_k[l] = static_cast<__nv_bfloat16*>(pool_k[l]);
    p.pool_v[l] = static_cast<__nv_bfloat16*>(pool_v[l]);
  }
  p.trash_row = trash_row;
  p.pool_rows = pool_rows;
  p.num_requests = num_requests;
  p.rows = rows;
  p.k_chunks = hidden / 64;
  p.layers = num_layers;
  p.row_tiles = (rows + append::kTileRows - 1) / append::kTileRows;
  p.eps = eps;
  // Two heads per tile once those tiles alone fill every SM (prefill-sized appends):
  // each context chunk then feeds twice the MMA work. Smaller appends keep one head
  // per tile, so their few row tiles still spread over the SMs.
  // Largest appends: 2-SM tiles of 256 rows x 2 heads, once they give every CTA pair
  // at least two tiles.
  const long long pair_tiles = static_cast<long long>((p.row_tiles + 1) / 2) * num_layers * 8;
  if (dev.append_pairs > 0 && pair_tiles >= 2ll * dev.append_pairs && pair_tiles < (1ll << 31)) {
    p.row_tiles = (p.row_tiles + 1) / 2;
    p.head_tiles = num_layers * 8;
    const int grid = 2 * dev.append_pairs;
    append::draft_append_pair_kernel<<<grid, append::kThreads, append::PairCfg::kSmemBytes, stream>>>(cm, wm, p);
    return launch_status();
  }
  const bool pair = static_cast<long long>(p.row_tiles) * num_layers * 8 >= dev.sms;
  p.head_tiles = num_layers * (pair ? 8 : 16);
  const long long tiles = static_cast<long long>(p.row_tiles) * p.head_tiles;
  if (tiles >= (1ll << 31)) return DSPARK_ERR_UNSUPPORTED;
  const int grid = tiles < dev.sms ? static_cast<int>(tiles) : dev.sms;
  if (pair)
    append::draft_append_kernel<2><<<grid, append::kThreads, append::Cfg<2>::kSmemBytes, stream>>>(cm, wm, p);
  else
    append::draft_append_kernel<1><<<grid, append::kThreads, append::Cfg<1>::kSmemBytes, stream>>>(cm, wm, p);
  return launch_status();
}

namespace {
// Stochastic scratch: the row statistics, then (256-byte aligned) the table of
// x / T for every bf16 bit pattern.
size_t stochastic_table_offset(int rows) {
  return (static_cast<size_t>(rows) * sizeof(sampling::RowStats) + 255) & ~static_cast<size_t>(255);
}
}  // namespace

size_t dspark_stochastic_scratch_bytes(int rows) {
  return rows > 0 ? stochastic_table_offset(rows) + sampling::kScaledTableSize * sizeof(double) : 0;
}

int dspark_stochastic_accept(const void* logits, long long ld, int dtype, int vocab, double temperature,
                             int target_rows, const double* q, int draft_rows, const long long* tokens,
                             const int32_t* cu_n, int num_requests, const double* uniforms, int u_stride,
                             const long long* eos, int n_eos, const int32_t* budget, long long* emitted,
                             int32_t* result, void* scratch, size_t scratch_bytes, cudaStream_t stream) {
  if (!logits || !cu_n || !uniforms || !budget || !emitted || !result || !scratch || vocab < 1 || ld < vocab ||
      (dtype != DSPARK_DTYPE_BF16 && dtype != DSPARK_DTYPE_F32) || !(temperature > 0.0) ||
      !std::isfinite(temperature) || num_requests < 1 || target_rows != draft_rows + num_requests ||
      draft_rows < 0 || (draft_rows > 0 && (!q || !tokens)) || u_stride < 1 || n_eos < 0 || (n_eos > 0 && !eos) ||
      scratch_bytes < dspark_stochastic_scratch_bytes(target_rows + draft_rows) || !aligned(scratch, 16))
    return DSPARK_ERR_INVALID_ARGUMENT;
  sampling::Params p{};
  p.logits = logits;
  p.ld = ld;
  p.dtype = dtype == DSPARK_DTYPE_BF16 ? 0 : 1;
  p.vocab = vocab;
  p.temperature = temperature;
  p.target_rows = target_rows;
  p.q = q;
  p.draft_rows = draft_rows;
  p.stats = static_cast<sampling::RowStats*>(scratch);
  p.scaled = nullptr;
  if (dtype == DSPARK_DTYPE_BF16) {
    double* table = reinterpret_cast<double*>(static_cast<uint8_t*>(scratch) +
                                              stochastic_table_offset(target_rows + draft_rows));
    sampling::scaled_table_kernel<<<sampling::kScaledTableSize / 256, 256, 0, stream>>>(table, temperature);
    const int st0 = launch_status();
    if (st0 != DSPARK_OK) return st0;
    p.scaled = table;
  }
  p.tokens = tokens;
  p.cu_n = cu_n;
  p.num_requests = num_requests;
  p.uniforms = uniforms;
  p.u_stride = u_stride;
  p.eos = eos;
  p.n_eos = n_eos;
  p.budget = budget;
  p.emitted = emitted;
  p.result = result;
  sampling::law_stats_kernel<<<target_rows + draft_rows, sampling::kThreads, 0, stream>>>(p);
  int st = launch_status();
  if (st != DSPARK_OK) return st;
  sampling::stochastic_accept_kernel<<<num_requests, sampling::kThreads, 0, stream>>>(p);
  return launch_status();
}

size_t dspark_propose_scratch_bytes(void) { return sampling::kScaledTableSize * sizeof(double); }

int dspark_stochastic_propose(const void* base, long long ld_base, const int32_t* row_index, const void* proj,
                              long long ld_proj, int vocab, double temperature, const double* uniforms, int rows,
                              double* law, long long ld_law, long long* tokens, int32_t* status, void* scratch,
                              size_t scratch_bytes, cudaStream_t stream) {
  if (rows < 0 || vocab < 1 || ld_base < vocab || ld_proj < vocab || ld_law < vocab || !(temperature > 0.0) ||
      !std::isfinite(temperature))
    return DSPARK_ERR_INVALID_ARGUMENT;
  if (rows == 0) return DSPARK_OK;
  if (!base || !proj || !uniforms || !law || !tokens || !status || !scratch ||
      scratch_bytes < dspark_propose_scratch_bytes() || !aligned(scratch, 16) || !aligned(law, 8))
    return DSPARK_ERR_INVALID_ARGUMENT;
  double* table = static_cast<double*>(scratch);
  sampling::scaled_table_kernel<<<sampling::kScaledTableSize / 256, 256, 0, stream>>>(table, temperature);
  int st = launch_status();
  if (st != DSPARK_OK) return st;
  sampling::ProposeParams p{};
  p.base = static_cast<const unsigned short*>(base);
  p.ld_base = ld_base;
  p.row_index = row_index;
  p.proj = static_cast<const unsigned short*>(proj);
  p.ld_proj = ld_proj;
  p.vocab = vocab;
  p.scaled = table;
  p.uniforms = uniforms;
  p.law = law;
  p.ld_law = ld_law;
  p.tokens = tokens;
  p.status = status;
  p.rows = rows;
  // Two CTAs per row (a cluster) when twice the rows still fit the SMs at once and
  // each half of the row fits the per-CTA tile totals; one CTA per row otherwise.
  DeviceInfo dev;
  st = current_device_info(&dev);
  if (st != DSPARK_OK) return st;
  const long long tiles = (static_cast<long long>(vocab) + sampling::kThreads * 8 - 1) / (sampling::kThreads * 8);
  if (2ll * rows <= dev.sms && (tiles + 1) / 2 <= sampling::kPairMaxTiles)
    sampling::propose_law_pair_kernel<<<2 * rows, sampling::kThreads, 0, stream>>>(p);
  else
    sampling::propose_law_kernel<<<rows, sampling::kThreads, 0, stream>>>(p);
  return launch_status();
}

int dspark_train_plan(int num_seqs, const int32_t* ctx_len, const int32_t* num_blocks, const int32_t* anchors,
                      int block_size, int grid_limit, int32_t* plan, long long plan_capacity, long long* plan_words) {
  using namespace train;
  if (num_seqs < 1 || !ctx_len || !num_blocks || !anchors || !plan_words || block_size < kMinBlock ||
      block_size > kMaxBlock || grid_limit < 1 || grid_limit > 65535)
    return DSPARK_ERR_INVALID_ARGUMENT;
  // Packed offsets of every sequence: queries = its blocks' rows, keys = context then block rows.
  struct Tile {
    int item[kItemWords];
    int cost;
  };
  std::vector<Tile> tiles;
  long long q_off = 0, k_off = 0, a_off = 0;
  for (int s = 0; s < num_seqs; ++s) {
    const long long ctx = ctx_len[s], nb = num_blocks[s];
    if (ctx < 0 || nb < 0) return DSPARK_ERR_INVALID_ARGUMENT;
    const long long nq = nb * block_size;
    if (q_off + nq >= (1ll << 31) || k_off + ctx + nq >= (1ll << 31)) return DSPARK_ERR_UNSUPPORTED;
    for (long long t0 = 0; t0 < nq; t0 += kTileQ) {
      Tile tile{};
      const int n = static_cast<int>(std::min<long long>(kTileQ, nq - t0));
      const int b0 = static_cast<int>(t0 / block_size), b1 = static_cast<int>((t0 + n - 1) / block_size);
      int ctx_keys = 0;
      for (int b = b0; b <= b1; ++b) {
        const int a = static_cast<int>(std::max<long long>(0, std::min<long long>(anchors[a_off + b], ctx)));
        tile.item[kIAnchors + b - b0] = a;
        ctx_keys = std::max(ctx_keys, a);
      }
      tile.item[kIQRow0] = static_cast<int>(q_off + t0);
      tile.item[kINq] = n;
      tile.item[kIKBase] = static_cast<int>(k_off);
      tile.item[kICtxKeys] = ctx_keys;
      tile.item[kIBlkKey0] = static_cast<int>(k_off + ctx + static_cast<long long>(b0) * block_size);
      tile.item[kIPhase] = static_cast<int>(t0 % block_size);
      tile.item[kINBlocks] = b1 - b0 + 1;
      tile.item[kIBlockSize] = block_size;
      // one key block of tile overhead (Q load, epilogue) on top of the key blocks
      tile.cost = (ctx_keys + kKeyBlock - 1) / kKeyBlock + 2;
      for (int h = 0; h < kKVHeads; ++h) {
        tile.item[kIHead] = h;
        tiles.push_back(tile);
      }
    }
    q_off += nq;
    k_off += ctx + nq;
    a_off += nb;
  }
  const int n_items = static_cast<int>(tiles.size());
  const int grid = std::max(1, std::min(grid_limit, n_items));
  const long long words = plan_items_at(grid) + static_cast<long long>(n_items) * kItemWords;
  *plan_words = words;
  if (plan == nullptr) return DSPARK_OK;            // size query
  if (plan_capacity < words) return DSPARK_ERR_INVALID_ARGUMENT;
  // Largest tile first onto the least-loaded CTA.
  std::vector<int> order(n_items);
  std::iota(order.begin(), order.end(), 0);
  std::stable_sort(order.begin(), order.end(), [&](int a, int b) { return tiles[a].cost > tiles[b].cost; });
  using Load = std::pair<long long, int>;
  std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
  for (int c = 0; c < grid; ++c) heap.push({0, c});
  std::vector<std::vector<int>> per_cta(grid);
  for (int i : order) {
    Load l = heap.top();
    heap.pop();
    per_cta[l.second].push_back(i);
    heap.push({l.first + tiles[i].cost, l.second});
  }
  std::fill(plan, plan + words, 0);
  plan[0] = kPlanMagic;
  plan[1] = n_items;
  plan[2] = grid;
  plan[3] = static_cast<int>(q_off);
  plan[4] = static_cast<int>(k_off);
  int* items = plan + plan_items_at(grid);
  int next = 0;
  for (int c = 0; c < grid; ++c) {
    plan[kPlanHeader + c] = next;
    for (int i : per_cta[c]) std::copy(tiles[i].item, tiles[i].item + kItemWords, items + (next++) * kItemWords);
  }
  plan[kPlanHeader + grid] = next;
  return DSPARK_OK;
}

int dspark_train_attn(const void* q, const void* k, const void* v, int total_q, long long total_k,
                      const int32_t* plan, int grid, float scale, void* out, cudaStream_t stream) {
  if (!q || !k || !v || !plan || !out || total_q < 1 || total_k < 1 || total_k >= (1ll << 31) || grid < 1 ||
      grid > 65535 || !(scale > 0.f) || !aligned(q, 16) || !aligned(k, 16) || !aligned(v, 16) ||
      !aligned(out, 16) || !aligned(plan, 16))
    return DSPARK_ERR_INVALID_ARGUMENT;
  DeviceInfo dev;
  int st = current_device_info(&dev);
  if (st != DSPARK_OK) return st;
  CUtensorMap qm, km, vm;
  if ((st = encode_rows_map(&qm, q, total_q, 16, 2, train::kTileQ)) != DSPARK_OK) return st;
  if ((st = encode_rows_map(&km, k, total_k, kKVHeads, 1, train::kKeyBlock)) != DSPARK_OK) return st;
  if ((st = encode_rows_map(&vm, v, total_k, kKVHeads, 1, train::kKeyBlock)) != DSPARK_OK) return st;
  train::train_attn_kernel<<<grid, train::kThreads, train::kSmemBytes, stream>>>(
      qm, km, vm, plan, static_cast<__nv_bfloat16*>(out), total_q, static_cast<int>(total_k),
      scale * 1.4426950408889634f);
  return launch_status();
}

}  // extern "C"

// ---------------------------------------------------------------------------
// Allocation-free variant of dspark_varlen_attn.
//
// Some callers cannot allocate device memory for a workspace: a host that
// embeds this library through a C FFI (Go, Java) and has no access to the
// framework allocator that owns the GPU, or a serving process that has handed
// nearly all HBM to its KV-cache pool up front, where an extra cudaMalloc
// fails or fragments the pool and a cudaMalloc/cudaFree pair would also
// synchronise the device in the middle of a decode step. For them the
// split-item partials live in the static array below instead of a
// caller-provided workspace.
// ---------------------------------------------------------------------------
namespace {

// The scratch holds the partials of at most this many persistent CTAs; the
// entry point never launches more. Its size does not depend on the inputs.
constexpr int kNoAllocMaxCtas = 148;
constexpr size_t kNoAllocScratchBytes = workspace_for_grid(kNoAllocMaxCtas);

// 148 CTAs x (2 x 66 KB of fp32 partials + 384 B of merge entries) = 18.8 MiB. Every
// GPU that loads this library holds it until the process exits.
static __device__ __align__(256) unsigned char g_noalloc_scratch[kNoAllocScratchBytes];

void* g_noalloc_ptr[kMaxDevices] = {};

}  // namespace

extern "C" size_t dspark_varlen_attn_noalloc_scratch_bytes(void) { return kNoAllocScratchBytes; }

extern "C" int dspark_varlen_attn_noalloc(const void* q, const void* k, const void* v, const int32_t* cu_q,
                                          const int32_t* cu_k, int num_requests, int total_q, long long key_rows,
                                          int max_q, int max_k, float scale, void* out, cudaStream_t stream) {
  (void)max_q;
  (void)max_k;
  if (!common_ok(q, out, cu_q, num_requests, total_q, scale, DSPARK_DTYPE_BF16) || !k || !v || !cu_k ||
      key_rows < 1)
    return DSPARK_ERR_INVALID_ARGUMENT;
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess) return DSPARK_ERR_CUDA;
  DeviceInfo info;
  int st = device_info(dev, &info);
  if (st != DSPARK_OK) return st;
  void* scratch = nullptr;
  {
    // Once per device, with that device current: the host-side symbol is not a
    // device address, so ask the runtime for this device's copy of the array.
    std::lock_guard<std::mutex> lock(g_mu);
    if (g_noalloc_ptr[dev] == nullptr) {
      void* ptr = nullptr;
      if (cudaGetSymbolAddress(&ptr, g_noalloc_scratch) != cudaSuccess || ptr == nullptr) return DSPARK_ERR_CUDA;
      g_noalloc_ptr[dev] = ptr;
    }
    scratch = g_noalloc_ptr[dev];
  }
  const int grid = info.sms < kNoAllocMaxCtas ? info.sms : kNoAllocMaxCtas;
  if (workspace_for_grid(grid) > kNoAllocScratchBytes) return DSPARK_ERR_UNSUPPORTED;
  AttnParams p = base_params(q, out, cu_q, num_requests, total_q, scale, 1);
  p.mode = kModeVarlen;
  p.cu_k = cu_k;
  bind_workspace(p, scratch, grid);
  p.rows_a = key_rows;
  CUtensorMap ka, va;
  if ((st = encode_kv_map(&ka, k, key_rows)) != DSPARK_OK) return st;
  if ((st = encode_kv_map(&va, v, key_rows)) != DSPARK_OK) return st;
  attn_bf16_kernel<true, false><<<grid, kAttnThreads, kAttnSmemBytes, stream>>>(ka, va, ka, va, p);
  if ((st = launch_status()) != DSPARK_OK) return st;
  return launch_merge(p, stream);
}
