// Helpers for 2-SM (CTA pair) tcgen05 kernels on sm_100a: cluster rank and
// barriers, remote mbarrier arrivals, pair-wide TMEM allocation, the cta_group::2
// MMA forms and their multicast commits. A pair kernel is launched with clusters
// of two CTAs; rank 0 issues every MMA, whose A rows and accumulator rows are each
// CTA's own 128 rows and whose B operand is split by N between the two CTAs'
// shared memory at the same address. No copy here multicasts: each CTA loads its
// own half with its own TMA copies, whose bytes may count on rank 0's barrier.
#pragma once
#include "train.cuh"

namespace dspark {
namespace pair {

using train::wait_or_abort;

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_index() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
  return r;
}

// All threads of both CTAs; orders every earlier memory access of each before
// anything after it in the other. Split into its halves where some threads have
// work to do in between (each thread arrives, then waits, once per phase).
__device__ __forceinline__ void cluster_arrive() {
  asm volatile("barrier.cluster.arrive.release.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_wait() {
  asm volatile("barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

__device__ __forceinline__ void cluster_sync() {
  cluster_arrive();
  cluster_wait();
}

// Address of the same shared-memory variable in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t cluster_addr(uint32_t local, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local), "r"(rank));
  return r;
}

// One arrival on the mbarrier at `local`'s offset in rank 0 (default .release.cta
// semantics, as for any arrival; the TMEM stores it follows have completed, and
// their tcgen05.fence::before_thread_sync orders them before it).
__device__ __forceinline__ void arrive_rank0(uint32_t local) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr(local, 0)) : "memory");
}

// A 2-D TMA load into this CTA's shared memory whose bytes are counted on an
// mbarrier of either CTA of the pair (cluster address; `.cta_group::2`, no multicast).
__device__ __forceinline__ void tma_load_2d_pair(uint32_t dst, const CUtensorMap* m, int c0, int c1,
                                                 uint32_t cluster_bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(c0), "r"(c1), "r"(cluster_bar)
      : "memory");
}

// The pair kernel's bounded wait (default .acquire.cta semantics, as for a
// barrier that only this CTA arrives on).
__device__ __forceinline__ bool pair_wait(uint32_t bar, uint32_t parity, volatile int* abort_flag) {
  return wait_or_abort(bar, parity, abort_flag);
}

// TMEM of both CTAs at the same columns: one warp of each CTA (the same warp).
__device__ __forceinline__ void tmem_alloc_pair(uint32_t slot_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(slot_smem), "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}

// Instruction descriptor of a 2-SM kind::f16 MMA: fp32 D, bf16 A and B, A
// K-major, B K-major (b_mn = 0) or N-major (b_mn = 1), M = 256, N = 128.
__host__ __device__ constexpr uint32_t instr_desc_pair(uint32_t b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (b_mn << 16) | ((128u >> 3) << 17) | ((256u >> 4) << 24);
}

// 2-SM MMA, A from shared memory: D rows of each CTA from its own A rows; B is
// the N/2 columns each CTA holds at the same address. One thread of rank 0.
__device__ __forceinline__ void umma_pair_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 2-SM MMA, A from each CTA's TMEM (128 lanes x 8 columns of packed bf16 pairs).
__device__ __forceinline__ void umma_pair_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the mbarrier at `bar`'s offset in both CTAs when every 2-SM MMA
// this thread issued so far is done.
__device__ __forceinline__ void umma_commit_pair(uint32_t bar) {
  asm volatile(
      "{\n\t.reg .b16 m;\n\t"
      "mov.b16 m, 3;\n\t"
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], m;\n\t}" ::"r"(
          bar)
      : "memory");
}

// The same, arriving on this CTA's barrier only.
__device__ __forceinline__ void umma_commit_pair_local(uint32_t bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar) : "memory");
}

}  // namespace pair
}  // namespace dspark
