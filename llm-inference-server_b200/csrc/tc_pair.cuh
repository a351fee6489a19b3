// tcgen05 CTA-pair (cta_group::2) helpers for sm_100a: cluster rank and barrier, remote
// mbarrier arrivals in the leader CTA, pair-counted TMA loads, pair TMEM allocation, and
// M = 256 MMAs whose operands come from both CTAs' shared memory (each CTA holds half of
// A's rows and half of B's N extent), committed to both CTAs' barriers.  No load here uses
// cluster multicast: every CTA loads its own half from this GPU's memory.
#pragma once

#include <stdint.h>

#include "pa_common.cuh"
#include "tc_common.cuh"

namespace pa {

__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// Every thread of both CTAs (the non-.aligned form: callers reconverge their warp first).
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}
// shared::cluster address of the variable at local address `a` in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t mapa_rank(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
// Arrive on a barrier of the peer CTA (the default .release.cta form, as CUTLASS's cluster
// pipelines use: a .cluster-scope release costs a cluster-wide memory fence per arrival).
// What the arrival publishes stays on the arriving SM — its own TMEM reads and writes,
// ordered by tcgen05.fence::before_thread_sync, and its own shared-memory P, ordered for
// its tensor core by fence.proxy.async — so the MMA it unblocks needs no wider fence.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_remote(uint32_t cluster_addr, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cluster.b64 _, [%0], %1;" ::"r"(cluster_addr), "r"(bytes)
               : "memory");
}
// Bounded wait (arrivals and transfers may come from the peer CTA).
__device__ __forceinline__ bool mbar_wait_cl(uint64_t* bar, uint32_t parity) { return mbar_wait(bar, parity); }
// Tiled 3-D load into this CTA's shared memory whose completion is counted on an
// mbarrier that may sit in the peer CTA of the pair (`bar_cluster` is a shared::cluster
// address).
__device__ __forceinline__ void tma_load_3d_pair(void* smem_dst, const CUtensorMap* map, int c0, int c1, int c2,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4}], [%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar_cluster)
      : "memory");
}

// ------------------------------------------------------------------ tcgen05, pair forms
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* smem_dst, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(smem_dst)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// D (+)= A[smem] * B[smem] over both CTAs of the pair (M = 256: 128 rows per CTA).
__device__ __forceinline__ void umma_pair_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D (+)= A[tmem] * B[smem] over both CTAs of the pair.
__device__ __forceinline__ void umma_pair_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive once on the barrier at local offset `bar` in BOTH CTAs of the pair when every
// tcgen05 operation this thread issued so far completes.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(uint16_t(3))
      : "memory");
}

// Tiled 2-D load into this CTA's shared memory whose completion is counted on an
// mbarrier that may sit in the peer CTA of the pair (`bar_cluster` is a shared::cluster
// address).  c0 is the innermost coordinate (its byte offset a multiple of 16).
__device__ __forceinline__ void tma_load_2d_pair(void* smem_dst, const CUtensorMap* map, int c0, int c1,
                                                 uint32_t bar_cluster) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar_cluster)
      : "memory");
}

}  // namespace pa
