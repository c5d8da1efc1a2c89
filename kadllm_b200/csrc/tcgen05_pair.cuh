// CTA-pair (cta_group::2) tensor-core primitives and the tensor-map (TMA) copies
// used by the persistent GEMM.
//
// A CTA pair is the two CTAs of a 2-CTA cluster (%cluster_ctarank 0 and 1).
// One thread of rank 0 issues tcgen05.mma.cta_group::2: the A operand's rows
// 0-127 and the B operand's rows 0-127 come from rank 0's shared memory, rows
// 128-255 of both from rank 1's shared memory at the same offsets, and the
// 256-row accumulator lands in the two CTAs' tensor memories (rows 0-127 in rank
// 0's, 128-255 in rank 1's) at the same column.  Every tcgen05 instruction of a
// kernel that uses these must be the cta_group::2 form.
//
// Operand layout: K-major, 128-byte swizzle.  A tensor-map copy of a box of 64
// BF16 (128 bytes) x R rows writes R rows of 128 bytes, row r at r * 128, its
// 16-byte chunks permuted by (r % 8); groups of 8 rows are 1024 bytes apart.
// The matrix descriptor of such a tile (1024-byte aligned) has SBO = 1024 and
// swizzle mode 2; the K = 16 slice j of the 64-wide row starts 32 * j bytes in.
#pragma once
#include <cuda.h>

#include "tcgen05.cuh"

namespace kb {
namespace tc2 {

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_id() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;\n" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t num_clusters() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;\n" : "=r"(r));
  return r;
}
// Every thread of both CTAs; release / acquire at cluster scope.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\nbarrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;\n" ::: "memory"); }
// shared::cluster address of the same shared-memory location in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t peer_addr(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}
// Arrive once on an mbarrier given by its shared::cluster address (possibly the peer's).
__device__ __forceinline__ void arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(cluster_addr) : "memory");
}

// K-major, 128-byte-swizzle matrix descriptor (version 1, SBO 1024 bytes).
__device__ __forceinline__ uint64_t desc_sw128(uint32_t saddr) {
  return uint64_t((saddr >> 4) & 0x3FFFu) | (uint64_t(1) << 16) | (uint64_t(1024 >> 4) << 32) |
         (uint64_t(1) << 46) | (uint64_t(2) << 61);
}

// D[tmem] (+)= A * B over the pair; issued by one thread of rank 0.
__device__ __forceinline__ void mma(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                    bool accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(uint32_t(accumulate))
      : "memory");
}
// Arrive once on the mbarrier at `cluster_addr` (this CTA's or the peer's) when every
// pair MMA this thread issued so far has completed.
__device__ __forceinline__ void commit(uint32_t cluster_addr) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];\n" ::"r"(cluster_addr)
               : "memory");
}
// Whole warp, in both CTAs of the pair: allocate `cols` TMEM columns at the same address.
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_u32(slot)), "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
}
__device__ __forceinline__ void tmem_free(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(base), "r"(cols) : "memory");
}

// Tensor-map copy of the box at (x = inner coordinate, y = row) into this CTA's shared
// memory; its bytes complete on the mbarrier at `bar_cluster_addr`, which may be the
// peer CTA's (the pair's forms: no multicast).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y,
                                            uint32_t bar_cluster_addr) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster_addr)
      : "memory");
}
// Tensor-map copy into this CTA's shared memory completing on this CTA's mbarrier
// (the single-CTA form, used by the epilogue for its residual tiles).
__device__ __forceinline__ void tma_load_2d_cta(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3}], [%4];\n" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
// Tensor-map store of a shared-memory box to global memory at (x, y); boxes clip at
// the tensor's edges.  Completion is tracked by bulk groups.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, int x, int y, const void* src) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%1, %2}], [%3];\n" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(x), "r"(y), "r"(smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }
// Wait until at most N committed bulk groups still read their shared-memory sources.
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}
// Wait until every committed bulk group has completed (writes visible).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

__device__ __forceinline__ void prefetch_map(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];\n" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

}  // namespace tc2
}  // namespace kb
