// PTX wrappers for the CTA-pair (cta_group::2) tensor-core path of sm_100a:
// cluster rank / barrier, shared::cluster address mapping, remote mbarrier
// arrivals, pair-wide TMEM allocation, the 2-SM MMA and its commit, and the
// TMA tile load whose completion is counted on the pair leader's mbarrier.
// Written from the PTX ISA chapters on tcgen05, cp.async.bulk.tensor,
// mbarrier and clusters.  Every CTA fetches its own half of each operand
// tile from this GPU's memory with a plain (single-destination) TMA copy.
#pragma once

#include "tc_gemm.cuh"

namespace lrl {
namespace tc2 {

using tc::smem_addr;

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;\n" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t cluster_id_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%clusterid.x;\n" : "=r"(r));
  return r;
}

__device__ __forceinline__ uint32_t nclusters_x() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%nclusterid.x;\n" : "=r"(r));
  return r;
}

// every thread of both CTAs; release/acquire orders the shared-memory writes
// (barrier initialisation, remote arrivals) of one CTA before the other's
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n" ::: "memory");
  asm volatile("barrier.cluster.wait.acquire.aligned;\n" ::: "memory");
}

// shared::cta address of this CTA -> shared::cluster address of the same
// offset in CTA `rank` of the cluster
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;\n" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

// arrive (count 1) on an mbarrier named by its shared::cluster address
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];\n" ::"r"(cluster_addr) : "memory");
}

// TMEM allocation for a CTA pair: one warp of EACH CTA executes it; both get
// the same column base written to their `dst_smem`.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;\n" ::"r"(smem_addr(dst_smem)),
               "r"(ncols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;\n" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;\n" ::"r"(taddr), "r"(ncols) : "memory");
}

// D[tmem] (+)= A * B over the pair: A's rows are split between the two CTAs'
// shared memory (same offsets), as are B's rows; each CTA's TMEM receives the
// accumulator rows of its A half.  Issued by one thread of the even CTA.
__device__ __forceinline__ void umma_bf16_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// block-scaled-free fp8 MMA over the pair (E4M3/E5M2 operands, fp32 accum)
__device__ __forceinline__ void umma_f8_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// MMA completion signal: arrive on the mbarrier at the same shared offset in
// every CTA of `mask` once all tcgen05 ops issued so far by this thread have
// completed (a tcgen05.commit, which moves no data).
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar, uint16_t mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;\n" ::"r"(
          smem_addr(bar)),
      "h"(mask)
      : "memory");
}

// 2-D tile load into this CTA's shared memory; the transferred bytes are
// counted on the mbarrier at shared::cluster address `bar_cluster`, which may
// be the pair leader's barrier.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, "
      "%4}], [%2];\n" ::"r"(smem_addr(dst)),
      "l"(map), "r"(bar_cluster), "r"(c0), "r"(c1)
      : "memory");
}

// L2 eviction policy for one access (PTX `createpolicy`): code 1 keeps the
// lines (evict_last), 2 lets them go first (evict_first), 0 is evict_normal.
__device__ __forceinline__ uint64_t l2_policy(int code) {
  uint64_t p;
  if (code == 1)
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;\n" : "=l"(p));
  else if (code == 2)
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;\n" : "=l"(p));
  else
    asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;\n" : "=l"(p));
  return p;
}

// tma_load_2d_pair with an L2 cache policy
__device__ __forceinline__ void tma_load_2d_pair_hint(void* dst, const CUtensorMap* map, uint32_t bar_cluster,
                                                      int c0, int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint "
      "[%0], [%1, {%3, %4}], [%2], %5;\n" ::"r"(smem_addr(dst)),
      "l"(map), "r"(bar_cluster), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// MN-major operand tile (128-byte swizzle): 64 MN elements (128 B) per row,
// rows along K, 8-row swizzle atoms 1024 B apart (SBO), 64-wide MN slabs
// `lbo` bytes apart (LBO).
__device__ __forceinline__ uint64_t sw128_mnmajor_desc(uint32_t saddr, uint32_t lbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// kind::f16 instruction descriptor with operand majorness: bit 15 = A is
// MN-major, bit 16 = B is MN-major.
__host__ __device__ constexpr uint32_t idesc_bf16_f32_major(int M, int N, bool a_mn, bool b_mn) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}


// try_wait with a suspend-time hint (ns): a waiting warp sleeps until the
// phase completes or the hint expires, instead of re-polling every short
// system-defined window
__device__ __forceinline__ bool mbar_try_wait_hint(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// bounded wait (see tc::mbar_wait) that sleeps between polls when hint_ns > 0
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, volatile int* err, int code,
                                                uint32_t hint_ns) {
  if (hint_ns == 0) return tc::mbar_wait(bar, parity, err, code);
  const long long t0 = clock64();
  while (!mbar_try_wait_hint(bar, parity, hint_ns)) {
    if (*err != tc::kErrNone) return false;
    if (clock64() - t0 > tc::kWaitCycles) {
      *err = code;
      return false;
    }
  }
  return true;
}

// ---- epilogue: TMA bulk stores from shared memory --------------------------------
// tcgen05.ld without the wait (issue several, then one tcgen05.wait::ld)
__device__ __forceinline__ void tmem_ld32_nowait(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,"
      "%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;\n" ::: "memory"); }

// generic-proxy shared-memory writes -> visible to the TMA (async proxy)
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;\n" ::: "memory");
}

// 2-D tile store shared -> global (rows / columns outside the tensor are
// clipped by the TMA unit)
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];\n" ::"l"(map),
               "r"(smem_addr(src)), "r"(c0), "r"(c1)
               : "memory");
}

// 2-D tile element-wise add into global memory (fp32), performed in L2
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.bulk_group [%0, {%2, %3}], [%1];\n" ::"l"(
                   map),
               "r"(smem_addr(src)), "r"(c0), "r"(c1)
               : "memory");
}

// tma_store_2d / tma_reduce_add_2d with an L2 cache policy
__device__ __forceinline__ void tma_store_2d_hint(const CUtensorMap* map, const void* src, int c0, int c1,
                                                  uint64_t policy) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;\n"
               ::"l"(map), "r"(smem_addr(src)), "r"(c0), "r"(c1), "l"(policy)
               : "memory");
}

__device__ __forceinline__ void tma_reduce_add_2d_hint(const CUtensorMap* map, const void* src, int c0, int c1,
                                                       uint64_t policy) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], "
      "%4;\n" ::"l"(map),
      "r"(smem_addr(src)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;\n" ::: "memory"); }

// at most N of this thread's bulk groups still read their shared-memory source
template <int N>
__device__ __forceinline__ void bulk_wait_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;\n" ::"n"(N) : "memory");
}

// all of this thread's bulk groups complete
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;\n" ::: "memory"); }

}  // namespace tc2
}  // namespace lrl
