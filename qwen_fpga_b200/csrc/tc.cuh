// sm_100a primitives of the batched engine (batch.cu): mbarriers, bulk
// copies, tcgen05 MMA / TMEM, bounded waits.  Everything is inline PTX from
// the public PTX ISA; no multicast form is used anywhere.
#pragma once
#include <cstdint>

#include <cuda_runtime.h>

namespace qb {
namespace tc {

constexpr unsigned long long WAIT_NS = 2000000000ull;   // every device wait ends after 2 s

__device__ __forceinline__ unsigned smem_u32(const void* p) { return (unsigned)__cvta_generic_to_shared(p); }
__device__ __forceinline__ unsigned long long gtime() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---- mbarriers
__device__ __forceinline__ void mbar_init(unsigned bar, unsigned count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" :: "r"(bar), "r"(count) : "memory");
}
__device__ __forceinline__ void mbar_init_fence() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
__device__ __forceinline__ bool mbar_try(unsigned bar, unsigned parity) {
  unsigned ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok) : "r"(bar), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ void mbar_arrive(unsigned bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" :: "r"(bar) : "memory");
}
__device__ __forceinline__ void mbar_expect(unsigned bar, unsigned bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" :: "r"(bar), "r"(bytes) : "memory");
}
// try_wait that may suspend the thread (up to the hint, in ns) until the
// phase completes: waiting threads take no issue slots from the SM's others
__device__ __forceinline__ bool mbar_try_sleep(unsigned bar, unsigned parity) {
  unsigned ok;
  asm volatile("{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3; selp.u32 %0, 1, 0, p; }"
               : "=r"(ok) : "r"(bar), "r"(parity), "r"(100000u) : "memory");
  return ok != 0;
}
// Bounded wait for phase `parity` (one thread or many).  On time-out the
// first error wins into err[0..2] = {ERR_WAIT, site, value}; returns false.
__device__ __forceinline__ bool mbar_wait(unsigned bar, unsigned parity, int* err, int site, int value) {
  if (mbar_try(bar, parity)) return true;
  const unsigned long long t0 = gtime();
  while (!mbar_try_sleep(bar, parity)) {
    if (gtime() - t0 > WAIT_NS) {
      if (atomicCAS(err, 0, 3) == 0) { err[1] = site; err[2] = value; }
      return false;
    }
  }
  return true;
}

// ---- bulk copies (global -> shared, completion on an mbarrier); 16-byte
// aligned addresses, size a multiple of 16
__device__ __forceinline__ unsigned long long policy_evict_first() {
  unsigned long long p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ unsigned long long policy_evict_last() {
  unsigned long long p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void bulk_g2s(unsigned dst, const void* src, unsigned bytes, unsigned bar,
                                         unsigned long long pol) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;"
               :: "r"(dst), "l"(src), "r"(bytes), "r"(bar), "l"(pol) : "memory");
}

// ---- tcgen05
// Shared-memory matrix descriptor, canonical K-major layout without swizzle:
// start address, leading byte offset (between the two 16-byte core-matrix
// columns of one K = 32 step), stride byte offset (between 8-row groups),
// descriptor version 1.
__device__ __forceinline__ unsigned long long desc(unsigned addr, unsigned lbo, unsigned sbo) {
  return (unsigned long long)((addr >> 4) & 0x3fffu) | (unsigned long long)((lbo >> 4) & 0x3fffu) << 16 |
         (unsigned long long)((sbo >> 4) & 0x3fffu) << 32 | 1ull << 46;
}
// Instruction descriptor of kind::i8: s32 accumulators, signed int8 A and B,
// both K-major, N columns, M rows.
__host__ __device__ constexpr unsigned idesc_i8(int M, int N) {
  return (2u << 4) | (1u << 7) | (1u << 10) | ((unsigned)(N >> 3) << 17) | ((unsigned)(M >> 4) << 24);
}
// D[tmem] (+)= A[M x 32] * B[N x 32]^T, one int8 K-step; issued by one thread.
__device__ __forceinline__ void mma_i8(unsigned tmem, unsigned long long a, unsigned long long b, unsigned idesc,
                                       unsigned accumulate) {
  asm volatile("{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
               "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}"
               :: "r"(tmem), "l"(a), "l"(b), "r"(idesc), "r"(accumulate) : "memory");
}
// Arrive (once) on an mbarrier when every tcgen05 op this thread issued so far has completed.
__device__ __forceinline__ void commit(unsigned bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               :: "r"(bar) : "memory");
}
__device__ __forceinline__ void fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// generic-proxy shared-memory writes -> visible to the async proxy (tensor core, bulk copies)
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

// TMEM allocation by one whole warp; the base address lands in *slot (smem).
template <int NCOLS>
__device__ __forceinline__ void tmem_alloc(unsigned* slot) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
               :: "r"(smem_u32(slot)), "n"(NCOLS) : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
template <int NCOLS>
__device__ __forceinline__ void tmem_free(unsigned base) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" :: "r"(base), "n"(NCOLS) : "memory");
}
// 16 consecutive 32-bit TMEM columns of this warp's 32 lanes (lane = row).
__device__ __forceinline__ void tmem_ld16(unsigned addr, unsigned (&r)[16]) {
  asm volatile("tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
               : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
                 "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
               : "r"(addr) : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }

// ---- thread-block clusters (distributed shared memory)
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
__device__ __forceinline__ unsigned cluster_ctarank() {
  unsigned r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// The address of `addr` (this CTA's shared memory) in CTA `rank` of the cluster.
__device__ __forceinline__ unsigned mapa(unsigned addr, unsigned rank) {
  unsigned r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
__device__ __forceinline__ int ld_dsmem(unsigned addr) {
  int v;
  asm volatile("ld.shared::cluster.u32 %0, [%1];" : "=r"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ int4 ld_dsmem_v4(unsigned addr) {
  int4 v;
  asm volatile("ld.shared::cluster.v4.u32 {%0,%1,%2,%3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

// ---- programmatic dependent launch (no-ops for a launch without the attribute)
__device__ __forceinline__ void grid_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void grid_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

}  // namespace tc
}  // namespace qb
