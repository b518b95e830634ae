// Inline-PTX building blocks for sm_100a: mbarriers, cp.async / bulk copies, tcgen05
// (TMEM allocation, UMMA issue, commit, TMEM loads) and the device error flag.
//
// UMMA operand descriptors follow the sm_100 shared-memory descriptor format: start address,
// leading-dimension byte offset (LBO) and stride-dimension byte offset (SBO), all >> 4,
// version 1 in bits 46-47, layout type in bits 61-63 (0 = no swizzle). For K-major operands
// without swizzle the canonical layout is ((8 rows, n), 2 K-halves) : ((16 B, SBO), LBO):
// a "core matrix" is 8 rows of 16 contiguous bytes; SBO steps to the next 8 rows and LBO to
// the next 16 bytes of K.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>

namespace ixb {

// Error bits of the device flag.
enum : unsigned { DEV_ERR_WAIT_TIMEOUT = 1u, DEV_ERR_BAD_ARGS = 2u };

// A bounded wait gives up after this many nanoseconds of %globaltimer: seconds, far above any
// legitimate wait in these kernels.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
// Suspend hint (ns) for mbarrier.try_wait: a waiting warp sleeps instead of spinning on issue
// slots the working warps need; the phase completing wakes it.
constexpr uint32_t kSuspendHintNs = 20000;

// The library is one translation unit (ixb_api.cu includes every kernel header), so the
// flag is defined here; the host reads and clears it with cudaMemcpyFromSymbol.
__device__ unsigned int g_dev_error = 0;

__device__ __forceinline__ void set_dev_error(unsigned bits) { atomicOr(&g_dev_error, bits); }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// True in exactly one active lane of the (converged) warp.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred = 0;
  asm volatile(
      "{\n\t.reg .pred P1;\n\t"
      "elect.sync _|P1, 0xffffffff;\n\t"
      "selp.b32 %0, 1, 0, P1;\n\t}"
      : "+r"(pred));
  return pred != 0;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(kSuspendHintNs)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ unsigned long long global_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}
__device__ __forceinline__ bool wait_timed_out() {
  return (*reinterpret_cast<volatile unsigned int*>(&g_dev_error) & DEV_ERR_WAIT_TIMEOUT) != 0;
}
// Bounded wait: returns false (and raises the device flag) if the phase never completes. Once any
// wait has timed out, later waits give up at once, so a stuck launch ends after one time limit.
// The clock and the flag (a global load) are checked every 16th retry only, so a warp that keeps
// retrying costs the working warps few issue slots and no memory traffic.
__device__ __forceinline__ bool mbar_wait_for(uint64_t* bar, uint32_t parity, unsigned long long limit_ns) {
  if (mbar_try_wait(bar, parity)) return true;
  const unsigned long long t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((i & 15) == 0 && (global_ns() - t0 > limit_ns || wait_timed_out())) break;
  }
  set_dev_error(DEV_ERR_WAIT_TIMEOUT);
  return false;
}
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
  return mbar_wait_for(bar, parity, kWaitLimitNs);
}

// ---------------------------------------------------------------- programmatic dependent launch
// The kernels of one network step are launched so that each may start while the previous one
// drains: a kernel sets up (shared memory, TMEM, barriers, constant loads) and then waits here
// until the previous grid has completed and its writes are visible, before it touches any
// activation. Without the launch attribute the wait returns at once.
__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel in the stream begin its setup once every CTA of this grid has started.
__device__ __forceinline__ void grid_dep_launch() { asm volatile("griddepcontrol.launch_dependents;" :::); }

// ---------------------------------------------------------------- copies
// 16-byte global -> shared copy; src_bytes 0 zero-fills the destination.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
__device__ __forceinline__ void cp_async8(void* dst, const void* src, uint32_t src_bytes) {
  asm volatile("cp.async.ca.shared.global [%0], [%1], 8, %2;" ::"r"(smem_u32(dst)), "l"(src), "r"(src_bytes)
               : "memory");
}
// Arrive on bar once every cp.async this thread issued before has completed; the arrival is
// one of the barrier's expected arrivals (no pending-count increment).
__device__ __forceinline__ void cp_async_mbar_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}
// Order this thread's generic-proxy shared-memory writes before async-proxy reads (UMMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// Bulk (TMA engine, non-tensor) copy global -> shared, completing tx bytes on bar.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Thread-block clusters: this CTA's rank, the shared::cluster address of a shared-memory location
// in CTA `rank`, stores there, and a barrier over every thread of the cluster (release / acquire:
// the shared-memory writes of each CTA before it are visible to all after it).
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ uint32_t cluster_addr(const void* p, uint32_t rank) {
  uint32_t a;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(a) : "r"(smem_u32(p)), "r"(rank));
  return a;
}
__device__ __forceinline__ void st_cluster_u8(uint32_t a, uint32_t v) {
  asm volatile("st.shared::cluster.u8 [%0], %1;" ::"r"(a), "h"((unsigned short)v) : "memory");
}
__device__ __forceinline__ void st_cluster_u16(uint32_t a, uint32_t v) {
  asm volatile("st.shared::cluster.u16 [%0], %1;" ::"r"(a), "h"((unsigned short)v) : "memory");
}
__device__ __forceinline__ void st_cluster_u32(uint32_t a, uint32_t v) {
  asm volatile("st.shared::cluster.u32 [%0], %1;" ::"r"(a), "r"(v) : "memory");
}
__device__ __forceinline__ void st_cluster_f4(uint32_t a, float4 v) {
  asm volatile("st.shared::cluster.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(a), "f"(v.x), "f"(v.y), "f"(v.z), "f"(v.w)
               : "memory");
}
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// A hint that brings `bytes` (a multiple of 16, 16-byte aligned) of global memory into the L2.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(cols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(cols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// K-major, no-swizzle UMMA shared-memory descriptor.
__device__ __forceinline__ uint64_t umma_desc(uint32_t saddr, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for sm_100
  return d;                // base offset 0, legacy LBO mode, layout type 0 (no swizzle)
}

// Instruction descriptor of tcgen05.mma kind::i8: s8 x s8 -> s32, both K-major.
__host__ __device__ constexpr uint32_t umma_idesc_s8(int m, int n) {
  return (2u << 4)                          // D format: S32
         | (1u << 7)                        // A format: signed 8-bit
         | (1u << 10)                       // B format: signed 8-bit
         | ((uint32_t)(n >> 3) << 17)       // N / 8
         | ((uint32_t)(m >> 4) << 24);      // M / 16
}
// The same with an unsigned 8-bit A (A format 0): u8 x s8 -> s32.
__host__ __device__ constexpr uint32_t umma_idesc_u8s8(int m, int n) { return umma_idesc_s8(m, n) & ~(7u << 7); }

// D[tmem] (+)= A[smem] * B[smem]^T, issued by one thread.
__device__ __forceinline__ void umma_s8(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on bar once every tcgen05 op this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}
// 32 lanes x 16 consecutive 32-bit columns: thread i of the warp gets lane (base lane + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
        "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
// 32 lanes x 16 consecutive 32-bit columns set to zero (thread i writes lane base + i).
__device__ __forceinline__ void tmem_zero16(uint32_t taddr) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1,%1};" ::"r"(taddr), "r"(0u)
      : "memory");
}
// 16 columns of this warp's 32 TMEM lanes set to b[0..15] (the same 16 values in every lane).
__device__ __forceinline__ void tmem_fill16(uint32_t taddr, const int4* b) {
  const int4 a0 = b[0], a1 = b[1], a2 = b[2], a3 = b[3];
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(a0.x), "r"(a0.y), "r"(a0.z), "r"(a0.w), "r"(a1.x), "r"(a1.y), "r"(a1.z), "r"(a1.w), "r"(a2.x), "r"(a2.y),
      "r"(a2.z), "r"(a2.w), "r"(a3.x), "r"(a3.y), "r"(a3.z), "r"(a3.w)
      : "memory");
}
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- integer helpers
// n / d for 0 <= n < 2^31 by a multiply: m = floor(2^32 (2^s - d) / d) + 1, s = ceil(log2 d),
// q = (umulhi(n, m) + n) >> s (division by invariant integers, Granlund & Montgomery 1994).
struct FastDiv {
  uint32_t d, m, s;
};
__host__ __device__ inline FastDiv make_fastdiv(uint32_t d) {
  uint32_t s = 0;
  while ((1ull << s) < d) ++s;
  const uint32_t m = (uint32_t)((((1ull << 32) * ((1ull << s) - d)) / d) + 1);
  return FastDiv{d, m, s};
}
__device__ __forceinline__ uint32_t fdiv(uint32_t n, const FastDiv& f) { return (__umulhi(n, f.m) + n) >> f.s; }

// ---------------------------------------------------------------- integer epilogue
// Arithmetic shift right by s (0..30) rounding half to even; s <= 0 shifts left.
__device__ __forceinline__ int rne_shift(int x, int s) {
  if (s <= 0) return x << (-s);
  int q = x >> s;
  int r = x - (q << s);
  int h = 1 << (s - 1);
  return q + ((r > h) | ((r == h) & (q & 1)));
}
__device__ __forceinline__ int clamp_i8(int x) { return min(max(x, -128), 127); }
__device__ __forceinline__ int add_sat(int a, int b) {
  int d;
  asm("add.sat.s32 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
  return d;
}

}  // namespace ixb
