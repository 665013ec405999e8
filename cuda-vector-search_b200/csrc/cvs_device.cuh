// Device-side building blocks for the sm_100a search kernels: mbarriers with
// bounded waits, TMA tile loads, tcgen05 (TMEM allocation, MMA issue, commit,
// TMEM loads) and the shared-memory matrix descriptor.
//
// Every wait in this file gives up after kWaitCycles SM clocks (about a second),
// records a code in the kernel's device error word and returns false, so a
// broken pipeline surfaces as CVS_ERR_DEVICE_TIMEOUT on the host instead of a
// hung GPU.
#pragma once

#include <cuda_fp16.h>
#include <cstdint>

namespace cvs {

constexpr long long kWaitCycles = 2000000000LL;  // ~1 s at 1.9 GHz

// Device error word codes (or-ed with a small site id in the low byte).
constexpr int kErrTimeout = 0x100;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void report_error(int* err, int code) {
  if (err != nullptr) atomicCAS(err, 0, code);
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile(
      "{ .reg .b64 st;\n\t"
      "mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile(
      "{ .reg .b64 st;\n\t"
      "mbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1; }" ::"r"(smem_u32(bar)),
      "r"(bytes)
      : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the waiting thread is parked until the
// phase completes or about `ns` nanoseconds pass, instead of re-issuing the
// polling loop (the single-thread producer and MMA loops otherwise spend issue
// slots, shared with the drain warps of their sub-partition, on spinning).
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

constexpr uint32_t kSuspendNs = 1000000;  // per try_wait; the overall wait stays bounded by kWaitCycles

// Waits for the phase with the given parity to complete. Returns false (after
// recording kErrTimeout|site in *err and raising *abort) if it does not complete
// within kWaitCycles, or if another role already raised *abort.
// `limit` (SM clocks) is kWaitCycles except where a test shortens it.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort,
                                          int* err, int site, long long limit = kWaitCycles) {
  if (mbar_try_wait(bar, parity)) return true;
  const long long t0 = clock64();
  while (true) {
    if (mbar_try_wait_suspend(bar, parity, kSuspendNs)) return true;
    if (*abort) return false;
    if (clock64() - t0 > limit) {
      *abort = 1;
      report_error(err, kErrTimeout | site);
      return false;
    }
  }
}

// Bounded wait that ignores the abort flag; used only to drain work that was
// already issued before leaving on an error path.
__device__ __forceinline__ void mbar_wait_drain(uint64_t* bar, uint32_t parity) {
  const long long t0 = clock64();
  while (!mbar_try_wait_suspend(bar, parity, kSuspendNs)) {
    if (clock64() - t0 > kWaitCycles) return;
  }
}

// ---------------------------------------------------------------------------
// Programmatic dependent launch
// ---------------------------------------------------------------------------
// Blocks until the grids this one depends on (the previous kernel on the
// stream, when launched with programmatic stream serialisation) have completed
// and their memory is visible; a no-op for an ordinary launch.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
// Lets the next kernel on the stream (if launched programmatically) start its
// prologue; it still waits for this grid's results with grid_dependency_wait.
__device__ __forceinline__ void grid_launch_dependents() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---------------------------------------------------------------------------
// TMA (tiled tensor copies global -> shared, completion on an mbarrier)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tma_prefetch_desc(const void* desc) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(desc)) : "memory");
}

__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

// 2-D tile load: box origin (x = inner/column coordinate, y = row coordinate).
// x * 2 bytes must be a multiple of 16 (all callers pass multiples of 64 halves).
__device__ __forceinline__ void tma_load_2d(void* smem_dst, const void* desc, uint64_t* bar, int x,
                                            int y, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(smem_u32(bar)), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// 2-D tile load into this CTA's shared memory whose completion is counted on an
// mbarrier of the even CTA of a tcgen05 CTA pair (bar_cluster: a shared::cluster
// address obtained with map_to_rank). No multicast: one destination CTA.
__device__ __forceinline__ void tma_load_2d_to_pair_bar(void* smem_dst, const void* desc,
                                                        uint32_t bar_cluster, int x, int y,
                                                        uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(desc)), "r"(bar_cluster), "r"(x), "r"(y), "l"(policy)
      : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05: tensor memory, MMA, commit, loads
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, fp16 inputs, fp32 accumulate, one CTA.
__device__ __forceinline__ void tc_mma_f16(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives (once) on the mbarrier when every tcgen05.mma issued so far by this
// thread has completed.
__device__ __forceinline__ void tc_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread i of the warp receives TMEM
// lane (base lane + i), columns [col, col + 32).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the
// 128-byte swizzle: rows of 128 bytes (64 halves), 8-row groups 1024 bytes
// apart. The tile base must be 1024-byte aligned; a K offset inside the
// 128-byte row is applied by adding (bytes >> 4) to the start address field.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);          // start address  [0,14)
  d |= static_cast<uint64_t>(1u) << 16;                          // LBO (unused)   [16,30)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;                  // SBO = 1024 B   [32,46)
  d |= static_cast<uint64_t>(1u) << 46;                          // sm100 version  [46,48)
  d |= static_cast<uint64_t>(2u) << 61;                          // SWIZZLE_128B   [61,64)
  return d;
}

// Instruction descriptor, kind::f16: fp16 A/B, fp32 D, both K-major.
__host__ __device__ constexpr uint32_t idesc_f16_f32(int m, int n) {
  return (1u << 4)                                    // D format: f32
         | (0u << 7) | (0u << 10)                     // A, B: f16
         | (static_cast<uint32_t>(n >> 3) << 17)      // N >> 3
         | (static_cast<uint32_t>(m >> 4) << 24);     // M >> 4
}

// ---------------------------------------------------------------------------
// Clusters and CTA pairs (tcgen05 cta_group::2)
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// Every thread of both CTAs of the cluster arrives and waits.
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile(
      "barrier.cluster.arrive.release.aligned;\n\t"
      "barrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Shared::cluster address of the same shared variable in CTA `rank`.
__device__ __forceinline__ uint32_t map_to_rank(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

// Arrive on an mbarrier of another CTA of the cluster. Release at CTA scope
// only: the one use is "this CTA's drain warps have read the accumulator"
// (their tcgen05.ld completed, tcgen05.wait::ld, before the arrive), an
// execution order the partner's MMA thread needs, not the visibility of this
// thread's memory writes at cluster scope -- waiting for those (the candidate
// appends in flight to global memory) made every arrive cost a round trip.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.release.cta.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
               : "memory");
}

__device__ __forceinline__ void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                   smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}

__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
               : "memory");
}

// Pair MMA, issued by one thread of the even CTA: A rows 0-127 and B rows
// 0..N/2-1 come from this CTA's shared memory, A rows 128-255 and the other
// half of B from the odd CTA's shared memory at the same offsets; each CTA's
// TMEM receives its 128 rows of D.
__device__ __forceinline__ void tc_mma_f16_pair(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc,
                                                uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrives once on the mbarrier at this offset in every CTA of cta_mask when all
// pair MMAs issued so far by this thread have completed.
__device__ __forceinline__ void tc_commit_pair(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

__device__ __forceinline__ uint32_t elect_one_lane() {
  uint32_t pred = 0;
  asm volatile(
      "{ .reg .b32 r;\n\t .reg .pred p;\n\t"
      "elect.sync r|p, 0xffffffff;\n\t"
      "selp.u32 %0, 1, 0, p; }"
      : "=r"(pred));
  return pred;
}

// ---------------------------------------------------------------------------
// Ordered 64-bit keys. A candidate (score, row) maps to a key such that a larger
// key ranks first: higher score first, then the smaller row id. Keys of
// distinct rows are distinct, so "top-k" over keys has no ties. Key 0 ranks
// after every real candidate and marks an empty slot.
// ---------------------------------------------------------------------------
__host__ __device__ __forceinline__ uint32_t ordered_bits(float s) {
#ifdef __CUDA_ARCH__
  const uint32_t u = __float_as_uint(s);
#else
  uint32_t u;
  __builtin_memcpy(&u, &s, 4);
#endif
  return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

__host__ __device__ __forceinline__ float score_of_bits(uint32_t o) {
  const uint32_t u = (o & 0x80000000u) ? (o & 0x7FFFFFFFu) : ~o;
#ifdef __CUDA_ARCH__
  return __uint_as_float(u);
#else
  float f;
  __builtin_memcpy(&f, &u, 4);
  return f;
#endif
}

__host__ __device__ __forceinline__ uint64_t make_key(float s, uint32_t row) {
  return (static_cast<uint64_t>(ordered_bits(s)) << 32) | static_cast<uint64_t>(~row);
}

__host__ __device__ __forceinline__ float key_score(uint64_t key) {
  return score_of_bits(static_cast<uint32_t>(key >> 32));
}

__host__ __device__ __forceinline__ uint32_t key_row(uint64_t key) {
  return ~static_cast<uint32_t>(key);
}

}  // namespace cvs
