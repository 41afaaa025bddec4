// Shared device helpers for the B200 (sm_100a) MXFP4/INT8 MoE kernels:
// status reporting, bounded mbarrier waits, bulk async copies, tcgen05
// (TMEM alloc / MMA / commit / load) and the MXFP4 -> INT8 nibble decode.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#include "dsv4_b200.h"

namespace dsv4 {

// ---------------------------------------------------------------------------
// Device-side status word.  A kernel that gives up on a wait records a code
// here (first writer wins) and runs to completion with garbage output instead
// of hanging the GPU; the host reads it with dsv4_b200_get_device_status().
// ---------------------------------------------------------------------------
// Defined here: the library is a single translation unit (dsv4_b200.cu).
__device__ int g_device_status = 0;

enum DeviceErr : int {
  kErrNone = 0,
  kErrWaitPackedFull = 0x101,
  kErrWaitAbEmpty = 0x102,
  kErrWaitAbFull = 0x103,
  kErrWaitAccFull = 0x104,
  kErrWaitPackedEmpty = 0x105,
  kErrWaitMeta = 0x106,
  kErrWaitAccEmpty = 0x107,
};

// Wait budget: ~2 s of %globaltimer per wait.
constexpr unsigned long long kWaitBudgetNs = 2000000000ull;

__device__ __forceinline__ unsigned long long globaltimer_ns() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void record_error(int code) {
  atomicCAS(&g_device_status, 0, code);
}

__device__ __forceinline__ bool device_error_pending() {
  return *reinterpret_cast<volatile int*>(&g_device_status) != 0;
}

// Optional pipeline timeline (compile with -DDSV4_TRACE; debug builds only):
// CTA 0 records clock64 at each hand-off of the first kTraceStages stages.
#ifdef DSV4_TRACE
constexpr int kTraceStages = 1024;
constexpr int kTraceEvents = 14;
__device__ long long g_trace[kTraceEvents][kTraceStages];
#define DSV4_TRACE_EV(ev, idx)                                                   \
  do {                                                                           \
    if (blockIdx.x == 0 && (idx) < kTraceStages) g_trace[ev][idx] = clock64();   \
  } while (0)
#else
#define DSV4_TRACE_EV(ev, idx) \
  do {                         \
  } while (0)
#endif

// Programmatic dependent launch: a kernel launched with programmatic stream
// serialisation may start before its predecessor in the stream finishes.
// pdl_entry() lets the next kernel in the stream be scheduled early and then
// waits until every predecessor has completed and its memory is visible, so
// it must run before the kernel's first global-memory access.  Without that
// launch attribute both instructions do nothing.
__device__ __forceinline__ void pdl_entry() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---------------------------------------------------------------------------
// mbarrier
// ---------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_fence_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

// try_wait with a suspend-time hint: a thread whose phase is not complete is
// parked (issuing nothing) until the phase completes or ~hint ns pass, so
// waiting warps do not steal issue slots from the decode warps.
constexpr uint32_t kWaitSuspendHintNs = 100000u;

__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kWaitSuspendHintNs)
      : "memory");
  return ok != 0;
}

// Non-blocking probe of a phase.
__device__ __forceinline__ bool mbar_test_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait: returns false (and records `code`) when the budget runs out
// or another wait in the grid already failed.
__device__ __forceinline__ bool mbar_wait(uint32_t bar, uint32_t parity, int code) {
  // a completed phase is seen by the non-blocking probe much sooner than by
  // try_wait, whose latency is ~245 cycles even when the phase is complete
  if (mbar_test_wait(bar, parity)) return true;
  if (mbar_try_wait(bar, parity)) return true;
  unsigned long long t0 = globaltimer_ns();
  uint32_t n = 0;
  while (!mbar_try_wait(bar, parity)) {
    if ((++n & 7u) == 0) {
      if (device_error_pending()) return false;
      if (globaltimer_ns() - t0 > kWaitBudgetNs) {
        record_error(code);
        return false;
      }
    }
  }
  return true;
}

// Cluster-scope forms for the CTA pair of a 2-SM MMA: barriers that the peer
// CTA arrives on (or that a pair commit signals) are waited on with
// acquire.cluster, remote arrivals release at cluster scope.
__device__ __forceinline__ bool mbar_try_wait_cl(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(kWaitSuspendHintNs)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_test_wait_cl(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Bounded wait, cluster scope (same budget and error recording as mbar_wait).
__device__ __forceinline__ bool mbar_wait_cl(uint32_t bar, uint32_t parity, int code) {
  if (mbar_test_wait_cl(bar, parity)) return true;
  if (mbar_try_wait_cl(bar, parity)) return true;
  unsigned long long t0 = globaltimer_ns();
  uint32_t n = 0;
  while (!mbar_try_wait_cl(bar, parity)) {
    if ((++n & 7u) == 0) {
      if (device_error_pending()) return false;
      if (globaltimer_ns() - t0 > kWaitBudgetNs) {
        record_error(code);
        return false;
      }
    }
  }
  return true;
}

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

// shared::cta address -> the shared::cluster address of the same offset in
// CTA `rank` of the cluster
__device__ __forceinline__ uint32_t mapa_shared(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}

// arrive on a barrier given by its shared::cluster address (this CTA's or the peer's)
__device__ __forceinline__ void mbar_arrive_cl(uint32_t cl_bar) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cl_bar)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx_cl(uint32_t cl_bar, uint32_t bytes) {
  asm volatile(
      "mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(cl_bar),
      "r"(bytes)
      : "memory");
}

// all threads of both CTAs of the cluster
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;"
               ::: "memory");
}

// ---------------------------------------------------------------------------
// Bulk async copies (TMA engine, untiled and tiled)
// ---------------------------------------------------------------------------
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

// global -> shared bulk copy; dst/src 16-byte aligned, bytes % 16 == 0.
__device__ __forceinline__ void bulk_g2s(uint32_t dst, const void* src, uint32_t bytes,
                                         uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1], %2, [%3], %4;" ::"r"(dst),
      "l"(src), "r"(bytes), "r"(bar), "l"(policy)
      : "memory");
}

// Tiled tensor-map (TMA) loads, no multicast, completion on an mbarrier.
// The shared-memory destination must be 128-byte aligned.
__device__ __forceinline__ void tma_load_3d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(bar), "l"(policy)
      : "memory");
}

// 3-D tile load of one CTA of a 2-SM pair: the bytes land in this CTA's
// shared memory and complete on the barrier at shared::cluster address
// `cl_bar` (the pair leader's).  Not a multicast load.
__device__ __forceinline__ void tma_load_3d_pair(uint32_t dst, const CUtensorMap* map, int c0,
                                                 int c1, int c2, uint32_t cl_bar,
                                                 uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(cl_bar), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            int c2, int c3, uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_2d(uint32_t dst, const CUtensorMap* map, int c0, int c1,
                                            uint32_t bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3}], [%4], %5;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(bar), "l"(policy)
      : "memory");
}

// Row gather: 4 rows (arbitrary row coordinates, out-of-range -> zeros) of a
// 2-D tensor map whose box is 1 row high, written as 4 consecutive box rows.
__device__ __forceinline__ void tma_gather4(uint32_t dst, const CUtensorMap* map, int x, int r0,
                                            int r1, int r2, int r3, uint32_t bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile::gather4.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(r0), "r"(r1), "r"(r2), "r"(r3), "r"(bar),
      "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Make generic-proxy shared-memory writes visible to the async proxy
// (tcgen05.mma operand reads).
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void named_bar_sync(int id, int threads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

// ---------------------------------------------------------------------------
// tcgen05 (5th-gen tensor core, TMEM accumulators)
// ---------------------------------------------------------------------------
__device__ __forceinline__ void tmem_alloc(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
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

// TMEM allocation for a 2-SM pair: the same warp index of both CTAs issues it.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(dst_smem),
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

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[tmem] * B[smem]^T: A (M=128 lanes x K int8, K-major,
// 4 int8 per 32-bit column) read from tensor memory.
__device__ __forceinline__ void mma_i8_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                          uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns per thread, registers -> TMEM.
__device__ __forceinline__ void tmem_st_x16(uint32_t taddr, const uint32_t (&v)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
      "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

// 32 lanes x 32 bits, 8 consecutive columns per thread, registers -> TMEM.
__device__ __forceinline__ void tmem_st_x8(uint32_t taddr, const uint32_t (&v)[8]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x8.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8};" ::"r"(taddr),
      "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7])
      : "memory");
}

// 32 lanes x 32 bits, 8 consecutive columns per thread, TMEM -> registers.
__device__ __forceinline__ void tmem_ld_x8(uint32_t taddr, uint32_t (&v)[8]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x8.b32 {%0,%1,%2,%3,%4,%5,%6,%7}, [%8];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7])
      : "r"(taddr)
      : "memory");
}

// tcgen05.wait::ld tied to the 8 destination registers of a load issued ahead.
__device__ __forceinline__ void tmem_ld_wait_regs8(uint32_t (&v)[8]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]),
                 "+r"(v[6]), "+r"(v[7])
               :
               : "memory");
}

__device__ __forceinline__ void tmem_st_wait() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 2-SM MMA (cta_group::2, issued by the pair leader): A from TMEM (each CTA
// holds its M/2 rows at the same column address), B from shared memory (each
// CTA holds N/2 rows at the same offset), D in each CTA's TMEM.
__device__ __forceinline__ void mma_i8_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc,
                                               uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on the barrier at shared::cluster address `cl_bar` (either CTA of the
// pair) once all pair MMAs issued so far by this thread complete.
__device__ __forceinline__ void mma_commit_pair(uint32_t cl_bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(cl_bar)
      : "memory");
}

// Arrive on `bar` once all tcgen05.mma issued so far by this thread complete.
__device__ __forceinline__ void mma_commit(uint32_t bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(bar)
      : "memory");
}

// 32 lanes x 32 bits, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld_x16(uint32_t taddr, int32_t (&v)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15])
      : "r"(taddr)
      : "memory");
}

// 32 lanes x 32 bits, 32 consecutive columns per thread, waited on at once.
__device__ __forceinline__ void tmem_ld_x32_wait(uint32_t taddr, int32_t (&v)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]),
        "=r"(v[7]), "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]),
        "=r"(v[14]), "=r"(v[15]), "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]),
        "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]), "=r"(v[24]), "=r"(v[25]),
        "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
      : "r"(taddr)
      : "memory");
}

__device__ __forceinline__ void tmem_ld_wait() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Wait for outstanding tcgen05.ld with the destination registers tied to the
// wait, so no use of them can be scheduled above it (for loads issued ahead).
__device__ __forceinline__ void tmem_ld_wait_regs(int32_t (&v)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(v[0]), "+r"(v[1]), "+r"(v[2]), "+r"(v[3]), "+r"(v[4]), "+r"(v[5]),
                 "+r"(v[6]), "+r"(v[7]), "+r"(v[8]), "+r"(v[9]), "+r"(v[10]), "+r"(v[11]),
                 "+r"(v[12]), "+r"(v[13]), "+r"(v[14]), "+r"(v[15])
               :
               : "memory");
}

// Shared-memory matrix descriptor, K-major, 128-byte swizzle: 8-row atoms of
// 8 x 128 B stacked every 1024 B (stride byte offset), version 1, layout
// SWIZZLE_128B (2).  Start address must be 1024-aligned apart from the
// in-row K offset (0/32/64/96 B), which the hardware folds into the swizzle.
__device__ __forceinline__ uint64_t smem_desc_sw128(uint32_t saddr) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4);   // start address
  d |= static_cast<uint64_t>(1u) << 16;                   // LBO (unused for SW128 K-major)
  d |= static_cast<uint64_t>(1024u >> 4) << 32;           // SBO = 1024 B
  d |= static_cast<uint64_t>(1u) << 46;                   // descriptor version (sm100)
  d |= static_cast<uint64_t>(2u) << 61;                   // SWIZZLE_128B
  return d;
}

// Instruction descriptor for kind::i8: u8 (A) x s8 (B) -> s32, both K-major.
__device__ __forceinline__ uint32_t idesc_u8s8(uint32_t m, uint32_t n) {
  return (2u << 4)            // D format S32
         | (0u << 7)          // A unsigned int8
         | (1u << 10)         // B signed int8
         | ((n >> 3) << 17)   // N / 8
         | ((m >> 4) << 24);  // M / 16
}

// Instruction descriptor for kind::i8: s8 x s8 -> s32, both K-major.
__device__ __forceinline__ uint32_t idesc_i8(uint32_t m, uint32_t n) {
  return (2u << 4)            // D format S32
         | (1u << 7)          // A signed int8
         | (1u << 10)         // B signed int8
         | ((n >> 3) << 17)   // N / 8
         | ((m >> 4) << 24);  // M / 16
}

// ---------------------------------------------------------------------------
// MXFP4 -> INT8 decode.
// Code nibble c: magnitude index c & 7 into {0,1,2,3,4,6,8,12}, sign c & 8,
// value = +/- (mag << shift), shift in [0,3] (max 96, fits int8).
// prmt with a raw nibble selector copies byte (c & 7) of {t1,t0} when c < 8
// and replicates its sign bit (0, the table bytes are positive) when c >= 8:
// that yields the positive part P.  Flipping every nibble's bit 3 yields the
// negative part N.  P and N are disjoint per byte, so P - N = P | (-N) with a
// borrow-free per-byte negate (N <= 0x60).
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
  uint32_t r;
  asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
  return r;
}

__device__ __forceinline__ uint32_t neg_bytes_or(uint32_t p, uint32_t n) {
  // p | ((0x80808080 - n) ^ 0x80808080)
  return p | ((0x80808080u - n) ^ 0x80808080u);
}

// Decode the 8 nibbles of `q` (low nibble first) into 8 int8:
// lo <- nibbles 0..3, hi <- nibbles 4..7.
__device__ __forceinline__ void decode8(uint32_t q, uint32_t t0, uint32_t t1, uint32_t& lo,
                                        uint32_t& hi) {
  const uint32_t qn = q ^ 0x88888888u;
  const uint32_t p_lo = prmt(t0, t1, q);
  const uint32_t n_lo = prmt(t0, t1, qn);
  const uint32_t p_hi = prmt(t0, t1, q >> 16);
  const uint32_t n_hi = prmt(t0, t1, qn >> 16);
  lo = neg_bytes_or(p_lo, n_lo);
  hi = neg_bytes_or(p_hi, n_hi);
}

// Same result as decode8, with 4 of its 11 integer ops moved from the ALU
// pipe to the FMA pipe: x >> 16 as umulhi(x, 65536) and 0x80808080 - n as
// n * (-1) + 0x80808080.  m1 (= 0xFFFFFFFF) and hi16 (= 65536) must be
// run-time values (kernel parameters) so they are not folded back into ALU ops.
__device__ __forceinline__ void decode8_fma(uint32_t q, uint32_t t0, uint32_t t1, uint32_t m1,
                                            uint32_t hi16, uint32_t& lo, uint32_t& hi) {
  const uint32_t qn = q ^ 0x88888888u;
  const uint32_t qh = __umulhi(q, hi16);  // q >> 16 on the FMA pipe
  const uint32_t p_lo = prmt(t0, t1, q);
  const uint32_t n_lo = prmt(t0, t1, qn);
  const uint32_t p_hi = prmt(t0, t1, qh);
  const uint32_t n_hi = prmt(t0, t1, qh ^ 0x8888u);
  lo = p_lo | ((n_lo * m1 + 0x80808080u) ^ 0x80808080u);
  hi = p_hi | ((n_hi * m1 + 0x80808080u) ^ 0x80808080u);
}

// Biased-unsigned variant: each output byte is 0x80 + value (value in
// [-96, 96]).  P and N as in decode8_fma; 0x80 + P - N is formed with two
// IMADs on the FMA pipe (no byte carries or borrows: every byte stays in
// [0x20, 0xE0]).  Per 8 weights: 6 ALU ops (2 xor, 4 prmt) and 5 FMA-pipe ops
// (1 multiply-high, 4 IMAD), against 8 ALU + 3 FMA for decode8_fma; measured
// ~10% more stages per SM cycle in isolation.  one / m1 / hi16 (1,
// 0xFFFFFFFF, 65536) must be run-time values so they are not folded into ALU
// ops.  An MMA that reads these bytes as
// unsigned computes acc + 128 * sum(b); the caller subtracts that.
__device__ __forceinline__ void decode8_u8(uint32_t q, uint32_t t0, uint32_t t1, uint32_t one,
                                          uint32_t m1, uint32_t hi16, uint32_t& lo, uint32_t& hi) {
  const uint32_t qn = q ^ 0x88888888u;
  const uint32_t qh = __umulhi(q, hi16);  // q >> 16 on the FMA pipe
  const uint32_t p_lo = prmt(t0, t1, q);
  const uint32_t n_lo = prmt(t0, t1, qn);
  const uint32_t p_hi = prmt(t0, t1, qh);
  const uint32_t n_hi = prmt(t0, t1, qh ^ 0x8888u);
  lo = n_lo * m1 + (p_lo * one + 0x80808080u);
  hi = n_hi * m1 + (p_hi * one + 0x80808080u);
}

__device__ __forceinline__ void decode_tables(uint32_t shift, uint32_t& t0, uint32_t& t1) {
  t0 = 0x03020100u << shift;
  t1 = 0x0C080604u << shift;
}

}  // namespace dsv4
