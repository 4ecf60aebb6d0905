// Device-side building blocks shared by the KernelSwift-B200 kernels (sm_100a only).
//
//  * mbarrier helpers whose waits are bounded: a wait that exceeds its time
//    budget records an error code in a status word, raises a CTA-local abort
//    flag and returns false, so no kernel can spin forever;
//  * TMA (cp.async.bulk.tensor) tile and gather4 loads completing on an mbarrier;
//  * tcgen05 wrappers: TMEM alloc/dealloc, MMA (kind::f16, cta_group 1 and 2),
//    commit, TMEM loads, fences;
//  * UMMA shared-memory / instruction descriptors for the 128-byte-swizzled
//    canonical layouts that TMA writes.
//
// Every TMA load here writes only the issuing CTA's own shared memory and reads
// only this GPU's global memory.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ks {

// ------------------------------------------------------------------ status
enum DeviceError : int {
  DEV_OK = 0,
  DEV_TIMEOUT = 1,  // a bounded wait ran out
  DEV_BOUNDS = 2,   // an index check failed; the access was skipped
};

__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count)
               : "memory");
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{ .reg .b64 st; mbarrier.arrive.shared::cta.b64 st, [%0]; }" ::"r"(smem_u32(bar))
               : "memory");
}

// Arrive on the barrier at the same shared-memory offset in CTA `cta` of the cluster.
__device__ __forceinline__ void mbar_arrive_cluster(uint64_t* bar, uint32_t cta) {
  asm volatile(
      "{ .reg .b32 ra; mapa.shared::cluster.u32 ra, %0, %1;"
      " mbarrier.arrive.shared::cluster.b64 _, [ra]; }" ::"r"(smem_u32(bar)),
      "r"(cta)
      : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ bool mbar_test_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.try_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;"
      " selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Non-blocking probes (mbarrier.test_wait): for loops that poll several barriers;
// try_wait may suspend the thread on the first incomplete barrier it probes.
__device__ __forceinline__ bool mbar_poll(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2; selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool mbar_poll_cluster(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{ .reg .pred p; mbarrier.test_wait.parity.acquire.cluster.shared::cta.b64 p, [%1], %2;"
      " selp.u32 %0, 1, 0, p; }"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// Shared state every bounded wait consults: the CTA-local abort flag (in shared
// memory), the global status word and the time budget of one wait.
struct WaitCtx {
  volatile int* abort;  // shared memory
  int* status;          // global memory (4 ints: code and where the first timeout was), may be null
  uint64_t budget_ns;
  int tag = 0;          // caller's progress marker, reported with a timeout
};

// Budgets are enforced with the SM cycle counter (cheap to read, unlike
// %globaltimer): at most 2 cycles per ns below 2 GHz, so a budget of B ns
// expires after at most 2B cycles, i.e. between B/2 and 2B ns of wall time for
// SM clocks from 1 to 2 GHz.
__device__ __forceinline__ uint64_t budget_cycles(uint64_t budget_ns) { return budget_ns * 2; }

__device__ __forceinline__ void raise_error(const WaitCtx& w, int code) {
  *w.abort = 1;
  if (w.status) atomicCAS(w.status, 0, code);
}
// A timed-out wait also records where it happened (first one only):
// status[1] = block, status[2] = thread << 20 | barrier's shared-memory offset << 1 | parity,
// status[3] = the waiting thread's progress tag.
__device__ __forceinline__ void raise_timeout(const WaitCtx& w, uint32_t bar, uint32_t parity) {
  *w.abort = 1;
  if (w.status && atomicCAS(w.status, 0, DEV_TIMEOUT) == 0) {
    w.status[1] = (int)blockIdx.x;
    w.status[2] = (int)((threadIdx.x << 20) | ((bar & 0x7FFFFu) << 1) | (parity & 1u));
    w.status[3] = w.tag;
  }
}

// An index outside its table was found; the access it named was skipped.  Records
// DEV_BOUNDS (first error only) with status[1] = `where` (e.g. the query row) and
// status[3] = `value` (e.g. the table size the index reached).  Unlike a timeout it
// does not abort the CTA.
__device__ __forceinline__ void report_bounds(int* status, int where, int value) {
  if (status && atomicCAS(status, 0, DEV_BOUNDS) == 0) {
    status[1] = where;
    status[2] = 0;
    status[3] = value;
  }
}

// Wait until the phase with `parity` of `bar` completes.  Returns false when the
// CTA is aborting (unless `drain`) or the budget ran out (then the error is
// recorded).  `drain` waits are the ones that make sure copies and MMAs already
// in flight have landed before the CTA exits; they ignore the abort flag but
// keep the time budget.
__device__ __forceinline__ bool mbar_wait_body(uint64_t* bar, uint32_t parity, const WaitCtx& w,
                                               bool cluster_scope, bool drain) {
  const uint32_t b = smem_u32(bar);
  if (cluster_scope ? mbar_test_cluster(b, parity) : mbar_test(b, parity)) return true;
  const uint64_t t0 = clock64();
  const uint64_t lim = budget_cycles(w.budget_ns);
  for (;;) {
    // try_wait without a suspend-time hint: with a hint, a waiting thread was seen
    // (rarely) never to return although the phase had completed.
    if (cluster_scope ? mbar_test_cluster(b, parity) : mbar_test(b, parity)) return true;
    if (!drain && *w.abort) return false;
    if ((uint64_t)clock64() - t0 > lim) {
      raise_timeout(w, b, parity);
      return false;
    }
  }
}
__device__ __noinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, const WaitCtx& w,
                                       bool cluster_scope = false, bool drain = false) {
  return mbar_wait_body(bar, parity, w, cluster_scope, drain);
}
// The same wait compiled into the caller.  A call keeps every register that is
// live across it (e.g. the destination of a load still in flight) in a saved
// register or on the stack, and saving one waits for its load to land: loops
// that keep loads in flight across a wait use this form.
__device__ __forceinline__ bool mbar_wait_inl(uint64_t* bar, uint32_t parity, const WaitCtx& w,
                                              bool cluster_scope = false) {
  return mbar_wait_body(bar, parity, w, cluster_scope, false);
}

// ------------------------------------------------------------------ clusters
__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// All threads of every CTA in the cluster.
__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::
                   : "memory");
}

// One lane of a fully active warp (the lowest) is elected; all 32 lanes must call.
__device__ __forceinline__ bool elect_one() {
  uint32_t pred;
  asm volatile("{ .reg .pred p; elect.sync _|p, 0xffffffff; selp.u32 %0, 1, 0, p; }" : "=r"(pred));
  return pred != 0;
}

// ------------------------------------------------------------------ proxies / fences
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
__device__ __forceinline__ void named_bar_sync(uint32_t id, uint32_t nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}

// 2D tile load (no multicast) into this CTA's shared memory.
__device__ __forceinline__ void tma_load_2d(const CUtensorMap* m, uint64_t* bar, void* dst,
                                            int32_t x, int32_t y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// 2D tile store from this CTA's shared memory to global memory, tracked as a bulk
// group of the issuing thread (x, y >= 0; x times the element size a multiple of 16).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* m, const void* src, int32_t x,
                                             int32_t y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(m)),
               "r"(smem_u32(src)), "r"(x), "r"(y)
               : "memory");
}
__device__ __forceinline__ void bulk_commit_group() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}
// Wait until at most N of this thread's bulk groups still read shared memory.
template <int N>
__device__ __forceinline__ void bulk_wait_group_read() {
  asm volatile("cp.async.bulk.wait_group.read %0;" ::"n"(N) : "memory");
}
// Wait until at most N of this thread's bulk groups are incomplete.
template <int N>
__device__ __forceinline__ void bulk_wait_group() {
  asm volatile("cp.async.bulk.wait_group %0;" ::"n"(N) : "memory");
}

// Four rows (y0..y3) of a 2D tensor, columns [x, x + box_w), into four consecutive
// box rows in this CTA's shared memory.  No multicast.
__device__ __forceinline__ void tma_gather4(const CUtensorMap* m, uint64_t* bar, void* dst,
                                            int32_t x, int32_t y0, int32_t y1, int32_t y2,
                                            int32_t y3) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cta.global.tile::gather4.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%3, %4, %5, %6, %7}], [%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y0), "r"(y1), "r"(y2),
      "r"(y3)
      : "memory");
}

// ------------------------------------------------------------------ predicated loads
// 16 bytes from global memory (cached in L2 only) when `pred`, else zeros.  The
// zeros are written first and the load is predicated, so nothing consumes the
// loaded value here: the thread runs on until it uses the registers (a
// `pred ? load : 0` select would wait for the load on the spot).
__device__ __forceinline__ uint4 ldcg_or_zero(const void* ptr, bool pred) {
  uint4 v;
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %5, 0;"
      " mov.b32 %0, 0; mov.b32 %1, 0; mov.b32 %2, 0; mov.b32 %3, 0;"
      " @p ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4]; }"
      : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
      : "l"(ptr), "r"((int)pred));
  return v;
}

// 32-bit load through the read-only path when `pred`, else `fallback` (same idea).
__device__ __forceinline__ int32_t ldg_s32_or(const int32_t* ptr, bool pred, int32_t fallback) {
  int32_t v;
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %3, 0; mov.b32 %0, %2;"
      " @p ld.global.nc.b32 %0, [%1]; }"
      : "=r"(v)
      : "l"(ptr), "r"(fallback), "r"((int)pred));
  return v;
}

// ------------------------------------------------------------------ cp.async (16 bytes)
// Copy 16 bytes global -> shared (L2 only); src_bytes < 16 zero-fills the rest.
__device__ __forceinline__ void cp_async16(void* dst, const void* src, uint32_t src_bytes = 16) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(dst)), "l"(src),
               "r"(src_bytes)
               : "memory");
}
// Arrive on `bar` once every cp.async this thread issued so far has landed (the
// arrival counts against the barrier's expected count).
__device__ __forceinline__ void cp_async_arrive(uint64_t* bar) {
  asm volatile("cp.async.mbarrier.arrive.noinc.shared::cta.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void cp_async_wait_all() {
  asm volatile("cp.async.wait_all;" ::: "memory");
}

// ------------------------------------------------------------------ tcgen05
template <int CG>
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
  else
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
template <int CG>
__device__ __forceinline__ void tmem_relinquish() {
  if constexpr (CG == 1)
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  else
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
template <int CG>
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  if constexpr (CG == 1)
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
  else
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, bf16 inputs, fp32 accumulate.
__device__ __forceinline__ void umma_bf16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                             uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
__device__ __forceinline__ void umma_bf16_ss_cg2(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                                 uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;"
      " tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, e4m3 (fp8) inputs, fp32 accumulate; one
// instruction contracts K = 32 elements (32 bytes of each K-major row).
__device__ __forceinline__ void umma_f8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                           uint32_t idesc, uint32_t accumulate) {
  asm volatile(
      "{ .reg .pred p; setp.ne.b32 p, %4, 0;"
      " tcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p; }" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// cta_group::2 MMA with descriptors passed as (low, high) words: the start address
// sits in the low 14 bits, so per-MMA offsets are single 32-bit adds.
__device__ __forceinline__ void umma_cg2_w(uint32_t d, uint32_t alo, uint32_t ahi, uint32_t blo,
                                           uint32_t bhi, uint32_t idesc, uint32_t acc) {
  asm volatile(
      "{ .reg .pred p; .reg .b64 ad, bd; setp.ne.b32 p, %6, 0; mov.b64 ad, {%1, %2};"
      " mov.b64 bd, {%3, %4}; tcgen05.mma.cta_group::2.kind::f16 [%0], ad, bd, %5, p; }" ::"r"(d),
      "r"(alo), "r"(ahi), "r"(blo), "r"(bhi), "r"(idesc), "r"(acc)
      : "memory");
}

// Arrive (once) on `bar` when every previously issued tcgen05 op of this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
          smem_u32(bar))
      : "memory");
}
// 2-CTA form: arrive on the barrier at the same offset in every CTA of `cta_mask`.
__device__ __forceinline__ void umma_commit_cg2(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
      " [%0], %1;" ::"r"(smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

__device__ __forceinline__ void tmem_wait_ld() {
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_wait_st() {
  asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}

// 32 lanes x 32-bit, N consecutive columns -> r[0..N).
#define KS_TMEM_LD_X16(taddr, r)                                                              \
  asm volatile(                                                                                \
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13," \
      "%14,%15}, [%16];"                                                                       \
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),    \
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),             \
        "=r"(r[13]), "=r"(r[14]), "=r"(r[15])                                                  \
      : "r"(taddr))

__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t* r) { KS_TMEM_LD_X16(taddr, r); }

__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t* r) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,"
      "%15,%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
        "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]),
        "=r"(r[14]), "=r"(r[15]), "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]),
        "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]), "=r"(r[25]),
        "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}

__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t* r) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,"
      "%14,%15,%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
      "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
      "r"(r[15])
      : "memory");
}

// ------------------------------------------------------------------ UMMA descriptors
// Shared-memory matrix descriptor for the 128-byte-swizzled canonical layout that a
// TMA load with CU_TENSOR_MAP_SWIZZLE_128B and a 128-byte-wide box produces:
// rows of 128 bytes, 8-row (1024-byte) swizzle atoms.
//   K-major operand : start = row 0 of the atom column; LBO unused (1); SBO = 1024
//                     (next 8 rows).  Step along K inside the 128-byte row by adding
//                     the byte offset to the start address.
//   MN-major operand: start = first K row; LBO = byte stride between 64-element MN
//                     blocks; SBO = 1024 (next 8 K rows).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t saddr, uint32_t lbo_bytes,
                                                uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFF);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFF) << 32;
  d |= (uint64_t)1 << 46;  // descriptor version for tcgen05
  d |= (uint64_t)2 << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor, kind::f16: bf16 A and B, fp32 D.
//   bits 4-5 D format (1 = f32), 7-9 A format (1 = bf16), 10-12 B format (1 = bf16),
//   15 A major (0 = K, 1 = MN), 16 B major, 17-22 N>>3, 24-28 M>>4.
__host__ __device__ constexpr uint32_t idesc_bf16_f32(int M, int N, bool a_mn_major,
                                                      bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn_major ? 1u : 0u) << 15) |
         ((b_mn_major ? 1u : 0u) << 16) | ((uint32_t)(N >> 3) << 17) |
         ((uint32_t)(M >> 4) << 24);
}

// Instruction descriptor, kind::f8f6f4: e4m3 A and B (format code 0), fp32 D,
// both K-major; same field positions as idesc_bf16_f32.
__host__ __device__ constexpr uint32_t idesc_e4m3_f32(int M, int N) {
  return (1u << 4) | ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

// ------------------------------------------------------------------ bf16 arithmetic
// Two fp32 -> bf16x2 with ReLU, round to nearest even (lo in bits 0-15).
__device__ __forceinline__ uint32_t cvt_relu_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.relu.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
__device__ __forceinline__ uint32_t cvt_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// Lane-wise bf16 product, correctly rounded (round to nearest even).
__device__ __forceinline__ uint32_t mul_bf16x2(uint32_t a, uint32_t b) {
  uint32_t r;
  asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(b));
  return r;
}
__device__ __forceinline__ float bf16lo_f32(uint32_t v) { return __uint_as_float(v << 16); }
__device__ __forceinline__ float bf16hi_f32(uint32_t v) { return __uint_as_float(v & 0xFFFF0000u); }

}  // namespace ks
