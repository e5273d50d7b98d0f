// Shared device helpers for the sm_100a kernels: mbarriers with bounded waits, TMA tile loads,
// tcgen05 (TMEM alloc / MMA / ld / st / commit) wrappers, UMMA descriptors.
//
// Every wait in these kernels is bounded by a %globaltimer budget: on expiry the waiting thread
// raises the CTA's abort flag and records an error code in the library status word, so a protocol
// bug ends the kernel with an error instead of hanging the GPU.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/vomni_b200.h"

#define VOMNI_DEV __device__ __forceinline__

namespace vomni {

// Budget for one mbarrier wait. A healthy wait ends in microseconds (it depends only on this CTA's
// own TMA loads and MMAs); two seconds means the protocol is broken.
constexpr uint64_t kWaitBudgetNs = 2000000000ull;

VOMNI_DEV uint32_t smem_u32(const void* p) { return static_cast<uint32_t>(__cvta_generic_to_shared(p)); }

VOMNI_DEV uint64_t globaltimer() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
VOMNI_DEV void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
// Programmatic dependent launch: let the next kernel on the stream start its CTAs once every CTA of
// this grid has issued the trigger; the dependent's wait blocks until this grid has completed and its
// memory is visible (a no-op when the kernel was not launched as a dependent).
VOMNI_DEV void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
VOMNI_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
VOMNI_DEV void fence_mbar_init() { asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory"); }
VOMNI_DEV void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar)) : "memory");
}
VOMNI_DEV void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
VOMNI_DEV bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the phase completes (or
// the hint elapses) instead of spinning, so waiting producer / MMA / softmax threads do not take
// issue slots from the warps doing the math.
VOMNI_DEV bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

// Wait until the phase with parity `parity` of `bar` has completed. Returns false (and raises
// `*abort`) when the budget runs out or another thread of the CTA already aborted.
VOMNI_DEV bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort, int* status, int code,
                         uint64_t budget_ns = kWaitBudgetNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, 200000u)) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > budget_ns) {
      *abort = 1;
      if (status) atomicCAS(status, 0, code);
      return false;
    }
  }
}

// mbar_wait without the suspend hint: the waiting thread polls with plain try_wait (same budget and
// abort handling). For the attention kernel, whose MMA and softmax hand-offs are latency-critical:
// measured 0.75 % faster there than the suspending form.
VOMNI_DEV bool mbar_wait_spin(uint64_t* bar, uint32_t parity, volatile int* abort, int* status, int code,
                              uint64_t budget_ns = kWaitBudgetNs) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer();
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if (*abort) return false;
    if (globaltimer() - t0 > budget_ns) {
      *abort = 1;
      if (status) atomicCAS(status, 0, code);
      return false;
    }
  }
}

// Bounded wait until a 32-bit ready word, written by a stream memory operation after copies on
// another stream, reaches `target` (wrap-safe). Acquire, then order the async proxy (TMA reads of
// the copied data) after it.
VOMNI_DEV bool ready_wait(const unsigned* word, unsigned target, volatile int* abort, int* status, int code,
                          uint64_t budget_ns = kWaitBudgetNs) {
  const uint64_t t0 = globaltimer();
  while (true) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(word) : "memory");
    if (static_cast<int>(v - target) >= 0) {
      asm volatile("fence.proxy.async.global;" ::: "memory");
      return true;
    }
    if (*abort) return false;
    if (globaltimer() - t0 > budget_ns) {
      *abort = 1;
      if (status) atomicCAS(status, 0, code);
      return false;
    }
    __nanosleep(500);
  }
}

// ---------------------------------------------------------------- TMA (no multicast anywhere)
// Untiled bulk copy of `bytes` (a multiple of 16; both addresses 16-byte aligned) from global memory
// into this CTA's shared memory, completing on `bar` through its transaction count.
VOMNI_DEV void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
// Orders this thread's earlier generic-proxy shared-memory accesses (and, through a preceding
// barrier, other threads') before its later async-proxy ones, e.g. a bulk copy into a reused slot.
VOMNI_DEV void fence_proxy_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
VOMNI_DEV void tma_prefetch_desc(const CUtensorMap* m) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(m)) : "memory");
}
VOMNI_DEV void tma_load_3d(const CUtensorMap* m, uint64_t* bar, void* dst, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z)
      : "memory");
}
VOMNI_DEV void tma_load_2d(const CUtensorMap* m, uint64_t* bar, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}

// ---------------------------------------------------------------- tcgen05 / TMEM
VOMNI_DEV void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols)
               : "memory");
}
VOMNI_DEV void tmem_relinquish() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory"); }
VOMNI_DEV void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
VOMNI_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
VOMNI_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
// Arrive once on `bar` when every tcgen05 async op issued so far by this thread has completed.
VOMNI_DEV void tc_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// ---------------------------------------------------------------- CTA pairs (cta_group::2)
// A cluster of two CTAs on two SMs shares one MMA: the even CTA (rank 0) issues it, A rows are
// split between the CTAs (128 each), B columns too (N/2 each), and each CTA's TMEM receives its
// 128 rows of D. No TMA multicast is used anywhere: each CTA loads its own operand halves.
VOMNI_DEV uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
// shared::cluster address of the variable at this CTA's shared address `a` in CTA `rank`.
VOMNI_DEV uint32_t mapa_shared(uint32_t a, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(a), "r"(rank));
  return r;
}
VOMNI_DEV void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of another CTA of the cluster. The data it publishes is TMEM that the
// arriving thread has already completed (tcgen05.wait::st + tcgen05.fence::before_thread_sync)
// and that only the peer's tensor pipe reads, so the default (CTA-scope) release suffices.
VOMNI_DEV void mbar_arrive_cluster(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
// Tile load into this CTA's shared memory whose completion is counted on the mbarrier at
// shared::cluster address `bar_cluster` (this CTA's or its pair leader's). Not a multicast.
VOMNI_DEV void tma_load_3d_pair(const CUtensorMap* m, uint32_t bar_cluster, void* dst, int x, int y, int z) {
  asm volatile(
      "cp.async.bulk.tensor.3d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y), "r"(z)
      : "memory");
}
VOMNI_DEV void tma_load_2d_pair(const CUtensorMap* m, uint32_t bar_cluster, void* dst, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(m)), "r"(bar_cluster), "r"(x), "r"(y)
      : "memory");
}
VOMNI_DEV void mma_f8_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}
VOMNI_DEV void tmem_cp_32x128b_warpx4_pair(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::2.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}
VOMNI_DEV void mma_mxf8_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum,
                                uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
VOMNI_DEV void tmem_alloc_pair(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)), "r"(ncols)
               : "memory");
}
VOMNI_DEV void tmem_relinquish_pair() { asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory"); }
VOMNI_DEV void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// Arrive once on the mbarrier at this shared offset in both CTAs of the pair when every tcgen05
// op issued so far by this thread (pair MMAs included) has completed.
VOMNI_DEV void tc_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(static_cast<uint16_t>(3))
      : "memory");
}
VOMNI_DEV void mma_f16_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}
VOMNI_DEV void mma_f16_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::2.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}

// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f16 (bf16 operands, fp32 accumulate).
VOMNI_DEV void mma_f16_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem desc], kind::f16. A is K-major in TMEM: one row per lane,
// two bf16 per 32-bit column.
VOMNI_DEV void mma_f16_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc], kind::f8f6f4 (fp8 e4m3 operands, fp32 accumulate).
VOMNI_DEV void mma_f8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f8f6f4 [%0], %1, %2, %3, p;\n\t}" ::"r"(
          d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum)
      : "memory");
}

// D[tmem] (+)= A[smem] * B[smem] with per-32-element UE8M0 block scales read from TMEM
// (kind::mxf8f6f4.block_scale, e4m3 operands, fp32 accumulate). The instruction descriptor's
// a_sf_id / b_sf_id select which byte of each 32-bit scale word this K=32 step uses.
VOMNI_DEV void mma_mxf8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t accum,
                           uint32_t sfa_tmem, uint32_t sfb_tmem) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::mxf8f6f4.block_scale [%0], %1, %2, %3, [%5], [%6], p;\n\t}" ::"r"(d_tmem),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accum), "r"(sfa_tmem), "r"(sfb_tmem)
      : "memory");
}
// Shared memory -> TMEM copy of 32 rows x 128 bits, replicated into all four lane quadrants.
VOMNI_DEV void tmem_cp_32x128b_warpx4(uint32_t taddr, uint64_t sdesc) {
  asm volatile("tcgen05.cp.cta_group::1.32x128b.warpx4 [%0], %1;" ::"r"(taddr), "l"(sdesc) : "memory");
}

// 32 lanes x 32 consecutive 32-bit columns: thread t of the warp gets lane (warp%4)*32 + t.
VOMNI_DEV void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]), "=r"(r[16]),
        "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]), "=r"(r[24]),
        "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
}
// Completes the preceding tcgen05.ld; the registers are threaded through so no use of them can be
// scheduled above the wait. tcgen05.ld / tcgen05.st carry no "memory" clobber (they touch only
// TMEM and registers), so independent math can be scheduled across them; their order against
// each other (both asm volatile) and against the barrier fences (which do clobber memory) stays.
VOMNI_DEV void tmem_ld_wait(uint32_t (&r)[32]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15]),
                 "+r"(r[16]), "+r"(r[17]), "+r"(r[18]), "+r"(r[19]), "+r"(r[20]), "+r"(r[21]), "+r"(r[22]),
                 "+r"(r[23]), "+r"(r[24]), "+r"(r[25]), "+r"(r[26]), "+r"(r[27]), "+r"(r[28]), "+r"(r[29]),
                 "+r"(r[30]), "+r"(r[31])
               :
               : "memory");
}
VOMNI_DEV void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, %15, "
      "%16};" ::"r"(taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]));
}
VOMNI_DEV void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ---------------------------------------------------------------- UMMA descriptors
// Shared-memory matrix descriptor (sm_100 format): start address, leading / stride byte offsets
// (16-byte units), version 1, layout type in bits 61-63 (2 = 128-byte swizzle).
constexpr uint32_t kLayoutSW128 = 2;
VOMNI_DEV uint64_t make_sdesc(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes, uint32_t layout) {
  uint64_t d = 0;
  d |= static_cast<uint64_t>((saddr >> 4) & 0x3FFFu);
  d |= static_cast<uint64_t>((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= static_cast<uint64_t>((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= static_cast<uint64_t>(1) << 46;
  d |= static_cast<uint64_t>(layout & 0x7u) << 61;
  return d;
}
// Instruction descriptor, kind::f16 with bf16 A/B and fp32 D. b_mn_major: B stored N-contiguous.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool b_mn_major) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((b_mn_major ? 1u : 0u) << 16) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}
// kind::f16 descriptor with either operand MN-major (A: bit 15, B: bit 16).
__host__ __device__ constexpr uint32_t idesc_bf16_mn(int m, int n, bool a_mn_major, bool b_mn_major) {
  return idesc_bf16(m, n, b_mn_major) | ((a_mn_major ? 1u : 0u) << 15);
}
// Instruction descriptor, kind::mxf8f6f4.block_scale: e4m3 A/B (K-major), UE8M0 scales (bit 23),
// fp32 D, scale byte `sf_id` of each 32-bit scale word for both A (bits 29-30) and B (bits 4-5).
__host__ __device__ constexpr uint32_t idesc_mxf8(int m, int n, uint32_t sf_id) {
  return ((sf_id & 3u) << 4) | (static_cast<uint32_t>(n >> 3) << 17) | (1u << 23) |
         (static_cast<uint32_t>(m >> 4) << 24) | ((sf_id & 3u) << 29);
}
// Instruction descriptor, kind::f8f6f4 with e4m3 A/B (both K-major) and fp32 D.
__host__ __device__ constexpr uint32_t idesc_e4m3(int m, int n) {
  return (1u << 4) | (0u << 7) | (0u << 10) | (static_cast<uint32_t>(n >> 3) << 17) | (static_cast<uint32_t>(m >> 4) << 24);
}

// ---------------------------------------------------------------- math
VOMNI_DEV float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

// Packed fp32 pairs (sm_100 `.f32x2` arithmetic): one instruction operates on two fp32 values held
// in a 64-bit register pair, halving the issue slots of elementwise fp32 work. Each lane of the
// pair is rounded exactly as the scalar instruction would round it.
VOMNI_DEV uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
VOMNI_DEV void f2_unpack(uint64_t v, float& lo, float& hi) { asm("mov.b64 {%0, %1}, %2;" : "=f"(lo), "=f"(hi) : "l"(v)); }
VOMNI_DEV uint64_t f2_fma(uint64_t a, uint64_t b, uint64_t c) {
  uint64_t r;
  asm("fma.rn.f32x2 %0, %1, %2, %3;" : "=l"(r) : "l"(a), "l"(b), "l"(c));
  return r;
}
VOMNI_DEV uint64_t f2_add(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("add.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
VOMNI_DEV uint64_t f2_mul(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("mul.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}
VOMNI_DEV uint64_t f2_sub(uint64_t a, uint64_t b) {
  uint64_t r;
  asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(a), "l"(b));
  return r;
}

// 2^x for a pair of fp32 values on the FMA pipe, so that a share of the softmax exponentials
// bypasses the MUFU unit (which delivers 16 results per clock per SM, the same rate as the tensor
// pipe needs them at head dim 128). Method: Cody-Waite range reduction x = n + f with n = rint(x),
// obtained by adding 1.5 * 2^23 so that n lands in the low mantissa bits, and f in [-0.5, 0.5];
// 2^f from a degree-3 polynomial whose coefficients were fitted by a Remez exchange minimising the
// relative error on [-0.5, 0.5] (max 7.5e-5 = 2^-13.7, far below the bf16 rounding that softmax
// probabilities get); 2^n is added into the exponent field as an integer. That addition is exact
// while the result stays a normal number (n >= -125); below x = -125.5 the result is 0, as the
// flush-to-zero MUFU exponential gives 0 for results under 2^-126. The reduction and the polynomial
// run as `.f32x2` pairs (6 instructions for two values).
constexpr float kExp2Round = 12582912.f;  // 1.5 * 2^23
constexpr float kExp2C3 = 0.0551716685f, kExp2C2 = 0.2426111251f, kExp2C1 = 0.6932609677f, kExp2C0 = 0.9999280572f;
VOMNI_DEV void exp2_poly2(float x0, float x1, float& p0, float& p1) {
  const uint64_t x = f2_pack(x0, x1);
  const uint64_t rnd = f2_pack(kExp2Round, kExp2Round);
  const uint64_t t = f2_add(x, rnd);
  const uint64_t f = f2_sub(x, f2_sub(t, rnd));
  uint64_t p = f2_fma(f2_pack(kExp2C3, kExp2C3), f, f2_pack(kExp2C2, kExp2C2));
  p = f2_fma(p, f, f2_pack(kExp2C1, kExp2C1));
  p = f2_fma(p, f, f2_pack(kExp2C0, kExp2C0));
  float plo, phi, tlo, thi;
  f2_unpack(p, plo, phi);
  f2_unpack(t, tlo, thi);
  // (bits(t) - bits(1.5 * 2^23)) << 23 == n << 23 (mod 2^32): the constant's 23 low bits are 0.
  const float r0 = __int_as_float(__float_as_int(plo) + (__float_as_int(tlo) << 23));
  const float r1 = __int_as_float(__float_as_int(phi) + (__float_as_int(thi) << 23));
  p0 = x0 > -125.5f ? r0 : 0.f;
  p1 = x1 > -125.5f ? r1 : 0.f;
}
// a += bf16 lo half of `pk`, b += bf16 hi half, exactly (sm_100 mixed-precision add: the bf16 operand
// is widened exactly, the sum rounded once to fp32) — one instruction per value.
VOMNI_DEV void add_bf16x2_f32(float& a, float& b, uint32_t pk) {
  asm("{\n\t.reg .b16 lo, hi;\n\tmov.b32 {lo, hi}, %2;\n\tadd.rn.f32.bf16 %0, lo, %0;\n\tadd.rn.f32.bf16 %1, hi, %1;\n\t}"
      : "+f"(a), "+f"(b)
      : "r"(pk));
}
// Two fp32 -> packed bf16x2 (round to nearest even); `lo` lands in bits 0-15.
VOMNI_DEV uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}
// Two fp32 -> two e4m3 (round to nearest even, saturate to +-448); lo in byte 0.
VOMNI_DEV uint16_t e4m3x2(float lo, float hi) {
  uint16_t r;
  asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(r) : "f"(hi), "f"(lo));
  return r;
}
// GELU with the tanh approximation in fp32 (torch's gelu(approximate="tanh") formula).
VOMNI_DEV float gelu_tanh(float x) {
  const float kBeta = 0.7978845608028654f;  // sqrt(2 / pi)
  const float kKappa = 0.044715f;
  const float x3 = x * x * x;
  const float inner = kBeta * (x + kKappa * x3);
  return 0.5f * x * (1.f + tanhf(inner));
}

}  // namespace vomni
