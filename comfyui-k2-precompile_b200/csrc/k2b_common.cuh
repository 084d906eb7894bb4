// k2b_common.cuh -- sm_100a building blocks shared by the k2b kernels:
// bounded mbarrier waits, TMA loads, tcgen05 (TMEM alloc / MMA / commit /
// ld / st), UMMA shared-memory descriptors, and the exact scalar helpers that
// the CPU oracle restates bit for bit (bf16/fp16 rounding, exp, quantisation).
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace k2b {

// ------------------------------------------------------------------ errors
// Device-side error word of the library (one per loaded .so).  Kernels never
// trap: a wait that runs out of time records a code here, raises the CTA's
// abort flag, and every role of the CTA unwinds to the teardown.
__device__ int g_error;

enum DeviceError : int {
  ERR_WAIT_PRODUCER = 1 << 0,
  ERR_WAIT_MMA = 1 << 1,
  ERR_WAIT_UNPACK = 1 << 2,
  ERR_WAIT_EPILOGUE = 1 << 3,
  ERR_WAIT_SOFTMAX = 1 << 4,
  ERR_WAIT_LOAD = 1 << 5,
  ERR_WAIT_SELFTEST = 1 << 6,
};

// Upper bound for any single mbarrier wait.  Normal waits are microseconds.
constexpr unsigned long long kWaitLimitNs = 2000000000ull;
// Bound for the teardown wait on copies/MMAs still in flight after an abort.
constexpr unsigned long long kDrainLimitNs = 200000000ull;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ unsigned long long global_timer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ---------------------------------------------------------------- mbarrier
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.expect_tx.shared::cta.b64 st, [%0], %1;\n\t}" ::"r"(
                   smem_u32(bar)),
               "r"(bytes)
               : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait that may suspend the thread until the phase completes or
// `hint_ns` elapses: a waiting warp then issues nothing, instead of polling.
__device__ __forceinline__ bool mbar_try_wait_sleep(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\tselp.b32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
constexpr uint32_t kWaitSleepNs = 1000000;  // 1 ms per suspension

// Bounded waits.  Reading %globaltimer costs a few hundred cycles, which on
// the MMA <-> epilogue handoff chain of the GEMM is paid every K group (traced:
// ~300 cycles per wait).  So every wait polls first and only starts its clock
// after kWaitPollsPerCheck failed polls, then looks at the clock once per
// kWaitPollsPerCheck polls: a wait that completes within a few polls never
// reads the timer, and every wait still gives up within its limit (plus at
// most kWaitPollsPerCheck suspended polls).
constexpr uint32_t kWaitPollsPerCheck = 16;

// Bounded wait for the completion of phase `parity` of `bar`.  Returns false
// (after raising *abort and recording `code`) if the CTA was aborted or the
// wait exceeded `limit_ns`.  Between checks the thread sleeps in try_wait
// (woken by the phase completing), so waiting warps leave the issue slots to
// the warps doing work.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int code,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  const uint32_t a = smem_u32(bar);
  if (mbar_try_wait(a, parity)) return true;
  unsigned long long t0 = 0;
  for (uint32_t polls = 1;; ++polls) {
    if (mbar_try_wait_sleep(a, parity, kWaitSleepNs)) return true;
    if (*abort_flag) return false;
    if (polls % kWaitPollsPerCheck == 0) {
      const unsigned long long now = global_timer();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > limit_ns) {
        *abort_flag = 1;
        atomicOr(&g_error, code);
        return false;
      }
    }
  }
}

// mbar_wait on 32-bit shared-memory addresses (barrier and abort flag), for
// loops that cannot spare registers for generic pointers.
__device__ __forceinline__ bool mbar_wait_s(uint32_t a, uint32_t parity, uint32_t abort_addr, int code) {
  if (mbar_try_wait(a, parity)) return true;
  unsigned long long t0 = 0;
  for (uint32_t polls = 1;; ++polls) {
    if (mbar_try_wait_sleep(a, parity, kWaitSleepNs)) return true;
    int ab;
    asm volatile("ld.volatile.shared.b32 %0, [%1];" : "=r"(ab) : "r"(abort_addr) : "memory");
    if (ab) return false;
    if (polls % kWaitPollsPerCheck == 0) {
      const unsigned long long now = global_timer();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitLimitNs) {
        asm volatile("st.volatile.shared.b32 [%0], %1;" ::"r"(abort_addr), "r"(1) : "memory");
        atomicOr(&g_error, code);
        return false;
      }
    }
  }
}
__device__ __forceinline__ void mbar_arrive_s(uint32_t a) {
  asm volatile("{\n\t.reg .b64 st;\n\tmbarrier.arrive.shared::cta.b64 st, [%0];\n\t}" ::"r"(a) : "memory");
}
__device__ __forceinline__ float4 lds128(uint32_t a) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(a));
  return v;
}

// mbar_wait for phases completed by arrivals from the other CTA of the pair.
__device__ __forceinline__ bool mbar_wait_cluster(uint64_t* bar, uint32_t parity, volatile int* abort_flag, int code) {
  const uint32_t a = smem_u32(bar);
  unsigned long long t0 = 0;
  for (uint32_t polls = 0;; ++polls) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.b32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(a), "r"(parity), "r"(kWaitSleepNs)
        : "memory");
    if (ok) return true;
    if (*abort_flag) return false;
    if (polls % kWaitPollsPerCheck == kWaitPollsPerCheck - 1) {
      const unsigned long long now = global_timer();
      if (t0 == 0) {
        t0 = now;
      } else if (now - t0 > kWaitLimitNs) {
        *abort_flag = 1;
        atomicOr(&g_error, code);
        return false;
      }
    }
  }
}

// Teardown-only wait (ignores the abort flag): lets async copies or MMAs that
// were already issued land before the CTA releases its shared memory / TMEM.
__device__ __forceinline__ void mbar_drain(uint64_t* bar, uint32_t parity) {
  const uint32_t a = smem_u32(bar);
  const unsigned long long t0 = global_timer();
  while (!mbar_try_wait(a, parity)) {
    if (global_timer() - t0 > kDrainLimitNs) return;
  }
}

// --------------------------------------------------------------------- TMA
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4}], [%2];" ::"r"(
          smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y)
      : "memory");
}
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y, int z,
                                            int w) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%3, %4, %5, %6}], "
      "[%2];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(smem_u32(bar)), "r"(x), "r"(y), "r"(z), "r"(w)
      : "memory");
}
// Untiled bulk copy global -> shared (addresses and size 16-byte aligned).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
                   smem_u32(dst)),
               "l"(src), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ----------------------------------------------------------------- tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// ---- CTA pair (cluster of 2) forms: the pair shares one MMA issued by
// cluster rank 0; TMEM is allocated at the same columns in both CTAs.
__device__ __forceinline__ uint32_t cluster_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Address of this CTA's shared-memory word `addr` in cluster CTA `rank`.
__device__ __forceinline__ uint32_t cluster_map(uint32_t addr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(addr), "r"(rank));
  return r;
}
// Arrive on an mbarrier of another CTA of the cluster (cluster_map address).
// Default (release) semantics, as the CTA-pair pipelines of CUTLASS use: a
// cluster-scope release here measured ~800 cycles per arrival.
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
  asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
// M = 256 MMA over the pair: A rows 0-127 / 128-255 and B columns 0-N/2-1 /
// N/2.. from the two CTAs' shared memory at the same offsets; each CTA's TMEM
// receives its 128 rows.
__device__ __forceinline__ void mma_i8_pair(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, "
      "p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// The same pair MMA on e4m3 x e4m3 operands with fp32 accumulators
// (kind::f8f6f4, K = 32 per instruction like kind::i8).
__device__ __forceinline__ void mma_f8_pair(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                           uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::2.kind::f8f6f4 [%0], %1, %2, %3, "
      "p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Completion of the pair's prior MMAs arrives on the mbarrier at this offset
// in both CTAs.
__device__ __forceinline__ void mma_commit_pair(uint64_t* bar) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"((uint16_t)3)
      : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem] * B[smem]^T, int8 x int8 -> int32.
__device__ __forceinline__ void mma_i8_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, "
      "p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[smem] * B[smem], bf16 x bf16 -> fp32.
__device__ __forceinline__ void mma_bf16_ss(uint32_t d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, "
      "p;\n\t}" ::"r"(d),
      "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem], bf16 x bf16 -> fp32.
__device__ __forceinline__ void mma_bf16_ts(uint32_t d, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc,
                                            uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\ttcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, "
      "p;\n\t}" ::"r"(d),
      "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive on `bar` once every tcgen05 operation issued so far by this thread completes.
__device__ __forceinline__ void mma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}
// max(a, b, c) in one instruction (NaN operands are ignored, as by fmaxf).
__device__ __forceinline__ float fmax3(float a, float b, float c) {
  float r;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(r) : "f"(a), "f"(b), "f"(c));
  return r;
}
__device__ __forceinline__ void tmem_wait_ld() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_wait_st() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }
// tcgen05.wait::ld that also "writes" the destination registers of the
// preceding tcgen05.ld, so no use of them can be scheduled above the wait.
__device__ __forceinline__ void tmem_wait_ld_regs(uint32_t (&r)[16]) {
  asm volatile("tcgen05.wait::ld.sync.aligned;"
               : "+r"(r[0]), "+r"(r[1]), "+r"(r[2]), "+r"(r[3]), "+r"(r[4]), "+r"(r[5]), "+r"(r[6]), "+r"(r[7]),
                 "+r"(r[8]), "+r"(r[9]), "+r"(r[10]), "+r"(r[11]), "+r"(r[12]), "+r"(r[13]), "+r"(r[14]), "+r"(r[15])
               :
               : "memory");
}

// 32 lanes x 16 columns of 32-bit: thread i of the warp receives its lane's 16 columns.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]), "=r"(r[8]),
        "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr)
      : "memory");
}
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};" ::"r"(
          taddr),
      "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]), "r"(r[9]),
      "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15])
      : "memory");
}

__device__ __forceinline__ void setmaxnreg_dec32() { asm volatile("setmaxnreg.dec.sync.aligned.u32 32;"); }
__device__ __forceinline__ void setmaxnreg_inc112() { asm volatile("setmaxnreg.inc.sync.aligned.u32 112;"); }

// UMMA shared-memory descriptor for a 128B-swizzled tile (sm_100 version 1).
// K-major: rows of 128 B, 8-row atoms 1024 B apart (SBO), LBO unused (1).
// MN-major: 128 B of MN per K row, 8 K rows per atom (SBO between K atoms),
// LBO between 64-element MN blocks.
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr, uint32_t lbo_bytes, uint32_t sbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr >> 4) & 0x3FFFu);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo_bytes >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1u << 46;  // descriptor version (sm_100)
  d |= (uint64_t)2u << 61;  // SWIZZLE_128B
  return d;
}

// Instruction descriptor: c_fmt {0:f16,1:f32,2:s32}, a/b fmt {i8: 0 u8 / 1 s8;
// f16-kind: 0 f16 / 1 bf16; f8f6f4-kind: 0 e4m3 / 1 e5m2}, majors {0:K, 1:MN}.
__host__ __device__ constexpr uint32_t make_idesc(uint32_t c_fmt, uint32_t a_fmt, uint32_t b_fmt, uint32_t a_major,
                                                  uint32_t b_major, uint32_t m, uint32_t n) {
  return (c_fmt << 4) | (a_fmt << 7) | (b_fmt << 10) | (a_major << 15) | (b_major << 16) | ((n >> 3) << 17) |
         ((m >> 4) << 24);
}

// ------------------------------------------------------- packed fp32 math
// Float pairs kept in 64-bit registers so fma.rn.f32x2 consumes them without
// repacking.
__device__ __forceinline__ uint64_t f2_pack(float lo, float hi) {
  uint64_t r;
  asm("mov.b64 %0, {%1, %2};" : "=l"(r) : "f"(lo), "f"(hi));
  return r;
}
__device__ __forceinline__ float f2_lo(uint64_t v) { return __uint_as_float((uint32_t)v); }
__device__ __forceinline__ float f2_hi(uint64_t v) { return __uint_as_float((uint32_t)(v >> 32)); }
// acc = fma(fma({x0,x1}, sa, sb), sw, acc) on a float pair, the two drained
// TMEM words x0/x1 given as raw bits.
__device__ __forceinline__ void dequant_acc2(uint64_t& acc, uint32_t x0, uint32_t x1, uint64_t sa2, uint64_t sb2,
                                             uint64_t sw2) {
  asm("{\n\t.reg .b64 f, u;\n\tmov.b64 f, {%1, %2};\n\tfma.rn.f32x2 u, f, %3, %4;\n\tfma.rn.f32x2 %0, u, %5, "
      "%0;\n\t}"
      : "+l"(acc)
      : "r"(x0), "r"(x1), "l"(sa2), "l"(sb2), "l"(sw2));
}
__device__ __forceinline__ float2 ffma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\tmov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, "
      "%7};\n\tfma.rn.f32x2 rd, ra, rb, rc;\n\tmov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}

__device__ __forceinline__ uint32_t pack_bf16x2(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ------------------------------------------------- exact scalar contract

// Unnormalised Walsh-Hadamard transform of a 128-column group: seven
// butterfly stages (a, b) -> (a + b, a - b) over index bit lh (partner
// distance h = 1 << lh), each sum rounded to fp32, in the contract's order
// h = 2, 4, 8, 1, 16, 32, 64 (oracle: k2o_hadamard128).  Any stage order
// gives the same transform in exact arithmetic; this one lets the
// norm_quant kernel run every stage but one on packed f32x2 pairs.
__host__ __device__ constexpr int hadamard_stage_bit(int st) { return st < 3 ? st + 1 : (st == 3 ? 0 : st); }
// In-register transform of 128 fp32 values; counted stage loop so every
// index is a compile-time constant.
__device__ __forceinline__ void hadamard128_regs(float (&v)[128]) {
#pragma unroll
  for (int st = 0; st < 7; ++st) {
    const int lh = hadamard_stage_bit(st);
    const int h = 1 << lh;
#pragma unroll
    for (int i = 0; i < 64; ++i) {
      const int lo = ((i >> lh) << (lh + 1)) | (i & (h - 1));
      const float a = v[lo], b = v[lo + h];
      v[lo] = __fadd_rn(a, b);
      v[lo + h] = __fsub_rn(a, b);
    }
  }
}
// These helpers are restated bit for bit by oracle/k2_oracle.c.
__device__ __forceinline__ float bf16_round(float x) { return __bfloat162float(__float2bfloat16_rn(x)); }

// fp32(1/sqrt(128)), the normalisation of the Sylvester H128 block.
constexpr float kHadamardScale = 0.0883883461356163024902343750f;

// exp(x): Cody-Waite range reduction x = n*ln2 + r with ln2 split in two
// parts (the hi/lo split published in fdlibm's e_expf.c: ln2_hi = 0.693145751953125
// has trailing zero bits so n*ln2_hi is exact), then the degree-7 Taylor
// polynomial of exp(r) (coefficients 1/k!) in Horner form and exponent-field
// scaling by 2^n (oracle: k2o_exp).
__device__ __forceinline__ float exp_contract(float x) {
  if (x != x) return x;
  if (x > 88.72283935546875f) return __int_as_float(0x7f800000);
  if (x < -103.972084045410156f) return 0.0f;
  float n = rintf(__fmul_rn(x, 1.44269502162933349609375f));
  float r = __fmaf_rn(n, -0.693145751953125f, x);
  r = __fmaf_rn(n, -1.428606765330187045037746429443359375e-06f, r);
  float p = 1.98412698412698412526e-4f;
  p = __fmaf_rn(p, r, 1.38888888888888894189e-3f);
  p = __fmaf_rn(p, r, 8.33333333333333321769e-3f);
  p = __fmaf_rn(p, r, 4.16666666666666643537e-2f);
  p = __fmaf_rn(p, r, 1.66666666666666657415e-1f);
  p = __fmaf_rn(p, r, 0.5f);
  p = __fmaf_rn(p, r, 1.0f);
  p = __fmaf_rn(p, r, 1.0f);
  int e = (int)n;
  if (e > 127) {
    p = __fmul_rn(p, 1.7014118346046923e38f);
    e -= 127;
  }
  if (e < -126) {
    p = __fmul_rn(p, 1.1754943508222875e-38f);
    e += 126;
  }
  return __fmul_rn(p, __int_as_float((e + 127) << 23));
}
__device__ __forceinline__ float silu_contract(float x) {
  return __fdiv_rn(x, __fadd_rn(1.0f, exp_contract(-x)));
}
__device__ __forceinline__ float sigmoid_contract(float x) {
  return __fdiv_rn(1.0f, __fadd_rn(1.0f, exp_contract(-x)));
}

// ------------------------------------------- group-128 INT4 quantisation
// Input: the 128 raw outputs u of hadamard128_regs (no 1/sqrt(128) applied).
// Contract (oracle: k2o_quant_group128):
//   scale = fp16(min(fp32(max|u| * kQuantScale), 65504)),
//           kQuantScale = fp32(1 / (7 * sqrt(128)))
//   c     = fp32(kHadamardScale * fp32(1 / scale))     (0 for a zero scale)
//   code  = clamp(rne(u * c), -8, 7)                    (exact product)
// The rounding is one fma(u, c, 1.5*2^23 + 8): the sum lies on the integer
// grid, so its fp32 bits are 0x4B400000 + (code + 8) and the low nibble holds
// the offset-8 code.  When the scale is a normal fp16 that was not clamped,
// |u * c| <= 7 * (1 + 2^-11 + 2^-21) < 7.5, so the clamp cannot bind and is
// skipped.  Codes of NaN inputs are unspecified (the scale ignores NaN).
constexpr float kRoundMagic = 12582912.0f;   // 1.5 * 2^23
constexpr float kRoundMagic8 = 12582920.0f;  // 1.5 * 2^23 + 8
constexpr float kQuantScale = 0.012626906856894493103027343750f;
struct QuantGroup {
  __half scale;
  float sd;  // the scale as fp32
  float c;
  bool clamp;
};
__device__ __forceinline__ QuantGroup quant_scale(float amax_raw) {
  QuantGroup g;
  const float sf = __fmul_rn(amax_raw, kQuantScale);
  g.scale = __float2half_rn(fminf(sf, 65504.0f));
  g.sd = __half2float(g.scale);
  g.c = 0.0f;
  g.clamp = !(g.sd >= 6.103515625e-05f) || !(sf <= 65504.0f);
  return g;
}
__device__ __forceinline__ QuantGroup quant_group(float amax_raw) {
  QuantGroup g = quant_scale(amax_raw);
  g.c = g.sd > 0.0f ? __fmul_rn(kHadamardScale, __frcp_rn(g.sd)) : 0.0f;
  return g;
}
// Table form of c: with sd = m * 2^e (m in [1, 2)), fp32(1/sd) = 2^-e *
// fp32(1/m) and fp32(H * 2^-e * r) = 2^-e * fp32(H * r), because scaling by a
// power of two is exact while everything stays normal (every positive fp16,
// its reciprocal and H times it do).  So tab[i] = fp32(H * fp32(1 / (1 +
// i/1024))) over the 1024 fp16 significands gives the contract's c exactly;
// fp16 subnormals are normal fp32 and index the same table.
__device__ __forceinline__ void quant_table_init(float* tab, int tid, int nthreads) {
  for (int i = tid; i < 1024; i += nthreads)
    tab[i] = __fmul_rn(kHadamardScale, __frcp_rn(1.0f + (float)i * (1.0f / 1024.0f)));
}
__device__ __forceinline__ float quant_c_table(float sd, const float* tab) {
  const uint32_t b = __float_as_uint(sd);
  const uint32_t t = __float_as_uint(tab[(b >> 13) & 1023u]);
  return b ? __uint_as_float(t - ((b & 0x7F800000u) - 0x3F800000u)) : 0.0f;
}
// fp32 bits 0x4B400000 + (code + 8): low nibble = code + 8, bits 4..21 zero.
__device__ __forceinline__ uint32_t quant_bits(float u, float c, bool clamp) {
  float r = __fmaf_rn(u, c, kRoundMagic8);
  if (clamp) r = fminf(fmaxf(r, kRoundMagic), kRoundMagic + 15.0f);
  return __float_as_uint(r);
}
// Four INT4 codes (the low 16 bits of w: nibble i = column i, two's
// complement) -> four e4m3 bytes in column order.  Two byte-permute lookups
// (codes 0..7 and codes -8..-1, indexed by the nibble's low three bits) and a
// per-byte select on the nibble's sign bit, itself spread to a byte mask by a
// third byte-permute.  e4m3(v) for v = 0..7: 00 38 40 44 48 4A 4C 4E; for
// v = -8..-1: D0 CE CC CA C8 C4 C0 B8.
__device__ __forceinline__ uint32_t e4m3x4_from_s4x4(uint32_t w) {
  const uint32_t sel = w & 0x7777u;
  const uint32_t pos = __byte_perm(0x44403800u, 0x4E4C4A48u, sel);
  const uint32_t neg = __byte_perm(0xCACCCED0u, 0xB8C0C4C8u, sel);
  const uint32_t m = __byte_perm(0x0000FF00u, 0u, (w >> 3) & 0x1111u);
  return (pos & ~m) | (neg & m);
}
// 32 packed codes (16 bytes, column order) -> 32 e4m3 bytes: lo = columns
// 0..15, hi = columns 16..31.
__device__ __forceinline__ void unpack_chunk(uint4 v, uint4& lo, uint4& hi) {
  lo = make_uint4(e4m3x4_from_s4x4(v.x), e4m3x4_from_s4x4(v.x >> 16), e4m3x4_from_s4x4(v.y),
                  e4m3x4_from_s4x4(v.y >> 16));
  hi = make_uint4(e4m3x4_from_s4x4(v.z), e4m3x4_from_s4x4(v.z >> 16), e4m3x4_from_s4x4(v.w),
                  e4m3x4_from_s4x4(v.w >> 16));
}
// Sum of 0x4B400000 << 4j over j = 0..7, mod 2^32: what the exponent bits of
// eight quant_bits words add to an 8-nibble shift-and-add pack.
__host__ __device__ constexpr uint32_t pack_bias8() {
  uint32_t s = 0;
  for (int j = 0; j < 8; ++j) s += 0x4B400000u << (4 * j);
  return s;
}
// Eight quant_bits words -> eight two's-complement nibbles, element j in
// bits 4j..4j+3.  Bits 4..21 of every word are zero, so the shifted sum of
// the low nibbles carries nothing; the exponent bits add a known constant.
__device__ __forceinline__ uint32_t pack8_codes(const uint32_t (&b)[8]) {
  uint32_t s = b[0];
#pragma unroll
  for (int j = 1; j < 8; ++j) s += b[j] << (4 * j);
  return (s - pack_bias8()) ^ 0x88888888u;
}

}  // namespace k2b
