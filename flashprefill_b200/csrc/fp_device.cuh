// Device-side building blocks for the sm_100a kernels: mbarriers with bounded waits,
// TMA tile loads/stores, and the tcgen05 (5th-generation tensor core) primitives:
// TMEM allocation, MMA issue/commit, and TMEM <-> register moves.
//
// Every wait in this library is bounded.  A wait that runs out of time (or sees the
// CTA-wide abort flag) returns false; the caller records an error bit in the device
// error word, stops issuing work and falls through to its teardown, so the GPU context
// stays usable and the host reports the failure.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

namespace fpb {

// A single wait never legitimately lasts longer than this; 1 s of global time.
constexpr uint64_t kWaitLimitNs = 1000000000ull;
// The limit the kernels apply (kWaitLimitNs unless a test shortens it through
// fpb_test_set_fault), and the one-shot test hook that makes the next attention launch skip
// one key load so that a wait runs out (the producer that consumes it clears it).
__device__ uint64_t g_wait_limit_ns = kWaitLimitNs;
__device__ int g_test_withhold;
#ifndef FPB_SLEEP_HINT_NS
#define FPB_SLEEP_HINT_NS 20000
#endif
constexpr uint32_t kSleepHintNs = FPB_SLEEP_HINT_NS;  // suspend hint of the sleeping waits

// Error bits written into the device error word (workspace offset 0).
enum : uint32_t {
  kErrWaitTimeout = 1u << 0,   // an mbarrier wait ran out of time
  kErrBadSeqlens = 1u << 1,    // cu_seqlens not monotone / last != total tokens
  kErrSeqTooLong = 1u << 2,    // a sequence is longer than max_seq_len
  kErrIndexRange = 1u << 3,    // a block index outside [0, qb] was read
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// ------------------------------------------------------------------ mbarrier
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
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in hardware until the phase
// completes or about hint_ns elapses, instead of spinning on issue slots.
__device__ __forceinline__ bool mbar_test_sleep(uint64_t* bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}
// Non-blocking probe (never suspends the thread).
__device__ __forceinline__ bool mbar_probe(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n .reg .pred p;\n mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n selp.u32 %0, 1, 0, p;\n}\n"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// The bounded waits below read the global timer only every kTimerEvery polls: a timer read
// per poll, from every spinning thread, would load the SM's special-register path that the
// softmax's exp2 instructions also use.
#ifndef FPB_TIMER_EVERY
#define FPB_TIMER_EVERY 32
#endif
constexpr uint32_t kTimerEvery = FPB_TIMER_EVERY;

// Waits for the phase with the given parity to complete.  Returns false on timeout or
// when another thread of the CTA has raised *abort (the CTA is shutting down).
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_test(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns(), lim = g_wait_limit_ns;
  for (uint32_t i = 1;; ++i) {
    if (mbar_test(bar, parity)) return true;
    if (i % kTimerEvery == 0) {
      if (*abort) return false;
      if (global_timer_ns() - t0 > lim) {
        *abort = 1;
        return false;
      }
    }
  }
}

// The same with non-blocking probes (mbarrier.test_wait) instead of try_wait.
__device__ __forceinline__ bool mbar_wait_probe(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_probe(bar, parity)) return true;
  const uint64_t t0 = global_timer_ns(), lim = g_wait_limit_ns;
  for (uint32_t i = 1;; ++i) {
    if (mbar_probe(bar, parity)) return true;
    if (i % kTimerEvery == 0) {
      if (*abort) return false;
      if (global_timer_ns() - t0 > lim) {
        *abort = 1;
        return false;
      }
    }
  }
}

// Bounded wait that sleeps between polls (for waits that are usually long).
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, volatile int* abort) {
  if (mbar_test_sleep(bar, parity, kSleepHintNs)) return true;
  const uint64_t t0 = global_timer_ns(), lim = g_wait_limit_ns;
  while (true) {
    if (mbar_test_sleep(bar, parity, kSleepHintNs)) return true;
    if (*abort) return false;
    if (global_timer_ns() - t0 > lim) {
      *abort = 1;
      return false;
    }
  }
}
__device__ __forceinline__ bool mbar_wait_warp_sleep(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const uint64_t t0 = global_timer_ns(), lim = g_wait_limit_ns;
  while (true) {
    if (__all_sync(0xffffffffu, mbar_test_sleep(bar, parity, kSleepHintNs))) return true;
    const bool stop = (*abort != 0) || (global_timer_ns() - t0 > lim);
    if (__any_sync(0xffffffffu, stop)) {
      *abort = 1;
      return false;
    }
  }
}

// Warp-uniform variant for warps whose lanes then execute warp-collective instructions
// (tcgen05.ld/st, shuffles): every lane returns the same value.
template <bool kProbe = false>
__device__ __forceinline__ bool mbar_wait_warp(uint64_t* bar, uint32_t parity, volatile int* abort) {
  const uint64_t t0 = global_timer_ns(), lim = g_wait_limit_ns;
  for (uint32_t i = 1;; ++i) {
    const bool done = kProbe ? mbar_probe(bar, parity) : mbar_test(bar, parity);
    if (__all_sync(0xffffffffu, done)) return true;
    if (i % kTimerEvery == 0) {
      const bool stop = (*abort != 0) || (global_timer_ns() - t0 > lim);
      if (__any_sync(0xffffffffu, stop)) {
        *abort = 1;
        return false;
      }
    }
  }
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            int c2, int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], "
      "[%6];" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar))
      : "memory");
}
// Same with an L2 eviction-priority hint (createpolicy result).
__device__ __forceinline__ void tma_load_4d_hint(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                                 int c2, int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, {%2, "
      "%3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(map), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}
__device__ __forceinline__ void tma_store_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.tensor.4d.global.shared::cta.bulk_group [%0, {%1, %2, %3, %4}], [%5];" ::"l"(map),
               "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(src))
               : "memory");
}
__device__ __forceinline__ void tma_store_4d_hint(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                                  int c3, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%1, %2, %3, %4}], [%5], %6;" ::"l"(map),
      "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(smem_u32(src)), "l"(policy)
      : "memory");
}
// 16-byte global store with an L2 cache policy (e.g. evict-first for streamed output).
__device__ __forceinline__ void st_global_hint(uint4* p, uint4 v, uint64_t policy) {
  asm volatile("st.global.L2::cache_hint.v4.u32 [%0], {%1, %2, %3, %4}, %5;" ::"l"(p), "r"(v.x), "r"(v.y), "r"(v.z),
               "r"(v.w), "l"(policy)
               : "memory");
}
// Wait until every bulk store issued by this thread has completed (global writes done).
__device__ __forceinline__ void tma_store_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Commit the bulk stores issued so far and wait until their shared-memory source has been read.
__device__ __forceinline__ void tma_store_commit_and_wait_read() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory");
}
__device__ __forceinline__ void tma_store_commit_and_wait() {
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
  asm volatile("cp.async.bulk.wait_group 0;" ::: "memory");
}
__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
// L2 prefetch of one TMA box (no shared-memory destination, no barrier).
__device__ __forceinline__ void tma_prefetch_4d(const CUtensorMap* map, int c0, int c1, int c2, int c3) {
  asm volatile("cp.async.bulk.prefetch.tensor.4d.L2.global.tile [%0, {%1, %2, %3, %4}];" ::"l"(map), "r"(c0), "r"(c1),
               "r"(c2), "r"(c3)
               : "memory");
}
__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t* dst_smem, uint32_t ncols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(dst_smem)),
               "r"(ncols)
               : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols) : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// D[tmem] (+)= A[smem] * B[smem]^T, kind::f16 (bf16 or fp16 operands, fp32 accumulate).
__device__ __forceinline__ void umma_ss(uint32_t d_tmem, uint64_t a_desc, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}\n" ::"r"(d_tmem),
      "l"(a_desc), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// D[tmem] (+)= A[tmem] * B[smem]^T.
__device__ __forceinline__ void umma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t b_desc, uint32_t idesc,
                                        uint32_t accumulate) {
  asm volatile(
      "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
      " tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n}\n" ::"r"(d_tmem),
      "r"(a_tmem), "l"(b_desc), "r"(idesc), "r"(accumulate)
      : "memory");
}
// Arrive (once) on an mbarrier when every tcgen05.mma issued so far by this thread is done.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
               : "memory");
}

// Shared-memory matrix descriptor for a tile written by TMA with 128-byte swizzling.
// start: smem byte address; lbo/sbo: leading / stride byte offsets.  Bits 46-48 hold the
// fixed value 0b001; bits 61-63 select the 128B swizzle mode (value 2).
__device__ __forceinline__ uint64_t sdesc_sw128(uint32_t start, uint32_t lbo, uint32_t sbo) {
  uint64_t d = 0;
  d |= (uint64_t)((start & 0x3FFFFu) >> 4);
  d |= (uint64_t)((lbo >> 4) & 0x3FFFu) << 16;
  d |= (uint64_t)((sbo >> 4) & 0x3FFFu) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// Instruction descriptor for kind::f16: fp32 accumulator, A/B both bf16 (or both fp16),
// A K-major, B K-major (b_mn_major=0) or MN-major (b_mn_major=1), shape M x N.
__host__ __device__ constexpr uint32_t idesc_f16(int M, int N, bool bf16, bool b_mn_major) {
  return (1u << 4) | ((bf16 ? 1u : 0u) << 7) | ((bf16 ? 1u : 0u) << 10) | ((b_mn_major ? 1u : 0u) << 16) |
         ((uint32_t)(N >> 3) << 17) | ((uint32_t)(M >> 4) << 24);
}

#define FPB_R32(a) \
  "=r"(a[0]), "=r"(a[1]), "=r"(a[2]), "=r"(a[3]), "=r"(a[4]), "=r"(a[5]), "=r"(a[6]), "=r"(a[7]), "=r"(a[8]), \
      "=r"(a[9]), "=r"(a[10]), "=r"(a[11]), "=r"(a[12]), "=r"(a[13]), "=r"(a[14]), "=r"(a[15]), "=r"(a[16]),  \
      "=r"(a[17]), "=r"(a[18]), "=r"(a[19]), "=r"(a[20]), "=r"(a[21]), "=r"(a[22]), "=r"(a[23]), "=r"(a[24]),  \
      "=r"(a[25]), "=r"(a[26]), "=r"(a[27]), "=r"(a[28]), "=r"(a[29]), "=r"(a[30]), "=r"(a[31])
#define FPB_W32(a)                                                                                                \
  "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7]), "r"(a[8]), "r"(a[9]),  \
      "r"(a[10]), "r"(a[11]), "r"(a[12]), "r"(a[13]), "r"(a[14]), "r"(a[15]), "r"(a[16]), "r"(a[17]), "r"(a[18]), \
      "r"(a[19]), "r"(a[20]), "r"(a[21]), "r"(a[22]), "r"(a[23]), "r"(a[24]), "r"(a[25]), "r"(a[26]), "r"(a[27]), \
      "r"(a[28]), "r"(a[29]), "r"(a[30]), "r"(a[31])

// Thread i of the warp receives 32 consecutive 32-bit columns [col, col+32) of TMEM lane
// (lane base of taddr) + i.  A warp may only touch the 32-lane quarter (warp_id % 4).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : FPB_R32(r)
      : "r"(taddr));
}
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32};" ::"r"(taddr),
      FPB_W32(r)
      : "memory");
}
#define FPB_W16(a)                                                                                               \
  "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(a[4]), "r"(a[5]), "r"(a[6]), "r"(a[7]), "r"(a[8]), "r"(a[9]), \
      "r"(a[10]), "r"(a[11]), "r"(a[12]), "r"(a[13]), "r"(a[14]), "r"(a[15])
__device__ __forceinline__ void tmem_st16(uint32_t taddr, const uint32_t (&r)[16]) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], {%1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16};" ::"r"(taddr),
      FPB_W16(r)
      : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() { asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory"); }
__device__ __forceinline__ void tmem_st_wait() { asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory"); }

// ------------------------------------------------------------------ misc
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// ---- packed fp32 pairs (sm_100 f32x2 instructions) and 3-input max
__device__ __forceinline__ void fma2(float& d0, float& d1, float a0, float a1, float b0, float b1, float c0, float c1) {
  asm("{\n .reg .b64 ra, rb, rc, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n mov.b64 rc, {%6, %7};\n"
      " fma.rn.f32x2 rd, ra, rb, rc;\n mov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1), "f"(c0), "f"(c1));
}
__device__ __forceinline__ void add2(float& d0, float& d1, float a0, float a1, float b0, float b1) {
  asm("{\n .reg .b64 ra, rb, rd;\n mov.b64 ra, {%2, %3};\n mov.b64 rb, {%4, %5};\n"
      " add.rn.f32x2 rd, ra, rb;\n mov.b64 {%0, %1}, rd;\n}\n"
      : "=f"(d0), "=f"(d1)
      : "f"(a0), "f"(a1), "f"(b0), "f"(b1));
}
__device__ __forceinline__ float max3(float a, float b, float c) {
  float d;
  asm("max.f32 %0, %1, %2, %3;" : "=f"(d) : "f"(a), "f"(b), "f"(c));
  return d;
}

// 2^x for a pair of x <= 0 on the FMA pipe (takes load off the 16/clk/SM MUFU unit).
// Cody-Waite style split x = n + f with n = round(x) (adding 1.5*2^23 rounds to an integer)
// and f in [-0.5, 0.5]; 2^f by a degree-3 polynomial whose coefficients were fitted here
// for minimal relative error with the constant term fixed to 1 (so 2^0 = 1 exactly; max
// relative error 1.0e-4, far below the 2^-9 of the bf16 P it feeds); 2^n is applied by
// adding n to the exponent field.  x is clamped at -126 (the result there is < 2^-125).
__device__ __forceinline__ void exp2_poly2(float x0, float x1, float& y0, float& y1) {
  constexpr float kShift = 12582912.0f;  // 1.5 * 2^23
  constexpr float C1 = 0.6932829022407532f, C2 = 0.2422109693288803f, C3 = 0.05500892922282219f;
  x0 = fmaxf(x0, -126.f);
  x1 = fmaxf(x1, -126.f);
  float j0, j1, t0, t1, f0, f1, p0, p1;
  add2(j0, j1, x0, x1, kShift, kShift);
  add2(t0, t1, j0, j1, -kShift, -kShift);
  fma2(f0, f1, t0, t1, -1.f, -1.f, x0, x1);
  fma2(p0, p1, C3, C3, f0, f1, C2, C2);
  fma2(p0, p1, p0, p1, f0, f1, C1, C1);
  fma2(p0, p1, p0, p1, f0, f1, 1.f, 1.f);
  y0 = __int_as_float(__float_as_int(p0) + (__float_as_int(j0) << 23));
  y1 = __int_as_float(__float_as_int(p1) + (__float_as_int(j1) << 23));
}

// Register reallocation between warpgroups.  The sum over the CTA must not exceed the
// registers the CTA was launched with (the host checks the kernel's register count).
template <int N>
__device__ __forceinline__ void regs_inc() { asm volatile("setmaxnreg.inc.sync.aligned.u32 %0;" ::"n"(N)); }
template <int N>
__device__ __forceinline__ void regs_dec() { asm volatile("setmaxnreg.dec.sync.aligned.u32 %0;" ::"n"(N)); }

__device__ __forceinline__ void named_bar_sync(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Ordered-int encoding so that atomicMax on int gives the float maximum.
__device__ __forceinline__ int float_to_ordered(float f) {
  int i = __float_as_int(f);
  return i >= 0 ? i : i ^ 0x7FFFFFFF;
}
__device__ __forceinline__ float ordered_to_float(int i) { return __int_as_float(i >= 0 ? i : i ^ 0x7FFFFFFF); }

template <typename T>
struct DT;
template <>
struct DT<__nv_bfloat16> {
  static constexpr bool is_bf16 = true;
  __device__ static __forceinline__ uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  // the two values of a packed pair, widened back to fp32 (exact)
  __device__ static __forceinline__ float lo(uint32_t p) { return __uint_as_float(p << 16); }
  __device__ static __forceinline__ float hi(uint32_t p) { return __uint_as_float(p & 0xFFFF0000u); }
  __device__ static __forceinline__ float to_f(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ static __forceinline__ __nv_bfloat16 from_f(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct DT<__half> {
  static constexpr bool is_bf16 = false;
  __device__ static __forceinline__ uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ static __forceinline__ float lo(uint32_t p) { return __half2float(__ushort_as_half((unsigned short)p)); }
  __device__ static __forceinline__ float hi(uint32_t p) {
    return __half2float(__ushort_as_half((unsigned short)(p >> 16)));
  }
  __device__ static __forceinline__ float to_f(__half x) { return __half2float(x); }
  __device__ static __forceinline__ __half from_f(float x) { return __float2half_rn(x); }
};

}  // namespace fpb
