// Block-sparse causal GQA attention forward on the 5th-generation tensor cores.
//
// Reference: ops/flashprefill_native_forward.py:228-344 (_flash_forward) and
// ops/flashprefill_varlen_func.py:449-575 (_flash_block_sparse_varlen): for each query
// block and each selected key block (ascending), S = (Q K^T) * c with c = scale*log2(e),
// the diagonal block masked causally, online softmax in exp2, P rounded to the input
// dtype for the P V product, O = acc / l stored in the input dtype.  A row whose list is
// empty outputs zeros (the reference starts l at 1.0 and acc at 0).
//
// Persistent kernel, one CTA per SM, 384 threads.  A work item is one query block of two
// query heads ("tiles" a and b); items are handed out heavy-first by an atomic counter.
//   warp 0      scheduler (fetches items into a 2-slot smem ring) + TMA producer of Q and K
//   warp 1      TMEM owner + tcgen05.mma issuer
//   warp 2      TMA producer of V
//   warps 4-7   softmax / epilogue of tile a, warps 8-11 of tile b; one TMEM lane (= one
//               query row) per thread
// MMA issue order per item: S_a(0), S_b(0), then for each block j: PV_a(j), S_a(j+1),
// PV_b(j), S_b(j+1).  The tensor core therefore works on one tile while the other tile's
// softmax runs, and because PV_x(j) is issued before S_x(j+1), O_x is final whenever
// S_x(j+1) completes: the exact running-max rescale of O (as in the reference) never waits.
// TMEM columns: S_a [0,128), S_b [128,256), O_a [256,384), O_b [384,512).  P (16-bit
// pairs) is written over the first 64 columns of S and read by the TS-form MMA.
// The largest P of a row is exactly 1.0, which keeps the bf16 rounding of P at the
// reference's level (a lazy max that lets P grow above 1 adds up to one bf16 ulp of P).
#include "fp_common.cuh"

namespace fpb {

struct AttnArgs {
  SeqProblem P;
  float c;                   // fp32(1/sqrt(D)) * fp32(log2 e)
  const int32_t* idx;        // [hq][tiles_ub][cap] ascending block lists
  const int32_t* cnt;        // [hq][tiles_ub]
  int* counter;              // work-item counter, zero at launch
  int profile;               // accumulate g_attn_prof
  int total_items;           // tiles_ub * pairs
  int pairs;                 // ceil(hq / 2)
  void* out;                 // output base (masked-store path)
  int64_t o_sb, o_ss, o_sh;  // output strides in elements
};

constexpr int kAttnThreads = 384;
#ifndef FPB_SOFTMAX_PROBE
#define FPB_SOFTMAX_PROBE 0
#endif
constexpr bool kSoftmaxProbe = FPB_SOFTMAX_PROBE;
// Register split (per thread): the kernel is compiled for 168 (= 65536 / 384, rounded down
// to a multiple of 8); role warps 0-3 give back to 80 and the two softmax warpgroups grow
// to 208: 128*80 + 256*208 = 63488 <= 384*168 = 64512.  The host refuses to launch unless the compiled
// register count is exactly kAttnLaunchRegs.
constexpr int kAttnLaunchRegs = 168, kAttnRoleRegs = 80, kAttnSoftmaxRegs = 208;
static_assert(128 * kAttnRoleRegs + 256 * kAttnSoftmaxRegs <= kAttnThreads * kAttnLaunchRegs, "register split");

// Opt-in instrumentation (FLASHPREFILL_B200_PROFILE=1): cycles spent per wait / phase,
// summed over CTAs.  Indices: see kProfNames in fp_api.cu.
constexpr int kProfSlots = 24;
__device__ unsigned long long g_attn_prof[kProfSlots];
struct ProfAcc {  // counters live in shared memory, flushed once per CTA
  unsigned long long* sm;
  __device__ void add(int i, unsigned long long c) {
    if (sm) atomicAdd(sm + i, c);
  }
};
__device__ __forceinline__ unsigned long long clk() { return clock64(); }
#define FPB_TW(slot, call)                   \
  ({                                         \
    const unsigned long long t0_ = clk();    \
    const bool r_ = (call);                  \
    pa.add(slot, clk() - t0_);               \
    r_;                                      \
  })
constexpr uint32_t kAttnTile = 128 * 128 * 2;
constexpr uint32_t kAttnHalf = kAttnTile / 2;

__host__ __device__ constexpr size_t attn_smem_bytes() { return (size_t)kAttnTile * 6 + 1024 + 1024; }

// One work item as published by the scheduler in the smem ring.
struct ItemInfo {
  int valid;  // 0: no more work, 1: item, 2: empty slot of the grid (skip)
  int start, len, nb, tile_base, bcoord, qb;
  int h[2];   // query heads of tiles a, b (-1: none)
  int n[2];   // list lengths
  int pad[3];
};

template <typename T>
__global__ void __launch_bounds__(kAttnThreads, 1)
    sparse_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                       const AttnArgs A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                   // [2] tiles
  uint8_t* sK = smem + 2 * kAttnTile;   // [2] slots
  uint8_t* sV = smem + 4 * kAttnTile;   // [2] slots
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * kAttnTile);
  uint64_t* item_full = bars + 0;
  uint64_t* item_empty = bars + 2;
  uint64_t* q_full = bars + 4;
  uint64_t* q_empty = bars + 6;
  uint64_t* k_full = bars + 8;
  uint64_t* k_empty = bars + 10;
  uint64_t* v_full = bars + 12;
  uint64_t* v_empty = bars + 14;
  uint64_t* s_full = bars + 16;
  uint64_t* p_full = bars + 18;
  uint64_t* o_full = bars + 20;
  uint64_t* o_empty = bars + 22;
  uint64_t* mma_done = bars + 24;
  uint64_t* epi = bars + 26;  // [2] bounded sync of a tile's 128 epilogue threads
  ItemInfo* ring = reinterpret_cast<ItemInfo*>(bars + 28);  // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ring + 2);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  unsigned long long* prof_smem = reinterpret_cast<unsigned long long*>(tmem_slot + 4);  // [kProfSlots]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(item_full + i, 1);
      mbar_init(item_empty + i, 2 + 256);
      mbar_init(q_full + i, 1);
      mbar_init(q_empty + i, 1);
      mbar_init(k_full + i, 1);
      mbar_init(k_empty + i, 1);
      mbar_init(v_full + i, 1);
      mbar_init(v_empty + i, 1);
      mbar_init(s_full + i, 1);
      mbar_init(p_full + i, 128);
      mbar_init(o_full + i, 1);
      mbar_init(o_empty + i, 128);
      mbar_init(epi + i, 128);
    }
    mbar_init(mma_done, 1);
    *abort = 0;
    for (int i = 0; i < kProfSlots; ++i) prof_smem[i] = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 512);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  ProfAcc pa;
  // one recording thread per role / per softmax warpgroup (threads 128 and 256)
  pa.sm = (A.profile && (threadIdx.x < 128 ? lane == 0 : (threadIdx.x & 127) == 0)) ? prof_smem : nullptr;
  const unsigned long long t_kernel0 = clk();

  auto list_of = [&](const ItemInfo& f, int h) -> const int32_t* {
    return A.idx + ((int64_t)h * A.P.tiles_ub + f.tile_base + f.qb) * A.P.cap;
  };

  if (warp < 4) {
  regs_dec<kAttnRoleRegs>();
  if (warp == 0) {
    // ------------------------------------------------------------ scheduler + Q/K producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      const uint64_t stream_once = l2_policy_evict_first();
      uint32_t it = 0, kseq = 0, qld[2] = {0, 0};
      while (true) {
        const int slot = it & 1;
        if (!FPB_TW(15, mbar_wait(item_empty + slot, ((it >> 1) & 1) ^ 1, abort))) break;
        ItemInfo f{};
        const int id = atomicAdd(A.counter, 1);
        if (id >= A.total_items) {
          f.valid = 0;
        } else {
          SeqInfo s;
          int qb;
          const bool single = A.pairs < 0;
          const int np = single ? -A.pairs : A.pairs;
          const int pair = id % np;
          if (!decode_item(A.P, id / np, s, qb)) {
            f.valid = 2;
          } else {
            f.valid = 1;
            f.start = s.start;
            f.len = s.len;
            f.nb = s.nb;
            f.tile_base = s.tile_base;
            f.bcoord = s.bcoord;
            f.qb = qb;
            for (int x = 0; x < 2; ++x) {
              const int h = single ? (x == 0 ? pair : A.P.hq) : 2 * pair + x;
              f.h[x] = h < A.P.hq ? h : -1;
              int n = 0;
              if (f.h[x] >= 0) n = __ldg(A.cnt + (int64_t)h * A.P.tiles_ub + s.tile_base + qb);
              f.n[x] = max(0, min(n, qb + 1));
            }
          }
        }
        ring[slot] = f;
        mbar_arrive(item_full + slot);
        if (f.valid == 1) pa.add(19, 1);
        ++it;
        if (f.valid == 0) break;
        if (f.valid == 2) continue;
        const int qrow = f.start + f.qb * kBlock;
        bool ok = true;
        
#pragma unroll
        for (int x = 0; x < 2 && ok; ++x) {
          if (f.h[x] < 0 || f.n[x] == 0) continue;
          if (!FPB_TW(14, mbar_wait(q_empty + x, (qld[x] & 1) ^ 1, abort))) { ok = false; break; }
          ++qld[x];
          uint8_t* dst = sQ + x * kAttnTile;
          mbar_arrive_expect_tx(q_full + x, kAttnTile);
          tma_load_4d_hint(dst, &tm_q, q_full + x, 0, f.h[x], qrow, f.bcoord, stream_once);
          tma_load_4d_hint(dst + kAttnHalf, &tm_q, q_full + x, 64, f.h[x], qrow, f.bcoord, stream_once);
        }
        const int hk[2] = {f.h[0] >= 0 ? f.h[0] / (A.P.hq / A.P.hk) : 0,
                           f.h[1] >= 0 ? f.h[1] / (A.P.hq / A.P.hk) : 0};
        const int32_t* lst[2] = {f.h[0] >= 0 ? list_of(f, f.h[0]) : nullptr, f.h[1] >= 0 ? list_of(f, f.h[1]) : nullptr};
        const int nmax = max(f.n[0], f.n[1]);
        for (int j = 0; j < nmax && ok; ++j) {
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            if (j >= f.n[x]) continue;
            int kb = __ldg(lst[x] + j);
            if (kb < 0 || kb > f.qb) {
              raise_error(A.P.err, kErrIndexRange);
              kb = f.qb;
            }
            const int sl = kseq & 1;
            if (!FPB_TW(13, mbar_wait(k_empty + sl, ((kseq >> 1) & 1) ^ 1, abort))) { ok = false; break; }
            ++kseq;
            uint8_t* dst = sK + sl * kAttnTile;
            const int krow = f.start + kb * kBlock;
            mbar_arrive_expect_tx(k_full + sl, kAttnTile);
            tma_load_4d(dst, &tm_k, k_full + sl, 0, hk[x], krow, f.bcoord);
            tma_load_4d(dst + kAttnHalf, &tm_k, k_full + sl, 64, hk[x], krow, f.bcoord);
          }
        }
        if (!ok) break;
      }
      if (*abort) {  // let loads still in flight land before the CTA exits
        volatile int no_abort = 0;
        for (uint32_t s = (kseq > 2 ? kseq - 2 : 0); s < kseq; ++s) mbar_wait(k_full + (s & 1), (s >> 1) & 1, &no_abort);
        for (int x = 0; x < 2; ++x)
          if (qld[x]) mbar_wait(q_full + x, (qld[x] - 1) & 1, &no_abort);
      }
    }
  } else if (warp == 2) {
    // ------------------------------------------------------------ V producer
    if (lane == 0) {
      prefetch_tmap(&tm_v);
      uint32_t it = 0, vseq = 0;
      while (true) {
        const int slot = it & 1;
        if (!FPB_TW(17, mbar_wait(item_full + slot, (it >> 1) & 1, abort))) break;
        const ItemInfo f = ring[slot];
        mbar_arrive(item_empty + slot);
        ++it;
        if (f.valid == 0) break;
        if (f.valid == 2) continue;
        bool ok = true;
        const int nmax = max(f.n[0], f.n[1]);
        for (int j = 0; j < nmax && ok; ++j) {
#pragma unroll
          for (int x = 0; x < 2; ++x) {
            if (j >= f.n[x]) continue;
            int kb = __ldg(list_of(f, f.h[x]) + j);
            if (kb < 0 || kb > f.qb) kb = f.qb;
            const int hk = f.h[x] / (A.P.hq / A.P.hk);
            const int sl = vseq & 1;
            if (!FPB_TW(16, mbar_wait(v_empty + sl, ((vseq >> 1) & 1) ^ 1, abort))) { ok = false; break; }
            ++vseq;
            uint8_t* dst = sV + sl * kAttnTile;
            const int krow = f.start + kb * kBlock;
            mbar_arrive_expect_tx(v_full + sl, kAttnTile);
            tma_load_4d(dst, &tm_v, v_full + sl, 0, hk, krow, f.bcoord);
            tma_load_4d(dst + kAttnHalf, &tm_v, v_full + sl, 64, hk, krow, f.bcoord);
          }
        }
        if (!ok) break;
      }
      if (*abort) {
        volatile int no_abort = 0;
        for (uint32_t s = (vseq > 2 ? vseq - 2 : 0); s < vseq; ++s) mbar_wait(v_full + (s & 1), (s >> 1) & 1, &no_abort);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(128, 128, DT<T>::is_bf16, false);
      constexpr uint32_t id_o = idesc_f16(128, 128, DT<T>::is_bf16, true);
      uint32_t it = 0, kc = 0, vc = 0, qc[2] = {0, 0}, pc[2] = {0, 0}, oc[2] = {0, 0};
      bool ok = true;
      auto issue_s = [&](int x) -> bool {
        const int sl = kc & 1;
        if (!FPB_TW(1, mbar_wait(k_full + sl, (kc >> 1) & 1, abort))) return false;
        ++kc;
        tc_fence_after();
        const uint32_t q_base = smem_u32(sQ + x * kAttnTile);
        const uint32_t k_base = smem_u32(sK + sl * kAttnTile);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = (ks >> 2) * kAttnHalf + (ks & 3) * 32;
          umma_ss(tmem + x * 128, sdesc_sw128(q_base + off, 16, 1024), sdesc_sw128(k_base + off, 16, 1024), id_s,
                  ks > 0);
        }
        umma_commit(k_empty + sl);
        umma_commit(s_full + x);
        return true;
      };
      while (ok) {
        const int slot = it & 1;
        if (!FPB_TW(4, mbar_wait(item_full + slot, (it >> 1) & 1, abort))) break;
        const ItemInfo f = ring[slot];
        mbar_arrive(item_empty + slot);
        ++it;
        if (f.valid == 0) break;
        if (f.valid == 2) continue;
        bool act[2];
        for (int x = 0; x < 2; ++x) act[x] = f.h[x] >= 0 && f.n[x] > 0;
        
#pragma unroll
        for (int x = 0; x < 2 && ok; ++x) {
          if (!act[x]) continue;
          ok = FPB_TW(3, mbar_wait(q_full + x, qc[x] & 1, abort) && mbar_wait(o_empty + x, (oc[x] & 1) ^ 1, abort));
          ++qc[x];
          ++oc[x];
        }
        for (int x = 0; x < 2 && ok; ++x)
          if (act[x]) ok = issue_s(x);
        const int nmax = max(f.n[0], f.n[1]);
        for (int j = 0; j < nmax && ok; ++j) {
          
#pragma unroll
        for (int x = 0; x < 2 && ok; ++x) {
            if (j >= f.n[x]) continue;
            if (!FPB_TW(0, mbar_wait(p_full + x, pc[x] & 1, abort))) { ok = false; break; }
            ++pc[x];
            const int sl = vc & 1;
            if (!FPB_TW(2, mbar_wait(v_full + sl, (vc >> 1) & 1, abort))) { ok = false; break; }
            ++vc;
            tc_fence_after();
            const uint32_t v_base = smem_u32(sV + sl * kAttnTile);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              // A = P (TMEM, 16-bit pairs: 8 columns per 16 keys); B = V rows ks*16.. (MN-major)
              umma_ts(tmem + 256 + x * 128, tmem + x * 128 + ks * 8,
                      sdesc_sw128(v_base + ks * 2048, kAttnHalf, 1024), id_o, (j > 0 || ks > 0) ? 1u : 0u);
            }
            umma_commit(v_empty + sl);
            if (j == f.n[x] - 1) umma_commit(o_full + x);
            else ok = issue_s(x);
          }
        }
      }
      umma_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort);
    }
  }
  } else {
    regs_inc<kAttnSoftmaxRegs>();
    // ------------------------------------------------------------ softmax + epilogue
    const int x = (warp - 4) >> 2;     // tile
    const int quad = warp & 3;
    const int r = quad * 32 + lane;    // query row within the block (= TMEM lane)
    const int et = r;                  // thread index within the tile's warpgroup
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t t_s = tmem + x * 128 + lane_off;
    const uint32_t t_o = tmem + 256 + x * 128 + lane_off;
    uint8_t* stage = sQ + x * kAttnTile;
    const float c = A.c;
    uint32_t it = 0, sc = 0, oc = 0, ep = 0;
    auto group_sync = [&]() -> bool {  // all 128 threads of this tile, bounded
      mbar_arrive(epi + x);
      return FPB_TW(12, mbar_wait_warp(epi + x, (ep++) & 1, abort));
    };
    while (true) {
      const int slot = it & 1;
      if (!FPB_TW(7, mbar_wait_warp(item_full + slot, (it >> 1) & 1, abort))) break;
      const ItemInfo f = ring[slot];
      mbar_arrive(item_empty + slot);
      ++it;
      if (f.valid == 0) break;
      if (f.valid == 2) continue;
      const int hx = x ? f.h[1] : f.h[0];
      if (hx < 0) continue;
      const int n = x ? f.n[1] : f.n[0];
      const int vr = min(kBlock, f.len - f.qb * kBlock);
      T* orow = reinterpret_cast<T*>(A.out) + (int64_t)f.bcoord * A.o_sb +
                (int64_t)(f.start + f.qb * kBlock) * A.o_ss + (int64_t)hx * A.o_sh;
      if (n == 0) {  // empty list: zeros (the reference's acc = 0, l = 1)
        if (r < vr) {
          uint4* dst = reinterpret_cast<uint4*>(orow + (int64_t)r * A.o_ss);
#pragma unroll
          for (int i = 0; i < 16; ++i) dst[i] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      // lists are ascending and causal, so only the last entry can be the diagonal block
      int last_kb = __ldg(list_of(f, hx) + n - 1);
      if (last_kb < 0 || last_kb > f.qb) last_kb = f.qb;
      const bool last_is_diag = last_kb == f.qb;
      float m_use = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < n; ++j) {
        const bool diag = last_is_diag && j == n - 1;
        if (!FPB_TW(5, mbar_wait_warp<kSoftmaxProbe>(s_full + x, sc & 1, abort))) { ok = false; break; }
        ++sc;
        tc_fence_after();
        // the whole 128-column row of S in registers: four loads, one wait
        const unsigned long long tp1 = clk();
        pa.add(20, 1);
        uint32_t ua[32], ub[32], uc[32], ud[32];
        tmem_ld32(t_s, ua);
        tmem_ld32(t_s + 32, ub);
        tmem_ld32(t_s + 64, uc);
        tmem_ld32(t_s + 96, ud);
        tmem_ld_wait();
        pa.add(22, clk() - tp1);
#define FPB_U(i) ((i) < 32 ? ua[(i)] : (i) < 64 ? ub[(i) - 32] : (i) < 96 ? uc[(i) - 64] : ud[(i) - 96])
        if (diag) {  // only the diagonal block needs the causal mask
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i > r) FPB_U(i) = __float_as_uint(-INFINITY);
        }
        float mx = -INFINITY, m1 = -INFINITY;
#pragma unroll
        for (int i = 0; i < 128; i += 4) {
          mx = max3(mx, __uint_as_float(FPB_U(i)), __uint_as_float(FPB_U(i + 1)));
          m1 = max3(m1, __uint_as_float(FPB_U(i + 2)), __uint_as_float(FPB_U(i + 3)));
        }
        mx = fmaxf(mx, m1);
        const float m_blk = mx * c;
        float scale_o = 1.f;
        if (j == 0) {
          m_use = m_blk;
        } else if (m_blk > m_use) {
          scale_o = ex2_approx(m_use - m_blk);
          m_use = m_blk;
          l *= scale_o;
        }
        const unsigned long long tp3 = clk();
        pa.add(8, tp3 - tp1);
        // P = exp2(s*c - m), written as 16-bit pairs over S columns [0, 64); one pair in
        // four is evaluated on the FMA pipe (exp2_poly2), the rest by ex2.approx.
        const float neg_m = -m_use;
        float rs = 0.f, rs1 = 0.f;
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const int e = ch * 32 + i;
            float x0, x1, p0, p1;
            fma2(x0, x1, __uint_as_float(FPB_U(e)), __uint_as_float(FPB_U(e + 1)), c, c, neg_m, neg_m);
            if (((i >> 1) & 3) == 3) {
              exp2_poly2(x0, x1, p0, p1);  // masked (-inf) entries give 2^-126 here, negligible
            } else {
              p0 = ex2_approx(x0);
              p1 = ex2_approx(x1);
            }
            add2(rs, rs1, rs, rs1, p0, p1);
            pk[i >> 1] = DT<T>::pack(p0, p1);
          }
          tmem_st16(t_s + ch * 16, pk);
        }
#undef FPB_U
        const unsigned long long tst = clk();
        pa.add(10, tst - tp3);
        rs += rs1;
        if (__any_sync(0xffffffffu, scale_o != 1.f)) {
          // O_x holds blocks 0..j-1 (PV_x(j-1) completed before S_x(j) did); rescale it
          // before PV_x(j) is allowed to start (p_full below)
          pa.add(21, 1);
#pragma unroll 1
          for (int h2 = 0; h2 < 2; ++h2) {
            uint32_t oa[32], ob[32];
            tmem_ld32(t_o + h2 * 64, oa);
            tmem_ld32(t_o + h2 * 64 + 32, ob);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) {
              oa[i] = __float_as_uint(__uint_as_float(oa[i]) * scale_o);
              ob[i] = __float_as_uint(__uint_as_float(ob[i]) * scale_o);
            }
            tmem_st32(t_o + h2 * 64, oa);
            tmem_st32(t_o + h2 * 64 + 32, ob);
          }
          pa.add(9, clk() - tst);
        }
        tmem_st_wait();
        pa.add(23, clk() - tst);
        l += rs;
        tc_fence_before();
        mbar_arrive(p_full + x);
      }
      if (!ok) break;
      // ---- epilogue: O / l -> smem (SW128 layout, in the Q tile) -> global
      if (!FPB_TW(6, mbar_wait_warp(o_full + x, oc & 1, abort))) break;
      ++oc;
      tc_fence_after();
      const unsigned long long te0 = clk();
      const float inv = 1.f / l;
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t u[32];
        tmem_ld32(t_o + ch * 32, u);
        tmem_ld_wait();
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 16; ++i)
          pk[i] = DT<T>::pack(__uint_as_float(u[2 * i]) * inv, __uint_as_float(u[2 * i + 1]) * inv);
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4) {
          const int cidx = ch * 4 + q4;  // 16-byte chunk 0..15 of the row
          uint8_t* dst = stage + (cidx >> 3) * kAttnHalf + r * 128 + (((cidx & 7) ^ (r & 7)) << 4);
          *reinterpret_cast<uint4*>(dst) = make_uint4(pk[q4 * 4], pk[q4 * 4 + 1], pk[q4 * 4 + 2], pk[q4 * 4 + 3]);
        }
      }
      tc_fence_before();
      mbar_arrive(o_empty + x);
      fence_proxy_async_smem();
      if (!group_sync()) break;
      if (vr == kBlock) {
        if (et == 0) {
          const int qrow = f.start + f.qb * kBlock;
          tma_store_4d(&tm_o, stage, 0, hx, qrow, f.bcoord);
          tma_store_4d(&tm_o, stage + kAttnHalf, 64, hx, qrow, f.bcoord);
          tma_store_commit_and_wait();
          mbar_arrive(q_empty + x);
        }
      } else {
        for (int e = et; e < vr * 16; e += 128) {
          const int rr = e >> 4, cidx = e & 15;
          const uint4 v =
              *reinterpret_cast<const uint4*>(stage + (cidx >> 3) * kAttnHalf + rr * 128 + (((cidx & 7) ^ (rr & 7)) << 4));
          *reinterpret_cast<uint4*>(orow + (int64_t)rr * A.o_ss + cidx * 8) = v;
        }
        if (!group_sync()) break;
        if (et == 0) mbar_arrive(q_empty + x);
      }
      pa.add(11, clk() - te0);
    }
  }

  if (threadIdx.x == 0) pa.add(18, clk() - t_kernel0);
  tc_fence_before();
  __syncthreads();
  if (A.profile && threadIdx.x < kProfSlots) atomicAdd(&g_attn_prof[threadIdx.x], prof_smem[threadIdx.x]);
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && *abort) raise_error(A.P.err, kErrWaitTimeout);
}

}  // namespace fpb
