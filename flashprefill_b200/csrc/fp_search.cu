// Fused block search: pooled-key scores, per-block max / exp-sum, normalisation,
// threshold + structural rules, and compaction into an ascending int32 block list --
// one CTA per (query block, query head), nothing but the list and its count written.
//
// Reference semantics (paths relative to the reference project):
//   scores   ops/flashprefill_native_forward.py:129-188, ops/flashprefill_varlen_func.py:158-217
//            s[r,kb] = c * (q_r . mk_kb), c = fp32(1/sqrt(D)) * fp32(log2 e); row r of query
//            block qb is causal for kb iff qb*128 + r >= kb*128 + 127 (so the diagonal block
//            sees only row 127, and zero-padded rows past the sequence end count as s = 0);
//            m[kb] = max_r s, p[kb] = sum_r exp2(s - m).
//   normalise native:388-403 (dense: pw / (sum pw + 1e-9)), varlen:240-304,656 (pw only),
//            pw[kb] = p[kb] * exp2(m[kb] - max_kb m).
//   select   native:347-385, varlen:327-409: score >= alpha * max score, or kb < sink, or
//            0 <= qb - kb < window, or qb >= nb - last_n; AND kb <= qb.  Dense min_budget > 0
//            also forces the top-min_budget scores in (ties: lower block index first).
//   output   ascending block indices (what the reference's sort / boolean compaction yields,
//            native:379-383, varlen:683-698) and the per-row count.
//
// The reference materialises (NB, NB, Hq) fp32 score and max tensors and sorts an int64
// copy; here everything after the MMA stays on chip.  Roles (192 threads): warp 0 issues
// TMA loads (query block once, pooled-key tiles of 128 blocks into a 2-stage ring), warp 1
// issues tcgen05.mma D[kb, r] = mk_kb . q_r into a double-buffered 128x128 fp32 TMEM
// accumulator, warps 2-5 read one TMEM lane (= one key block) each and reduce its 128
// query rows.
//
// exp2 work is skipped where it cannot change the result: with M = max_kb m, every
// block's pw <= 128 * 2^(m - M) while the best block has pw >= 1, so a block with
// m < M + log2(alpha) - 8 scores below alpha/2 of the maximum and cannot pass the
// threshold.  A running lower bound of M is used while scanning, which only widens the
// set of evaluated blocks.  (With min_budget > 0 every causal block is evaluated.)
#include "fp_common.cuh"

namespace fpb {

struct SearchArgs {
  SeqProblem P;
  float c;          // score scale in log2 units
  float alpha;
  float cand_off;   // log2(alpha) - 8, or -inf to evaluate every block
  int sink, window, last_n, min_budget;
  int normalize;    // dense path: divide by (sum + 1e-9)
  int32_t* idx;     // [hq][tiles_ub][cap]
  int32_t* cnt;     // [hq][tiles_ub]
  int* counter;     // persistent kernel: work-item counter, zero at launch
  int total_items;  // persistent kernel: tiles_ub * hq
  unsigned long long* prof;  // persistent kernel: optional per-phase cycle sums (kSpSlots)
};
// Instrumentation of the persistent search: compiled in with -DFPB_SEARCH_PROFILE=1, enabled
// at run time with FLASHPREFILL_B200_SEARCH_PROFILE=1.
#ifndef FPB_SEARCH_PROFILE
#define FPB_SEARCH_PROFILE 0
#endif
enum SearchProf {
  kSpProdItem, kSpProdQ, kSpProdMk, kSpMmaQ, kSpMmaMk, kSpMmaAcc, kSpEpiItem, kSpEpiArr, kSpEpiAcc, kSpEpiLd,
  kSpEpiMax, kSpEpiExp, kSpEpiTiles, kSpEpiExpTiles, kSpSelItem, kSpSelArr, kSpSelWork, kSpCta, kSpSlots
};
static const char* const kSearchProfNames[kSpSlots] = {
    "prod_wait_item_slot", "prod_wait_q_slot", "prod_wait_mk_stage", "mma_wait_q", "mma_wait_mk", "mma_wait_acc",
    "epi_wait_item", "epi_wait_arrays", "epi_wait_acc", "epi_tmem_ld", "epi_max_pass", "epi_exp_pass", "epi_tiles",
    "epi_tiles_with_exp", "sel_wait_item", "sel_wait_arrays", "sel_work", "cta_cycles"};

constexpr int kSearchThreads = 192;
constexpr uint32_t kTileBytes = 128 * 128 * 2;  // one 128x128 16-bit tile (two 64-column TMA boxes)
constexpr uint32_t kHalfTile = kTileBytes / 2;

__host__ __device__ constexpr size_t search_smem_bytes(int cap) {
  // Q + 2 pooled-key stages + m/p arrays + top-k marks + barriers/scalars + alignment slack
  return 3 * (size_t)kTileBytes + 8 * (size_t)cap + (size_t)((cap + 31) / 32) * 4 + 384 + 1024;
}

// Sum / max over a group of 128 threads (four warps from warp `base`), using named barrier
// `bar` (the group's warps only).
template <int kBase = 2, int kBar = 1>
__device__ __forceinline__ float epi_reduce_sum(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  const int wq = (threadIdx.x >> 5) - kBase;
  named_bar_sync(kBar, 128);
  if ((threadIdx.x & 31) == 0) red[wq] = v;
  named_bar_sync(kBar, 128);
  return (red[0] + red[1]) + (red[2] + red[3]);
}
template <int kBase = 2, int kBar = 1>
__device__ __forceinline__ float epi_reduce_max(float v, float* red) {
#pragma unroll
  for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  const int wq = (threadIdx.x >> 5) - kBase;
  named_bar_sync(kBar, 128);
  if ((threadIdx.x & 31) == 0) red[wq] = v;
  named_bar_sync(kBar, 128);
  return fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
}

template <typename T>
__global__ void __launch_bounds__(kSearchThreads, 1)
    block_search_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_mk,
                        const SearchArgs A) {
  const int hq = blockIdx.x % A.P.hq;
  SeqInfo s;
  int qb;
  if (!decode_item(A.P, blockIdx.x / A.P.hq, s, qb)) return;
  const int hk = hq / (A.P.hq / A.P.hk);
  const int row = s.tile_base + qb;
  int32_t* out_idx = A.idx + ((int64_t)hq * A.P.tiles_ub + row) * A.P.cap;
  int32_t* out_cnt = A.cnt + (int64_t)hq * A.P.tiles_ub + row;

  // Rows in the last-N band, or alpha <= 0: every causal block is selected.
  if (qb >= s.nb - A.last_n || A.alpha <= 0.f) {
    for (int kb = threadIdx.x; kb <= qb; kb += blockDim.x) out_idx[kb] = kb;
    if (threadIdx.x == 0) *out_cnt = qb + 1;
    return;
  }

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sMK = smem + kTileBytes;  // 2 stages
  float* m_arr = reinterpret_cast<float*>(smem + 3 * kTileBytes);
  float* p_arr = m_arr + A.P.cap;
  uint32_t* marks = reinterpret_cast<uint32_t*>(p_arr + A.P.cap);
  uint8_t* tail = reinterpret_cast<uint8_t*>(marks + (A.P.cap + 31) / 32);
  tail = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(tail) + 15) & ~uintptr_t(15));
  uint64_t* bars = reinterpret_cast<uint64_t*>(tail);
  uint64_t* q_full = bars + 0;
  uint64_t* mk_full = bars + 1;    // [2]
  uint64_t* mk_empty = bars + 3;   // [2]
  uint64_t* acc_full = bars + 5;   // [2]
  uint64_t* acc_empty = bars + 7;  // [2]
  uint64_t* mma_done = bars + 9;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 10);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* mrun = reinterpret_cast<int*>(tmem_slot + 2);
  float* red = reinterpret_cast<float*>(tmem_slot + 4);   // 4 floats
  int* red_i = reinterpret_cast<int*>(tmem_slot + 8);     // 4 ints
  int* red_k = reinterpret_cast<int*>(tmem_slot + 12);    // 4 ints
  int* failed_flag = reinterpret_cast<int*>(tmem_slot + 16);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int ntiles = qb / kBlock + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(mk_full + i, 1);
      mbar_init(mk_empty + i, 1);
      mbar_init(acc_full + i, 1);
      mbar_init(acc_empty + i, 128);
    }
    mbar_init(mma_done, 1);
    *abort = 0;
    *mrun = float_to_ordered(-INFINITY);
    *failed_flag = 0;
    fence_mbar_init();
  }
  if (warp == 1) {
    tmem_alloc(tmem_slot, 256);
    tmem_relinquish();
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_mk);
      const int qrow = s.start + qb * kBlock - A.P.q_off;  // may be negative: rows before the chunk load as zeros
      mbar_arrive_expect_tx(q_full, kTileBytes);
      tma_load_4d(sQ, &tm_q, q_full, 0, hq, qrow, s.bcoord);
      tma_load_4d(sQ + kHalfTile, &tm_q, q_full, 64, hq, qrow, s.bcoord);
      int issued = 0;
      for (int t = 0; t < ntiles; ++t) {
        const int st = t & 1;
        if (!mbar_wait(mk_empty + st, ((t >> 1) & 1) ^ 1, abort)) break;
        mbar_arrive_expect_tx(mk_full + st, kTileBytes);
        uint8_t* dst = sMK + st * kTileBytes;
        const int mrow = s.tile_base + t * kBlock;
        tma_load_4d(dst, &tm_mk, mk_full + st, 0, hk, mrow, 0);
        tma_load_4d(dst + kHalfTile, &tm_mk, mk_full + st, 64, hk, mrow, 0);
        issued = t + 1;
      }
      if (*abort) {  // let loads still in flight land before the CTA exits
        volatile int no_abort = 0;
        for (int t = (issued > 2 ? issued - 2 : 0); t < issued; ++t)
          mbar_wait(mk_full + (t & 1), (t >> 1) & 1, &no_abort);
        mbar_wait(q_full, 0, &no_abort);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(128, 128, DT<T>::is_bf16, false);
      const uint32_t q_base = smem_u32(sQ);
      if (mbar_wait(q_full, 0, abort)) {
        for (int t = 0; t < ntiles; ++t) {
          const int st = t & 1, acc = t & 1;
          if (!mbar_wait(mk_full + st, (t >> 1) & 1, abort)) break;
          if (!mbar_wait(acc_empty + acc, ((t >> 1) & 1) ^ 1, abort)) break;
          tc_fence_after();
          const uint32_t a_base = smem_u32(sMK + st * kTileBytes);
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t off = (ks >> 2) * kHalfTile + (ks & 3) * 32;
            umma_ss(tmem + acc * 128, sdesc_sw128(a_base + off, 16, 1024), sdesc_sw128(q_base + off, 16, 1024),
                    idesc, ks > 0);
          }
          umma_commit(mk_empty + st);
          umma_commit(acc_full + acc);
        }
      }
      umma_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort);
    }
  } else {
    // ------------------------------------------------------------ epilogue (warps 2..5)
    const int quad = warp & 3;
    const int et = threadIdx.x - 64;       // 0..127 within the epilogue group
    const int lrow = quad * 32 + lane;     // TMEM lane = key block within the tile
    const int vr = min(kBlock, s.len - qb * kBlock);  // valid query rows of this block
    const float c = A.c;
    bool ok = true;
    for (int t = 0; t < ntiles; ++t) {
      const int acc = t & 1;
      if (!mbar_wait_warp(acc_full + acc, (t >> 1) & 1, abort)) { ok = false; break; }
      tc_fence_after();
      const int kb = t * kBlock + lrow;
      const uint32_t taddr = tmem + acc * 128 + ((uint32_t)(quad * 32) << 16);
      // the 128 scores of this key block, kept in registers for both passes
      uint32_t ua[32], ub[32], uc[32], ud[32];
      tmem_ld32(taddr, ua);
      tmem_ld32(taddr + 32, ub);
      tmem_ld32(taddr + 64, uc);
      tmem_ld32(taddr + 96, ud);
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(acc_empty + acc);  // the accumulator may be overwritten by tile t + 2
#define FPB_S(i) __uint_as_float((i) < 32 ? ua[(i)] : (i) < 64 ? ub[(i) - 32] : (i) < 96 ? uc[(i) - 64] : ud[(i) - 96])
      float mx, s127;
      if (vr == kBlock) {
        float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
        for (int i = 0; i < 128; i += 4) {
          m0 = max3(m0, FPB_S(i), FPB_S(i + 1));
          m1 = max3(m1, FPB_S(i + 2), FPB_S(i + 3));
        }
        mx = fmaxf(m0, m1);
        s127 = FPB_S(127);
      } else {  // a sequence's last, partial query block: padded rows have q = 0, s = 0
        mx = 0.f;
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i < vr) mx = fmaxf(mx, FPB_S(i));
        s127 = 0.f;
      }
      const bool causal = kb <= qb;
      const bool diag = kb == qb;
      float m = -INFINITY;
      if (causal) m = __fmul_rn(diag ? s127 : mx, c);
      // running lower bound of the row maximum
      float wm = m;
#pragma unroll
      for (int o = 16; o; o >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, o));
      const float m_est = fmaxf(wm, ordered_to_float(*(volatile int*)mrun));
      if (lane == 0 && wm > -INFINITY) atomicMax(mrun, float_to_ordered(wm));
      const bool cand = causal && (m >= m_est + A.cand_off);
      float p = 0.f;
      if (__any_sync(0xffffffffu, cand && !diag)) {
        // p = sum_r exp2(s_r c - m): one FMA per score (the reference rounds s c first; the
        // difference is below one ulp of the exponent and only matters at the threshold)
        const float nm = -m;
        float p0 = 0.f, p1 = 0.f;
        if (vr == kBlock) {
#pragma unroll
          for (int i = 0; i < 128; i += 2) {
            float x0, x1;
            fma2(x0, x1, FPB_S(i), FPB_S(i + 1), c, c, nm, nm);
            add2(p0, p1, p0, p1, ex2_approx(x0), ex2_approx(x1));
          }
          p = p0 + p1;
        } else {
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i < vr) p += ex2_approx(__fmaf_rn(FPB_S(i), c, nm));
          p += (float)(kBlock - vr) * ex2_approx(-m);
        }
      }
#undef FPB_S
      if (diag) p = 1.f;
      if (causal) {
        m_arr[kb] = m;
        p_arr[kb] = cand ? p : -1.f;
      }
    }
    // ---- normalise, threshold, compact (the failure decision is taken once for all 4 warps)
    if (!ok) *failed_flag = 1;
    named_bar_sync(1, 128);
    if (et == 0 && *abort) *failed_flag = 1;
    named_bar_sync(1, 128);
    const bool failed = *(volatile int*)failed_flag != 0;
    if (failed) {
      if (et == 0) *out_cnt = 0;
    } else {
      const float M = ordered_to_float(*(volatile int*)mrun);
      // pw[kb] = p[kb] * 2^(m[kb] - M).  The reference selects score >= alpha * max score with
      // score = pw / (sum pw + 1e-9) on the dense path and score = pw on the varlen path; both
      // are the test pw >= alpha * max pw up to the rounding of one division, which moves the
      // decision only for scores within a few ulps of the threshold.
      float best = 0.f;
      for (int kb = et; kb <= qb; kb += 128) {
        const float pv = p_arr[kb];
        const float pw = pv >= 0.f ? __fmul_rn(pv, ex2_approx(__fsub_rn(m_arr[kb], M))) : -1.f;
        p_arr[kb] = pw;
        best = fmaxf(best, pw);
      }
      const float thr = __fmul_rn(epi_reduce_max(best, red), A.alpha);
      // dense min_budget: force the top-k scores in (ties -> lower block index)
      const int nwords = (qb + 1 + 31) / 32;
      const int kbudget = min(A.min_budget, qb + 1);
      if (kbudget > 0) {
        for (int wd = et; wd < nwords; wd += 128) marks[wd] = 0u;
        named_bar_sync(1, 128);
      }
      for (int it = 0; it < kbudget; ++it) {
        float bv = -INFINITY;
        int bk = 0x7fffffff;
        for (int kb = et; kb <= qb; kb += 128) {
          if (marks[kb >> 5] & (1u << (kb & 31))) continue;
          const float v = fmaxf(p_arr[kb], 0.f);
          if (v > bv || (v == bv && kb < bk)) { bv = v; bk = kb; }
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) {
          const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
          const int ok2 = __shfl_xor_sync(0xffffffffu, bk, o);
          if (ov > bv || (ov == bv && ok2 < bk)) { bv = ov; bk = ok2; }
        }
        const int wq = warp - 2;
        if (lane == 0) { red[wq] = bv; red_k[wq] = bk; }
        named_bar_sync(1, 128);
        if (et == 0) {
          float v0 = red[0];
          int k0 = red_k[0];
          for (int j = 1; j < 4; ++j)
            if (red[j] > v0 || (red[j] == v0 && red_k[j] < k0)) { v0 = red[j]; k0 = red_k[j]; }
          if (k0 <= qb) marks[k0 >> 5] |= 1u << (k0 & 31);
        }
        named_bar_sync(1, 128);
      }
      // selection + ascending compaction: thread et owns the contiguous blocks
      // [et * chunk, et * chunk + chunk); one block-wide exclusive scan of the counts
      const int chunk = (qb + 128) / 128;  // ceil((qb + 1) / 128)
      const int kb0 = et * chunk, kb1 = min(qb + 1, kb0 + chunk);
      auto selected = [&](int kb) -> bool {
        const float pw = p_arr[kb];
        bool sel = (pw >= 0.f && pw >= thr) || kb < A.sink || (qb - kb) < A.window;
        if (kbudget > 0) sel = sel || ((marks[kb >> 5] >> (kb & 31)) & 1u);
        return sel;
      };
      int mine = 0;
      for (int kb = kb0; kb < kb1; ++kb) mine += selected(kb);
      int incl = mine;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
      }
      const int wq = warp - 2;
      if (lane == 31) red_i[wq] = incl;
      named_bar_sync(1, 128);
      int pre = incl - mine;
      for (int j = 0; j < wq; ++j) pre += red_i[j];
      const int base = red_i[0] + red_i[1] + red_i[2] + red_i[3];
      for (int kb = kb0; kb < kb1; ++kb)
        if (selected(kb)) out_idx[pre++] = kb;
      if (et == 0) *out_cnt = base;
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 256);
  }
  if (threadIdx.x == 0 && *abort) raise_error(A.P.err, kErrWaitTimeout);
}

// ---------------------------------------------------------------------------------------
// Persistent variant (sequences of up to kSearchMaxCap blocks): one CTA per SM loops over
// the same (query block, head) items, fetched heavy-first from an atomic counter, so the
// per-item latencies overlap instead of adding up:
//   warp 0      scheduler + TMA producer: item ring, query block (2 slots), pooled-key tiles
//               (2 stages)
//   warp 1      TMEM owner + tcgen05.mma issuer (double-buffered accumulator)
//   warps 4-7 / 8-11  tile epilogue groups 0 / 1 (the tiles with even / odd global index):
//               per key block m and p (as above) into per-item arrays (double-buffered, so
//               the next item's tiles proceed while ...)
//   warps 12-15 / 16-19  selection groups 0 / 1: ... the previous items (array slot 0 / 1)
//               are normalised, thresholded and compacted.
// Warps 2 and 3 are idle: every SM sub-partition (warp % 4) then holds one role or idle
// warp, two epilogue warps and two selection warps, which matters because each
// sub-partition has its own quarter of the register file.
constexpr int kSearchPThreads = 640;
// Register split: compiled for 96 (= 65536 / 640, rounded down to a multiple of 8); role,
// idle and selection warps give back to 64, the epilogue warps grow to 144: per
// sub-partition 3*64 + 2*144 = 480 = 5*96.
// Tile-epilogue groups (4 warps each, tiles dealt round robin) and selection groups (4 warps
// each, items dealt round robin); the two counts add up to 4.  Measured at 128K: 2 + 2 gives a
// 0.803 ms search stage, 3 + 1 0.811 ms (cfg3: 2.25 / 2.31 ms).
#ifndef FPB_SEARCH_EPI_GROUPS
#define FPB_SEARCH_EPI_GROUPS 2
#endif
constexpr int kSearchEpiGroups = FPB_SEARCH_EPI_GROUPS, kSearchSelGroups = 4 - kSearchEpiGroups;
static_assert(kSearchEpiGroups >= 2 && kSearchEpiGroups <= 3, "epilogue groups");
constexpr int kSearchSelWarp0 = 4 + 4 * kSearchEpiGroups;  // first selection warp
constexpr int kSearchPLaunchRegs = 96, kSearchPRoleRegs = 64, kSearchPEpiRegs = kSearchEpiGroups == 2 ? 144 : 112;
static_assert((128 + 128 * kSearchSelGroups) * kSearchPRoleRegs + 128 * kSearchEpiGroups * kSearchPEpiRegs <=
                  kSearchPThreads * kSearchPLaunchRegs, "split");
constexpr int kSearchRing = 4;
// 1: one exp2 pair in four of the persistent search's exp pass on the FMA pipe; 0: all on MUFU
// (measured at 128K: 0.807 ms with all on MUFU, 0.813 with the quarter on the FMA pipe)
#ifndef FPB_SEARCH_POLY
#define FPB_SEARCH_POLY 0
#endif
constexpr bool kSearchPoly = FPB_SEARCH_POLY;
constexpr int kSearchMaxCap = 2048;
constexpr int kSearchStages = 4;  // pooled-key tiles in flight and TMEM accumulators (2 per epilogue group)

__host__ __device__ constexpr size_t search_p_smem_bytes(int cap) {
  // Q x2, pooled keys x4, two item slots of (m, p, top-k marks), barriers / ring, alignment
  return (2 + kSearchStages) * (size_t)kTileBytes + 2 * (8 * (size_t)cap + (size_t)((cap + 31) / 32) * 4) + 1024 +
         1024;
}

// Tiles of a row are visited last first (diagonal and window blocks), then from the first
// (sink blocks): the blocks that usually hold the row maximum come first, so the running
// estimate that lets the exp2 pass skip most key blocks is close to final early.
__device__ __forceinline__ int tile_order(int j, int ntiles) { return j == 0 ? ntiles - 1 : j - 1; }

struct SearchItem {
  int valid;  // 0: no more work, 1: item, 2: empty slot of the grid (skip)
  int fast;   // every causal block selected (last-N rows or alpha <= 0): no tiles
  int start, len, tile_base, bcoord, qb, h;
  int pad[8];
};

template <typename T>
__global__ void __launch_bounds__(kSearchPThreads, 1)
    block_search_persistent_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_mk,
                                   const SearchArgs A) {
#if FPB_SEARCH_PROFILE
  const long long t_k0 = clock64();
  // per-role accumulators (one recording thread per role), flushed at the end
  unsigned long long pacc[kSpSlots] = {};
#define SP_TW(slot, call)                        \
  ({                                             \
    const long long t0_ = clock64();             \
    const bool r_ = (call);                      \
    if (A.prof) pacc[slot] += clock64() - t0_;   \
    r_;                                          \
  })
#define SP_T() clock64()
#define SP_ON (A.prof != nullptr)
#else
#define SP_TW(slot, call) (call)
#define SP_T() 0ll
#define SP_ON false
  unsigned long long pacc[kSpSlots];
#endif
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                   // [2]
  uint8_t* sMK = smem + 2 * kTileBytes;  // [stages]
  const int cap = A.P.cap;
  const int ncw = (cap + 31) / 32;
  float* arr = reinterpret_cast<float*>(smem + (2 + kSearchStages) * kTileBytes);  // [2]{m[cap], p[cap]}
  uint32_t* marks_all = reinterpret_cast<uint32_t*>(arr + 4 * cap);  // [2][ncw]
  uint8_t* misc = reinterpret_cast<uint8_t*>(
      (reinterpret_cast<uintptr_t>(marks_all + 2 * ncw) + 15) & ~uintptr_t(15));
  uint64_t* bars = reinterpret_cast<uint64_t*>(misc);
  uint64_t* item_full = bars + 0;    // [ring]
  uint64_t* item_empty = bars + 4;   // [ring]
  uint64_t* q_full = bars + 8;       // [2]
  uint64_t* q_empty = bars + 10;     // [2]
  uint64_t* arr_full = bars + 12;    // [2] an item's m / p complete
  uint64_t* arr_empty = bars + 14;   // [2] an item's m / p consumed
  uint64_t* mma_done = bars + 16;
  uint64_t* mk_full = bars + 17;     // [stages]
  uint64_t* mk_empty = bars + 21;    // [stages]
  uint64_t* acc_full = bars + 25;    // [stages]
  uint64_t* acc_empty = bars + 29;   // [stages]
  SearchItem* ring = reinterpret_cast<SearchItem*>(misc + 512);  // [ring]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(misc + 768);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* mrun = reinterpret_cast<int*>(tmem_slot + 2);     // [2] running max per item slot (ordered int)
  float* red_all = reinterpret_cast<float*>(tmem_slot + 4);  // [2 groups][4] selection reductions
  int* red_i_all = reinterpret_cast<int*>(tmem_slot + 12);   // [2][4]
  int* red_k_all = reinterpret_cast<int*>(tmem_slot + 20);   // [2][4]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < kSearchRing; ++i) {
      mbar_init(item_full + i, 1);
      mbar_init(item_empty + i, 1 + 256 + 256);  // MMA issuer, tile epilogue, selection
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(q_full + i, 1);
      mbar_init(q_empty + i, 1);
      mbar_init(arr_full + i, 128 * kSearchEpiGroups);
      mbar_init(arr_empty + i, 128);
      mrun[i] = float_to_ordered(-INFINITY);
    }
    for (int i = 0; i < kSearchStages; ++i) {
      mbar_init(mk_full + i, 1);
      mbar_init(mk_empty + i, 1);
      mbar_init(acc_full + i, 1);
      mbar_init(acc_empty + i, 128);
    }
    mbar_init(mma_done, 1);
    *abort = 0;
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
  const int group = A.P.hq / A.P.hk;

  const bool epi_warp = warp >= 4 && warp < kSearchSelWarp0;
  if (warp == 0) {
    // ------------------------------------------------------------ scheduler + TMA producer
    regs_dec<kSearchPRoleRegs>();
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_mk);
      uint32_t it = 0, qn = 0, tn = 0;
      bool ok = true;
      while (ok) {
        const int slot = it % kSearchRing;
        if (!SP_TW(kSpProdItem, mbar_wait_sleep(item_empty + slot, ((it / kSearchRing) & 1) ^ 1, abort))) break;
        SearchItem f{};
        const int id = atomicAdd(A.counter, 1);
        if (id >= A.total_items) {
          f.valid = 0;
        } else {
          SeqInfo sq;
          int qb;
          const int tile = id / A.P.hq;
          if (!decode_item(A.P, tile, sq, qb)) {
            f.valid = 2;
          } else {
            f.valid = 1;
            f.fast = (qb >= sq.nb - A.last_n || !(A.alpha > 0.f)) ? 1 : 0;
            f.start = sq.start;
            f.len = sq.len;
            f.tile_base = sq.tile_base;
            f.bcoord = sq.bcoord;
            f.qb = qb;
            f.h = id - tile * A.P.hq;
          }
        }
        ring[slot] = f;
        mbar_arrive(item_full + slot);
        ++it;
        if (f.valid == 0) break;
        if (f.valid != 1 || f.fast) continue;
        const int qs = qn & 1;
        if (!SP_TW(kSpProdQ, mbar_wait_sleep(q_empty + qs, ((qn >> 1) & 1) ^ 1, abort))) break;
        ++qn;
        const int qrow = f.start + f.qb * kBlock - A.P.q_off;  // rows before a chunk load as zeros
        mbar_arrive_expect_tx(q_full + qs, kTileBytes);
        tma_load_4d(sQ + qs * kTileBytes, &tm_q, q_full + qs, 0, f.h, qrow, f.bcoord);
        tma_load_4d(sQ + qs * kTileBytes + kHalfTile, &tm_q, q_full + qs, 64, f.h, qrow, f.bcoord);
        const int hk = f.h / group, ntiles = f.qb / kBlock + 1;
        for (int j = 0; j < ntiles; ++j, ++tn) {
          const int t = tile_order(j, ntiles);
          const int st = tn % kSearchStages;
          if (!SP_TW(kSpProdMk, mbar_wait_sleep(mk_empty + st, ((tn / kSearchStages) & 1) ^ 1, abort))) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(mk_full + st, kTileBytes);
          uint8_t* dst = sMK + st * kTileBytes;
          const int mrow = f.tile_base + t * kBlock;
          tma_load_4d(dst, &tm_mk, mk_full + st, 0, hk, mrow, 0);
          tma_load_4d(dst + kHalfTile, &tm_mk, mk_full + st, 64, hk, mrow, 0);
        }
      }
      if (*abort) {  // let loads still in flight land before the CTA exits
        volatile int no_abort = 0;
        for (int sl = 0; sl < 2; ++sl) {
          const uint32_t nt = (tn + 1 - sl) >> 1, nq = (qn + 1 - sl) >> 1;
          if (nt) mbar_wait(mk_full + sl, (nt - 1) & 1, &no_abort);
          if (nq) mbar_wait(q_full + sl, (nq - 1) & 1, &no_abort);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    regs_dec<kSearchPRoleRegs>();
    if (lane == 0) {
      constexpr uint32_t idesc = idesc_f16(128, 128, DT<T>::is_bf16, false);
      uint32_t it = 0, qc = 0, tc = 0;
      bool ok = true;
      while (ok) {
        const int slot = it % kSearchRing;
        if (!mbar_wait_sleep(item_full + slot, (it / kSearchRing) & 1, abort)) break;
        const SearchItem f = ring[slot];
        if (f.valid == 0) break;
        if (f.valid == 1 && !f.fast) {
          const int qs = qc & 1;
          if (!SP_TW(kSpMmaQ, mbar_wait(q_full + qs, (qc >> 1) & 1, abort))) break;
          const uint32_t q_base = smem_u32(sQ + qs * kTileBytes);
          const int ntiles = f.qb / kBlock + 1;
          for (int t = 0; t < ntiles; ++t, ++tc) {
            const int st = tc % kSearchStages;  // pooled-key stage = accumulator
            const uint32_t ph = (tc / kSearchStages) & 1;
            if (!SP_TW(kSpMmaMk, mbar_wait(mk_full + st, ph, abort))) { ok = false; break; }
            if (!SP_TW(kSpMmaAcc, mbar_wait(acc_empty + st, ph ^ 1, abort))) { ok = false; break; }
            tc_fence_after();
            const uint32_t a_base = smem_u32(sMK + st * kTileBytes);
#pragma unroll
            for (int ks = 0; ks < 8; ++ks) {
              const uint32_t off = (ks >> 2) * kHalfTile + (ks & 3) * 32;
              umma_ss(tmem + st * 128, sdesc_sw128(a_base + off, 16, 1024), sdesc_sw128(q_base + off, 16, 1024),
                      idesc, ks > 0);
            }
            umma_commit(mk_empty + st);
            umma_commit(acc_full + st);
          }
          if (!ok) break;
          umma_commit(q_empty + qs);
          ++qc;
        }
        mbar_arrive(item_empty + slot);
        ++it;
      }
      umma_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort);
    }
  } else if (warp < 4) {
    regs_dec<kSearchPRoleRegs>();  // idle
  } else if (epi_warp) {
    // ------------------------------------------------------------ tile epilogue (warps 4..11)
    regs_inc<kSearchPEpiRegs>();
    const int eg = (warp - 4) >> 2;     // group: tiles with tc % kSearchEpiGroups == eg
    const int quad = warp & 3;
    const int lrow = quad * 32 + lane;  // TMEM lane = key block within the tile
    const float c = A.c;
    uint32_t it = 0, tc = 0, an = 0;
    while (true) {
      const int slot = it % kSearchRing;
      if (!SP_TW(kSpEpiItem, mbar_wait_warp_sleep(item_full + slot, (it / kSearchRing) & 1, abort))) break;
      const SearchItem f = ring[slot];
      if (f.valid == 0) break;
      bool ok = true;
      if (f.valid == 1 && !f.fast) {
        const int a = an & 1;
        if (!SP_TW(kSpEpiArr, mbar_wait_warp_sleep(arr_empty + a, ((an >> 1) & 1) ^ 1, abort))) break;
        ++an;
        float* m_arr = arr + a * 2 * cap;
        float* p_arr = m_arr + cap;
        int* mr = mrun + a;
        const int qb = f.qb;
        const int vr = min(kBlock, f.len - qb * kBlock);  // valid query rows of this block
        const int ntiles = qb / kBlock + 1;
        for (int j = 0; j < ntiles; ++j, ++tc) {
          const int t = tile_order(j, ntiles);
          if ((int)(tc % kSearchEpiGroups) != eg) continue;  // another group's tile
          const int acc = tc % kSearchStages;
          if (!SP_TW(kSpEpiAcc, mbar_wait_warp_sleep(acc_full + acc, (tc / kSearchStages) & 1, abort))) {
            ok = false;
            break;
          }
          tc_fence_after();
          const long long te1 = SP_T();
          const int kb = t * kBlock + lrow;
          const uint32_t taddr = tmem + acc * 128 + ((uint32_t)(quad * 32) << 16);
          // the 128 scores of this key block, read from TMEM 64 at a time (once for the max,
          // again for the exponentials)
          uint32_t ua[32], ub[32];
          float mx = vr == kBlock ? -INFINITY : 0.f, s127 = 0.f;  // padded rows (q = 0) score 0
#pragma unroll
          for (int hb = 0; hb < 2; ++hb) {
            tmem_ld32(taddr + hb * 64, ua);
            tmem_ld32(taddr + hb * 64 + 32, ub);
            tmem_ld_wait();
#define FPB_S(i) __uint_as_float((i) < 32 ? ua[(i)] : ub[(i) - 32])
            if (vr == kBlock) {
              float m0 = -INFINITY, m1 = -INFINITY;
#pragma unroll
              for (int i = 0; i < 64; i += 4) {
                m0 = max3(m0, FPB_S(i), FPB_S(i + 1));
                m1 = max3(m1, FPB_S(i + 2), FPB_S(i + 3));
              }
              mx = fmaxf(mx, fmaxf(m0, m1));
              if (hb == 1) s127 = FPB_S(63);
            } else {
#pragma unroll
              for (int i = 0; i < 64; ++i)
                if (hb * 64 + i < vr) mx = fmaxf(mx, FPB_S(i));
            }
#undef FPB_S
          }
          const long long te2 = SP_T();
          const bool causal = kb <= qb;
          const bool diag = kb == qb;
          float m = -INFINITY;
          if (causal) m = __fmul_rn(diag ? s127 : mx, c);
          float wm = m;  // running lower bound of the row maximum
#pragma unroll
          for (int o = 16; o; o >>= 1) wm = fmaxf(wm, __shfl_xor_sync(0xffffffffu, wm, o));
          const float m_est = fmaxf(wm, ordered_to_float(*(volatile int*)mr));
          if (lane == 0 && wm > -INFINITY) atomicMax(mr, float_to_ordered(wm));
          const bool cand = causal && (m >= m_est + A.cand_off);
          float p = 0.f;
          const long long te3 = SP_T();
          const bool any_exp = __any_sync(0xffffffffu, cand && !diag);
          if (any_exp) {
            const float nm = -m;
            float p0 = 0.f, p1 = 0.f;
#pragma unroll
            for (int hb = 0; hb < 2; ++hb) {
              tmem_ld32(taddr + hb * 64, ua);
              tmem_ld32(taddr + hb * 64 + 32, ub);
              tmem_ld_wait();
#define FPB_S(i) __uint_as_float((i) < 32 ? ua[(i)] : ub[(i) - 32])
              if (vr == kBlock) {
                // one pair in four on the FMA pipe (exp2_poly2, relative error ~1e-4), the
                // rest by ex2.approx: the sum only has to resolve the 1e-3 threshold band
#pragma unroll
                for (int i = 0; i < 64; i += 2) {
                  float x0, x1, e0, e1;
                  fma2(x0, x1, FPB_S(i), FPB_S(i + 1), c, c, nm, nm);
                  if (kSearchPoly && ((i >> 1) & 3) == 3) {
                    exp2_poly2(x0, x1, e0, e1);
                  } else {
                    e0 = ex2_approx(x0);
                    e1 = ex2_approx(x1);
                  }
                  add2(p0, p1, p0, p1, e0, e1);
                }
              } else {
#pragma unroll
                for (int i = 0; i < 64; ++i)
                  if (hb * 64 + i < vr) p0 += ex2_approx(__fmaf_rn(FPB_S(i), c, nm));
              }
#undef FPB_S
            }
            p = p0 + p1;
            if (vr < kBlock) p += (float)(kBlock - vr) * ex2_approx(-m);
          }
          tc_fence_before();
          mbar_arrive(acc_empty + acc);  // the accumulator may be overwritten by tile tc + 2
          if (diag) p = 1.f;
          if (causal) {
            m_arr[kb] = m;
            p_arr[kb] = cand ? p : -1.f;
          }
          if (SP_ON) {
            const long long te4 = SP_T();
            pacc[kSpEpiLd] += te2 - te1;
            pacc[kSpEpiMax] += te3 - te2;
            pacc[kSpEpiExp] += te4 - te3;
            pacc[kSpEpiTiles] += 1;
            pacc[kSpEpiExpTiles] += any_exp;
          }
        }
        if (!ok) break;
        mbar_arrive(arr_full + a);
      }
      mbar_arrive(item_empty + slot);
      ++it;
    }
  } else {
    // ------------------------------------------------------------ selection (warps 12..19)
    regs_dec<kSearchPRoleRegs>();
    const int sg = (warp - kSearchSelWarp0) >> 2;  // group: items dealt round robin (fast ones too)
    const int es = threadIdx.x - 32 * kSearchSelWarp0 - sg * 128;  // 0..127
    const int wq = (warp - kSearchSelWarp0) & 3;
    float* red = red_all + sg * 4;
    int* red_i = red_i_all + sg * 4;
    int* red_k = red_k_all + sg * 4;
    uint32_t it = 0, an = 0, fn = 0;
    while (true) {
      const int slot = it % kSearchRing;
      if (!SP_TW(kSpSelItem, mbar_wait_warp_sleep(item_full + slot, (it / kSearchRing) & 1, abort))) break;
      const long long ts0 = SP_T();
      const SearchItem f = ring[slot];
      if (f.valid == 0) break;
      if (f.valid == 1) {
        const int qb = f.qb;
        const int row = f.tile_base + qb;
        int32_t* out_idx = A.idx + ((int64_t)f.h * A.P.tiles_ub + row) * cap;
        int32_t* out_cnt = A.cnt + (int64_t)f.h * A.P.tiles_ub + row;
        if (f.fast) {  // every causal block
          if ((fn++ % kSearchSelGroups) == (uint32_t)sg) {
            for (int kb = es; kb <= qb; kb += 128) out_idx[kb] = kb;
            if (es == 0) *out_cnt = qb + 1;
          }
        } else if ((an++ % kSearchSelGroups) != (uint32_t)sg) {
          // another group's item
        } else {
          const int a = (an - 1) & 1;  // the item's array slot
          if (!SP_TW(kSpSelArr, mbar_wait_warp_sleep(arr_full + a, ((an - 1) >> 1) & 1, abort))) break;
          float* m_arr = arr + a * 2 * cap;
          float* p_arr = m_arr + cap;
          uint32_t* marks = marks_all + a * ncw;
          const float M = ordered_to_float(*(volatile int*)(mrun + a));
          // pw >= alpha * max pw  (see the per-item kernel above)
          float best = 0.f;
#pragma unroll 4
          for (int kb = es; kb <= qb; kb += 128) {
            const float pv = p_arr[kb];
            const float pw = pv >= 0.f ? __fmul_rn(pv, ex2_approx(__fsub_rn(m_arr[kb], M))) : -1.f;
            p_arr[kb] = pw;
            best = fmaxf(best, pw);
          }
          // row maximum of pw over the group (named barrier 2 + sg)
#pragma unroll
          for (int o = 16; o; o >>= 1) best = fmaxf(best, __shfl_xor_sync(0xffffffffu, best, o));
          named_bar_sync(2 + sg, 128);
          if (lane == 0) red[wq] = best;
          named_bar_sync(2 + sg, 128);
          const float thr = __fmul_rn(fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3])), A.alpha);
          const int nwords = (qb + 1 + 31) / 32;
          const int kbudget = min(A.min_budget, qb + 1);
          if (kbudget > 0) {
            for (int wd = es; wd < nwords; wd += 128) marks[wd] = 0u;
            named_bar_sync(2 + sg, 128);
          }
          for (int r2 = 0; r2 < kbudget; ++r2) {
            float bv = -INFINITY;
            int bk = 0x7fffffff;
            for (int kb = es; kb <= qb; kb += 128) {
              if (marks[kb >> 5] & (1u << (kb & 31))) continue;
              const float v = fmaxf(p_arr[kb], 0.f);
              if (v > bv || (v == bv && kb < bk)) { bv = v; bk = kb; }
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) {
              const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
              const int ok2 = __shfl_xor_sync(0xffffffffu, bk, o);
              if (ov > bv || (ov == bv && ok2 < bk)) { bv = ov; bk = ok2; }
            }
            if (lane == 0) { red[wq] = bv; red_k[wq] = bk; }
            named_bar_sync(2 + sg, 128);
            if (es == 0) {
              float v0 = red[0];
              int k0 = red_k[0];
              for (int j = 1; j < 4; ++j)
                if (red[j] > v0 || (red[j] == v0 && red_k[j] < k0)) { v0 = red[j]; k0 = red_k[j]; }
              if (k0 <= qb) marks[k0 >> 5] |= 1u << (k0 & 31);
            }
            named_bar_sync(2 + sg, 128);
          }
          // selection + ascending compaction: warp wq owns the contiguous key blocks
          // [wq * span, wq * span + span), visited 32 at a time (one per lane, ballot +
          // popcount); one barrier combines the four warp totals
          const int span = ((qb + 1 + 127) / 128) * 32;
          const int w0 = wq * span, w1 = min(qb + 1, w0 + span);
          auto selected = [&](int kb) -> bool {
            if (kb >= w1) return false;
            const float pw = p_arr[kb];
            bool sel = (pw >= 0.f && pw >= thr) || kb < A.sink || (qb - kb) < A.window;
            if (kbudget > 0) sel = sel || ((marks[kb >> 5] >> (kb & 31)) & 1u);
            return sel;
          };
          int wcount = 0;
          for (int k0 = w0; k0 < w1; k0 += 32) wcount += __popc(__ballot_sync(0xffffffffu, selected(k0 + lane)));
          if (lane == 0) red_i[wq] = wcount;
          named_bar_sync(2 + sg, 128);
          int pre = 0;
          for (int j = 0; j < wq; ++j) pre += red_i[j];
          const int total = red_i[0] + red_i[1] + red_i[2] + red_i[3];
          for (int k0 = w0; k0 < w1; k0 += 32) {
            const bool sel = selected(k0 + lane);
            const uint32_t bal = __ballot_sync(0xffffffffu, sel);
            if (sel) out_idx[pre + __popc(bal & ((1u << lane) - 1u))] = k0 + lane;
            pre += __popc(bal);
          }
          if (es == 0) *out_cnt = total;
          named_bar_sync(2 + sg, 128);  // every thread has read M, red_i and this item's arrays
          if (es == 0) mrun[a] = float_to_ordered(-INFINITY);
          mbar_arrive(arr_empty + a);
        }
      }
      if (SP_ON) pacc[kSpSelWork] += SP_T() - ts0;
      mbar_arrive(item_empty + slot);
      ++it;
    }
  }
  // recording threads: producer, issuer, the first epilogue thread of group 0, the first selection thread
#if FPB_SEARCH_PROFILE
  if (A.prof && (threadIdx.x == 0 || threadIdx.x == 32 || threadIdx.x == 128 || threadIdx.x == 32 * kSearchSelWarp0)) {
    pacc[kSpCta] = threadIdx.x == 0 ? clock64() - t_k0 : 0;
    for (int i = 0; i < kSpSlots; ++i)
      if (pacc[i]) atomicAdd(A.prof + i, pacc[i]);
  }
#endif
#undef SP_TW
#undef SP_T
#undef SP_ON

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && *abort) raise_error(A.P.err, kErrWaitTimeout);
}

}  // namespace fpb
