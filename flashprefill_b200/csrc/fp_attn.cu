// Block-sparse causal GQA attention forward on the 5th-generation tensor cores.
//
// Reference: ops/flashprefill_native_forward.py:228-344 (_flash_forward) and
// ops/flashprefill_varlen_func.py:449-575 (_flash_block_sparse_varlen): for each query
// block and each selected key block (ascending), S = (Q K^T) * c with c = scale*log2(e),
// the diagonal block masked causally, online softmax in exp2, P rounded to the input
// dtype for the P V product, O = acc / l stored in the input dtype.  A row whose list is
// empty outputs zeros (the reference starts l at 1.0 and acc at 0).
//
// One CTA per (query block, query head) with 192 threads:
//   warp 0      TMA producer: Q once, then K and V of each listed block into a 2-stage ring
//   warp 1      tcgen05.mma issuer: S_j = Q K_j^T (both operands K-major, SW128 smem) into
//               a double-buffered TMEM S; O += P_j V_j with P read from TMEM (16-bit pairs
//               written in place of S_j) and V MN-major from smem
//   warps 2-5   softmax: one TMEM lane (= one query row) per thread.  The running row max
//               is exact, as in the reference: whenever a block raises it, O (in TMEM) is
//               rescaled after the previous P V product has landed.  The largest P of a row
//               is therefore exactly 1.0, which keeps the bf16 rounding of P at the
//               reference's level (a lazy max that lets P grow above 1 adds up to one bf16
//               ulp of P to the output).
// TMEM columns: S0 [0,128), S1 [128,256), O [256,384).
#include "fp_common.cuh"

namespace fpb {

struct AttnArgs {
  SeqProblem P;
  float c;                   // fp32(1/sqrt(D)) * fp32(log2 e)
  float rescale_thr;         // move the running max only if a block exceeds it by more than this
  const int32_t* idx;        // [hq][tiles_ub][cap] ascending block lists
  const int32_t* cnt;        // [hq][tiles_ub]
  void* out;                 // output base (masked-store path)
  int64_t o_sb, o_ss, o_sh;  // output strides in elements
};

constexpr int kAttnThreads = 192;
constexpr int kKVStages = 2;
constexpr uint32_t kAttnTile = 128 * 128 * 2;
constexpr uint32_t kAttnHalf = kAttnTile / 2;
constexpr float kRescaleThreshold = 0.f;  // exact running max (reference numerics)

__host__ __device__ constexpr size_t attn_smem_bytes() {
  return (size_t)kAttnTile * (1 + 2 * kKVStages) + 256 + 1024;
}

template <typename T>
__global__ void __launch_bounds__(kAttnThreads, 1)
    sparse_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                       const AttnArgs A) {
  const int hq = blockIdx.x % A.P.hq;
  SeqInfo s;
  int qb;
  if (!decode_item(A.P, blockIdx.x / A.P.hq, s, qb)) return;
  const int hk = hq / (A.P.hq / A.P.hk);
  const int row = s.tile_base + qb;
  const int32_t* list = A.idx + ((int64_t)hq * A.P.tiles_ub + row) * A.P.cap;
  int n = __ldg(A.cnt + (int64_t)hq * A.P.tiles_ub + row);
  n = max(0, min(n, qb + 1));

  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;
  uint8_t* sK = smem + kAttnTile;
  uint8_t* sV = sK + kKVStages * kAttnTile;
  uint64_t* bars = reinterpret_cast<uint64_t*>(sV + kKVStages * kAttnTile);
  uint64_t* q_full = bars + 0;
  uint64_t* k_full = bars + 1;     // [2]
  uint64_t* v_full = bars + 3;     // [2]
  uint64_t* kv_empty = bars + 5;   // [2]
  uint64_t* s_full = bars + 7;     // [2]
  uint64_t* p_full = bars + 9;     // [2]
  uint64_t* pv_done = bars + 11;
  uint64_t* mma_done = bars + 12;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 13);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(k_full + i, 1);
      mbar_init(v_full + i, 1);
      mbar_init(kv_empty + i, 1);
      mbar_init(s_full + i, 1);
      mbar_init(p_full + i, 128);
    }
    mbar_init(pv_done, 1);
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
  const uint32_t tmem_o = tmem + 256;

  if (warp == 0) {
    // ------------------------------------------------------------ TMA producer
    if (lane == 0) {
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      const int qrow = s.start + qb * kBlock;
      mbar_arrive_expect_tx(q_full, kAttnTile);
      tma_load_4d(sQ, &tm_q, q_full, 0, hq, qrow, s.bcoord);
      tma_load_4d(sQ + kAttnHalf, &tm_q, q_full, 64, hq, qrow, s.bcoord);
      const uint64_t keep = l2_policy_evict_last();
      int issued = 0;
      for (int j = 0; j < n; ++j) {
        const int st = j & 1;
        if (!mbar_wait(kv_empty + st, ((j >> 1) & 1) ^ 1, abort)) break;
        int kb = __ldg(list + j);
        if (kb < 0 || kb > qb) {
          raise_error(A.P.err, kErrIndexRange);
          kb = qb;
        }
        const int krow = s.start + kb * kBlock;
        mbar_arrive_expect_tx(k_full + st, kAttnTile);
        tma_load_4d_hint(sK + st * kAttnTile, &tm_k, k_full + st, 0, hk, krow, s.bcoord, keep);
        tma_load_4d_hint(sK + st * kAttnTile + kAttnHalf, &tm_k, k_full + st, 64, hk, krow, s.bcoord, keep);
        mbar_arrive_expect_tx(v_full + st, kAttnTile);
        tma_load_4d_hint(sV + st * kAttnTile, &tm_v, v_full + st, 0, hk, krow, s.bcoord, keep);
        tma_load_4d_hint(sV + st * kAttnTile + kAttnHalf, &tm_v, v_full + st, 64, hk, krow, s.bcoord, keep);
        issued = j + 1;
      }
      if (*abort) {  // let loads still in flight land before the CTA exits
        volatile int no_abort = 0;
        for (int j = (issued > 2 ? issued - 2 : 0); j < issued; ++j) {
          mbar_wait(k_full + (j & 1), (j >> 1) & 1, &no_abort);
          mbar_wait(v_full + (j & 1), (j >> 1) & 1, &no_abort);
        }
        mbar_wait(q_full, 0, &no_abort);
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      constexpr uint32_t id_s = idesc_f16(128, 128, DT<T>::is_bf16, false);
      constexpr uint32_t id_o = idesc_f16(128, 128, DT<T>::is_bf16, true);
      const uint32_t q_base = smem_u32(sQ);
      bool ok = mbar_wait(q_full, 0, abort);
      auto issue_s = [&](int j) -> bool {
        const int st = j & 1;
        if (!mbar_wait(k_full + st, (j >> 1) & 1, abort)) return false;
        tc_fence_after();
        const uint32_t k_base = smem_u32(sK + st * kAttnTile);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = (ks >> 2) * kAttnHalf + (ks & 3) * 32;
          umma_ss(tmem + st * 128, sdesc_sw128(q_base + off, 16, 1024), sdesc_sw128(k_base + off, 16, 1024), id_s,
                  ks > 0);
        }
        umma_commit(s_full + st);
        return true;
      };
      if (ok && n > 0) ok = issue_s(0);
      for (int j = 0; ok && j < n; ++j) {
        const int st = j & 1;
        if (j + 1 < n && !issue_s(j + 1)) { ok = false; break; }
        if (!mbar_wait(p_full + st, (j >> 1) & 1, abort)) { ok = false; break; }
        if (!mbar_wait(v_full + st, (j >> 1) & 1, abort)) { ok = false; break; }
        tc_fence_after();
        const uint32_t v_base = smem_u32(sV + st * kAttnTile);
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          // A = P (TMEM, 16-bit pairs: 8 columns per 16 keys); B = V rows ks*16.. (MN-major)
          umma_ts(tmem_o, tmem + st * 128 + ks * 8, sdesc_sw128(v_base + ks * 2048, kAttnHalf, 1024), id_o,
                  (j > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(kv_empty + st);
        umma_commit(pv_done);
      }
      umma_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort);
    }
  } else {
    // ------------------------------------------------------------ softmax + epilogue
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row within the block (= TMEM lane)
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const float c = A.c;
    float m_use = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n; ++j) {
      const int st = j & 1;
      int kb = __ldg(list + j);
      if (kb < 0 || kb > qb) kb = qb;
      const bool diag = kb == qb;
      if (!mbar_wait_warp(s_full + st, (j >> 1) & 1, abort)) { ok = false; break; }
      tc_fence_after();
      float sv[128];
#pragma unroll
      for (int ch = 0; ch < 4; ++ch) {
        uint32_t u[32];
        tmem_ld32(tmem + st * 128 + lane_off + ch * 32, u);
        tmem_ld_wait();
#pragma unroll
        for (int i = 0; i < 32; ++i) sv[ch * 32 + i] = __uint_as_float(u[i]);
      }
      if (diag) {
#pragma unroll
        for (int i = 0; i < 128; ++i)
          if (i > r) sv[i] = -INFINITY;
      }
      float mx0 = sv[0], mx1 = sv[1], mx2 = sv[2], mx3 = sv[3];
#pragma unroll
      for (int i = 4; i < 128; i += 4) {
        mx0 = fmaxf(mx0, sv[i]);
        mx1 = fmaxf(mx1, sv[i + 1]);
        mx2 = fmaxf(mx2, sv[i + 2]);
        mx3 = fmaxf(mx3, sv[i + 3]);
      }
      const float m_blk = fmaxf(fmaxf(mx0, mx1), fmaxf(mx2, mx3)) * c;
      float scale_o = 1.f;
      if (j == 0) {
        m_use = m_blk;
      } else if (m_blk > m_use + A.rescale_thr) {
        scale_o = ex2_approx(m_use - m_blk);
        m_use = m_blk;
        l *= scale_o;
      }
      if (__any_sync(0xffffffffu, scale_o != 1.f)) {
        // O holds the sum up to block j-1: wait for that P V product, then rescale in TMEM
        if (!mbar_wait_warp(pv_done, (j - 1) & 1, abort)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int ch = 0; ch < 4; ++ch) {
          uint32_t u[32];
          tmem_ld32(tmem_o + lane_off + ch * 32, u);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) u[i] = __float_as_uint(__uint_as_float(u[i]) * scale_o);
          tmem_st32(tmem_o + lane_off + ch * 32, u);
        }
        tmem_st_wait();
      }
      const float neg_m = -m_use;
      float rs0 = 0.f, rs1 = 0.f;
      uint32_t pk[64];
#pragma unroll
      for (int i = 0; i < 128; i += 2) {
        const float p0 = ex2_approx(fmaf(sv[i], c, neg_m));
        const float p1 = ex2_approx(fmaf(sv[i + 1], c, neg_m));
        rs0 += p0;
        rs1 += p1;
        pk[i >> 1] = DT<T>::pack(p0, p1);
      }
      l += rs0 + rs1;
      {
        uint32_t (&lo)[32] = *reinterpret_cast<uint32_t(*)[32]>(&pk[0]);
        uint32_t (&hi)[32] = *reinterpret_cast<uint32_t(*)[32]>(&pk[32]);
        tmem_st32(tmem + st * 128 + lane_off, lo);
        tmem_st32(tmem + st * 128 + lane_off + 32, hi);
      }
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(p_full + st);
    }

    // ---- epilogue: O / l -> smem (SW128 layout, reusing the Q tile) -> global
    float inv = 0.f;
    const bool have = __all_sync(0xffffffffu, ok && n > 0 && !*abort);
    if (have) {
      if (!mbar_wait_warp(pv_done, (n - 1) & 1, abort)) ok = false;
      tc_fence_after();
      inv = 1.f / l;
    }
    const bool use_tmem = have && ok;
#pragma unroll
    for (int ch = 0; ch < 4; ++ch) {
      uint32_t u[32];
      if (use_tmem) {
        tmem_ld32(tmem_o + lane_off + ch * 32, u);
        tmem_ld_wait();
      } else {
#pragma unroll
        for (int i = 0; i < 32; ++i) u[i] = 0u;
      }
      uint32_t pk[16];
#pragma unroll
      for (int i = 0; i < 16; ++i)
        pk[i] = DT<T>::pack(__uint_as_float(u[2 * i]) * inv, __uint_as_float(u[2 * i + 1]) * inv);
#pragma unroll
      for (int q4 = 0; q4 < 4; ++q4) {
        const int cidx = ch * 4 + q4;  // 16-byte chunk 0..15 of the row
        const int half = cidx >> 3, c8 = cidx & 7;
        uint8_t* dst = sQ + half * kAttnHalf + r * 128 + ((c8 ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(pk[q4 * 4], pk[q4 * 4 + 1], pk[q4 * 4 + 2], pk[q4 * 4 + 3]);
      }
    }
    fence_proxy_async_smem();
    named_bar_sync(1, 128);
    const int vr = min(kBlock, s.len - qb * kBlock);
    const int et = threadIdx.x - 64;
    if (vr == kBlock) {
      if (et == 0) {
        const int qrow = s.start + qb * kBlock;
        tma_store_4d(&tm_o, sQ, 0, hq, qrow, s.bcoord);
        tma_store_4d(&tm_o, sQ + kAttnHalf, 64, hq, qrow, s.bcoord);
        tma_store_commit_and_wait();
      }
    } else {
      T* ob = reinterpret_cast<T*>(A.out) + (int64_t)s.bcoord * A.o_sb +
              (int64_t)(s.start + qb * kBlock) * A.o_ss + (int64_t)hq * A.o_sh;
      for (int e = et; e < vr * 16; e += 128) {
        const int rr = e >> 4, cidx = e & 15;
        const int half = cidx >> 3, c8 = cidx & 7;
        const uint4 v = *reinterpret_cast<const uint4*>(sQ + half * kAttnHalf + rr * 128 + ((c8 ^ (rr & 7)) << 4));
        *reinterpret_cast<uint4*>(ob + (int64_t)rr * A.o_ss + cidx * 8) = v;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && *abort) raise_error(A.P.err, kErrWaitTimeout);
}

}  // namespace fpb
