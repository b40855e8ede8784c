// Block-sparse causal GQA attention forward, head-pair kernel (5th-generation tensor cores).
//
// Reference: ops/flashprefill_native_forward.py:228-344 (_flash_forward) and
// ops/flashprefill_varlen_func.py:449-575 (_flash_block_sparse_varlen): for each query block and
// each selected key block (ascending), S = (Q K^T) * c with c = scale*log2(e), the diagonal block
// masked causally, online softmax in exp2, P rounded to the input dtype for the P V product,
// O = acc / l stored in the input dtype.  A row whose list is empty outputs zeros.
//
// A work item is one query block of TWO query heads of the same KV head (a head pair; with an
// odd group size the last pair of a group has one head).  The two heads' block lists are walked
// as one ascending union: every key/value tile of the union is loaded once into a two-stage ring
// and serves the MMAs of whichever of the two heads lists it.  At long contexts most selected
// blocks are structural (sinks, local window, last rows) and shared by the heads of a group, so
// the union is barely longer than either list and K/V traffic halves.
//
// The two heads are two "tiles" in flight on the tensor core, in ping-pong: the MMA issuer
// issues, for each union block, PV_0(previous) and S_0(this), then PV_1(previous) and
// S_1(this); while the tensor core works for one tile, the other tile's softmax runs.  P is
// written over S in TMEM (16-bit pairs in S columns 0..63) and read by the TS-form MMA, so
// S_t(next) is issued after PV_t(previous), which the in-order tensor pipe keeps ordered.
//
// Persistent kernel, one CTA per SM, 384 threads:
//   warp 0        scheduler + TMA producer: item fetch, Q_0/Q_1, union walk, K/V ring
//   warp 1        TMEM owner + tcgen05.mma issuer
//   warps 4-7     softmax + epilogue of tile 0 (one thread per query row, 128 columns)
//   warps 8-11    softmax + epilogue of tile 1
// TMEM columns: S_0 [0,128), S_1 [128,256), O_0 [256,384), O_1 [384,512).
// Shared memory: Q_0, Q_1, K[2], V[2] (32 KB each, 128-byte swizzled) and the barriers.
// The epilogue writes O / l from registers straight to global memory (each thread one row of
// 256 contiguous bytes), so no staging tile holds back the next item's loads.
#include "fp_common.cuh"

namespace fpb {

struct Attn2Args {
  SeqProblem P;
  float c;               // fp32(1/sqrt(D)) * fp32(log2 e)
  const int32_t* idx;    // [hq][tiles_ub][cap] ascending block lists
  const int32_t* cnt;    // [hq][tiles_ub]
  int* counter;          // work-item counter, zero at launch
  int total_items;       // tiles_ub * hk * ppg
  int ppg;               // head pairs per KV head: ceil(G / 2)
  void* out;             // output base
  int64_t o_sb, o_ss, o_sh;  // output strides in elements
};

constexpr int kA2Threads = 384;
// Register split: compiled for 168 per thread (384 x 168 = 64512 <= 65536); warps 0-3 give back
// to 80, the two softmax warpgroups grow to 208: 128 * 80 + 256 * 208 = 63488.
constexpr int kA2LaunchRegs = 168, kA2RoleRegs = 80, kA2SoftRegs = 208;
static_assert(128 * kA2RoleRegs + 256 * kA2SoftRegs <= kA2Threads * kA2LaunchRegs, "register split");
#ifndef FPB_A2_POLY_EVERY
#define FPB_A2_POLY_EVERY 3
#endif
constexpr int kA2PolyEvery = FPB_A2_POLY_EVERY;  // one exp2 pair in kA2PolyEvery on the FMA pipe
constexpr uint32_t kA2Tile = 128 * 128 * 2;
constexpr uint32_t kA2Half = kA2Tile / 2;

__host__ __device__ constexpr size_t attn2_smem_bytes() { return (size_t)kA2Tile * 6 + 1024 + 1024; }

struct Item2 {
  int valid;  // 0: no more work, 1: item, 2: nothing to do (padding tile of the grid)
  int start, len, bcoord, qb, row;
  int h[2];     // query heads of the two tiles (h[1] = -1: single-head item)
  int n[2];     // listed blocks per tile
  int diag[2];  // the tile's last listed block is the diagonal block (causal mask)
  int pad[4];
};

template <typename T>
__global__ void __launch_bounds__(kA2Threads, 1)
    sparse_attn2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const Attn2Args A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                  // [2] tiles
  uint8_t* sK = smem + 2 * kA2Tile;    // [2] stages
  uint8_t* sV = smem + 4 * kA2Tile;    // [2] stages
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * kA2Tile);
  uint64_t* item_full = bars + 0;   // [slot]
  uint64_t* item_empty = bars + 2;  // [slot]
  uint64_t* q_full = bars + 4;      // [tile]
  uint64_t* q_empty = bars + 6;
  uint64_t* k_full = bars + 8;      // [stage]
  uint64_t* k_empty = bars + 10;
  uint64_t* v_full = bars + 12;
  uint64_t* v_empty = bars + 14;
  uint64_t* s_full = bars + 16;     // [tile]
  uint64_t* p_full = bars + 18;
  uint64_t* o_full = bars + 20;
  uint64_t* o_empty = bars + 22;
  uint64_t* mma_done = bars + 24;
  Item2* ring = reinterpret_cast<Item2*>(bars + 32);          // [slot], 64 bytes each
  volatile int* umask = reinterpret_cast<volatile int*>(ring + 2);  // [stage]: tiles | last << 2
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ring + 3);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(item_full + i, 1);
      mbar_init(item_empty + i, 1 + 256);
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
  const int npairs = A.P.hk * A.ppg;

  if (warp < 4) {
    regs_dec<kA2RoleRegs>();
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------ scheduler + producer
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      prefetch_tmap(&tm_v);
      const uint64_t stream_once = l2_policy_evict_first();
      uint32_t it = 0, kvseq = 0, qld[2] = {0, 0};
      bool ok = true;
      while (ok) {
        const int slot = it & 1;
        if (!mbar_wait_sleep(item_empty + slot, ((it >> 1) & 1) ^ 1, abort)) break;
        Item2 f{};
        const int id = atomicAdd(A.counter, 1);
        const int32_t* lst[2] = {nullptr, nullptr};
        if (id >= A.total_items) {
          f.valid = 0;
        } else {
          const int tile = id / npairs, pr = id - tile * npairs;
          const int hk = pr / A.ppg, ip = pr - hk * A.ppg;
          SeqInfo s;
          int qb;
          if (!decode_item(A.P, tile, s, qb)) {
            f.valid = 2;
          } else {
            f.valid = 1;
            f.start = s.start;
            f.len = s.len;
            f.bcoord = s.bcoord;
            f.qb = qb;
            f.row = s.tile_base + qb;
            f.h[0] = hk * group + 2 * ip;
            f.h[1] = 2 * ip + 1 < group ? f.h[0] + 1 : -1;
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              f.n[t] = 0;
              f.diag[t] = 0;
              if (f.h[t] < 0) continue;
              const int64_t row = (int64_t)f.h[t] * A.P.tiles_ub + f.row;
              f.n[t] = max(0, min(__ldg(A.cnt + row), qb + 1));
              lst[t] = A.idx + row * A.P.cap;
              if (f.n[t] > 0) {
                const int last = __ldg(lst[t] + f.n[t] - 1);
                f.diag[t] = last == qb || last < 0 || last > qb;
              }
            }
          }
        }
        ring[slot] = f;
        mbar_arrive(item_full + slot);
        ++it;
        if (f.valid == 0) break;
        if (f.valid != 1 || (f.n[0] == 0 && f.n[1] == 0)) continue;
        const int hkv = f.h[0] / group;
        const int qrow = f.start + f.qb * kBlock;
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          if (f.n[t] == 0) continue;
          if (!mbar_wait_sleep(q_empty + t, (qld[t] & 1) ^ 1, abort)) { ok = false; break; }
          ++qld[t];
          mbar_arrive_expect_tx(q_full + t, kA2Tile);
          tma_load_4d_hint(sQ + t * kA2Tile, &tm_q, q_full + t, 0, f.h[t], qrow, f.bcoord, stream_once);
          tma_load_4d_hint(sQ + t * kA2Tile + kA2Half, &tm_q, q_full + t, 64, f.h[t], qrow, f.bcoord, stream_once);
        }
        if (!ok) break;
        // union of the two ascending lists, one K/V tile per distinct block
        int j0 = 0, j1 = 0;
        int a0 = f.n[0] > 0 ? __ldg(lst[0]) : 0x7fffffff;
        int a1 = f.n[1] > 0 ? __ldg(lst[1]) : 0x7fffffff;
        while (j0 < f.n[0] || j1 < f.n[1]) {
          int kb = min(a0, a1);
          int m = 0;
          if (a0 == kb) {
            m |= 1;
            ++j0;
            a0 = j0 < f.n[0] ? __ldg(lst[0] + j0) : 0x7fffffff;
          }
          if (a1 == kb) {
            m |= 2;
            ++j1;
            a1 = j1 < f.n[1] ? __ldg(lst[1] + j1) : 0x7fffffff;
          }
          if (j0 >= f.n[0] && j1 >= f.n[1]) m |= 4;  // the item's last union block
          if (kb < 0 || kb > f.qb) {
            raise_error(A.P.err, kErrIndexRange);
            kb = f.qb;
          }
          const int krow = f.start + kb * kBlock;
          const int st = kvseq & 1;
          const uint32_t ph = (kvseq >> 1) & 1;
          if (!mbar_wait_sleep(k_empty + st, ph ^ 1, abort)) { ok = false; break; }
          umask[st] = m;
          // test hook (one-shot): the first producer to reach a key load while it is armed
          // skips that load, so the MMA issuer's wait runs out
          bool withhold = false;
          if (kvseq == 0 && *(volatile int*)&g_test_withhold != 0) withhold = atomicExch(&g_test_withhold, 0) != 0;
          if (!withhold) {
            mbar_arrive_expect_tx(k_full + st, kA2Tile);
            tma_load_4d(sK + st * kA2Tile, &tm_k, k_full + st, 0, hkv, krow, f.bcoord);
            tma_load_4d(sK + st * kA2Tile + kA2Half, &tm_k, k_full + st, 64, hkv, krow, f.bcoord);
          }
          if (!mbar_wait_sleep(v_empty + st, ph ^ 1, abort)) { ok = false; ++kvseq; break; }
          mbar_arrive_expect_tx(v_full + st, kA2Tile);
          tma_load_4d(sV + st * kA2Tile, &tm_v, v_full + st, 0, hkv, krow, f.bcoord);
          tma_load_4d(sV + st * kA2Tile + kA2Half, &tm_v, v_full + st, 64, hkv, krow, f.bcoord);
          ++kvseq;
        }
      }
      if (*abort) {  // let loads still in flight land before the CTA exits
        volatile int no_abort = 0;
        for (uint32_t q = kvseq > 2 ? kvseq - 2 : 0; q < kvseq; ++q) {
          mbar_wait(k_full + (q & 1), (q >> 1) & 1, &no_abort);
          no_abort = 0;
          mbar_wait(v_full + (q & 1), (q >> 1) & 1, &no_abort);
          no_abort = 0;
        }
        for (int t = 0; t < 2; ++t)
          if (qld[t]) {
            mbar_wait(q_full + t, (qld[t] - 1) & 1, &no_abort);
            no_abort = 0;
          }
      }
    } else if (warp == 1 && lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t id_s = idesc_f16(128, 128, DT<T>::is_bf16, false);
      constexpr uint32_t id_o = idesc_f16(128, 128, DT<T>::is_bf16, true);
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV);
      uint32_t it = 0, kvseq = 0, qc[2] = {0, 0}, pc[2] = {0, 0}, oc[2] = {0, 0};
      int users[2] = {0, 0};
      bool ok = true;
      while (ok) {
        const int slot = it & 1;
        if (!mbar_wait_sleep(item_full + slot, (it >> 1) & 1, abort)) break;
        const Item2 f = ring[slot];
        mbar_arrive(item_empty + slot);
        ++it;
        if (f.valid == 0) break;
        if (f.valid != 1 || (f.n[0] == 0 && f.n[1] == 0)) continue;
        int pend[2] = {-1, -1};           // union sequence number of the block whose PV is due
        bool first[2] = {true, true}, qw[2] = {false, false};
        auto issue_pv = [&](int t) -> bool {
          const int q = pend[t], st = q & 1;
          if (first[t]) {  // the previous item's epilogue must have read O_t
            if (!mbar_wait(o_empty + t, (oc[t] & 1) ^ 1, abort)) return false;
            ++oc[t];
          }
          if (!mbar_wait(p_full + t, pc[t] & 1, abort)) return false;
          ++pc[t];
          if (!mbar_wait(v_full + st, (q >> 1) & 1, abort)) return false;
          tc_fence_after();
          const uint32_t t_s = tmem + t * 128, t_o = tmem + 256 + t * 128;
          const uint32_t vb = v_base + st * kA2Tile;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)  // A = P (TMEM, 8 packed columns per 16 keys), B = V (MN-major)
            umma_ts(t_o, t_s + ks * 8, sdesc_sw128(vb + ks * 2048, kA2Half, 1024), id_o,
                    (!first[t] || ks > 0) ? 1u : 0u);
          first[t] = false;
          if (--users[st] == 0) umma_commit(v_empty + st);
          pend[t] = -1;
          return true;
        };
        bool last = false;
        while (!last && ok) {
          const int st = kvseq & 1;
          if (!mbar_wait(k_full + st, (kvseq >> 1) & 1, abort)) { ok = false; break; }
          const int m = umask[st];
          last = (m & 4) != 0;
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (pend[t] >= 0 && !issue_pv(t)) { ok = false; break; }
            if (m & (1 << t)) {
              if (!qw[t]) {
                if (!mbar_wait(q_full + t, qc[t] & 1, abort)) { ok = false; break; }
                ++qc[t];
                qw[t] = true;
              }
              tc_fence_after();
              const uint32_t qb_ = q_base + t * kA2Tile, kb_ = k_base + st * kA2Tile;
#pragma unroll
              for (int ks = 0; ks < 8; ++ks) {
                const uint32_t off = (ks >> 2) * kA2Half + (ks & 3) * 32;
                umma_ss(tmem + t * 128, sdesc_sw128(qb_ + off, 16, 1024), sdesc_sw128(kb_ + off, 16, 1024), id_s,
                        ks > 0);
              }
              umma_commit(s_full + t);
              pend[t] = (int)kvseq;
            }
          }
          if (!ok) break;
          umma_commit(k_empty + st);
          users[st] = __popc(m & 3);
          ++kvseq;
        }
        if (!ok) break;
#pragma unroll
        for (int t = 0; t < 2; ++t)
          if (pend[t] >= 0 && !issue_pv(t)) ok = false;
        if (!ok) break;
#pragma unroll
        for (int t = 0; t < 2; ++t)
          if (f.n[t] > 0) {
            umma_commit(o_full + t);
            umma_commit(q_empty + t);  // the item's last read of Q_t
          }
      }
      umma_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort);
    }
  } else {
    regs_inc<kA2SoftRegs>();
    // ------------------------------------------------------------ softmax + epilogue of tile t
    const int t = (warp - 4) >> 2;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;  // query row within the block (= TMEM lane)
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t t_s = tmem + t * 128 + lane_off;
    const uint32_t t_o = tmem + 256 + t * 128 + lane_off;
    const float c = A.c;
    uint32_t it = 0, sc = 0, oc = 0;
    while (true) {
      const int slot = it & 1;
      if (!mbar_wait_warp_sleep(item_full + slot, (it >> 1) & 1, abort)) break;
      const Item2 f = ring[slot];
      mbar_arrive(item_empty + slot);
      ++it;
      if (f.valid == 0) break;
      if (f.valid != 1 || f.h[t] < 0) continue;
      const int n = f.n[t];
      const int vr = min(kBlock, f.len - f.qb * kBlock);
      T* orow = reinterpret_cast<T*>(A.out) + (int64_t)f.bcoord * A.o_sb +
                (int64_t)(f.start + f.qb * kBlock + r) * A.o_ss + (int64_t)f.h[t] * A.o_sh;
      if (n == 0) {  // empty list: zeros (the reference's acc = 0, l = 1)
        if (r < vr) {
          uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
          for (int i = 0; i < 16; ++i) dst[i] = make_uint4(0, 0, 0, 0);
        }
        continue;
      }
      float m_use = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < n; ++j) {
        if (!mbar_wait_warp_sleep(s_full + t, sc & 1, abort)) { ok = false; break; }
        ++sc;
        tc_fence_after();
        uint32_t u[128];
        tmem_ld32(t_s, *reinterpret_cast<uint32_t(*)[32]>(u));
        tmem_ld32(t_s + 32, *reinterpret_cast<uint32_t(*)[32]>(u + 32));
        tmem_ld32(t_s + 64, *reinterpret_cast<uint32_t(*)[32]>(u + 64));
        tmem_ld32(t_s + 96, *reinterpret_cast<uint32_t(*)[32]>(u + 96));
        tmem_ld_wait();
        if (f.diag[t] && j == n - 1) {  // only the diagonal block needs the causal mask
#pragma unroll
          for (int i = 0; i < 128; ++i)
            if (i > r) u[i] = __float_as_uint(-INFINITY);
        }
        float m0 = -INFINITY, m1 = -INFINITY, m2 = -INFINITY, m3 = -INFINITY;
#pragma unroll
        for (int i = 0; i < 128; i += 8) {
          m0 = max3(m0, __uint_as_float(u[i]), __uint_as_float(u[i + 1]));
          m1 = max3(m1, __uint_as_float(u[i + 2]), __uint_as_float(u[i + 3]));
          m2 = max3(m2, __uint_as_float(u[i + 4]), __uint_as_float(u[i + 5]));
          m3 = max3(m3, __uint_as_float(u[i + 6]), __uint_as_float(u[i + 7]));
        }
        const float m_blk = fmaxf(fmaxf(m0, m1), fmaxf(m2, m3)) * c;
        float scale_o = 1.f;
        if (j == 0) {
          m_use = m_blk;
        } else if (m_blk > m_use) {
          scale_o = ex2_approx(m_use - m_blk);
          m_use = m_blk;
          l *= scale_o;
        }
        // P = exp2(s*c - m) as 16-bit pairs over S columns [0, 64); one pair in kA2PolyEvery
        // on the FMA pipe (exp2_poly2), the rest by ex2.approx
        const float neg_m = -m_use;
        float rs0 = 0.f, rs1 = 0.f;
        // packed pair k overwrites u[k] (u[2k] and u[2k+1] are read first), so no second array
#pragma unroll
        for (int k = 0; k < 64; ++k) {
          float x0, x1, p0, p1;
          fma2(x0, x1, __uint_as_float(u[2 * k]), __uint_as_float(u[2 * k + 1]), c, c, neg_m, neg_m);
          if ((k % kA2PolyEvery) == kA2PolyEvery - 1) {
            exp2_poly2(x0, x1, p0, p1);  // masked (-inf) entries give 2^-126 here, negligible
          } else {
            p0 = ex2_approx(x0);
            p1 = ex2_approx(x1);
          }
          add2(rs0, rs1, rs0, rs1, p0, p1);
          u[k] = DT<T>::pack(p0, p1);
        }
        tmem_st32(t_s, *reinterpret_cast<uint32_t(*)[32]>(u));
        tmem_st32(t_s + 32, *reinterpret_cast<uint32_t(*)[32]>(u + 32));
        if (__any_sync(0xffffffffu, scale_o != 1.f)) {
          // O_t holds the blocks before this one (PV_t(previous) completed before S_t(this)
          // did); rescale this row before PV_t(this) may start (p_full below)
#pragma unroll
          for (int ch = 0; ch < 4; ++ch) {
            uint32_t o[32];
            tmem_ld32(t_o + ch * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] = __float_as_uint(__uint_as_float(o[i]) * scale_o);
            tmem_st32(t_o + ch * 32, o);
          }
        }
        tmem_st_wait();
        l += rs0 + rs1;
        tc_fence_before();
        mbar_arrive(p_full + t);
      }
      if (!ok) break;
      // ---- epilogue: O / l straight from TMEM to this thread's output row
      if (!mbar_wait_warp_sleep(o_full + t, oc & 1, abort)) break;
      ++oc;
      tc_fence_after();
      uint32_t o[128];
      tmem_ld32(t_o, *reinterpret_cast<uint32_t(*)[32]>(o));
      tmem_ld32(t_o + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
      tmem_ld32(t_o + 64, *reinterpret_cast<uint32_t(*)[32]>(o + 64));
      tmem_ld32(t_o + 96, *reinterpret_cast<uint32_t(*)[32]>(o + 96));
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(o_empty + t);  // O_t may be overwritten by the next item's first PV
      const float inv = 1.f / l;
      if (r < vr) {
        const uint64_t pol = l2_policy_evict_first();  // the output is not read again here
        uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
        for (int q4 = 0; q4 < 16; ++q4) {
          uint32_t pk[4];
#pragma unroll
          for (int i = 0; i < 4; ++i)
            pk[i] = DT<T>::pack(__uint_as_float(o[q4 * 8 + 2 * i]) * inv, __uint_as_float(o[q4 * 8 + 2 * i + 1]) * inv);
          st_global_hint(dst + q4, make_uint4(pk[0], pk[1], pk[2], pk[3]), pol);
        }
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
