// Block-sparse causal GQA attention forward on the 5th-generation tensor cores.
//
// Reference: ops/flashprefill_native_forward.py:228-344 (_flash_forward) and
// ops/flashprefill_varlen_func.py:449-575 (_flash_block_sparse_varlen): for each query
// block and each selected key block (ascending), S = (Q K^T) * c with c = scale*log2(e),
// the diagonal block masked causally, online softmax in exp2, P rounded to the input
// dtype for the P V product, O = acc / l stored in the input dtype.  A row whose list is
// empty outputs zeros (the reference starts l at 1.0 and acc at 0).
//
// Persistent kernel, one CTA per SM, 640 threads (20 warps), running two independent
// pipelines that share the tensor core.  A work item is one (query block, query head), or
// one chunk of a long row (fp_split.cu); each pipeline fetches its own items, heavy-first,
// from one atomic counter.
//   warp 0 / warp 2    scheduler + TMA producer (Q, then K and V of each listed block)
//                      of pipeline 0 / 1, with single-slot Q, K and V buffers
//   warp 1 / warp 3    tcgen05.mma issuer of pipeline 0 / 1 (warp 1 owns the TMEM
//                      allocation): S_x(j) = Q K^T when K_x(j) has landed, PV_x(j) when
//                      P_x(j) and V_x(j) are ready
//   warps 4-11 / 12-19 softmax / epilogue of pipeline 0 / 1: two warpgroups per pipeline,
//                      thread (half hh, row r) owns 64 columns of query row r (= TMEM lane)
// While one pipeline's softmax runs, the tensor core works for the other.  PV_x(j) is
// issued before S_x(j+1), so O_x is final whenever S_x(j+1) completes: the exact
// running-max rescale of O (as in the reference) never waits.
// TMEM columns: S_0 [0,128), S_1 [128,256), O_0 [256,384), O_1 [384,512).  P (16-bit
// pairs) is written over the first 64 columns of S and read by the TS-form MMA.
// The largest P of a row is exactly 1.0, which keeps the bf16 rounding of P at the
// reference's level (a lazy max that lets P grow above 1 adds up to one bf16 ulp of P).
#include "fp_common.cuh"
#include "fp_split.cu"

namespace fpb {

constexpr int kMaxOutPeers = 7;  // peers of an output gather (8 GPUs of one NVSwitch domain)

struct AttnArgs {
  SeqProblem P;
  float c;                   // fp32(1/sqrt(D)) * fp32(log2 e)
  const int32_t* idx;        // [hq][tiles_ub][cap] ascending block lists
  const int32_t* cnt;        // [hq][tiles_ub]
  int* counter;              // work-item counter, zero at launch
  int profile;               // accumulate g_attn_prof
  int trace;                 // record g_attn_trace for CTA 0
  int alt_issue;             // one MMA issuer alternating between the pipelines (else one per pipeline)
  int total_items;           // tiles_ub * hq
  void* out;                 // output base (masked-store path)
  int64_t o_sb, o_ss, o_sh;  // output strides in elements
  // long rows split into chunks (fp_split.cu); split = 0 processes every row whole
  int split;
  const SplitEntry* sp_entries;
  const int* sp_head;        // plan header: [0] chunk entries, [3] split threshold
  const int* sp_rowidx;      // [hq][tiles_ub] split-row index or -1 (rows over the threshold)
  int* sp_counters;          // chunks finished per split row, at the row's first entry
  float* sp_part;            // per chunk entry: O [128][128], m [128], l [2][128]
  // other GPUs' copies of the output (same layout and strides as `out`, reached over
  // NVLink): the epilogue writes every output tile there too (kernel instance kPeers)
  int n_peers;
  void* peer_out[kMaxOutPeers];
};

constexpr int kAttnThreads = 640;
// One exp2 pair in kPolyEvery is evaluated on the FMA pipe (exp2_poly2), the rest by MUFU.
#ifndef FPB_POLY_EVERY
#define FPB_POLY_EVERY 4
#endif
constexpr int kPolyEvery = FPB_POLY_EVERY;
#ifndef FPB_SOFTMAX_PROBE
#define FPB_SOFTMAX_PROBE 0
#endif
constexpr bool kSoftmaxProbe = FPB_SOFTMAX_PROBE;

// Register split (per thread): the kernel is compiled for 96 (= 65536 / 640, rounded down
// to a multiple of 8); role warps 0-3 give back to 64 and the four softmax warpgroups grow
// to 104: 128*64 + 512*104 = 61440 <= 640*96 = 61440.  The host refuses to launch unless
// the compiled register count is exactly kAttnLaunchRegs.
constexpr int kAttnLaunchRegs = 96, kAttnRoleRegs = 64, kAttnSoftmaxRegs = 104;
static_assert(128 * kAttnRoleRegs + 512 * kAttnSoftmaxRegs <= kAttnThreads * kAttnLaunchRegs, "register split");

// Instrumentation, compiled in only with -DFPB_ATTN_PROFILE=1 (build flag), then enabled at
// run time by FLASHPREFILL_B200_PROFILE=1 (cycles spent per wait / phase, summed over CTAs;
// indices: kProfNames in fp_api.cu) and FLASHPREFILL_B200_TRACE=<file> (event trace of CTA 0:
// (clock, kind << 56 | a << 28 | b) pairs).  In the default build every hook below is empty
// and no clock is read on the hot path.
#ifndef FPB_ATTN_PROFILE
#define FPB_ATTN_PROFILE 0
#endif
constexpr int kProfSlots = 25;
constexpr int kTraceCap = 1 << 16;
#if FPB_ATTN_PROFILE
__device__ unsigned long long g_attn_prof[kProfSlots];
__device__ unsigned long long g_attn_trace[2 * kTraceCap];
__device__ unsigned int g_attn_trace_n;
struct ProfAcc {  // counters live in shared memory, flushed once per CTA
  unsigned long long* sm;
  __device__ void add(int i, unsigned long long c) {
    if (sm) atomicAdd(sm + i, c);
  }
};
__device__ __forceinline__ unsigned long long clk() { return clock64(); }
#define trace(on, kind, a, b) trace_((on), trace_ctr, (kind), (a), (b))
__device__ __forceinline__ void trace_(bool on, unsigned* ctr, uint32_t kind, uint32_t a, uint32_t b) {
  if (!on) return;
  const unsigned long long now = clock64();
  const unsigned i = atomicAdd(ctr, 1u);  // shared-memory counter: short round trip
  if (i < kTraceCap) {
    g_attn_trace[2 * i] = now;
    g_attn_trace[2 * i + 1] = ((unsigned long long)kind << 56) | ((unsigned long long)a << 28) | b;
  }
}
#define FPB_TW(slot, call)                   \
  ({                                         \
    const unsigned long long t0_ = clk();    \
    const bool r_ = (call);                  \
    pa.add(slot, clk() - t0_);               \
    r_;                                      \
  })
#else
struct ProfAcc {
  unsigned long long* sm;
  __device__ __forceinline__ void add(int, unsigned long long) {}
};
__device__ __forceinline__ unsigned long long clk() { return 0; }
#define trace(on, kind, a, b) ((void)0)
#define FPB_TW(slot, call) (call)
#endif
constexpr uint32_t kAttnTile = 128 * 128 * 2;
constexpr uint32_t kAttnHalf = kAttnTile / 2;

// 6 tiles, alignment slack, barriers / item ring / counters, row max and sum exchange (6 KB)
__host__ __device__ constexpr size_t attn_smem_bytes() { return (size_t)kAttnTile * 6 + 1024 + 1024 + 6400; }

// One work item as published by a pipeline's scheduler in its smem ring.
struct ItemInfo {
  int valid;  // 0: no more work, 1: item, 2: empty slot of the grid (skip)
  int start, len, tile_base, bcoord, qb, h, n, last_kb;
  int j0;     // first list entry of this item (a chunk of a split row; 0 otherwise)
  int chunk;  // split_code(entry, chunk, nchunks) of a chunk of a split row, or -1 for a whole row
  int pad[5];
};

// A chunk of a split row stores its unnormalised O (this thread's row, 64 columns from TMEM
// address t_o) as fp32 to dst.  Out of line for the same reason as split_merge_row.
__device__ __noinline__ void split_store_partial(uint32_t t_o, float* dst) {
  float4* po = reinterpret_cast<float4*>(dst);
#pragma unroll 1
  for (int h = 0; h < 2; ++h) {
    uint32_t o[32];
    tmem_ld32(t_o + h * 32, o);
    tmem_ld_wait();
#pragma unroll
    for (int i = 0; i < 8; ++i)
      po[h * 8 + i] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]),
                                  __uint_as_float(o[4 * i + 2]), __uint_as_float(o[4 * i + 3]));
  }
}

// The last chunk of a split row to finish merges the partial results of all its chunks (row
// r, columns hh*64..+64 of this thread):  O = sum_c O_c 2^(m_c - M) / sum_c l_c 2^(m_c - M).
// Kept out of line so the kernel's register allocation is not shaped by it.
// Consecutive chunks' partials are `stride` floats apart.
template <typename T>
__device__ __noinline__ void split_merge_row(const float* p0, int nchunks, int r, int hh, int vr, T* orow,
                                             int64_t o_ss, int64_t stride = kSplitPartBytes / 4) {
  float M = -INFINITY;
  for (int cix = 0; cix < nchunks; ++cix)
    M = fmaxf(M, __ldcg(p0 + (int64_t)cix * stride + 128 * 128 + r));
  float Lsum = 0.f;
  for (int cix = 0; cix < nchunks; ++cix) {
    const float* pc = p0 + (int64_t)cix * stride + 128 * 128;
    Lsum += (__ldcg(pc + 128 + r) + __ldcg(pc + 256 + r)) * ex2_approx(__ldcg(pc + r) - M);
  }
  const float invL = 1.f / Lsum;
  // 16 columns at a time, so the merge holds few registers
#pragma unroll 1
  for (int g = 0; g < 4; ++g) {
    float acc[16];
#pragma unroll
    for (int i = 0; i < 16; ++i) acc[i] = 0.f;
    for (int cix = 0; cix < nchunks; ++cix) {
      const float* pc = p0 + (int64_t)cix * stride;
      const float sc = ex2_approx(__ldcg(pc + 128 * 128 + r) - M);
      const float4* src = reinterpret_cast<const float4*>(pc + r * 128 + hh * 64 + g * 16);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const float4 v4 = __ldcg(src + i);
        acc[4 * i] += v4.x * sc;
        acc[4 * i + 1] += v4.y * sc;
        acc[4 * i + 2] += v4.z * sc;
        acc[4 * i + 3] += v4.w * sc;
      }
    }
    if (r < vr) {
      uint4* dst = reinterpret_cast<uint4*>(orow + (int64_t)r * o_ss + hh * 64 + g * 16);
#pragma unroll
      for (int q = 0; q < 2; ++q) {
        uint32_t pk[4];
#pragma unroll
        for (int i = 0; i < 4; ++i)
          pk[i] = DT<T>::pack(acc[q * 8 + 2 * i] * invL, acc[q * 8 + 2 * i + 1] * invL);
        dst[q] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
    }
  }
}

// Epilogue of one chunk of a split row, for the 256 epilogue threads of a pipeline (row r,
// half hh): stores the unnormalised O, the running max m and the row sum l of this chunk;
// the chunk that finishes its row last merges all of them into the output.  Arrives on
// o_empty once O is read, and passes the pipeline's group barrier (epi) twice, at phases ep
// and ep + 1.  Returns false if a barrier wait gave up.  Kept out of line: inlined, its
// code raised the kernel's register pressure and slowed the softmax loop.
template <typename T>
__device__ __noinline__ bool split_chunk_epilogue(uint32_t t_o, int code, float m_use, float l, int r, int hh,
                                                  int vr, T* orow, int64_t o_ss, float* sp_part, int* sp_counters,
                                                  int* last_chunk, uint64_t* epi, uint64_t* o_empty, uint32_t ep,
                                                  volatile int* abort) {
  const int entry = code & (kSplitMaxEntries - 1), nchunks = code >> 24;
  const int e0 = entry - ((code >> 17) & 127);  // the row's first entry
  float* part = sp_part + (int64_t)entry * (kSplitPartBytes / 4);
  split_store_partial(t_o, part + r * 128 + hh * 64);
  tc_fence_before();
  mbar_arrive(o_empty);  // O may be overwritten by the next item's first PV
  if (hh == 0) part[128 * 128 + r] = m_use;
  part[128 * 128 + 128 + hh * 128 + r] = l;
  __threadfence();
  mbar_arrive(epi);
  if (!mbar_wait_warp_sleep(epi, ep & 1, abort)) return false;
  if (hh == 0 && r == 0) *last_chunk = atomicAdd(sp_counters + e0, 1) == nchunks - 1;
  mbar_arrive(epi);
  if (!mbar_wait_warp_sleep(epi, (ep + 1) & 1, abort)) return false;
  if (*(volatile int*)last_chunk) {
    __threadfence();
    split_merge_row<T>(sp_part + (int64_t)e0 * (kSplitPartBytes / 4), nchunks, r, hh, vr, orow, o_ss);
  }
  return true;
}

// Copy `bytes` (a multiple of 16) from src to the same byte offset of every peer output.
__device__ __forceinline__ void copy_row_to_peers(const AttnArgs& A, int64_t byte_off, const void* src, int bytes) {
  for (int p = 0; p < A.n_peers; ++p) {
    uint4* dst = reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(A.peer_out[p]) + byte_off);
    for (int i = 0; i < bytes / 16; ++i) dst[i] = reinterpret_cast<const uint4*>(src)[i];
  }
}

template <typename T, bool kPeers>
__global__ void __launch_bounds__(kAttnThreads, 1)
    sparse_attn_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                       const __grid_constant__ CUtensorMap tm_v, const __grid_constant__ CUtensorMap tm_o,
                       const AttnArgs A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // pipeline x owns [x * 3 tiles): Q, K, V
  uint64_t* bars = reinterpret_cast<uint64_t*>(smem + 6 * kAttnTile);
  uint64_t* item_full = bars + 0;    // [pipeline][slot]
  uint64_t* item_empty = bars + 4;   // [pipeline][slot]
  uint64_t* q_full = bars + 8;       // [pipeline]
  uint64_t* q_empty = bars + 10;
  uint64_t* k_full = bars + 12;
  uint64_t* k_empty = bars + 14;
  uint64_t* v_full = bars + 16;
  uint64_t* v_empty = bars + 18;
  uint64_t* s_full = bars + 20;
  uint64_t* p_full = bars + 22;
  uint64_t* o_full = bars + 24;
  uint64_t* o_empty = bars + 26;
  uint64_t* epi = bars + 28;         // bounded sync of a pipeline's 128 epilogue threads
  uint64_t* mma_done = bars + 30;   // [pipeline]
  uint64_t* mx_bar = bars + 32;      // [pipeline] row-max exchange of the two halves
  uint64_t* stage_free = bars + 34;  // [pipeline] epilogue done with the V tile (output staging)
  ItemInfo* ring = reinterpret_cast<ItemInfo*>(bars + 40);  // [pipeline][slot]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ring + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  unsigned* trace_ctr = tmem_slot + 3;
  unsigned long long* prof_smem = reinterpret_cast<unsigned long long*>(tmem_slot + 4);  // [kProfSlots]
  float* xchg = reinterpret_cast<float*>(smem + 6 * kAttnTile + 1024);  // 1536 floats

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int i = 0; i < 4; ++i) {
      mbar_init(item_full + i, 1);
      mbar_init(item_empty + i, 1 + 256);
    }
    for (int x = 0; x < 2; ++x) {
      mbar_init(q_full + x, 1);
      mbar_init(q_empty + x, 1);
      mbar_init(k_full + x, 1);
      mbar_init(k_empty + x, 1);
      mbar_init(v_full + x, 1);
      mbar_init(v_empty + x, 1);
      mbar_init(s_full + x, 1);
      mbar_init(p_full + x, 256);
      mbar_init(o_full + x, 1);
      mbar_init(o_empty + x, 256);
      mbar_init(epi + x, 256);
      mbar_init(mx_bar + x, 256);
      mbar_init(stage_free + x, 1);
    }
    mbar_init(mma_done, 1);
    mbar_init(mma_done + 1, 1);
    *abort = 0;
    *trace_ctr = 0;
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
  const int group = A.P.hq / A.P.hk;
  const bool tr = A.trace && blockIdx.x == 0;

  if (warp < 4) {
  regs_dec<kAttnRoleRegs>();
  if ((warp == 0 || warp == 2) && lane == 0) {
    // ------------------------------------------------------------ scheduler + producer of pipeline x
    const int x = warp >> 1;
    uint8_t* sQ = smem + x * 3 * kAttnTile;
    uint8_t* sK = sQ + kAttnTile;
    uint8_t* sV = sK + kAttnTile;
    prefetch_tmap(&tm_q);
    prefetch_tmap(&tm_k);
    prefetch_tmap(&tm_v);
    const uint64_t stream_once = l2_policy_evict_first();
    uint32_t it = 0, kseq = 0, vseq = 0, qld = 0, sfc = 0;
    // chunks of split rows come first in the work order (they are the longest work)
    const int n_ent = A.split ? A.sp_head[0] : 0;
    const int split_thr = A.split ? A.sp_head[3] : 0x7fffffff;  // only rows above it can be split
    bool ok = true;
    while (ok) {
      const int slot = it & 1;
      if (!FPB_TW(15, mbar_wait_sleep(item_empty + 2 * x + slot, ((it >> 1) & 1) ^ 1, abort))) break;
      ItemInfo f{};
      const int id = atomicAdd(A.counter, 1);
      const int32_t* lst = nullptr;
      if (id >= n_ent + A.total_items) {
        f.valid = 0;
      } else {
        SeqInfo s;
        int qb;
        const SplitEntry se = id < n_ent ? A.sp_entries[id] : SplitEntry{id - n_ent, 0, 0, -1};
        const int tile = se.item / A.P.hq, h = se.item - tile * A.P.hq;
        if (!decode_item(A.P, tile, s, qb)) {
          f.valid = 2;
        } else {
          f.valid = 1;
          f.start = s.start;
          f.len = s.len;
          f.tile_base = s.tile_base;
          f.bcoord = s.bcoord;
          f.qb = qb;
          f.h = h;
          const int64_t row = (int64_t)f.h * A.P.tiles_ub + s.tile_base + qb;
          const int n_row = max(0, min(__ldg(A.cnt + row), qb + 1));
          f.chunk = -1;
          if (id < n_ent) {  // one chunk of a split row
            f.j0 = se.chunk * kSplitChunk;
            f.n = min(kSplitChunk, n_row - f.j0);
            f.chunk = split_code(id, se.chunk, se.nchunks);
          } else {
            f.n = n_row;
            if (n_row > split_thr && __ldg(A.sp_rowidx + row) >= 0) f.valid = 2;  // done as chunks
          }
          lst = A.idx + row * A.P.cap + f.j0;
          f.last_kb = f.n > 0 ? __ldg(lst + f.n - 1) : -1;
        }
      }
      ring[2 * x + slot] = f;
      mbar_arrive(item_full + 2 * x + slot);
      if (f.valid == 1) pa.add(19, 1);
      ++it;
      if (f.valid == 0) break;
      if (f.valid == 2 || f.n == 0) continue;
      const int hk = f.h / group;
      if (!FPB_TW(14, mbar_wait_sleep(q_empty + x, (qld & 1) ^ 1, abort))) break;
      ++qld;
      const int qrow = f.start + f.qb * kBlock;
      mbar_arrive_expect_tx(q_full + x, kAttnTile);
      tma_load_4d_hint(sQ, &tm_q, q_full + x, 0, f.h, qrow, f.bcoord, stream_once);
      tma_load_4d_hint(sQ + kAttnHalf, &tm_q, q_full + x, 64, f.h, qrow, f.bcoord, stream_once);
      for (int j = 0; j < f.n; ++j) {
        int kb = __ldg(lst + j);
        if (kb < 0 || kb > f.qb) {
          raise_error(A.P.err, kErrIndexRange);
          kb = f.qb;
        }
        const int krow = f.start + kb * kBlock;
        if (!FPB_TW(13, mbar_wait_sleep(k_empty + x, (kseq & 1) ^ 1, abort))) { ok = false; break; }
        trace(tr, 1, x, kseq);
        ++kseq;
        // test hook (one-shot): the first producer to reach a key load while it is armed skips
        // that load, so its MMA issuer's wait runs out
        bool withhold = false;
        if (kseq == 1 && *(volatile int*)&g_test_withhold != 0) withhold = atomicExch(&g_test_withhold, 0) != 0;
        if (!withhold) {
          mbar_arrive_expect_tx(k_full + x, kAttnTile);
          tma_load_4d(sK, &tm_k, k_full + x, 0, hk, krow, f.bcoord);
          tma_load_4d(sK + kAttnHalf, &tm_k, k_full + x, 64, hk, krow, f.bcoord);
        }
        if (!FPB_TW(16, mbar_wait_sleep(v_empty + x, (vseq & 1) ^ 1, abort))) { ok = false; break; }
        if (j == 0 && qld > 1) {  // the previous item's epilogue stages its output in the V tile
          if (!FPB_TW(16, mbar_wait_sleep(stage_free + x, sfc & 1, abort))) { ok = false; break; }
          ++sfc;
        }
        trace(tr, 2, x, vseq);
        ++vseq;
        mbar_arrive_expect_tx(v_full + x, kAttnTile);
        tma_load_4d(sV, &tm_v, v_full + x, 0, hk, krow, f.bcoord);
        tma_load_4d(sV + kAttnHalf, &tm_v, v_full + x, 64, hk, krow, f.bcoord);
      }
    }
    if (*abort) {  // let loads still in flight land before the CTA exits
      volatile int no_abort = 0;
      if (kseq) mbar_wait(k_full + x, (kseq - 1) & 1, &no_abort);
      if (vseq) mbar_wait(v_full + x, (vseq - 1) & 1, &no_abort);
      if (qld) mbar_wait(q_full + x, (qld - 1) & 1, &no_abort);
    }
  } else if (A.alt_issue && warp == 1 && lane == 0) {
    // ------------------------------------------------------------ MMA issuer (both pipelines)
    // PV_x(j) and S_x(j+1) are issued back to back, and the pipelines take turns: while the
    // tensor core works for one pipeline, the other one's softmax runs.  A pipeline whose
    // turn it is but that waits for loads or an item (not for its softmax) lets the other go.
    constexpr uint32_t id_s = idesc_f16(128, 128, DT<T>::is_bf16, false);
    constexpr uint32_t id_o = idesc_f16(128, 128, DT<T>::is_bf16, true);
    enum { kNeedItem = 0, kNeedS = 1, kNeedPV = 2, kDone = 3 };
    int st[2] = {kNeedItem, kNeedItem}, jj[2] = {0, 0}, nn[2] = {0, 0};
    uint32_t it[2] = {0, 0}, qc[2] = {0, 0}, kc[2] = {0, 0}, vc[2] = {0, 0}, pc[2] = {0, 0}, oc[2] = {0, 0};
    int turn = 0;
    uint64_t last_progress = global_timer_ns();
    auto try_s = [&](int x) -> bool {
      if (st[x] != kNeedS) return false;
      if (!(jj[x] > 0 || mbar_probe(q_full + x, qc[x] & 1))) return false;
      if (!mbar_probe(k_full + x, kc[x] & 1)) return false;
      if (jj[x] == 0) ++qc[x];
      ++kc[x];
      tc_fence_after();
      const uint32_t q_base = smem_u32(smem + x * 3 * kAttnTile);
      const uint32_t k_base = q_base + kAttnTile;
#pragma unroll
      for (int ks = 0; ks < 8; ++ks) {
        const uint32_t off = (ks >> 2) * kAttnHalf + (ks & 3) * 32;
        umma_ss(tmem + x * 128, sdesc_sw128(q_base + off, 16, 1024), sdesc_sw128(k_base + off, 16, 1024), id_s,
                ks > 0);
      }
      umma_commit(k_empty + x);
      umma_commit(s_full + x);
      if (jj[x] == nn[x] - 1) umma_commit(q_empty + x);  // the item's last read of Q
      trace(tr, 3, x, kc[x]);
      st[x] = kNeedPV;
      return true;
    };
    auto pv_ready = [&](int x) -> bool {
      return st[x] == kNeedPV && (jj[x] > 0 || mbar_probe(o_empty + x, (oc[x] & 1) ^ 1)) &&
             mbar_probe(p_full + x, pc[x] & 1) && mbar_probe(v_full + x, vc[x] & 1);
    };
    auto issue_pv = [&](int x) {
      if (jj[x] == 0) ++oc[x];
      ++pc[x];
      ++vc[x];
      tc_fence_after();
      const uint32_t v_base = smem_u32(smem + x * 3 * kAttnTile + 2 * kAttnTile);
#pragma unroll
      for (int ks = 0; ks < 8; ++ks)
        umma_ts(tmem + 256 + x * 128, tmem + x * 128 + ks * 8, sdesc_sw128(v_base + ks * 2048, kAttnHalf, 1024),
                id_o, (jj[x] > 0 || ks > 0) ? 1u : 0u);
      umma_commit(v_empty + x);
      trace(tr, 4, x, pc[x]);
      if (jj[x] == nn[x] - 1) {
        umma_commit(o_full + x);
        st[x] = kNeedItem;
      } else {
        ++jj[x];
        st[x] = kNeedS;
      }
    };
    while (st[0] != kDone || st[1] != kDone) {
      bool progress = false;
#pragma unroll
      for (int x = 0; x < 2; ++x) {
        if (st[x] == kNeedItem) {
          const int slot = it[x] & 1;
          if (mbar_probe(item_full + 2 * x + slot, (it[x] >> 1) & 1)) {
            const ItemInfo f = ring[2 * x + slot];
            mbar_arrive(item_empty + 2 * x + slot);
            ++it[x];
            progress = true;
            if (f.valid == 0) {
              st[x] = kDone;
            } else if (f.valid == 1 && f.n > 0) {
              st[x] = kNeedS;
              jj[x] = 0;
              nn[x] = f.n;
            }
          }
        }
        if (try_s(x)) progress = true;
      }
      const int y = turn, z = turn ^ 1;
      if (pv_ready(y)) {
        issue_pv(y);
        try_s(y);
        turn = z;
        progress = true;
      } else if (st[y] != kNeedPV && pv_ready(z)) {
        issue_pv(z);
        try_s(z);
        progress = true;
      }
      if (progress) {
        last_progress = global_timer_ns();
      } else if (*abort || global_timer_ns() - last_progress > g_wait_limit_ns) {
        *abort = 1;
        break;
      }
    }
    umma_commit(mma_done);
    volatile int no_abort = 0;
    mbar_wait(mma_done, 0, &no_abort);
  } else if (!A.alt_issue && (warp == 1 || warp == 3) && lane == 0) {
    // ------------------------------------------------------------ MMA issuer of pipeline x
    // One issuing thread per pipeline: tcgen05.mma issue stalls while the tensor core's
    // instruction queue is full (about one group of eight), so an issuer shared by both
    // pipelines would hold one pipeline's ready MMAs behind the other's.
    const int x = warp >> 1;
    constexpr uint32_t id_s = idesc_f16(128, 128, DT<T>::is_bf16, false);
    constexpr uint32_t id_o = idesc_f16(128, 128, DT<T>::is_bf16, true);
    const uint32_t q_base = smem_u32(smem + x * 3 * kAttnTile);
    const uint32_t k_base = q_base + kAttnTile, v_base = q_base + 2 * kAttnTile;
    const uint32_t t_s = tmem + x * 128, t_o = tmem + 256 + x * 128;
    uint32_t it = 0, qc = 0, kc = 0, vc = 0, pc = 0, oc = 0;
    bool ok = true;
    while (ok) {
      const int slot = it & 1;
      if (!FPB_TW(4, mbar_wait_sleep(item_full + 2 * x + slot, (it >> 1) & 1, abort))) break;
      const ItemInfo f = ring[2 * x + slot];
      mbar_arrive(item_empty + 2 * x + slot);
      ++it;
      if (f.valid == 0) break;
      if (f.valid != 1 || f.n == 0) continue;
      for (int j = 0; j < f.n; ++j) {
        if (j == 0) {
          if (!FPB_TW(3, mbar_wait_sleep(q_full + x, qc & 1, abort))) { ok = false; break; }
          ++qc;
        }
        if (!FPB_TW(1, mbar_wait_sleep(k_full + x, kc & 1, abort))) { ok = false; break; }
        ++kc;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          const uint32_t off = (ks >> 2) * kAttnHalf + (ks & 3) * 32;
          umma_ss(t_s, sdesc_sw128(q_base + off, 16, 1024), sdesc_sw128(k_base + off, 16, 1024), id_s, ks > 0);
        }
        umma_commit(k_empty + x);
        umma_commit(s_full + x);
        if (j == f.n - 1) umma_commit(q_empty + x);  // the item's last read of Q
        trace(tr, 3, x, kc);
        if (j == 0) {  // the previous item's epilogue must have read O
          if (!FPB_TW(3, mbar_wait_sleep(o_empty + x, (oc & 1) ^ 1, abort))) { ok = false; break; }
          ++oc;
        }
        if (!FPB_TW(0, mbar_wait_sleep(p_full + x, pc & 1, abort))) { ok = false; break; }
        ++pc;
        if (!FPB_TW(2, mbar_wait_sleep(v_full + x, vc & 1, abort))) { ok = false; break; }
        ++vc;
        tc_fence_after();
#pragma unroll
        for (int ks = 0; ks < 8; ++ks) {
          // A = P (TMEM, 16-bit pairs: 8 columns per 16 keys); B = V rows ks*16.. (MN-major)
          umma_ts(t_o, t_s + ks * 8, sdesc_sw128(v_base + ks * 2048, kAttnHalf, 1024), id_o,
                  (j > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(v_empty + x);
        trace(tr, 4, x, pc);
        if (j == f.n - 1) umma_commit(o_full + x);
      }
    }
    umma_commit(mma_done + x);
    volatile int no_abort = 0;
    mbar_wait(mma_done + x, 0, &no_abort);
  }
  } else {
    regs_inc<kAttnSoftmaxRegs>();
    // ------------------------------------------------------------ softmax + epilogue of pipeline x
    // Two warpgroups per pipeline: thread (hh, r) owns columns [64*hh, 64*hh + 64) of query
    // row r in S, P and O.  The two halves of a row agree on its running max through shared
    // memory once per block (mx_bar); each keeps its own partial row sum.
    const int w = warp - 4;
    const int x = w >> 3;
    const int hh = (w >> 2) & 1;
    const int quad = warp & 3;
    const int r = quad * 32 + lane;    // query row within the block (= TMEM lane)
    const uint32_t lane_off = (uint32_t)(quad * 32) << 16;
    const uint32_t t_s = tmem + x * 128 + lane_off;
    const uint32_t t_o = tmem + 256 + x * 128 + lane_off + hh * 64;
    float* xch = xchg + x * 512;                // row max: [parity][half][row]
    float* xl = xchg + 1024 + x * 256;          // row sum: [half][row]
    int* last_chunk = reinterpret_cast<int*>(xchg + 1536) + x;  // this pipeline finished a split row
    const float c = A.c;
    const bool rec = tr && r == 0 && hh == 0;
    uint32_t it = 0, sc = 0, oc = 0, ep = 0, mp = 0;
    auto group_sync = [&]() -> bool {  // all 256 threads of this pipeline, bounded
      mbar_arrive(epi + x);
      return FPB_TW(12, mbar_wait_warp_sleep(epi + x, (ep++) & 1, abort));
    };
    while (true) {
      const int slot = it & 1;
      if (!FPB_TW(7, mbar_wait_warp_sleep(item_full + 2 * x + slot, (it >> 1) & 1, abort))) break;
      const ItemInfo f = ring[2 * x + slot];
      mbar_arrive(item_empty + 2 * x + slot);
      ++it;
      if (f.valid == 0) break;
      if (f.valid == 2) continue;
      const int hx = f.h;
      const int n = f.n;
      const int vr = min(kBlock, f.len - f.qb * kBlock);
      T* orow = reinterpret_cast<T*>(A.out) + (int64_t)f.bcoord * A.o_sb +
                (int64_t)(f.start + f.qb * kBlock) * A.o_ss + (int64_t)hx * A.o_sh;
      if (n == 0) {  // empty list: zeros (the reference's acc = 0, l = 1)
        if (r < vr) {
          uint4* dst = reinterpret_cast<uint4*>(orow + (int64_t)r * A.o_ss + hh * 64);
#pragma unroll
          for (int i = 0; i < 8; ++i) dst[i] = make_uint4(0, 0, 0, 0);
          if constexpr (kPeers)
            copy_row_to_peers(A, reinterpret_cast<const uint8_t*>(dst) - reinterpret_cast<const uint8_t*>(A.out),
                              dst, 128);
        }
        continue;
      }
      // lists are ascending and causal, so only the last entry can be the diagonal block
      const bool last_is_diag = f.last_kb == f.qb || f.last_kb < 0 || f.last_kb > f.qb;
      float m_use = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < n; ++j) {
        const bool diag = last_is_diag && j == n - 1;
        if (!FPB_TW(5, mbar_wait_warp_sleep(s_full + x, sc & 1, abort))) { ok = false; break; }
        ++sc;
        tc_fence_after();
        const unsigned long long tp1 = clk();
        trace(rec, 5, x, j);
        pa.add(20, 1);
        uint32_t ua[32], ub[32];
        tmem_ld32(t_s + hh * 64, ua);
        tmem_ld32(t_s + hh * 64 + 32, ub);
        tmem_ld_wait();
        pa.add(22, clk() - tp1);
#define FPB_U(i) ((i) < 32 ? ua[(i)] : ub[(i) - 32])
        if (diag) {  // only the diagonal block needs the causal mask
#pragma unroll
          for (int i = 0; i < 64; ++i)
            if (hh * 64 + i > r) FPB_U(i) = __float_as_uint(-INFINITY);
        }
        float mx = -INFINITY, m1 = -INFINITY;
#pragma unroll
        for (int i = 0; i < 64; i += 4) {
          mx = max3(mx, __uint_as_float(FPB_U(i)), __uint_as_float(FPB_U(i + 1)));
          m1 = max3(m1, __uint_as_float(FPB_U(i + 2)), __uint_as_float(FPB_U(i + 3)));
        }
        mx = fmaxf(mx, m1);
        // exchange with the other half of the row (double-buffered by block parity)
        xch[(mp & 1) * 256 + hh * 128 + r] = mx;
        mbar_arrive(mx_bar + x);
        if (!FPB_TW(24, mbar_wait_warp_sleep(mx_bar + x, mp & 1, abort))) { ok = false; break; }
        mx = fmaxf(mx, xch[(mp & 1) * 256 + (hh ^ 1) * 128 + r]);
        ++mp;
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
        // P = exp2(s*c - m) as 16-bit pairs over S columns [32*hh, 32*hh + 32) (the S values
        // there, the other half's, were read before the exchange above); one pair in four
        // is evaluated on the FMA pipe (exp2_poly2), the rest by ex2.approx.
        const float neg_m = -m_use;
        float rs = 0.f, rs1 = 0.f;
#pragma unroll
        for (int ch = 0; ch < 2; ++ch) {
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) {
            const int e = ch * 32 + i;
            float x0, x1, p0, p1;
            fma2(x0, x1, __uint_as_float(FPB_U(e)), __uint_as_float(FPB_U(e + 1)), c, c, neg_m, neg_m);
            if (((i >> 1) % kPolyEvery) == kPolyEvery - 1) {
              exp2_poly2(x0, x1, p0, p1);  // masked (-inf) entries give 2^-126 here, negligible
            } else {
              p0 = ex2_approx(x0);
              p1 = ex2_approx(x1);
            }
            add2(rs, rs1, rs, rs1, p0, p1);
            pk[i >> 1] = DT<T>::pack(p0, p1);
          }
          tmem_st16(t_s + hh * 32 + ch * 16, pk);
        }
#undef FPB_U
        const unsigned long long tst = clk();
        pa.add(10, tst - tp3);
        rs += rs1;
        if (__any_sync(0xffffffffu, scale_o != 1.f)) {
          // O_x holds blocks 0..j-1 (PV_x(j-1) completed before S_x(j) did); rescale this
          // thread's 64 columns before PV_x(j) is allowed to start (p_full below)
          pa.add(21, 1);
          uint32_t oa[32], ob[32];
          tmem_ld32(t_o, oa);
          tmem_ld32(t_o + 32, ob);
          tmem_ld_wait();
#pragma unroll
          for (int i = 0; i < 32; ++i) {
            oa[i] = __float_as_uint(__uint_as_float(oa[i]) * scale_o);
            ob[i] = __float_as_uint(__uint_as_float(ob[i]) * scale_o);
          }
          tmem_st32(t_o, oa);
          tmem_st32(t_o + 32, ob);
          pa.add(9, clk() - tst);
        }
        tmem_st_wait();
        pa.add(23, clk() - tst);
        l += rs;
        tc_fence_before();
        mbar_arrive(p_full + x);
        trace(rec, 6, x, j);
      }
      if (!ok) break;
      // ---- epilogue: O / l -> smem (SW128 layout, in the V tile) -> global by TMA
      if (!FPB_TW(6, mbar_wait_warp_sleep(o_full + x, oc & 1, abort))) break;
      ++oc;
      tc_fence_after();
      const unsigned long long te0 = clk();
      if (f.chunk >= 0) {  // a chunk of a split row
        const bool ok2 = split_chunk_epilogue<T>(t_o, f.chunk, m_use, l, r, hh, vr, orow, A.o_ss, A.sp_part,
                                                 A.sp_counters, last_chunk, epi + x, o_empty + x, ep, abort);
        ep += 2;
        if (!ok2) break;
        if constexpr (kPeers) {
          if (*(volatile int*)last_chunk && r < vr) {  // this chunk merged the row: send it on
            const T* src = orow + (int64_t)r * A.o_ss + hh * 64;
            copy_row_to_peers(A, reinterpret_cast<const uint8_t*>(src) - reinterpret_cast<const uint8_t*>(A.out),
                              src, 128);
          }
        }
        if (hh * 128 + r == 0) mbar_arrive(stage_free + x);  // the V tile was not used for staging
        pa.add(11, clk() - te0);
        continue;
      }
      uint32_t oa[32], ob[32];
      tmem_ld32(t_o, oa);
      tmem_ld32(t_o + 32, ob);
      xl[hh * 128 + r] = l;
      tmem_ld_wait();
      tc_fence_before();
      mbar_arrive(o_empty + x);  // O_x may be overwritten by the next item's first PV
      if (!group_sync()) break;
      const float inv = 1.f / (l + xl[(hh ^ 1) * 128 + r]);
      uint8_t* stage = smem + x * 3 * kAttnTile + 2 * kAttnTile;  // V tile: its last PV has completed
#pragma unroll
      for (int q4 = 0; q4 < 8; ++q4) {
        uint32_t pk[4];
#pragma unroll
        for (int i = 0; i < 4; ++i) {
          const int e = q4 * 8 + 2 * i;
          const float v0 = __uint_as_float(e < 32 ? oa[e] : ob[e - 32]) * inv;
          const float v1 = __uint_as_float(e + 1 < 32 ? oa[e + 1] : ob[e - 31]) * inv;
          pk[i] = DT<T>::pack(v0, v1);
        }
        uint8_t* dst = stage + hh * kAttnHalf + r * 128 + ((q4 ^ (r & 7)) << 4);
        *reinterpret_cast<uint4*>(dst) = make_uint4(pk[0], pk[1], pk[2], pk[3]);
      }
      fence_proxy_async_smem();
      if (!group_sync()) break;
      const int et = hh * 128 + r;
      if constexpr (kPeers) {
        // the staged tile to every peer's output, 16 bytes per store, rows r < vr
        const int64_t row0 = reinterpret_cast<const uint8_t*>(orow) - reinterpret_cast<const uint8_t*>(A.out);
        for (int p = 0; p < A.n_peers; ++p) {
          uint8_t* pbase = reinterpret_cast<uint8_t*>(A.peer_out[p]) + row0;
          for (int e = et; e < vr * 16; e += 256) {
            const int rr = e >> 4, cidx = e & 15;
            const uint4 v = *reinterpret_cast<const uint4*>(stage + (cidx >> 3) * kAttnHalf + rr * 128 +
                                                           (((cidx & 7) ^ (rr & 7)) << 4));
            *reinterpret_cast<uint4*>(pbase + ((int64_t)rr * A.o_ss + cidx * 8) * (int64_t)sizeof(T)) = v;
          }
        }
        if (!group_sync()) break;
      }
      if (vr == kBlock) {
        if (et == 0) {
          const int qrow = f.start + f.qb * kBlock;
          const uint64_t pol = l2_policy_evict_first();  // the output is not read again here
          tma_store_4d_hint(&tm_o, stage, 0, hx, qrow, f.bcoord, pol);
          tma_store_4d_hint(&tm_o, stage + kAttnHalf, 64, hx, qrow, f.bcoord, pol);
          tma_store_commit_and_wait_read();
          mbar_arrive(stage_free + x);
        }
      } else {  // a sequence's last, partial block: only its rows may be written
        for (int e = et; e < vr * 16; e += 256) {
          const int rr = e >> 4, cidx = e & 15;
          const uint4 v =
              *reinterpret_cast<const uint4*>(stage + (cidx >> 3) * kAttnHalf + rr * 128 + (((cidx & 7) ^ (rr & 7)) << 4));
          *reinterpret_cast<uint4*>(orow + (int64_t)rr * A.o_ss + cidx * 8) = v;
        }
        if (!group_sync()) break;
        if (et == 0) mbar_arrive(stage_free + x);
      }
      pa.add(11, clk() - te0);
    }
    // the epilogue waits only until its stores have read the staging tile; their global
    // writes must be complete before the thread exits
    tma_store_wait_all();
    if constexpr (kPeers) __threadfence_system();  // peer stores ordered before what follows
  }

  if (threadIdx.x == 0) pa.add(18, clk() - t_kernel0);
  tc_fence_before();
  __syncthreads();
#if FPB_ATTN_PROFILE
  if (A.profile && threadIdx.x < kProfSlots) atomicAdd(&g_attn_prof[threadIdx.x], prof_smem[threadIdx.x]);
  if (tr && threadIdx.x == 0) g_attn_trace_n = *trace_ctr;
#endif
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if (threadIdx.x == 0 && *abort) raise_error(A.P.err, kErrWaitTimeout);
}

}  // namespace fpb
