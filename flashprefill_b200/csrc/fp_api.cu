// Host side of the C ABI declared in include/flashprefill_b200.h: argument validation,
// workspace layout, TMA tensor maps and kernel launches.  Built as one translation unit
// with the kernels (unity build) into libflashprefill_b200.so.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cmath>
#include <cstdarg>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>
#include <string>

#include "../../include/flashprefill_b200.h"
#include "fp_attn.cu"
#include "fp_attn2.cu"
#include "fp_mean.cu"
#include "fp_search.cu"

namespace fpb {
namespace {

thread_local std::string g_last_error;

int fail(int code, const char* fmt, ...) {
  char buf[512];
  va_list ap;
  va_start(ap, fmt);
  vsnprintf(buf, sizeof(buf), fmt, ap);
  va_end(ap);
  g_last_error = buf;
  return code;
}

#define FPB_CHECK_ARG(cond, ...)                       \
  do {                                                 \
    if (!(cond)) return fail(FPB_EINVAL, __VA_ARGS__); \
  } while (0)

#define FPB_CUDA(call)                                                                            \
  do {                                                                                            \
    cudaError_t e_ = (call);                                                                      \
    if (e_ != cudaSuccess) return fail(FPB_ECUDA, "%s failed: %s", #call, cudaGetErrorString(e_)); \
  } while (0)

#define FPB_TRY(x)                 \
  do {                             \
    int rc_ = (x);                 \
    if (rc_ != FPB_OK) return rc_; \
  } while (0)

// ------------------------------------------------------------------ workspace layout
struct Layout {
  int64_t err, cu_tile, mk, cnt, idx, total;
  int tiles, cap;
  // Optional tail (long rows split into chunks, fp_split.cu): used when the caller's workspace
  // reaches total_split; base_total is the required minimum.
  int64_t base_total, sp_head, sp_entries, sp_rowidx, sp_counters, sp_part, total_split;
  int max_chunks, max_split_rows;
};

int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

// Bounds that keep every workspace offset and kernel index in range: at most 2^30 query-block
// rows (tiles) per call, and at most 2^34 list entries (hq * tiles * cap, 64 GiB of lists).
constexpr int64_t kMaxTiles = int64_t(1) << 30;
constexpr int64_t kMaxListEntries = int64_t(1) << 34;

// Rejects sizes whose tile count or list area would leave those bounds.
int check_tiles(int64_t tiles, int64_t cap, int hq) {
  if (tiles >= kMaxTiles || (int64_t)hq * tiles * cap > kMaxListEntries)
    return fail(FPB_EINVAL, "problem too large: %lld query-block rows x %lld blocks x %d heads", (long long)tiles,
                (long long)cap, hq);
  return FPB_OK;
}

// varlen=0: a=batch, b=seqlen; varlen=1: a=nseq, b=total_tokens, c=max_seq_len
Layout make_layout(int varlen, int a, int b, int c, int hq, int hk) {
  Layout L{};
  const int nseq = a;
  if (!varlen) {
    const int nb = (b + kBlock - 1) / kBlock;
    L.tiles = (int)std::min<int64_t>((int64_t)a * nb, kMaxTiles);  // callers reject more (check_tiles)
    L.cap = nb;
  } else {
    // sum ceil(len_i/128) <= ceil(T/128) + nseq
    L.tiles = (int)std::min<int64_t>((int64_t)(b + kBlock - 1) / kBlock + a, kMaxTiles);
    L.cap = (c + kBlock - 1) / kBlock;
    if (L.cap < 1) L.cap = 1;
  }
  int64_t off = 0;
  L.err = off;
  off += 256;
  L.cu_tile = off;
  off = align256(off + 4 * (int64_t)(nseq + 1));
  L.mk = off;
  off = align256(off + (int64_t)L.tiles * hk * kHeadDim * 2);
  L.cnt = off;
  off = align256(off + 4 * (int64_t)hq * L.tiles);
  L.idx = off;
  off = align256(off + 4 * (int64_t)hq * L.tiles * L.cap);
  L.base_total = off;
  // split region: enough chunks for two full-length rows per sequence and head (the last-N
  // band at its default width) plus a quarter more; further long rows stay whole
  const int chunks_per_row = (L.cap + kSplitChunk - 1) / kSplitChunk;
  L.max_chunks = L.cap > kSplitChunk ? (int)std::min<int64_t>(2LL * nseq * hq * chunks_per_row * 5 / 4, 1 << 16) : 0;
  L.max_split_rows = L.max_chunks;
  L.sp_head = off;
  off = align256(off + kPlanHeadBytes);
  L.sp_entries = off;
  off = align256(off + 16 * (int64_t)L.max_chunks);
  L.sp_rowidx = off;
  off = align256(off + 4 * (int64_t)hq * L.tiles);
  L.sp_counters = off;
  off = align256(off + 4 * (int64_t)L.max_split_rows);
  L.sp_part = off;
  off = align256(off + kSplitPartBytes * L.max_chunks);
  L.total_split = L.max_chunks > 0 ? off : L.base_total;
  L.total = L.total_split;  // what callers should allocate
  return L;
}

// ------------------------------------------------------------------ tensor maps
PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 4-D map over (128, heads, rows, batch) 16-bit elements, box (64, 1, 128, 1), 128B swizzle.
// Strides in elements for dims 1..3.  Size-1 dimensions get a harmless stride.
int make_map(CUtensorMap* map, const void* base, int dtype, int64_t heads, int64_t rows, int64_t batch,
             int64_t s_head, int64_t s_row, int64_t s_batch, const char* what) {
  auto enc = get_encode_fn();
  if (!enc) return fail(FPB_ECUDA, "cuTensorMapEncodeTiled is unavailable (driver too old?)");
  if (heads == 1) s_head = 8;
  if (batch == 1) s_batch = s_row * rows + 8;
  const cuuint64_t dims[4] = {(cuuint64_t)kHeadDim, (cuuint64_t)heads, (cuuint64_t)rows, (cuuint64_t)batch};
  const cuuint64_t strides[3] = {(cuuint64_t)s_head * 2, (cuuint64_t)s_row * 2, (cuuint64_t)s_batch * 2};
  const cuuint32_t box[4] = {64, 1, 128, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = enc(map, dtype == FPB_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16, 4,
                   const_cast<void*>(base), dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                   CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                   CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(FPB_ECUDA, "cuTensorMapEncodeTiled(%s) failed with CUresult %d", what, (int)r);
  return FPB_OK;
}

// ------------------------------------------------------------------ argument checks
int check_ptr(const void* p, const char* what) {
  FPB_CHECK_ARG(p != nullptr, "%s is NULL", what);
  FPB_CHECK_ARG((reinterpret_cast<uintptr_t>(p) & 15) == 0, "%s must be 16-byte aligned", what);
  return FPB_OK;
}
int check_strides(const int64_t* st, int n, const char* what) {
  FPB_CHECK_ARG(st != nullptr, "%s strides are NULL", what);
  for (int i = 0; i < n; ++i) {
    FPB_CHECK_ARG(st[i] >= 0 && st[i] % 8 == 0, "%s stride[%d]=%lld must be a non-negative multiple of 8 elements",
                  what, i, (long long)st[i]);
    FPB_CHECK_ARG(st[i] * 2 < (int64_t(1) << 40), "%s stride[%d] too large", what, i);
  }
  return FPB_OK;
}
int check_common(int dtype, int hq, int hk, int head_dim, int block_size) {
  FPB_CHECK_ARG(dtype == FPB_BF16 || dtype == FPB_FP16, "dtype must be FPB_BF16 or FPB_FP16 (got %d)", dtype);
  FPB_CHECK_ARG(head_dim == kHeadDim, "head_dim must be 128 (got %d)", head_dim);
  FPB_CHECK_ARG(block_size == kBlock, "block_size must be 128 (got %d)", block_size);
  FPB_CHECK_ARG(hq >= 1 && hk >= 1 && hq % hk == 0, "num_q_heads (%d) must be a multiple of num_kv_heads (%d)", hq,
                hk);
  return FPB_OK;
}

// Work-item counter of the persistent attention kernel (inside the 256-byte error block).
constexpr int64_t kCounterOffset = 64;         // attention work-item counter
constexpr int64_t kSearchCounterOffset = 128;  // persistent search work-item counter

int sm_count(int* out) {
  int dev = 0;
  FPB_CUDA(cudaGetDevice(&dev));
  static int cache[64] = {};
  if (dev >= 0 && dev < 64 && cache[dev] > 0) {
    *out = cache[dev];
    return FPB_OK;
  }
  int n = 0;
  FPB_CUDA(cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev));
  if (dev >= 0 && dev < 64) cache[dev] = n;
  *out = n;
  return FPB_OK;
}

template <typename KernelT>
int set_smem(KernelT kernel, size_t bytes) {
  FPB_CUDA(cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)bytes));
  return FPB_OK;
}

// ------------------------------------------------------------------ stage launchers
struct Geometry {
  int varlen, nseq, seqlen, total_tokens, max_seq_len, batch;
  int hq, hk, dtype;
  const int32_t* cu_seqlens;
  int qb_lo = 0, qb_hi = -1;  // dense: query blocks [qb_lo, qb_hi) only (qb_hi < 0: all)
  int q_off = 0;              // dense chunked prefill: q/out hold key positions [q_off, seqlen)
};

// Query-block rows of work (search items and attention items per head): dense covers the
// chosen query blocks of every batch entry, varlen the layout's upper bound of blocks.
int work_tiles(const Geometry& g, const Layout& L) {
  if (g.varlen) return L.tiles;
  const int nb = (g.seqlen + kBlock - 1) / kBlock;
  const int hi = g.qb_hi < 0 ? nb : g.qb_hi;
  return g.batch * (hi - g.qb_lo);
}

SeqProblem make_problem(const Geometry& g, const Layout& L, uint8_t* ws) {
  SeqProblem P{};
  P.varlen = g.varlen;
  P.nseq = g.varlen ? g.nseq : g.batch;
  P.seqlen = g.seqlen;
  P.nb_dense = g.varlen ? 0 : (g.seqlen + kBlock - 1) / kBlock;
  P.row_lo = g.varlen ? 0 : g.qb_lo;
  P.nrows = g.varlen ? 0 : (g.qb_hi < 0 ? P.nb_dense : g.qb_hi) - g.qb_lo;
  P.q_off = g.varlen ? 0 : g.q_off;
  P.tiles_ub = L.tiles;
  P.cap = L.cap;
  P.hq = g.hq;
  P.hk = g.hk;
  P.cu_seqlens = g.cu_seqlens;
  P.cu_tile = reinterpret_cast<const int*>(ws + L.cu_tile);
  P.err = reinterpret_cast<uint32_t*>(ws + L.err);
  return P;
}

float score_scale() { return (float)(1.0 / std::sqrt((double)kHeadDim)) * 1.4426950408889634f; }

// q/k strides as {batch, row, head} (varlen: batch stride unused)
int run_search(const Geometry& g, const void* q, const void* k, const int64_t qs[3], const int64_t ks[3], int sink,
               int window, float alpha, int last_n, int min_budget, int mean_model, uint8_t* ws, const Layout& L,
               cudaStream_t stream) {
  FPB_CHECK_ARG(mean_model == 4 || mean_model == 8, "mean_model must be 4 or 8 (got %d)", mean_model);
  FPB_CHECK_ARG(min_budget >= 0, "min_budget must be >= 0");
  const size_t smem = search_smem_bytes(L.cap);
  FPB_CHECK_ARG(smem <= 227 * 1024, "sequence too long for the on-chip block search (%d blocks)", L.cap);
  SeqProblem P = make_problem(g, L, ws);
  FPB_CUDA(cudaMemsetAsync(ws + L.err, 0, 4, stream));
  if (g.varlen) {
    varlen_prep_kernel<<<1, 1024, 0, stream>>>(g.cu_seqlens, g.nseq, g.total_tokens, L.cap,
                                               reinterpret_cast<int*>(ws + L.cu_tile), P.err);
    FPB_CUDA(cudaGetLastError());
  }
  const int rows = g.varlen ? g.total_tokens : g.seqlen;
  const int batch = g.varlen ? 1 : g.batch;
  {
    dim3 grid(L.tiles, g.hk);
    if (g.dtype == FPB_BF16) {
      auto* mk = reinterpret_cast<__nv_bfloat16*>(ws + L.mk);
      auto* kp = reinterpret_cast<const __nv_bfloat16*>(k);
      if (mean_model == 4) block_mean_kernel<__nv_bfloat16, 4><<<grid, 128, 0, stream>>>(kp, ks[0], ks[1], ks[2], mk, P);
      else block_mean_kernel<__nv_bfloat16, 8><<<grid, 256, 0, stream>>>(kp, ks[0], ks[1], ks[2], mk, P);
    } else {
      auto* mk = reinterpret_cast<__half*>(ws + L.mk);
      auto* kp = reinterpret_cast<const __half*>(k);
      if (mean_model == 4) block_mean_kernel<__half, 4><<<grid, 128, 0, stream>>>(kp, ks[0], ks[1], ks[2], mk, P);
      else block_mean_kernel<__half, 8><<<grid, 256, 0, stream>>>(kp, ks[0], ks[1], ks[2], mk, P);
    }
    FPB_CUDA(cudaGetLastError());
  }
  CUtensorMap tm_q, tm_mk;
  FPB_TRY(make_map(&tm_q, q, g.dtype, g.hq, rows - g.q_off, batch, qs[2], qs[1], qs[0], "q"));
  FPB_TRY(make_map(&tm_mk, ws + L.mk, g.dtype, g.hk, L.tiles, 1, kHeadDim, (int64_t)g.hk * kHeadDim, 0, "pooled k"));
  SearchArgs A{};
  A.P = P;
  A.c = score_scale();
  A.alpha = alpha;
  A.cand_off = (min_budget > 0 || !(alpha > 0.f)) ? -INFINITY : std::log2(alpha) - 8.0f;
  A.sink = sink;
  A.window = window;
  A.last_n = last_n;
  A.min_budget = g.varlen ? 0 : min_budget;
  A.normalize = g.varlen ? 0 : 1;
  A.idx = reinterpret_cast<int32_t*>(ws + L.idx);
  A.cnt = reinterpret_cast<int32_t*>(ws + L.cnt);
  const unsigned grid = (unsigned)work_tiles(g, L) * (unsigned)g.hq;
  const size_t psmem = search_p_smem_bytes(L.cap);
  const bool persistent = L.cap <= kSearchMaxCap && psmem <= 227 * 1024 &&
                          std::getenv("FLASHPREFILL_B200_SEARCH_PER_ITEM") == nullptr;
  if (persistent) {
    A.counter = reinterpret_cast<int*>(ws + L.err + kSearchCounterOffset);
    A.total_items = (int)grid;
    FPB_CUDA(cudaMemsetAsync(A.counter, 0, sizeof(int), stream));
    int sms = 0;
    FPB_TRY(sm_count(&sms));
    const unsigned pgrid = (unsigned)std::min<long long>(sms, grid);
    {
      cudaFuncAttributes fa{};
      FPB_CUDA(cudaFuncGetAttributes(&fa, g.dtype == FPB_BF16 ? (const void*)block_search_persistent_kernel<__nv_bfloat16>
                                                               : (const void*)block_search_persistent_kernel<__half>));
      if (fa.numRegs != kSearchPLaunchRegs || fa.maxThreadsPerBlock < kSearchPThreads)
        return fail(FPB_ECUDA,
                    "search kernel compiled with %d registers/thread (%d expected by its register split), "
                    "at most %d threads per block (%d needed), %zu bytes static shared memory",
                    fa.numRegs, kSearchPLaunchRegs, fa.maxThreadsPerBlock, kSearchPThreads, fa.sharedSizeBytes);
    }
    unsigned long long* sprof = nullptr;
#if FPB_SEARCH_PROFILE  // debug build only: per-phase cycle sums (allocates and synchronises)
    if (std::getenv("FLASHPREFILL_B200_SEARCH_PROFILE")) {
      FPB_CUDA(cudaMalloc(&sprof, sizeof(unsigned long long) * kSpSlots));
      FPB_CUDA(cudaMemsetAsync(sprof, 0, sizeof(unsigned long long) * kSpSlots, stream));
    }
#endif
    A.prof = sprof;
    if (g.dtype == FPB_BF16) {
      FPB_TRY(set_smem(block_search_persistent_kernel<__nv_bfloat16>, psmem));
      block_search_persistent_kernel<__nv_bfloat16><<<pgrid, kSearchPThreads, psmem, stream>>>(tm_q, tm_mk, A);
    } else {
      FPB_TRY(set_smem(block_search_persistent_kernel<__half>, psmem));
      block_search_persistent_kernel<__half><<<pgrid, kSearchPThreads, psmem, stream>>>(tm_q, tm_mk, A);
    }
    if (sprof) {
      unsigned long long h[kSpSlots];
      FPB_CUDA(cudaMemcpyAsync(h, sprof, sizeof(h), cudaMemcpyDeviceToHost, stream));
      FPB_CUDA(cudaStreamSynchronize(stream));
      fprintf(stderr, "[fpb search profile] grid=%u\n", pgrid);
      for (int i = 0; i < kSpSlots; ++i) fprintf(stderr, "[fpb search profile] %-22s %llu\n", kSearchProfNames[i], h[i]);
      cudaFree(sprof);
    }
  } else if (g.dtype == FPB_BF16) {
    FPB_TRY(set_smem(block_search_kernel<__nv_bfloat16>, smem));
    block_search_kernel<__nv_bfloat16><<<grid, kSearchThreads, smem, stream>>>(tm_q, tm_mk, A);
  } else {
    FPB_TRY(set_smem(block_search_kernel<__half>, smem));
    block_search_kernel<__half><<<grid, kSearchThreads, smem, stream>>>(tm_q, tm_mk, A);
  }
  FPB_CUDA(cudaGetLastError());
  return FPB_OK;
}

// Head-pair attention kernel (fp_attn2.cu) over the block lists in the workspace; with split,
// the long-row plan runs first in head-pair mode.
int run_attention2(const Geometry& g, const Layout& L, const CUtensorMap& tm_q, const CUtensorMap& tm_k,
                   const CUtensorMap& tm_v, const AttnArgs& A1, uint8_t* ws, bool split, cudaStream_t stream,
                   void* const* out_peers, int n_peers) {
  Attn2Args A{};
  A.P = A1.P;
  A.c = A1.c;
  A.idx = A1.idx;
  A.cnt = A1.cnt;
  A.counter = A1.counter;
  const int group = g.hq / g.hk;
  A.ppg = (group + 1) / 2;
  A.total_items = work_tiles(g, L) * g.hk * A.ppg;
  A.out = A1.out;
  A.o_sb = A1.o_sb;
  A.o_ss = A1.o_ss;
  A.o_sh = A1.o_sh;
  int sms = 0;
  FPB_TRY(sm_count(&sms));
  const unsigned grid = (unsigned)std::max(1, std::min(sms, A.total_items));
  A.split = split && L.max_chunks >= 2;
  if (A.split) {
    SplitArgs S{};
    S.P = A.P;
    S.cnt = A.cnt;
    S.total_items = A.total_items;
    S.ppg = A.ppg;
    S.max_chunks = L.max_chunks / 2;  // two tiles' partials per entry in the same area
    S.pipelines = (int)grid;
    S.entries = reinterpret_cast<SplitEntry*>(ws + L.sp_entries);
    S.head = reinterpret_cast<int*>(ws + L.sp_head);
    S.rowidx = reinterpret_cast<int*>(ws + L.sp_rowidx);
    S.counters = reinterpret_cast<int*>(ws + L.sp_counters);
    FPB_CUDA(cudaMemsetAsync(S.head, 0, kPlanHeadClear, stream));
    split_scan_kernel<<<(unsigned)((A.total_items + kScanThreads - 1) / kScanThreads), kScanThreads, 0, stream>>>(S);
    split_plan_kernel<<<1, kPlanThreads, 0, stream>>>(S);
    FPB_CUDA(cudaGetLastError());
    A.sp_entries = S.entries;
    A.sp_head = S.head;
    A.sp_rowidx = S.rowidx;
    A.sp_counters = S.counters;
    A.sp_part = reinterpret_cast<float*>(ws + L.sp_part);
  }
  A.n_peers = n_peers;
  for (int i = 0; i < n_peers; ++i) A.peer_out[i] = out_peers[i];
  using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, Attn2Args);
  // the peer-writing instance only when there are peers: the plain one is the hot path
  const KernelFn kern =
      g.dtype == FPB_BF16
          ? (n_peers ? sparse_attn2_kernel<__nv_bfloat16, true> : sparse_attn2_kernel<__nv_bfloat16, false>)
          : (n_peers ? sparse_attn2_kernel<__half, true> : sparse_attn2_kernel<__half, false>);
  {
    cudaFuncAttributes fa{};
    FPB_CUDA(cudaFuncGetAttributes(&fa, (const void*)kern));
    if (fa.numRegs != kA2LaunchRegs)
      return fail(FPB_ECUDA, "head-pair attention kernel compiled with %d registers/thread, %d expected by its "
                  "register split", fa.numRegs, kA2LaunchRegs);
  }
  const size_t smem = attn2_smem_bytes();
  FPB_TRY(set_smem(kern, smem));
#if FPB_ATTN_PROFILE
  A.profile = std::getenv("FLASHPREFILL_B200_PROFILE") != nullptr;
  if (A.profile) {
    static const unsigned long long zeros[kA2ProfSlots] = {};
    FPB_CUDA(cudaMemcpyToSymbolAsync(g_attn2_prof, zeros, sizeof(zeros), 0, cudaMemcpyHostToDevice, stream));
  }
  A.trace = std::getenv("FLASHPREFILL_B200_TRACE") != nullptr;
  if (A.trace) {
    static const unsigned int zero = 0;
    FPB_CUDA(cudaMemcpyToSymbolAsync(g_attn2_trace_n, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, stream));
  }
#endif
  kern<<<grid, kA2Threads, smem, stream>>>(tm_q, tm_k, tm_v, A);
  FPB_CUDA(cudaGetLastError());
#if FPB_ATTN_PROFILE
  if (A.profile) {  // debug instrumentation: synchronises and prints per-phase cycle sums
    unsigned long long h[kA2ProfSlots];
    FPB_CUDA(cudaMemcpyFromSymbolAsync(h, g_attn2_prof, sizeof(h), 0, cudaMemcpyDeviceToHost, stream));
    FPB_CUDA(cudaStreamSynchronize(stream));
    static const char* names[kA2ProfSlots] = {
        "sm_wait_s_full", "sm_tmem_ld_S", "sm_max", "sm_exp_pack_st", "sm_rescale", "sm_st_wait_arrive",
        "sm_blocks", "sm_rescales", "sm_wait_o_full", "mma_wait_k_full", "mma_wait_p_full", "mma_wait_v_full",
        "mma_wait_o_empty", "mma_wait_q_full", "mma_union_blocks", "cta_cycles(4 roles)", "mma_wait_item",
        "prod_wait_k_empty", "prod_wait_v_empty", "prod_wait_q_empty", "prod_wait_item_empty", "sm_epilogue",
        "-", "-"};
    fprintf(stderr, "[fpb attn2 profile] grid=%u\n", grid);
    for (int i = 0; i < kA2ProfSlots; ++i) fprintf(stderr, "[fpb attn2 profile] %-24s %llu\n", names[i], h[i]);
  }
  {
    unsigned long long gu[4];
    FPB_CUDA(cudaMemcpyFromSymbolAsync(gu, g_attn2_gaveup, sizeof(gu), 0, cudaMemcpyDeviceToHost, stream));
    FPB_CUDA(cudaStreamSynchronize(stream));
    if (gu[0]) fprintf(stderr, "[fpb attn2] first wait that gave up: block %llu thread %llu slot %llu\n", gu[0] - 1, gu[1], gu[2]);
  }
  if (A.trace) {  // debug: CTA 0's event trace, written to the file the variable names
    unsigned int n = 0;
    FPB_CUDA(cudaMemcpyFromSymbolAsync(&n, g_attn2_trace_n, sizeof(n), 0, cudaMemcpyDeviceToHost, stream));
    FPB_CUDA(cudaStreamSynchronize(stream));
    n = std::min(n, (unsigned)kA2TraceCap);
    std::vector<unsigned long long> buf(2 * (size_t)n + 1);
    FPB_CUDA(cudaMemcpyFromSymbol(buf.data(), g_attn2_trace, 16 * (size_t)n));
    if (FILE* fh = std::fopen(std::getenv("FLASHPREFILL_B200_TRACE"), "wb")) {
      std::fwrite(buf.data(), 16, n, fh);
      std::fclose(fh);
    }
  }
#endif
  return FPB_OK;
}

int run_attention(const Geometry& g, const void* q, const void* k, const void* v, void* o, const int64_t qs[3],
                  const int64_t ks[3], const int64_t vs[3], const int64_t os[3], uint8_t* ws, const Layout& L,
                  size_t ws_bytes, cudaStream_t stream, int64_t listed_lower_bound = 0,
                  void* const* out_peers = nullptr, int n_peers = 0) {
  SeqProblem P = make_problem(g, L, ws);
  const int rows = g.varlen ? g.total_tokens : g.seqlen;
  const int batch = g.varlen ? 1 : g.batch;
  CUtensorMap tm_q, tm_k, tm_v, tm_o;
  FPB_TRY(make_map(&tm_q, q, g.dtype, g.hq, rows - g.q_off, batch, qs[2], qs[1], qs[0], "q"));
  FPB_TRY(make_map(&tm_k, k, g.dtype, g.hk, rows, batch, ks[2], ks[1], ks[0], "k"));
  FPB_TRY(make_map(&tm_v, v, g.dtype, g.hk, rows, batch, vs[2], vs[1], vs[0], "v"));
  FPB_TRY(make_map(&tm_o, o, g.dtype, g.hq, rows - g.q_off, batch, os[2], os[1], os[0], "out"));
  AttnArgs A{};
  A.P = P;
  A.c = score_scale();
  A.total_items = work_tiles(g, L) * g.hq;
  A.counter = reinterpret_cast<int*>(ws + L.err + kCounterOffset);
  FPB_CUDA(cudaMemsetAsync(A.counter, 0, sizeof(int), stream));
  A.idx = reinterpret_cast<const int32_t*>(ws + L.idx);
  A.cnt = reinterpret_cast<const int32_t*>(ws + L.cnt);
  A.out = o;
  A.o_sb = os[0];
  A.o_ss = os[1];
  A.o_sh = os[2];
  int sms = 0;
  FPB_TRY(sm_count(&sms));
  const unsigned grid = (unsigned)std::min(sms, A.total_items);
  // long rows as parallel chunks when the workspace holds the split area
  A.split = L.max_chunks > 0 && (int64_t)ws_bytes >= L.total_split && std::getenv("FLASHPREFILL_B200_NO_SPLIT") == nullptr;
  // No row can pass the plan's threshold if even the longest possible row is within it for
  // the fewest blocks the lists can hold: then the plan is not run at all.
  if (A.split && listed_lower_bound > 0 &&
      (int64_t)std::min(L.cap, ((g.varlen ? g.max_seq_len : g.seqlen) + kBlock - 1) / kBlock) * kSplitThrDen * 2 * (int64_t)grid <=
          listed_lower_bound * kSplitThrNum)
    A.split = 0;
  // the head-pair kernel serves every call without a split plan or peer outputs
  // the head-pair kernel unless the per-head kernel is asked for (FLASHPREFILL_B200_ATTN=v1)
  const char* which = std::getenv("FLASHPREFILL_B200_ATTN");
  const bool v2 = which ? std::strcmp(which, "v1") != 0 : true;
  if (v2) return run_attention2(g, L, tm_q, tm_k, tm_v, A, ws, A.split, stream, out_peers, n_peers);
  FPB_CHECK_ARG(g.q_off == 0, "chunked prefill needs the head-pair attention kernel (unset FLASHPREFILL_B200_ATTN)");
  if (A.split) {
    SplitArgs S{};
    S.P = P;
    S.cnt = A.cnt;
    S.total_items = A.total_items;
    S.max_chunks = L.max_chunks;
    S.pipelines = 2 * (int)grid;
    S.entries = reinterpret_cast<SplitEntry*>(ws + L.sp_entries);
    S.head = reinterpret_cast<int*>(ws + L.sp_head);
    S.rowidx = reinterpret_cast<int*>(ws + L.sp_rowidx);
    S.counters = reinterpret_cast<int*>(ws + L.sp_counters);
    FPB_CUDA(cudaMemsetAsync(S.head, 0, kPlanHeadClear, stream));
    split_scan_kernel<<<(unsigned)((A.total_items + kScanThreads - 1) / kScanThreads), kScanThreads, 0, stream>>>(S);
    split_plan_kernel<<<1, kPlanThreads, 0, stream>>>(S);
    FPB_CUDA(cudaGetLastError());
    A.sp_entries = S.entries;
    A.sp_head = S.head;
    A.sp_rowidx = S.rowidx;
    A.sp_counters = S.counters;
    A.sp_part = reinterpret_cast<float*>(ws + L.sp_part);
  }
  A.alt_issue = std::getenv("FLASHPREFILL_B200_ISSUE") && std::strcmp(std::getenv("FLASHPREFILL_B200_ISSUE"), "alt") == 0;
#if FPB_ATTN_PROFILE
  A.profile = std::getenv("FLASHPREFILL_B200_PROFILE") != nullptr;
  A.trace = std::getenv("FLASHPREFILL_B200_TRACE") != nullptr;
  if (A.trace) {
    static const unsigned int zero = 0;
    FPB_CUDA(cudaMemcpyToSymbolAsync(g_attn_trace_n, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, stream));
  }
  if (A.profile) {
    static const unsigned long long zeros[kProfSlots] = {};
    FPB_CUDA(cudaMemcpyToSymbolAsync(g_attn_prof, zeros, sizeof(zeros), 0, cudaMemcpyHostToDevice, stream));
  }
#else
  A.profile = 0;
  A.trace = 0;
#endif
  A.n_peers = n_peers;
  for (int i = 0; i < n_peers; ++i) A.peer_out[i] = out_peers[i];
  // the peer-writing instance only when there are peers: the plain one is the hot path
  using KernelFn = void (*)(CUtensorMap, CUtensorMap, CUtensorMap, CUtensorMap, AttnArgs);
  const KernelFn kern =
      g.dtype == FPB_BF16 ? (n_peers ? sparse_attn_kernel<__nv_bfloat16, true> : sparse_attn_kernel<__nv_bfloat16, false>)
                          : (n_peers ? sparse_attn_kernel<__half, true> : sparse_attn_kernel<__half, false>);
  {
    cudaFuncAttributes fa{};
    FPB_CUDA(cudaFuncGetAttributes(&fa, (const void*)kern));
    if (fa.numRegs != kAttnLaunchRegs)
      return fail(FPB_ECUDA, "attention kernel compiled with %d registers/thread, %d expected by its register split",
                  fa.numRegs, kAttnLaunchRegs);
  }
  const size_t smem = attn_smem_bytes();
  FPB_TRY(set_smem(kern, smem));
  kern<<<grid, kAttnThreads, smem, stream>>>(tm_q, tm_k, tm_v, tm_o, A);
  FPB_CUDA(cudaGetLastError());
#if FPB_ATTN_PROFILE
  if (A.trace) {  // debug: CTA 0's event trace, written to the file the variable names
    unsigned int n = 0;
    FPB_CUDA(cudaMemcpyFromSymbolAsync(&n, g_attn_trace_n, sizeof(n), 0, cudaMemcpyDeviceToHost, stream));
    FPB_CUDA(cudaStreamSynchronize(stream));
    n = std::min(n, (unsigned)kTraceCap);
    std::vector<unsigned long long> buf(2 * (size_t)n + 1);
    FPB_CUDA(cudaMemcpyFromSymbol(buf.data(), g_attn_trace, 16 * (size_t)n));
    if (FILE* fh = std::fopen(std::getenv("FLASHPREFILL_B200_TRACE"), "wb")) {
      std::fwrite(buf.data(), 16, n, fh);
      std::fclose(fh);
    }
  }
  if (A.profile) {  // debug instrumentation: synchronises and prints per-phase cycle sums
    unsigned long long h[kProfSlots];
    FPB_CUDA(cudaMemcpyFromSymbolAsync(h, g_attn_prof, sizeof(h), 0, cudaMemcpyDeviceToHost, stream));
    FPB_CUDA(cudaStreamSynchronize(stream));
    static const char* names[kProfSlots] = {
        "mma_blk_p_full", "mma_blk_k_full", "mma_blk_v_full", "mma_blk_q_or_o", "mma_wait_item",
        "sm_wait_s_full", "sm_wait_o_full", "sm_wait_item", "sm_pass1", "sm_rescale", "sm_pass2", "sm_epilogue",
        "sm_epi_sync", "prod_wait_k_empty", "prod_wait_q_empty", "prod_wait_item_empty", "prod_wait_v_empty", "mma_pipe_done",
        "cta_total_cycles", "items", "softmax_block_iters", "rescales", "sm_tmem_ld_S", "sm_tmem_st_P_wait", "sm_wait_rowmax"};
    fprintf(stderr, "[fpb profile] grid=%u\n", grid);
    for (int i = 0; i < kProfSlots; ++i) fprintf(stderr, "[fpb profile] %-26s %llu\n", names[i], h[i]);
  }
#endif
  return FPB_OK;
}

int check_dense(const void* q, const void* k, int dtype, int batch, int seqlen, int hq, int hk, int head_dim,
                const int64_t* qs, const int64_t* ks, int block_size) {
  FPB_TRY(check_common(dtype, hq, hk, head_dim, block_size));
  FPB_CHECK_ARG(batch >= 1 && seqlen >= 1, "batch (%d) and seqlen (%d) must be >= 1", batch, seqlen);
  FPB_CHECK_ARG((int64_t)seqlen + kBlock < (int64_t(1) << 31), "seqlen too large");
  {
    const int64_t nb = ((int64_t)seqlen + kBlock - 1) / kBlock;
    FPB_TRY(check_tiles((int64_t)batch * nb, nb, hq));
  }
  FPB_TRY(check_ptr(q, "q"));
  FPB_TRY(check_ptr(k, "k"));
  FPB_TRY(check_strides(qs, 3, "q"));
  FPB_TRY(check_strides(ks, 3, "k"));
  return FPB_OK;
}

int check_dense_vo(const void* v, const void* o, const int64_t* vs, const int64_t* os) {
  FPB_TRY(check_ptr(v, "v"));
  FPB_TRY(check_ptr(o, "out"));
  FPB_TRY(check_strides(vs, 3, "v"));
  FPB_TRY(check_strides(os, 3, "out"));
  return FPB_OK;
}

int check_varlen(const void* q, const void* k, int dtype, const int32_t* cu, int nseq, int total, int max_len, int hq,
                 int hk, int head_dim, const int64_t* qs, const int64_t* ks, int block_size) {
  FPB_TRY(check_common(dtype, hq, hk, head_dim, block_size));
  FPB_CHECK_ARG(nseq >= 1, "cu_seqlens must hold at least 2 entries");
  FPB_CHECK_ARG(total >= 0 && max_len >= 0, "total_tokens and max_seq_len must be >= 0");
  FPB_CHECK_ARG((int64_t)total + kBlock < (int64_t(1) << 31) && (int64_t)max_len + kBlock < (int64_t(1) << 31),
                "total_tokens or max_seq_len too large");
  FPB_TRY(check_tiles(((int64_t)total + kBlock - 1) / kBlock + nseq, std::max<int64_t>(1, ((int64_t)max_len + kBlock - 1) / kBlock), hq));
  FPB_CHECK_ARG(cu != nullptr && (reinterpret_cast<uintptr_t>(cu) & 3) == 0,
                "cu_seqlens must be an aligned int32 pointer");
  FPB_TRY(check_ptr(q, "q"));
  FPB_TRY(check_ptr(k, "k"));
  FPB_TRY(check_strides(qs, 2, "q"));
  FPB_TRY(check_strides(ks, 2, "k"));
  return FPB_OK;
}

int check_varlen_vo(const void* v, const void* o, const int64_t* vs, const int64_t* os) {
  FPB_TRY(check_ptr(v, "v"));
  FPB_TRY(check_ptr(o, "o"));
  FPB_TRY(check_strides(vs, 2, "v"));
  FPB_TRY(check_strides(os, 2, "o"));
  return FPB_OK;
}

int check_ws(const void* ws, size_t bytes, const Layout& L) {
  FPB_CHECK_ARG(ws != nullptr && (reinterpret_cast<uintptr_t>(ws) & 255) == 0,
                "workspace must be a 256-byte aligned device pointer");
  FPB_CHECK_ARG((int64_t)bytes >= L.base_total, "workspace too small: %zu bytes given, %lld needed", bytes,
                (long long)L.base_total);
  return FPB_OK;
}

void s3(const int64_t* s2, int64_t out[3]) {  // varlen {token, head} -> {batch, row, head}
  out[0] = 0;
  out[1] = s2[0];
  out[2] = s2[1];
}

}  // namespace
}  // namespace fpb

using namespace fpb;

extern "C" {

int fpb_version(void) { return 100; }

const char* fpb_last_error(void) { return g_last_error.c_str(); }

size_t fpb_dense_workspace_bytes(int batch, int seqlen, int hq, int hk, int head_dim) {
  (void)head_dim;
  if (batch < 1 || seqlen < 1 || hq < 1 || hk < 1) return 0;
  return (size_t)make_layout(0, batch, seqlen, 0, hq, hk).total;
}

size_t fpb_varlen_workspace_bytes(int total_tokens, int nseq, int max_seq_len, int hq, int hk, int head_dim) {
  (void)head_dim;
  if (nseq < 1 || total_tokens < 0 || hq < 1 || hk < 1) return 0;
  return (size_t)make_layout(1, nseq, total_tokens, max_seq_len, hq, hk).total;
}

int fpb_workspace_layout(int varlen, int a, int b, int c, int hq, int hk, int head_dim, int64_t* out8) {
  (void)head_dim;
  FPB_CHECK_ARG(out8 != nullptr, "out8 is NULL");
  FPB_CHECK_ARG(a >= 1 && b >= 0 && hq >= 1 && hk >= 1, "invalid sizes");
  const Layout L = make_layout(varlen, a, b, c, hq, hk);
  out8[0] = L.err;
  out8[1] = L.cu_tile;
  out8[2] = L.mk;
  out8[3] = L.cnt;
  out8[4] = L.idx;
  out8[5] = L.total;
  out8[6] = L.tiles;
  out8[7] = L.cap;
  return FPB_OK;
}

int fpb_search_dense(const void* q, const void* k, int dtype, int batch, int seqlen, int hq, int hk, int head_dim,
                     const int64_t* q_strides, const int64_t* k_strides, int block_size, int attention_sink,
                     int window_size, float alpha, int last_n_block_full, int min_budget, int mean_model,
                     void* workspace, size_t workspace_bytes, void* stream) {
  FPB_TRY(check_dense(q, k, dtype, batch, seqlen, hq, hk, head_dim, q_strides, k_strides, block_size));
  const Layout L = make_layout(0, batch, seqlen, 0, hq, hk);
  FPB_TRY(check_ws(workspace, workspace_bytes, L));
  Geometry g{0, batch, seqlen, 0, 0, batch, hq, hk, dtype, nullptr};
  return run_search(g, q, k, q_strides, k_strides, attention_sink, window_size, alpha, last_n_block_full, min_budget,
                    mean_model, static_cast<uint8_t*>(workspace), L, static_cast<cudaStream_t>(stream));
}

int fpb_search_varlen(const void* q, const void* k, int dtype, const int32_t* cu_seqlens, int nseq, int total_tokens,
                      int max_seq_len, int hq, int hk, int head_dim, const int64_t* q_strides,
                      const int64_t* k_strides, int block_size, int attention_sink, int window_size, float alpha,
                      int last_n_block, int mean_model, void* workspace, size_t workspace_bytes, void* stream) {
  FPB_TRY(check_varlen(q, k, dtype, cu_seqlens, nseq, total_tokens, max_seq_len, hq, hk, head_dim, q_strides,
                       k_strides, block_size));
  const Layout L = make_layout(1, nseq, total_tokens, max_seq_len, hq, hk);
  FPB_TRY(check_ws(workspace, workspace_bytes, L));
  if (total_tokens == 0) return FPB_OK;
  Geometry g{1, nseq, 0, total_tokens, max_seq_len, 1, hq, hk, dtype, cu_seqlens};
  int64_t qs[3], ks[3];
  s3(q_strides, qs);
  s3(k_strides, ks);
  return run_search(g, q, k, qs, ks, attention_sink, window_size, alpha, last_n_block, 0, mean_model,
                    static_cast<uint8_t*>(workspace), L, static_cast<cudaStream_t>(stream));
}

int fpb_attention_dense(const void* q, const void* k, const void* v, void* out, int dtype, int batch, int seqlen,
                        int hq, int hk, int head_dim, const int64_t* q_strides, const int64_t* k_strides,
                        const int64_t* v_strides, const int64_t* o_strides, int block_size, void* workspace,
                        size_t workspace_bytes, void* stream) {
  FPB_TRY(check_dense(q, k, dtype, batch, seqlen, hq, hk, head_dim, q_strides, k_strides, block_size));
  FPB_TRY(check_dense_vo(v, out, v_strides, o_strides));
  const Layout L = make_layout(0, batch, seqlen, 0, hq, hk);
  FPB_TRY(check_ws(workspace, workspace_bytes, L));
  Geometry g{0, batch, seqlen, 0, 0, batch, hq, hk, dtype, nullptr};
  return run_attention(g, q, k, v, out, q_strides, k_strides, v_strides, o_strides, static_cast<uint8_t*>(workspace),
                       L, workspace_bytes, static_cast<cudaStream_t>(stream));
}

int fpb_attention_varlen(const void* q, const void* k, const void* v, void* o, int dtype, const int32_t* cu_seqlens,
                         int nseq, int total_tokens, int max_seq_len, int hq, int hk, int head_dim,
                         const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                         const int64_t* o_strides, int block_size, void* workspace, size_t workspace_bytes,
                         void* stream) {
  FPB_TRY(check_varlen(q, k, dtype, cu_seqlens, nseq, total_tokens, max_seq_len, hq, hk, head_dim, q_strides,
                       k_strides, block_size));
  FPB_TRY(check_varlen_vo(v, o, v_strides, o_strides));
  const Layout L = make_layout(1, nseq, total_tokens, max_seq_len, hq, hk);
  FPB_TRY(check_ws(workspace, workspace_bytes, L));
  if (total_tokens == 0) return FPB_OK;
  Geometry g{1, nseq, 0, total_tokens, max_seq_len, 1, hq, hk, dtype, cu_seqlens};
  int64_t qs[3], ks[3], vs[3], os[3];
  s3(q_strides, qs);
  s3(k_strides, ks);
  s3(v_strides, vs);
  s3(o_strides, os);
  return run_attention(g, q, k, v, o, qs, ks, vs, os, static_cast<uint8_t*>(workspace), L, workspace_bytes,
                       static_cast<cudaStream_t>(stream));
}

// Fewest listed blocks a dense search can return: its lists hold at least the structural
// blocks of every row (sinks, the local window, and whole rows for the last-N query blocks).
int64_t dense_listed_lower_bound(int batch, int seqlen, int hq, int sink, int window, int last_n, int qb_lo = 0,
                                 int qb_hi = -1) {
  const int64_t nb = (seqlen + kBlock - 1) / kBlock;
  int64_t per_head = 0;
  for (int64_t qb = qb_lo; qb < (qb_hi < 0 ? nb : qb_hi); ++qb)
    if (qb >= nb - last_n) {
      per_head += qb + 1;
    } else {  // |[0, sink) U (qb - window, qb]| within [0, qb]
      const int64_t s_end = std::min<int64_t>(std::max(sink, 0), qb + 1), w_lo = std::max<int64_t>(0, qb - window + 1);
      const int64_t w_n = window > 0 ? qb + 1 - w_lo : 0;
      per_head += s_end + w_n - (window > 0 ? std::max<int64_t>(0, s_end - w_lo) : 0);
    }
  return per_head * hq * batch;
}

int fpb_prefill_dense(const void* q, const void* k, const void* v, void* out, int dtype, int batch, int seqlen,
                      int hq, int hk, int head_dim, const int64_t* q_strides, const int64_t* k_strides,
                      const int64_t* v_strides, const int64_t* o_strides, int block_size, int attention_sink,
                      int window_size, float alpha, int last_n_block_full, int min_budget, int mean_model,
                      void* workspace, size_t workspace_bytes, void* stream) {
  FPB_TRY(check_dense(q, k, dtype, batch, seqlen, hq, hk, head_dim, q_strides, k_strides, block_size));
  FPB_TRY(check_dense_vo(v, out, v_strides, o_strides));
  const Layout L = make_layout(0, batch, seqlen, 0, hq, hk);
  FPB_TRY(check_ws(workspace, workspace_bytes, L));
  Geometry g{0, batch, seqlen, 0, 0, batch, hq, hk, dtype, nullptr};
  auto* ws = static_cast<uint8_t*>(workspace);
  auto st = static_cast<cudaStream_t>(stream);
  FPB_TRY(run_search(g, q, k, q_strides, k_strides, attention_sink, window_size, alpha, last_n_block_full, min_budget,
                     mean_model, ws, L, st));
  return run_attention(g, q, k, v, out, q_strides, k_strides, v_strides, o_strides, ws, L, workspace_bytes, st,
                       dense_listed_lower_bound(batch, seqlen, hq, attention_sink, window_size, last_n_block_full));
}

int fpb_prefill_dense_rows(const void* q, const void* k, const void* v, void* out, int dtype, int batch,
                           int seqlen, int hq, int hk, int head_dim, const int64_t* q_strides,
                           const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                           int block_size, int attention_sink, int window_size, float alpha, int last_n_block_full,
                           int min_budget, int mean_model, int q_block_begin, int q_block_end, void* workspace,
                           size_t workspace_bytes, void* stream) {
  FPB_TRY(check_dense(q, k, dtype, batch, seqlen, hq, hk, head_dim, q_strides, k_strides, block_size));
  FPB_TRY(check_dense_vo(v, out, v_strides, o_strides));
  const int nb = (seqlen + kBlock - 1) / kBlock;
  FPB_CHECK_ARG(0 <= q_block_begin && q_block_begin < q_block_end && q_block_end <= nb,
                "query-block range [%d, %d) must be non-empty and within [0, %d)", q_block_begin, q_block_end, nb);
  const Layout L = make_layout(0, batch, seqlen, 0, hq, hk);
  FPB_TRY(check_ws(workspace, workspace_bytes, L));
  Geometry g{0, batch, seqlen, 0, 0, batch, hq, hk, dtype, nullptr, q_block_begin, q_block_end};
  auto* ws = static_cast<uint8_t*>(workspace);
  auto st = static_cast<cudaStream_t>(stream);
  FPB_TRY(run_search(g, q, k, q_strides, k_strides, attention_sink, window_size, alpha, last_n_block_full, min_budget,
                     mean_model, ws, L, st));
  return run_attention(g, q, k, v, out, q_strides, k_strides, v_strides, o_strides, ws, L, workspace_bytes, st,
                       dense_listed_lower_bound(batch, seqlen, hq, attention_sink, window_size, last_n_block_full,
                                                q_block_begin, q_block_end));
}

int fpb_prefill_dense_chunk(const void* q, const void* k, const void* v, void* out, int dtype, int batch, int q_len,
                            int kv_len, int hq, int hk, int head_dim, const int64_t* q_strides,
                            const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                            int block_size, int attention_sink, int window_size, float alpha, int last_n_block_full,
                            int min_budget, int mean_model, void* workspace, size_t workspace_bytes, void* stream) {
  FPB_TRY(check_dense(q, k, dtype, batch, kv_len, hq, hk, head_dim, q_strides, k_strides, block_size));
  FPB_TRY(check_dense_vo(v, out, v_strides, o_strides));
  FPB_CHECK_ARG(q_len >= 1 && q_len <= kv_len, "q_len (%d) must be in [1, kv_len = %d]", q_len, kv_len);
  const Layout L = make_layout(0, batch, kv_len, 0, hq, hk);
  FPB_TRY(check_ws(workspace, workspace_bytes, L));
  const int q_off = kv_len - q_len;
  const int nb = (kv_len + kBlock - 1) / kBlock;
  Geometry g{0, batch, kv_len, 0, 0, batch, hq, hk, dtype, nullptr, q_off / kBlock, nb, q_off};
  auto* ws = static_cast<uint8_t*>(workspace);
  auto st = static_cast<cudaStream_t>(stream);
  FPB_TRY(run_search(g, q, k, q_strides, k_strides, attention_sink, window_size, alpha, last_n_block_full, min_budget,
                     mean_model, ws, L, st));
  return run_attention(g, q, k, v, out, q_strides, k_strides, v_strides, o_strides, ws, L, workspace_bytes, st,
                       dense_listed_lower_bound(batch, kv_len, hq, attention_sink, window_size, last_n_block_full,
                                                q_off / kBlock, nb));
}

int fpb_prefill_dense_peers(const void* q, const void* k, const void* v, void* out, int dtype, int batch, int seqlen,
                            int hq, int hk, int head_dim, const int64_t* q_strides, const int64_t* k_strides,
                            const int64_t* v_strides, const int64_t* o_strides, int block_size, int attention_sink,
                            int window_size, float alpha, int last_n_block_full, int min_budget, int mean_model,
                            void* workspace, size_t workspace_bytes, void* const* out_peers, int n_peers,
                            void* stream) {
  FPB_CHECK_ARG(n_peers >= 0 && n_peers <= kMaxOutPeers, "n_peers (%d) must be in [0, %d]", n_peers, kMaxOutPeers);
  FPB_CHECK_ARG(n_peers == 0 || out_peers != nullptr, "out_peers is NULL");
  for (int i = 0; i < n_peers; ++i)
    FPB_CHECK_ARG(out_peers[i] != nullptr && reinterpret_cast<uintptr_t>(out_peers[i]) % 16 == 0,
                  "out_peers[%d] must be a 16-byte aligned device pointer", i);
  FPB_TRY(check_dense(q, k, dtype, batch, seqlen, hq, hk, head_dim, q_strides, k_strides, block_size));
  FPB_TRY(check_dense_vo(v, out, v_strides, o_strides));
  const Layout L = make_layout(0, batch, seqlen, 0, hq, hk);
  FPB_TRY(check_ws(workspace, workspace_bytes, L));
  Geometry g{0, batch, seqlen, 0, 0, batch, hq, hk, dtype, nullptr};
  auto* ws = static_cast<uint8_t*>(workspace);
  auto st = static_cast<cudaStream_t>(stream);
  FPB_TRY(run_search(g, q, k, q_strides, k_strides, attention_sink, window_size, alpha, last_n_block_full, min_budget,
                     mean_model, ws, L, st));
  return run_attention(g, q, k, v, out, q_strides, k_strides, v_strides, o_strides, ws, L, workspace_bytes, st,
                       dense_listed_lower_bound(batch, seqlen, hq, attention_sink, window_size, last_n_block_full),
                       out_peers, n_peers);
}

int fpb_prefill_varlen(const void* q, const void* k, const void* v, void* o, int dtype, const int32_t* cu_seqlens,
                       int nseq, int total_tokens, int max_seq_len, int hq, int hk, int head_dim,
                       const int64_t* q_strides, const int64_t* k_strides, const int64_t* v_strides,
                       const int64_t* o_strides, int block_size, int attention_sink, int window_size, float alpha,
                       int last_n_block, int mean_model, void* workspace, size_t workspace_bytes, void* stream) {
  FPB_TRY(check_varlen(q, k, dtype, cu_seqlens, nseq, total_tokens, max_seq_len, hq, hk, head_dim, q_strides,
                       k_strides, block_size));
  FPB_TRY(check_varlen_vo(v, o, v_strides, o_strides));
  const Layout L = make_layout(1, nseq, total_tokens, max_seq_len, hq, hk);
  FPB_TRY(check_ws(workspace, workspace_bytes, L));
  if (total_tokens == 0) return FPB_OK;
  Geometry g{1, nseq, 0, total_tokens, max_seq_len, 1, hq, hk, dtype, cu_seqlens};
  int64_t qs[3], ks[3], vs[3], os[3];
  s3(q_strides, qs);
  s3(k_strides, ks);
  s3(v_strides, vs);
  s3(o_strides, os);
  auto* ws = static_cast<uint8_t*>(workspace);
  auto st = static_cast<cudaStream_t>(stream);
  FPB_TRY(run_search(g, q, k, qs, ks, attention_sink, window_size, alpha, last_n_block, 0, mean_model, ws, L, st));
  return run_attention(g, q, k, v, o, qs, ks, vs, os, ws, L, workspace_bytes, st);
}

int fpb_test_set_fault(int withhold_first_load, unsigned long long wait_limit_ns) {
  FPB_CHECK_ARG(wait_limit_ns >= 1000000ull && wait_limit_ns <= kWaitLimitNs,
                "wait_limit_ns must be in [1 ms, 1 s]");
  const int w = withhold_first_load ? 1 : 0;
  const uint64_t lim = wait_limit_ns;
  FPB_CUDA(cudaMemcpyToSymbol(g_test_withhold, &w, sizeof(w)));
  FPB_CUDA(cudaMemcpyToSymbol(g_wait_limit_ns, &lim, sizeof(lim)));
  return FPB_OK;
}

int fpb_read_device_error(const void* workspace, uint32_t* flags, void* stream) {
  FPB_CHECK_ARG(workspace != nullptr && flags != nullptr, "NULL argument");
  auto st = static_cast<cudaStream_t>(stream);
  uint32_t h = 0;
  FPB_CUDA(cudaMemcpyAsync(&h, workspace, 4, cudaMemcpyDeviceToHost, st));
  FPB_CUDA(cudaStreamSynchronize(st));
  *flags = h;
  if (h) return fail(FPB_EDEVICE, "device error bits 0x%x", h);
  return FPB_OK;
}

}  // extern "C"

#include "fp_noalloc.cu"
