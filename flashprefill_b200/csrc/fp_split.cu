// Long rows of the block-sparse attention split into chunks.
//
// The attention processes one (query block, head) row per pipeline.  A row whose block list
// is long -- the last-N rows select every causal block (ops/flashprefill_native_forward.py:
// 347-385, "qb >= NB - last_n"), 1,024 blocks at 128K tokens -- would then take as long as
// all the other work together and set the kernel's duration on its own.  Such rows are cut
// into chunks of kSplitChunk listed blocks.  Each chunk is a separate work item; its
// pipeline writes the unnormalised O, the running max m and the row sum l of its chunk to
// workspace scratch, and the chunk that finishes its row last merges the partials:
//   O = sum_c O_c 2^(m_c - M) / sum_c l_c 2^(m_c - M),  M = max_c m_c,
// the same online-softmax algebra the reference applies block by block (native:317-333).
//
// The plan runs between the search and the attention in two launches: split_scan_kernel sums
// the listed blocks of all rows and collects the rows longer than one chunk; split_plan_kernel
// (one CTA) sets the split threshold and gives each candidate over it its chunk entries by a
// block-wide exclusive scan, within the workspace's chunk budget (rows beyond it stay whole).
// A row is split only if it is longer than 1.2x the listed blocks per attention pipeline:
// shorter rows are absorbed by the heavy-first order, and splitting costs Q reloads and
// partial-result traffic (at 128K tokens with all 32 heads on one GPU, rows of 1.08x the
// average ran 3% slower split; at 256K, rows of 1.26x ran 10% faster split).  The merge adds
// the chunks of a row in chunk order, so the output does not depend on where the plan put
// their entries.
#pragma once
#include "fp_common.cuh"

namespace fpb {

constexpr int kSplitChunk = 64;  // listed key blocks per chunk
// per chunk: O [128][128] f32, m [128] f32, l [2 halves][128] f32
constexpr int64_t kSplitPartBytes = 128 * 128 * 4 + 128 * 4 + 2 * 128 * 4;
constexpr int kPlanThreads = 1024;
// split threshold: kSplitThrNum / kSplitThrDen x the listed blocks per attention pipeline
constexpr int kSplitThrNum = 6, kSplitThrDen = 5;
// The attention carries a chunk as one int: entry (17 bits) | chunk (7) << 17 | nchunks (7) << 24,
// so entries stay below 2^17 and rows of more than 127 chunks (8,128 blocks) stay whole.
constexpr int kSplitMaxEntries = 1 << 17, kSplitMaxRowChunks = 127;
__host__ __device__ inline int split_code(int entry, int chunk, int nchunks) {
  return entry | (chunk << 17) | (nchunks << 24);
}

struct SplitEntry {
  int item;     // attention work item (tile * hq + head)
  int chunk;    // chunk index within the row
  int nchunks;  // chunks of the row
  int srow;     // split-row index (completion counter)
};

// Plan header at the start of the split region (ints): [0] chunk entries used, [1] rows split,
// [2] long rows left whole, [3] split threshold (listed blocks), [4] candidates found,
// [6..7] listed blocks in total (u64).  The host zeroes its first kPlanHeadClear bytes.
// Candidate rows (int4: item, row, listed blocks, -) follow at byte kPlanCandOffset.
constexpr int kPlanHeadClear = 32, kPlanCandOffset = 256;
constexpr int kPlanMaxRows = 2048;  // rows over one chunk a plan holds; further long rows stay whole
constexpr int64_t kPlanHeadBytes = kPlanCandOffset + 16 * (int64_t)kPlanMaxRows;

struct SplitArgs {
  SeqProblem P;
  const int32_t* cnt;  // [hq][tiles_ub]
  int total_items;     // tiles_ub * hq (head items), or tiles * hk * ppg (head-pair items)
  int ppg;             // > 0: items are head pairs (ceil(G/2) per KV head) of the head-pair kernel
  int max_chunks;
  int pipelines;       // attention pipelines (2 per CTA)
  SplitEntry* entries;
  int* head;           // plan header (above)
  int* rowidx;         // [hq][tiles_ub]: split-row index or -1, written for candidate rows only
  int* counters;       // [max_chunks]: chunks finished, indexed by the row's first entry (head
                       // pairs: two counters per entry, [2 * entry + tile])
};

// Pass 1, over all rows (one item per thread): listed blocks in total, and the rows longer
// than one chunk as candidates.
constexpr int kScanThreads = 256;
__global__ void __launch_bounds__(kScanThreads) split_scan_kernel(const SplitArgs A) {
  const int id = blockIdx.x * kScanThreads + threadIdx.x;
  int n = 0, row = -1;
  if (id < A.total_items && A.ppg == 0) {
    const int tile = id / A.P.hq, h = id - tile * A.P.hq;
    SeqInfo s;
    int qb;
    if (decode_item(A.P, tile, s, qb)) {
      row = h * A.P.tiles_ub + s.tile_base + qb;
      n = max(0, min(__ldg(A.cnt + row), qb + 1));
    }
  } else if (id < A.total_items) {  // a head pair: the longer of its two lists
    const int group = A.P.hq / A.P.hk, npairs = A.P.hk * A.ppg;
    const int tile = id / npairs, pr = id - tile * npairs;
    const int hk = pr / A.ppg, ip = pr - hk * A.ppg;
    SeqInfo s;
    int qb;
    if (decode_item(A.P, tile, s, qb)) {
      row = id;
      for (int t = 0; t < 2 && 2 * ip + t < group; ++t) {
        const int h = hk * group + 2 * ip + t;
        n = max(n, max(0, min(__ldg(A.cnt + (int64_t)h * A.P.tiles_ub + s.tile_base + qb), qb + 1)));
      }
    }
  }
  if (n > kSplitChunk) {
    const int slot = atomicAdd(A.head + 4, 1);
    if (slot < kPlanMaxRows)
      reinterpret_cast<int4*>(reinterpret_cast<uint8_t*>(A.head) + kPlanCandOffset)[slot] = make_int4(id, row, n, 0);
    else
      atomicAdd(A.head + 2, 1);  // the plan then splits no row at all
  }
  unsigned long long t = n;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) t += __shfl_xor_sync(0xffffffffu, t, o);
  if ((threadIdx.x & 31) == 0 && t) atomicAdd(reinterpret_cast<unsigned long long*>(A.head + 6), t);
}

// Pass 2, one CTA: the threshold, and chunk entries for the candidates over it (block-wide
// exclusive scan of their chunk counts).
__global__ void __launch_bounds__(kPlanThreads, 1) split_plan_kernel(const SplitArgs A) {
  __shared__ int warp_sums[32];
  __shared__ int n_split;
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const unsigned long long total = *reinterpret_cast<const unsigned long long*>(A.head + 6);
  const long long thr =
      max((long long)kSplitChunk, (long long)(total * kSplitThrNum / (kSplitThrDen * (unsigned long long)max(1, A.pipelines))));
  if (A.head[4] > kPlanMaxRows) {  // candidates lost: no row is split (the attention reads no rowidx)
    if (tid == 0) A.head[3] = 0x7fffffff;
    return;
  }
  const int nc = A.head[4];
  const int4* cand = reinterpret_cast<const int4*>(reinterpret_cast<const uint8_t*>(A.head) + kPlanCandOffset);
  if (tid == 0) n_split = 0;
  constexpr int kPer = kPlanMaxRows / kPlanThreads;
  int chunks[kPer], my = 0, left_whole = 0;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int ci = tid * kPer + k;
    const int nk = ci < nc ? cand[ci].z : 0;
    chunks[k] = nk > thr ? (nk + kSplitChunk - 1) / kSplitChunk : 0;
    if (chunks[k] > kSplitMaxRowChunks) {
      chunks[k] = 0;
      ++left_whole;
    }
    my += chunks[k];
  }
  int inc = my;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int y = __shfl_up_sync(0xffffffffu, inc, o);
    if (lane >= o) inc += y;
  }
  if (lane == 31) warp_sums[wid] = inc;
  __syncthreads();
  if (wid == 0) {
    int v = warp_sums[lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += y;
    }
    warp_sums[lane] = v;  // inclusive
  }
  __syncthreads();
  int e = inc - my + (wid > 0 ? warp_sums[wid - 1] : 0);
  int used_e = 0;
#pragma unroll
  for (int k = 0; k < kPer; ++k) {
    const int ci = tid * kPer + k, c = chunks[k];
    if (ci >= nc) break;
    const int4 cd = cand[ci];
    // entries advance for every split candidate, so those that fit are a prefix of the array
    if (c > 0 && e + c <= A.max_chunks) {
      A.rowidx[cd.y] = ci;
      A.counters[A.ppg ? 2 * e : e] = 0;
      if (A.ppg) A.counters[2 * e + 1] = 0;
      for (int k2 = 0; k2 < c; ++k2) A.entries[e + k2] = SplitEntry{cd.x, k2, c, ci};
      used_e = e + c;
      atomicAdd(&n_split, 1);
    } else {
      A.rowidx[cd.y] = -1;
      left_whole += c > 0;
    }
    e += c;
  }
  if (left_whole) atomicAdd(A.head + 2, left_whole);
  if (used_e) atomicMax(A.head + 0, used_e);
  __syncthreads();
  if (tid == 0) {
    A.head[1] = n_split;
    A.head[3] = (int)thr;
  }
}

}  // namespace fpb
