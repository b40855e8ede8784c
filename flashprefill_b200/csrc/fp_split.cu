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
// split_plan_kernel runs between the search and the attention: one CTA walks the items in
// the attention's order (heavy first), counts the chunks of every row longer than
// kSplitChunk, and assigns chunk entries by a block-wide exclusive scan, so the longest rows
// get the workspace's chunk budget first; rows beyond the budget stay whole.
#pragma once
#include "fp_common.cuh"

namespace fpb {

constexpr int kSplitChunk = 64;  // listed key blocks per chunk
// per chunk: O [128][128] f32, m [128] f32, l [2 halves][128] f32
constexpr int64_t kSplitPartBytes = 128 * 128 * 4 + 128 * 4 + 2 * 128 * 4;
constexpr int kPlanThreads = 1024;

struct SplitEntry {
  int item;     // attention work item (tile * hq + head)
  int chunk;    // chunk index within the row
  int nchunks;  // chunks of the row
  int srow;     // split-row index (completion counter)
};

struct SplitArgs {
  SeqProblem P;
  const int32_t* cnt;  // [hq][tiles_ub]
  int total_items;     // tiles_ub * hq
  int max_chunks, max_rows;
  SplitEntry* entries;
  int* head;           // [0] entries used, [1] rows split, [2] long rows left whole (zeroed by the host)
  int* rowidx;         // [hq][tiles_ub]: split-row index or -1
  int* counters;       // [max_rows]
};

__global__ void __launch_bounds__(kPlanThreads, 1) split_plan_kernel(const SplitArgs A) {
  __shared__ int warp_sums[2][32];
  const int tid = threadIdx.x, lane = tid & 31, wid = tid >> 5;
  const int per = (A.total_items + kPlanThreads - 1) / kPlanThreads;
  const int i0 = min(A.total_items, tid * per), i1 = min(A.total_items, i0 + per);
  auto row_chunks = [&](int id, int& row) -> int {
    const int tile = id / A.P.hq, h = id - tile * A.P.hq;
    SeqInfo s;
    int qb;
    row = -1;
    if (!decode_item(A.P, tile, s, qb)) return 0;
    row = h * A.P.tiles_ub + s.tile_base + qb;
    const int n = max(0, min(__ldg(A.cnt + row), qb + 1));
    return n > kSplitChunk ? (n + kSplitChunk - 1) / kSplitChunk : 0;
  };
  int my_chunks = 0, my_rows = 0;
  for (int id = i0; id < i1; ++id) {
    int row;
    const int c = row_chunks(id, row);
    my_chunks += c;
    my_rows += c > 0;
  }
  // block-wide exclusive scan of (chunks, rows) in item order
  int inc_c = my_chunks, inc_r = my_rows;
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int yc = __shfl_up_sync(0xffffffffu, inc_c, o), yr = __shfl_up_sync(0xffffffffu, inc_r, o);
    if (lane >= o) {
      inc_c += yc;
      inc_r += yr;
    }
  }
  if (lane == 31) {
    warp_sums[0][wid] = inc_c;
    warp_sums[1][wid] = inc_r;
  }
  __syncthreads();
  if (wid == 0) {
    int vc = warp_sums[0][lane], vr = warp_sums[1][lane];
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int yc = __shfl_up_sync(0xffffffffu, vc, o), yr = __shfl_up_sync(0xffffffffu, vr, o);
      if (lane >= o) {
        vc += yc;
        vr += yr;
      }
    }
    warp_sums[0][lane] = vc;  // inclusive
    warp_sums[1][lane] = vr;
  }
  __syncthreads();
  // Offsets advance for every long row whether or not it fits, so the rows that fit are
  // exactly a prefix (in item order) and their entries are contiguous from 0.
  int e = inc_c - my_chunks + (wid > 0 ? warp_sums[0][wid - 1] : 0);
  int sr = inc_r - my_rows + (wid > 0 ? warp_sums[1][wid - 1] : 0);
  int used_e = 0, used_r = 0, left_whole = 0;
  for (int id = i0; id < i1; ++id) {
    int row;
    const int c = row_chunks(id, row);
    if (row < 0) continue;
    if (c > 0 && e + c <= A.max_chunks && sr < A.max_rows) {
      A.rowidx[row] = sr;
      A.counters[sr] = 0;
      for (int k = 0; k < c; ++k) A.entries[e + k] = SplitEntry{id, k, c, sr};
      used_e = e + c;
      used_r = sr + 1;
    } else {
      A.rowidx[row] = -1;
      left_whole += c > 0;
    }
    e += c;
    sr += c > 0;
  }
  if (left_whole) atomicAdd(A.head + 2, left_whole);
  if (used_e) {
    atomicMax(A.head + 0, used_e);
    atomicMax(A.head + 1, used_r);
  }
}

}  // namespace fpb
