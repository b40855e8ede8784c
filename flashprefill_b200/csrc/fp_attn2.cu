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
// Shared memory: Q_0, Q_1, K[2], V[2] (32 KB each, 128-byte swizzled), 4 KB of output
// staging per softmax warp, and the barriers.
// The epilogue takes O / l from TMEM into registers and writes each warp's 32 rows through its
// own staging area, half a row at a time, as whole 128-byte lines (a thread storing its own
// 256-byte row makes every store instruction touch 32 lines, and that burst holds up the
// shared-memory and barrier traffic of the producer and the MMA issuer at every item boundary).
// The staging area is the warp's own, so it never holds back the next item's loads.
#include <type_traits>

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
  int profile;           // instrumented builds: accumulate g_attn2_prof
  int trace;             // instrumented builds: record CTA 0's events in g_attn2_trace
  // long rows split into chunks (fp_split.cu, head-pair items); split = 0 runs every item whole
  int split;
  const SplitEntry* sp_entries;
  const int* sp_head;    // plan header: [0] chunk entries, [3] split threshold
  const int* sp_rowidx;  // [items]: split-row index or -1 (items over the threshold)
  int* sp_counters;      // [2 * entry + tile]: chunks finished, at the row's first entry
  float* sp_part;        // per chunk entry and tile: O [128][128], m [128], l [2][128]
  // other GPUs' copies of the output (same layout and strides as `out`, reached over NVLink):
  // the epilogue writes every output row there too (kernel instance kPeers)
  int n_peers;
  void* peer_out[kMaxOutPeers];
  void* out;             // output base
  int64_t o_sb, o_ss, o_sh;  // output strides in elements
};

// 1: each tile's P goes to a shared-memory tile of its own instead of over S in TMEM, so S_t(next)
// may be issued as soon as the softmax has read S_t into registers and runs under the softmax of
// this block (the K ring then has one stage: Q, K, V[2], P[2] take 224 KB)
#ifndef FPB_A2_PSMEM
#define FPB_A2_PSMEM 0
#endif
constexpr int kA2Threads = 384;
// Register split: compiled for 168 per thread (384 x 168 = 64512 <= 65536); warps 0-3 give back
// to 80, the two softmax warpgroups grow to 208: 128 * 80 + 256 * 208 = 63488.
constexpr int kA2LaunchRegs = 168, kA2RoleRegs = FPB_A2_PSMEM ? 88 : 80, kA2SoftRegs = 208;
static_assert(128 * kA2RoleRegs + 256 * kA2SoftRegs <= kA2Threads * kA2LaunchRegs, "register split");
#ifndef FPB_A2_POLY_EVERY
#define FPB_A2_POLY_EVERY 1000
#endif
// 1: the exp passes of the two tiles' softmax warps on one SM sub-partition take turns
#ifndef FPB_A2_TURNS
#define FPB_A2_TURNS 0
#endif
constexpr int kA2PolyEvery = FPB_A2_POLY_EVERY;  // one exp2 pair in kA2PolyEvery on the FMA pipe
// MMA issuing threads: 2 = one per tile (warps 1 and 3), each walking the union and issuing its
// tile's S and PV; 1 = one thread for both tiles (warp 1)
#ifndef FPB_A2_ISSUERS
#define FPB_A2_ISSUERS 1
#endif
constexpr int kA2Issuers = FPB_A2_ISSUERS;
constexpr uint32_t kA2Tile = 128 * 128 * 2;
constexpr uint32_t kA2Half = kA2Tile / 2;

// Rings: three K stages (a key tile is needed as soon as its S can be issued) and two V stages.
// Pipeline variants, measured at 128K tokens on one B200 (attention ms): two K stages 2.80
// (three 2.85); one producer thread for K and V 2.80 (a second one for V 3.21); Q released
// after the item's last MMA 2.80 (after its last S 2.87); one MMA issuer 2.80 (one per tile
// 3.17-3.58).  Every extra polling thread takes issue slots from the softmax warps.
#ifndef FPB_A2_KSTAGES
#define FPB_A2_KSTAGES (FPB_A2_PSMEM ? 1 : 2)
#endif
// 1: a second producer thread (warp 2) loads the V tiles; 0: the K producer loads both
#ifndef FPB_A2_SPLIT_PRODUCER
#define FPB_A2_SPLIT_PRODUCER 0
#endif
// 1: Q_t is released after the item's last S_t; 0: after the item's last MMA
#ifndef FPB_A2_EARLY_QFREE
#define FPB_A2_EARLY_QFREE 0
#endif
// 1: the producer prefetches an item's Q tiles into L2 as soon as it has fetched the item, before
// it waits for the Q buffers to be free
#ifndef FPB_A2_QPREFETCH
#define FPB_A2_QPREFETCH 0
#endif
// 1: the producer issues an item's first K/V loads before it waits for the Q buffers
#ifndef FPB_A2_KFIRST
#define FPB_A2_KFIRST 0
#endif
constexpr bool kA2KFirst = FPB_A2_KFIRST;
// > 0: the producer prefetches into L2 the K and V tiles of the list entries this far ahead of
// the ones it loads
#ifndef FPB_A2_AHEAD
#define FPB_A2_AHEAD 0
#endif
constexpr int kA2Ahead = FPB_A2_AHEAD;
#ifndef FPB_A2_ORDER
#define FPB_A2_ORDER 0
#endif
constexpr int kA2Order = FPB_A2_ORDER, kA2HotTiles = 8;
// 1: the MMA issuer's waits suspend between polls (try_wait with a time hint); 0: they spin
#ifndef FPB_A2_MMA_SLEEP
#define FPB_A2_MMA_SLEEP 0
#endif
constexpr int kA2KStages = FPB_A2_KSTAGES, kA2VStages = 2;
// Timing experiments only (wrong results): skip the exp2 pass / the O rescale
#ifndef FPB_A2_TIMING_NOEXP
#define FPB_A2_TIMING_NOEXP 0
#endif
#ifndef FPB_A2_TIMING_NOSOFTMAX
#define FPB_A2_TIMING_NOSOFTMAX 0
#endif
#ifndef FPB_A2_TIMING_NORESCALE
#define FPB_A2_TIMING_NORESCALE 0
#endif
// Timing experiments only: 1 = no K/V tile loads (the full barriers are arrived without data),
// 2 = every K/V load reads the sequence's first key block (always an L2 hit)
#ifndef FPB_A2_TIMING_KV
#define FPB_A2_TIMING_KV 0
#endif
// 1: the softmax warps poll for S without suspending (0: try_wait with a suspend-time hint)
#ifndef FPB_A2_SM_SPIN
#define FPB_A2_SM_SPIN 0
#endif
#if FPB_A2_SM_SPIN
#define A2_SM_WAIT mbar_wait_warp<false>
#else
#define A2_SM_WAIT mbar_wait_warp_sleep
#endif
// 1: the K/V producer's waits spin (0: try_wait with a suspend-time hint)
#ifndef FPB_A2_PROD_SPIN
#define FPB_A2_PROD_SPIN 0
#endif
#if FPB_A2_PROD_SPIN
#define A2_PROD_WAIT mbar_wait
#else
#define A2_PROD_WAIT mbar_wait_sleep
#endif
// 1: the MMA issuer polls with mbarrier.test_wait (never suspends) instead of try_wait
#ifndef FPB_A2_MMA_PROBE
#define FPB_A2_MMA_PROBE 0
#endif
#if FPB_A2_MMA_SLEEP
#define A2_MMA_WAIT mbar_wait_sleep
#elif FPB_A2_MMA_PROBE
#define A2_MMA_WAIT mbar_wait_probe
#else
#define A2_MMA_WAIT mbar_wait
#endif
constexpr bool kA2SplitProducer = FPB_A2_SPLIT_PRODUCER, kA2EarlyQFree = FPB_A2_EARLY_QFREE;
// 1: the epilogue stages each warp's 32 output rows through shared memory, half a row at a
// time, and stores them with consecutive lanes on consecutive 16-byte pieces of a row (whole
// 128-byte lines); 0: each thread stores its own 256-byte row (32 lines per warp instruction)
#ifndef FPB_A2_STAGE_OUT
#define FPB_A2_STAGE_OUT 1
#endif
constexpr bool kA2PSmem = FPB_A2_PSMEM;
// 1: the softmax warps signal p_full / s_free / o_empty with one arrival per warp (lane 0, after
// the warp has synchronised) instead of one per thread: 4 arrivals per tile instead of 128
#ifndef FPB_A2_WARP_ARRIVE
#define FPB_A2_WARP_ARRIVE 0
#endif
constexpr int kA2RowArrivals = FPB_A2_WARP_ARRIVE ? 4 : 128;
static_assert(!kA2PSmem || (!FPB_A2_TIMING_NOSOFTMAX && kA2Issuers == 1 && !kA2EarlyQFree),
              "the shared-memory P pipeline has one MMA issuer and a full softmax");
// the output staging areas (8 softmax warps x 32 rows x 128 B), or the two P tiles, whose halves
// the warps of each tile use as staging areas
// 1: three Q buffers.  Tile 1's Q always uses buffer 2; tile 0's alternates between buffers 0
// and 1 from one item to the next, so the producer loads the next item's Q_0 while this item
// runs, and the item's epilogue stages its output rows in its own Q_0 buffer (free once its
// MMAs are done).  The producer reuses a Q_0 buffer after the epilogue of the item two back.
#ifndef FPB_A2_QROT
#define FPB_A2_QROT 0
#endif
constexpr bool kA2QRot = FPB_A2_QROT;
static_assert(!kA2QRot || (!kA2PSmem && kA2Issuers == 1 && !kA2EarlyQFree && !kA2KFirst && !kA2SplitProducer),
              "the rotating Q buffers run with the default pipeline");
constexpr int kA2QTiles = kA2QRot ? 3 : 2;
constexpr int kA2StageBytes =
    FPB_A2_PSMEM ? 2 * (int)kA2Tile : (FPB_A2_STAGE_OUT && !FPB_A2_QROT) ? (int)kA2Tile : 0;
__host__ __device__ constexpr size_t attn2_smem_bytes() {
  return (size_t)kA2Tile * (kA2QTiles + kA2KStages + kA2VStages) + kA2StageBytes + 1024 + 1024;
}

// Instrumentation (build flag -DFPB_ATTN_PROFILE=1, run time FLASHPREFILL_B200_PROFILE=1): cycle
// sums per phase over all CTAs, recorded by one thread per role (kA2ProfNames in fp_api.cu).
constexpr int kA2ProfSlots = 24;
#if FPB_ATTN_PROFILE
__device__ unsigned long long g_attn2_prof[kA2ProfSlots];
#define A2_CLK() clock64()
#define A2_ADD(slot, v) \
  do {                  \
    if (prof) atomicAdd(prof + (slot), (unsigned long long)(v)); \
  } while (0)
// the first wait of the launch that gives up: (block, thread, profile slot, clock)
__device__ unsigned long long g_attn2_gaveup[4];
#define A2_W(slot, call)                                                       \
  ({                                                                           \
    const unsigned long long t0_ = clock64();                                  \
    const bool r_ = (call);                                                    \
    A2_ADD(slot, clock64() - t0_);                                             \
    if (!r_ && atomicCAS(&g_attn2_gaveup[0], 0ull, 1ull + blockIdx.x) == 0ull) { \
      g_attn2_gaveup[1] = threadIdx.x;                                         \
      g_attn2_gaveup[2] = (slot);                                              \
      g_attn2_gaveup[3] = t0_;                                                 \
    }                                                                          \
    r_;                                                                        \
  })
// event trace of CTA 0 (FLASHPREFILL_B200_TRACE=<file>): (clock, kind << 32 | value) pairs
constexpr int kA2TraceCap = 1 << 16;
__device__ unsigned long long g_attn2_trace[2 * kA2TraceCap];
__device__ unsigned int g_attn2_trace_n;
#define A2_EV(kind, val)                                                                         \
  do {                                                                                           \
    if (trace_on) {                                                                              \
      const unsigned long long now_ = clock64();                                                 \
      const unsigned i_ = atomicAdd(trace_ctr, 1u); /* shared memory: short round trip */        \
      if (i_ < kA2TraceCap) {                                                                    \
        g_attn2_trace[2 * i_] = now_;                                                            \
        g_attn2_trace[2 * i_ + 1] = ((unsigned long long)(kind) << 32) | (unsigned)(val);        \
      }                                                                                          \
    }                                                                                            \
  } while (0)
#else
#define A2_CLK() 0ull
#define A2_ADD(slot, v) ((void)0)
#define A2_W(slot, call) (call)
#define A2_EV(kind, val) ((void)0)
#endif

struct Item2 {
  int valid;  // 0: no more work, 1: item, 2: nothing to do (padding tile, or a row done as chunks)
  int start, len, bcoord, qb, row;
  int h[2];      // query heads of the two tiles (h[1] = -1: single-head item)
  int n[2];      // listed blocks per tile in this item (a chunk: its share of the list)
  int diag[2];   // the tile's last block in this item is the diagonal block (causal mask)
  int nfull[2];  // listed blocks per tile in the whole row
  int chunk;     // split_code(entry, chunk, nchunks) of a chunk of a split row, or -1
  int pad[5];
};
static_assert(sizeof(Item2) == 80, "item ring slot");

// 16-byte store of output chunk q4 of a row to every peer copy of the output (plain stores over
// NVLink into CUDA-IPC mappings; no TMA, no multicast).
__device__ __forceinline__ void store_to_peers(const Attn2Args& A, int64_t byte_off, uint4 v) {
  for (int p = 0; p < A.n_peers; ++p)
    *reinterpret_cast<uint4*>(reinterpret_cast<uint8_t*>(A.peer_out[p]) + byte_off) = v;
}

// The 32 output rows a warp has just written (lane l: row pointer `row`, written iff `valid`)
// sent on to every peer copy of the output.  Each lane wrote a whole 256-byte row; read back
// (visible to the warp after __syncwarp), the rows go out with consecutive lanes on consecutive
// 16-byte pieces of a row, so the NVLink writes are full 256-byte segments.  Whole warp only.
template <typename T>
__device__ __forceinline__ void warp_rows_to_peers(const Attn2Args& A, const T* row, bool valid) {
  __syncwarp();
  const unsigned vmask = __ballot_sync(0xffffffffu, valid);
  const int lane = threadIdx.x & 31;
  const long long mine = reinterpret_cast<long long>(row);
#pragma unroll 4
  for (int i = 0; i < 16; ++i) {
    const int c = i * 32 + lane, rl = c >> 4, piece = c & 15;
    const long long src = __shfl_sync(0xffffffffu, mine, rl);
    if ((vmask >> rl) & 1u) {
      const uint4* p = reinterpret_cast<const uint4*>(src) + piece;
      store_to_peers(A, reinterpret_cast<const uint8_t*>(p) - reinterpret_cast<const uint8_t*>(A.out), *p);
    }
  }
}

template <typename T, bool kPeers>
__global__ void __launch_bounds__(kA2Threads, 1)
    sparse_attn2_kernel(const __grid_constant__ CUtensorMap tm_q, const __grid_constant__ CUtensorMap tm_k,
                        const __grid_constant__ CUtensorMap tm_v, const Attn2Args A) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sQ = smem;                               // [kA2QTiles] tiles
  uint8_t* sK = smem + kA2QTiles * kA2Tile;         // [kA2KStages]
  uint8_t* sV = sK + kA2KStages * kA2Tile;          // [kA2VStages]
  uint8_t* sStage = sV + kA2VStages * kA2Tile;     // [softmax warp] 32 rows x 128 B (FPB_A2_STAGE_OUT)
  (void)sStage;                                     // FPB_A2_PSMEM: also the P tile (128 rows x 128 keys)
  uint64_t* bars = reinterpret_cast<uint64_t*>(sStage + kA2StageBytes);
  uint64_t* item_full = bars + 0;   // [slot]
  uint64_t* item_empty = bars + 2;  // [slot]
  uint64_t* q_full = bars + 4;      // [tile]
  uint64_t* q_empty = bars + 6;
  uint64_t* k_full = bars + 8;      // [K stage], 4 reserved
  uint64_t* k_empty = bars + 12;    // [K stage] (tile 0's, or the single issuer's)
  uint64_t* v_full = bars + 27;     // [V stage]
  uint64_t* v_empty = bars + 29;    // [V stage] (tile 0's, or the single issuer's)
  // With one issuer per tile each tile releases stages on barriers of its own: a tile that
  // lists few blocks runs ahead, and on a shared counting barrier its release of a later use
  // of a stage could complete an earlier use's phase before the other tile is done with it.
  uint64_t* k_empty1 = bars + 121;  // [K stage] tile 1's (after the profile counters)
  uint64_t* v_empty1 = bars + 124;  // [V stage] tile 1's
  uint64_t* s_full = bars + 16;     // [tile]
  uint64_t* p_full = bars + 18;
  uint64_t* o_full = bars + 20;
  uint64_t* o_empty = bars + 22;
  uint64_t* mma_done = bars + 24;
  uint64_t* epi = bars + 25;        // [tile]: bounded sync of a tile's 128 softmax threads
  uint64_t* s_free = bars + 64;     // [tile] (FPB_A2_PSMEM): the softmax has read S_t into registers
  uint64_t* p_grant = bars + 66;    // [tile] (FPB_A2_PSMEM): P_t was read by its PV, P_t may be written
  uint64_t* q_full_b = bars + 70;   // (FPB_A2_QROT): Q buffer 2 (tile 1) loaded; q_full[0/1]: buffers 0/1
  uint64_t* stg_done = bars + 71;   // [Q_0 buffer] (FPB_A2_QROT): every softmax thread is past an item
  Item2* ring = reinterpret_cast<Item2*>(bars + 32);          // [slot], 80 bytes each
  int* umask_raw = reinterpret_cast<int*>(ring + 2);
  volatile int* umask = umask_raw;  // [K stage]: tiles | last << 2
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(umask_raw + 4);
  volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
  volatile int* last_chunk = reinterpret_cast<volatile int*>(tmem_slot + 2);  // [tile]
  volatile int* pp_want = reinterpret_cast<volatile int*>(tmem_slot + 4);  // [tile][quad]
  volatile int* pp_turn = reinterpret_cast<volatile int*>(tmem_slot + 12);  // [quad]
  unsigned long long* prof_sm = reinterpret_cast<unsigned long long*>(bars + 96);  // [kA2ProfSlots]

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  // the recording thread of each role (producer, MMA issuer, row 0 of each softmax tile)
  unsigned long long* prof =
      (A.profile && (threadIdx.x == 0 || threadIdx.x == 32 || threadIdx.x == 128 || threadIdx.x == 256)) ? prof_sm
                                                                                                           : nullptr;
  (void)prof;
  unsigned* trace_ctr = reinterpret_cast<unsigned*>(prof_sm + kA2ProfSlots);
  (void)trace_ctr;
  const bool trace_on = A.trace && blockIdx.x == 0 &&
                        (threadIdx.x == 0 || threadIdx.x == 32 || threadIdx.x == 64 || threadIdx.x == 128 ||
                         threadIdx.x == 256);
  (void)trace_on;
  const unsigned long long t_kernel0 = A2_CLK();
  (void)t_kernel0;
  if (threadIdx.x < kA2ProfSlots + 1) prof_sm[threadIdx.x] = 0;  // counters and the trace index
  if (threadIdx.x == 0) {
    for (int i = 0; i < kA2KStages; ++i) {
      mbar_init(k_full + i, 1);
      mbar_init(k_empty + i, 1);
      mbar_init(k_empty1 + i, 1);
    }
    for (int i = 0; i < 2; ++i) {
      mbar_init(item_full + i, 1);
      mbar_init(item_empty + i, kA2Issuers + (kA2SplitProducer ? 1 : 0) + 256);  // issuer(s), V producer, softmax
      mbar_init(q_full + i, 1);
      mbar_init(q_empty + i, 1);
      mbar_init(v_full + i, 1);
      mbar_init(v_empty + i, 1);
      mbar_init(v_empty1 + i, 1);
      mbar_init(s_full + i, 1);
      mbar_init(p_full + i, kA2RowArrivals);
      mbar_init(o_full + i, 1);
      mbar_init(o_empty + i, kA2RowArrivals);
      mbar_init(epi + i, 128);
      mbar_init(s_free + i, kA2RowArrivals);
      mbar_init(p_grant + i, 1);
      mbar_init(stg_done + i, 256);
    }
    mbar_init(q_full_b, 1);
    mbar_init(mma_done, kA2Issuers);
    for (int i = 0; i < 12; ++i) pp_want[i] = 0;  // want flags, then the turn and two exit counters
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
    // Union of a head pair's two ascending lists: calls visit(kb, mask) once per distinct block in
    // ascending order (mask bit t: tile t lists it; bit 2: the item's last union block).  The
    // K and the V producer walk the same union, so both number its blocks alike.
    auto walk_union = [&](const int32_t* l0, int n0, const int32_t* l1, int n1, int qb, auto&& visit,
                          auto&& ahead) -> bool {
      int j0 = 0, j1 = 0;
      int a0 = n0 > 0 ? __ldg(l0) : 0x7fffffff;
      int a1 = n1 > 0 ? __ldg(l1) : 0x7fffffff;
      if (kA2Ahead > 0) {  // the first entries' tiles, then one entry per advance, kA2Ahead ahead
        for (int j = 1; j < kA2Ahead && j < n0; ++j) ahead(__ldg(l0 + j));
        for (int j = 1; j < kA2Ahead && j < n1; ++j) ahead(__ldg(l1 + j));
      }
      while (j0 < n0 || j1 < n1) {
        int kb = min(a0, a1);
        int m = 0;
        if (a0 == kb) {
          m |= 1;
          ++j0;
          a0 = j0 < n0 ? __ldg(l0 + j0) : 0x7fffffff;
          if (kA2Ahead > 0 && j0 + kA2Ahead - 1 < n0) ahead(__ldg(l0 + j0 + kA2Ahead - 1));
        }
        if (a1 == kb) {
          m |= 2;
          ++j1;
          a1 = j1 < n1 ? __ldg(l1 + j1) : 0x7fffffff;
          if (kA2Ahead > 0 && j1 + kA2Ahead - 1 < n1) ahead(__ldg(l1 + j1 + kA2Ahead - 1));
        }
        if (j0 >= n0 && j1 >= n1) m |= 4;
        if (kb < 0 || kb > qb) {
          raise_error(A.P.err, kErrIndexRange);
          kb = qb;
        }
        if (!visit(kb, m)) return false;
      }
      return true;
    };
    // Visit order of whole items (position -> item id = tile * npairs + pair).  Default: heavy
    // tiles first, all pairs of a tile together.  FPB_A2_ORDER=1: the kA2HotTiles heaviest tiles
    // first as before, then KV head by KV head, so that the items in flight share one KV head's
    // K/V and its re-reads hit L2.
    auto visit_order = [&](int pos) -> int {
      if (kA2Order == 0) return pos;
      const int ntiles = A.total_items / npairs, hot = min(kA2HotTiles, ntiles);
      if (pos < hot * npairs) return pos;
      const int r = pos - hot * npairs, rest = ntiles - hot;
      const int hk = r / (rest * A.ppg), w = r - hk * rest * A.ppg;
      return (hot + w / A.ppg) * npairs + hk * A.ppg + w % A.ppg;
    };
    if (warp == 0 && lane == 0) {
      // ------------------------------------------------------------ scheduler + K producer
      prefetch_tmap(&tm_q);
      prefetch_tmap(&tm_k);
      const uint64_t stream_once = l2_policy_evict_first();
      uint32_t it = 0, kseq = 0, qld[2] = {0, 0};
      uint32_t pq = 0, qldx0 = 0, qldx1 = 0;  // FPB_A2_QROT: items started, loads per Q_0 buffer
      // chunks of split rows come first in the work order (they are the longest work)
      const int n_ent = A.split ? A.sp_head[0] : 0;
      const int split_thr = A.split ? A.sp_head[3] : 0x7fffffff;  // only rows above it can be split
      bool ok = true;
      while (ok) {
        const int slot = it & 1;
        if (!A2_W(20, A2_PROD_WAIT(item_empty + slot, ((it >> 1) & 1) ^ 1, abort))) break;
        Item2 f{};
        A2_EV(20, it);
        const int id = atomicAdd(A.counter, 1);
        A2_EV(21, id);
        const int32_t* lst[2] = {nullptr, nullptr};
        if (id >= n_ent + A.total_items) {
          f.valid = 0;
        } else {
          const SplitEntry se = id < n_ent ? A.sp_entries[id] : SplitEntry{visit_order(id - n_ent), 0, 0, -1};
          const int tile = se.item / npairs, pr = se.item - tile * npairs;
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
            f.chunk = id < n_ent ? split_code(id, se.chunk, se.nchunks) : -1;
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              f.n[t] = f.nfull[t] = f.diag[t] = 0;
              if (f.h[t] < 0) continue;
              const int64_t row = (int64_t)f.h[t] * A.P.tiles_ub + f.row;
              f.nfull[t] = max(0, min(__ldg(A.cnt + row), qb + 1));
              const int j0 = id < n_ent ? se.chunk * kSplitChunk : 0;
              f.n[t] = id < n_ent ? max(0, min(kSplitChunk, f.nfull[t] - j0)) : f.nfull[t];
              lst[t] = A.idx + row * A.P.cap + j0;
              if (f.n[t] > 0) {
                const int last = __ldg(lst[t] + f.n[t] - 1);
                f.diag[t] = last == qb || last < 0 || last > qb;
              }
            }
            // a whole row that the plan cut into chunks is done by its chunk items
            if (id >= n_ent && max(f.nfull[0], f.nfull[1]) > split_thr && __ldg(A.sp_rowidx + se.item) >= 0)
              f.valid = 2;
          }
        }
        A2_EV(22, f.n[0] + f.n[1]);
        ring[slot] = f;
        mbar_arrive(item_full + slot);
        ++it;
        if (f.valid == 0) break;
        if (f.valid != 1 || (f.n[0] == 0 && f.n[1] == 0)) continue;
        const int hkv = f.h[0] / group;
        const int qrow = f.start + f.qb * kBlock - A.P.q_off;  // rows before a chunk load as zeros
#if FPB_A2_QPREFETCH
#pragma unroll
        for (int t = 0; t < 2; ++t)
          if (f.n[t] > 0) {
            tma_prefetch_4d(&tm_q, 0, f.h[t], qrow, f.bcoord);
            tma_prefetch_4d(&tm_q, 64, f.h[t], qrow, f.bcoord);
          }
#endif
        // Q_0 and Q_1 of the item: before its first K/V tiles, or (FPB_A2_KFIRST) right after them,
        // so that the item's first K/V loads do not queue behind the wait for the Q buffers
        bool q_pending = true;
        auto load_q = [&]() -> bool {
          q_pending = false;
#pragma unroll
          for (int t = 0; t < 2; ++t) {
            if (f.n[t] == 0) continue;
            if (!A2_W(19, A2_PROD_WAIT(q_empty + t, (qld[t] & 1) ^ 1, abort))) return false;
            A2_EV(23, t);
            ++qld[t];
            mbar_arrive_expect_tx(q_full + t, kA2Tile);
            tma_load_4d_hint(sQ + t * kA2Tile, &tm_q, q_full + t, 0, f.h[t], qrow, f.bcoord, stream_once);
            tma_load_4d_hint(sQ + t * kA2Tile + kA2Half, &tm_q, q_full + t, 64, f.h[t], qrow, f.bcoord,
                             stream_once);
          }
          return true;
        };
        // FPB_A2_QROT: Q_0 into buffer pq & 1 once the epilogue of the item two back is done;
        // Q_1 into buffer 2 after the item's first K/V, once the last item's MMAs are done
        auto load_q0 = [&]() -> bool {
          if (f.n[0] == 0) return true;
          const int xs = pq & 1;
          if (pq >= 2 && !A2_W(19, A2_PROD_WAIT(stg_done + xs, ((pq - 2) >> 1) & 1, abort))) return false;
          if (xs) ++qldx1; else ++qldx0;
          mbar_arrive_expect_tx(q_full + xs, kA2Tile);
          tma_load_4d_hint(sQ + xs * kA2Tile, &tm_q, q_full + xs, 0, f.h[0], qrow, f.bcoord, stream_once);
          tma_load_4d_hint(sQ + xs * kA2Tile + kA2Half, &tm_q, q_full + xs, 64, f.h[0], qrow, f.bcoord,
                           stream_once);
          return true;
        };
        auto load_q1 = [&]() -> bool {
          q_pending = false;
          if (f.n[1] == 0) return true;
          if (!A2_W(19, A2_PROD_WAIT(q_empty + 1, (qld[1] & 1) ^ 1, abort))) return false;
          ++qld[1];
          mbar_arrive_expect_tx(q_full_b, kA2Tile);
          tma_load_4d_hint(sQ + 2 * kA2Tile, &tm_q, q_full_b, 0, f.h[1], qrow, f.bcoord, stream_once);
          tma_load_4d_hint(sQ + 2 * kA2Tile + kA2Half, &tm_q, q_full_b, 64, f.h[1], qrow, f.bcoord, stream_once);
          return true;
        };
        if (kA2QRot) {
          if (!load_q0()) break;
        } else if (!kA2KFirst && !load_q()) {
          break;
        }
        ok = walk_union(lst[0], f.n[0], lst[1], f.n[1], f.qb, [&](int kb, int m) -> bool {
          const int st = kseq % kA2KStages;
          const uint32_t ph = (kseq / kA2KStages) & 1;
          A2_EV(24, kseq);
          if (!A2_W(17, A2_PROD_WAIT(k_empty + st, ph ^ 1, abort))) return false;
          if (kA2Issuers == 2 && !A2_W(22, mbar_wait_sleep(k_empty1 + st, ph ^ 1, abort))) return false;
          umask[st] = m;
          // test hook (one-shot): the first producer to reach a key load while it is armed
          // skips that load, so the MMA issuer's wait runs out
          bool withhold = false;
          if (kseq == 0 && *(volatile int*)&g_test_withhold != 0) withhold = atomicExch(&g_test_withhold, 0) != 0;
          A2_EV(7, kseq);
          if (FPB_A2_TIMING_KV == 1) {
            mbar_arrive(k_full + st);
          } else if (!withhold) {
            const int krow = f.start + (FPB_A2_TIMING_KV == 2 ? 0 : kb) * kBlock;
            mbar_arrive_expect_tx(k_full + st, kA2Tile);
            tma_load_4d(sK + st * kA2Tile, &tm_k, k_full + st, 0, hkv, krow, f.bcoord);
            tma_load_4d(sK + st * kA2Tile + kA2Half, &tm_k, k_full + st, 64, hkv, krow, f.bcoord);
          }
          if (!kA2SplitProducer) {  // this thread loads the V tile too
            const int vs = kseq & 1;
            const uint32_t vph = ((kseq >> 1) & 1) ^ 1;
            if (!A2_W(18, A2_PROD_WAIT(v_empty + vs, vph, abort))) return false;
            if (kA2Issuers == 2 && !A2_W(22, mbar_wait_sleep(v_empty1 + vs, vph, abort))) return false;
            const int vrow = f.start + (FPB_A2_TIMING_KV == 2 ? 0 : kb) * kBlock;
            if (FPB_A2_TIMING_KV == 1) {
              mbar_arrive(v_full + vs);
            } else {
              mbar_arrive_expect_tx(v_full + vs, kA2Tile);
              tma_load_4d(sV + vs * kA2Tile, &tm_v, v_full + vs, 0, hkv, vrow, f.bcoord);
              tma_load_4d(sV + vs * kA2Tile + kA2Half, &tm_v, v_full + vs, 64, hkv, vrow, f.bcoord);
            }
          }
          ++kseq;
          if (q_pending && !(kA2QRot ? load_q1() : load_q())) return false;
          return true;
        }, [&](int kb) {  // L2 prefetch of a block's K and V tiles, kA2Ahead list entries ahead
          if (kb < 0 || kb > f.qb) return;
          const int row = f.start + kb * kBlock;
          tma_prefetch_4d(&tm_k, 0, hkv, row, f.bcoord);
          tma_prefetch_4d(&tm_k, 64, hkv, row, f.bcoord);
          tma_prefetch_4d(&tm_v, 0, hkv, row, f.bcoord);
          tma_prefetch_4d(&tm_v, 64, hkv, row, f.bcoord);
        });
        ++pq;
      }
      if (*abort) {  // let loads still in flight land before the CTA exits
        volatile int no_abort = 0;
        for (uint32_t q = kseq > kA2KStages ? kseq - kA2KStages : 0; q < kseq; ++q) {
          mbar_wait(k_full + q % kA2KStages, (q / kA2KStages) & 1, &no_abort);
          no_abort = 0;
        }
        if (!kA2SplitProducer)
          for (uint32_t q = kseq > 2 ? kseq - 2 : 0; q < kseq; ++q) {
            mbar_wait(v_full + (q & 1), (q >> 1) & 1, &no_abort);
            no_abort = 0;
          }
        if (kA2QRot) {
          if (qldx0) mbar_wait(q_full, (qldx0 - 1) & 1, &no_abort);
          no_abort = 0;
          if (qldx1) mbar_wait(q_full + 1, (qldx1 - 1) & 1, &no_abort);
          no_abort = 0;
          if (qld[1]) mbar_wait(q_full_b, (qld[1] - 1) & 1, &no_abort);
          no_abort = 0;
        } else {
          for (int t = 0; t < 2; ++t)
            if (qld[t]) {
              mbar_wait(q_full + t, (qld[t] - 1) & 1, &no_abort);
              no_abort = 0;
            }
        }
      }
    } else if (kA2SplitProducer && warp == 2 && lane == 0) {
      // ------------------------------------------------------------ V producer
      prefetch_tmap(&tm_v);
      uint32_t it = 0, vseq = 0;
      while (true) {
        const int slot = it & 1;
        if (!A2_W(23, mbar_wait_sleep(item_full + slot, (it >> 1) & 1, abort))) break;
        const Item2 f = ring[slot];
        mbar_arrive(item_empty + slot);
        ++it;
        if (f.valid == 0) break;
        if (f.valid != 1 || (f.n[0] == 0 && f.n[1] == 0)) continue;
        const int hkv = f.h[0] / group;
        const int j0 = f.chunk >= 0 ? ((f.chunk >> 17) & 127) * kSplitChunk : 0;
        const int32_t* l0 = A.idx + ((int64_t)f.h[0] * A.P.tiles_ub + f.row) * A.P.cap + j0;
        const int32_t* l1 = f.h[1] >= 0 ? A.idx + ((int64_t)f.h[1] * A.P.tiles_ub + f.row) * A.P.cap + j0 : l0;
        if (!walk_union(l0, f.n[0], l1, f.n[1], f.qb, [&](int kb, int) -> bool {
              const int st = vseq & 1;
              if (!A2_W(18, mbar_wait_sleep(v_empty + st, ((vseq >> 1) & 1) ^ 1, abort))) return false;
              if (kA2Issuers == 2 && !A2_W(22, mbar_wait_sleep(v_empty1 + st, ((vseq >> 1) & 1) ^ 1, abort))) return false;
              A2_EV(8, vseq);
              const int vrow = f.start + kb * kBlock;
              mbar_arrive_expect_tx(v_full + st, kA2Tile);
              tma_load_4d(sV + st * kA2Tile, &tm_v, v_full + st, 0, hkv, vrow, f.bcoord);
              tma_load_4d(sV + st * kA2Tile + kA2Half, &tm_v, v_full + st, 64, hkv, vrow, f.bcoord);
              ++vseq;
              return true;
            }, [](int) {}))
          break;
      }
      if (*abort) {
        volatile int no_abort = 0;
        for (uint32_t q = vseq > 2 ? vseq - 2 : 0; q < vseq; ++q) {
          mbar_wait(v_full + (q & 1), (q >> 1) & 1, &no_abort);
          no_abort = 0;
        }
      }
    } else if (kA2Issuers == 2 && (warp == 1 || warp == 3) && lane == 0) {
      // ------------------------------------------------------------ MMA issuer of one tile
      // Each tile has its own issuing thread, so one tile's waits (its softmax, its loads)
      // never hold back the other tile's MMAs.  Both walk every union block: a block the tile
      // does not list still gets the tile's arrivals on the stage's empty barriers (count 2).
      constexpr uint32_t id_s = idesc_f16(128, 128, DT<T>::is_bf16, false);
      constexpr uint32_t id_o = idesc_f16(128, 128, DT<T>::is_bf16, true);
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV);
      auto run = [&](auto tt) {
        constexpr int t = decltype(tt)::value;
        uint64_t* my_k_empty = t ? k_empty1 : k_empty;
        uint64_t* my_v_empty = t ? v_empty1 : v_empty;
        uint32_t it = 0, kvseq = 0, qc = 0, pc = 0, oc = 0;
        bool ok = true;
        while (ok) {
          const int slot = it & 1;
          if (!A2_W(16, mbar_wait_sleep(item_full + slot, (it >> 1) & 1, abort))) break;
          const int valid = ring[slot].valid, n0 = ring[slot].n[0], n1 = ring[slot].n[1];
          const int n_t = t ? n1 : n0;
          mbar_arrive(item_empty + slot);
          ++it;
          if (valid == 0) break;
          if (valid != 1 || (n0 == 0 && n1 == 0)) continue;
          int pend = -1, s_left = n_t;
          bool first = true, qw = false;
          auto issue_pv = [&]() -> bool {
            const int st = pend & 1;
            if (first) {  // the previous item's epilogue must have read O_t
              if (!A2_W(12, A2_MMA_WAIT(o_empty + t, (oc & 1) ^ 1, abort))) return false;
              ++oc;
            }
            if (!A2_W(10, A2_MMA_WAIT(p_full + t, pc & 1, abort))) return false;
            ++pc;
            if (!A2_W(11, A2_MMA_WAIT(v_full + st, (pend >> 1) & 1, abort))) return false;
            tc_fence_after();
            const uint32_t vb = v_base + st * kA2Tile;
#pragma unroll
            for (int ks = 0; ks < 8; ++ks)  // A = P (TMEM, 8 packed columns per 16 keys), B = V (MN-major)
              umma_ts(tmem + 256 + t * 128, tmem + t * 128 + ks * 8, sdesc_sw128(vb + ks * 2048, kA2Half, 1024),
                      id_o, (!first || ks > 0) ? 1u : 0u);
            umma_commit(my_v_empty + st);
            first = false;
            pend = -1;
            return true;
          };
          bool last = false;
          while (!last) {
            const int ks_ = kvseq % kA2KStages, vs = kvseq & 1;
            if (!A2_W(9, A2_MMA_WAIT(k_full + ks_, (kvseq / kA2KStages) & 1, abort))) { ok = false; break; }
            const int m = umask[ks_];
            last = (m & 4) != 0;
            if (pend >= 0 && !issue_pv()) { ok = false; break; }
            if (m & (1 << t)) {
              if (!qw) {
                if (!A2_W(13, A2_MMA_WAIT(q_full + t, qc & 1, abort))) { ok = false; break; }
                ++qc;
                qw = true;
              }
              tc_fence_after();
              const uint32_t qb_ = q_base + t * kA2Tile, kb_ = k_base + ks_ * kA2Tile;
#pragma unroll
              for (int ks = 0; ks < 8; ++ks) {
                const uint32_t off = (ks >> 2) * kA2Half + (ks & 3) * 32;
                umma_ss(tmem + t * 128, sdesc_sw128(qb_ + off, 16, 1024), sdesc_sw128(kb_ + off, 16, 1024), id_s,
                        ks > 0);
              }
              umma_commit(s_full + t);
              if (kA2EarlyQFree && --s_left == 0) umma_commit(q_empty + t);  // the item's last read of Q_t
              pend = (int)kvseq;
            } else {
              // This tile does not use the block's V tile.  It still releases it, but only once
              // the tile has landed: released earlier, a tile that skips many blocks could run
              // a V stage's barrier two phases ahead of the producer waiting on it.
              if (!A2_W(11, A2_MMA_WAIT(v_full + vs, (kvseq >> 1) & 1, abort))) { ok = false; break; }
              umma_commit(my_v_empty + vs);
            }
            umma_commit(my_k_empty + ks_);
            ++kvseq;
          }
          if (!ok) break;
          if (pend >= 0 && !issue_pv()) break;
          if (n_t > 0) {
            umma_commit(o_full + t);
            if (!kA2EarlyQFree) umma_commit(q_empty + t);
          }
        }
      };
      if (warp == 1) run(std::integral_constant<int, 0>{});
      else run(std::integral_constant<int, 1>{});
      umma_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort);
    } else if (kA2PSmem && warp == 1 && lane == 0) {
      // ------------------------------------------------------------ MMA issuer, P in shared memory
      // Two cursors over the item's union blocks, each advanced as soon as its barriers have
      // completed (non-blocking probes, one bounded clock for the whole item):
      //   S cursor:  S_0, S_1 of block s (K(s) loaded; S_t free: the softmax has read S_t), then
      //              k_empty; it runs at most two blocks ahead of the PV cursor;
      //   PV cursor: PV_0, PV_1 of block v < s (P_t written; V(v) loaded; O_t read by the last
      //              epilogue for the item's first PV_t), each followed by a commit to p_grant_t
      //              (P_t may be written again), then v_empty.
      constexpr uint32_t id_s = idesc_f16(128, 128, DT<T>::is_bf16, false);
      constexpr uint32_t id_o = idesc_f16(128, 128, DT<T>::is_bf16, true);
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV), p_base = smem_u32(sStage);
      volatile int* imask = reinterpret_cast<volatile int*>(tmem_slot + 16);  // [block & 3] masks between the cursors
      uint32_t it = 0, kvseq = 0, qc[2] = {0, 0}, pc[2] = {0, 0}, oc[2] = {0, 0}, sf[2] = {0, 0}, ns[2] = {0, 0};
      bool ok = true;
      while (ok) {
        const int slot = it & 1;
        if (!A2_W(16, mbar_wait_sleep(item_full + slot, (it >> 1) & 1, abort))) break;
        const int valid = ring[slot].valid, n0 = ring[slot].n[0], n1 = ring[slot].n[1];
        mbar_arrive(item_empty + slot);
        ++it;
        if (valid == 0) break;
        if (valid != 1 || (n0 == 0 && n1 == 0)) continue;
        const uint32_t base = kvseq;                  // sequence number of the item's first block
        uint32_t sq = base, vq = base, s_end = 0xffffffffu;  // s_end: one past the item's last block
        int s_t = 0, v_t = 0;                         // next tile within the cursor's block
        bool k_ready = false, qw0 = false, qw1 = false, first0 = true, first1 = true;
        int ms = 0;
        const uint64_t lim = g_wait_limit_ns;
        uint64_t t_last = global_timer_ns();
        uint32_t polls = 0;
        while (vq != s_end) {
          bool moved = false;
          // ---- S cursor
          if (sq != s_end && sq - vq < 2) {
            const int ks_ = sq % kA2KStages;
            if (!k_ready && mbar_probe(k_full + ks_, (sq / kA2KStages) & 1)) {
              ms = umask[ks_];
              imask[sq & 3] = ms;
              k_ready = true;
            }
            while (k_ready && s_t < 2) {
              if (!((ms >> s_t) & 1)) { ++s_t; continue; }
              const int t = s_t;
              const bool qready = t ? qw1 : qw0;
              if (!qready) {
                if (!mbar_probe(q_full + t, qc[t] & 1)) break;
                ++qc[t];
                if (t) qw1 = true; else qw0 = true;
              }
              if (ns[t] > 0) {
                if (!mbar_probe(s_free + t, sf[t] & 1)) break;
                ++sf[t];
              }
              ++ns[t];
              tc_fence_after();
              const uint32_t qb_ = q_base + t * kA2Tile, kb_ = k_base + ks_ * kA2Tile;
#pragma unroll
              for (int ks = 0; ks < 8; ++ks) {
                const uint32_t off = (ks >> 2) * kA2Half + (ks & 3) * 32;
                umma_ss(tmem + t * 128, sdesc_sw128(qb_ + off, 16, 1024), sdesc_sw128(kb_ + off, 16, 1024), id_s,
                        ks > 0);
              }
              umma_commit(s_full + t);
              ++s_t;
              moved = true;
            }
            if (k_ready && s_t == 2) {
              umma_commit(k_empty + ks_);
              if (ms & 4) s_end = sq + 1;
              ++sq;
              s_t = 0;
              k_ready = false;
              moved = true;
            }
          }
          // ---- PV cursor
          if (vq != sq) {
            const int mv = imask[vq & 3], st = vq & 1;
            while (v_t < 2) {
              if (!((mv >> v_t) & 1)) { ++v_t; continue; }
              const int t = v_t;
              const bool fst = t ? first1 : first0;
              if (fst && !mbar_probe(o_empty + t, (oc[t] & 1) ^ 1)) break;
              if (!mbar_probe(p_full + t, pc[t] & 1)) break;
              if (!mbar_probe(v_full + st, (vq >> 1) & 1)) break;
              if (fst) ++oc[t];
              ++pc[t];
              tc_fence_after();
              const uint32_t t_o = 256 + t * 128, vb = v_base + st * kA2Tile;
#pragma unroll
              for (int ks = 0; ks < 8; ++ks) {  // A = P_t (shared memory, K-major like Q), B = V (MN-major)
                const uint32_t off = t * kA2Tile + (ks >> 2) * kA2Half + (ks & 3) * 32;
                umma_ss(tmem + t_o, sdesc_sw128(p_base + off, 16, 1024), sdesc_sw128(vb + ks * 2048, kA2Half, 1024),
                        id_o, (!fst || ks > 0) ? 1u : 0u);
              }
              umma_commit(p_grant + t);
              if (t) first1 = false; else first0 = false;
              ++v_t;
              moved = true;
            }
            if (v_t == 2) {
              umma_commit(v_empty + st);  // both of the block's PVs are issued
              ++vq;
              v_t = 0;
              moved = true;
            }
          }
          if (moved) {
            polls = 0;
            t_last = global_timer_ns();
          } else if (++polls % kTimerEvery == 0) {
            if (*abort || global_timer_ns() - t_last > lim) {
              *abort = 1;
              ok = false;
              break;
            }
          }
        }
        kvseq = sq;
        if (!ok) break;
        if (n0 > 0) {
          umma_commit(o_full);
          umma_commit(q_empty);
        }
        if (n1 > 0) {
          umma_commit(o_full + 1);
          umma_commit(q_empty + 1);
        }
      }
      umma_commit(mma_done);
      volatile int no_abort = 0;
      mbar_wait(mma_done, 0, &no_abort);
    } else if (kA2Issuers == 1 && !kA2PSmem && warp == 1 && lane == 0) {
      // ------------------------------------------------------------ MMA issuer
      constexpr uint32_t id_s = idesc_f16(128, 128, DT<T>::is_bf16, false);
      constexpr uint32_t id_o = idesc_f16(128, 128, DT<T>::is_bf16, true);
      const uint32_t q_base = smem_u32(sQ), k_base = smem_u32(sK), v_base = smem_u32(sV);
      // Per-tile state is indexed only by compile-time tile numbers (generic lambdas over
      // std::integral_constant) and per-stage counters are two scalars, so nothing of it lives
      // in local memory.
      uint32_t it = 0, kvseq = 0, qc[2] = {0, 0}, pc[2] = {0, 0}, oc[2] = {0, 0};
      uint32_t pi = 0, qcx0 = 0, qcx1 = 0;  // FPB_A2_QROT: items started, waits per Q_0 buffer
      int users0 = 0, users1 = 0;  // PVs still to be issued on the V tile of stage 0 / 1
      using T0 = std::integral_constant<int, 0>;
      using T1 = std::integral_constant<int, 1>;
      bool ok = true;
      while (ok) {
        const int slot = it & 1;
        if (!A2_W(16, mbar_wait_sleep(item_full + slot, (it >> 1) & 1, abort))) break;
        const int valid = ring[slot].valid, n0 = ring[slot].n[0], n1 = ring[slot].n[1];
        mbar_arrive(item_empty + slot);
        ++it;
        if (valid == 0) break;
        if (valid != 1 || (n0 == 0 && n1 == 0)) continue;
        int pend[2] = {-1, -1};  // union sequence number of the block whose PV is due
        bool first[2] = {true, true}, qw[2] = {false, false};
        int s_left[2] = {n0, n1};  // S MMAs still to issue per tile; Q_t is free after the last
        const int xs = pi & 1;     // FPB_A2_QROT: this item's Q_0 buffer
        auto issue_pv = [&](auto tt) -> bool {
          constexpr int t = decltype(tt)::value;
          const int q = pend[t], st = q & 1;
          if (first[t]) {  // the previous item's epilogue must have read O_t
            if (!A2_W(12, A2_MMA_WAIT(o_empty + t, (oc[t] & 1) ^ 1, abort))) return false;
            ++oc[t];
          }
          A2_EV(3, t);
          if (!A2_W(10, A2_MMA_WAIT(p_full + t, pc[t] & 1, abort))) return false;
          ++pc[t];
          if (!A2_W(11, A2_MMA_WAIT(v_full + st, (q >> 1) & 1, abort))) return false;
          A2_EV(11, t);
          tc_fence_after();
          constexpr uint32_t t_s = t * 128, t_o = 256 + t * 128;
          const uint32_t vb = v_base + st * kA2Tile;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks)  // A = P (TMEM, 8 packed columns per 16 keys), B = V (MN-major)
            umma_ts(tmem + t_o, tmem + t_s + ks * 8, sdesc_sw128(vb + ks * 2048, kA2Half, 1024), id_o,
                    (!first[t] || ks > 0) ? 1u : 0u);
          A2_EV(2, t);
          first[t] = false;
          if (st == 0) {
            if (--users0 == 0) umma_commit(v_empty);
          } else {
            if (--users1 == 0) umma_commit(v_empty + 1);
          }
          pend[t] = -1;
          return true;
        };
        auto issue_s = [&](auto tt, int st) -> bool {
          constexpr int t = decltype(tt)::value;
          if (!qw[t]) {
            if (kA2QRot && t == 0) {
              if (!A2_W(13, A2_MMA_WAIT(q_full + xs, (xs ? qcx1 : qcx0) & 1, abort))) return false;
              if (xs) ++qcx1; else ++qcx0;
            } else {
              if (!A2_W(13, A2_MMA_WAIT(kA2QRot ? q_full_b : q_full + t, qc[t] & 1, abort))) return false;
              ++qc[t];
            }
            qw[t] = true;
          }
          tc_fence_after();
          A2_EV(13, t);
          const uint32_t qb_ = q_base + (kA2QRot ? (t ? 2 : xs) : t) * kA2Tile, kb_ = k_base + st * kA2Tile;
#pragma unroll
          for (int ks = 0; ks < 8; ++ks) {
            const uint32_t off = (ks >> 2) * kA2Half + (ks & 3) * 32;
            umma_ss(tmem + t * 128, sdesc_sw128(qb_ + off, 16, 1024), sdesc_sw128(kb_ + off, 16, 1024), id_s,
                    ks > 0);
          }
          umma_commit(s_full + t);
          A2_EV(1, (t << 16) | (kvseq & 0xffff));
          // the item's last read of Q_t: the next item's Q_t may load while this one finishes
          if (kA2EarlyQFree && --s_left[t] == 0) umma_commit(q_empty + t);
          pend[t] = (int)kvseq;
          return true;
        };
        bool last = false;
        while (!last && ok) {
          const int ks_ = kvseq % kA2KStages, st = kvseq & 1;  // K stage, V stage of this union block
          A2_EV(9, kvseq);
          if (!A2_W(9, A2_MMA_WAIT(k_full + ks_, (kvseq / kA2KStages) & 1, abort))) { ok = false; break; }
          A2_EV(10, kvseq);
          A2_ADD(14, 1);
          const int m = umask[ks_];
          last = (m & 4) != 0;
          // tile 0: PV of its previous block, then S of this one; then the same for tile 1
          if (pend[0] >= 0 && !issue_pv(T0{})) { ok = false; break; }
          if ((m & 1) && !issue_s(T0{}, ks_)) { ok = false; break; }
          if (pend[1] >= 0 && !issue_pv(T1{})) { ok = false; break; }
          if ((m & 2) && !issue_s(T1{}, ks_)) { ok = false; break; }
          umma_commit(k_empty + ks_);
          if (st == 0) users0 = __popc(m & 3); else users1 = __popc(m & 3);
          ++kvseq;
        }
        if (!ok) break;
        if (pend[0] >= 0 && !issue_pv(T0{})) break;
        if (pend[1] >= 0 && !issue_pv(T1{})) break;
        if (n0 > 0) {
          umma_commit(o_full);
          if (!kA2EarlyQFree && !kA2QRot) umma_commit(q_empty);
        }
        if (n1 > 0) {
          umma_commit(o_full + 1);
          if (!kA2EarlyQFree) umma_commit(q_empty + 1);
        }
        ++pi;
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
    uint32_t it = 0, sc = 0, oc = 0, ep = 0, pw = 0;
    uint32_t ps = 0;  // FPB_A2_QROT: items started (the issuer works on them)
    // a tile's per-row event: every thread's arrival, or (FPB_A2_WARP_ARRIVE) the warp's, once all
    // its lanes are past their fences
    auto row_arrive = [&](uint64_t* bar) {
      if (kA2RowArrivals == 128) {
        mbar_arrive(bar);
      } else {
        __syncwarp();
        if (lane == 0) mbar_arrive(bar);
      }
    };
    auto group_sync = [&]() -> bool {  // the tile's 128 softmax threads, bounded
      mbar_arrive(epi + t);
      return A2_W(22, mbar_wait_warp_sleep(epi + t, (ep++) & 1, abort));
    };
    while (true) {
      const int slot = it & 1;
      if (!A2_W(23, mbar_wait_warp_sleep(item_full + slot, (it >> 1) & 1, abort))) break;
      // this tile's fields as scalars (a struct indexed by the runtime tile would live in local memory)
      const Item2* fp = ring + slot;
      const int valid = fp->valid, h_t = fp->h[t], n = fp->n[t], diag_t = fp->diag[t], nfull_t = fp->nfull[t];
      const int start = fp->start, len = fp->len, bcoord = fp->bcoord, qbk = fp->qb, chunk = fp->chunk;
      // FPB_A2_QROT: every softmax thread reports once per item the issuer works on that it is
      // done with it (its epilogue staged rows in the item's Q_0 buffer)
      const bool issued = valid == 1 && (fp->n[0] > 0 || fp->n[1] > 0);
      uint8_t* const stage_base = kA2QRot ? sQ + (ps & 1) * kA2Tile : sStage;
      auto item_end = [&]() {
        if (kA2QRot && issued) {
          mbar_arrive(stg_done + (ps & 1));
          ++ps;
        }
      };
      mbar_arrive(item_empty + slot);
      ++it;
      if (valid == 0) break;
      if (valid != 1 || h_t < 0) {
        item_end();
        continue;
      }
      // rows this thread may write: inside the sequence and (chunked prefill) at or after q_off
      const int vr = min(kBlock, len - qbk * kBlock);
      const bool row_out = r < vr && qbk * kBlock + r >= A.P.q_off;
      T* orow = reinterpret_cast<T*>(A.out) + (int64_t)bcoord * A.o_sb +
                (int64_t)(start + qbk * kBlock + r - A.P.q_off) * A.o_ss + (int64_t)h_t * A.o_sh;
      if (n == 0) {  // empty list: zeros (the reference's acc = 0, l = 1); a chunk item only
                     // writes them for a row with no blocks at all, in its first chunk
        const bool zero_row = row_out && (chunk < 0 || (nfull_t == 0 && ((chunk >> 17) & 127) == 0));
        if (zero_row) {
          uint4* dst = reinterpret_cast<uint4*>(orow);
#pragma unroll
          for (int i = 0; i < 16; ++i) dst[i] = make_uint4(0, 0, 0, 0);
        }
        if constexpr (kPeers) warp_rows_to_peers<T>(A, orow, zero_row);
        item_end();
        continue;
      }
      float m_use = -INFINITY, l = 0.f;
      bool ok = true;
      for (int j = 0; j < n; ++j) {
        if (!A2_W(0, A2_SM_WAIT(s_full + t, sc & 1, abort))) { ok = false; break; }
        ++sc;
        tc_fence_after();
        const unsigned long long tp0 = A2_CLK();
        (void)tp0;
        A2_EV(5, (t << 16) | j);
        if (FPB_A2_TIMING_NOSOFTMAX) {  // timing experiment only: P = whatever S holds
          tc_fence_before();
          row_arrive(p_full + t);
          l = 1.f;
          continue;
        }
        uint32_t u[128];
        tmem_ld32(t_s, *reinterpret_cast<uint32_t(*)[32]>(u));
        tmem_ld32(t_s + 32, *reinterpret_cast<uint32_t(*)[32]>(u + 32));
        tmem_ld32(t_s + 64, *reinterpret_cast<uint32_t(*)[32]>(u + 64));
        tmem_ld32(t_s + 96, *reinterpret_cast<uint32_t(*)[32]>(u + 96));
        tmem_ld_wait();
        if (kA2PSmem) {  // S_t is in registers: the next S_t may be issued
          tc_fence_before();
          row_arrive(s_free + t);
        }
        const unsigned long long tp1 = A2_CLK();
        (void)tp1;
        A2_ADD(1, tp1 - tp0);
        if (diag_t && j == n - 1) {  // only the diagonal block needs the causal mask
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
        const unsigned long long tp2 = A2_CLK();
        (void)tp2;
        A2_ADD(2, tp2 - tp1);
        const float neg_m = -m_use;
        float rs0 = 0.f, rs1 = 0.f;
#if FPB_A2_TURNS == 1
        // Turn taking per SM sub-partition (Peterson's two-party lock): the exp passes of this
        // warp and of the other tile's warp on the same sub-partition alternate.
        if (lane == 0) {
          pp_want[t * 4 + quad] = 1;
          pp_turn[quad] = 1 - t;
          __threadfence_block();
          const uint64_t tw0 = global_timer_ns();
          while (pp_want[(1 - t) * 4 + quad] && pp_turn[quad] == 1 - t)
            if (global_timer_ns() - tw0 > 4000) break;
        }
        __syncwarp();
#elif FPB_A2_TURNS == 2
        // Turn taking per tile: a warp starts its exp pass when no warp of the other tile wants
        // one, or when it is this tile's turn; the last of this tile's four warps to finish hands
        // the turn over.  All four warps of a tile follow one order, so the tiles' exp passes
        // alternate as wholes.  It only orders work: after a bounded wait the pass goes ahead.
        if (lane == 0) {
          pp_want[t * 4 + quad] = 1;
          __threadfence_block();
          const uint64_t tw0 = global_timer_ns();
          while (pp_turn[0] != t && (pp_want[(1 - t) * 4] | pp_want[(1 - t) * 4 + 1] | pp_want[(1 - t) * 4 + 2] |
                                     pp_want[(1 - t) * 4 + 3]))
            if (global_timer_ns() - tw0 > 4000) break;
        }
        __syncwarp();
#endif
        // packed pair k overwrites u[k] (u[2k] and u[2k+1] are read first), so no second array
#pragma unroll
        for (int k = 0; k < 64; ++k) {
          float x0, x1, p0, p1;
          fma2(x0, x1, __uint_as_float(u[2 * k]), __uint_as_float(u[2 * k + 1]), c, c, neg_m, neg_m);
          if (FPB_A2_TIMING_NOEXP) {  // timing experiment only: wrong results
            p0 = x0;
            p1 = x1;
          } else if ((k % kA2PolyEvery) == kA2PolyEvery - 1) {
            exp2_poly2(x0, x1, p0, p1);  // masked (-inf) entries give 2^-126 here, negligible
          } else {
            p0 = ex2_approx(x0);
            p1 = ex2_approx(x1);
          }
          add2(rs0, rs1, rs0, rs1, p0, p1);
          u[k] = DT<T>::pack(p0, p1);
        }
#if FPB_A2_TURNS == 1
        __syncwarp();
        if (lane == 0) {
          __threadfence_block();
          pp_want[t * 4 + quad] = 0;
        }
#elif FPB_A2_TURNS == 2
        __syncwarp();
        if (lane == 0) {
          __threadfence_block();
          pp_want[t * 4 + quad] = 0;
          if (atomicAdd(const_cast<int*>(pp_turn) + 1 + t, 1) % 4 == 3) pp_turn[0] = 1 - t;  // last of 4 warps
        }
#endif
        if (kA2PSmem) {
          // P_t may be written once its last PV has read it (p_grant_t; the first write of the
          // launch has none before it).  Row r in the TMA layout of a K-major 128-byte-swizzled
          // tile: keys [64h, 64h+64) at h * 16 KB + r * 128, 16-byte piece c at (c ^ (r & 7)) * 16
          if (pw > 0 && !A2_W(5, mbar_wait_warp(p_grant + t, (pw - 1) & 1, abort))) { ok = false; break; }
          ++pw;
          uint4* prow = reinterpret_cast<uint4*>(sStage + t * kA2Tile + r * 128);
#pragma unroll
          for (int c16 = 0; c16 < 16; ++c16)
            prow[(c16 >> 3) * (kA2Half / 16) + ((c16 & 7) ^ (r & 7))] =
                make_uint4(u[4 * c16], u[4 * c16 + 1], u[4 * c16 + 2], u[4 * c16 + 3]);
        } else {
          tmem_st32(t_s, *reinterpret_cast<uint32_t(*)[32]>(u));
          tmem_st32(t_s + 32, *reinterpret_cast<uint32_t(*)[32]>(u + 32));
        }
        const unsigned long long tp3 = A2_CLK();
        (void)tp3;
        A2_ADD(3, tp3 - tp2);
        A2_ADD(6, 1);
        if (!FPB_A2_TIMING_NORESCALE && __any_sync(0xffffffffu, scale_o != 1.f)) {
          A2_ADD(7, 1);
          // O_t holds the blocks before this one (PV_t(previous) completed before S_t(this)
          // did); rescale this row before PV_t(this) may start (p_full below).  u[64..127]
          // are free (their S values are packed into u[0..63], which the P stores still read).
#pragma unroll
          for (int hh = 0; hh < 2; ++hh) {
            tmem_ld32(t_o + hh * 64, *reinterpret_cast<uint32_t(*)[32]>(u + 64));
            tmem_ld32(t_o + hh * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(u + 96));
            tmem_ld_wait();
#pragma unroll
            for (int i = 64; i < 128; i += 2) {
              float a0, a1;
              fma2(a0, a1, __uint_as_float(u[i]), __uint_as_float(u[i + 1]), scale_o, scale_o, 0.f, 0.f);
              u[i] = __float_as_uint(a0);
              u[i + 1] = __float_as_uint(a1);
            }
            tmem_st32(t_o + hh * 64, *reinterpret_cast<uint32_t(*)[32]>(u + 64));
            tmem_st32(t_o + hh * 64 + 32, *reinterpret_cast<uint32_t(*)[32]>(u + 96));
            if (hh == 0) tmem_st_wait();  // the second half reloads into the same registers
          }
        }
        const unsigned long long tp4 = A2_CLK();
        (void)tp4;
        A2_ADD(4, tp4 - tp3);
        tmem_st_wait();
        l += rs0 + rs1;
        if (kA2PSmem) fence_proxy_async_smem();  // P (generic-proxy stores) visible to the MMA
        tc_fence_before();
        row_arrive(p_full + t);
        A2_EV(6, (t << 16) | j);
        A2_ADD(5, A2_CLK() - tp4);
      }
      if (!ok) break;
      // ---- epilogue: O / l straight from TMEM to this thread's output row
      if (!A2_W(8, mbar_wait_warp_sleep(o_full + t, oc & 1, abort))) break;
      ++oc;
      tc_fence_after();
      const unsigned long long te0 = A2_CLK();
      (void)te0;
      uint32_t o[128];
      tmem_ld32(t_o, *reinterpret_cast<uint32_t(*)[32]>(o));
      tmem_ld32(t_o + 32, *reinterpret_cast<uint32_t(*)[32]>(o + 32));
      tmem_ld32(t_o + 64, *reinterpret_cast<uint32_t(*)[32]>(o + 64));
      tmem_ld32(t_o + 96, *reinterpret_cast<uint32_t(*)[32]>(o + 96));
      tmem_ld_wait();
      tc_fence_before();
      row_arrive(o_empty + t);  // O_t may be overwritten by the next item's first PV
      if (chunk >= 0) {  // a chunk of a split row: store the partial, the row's last chunk merges
        const int code = chunk;
        const int entry = code & (kSplitMaxEntries - 1), cix = (code >> 17) & 127;
        const int e0 = entry - cix, nch = (nfull_t + kSplitChunk - 1) / kSplitChunk;
        constexpr int64_t kStride = 2 * (kSplitPartBytes / 4);  // floats between a tile's chunk partials
        float* part = A.sp_part + (int64_t)entry * kStride + t * (kSplitPartBytes / 4);
        float4* po = reinterpret_cast<float4*>(part + r * 128);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          po[i] = make_float4(__uint_as_float(o[4 * i]), __uint_as_float(o[4 * i + 1]), __uint_as_float(o[4 * i + 2]),
                              __uint_as_float(o[4 * i + 3]));
        part[128 * 128 + r] = m_use;
        part[128 * 128 + 128 + r] = l;
        part[128 * 128 + 256 + r] = 0.f;
        __threadfence();
        if (!group_sync()) break;
        if (r == 0) last_chunk[t] = atomicAdd(A.sp_counters + 2 * e0 + t, 1) == nch - 1;
        if (!group_sync()) break;
        if (last_chunk[t]) {  // the same for every thread of the tile
          if (row_out) {
            __threadfence();
            T* oblk = orow - (int64_t)r * A.o_ss;
            const float* p0 = A.sp_part + (int64_t)e0 * kStride + t * (kSplitPartBytes / 4);
            split_merge_row<T>(p0, nch, r, 0, vr, oblk, A.o_ss, kStride);
            split_merge_row<T>(p0, nch, r, 1, vr, oblk, A.o_ss, kStride);
          }
          if constexpr (kPeers) warp_rows_to_peers<T>(A, orow, row_out);  // the merged rows, sent on
        }
        A2_ADD(21, A2_CLK() - te0);
        item_end();
        continue;
      }
      const float inv = 1.f / l;
      if (kA2StageBytes > 0 || kA2QRot) {
        // lane = row; half h of the 32 rows goes through shared memory (piece q of a row at slot
        // q ^ (row & 7), conflict-free both ways), then out four rows per store instruction
        const uint64_t pol = l2_policy_evict_first();
        // tile t's warps use [t * half, (t + 1) * half) of the area (with P in shared memory:
        // of P_t, which its last PV has read: o_full_t is committed after it)
        uint4* stg = reinterpret_cast<uint4*>(stage_base + t * (kA2PSmem ? kA2Tile : kA2Tile / 2)) + quad * 256;
        const unsigned vmask = __ballot_sync(0xffffffffu, row_out);
        const long long mine = reinterpret_cast<long long>(orow);
        long long rows[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) rows[i] = __shfl_sync(0xffffffffu, mine, 4 * i + (lane >> 3));
#pragma unroll
        for (int h = 0; h < 2; ++h) {
#pragma unroll
          for (int q = 0; q < 8; ++q) {
            const int q4 = h * 8 + q;
            uint32_t pk[4];
#pragma unroll
            for (int i = 0; i < 4; ++i)
              pk[i] = DT<T>::pack(__uint_as_float(o[q4 * 8 + 2 * i]) * inv, __uint_as_float(o[q4 * 8 + 2 * i + 1]) * inv);
            stg[lane * 8 + (q ^ (lane & 7))] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int rr = 4 * i + (lane >> 3), pc = lane & 7;
            if ((vmask >> rr) & 1u)
              st_global_hint(reinterpret_cast<uint4*>(rows[i]) + h * 8 + pc, stg[rr * 8 + (pc ^ (rr & 7))], pol);
          }
          __syncwarp();
        }
      } else if (row_out) {
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
      if constexpr (kPeers) warp_rows_to_peers<T>(A, orow, row_out);
      A2_ADD(21, A2_CLK() - te0);
      item_end();
    }
  }

  A2_ADD(15, A2_CLK() - t_kernel0);
  tc_fence_before();
  __syncthreads();
#if FPB_ATTN_PROFILE
  if (A.profile && threadIdx.x < kA2ProfSlots) atomicAdd(&g_attn2_prof[threadIdx.x], prof_sm[threadIdx.x]);
  if (A.trace && blockIdx.x == 0 && threadIdx.x == 0) g_attn2_trace_n = *trace_ctr;
#endif
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, 512);
  }
  if constexpr (kPeers) __threadfence_system();  // peer stores ordered before what follows
  if (threadIdx.x == 0 && *abort) raise_error(A.P.err, kErrWaitTimeout);
}

}  // namespace fpb
