// Dense prefill that allocates nothing: for callers that cannot call cudaMalloc or hand
// over a workspace -- code running inside a CUDA-graph-managed or custom-allocator
// runtime that forbids allocation on its hot path, or plain C hosts without an allocator
// of their own.  The workspace (error word, pooled keys, block counts and lists) lives in
// one file-scope device array of fixed size instead.
//
// The array is part of the library's device image, so every GPU that loads the library
// holds kNoAllocScratchBytes until the process exits.  In host code its name is only a
// host-side stand-in: its device address is fetched with cudaGetSymbolAddress, once per
// device, on the first call made with that device current (so make that first call
// before any stream capture).  All calls share the array and it keeps the last call's
// contents; the error word is cleared at the start of each call and every list entry a
// call reads is written by that call.  Calls that overlap on the GPU (different streams
// or threads, same device) race on the array.
#include <mutex>

namespace fpb {

constexpr size_t kNoAllocScratchBytes = size_t(32) << 20;  // 32 MiB
constexpr int kNoAllocMaxDevices = 64;

static __device__ __align__(256) uint8_t g_noalloc_scratch[kNoAllocScratchBytes];

namespace {
std::mutex g_noalloc_mu;
void* g_noalloc_ptr[kNoAllocMaxDevices] = {};

// Device address of g_noalloc_scratch on the current device (looked up once per device).
int noalloc_scratch(void** out) {
  int dev = -1;
  FPB_CUDA(cudaGetDevice(&dev));
  FPB_CHECK_ARG(dev >= 0 && dev < kNoAllocMaxDevices, "device %d out of range for the no-allocation path", dev);
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(FPB_ECUDA, "cudaGetSymbolAddress(no-allocation scratch) failed on device %d: %s", dev,
                  cudaGetErrorString(e));
    g_noalloc_ptr[dev] = p;
  }
  *out = g_noalloc_ptr[dev];
  return FPB_OK;
}
}  // namespace
}  // namespace fpb

extern "C" int fpb_noalloc_read_device_error(uint32_t* flags, void* stream) {
  using namespace fpb;
  FPB_CHECK_ARG(flags != nullptr, "flags is NULL");
  void* ws = nullptr;
  FPB_TRY(noalloc_scratch(&ws));
  return fpb_read_device_error(ws, flags, stream);
}

extern "C" int fpb_prefill_dense_noalloc(const void* q, const void* k, const void* v, void* out, int dtype,
                                         int batch, int seqlen, int hq, int hk, int head_dim,
                                         const int64_t* q_strides, const int64_t* k_strides,
                                         const int64_t* v_strides, const int64_t* o_strides, int block_size,
                                         int attention_sink, int window_size, float alpha, int last_n_block_full,
                                         int min_budget, int mean_model, void* stream) {
  using namespace fpb;
  FPB_CHECK_ARG(batch >= 1 && seqlen >= 1 && hq >= 1 && hk >= 1, "batch, seqlen and head counts must be >= 1");
  FPB_TRY(check_dense(q, k, dtype, batch, seqlen, hq, hk, head_dim, q_strides, k_strides, block_size));
  const Layout L = make_layout(0, batch, seqlen, 0, hq, hk);
  // the required part of the workspace must fit; the optional long-row split area is used
  // only where it fits as well
  FPB_CHECK_ARG((size_t)L.base_total <= kNoAllocScratchBytes,
                "problem needs %lld bytes of scratch; the no-allocation path holds at most %zu (32 MiB) -- use "
                "fpb_prefill_dense with a caller workspace", (long long)L.base_total, kNoAllocScratchBytes);
  void* ws = nullptr;
  FPB_TRY(noalloc_scratch(&ws));
  return fpb_prefill_dense(q, k, v, out, dtype, batch, seqlen, hq, hk, head_dim, q_strides, k_strides, v_strides,
                           o_strides, block_size, attention_sink, window_size, alpha, last_n_block_full, min_budget,
                           mean_model, ws, kNoAllocScratchBytes, stream);
}
