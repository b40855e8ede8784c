// Pooled keys (mean of each 128-token key block) and the varlen prep kernel.
//
// Reference: ops/flashprefill_native_forward.py:22-67 (compute_mean_vector) and
// ops/flashprefill_varlen_func.py:35-85 (compute_mean_vector_varlen): the block sum is
// formed in the INPUT dtype and divided by the number of valid rows, and the result is
// stored in the input dtype.  Because every partial sum rounds to 16 bits, the order of
// the additions decides the low bits of the mean, and those bits move blocks across the
// selection threshold.  This kernel reproduces the order of Triton's reduction of a
// 128x128 16-bit tile with W warps: thread (w, l, column group) adds rows
// rep*2W + 2w + l sequentially, lane pairs l=0/1 are combined, then the W warp partials
// are combined by xor shuffles of distance W/2, ..., 1.  W = 4 or 8 (the reference's
// autotuner picks one of the two).
//
// HBM-bound: reads S*Hk*D*2 bytes once with 16-byte loads, writes NB*Hk*D*2 bytes.
#include "fp_common.cuh"

namespace fpb {

// Fills cu_tile = [0, cumsum(ceil(len_i/128))] (reference varlen:8-18) and validates
// cu_seqlens on the device (no host synchronisation).  One CTA of 1024 threads.
__global__ void varlen_prep_kernel(const int* __restrict__ cu_seqlens, int nseq, int total_tokens, int cap,
                                   int* __restrict__ cu_tile, uint32_t* err) {
  __shared__ int warp_sums[32];
  __shared__ int carry;
  if (threadIdx.x == 0) carry = 0;
  __syncthreads();
  for (int base = 0; base < nseq; base += blockDim.x) {
    const int i = base + threadIdx.x;
    int nb = 0;
    if (i < nseq) {
      const int a = cu_seqlens[i], b = cu_seqlens[i + 1];
      int len = b - a;
      if (len < 0 || a < 0 || b > total_tokens) {
        raise_error(err, kErrBadSeqlens);
        len = 0;
      }
      nb = (len + kBlock - 1) / kBlock;
      if (nb > cap) raise_error(err, kErrSeqTooLong);
    }
    // block-wide inclusive scan of nb
    int v = nb;
    const int lane = threadIdx.x & 31, wid = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
      const int t = __shfl_up_sync(0xffffffffu, v, o);
      if (lane >= o) v += t;
    }
    if (lane == 31) warp_sums[wid] = v;
    __syncthreads();
    if (wid == 0) {
      int w = (lane < (int)(blockDim.x >> 5)) ? warp_sums[lane] : 0;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int t = __shfl_up_sync(0xffffffffu, w, o);
        if (lane >= o) w += t;
      }
      warp_sums[lane] = w;
    }
    __syncthreads();
    const int incl = v + (wid > 0 ? warp_sums[wid - 1] : 0) + carry;
    if (i < nseq) cu_tile[i + 1] = incl;
    __syncthreads();
    if (threadIdx.x == blockDim.x - 1) carry = incl;
    __syncthreads();
  }
  if (threadIdx.x == 0) {
    cu_tile[0] = 0;
    if (cu_seqlens[0] != 0 || cu_seqlens[nseq] != total_tokens) raise_error(err, kErrBadSeqlens);
  }
}

template <typename T, int W>
__global__ void __launch_bounds__(W * 32) block_mean_kernel(const T* __restrict__ k, int64_t sb, int64_t ss,
                                                            int64_t sh, T* __restrict__ mk, SeqProblem P) {
  SeqInfo s;
  int kb;
  if (!decode_block(P, blockIdx.x, s, kb)) return;
  const int hk = blockIdx.y;
  const int t = threadIdx.x, w = t >> 5, l = (t >> 4) & 1, cg = t & 15;
  const int n_valid = min(kBlock, s.len - kb * kBlock);
  const T* base = k + (int64_t)s.bcoord * sb + (int64_t)(s.start + kb * kBlock) * ss + (int64_t)hk * sh + cg * 8;
  constexpr int REPS = kBlock / (2 * W);
  float acc[8];
#pragma unroll
  for (int rep = 0; rep < REPS; ++rep) {
    const int row = rep * 2 * W + 2 * w + l;
    uint4 raw = make_uint4(0, 0, 0, 0);
    if (row < n_valid) raw = __ldg(reinterpret_cast<const uint4*>(base + (int64_t)row * ss));
    const T* x = reinterpret_cast<const T*>(&raw);
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float xv = DT<T>::to_f(x[i]);
      acc[i] = rep == 0 ? xv : DT<T>::to_f(DT<T>::from_f(acc[i] + xv));
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const float o = __shfl_xor_sync(0xffffffffu, acc[i], 16);
    acc[i] = DT<T>::to_f(DT<T>::from_f(acc[i] + o));
  }
  __shared__ float part[W][kHeadDim];
  if (l == 0) {
#pragma unroll
    for (int i = 0; i < 8; ++i) part[w][cg * 8 + i] = acc[i];
  }
  __syncthreads();
  if (t < kHeadDim) {
    float v[W];
#pragma unroll
    for (int j = 0; j < W; ++j) v[j] = part[j][t];
#pragma unroll
    for (int n = W / 2; n >= 1; n >>= 1) {
      float nv[W];
#pragma unroll
      for (int j = 0; j < W; ++j) nv[j] = DT<T>::to_f(DT<T>::from_f(v[j] + v[j ^ n]));
#pragma unroll
      for (int j = 0; j < W; ++j) v[j] = nv[j];
    }
    const float mean = n_valid > 0 ? __fdiv_rn(v[0], (float)n_valid) : 0.f;
    mk[((int64_t)(s.tile_base + kb) * P.hk + hk) * kHeadDim + t] = DT<T>::from_f(mean);
  }
}

}  // namespace fpb
