/* flashprefill_b200 -- C ABI of the B200 (sm_100a) sparse-prefill operator.
 *
 * The library replaces the device work behind the two public entry points of
 * FlashPrefill (qhfan/FlashPrefill, paths relative to that project):
 *   ops/flashprefill_native_forward.py:481-499  flash_prefill(q, k, v, out, block_size,
 *       attention_sink, window_size, alpha, last_n_block_full, min_budget)
 *   ops/flashprefill_varlen_func.py:723-743     flash_prefill_varlen_func(q, k, v, o,
 *       cu_seqlens, max_seq_len, alpha, block_size, attention_sink, window_size, last_n_block)
 * Those Python functions launch Triton kernels; here the same work is three CUDA kernels
 * (pooled keys, fused block search, tcgen05 block-sparse attention).  All pointers are
 * device pointers unless stated; all calls are asynchronous on `stream` (a cudaStream_t,
 * NULL = legacy default stream) and never synchronise the host, except
 * fpb_read_device_error.  Return value: FPB_OK or an FPB_E* code; fpb_last_error()
 * describes the most recent failure of the calling thread.
 *
 * Tensor layout: dense q/k/v/out are (batch, seq, heads, 128) with the last dimension
 * contiguous and strides given in ELEMENTS as {batch, seq, head}; varlen tensors are
 * (tokens, heads, 128) with strides {token, head}.  Strides must be multiples of 8
 * elements (16 bytes) and base pointers 16-byte aligned.  dtype: FPB_BF16 or FPB_FP16;
 * q, k, v and out share it.  head_dim and block_size must be 128.
 *
 * Workspace: the caller provides `workspace` of at least the size returned by the
 * matching *_workspace_bytes function (the reference allocates its temporaries from the
 * PyTorch caching allocator, native:419-434 / varlen:596-663; here they are one caller
 * buffer).  It holds the device error word, cu_tile, the pooled keys, and the per-head
 * block lists.  Its layout is reported by fpb_workspace_layout.
 */
#ifndef FLASHPREFILL_B200_H
#define FLASHPREFILL_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define FPB_API __attribute__((visibility("default")))
#else
#define FPB_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

#define FPB_OK 0
#define FPB_EINVAL 1   /* invalid argument (shape, dtype, stride, alignment, size) */
#define FPB_ECUDA 2    /* a CUDA runtime/driver call or a kernel launch failed */
#define FPB_EDEVICE 3  /* fpb_read_device_error found error bits set */

#define FPB_BF16 0
#define FPB_FP16 1

/* Device error bits (fpb_read_device_error). */
#define FPB_DEV_WAIT_TIMEOUT 1u   /* a pipeline wait ran out of time; the kernel bailed out */
#define FPB_DEV_BAD_SEQLENS 2u    /* cu_seqlens not non-decreasing from 0 to total_tokens */
#define FPB_DEV_SEQ_TOO_LONG 4u   /* a sequence longer than max_seq_len (rows skipped) */
#define FPB_DEV_INDEX_RANGE 8u    /* a block list held an index outside [0, query block] */

/* Library version (major*10000 + minor*100 + patch). */
FPB_API int fpb_version(void);

/* Message for the last failing call on this thread ("" if none). */
FPB_API const char* fpb_last_error(void);

/* Workspace size for the dense entry points (replaces the temporaries of
 * ops/flashprefill_native_forward.py:419-434 and deal_output_score's outputs :379-385). */
FPB_API size_t fpb_dense_workspace_bytes(int batch, int seqlen, int hq, int hk, int head_dim);

/* Workspace size for the varlen entry points (replaces
 * ops/flashprefill_varlen_func.py:596-698).  Sized from host-known bounds only, so no
 * device->host copy of cu_seqlens is needed. */
FPB_API size_t fpb_varlen_workspace_bytes(int total_tokens, int nseq, int max_seq_len, int hq, int hk,
                                          int head_dim);

/* Byte offsets inside the workspace.  out[8] = {error word, cu_tile (int32[nseq+1]),
 * pooled keys (dtype[tiles][hk][128]), counts (int32[hq][tiles]), block lists
 * (int32[hq][tiles][cap]), total bytes, tiles, cap}.  Row `tile_base(seq)+qb` of head h:
 * counts[h*tiles + row] entries at lists[(h*tiles + row)*cap ...], ascending.
 * varlen = 0: a = batch, b = seqlen, c ignored.  varlen = 1: a = nseq, b = total_tokens,
 * c = max_seq_len.  (The reference keeps the same information as block_index/counts,
 * native:377-385, or out_index/out_number_cu, varlen:683-698.) */
FPB_API int fpb_workspace_layout(int varlen, int a, int b, int c, int hq, int hk, int head_dim, int64_t* out8);

/* Whole operator, dense layout: replaces FlashPrefill.forward
 * (ops/flashprefill_native_forward.py:405-476).  Writes out in place.
 * mean_model: 4 or 8, the warp count whose reduction order the pooled-key sum follows
 * (the reference autotunes it, native:7-20). */
FPB_API int fpb_prefill_dense(const void* q, const void* k, const void* v, void* out, int dtype, int batch,
                              int seqlen, int hq, int hk, int head_dim, const int64_t* q_strides,
                              const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                              int block_size, int attention_sink, int window_size, float alpha,
                              int last_n_block_full, int min_budget, int mean_model, void* workspace,
                              size_t workspace_bytes, void* stream);

/* Whole operator, packed varlen layout: replaces FlashPrefill_varlen.forward
 * (ops/flashprefill_varlen_func.py:577-720).  cu_seqlens: device int32[nseq+1]. */
FPB_API int fpb_prefill_varlen(const void* q, const void* k, const void* v, void* o, int dtype,
                               const int32_t* cu_seqlens, int nseq, int total_tokens, int max_seq_len, int hq,
                               int hk, int head_dim, const int64_t* q_strides, const int64_t* k_strides,
                               const int64_t* v_strides, const int64_t* o_strides, int block_size,
                               int attention_sink, int window_size, float alpha, int last_n_block, int mean_model,
                               void* workspace, size_t workspace_bytes, void* stream);

/* fpb_prefill_dense for one rank of a head-sharded layer that also needs the full output on
 * every GPU (the gather of head shards; the reference has no multi-GPU path of its own).
 * `out` is this rank's head slice of its full (B, S, Hq, D) output; out_peers[i] is the
 * address of the same slice in another GPU's copy of that output (identical layout and
 * strides), reachable from this GPU (peer access or a symmetric-memory mapping).  The
 * attention epilogue writes every output tile to `out` and, with 16-byte stores over
 * NVLink, to each peer, so the gather overlaps the attention.  The call returns when the
 * work is queued: the caller orders the peers' reads after every rank's kernel (a
 * cross-GPU barrier on the stream).  n_peers <= 7. */
FPB_API int fpb_prefill_dense_peers(const void* q, const void* k, const void* v, void* out, int dtype, int batch,
                                    int seqlen, int hq, int hk, int head_dim, const int64_t* q_strides,
                                    const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                                    int block_size, int attention_sink, int window_size, float alpha,
                                    int last_n_block_full, int min_budget, int mean_model, void* workspace,
                                    size_t workspace_bytes, void* const* out_peers, int n_peers, void* stream);

/* fpb_prefill_dense restricted to the query blocks [q_block_begin, q_block_end) of every batch
 * entry: their block lists are searched and their output rows written, with the selection
 * rules of the whole sequence (the last-N rule still refers to the sequence's last blocks);
 * other output rows are left untouched.  The union over a partition of [0, ceil(S/128)) of
 * such calls equals one fpb_prefill_dense call.  It serves a 2-D split of one layer over
 * GPUs (KV-head groups x query-block ranges, each GPU holding its heads' whole K/V) when
 * there are more GPUs than KV heads.  The reference runs whole layers only
 * (ops/flashprefill_native_forward.py:481-499); q/k/v/out and the workspace are as in
 * fpb_prefill_dense. */
FPB_API int fpb_prefill_dense_rows(const void* q, const void* k, const void* v, void* out, int dtype, int batch,
                                   int seqlen, int hq, int hk, int head_dim, const int64_t* q_strides,
                                   const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                                   int block_size, int attention_sink, int window_size, float alpha,
                                   int last_n_block_full, int min_budget, int mean_model, int q_block_begin,
                                   int q_block_end, void* workspace, size_t workspace_bytes, void* stream);

/* Chunked (prefix) prefill: the queries are the last q_len positions of a kv_len-token sequence
 * (q and out (B, q_len, Hq, D); k and v (B, kv_len, Hk, D), the cached prefix followed by the
 * chunk).  Block structure, pooled keys and the selection rules are those of the whole
 * kv_len-token sequence (the last-N rule refers to its last blocks); a query block that starts
 * before the chunk scores its missing rows as zero rows, as the search scores the padded rows of
 * a partial last block.  The workspace is that of fpb_prefill_dense for kv_len tokens.  With
 * q_len = kv_len it equals fpb_prefill_dense.  No counterpart in the reference, which sends
 * chunked prefills to dense attention (patches/patch_loader_vllm_0_10_0.py:272-300,
 * ruler/models/llama.py:310-333). */
FPB_API int fpb_prefill_dense_chunk(const void* q, const void* k, const void* v, void* out, int dtype, int batch,
                                    int q_len, int kv_len, int hq, int hk, int head_dim, const int64_t* q_strides,
                                    const int64_t* k_strides, const int64_t* v_strides,
                                    const int64_t* o_strides, int block_size, int attention_sink,
                                    int window_size, float alpha, int last_n_block_full, int min_budget,
                                    int mean_model, void* workspace, size_t workspace_bytes, void* stream);

/* Search stage only (pooled keys + block lists into the workspace): replaces
 * compute_mean_vector + compute_block_score + normalize_scores + deal_output_score
 * (ops/flashprefill_native_forward.py:22-188,347-403). */
FPB_API int fpb_search_dense(const void* q, const void* k, int dtype, int batch, int seqlen, int hq, int hk,
                             int head_dim, const int64_t* q_strides, const int64_t* k_strides, int block_size,
                             int attention_sink, int window_size, float alpha, int last_n_block_full,
                             int min_budget, int mean_model, void* workspace, size_t workspace_bytes, void* stream);

/* Search stage only, varlen: replaces ops/flashprefill_varlen_func.py:8-18,35-409,656-698. */
FPB_API int fpb_search_varlen(const void* q, const void* k, int dtype, const int32_t* cu_seqlens, int nseq,
                              int total_tokens, int max_seq_len, int hq, int hk, int head_dim,
                              const int64_t* q_strides, const int64_t* k_strides, int block_size,
                              int attention_sink, int window_size, float alpha, int last_n_block, int mean_model,
                              void* workspace, size_t workspace_bytes, void* stream);

/* Attention stage only, over the block lists already in the workspace (written by
 * fpb_search_* or by the caller): replaces _flash_forward
 * (ops/flashprefill_native_forward.py:228-344). */
FPB_API int fpb_attention_dense(const void* q, const void* k, const void* v, void* out, int dtype, int batch,
                                int seqlen, int hq, int hk, int head_dim, const int64_t* q_strides,
                                const int64_t* k_strides, const int64_t* v_strides, const int64_t* o_strides,
                                int block_size, void* workspace, size_t workspace_bytes, void* stream);

/* Attention stage only, varlen: replaces _flash_block_sparse_varlen
 * (ops/flashprefill_varlen_func.py:449-575).  Needs cu_tile in the workspace, which
 * fpb_search_varlen writes. */
FPB_API int fpb_attention_varlen(const void* q, const void* k, const void* v, void* o, int dtype,
                                 const int32_t* cu_seqlens, int nseq, int total_tokens, int max_seq_len, int hq,
                                 int hk, int head_dim, const int64_t* q_strides, const int64_t* k_strides,
                                 const int64_t* v_strides, const int64_t* o_strides, int block_size,
                                 void* workspace, size_t workspace_bytes, void* stream);

/* Dense prefill that allocates nothing, for callers that cannot call cudaMalloc or pass
 * a workspace (runtimes that forbid allocation on their hot path, hosts without a device
 * allocator).  No counterpart in the reference.  Same arguments and results as
 * fpb_prefill_dense without the workspace: it uses a 32 MiB device array inside the
 * library, held by every GPU that loads the library until exit.  Problems whose required
 * workspace (the error word, pooled keys, counts and block lists: every part of
 * fpb_dense_workspace_bytes except the optional long-row split area) exceeds 32 MiB are
 * rejected with FPB_EINVAL (e.g. 32K tokens with 32/8 heads fit; 128K do not); long rows
 * are split only when the split area fits in the array as well.  The first call on a
 * device looks up the array's address on that device and should come before any stream
 * capture.  Calls share the array: calls that overlap on the GPU race.  Device-side errors
 * of these calls are read with fpb_noalloc_read_device_error. */
FPB_API int fpb_prefill_dense_noalloc(const void* q, const void* k, const void* v, void* out, int dtype, int batch,
                                      int seqlen, int hq, int hk, int head_dim, const int64_t* q_strides,
                                      const int64_t* k_strides, const int64_t* v_strides,
                                      const int64_t* o_strides, int block_size, int attention_sink,
                                      int window_size, float alpha, int last_n_block_full, int min_budget,
                                      int mean_model, void* stream);

/* fpb_read_device_error for the no-allocation path: synchronises `stream` and reads the
 * error word of the current device's fixed scratch array (the last
 * fpb_prefill_dense_noalloc call on that device).  No counterpart in the reference. */
FPB_API int fpb_noalloc_read_device_error(uint32_t* flags, void* stream);

/* Test hook, no counterpart in the reference: on the current device, sets the limit of every
 * bounded device-side wait (default 1 s; accepted range 1 ms .. 1 s) and, when
 * withhold_first_load is non-zero, arms a one-shot fault: the next attention launch on the
 * device skips one key-tile load (the first producer to reach one consumes the fault), so
 * that one of its waits runs out and the call reports FPB_DEV_WAIT_TIMEOUT through the
 * error word.  Call it again with (0, 1000000000) to restore normal operation.  For tests
 * of the timeout path only. */
FPB_API int fpb_test_set_fault(int withhold_first_load, unsigned long long wait_limit_ns);

/* Synchronises `stream`, copies the device error word of `workspace` to *flags and
 * returns FPB_EDEVICE if any bit is set.  No counterpart in the reference, which has no
 * device-side error reporting. */
FPB_API int fpb_read_device_error(const void* workspace, uint32_t* flags, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FLASHPREFILL_B200_H */
