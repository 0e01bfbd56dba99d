/*
 * flashdecode.h - C ABI of the B200 (sm_100a) paged-KV GQA decode operator.
 *
 * All pointers are device pointers unless stated otherwise.  No torch types
 * appear here; the library is loadable with dlopen/ctypes/cgo alike.
 *
 * Tensor layouts (row-major, contiguous):
 *   q             [B, 1, Hq, D]                 (bf16 or fp16)
 *   k_cache/v_cache [num_blocks, page, Hkv, D]  (same dtype as q, "NHD")
 *   block_table   [B, block_table_stride]       int32 physical page ids
 *   cache_seqlens [B]                           int32 tokens per sequence
 *   out           [B, 1, Hq, D]                 (dtype of q, or fp32)
 *   lse           [B, Hq]                       fp32 natural-log LSE (nullable)
 * Query head h reads KV head h / (Hq / Hkv).  Entries of block_table past
 * ceil(cache_seqlens[b] / page) are never read (they may be -1).
 */
#ifndef FLASHDECODE_H_
#define FLASHDECODE_H_

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* dtype codes */
#define FD_DTYPE_BF16 0
#define FD_DTYPE_FP16 1
#define FD_DTYPE_FP32 2 /* output only */
#define FD_DTYPE_E4M3 3 /* K/V cache only (fd_decode_paged_fp8) */

/* status codes */
#define FD_OK 0
#define FD_ERR_INVALID_ARG 1    /* a size/shape argument is out of range     */
#define FD_ERR_UNSUPPORTED 2    /* valid request this build does not handle  */
#define FD_ERR_WORKSPACE 3      /* workspace missing or too small            */
#define FD_ERR_CUDA 4           /* a CUDA runtime/driver call failed         */
#define FD_ERR_DEVICE_TIMEOUT 5 /* a bounded in-kernel wait ran out          */
#define FD_ERR_BAD_PAGE 6       /* a block_table id inside a sequence's range
                                   lies outside [0, num_blocks) (reported by
                                   fd_device_status; those rows read as 0)   */

/*
 * run_kernel - drop-in for the reference operator surface.
 *
 * Replaces: the `extern "C" void run_kernel(...)` declared by the reference
 * evaluator's binding (scripts/evaluate_flashattn_submission.py:29-44) and
 * defined by every submission, e.g.
 * submission-oj/best_flashattn_kvcache_decode.cu:1186-1426.
 * Same 15 arguments and meaning: bf16 tensors, softmax scale 1/sqrt(headdim),
 * block_table row stride = num_blocks / batch_size, seqlen_k is the maximum
 * sequence length (a scheduling hint; per-row lengths come from
 * cache_seqlens), no LSE output, launched on the legacy default stream,
 * asynchronous.  Like the reference it returns void and silently does nothing
 * on arguments it rejects; unlike the reference the reason is kept and can be
 * read with fd_last_error().  Unsupported-by-the-reference shapes (any head
 * group, page sizes other than 16, fp16 is not reachable here) are computed
 * rather than rejected.  seqlen_q > 1 and causal are honoured as in
 * fd_decode_paged_mq (the reference's fast paths reject them and its
 * fallback kernel assumes one query token).
 */
void run_kernel(const void* q, const void* k_cache_paged, const void* v_cache_paged, void* output,
                const int32_t* cache_seqlens, const int32_t* block_table, int64_t batch_size,
                int64_t seqlen_k, int64_t seqlen_q, int64_t num_heads, int64_t num_heads_k,
                int64_t headdim, int64_t page_block_size, int64_t num_blocks, int64_t causal);

/*
 * fd_decode_paged - the extended entry point (stream, dtype, scale, LSE,
 * explicit block_table stride, caller workspace).
 *
 * Replaces: the same reference run_kernel (best_flashattn_kvcache_decode.cu
 * :1186-1426) with the arguments the reference hard-codes made explicit:
 * softmax scale (best :286-287), block_table stride (best :1213), stream
 * (reference launches on the default stream), LSE output (reference emits
 * none; flash_attn_with_kvcache's return_softmax_lse, which the evaluator's
 * oracle call at evaluate_flashattn_submission.py:232-247 wraps).
 *
 * dtype:        FD_DTYPE_BF16 or FD_DTYPE_FP16 for q/k/v.
 * out_dtype:    FD_DTYPE_FP32 or the value of dtype.
 * max_seqlen_k: upper bound on cache_seqlens (0 = unknown); only sizes the grid.
 * workspace:    device buffer of at least fd_decode_workspace_size(...) bytes,
 *               zero-filled once before its first use (cudaMemset); the
 *               kernel keeps it consistent from then on (its counters carry a
 *               per-launch epoch and are cleared when a launch completes), so
 *               it never needs clearing again, also after a call that
 *               reported FD_ERR_DEVICE_TIMEOUT.  Or NULL: the library then
 *               uses a buffer of its own for this (device, stream) pair,
 *               allocated and zero-filled on the stream's first call and kept
 *               until the process exits, so calls on different streams never
 *               share one.  It grows to the largest shape the stream has
 *               seen; an outgrown buffer is kept too (a CUDA graph captured
 *               on the stream may still use it).  A call being captured into
 *               a CUDA graph may allocate it (the allocation is made outside
 *               the graph).  One workspace must not be used by two calls
 *               that can run at the same time.
 * stream:       cudaStream_t (NULL = legacy default stream).
 * Returns FD_OK or an FD_ERR_* code; launches are asynchronous.  Errors met
 * inside a kernel (a bounded wait that ran out, a block_table id outside the
 * pool) are reported later by fd_device_status.
 */
int fd_decode_paged(const void* q, const void* k_cache, const void* v_cache, void* out, float* lse,
                    const int32_t* cache_seqlens, const int32_t* block_table,
                    int64_t block_table_stride, int64_t batch_size, int64_t num_heads,
                    int64_t num_heads_k, int64_t headdim, int64_t page_block_size,
                    int64_t num_blocks, int dtype, int out_dtype, float softmax_scale,
                    int64_t max_seqlen_k, void* workspace, size_t workspace_bytes, void* stream);

/*
 * fd_decode_paged_mq - fd_decode_paged for seqlen_q >= 1 query tokens per
 * sequence (speculative / multi-token decode), with an optional causal mask.
 * q and out are [B, seqlen_q, Hq, D]; lse (nullable) is [B, Hq, seqlen_q].
 * The cached keys of sequence b are its cache_seqlens[b] tokens; with causal
 * != 0 query token i sits at position cache_seqlens[b] - seqlen_q + i and
 * sees keys up to that position (bottom-right alignment, as in
 * flash_attn_with_kvcache); without it every query token sees all keys.
 * Replaces: the seqlen_q and causal arguments of the reference run_kernel
 * (best_flashattn_kvcache_decode.cu:1186-1201), which its fast paths reject
 * (best :1235-1242) and its fallback ignores.
 */
int fd_decode_paged_mq(const void* q, const void* k_cache, const void* v_cache, void* out,
                       float* lse, const int32_t* cache_seqlens, const int32_t* block_table,
                       int64_t block_table_stride, int64_t batch_size, int64_t seqlen_q,
                       int64_t num_heads, int64_t num_heads_k, int64_t headdim,
                       int64_t page_block_size, int64_t num_blocks, int dtype, int out_dtype,
                       float softmax_scale, int causal, int64_t max_seqlen_k, void* workspace,
                       size_t workspace_bytes, void* stream);

/* Workspace bytes fd_decode_paged_mq needs (same role as fd_decode_workspace_size). */
size_t fd_decode_workspace_size_mq(int64_t batch_size, int64_t seqlen_q, int64_t num_heads,
                                   int64_t num_heads_k, int64_t headdim);

/*
 * fd_append_kv_paged - write a step's new keys and values into the paged cache.
 *
 * Replaces: the cache update flash_attn_with_kvcache performs when given
 * k / v (the reference evaluator passes None for both,
 * scripts/evaluate_flashattn_submission.py:233-239, so no reference
 * submission implements it).  k_new / v_new are [B, seqlen_new, Hkv, D];
 * row t of sequence b is stored at position max(cache_seqlens[b], 0) + t,
 * i.e. page block_table[b * block_table_stride + pos / page_block_size],
 * row pos % page_block_size.  cache_seqlens is not modified (the caller
 * advances it, as with flash_attn).  A row whose position lies past the
 * block table, or whose page id is outside [0, num_blocks), is skipped.
 */
int fd_append_kv_paged(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                       const int32_t* cache_seqlens, const int32_t* block_table,
                       int64_t block_table_stride, int64_t batch_size, int64_t seqlen_new,
                       int64_t num_heads_k, int64_t headdim, int64_t page_block_size,
                       int64_t num_blocks, int dtype, void* stream);

/*
 * fd_decode_paged_kvappend - fd_append_kv_paged, then fd_decode_paged_mq over
 * max(cache_seqlens[b], 0) + seqlen_new keys per sequence.
 *
 * Replaces: flash_attn_with_kvcache(q, k_cache, v_cache, k, v, cache_seqlens,
 * block_table=..., causal=...) with k / v given, the call the reference
 * evaluator makes with k = v = None (evaluate_flashattn_submission.py
 * :232-247).  With causal, query token i sits at position
 * max(cache_seqlens[b], 0) + seqlen_new - seqlen_q + i.  Arguments the
 * attention half would reject are checked before the cache is written.
 * max_seqlen_k bounds the attended length (cached + appended), 0 = unknown.
 */
int fd_decode_paged_kvappend(const void* q, void* k_cache, void* v_cache, const void* k_new,
                             const void* v_new, void* out, float* lse,
                             const int32_t* cache_seqlens, const int32_t* block_table,
                             int64_t block_table_stride, int64_t batch_size, int64_t seqlen_q,
                             int64_t seqlen_new, int64_t num_heads, int64_t num_heads_k,
                             int64_t headdim, int64_t page_block_size, int64_t num_blocks,
                             int dtype, int out_dtype, float softmax_scale, int causal,
                             int64_t max_seqlen_k, void* workspace, size_t workspace_bytes,
                             void* stream);

/*
 * fd_decode_paged_fp8 - decode over an e4m3 (FP8) KV cache with per-KV-head
 * scales: the attended key/value of token t, KV head h, is
 * k_cache[...] * k_scale[h] / v_cache[...] * v_scale[h].
 *
 * Replaces: nothing in the reference (its caches are bf16, best :1186-1211);
 * this is the FP8-cache extension of the same decode, halving the bytes the
 * HBM-bound kernel reads.  q (bf16 or fp16, q_dtype), out (q_dtype or fp32)
 * and lse keep fd_decode_paged_mq's layouts and meaning; k_cache / v_cache
 * are [num_blocks, page, Hkv, 128] e4m3 bytes; k_scale / v_scale are device
 * fp32 [Hkv].  With k_new / v_new (16-bit [B, seqlen_new, Hkv, 128]) given,
 * they are first quantised into the cache at cache_seqlens[b] + t as by
 * fd_append_kv_paged_fp8 and attention covers cache_seqlens[b] + seqlen_new
 * keys; pass NULL for both otherwise.  Supported: head dim 128,
 * seqlen_q * (Hq / Hkv) <= 16, page a multiple of 16, 16-byte aligned
 * q / caches (FD_ERR_UNSUPPORTED otherwise).  Workspace: at least
 * fd_decode_workspace_size_fp8(...) bytes, 256-byte aligned and zero-filled
 * before its first use, or NULL (as for fd_decode_paged).
 */
int fd_decode_paged_fp8(const void* q, void* k_cache, void* v_cache, const float* k_scale,
                        const float* v_scale, const void* k_new, const void* v_new,
                        int64_t seqlen_new, void* out, float* lse, const int32_t* cache_seqlens,
                        const int32_t* block_table, int64_t block_table_stride,
                        int64_t batch_size, int64_t seqlen_q, int64_t num_heads,
                        int64_t num_heads_k, int64_t headdim, int64_t page_block_size,
                        int64_t num_blocks, int q_dtype, int out_dtype, float softmax_scale,
                        int causal, int64_t max_seqlen_k, void* workspace, size_t workspace_bytes,
                        void* stream);

/* Workspace bytes fd_decode_paged_fp8 needs (0 for unsupported shapes). */
size_t fd_decode_workspace_size_fp8(int64_t batch_size, int64_t seqlen_q, int64_t num_heads,
                                    int64_t num_heads_k, int64_t headdim);

/*
 * fd_append_kv_paged_fp8 - fd_append_kv_paged into an e4m3 cache: each new
 * 16-bit value x (src_dtype bf16 or fp16) of KV head h is stored as
 * e4m3(x / scale[h]), rounded to nearest even and saturated at +-448.
 * Replaces: nothing in the reference (see fd_decode_paged_fp8).
 */
int fd_append_kv_paged_fp8(const void* k_new, const void* v_new, void* k_cache, void* v_cache,
                           const float* k_scale, const float* v_scale,
                           const int32_t* cache_seqlens, const int32_t* block_table,
                           int64_t block_table_stride, int64_t batch_size, int64_t seqlen_new,
                           int64_t num_heads_k, int64_t headdim, int64_t page_block_size,
                           int64_t num_blocks, int src_dtype, void* stream);

/*
 * fd_decode_paged_noalloc - fd_decode_paged for callers that cannot allocate
 * device memory: a process whose framework allocator already holds nearly
 * all of the GPU's memory (a library cudaMalloc would fail or fragment that
 * pool), or a serving loop that allocates everything at start-up and forbids
 * allocation afterwards.  Same arguments as fd_decode_paged without the
 * workspace: the split scratch is a fixed 8 MiB array inside the library's
 * device image, held on every GPU that loads the library until the process
 * exits.  Shapes needing more scratch than that (fd_decode_workspace_size >
 * 8 MiB) are rejected with FD_ERR_WORKSPACE.  Calls no cudaMalloc/cudaFree
 * or other allocating routine.  The first call on a device looks up the
 * array's device address (cudaGetSymbolAddress, that device current), so make
 * that first call before any stream capture.  All calls share the array and
 * it keeps the previous call's contents (the call clears what must start at
 * zero): calls that can overlap on the GPU race with each other.  Shapes the
 * CUDA-core kernel takes (head dim other than 128, more than 16 query heads
 * per KV head, pages not a multiple of 16, q/k/v not 16-byte aligned) use no
 * scratch and are never refused for its size.  Kernel-side errors are read
 * with fd_device_status, as for fd_decode_paged.
 * No counterpart in the reference, whose run_kernel always cudaMallocs its
 * split workspace on first use.
 */
int fd_decode_paged_noalloc(const void* q, const void* k_cache, const void* v_cache, void* out,
                            float* lse, const int32_t* cache_seqlens, const int32_t* block_table,
                            int64_t block_table_stride, int64_t batch_size, int64_t num_heads,
                            int64_t num_heads_k, int64_t headdim, int64_t page_block_size,
                            int64_t num_blocks, int dtype, int out_dtype, float softmax_scale,
                            int64_t max_seqlen_k, void* stream);

/*
 * fd_decode_workspace_size - bytes of workspace fd_decode_paged needs for
 * these shapes on the current device.
 * Replaces: reserve_split_workspace sizing (best :1078-1133, :1343-1348),
 * exposed so callers can own the memory.
 */
size_t fd_decode_workspace_size(int64_t batch_size, int64_t num_heads, int64_t num_heads_k,
                                int64_t headdim);

/*
 * fd_combine_lse - merge n_parts partial attention results computed over
 * disjoint KV ranges into one (the cross-GPU split-KV exchange step).
 * part_o   part j at part_o + j * part_o_stride: [rows, headdim] fp32, each
 *          part already normalised (part_o_stride 0 = rows * headdim);
 * part_lse part j at part_lse + j * part_lse_stride: [rows] fp32 natural
 *          log, -inf = empty part (part_lse_stride 0 = rows);
 * out      [rows, headdim] of out_dtype; lse_out [rows] (nullable).
 * The strides let one gathered buffer of per-part [O | LSE] blocks be merged
 * in place.
 * Replaces: combine_split_lse_kernel (best :956-1037) and combine_lse_kernel
 * _v11 (v11_best_hybrid/..._v11_best_hybrid.cu:574-614), including the rule
 * that empty parts get weight zero.
 */
int fd_combine_lse(const float* part_o, int64_t part_o_stride, const float* part_lse,
                   int64_t part_lse_stride, int64_t n_parts, int64_t rows, int64_t headdim,
                   void* out, int out_dtype, float* lse_out, void* stream);

/*
 * Cross-GPU split-KV decode over peer memory (one process per GPU of a node).
 *
 * Each rank holds a page range of every sequence (its own cache_seqlens and
 * block_table describe that range) and an exchange buffer of
 * fd_xgpu_buffer_size() bytes made by fd_xgpu_alloc; the ranks swap the
 * 64-byte IPC handles (any host channel) and map each other's buffers with
 * fd_xgpu_open.  fd_decode_paged_xgpu then runs one step: the decode kernel
 * writes this rank's partial (O, LSE) for every output row straight into
 * every rank's buffer over NVLink and flags it; a merge kernel waits (bounded,
 * FD_ERR_DEVICE_TIMEOUT in the device status word on expiry) for all ranks'
 * flags and writes out [B, sq, Hq, D] and lse [B, Hq, sq] on every rank.
 * xbufs: host array of `world` device pointers, entry rank = own buffer.
 * step: call counter, the same on every rank, +1 per call (the buffer is
 * double-buffered by its parity).  Needs the tensor-core path (head dim 128,
 * seqlen_q * Hq / Hkv <= 16) and batch_size <= 512.
 * Replaces: the reference's split combine (best_flashattn_kvcache_decode.cu
 * :956-1037, :1420-1425) with the splits on different GPUs; the reference has
 * no multi-GPU code.
 */
size_t fd_xgpu_buffer_size(int64_t batch_size, int64_t seqlen_q, int64_t num_heads, int world);
int fd_xgpu_alloc(size_t bytes, void** ptr, void* ipc_handle);
int fd_xgpu_open(const void* ipc_handle, void** ptr);
int fd_xgpu_close(void* ptr);
int fd_xgpu_free(void* ptr);
int fd_decode_paged_xgpu(const void* q, const void* k_cache, const void* v_cache,
                         const int32_t* cache_seqlens, const int32_t* block_table,
                         int64_t block_table_stride, int64_t batch_size, int64_t seqlen_q,
                         int64_t num_heads, int64_t num_heads_k, int64_t headdim,
                         int64_t page_block_size, int64_t num_blocks, int dtype, int out_dtype,
                         float softmax_scale, int causal, int64_t max_seqlen_k, int rank,
                         int world, void* const* xbufs, uint64_t step, void* out, float* lse,
                         void* workspace, size_t workspace_bytes, void* stream);

/*
 * fd_decode_paged_fp8_xgpu - fd_decode_paged_xgpu over an e4m3 KV cache:
 * the same step, exchange buffers and merge, with k_cache / v_cache and
 * k_scale / v_scale as in fd_decode_paged_fp8 (q of type q_dtype, bf16 or
 * fp16; no cache append).  Same limits as fd_decode_paged_fp8 and
 * batch_size <= 512.
 * Replaces: nothing in the reference (no FP8 cache, no multi-GPU code).
 */
int fd_decode_paged_fp8_xgpu(const void* q, const void* k_cache, const void* v_cache,
                             const float* k_scale, const float* v_scale,
                             const int32_t* cache_seqlens, const int32_t* block_table,
                             int64_t block_table_stride, int64_t batch_size, int64_t seqlen_q,
                             int64_t num_heads, int64_t num_heads_k, int64_t headdim,
                             int64_t page_block_size, int64_t num_blocks, int q_dtype,
                             int out_dtype, float softmax_scale, int causal, int64_t max_seqlen_k,
                             int rank, int world, void* const* xbufs, uint64_t step, void* out,
                             float* lse, void* workspace, size_t workspace_bytes, void* stream);

/* Status of the last call made on this host thread, and its message. */
int fd_last_error(void);
const char* fd_error_string(int code);
const char* fd_last_error_message(void);

/*
 * fd_device_status - read and clear the current device's status word: the
 * first error a kernel of this library met there since the last read,
 * whatever entry point and workspace the call used.  FD_ERR_DEVICE_TIMEOUT:
 * a bounded in-kernel wait ran out (that call's results are incomplete);
 * FD_ERR_BAD_PAGE: a block_table entry inside a sequence's length was
 * outside [0, num_blocks) (its rows were read as zeros, nothing outside the
 * cache was touched).  FD_OK otherwise.  Synchronises the current device.
 * Replaces: nothing in the reference, whose kernels report no errors and
 * gather through block_table unchecked (best :741-742).
 */
int fd_device_status(void);

/*
 * fd_library_workspace_bytes - bytes of workspace the library holds on the
 * current device for calls that passed workspace = NULL (all streams,
 * outgrown buffers included).
 * Replaces: nothing in the reference (its workspace is one process-global
 * buffer, best :17-20); lets a caller account for the library's memory.
 */
size_t fd_library_workspace_bytes(void);

/*
 * fd_selftest_bounded_wait - launch a one-warp kernel that waits on an
 * mbarrier nothing arrives on, with the same bounded wait the decode kernel
 * uses, and report what happened.  Returns FD_ERR_DEVICE_TIMEOUT when the
 * wait gave up as designed (the CUDA context stays usable), FD_OK if the
 * barrier completed, FD_ERR_CUDA on a launch failure.  *waited_ns (nullable,
 * host pointer) receives the time the wait took.  Synchronises the device.
 * No counterpart in the reference, which has no bounded waits.
 */
int fd_selftest_bounded_wait(uint64_t budget_ns, uint64_t* waited_ns);

/* Library version string. */
const char* fd_version(void);

#ifdef __cplusplus
}
#endif

#endif /* FLASHDECODE_H_ */
