/*
 * dsa_b200.h -- C ABI of the B200 (sm_100a) DSA decode kernels.
 *
 * Two operators, both destination-passing style (the caller owns inputs,
 * outputs and the scratch workspace; nothing here allocates device memory):
 *
 *   dsa_indexer_run    -- FP8 lightning indexer + top-2048 select.
 *     Replaces the reference entry point
 *       run(q_index_fp8, k_index_cache_fp8, weights, seq_lens, block_table,
 *           topk_indices)
 *     at dsa_indexer/solution/triton/kernel.py:364-436 and its host driver
 *     dsa_topk_run_ms (kernel.py:190-319).
 *
 *   dsa_attention_run  -- sparse MLA attention over the selected slots.
 *     Replaces the reference entry point
 *       run(q_nope, q_pe, ckv_cache, kpe_cache, sparse_indices, sm_scale,
 *           output, lse)
 *     at dsa_attention/solution/triton/kernel.py:240-252 and its host driver
 *     dsa_sparse_attention (kernel.py:174-218).
 *
 * All pointers are device pointers except where stated; all launches go to
 * `stream` (a cudaStream_t passed as void*), so calls are CUDA-graph
 * capturable.  No call synchronises the device or reads device memory on the
 * host (unlike the reference indexer, which reads seq_lens on the host at
 * kernel.py:375).
 *
 * Every function returns a dsa_status (0 == DSA_OK).  Argument errors are
 * detected on the host before anything is launched.  Data-dependent errors
 * (a page id outside the pool, a seq_len larger than the block table, a
 * sparse index outside the cache, a bounded wait that ran out) are recorded
 * by the kernels as bits of a sticky 32-bit word at the start of the
 * workspace; dsa_read_device_status() reads and optionally clears it.
 */
#ifndef DSA_B200_H_
#define DSA_B200_H_

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define DSA_API __attribute__((visibility("default")))
#else
#define DSA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (host side) ---------------------------------------- */
#define DSA_OK                       0
#define DSA_ERR_INVALID_ARGUMENT     1
#define DSA_ERR_MISALIGNED           2
#define DSA_ERR_WORKSPACE_TOO_SMALL  3
#define DSA_ERR_CUDA                 4
#define DSA_ERR_UNSUPPORTED_DEVICE   5
#define DSA_ERR_TENSOR_MAP           6

/* ---- sticky device status bits (first uint32 of each workspace) ------ */
#define DSA_DEV_BAD_SEQ_LEN   0x1u  /* seq_len < 0 or > max_pages*64; clamped   */
#define DSA_DEV_BAD_PAGE      0x2u  /* block_table entry outside [0, num_pages) */
#define DSA_DEV_BAD_INDEX     0x4u  /* sparse index outside [-1, num_slots)     */
#define DSA_DEV_WAIT_TIMEOUT  0x8u  /* a bounded pipeline wait gave up          */
#define DSA_DEV_STALE_WORKSPACE 0x10u /* workspace contents did not match: a merge */
                                      /* counter not zero on entry, or an indexer */
                                      /* histogram not matching its scores        */

/* Shape constants of the two contest definitions
 * dsa_topk_indexer_fp8_h64_d128_topk2048_ps64 and
 * dsa_sparse_attention_h16_ckv512_kpe64_topk2048_ps64. */
#define DSA_PAGE_SIZE        64
#define DSA_INDEX_HEADS      64
#define DSA_INDEX_DIM        128
#define DSA_INDEX_PAGE_BYTES 8448  /* 64*128 fp8 + 64 fp32 scales (kernel.py:80) */
#define DSA_TOPK             2048
#define DSA_ATTN_HEADS       16
#define DSA_CKV_DIM          512
#define DSA_KPE_DIM          64

/* Version of this ABI (bumped on any signature change). */
DSA_API int dsa_b200_abi_version(void);

/* Human-readable text for a dsa_status value; never NULL. */
DSA_API const char* dsa_b200_status_string(int status);

/* Bytes of device workspace dsa_indexer_run needs for this batch and block
 * table width: a 256-byte header, 32 KiB of per-request ready counters
 * (the score kernel counts each request's scored tiles there and the top-k
 * select of that request starts once they are all counted; the counters
 * carry over from call to call and are never reset), a [batch, 2048] uint32
 * radix histogram (cleared by the call itself, on its stream, before the
 * scores are added) and [batch, max_pages*64] fp32 score rows.  Zero-fill a
 * workspace once before its first use, so that the status word in its
 * header starts clear and the ready counters start consistent. */
DSA_API size_t dsa_indexer_workspace_bytes(int32_t batch, int32_t max_pages);

/* FP8 lightning indexer, decode (one query token per request).
 *
 *   q_index_fp8       [batch, 64, 128] float8_e4m3fn, contiguous
 *   k_index_cache_fp8 num_pages pages of 8448 bytes: 64x128 fp8 then 64 fp32
 *                     scales (the [num_pages, 64, 1, 132] uint8 cache viewed
 *                     as bytes), 16-byte aligned
 *   weights           [batch, 64] fp32
 *   seq_lens          [batch] int32 (device memory; never read on the host)
 *   block_table       [batch, max_pages] int32
 *   topk_indices      [batch, 2048] int32 output: global slot ids
 *                     block_table[b, t/64]*64 + t%64 of the top-min(L,2048)
 *                     tokens, score descending, ties by lower token index,
 *                     then -1 padding.
 *
 * Mirrors dsa_indexer/solution/triton/kernel.py:364 (argument order and
 * meaning), plus the sizes a C caller must pass explicitly. */
DSA_API int dsa_indexer_run(const void* q_index_fp8, const void* k_index_cache_fp8,
                    int64_t num_pages, const float* weights,
                    const int32_t* seq_lens, const int32_t* block_table,
                    int32_t batch, int32_t max_pages, int32_t* topk_indices,
                    void* workspace, size_t workspace_bytes, void* stream);

/* Bytes of device workspace dsa_attention_run needs for num_tokens queries
 * on this device: a 256-byte header, two split-softmax partial records per
 * CTA (a token segment's O in fp32 and its per-head max and sum, 32.1 KiB
 * each) and two merge counters per token, placed at the end of the
 * workspace.  Zero-fill a workspace once before its first use (status word
 * and counters start at zero) and pass the same workspace_bytes to every
 * call on it.  Every call leaves the counters at zero again, including one
 * that gave up on a bounded wait (DSA_DEV_WAIT_TIMEOUT).  A counter found
 * non-zero on entry (the workspace was changed from outside, or two calls on
 * it overlapped) is reported as DSA_DEV_STALE_WORKSPACE by this and every
 * later call until the workspace is zero-filled again. */
DSA_API size_t dsa_attention_workspace_bytes(int32_t num_tokens);

/* Sparse MLA attention, one query token per row of sparse_indices.
 * Launched with programmatic stream serialization: it may be scheduled while
 * the previous kernel on `stream` drains, and touches global memory only
 * after that kernel has completed.
 *
 *   q_nope          [num_tokens, 16, 512] bf16
 *   q_pe            [num_tokens, 16, 64]  bf16
 *   ckv_cache       num_slots rows of 512 bf16 ([pages, 64, 512] flattened)
 *   kpe_cache       num_slots rows of 64 bf16  ([pages, 64, 64] flattened)
 *   sparse_indices  [num_tokens, 2048] int32 global slot ids, -1 = padding
 *   output          [num_tokens, 16, 512] bf16
 *   lse             [num_tokens, 16] fp32, base-2 log-sum-exp of the scaled
 *                   logits; -inf (and output 0) for a row with no valid index
 *
 * Mirrors dsa_attention/solution/triton/kernel.py:241 (argument order and
 * meaning), plus the sizes a C caller must pass explicitly. */
DSA_API int dsa_attention_run(const void* q_nope, const void* q_pe,
                      const void* ckv_cache, const void* kpe_cache,
                      int64_t num_slots, const int32_t* sparse_indices,
                      int32_t num_tokens, float sm_scale,
                      void* output, float* lse,
                      void* workspace, size_t workspace_bytes, void* stream);

/* Size of the scratch array compiled into the library for
 * dsa_indexer_run_noalloc: the 256-byte header, the per-request ready
 * counters (32 KiB), 64 radix histograms and 1,048,576 fp32 score slots
 * (4.5 MiB per GPU that loads the library). */
#define DSA_NOALLOC_SCRATCH_BYTES (256u + 32768u + 64u * 2048u * 4u + 1048576u * 4u)

/* dsa_indexer_run without a workspace argument, for callers that cannot
 * allocate device memory when they call: hosts that reach this library
 * through C / JNI / FFI while another allocator owns the device memory, and
 * serving loops that allow no cudaMalloc after warm-up.  Scratch comes from
 * a fixed array inside the library (DSA_NOALLOC_SCRATCH_BYTES), so the
 * problem must fit: dsa_indexer_workspace_bytes(batch, max_pages) may not
 * exceed it (e.g. 64 requests x 256 pages, or 8 requests x 2048 pages);
 * otherwise the call returns DSA_ERR_WORKSPACE_TOO_SMALL before touching the
 * device.  Nothing is allocated or freed.
 *   - The first call on a device looks up the array's device address, so
 *     make it before capturing any stream.
 *   - All calls share the one array: calls whose work overlaps on the GPU
 *     (other streams, other threads) race and corrupt each other's results.
 *   - Data-dependent device errors are recorded in the array's status word,
 *     which this entry point gives no way to read; use dsa_indexer_run when
 *     they must be observed.
 * Arguments have the meaning of dsa_indexer_run.  No counterpart in the
 * reference, which always allocates its scratch through PyTorch. */
DSA_API int dsa_indexer_run_noalloc(const void* q_index_fp8, const void* k_index_cache_fp8,
                                    int64_t num_pages, const float* weights,
                                    const int32_t* seq_lens, const int32_t* block_table,
                                    int32_t batch, int32_t max_pages, int32_t* topk_indices,
                                    void* stream);

/* Bytes of device workspace dsa_indexer_prefill_run needs: a 256-byte header,
 * a [num_rows, 2048] uint32 radix histogram (cleared by the call), [num_rows,
 * max_pages*64] fp32 score rows and the row-group plan (about
 * (num_rows + 3*num_requests)/4 groups of 16 bytes, plus 4 bytes per row and
 * per request).  Zero-fill it once before its first use. */
DSA_API size_t dsa_indexer_prefill_workspace_bytes(int32_t num_rows, int32_t num_requests,
                                                   int32_t max_pages);

/* FP8 lightning indexer for many query rows per request (prefill, chunked
 * prefill, speculative rows): row t of request r is the decode problem
 * (q[t], weights[t], seq_lens[t], block_table[r]).
 *
 *   q_index_fp8       [num_rows, 64, 128] float8_e4m3fn, 16-byte aligned
 *   k_index_cache_fp8 as for dsa_indexer_run
 *   weights           [num_rows, 64] fp32, 16-byte aligned
 *   seq_lens          [num_rows] int32: tokens row t sees (causal rows of a
 *                     prefill chunk see growing prefixes)
 *   block_table       [num_requests, max_pages] int32
 *   cu_seqlens_q      [num_requests + 1] int32: request r owns rows
 *                     [cu_seqlens_q[r], cu_seqlens_q[r+1]); 0 and num_rows
 *                     at the ends (a violation sets DSA_DEV_BAD_SEQ_LEN)
 *   topk_indices      [num_rows, 2048] int32 output, as for dsa_indexer_run
 *
 * Rows are scored four at a time per request as one FP8 tensor-core GEMM
 * (N = 4 rows x 64 heads), so each 128-token K tile is read once per four
 * rows.  With cu_seqlens_q = 0..num_rows it computes exactly what
 * dsa_indexer_run computes.  No counterpart in the reference, whose indexer
 * definition is decode-only (one query per request). */
DSA_API int dsa_indexer_prefill_run(const void* q_index_fp8, const void* k_index_cache_fp8,
                                    int64_t num_pages, const float* weights,
                                    const int32_t* seq_lens, const int32_t* block_table,
                                    const int32_t* cu_seqlens_q, int32_t num_rows,
                                    int32_t num_requests, int32_t max_pages,
                                    int32_t* topk_indices, void* workspace, size_t workspace_bytes,
                                    void* stream);

/* Quantises new indexer keys into the paged FP8 K cache (the step before
 * dsa_indexer_run in a serving loop).
 *
 *   k                  [num_tokens, 128] bf16, 8-byte aligned
 *   slot_mapping       [num_tokens] int64 global slot ids (page*64 + token);
 *                      negative = padding, skipped
 *   k_index_cache_fp8  num_pages pages of 8448 bytes (the layout
 *                      dsa_indexer_run reads), 16-byte aligned
 *   ue8m0              non-zero: round each scale up to a power of two
 *   status             optional device word (NULL = none): DSA_DEV_BAD_INDEX
 *                      is OR-ed in for a slot >= num_pages*64 (not written)
 *
 * Per token: scale = max(1e-4, max|k|)/448 (ue8m0: 2^ceil(log2 scale)),
 * fp8 = e4m3(k/scale) round-to-nearest-even, stored at the token's row and
 * scale slot.  The reference only defines the page layout
 * (dsa_indexer/solution/triton/kernel.py:80,120-124); the arithmetic is the
 * published vLLM indexer cache writer (indexer_k_quant_and_cache). */
DSA_API int dsa_index_cache_write(const void* k, const int64_t* slot_mapping, int32_t num_tokens,
                                  void* k_index_cache_fp8, int64_t num_pages, int32_t ue8m0,
                                  uint32_t* status, void* stream);

/* Copies the sticky device status word of `workspace` to *status_out
 * (synchronising `stream`), and zeroes it when `clear` is non-zero.
 * No counterpart in the reference, which has no error channel
 * (errors there surface as Python exceptions, FAQ.md:238-240). */
DSA_API int dsa_read_device_status(void* workspace, uint32_t* status_out, int clear,
                           void* stream);

/* ---- test hook ---------------------------------------------------------
 * Arms one fault for the next call of the operator it names, made by any
 * thread of this process (the call consumes it).
 * DSA_TEST_SKIP_ARRIVAL, for the next dsa_attention_run: makes,
 * in every CTA, the producers of its second tile issue no copy and no
 * arrival for it, and every bounded wait of that launch gives up after
 * `wait_limit_ns` instead of 2 s.  The launch then ends with
 * DSA_DEV_WAIT_TIMEOUT set and its output void; every wait stays bounded and
 * the workspace's merge counters are left at zero, so the next call is
 * exact.  kind DSA_TEST_NONE disarms every armed fault.  For tests of the
 * failure path only; no counterpart in the reference. */
#define DSA_TEST_NONE         0
#define DSA_TEST_SKIP_ARRIVAL 1
/* DSA_TEST_SKIP_READY, for the next dsa_indexer_run (the no-allocation entry
 * point included): the score kernel publishes no ready count for request 0,
 * and the select's wait for a request's ready count gives up after
 * `wait_limit_ns` instead of 2 s.  The call ends with DSA_DEV_WAIT_TIMEOUT set
 * and row 0 written as all -1; the other rows are exact, and the select
 * resynchronises request 0's consumed count with its scored count, so the
 * next call is exact. */
#define DSA_TEST_SKIP_READY   2
DSA_API int dsa_b200_test_inject(int kind, uint64_t wait_limit_ns);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* DSA_B200_H_ */
