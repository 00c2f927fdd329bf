/*
 * fpv2_b200.h - C ABI of the B200 (sm_100a) FlashPrefill V2 prefill-attention path.
 *
 * Every entry point is stream-ordered and asynchronous: it validates its
 * scalar arguments, enqueues its kernels on `stream` (a cudaStream_t passed
 * as void*, NULL = legacy default stream) and returns. Nothing here
 * synchronises the host, and no entry point allocates device memory: the
 * caller owns every input, output and the stream.
 *
 * Tensors are dense, row-major, device-resident:
 *   q            [q_heads,  padded_q_len, head_dim]
 *   k, v         [kv_heads, padded_k_len, head_dim]
 *   pooled_k/v   [kv_heads, num_blocks,   head_dim]   num_blocks = padded_k_len / block_k
 *   selected     uint8 (0/1) [kv_heads, num_tiles, num_blocks], num_tiles = padded_q_len / tile_q
 *   *_ids        int32 [kv_heads, num_tiles, num_blocks]   (full-width padded lists)
 *   *_counts     int32 [kv_heads, num_tiles]
 * Query row r of q head hq belongs to KV head hq / (q_heads / kv_heads); a
 * selection tile packs the tile_q rows of all q heads of one KV head.
 *
 * Return value: FPV2_OK or an FPV2_ERR_* code; fpv2_last_error() gives the
 * message of the calling thread's last failure.
 */
#ifndef FPV2_B200_H
#define FPV2_B200_H

#include <stdint.h>

#if defined(__GNUC__)
#define FPV2_API __attribute__((visibility("default")))
#else
#define FPV2_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* element types */
#define FPV2_F16 0
#define FPV2_BF16 1
#define FPV2_F32 2

/* status codes */
#define FPV2_OK 0
#define FPV2_ERR_INVALID_ARGUMENT 1 /* a shape, pointer or scalar is out of contract */
#define FPV2_ERR_UNSUPPORTED 2      /* valid request this build cannot run (device, dtype) */
#define FPV2_ERR_CUDA 3             /* a CUDA runtime call or kernel launch failed */
#define FPV2_ERR_DEVICE_TIMEOUT 4   /* a kernel's bounded wait expired (see fpv2_device_status) */

/* Library version (major * 10000 + minor * 100 + patch). */
FPV2_API int fpv2_version(void);

/* Message of the calling thread's most recent failed call ("" if none). */
FPV2_API const char* fpv2_last_error(void);

/*
 * Kernels this library has launched in this process, all devices and threads
 * (no counterpart in the reference): the difference across a region of calls
 * is how many of the library's kernels ran there.
 */
FPV2_API int64_t fpv2_launch_count(void);

/* FPV2_OK when `device` is an sm_100 GPU this build can run on. */
FPV2_API int fpv2_device_supported(int device);

/*
 * Device status word of the current device. Kernels that give up a bounded
 * wait set a bit here instead of hanging; this call synchronises `stream`,
 * returns the word and clears it when `clear` is non-zero. Bits: 1 a bounded
 * wait expired, 2 TMEM allocation failed, 4 a split-work entry failed its
 * bounds check, 8 (debug builds only, `build.py --debug-bounds`) a block-list
 * entry, count or page index was out of range; kernels clamp such values into
 * range in every build, as the reference clips its lists.
 */
FPV2_API int fpv2_device_status(void* stream, int clear, int32_t* status_out);

/* Upper bound, in milliseconds, for any single wait inside a kernel (default 2000). */
FPV2_API int fpv2_set_wait_budget_ms(double milliseconds);

/*
 * Mean-pool the sequence axis of x [heads, length, head_dim] into blocks of
 * block_size rows: out [heads, length / block_size, head_dim].
 * The mean is exact (float64 sum), rounded to float32, then to out_dtype.
 * Replaces fpv2/selection.py:68-80 (pool_blocks).
 */
FPV2_API int fpv2_pool_blocks(const void* x, int x_dtype, int64_t heads, int64_t length,
                     int32_t head_dim, int32_t block_size, void* out, int out_dtype,
                     void* stream);

/*
 * Index stage on caller-pooled keys: selection mask [kv_heads, num_tiles, num_blocks].
 * Scores are scale * q . pooled_k in float32; per (KV head, tile) the block
 * energies sum exp(score - tile max) over the tile's fully visible blocks and
 * visible rows; a block is kept when its energy is >= alpha * max energy, and
 * sink / local-window / diagonal / dense-tail blocks are forced, all limited
 * to causally visible blocks. `offset` is the absolute key position of query
 * row 0; rows >= query_length are padding. `raw_scores` (nullable) receives
 * the unmasked scale * q . pooled_k scores [kv_heads, G, padded_q_len, num_blocks].
 * `workspace` (nullable, 256-byte aligned, `workspace_bytes` long): with
 * float32 pooled keys and 16-bit queries, a workspace of
 * fpv2_select_workspace_bytes() bytes holds the keys' three 16-bit parts so
 * the tensor cores score them at float32 precision; without it those inputs
 * are scored on the CUDA cores (same results).
 * Replaces fpv2/selection.py:109-201 (block_scores_and_select).
 */
FPV2_API int fpv2_block_select(const void* q, int q_dtype, const void* pooled_k, int k_dtype,
                      int32_t q_heads, int32_t kv_heads, int32_t padded_q_len,
                      int32_t num_blocks, int32_t head_dim, int32_t offset,
                      int32_t query_length, float scale, int32_t block_k, int32_t tile_q,
                      float alpha, int32_t sink_tokens, int32_t window_tokens,
                      int32_t last_n_blocks, uint8_t* selected, float* raw_scores,
                      void* workspace, int64_t workspace_bytes, void* stream);

/*
 * Workspace bytes that let fpv2_block_select / fpv2_index_stage score float32
 * pooled keys on the tensor cores (0 when the dtypes do not need any): three
 * 16-bit parts of the keys, [3][kv_heads][num_blocks][head_dim] in the query
 * dtype, and two ints per KV head (the head's largest magnitude and the
 * power-of-two exponent that scales a head beyond the 16-bit range into it;
 * the head's scores are scaled back). No
 * counterpart in the reference (reference.py:45-51 scores float32 pooled keys
 * with MLX's einsum).
 */
FPV2_API int64_t fpv2_select_workspace_bytes(int q_dtype, int k_dtype, int32_t kv_heads,
                                    int32_t num_blocks, int32_t head_dim);

/*
 * Mask -> padded block lists. selected_ids lists the selected blocks
 * ascending followed by every other block ascending; pruned_ids likewise for
 * the blocks that are not selected and end (clamped to key_length) at or
 * before the tile's first query position.
 * Replaces fpv2/kernel.py:141-184 (compact_block_indices).
 */
FPV2_API int fpv2_compact_block_indices(const uint8_t* selected, int32_t kv_heads, int32_t num_tiles,
                               int32_t num_blocks, int32_t block_k, int32_t tile_q,
                               int32_t offset, int32_t query_length, int32_t key_length,
                               int32_t* selected_ids, int32_t* selected_counts,
                               int32_t* pruned_ids, int32_t* pruned_counts, void* stream);

/*
 * Fused index stage of the attention hook: pools K and V into pooled_k /
 * pooled_v (written as `pooled_dtype`: the input dtype, as fpv2/patch.py:137-138
 * pools, or FPV2_F32, as fpv2/reference.py:45-48 pools), selects on those
 * pooled keys and writes the four list/count arrays. `selected` (nullable)
 * also receives the mask. `workspace` as for fpv2_block_select (used when
 * pooled_dtype is FPV2_F32 and the inputs are 16-bit).
 * Replaces the pool_blocks x2 -> block_scores_and_select -> compact_block_indices
 * sequence of fpv2/patch.py:137-153.
 */
FPV2_API int fpv2_index_stage(const void* q, const void* k, const void* v, int dtype,
                     int32_t q_heads, int32_t kv_heads, int32_t padded_q_len,
                     int32_t padded_k_len, int32_t head_dim, int32_t offset,
                     int32_t query_length, int32_t key_length, float scale,
                     int32_t block_k, int32_t tile_q, float alpha, int32_t sink_tokens,
                     int32_t window_tokens, int32_t last_n_blocks, int pooled_dtype,
                     void* pooled_k, void* pooled_v, int32_t* selected_ids,
                     int32_t* selected_counts, int32_t* pruned_ids, int32_t* pruned_counts,
                     uint8_t* selected, void* workspace, int64_t workspace_bytes,
                     void* stream);

/*
 * Block-sparse attention over the lists: per query row, online softmax in
 * base 2 over the selected blocks (causal and key_length masked), then, when
 * mean_correction is set, the pruned blocks as pooled K/V entries with logits
 * shifted by log2(block_k). q/k/v/out share `dtype` (FPV2_F16 or FPV2_BF16);
 * pooled_k/pooled_v are `pooled_dtype` (dtype or FPV2_F32) and are rounded
 * to `dtype` on load. Ids are clipped to [0, num_blocks-1] and counts to
 * [0, num_blocks]; the pruned ids of a tile are treated as a set.
 * Rows >= query_length are padding; their output is unspecified.
 * `workspace` (nullable) is caller-owned device scratch of at least
 * FPV2_ATTN_WORKSPACE_BYTES: the kernel's work-queue counter, rewritten on
 * `stream` by every call (calls sharing one workspace must be stream-ordered).
 * Without it the work is distributed statically (same results, slower). A
 * 256-byte aligned workspace of fpv2_attention_workspace_bytes() bytes also
 * holds, for bf16 inputs, an exact fp16 copy of V so that P is held at fp16
 * precision in the P.V product (11 significant bits instead of bf16's 8), and
 * the partial results of long work items, which are then split into segments
 * over the GPU; smaller workspaces run without either (results within the
 * same output tolerance, slightly less precise).
 * Replaces fpv2/kernel.py:441-590 (sparse_attention) and its Metal kernel
 * fpv2/kernel.py:187-414.
 */
#define FPV2_ATTN_WORKSPACE_BYTES 16
FPV2_API int fpv2_sparse_attention(const void* q, const void* k, const void* v, const void* pooled_k,
                          const void* pooled_v, int pooled_dtype,
                          const int32_t* selected_ids, const int32_t* selected_counts,
                          const int32_t* pruned_ids, const int32_t* pruned_counts, int dtype,
                          int32_t q_heads, int32_t kv_heads, int32_t padded_q_len,
                          int32_t padded_k_len, int32_t head_dim, int32_t offset,
                          int32_t query_length, int32_t key_length, float scale,
                          int32_t block_k, int32_t tile_q, int32_t mean_correction,
                          void* out, void* workspace, int64_t workspace_bytes,
                          void* stream);

/*
 * Workspace size for fpv2_sparse_attention / _multicast / _paged that enables
 * (a) for bf16 inputs, the fp16 P.V product on an exact fp16 copy of V (the
 * reference multiplies a float32 P by V upcast to float32, fpv2/kernel.py:
 * 234-235, 322; fp16 P comes 8x closer to that than bf16 P), and (b) the split
 * of long work items (the dense-tail tiles that walk every key block) into
 * segments spread over the SMs. Any smaller workspace of at least
 * FPV2_ATTN_WORKSPACE_BYTES runs without them. Never smaller than
 * FPV2_ATTN_WORKSPACE_BYTES. No counterpart in the reference.
 */
FPV2_API int64_t fpv2_attention_workspace_bytes(int dtype, int32_t q_heads, int32_t kv_heads,
                                       int32_t padded_q_len, int32_t padded_k_len,
                                       int32_t head_dim, int32_t block_k, int32_t tile_q,
                                       int pooled_dtype, int32_t mean_correction);

/*
 * fpv2_sparse_attention for the head-parallel multi-GPU layer, with the output
 * all-gather fused into the kernel (no counterpart in the reference, which runs
 * on one device; it replaces the NCCL all-gather that reassembles the layer
 * output). `out_multicast` is the NVLink multicast address of a full output
 * [heads_total, padded_q_len, head_dim] buffer bound on every rank (for
 * example torch symmetric memory); this call's query head hq is written to
 * head `head_offset + hq` of every rank's buffer as each output tile
 * completes, with 16-byte multimem stores. Needs the tcgen05 path (bf16/fp16,
 * head_dim 64, 96, 128 or 256, 16-byte aligned pointers), else FPV2_ERR_UNSUPPORTED.
 * The caller orders the ranks around the call (a cross-rank barrier after it
 * before reading the buffer, and before reusing it).
 */
FPV2_API int fpv2_sparse_attention_multicast(
    const void* q, const void* k, const void* v, const void* pooled_k, const void* pooled_v,
    int pooled_dtype, const int32_t* selected_ids, const int32_t* selected_counts,
    const int32_t* pruned_ids, const int32_t* pruned_counts, int dtype, int32_t q_heads,
    int32_t kv_heads, int32_t padded_q_len, int32_t padded_k_len, int32_t head_dim,
    int32_t offset, int32_t query_length, int32_t key_length, float scale, int32_t block_k,
    int32_t tile_q, int32_t mean_correction, void* out_multicast, int32_t head_offset,
    int32_t heads_total, void* workspace, int64_t workspace_bytes, void* stream);

/*
 * fpv2_sparse_attention for callers that cannot allocate device memory (no
 * counterpart in the reference). Same arguments as fpv2_sparse_attention
 * without the workspace, and the results that call gives with a workspace of
 * FPV2_NOALLOC_SCRATCH_BYTES: the kernel's work-queue counter
 * lives in a FPV2_NOALLOC_SCRATCH_BYTES array compiled into the library, held
 * by every GPU that loads it until exit. Every call on a device shares that
 * array (it is cleared on `stream` before each launch), so calls that overlap
 * on the GPU race. The first call on a device looks up the array's address;
 * make it before any stream capture, and do not use the library across a
 * cudaDeviceReset of that device (the cached address would be stale). The
 * scratch holds no fp16 copy of V and no split results (see
 * fpv2_attention_workspace_bytes), so bf16 inputs keep P in bf16 here; the
 * output stays within the same tolerance. Problems with more than
 * FPV2_NOALLOC_MAX_WORK_ITEMS work items (128-row chunks of selection tiles)
 * are rejected with FPV2_ERR_INVALID_ARGUMENT.
 */
#define FPV2_NOALLOC_SCRATCH_BYTES 256
#define FPV2_NOALLOC_MAX_WORK_ITEMS (1 << 24)
FPV2_API int fpv2_sparse_attention_noalloc(
    const void* q, const void* k, const void* v, const void* pooled_k, const void* pooled_v,
    int pooled_dtype, const int32_t* selected_ids, const int32_t* selected_counts,
    const int32_t* pruned_ids, const int32_t* pruned_counts, int dtype, int32_t q_heads,
    int32_t kv_heads, int32_t padded_q_len, int32_t padded_k_len, int32_t head_dim,
    int32_t offset, int32_t query_length, int32_t key_length, float scale, int32_t block_k,
    int32_t tile_q, int32_t mean_correction, void* out, void* stream);

/*
 * Paged K/V (no counterpart in the reference, whose MLX KV cache is one
 * contiguous array; this is the serving-side form of the same call): k_pages
 * and v_pages are page pools [num_pages, page_size, kv_heads, head_dim] in the
 * token-major layout of paged KV caches, and key position p of the sequence is
 * row p % page_size of page block_table[p / page_size] (table_len entries,
 * covering padded_k_len). The block lists, pooled K/V and every other argument
 * are those of fpv2_sparse_attention (lists hold logical block indices).
 * Needs the tcgen05 path: bf16/fp16, head_dim 64/96/128, block_k a multiple of
 * 128, page_size a multiple of 8 that divides 128 or is a multiple of 128;
 * else FPV2_ERR_UNSUPPORTED. Out-of-range table entries are clamped.
 */
FPV2_API int fpv2_sparse_attention_paged(
    const void* q, const void* k_pages, const void* v_pages, const int32_t* block_table,
    int32_t table_len, int32_t num_pages, int32_t page_size, const void* pooled_k,
    const void* pooled_v, int pooled_dtype, const int32_t* selected_ids,
    const int32_t* selected_counts, const int32_t* pruned_ids, const int32_t* pruned_counts,
    int dtype, int32_t q_heads, int32_t kv_heads, int32_t padded_q_len, int32_t padded_k_len,
    int32_t head_dim, int32_t offset, int32_t query_length, int32_t key_length, float scale,
    int32_t block_k, int32_t tile_q, int32_t mean_correction, void* out, void* workspace,
    int64_t workspace_bytes, void* stream);

/*
 * fpv2_pool_blocks for a sequence held in a page pool (see
 * fpv2_sparse_attention_paged): out [kv_heads, length / block_size, head_dim]
 * in out_dtype, with the same exact-mean definition. The pool is bf16/fp16,
 * head_dim a multiple of 8.
 */
FPV2_API int fpv2_pool_pages(const void* pages, const int32_t* block_table, int32_t table_len,
                             int32_t num_pages, int32_t page_size, int32_t kv_heads,
                             int32_t head_dim, int32_t length, int32_t block_size, int dtype,
                             void* out, int out_dtype, void* stream);

/*
 * Which kernel family the two stages would use for this shape:
 * bit 0 set = tcgen05 index stage, bit 1 set = tcgen05 attention
 * (otherwise the generic CUDA-core kernels run), bit 2 set = the attention
 * takes two 128-row chunks of a selection tile per K/V stream (tiles of
 * several chunks at the same query positions).
 */
FPV2_API int fpv2_fast_path_mask(int dtype, int32_t q_heads, int32_t kv_heads, int32_t head_dim,
                        int32_t block_k, int32_t tile_q, int32_t num_blocks);

/*
 * Test hook for failure detection: launches one CTA that waits on an
 * mbarrier nothing ever arrives at, with a budget of `budget_ms`. Returns
 * FPV2_ERR_DEVICE_TIMEOUT (and leaves the context usable) when the bounded
 * wait gave up as designed.
 */
FPV2_API int fpv2_selftest_wait_timeout(double budget_ms, void* stream);

#ifdef __cplusplus
}
#endif

#endif /* FPV2_B200_H */
