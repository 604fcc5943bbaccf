/*
 * memopt_b200.h — C-ABI of the B200 (sm_100a) KV-cache data plane.
 *
 * Every entry point takes plain pointers and sizes; no PyTorch types cross
 * this boundary.  Device pointers must point to memory of the device that is
 * current on the calling thread.  `stream` is a cudaStream_t passed as void*
 * (NULL = legacy default stream).  All kernel entry points are asynchronous
 * with respect to the host: they enqueue work on `stream` and return a
 * status code describing argument validation and launch errors only.
 *
 * Reference interfaces replaced (paths relative to the reference project
 * TheRadDani/memopt-transformer-runtime):
 *   pool / free-list ........ src/csrc/kv_cache.cu:83-201, kv_cache.h:24-54
 *   write_cache ............. src/csrc/kv_cache.cu:228-348, kv_cache.h:69-73
 *   evict_cache ............. src/csrc/kv_cache.cu:379-559, kv_cache.h:88-92
 *   evict_tokens ............ src/csrc/kv_cache.cu:609-1156, kv_cache.h:117-122
 *   quantize / dequantize ... src/csrc/quantization.cu:104-428, quantization.h:22,35
 *   dynamic_sparse_attention  src/csrc/attention.cu:98-521, attention.h:21-29
 * The Python-facing module `memopt_C` (src/csrc/extension.cpp:10-124) is a
 * thin wrapper that validates tensors and forwards to these functions.
 */
#ifndef MEMOPT_B200_H
#define MEMOPT_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif
#ifdef __cplusplus
extern "C" {
#endif

/* ------------------------------------------------------------------------ */
/* Status codes                                                               */
/* ------------------------------------------------------------------------ */
#define MEMOPT_OK                    0
#define MEMOPT_ERR_INVALID_ARG      (-1)
#define MEMOPT_ERR_NOT_INITIALIZED  (-2)
#define MEMOPT_ERR_UNSUPPORTED      (-3)
#define MEMOPT_ERR_CUDA             (-4)
#define MEMOPT_ERR_OUT_OF_RANGE     (-5)
#define MEMOPT_ERR_WORKSPACE        (-6)
#define MEMOPT_ERR_TIMEOUT          (-7)

/* Version of this ABI (bumped on any signature change). */
int memopt_abi_version(void);
/* Static description of a status code. */
const char* memopt_status_string(int status);
/* Human-readable message of the last failing call on this host thread. */
const char* memopt_last_error(void);

/* ------------------------------------------------------------------------ */
/* Page pool free-list (host side).                                           */
/* Replaces KVCachePool / init_pool / allocate_block / free_block /           */
/* free_blocks_count (kv_cache.cu:83-201).  The pool's device memory is owned */
/* by the caller (the Python module allocates it with the caching allocator); */
/* this library keeps the FIFO free-list and the pool geometry.               */
/* ------------------------------------------------------------------------ */

/* (Re)initialise the free-list with blocks 0..num_blocks-1 in FIFO order.
 * Returns MEMOPT_OK, or MEMOPT_ERR_INVALID_ARG (the pool is then left
 * uninitialised).  Same geometry as the live pool -> no-op (kv_cache.cu:116). */
int memopt_pool_init(int num_blocks, int block_size, int num_heads, int head_dim);
/* Drop the pool: afterwards every pool call reports NOT_INITIALIZED. */
void memopt_pool_reset(void);
int memopt_pool_is_initialized(void);
/* Writes the live geometry; NOT_INITIALIZED when there is no pool. */
int memopt_pool_config(int* num_blocks, int* block_size, int* num_heads, int* head_dim);
/* Pops the oldest free block: >=0 on success, -1 when exhausted,
 * MEMOPT_ERR_NOT_INITIALIZED (-2) without a pool (kv_cache.cu:163-172). */
int memopt_pool_allocate_block(void);
/* Pushes a block back (kv_cache.cu:179-185): OK, NOT_INITIALIZED or OUT_OF_RANGE. */
int memopt_pool_free_block(int block_idx);
/* Number of free blocks, 0 without a pool (kv_cache.cu:198-201). */
int memopt_pool_free_blocks_count(void);

/* ------------------------------------------------------------------------ */
/* Pages spread over several GPUs (no reference counterpart: the reference's  */
/* pool lives on one device, kv_cache.cu:97 and README "Future Work").  A     */
/* page is (owner device, block).  Host-side, process-wide; every rank of an  */
/* SPMD job makes the same calls and so holds the same state.                 */
/* ------------------------------------------------------------------------ */

/* One FIFO free-list per device with blocks 0..blocks_per_device[d]-1. */
int memopt_mdpool_init(int num_devices, const int* blocks_per_device);
void memopt_mdpool_reset(void);
/* Oldest free block of preferred_device, else of the device with the most
 * free blocks (lowest index on ties); writes the owner to *device_out.
 * Returns the block, -1 when every device is exhausted, or an error code. */
int memopt_mdpool_allocate(int preferred_device, int* device_out);
/* Returns a block to its device's free-list (INVALID_ARG if already free). */
int memopt_mdpool_free(int device, int block);
int memopt_mdpool_free_count(int device);
/* Gather plan of n pages (page_dev/page_blk; blk < 0 = no page) for
 * home_device: local_blk[i] is the block to read on the home device: its own
 * block for pages it owns, else a staging block staging_base + k.  Each
 * distinct remote page gets one copy k (copy_src_dev/blk -> copy_dst_blk),
 * grouped by owner in device order, so the pages of one owner land in
 * consecutive staging blocks.  Copy arrays hold up to n entries.
 * MEMOPT_ERR_WORKSPACE when more than staging_capacity pages are remote. */
int memopt_mdpool_plan(const int32_t* page_dev, const int32_t* page_blk, int n, int home_device,
                       int staging_base, int staging_capacity, int32_t* local_blk, int32_t* copy_src_dev,
                       int32_t* copy_src_blk, int32_t* copy_dst_blk, int* n_copies);
/* Device page copy on the current device: dst[dst_ids[i]] = src[src_ids[i]]
 * for num_pages pages of page_bytes (a multiple of 16) each; NULL ids mean
 * 0..num_pages-1 (a packed buffer); negative ids are skipped.  Packs pages
 * for a transfer between GPUs and unpacks them. */
int memopt_copy_pages(const void* src_pool, const int32_t* src_ids, void* dst_pool, const int32_t* dst_ids,
                      int num_pages, int64_t page_bytes, void* stream);

/* ------------------------------------------------------------------------ */
/* write_cache (kv_cache.cu:228-348).                                         */
/* keys/values: fp16 [num_tokens, num_heads, head_dim], contiguous.           */
/* slot_mapping: int32 [num_tokens], slot = block * block_size + position.    */
/* Slots outside [0, num_blocks*block_size) are skipped (the reference writes */
/* out of bounds); when `bad_slot_count` (device int32, nullable) is given,   */
/* the kernel atomically adds the number of skipped tokens to it.             */
/* ------------------------------------------------------------------------ */

/* fp16 pool, reference layout [num_blocks, block_size, num_heads, head_dim]. */
int memopt_write_cache_f16(const void* keys, const void* values,
                           const int32_t* slot_mapping, int64_t num_tokens,
                           int num_heads, int head_dim,
                           void* key_pool, void* value_pool,
                           int64_t num_blocks, int block_size,
                           int32_t* bad_slot_count, void* stream);

/* INT4 pool with on-the-fly quantisation (new page format, no reference
 * counterpart for the fused op; the codes follow quantization.cu:129-202).
 * kv_pages: uint8 [num_blocks, num_heads, page_bytes], one contiguous page per
 * (block, head) laid out as
 *   K codes  [block_size][head_dim/2]   (byte i of a row = q[2i] | q[2i+1] << 4)
 *   V codes  [block_size][head_dim/2]   same bytes; for head_dim 128 byte i of
 *                                        row pos is stored at i ^ 32 when bit 1
 *                                        of pos is set
 *   K scales [block_size][head_dim/64]  fp16
 *   V scales [block_size/16][head_dim/64][16] fp16, token r of a 16-token tile
 *                                        at slot 2(r&3) + ((r>>2)&1) + 8(r>>3)
 * page_bytes = memopt_int4_page_bytes(block_size, head_dim).  Groups are 64
 * consecutive head_dim elements of one (token, head); the code is computed
 * from the fp32 scale absmax/7 (1.0 for an all-zero group) and the stored
 * scale is that fp32 scale rounded to fp16.  head_dim % 64 == 0 and
 * block_size % 16 == 0.  The V permutations serve the decode kernel's
 * conflict-free shared-memory fragment loads; every token still owns whole
 * 32-byte sectors of its K and V rows. */
size_t memopt_int4_page_bytes(int block_size, int head_dim);
int memopt_write_cache_int4(const void* keys, const void* values,
                            const int32_t* slot_mapping, int64_t num_tokens,
                            int num_heads, int head_dim, uint8_t* kv_pages,
                            int64_t num_blocks, int block_size,
                            int32_t* bad_slot_count, void* stream);

/* ------------------------------------------------------------------------ */
/* INT4 quantize / dequantize (quantization.cu:104-203, 232-270, 294-428).    */
/* Groups of `group_size` (must be 64) consecutive elements of the flat input.*/
/* ------------------------------------------------------------------------ */
int memopt_quantize_int4(const void* input_f16, int64_t numel, int group_size,
                         uint8_t* packed, float* scales, void* stream);
/* numel = number of fp16 outputs; numel / group_size groups are written.     */
int memopt_dequantize_int4(const uint8_t* packed, const float* scales,
                           int64_t numel, int group_size,
                           void* output_f16, void* stream);

/* ------------------------------------------------------------------------ */
/* evict_tokens (kv_cache.cu:640-1156): per (sequence, head) Ada-KV eviction  */
/* with the reference's exact 32-step fp32 bisection threshold, sink boost,   */
/* partial zeroing of evicted rows and per-block vote/unlink.                 */
/* scores: fp32 [num_seqs, num_heads, seq_len]; block_tables int32           */
/* [num_seqs, max_blocks_per_seq] (mutated); is_block_free int32              */
/* [total_pool_blocks] (mutated); key/value pool fp16 in reference layout.    */
/* Optional compaction outputs (nullable): retained_idx int32                 */
/* [num_seqs, num_heads, seq_len] — ascending indices of the kept tokens,     */
/* padded with -1 — and retained_count int32 [num_seqs, num_heads].          */
/* seq_len <= 32768 (the reference stops at 4096).                            */
/* ------------------------------------------------------------------------ */
int memopt_evict_tokens(const float* scores, int num_seqs, int num_heads, int seq_len,
                        int32_t* block_tables, int max_blocks_per_seq,
                        int32_t* is_block_free, int total_pool_blocks,
                        void* key_pool, void* value_pool,
                        int pool_num_blocks, int block_size, int head_dim,
                        float retain_ratio, int num_sink_tokens,
                        int32_t* retained_idx, int32_t* retained_count,
                        void* stream);

/* ------------------------------------------------------------------------ */
/* Exact sink-aware top-k eviction with compaction (new; the reference's      */
/* evict_tokens frees no memory).  Per sequence b: token score = sum over     */
/* heads of scores[b, h, t] (fp32, heads in order); tokens < num_sink_tokens  */
/* are always kept; tokens at/after context_lens[b] or on a page whose entry  */
/* is < 0 or >= pool_num_blocks are never kept; keep = max(1, min(L,         */
/* ceil(r*L))) over the L valid tokens; the keep largest survive (ties: lower */
/* index first; NaN lowest).  Their K/V rows (all heads) move in token order  */
/* to positions 0..keep-1 over the sequence's valid pages; block_tables[b]    */
/* becomes the first ceil(keep/block_size) valid pages then -1, the other     */
/* valid pages are listed in freed_pages[b] (freed_count[b] of them, -1 pad)  */
/* for the caller to release; context_lens[b] = keep.                          */
/* scores fp32 [num_seqs, num_heads, max_len]; kept_idx int32 [num_seqs,      */
/* max_len] (ascending original indices, -1 pad); kept_count int32            */
/* [num_seqs]; freed_pages int32 [num_seqs, max_blocks_per_seq]; freed_count  */
/* int32 [num_seqs].  max_blocks_per_seq <= 16384 and <= max(2048, max_len)  */
/* (sequences beyond 32768 tokens or 2048 pages use a streaming select); fp16 */
/* pools in reference layout; a physical page appears at most once in the   */
/* tables.  Rows move in place.  The workspace (16-byte aligned,               */
/* memopt_evict_topk_workspace_size() bytes: about 20 B per token, no K/V    */
/* rows) holds tables, ordinals and move flags.                                */
/* ------------------------------------------------------------------------ */
size_t memopt_evict_topk_workspace_size(int num_seqs, int max_len, int num_heads, int head_dim);
int memopt_evict_topk_compact(const float* scores, int num_seqs, int num_heads, int max_len,
                              int32_t* block_tables, int max_blocks_per_seq, int32_t* context_lens,
                              void* key_pool, void* value_pool, int pool_num_blocks, int block_size,
                              int head_dim, float retain_ratio, int num_sink_tokens,
                              int32_t* kept_idx, int32_t* kept_count, int32_t* freed_pages,
                              int32_t* freed_count, void* workspace, size_t workspace_bytes,
                              void* stream);

/* The same operator on an INT4 pool: kv_pages [pool_num_blocks][num_heads]   */
/* [page bytes] as written by write_cache (head_dim 64 or 128, block_size a   */
/* multiple of 16, <= 64 heads); each kept token's codes and scales move with */
/* it (the position-dependent V row and V scale layout re-laid out).          */
int memopt_evict_topk_compact_int4(const float* scores, int num_seqs, int num_heads, int max_len,
                                   int32_t* block_tables, int max_blocks_per_seq, int32_t* context_lens,
                                   uint8_t* kv_pages, int pool_num_blocks, int block_size, int head_dim,
                                   float retain_ratio, int num_sink_tokens, int32_t* kept_idx, int32_t* kept_count,
                                   int32_t* freed_pages, int32_t* freed_count, void* workspace,
                                   size_t workspace_bytes, void* stream);

/* Outcome of the last evict_topk_compact* call that used `workspace` on
 * `stream` (no reference counterpart).  Synchronises the stream.  Every row
 * move waits, with a bound, for the rows at its destination to be read; a
 * wait that runs out skips that row's store (the destination keeps its old
 * contents, so no kept row is overwritten before it is read) and is reported
 * here as MEMOPT_ERR_TIMEOUT: the pool, block tables and lengths are then
 * only partly compacted. */
int memopt_evict_topk_status(const void* workspace, int num_seqs, int max_len, void* stream);
/* Test hook (process-wide): bound of the row movers' flag waits in polls
 * (0 = the default, over a second) and, when withhold_read_flags != 0, movers
 * that never publish their "read" flags, so that every wait on one runs out.
 * Only for testing the failure path above. */
int memopt_evict_topk_set_test_hooks(uint32_t flag_poll_limit, int withhold_read_flags);

/* Head-sharded form of the same operator (the one cross-GPU exchange of the  */
/* data plane): with the heads of every sequence split over G ranks, rank r   */
/* writes the fp32 sum of its own heads' scores (heads in order) with         */
/* memopt_evict_topk_head_sum -> sums [num_seqs, max_len]; the G rows are      */
/* exchanged (an all-gather) into partial_sums [G, num_seqs, max_len] in rank */
/* order, and memopt_evict_topk_compact_parts ranks tokens by the fp32 sum of */
/* the G parts in rank order, then compacts this rank's pool (num_heads =     */
/* the heads this rank holds).  All ranks reach the same decision; with G = 1 */
/* the result equals memopt_evict_topk_compact's bit for bit.                  */
int memopt_evict_topk_head_sum(const float* scores, int num_seqs, int num_heads, int max_len,
                               float* sums, void* stream);
int memopt_evict_topk_compact_parts(const float* partial_sums, int num_parts, int num_seqs, int max_len,
                                    int32_t* block_tables, int max_blocks_per_seq, int32_t* context_lens,
                                    void* key_pool, void* value_pool, int pool_num_blocks, int block_size,
                                    int num_heads, int head_dim, float retain_ratio, int num_sink_tokens,
                                    int32_t* kept_idx, int32_t* kept_count, int32_t* freed_pages,
                                    int32_t* freed_count, void* workspace, size_t workspace_bytes,
                                    void* stream);

/* ------------------------------------------------------------------------ */
/* evict_cache (kv_cache.cu:379-559): per (physical block, head) keep the     */
/* max(1, (int)(r*block_size)) highest scores, zero the full head rows of the */
/* rest.  scores fp32 [num_blocks, block_size, num_heads].                    */
/* ------------------------------------------------------------------------ */
int memopt_evict_cache(const float* scores, int num_blocks, int block_size,
                       int num_heads, int head_dim,
                       void* key_pool, void* value_pool,
                       float retain_ratio, void* stream);

/* ------------------------------------------------------------------------ */
/* dynamic_sparse_attention (attention.cu:98-521).                            */
/* out[b,q,h,:] = softmax(q.K^T / sqrt(head_dim)) V over the tokens           */
/* [max(0, ctx_b - W), ctx_b) of every logical page whose block-table entry   */
/* is >= 0 (and < num_blocks); no causal mask; W = max_seq_len when           */
/* window_size <= 0 or > max_seq_len; rows with no visible token are 0.       */
/* query/out fp16 [batch, q_len, num_heads, head_dim]; head_dim in {64,128};  */
/* block_size in {16,32}.  `workspace` holds split-K partials and tickets:    */
/* size it with memopt_paged_attention_workspace_size(); its first            */
/* memopt_paged_attention_ticket_bytes() bytes must be zero before the first  */
/* use and every completed call leaves them zero again.                       */
/* ------------------------------------------------------------------------ */
size_t memopt_paged_attention_workspace_size(int batch, int q_len, int num_heads,
                                             int head_dim, int max_blocks_per_seq,
                                             int block_size, int max_seq_len,
                                             int window_size);
/* The same for the _ex entry points: pools holding num_kv_heads heads.      */
size_t memopt_paged_attention_workspace_size_ex(int batch, int q_len, int num_heads, int num_kv_heads,
                                                int head_dim, int max_blocks_per_seq, int block_size,
                                                int max_seq_len, int window_size);
/* Workspace of memopt_paged_attention_int4 / _int4_ex: the size above plus,  */
/* for q_len >= 64 (head_dim 64/128, block_size 16/32), an fp16 scratch of   */
/* batch * max_blocks_per_seq pages into which the call dequantises the      */
/* sequences' INT4 pages before running the tcgen05 prefill kernel on them,  */
/* as the reference dequantises an INT4 cache before fp16 attention          */
/* (quantization.cu:371-428 -> attention.cu:371-521).  Ticket rules as above; */
/* such calls need a 256-byte aligned workspace (cudaMalloc's alignment).    */
size_t memopt_paged_attention_int4_workspace_size_ex(int batch, int q_len, int num_heads, int num_kv_heads,
                                                     int head_dim, int max_blocks_per_seq, int block_size,
                                                     int max_seq_len, int window_size);
/* Bytes at the start of the workspace that hold tickets (must start zeroed). */
size_t memopt_paged_attention_ticket_bytes(int batch, int q_len, int num_heads);

/* fp16 pool, reference layout [num_blocks, block_size, num_heads, head_dim]. */
int memopt_paged_attention_f16(const void* query, const void* key_pool,
                               const void* value_pool,
                               const int32_t* block_tables,
                               const int32_t* context_lens,
                               int batch, int q_len, int num_heads, int head_dim,
                               int max_blocks_per_seq, int64_t num_blocks,
                               int block_size, int max_seq_len, int window_size,
                               void* out, void* workspace, size_t workspace_bytes,
                               void* stream);

/* Extended attention (no reference counterpart for the options):          */
/* num_kv_heads divides num_heads; the pools (fp16 [NB, BS, num_kv_heads, D]  */
/* or INT4 pages [NB, num_kv_heads, page_bytes]) hold num_kv_heads heads and  */
/* query head h reads KV head h / (num_heads / num_kv_heads) (grouped-query   */
/* attention).  causal != 0: query row i of the q_len rows is the token at    */
/* ctx - q_len + i and sees [max(0, c_i - W), c_i) with c_i = ctx - q_len +   */
/* i + 1.  num_kv_heads == num_heads and causal == 0 is exactly the call      */
/* above.  The workspace size is the same.                                    */
int memopt_paged_attention_f16_ex(const void* query, const void* key_pool,
                                  const void* value_pool, const int32_t* block_tables,
                                  const int32_t* context_lens, int batch, int q_len,
                                  int num_heads, int num_kv_heads, int head_dim,
                                  int max_blocks_per_seq, int64_t num_blocks, int block_size,
                                  int max_seq_len, int window_size, int causal, void* out,
                                  void* workspace, size_t workspace_bytes, void* stream);
int memopt_paged_attention_int4_ex(const void* query, const uint8_t* kv_pages,
                                   const int32_t* block_tables, const int32_t* context_lens,
                                   int batch, int q_len, int num_heads, int num_kv_heads,
                                   int head_dim, int max_blocks_per_seq, int64_t num_blocks,
                                   int block_size, int max_seq_len, int window_size, int causal,
                                   void* out, void* workspace, size_t workspace_bytes,
                                   void* stream);

/* No counterpart in the reference.  Same as memopt_paged_attention_f16, but
 * for callers that cannot allocate device memory at call time (hosts with
 * their own allocator-free runtime, or steps where allocator calls are not
 * allowed): the split-K scratch is a fixed 4 MiB array inside this library's
 * device image, so the call allocates nothing.  Calls needing more scratch
 * than memopt_paged_attention_noalloc_max_bytes() return
 * MEMOPT_ERR_WORKSPACE; calls with invalid arguments are rejected before the
 * scratch is touched.  The first call on a device looks up the array's
 * address; CUDA loads the module that holds the array lazily, so that first
 * call is also when the 4 MiB are committed on that device and it can fail
 * with an out-of-memory error (MEMOPT_ERR_CUDA): make it at start-up, before
 * any stream capture.  From then on the array stays on that GPU until the
 * process exits.  All calls share the array: calls that overlap on the GPU
 * race.  The ticket region is cleared at the start of every call. */
size_t memopt_paged_attention_noalloc_max_bytes(void);
int memopt_paged_attention_f16_noalloc(const void* query, const void* key_pool,
                                       const void* value_pool,
                                       const int32_t* block_tables,
                                       const int32_t* context_lens,
                                       int batch, int q_len, int num_heads, int head_dim,
                                       int max_blocks_per_seq, int64_t num_blocks,
                                       int block_size, int max_seq_len, int window_size,
                                       void* out, void* stream);

/* INT4 pool written by memopt_write_cache_int4 (kv_pages as described
 * there); K/V element value is (code - 8) * float(scale_fp16), dequantised
 * inside the kernel. */
int memopt_paged_attention_int4(const void* query, const uint8_t* kv_pages,
                                const int32_t* block_tables,
                                const int32_t* context_lens,
                                int batch, int q_len, int num_heads, int head_dim,
                                int max_blocks_per_seq, int64_t num_blocks,
                                int block_size, int max_seq_len, int window_size,
                                void* out, void* workspace, size_t workspace_bytes,
                                void* stream);

#ifdef __cplusplus
}
#endif
#if defined(__GNUC__)
#pragma GCC visibility pop
#endif
#endif /* MEMOPT_B200_H */
