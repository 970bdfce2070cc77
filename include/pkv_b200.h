/*
 * pkv_b200.h -- C ABI of the B200 paged-KV library (libpkv_b200.so).
 *
 * The library implements AgentRL's paged-KV hot path: the block allocator and
 * its block tables (host C++), and the device kernels for sm_100a that append
 * K/V into pages, gather pages back into contiguous caches, run paged GQA
 * decode attention, chunked-prefill and speculative-verify attention over
 * pages, and apply copy-on-write forks and frees to the device block tables.
 *
 * The reference (AgentRL, Python) has no native code, so there is no existing
 * FFI to keep; each entry point below names the Python call it replaces.  The
 * Python package `randomrepo_b200` binds these through ctypes and exposes the
 * reference's own classes (`PagedKVAllocator`, `PagedKVCacheStore`,
 * `PagedKVSequenceView`) on top.
 *
 * Conventions
 *  - Every function returns a status (0 = success).  On failure
 *    pkv_last_error() returns a message for the calling thread.  The status
 *    tells the binding which Python exception the reference raises:
 *    PKV_ERR_VALUE -> ValueError, PKV_ERR_KEY -> KeyError,
 *    PKV_ERR_RUNTIME -> RuntimeError, PKV_ERR_INDEX -> IndexError.
 *  - Device pointers are plain CUDA device addresses; `stream` is a
 *    cudaStream_t passed as void* (NULL = legacy default stream).  Kernels are
 *    asynchronous on that stream and never synchronize the host.
 *  - KV pool layout (one allocation for all layers):
 *        pool[layer][block][kv_head][state(0=K,1=V)][slot][head_dim]
 *    The K (or V) rows of one block and one KV head form a "page"; the pages
 *    of one block are contiguous.  When a row is a multiple of 128 bytes and
 *    block_size a multiple of 8, each page is stored pre-swizzled: cut into
 *    128-byte column slabs, each slab holding the page's rows at 128 bytes
 *    apiece with the 16-byte chunks of row t permuted by XOR (t mod 8) (the
 *    layout TMA's 128-byte swizzle produces).  Otherwise pages are row-major.
 *    Read and write the pool through pkv_scatter_tokens / pkv_gather_tokens.
 *  - Block tables: int32 [rows][table_stride]; row r belongs to the sequence
 *    the allocator mapped to row r; entries past the sequence's block count
 *    are unspecified.  Context lengths: int32 [rows].
 */
#ifndef PKV_B200_H
#define PKV_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* The library is built with hidden visibility; everything declared here is
 * exported. */
#if defined(__GNUC__)
#pragma GCC visibility push(default)
#endif

enum pkv_status {
  PKV_OK = 0,
  PKV_ERR_VALUE = 1,    /* ValueError in the reference */
  PKV_ERR_KEY = 2,      /* KeyError */
  PKV_ERR_RUNTIME = 3,  /* RuntimeError (pool exhausted) */
  PKV_ERR_INDEX = 4,    /* IndexError (logical block past the table) */
  PKV_ERR_ARG = 5,      /* invalid argument to a kernel entry point */
  PKV_ERR_CUDA = 6,     /* CUDA launch / runtime error */
  PKV_ERR_UNSUPPORTED = 7, /* shape or dtype the kernels are not built for */
  PKV_ERR_CAPACITY = 8     /* device block tables must grow first (see pkv_step_info) */
};

enum pkv_dtype { PKV_F32 = 0, PKV_F16 = 1, PKV_BF16 = 2 };

/* Message of the last failure on this thread ("" if none). */
const char* pkv_last_error(void);

/* Library version string, e.g. "pkv_b200 1.0 sm_100a". */
const char* pkv_version(void);

/* ------------------------------------------------------------------------ */
/* Host block allocator                                                      */
/* ------------------------------------------------------------------------ */

typedef struct pkv_allocator pkv_allocator;

typedef struct pkv_allocator_stats {
  int64_t total_blocks;
  int64_t block_size_tokens;
  int64_t free_block_count;        /* PagedKVAllocator.free_block_count */
  int64_t used_block_count;        /* .used_block_count */
  int64_t block_reuse_count;       /* .block_reuse_count */
  int64_t max_blocks_in_use;       /* .max_blocks_in_use (high watermark) */
  int64_t resident_sequence_count; /* .resident_sequence_count */
  int64_t row_capacity;            /* rows the device table must have */
  int64_t max_blocks_per_row;      /* columns the device table must have */
  int64_t shared_block_count;      /* blocks with refcount > 1 (forks) */
} pkv_allocator_stats;

/* PagedKVAllocator.__init__ (agentrl/generation/paged_kv.py:34-48).
 * Returns NULL and sets *status on invalid sizes. */
pkv_allocator* pkv_allocator_create(int64_t total_blocks, int64_t block_size_tokens, int32_t* status);
void pkv_allocator_destroy(pkv_allocator* a);

/* PagedKVAllocator.reserve (paged_kv.py:78-91): lowest free ids first. */
int32_t pkv_allocator_reserve(pkv_allocator* a, int64_t sequence_id, int64_t token_count);
/* PagedKVAllocator.append_tokens (paged_kv.py:93-110).  A shared partial
 * tail block (after pkv_allocator_fork) is first replaced by a private copy. */
int32_t pkv_allocator_append_tokens(pkv_allocator* a, int64_t sequence_id, int64_t token_count);
/* PagedKVAllocator.release (paged_kv.py:112-120); shared blocks are freed
 * when their last owner releases them. */
int32_t pkv_allocator_release(pkv_allocator* a, int64_t sequence_id);
/* Copy-on-write fork: `child` shares all of `parent`'s blocks (no reference
 * counterpart; used to share a GRPO group's prompt pages). */
int32_t pkv_allocator_fork(pkv_allocator* a, int64_t parent_id, int64_t child_id);
/* PagedKVAllocator.logical_to_physical (paged_kv.py:122-127). */
int32_t pkv_allocator_logical_to_physical(pkv_allocator* a, int64_t sequence_id, int64_t logical_block_index,
                                          int64_t* block_out);
/* PagedKVAllocator.view (paged_kv.py:129-139).  Writes up to `capacity`
 * block ids; *num_blocks gets the full count. */
int32_t pkv_allocator_view(pkv_allocator* a, int64_t sequence_id, int64_t* token_count, int32_t* blocks,
                           int64_t capacity, int64_t* num_blocks);
/* PagedKVAllocator.has_sequence (paged_kv.py:154-157): 1 or 0. */
int32_t pkv_allocator_has_sequence(pkv_allocator* a, int64_t sequence_id);
/* Counters behind PagedKVAllocator's properties and metrics() (paged_kv.py:50-76,141-152). */
int32_t pkv_allocator_get_stats(pkv_allocator* a, pkv_allocator_stats* out);
/* Refcount of one block (0 = free). */
int32_t pkv_allocator_refcount(pkv_allocator* a, int64_t block, int32_t* out);
/* Device block-table row of a sequence. */
int32_t pkv_allocator_row(pkv_allocator* a, int64_t sequence_id, int32_t* row_out);

/* One decode step: append one token to each of `n` sequences, in order
 * (the per-token append_tokens(seq, 1) calls of agentrl/generation/continuous.py:492-493).
 * Per entry i it writes the table row, the new token count, the block
 * newly allocated for the token (-1 if the token fits the current tail) and
 * (if token_blocks_out is not NULL) the block that holds the token.
 * rows/lens/new_blocks are what pkv_decode_attention consumes; the fused
 * kernel itself stores the new block and length into the device tables, so
 * they are not recorded as pending device updates (pkv_allocator_touch_rows
 * records them when no fused kernel will run).  On failure (unknown id, pool
 * exhausted) the steps already taken stay applied (as with the reference's
 * sequential calls) and *done gets their count. */
int32_t pkv_allocator_decode_step(pkv_allocator* a, const int64_t* sequence_ids, int64_t n, int32_t* rows_out,
                                  int32_t* lens_out, int32_t* new_blocks_out, int32_t* token_blocks_out,
                                  int64_t* done);
/* Shrink sequences to token_counts[i] tokens (no reference counterpart: it
 * rolls back speculative drafts a verify step rejected).  Blocks past the new
 * end are released (a shared block only drops one reference).  A count above
 * the current one is a ValueError; an unknown id a KeyError. */
int32_t pkv_allocator_truncate(pkv_allocator* a, const int64_t* sequence_ids, const int64_t* token_counts,
                               int64_t n);
/* pkv_allocator_truncate plus the store's per-block fill bookkeeping in the
 * same pass (block_fill [fill_n]: tokens stored per block, -1 = none): a
 * block that becomes free gets -1, a sequence's new partial tail block at
 * most the tokens it still holds. */
int32_t pkv_allocator_truncate_fill(pkv_allocator* a, const int64_t* sequence_ids, const int64_t* token_counts,
                                    int64_t n, int32_t* block_fill, int64_t fill_n);
/* Token counts of n sequences (KeyError for an unknown id): the
 * PagedKVSequenceView.token_count of each, without building the views. */
int32_t pkv_allocator_token_counts(pkv_allocator* a, const int64_t* sequence_ids, int64_t n, int64_t* counts_out);
/* Free blocks that appending one token to each of n sequences takes:
 * need_out[i] = 1 when sequence i's next token starts a new block or lands in
 * a partial tail block still shared by a fork (copied on write), else 0.  It
 * generalises the growth test of ContinuousBatchingOrchestrator's admission
 * (agentrl/generation/continuous.py:915-919: max(1, len) % block_size == 0)
 * to copy-on-write forks, which the reference does not have. */
int32_t pkv_allocator_growth_blocks(pkv_allocator* a, const int64_t* sequence_ids, int64_t n, int32_t* need_out);
/* Layout of a prefill / verify chunk per sequence -- its last q_lens[i]
 * tokens (no reference counterpart: the reference prefills into HF caches):
 * the table row, the tokens before the chunk (past), and the pool slot
 * (block * block_size + offset) of every chunk token, packed in order into
 * slots_out (capacity slots_capacity); block_fill (optional) is raised to
 * cover the chunk tokens.  A chunk longer than its sequence is a ValueError. */
int32_t pkv_allocator_chunk_slots(pkv_allocator* a, const int64_t* sequence_ids, const int64_t* q_lens, int64_t n,
                                  int32_t* rows_out, int32_t* past_out, int64_t* slots_out, int64_t slots_capacity,
                                  int32_t* block_fill, int64_t fill_n);
/* Record the length and last table entry of the given rows as pending device
 * updates. */
int32_t pkv_allocator_touch_rows(pkv_allocator* a, const int32_t* rows, int64_t n);

/* Device-mirror synchronisation.  Every allocator call records which table
 * entries, refcounts and lengths changed and which blocks must be copied
 * (copy-on-write).  pkv_allocator_pending_updates reports the sizes;
 * pkv_allocator_drain_updates writes them into one int32 buffer laid out as
 *   [n_table, n_ref, n_len, n_copy,
 *    n_table x (row, col, block), n_ref x (block, refcount),
 *    n_len x (row, len), n_copy x (src_block, dst_block)]
 * with the CURRENT host values, and clears the record.  The buffer is what
 * pkv_apply_updates (device) consumes.  Returns the number of int32 written. */
int32_t pkv_allocator_pending_updates(pkv_allocator* a, int64_t* n_table, int64_t* n_ref, int64_t* n_len,
                                      int64_t* n_copy);
int32_t pkv_allocator_drain_updates(pkv_allocator* a, int32_t* out, int64_t capacity, int64_t* written);

/* ------------------------------------------------------------------------ */
/* Device kernels (sm_100a)                                                  */
/* ------------------------------------------------------------------------ */

typedef struct pkv_pool_geom {
  int32_t num_layers;
  int32_t num_blocks;
  int32_t num_kv_heads;
  int32_t block_size;   /* tokens per block */
  int32_t head_dim;
  int32_t dtype;        /* enum pkv_dtype */
} pkv_pool_geom;

/* Bytes of the KV pool for a geometry. */
int64_t pkv_pool_bytes(const pkv_pool_geom* g);

/* Apply a drained update buffer (pkv_allocator_drain_updates) to the device
 * block tables, refcounts and lengths, then copy whole blocks (all layers,
 * K and V) for the copy-on-write pairs, in order.  `updates` is a DEVICE copy
 * of the buffer and `host_updates` the host buffer it was copied from (read
 * for the counts and to order chained copies).
 * Replaces nothing in the reference (whose tables live in Python dicts,
 * paged_kv.py:44-45); it is the fork/free/COW table and refcount kernel. */
int32_t pkv_apply_updates(const pkv_pool_geom* g, void* pool, int32_t* block_tables, int32_t table_stride,
                          int32_t num_rows, int32_t* refcounts, int32_t* context_lens, const int32_t* updates,
                          const int32_t* host_updates, void* stream);

/* Scatter `n_tokens` token rows of K and V into their pool slots, for layers
 * [layer0, layer0 + n_layers).  Token t of layer l, head h is read from
 *   src + l*src_layer_stride + h*src_head_stride + t*src_token_stride
 * (element strides, innermost head_dim contiguous) and written to slot
 * slot_mapping[t] = block * block_size + offset.  A slot < 0 is skipped.
 * Replaces the per-block clone of write_sequence_cache (paged_kv.py:259-269)
 * and the per-step K/V append DynamicLayer.update (transformers
 * cache_utils.py:119-120). */
int32_t pkv_scatter_tokens(const pkv_pool_geom* g, void* pool, int32_t layer0, int32_t n_layers, const void* k_src,
                           const void* v_src, int64_t src_layer_stride, int64_t src_head_stride,
                           int64_t src_token_stride, const int64_t* slot_mapping, int64_t n_tokens, void* stream);

/* Gather: the inverse of pkv_scatter_tokens into dst buffers with the same
 * stride convention.  Replaces read_sequence_legacy_cache's torch.cat of the
 * block chunks (paged_kv.py:302-321). */
int32_t pkv_gather_tokens(const pkv_pool_geom* g, const void* pool, int32_t layer0, int32_t n_layers, void* k_dst,
                          void* v_dst, int64_t dst_layer_stride, int64_t dst_head_stride, int64_t dst_token_stride,
                          const int64_t* slot_mapping, int64_t n_tokens, void* stream);

/* Copy whole blocks (every layer, K and V) src[i] -> dst[i]. */
int32_t pkv_copy_blocks(const pkv_pool_geom* g, void* pool, const int32_t* src_blocks, const int32_t* dst_blocks,
                        int64_t n, void* stream);

/* KV heads one decode work item covers: 2 when num_kv_heads is even, else 1. */
int32_t pkv_decode_heads_per_item(int32_t num_kv_heads);

/* Plan one decode step (host): cut each sequence's pages into work items of
 * at most *pages_per_split_out (<= 32) pages for one group of
 * pkv_decode_heads_per_item KV heads, sized for the warps of `num_sms`
 * persistent CTAs.  seq_lens[b] counts the step's token; a sequence may hold
 * up to 32768 tokens.  With items_out == NULL only the counts are returned; else
 * items_out (capacity in quadruples) receives *n_items_out int32 quadruples
 *   {sequence, split << 8 | head_group, splits of the sequence, workspace slot of split 0}
 * (by decreasing page count: full-size items first, the smallest last, so a
 * persistent grid's tail holds the shortest items), followed by
 * *n_combine_out quadruples {sequence, head_group, splits, slot of split 0},
 * one per (sequence, head group) cut into several items. */
int32_t pkv_decode_plan(const int32_t* seq_lens, int32_t batch, int32_t num_kv_heads, int32_t head_dim,
                        int32_t num_sms, int32_t* pages_per_split_out, int32_t* items_out, int64_t items_capacity,
                        int64_t* n_items_out, int64_t* n_combine_out);

/* Bytes of device workspace pkv_decode_attention needs for `batch`
 * sequences and `n_items` work items. */
int64_t pkv_decode_workspace_bytes(int32_t batch, int32_t num_kv_heads, int32_t head_dim, int64_t n_items);

/* Paged GQA decode attention for one layer, optionally fused with the K/V
 * append of the step's token.
 *   q      [batch][num_q_heads][head_dim] (bf16 or f16, same as the pool)
 *   k_new, v_new [batch][num_kv_heads][head_dim] or NULL (no append)
 *   block_tables  int32 [table_rows][table_stride]
 *   rows[b]       table row of entry b
 *   seq_lens[b]   tokens in the cache INCLUDING the step's token
 *   new_blocks[b] block allocated for the step's token or -1 (may be NULL)
 *   work_items    the plan of pkv_decode_plan for these seq_lens (device copy:
 *                 n_items items then n_combine combine entries)
 *   out    [batch][num_q_heads][head_dim]
 *   workspace: pkv_decode_workspace_bytes() bytes, zeroed once before first
 *              use; every launch leaves it ready for the next one.  Its first
 *              int32 is an error word: 0, or 1 (a bounded wait gave up),
 *              3 (a work item outside the launch was skipped), 4 (a block id
 *              outside the pool was replaced by block 0).
 * With k_new != NULL the kernel writes the token's K/V into its slot
 * (position seq_lens[b]-1), and stores new_blocks[b] (when >= 0) into the
 * table and seq_lens[b] into context_lens[rows[b]].
 * Replaces HF sdpa_attention_forward with GQA (transformers
 * integrations/sdpa_attention.py:40-62) over the stacked resident caches of
 * agentrl/generation/continuous.py:476-483, and the torch.cat append of
 * transformers cache_utils.py:119-120.  Requires block_size 16, head_dim 64
 * or 128, bf16/f16, num_q_heads / num_kv_heads <= 8. */
int32_t pkv_decode_attention(const pkv_pool_geom* g, void* pool, int32_t layer, const void* q, const void* k_new,
                             const void* v_new, int32_t* block_tables, int32_t table_stride, int32_t table_rows,
                             int32_t* context_lens,
                             const int32_t* rows, const int32_t* seq_lens, const int32_t* new_blocks,
                             const int32_t* work_items, int32_t n_items, int32_t n_combine, int32_t batch,
                             int32_t num_q_heads, int32_t pages_per_split, float scale, void* out, void* workspace,
                             int64_t workspace_bytes, void* stream);

/* pkv_decode_attention for callers that may not allocate device memory (no
 * counterpart in the reference).  Some hosts of this library -- a serving
 * framework that owns all GPU memory through its own arena so that its
 * accounting stays exact and no cudaMalloc/cudaFree stalls the device, or a
 * plugin interface that only passes buffers it allocated -- provide inputs
 * and outputs but no workspace.  This entry point takes the same arguments
 * minus the workspace and uses a 16 MiB scratch array that lives in the
 * library's device memory on every GPU that loads it, until process exit.  It
 * never calls cudaMalloc, cudaFree or any allocating routine.
 *  - A step whose workspace (pkv_decode_workspace_bytes) exceeds 16 MiB is
 *    rejected with PKV_ERR_ARG and a message; nothing is launched.
 *  - The first call on a device looks up the scratch's device address (with
 *    that device current); make that first call before any stream capture.
 *  - All calls share the one scratch: calls that overlap on the GPU (other
 *    streams, other threads) race and corrupt each other's results.  Each call
 *    clears the parts that must start at zero. */
int32_t pkv_decode_attention_noalloc(const pkv_pool_geom* g, void* pool, int32_t layer, const void* q,
                                     const void* k_new, const void* v_new, int32_t* block_tables,
                                     int32_t table_stride, int32_t table_rows, int32_t* context_lens,
                                     const int32_t* rows, const int32_t* seq_lens, const int32_t* new_blocks,
                                     const int32_t* work_items, int32_t n_items, int32_t n_combine, int32_t batch,
                                     int32_t num_q_heads, int32_t pages_per_split, float scale, void* out,
                                     void* stream);

/* The error word of the no-alloc decode calls on the current device (no
 * counterpart in the reference): 0, or the codes of pkv_decode_attention's
 * workspace error word -- 1 (a bounded wait gave up), 3 (a work item outside
 * the launch was skipped), 4 (a block id outside the pool was replaced by
 * block 0).  Each pkv_decode_attention_noalloc call clears the word when it
 * starts, so read it after the calls it should cover and before the next
 * one.  The word is copied in stream order on `stream` (after the calls
 * issued there so far) and the function waits for that copy; *error_out is 0
 * when no no-alloc call has run on the device yet. */
int32_t pkv_decode_noalloc_error(int32_t* error_out, void* stream);

/* ------------------------------------------------------------------------ */
/* Chunked prefill / speculative verify over pages                           */
/* ------------------------------------------------------------------------ */

/* Chunk positions one prefill work item covers: 2 x 128 / G with G =
 * num_q_heads / num_kv_heads (the G query heads of a position share a row
 * block of a 128-row tile, and an item holds two tiles); 0 for head counts
 * the kernel does not support. */
int32_t pkv_prefill_positions_per_item(int32_t num_q_heads, int32_t num_kv_heads);

/* Plan a prefill / verify launch (host).  Sequence i has table row rows[i],
 * past_lens[i] tokens before its chunk and q_lens[i] chunk queries, packed in
 * q in sequence order.  Output: int32 [n_items + n_combine][8] records, the
 * work items (longest key range first) then the combine entries.  With
 * split_waves > 0 and fewer than split_waves x num_sms items (a verify step),
 * the keys of an item whose queries fit one tile are cut into ranges (about
 * split_waves CTAs per SM in all) that each write a partial into one of
 * *n_slots_out workspace slots, merged by a combine entry; 0 keeps one CTA
 * per item.  Records are written when items_out is non-NULL and the capacity (in
 * records) suffices (else PKV_ERR_CAPACITY); the counts are always set. */
int32_t pkv_prefill_plan(const int32_t* rows, const int32_t* past_lens, const int32_t* q_lens, int32_t n_seqs,
                         int32_t num_q_heads, int32_t num_kv_heads, int32_t num_sms, int32_t split_waves,
                         int32_t* work_items_out, int64_t items_capacity, int64_t* n_items_out,
                         int64_t* n_combine_out, int64_t* n_slots_out);

/* Bytes of workspace pkv_prefill_attention needs for n_slots partials. */
int64_t pkv_prefill_workspace_bytes(int64_t n_slots, int32_t head_dim);

/* Causal paged attention for chunks of queries after cached tokens, one layer
 * (tcgen05 tensor cores, fp32 accumulation in tensor memory).
 *   q, out        [total_q][num_q_heads][head_dim], pool dtype (bf16 / f16)
 *   block_tables  int32 [table_rows][table_stride] (device; every block of
 *                 past + chunk tokens present, the chunk's K/V already
 *                 written, e.g. by pkv_scatter_tokens)
 *   work_items    device copy of pkv_prefill_plan's records (n_items work
 *                 items, then n_combine combine entries)
 *   error_word    device int32, 0 before the call; afterwards 0, or 1 (a
 *                 bounded wait gave up), 3 (an item outside the launch was
 *                 skipped), 4 (a block id outside the pool was replaced by 0)
 *   workspace     pkv_prefill_workspace_bytes(n_slots) bytes (may be NULL
 *                 when n_slots is 0); no initial contents needed
 * Query i of a chunk after `past` tokens attends to keys 0 .. past + i.
 * Replaces the attention of the HF forward per prefill chunk
 * (agentrl/generation/prefill.py:96-104; transformers
 * integrations/sdpa_attention.py:40-62 with a causal mask after a past) and
 * of the speculative verify forward (agentrl/generation/speculative.py:229-264,
 * rows prefix_len-1 .. prefix_len-1+k: a chunk of k+1 queries after
 * prefix_len-1 tokens).  Requires block_size 16, head_dim 64 or 128. */
int32_t pkv_prefill_attention(const pkv_pool_geom* g, const void* pool, int32_t layer, const void* q,
                              const int32_t* block_tables, int32_t table_stride, int32_t table_rows,
                              const int32_t* work_items, int32_t n_items, int32_t n_combine, int64_t total_q,
                              int32_t num_q_heads, float scale, void* out, int32_t* error_word, void* workspace,
                              int64_t workspace_bytes, int64_t n_slots, void* stream);

/* Positions of a chunk one verify work item covers: 32 / G query columns of
 * one KV head (G = num_q_heads / num_kv_heads); 0 when G > 32 or the head
 * counts are invalid. */
int32_t pkv_verify_positions_per_item(int32_t num_q_heads, int32_t num_kv_heads);

/* Plan a pkv_verify_attention launch (host); arguments as for
 * pkv_prefill_plan.  A sequence's chunk is cut into items of
 * pkv_verify_positions_per_item positions, one per KV head.  With num_sms > 0
 * the launch is a persistent grid of *n_ctas_out = min(num_sms, items) CTAs,
 * one per SM, each working through a list of items: items longer than half
 * an SM's share of the KV tiles (of 128 keys) are cut into key ranges of at
 * least two tiles, each writing a partial into one of *n_slots_out workspace
 * slots that a combine entry merges, and the items go longest first to the
 * CTA with the fewest tiles so far.  num_sms = 0 gives one CTA per item and no
 * combine entries (a fixed record count, as a recorded CUDA graph needs).
 * Records: int32 [n_items + n_combine][8]; record c < n_ctas is CTA c's first
 * item, whose last field is (f << 8) | m: the CTA's other m <= 127 items are
 * records f .. f+m-1 (more CTAs than num_sms only beyond 128 items per SM);
 * then the combine entries {first slot, slots, query index, kv_head << 16 |
 * positions}.  An item record is {table row, first position, query index,
 * kv_head << 16 | positions, first KV tile | (end KV tile << 16) (0: all),
 * combine entry (-1: none), partial slot (-1: none), list}. */
int32_t pkv_verify_plan(const int32_t* rows, const int32_t* past_lens, const int32_t* q_lens, int32_t n_seqs,
                        int32_t num_q_heads, int32_t num_kv_heads, int32_t num_sms, int32_t* work_items_out,
                        int64_t items_capacity, int64_t* n_items_out, int64_t* n_ctas_out, int64_t* n_combine_out,
                        int64_t* n_slots_out);

/* The speculative-verify read (short chunks after long cached prefixes), one
 * layer: the same result as pkv_prefill_attention, from a kernel that puts the
 * 128 keys of a KV tile on the tensor-core rows and the <= 32 (position,
 * head) query columns of an item on N, so that short chunks do not leave a
 * 128-row query tile mostly empty, and streams each CTA's items through one
 * pipeline.  Arguments as for pkv_prefill_attention with pkv_verify_plan's
 * records and n_ctas; workspace pkv_prefill_workspace_bytes(n_slots, 128)
 * for the key-range partials, merged by a second (programmatic dependent)
 * launch.
 * Replaces the attention of the speculative verify forward
 * (agentrl/generation/speculative.py:229-264, rows prefix_len-1 ..
 * prefix_len-1+k).  Requires block_size 16, head_dim 128, bf16 or f16, at most
 * 32 query heads per KV head. */
int32_t pkv_verify_attention(const pkv_pool_geom* g, const void* pool, int32_t layer, const void* q,
                             const int32_t* block_tables, int32_t table_stride, int32_t table_rows,
                             const int32_t* work_items, int32_t n_items, int32_t n_ctas, int32_t n_combine,
                             int64_t total_q, int32_t num_q_heads, float scale, void* out, int32_t* error_word,
                             void* workspace, int64_t workspace_bytes, int64_t n_slots, void* stream);

/* ------------------------------------------------------------------------ */
/* Native decode-step runtime                                                */
/* ------------------------------------------------------------------------ */

/* One decode step as uploaded to the device (device pointers are valid until
 * the stepper's next upload). */
typedef struct pkv_step_info {
  int32_t batch;            /* sequences in the step (appended so far on failure) */
  int32_t pages_per_split;
  int32_t n_items;
  int32_t n_combine;
  int32_t n_copies;         /* copy-on-write block copies applied before the step */
  int32_t need_rows;        /* device table rows / columns the step needs */
  int32_t need_cols;
  int32_t need_items;       /* fixed-step mode: the work items a step needs beyond the capacity (else 0) */
  const int32_t* rows;      /* device [batch] */
  const int32_t* seq_lens;  /* device [batch] (tokens incl. the step's token) */
  const int32_t* new_blocks;/* device [batch] */
  const int32_t* items;     /* device: n_items work items, then n_combine entries */
  const int64_t* slots;     /* device [batch]: pool slot of each step token */
} pkv_step_info;

typedef struct pkv_stepper pkv_stepper;

/* A stepper runs decode steps of one allocator / pool on one stream: it owns
 * a small ring of pinned staging buffers and the decode workspace.  It
 * replaces the per-step Python work around AgentRL's decode loop
 * (agentrl/generation/continuous.py:443-497: per-sequence append_tokens,
 * cache stack / split) with one C call per step plus one per layer. */
pkv_stepper* pkv_stepper_create(pkv_allocator* a, const pkv_pool_geom* g, void* pool, int32_t* status);
void pkv_stepper_destroy(pkv_stepper* st);
/* The device block tables (int32 [table_rows][table_stride]), lengths and
 * refcounts the stepper keeps in sync; rebind after growing them. */
int32_t pkv_stepper_bind_tables(pkv_stepper* st, int32_t* block_tables, int32_t table_stride, int32_t table_rows,
                                int32_t* context_lens, int32_t* refcounts);
/* Fixed-step mode, for decode steps recorded once in a CUDA graph and
 * replayed: from now on every upload writes the step descriptor into one
 * device block whose header carries the step's counts, the attention
 * launches always have the same arguments (capacities, that block, a
 * workspace sized now) and the kernels read the counts at run time.
 * max_batch bounds the sequences of a step, max_items its work items (0: a
 * default of KV-head groups x max_batch + 4 x the persistent grid's warps); a
 * step beyond them fails with PKV_ERR_UNSUPPORTED.  The device tables must
 * not be rebound while a graph holds such launches.  No counterpart in the
 * reference (its decode loop is eager Python). */
int32_t pkv_stepper_fix_steps(pkv_stepper* st, int32_t max_batch, int32_t max_items, void* stream);
/* The fixed-step capacities in force (0, 0 when the mode is off). */
int32_t pkv_stepper_fixed_capacity(pkv_stepper* st, int32_t* max_batch, int32_t* max_items);
/* Optional: a host int32 array [n_blocks] of tokens stored per block that the
 * stepper keeps current -- a copy-on-write copy gives the new block its
 * source's count, an uploaded step sets the count of the block each step
 * token went to.  The array must outlive the stepper or be unbound (n 0). */
int32_t pkv_stepper_bind_fill(pkv_stepper* st, int32_t* block_fill, int64_t n_blocks);
/* Apply the allocator's pending updates on `stream` (as pkv_apply_updates);
 * up to copies_cap copy-on-write (src, dst) pairs are reported.  Returns
 * PKV_ERR_CAPACITY with *need_rows / *need_cols when the tables must grow. */
int32_t pkv_stepper_sync(pkv_stepper* st, void* stream, int32_t* copies_out, int64_t copies_cap, int32_t* n_copies,
                         int32_t* need_rows, int32_t* need_cols);
/* Step phase 1 (host only): append one token to each sequence in order
 * (pkv_allocator_decode_step).  Optional host outputs: table rows, new token
 * counts and the block holding each step token. */
int32_t pkv_stepper_begin(pkv_stepper* st, const int64_t* sequence_ids, int32_t n, pkv_step_info* info,
                          int32_t* rows_out, int32_t* lens_out, int32_t* token_blocks_out);
/* Step phase 2: apply pending updates, plan, upload the descriptor on
 * `stream`.  PKV_ERR_CAPACITY (info->need_rows / need_cols set, nothing
 * launched) asks the caller to grow and rebind the tables and call again.
 * In fixed-step mode a step with more work items than the capacity fails
 * with PKV_ERR_UNSUPPORTED and info->need_items set: fix the steps again
 * with room for them (graphs recorded before hold the old block) and call
 * again. */
int32_t pkv_stepper_upload(pkv_stepper* st, void* stream, pkv_step_info* info, int32_t* copies_out,
                           int64_t copies_cap);
/* Fused append + paged decode attention of the uploaded step for one layer
 * (pkv_decode_attention with the stepper's descriptor and workspace). */
int32_t pkv_stepper_attention(pkv_stepper* st, int32_t layer, const void* q, const void* k_new, const void* v_new,
                              int32_t num_q_heads, float scale, void* out, void* stream);
/* begin + upload + attention of one layer in one call (a one-layer step, or
 * a step and its first layer).  On PKV_ERR_CAPACITY the step is begun but
 * nothing is launched: grow and rebind the tables, then call
 * pkv_stepper_upload and pkv_stepper_attention. */
int32_t pkv_stepper_step(pkv_stepper* st, const int64_t* sequence_ids, int32_t n, int32_t layer, const void* q,
                         const void* k_new, const void* v_new, int32_t num_q_heads, float scale, void* out,
                         void* stream, pkv_step_info* info, int32_t* rows_out, int32_t* lens_out,
                         int32_t* token_blocks_out, int32_t* copies_out, int64_t copies_cap);
/* pkv_stepper_step with q / k_new / v_new and out in HOST memory (pinned for
 * the copies to overlap; q and out [n][num_q_heads][head_dim], k_new and
 * v_new [n][num_kv_heads][head_dim], the pool's dtype; k_new / v_new both
 * NULL for attention without the append).  The stepper stages the inputs in
 * device buffers of its own: they cross on its copy stream ahead of the step
 * descriptor (one copy when inputs_packed is 1: q, k_new and v_new are
 * consecutive parts of ONE host allocation, back to back; else three), the
 * output crosses on a second stream of the stepper after the step's
 * kernels, so a step's input copy and the previous step's output copy run
 * while the kernels of the step between them do.  Host pointers are read and
 * written asynchronously: q / k_new / v_new must stay unchanged and out must
 * not be read until `stream` has passed pkv_stepper_host_fence.  This is the
 * host-facing form of the reference's decode step, whose q / k / v come from
 * the model on the same device (agentrl/generation/continuous.py:407-497).
 * On PKV_ERR_CAPACITY the step is begun and its inputs staged: grow and
 * rebind the tables, then call pkv_stepper_upload and
 * pkv_stepper_attention_host. */
int32_t pkv_stepper_step_host(pkv_stepper* st, const int64_t* sequence_ids, int32_t n, int32_t layer,
                              const void* q_host, const void* k_new_host, const void* v_new_host,
                              int32_t inputs_packed, int32_t num_q_heads, float scale, void* out_host, void* stream, pkv_step_info* info,
                              int32_t* rows_out, int32_t* lens_out, int32_t* token_blocks_out);
/* The attention + output copy of a host step whose inputs were staged by
 * pkv_stepper_step_host and whose descriptor is uploaded (the capacity retry). */
int32_t pkv_stepper_attention_host(pkv_stepper* st, int32_t layer, int32_t num_q_heads, float scale, void* out_host,
                                   void* stream);
/* Make `stream` wait for every output copy of the host steps issued so far;
 * once `stream` has run past this point their out buffers hold the results. */
int32_t pkv_stepper_host_fence(pkv_stepper* st, void* stream);
/* Page-locked host memory for a host step's inputs (q / k_new / v_new):
 * write-combined unless write_combined is 0.  The GPU reads write-combined
 * memory over PCIe without snooping the host's caches, which on the hosts
 * measured here doubled host-to-device bandwidth for 1-16 MB copies (about
 * 50 GB/s against 16-38 GB/s from cacheable page-locked memory); host reads
 * of it are slow, so use it only for data the host writes and the GPU reads,
 * and default page-locked memory for outputs.  Free with pkv_host_free. */
int32_t pkv_host_alloc(int64_t bytes, int32_t write_combined, void** ptr_out);
int32_t pkv_host_free(void* ptr);
/* The copy-on-write (src, dst) block pairs the last sync / upload applied
 * (*n_pairs gets their count; up to `capacity` pairs are written). */
int32_t pkv_stepper_copies(pkv_stepper* st, int32_t* pairs_out, int64_t capacity, int64_t* n_pairs);
/* The decode workspace's error word (synchronous read; 0 = no error). */
int32_t pkv_stepper_error(pkv_stepper* st, int32_t* device_error);
/* Kernels the stepper has launched so far. */
int64_t pkv_stepper_launches(pkv_stepper* st);
/* Nanoseconds the host has spent blocked on the stepper's staging ring so far
 * (it waits there only when it runs eight steps ahead of the device); with a
 * wall-clock reading around a loop of steps it separates the host's own work
 * per step from waiting.  No reference counterpart (measurement). */
int64_t pkv_stepper_host_wait_ns(pkv_stepper* st);
/* Time `count` of the following attention launches, every `every`-th one,
 * with CUDA events recorded right around the decode kernels on their stream
 * (count 0 turns timing off; sampling keeps the event calls' host time off
 * most steps). */
int32_t pkv_stepper_time_launches(pkv_stepper* st, int64_t count, int64_t every);
/* Device milliseconds of the timed launches so far (waits for the last). */
int32_t pkv_stepper_launch_times(pkv_stepper* st, float* ms_out, int64_t capacity, int64_t* n_out);

/* ---------------------------------------------------------------------------
 * Fused elementwise layers of a Qwen2-family decoder (bf16 / f16), each one
 * launch doing what the HF modules do in several, with the same roundings
 * (transformers models/qwen2/modeling_qwen2.py).  No reference counterpart:
 * AgentRL runs those modules eagerly inside its HF forwards
 * (agentrl/generation/continuous.py:407-497).
 * ------------------------------------------------------------------------- */

/* Qwen2RMSNorm: out = w * to_dtype(x * rsqrt(mean(x^2) + eps)), x in fp32,
 * rows x hidden (hidden <= 8192).  With residual (and sum_out) non-NULL, x is
 * first to_dtype(x + residual) -- Qwen2DecoderLayer's residual add -- and that
 * sum is written to sum_out. */
int32_t pkv_rms_norm(const void* x, const void* residual, void* sum_out, const void* weight, void* out, int64_t rows,
                     int32_t hidden, float eps, int32_t dtype, void* stream);
/* apply_rotary_pos_emb for the q and k of `rows` tokens: q rows of q_heads *
 * head_dim, k rows of kv_heads * head_dim, q_ld / k_ld elements apart (three
 * tensors, or one packed q|k|v projection row), cos / sin [rows][head_dim];
 * out = to_dtype(to_dtype(x * cos) + to_dtype(rotate_half(x) * sin)) into
 * contiguous q_out [rows][q_heads][head_dim] / k_out.  With v and v_out
 * non-NULL the v rows (v_ld apart) are copied to contiguous v_out too. */
int32_t pkv_rope(const void* q, const void* k, const void* v, const void* cos, const void* sin, void* q_out,
                 void* k_out, void* v_out, int64_t rows, int64_t q_ld, int64_t k_ld, int64_t v_ld, int32_t q_heads,
                 int32_t kv_heads, int32_t head_dim, int32_t dtype, void* stream);
/* Qwen2MLP's act_fn(gate) * up with SiLU: out[r][c] = to_dtype(to_dtype(
 * silu(gate)) * up) for rows x cols, gate / up rows ld_in elements apart. */
int32_t pkv_silu_mul(const void* gate, const void* up, void* out, int64_t rows, int64_t cols, int64_t ld_in,
                     int32_t dtype, void* stream);

/* ---------------------------------------------------------------------------
 * Vocabulary rows: token log-probabilities, token selection, speculative
 * accept / reject.  Logits are fp32 rows of `vocab` columns, row r at
 * logits + r * ld (ld >= vocab).  Each launch streams the rows once.  The
 * workspace is device scratch of at least the size the matching
 * *_workspace_bytes call returns.  `tickets` is an int32 device array
 * (n_rows entries for the row entry points, pkv_spec_tickets for
 * pkv_spec_accept) that is zero-filled once before its first use: the
 * kernels leave it zero again, so one array serves every later launch.
 * Launches sharing a workspace or a ticket array must run in stream order.
 * ------------------------------------------------------------------------- */

/* Workspace bytes for pkv_token_logprobs / pkv_sample_tokens over n_rows rows
 * (-1 for invalid arguments). */
int64_t pkv_sampling_workspace_bytes(int64_t n_rows, int32_t vocab);

/* Replaces torch.log_softmax(logits, -1).gather(-1, tokens) of the
 * old-policy pass (agentrl/core/rollout.py:462-465): logprobs_out[r] =
 * logits[r][tokens[r]] - logsumexp(logits[r]) (NaN for a token outside
 * [0, vocab)), lse_out[r] = logsumexp(logits[r]).  Either output may be NULL
 * (logprobs_out needs tokens). */
int32_t pkv_token_logprobs(const float* logits, int64_t ld, int32_t n_rows, int32_t vocab, const int64_t* tokens,
                           float* logprobs_out, float* lse_out, int32_t* tickets, void* workspace,
                           int64_t workspace_bytes, void* stream);

/* Replaces the rollout's next-token choice (agentrl/core/rollout.py:307-315)
 * and the log-probability recorded for it: with do_sample = 0, tokens_out[r]
 * = argmax of row r (first index of the maximum); otherwise a draw from
 * softmax(race_logits[r] / temperature) (race_logits NULL = logits; pass
 * top-p filtered logits there, -inf for dropped columns), made with the
 * Gumbel-max trick from a counter-based hash of (seed, offset, r, column).
 * logprobs_out[r] = log_softmax(logits[r])[tokens_out[r]] (temperature 1);
 * argmax_out[r] = argmax of logits[r].  logprobs_out and argmax_out may be
 * NULL. */
int32_t pkv_sample_tokens(const float* logits, const float* race_logits, int64_t ld, int32_t n_rows, int32_t vocab,
                          float temperature, int32_t do_sample, uint64_t seed, uint64_t offset, int64_t* tokens_out,
                          float* logprobs_out, int64_t* argmax_out, int32_t* tickets, void* workspace,
                          int64_t workspace_bytes, void* stream);

/* Workspace bytes and ticket count for pkv_spec_accept (-1 for invalid
 * arguments). */
int64_t pkv_spec_workspace_bytes(int32_t batch, int32_t k, int32_t vocab);
int64_t pkv_spec_tickets(int32_t batch, int32_t k);

/* Replaces SpeculativeRolloutOrchestrator._verify_draft
 * (agentrl/generation/speculative.py:217-274) for a batch of sequences.
 * target_logits [batch][k + 1][ld]: row i is the target's prediction after
 * the sequence's last accepted token and drafts 0..i-1 (row k is the bonus
 * row); draft_logits [batch][k][ld]: the draft's logits that proposed draft
 * i; draft_tokens [batch][k]; n_draft[b] <= k drafts are valid (the draft
 * stops after eos, speculative.py:210-211).  Draft i is accepted when u <=
 * min(1, exp(lp_target - log(p_draft + 1e-12))), p_draft from softmax(draft
 * logits / draft_temperature) and u = uniforms[b][i] (NULL: hashed from
 * seed / offset); the first rejection draws a correction from
 * max(p_target - p_draft, 0) (p_target itself if that is all zero), and
 * accepting all n_draft drafts draws a bonus token from p_target of row
 * n_draft; both draws are argmax when do_sample = 0.  An accepted
 * eos_token_id (< 0: none) ends the round without a draw.  Outputs:
 * tokens_out / logprobs_out [batch][k + 1] (the emitted tokens and their
 * target log-probabilities, -1 / 0 past n_out), n_out[b] (tokens emitted;
 * -1 when a draft token lies outside the vocabulary) and n_accepted[b]. */
int32_t pkv_spec_accept(const float* target_logits, const float* draft_logits, int64_t ld,
                        const int64_t* draft_tokens, const int32_t* n_draft, const float* uniforms, int32_t batch,
                        int32_t k, int32_t vocab, float draft_temperature, int32_t do_sample, int64_t eos_token_id,
                        uint64_t seed, uint64_t offset, int64_t* tokens_out, float* logprobs_out, int32_t* n_out,
                        int32_t* n_accepted, int32_t* tickets, void* workspace, int64_t workspace_bytes,
                        void* stream);

#if defined(__GNUC__)
#pragma GCC visibility pop
#endif

#ifdef __cplusplus
}
#endif

#endif /* PKV_B200_H */
