// Entry points shared between the library's translation units (not exported).
#pragma once
#include <stdint.h>

#include "pkv_b200.h"

// Decode launch shape.  A warp owns a ring of bulk-copy stages totalling
// PKV_DECODE_RING_BYTES / warps; stages of 16 KB or more (D = 128, two KV
// heads) run PKV_DECODE_WARPS_BIG warps per CTA, smaller stages 8.  The
// planner sizes work items for about PKV_DECODE_ITEMS_PER_WARP items per warp
// of the persistent grid.
#ifndef PKV_DECODE_WARPS_BIG
#define PKV_DECODE_WARPS_BIG 5
#endif
#ifndef PKV_DECODE_RING_BYTES
#define PKV_DECODE_RING_BYTES (200 * 1024)
#endif
#ifndef PKV_DECODE_ITEMS_PER_WARP
#define PKV_DECODE_ITEMS_PER_WARP 3
#endif
// Splits of one (sequence, head) the split-K combine loads per round (its
// registers, hence how many of its blocks stay resident beside the decode CTA).
#ifndef PKV_COMBINE_BATCH
#define PKV_COMBINE_BATCH 16
#endif
// Work-item order of the decode plan: 1 = items by decreasing page count
// (the grid's tail holds the smallest items: 54.8-55.8 vs 55.9-57.1 us per
// microbench launch); 0 = sequences by decreasing length, each sequence's
// items together.
#ifndef PKV_DECODE_ORDER
#define PKV_DECODE_ORDER 1
#endif
// Prefer the largest shared-memory carveout for the decode and combine kernels.
#ifndef PKV_CARVEOUT_MAX
#define PKV_CARVEOUT_MAX 0
#endif
// Launch the decode grid as a programmatic dependent of the kernel before it
// on the stream (its CTAs get resident during that kernel's last blocks).
#ifndef PKV_DECODE_PDL
#define PKV_DECODE_PDL 0
#endif

// pkv_decode_attention plus length / refcount updates the decode does not
// read, applied by the kernel itself: `deferred` holds deferred_refs
// (block, refcount) pairs then deferred_lens (row, length) pairs.
// Fixed-step mode (for launches recorded in a CUDA graph): with step_header
// non-NULL the kernels read {n_items, n_combine, batch, pages_per_split,
// deferred_refs, deferred_lens} from it at run time (the arguments then give
// capacities), and the combine entries come from combine_entries (otherwise
// they follow the n_items work items).
int32_t pkv_decode_attention_ex(const pkv_pool_geom* g, void* pool, int32_t layer, const void* q, const void* k_new,
                                const void* v_new, int32_t* block_tables, int32_t table_stride, int32_t table_rows,
                                int32_t* context_lens, const int32_t* rows, const int32_t* seq_lens,
                                const int32_t* new_blocks, const int32_t* work_items, int32_t n_items,
                                int32_t n_combine, int32_t batch, int32_t num_q_heads, int32_t pages_per_split,
                                float scale, void* out, void* workspace, int64_t workspace_bytes, void* stream,
                                const int32_t* deferred, int32_t deferred_refs, int32_t deferred_lens,
                                int32_t* refcounts, const int32_t* step_header, const int32_t* combine_entries);
