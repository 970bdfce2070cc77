// Byte-exact K/V movement between contiguous caches and the paged pool, the
// copy-on-write block copy, and the block-table / refcount update kernel.
//
// All of these are HBM-bound copies: each thread moves 16-byte vectors where
// the row size, strides and pointers allow it (8/4/2-byte vectors otherwise),
// grids are sized as a multiple of the SM count and loop over the work.
#include "pkv_device.cuh"
#include "pkv_error.h"

#include <string>
#include <unordered_set>

namespace pkv {
namespace {

int elem_size(int32_t dtype) { return dtype == PKV_F32 ? 4 : 2; }

bool check_geom(const pkv_pool_geom* g) {
  if (!g || g->num_layers <= 0 || g->num_blocks <= 0 || g->num_kv_heads <= 0 || g->block_size <= 0 ||
      g->head_dim <= 0 || g->dtype < PKV_F32 || g->dtype > PKV_BF16) {
    pkv_set_error("invalid pool geometry");
    return false;
  }
  return true;
}

int num_sms() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

int32_t launch_status(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    pkv_set_error(std::string(what) + ": " + cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}

// Largest vector width (bytes) dividing every quantity in `vals`.
int vec_width(std::initializer_list<int64_t> vals) {
  for (int w : {16, 8, 4, 2}) {
    bool ok = true;
    for (int64_t v : vals) ok = ok && (v % w == 0);
    if (ok) return w;
  }
  return 0;
}

template <int W>
struct VecT;
template <>
struct VecT<16> { using type = uint4; };
template <>
struct VecT<8> { using type = uint2; };
template <>
struct VecT<4> { using type = uint32_t; };
template <>
struct VecT<2> { using type = uint16_t; };

// One work item = one vector of one (layer, token, state, head) row.
template <int W, bool kToPool>
__global__ void __launch_bounds__(256) move_tokens_kernel(char* __restrict__ pool, char* __restrict__ k_buf,
                                                          char* __restrict__ v_buf, const int64_t* __restrict__ slots,
                                                          int64_t n_tokens, int32_t layer0, int32_t n_layers,
                                                          int32_t num_blocks, int32_t num_kv_heads, int32_t block_size,
                                                          int64_t row_bytes, int64_t layer_stride_b,
                                                          int64_t head_stride_b, int64_t token_stride_b) {
  using V = typename VecT<W>::type;
  const int64_t vecs = row_bytes / W;
  const bool swizzled = page_swizzled(block_size, row_bytes);
  const int64_t total = (int64_t)n_layers * n_tokens * 2 * num_kv_heads * vecs;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    int64_t r = i;
    const int64_t vec = r % vecs;
    r /= vecs;
    const int64_t head = r % num_kv_heads;
    r /= num_kv_heads;
    const int64_t state = r % 2;
    r /= 2;
    const int64_t tok = r % n_tokens;
    const int64_t layer = r / n_tokens;
    const int64_t slot = slots[tok];
    if (slot < 0) continue;
    const int64_t block = slot / block_size;
    const int64_t off = slot % block_size;
    const int64_t page = page_offset(layer0 + layer, block, head, state, num_blocks, num_kv_heads, block_size,
                                     row_bytes);
    V* p = reinterpret_cast<V*>(pool + page + row_byte_offset(off, vec * W, block_size, row_bytes, swizzled));
    char* base = state == 0 ? k_buf : v_buf;
    V* b = reinterpret_cast<V*>(base + layer * layer_stride_b + head * head_stride_b + tok * token_stride_b) + vec;
    if (kToPool) {
      *p = *b;
    } else {
      *b = *p;
    }
  }
}

template <bool kToPool>
int32_t move_tokens(const pkv_pool_geom* g, void* pool, int32_t layer0, int32_t n_layers, const void* k, const void* v,
                    int64_t ls, int64_t hs, int64_t ts, const int64_t* slots, int64_t n_tokens, void* stream) {
  pkv_clear_error();
  if (!check_geom(g)) return PKV_ERR_ARG;
  if (n_tokens < 0 || n_layers < 0 || layer0 < 0 || layer0 + n_layers > g->num_layers) {
    pkv_set_error("token or layer range out of bounds");
    return PKV_ERR_ARG;
  }
  if (n_tokens == 0 || n_layers == 0) return PKV_OK;
  if (!pool || !k || !v || !slots) {
    pkv_set_error("null pointer");
    return PKV_ERR_ARG;
  }
  const int64_t es = elem_size(g->dtype);
  const int64_t row_bytes = (int64_t)g->head_dim * es;
  const int w = vec_width({row_bytes, ls * es, hs * es, ts * es, (int64_t)(uintptr_t)pool, (int64_t)(uintptr_t)k,
                           (int64_t)(uintptr_t)v});
  if (!w) {
    pkv_set_error("buffers are not 2-byte aligned");
    return PKV_ERR_ARG;
  }
  const int64_t total = (int64_t)n_layers * n_tokens * 2 * g->num_kv_heads * (row_bytes / w);
  const int64_t want = (total + 255) / 256;
  const int blocks = (int)std::min<int64_t>(want, (int64_t)num_sms() * 8);
  auto s = static_cast<cudaStream_t>(stream);
  char* kb = (char*)k;
  char* vb = (char*)v;
  char* pb = (char*)pool;
#define PKV_MOVE(WW)                                                                                              \
  move_tokens_kernel<WW, kToPool><<<blocks, 256, 0, s>>>(pb, kb, vb, slots, n_tokens, layer0, n_layers,            \
                                                         g->num_blocks, g->num_kv_heads, g->block_size, row_bytes, \
                                                         ls * es, hs * es, ts * es)
  switch (w) {
    case 16: PKV_MOVE(16); break;
    case 8: PKV_MOVE(8); break;
    case 4: PKV_MOVE(4); break;
    default: PKV_MOVE(2); break;
  }
#undef PKV_MOVE
  return launch_status(kToPool ? "pkv_scatter_tokens" : "pkv_gather_tokens");
}

// Copy whole blocks: per (pair, layer) the (head, state, slot, dim) sub-array
// of a block is one contiguous run of Hkv*2*bs*D elements.
__global__ void __launch_bounds__(256) copy_blocks_kernel(uint4* __restrict__ pool, const int32_t* __restrict__ src,
                                                          const int32_t* __restrict__ dst, int64_t n_pairs,
                                                          int32_t pair_stride, int32_t num_layers,
                                                          int32_t num_blocks, int64_t block_vecs) {
  const int64_t total = n_pairs * num_layers * block_vecs;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t vec = i % block_vecs;
    const int64_t r = i / block_vecs;
    const int64_t layer = r % num_layers;
    const int64_t pair = r / num_layers;
    const int64_t s = src[pair * pair_stride], d = dst[pair * pair_stride];
    pool[(layer * num_blocks + d) * block_vecs + vec] = pool[(layer * num_blocks + s) * block_vecs + vec];
  }
}

__global__ void __launch_bounds__(256) apply_updates_kernel(int32_t* __restrict__ tables, int32_t table_stride,
                                                            int32_t num_rows, int32_t* __restrict__ refcounts,
                                                            int32_t num_blocks, int32_t* __restrict__ lens,
                                                            const int32_t* __restrict__ upd, int64_t n_table,
                                                            int64_t n_ref, int64_t n_len) {
  const int64_t total = n_table + n_ref + n_len;
  const int32_t* tab = upd + 4;
  const int32_t* ref = tab + 3 * n_table;
  const int32_t* len = ref + 2 * n_ref;
  for (int64_t i = blockIdx.x * (int64_t)blockDim.x + threadIdx.x; i < total; i += (int64_t)gridDim.x * blockDim.x) {
    if (i < n_table) {
      const int32_t row = tab[3 * i], col = tab[3 * i + 1];
      if (row >= 0 && row < num_rows && col >= 0 && col < table_stride)
        tables[(int64_t)row * table_stride + col] = tab[3 * i + 2];
    } else if (i < n_table + n_ref) {
      const int64_t j = i - n_table;
      const int32_t b = ref[2 * j];
      if (b >= 0 && b < num_blocks) refcounts[b] = ref[2 * j + 1];
    } else {
      const int64_t j = i - n_table - n_ref;
      const int32_t row = len[2 * j];
      if (row >= 0 && row < num_rows) lens[row] = len[2 * j + 1];
    }
  }
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" {

int64_t pkv_pool_bytes(const pkv_pool_geom* g) {
  return (int64_t)g->num_layers * g->num_blocks * 2 * g->num_kv_heads * g->block_size * g->head_dim *
         elem_size(g->dtype);
}

int32_t pkv_scatter_tokens(const pkv_pool_geom* g, void* pool, int32_t layer0, int32_t n_layers, const void* k_src,
                           const void* v_src, int64_t src_layer_stride, int64_t src_head_stride,
                           int64_t src_token_stride, const int64_t* slot_mapping, int64_t n_tokens, void* stream) {
  return move_tokens<true>(g, pool, layer0, n_layers, k_src, v_src, src_layer_stride, src_head_stride,
                           src_token_stride, slot_mapping, n_tokens, stream);
}

int32_t pkv_gather_tokens(const pkv_pool_geom* g, const void* pool, int32_t layer0, int32_t n_layers, void* k_dst,
                          void* v_dst, int64_t dst_layer_stride, int64_t dst_head_stride, int64_t dst_token_stride,
                          const int64_t* slot_mapping, int64_t n_tokens, void* stream) {
  return move_tokens<false>(g, const_cast<void*>(pool), layer0, n_layers, k_dst, v_dst, dst_layer_stride,
                            dst_head_stride, dst_token_stride, slot_mapping, n_tokens, stream);
}

int32_t pkv_copy_blocks(const pkv_pool_geom* g, void* pool, const int32_t* src_blocks, const int32_t* dst_blocks,
                        int64_t n, void* stream) {
  pkv_clear_error();
  if (!check_geom(g)) return PKV_ERR_ARG;
  if (n <= 0) return PKV_OK;
  const int64_t block_bytes = 2ll * g->num_kv_heads * g->block_size * g->head_dim * elem_size(g->dtype);
  if (block_bytes % 16 != 0 || ((uintptr_t)pool % 16) != 0) {
    pkv_set_error("block copy needs 16-byte aligned blocks");
    return PKV_ERR_ARG;
  }
  const int64_t vecs = block_bytes / 16;
  const int64_t total = n * g->num_layers * vecs;
  const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 8);
  copy_blocks_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<uint4*>(pool), src_blocks, dst_blocks, n, 1, g->num_layers, g->num_blocks, vecs);
  return launch_status("pkv_copy_blocks");
}

int32_t pkv_apply_updates(const pkv_pool_geom* g, void* pool, int32_t* block_tables, int32_t table_stride,
                          int32_t num_rows, int32_t* refcounts, int32_t* context_lens, const int32_t* updates,
                          const int32_t* host_updates, void* stream) {
  pkv_clear_error();
  if (!check_geom(g)) return PKV_ERR_ARG;
  if (!updates || !host_updates) {
    pkv_set_error("null update buffer");
    return PKV_ERR_ARG;
  }
  const int64_t nt = host_updates[0], nr = host_updates[1], nl = host_updates[2], nc = host_updates[3];
  auto s = static_cast<cudaStream_t>(stream);
  const int64_t total = nt + nr + nl;
  if (total > 0) {
    const int blocks = (int)std::min<int64_t>((total + 255) / 256, (int64_t)num_sms() * 4);
    apply_updates_kernel<<<blocks, 256, 0, s>>>(block_tables, table_stride, num_rows, refcounts, g->num_blocks,
                                                 context_lens, updates, nt, nr, nl);
    int32_t st = launch_status("pkv_apply_updates");
    if (st != PKV_OK) return st;
  }
  if (nc <= 0) return PKV_OK;
  // Copy-on-write pairs follow the three update sections as interleaved
  // (src, dst) int32 pairs and must take effect in order.  Pairs are copied in
  // waves in which no block is touched twice, one launch per wave (a chain
  // A->B, B->C gives two waves); the table kernel above never writes the pool.
  const int64_t block_bytes = 2ll * g->num_kv_heads * g->block_size * g->head_dim * elem_size(g->dtype);
  if (block_bytes % 16 != 0 || ((uintptr_t)pool % 16) != 0) {
    pkv_set_error("block copy needs 16-byte aligned blocks");
    return PKV_ERR_ARG;
  }
  const int64_t off = 4 + 3 * nt + 2 * nr + 2 * nl;
  const int32_t* hp = host_updates + off;
  const int32_t* dp = updates + off;
  const int64_t vecs = block_bytes / 16;
  int64_t start = 0;
  while (start < nc) {
    std::unordered_set<int32_t> touched;
    int64_t end = start;
    while (end < nc && !touched.count(hp[2 * end]) && !touched.count(hp[2 * end + 1])) {
      touched.insert(hp[2 * end]);
      touched.insert(hp[2 * end + 1]);
      ++end;
    }
    const int64_t n = end - start;
    const int64_t tot = n * g->num_layers * vecs;
    const int blocks = (int)std::min<int64_t>((tot + 255) / 256, (int64_t)num_sms() * 8);
    copy_blocks_kernel<<<blocks, 256, 0, s>>>(static_cast<uint4*>(pool), dp + 2 * start, dp + 2 * start + 1, n, 2,
                                              g->num_layers, g->num_blocks, vecs);
    int32_t st = launch_status("pkv_apply_updates(copy)");
    if (st != PKV_OK) return st;
    start = end;
  }
  return PKV_OK;
}

}  // extern "C"
