// Chunked-prefill and speculative-verify attention over pages (sm_100a, tcgen05).
//
// Replaces, for one layer, the causal attention of AgentRL's chunked prefill
// (agentrl/generation/prefill.py:96-104: an HF forward per chunk of <= 512
// prompt tokens over the cache of the previous chunks) and of the speculative
// verify forward (agentrl/generation/speculative.py:229-264, whose rows
// prefix_len-1 .. prefix_len-1+k are k+1 causal queries after prefix_len-1
// cached tokens).  Both are "a chunk of queries after `past` cached tokens":
// query i of a chunk sees keys 0 .. past+i (HF's causal mask with a past
// offset, integrations/sdpa_attention.py:40-62), with GQA (query head h reads
// KV head h / (Hq/Hkv)).  The chunk's own K/V are written into their pages
// first (pkv_scatter_tokens), so every key is read from the pool.
//
// Tiles: a CTA owns one work item = (sequence, KV head, up to 128/G chunk
// positions), whose G = Hq/Hkv query heads per position are packed into the
// 128 rows of one tcgen05 tile (row = position * G + head), so the KV head's
// pages are read once for all of its query heads.  Keys stream in tiles of
// 128 (8 pages).  Roles (192 threads):
//   warp 4      producer: per KV tile, 2 KB cp.async.bulk copies of every
//               page's 64-dim K and V slabs into a 2-stage ring (the pool's
//               pages are pre-swizzled, so the slabs land directly in the
//               128-byte-swizzled canonical operand layouts; no tensor map,
//               no multicast);
//   warp 5      allocates 512 tensor-memory columns; lane 0 issues the MMAs:
//               S_j = Q K_j^T into one of two S buffers (M=128, N=128,
//               K-major A and B), and O += P_j V_j (K-major P, MN-major V)
//               into the O accumulator, committing each to mbarriers;
//   warps 0-3   one thread per tile row: Q load (swizzled into shared
//               memory), online softmax on S read from tensor memory
//               (tcgen05.ld), P written as 16-bit into a double-buffered
//               shared tile, lazy rescaling of O in tensor memory (only
//               when a row maximum grows by more than 2^8), and the
//               epilogue O / l -> out.
// S_{j+1} runs on the tensor cores while warps 0-3 turn S_j into P_j.
//
// Every mbarrier wait is bounded; a timed-out role records an error word and
// skips the rest of its work, the MMA thread waits (bounded) for its last
// MMAs and the producer for its copies before tensor memory is freed.
#include "pkv_device.cuh"
#include "pkv_error.h"

#include <algorithm>
#include <string>
#include <type_traits>
#include <vector>

namespace pkv {
namespace {

constexpr int kRows = 128;             // tile rows (M)
constexpr int kKeys = 128;             // keys per KV tile (N of S, K of P.V)
constexpr int kPageRows = 16;          // block_size
constexpr int kPagesPerTile = kKeys / kPageRows;
constexpr int kThreads = 192;
constexpr int kSoftmaxThreads = 128;
constexpr int kTmemCols = 512;         // S buffers 2 x kKeys, O head_dim
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;    // keep a stale row maximum while the new one exceeds it by <= 2^8

template <int D>
struct PCfg {
  static constexpr int kSlabs = D / 64;                    // 64-dim (128-byte) slabs per row
  static constexpr int kQSlabBytes = kRows * 128;
  static constexpr int kQBytes = kSlabs * kQSlabBytes;
  static constexpr int kKVSlabBytes = kKeys * 128;         // one slab of a KV tile
  static constexpr int kKBytes = kSlabs * kKVSlabBytes;    // K (or V) of one KV tile
  static constexpr int kStageBytes = 2 * kKBytes;
  static constexpr int kPSlabBytes = kRows * 128;          // 64 keys of P
  static constexpr int kPBytes = (kKeys / 64) * kPSlabBytes;
  static constexpr int kOffKV = kQBytes;
  static constexpr int kOffP = kOffKV + 2 * kStageBytes;
  static constexpr int kOffBar = kOffP + 2 * kPBytes;
  static constexpr int kSmemBytes = kOffBar + 256 + 1024;  // + barriers, + alignment slack
  static constexpr int kCopiesPerPage = 2 * kSlabs;        // K and V slabs of one page
  static constexpr uint32_t kPageSlabBytes = kPageRows * 128;
};

// Work item (int4): {table row, position of the tile's first query, index of
// that query in the packed q, kv_head << 16 | positions in the tile}.
struct PrefillParams {
  const void* q;    // [total_q][hq][D]
  void* out;        // [total_q][hq][D]
  const char* pool;
  const int32_t* tables;
  const int4* items;
  int32_t* error;
  int64_t total_q;
  int32_t n_items;
  int32_t table_stride;
  int32_t table_rows;
  int32_t hq;
  int32_t hkv;
  int32_t group;
  int32_t layer;
  int32_t num_blocks;
  float scale_log2;
};

struct Bars {
  uint64_t q_full;       // 128 Q-writer arrivals
  uint64_t kv_full[2];   // producer expect_tx + bulk-copy bytes
  uint64_t kv_empty[2];  // MMA commit after P_j V_j
  uint64_t s_full[2];    // MMA commit after S_j
  uint64_t p_full[2];    // 128 softmax arrivals: P_j written, O rescaled, S_j read
  uint64_t o_done[2];    // MMA commit after P_j V_j
  uint64_t mma_done;     // final commit of the MMA thread
  uint32_t tmem_base;
  int32_t abort;
};

__device__ __forceinline__ void record_error(const PrefillParams& p, volatile int32_t* abort, int32_t code) {
  *abort = 1;
  atomicExch(p.error, code);
}

// Bounded wait unless the CTA already gave up.
__device__ __forceinline__ bool wait_or_abort(uint64_t* bar, uint32_t parity, const PrefillParams& p,
                                              volatile int32_t* abort) {
  if (*abort) return false;
  if (mbar_wait_bounded(bar, parity)) return true;
  record_error(p, abort, kDevWaitTimeout);
  return false;
}

template <int D, typename T>
__global__ void __launch_bounds__(kThreads, 1) paged_prefill_kernel(const __grid_constant__ PrefillParams p) {
  using C = PCfg<D>;
  constexpr uint32_t kAbFormat = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t kIdescS = umma_idesc_f16(kAbFormat, 0, 0, kRows, kKeys);
  constexpr uint32_t kIdescO = umma_idesc_f16(kAbFormat, 0, 1, kRows, D);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
  uint8_t* q_s = smem;
  uint8_t* kv_s = smem + C::kOffKV;
  uint8_t* p_s = smem + C::kOffP;
  Bars* bars = reinterpret_cast<Bars*>(smem + C::kOffBar);
  volatile int32_t* abort = &bars->abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  const int4 item = p.items[blockIdx.x];
  const int row = item.x, pos0 = item.y, qrow0 = item.z, h = item.w >> 16, nt = item.w & 0xffff;
  const int kv_len = pos0 + nt;  // keys the tile's last query sees
  const bool ok = row >= 0 && row < p.table_rows && h >= 0 && h < p.hkv && nt >= 1 && nt * p.group <= kRows &&
                  pos0 >= 0 && qrow0 >= 0 && (int64_t)qrow0 + nt <= p.total_q &&
                  (kv_len + kPageRows - 1) / kPageRows <= p.table_stride;
  if (!ok) {  // uniform across the CTA: nothing initialised yet
    if (tid == 0) atomicExch(p.error, kDevBadItem);
    return;
  }
  const int n_tiles = (kv_len + kKeys - 1) / kKeys;

  if (tid == 0) {
    mbar_init(&bars->q_full, kSoftmaxThreads);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&bars->kv_full[i], 1);
      mbar_init(&bars->kv_empty[i], 1);
      mbar_init(&bars->s_full[i], 1);
      mbar_init(&bars->p_full[i], kSoftmaxThreads);
      mbar_init(&bars->o_done[i], 1);
    }
    mbar_init(&bars->mma_done, 1);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == 5) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = bars->tmem_base;
  const uint32_t tmem_o = tmem + 2 * kKeys;

  if (warp == 4) {
    // ---------------- producer ----------------
    const char* layer_base = p.pool;
    const int32_t* trow = p.tables + (int64_t)row * p.table_stride;
    int issued = 0;
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      if (j >= 2 && !__all_sync(0xffffffffu, wait_or_abort(&bars->kv_empty[st], ((j >> 1) - 1) & 1, p, abort)))
        break;
      const int key0 = j * kKeys;
      const int pages = min(kPagesPerTile, (kv_len - key0 + kPageRows - 1) / kPageRows);
      const int copies = pages * C::kCopiesPerPage;
      if (lane == 0) mbar_arrive_expect_tx(&bars->kv_full[st], copies * C::kPageSlabBytes);
      __syncwarp();
      uint8_t* stage = kv_s + st * C::kStageBytes;
      for (int c = lane; c < copies; c += 32) {
        const int pg = c / C::kCopiesPerPage;
        const int kv = (c / C::kSlabs) & 1;
        const int slab = c % C::kSlabs;
        int blk = __ldg(trow + key0 / kPageRows + pg);
        if (blk < 0 || blk >= p.num_blocks) {
          atomicExch(p.error, kDevBadBlock);
          blk = 0;
        }
        const char* src = layer_base +
                          page_offset(p.layer, blk, h, kv, p.num_blocks, p.hkv, kPageRows, D * 2) +
                          slab * C::kPageSlabBytes;
        bulk_copy_g2s(stage + kv * C::kKBytes + slab * C::kKVSlabBytes + pg * C::kPageSlabBytes, src,
                      C::kPageSlabBytes, &bars->kv_full[st]);
      }
      issued = j + 1;
    }
    // Copies still in flight must land before the CTA frees its memory.
    if (lane == 0) {
      for (int j = max(0, issued - 2); j < issued; ++j) mbar_wait_bounded(&bars->kv_full[j & 1], (j >> 1) & 1);
    }
  } else if (warp == 5) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t q_addr = smem_u32(q_s);
      const uint32_t kv_addr = smem_u32(kv_s);
      const uint32_t p_addr = smem_u32(p_s);
      auto issue_pv = [&](int i) -> bool {
        if (!wait_or_abort(&bars->p_full[i & 1], (i >> 1) & 1, p, abort)) return false;
        tc_fence_after_sync();
        const int valid = min(kKeys, kv_len - i * kKeys);
        const int steps = (valid + 15) / 16;
        const uint32_t v_base = kv_addr + (i & 1) * C::kStageBytes + C::kKBytes;
        const uint32_t pb = p_addr + (i & 1) * C::kPBytes;
        for (int ks = 0; ks < steps; ++ks) {
          const uint64_t adesc = umma_desc_sw128(pb + (ks >> 2) * C::kPSlabBytes + (ks & 3) * 32, 16, 1024);
          const uint64_t bdesc = umma_desc_sw128(v_base + ks * 2048, C::kKVSlabBytes, 1024);
          umma_f16_ss(tmem_o, adesc, bdesc, kIdescO, (i > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(&bars->o_done[i & 1]);
        umma_commit(&bars->kv_empty[i & 1]);
        return true;
      };
      bool alive = wait_or_abort(&bars->q_full, 0, p, abort);
      if (alive) tc_fence_after_sync();
      for (int j = 0; alive && j < n_tiles; ++j) {
        const int st = j & 1;
        if (!wait_or_abort(&bars->kv_full[st], (j >> 1) & 1, p, abort)) {
          alive = false;
          break;
        }
        tc_fence_after_sync();
        const uint32_t k_base = kv_addr + st * C::kStageBytes;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * C::kQSlabBytes + (ks & 3) * 32;
          const uint64_t adesc = umma_desc_sw128(q_addr + off, 16, 1024);
          const uint64_t bdesc = umma_desc_sw128(k_base + (ks >> 2) * C::kKVSlabBytes + (ks & 3) * 32, 16, 1024);
          umma_f16_ss(tmem + st * kKeys, adesc, bdesc, kIdescS, ks > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[st]);
        if (j > 0 && !issue_pv(j - 1)) alive = false;
      }
      if (alive) issue_pv(n_tiles - 1);
      // Every MMA issued must complete before tensor memory is freed.
      umma_commit(&bars->mma_done);
      mbar_wait_bounded(&bars->mma_done, 0);
    }
    __syncwarp();
  } else {
    // ---------------- softmax / epilogue (thread = tile row) ----------------
    const int r = tid;
    const int group = p.group;
    const int rows_valid = nt * group;
    const T* qbase = static_cast<const T*>(p.q);
    {
      const bool in = r < rows_valid;
      const T* src = qbase + (((int64_t)qrow0 + r / group) * p.hq + (int64_t)h * group + r % group) * D;
#pragma unroll
      for (int c = 0; c < D / 8; ++c) {
        uint4 v = make_uint4(0, 0, 0, 0);
        if (in) v = __ldg(reinterpret_cast<const uint4*>(src) + c);
        *reinterpret_cast<uint4*>(q_s + (c >> 3) * C::kQSlabBytes + swz128(r, c & 7)) = v;
      }
      fence_proxy_async_smem();
      mbar_arrive(&bars->q_full);
    }
    const int pos_r = pos0 + min(r / group, nt - 1);  // padding rows repeat the last position
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    float m_run = -INFINITY, l_run = 0.f;
    bool alive = true;
    for (int j = 0; j < n_tiles; ++j) {
      const int st = j & 1;
      if (!__all_sync(0xffffffffu, wait_or_abort(&bars->s_full[st], (j >> 1) & 1, p, abort))) {
        alive = false;
        break;
      }
      tc_fence_after_sync();
      const uint32_t s_addr = tmem + lane_base + st * kKeys;
      const int key0 = j * kKeys;
      // Pass 1: row maximum over the visible keys.
      float mx = -INFINITY;
#pragma unroll 1
      for (int cc = 0; cc < kKeys / 32; ++cc) {
        float v[32];
        tmem_ld32(s_addr + cc * 32, v);
#pragma unroll
        for (int i = 0; i < 32; ++i)
          if (key0 + cc * 32 + i <= pos_r) mx = fmaxf(mx, v[i]);
      }
      mx *= p.scale_log2;
      float alpha = 1.f;
      bool rescale = false;
      if (mx > m_run + kRescaleLog2) {
        alpha = exp2f(m_run - mx);
        l_run *= alpha;
        m_run = mx;
        rescale = j > 0;
      }
      // P_j goes into the buffer P_{j-2} used: that product must be done.
      if (j >= 2 &&
          !__all_sync(0xffffffffu, wait_or_abort(&bars->o_done[st], ((j >> 1) - 1) & 1, p, abort))) {
        alive = false;
        break;
      }
      // Pass 2: P = exp2(S * scale * log2e - m) for visible keys, 0 elsewhere.
      uint8_t* pb = p_s + st * C::kPBytes;
#pragma unroll 1
      for (int cc = 0; cc < kKeys / 32; ++cc) {
        float v[32];
        tmem_ld32(s_addr + cc * 32, v);
        uint32_t pk[16];
#pragma unroll
        for (int i = 0; i < 32; i += 2) {
          const float p0 = key0 + cc * 32 + i <= pos_r ? exp2f(fmaf(v[i], p.scale_log2, -m_run)) : 0.f;
          const float p1 = key0 + cc * 32 + i + 1 <= pos_r ? exp2f(fmaf(v[i + 1], p.scale_log2, -m_run)) : 0.f;
          l_run += p0 + p1;
          pk[i >> 1] = MmaOp<T>::pack(p0, p1);
        }
        uint8_t* prow = pb + (cc >> 1) * C::kPSlabBytes;
#pragma unroll
        for (int c = 0; c < 4; ++c)
          *reinterpret_cast<uint4*>(prow + swz128(r, (cc & 1) * 4 + c)) =
              make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
      }
      // Last tile: V rows past the sequence inside its last page are zeroed
      // so that their zero probabilities multiply finite values.
      if (j == n_tiles - 1 && (kv_len & (kPageRows - 1)) != 0) {
        if (!__all_sync(0xffffffffu, wait_or_abort(&bars->kv_full[st], (j >> 1) & 1, p, abort))) {
          alive = false;
          break;
        }
        const int first = kv_len - key0;                       // first stale row of the tile
        const int last = (first + kPageRows - 1) & ~(kPageRows - 1);
        uint8_t* vb = kv_s + st * C::kStageBytes + C::kKBytes;
        for (int c = r; c < (last - first) * 8 * C::kSlabs; c += kSoftmaxThreads) {
          const int slab = c / ((last - first) * 8);
          const int rem = c % ((last - first) * 8);
          *reinterpret_cast<uint4*>(vb + slab * C::kKVSlabBytes + swz128(first + rem / 8, rem & 7)) =
              make_uint4(0, 0, 0, 0);
        }
      }
      // O *= alpha for rows whose maximum moved (after P_{j-1} V_{j-1} is done).
      if (__any_sync(0xffffffffu, rescale)) {
        if (!__all_sync(0xffffffffu,
                        wait_or_abort(&bars->o_done[(j - 1) & 1], ((j - 1) >> 1) & 1, p, abort))) {
          alive = false;
          break;
        }
        tc_fence_after_sync();
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          float v[32];
          tmem_ld32(tmem_o + lane_base + cc * 32, v);
#pragma unroll
          for (int i = 0; i < 32; ++i) v[i] *= alpha;
          tmem_st32(tmem_o + lane_base + cc * 32, v);
        }
      }
      fence_proxy_async_smem();
      tc_fence_before_sync();
      mbar_arrive(&bars->p_full[st]);
    }
    if (alive) {
      const int last = n_tiles - 1;
      if (__all_sync(0xffffffffu, wait_or_abort(&bars->o_done[last & 1], (last >> 1) & 1, p, abort))) {
        tc_fence_after_sync();
        const float inv_l = 1.f / l_run;
        T* dst = static_cast<T*>(p.out) + (((int64_t)qrow0 + r / group) * p.hq + (int64_t)h * group + r % group) * D;
#pragma unroll 1
        for (int cc = 0; cc < D / 32; ++cc) {
          float v[32];
          tmem_ld32(tmem_o + lane_base + cc * 32, v);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 32; i += 2) pk[i >> 1] = MmaOp<T>::pack(v[i] * inv_l, v[i + 1] * inv_l);
          if (r < rows_valid) {
#pragma unroll
            for (int c = 0; c < 4; ++c)
              reinterpret_cast<uint4*>(dst + cc * 32)[c] = make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2],
                                                                      pk[4 * c + 3]);
          }
        }
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == 5) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, typename T>
cudaError_t launch_prefill(const PrefillParams& prm, cudaStream_t stream) {
  using C = PCfg<D>;
  static_assert(C::kSmemBytes <= 232448, "prefill tile exceeds the shared memory of one CTA");
  auto kern = paged_prefill_kernel<D, T>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (err != cudaSuccess) return err;
  kern<<<prm.n_items, kThreads, C::kSmemBytes, stream>>>(prm);
  return cudaGetLastError();
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int32_t pkv_prefill_positions_per_item(int32_t num_q_heads, int32_t num_kv_heads) {
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads != 0) return 0;
  const int group = num_q_heads / num_kv_heads;
  return group > kRows ? 0 : kRows / group;
}

extern "C" int32_t pkv_prefill_plan(const int32_t* rows, const int32_t* past_lens, const int32_t* q_lens,
                                    int32_t n_seqs, int32_t num_q_heads, int32_t num_kv_heads, int32_t* items_out,
                                    int64_t items_capacity, int64_t* n_items_out) {
  pkv_clear_error();
  const int ppi = pkv_prefill_positions_per_item(num_q_heads, num_kv_heads);
  if (ppi <= 0 || num_kv_heads > 0x7fff) {
    pkv_set_error("num_q_heads must be a positive multiple of num_kv_heads with at most 128 query heads per KV head");
    return PKV_ERR_UNSUPPORTED;
  }
  if (n_seqs < 0 || !n_items_out || (n_seqs > 0 && (!rows || !past_lens || !q_lens))) {
    pkv_set_error("invalid plan arguments");
    return PKV_ERR_ARG;
  }
  struct Entry {
    int64_t kv_len;
    int32_t v[4];
  };
  std::vector<Entry> entries;
  int64_t qrow = 0;
  for (int32_t i = 0; i < n_seqs; ++i) {
    if (rows[i] < 0 || past_lens[i] < 0 || q_lens[i] < 0) {
      pkv_set_error("negative row, past length or query count for sequence " + std::to_string(i));
      return PKV_ERR_VALUE;
    }
    if ((int64_t)past_lens[i] + q_lens[i] > INT32_MAX || qrow + q_lens[i] > INT32_MAX) {
      pkv_set_error("sequence or query count too large");
      return PKV_ERR_VALUE;
    }
    for (int32_t t0 = 0; t0 < q_lens[i]; t0 += ppi) {
      const int32_t n = std::min(ppi, q_lens[i] - t0);
      for (int32_t hk = 0; hk < num_kv_heads; ++hk)
        entries.push_back({(int64_t)past_lens[i] + t0 + n,
                           {rows[i], past_lens[i] + t0, static_cast<int32_t>(qrow + t0), (hk << 16) | n}});
    }
    qrow += q_lens[i];
  }
  *n_items_out = static_cast<int64_t>(entries.size());
  if (!items_out) return PKV_OK;
  if ((int64_t)entries.size() > items_capacity) {
    pkv_set_error("item buffer too small: need " + std::to_string(entries.size()) + " items");
    return PKV_ERR_CAPACITY;
  }
  // Longest key range first, so the grid's tail holds the short tiles.
  std::stable_sort(entries.begin(), entries.end(),
                   [](const Entry& a, const Entry& b) { return a.kv_len > b.kv_len; });
  for (size_t i = 0; i < entries.size(); ++i)
    for (int k = 0; k < 4; ++k) items_out[4 * i + k] = entries[i].v[k];
  return PKV_OK;
}

extern "C" int32_t pkv_prefill_attention(const pkv_pool_geom* g, const void* pool, int32_t layer, const void* q,
                                         const int32_t* block_tables, int32_t table_stride, int32_t table_rows,
                                         const int32_t* work_items, int32_t n_items, int64_t total_q,
                                         int32_t num_q_heads, float scale, void* out, int32_t* error_word,
                                         void* stream) {
  pkv_clear_error();
  if (!g || g->block_size != kPageRows) {
    pkv_set_error("paged prefill attention needs block_size 16");
    return PKV_ERR_UNSUPPORTED;
  }
  if (g->dtype != PKV_BF16 && g->dtype != PKV_F16) {
    pkv_set_error("paged prefill attention supports bf16 and f16 pools");
    return PKV_ERR_UNSUPPORTED;
  }
  if (g->head_dim != 64 && g->head_dim != 128) {
    pkv_set_error("paged prefill attention supports head_dim 64 and 128");
    return PKV_ERR_UNSUPPORTED;
  }
  if (pkv_prefill_positions_per_item(num_q_heads, g->num_kv_heads) <= 0 || g->num_kv_heads > 0x7fff) {
    pkv_set_error("num_q_heads must be a positive multiple of num_kv_heads with at most 128 query heads per KV head");
    return PKV_ERR_UNSUPPORTED;
  }
  if (layer < 0 || layer >= g->num_layers || n_items < 0 || total_q < 0 || table_stride <= 0 || table_rows <= 0 ||
      !(scale > 0.f)) {
    pkv_set_error("invalid layer, item, query, table or scale arguments");
    return PKV_ERR_ARG;
  }
  if (n_items == 0) return PKV_OK;
  if (!pool || !q || !out || !block_tables || !work_items || !error_word) {
    pkv_set_error("null pointer argument");
    return PKV_ERR_ARG;
  }
  if ((uintptr_t)pool % 16 != 0 || (uintptr_t)q % 16 != 0 || (uintptr_t)out % 16 != 0 ||
      (uintptr_t)work_items % 16 != 0) {
    pkv_set_error("pool, q, out and work_items must be 16-byte aligned");
    return PKV_ERR_ARG;
  }
  PrefillParams prm;
  prm.q = q;
  prm.out = out;
  prm.pool = static_cast<const char*>(pool);
  prm.tables = block_tables;
  prm.items = reinterpret_cast<const int4*>(work_items);
  prm.error = error_word;
  prm.total_q = total_q;
  prm.n_items = n_items;
  prm.table_stride = table_stride;
  prm.table_rows = table_rows;
  prm.hq = num_q_heads;
  prm.hkv = static_cast<int32_t>(g->num_kv_heads);
  prm.group = num_q_heads / static_cast<int32_t>(g->num_kv_heads);
  prm.layer = layer;
  prm.num_blocks = static_cast<int32_t>(g->num_blocks);
  prm.scale_log2 = scale * kLog2e;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err;
  if (g->head_dim == 128)
    err = g->dtype == PKV_BF16 ? launch_prefill<128, __nv_bfloat16>(prm, s) : launch_prefill<128, __half>(prm, s);
  else
    err = g->dtype == PKV_BF16 ? launch_prefill<64, __nv_bfloat16>(prm, s) : launch_prefill<64, __half>(prm, s);
  if (err != cudaSuccess) {
    pkv_set_error(std::string("prefill launch failed: ") + cudaGetErrorString(err));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}
