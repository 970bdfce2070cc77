// Paged GQA decode attention for sm_100a, fused with the step's K/V append.
//
// Replaces, for one decode step of one layer, what AgentRL's continuous loop
// does through HF (agentrl/generation/continuous.py:476-483): the torch.cat
// append into each resident cache (transformers cache_utils.py:119-120) and
// sdpa_attention_forward with GQA (integrations/sdpa_attention.py:40-62).
//
// Work decomposition: one CTA per (split work item, KV head).  A work item is
// `pages_per_split` consecutive 16-token pages of one sequence; the host lays
// the items out with split_offsets.  The CTA serves all G = Hq/Hkv query heads
// of its KV head from a single read of each page (GQA reuse).
//
// Inside the CTA, 4 warps take interleaved pages, each warp running its own
// 3-stage TMA pipeline: one lane arms an mbarrier and issues 128-byte-swizzled
// 3-D tensor loads of the page's K and V rows (no multicast).  Per page the
// warp computes S^T[16 tokens x 8 heads] = K Q^T and O^T[D x 8] += V^T P^T
// with mma.sync m16n8k16 (A fragments by ldmatrix from the swizzled stage,
// P^T fragments by movmatrix.trans from the S^T accumulators), and keeps the
// online softmax per head with warp shuffles (Milakov & Gimelshein 2018).
// The 4 warps merge through shared memory; a sequence with several splits
// writes (O, m, l) partials to the workspace and the last CTA to finish (an
// atomic ticket, no spinning) combines them.
//
// Arithmetic: fp32 scores and accumulation, P rounded to the input dtype for
// the P.V product, output rounded once to the input dtype.
#include "pkv_device.cuh"
#include "pkv_error.h"

#include <cudaTypedefs.h>

#include <map>
#include <mutex>
#include <string>
#include <tuple>

namespace pkv {
namespace {

constexpr int kWarps = 4;
constexpr int kStages = 3;
constexpr int kMaxSplitsPerSeq = 64;
constexpr float kLog2e = 1.4426950408889634f;

template <int D>
struct Geo {
  static constexpr int kHalves = D / 64;            // 128-byte TMA boxes per row
  static constexpr int kPageBytes = 16 * D * 2;     // one K (or V) page of one head
  static constexpr int kStageBytes = 2 * kPageBytes;
  static constexpr int kSmemBytes = kWarps * kStages * kStageBytes + 1024;
  static constexpr int kVecsPerRow = D * 2 / 16;    // 16-byte chunks per token row
};

struct DecodeParams {
  const void* q;
  const void* k_new;
  const void* v_new;
  void* out;
  void* pool;
  int32_t* tables;
  int32_t* ctx_lens;
  const int32_t* rows;
  const int32_t* seq_lens;
  const int32_t* new_blocks;
  const int32_t* split_offsets;
  float* ws_ml;
  float* ws_o;
  int32_t* ws_counters;
  int32_t* ws_error;
  int32_t table_stride;
  int32_t batch;
  int32_t hq;
  int32_t hkv;
  int32_t group;
  int32_t layer;
  int32_t num_blocks;
  int32_t pages_per_split;
  float scale_log2;
};

template <int D, typename T>
__global__ void __launch_bounds__(kWarps * 32) paged_decode_kernel(const __grid_constant__ CUtensorMap tmap,
                                                                   const DecodeParams p) {
  using G = Geo<D>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bars[kWarps * kStages];
  __shared__ float s_m[kWarps][8];
  __shared__ float s_l[kWarps][8];
  __shared__ float s_w[kMaxSplitsPerSeq][8];
  __shared__ int s_last;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;
  const int item = blockIdx.x;
  const int h = blockIdx.y;

  // Sequence owning this work item: largest b with split_offsets[b] <= item.
  int lo = 0, hi = p.batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (__ldg(p.split_offsets + mid) <= item) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  const int first_item = __ldg(p.split_offsets + b);
  const int nsplits = __ldg(p.split_offsets + b + 1) - first_item;
  const int split = item - first_item;
  const int row = __ldg(p.rows + b);
  const int len = __ldg(p.seq_lens + b);
  const int npages = (len + 15) >> 4;
  const int pg0 = split * p.pages_per_split;
  const int pg1 = min(pg0 + p.pages_per_split, npages);
  const int last_page = npages - 1;
  const int new_block = p.new_blocks ? __ldg(p.new_blocks + b) : -1;
  int32_t* table_row = p.tables + (int64_t)row * p.table_stride;
  if (nsplits > kMaxSplitsPerSeq) {  // the host never builds such offsets; refuse rather than overflow
    if (tid == 0) atomicExch(p.ws_error, kDevBadSplits);
    return;
  }
  const T* kn = static_cast<const T*>(p.k_new);
  const T* vn = static_cast<const T*>(p.v_new);

  // Fused append: write the step's K/V row into its slot (for later steps;
  // this step patches it into shared memory below).
  if (kn != nullptr && pg1 == npages) {
    const int pos = len - 1;
    const int blk = new_block >= 0 ? new_block : table_row[pos >> 4];
    const int slot = pos & 15;
    if (tid < 2 * G::kVecsPerRow) {
      const int state = tid / G::kVecsPerRow;
      const int vec = tid % G::kVecsPerRow;
      const T* src = (state == 0 ? kn : vn) + ((int64_t)b * p.hkv + h) * D;
      const int64_t prow = pool_row_index(p.layer, blk, state, h, slot, p.num_blocks, p.hkv, 16);
      reinterpret_cast<uint4*>(static_cast<T*>(p.pool) + prow * D)[vec] = reinterpret_cast<const uint4*>(src)[vec];
    }
    if (h == 0 && tid == 0) {
      if (new_block >= 0) table_row[pos >> 4] = new_block;
      p.ctx_lens[row] = len;
    }
  }

  if (tid == 0) {
    prefetch_tmap(&tmap);
    for (int i = 0; i < kWarps * kStages; ++i) mbar_init(&bars[i], 1);
    fence_barrier_init();
  }
  __syncthreads();

  // Q^T fragments (B operand, col layout): head = lane/4, dims 2*(lane%4)+{0,1} (+8).
  constexpr int KK = D / 16;
  uint32_t qf[KK][2];
  {
    const int g = lane >> 2;
    const T* qrow = static_cast<const T*>(p.q) + ((int64_t)b * p.hq + h * p.group + g) * D;
#pragma unroll
    for (int kk = 0; kk < KK; ++kk) {
      if (g < p.group) {
        qf[kk][0] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * (lane & 3));
        qf[kk][1] = *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 8 + 2 * (lane & 3));
      } else {
        qf[kk][0] = 0u;
        qf[kk][1] = 0u;
      }
    }
  }

  const int span = pg1 - pg0;
  const int n_my = span > warp ? (span - warp + kWarps - 1) / kWarps : 0;
  uint8_t* wsm = smem + warp * kStages * G::kStageBytes;
  uint64_t* wbar = bars + warp * kStages;

  auto issue = [&](int i) {
    const int pg = pg0 + warp + i * kWarps;
    const int st = i % kStages;
    const int blk = (pg == last_page && new_block >= 0) ? new_block : table_row[pg];
    uint8_t* dst = wsm + st * G::kStageBytes;
    const int rk = ((blk * 2 + 0) * p.hkv + h) * 16;
    const int rv = ((blk * 2 + 1) * p.hkv + h) * 16;
    mbar_arrive_expect_tx(&wbar[st], G::kStageBytes);
#pragma unroll
    for (int j = 0; j < G::kHalves; ++j) {
      tma_load_3d(dst + j * 2048, &tmap, 64 * j, rk, p.layer, &wbar[st]);
      tma_load_3d(dst + G::kPageBytes + j * 2048, &tmap, 64 * j, rv, p.layer, &wbar[st]);
    }
  };

  int issued = min(kStages, n_my);
  if (lane == 0) {
    for (int i = 0; i < issued; ++i) issue(i);
  }
  __syncwarp();

  float m_a = -INFINITY, m_b = -INFINITY, l_a = 0.f, l_b = 0.f;
  float oacc[KK][4];
#pragma unroll
  for (int mt = 0; mt < KK; ++mt) oacc[mt][0] = oacc[mt][1] = oacc[mt][2] = oacc[mt][3] = 0.f;

  int failed_at = -1;
  for (int i = 0; i < n_my; ++i) {
    const int st = i % kStages;
    const bool ok = mbar_wait_bounded(&wbar[st], (i / kStages) & 1);
    if (!__all_sync(0xffffffffu, ok)) {  // warp-uniform exit
      failed_at = i;
      break;
    }
    const int pg = pg0 + warp + i * kWarps;
    const int valid = min(16, len - pg * 16);
    uint8_t* stage = wsm + st * G::kStageBytes;
    const uint32_t sk = smem_u32(stage);
    const uint32_t sv = sk + G::kPageBytes;

    if (pg == last_page) {
      // Patch the step's token (the slot may have been read before the
      // append above landed) and zero V rows past the context so that
      // masked probabilities multiply finite values.
      if (kn != nullptr && lane < 2 * G::kVecsPerRow) {
        const int state = lane / G::kVecsPerRow;
        const int vec = lane % G::kVecsPerRow;
        const T* src = (state == 0 ? kn : vn) + ((int64_t)b * p.hkv + h) * D;
        const int slot = valid - 1;
        uint8_t* dst = stage + state * G::kPageBytes + (vec >> 3) * 2048 + swz128(slot, vec & 7);
        *reinterpret_cast<uint4*>(dst) = reinterpret_cast<const uint4*>(src)[vec];
      }
      for (int c = lane; c < (16 - valid) * G::kVecsPerRow; c += 32) {
        const int r = valid + c / G::kVecsPerRow;
        const int vec = c % G::kVecsPerRow;
        *reinterpret_cast<uint4*>(stage + G::kPageBytes + (vec >> 3) * 2048 + swz128(r, vec & 7)) =
            make_uint4(0u, 0u, 0u, 0u);
      }
      __syncwarp();
    }

    // S^T = K Q^T  (M = 16 tokens, N = 8 heads, K = D)
    float sacc[4] = {0.f, 0.f, 0.f, 0.f};
    {
      const int tok = (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
      for (int kk = 0; kk < KK; ++kk) {
        const int dim = kk * 16 + 8 * (lane >> 4);
        uint32_t a[4];
        ldmatrix_x4(sk + (dim >> 6) * 2048 + swz128(tok, (dim & 63) >> 3), a[0], a[1], a[2], a[3]);
        MmaOp<T>::run(sacc, a, qf[kk]);
      }
    }

    // Online softmax per head column (heads 2*(lane%4) and +1).
    const bool va = (lane >> 2) < valid;
    const bool vb = (lane >> 2) + 8 < valid;
    const float s0 = va ? sacc[0] * p.scale_log2 : -INFINITY;
    const float s1 = va ? sacc[1] * p.scale_log2 : -INFINITY;
    const float s2 = vb ? sacc[2] * p.scale_log2 : -INFINITY;
    const float s3 = vb ? sacc[3] * p.scale_log2 : -INFINITY;
    float mx_a = fmaxf(s0, s2), mx_b = fmaxf(s1, s3);
#pragma unroll
    for (int off = 4; off < 32; off <<= 1) {
      mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
      mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
    }
    const float mn_a = fmaxf(m_a, mx_a), mn_b = fmaxf(m_b, mx_b);
    const float al_a = exp2f(m_a - mn_a), al_b = exp2f(m_b - mn_b);
    const float p0 = exp2f(s0 - mn_a), p1 = exp2f(s1 - mn_b);
    const float p2 = exp2f(s2 - mn_a), p3 = exp2f(s3 - mn_b);
    l_a = l_a * al_a + p0 + p2;
    l_b = l_b * al_b + p1 + p3;
    m_a = mn_a;
    m_b = mn_b;
#pragma unroll
    for (int mt = 0; mt < KK; ++mt) {
      oacc[mt][0] *= al_a;
      oacc[mt][1] *= al_b;
      oacc[mt][2] *= al_a;
      oacc[mt][3] *= al_b;
    }
    uint32_t pb[2];
    pb[0] = movmatrix_trans(MmaOp<T>::pack(p0, p1));
    pb[1] = movmatrix_trans(MmaOp<T>::pack(p2, p3));

    // O^T += V^T P^T  (M = D dims in tiles of 16, N = 8 heads, K = 16 tokens)
    {
      const int tok = (lane & 7) + 8 * (lane >> 4);
#pragma unroll
      for (int mt = 0; mt < KK; ++mt) {
        const int dim = mt * 16 + 8 * ((lane >> 3) & 1);
        uint32_t a[4];
        ldmatrix_x4_trans(sv + (dim >> 6) * 2048 + swz128(tok, (dim & 63) >> 3), a[0], a[1], a[2], a[3]);
        MmaOp<T>::run(oacc[mt], a, pb);
      }
    }

    if (i + kStages < n_my) {
      __syncwarp();
      fence_proxy_async_smem();
      if (lane == 0) issue(i + kStages);
      ++issued;
      __syncwarp();
    }
  }

  if (failed_at >= 0) {
    // Record the failure, then give the loads still in flight one more
    // bounded wait each before this warp's stages are reused or released.
    if (lane == 0) atomicExch(p.ws_error, kDevWaitTimeout);
    for (int i = failed_at; i < issued; ++i) mbar_wait_bounded(&wbar[i % kStages], (i / kStages) & 1);
  }
#pragma unroll
  for (int off = 4; off < 32; off <<= 1) {
    l_a += __shfl_xor_sync(0xffffffffu, l_a, off);
    l_b += __shfl_xor_sync(0xffffffffu, l_b, off);
  }
  __syncthreads();  // every warp is done with its stages: reuse them for the merge

  float* red = reinterpret_cast<float*>(smem);  // [kWarps][8][D]
  {
    float* wr = red + warp * 8 * D;
    const int ha = 2 * (lane & 3), hb = ha + 1;
#pragma unroll
    for (int mt = 0; mt < KK; ++mt) {
      const int d0 = mt * 16 + (lane >> 2);
      wr[ha * D + d0] = oacc[mt][0];
      wr[hb * D + d0] = oacc[mt][1];
      wr[ha * D + d0 + 8] = oacc[mt][2];
      wr[hb * D + d0 + 8] = oacc[mt][3];
    }
    if (lane < 4) {
      s_m[warp][ha] = n_my > 0 ? m_a : -INFINITY;
      s_m[warp][hb] = n_my > 0 ? m_b : -INFINITY;
      s_l[warp][ha] = n_my > 0 ? l_a : 0.f;
      s_l[warp][hb] = n_my > 0 ? l_b : 0.f;
    }
  }
  __syncthreads();

  const int group = p.group;
  T* out = static_cast<T*>(p.out);
  const int64_t wi = (int64_t)item * p.hkv + h;
  for (int idx = tid; idx < group * D; idx += kWarps * 32) {
    const int g = idx / D, d = idx % D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) mm = fmaxf(mm, s_m[w][g]);
    float o = 0.f, l = 0.f;
#pragma unroll
    for (int w = 0; w < kWarps; ++w) {
      const float wgt = exp2f(s_m[w][g] - mm);
      o += wgt * red[(w * 8 + g) * D + d];
      l += wgt * s_l[w][g];
    }
    if (nsplits == 1) {
      out[((int64_t)b * p.hq + h * group + g) * D + d] = MmaOp<T>::from_float(o / l);
    } else {
      p.ws_o[(wi * 8 + g) * D + d] = o;
      if (d == 0) {
        p.ws_ml[wi * 16 + g] = mm;
        p.ws_ml[wi * 16 + 8 + g] = l;
      }
    }
  }
  if (nsplits == 1) return;

  // Split-K combine by the last CTA of this (sequence, KV head).
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    const int ticket = atomicAdd(p.ws_counters + (int64_t)b * p.hkv + h, 1);
    s_last = ticket == nsplits - 1;
  }
  __syncthreads();
  if (!s_last) return;
  __threadfence();
  const int64_t base = (int64_t)first_item * p.hkv + h;
  if (tid < group) {
    const int g = tid;
    float mm = -INFINITY;
    for (int s = 0; s < nsplits; ++s) mm = fmaxf(mm, __ldcg(p.ws_ml + (base + (int64_t)s * p.hkv) * 16 + g));
    float l = 0.f;
    for (int s = 0; s < nsplits; ++s) {
      const int64_t si = base + (int64_t)s * p.hkv;
      const float wgt = exp2f(__ldcg(p.ws_ml + si * 16 + g) - mm);
      s_w[s][g] = wgt;
      l += wgt * __ldcg(p.ws_ml + si * 16 + 8 + g);
    }
    s_l[0][g] = 1.f / l;
  }
  __syncthreads();
  for (int idx = tid; idx < group * D; idx += kWarps * 32) {
    const int g = idx / D, d = idx % D;
    float o = 0.f;
    for (int s = 0; s < nsplits; ++s)
      o += s_w[s][g] * __ldcg(p.ws_o + ((base + (int64_t)s * p.hkv) * 8 + g) * D + d);
    out[((int64_t)b * p.hq + h * group + g) * D + d] = MmaOp<T>::from_float(o * s_l[0][g]);
  }
  if (tid == 0) p.ws_counters[(int64_t)b * p.hkv + h] = 0;
}

// ---------------------------------------------------------------------------
// Host side: tensor maps and launch.

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

// Pool viewed as a 3-D tensor {head_dim, rows of one layer, layers} with
// 128-byte-swizzled boxes of {64 elements, 16 rows, 1}: one box is one half
// (64 dims) of one K or V page of one KV head.
bool make_pool_map(const pkv_pool_geom* g, void* pool, CUtensorMap* out) {
  using Key = std::tuple<uintptr_t, int, int, int, int, int>;
  static std::map<Key, CUtensorMap> cache;
  static std::mutex mu;
  Key key{(uintptr_t)pool, g->num_layers, g->num_blocks, g->num_kv_heads, g->head_dim, g->dtype};
  std::lock_guard<std::mutex> lock(mu);
  auto it = cache.find(key);
  if (it != cache.end()) {
    *out = it->second;
    return true;
  }
  auto encode = get_encode_fn();
  if (!encode) {
    pkv_set_error("cuTensorMapEncodeTiled is unavailable from the driver");
    return false;
  }
  const uint64_t rows = (uint64_t)g->num_blocks * 2 * g->num_kv_heads * 16;
  cuuint64_t dims[3] = {(cuuint64_t)g->head_dim, rows, (cuuint64_t)g->num_layers};
  cuuint64_t strides[2] = {(cuuint64_t)g->head_dim * 2, rows * g->head_dim * 2};
  cuuint32_t box[3] = {64, 16, 1};
  cuuint32_t estr[3] = {1, 1, 1};
  CUtensorMap map;
  CUresult r = encode(&map, g->dtype == PKV_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                      3, pool, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                      CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) {
    pkv_set_error("cuTensorMapEncodeTiled failed with CUresult " + std::to_string((int)r));
    return false;
  }
  if (cache.size() > 64) cache.clear();
  cache.emplace(key, map);
  *out = map;
  return true;
}

int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

struct WsLayout {
  int64_t counters, ml, o, total;
};

WsLayout ws_layout(int32_t batch, int32_t hkv, int32_t head_dim, int64_t splits) {
  WsLayout w;
  w.counters = 256;
  w.ml = w.counters + align256((int64_t)batch * hkv * 4);
  w.o = w.ml + align256(splits * hkv * 16 * 4);
  w.total = w.o + align256(splits * hkv * 8 * head_dim * 4);
  return w;
}

template <int D, typename T>
int32_t launch_decode(const CUtensorMap& map, const DecodeParams& prm, int64_t total_splits, cudaStream_t s) {
  using G = Geo<D>;
  static bool attr_set = false;
  if (!attr_set) {
    cudaFuncSetAttribute(paged_decode_kernel<D, T>, cudaFuncAttributeMaxDynamicSharedMemorySize, G::kSmemBytes);
    attr_set = true;
  }
  dim3 grid((unsigned)total_splits, (unsigned)prm.hkv);
  paged_decode_kernel<D, T><<<grid, kWarps * 32, G::kSmemBytes, s>>>(map, prm);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    pkv_set_error(std::string("pkv_decode_attention launch: ") + cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" {

int64_t pkv_decode_workspace_bytes(int32_t batch, int32_t num_kv_heads, int32_t head_dim, int64_t max_splits_total) {
  return ws_layout(batch, num_kv_heads, head_dim, max_splits_total).total;
}

int32_t pkv_decode_attention(const pkv_pool_geom* g, void* pool, int32_t layer, const void* q, const void* k_new,
                             const void* v_new, int32_t* block_tables, int32_t table_stride, int32_t* context_lens,
                             const int32_t* rows, const int32_t* seq_lens, const int32_t* new_blocks,
                             const int32_t* split_offsets, int32_t batch, int32_t num_q_heads,
                             int32_t pages_per_split, int64_t total_splits, float scale, void* out,
                             void* workspace, int64_t workspace_bytes, void* stream) {
  pkv_clear_error();
  if (!g || g->block_size != 16) {
    pkv_set_error("paged decode attention needs block_size 16");
    return PKV_ERR_UNSUPPORTED;
  }
  if (g->dtype != PKV_BF16 && g->dtype != PKV_F16) {
    pkv_set_error("paged decode attention supports bf16 and f16 pools");
    return PKV_ERR_UNSUPPORTED;
  }
  if (g->head_dim != 64 && g->head_dim != 128) {
    pkv_set_error("paged decode attention supports head_dim 64 and 128");
    return PKV_ERR_UNSUPPORTED;
  }
  if (num_q_heads <= 0 || num_q_heads % g->num_kv_heads != 0 || num_q_heads / g->num_kv_heads > 8) {
    pkv_set_error("num_q_heads must be a multiple of num_kv_heads with at most 8 query heads per KV head");
    return PKV_ERR_UNSUPPORTED;
  }
  if (layer < 0 || layer >= g->num_layers || batch <= 0 || pages_per_split <= 0 || total_splits < batch ||
      total_splits > INT32_MAX) {
    pkv_set_error("invalid layer, batch or split arguments");
    return PKV_ERR_ARG;
  }
  if (!pool || !q || !out || !block_tables || !rows || !seq_lens || !split_offsets || !workspace ||
      (k_new != nullptr) != (v_new != nullptr) || (k_new && !context_lens)) {
    pkv_set_error("null pointer argument");
    return PKV_ERR_ARG;
  }
  if ((uintptr_t)pool % 16 != 0 || (uintptr_t)q % 16 != 0 || (uintptr_t)out % 16 != 0 ||
      (k_new && ((uintptr_t)k_new % 16 || (uintptr_t)v_new % 16))) {
    pkv_set_error("pool, q, out, k_new and v_new must be 16-byte aligned");
    return PKV_ERR_ARG;
  }
  if ((int64_t)g->num_blocks * 2 * g->num_kv_heads * 16 >= INT32_MAX) {
    pkv_set_error("pool too large for 32-bit TMA row coordinates");
    return PKV_ERR_UNSUPPORTED;
  }
  const WsLayout wl = ws_layout(batch, g->num_kv_heads, g->head_dim, total_splits);
  if (workspace_bytes < wl.total) {
    pkv_set_error("workspace too small: need " + std::to_string(wl.total) + " bytes");
    return PKV_ERR_ARG;
  }
  CUtensorMap map;
  if (!make_pool_map(g, pool, &map)) return PKV_ERR_CUDA;

  DecodeParams prm;
  prm.q = q;
  prm.k_new = k_new;
  prm.v_new = v_new;
  prm.out = out;
  prm.pool = pool;
  prm.tables = block_tables;
  prm.ctx_lens = context_lens;
  prm.rows = rows;
  prm.seq_lens = seq_lens;
  prm.new_blocks = new_blocks;
  prm.split_offsets = split_offsets;
  char* ws = static_cast<char*>(workspace);
  prm.ws_error = reinterpret_cast<int32_t*>(ws);
  prm.ws_counters = reinterpret_cast<int32_t*>(ws + wl.counters);
  prm.ws_ml = reinterpret_cast<float*>(ws + wl.ml);
  prm.ws_o = reinterpret_cast<float*>(ws + wl.o);
  prm.table_stride = table_stride;
  prm.batch = batch;
  prm.hq = num_q_heads;
  prm.hkv = g->num_kv_heads;
  prm.group = num_q_heads / g->num_kv_heads;
  prm.layer = layer;
  prm.num_blocks = g->num_blocks;
  prm.pages_per_split = pages_per_split;
  prm.scale_log2 = scale * kLog2e;
  auto s = static_cast<cudaStream_t>(stream);
  if (g->head_dim == 128) {
    return g->dtype == PKV_BF16 ? launch_decode<128, __nv_bfloat16>(map, prm, total_splits, s)
                                : launch_decode<128, __half>(map, prm, total_splits, s);
  }
  return g->dtype == PKV_BF16 ? launch_decode<64, __nv_bfloat16>(map, prm, total_splits, s)
                              : launch_decode<64, __half>(map, prm, total_splits, s);
}

}  // extern "C"
