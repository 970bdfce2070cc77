// Paged GQA decode attention for sm_100a, fused with the step's K/V append.
//
// Replaces, for one decode step of one layer, what AgentRL's continuous loop
// does through HF (agentrl/generation/continuous.py:476-483): the torch.cat
// append into each resident cache (transformers cache_utils.py:119-120) and
// sdpa_attention_forward with GQA (integrations/sdpa_attention.py:40-62).
//
// Work: pkv_decode_plan (host) cuts every sequence's pages into work items of
// at most `pages_per_split` (<= 32) pages for a group of HPC KV heads (HPC = 2
// when the KV head count is even, else 1), largest items first.  A persistent
// grid (one CTA per SM) runs independent warps; each warp takes the next item
// from an atomic counter (dynamic, largest-first scheduling) and owns it
// entirely, so no barrier ever couples warps.
//
// Per warp: a private ring of kStages shared-memory stages (5 warps x 2
// stages of 16 KB at D = 128 with two KV heads per item; 8 warps x 3 stages
// of 8 KB otherwise: PKV_DECODE_* in pkv_internal.h).  One stage holds
// one block's K and V pages of the item's HPC heads -- adjacent in the pool
// and stored pre-swizzled (pkv_device.cuh) -- filled by one cp.async.bulk
// (no tensor map, no multicast) whose completion is counted on the stage's
// mbarrier.  The warp keeps kStages copies in flight, and the stream runs on
// across item boundaries: the next item's descriptor and block ids are
// prefetched while the current item computes.  Per page and KV head the warp
// computes S^T[16 tokens x 8 query heads] = K Q^T and O^T[D x 8] += V^T P^T
// with mma.sync m16n8k16 (ldmatrix / ldmatrix.trans fragments straight from
// the swizzled stage, P^T by movmatrix.trans) and keeps an online softmax per
// query head with warp shuffles (Milakov & Gimelshein 2018); all G = Hq/Hkv
// query heads of a KV head are served from one read of its pages.
//
// Item epilogue: a sequence with one item writes its output from registers;
// otherwise the item writes its unnormalised (O, m, l) partial to the
// workspace (plain stores, no fence) and a second, fully parallel kernel --
// a programmatic dependent of the decode grid -- combines the partials of each
// such (sequence, head group).  Combining inside the decode kernel (the last
// item of a sequence, by atomic ticket) put one warp on a chain of L2 round
// trips while HBM was saturated and cost ~45% more time.
//
// Every mbarrier wait is bounded; on a timeout the warp records an error word
// in the workspace, waits (bounded) for its copies in flight and exits.
//
// Arithmetic: fp32 scores and accumulation, P rounded to the input dtype for
// the P.V product, output rounded once to the input dtype.
#include "pkv_device.cuh"
#include "pkv_error.h"
#include "pkv_internal.h"

#include <algorithm>
#include <atomic>
#include <mutex>
#include <string>
#include <vector>

namespace pkv {
namespace {

constexpr int kMaxSplitsPerSeq = 64;
constexpr int kMaxPagesPerItem = 32;
constexpr float kLog2e = 1.4426950408889634f;

template <int D, int HPC>
struct Cfg {
  static constexpr int kPageBytes = 16 * D * 2;         // one K (or V) page of one head
  static constexpr int kHeadBytes = 2 * kPageBytes;     // K + V of one head in one block
  static constexpr int kStageBytes = HPC * kHeadBytes;  // one ring stage = one block, HPC heads
  static constexpr int kWarps = kStageBytes >= 16384 ? PKV_DECODE_WARPS_BIG : 8;
  static constexpr int kStages = PKV_DECODE_RING_BYTES / (kWarps * kStageBytes) > 8
                                     ? 8
                                     : PKV_DECODE_RING_BYTES / (kWarps * kStageBytes);
  static constexpr int kSmemBytes = kWarps * kStages * kStageBytes + 1024;
  static constexpr int kVecsPerRow = D * 2 / 16;        // 16-byte chunks per token row
};

// Work item as laid out by pkv_decode_plan: {sequence, split << 8 | head_group,
// nsplits, workspace slot of split 0}.  The splits of one (sequence, head
// group) own consecutive workspace slots.
struct DecodeParams {
  const void* q;
  const void* k_new;
  const void* v_new;
  void* out;
  char* pool;
  int32_t* tables;
  int32_t* ctx_lens;
  const int32_t* rows;
  const int32_t* seq_lens;
  const int32_t* new_blocks;
  const int4* items;
  float* ws_ml;
  float* ws_o;
  int32_t* ws_sched;     // [0] next item, [1] warps done
  // Length / refcount updates the decode does not read, applied on the way
  // (the stepper defers them here instead of launching a table kernel):
  // n_ref (block, refcount) pairs then n_len (row, length) pairs.
  const int32_t* deferred;
  int32_t deferred_refs;
  int32_t deferred_lens;
  int32_t* refcounts;
  int32_t* ws_error;
  // Fixed-step mode (a launch recorded once in a CUDA graph and replayed for
  // every step): when set, n_items, n_combine, batch, pages_per_split and the
  // deferred-update counts are read from here at run time:
  // {n_items, n_combine, batch, pages_per_split, deferred_refs, deferred_lens}.
  const int32_t* step_header;
  int32_t n_combine;
  int32_t n_items;
  int32_t batch;
  int32_t table_stride;
  int32_t table_rows;
  int32_t hq;
  int32_t hkv;
  int32_t group;
  int32_t layer;
  int32_t num_blocks;
  int32_t pages_per_split;
  float scale_log2;
};

// A work item must name a sequence of the batch whose table row exists, a
// head group of the pool, a split inside the sequence's pages and a workspace
// slot inside the item list.
template <int HPC>
__device__ __forceinline__ bool item_ok(const int4 item, const DecodeParams& p) {
  const int b = item.x, split = item.y >> 8, hg = item.y & 0xff;
  if (b < 0 || b >= p.batch || (hg + 1) * HPC > p.hkv || item.z < 1 || item.z > kMaxSplitsPerSeq) return false;
  if (split < 0 || split >= item.z || item.w < 0 || item.w + item.z > p.n_items) return false;
  const int row = __ldg(p.rows + b);
  const int len = __ldg(p.seq_lens + b);
  return row >= 0 && row < p.table_rows && len > 0 && (len + 15) / 16 <= p.table_stride &&
         split * p.pages_per_split < (len + 15) / 16;
}

// A block id from the table or the step descriptor must lie in the pool; a bad
// one is replaced by block 0 (and reported) so that no copy leaves the pool.
__device__ __forceinline__ int checked_block(int blk, const DecodeParams& p) {
  if (blk >= 0 && blk < p.num_blocks) return blk;
  atomicExch(p.ws_error, kDevBadBlock);
  return 0;
}

// Everything a warp needs about one item, in registers (warp-uniform except blk).
struct Item {
  int idx;  // -1: none
  int b, split, hg, nsplits, slot0, len, npages, pg0, pg1, row, newb;
  int blk;  // this lane's block: page pg0 + lane
};

// Take the next item.  A warp's first item is its global warp index (no
// atomic round trip before its first copy); later ones come from the
// launch's counter, past the first items.  Each warp draws until it gets an
// out-of-range index, once; the warp that does so last resets the counters
// for the next launch (by then no warp of this launch draws again).
__device__ __forceinline__ int fetch_item(const DecodeParams& p, int lane, int gwarp, int total_warps, bool first) {
  int idx = 0;
  if (lane == 0) {
    idx = first ? gwarp : total_warps + atomicAdd(p.ws_sched, 1);
    if (idx >= p.n_items) {
      const int done = atomicAdd(p.ws_sched + 1, 1);
      if (done == total_warps - 1) {
        atomicExch(p.ws_sched, 0);
        atomicExch(p.ws_sched + 1, 0);
      }
    }
  }
  idx = __shfl_sync(0xffffffffu, idx, 0);
  return idx < p.n_items ? idx : -1;
}

template <int HPC>
__device__ __forceinline__ Item next_item(const DecodeParams& p, int lane, int gwarp, int total_warps, bool first) {
  Item m;
  for (;;) {
    m.idx = fetch_item(p, lane, gwarp, total_warps, first);
    first = false;
    if (m.idx < 0) return m;
    const int4 it = p.items[m.idx];
    if (item_ok<HPC>(it, p)) {
      m.b = it.x;
      m.split = it.y >> 8;
      m.hg = it.y & 0xff;
      m.nsplits = it.z;
      m.slot0 = it.w;
      break;
    }
    if (lane == 0) atomicExch(p.ws_error, kDevBadItem);
  }
  m.len = __ldg(p.seq_lens + m.b);
  m.row = __ldg(p.rows + m.b);
  m.newb = p.new_blocks ? __ldg(p.new_blocks + m.b) : -1;
  m.npages = (m.len + 15) >> 4;
  m.pg0 = m.split * p.pages_per_split;
  m.pg1 = min(m.pg0 + p.pages_per_split, m.npages);
  const int pg = m.pg0 + lane;
  m.blk = 0;
  if (pg < m.pg1)
    m.blk = checked_block((pg == m.npages - 1 && m.newb >= 0) ? m.newb
                                                              : p.tables[(int64_t)m.row * p.table_stride + pg],
                          p);
  return m;
}

// The launch's per-step values: from the parameters, or from the step header.
__device__ __forceinline__ DecodeParams step_params(const DecodeParams& in) {
  DecodeParams p = in;
  if (in.step_header) {
    const int32_t* h = in.step_header;
    p.n_items = h[0];
    p.n_combine = h[1];
    p.batch = h[2];
    p.pages_per_split = h[3];
    p.deferred_refs = h[4];
    p.deferred_lens = h[5];
  }
  return p;
}

template <int D, int HPC, typename T>
__global__ void __launch_bounds__(Cfg<D, HPC>::kWarps * 32, 1) paged_decode_kernel(const DecodeParams launch_p) {
  const DecodeParams p = step_params(launch_p);
  using C = Cfg<D, HPC>;
  constexpr int KK = D / 16;
  constexpr int S = C::kStages;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bars[C::kWarps * S];

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int total_warps = gridDim.x * C::kWarps;
  const int gwarp = blockIdx.x * C::kWarps + warp;
  uint8_t* ring = smem + warp * S * C::kStageBytes;
  uint64_t* full = bars + warp * S;
  if (lane == 0) {
    for (int i = 0; i < S; ++i) mbar_init(&full[i], 1);
    fence_barrier_init();
  }
  __syncwarp();

  // Launched as a programmatic dependent of the previous step's kernels
  // (PKV_DECODE_PDL), this CTA got resident and set up its barriers while
  // they ran; wait for them here, before the first global access.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // Let the split-K combine grid get resident now; it waits in hardware for
  // this grid to complete before it reads the partials.
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");

  if (p.deferred) {
    const int n = p.deferred_refs + p.deferred_lens;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
      const int32_t a = p.deferred[2 * i], v = p.deferred[2 * i + 1];
      if (i < p.deferred_refs) {
        if (a >= 0 && a < p.num_blocks) p.refcounts[a] = v;
      } else if (a >= 0 && a < p.table_rows) {
        p.ctx_lens[a] = v;
      }
    }
  }

  const T* kn = static_cast<const T*>(p.k_new);
  const T* vn = static_cast<const T*>(p.v_new);
  T* out = static_cast<T*>(p.out);
  const int group = p.group;
  const char* layer_base = p.pool + (int64_t)p.layer * p.num_blocks * p.hkv * C::kHeadBytes;

  Item cur = next_item<HPC>(p, lane, gwarp, total_warps, true);
  Item nxt;
  nxt.idx = -1;
  if (cur.idx >= 0) nxt = next_item<HPC>(p, lane, gwarp, total_warps, false);
  int issued = 0, consumed = 0;
  bool iss_next = false;
  int iss_pg = cur.pg0;
  // Pages are read once per step: evict them first, so the split partials
  // this kernel writes are still in L2 when the combine kernel reads them.
  const uint64_t kv_policy = l2_evict_first_policy();

  // Keep kStages copies in flight along the stream cur -> nxt.
  auto issue_ahead = [&]() {
    while (issued - consumed < S) {
      const Item& m = iss_next ? nxt : cur;
      if (m.idx < 0) break;
      if (iss_pg >= m.pg1) {
        if (iss_next) break;
        iss_next = true;
        iss_pg = nxt.pg0;
        continue;
      }
      const int blk = __shfl_sync(0xffffffffu, m.blk, iss_pg - m.pg0);
      if (lane == 0) {
        const int st = issued % S;
        mbar_arrive_expect_tx(&full[st], C::kStageBytes);
        bulk_copy_g2s_hint(ring + st * C::kStageBytes,
                           layer_base + ((int64_t)blk * p.hkv + m.hg * HPC) * C::kHeadBytes, C::kStageBytes,
                           &full[st], kv_policy);
      }
      ++issued;
      ++iss_pg;
    }
  };

  while (cur.idx >= 0) {
    // Q^T fragments (B operand, col layout): query head lane/4, dims 2*(lane%4)+{0,1} (+8).
    uint32_t qf[HPC][KK][2];
#pragma unroll
    for (int hh = 0; hh < HPC; ++hh) {
      const int gq = lane >> 2;
      const bool in = gq < group;
      const T* qrow =
          static_cast<const T*>(p.q) + ((int64_t)cur.b * p.hq + (cur.hg * HPC + hh) * group + (in ? gq : 0)) * D;
#pragma unroll
      for (int kk = 0; kk < KK; ++kk) {
        qf[hh][kk][0] = in ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 2 * (lane & 3)) : 0u;
        qf[hh][kk][1] = in ? *reinterpret_cast<const uint32_t*>(qrow + kk * 16 + 8 + 2 * (lane & 3)) : 0u;
      }
    }
    float m_a[HPC], m_b[HPC], l_a[HPC], l_b[HPC];
    float oacc[HPC][KK][4];
#pragma unroll
    for (int hh = 0; hh < HPC; ++hh) {
      m_a[hh] = m_b[hh] = -INFINITY;
      l_a[hh] = l_b[hh] = 0.f;
#pragma unroll
      for (int mt = 0; mt < KK; ++mt) oacc[hh][mt][0] = oacc[hh][mt][1] = oacc[hh][mt][2] = oacc[hh][mt][3] = 0.f;
    }

    for (int pg = cur.pg0; pg < cur.pg1; ++pg) {
      issue_ahead();
      const int st = consumed % S;
      const bool ok = mbar_wait_bounded(&full[st], (consumed / S) & 1);
      if (!__all_sync(0xffffffffu, ok)) {
        // Record the failure, wait (bounded) for the copies still in flight, leave.
        if (lane == 0) {
          atomicExch(p.ws_error, kDevWaitTimeout);
          for (int k = consumed + 1; k < issued; ++k) mbar_wait_bounded(&full[k % S], (k / S) & 1);
        }
        __syncwarp();
        return;
      }
      uint8_t* stage = ring + st * C::kStageBytes;
      const int valid = min(16, cur.len - pg * 16);

      if (pg == cur.npages - 1) {
        // The step's token: write it to its slot in the pool (for later steps)
        // and patch it into the stage (the copy may predate that write); then
        // zero V rows past the context so masked probabilities multiply finite
        // values.
        const int slot = valid - 1;
#pragma unroll
        for (int hh = 0; hh < HPC; ++hh) {
          if (kn != nullptr && lane < 2 * C::kVecsPerRow) {
            const int state = lane / C::kVecsPerRow, vec = lane % C::kVecsPerRow;
            const int h = cur.hg * HPC + hh;
            const uint4 val =
                reinterpret_cast<const uint4*>((state == 0 ? kn : vn) + ((int64_t)cur.b * p.hkv + h) * D)[vec];
            const int64_t inpage = row_byte_offset(slot, vec * 16, 16, D * 2, true);
            *reinterpret_cast<uint4*>(stage + hh * C::kHeadBytes + state * C::kPageBytes + inpage) = val;
            const int blk = checked_block(
                cur.newb >= 0 ? cur.newb : p.tables[(int64_t)cur.row * p.table_stride + pg], p);
            *reinterpret_cast<uint4*>(p.pool + page_offset(p.layer, blk, h, state, p.num_blocks, p.hkv, 16, D * 2) +
                                      inpage) = val;
          }
          for (int c = lane; c < (16 - valid) * C::kVecsPerRow; c += 32) {
            const int r = valid + c / C::kVecsPerRow, vec = c % C::kVecsPerRow;
            *reinterpret_cast<uint4*>(stage + hh * C::kHeadBytes + C::kPageBytes +
                                      row_byte_offset(r, vec * 16, 16, D * 2, true)) = make_uint4(0u, 0u, 0u, 0u);
          }
        }
        if (kn != nullptr && cur.hg == 0 && lane == 0) {
          if (cur.newb >= 0) p.tables[(int64_t)cur.row * p.table_stride + pg] = cur.newb;
          p.ctx_lens[cur.row] = cur.len;
        }
        __syncwarp();
      }

      const bool va = (lane >> 2) < valid;
      const bool vb = (lane >> 2) + 8 < valid;
#pragma unroll
      for (int hh = 0; hh < HPC; ++hh) {
        const uint32_t sk = smem_u32(stage + hh * C::kHeadBytes);
        const uint32_t sv = sk + C::kPageBytes;
        // S^T = K Q^T  (M = 16 tokens, N = 8 query heads, K = D), two accumulator chains.
        float s0[4] = {0.f, 0.f, 0.f, 0.f}, s1[4] = {0.f, 0.f, 0.f, 0.f};
        {
          const int tok = (lane & 7) + 8 * ((lane >> 3) & 1);
#pragma unroll
          for (int kk = 0; kk < KK; ++kk) {
            const int dim = kk * 16 + 8 * (lane >> 4);
            uint32_t a[4];
            ldmatrix_x4(sk + (dim >> 6) * 2048 + swz128(tok, (dim & 63) >> 3), a[0], a[1], a[2], a[3]);
            MmaOp<T>::run((kk & 1) ? s1 : s0, a, qf[hh][kk]);
          }
        }
        const float x0 = va ? (s0[0] + s1[0]) * p.scale_log2 : -INFINITY;
        const float x1 = va ? (s0[1] + s1[1]) * p.scale_log2 : -INFINITY;
        const float x2 = vb ? (s0[2] + s1[2]) * p.scale_log2 : -INFINITY;
        const float x3 = vb ? (s0[3] + s1[3]) * p.scale_log2 : -INFINITY;
        float mx_a = fmaxf(x0, x2), mx_b = fmaxf(x1, x3);
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          mx_a = fmaxf(mx_a, __shfl_xor_sync(0xffffffffu, mx_a, off));
          mx_b = fmaxf(mx_b, __shfl_xor_sync(0xffffffffu, mx_b, off));
        }
        const float mn_a = fmaxf(m_a[hh], mx_a), mn_b = fmaxf(m_b[hh], mx_b);
        const float al_a = exp2f(m_a[hh] - mn_a), al_b = exp2f(m_b[hh] - mn_b);
        const float p0 = exp2f(x0 - mn_a), p1 = exp2f(x1 - mn_b);
        const float p2 = exp2f(x2 - mn_a), p3 = exp2f(x3 - mn_b);
        l_a[hh] = l_a[hh] * al_a + p0 + p2;
        l_b[hh] = l_b[hh] * al_b + p1 + p3;
        m_a[hh] = mn_a;
        m_b[hh] = mn_b;
        uint32_t pb[2];
        pb[0] = movmatrix_trans(MmaOp<T>::pack(p0, p1));
        pb[1] = movmatrix_trans(MmaOp<T>::pack(p2, p3));
        // O^T += V^T P^T  (M = D dims in tiles of 16, N = 8 query heads, K = 16 tokens)
        const int tok = (lane & 7) + 8 * (lane >> 4);
#pragma unroll
        for (int mt = 0; mt < KK; ++mt) {
          oacc[hh][mt][0] *= al_a;
          oacc[hh][mt][1] *= al_b;
          oacc[hh][mt][2] *= al_a;
          oacc[hh][mt][3] *= al_b;
          const int dim = mt * 16 + 8 * ((lane >> 3) & 1);
          uint32_t a[4];
          ldmatrix_x4_trans(sv + (dim >> 6) * 2048 + swz128(tok, (dim & 63) >> 3), a[0], a[1], a[2], a[3]);
          MmaOp<T>::run(oacc[hh][mt], a, pb);
        }
      }
      // The stage is read; order those reads before the next bulk copy into it.
      __syncwarp();
      fence_proxy_async_smem();
      ++consumed;
    }

    // ---- item epilogue ----
    const int ha = 2 * (lane & 3), hb = ha + 1;
    if (cur.nsplits == 1) {
#pragma unroll
      for (int hh = 0; hh < HPC; ++hh) {
        float la = l_a[hh], lb = l_b[hh];
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          la += __shfl_xor_sync(0xffffffffu, la, off);
          lb += __shfl_xor_sync(0xffffffffu, lb, off);
        }
        const float ia = 1.f / la, ib = 1.f / lb;
        T* oa = out + ((int64_t)cur.b * p.hq + (cur.hg * HPC + hh) * group + ha) * D;
        T* ob = oa + D;
#pragma unroll
        for (int mt = 0; mt < KK; ++mt) {
          const int d0 = mt * 16 + (lane >> 2);
          if (ha < group) {
            oa[d0] = MmaOp<T>::from_float(oacc[hh][mt][0] * ia);
            oa[d0 + 8] = MmaOp<T>::from_float(oacc[hh][mt][2] * ia);
          }
          if (hb < group) {
            ob[d0] = MmaOp<T>::from_float(oacc[hh][mt][1] * ib);
            ob[d0 + 8] = MmaOp<T>::from_float(oacc[hh][mt][3] * ib);
          }
        }
      }
    } else {
      const int64_t slot = (int64_t)cur.slot0 + cur.split;
#pragma unroll
      for (int hh = 0; hh < HPC; ++hh) {
        float la = l_a[hh], lb = l_b[hh];
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) {
          la += __shfl_xor_sync(0xffffffffu, la, off);
          lb += __shfl_xor_sync(0xffffffffu, lb, off);
        }
        float* wo = p.ws_o + (slot * HPC + hh) * 8 * D;
#pragma unroll
        for (int mt = 0; mt < KK; ++mt) {
          const int d0 = mt * 16 + (lane >> 2);
          wo[ha * D + d0] = oacc[hh][mt][0];
          wo[hb * D + d0] = oacc[hh][mt][1];
          wo[ha * D + d0 + 8] = oacc[hh][mt][2];
          wo[hb * D + d0 + 8] = oacc[hh][mt][3];
        }
        if (lane < 4) {
          float* ml = p.ws_ml + (slot * HPC + hh) * 16;
          ml[ha] = m_a[hh];
          ml[hb] = m_b[hh];
          ml[8 + ha] = la;
          ml[8 + hb] = lb;
        }
      }
    }

    // ---- advance the stream ----
    cur = nxt;
    if (iss_next) {
      iss_next = false;
    } else {
      iss_pg = cur.pg0;
    }
    nxt.idx = -1;
    if (cur.idx >= 0) nxt = next_item<HPC>(p, lane, gwarp, total_warps, false);
  }
}

// Split-K combine: entries {sequence, head_group, nsplits, workspace slot of
// split 0} follow the decode items in the plan; grid = (entry, query head of
// the group), one warp each.  out = sum_s w_s O_s / sum_s w_s l_s with
// w_s = 2^(m_s - max_s m_s).  Lane s (and s + 32) reads split s's max and sum,
// warp shuffles give the weights, then lane i loads dims 4i..4i+3 of every
// split at once: about two memory round trips per warp.  Launched as a
// programmatic dependent of the decode grid: its CTAs become resident early
// and griddepcontrol.wait holds them (in hardware, no spinning) until the
// decode grid has completed and its partials are visible.
constexpr int kCombineThreads = 32;

template <int D, int HPC>
__device__ __forceinline__ bool entry_ok(const DecodeParams& p, const int4 en) {
  const int b = en.x, hg = en.y, ns = en.z, slot0 = en.w;
  return b >= 0 && b < p.batch && (hg + 1) * HPC <= p.hkv && ns >= 2 && ns <= kMaxSplitsPerSeq && slot0 >= 0 &&
         slot0 + ns <= p.n_items;
}

// Merge one (entry, query head); the entry has been checked.
template <int D, int HPC, typename T>
__device__ __forceinline__ void combine_one(const DecodeParams& p, const int4 en, int hh, int gq) {
  const int b = en.x, hg = en.y, ns = en.z, slot0 = en.w;
  const int lane = threadIdx.x;
  float m0 = -INFINITY, l0 = 0.f, m1 = -INFINITY, l1 = 0.f;
  if (lane < ns) {
    const float* ml = p.ws_ml + ((int64_t)(slot0 + lane) * HPC + hh) * 16;
    m0 = ml[gq];
    l0 = ml[8 + gq];
  }
  if (lane + 32 < ns) {
    const float* ml = p.ws_ml + ((int64_t)(slot0 + lane + 32) * HPC + hh) * 16;
    m1 = ml[gq];
    l1 = ml[8 + gq];
  }
  float mm = fmaxf(m0, m1);
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) mm = fmaxf(mm, __shfl_xor_sync(0xffffffffu, mm, off));
  const float w0 = lane < ns ? exp2f(m0 - mm) : 0.f;
  const float w1 = lane + 32 < ns ? exp2f(m1 - mm) : 0.f;
  float l = w0 * l0 + w1 * l1;
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) l += __shfl_xor_sync(0xffffffffu, l, off);
  const float inv = 1.f / l;
  constexpr int kQuads = D / 4;
  const bool active = lane < kQuads;
  const float4* src = reinterpret_cast<const float4*>(p.ws_o + (((int64_t)slot0 * HPC + hh) * 8 + gq) * D) + lane;
  const int64_t stride = (int64_t)HPC * 8 * D / 4;  // float4s from one split to the next
  float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
  constexpr int kBatch = PKV_COMBINE_BATCH;  // splits loaded per round
  for (int s0 = 0; s0 < ns; s0 += kBatch) {
    float4 x[kBatch];
#pragma unroll
    for (int k = 0; k < kBatch; ++k)
      x[k] = (active && s0 + k < ns) ? src[(s0 + k) * stride] : make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
    for (int k = 0; k < kBatch; ++k) {
      const int sidx = s0 + k;
      const float w = __shfl_sync(0xffffffffu, sidx < 32 ? w0 : w1, sidx & 31);
      if (sidx < ns) {
        acc.x += w * x[k].x;
        acc.y += w * x[k].y;
        acc.z += w * x[k].z;
        acc.w += w * x[k].w;
      }
    }
  }
  if (!active) return;
  T* dst = static_cast<T*>(p.out) + ((int64_t)b * p.hq + (hg * HPC + hh) * p.group + gq) * D + 4 * lane;
  dst[0] = MmaOp<T>::from_float(acc.x * inv);
  dst[1] = MmaOp<T>::from_float(acc.y * inv);
  dst[2] = MmaOp<T>::from_float(acc.z * inv);
  dst[3] = MmaOp<T>::from_float(acc.w * inv);
}

template <int D, int HPC, typename T>
__global__ void __launch_bounds__(kCombineThreads) paged_decode_combine_kernel(const DecodeParams launch_p,
                                                                               const int4* entries) {
  // The step header and the entries come from the step's descriptor, which
  // was in place before the decode grid started: read them while that grid
  // still runs, then wait for its partials.
  const DecodeParams p = step_params(launch_p);
  const int pi = blockIdx.y;
  // blockIdx.y = head of the item's KV-head group x query head of its group
  const int hh = pi / launch_p.group, gq = pi % launch_p.group;
  const int e0 = blockIdx.x;
  const bool live = gq < p.group && e0 < p.n_combine;
  int4 en = make_int4(0, 0, 0, 0);
  bool ok = false;
  if (live) {
    en = entries[e0];
    ok = entry_ok<D, HPC>(p, en);
  }
  asm volatile("griddepcontrol.wait;" ::: "memory");
  // The next step's decode grid may get resident now (it waits in hardware
  // for this grid before its first global access).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  if (gq >= p.group) return;
  if (live && !ok && threadIdx.x == 0) atomicExch(p.ws_error, kDevBadItem);
  if (ok) combine_one<D, HPC, T>(p, en, hh, gq);
  // One (entry, query head) per block; a fixed-step launch has a fixed grid
  // and strides over however many entries the step has.
  for (int e = e0 + gridDim.x; e < p.n_combine; e += gridDim.x) {
    const int4 x = entries[e];
    if (entry_ok<D, HPC>(p, x)) {
      combine_one<D, HPC, T>(p, x, hh, gq);
    } else if (threadIdx.x == 0) {
      atomicExch(p.ws_error, kDevBadItem);
    }
  }
}

// ---------------------------------------------------------------------------
// Host side.

int num_sms_cached() {
  static int sms = 0;
  if (!sms) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    if (sms <= 0) sms = 148;
  }
  return sms;
}

int heads_per_item(int num_kv_heads) { return num_kv_heads % 2 == 0 ? 2 : 1; }

int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

int warps_per_cta(int head_dim, int hpc) {
  const int stage = hpc * 2 * 16 * head_dim * 2;
  return stage >= 16384 ? PKV_DECODE_WARPS_BIG : 8;
}

struct WsLayout {
  int64_t sched, ml, o, total;
};

// Workspace: [error word][scheduler counters][partial m, l][partial O].
WsLayout ws_layout(int32_t batch, int32_t hkv, int32_t head_dim, int64_t n_items) {
  (void)batch;
  const int hpc = heads_per_item(hkv);
  WsLayout w;
  w.sched = 64;
  w.ml = 256;
  w.o = w.ml + align256(n_items * hpc * 16 * 4);
  w.total = w.o + align256(n_items * hpc * 8 * head_dim * 4);
  return w;
}

// cudaFuncSetAttribute once per device (the attribute is per device).
constexpr int kAttrDevices = 64;

template <typename Fn>
int32_t ensure_smem_attr(Fn* fn, int bytes, std::atomic<bool>* done) {
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kAttrDevices) dev = -1;
  if (dev >= 0 && done[dev].load(std::memory_order_acquire)) return PKV_OK;
  cudaError_t e = cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) {
    pkv_set_error(std::string("pkv_decode_attention: cudaFuncSetAttribute: ") + cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  if (dev >= 0) done[dev].store(true, std::memory_order_release);
  return PKV_OK;
}

template <int D, int HPC, typename T>
int32_t launch_decode(const DecodeParams& prm, const int4* entries, cudaStream_t s) {
  using C = Cfg<D, HPC>;
  static std::atomic<bool> attr_done[kAttrDevices];
  if (int32_t st = ensure_smem_attr(paged_decode_kernel<D, HPC, T>, C::kSmemBytes, attr_done)) return st;
#if PKV_CARVEOUT_MAX
  {
    // Both kernels of a step prefer the largest shared-memory carveout, so an
    // SM that runs the combine between two decode grids keeps its split.
    static std::atomic<bool> carve_done[kAttrDevices];
    int dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess && dev >= 0 && dev < kAttrDevices && !carve_done[dev].load()) {
      cudaFuncSetAttribute(paged_decode_kernel<D, HPC, T>, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
      cudaFuncSetAttribute(paged_decode_combine_kernel<D, HPC, T>, cudaFuncAttributePreferredSharedMemoryCarveout,
                           cudaSharedmemCarveoutMaxShared);
      carve_done[dev].store(true);
    }
  }
#endif
  // A fixed-step launch does not know its item count on the host: it always
  // runs the persistent grid (idle warps fetch an out-of-range item and
  // leave) and the combine kernel.
  const bool fixed = prm.step_header != nullptr;
  const int grid =
      fixed ? num_sms_cached() : std::max(1, std::min((prm.n_items + C::kWarps - 1) / C::kWarps, num_sms_cached()));
#if PKV_DECODE_PDL
  {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((unsigned)grid);
    cfg.blockDim = dim3(C::kWarps * 32);
    cfg.dynamicSmemBytes = C::kSmemBytes;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t le = cudaLaunchKernelEx(&cfg, paged_decode_kernel<D, HPC, T>, prm);
    if (le != cudaSuccess) {
      pkv_set_error(std::string("pkv_decode_attention launch: ") + cudaGetErrorString(le));
      return PKV_ERR_CUDA;
    }
  }
#else
  paged_decode_kernel<D, HPC, T><<<grid, C::kWarps * 32, C::kSmemBytes, s>>>(prm);
#endif
  if (fixed || prm.n_combine > 0) {
    cudaLaunchConfig_t cfg = {};
    // One block per (entry, query head): n_combine is the step's count, or
    // its capacity for a fixed-step launch (whose blocks past the step's
    // count return at once).
    cfg.gridDim = dim3((unsigned)std::max(1, prm.n_combine), HPC * prm.group);
    cfg.blockDim = dim3(kCombineThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t le = cudaLaunchKernelEx(&cfg, paged_decode_combine_kernel<D, HPC, T>, prm, entries);
    if (le != cudaSuccess) {
      pkv_set_error(std::string("pkv_decode_attention combine launch: ") + cudaGetErrorString(le));
      return PKV_ERR_CUDA;
    }
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    pkv_set_error(std::string("pkv_decode_attention launch: ") + cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}

template <int D, typename T>
int32_t launch_for_heads(const DecodeParams& prm, const int4* entries, cudaStream_t s) {
  return heads_per_item(prm.hkv) == 2 ? launch_decode<D, 2, T>(prm, entries, s)
                                      : launch_decode<D, 1, T>(prm, entries, s);
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" {

int32_t pkv_decode_heads_per_item(int32_t num_kv_heads) { return heads_per_item(num_kv_heads); }

int32_t pkv_decode_plan(const int32_t* seq_lens, int32_t batch, int32_t num_kv_heads, int32_t head_dim,
                        int32_t num_sms, int32_t* pages_per_split_out, int32_t* items_out, int64_t items_capacity,
                        int64_t* n_items_out, int64_t* n_combine_out) {
  pkv_clear_error();
  if (batch <= 0 || num_kv_heads <= 0 || !seq_lens || !pages_per_split_out || !n_items_out || !n_combine_out) {
    pkv_set_error("pkv_decode_plan: invalid arguments");
    return PKV_ERR_ARG;
  }
  const int hpc = heads_per_item(num_kv_heads);
  const int groups = num_kv_heads / hpc;
  if (num_sms <= 0) num_sms = 148;
  int64_t total_pages = 0;
  int32_t max_pages = 1;
  for (int b = 0; b < batch; ++b) {
    if (seq_lens[b] <= 0) {
      pkv_set_error("pkv_decode_plan: every sequence needs at least one token (the step's token)");
      return PKV_ERR_ARG;
    }
    const int32_t pages = (seq_lens[b] + 15) / 16;
    total_pages += pages;
    max_pages = std::max(max_pages, pages);
  }
  if (max_pages > kMaxPagesPerItem * kMaxSplitsPerSeq) {
    pkv_set_error("pkv_decode_plan: a sequence exceeds " + std::to_string(16 * kMaxPagesPerItem * kMaxSplitsPerSeq) +
                  " tokens");
    return PKV_ERR_UNSUPPORTED;
  }
  // About PKV_DECODE_ITEMS_PER_WARP (3) items per warp of the persistent grid (dynamic scheduling evens
  // out the rest), 4..32 pages per item, at most kMaxSplitsPerSeq items per
  // sequence and head group.
  const int64_t work = total_pages * groups;
  const int64_t warps = (int64_t)num_sms * warps_per_cta(head_dim, hpc);
  int32_t pps = (int32_t)std::min<int64_t>(kMaxPagesPerItem,
                                           std::max<int64_t>(4, (work + warps * PKV_DECODE_ITEMS_PER_WARP - 1) /
                                                                    (warps * PKV_DECODE_ITEMS_PER_WARP)));
  pps = std::max(pps, (max_pages + kMaxSplitsPerSeq - 1) / kMaxSplitsPerSeq);
  int64_t n = 0, nc = 0;
  for (int b = 0; b < batch; ++b) {
    const int64_t ns = ((seq_lens[b] + 15) / 16 + pps - 1) / pps;
    n += groups * ns;
    if (ns > 1) nc += groups;
  }
  *pages_per_split_out = pps;
  *n_items_out = n;
  *n_combine_out = nc;
  if (!items_out) return PKV_OK;
  if (items_capacity < n + nc) {
    pkv_set_error("pkv_decode_plan: item buffer too small");
    return PKV_ERR_ARG;
  }
  // Sequences ordered by (pages descending, index ascending): a counting
  // sort over the page counts (max_pages buckets) for large batches, a
  // comparison sort of packed keys for small ones.  With PKV_DECODE_ORDER 1
  // the items are then placed by decreasing page count (below), else each
  // sequence's items stay together (head group, then split).
  thread_local std::vector<int32_t> order;
  thread_local std::vector<int32_t> slot_of;
  thread_local std::vector<int32_t> bucket;
  order.resize(batch);
  slot_of.resize(batch);
  {
    int32_t sl = 0;
    for (int b = 0; b < batch; ++b) {
      const int32_t pages = (seq_lens[b] + 15) / 16;
      slot_of[b] = sl;
      sl += groups * ((pages + pps - 1) / pps);
    }
  }
  if (batch >= 64 && max_pages <= 4 * batch + 64) {
    bucket.assign(max_pages + 2, 0);
    for (int b = 0; b < batch; ++b) ++bucket[(seq_lens[b] + 15) / 16];
    // Start of each page count's run, longest first.
    int32_t at = 0;
    for (int32_t pg = max_pages; pg >= 1; --pg) {
      const int32_t n = bucket[pg];
      bucket[pg] = at;
      at += n;
    }
    for (int b = 0; b < batch; ++b) order[bucket[(seq_lens[b] + 15) / 16]++] = b;
  } else {
    thread_local std::vector<int64_t> keys;
    keys.resize(batch);
    for (int b = 0; b < batch; ++b) {
      const int64_t pages = (seq_lens[b] + 15) / 16;
      keys[b] = ((int64_t)(0x7fffffff - pages) << 32) | b;  // ascending key = descending length
    }
    std::sort(keys.begin(), keys.end());
    for (int b = 0; b < batch; ++b) order[b] = (int32_t)(keys[b] & 0xffffffff);
  }
  int32_t* o = items_out;
#if PKV_DECODE_ORDER == 1
  // Items by decreasing page count: every full-size item (pps pages) first,
  // in the sequence order above, then the remainders from the largest to the
  // smallest, so the grid's tail holds the shortest items.  One pass: each
  // item is written straight to its place among the items of its size.
  {
    int64_t start[kMaxPagesPerItem + 2] = {};
    for (int32_t b : order) {
      const int32_t pages = (seq_lens[b] + 15) / 16;
      start[pps] += (int64_t)groups * (pages / pps);
      if (pages % pps) start[pages % pps] += groups;
    }
    int64_t at = 0;
    for (int32_t pg = pps; pg >= 1; --pg) {
      const int64_t c = start[pg];
      start[pg] = at;
      at += c;
    }
    for (int32_t b : order) {
      const int32_t pages = (seq_lens[b] + 15) / 16;
      const int32_t ns = (pages + pps - 1) / pps;
      const int32_t full = pages / pps;
      for (int hg = 0; hg < groups; ++hg) {
        for (int sp = 0; sp < ns; ++sp) {
          int32_t* q = items_out + 4 * start[sp < full ? pps : pages % pps]++;
          q[0] = b;
          q[1] = (sp << 8) | hg;
          q[2] = ns;
          q[3] = slot_of[b] + hg * ns;
        }
      }
    }
    o += 4 * n;
  }
#else
  for (int32_t b : order) {
    const int32_t pages = (seq_lens[b] + 15) / 16;
    const int32_t ns = (pages + pps - 1) / pps;
    for (int hg = 0; hg < groups; ++hg) {
      for (int sp = 0; sp < ns; ++sp) {
        o[0] = b;
        o[1] = (sp << 8) | hg;
        o[2] = ns;
        o[3] = slot_of[b] + hg * ns;
        o += 4;
      }
    }
  }
#endif
  // Combine entries {sequence, head_group, nsplits, slot of split 0}.
  int32_t slot = 0;
  for (int b = 0; b < batch; ++b) {
    const int32_t ns = ((seq_lens[b] + 15) / 16 + pps - 1) / pps;
    for (int hg = 0; hg < groups; ++hg) {
      if (ns > 1) {
        o[0] = b;
        o[1] = hg;
        o[2] = ns;
        o[3] = slot;
        o += 4;
      }
      slot += ns;
    }
  }
  return PKV_OK;
}

int64_t pkv_decode_workspace_bytes(int32_t batch, int32_t num_kv_heads, int32_t head_dim, int64_t n_items) {
  return ws_layout(batch, num_kv_heads, head_dim, n_items).total;
}

int32_t pkv_decode_attention(const pkv_pool_geom* g, void* pool, int32_t layer, const void* q, const void* k_new,
                             const void* v_new, int32_t* block_tables, int32_t table_stride, int32_t table_rows,
                             int32_t* context_lens,
                             const int32_t* rows, const int32_t* seq_lens, const int32_t* new_blocks,
                             const int32_t* work_items, int32_t n_items, int32_t n_combine, int32_t batch,
                             int32_t num_q_heads, int32_t pages_per_split, float scale, void* out, void* workspace,
                             int64_t workspace_bytes, void* stream) {
  return pkv_decode_attention_ex(g, pool, layer, q, k_new, v_new, block_tables, table_stride, table_rows,
                                 context_lens, rows, seq_lens, new_blocks, work_items, n_items, n_combine, batch,
                                 num_q_heads, pages_per_split, scale, out, workspace, workspace_bytes, stream,
                                 nullptr, 0, 0, nullptr, nullptr, nullptr);
}

}  // extern "C"

int32_t pkv_decode_attention_ex(const pkv_pool_geom* g, void* pool, int32_t layer, const void* q, const void* k_new,
                                const void* v_new, int32_t* block_tables, int32_t table_stride, int32_t table_rows,
                                int32_t* context_lens, const int32_t* rows, const int32_t* seq_lens,
                                const int32_t* new_blocks, const int32_t* work_items, int32_t n_items,
                                int32_t n_combine, int32_t batch, int32_t num_q_heads, int32_t pages_per_split,
                                float scale, void* out, void* workspace, int64_t workspace_bytes, void* stream,
                                const int32_t* deferred, int32_t deferred_refs, int32_t deferred_lens,
                                int32_t* refcounts, const int32_t* step_header, const int32_t* combine_entries) {
  pkv_clear_error();
  if (deferred && (!refcounts || !context_lens || deferred_refs < 0 || deferred_lens < 0)) {
    pkv_set_error("deferred updates need the refcount and length arrays");
    return PKV_ERR_ARG;
  }
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
  if (num_q_heads <= 0 || num_q_heads % g->num_kv_heads != 0 || num_q_heads / g->num_kv_heads > 8 ||
      g->num_kv_heads > 255 * 2) {
    pkv_set_error("num_q_heads must be a multiple of num_kv_heads with at most 8 query heads per KV head");
    return PKV_ERR_UNSUPPORTED;
  }
  if (layer < 0 || layer >= g->num_layers || batch <= 0 || pages_per_split <= 0 ||
      pages_per_split > kMaxPagesPerItem || n_items < batch || n_combine < 0 || n_combine > n_items) {
    pkv_set_error("invalid layer, batch, item or split arguments");
    return PKV_ERR_ARG;
  }
  if (!pool || !q || !out || !block_tables || !rows || !seq_lens || !work_items || !workspace ||
      (k_new != nullptr) != (v_new != nullptr) || (k_new && !context_lens)) {
    pkv_set_error("null pointer argument");
    return PKV_ERR_ARG;
  }
  if ((uintptr_t)pool % 16 != 0 || (uintptr_t)q % 16 != 0 || (uintptr_t)out % 16 != 0 ||
      (uintptr_t)work_items % 16 != 0 || (k_new && ((uintptr_t)k_new % 16 || (uintptr_t)v_new % 16))) {
    pkv_set_error("pool, q, out, work_items, k_new and v_new must be 16-byte aligned");
    return PKV_ERR_ARG;
  }
  const WsLayout wl = ws_layout(batch, g->num_kv_heads, g->head_dim, n_items);
  if (workspace_bytes < wl.total) {
    pkv_set_error("workspace too small: need " + std::to_string(wl.total) + " bytes");
    return PKV_ERR_ARG;
  }
  DecodeParams prm;
  prm.q = q;
  prm.k_new = k_new;
  prm.v_new = v_new;
  prm.out = out;
  prm.pool = static_cast<char*>(pool);
  prm.tables = block_tables;
  prm.ctx_lens = context_lens;
  prm.rows = rows;
  prm.seq_lens = seq_lens;
  prm.new_blocks = new_blocks;
  prm.items = reinterpret_cast<const int4*>(work_items);
  char* ws = static_cast<char*>(workspace);
  prm.ws_error = reinterpret_cast<int32_t*>(ws);
  prm.ws_sched = reinterpret_cast<int32_t*>(ws + wl.sched);
  prm.deferred = deferred;
  prm.deferred_refs = deferred ? deferred_refs : 0;
  prm.deferred_lens = deferred ? deferred_lens : 0;
  prm.refcounts = refcounts;
  prm.ws_ml = reinterpret_cast<float*>(ws + wl.ml);
  prm.ws_o = reinterpret_cast<float*>(ws + wl.o);
  prm.step_header = step_header;
  prm.n_combine = n_combine;
  prm.n_items = n_items;
  prm.batch = batch;
  prm.table_stride = table_stride;
  prm.table_rows = table_rows;
  prm.hq = num_q_heads;
  prm.hkv = g->num_kv_heads;
  prm.group = num_q_heads / g->num_kv_heads;
  prm.layer = layer;
  prm.num_blocks = g->num_blocks;
  prm.pages_per_split = pages_per_split;
  prm.scale_log2 = scale * kLog2e;
  auto s = static_cast<cudaStream_t>(stream);
  const int4* entries = combine_entries ? reinterpret_cast<const int4*>(combine_entries)
                                        : reinterpret_cast<const int4*>(work_items) + n_items;
  if (g->head_dim == 128)
    return g->dtype == PKV_BF16 ? launch_for_heads<128, __nv_bfloat16>(prm, entries, s)
                                : launch_for_heads<128, __half>(prm, entries, s);
  return g->dtype == PKV_BF16 ? launch_for_heads<64, __nv_bfloat16>(prm, entries, s)
                              : launch_for_heads<64, __half>(prm, entries, s);
}

extern "C" {

// ---------------------------------------------------------------------------
// Decode without a caller-provided workspace.
//
// Some callers of this library may not allocate device memory while they
// run: an inference server or framework that owns every byte of the GPU
// through its own arena (so that memory accounting stays exact and no
// cudaMalloc / cudaFree ever stalls the device), or a plugin interface that
// only hands the library buffers it allocated itself.  They can pass their
// inputs and outputs but cannot provide the decode workspace.  For them,
// pkv_decode_attention_noalloc takes its scratch (error word, scheduler
// counters, split-K partials) from a fixed array in this file's device
// memory instead.  The array exists on every GPU that loads this library and
// stays allocated until the process exits.
namespace {
constexpr int64_t kStaticScratchBytes = 16ll << 20;  // 16 MiB
__device__ __align__(256) unsigned char g_decode_scratch[kStaticScratchBytes];
constexpr int kMaxDevices = 64;
std::mutex g_scratch_mutex;
void* g_scratch_addr[kMaxDevices] = {};
}  // namespace

int32_t pkv_decode_attention_noalloc(const pkv_pool_geom* g, void* pool, int32_t layer, const void* q,
                                     const void* k_new, const void* v_new, int32_t* block_tables,
                                     int32_t table_stride, int32_t table_rows, int32_t* context_lens,
                                     const int32_t* rows, const int32_t* seq_lens, const int32_t* new_blocks,
                                     const int32_t* work_items, int32_t n_items, int32_t n_combine, int32_t batch,
                                     int32_t num_q_heads, int32_t pages_per_split, float scale, void* out,
                                     void* stream) {
  pkv_clear_error();
  if (!g) {
    pkv_set_error("null pool geometry");
    return PKV_ERR_ARG;
  }
  const int64_t need = ws_layout(batch, g->num_kv_heads, g->head_dim, n_items).total;
  if (need > kStaticScratchBytes) {
    pkv_set_error("pkv_decode_attention_noalloc: this step needs " + std::to_string(need) +
                  " bytes of scratch, more than the 16 MiB static scratch (fewer or shorter sequences per "
                  "call, or pkv_decode_attention with a workspace)");
    return PKV_ERR_ARG;
  }
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    pkv_set_error(std::string("pkv_decode_attention_noalloc: cudaGetDevice: ") + cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    pkv_set_error("pkv_decode_attention_noalloc: device index out of range");
    return PKV_ERR_UNSUPPORTED;
  }
  void* scratch = nullptr;
  {
    // The array's name is only a host-side stand-in: its device address must
    // be looked up, once per device, with that device current.
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    if (!g_scratch_addr[dev]) {
      e = cudaGetSymbolAddress(&g_scratch_addr[dev], g_decode_scratch);
      if (e != cudaSuccess) {
        g_scratch_addr[dev] = nullptr;
        pkv_set_error(std::string("pkv_decode_attention_noalloc: cudaGetSymbolAddress: ") + cudaGetErrorString(e));
        return PKV_ERR_CUDA;
      }
    }
    scratch = g_scratch_addr[dev];
  }
  // The scratch keeps the previous call's contents: clear the error word and
  // the scheduler counters, which the kernels expect at zero.  (The split-K
  // partials are always written before they are read.)
  e = cudaMemsetAsync(scratch, 0, 256, static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) {
    pkv_set_error(std::string("pkv_decode_attention_noalloc: cudaMemsetAsync: ") + cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  return pkv_decode_attention(g, pool, layer, q, k_new, v_new, block_tables, table_stride, table_rows, context_lens,
                              rows, seq_lens, new_blocks, work_items, n_items, n_combine, batch, num_q_heads,
                              pages_per_split, scale, out, scratch, kStaticScratchBytes, stream);
}

int32_t pkv_decode_noalloc_error(int32_t* error_out, void* stream) {
  pkv_clear_error();
  if (!error_out) {
    pkv_set_error("pkv_decode_noalloc_error: error_out must not be NULL");
    return PKV_ERR_ARG;
  }
  *error_out = 0;
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) {
    pkv_set_error(std::string("pkv_decode_noalloc_error: cudaGetDevice: ") + cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  if (dev < 0 || dev >= kMaxDevices) {
    pkv_set_error("pkv_decode_noalloc_error: device index out of range");
    return PKV_ERR_UNSUPPORTED;
  }
  void* scratch = nullptr;
  {
    std::lock_guard<std::mutex> lock(g_scratch_mutex);
    scratch = g_scratch_addr[dev];
  }
  if (!scratch) return PKV_OK;  // no no-alloc call on this device yet
  // The error word is the scratch's first int32; read it in stream order,
  // after the calls issued so far on `stream`, and wait for the copy.
  auto s = static_cast<cudaStream_t>(stream);
  e = cudaMemcpyAsync(error_out, scratch, sizeof(int32_t), cudaMemcpyDeviceToHost, s);
  if (e == cudaSuccess) e = cudaStreamSynchronize(s);
  if (e != cudaSuccess) {
    pkv_set_error(std::string("pkv_decode_noalloc_error: ") + cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}

}  // extern "C"
