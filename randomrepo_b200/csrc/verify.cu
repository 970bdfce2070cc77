// Speculative-verify attention over pages, keys on the tensor-core rows (sm_100a, tcgen05).
//
// Replaces, for one layer, the attention of AgentRL's speculative verify
// forward (agentrl/generation/speculative.py:229-264: rows prefix_len-1 ..
// prefix_len-1+k of its full causal forward are k+1 queries after
// prefix_len-1 cached tokens; HF's causal mask with a past offset,
// transformers integrations/sdpa_attention.py:40-62, with GQA).  It computes
// what the chunked-prefill kernel (prefill.cu) computes for a short chunk, with
// the tile transposed: there a 128-row query tile holds (position, head) rows,
// and a verify item fills only G x (k+1) of them (30 at 12 query / 2 KV heads,
// k = 4).  Here, per KV tile of 128 keys,
//   S^T  = K Q^T     M = 128 keys, N = 32 query columns, K = head_dim,
//   O^T += V^T P^T   M = head_dim, N = 32, K = the tile's keys,
// A and B both in shared memory: K (K-major) and V (MN-major: V^T) straight
// from the pool's pre-swizzled page slabs, Q (K-major) and P^T (MN-major: one
// 64-byte row per key) written by the softmax threads.  Column c = position *
// G + head of the item's queries; an item holds 32 / G positions of one
// sequence and KV head, over a range of its KV tiles.
//
// The grid is persistent: one CTA per SM (192 threads, 225 KB of shared
// memory, 128 tensor-memory columns) works through a list of items the host
// plan balanced across the SMs (record c is CTA c's first item; the rest are
// copied into shared memory once).  Barrier phases count the CTA's KV tiles
// g across items.  Roles:
//   warps 0-3  softmax, thread = key of the tile (its tensor-memory lane): a
//              32-column tcgen05.ld of S^T; on an item's first tile the exact
//              column maxima over the 128 keys (a shuffle transpose-reduction
//              in each warp, four partials through shared memory at a
//              barrier), on later tiles only a test whether some logit exceeds
//              its column's running maximum by more than 2^8 (then the exact
//              maxima, and O^T rescaled in tensor memory); P^T stored as the
//              key's 64-byte row; query columns of the items two ahead copied
//              with cp.async; in the epilogue thread = head_dim row of O^T,
//              the output staged through shared memory as 16-byte stores;
//   warp 4     producer, lanes 0-15 for K and 16-31 for V on their own: 2 KB
//              cp.async.bulk copies of every page's slabs into a 2-stage K
//              and a 3-stage V ring (no tensor map, no multicast), the next
//              tile's block ids read before the wait for a free stage;
//   warp 5     allocates tensor memory (S^T double-buffered, O^T); lane 0
//              issues the next S and the next P V, each as soon as its
//              operands are in.
// A key range that is not the whole sequence writes an unnormalised partial
// (prefill.cu's slot format), merged by paged_verify_combine_kernel, launched
// as a programmatic dependent of this grid.
//
// Every wait is bounded; a timed-out role records an error word and skips the
// rest of its work, the MMA thread waits (bounded) for its last MMAs and the
// producer for its copies before tensor memory is freed.
#include "pkv_device.cuh"
#include "pkv_error.h"
#include "pkv_prefill.cuh"

#include <algorithm>
#include <queue>
#include <string>
#include <type_traits>
#include <utility>
#include <vector>

namespace pkv {
namespace {

constexpr int kVD = 128;                 // head_dim
constexpr int kCols = 32;                // query columns of an item (N)
constexpr int kVThreads = 192;
constexpr int kSoftThreads = 128;
constexpr int kVProducerWarp = 4;
constexpr int kVMmaWarp = 5;
constexpr int kVTmemCols = 128;          // S^T buffers at columns 0 and 32, O^T at 64
constexpr int kNK = 2;                   // K ring stages (one KV tile each)
constexpr int kNV = 3;                   // V ring stages: V(g) waits for P V(g - 3), K(g) only for S(g - 2)
constexpr int kVSlabBytes = kKeys * 128; // one 64-dim slab of a KV tile
constexpr int kVTileBytes = 2 * kVSlabBytes;
constexpr int kQSlab = kCols * 128;      // one 64-dim slab of the query columns
constexpr int kQBytes = 2 * kQSlab;      // one item's query columns
constexpr int kNQ = 3;                   // query buffers: item i in buffer i % 3
constexpr int kPBytes = kKeys * 128;     // P^T of one tile: 128 key rows of 128 bytes (64 used)
constexpr int kMaxList = 128;            // work items one CTA holds in shared memory
constexpr int64_t kItemCost = 2;         // fixed work of one item, in KV tiles (plan balance)
constexpr int64_t kCombineCost = 5;      // the combine launch, in KV tiles (plan: cut or not)
constexpr int kOffQ = 0;
constexpr int kOffP = kOffQ + kNQ * kQBytes;       // two buffers, tiles alternate
constexpr int kOffK = kOffP + 2 * kPBytes;
constexpr int kOffV = kOffK + kNK * kVTileBytes;
constexpr int kOffBar = kOffV + kNV * kVTileBytes;
constexpr uint32_t kPageSlab = kPageRows * 128;

// Barrier phases are counted over the CTA's whole sequence of KV tiles g (and
// items i), across item boundaries: ring stage g % stages, parity (g / stages) & 1.
struct VBars {
  uint64_t q_full[kNQ];     // 128 arrivals: item i's query columns in buffer i % 3
  uint64_t k_full[kNK];     // producer expect_tx + copy bytes
  uint64_t k_empty[kNK];    // MMA commit after S(g)
  uint64_t v_full[kNV];
  uint64_t v_empty[kNV];    // MMA commit after P V(g)
  uint64_t s_full[2];       // MMA commit after S(g), per S^T buffer
  uint64_t p_full[2];       // 128 softmax arrivals: P^T(g) stored (and O^T rescaled), per P^T buffer
  uint64_t pv_done;         // MMA commit after P V(g)
  uint64_t o_done;          // MMA commit after an item's last P V
  uint64_t mma_done;        // final commit of the MMA thread
  uint64_t list_full;       // 128 arrivals: the CTA's later items copied into `list`
  uint32_t tmem_base;
  int32_t abort;
  float red[2][4][kCols];   // per-warp column maxima, double-buffered by tile parity
  float lsum[4][kCols];     // per-warp column sums (epilogue)
  int4 list[kMaxList - 1][2];  // the CTA's items after its first
};
constexpr int kVSmemBytes = kOffBar + 8192 + 1024;  // + barriers and item list, + alignment slack

// One work item as every role of the CTA decodes it; bad: outside the launch.
struct VItem {
  int row, pos0, qrow0, h, nt, ncols, kv_len, n_tiles, kt_lo, n, slot, entry;
  bool bad;
};

__device__ __forceinline__ VItem decode_item(const PrefillParams& p, int4 a, int4 b) {
  VItem it;
  it.row = a.x;
  it.pos0 = a.y;
  it.qrow0 = a.z;
  it.h = a.w >> 16;
  it.nt = a.w & 0xffff;
  it.ncols = it.nt * p.group;
  it.kv_len = it.pos0 + it.nt;  // keys the item's last query sees
  it.n_tiles = (it.kv_len + kKeys - 1) / kKeys;
  it.kt_lo = b.x & 0xffff;
  const int kt_hi = (b.x >> 16) > 0 ? (b.x >> 16) : it.n_tiles;
  it.slot = b.z;
  it.entry = b.y;
  const bool ok = it.row >= 0 && it.row < p.table_rows && it.h >= 0 && it.h < p.hkv && it.nt >= 1 &&
                  it.nt <= p.ppi && it.ncols <= kCols && it.pos0 >= 0 && it.qrow0 >= 0 &&
                  (int64_t)it.qrow0 + it.nt <= p.total_q &&
                  (it.kv_len + kPageRows - 1) / kPageRows <= p.table_stride && it.kt_lo >= 0 &&
                  it.kt_lo < kt_hi && kt_hi <= it.n_tiles && it.slot >= -1 && it.slot < p.n_slots &&
                  it.entry >= -1 && it.entry < p.n_combine && (it.slot >= 0) == (it.entry >= 0) &&
                  (it.slot >= 0 || (it.kt_lo == 0 && kt_hi == it.n_tiles));
  it.bad = !ok;
  it.n = ok ? kt_hi - it.kt_lo : 0;
  return it;
}

// Non-blocking test of phase `parity` of `bar`.
__device__ __forceinline__ bool mbar_test(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// 16-byte asynchronous copy global -> shared (zero-filled when !valid), and
// the wait for this thread's copies but the most recent `n` groups.
__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc, bool valid) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16, %2;" ::"r"(smem_u32(smem_dst)), "l"(gsrc),
               "r"(valid ? 16 : 0)
               : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
__device__ __forceinline__ void cp_async_wait_all_but_one() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// The 128 softmax threads: barrier 1, returning whether any of them passed `pred`.
__device__ __forceinline__ bool softmax_bar_any(bool pred) {
  uint32_t r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.u32 p, %1, 0;\n\t"
      "bar.red.or.pred q, 1, 128, p;\n\t"
      "selp.u32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"(static_cast<uint32_t>(pred))
      : "memory");
  return r != 0;
}

// Warp transpose-reduction: lane l holds 32 values (one per column); on return
// lane l holds op over the 32 lanes of column l (31 shuffles; v is consumed).
template <bool kMax>
__device__ __forceinline__ float warp_columns(float (&v)[32], int lane) {
#pragma unroll
  for (int w = 16; w >= 1; w >>= 1) {
    const bool hi = (lane & w) != 0;
#pragma unroll
    for (int i = 0; i < w; ++i) {
      const float send = hi ? v[i] : v[i + w];
      const float keep = hi ? v[i + w] : v[i];
      const float recv = __shfl_xor_sync(0xffffffffu, send, w);
      v[i] = kMax ? fmaxf(keep, recv) : keep + recv;
    }
  }
  return v[0];
}

template <typename T>
__global__ void __launch_bounds__(kVThreads, 1) paged_verify_kernel(const __grid_constant__ PrefillParams p) {
  constexpr uint32_t kFmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t kIdescS = umma_idesc_f16(kFmt, 0, 0, kKeys, kCols);  // K-major K, K-major Q
  constexpr uint32_t kIdescO = umma_idesc_f16(kFmt, 1, 1, kVD, kCols);    // MN-major V^T, MN-major P^T

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
  uint8_t* q_s = smem + kOffQ;
  uint8_t* p_s = smem + kOffP;
  uint8_t* k_s = smem + kOffK;
  uint8_t* v_s = smem + kOffV;
  VBars* bars = reinterpret_cast<VBars*>(smem + kOffBar);
  volatile int32_t* abort = &bars->abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  // The combine grid may be scheduled once every CTA of this grid has started
  // (it waits for this grid's completion before reading the partials).
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
  // The CTA's first work item is record blockIdx.x; its last field gives the
  // rest of the CTA's list: (first record << 8) | count, contiguous.  The
  // (cold) loads are in flight while the barriers and tensor memory are set up.
  const int4 head_a = p.items[2 * blockIdx.x];
  const int4 head_b = p.items[2 * blockIdx.x + 1];
  if (tid == 0) {
    for (int x = 0; x < kNQ; ++x) mbar_init(&bars->q_full[x], kSoftThreads);
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars->s_full[x], 1);
      mbar_init(&bars->p_full[x], kSoftThreads);
    }
    for (int x = 0; x < kNK; ++x) {
      mbar_init(&bars->k_full[x], 1);
      mbar_init(&bars->k_empty[x], 1);
    }
    for (int x = 0; x < kNV; ++x) {
      mbar_init(&bars->v_full[x], 1);
      mbar_init(&bars->v_empty[x], 1);
    }
    mbar_init(&bars->pv_done, 1);
    mbar_init(&bars->o_done, 1);
    mbar_init(&bars->mma_done, 1);
    mbar_init(&bars->list_full, kSoftThreads);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == kVMmaWarp) tmem_alloc(&bars->tmem_base, kVTmemCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = bars->tmem_base;

  const VItem first = decode_item(p, head_a, head_b);
  const int follow_off = head_b.w >> 8, follow_cnt = head_b.w & 0xff;
  const bool list_ok = follow_cnt <= kMaxList - 1 && (follow_cnt == 0 || (follow_off >= 0 &&
                       (int64_t)follow_off + follow_cnt <= p.n_items));
  const int n_list = first.bad ? 0 : 1 + (list_ok ? follow_cnt : 0);
  // Item k of the CTA's list (k >= 1 read from shared memory once list_full
  // has completed; n = 0 past the list or for a record outside the launch).
  auto item_at = [&](int k) -> VItem {
    if (k == 0) return first;
    VItem none;
    none.n = 0;
    none.bad = false;
    if (k >= n_list) return none;
    return decode_item(p, bars->list[k - 1][0], bars->list[k - 1][1]);
  };

  if (warp == kVProducerWarp) {
    // ---------------- producer ----------------
    // Lanes 0-15 stream K, lanes 16-31 V, each half on its own through the
    // CTA's items: lane l of a half copies slab (l & 1) of page (l >> 1) of a
    // tile (at most 8 pages x 2 slabs), and loads its block id for the next
    // tile (of this item or the next) before it waits for a free stage, so
    // the table read is off the copy chain.
    const int state = lane >> 4;  // 0 = K, 1 = V
    const int hl = lane & 15;
    const unsigned half = state ? 0xffff0000u : 0x0000ffffu;
    const int ns = state ? kNV : kNK;
    uint8_t* ring = state ? v_s : k_s;
    uint64_t* fulls = state ? bars->v_full : bars->k_full;
    uint64_t* empties = state ? bars->v_empty : bars->k_empty;
    auto block_of = [&](const VItem& it, int t) -> int {  // this lane's page of KV tile t, -1 past the sequence
      const int pg = t * kPagesPerTile + (hl >> 1);
      return pg * kPageRows < it.kv_len ? __ldg(p.tables + (int64_t)it.row * p.table_stride + pg) : -1;
    };
    bool run = n_list > 1 ? __all_sync(half, wait_or_abort(&bars->list_full, 0, p, abort)) : true;
    int blk = first.n > 0 ? block_of(first, first.kt_lo) : -1;
    int g = 0;
    for (int k = 0; run && k < n_list; ++k) {
      const VItem it = item_at(k);
      if (it.n == 0) break;
      const VItem nx = item_at(k + 1);
      for (int j = 0; j < it.n; ++j) {
        const int nblk = j + 1 < it.n ? block_of(it, it.kt_lo + j + 1) : (nx.n > 0 ? block_of(nx, nx.kt_lo) : -1);
        const int st = g % ns;
        // Stage free once S(g - ns) (K) or P V(g - ns) (V) completed.
        if (g >= ns && !__all_sync(half, wait_or_abort(&empties[st], ((g / ns) - 1) & 1, p, abort))) {
          run = false;
          break;
        }
        const int key0 = (it.kt_lo + j) * kKeys;
        const int pages = min(kPagesPerTile, (it.kv_len - key0 + kPageRows - 1) / kPageRows);
        if (hl == 0) mbar_arrive_expect_tx(&fulls[st], pages * 2 * kPageSlab);
        __syncwarp(half);
        if ((hl >> 1) < pages) {
          int b = blk;
          if (b < 0 || b >= p.num_blocks) {
            atomicExch(p.error, kDevBadBlock);
            b = 0;
          }
          const char* src = p.pool +
                            page_offset(p.layer, b, it.h, state, p.num_blocks, p.hkv, kPageRows, kVD * 2) +
                            (hl & 1) * kPageSlab;
          bulk_copy_g2s(ring + st * kVTileBytes + (hl & 1) * kVSlabBytes + (hl >> 1) * kPageSlab, src, kPageSlab,
                        &fulls[st]);
        }
        blk = nblk;
        ++g;
      }
    }
    // Copies still in flight must land before the CTA frees its memory.
    if (hl == 0)
      for (int c = max(0, g - ns); c < g; ++c) mbar_wait_bounded(&fulls[c % ns], (c / ns) & 1);
    __syncwarp();
  } else if (warp == kVMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t q_addr = smem_u32(q_s);
      const uint32_t p_addr = smem_u32(p_s);
      const uint32_t k_addr = smem_u32(k_s);
      const uint32_t v_addr = smem_u32(v_s);
      auto issue_s = [&](int g, int qbuf) {  // S^T(g) = K(g) Q^T into buffer g & 1
        const uint32_t kb = k_addr + (g % kNK) * kVTileBytes;
        const uint32_t qb = q_addr + qbuf * kQBytes;
#pragma unroll
        for (int ks = 0; ks < kVD / 16; ++ks) {
          const uint64_t adesc = umma_desc_sw128(kb + (ks >> 2) * kVSlabBytes + (ks & 3) * 32, 16, 1024);
          const uint64_t bdesc = umma_desc_sw128(qb + (ks >> 2) * kQSlab + (ks & 3) * 32, 16, 1024);
          umma_f16_ss(tmem + (g & 1) * kCols, adesc, bdesc, kIdescS, ks > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[g & 1]);
        umma_commit(&bars->k_empty[g % kNK]);
      };
      auto issue_pv = [&](int g, const VItem& it, int j) {  // O^T += V(g)^T P^T(g), one page (16 keys) per MMA
        const int key0 = (it.kt_lo + j) * kKeys;
        const int steps = min(kPagesPerTile, (it.kv_len - key0 + kPageRows - 1) / kPageRows);
        const uint32_t vb = v_addr + (g % kNV) * kVTileBytes;
        const uint32_t pb = p_addr + (g & 1) * kPBytes;
        for (int ks = 0; ks < steps; ++ks) {
          const uint64_t adesc = umma_desc_sw128(vb + ks * 2048, kVSlabBytes, 1024);
          const uint64_t bdesc = umma_desc_sw128(pb + ks * 2048, kVSlabBytes, 1024);
          umma_f16_ss(tmem + 2 * kCols, adesc, bdesc, kIdescO, (j > 0 || ks > 0) ? 1u : 0u);
        }
        umma_commit(&bars->v_empty[g % kNV]);
        umma_commit(&bars->pv_done);
        if (j == it.n - 1) umma_commit(&bars->o_done);
      };
      bool alive = first.n > 0 && (n_list < 2 || wait_or_abort(&bars->list_full, 0, p, abort));
      // Two cursors over the CTA's tiles: the next S and the next P V.  Each is
      // issued as soon as its operands are in: S(g) once K(g) has landed (and
      // its item's query columns), and P V(g-2) was issued (its S^T buffer was
      // last read by softmax(g-2), done before that); P V(g) once S(g) was
      // issued, P^T(g) is stored and V(g) has landed.
      int s_k = 0, s_j = 0, s_g = 0;  // next S: item, tile of the item, tile of the CTA
      int v_k = 0, v_j = 0, v_g = 0;  // next P V
      VItem s_it = first, v_it = first;
      long long idle0 = clock64();
      while (alive && v_it.n > 0) {
        bool did = false;
        if (s_it.n > 0 && s_g <= v_g + 1 && (s_j > 0 || mbar_test(&bars->q_full[s_k % kNQ], (s_k / kNQ) & 1)) &&
            mbar_test(&bars->k_full[s_g % kNK], (s_g / kNK) & 1)) {
          tc_fence_after_sync();
          issue_s(s_g, s_k % kNQ);
          ++s_g;
          if (++s_j == s_it.n) {
            s_j = 0;
            s_it = item_at(++s_k);
          }
          did = true;
        }
        if (v_g < s_g && mbar_test(&bars->p_full[v_g & 1], (v_g >> 1) & 1) &&
            mbar_test(&bars->v_full[v_g % kNV], (v_g / kNV) & 1)) {
          tc_fence_after_sync();
          issue_pv(v_g, v_it, v_j);
          ++v_g;
          if (++v_j == v_it.n) {
            v_j = 0;
            v_it = item_at(++v_k);
          }
          did = true;
        }
        if (did) {
          idle0 = clock64();
        } else if (*abort) {
          alive = false;
        } else if (clock64() - idle0 > kWaitLimitCycles) {
          record_error(p, abort, kDevWaitTimeout);
          alive = false;
        } else {
          __nanosleep(32);
        }
      }
      // Every MMA issued must complete before tensor memory is freed.
      umma_commit(&bars->mma_done);
      mbar_wait_bounded(&bars->mma_done, 0);
    }
    __syncwarp();
  } else {
    // ---------------- softmax / epilogue (warps 0-3) ----------------
    const uint32_t lane_base = static_cast<uint32_t>(warp * 32) << 16;
    const uint32_t o_addr = tmem + lane_base + 2 * kCols;
    const float sl2 = p.scale_log2;
    // The rest of the CTA's list into shared memory, once.
    if (list_ok && tid < follow_cnt) {
      bars->list[tid][0] = p.items[2 * (follow_off + tid)];
      bars->list[tid][1] = p.items[2 * (follow_off + tid) + 1];
    }
    mbar_arrive(&bars->list_full);
    if (first.bad && tid == 0) atomicExch(p.error, kDevBadItem);
    bool fail = n_list > 1 && !__all_sync(0xffffffffu, wait_or_abort(&bars->list_full, 0, p, abort));
    // Query columns of item k into buffer k % 3 with cp.async (thread t: 4 of
    // the 16 chunks of column t / 4; zero for unused columns), K-major with
    // the 128-byte swizzle.  Item k+2's copies start at item k's first tile
    // (its buffer was item k-1's, whose S products have completed by then)
    // and item k+1's are waited for there, so that its columns are in long
    // before its first S: one commit group per item.
    const int qc = tid >> 2, qc0 = (tid & 3) * 4;
    auto q_issue = [&](int k) {
      const VItem q_it = item_at(k);
      if (q_it.n > 0) {
        const bool in = qc < q_it.ncols;
        const T* src = static_cast<const T*>(p.q) +
                       (((int64_t)q_it.qrow0 + (in ? qc / p.group : 0)) * p.hq + (int64_t)q_it.h * p.group +
                        (in ? qc % p.group : 0)) * kVD;
        uint8_t* qb = q_s + (k % kNQ) * kQBytes;
#pragma unroll
        for (int c4 = 0; c4 < 4; ++c4) {
          const int ch = qc0 + c4;
          cp_async16(qb + (ch >> 3) * kQSlab + swz128(qc, ch & 7), reinterpret_cast<const uint4*>(src) + ch, in);
        }
      }
      cp_async_commit();
    };
    auto q_publish = [&](int k) {  // every group but the newest has landed: item k's columns are in
      cp_async_wait_all_but_one();
      if (item_at(k).n > 0) {
        fence_proxy_async_smem();
        mbar_arrive(&bars->q_full[k % kNQ]);
      }
    };
    q_issue(0);
    q_issue(1);
    q_publish(0);
    float mrep[kCols];   // every column's running maximum, in every thread
    float lpart[kCols];  // this key's share of every column's sum
    int g = 0;
    for (int k = 0; k < n_list && !fail; ++k) {
      const VItem it = item_at(k);
      if (it.bad && tid == 0) atomicExch(p.error, kDevBadItem);
      if (it.n == 0) break;
      const uint32_t colmask = it.ncols >= 32 ? 0xffffffffu : ((1u << it.ncols) - 1u);
      float m_run = -INFINITY;  // running maximum of column `lane` (the same in all four warps)
#pragma unroll
      for (int c = 0; c < kCols; ++c) {
        mrep[c] = -INFINITY;
        lpart[c] = 0.f;
      }
      for (int j = 0; j < it.n; ++j, ++g) {
        const bool got =
            !fail && __all_sync(0xffffffffu, wait_or_abort(&bars->s_full[g & 1], (g >> 1) & 1, p, abort));
        // S(g) completed, so every earlier S did: item k-1's query buffer is
        // free for item k+2's columns.
        if (j == 0 && got) {
          q_issue(k + 2);
          q_publish(k + 1);
        }
        const int key0 = (it.kt_lo + j) * kKeys;
        const uint32_t s_addr = tmem + lane_base + (g & 1) * kCols;
        // Columns this key is visible to.  A tile wholly before the diagonal
        // has every key loaded and visible; there the unused columns (zero
        // query rows, S = 0) are kept like the others.  From the diagonal on,
        // a key sees the columns whose position is >= the key (none past the
        // sequence).
        const bool masked = key0 + kKeys - 1 > it.pos0;
        uint32_t vis = 0xffffffffu;
        if (masked) {
          const int dk = key0 + tid - it.pos0;
          vis = dk >= it.nt ? 0u : (dk > 0 ? colmask & ~((1u << (dk * p.group)) - 1u) : colmask);
        }
        // x = S * scale * log2(e) - m per column (-inf where not visible); the
        // running maxima only move when some x exceeds 2^8.
        float xm[kCols];
        float xmax = -INFINITY;
        if (got) tc_fence_after_sync();
        if (got && j > 0) {
          uint32_t sr[kCols];
          tmem_ld32_bits(s_addr, sr);
          if (masked) {
#pragma unroll
            for (int c = 0; c < kCols; ++c)
              xm[c] = ((vis >> c) & 1u) ? fmaf(__uint_as_float(sr[c]), sl2, -mrep[c]) : -INFINITY;
          } else {
#pragma unroll
            for (int c = 0; c < kCols; ++c) xm[c] = fmaf(__uint_as_float(sr[c]), sl2, -mrep[c]);
          }
#pragma unroll
          for (int c = 0; c < kCols; ++c) xmax = fmaxf(xmax, xm[c]);
        }
        // An item's first tile sets the running maxima from its exact column
        // maxima (nothing accumulated yet to rescale).
        if (j == 0) {
          if (got) {
            uint32_t sr[kCols];
            tmem_ld32_bits(s_addr, sr);
            float v[kCols];
#pragma unroll
            for (int c = 0; c < kCols; ++c) v[c] = ((vis >> c) & 1u) ? __uint_as_float(sr[c]) * sl2 : -INFINITY;
            bars->red[g & 1][warp][lane] = warp_columns<true>(v, lane);
          }
          if (softmax_bar_any(!got)) {
            fail = true;
            break;
          }
          m_run = fmaxf(fmaxf(bars->red[g & 1][0][lane], bars->red[g & 1][1][lane]),
                        fmaxf(bars->red[g & 1][2][lane], bars->red[g & 1][3][lane]));
          uint32_t sr[kCols];
          tmem_ld32_bits(s_addr, sr);
#pragma unroll
          for (int c = 0; c < kCols; ++c) {
            mrep[c] = __shfl_sync(0xffffffffu, m_run, c);
            xm[c] = ((vis >> c) & 1u) ? fmaf(__uint_as_float(sr[c]), sl2, -mrep[c]) : -INFINITY;
          }
        } else if (softmax_bar_any(!got || xmax > kRescaleLog2)) {
          // One barrier per tile makes both decisions (stop; move the maxima)
          // the same in all four warps.
          // Column maxima of this tile: a transpose-reduction in each warp,
          // the four warps' partials through shared memory at a second barrier.
          if (got) {
            uint32_t sr[kCols];
            tmem_ld32_bits(s_addr, sr);
            float v[kCols];
#pragma unroll
            for (int c = 0; c < kCols; ++c) v[c] = ((vis >> c) & 1u) ? __uint_as_float(sr[c]) * sl2 : -INFINITY;
            bars->red[g & 1][warp][lane] = warp_columns<true>(v, lane);
          }
          if (softmax_bar_any(!got)) {
            fail = true;
            break;
          }
          const float t = fmaxf(fmaxf(bars->red[g & 1][0][lane], bars->red[g & 1][1][lane]),
                                fmaxf(bars->red[g & 1][2][lane], bars->red[g & 1][3][lane]));
          const float m_new = t > m_run + kRescaleLog2 ? t : m_run;
          // O^T *= alpha per column (this thread's head_dim row), after P V(g-1) completed.
          const bool rescale_o =
              j > 0 && !fail && __all_sync(0xffffffffu, wait_or_abort(&bars->pv_done, (g - 1) & 1, p, abort));
          if (j > 0 && !rescale_o) fail = true;  // the next barrier stops every warp
          if (rescale_o) {
            tc_fence_after_sync();
            float o[kCols];
            tmem_ld32(o_addr, o);
#pragma unroll
            for (int c = 0; c < kCols; ++c) {
              const float mn = __shfl_sync(0xffffffffu, m_new, c);
              const float alpha = mn == mrep[c] ? 1.f : ex2_approx(mrep[c] - mn);
              mrep[c] = mn;
              lpart[c] *= alpha;
              o[c] *= alpha;
            }
            tmem_st32(o_addr, o);
          } else {
#pragma unroll
            for (int c = 0; c < kCols; ++c) {
              const float mn = __shfl_sync(0xffffffffu, m_new, c);
              lpart[c] *= mn == mrep[c] ? 1.f : ex2_approx(mrep[c] - mn);
              mrep[c] = mn;
            }
          }
          m_run = m_new;
          uint32_t sr[kCols];
          tmem_ld32_bits(s_addr, sr);
#pragma unroll
          for (int c = 0; c < kCols; ++c)
            xm[c] = ((vis >> c) & 1u) ? fmaf(__uint_as_float(sr[c]), sl2, -mrep[c]) : -INFINITY;
        }
        // P^T row of this key: 2^x (0 where x = -inf).
        uint32_t pk[kCols / 2];
#pragma unroll
        for (int c2 = 0; c2 < kCols / 2; ++c2) {
          const float p0 = ex2_approx(xm[2 * c2]);
          const float p1 = ex2_approx(xm[2 * c2 + 1]);
          lpart[2 * c2] += p0;
          lpart[2 * c2 + 1] += p1;
          pk[c2] = MmaOp<T>::pack(p0, p1);
        }
        uint8_t* prow = p_s + (g & 1) * kPBytes;
#pragma unroll
        for (int q4 = 0; q4 < 4; ++q4)
          *reinterpret_cast<uint4*>(prow + swz128(tid, q4)) =
              make_uint4(pk[4 * q4], pk[4 * q4 + 1], pk[4 * q4 + 2], pk[4 * q4 + 3]);
        // The sequence's last KV tile: V rows past the sequence inside its
        // last page are zeroed so that their zero probabilities multiply
        // finite values.  V(g) is copied once P V(g - kNV) completed, which
        // S(g) implies, so its stage has been filled g / kNV or g / kNV + 1
        // times: the parity tells the two apart.
        if (it.kt_lo + j == it.n_tiles - 1 && (it.kv_len & (kPageRows - 1)) != 0) {
          if (__all_sync(0xffffffffu, wait_or_abort(&bars->v_full[g % kNV], (g / kNV) & 1, p, abort))) {
            const int first_row = it.kv_len - key0;
            const int last_row = (first_row + kPageRows - 1) & ~(kPageRows - 1);
            uint8_t* vb = v_s + (g % kNV) * kVTileBytes;
            for (int e = tid; e < (last_row - first_row) * 16; e += kSoftThreads) {
              const int slab = e / ((last_row - first_row) * 8);
              const int rem = e % ((last_row - first_row) * 8);
              *reinterpret_cast<uint4*>(vb + slab * kVSlabBytes + swz128(first_row + rem / 8, rem & 7)) =
                  make_uint4(0, 0, 0, 0);
            }
          } else {
            fail = true;
          }
        }
        fence_proxy_async_smem();
        tc_fence_before_sync();
        mbar_arrive(&bars->p_full[g & 1]);
      }
      // Epilogue of the item.  Column sums: lane c of each warp gets its
      // warp's share, the four shares meet in shared memory at a barrier that
      // also makes the decision to stop the same in all four warps.
      bars->lsum[warp][lane] = warp_columns<false>(lpart, lane);
      fail = softmax_bar_any(fail);
      const float lsum_c =
          (bars->lsum[0][lane] + bars->lsum[1][lane]) + (bars->lsum[2][lane] + bars->lsum[3][lane]);
      // The output step has barriers of its own: whether it runs is decided
      // the same in all four warps.
      const bool o_in = !fail && __all_sync(0xffffffffu, wait_or_abort(&bars->o_done, k & 1, p, abort));
      if (softmax_bar_any(!o_in)) fail = true;
      if (!fail) {
        tc_fence_after_sync();
        float o[kCols];
        tmem_ld32(o_addr, o);  // this thread's head_dim row `tid` of O^T: one value per column
        tc_fence_before_sync();
        if (it.slot >= 0) {
          float* part = p.partials + (int64_t)it.slot * (2 * kRows + kRows * kVD);
          if (warp == 0 && lane < it.ncols) {
            part[lane] = m_run;
            part[kRows + lane] = lsum_c;
          }
#pragma unroll
          for (int c = 0; c < kCols; ++c)
            if (c < it.ncols) part[2 * kRows + c * kVD + tid] = o[c];
        } else {
          // O / l in the output dtype, staged in shared memory (the P^T
          // buffers: the item's products have completed) as [column][head_dim],
          // then written one 16-byte chunk per thread and step: each column is
          // a 256-byte row of the output.
          const float inv_c = 1.f / lsum_c;  // lane c: column c
          T* stage = reinterpret_cast<T*>(p_s);
#pragma unroll
          for (int c = 0; c < kCols; ++c)
            stage[c * kVD + tid] = MmaOp<T>::from_float(o[c] * __shfl_sync(0xffffffffu, inv_c, c));
          asm volatile("bar.sync 1, 128;" ::: "memory");
          for (int e = tid; e < it.ncols * (kVD / 8); e += kSoftThreads) {
            const int c = e / (kVD / 8), ch = e % (kVD / 8);
            T* dst = static_cast<T*>(p.out) +
                     (((int64_t)it.qrow0 + c / p.group) * p.hq + (int64_t)it.h * p.group + c % p.group) * kVD;
            reinterpret_cast<uint4*>(dst)[ch] = reinterpret_cast<const uint4*>(stage + c * kVD)[ch];
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");  // the stage is free again for the next item's P^T
        }
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == kVMmaWarp) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kVTmemCols);
  }
}

// Merge the key-range partials of one item (one CTA per combine entry):
// every slot's m and l in one round of loads (thread = slot x column), then
// per column r: m = max_s m_s and weights w_s = 2^(m_s - m) / sum_s 2^(m_s -
// m) l_s, then out[r][d] = sum_s w_s O_s[r][d] with thread = head_dim element
// and 8 rows per thread, so each slot's rows are read as coalesced 512-byte
// runs with 16 loads in flight per thread; the rows leave through shared
// memory as 16-byte stores.
constexpr int kCombineThreads = 512;
template <typename T>
__global__ void __launch_bounds__(kCombineThreads) paged_verify_combine_kernel(const __grid_constant__ PrefillParams p,
                                                                               const int4* entries) {
  __shared__ float wsm[64][kCols];
  __shared__ float lsm[64][kCols];
  __shared__ __align__(16) T stage[kCols * kVD];
  const int4 e = entries[2 * blockIdx.x];  // records are two int4 apart
  const int slot0 = e.x, ns = e.y, qrow0 = e.z, h = e.w >> 16, nt = e.w & 0xffff;
  const int tid = threadIdx.x;
  const int group = p.group;
  const int ncols = nt * group;
  if (slot0 < 0 || ns < 1 || ns > 64 || slot0 + ns > p.n_slots || nt < 1 || ncols > kCols || qrow0 < 0 ||
      (int64_t)qrow0 + nt > p.total_q || h < 0 || h >= p.hkv) {
    if (tid == 0) atomicExch(p.error, kDevBadItem);
    return;
  }
  constexpr int kSlotFloats = 2 * kRows + kRows * kVD;
  const float* base = p.partials + (int64_t)slot0 * kSlotFloats;
  // Launched as a programmatic dependent of the verify grid: the partials are
  // complete (and visible) once that grid has finished.
  asm volatile("griddepcontrol.wait;" ::: "memory");
  for (int idx = tid; idx < ns * ncols; idx += kCombineThreads) {
    const int s = idx / ncols, c = idx % ncols;
    wsm[s][c] = base[(int64_t)s * kSlotFloats + c];
    lsm[s][c] = base[(int64_t)s * kSlotFloats + kRows + c];
  }
  __syncthreads();
  if (tid < ncols) {
    float m = -INFINITY;
    for (int s = 0; s < ns; ++s) m = fmaxf(m, wsm[s][tid]);
    float l = 0.f;
    for (int s = 0; s < ns; ++s) l += wsm[s][tid] == -INFINITY ? 0.f : ex2_approx(wsm[s][tid] - m) * lsm[s][tid];
    const float inv_l = 1.f / l;
    for (int s = 0; s < ns; ++s) wsm[s][tid] = wsm[s][tid] == -INFINITY ? 0.f : ex2_approx(wsm[s][tid] - m) * inv_l;
  }
  __syncthreads();
  const int d = tid & (kVD - 1), g = tid >> 7;  // rows g, g + 4, ...
  const float* o = base + 2 * kRows + d;
  float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
#pragma unroll 2
  for (int s = 0; s < ns; ++s) {
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int r = g + 4 * i;
      if (r < ncols) acc[i] += wsm[s][r] * o[(int64_t)s * kSlotFloats + r * kVD];
    }
  }
#pragma unroll
  for (int i = 0; i < 8; ++i) {
    const int r = g + 4 * i;
    if (r < ncols) stage[r * kVD + d] = MmaOp<T>::from_float(acc[i]);
  }
  __syncthreads();
  for (int x = tid; x < ncols * (kVD / 8); x += kCombineThreads) {
    const int r = x / (kVD / 8), ch = x % (kVD / 8);
    T* dst = static_cast<T*>(p.out) + (((int64_t)qrow0 + r / group) * p.hq + (int64_t)h * group + r % group) * kVD;
    reinterpret_cast<uint4*>(dst)[ch] = reinterpret_cast<const uint4*>(stage + r * kVD)[ch];
  }
}

template <typename T>
cudaError_t launch_verify(const PrefillParams& prm, int32_t n_ctas, int32_t n_combine, cudaStream_t stream) {
  static_assert(sizeof(VBars) <= 8192, "barrier block overflows its slot");
  static_assert(kVSmemBytes <= 232448, "verify tile exceeds the shared memory of one CTA");
  auto kern = paged_verify_kernel<T>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kVSmemBytes);
  if (err != cudaSuccess) return err;
  kern<<<n_ctas, kVThreads, kVSmemBytes, stream>>>(prm);
  err = cudaGetLastError();
  if (err != cudaSuccess || n_combine == 0) return err;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3((unsigned)n_combine);
  cfg.blockDim = dim3(kCombineThreads);
  cfg.dynamicSmemBytes = 0;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, paged_verify_combine_kernel<T>, prm, prm.items + 2 * prm.n_items);
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int32_t pkv_verify_positions_per_item(int32_t num_q_heads, int32_t num_kv_heads) {
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads != 0) return 0;
  const int group = num_q_heads / num_kv_heads;
  return group > kCols ? 0 : kCols / group;
}

extern "C" int32_t pkv_verify_plan(const int32_t* rows, const int32_t* past_lens, const int32_t* q_lens,
                                   int32_t n_seqs, int32_t num_q_heads, int32_t num_kv_heads, int32_t num_sms,
                                   int32_t* items_out, int64_t items_capacity, int64_t* n_items_out,
                                   int64_t* n_ctas_out, int64_t* n_combine_out, int64_t* n_slots_out) {
  pkv_clear_error();
  const int ppv = pkv_verify_positions_per_item(num_q_heads, num_kv_heads);
  if (ppv <= 0 || num_kv_heads > 0x7fff) {
    pkv_set_error("num_q_heads must be a positive multiple of num_kv_heads with at most 32 query heads per KV head");
    return PKV_ERR_UNSUPPORTED;
  }
  if (n_seqs < 0 || num_sms < 0 || !n_items_out || !n_ctas_out || !n_combine_out || !n_slots_out ||
      (n_seqs > 0 && (!rows || !past_lens || !q_lens))) {
    pkv_set_error("invalid plan arguments");
    return PKV_ERR_ARG;
  }
  struct Entry {
    int64_t work;  // KV tiles the item streams
    int32_t v[8];
  };
  std::vector<Entry> base;
  int64_t qrow = 0, total = 0;
  for (int32_t i = 0; i < n_seqs; ++i) {
    if (rows[i] < 0 || past_lens[i] < 0 || q_lens[i] < 0) {
      pkv_set_error("negative row, past length or query count for sequence " + std::to_string(i));
      return PKV_ERR_VALUE;
    }
    if ((int64_t)past_lens[i] + q_lens[i] > INT32_MAX || qrow + q_lens[i] > INT32_MAX ||
        (int64_t)past_lens[i] + q_lens[i] > (int64_t)0xffff * kKeys) {
      pkv_set_error("sequence or query count too large");
      return PKV_ERR_VALUE;
    }
    for (int32_t t0 = 0; t0 < q_lens[i]; t0 += ppv) {
      const int32_t n = std::min(ppv, q_lens[i] - t0);
      const int64_t kv_len = (int64_t)past_lens[i] + t0 + n;
      for (int32_t hk = 0; hk < num_kv_heads; ++hk) {
        base.push_back({(kv_len + kKeys - 1) / kKeys,
                        {rows[i], past_lens[i] + t0, static_cast<int32_t>(qrow + t0), (hk << 16) | n, 0, -1, -1, -1}});
        total += base.back().work;
      }
    }
    qrow += q_lens[i];
  }
  // num_sms > 0: a persistent grid of one CTA per SM, each working through a
  // list of items.  An item costs its KV tiles plus kItemCost tiles' worth of
  // fixed work (its first tile's exact maxima, its epilogue, the hand-over to
  // the next item); the items go, costliest first, to the CTA with the least
  // cost so far.  Two candidate item sets are balanced this way: the items as
  // they are, and the items costing more than an SM's share cut into key
  // ranges (at least two tiles each; each writes a partial, merged by a
  // combine entry in a second launch that costs about kCombineCost tiles).
  // The cut is kept only when its balanced makespan plus that is the
  // smaller.  num_sms = 0: one CTA per item, no cut.
  std::vector<Entry> items, combine;
  int32_t n_slots = 0;
  const int64_t cost_total = total + kItemCost * (int64_t)base.size();
  const int64_t share = num_sms > 0 ? (cost_total + num_sms - 1) / num_sms : 0;
  const int64_t target = std::max<int64_t>(2, share - kItemCost);
  for (const Entry& e : base) {
    const int64_t ns =
        num_sms == 0 ? 1 : std::min<int64_t>({64, (e.work + target - 1) / target, e.work / 2});
    if (ns < 2) {
      items.push_back(e);
      continue;
    }
    int32_t lo = 0;
    for (int64_t s2 = 0; s2 < ns; ++s2) {
      const int32_t hi = static_cast<int32_t>((e.work * (s2 + 1)) / ns);
      Entry r = e;
      r.work = hi - lo;
      r.v[4] = lo | (hi << 16);
      r.v[5] = static_cast<int32_t>(combine.size());
      r.v[6] = n_slots + static_cast<int32_t>(s2);
      items.push_back(r);
      lo = hi;
    }
    combine.push_back({0, {n_slots, static_cast<int32_t>(ns), e.v[2], e.v[3], 0, 0, 0, 0}});
    n_slots += static_cast<int32_t>(ns);
  }
  auto by_work = [](const Entry& a, const Entry& b) { return a.work > b.work; };
  if (!combine.empty()) {
    // Makespan (in tiles) of the costliest-first balance over num_sms CTAs.
    auto makespan = [&](std::vector<Entry> its) {
      std::stable_sort(its.begin(), its.end(), by_work);
      std::priority_queue<int64_t, std::vector<int64_t>, std::greater<int64_t>> loads;
      for (int64_t c = 0; c < std::min<int64_t>(num_sms, (int64_t)its.size()); ++c) loads.push(0);
      int64_t worst = 0;
      for (const Entry& e : its) {
        const int64_t l = loads.top() + e.work + kItemCost;
        loads.pop();
        loads.push(l);
        worst = std::max(worst, l);
      }
      return worst;
    };
    if (makespan(items) + kCombineCost >= makespan(base)) {
      items = base;
      combine.clear();
      n_slots = 0;
    }
  }
  std::stable_sort(items.begin(), items.end(), by_work);
  const int64_t n_items = static_cast<int64_t>(items.size());
  if (n_items >= (int64_t(1) << 23)) {
    pkv_set_error("too many verify work items in one launch");
    return PKV_ERR_VALUE;
  }
  // A CTA holds at most kMaxList items: more CTAs than SMs (a second wave)
  // only for batches beyond kMaxList items per SM.
  const int64_t n_ctas = num_sms > 0 ? std::max<int64_t>(std::min<int64_t>(num_sms, n_items),
                                                         (n_items + kMaxList - 1) / kMaxList)
                                     : n_items;
  *n_items_out = n_items;
  *n_ctas_out = n_ctas;
  *n_combine_out = static_cast<int64_t>(combine.size());
  *n_slots_out = n_slots;
  if (!items_out) return PKV_OK;
  if (n_items + (int64_t)combine.size() > items_capacity) {
    pkv_set_error("item buffer too small: need " + std::to_string(n_items + combine.size()) + " records");
    return PKV_ERR_CAPACITY;
  }
  // Costliest first to the least-loaded CTA (with room left).  Record c < n_ctas
  // is CTA c's first item; the CTA's other items follow contiguously from
  // record n_ctas on, and the first item's last field is (their first record
  // << 8) | their count.
  std::vector<std::vector<int64_t>> lists(static_cast<size_t>(n_ctas));
  {
    using Load = std::pair<int64_t, int64_t>;  // (tiles, cta)
    std::priority_queue<Load, std::vector<Load>, std::greater<Load>> heap;
    for (int64_t c = 0; c < n_ctas; ++c) heap.push({0, c});
    for (int64_t k = 0; k < n_items; ++k) {
      Load l = heap.top();
      heap.pop();
      lists[l.second].push_back(k);
      if ((int64_t)lists[l.second].size() < kMaxList) heap.push({l.first + items[k].work + kItemCost, l.second});
    }
  }
  // CTAs with neighbouring indices run on the two SMs of one TPC: the lists,
  // ordered by cost, go heaviest and lightest alternately, so that no pair of
  // neighbours holds two of the heaviest lists.
  {
    std::vector<std::pair<int64_t, int64_t>> by_cost;  // (-cost, list)
    for (int64_t c = 0; c < n_ctas; ++c) {
      int64_t cost = 0;
      for (int64_t k : lists[c]) cost += items[k].work + kItemCost;
      by_cost.push_back({-cost, c});
    }
    std::stable_sort(by_cost.begin(), by_cost.end());
    std::vector<std::vector<int64_t>> mixed(static_cast<size_t>(n_ctas));
    for (int64_t c = 0, lo = 0, hi = n_ctas - 1; lo <= hi; ++c)
      mixed[c] = std::move(lists[by_cost[(c & 1) ? hi-- : lo++].second]);
    lists.swap(mixed);
  }
  int64_t next_rec = n_ctas;
  for (int64_t c = 0; c < n_ctas; ++c) {
    const std::vector<int64_t>& li = lists[c];
    const int64_t cnt = static_cast<int64_t>(li.size()) - 1;
    for (size_t k = 0; k < li.size(); ++k) {
      Entry e = items[li[k]];
      e.v[7] = k == 0 ? static_cast<int32_t>((cnt > 0 ? next_rec : 0) << 8 | cnt) : -1;
      std::copy(e.v, e.v + 8, items_out + 8 * (k == 0 ? c : next_rec + (int64_t)k - 1));
    }
    next_rec += cnt;
  }
  int32_t* o = items_out + 8 * n_items;
  for (const Entry& e : combine) o = std::copy(e.v, e.v + 8, o);
  return PKV_OK;
}

extern "C" int32_t pkv_verify_attention(const pkv_pool_geom* g, const void* pool, int32_t layer, const void* q,
                                        const int32_t* block_tables, int32_t table_stride, int32_t table_rows,
                                        const int32_t* work_items, int32_t n_items, int32_t n_ctas,
                                        int32_t n_combine, int64_t total_q, int32_t num_q_heads, float scale,
                                        void* out,
                                        int32_t* error_word, void* workspace, int64_t workspace_bytes,
                                        int64_t n_slots, void* stream) {
  pkv_clear_error();
  if (!g || g->block_size != kPageRows || g->head_dim != kVD) {
    pkv_set_error("paged verify attention needs block_size 16 and head_dim 128");
    return PKV_ERR_UNSUPPORTED;
  }
  if (g->dtype != PKV_BF16 && g->dtype != PKV_F16) {
    pkv_set_error("paged verify attention supports bf16 and f16 pools");
    return PKV_ERR_UNSUPPORTED;
  }
  if (pkv_verify_positions_per_item(num_q_heads, g->num_kv_heads) <= 0 || g->num_kv_heads > 0x7fff) {
    pkv_set_error("num_q_heads must be a positive multiple of num_kv_heads with at most 32 query heads per KV head");
    return PKV_ERR_UNSUPPORTED;
  }
  if (layer < 0 || layer >= g->num_layers || n_items < 0 || n_combine < 0 || n_slots < 0 || n_slots > INT32_MAX ||
      total_q < 0 || table_stride <= 0 || table_rows <= 0 || !(scale > 0.f) ||
      (n_items > 0 && (n_ctas < 1 || n_ctas > n_items))) {
    pkv_set_error("invalid layer, item, CTA, combine, query, table or scale arguments");
    return PKV_ERR_ARG;
  }
  if ((n_combine > 0 || n_slots > 0) &&
      (!workspace || (uintptr_t)workspace % 16 != 0 ||
       workspace_bytes < pkv_prefill_workspace_bytes(n_slots, g->head_dim))) {
    pkv_set_error("workspace too small or misaligned: need " +
                  std::to_string(pkv_prefill_workspace_bytes(n_slots, g->head_dim)) + " bytes, 16-byte aligned");
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
  prm.partials = static_cast<float*>(workspace);
  prm.n_slots = static_cast<int32_t>(n_slots);
  prm.total_q = total_q;
  prm.n_items = n_items;
  prm.table_stride = table_stride;
  prm.table_rows = table_rows;
  prm.hq = num_q_heads;
  prm.hkv = static_cast<int32_t>(g->num_kv_heads);
  prm.group = num_q_heads / static_cast<int32_t>(g->num_kv_heads);
  prm.ppi = kCols / prm.group;
  prm.layer = layer;
  prm.num_blocks = static_cast<int32_t>(g->num_blocks);
  prm.scale_log2 = scale * kLog2e;
  prm.n_combine = n_combine;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const cudaError_t err = g->dtype == PKV_BF16 ? launch_verify<__nv_bfloat16>(prm, n_ctas, n_combine, s)
                                               : launch_verify<__half>(prm, n_ctas, n_combine, s);
  if (err != cudaSuccess) {
    pkv_set_error(std::string("verify launch failed: ") + cudaGetErrorString(err));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}
