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
// Tiles: a CTA owns one work item = (sequence, KV head, up to 2 x 128/G chunk
// positions).  The G = Hq/Hkv query heads of a position are packed into the
// rows of a 128-row tcgen05 tile (row = position * G + head), and the item's
// positions fill two such query tiles, A and B, that share every K/V tile the
// CTA loads: the KV head's pages are read once for 2 x 128 query rows.  Keys
// stream in tiles of 128 (8 pages).  Roles (320 threads):
//   warp 8      producer: per KV tile, 2 KB cp.async.bulk copies of every
//               page's 64-dim K (then V) slabs into separate K and V rings
//               (the pool's pages are pre-swizzled, so the slabs land directly
//               in the 128-byte-swizzled canonical operand layouts; no tensor
//               map, no multicast);
//   warp 9      allocates all 512 tensor-memory columns (S_A, S_B, O_A, O_B);
//               lane 0 issues S_X = Q_X K_j^T (M=128, N=128, both operands
//               K-major in shared memory) and O_X += P_X V_j with P_X read
//               from tensor memory (it overwrites S_X in place) and V
//               MN-major in shared memory, in the order S_A(j), P_B V(j-1),
//               S_B(j), P_A V(j), so the tensor cores work on one tile while
//               the other tile's softmax runs;
//   warps 0-3   softmax of tile A, warps 4-7 of tile B (thread = tile row):
//               Q load (swizzled into shared memory), one 128-column
//               tcgen05.ld of S per KV tile, online softmax in base 2 with a
//               lazily kept row maximum (O is rescaled in tensor memory only
//               when the maximum grows by more than 2^8), P stored back into
//               tensor memory as packed 16-bit pairs, and the epilogue O / l.
// Completion of S_X(j) also implies completion of P_X V(j-1) (MMAs complete
// in issue order), so the O rescale needs no separate wait.
//
// Every mbarrier wait is bounded; a timed-out role records an error word and
// skips the rest of its work, the MMA thread waits (bounded) for its last
// MMAs and the producer for its copies before tensor memory is freed.
#include "pkv_device.cuh"
#include "pkv_error.h"
#include "pkv_prefill.cuh"

#include <algorithm>
#include <string>
#include <type_traits>
#include <vector>

namespace pkv {
namespace {

constexpr int kProducerWarp = 8;
constexpr int kMmaWarp = 9;
constexpr int kThreads = 320;
constexpr int kTileThreads = 128;      // softmax threads per query tile
constexpr int kTmemCols = 512;         // S_A, S_B (kKeys each), O_A, O_B (head_dim each)
#ifndef PKV_PREFILL_POLY_PAIRS
#define PKV_PREFILL_POLY_PAIRS 0       // of every 8 probability pairs, those whose 2^x runs on the FMA pipes
#endif

template <int D>
struct PCfg {
  static constexpr int kSlabs = D / 64;                    // 64-dim (128-byte) slabs per row
  static constexpr int kQSlabBytes = kRows * 128;
  static constexpr int kQBytes = kSlabs * kQSlabBytes;     // one query tile
  static constexpr int kKVSlabBytes = kKeys * 128;         // one slab of a KV tile
  static constexpr int kTileBytes = kSlabs * kKVSlabBytes; // K (or V) of one KV tile
  static constexpr int kKStages = D == 128 ? 3 : 4;
  static constexpr int kVStages = D == 128 ? 2 : 4;
  static constexpr int kOffK = 2 * kQBytes;
  static constexpr int kOffV = kOffK + kKStages * kTileBytes;
  static constexpr int kOffBar = kOffV + kVStages * kTileBytes;
  static constexpr int kSmemBytes = kOffBar + 256 + 1024;  // + barriers, + alignment slack
  static constexpr uint32_t kPageSlabBytes = kPageRows * 128;
};

template <int NK, int NV>
struct Bars {
  uint64_t q_full[2];    // 128 Q-writer arrivals per query tile
  uint64_t k_full[NK];   // producer expect_tx + bulk-copy bytes
  uint64_t k_empty[NK];  // MMA commit after the tile's last S MMA
  uint64_t v_full[NV];
  uint64_t v_empty[NV];  // MMA commit after the tile's last P.V MMA
  uint64_t s_full[2];    // MMA commit after S_X(j)
  uint64_t p_full[2];    // 128 softmax arrivals: P_X(j) stored, O_X rescaled
  uint64_t o_done[2];    // MMA commit after the last P_X V MMA
  uint64_t mma_done;     // final commit of the MMA thread
  uint32_t tmem_base;
  int32_t abort;
};

template <int D, typename T, int kPoly>
__global__ void __launch_bounds__(kThreads, 1) paged_prefill_kernel(const __grid_constant__ PrefillParams p) {
  using C = PCfg<D>;
  constexpr int NK = C::kKStages, NV = C::kVStages;
  constexpr uint32_t kAbFormat = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
  constexpr uint32_t kIdescS = umma_idesc_f16(kAbFormat, 0, 0, kRows, kKeys);
  constexpr uint32_t kIdescO = umma_idesc_f16(kAbFormat, 0, 1, kRows, D);

  extern __shared__ uint8_t smem_raw[];
  const uint32_t raw_s = smem_u32(smem_raw);
  uint8_t* smem = smem_raw + ((1024u - (raw_s & 1023u)) & 1023u);
  uint8_t* q_s = smem;
  uint8_t* k_s = smem + C::kOffK;
  uint8_t* v_s = smem + C::kOffV;
  Bars<NK, NV>* bars = reinterpret_cast<Bars<NK, NV>*>(smem + C::kOffBar);
  volatile int32_t* abort = &bars->abort;

  const int tid = threadIdx.x;
  const int warp = tid >> 5;
  const int lane = tid & 31;

  const int4 item = p.items[2 * blockIdx.x];
  const int4 ext = p.items[2 * blockIdx.x + 1];
  const int row = item.x, pos0 = item.y, qrow0 = item.z, h = item.w >> 16, nt = item.w & 0xffff;
  const int group = p.group, ppi = p.ppi;
  const int kv_len = pos0 + nt;  // keys the item's last query sees
  const int n_tiles = (kv_len + kKeys - 1) / kKeys;    // KV tiles of the whole key range
  const int kt_lo = ext.x, kt_hi = ext.y > 0 ? ext.y : n_tiles, slot = ext.z;
  const bool ranged = kt_lo != 0 || kt_hi != n_tiles || slot >= 0;  // a key range of a one-tile item
  const bool ok = row >= 0 && row < p.table_rows && h >= 0 && h < p.hkv && nt >= 1 && nt <= 2 * ppi &&
                  ppi * group <= kRows && pos0 >= 0 && qrow0 >= 0 && (int64_t)qrow0 + nt <= p.total_q &&
                  (kv_len + kPageRows - 1) / kPageRows <= p.table_stride && kt_lo >= 0 && kt_lo < kt_hi &&
                  kt_hi <= n_tiles && slot >= -1 && slot < p.n_slots && (!ranged || nt <= ppi);
  if (!ok) {  // uniform across the CTA: nothing initialised yet
    if (tid == 0) atomicExch(p.error, kDevBadItem);
    return;
  }
  const int n_range = kt_hi - kt_lo;
  // Two modes.  Shared: tile A holds the first ppi positions, tile B the rest,
  // and both read KV tile j at step j (one load serves both).  Split (all
  // positions fit tile A and the CTA's key range has >= 2 KV tiles): tile B
  // takes the same queries over the second half of the range, each half
  // streams its own K/V, and the two partial softmaxes are merged at the end.
  const bool split = nt <= ppi && n_range >= 2;
  const int nt_a = min(nt, ppi);
  const int n_a = split ? (n_range + 1) / 2
                        : (ranged ? n_range : (pos0 + nt_a + kKeys - 1) / kKeys);  // KV tiles of tile A
  const int n_b = split ? n_range - n_a : (nt > ppi ? n_tiles : 0);              // KV tiles of tile B
  const int a_tile0 = kt_lo;                                                       // A's first KV tile
  const int b_tile0 = split ? kt_lo + n_a : 0;                                     // B's first KV tile
  const int n_steps = max(n_a, n_b);
  const bool two_q = n_b > 0 && !split;  // tile B has queries of its own
  // Index of tile x's step-j K (or V) tile in the order the MMAs consume them:
  // shared mode one per step; split mode A(0), B(0), A(1), B(1), ... then A's rest.
  auto use_idx = [&](int x, int j) { return split ? (x == 0 ? j + min(j, n_b) : 2 * j + 1) : j; };
  const int n_loads = split ? n_a + n_b : n_steps;
  auto load_tile = [&](int c) {  // KV tile of load c
    if (!split) return a_tile0 + c;
    return c < 2 * n_b ? ((c & 1) ? b_tile0 + (c >> 1) : a_tile0 + (c >> 1)) : a_tile0 + c - n_b;
  };

  if (tid == 0) {
    for (int x = 0; x < 2; ++x) {
      mbar_init(&bars->q_full[x], kTileThreads);
      mbar_init(&bars->s_full[x], 1);
      mbar_init(&bars->p_full[x], kTileThreads);
      mbar_init(&bars->o_done[x], 1);
    }
    for (int i = 0; i < NK; ++i) {
      mbar_init(&bars->k_full[i], 1);
      mbar_init(&bars->k_empty[i], 1);
    }
    for (int i = 0; i < NV; ++i) {
      mbar_init(&bars->v_full[i], 1);
      mbar_init(&bars->v_empty[i], 1);
    }
    mbar_init(&bars->mma_done, 1);
    bars->abort = 0;
    fence_barrier_init();
  }
  if (warp == kMmaWarp) tmem_alloc(&bars->tmem_base, kTmemCols);
  tc_fence_before_sync();
  __syncthreads();
  tc_fence_after_sync();
  const uint32_t tmem = bars->tmem_base;

  if (warp == kProducerWarp) {
    // ---------------- producer ----------------
    const int32_t* trow = p.tables + (int64_t)row * p.table_stride;
    // K (state 0) or V (state 1) pages of KV tile t into one ring stage.
    auto issue = [&](int state, int t, uint8_t* stage, uint64_t* full) {
      const int key0 = t * kKeys;
      const int pages = min(kPagesPerTile, (kv_len - key0 + kPageRows - 1) / kPageRows);
      const int copies = pages * C::kSlabs;
      if (lane == 0) mbar_arrive_expect_tx(full, copies * C::kPageSlabBytes);
      __syncwarp();
      for (int c = lane; c < copies; c += 32) {
        const int pg = c / C::kSlabs, slab = c % C::kSlabs;
        int blk = __ldg(trow + key0 / kPageRows + pg);
        if (blk < 0 || blk >= p.num_blocks) {
          atomicExch(p.error, kDevBadBlock);
          blk = 0;
        }
        const char* src = p.pool + page_offset(p.layer, blk, h, state, p.num_blocks, p.hkv, kPageRows, D * 2) +
                          slab * C::kPageSlabBytes;
        bulk_copy_g2s(stage + slab * C::kKVSlabBytes + pg * C::kPageSlabBytes, src, C::kPageSlabBytes, full);
      }
    };
    int k_issued = 0, v_issued = 0;
    // K runs one load ahead of V: S(j) needs its K before P V(j-1) needs its V.
    for (int s = 0; s <= n_loads; ++s) {
      if (s < n_loads) {
        const int st = s % NK;
        if (s >= NK &&
            !__all_sync(0xffffffffu, wait_or_abort(&bars->k_empty[st], ((s / NK) - 1) & 1, p, abort)))
          break;
        issue(0, load_tile(s), k_s + st * C::kTileBytes, &bars->k_full[st]);
        k_issued = s + 1;
      }
      if (s >= 1) {
        const int c = s - 1, st = c % NV;
        if (c >= NV && !__all_sync(0xffffffffu, wait_or_abort(&bars->v_empty[st], ((c / NV) - 1) & 1, p, abort)))
          break;
        issue(1, load_tile(c), v_s + st * C::kTileBytes, &bars->v_full[st]);
        v_issued = c + 1;
      }
    }
    // Copies still in flight must land before the CTA frees its memory.
    if (lane == 0) {
      for (int c = max(0, k_issued - NK); c < k_issued; ++c) mbar_wait_bounded(&bars->k_full[c % NK], (c / NK) & 1);
      for (int c = max(0, v_issued - NV); c < v_issued; ++c) mbar_wait_bounded(&bars->v_full[c % NV], (c / NV) & 1);
    }
  } else if (warp == kMmaWarp) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t q_addr = smem_u32(q_s);
      const uint32_t k_addr = smem_u32(k_s);
      const uint32_t v_addr = smem_u32(v_s);
      // S_x(j) = Q K^T; in split mode both tiles use tile A's queries.
      auto s_mma = [&](int x, int j) -> bool {
        const int c = use_idx(x, j), kst = c % NK;
        if (!wait_or_abort(&bars->k_full[kst], (c / NK) & 1, p, abort)) return false;
        tc_fence_after_sync();
        const uint32_t qb = q_addr + (two_q ? x : 0) * C::kQBytes;
        const uint32_t kb = k_addr + kst * C::kTileBytes;
#pragma unroll
        for (int ks = 0; ks < D / 16; ++ks) {
          const uint32_t off = (ks >> 2) * C::kQSlabBytes + (ks & 3) * 32;
          const uint64_t adesc = umma_desc_sw128(qb + off, 16, 1024);
          const uint64_t bdesc = umma_desc_sw128(kb + (ks >> 2) * C::kKVSlabBytes + (ks & 3) * 32, 16, 1024);
          umma_f16_ss(tmem + x * kKeys, adesc, bdesc, kIdescS, ks > 0 ? 1u : 0u);
        }
        umma_commit(&bars->s_full[x]);
        // The K tile is free once every S that reads it is issued before this commit.
        if (split || x == 1 || n_b == 0) umma_commit(&bars->k_empty[kst]);
        return true;
      };
      auto pv_mma = [&](int x, int j) -> bool {
        const int c = use_idx(x, j), vst = c % NV;
        if (!wait_or_abort(&bars->p_full[x], j & 1, p, abort)) return false;
        if (!wait_or_abort(&bars->v_full[vst], (c / NV) & 1, p, abort)) return false;
        tc_fence_after_sync();
        const int t = x == 0 ? a_tile0 + j : b_tile0 + j;
        const int steps = (min(kKeys, kv_len - t * kKeys) + 15) / 16;
        const uint32_t vb = v_addr + vst * C::kTileBytes;
        for (int ks = 0; ks < steps; ++ks) {
          const uint64_t bdesc = umma_desc_sw128(vb + ks * 2048, C::kKVSlabBytes, 1024);
          umma_f16_ts(tmem + 2 * kKeys + x * D, tmem + x * kKeys + ks * 8, bdesc, kIdescO,
                      (j > 0 || ks > 0) ? 1u : 0u);
        }
        if (split || x == 1 || n_b == 0) umma_commit(&bars->v_empty[vst]);
        if (j == (x == 0 ? n_a : n_b) - 1) umma_commit(&bars->o_done[x]);
        return true;
      };
      bool alive = wait_or_abort(&bars->q_full[0], 0, p, abort);
      if (alive && two_q) alive = wait_or_abort(&bars->q_full[1], 0, p, abort);
      // Order per step: S_A(j), P_B V(j-1), S_B(j), P_A V(j): the tensor pipe
      // runs one tile's products while the other tile's softmax works.
      for (int j = 0; alive && j < n_steps; ++j) {
        if (j < n_a && !s_mma(0, j)) alive = false;
        if (alive && j > 0 && j - 1 < n_b && !pv_mma(1, j - 1)) alive = false;
        if (alive && j < n_b && !s_mma(1, j)) alive = false;
        if (alive && j < n_a && !pv_mma(0, j)) alive = false;
      }
      if (alive && n_b == n_steps && n_b > 0) pv_mma(1, n_b - 1);
      // Every MMA issued must complete before tensor memory is freed.
      umma_commit(&bars->mma_done);
      mbar_wait_bounded(&bars->mma_done, 0);
    }
    __syncwarp();
  } else {
    // ---------------- softmax / epilogue: tile x, thread = tile row ----------------
    const int x = warp >> 2;
    const int r = tid & (kTileThreads - 1);
    const int nt_x = (split || x == 0) ? nt_a : nt - nt_a;
    const int n_x = x == 0 ? n_a : n_b;
    const int row_block = split ? 0 : x;                         // which positions the tile's rows hold
    const int rows_valid = nt_x * group;
    const int pos_first = pos0 + row_block * ppi;                // tile's first position
    const int pos_r = pos_first + min(r / group, nt_x - 1);      // padding rows repeat the last position
    const int64_t qrow = (int64_t)qrow0 + row_block * ppi + r / group;  // this row's query
    const uint32_t lane_base = static_cast<uint32_t>((warp & 3) * 32) << 16;
    const uint32_t s_addr = tmem + lane_base + x * kKeys;
    const uint32_t o_addr = tmem + lane_base + 2 * kKeys + x * D;
    float m_run = -INFINITY, l_run = 0.f;
    bool alive = true;
    if (n_x > 0) {
      if (x == 0 || two_q) {
        const T* src = static_cast<const T*>(p.q) + (qrow * p.hq + (int64_t)h * group + r % group) * D;
        uint8_t* qt = q_s + x * C::kQBytes;
        const bool in = r < rows_valid;
#pragma unroll
        for (int c = 0; c < D / 8; ++c) {
          uint4 v = make_uint4(0, 0, 0, 0);
          if (in) v = __ldg(reinterpret_cast<const uint4*>(src) + c);
          *reinterpret_cast<uint4*>(qt + (c >> 3) * C::kQSlabBytes + swz128(r, c & 7)) = v;
        }
        fence_proxy_async_smem();
        mbar_arrive(&bars->q_full[x]);
      }
      const float sl2 = p.scale_log2;
      for (int j = 0; j < n_x; ++j) {
        if (!__all_sync(0xffffffffu, wait_or_abort(&bars->s_full[x], j & 1, p, abort))) {
          alive = false;
          break;
        }
        tc_fence_after_sync();
        const int t = x == 0 ? a_tile0 + j : b_tile0 + j;  // KV tile
        const int key0 = t * kKeys;
        const bool masked = key0 + kKeys - 1 > pos_first;  // crosses the causal diagonal of this tile
        const int lim = pos_r - key0;                      // visible columns: c <= lim
        // Pass 1: row maximum of the visible keys (one 128-column read).
        float m4[4] = {-INFINITY, -INFINITY, -INFINITY, -INFINITY};
        {
          uint32_t sr[128];
          tmem_ld128(s_addr, sr);
          if (masked) {
#pragma unroll
            for (int c = 0; c < kKeys; c += 2)
              m4[(c >> 1) & 3] = fmax3(m4[(c >> 1) & 3], c <= lim ? __uint_as_float(sr[c]) : -INFINITY,
                                       c + 1 <= lim ? __uint_as_float(sr[c + 1]) : -INFINITY);
          } else {
#pragma unroll
            for (int c = 0; c < kKeys; c += 2)
              m4[(c >> 1) & 3] = fmax3(m4[(c >> 1) & 3], __uint_as_float(sr[c]), __uint_as_float(sr[c + 1]));
          }
        }
        const float mx = fmax3(m4[0], m4[1], fmaxf(m4[2], m4[3])) * sl2;
        float alpha = 1.f;
        bool rescale = false;
        if (mx > m_run + kRescaleLog2) {
          alpha = ex2_approx(m_run - mx);
          l_run *= alpha;
          m_run = mx;
          rescale = j > 0;
        }
        // Pass 2, per 32 columns: P = 2^(S * scale * log2e - m) for visible
        // keys, 0 elsewhere, packed 16-bit pairs over the first 64 columns of
        // S (each part is read before its pairs land on columns already read;
        // re-reading S keeps the register peak low).  kPoly of every 8 pairs
        // take 2^x from the FMA pipes, the rest from the multi-function unit.
        const float2 sc2 = make_float2(sl2, sl2), nm2 = make_float2(-m_run, -m_run);
        float2 l2[2] = {make_float2(0.f, 0.f), make_float2(0.f, 0.f)};
#pragma unroll
        for (int part = 0; part < kKeys / 32; ++part) {
          uint32_t sr[32];
          tmem_ld32_bits(s_addr + part * 32, sr);
          uint32_t pk[16];
#pragma unroll
          for (int i = 0; i < 16; ++i) {
            const int c = part * 32 + 2 * i;
            const float2 xv = fma2(make_float2(__uint_as_float(sr[2 * i]), __uint_as_float(sr[2 * i + 1])), sc2, nm2);
            float2 pv;
            if ((i & 7) < kPoly) {
              pv = exp2_poly2(xv);
            } else {
              pv = make_float2(ex2_approx(xv.x), ex2_approx(xv.y));
            }
            if (masked) {
              pv.x = c <= lim ? pv.x : 0.f;
              pv.y = c + 1 <= lim ? pv.y : 0.f;
            }
            l2[i & 1] = add2(l2[i & 1], pv);
            pk[i] = MmaOp<T>::pack(pv.x, pv.y);
          }
          tmem_st16_nowait(s_addr + part * 16, pk);
        }
        l_run += (l2[0].x + l2[0].y) + (l2[1].x + l2[1].y);
        // The item's last KV tile: V rows past the sequence inside its last
        // page are zeroed (by the tile whose product reads it first) so that
        // their zero probabilities multiply finite values.
        const bool zero_owner = split || n_b == 0 || ((x == 0) == (n_a == n_tiles));
        if (zero_owner && t == n_tiles - 1 && (kv_len & (kPageRows - 1)) != 0) {
          const int c = use_idx(x, j);
          if (!__all_sync(0xffffffffu, wait_or_abort(&bars->v_full[c % NV], (c / NV) & 1, p, abort))) {
            alive = false;
            break;
          }
          const int first = kv_len - key0;                       // first stale row of the tile
          const int last = (first + kPageRows - 1) & ~(kPageRows - 1);
          uint8_t* vb = v_s + (c % NV) * C::kTileBytes;
          for (int e = r; e < (last - first) * 8 * C::kSlabs; e += kTileThreads) {
            const int slab = e / ((last - first) * 8);
            const int rem = e % ((last - first) * 8);
            *reinterpret_cast<uint4*>(vb + slab * C::kKVSlabBytes + swz128(first + rem / 8, rem & 7)) =
                make_uint4(0, 0, 0, 0);
          }
          fence_proxy_async_smem();
        }
        // O *= alpha for rows whose maximum moved; P V(j-1) completed before S(j).
        if (__any_sync(0xffffffffu, rescale)) {
#pragma unroll 1
          for (int cc = 0; cc < D / 32; ++cc) {
            float v[32];
            tmem_ld32(o_addr + cc * 32, v);
#pragma unroll
            for (int i = 0; i < 32; ++i) v[i] *= alpha;
            tmem_st32(o_addr + cc * 32, v);
          }
        }
        tmem_wait_st();
        tc_fence_before_sync();
        mbar_arrive(&bars->p_full[x]);
      }
    }
    // Epilogue.  Split mode: tile B hands its row maximum and sum to tile A
    // through shared memory (tile B's unused query buffer), and tile A merges
    // the two partial results: O = (O_A 2^(m_A-m) + O_B 2^(m_B-m)) / (l_A
    // 2^(m_A-m) + l_B 2^(m_B-m)), m = max(m_A, m_B).
    float* xchg = reinterpret_cast<float*>(q_s + C::kQBytes);
    if (split) {
      if (x == 1) {
        xchg[r] = m_run;
        xchg[kTileThreads + r] = l_run;
      }
      asm volatile("bar.sync 1, 256;" ::: "memory");  // the 8 softmax warps, once, on every path
    }
    if (x == 0 || two_q) {
      bool done = alive && __all_sync(0xffffffffu, wait_or_abort(&bars->o_done[x], 0, p, abort));
      if (split) done = done && __all_sync(0xffffffffu, wait_or_abort(&bars->o_done[1], 0, p, abort));
      if (done) {
        tc_fence_after_sync();
        // Merge weights: 2^(m_x - m) per tile, m = the larger row maximum
        // (rows that saw no key in a key range have m_x = -inf, weight 0).
        float m_b = -INFINITY, l_b = 0.f;
        if (split) {
          m_b = xchg[r];
          l_b = xchg[kTileThreads + r];
        }
        const float m = fmaxf(m_run, m_b);
        const float wa = m == -INFINITY ? 0.f : ex2_approx(m_run - m);
        const float wb = (split && m != -INFINITY) ? ex2_approx(m_b - m) : 0.f;
        const float l = l_run * wa + l_b * wb;
        if (slot >= 0) {
          // Unnormalised partial of this key range: m, l and O in fp32.
          float* part = p.partials + (int64_t)slot * (2 * kRows + kRows * D);
          if (r < rows_valid) {
            part[r] = m;
            part[kRows + r] = l;
          }
          float* orow = part + 2 * kRows + (int64_t)r * D;
#pragma unroll 1
          for (int cc = 0; cc < D / 32; ++cc) {
            float v[32];
            tmem_ld32(o_addr + cc * 32, v);
            if (split) {
              float vb[32];
              tmem_ld32(o_addr + D + cc * 32, vb);  // O_B, same lanes
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = v[i] * wa + vb[i] * wb;
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] *= wa;
            }
            if (r < rows_valid) {
#pragma unroll
              for (int c = 0; c < 8; ++c)
                reinterpret_cast<float4*>(orow + cc * 32)[c] =
                    make_float4(v[4 * c], v[4 * c + 1], v[4 * c + 2], v[4 * c + 3]);
            }
          }
        } else {
          const float inv_l = 1.f / l;
          const float sa = wa * inv_l, sb = wb * inv_l;
          T* dst = static_cast<T*>(p.out) + (qrow * p.hq + (int64_t)h * group + r % group) * D;
#pragma unroll 1
          for (int cc = 0; cc < D / 32; ++cc) {
            float v[32];
            tmem_ld32(o_addr + cc * 32, v);
            if (split) {
              float vb[32];
              tmem_ld32(o_addr + D + cc * 32, vb);  // O_B, same lanes
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] = v[i] * sa + vb[i] * sb;
            } else {
#pragma unroll
              for (int i = 0; i < 32; ++i) v[i] *= sa;
            }
            uint32_t pk[16];
#pragma unroll
            for (int i = 0; i < 32; i += 2) pk[i >> 1] = MmaOp<T>::pack(v[i], v[i + 1]);
            if (r < rows_valid) {
#pragma unroll
              for (int c = 0; c < 4; ++c)
                reinterpret_cast<uint4*>(dst + cc * 32)[c] =
                    make_uint4(pk[4 * c], pk[4 * c + 1], pk[4 * c + 2], pk[4 * c + 3]);
            }
          }
        }
      }
    }
  }

  tc_fence_before_sync();
  __syncthreads();
  if (warp == kMmaWarp) {
    tc_fence_after_sync();
    tmem_dealloc(tmem, kTmemCols);
  }
}

template <int D, typename T>
cudaError_t launch_prefill(const PrefillParams& prm, int32_t n_combine, cudaStream_t stream) {
  using C = PCfg<D>;
  static_assert(C::kSmemBytes <= 232448, "prefill tile exceeds the shared memory of one CTA");
  static_assert(sizeof(Bars<C::kKStages, C::kVStages>) <= 256, "barrier block overflows its slot");
  auto kern = paged_prefill_kernel<D, T, PKV_PREFILL_POLY_PAIRS>;
  cudaError_t err = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, C::kSmemBytes);
  if (err != cudaSuccess) return err;
  kern<<<prm.n_items, kThreads, C::kSmemBytes, stream>>>(prm);
  err = cudaGetLastError();
  if (err != cudaSuccess || n_combine == 0) return err;
  paged_prefill_combine_kernel<D, T><<<n_combine, kRows, 0, stream>>>(prm, prm.items + 2 * prm.n_items);
  return cudaGetLastError();
}

}  // namespace
}  // namespace pkv


using namespace pkv;

extern "C" int32_t pkv_prefill_positions_per_item(int32_t num_q_heads, int32_t num_kv_heads) {
  if (num_kv_heads <= 0 || num_q_heads <= 0 || num_q_heads % num_kv_heads != 0) return 0;
  const int group = num_q_heads / num_kv_heads;
  return group > kRows ? 0 : 2 * (kRows / group);  // two query tiles of kRows / group positions
}

extern "C" int64_t pkv_prefill_workspace_bytes(int64_t n_slots, int32_t head_dim) {
  if (n_slots <= 0) return 0;
  return n_slots * (int64_t)(2 * kRows + kRows * head_dim) * (int64_t)sizeof(float);
}

extern "C" int32_t pkv_prefill_plan(const int32_t* rows, const int32_t* past_lens, const int32_t* q_lens,
                                    int32_t n_seqs, int32_t num_q_heads, int32_t num_kv_heads, int32_t num_sms,
                                    int32_t split_waves, int32_t* items_out, int64_t items_capacity,
                                    int64_t* n_items_out, int64_t* n_combine_out, int64_t* n_slots_out) {
  pkv_clear_error();
  const int ppi = pkv_prefill_positions_per_item(num_q_heads, num_kv_heads);  // two query tiles
  if (ppi <= 0 || num_kv_heads > 0x7fff) {
    pkv_set_error("num_q_heads must be a positive multiple of num_kv_heads with at most 128 query heads per KV head");
    return PKV_ERR_UNSUPPORTED;
  }
  if (n_seqs < 0 || num_sms < 0 || split_waves < 0 || !n_items_out || !n_combine_out || !n_slots_out ||
      (n_seqs > 0 && (!rows || !past_lens || !q_lens))) {
    pkv_set_error("invalid plan arguments");
    return PKV_ERR_ARG;
  }
  const int tile_positions = ppi / 2;
  struct Entry {
    int64_t work;  // KV tiles the CTA streams
    int32_t v[8];
  };
  std::vector<Entry> base;
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
      const int64_t kv_len = (int64_t)past_lens[i] + t0 + n;
      for (int32_t hk = 0; hk < num_kv_heads; ++hk)
        base.push_back({(kv_len + kKeys - 1) / kKeys,
                        {rows[i], past_lens[i] + t0, static_cast<int32_t>(qrow + t0), (hk << 16) | n, 0, 0, -1, 0}});
    }
    qrow += q_lens[i];
  }
  // Few items (a verify step): cut the keys of one-tile items into ranges of
  // about `target` KV tiles so that about split_waves CTAs per SM share the
  // work; each range writes a partial and a combine entry merges them.
  std::vector<Entry> items, combine;
  int32_t n_slots = 0;
  const int64_t slots_wanted = (int64_t)split_waves * num_sms;
  if (split_waves > 0 && num_sms > 0 && (int64_t)base.size() < slots_wanted) {
    int64_t total = 0;
    for (const Entry& e : base) total += e.work;
    const int64_t target = std::max<int64_t>(2, (total + slots_wanted - 1) / slots_wanted);
    for (const Entry& e : base) {
      const int32_t nt = e.v[3] & 0xffff;
      const int64_t ns = std::min<int64_t>(64, (e.work + target - 1) / target);
      if (nt > tile_positions || ns < 2) {
        items.push_back(e);
        continue;
      }
      int32_t lo = 0;
      for (int64_t s2 = 0; s2 < ns; ++s2) {
        const int32_t hi = static_cast<int32_t>((e.work * (s2 + 1)) / ns);
        Entry r = e;
        r.work = hi - lo;
        r.v[4] = lo;
        r.v[5] = hi;
        r.v[6] = n_slots + static_cast<int32_t>(s2);
        items.push_back(r);
        lo = hi;
      }
      combine.push_back({0, {n_slots, static_cast<int32_t>(ns), e.v[2], e.v[3], 0, 0, 0, 0}});
      n_slots += static_cast<int32_t>(ns);
    }
  } else {
    items = std::move(base);
  }
  *n_items_out = static_cast<int64_t>(items.size());
  *n_combine_out = static_cast<int64_t>(combine.size());
  *n_slots_out = n_slots;
  if (!items_out) return PKV_OK;
  if ((int64_t)(items.size() + combine.size()) > items_capacity) {
    pkv_set_error("item buffer too small: need " + std::to_string(items.size() + combine.size()) + " records");
    return PKV_ERR_CAPACITY;
  }
  // Longest key range first, so the grid's tail holds the short ones.
  std::stable_sort(items.begin(), items.end(), [](const Entry& a, const Entry& b) { return a.work > b.work; });
  int32_t* o = items_out;
  for (const Entry& e : items) o = std::copy(e.v, e.v + 8, o);
  for (const Entry& e : combine) o = std::copy(e.v, e.v + 8, o);
  return PKV_OK;
}

extern "C" int32_t pkv_prefill_attention(const pkv_pool_geom* g, const void* pool, int32_t layer, const void* q,
                                         const int32_t* block_tables, int32_t table_stride, int32_t table_rows,
                                         const int32_t* work_items, int32_t n_items, int32_t n_combine,
                                         int64_t total_q, int32_t num_q_heads, float scale, void* out,
                                         int32_t* error_word, void* workspace, int64_t workspace_bytes,
                                         int64_t n_slots, void* stream) {
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
  if (layer < 0 || layer >= g->num_layers || n_items < 0 || n_combine < 0 || n_slots < 0 || n_slots > INT32_MAX ||
      total_q < 0 || table_stride <= 0 || table_rows <= 0 || !(scale > 0.f)) {
    pkv_set_error("invalid layer, item, combine, query, table or scale arguments");
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
  prm.ppi = kRows / prm.group;
  prm.layer = layer;
  prm.num_blocks = static_cast<int32_t>(g->num_blocks);
  prm.scale_log2 = scale * kLog2e;
  prm.n_combine = n_combine;
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  cudaError_t err;
  if (g->head_dim == 128)
    err = g->dtype == PKV_BF16 ? launch_prefill<128, __nv_bfloat16>(prm, n_combine, s) : launch_prefill<128, __half>(prm, n_combine, s);
  else
    err = g->dtype == PKV_BF16 ? launch_prefill<64, __nv_bfloat16>(prm, n_combine, s) : launch_prefill<64, __half>(prm, n_combine, s);
  if (err != cudaSuccess) {
    pkv_set_error(std::string("prefill launch failed: ") + cudaGetErrorString(err));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}
