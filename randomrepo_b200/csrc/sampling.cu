// Token selection, token log-probabilities and speculative accept / reject
// over fp32 logits, for sm_100a.
//
// Replaces the per-token vocabulary work around AgentRL's rollouts:
//  * the old-policy pass's log_softmax + gather over the vocabulary
//    (agentrl/core/rollout.py:456-472), applied to rows of logits the
//    rollout already has instead of a second full forward;
//  * next-token selection (rollout.py:307-315): argmax, or a draw from
//    softmax(logits / temperature);
//  * the speculative verify's accept / reject, correction draw and bonus draw
//    (agentrl/generation/speculative.py:217-274), for a whole batch at once.
//
// All of it streams rows of `vocab` fp32 logits (151 936 for Qwen2: 594 KB a
// row) from HBM once.  Each CTA streams a span of one row with kUnroll
// float4 loads in flight per thread (coalesced, evict-first), folding them
// into per-thread state, then reduces the state across the CTA.  The host
// cuts rows into as many spans as it takes to put about four CTAs on every
// SM (none for a batch of thousands of rows, a few for a handful).  A row of
// one span is finished by its CTA; otherwise each CTA writes one partial
// record and the CTA that takes the row's last ticket (an atomic after a
// release fence -- nothing ever waits) merges the partials, writes the row's
// results and re-arms the ticket for the next launch, so the tickets stay
// zero between launches (and across CUDA-graph replays).
//
// Per element a CTA keeps the log-sum-exp pair (max, sum 2^((x - max) log2 e)),
// the argmax (first index among equal maxima, as torch.argmax) and, to draw a
// sample, a Gumbel-max race: key = x / T + g with g = -log(-log u) and u
// uniform in (0, 1); the column with the largest key is a draw from
// softmax(x / T) (Gumbel 1954; the "Gumbel-max trick").  u comes from a
// counter-based hash of (seed, offset, row, column pair): SplitMix64's output
// function (Steele, Lea & Flood 2014), so a draw needs no RNG state.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <algorithm>
#include <string>

#include "pkv_b200.h"
#include "pkv_error.h"

namespace pkv {
namespace {

constexpr int kThreads = 256;
constexpr int kWarpsPerCta = kThreads / 32;
constexpr int kUnroll = 4;                   // float4 loads in flight per thread
constexpr int kGroup = 4 * kUnroll;          // columns a thread folds in per iteration
constexpr int kSpanQuantum = 4 * kThreads;   // spans are multiples of this many columns
constexpr int kMinSpan = 4096;               // columns below which a row is not split further
constexpr int kCtasPerSm = 4;                // split target: resident CTAs per SM (<= 64 registers)
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr int kMaxDrafts = 16;

// ---------------------------------------------------------------------------
// Counter-based randomness.

__device__ __forceinline__ uint64_t mix64(uint64_t z) {
  z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
  z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
  return z ^ (z >> 31);
}

// One key per (seed, offset, stream, row); columns are hashed off it.
__device__ __forceinline__ uint64_t row_key(uint64_t seed, uint64_t offset, uint32_t stream, uint64_t row) {
  return mix64(mix64(seed + 0x9e3779b97f4a7c15ull * (offset + 1)) ^ (row * 4 + stream));
}

// u in [0, 1) (the range torch.rand draws from).
__device__ __forceinline__ float uniform_co(uint64_t h) { return (float)(uint32_t)(h >> 40) * 0x1p-24f; }

// Column v's 23 random bits: one SplitMix64 output serves the column pair
// (2m, 2m + 1), bits 41..63 for the even column and 18..40 for the odd one,
// so a race over consecutive columns hashes once per two.
__device__ __forceinline__ uint64_t pair_hash(uint64_t key, int v) {
  return mix64(key + (uint64_t)((uint32_t)v >> 1) * 0xd1b54a32d192ed03ull);
}
__device__ __forceinline__ uint32_t pair_bits(uint64_t h, int v) {
  return (uint32_t)((v & 1) ? (h >> 18) : (h >> 41)) & 0x7fffffu;
}

// g = -log(E), E = -log(u), u = (i + 1/2) 2^-23.  E needs relative accuracy
// where it is small (u near 1: the keys that win races): there it is the
// Taylor series of -log(1 - w) in w = 1 - u (exact in float), five terms
// below w = 2^-6 (truncation ~w^5 / 6 relative), elsewhere the fast log,
// whose ~1e-7 absolute error is then a relative one below 1e-5.  The outer
// log only shifts keys by its absolute error.
__device__ __forceinline__ float gumbel_of(uint32_t i) {
  const float u = ((float)i + 0.5f) * 0x1p-23f;
  const float w = ((float)(0x7fffffu - i) + 0.5f) * 0x1p-23f;
  const float series = w * (1.f + w * (0.5f + w * (1.f / 3.f + w * (0.25f + w * 0.2f))));
  const float e = w < 0x1p-6f ? series : -__logf(u);
  return -__logf(e);
}

__device__ __forceinline__ float gumbel(uint64_t key, int v) { return gumbel_of(pair_bits(pair_hash(key, v), v)); }

// ---------------------------------------------------------------------------
// Reductions.

// Log-sum-exp pairs in base 2: value = m2 + log2(s) over the scaled logits.
__device__ __forceinline__ void lse_merge(float& m, float& s, float m2, float s2) {
  const float mn = fmaxf(m, m2);
  if (mn == -INFINITY) return;
  s = s * exp2f(m - mn) + s2 * exp2f(m2 - mn);
  m = mn;
}

// Larger key wins; equal keys go to the smaller column (-1 = none loses).
__device__ __forceinline__ void arg_merge(float& key, int& idx, float key2, int idx2) {
  if (key2 > key || (key2 == key && (unsigned)idx2 < (unsigned)idx)) {
    key = key2;
    idx = idx2;
  }
}

__device__ __forceinline__ void warp_lse(float& m, float& s) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float m2 = __shfl_xor_sync(0xffffffffu, m, off);
    const float s2 = __shfl_xor_sync(0xffffffffu, s, off);
    lse_merge(m, s, m2, s2);
  }
}

__device__ __forceinline__ void warp_arg(float& key, int& idx) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) {
    const float k2 = __shfl_xor_sync(0xffffffffu, key, off);
    const int i2 = __shfl_xor_sync(0xffffffffu, idx, off);
    arg_merge(key, idx, k2, i2);
  }
}

__device__ __forceinline__ float warp_sum(float x) {
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

// Load iteration `i0` of a thread's stream over columns [.., v_end) of a
// row: kGroup columns, x[q] at column col[q] (rising with q), -inf past v_end.
// VEC: kUnroll float4 loads (v_end a multiple of 4); else kGroup scalar loads.
template <bool VEC>
__device__ __forceinline__ void load_group(const float* __restrict__ row, int i0, int v_end, float (&x)[kGroup],
                                           int (&col)[kGroup]) {
  if (VEC) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
    const int f_end = v_end >> 2;
#pragma unroll
    for (int u = 0; u < kUnroll; ++u) {
      const int j = i0 + u * kThreads;
      const float4 t = j < f_end ? __ldcs(r4 + j) : make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      x[4 * u + 0] = t.x;
      x[4 * u + 1] = t.y;
      x[4 * u + 2] = t.z;
      x[4 * u + 3] = t.w;
#pragma unroll
      for (int e = 0; e < 4; ++e) col[4 * u + e] = 4 * j + e;
    }
  } else {
#pragma unroll
    for (int q = 0; q < kGroup; ++q) {
      const int j = i0 + q * kThreads;
      x[q] = j < v_end ? __ldcs(row + j) : -INFINITY;
      col[q] = j;
    }
  }
}

// A thread's first load index and the stride between its iterations over a
// span [v_begin, v_end) (in float4s for VEC, in floats otherwise).
template <bool VEC>
__device__ __forceinline__ int first_index(int v_begin) {
  return (VEC ? (v_begin >> 2) : v_begin) + (int)threadIdx.x;
}
template <bool VEC>
__device__ __forceinline__ int end_index(int v_end) {
  return VEC ? (v_end >> 2) : v_end;
}
constexpr int kIterStride = kThreads * kUnroll;    // float4s per iteration of the CTA (VEC)
constexpr int kIterStrideScalar = kThreads * kGroup;

// Release this CTA's partial and take a ticket; true in the row's last CTA
// (which then sees every partial of the row).
__device__ __forceinline__ bool last_of_row(int32_t* ticket, int n) {
  __shared__ int s_last;
  __syncthreads();  // the partial is written by thread 0 before this point
  if (threadIdx.x == 0) {
    __threadfence();
    s_last = atomicAdd(ticket, 1) == n - 1;
  }
  __syncthreads();
  if (s_last) __threadfence();
  return s_last;
}

// ---------------------------------------------------------------------------
// Row statistics: log-sum-exp, argmax, an optional race, token gathers.

struct RowPart {
  float m, s;       // base-2 log-sum-exp pair of x * lse_scale
  float amax;       // argmax of x
  int aidx;
  float rkey;       // race winner
  int ridx;
  int pad[2];
};

struct RowArgs {
  const float* x;          // row r at x + r * ld
  const float* race_x;     // race logits (same layout), or null for x
  int64_t ld;
  int32_t rows, vocab;
  int32_t splits, span;    // CTAs per row and columns per CTA (a multiple of kSpanQuantum)
  float lse_scale;         // statistics of x * lse_scale (> 0)
  float race_scale;        // race key = race_x * race_scale + gumbel
  int32_t race;            // 0: token = argmax; 1: token = race winner
  uint64_t seed, offset;
  // Row r's gathered token: tokens[(r / rpg) * tpg + r % rpg] when
  // r % rpg < tpg, else none.
  const int64_t* tokens;
  int32_t rpg, tpg;
  RowPart* parts;          // [rows][splits] (splits > 1)
  int32_t* tickets;        // [rows], zero between launches
  float* lse_out;          // [rows] natural-log log-sum-exp of x * lse_scale
  float* lp_out;           // [rows] x[token] * lse_scale - lse (NaN for a token outside the vocabulary)
  int64_t* tok_out;        // [rows] race winner (race) or argmax
  float* tok_lp_out;       // [rows] x[tok_out] * lse_scale - lse
  int64_t* amax_out;       // [rows] argmax of x
};

// Merge of the per-thread states of a CTA into thread 0's (smem + warp shuffles).
__device__ __forceinline__ RowPart cta_reduce(RowPart t) {
  warp_lse(t.m, t.s);
  warp_arg(t.amax, t.aidx);
  warp_arg(t.rkey, t.ridx);
  __shared__ RowPart sp[kWarpsPerCta];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sp[warp] = t;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kWarpsPerCta; ++w) {
      lse_merge(t.m, t.s, sp[w].m, sp[w].s);
      arg_merge(t.amax, t.aidx, sp[w].amax, sp[w].aidx);
      arg_merge(t.rkey, t.ridx, sp[w].rkey, sp[w].ridx);
    }
  }
  return t;
}

// RACE: 0 none, 1 race over x, 2 race over race_x.
template <bool VEC, int RACE>
__global__ void __launch_bounds__(kThreads) row_stats_kernel(const RowArgs a) {
  const int r = blockIdx.x / a.splits, c = blockIdx.x - r * a.splits;
  const int v_begin = c * a.span, v_end = min(a.vocab, v_begin + a.span);
  const float* row = a.x + (int64_t)r * a.ld;
  const float* rrow = RACE == 2 ? a.race_x + (int64_t)r * a.ld : row;
  const float k2 = a.lse_scale * kLog2e;
  const uint64_t key = RACE ? row_key(a.seed, a.offset, 0, (uint64_t)r) : 0;
  RowPart t{-INFINITY, 0.f, -INFINITY, -1, -INFINITY, -1, {0, 0}};
  const int i_end = end_index<VEC>(v_end);
  for (int i = first_index<VEC>(v_begin); i < i_end; i += VEC ? kIterStride : kIterStrideScalar) {
    float x[kGroup];
    int col[kGroup];
    load_group<VEC>(row, i, v_end, x, col);
    float rx[kGroup];
    if (RACE == 2) load_group<VEC>(rrow, i, v_end, rx, col);
    float gm = -INFINITY;
#pragma unroll
    for (int q = 0; q < kGroup; ++q) gm = fmaxf(gm, x[q]);
    if (gm == -INFINITY) continue;
    // Rescale the running sum once per group, then one 2^y per column.
    const float gy = gm * k2;
    if (gy > t.m) {
      t.s *= exp2f(t.m - gy);
      t.m = gy;
    }
#pragma unroll
    for (int q = 0; q < kGroup; ++q) {
      t.s += exp2f(fmaf(x[q], k2, -t.m));
      if (x[q] > t.amax) {
        t.amax = x[q];
        t.aidx = col[q];
      }
    }
    if (RACE) {
      // Vector loads give consecutive columns, so pairs (2m, 2m + 1) share one hash.
#pragma unroll
      for (int q = 0; q < kGroup; q += 2) {
        const uint64_t h = VEC ? pair_hash(key, col[q]) : 0;
#pragma unroll
        for (int p = 0; p < 2; ++p) {
          const float v = RACE == 2 ? rx[q + p] : x[q + p];
          if (v == -INFINITY) continue;
          const uint64_t hh = VEC ? h : pair_hash(key, col[q + p]);
          const float kk = fmaf(v, a.race_scale, gumbel_of(pair_bits(hh, col[q + p])));
          if (kk > t.rkey) {
            t.rkey = kk;
            t.ridx = col[q + p];
          }
        }
      }
    }
  }
  t = cta_reduce(t);
  const int lane = threadIdx.x & 31;
  if (a.splits > 1) {
    if (threadIdx.x == 0) a.parts[(int64_t)r * a.splits + c] = t;
    if (!last_of_row(a.tickets + r, a.splits)) return;
    // The row's last CTA: merge the partials (warp 0), write the results.
    if (threadIdx.x >= 32) return;
    RowPart u{-INFINITY, 0.f, -INFINITY, -1, -INFINITY, -1, {0, 0}};
    for (int i = lane; i < a.splits; i += 32) {
      const RowPart* p = a.parts + (int64_t)r * a.splits + i;
      lse_merge(u.m, u.s, __ldcg(&p->m), __ldcg(&p->s));
      arg_merge(u.amax, u.aidx, __ldcg(&p->amax), __ldcg(&p->aidx));
      arg_merge(u.rkey, u.ridx, __ldcg(&p->rkey), __ldcg(&p->ridx));
    }
    warp_lse(u.m, u.s);
    warp_arg(u.amax, u.aidx);
    warp_arg(u.rkey, u.ridx);
    t = u;
    if (lane == 0) a.tickets[r] = 0;
  }
  if (threadIdx.x != 0) return;
  const float lse = (t.m + log2f(t.s)) * kLn2;
  if (a.lse_out) a.lse_out[r] = lse;
  if (a.lp_out && a.tokens) {
    const int g = r / a.rpg, i = r - g * a.rpg;
    if (i < a.tpg) {
      const int64_t tok = a.tokens[(int64_t)g * a.tpg + i];
      a.lp_out[r] = (tok >= 0 && tok < a.vocab) ? row[tok] * a.lse_scale - lse : NAN;
    }
  }
  const int tok = (RACE && t.ridx >= 0) ? t.ridx : t.aidx;
  if (a.tok_out) a.tok_out[r] = tok;
  if (a.tok_lp_out) a.tok_lp_out[r] = tok >= 0 ? row[tok] * a.lse_scale - lse : NAN;
  if (a.amax_out) a.amax_out[r] = t.aidx;
}

// ---------------------------------------------------------------------------
// Speculative accept / reject.

struct AccPart {
  float sum_w;      // sum of max(p_target - p_draft, 0) over the chunk
  float key_w;      // correction race (or argmax) over those weights
  int idx_w;
  float key_p;      // race (or argmax) over the target distribution
  int idx_p;
  int pad[3];
};

struct AccArgs {
  const float* xt;         // target logits [batch][k + 1][ld]
  const float* xd;         // draft logits [batch][k][ld]
  int64_t ld;
  int32_t batch, k, vocab;
  int32_t splits, span;    // CTAs per sequence and columns per CTA
  const int64_t* dtok;     // [batch][k]
  const int32_t* n_draft;  // [batch]
  const float* uniforms;   // [batch][k], or null: hashed from (seed, offset)
  float inv_t_draft;       // 1 / the draft's sampling temperature
  int32_t do_sample;
  int64_t eos;             // < 0: none
  uint64_t seed, offset;
  const float* lse_t;      // [batch][k + 1]
  const float* lp_t;       // [batch][k + 1]: target log-prob of draft i at row i
  const float* lp_d;       // [batch][k]: draft log-prob (at its temperature) of draft i
  const float* lse_d;      // [batch][k]
  AccPart* parts;          // [batch][splits] (splits > 1)
  int32_t* tickets;        // [batch]
  int64_t* tok_out;        // [batch][k + 1]
  float* lp_out;           // [batch][k + 1]
  int32_t* n_out;          // [batch]: tokens emitted (-1: a draft token outside the vocabulary)
  int32_t* n_acc;          // [batch]: draft tokens accepted
};

struct Decision {
  int m;        // accepted drafts; the target row the draw uses
  int stop;     // an accepted draft was eos: nothing is drawn
  int reject;   // draft m was rejected: correction draw, else bonus draw
  int bad;      // a draft token outside the vocabulary
};

// speculative.py:244-256: draft i is kept when u_i <= min(1, exp(lp_target -
// lp_draft)), lp_draft = log(p_draft + 1e-12); the first rejection ends the
// round, and an accepted eos ends it without a draw.
__device__ Decision decide(const AccArgs& a, int b) {
  Decision d{0, 0, 0, 0};
  const int nd = min(max(a.n_draft[b], 0), a.k);
  const uint64_t ukey = row_key(a.seed, a.offset, 1, (uint64_t)b);
  for (int i = 0; i < nd; ++i) {
    const int64_t tok = a.dtok[(int64_t)b * a.k + i];
    if (tok < 0 || tok >= a.vocab) {
      d.bad = 1;
      d.m = i;
      return d;
    }
    const float plp = a.lp_t[(int64_t)b * (a.k + 1) + i];
    const float dlp = logf(expf(a.lp_d[(int64_t)b * a.k + i]) + 1e-12f);
    const float acc = fminf(1.f, expf(plp - dlp));
    const float u = a.uniforms ? a.uniforms[(int64_t)b * a.k + i] : uniform_co(mix64(ukey + (uint64_t)i));
    if (u <= acc) {
      if (tok == a.eos) {
        d.m = i + 1;
        d.stop = 1;
        return d;
      }
      continue;
    }
    d.m = i;
    d.reject = 1;
    return d;
  }
  d.m = nd;
  return d;
}

template <bool VEC>
__global__ void __launch_bounds__(kThreads) spec_accept_kernel(const AccArgs a) {
  const int b = blockIdx.x / a.splits, c = blockIdx.x - b * a.splits;
  __shared__ Decision sd;
  if (threadIdx.x == 0) sd = decide(a, b);
  __syncthreads();
  const Decision d = sd;
  const int K1 = a.k + 1;
  if (d.stop || d.bad) {
    // No draw: the first CTA of the sequence writes its results.
    if (c != 0 || threadIdx.x > (unsigned)a.k) return;
    const int i = threadIdx.x;
    const int64_t o = (int64_t)b * K1 + i;
    if (i < d.m) {
      a.tok_out[o] = a.dtok[(int64_t)b * a.k + i];
      a.lp_out[o] = a.lp_t[o];
    } else {
      a.tok_out[o] = -1;
      a.lp_out[o] = 0.f;
    }
    if (i == 0) {
      a.n_out[b] = d.bad ? -1 : d.m;
      a.n_acc[b] = d.m;
    }
    return;
  }

  const int v_begin = c * a.span, v_end = min(a.vocab, v_begin + a.span);
  const int64_t trow = (int64_t)b * K1 + d.m;
  const int64_t drow = (int64_t)b * a.k + d.m;  // read only on a rejection (d.m < n_draft <= k)
  const float* xt = a.xt + trow * a.ld;
  const float* xd = a.xd + drow * a.ld;
  const bool sample = a.do_sample != 0;
  const uint64_t key = row_key(a.seed, a.offset, 2, (uint64_t)b);
  const float lt2 = a.lse_t[trow] * kLog2e;
  const float ld2 = d.reject ? a.lse_d[drow] * kLog2e : 0.f;
  const float kd = a.inv_t_draft * kLog2e;
  AccPart t{0.f, -INFINITY, -1, -INFINITY, -1, {0, 0, 0}};
  const int i_end = end_index<VEC>(v_end);
  for (int i = first_index<VEC>(v_begin); i < i_end; i += VEC ? kIterStride : kIterStrideScalar) {
    float x[kGroup], y[kGroup];
    int col[kGroup];
    load_group<VEC>(xt, i, v_end, x, col);
    if (d.reject) load_group<VEC>(xd, i, v_end, y, col);
#pragma unroll
    for (int q = 0; q < kGroup; ++q) {
      if (x[q] == -INFINITY) continue;
      const float g = sample ? gumbel(key, col[q]) : 0.f;
      if (d.reject) {
        // correction_probs = clamp(p_target - p_draft, 0) (speculative.py:251)
        const float w = fmaxf(exp2f(fmaf(x[q], kLog2e, -lt2)) - exp2f(fmaf(y[q], kd, -ld2)), 0.f);
        t.sum_w += w;
        const float kw = sample ? (w > 0.f ? __logf(w) + g : -INFINITY) : w;
        if (kw > t.key_w) {
          t.key_w = kw;
          t.idx_w = col[q];
        }
      }
      const float kp = x[q] + g;
      if (kp > t.key_p) {
        t.key_p = kp;
        t.idx_p = col[q];
      }
    }
  }
  t.sum_w = warp_sum(t.sum_w);
  warp_arg(t.key_w, t.idx_w);
  warp_arg(t.key_p, t.idx_p);
  __shared__ AccPart sp[kWarpsPerCta];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sp[warp] = t;
  __syncthreads();
  if (threadIdx.x == 0) {
    for (int w = 1; w < kWarpsPerCta; ++w) {
      t.sum_w += sp[w].sum_w;
      arg_merge(t.key_w, t.idx_w, sp[w].key_w, sp[w].idx_w);
      arg_merge(t.key_p, t.idx_p, sp[w].key_p, sp[w].idx_p);
    }
  }
  if (a.splits > 1) {
    if (threadIdx.x == 0) a.parts[(int64_t)b * a.splits + c] = t;
    if (!last_of_row(a.tickets + b, a.splits)) return;
    if (warp != 0) return;
    AccPart u{0.f, -INFINITY, -1, -INFINITY, -1, {0, 0, 0}};
    for (int i = lane; i < a.splits; i += 32) {
      const AccPart* p = a.parts + (int64_t)b * a.splits + i;
      u.sum_w += __ldcg(&p->sum_w);
      arg_merge(u.key_w, u.idx_w, __ldcg(&p->key_w), __ldcg(&p->idx_w));
      arg_merge(u.key_p, u.idx_p, __ldcg(&p->key_p), __ldcg(&p->idx_p));
    }
    u.sum_w = warp_sum(u.sum_w);
    warp_arg(u.key_w, u.idx_w);
    warp_arg(u.key_p, u.idx_p);
    t = u;
    if (lane == 0) a.tickets[b] = 0;
  } else if (warp != 0) {
    return;
  }
  // Warp 0 of the finishing CTA; lane 0 holds the merged record (broadcast).
  t.sum_w = __shfl_sync(0xffffffffu, t.sum_w, 0);
  t.idx_w = __shfl_sync(0xffffffffu, t.idx_w, 0);
  t.idx_p = __shfl_sync(0xffffffffu, t.idx_p, 0);
  // An all-zero correction falls back to the target distribution itself
  // (speculative.py:252-253).
  const int tok = (d.reject && t.sum_w > 0.f && t.idx_w >= 0) ? t.idx_w : t.idx_p;
  for (int i = lane; i <= a.k; i += 32) {
    const int64_t o = (int64_t)b * K1 + i;
    if (i < d.m) {
      a.tok_out[o] = a.dtok[(int64_t)b * a.k + i];
      a.lp_out[o] = a.lp_t[o];
    } else if (i == d.m) {
      a.tok_out[o] = tok;
      a.lp_out[o] = tok >= 0 ? xt[tok] - a.lse_t[trow] : NAN;
    } else {
      a.tok_out[o] = -1;
      a.lp_out[o] = 0.f;
    }
  }
  if (lane == 0) {
    a.n_out[b] = d.m + 1;
    a.n_acc[b] = d.m;
  }
}

// ---------------------------------------------------------------------------
// Host side.

int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

// SM count of the current device (queried once per device).
int num_sms() {
  constexpr int kMaxDevices = 64;
  static int cache[kMaxDevices] = {};
  int dev = 0;
  cudaGetDevice(&dev);
  if (dev < 0 || dev >= kMaxDevices) dev = 0;
  if (cache[dev] == 0) {
    int sms = 0;
    cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    cache[dev] = sms > 0 ? sms : 148;
  }
  return cache[dev];
}

// Most CTAs one row is ever cut into.
int32_t max_splits(int32_t vocab) { return (vocab + kMinSpan - 1) / kMinSpan; }

// Cut each of `rows` rows into spans so that the launch has about
// kCtasPerSm CTAs per SM, never spans under kMinSpan columns.
void plan_split(int64_t rows, int32_t vocab, int32_t* splits, int32_t* span) {
  const int64_t target = (int64_t)num_sms() * kCtasPerSm;
  int64_t sp = rows > 0 ? (target + rows - 1) / rows : 1;
  sp = std::max<int64_t>(1, std::min<int64_t>(sp, max_splits(vocab)));
  const int64_t per = (vocab + sp - 1) / sp;
  *span = (int32_t)((per + kSpanQuantum - 1) / kSpanQuantum * kSpanQuantum);
  *splits = (int32_t)((vocab + *span - 1) / *span);
}

// Row workspace: RowPart x rows x splits (scratch: written before it is read).
int64_t row_ws_bytes(int64_t rows, int32_t vocab) {
  return align256(rows * max_splits(vocab) * (int64_t)sizeof(RowPart));
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// float4 loads: rows start on 16 bytes and a load never passes the row's
// last column.
bool vec_ok(int64_t ld, int32_t vocab, const void* p) { return ld % 4 == 0 && vocab % 4 == 0 && aligned16(p); }

int32_t check_rows(const float* x, int64_t ld, int64_t rows, int32_t vocab, const char* who) {
  if (!x || rows < 0 || vocab <= 0 || ld < vocab) {
    pkv_set_error(std::string(who) + ": logits must be non-null with rows >= 0, vocab >= 1 and ld >= vocab");
    return PKV_ERR_ARG;
  }
  if (rows * (int64_t)max_splits(vocab) > INT32_MAX) {
    pkv_set_error(std::string(who) + ": too many rows for one launch");
    return PKV_ERR_ARG;
  }
  return PKV_OK;
}

template <bool VEC>
void launch_rows_t(const RowArgs& a, unsigned grid, cudaStream_t s) {
  if (!a.race)
    row_stats_kernel<VEC, 0><<<grid, kThreads, 0, s>>>(a);
  else if (!a.race_x)
    row_stats_kernel<VEC, 1><<<grid, kThreads, 0, s>>>(a);
  else
    row_stats_kernel<VEC, 2><<<grid, kThreads, 0, s>>>(a);
}

int32_t launch_rows(RowArgs a, bool vec, cudaStream_t s, const char* who) {
  if (a.rows == 0) return PKV_OK;
  plan_split(a.rows, a.vocab, &a.splits, &a.span);
  const unsigned grid = (unsigned)((int64_t)a.rows * a.splits);
  if (vec)
    launch_rows_t<true>(a, grid, s);
  else
    launch_rows_t<false>(a, grid, s);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    pkv_set_error(std::string(who) + ": " + cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}

// Speculative workspace (scratch): [lse_t, lp_t: batch (k+1)][lse_d, lp_d:
// batch k][RowPart: batch (2k+1) x splits][AccPart: batch x splits].
// Tickets: batch (2k+1) row tickets, then batch accept tickets.
struct SpecWs {
  int64_t lse_t, lp_t, lse_d, lp_d, row_parts, acc_parts, total;
};

SpecWs spec_ws(int64_t batch, int32_t k, int32_t vocab) {
  SpecWs w;
  const int64_t nt = batch * (k + 1), nd = batch * k, nc = max_splits(vocab);
  w.lse_t = 0;
  w.lp_t = w.lse_t + align256(nt * 4);
  w.lse_d = w.lp_t + align256(nt * 4);
  w.lp_d = w.lse_d + align256(nd * 4);
  w.row_parts = w.lp_d + align256(nd * 4);
  w.acc_parts = w.row_parts + align256((nt + nd) * nc * (int64_t)sizeof(RowPart));
  w.total = w.acc_parts + align256(batch * nc * (int64_t)sizeof(AccPart));
  return w;
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" int64_t pkv_sampling_workspace_bytes(int64_t n_rows, int32_t vocab) {
  if (n_rows < 0 || vocab <= 0) return -1;
  return row_ws_bytes(n_rows, vocab);
}

extern "C" int32_t pkv_token_logprobs(const float* logits, int64_t ld, int32_t n_rows, int32_t vocab,
                                      const int64_t* tokens, float* logprobs_out, float* lse_out, int32_t* tickets,
                                      void* workspace, int64_t workspace_bytes, void* stream) {
  pkv_clear_error();
  if (int32_t st = check_rows(logits, ld, n_rows, vocab, "pkv_token_logprobs")) return st;
  if ((logprobs_out && !tokens) || (!logprobs_out && !lse_out)) {
    pkv_set_error("pkv_token_logprobs: give tokens with logprobs_out, and at least one output");
    return PKV_ERR_ARG;
  }
  if (!tickets || !workspace || workspace_bytes < row_ws_bytes(n_rows, vocab)) {
    pkv_set_error("pkv_token_logprobs: null tickets, or a workspace smaller than pkv_sampling_workspace_bytes");
    return PKV_ERR_ARG;
  }
  RowArgs a = {};
  a.x = logits;
  a.ld = ld;
  a.rows = n_rows;
  a.vocab = vocab;
  a.lse_scale = 1.f;
  a.race_scale = 1.f;
  a.tokens = tokens;
  a.rpg = 1;
  a.tpg = 1;
  a.lse_out = lse_out;
  a.lp_out = logprobs_out;
  a.tickets = tickets;
  a.parts = static_cast<RowPart*>(workspace);
  const bool vec = vec_ok(ld, vocab, logits);
  return launch_rows(a, vec, static_cast<cudaStream_t>(stream), "pkv_token_logprobs");
}

extern "C" int32_t pkv_sample_tokens(const float* logits, const float* race_logits, int64_t ld, int32_t n_rows,
                                     int32_t vocab, float temperature, int32_t do_sample, uint64_t seed,
                                     uint64_t offset, int64_t* tokens_out, float* logprobs_out, int64_t* argmax_out,
                                     int32_t* tickets, void* workspace, int64_t workspace_bytes, void* stream) {
  pkv_clear_error();
  if (int32_t st = check_rows(logits, ld, n_rows, vocab, "pkv_sample_tokens")) return st;
  if (!tokens_out) {
    pkv_set_error("pkv_sample_tokens: tokens_out is required");
    return PKV_ERR_ARG;
  }
  if (do_sample && !(temperature > 0.f)) {
    pkv_set_error("pkv_sample_tokens: sampling needs a temperature > 0");
    return PKV_ERR_ARG;
  }
  if (!tickets || !workspace || workspace_bytes < row_ws_bytes(n_rows, vocab)) {
    pkv_set_error("pkv_sample_tokens: null tickets, or a workspace smaller than pkv_sampling_workspace_bytes");
    return PKV_ERR_ARG;
  }
  RowArgs a = {};
  a.x = logits;
  a.race_x = race_logits;
  a.ld = ld;
  a.rows = n_rows;
  a.vocab = vocab;
  a.lse_scale = 1.f;
  a.race = do_sample ? 1 : 0;
  a.race_scale = do_sample ? 1.f / temperature : 1.f;
  a.seed = seed;
  a.offset = offset;
  a.tok_out = tokens_out;
  a.tok_lp_out = logprobs_out;
  a.amax_out = argmax_out;
  a.tickets = tickets;
  a.parts = static_cast<RowPart*>(workspace);
  const bool vec = vec_ok(ld, vocab, logits) && (!race_logits || aligned16(race_logits));
  return launch_rows(a, vec, static_cast<cudaStream_t>(stream), "pkv_sample_tokens");
}

extern "C" int64_t pkv_spec_workspace_bytes(int32_t batch, int32_t k, int32_t vocab) {
  if (batch < 0 || k < 1 || k > kMaxDrafts || vocab <= 0) return -1;
  return spec_ws(batch, k, vocab).total;
}

extern "C" int64_t pkv_spec_tickets(int32_t batch, int32_t k) {
  if (batch < 0 || k < 1 || k > kMaxDrafts) return -1;
  return (int64_t)batch * (2 * k + 2);
}

extern "C" int32_t pkv_spec_accept(const float* target_logits, const float* draft_logits, int64_t ld,
                                   const int64_t* draft_tokens, const int32_t* n_draft, const float* uniforms,
                                   int32_t batch, int32_t k, int32_t vocab, float draft_temperature,
                                   int32_t do_sample, int64_t eos_token_id, uint64_t seed, uint64_t offset,
                                   int64_t* tokens_out, float* logprobs_out, int32_t* n_out, int32_t* n_accepted,
                                   int32_t* tickets, void* workspace, int64_t workspace_bytes, void* stream) {
  pkv_clear_error();
  const char* who = "pkv_spec_accept";
  if (k < 1 || k > kMaxDrafts) {
    pkv_set_error("pkv_spec_accept: k must be in [1, 16]");
    return PKV_ERR_ARG;
  }
  if (int32_t st = check_rows(target_logits, ld, (int64_t)batch * (k + 1), vocab, who)) return st;
  if (int32_t st = check_rows(draft_logits, ld, (int64_t)batch * k, vocab, who)) return st;
  if (!draft_tokens || !n_draft || !tokens_out || !logprobs_out || !n_out || !n_accepted) {
    pkv_set_error("pkv_spec_accept: null draft tokens, draft counts or outputs");
    return PKV_ERR_ARG;
  }
  if (!(draft_temperature > 0.f)) {
    pkv_set_error("pkv_spec_accept: the draft temperature must be > 0");
    return PKV_ERR_ARG;
  }
  const SpecWs w = spec_ws(batch, k, vocab);
  if (!tickets || !workspace || workspace_bytes < w.total) {
    pkv_set_error("pkv_spec_accept: null tickets, or a workspace smaller than pkv_spec_workspace_bytes");
    return PKV_ERR_ARG;
  }
  if (batch == 0) return PKV_OK;
  char* base = static_cast<char*>(workspace);
  cudaStream_t s = static_cast<cudaStream_t>(stream);
  const int32_t nc = max_splits(vocab);
  const bool vec = vec_ok(ld, vocab, target_logits) && aligned16(draft_logits);
  RowPart* parts = reinterpret_cast<RowPart*>(base + w.row_parts);
  const int64_t nt = (int64_t)batch * (k + 1), nd = (int64_t)batch * k;

  // Target rows: log-sum-exp at temperature 1 and the log-prob of each draft
  // token at the row that predicts it (row i predicts draft i; row k, the
  // bonus row, gathers nothing).
  RowArgs t = {};
  t.x = target_logits;
  t.ld = ld;
  t.rows = (int32_t)nt;
  t.vocab = vocab;
  t.lse_scale = 1.f;
  t.race_scale = 1.f;
  t.tokens = draft_tokens;
  t.rpg = k + 1;
  t.tpg = k;
  t.tickets = tickets;
  t.parts = parts;
  t.lse_out = reinterpret_cast<float*>(base + w.lse_t);
  t.lp_out = reinterpret_cast<float*>(base + w.lp_t);
  if (int32_t st = launch_rows(t, vec, s, who)) return st;
  // Draft rows: the same at the draft's temperature (speculative.py:200-203).
  RowArgs d = t;
  d.x = draft_logits;
  d.rows = (int32_t)nd;
  d.lse_scale = 1.f / draft_temperature;
  d.rpg = k;
  d.tpg = k;
  d.tickets = tickets + nt;
  d.parts = parts + nt * nc;
  d.lse_out = reinterpret_cast<float*>(base + w.lse_d);
  d.lp_out = reinterpret_cast<float*>(base + w.lp_d);
  if (int32_t st = launch_rows(d, vec, s, who)) return st;

  AccArgs a = {};
  a.xt = target_logits;
  a.xd = draft_logits;
  a.ld = ld;
  a.batch = batch;
  a.k = k;
  a.vocab = vocab;
  plan_split(batch, vocab, &a.splits, &a.span);
  a.dtok = draft_tokens;
  a.n_draft = n_draft;
  a.uniforms = uniforms;
  a.inv_t_draft = 1.f / draft_temperature;
  a.do_sample = do_sample;
  a.eos = eos_token_id;
  a.seed = seed;
  a.offset = offset;
  a.lse_t = t.lse_out;
  a.lp_t = t.lp_out;
  a.lse_d = d.lse_out;
  a.lp_d = d.lp_out;
  a.parts = reinterpret_cast<AccPart*>(base + w.acc_parts);
  a.tickets = tickets + nt + nd;
  a.tok_out = tokens_out;
  a.lp_out = logprobs_out;
  a.n_out = n_out;
  a.n_acc = n_accepted;
  const unsigned grid = (unsigned)((int64_t)batch * a.splits);
  if (vec)
    spec_accept_kernel<true><<<grid, kThreads, 0, s>>>(a);
  else
    spec_accept_kernel<false><<<grid, kThreads, 0, s>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    pkv_set_error(std::string("pkv_spec_accept: ") + cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}
