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
// row) from HBM once.  A row is cut into chunks of kChunk columns, one CTA
// each (grid = rows x chunks, so a handful of rows already covers the 148
// SMs).  Each CTA reduces its chunk in registers and writes one partial
// record; the CTA that takes the row's last ticket (an atomic after a release
// fence -- nothing ever waits) merges the row's partials, writes the row's
// results and re-arms the ticket for the next launch, so the tickets stay
// zero between launches (and across CUDA-graph replays).
//
// Per element a CTA keeps the log-sum-exp pair (max, sum 2^((x - max) log2 e)),
// the argmax (first index among equal maxima, as torch.argmax) and, to draw a
// sample, a Gumbel-max race: key = x / T + g with g = -log(-log u) and u
// uniform in (0, 1); the column with the largest key is a draw from
// softmax(x / T) (Gumbel 1954; the "Gumbel-max trick").  u comes from a
// counter-based hash of (seed, offset, row, column): SplitMix64's output
// function (Steele, Lea & Flood 2014), so a draw needs no RNG state.
#include <cuda_runtime.h>
#include <math.h>
#include <stdint.h>

#include <string>

#include "pkv_b200.h"
#include "pkv_error.h"

namespace pkv {
namespace {

constexpr int kThreads = 256;
constexpr int kWarpsPerCta = kThreads / 32;
constexpr int kChunk = 8192;               // columns of one row per CTA
constexpr int kPer = kChunk / kThreads;    // 32 per thread
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

// u in (0, 1) from 23 hashed bits: (i + 1/2) 2^-23, so -log u > 0 always.
__device__ __forceinline__ float uniform_open(uint64_t h) {
  return ((float)(uint32_t)(h >> 41) + 0.5f) * 0x1p-23f;
}

// u in [0, 1) (the range torch.rand draws from).
__device__ __forceinline__ float uniform_co(uint64_t h) { return (float)(uint32_t)(h >> 40) * 0x1p-24f; }

__device__ __forceinline__ float gumbel(uint64_t key, int v) {
  const float u = uniform_open(mix64(key + (uint64_t)(uint32_t)v * 0xd1b54a32d192ed03ull));
  return -logf(-logf(u));
}

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

// Column of register q of this thread in the chunk starting at v0.  With
// float4 loads a thread holds 4 adjacent columns per load; either way the
// columns of one thread rise with q, so strict comparisons keep the first
// index of a tie inside the thread.
template <bool VEC>
__device__ __forceinline__ int col_of(int v0, int q) {
  if (VEC) return v0 + 4 * ((q >> 2) * kThreads + (int)threadIdx.x) + (q & 3);
  return v0 + q * kThreads + (int)threadIdx.x;
}

// Load this thread's kPer columns of a row chunk; columns >= vocab read -inf.
template <bool VEC>
__device__ __forceinline__ void load_chunk(const float* __restrict__ row, int v0, int vocab, float (&x)[kPer]) {
  if (VEC) {
    const float4* r4 = reinterpret_cast<const float4*>(row);
#pragma unroll
    for (int j = 0; j < kPer / 4; ++j) {
      const int c = col_of<true>(v0, 4 * j);
      float4 t = make_float4(-INFINITY, -INFINITY, -INFINITY, -INFINITY);
      if (c < vocab) t = __ldcs(r4 + (c >> 2));
      x[4 * j + 0] = t.x;
      x[4 * j + 1] = c + 1 < vocab ? t.y : -INFINITY;
      x[4 * j + 2] = c + 2 < vocab ? t.z : -INFINITY;
      x[4 * j + 3] = c + 3 < vocab ? t.w : -INFINITY;
    }
  } else {
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      const int c = col_of<false>(v0, q);
      x[q] = c < vocab ? __ldcs(row + c) : -INFINITY;
    }
  }
}

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
  int32_t rows, vocab, nchunks;
  float lse_scale;         // statistics of x * lse_scale (> 0)
  float race_scale;        // race key = race_x * race_scale + gumbel
  int32_t race;            // 0: token = argmax; 1: token = race winner
  uint64_t seed, offset;
  // Row r's gathered token: tokens[(r / rpg) * tpg + r % rpg] when
  // r % rpg < tpg, else none.
  const int64_t* tokens;
  int32_t rpg, tpg;
  RowPart* parts;          // [rows][nchunks]
  int32_t* tickets;        // [rows], zero between launches
  float* lse_out;          // [rows] natural-log log-sum-exp of x * lse_scale
  float* lp_out;           // [rows] x[token] * lse_scale - lse (NaN for a token outside the vocabulary)
  int64_t* tok_out;        // [rows] race winner (race) or argmax
  float* tok_lp_out;       // [rows] x[tok_out] * lse_scale - lse
  int64_t* amax_out;       // [rows] argmax of x
};

template <bool VEC>
__global__ void __launch_bounds__(kThreads) row_stats_kernel(const RowArgs a) {
  const int r = blockIdx.x / a.nchunks, c = blockIdx.x - r * a.nchunks;
  const int v0 = c * kChunk;
  const float* row = a.x + (int64_t)r * a.ld;
  float x[kPer];
  load_chunk<VEC>(row, v0, a.vocab, x);

  float amax = -INFINITY;
  int aidx = -1;
#pragma unroll
  for (int q = 0; q < kPer; ++q)
    if (x[q] > amax) {
      amax = x[q];
      aidx = col_of<VEC>(v0, q);
    }
  const float k2 = a.lse_scale * kLog2e;
  float m = amax == -INFINITY ? -INFINITY : amax * k2;
  float s = 0.f;
  if (amax != -INFINITY) {
#pragma unroll
    for (int q = 0; q < kPer; ++q) s += exp2f(fmaf(x[q], k2, -m));
  }
  float rkey = -INFINITY;
  int ridx = -1;
  if (a.race) {
    const uint64_t key = row_key(a.seed, a.offset, 0, (uint64_t)r);
    if (a.race_x) load_chunk<VEC>(a.race_x + (int64_t)r * a.ld, v0, a.vocab, x);
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      if (x[q] == -INFINITY) continue;
      const int v = col_of<VEC>(v0, q);
      const float kk = fmaf(x[q], a.race_scale, gumbel(key, v));
      if (kk > rkey) {
        rkey = kk;
        ridx = v;
      }
    }
  }

  warp_lse(m, s);
  warp_arg(amax, aidx);
  warp_arg(rkey, ridx);
  __shared__ RowPart sp[kWarpsPerCta];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sp[warp] = RowPart{m, s, amax, aidx, rkey, ridx, {0, 0}};
  __syncthreads();
  if (threadIdx.x == 0) {
    RowPart t = sp[0];
    for (int w = 1; w < kWarpsPerCta; ++w) {
      lse_merge(t.m, t.s, sp[w].m, sp[w].s);
      arg_merge(t.amax, t.aidx, sp[w].amax, sp[w].aidx);
      arg_merge(t.rkey, t.ridx, sp[w].rkey, sp[w].ridx);
    }
    a.parts[(int64_t)r * a.nchunks + c] = t;
  }
  if (!last_of_row(a.tickets + r, a.nchunks)) return;

  // The row's last CTA: merge the partials (warp 0), write the results.
  if (warp != 0) return;
  RowPart t{-INFINITY, 0.f, -INFINITY, -1, -INFINITY, -1, {0, 0}};
  for (int i = lane; i < a.nchunks; i += 32) {
    const RowPart* p = a.parts + (int64_t)r * a.nchunks + i;
    const float pm = __ldcg(&p->m), ps = __ldcg(&p->s), pa = __ldcg(&p->amax), pk = __ldcg(&p->rkey);
    const int pai = __ldcg(&p->aidx), pri = __ldcg(&p->ridx);
    lse_merge(t.m, t.s, pm, ps);
    arg_merge(t.amax, t.aidx, pa, pai);
    arg_merge(t.rkey, t.ridx, pk, pri);
  }
  warp_lse(t.m, t.s);
  warp_arg(t.amax, t.aidx);
  warp_arg(t.rkey, t.ridx);
  if (lane != 0) return;
  const float lse = (t.m + log2f(t.s)) * kLn2;
  if (a.lse_out) a.lse_out[r] = lse;
  if (a.lp_out && a.tokens) {
    const int g = r / a.rpg, i = r - g * a.rpg;
    if (i < a.tpg) {
      const int64_t tok = a.tokens[(int64_t)g * a.tpg + i];
      a.lp_out[r] = (tok >= 0 && tok < a.vocab) ? row[tok] * a.lse_scale - lse : NAN;
    }
  }
  const int tok = (a.race && t.ridx >= 0) ? t.ridx : t.aidx;
  if (a.tok_out) a.tok_out[r] = tok;
  if (a.tok_lp_out) a.tok_lp_out[r] = tok >= 0 ? row[tok] * a.lse_scale - lse : NAN;
  if (a.amax_out) a.amax_out[r] = t.aidx;
  a.tickets[r] = 0;
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
  int32_t batch, k, vocab, nchunks;
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
  AccPart* parts;          // [batch][nchunks]
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
  const int b = blockIdx.x / a.nchunks, c = blockIdx.x - b * a.nchunks;
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

  const int v0 = c * kChunk;
  const int64_t trow = (int64_t)b * K1 + d.m;
  const float* xt = a.xt + trow * a.ld;
  float x[kPer];
  load_chunk<VEC>(xt, v0, a.vocab, x);
  const bool sample = a.do_sample != 0;
  const uint64_t key = row_key(a.seed, a.offset, 2, (uint64_t)b);
  float sum_w = 0.f, key_w = -INFINITY, key_p = -INFINITY;
  int idx_w = -1, idx_p = -1;
  if (d.reject) {
    const int64_t drow = (int64_t)b * a.k + d.m;
    float y[kPer];
    load_chunk<VEC>(a.xd + drow * a.ld, v0, a.vocab, y);
    const float lt2 = a.lse_t[trow] * kLog2e;
    const float ld2 = a.lse_d[drow] * kLog2e;
    const float kd = a.inv_t_draft * kLog2e;
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      if (x[q] == -INFINITY) continue;
      const int v = col_of<VEC>(v0, q);
      // correction_probs = clamp(p_target - p_draft, 0) (speculative.py:251)
      const float w = fmaxf(exp2f(fmaf(x[q], kLog2e, -lt2)) - exp2f(fmaf(y[q], kd, -ld2)), 0.f);
      sum_w += w;
      float g = 0.f;
      if (sample) g = gumbel(key, v);
      const float kw = sample ? (w > 0.f ? logf(w) + g : -INFINITY) : w;
      if (kw > key_w) {
        key_w = kw;
        idx_w = v;
      }
      const float kp = sample ? x[q] + g : x[q];
      if (kp > key_p) {
        key_p = kp;
        idx_p = v;
      }
    }
  } else {
#pragma unroll
    for (int q = 0; q < kPer; ++q) {
      if (x[q] == -INFINITY) continue;
      const int v = col_of<VEC>(v0, q);
      const float kp = sample ? x[q] + gumbel(key, v) : x[q];
      if (kp > key_p) {
        key_p = kp;
        idx_p = v;
      }
    }
  }
  sum_w = warp_sum(sum_w);
  warp_arg(key_w, idx_w);
  warp_arg(key_p, idx_p);
  __shared__ AccPart sp[kWarpsPerCta];
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (lane == 0) sp[warp] = AccPart{sum_w, key_w, idx_w, key_p, idx_p, {0, 0, 0}};
  __syncthreads();
  if (threadIdx.x == 0) {
    AccPart t = sp[0];
    for (int w = 1; w < kWarpsPerCta; ++w) {
      t.sum_w += sp[w].sum_w;
      arg_merge(t.key_w, t.idx_w, sp[w].key_w, sp[w].idx_w);
      arg_merge(t.key_p, t.idx_p, sp[w].key_p, sp[w].idx_p);
    }
    a.parts[(int64_t)b * a.nchunks + c] = t;
  }
  if (!last_of_row(a.tickets + b, a.nchunks)) return;
  if (warp != 0) return;

  AccPart t{0.f, -INFINITY, -1, -INFINITY, -1, {0, 0, 0}};
  for (int i = lane; i < a.nchunks; i += 32) {
    const AccPart* p = a.parts + (int64_t)b * a.nchunks + i;
    t.sum_w += __ldcg(&p->sum_w);
    arg_merge(t.key_w, t.idx_w, __ldcg(&p->key_w), __ldcg(&p->idx_w));
    arg_merge(t.key_p, t.idx_p, __ldcg(&p->key_p), __ldcg(&p->idx_p));
  }
  t.sum_w = warp_sum(t.sum_w);
  warp_arg(t.key_w, t.idx_w);
  warp_arg(t.key_p, t.idx_p);
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
    a.tickets[b] = 0;
  }
}

// ---------------------------------------------------------------------------
// Host side.

int64_t align256(int64_t x) { return (x + 255) & ~int64_t(255); }

int32_t nchunks_of(int32_t vocab) { return (vocab + kChunk - 1) / kChunk; }

// Row workspace: RowPart x rows x nchunks (scratch: written before it is read).
int64_t row_ws_bytes(int64_t rows, int32_t vocab) {
  return align256(rows * nchunks_of(vocab) * (int64_t)sizeof(RowPart));
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
  if (rows * (int64_t)nchunks_of(vocab) > INT32_MAX) {
    pkv_set_error(std::string(who) + ": too many rows for one launch");
    return PKV_ERR_ARG;
  }
  return PKV_OK;
}

int32_t launch_rows(RowArgs a, bool vec, cudaStream_t s, const char* who) {
  if (a.rows == 0) return PKV_OK;
  const unsigned grid = (unsigned)((int64_t)a.rows * a.nchunks);
  if (vec)
    row_stats_kernel<true><<<grid, kThreads, 0, s>>>(a);
  else
    row_stats_kernel<false><<<grid, kThreads, 0, s>>>(a);
  const cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) {
    pkv_set_error(std::string(who) + ": " + cudaGetErrorString(e));
    return PKV_ERR_CUDA;
  }
  return PKV_OK;
}

// Speculative workspace (scratch): [lse_t, lp_t: batch (k+1)][lse_d, lp_d:
// batch k][RowPart: batch (2k+1) x nchunks][AccPart: batch x nchunks].
// Tickets: batch (2k+1) row tickets, then batch accept tickets.
struct SpecWs {
  int64_t lse_t, lp_t, lse_d, lp_d, row_parts, acc_parts, total;
};

SpecWs spec_ws(int64_t batch, int32_t k, int32_t vocab) {
  SpecWs w;
  const int64_t nt = batch * (k + 1), nd = batch * k, nc = nchunks_of(vocab);
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
  a.nchunks = nchunks_of(vocab);
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
  a.nchunks = nchunks_of(vocab);
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
  const int32_t nc = nchunks_of(vocab);
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
  t.nchunks = nc;
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
  a.nchunks = nc;
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
  const unsigned grid = (unsigned)((int64_t)batch * nc);
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
