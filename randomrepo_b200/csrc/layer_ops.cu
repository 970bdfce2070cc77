// Fused elementwise layers of a Qwen2-family decoder step (sm_100a).
//
// A graphed decode step of HF's Qwen2 spends more device time in its eager
// elementwise ops than in attention: RMSNorm is seven kernels (cast, pow,
// mean, add, rsqrt, two multiplies), rotary embedding ten (two multiplies,
// slice, negate, cat and add, for q and for k), the MLP's SiLU and product
// two, the residual add one.  These kernels do the same arithmetic in one
// pass each, with the roundings where torch rounds, so their outputs equal the
// modules' (transformers models/qwen2/modeling_qwen2.py: Qwen2RMSNorm.forward,
// rotate_half / apply_rotary_pos_emb, Qwen2MLP.forward, and the residual adds
// of Qwen2DecoderLayer.forward):
//
//  * rms_norm: y = w * to_dtype(x * rsqrt(mean(x^2) + eps)) with x in fp32,
//    optionally on x = to_dtype(a + b) (the residual add), whose sum is also
//    written out; the mean is a fp32 tree sum (torch's reduction order
//    differs, so the variance can differ in its last bits);
//  * rope: out = to_dtype(to_dtype(x * cos) + to_dtype(rotate_half(x) * sin))
//    for every q and k head of a token row, written head-major [rows][heads][D];
//  * silu_mul: out = to_dtype(to_dtype(g / (1 + exp(-g))) * u).
//
// All three are bandwidth-bound and, at decode batch sizes, latency-bound
// (a step's rows are 100 KB-1 MB): the fast paths move 16-byte vectors of
// eight elements -- a warp per row for the norm (shuffles only, no block
// barrier), eight consecutive columns per thread for the SiLU product, and
// for rope eight columns of a head's first half with the eight they pair with
// in its second half -- and general kernels take shapes whose rows are not
// multiples of eight elements.
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>

#include <string>

#include "pkv_b200.h"
#include "pkv_error.h"

namespace pkv {
namespace {

template <typename T>
struct Cvt;
template <>
struct Cvt<__nv_bfloat16> {
  static __device__ __forceinline__ float f(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 t(float x) { return __float2bfloat16_rn(x); }
};
template <>
struct Cvt<__half> {
  static __device__ __forceinline__ float f(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half t(float x) { return __float2half_rn(x); }
};

// Round a float to T and back (the value torch keeps after an op in T).
template <typename T>
__device__ __forceinline__ float rnd(float x) {
  return Cvt<T>::f(Cvt<T>::t(x));
}

constexpr int kNormThreads = 256;

template <typename T>
__global__ void __launch_bounds__(kNormThreads) rms_norm_kernel(const T* __restrict__ a, const T* __restrict__ b,
                                                                T* __restrict__ sum_out, const T* __restrict__ w,
                                                                T* __restrict__ out, int hidden, float eps) {
  const int64_t row = blockIdx.x;
  const T* ar = a + row * hidden;
  const T* br = b ? b + row * hidden : nullptr;
  // Each thread keeps its columns' fp32 values between the two passes.
  constexpr int kMaxPerThread = 32;  // hidden <= 8192
  float xs[kMaxPerThread];
  float ss = 0.f;
#pragma unroll
  for (int j = 0; j < kMaxPerThread; ++j) {
    const int c = threadIdx.x + j * kNormThreads;
    xs[j] = 0.f;
    if (c < hidden) {
      float x = Cvt<T>::f(ar[c]);
      if (br) {
        x = rnd<T>(x + Cvt<T>::f(br[c]));
        sum_out[row * hidden + c] = Cvt<T>::t(x);
      }
      xs[j] = x;
      ss = fmaf(x, x, ss);
    }
  }
  __shared__ float red[kNormThreads / 32];
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
  __syncthreads();
  if (threadIdx.x < 32) {
    float v = threadIdx.x < kNormThreads / 32 ? red[threadIdx.x] : 0.f;
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
    if (threadIdx.x == 0) red[0] = v;
  }
  __syncthreads();
  const float inv = rsqrtf(red[0] / (float)hidden + eps);
#pragma unroll
  for (int j = 0; j < kMaxPerThread; ++j) {
    const int c = threadIdx.x + j * kNormThreads;
    if (c < hidden) out[row * hidden + c] = Cvt<T>::t(Cvt<T>::f(w[c]) * rnd<T>(xs[j] * inv));
  }
}

// Eight elements of T in one 16-byte vector.
template <typename T>
struct Vec8 {
  uint4 raw;
  __device__ __forceinline__ float get(int i) const {
    const T* e = reinterpret_cast<const T*>(&raw);
    return Cvt<T>::f(e[i]);
  }
  __device__ __forceinline__ void set(int i, float v) {
    T* e = reinterpret_cast<T*>(&raw);
    e[i] = Cvt<T>::t(v);
  }
};

template <typename T>
__device__ __forceinline__ Vec8<T> ld8(const T* p) {
  Vec8<T> v;
  v.raw = *reinterpret_cast<const uint4*>(p);
  return v;
}

template <typename T>
__device__ __forceinline__ void st8(T* p, const Vec8<T>& v) {
  *reinterpret_cast<uint4*>(p) = v.raw;
}

constexpr int kNormWarps = 4;

// A warp per row; hidden % 8 == 0 and 16-byte aligned rows.  Pass 1 folds the
// residual (storing the sum) and accumulates x^2; pass 2 re-reads the row
// (its own sum writes, or the input, from L1 / L2) and writes the output.
template <typename T>
__global__ void __launch_bounds__(kNormWarps * 32) rms_norm_warp_kernel(const T* __restrict__ a,
                                                                        const T* __restrict__ b,
                                                                        T* __restrict__ sum_out,
                                                                        const T* __restrict__ w,
                                                                        T* __restrict__ out, int64_t rows,
                                                                        int hidden, float eps) {
  const int64_t row = (int64_t)blockIdx.x * kNormWarps + (threadIdx.x >> 5);
  if (row >= rows) return;
  const int lane = threadIdx.x & 31;
  const int nvec = hidden >> 3;
  const T* ar = a + row * hidden;
  const T* br = b ? b + row * hidden : nullptr;
  T* sr = sum_out ? sum_out + row * hidden : nullptr;
  float ss = 0.f;
  for (int v = lane; v < nvec; v += 32) {
    Vec8<T> x = ld8(ar + 8 * v);
    if (br) {
      const Vec8<T> y = ld8(br + 8 * v);
#pragma unroll
      for (int i = 0; i < 8; ++i) x.set(i, x.get(i) + y.get(i));
      st8(sr + 8 * v, x);
    }
#pragma unroll
    for (int i = 0; i < 8; ++i) ss = fmaf(x.get(i), x.get(i), ss);
  }
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, off);
  const float inv = rsqrtf(ss / (float)hidden + eps);
  const T* src = sr ? sr : ar;
  T* orow = out + row * hidden;
  for (int v = lane; v < nvec; v += 32) {
    const Vec8<T> x = ld8(src + 8 * v);
    const Vec8<T> g = ld8(w + 8 * v);
    Vec8<T> o;
#pragma unroll
    for (int i = 0; i < 8; ++i) o.set(i, g.get(i) * rnd<T>(x.get(i) * inv));
    st8(orow + 8 * v, o);
  }
}

// Rope on 16-byte vectors: a thread takes columns [8j, 8j + 8) of a head's
// first half and the eight they pair with in its second half (d % 16 == 0,
// row strides multiples of 8 elements).  One CTA per token row.
template <typename T>
__global__ void rope_vec_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                                const T* __restrict__ cosv, const T* __restrict__ sinv, T* __restrict__ q_out,
                                T* __restrict__ k_out, T* __restrict__ v_out, int64_t q_ld, int64_t k_ld,
                                int64_t v_ld, int hq, int hkv, int d) {
  const int64_t row = blockIdx.x;
  const int half = d >> 1, per_head = half >> 3;
  const T* c = cosv + row * d;
  const T* s = sinv + row * d;
  const int n = (hq + hkv) * per_head;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int h = i / per_head, e = (i - h * per_head) * 8;
    const bool is_q = h < hq;
    const T* x = is_q ? q + row * q_ld + h * d : k + row * k_ld + (h - hq) * d;
    T* o = is_q ? q_out + (row * hq + h) * d : k_out + (row * hkv + (h - hq)) * d;
    const Vec8<T> lo = ld8(x + e), hi = ld8(x + e + half);
    const Vec8<T> cl = ld8(c + e), ch = ld8(c + e + half), sl = ld8(s + e), sh = ld8(s + e + half);
    Vec8<T> ol, oh;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      // rotate_half: first half pairs with -second half, second half with first half.
      ol.set(j, rnd<T>(lo.get(j) * cl.get(j)) + rnd<T>(-hi.get(j) * sl.get(j)));
      oh.set(j, rnd<T>(hi.get(j) * ch.get(j)) + rnd<T>(lo.get(j) * sh.get(j)));
    }
    st8(o + e, ol);
    st8(o + e + half, oh);
  }
  if (v) {
    for (int i = threadIdx.x; i < hkv * d / 8; i += blockDim.x) st8(v_out + row * hkv * d + 8 * i, ld8(v + row * v_ld + 8 * i));
  }
}

// SiLU product on 16-byte vectors (cols % 8 == 0, ld_in % 8 == 0): a CTA
// takes 2048 columns of one row, a thread eight of them.
template <typename T>
__global__ void silu_mul_vec_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ out, int chunks,
                                    int64_t ld_in, int cols) {
  const int64_t r = blockIdx.x / chunks;
  const int c0 = (int)(blockIdx.x - r * chunks) * 2048;
  const int c = c0 + 8 * threadIdx.x;
  if (c >= cols) return;
  const Vec8<T> gv = ld8(g + r * ld_in + c), uv = ld8(u + r * ld_in + c);
  Vec8<T> o;
#pragma unroll
  for (int j = 0; j < 8; ++j) {
    const float x = gv.get(j);
    o.set(j, rnd<T>(x / (1.f + expf(-x))) * uv.get(j));
  }
  st8(out + r * (int64_t)cols + c, o);
}

// One CTA per token row: q heads, then k heads (rotated), then v heads
// (copied, when given); inputs rows q_ld / k_ld / v_ld elements apart (one
// packed q|k|v projection row, or three tensors), outputs contiguous.
template <typename T>
__global__ void rope_kernel(const T* __restrict__ q, const T* __restrict__ k, const T* __restrict__ v,
                            const T* __restrict__ cosv, const T* __restrict__ sinv, T* __restrict__ q_out,
                            T* __restrict__ k_out, T* __restrict__ v_out, int64_t q_ld, int64_t k_ld, int64_t v_ld,
                            int hq, int hkv, int d) {
  const int64_t row = blockIdx.x;
  const int half = d >> 1;
  const T* c = cosv + row * d;
  const T* s = sinv + row * d;
  const int n = (hq + hkv) * d;
  for (int i = threadIdx.x; i < n; i += blockDim.x) {
    const int h = i / d, e = i - h * d;
    const bool is_q = h < hq;
    const T* x = is_q ? q + row * q_ld + h * d : k + row * k_ld + (h - hq) * d;
    T* o = is_q ? q_out + (row * hq + h) * d : k_out + (row * hkv + (h - hq)) * d;
    const float xv = Cvt<T>::f(x[e]);
    const float rot = e < half ? -Cvt<T>::f(x[e + half]) : Cvt<T>::f(x[e - half]);
    o[e] = Cvt<T>::t(rnd<T>(xv * Cvt<T>::f(c[e])) + rnd<T>(rot * Cvt<T>::f(s[e])));
  }
  if (v) {
    for (int i = threadIdx.x; i < hkv * d; i += blockDim.x) v_out[row * hkv * d + i] = v[row * v_ld + i];
  }
}

constexpr int kSiluCols = 2048;  // columns per CTA

template <typename T>
__global__ void silu_mul_kernel(const T* __restrict__ g, const T* __restrict__ u, T* __restrict__ out, int chunks,
                                int64_t ld_in, int cols) {
  // CTA = (row, chunk of kSiluCols columns) of a [rows][cols] result; gate /
  // up rows are ld_in elements apart.
  const int64_t r = blockIdx.x / chunks;
  const int c0 = (int)(blockIdx.x - r * chunks) * kSiluCols;
  const int c1 = min(cols, c0 + kSiluCols);
  const T* gr = g + r * ld_in;
  const T* ur = u + r * ld_in;
  T* orow = out + r * cols;
  for (int c = c0 + threadIdx.x; c < c1; c += blockDim.x) {
    const float gv = Cvt<T>::f(gr[c]);
    const float sv = rnd<T>(gv / (1.f + expf(-gv)));
    orow[c] = Cvt<T>::t(sv * Cvt<T>::f(ur[c]));
  }
}

bool aligned16(const void* p) { return ((uintptr_t)p & 15) == 0; }

int32_t cuda_status(cudaError_t e, const char* what) {
  if (e == cudaSuccess) return PKV_OK;
  pkv_set_error(std::string(what) + ": " + cudaGetErrorString(e));
  return PKV_ERR_CUDA;
}

}  // namespace
}  // namespace pkv

using namespace pkv;

extern "C" {

int32_t pkv_rms_norm(const void* x, const void* residual, void* sum_out, const void* weight, void* out, int64_t rows,
                     int32_t hidden, float eps, int32_t dtype, void* stream) {
  pkv_clear_error();
  if (!x || !weight || !out || rows < 0 || hidden <= 0 || hidden > 32 * kNormThreads ||
      (residual != nullptr) != (sum_out != nullptr)) {
    pkv_set_error("pkv_rms_norm: invalid arguments (hidden 1..8192; residual and sum_out together)");
    return PKV_ERR_ARG;
  }
  if (dtype != PKV_BF16 && dtype != PKV_F16) {
    pkv_set_error("pkv_rms_norm: bf16 or f16");
    return PKV_ERR_UNSUPPORTED;
  }
  if (rows == 0) return PKV_OK;
  auto s = static_cast<cudaStream_t>(stream);
  const bool vec = hidden % 8 == 0 && aligned16(x) && aligned16(weight) && aligned16(out) && aligned16(residual) &&
                   aligned16(sum_out);
  if (vec) {
    const unsigned blocks = (unsigned)((rows + kNormWarps - 1) / kNormWarps);
    if (dtype == PKV_BF16) {
      using T = __nv_bfloat16;
      rms_norm_warp_kernel<T><<<blocks, kNormWarps * 32, 0, s>>>(
          static_cast<const T*>(x), static_cast<const T*>(residual), static_cast<T*>(sum_out),
          static_cast<const T*>(weight), static_cast<T*>(out), rows, hidden, eps);
    } else {
      using T = __half;
      rms_norm_warp_kernel<T><<<blocks, kNormWarps * 32, 0, s>>>(
          static_cast<const T*>(x), static_cast<const T*>(residual), static_cast<T*>(sum_out),
          static_cast<const T*>(weight), static_cast<T*>(out), rows, hidden, eps);
    }
    return cuda_status(cudaGetLastError(), "pkv_rms_norm launch");
  }
  if (dtype == PKV_BF16) {
    using T = __nv_bfloat16;
    rms_norm_kernel<T><<<(unsigned)rows, kNormThreads, 0, s>>>(
        static_cast<const T*>(x), static_cast<const T*>(residual), static_cast<T*>(sum_out),
        static_cast<const T*>(weight), static_cast<T*>(out), hidden, eps);
  } else {
    using T = __half;
    rms_norm_kernel<T><<<(unsigned)rows, kNormThreads, 0, s>>>(
        static_cast<const T*>(x), static_cast<const T*>(residual), static_cast<T*>(sum_out),
        static_cast<const T*>(weight), static_cast<T*>(out), hidden, eps);
  }
  return cuda_status(cudaGetLastError(), "pkv_rms_norm launch");
}

int32_t pkv_rope(const void* q, const void* k, const void* v, const void* cos, const void* sin, void* q_out,
                 void* k_out, void* v_out, int64_t rows, int64_t q_ld, int64_t k_ld, int64_t v_ld, int32_t q_heads,
                 int32_t kv_heads, int32_t head_dim, int32_t dtype, void* stream) {
  pkv_clear_error();
  if (!q || !k || !cos || !sin || !q_out || !k_out || (v != nullptr) != (v_out != nullptr) || rows < 0 ||
      q_heads <= 0 || kv_heads <= 0 || head_dim <= 0 || head_dim % 2 || q_ld < (int64_t)q_heads * head_dim ||
      k_ld < (int64_t)kv_heads * head_dim || (v && v_ld < (int64_t)kv_heads * head_dim)) {
    pkv_set_error("pkv_rope: invalid arguments");
    return PKV_ERR_ARG;
  }
  if (dtype != PKV_BF16 && dtype != PKV_F16) {
    pkv_set_error("pkv_rope: bf16 or f16");
    return PKV_ERR_UNSUPPORTED;
  }
  if (rows == 0) return PKV_OK;
  auto s = static_cast<cudaStream_t>(stream);
  const bool vec = head_dim % 16 == 0 && q_ld % 8 == 0 && k_ld % 8 == 0 && (!v || v_ld % 8 == 0) && aligned16(q) &&
                   aligned16(k) && aligned16(v) && aligned16(cos) && aligned16(sin) && aligned16(q_out) &&
                   aligned16(k_out) && aligned16(v_out);
  if (vec) {
    const int threads = 128;
    if (dtype == PKV_BF16) {
      using T = __nv_bfloat16;
      rope_vec_kernel<T><<<(unsigned)rows, threads, 0, s>>>(
          static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<const T*>(cos),
          static_cast<const T*>(sin), static_cast<T*>(q_out), static_cast<T*>(k_out), static_cast<T*>(v_out), q_ld,
          k_ld, v_ld, q_heads, kv_heads, head_dim);
    } else {
      using T = __half;
      rope_vec_kernel<T><<<(unsigned)rows, threads, 0, s>>>(
          static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<const T*>(cos),
          static_cast<const T*>(sin), static_cast<T*>(q_out), static_cast<T*>(k_out), static_cast<T*>(v_out), q_ld,
          k_ld, v_ld, q_heads, kv_heads, head_dim);
    }
    return cuda_status(cudaGetLastError(), "pkv_rope launch");
  }
  const int threads = 256;
  if (dtype == PKV_BF16) {
    using T = __nv_bfloat16;
    rope_kernel<T><<<(unsigned)rows, threads, 0, s>>>(
        static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<const T*>(cos),
        static_cast<const T*>(sin), static_cast<T*>(q_out), static_cast<T*>(k_out), static_cast<T*>(v_out), q_ld,
        k_ld, v_ld, q_heads, kv_heads, head_dim);
  } else {
    using T = __half;
    rope_kernel<T><<<(unsigned)rows, threads, 0, s>>>(
        static_cast<const T*>(q), static_cast<const T*>(k), static_cast<const T*>(v), static_cast<const T*>(cos),
        static_cast<const T*>(sin), static_cast<T*>(q_out), static_cast<T*>(k_out), static_cast<T*>(v_out), q_ld,
        k_ld, v_ld, q_heads, kv_heads, head_dim);
  }
  return cuda_status(cudaGetLastError(), "pkv_rope launch");
}

int32_t pkv_silu_mul(const void* gate, const void* up, void* out, int64_t rows, int64_t cols, int64_t ld_in,
                     int32_t dtype, void* stream) {
  pkv_clear_error();
  if (!gate || !up || !out || rows < 0 || cols <= 0 || cols > (1 << 30) || ld_in < cols) {
    pkv_set_error("pkv_silu_mul: invalid arguments");
    return PKV_ERR_ARG;
  }
  if (dtype != PKV_BF16 && dtype != PKV_F16) {
    pkv_set_error("pkv_silu_mul: bf16 or f16");
    return PKV_ERR_UNSUPPORTED;
  }
  if (rows == 0) return PKV_OK;
  const int chunks = (int)((cols + kSiluCols - 1) / kSiluCols);
  if (rows * chunks > 0x7fffffffll) {
    pkv_set_error("pkv_silu_mul: too many rows");
    return PKV_ERR_ARG;
  }
  auto s = static_cast<cudaStream_t>(stream);
  const unsigned blocks = (unsigned)(rows * chunks);
  if (cols % 8 == 0 && ld_in % 8 == 0 && aligned16(gate) && aligned16(up) && aligned16(out)) {
    if (dtype == PKV_BF16) {
      using T = __nv_bfloat16;
      silu_mul_vec_kernel<T><<<blocks, kSiluCols / 8, 0, s>>>(static_cast<const T*>(gate), static_cast<const T*>(up),
                                                              static_cast<T*>(out), chunks, ld_in, (int)cols);
    } else {
      using T = __half;
      silu_mul_vec_kernel<T><<<blocks, kSiluCols / 8, 0, s>>>(static_cast<const T*>(gate), static_cast<const T*>(up),
                                                              static_cast<T*>(out), chunks, ld_in, (int)cols);
    }
    return cuda_status(cudaGetLastError(), "pkv_silu_mul launch");
  }
  const int threads = 256;
  if (dtype == PKV_BF16) {
    using T = __nv_bfloat16;
    silu_mul_kernel<T><<<blocks, threads, 0, s>>>(static_cast<const T*>(gate), static_cast<const T*>(up),
                                                  static_cast<T*>(out), chunks, ld_in, (int)cols);
  } else {
    using T = __half;
    silu_mul_kernel<T><<<blocks, threads, 0, s>>>(static_cast<const T*>(gate), static_cast<const T*>(up),
                                                  static_cast<T*>(out), chunks, ld_in, (int)cols);
  }
  return cuda_status(cudaGetLastError(), "pkv_silu_mul launch");
}

}  // extern "C"
