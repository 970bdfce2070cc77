// Pieces shared by the two paged attention kernels for query chunks: the
// chunked-prefill kernel (prefill.cu, queries on the tensor-core rows) and the
// speculative-verify kernel (verify.cu, keys on the rows).  Both take their
// launch parameters in PrefillParams and write key-range partials in the same
// slot format; the records below are the prefill kernel's (verify.cu
// documents its own, which add per-CTA item lists).
#pragma once

#include "pkv_device.cuh"

// Internal linkage: each kernel file gets its own copy of these kernels.
namespace pkv {
namespace {

constexpr int kRows = 128;             // rows of one prefill query tile; rows of a partial slot
constexpr int kKeys = 128;             // keys per KV tile
constexpr int kPageRows = 16;          // block_size
constexpr int kPagesPerTile = kKeys / kPageRows;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kRescaleLog2 = 8.f;    // keep a stale running maximum while the new one exceeds it by <= 2^8

// Prefill work item (two int4): {table row, position of the item's first query, index
// of that query in the packed q, kv_head << 16 | positions in the item} and
// {first KV tile, one past the last KV tile (0: all of them), partial slot
// (-1: write the output), 0}.  A combine entry (two int4) is {first slot,
// slots, query index, kv_head << 16 | positions}; it merges the slots of one
// group of queries.  A partial slot holds m[128], l[128] and O[128][D] in
// fp32 for rows r = position * G + head (G = query heads per KV head): m the
// running maximum of the scaled logits in base 2, l the sum of 2^(x - m) and O
// the unnormalised sum of 2^(x - m) V.
struct PrefillParams {
  const void* q;    // [total_q][hq][D]
  void* out;        // [total_q][hq][D]
  const char* pool;
  const int32_t* tables;
  const int4* items;
  int32_t* error;
  float* partials;  // n_slots x (m[128], l[128], O[128][D]) fp32
  int32_t n_slots;
  int64_t total_q;
  int32_t n_items;
  int32_t table_stride;
  int32_t table_rows;
  int32_t hq;
  int32_t hkv;
  int32_t group;
  int32_t ppi;      // positions per query tile (prefill: kRows / group; verify: 32 / group)
  int32_t layer;
  int32_t num_blocks;
  float scale_log2;
  int32_t n_combine;   // combine entries (after the items in `items`)
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

// Merge the key-range partials of one group of queries: per row, m = max m_s,
// O = sum_s 2^(m_s - m) O_s / sum_s 2^(m_s - m) l_s, written in the output dtype.
// One block per combine entry, one thread per row.
template <int D, typename T>
__global__ void __launch_bounds__(kRows) paged_prefill_combine_kernel(const __grid_constant__ PrefillParams p,
                                                                     const int4* entries) {
  const int4 e = entries[2 * blockIdx.x];  // records are two int4 apart
  const int slot0 = e.x, ns = e.y, qrow0 = e.z, h = e.w >> 16, nt = e.w & 0xffff;
  const int r = threadIdx.x;
  const int group = p.group;
  if (slot0 < 0 || ns < 1 || slot0 + ns > p.n_slots || nt < 1 || nt * group > kRows || qrow0 < 0 ||
      (int64_t)qrow0 + nt > p.total_q || h < 0 || h >= p.hkv) {
    if (r == 0) atomicExch(p.error, kDevBadItem);
    return;
  }
  if (r >= nt * group) return;
  constexpr int kSlotFloats = 2 * kRows + kRows * D;
  const float* base = p.partials + (int64_t)slot0 * kSlotFloats;
  float m = -INFINITY;
  for (int s = 0; s < ns; ++s) m = fmaxf(m, base[(int64_t)s * kSlotFloats + r]);
  float l = 0.f;
  for (int s = 0; s < ns; ++s) {
    const float ms = base[(int64_t)s * kSlotFloats + r];
    l += ms == -INFINITY ? 0.f : ex2_approx(ms - m) * base[(int64_t)s * kSlotFloats + kRows + r];
  }
  const float inv_l = 1.f / l;
  T* dst = static_cast<T*>(p.out) + (((int64_t)qrow0 + r / group) * p.hq + (int64_t)h * group + r % group) * D;
#pragma unroll 1
  for (int d = 0; d < D; d += 8) {
    float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int s = 0; s < ns; ++s) {
      const float* ps = base + (int64_t)s * kSlotFloats;
      const float ms = ps[r];
      const float w = ms == -INFINITY ? 0.f : ex2_approx(ms - m) * inv_l;
      const float4 a = *reinterpret_cast<const float4*>(ps + 2 * kRows + (int64_t)r * D + d);
      const float4 b = *reinterpret_cast<const float4*>(ps + 2 * kRows + (int64_t)r * D + d + 4);
      acc[0] += w * a.x; acc[1] += w * a.y; acc[2] += w * a.z; acc[3] += w * a.w;
      acc[4] += w * b.x; acc[5] += w * b.y; acc[6] += w * b.z; acc[7] += w * b.w;
    }
    *reinterpret_cast<uint4*>(dst + d) = make_uint4(MmaOp<T>::pack(acc[0], acc[1]), MmaOp<T>::pack(acc[2], acc[3]),
                                                    MmaOp<T>::pack(acc[4], acc[5]), MmaOp<T>::pack(acc[6], acc[7]));
  }
}

}  // namespace
}  // namespace pkv
