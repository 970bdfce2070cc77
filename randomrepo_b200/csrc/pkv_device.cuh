// Device helpers shared by the paged-KV kernels (sm_100a).
//
// Inline PTX for: mbarriers with bounded waits, TMA tensor loads (no cluster
// multicast anywhere in this library), ldmatrix / movmatrix / mma.sync
// fragments, and the 128-byte shared-memory swizzle that TMA applies.
#pragma once

#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "pkv_b200.h"

namespace pkv {

// Error word values written into a kernel's error slot (host reads them back).
enum DeviceError : int32_t {
  kDevOk = 0,
  kDevWaitTimeout = 1,  // an mbarrier wait hit its iteration limit
  kDevBadSplits = 2,    // a sequence was given more split work items than a kernel supports
  kDevBadItem = 3,      // a work item named a sequence, head group or split outside the launch
  kDevBadBlock = 4,     // a block id outside the pool (replaced by block 0, no access left the pool)
};

// Upper bound of one mbarrier wait, in SM clock cycles (~1 s at 2 GHz).
constexpr long long kWaitLimitCycles = 2000000000ll;

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_barrier_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// Wait for phase `parity` of `bar` to complete.  Returns false (and the
// caller must record an error and leave) if the wait exceeds kWaitLimitCycles.
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t* bar, uint32_t parity) {
  if (mbar_try_wait(bar, parity)) return true;
  long long start = clock64();
  while (!mbar_try_wait(bar, parity)) {
    if (clock64() - start > kWaitLimitCycles) return false;
  }
  return true;
}

// 3-D tiled TMA load into shared memory, completion counted on `bar`.
__device__ __forceinline__ void tma_load_3d(void* smem_dst, const CUtensorMap* map, int32_t x, int32_t y, int32_t z,
                                            uint64_t* bar) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4}], "
      "[%5];" ::"r"(smem_u32(smem_dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(z), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Byte offset of (row, 16-byte chunk) inside a region written by TMA with
// CU_TENSOR_MAP_SWIZZLE_128B: 128-byte rows, chunk index XOR (row mod 8).
// The region must start on a 1024-byte boundary.
__device__ __forceinline__ uint32_t swz128(uint32_t row, uint32_t chunk) {
  return row * 128u + ((chunk ^ (row & 7u)) << 4);
}

__device__ __forceinline__ void ldmatrix_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldmatrix_x4_trans(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2,
                                                  uint32_t& r3) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0, %1, %2, %3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ uint32_t movmatrix_trans(uint32_t x) {
  uint32_t y;
  asm volatile("movmatrix.sync.aligned.m8n8.trans.b16 %0, %1;" : "=r"(y) : "r"(x));
  return y;
}

template <typename T>
struct MmaOp;

template <>
struct MmaOp<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float* d, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ __forceinline__ static __nv_bfloat16 from_float(float x) { return __float2bfloat16_rn(x); }
};

template <>
struct MmaOp<__half> {
  __device__ __forceinline__ static void run(float* d, const uint32_t* a, const uint32_t* b) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b[0]), "r"(b[1]));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t*>(&v);
  }
  __device__ __forceinline__ static __half from_float(float x) { return __float2half_rn(x); }
};

// KV pool layout: pool[layer][block][kv_head][state (0=K, 1=V)][slot][head_dim].
// One (layer, block, kv_head, state) run of block_size rows is a "page"; the
// K and V pages of one head in one block are adjacent, and so are the heads
// of one block, so a block's pages for a group of heads move with one bulk copy.
//
// When a row is a multiple of 128 bytes and block_size a multiple of 8, a page
// is stored pre-swizzled: it is cut into 128-byte column slabs (64 bf16 dims
// each), a slab holds the page's rows at 128 bytes apiece, and the 16-byte
// chunks of row t are permuted by XOR with (t mod 8).  That is the 128-byte
// swizzle TMA applies, so a linear copy of a page into 1024-byte aligned shared
// memory is directly bank-conflict free for ldmatrix and is the canonical
// SWIZZLE_128B operand layout of tcgen05 (K-major for K, MN-major for V).
// Other geometries (rows of 64 bytes, block sizes such as 2) use plain
// row-major pages.
__host__ __device__ __forceinline__ bool page_swizzled(int64_t block_size, int64_t row_bytes) {
  return row_bytes % 128 == 0 && block_size % 8 == 0;
}

// Byte offset of page (layer, block, head, state) from the pool base.
__host__ __device__ __forceinline__ int64_t page_offset(int64_t layer, int64_t block, int64_t head, int64_t state,
                                                        int64_t num_blocks, int64_t num_kv_heads, int64_t block_size,
                                                        int64_t row_bytes) {
  return (((layer * num_blocks + block) * num_kv_heads + head) * 2 + state) * block_size * row_bytes;
}

// Byte offset, inside a page, of byte `b` of row `t`.
__host__ __device__ __forceinline__ int64_t row_byte_offset(int64_t t, int64_t b, int64_t block_size, int64_t row_bytes,
                                                            bool swizzled) {
  if (!swizzled) return t * row_bytes + b;
  const int64_t chunk = b >> 4;
  return (chunk >> 3) * block_size * 128 + t * 128 + (((chunk & 7) ^ (t & 7)) << 4) + (b & 15);
}

}  // namespace pkv
