// TMA tensor maps over the page pool and queries, and the device-side TMA /
// mbarrier helpers shared by the decode and prefill kernels.
#pragma once

#include <cuda.h>

#include "mi_common.cuh"

namespace mi {

// Tensor map over one layer's pool kv_data[P][2][ps][Hkv][D] (bf16/fp16),
// 128-byte swizzle, cached per pool. Per-head boxes: dims (d, head, slot,
// page*2 + kv), box = 64 d x 1 head x 16 slots x 1. All-heads boxes: dims
// (d, slot, head, page*2 + kv), box = 64 d x 16 slots x Hkv heads x 1, which
// lands in shared memory exactly as Hkv per-head boxes placed one after the
// other ([head][slot][64 d]), in one TMA operation.
bool pool_tensor_map(const void *kv, int64_t num_pages, int ps, int hkv, int d, int dtype,
                     CUtensorMap *out, bool all_heads = false);
// Whole-tile tensor map over the same pool: dims (64 d, slot, head, d / 64,
// page*2 + kv), box = 64 x 16 x Hkv x d/64 x 2: one TMA operation brings a
// 16-token tile of K and V, all heads and both halves of head_dim, laid out
// as [kv][d-half][head][slot][64 d]. Cached per pool.
bool pool_tile_tensor_map(const void *kv, int64_t num_pages, int ps, int hkv, int d, int dtype,
                          CUtensorMap *out);
// Tensor map over rows[n][h][d] (element strides sn, sh; d contiguous):
// dims (d, h, n), box = 64 d x box_h x box_n, 128-byte swizzle. Not cached.
bool rows_tensor_map(const void *base, int64_t n, int h, int d, int64_t sn, int64_t sh,
                     int box_h, int box_n, int dtype, CUtensorMap *out);

// 3-/4-D TMA tile loads completing on an mbarrier, with an L2 cache policy.
__device__ __forceinline__ void tma_load_4d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, int c3, uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5}], [%6], %7;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
      "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_5d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, int c3, int c4, uint64_t *bar,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.5d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4, %5, %6}], [%7], %8;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(c4),
      "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

__device__ __forceinline__ void tma_load_3d(void *dst, const CUtensorMap *map, int c0, int c1,
                                            int c2, uint64_t *bar, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.3d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      ".L2::cache_hint [%0], [%1, {%2, %3, %4}], [%5], %6;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(smem_u32(bar)),
      "l"(policy)
      : "memory");
}

// L2 eviction priorities for TMA loads. Decode reads its KV stream once
// (evict-first, so it does not push partials and metadata out of L2) and
// reuses the queries for every KV tile (evict-last); prefill the other way
// round.
__device__ __forceinline__ uint64_t evict_first_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}
__device__ __forceinline__ uint64_t evict_last_policy() {
  uint64_t pol;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
  return pol;
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

// Offset of 16-byte chunk `c` of row `r` in a 128-byte-swizzled box whose
// base is 1024-byte aligned (the hardware XORs the chunk with row % 8).
__device__ __forceinline__ uint32_t swz(int r, int c) {
  return static_cast<uint32_t>(r * 128 + ((c ^ (r & 7)) << 4));
}

}  // namespace mi
