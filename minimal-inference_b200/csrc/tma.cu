// Host side of the TMA tensor maps (cuTensorMapEncodeTiled through the
// runtime's driver entry point; no libcuda link needed).
#include <cudaTypedefs.h>

#include <mutex>

#include "tma.cuh"

namespace mi {
namespace {

PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &ptr, 12000,
                                         cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(ptr);
  });
  return fn;
}

CUtensorMapDataType map_type(int dtype) {
  return dtype == MI_DTYPE_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16
                                : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
}

struct MapEntry {
  const void *base;
  int64_t pages;
  int ps, hkv, d, dtype, all_heads;
  CUtensorMap map;
};

std::mutex g_map_mu;
MapEntry g_maps[512];
int g_map_count = 0, g_map_next = 0;

}  // namespace

bool pool_tensor_map(const void *kv, int64_t num_pages, int ps, int hkv, int d, int dtype,
                     CUtensorMap *out, bool all_heads) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  const int ah = all_heads ? 1 : 0;
  for (int i = 0; i < g_map_count; ++i) {
    const MapEntry &e = g_maps[i];
    if (e.base == kv && e.pages == num_pages && e.ps == ps && e.hkv == hkv && e.d == d &&
        e.dtype == dtype && e.all_heads == ah) {
      *out = e.map;
      return true;
    }
  }
  auto fn = encode_fn();
  if (!fn) return false;
  const cuuint64_t es = 2;
  const cuuint64_t slot_stride = static_cast<cuuint64_t>(hkv) * d * es;
  const cuuint64_t head_stride = static_cast<cuuint64_t>(d) * es;
  const cuuint64_t plane_stride = static_cast<cuuint64_t>(ps) * hkv * d * es;
  // per-head boxes: dims (d, head, slot, plane); all-heads boxes: dims
  // (d, slot, head, plane), so a box lands as [head][slot][64 d] like the
  // per-head boxes side by side
  cuuint64_t dims[4] = {static_cast<cuuint64_t>(d),
                        static_cast<cuuint64_t>(all_heads ? ps : hkv),
                        static_cast<cuuint64_t>(all_heads ? hkv : ps),
                        static_cast<cuuint64_t>(num_pages) * 2};
  cuuint64_t strides[3] = {all_heads ? slot_stride : head_stride,
                           all_heads ? head_stride : slot_stride, plane_stride};
  cuuint32_t box[4] = {64, all_heads ? 16u : 1u, all_heads ? static_cast<cuuint32_t>(hkv) : 16u,
                       1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  MapEntry e{kv, num_pages, ps, hkv, d, dtype, ah, {}};
  if (fn(&e.map, map_type(dtype), 4, const_cast<void *>(kv), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  if (g_map_count < 512) {
    g_maps[g_map_count++] = e;
  } else {
    g_maps[g_map_next] = e;
    g_map_next = (g_map_next + 1) % 512;
  }
  *out = e.map;
  return true;
}

bool pool_tile_tensor_map(const void *kv, int64_t num_pages, int ps, int hkv, int d, int dtype,
                          CUtensorMap *out) {
  std::lock_guard<std::mutex> lock(g_map_mu);
  for (int i = 0; i < g_map_count; ++i) {
    const MapEntry &e = g_maps[i];
    if (e.base == kv && e.pages == num_pages && e.ps == ps && e.hkv == hkv && e.d == d &&
        e.dtype == dtype && e.all_heads == 2) {
      *out = e.map;
      return true;
    }
  }
  auto fn = encode_fn();
  if (!fn || d % 64) return false;
  const cuuint64_t es = 2;
  cuuint64_t dims[5] = {64, static_cast<cuuint64_t>(ps), static_cast<cuuint64_t>(hkv),
                        static_cast<cuuint64_t>(d / 64), static_cast<cuuint64_t>(num_pages) * 2};
  cuuint64_t strides[4] = {static_cast<cuuint64_t>(hkv) * d * es,       // slot
                           static_cast<cuuint64_t>(d) * es,             // head
                           64 * es,                                     // d-half
                           static_cast<cuuint64_t>(ps) * hkv * d * es}; // plane
  cuuint32_t box[5] = {64, 16, static_cast<cuuint32_t>(hkv), static_cast<cuuint32_t>(d / 64), 2};
  cuuint32_t estr[5] = {1, 1, 1, 1, 1};
  MapEntry e{kv, num_pages, ps, hkv, d, dtype, 2, {}};
  if (fn(&e.map, map_type(dtype), 5, const_cast<void *>(kv), dims, strides, box, estr,
         CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
         CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) != CUDA_SUCCESS)
    return false;
  if (g_map_count < 512) {
    g_maps[g_map_count++] = e;
  } else {
    g_maps[g_map_next] = e;
    g_map_next = (g_map_next + 1) % 512;
  }
  *out = e.map;
  return true;
}

bool rows_tensor_map(const void *base, int64_t n, int h, int d, int64_t sn, int64_t sh,
                     int box_h, int box_n, int dtype, CUtensorMap *out) {
  auto fn = encode_fn();
  if (!fn || (reinterpret_cast<uintptr_t>(base) & 15) || (sn * 2) % 16 || (sh * 2) % 16)
    return false;
  cuuint64_t dims[3] = {static_cast<cuuint64_t>(d), static_cast<cuuint64_t>(h),
                        static_cast<cuuint64_t>(n)};
  cuuint64_t strides[2] = {static_cast<cuuint64_t>(sh) * 2, static_cast<cuuint64_t>(sn) * 2};
  cuuint32_t box[3] = {64, static_cast<cuuint32_t>(box_h), static_cast<cuuint32_t>(box_n)};
  cuuint32_t estr[3] = {1, 1, 1};
  return fn(out, map_type(dtype), 3, const_cast<void *>(base), dims, strides, box, estr,
            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
            CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
            CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace mi
