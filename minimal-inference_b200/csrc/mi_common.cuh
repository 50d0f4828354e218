// Shared helpers for the paged-KV kernels (sm_100a).
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <atomic>
#include <utility>

#include "../../include/mi_paged.h"

namespace mi {

// ---------------------------------------------------------------------------
// host-side error reporting
// ---------------------------------------------------------------------------
void set_error(const char *fmt, ...);
int fail(int code, const char *fmt, ...);
int check_launch(const char *what);
int num_sms();

// Raise `kernel`'s dynamic shared-memory limit to `bytes` once per device
// (`done` keeps one bit per device; safe when several host threads launch).
// Setting the attribute twice is harmless, so racing first calls need no lock.
template <typename K>
cudaError_t smem_limit_once(std::atomic<unsigned long long> &done, K kernel, int bytes) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e;
  const unsigned long long bit = 1ull << (dev & 63);
  if (done.load(std::memory_order_acquire) & bit) return cudaSuccess;
  e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess) done.fetch_or(bit, std::memory_order_release);
  return e;
}

#define MI_REQUIRE(cond, ...)                           \
  do {                                                  \
    if (!(cond)) return ::mi::fail(MI_ERR_INVALID, __VA_ARGS__); \
  } while (0)

// ---------------------------------------------------------------------------
// element types
// ---------------------------------------------------------------------------
template <typename T> struct Elt;
template <> struct Elt<float> {
  __device__ __forceinline__ static float to(float x) { return x; }
  __device__ __forceinline__ static float from(float x) { return x; }
};
template <> struct Elt<__half> {
  __device__ __forceinline__ static float to(__half x) { return __half2float(x); }
  __device__ __forceinline__ static __half from(float x) { return __float2half_rn(x); }
};
template <> struct Elt<__nv_bfloat16> {
  __device__ __forceinline__ static float to(__nv_bfloat16 x) { return __bfloat162float(x); }
  __device__ __forceinline__ static __nv_bfloat16 from(float x) { return __float2bfloat16_rn(x); }
};

inline int elt_size(int dtype) { return dtype == MI_DTYPE_F32 ? 4 : 2; }

// OR a status bit into the caller's device status word (if any).
__device__ __forceinline__ void flag(int32_t *status, int32_t bit) {
  if (status) atomicOr(status, bit);
}

__device__ __forceinline__ int cdiv(int a, int b) { return (a + b - 1) / b; }

// Token count of request b: (n-1)*ps + last if n > 0 pages, else 0
// (FlashInfer paged_kv_t::get_length semantics). last is clamped to
// [0, ps] so a malformed value can never index past the request's pages.
__device__ __forceinline__ int kv_len_of(const int32_t *indptr, const int32_t *last, int b,
                                         int ps) {
  const int n = indptr[b + 1] - indptr[b];
  return n > 0 ? (n - 1) * ps + min(max(last[b], 0), ps) : 0;
}

// ---------------------------------------------------------------------------
// PTX wrappers: mbarrier, bulk copy (TMA engine), ldmatrix, mma.sync
// ---------------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void *p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
               "r"(bytes)
               : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t phase) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(phase)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait: gives up after `limit_ns` of wall time and returns false (the
// caller records MI_STATUS_TIMEOUT and stops), so a lost transaction can never
// hang the GPU.
constexpr uint64_t kWaitLimitNs = 2000000000ull;  // 2 s
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t phase,
                                                  uint64_t limit_ns = kWaitLimitNs) {
  if (mbar_try_wait(bar, phase)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t i = 1;; ++i) {
    if (mbar_try_wait(bar, phase)) return true;
    if ((i & 255u) == 0 && global_ns() - t0 > limit_ns) return false;
  }
}

// Bulk global->shared copy through the TMA engine, completing on an mbarrier.
// dst/src 16-byte aligned, bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes,
                                         uint64_t *bar) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar))
      : "memory");
}

// Non-blocking prefetch of the 128-byte line holding `p` into this SM's L1.
__device__ __forceinline__ void prefetch_l1(const void *p) {
  asm volatile("prefetch.global.L1 [%0];" ::"l"(p));
}

__device__ __forceinline__ void ldsm_x4(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3,
                                        uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

__device__ __forceinline__ void ldsm_x4_t(uint32_t &r0, uint32_t &r1, uint32_t &r2, uint32_t &r3,
                                          uint32_t addr) {
  asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
               : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
               : "r"(addr));
}

template <typename T> struct Mma;
// D = A(16x16, row) * B(16x8, col) + D, fp32 accumulate.
template <> struct Mma<__nv_bfloat16> {
  __device__ __forceinline__ static void run(float *d, const uint32_t *a, uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __nv_bfloat162 v = __floats2bfloat162_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
  }
};
template <> struct Mma<__half> {
  __device__ __forceinline__ static void run(float *d, const uint32_t *a, uint32_t b0,
                                             uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, "
        "{%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
  }
  __device__ __forceinline__ static uint32_t pack(float lo, float hi) {
    __half2 v = __floats2half2_rn(lo, hi);
    return *reinterpret_cast<uint32_t *>(&v);
  }
};

// One RoPE output element before its final rounding (model.py:101-107):
// round(round(x*c) + round(r*s)) with the outer round done by the store; no
// FMA contraction, so pages and queries hold the reference's bits. Shared by
// the append kernel and the decode kernel's fused append.
template <typename T>
__device__ __forceinline__ float rope1(float x, float r, float c, float s) {
  const float a = Elt<T>::to(Elt<T>::from(__fmul_rn(x, c)));
  const float b = Elt<T>::to(Elt<T>::from(__fmul_rn(r, s)));
  return __fadd_rn(a, b);
}

// Programmatic dependent launch. A kernel launched with launch_pdl() may
// start while its predecessor in the stream is still running; it must call
// pdl_wait() before touching any memory (pdl_wait returns once every
// prerequisite grid has completed and its writes are visible). pdl_trigger()
// lets the next PDL-launched kernel get scheduled early.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_trigger() {
  asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

template <typename... KArgs, typename... Args>
inline cudaError_t launch_pdl(void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                              cudaStream_t stream, Args &&...args) {
  cudaLaunchConfig_t cfg{};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = stream;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}
__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

}  // namespace mi
