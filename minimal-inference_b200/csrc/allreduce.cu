// Tensor-parallel decode: all-reduce of a row-parallel GEMM's partial sums
// over NVLink peer memory, fused with the residual add and RMSNorm that
// follow it.
//
// In a tensor-parallel decoder layer (o_proj and down_proj split by input
// columns) every rank holds a partial [rows, hidden] sum; the reference
// model's next operations are `h = h + x` and F.rms_norm(h) (model.py:115-122,
// :333-343), which the unsharded path runs as add_rmsnorm. Here one kernel
// does all three for decode-sized row counts:
//   * every rank's GEMM has written its partial into its own region of a
//     symmetric buffer (same offset on every rank, each rank's buffer mapped
//     into every other rank's address space);
//   * block b of every rank publishes "partial ready" to its peers by storing
//     its epoch into their flag arrays (P2P store, release, system scope),
//     then waits (bounded) until every peer's block b has done the same;
//   * block b then owns row b (and b + grid, ...): it reads the row from all
//     ranks' partials (P2P loads), sums in fp32, rounds like the all-reduce
//     result, adds the residual (rounded like `h + x`), and normalises.
// Reuse: a call site's region is rewritten only by a later call's GEMM on
// this rank, which runs after this rank's kernel for the call in between has
// passed its own barrier, i.e. after every peer finished reading it.
// No multicast, no TMA: plain loads and stores over NVLink.
#include <cuda.h>
#include <string.h>

#include <mutex>

#include "mi_common.cuh"

namespace mi {
namespace {

constexpr int kArBlocks = 256;  // max rows per call == flag slots per rank
constexpr uint64_t kArWaitNs = 10000000000ull;  // 10 s default: ranks may drift apart
std::atomic<uint64_t> g_peer_wait_ns{kArWaitNs};

struct ArParams {
  const unsigned long long *peer_base;  // [world] each rank's buffer base, in this address space
  int64_t data_off;                     // this call site's [rows][hidden] partial
  int64_t flag_off;                     // flags [world][kArBlocks] uint32
  unsigned *counters;                   // [kArBlocks] this rank's epoch per block
  int rank, world, rows, hidden;
  void *residual;
  const void *weight;
  void *out;
  float eps;
  int32_t *status;
  uint64_t wait_ns;  // give-up limit of the barrier with the peers
};

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
  unsigned v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

template <typename T, int V>
__global__ void __launch_bounds__(1024) ar_add_rmsnorm_kernel(const ArParams p) {
  __shared__ float s_part[32];
  __shared__ int s_ok;
  const int b = blockIdx.x;
  // ---- barrier with the peers' block b -------------------------------------
  if (threadIdx.x == 0) {
    const unsigned e = p.counters[b] + 1u;
    p.counters[b] = e;
    for (int q = 0; q < p.world; ++q)
      if (q != p.rank)
        st_release_sys(reinterpret_cast<unsigned *>(p.peer_base[q] + p.flag_off) +
                           p.rank * kArBlocks + b, e);
    const unsigned *mine = reinterpret_cast<const unsigned *>(p.peer_base[p.rank] + p.flag_off);
    int ok = 1;
    const uint64_t t0 = global_ns();
    for (int q = 0; q < p.world && ok; ++q) {
      if (q == p.rank) continue;
      for (uint32_t i = 0; static_cast<int>(ld_acquire_sys(mine + q * kArBlocks + b) - e) < 0; ++i) {
        if ((i & 255u) == 255u && global_ns() - t0 > p.wait_ns) {
          ok = 0;
          break;
        }
      }
    }
    if (!ok) flag(p.status, MI_STATUS_TIMEOUT);
    s_ok = ok;
  }
  __syncthreads();
  if (!s_ok) return;
  // ---- rows b, b + grid, ...: sum of partials + residual, RMSNorm ----------
  const int nvec = p.hidden >> 3;
  for (int row = b; row < p.rows; row += gridDim.x) {
    const int64_t rbase = static_cast<int64_t>(row) * p.hidden;
    uint4 *rr = reinterpret_cast<uint4 *>(static_cast<T *>(p.residual) + rbase);
    float h[V][8];
    float ss = 0.f;
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int i = threadIdx.x + v * blockDim.x;
      if (i < nvec) {
        float acc[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
        for (int q = 0; q < p.world; ++q) {
          const uint4 *src = reinterpret_cast<const uint4 *>(p.peer_base[q] + p.data_off) +
                             rbase / 8 + i;
          const uint4 x = __ldcg(src);
          const T *xe = reinterpret_cast<const T *>(&x);
#pragma unroll
          for (int j = 0; j < 8; ++j) acc[j] += Elt<T>::to(xe[j]);
        }
        uint4 rv = rr[i];
        T *re = reinterpret_cast<T *>(&rv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float a = Elt<T>::to(Elt<T>::from(acc[j]));  // the all-reduced value
          re[j] = Elt<T>::from(__fadd_rn(Elt<T>::to(re[j]), a));
          h[v][j] = Elt<T>::to(re[j]);
          ss = fmaf(h[v][j], h[v][j], ss);
        }
        rr[i] = rv;
      }
    }
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < static_cast<int>((blockDim.x + 31) >> 5); ++w) tot += s_part[w];
    const float inv = rsqrtf(tot / p.hidden + p.eps);
    const uint4 *wr = reinterpret_cast<const uint4 *>(p.weight);
    uint4 *yr = reinterpret_cast<uint4 *>(static_cast<T *>(p.out) + rbase);
#pragma unroll
    for (int v = 0; v < V; ++v) {
      const int i = threadIdx.x + v * blockDim.x;
      if (i < nvec) {
        const uint4 wv = wr[i];
        const T *we = reinterpret_cast<const T *>(&wv);
        uint4 ov;
        T *oe = reinterpret_cast<T *>(&ov);
#pragma unroll
        for (int j = 0; j < 8; ++j) oe[j] = Elt<T>::from(h[v][j] * inv * Elt<T>::to(we[j]));
        yr[i] = ov;
      }
    }
    __syncthreads();  // s_part is reused by the next row
  }
}

template <typename T>
int launch_ar(const ArParams &p, cudaStream_t s) {
  const int nvec = p.hidden / 8;
  const int threads = nvec < 1024 ? ((nvec + 31) / 32) * 32 : 1024;
  const int v = (nvec + threads - 1) / threads;
  const int grid = p.rows;
  if (v == 1)
    ar_add_rmsnorm_kernel<T, 1><<<grid, threads, 0, s>>>(p);
  else if (v == 2)
    ar_add_rmsnorm_kernel<T, 2><<<grid, threads, 0, s>>>(p);
  else
    ar_add_rmsnorm_kernel<T, 4><<<grid, threads, 0, s>>>(p);
  return check_launch("ar_add_rmsnorm_kernel");
}

}  // namespace
}  // namespace mi

extern "C" int mi_allreduce_add_rmsnorm(const unsigned long long *peer_bases, int64_t data_off,
                                        int64_t flag_off, uint32_t *block_counters,
                                        int32_t rank, int32_t world, void *residual,
                                        const void *weight, void *out, int32_t rows,
                                        int32_t hidden, float eps, int32_t dtype,
                                        int32_t *status, mi_stream_t stream) {
  using namespace mi;
  MI_REQUIRE(world >= 1 && world <= 64 && rank >= 0 && rank < world,
             "allreduce: bad rank %d / world %d", rank, world);
  MI_REQUIRE(rows >= 0 && rows <= kArBlocks, "allreduce: rows %d outside [0, %d]", rows,
             kArBlocks);
  if (rows == 0) return MI_OK;
  MI_REQUIRE(peer_bases && block_counters && residual && weight && out,
             "allreduce: null pointer argument");
  MI_REQUIRE(dtype == MI_DTYPE_BF16 || dtype == MI_DTYPE_F16, "allreduce: dtype must be 16-bit");
  MI_REQUIRE(hidden > 0 && hidden % 8 == 0 && hidden / 8 <= 4 * 1024,
             "allreduce: hidden %d must be a multiple of 8 up to 32768", hidden);
  MI_REQUIRE(data_off % 16 == 0 && flag_off % 16 == 0, "allreduce: offsets must be 16-byte aligned");
  MI_REQUIRE((reinterpret_cast<uintptr_t>(residual) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(weight) & 15) == 0 &&
                 (reinterpret_cast<uintptr_t>(out) & 15) == 0,
             "allreduce: residual / weight / out must be 16-byte aligned");
  ArParams p{peer_bases, data_off, flag_off, block_counters, rank, world, rows, hidden,
             residual, weight, out, eps, status, g_peer_wait_ns.load(std::memory_order_relaxed)};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  return dtype == MI_DTYPE_BF16 ? launch_ar<__nv_bfloat16>(p, s) : launch_ar<__half>(p, s);
}

extern "C" int mi_set_peer_wait_limit_ns(int64_t ns) {
  mi::g_peer_wait_ns.store(ns > 0 ? static_cast<uint64_t>(ns) : mi::kArWaitNs,
                           std::memory_order_relaxed);
  return MI_OK;
}

// ---------------------------------------------------------------------------
// Peer mappings for the symmetric buffer: plain CUDA IPC (cudaIpcGetMemHandle
// / cudaIpcOpenMemHandle), which maps a peer's allocation over NVLink P2P and
// binds nothing to an NVLink multicast object.
// ---------------------------------------------------------------------------
namespace mi {
namespace {
using AddrRangeFn = CUresult (*)(CUdeviceptr *, size_t *, CUdeviceptr);

AddrRangeFn addr_range_fn() {
  static AddrRangeFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void *ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &ptr, 12000, cudaEnableDefault,
                                         &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<AddrRangeFn>(ptr);
  });
  return fn;
}
}  // namespace
}  // namespace mi

extern "C" int mi_ipc_export(const void *ptr, void *handle_out, int64_t *offset_out) {
  using namespace mi;
  MI_REQUIRE(ptr && handle_out && offset_out, "ipc_export: null pointer argument");
  static_assert(sizeof(cudaIpcMemHandle_t) <= MI_IPC_HANDLE_BYTES, "IPC handle size");
  auto fn = addr_range_fn();
  if (!fn) return fail(MI_ERR_CUDA, "ipc_export: cuMemGetAddressRange unavailable");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(MI_ERR_INVALID, "ipc_export: %p is not device memory", ptr);
  cudaIpcMemHandle_t h;
  const cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void *>(base));
  if (e != cudaSuccess)
    return fail(MI_ERR_CUDA,
                "ipc_export: cudaIpcGetMemHandle: %s (memory from cudaMalloc is needed; "
                "expandable segments of the caching allocator cannot be exported)",
                cudaGetErrorString(e));
  memset(handle_out, 0, MI_IPC_HANDLE_BYTES);
  memcpy(handle_out, &h, sizeof(h));
  *offset_out = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return MI_OK;
}

extern "C" int mi_ipc_open(const void *handle, void **base_out) {
  using namespace mi;
  MI_REQUIRE(handle && base_out, "ipc_open: null pointer argument");
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  void *base = nullptr;
  const cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(MI_ERR_CUDA, "ipc_open: cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  }
  *base_out = base;
  return MI_OK;
}

extern "C" int mi_ipc_close(void *base) {
  using namespace mi;
  MI_REQUIRE(base, "ipc_close: null pointer");
  const cudaError_t e = cudaIpcCloseMemHandle(base);
  if (e != cudaSuccess) {
    cudaGetLastError();
    return fail(MI_ERR_CUDA, "ipc_close: cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  }
  return MI_OK;
}
