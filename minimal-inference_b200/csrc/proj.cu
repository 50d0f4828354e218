// Small-M projections of the decode step: Y[M, N] = X[M, K] W[N, K]^T (+ b)
// for M <= 32 token rows (model.py's nn.Linear layers at decode batch sizes).
//
// At a few rows the step streams W once from HBM and does almost no math, so
// the kernel is built for bandwidth: W tiles of 128 rows x 64 K (16 KB) come
// in by TMA through a five-stage ring; the tensor core computes the
// transposed product Y^T = W X^T with W as the 128-row operand and the (at
// most) 32 token rows as the N = 32 operand (tcgen05 kind::f16, fp32
// accumulator in 32 TMEM columns). K is split across CTAs so that every SM
// streams (up to two CTAs per SM): the splits of one 128-column block form a
// thread-block cluster, each leaves its fp32 partial in its own shared
// memory, and after a cluster barrier each sums its share of the rows over
// all ranks' partials in rank order (distributed shared memory), so the
// result does not depend on which split finished first. Launched as a
// programmatic dependent: the first stages of W (which no kernel writes) are
// requested before the wait for the predecessor, only X after it.
// 192 threads: warp 0 TMA producer, warp 1 MMA issuer (one thread),
// warps 2-5 epilogue (thread = TMEM lane = output column).
#include <algorithm>
#include <type_traits>

#include "tma.cuh"
#include "umma.cuh"

namespace mi {
namespace {

constexpr int kPBN = 128;      // output columns (W rows) per block
constexpr int kPBK = 64;       // K per stage (one 128-byte swizzled row)
constexpr int kPBM = 32;       // token rows (MMA N)
constexpr int kPStages = 5;
constexpr int kPMaxSplits = 8;  // cluster size (portable limit)
constexpr int kPThreads = 192;
constexpr int kPWBytes = kPBN * 128;  // 16 KB
constexpr int kPXBytes = kPBM * 128;  // 4 KB
constexpr int kPSmem = kPStages * (kPWBytes + kPXBytes) + 256 + 1024;

struct ProjParams {
  void *y;
  const void *bias;  // [N] or null
  int32_t *status;
  int m, n, k, ldy, splits, ksteps;  // splits = cluster size along K
};

// all threads of all CTAs of the cluster; orders each thread's earlier
// shared-memory writes before the other CTAs' reads after it
__device__ __forceinline__ void cluster_sync_all() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" :::
                   "memory");
}

// 16 bytes at the same shared-memory offset in cluster rank `rank`
__device__ __forceinline__ float4 ld_cluster_v4(uint32_t local_addr, uint32_t rank) {
  uint32_t remote;
  float4 v;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(remote) : "r"(local_addr), "r"(rank));
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
               : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
               : "r"(remote)
               : "memory");
  return v;
}

template <typename T>
__global__ void __launch_bounds__(kPThreads, 2)
    proj_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap xmap,
                const ProjParams p) {
  extern __shared__ unsigned char smem_raw[];
  unsigned char *smem = reinterpret_cast<unsigned char *>(
      (reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  unsigned char *sw = smem;                                 // [stage][128 rows][128 B]
  unsigned char *sx = smem + kPStages * kPWBytes;           // [stage][32 rows][128 B]
  uint64_t *bars = reinterpret_cast<uint64_t *>(sx + kPStages * kPXBytes);
  uint64_t *full = bars, *empty = bars + kPStages, *done = bars + 2 * kPStages;
  uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(bars + 2 * kPStages + 1);
  float *part = reinterpret_cast<float *>(sw);  // [32 rows][128 cols], once the stages are idle

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int nb = blockIdx.x / p.splits, split = blockIdx.x % p.splits;
  // this CTA's K steps: an even share, the first (ksteps % splits) one longer
  const int base = p.ksteps / p.splits, extra = p.ksteps % p.splits;
  const int k0 = split * base + min(split, extra);
  const int nk = base + (split < extra ? 1 : 0);

  if (warp == 1) {
    if (lane == 0) {
      for (int i = 0; i < kPStages; ++i) {
        mbar_init(&full[i], 1);
        mbar_init(&empty[i], 1);
      }
      mbar_init(done, 1);
    }
    __syncwarp();
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 32;" ::"r"(
                     smem_u32(tmem_slot))
                 : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  fence_mbar_init();
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  bool ok = true;
  float v[32];  // epilogue: this thread's column of the accumulator, rows 0..31

  if (warp == 0) {
    // ============================ producer ==================================
    if (lane == 0) {
      const uint64_t pol_w = evict_first_policy(), pol_x = evict_last_policy();
      // the first stages' W before the predecessor is waited for; X (its
      // output) after
      const int npre = min(nk, kPStages);
      for (int i = 0; i < npre; ++i) {
        mbar_arrive_expect_tx(&full[i], kPWBytes + kPXBytes);
        tma_load_3d(sw + i * kPWBytes, &wmap, (k0 + i) * kPBK, 0, nb * kPBN, &full[i], pol_w);
      }
      pdl_wait();
      for (int i = 0; i < npre; ++i)
        tma_load_3d(sx + i * kPXBytes, &xmap, (k0 + i) * kPBK, 0, 0, &full[i], pol_x);
      for (int i = npre; i < nk; ++i) {
        const int st = i % kPStages;
        if (!mbar_wait_bounded(&empty[st], ((i / kPStages) - 1) & 1)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(&full[st], kPWBytes + kPXBytes);
        const int kc = (k0 + i) * kPBK;
        tma_load_3d(sw + st * kPWBytes, &wmap, kc, 0, nb * kPBN, &full[st], pol_w);
        tma_load_3d(sx + st * kPXBytes, &xmap, kc, 0, 0, &full[st], pol_x);
      }
      // no copy may be in flight when the CTA retires
      for (int i = max(0, nk - kPStages); i < nk && ok; ++i)
        if (!mbar_wait_bounded(&full[i % kPStages], (i / kPStages) & 1)) ok = false;
    }
    __syncwarp();
  } else if (warp == 1) {
    // ============================ MMA issuer ================================
    if (lane == 0) {
      const uint32_t fmt = std::is_same<T, __nv_bfloat16>::value ? 1u : 0u;
      const uint32_t idesc = umma_idesc(fmt, false, kPBM, kPBN);
      for (int i = 0; i < nk; ++i) {
        const int st = i % kPStages;
        if (!mbar_wait_bounded(&full[st], (i / kPStages) & 1)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t wa = smem_u32(sw + st * kPWBytes), xa = smem_u32(sx + st * kPXBytes);
#pragma unroll
        for (int kk = 0; kk < kPBK / 16; ++kk)
          umma(tmem, umma_desc(wa + kk * 32, 16, 1024), umma_desc(xa + kk * 32, 16, 1024), idesc,
               (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[st]);
      }
      // the accumulator is final once every product has landed (a commit
      // tracks all of this thread's earlier tensor-core operations)
      umma_commit(done);
    }
    __syncwarp();
  } else {
    // ============================ epilogue ==================================
    const int qd = warp & 3;
    const int cl = qd * 32 + lane;  // column in the block = TMEM lane
    const uint32_t taddr = tmem + (static_cast<uint32_t>(qd * 32) << 16);
    if (!__all_sync(0xffffffffu, mbar_wait_bounded(done, 0))) ok = false;
    pdl_wait();  // (returns at once: the producer has waited) y is written below
    tc_fence_after();
    tmem_ld32(taddr, v);
    tmem_wait_ld();
    if (p.splits == 1) {
      const int col = nb * kPBN + cl;
      if (ok && col < p.n) {
        const float b = p.bias ? Elt<T>::to(static_cast<const T *>(p.bias)[col]) : 0.f;
        T *y = static_cast<T *>(p.y);
#pragma unroll
        for (int r = 0; r < kPBM; ++r)
          if (r < p.m) y[static_cast<int64_t>(r) * p.ldy + col] = Elt<T>::from(v[r] + b);
      }
    } else {
      // every product has landed (done), so no copy or MMA still uses the
      // stage buffers: the partial goes there
#pragma unroll
      for (int r = 0; r < kPBM; ++r) part[r * kPBN + cl] = ok ? v[r] : 0.f;
    }
  }
  if (p.splits > 1) {
    cluster_sync_all();  // every rank's partial is in its shared memory
    if (warp >= 2) {
      // this rank's rows: split, split + splits, ...; a thread takes 4
      // columns of every 4th of them and sums the ranks' partials in rank
      // order (all ranks' 16-byte loads in flight first)
      const int t = threadIdx.x - 64;
      const int c4 = (t & 31) * 4, sub = t >> 5;
      const int col0 = nb * kPBN + c4;
      T *y = static_cast<T *>(p.y);
      for (int r = split + sub * p.splits; r < p.m; r += 4 * p.splits) {
        const uint32_t a = smem_u32(part + r * kPBN + c4);
        float4 pv[kPMaxSplits];
#pragma unroll
        for (int q = 0; q < kPMaxSplits; ++q)
          if (q < p.splits) pv[q] = ld_cluster_v4(a, static_cast<uint32_t>(q));
        float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int q = 0; q < kPMaxSplits; ++q)
          if (q < p.splits) {
            acc.x += pv[q].x;
            acc.y += pv[q].y;
            acc.z += pv[q].z;
            acc.w += pv[q].w;
          }
        const float vals[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
        for (int e = 0; e < 4; ++e) {
          const int col = col0 + e;
          if (col < p.n) {
            const float b = p.bias ? Elt<T>::to(static_cast<const T *>(p.bias)[col]) : 0.f;
            y[static_cast<int64_t>(r) * p.ldy + col] = Elt<T>::from(vals[e] + b);
          }
        }
      }
    }
    cluster_sync_all();  // no rank leaves while another still reads its partial
  }
  if (!ok && lane == 0) flag(p.status, MI_STATUS_TIMEOUT);
  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 32;" ::"r"(tmem) : "memory");
  }
}

// Clusters of `size` CTAs of proj_kernel<T> resident at once on the current
// device (cached per device and size; 0 if the query fails).
template <typename T>
int proj_max_clusters(int size) {
  static std::atomic<int> cache[64][kPMaxSplits + 1];  // count + 1; 0: not queried
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev >= 64) return 0;
  const int v = cache[dev][size].load();
  if (v > 0) return v - 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(size * 64);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = kPSmem;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = size;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int num = 0;
  if (cudaOccupancyMaxActiveClusters(&num, proj_kernel<T>, &cfg) != cudaSuccess) {
    cudaGetLastError();
    num = 0;
  }
  cache[dev][size].store(num + 1);
  return num;
}

template <typename T>
int launch_proj(const void *x, int64_t ldx, const void *w, int64_t ldw, const void *bias,
                void *y, int64_t ldy, int m, int n, int k, int dtype, int32_t *status,
                cudaStream_t s) {
  CUtensorMap wmap, xmap;
  if (!rows_tensor_map(w, n, 1, k, ldw, ldw, 1, kPBN, dtype, &wmap) ||
      !rows_tensor_map(x, m, 1, k, ldx, ldx, 1, kPBM, dtype, &xmap))
    return fail(MI_ERR_INVALID, "mi_proj_small_m: tensor map (pointers 16-byte aligned, "
                                "row strides a multiple of 8 elements)");
  const int nblocks = (n + kPBN - 1) / kPBN;
  const int ksteps = k / kPBK;
  static std::atomic<unsigned long long> attr_set{0};
  if (smem_limit_once(attr_set, proj_kernel<T>, kPSmem) != cudaSuccess)
    return check_launch("proj_kernel smem attribute");
  // K split: enough CTAs for two per SM, at most 8 (one cluster) and at
  // least 4 K steps (64 KB of W) each; fewer when under 85 % of the
  // clusters would be resident at once (then the most that all fit)
  const int want = std::max(1, std::min({2 * num_sms() / nblocks, ksteps / 4, kPMaxSplits}));
  int splits = want;
  if (want > 1 && 100 * proj_max_clusters<T>(want) < 85 * nblocks) {
    splits = 1;
    for (int c = want - 1; c > 1; --c)
      if (nblocks <= proj_max_clusters<T>(c)) {
        splits = c;
        break;
      }
  }
  ProjParams p{y, bias, status, m, n, k, static_cast<int>(ldy), splits, ksteps};
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(nblocks * splits);
  cfg.blockDim = dim3(kPThreads);
  cfg.dynamicSmemBytes = kPSmem;
  cfg.stream = s;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = splits;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cudaLaunchKernelEx(&cfg, proj_kernel<T>, wmap, xmap, p);
  return check_launch("proj_kernel");
}

}  // namespace
}  // namespace mi

extern "C" int mi_proj_small_m(const void *x, int64_t ldx, const void *w, int64_t ldw,
                               const void *bias, void *y, int64_t ldy, int32_t m, int32_t n,
                               int32_t k, int32_t dtype, int32_t *status, mi_stream_t stream) {
  using namespace mi;
  MI_REQUIRE(dtype == MI_DTYPE_BF16 || dtype == MI_DTYPE_F16, "mi_proj_small_m: bf16 / fp16 only");
  MI_REQUIRE(m >= 0 && m <= kPBM, "mi_proj_small_m: m = %d outside [0, 32]", m);
  if (m == 0) return MI_OK;
  MI_REQUIRE(x && w && y && status, "mi_proj_small_m: null pointer");
  MI_REQUIRE(n > 0 && k > 0 && k % kPBK == 0, "mi_proj_small_m: n = %d, k = %d (k a multiple of 64)",
             n, k);
  MI_REQUIRE(ldx >= k && ldw >= k && ldy >= n, "mi_proj_small_m: leading dimensions");
  MI_REQUIRE(ldy <= INT32_MAX && static_cast<int64_t>(m) * ldy <= (int64_t(1) << 40),
             "mi_proj_small_m: sizes");
  return dtype == MI_DTYPE_BF16
             ? launch_proj<__nv_bfloat16>(x, ldx, w, ldw, bias, y, ldy, m, n, k, dtype, status,
                                          stream)
             : launch_proj<__half>(x, ldx, w, ldw, bias, y, ldy, m, n, k, dtype, status, stream);
}
