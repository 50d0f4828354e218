// Decode-step glue around the paged path: fused residual-add + RMSNorm and
// fused SiLU-and-multiply.
//
// The reference runs, per decoder layer, `residual + x` then F.rms_norm
// (model.py:115-122, :333-343) and `F.silu(gate) * up` (model.py:311) as
// separate torch kernels. At decode batch sizes (tens of rows) each of those
// is latency bound, so one launch each here, with one 16-byte vector per
// thread and the row held in registers between the sum of squares and the
// scaling pass.
//
// Numerics follow torch: the residual sum is rounded to the storage type
// before the norm sees it (torch's `x + y`), the norm accumulates in fp32 and
// rounds once; silu(gate) is rounded to the storage type before the multiply
// and the product is rounded again (torch's `F.silu(g) * u`).
#include <algorithm>

#include "mi_common.cuh"

namespace mi {
namespace {

__device__ __forceinline__ float block_sum(float v, float *s_part) {
  v = warp_sum(v);
  const int nw = (blockDim.x + 31) >> 5;
  if ((threadIdx.x & 31) == 0) s_part[threadIdx.x >> 5] = v;
  __syncthreads();
  float t = 0.f;
  for (int i = 0; i < nw; ++i) t += s_part[i];
  return t;
}

// 16-bit types, hidden % 8 == 0, 16-byte aligned rows: thread t owns the
// 8-element vectors t, t + blockDim, ... (at most V of them).
template <typename T, int V>
__global__ void __launch_bounds__(1024) add_rmsnorm_vec_kernel(
    const T *__restrict__ x, T *__restrict__ residual, const T *__restrict__ w, T *__restrict__ y,
    int hidden, float eps, int has_x) {
  pdl_trigger();  // a programmatic-dependent successor waits for this grid itself
  __shared__ float s_part[32];
  const int nvec = hidden >> 3;
  const int64_t base = static_cast<int64_t>(blockIdx.x) * hidden;
  const uint4 *xr = reinterpret_cast<const uint4 *>(x + base);
  uint4 *rr = reinterpret_cast<uint4 *>(residual + base);
  const uint4 *wr = reinterpret_cast<const uint4 *>(w);
  uint4 *yr = reinterpret_cast<uint4 *>(y + base);
  float h[V][8];
  float ss = 0.f;
#pragma unroll
  for (int v = 0; v < V; ++v) {
    const int i = threadIdx.x + v * blockDim.x;
    if (i < nvec) {
      uint4 rv = rr[i];
      const T *re = reinterpret_cast<const T *>(&rv);
      if (has_x) {
        const uint4 xv = xr[i];
        const T *xe = reinterpret_cast<const T *>(&xv);
        uint4 sv;
        T *se = reinterpret_cast<T *>(&sv);
#pragma unroll
        for (int j = 0; j < 8; ++j) se[j] = Elt<T>::from(__fadd_rn(Elt<T>::to(re[j]), Elt<T>::to(xe[j])));
        rr[i] = sv;
        rv = sv;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        h[v][j] = Elt<T>::to(re[j]);
        ss = fmaf(h[v][j], h[v][j], ss);
      }
    }
  }
  const float inv = rsqrtf(block_sum(ss, s_part) / hidden + eps);
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
}

// Any type / shape: two passes over the row (the second re-reads the
// residual this thread wrote).
template <typename T>
__global__ void __launch_bounds__(256) add_rmsnorm_kernel(
    const T *__restrict__ x, T *__restrict__ residual, const T *__restrict__ w, T *__restrict__ y,
    int hidden, float eps, int has_x) {
  pdl_trigger();  // a programmatic-dependent successor waits for this grid itself
  __shared__ float s_part[32];
  const int64_t base = static_cast<int64_t>(blockIdx.x) * hidden;
  T *rr = residual + base;
  float ss = 0.f;
  for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
    float hv = Elt<T>::to(rr[i]);
    if (has_x) {
      const T hs = Elt<T>::from(__fadd_rn(hv, Elt<T>::to(x[base + i])));
      rr[i] = hs;
      hv = Elt<T>::to(hs);
    }
    ss = fmaf(hv, hv, ss);
  }
  const float inv = rsqrtf(block_sum(ss, s_part) / hidden + eps);
  for (int i = threadIdx.x; i < hidden; i += blockDim.x)
    y[base + i] = Elt<T>::from(Elt<T>::to(rr[i]) * inv * Elt<T>::to(w[i]));
}

template <typename T>
__device__ __forceinline__ T silu_mul_one(T g, T u) {
  const float gf = Elt<T>::to(g);
  const float s = Elt<T>::to(Elt<T>::from(gf / (1.f + expf(-gf))));
  return Elt<T>::from(s * Elt<T>::to(u));
}

// gate_up rows are [gate(inter) | up(inter)]; out rows are [inter].
// VEC elements per thread step (8 for 16-bit types with aligned rows, else 1).
template <typename T, int VEC>
__global__ void __launch_bounds__(256) silu_mul_kernel(const T *__restrict__ gu, T *__restrict__ out,
                                                       int rows, int inter) {
  pdl_trigger();  // a programmatic-dependent successor waits for this grid itself
  const int per_row = inter / VEC;
  const int64_t n = static_cast<int64_t>(rows) * per_row;
  for (int64_t idx = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; idx < n;
       idx += static_cast<int64_t>(gridDim.x) * blockDim.x) {
    const int64_t r = idx / per_row;
    const int c = static_cast<int>(idx - r * per_row) * VEC;
    const T *g = gu + r * 2 * inter + c;
    T *o = out + r * inter + c;
    if constexpr (VEC == 8) {
      const uint4 gv = *reinterpret_cast<const uint4 *>(g);
      const uint4 uv = *reinterpret_cast<const uint4 *>(g + inter);
      const T *ge = reinterpret_cast<const T *>(&gv);
      const T *ue = reinterpret_cast<const T *>(&uv);
      uint4 ov;
      T *oe = reinterpret_cast<T *>(&ov);
#pragma unroll
      for (int j = 0; j < 8; ++j) oe[j] = silu_mul_one(ge[j], ue[j]);
      *reinterpret_cast<uint4 *>(o) = ov;
    } else {
      o[0] = silu_mul_one(g[0], g[inter]);
    }
  }
}

bool aligned16(const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

template <typename T>
int launch_add_rmsnorm(const void *x, void *residual, const void *weight, void *out, int rows,
                       int hidden, float eps, cudaStream_t s) {
  const T *xp = static_cast<const T *>(x);
  T *rp = static_cast<T *>(residual);
  const T *wp = static_cast<const T *>(weight);
  T *yp = static_cast<T *>(out);
  const int has_x = x != nullptr;
  const int nvec = hidden / 8;
  const bool vec = sizeof(T) == 2 && hidden % 8 == 0 && nvec <= 4 * 1024 &&
                   (!x || aligned16(x)) && aligned16(residual) && aligned16(weight) &&
                   aligned16(out);
  if (vec) {
    int threads = nvec < 1024 ? ((nvec + 31) / 32) * 32 : 1024;
    const int v = (nvec + threads - 1) / threads;
    if (v == 1) {
      add_rmsnorm_vec_kernel<T, 1><<<rows, threads, 0, s>>>(xp, rp, wp, yp, hidden, eps, has_x);
    } else if (v == 2) {
      add_rmsnorm_vec_kernel<T, 2><<<rows, threads, 0, s>>>(xp, rp, wp, yp, hidden, eps, has_x);
    } else {
      add_rmsnorm_vec_kernel<T, 4><<<rows, threads, 0, s>>>(xp, rp, wp, yp, hidden, eps, has_x);
    }
    return check_launch("add_rmsnorm_vec_kernel");
  }
  add_rmsnorm_kernel<T><<<rows, 256, 0, s>>>(xp, rp, wp, yp, hidden, eps, has_x);
  return check_launch("add_rmsnorm_kernel");
}

template <typename T>
int launch_silu_mul(const void *gate_up, void *out, int rows, int inter, cudaStream_t s) {
  const T *gp = static_cast<const T *>(gate_up);
  T *op = static_cast<T *>(out);
  const bool vec = sizeof(T) == 2 && inter % 8 == 0 && aligned16(gate_up) && aligned16(out);
  const int64_t n = static_cast<int64_t>(rows) * (vec ? inter / 8 : inter);
  const int64_t cap = static_cast<int64_t>(num_sms()) * 8;
  const int blocks = static_cast<int>(std::min<int64_t>((n + 255) / 256, cap));
  if (vec)
    silu_mul_kernel<T, 8><<<blocks, 256, 0, s>>>(gp, op, rows, inter);
  else
    silu_mul_kernel<T, 1><<<blocks, 256, 0, s>>>(gp, op, rows, inter);
  return check_launch("silu_mul_kernel");
}

}  // namespace
}  // namespace mi

extern "C" int mi_add_rmsnorm(const void *x, void *residual, const void *weight, void *out,
                              int32_t rows, int32_t hidden, float eps, int32_t dtype,
                              mi_stream_t stream) {
  using namespace mi;
  MI_REQUIRE(rows >= 0 && hidden > 0, "add_rmsnorm: bad shape rows=%d hidden=%d", rows, hidden);
  if (rows == 0) return MI_OK;
  MI_REQUIRE(residual && weight && out, "add_rmsnorm: null pointer argument");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case MI_DTYPE_BF16:
      return launch_add_rmsnorm<__nv_bfloat16>(x, residual, weight, out, rows, hidden, eps, s);
    case MI_DTYPE_F16:
      return launch_add_rmsnorm<__half>(x, residual, weight, out, rows, hidden, eps, s);
    case MI_DTYPE_F32:
      return launch_add_rmsnorm<float>(x, residual, weight, out, rows, hidden, eps, s);
    default:
      return fail(MI_ERR_INVALID, "add_rmsnorm: bad dtype %d", dtype);
  }
}

extern "C" int mi_silu_mul(const void *gate_up, void *out, int32_t rows, int32_t inter,
                           int32_t dtype, mi_stream_t stream) {
  using namespace mi;
  MI_REQUIRE(rows >= 0 && inter > 0, "silu_mul: bad shape rows=%d inter=%d", rows, inter);
  if (rows == 0) return MI_OK;
  MI_REQUIRE(gate_up && out, "silu_mul: null pointer argument");
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case MI_DTYPE_BF16: return launch_silu_mul<__nv_bfloat16>(gate_up, out, rows, inter, s);
    case MI_DTYPE_F16: return launch_silu_mul<__half>(gate_up, out, rows, inter, s);
    case MI_DTYPE_F32: return launch_silu_mul<float>(gate_up, out, rows, inter, s);
    default: return fail(MI_ERR_INVALID, "silu_mul: bad dtype %d", dtype);
  }
}
