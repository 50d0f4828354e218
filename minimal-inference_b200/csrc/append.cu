// Kernel (1): paged KV append with fused RoPE on K (and optionally Q).
//
// Replaces the reference's RoPE glue (model.py:169-170 -> apply_rotary_emb,
// model.py:92-107: ~5 elementwise launches per tensor) plus the K/V
// permute-copies (model.py:203-204) and flashinfer.page.append_paged_kv_cache
// (model.py:207-216) with one launch per layer.
//
// Addressing follows FlashInfer's append (page.cuh:259-283): token i of
// request b at position p goes to page kv_indices[kv_indptr[b] + p/ps], slot
// p%ps. RoPE reproduces the reference's rounding exactly: each of x*cos,
// rot*sin and their sum is rounded to the storage type, with no FMA
// contraction (explicit __fmul_rn/__fadd_rn), so pages hold the same bits as
// the reference's.
//
// Layout: one CTA row per token (blockIdx.x), threads over 16-byte chunks of
// the token's Q/K/V head rows (blockIdx.y spreads wide tokens). Every access
// is a 16-byte vector load/store on the fast path; page rows are contiguous
// head_dim runs, so stores are fully coalesced within a head.
#include "mi_common.cuh"

namespace mi {
namespace {

struct AppendParams {
  const void *k;
  int64_t ksn, ksh;
  const void *v;
  int64_t vsn, vsh;
  const int32_t *batch_indices, *positions;
  int nnz;
  void *kv;
  int64_t num_pages;
  int ps, hkv, d;
  const int32_t *indices, *indptr;
  int batch;
  const void *cos, *sin;
  int max_pos;
  const int32_t *rope_pos;
  const void *q_in;
  int64_t qisn, qish;
  void *q_out;
  int64_t qosn, qosh;
  int hq;
  int scratch;
  int32_t *status;
};

template <typename T, int VEC>
__device__ __forceinline__ void load_vec(float (&dst)[VEC], const T *src) {
  if constexpr (VEC * sizeof(T) == 16) {
    uint4 u = *reinterpret_cast<const uint4 *>(src);
    const T *e = reinterpret_cast<const T *>(&u);
#pragma unroll
    for (int j = 0; j < VEC; ++j) dst[j] = Elt<T>::to(e[j]);
  } else {
#pragma unroll
    for (int j = 0; j < VEC; ++j) dst[j] = Elt<T>::to(src[j]);
  }
}

template <typename T, int VEC>
__device__ __forceinline__ void store_vec(T *dst, const float (&src)[VEC]) {
  if constexpr (VEC * sizeof(T) == 16) {
    uint4 u;
    T *e = reinterpret_cast<T *>(&u);
#pragma unroll
    for (int j = 0; j < VEC; ++j) e[j] = Elt<T>::from(src[j]);
    *reinterpret_cast<uint4 *>(dst) = u;
  } else {
#pragma unroll
    for (int j = 0; j < VEC; ++j) dst[j] = Elt<T>::from(src[j]);
  }
}

template <typename T, int VEC>
__device__ __forceinline__ void copy_vec(T *dst, const T *src) {
  if constexpr (VEC * sizeof(T) == 16) {
    *reinterpret_cast<uint4 *>(dst) = *reinterpret_cast<const uint4 *>(src);
  } else {
#pragma unroll
    for (int j = 0; j < VEC; ++j) dst[j] = src[j];
  }
}

// Rotate chunk `c` of a head row: out = x*cos + rotate_half(x)*sin where
// rotate_half(x) = cat(-x2, x1) (model.py:101-107).
template <typename T, int VEC>
__device__ __forceinline__ void rope_chunk(float (&out)[VEC], const T *row, int c, int nchunk,
                                           const T *cos_row, const T *sin_row) {
  const int half = nchunk / 2;
  float x[VEC], r[VEC], cs[VEC], sn[VEC];
  load_vec<T, VEC>(x, row + c * VEC);
  const int pc = c < half ? c + half : c - half;
  load_vec<T, VEC>(r, row + pc * VEC);
  load_vec<T, VEC>(cs, cos_row + c * VEC);
  load_vec<T, VEC>(sn, sin_row + c * VEC);
  const bool neg = c < half;
#pragma unroll
  for (int j = 0; j < VEC; ++j) out[j] = rope1<T>(x[j], neg ? -r[j] : r[j], cs[j], sn[j]);
}

template <typename T, int VEC>
__global__ void __launch_bounds__(256) append_kernel(const AppendParams p) {
  pdl_wait();     // predecessors' writes (q/k/v producers, readers of q_out) are done
  pdl_trigger();  // the attention kernel that follows may get scheduled now
  const int nchunk = p.d / VEC;
  const int nq = p.q_in ? p.hq * nchunk : 0;
  const int nk = p.hkv * nchunk;
  const int items = nq + 2 * nk;
  const bool rope = p.cos != nullptr;
  const T *kin = static_cast<const T *>(p.k);
  const T *vin = static_cast<const T *>(p.v);
  T *kv = static_cast<T *>(p.kv);
  const int64_t row = static_cast<int64_t>(p.hkv) * p.d;  // one slot's K (or V) row

  for (int i = blockIdx.x; i < p.nnz; i += gridDim.x) {
    const int b = p.batch_indices[i];
    const int pos = p.positions[i];
    const int rp = p.rope_pos ? p.rope_pos[i] : pos;
    const bool rope_ok = !rope || (rp >= 0 && rp < p.max_pos);
    int64_t page = -1;  // -1 bad batch index/position, -2 bad page id
    int slot = 0;
    if (b >= 0 && b < p.batch && pos >= 0) {
      const int it = p.indptr[b] + pos / p.ps;
      slot = pos % p.ps;
      if (it < p.indptr[b + 1]) {
        const int pg = p.indices[it];
        page = (pg >= 0 && pg < p.num_pages) ? pg : -2;
      } else if (p.scratch >= 0) {
        page = p.scratch;  // padding lane: its page slot lies past its pages
      }
    }
    if (blockIdx.y == 0 && threadIdx.x == 0) {
      if (!(b >= 0 && b < p.batch)) flag(p.status, MI_STATUS_BAD_BATCH_INDEX);
      else if (page == -1 || !rope_ok) flag(p.status, MI_STATUS_BAD_POSITION);
      else if (page == -2) flag(p.status, MI_STATUS_BAD_PAGE);
    }
    if (!rope_ok) continue;
    const T *cos_row = rope ? static_cast<const T *>(p.cos) + static_cast<int64_t>(rp) * p.d : nullptr;
    const T *sin_row = rope ? static_cast<const T *>(p.sin) + static_cast<int64_t>(rp) * p.d : nullptr;

    for (int w = blockIdx.y * blockDim.x + threadIdx.x; w < items; w += gridDim.y * blockDim.x) {
      if (w < nq) {  // rotate a query chunk into q_out
        const int h = w / nchunk, c = w % nchunk;
        const T *src = static_cast<const T *>(p.q_in) + i * p.qisn + h * p.qish;
        T *dst = static_cast<T *>(p.q_out) + i * p.qosn + h * p.qosh + c * VEC;
        float o[VEC];
        rope_chunk<T, VEC>(o, src, c, nchunk, cos_row, sin_row);
        store_vec<T, VEC>(dst, o);
        continue;
      }
      if (page < 0) continue;
      const int wk = w - nq;
      const int which = wk < nk ? 0 : 1;  // 0: K, 1: V
      const int hw = wk - which * nk;
      const int h = hw / nchunk, c = hw % nchunk;
      T *dst = kv + ((page * 2 + which) * p.ps + slot) * row + static_cast<int64_t>(h) * p.d + c * VEC;
      if (which == 0) {
        const T *src = kin + i * p.ksn + h * p.ksh;
        if (rope) {
          float o[VEC];
          rope_chunk<T, VEC>(o, src, c, nchunk, cos_row, sin_row);
          store_vec<T, VEC>(dst, o);
        } else {
          copy_vec<T, VEC>(dst, src + c * VEC);
        }
      } else {
        copy_vec<T, VEC>(dst, vin + i * p.vsn + h * p.vsh + c * VEC);
      }
    }
  }
}

template <typename T>
int launch_append(const AppendParams &p, bool vec_ok, cudaStream_t stream) {
  constexpr int V16 = 16 / sizeof(T);
  const int vec = vec_ok ? V16 : 1;
  const int nchunk = p.d / vec;
  const int items = (p.q_in ? p.hq * nchunk : 0) + 2 * p.hkv * nchunk;
  const int threads = 256;
  int gy = (items + threads - 1) / threads;
  int gx = p.nnz < (1 << 20) ? p.nnz : (1 << 20);
  dim3 grid(gx, gy);
  cudaError_t e = vec_ok ? launch_pdl(append_kernel<T, V16>, grid, dim3(threads), 0, stream, p)
                         : launch_pdl(append_kernel<T, 1>, grid, dim3(threads), 0, stream, p);
  if (e != cudaSuccess) return fail(MI_ERR_CUDA, "append_kernel launch: %s", cudaGetErrorString(e));
  return check_launch("append_kernel");
}

bool aligned16(const void *ptr) { return (reinterpret_cast<uintptr_t>(ptr) & 15u) == 0; }

}  // namespace
}  // namespace mi

extern "C" int mi_append_paged_kv_cache(
    const void *append_key, int64_t k_stride_n, int64_t k_stride_h,
    const void *append_value, int64_t v_stride_n, int64_t v_stride_h,
    const int32_t *batch_indices, const int32_t *positions, int32_t nnz,
    void *kv_data, int64_t num_pages, int32_t page_size, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype,
    const int32_t *kv_indices, const int32_t *kv_indptr, int32_t batch_size,
    const void *rope_cos, const void *rope_sin, int32_t rope_max_pos,
    const int32_t *rope_positions,
    const void *q_in, int64_t q_in_stride_n, int64_t q_in_stride_h,
    void *q_out, int64_t q_out_stride_n, int64_t q_out_stride_h, int32_t num_qo_heads,
    int32_t scratch_page, int32_t *status, mi_stream_t stream) {
  using namespace mi;
  MI_REQUIRE(nnz >= 0 && batch_size >= 0, "append: negative nnz/batch_size");
  if (nnz == 0) return MI_OK;
  MI_REQUIRE(append_key && append_value && batch_indices && positions && kv_data && kv_indices &&
                 kv_indptr,
             "append: null pointer argument");
  MI_REQUIRE(page_size > 0 && num_kv_heads > 0 && head_dim > 0 && num_pages > 0,
             "append: bad pool geometry");
  MI_REQUIRE(dtype == MI_DTYPE_F32 || dtype == MI_DTYPE_F16 || dtype == MI_DTYPE_BF16,
             "append: bad dtype %d", dtype);
  MI_REQUIRE(scratch_page < num_pages, "append: scratch_page %d outside the pool", scratch_page);
  const bool rope = rope_cos != nullptr || rope_sin != nullptr;
  MI_REQUIRE(!rope || (rope_cos && rope_sin && rope_max_pos > 0 && head_dim % 2 == 0),
             "append: RoPE needs both tables, rope_max_pos > 0 and an even head_dim");
  MI_REQUIRE(!q_in || (rope && q_out && num_qo_heads > 0),
             "append: query rotation needs RoPE tables, q_out and num_qo_heads");
  const int es = elt_size(dtype);
  const int v16 = 16 / es;
  bool vec_ok = head_dim % (2 * v16) == 0;
  const void *ptrs[] = {append_key, append_value, kv_data, rope_cos, rope_sin, q_in, q_out};
  for (const void *ptr : ptrs) vec_ok = vec_ok && (ptr == nullptr || aligned16(ptr));
  const int64_t strides[] = {k_stride_n, k_stride_h, v_stride_n, v_stride_h,
                             q_in ? q_in_stride_n : 0, q_in ? q_in_stride_h : 0,
                             q_in ? q_out_stride_n : 0, q_in ? q_out_stride_h : 0};
  for (int64_t s : strides) vec_ok = vec_ok && (s % v16 == 0);

  AppendParams p{append_key, k_stride_n, k_stride_h, append_value, v_stride_n, v_stride_h,
                 batch_indices, positions, nnz, kv_data, num_pages, page_size, num_kv_heads,
                 head_dim, kv_indices, kv_indptr, batch_size, rope ? rope_cos : nullptr,
                 rope ? rope_sin : nullptr, rope_max_pos, rope_positions, q_in, q_in_stride_n,
                 q_in_stride_h, q_out, q_out_stride_n, q_out_stride_h, num_qo_heads,
                 scratch_page, status};
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  switch (dtype) {
    case MI_DTYPE_F32: return launch_append<float>(p, vec_ok, s);
    case MI_DTYPE_F16: return launch_append<__half>(p, vec_ok, s);
    default: return launch_append<__nv_bfloat16>(p, vec_ok, s);
  }
}
