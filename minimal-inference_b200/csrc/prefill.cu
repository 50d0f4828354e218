// Kernel (3): paged prefill attention.
//
// Replaces FlashInfer's BatchPrefillWithPagedKVCacheWrapper as the reference
// uses it (scheduler.py:530-534 ctor, :704-716 plan, model.py:219-235 run):
// ragged queries split by qo_indptr attend to their request's pages, causal
// with bottom-right alignment (query i of qo_len sees keys
// j <= kv_len - qo_len + i), native GQA (no head padding).
//
// This file holds the generic path: one warp per (query row, query head),
// online softmax over the visible keys, any dtype (fp32 parity configs
// included) and any head_dim <= 256. The tensor-core path lives in
// prefill_tc2.cu.
#include "mi_common.cuh"
#include "prefill.cuh"

namespace mi {
namespace {

constexpr int kRowsPerCta = 4;

template <typename T, int DPL>
__global__ void __launch_bounds__(128) prefill_generic_kernel(const PrefillParams p) {
  const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
  const int qi = blockIdx.x * kRowsPerCta + warp;
  const int hqi = blockIdx.y;
  if (qi >= p.total_q) return;
  // request of this query row: last b with qo_indptr[b] <= qi
  int lo = 0, hi = p.batch - 1;
  while (lo < hi) {
    const int mid = (lo + hi + 1) >> 1;
    if (p.qo_indptr[mid] <= qi) lo = mid; else hi = mid - 1;
  }
  const int b = lo;
  const int q0 = p.qo_indptr[b], qo_len = p.qo_indptr[b + 1] - q0;
  const int i = qi - q0;
  T *orow = static_cast<T *>(p.out) + (static_cast<int64_t>(qi) * p.hq + hqi) * p.d;
  if (i < 0 || i >= qo_len) return;  // row outside every request (malformed indptr)
  const int kvlen = kv_len_of(p.indptr, p.last, b, p.ps);
  int limit = kvlen;
  if (p.causal) limit = min(kvlen, kvlen - qo_len + i + 1);
  const int h = hqi / p.group;
  const T *qr = static_cast<const T *>(p.q) + static_cast<int64_t>(qi) * p.qsn +
                static_cast<int64_t>(hqi) * p.qsh;
  float qv[DPL], acc[DPL];
#pragma unroll
  for (int j = 0; j < DPL; ++j) {
    const int dd = j * 32 + lane;
    qv[j] = dd < p.d ? Elt<T>::to(qr[dd]) : 0.f;
    acc[j] = 0.f;
  }
  float m = -INFINITY, l = 0.f;
  const T *kv = static_cast<const T *>(p.kv);
  const int64_t slot_elems = static_cast<int64_t>(p.hkv) * p.d;
  for (int t = 0; t < limit; ++t) {
    const int64_t page = p.indices[p.indptr[b] + t / p.ps];
    if (page < 0 || page >= p.num_pages) {
      if (lane == 0) flag(p.status, MI_STATUS_BAD_PAGE);
      continue;
    }
    const T *kr = kv + ((page * 2) * p.ps + t % p.ps) * slot_elems + static_cast<int64_t>(h) * p.d;
    const T *vr = kr + static_cast<int64_t>(p.ps) * slot_elems;
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const int dd = j * 32 + lane;
      if (dd < p.d) s += qv[j] * Elt<T>::to(kr[dd]);
    }
    s = warp_sum(s) * p.scale_log2;
    const float mn = fmaxf(m, s);
    const float corr = exp2f(m - mn);
    const float pr = exp2f(s - mn);
    l = l * corr + pr;
#pragma unroll
    for (int j = 0; j < DPL; ++j) {
      const int dd = j * 32 + lane;
      acc[j] = acc[j] * corr + (dd < p.d ? pr * Elt<T>::to(vr[dd]) : 0.f);
    }
    m = mn;
  }
  const float inv = l > 0.f ? 1.f / l : 0.f;
#pragma unroll
  for (int j = 0; j < DPL; ++j) {
    const int dd = j * 32 + lane;
    if (dd < p.d) orow[dd] = Elt<T>::from(acc[j] * inv);
  }
  if (p.lse && lane == 0)
    p.lse[static_cast<int64_t>(qi) * p.hq + hqi] = l > 0.f ? (m + __log2f(l)) * kLn2 : -INFINITY;
}

template <typename T>
int launch_generic(const PrefillParams &p, cudaStream_t s) {
  dim3 grid((p.total_q + kRowsPerCta - 1) / kRowsPerCta, p.hq);
  if (p.d <= 32) prefill_generic_kernel<T, 1><<<grid, 128, 0, s>>>(p);
  else if (p.d <= 64) prefill_generic_kernel<T, 2><<<grid, 128, 0, s>>>(p);
  else if (p.d <= 128) prefill_generic_kernel<T, 4><<<grid, 128, 0, s>>>(p);
  else prefill_generic_kernel<T, 8><<<grid, 128, 0, s>>>(p);
  return check_launch("prefill_generic_kernel");
}

}  // namespace
}  // namespace mi

extern "C" size_t mi_paged_prefill_workspace_size(int32_t total_q, int32_t batch_size,
                                                  int32_t num_qo_heads, int32_t head_dim) {
  (void)total_q;
  (void)batch_size;
  (void)num_qo_heads;
  (void)head_dim;
  return 256;  // the tensor-core kernel's two work-item counters
}

extern "C" int mi_paged_prefill(
    const void *q, int64_t q_stride_n, int64_t q_stride_h,
    const int32_t *qo_indptr, int32_t total_q,
    const void *kv_data, int64_t num_pages, int32_t page_size, int32_t num_kv_heads,
    int32_t head_dim, int32_t dtype,
    const int32_t *kv_indptr, const int32_t *kv_indices, const int32_t *kv_last_page_len,
    int32_t batch_size, int32_t num_qo_heads, int32_t causal, float sm_scale,
    void *out, float *lse, void *workspace, size_t workspace_bytes, int32_t *status,
    mi_stream_t stream) {
  using namespace mi;
  MI_REQUIRE(total_q >= 0 && batch_size >= 0, "prefill: negative total_q/batch_size");
  if (total_q == 0 || batch_size == 0) return MI_OK;
  MI_REQUIRE(q && qo_indptr && kv_data && kv_indptr && kv_indices && kv_last_page_len && out,
             "prefill: null pointer argument");
  MI_REQUIRE(page_size > 0 && num_kv_heads > 0 && head_dim > 0 && head_dim <= 256 &&
                 num_pages > 0,
             "prefill: bad pool geometry");
  MI_REQUIRE(num_qo_heads >= num_kv_heads && num_qo_heads % num_kv_heads == 0,
             "prefill: num_qo_heads %d is not a multiple of num_kv_heads %d", num_qo_heads,
             num_kv_heads);
  MI_REQUIRE(dtype == MI_DTYPE_F32 || dtype == MI_DTYPE_F16 || dtype == MI_DTYPE_BF16,
             "prefill: bad dtype %d", dtype);
  MI_REQUIRE(num_qo_heads <= 65535, "prefill: too many heads");
  PrefillParams p{q, q_stride_n, q_stride_h, qo_indptr, total_q, kv_data, num_pages, page_size,
                  num_kv_heads, head_dim, kv_indptr, kv_indices, kv_last_page_len, batch_size,
                  num_qo_heads, num_qo_heads / num_kv_heads, causal != 0, sm_scale * kLog2e,
                  out, lse, status, nullptr};
  // work-item counters for the persistent tensor-core kernel (without a
  // workspace it falls back to a fixed round robin)
  if (workspace && workspace_bytes >= 256 && (reinterpret_cast<uintptr_t>(workspace) & 15) == 0)
    p.ctr = static_cast<unsigned *>(workspace);
  cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
  // tensor cores (two query tiles per work item) where they cover the shape
  const int rc = launch_prefill_tc2(p, dtype, s);
  if (rc >= 0) return rc;
  switch (dtype) {
    case MI_DTYPE_F32: return launch_generic<float>(p, s);
    case MI_DTYPE_F16: return launch_generic<__half>(p, s);
    default: return launch_generic<__nv_bfloat16>(p, s);
  }
}
