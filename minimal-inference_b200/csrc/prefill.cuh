// Arguments shared by the generic (prefill.cu) and tensor-core
// (prefill_tc2.cu) paged prefill kernels.
#pragma once

#include "mi_common.cuh"

namespace mi {

struct PrefillParams {
  const void *q;
  int64_t qsn, qsh;
  const int32_t *qo_indptr;
  int total_q;
  const void *kv;
  int64_t num_pages;
  int ps, hkv, d;
  const int32_t *indptr, *indices, *last;
  int batch, hq, group, causal;
  float scale_log2;
  void *out;
  float *lse;
  int32_t *status;
  unsigned *ctr;  // [2] work-item counters in the workspace (zero between calls), or null
};

// Tensor-core path (prefill_tc2.cu): two query tiles per work item. Returns
// -1 (nothing launched) when the shape or layout is outside its coverage, so
// the caller runs the generic kernel instead.
int launch_prefill_tc2(const PrefillParams &p, int dtype, cudaStream_t s);

}  // namespace mi
