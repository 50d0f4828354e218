// Stream-K TMA decode kernel (decode_sk.cu): arguments and entry points used
// by the mi_paged_decode dispatcher in decode.cu.
#pragma once

#include "mi_common.cuh"

namespace mi {

struct SkArgs {
  const void *q;
  int64_t qsb, qsh;
  const void *kv;
  int64_t num_pages;
  int ps, hkv, d, dtype;
  const int32_t *indptr, *indices, *last;
  int batch, hq;
  float sm_scale;
  void *out;
  float *lse;
  void *ws;
  size_t ws_bytes;
  int32_t *status;
  cudaStream_t stream;
  // fused append (mi_paged_decode_append); k_new == nullptr: plain decode
  const void *k_new = nullptr, *v_new = nullptr;
  int64_t ksb = 0, ksh = 0, vsb = 0, vsh = 0;
  const void *rope_cos = nullptr, *rope_sin = nullptr;
  int rope_max = 0;
};

// Workspace bytes the stream-K kernel needs for this shape.
size_t decode_sk_workspace_bytes(int batch, int hq, int hkv, int d);
// Launches the stream-K kernel; returns -1 (nothing launched) when the
// shape, alignment or workspace is outside its coverage.
int launch_decode_sk(const SkArgs &a);

}  // namespace mi
