// Tensor-core (tcgen05) cross-depth masked attention.  Not yet enabled: every
// call is routed to the CUDA-core kernels.
#include "attn.cuh"

namespace pe {

bool attn_tc_eligible(int, int64_t, int64_t, int, int, int, int, const void*, int64_t,
                      const void*, int64_t, const void*, int64_t) {
  return false;
}

int attn_fwd_tc_launch(int64_t, int, int, const void*, int64_t, const void*, int64_t,
                       const void*, int64_t, void*, int64_t, float*, const MaskSpec&, int*,
                       cudaStream_t) {
  set_error("tcgen05 attention not built");
  return PE_ERR_UNSUPPORTED;
}

int attn_bwd_tc_launch(int64_t, int, int, const void*, int64_t, const void*, int64_t,
                       const void*, int64_t, const void*, int64_t, const void*, int64_t,
                       const float*, void*, int64_t, void*, int64_t, void*, int64_t, float*,
                       const MaskSpec&, int*, cudaStream_t) {
  set_error("tcgen05 attention not built");
  return PE_ERR_UNSUPPORTED;
}

}  // namespace pe
