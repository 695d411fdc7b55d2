// Generic CUDA-core attention backward, double instantiations (simt_kernels.cuh).
#include "simt_kernels.cuh"

namespace tsa {

cudaError_t simt_backward_f64(const ts_attn_bwd_params& bp, void* ws, cudaStream_t st, const DropoutArgs* drop) {
  return simt_bwd_t<double>(bp, ws, drop, st);
}

}  // namespace tsa
