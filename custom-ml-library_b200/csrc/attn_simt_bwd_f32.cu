// Generic CUDA-core attention backward, float instantiations (simt_kernels.cuh).
#include "simt_kernels.cuh"

namespace tsa {

cudaError_t simt_backward_f32(const ts_attn_bwd_params& bp, void* ws, cudaStream_t st, const DropoutArgs* drop) {
  return simt_bwd_t<float>(bp, ws, drop, st);
}

}  // namespace tsa
