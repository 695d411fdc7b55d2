// Generic CUDA-core attention backward, __half instantiations (simt_kernels.cuh).
#include "simt_kernels.cuh"

namespace tsa {

cudaError_t simt_backward_f16(const ts_attn_bwd_params& bp, void* ws, cudaStream_t st, const DropoutArgs* drop) {
  return simt_bwd_t<__half>(bp, ws, drop, st);
}

}  // namespace tsa
