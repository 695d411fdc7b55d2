// Generic CUDA-core attention backward, __nv_bfloat16 instantiations (simt_kernels.cuh).
#include "simt_kernels.cuh"

namespace tsa {

cudaError_t simt_backward_bf16(const ts_attn_bwd_params& bp, void* ws, cudaStream_t st, const DropoutArgs* drop) {
  return simt_bwd_t<__nv_bfloat16>(bp, ws, drop, st);
}

}  // namespace tsa
