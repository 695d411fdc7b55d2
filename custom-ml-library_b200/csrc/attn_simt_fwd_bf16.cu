// Generic CUDA-core attention forward, __nv_bfloat16 instantiations (simt_kernels.cuh).
#include "simt_kernels.cuh"

namespace tsa {

cudaError_t simt_forward_bf16(const ts_attn_params& p, cudaStream_t st, const DropoutArgs* drop) {
  return simt_fwd_t<__nv_bfloat16>(p, drop, st);
}

}  // namespace tsa
