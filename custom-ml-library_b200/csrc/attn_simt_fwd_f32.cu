// Generic CUDA-core attention forward, float instantiations (simt_kernels.cuh).
#include "simt_kernels.cuh"

namespace tsa {

cudaError_t simt_forward_f32(const ts_attn_params& p, cudaStream_t st, const DropoutArgs* drop) {
  return simt_fwd_t<float>(p, drop, st);
}

}  // namespace tsa
