// Generic CUDA-core attention forward, double instantiations (simt_kernels.cuh).
#include "simt_kernels.cuh"

namespace tsa {

cudaError_t simt_forward_f64(const ts_attn_params& p, cudaStream_t st, const DropoutArgs* drop) {
  return simt_fwd_t<double>(p, drop, st);
}

}  // namespace tsa
