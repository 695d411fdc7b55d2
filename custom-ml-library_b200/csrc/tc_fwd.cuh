// Entry points of the tcgen05 prefill forward (attn_fwd_tc.cu).
#pragma once
#include "common.cuh"

namespace tsa {
// True when the tensor-core kernel takes this problem.
bool tc_fwd_supported(const ts_attn_params& p);
cudaError_t tc_forward(const ts_attn_params& p, uint32_t* fault, cudaStream_t stream);
}  // namespace tsa
