// Entry points of the tcgen05 prefill forward (attn_fwd_tc.cu).
#pragma once
#include "common.cuh"
#include "dropout.cuh"

namespace tsa {
// True when the tensor-core kernel takes this problem.
bool tc_fwd_supported(const ts_attn_params& p);
// `drop` set: attention dropout on P before P.V (the generic kernels' mask).
cudaError_t tc_forward(const ts_attn_params& p, uint32_t* fault, cudaStream_t stream,
                       const DropoutArgs* drop = nullptr);
}  // namespace tsa
