// Entry points of the tcgen05 attention backward (attn_bwd_tc.cu).
#pragma once
#include "common.cuh"
#include "dropout.cuh"

namespace tsa {
// True when the tensor-core backward takes this problem.
bool tc_bwd_supported(const ts_attn_bwd_params& bp);
// Workspace bytes: fp32 row deltas + fp32 dQ accumulator.
size_t tc_bwd_workspace(const ts_attn_bwd_params& bp);
// `drop` set: the VJP of a forward that applied this dropout (mask regenerated).
cudaError_t tc_backward(const ts_attn_bwd_params& bp, void* workspace, size_t workspace_bytes, uint32_t* fault,
                        cudaStream_t stream, const DropoutArgs* drop = nullptr);
}  // namespace tsa
