// Entry points of the generic CUDA-core attention kernels (attn_simt.cu).
#pragma once
#include "common.cuh"
#include "dropout.cuh"

namespace tsa {
// Forward O (+ LSE) for any dtype / head dims <= 256 / masks; attention dropout when `drop` is set.
cudaError_t simt_forward(const ts_attn_params& p, cudaStream_t stream, const DropoutArgs* drop = nullptr);
// Bytes of workspace simt_backward needs (row deltas in the accumulation type).
size_t simt_backward_workspace(const ts_attn_bwd_params& bp);
// delta[b,h,i] = sum_c dO * O in fp32 (half / fp32 inputs), the backward preprocess.
cudaError_t simt_delta_f32(const ts_attn_bwd_params& bp, float* delta, cudaStream_t stream);
// dQ, dK, dV from the saved LSE (with the forward's dropout mask regenerated when `drop` is set).
cudaError_t simt_backward(const ts_attn_bwd_params& bp, void* workspace, cudaStream_t stream,
                          const DropoutArgs* drop = nullptr);
}  // namespace tsa
