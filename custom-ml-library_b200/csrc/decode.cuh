// Entry points of the split-K decode kernels (decode.cu).
#pragma once
#include "common.cuh"

namespace tsa {
// True when the split-K kernel takes this problem (else the caller uses the
// generic forward kernel).
bool decode_supported(const ts_attn_params& p);
// Workspace bytes for the per-split partials (0 when one split suffices).
size_t decode_workspace(const ts_attn_params& p);
cudaError_t decode_forward(const ts_attn_params& p, void* workspace, size_t workspace_bytes,
                           uint32_t* fault, cudaStream_t stream);
// The split kernel for 2+ query rows per KV head (decode_group.cu); partials in
// decode_forward's workspace layout, merged by its combine kernel.
cudaError_t decode_group_forward(const ts_attn_params& p, int split_keys, int max_splits, float* ws_acc,
                                 float* ws_ml, uint32_t* fault, cudaStream_t stream);
}  // namespace tsa
