// Entry points of the rotary-embedding kernels (rope.cu).
#pragma once
#include "common.cuh"

namespace tsa {
cudaError_t rope_apply(const ts_view4& x, const ts_view4& y, int dtype, int batch, int heads, int seq,
                       int channels, int rotary_dim, int64_t offset, const int32_t* positions,
                       const float* inv_freq, int inverse, cudaStream_t stream);
cudaError_t kv_append_rope(const ts_kv_append_params& p, const float* inv_freq, int rotary_dim,
                           cudaStream_t stream);
}  // namespace tsa
