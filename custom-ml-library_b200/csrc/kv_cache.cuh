// Entry points of the KV-cache maintenance kernels (kv_cache.cu).
#pragma once
#include "common.cuh"

namespace tsa {
cudaError_t kv_append(const ts_kv_append_params& p, cudaStream_t stream);
cudaError_t kv_reorder(const ts_view4& src, const ts_view4& dst, int dtype, int batch, int heads,
                       int length, int channels, const int32_t* index, cudaStream_t stream);
}  // namespace tsa
