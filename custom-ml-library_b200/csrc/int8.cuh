// Entry points of the int8 KV-cache kernels: quantising append and
// dequantisation (kv_int8.cu), fused-dequant split-K decode (decode_int8.cu).
#pragma once
#include "common.cuh"

namespace tsa {
cudaError_t kv_append_int8(const ts_kv_append_params& p, float* key_scales, float* value_scales,
                           cudaStream_t stream);
cudaError_t kv_dequant_int8(const ts_view4& src, const float* scales, int64_t scale_capacity, const ts_view4& dst,
                            int dtype, int batch, int heads, int length, int channels, cudaStream_t stream);
// True when the fused int8 decode takes this problem.
bool decode_int8_supported(const ts_attn_params& p);
size_t decode_int8_workspace(const ts_attn_params& p);
cudaError_t decode_int8_forward(const ts_attn_params& p, const float* k_scale, const float* v_scale,
                                int64_t scale_capacity, void* ws, size_t ws_bytes, uint32_t* fault,
                                cudaStream_t stream);
}  // namespace tsa
