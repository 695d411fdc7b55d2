// Dtype dispatch of the generic CUDA-core attention kernels (their templates
// are in simt_kernels.cuh, instantiated per dtype in attn_simt_{fwd,bwd}_*.cu),
// the fp32 row-delta preprocess and the dropout keep-mask kernel.
#include "simt_kernels.cuh"

namespace tsa {

cudaError_t simt_forward_f32(const ts_attn_params& p, cudaStream_t st, const DropoutArgs* drop);
cudaError_t simt_forward_f64(const ts_attn_params& p, cudaStream_t st, const DropoutArgs* drop);
cudaError_t simt_forward_f16(const ts_attn_params& p, cudaStream_t st, const DropoutArgs* drop);
cudaError_t simt_forward_bf16(const ts_attn_params& p, cudaStream_t st, const DropoutArgs* drop);
cudaError_t simt_backward_f32(const ts_attn_bwd_params& bp, void* ws, cudaStream_t st, const DropoutArgs* drop);
cudaError_t simt_backward_f64(const ts_attn_bwd_params& bp, void* ws, cudaStream_t st, const DropoutArgs* drop);
cudaError_t simt_backward_f16(const ts_attn_bwd_params& bp, void* ws, cudaStream_t st, const DropoutArgs* drop);
cudaError_t simt_backward_bf16(const ts_attn_bwd_params& bp, void* ws, cudaStream_t st, const DropoutArgs* drop);

cudaError_t simt_delta_f32(const ts_attn_bwd_params& bp, float* delta, cudaStream_t st) {
  const int rows = bp.fwd.batch * bp.fwd.q_heads * bp.fwd.q_len;
  const dim3 grid(ceil_div(rows * 32, 256));
  switch (bp.fwd.dtype) {
    case TS_F32: simt_bwd_delta_kernel<float><<<grid, 256, 0, st>>>(bp, delta); break;
    case TS_F16: simt_bwd_delta_kernel<__half><<<grid, 256, 0, st>>>(bp, delta); break;
    case TS_BF16: simt_bwd_delta_kernel<__nv_bfloat16><<<grid, 256, 0, st>>>(bp, delta); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t simt_forward(const ts_attn_params& p, cudaStream_t st, const DropoutArgs* drop) {
  switch (p.dtype) {
    case TS_F32: return simt_forward_f32(p, st, drop);
    case TS_F64: return simt_forward_f64(p, st, drop);
    case TS_F16: return simt_forward_f16(p, st, drop);
    case TS_BF16: return simt_forward_bf16(p, st, drop);
  }
  return cudaErrorInvalidValue;
}

size_t simt_backward_workspace(const ts_attn_bwd_params& bp) {
  const size_t acc = bp.fwd.dtype == TS_F64 ? 8 : 4;
  return acc * (size_t)bp.fwd.batch * bp.fwd.q_heads * bp.fwd.q_len;
}

cudaError_t simt_backward(const ts_attn_bwd_params& bp, void* ws, cudaStream_t st, const DropoutArgs* drop) {
  switch (bp.fwd.dtype) {
    case TS_F32: return simt_backward_f32(bp, ws, st, drop);
    case TS_F64: return simt_backward_f64(bp, ws, st, drop);
    case TS_F16: return simt_backward_f16(bp, ws, st, drop);
    case TS_BF16: return simt_backward_bf16(bp, ws, st, drop);
  }
  return cudaErrorInvalidValue;
}

// One CTA per (query row, head, batch row); threads over keys in groups of 8.
__global__ void dropout_mask_kernel(DropoutArgs d, int heads, int q_len, int kv_len, uint8_t* mask) {
  const int i = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const uint32_t bh = (uint32_t)(b * heads + h);
  uint8_t* row = mask + (((int64_t)b * heads + h) * q_len + i) * kv_len;
  for (int j8 = threadIdx.x; j8 * 8 < kv_len; j8 += blockDim.x) {
    const uint32_t bits = dropout_keep8(d, bh, (uint32_t)i, (uint32_t)j8);
    for (int k = 0; k < 8 && j8 * 8 + k < kv_len; ++k) row[j8 * 8 + k] = (bits >> k) & 1u;
  }
}

cudaError_t dropout_mask(const DropoutArgs& d, int batch, int heads, int q_len, int kv_len, uint8_t* mask,
                         cudaStream_t st) {
  if (q_len > 65535 * 32 || heads > 65535 || batch > 65535) return cudaErrorInvalidValue;
  dropout_mask_kernel<<<dim3(q_len, heads, batch), 128, 0, st>>>(d, heads, q_len, kv_len, mask);
  return cudaGetLastError();
}

}  // namespace tsa
