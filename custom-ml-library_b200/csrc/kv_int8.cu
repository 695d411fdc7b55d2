// int8 KV storage (tensorsmith nn/cache.py:47-52, 70-82, 91-98): symmetric
// per-token/head quantisation on append and dequantisation for callers that
// want the float prefix back.
//
// Quantisation of one row x[0:C] (after rounding to the cache's compute dtype,
// :68 `astype(self.dtype)`):
//   scale = max(max_c |x_c| / 127, 1e-8)         (fp32, correctly rounded)
//   q_c   = round_half_even(x_c / scale)         (fp32 division, :74)
// Dequantisation: dtype(float(q_c) * scale)       (:94-99).
// One warp per row: a butterfly max over the row, then a second pass writes
// the bytes (the row is in L1 from the first pass).
#include "int8.cuh"

namespace tsa {

template <typename S, typename C>
__device__ __forceinline__ float to_compute(S x) {
  return (float)Elem<C>::to_acc(Elem<C>::from_acc((typename Elem<C>::acc)Elem<S>::to_acc(x)));
}
// fp64 into a half-precision cache rounds once, as numpy's astype does.
template <>
__device__ __forceinline__ float to_compute<double, __half>(double x) {
  return __half2float(__double2half(x));
}
template <>
__device__ __forceinline__ float to_compute<double, __nv_bfloat16>(double x) {
  return __bfloat162float(__double2bfloat16(x));
}

template <typename S, typename C>
__device__ __forceinline__ void quantize_row(const S* src, int64_t src_stride, int8_t* dst, int64_t dst_stride,
                                             int channels, float* scale_out) {
  const int lane = threadIdx.x & 31;
  float amax = 0.f;
  for (int c = lane; c < channels; c += 32) amax = fmaxf(amax, fabsf(to_compute<S, C>(src[c * src_stride])));
#pragma unroll
  for (int off = 16; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
  const float scale = fmaxf(__fdiv_rn(amax, 127.f), 1e-8f);
  for (int c = lane; c < channels; c += 32) {
    int q = __float2int_rn(__fdiv_rn(to_compute<S, C>(src[c * src_stride]), scale));
    q = q > 127 ? 127 : (q < -128 ? -128 : q);
    dst[c * dst_stride] = (int8_t)q;
  }
  if (lane == 0) *scale_out = scale;
}

// grid (step blocks, heads, batch), 64 threads: warp 0 quantises the key row,
// warp 1 the value row of each step.
template <typename S, typename C>
__global__ void kv_append_int8_kernel(ts_kv_append_params p, float* key_scales, float* value_scales) {
  const int b = blockIdx.z, h = blockIdx.y, warp = threadIdx.x >> 5;
  const int64_t pos = p.positions ? (int64_t)p.positions[b] : p.position;
  const int64_t srow = ((int64_t)b * p.heads + h) * p.capacity;
  for (int t = blockIdx.x; t < p.steps; t += gridDim.x) {
    const int64_t dst_t = pos + t;
    if (dst_t < 0 || dst_t >= p.capacity) continue;  // rejected on the host; never written
    const ts_view4& sv = warp == 0 ? p.key : p.value;
    const ts_view4& dv = warp == 0 ? p.key_cache : p.value_cache;
    const S* src = reinterpret_cast<const S*>(sv.data) + b * sv.stride[0] + h * sv.stride[1] + t * sv.stride[2];
    int8_t* dst = reinterpret_cast<int8_t*>(dv.data) + b * dv.stride[0] + h * dv.stride[1] + dst_t * dv.stride[2];
    float* so = (warp == 0 ? key_scales : value_scales) + srow + dst_t;
    quantize_row<S, C>(src, sv.stride[3], dst, dv.stride[3], warp == 0 ? p.head_dim : p.value_dim, so);
  }
  if (p.positions_out && h == 0 && blockIdx.x == 0 && threadIdx.x == 0)
    p.positions_out[b] = (int32_t)(pos + p.steps);
}

template <typename S>
static cudaError_t append_int8_src(const ts_kv_append_params& p, float* ks, float* vs, dim3 grid,
                                   cudaStream_t st) {
  switch (p.cache_dtype) {
    case TS_F32: kv_append_int8_kernel<S, float><<<grid, 64, 0, st>>>(p, ks, vs); break;
    case TS_F64: kv_append_int8_kernel<S, double><<<grid, 64, 0, st>>>(p, ks, vs); break;
    case TS_F16: kv_append_int8_kernel<S, __half><<<grid, 64, 0, st>>>(p, ks, vs); break;
    case TS_BF16: kv_append_int8_kernel<S, __nv_bfloat16><<<grid, 64, 0, st>>>(p, ks, vs); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

cudaError_t kv_append_int8(const ts_kv_append_params& p, float* key_scales, float* value_scales,
                           cudaStream_t st) {
  const dim3 grid(p.steps < 65535 ? p.steps : 65535, p.heads, p.batch);
  switch (p.src_dtype) {
    case TS_F32: return append_int8_src<float>(p, key_scales, value_scales, grid, st);
    case TS_F64: return append_int8_src<double>(p, key_scales, value_scales, grid, st);
    case TS_F16: return append_int8_src<__half>(p, key_scales, value_scales, grid, st);
    case TS_BF16: return append_int8_src<__nv_bfloat16>(p, key_scales, value_scales, grid, st);
  }
  return cudaErrorInvalidValue;
}

// dst[b, h, t, c] = T(float(src[b, h, t, c]) * scales[b, h, t]) for t < length.
template <typename T>
__global__ void kv_dequant_int8_kernel(ts_view4 src, const float* scales, int64_t cap, ts_view4 dst, int heads,
                                       int length, int channels) {
  const int b = blockIdx.z, h = blockIdx.y;
  for (int t = blockIdx.x; t < length; t += gridDim.x) {
    const float sc = scales[((int64_t)b * heads + h) * cap + t];
    const int8_t* s = reinterpret_cast<const int8_t*>(src.data) + b * src.stride[0] + h * src.stride[1] +
                      t * src.stride[2];
    T* d = reinterpret_cast<T*>(dst.data) + b * dst.stride[0] + h * dst.stride[1] + t * dst.stride[2];
    for (int c = threadIdx.x; c < channels; c += blockDim.x)
      d[c * dst.stride[3]] = Elem<T>::from_acc((typename Elem<T>::acc)((float)s[c * src.stride[3]] * sc));
  }
}

cudaError_t kv_dequant_int8(const ts_view4& src, const float* scales, int64_t cap, const ts_view4& dst, int dtype,
                            int batch, int heads, int length, int channels, cudaStream_t st) {
  if (length <= 0) return cudaSuccess;
  const dim3 grid(length < 65535 ? length : 65535, heads, batch);
  switch (dtype) {
    case TS_F32: kv_dequant_int8_kernel<float><<<grid, 128, 0, st>>>(src, scales, cap, dst, heads, length, channels); break;
    case TS_F64: kv_dequant_int8_kernel<double><<<grid, 128, 0, st>>>(src, scales, cap, dst, heads, length, channels); break;
    case TS_F16: kv_dequant_int8_kernel<__half><<<grid, 128, 0, st>>>(src, scales, cap, dst, heads, length, channels); break;
    case TS_BF16:
      kv_dequant_int8_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(src, scales, cap, dst, heads, length, channels);
      break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace tsa
