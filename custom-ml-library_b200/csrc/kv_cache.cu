// KV-cache maintenance kernels: chunk append (nn/cache.py:54-86) and batch-row
// reorder for beam search (nn/cache.py:110-123).  Both are pure data movement
// (HBM-bound): each thread moves 16-byte vectors when the rows allow it.
#include "common.cuh"
#include "kv_cache.cuh"

namespace tsa {

template <typename S, typename D>
__device__ __forceinline__ D convert_elem(S x) {
  return Elem<D>::from_acc((typename Elem<D>::acc)Elem<S>::to_acc(x));
}

struct AppendLaunch {
  ts_kv_append_params p;
};

// One CTA per (row b, head h, block of steps); threads stride over channels.
template <typename S, typename D>
__global__ void kv_append_kernel(AppendLaunch L) {
  const ts_kv_append_params& p = L.p;
  const int b = blockIdx.z, h = blockIdx.y;
  const int64_t pos = p.positions ? (int64_t)p.positions[b] : p.position;
  for (int t = blockIdx.x; t < p.steps; t += gridDim.x) {
    const int64_t dst_t = pos + t;
    if (dst_t < 0 || dst_t >= p.capacity) continue;  // rejected on the host; never written
    const S* ks = reinterpret_cast<const S*>(p.key.data) + b * p.key.stride[0] + h * p.key.stride[1] +
                  t * p.key.stride[2];
    const S* vs = reinterpret_cast<const S*>(p.value.data) + b * p.value.stride[0] +
                  h * p.value.stride[1] + t * p.value.stride[2];
    D* kd = reinterpret_cast<D*>(p.key_cache.data) + b * p.key_cache.stride[0] +
            h * p.key_cache.stride[1] + dst_t * p.key_cache.stride[2];
    D* vd = reinterpret_cast<D*>(p.value_cache.data) + b * p.value_cache.stride[0] +
            h * p.value_cache.stride[1] + dst_t * p.value_cache.stride[2];
    for (int c = threadIdx.x; c < p.head_dim; c += blockDim.x)
      kd[c * p.key_cache.stride[3]] = convert_elem<S, D>(ks[c * p.key.stride[3]]);
    for (int c = threadIdx.x; c < p.value_dim; c += blockDim.x)
      vd[c * p.value_cache.stride[3]] = convert_elem<S, D>(vs[c * p.value.stride[3]]);
  }
  if (p.positions_out && h == 0 && blockIdx.x == 0 && threadIdx.x == 0)
    p.positions_out[b] = (int32_t)(pos + p.steps);
}

// Same-dtype fast path: 16-byte vectors, rows contiguous in channels.
__global__ void kv_append_vec_kernel(AppendLaunch L, int vec_k, int vec_v) {
  const ts_kv_append_params& p = L.p;
  const int b = blockIdx.z, h = blockIdx.y;
  const int64_t pos = p.positions ? (int64_t)p.positions[b] : p.position;
  const int esz = p.cache_dtype == TS_F64 ? 8 : (p.cache_dtype == TS_F32 ? 4 : 2);
  for (int t = blockIdx.x; t < p.steps; t += gridDim.x) {
    const int64_t dst_t = pos + t;
    if (dst_t < 0 || dst_t >= p.capacity) continue;
    const char* ks = reinterpret_cast<const char*>(p.key.data) +
                     (b * p.key.stride[0] + h * p.key.stride[1] + t * p.key.stride[2]) * esz;
    const char* vs = reinterpret_cast<const char*>(p.value.data) +
                     (b * p.value.stride[0] + h * p.value.stride[1] + t * p.value.stride[2]) * esz;
    char* kd = reinterpret_cast<char*>(p.key_cache.data) +
               (b * p.key_cache.stride[0] + h * p.key_cache.stride[1] + dst_t * p.key_cache.stride[2]) * esz;
    char* vd = reinterpret_cast<char*>(p.value_cache.data) +
               (b * p.value_cache.stride[0] + h * p.value_cache.stride[1] + dst_t * p.value_cache.stride[2]) *
                   esz;
    for (int c = threadIdx.x; c < vec_k; c += blockDim.x)
      reinterpret_cast<uint4*>(kd)[c] = reinterpret_cast<const uint4*>(ks)[c];
    for (int c = threadIdx.x; c < vec_v; c += blockDim.x)
      reinterpret_cast<uint4*>(vd)[c] = reinterpret_cast<const uint4*>(vs)[c];
  }
  if (p.positions_out && h == 0 && blockIdx.x == 0 && threadIdx.x == 0)
    p.positions_out[b] = (int32_t)(pos + p.steps);
}

template <typename S>
static cudaError_t append_src(const AppendLaunch& L, dim3 grid, int threads, cudaStream_t st) {
  switch (L.p.cache_dtype) {
    case TS_F32: kv_append_kernel<S, float><<<grid, threads, 0, st>>>(L); break;
    case TS_F64: kv_append_kernel<S, double><<<grid, threads, 0, st>>>(L); break;
    case TS_F16: kv_append_kernel<S, __half><<<grid, threads, 0, st>>>(L); break;
    case TS_BF16: kv_append_kernel<S, __nv_bfloat16><<<grid, threads, 0, st>>>(L); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

static int esize(int dtype) { return dtype == TS_F64 ? 8 : (dtype == TS_F32 ? 4 : 2); }

static bool vec_ok(const ts_view4& v, int channels, int esz) {
  if (v.stride[3] != 1) return false;
  if ((channels * esz) % 16) return false;
  for (int i = 0; i < 3; ++i)
    if ((v.stride[i] * esz) % 16) return false;
  return reinterpret_cast<uintptr_t>(v.data) % 16 == 0;
}

cudaError_t kv_append(const ts_kv_append_params& p, cudaStream_t st) {
  AppendLaunch L{p};
  const int blocks_t = p.steps < 65535 ? p.steps : 65535;
  dim3 grid(blocks_t, p.heads, p.batch);
  const int esz = esize(p.cache_dtype);
  if (p.src_dtype == p.cache_dtype && vec_ok(p.key, p.head_dim, esz) && vec_ok(p.value, p.value_dim, esz) &&
      vec_ok(p.key_cache, p.head_dim, esz) && vec_ok(p.value_cache, p.value_dim, esz)) {
    const int vk = p.head_dim * esz / 16, vv = p.value_dim * esz / 16;
    const int threads = ((vk > vv ? vk : vv) + 31) / 32 * 32;
    kv_append_vec_kernel<<<grid, threads, 0, st>>>(L, vk, vv);
    return cudaGetLastError();
  }
  const int threads = 128;
  switch (p.src_dtype) {
    case TS_F32: return append_src<float>(L, grid, threads, st);
    case TS_F64: return append_src<double>(L, grid, threads, st);
    case TS_F16: return append_src<__half>(L, grid, threads, st);
    case TS_BF16: return append_src<__nv_bfloat16>(L, grid, threads, st);
  }
  return cudaErrorInvalidValue;
}

// dst[b, h, t, c] = src[index[b], h, t, c] for t < length.
template <typename T>
__global__ void kv_reorder_kernel(ts_view4 src, ts_view4 dst, int heads, int length, int channels,
                                  const int32_t* index) {
  const int b = blockIdx.z, h = blockIdx.y;
  const int sb = index[b];
  for (int t = blockIdx.x; t < length; t += gridDim.x) {
    const T* s = reinterpret_cast<const T*>(src.data) + sb * src.stride[0] + h * src.stride[1] +
                 t * src.stride[2];
    T* d = reinterpret_cast<T*>(dst.data) + b * dst.stride[0] + h * dst.stride[1] + t * dst.stride[2];
    for (int c = threadIdx.x; c < channels; c += blockDim.x) d[c * dst.stride[3]] = s[c * src.stride[3]];
  }
}

cudaError_t kv_reorder(const ts_view4& src, const ts_view4& dst, int dtype, int batch, int heads,
                       int length, int channels, const int32_t* index, cudaStream_t st) {
  if (length <= 0) return cudaSuccess;
  dim3 grid(length < 65535 ? length : 65535, heads, batch);
  switch (dtype) {
    case TS_F32: kv_reorder_kernel<float><<<grid, 128, 0, st>>>(src, dst, heads, length, channels, index); break;
    case TS_F64: kv_reorder_kernel<double><<<grid, 128, 0, st>>>(src, dst, heads, length, channels, index); break;
    case TS_F16: kv_reorder_kernel<__half><<<grid, 128, 0, st>>>(src, dst, heads, length, channels, index); break;
    case TS_BF16:
      kv_reorder_kernel<__nv_bfloat16><<<grid, 128, 0, st>>>(src, dst, heads, length, channels, index);
      break;
    case TS_I8: kv_reorder_kernel<int8_t><<<grid, 128, 0, st>>>(src, dst, heads, length, channels, index); break;
    default: return cudaErrorInvalidValue;
  }
  return cudaGetLastError();
}

}  // namespace tsa
