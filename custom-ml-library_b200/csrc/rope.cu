// Rotary position embedding (tensorsmith nn/attention.py:255-296) and its
// fusion with the KV-cache append (nn/cache.py:54-86).
//
// Interleaved pairs: for pair i of a row at absolute position pos,
//   angle = pos * inv_freq[i]            (fp32, inv_freq = base^(-2i/dim))
//   y[2i]   = x[2i]   * cos - x[2i+1] * sin
//   y[2i+1] = x[2i+1] * cos + x[2i]   * sin
// with cos / sin rounded to the element type first and every product and sum
// rounded to it, as the reference evaluates `part * cos + rotate(part) * sin`
// in the input dtype.  Channels past rotary_dim are copied unchanged.  The
// inverse rotation (sin negated) is the VJP (:287-293).
//
// One CTA per (sequence position, batch row): its threads compute sin/cos of
// the position's pairs once and apply them to every head, with consecutive
// threads touching consecutive pairs (coalesced).
#include "common.cuh"
#include "rope.cuh"

namespace tsa {

template <typename T>
__device__ __forceinline__ typename Elem<T>::acc rnd(typename Elem<T>::acc x) {
  return Elem<T>::to_acc(Elem<T>::from_acc(x));
}

struct RopeLaunch {
  ts_view4 x, y;        // [B, H, T, C] in / out (may alias)
  int batch, heads, seq, channels, rotary_dim;
  int64_t offset;       // position of t = 0 when positions == NULL
  const int32_t* positions;
  const float* inv_freq;  // [rotary_dim / 2]
  float sign;           // +1 forward, -1 inverse (VJP)
  // KV-append fusion: when cache.data != NULL, y is ignored and rows go to
  // cache[b, h, pos_b + t] (pos_b = positions[b] or offset); value rows copied.
  ts_view4 vx, vcache;
  ts_view4 cache;
  int value_dim;
  int32_t* positions_out;
};

template <typename T, typename C>
__global__ void rope_kernel(RopeLaunch L) {
  using A = typename Elem<T>::acc;
  const int t = blockIdx.x, b = blockIdx.y;
  const int64_t base = L.positions ? (int64_t)L.positions[b] : L.offset;
  const int64_t pos = base + t;
  const bool to_cache = L.cache.data != nullptr;
  const int pairs = L.rotary_dim / 2;
  for (int i = threadIdx.x; i < pairs; i += blockDim.x) {
    const float angle = (float)pos * L.inv_freq[i];
    float sf, cf;
    sincosf(angle, &sf, &cf);
    const A c = rnd<T>((A)cf), s = rnd<T>((A)sf) * (A)L.sign;
    for (int h = 0; h < L.heads; ++h) {
      const T* xp = reinterpret_cast<const T*>(L.x.data) + b * L.x.stride[0] + h * L.x.stride[1] +
                    t * L.x.stride[2];
      const A x0 = Elem<T>::to_acc(xp[(2 * i) * L.x.stride[3]]);
      const A x1 = Elem<T>::to_acc(xp[(2 * i + 1) * L.x.stride[3]]);
      const A y0 = rnd<T>(rnd<T>(x0 * c) - rnd<T>(x1 * s));
      const A y1 = rnd<T>(rnd<T>(x1 * c) + rnd<T>(x0 * s));
      if (to_cache) {
        C* cp = reinterpret_cast<C*>(L.cache.data) + b * L.cache.stride[0] + h * L.cache.stride[1] +
                pos * L.cache.stride[2];
        cp[(2 * i) * L.cache.stride[3]] = Elem<C>::from_acc((typename Elem<C>::acc)y0);
        cp[(2 * i + 1) * L.cache.stride[3]] = Elem<C>::from_acc((typename Elem<C>::acc)y1);
      } else {
        T* yp = reinterpret_cast<T*>(L.y.data) + b * L.y.stride[0] + h * L.y.stride[1] + t * L.y.stride[2];
        yp[(2 * i) * L.y.stride[3]] = Elem<T>::from_acc(y0);
        yp[(2 * i + 1) * L.y.stride[3]] = Elem<T>::from_acc(y1);
      }
    }
  }
  // Channels past rotary_dim, and (fused append) the value rows.
  for (int h = 0; h < L.heads; ++h) {
    const T* xp = reinterpret_cast<const T*>(L.x.data) + b * L.x.stride[0] + h * L.x.stride[1] + t * L.x.stride[2];
    for (int c = L.rotary_dim + threadIdx.x; c < L.channels; c += blockDim.x) {
      const T v = xp[c * L.x.stride[3]];
      if (to_cache) {
        C* cp = reinterpret_cast<C*>(L.cache.data) + b * L.cache.stride[0] + h * L.cache.stride[1] +
                pos * L.cache.stride[2];
        cp[c * L.cache.stride[3]] = Elem<C>::from_acc((typename Elem<C>::acc)Elem<T>::to_acc(v));
      } else {
        T* yp = reinterpret_cast<T*>(L.y.data) + b * L.y.stride[0] + h * L.y.stride[1] + t * L.y.stride[2];
        yp[c * L.y.stride[3]] = v;
      }
    }
    if (to_cache) {
      const T* vp = reinterpret_cast<const T*>(L.vx.data) + b * L.vx.stride[0] + h * L.vx.stride[1] +
                    t * L.vx.stride[2];
      C* cp = reinterpret_cast<C*>(L.vcache.data) + b * L.vcache.stride[0] + h * L.vcache.stride[1] +
              pos * L.vcache.stride[2];
      for (int c = threadIdx.x; c < L.value_dim; c += blockDim.x)
        cp[c * L.vcache.stride[3]] =
            Elem<C>::from_acc((typename Elem<C>::acc)Elem<T>::to_acc(vp[c * L.vx.stride[3]]));
    }
  }
  if (L.positions_out && t == 0 && threadIdx.x == 0) L.positions_out[b] = (int32_t)(base + L.seq);
}

template <typename T>
static cudaError_t launch_t(const RopeLaunch& L, int cache_dtype, cudaStream_t st) {
  const dim3 grid(L.seq, L.batch);
  const int threads = 128;
  if (!L.cache.data) {
    rope_kernel<T, T><<<grid, threads, 0, st>>>(L);
  } else {
    switch (cache_dtype) {
      case TS_F32: rope_kernel<T, float><<<grid, threads, 0, st>>>(L); break;
      case TS_F64: rope_kernel<T, double><<<grid, threads, 0, st>>>(L); break;
      case TS_F16: rope_kernel<T, __half><<<grid, threads, 0, st>>>(L); break;
      case TS_BF16: rope_kernel<T, __nv_bfloat16><<<grid, threads, 0, st>>>(L); break;
      default: return cudaErrorInvalidValue;
    }
  }
  return cudaGetLastError();
}

static cudaError_t launch(const RopeLaunch& L, int dtype, int cache_dtype, cudaStream_t st) {
  switch (dtype) {
    case TS_F32: return launch_t<float>(L, cache_dtype, st);
    case TS_F64: return launch_t<double>(L, cache_dtype, st);
    case TS_F16: return launch_t<__half>(L, cache_dtype, st);
    case TS_BF16: return launch_t<__nv_bfloat16>(L, cache_dtype, st);
  }
  return cudaErrorInvalidValue;
}

cudaError_t rope_apply(const ts_view4& x, const ts_view4& y, int dtype, int batch, int heads, int seq,
                       int channels, int rotary_dim, int64_t offset, const int32_t* positions,
                       const float* inv_freq, int inverse, cudaStream_t st) {
  RopeLaunch L = {};
  L.x = x;
  L.y = y;
  L.batch = batch;
  L.heads = heads;
  L.seq = seq;
  L.channels = channels;
  L.rotary_dim = rotary_dim;
  L.offset = offset;
  L.positions = positions;
  L.inv_freq = inv_freq;
  L.sign = inverse ? -1.f : 1.f;
  return launch(L, dtype, dtype, st);
}

cudaError_t kv_append_rope(const ts_kv_append_params& p, const float* inv_freq, int rotary_dim, cudaStream_t st) {
  RopeLaunch L = {};
  L.x = p.key;
  L.batch = p.batch;
  L.heads = p.heads;
  L.seq = p.steps;
  L.channels = p.head_dim;
  L.rotary_dim = rotary_dim;
  L.offset = p.position;
  L.positions = p.positions;
  L.inv_freq = inv_freq;
  L.sign = 1.f;
  L.vx = p.value;
  L.vcache = p.value_cache;
  L.cache = p.key_cache;
  L.value_dim = p.value_dim;
  L.positions_out = p.positions_out;
  return launch(L, p.src_dtype, p.cache_dtype, st);
}

}  // namespace tsa
