// Templates of the generic CUDA-core attention kernels and their launchers,
// instantiated per dtype in attn_simt_{fwd,bwd}_{f32,f64,f16,bf16}.cu so the
// instantiations compile in parallel.
//
// The kernels cover every dtype
// (f32 / f64 / f16 / bf16), any head dims up to 256, Dv != D, GQA, causal
// offset, boolean / additive masks with broadcast strides and per-row valid
// key counts.  They are the exact-arithmetic path (fp32 ≤1e-4 relative to the
// reference) and the fallback for shapes the tensor-core kernel does not take.
//
// Semantics follow tensorsmith's nn/attention.py:
//   scores      :102-113  s = scale * q.k (+ additive mask), -inf where masked
//   forward     :175-198  online softmax, output a/l, LSE = m + log l (-inf if l = 0)
//   backward    :220-244  p = exp(s - LSE), ds = p (dO.v - rowsum(dO*O)) * scale
//   GQA reduce  :245-247  dK/dV summed over the query heads of a KV group
//   dropout     :140-144, 212-216 (kDrop instantiations): P.V uses p * keep / (1 - p),
//               dP is multiplied by the same factor; the mask is regenerated from a
//               counter-based generator (dropout.cuh) in every kernel.
//
// Thread layout: a group of G consecutive threads owns one row (a query row in
// the forward / dQ kernels, a key row in the dK/dV kernel).  Thread g of the
// group holds channels g, g+G, g+2G, ... so the G threads of a group read
// consecutive shared-memory words (no bank conflicts) and a row's dot product
// is a G-lane butterfly.
#pragma once
#include "dropout.cuh"
#include "simt.cuh"

namespace tsa {

template <typename A> struct SimtCfg {
  static constexpr int DPT = sizeof(A) == 8 ? 16 : 32;  // channels per thread
};
constexpr int kSimtThreads = 128;
constexpr int kSimtKeys = 32;     // keys staged per shared-memory tile
constexpr int kSimtQRows = 32;    // query rows staged per tile (dK/dV kernel)
constexpr int kStageBatch = 8;    // global loads in flight per thread while staging a tile

struct RowCtx {
  int b, h, hk, kv_end, offset;
};

__device__ __forceinline__ int row_kv_end(const ts_attn_params& p, int b) {
  int end = p.kv_len;
  if (p.kv_lens) end = min(end, max(0, p.kv_lens[b]));
  return end;
}
__device__ __forceinline__ int64_t row_offset(const ts_attn_params& p, int b) {
  if (!p.is_causal) return 0;
  if (p.kv_lens) return (int64_t)max(0, p.kv_lens[b]) - p.q_len;
  return p.causal_offset;
}

template <typename A>
__device__ __forceinline__ bool mask_apply(const ts_attn_params& p, int b, int h, int i, int j,
                                           A& s) {
  if (p.mask_kind == TS_MASK_NONE) return true;
  const int64_t idx = (int64_t)b * p.mask_stride[0] + (int64_t)h * p.mask_stride[1] +
                      (int64_t)i * p.mask_stride[2] + (int64_t)j * p.mask_stride[3];
  if (p.mask_kind == TS_MASK_BOOL) return reinterpret_cast<const uint8_t*>(p.mask)[idx] != 0;
  s += reinterpret_cast<const A*>(p.mask)[idx];
  return true;
}

template <typename T>
__device__ __forceinline__ const T* at4(const ts_view4& v, int b, int h, int t, int c) {
  return reinterpret_cast<const T*>(v.data) + (int64_t)b * v.stride[0] + (int64_t)h * v.stride[1] +
         (int64_t)t * v.stride[2] + (int64_t)c * v.stride[3];
}
template <typename T>
__device__ __forceinline__ T* at4w(const ts_view4& v, int b, int h, int t, int c) {
  return reinterpret_cast<T*>(v.data) + (int64_t)b * v.stride[0] + (int64_t)h * v.stride[1] +
         (int64_t)t * v.stride[2] + (int64_t)c * v.stride[3];
}

template <int G, typename A>
__device__ __forceinline__ A group_sum(A x) {
#pragma unroll
  for (int off = G / 2; off > 0; off >>= 1) x += __shfl_xor_sync(0xffffffffu, x, off);
  return x;
}

// Cooperative load of keys [k0, k0 + kSimtKeys) of (b, hk) into shared memory,
// converted to the accumulation type; rows at or beyond `end` are zero.
template <typename T, typename A>
__device__ __forceinline__ void stage_rows(A* dst, const ts_view4& src, int b, int hk, int k0,
                                           int rows, int end, int C) {
  // kStageBatch loads per thread are issued before any of them is stored, so
  // their latencies overlap instead of adding up one element at a time.
  const int n = rows * C;
  for (int base = threadIdx.x; base < n; base += blockDim.x * kStageBatch) {
    A tmp[kStageBatch];
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int idx = base + u * blockDim.x;
      const int r = idx / C, c = idx - r * C, t = k0 + r;
      tmp[u] = (idx < n && t < end) ? Elem<T>::to_acc(*at4<T>(src, b, hk, t, c)) : A(0);
    }
#pragma unroll
    for (int u = 0; u < kStageBatch; ++u) {
      const int idx = base + u * blockDim.x;
      if (idx < n) dst[idx] = tmp[u];
    }
  }
}

// ---------------------------------------------------------------------------
// Forward: one query row per G-thread group.
// ---------------------------------------------------------------------------
template <typename T, int G, bool kDrop>
__global__ void __launch_bounds__(kSimtThreads) simt_fwd_kernel(ts_attn_params p, DropoutArgs drop) {
  using A = typename Elem<T>::acc;
  constexpr int DPT = SimtCfg<A>::DPT;
  constexpr int R = kSimtThreads / G;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int D = p.head_dim, Dv = p.value_dim;
  A* ks = reinterpret_cast<A*>(smem_raw);
  A* vs = ks + kSimtKeys * D;

  const int g = threadIdx.x % G, rloc = threadIdx.x / G;
  const int b = blockIdx.z, h = blockIdx.y;
  const int i = blockIdx.x * R + rloc;
  const int hk = h / (p.q_heads / p.kv_heads);
  const bool row_ok = i < p.q_len;
  const int64_t offset = row_offset(p, b);
  int kv_end = row_kv_end(p, b);
  if (p.is_causal) {
    const int64_t last = min(blockIdx.x * R + R - 1, p.q_len - 1);
    kv_end = (int)i64max(0, i64min(kv_end, last + offset + 1));
  }
  const A scale = (A)p.scale;

  A q[DPT], o[DPT];
#pragma unroll
  for (int k = 0; k < DPT; ++k) {
    const int d = g + G * k;
    q[k] = (row_ok && d < D) ? Elem<T>::to_acc(*at4<T>(p.q, b, h, i, d)) * scale : A(0);
    o[k] = A(0);
  }
  A m = neg_inf<A>(), l = A(0);

  for (int k0 = 0; k0 < kv_end; k0 += kSimtKeys) {
    __syncthreads();
    stage_rows<T, A>(ks, p.k, b, hk, k0, kSimtKeys, kv_end, D);
    stage_rows<T, A>(vs, p.v, b, hk, k0, kSimtKeys, kv_end, Dv);
    __syncthreads();
    A s[kSimtKeys];
    A tile_max = neg_inf<A>();
#pragma unroll
    for (int jj = 0; jj < kSimtKeys; ++jj) {
      A part = A(0);
#pragma unroll
      for (int k = 0; k < DPT; ++k) {
        const int d = g + G * k;
        if (d < D) part += q[k] * ks[jj * D + d];
      }
      A sc = group_sum<G>(part);
      const int j = k0 + jj;
      bool ok = row_ok && j < kv_end && (!p.is_causal || (int64_t)i + offset >= j);
      if (ok) ok = mask_apply<A>(p, b, h, i, j, sc);
      s[jj] = ok ? sc : neg_inf<A>();
      tile_max = s[jj] > tile_max ? s[jj] : tile_max;
    }
    const A m_new = tile_max > m ? tile_max : m;
    const A safe = m_new == neg_inf<A>() ? A(0) : m_new;
    const A corr = acc_exp(m - safe);
    l *= corr;
#pragma unroll
    for (int k = 0; k < DPT; ++k) o[k] *= corr;
    uint32_t keep = 0xffffffffu;
    if constexpr (kDrop) {
      keep = 0;
      const uint32_t bh = (uint32_t)(b * p.q_heads + h);
#pragma unroll
      for (int j8 = 0; j8 < kSimtKeys / 8; ++j8)
        keep |= dropout_keep8(drop, bh, (uint32_t)i, (uint32_t)(k0 / 8 + j8)) << (8 * j8);
    }
#pragma unroll
    for (int jj = 0; jj < kSimtKeys; ++jj) {
      const A pj = acc_exp(s[jj] - safe);
      l += pj;
      const A pv = kDrop ? ((keep >> jj) & 1u ? pj * dropout_scale<A>(drop) : A(0)) : pj;
#pragma unroll
      for (int k = 0; k < DPT; ++k) {
        const int d = g + G * k;
        if (d < Dv) o[k] += pv * vs[jj * Dv + d];
      }
    }
    m = m_new;
  }
  if (!row_ok) return;
  const A inv = l > A(0) ? A(1) / l : A(0);
#pragma unroll
  for (int k = 0; k < DPT; ++k) {
    const int d = g + G * k;
    if (d < Dv) *at4w<T>(p.o, b, h, i, d) = Elem<T>::from_acc(o[k] * inv);
  }
  if (p.lse && g == 0) {
    const A lse = l > A(0) ? m + acc_log(l) : neg_inf<A>();
    reinterpret_cast<A*>(p.lse)[(int64_t)b * p.lse_stride[0] + (int64_t)h * p.lse_stride[1] +
                                (int64_t)i * p.lse_stride[2]] = lse;
  }
}

// ---------------------------------------------------------------------------
// Backward preprocess: delta[b,h,i] = sum_c dO * O   (nn/attention.py:231)
// One warp per query row.
// ---------------------------------------------------------------------------
template <typename T>
__global__ void simt_bwd_delta_kernel(ts_attn_bwd_params bp, typename Elem<T>::acc* delta) {
  using A = typename Elem<T>::acc;
  const ts_attn_params& p = bp.fwd;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int rows = p.batch * p.q_heads * p.q_len;
  if (warp >= rows) return;
  const int i = warp % p.q_len, h = (warp / p.q_len) % p.q_heads, b = warp / (p.q_len * p.q_heads);
  A acc = A(0);
  for (int c = lane; c < p.value_dim; c += 32)
    acc += Elem<T>::to_acc(*at4<T>(bp.dout, b, h, i, c)) * Elem<T>::to_acc(*at4<T>(p.o, b, h, i, c));
  acc = group_sum<32>(acc);
  if (lane == 0) delta[warp] = acc;
}

// ---------------------------------------------------------------------------
// dQ: one query row per group; loops over the row's visible keys.
// ---------------------------------------------------------------------------
template <typename T, int G, bool kDrop>
__global__ void __launch_bounds__(kSimtThreads)
    simt_bwd_dq_kernel(ts_attn_bwd_params bp, const typename Elem<T>::acc* delta, DropoutArgs drop) {
  using A = typename Elem<T>::acc;
  constexpr int DPT = SimtCfg<A>::DPT;
  constexpr int R = kSimtThreads / G;
  const ts_attn_params& p = bp.fwd;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int D = p.head_dim, Dv = p.value_dim;
  A* ks = reinterpret_cast<A*>(smem_raw);
  A* vs = ks + kSimtKeys * D;

  const int g = threadIdx.x % G, rloc = threadIdx.x / G;
  const int b = blockIdx.z, h = blockIdx.y;
  const int i = blockIdx.x * R + rloc;
  const int hk = h / (p.q_heads / p.kv_heads);
  const bool row_ok = i < p.q_len;
  const int64_t offset = row_offset(p, b);
  int kv_end = row_kv_end(p, b);
  if (p.is_causal) {
    const int64_t last = min(blockIdx.x * R + R - 1, p.q_len - 1);
    kv_end = (int)i64max(0, i64min(kv_end, last + offset + 1));
  }
  const A scale = (A)p.scale;
  const int64_t row = ((int64_t)b * p.q_heads + h) * p.q_len + i;
  A lse = A(0), dlt = A(0);
  bool live = false;
  if (row_ok) {
    const A lv = reinterpret_cast<const A*>(p.lse)[(int64_t)b * p.lse_stride[0] +
                                                   (int64_t)h * p.lse_stride[1] + (int64_t)i * p.lse_stride[2]];
    live = lv != neg_inf<A>();
    lse = live ? lv : A(0);
    dlt = delta[row];
  }
  A q[DPT], dO[DPT], dq[DPT];
#pragma unroll
  for (int k = 0; k < DPT; ++k) {
    const int d = g + G * k;
    q[k] = (row_ok && d < D) ? Elem<T>::to_acc(*at4<T>(p.q, b, h, i, d)) : A(0);
    dO[k] = (row_ok && d < Dv) ? Elem<T>::to_acc(*at4<T>(bp.dout, b, h, i, d)) : A(0);
    dq[k] = A(0);
  }
  for (int k0 = 0; k0 < kv_end; k0 += kSimtKeys) {
    __syncthreads();
    stage_rows<T, A>(ks, p.k, b, hk, k0, kSimtKeys, kv_end, D);
    stage_rows<T, A>(vs, p.v, b, hk, k0, kSimtKeys, kv_end, Dv);
    __syncthreads();
    uint32_t keep = 0xffffffffu;
    if constexpr (kDrop) {
      keep = 0;
      const uint32_t bh = (uint32_t)(b * p.q_heads + h);
#pragma unroll
      for (int j8 = 0; j8 < kSimtKeys / 8; ++j8)
        keep |= dropout_keep8(drop, bh, (uint32_t)i, (uint32_t)(k0 / 8 + j8)) << (8 * j8);
    }
#pragma unroll 4
    for (int jj = 0; jj < kSimtKeys; ++jj) {
      A sp = A(0), dp = A(0);
#pragma unroll
      for (int k = 0; k < DPT; ++k) {
        const int d = g + G * k;
        if (d < D) sp += q[k] * ks[jj * D + d];
        if (d < Dv) dp += dO[k] * vs[jj * Dv + d];
      }
      sp = group_sum<G>(sp) * scale;
      dp = group_sum<G>(dp);
      const int j = k0 + jj;
      bool ok = live && j < kv_end && (!p.is_causal || (int64_t)i + offset >= j);
      if (ok) ok = mask_apply<A>(p, b, h, i, j, sp);
      const A pr = ok ? acc_exp(sp - lse) : A(0);
      if constexpr (kDrop) dp = (keep >> jj) & 1u ? dp * dropout_scale<A>(drop) : A(0);
      const A ds = pr * (dp - dlt) * scale;
#pragma unroll
      for (int k = 0; k < DPT; ++k) {
        const int d = g + G * k;
        if (d < D) dq[k] += ds * ks[jj * D + d];
      }
    }
  }
  if (!row_ok) return;
#pragma unroll
  for (int k = 0; k < DPT; ++k) {
    const int d = g + G * k;
    if (d < D) *at4w<T>(bp.dq, b, h, i, d) = Elem<T>::from_acc(dq[k]);
  }
}

// ---------------------------------------------------------------------------
// dK / dV: one key row per group; loops over every query head of the KV
// group and the query rows that see the key (GQA reduction in registers).
// ---------------------------------------------------------------------------
template <typename T, int G, bool kDrop>
__global__ void __launch_bounds__(kSimtThreads)
    simt_bwd_dkdv_kernel(ts_attn_bwd_params bp, const typename Elem<T>::acc* delta, DropoutArgs drop) {
  using A = typename Elem<T>::acc;
  constexpr int DPT = SimtCfg<A>::DPT;
  constexpr int R = kSimtThreads / G;
  const ts_attn_params& p = bp.fwd;
  extern __shared__ __align__(16) unsigned char smem_raw[];
  const int D = p.head_dim, Dv = p.value_dim;
  A* qs = reinterpret_cast<A*>(smem_raw);  // [kSimtQRows][D]
  A* gs = qs + kSimtQRows * D;             // [kSimtQRows][Dv]
  A* ls = gs + kSimtQRows * Dv;            // [kSimtQRows] lse (0 where fully masked)
  A* ds_ = ls + kSimtQRows;                // [kSimtQRows] delta
  uint8_t* lv = reinterpret_cast<uint8_t*>(ds_ + kSimtQRows);  // row has finite lse

  const int g = threadIdx.x % G, rloc = threadIdx.x / G;
  const int b = blockIdx.z, hk = blockIdx.y;
  const int j = blockIdx.x * R + rloc;
  const int rep = p.q_heads / p.kv_heads;
  const int kv_end = row_kv_end(p, b);
  const bool key_ok = j < kv_end;
  const int64_t offset = row_offset(p, b);
  const A scale = (A)p.scale;

  A kr[DPT], vr[DPT], dk[DPT], dv[DPT];
#pragma unroll
  for (int k = 0; k < DPT; ++k) {
    const int d = g + G * k;
    kr[k] = (key_ok && d < D) ? Elem<T>::to_acc(*at4<T>(p.k, b, hk, j, d)) : A(0);
    vr[k] = (key_ok && d < Dv) ? Elem<T>::to_acc(*at4<T>(p.v, b, hk, j, d)) : A(0);
    dk[k] = A(0);
    dv[k] = A(0);
  }
  // First query row that can see the block's first key.
  int i_begin = 0;
  if (p.is_causal) i_begin = (int)i64max(0, (int64_t)blockIdx.x * R - offset);
  i_begin = (i_begin / kSimtQRows) * kSimtQRows;
  const bool block_live = blockIdx.x * R < kv_end;

  for (int r = 0; r < rep && block_live; ++r) {
    const int h = hk * rep + r;
    for (int i0 = i_begin; i0 < p.q_len; i0 += kSimtQRows) {
      __syncthreads();
      stage_rows<T, A>(qs, p.q, b, h, i0, kSimtQRows, p.q_len, D);
      stage_rows<T, A>(gs, bp.dout, b, h, i0, kSimtQRows, p.q_len, Dv);
      if (threadIdx.x < kSimtQRows) {
        const int i = i0 + threadIdx.x;
        A lval = neg_inf<A>();
        A dval = A(0);
        if (i < p.q_len) {
          lval = reinterpret_cast<const A*>(p.lse)[(int64_t)b * p.lse_stride[0] + (int64_t)h * p.lse_stride[1] +
                                                   (int64_t)i * p.lse_stride[2]];
          dval = delta[((int64_t)b * p.q_heads + h) * p.q_len + i];
        }
        lv[threadIdx.x] = (i < p.q_len && lval != neg_inf<A>()) ? 1 : 0;
        ls[threadIdx.x] = lv[threadIdx.x] ? lval : A(0);
        ds_[threadIdx.x] = dval;
      }
      __syncthreads();
#pragma unroll 2
      for (int ii = 0; ii < kSimtQRows; ++ii) {
        const int i = i0 + ii;
        A sp = A(0), dp = A(0);
#pragma unroll
        for (int k = 0; k < DPT; ++k) {
          const int d = g + G * k;
          if (d < D) sp += kr[k] * qs[ii * D + d];
          if (d < Dv) dp += vr[k] * gs[ii * Dv + d];
        }
        sp = group_sum<G>(sp) * scale;
        dp = group_sum<G>(dp);
        bool ok = key_ok && lv[ii] && (!p.is_causal || (int64_t)i + offset >= j);
        if (ok) ok = mask_apply<A>(p, b, h, i, j, sp);
        const A pr = ok ? acc_exp(sp - ls[ii]) : A(0);
        A pv = pr;
        if constexpr (kDrop) {
          const A f = dropout_keep(drop, (uint32_t)(b * p.q_heads + h), (uint32_t)i, (uint32_t)j)
                          ? dropout_scale<A>(drop) : A(0);
          pv = pr * f;
          dp = dp * f;
        }
        const A dsv = pr * (dp - ds_[ii]) * scale;
#pragma unroll
        for (int k = 0; k < DPT; ++k) {
          const int d = g + G * k;
          if (d < Dv) dv[k] += pv * gs[ii * Dv + d];
          if (d < D) dk[k] += dsv * qs[ii * D + d];
        }
      }
    }
  }
  if (j >= p.kv_len) return;
#pragma unroll
  for (int k = 0; k < DPT; ++k) {
    const int d = g + G * k;
    if (d < D) *at4w<T>(bp.dk, b, hk, j, d) = Elem<T>::from_acc(dk[k]);
    if (d < Dv) *at4w<T>(bp.dv, b, hk, j, d) = Elem<T>::from_acc(dv[k]);
  }
}

// ---------------------------------------------------------------------------
// Host-side launchers
// ---------------------------------------------------------------------------
template <typename A> inline int simt_group(int dmax) {
  const int dpt = SimtCfg<A>::DPT;
  int g = 1;
  while (g * dpt < dmax) g <<= 1;
  return g;
}

template <typename T, int G>
inline cudaError_t launch_fwd_g(const ts_attn_params& p, const DropoutArgs* drop, cudaStream_t st) {
  using A = typename Elem<T>::acc;
  constexpr int R = kSimtThreads / G;
  const size_t smem = sizeof(A) * kSimtKeys * (p.head_dim + p.value_dim);
  auto kern = drop ? simt_fwd_kernel<T, G, true> : simt_fwd_kernel<T, G, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(ceil_div(p.q_len, R), p.q_heads, p.batch);
  kern<<<grid, kSimtThreads, smem, st>>>(p, drop ? *drop : DropoutArgs{});
  return cudaGetLastError();
}

template <typename T, int G>
inline cudaError_t launch_bwd_g(const ts_attn_bwd_params& bp, typename Elem<T>::acc* delta,
                                const DropoutArgs* drop, cudaStream_t st) {
  const DropoutArgs d = drop ? *drop : DropoutArgs{};
  using A = typename Elem<T>::acc;
  constexpr int R = kSimtThreads / G;
  const ts_attn_params& p = bp.fwd;
  const int rows = p.batch * p.q_heads * p.q_len;
  simt_bwd_delta_kernel<T><<<ceil_div(rows * 32, 256), 256, 0, st>>>(bp, delta);
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  const size_t smem_dq = sizeof(A) * kSimtKeys * (p.head_dim + p.value_dim);
  auto kdq = drop ? simt_bwd_dq_kernel<T, G, true> : simt_bwd_dq_kernel<T, G, false>;
  e = cudaFuncSetAttribute(kdq, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_dq);
  if (e != cudaSuccess) return e;
  kdq<<<dim3(ceil_div(p.q_len, R), p.q_heads, p.batch), kSimtThreads, smem_dq, st>>>(bp, delta, d);
  e = cudaGetLastError();
  if (e != cudaSuccess) return e;

  const size_t smem_kv = sizeof(A) * (kSimtQRows * (p.head_dim + p.value_dim) + 2 * kSimtQRows) +
                         kSimtQRows;
  auto kkv = drop ? simt_bwd_dkdv_kernel<T, G, true> : simt_bwd_dkdv_kernel<T, G, false>;
  e = cudaFuncSetAttribute(kkv, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_kv);
  if (e != cudaSuccess) return e;
  kkv<<<dim3(ceil_div(p.kv_len, R), p.kv_heads, p.batch), kSimtThreads, smem_kv, st>>>(bp, delta, d);
  return cudaGetLastError();
}

// SMs of the current device (cached per device).
inline int simt_sm_count() {
  static int cached[64] = {0};
  int dev = 0;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
  if (cached[dev] == 0) {
    int n = 0;
    cached[dev] = cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) == cudaSuccess && n > 0 ? n : 148;
  }
  return cached[dev];
}

// Threads per row: the fewest that cover the channels (more channels per
// thread, fewer shuffles), widened while the grid of `rows` rows in `slices`
// (batch x head) grids would leave SMs idle (small problems: the BASELINE C1
// shape has 8 (b,h) slices of 256 rows).
template <typename A> inline int simt_group_for(int dmax, int rows, int slices) {
  int g = simt_group<A>(dmax);
  const int64_t want = 2 * (int64_t)simt_sm_count();
  while (g < 16 && (int64_t)ceil_div(rows, kSimtThreads / g) * slices < want) g <<= 1;
  return g;
}

template <typename T>
inline cudaError_t simt_fwd_t(const ts_attn_params& p, const DropoutArgs* drop, cudaStream_t st) {
  using A = typename Elem<T>::acc;
  switch (simt_group_for<A>(max(p.head_dim, p.value_dim), p.q_len, p.batch * p.q_heads)) {
    case 1: return launch_fwd_g<T, 1>(p, drop, st);
    case 2: return launch_fwd_g<T, 2>(p, drop, st);
    case 4: return launch_fwd_g<T, 4>(p, drop, st);
    case 8: return launch_fwd_g<T, 8>(p, drop, st);
    case 16: return launch_fwd_g<T, 16>(p, drop, st);
    default: return cudaErrorInvalidValue;
  }
}

template <typename T>
inline cudaError_t simt_bwd_t(const ts_attn_bwd_params& bp, void* ws, const DropoutArgs* drop, cudaStream_t st) {
  using A = typename Elem<T>::acc;
  A* delta = reinterpret_cast<A*>(ws);
  const ts_attn_params& p = bp.fwd;
  switch (simt_group_for<A>(max(p.head_dim, p.value_dim), min(p.q_len, p.kv_len),
                            p.batch * min(p.q_heads, p.kv_heads))) {
    case 1: return launch_bwd_g<T, 1>(bp, delta, drop, st);
    case 2: return launch_bwd_g<T, 2>(bp, delta, drop, st);
    case 4: return launch_bwd_g<T, 4>(bp, delta, drop, st);
    case 8: return launch_bwd_g<T, 8>(bp, delta, drop, st);
    case 16: return launch_bwd_g<T, 16>(bp, delta, drop, st);
    default: return cudaErrorInvalidValue;
  }
}

}  // namespace tsa
