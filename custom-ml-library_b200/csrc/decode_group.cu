// Split-K decode for several query rows per KV head: grouped-query attention
// (nn/attention.py:93-100 broadcasts each KV head to its query heads; here the
// group reads the KV head once) and multi-token decode steps.
//
// Same CTA shape and 4-stage bulk-copy ring of 32-key chunks as the one-row
// decode (decode.cu), with the layout that keeps the per-key work low when
// every key row meets several query rows:
//   * a lane holds 16 channels of a key row (32 bytes of a half-precision
//     row), so a row needs D/16 lanes and a dot product 3 butterfly levels at
//     D = 128;
//   * each lane exponentiates only the keys it holds, against the warp's
//     running max (butterfly over the row slots), and the accumulator is
//     rescaled only when that max grows (warp-uniform);
//   * dot products and P.V run as packed f32x2 FMAs;
//   * a CTA takes two query rows; larger groups are split over CTAs that are
//     adjacent in the grid, so their K/V reads meet in L2;
//   * 3 ring stages and at most 96 registers per thread let 4 CTAs share an
//     SM (the kernel is latency-bound: 4 CTAs ran 12 % faster than 3 with 4
//     stages).
// Partials use the workspace layout of decode.cu, so the caller's workspace
// size and the combine step are shared.
#include "decode.cuh"
#include "ptx.cuh"

namespace tsa {

namespace {
constexpr int kChunk = 32;
constexpr int kStages = 3;
constexpr int kComputeWarps = 4;
constexpr int kThreads = (kComputeWarps + 1) * 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

// 16 elements at `src` (16-byte aligned) -> 8 packed fp32 pairs.
template <typename T> struct Unpack16;
template <> struct Unpack16<__nv_bfloat16> {
  static __device__ __forceinline__ void run(const unsigned char* src, uint64_t (&f)[8]) {
    const uint4 a = *reinterpret_cast<const uint4*>(src), b = *reinterpret_cast<const uint4*>(src + 16);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) f[i] = ptx::f2pack(__uint_as_float(w[i] << 16), __uint_as_float(w[i] & 0xFFFF0000u));
  }
};
template <> struct Unpack16<__half> {
  static __device__ __forceinline__ void run(const unsigned char* src, uint64_t (&f)[8]) {
    const uint4 a = *reinterpret_cast<const uint4*>(src), b = *reinterpret_cast<const uint4*>(src + 16);
    const uint32_t w[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const float2 x = __half22float2(*reinterpret_cast<const __half2*>(&w[i]));
      f[i] = ptx::f2pack(x.x, x.y);
    }
  }
};
template <> struct Unpack16<float> {
  static __device__ __forceinline__ void run(const unsigned char* src, uint64_t (&f)[8]) {
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const uint4 a = *reinterpret_cast<const uint4*>(src + 16 * i);
      f[2 * i] = ptx::f2pack(__uint_as_float(a.x), __uint_as_float(a.y));
      f[2 * i + 1] = ptx::f2pack(__uint_as_float(a.z), __uint_as_float(a.w));
    }
  }
};

struct GroupLaunch {
  ts_attn_params p;
  int split_keys, max_splits;
  int n_groups;  // query-row groups of NQ rows per KV head (grid.x = splits * groups)
  float* ws_acc;
  float* ws_ml;
  uint32_t* fault;
};

__device__ __forceinline__ void group_row_range(const ts_attn_params& p, int b, int& end, int64_t& offset) {
  end = p.kv_len;
  offset = p.causal_offset;
  if (p.kv_lens) {
    end = min(end, max(0, p.kv_lens[b]));
    offset = (int64_t)end - p.q_len;
  }
  if (p.is_causal) end = (int)i64max(0, i64min(end, offset + p.q_len));
}
}  // namespace

template <typename T, int D, int NQ>
__global__ void __launch_bounds__(kThreads, 4) decode_group_kernel(GroupLaunch L) {
  const ts_attn_params& p = L.p;
  constexpr int kVec = 16;                   // elements per lane per row
  constexpr int kLanesPerRow = D / kVec;     // 4, 8, 16
  constexpr int kRowsPerWarp = 32 / kLanesPerRow;
  constexpr int kRowsPerWarpChunk = kChunk / kComputeWarps;  // 8
  constexpr int kIters = kRowsPerWarpChunk / kRowsPerWarp;
  constexpr int kRowBytes = D * (int)sizeof(T);
  constexpr int kStageBytes = kChunk * kRowBytes;

  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* kbuf = smem;
  unsigned char* vbuf = smem + kStages * kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * kStages * kStageBytes);
  uint64_t* empty = full + kStages;

  const int split = blockIdx.x / L.n_groups, grp = blockIdx.x - split * L.n_groups;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int rep = p.q_heads / p.kv_heads;
  const int n0 = grp * NQ;
  const int nq_used = min(NQ, rep * p.q_len - n0);
  int end;
  int64_t offset;
  group_row_range(p, b, end, offset);
  const int n_splits = max(1, ceil_div(end, L.split_keys));
  if (split >= n_splits) return;
  const int k_begin = split * L.split_keys;
  const int k_end = min(end, k_begin + L.split_keys);
  const int n_chunks = k_end > k_begin ? ceil_div(k_end - k_begin, kChunk) : 0;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], kComputeWarps);
    }
    ptx::fence_mbar_init();
  }
  __syncthreads();
  const T* kbase = reinterpret_cast<const T*>(p.k.data) + (int64_t)b * p.k.stride[0] + (int64_t)hk * p.k.stride[1];
  const T* vbase = reinterpret_cast<const T*>(p.v.data) + (int64_t)b * p.v.stride[0] + (int64_t)hk * p.v.stride[1];

  if (warp == kComputeWarps) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      const bool k_contig = p.k.stride[2] == D, v_contig = p.v.stride[2] == D;
      for (int c = 0; c < n_chunks; ++c) {
        const int s = c % kStages;
        if (c >= kStages && !ptx::mbar_wait(&empty[s], ((c / kStages) - 1) & 1, L.fault, FAULT_DEC_EMPTY)) break;
        const int r0 = k_begin + c * kChunk;
        const int rows = min(kChunk, k_end - r0);
        ptx::mbar_expect_tx(&full[s], 2u * rows * kRowBytes);
        unsigned char* kd = kbuf + s * kStageBytes;
        unsigned char* vd = vbuf + s * kStageBytes;
        if (k_contig) {
          ptx::bulk_g2s(kd, kbase + (int64_t)r0 * D, rows * kRowBytes, &full[s]);
        } else {
          for (int r = 0; r < rows; ++r)
            ptx::bulk_g2s(kd + r * kRowBytes, kbase + (int64_t)(r0 + r) * p.k.stride[2], kRowBytes, &full[s]);
        }
        if (v_contig) {
          ptx::bulk_g2s(vd, vbase + (int64_t)r0 * D, rows * kRowBytes, &full[s]);
        } else {
          for (int r = 0; r < rows; ++r)
            ptx::bulk_g2s(vd + r * kRowBytes, vbase + (int64_t)(r0 + r) * p.v.stride[2], kRowBytes, &full[s]);
        }
      }
      // Drain: every issued copy must land before the CTA exits.
      const int first = max(0, n_chunks - kStages);
      for (int c = first; c < n_chunks; ++c)
        if (!ptx::mbar_wait(&full[c % kStages], (c / kStages) & 1, L.fault, FAULT_DEC_FULL)) break;
    }
    return;
  }

  // ------------------------------- compute --------------------------------
  const int sub = lane / kLanesPerRow;
  const int cvec = lane % kLanesPerRow;
  const float qscale = (float)p.scale * kLog2e;
  uint64_t qf[NQ][8];
#pragma unroll
  for (int n = 0; n < NQ; ++n) {
    const int r = (n0 + n) / p.q_len, t = (n0 + n) - r * p.q_len;
    const bool live = n < nq_used;
    const int h = hk * rep + (live ? r : 0);
    const T* qp = reinterpret_cast<const T*>(p.q.data) + (int64_t)b * p.q.stride[0] + (int64_t)h * p.q.stride[1] +
                  (int64_t)(live ? t : 0) * p.q.stride[2];
#pragma unroll
    for (int i = 0; i < 8; ++i) {
      const int e = cvec * kVec + 2 * i;
      const float a0 = live ? Elem<T>::to_acc(qp[(int64_t)e * p.q.stride[3]]) * qscale : 0.f;
      const float a1 = live ? Elem<T>::to_acc(qp[(int64_t)(e + 1) * p.q.stride[3]]) * qscale : 0.f;
      qf[n][i] = ptx::f2pack(a0, a1);
    }
  }
  float m[NQ], l[NQ];
  uint64_t acc[NQ][8];
#pragma unroll
  for (int n = 0; n < NQ; ++n) {
    m[n] = -INFINITY;
    l[n] = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[n][i] = 0ull;
  }
  bool ok = true;
  for (int c = 0; c < n_chunks && ok; ++c) {
    const int s = c % kStages;
    const int r0 = k_begin + c * kChunk;
    int key[kIters];
#pragma unroll
    for (int it = 0; it < kIters; ++it) key[it] = r0 + warp * kRowsPerWarpChunk + it * kRowsPerWarp + sub;
    if (!ptx::mbar_wait(&full[s], (c / kStages) & 1, L.fault, FAULT_DEC_FULL)) {
      ok = false;
      break;
    }
    const unsigned char* kd = kbuf + s * kStageBytes;
    const unsigned char* vd = vbuf + s * kStageBytes;
    float sc[NQ][kIters];
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      const int row = warp * kRowsPerWarpChunk + it * kRowsPerWarp + sub;
      uint64_t kf[8];
      Unpack16<T>::run(kd + row * kRowBytes + cvec * kVec * (int)sizeof(T), kf);
#pragma unroll
      for (int n = 0; n < NQ; ++n) {
        uint64_t d2 = ptx::fma2(qf[n][0], kf[0], 0ull);
        uint64_t e2 = ptx::fma2(qf[n][1], kf[1], 0ull);
#pragma unroll
        for (int i = 2; i < 8; i += 2) {
          d2 = ptx::fma2(qf[n][i], kf[i], d2);
          e2 = ptx::fma2(qf[n][i + 1], kf[i + 1], e2);
        }
        float d0, d1, e0, e1;
        ptx::f2unpack(d2, d0, d1);
        ptx::f2unpack(e2, e0, e1);
        float part = (d0 + d1) + (e0 + e1);
#pragma unroll
        for (int off = kLanesPerRow / 2; off > 0; off >>= 1) part += __shfl_xor_sync(0xffffffffu, part, off);
        sc[n][it] = part;
      }
    }
    // Online softmax with the warp's running max; each lane exponentiates its own keys.
#pragma unroll
    for (int n = 0; n < NQ; ++n) {
      const int64_t limit = offset + (n0 + n) % p.q_len;
      float mx = -INFINITY;
#pragma unroll
      for (int it = 0; it < kIters; ++it) {
        const bool vis = key[it] < k_end && (!p.is_causal || (int64_t)key[it] <= limit);
        sc[n][it] = vis ? sc[n][it] : -INFINITY;
        mx = fmaxf(mx, sc[n][it]);
      }
#pragma unroll
      for (int off = kLanesPerRow; off < 32; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      if (mx > m[n]) {  // warp-uniform: m and mx are the same on every lane
        const float corr = ptx::ex2(m[n] - mx);
        l[n] *= corr;
        const uint64_t c2 = ptx::f2pack(corr, corr);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[n][i] = ptx::fma2(acc[n][i], c2, 0ull);
        m[n] = mx;
      }
      const float safe = m[n] == -INFINITY ? 0.f : m[n];
#pragma unroll
      for (int it = 0; it < kIters; ++it) {
        sc[n][it] = ptx::ex2(sc[n][it] - safe);
        l[n] += sc[n][it];
      }
    }
    // P.V.  Rows past the valid range have p = 0, but their stale bytes may
    // not be finite, so they are skipped rather than multiplied by zero.
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      const int row = warp * kRowsPerWarpChunk + it * kRowsPerWarp + sub;
      if (key[it] < k_end) {
        uint64_t vf[8];
        Unpack16<T>::run(vd + row * kRowBytes + cvec * kVec * (int)sizeof(T), vf);
#pragma unroll
        for (int n = 0; n < NQ; ++n) {
          const uint64_t w2 = ptx::f2pack(sc[n][it], sc[n][it]);
#pragma unroll
          for (int i = 0; i < 8; ++i) acc[n][i] = ptx::fma2(w2, vf[i], acc[n][i]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&empty[s]);
  }
  // Merge the row slots of the warp: lanes holding the same channels, and the
  // per-lane partial sums of p.
  float accf[NQ][kVec];
#pragma unroll
  for (int n = 0; n < NQ; ++n) {
#pragma unroll
    for (int i = 0; i < 8; ++i) ptx::f2unpack(acc[n][i], accf[n][2 * i], accf[n][2 * i + 1]);
#pragma unroll
    for (int off = kLanesPerRow; off < 32; off <<= 1) {
      l[n] += __shfl_xor_sync(0xffffffffu, l[n], off);
#pragma unroll
      for (int e = 0; e < kVec; ++e) accf[n][e] += __shfl_xor_sync(0xffffffffu, accf[n][e], off);
    }
  }
  // Merge the 4 compute warps through shared memory (the stages are free now).
  asm volatile("bar.sync 1, %0;" ::"r"(kComputeWarps * 32));
  float* red = reinterpret_cast<float*>(smem);
  constexpr int kStride = D + 2;
  if (lane < kLanesPerRow) {
#pragma unroll
    for (int n = 0; n < NQ; ++n)
#pragma unroll
      for (int e = 0; e < kVec; ++e) red[(warp * NQ + n) * kStride + cvec * kVec + e] = accf[n][e];
  }
  if (lane == 0) {
#pragma unroll
    for (int n = 0; n < NQ; ++n) {
      red[(warp * NQ + n) * kStride + D] = m[n];
      red[(warp * NQ + n) * kStride + D + 1] = l[n];
    }
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kComputeWarps * 32));
  if (!ok) return;
  for (int idx = threadIdx.x; idx < nq_used * D; idx += kComputeWarps * 32) {
    const int n = idx / D, d = idx - n * D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kComputeWarps; ++w) mm = fmaxf(mm, red[(w * NQ + n) * kStride + D]);
    const float safe = mm == -INFINITY ? 0.f : mm;
    float ll = 0.f, aa = 0.f;
#pragma unroll
    for (int w = 0; w < kComputeWarps; ++w) {
      const float f = ptx::ex2(red[(w * NQ + n) * kStride + D] - safe);
      ll += red[(w * NQ + n) * kStride + D + 1] * f;
      aa += red[(w * NQ + n) * kStride + d] * f;
    }
    const int r = (n0 + n) / p.q_len, t = (n0 + n) - r * p.q_len, h = hk * rep + r;
    const int64_t row = ((int64_t)b * p.q_heads + h) * p.q_len + t;
    if (n_splits == 1) {
      T* op = reinterpret_cast<T*>(p.o.data) + (int64_t)b * p.o.stride[0] + (int64_t)h * p.o.stride[1] +
              (int64_t)t * p.o.stride[2] + (int64_t)d * p.o.stride[3];
      *op = Elem<T>::from_acc(ll > 0.f ? aa / ll : 0.f);
      if (d == 0 && p.lse)
        reinterpret_cast<float*>(p.lse)[(int64_t)b * p.lse_stride[0] + (int64_t)h * p.lse_stride[1] +
                                        (int64_t)t * p.lse_stride[2]] = ll > 0.f ? (mm + __log2f(ll)) * kLn2 : -INFINITY;
    } else {
      L.ws_acc[(row * L.max_splits + split) * D + d] = aa;
      if (d == 0) {
        L.ws_ml[(row * L.max_splits + split) * 2 + 0] = mm;
        L.ws_ml[(row * L.max_splits + split) * 2 + 1] = ll;
      }
    }
  }
}

// Two query rows per CTA measured best on B200 (bf16, D=128, 8 KV heads x
// 32768 keys, 4 query heads per KV head: 1 row 2.35, 2 rows 2.65, 4 rows
// 2.36 TB/s): more rows per CTA cost registers and occupancy, fewer rows
// re-read K/V from L2 too often.
constexpr int kGroupRows = 2;

template <typename T, int D, int NQ>
static cudaError_t launch_group(const GroupLaunch& L, cudaStream_t st) {
  const size_t stage = 2ull * kStages * kChunk * D * sizeof(T);
  const size_t red = (size_t)kComputeWarps * NQ * (D + 2) * sizeof(float);
  const size_t smem = (stage > red ? stage : red) + 2 * kStages * sizeof(uint64_t);
  auto kern = decode_group_kernel<T, D, NQ>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<dim3(L.max_splits * L.n_groups, L.p.kv_heads, L.p.batch), kThreads, smem, st>>>(L);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t group_nq_dispatch(const GroupLaunch& L, cudaStream_t st) {
  return launch_group<T, D, kGroupRows>(L, st);
}

cudaError_t decode_group_forward(const ts_attn_params& p, int split_keys, int max_splits, float* ws_acc,
                                 float* ws_ml, uint32_t* fault, cudaStream_t st) {
  GroupLaunch L;
  L.p = p;
  L.split_keys = split_keys;
  L.max_splits = max_splits;
  const int nq = (p.q_heads / p.kv_heads) * p.q_len;
  L.n_groups = ceil_div(nq, kGroupRows);
  L.ws_acc = ws_acc;
  L.ws_ml = ws_ml;
  L.fault = fault;
  switch (p.dtype) {
    case TS_F16:
      if (p.head_dim == 64) return group_nq_dispatch<__half, 64>(L, st);
      if (p.head_dim == 128) return group_nq_dispatch<__half, 128>(L, st);
      if (p.head_dim == 256) return group_nq_dispatch<__half, 256>(L, st);
      break;
    case TS_BF16:
      if (p.head_dim == 64) return group_nq_dispatch<__nv_bfloat16, 64>(L, st);
      if (p.head_dim == 128) return group_nq_dispatch<__nv_bfloat16, 128>(L, st);
      if (p.head_dim == 256) return group_nq_dispatch<__nv_bfloat16, 256>(L, st);
      break;
    case TS_F32:
      if (p.head_dim == 64) return group_nq_dispatch<float, 64>(L, st);
      if (p.head_dim == 128) return group_nq_dispatch<float, 128>(L, st);
      break;
  }
  return cudaErrorInvalidValue;
}

}  // namespace tsa
