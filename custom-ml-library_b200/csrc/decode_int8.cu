// Split-K decode over an int8 KV cache with fused dequantisation.
//
// tensorsmith's quantized KVCache stores symmetric int8 rows with one fp32
// scale per token and head (nn/cache.py:47-52, 70-82) and dequantises the
// whole active prefix before attention (:91-98).  Here the decode reads the
// int8 rows directly: K and V bytes stream through shared memory in 32-row
// chunks (cp.async.bulk, 4-stage ring, as the half-precision decode), each
// byte becomes a float with one byte permute and one add (no conversion
// unit), and the per-row scales fold into the score (s = k_scale * q.k8) and
// into the probability used for P.V (p * v_scale).  Half the bytes of an fp16
// cache per step.
#include <type_traits>

#include "int8.cuh"
#include "ptx.cuh"

namespace tsa {

namespace {
constexpr int kChunk = 32;
constexpr int kStages = 4;
constexpr int kComputeWarps = 4;
constexpr int kThreads = (kComputeWarps + 1) * 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;
constexpr float kMagic = 8388608.f + 128.f;  // 2^23 + the byte bias

// 16 signed bytes -> 8 packed float pairs: bias each byte to unsigned, splice
// it under the exponent of 2^23 (one byte permute per element) and subtract
// 2^23 + 128 with packed adds.
__device__ __forceinline__ void unpack_i8x16(const uint4& v, uint64_t (&f)[8]) {
  const uint32_t w[4] = {v.x ^ 0x80808080u, v.y ^ 0x80808080u, v.z ^ 0x80808080u, v.w ^ 0x80808080u};
  const uint64_t bias = ptx::f2pack(-kMagic, -kMagic);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const float a = __uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7540));
    const float b = __uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7541));
    const float c = __uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7542));
    const float d = __uint_as_float(__byte_perm(w[i], 0x4B000000u, 0x7543));
    f[2 * i] = ptx::add2(ptx::f2pack(a, b), bias);
    f[2 * i + 1] = ptx::add2(ptx::f2pack(c, d), bias);
  }
}

__device__ __forceinline__ int dp2a_lo(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.lo.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
__device__ __forceinline__ int dp2a_hi(uint32_t a, uint32_t b, int c) {
  int d;
  asm("dp2a.hi.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
  return d;
}
}  // namespace

struct Int8Launch {
  ts_attn_params p;        // k / v views address int8 storage
  const float* k_scale;    // [B, Hkv, capacity] contiguous
  const float* v_scale;
  int64_t scale_row_stride;  // capacity (elements between consecutive heads)
  int split_keys, max_splits;
  int n_groups;            // query-row groups of NQ rows per KV head (grid.x = splits * groups)
  float* ws_acc;
  float* ws_ml;
  uint32_t* fault;
};

__device__ __forceinline__ void int8_row_range(const ts_attn_params& p, int b, int& end, int64_t& offset) {
  end = p.kv_len;
  offset = p.causal_offset;
  if (p.kv_lens) {
    end = min(end, max(0, p.kv_lens[b]));
    offset = (int64_t)end - p.q_len;
  }
  if (p.is_causal) end = (int)i64max(0, i64min(end, offset + p.q_len));
}

// Lane layout per chunk of 32 keys: warp w owns keys [8w, 8w + 8); a key row
// of D bytes is spread over D/16 lanes (16 bytes each), so one warp step covers
// 32 / (D/16) rows.  Scores: for half-precision queries the query row is held
// as int16 (symmetric, per row, 2^-15 of its max magnitude) and q . k8 is an
// exact int32 sum of dp2a products -- no conversion of K at all; fp32 queries
// keep an fp32 dot product over unpacked K.  Softmax: every lane exponentiates
// only the keys it holds, with the warp's running max; P.V: p * v_scale times
// the unpacked V row, packed f32x2 FMAs.
template <typename T, int D, int NQ>
__global__ void __launch_bounds__(kThreads, 4) decode_int8_kernel(Int8Launch L) {
  constexpr bool kIntQ = !std::is_same<T, float>::value;
  const ts_attn_params& p = L.p;
  constexpr int kVec = 16;                 // int8 elements per 16-byte vector
  constexpr int kLanesPerRow = D / kVec;   // 4, 8, 16
  constexpr int kRowsPerWarp = 32 / kLanesPerRow;
  constexpr int kRowsPerWarpChunk = kChunk / kComputeWarps;  // 8
  constexpr int kIters = kRowsPerWarpChunk / kRowsPerWarp;
  constexpr int kRowBytes = D;
  constexpr int kStageBytes = kChunk * kRowBytes;

  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* kbuf = smem;
  unsigned char* vbuf = smem + kStages * kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * kStages * kStageBytes);
  uint64_t* empty = full + kStages;

  // Groups of one split are adjacent in grid.x so their K/V reads meet in L2.
  const int split = blockIdx.x / L.n_groups, grp = blockIdx.x - split * L.n_groups;
  const int hk = blockIdx.y, b = blockIdx.z;
  const int rep = p.q_heads / p.kv_heads;
  const int n0 = grp * NQ;                          // first query row of this group
  const int nq_used = min(NQ, rep * p.q_len - n0);  // live rows of this group
  int end;
  int64_t offset;
  int8_row_range(p, b, end, offset);
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
  const int8_t* kbase = reinterpret_cast<const int8_t*>(p.k.data) + (int64_t)b * p.k.stride[0] +
                        (int64_t)hk * p.k.stride[1];
  const int8_t* vbase = reinterpret_cast<const int8_t*>(p.v.data) + (int64_t)b * p.v.stride[0] +
                        (int64_t)hk * p.v.stride[1];
  const float* ksc = L.k_scale + ((int64_t)b * p.kv_heads + hk) * L.scale_row_stride;
  const float* vsc = L.v_scale + ((int64_t)b * p.kv_heads + hk) * L.scale_row_stride;

  if (warp == kComputeWarps) {
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
      const int first = max(0, n_chunks - kStages);
      for (int c = first; c < n_chunks; ++c)
        if (!ptx::mbar_wait(&full[c % kStages], (c / kStages) & 1, L.fault, FAULT_DEC_FULL)) break;
    }
    return;
  }

  const int sub = lane / kLanesPerRow;
  const int cvec = lane % kLanesPerRow;
  const float qscale = (float)p.scale * kLog2e;
  // Queries: fp32 pairs, or int16 pairs plus one fp32 step per row.
  uint64_t qf[kIntQ ? 1 : NQ][8];
  uint32_t q16[kIntQ ? NQ : 1][8];
  float qstep[NQ];
#pragma unroll
  for (int n = 0; n < NQ; ++n) {
    const int r = (n0 + n) / p.q_len, t = (n0 + n) - r * p.q_len;
    const bool live = n < nq_used;
    const int h = hk * rep + (live ? r : 0);
    const T* qp = reinterpret_cast<const T*>(p.q.data) + (int64_t)b * p.q.stride[0] + (int64_t)h * p.q.stride[1] +
                  (int64_t)(live ? t : 0) * p.q.stride[2];
    float qv[kVec];
#pragma unroll
    for (int e = 0; e < kVec; ++e)
      qv[e] = live ? Elem<T>::to_acc(qp[(int64_t)(cvec * kVec + e) * p.q.stride[3]]) * qscale : 0.f;
    if constexpr (kIntQ) {
      float amax = 0.f;
#pragma unroll
      for (int e = 0; e < kVec; ++e) amax = fmaxf(amax, fabsf(qv[e]));
#pragma unroll
      for (int off = kLanesPerRow / 2; off > 0; off >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, off));
      const float inv = amax > 0.f ? 32767.f / amax : 0.f;
      qstep[n] = amax * (1.f / 32767.f);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const int lo = max(-32767, min(32767, __float2int_rn(qv[2 * i] * inv)));
        const int hi = max(-32767, min(32767, __float2int_rn(qv[2 * i + 1] * inv)));
        q16[n][i] = ((uint32_t)lo & 0xFFFFu) | ((uint32_t)hi << 16);
      }
    } else {
      qstep[n] = 1.f;
#pragma unroll
      for (int i = 0; i < 8; ++i) qf[n][i] = ptx::f2pack(qv[2 * i], qv[2 * i + 1]);
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
    // Scales of this lane's rows (issued before the wait so their latency overlaps it).
    float ks[kIters], vs[kIters];
    int key[kIters];
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      key[it] = r0 + warp * kRowsPerWarpChunk + it * kRowsPerWarp + sub;
      const bool in = key[it] < k_end;
      ks[it] = in ? __ldg(ksc + key[it]) : 0.f;
      vs[it] = in ? __ldg(vsc + key[it]) : 0.f;
    }
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
      const uint4 kw = *reinterpret_cast<const uint4*>(kd + row * kRowBytes + cvec * 16);
      if constexpr (kIntQ) {
#pragma unroll
        for (int n = 0; n < NQ; ++n) {
          int dot = 0;
          dot = dp2a_lo(q16[n][0], kw.x, dot);
          dot = dp2a_hi(q16[n][1], kw.x, dot);
          dot = dp2a_lo(q16[n][2], kw.y, dot);
          dot = dp2a_hi(q16[n][3], kw.y, dot);
          dot = dp2a_lo(q16[n][4], kw.z, dot);
          dot = dp2a_hi(q16[n][5], kw.z, dot);
          dot = dp2a_lo(q16[n][6], kw.w, dot);
          dot = dp2a_hi(q16[n][7], kw.w, dot);
#pragma unroll
          for (int off = kLanesPerRow / 2; off > 0; off >>= 1) dot += __shfl_xor_sync(0xffffffffu, dot, off);
          sc[n][it] = (float)dot * (qstep[n] * ks[it]);
        }
      } else {
        uint64_t kf[8];
        unpack_i8x16(kw, kf);
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
          sc[n][it] = part * ks[it];
        }
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
    // P.V: rows past the valid range have p = 0 and finite (int8) values.
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      const int row = warp * kRowsPerWarpChunk + it * kRowsPerWarp + sub;
      uint64_t vf[8];
      unpack_i8x16(*reinterpret_cast<const uint4*>(vd + row * kRowBytes + cvec * 16), vf);
#pragma unroll
      for (int n = 0; n < NQ; ++n) {
        const float w = sc[n][it] * vs[it];
        const uint64_t w2 = ptx::f2pack(w, w);
#pragma unroll
        for (int i = 0; i < 8; ++i) acc[n][i] = ptx::fma2(w2, vf[i], acc[n][i]);
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

// One CTA per output row, one thread per channel: merge the row's split partials.
template <typename T>
__global__ void decode_int8_combine(Int8Launch L) {
  const ts_attn_params& p = L.p;
  const int64_t row = blockIdx.x;
  const int t = (int)(row % p.q_len), h = (int)((row / p.q_len) % p.q_heads), b = (int)(row / ((int64_t)p.q_len * p.q_heads));
  int end;
  int64_t offset;
  int8_row_range(p, b, end, offset);
  const int n_splits = max(1, ceil_div(end, L.split_keys));
  if (n_splits == 1) return;
  const int D = p.value_dim;
  float mm = -INFINITY;
  for (int s = 0; s < n_splits; ++s) mm = fmaxf(mm, L.ws_ml[(row * L.max_splits + s) * 2]);
  const float safe = mm == -INFINITY ? 0.f : mm;
  float ll = 0.f;
  for (int s = 0; s < n_splits; ++s)
    ll += L.ws_ml[(row * L.max_splits + s) * 2 + 1] * ptx::ex2(L.ws_ml[(row * L.max_splits + s) * 2] - safe);
  const float inv = ll > 0.f ? 1.f / ll : 0.f;
  for (int d = threadIdx.x; d < D; d += blockDim.x) {
    float aa = 0.f;
    for (int s = 0; s < n_splits; ++s)
      aa += L.ws_acc[(row * L.max_splits + s) * D + d] * ptx::ex2(L.ws_ml[(row * L.max_splits + s) * 2] - safe);
    T* op = reinterpret_cast<T*>(p.o.data) + (int64_t)b * p.o.stride[0] + (int64_t)h * p.o.stride[1] +
            (int64_t)t * p.o.stride[2] + (int64_t)d * p.o.stride[3];
    *op = Elem<T>::from_acc(aa * inv);
  }
  if (threadIdx.x == 0 && p.lse)
    reinterpret_cast<float*>(p.lse)[(int64_t)b * p.lse_stride[0] + (int64_t)h * p.lse_stride[1] +
                                    (int64_t)t * p.lse_stride[2]] = ll > 0.f ? (mm + __log2f(ll)) * kLn2 : -INFINITY;
}

// At most two query rows per CTA: as for the half-precision grouped decode,
// more rows cost registers and occupancy than the shared K/V pass saves.
static int int8_pick_nq(int nq) { return nq <= 1 ? 1 : 2; }

bool decode_int8_supported(const ts_attn_params& p) {
  if (p.dtype != TS_F16 && p.dtype != TS_BF16 && p.dtype != TS_F32) return false;
  if (p.head_dim != p.value_dim || p.mask_kind != TS_MASK_NONE) return false;
  if (p.head_dim != 64 && p.head_dim != 128 && p.head_dim != 256) return false;
  const ts_view4* views[2] = {&p.k, &p.v};
  for (const ts_view4* v : views) {
    if (v->stride[3] != 1 || v->stride[2] % 16 || v->stride[1] % 16 || v->stride[0] % 16) return false;
    if (reinterpret_cast<uintptr_t>(v->data) % 16) return false;
  }
  return true;
}

static int int8_split_keys(const ts_attn_params& p) {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  const int64_t keys = (int64_t)p.batch * p.kv_heads * p.kv_len;
  const int64_t target = (int64_t)sms * 6 * 4;  // about 4 waves, at least 512 keys per split (see decode.cu)
  int64_t s = (keys + target - 1) / target;
  s = ((s + kChunk - 1) / kChunk) * kChunk;
  return (int)(s < 512 ? 512 : (s > 8192 ? 8192 : s));
}

size_t decode_int8_workspace(const ts_attn_params& p) {
  const int sk = int8_split_keys(p);
  const int max_splits = ceil_div(p.kv_len, sk);
  if (max_splits <= 1) return 0;
  return (size_t)p.batch * p.q_heads * p.q_len * max_splits * (p.value_dim + 2) * sizeof(float);
}

template <typename T, int D, int NQ>
static cudaError_t launch_int8(const Int8Launch& L, cudaStream_t st) {
  const size_t stage = 2ull * kStages * kChunk * D;
  const size_t red = (size_t)kComputeWarps * NQ * (D + 2) * sizeof(float);
  const size_t smem = (stage > red ? stage : red) + 2 * kStages * sizeof(uint64_t);
  auto kern = decode_int8_kernel<T, D, NQ>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  kern<<<dim3(L.max_splits * L.n_groups, L.p.kv_heads, L.p.batch), kThreads, smem, st>>>(L);
  e = cudaGetLastError();
  if (e != cudaSuccess || L.max_splits <= 1) return e;
  decode_int8_combine<T><<<L.p.batch * L.p.q_heads * L.p.q_len, 128, 0, st>>>(L);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t int8_nq(const Int8Launch& L, cudaStream_t st) {
  switch (int8_pick_nq((L.p.q_heads / L.p.kv_heads) * L.p.q_len)) {
    case 1: return launch_int8<T, D, 1>(L, st);
    case 2: return launch_int8<T, D, 2>(L, st);
  }
  return cudaErrorInvalidValue;
}

template <typename T>
static cudaError_t int8_dim(const Int8Launch& L, cudaStream_t st) {
  switch (L.p.head_dim) {
    case 64: return int8_nq<T, 64>(L, st);
    case 128: return int8_nq<T, 128>(L, st);
    case 256: return int8_nq<T, 256>(L, st);
  }
  return cudaErrorInvalidValue;
}

cudaError_t decode_int8_forward(const ts_attn_params& p, const float* k_scale, const float* v_scale,
                                int64_t scale_row_stride, void* ws, size_t ws_bytes, uint32_t* fault,
                                cudaStream_t st) {
  Int8Launch L;
  L.p = p;
  L.k_scale = k_scale;
  L.v_scale = v_scale;
  L.scale_row_stride = scale_row_stride;
  L.split_keys = int8_split_keys(p);
  L.max_splits = max(1, ceil_div(p.kv_len, L.split_keys));
  const int nq = (p.q_heads / p.kv_heads) * p.q_len;
  L.n_groups = ceil_div(nq, int8_pick_nq(nq));
  const size_t rows = (size_t)p.batch * p.q_heads * p.q_len;
  L.ws_acc = reinterpret_cast<float*>(ws);
  L.ws_ml = L.ws_acc ? L.ws_acc + rows * L.max_splits * p.value_dim : nullptr;
  L.fault = fault;
  if (L.max_splits > 1 && ws_bytes < decode_int8_workspace(p)) return cudaErrorInvalidValue;
  switch (p.dtype) {
    case TS_F16: return int8_dim<__half>(L, st);
    case TS_BF16: return int8_dim<__nv_bfloat16>(L, st);
    case TS_F32: return int8_dim<float>(L, st);
  }
  return cudaErrorInvalidValue;
}

}  // namespace tsa
