// Split-K KV-cache decode attention (HBM-bound).
//
// A few query tokens per row (decode: one) attend to a long cached prefix.
// The keys of each (batch row, KV head) are cut into splits of `split_keys`;
// one CTA streams one split through shared memory and a combine kernel merges
// the per-split partial softmax states.  Replaces, for cached decoding, the
// dense call of nn/attention.py:132-145 made by nn/transformer.py:144-154; the
// key-valid rule per row follows the padded-cache mask of
// docs/transformers.md:52-55.
//
// CTA = 4 compute warps + 1 producer warp.  The producer lane streams K and V
// chunks of 32 rows with untiled bulk copies (cp.async.bulk, one copy per
// chunk when rows are contiguous, else one per row) into a 4-stage ring
// guarded by full/empty mbarriers.  Each compute warp takes 8 rows of every
// chunk: a 16-byte vector of a row per lane (8 lanes/row at 128 B rows, 16 at
// 256 B, 32 at 512 B), dot products by lane butterflies, exp2-domain online
// softmax per warp, and P.V accumulated on the lanes that hold the row's
// channels.  All query heads of a KV group (GQA) and all query tokens share
// one pass over the keys, so K/V bytes are read once per KV head.
#include "decode.cuh"
#include "ptx.cuh"

namespace tsa {

constexpr int kDecChunk = 32;
constexpr int kDecStages = 4;
constexpr int kDecComputeWarps = 4;
constexpr int kDecThreads = (kDecComputeWarps + 1) * 32;
constexpr float kLog2e = 1.4426950408889634f;
constexpr float kLn2 = 0.6931471805599453f;

template <typename T> struct Vec16;
template <> struct Vec16<__half> {
  static __device__ __forceinline__ void unpack(const uint4& v, float* f) {
    const __half2* h = reinterpret_cast<const __half2*>(&v);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 x = __half22float2(h[e]);
      f[2 * e] = x.x;
      f[2 * e + 1] = x.y;
    }
  }
};
template <> struct Vec16<__nv_bfloat16> {
  static __device__ __forceinline__ void unpack(const uint4& v, float* f) {
    const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&v);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
      float2 x = __bfloat1622float2(h[e]);
      f[2 * e] = x.x;
      f[2 * e + 1] = x.y;
    }
  }
};
template <> struct Vec16<float> {
  static __device__ __forceinline__ void unpack(const uint4& v, float* f) {
    f[0] = __uint_as_float(v.x);
    f[1] = __uint_as_float(v.y);
    f[2] = __uint_as_float(v.z);
    f[3] = __uint_as_float(v.w);
  }
};

struct DecodeLaunch {
  ts_attn_params p;
  int split_keys;   // keys per split (multiple of kDecChunk)
  int max_splits;   // splits of the longest row
  float* ws_acc;    // [rows][max_splits][Dv] unnormalised partial outputs
  float* ws_ml;     // [rows][max_splits][2]  (running max in log2 units, sum)
  uint32_t* fault;
};

// Keys row b can see: [0, end_b); offset_b positions the first query token.
__device__ __forceinline__ void decode_row_range(const ts_attn_params& p, int b, int& end,
                                                 int64_t& offset) {
  end = p.kv_len;
  offset = p.causal_offset;
  if (p.kv_lens) {
    end = min(end, max(0, p.kv_lens[b]));
    offset = (int64_t)end - p.q_len;
  }
  if (p.is_causal) end = (int)i64max(0, i64min(end, offset + p.q_len));
}

template <typename T, int D, int NQ>
__global__ void __launch_bounds__(kDecThreads) decode_split_kernel(DecodeLaunch L) {
  const ts_attn_params& p = L.p;
  constexpr int kVec = 16 / (int)sizeof(T);
  constexpr int kLanesPerRow = D / kVec;
  constexpr int kRowsPerWarp = 32 / kLanesPerRow;
  constexpr int kRowsPerWarpChunk = kDecChunk / kDecComputeWarps;  // 8
  constexpr int kIters = kRowsPerWarpChunk / kRowsPerWarp;
  constexpr int kRowBytes = D * (int)sizeof(T);
  constexpr int kStageBytes = kDecChunk * kRowBytes;

  extern __shared__ __align__(128) unsigned char smem[];
  unsigned char* kbuf = smem;
  unsigned char* vbuf = smem + kDecStages * kStageBytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + 2 * kDecStages * kStageBytes);
  uint64_t* empty = full + kDecStages;

  const int split = blockIdx.x, hk = blockIdx.y, b = blockIdx.z;
  const int rep = p.q_heads / p.kv_heads;
  const int nq_used = rep * p.q_len;
  int end;
  int64_t offset;
  decode_row_range(p, b, end, offset);
  const int n_splits = max(1, ceil_div(end, L.split_keys));
  if (split >= n_splits) return;
  const int k_begin = split * L.split_keys;
  const int k_end = min(end, k_begin + L.split_keys);
  const int n_chunks = k_end > k_begin ? ceil_div(k_end - k_begin, kDecChunk) : 0;

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    for (int s = 0; s < kDecStages; ++s) {
      ptx::mbar_init(&full[s], 1);
      ptx::mbar_init(&empty[s], kDecComputeWarps);
    }
    ptx::fence_mbar_init();
  }
  __syncthreads();

  const T* kbase = reinterpret_cast<const T*>(p.k.data) + (int64_t)b * p.k.stride[0] +
                   (int64_t)hk * p.k.stride[1];
  const T* vbase = reinterpret_cast<const T*>(p.v.data) + (int64_t)b * p.v.stride[0] +
                   (int64_t)hk * p.v.stride[1];

  if (warp == kDecComputeWarps) {
    // ------------------------------ producer ------------------------------
    if (lane == 0) {
      const bool k_contig = p.k.stride[2] == D, v_contig = p.v.stride[2] == D;
      for (int c = 0; c < n_chunks; ++c) {
        const int s = c % kDecStages;
        if (c >= kDecStages &&
            !ptx::mbar_wait(&empty[s], ((c / kDecStages) - 1) & 1, L.fault, FAULT_DEC_EMPTY))
          break;
        const int r0 = k_begin + c * kDecChunk;
        const int rows = min(kDecChunk, k_end - r0);
        ptx::mbar_expect_tx(&full[s], 2u * rows * kRowBytes);
        unsigned char* kd = kbuf + s * kStageBytes;
        unsigned char* vd = vbuf + s * kStageBytes;
        if (k_contig) {
          ptx::bulk_g2s(kd, kbase + (int64_t)r0 * D, rows * kRowBytes, &full[s]);
        } else {
          for (int r = 0; r < rows; ++r)
            ptx::bulk_g2s(kd + r * kRowBytes, kbase + (int64_t)(r0 + r) * p.k.stride[2], kRowBytes,
                          &full[s]);
        }
        if (v_contig) {
          ptx::bulk_g2s(vd, vbase + (int64_t)r0 * D, rows * kRowBytes, &full[s]);
        } else {
          for (int r = 0; r < rows; ++r)
            ptx::bulk_g2s(vd + r * kRowBytes, vbase + (int64_t)(r0 + r) * p.v.stride[2], kRowBytes,
                          &full[s]);
        }
      }
      // Drain: every issued copy must land before the CTA exits.
      const int first = max(0, n_chunks - kDecStages);
      for (int c = first; c < n_chunks; ++c)
        if (!ptx::mbar_wait(&full[c % kDecStages], (c / kDecStages) & 1, L.fault, FAULT_DEC_FULL)) break;
    }
    return;
  }

  // ------------------------------- compute --------------------------------
  const int sub = lane / kLanesPerRow;        // row slot of this lane within a warp step
  const int cvec = lane % kLanesPerRow;       // 16-byte vector index within the row
  const float qscale = (float)p.scale * kLog2e;
  float q[NQ][kVec];
#pragma unroll
  for (int n = 0; n < NQ; ++n) {
    const int r = n / p.q_len, t = n - r * p.q_len;
    const bool live = n < nq_used;
    const int h = hk * rep + (live ? r : 0);
    const T* qp = reinterpret_cast<const T*>(p.q.data) + (int64_t)b * p.q.stride[0] +
                  (int64_t)h * p.q.stride[1] + (int64_t)(live ? t : 0) * p.q.stride[2];
#pragma unroll
    for (int e = 0; e < kVec; ++e)
      q[n][e] = live ? Elem<T>::to_acc(qp[(int64_t)(cvec * kVec + e) * p.q.stride[3]]) * qscale : 0.f;
  }
  float m[NQ], l[NQ], acc[NQ][kVec];
#pragma unroll
  for (int n = 0; n < NQ; ++n) {
    m[n] = -INFINITY;
    l[n] = 0.f;
#pragma unroll
    for (int e = 0; e < kVec; ++e) acc[n][e] = 0.f;
  }

  bool ok = true;
  for (int c = 0; c < n_chunks && ok; ++c) {
    const int s = c % kDecStages;
    if (!ptx::mbar_wait(&full[s], (c / kDecStages) & 1, L.fault, FAULT_DEC_FULL)) {
      ok = false;
      break;
    }
    const int r0 = k_begin + c * kDecChunk;
    const unsigned char* kd = kbuf + s * kStageBytes;
    const unsigned char* vd = vbuf + s * kStageBytes;
    float sc[NQ][kRowsPerWarpChunk];
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      const int row = warp * kRowsPerWarpChunk + it * kRowsPerWarp + sub;
      float kf[kVec];
      const uint4 kv = *reinterpret_cast<const uint4*>(kd + row * kRowBytes + cvec * 16);
      Vec16<T>::unpack(kv, kf);
#pragma unroll
      for (int n = 0; n < NQ; ++n) {
        float part = 0.f;
#pragma unroll
        for (int e = 0; e < kVec; ++e) part = fmaf(q[n][e], kf[e], part);
#pragma unroll
        for (int off = kLanesPerRow / 2; off > 0; off >>= 1)
          part += __shfl_xor_sync(0xffffffffu, part, off);
        // Gather the scores of every row slot of this step into all lanes.
#pragma unroll
        for (int rs = 0; rs < kRowsPerWarp; ++rs)
          sc[n][it * kRowsPerWarp + rs] = __shfl_sync(0xffffffffu, part, rs * kLanesPerRow);
      }
    }
    // Masks: key range of the split, and the causal rule per query token.
#pragma unroll
    for (int n = 0; n < NQ; ++n) {
      const int t = n % p.q_len;
      float mx = -INFINITY;
#pragma unroll
      for (int rr = 0; rr < kRowsPerWarpChunk; ++rr) {
        const int key = r0 + warp * kRowsPerWarpChunk + rr;
        const bool vis = key < k_end && (!p.is_causal || (int64_t)key <= offset + t);
        sc[n][rr] = vis ? sc[n][rr] : -INFINITY;
        mx = fmaxf(mx, sc[n][rr]);
      }
      const float m_new = fmaxf(m[n], mx);
      const float safe = m_new == -INFINITY ? 0.f : m_new;
      const float corr = ptx::ex2(m[n] - safe);
      l[n] *= corr;
#pragma unroll
      for (int e = 0; e < kVec; ++e) acc[n][e] *= corr;
      m[n] = m_new;
#pragma unroll
      for (int rr = 0; rr < kRowsPerWarpChunk; ++rr) {
        sc[n][rr] = ptx::ex2(sc[n][rr] - safe);
        l[n] += sc[n][rr];
      }
    }
#pragma unroll
    for (int it = 0; it < kIters; ++it) {
      const int rr = it * kRowsPerWarp + sub;
      const int row = warp * kRowsPerWarpChunk + rr;
      float vf[kVec];
      const uint4 vv = *reinterpret_cast<const uint4*>(vd + row * kRowBytes + cvec * 16);
      Vec16<T>::unpack(vv, vf);
      // Rows past the valid range hold stale bytes; their probability is 0,
      // but 0 * NaN would poison the sum, so skip them explicitly.
      const bool row_valid = r0 + row < k_end;
#pragma unroll
      for (int n = 0; n < NQ; ++n) {
        float pr = 0.f;
#pragma unroll
        for (int rs = 0; rs < kRowsPerWarp; ++rs)
          if (rs == sub) pr = sc[n][it * kRowsPerWarp + rs];
        if (row_valid) {
#pragma unroll
          for (int e = 0; e < kVec; ++e) acc[n][e] = fmaf(pr, vf[e], acc[n][e]);
        }
      }
    }
    __syncwarp();
    if (lane == 0) ptx::mbar_arrive(&empty[s]);
  }

  // Merge the row slots of the warp (lanes holding the same channels).
#pragma unroll
  for (int n = 0; n < NQ; ++n)
#pragma unroll
    for (int e = 0; e < kVec; ++e)
#pragma unroll
      for (int off = kLanesPerRow; off < 32; off <<= 1)
        acc[n][e] += __shfl_xor_sync(0xffffffffu, acc[n][e], off);

  // Merge the 4 compute warps through shared memory (stages are free now).
  asm volatile("bar.sync 1, %0;" ::"r"(kDecComputeWarps * 32));
  float* red = reinterpret_cast<float*>(smem);  // [warps][NQ][D + 2]
  constexpr int kStride = D + 2;
  if (lane < kLanesPerRow) {
#pragma unroll
    for (int n = 0; n < NQ; ++n)
#pragma unroll
      for (int e = 0; e < kVec; ++e) red[(warp * NQ + n) * kStride + cvec * kVec + e] = acc[n][e];
  }
  if (lane == 0) {
#pragma unroll
    for (int n = 0; n < NQ; ++n) {
      red[(warp * NQ + n) * kStride + D] = m[n];
      red[(warp * NQ + n) * kStride + D + 1] = l[n];
    }
  }
  asm volatile("bar.sync 1, %0;" ::"r"(kDecComputeWarps * 32));
  if (!ok) return;
  const int rows_total = p.batch * p.q_heads * p.q_len;
  (void)rows_total;
  for (int idx = threadIdx.x; idx < nq_used * D; idx += kDecComputeWarps * 32) {
    const int n = idx / D, d = idx - n * D;
    float mm = -INFINITY;
#pragma unroll
    for (int w = 0; w < kDecComputeWarps; ++w) mm = fmaxf(mm, red[(w * NQ + n) * kStride + D]);
    const float safe = mm == -INFINITY ? 0.f : mm;
    float ll = 0.f, aa = 0.f;
#pragma unroll
    for (int w = 0; w < kDecComputeWarps; ++w) {
      const float f = ptx::ex2(red[(w * NQ + n) * kStride + D] - safe);
      ll += red[(w * NQ + n) * kStride + D + 1] * f;
      aa += red[(w * NQ + n) * kStride + d] * f;
    }
    const int r = n / p.q_len, t = n - r * p.q_len, h = hk * rep + r;
    const int64_t row = ((int64_t)b * p.q_heads + h) * p.q_len + t;
    if (n_splits == 1) {
      T* op = reinterpret_cast<T*>(p.o.data) + (int64_t)b * p.o.stride[0] + (int64_t)h * p.o.stride[1] +
              (int64_t)t * p.o.stride[2] + (int64_t)d * p.o.stride[3];
      *op = Elem<T>::from_acc(ll > 0.f ? aa / ll : 0.f);
      if (d == 0 && p.lse)
        reinterpret_cast<float*>(p.lse)[(int64_t)b * p.lse_stride[0] + (int64_t)h * p.lse_stride[1] + (int64_t)t * p.lse_stride[2]] =
            ll > 0.f ? (mm + __log2f(ll)) * kLn2 : -INFINITY;
    } else {
      L.ws_acc[(row * L.max_splits + split) * D + d] = aa;
      if (d == 0) {
        L.ws_ml[(row * L.max_splits + split) * 2 + 0] = mm;
        L.ws_ml[(row * L.max_splits + split) * 2 + 1] = ll;
      }
    }
  }
}

// One warp per output row: merge the row's split partials.
template <typename T, int D>
__global__ void decode_combine_kernel(DecodeLaunch L) {
  const ts_attn_params& p = L.p;
  const int warp = (blockIdx.x * blockDim.x + threadIdx.x) >> 5, lane = threadIdx.x & 31;
  const int rows = p.batch * p.q_heads * p.q_len;
  if (warp >= rows) return;
  const int t = warp % p.q_len, h = (warp / p.q_len) % p.q_heads, b = warp / (p.q_len * p.q_heads);
  int end;
  int64_t offset;
  decode_row_range(p, b, end, offset);
  const int n_splits = max(1, ceil_div(end, L.split_keys));
  if (n_splits == 1) return;
  const int64_t row = warp;
  float mm = -INFINITY;
  for (int s = 0; s < n_splits; ++s) mm = fmaxf(mm, L.ws_ml[(row * L.max_splits + s) * 2]);
  const float safe = mm == -INFINITY ? 0.f : mm;
  float ll = 0.f;
  for (int s = 0; s < n_splits; ++s)
    ll += L.ws_ml[(row * L.max_splits + s) * 2 + 1] * ptx::ex2(L.ws_ml[(row * L.max_splits + s) * 2] - safe);
  const float inv = ll > 0.f ? 1.f / ll : 0.f;
  for (int d = lane; d < D; d += 32) {
    float aa = 0.f;
    for (int s = 0; s < n_splits; ++s)
      aa += L.ws_acc[(row * L.max_splits + s) * D + d] *
            ptx::ex2(L.ws_ml[(row * L.max_splits + s) * 2] - safe);
    T* op = reinterpret_cast<T*>(p.o.data) + (int64_t)b * p.o.stride[0] + (int64_t)h * p.o.stride[1] +
            (int64_t)t * p.o.stride[2] + (int64_t)d * p.o.stride[3];
    *op = Elem<T>::from_acc(aa * inv);
  }
  if (lane == 0 && p.lse)
    reinterpret_cast<float*>(p.lse)[(int64_t)b * p.lse_stride[0] + (int64_t)h * p.lse_stride[1] + (int64_t)t * p.lse_stride[2]] =
        ll > 0.f ? (mm + __log2f(ll)) * kLn2 : -INFINITY;
}

// ---------------------------------------------------------------------------
// Host side
// ---------------------------------------------------------------------------
static int pick_nq(int nq) {
  if (nq <= 1) return 1;
  if (nq <= 2) return 2;
  if (nq <= 4) return 4;
  if (nq <= 8) return 8;
  return 0;
}

bool decode_supported(const ts_attn_params& p) {
  if (p.dtype != TS_F16 && p.dtype != TS_BF16 && p.dtype != TS_F32) return false;
  if (p.head_dim != p.value_dim || p.mask_kind != TS_MASK_NONE) return false;
  const int esz = p.dtype == TS_F32 ? 4 : 2;
  const int D = p.head_dim;
  const bool dim_ok = esz == 2 ? (D == 64 || D == 128 || D == 256) : (D == 64 || D == 128);
  if (!dim_ok) return false;
  if (pick_nq((p.q_heads / p.kv_heads) * p.q_len) == 0) return false;
  // 16-byte vector rows: channel stride 1, row stride and bases 16-byte aligned.
  const ts_view4* views[2] = {&p.k, &p.v};
  for (const ts_view4* v : views) {
    if (v->stride[3] != 1) return false;
    if ((v->stride[2] * esz) % 16 || (v->stride[1] * esz) % 16 || (v->stride[0] * esz) % 16) return false;
    if (reinterpret_cast<uintptr_t>(v->data) % 16) return false;
  }
  return true;
}

static int decode_split_keys(const ts_attn_params& p, int sm_count) {
  // Aim for about 4 waves of 3 CTAs per SM over the longest-row estimate, with
  // at least 512 keys (16 chunks) per split: short splits spend their time
  // filling the 4-stage ring, too few waves leave ragged rows unbalanced.
  const int64_t keys = (int64_t)p.batch * p.kv_heads * p.kv_len;
  const int64_t target_ctas = (int64_t)sm_count * 3 * 4;
  int64_t s = (keys + target_ctas - 1) / target_ctas;
  s = ((s + kDecChunk - 1) / kDecChunk) * kDecChunk;
  s = s < 512 ? 512 : (s > 8192 ? 8192 : s);
  return (int)s;
}

static int device_sms() {
  int dev = 0, sms = 148;
  if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms;
}

size_t decode_workspace(const ts_attn_params& p) {
  const int sk = decode_split_keys(p, device_sms());
  const int max_splits = ceil_div(p.kv_len, sk);
  if (max_splits <= 1) return 0;
  const size_t rows = (size_t)p.batch * p.q_heads * p.q_len;
  return rows * max_splits * (p.value_dim + 2) * sizeof(float);
}

template <typename T, int D, int NQ>
static cudaError_t launch_decode(const DecodeLaunch& L, cudaStream_t st) {
  constexpr int kRowBytes = D * (int)sizeof(T);
  const size_t stage_bytes = 2ull * kDecStages * kDecChunk * kRowBytes;
  const size_t red_bytes = (size_t)kDecComputeWarps * NQ * (D + 2) * sizeof(float);
  const size_t smem = (stage_bytes > red_bytes ? stage_bytes : red_bytes) + 2 * kDecStages * sizeof(uint64_t);
  auto kern = decode_split_kernel<T, D, NQ>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return e;
  dim3 grid(L.max_splits, L.p.kv_heads, L.p.batch);
  kern<<<grid, kDecThreads, smem, st>>>(L);
  e = cudaGetLastError();
  if (e != cudaSuccess || L.max_splits <= 1) return e;
  const int rows = L.p.batch * L.p.q_heads * L.p.q_len;
  decode_combine_kernel<T, D><<<ceil_div(rows * 32, 256), 256, 0, st>>>(L);
  return cudaGetLastError();
}

template <typename T, int D>
static cudaError_t decode_nq(const DecodeLaunch& L, cudaStream_t st) {
  switch (pick_nq((L.p.q_heads / L.p.kv_heads) * L.p.q_len)) {
    case 1: return launch_decode<T, D, 1>(L, st);
    case 2: return launch_decode<T, D, 2>(L, st);
    case 4: return launch_decode<T, D, 4>(L, st);
    case 8: return launch_decode<T, D, 8>(L, st);
  }
  return cudaErrorInvalidValue;
}

template <typename T, int D>
static cudaError_t combine_only(const DecodeLaunch& L, cudaStream_t st) {
  const int rows = L.p.batch * L.p.q_heads * L.p.q_len;
  decode_combine_kernel<T, D><<<ceil_div(rows * 32, 256), 256, 0, st>>>(L);
  return cudaGetLastError();
}

static cudaError_t decode_combine(const DecodeLaunch& L, cudaStream_t st) {
  const int D = L.p.head_dim;
  switch (L.p.dtype) {
    case TS_F16:
      if (D == 64) return combine_only<__half, 64>(L, st);
      if (D == 128) return combine_only<__half, 128>(L, st);
      if (D == 256) return combine_only<__half, 256>(L, st);
      break;
    case TS_BF16:
      if (D == 64) return combine_only<__nv_bfloat16, 64>(L, st);
      if (D == 128) return combine_only<__nv_bfloat16, 128>(L, st);
      if (D == 256) return combine_only<__nv_bfloat16, 256>(L, st);
      break;
    case TS_F32:
      if (D == 64) return combine_only<float, 64>(L, st);
      if (D == 128) return combine_only<float, 128>(L, st);
      break;
  }
  return cudaErrorInvalidValue;
}

cudaError_t decode_forward(const ts_attn_params& p, void* ws, size_t ws_bytes, uint32_t* fault,
                           cudaStream_t st) {
  DecodeLaunch L;
  L.p = p;
  L.split_keys = decode_split_keys(p, device_sms());
  L.max_splits = ceil_div(p.kv_len, L.split_keys);
  if (L.max_splits < 1) L.max_splits = 1;
  const size_t rows = (size_t)p.batch * p.q_heads * p.q_len;
  L.ws_acc = reinterpret_cast<float*>(ws);
  L.ws_ml = L.ws_acc ? L.ws_acc + rows * L.max_splits * p.value_dim : nullptr;
  L.fault = fault;
  if (L.max_splits > 1 && ws_bytes < decode_workspace(p)) return cudaErrorInvalidValue;
  // Several query rows per KV head (GQA groups, multi-token steps): the grouped kernel.
  if ((p.q_heads / p.kv_heads) * p.q_len >= 2) {
    const cudaError_t e = decode_group_forward(p, L.split_keys, L.max_splits, L.ws_acc, L.ws_ml, fault, st);
    if (e != cudaSuccess || L.max_splits <= 1) return e;
    return decode_combine(L, st);
  }
  const int D = p.head_dim;
  switch (p.dtype) {
    case TS_F16:
      if (D == 64) return decode_nq<__half, 64>(L, st);
      if (D == 128) return decode_nq<__half, 128>(L, st);
      if (D == 256) return decode_nq<__half, 256>(L, st);
      break;
    case TS_BF16:
      if (D == 64) return decode_nq<__nv_bfloat16, 64>(L, st);
      if (D == 128) return decode_nq<__nv_bfloat16, 128>(L, st);
      if (D == 256) return decode_nq<__nv_bfloat16, 256>(L, st);
      break;
    case TS_F32:
      if (D == 64) return decode_nq<float, 64>(L, st);
      if (D == 128) return decode_nq<float, 128>(L, st);
      break;
  }
  return cudaErrorInvalidValue;
}

}  // namespace tsa
