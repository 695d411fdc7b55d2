/*
 * ts_attn.h -- C ABI of the B200 attention engine for tensorsmith.
 *
 * The engine replaces the compute behind tensorsmith's attention path
 * (tensorsmith 0.3.0; file:line below are relative to the tensorsmith project
 * root).  Every entry point takes plain device pointers, element strides and
 * sizes; the caller owns all memory (outputs and workspaces included).  Calls
 * are asynchronous on the given CUDA stream (a cudaStream_t passed as void*,
 * NULL = legacy default stream) of the current device.  Every entry point
 * returns TS_OK (0) or a negative ts_status and never aborts the process.
 *
 * Layout convention: a 4-D view [batch, heads, sequence, channels] is a base
 * pointer plus four ELEMENT strides, so tensors coming from tensorsmith's
 * reshape/permute (nn/transformer.py:124-138, memory order B,T,H,D) are
 * accepted without a copy.
 */
#ifndef TS_ATTN_H
#define TS_ATTN_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#define TS_ATTN_ABI_VERSION 1

#if defined(__GNUC__)
#define TS_ATTN_API __attribute__((visibility("default")))
#else
#define TS_ATTN_API
#endif

/* Element types.  Half types compute in fp32 with fp32 softmax statistics,
 * as the reference does (nn/attention.py:63); fp64 computes in fp64. */
typedef enum ts_dtype { TS_F32 = 0, TS_F16 = 1, TS_BF16 = 2, TS_F64 = 3, TS_I8 = 4 } ts_dtype;
/* TS_I8 is a storage type only: the int8 KV cache of nn/cache.py:47-52
 * (ts_kv_append_int8, ts_kv_dequant_int8, ts_kv_reorder and the K/V views of
 * ts_attn_decode_int8).  No attention entry point computes in it. */

/* Optional attention mask of nn/attention.py:64-76, 105-107:
 * BOOL  -- uint8 0/1, True (1) = allowed, False -> score -inf;
 * ADD   -- values added to the scaled scores: fp32, or fp64 when dtype is TS_F64. */
typedef enum ts_mask_kind { TS_MASK_NONE = 0, TS_MASK_BOOL = 1, TS_MASK_ADD_F32 = 2 } ts_mask_kind;

typedef enum ts_status {
  TS_OK = 0,
  TS_ERR_INVALID_ARGUMENT = -1, /* shape / stride / pointer / value check failed */
  TS_ERR_UNSUPPORTED = -2,      /* combination not implemented by any kernel */
  TS_ERR_WORKSPACE = -3,        /* workspace missing or smaller than required */
  TS_ERR_LAUNCH = -4,           /* kernel launch or driver call failed */
  TS_ERR_DEVICE_TIMEOUT = -5,   /* a bounded wait inside a kernel gave up */
  TS_ERR_CAPACITY = -6          /* KV-cache append would exceed the capacity */
} ts_status;

/* Which kernel family ts_attn_fwd would run (for tests and diagnostics). */
typedef enum ts_fwd_path {
  TS_PATH_NONE = 0,
  TS_PATH_TCGEN05 = 1, /* bf16/f16 tensor-core prefill (tcgen05 + TMEM + TMA) */
  TS_PATH_SIMT = 2,    /* generic CUDA-core path (any dtype/dim/mask) */
  TS_PATH_DECODE = 3   /* split-K HBM-streaming decode */
} ts_fwd_path;

/* A [B, H, T, C] view: base pointer + element strides (b, h, t, c). */
typedef struct ts_view4 {
  void* data;
  int64_t stride[4];
} ts_view4;

/* Forward / decode problem.  Mirrors the arguments of
 * scaled_dot_product_attention (nn/attention.py:16-29). */
typedef struct ts_attn_params {
  ts_view4 q;  /* [B, Hq,  Tq, D]  */
  ts_view4 k;  /* [B, Hkv, Tk, D]  */
  ts_view4 v;  /* [B, Hkv, Tk, Dv] */
  ts_view4 o;  /* [B, Hq,  Tq, Dv] output, same dtype as q */
  /* optional [B, Hq, Tq] natural-log normaliser (-inf = fully masked row);
   * fp32, or fp64 when dtype is TS_F64 */
  void* lse;
  int64_t lse_stride[3];
  int32_t dtype; /* ts_dtype of q, k, v and o */
  int32_t batch, q_heads, kv_heads, q_len, kv_len, head_dim, value_dim;
  double scale;          /* softmax scale; the reference default is 1/sqrt(D) (nn/attention.py:60) */
  int32_t is_causal;     /* key j visible to query i iff i + offset >= j (nn/attention.py:108-111) */
  int64_t causal_offset; /* absolute position of query 0 in the key sequence */
  /* Optional per-row valid key count [B] (int32, device).  Keys j >= kv_lens[b]
   * are masked.  When set together with is_causal, the queries of row b sit at
   * the end of its valid keys: offset_b = kv_lens[b] - q_len (causal_offset is
   * then ignored).  Expresses tensorsmith's padded-cache + key-valid-mask idiom
   * (docs/transformers.md:52-55) without a mask tensor. */
  const int32_t* kv_lens;
  int32_t mask_kind;  /* ts_mask_kind */
  const void* mask;   /* [B, Hq, Tq, Tk] with broadcast (0) strides allowed */
  int64_t mask_stride[4];
} ts_attn_params;

/* Backward problem: the forward problem plus upstream and gradient views. */
typedef struct ts_attn_bwd_params {
  ts_attn_params fwd; /* q, k, v, o (forward output) and lse (required) */
  ts_view4 dout;      /* [B, Hq,  Tq, Dv] upstream gradient, dtype of q */
  ts_view4 dq;        /* [B, Hq,  Tq, D]  */
  ts_view4 dk;        /* [B, Hkv, Tk, D]  (summed over the query-head group) */
  ts_view4 dv;        /* [B, Hkv, Tk, Dv] */
} ts_attn_bwd_params;

/* KV-cache append: write a [B, H, steps, C] chunk at positions
 * [pos_b, pos_b + steps) of [B, H, capacity, C] caches. */
typedef struct ts_kv_append_params {
  ts_view4 key, value;             /* new chunk */
  ts_view4 key_cache, value_cache; /* preallocated storage */
  int32_t src_dtype;               /* ts_dtype of key/value (cast on write) */
  int32_t cache_dtype;             /* ts_dtype of the caches */
  int32_t batch, heads, steps, head_dim, value_dim, capacity;
  int64_t position;          /* write offset for every row when positions == NULL */
  const int32_t* positions;  /* optional [B] per-row write offsets (device) */
  int32_t* positions_out;    /* optional [B]: receives positions[b] + steps */
} ts_kv_append_params;

/* ABI version (TS_ATTN_ABI_VERSION) of the loaded library. */
TS_ATTN_API int ts_attn_abi_version(void);

/* Static description of a status code. */
TS_ATTN_API const char* ts_attn_strerror(int status);

/* Build provenance (no counterpart in tensorsmith): SHA-256, as 64 hex digits,
 * of the sources this library was compiled from -- every csrc/*.cu, csrc/*.cuh
 * and include/*.h, hashed in file-name order as name, NUL, contents, NUL.  The
 * Python loader refuses a library whose digest differs from the tree's. */
TS_ATTN_API const char* ts_attn_source_digest(void);

/* Kernel family ts_attn_fwd / ts_attn_decode would select (ts_fwd_path), or a
 * negative ts_status when the parameters are invalid. */
TS_ATTN_API int ts_attn_fwd_path(const ts_attn_params* params, int decode);

/* Prefill / training forward: O and (optionally) LSE.  Replaces the dense,
 * streaming and native forwards of nn/attention.py:132-198 (the native slot
 * :146-174 is where tensorsmith plugs a vendor kernel).  On the tensor-core
 * path the library picks the kernel by shape (two query tiles per CTA for two
 * or more 128-row tiles); the environment variable TS_FWD_KERNEL = "pair",
 * "tile" or "persistent", read at every call, forces one for tests and
 * measurements.  Results are the same within the stated tolerances. */
TS_ATTN_API int ts_attn_fwd(const ts_attn_params* params, void* stream);

/* Workspace bytes ts_attn_bwd needs (fp32 row statistics, plus an fp32 dQ
 * accumulator on the tensor-core path). */
TS_ATTN_API size_t ts_attn_bwd_workspace_size(const ts_attn_bwd_params* params);

/* Kernel family ts_attn_bwd would run (TS_PATH_TCGEN05 or TS_PATH_SIMT), or a
 * negative ts_status when the parameters are invalid. */
TS_ATTN_API int ts_attn_bwd_path(const ts_attn_bwd_params* params);

/* Backward: dQ, dK, dV from recomputed probabilities (LSE of the forward).
 * Replaces the dense / blockwise VJP and the GQA reduction of
 * nn/attention.py:200-248. */
TS_ATTN_API int ts_attn_bwd(const ts_attn_bwd_params* params, void* workspace, size_t workspace_bytes,
                void* stream);

/* Workspace bytes ts_attn_decode needs (per-split partial results). */
TS_ATTN_API size_t ts_attn_decode_workspace_size(const ts_attn_params* params);

/* Cached decode: a few query tokens against a long KV cache, split along the
 * keys and combined.  Same semantics as ts_attn_fwd; replaces the cached call
 * of nn/transformer.py:144-154 into nn/attention.py:132-145.  A grouped-query
 * step (one query token, 2-128 query heads per KV head, no mask, at least 64
 * (batch, KV head) pairs) runs on the tcgen05 prefill kernel with the query
 * heads of each KV head as the rows of one tile (ts_attn_fwd_path(params, 1)
 * then returns TS_PATH_TCGEN05).  Problems neither kernel family takes
 * (ts_attn_fwd_path(params, 1) != TS_PATH_DECODE) run exactly as ts_attn_fwd;
 * only TS_PATH_DECODE needs a workspace. */
TS_ATTN_API int ts_attn_decode(const ts_attn_params* params, void* workspace, size_t workspace_bytes,
                   void* stream);

/* KVCache.append slice write (nn/cache.py:54-86, unquantized storage). */
TS_ATTN_API int ts_kv_append(const ts_kv_append_params* params, void* stream);

/* Interleaved-pair rotary embedding of nn/attention.py:255-296 on a
 * [B, H, T, C] view: y = rope(x) at positions (positions[b] or offset) + t,
 * first rotary_dim (even) channels, inv_freq[i] = base^(-2i/rotary_dim) as
 * fp32 (rotary_dim/2 entries, device).  inverse != 0 applies the inverse
 * rotation (the VJP of :287-293).  y may alias x. */
TS_ATTN_API int ts_rope(ts_view4 x, ts_view4 y, int32_t dtype, int32_t batch, int32_t heads, int32_t seq,
                        int32_t channels, int32_t rotary_dim, int64_t offset, const int32_t* positions,
                        const float* inv_freq, int32_t inverse, void* stream);

/* KVCache.append with the key rotation of the attention module fused into the
 * write (nn/transformer.py:139-142 followed by nn/cache.py:54-86): keys are
 * rotated at their cache positions, values copied. */
TS_ATTN_API int ts_kv_append_rope(const ts_kv_append_params* params, const float* inv_freq, int32_t rotary_dim,
                                  void* stream);

/* KVCache.reorder batch gather (nn/cache.py:110-123): dst[b] = src[index[b]].
 * src and dst must not overlap. */
TS_ATTN_API int ts_kv_reorder(ts_view4 src, ts_view4 dst, int32_t dtype, int32_t batch, int32_t heads,
                  int32_t length, int32_t channels, const int32_t* index, void* stream);

/* Size of the fixed device scratch ts_attn_decode_noalloc uses (8 MiB per GPU). */
#define TS_ATTN_NOALLOC_SCRATCH_BYTES ((size_t)8 << 20)

/* Decode for callers that cannot allocate device memory (no counterpart in
 * tensorsmith): e.g. a serving loop whose allocator already gave all free HBM
 * to KV-cache pages, or host code that must not call cudaMalloc (which may
 * synchronise the device) between decode steps.  Same semantics and kernels as
 * ts_attn_decode, but the split partials live in a fixed library-owned device
 * array of TS_ATTN_NOALLOC_SCRATCH_BYTES on every GPU that loads the library,
 * held until exit.  The first call in a CUDA context looks up the array's
 * device address (make it before any stream capture; a context recreated after
 * cudaDeviceReset looks it up again); calls that overlap on the GPU share the
 * array and race.  Returns TS_ERR_WORKSPACE, launching nothing, when
 * the problem needs more scratch than that.  Allocates nothing. */
TS_ATTN_API int ts_attn_decode_noalloc(const ts_attn_params* params, void* stream);

/* Attention dropout of nn/attention.py:140-144 (forward) and :212-216
 * (backward): P.V uses p * keep / (1 - p) with keep = (u >= p), u uniform on
 * the 2^16 points k * 2^-16 of [0, 1) per (batch, query head, query row, key);
 * dP is multiplied by the same factor; LSE stays the softmax normaliser.  u
 * comes from a counter-based generator (Philox4x32-10, 16 bits per key) keyed
 * by (seed, offset), so a backward given the forward's (seed, offset)
 * regenerates its mask without storing it. */
typedef struct ts_dropout {
  double p;        /* drop probability, 0 <= p < 1 */
  uint64_t seed;   /* generator key */
  uint64_t offset; /* call counter; a forward and its backward pass the same value */
} ts_dropout;

/* ts_attn_fwd with dropout: the tcgen05 kernel where ts_attn_fwd would use it,
 * the generic CUDA-core kernels otherwise (every dtype / shape / mask of
 * ts_attn_fwd).  p = 0 is exactly ts_attn_fwd (same kernel selection). */
TS_ATTN_API int ts_attn_fwd_dropout(const ts_attn_params* params, const ts_dropout* dropout, void* stream);

/* Workspace bytes ts_attn_bwd_dropout needs. */
TS_ATTN_API size_t ts_attn_bwd_dropout_workspace_size(const ts_attn_bwd_params* params);

/* ts_attn_bwd for a forward made by ts_attn_fwd_dropout with the same dropout
 * arguments (p = 0 is exactly ts_attn_bwd). */
TS_ATTN_API int ts_attn_bwd_dropout(const ts_attn_bwd_params* params, const ts_dropout* dropout, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* The keep mask those calls use, as uint8 0/1 [batch, heads, q_len, kv_len]
 * (contiguous; heads = query heads). */
TS_ATTN_API int ts_attn_dropout_mask(const ts_dropout* dropout, int32_t batch, int32_t heads, int32_t q_len,
                                     int32_t kv_len, uint8_t* mask, void* stream);

/* Quantising KVCache.append of nn/cache.py:54-86 with quantized=True.
 * key_cache / value_cache are int8 views; params->cache_dtype is the cache's
 * compute dtype (rows are rounded to it first, :68).  Per row:
 * scale = max(max|x| / 127, 1e-8) in fp32, q = round_half_even(x / scale)
 * (:70-75).  key_scales / value_scales are contiguous fp32 [batch, heads,
 * capacity] (the reference's [B, H, capacity, 1]). */
TS_ATTN_API int ts_kv_append_int8(const ts_kv_append_params* params, float* key_scales, float* value_scales,
                                  void* stream);

/* KVCache.get of a quantized cache (nn/cache.py:88-99):
 * dst[b, h, t, c] = dtype(float(src[b, h, t, c]) * scales[b, h, t]) for
 * t < length; scales contiguous [batch, heads, scale_capacity]. */
TS_ATTN_API int ts_kv_dequant_int8(ts_view4 src, const float* scales, int64_t scale_capacity, ts_view4 dst,
                                   int32_t dtype, int32_t batch, int32_t heads, int32_t length, int32_t channels,
                                   void* stream);

/* Workspace bytes ts_attn_decode_int8 needs (0 when one split suffices). */
TS_ATTN_API size_t ts_attn_decode_int8_workspace_size(const ts_attn_params* params);

/* Decode straight from an int8 KV cache (replaces nn/cache.py:91-99 followed
 * by nn/attention.py:132-145): params->k / params->v are int8 views (element
 * strides = bytes), params->dtype is the dtype of q and o, scales as in
 * ts_kv_append_int8 with `scale_capacity` keys per (row, head).  Scores are
 * k_scale * (q . k8) and probabilities meet v_scale * v8, in fp32; the
 * dequantised rows are never written.  Same masking rules as ts_attn_decode
 * (causal, causal_offset, kv_lens; no explicit mask).  TS_ERR_UNSUPPORTED when
 * the shape is outside the kernel (head_dim = value_dim in {64, 128, 256},
 * 16-byte aligned rows): dequantise with ts_kv_dequant_int8 and call
 * ts_attn_fwd instead. */
TS_ATTN_API int ts_attn_decode_int8(const ts_attn_params* params, const float* key_scales,
                                    const float* value_scales, int64_t scale_capacity, void* workspace,
                                    size_t workspace_bytes, void* stream);

/* Reads and clears the device fault word written by kernels whose bounded
 * waits gave up.  Synchronises `stream`.  Returns TS_OK or
 * TS_ERR_DEVICE_TIMEOUT; *info (optional) receives the recorded site code. */
TS_ATTN_API int ts_attn_device_status(void* stream, uint32_t* info);

#ifdef __cplusplus
}
#endif

#endif /* TS_ATTN_H */
