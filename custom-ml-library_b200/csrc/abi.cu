// extern "C" entry points of libts_attn.so (declared in include/ts_attn.h):
// argument validation, kernel selection and the device fault word.
#include <cmath>
#include <cstdio>
#include <mutex>

#include "common.cuh"
#include "decode.cuh"
#include "int8.cuh"
#include "kv_cache.cuh"
#include "rope.cuh"
#include "simt.cuh"
#include "symbols.cuh"
#include "tc_bwd.cuh"
#include "tc_fwd.cuh"

namespace {

// Fault word written by kernels whose bounded waits gave up (per device).
__device__ uint32_t g_fault_word;

uint32_t* fault_ptr() { return static_cast<uint32_t*>(tsa::device_symbol_address(&g_fault_word)); }

inline cudaStream_t as_stream(void* s) { return reinterpret_cast<cudaStream_t>(s); }

int from_cuda(cudaError_t e) {
  if (e == cudaSuccess) return TS_OK;
  if (e == cudaErrorInvalidValue) return TS_ERR_INVALID_ARGUMENT;
  return TS_ERR_LAUNCH;
}

bool dtype_ok(int d) { return d == TS_F32 || d == TS_F16 || d == TS_BF16 || d == TS_F64; }

int check_params(const ts_attn_params* p) {
  if (!p) return TS_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(p->dtype)) return TS_ERR_UNSUPPORTED;
  if (p->batch <= 0 || p->q_heads <= 0 || p->kv_heads <= 0 || p->q_len <= 0 || p->kv_len <= 0 ||
      p->head_dim <= 0 || p->value_dim <= 0)
    return TS_ERR_INVALID_ARGUMENT;
  if (p->q_heads % p->kv_heads) return TS_ERR_INVALID_ARGUMENT;
  if (p->head_dim > 256 || p->value_dim > 256) return TS_ERR_UNSUPPORTED;
  if (!p->q.data || !p->k.data || !p->v.data || !p->o.data) return TS_ERR_INVALID_ARGUMENT;
  if (p->causal_offset < 0) return TS_ERR_INVALID_ARGUMENT;
  if (!(p->scale == p->scale) || p->scale > 1.0e300 || p->scale < -1.0e300) return TS_ERR_INVALID_ARGUMENT;
  if (p->mask_kind < TS_MASK_NONE || p->mask_kind > TS_MASK_ADD_F32) return TS_ERR_INVALID_ARGUMENT;
  if (p->mask_kind != TS_MASK_NONE && !p->mask) return TS_ERR_INVALID_ARGUMENT;
  return TS_OK;
}

}  // namespace

namespace tsa {

void* device_symbol_address(const void* symbol) {
  // CUresult cuCtxGetId(CUcontext ctx, unsigned long long* id); ctx = NULL: the current context.
  typedef int (*CtxGetIdFn)(void*, unsigned long long*);
  struct Entry {
    const void* symbol;
    unsigned long long ctx;
    void* ptr;
  };
  constexpr int kEntries = 256;
  static Entry cache[kEntries];
  static int used = 0;
  static CtxGetIdFn ctx_get_id = nullptr;
  static std::once_flag once;
  static std::mutex lock;
  std::call_once(once, [] {
    void* fn = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuCtxGetId", &fn, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      ctx_get_id = reinterpret_cast<CtxGetIdFn>(fn);
  });
  std::lock_guard<std::mutex> guard(lock);
  unsigned long long ctx = 0;
  bool have_ctx = ctx_get_id && ctx_get_id(nullptr, &ctx) == 0;
  if (have_ctx)
    for (int i = 0; i < used; ++i)
      if (cache[i].symbol == symbol && cache[i].ctx == ctx) return cache[i].ptr;
  void* ptr = nullptr;
  if (cudaGetSymbolAddress(&ptr, symbol) != cudaSuccess || ptr == nullptr) return nullptr;
  // The lookup above makes the device's primary context current if nothing was.
  if (!have_ctx) have_ctx = ctx_get_id && ctx_get_id(nullptr, &ctx) == 0;
  if (have_ctx && used < kEntries) cache[used++] = Entry{symbol, ctx, ptr};
  return ptr;
}

}  // namespace tsa

extern "C" {

int ts_attn_abi_version(void) { return TS_ATTN_ABI_VERSION; }

#ifndef TS_SOURCE_DIGEST
#define TS_SOURCE_DIGEST "unknown"
#endif
const char* ts_attn_source_digest(void) { return TS_SOURCE_DIGEST; }

const char* ts_attn_strerror(int status) {
  switch (status) {
    case TS_OK: return "ok";
    case TS_ERR_INVALID_ARGUMENT: return "invalid argument (shape, stride, pointer or value)";
    case TS_ERR_UNSUPPORTED: return "unsupported dtype / dimension combination";
    case TS_ERR_WORKSPACE: return "workspace missing or too small";
    case TS_ERR_LAUNCH: return "CUDA kernel launch or driver call failed";
    case TS_ERR_DEVICE_TIMEOUT: return "a bounded wait inside an engine kernel gave up";
    case TS_ERR_CAPACITY: return "KV-cache capacity exceeded or empty append";
  }
  return "unknown status";
}

int ts_attn_fwd_path(const ts_attn_params* p, int decode) {
  const int st = check_params(p);
  if (st != TS_OK) return st;
  ts_attn_params view;
  if (decode && tsa::gqa_decode_view(*p, &view)) return TS_PATH_TCGEN05;
  if (decode && tsa::decode_supported(*p)) return TS_PATH_DECODE;
  if (tsa::tc_fwd_supported(*p)) return TS_PATH_TCGEN05;
  return TS_PATH_SIMT;
}

int ts_attn_fwd(const ts_attn_params* p, void* stream) {
  const int st = check_params(p);
  if (st != TS_OK) return st;
  if (tsa::tc_fwd_supported(*p)) return from_cuda(tsa::tc_forward(*p, fault_ptr(), as_stream(stream)));
  return from_cuda(tsa::simt_forward(*p, as_stream(stream)));
}

size_t ts_attn_decode_workspace_size(const ts_attn_params* p) {
  ts_attn_params view;
  if (check_params(p) != TS_OK || tsa::gqa_decode_view(*p, &view) || !tsa::decode_supported(*p)) return 0;
  return tsa::decode_workspace(*p);
}

int ts_attn_decode(const ts_attn_params* p, void* workspace, size_t workspace_bytes, void* stream) {
  const int st = check_params(p);
  if (st != TS_OK) return st;
  // A grouped-query step over enough (batch, KV head) pairs runs on the
  // tensor cores, the query heads of each KV head as the rows of one tile.
  ts_attn_params view;
  if (tsa::gqa_decode_view(*p, &view)) return from_cuda(tsa::tc_forward(view, fault_ptr(), as_stream(stream)));
  // Problems the split-K kernels do not take (many query rows, explicit masks,
  // value_dim != head_dim) go where ts_attn_fwd would send them; neither path
  // needs a workspace.
  if (!tsa::decode_supported(*p)) return ts_attn_fwd(p, stream);
  const size_t need = tsa::decode_workspace(*p);
  if (need && (!workspace || workspace_bytes < need)) return TS_ERR_WORKSPACE;
  return from_cuda(tsa::decode_forward(*p, workspace, workspace_bytes, fault_ptr(), as_stream(stream)));
}

size_t ts_attn_bwd_workspace_size(const ts_attn_bwd_params* bp) {
  if (!bp || check_params(&bp->fwd) != TS_OK) return 0;
  if (tsa::tc_bwd_supported(*bp)) return tsa::tc_bwd_workspace(*bp);
  return tsa::simt_backward_workspace(*bp);
}

int ts_attn_bwd_path(const ts_attn_bwd_params* bp) {
  if (!bp) return TS_ERR_INVALID_ARGUMENT;
  const int st = check_params(&bp->fwd);
  if (st != TS_OK) return st;
  return tsa::tc_bwd_supported(*bp) ? TS_PATH_TCGEN05 : TS_PATH_SIMT;
}

int ts_attn_bwd(const ts_attn_bwd_params* bp, void* workspace, size_t workspace_bytes, void* stream) {
  if (!bp) return TS_ERR_INVALID_ARGUMENT;
  const int st = check_params(&bp->fwd);
  if (st != TS_OK) return st;
  if (!bp->fwd.lse || !bp->dout.data || !bp->dq.data || !bp->dk.data || !bp->dv.data)
    return TS_ERR_INVALID_ARGUMENT;
  if (tsa::tc_bwd_supported(*bp)) {
    if (!workspace || workspace_bytes < tsa::tc_bwd_workspace(*bp)) return TS_ERR_WORKSPACE;
    return from_cuda(tsa::tc_backward(*bp, workspace, workspace_bytes, fault_ptr(), as_stream(stream)));
  }
  const size_t need = tsa::simt_backward_workspace(*bp);
  if (!workspace || workspace_bytes < need) return TS_ERR_WORKSPACE;
  return from_cuda(tsa::simt_backward(*bp, workspace, as_stream(stream)));
}

int ts_kv_append(const ts_kv_append_params* p, void* stream) {
  if (!p) return TS_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(p->src_dtype) || !dtype_ok(p->cache_dtype)) return TS_ERR_UNSUPPORTED;
  if (p->batch <= 0 || p->heads <= 0 || p->head_dim <= 0 || p->value_dim <= 0 || p->capacity <= 0)
    return TS_ERR_INVALID_ARGUMENT;
  if (!p->key.data || !p->value.data || !p->key_cache.data || !p->value_cache.data)
    return TS_ERR_INVALID_ARGUMENT;
  if (p->steps <= 0) return TS_ERR_CAPACITY;
  if (!p->positions && (p->position < 0 || p->position + p->steps > p->capacity)) return TS_ERR_CAPACITY;
  return from_cuda(tsa::kv_append(*p, as_stream(stream)));
}

int ts_rope(ts_view4 x, ts_view4 y, int32_t dtype, int32_t batch, int32_t heads, int32_t seq, int32_t channels,
            int32_t rotary_dim, int64_t offset, const int32_t* positions, const float* inv_freq, int32_t inverse,
            void* stream) {
  if (!dtype_ok(dtype)) return TS_ERR_UNSUPPORTED;
  if (!x.data || !y.data || !inv_freq || batch <= 0 || heads <= 0 || seq <= 0 || channels <= 0)
    return TS_ERR_INVALID_ARGUMENT;
  if (rotary_dim <= 0 || rotary_dim % 2 || rotary_dim > channels || offset < 0) return TS_ERR_INVALID_ARGUMENT;
  return from_cuda(tsa::rope_apply(x, y, dtype, batch, heads, seq, channels, rotary_dim, offset, positions, inv_freq,
                                   inverse, as_stream(stream)));
}

int ts_kv_append_rope(const ts_kv_append_params* p, const float* inv_freq, int32_t rotary_dim, void* stream) {
  if (!p) return TS_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(p->src_dtype) || !dtype_ok(p->cache_dtype)) return TS_ERR_UNSUPPORTED;
  if (p->batch <= 0 || p->heads <= 0 || p->head_dim <= 0 || p->value_dim <= 0 || p->capacity <= 0 || !inv_freq)
    return TS_ERR_INVALID_ARGUMENT;
  if (!p->key.data || !p->value.data || !p->key_cache.data || !p->value_cache.data) return TS_ERR_INVALID_ARGUMENT;
  if (rotary_dim <= 0 || rotary_dim % 2 || rotary_dim > p->head_dim) return TS_ERR_INVALID_ARGUMENT;
  if (p->steps <= 0) return TS_ERR_CAPACITY;
  if (!p->positions && (p->position < 0 || p->position + p->steps > p->capacity)) return TS_ERR_CAPACITY;
  return from_cuda(tsa::kv_append_rope(*p, inv_freq, rotary_dim, as_stream(stream)));
}

int ts_kv_reorder(ts_view4 src, ts_view4 dst, int32_t dtype, int32_t batch, int32_t heads, int32_t length,
                  int32_t channels, const int32_t* index, void* stream) {
  if (!dtype_ok(dtype) && dtype != TS_I8) return TS_ERR_UNSUPPORTED;
  if (!src.data || !dst.data || !index || batch <= 0 || heads <= 0 || length < 0 || channels <= 0)
    return TS_ERR_INVALID_ARGUMENT;
  return from_cuda(tsa::kv_reorder(src, dst, dtype, batch, heads, length, channels, index, as_stream(stream)));
}

}  // extern "C"

namespace {
bool make_dropout(const ts_dropout* d, tsa::DropoutArgs& out) {
  if (!d || !(d->p >= 0.0) || !(d->p < 1.0)) return false;
  out.p = (float)d->p;
  out.keep_min = (uint32_t)std::ceil(d->p * 65536.0);
  out.inv_keep_f = 1.0f / (float)(1.0 - d->p);
  out.inv_keep_d = 1.0 / (1.0 - d->p);
  out.seed = d->seed;
  out.offset = d->offset;
  return true;
}
}  // namespace

extern "C" {

int ts_attn_fwd_dropout(const ts_attn_params* p, const ts_dropout* d, void* stream) {
  const int st = check_params(p);
  if (st != TS_OK) return st;
  tsa::DropoutArgs args;
  if (!make_dropout(d, args)) return TS_ERR_INVALID_ARGUMENT;
  if (d->p == 0.0) return ts_attn_fwd(p, stream);  // no dropout: the plain path selection
  if (tsa::tc_fwd_supported(*p)) return from_cuda(tsa::tc_forward(*p, fault_ptr(), as_stream(stream), &args));
  return from_cuda(tsa::simt_forward(*p, as_stream(stream), &args));
}

size_t ts_attn_bwd_dropout_workspace_size(const ts_attn_bwd_params* bp) {
  if (!bp || check_params(&bp->fwd) != TS_OK) return 0;
  const size_t simt = tsa::simt_backward_workspace(*bp);
  if (!tsa::tc_bwd_supported(*bp)) return simt;
  const size_t tc = tsa::tc_bwd_workspace(*bp);
  return tc > simt ? tc : simt;
}

int ts_attn_bwd_dropout(const ts_attn_bwd_params* bp, const ts_dropout* d, void* workspace, size_t workspace_bytes,
                        void* stream) {
  if (!bp) return TS_ERR_INVALID_ARGUMENT;
  const int st = check_params(&bp->fwd);
  if (st != TS_OK) return st;
  if (!bp->fwd.lse || !bp->dout.data || !bp->dq.data || !bp->dk.data || !bp->dv.data)
    return TS_ERR_INVALID_ARGUMENT;
  tsa::DropoutArgs args;
  if (!make_dropout(d, args)) return TS_ERR_INVALID_ARGUMENT;
  if (d->p == 0.0) return ts_attn_bwd(bp, workspace, workspace_bytes, stream);  // the plain path selection
  if (tsa::tc_bwd_supported(*bp)) {
    if (!workspace || workspace_bytes < tsa::tc_bwd_workspace(*bp)) return TS_ERR_WORKSPACE;
    return from_cuda(tsa::tc_backward(*bp, workspace, workspace_bytes, fault_ptr(), as_stream(stream), &args));
  }
  if (!workspace || workspace_bytes < tsa::simt_backward_workspace(*bp)) return TS_ERR_WORKSPACE;
  return from_cuda(tsa::simt_backward(*bp, workspace, as_stream(stream), &args));
}

int ts_attn_dropout_mask(const ts_dropout* d, int32_t batch, int32_t heads, int32_t q_len, int32_t kv_len,
                         uint8_t* mask, void* stream) {
  tsa::DropoutArgs args;
  if (!make_dropout(d, args) || !mask || batch <= 0 || heads <= 0 || q_len <= 0 || kv_len <= 0)
    return TS_ERR_INVALID_ARGUMENT;
  return from_cuda(tsa::dropout_mask(args, batch, heads, q_len, kv_len, mask, as_stream(stream)));
}

int ts_kv_append_int8(const ts_kv_append_params* p, float* key_scales, float* value_scales, void* stream) {
  if (!p) return TS_ERR_INVALID_ARGUMENT;
  if (!dtype_ok(p->src_dtype) || !dtype_ok(p->cache_dtype)) return TS_ERR_UNSUPPORTED;
  if (p->batch <= 0 || p->heads <= 0 || p->head_dim <= 0 || p->value_dim <= 0 || p->capacity <= 0)
    return TS_ERR_INVALID_ARGUMENT;
  if (!p->key.data || !p->value.data || !p->key_cache.data || !p->value_cache.data || !key_scales || !value_scales)
    return TS_ERR_INVALID_ARGUMENT;
  if (p->steps <= 0) return TS_ERR_CAPACITY;
  if (!p->positions && (p->position < 0 || p->position + p->steps > p->capacity)) return TS_ERR_CAPACITY;
  return from_cuda(tsa::kv_append_int8(*p, key_scales, value_scales, as_stream(stream)));
}

int ts_kv_dequant_int8(ts_view4 src, const float* scales, int64_t scale_capacity, ts_view4 dst, int32_t dtype,
                       int32_t batch, int32_t heads, int32_t length, int32_t channels, void* stream) {
  if (!dtype_ok(dtype)) return TS_ERR_UNSUPPORTED;
  if (!src.data || !dst.data || !scales || batch <= 0 || heads <= 0 || length < 0 || channels <= 0 ||
      scale_capacity < length)
    return TS_ERR_INVALID_ARGUMENT;
  return from_cuda(tsa::kv_dequant_int8(src, scales, scale_capacity, dst, dtype, batch, heads, length, channels,
                                        as_stream(stream)));
}

size_t ts_attn_decode_int8_workspace_size(const ts_attn_params* p) {
  if (check_params(p) != TS_OK || !tsa::decode_int8_supported(*p)) return 0;
  return tsa::decode_int8_workspace(*p);
}

int ts_attn_decode_int8(const ts_attn_params* p, const float* key_scales, const float* value_scales,
                        int64_t scale_capacity, void* workspace, size_t workspace_bytes, void* stream) {
  const int st = check_params(p);
  if (st != TS_OK) return st;
  if (!key_scales || !value_scales || scale_capacity < p->kv_len) return TS_ERR_INVALID_ARGUMENT;
  if (!tsa::decode_int8_supported(*p)) return TS_ERR_UNSUPPORTED;
  const size_t need = tsa::decode_int8_workspace(*p);
  if (need && (!workspace || workspace_bytes < need)) return TS_ERR_WORKSPACE;
  return from_cuda(tsa::decode_int8_forward(*p, key_scales, value_scales, scale_capacity, workspace,
                                            workspace_bytes, fault_ptr(), as_stream(stream)));
}

int ts_attn_device_status(void* stream, uint32_t* info) {
  uint32_t* f = fault_ptr();
  if (!f) return TS_ERR_LAUNCH;
  uint32_t host = 0;
  cudaStream_t s = as_stream(stream);
  if (cudaMemcpyAsync(&host, f, sizeof(uint32_t), cudaMemcpyDeviceToHost, s) != cudaSuccess) return TS_ERR_LAUNCH;
  if (cudaStreamSynchronize(s) != cudaSuccess) return TS_ERR_LAUNCH;
  if (info) *info = host;
  if (host) {
    const uint32_t zero = 0;
    if (cudaMemcpyAsync(f, &zero, sizeof(uint32_t), cudaMemcpyHostToDevice, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
      return TS_ERR_LAUNCH;
    return TS_ERR_DEVICE_TIMEOUT;
  }
  return TS_OK;
}

}  // extern "C"
