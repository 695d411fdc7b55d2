// ts_attn_decode_noalloc: the split-K decode for callers that cannot allocate
// device memory when they decode.
//
// Who needs it: a serving loop whose allocator has already handed every free
// byte of HBM to KV-cache pages, or host code that must not call cudaMalloc
// between decode steps (cudaMalloc may synchronise the device and stall the
// token loop).  Such callers cannot provide the workspace ts_attn_decode asks
// for, so this entry point keeps the split partials in one fixed scratch array
// that belongs to the library.
//
// The scratch is the file-scope device array below: kNoAllocScratchBytes
// (TS_ATTN_NOALLOC_SCRATCH_BYTES, 8 MiB) on every GPU that loads the library,
// held until the process exits.  Host code cannot use the array's name as a
// device address (on the host it names a stand-in object), so the first call
// on each device looks the real address up with cudaGetSymbolAddress while
// that device is current and caches it under the context's unique id (a
// context recreated after cudaDeviceReset looks it up again); make that first
// call before any stream capture.  Every call on a device shares the array, so calls that
// overlap on the GPU (different streams, or threads, without ordering) race on
// it.  No byte of it has to start at zero: a call writes each partial before
// it reads it, so the contents left by the previous call are never used.
// Problems whose partials need more than the scratch size are rejected with
// TS_ERR_WORKSPACE before anything is launched.  No cudaMalloc, cudaFree or
// allocating library routine is called here.
#include "common.cuh"
#include "symbols.cuh"

namespace {

constexpr size_t kNoAllocScratchBytes = TS_ATTN_NOALLOC_SCRATCH_BYTES;
static_assert(kNoAllocScratchBytes == (size_t)8 << 20, "scratch size is part of the ABI contract");

static __device__ __align__(256) unsigned char g_decode_scratch[kNoAllocScratchBytes];

}  // namespace

extern "C" int ts_attn_decode_noalloc(const ts_attn_params* params, void* stream) {
  const int path = ts_attn_fwd_path(params, 1);  // validates the problem
  if (path < 0) return path;
  if (path != TS_PATH_DECODE) return ts_attn_decode(params, nullptr, 0, stream);  // needs no scratch
  const size_t need = ts_attn_decode_workspace_size(params);
  if (need > kNoAllocScratchBytes) return TS_ERR_WORKSPACE;
  void* scratch = tsa::device_symbol_address(&g_decode_scratch);
  if (scratch == nullptr) return TS_ERR_LAUNCH;
  return ts_attn_decode(params, scratch, kNoAllocScratchBytes, stream);
}
