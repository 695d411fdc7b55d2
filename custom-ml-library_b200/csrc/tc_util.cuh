// Helpers shared by the tcgen05 kernels: bounded mbarrier waits that also
// stop as soon as any CTA recorded a fault, and host-side TMA tensor-map
// encoding for [B, H, T, C] bf16/f16 views (128-byte swizzle, 64-channel boxes).
#pragma once
#include <cuda.h>

#include <mutex>

#include "ptx.cuh"

namespace tsa {

__device__ __forceinline__ bool fault_set(const uint32_t* fault) {
  return fault && *reinterpret_cast<const volatile uint32_t*>(fault) != 0u;
}

// Bounded wait that also gives up as soon as any CTA recorded a fault.
__device__ __forceinline__ bool wait_bar(uint64_t* bar, uint32_t parity, uint32_t* fault,
                                         uint32_t site) {
  if (ptx::mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = global_ns();
  for (uint32_t it = 1;; ++it) {
    if (ptx::mbar_try_wait(bar, parity)) return true;
    if ((it & 255u) == 0u) {
      if (fault_set(fault)) return false;
      if (global_ns() - t0 > kWaitLimitNs) {
        record_fault(fault, site);
        return false;
      }
    }
  }
}

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*,
                                  CUtensorMapInterleave, CUtensorMapSwizzle, CUtensorMapL2promotion,
                                  CUtensorMapFloatOOBfill);

// cuTensorMapEncodeTiled through the runtime's driver entry point (no -lcuda).
inline EncodeTiledFn encode_fn() {
  static EncodeTiledFn fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* ptr = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &ptr, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<EncodeTiledFn>(ptr);
  });
  return fn;
}

// cudaFuncSetAttribute(MaxDynamicSharedMemorySize) for `kern` on the current
// device, called once per (kernel, device): the attribute persists, and small
// problems (a few microseconds of GPU work) otherwise pay the call every launch.
inline cudaError_t ensure_max_smem(const void* kern, int bytes) {
  struct Entry {
    const void* kern;
    int device;
  };
  constexpr int kEntries = 512;
  static Entry done[kEntries];
  static int used = 0;
  static std::mutex lock;
  int device = -1;
  cudaError_t e = cudaGetDevice(&device);
  if (e != cudaSuccess) return e;
  std::lock_guard<std::mutex> guard(lock);
  for (int i = 0; i < used; ++i)
    if (done[i].kern == kern && done[i].device == device) return cudaSuccess;
  e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e == cudaSuccess && used < kEntries) done[used++] = Entry{kern, device};
  return e;
}

// A 2-byte-element view a TMA map can address: unit channel stride, 16-byte
// aligned base and strides.
inline bool view_tma_ok(const ts_view4& v) {
  if (v.stride[3] != 1) return false;
  if (reinterpret_cast<uintptr_t>(v.data) % 16) return false;
  for (int i = 0; i < 3; ++i)
    if ((v.stride[i] * 2) % 16 || v.stride[i] <= 0) return false;
  return true;
}

// 4-D map (channels, sequence, heads, batch), box {64, box_rows, 1, 1},
// 128-byte swizzle, zero fill outside the tensor.
inline bool make_map(CUtensorMap* map, const ts_view4& v, int dtype, int batch, int heads, int len,
                     int channels, int box_rows) {
  if (!encode_fn()) return false;
  const cuuint64_t dims[4] = {(cuuint64_t)channels, (cuuint64_t)len, (cuuint64_t)heads, (cuuint64_t)batch};
  const cuuint64_t strides[3] = {(cuuint64_t)v.stride[2] * 2, (cuuint64_t)v.stride[1] * 2,
                                 (cuuint64_t)v.stride[0] * 2};
  const cuuint32_t box[4] = {64, (cuuint32_t)box_rows, 1, 1};
  const cuuint32_t estr[4] = {1, 1, 1, 1};
  const CUtensorMapDataType dt =
      dtype == TS_BF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16;
  return encode_fn()(map, dt, 4, v.data, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                     CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                     CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace tsa
