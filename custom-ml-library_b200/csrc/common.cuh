// Shared device helpers of the attention engine: element conversion, fault
// reporting for bounded waits, and small integer utilities.
#pragma once

#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include "../../include/ts_attn.h"

namespace tsa {

// ---------------------------------------------------------------------------
// Element conversion
// ---------------------------------------------------------------------------
template <typename T> struct Elem;
template <> struct Elem<float> {
  using acc = float;
  static __device__ __forceinline__ float to_acc(float x) { return x; }
  static __device__ __forceinline__ float from_acc(float x) { return x; }
};
template <> struct Elem<double> {
  using acc = double;
  static __device__ __forceinline__ double to_acc(double x) { return x; }
  static __device__ __forceinline__ double from_acc(double x) { return x; }
};
template <> struct Elem<__half> {
  using acc = float;
  static __device__ __forceinline__ float to_acc(__half x) { return __half2float(x); }
  static __device__ __forceinline__ __half from_acc(float x) { return __float2half_rn(x); }
};
template <> struct Elem<__nv_bfloat16> {
  using acc = float;
  static __device__ __forceinline__ float to_acc(__nv_bfloat16 x) { return __bfloat162float(x); }
  static __device__ __forceinline__ __nv_bfloat16 from_acc(float x) { return __float2bfloat16_rn(x); }
};

template <typename A> __device__ __forceinline__ A neg_inf();
template <> __device__ __forceinline__ float neg_inf<float>() { return -__int_as_float(0x7f800000); }
template <> __device__ __forceinline__ double neg_inf<double>() {
  return -__longlong_as_double(0x7ff0000000000000ll);
}

__device__ __forceinline__ float acc_exp(float x) { return expf(x); }
__device__ __forceinline__ double acc_exp(double x) { return exp(x); }
__device__ __forceinline__ float acc_log(float x) { return logf(x); }
__device__ __forceinline__ double acc_log(double x) { return log(x); }

// ---------------------------------------------------------------------------
// Fault reporting: kernels never trap.  A wait that gives up records a site
// code in the fault word (owned by the host library, passed by pointer) and
// the kernel unwinds normally.
// ---------------------------------------------------------------------------
enum FaultSite : uint32_t {
  FAULT_NONE = 0,
  FAULT_FWD_Q = 0x101,
  FAULT_FWD_KV = 0x102,
  FAULT_FWD_S = 0x103,
  FAULT_FWD_P = 0x104,
  FAULT_FWD_O = 0x105,
  FAULT_FWD_EMPTY = 0x106,
  FAULT_FWD_DRAIN = 0x107,
  FAULT_DEC_FULL = 0x201,
  FAULT_DEC_EMPTY = 0x202,
};

__device__ __forceinline__ void record_fault(uint32_t* fault, uint32_t site) {
  if (fault) atomicCAS(fault, 0u, site);
}

__device__ __forceinline__ uint64_t global_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Upper bound of any single wait inside an engine kernel.  Every wait in the
// pipeline normally completes within microseconds.
constexpr uint64_t kWaitLimitNs = 2000000000ull;

__host__ __device__ __forceinline__ int ceil_div(int a, int b) { return (a + b - 1) / b; }
__host__ __device__ __forceinline__ int64_t i64max(int64_t a, int64_t b) { return a > b ? a : b; }
__host__ __device__ __forceinline__ int64_t i64min(int64_t a, int64_t b) { return a < b ? a : b; }

}  // namespace tsa
