// Device addresses of the library's file-scope __device__ variables (the
// fault word, the no-allocation decode scratch).
#pragma once

namespace tsa {

// Device address of `symbol` (the host-side name of a file-scope __device__
// variable) in the calling thread's current CUDA context, or nullptr.  The
// address is looked up with cudaGetSymbolAddress the first time a context asks
// and cached under that context's unique id (cuCtxGetId), so a context that is
// destroyed and recreated (cudaDeviceReset) gets a fresh lookup instead of a
// stale pointer.  Thread-safe.
void* device_symbol_address(const void* symbol);

}  // namespace tsa
