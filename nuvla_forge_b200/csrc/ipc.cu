// Peer-mapped device buffers for the fused collectives (CUDA IPC, no multicast).
//
// Each rank allocates one buffer, exports a CUDA IPC handle, and opens every
// peer's handle; the resulting pointers are peer mappings over NVLink that the
// kernels in comm.cu address with plain loads and stores. No NVLink multicast
// object is ever created, so a rank that exits cannot leave peers bound to a
// multicast group.
#include <cuda_runtime.h>
#include <stdint.h>
#include <string.h>

#include "nfb_api.h"

#define NFB_API extern "C" __attribute__((visibility("default")))

NFB_API int nfb_ipc_handle_bytes() { return (int)sizeof(cudaIpcMemHandle_t); }

// Allocate `bytes` of zeroed device memory on the current device and export its IPC handle.
NFB_API int nfb_ipc_alloc(uint64_t bytes, void** ptr, void* handle_out) {
  void* p = nullptr;
  cudaError_t e = cudaMalloc(&p, bytes);
  if (e != cudaSuccess) return (int)e;
  e = cudaMemset(p, 0, bytes);
  if (e != cudaSuccess) { cudaFree(p); return (int)e; }
  cudaIpcMemHandle_t h;
  e = cudaIpcGetMemHandle(&h, p);
  if (e != cudaSuccess) { cudaFree(p); return (int)e; }
  memcpy(handle_out, &h, sizeof(h));
  *ptr = p;
  return 0;
}

// Map a peer's exported buffer into this process (peer access enabled lazily).
NFB_API int nfb_ipc_open(const void* handle, void** ptr) {
  cudaIpcMemHandle_t h;
  memcpy(&h, handle, sizeof(h));
  return (int)cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess);
}

NFB_API int nfb_ipc_close(void* ptr) { return (int)cudaIpcCloseMemHandle(ptr); }

NFB_API int nfb_ipc_free(void* ptr) { return (int)cudaFree(ptr); }

NFB_API int nfb_device_synchronize() { return (int)cudaDeviceSynchronize(); }

// Asynchronous copy between any two device addresses of this process (a peer's
// IPC-mapped memory included; the copy engine moves it over NVLink).
NFB_API int nfb_copy_async(void* dst, const void* src, int64_t bytes, void* stream) {
  if (bytes <= 0) return 0;
  return (int)cudaMemcpyAsync(dst, src, (size_t)bytes, cudaMemcpyDefault, (cudaStream_t)stream);
}

// Debug words of the translation units that carry device checks (all zero in release builds).
#ifdef NFB_DEBUG
extern "C" uint32_t nfb_debug_word_ce_rows();
extern "C" uint32_t nfb_debug_word_ce_tc();
extern "C" uint32_t nfb_debug_word_gemm();
extern "C" void nfb_debug_reset_ce_rows();
extern "C" void nfb_debug_reset_ce_tc();
extern "C" void nfb_debug_reset_gemm();
#endif

// First failed device check of the debug build (kDebugCheck << 24 | site), 0 if none or release.
NFB_API uint32_t nfb_debug_status() {
#ifdef NFB_DEBUG
  uint32_t v = nfb_debug_word_ce_rows();
  if (!v) v = nfb_debug_word_ce_tc();
  if (!v) v = nfb_debug_word_gemm();
  return v;
#else
  return 0;
#endif
}

NFB_API void nfb_debug_reset() {
#ifdef NFB_DEBUG
  nfb_debug_reset_ce_rows();
  nfb_debug_reset_ce_tc();
  nfb_debug_reset_gemm();
#endif
}

// 1 in the debug build (device checks compiled in), 0 otherwise.
NFB_API int nfb_is_debug_build() {
#ifdef NFB_DEBUG
  return 1;
#else
  return 0;
#endif
}
