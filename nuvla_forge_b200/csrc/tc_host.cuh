// Host-side helpers shared by the tcgen05 GEMM launchers: TMA tensor maps
// (cuTensorMapEncodeTiled through the runtime's driver entry point, so no
// libcuda link is needed), SM count and the tile shape.
#pragma once

#include <cudaTypedefs.h>

#include "tc_gemm.cuh"

namespace nfb {
namespace tc {

static PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;

static int get_encode() {
  if (g_encode) return 0;
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q);
  if (e != cudaSuccess || q != cudaDriverEntryPointSuccess || fn == nullptr) return (int)cudaErrorNotSupported;
  g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
  return 0;
}

// Make the context of the device that owns `p` current in this host thread. Threads that torch
// starts (the autograd engine's device threads, Python threads) may have no current context;
// encoding a tensor map then fails, so every tensor-map builder binds the operand's device first.
static int bind_device_of(const void* p) {
  cudaPointerAttributes a;
  cudaError_t e = cudaPointerGetAttributes(&a, p);
  if (e != cudaSuccess) {
    cudaGetLastError();   // not a pointer the runtime knows: leave the thread's context alone
    return 0;
  }
  if (a.type != cudaMemoryTypeDevice && a.type != cudaMemoryTypeManaged) return 0;
  e = cudaSetDevice(a.device);
  return e == cudaSuccess ? 0 : (int)e;
}

// 2-D bf16 row-major [rows, cols] with row stride `ld` elements; box = box_rows x 64 columns, 128B swizzle.
static int make_tmap(CUtensorMap* m, const void* base, int64_t rows, int64_t cols, int64_t ld, int box_rows) {
  int rc = get_encode();
  if (rc) return rc;
  rc = bind_device_of(base);
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || ((ld * 2) % 16) || cols % 8) return (int)cudaErrorInvalidValue;
  cuuint64_t dims[2] = {(cuuint64_t)cols, (cuuint64_t)rows};
  cuuint64_t strides[1] = {(cuuint64_t)(ld * 2)};
  cuuint32_t box[2] = {(cuuint32_t)BK, (cuuint32_t)box_rows};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

static int sm_count() {
  int dev = 0, n = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
  return n;
}

static GemmShape make_shape(int M, int N, int K) {
  GemmShape s;
  s.M = M; s.N = N; s.K = K;
  s.m_tiles = (M + BM - 1) / BM;
  s.n_tiles = (N + BN - 1) / BN;
  s.k_tiles = (K + BK - 1) / BK;
  s.group = 8;
  return s;
}

}  // namespace tc
}  // namespace nfb
