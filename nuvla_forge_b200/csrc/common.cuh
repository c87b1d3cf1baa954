// Shared device helpers for the nuvla_forge_b200 kernels (sm_100a only).
//
// Everything in this library is exported through a C ABI (extern "C") so the
// Python side can call it through ctypes without compiling against torch
// headers. Every entry point returns a cudaError_t (0 == success) and takes the
// CUDA stream it must launch on; none of them allocates memory: scratch space is
// always passed in by the caller.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <type_traits>
#include <cuda_fp16.h>
#include <stdint.h>

#include "nfb_api.h"

#define NFB_API extern "C" __attribute__((visibility("default")))

#ifndef NFB_CHECK_LAUNCH
#define NFB_CHECK_LAUNCH() return (int)cudaGetLastError()
#endif

namespace nfb {

// dtype codes shared with Python (nuvla_forge_b200/_native.py).
enum DType : int { kF32 = 0, kBF16 = 1, kF16 = 2 };

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__nv_bfloat16 v) { return __bfloat162float(v); }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

template <typename T> __device__ __forceinline__ T from_f32(float v);
template <> __device__ __forceinline__ float from_f32<float>(float v) { return v; }
template <> __device__ __forceinline__ __nv_bfloat16 from_f32<__nv_bfloat16>(float v) { return __float2bfloat16_rn(v); }
template <> __device__ __forceinline__ __half from_f32<__half>(float v) { return __float2half_rn(v); }

// 16-byte vector of T (8 x bf16/fp16 or 4 x fp32).
template <typename T> struct Vec16 {
  static constexpr int N = 16 / sizeof(T);
  union { uint4 u; T v[N]; };
};

// A 16-byte vector to / from fp32, two 16-bit elements per 32-bit word at a time: a bf16 is the top
// half of the fp32 with the same value (widening is a shift or a mask), and one packed conversion
// rounds two floats (round to nearest even, as the scalar conversions do), halving the conversion
// instructions of the bandwidth-bound kernels.
template <typename T>
__device__ __forceinline__ void unpack16(const uint4& u, float* out) {
  const uint32_t w[4] = {u.x, u.y, u.z, u.w};
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int k = 0; k < 4; ++k) out[k] = __uint_as_float(w[k]);
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      out[2 * k] = __uint_as_float(w[k] << 16);
      out[2 * k + 1] = __uint_as_float(w[k] & 0xFFFF0000u);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const float2 f = __half22float2(*reinterpret_cast<const __half2*>(&w[k]));
      out[2 * k] = f.x;
      out[2 * k + 1] = f.y;
    }
  }
}

template <typename T>
__device__ __forceinline__ uint4 pack16(const float* in) {
  uint32_t w[4];
  if constexpr (sizeof(T) == 4) {
#pragma unroll
    for (int k = 0; k < 4; ++k) w[k] = __float_as_uint(in[k]);
  } else if constexpr (std::is_same<T, __nv_bfloat16>::value) {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const __nv_bfloat162 h = __floats2bfloat162_rn(in[2 * k], in[2 * k + 1]);
      w[k] = *reinterpret_cast<const uint32_t*>(&h);
    }
  } else {
#pragma unroll
    for (int k = 0; k < 4; ++k) {
      const __half2 h = __floats2half2_rn(in[2 * k], in[2 * k + 1]);
      w[k] = *reinterpret_cast<const uint32_t*>(&h);
    }
  }
  return make_uint4(w[0], w[1], w[2], w[3]);
}

template <typename T>
__device__ __forceinline__ void load16(const T* p, float* out) {
  unpack16<T>(*reinterpret_cast<const uint4*>(p), out);
}

template <typename T>
__device__ __forceinline__ void store16(T* p, const float* in) {
  *reinterpret_cast<uint4*>(p) = pack16<T>(in);
}

// Streaming (evict-first) variants for data that is touched exactly once.
template <typename T>
__device__ __forceinline__ void load16_stream(const T* p, float* out) {
  unpack16<T>(__ldcs(reinterpret_cast<const uint4*>(p)), out);
}

template <typename T>
__device__ __forceinline__ void store16_stream(T* p, const float* in) {
  __stcs(reinterpret_cast<uint4*>(p), pack16<T>(in));
}

// 8 consecutive elements of T (one 16-byte vector for 2-byte types, two for fp32).
template <typename T>
__device__ __forceinline__ void load8(const T* p, float* out) {
  if constexpr (sizeof(T) == 2) load16<T>(p, out);
  else { load16<T>(p, out); load16<T>(p + 4, out + 4); }
}
template <typename T>
__device__ __forceinline__ void store8(T* p, const float* in) {
  if constexpr (sizeof(T) == 2) store16<T>(p, in);
  else { store16<T>(p, in); store16<T>(p + 4, in + 4); }
}
template <typename T>
__device__ __forceinline__ void load8_stream(const T* p, float* out) {
  if constexpr (sizeof(T) == 2) load16_stream<T>(p, out);
  else { load16_stream<T>(p, out); load16_stream<T>(p + 4, out + 4); }
}
// Round 8 floats through T (so later math sees exactly what was stored).
template <typename T>
__device__ __forceinline__ void round8(float* v) {
#pragma unroll
  for (int j = 0; j < 8; ++j) v[j] = to_f32(from_f32<T>(v[j]));
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
  return v;
}

__device__ __forceinline__ float sigmoidf_fast(float x) {
  return __fdividef(1.0f, 1.0f + __expf(-x));
}

// Nanosecond global timer, used to bound every spin-wait in the library.
__device__ __forceinline__ uint64_t globaltimer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// System-scope release store / acquire load on 32-bit flags living in memory
// that other GPUs read and write through NVLink peer mappings.
__device__ __forceinline__ void st_release_sys(uint32_t* p, uint32_t v) {
  asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
__device__ __forceinline__ uint32_t ld_acquire_sys(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}
__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Error codes written into a caller-provided device status word when a bounded
// wait gives up. The host reads the word after the step and raises.
enum Status : uint32_t {
  kOk = 0,
  kTimeoutBarrier = 1,
  kTimeoutFlag = 2,
  kBadArgument = 3,
};

__device__ __forceinline__ void set_status(uint32_t* status, uint32_t code, uint32_t where) {
  if (status) {
    atomicCAS(status, 0u, (code << 24) | (where & 0xFFFFFFu));
  }
}

// ---------------------------------------------------------------------------
// Debug build (-DNFB_DEBUG, libnfb200_debug.so): device-side bounds and argument checks that a
// host cannot make cheaply (label values, peer addresses, derived indices). A failed check
// records (kDebugCheck << 24 | site) in this translation unit's debug word -- the first failure
// wins -- and the guarded access is skipped; no trap, so the context stays usable and the host
// reads the word with nfb_debug_status(). In release builds NFB_DCHECK compiles to nothing.
// NFB_DEBUG_TU(name) defines the word and its host accessors once per .cu file.
// ---------------------------------------------------------------------------
constexpr uint32_t kDebugCheck = 4;

#ifdef NFB_DEBUG
#define NFB_DEBUG_TU(name)                                                                          \
  static __device__ uint32_t g_nfb_dbg_word;                                                        \
  __device__ __forceinline__ void nfb_dbg_fail(uint32_t site) {                                     \
    atomicCAS(&g_nfb_dbg_word, 0u, (nfb::kDebugCheck << 24) | (site & 0xFFFFFFu));                  \
  }                                                                                                 \
  extern "C" __attribute__((visibility("default"))) uint32_t nfb_debug_word_##name() {             \
    uint32_t v = 0;                                                                                 \
    cudaMemcpyFromSymbol(&v, g_nfb_dbg_word, sizeof(v));                                            \
    return v;                                                                                       \
  }                                                                                                 \
  extern "C" __attribute__((visibility("default"))) void nfb_debug_reset_##name() {                \
    const uint32_t z = 0;                                                                           \
    cudaMemcpyToSymbol(g_nfb_dbg_word, &z, sizeof(z));                                              \
  }
// Evaluate `cond`; if false, record `site` and run `on_fail` (e.g. `return` or `continue`).
#define NFB_DCHECK(cond, site, on_fail) \
  do {                                  \
    if (!(cond)) {                      \
      nfb_dbg_fail(site);               \
      on_fail;                          \
    }                                   \
  } while (0)
#else
#define NFB_DEBUG_TU(name)
#define NFB_DCHECK(cond, site, on_fail) \
  do {                                  \
  } while (0)
#endif

// Spin until *flag >= target (wrap-safe comparison of epochs), at most
// timeout_ns. Returns true on success.
__device__ __forceinline__ bool wait_flag_geq(const uint32_t* flag, uint32_t target, uint64_t timeout_ns) {
  uint64_t t0 = globaltimer_ns();
  while (true) {
    uint32_t v = ld_acquire_sys(flag);
    if ((int32_t)(v - target) >= 0) return true;
    if (globaltimer_ns() - t0 > timeout_ns) return false;
    __nanosleep(64);
  }
}

}  // namespace nfb
