// Hardware characterisation: throughput of back-to-back tcgen05.mma instructions by shape and
// operand source (one CTA per SM, all SMs busy). The attention kernels' MMAs are small (N = 64 or
// 128, K = 16 per instruction), and whether an instruction runs at the tensor core's full rate
// depends on its shape and on where A comes from; this measures it instead of assuming it.
// Modes: 0 = A and B from shared memory (K-major), 1 = B MN-major, 2 = A from TMEM, B MN-major.
// Operands are zero-filled shared memory; every wait is bounded (clock64) and reports through out[1].
#include "tc_gemm.cuh"

namespace nfb {
namespace mmaprobe {

using namespace nfb::tc;

template <int N, int MODE>
__global__ void __launch_bounds__(128, 1) mma_rate_kernel(int iters, unsigned long long* out) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* s = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  __shared__ uint64_t bar;
  __shared__ uint32_t tbase;
  for (int i = threadIdx.x; i < 65536 / 4; i += blockDim.x) reinterpret_cast<uint32_t*>(s)[i] = 0u;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
  }
  if (threadIdx.x < 32) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], 512;" ::"r"(smem_u32(&tbase)) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t t = tbase;
  if (threadIdx.x == 0) {
    constexpr uint32_t id = idesc_bf16(128, N, false, MODE != 0);
    const uint64_t da = sw128_desc(smem_u32(s));
    const uint64_t db = MODE == 0 ? sw128_desc(smem_u32(s + 32768)) : sw128_mn_desc(smem_u32(s + 32768));
    const long long c0 = clock64();
    for (int i = 0; i < iters; ++i) {
      const uint32_t acc = i > 0 ? 1u : 0u;
      if (MODE == 2) {
        asm volatile(
            "{\n\t.reg .pred p;\n\tsetp.ne.b32 p, %4, 0;\n\t"
            "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
            ::"r"(t), "r"(t + 256u + (uint32_t)((i & 7) * 8)), "l"(db + (uint64_t)(((i & 3) * 2048) >> 4)), "r"(id),
              "r"(acc)
            : "memory");
      } else {
        umma_bf16(t, da + (uint64_t)(((i & 3) * 32) >> 4), db + (uint64_t)(((i & 3) * (MODE ? 2048 : 32)) >> 4), id,
                  acc);
      }
    }
    umma_commit(&bar);
    uint32_t ok = 0;
    while (!ok && clock64() - c0 < 4000000000ll) ok = mbar_try_wait(&bar, 0u) ? 1u : 0u;
    const long long c1 = clock64();
    if (blockIdx.x == 0) {
      out[0] = (unsigned long long)(c1 - c0);
      out[1] = ok;
    }
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if (threadIdx.x < 32) asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, 512;" ::"r"(t) : "memory");
}

template <int N, int MODE>
static int launch(int iters, unsigned long long* out, int sms, cudaStream_t st) {
  const int smem = 200 * 1024;   // keeps one CTA (and its 512 TMEM columns) per SM
  cudaError_t e = cudaFuncSetAttribute(mma_rate_kernel<N, MODE>, cudaFuncAttributeMaxDynamicSharedMemorySize, smem);
  if (e != cudaSuccess) return (int)e;
  mma_rate_kernel<N, MODE><<<sms, 128, smem, st>>>(iters, out);
  return (int)cudaGetLastError();
}

}  // namespace mmaprobe
}  // namespace nfb

using namespace nfb::mmaprobe;

// out (device, 2 x uint64): SM cycles for `iters` back-to-back M128 x n x K16 bf16 MMAs issued by
// CTA 0 (issue of the first to completion of the last), and 1 if the completion was observed.
// mode: 0 both operands K-major in shared memory, 1 B MN-major, 2 A from TMEM and B MN-major.
NFB_API int nfb_mma_rate(int mode, int n, int iters, unsigned long long* out, int sms, void* stream) {
  cudaStream_t st = (cudaStream_t)stream;
  if (iters < 1 || sms < 1) return (int)cudaErrorInvalidValue;
  if (mode == 0 && n == 64) return launch<64, 0>(iters, out, sms, st);
  if (mode == 0 && n == 128) return launch<128, 0>(iters, out, sms, st);
  if (mode == 0 && n == 256) return launch<256, 0>(iters, out, sms, st);
  if (mode == 1 && n == 64) return launch<64, 1>(iters, out, sms, st);
  if (mode == 1 && n == 128) return launch<128, 1>(iters, out, sms, st);
  if (mode == 2 && n == 64) return launch<64, 2>(iters, out, sms, st);
  if (mode == 2 && n == 128) return launch<128, 2>(iters, out, sms, st);
  return (int)cudaErrorInvalidValue;
}
