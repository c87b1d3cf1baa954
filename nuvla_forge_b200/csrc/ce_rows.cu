// Cross-entropy row kernels over a materialised logit chunk.
//
// Parity: nuvla_forge/kernels/chunked_ce.py:49-98 (_ce_fwd_bwd): per row, an
// online max / sum-exp sweep gives the log-sum-exp, the row's loss is
// (lse - logit[target]) / count, and a second sweep overwrites the logits in
// place with (softmax - onehot) / count; ignored rows get zero loss and zero
// gradient. Differences: the valid-token count is read from device memory
// (the reference synchronises the host with .item() on every call), rows are
// processed with 16-byte vectors, and the chunk may be bf16 or fp32.
#include "common.cuh"

NFB_DEBUG_TU(ce_rows)

namespace nfb {

struct MS { float m, s; };

__device__ __forceinline__ MS ms_merge(MS a, MS b) {
  const float m = fmaxf(a.m, b.m);
  if (m == -INFINITY) return {m, 0.f};
  return {m, a.s * __expf(a.m - m) + b.s * __expf(b.m - m)};
}

template <typename T, bool VEC>
__global__ void __launch_bounds__(512) ce_rows_kernel(T* logits, int64_t ld, const int64_t* targets,
                                                      int64_t V, int64_t ignore_index, const float* count,
                                                      float* loss_rows) {
  __shared__ MS red[16];
  __shared__ float s_lse;
  const int64_t row = blockIdx.x;
  T* base = logits + row * ld;
  const int64_t tgt = targets[row];
  const float inv = 1.f / fmaxf(*count, 1.f);
  const int64_t nv = VEC ? V / 8 : 0;  // rows not 16-byte aligned take the scalar loops only
  if (tgt == ignore_index) {
    float z[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int64_t i = threadIdx.x; i < nv; i += blockDim.x) store8<T>(base + i * 8, z);
    for (int64_t c = nv * 8 + threadIdx.x; c < V; c += blockDim.x) base[c] = from_f32<T>(0.f);
    if (threadIdx.x == 0) loss_rows[row] = 0.f;
    return;
  }
  // debug build: a label outside [0, V) would read (and later write) past the row
  NFB_DCHECK(tgt >= 0 && tgt < V, 1001, return);
  MS acc{-INFINITY, 0.f};
  for (int64_t i = threadIdx.x; i < nv; i += blockDim.x) {
    float v[8];
    load8<T>(base + i * 8, v);
    float m = v[0];
#pragma unroll
    for (int j = 1; j < 8; ++j) m = fmaxf(m, v[j]);
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 8; ++j) s += __expf(v[j] - m);
    acc = ms_merge(acc, MS{m, s});
  }
  for (int64_t c = nv * 8 + threadIdx.x; c < V; c += blockDim.x) acc = ms_merge(acc, MS{to_f32(base[c]), 1.f});
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    MS other{__shfl_xor_sync(0xffffffffu, acc.m, o), __shfl_xor_sync(0xffffffffu, acc.s, o)};
    acc = ms_merge(acc, other);
  }
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    MS t = red[0];
    for (int w = 1; w < (int)(blockDim.x >> 5); ++w) t = ms_merge(t, red[w]);
    const float lse = t.m + __logf(t.s);
    s_lse = lse;
    loss_rows[row] = (lse - to_f32(base[tgt])) * inv;
  }
  __syncthreads();
  const float lse = s_lse;
  for (int64_t i = threadIdx.x; i < nv; i += blockDim.x) {
    float v[8];
    load8<T>(base + i * 8, v);
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      const float p = __expf(v[j] - lse);
      v[j] = ((i * 8 + j == tgt) ? p - 1.f : p) * inv;
    }
    store8<T>(base + i * 8, v);
  }
  for (int64_t c = nv * 8 + threadIdx.x; c < V; c += blockDim.x) {
    const float p = __expf(to_f32(base[c]) - lse);
    base[c] = from_f32<T>(((c == tgt) ? p - 1.f : p) * inv);
  }
}

__global__ void count_valid_kernel(const int64_t* targets, int64_t n, int64_t ignore_index, float* out) {
  __shared__ int red[32];
  int c = 0;
  for (int64_t i = threadIdx.x; i < n; i += blockDim.x) c += targets[i] != ignore_index;
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) c += __shfl_xor_sync(0xffffffffu, c, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = c;
  __syncthreads();
  if (threadIdx.x == 0) {
    int t = 0;
    for (int w = 0; w < (int)(blockDim.x >> 5); ++w) t += red[w];
    *out = (float)t;
  }
}

}  // namespace nfb

using namespace nfb;

NFB_API int nfb_ce_rows(int dtype, void* logits, int64_t ld, const int64_t* targets, int64_t rows, int64_t V,
                        int64_t ignore_index, const float* count, float* loss_rows, void* stream) {
  if (rows == 0) return 0;
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t es = dtype == kF32 ? 4 : 2;
  const bool vec = ((reinterpret_cast<uintptr_t>(logits) & 15) == 0) && ((ld * es) % 16 == 0);
  if (dtype == kBF16) {
    if (vec) ce_rows_kernel<__nv_bfloat16, true><<<(unsigned)rows, 512, 0, st>>>((__nv_bfloat16*)logits, ld, targets, V, ignore_index, count, loss_rows);
    else ce_rows_kernel<__nv_bfloat16, false><<<(unsigned)rows, 512, 0, st>>>((__nv_bfloat16*)logits, ld, targets, V, ignore_index, count, loss_rows);
  } else if (dtype == kF32) {
    if (vec) ce_rows_kernel<float, true><<<(unsigned)rows, 512, 0, st>>>((float*)logits, ld, targets, V, ignore_index, count, loss_rows);
    else ce_rows_kernel<float, false><<<(unsigned)rows, 512, 0, st>>>((float*)logits, ld, targets, V, ignore_index, count, loss_rows);
  } else {
    return (int)cudaErrorInvalidValue;
  }
  return (int)cudaGetLastError();
}

NFB_API int nfb_count_valid(const int64_t* targets, int64_t n, int64_t ignore_index, float* out, void* stream) {
  count_valid_kernel<<<1, 1024, 0, (cudaStream_t)stream>>>(targets, n, ignore_index, out);
  return (int)cudaGetLastError();
}
