// Flat-buffer optimizer and gradient kernels.
//
// The training runtime keeps every trainable parameter of a replica (DDP) or
// of a shard (FSDP) in ONE contiguous fp32 master buffer with matching fp32
// gradient, exp_avg and exp_avg_sq buffers, and the bf16 weights the model
// computes with are views of one contiguous bf16 buffer. So the whole
// optimizer step is one launch instead of torch's multi-tensor chunking, and
// the global gradient norm is one deterministic reduction whose result stays
// on the device (no host sync for clip_grad_norm_).
//
// AdamW math is the decoupled-weight-decay Adam of Loshchilov & Hutter, in
// the same order as torch.optim.AdamW (which the reference uses with
// fused=True, nuvla_forge/train.py:170-173):
//   p *= 1 - lr*wd;  m = b1*m + (1-b1)*g;  v = b2*v + (1-b2)*g^2
//   p -= (lr / bc1) * m / (sqrt(v) / sqrt(bc2) + eps)
// Clipping follows torch.nn.utils.clip_grad_norm_: coef = min(1, max_norm / (norm + 1e-6)).
#include "common.cuh"

namespace nfb {

struct AdamArgs {
  float* param; const float* grad; float* m; float* v;
  void* param_lp;          // optional low-precision copy of param (bf16), may be null
  int64_t n;
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, grad_scale;
  const float* norm2;      // optional device norm^2 for clipping
  float max_norm;
};

__device__ __forceinline__ float clip_coef(const float* norm2, float max_norm) {
  if (norm2 == nullptr || max_norm <= 0.f) return 1.f;
  float c = max_norm / (sqrtf(*norm2) + 1e-6f);
  return c < 1.f ? c : 1.f;
}

__device__ __forceinline__ void adam_one(float& p, float g, float& m, float& v, const AdamArgs& a) {
  p = p * (1.f - a.lr * a.wd);
  m = a.beta1 * m + (1.f - a.beta1) * g;
  v = a.beta2 * v + (1.f - a.beta2) * g * g;
  const float denom = sqrtf(v) / a.bc2_sqrt + a.eps;
  p = p - (a.lr / a.bc1) * (m / denom);
}

__global__ void __launch_bounds__(256) adamw_kernel(AdamArgs a) {
  const float coef = clip_coef(a.norm2, a.max_norm) * a.grad_scale;
  const int64_t nv = a.n / 4;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    float4 p = reinterpret_cast<float4*>(a.param)[i];
    float4 g = __ldcs(reinterpret_cast<const float4*>(a.grad) + i);
    float4 m = reinterpret_cast<float4*>(a.m)[i];
    float4 v = reinterpret_cast<float4*>(a.v)[i];
    adam_one(p.x, g.x * coef, m.x, v.x, a);
    adam_one(p.y, g.y * coef, m.y, v.y, a);
    adam_one(p.z, g.z * coef, m.z, v.z, a);
    adam_one(p.w, g.w * coef, m.w, v.w, a);
    reinterpret_cast<float4*>(a.param)[i] = p;
    reinterpret_cast<float4*>(a.m)[i] = m;
    reinterpret_cast<float4*>(a.v)[i] = v;
    if (a.param_lp) {
      __nv_bfloat162 lo = __floats2bfloat162_rn(p.x, p.y), hi = __floats2bfloat162_rn(p.z, p.w);
      uint2 u; u.x = *reinterpret_cast<uint32_t*>(&lo); u.y = *reinterpret_cast<uint32_t*>(&hi);
      reinterpret_cast<uint2*>(a.param_lp)[i] = u;
    }
  }
  for (int64_t i = nv * 4 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < a.n; i += (int64_t)gridDim.x * blockDim.x) {
    float p = a.param[i], m = a.m[i], v = a.v[i];
    adam_one(p, a.grad[i] * coef, m, v, a);
    a.param[i] = p; a.m[i] = m; a.v[i] = v;
    if (a.param_lp) reinterpret_cast<__nv_bfloat16*>(a.param_lp)[i] = __float2bfloat16_rn(p);
  }
}

// Deterministic sum of squares: CTA partials then the last CTA (ticket) sums
// them in index order. partials: [grid] floats; ticket: one zeroed uint32 that
// the kernel leaves zeroed. Result written to *out (fp32), times `scale`^2.
template <typename T>
__global__ void __launch_bounds__(512) sumsq_kernel(const T* __restrict__ x, int64_t n, float scale,
                                                    float* partials, uint32_t* ticket, float* out, int accumulate) {
  __shared__ float red[32];
  __shared__ uint32_t s_t;
  float s = 0.f;
  constexpr int PER = 16 / sizeof(T);
  const int64_t nv = n / PER;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    float v[PER];
    load16<T>(x + i * PER, v);
#pragma unroll
    for (int j = 0; j < PER; ++j) s += v[j] * v[j];
  }
  for (int64_t i = nv * PER + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = to_f32(x[i]);
    s += v * v;
  }
  s = warp_sum(s);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) {
      partials[blockIdx.x] = t;
      __threadfence();
      s_t = atomicAdd(ticket, 1u);
    }
  }
  __syncthreads();
  if (s_t != gridDim.x - 1) return;
  __threadfence();
  if (threadIdx.x == 0) {
    float tot = 0.f;
    for (unsigned b = 0; b < gridDim.x; ++b) tot += __ldcg(partials + b);
    tot *= scale * scale;
    *out = accumulate ? (*out + tot) : tot;
    *ticket = 0u;
  }
}

// dst(fp32) = src * scale (overwrite) or dst += src * scale.
template <typename T>
__global__ void __launch_bounds__(256) accum_kernel(float* __restrict__ dst, const T* __restrict__ src, int64_t n,
                                                    float scale, int overwrite) {
  constexpr int PER = 16 / sizeof(T);
  const int64_t nv = n / PER;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nv; i += (int64_t)gridDim.x * blockDim.x) {
    float v[PER];
    load16_stream<T>(src + i * PER, v);
#pragma unroll
    for (int j = 0; j < PER; j += 4) {
      float4* d = reinterpret_cast<float4*>(dst + i * PER + j);
      float4 o = overwrite ? make_float4(0.f, 0.f, 0.f, 0.f) : *d;
      o.x += v[j] * scale; o.y += v[j + 1] * scale; o.z += v[j + 2] * scale; o.w += v[j + 3] * scale;
      *d = o;
    }
  }
  for (int64_t i = nv * PER + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x) {
    float v = to_f32(src[i]) * scale;
    dst[i] = overwrite ? v : dst[i] + v;
  }
}

template <typename TI, typename TO>
__global__ void __launch_bounds__(256) cast_kernel(TO* __restrict__ dst, const TI* __restrict__ src, int64_t n, float scale) {
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n; i += (int64_t)gridDim.x * blockDim.x)
    dst[i] = from_f32<TO>(to_f32(src[i]) * scale);
}

static int grid_for(int64_t work, int threads, int per_sm) {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  int64_t b = (work + threads - 1) / threads;
  int64_t cap = (int64_t)sms * per_sm;
  if (b > cap) b = cap;
  return (int)(b < 1 ? 1 : b);
}

}  // namespace nfb

using namespace nfb;

NFB_API int nfb_adamw_flat(float* param, const float* grad, float* m, float* v, void* param_bf16, int64_t n,
                           float lr, float beta1, float beta2, float eps, float wd, int64_t step,
                           float grad_scale, const float* norm2, float max_norm, void* stream) {
  if (n == 0) return 0;
  if ((reinterpret_cast<uintptr_t>(param) | reinterpret_cast<uintptr_t>(grad) | reinterpret_cast<uintptr_t>(m) |
       reinterpret_cast<uintptr_t>(v)) & 15) return (int)cudaErrorInvalidValue;
  if (param_bf16 && (reinterpret_cast<uintptr_t>(param_bf16) & 7)) return (int)cudaErrorInvalidValue;
  AdamArgs a;
  a.param = param; a.grad = grad; a.m = m; a.v = v; a.param_lp = param_bf16; a.n = n;
  a.lr = lr; a.beta1 = beta1; a.beta2 = beta2; a.eps = eps; a.wd = wd;
  a.bc1 = 1.f - powf(beta1, (float)step);
  a.bc2_sqrt = sqrtf(1.f - powf(beta2, (float)step));
  a.grad_scale = grad_scale; a.norm2 = norm2; a.max_norm = max_norm;
  adamw_kernel<<<grid_for(n / 4 + 1, 256, 8), 256, 0, (cudaStream_t)stream>>>(a);
  return (int)cudaGetLastError();
}

// Number of partial slots nfb_sumsq needs.
NFB_API int nfb_sumsq_slots() {
  int dev = 0, sms = 148;
  cudaGetDevice(&dev);
  cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
  return sms * 2;
}

NFB_API int nfb_sumsq(int dtype, const void* x, int64_t n, float scale, float* partials, uint32_t* ticket,
                      float* out, int accumulate, void* stream) {
  const int grid = nfb_sumsq_slots();
  cudaStream_t st = (cudaStream_t)stream;
  if (reinterpret_cast<uintptr_t>(x) & 15) return (int)cudaErrorInvalidValue;
  if (dtype == kF32) sumsq_kernel<float><<<grid, 512, 0, st>>>((const float*)x, n, scale, partials, ticket, out, accumulate);
  else if (dtype == kBF16) sumsq_kernel<__nv_bfloat16><<<grid, 512, 0, st>>>((const __nv_bfloat16*)x, n, scale, partials, ticket, out, accumulate);
  else return (int)cudaErrorInvalidValue;
  return (int)cudaGetLastError();
}

NFB_API int nfb_accum(int src_dtype, float* dst, const void* src, int64_t n, float scale, int overwrite, void* stream) {
  if (n == 0) return 0;
  if ((reinterpret_cast<uintptr_t>(dst) | reinterpret_cast<uintptr_t>(src)) & 15) return (int)cudaErrorInvalidValue;
  cudaStream_t st = (cudaStream_t)stream;
  const int g = grid_for(n / 8 + 1, 256, 8);
  if (src_dtype == kBF16) accum_kernel<__nv_bfloat16><<<g, 256, 0, st>>>(dst, (const __nv_bfloat16*)src, n, scale, overwrite);
  else if (src_dtype == kF16) accum_kernel<__half><<<g, 256, 0, st>>>(dst, (const __half*)src, n, scale, overwrite);
  else if (src_dtype == kF32) accum_kernel<float><<<g, 256, 0, st>>>(dst, (const float*)src, n, scale, overwrite);
  else return (int)cudaErrorInvalidValue;
  return (int)cudaGetLastError();
}

NFB_API int nfb_cast(int src_dtype, int dst_dtype, void* dst, const void* src, int64_t n, float scale, void* stream) {
  if (n == 0) return 0;
  cudaStream_t st = (cudaStream_t)stream;
  const int g = grid_for(n, 256, 8);
  if (src_dtype == kF32 && dst_dtype == kBF16) cast_kernel<float, __nv_bfloat16><<<g, 256, 0, st>>>((__nv_bfloat16*)dst, (const float*)src, n, scale);
  else if (src_dtype == kBF16 && dst_dtype == kF32) cast_kernel<__nv_bfloat16, float><<<g, 256, 0, st>>>((float*)dst, (const __nv_bfloat16*)src, n, scale);
  else if (src_dtype == kF32 && dst_dtype == kF32) cast_kernel<float, float><<<g, 256, 0, st>>>((float*)dst, (const float*)src, n, scale);
  else if (src_dtype == kBF16 && dst_dtype == kBF16) cast_kernel<__nv_bfloat16, __nv_bfloat16><<<g, 256, 0, st>>>((__nv_bfloat16*)dst, (const __nv_bfloat16*)src, n, scale);
  else return (int)cudaErrorInvalidValue;
  return (int)cudaGetLastError();
}
