// On-device image preparation: uint8 camera frames -> normalised bf16.
//
// Parity: nuvla_forge/data/loader.py:186-196 (normalise_images), which runs
// four eager elementwise kernels plus two small host->device constructions per
// call. Two kernels here:
//
// * nfb_image_normalize: [.., 3, H, W] uint8 -> same layout in bf16/fp16/fp32,
//   out = (v / 255 - mean[c]) / std[c]; one pass, one launch.
// * nfb_image_patchify: [n_img, H, W, 3] uint8 (HWC, as the loader produces
//   it, so the host never transposes) -> [n_img, (H/p)*(W/p), Kpad] bf16 patch
//   rows in (c, ky, kx) order, i.e. exactly the rows that multiply a
//   Conv2d-shaped [D, 3, p, p] patch-embedding weight. Columns K..Kpad are
//   zero so the patch GEMM's K stays a multiple of 8. One CTA owns one strip
//   of p image rows: the strip is contiguous in HWC, so it is read once with
//   16-byte loads into shared memory and the strip's patches are written out
//   contiguously (p = 14 / 16 with 16-byte image rows: the tiled kernel below;
//   other shapes: a per-element gather through a column table).
#include "common.cuh"

namespace nfb {

struct NormConst { float scale[3]; float bias[3]; };

template <typename TO>
__global__ void image_normalize_kernel(const uint8_t* __restrict__ in, TO* __restrict__ out,
                                       int64_t n, int64_t hw, NormConst k) {
  // 16 bytes per thread per step
  const int64_t nvec = n / 16;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < nvec; i += (int64_t)gridDim.x * blockDim.x) {
    uint4 u = __ldcs(reinterpret_cast<const uint4*>(in) + i);
    const uint8_t* b = reinterpret_cast<const uint8_t*>(&u);
    float o[16];
#pragma unroll
    for (int j = 0; j < 16; ++j) {
      const int64_t e = i * 16 + j;
      const int c = (int)((e / hw) % 3);
      o[j] = (float)b[j] * k.scale[c] + k.bias[c];
    }
    constexpr int PER = 16 / sizeof(TO);
#pragma unroll
    for (int j = 0; j < 16; j += PER) store16<TO>(out + i * 16 + j, o + j);
  }
  // tail
  for (int64_t e = nvec * 16 + (int64_t)blockIdx.x * blockDim.x + threadIdx.x; e < n; e += (int64_t)gridDim.x * blockDim.x) {
    const int c = (int)((e / hw) % 3);
    out[e] = from_f32<TO>((float)in[e] * k.scale[c] + k.bias[c]);
  }
}

template <typename TO>
__global__ void __launch_bounds__(256) image_patchify_kernel(const uint8_t* __restrict__ in, TO* __restrict__ out,
                                                             int H, int W, int p, int kpad, NormConst k) {
  extern __shared__ __align__(16) uint8_t smem[];
  // [kpad] offsets of each patch-row column inside the strip (or -1 for the zero
  // padding), computed once per CTA so the hot loop has no divisions; then the strip.
  int* koff = reinterpret_cast<int*>(smem);
  uint8_t* strip = smem + ((kpad * 4 + 15) / 16) * 16;
  const int rows_of_patches = H / p;
  const int64_t img = blockIdx.x / rows_of_patches;
  const int py = blockIdx.x % rows_of_patches;
  const int64_t strip_bytes = (int64_t)p * W * 3;
  const uint8_t* src = in + img * (int64_t)H * W * 3 + (int64_t)py * strip_bytes;
  if ((reinterpret_cast<uintptr_t>(src) & 15) == 0 && (strip_bytes & 15) == 0) {
    for (int64_t i = threadIdx.x; i < strip_bytes / 16; i += blockDim.x)
      reinterpret_cast<uint4*>(strip)[i] = __ldcs(reinterpret_cast<const uint4*>(src) + i);
  } else {
    for (int64_t i = threadIdx.x; i < strip_bytes; i += blockDim.x) strip[i] = src[i];
  }
  const int K = 3 * p * p;
  const int pp = p * p;
  for (int kk = threadIdx.x; kk < kpad; kk += blockDim.x) {
    if (kk < K) {
      const int c = kk / pp;
      const int rem = kk - c * pp;
      const int ky = rem / p;
      const int kx = rem - ky * p;
      koff[kk] = ((ky * W + kx) * 3 + c) | (c << 28);
    } else {
      koff[kk] = -1;
    }
  }
  __syncthreads();
  const int pw = W / p;
  TO* dst = out + (img * rows_of_patches + py) * (int64_t)pw * kpad;
  constexpr int PER = 16 / sizeof(TO);
  const int vec_per_patch = kpad / PER;
  for (int v = threadIdx.x; v < pw * vec_per_patch; v += blockDim.x) {
    const int px = v / vec_per_patch;
    const int k0 = (v % vec_per_patch) * PER;
    float o[PER];
#pragma unroll
    for (int j = 0; j < PER; ++j) {
      const int e = koff[k0 + j];
      if (e >= 0) {
        const int c = e >> 28;
        const float val = (float)strip[(e & 0x0FFFFFFF) + px * p * 3];
        o[j] = val * k.scale[c] + k.bias[c];
      } else {
        o[j] = 0.f;
      }
    }
    store16<TO>(dst + (int64_t)px * kpad + k0, o);
  }
}

constexpr int kPatchGroup = 16;

// Two floats as one packed pair of 2-byte values (round to nearest even).
template <typename TO>
__device__ __forceinline__ uint32_t pack_pair(float a, float b) {
  if constexpr (std::is_same<TO, __nv_bfloat16>::value) {
    const __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  } else {
    const __half2 h = __floats2half2_rn(a, b);
    return *reinterpret_cast<const uint32_t*>(&h);
  }
}

// Tiled variant for even patch sizes with 16-byte image rows (the ViT's 448 x 448, p = 14). The
// strip is copied into shared memory with each image row padded by 16 bytes; a task is one image
// row (ky) of one patch (px): 3p consecutive bytes, read as aligned 32-bit words and realigned with
// funnel shifts, written as bf16 pairs into a shared-memory copy of the strip's patch rows; then the
// CTA writes its patch rows (contiguous in the output) with 16-byte stores, 16 patches at a time. A warp's 32 tasks are
// 8 patches x 4 image rows and patch rows sit 2 * kpad + 16 bytes apart, so for p = 14 the pair
// stores of a warp fall in 32 different banks (the per-element gather from one unpadded strip
// was bound by bank conflicts).
template <typename TO, int P>
__global__ void __launch_bounds__(256) image_patchify_tiled_kernel(const uint8_t* __restrict__ in,
                                                                   TO* __restrict__ out, int H, int W,
                                                                   int kpad, NormConst k) {
  static_assert(P % 2 == 0 && sizeof(TO) == 2, "even patch size, 2-byte output");
  constexpr int K = 3 * P * P;
  constexpr int RUN = 3 * P;                 // bytes of one image row of one patch
  constexpr int NWORD = (RUN + 3 + 3) / 4;   // aligned words that cover the run at any offset
  constexpr int kGroup = kPatchGroup;        // patch rows staged at a time
  extern __shared__ __align__(16) uint8_t smem[];
  const int row_bytes = W * 3;               // multiple of 16 (checked by the launcher)
  const int rs = row_bytes + 16;             // padded image row in shared memory
  const int os = kpad * 2 + 16;              // padded patch row in shared memory
  uint8_t* strip = smem;
  uint8_t* rows = smem + P * rs;
  const int rows_of_patches = H / P, pw = W / P;
  const int64_t img = blockIdx.x / rows_of_patches;
  const int py = blockIdx.x % rows_of_patches;
  const uint4* src = reinterpret_cast<const uint4*>(in + (img * H + (int64_t)py * P) * row_bytes);
  const int cpr_in = row_bytes / 16, nin = P * cpr_in;
  constexpr int kLd = 5;
  for (int base = threadIdx.x; base < nin; base += kLd * blockDim.x) {
    uint4 v[kLd];
#pragma unroll
    for (int u = 0; u < kLd; ++u) {
      const int i = base + u * blockDim.x;
      if (i < nin) v[u] = __ldcs(src + i);
    }
#pragma unroll
    for (int u = 0; u < kLd; ++u) {
      const int i = base + u * blockDim.x;
      if (i < nin) *reinterpret_cast<uint4*>(strip + (i / cpr_in) * rs + (i % cpr_in) * 16) = v[u];
    }
  }
  // zero padding columns K..kpad of every patch row
  const int nstage = pw < kGroup ? pw : kGroup;
  for (int i = threadIdx.x; i < nstage * (kpad - K); i += blockDim.x) {
    const int r = i / (kpad - K), c = K + i % (kpad - K);
    *reinterpret_cast<TO*>(rows + r * os + c * 2) = from_f32<TO>(0.f);
  }
  __syncthreads();
  // the strip's patches in groups of kGroup (staging for one group only keeps more CTAs resident)
  const int cpr_out = kpad / 8, kyb = (P + 3) / 4;
  TO* strip_out = out + ((img * rows_of_patches + py) * (int64_t)pw) * kpad;
  for (int g0 = 0; g0 < pw; g0 += kGroup) {
    const int ng = pw - g0 < kGroup ? pw - g0 : kGroup;
    const int pxb = (ng + 7) / 8;
    for (int t = threadIdx.x; t < pxb * kyb * 32; t += blockDim.x) {
      const int blk = t >> 5;
      const int r = (blk % pxb) * 8 + (t & 7);          // patch row within the group
      const int ky = (blk / pxb) * 4 + ((t >> 3) & 3);
      if (r >= ng || ky >= P) continue;
      const int b0 = ky * rs + (g0 + r) * RUN;
      const uint32_t* w = reinterpret_cast<const uint32_t*>(strip) + (b0 >> 2);
      const uint32_t sh = (uint32_t)(b0 & 3) * 8;
      uint32_t wv[NWORD];
#pragma unroll
      for (int i = 0; i < NWORD; ++i) wv[i] = w[i];
      uint32_t v[(RUN + 3) / 4];
#pragma unroll
      for (int i = 0; i < (RUN + 3) / 4; ++i) v[i] = __funnelshift_r(wv[i], wv[i + 1], sh);
      uint8_t* dst = rows + r * os + ky * P * 2;
#pragma unroll
      for (int c = 0; c < 3; ++c) {
#pragma unroll
        for (int kx = 0; kx < P; kx += 2) {
          const int t0 = kx * 3 + c, t1 = (kx + 1) * 3 + c;
          const float f0 = (float)((v[t0 >> 2] >> (8 * (t0 & 3))) & 0xFFu);
          const float f1 = (float)((v[t1 >> 2] >> (8 * (t1 & 3))) & 0xFFu);
          *reinterpret_cast<uint32_t*>(dst + (c * P * P + kx) * 2) =
              pack_pair<TO>(fmaf(f0, k.scale[c], k.bias[c]), fmaf(f1, k.scale[c], k.bias[c]));
        }
      }
    }
    __syncthreads();
    uint4* dst = reinterpret_cast<uint4*>(strip_out + (int64_t)g0 * kpad);
    for (int i = threadIdx.x; i < ng * cpr_out; i += blockDim.x)
      dst[i] = *reinterpret_cast<const uint4*>(rows + (i / cpr_out) * os + (i % cpr_out) * 16);
    if (g0 + kGroup < pw) __syncthreads();  // the next group reuses the staging rows
  }
}

static NormConst make_const(const float* mean, const float* std) {
  NormConst k;
  for (int c = 0; c < 3; ++c) {
    k.scale[c] = 1.0f / (255.0f * std[c]);
    k.bias[c] = -mean[c] / std[c];
  }
  return k;
}

}  // namespace nfb

using namespace nfb;

// in: uint8 [..., 3, H, W] contiguous, n elements; out dtype 0 f32, 1 bf16, 2 f16.
NFB_API int nfb_image_normalize(int out_dtype, const void* in, void* out, int64_t n, int64_t hw,
                                const float* mean, const float* std, void* stream) {
  if (n == 0) return 0;
  if ((reinterpret_cast<uintptr_t>(in) & 15) || (reinterpret_cast<uintptr_t>(out) & 15)) return (int)cudaErrorInvalidValue;
  NormConst k = make_const(mean, std);
  cudaStream_t st = (cudaStream_t)stream;
  int64_t blocks = (n / 16 + 255) / 256;
  if (blocks > 148 * 16) blocks = 148 * 16;
  if (blocks < 1) blocks = 1;
  const uint8_t* src = (const uint8_t*)in;
  if (out_dtype == kBF16) image_normalize_kernel<__nv_bfloat16><<<(int)blocks, 256, 0, st>>>(src, (__nv_bfloat16*)out, n, hw, k);
  else if (out_dtype == kF16) image_normalize_kernel<__half><<<(int)blocks, 256, 0, st>>>(src, (__half*)out, n, hw, k);
  else if (out_dtype == kF32) image_normalize_kernel<float><<<(int)blocks, 256, 0, st>>>(src, (float*)out, n, hw, k);
  else return (int)cudaErrorInvalidValue;
  return (int)cudaGetLastError();
}

// in: uint8 [n_img, H, W, 3]; out: [n_img, (H/p)*(W/p), kpad]; kpad % 8 == 0, kpad >= 3*p*p.
NFB_API int nfb_image_patchify(int out_dtype, const void* in, void* out, int64_t n_img, int H, int W, int p,
                               int kpad, const float* mean, const float* std, void* stream) {
  if (n_img == 0) return 0;
  if (H % p || W % p || kpad < 3 * p * p || kpad % 8) return (int)cudaErrorInvalidValue;
  NormConst k = make_const(mean, std);
  cudaStream_t st = (cudaStream_t)stream;
  const int64_t grid = n_img * (H / p);
  const size_t tiled_smem = (size_t)p * (W * 3 + 16) + (size_t)(W / p < kPatchGroup ? W / p : kPatchGroup) * (kpad * 2 + 16);
  const bool aligned = ((reinterpret_cast<uintptr_t>(in) | reinterpret_cast<uintptr_t>(out)) & 15) == 0;
  if ((p == 14 || p == 16) && (W * 3) % 16 == 0 && aligned && tiled_smem <= 200 * 1024 &&
      (out_dtype == kBF16 || out_dtype == kF16)) {
#define NFB_PATCH_TILED(TO, P)                                                                               \
    do {                                                                                                   \
      cudaFuncSetAttribute(image_patchify_tiled_kernel<TO, P>, cudaFuncAttributeMaxDynamicSharedMemorySize, \
                           (int)tiled_smem);                                                               \
      image_patchify_tiled_kernel<TO, P><<<(unsigned)grid, 256, tiled_smem, st>>>(                          \
          (const uint8_t*)in, (TO*)out, H, W, kpad, k);                                                    \
    } while (0)
    if (out_dtype == kBF16) {
      if (p == 14) NFB_PATCH_TILED(__nv_bfloat16, 14); else NFB_PATCH_TILED(__nv_bfloat16, 16);
    } else {
      if (p == 14) NFB_PATCH_TILED(__half, 14); else NFB_PATCH_TILED(__half, 16);
    }
#undef NFB_PATCH_TILED
    return (int)cudaGetLastError();
  }
  const size_t smem = ((size_t)kpad * 4 + 15) / 16 * 16 + ((size_t)p * W * 3 + 15) / 16 * 16;
  if (smem > 200 * 1024) return (int)cudaErrorInvalidValue;
  if (out_dtype == kBF16) {
    if (smem > 48 * 1024) cudaFuncSetAttribute(image_patchify_kernel<__nv_bfloat16>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    image_patchify_kernel<__nv_bfloat16><<<(unsigned)grid, 256, smem, st>>>((const uint8_t*)in, (__nv_bfloat16*)out, H, W, p, kpad, k);
  } else if (out_dtype == kF16) {
    if (smem > 48 * 1024) cudaFuncSetAttribute(image_patchify_kernel<__half>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    image_patchify_kernel<__half><<<(unsigned)grid, 256, smem, st>>>((const uint8_t*)in, (__half*)out, H, W, p, kpad, k);
  } else {
    return (int)cudaErrorInvalidValue;
  }
  return (int)cudaGetLastError();
}
