// Cross entropy on the tcgen05 GEMM: the [M, V] logits exist only in TMEM.
//
// Parity: nuvla_forge/kernels/chunked_ce.py:120-208 computes the same mean CE and
// its gradients during forward, but materialises an fp32 [chunk, V] logit tile
// per chunk and syncs the host for the valid-token count. Here:
//
//   pass 1 (nfb_ce_tc_stats): logits tile = h[128 rows] x W[256 vocab]^T in TMEM;
//          the epilogue reduces each row's 256 logits to an online-softmax
//          partial (max, sum exp) per vocab tile and picks out the target logit.
//   merge  (nfb_ce_tc_merge): per row, merge the partials into the log-sum-exp
//          and the row's loss / count (count read from device memory).
//   pass 2 (nfb_ce_tc_grad): recompute the logits tile in TMEM; the epilogue
//          writes dlogits = (softmax - onehot) / count as bf16 for the two
//          gradient GEMMs (d_hidden = dl W, d_W += dl^T h), which the caller
//          runs per row chunk so only a [chunk, V] bf16 buffer ever exists.
//
// nfb_tc_gemm_bf16 exposes the same core as a plain C = A B^T GEMM (bf16 or
// fp32 output), used by the tests to check the core against cuBLAS.
#include <cudaTypedefs.h>

#include "tc_gemm.cuh"
#include "tc_host.cuh"

NFB_DEBUG_TU(ce_tc)

namespace nfb {
namespace tc {

template <class Epi, bool A_MN, bool B_MN>
__global__ void __launch_bounds__(kThreads, 1) tc_kernel(const __grid_constant__ CUtensorMap ta,
                                                        const __grid_constant__ CUtensorMap tb, GemmShape sh,
                                                        Epi epi, uint32_t* status) {
  Epi e = epi;
  NoGate g;
  gemm_body<A_MN, B_MN>(&ta, &tb, sh, e, status, g);
}

// A K-major operand [rows, K] is read in boxes of 64 K x box_rows rows; an MN-major one, stored
// [K, rows] with rows contiguous, in boxes of 64 rows x BK K (the core loads box_rows / 64 of them).
template <class Epi, bool A_MN, bool B_MN>
static int launch_t(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, const Epi& epi,
                    uint32_t* status, cudaStream_t st) {
  if (M <= 0 || N <= 0 || K <= 0) return 0;
  CUtensorMap ta, tb;
  int rc = A_MN ? make_tmap(&ta, A, K, M, lda, BK) : make_tmap(&ta, A, M, K, lda, BM);
  if (rc) return rc;
  rc = B_MN ? make_tmap(&tb, B, K, N, ldb, BK) : make_tmap(&tb, B, N, K, ldb, BN);
  if (rc) return rc;
  GemmShape sh = make_shape(M, N, K);
  cudaError_t e = cudaFuncSetAttribute(tc_kernel<Epi, A_MN, B_MN>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       (int)kSmemBytes);
  if (e != cudaSuccess) return (int)e;
  const int tiles = sh.m_tiles * sh.n_tiles;
  const int grid = tiles < sm_count() ? tiles : sm_count();
  tc_kernel<Epi, A_MN, B_MN><<<grid, kThreads, kSmemBytes, st>>>(ta, tb, sh, epi, status);
  return (int)cudaGetLastError();
}

template <class Epi>
static int launch(const void* A, int64_t lda, const void* B, int64_t ldb, int M, int N, int K, const Epi& epi,
                  uint32_t* status, cudaStream_t st) {
  return launch_t<Epi, false, false>(A, lda, B, ldb, M, N, K, epi, status, st);
}

// ---------------------------------------------------------------------------
// Epilogues (one TMEM lane = one output row per thread)
// ---------------------------------------------------------------------------

struct CeStatsEpi {
  const int64_t* targets;
  float* pmax;   // [M, n_tiles]
  float* psum;   // [M, n_tiles]
  float* tlogit; // [M]

  __device__ void row(int m0, int n0, int r, uint32_t taddr, const GemmShape& sh) {
    const int m = m0 + r;
    const int64_t tgt = m < sh.M ? targets[m] : -1;
    // debug build: a label outside [0, V) (other than the ignore value, < 0) never matches a column,
    // so its target logit would silently stay unset
    if (n0 == 0 && m < sh.M) NFB_DCHECK(tgt < (int64_t)sh.N, 1101, (void)0);
    float mx = -INFINITY, sum = 0.f;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float v[32];
      tmem_ld32(taddr + c, v);
      const int n = n0 + c;
      float cm = -INFINITY;
#pragma unroll
      for (int j = 0; j < 32; ++j) if (n + j < sh.N) cm = fmaxf(cm, v[j]);
      if (cm > mx) {
        sum = (mx == -INFINITY) ? 0.f : sum * __expf(mx - cm);
        mx = cm;
      }
      if (mx != -INFINITY) {
#pragma unroll
        for (int j = 0; j < 32; ++j) if (n + j < sh.N) sum += __expf(v[j] - mx);
      }
      if (tgt >= n && tgt < n + 32) {
#pragma unroll
        for (int j = 0; j < 32; ++j) if (tgt == n + j) tlogit[m] = v[j];
      }
    }
    if (m < sh.M) {
      const int64_t idx = (int64_t)m * sh.n_tiles + n0 / BN;
      pmax[idx] = mx;
      psum[idx] = sum;
    }
  }
};

struct CeGradEpi {
  const int64_t* targets;
  const float* lse;
  const float* count;
  __nv_bfloat16* dl;
  int64_t ldd;
  int64_t ignore_index;
  int vec_ok;

  __device__ void row(int m0, int n0, int r, uint32_t taddr, const GemmShape& sh) {
    const int m = m0 + r;
    const int64_t tgt = m < sh.M ? targets[m] : ignore_index;
    const bool valid = m < sh.M && tgt != ignore_index;
    const float inv = 1.f / fmaxf(*count, 1.f);
    const float l = valid ? lse[m] : 0.f;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float v[32];
      tmem_ld32(taddr + c, v);
      if (m >= sh.M) continue;
      const int n = n0 + c;
#pragma unroll
      for (int j = 0; j < 32; ++j) {
        float p = valid ? __expf(v[j] - l) * inv : 0.f;
        if (valid && tgt == n + j) p -= inv;
        v[j] = p;
      }
      __nv_bfloat16* dst = dl + (int64_t)m * ldd + n;
      if (vec_ok && n + 32 <= sh.N) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) store16<__nv_bfloat16>(dst + j, v + j);
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) if (n + j < sh.N) dst[j] = __float2bfloat16_rn(v[j]);
      }
    }
  }
};

__global__ void ce_merge_kernel(const float* pmax, const float* psum, const float* tlogit, const int64_t* targets,
                                const float* count, int M, int n_tiles, int64_t ignore_index, float* lse_out,
                                float* loss_rows) {
  const int m = blockIdx.x * blockDim.x + threadIdx.x;
  if (m >= M) return;
  float mx = -INFINITY, s = 0.f;
  for (int t = 0; t < n_tiles; ++t) {
    const float pm = pmax[(int64_t)m * n_tiles + t];
    const float ps = psum[(int64_t)m * n_tiles + t];
    if (pm == -INFINITY) continue;
    if (pm > mx) {
      s = (mx == -INFINITY) ? 0.f : s * __expf(mx - pm);
      mx = pm;
    }
    s += ps * __expf(pm - mx);
  }
  const float lse = mx + __logf(s);
  lse_out[m] = lse;
  const int64_t tgt = targets[m];
  const float inv = 1.f / fmaxf(*count, 1.f);
  loss_rows[m] = (tgt == ignore_index) ? 0.f : (lse - tlogit[m]) * inv;
}

}  // namespace tc
}  // namespace nfb

using namespace nfb;
using namespace nfb::tc;

// C[M, N] = A[M, K] @ B[N, K]^T, A/B bf16 with row strides lda/ldb; C bf16 (out_f32=0) or fp32.
// C[M, N] (=|+=) A B^T with A K-major [M, K] (a_mn = 0) or MN-major [K, M] (a_mn = 1), B K-major [N, K]
// or MN-major [K, N]; C bf16 or fp32 (out_f32), accumulate (fp32 only) adds into C.
NFB_API int nfb_tc_gemm_ex(const void* A, const void* B, void* C, int M, int N, int K, int64_t lda, int64_t ldb,
                           int64_t ldc, int out_f32, int a_mn, int b_mn, int accumulate, uint32_t* status,
                           void* stream) {
  if (accumulate && !out_f32) return (int)cudaErrorInvalidValue;
  StoreEpi epi{};
  epi.C = C; epi.ldc = ldc; epi.out_f32 = out_f32; epi.accumulate = accumulate;
  const int es = out_f32 ? 4 : 2;
  epi.vec_ok = ((reinterpret_cast<uintptr_t>(C) & 15) == 0) && ((ldc * es) % 16 == 0);
  cudaStream_t st = (cudaStream_t)stream;
  if (a_mn && b_mn) return launch_t<StoreEpi, true, true>(A, lda, B, ldb, M, N, K, epi, status, st);
  if (a_mn) return launch_t<StoreEpi, true, false>(A, lda, B, ldb, M, N, K, epi, status, st);
  if (b_mn) return launch_t<StoreEpi, false, true>(A, lda, B, ldb, M, N, K, epi, status, st);
  return launch_t<StoreEpi, false, false>(A, lda, B, ldb, M, N, K, epi, status, st);
}

NFB_API int nfb_tc_gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, int64_t lda, int64_t ldb,
                             int64_t ldc, int out_f32, uint32_t* status, void* stream) {
  return nfb_tc_gemm_ex(A, B, C, M, N, K, lda, ldb, ldc, out_f32, 0, 0, 0, status, stream);
}

NFB_API int nfb_ce_tc_tiles(int V) { return (V + BN - 1) / BN; }

// Pass 1: online-softmax partials per (row, vocab tile) and the target logit.
NFB_API int nfb_ce_tc_stats(const void* hidden, int64_t ldh, const void* weight, int64_t ldw, const int64_t* targets,
                            int M, int V, int H, float* pmax, float* psum, float* tlogit, uint32_t* status,
                            void* stream) {
  CeStatsEpi epi{targets, pmax, psum, tlogit};
  return launch(hidden, ldh, weight, ldw, M, V, H, epi, status, (cudaStream_t)stream);
}

NFB_API int nfb_ce_tc_merge(const float* pmax, const float* psum, const float* tlogit, const int64_t* targets,
                            const float* count, int M, int V, int64_t ignore_index, float* lse, float* loss_rows,
                            void* stream) {
  if (M <= 0) return 0;
  ce_merge_kernel<<<(M + 255) / 256, 256, 0, (cudaStream_t)stream>>>(pmax, psum, tlogit, targets, count, M,
                                                                     (V + BN - 1) / BN, ignore_index, lse, loss_rows);
  return (int)cudaGetLastError();
}

// Pass 2: dl[M, V] = (softmax - onehot) / count in bf16, recomputing the logits in TMEM.
NFB_API int nfb_ce_tc_grad(const void* hidden, int64_t ldh, const void* weight, int64_t ldw, const int64_t* targets,
                           const float* lse, const float* count, int64_t ignore_index, int M, int V, int H, void* dl,
                           int64_t ldd, uint32_t* status, void* stream) {
  CeGradEpi epi;
  epi.targets = targets; epi.lse = lse; epi.count = count; epi.dl = (__nv_bfloat16*)dl; epi.ldd = ldd;
  epi.ignore_index = ignore_index;
  epi.vec_ok = ((reinterpret_cast<uintptr_t>(dl) & 15) == 0) && ((ldd * 2) % 16 == 0);
  return launch(hidden, ldh, weight, ldw, M, V, H, epi, status, (cudaStream_t)stream);
}
