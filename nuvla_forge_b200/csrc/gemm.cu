// Entry points of the CTA-pair tcgen05 GEMM (gemm2.cuh) used by every linear layer of the model.
//
// Parity: the reference's linear layers are nn.Linear / F.linear on cuBLAS
// (nuvla_forge/model/dit.py:75-76, 91-92, 99-101; nuvla_forge/model/nuvla.py:112, 123). Here
// their forward, input-gradient and weight-gradient GEMMs run on this kernel:
//   nfb_gemm       C = A B^T (+ bias) (+ residual), bf16 or fp32 output (forward, dgrad)
//   nfb_gemm_acc   fp32 C (+)= A B^T with ordered split-K (wgrad into an fp32 gradient buffer)
#include <cudaTypedefs.h>

#include <stdio.h>
#include <string.h>

#include <mutex>

#include "gemm2.cuh"
#include "nfb_api.h"
#include "tc_host.cuh"

using namespace nfb;
using namespace nfb::g2;

NFB_DEBUG_TU(gemm)

// Where the last failing GEMM call of this host thread stopped ("" if none).
static thread_local char g_gemm_err[160] = "";

static int gemm_fail(int rc, const char* site) {
  snprintf(g_gemm_err, sizeof(g_gemm_err), "%s (cuda error %d)", site, rc);
  return rc;
}

namespace {

template <class Epi, bool A_MN, bool B_MN>
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(threads_for<Epi>(), 1)
    gemm_pair_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb,
                     const __grid_constant__ CUtensorMap tc, const __grid_constant__ CUtensorMap td, Work w,
                     Epi epi, uint32_t* status) {
  Epi e = epi;
  gemm_pair_body<A_MN, B_MN>(&ta, &tb, &tc, &td, w, e, status);
}

// Co-resident clusters of a kernel (cached per device and kernel).
struct ClusterCache {
  const void* fn[64];
  int dev[64];
  int clusters[64];
  int n = 0;
};
static ClusterCache g_cc;
static std::mutex g_cc_mu;

template <class K>
static int max_clusters(K kernel, int* out, size_t smem_bytes, int threads) {
  int dev = 0;
  cudaGetDevice(&dev);
  std::lock_guard<std::mutex> lock(g_cc_mu);
  for (int i = 0; i < g_cc.n; ++i) {
    if (g_cc.fn[i] == (const void*)kernel && g_cc.dev[i] == dev) { *out = g_cc.clusters[i]; return 0; }
  }
  cudaError_t e = cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem_bytes);
  if (e != cudaSuccess) return (int)e;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(2 * 74, 1, 1);
  cfg.blockDim = dim3(threads, 1, 1);
  cfg.dynamicSmemBytes = smem_bytes;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  int n = 0;
  e = cudaOccupancyMaxActiveClusters(&n, kernel, &cfg);
  if (e != cudaSuccess) return (int)e;
  if (n <= 0) return (int)cudaErrorLaunchOutOfResources;
  if (g_cc.n < 64) {
    g_cc.fn[g_cc.n] = (const void*)kernel;
    g_cc.dev[g_cc.n] = dev;
    g_cc.clusters[g_cc.n] = n;
    ++g_cc.n;
  }
  *out = n;
  return 0;
}

static Work make_work(int M, int N, int K) {
  Work w;
  w.M = M; w.N = N; w.K = K;
  w.m_tiles = (M + TM - 1) / TM;
  w.n_tiles = (N + TN - 1) / TN;
  w.k_blocks = (K + BK - 1) / BK;
  w.splits = 1;
  w.kb_per_split = w.k_blocks;
  w.group = 8;
  w.items = w.m_tiles * w.n_tiles;
  return w;
}

// Split count for a weight-gradient GEMM: the smallest one whose last wave keeps >= 85% of the
// clusters busy, at most 4 (a tile's slices are added one after the other, so the epilogue chain
// grows with the split count), with at least 8 K blocks (512 of K) per slice.
static int choose_splits(int tiles, int k_blocks, int clusters) {
  int best = 1;
  double best_eff = 0.0;
  int smax = k_blocks / 8;
  if (smax > 4) smax = 4;
  if (smax < 1) smax = 1;
  for (int s = 1; s <= smax; ++s) {
    const int items = tiles * s;
    const int waves = (items + clusters - 1) / clusters;
    const double eff = (double)items / ((double)waves * clusters);
    if (eff >= 0.85) return s;
    if (eff > best_eff + 0.02) { best_eff = eff; best = s; }
  }
  return best;
}

// K-major operand stored [rows, K] -> boxes of 64 K x 128 rows; MN-major operand stored
// [K, rows] -> boxes of 64 rows-columns x 64 K (the kernel loads two per 128 rows).
static int operand_map(CUtensorMap* m, const void* p, int rows, int K, int64_t ld, bool mn) {
  return mn ? tc::make_tmap(m, p, K, rows, ld, BK) : tc::make_tmap(m, p, rows, K, ld, HALF);
}

// fp32 map for the accumulating epilogue: [M, N] with row stride ldc, 32 x 32 boxes, 128-byte swizzle.
static int output_map_f32(CUtensorMap* m, const void* C, int M, int N, int64_t ldc) {
  int rc = tc::get_encode();
  if (rc) return rc;
  rc = tc::bind_device_of(C);
  if (rc) return rc;
  cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)(ldc * 4)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tc::g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<void*>(C), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

// Output map for the staged epilogue: bf16 [M, N] with row stride ldc, 32 x 32 boxes, 64-byte swizzle.
static int output_map(CUtensorMap* m, const void* C, int M, int N, int64_t ldc) {
  int rc = tc::get_encode();
  if (rc) return rc;
  rc = tc::bind_device_of(C);
  if (rc) return rc;
  cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)(ldc * 2)};
  cuuint32_t box[2] = {32, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tc::g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(C), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_64B,
                            CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

// Map for the SwiGLU-backward epilogue: bf16 [M, N] with row stride ldc, 32-row x 64-column boxes
// (128-byte rows), 128-byte swizzle.
static int output_map_wide(CUtensorMap* m, const void* C, int M, int N, int64_t ldc) {
  int rc = tc::get_encode();
  if (rc) return rc;
  rc = tc::bind_device_of(C);
  if (rc) return rc;
  cuuint64_t dims[2] = {(cuuint64_t)N, (cuuint64_t)M};
  cuuint64_t strides[1] = {(cuuint64_t)(ldc * 2)};
  cuuint32_t box[2] = {64, 32};
  cuuint32_t estr[2] = {1, 1};
  CUresult r = tc::g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(C), dims, strides, box, estr,
                            CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                            CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

template <class Epi, bool A_MN, bool B_MN>
static int launch(const void* A, int64_t lda, const void* B, int64_t ldb, Work w, const Epi& epi, uint32_t* status,
                  cudaStream_t st, const CUtensorMap* tc_map = nullptr, const CUtensorMap* td_map = nullptr) {
  CUtensorMap ta, tb, tcm, tdm;
  if (tc_map) tcm = *tc_map;
  else memset(&tcm, 0, sizeof(tcm));
  if (td_map) tdm = *td_map;
  else memset(&tdm, 0, sizeof(tdm));
  int rc = operand_map(&ta, A, w.M, w.K, lda, A_MN);
  if (rc) return gemm_fail(rc, "tensor map of A");
  rc = operand_map(&tb, B, w.N, w.K, ldb, B_MN);
  if (rc) return gemm_fail(rc, "tensor map of B");
  auto kern = gemm_pair_kernel<Epi, A_MN, B_MN>;
  int clusters = 0;
  rc = max_clusters(kern, &clusters, smem_bytes_for<Epi>(), threads_for<Epi>());
  if (rc) return gemm_fail(rc, "cluster occupancy query");
  const int grid_clusters = w.items < clusters ? w.items : clusters;
  cudaError_t pending = cudaGetLastError();     // an error left by an earlier call of this thread
  if (pending != cudaSuccess) return gemm_fail((int)pending, "error pending before the launch");
  kern<<<2 * grid_clusters, threads_for<Epi>(), smem_bytes_for<Epi>(), st>>>(ta, tb, tcm, tdm, w, epi, status);
  rc = (int)cudaGetLastError();
  return rc ? gemm_fail(rc, "kernel launch") : 0;
}

template <class Epi>
static int dispatch(const void* A, int64_t lda, const void* B, int64_t ldb, Work w, const Epi& epi, int a_mn,
                    int b_mn, uint32_t* status, cudaStream_t st, const CUtensorMap* tc_map = nullptr) {
  if (a_mn && b_mn) return launch<Epi, true, true>(A, lda, B, ldb, w, epi, status, st, tc_map);
  if (a_mn) return launch<Epi, true, false>(A, lda, B, ldb, w, epi, status, st, tc_map);
  if (b_mn) return launch<Epi, false, true>(A, lda, B, ldb, w, epi, status, st, tc_map);
  return launch<Epi, false, false>(A, lda, B, ldb, w, epi, status, st, tc_map);
}

static bool al16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

NFB_API const char* nfb_gemm_last_error() { return g_gemm_err; }

NFB_API int nfb_gemm(const void* A, const void* B, void* C, int M, int N, int K, int64_t lda, int64_t ldb,
                     int64_t ldc, int a_mn, int b_mn, int out_f32, const void* bias, const void* R, int64_t ldr,
                     uint32_t* status, void* stream) {
  if (M <= 0 || N <= 0) return 0;
  if (K <= 0) return (int)cudaErrorInvalidValue;
  LinearEpi epi;
  epi.C = C; epi.ldc = ldc;
  epi.bias = reinterpret_cast<const __nv_bfloat16*>(bias);
  epi.R = reinterpret_cast<const __nv_bfloat16*>(R);
  epi.ldr = ldr;
  epi.out_f32 = out_f32;
  const int es = out_f32 ? 4 : 2;
  epi.vec_ok = al16(C) && (ldc * es) % 16 == 0 && (!bias || al16(bias)) && (!R || (al16(R) && (ldr * 2) % 16 == 0));
  epi.chunk = 0;
  epi.use_tma = 0;
  CUtensorMap tcm;
  if (!out_f32 && al16(C) && (ldc * 2) % 16 == 0 && N % 8 == 0 && output_map(&tcm, C, M, N, ldc) == 0)
    epi.use_tma = 1;
  return dispatch(A, lda, B, ldb, make_work(M, N, K), epi, a_mn, b_mn, status, (cudaStream_t)stream,
                  epi.use_tma ? &tcm : nullptr);
}

NFB_API int nfb_gemm_acc(const void* A, const void* B, float* C, int M, int N, int K, int64_t lda, int64_t ldb,
                         int64_t ldc, int a_mn, int b_mn, int accumulate, int splits, uint32_t* flags,
                         int64_t flag_words, uint32_t epoch, uint32_t* status, void* stream) {
  if (M <= 0 || N <= 0) return 0;
  if (K <= 0) return (int)cudaErrorInvalidValue;
  Work w = make_work(M, N, K);
  const int tiles = w.m_tiles * w.n_tiles;
  if (splits <= 0) {
    int clusters = 0;
    int rc = max_clusters(gemm_pair_kernel<AccumF32Epi, true, true>, &clusters, smem_bytes_for<AccumF32Epi>(), threads_for<AccumF32Epi>());
    if (rc) return rc;
    splits = choose_splits(tiles, w.k_blocks, clusters);
  }
  if (splits > w.k_blocks) splits = w.k_blocks;
  if (splits > 255) splits = 255;
  if (splits > 1 && (flags == nullptr || (int64_t)tiles * 8 > flag_words)) splits = 1;
  w.splits = splits;
  w.kb_per_split = (w.k_blocks + splits - 1) / splits;
  w.splits = (w.k_blocks + w.kb_per_split - 1) / w.kb_per_split;   // no empty slice
  w.items = tiles * w.splits;
  AccumF32Epi epi;
  epi.C = C; epi.ldc = ldc; epi.accumulate = accumulate;
  epi.vec_ok = al16(C) && (ldc * 4) % 16 == 0;
  epi.flags = flags;
  epi.epoch = epoch & 0xFFFFFFu;
  epi.chunk = 0;
  epi.use_tma = 0;
  CUtensorMap tcm;
  if (epi.vec_ok && N % 4 == 0 && output_map_f32(&tcm, C, M, N, ldc) == 0) epi.use_tma = 1;
  return dispatch(A, lda, B, ldb, w, epi, a_mn, b_mn, status, (cudaStream_t)stream, epi.use_tma ? &tcm : nullptr);
}

// act [M, F] = silu(gate) * up with (gate | up) = X W^T, W [2F, K] interleaved in 128-row blocks
// (gate rows of hidden units [128 b, 128 b + 128), then their up rows); the pre-activations go to
// ab [M, 2F] in the same interleaved order. F must be a multiple of 128.
NFB_API int nfb_gemm_swiglu_fwd(const void* X, const void* W, void* ab, void* act, int M, int F, int K, int64_t ldx,
                                int64_t ldw, int64_t ldab, int64_t ldact, uint32_t* status, void* stream) {
  if (M <= 0) return 0;
  if (K <= 0 || F <= 0 || F % 128) return gemm_fail((int)cudaErrorInvalidValue, "swiglu: F must be a multiple of 128");
  CUtensorMap tab, tact;
  int rc = output_map_wide(&tab, ab, M, 2 * F, ldab);
  if (rc) return gemm_fail(rc, "tensor map of ab");
  rc = output_map_wide(&tact, act, M, F, ldact);
  if (rc) return gemm_fail(rc, "tensor map of act");
  SwiGluFwdEpi epi;
  epi.chunk = 0;
  return launch<SwiGluFwdEpi, false, false>(X, ldx, W, ldw, make_work(M, 2 * F, K), epi, status,
                                            (cudaStream_t)stream, &tab, &tact);
}

// d_ab [M, 2F] (interleaved like ab) from dY [M, D] and the down projection W_down [D, F]:
// d_act = dY W_down on the tensor cores, then the SwiGLU backward in the epilogue (reads ab).
NFB_API int nfb_gemm_swiglu_bwd(const void* dY, const void* Wd, const void* ab, void* dab, int M, int F, int D,
                                int64_t ldy, int64_t ldw, int64_t ldab, int64_t lddab, uint32_t* status, void* stream) {
  if (M <= 0) return 0;
  if (D <= 0 || F <= 0 || F % 128) return gemm_fail((int)cudaErrorInvalidValue, "swiglu: F must be a multiple of 128");
  if (!al16(ab) || (ldab * 2) % 16) return gemm_fail((int)cudaErrorInvalidValue, "swiglu: ab rows not 16-byte aligned");
  CUtensorMap tdab, tab;
  int rc = output_map_wide(&tdab, dab, M, 2 * F, lddab);
  if (rc) return gemm_fail(rc, "tensor map of d_ab");
  rc = output_map_wide(&tab, ab, M, 2 * F, ldab);   // the same 32 x 64 boxes, read by TMA loads
  if (rc) return gemm_fail(rc, "tensor map of ab");
  SwiGluBwdEpi epi;
  epi.loads = 0;
  epi.done = 0;
  epi.inited = 0;
  return launch<SwiGluBwdEpi, false, true>(dY, ldy, Wd, ldw, make_work(M, F, D), epi, status, (cudaStream_t)stream,
                                           &tdab, &tab);
}

// Split count nfb_gemm_acc picks for this shape when given splits = 0 (for callers sizing flags).
NFB_API int nfb_gemm_acc_splits(int M, int N, int K) {
  Work w = make_work(M, N, K);
  int clusters = 0;
  if (max_clusters(gemm_pair_kernel<AccumF32Epi, true, true>, &clusters, smem_bytes_for<AccumF32Epi>(), threads_for<AccumF32Epi>())) return 1;
  return choose_splits(w.m_tiles * w.n_tiles, w.k_blocks, clusters);
}

NFB_API int nfb_gemm_max_clusters() {
  int clusters = 0;
  if (max_clusters(gemm_pair_kernel<LinearEpi, false, false>, &clusters, smem_bytes_for<LinearEpi>(), threads_for<LinearEpi>())) return -1;
  return clusters;
}

// ---------------------------------------------------------------------------
// Small GEMM on the CUDA cores for the layers whose widths the tensor-core kernel cannot tile
// (a 3-wide waypoint input or output): C[m, n] (=|+=) sum_k A[m, k] B[n, k] (+ bias[n]),
// every operand addressed through (row, column) strides, so the transposed products of the
// backward pass need no copies. fp32 accumulation; one thread per output element.
// ---------------------------------------------------------------------------
namespace {

template <typename TA, typename TC>
__global__ void gemm_small_kernel(const TA* __restrict__ A, int64_t sam, int64_t sak, const TA* __restrict__ B,
                                  int64_t sbn, int64_t sbk, TC* __restrict__ C, int64_t scm, int64_t scn,
                                  const TA* __restrict__ bias, int M, int N, int K, int accumulate) {
  const int64_t idx = (int64_t)blockIdx.x * blockDim.x + threadIdx.x;
  if (idx >= (int64_t)M * N) return;
  const int m = (int)(idx / N);
  const int n = (int)(idx - (int64_t)m * N);
  // debug build: strides that would make an operand walk backwards past its base
  NFB_DCHECK(sam >= 0 && sak >= 0 && sbn >= 0 && sbk >= 0 && scm >= 0 && scn >= 0, 1201, return);
  const TA* a = A + m * sam;
  const TA* b = B + n * sbn;
  float s = 0.f;
  for (int k = 0; k < K; ++k) s += to_f32(a[k * sak]) * to_f32(b[k * sbk]);
  if (bias) s += to_f32(bias[n]);
  TC* c = C + m * scm + n * scn;
  if (accumulate) s += to_f32(*c);
  *c = from_f32<TC>(s);
}

}  // namespace

NFB_API int nfb_gemm_small(int dtype, int out_f32, const void* A, int64_t sam, int64_t sak, const void* B,
                           int64_t sbn, int64_t sbk, void* C, int64_t scm, int64_t scn, const void* bias, int M, int N,
                           int K, int accumulate, void* stream) {
  if ((int64_t)M * N == 0) return 0;
  const int64_t total = (int64_t)M * N;
  const int threads = 256;
  const unsigned grid = (unsigned)((total + threads - 1) / threads);
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == kBF16 && out_f32) {
    gemm_small_kernel<__nv_bfloat16, float><<<grid, threads, 0, st>>>(
        (const __nv_bfloat16*)A, sam, sak, (const __nv_bfloat16*)B, sbn, sbk, (float*)C, scm, scn,
        (const __nv_bfloat16*)bias, M, N, K, accumulate);
  } else if (dtype == kBF16) {
    gemm_small_kernel<__nv_bfloat16, __nv_bfloat16><<<grid, threads, 0, st>>>(
        (const __nv_bfloat16*)A, sam, sak, (const __nv_bfloat16*)B, sbn, sbk, (__nv_bfloat16*)C, scm, scn,
        (const __nv_bfloat16*)bias, M, N, K, accumulate);
  } else if (dtype == kF32) {
    gemm_small_kernel<float, float><<<grid, threads, 0, st>>>((const float*)A, sam, sak, (const float*)B, sbn, sbk,
                                                              (float*)C, scm, scn, (const float*)bias, M, N, K,
                                                              accumulate);
  } else {
    return (int)cudaErrorInvalidValue;
  }
  return (int)cudaGetLastError();
}
