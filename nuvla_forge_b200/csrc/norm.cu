// Fused gated residual + RMSNorm + adaLN-Zero modulation, forward and backward.
//
//   h   = x + g * y                 g = gate[b] (GATE_VEC), 1 (GATE_ONE); no residual when GATE_NONE (h = x)
//   out = rmsnorm(h) * w * (1 + scale[b]) + shift[b]      (MOD); out = rmsnorm(h) * w otherwise
//
// Row m belongs to sample b = m / T. Parity with the reference Triton kernels
// (nuvla_forge/kernels/adaln_rmsnorm.py:61-162) in what is computed; the
// schedule is our own:
//
// * A "team" of K warps owns one row; each thread owns NV=2 chunks of 8
//   contiguous columns, so a team covers K*512 columns (N <= 8192, K <= 16).
//   Several teams share a CTA so that enough rows are in flight per SM.
// * Backward is ONE launch. The per-sample reductions (dgate, dscale, dshift)
//   and the global dweight are deterministic and lock-free: each CTA owns one
//   sample and a strided set of its rows, keeps its column partials in
//   registers, folds its teams together in shared memory in a fixed order and
//   writes one partial row to scratch. The last CTA of a sample (atomic ticket)
//   sums that sample's partials in index order; the last sample to finish sums
//   the per-sample dweight rows in index order. Ticket counters reset
//   themselves, so the scratch needs zeroing only once when it is created.
//   dscale and dweight share one accumulator A = sum_t dout * xhat, because
//   dscale[b] = w * A_b and dweight = sum_b (1 + scale[b]) * A_b.
#include "common.cuh"

namespace nfb {

enum GateMode : int { GATE_NONE = 0, GATE_ONE = 1, GATE_VEC = 2 };
constexpr int NV = 2;        // 8-column chunks per thread
constexpr int CPT = NV * 8;  // columns per thread

struct NormFwdArgs {
  const void* x; const void* y; const void* gate; const void* weight;
  const void* scale; const void* shift;
  void* h; void* out; float* rstd;
  int64_t M, N, T;
  int64_t sx, sy, sh, so;        // row strides (elements)
  int64_t sg, ss, ssh;           // row strides of gate / scale / shift ([B, N] views)
  float eps;
  int w_f32;                     // weight stored as fp32 (else same dtype as x)
};

struct NormBwdArgs {
  const void* dh_up;  // may be null (treated as zero)
  const void* dout;
  const void* h;      // the residual stream saved by forward (x when GATE_NONE)
  const void* y;
  const void* gate; const void* weight; const void* scale;
  const float* rstd;
  void* dx; void* dy;
  void* dgate; void* dscale; void* dshift; void* dweight;
  float* partials;    // [B*P][3][N]
  float* dwb;         // [B][N]
  uint32_t* tickets;  // [B + 1], zero on entry, zero again on exit
  int64_t M, N, T, B, P;
  int64_t s_dhup, s_dout, s_h, s_y, s_dx, s_dy;
  int64_t sg, ss;
  int w_f32;
};

__device__ __forceinline__ void named_bar(int id, int nthreads) {
  asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(nthreads) : "memory");
}

// Sum over the K warps of one team. red: [2][K] floats for this team.
__device__ __forceinline__ float team_sum(float v, float* red, int parity, int wt, int K, int bar_id) {
  v = warp_sum(v);
  if (K == 1) return v;
  if ((threadIdx.x & 31) == 0) red[parity * K + wt] = v;
  named_bar(bar_id, K * 32);
  float s = 0.f;
  for (int k = 0; k < K; ++k) s += red[parity * K + k];
  return s;
}

template <typename T>
__device__ __forceinline__ void load_chunk(const T* base, int64_t col, int64_t N, float* out) {
  if (col < N) load8<T>(base + col, out);
  else {
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = 0.f;
  }
}

template <typename T>
__device__ __forceinline__ void load_weight_chunk(const void* w, int w_f32, int64_t col, int64_t N, float* out) {
  if (col >= N) {
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = 0.f;
    return;
  }
  if (w_f32) {
    load16<float>(reinterpret_cast<const float*>(w) + col, out);
    load16<float>(reinterpret_cast<const float*>(w) + col + 4, out + 4);
  } else {
    load8<T>(reinterpret_cast<const T*>(w) + col, out);
  }
}

// ---------------------------------------------------------------------------
// Forward
// ---------------------------------------------------------------------------
template <typename T, int GATE, bool MOD>
__global__ void __launch_bounds__(512) norm_fwd_kernel(NormFwdArgs a, int K, int R) {
  extern __shared__ float smem[];
  const int tid = threadIdx.x;
  const int team = tid / (K * 32);
  const int tt = tid % (K * 32);       // thread index within team
  const int wt = tt / 32;              // warp index within team
  float* red = smem + team * 2 * K;
  const int bar_id = 1 + team;
  const int64_t N = a.N;

  int parity = 0;
  for (int64_t row = (int64_t)blockIdx.x * R + team; row < a.M; row += (int64_t)gridDim.x * R) {
    const int64_t b = row / a.T;
    const T* xr = reinterpret_cast<const T*>(a.x) + row * a.sx;
    float hv[CPT];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = ((int64_t)i * K * 32 + tt) * 8;
      float xv[8];
      load_chunk<T>(xr, col, N, xv);
      if (GATE != GATE_NONE) {
        float yv[8];
        load_chunk<T>(reinterpret_cast<const T*>(a.y) + row * a.sy, col, N, yv);
        if (GATE == GATE_VEC) {
          float gv[8];
          load_chunk<T>(reinterpret_cast<const T*>(a.gate) + b * a.sg, col, N, gv);
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[j] = xv[j] + gv[j] * yv[j];
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) xv[j] = xv[j] + yv[j];
        }
        // h is stored in the activation dtype; the norm uses the rounded value
        // so that forward and backward see the same h.
        round8<T>(xv);
        if (col < N) store8<T>(reinterpret_cast<T*>(a.h) + row * a.sh + col, xv);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) { hv[i * 8 + j] = xv[j]; ss += xv[j] * xv[j]; }
    }
    ss = team_sum(ss, red, parity, wt, K, bar_id);
    parity ^= 1;
    const float rstd = rsqrtf(ss / (float)N + a.eps);
    if (tt == 0) a.rstd[row] = rstd;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = ((int64_t)i * K * 32 + tt) * 8;
      if (col >= N) continue;
      float wv[8];
      load_weight_chunk<T>(a.weight, a.w_f32, col, N, wv);
      float o[8];
      if (MOD) {
        float sc[8], sf[8];
        load8<T>(reinterpret_cast<const T*>(a.scale) + b * a.ss + col, sc);
        load8<T>(reinterpret_cast<const T*>(a.shift) + b * a.ssh + col, sf);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = hv[i * 8 + j] * rstd * wv[j] * (1.f + sc[j]) + sf[j];
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = hv[i * 8 + j] * rstd * wv[j];
      }
      store8<T>(reinterpret_cast<T*>(a.out) + row * a.so + col, o);
    }
  }
}

// Warp-per-row forward for N <= 4096: each lane owns NW chunks of 8 columns,
// the row reduction is a warp shuffle (no shared memory, no named barriers),
// and all chunk loads of a row are issued before any of them is used.
template <typename T, int GATE, bool MOD, int NW>
__global__ void __launch_bounds__(256) norm_fwd_warp_kernel(NormFwdArgs a) {
  const int lane = threadIdx.x & 31;
  const int64_t warps = (int64_t)gridDim.x * (blockDim.x >> 5);
  const int64_t N = a.N;
  for (int64_t row = (int64_t)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < a.M; row += warps) {
    const int64_t b = row / a.T;
    float hv[NW][8];
    float ss = 0.f;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      const int64_t col = ((int64_t)i * 32 + lane) * 8;
      load_chunk<T>(reinterpret_cast<const T*>(a.x) + row * a.sx, col, N, hv[i]);
      if (GATE != GATE_NONE) {
        float yv[8];
        load_chunk<T>(reinterpret_cast<const T*>(a.y) + row * a.sy, col, N, yv);
        if (GATE == GATE_VEC) {
          float gv[8];
          load_chunk<T>(reinterpret_cast<const T*>(a.gate) + b * a.sg, col, N, gv);
#pragma unroll
          for (int j = 0; j < 8; ++j) hv[i][j] += gv[j] * yv[j];
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) hv[i][j] += yv[j];
        }
        round8<T>(hv[i]);
        if (col < N) store8<T>(reinterpret_cast<T*>(a.h) + row * a.sh + col, hv[i]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += hv[i][j] * hv[i][j];
    }
    ss = warp_sum(ss);
    const float rstd = rsqrtf(ss / (float)N + a.eps);
    if (lane == 0) a.rstd[row] = rstd;
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      const int64_t col = ((int64_t)i * 32 + lane) * 8;
      if (col >= N) continue;
      float wv[8], o[8];
      load_weight_chunk<T>(a.weight, a.w_f32, col, N, wv);
      if (MOD) {
        float sc[8], sf[8];
        load8<T>(reinterpret_cast<const T*>(a.scale) + b * a.ss + col, sc);
        load8<T>(reinterpret_cast<const T*>(a.shift) + b * a.ssh + col, sf);
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = hv[i][j] * rstd * wv[j] * (1.f + sc[j]) + sf[j];
      } else {
#pragma unroll
        for (int j = 0; j < 8; ++j) o[j] = hv[i][j] * rstd * wv[j];
      }
      store8<T>(reinterpret_cast<T*>(a.out) + row * a.so + col, o);
    }
  }
}

// ---------------------------------------------------------------------------
// Backward
// ---------------------------------------------------------------------------
template <typename T, int GATE, bool MOD>
__global__ void __launch_bounds__(512, (GATE == GATE_VEC || MOD) ? 1 : 2) norm_bwd_kernel(NormBwdArgs a, int K, int R) {
  extern __shared__ float smem[];
  const int tid = threadIdx.x;
  const int team = tid / (K * 32);
  const int tt = tid % (K * 32);
  const int wt = tt / 32;
  const int nthreads = blockDim.x;
  const int64_t N = a.N;
  float* ws_s = smem;                        // [N]  w * (1 + scale[b])
  float* gv_s = smem + N;                    // [N]  gate[b]
  float* red = smem + 2 * N + team * 2 * K;  // [R][2][K]
  float* tpart = smem + 2 * N + R * 2 * K;   // [R][3][N] team partials (R > 1 only)
  __shared__ uint32_t s_ticket;
  const int bar_id = 1 + team;
  const int64_t b = blockIdx.x / a.P;
  const int64_t p = blockIdx.x % a.P;

  for (int64_t c = tid; c < N; c += nthreads) {
    float w = a.w_f32 ? reinterpret_cast<const float*>(a.weight)[c]
                      : to_f32(reinterpret_cast<const T*>(a.weight)[c]);
    float s1 = MOD ? 1.f + to_f32(reinterpret_cast<const T*>(a.scale)[b * a.ss + c]) : 1.f;
    ws_s[c] = w * s1;
    gv_s[c] = (GATE == GATE_VEC) ? to_f32(reinterpret_cast<const T*>(a.gate)[b * a.sg + c]) : 1.f;
  }
  __syncthreads();

  float accA[CPT], accD[CPT], accG[CPT];
#pragma unroll
  for (int j = 0; j < CPT; ++j) { accA[j] = 0.f; accD[j] = 0.f; accG[j] = 0.f; }

  const float invN = 1.f / (float)N;
  int parity = 0;
  // Rows of sample b handled by this CTA: t = p*R + team, stepping P*R.
  for (int64_t t = p * R + team; t < a.T; t += a.P * R) {
    const int64_t row = b * a.T + t;
    const float rstd = a.rstd[row];
    const T* dout_r = reinterpret_cast<const T*>(a.dout) + row * a.s_dout;
    const T* h_r = reinterpret_cast<const T*>(a.h) + row * a.s_h;
    // pass 1: row dot product and the per-column accumulators
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = ((int64_t)i * K * 32 + tt) * 8;
      float dv[8], hv[8];
      load_chunk<T>(dout_r, col, N, dv);
      load_chunk<T>(h_r, col, N, hv);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = hv[j] * rstd;
        const float w = (col < N) ? ws_s[col + j] : 0.f;
        dot += dv[j] * w * xh;
        accA[i * 8 + j] += dv[j] * xh;
        if (MOD) accD[i * 8 + j] += dv[j];
      }
    }
    dot = team_sum(dot, red, parity, wt, K, bar_id) * invN;
    parity ^= 1;
    // pass 2: the row is re-read (L1-resident) rather than kept in registers
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = ((int64_t)i * K * 32 + tt) * 8;
      if (col >= N) continue;
      float dv[8], hv[8], dh[8];
      load8<T>(dout_r + col, dv);
      load8<T>(h_r + col, hv);
      if (a.dh_up != nullptr) load8<T>(reinterpret_cast<const T*>(a.dh_up) + row * a.s_dhup + col, dh);
      else {
#pragma unroll
        for (int j = 0; j < 8; ++j) dh[j] = 0.f;
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = hv[j] * rstd;
        dh[j] += rstd * (dv[j] * ws_s[col + j] - xh * dot);
      }
      store8<T>(reinterpret_cast<T*>(a.dx) + row * a.s_dx + col, dh);
      if (GATE == GATE_VEC) {
        float yv[8], dyv[8];
        load8<T>(reinterpret_cast<const T*>(a.y) + row * a.s_y + col, yv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          dyv[j] = dh[j] * gv_s[col + j];
          accG[i * 8 + j] += dh[j] * yv[j];
        }
        store8<T>(reinterpret_cast<T*>(a.dy) + row * a.s_dy + col, dyv);
      } else if (GATE == GATE_ONE) {
        if (a.dy != nullptr) store8<T>(reinterpret_cast<T*>(a.dy) + row * a.s_dy + col, dh);
      }
    }
  }

  // ---- fold teams (fixed order) and write this CTA's partial row ----------
  float* part = a.partials + (size_t)blockIdx.x * 3 * N;
  if (R == 1) {
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = ((int64_t)i * K * 32 + tt) * 8;
      if (col >= N) continue;
      store16<float>(part + col, accA + i * 8); store16<float>(part + col + 4, accA + i * 8 + 4);
      store16<float>(part + N + col, accD + i * 8); store16<float>(part + N + col + 4, accD + i * 8 + 4);
      store16<float>(part + 2 * N + col, accG + i * 8); store16<float>(part + 2 * N + col + 4, accG + i * 8 + 4);
    }
  } else {
    float* mine = tpart + (size_t)team * 3 * N;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = ((int64_t)i * K * 32 + tt) * 8;
      if (col >= N) continue;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        mine[col + j] = accA[i * 8 + j];
        mine[N + col + j] = accD[i * 8 + j];
        mine[2 * N + col + j] = accG[i * 8 + j];
      }
    }
    __syncthreads();
    for (int64_t c = tid; c < 3 * N; c += nthreads) {
      float s = 0.f;
      for (int r = 0; r < R; ++r) s += tpart[(size_t)r * 3 * N + c];
      part[c] = s;
    }
  }

  // ---- last CTA of this sample reduces the sample's partials --------------
  __threadfence();
  __syncthreads();
  if (tid == 0) s_ticket = atomicAdd(&a.tickets[b], 1u);
  __syncthreads();
  if (s_ticket != (uint32_t)(a.P - 1)) return;
  __threadfence();

  const float* sp = a.partials + (size_t)b * a.P * 3 * N;
  for (int64_t c = tid; c < N; c += nthreads) {
    float A = 0.f, D = 0.f, G = 0.f;
    for (int64_t q = 0; q < a.P; ++q) {
      const float* pq = sp + (size_t)q * 3 * N;
      A += __ldcg(pq + c);
      if (MOD) D += __ldcg(pq + N + c);
      if (GATE == GATE_VEC) G += __ldcg(pq + 2 * N + c);
    }
    float w = a.w_f32 ? reinterpret_cast<const float*>(a.weight)[c]
                      : to_f32(reinterpret_cast<const T*>(a.weight)[c]);
    float s1 = 1.f;
    if (MOD) {
      s1 = 1.f + to_f32(reinterpret_cast<const T*>(a.scale)[b * a.ss + c]);
      reinterpret_cast<T*>(a.dscale)[b * N + c] = from_f32<T>(w * A);
      reinterpret_cast<T*>(a.dshift)[b * N + c] = from_f32<T>(D);
    }
    if (GATE == GATE_VEC) reinterpret_cast<T*>(a.dgate)[b * N + c] = from_f32<T>(G);
    a.dwb[b * N + c] = s1 * A;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) {
    a.tickets[b] = 0u;
    s_ticket = atomicAdd(&a.tickets[a.B], 1u);
  }
  __syncthreads();
  if (s_ticket != (uint32_t)(a.B - 1)) return;
  __threadfence();
  for (int64_t c = tid; c < N; c += nthreads) {
    float s = 0.f;
    for (int64_t q = 0; q < a.B; ++q) s += __ldcg(a.dwb + q * N + c);
    if (a.w_f32) reinterpret_cast<float*>(a.dweight)[c] = s;
    else reinterpret_cast<T*>(a.dweight)[c] = from_f32<T>(s);
  }
  if (tid == 0) a.tickets[a.B] = 0u;
}

// ---------------------------------------------------------------------------
// Launch helpers
// ---------------------------------------------------------------------------
static int g_num_sms = 0;
static int num_sms() {
  if (g_num_sms == 0) {
    int dev = 0;
    cudaGetDevice(&dev);
    cudaDeviceGetAttribute(&g_num_sms, cudaDevAttrMultiProcessorCount, dev);
    if (g_num_sms <= 0) g_num_sms = 148;
  }
  return g_num_sms;
}

static inline int team_warps(int64_t N) { return (int)((N + 511) / 512); }

template <typename T, int GATE, bool MOD, int NW>
static int launch_fwd_warp(const NormFwdArgs& a, cudaStream_t st) {
  const int64_t want = (a.M + 7) / 8;
  const int64_t cap = (int64_t)num_sms() * 8;
  const int grid = (int)(want < cap ? want : cap);
  norm_fwd_warp_kernel<T, GATE, MOD, NW><<<grid < 1 ? 1 : grid, 256, 0, st>>>(a);
  return (int)cudaGetLastError();
}

template <typename T, int GATE, bool MOD>
static int launch_fwd(const NormFwdArgs& a, cudaStream_t st) {
  const int64_t nw = (a.N + 255) / 256;
  if (nw <= 1) return launch_fwd_warp<T, GATE, MOD, 1>(a, st);
  if (nw <= 2) return launch_fwd_warp<T, GATE, MOD, 2>(a, st);
  if (nw <= 4) return launch_fwd_warp<T, GATE, MOD, 4>(a, st);
  if (nw <= 6) return launch_fwd_warp<T, GATE, MOD, 6>(a, st);
  if (nw <= 8) return launch_fwd_warp<T, GATE, MOD, 8>(a, st);
  if (nw <= 12) return launch_fwd_warp<T, GATE, MOD, 12>(a, st);
  if (nw <= 16) return launch_fwd_warp<T, GATE, MOD, 16>(a, st);
  const int K = team_warps(a.N);
  int R = 1;
  while (R * 2 * K * 32 <= 256 && R * 2 <= 8) R *= 2;
  const int threads = R * K * 32;
  int64_t want = (a.M + R - 1) / R;
  int64_t cap = (int64_t)num_sms() * (2048 / threads);
  int grid = (int)(want < cap ? want : cap);
  if (grid < 1) grid = 1;
  size_t sm = (size_t)R * 2 * K * sizeof(float);
  norm_fwd_kernel<T, GATE, MOD><<<grid, threads, sm, st>>>(a, K, R);
  return (int)cudaGetLastError();
}

// Scratch sizes the Python side must provide for a backward call.
NFB_API int64_t nfb_norm_bwd_P(int64_t M, int64_t N, int64_t B) {
  const int64_t T = M / B;
  const int K = team_warps(N);
  int R = 1;
  while (R * 2 * K * 32 <= 512 && R * 2 <= 8 && (size_t)R * 2 * 3 * N * 4 <= 160 * 1024) R *= 2;
  int64_t target = (2 * (int64_t)num_sms() + B - 1) / B;  // ~2 CTAs per SM overall
  int64_t maxP = (T + R - 1) / R;
  int64_t P = target < maxP ? target : maxP;
  return P < 1 ? 1 : P;
}

template <typename T, int GATE, bool MOD>
static int launch_bwd(const NormBwdArgs& a, cudaStream_t st) {
  const int K = team_warps(a.N);
  int R = 1;
  while (R * 2 * K * 32 <= 512 && R * 2 <= 8 && (size_t)R * 2 * 3 * a.N * 4 <= 160 * 1024) R *= 2;
  const int threads = R * K * 32;
  size_t sm = (size_t)(2 * a.N + R * 2 * K) * sizeof(float) + (R > 1 ? (size_t)R * 3 * a.N * sizeof(float) : 0);
  if (sm > 48 * 1024) {
    cudaFuncSetAttribute(norm_bwd_kernel<T, GATE, MOD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  }
  const int grid = (int)(a.B * a.P);
  norm_bwd_kernel<T, GATE, MOD><<<grid, threads, sm, st>>>(a, K, R);
  return (int)cudaGetLastError();
}

template <typename T>
static int dispatch_fwd(const NormFwdArgs& a, int gate, int mod, cudaStream_t st) {
  if (gate == GATE_NONE) return mod ? launch_fwd<T, GATE_NONE, true>(a, st) : launch_fwd<T, GATE_NONE, false>(a, st);
  if (gate == GATE_ONE) return mod ? launch_fwd<T, GATE_ONE, true>(a, st) : launch_fwd<T, GATE_ONE, false>(a, st);
  return mod ? launch_fwd<T, GATE_VEC, true>(a, st) : launch_fwd<T, GATE_VEC, false>(a, st);
}

template <typename T>
static int dispatch_bwd(const NormBwdArgs& a, int gate, int mod, cudaStream_t st) {
  if (gate == GATE_NONE) return mod ? launch_bwd<T, GATE_NONE, true>(a, st) : launch_bwd<T, GATE_NONE, false>(a, st);
  if (gate == GATE_ONE) return mod ? launch_bwd<T, GATE_ONE, true>(a, st) : launch_bwd<T, GATE_ONE, false>(a, st);
  return mod ? launch_bwd<T, GATE_VEC, true>(a, st) : launch_bwd<T, GATE_VEC, false>(a, st);
}

}  // namespace nfb

using namespace nfb;

// Forward. dtype: 1 = bf16, 2 = fp16. Pointers/strides are described in
// NormFwdArgs; every row start and stride must be 16-byte aligned.
NFB_API int nfb_norm_fwd(int dtype, int gate_mode, int mod,
                         const void* x, const void* y, const void* gate, const void* weight,
                         const void* scale, const void* shift,
                         void* h, void* out, float* rstd,
                         int64_t M, int64_t N, int64_t T,
                         int64_t sx, int64_t sy, int64_t sh, int64_t so,
                         int64_t sg, int64_t ss, int64_t ssh,
                         float eps, int w_f32, void* stream) {
  if (N <= 0 || N > 8192 || (N % 8) != 0 || M < 0 || T <= 0) return (int)cudaErrorInvalidValue;
  if (M == 0) return 0;
  NormFwdArgs a{x, y, gate, weight, scale, shift, h, out, rstd, M, N, T, sx, sy, sh, so, sg, ss, ssh, eps, w_f32};
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == kF32) return dispatch_fwd<float>(a, gate_mode, mod, st);
  if (dtype == kBF16) return dispatch_fwd<__nv_bfloat16>(a, gate_mode, mod, st);
  if (dtype == kF16) return dispatch_fwd<__half>(a, gate_mode, mod, st);
  return (int)cudaErrorInvalidValue;
}

NFB_API int nfb_norm_bwd(int dtype, int gate_mode, int mod,
                         const void* dh_up, const void* dout, const void* h, const void* y,
                         const void* gate, const void* weight, const void* scale, const float* rstd,
                         void* dx, void* dy, void* dgate, void* dscale, void* dshift, void* dweight,
                         float* partials, float* dwb, uint32_t* tickets,
                         int64_t M, int64_t N, int64_t T, int64_t P,
                         int64_t s_dhup, int64_t s_dout, int64_t s_h, int64_t s_y, int64_t s_dx, int64_t s_dy,
                         int64_t sg, int64_t ss, int w_f32, void* stream) {
  if (N <= 0 || N > 8192 || (N % 8) != 0 || T <= 0 || M % T != 0 || P <= 0) return (int)cudaErrorInvalidValue;
  if (M == 0) return 0;
  const int64_t B = M / T;
  NormBwdArgs a{dh_up, dout, h, y, gate, weight, scale, rstd, dx, dy, dgate, dscale, dshift, dweight,
                partials, dwb, tickets, M, N, T, B, P, s_dhup, s_dout, s_h, s_y, s_dx, s_dy, sg, ss, w_f32};
  cudaStream_t st = (cudaStream_t)stream;
  if (dtype == kF32) return dispatch_bwd<float>(a, gate_mode, mod, st);
  if (dtype == kBF16) return dispatch_bwd<__nv_bfloat16>(a, gate_mode, mod, st);
  if (dtype == kF16) return dispatch_bwd<__half>(a, gate_mode, mod, st);
  return (int)cudaErrorInvalidValue;
}

NFB_API int nfb_num_sms() { return num_sms(); }

// ===========================================================================
// Allocation-free variant of the norm backward (nfb_norm_bwd_noalloc).
//
// This entry point has no counterpart in the reference implementation.
//
// Who it is for: callers that cannot allocate device memory at the point
// where they run the backward. Examples are a host framework that owns every
// device allocation through a fixed memory plan made before the first step
// (its accounting forbids raw allocations later), and plugin or callback
// code inside another engine whose contract says the call must not allocate,
// because a device allocation can block on work already queued on the GPU.
// nfb_norm_bwd needs the caller to pass scratch buffers (per-CTA partial
// rows, per-sample rows and ticket counters); this variant instead uses one
// file-scope device array of fixed size, so the caller passes only the
// inputs and outputs.
//
// Limit: the scratch holds kNoAllocScratchFloats floats (4 MiB). A call needs
// B*N floats for per-sample rows plus 3*N*B*P floats of CTA partials, with
// P >= 1 CTAs per sample, and B+1 ticket slots (B <= kNoAllocMaxSamples).
// Larger problems are rejected with cudaErrorInvalidValue and a message
// readable through nfb_noalloc_last_error(); the number of CTAs per sample is
// lowered (never below 1) to fit the scratch, which changes only the
// summation grouping, not the result beyond rounding.
//
// Every GPU that loads this library holds the array until the process exits.
// The first call on each device looks up the array's device address with
// cudaGetSymbolAddress while that device is current and caches it; make that
// first call before any stream capture. All calls on a device share the
// array: it keeps the previous call's contents, the ticket counters are
// cleared with cudaMemsetAsync on the call's stream at the start of every
// call, and calls whose executions overlap on the GPU (for example on two
// streams without ordering between them) race on the scratch and give wrong
// results. The call makes no cudaMalloc/cudaFree and no allocating library
// call.
// ===========================================================================
#include <mutex>
#include <stdio.h>

namespace nfb {

constexpr int64_t kNoAllocScratchFloats = 1 << 20;  // 4 MiB of fp32
constexpr int64_t kNoAllocMaxSamples = 1023;        // ticket slots = samples + 1
constexpr int64_t kNoAllocTicketWords = kNoAllocMaxSamples + 1;
constexpr int kNoAllocMaxDevices = 64;

// [0, kNoAllocScratchFloats): partials then per-sample rows; then the tickets.
static __device__ __align__(256) float g_noalloc_scratch[kNoAllocScratchFloats + kNoAllocTicketWords];

static float* g_noalloc_ptr[kNoAllocMaxDevices] = {nullptr};
static std::mutex g_noalloc_mu;
static thread_local char g_noalloc_msg[256] = "";

static int noalloc_fail(int rc, const char* msg) {
  snprintf(g_noalloc_msg, sizeof(g_noalloc_msg), "%s", msg);
  return rc;
}

// Device address of the scratch array for the current device (looked up once per device).
static int noalloc_scratch(float** out) {
  int dev = 0;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return noalloc_fail((int)e, "cudaGetDevice failed");
  if (dev < 0 || dev >= kNoAllocMaxDevices) return noalloc_fail((int)cudaErrorInvalidDevice, "device ordinal too large");
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (g_noalloc_ptr[dev] == nullptr) {
    void* p = nullptr;
    e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr) return noalloc_fail((int)e, "cudaGetSymbolAddress(g_noalloc_scratch) failed");
    g_noalloc_ptr[dev] = static_cast<float*>(p);
  }
  *out = g_noalloc_ptr[dev];
  return 0;
}

}  // namespace nfb

// Message describing why the last nfb_norm_bwd_noalloc call on this host thread failed ("" if none).
NFB_API const char* nfb_noalloc_last_error() { return nfb::g_noalloc_msg; }

// Capacity of the allocation-free scratch, in fp32 elements.
NFB_API int64_t nfb_noalloc_scratch_floats() { return nfb::kNoAllocScratchFloats; }

// Same contract and outputs as nfb_norm_bwd, without the partials/dwb/tickets/P arguments.
NFB_API int nfb_norm_bwd_noalloc(int dtype, int gate_mode, int mod,
                                 const void* dh_up, const void* dout, const void* h, const void* y,
                                 const void* gate, const void* weight, const void* scale, const float* rstd,
                                 void* dx, void* dy, void* dgate, void* dscale, void* dshift, void* dweight,
                                 int64_t M, int64_t N, int64_t T,
                                 int64_t s_dhup, int64_t s_dout, int64_t s_h, int64_t s_y, int64_t s_dx,
                                 int64_t s_dy, int64_t sg, int64_t ss, int w_f32, void* stream) {
  using namespace nfb;
  g_noalloc_msg[0] = '\0';
  if (N <= 0 || N > 8192 || (N % 8) != 0 || T <= 0 || M % T != 0)
    return noalloc_fail((int)cudaErrorInvalidValue, "invalid shape: need 0 < N <= 8192, N % 8 == 0, M % T == 0");
  if (M == 0) return 0;
  const int64_t B = M / T;
  if (B > kNoAllocMaxSamples)
    return noalloc_fail((int)cudaErrorInvalidValue, "too many samples for the allocation-free scratch (max 1023)");
  const int64_t rows_floats = B * N;
  if (rows_floats + 3 * N * B > kNoAllocScratchFloats)
    return noalloc_fail((int)cudaErrorInvalidValue,
                        "problem too large for the allocation-free scratch: need B*N + 3*N*B floats <= 1048576");
  int64_t P = nfb_norm_bwd_P(M, N, B);
  const int64_t p_fit = (kNoAllocScratchFloats - rows_floats) / (3 * N * B);
  if (P > p_fit) P = p_fit;
  float* scratch = nullptr;
  int rc = noalloc_scratch(&scratch);
  if (rc != 0) return rc;
  float* partials = scratch;
  float* dwb = scratch + B * P * 3 * N;
  uint32_t* tickets = reinterpret_cast<uint32_t*>(scratch + kNoAllocScratchFloats);
  cudaStream_t st = (cudaStream_t)stream;
  cudaError_t e = cudaMemsetAsync(tickets, 0, (size_t)(B + 1) * sizeof(uint32_t), st);
  if (e != cudaSuccess) return noalloc_fail((int)e, "cudaMemsetAsync of the ticket counters failed");
  NormBwdArgs a{dh_up, dout, h, y, gate, weight, scale, rstd, dx, dy, dgate, dscale, dshift, dweight,
                partials, dwb, tickets, M, N, T, B, P, s_dhup, s_dout, s_h, s_y, s_dx, s_dy, sg, ss, w_f32};
  if (dtype == kF32) rc = dispatch_bwd<float>(a, gate_mode, mod, st);
  else if (dtype == kBF16) rc = dispatch_bwd<__nv_bfloat16>(a, gate_mode, mod, st);
  else if (dtype == kF16) rc = dispatch_bwd<__half>(a, gate_mode, mod, st);
  else return noalloc_fail((int)cudaErrorInvalidValue, "unsupported dtype code");
  if (rc != 0) return noalloc_fail(rc, "kernel launch failed");
  return 0;
}
