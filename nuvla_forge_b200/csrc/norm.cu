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

// 8 consecutive fp32 values of a shared-memory row as two 16-byte loads (zeros past N): with
// each lane reading its own 32 bytes, scalar loads would hit the same banks 8 ways.
__device__ __forceinline__ void lds8(const float* row, int64_t col, int64_t N, float* out) {
  if (col < N) {
    const float4 a = *reinterpret_cast<const float4*>(row + col);
    const float4 b = *reinterpret_cast<const float4*>(row + col + 4);
    out[0] = a.x; out[1] = a.y; out[2] = a.z; out[3] = a.w;
    out[4] = b.x; out[5] = b.y; out[6] = b.z; out[7] = b.w;
  } else {
#pragma unroll
    for (int j = 0; j < 8; ++j) out[j] = 0.f;
  }
}

// 8 elements held as raw loaded vectors (16 bytes for 16-bit types, 32 for fp32); zeros past N or
// for a null row.
template <typename T>
struct RawChunk {
  uint4 u[sizeof(T) == 2 ? 1 : 2];
  __device__ __forceinline__ void load(const T* base, int64_t col, int64_t N) {
    if (base != nullptr && col < N) {
      u[0] = *reinterpret_cast<const uint4*>(base + col);
      if (sizeof(T) == 4) u[sizeof(T) == 2 ? 0 : 1] = *reinterpret_cast<const uint4*>(base + col + 4);
    } else {
#pragma unroll
      for (int k = 0; k < (sizeof(T) == 2 ? 1 : 2); ++k) u[k] = make_uint4(0u, 0u, 0u, 0u);
    }
  }
  __device__ __forceinline__ void get(float* out) const {
    unpack16<T>(u[0], out);
    if (sizeof(T) == 4) unpack16<T>(u[sizeof(T) == 2 ? 0 : 1], out + 4);
  }
};

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
    float yv[GATE != GATE_NONE ? NW : 1][8];
    float ss = 0.f;
    // every load of the row is issued before the first store: the compiler may not move a load
    // across a store that could alias it, which would serialise one round trip per chunk
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      const int64_t col = ((int64_t)i * 32 + lane) * 8;
      load_chunk<T>(reinterpret_cast<const T*>(a.x) + row * a.sx, col, N, hv[i]);
      if (GATE != GATE_NONE) load_chunk<T>(reinterpret_cast<const T*>(a.y) + row * a.sy, col, N, yv[i % (GATE != GATE_NONE ? NW : 1)]);
    }
#pragma unroll
    for (int i = 0; i < NW; ++i) {
      const int64_t col = ((int64_t)i * 32 + lane) * 8;
      if (GATE != GATE_NONE) {
        const float* y8 = yv[i % (GATE != GATE_NONE ? NW : 1)];
        if (GATE == GATE_VEC) {
          float gv[8];
          load_chunk<T>(reinterpret_cast<const T*>(a.gate) + b * a.sg, col, N, gv);
#pragma unroll
          for (int j = 0; j < 8; ++j) hv[i][j] += gv[j] * y8[j];
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) hv[i][j] += y8[j];
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
    // Every HBM load of the row (dout, h, and pass 2's dh_up and y) is issued here, before the
    // team barrier and before any store: a load may not be moved across a store that could alias
    // it, so HBM loads issued after the first store would each cost a serial round trip.
    // (kept as raw 16-byte vectors until used, to spare registers)
    RawChunk<T> dhv[NV], yv[GATE == GATE_VEC ? NV : 1];
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = ((int64_t)i * K * 32 + tt) * 8;
      dhv[i].load(a.dh_up != nullptr ? reinterpret_cast<const T*>(a.dh_up) + row * a.s_dhup : nullptr, col, N);
      if (GATE == GATE_VEC)
        yv[i % (GATE == GATE_VEC ? NV : 1)].load(reinterpret_cast<const T*>(a.y) + row * a.s_y, col, N);
    }
    // pass 1: row dot product and the per-column accumulators
    float dot = 0.f;
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = ((int64_t)i * K * 32 + tt) * 8;
      float dv[8], hv[8];
      load_chunk<T>(dout_r, col, N, dv);
      load_chunk<T>(h_r, col, N, hv);
      float w8[8];
      lds8(ws_s, col, N, w8);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = hv[j] * rstd;
        dot += dv[j] * w8[j] * xh;
        accA[i * 8 + j] += dv[j] * xh;
        if (MOD) accD[i * 8 + j] += dv[j];
      }
    }
    dot = team_sum(dot, red, parity, wt, K, bar_id) * invN;
    parity ^= 1;
    // pass 2: dout and h are re-read (L1-resident; a reload after a store costs an L1 round trip only)
#pragma unroll
    for (int i = 0; i < NV; ++i) {
      const int64_t col = ((int64_t)i * K * 32 + tt) * 8;
      if (col >= N) continue;
      float dv[8], hv[8], dh[8];
      load8<T>(dout_r + col, dv);
      load8<T>(h_r + col, hv);
      dhv[i].get(dh);
      float w8[8];
      lds8(ws_s, col, N, w8);
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float xh = hv[j] * rstd;
        dh[j] += rstd * (dv[j] * w8[j] - xh * dot);
      }
      store8<T>(reinterpret_cast<T*>(a.dx) + row * a.s_dx + col, dh);
      if (GATE == GATE_VEC) {
        float dyv[8], y8[8];
        yv[i % (GATE == GATE_VEC ? NV : 1)].get(y8);
#pragma unroll
        float g8[8];
        lds8(gv_s, col, N, g8);
        for (int j = 0; j < 8; ++j) {
          dyv[j] = dh[j] * g8[j];
          accG[i * 8 + j] += dh[j] * y8[j];
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
  // Sum of the sample's P partial rows in a fixed order. A column quad (four columns, one 16-byte
  // load per partial row) is shared by S consecutive lanes, lane s taking rows s, s + S, ... into
  // four interleaved sums; a butterfly of shuffles then adds the S lane sums. With one sample
  // (P = 2 x SMs rows) the single last CTA otherwise waits on P / 4 dependent L2 round trips per
  // column.
  const int64_t nq4 = N / 4;
  int S = 1;
  while (S < 8 && nq4 * S * 2 <= nthreads) S *= 2;
  auto fold4 = [&](int64_t off, int s, bool live) -> float4 {
    float4 acc[4];
#pragma unroll
    for (int k = 0; k < 4; ++k) acc[k] = make_float4(0.f, 0.f, 0.f, 0.f);
    if (live) {
      const float* base = sp + off;
      const size_t rs = (size_t)3 * N;
      int64_t q = s;
      for (; q + 3 * S < a.P; q += 4 * S) {
#pragma unroll
        for (int k = 0; k < 4; ++k) {
          const float4 v = __ldcg(reinterpret_cast<const float4*>(base + (size_t)(q + k * S) * rs));
          acc[k].x += v.x; acc[k].y += v.y; acc[k].z += v.z; acc[k].w += v.w;
        }
      }
      for (; q < a.P; q += S) {
        const float4 v = __ldcg(reinterpret_cast<const float4*>(base + (size_t)q * rs));
        acc[0].x += v.x; acc[0].y += v.y; acc[0].z += v.z; acc[0].w += v.w;
      }
    }
    float4 r;
    r.x = (acc[0].x + acc[1].x) + (acc[2].x + acc[3].x);
    r.y = (acc[0].y + acc[1].y) + (acc[2].y + acc[3].y);
    r.z = (acc[0].z + acc[1].z) + (acc[2].z + acc[3].z);
    r.w = (acc[0].w + acc[1].w) + (acc[2].w + acc[3].w);
    // lanes of one quad are S consecutive lanes of one warp (S divides 32)
    for (int o = 1; o < S; o <<= 1) {
      r.x += __shfl_xor_sync(0xffffffffu, r.x, o);
      r.y += __shfl_xor_sync(0xffffffffu, r.y, o);
      r.z += __shfl_xor_sync(0xffffffffu, r.z, o);
      r.w += __shfl_xor_sync(0xffffffffu, r.w, o);
    }
    return r;
  };
  // the loop bound is padded to whole warps (nthreads is a multiple of 32), so every lane of a
  // warp runs the same iterations and the shuffles see the full warp
  const int64_t items = nq4 * S, items_pad = (items + 31) / 32 * 32;
  for (int64_t it = tid; it < items_pad; it += nthreads) {
    const bool live = it < items;
    const int64_t c0 = (it / S) * 4;
    const int s = (int)(it % S);
    const float4 A4 = fold4(c0, s, live);
    const float4 D4 = MOD ? fold4(N + c0, s, live) : make_float4(0.f, 0.f, 0.f, 0.f);
    const float4 G4 = GATE == GATE_VEC ? fold4(2 * N + c0, s, live) : make_float4(0.f, 0.f, 0.f, 0.f);
    if (!live || s != 0) continue;
    const float Av[4] = {A4.x, A4.y, A4.z, A4.w}, Dv[4] = {D4.x, D4.y, D4.z, D4.w};
    const float Gv[4] = {G4.x, G4.y, G4.z, G4.w};
#pragma unroll
    for (int j = 0; j < 4; ++j) {
      const int64_t c = c0 + j;
      float w = a.w_f32 ? reinterpret_cast<const float*>(a.weight)[c]
                        : to_f32(reinterpret_cast<const T*>(a.weight)[c]);
      float s1 = 1.f;
      if (MOD) {
        s1 = 1.f + to_f32(reinterpret_cast<const T*>(a.scale)[b * a.ss + c]);
        reinterpret_cast<T*>(a.dscale)[b * N + c] = from_f32<T>(w * Av[j]);
        reinterpret_cast<T*>(a.dshift)[b * N + c] = from_f32<T>(Dv[j]);
      }
      if (GATE == GATE_VEC) reinterpret_cast<T*>(a.dgate)[b * N + c] = from_f32<T>(Gv[j]);
      a.dwb[b * N + c] = s1 * Av[j];
    }
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
    float s0 = 0.f, s1 = 0.f, s2 = 0.f, s3 = 0.f;
    int64_t q = 0;
    for (; q + 4 <= a.B; q += 4) {
      s0 += __ldcg(a.dwb + q * N + c);
      s1 += __ldcg(a.dwb + (q + 1) * N + c);
      s2 += __ldcg(a.dwb + (q + 2) * N + c);
      s3 += __ldcg(a.dwb + (q + 3) * N + c);
    }
    for (; q < a.B; ++q) s0 += __ldcg(a.dwb + q * N + c);
    const float s = (s0 + s1) + (s2 + s3);
    if (a.w_f32) reinterpret_cast<float*>(a.dweight)[c] = s;
    else reinterpret_cast<T*>(a.dweight)[c] = from_f32<T>(s);
  }
  if (tid == 0) a.tickets[a.B] = 0u;
}

// ---------------------------------------------------------------------------
// Bulk-copy pipelined kernels (N % 8 == 0, 16-byte aligned rows)
//
// One producer thread streams whole rows of every input tensor into a
// shared-memory ring of up to kStagesMax stages with 1-D bulk async copies
// (cp.async.bulk ... mbarrier::complete_tx; no multicast), so the bytes in
// flight per SM do not depend on registers. A stage holds G rows; thread group
// g (nt threads) owns row g of every stage and NV2 fixed 8-column chunks of
// it for the whole kernel, so per-column accumulators stay in registers. The
// forward walks a contiguous block range per CTA and caches the per-sample
// coefficients in registers; the backward prefetches its rows' rstd into
// shared memory. Selected with nfb_norm_set_impl(1); the warp/team kernels
// stay the default (see g_norm_impl for the measured comparison).
// ---------------------------------------------------------------------------
constexpr int kStagesMax = 8;
constexpr uint64_t kCopyWaitNs = 2000000000ull;

__device__ __forceinline__ uint32_t s_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

__device__ __forceinline__ void bar_init(uint64_t* b, uint32_t n) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(s_u32(b)), "r"(n) : "memory");
}
__device__ __forceinline__ void bar_expect(uint64_t* b, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(s_u32(b)), "r"(bytes) : "memory");
}
__device__ __forceinline__ bool bar_try(uint64_t* b, uint32_t parity) {
  uint32_t ok;
  asm volatile("{\n\t.reg .pred p;\n\tmbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\tselp.u32 %0, 1, 0, p;\n\t}"
               : "=r"(ok) : "r"(s_u32(b)), "r"(parity) : "memory");
  return ok != 0;
}
__device__ __forceinline__ bool bar_wait(uint64_t* b, uint32_t parity) {
  if (bar_try(b, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  while (!bar_try(b, parity)) {
    if (globaltimer_ns() - t0 > kCopyWaitNs) return false;
  }
  return true;
}
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* b) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(s_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(s_u32(b)) : "memory");
}

struct TmaGeom { int G; int stages; int nt; int rcap; };  // rows (= thread groups) per stage, stages, threads per group, rstd slots

// ---------------- forward ----------------
// Group g (nt threads) owns row g of every stage; one CTA barrier per stage.
template <typename T, int GATE, bool MOD, int NV2>
__global__ void __launch_bounds__(512, 1) norm_fwd_tma_kernel(NormFwdArgs a, TmaGeom g, uint32_t* status) {
  extern __shared__ __align__(128) uint8_t tsmem[];
  const int64_t N = a.N;
  const int ntens = GATE != GATE_NONE ? 2 : 1;
  const size_t rowb = (size_t)N * sizeof(T);
  const size_t stage_b = (size_t)g.G * ntens * rowb;
  uint64_t* full = reinterpret_cast<uint64_t*>(tsmem + (size_t)g.stages * stage_b);
  float* red = reinterpret_cast<float*>(full + kStagesMax);           // [G][warps per group]
  __shared__ int s_abort;
  const int tid = threadIdx.x;
  const int grp = tid / g.nt, lt = tid % g.nt, wpg = g.nt >> 5, wl = lt >> 5;
  const int64_t nblocks = (a.M + g.G - 1) / g.G;
  if (tid == 0) {
    for (int s = 0; s < g.stages; ++s) bar_init(&full[s], 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  auto issue = [&](int64_t blk, int stage) {
    const int64_t r0 = blk * g.G;
    const int rows = (int)min((int64_t)g.G, a.M - r0);
    bar_expect(&full[stage], (uint32_t)(rows * ntens * rowb));
    uint8_t* st = tsmem + (size_t)stage * stage_b;
    for (int r = 0; r < rows; ++r) {
      bulk_g2s(st + (size_t)(r * ntens) * rowb, reinterpret_cast<const T*>(a.x) + (r0 + r) * a.sx, (uint32_t)rowb, &full[stage]);
      if (GATE != GATE_NONE)
        bulk_g2s(st + (size_t)(r * ntens + 1) * rowb, reinterpret_cast<const T*>(a.y) + (r0 + r) * a.sy, (uint32_t)rowb, &full[stage]);
    }
  };
  // contiguous block range per CTA, so the per-sample coefficients change rarely
  const int64_t blk0 = nblocks * blockIdx.x / gridDim.x, blk1 = nblocks * (blockIdx.x + 1) / gridDim.x;
  if (tid == 0)
    for (int s = 0; s < g.stages; ++s)
      if (blk0 + s < blk1) issue(blk0 + s, s);
  constexpr bool kCache = NV2 <= 2;   // per-thread copies of weight*(1+scale), shift, gate for the current sample
  float cw[kCache ? NV2 * 8 : 1], csf[(kCache && MOD) ? NV2 * 8 : 1], cg[(kCache && GATE == GATE_VEC) ? NV2 * 8 : 1];
  int64_t cb = -1;
  int64_t i = 0;
  for (int64_t blk = blk0; blk < blk1; ++blk, ++i) {
    const int stage = (int)(i % g.stages);
    if (!bar_wait(&full[stage], (uint32_t)((i / g.stages) & 1))) {
      if (tid == 0) { set_status(status, kTimeoutFlag, 20); s_abort = 1; }
    }
    __syncthreads();
    if (s_abort) break;
    const int64_t row = blk * g.G + grp;
    const bool active = row < a.M;
    const T* st = reinterpret_cast<const T*>(tsmem + (size_t)stage * stage_b) + (size_t)(grp * ntens) * N;
    const int64_t b = active ? row / a.T : 0;
    if (kCache && active && b != cb) {
      cb = b;
#pragma unroll
      for (int c = 0; c < NV2; ++c) {
        const int64_t col = ((int64_t)c * g.nt + lt) * 8;
        if (col >= N) continue;
        float wv[8];
        load_weight_chunk<T>(a.weight, a.w_f32, col, N, wv);
        if (MOD) {
          float sc[8], sf[8];
          load8<T>(reinterpret_cast<const T*>(a.scale) + b * a.ss + col, sc);
          load8<T>(reinterpret_cast<const T*>(a.shift) + b * a.ssh + col, sf);
#pragma unroll
          for (int j = 0; j < 8; ++j) { wv[j] *= 1.f + sc[j]; csf[(c * 8 + j) % (MOD ? NV2 * 8 : 1)] = sf[j]; }
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) cw[(c * 8 + j) % (kCache ? NV2 * 8 : 1)] = wv[j];
        if (GATE == GATE_VEC) {
          float gv[8];
          load8<T>(reinterpret_cast<const T*>(a.gate) + b * a.sg + col, gv);
#pragma unroll
          for (int j = 0; j < 8; ++j) cg[(c * 8 + j) % (GATE == GATE_VEC ? NV2 * 8 : 1)] = gv[j];
        }
      }
    }
    float h[NV2][8];
    float ss = 0.f;
#pragma unroll
    for (int c = 0; c < NV2; ++c) {
      const int64_t col = ((int64_t)c * g.nt + lt) * 8;
      if (!active || col >= N) {
#pragma unroll
        for (int j = 0; j < 8; ++j) h[c][j] = 0.f;
        continue;
      }
      load8<T>(st + col, h[c]);
      if (GATE != GATE_NONE) {
        float yv[8];
        load8<T>(st + N + col, yv);
        if (GATE == GATE_VEC) {
          float gv[8];
          if (kCache) {
#pragma unroll
            for (int j = 0; j < 8; ++j) gv[j] = cg[(c * 8 + j) % (kCache && GATE == GATE_VEC ? NV2 * 8 : 1)];
          } else {
            load8<T>(reinterpret_cast<const T*>(a.gate) + b * a.sg + col, gv);
          }
#pragma unroll
          for (int j = 0; j < 8; ++j) h[c][j] += gv[j] * yv[j];
        } else {
#pragma unroll
          for (int j = 0; j < 8; ++j) h[c][j] += yv[j];
        }
        round8<T>(h[c]);
        store8<T>(reinterpret_cast<T*>(a.h) + row * a.sh + col, h[c]);
      }
#pragma unroll
      for (int j = 0; j < 8; ++j) ss += h[c][j] * h[c][j];
    }
    ss = warp_sum(ss);
    if ((lt & 31) == 0) red[grp * wpg + wl] = ss;
    __syncthreads();   // row sums visible; every thread is done reading this stage
    if (tid == 0 && blk + g.stages < blk1) issue(blk + g.stages, stage);
    float tot = 0.f;
    for (int w = 0; w < wpg; ++w) tot += red[grp * wpg + w];
    if (active) {
      const float rstd = rsqrtf(tot / (float)N + a.eps);
      if (lt == 0) a.rstd[row] = rstd;
#pragma unroll
      for (int c = 0; c < NV2; ++c) {
        const int64_t col = ((int64_t)c * g.nt + lt) * 8;
        if (col >= N) continue;
        float o[8];
        if (kCache) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            const int q = (c * 8 + j) % (kCache ? NV2 * 8 : 1);
            o[j] = h[c][j] * rstd * cw[q] + (MOD ? csf[q % (MOD ? NV2 * 8 : 1)] : 0.f);
          }
        } else {
          float wv[8];
          load_weight_chunk<T>(a.weight, a.w_f32, col, N, wv);
          if (MOD) {
            float sc[8], sf[8];
            load8<T>(reinterpret_cast<const T*>(a.scale) + b * a.ss + col, sc);
            load8<T>(reinterpret_cast<const T*>(a.shift) + b * a.ssh + col, sf);
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = h[c][j] * rstd * (wv[j] * (1.f + sc[j])) + sf[j];
          } else {
#pragma unroll
            for (int j = 0; j < 8; ++j) o[j] = h[c][j] * rstd * wv[j];
          }
        }
        store8<T>(reinterpret_cast<T*>(a.out) + row * a.so + col, o);
      }
    }
    __syncthreads();   // red[] reuse
  }
  if (tid == 0) {
    for (int s = 0; s < g.stages; ++s) {
      const int64_t k = i + s;
      if (blk0 + k >= blk1) break;
      const uint64_t t0 = globaltimer_ns();
      while (!bar_try(&full[k % g.stages], (uint32_t)((k / g.stages) & 1))) {
        if (globaltimer_ns() - t0 > kCopyWaitNs) break;
      }
    }
  }
}

// ---------------- backward ----------------
template <typename T, int GATE, bool MOD, int NV2>
__global__ void __launch_bounds__(512, 1) norm_bwd_tma_kernel(NormBwdArgs a, TmaGeom g, uint32_t* status) {
  extern __shared__ __align__(128) uint8_t tsmem[];
  const int64_t N = a.N;
  const bool has_up = a.dh_up != nullptr;
  const int ntens = 2 + (has_up ? 1 : 0) + (GATE == GATE_VEC ? 1 : 0);
  const int i_up = 2, i_y = has_up ? 3 : 2;
  const size_t rowb = (size_t)N * sizeof(T);
  const size_t stage_b = (size_t)g.G * ntens * rowb;
  uint64_t* full = reinterpret_cast<uint64_t*>(tsmem + (size_t)g.stages * stage_b);
  float* red = reinterpret_cast<float*>(full + kStagesMax);       // [G][warps per group]
  float* ws_s = red + 32;                                          // [N]
  float* gv_s = ws_s + N;                                          // [N]
  float* rs_s = gv_s + N;                                          // [g.rcap] rstd of this CTA's rows
  __shared__ int s_abort;
  __shared__ uint32_t s_ticket;
  const int tid = threadIdx.x;
  const int grp = tid / g.nt, lt = tid % g.nt, wpg = g.nt >> 5, wl = lt >> 5;
  const int64_t b = blockIdx.x / a.P, p = blockIdx.x % a.P;
  const int64_t nblk_s = (a.T + g.G - 1) / g.G;
  for (int64_t c = tid; c < N; c += blockDim.x) {
    const float w = a.w_f32 ? reinterpret_cast<const float*>(a.weight)[c] : to_f32(reinterpret_cast<const T*>(a.weight)[c]);
    const float s1 = MOD ? 1.f + to_f32(reinterpret_cast<const T*>(a.scale)[b * a.ss + c]) : 1.f;
    ws_s[c] = w * s1;
    gv_s[c] = (GATE == GATE_VEC) ? to_f32(reinterpret_cast<const T*>(a.gate)[b * a.sg + c]) : 1.f;
  }
  const int64_t my_blocks = nblk_s > p ? (nblk_s - p + a.P - 1) / a.P : 0;
  const bool rs_pre = my_blocks * g.G <= g.rcap;
  if (rs_pre)
    for (int64_t e = tid; e < my_blocks * g.G; e += blockDim.x) {
      const int64_t t = (p + (e / g.G) * a.P) * g.G + e % g.G;
      rs_s[e] = t < a.T ? a.rstd[b * a.T + t] : 0.f;
    }
  if (tid == 0) {
    for (int s = 0; s < g.stages; ++s) bar_init(&full[s], 1);
    s_abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  __syncthreads();
  auto issue = [&](int64_t kb, int stage) {
    const int64_t t0 = kb * g.G;
    const int rows = (int)min((int64_t)g.G, a.T - t0);
    bar_expect(&full[stage], (uint32_t)(rows * ntens * rowb));
    uint8_t* st = tsmem + (size_t)stage * stage_b;
    for (int r = 0; r < rows; ++r) {
      const int64_t row = b * a.T + t0 + r;
      uint8_t* d = st + (size_t)(r * ntens) * rowb;
      bulk_g2s(d, reinterpret_cast<const T*>(a.dout) + row * a.s_dout, (uint32_t)rowb, &full[stage]);
      bulk_g2s(d + rowb, reinterpret_cast<const T*>(a.h) + row * a.s_h, (uint32_t)rowb, &full[stage]);
      if (has_up) bulk_g2s(d + (size_t)i_up * rowb, reinterpret_cast<const T*>(a.dh_up) + row * a.s_dhup, (uint32_t)rowb, &full[stage]);
      if (GATE == GATE_VEC) bulk_g2s(d + (size_t)i_y * rowb, reinterpret_cast<const T*>(a.y) + row * a.s_y, (uint32_t)rowb, &full[stage]);
    }
  };
  float accA[NV2 * 8], accD[NV2 * 8], accG[NV2 * 8];
#pragma unroll
  for (int j = 0; j < NV2 * 8; ++j) { accA[j] = 0.f; accD[j] = 0.f; accG[j] = 0.f; }
  const float invN = 1.f / (float)N;
  if (tid == 0)
    for (int s = 0; s < g.stages; ++s)
      if (p + (int64_t)s * a.P < nblk_s) issue(p + (int64_t)s * a.P, s);
  int64_t i = 0;
  for (int64_t kb = p; kb < nblk_s; kb += a.P, ++i) {
    const int stage = (int)(i % g.stages);
    if (!bar_wait(&full[stage], (uint32_t)((i / g.stages) & 1))) {
      if (tid == 0) { set_status(status, kTimeoutFlag, 21); s_abort = 1; }
    }
    __syncthreads();
    if (s_abort) break;
    const int64_t t = kb * g.G + grp;
    const bool active = t < a.T;
    const int64_t row = b * a.T + t;
    const T* st = reinterpret_cast<const T*>(tsmem + (size_t)stage * stage_b) + (size_t)(grp * ntens) * N;
    const float rstd = !active ? 0.f : rs_pre ? rs_s[i * g.G + grp] : a.rstd[row];
    float dot = 0.f;
    if (active) {
#pragma unroll
      for (int c = 0; c < NV2; ++c) {
        const int64_t col = ((int64_t)c * g.nt + lt) * 8;
        if (col >= N) continue;
        float dv[8], hv[8];
        load8<T>(st + col, dv);
        load8<T>(st + N + col, hv);
#pragma unroll
        for (int j = 0; j < 8; ++j) {
          const float xh = hv[j] * rstd;
          dot += dv[j] * ws_s[col + j] * xh;
          accA[c * 8 + j] += dv[j] * xh;
          if (MOD) accD[c * 8 + j] += dv[j];
        }
      }
    }
    dot = warp_sum(dot);
    if ((lt & 31) == 0) red[grp * wpg + wl] = dot;
    __syncthreads();
    float tot = 0.f;
    for (int w = 0; w < wpg; ++w) tot += red[grp * wpg + w];
    const float d_r = tot * invN;
    if (active) {
#pragma unroll
      for (int c = 0; c < NV2; ++c) {
        const int64_t col = ((int64_t)c * g.nt + lt) * 8;
        if (col >= N) continue;
        float dv[8], hv[8], dh[8];
        load8<T>(st + col, dv);
        load8<T>(st + N + col, hv);
        if (has_up) load8<T>(st + (size_t)i_up * N + col, dh);
        else {
#pragma unroll
          for (int j = 0; j < 8; ++j) dh[j] = 0.f;
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) dh[j] += rstd * (dv[j] * ws_s[col + j] - hv[j] * rstd * d_r);
        store8<T>(reinterpret_cast<T*>(a.dx) + row * a.s_dx + col, dh);
        if (GATE == GATE_VEC) {
          float yv[8], dyv[8];
          load8<T>(st + (size_t)i_y * N + col, yv);
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            dyv[j] = dh[j] * gv_s[col + j];
            accG[c * 8 + j] += dh[j] * yv[j];
          }
          store8<T>(reinterpret_cast<T*>(a.dy) + row * a.s_dy + col, dyv);
        } else if (GATE == GATE_ONE && a.dy != nullptr) {
          store8<T>(reinterpret_cast<T*>(a.dy) + row * a.s_dy + col, dh);
        }
      }
    }
    __syncthreads();    // stage and red[] free
    if (tid == 0 && kb + (int64_t)g.stages * a.P < nblk_s) issue(kb + (int64_t)g.stages * a.P, stage);
  }
  if (tid == 0) {
    for (int s = 0; s < g.stages; ++s) {
      const int64_t k = i + s;
      if (p + k * a.P >= nblk_s) break;
      const uint64_t t0 = globaltimer_ns();
      while (!bar_try(&full[k % g.stages], (uint32_t)((k / g.stages) & 1))) {
        if (globaltimer_ns() - t0 > kCopyWaitNs) break;
      }
    }
  }
  __syncthreads();
  if (s_abort) return;
  // fold the groups' column accumulators in shared memory (group order fixed), then write the CTA partial
  float* fold = reinterpret_cast<float*>(tsmem);    // stages are drained: reuse as [G][3][N]
#pragma unroll
  for (int c = 0; c < NV2; ++c) {
    const int64_t col = ((int64_t)c * g.nt + lt) * 8;
    if (col >= N) continue;
    float* f = fold + (size_t)grp * 3 * N;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
      f[col + j] = accA[c * 8 + j];
      f[N + col + j] = accD[c * 8 + j];
      f[2 * N + col + j] = accG[c * 8 + j];
    }
  }
  __syncthreads();
  float* part = a.partials + (size_t)blockIdx.x * 3 * N;
  for (int64_t e = tid; e < 3 * N; e += blockDim.x) {
    float v = 0.f;
    for (int q = 0; q < g.G; ++q) v += fold[(size_t)q * 3 * N + e];
    part[e] = v;
  }
  __threadfence();
  __syncthreads();
  if (tid == 0) s_ticket = atomicAdd(&a.tickets[b], 1u);
  __syncthreads();
  if (s_ticket != (uint32_t)(a.P - 1)) return;
  __threadfence();
  const float* sp = a.partials + (size_t)b * a.P * 3 * N;
  for (int64_t c = tid; c < N; c += blockDim.x) {
    float A = 0.f, D = 0.f, Gs = 0.f;
    for (int64_t q = 0; q < a.P; ++q) {
      const float* pq = sp + (size_t)q * 3 * N;
      A += __ldcg(pq + c);
      if (MOD) D += __ldcg(pq + N + c);
      if (GATE == GATE_VEC) Gs += __ldcg(pq + 2 * N + c);
    }
    const float w = a.w_f32 ? reinterpret_cast<const float*>(a.weight)[c] : to_f32(reinterpret_cast<const T*>(a.weight)[c]);
    float s1 = 1.f;
    if (MOD) {
      s1 = 1.f + to_f32(reinterpret_cast<const T*>(a.scale)[b * a.ss + c]);
      reinterpret_cast<T*>(a.dscale)[b * N + c] = from_f32<T>(w * A);
      reinterpret_cast<T*>(a.dshift)[b * N + c] = from_f32<T>(D);
    }
    if (GATE == GATE_VEC) reinterpret_cast<T*>(a.dgate)[b * N + c] = from_f32<T>(Gs);
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
  for (int64_t c = tid; c < N; c += blockDim.x) {
    float sacc = 0.f;
    for (int64_t q = 0; q < a.B; ++q) sacc += __ldcg(a.dwb + q * N + c);
    if (a.w_f32) reinterpret_cast<float*>(a.dweight)[c] = sacc;
    else reinterpret_cast<T*>(a.dweight)[c] = from_f32<T>(sacc);
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

static inline int nv2_for(int64_t N) { return (int)((N / 8 + 255) / 256); }

constexpr size_t kSmemCap = 227 * 1024;   // opt-in dynamic shared memory per CTA

static size_t tma_smem(const TmaGeom& g, int64_t N, size_t esize, int ntens, bool bwd) {
  size_t stages = (size_t)g.stages * g.G * ntens * N * esize;
  if (bwd && stages < (size_t)g.G * 3 * N * 4) stages = (size_t)g.G * 3 * N * 4;
  return stages + kStagesMax * 8 + 32 * 4 + (bwd ? (2 * N + g.rcap) * 4 : 0) + 128;
}

// Rows per stage G (one thread group of nt threads each, G * nt <= 512) and
// the stage count that fit about 150 KB of staging; stages == 0 when even two
// single-row stages do not fit in shared memory.
static TmaGeom tma_geom(int64_t N, size_t esize, int ntens, bool bwd) {
  TmaGeom g;
  const int nv2 = nv2_for(N);
  const int64_t chunks = (N / 8 + nv2 - 1) / nv2;
  g.nt = (int)((chunks + 31) / 32 * 32);
  g.rcap = bwd ? 2048 : 0;
  int G = 512 / g.nt;
  G = G < 1 ? 1 : (G > 8 ? 8 : G);
  const size_t row_set = (size_t)ntens * N * esize;
  while (G > 1 && 2 * (size_t)G * row_set > 150 * 1024) G >>= 1;
  for (;; G >>= 1) {
    g.G = G;
    int st = (int)(150 * 1024 / ((size_t)G * row_set));
    if (bwd) {   // the stage area is reused to fold G x 3 x N fp32 accumulators at the end
      const size_t need = (size_t)G * 3 * N * 4;
      while ((size_t)st * G * row_set < need) ++st;
    }
    g.stages = st < 2 ? 2 : (st > kStagesMax ? kStagesMax : st);
    if (tma_smem(g, N, esize, ntens, bwd) <= kSmemCap) return g;
    if (G == 1) break;
  }
  g.stages = 0;
  return g;
}

// Device status word (per device) for the pipelined kernels' bounded waits; nonzero after a copy timed out.
static uint32_t* g_status_dev[64] = {};
NFB_API void nfb_norm_set_status(uint32_t* status) {
  int d = 0;
  cudaGetDevice(&d);
  if (d >= 0 && d < 64) g_status_dev[d] = status;
}
static uint32_t* cur_status() {
  int d = 0;
  cudaGetDevice(&d);
  return (d >= 0 && d < 64) ? g_status_dev[d] : nullptr;
}
// 0 (default): register-resident warp/team kernels. 1: bulk-copy pipelined kernels where the rows
// allow them. Measured on B200 (adaLN fwd+bwd, B8 x T2048 x N1536 bf16): 0.297 ms for 0 against
// 0.469 ms for 1 -- with one CTA of 12 warps per SM the pipelined kernels stall on issue latency and
// per-stage barriers (ncu: "wait", "barrier" and "short scoreboard" stalls, DRAM 21%), while the
// warp/team kernels keep 32+ warps per SM loading straight into registers.
static int g_norm_impl = 0;
NFB_API void nfb_norm_set_impl(int impl) { g_norm_impl = impl; }
NFB_API int nfb_norm_get_impl() { return g_norm_impl; }

static inline bool al16(const void* p, int64_t stride_elems, size_t es) {
  return p == nullptr || (((reinterpret_cast<uintptr_t>(p) & 15) == 0) && ((stride_elems * (int64_t)es) % 16 == 0));
}
template <typename T>
static bool tma_ok_fwd(const NormFwdArgs& a, int gate) {
  return g_norm_impl == 1 && a.N % 8 == 0 && a.N <= 8192 && al16(a.x, a.sx, sizeof(T)) && al16(a.y, a.sy, sizeof(T)) &&
         tma_geom(a.N, sizeof(T), gate != GATE_NONE ? 2 : 1, false).stages > 0;
}
template <typename T>
static bool tma_ok_bwd(const NormBwdArgs& a, int gate) {
  return g_norm_impl == 1 && a.N % 8 == 0 && a.N <= 8192 && al16(a.dout, a.s_dout, sizeof(T)) && al16(a.h, a.s_h, sizeof(T)) &&
         al16(a.dh_up, a.s_dhup, sizeof(T)) && al16(a.y, a.s_y, sizeof(T)) &&
         tma_geom(a.N, sizeof(T), 2 + (a.dh_up ? 1 : 0) + (gate == GATE_VEC ? 1 : 0), true).stages > 0;
}

template <typename T, int GATE, bool MOD, int NV2>
static int launch_fwd_tma(const NormFwdArgs& a, cudaStream_t st) {
  const int ntens = GATE != GATE_NONE ? 2 : 1;
  TmaGeom g = tma_geom(a.N, sizeof(T), ntens, false);
  const size_t sm = tma_smem(g, a.N, sizeof(T), ntens, false);
  cudaFuncSetAttribute(norm_fwd_tma_kernel<T, GATE, MOD, NV2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  const int64_t nblocks = (a.M + g.G - 1) / g.G;
  const int grid = (int)(nblocks < num_sms() ? nblocks : num_sms());
  norm_fwd_tma_kernel<T, GATE, MOD, NV2><<<grid, g.G * g.nt, sm, st>>>(a, g, cur_status());
  return (int)cudaGetLastError();
}

template <typename T, int GATE, bool MOD, int NV2>
static int launch_bwd_tma(const NormBwdArgs& a, cudaStream_t st) {
  const int ntens = 2 + (a.dh_up ? 1 : 0) + (GATE == GATE_VEC ? 1 : 0);
  TmaGeom g = tma_geom(a.N, sizeof(T), ntens, true);
  const size_t sm = tma_smem(g, a.N, sizeof(T), ntens, true);
  cudaFuncSetAttribute(norm_bwd_tma_kernel<T, GATE, MOD, NV2>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)sm);
  norm_bwd_tma_kernel<T, GATE, MOD, NV2><<<(int)(a.B * a.P), g.G * g.nt, sm, st>>>(a, g, cur_status());
  return (int)cudaGetLastError();
}

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
  if (tma_ok_fwd<T>(a, GATE)) {
    switch (nv2_for(a.N)) {
      case 1: return launch_fwd_tma<T, GATE, MOD, 1>(a, st);
      case 2: return launch_fwd_tma<T, GATE, MOD, 2>(a, st);
      case 3: return launch_fwd_tma<T, GATE, MOD, 3>(a, st);
      default: return launch_fwd_tma<T, GATE, MOD, 4>(a, st);
    }
  }
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
  if (g_norm_impl == 1 && N % 8 == 0 && N <= 8192) {
    // pipelined kernel: one wave with one CTA per SM (each keeps several stages
    // of rows in flight); never more CTAs than rows
    int64_t P = ((int64_t)num_sms() + B - 1) / B;
    if (P > T) P = T;
    return P < 1 ? 1 : P;
  }
  // team kernel: about two CTAs per SM, each with R row-teams
  const int K = team_warps(N);
  int R = 1;
  while (R * 2 * K * 32 <= 512 && R * 2 <= 8 && (size_t)R * 2 * 3 * N * 4 <= 160 * 1024) R *= 2;
  int64_t target = (2 * (int64_t)num_sms() + B - 1) / B;
  int64_t maxP = (T + R - 1) / R;
  int64_t P = target < maxP ? target : maxP;
  return P < 1 ? 1 : P;
}

template <typename T, int GATE, bool MOD>
static int launch_bwd(const NormBwdArgs& a, cudaStream_t st) {
  if (tma_ok_bwd<T>(a, GATE)) {
    switch (nv2_for(a.N)) {
      case 1: return launch_bwd_tma<T, GATE, MOD, 1>(a, st);
      case 2: return launch_bwd_tma<T, GATE, MOD, 2>(a, st);
      case 3: return launch_bwd_tma<T, GATE, MOD, 3>(a, st);
      default: return launch_bwd_tma<T, GATE, MOD, 4>(a, st);
    }
  }
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
