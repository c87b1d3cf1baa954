// Blackwell (sm_100a) tensor-core GEMM core: TMA + mbarrier pipeline + tcgen05.mma + TMEM.
//
//   C[m, n] = sum_k A[m, k] * B[n, k]          A: [M, K] bf16, B: [N, K] bf16
//
// Each operand is either K-major (rows of K contiguous: A stored [M, K], B [N, K]) or MN-major
// (A stored as [K, M] with M contiguous, B as [K, N]), chosen at compile time; an MN-major tile
// is loaded as 64-column TMA boxes and described to tcgen05.mma with its transpose bit.
//
// One persistent CTA per SM, 6 warps with fixed roles:
//   warp 0      TMA producer: one elected lane streams 128x64 A tiles and 256x64 B tiles
//               (128-byte swizzle) into a kStages-deep shared-memory ring.
//   warp 1      MMA issuer: one elected lane issues tcgen05.mma (M=128, N=256, K=16,
//               bf16 x bf16 -> fp32) into one of two TMEM accumulators (2 x 256 columns).
//   warps 2-5   epilogue: tcgen05.ld the finished accumulator (warp w reads TMEM lanes
//               32*(w%4)..+31, i.e. one output row per thread) and hand each row's fp32
//               values to an Epilogue functor; then release the accumulator.
// Two accumulators let the epilogue of tile i overlap the main loop of tile i+1.
// No TMA multicast and no clusters are used.
//
// A Gate policy can add worker warps (warp 6 onward) and make the producer wait
// until the B rows of an N-block are ready before loading them (NoGate: none).
//
// Every mbarrier wait is bounded by %globaltimer. On timeout a role records an
// error code in the caller's status word, raises the CTA-wide abort flag and
// stops; the other roles see the flag and stop too; the producer waits (bounded)
// for its outstanding copies; all warps meet at the final barrier where TMEM is
// freed. A stuck pipeline therefore ends with an error status, not a hang.
#pragma once

#include <cuda.h>
#include "common.cuh"

namespace nfb {
namespace tc {

constexpr int BM = 128;
constexpr int BN = 256;
constexpr int BK = 64;                    // one 128-byte swizzle atom of bf16
constexpr int kStages = 4;
constexpr int kATileBytes = BM * BK * 2;  // 16 KB
constexpr int kBTileBytes = BN * BK * 2;  // 32 KB
constexpr int kStageBytes = kATileBytes + kBTileBytes;
constexpr int kThreads = 192;
constexpr int kEpiWarp0 = 2;
constexpr uint32_t kTmemCols = 512;       // two 256-column fp32 accumulators
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s per wait

struct alignas(8) Shared {
  uint64_t full[kStages];
  uint64_t empty[kStages];
  uint64_t tmem_full[2];
  uint64_t tmem_empty[2];
  uint64_t mma_drain;
  uint32_t tmem_base;
  int abort;
};

// smem layout: [1 KB-aligned stage buffers][Shared (1 KB slot)][gate area]
constexpr size_t kSharedSlot = 1024;
static_assert(sizeof(Shared) <= kSharedSlot, "Shared must fit its slot");
constexpr size_t kSmemBytes = (size_t)kStages * kStageBytes + kSharedSlot + 1024;

// Default gate: no worker warps, every N-block always ready.
struct NoGate {
  static constexpr int kWarps = 0;
  static constexpr size_t kSmemBytes = 0;
  __device__ __forceinline__ void bind(uint8_t*) {}   // every thread: locate the gate's shared memory
  __device__ __forceinline__ void init() {}           // thread 0, before the CTA barrier
  __device__ __forceinline__ bool wait_nblock(int, volatile int*) { return true; }
  __device__ __forceinline__ void worker(int, uint8_t*, volatile int*) {}
};

template <class Gate>
constexpr size_t smem_bytes() { return kSmemBytes + Gate::kSmemBytes; }
template <class Gate>
constexpr int threads_for() { return kThreads + 32 * Gate::kWarps; }

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes) : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity)
      : "memory");
  return ok != 0;
}

// try_wait with a suspend-time hint: a thread whose phase is not complete sleeps in the barrier
// unit until the phase completes or `ns` elapse, instead of re-polling (less issue activity and
// power while a role idles, e.g. the epilogue during a main loop).
__device__ __forceinline__ bool mbar_try_wait_sleep(uint64_t* bar, uint32_t parity, uint32_t ns) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(smem_u32(bar)), "r"(parity), "r"(ns)
      : "memory");
  return ok != 0;
}

// Bounded wait with the suspend hint (same contract as mbar_wait below).
__device__ __forceinline__ bool mbar_wait_sleep(uint64_t* bar, uint32_t parity, volatile int* abort_flag,
                                                uint32_t hint_ns = 20000u) {
  if (mbar_try_wait_sleep(bar, parity, hint_ns)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait_sleep(bar, parity, hint_ns)) return true;
    if ((++spins & 15u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitNs) return false;
    }
  }
}

// Bounded wait for the phase with the given parity. Returns false on timeout
// or when another role has raised the abort flag.
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, volatile int* abort_flag) {
  if (mbar_try_wait(bar, parity)) return true;
  const uint64_t t0 = globaltimer_ns();
  uint32_t spins = 0;
  while (true) {
    if (mbar_try_wait(bar, parity)) return true;
    if ((++spins & 255u) == 0) {
      if (*abort_flag) return false;
      if (globaltimer_ns() - t0 > kWaitNs) return false;
    }
  }
}

__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void prefetch_tmap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// Shared-memory matrix descriptor for a K-major tile written by TMA with
// 128-byte swizzle: rows of 128 bytes, 8-row groups 1024 bytes apart.
__device__ __forceinline__ uint64_t sw128_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);          // start address
  d |= (uint64_t)1 << 16;                           // leading byte offset (unused for swizzled K-major)
  d |= (uint64_t)(1024 >> 4) << 32;                 // stride byte offset: 8 rows x 128 B
  d |= (uint64_t)1 << 46;                           // descriptor version (sm100)
  d |= (uint64_t)2 << 61;                           // layout: 128-byte swizzle
  return d;
}

// Shared-memory matrix descriptor for an MN-major tile written by TMA as boxes of
// [BK rows of K] x [64 MN columns] (128-byte rows, 128-byte swizzle): 8-row K
// groups 1024 bytes apart (stride byte offset), 64-column MN blocks one box
// (BK * 128 bytes) apart (leading byte offset).
__device__ __forceinline__ uint64_t sw128_mn_desc(uint32_t saddr) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);          // start address
  d |= (uint64_t)((BK * 128) >> 4) << 16;           // leading byte offset: next 64-column MN block
  d |= (uint64_t)(1024 >> 4) << 32;                 // stride byte offset: next 8 K rows
  d |= (uint64_t)1 << 46;                           // descriptor version (sm100)
  d |= (uint64_t)2 << 61;                           // layout: 128-byte swizzle
  return d;
}

// Instruction descriptor: kind::f16, A/B bf16, D fp32, M x N; bit 15 / 16 mark an
// MN-major ("transposed") A / B.
__host__ __device__ constexpr uint32_t idesc_bf16(int m, int n, bool a_mn = false, bool b_mn = false) {
  return (1u << 4) | (1u << 7) | (1u << 10) | ((a_mn ? 1u : 0u) << 15) | ((b_mn ? 1u : 0u) << 16) |
         ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void tmem_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
__device__ __forceinline__ void tmem_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// 32 consecutive fp32 columns of this thread's TMEM lane. The load and its
// wait are one asm statement so no use of the registers can be scheduled
// between them.
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float* v) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 "
      "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
      "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];\n\t"
      "tcgen05.wait::ld.sync.aligned;"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
        "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
      : "r"(taddr)
      : "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 2^x on the FMA pipe (no SFU), for softmax kernels that would otherwise be bound by the SFU's
// exp2 throughput. Range reduction x = n + f with n = round(x), found by adding 1.5 * 2^23 (the sum's
// low mantissa bits then hold n) and f in [-1/2, 1/2]; 2^f from a degree-3 polynomial fitted to 2^f on
// that interval (least squares on the relative error, reweighted toward equal ripple; maximum
// relative error 7.5e-5 in fp32, far below a bf16 step); 2^n is added to the exponent field. Inputs
// are clamped at -126 so the exponent cannot wrap: x <= -126 (and -inf) gives a value below 2^-125.
constexpr float kExp2C0 = 0.999928057f;
constexpr float kExp2C1 = 0.693260968f;
constexpr float kExp2C2 = 0.242611125f;
constexpr float kExp2C3 = 0.0551716648f;
__device__ __forceinline__ float ex2_poly(float x) {
  x = fmaxf(x, -126.f);
  const float t = x + 12582912.f;                 // 1.5 * 2^23: round(x) in the low mantissa bits
  const float f = x - (t - 12582912.f);           // in [-1/2, 1/2]
  const float p = fmaf(fmaf(fmaf(kExp2C3, f, kExp2C2), f, kExp2C1), f, kExp2C0);
  return __uint_as_float(__float_as_uint(p) + (__float_as_uint(t) << 23));
}

// Per-phase cycle accounting (a profiling aid, compiled in only when kOn): lane 0 of a warp adds the
// SM cycles spent since its previous mark to one of 8 counters (constant slot indices keep them in
// registers) and flushes them with one atomic add each into buf[base + slot] at the end.
template <bool kOn>
struct PhaseClock {
  __device__ __forceinline__ void start() {}
  __device__ __forceinline__ void mark(int) {}
  __device__ __forceinline__ void bind_events(uint64_t*, int) {}
  __device__ __forceinline__ void event(unsigned long long*, int) {}
  __device__ __forceinline__ void flush(unsigned long long*, int, int = 0) {}
};
template <>
struct PhaseClock<true> {
  long long t;
  uint32_t acc[8];
  uint64_t* ev = nullptr;      // shared-memory event buffer of this role (first CTA only)
  int n_ev = 0, cap = 0;
  __device__ __forceinline__ void start() {
    t = clock64();
#pragma unroll
    for (int i = 0; i < 8; ++i) acc[i] = 0;
  }
  __device__ __forceinline__ void mark(int slot) {
    const long long n = clock64();
    acc[slot] += (uint32_t)(n - t);
    t = n;
  }
  // timeline of the first CTA: lane 0 appends (code << 48 | SM clock) to a shared-memory buffer
  __device__ __forceinline__ void bind_events(uint64_t* buf, int capacity) {
    if (blockIdx.x == 0 && blockIdx.y == 0 && blockIdx.z == 0) {
      ev = buf;
      cap = capacity;
    }
  }
  __device__ __forceinline__ void event(unsigned long long*, int code) {
    if (ev != nullptr && (threadIdx.x & 31) == 0 && n_ev < cap)
      ev[n_ev++] = ((uint64_t)code << 48) | ((uint64_t)clock64() & 0xFFFFFFFFFFFFull);
  }
  // counters into buf[base + slot]; events (if bound) into buf[64 + ev_off + i]
  __device__ __forceinline__ void flush(unsigned long long* buf, int base, int ev_off = 0) {
    if (buf != nullptr && (threadIdx.x & 31) == 0) {
#pragma unroll
      for (int i = 0; i < 8; ++i)
        if (acc[i]) atomicAdd(buf + base + i, (unsigned long long)acc[i]);
      for (int i = 0; i < n_ev; ++i) buf[64 + ev_off + i] = ev[i];
    }
  }
};

struct TileCoord { int m_blk, n_blk; };

// Tile order: groups of `group` M-blocks; inside a group, N-major, so CTAs that
// run at the same time share B tiles (and the group's A rows stay in L2).
__device__ __forceinline__ TileCoord tile_coord(int t, int m_tiles, int n_tiles, int group) {
  const int per_group = group * n_tiles;
  const int g = t / per_group;
  const int within = t - g * per_group;
  const int rows_in_group = min(group, m_tiles - g * group);
  TileCoord c;
  c.n_blk = within / rows_in_group;
  c.m_blk = g * group + within % rows_in_group;
  return c;
}

struct GemmShape {
  int M, N, K;
  int m_tiles, n_tiles, k_tiles;
  int group;
};

// Plain store epilogue: C[m, n] (bf16 or fp32, row stride ldc), 16-byte
// vector stores when the rows allow them.
struct StoreEpi {
  void* C;
  int64_t ldc;
  int out_f32;
  int vec_ok;      // rows 16-byte aligned
  int accumulate;  // fp32 output only: C += A B^T

  __device__ void row(int m0, int n0, int r, uint32_t taddr, const GemmShape& sh) {
    const int m = m0 + r;
#pragma unroll 1
    for (int c = 0; c < BN; c += 32) {
      float v[32];
      tmem_ld32(taddr + c, v);
      if (m >= sh.M) continue;
      const int n = n0 + c;
      if (out_f32) {
        float* dst = reinterpret_cast<float*>(C) + (int64_t)m * ldc + n;
        if (accumulate) {
          if (vec_ok && n + 32 <= sh.N) {
#pragma unroll
            for (int j = 0; j < 32; j += 4) {
              const float4 o = *reinterpret_cast<const float4*>(dst + j);
              *reinterpret_cast<float4*>(dst + j) = make_float4(o.x + v[j], o.y + v[j + 1], o.z + v[j + 2], o.w + v[j + 3]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) if (n + j < sh.N) dst[j] += v[j];
          }
        } else if (vec_ok && n + 32 <= sh.N) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) if (n + j < sh.N) dst[j] = v[j];
        }
      } else {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(C) + (int64_t)m * ldc + n;
        if (vec_ok && n + 32 <= sh.N) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) store16<__nv_bfloat16>(dst + j, v + j);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) if (n + j < sh.N) dst[j] = __float2bfloat16_rn(v[j]);
        }
      }
    }
  }
};

// The persistent kernel body. Epi must provide:
//   __device__ void row(int tile_m0, int tile_n0, int row_in_tile, uint32_t tmem_row_addr, const GemmShape&)
// which reads the 256 accumulator columns of its row (tmem_ld32 at tmem_row_addr + c)
// and consumes them.
template <bool A_MN, bool B_MN, class Epi, class Gate>
__device__ void gemm_body(const CUtensorMap* tma_a, const CUtensorMap* tma_b, const GemmShape& sh, Epi& epi,
                          uint32_t* status, Gate& gate) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  Shared* S = reinterpret_cast<Shared*>(smem + (size_t)kStages * kStageBytes);
  uint8_t* gate_smem = smem + (size_t)kStages * kStageBytes + kSharedSlot;
  gate.bind(gate_smem);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  volatile int* abort_flag = &S->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&S->full[s], 1);
      mbar_init(&S->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&S->tmem_full[a], 1);
      mbar_init(&S->tmem_empty[a], 4);   // one arrive per epilogue warp
    }
    mbar_init(&S->mma_drain, 1);
    S->abort = 0;
    gate.init();
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&S->tmem_base)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = S->tmem_base;
  const int total_tiles = sh.m_tiles * sh.n_tiles;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0) {
      prefetch_tmap(tma_a);
      prefetch_tmap(tma_b);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        const TileCoord tc = tile_coord(t, sh.m_tiles, sh.n_tiles, sh.group);
        if (!gate.wait_nblock(tc.n_blk, abort_flag)) { ok = false; break; }
        for (int kb = 0; kb < sh.k_tiles; ++kb) {
          if (!mbar_wait(&S->empty[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          uint8_t* sa = smem + (size_t)stage * kStageBytes;
          uint8_t* sb = sa + kATileBytes;
          mbar_arrive_expect_tx(&S->full[stage], kStageBytes);
          if (A_MN) {
#pragma unroll
            for (int h = 0; h < BM / 64; ++h)
              tma_load_2d(sa + h * (BK * 128), tma_a, &S->full[stage], tc.m_blk * BM + 64 * h, kb * BK);
          } else {
            tma_load_2d(sa, tma_a, &S->full[stage], kb * BK, tc.m_blk * BM);
          }
          if (B_MN) {
#pragma unroll
            for (int h = 0; h < BN / 64; ++h)
              tma_load_2d(sb + h * (BK * 128), tma_b, &S->full[stage], tc.n_blk * BN + 64 * h, kb * BK);
          } else {
            tma_load_2d(sb, tma_b, &S->full[stage], kb * BK, tc.n_blk * BN);
          }
          ++issued;
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        set_status(status, kTimeoutFlag, 100);
        S->abort = 1;
      }
      // Drain: the most recent load of every stage must have landed before the
      // CTA may exit (bounded). Load i used stage i % kStages in phase (i / kStages) & 1.
      const uint32_t first = issued > (uint32_t)kStages ? issued - (uint32_t)kStages : 0u;
      for (uint32_t i = first; i < issued; ++i) {
        const uint64_t t0 = globaltimer_ns();
        while (!mbar_try_wait(&S->full[i % kStages], (i / kStages) & 1u)) {
          if (globaltimer_ns() - t0 > kWaitNs) break;
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0) {
      const uint32_t idesc = idesc_bf16(BM, BN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < total_tiles && ok; t += gridDim.x) {
        if (!mbar_wait(&S->tmem_empty[acc], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
        tmem_fence_after();
        const uint32_t tmem_d = tmem_base + (uint32_t)(acc * BN);
        for (int kb = 0; kb < sh.k_tiles; ++kb) {
          if (!mbar_wait(&S->full[stage], phase, abort_flag)) { ok = false; break; }
          tmem_fence_after();
          const uint32_t sa = smem_u32(smem + (size_t)stage * kStageBytes);
          const uint32_t sb = sa + kATileBytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            // K-major: the next 16 K columns are 32 bytes further along each row;
            // MN-major: they are the next 16 rows of 128 bytes
            const uint64_t ad = A_MN ? sw128_mn_desc(sa + kk * 16 * 128) : sw128_desc(sa + kk * 32);
            const uint64_t bd = B_MN ? sw128_mn_desc(sb + kk * 16 * 128) : sw128_desc(sb + kk * 32);
            umma_bf16(tmem_d, ad, bd, idesc, (kb > 0 || kk > 0) ? 1u : 0u);
          }
          umma_commit(&S->empty[stage]);   // frees this stage once the MMAs above are done
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit(&S->tmem_full[acc]);  // accumulator ready for the epilogue
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
      if (!ok) {
        set_status(status, kTimeoutFlag, 101);
        S->abort = 1;
      }
      // every MMA this thread issued must complete before TMEM is freed (bounded)
      umma_commit(&S->mma_drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&S->mma_drain, 0u)) {
        if (globaltimer_ns() - t0 > kWaitNs) break;
      }
    }
  } else if (warp >= kThreads / 32) {
    // ---------------- gate worker warps (6 ..) ----------------
    gate.worker(warp - kThreads / 32, gate_smem, abort_flag);
  } else {
    // ---------------- epilogue (warps 2..5) ----------------
    const int quarter = warp & 3;               // TMEM lanes 32*quarter .. +31
    const int row_in_tile = quarter * 32 + lane;
    int acc = 0;
    uint32_t acc_phase = 0;
    for (int t = blockIdx.x; t < total_tiles; t += gridDim.x) {
      bool ok = mbar_wait(&S->tmem_full[acc], acc_phase, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) {
          set_status(status, kTimeoutFlag, 102);
          S->abort = 1;
        }
        break;
      }
      tmem_fence_after();
      const TileCoord tc = tile_coord(t, sh.m_tiles, sh.n_tiles, sh.group);
      const uint32_t taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * BN);
      epi.row(tc.m_blk * BM, tc.n_blk * BN, row_in_tile, taddr, sh);
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&S->tmem_empty[acc]);
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
  }

  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

}  // namespace tc
}  // namespace nfb
