// Flash attention backward on the 5th-generation tensor cores (sm_100a).
//
// Given Q, K, V, O, dO in the projection-native [B, S, H, D] layout (D = 64 or 128, bf16) and the
// forward's row log-sum-exp, computes dQ, dK, dV for softmax(scale Q K^T) V with grouped-query
// attention (Hkv divides Hq) and an optional causal mask (key kv visible to query q iff
// kv <= q + Sk - Sq; the model uses it with Sq == Sk).
//
//   P = exp(scale S - lse),  S = Q K^T        dV = P^T dO
//   dP = dO V^T,  Delta = rowsum(dO . O)       dS = scale P . (dP - Delta)
//   dQ = dS K,  dK = dS^T Q
//
// Three launches:
//   attn_bwd_pre   Delta and lse * log2(e) per query row, padded to whole 128-query tiles
//                  (padding: lse = +inf, so padded queries get P = 0), and dQ accumulator = 0.
//   attn_bwd_kernel one CTA per (128-key tile, kv head, batch). K and V stay in shared memory;
//                  the CTA walks every query tile i of every query head of its group:
//                    S^T  = K Q_i^T   (M 128 keys, N 128 queries, K = D) -> TMEM
//                    dP^T = V dO_i^T  (same)                              -> TMEM
//                    8 compute warps (two threads per key row, 64 queries each) turn S^T into
//                    P^T (bf16, written back over S^T in TMEM) and dP^T into dS^T (bf16,
//                    128-byte-swizzled K-major tile in shared memory)
//                    dV  += P^T dO_i  (A = P^T from TMEM, B = dO_i read MN-major from its TMA tile)
//                    dK  += dS^T Q_i  (A = dS^T, B = Q_i read MN-major)
//                    dQ_i = dS K      (A = the dS^T tile read MN-major, B = K read MN-major)
//                  The compute warps are software-pipelined: step i's dK / dQ MMAs run while they
//                  compute P of step i+1; then each warp copies its 32 x 32 fp32 blocks of dQ_i
//                  from TMEM into its own slice of the (consumed) dS^T tile and adds them to the
//                  fp32 dQ accumulator with TMA reduce-adds (whole lines, performed in L2).
//                  dK and dV stay in TMEM for the whole walk (GQA heads accumulate there) and
//                  are written once at the end.
//   attn_bwd_post  dQ accumulator (fp32) -> bf16 dQ.
// Every wait is bounded by %globaltimer and reports through the status word (no hang, no trap);
// no cluster, no multicast. Parity: the reference differentiates F.scaled_dot_product_attention
// (nuvla_forge/model/dit.py:92) with autograd.
#include "tc_gemm.cuh"
#include "tc_host.cuh"

namespace nfb {
namespace attnb {

using namespace nfb::tc;

constexpr int T = 128;                 // keys per CTA, queries per tile
constexpr int kThreadsB = 320;         // producer, MMA, 8 compute warps
constexpr uint32_t kTmemColsB = 512;

struct BwdArgs {
  int B, Sq, Sk, Hq, Hkv, D, Sq_pad;
  int causal;
  float scale;                 // softmax scale
  float scale_log2;            // scale * log2(e)
  const float* lse2;           // [B, Hq, Sq_pad] lse * log2(e)
  const float* delta;          // [B, Hq, Sq_pad]
  __nv_bfloat16* dk;           // [B, Sk, Hkv, D]
  __nv_bfloat16* dv;
  int64_t sdk_b, sdk_s, sdk_h, sdv_b, sdv_s, sdv_h;
  uint32_t* status;
  unsigned long long* trace;   // per-phase cycle counters (traced instantiation only)
};

struct alignas(8) BwdShared {
  uint64_t kv_full;
  uint64_t qdo_full[3];
  uint64_t qdo_empty[3];
  uint64_t s_full;
  uint64_t dp_full;
  uint64_t p_ready;            // 256 arrivals: P^T written over S^T in TMEM
  uint64_t dv_done;            // dV MMA of the step complete (P^T consumed)
  uint64_t ds_ready;           // 256 arrivals: dS^T in smem, dP^T read
  uint64_t dq_full;
  uint64_t dq_free;            // 256 arrivals: dQ read from TMEM
  uint64_t acc_full;           // dK, dV complete
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

// smem: [K: D/64 x 16 KB][V][Q: stages][dO: stages][dS^T 32 KB][lse2, delta: stages x 1 KB][BwdShared]
template <int D>
struct LayoutB {
  static constexpr int kStages = D == 64 ? 3 : 2;
  static constexpr int kTile = T * D * 2;            // one [128 x D] bf16 tile
  static constexpr int kK = 0;
  static constexpr int kV = kK + kTile;
  static constexpr int kQ = kV + kTile;
  static constexpr int kDO = kQ + kStages * kTile;
  static constexpr int kDS = kDO + kStages * kTile;
  static constexpr int kRow = kDS + T * T * 2;       // per stage: 128 lse2 + 128 delta floats
  // D = 64: a separate dQ staging area (8 warps x 4 KB), so the next dS^T write need not wait for
  // the TMA to have read the staged dQ; D = 128 stages dQ in the warp's own (consumed) dS^T rows
  static constexpr bool kSepStage = D == 64;
  static constexpr int kStage = kRow + kStages * 1024;
  static constexpr int kS = kStage + (kSepStage ? 8 * 4096 : 0);
  static constexpr size_t kNeed = (size_t)kS + 256;   // + BwdShared
  // dynamic shared memory requested: the layout plus alignment slack, capped at the 227 KB limit
  // (the kernel checks at run time that the aligned layout fits what it was given)
  static constexpr size_t kLimit = 227 * 1024;
  static constexpr size_t kBytes = kNeed + 1024 < kLimit ? kNeed + 1024 : kLimit;
  static_assert(kNeed <= kLimit, "shared memory");
  // TMEM columns: S^T (P^T bf16 over it: queries 0-63 at +0, 64-127 at +64), dP^T, dV, dK, dQ
  static constexpr uint32_t cS = 0, cDP = 128, cDV = 256, cDK = 256 + D;
  static constexpr uint32_t cDQ = D == 64 ? 256 + 2 * D : cDP;   // D = 128: dQ over the consumed dP^T
};

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
        "r"(smem_u32(bar))
      : "memory");
}

// Element-wise add of a shared-memory box into the tensor (performed by L2), bulk-group completion.
__device__ __forceinline__ void tma_reduce_add_4d(const CUtensorMap* map, const void* src, int c0, int c1, int c2,
                                                  int c3) {
  asm volatile(
      "cp.reduce.async.bulk.tensor.4d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3, %4, %5}], [%1];"
      ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(c0), "r"(c1), "r"(c2), "r"(c3)
      : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }

// 1-D bulk copy global -> shared (16-byte aligned addresses, size a multiple of 16).
__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

// MN-major shared-memory descriptor with an explicit distance between 64-column MN blocks.
__device__ __forceinline__ uint64_t mn_desc(uint32_t saddr, uint32_t lbo_bytes) {
  uint64_t d = 0;
  d |= (uint64_t)((saddr & 0x3FFFF) >> 4);
  d |= (uint64_t)((lbo_bytes >> 4) & 0x3FFF) << 16;
  d |= (uint64_t)(1024 >> 4) << 32;
  d |= (uint64_t)1 << 46;
  d |= (uint64_t)2 << 61;
  return d;
}

// D (TMEM) (+)= A (TMEM, 128 lanes x 16 bf16 packed two per column) x B (shared memory descriptor).
__device__ __forceinline__ void umma_bf16_ts(uint32_t tmem_d, uint32_t tmem_a, uint64_t bdesc, uint32_t idesc,
                                             uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n\t}"
      ::"r"(tmem_d), "r"(tmem_a), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

__device__ __forceinline__ void tmem_st16_nowait(uint32_t taddr, const uint32_t* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x16.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16};"
      ::"r"(taddr), "r"(v[0]), "r"(v[1]), "r"(v[2]), "r"(v[3]), "r"(v[4]), "r"(v[5]), "r"(v[6]), "r"(v[7]),
        "r"(v[8]), "r"(v[9]), "r"(v[10]), "r"(v[11]), "r"(v[12]), "r"(v[13]), "r"(v[14]), "r"(v[15])
      : "memory");
}

__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// The 8 compute warps (256 threads) as one named barrier group.
__device__ __forceinline__ bool compute_all(bool v) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.and.pred q, 1, 256, p;\n\t"
      "selp.b32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((int)v)
      : "memory");
  return r != 0;
}

// First query tile whose queries can see a key of this key tile (causal), else 0.
__device__ __forceinline__ int first_qtile(const BwdArgs& a, int k0) {
  if (!a.causal) return 0;
  const int q_first = k0 - (a.Sk - a.Sq);      // smallest query that sees key k0
  return q_first <= 0 ? 0 : q_first / T;
}

template <int D, bool kTrace>
__global__ void __launch_bounds__(kThreadsB, 1)
    attn_bwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, const __grid_constant__ CUtensorMap tdo,
                    const __grid_constant__ CUtensorMap tdq, BwdArgs a) {
  using L = LayoutB<D>;
  constexpr int kDB = D / 64;
  constexpr int NS = L::kStages;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // the aligned layout must fit the allocation (the request is capped at the per-block limit)
  if ((size_t)(smem - smem_raw) + L::kNeed > L::kBytes) {
    if (threadIdx.x == 0) set_status(a.status, kTimeoutFlag, 143);
    return;
  }
  BwdShared* S = reinterpret_cast<BwdShared*>(smem + L::kS);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &S->abort;
  const int k0 = blockIdx.x * T, hk = blockIdx.y, b = blockIdx.z;
  const int G = a.Hq / a.Hkv;
  const int nq = (a.Sq + T - 1) / T;
  const int i0 = first_qtile(a, k0);
  const int per_head = nq - i0 > 0 ? nq - i0 : 0;
  const int n_tiles = G * per_head;              // (head, query tile) pairs this CTA walks

  if (threadIdx.x == 0) {
    mbar_init(&S->kv_full, 1);
    for (int s = 0; s < NS; ++s) {
      mbar_init(&S->qdo_full[s], 1);
      mbar_init(&S->qdo_empty[s], 1);
    }
    mbar_init(&S->s_full, 1);
    mbar_init(&S->dp_full, 1);
    mbar_init(&S->p_ready, 256);
    mbar_init(&S->dv_done, 1);
    mbar_init(&S->ds_ready, 256);
    mbar_init(&S->dq_full, 1);
    mbar_init(&S->dq_free, 256);
    mbar_init(&S->acc_full, 1);
    mbar_init(&S->drain, 1);
    S->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&S->tmem_base)), "r"(kTmemColsB) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem = S->tmem_base;

  if (warp == 0) {
    // ---------------- producer ----------------
    if (lane == 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
      prefetch_tmap(&tdo);
      mbar_arrive_expect_tx(&S->kv_full, 2 * L::kTile);
      for (int db = 0; db < kDB; ++db) {
        tma_load_4d(smem + L::kK + db * 16384, &tk, &S->kv_full, db * 64, hk, k0, b);
        tma_load_4d(smem + L::kV + db * 16384, &tv, &S->kv_full, db * 64, hk, k0, b);
      }
      bool ok = true;
      int issued = 0;
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int st = t % NS;
        const int use = t / NS;                    // how often this stage was filled before
        if (use >= 1 && !mbar_wait(&S->qdo_empty[st], (use - 1) & 1, abort_flag)) { ok = false; break; }
        const int h = hk * G + t / per_head;
        const int q0 = (i0 + t % per_head) * T;
        mbar_arrive_expect_tx(&S->qdo_full[st], 2 * L::kTile + 1024);
        for (int db = 0; db < kDB; ++db) {
          tma_load_4d(smem + L::kQ + st * L::kTile + db * 16384, &tq, &S->qdo_full[st], db * 64, h, q0, b);
          tma_load_4d(smem + L::kDO + st * L::kTile + db * 16384, &tdo, &S->qdo_full[st], db * 64, h, q0, b);
        }
        const int64_t row = ((int64_t)b * a.Hq + h) * a.Sq_pad + q0;
        bulk_load(smem + L::kRow + st * 1024, a.lse2 + row, 512, &S->qdo_full[st]);
        bulk_load(smem + L::kRow + st * 1024 + 512, a.delta + row, 512, &S->qdo_full[st]);
        ++issued;
      }
      if (!ok) {
        set_status(a.status, kTimeoutFlag, 140);
        S->abort = 1;
      }
      // drain (bounded): K/V and the latest Q/dO loads
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&S->kv_full, 0u) && globaltimer_ns() - t0 < kWaitNs) {}
      for (int t = issued > NS ? issued - NS : 0; t < issued; ++t) {
        const uint64_t t1 = globaltimer_ns();
        while (!mbar_try_wait(&S->qdo_full[t % NS], (t / NS) & 1) && globaltimer_ns() - t1 < kWaitNs) {}
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n_tiles > 0) {
      constexpr uint32_t id_s = idesc_bf16(T, T, false, false);     // S^T, dP^T
      constexpr uint32_t id_kv = idesc_bf16(T, D, false, true);     // dV, dK: A K-major, B MN-major
      constexpr uint32_t id_q = idesc_bf16(T, D, true, true);       // dQ: A (dS^T) and B (K) MN-major
      // shared-memory descriptors computed once; tile offsets are added to the start-address field
      const uint64_t dk = sw128_desc(smem_u32(smem + L::kK)), dv = sw128_desc(smem_u32(smem + L::kV));
      const uint64_t dk_mn = mn_desc(smem_u32(smem + L::kK), 16384);
      const uint64_t dq0 = sw128_desc(smem_u32(smem + L::kQ)), dq0_mn = mn_desc(smem_u32(smem + L::kQ), 16384);
      const uint64_t ddo0 = sw128_desc(smem_u32(smem + L::kDO)), ddo0_mn = mn_desc(smem_u32(smem + L::kDO), 16384);
      const uint64_t dds = sw128_desc(smem_u32(smem + L::kDS)), dds_mn = mn_desc(smem_u32(smem + L::kDS), 16384);
      auto off = [](int bytes) { return (uint64_t)(bytes >> 4); };
      auto issue_s = [&](int t) {        // S^T = K Q_t^T
        const uint64_t dq = dq0 + off((t % NS) * L::kTile);
#pragma unroll
        for (int db = 0; db < kDB; ++db)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + L::cS, dk + off(db * 16384 + kk * 32), dq + off(db * 16384 + kk * 32), id_s,
                      (db > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&S->s_full);
      };
      auto issue_dp = [&](int t) {       // dP^T = V dO_t^T
        const uint64_t ddo = ddo0 + off((t % NS) * L::kTile);
#pragma unroll
        for (int db = 0; db < kDB; ++db)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + L::cDP, dv + off(db * 16384 + kk * 32), ddo + off(db * 16384 + kk * 32), id_s,
                      (db > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&S->dp_full);
      };
      PhaseClock<kTrace> pc;
      pc.start();
      bool ok = mbar_wait(&S->kv_full, 0u, abort_flag) && mbar_wait(&S->qdo_full[0], 0u, abort_flag);
      pc.mark(1);
      if (ok) {
        tmem_fence_after();
        issue_s(0);
        issue_dp(0);
      }
      pc.mark(4);
      for (int t = 0; t < n_tiles && ok; ++t) {
        const int st = t % NS;
        const uint64_t dq_mn = dq0_mn + off(st * L::kTile);
        const uint64_t ddo_mn = ddo0_mn + off(st * L::kTile);
        // dV += P^T dO_t, P^T from TMEM (queries 0-63 at cS, 64-127 at cS + 64)
        if (!mbar_wait(&S->p_ready, t & 1, abort_flag)) { ok = false; break; }
        pc.mark(0);
        tmem_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16_ts(tmem + L::cDV, tmem + L::cS + (uint32_t)((kk >> 2) * 64 + (kk & 3) * 8),
                       ddo_mn + off(kk * 16 * 128), id_kv, (t > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&S->dv_done);
        pc.mark(4);
        if (t + 1 < n_tiles) {
          // S^T of the next step overwrites P^T: wait until the dV MMA has read it
          if (!mbar_wait(&S->qdo_full[(t + 1) % NS], ((t + 1) / NS) & 1, abort_flag)) { ok = false; break; }
          pc.mark(1);
          if (!mbar_wait(&S->dv_done, t & 1, abort_flag)) { ok = false; break; }
          pc.mark(2);
          tmem_fence_after();
          issue_s(t + 1);
          pc.mark(4);
        }
        // dK += dS^T Q_t
        if (!mbar_wait(&S->ds_ready, t & 1, abort_flag)) { ok = false; break; }
        pc.mark(3);
        tmem_fence_after();
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(tmem + L::cDK, dds + off(kb * 16384 + kk * 32), dq_mn + off((kb * 64 + kk * 16) * 128), id_kv,
                      (t > 0 || kb > 0 || kk > 0) ? 1u : 0u);
        // dQ_t = dS K (D = 64: own columns, free once the compute warps drained dQ of t-1)
        pc.mark(4);
        if (D == 64 && t >= 1 && !mbar_wait(&S->dq_free, (t - 1) & 1, abort_flag)) { ok = false; break; }
        pc.mark(5);
        tmem_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_bf16(tmem + L::cDQ, dds_mn + off(kk * 16 * 128), dk_mn + off(kk * 16 * 128), id_q, kk > 0 ? 1u : 0u);
        umma_commit(&S->dq_full);
        umma_commit(&S->qdo_empty[st]);
        pc.mark(4);
        if (t + 1 < n_tiles) {
          // D = 128: dQ_t occupies the dP^T columns until the compute warps have drained it
          if (D == 128 && !mbar_wait(&S->dq_free, t & 1, abort_flag)) { ok = false; break; }
          pc.mark(5);
          tmem_fence_after();
          issue_dp(t + 1);
          pc.mark(4);
        }
      }
      pc.flush(a.trace, 8);
      if (ok) umma_commit(&S->acc_full);
      if (!ok) {
        set_status(a.status, kTimeoutFlag, 141);
        S->abort = 1;
      }
      umma_commit(&S->drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&S->drain, 0u) && globaltimer_ns() - t0 < kWaitNs) {}
    }
  } else {
    // ---------------- compute warps 2..9 ----------------
    // Key row r = TMEM lane (quarter * 32 + lane); half 0 takes queries 0-63 of each tile, half 1
    // queries 64-127 (and dQ / dK / dV columns [half * D/2, +D/2)).
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int key = k0 + r;
    constexpr int HC = 64;
    // this warp's rows of the dS^T tile (block `half`, rows quarter*32..+31): 4 KB, also the
    // staging box of its dQ blocks once the MMAs have consumed dS^T
    uint8_t* slice = smem + L::kDS + half * 16384 + quarter * 4096;
    uint8_t* drow = slice + lane * 128;
    uint8_t* stage = L::kSepStage ? smem + L::kStage + (warp - 2) * 4096 : slice;   // dQ staging box
    uint8_t* srow = stage + lane * 128;
    bool ok = true;
    int prev_h = 0, prev_q0 = 0;
    PhaseClock<kTrace> pc;
    pc.start();
    // dQ of the previous step: TMEM -> this warp's slice -> TMA reduce-add into the accumulator
    auto drain_dq = [&](int tt) -> bool {
      const bool w = mbar_wait(&S->dq_full, tt & 1, abort_flag);
      if (!compute_all(w)) return false;
      pc.mark(2);
      tmem_fence_after();
#pragma unroll
      for (int bx = 0; bx < D / 64; ++bx) {
        const int col = half * (D / 2) + bx * 32;
        float g[32];
        tmem_ld32(tmem + lane_off + L::cDQ + (uint32_t)col, g);
        if (bx > 0 || L::kSepStage) {
          if (lane == 0) bulk_wait_read0();      // the previous box has been read out of the staging area
          __syncwarp();
        }
#pragma unroll
        for (int c = 0; c < 8; ++c)
          *reinterpret_cast<float4*>(srow + ((c ^ (lane & 7)) << 4)) =
              make_float4(g[4 * c], g[4 * c + 1], g[4 * c + 2], g[4 * c + 3]);
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        __syncwarp();
        if (lane == 0) {
          tma_reduce_add_4d(&tdq, stage, col, prev_h, prev_q0 + quarter * 32, b);
          bulk_commit();
        }
      }
      tmem_fence_before();
      mbar_arrive(&S->dq_free);
      pc.mark(3);
      return true;
    };
    for (int t = 0; t < n_tiles; ++t) {
      const int st = t % NS;
      const int h = hk * G + t / per_head;
      const int q0 = (i0 + t % per_head) * T;
      const float* lse2 = reinterpret_cast<const float*>(smem + L::kRow + st * 1024) + half * HC;
      const float* dlt = reinterpret_cast<const float*>(smem + L::kRow + st * 1024 + 512) + half * HC;
      // ---- P^T of step t ----
      bool w = mbar_wait(&S->qdo_full[st], (t / NS) & 1, abort_flag);
      w = w && mbar_wait(&S->s_full, t & 1, abort_flag);
      if (!compute_all(w)) { ok = false; break; }
      pc.mark(0);
      tmem_fence_after();
      float p[HC];
#pragma unroll
      for (int c = 0; c < HC; c += 32) tmem_ld32(tmem + lane_off + L::cS + (uint32_t)(half * HC + c), p + c);
      const int qb = q0 + half * HC;
      const int lim = key - (a.Sk - a.Sq);        // causal: queries q >= lim see this key
      const bool full = key < a.Sk && (!a.causal || qb >= lim);
#pragma unroll
      for (int c = 0; c < HC; c += 4) {
        // one quad in four on the FMA pipe (ex2_poly), the rest on the SFU
        const float4 l4 = *reinterpret_cast<const float4*>(lse2 + c);
        const float x0 = fmaf(p[c], a.scale_log2, -l4.x), x1 = fmaf(p[c + 1], a.scale_log2, -l4.y);
        const float x2 = fmaf(p[c + 2], a.scale_log2, -l4.z), x3 = fmaf(p[c + 3], a.scale_log2, -l4.w);
        if (((c >> 2) & 3) == 3) {
          p[c] = ex2_poly(x0); p[c + 1] = ex2_poly(x1); p[c + 2] = ex2_poly(x2); p[c + 3] = ex2_poly(x3);
        } else {
          p[c] = ex2_approx(x0); p[c + 1] = ex2_approx(x1); p[c + 2] = ex2_approx(x2); p[c + 3] = ex2_approx(x3);
        }
      }
      if (!full) {
#pragma unroll
        for (int c = 0; c < HC; ++c) p[c] = (key < a.Sk && (!a.causal || qb + c >= lim)) ? p[c] : 0.f;
      }
#pragma unroll
      for (int c0 = 0; c0 < HC; c0 += 32) {
        uint32_t pk[16];
#pragma unroll
        for (int c = 0; c < 16; ++c) pk[c] = pack_bf16(p[c0 + 2 * c], p[c0 + 2 * c + 1]);
        tmem_st16_nowait(tmem + lane_off + L::cS + (uint32_t)(half * HC + (c0 >> 1)), pk);
      }
      asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
      tmem_fence_before();
      mbar_arrive(&S->p_ready);
      pc.mark(1);
      // ---- dQ of step t-1 (its MMAs ran while P of step t was computed) ----
      if (t >= 1 && !drain_dq(t - 1)) { ok = false; break; }
      // ---- dS^T = scale * P^T . (dP^T - Delta) of step t ----
      w = mbar_wait(&S->dp_full, t & 1, abort_flag);
      if (!compute_all(w)) { ok = false; break; }
      pc.mark(4);
      tmem_fence_after();
      if (t >= 1 && !L::kSepStage) {
        if (lane == 0) bulk_wait_read0();        // the slice's dQ boxes have been read
        __syncwarp();
      }
#pragma unroll
      for (int c = 0; c < HC; c += 32) {
        float dp[32];
        tmem_ld32(tmem + lane_off + L::cDP + (uint32_t)(half * HC + c), dp);
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          const float4 d4 = *reinterpret_cast<const float4*>(dlt + c + j);
          dp[j] = a.scale * p[c + j] * (dp[j] - d4.x);
          dp[j + 1] = a.scale * p[c + j + 1] * (dp[j + 1] - d4.y);
          dp[j + 2] = a.scale * p[c + j + 2] * (dp[j + 2] - d4.z);
          dp[j + 3] = a.scale * p[c + j + 3] * (dp[j + 3] - d4.w);
        }
#pragma unroll
        for (int g8 = 0; g8 < 4; ++g8) {
          const int cc = (c >> 3) + g8;
          uint4 v;
          v.x = pack_bf16(dp[8 * g8 + 0], dp[8 * g8 + 1]);
          v.y = pack_bf16(dp[8 * g8 + 2], dp[8 * g8 + 3]);
          v.z = pack_bf16(dp[8 * g8 + 4], dp[8 * g8 + 5]);
          v.w = pack_bf16(dp[8 * g8 + 6], dp[8 * g8 + 7]);
          *reinterpret_cast<uint4*>(drow + ((cc ^ (r & 7)) << 4)) = v;
        }
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tmem_fence_before();
      mbar_arrive(&S->ds_ready);
      pc.mark(5);
      prev_h = h;
      prev_q0 = q0;
    }
    if (ok && n_tiles > 0 && !drain_dq(n_tiles - 1)) ok = false;
    if (lane == 0) bulk_wait_all();              // every dQ reduce-add performed before the CTA exits
    __syncwarp();
    pc.mark(6);
    // dK, dV rows (TMEM lane = key): this half's D/2 columns, written once
    if (ok && n_tiles > 0) {
      bool w = mbar_wait(&S->acc_full, 0u, abort_flag);
      if (compute_all(w)) {
        tmem_fence_after();
        // tcgen05.ld is warp-collective: every lane loads, only rows of real keys are stored
        const bool live = key < a.Sk;
        __nv_bfloat16* dkr = a.dk + (int64_t)b * a.sdk_b + (int64_t)key * a.sdk_s + (int64_t)hk * a.sdk_h;
        __nv_bfloat16* dvr = a.dv + (int64_t)b * a.sdv_b + (int64_t)key * a.sdv_s + (int64_t)hk * a.sdv_h;
#pragma unroll
        for (int c = 0; c < D / 2; c += 32) {
          float g[32];
          const int col = half * (D / 2) + c;
          tmem_ld32(tmem + lane_off + L::cDK + (uint32_t)col, g);
          if (live) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) store16<__nv_bfloat16>(dkr + col + j, g + j);
          }
          tmem_ld32(tmem + lane_off + L::cDV + (uint32_t)col, g);
          if (live) {
#pragma unroll
            for (int j = 0; j < 32; j += 8) store16<__nv_bfloat16>(dvr + col + j, g + j);
          }
        }
      } else {
        ok = false;
      }
    } else if (n_tiles == 0 && key < a.Sk) {
      // no query sees this key tile (causal): zero gradients
      __nv_bfloat16* dkr = a.dk + (int64_t)b * a.sdk_b + (int64_t)key * a.sdk_s + (int64_t)hk * a.sdk_h;
      __nv_bfloat16* dvr = a.dv + (int64_t)b * a.sdv_b + (int64_t)key * a.sdv_s + (int64_t)hk * a.sdv_h;
      for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 8) {
        *reinterpret_cast<uint4*>(dkr + c) = make_uint4(0u, 0u, 0u, 0u);
        *reinterpret_cast<uint4*>(dvr + c) = make_uint4(0u, 0u, 0u, 0u);
      }
    }
    pc.mark(7);
    pc.flush(a.trace, 0);
    if (!ok && lane == 0) {
      set_status(a.status, kTimeoutFlag, 142);
      S->abort = 1;
    }
  }

  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(kTmemColsB) : "memory");
  }
}

// Delta = rowsum(dO . O), lse2 = lse * log2(e), padded to Sq_pad (pad: lse2 = +inf, Delta = 0); one
// warp per (b, h, q) row.
__global__ void attn_bwd_pre_kernel(const __nv_bfloat16* o, const __nv_bfloat16* dout, const float* lse, int B,
                                    int Sq, int Hq, int D, int Sq_pad, int64_t so_b, int64_t so_s, int64_t so_h,
                                    int64_t sd_b, int64_t sd_s, int64_t sd_h, float* lse2, float* delta) {
  const int64_t row = ((int64_t)blockIdx.x * blockDim.x + threadIdx.x) >> 5;
  const int lane = threadIdx.x & 31;
  const int64_t rows = (int64_t)B * Hq * Sq_pad;
  if (row >= rows) return;
  const int q = (int)(row % Sq_pad);
  const int64_t bh = row / Sq_pad;
  const int h = (int)(bh % Hq), b = (int)(bh / Hq);
  if (q >= Sq) {
    if (lane == 0) {
      lse2[row] = INFINITY;
      delta[row] = 0.f;
    }
    return;
  }
  const __nv_bfloat16* orow = o + b * so_b + (int64_t)q * so_s + (int64_t)h * so_h;
  const __nv_bfloat16* drow = dout + b * sd_b + (int64_t)q * sd_s + (int64_t)h * sd_h;
  float s = 0.f;
  for (int c = lane * 8; c < D; c += 256) {
    float x[8], y[8];
    load16<__nv_bfloat16>(orow + c, x);
    load16<__nv_bfloat16>(drow + c, y);
#pragma unroll
    for (int j = 0; j < 8; ++j) s += x[j] * y[j];
  }
  s = warp_sum(s);
  if (lane == 0) {
    delta[row] = s;
    const float l = lse[((int64_t)b * Hq + h) * Sq + q];
    lse2[row] = l * 1.4426950408889634f;
  }
}

// dQ (bf16, any strides) from the fp32 accumulator [B, Sq, Hq, D].
__global__ void attn_bwd_post_kernel(const float* acc, __nv_bfloat16* dq, int B, int Sq, int Hq, int D, int64_t sb,
                                     int64_t ss, int64_t sh) {
  const int64_t n8 = (int64_t)B * Sq * Hq * D / 8;
  for (int64_t i = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; i < n8; i += (int64_t)gridDim.x * blockDim.x) {
    const int64_t e = i * 8;
    const int d = (int)(e % D);
    const int64_t r = e / D;
    const int h = (int)(r % Hq);
    const int64_t bs = r / Hq;
    const int s = (int)(bs % Sq), b = (int)(bs / Sq);
    float v[8];
    load16<float>(acc + e, v);
    load16<float>(acc + e + 4, v + 4);
    store16<__nv_bfloat16>(dq + b * sb + (int64_t)s * ss + (int64_t)h * sh + d, v);
  }
}

static int make_tmap_bshd(CUtensorMap* m, const void* base, int Bn, int Sn, int Hn, int Dn, int64_t sb, int64_t ss,
                          int64_t sh) {
  int rc = get_encode();
  if (rc) return rc;
  rc = bind_device_of(base);
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (sb * 2) % 16 || (ss * 2) % 16 || (sh * 2) % 16)
    return (int)cudaErrorInvalidValue;
  cuuint64_t dims[4] = {(cuuint64_t)Dn, (cuuint64_t)Hn, (cuuint64_t)Sn, (cuuint64_t)Bn};
  cuuint64_t strides[3] = {(cuuint64_t)(sh * 2), (cuuint64_t)(ss * 2), (cuuint64_t)(sb * 2)};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)T, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

// 4-D fp32 tensor map over the dQ accumulator [B, Sq, Hq, D] with 32 x 32 boxes (128-byte rows,
// 128-byte swizzle), the target of the TMA reduce-adds.
static int make_tmap_dq(CUtensorMap* m, const float* base, int Bn, int Sn, int Hn, int Dn) {
  int rc = get_encode();
  if (rc) return rc;
  rc = bind_device_of(base);
  if (rc) return rc;
  cuuint64_t dims[4] = {(cuuint64_t)Dn, (cuuint64_t)Hn, (cuuint64_t)Sn, (cuuint64_t)Bn};
  cuuint64_t strides[3] = {(cuuint64_t)Dn * 4, (cuuint64_t)Hn * Dn * 4, (cuuint64_t)Sn * Hn * Dn * 4};
  cuuint32_t box[4] = {32, 1, 32, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 4, const_cast<float*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

// Per-phase cycle counters: when set (nfb_attn_bwd_trace), launches run the traced instantiation.
static unsigned long long* g_trace = nullptr;

template <int D>
static int launch_bwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const CUtensorMap& tdo,
                      const CUtensorMap& tdq, BwdArgs a, cudaStream_t st) {
  const size_t smem = LayoutB<D>::kBytes;
  a.trace = g_trace;
  auto kern = g_trace ? attn_bwd_kernel<D, true> : attn_bwd_kernel<D, false>;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  dim3 grid((a.Sk + T - 1) / T, a.Hkv, a.B);
  kern<<<grid, kThreadsB, smem, st>>>(tq, tk, tv, tdo, tdq, a);
  return (int)cudaGetLastError();
}

}  // namespace attnb
}  // namespace nfb

using namespace nfb;
using namespace nfb::attnb;

// Scratch the backward needs (bytes): lse2 + delta [B, Hq, Sq_pad] fp32 and the fp32 dQ accumulator.
NFB_API int64_t nfb_attn_bwd_scratch_bytes(int B, int Sq, int Hq, int D) {
  const int64_t sq_pad = (int64_t)(Sq + T - 1) / T * T;
  return 2 * (int64_t)B * Hq * sq_pad * 4 + (int64_t)B * Sq * Hq * D * 4;
}

// dq / dk / dv from q, k, v, o, do (all [B, S, H, D] with element strides) and the forward's lse
// [B, Hq, Sq]; scratch: nfb_attn_bwd_scratch_bytes bytes, 16-byte aligned. Three launches.
NFB_API int nfb_attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout, const float* lse,
                         void* dq, void* dk, void* dv, void* scratch, int B, int Sq, int Sk, int Hq, int Hkv, int D,
                         const int64_t* strides, int causal, float scale, uint32_t* status, void* stream) {
  // strides: 7 x (b, s, h) for q, k, v, o, do, dq, dk, dv -> 24 values
  if ((D != 64 && D != 128) || B < 1 || Sq < 1 || Sk < 1 || Hkv < 1 || Hq % Hkv) return (int)cudaErrorInvalidValue;
  if (reinterpret_cast<uintptr_t>(scratch) & 15) return (int)cudaErrorInvalidValue;
  const int64_t* sq_ = strides;
  const int64_t* sk_ = strides + 3;
  const int64_t* sv_ = strides + 6;
  const int64_t* so_ = strides + 9;
  const int64_t* sdo_ = strides + 12;
  const int64_t* sdq_ = strides + 15;
  const int64_t* sdk_ = strides + 18;
  const int64_t* sdv_ = strides + 21;
  for (int i = 0; i < 24; ++i)
    if ((strides[i] * 2) % 16) return (int)cudaErrorInvalidValue;
  const void* outs[3] = {dq, dk, dv};
  for (const void* p : outs)
    if (reinterpret_cast<uintptr_t>(p) & 15) return (int)cudaErrorInvalidValue;
  cudaStream_t st = (cudaStream_t)stream;
  const int sq_pad = (Sq + T - 1) / T * T;
  float* lse2 = reinterpret_cast<float*>(scratch);
  float* delta = lse2 + (int64_t)B * Hq * sq_pad;
  float* acc = delta + (int64_t)B * Hq * sq_pad;
  cudaError_t e = cudaMemsetAsync(acc, 0, (size_t)B * Sq * Hq * D * 4, st);
  if (e != cudaSuccess) return (int)e;
  const int64_t rows = (int64_t)B * Hq * sq_pad;
  attn_bwd_pre_kernel<<<(unsigned)((rows * 32 + 255) / 256), 256, 0, st>>>(
      reinterpret_cast<const __nv_bfloat16*>(o), reinterpret_cast<const __nv_bfloat16*>(dout), lse, B, Sq, Hq, D,
      sq_pad, so_[0], so_[1], so_[2], sdo_[0], sdo_[1], sdo_[2], lse2, delta);
  e = cudaGetLastError();
  if (e != cudaSuccess) return (int)e;
  CUtensorMap tq, tk, tv, tdo;
  int rc = make_tmap_bshd(&tq, q, B, Sq, Hq, D, sq_[0], sq_[1], sq_[2]);
  if (rc) return rc;
  rc = make_tmap_bshd(&tk, k, B, Sk, Hkv, D, sk_[0], sk_[1], sk_[2]);
  if (rc) return rc;
  rc = make_tmap_bshd(&tv, v, B, Sk, Hkv, D, sv_[0], sv_[1], sv_[2]);
  if (rc) return rc;
  rc = make_tmap_bshd(&tdo, dout, B, Sq, Hq, D, sdo_[0], sdo_[1], sdo_[2]);
  if (rc) return rc;
  CUtensorMap tdq;
  rc = make_tmap_dq(&tdq, acc, B, Sq, Hq, D);
  if (rc) return rc;
  BwdArgs a;
  a.B = B; a.Sq = Sq; a.Sk = Sk; a.Hq = Hq; a.Hkv = Hkv; a.D = D; a.Sq_pad = sq_pad; a.causal = causal;
  a.scale = scale;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.lse2 = lse2; a.delta = delta;
  a.dk = reinterpret_cast<__nv_bfloat16*>(dk);
  a.dv = reinterpret_cast<__nv_bfloat16*>(dv);
  a.sdk_b = sdk_[0]; a.sdk_s = sdk_[1]; a.sdk_h = sdk_[2];
  a.sdv_b = sdv_[0]; a.sdv_s = sdv_[1]; a.sdv_h = sdv_[2];
  a.status = status;
  rc = D == 64 ? launch_bwd<64>(tq, tk, tv, tdo, tdq, a, st) : launch_bwd<128>(tq, tk, tv, tdo, tdq, a, st);
  if (rc) return rc;
  const int64_t n8 = (int64_t)B * Sq * Hq * D / 8;
  const unsigned grid = (unsigned)(n8 < 148 * 64 ? (n8 + 255) / 256 : 148 * 16);
  attn_bwd_post_kernel<<<grid > 0 ? grid : 1, 256, 0, st>>>(acc, reinterpret_cast<__nv_bfloat16*>(dq), B, Sq, Hq, D,
                                                            sdq_[0], sdq_[1], sdq_[2]);
  return (int)cudaGetLastError();
}

// Profiling aid: counters [1024] of uint64; the next backward launches add their per-phase SM
// cycles to (compute warps 0-7: wait S, P^T, wait dQ, dQ drain, wait dP, dS^T, final reduce-add
// wait, dK/dV epilogue; MMA issuer 8-13: wait P^T, wait Q/dO, wait dV done, wait dS^T, issue, wait
// dQ drained); nullptr switches it off.
NFB_API void nfb_attn_bwd_trace(void* counters) { g_trace = reinterpret_cast<unsigned long long*>(counters); }
