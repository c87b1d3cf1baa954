// Blackwell (sm_100a) CTA-pair tensor-core GEMM: cta_group::2 tcgen05.mma on 256 x 256 tiles.
//
//   C[m, n] = sum_k A[m, k] * B[n, k]          A, B bf16; fp32 accumulate in TMEM
//
// A cluster of two CTAs (one per SM) owns one 256 x 256 output tile at a time:
//   * CTA r of the pair loads rows [m0 + 128 r, +128) of A and rows [n0 + 128 r, +128) of B
//     (64 K columns per stage, 128-byte swizzle) into its own shared memory with plain TMA
//     loads (no multicast); both CTAs' loads complete on the LEADER's (rank 0) stage barrier,
//     which the leader arms with the bytes of both halves.
//   * the leader's elected MMA thread issues tcgen05.mma.cta_group::2 (M = 256, N = 256, K = 16):
//     the tensor cores of both SMs read A from their own CTA and the two B halves from both,
//     and each CTA's TMEM receives its 128 rows x 256 fp32 columns of the tile.
//   * tcgen05.commit with a CTA mask signals both CTAs' "stage empty" and "accumulator full"
//     barriers; the epilogue warps of both CTAs release the accumulator on the leader's barrier
//     with remote mbarrier arrives.
// Per CTA per stage the shared-memory operand traffic is 32 KB for 2 * 128 * 256 * 64 FLOP
// (the single-CTA 128 x 256 tile needs 48 KB for the same work), so the MMA is not bound by
// shared-memory bandwidth, and each B tile is fetched from L2 once per pair.
//
// Each operand is K-major (A [M, K], B [N, K], K contiguous) or MN-major (A stored [K, M],
// B stored [K, N]); MN-major tiles are loaded as 64-column boxes and described with the
// instruction descriptor's transpose bits. The three GEMMs of a linear layer map onto it as
//   forward  Y = X W^T:   A = X  (K-major),  B = W  (K-major)
//   dgrad    dX = dY W:   A = dY (K-major),  B = W  (MN-major)
//   wgrad    dW = dY^T X: A = dY (MN-major), B = X  (MN-major)
//
// Persistent: the grid is (co-resident clusters) x 2 CTAs, work items are taken round-robin.
// A work item is (tile, split): with split-K, consecutive items are the K slices of one tile and
// the epilogue accumulates them in order (split j waits, bounded, for split j-1's flag), so the
// result does not depend on timing. Every item of the kernel only waits for items with smaller
// indices, which co-resident clusters process in increasing order: no wait cycle exists.
//
// Roles per CTA (192 threads): warp 0 TMA producer, warp 1 MMA issuer (leader CTA) and TMEM
// allocator (both CTAs), warps 2-5 epilogue (warp w reads TMEM lanes 32 (w % 4) .. +31: one
// output row per thread). Two 256-column TMEM accumulators let the epilogue of one item
// overlap the main loop of the next.
//
// Every wait is bounded by %globaltimer: a timeout records a code in the status word, raises
// the CTA's abort flag (the other roles stop at their next wait), the producer waits (bounded)
// for the copies it can observe, and both CTAs meet at the closing cluster barrier before the
// TMEM is freed.
#pragma once

#include <cuda.h>

#include "common.cuh"
#include "tc_gemm.cuh"

namespace nfb {
namespace g2 {


using tc::mbar_arrive_expect_tx;
using tc::mbar_init;
using tc::mbar_try_wait;
using tc::mbar_wait_sleep;
using tc::prefetch_tmap;
using tc::smem_u32;
using tc::sw128_desc;
using tc::sw128_mn_desc;
using tc::tmem_fence_after;
using tc::tmem_fence_before;
using tc::tmem_ld32;

constexpr int TM = 256;                   // tile rows (128 per CTA)
constexpr int TN = 256;                   // tile columns (B rows: 128 per CTA)
constexpr int HALF = 128;
constexpr int BK = 64;
constexpr int kStages = 6;                // K stages of the main loop (an epilogue may use fewer)
constexpr int kABytes = HALF * BK * 2;    // 16 KB
constexpr int kBBytes = HALF * BK * 2;    // 16 KB
constexpr int kStageBytes = kABytes + kBBytes;
constexpr int kThreads = 192;
constexpr uint32_t kTmemCols = 512;       // two 256-column fp32 accumulators
constexpr uint64_t kWaitNs = 2000000000ull;

struct alignas(8) Shared {
  uint64_t full[kStages];     // leader: both CTAs' bytes of a stage landed
  uint64_t empty[kStages];    // every CTA: the MMAs reading a stage are done
  uint64_t tmem_full[2];      // every CTA: an accumulator is complete
  uint64_t tmem_empty[2];     // leader: the 8 epilogue warps of the pair read an accumulator
  uint64_t mma_drain;
  uint64_t epi_bar[8][4];     // per epilogue warp: TMA loads into its staging buffers (epilogues that read)
  uint32_t tmem_base;
  int abort;
};

constexpr size_t kSharedSlot = 1024;
static_assert(sizeof(Shared) <= kSharedSlot, "Shared must fit its slot");
// Epilogue staging: per epilogue warp four 32-row x 64-byte buffers (32 bf16 columns each), in the
// 64-byte swizzle of the TMA boxes; stores use two of them alternately, an epilogue that also reads
// a tensor (SwiGLU backward) uses all four as two (gate, up) sets.
constexpr int kEpiBufBytes = 32 * 64;
constexpr int kEpiWarpBufs = 4;
// Dynamic shared memory of a kernel instance: each epilogue type declares its main-loop stage count
// (kStages) and staging buffers per warp (kWarpBufs); one that streams a tensor in trades a stage for
// a deeper staging ring.
template <class Epi>
__host__ __device__ constexpr size_t smem_bytes_for() {
  return (size_t)Epi::kStages * kStageBytes + kSharedSlot + (size_t)Epi::kEpiWarps * Epi::kWarpBufs * kEpiBufBytes +
         1024;
}
// Threads of a CTA: the TMA producer warp, the MMA warp and the epilogue warps (four, one per TMEM
// lane quarter, or eight, two per quarter splitting the tile's columns).
template <class Epi>
__host__ __device__ constexpr int threads_for() { return 64 + 32 * Epi::kEpiWarps; }

__device__ __forceinline__ uint32_t cta_rank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}

// Address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to(uint32_t saddr, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(saddr), "r"(rank));
  return r;
}

// TMA tile load into this CTA's shared memory whose completion is counted on an mbarrier that
// may live in the peer CTA of the pair (cluster address).
__device__ __forceinline__ void tma_load_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(bar_cluster)
      : "memory");
}

__device__ __forceinline__ void umma_pair(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}"
      ::"r"(tmem_d), "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once the MMAs issued so far complete) on the mbarrier at this shared-memory offset
// in both CTAs of the pair.
__device__ __forceinline__ void umma_commit_pair(uint64_t* bar) {
  const uint16_t mask = 0x3;
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;"
      ::"r"(smem_u32(bar)), "h"(mask)
      : "memory");
}

__device__ __forceinline__ void umma_commit_local(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.b64 [%0];"
               ::"r"(smem_u32(bar)) : "memory");
}

// Arrive on an mbarrier of a CTA of the cluster. Only the TMEM reads before it need ordering, and
// tcgen05.fence::before_thread_sync gives that, so no cluster-wide release of global stores.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.relaxed.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// 2-D TMA store of a shared-memory box to global memory (bulk async-group of this thread).
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(x), "r"(y) : "memory");
}
__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// 2-D TMA reduction: global box (x, y) += shared-memory box (element-wise f32 add in L2).
__device__ __forceinline__ void tma_reduce_add_2d(const CUtensorMap* map, const void* src, int x, int y) {
  asm volatile("cp.reduce.async.bulk.tensor.2d.global.shared::cta.add.tile.bulk_group [%0, {%2, %3}], [%1];"
               ::"l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(src)), "r"(x), "r"(y) : "memory");
}
// Wait until at most one of this thread's bulk groups still reads shared memory.
__device__ __forceinline__ void bulk_wait_read1() { asm volatile("cp.async.bulk.wait_group.read 1;" ::: "memory"); }
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Wait until none of this thread's bulk groups still reads shared memory.
__device__ __forceinline__ void bulk_wait_read0() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }
// 2-D TMA load of one box into this CTA's shared memory, completion on an mbarrier of this CTA.
__device__ __forceinline__ void tma_load_box(void* dst, const CUtensorMap* map, uint64_t* bar, int x, int y) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_u32(bar))
      : "memory");
}
__device__ __forceinline__ void fence_async_smem() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }

struct Work {
  int M, N, K;
  int m_tiles, n_tiles;
  int k_blocks;
  int splits;          // K slices per tile (1: no split)
  int kb_per_split;    // 64-wide K blocks per slice (the last slice may be shorter)
  int group;           // tile raster: groups of `group` M tiles, N-major inside a group
  int items;           // m_tiles * n_tiles * splits
};

struct Item {
  int m_blk, n_blk, split, tile;
  int kb0, kb1;        // K blocks [kb0, kb1)
};

__device__ __forceinline__ Item item_at(const Work& w, int it) {
  Item r;
  r.tile = it / w.splits;
  r.split = it - r.tile * w.splits;
  const int per_group = w.group * w.n_tiles;
  const int g = r.tile / per_group;
  const int within = r.tile - g * per_group;
  const int rows_in_group = min(w.group, w.m_tiles - g * w.group);
  r.n_blk = within / rows_in_group;
  r.m_blk = g * w.group + within % rows_in_group;
  r.kb0 = r.split * w.kb_per_split;
  r.kb1 = min(w.k_blocks, r.kb0 + w.kb_per_split);
  return r;
}

// What an epilogue warp gets: its 32 rows start at row0 (lane l owns row row0 + l), the tile's
// columns start at n0; taddr is the TMEM address of (its first lane, the accumulator's column 0).
struct EpiCtx {
  int row0, n0;
  int col0, col1;      // the tile columns this warp handles (all 256 with four epilogue warps)
  int split, splits, tile;
  int slot;            // (tile's warp slot) = cta * 4 + quarter, for per-warp split-K flags
  uint32_t taddr;
  int lane;
  uint8_t* smem;            // this warp's two staging buffers (1024-byte aligned)
  const CUtensorMap* tmap_c; // output tensor map (bf16 [M, N], 32 x 32 boxes, 64-byte swizzle) or null
  const CUtensorMap* tmap_d; // second map of the same kind (a second output, or an input read by TMA) or null
  uint64_t* bar;             // this warp's two mbarriers for TMA loads into its staging buffers
};

// Epi must provide: __device__ bool warp(const EpiCtx&, const Work&, volatile int* abort, uint32_t* status)
// (every lane of the warp calls it; false = a bounded wait gave up) and __device__ void finish(const
// EpiCtx&) (every lane, after the warp's last tile: complete outstanding stores).
template <bool A_MN, bool B_MN, class Epi>
__device__ void gemm_pair_body(const CUtensorMap* tma_a, const CUtensorMap* tma_b, const CUtensorMap* tma_c,
                               const CUtensorMap* tma_d, const Work& w, Epi& epi, uint32_t* status) {
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  constexpr int kStages = Epi::kStages;
  static_assert(kStages <= g2::kStages, "stage barriers");
  static_assert(smem_bytes_for<Epi>() <= 227 * 1024, "shared memory budget");
  Shared* S = reinterpret_cast<Shared*>(smem + (size_t)kStages * kStageBytes);
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cta_rank();
  const bool leader = rank == 0;
  const int cluster = blockIdx.x >> 1;
  const int n_clusters = gridDim.x >> 1;
  volatile int* abort_flag = &S->abort;

  if (threadIdx.x == 0) {
    for (int s = 0; s < kStages; ++s) {
      mbar_init(&S->full[s], 1);
      mbar_init(&S->empty[s], 1);
    }
    for (int a = 0; a < 2; ++a) {
      mbar_init(&S->tmem_full[a], 1);
      mbar_init(&S->tmem_empty[a], 2 * Epi::kEpiWarps);   // every epilogue warp of both CTAs
    }
    mbar_init(&S->mma_drain, 1);
    S->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&S->tmem_base)), "r"(kTmemCols) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  cluster_sync();          // barriers of both CTAs initialised, TMEM allocated in both
  tmem_fence_after();
  const uint32_t tmem_base = S->tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer (both CTAs) ----------------
    if (lane == 0) {
      prefetch_tmap(tma_a);
      prefetch_tmap(tma_b);
      int stage = 0;
      uint32_t phase = 0;
      uint32_t issued = 0;
      bool ok = true;
      for (int it = cluster; it < w.items && ok; it += n_clusters) {
        const Item I = item_at(w, it);
        const int arow = I.m_blk * TM + HALF * (int)rank;
        const int brow = I.n_blk * TN + HALF * (int)rank;
        for (int kb = I.kb0; kb < I.kb1; ++kb) {
          if (!mbar_wait_sleep(&S->empty[stage], phase ^ 1u, abort_flag)) { ok = false; break; }
          uint8_t* sa = smem + (size_t)stage * kStageBytes;
          uint8_t* sb = sa + kABytes;
          const uint32_t bar = map_to(smem_u32(&S->full[stage]), 0);
          if (leader) mbar_arrive_expect_tx(&S->full[stage], 2 * kStageBytes);
          if (A_MN) {
            tma_load_pair(sa, tma_a, bar, arow, kb * BK);
            tma_load_pair(sa + BK * 128, tma_a, bar, arow + 64, kb * BK);
          } else {
            tma_load_pair(sa, tma_a, bar, kb * BK, arow);
          }
          if (B_MN) {
            tma_load_pair(sb, tma_b, bar, brow, kb * BK);
            tma_load_pair(sb + BK * 128, tma_b, bar, brow + 64, kb * BK);
          } else {
            tma_load_pair(sb, tma_b, bar, kb * BK, brow);
          }
          ++issued;
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
      }
      if (!ok) {
        set_status(status, kTimeoutFlag, 200 + rank);
        S->abort = 1;
        // The leader can observe the stage barriers; wait (bounded) for its latest loads.
        if (leader) {
          const uint32_t first = issued > (uint32_t)kStages ? issued - (uint32_t)kStages : 0u;
          for (uint32_t i = first; i < issued; ++i) {
            const uint64_t t0 = globaltimer_ns();
            while (!mbar_try_wait(&S->full[i % kStages], (i / kStages) & 1u)) {
              if (globaltimer_ns() - t0 > kWaitNs) break;
            }
          }
        } else {
          // the peer's copies complete on the leader's barriers: give them a bounded moment to land
          const uint64_t t0 = globaltimer_ns();
          while (globaltimer_ns() - t0 < 200000ull) { }
        }
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer (leader CTA only) ----------------
    if (leader && lane == 0) {
      const uint32_t idesc = tc::idesc_bf16(TM, TN, A_MN, B_MN);
      int stage = 0;
      uint32_t phase = 0;
      int acc = 0;
      uint32_t acc_phase = 0;
      bool ok = true;
      for (int it = cluster; it < w.items && ok; it += n_clusters) {
        const Item I = item_at(w, it);
        if (!mbar_wait_sleep(&S->tmem_empty[acc], acc_phase ^ 1u, abort_flag)) { ok = false; break; }
        tmem_fence_after();
        const uint32_t tmem_d = tmem_base + (uint32_t)(acc * TN);
        for (int kb = I.kb0; kb < I.kb1; ++kb) {
          if (!mbar_wait_sleep(&S->full[stage], phase, abort_flag)) { ok = false; break; }
          tmem_fence_after();
          const uint32_t sa = smem_u32(smem + (size_t)stage * kStageBytes);
          const uint32_t sb = sa + kABytes;
#pragma unroll
          for (int kk = 0; kk < BK / 16; ++kk) {
            const uint64_t ad = A_MN ? sw128_mn_desc(sa + kk * 16 * 128) : sw128_desc(sa + kk * 32);
            const uint64_t bd = B_MN ? sw128_mn_desc(sb + kk * 16 * 128) : sw128_desc(sb + kk * 32);
            umma_pair(tmem_d, ad, bd, idesc, (kb > I.kb0 || kk > 0) ? 1u : 0u);
          }
          umma_commit_pair(&S->empty[stage]);
          if (++stage == kStages) { stage = 0; phase ^= 1u; }
        }
        if (!ok) break;
        umma_commit_pair(&S->tmem_full[acc]);
        if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
      }
      if (!ok) {
        set_status(status, kTimeoutFlag, 202);
        S->abort = 1;
      }
      umma_commit_local(&S->mma_drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&S->mma_drain, 0u)) {
        if (globaltimer_ns() - t0 > kWaitNs) break;
      }
    }
  } else {
    // ---------------- epilogue (warps 2.., both CTAs) ----------------
    static_assert(Epi::kEpiWarps == 4 || Epi::kEpiWarps == 8, "epilogue warps");
    const int ew = warp - 2;                       // epilogue warp index
    const int quarter = warp & 3;                  // the TMEM lane quarter this warp may access
    const int cols = TN / (Epi::kEpiWarps / 4);    // tile columns per warp
    int acc = 0;
    uint32_t acc_phase = 0;
    const uint32_t empty_leader0 = map_to(smem_u32(&S->tmem_empty[0]), 0);
    const uint32_t empty_leader1 = map_to(smem_u32(&S->tmem_empty[1]), 0);
    EpiCtx c;
    c.lane = lane;
    c.smem = reinterpret_cast<uint8_t*>(S) + kSharedSlot + (size_t)ew * Epi::kWarpBufs * kEpiBufBytes;
    c.bar = S->epi_bar[ew];
    c.col0 = (ew >> 2) * cols;
    c.col1 = c.col0 + cols;
    c.tmap_c = tma_c;
    c.tmap_d = tma_d;
    for (int it = cluster; it < w.items; it += n_clusters) {
      const Item I = item_at(w, it);
      c.row0 = I.m_blk * TM + HALF * (int)rank + quarter * 32;
      c.n0 = I.n_blk * TN;
      epi.prefetch(c, w);        // loads that do not depend on the accumulator start under the main loop
      bool ok = mbar_wait_sleep(&S->tmem_full[acc], acc_phase, abort_flag);
      ok = __all_sync(0xffffffffu, ok);
      if (!ok) {
        if (lane == 0) {
          set_status(status, kTimeoutFlag, 203);
          S->abort = 1;
        }
        break;
      }
      tmem_fence_after();
      c.split = I.split;
      c.splits = w.splits;
      c.tile = I.tile;
      c.slot = (int)rank * 4 + quarter;
      c.taddr = tmem_base + ((uint32_t)(quarter * 32) << 16) + (uint32_t)(acc * TN);
      const bool eok = epi.warp(c, w, abort_flag, status);
      tmem_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive_cluster(acc ? empty_leader1 : empty_leader0);
      if (!eok) break;
      if (++acc == 2) { acc = 0; acc_phase ^= 1u; }
    }
    epi.finish(c);
  }

  tmem_fence_before();
  __syncthreads();
  __syncwarp();
  cluster_sync();          // the peer's MMAs and arrives that touch this CTA are over
  tmem_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemCols)
                 : "memory");
  }
}

// ---------------------------------------------------------------------------
// Epilogues
// ---------------------------------------------------------------------------

// Stage 32 fp32 values of row `r` (this lane) of a 32 x 32 bf16 box into the warp's next staging
// buffer and store the box at (x, y) of `map` with one TMA store. `chunk` counts the warp's
// staged boxes (the buffer alternates); every lane calls it.
__device__ __forceinline__ void stage_store(const EpiCtx& c, uint32_t& chunk, const float* v,
                                            const CUtensorMap* map, int x, int y) {
  // four staging buffers in rotation: up to three earlier stores may still be reading theirs
  uint8_t* buf = c.smem + (chunk & 3u) * kEpiBufBytes;
  if (chunk >= 4) {
    if (c.lane == 0) asm volatile("cp.async.bulk.wait_group.read 3;" ::: "memory");   // this buffer's last store read it
    __syncwarp();
  }
  const int r = c.lane;
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    Vec16<__nv_bfloat16> q;
#pragma unroll
    for (int e = 0; e < 8; ++e) q.v[e] = __float2bfloat16_rn(v[8 * j + e]);
    const int pj = j ^ ((r >> 1) & 3);             // 64-byte swizzle
    *reinterpret_cast<uint4*>(buf + r * 64 + pj * 16) = q.u;
  }
  fence_async_smem();
  __syncwarp();
  if (c.lane == 0) {
    tma_store_2d(map, buf, x, y);
    bulk_commit();
  }
  ++chunk;
}

// The same for a 32-row x 64-column bf16 box (128-byte rows: whole L2 lines), 128-byte swizzle, four
// 4 KB buffers per warp in rotation (epilogues with kWarpBufs >= 8).
__device__ __forceinline__ void stage_store_wide(const EpiCtx& c, uint32_t& chunk, const float* v,
                                                 const CUtensorMap* map, int x, int y) {
  uint8_t* buf = c.smem + (chunk & 3u) * (2 * kEpiBufBytes);
  if (chunk >= 4) {
    if (c.lane == 0) asm volatile("cp.async.bulk.wait_group.read 3;" ::: "memory");   // this buffer's last store read it
    __syncwarp();
  }
  const int r = c.lane;
#pragma unroll
  for (int j = 0; j < 8; ++j)
    *reinterpret_cast<uint4*>(buf + r * 128 + ((j ^ (r & 7)) << 4)) = pack16<__nv_bfloat16>(v + 8 * j);
  fence_async_smem();
  __syncwarp();
  if (c.lane == 0) {
    tma_store_2d(map, buf, x, y);
    bulk_commit();
  }
  ++chunk;
}

__device__ __forceinline__ void round_bf16(float* v, int n) {
  for (int i = 0; i < n; ++i) v[i] = __bfloat162float(__float2bfloat16_rn(v[i]));
}

// Y = acc (+ bias[n]) (+ R[m, n]) stored as bf16 (or fp32 with out_f32).
// bf16 output with a tensor map: each 32-column chunk of the warp's 32 rows is converted, written
// to a staging buffer (64-byte rows, 64-byte swizzle: 16-byte chunk j of row r sits at chunk
// j ^ ((r >> 1) & 3), so a warp's 16-byte writes hit every bank group evenly) and stored by one
// TMA store (full lines, out-of-range rows and columns clipped by the TMA unit); two buffers per
// warp alternate. Otherwise each thread stores its row directly.
struct LinearEpi {
  static constexpr int kEpiWarps = 4;
  static constexpr int kStages = g2::kStages;
  static constexpr int kWarpBufs = kEpiWarpBufs;
  __device__ __forceinline__ void prefetch(const EpiCtx&, const Work&) {}
  void* C;
  int64_t ldc;
  const __nv_bfloat16* bias;   // [N] or null
  const __nv_bfloat16* R;      // [M, N] residual or null
  int64_t ldr;
  int out_f32;
  int vec_ok;                  // C (and R) rows 16-byte aligned
  int use_tma;                 // bf16 output through the staged TMA store
  uint32_t chunk;              // chunks this warp has staged so far (buffer = chunk & 3)

  __device__ __forceinline__ void add_bias_res(float* v, int m, int n, int N, bool full) const {
    if (bias) {
      if (full) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          float b[8];
          load16<__nv_bfloat16>(bias + n + j, b);
#pragma unroll
          for (int q = 0; q < 8; ++q) v[j + q] += b[q];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) if (n + j < N) v[j] += __bfloat162float(bias[n + j]);
      }
    }
    if (R) {
      const __nv_bfloat16* r = R + (int64_t)m * ldr + n;
      if (full) {
#pragma unroll
        for (int j = 0; j < 32; j += 8) {
          float b[8];
          load16<__nv_bfloat16>(r + j, b);
#pragma unroll
          for (int q = 0; q < 8; ++q) v[j + q] += b[q];
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j) if (n + j < N) v[j] += __bfloat162float(r[j]);
      }
    }
  }

  __device__ bool warp(const EpiCtx& c, const Work& w, volatile int*, uint32_t*) {
    const int m = c.row0 + c.lane;
    const bool live = m < w.M;
    if (use_tma) {
#pragma unroll 1
      for (int cc = 0; cc < TN; cc += 32) {
        float v[32];
        tmem_ld32(c.taddr + cc, v);
        const int n = c.n0 + cc;
        if (c.row0 >= w.M || n >= w.N) continue;        // whole chunk outside C (warp-uniform)
        if (live) add_bias_res(v, m, n, w.N, vec_ok && n + 32 <= w.N);
        stage_store(c, chunk, v, c.tmap_c, n, c.row0);
      }
      return true;
    }
#pragma unroll 1
    for (int cc = 0; cc < TN; cc += 32) {
      float v[32];
      tmem_ld32(c.taddr + cc, v);
      const int n = c.n0 + cc;
      if (!live || n >= w.N) continue;
      const bool full = vec_ok && n + 32 <= w.N;
      add_bias_res(v, m, n, w.N, full);
      if (out_f32) {
        float* dst = reinterpret_cast<float*>(C) + (int64_t)m * ldc + n;
        if (full) {
#pragma unroll
          for (int j = 0; j < 32; j += 4) *reinterpret_cast<float4*>(dst + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) if (n + j < w.N) dst[j] = v[j];
        }
      } else {
        __nv_bfloat16* dst = reinterpret_cast<__nv_bfloat16*>(C) + (int64_t)m * ldc + n;
        if (full) {
#pragma unroll
          for (int j = 0; j < 32; j += 8) store16<__nv_bfloat16>(dst + j, v + j);
        } else {
#pragma unroll
          for (int j = 0; j < 32; ++j) if (n + j < w.N) dst[j] = __float2bfloat16_rn(v[j]);
        }
      }
    }
    return true;
  }

  __device__ void finish(const EpiCtx& c) {
    if (use_tma && c.lane == 0) bulk_wait_all();
    __syncwarp();
  }
};

// fp32 C = acc (overwrite) or C += acc (accumulate), with ordered split-K: split 0 writes (or
// adds to the caller's C), split j > 0 waits for split j-1 of the same rows and adds.
// flags: one 32-bit word per (tile, warp slot); a value (epoch << 8) | j means "splits < j done".
// With an fp32 tensor map (tmap_c: 32 x 32 boxes, 128-byte swizzle) each 32-column chunk is staged
// in shared memory and written by one TMA store, or added into C by one TMA reduction (the L2
// performs the read-add-write on full lines); a split releases its flag only after its
// reductions have completed, so the additions into C happen in split order (deterministic).
// Without a map (unaligned C) every thread reads and writes its own row.
struct AccumF32Epi {
  static constexpr int kEpiWarps = 4;
  static constexpr int kStages = g2::kStages;
  static constexpr int kWarpBufs = kEpiWarpBufs;
  __device__ __forceinline__ void prefetch(const EpiCtx&, const Work&) {}
  float* C;
  int64_t ldc;
  int accumulate;
  int vec_ok;
  int use_tma;
  uint32_t* flags;
  uint32_t epoch;
  uint32_t chunk;

  __device__ bool warp(const EpiCtx& c, const Work& w, volatile int* abort_flag, uint32_t* status) {
    const int m = c.row0 + c.lane;
    const bool live = m < w.M;
    uint32_t* flag = flags ? flags + (int64_t)c.tile * 8 + c.slot : nullptr;
    bool ok = true;
    if (c.split > 0) {
      if (c.lane == 0) {
        const uint32_t want = (epoch << 8) | (uint32_t)c.split;
        const uint64_t t0 = globaltimer_ns();
        uint32_t spins = 0;
        while (ld_acquire_gpu(flag) != want) {
          __nanosleep(128);
          if ((++spins & 63u) == 0 && (*abort_flag || globaltimer_ns() - t0 > kWaitNs)) { ok = false; break; }
        }
        if (!ok) set_status(status, kTimeoutFlag, 210);
        asm volatile("fence.proxy.async.global;" ::: "memory");   // the previous split's adds precede ours
      }
      ok = __shfl_sync(0xffffffffu, ok ? 1 : 0, 0) != 0;
      __syncwarp();
    }
    const bool add = accumulate || c.split > 0;
#pragma unroll 1
    for (int cc = 0; cc < TN; cc += 32) {
      float v[32];
      tmem_ld32(c.taddr + cc, v);
      const int n = c.n0 + cc;
      if (use_tma) {
        if (!ok || c.row0 >= w.M || n >= w.N) continue;           // warp-uniform
        uint8_t* buf = c.smem + (chunk & 1u) * 2 * kEpiBufBytes;   // 32 rows x 128 bytes
        if (chunk >= 2) {
          if (c.lane == 0) bulk_wait_read1();
          __syncwarp();
        }
        const int r = c.lane;
#pragma unroll
        for (int q = 0; q < 8; ++q)
          *reinterpret_cast<float4*>(buf + r * 128 + ((q ^ (r & 7)) << 4)) =
              make_float4(v[4 * q], v[4 * q + 1], v[4 * q + 2], v[4 * q + 3]);
        fence_async_smem();
        __syncwarp();
        if (c.lane == 0) {
          if (add) tma_reduce_add_2d(c.tmap_c, buf, n, c.row0);
          else tma_store_2d(c.tmap_c, buf, n, c.row0);
          bulk_commit();
        }
        ++chunk;
        continue;
      }
      if (!ok || !live || n >= w.N) continue;
      float* dst = C + (int64_t)m * ldc + n;
      if (vec_ok && n + 32 <= w.N) {
#pragma unroll
        for (int j = 0; j < 32; j += 4) {
          float4 o = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
          if (add) {
            const float4 p = *reinterpret_cast<const float4*>(dst + j);
            o.x += p.x; o.y += p.y; o.z += p.z; o.w += p.w;
          }
          *reinterpret_cast<float4*>(dst + j) = o;
        }
      } else {
#pragma unroll
        for (int j = 0; j < 32; ++j)
          if (n + j < w.N) dst[j] = add ? dst[j] + v[j] : v[j];
      }
    }
    if (ok && c.split + 1 < c.splits) {
      __syncwarp();
      if (c.lane == 0) {
        if (use_tma) {
          bulk_wait_all();                                        // our adds are performed in C
          asm volatile("fence.proxy.async.global;" ::: "memory");
        }
        __threadfence();
        asm volatile("st.release.gpu.global.u32 [%0], %1;" ::"l"(flag), "r"((epoch << 8) | (uint32_t)(c.split + 1))
                     : "memory");
      }
    }
    return ok;
  }

  __device__ void finish(const EpiCtx& c) {
    if (use_tma && c.lane == 0) bulk_wait_all();
    __syncwarp();
  }
};

// SwiGLU fused into the gate/up projection. The weight's rows are interleaved in 128-row blocks
// (block b of the output = 128 gate columns of hidden units [128 b, 128 b + 128), then the 128
// up columns of the same units), so each 256-column tile holds matching gate and up columns.
// The epilogue stores the pre-activations (the tile itself, bf16, needed by the backward) with
// the first map and act = silu(gate) * up for the tile's 128 hidden units with the second.
// Gate and up are rounded to bf16 before act is formed, as when act is computed from stored ab.
struct SwiGluFwdEpi {
  static constexpr int kEpiWarps = 4;
  // Stores gate, up (the backward's pre-activations) and silu(gate) * up for 64 hidden units at a
  // time as 32 x 64 boxes with 128-byte rows (whole L2 lines); one K stage fewer pays for the four
  // 4 KB staging buffers per warp.
  static constexpr int kStages = g2::kStages - 1;
  static constexpr int kWarpBufs = 8;
  __device__ __forceinline__ void prefetch(const EpiCtx&, const Work&) {}
  uint32_t chunk;

  __device__ bool warp(const EpiCtx& c, const Work& w, volatile int*, uint32_t*) {
    if (c.row0 >= w.M) {
      // every TMEM load is warp-collective: still read the accumulator, store nothing
#pragma unroll 1
      for (int cc = 0; cc < TN; cc += 32) { float v[32]; tmem_ld32(c.taddr + cc, v); }
      return true;
    }
    const int h0 = c.n0 / 2;                       // first hidden unit of this tile
#pragma unroll 1
    for (int cc = 0; cc < TN / 2; cc += 64) {
      float g[64], u[64];
      tmem_ld32(c.taddr + cc, g);
      tmem_ld32(c.taddr + cc + 32, g + 32);
      tmem_ld32(c.taddr + 128 + cc, u);
      tmem_ld32(c.taddr + 128 + cc + 32, u + 32);
      stage_store_wide(c, chunk, g, c.tmap_c, c.n0 + cc, c.row0);
      stage_store_wide(c, chunk, u, c.tmap_c, c.n0 + 128 + cc, c.row0);
      round_bf16(g, 64);
      round_bf16(u, 64);
#pragma unroll
      for (int j = 0; j < 64; ++j) g[j] = g[j] * sigmoidf_fast(g[j]) * u[j];
      stage_store_wide(c, chunk, g, c.tmap_d, h0 + cc, c.row0);
    }
    return true;
  }

  __device__ void finish(const EpiCtx& c) {
    if (c.lane == 0) bulk_wait_all();
    __syncwarp();
  }
};

// SwiGLU backward fused into the down projection's input gradient: the accumulator tile is
// d_act[m, j] for 256 hidden units j; the epilogue loads the stored pre-activations (gate, up) of
// those units from the interleaved ab [M, 2F] with TMA boxes (second map) into the warp's staging
// buffers -- the next chunk's boxes are in flight while this one is computed -- and stores
//   d_gate = d_act * up * s * (1 + gate (1 - s)),  d_up = d_act * gate * s,  s = sigmoid(gate)
// in place, then TMA-stores both boxes into d_ab (same interleaved layout, first map), so d_act
// never reaches memory and every global access is a full-line TMA transfer.
struct SwiGluBwdEpi {
  // The epilogue streams 4 bytes in and 4 bytes out per output element, as much DRAM traffic as the
  // main loop's arithmetic at D = 1024, and one warp per TMEM lane quarter left its loads, SFU and
  // shared-memory latencies exposed: eight epilogue warps (two per quarter, each half of the tile's
  // columns) hide them for one another. Each works on 64-column chunks whose (gate, up) boxes have
  // 128-byte rows (whole L2 lines) in one 8 KB staging set; a tile's first load is issued before its
  // accumulator is ready. One K stage fewer pays for the staging shared memory.
  static constexpr int kEpiWarps = 8;
  static constexpr int kStages = g2::kStages - 1;
  static constexpr int kWarpBufs = 4;               // one (gate, up) set of 4 KB boxes, in 2 KB units
  static constexpr int kBoxBytes = 32 * 128;
  uint32_t loads;     // lane 0: chunks whose loads this warp issued (counted over all its tiles)
  uint32_t done;      // chunks this warp stored (counted over all its tiles)
  uint32_t inited;

  // lane 0: load chunk `loads` (tile column j, a multiple of 64) into the staging set once the
  // previous chunk's stores have read it
  __device__ __forceinline__ void issue(const EpiCtx& c, int j) {
    bulk_wait_read0();
    const int gcol = 256 * (j >> 7) + (j & 127);
    uint8_t* gb = c.smem;
    uint8_t* ub = gb + kBoxBytes;
    mbar_arrive_expect_tx(&c.bar[0], 2 * kBoxBytes);
    tma_load_box(gb, c.tmap_d, &c.bar[0], gcol, c.row0);
    tma_load_box(ub, c.tmap_d, &c.bar[0], gcol + 128, c.row0);
    ++loads;
  }

  __device__ __forceinline__ static int live_chunks(const EpiCtx& c, const Work& w) {
    if (c.row0 >= w.M || c.n0 + c.col0 >= w.N) return 0;
    const int n = (w.N - c.n0 - c.col0 + 63) / 64;  // N is a multiple of 128
    const int m = (c.col1 - c.col0) / 64;
    return n < m ? n : m;
  }

  __device__ void prefetch(const EpiCtx& c, const Work& w) {
    if (!inited) {
      if (c.lane == 0) {
        mbar_init(&c.bar[0], 1);
        asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
      }
      __syncwarp();
      inited = 1;
    }
    if (c.lane == 0 && live_chunks(c, w) > 0) issue(c, c.n0 + c.col0);
  }

  __device__ bool warp(const EpiCtx& c, const Work& w, volatile int* abort_flag, uint32_t* status) {
    const int nch = live_chunks(c, w);               // live 64-column chunks of this warp's columns
    bool ok = true;
#pragma unroll 1
    for (int cc = c.col0; cc < c.col1; cc += 64) {
      float d[64];
      tmem_ld32(c.taddr + cc, d);                   // warp-collective: every lane, every chunk
      tmem_ld32(c.taddr + cc + 32, d + 32);
      const int k = (cc - c.col0) / 64;
      if (k >= nch) continue;                       // warp-uniform
      const uint32_t g = done;                      // this chunk's number, counted over the warp's tiles
      bool got = mbar_wait_sleep(&c.bar[0], g & 1u, abort_flag);
      got = __all_sync(0xffffffffu, got);
      if (!got) {
        if (c.lane == 0) set_status(status, kTimeoutFlag, 220);
        ok = false;
        break;
      }
      uint8_t* gb = c.smem;
      uint8_t* ub = gb + kBoxBytes;
      const int r = c.lane;
#pragma unroll
      for (int q = 0; q < 8; ++q) {
        const int off = r * 128 + ((q ^ (r & 7)) << 4);   // 128-byte swizzle of the TMA box
        float g8[8], u[8];
        load16<__nv_bfloat16>(reinterpret_cast<const __nv_bfloat16*>(gb + off), g8);
        load16<__nv_bfloat16>(reinterpret_cast<const __nv_bfloat16*>(ub + off), u);
        float dg[8], du[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) {
          const float sg = sigmoidf_fast(g8[e]);
          const float dd = d[8 * q + e];
          du[e] = dd * g8[e] * sg;
          dg[e] = dd * u[e] * sg * (1.f + g8[e] * (1.f - sg));
        }
        store16<__nv_bfloat16>(reinterpret_cast<__nv_bfloat16*>(gb + off), dg);
        store16<__nv_bfloat16>(reinterpret_cast<__nv_bfloat16*>(ub + off), du);
      }
      fence_async_smem();
      __syncwarp();
      if (c.lane == 0) {
        const int j = c.n0 + cc;
        const int gcol = 256 * (j >> 7) + (j & 127);
        tma_store_2d(c.tmap_c, gb, gcol, c.row0);
        tma_store_2d(c.tmap_c, ub, gcol + 128, c.row0);
        bulk_commit();
      }
      ++done;
      if (k + 1 < nch && c.lane == 0) issue(c, c.n0 + cc + 64);   // after this chunk's stores read the set
    }
    return ok;
  }

  __device__ void finish(const EpiCtx& c) {
    if (c.lane == 0) bulk_wait_all();
    __syncwarp();
  }
};

}  // namespace g2
}  // namespace nfb
