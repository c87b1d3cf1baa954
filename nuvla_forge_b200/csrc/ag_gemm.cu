// FSDP parameter all-gather fused into the first consuming tcgen05 GEMM.
//
//   Y[M, N] = X[M, K] @ W[N, K]^T       W = rows of a parameter unit's flat bf16 buffer
//
// A parameter unit's flat bf16 buffer is split into `world` contiguous shards;
// rank q keeps shard q at byte `shard_off` of its CUDA-IPC workspace, mapped
// into every rank. This ONE persistent kernel gathers the unit's flat range
// [lo, hi) into the local `full` buffer AND runs the GEMM that first consumes
// it, so the NVLink transfer overlaps the tensor-core tiles:
//
// * warp 6 of every CTA is the gather worker: one lane streams 16 KB chunks of
//   the shards (peer or local memory) into a two-buffer shared-memory ring
//   with 1-D bulk async copies (cp.async.bulk, mbarrier completion, no
//   multicast) and writes each chunk to `full` with a bulk store. A buffer is
//   reloaded as soon as its store has read it; once a store has completed
//   (checked lazily, two stores may stay in flight) the lane adds the chunk's
//   bytes to the ready counter of every W row block (BN rows) the chunk
//   overlaps (red.release.gpu).
// * Each CTA first takes its share of the chunks that hold W, in flat order,
//   so W's row blocks land first and in order; then its share of the rest of
//   the unit with the owners interleaved chunk by chunk and rotated by rank:
//   every rank needs W from the same one or two owners, but the remaining
//   bytes come from all owners at once, each rank starting at a different one,
//   so every link stays busy and no owner serves all the readers at once.
// * The tile order is M-major inside each N block (all M tiles of N block 0,
//   then N block 1, ...), so the first wave of tiles needs only the first few
//   row blocks. Before a tile's first B load the TMA producer waits until its
//   row block's counter is complete (ld.acquire.gpu, then fence.proxy.async so
//   the TMA reads see the bulk stores) -- bounded, like every wait here.
// * The kernel is launched cooperatively with one CTA per SM, so every CTA a
//   producer may wait on is resident. No wait depends on another rank: the
//   shards must be stable for the kernel's duration, which the caller
//   guarantees (an all-gather barrier after each optimizer step and the
//   reduce-scatter barriers before the next one).
//
// No counterpart kernel exists in the reference (torch FSDP there issues a
// separate NCCL all-gather of one flat parameter before each forward,
// nuvla_forge/train.py:158-160).
#include <cstdlib>

#include "tc_gemm.cuh"
#include "tc_host.cuh"

namespace nfb {
namespace tc {

constexpr int kAgMaxWorld = 8;
constexpr int kAgChunk = 16384;
constexpr int kAgBufs = 2;
constexpr int kAgPending = 2;   // bulk stores allowed in flight before the oldest is waited for (wait_group 2)
constexpr int kAgMaxNBlocks = 1024;
// Gather orders (see AgGate::rest_chunk); kOrderFlat is one list in flat order starting at W.
constexpr int kOrderFlat = 0, kOrderOwnFirst = 1, kOrderPeersFirst = 2, kOrderInterleaved = 3;

__device__ __forceinline__ void bulk_load(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
  asm volatile("cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];"
               ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
               : "memory");
}

__device__ __forceinline__ void bulk_store(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;"
               ::"l"(reinterpret_cast<uint64_t>(dst)), "r"(smem_u32(src)), "r"(bytes) : "memory");
  asm volatile("cp.async.bulk.commit_group;" ::: "memory");
}

__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// all but the kAgPending most recent bulk stores complete
__device__ __forceinline__ void bulk_wait_older() { asm volatile("cp.async.bulk.wait_group 2;" ::: "memory"); }
// every issued bulk store has finished reading its shared-memory source
__device__ __forceinline__ void bulk_wait_reads() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

struct AgGate {
  static constexpr int kWarps = 1;       // warp 6: the gather worker
  static constexpr size_t kSmemBytes = (size_t)kWarps * kAgBufs * kAgChunk + 64 + kAgMaxNBlocks / 8;

  uint64_t base[kAgMaxWorld];   // every rank's workspace base, mapped into this process
  int64_t shard_off;            // byte offset of the unit's shard inside each workspace
  int64_t shard_bytes;          // bytes per shard (multiple of 16)
  int world, rank;
  int order;                    // kOrder*
  uint8_t* full;                // local flat buffer being gathered
  int64_t lo, hi;               // flat byte range gathered by this launch
  int64_t w0, w_bytes, blk_bytes;  // W's flat byte offset, its size, bytes per BN-row block
  uint32_t* ready;              // [N blocks] bytes landed per W row block (zero at launch)
  uint32_t* status;

  uint8_t* buf;                 // shared memory (bound per thread)
  uint64_t* bar;
  uint32_t* known;              // producer-private bitmap of row blocks seen complete

  __device__ void bind(uint8_t* sm) {
    buf = sm;
    bar = reinterpret_cast<uint64_t*>(sm + (size_t)kWarps * kAgBufs * kAgChunk);
    known = reinterpret_cast<uint32_t*>(sm + (size_t)kWarps * kAgBufs * kAgChunk + 64);
  }
  __device__ void init() {
    for (int i = 0; i < kWarps * kAgBufs; ++i) mbar_init(&bar[i], 1);
    for (int i = 0; i < kAgMaxNBlocks / 32; ++i) known[i] = 0u;
  }

  __device__ __forceinline__ uint32_t expected(int g) const {
    const int64_t rest = w_bytes - (int64_t)g * blk_bytes;
    return (uint32_t)(rest < blk_bytes ? rest : blk_bytes);
  }

  // Producer lane: wait until W's row block g is complete in `full`.
  __device__ bool wait_nblock(int g, volatile int* abort_flag) {
    const uint32_t bit = 1u << (g & 31);
    if (known[g >> 5] & bit) return true;
    const uint32_t need = expected(g);
    const uint64_t t0 = globaltimer_ns();
    uint32_t spins = 0;
    while (ld_acquire_gpu(ready + g) < need) {
      if ((++spins & 63u) == 0) {
        if (*abort_flag) return false;
        if (globaltimer_ns() - t0 > kWaitNs) {
          set_status(status, kTimeoutFlag, 110);
          return false;
        }
      }
    }
    asm volatile("fence.proxy.async.global;" ::: "memory");
    known[g >> 5] |= bit;
    return true;
  }

  __device__ void signal(int64_t f0, int64_t f1) {
    const int64_t a = f0 > w0 ? f0 : w0;
    const int64_t b = f1 < w0 + w_bytes ? f1 : w0 + w_bytes;
    if (a >= b) return;
    const int g0 = (int)((a - w0) / blk_bytes), g1 = (int)((b - 1 - w0) / blk_bytes);
    for (int g = g0; g <= g1; ++g) {
      const int64_t lo_g = w0 + (int64_t)g * blk_bytes;
      const int64_t ga = a > lo_g ? a : lo_g;
      const int64_t gb = b < lo_g + blk_bytes ? b : lo_g + blk_bytes;
      red_release_gpu_add(ready + g, (uint32_t)(gb - ga));
    }
  }

  // Chunk lists. Chunks are shard-aligned: chunk c covers bytes [q*S + j*C, min(q*S + (j+1)*C, (q+1)*S))
  // of the flat unit, with q = c / cps, j = c % cps, clipped to [lo, hi).
  //   W list: the chunks overlapping W, in flat order (all ranks need them first, in this order).
  //   rest list: every other chunk, owners interleaved and rotated by rank (rest_chunk).
  __device__ __forceinline__ int64_t cps() const { return (shard_bytes + kAgChunk - 1) / kAgChunk; }
  __device__ __forceinline__ int64_t chunk_of(int64_t f) const {
    const int64_t q = f / shard_bytes;
    return q * cps() + (f - q * shard_bytes) / kAgChunk;
  }
  __device__ __forceinline__ int64_t w_first() const { return chunk_of(w0); }
  __device__ __forceinline__ int64_t w_last() const { return chunk_of(w0 + w_bytes - 1); }
  __device__ __forceinline__ int64_t c_first() const { return chunk_of(lo); }
  __device__ __forceinline__ int64_t c_last() const { return chunk_of(hi - 1); }

  // Owner q's chunks outside W (inside [lo, hi)): up to two ranges [p0a, p0b], [p1a, p1b].
  __device__ int64_t owner_rest(int q, int64_t k) const {
    const int64_t n = cps(), wf = w_first(), wl = w_last(), cf = c_first(), cl = c_last();
    int64_t a = (int64_t)q * n, b = a + n - 1;
    a = a > cf ? a : cf;
    b = b < cl ? b : cl;
    if (a > b) return -1;
    const int64_t p0a = a, p0b = (wf - 1 < b) ? wf - 1 : b;
    const int64_t p1a = (wl + 1 > a) ? wl + 1 : a, p1b = b;
    if (p0b >= p0a) {
      if (k <= p0b - p0a) return p0a + k;
      k -= p0b - p0a + 1;
    }
    if (p1b >= p1a && k <= p1b - p1a) return p1a + k;
    return -1;
  }

  // Number of owner q's chunks outside W.
  __device__ int64_t owner_rest_count(int q) const {
    const int64_t n = cps(), cf = c_first(), cl = c_last();
    int64_t a = (int64_t)q * n, b = a + n - 1;
    a = a > cf ? a : cf;
    b = b < cl ? b : cl;
    if (a > b) return 0;
    const int64_t ia = a > w_first() ? a : w_first(), ib = b < w_last() ? b : w_last();
    return (b - a + 1) - (ib >= ia ? ib - ia + 1 : 0);
  }

  // i-th entry of the rest list, or -1 for an entry to skip and -2 past the end. Orders:
  //   kOrderInterleaved: owners interleaved chunk by chunk, entry i from owner (rank + 1 + i) % world;
  //   kOrderPeersFirst:  owner by owner, rank+1, rank+2, ..., this rank's own shard last;
  //   kOrderOwnFirst:    owner by owner, this rank's own shard first, then rank+1, ...
  __device__ int64_t rest_chunk(int64_t i) const {
    if (order == kOrderInterleaved) {
      const int64_t k = i / world;
      if (k >= cps()) return -2;
      return owner_rest((int)((rank + 1 + i % world) % world), k);
    }
    for (int j = 0; j < world; ++j) {
      const int q = (rank + j + (order == kOrderOwnFirst ? 0 : 1)) % world;
      const int64_t n = owner_rest_count(q);
      if (i < n) return owner_rest(q, i);
      i -= n;
    }
    return -2;
  }

  __device__ bool chunk_range(int64_t c, int64_t& f0, int64_t& f1, int& q) const {
    const int64_t n = cps();
    q = (int)(c / n);
    f0 = (int64_t)q * shard_bytes + (c - (int64_t)q * n) * kAgChunk;
    f1 = f0 + kAgChunk < (int64_t)(q + 1) * shard_bytes ? f0 + kAgChunk : (int64_t)(q + 1) * shard_bytes;
    f0 = f0 > lo ? f0 : lo;
    f1 = f1 < hi ? f1 : hi;
    return f1 > f0;
  }

  // Gather worker: lane 0 of warp 6 issues every copy of this CTA's share of the W list and then of
  // the rest list (entries blockIdx.x, blockIdx.x + gridDim.x, ... of each), kAgBufs chunks in flight.
  __device__ void worker(int wi, uint8_t*, volatile int* abort_flag) {
    if ((threadIdx.x & 31) != 0) return;
    uint8_t* mybuf = buf + (size_t)wi * kAgBufs * kAgChunk;
    uint64_t* mybar = bar + wi * kAgBufs;
    const int64_t wf = w_first(), wl = w_last();
    int64_t next_i = blockIdx.x;
    int list = 0;   // 0: W list, then 1: rest list
    int64_t rf0[kAgBufs], rf1[kAgBufs];
    uint32_t rphase[kAgBufs];
    bool has[kAgBufs];
    for (int s = 0; s < kAgBufs; ++s) { rphase[s] = 0u; has[s] = false; }

    auto load_next = [&](int slot) -> bool {
      while (true) {
        int64_t c;
        if (order == kOrderFlat) {
          const int64_t total = cps() * world;
          if (next_i >= total) return false;
          c = (wf + next_i) % total;
        } else if (list == 0) {
          c = wf + next_i;
          if (c > wl) {            // this CTA's share of W is issued: continue with its share of the rest
            list = 1;
            next_i = blockIdx.x;
            continue;
          }
        } else {
          c = rest_chunk(next_i);
          if (c == -2) return false;
          if (c < 0) {
            next_i += gridDim.x;
            continue;
          }
        }
        next_i += gridDim.x;
        int64_t f0, f1;
        int q;
        if (!chunk_range(c, f0, f1, q)) continue;
        const uint8_t* src = reinterpret_cast<const uint8_t*>(base[q]) + shard_off + (f0 - (int64_t)q * shard_bytes);
        mbar_arrive_expect_tx(&mybar[slot], (uint32_t)(f1 - f0));
        bulk_load(mybuf + (size_t)slot * kAgChunk, src, (uint32_t)(f1 - f0), &mybar[slot]);
        rf0[slot] = f0;
        rf1[slot] = f1;
        return true;
      }
    };

    for (int s = 0; s < kAgBufs; ++s) {
      has[s] = load_next(s);
      if (!has[s]) break;
    }
    // Stores issued but not yet known complete, oldest first. A buffer is re-armed as soon as its
    // store has READ it; the chunk's bytes are published only once its store has COMPLETED, which
    // is waited for lazily (at most kAgPending stores stay in flight).
    int64_t pf0[kAgPending + 1], pf1[kAgPending + 1];
    int npend = 0;
    auto publish = [&](int n) {
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __threadfence();
      for (int k = 0; k < n; ++k) signal(pf0[k], pf1[k]);
      for (int k = n; k < npend; ++k) { pf0[k - n] = pf0[k]; pf1[k - n] = pf1[k]; }
      npend -= n;
    };
    int slot = 0;
    while (true) {
      bool any = false;
      for (int s = 0; s < kAgBufs; ++s) any |= has[s];
      if (!any) break;
      if (!has[slot]) { slot = (slot + 1) % kAgBufs; continue; }
      if (!mbar_wait(&mybar[slot], rphase[slot], abort_flag)) {
        set_status(status, kTimeoutFlag, 111);
        *abort_flag = 1;
        break;
      }
      rphase[slot] ^= 1u;
      has[slot] = false;
      bulk_store(full + rf0[slot], mybuf + (size_t)slot * kAgChunk, (uint32_t)(rf1[slot] - rf0[slot]));
      pf0[npend] = rf0[slot];
      pf1[npend] = rf1[slot];
      ++npend;
      if (npend > kAgPending) {
        bulk_wait_older();            // every store but the kAgPending newest has completed
        publish(npend - kAgPending);
      }
      bulk_wait_reads();              // this buffer has been read by its store: reuse it
      if (*abort_flag) break;
      has[slot] = load_next(slot);
      slot = (slot + 1) % kAgBufs;
    }
    bulk_wait_all();
    publish(npend);
    // copies still in flight must land before the CTA exits (bounded)
    for (int s = 0; s < kAgBufs; ++s) {
      if (!has[s]) continue;
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&mybar[s], rphase[s])) {
        if (globaltimer_ns() - t0 > kWaitNs) break;
      }
    }
  }
};

__global__ void __launch_bounds__(kThreads + 32 * AgGate::kWarps, 1)
    ag_gemm_kernel(const __grid_constant__ CUtensorMap ta, const __grid_constant__ CUtensorMap tb, GemmShape sh,
                   StoreEpi epi, AgGate gate, uint32_t* status) {
  StoreEpi e = epi;
  AgGate g = gate;
  gemm_body<false, false>(&ta, &tb, sh, e, status, g);
}

}  // namespace tc
}  // namespace nfb

using namespace nfb;
using namespace nfb::tc;

static bool al16(int64_t v) { return (v & 15) == 0; }

// Gather the unit's flat bytes [lo, hi) into `full` and compute Y = X @ W^T,
// W = the [N, K] bf16 rows at flat byte offset w_off of the unit. `bases`
// holds every rank's workspace base (device-visible in this process), `ready`
// at least ceil(N / 256) uint32 of scratch. Returns a CUDA error code.
NFB_API int nfb_ag_gemm(const uint64_t* bases, int rank, int world, int64_t shard_off, int64_t shard_bytes, void* full,
                        int64_t lo, int64_t hi, int64_t w_off, int N, int K, const void* X, int64_t ldx, int M,
                        void* Y, int64_t ldy, uint32_t* ready, uint32_t* status, void* stream) {
  if (world < 1 || world > kAgMaxWorld || rank < 0 || rank >= world || M < 1 || N < 1 || K < 8 || K % 8)
    return (int)cudaErrorInvalidValue;
  if (!al16(shard_off) || !al16(shard_bytes) || !al16(lo) || !al16(hi) || !al16(w_off) ||
      !al16((int64_t)reinterpret_cast<uintptr_t>(full)) || shard_bytes <= 0 || lo < 0 ||
      hi > shard_bytes * world || lo > w_off || w_off + (int64_t)N * K * 2 > hi)
    return (int)cudaErrorInvalidValue;
  const int nblk = (N + BN - 1) / BN;
  if (nblk > kAgMaxNBlocks) return (int)cudaErrorInvalidValue;
  cudaStream_t st = (cudaStream_t)stream;
  CUtensorMap ta, tb;
  int rc = make_tmap(&ta, X, M, K, ldx, BM);
  if (rc) return rc;
  rc = make_tmap(&tb, reinterpret_cast<uint8_t*>(full) + w_off, N, K, K, BN);
  if (rc) return rc;
  GemmShape sh = make_shape(M, N, K);
  sh.group = sh.m_tiles;   // M-major inside each N block: early tiles need only the first row blocks
  StoreEpi epi{};
  epi.C = Y; epi.ldc = ldy; epi.out_f32 = 0;
  epi.vec_ok = ((reinterpret_cast<uintptr_t>(Y) & 15) == 0) && ((ldy * 2) % 16 == 0);
  AgGate g{};
  for (int q = 0; q < world; ++q) g.base[q] = bases[q];
  g.shard_off = shard_off;
  g.shard_bytes = shard_bytes;
  g.world = world;
  g.rank = rank;
  {
    const char* e = getenv("NFB_AG_ORDER");
    // measured on 2 x B200: the flat order is fastest with one peer; with more peers each rank starts
    // its non-weight bytes at a different owner
    g.order = e ? atoi(e) : (world <= 2 ? kOrderFlat : kOrderPeersFirst);
    if (g.order < kOrderFlat || g.order > kOrderInterleaved) g.order = kOrderPeersFirst;
  }
  g.full = reinterpret_cast<uint8_t*>(full);
  g.lo = lo;
  g.hi = hi;
  g.w0 = w_off;
  g.w_bytes = (int64_t)N * K * 2;
  g.blk_bytes = (int64_t)BN * K * 2;
  g.ready = ready;
  g.status = status;
  cudaError_t e = cudaMemsetAsync(ready, 0, (size_t)nblk * sizeof(uint32_t), st);
  if (e != cudaSuccess) return (int)e;
  const size_t smem = smem_bytes<AgGate>();
  const int threads = threads_for<AgGate>();
  e = cudaFuncSetAttribute(ag_gemm_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  int per_sm = 0;
  e = cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, ag_gemm_kernel, threads, smem);
  if (e != cudaSuccess) return (int)e;
  if (per_sm < 1) return (int)cudaErrorCooperativeLaunchTooLarge;
  const int grid = sm_count();
  void* args[] = {&ta, &tb, &sh, &epi, &g, &status};
  e = cudaLaunchCooperativeKernel((const void*)ag_gemm_kernel, dim3(grid), dim3(threads), args, smem, st);
  return (int)e;
}

NFB_API int nfb_ag_gemm_max_nblocks() { return kAgMaxNBlocks; }
