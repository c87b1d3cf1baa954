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
// * warp 6 of every CTA is a gather worker: one lane streams 16 KB chunks of
//   the shards (peer or local memory) into a two-buffer shared-memory ring with
//   1-D bulk async copies (cp.async.bulk, mbarrier completion, no multicast)
//   and writes each chunk to `full` with a bulk store. After the store has
//   completed it adds the chunk's bytes to the ready counter of every W row
//   block (BN rows) the chunk overlaps (red.release.gpu).
// * Chunks are taken in a rotated order that starts at W's first byte, so W's
//   row blocks land first and in order; the rest of the unit follows.
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
#include "tc_gemm.cuh"
#include "tc_host.cuh"

namespace nfb {
namespace tc {

constexpr int kAgMaxWorld = 8;
constexpr int kAgChunk = 16384;
constexpr int kAgBufs = 2;
constexpr int kAgMaxNBlocks = 1024;

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

__device__ __forceinline__ uint32_t ld_acquire_gpu(const uint32_t* p) {
  uint32_t v;
  asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(uint32_t* p, uint32_t v) {
  asm volatile("red.release.gpu.global.add.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

struct AgGate {
  static constexpr int kWarps = 1;
  static constexpr size_t kSmemBytes = (size_t)kAgBufs * kAgChunk + 64 + kAgMaxNBlocks / 8;

  uint64_t base[kAgMaxWorld];   // every rank's workspace base, mapped into this process
  int64_t shard_off;            // byte offset of the unit's shard inside each workspace
  int64_t shard_bytes;          // bytes per shard (multiple of 16)
  int world;
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
    bar = reinterpret_cast<uint64_t*>(sm + (size_t)kAgBufs * kAgChunk);
    known = reinterpret_cast<uint32_t*>(sm + (size_t)kAgBufs * kAgChunk + 64);
  }
  __device__ void init() {
    for (int i = 0; i < kAgBufs; ++i) mbar_init(&bar[i], 1);
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

  // Gather worker (warp 6): one lane issues every copy of this CTA's chunks.
  __device__ void worker(int, uint8_t*, volatile int* abort_flag) {
    if ((threadIdx.x & 31) != 0) return;
    const int64_t S = shard_bytes;
    const int64_t cps = (S + kAgChunk - 1) / kAgChunk;
    const int64_t total = cps * world;
    const int64_t start = (w0 / S) * cps + (w0 % S) / kAgChunk;
    int64_t next_i = blockIdx.x;
    int64_t rf0[kAgBufs], rf1[kAgBufs];
    uint32_t rphase[kAgBufs] = {0u, 0u};
    bool has[kAgBufs] = {false, false};

    auto load_next = [&](int slot) -> bool {
      while (next_i < total) {
        const int64_t c = (start + next_i) % total;
        next_i += gridDim.x;
        const int q = (int)(c / cps);
        int64_t f0 = (int64_t)q * S + (c - (int64_t)q * cps) * kAgChunk;
        int64_t f1 = f0 + kAgChunk < (int64_t)(q + 1) * S ? f0 + kAgChunk : (int64_t)(q + 1) * S;
        f0 = f0 > lo ? f0 : lo;
        f1 = f1 < hi ? f1 : hi;
        if (f1 <= f0) continue;
        const uint8_t* src = reinterpret_cast<const uint8_t*>(base[q]) + shard_off + (f0 - (int64_t)q * S);
        mbar_arrive_expect_tx(&bar[slot], (uint32_t)(f1 - f0));
        bulk_load(buf + (size_t)slot * kAgChunk, src, (uint32_t)(f1 - f0), &bar[slot]);
        rf0[slot] = f0;
        rf1[slot] = f1;
        return true;
      }
      return false;
    };

    has[0] = load_next(0);
    has[1] = has[0] && load_next(1);
    int slot = 0;
    while (has[0] || has[1]) {
      if (!has[slot]) { slot ^= 1; continue; }
      if (!mbar_wait(&bar[slot], rphase[slot], abort_flag)) {
        set_status(status, kTimeoutFlag, 111);
        *abort_flag = 1;
        break;
      }
      rphase[slot] ^= 1u;
      has[slot] = false;
      bulk_store(full + rf0[slot], buf + (size_t)slot * kAgChunk, (uint32_t)(rf1[slot] - rf0[slot]));
      bulk_wait_all();   // the chunk is in `full` and the buffer is free
      asm volatile("fence.proxy.async.global;" ::: "memory");
      __threadfence();
      signal(rf0[slot], rf1[slot]);
      if (*abort_flag) break;
      has[slot] = load_next(slot);
      slot ^= 1;
    }
    // copies still in flight must land before the CTA exits (bounded)
    for (int s = 0; s < kAgBufs; ++s) {
      if (!has[s]) continue;
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&bar[s], rphase[s])) {
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
  gemm_body(&ta, &tb, sh, e, status, g);
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
NFB_API int nfb_ag_gemm(const uint64_t* bases, int world, int64_t shard_off, int64_t shard_bytes, void* full,
                        int64_t lo, int64_t hi, int64_t w_off, int N, int K, const void* X, int64_t ldx, int M,
                        void* Y, int64_t ldy, uint32_t* ready, uint32_t* status, void* stream) {
  if (world < 1 || world > kAgMaxWorld || M < 1 || N < 1 || K < 8 || K % 8) return (int)cudaErrorInvalidValue;
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
  StoreEpi epi;
  epi.C = Y; epi.ldc = ldy; epi.out_f32 = 0;
  epi.vec_ok = ((reinterpret_cast<uintptr_t>(Y) & 15) == 0) && ((ldy * 2) % 16 == 0);
  AgGate g{};
  for (int q = 0; q < world; ++q) g.base[q] = bases[q];
  g.shard_off = shard_off;
  g.shard_bytes = shard_bytes;
  g.world = world;
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
