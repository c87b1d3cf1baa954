// Fused collectives over NVLink 5 / NVSwitch peer memory (one process per GPU).
//
// Every rank owns one symmetric buffer (same size on every rank, mapped into
// every peer's address space through CUDA IPC handles, parallel/symm.py); kernels
// receive the base pointers of all ranks' buffers by value and address peer
// memory with ordinary loads and stores. Layout of a rank's symmetric buffer
// is decided by the host runtime (parallel/symm.py) and passed as byte offsets.
//
// Synchronisation: a CTA-pairwise barrier. CTA b of rank r signals CTA b of
// every peer by a system-scope release store into the peer's flag slot
// [slot][b][r] and waits with a system-scope acquire load on its own slots
// [slot][b][q]. Work is partitioned identically on every rank so CTA b only
// ever consumes data produced by the CTAs with index b on the peers. Flag
// values are monotonically increasing epochs supplied by the host, so flags
// never need resetting. Every wait is bounded (%globaltimer); on timeout the
// kernel records (code, where) in a status word, skips the rest of its work
// and returns, so the context stays usable and the host raises.
//
// What is fused, per reference collective site (nuvla_forge/train.py:157-167):
// * nfb_ar_twoshot: DDP bucket all-reduce. fp32 local gradient -> bf16 cast
//   pushed into each slice owner's inbox (phase 1) -> each owner reduces its
//   1/world slice locally and pushes the scaled bf16 result into every rank's
//   outbox (phase 2) -> fp32 unpack into the gradient buffer (phase 3).
//   2(N-1)/N of the bf16 bucket crosses NVLink per rank, all as posted writes.
// * nfb_ar_oneshot: small buckets, one barrier (double-buffered inboxes).
// * nfb_rs_push: FSDP reduce-scatter straight from the fp32 gradient (cast fused).
// * nfb_rs_f32: FSDP reduce-scatter of bf16 gradients into an fp32 shard,
//   fused with the 1/world scale and the shard's sum of squares (for the
//   global gradient-norm clip).
// * nfb_rs_adamw: reduce-scatter fused with the AdamW update of the fp32
//   master shard, writing the bf16 parameter shard for the next all-gather.
// * nfb_allgather: pull all peers' bf16 shards into a local full buffer.
// * nfb_allreduce_scalar: deterministic (rank-ordered) sum of one float.
#include "common.cuh"

namespace nfb {

constexpr int kMaxWorld = 8;
constexpr int kMaxCtas = 256;
constexpr int kSlots = 8;

struct Peers {
  uint64_t base[kMaxWorld];
};

__device__ __forceinline__ uint32_t* flag_ptr(uint64_t base, int64_t flag_off, int slot, int cta, int src_rank) {
  return reinterpret_cast<uint32_t*>(base + flag_off) + ((int64_t)(slot * kMaxCtas + cta) * kMaxWorld + src_rank);
}

// CTA-pairwise barrier across ranks; returns false (all threads) on timeout.
__device__ bool cta_barrier(const Peers& P, int rank, int world, int64_t flag_off, int slot, uint32_t value,
                            uint64_t timeout_ns, uint32_t* status, uint32_t where) {
  __shared__ int s_ok;
  __syncthreads();
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if ((int)threadIdx.x < world) {
    const int q = threadIdx.x;
    __threadfence_system();
    st_release_sys(flag_ptr(P.base[q], flag_off, slot, blockIdx.x, rank), value);
    if (!wait_flag_geq(flag_ptr(P.base[rank], flag_off, slot, blockIdx.x, q), value, timeout_ns)) {
      set_status(status, kTimeoutBarrier, where | ((uint32_t)q << 16));
      s_ok = 0;
    }
  }
  __syncthreads();
  return s_ok != 0;
}

__device__ __forceinline__ void f32x8_to_bf16(const float* in, uint4& out) {
  __nv_bfloat162 h[4];
#pragma unroll
  for (int j = 0; j < 4; ++j) h[j] = __floats2bfloat162_rn(in[2 * j], in[2 * j + 1]);
  out = *reinterpret_cast<uint4*>(h);
}

__device__ __forceinline__ void bf16x8_add(const uint4& u, float* acc) {
  const __nv_bfloat162* h = reinterpret_cast<const __nv_bfloat162*>(&u);
#pragma unroll
  for (int j = 0; j < 4; ++j) {
    float2 f = __bfloat1622float2(h[j]);
    acc[2 * j] += f.x;
    acc[2 * j + 1] += f.y;
  }
}

struct ArArgs {
  Peers peers;
  const float* src; float* dst;
  int64_t n;                 // elements, multiple of 8 * world
  int64_t send_off, recv_off, flag_off;
  int rank, world, slot;
  float scale;
  uint32_t epoch;
  uint64_t timeout_ns;
  uint32_t* status;
};

constexpr int kU = 4;  // 16-byte vectors per thread per iteration (memory-level parallelism)

__device__ __forceinline__ void load_f32x8(const float* p, float* f) {
  const float4* q = reinterpret_cast<const float4*>(p);
  float4 x0 = __ldcs(q), x1 = __ldcs(q + 1);
  f[0] = x0.x; f[1] = x0.y; f[2] = x0.z; f[3] = x0.w; f[4] = x1.x; f[5] = x1.y; f[6] = x1.z; f[7] = x1.w;
}

__device__ __forceinline__ void store_f32x8(float* p, const float* f, bool accumulate) {
  float4* q = reinterpret_cast<float4*>(p);
  if (accumulate) {
    float4 o0 = q[0], o1 = q[1];
    q[0] = make_float4(o0.x + f[0], o0.y + f[1], o0.z + f[2], o0.w + f[3]);
    q[1] = make_float4(o1.x + f[4], o1.y + f[5], o1.z + f[6], o1.w + f[7]);
  } else {
    q[0] = make_float4(f[0], f[1], f[2], f[3]);
    q[1] = make_float4(f[4], f[5], f[6], f[7]);
  }
}

// Push phase shared by the two-shot all-reduce and the reduce-scatter: CTA b
// casts its chunk of every destination slice to bf16 and writes it straight
// into the owner's inbox [rank][v] with (posted) NVLink stores.
__device__ __forceinline__ void push_slices(const ArArgs& a, int64_t slice_vecs, int64_t v0, int64_t v1) {
  for (int s = 0; s < a.world; ++s) {
    uint4* inbox = reinterpret_cast<uint4*>(a.peers.base[s] + a.send_off) + (int64_t)a.rank * slice_vecs;
    const float* src = a.src + (int64_t)s * slice_vecs * 8;
    for (int64_t v = v0 + threadIdx.x; v < v1; v += (int64_t)blockDim.x * kU) {
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t w = v + (int64_t)u * blockDim.x;
        if (w < v1) {
          float f[8];
          load_f32x8(src + w * 8, f);
          uint4 o;
          f32x8_to_bf16(f, o);
          inbox[w] = o;
        }
      }
    }
  }
}

// Reduce this rank's slice from its local inbox: out[j] = scale * sum_q inbox[q][v].
__device__ __forceinline__ void reduce_inbox(const ArArgs& a, int64_t slice_vecs, int64_t w, float* acc) {
  const uint4* inbox = reinterpret_cast<const uint4*>(a.peers.base[a.rank] + a.send_off);
  uint4 in[kMaxWorld];
#pragma unroll
  for (int q = 0; q < kMaxWorld; ++q)
    if (q < a.world) in[q] = __ldcg(inbox + (int64_t)q * slice_vecs + w);
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
  for (int q = 0; q < kMaxWorld; ++q)
    if (q < a.world) bf16x8_add(in[q], acc);
#pragma unroll
  for (int j = 0; j < 8; ++j) acc[j] *= a.scale;
}

// Two-shot all-reduce by pushes: (1) push bf16 slices to their owners' inboxes,
// (2) each owner reduces its slice locally and pushes the bf16 result into
// every rank's outbox, (3) every rank unpacks its outbox into fp32. All NVLink
// traffic is writes: 2(N-1)/N of the bf16 buffer per rank.
__global__ void __launch_bounds__(512) ar_twoshot_kernel(ArArgs a) {
  const int64_t slice_vecs = a.n / 8 / a.world;
  const int64_t per_cta = (slice_vecs + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = (int64_t)blockIdx.x * per_cta;
  const int64_t v1 = v0 + per_cta < slice_vecs ? v0 + per_cta : slice_vecs;

  push_slices(a, slice_vecs, v0, v1);
  if (!cta_barrier(a.peers, a.rank, a.world, a.flag_off, a.slot, 2u * a.epoch + 1u, a.timeout_ns, a.status, 1)) return;

  for (int64_t v = v0 + threadIdx.x; v < v1; v += (int64_t)blockDim.x * kU) {
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t w = v + (int64_t)u * blockDim.x;
      if (w < v1) {
        float acc[8];
        reduce_inbox(a, slice_vecs, w, acc);
        uint4 o;
        f32x8_to_bf16(acc, o);
#pragma unroll
        for (int q = 0; q < kMaxWorld; ++q)
          if (q < a.world)
            reinterpret_cast<uint4*>(a.peers.base[q] + a.recv_off)[(int64_t)a.rank * slice_vecs + w] = o;
      }
    }
  }
  if (!cta_barrier(a.peers, a.rank, a.world, a.flag_off, a.slot, 2u * a.epoch + 2u, a.timeout_ns, a.status, 2)) return;

  const uint4* outbox = reinterpret_cast<const uint4*>(a.peers.base[a.rank] + a.recv_off);
  for (int s = 0; s < a.world; ++s) {
    for (int64_t v = v0 + threadIdx.x; v < v1; v += (int64_t)blockDim.x * kU) {
#pragma unroll
      for (int u = 0; u < kU; ++u) {
        const int64_t w = v + (int64_t)u * blockDim.x;
        if (w < v1) {
          const int64_t idx = (int64_t)s * slice_vecs + w;
          float f[8];
#pragma unroll
          for (int j = 0; j < 8; ++j) f[j] = 0.f;
          bf16x8_add(__ldcg(outbox + idx), f);
          store_f32x8(a.dst + idx * 8, f, false);
        }
      }
    }
  }
}

// Chunk-pipelined two-shot all-reduce. Each CTA walks its slice range in chunks of `chunk`
// vectors; per chunk k: (A) push the bf16 cast of chunk k of every slice into its owner's inbox
// and post progress k+1 on slot_a; (B) once every peer posted chunk k on slot_a, reduce this
// rank's slice chunk k, push the scaled bf16 result into every rank's outbox and post on slot_b;
// (C) once every owner posted chunk k on slot_b, unpack chunk k of every slice into fp32. The loop
// issues A(k), B(k-1), C(k-2) in one iteration, so a chunk's push, reduce and unpack overlap the
// neighbouring chunks' and no CTA waits for the whole range of any phase. Progress values are
// epoch * 4096 + chunks done (monotonic across launches, compared wrap-safe). Reuse across
// launches is safe: a peer's next launch can only start after its unpack waited for this rank's
// last reduce, and its reduce waits for this rank's pushes of the new launch.
__device__ __forceinline__ void post_progress(const ArArgs& a, int slot, uint32_t value) {
  __syncthreads();
  if ((int)threadIdx.x < a.world) {
    __threadfence_system();
    st_release_sys(flag_ptr(a.peers.base[threadIdx.x], a.flag_off, slot, blockIdx.x, a.rank), value);
  }
}

__device__ __forceinline__ bool wait_progress(const ArArgs& a, int slot, uint32_t value, uint32_t where) {
  __shared__ int s_ok;
  if (threadIdx.x == 0) s_ok = 1;
  __syncthreads();
  if ((int)threadIdx.x < a.world) {
    const int q = threadIdx.x;
    if (!wait_flag_geq(flag_ptr(a.peers.base[a.rank], a.flag_off, slot, blockIdx.x, q), value, a.timeout_ns)) {
      set_status(a.status, kTimeoutBarrier, where | ((uint32_t)q << 16));
      s_ok = 0;
    }
  }
  __syncthreads();
  return s_ok != 0;
}

__global__ void __launch_bounds__(512, 2) ar_pipe_kernel(ArArgs a, int slot_b, int64_t chunk) {
  const int64_t slice_vecs = a.n / 8 / a.world;
  const int64_t per_cta = (slice_vecs + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = (int64_t)blockIdx.x * per_cta;
  const int64_t v1 = v0 + per_cta < slice_vecs ? v0 + per_cta : slice_vecs;
  const int nchunks = v1 > v0 ? (int)((v1 - v0 + chunk - 1) / chunk) : 0;
  const uint32_t base = a.epoch * 4096u;
  const uint4* outbox = reinterpret_cast<const uint4*>(a.peers.base[a.rank] + a.recv_off);
  for (int k = 0; k < nchunks + 2; ++k) {
    if (k < nchunks) {                                   // (A) push chunk k
      const int64_t c0 = v0 + (int64_t)k * chunk;
      const int64_t c1 = c0 + chunk < v1 ? c0 + chunk : v1;
      push_slices(a, slice_vecs, c0, c1);
      post_progress(a, a.slot, base + (uint32_t)k + 1u);
    }
    if (k >= 1 && k - 1 < nchunks) {                     // (B) reduce chunk k-1 and push the result
      const int kk = k - 1;
      if (!wait_progress(a, a.slot, base + (uint32_t)kk + 1u, 31)) return;
      const int64_t c0 = v0 + (int64_t)kk * chunk;
      const int64_t c1 = c0 + chunk < v1 ? c0 + chunk : v1;
      for (int64_t v = c0 + threadIdx.x; v < c1; v += (int64_t)blockDim.x * kU) {
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int64_t w = v + (int64_t)u * blockDim.x;
          if (w < c1) {
            float acc[8];
            reduce_inbox(a, slice_vecs, w, acc);
            uint4 o;
            f32x8_to_bf16(acc, o);
#pragma unroll
            for (int q = 0; q < kMaxWorld; ++q)
              if (q < a.world)
                reinterpret_cast<uint4*>(a.peers.base[q] + a.recv_off)[(int64_t)a.rank * slice_vecs + w] = o;
          }
        }
      }
      post_progress(a, slot_b, base + (uint32_t)kk + 1u);
    }
    if (k >= 2) {                                        // (C) unpack chunk k-2
      const int kk = k - 2;
      if (!wait_progress(a, slot_b, base + (uint32_t)kk + 1u, 32)) return;
      const int64_t c0 = v0 + (int64_t)kk * chunk;
      const int64_t c1 = c0 + chunk < v1 ? c0 + chunk : v1;
      for (int s = 0; s < a.world; ++s) {
        for (int64_t v = c0 + threadIdx.x; v < c1; v += (int64_t)blockDim.x * kU) {
#pragma unroll
          for (int u = 0; u < kU; ++u) {
            const int64_t w = v + (int64_t)u * blockDim.x;
            if (w < c1) {
              const int64_t idx = (int64_t)s * slice_vecs + w;
              float f[8];
#pragma unroll
              for (int j = 0; j < 8; ++j) f[j] = 0.f;
              bf16x8_add(__ldcg(outbox + idx), f);
              store_f32x8(a.dst + idx * 8, f, false);
            }
          }
        }
      }
    }
  }
}

// One-shot all-reduce for small buffers (latency-bound): every rank pushes its
// whole bf16 buffer into every peer's inbox [parity][rank], one barrier, then
// each rank sums the inboxes locally. Inboxes alternate by epoch parity, so a
// launch never overwrites an inbox a peer may still be reading.
__global__ void __launch_bounds__(512) ar_oneshot_kernel(ArArgs a, int64_t cap_vecs) {
  const int64_t nvec = a.n / 8;
  const int64_t per_cta = (nvec + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = (int64_t)blockIdx.x * per_cta;
  const int64_t v1 = v0 + per_cta < nvec ? v0 + per_cta : nvec;
  const int64_t par = (int64_t)(a.epoch & 1u) * a.world * cap_vecs;
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    float f[8];
    load_f32x8(a.src + v * 8, f);
    uint4 o;
    f32x8_to_bf16(f, o);
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < a.world) reinterpret_cast<uint4*>(a.peers.base[q] + a.send_off)[par + (int64_t)a.rank * cap_vecs + v] = o;
  }
  if (!cta_barrier(a.peers, a.rank, a.world, a.flag_off, a.slot, a.epoch, a.timeout_ns, a.status, 10)) return;
  const uint4* inbox = reinterpret_cast<const uint4*>(a.peers.base[a.rank] + a.send_off) + par;
  for (int64_t v = v0 + threadIdx.x; v < v1; v += blockDim.x) {
    float acc[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] = 0.f;
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < a.world) bf16x8_add(__ldcg(inbox + (int64_t)q * cap_vecs + v), acc);
#pragma unroll
    for (int j = 0; j < 8; ++j) acc[j] *= a.scale;
    store_f32x8(a.dst + v * 8, acc, false);
  }
}

// Deterministic block sum of `v` added into *out by the last CTA to finish (fixed CTA order);
// partials [gridDim], ticket zeroed before the first launch and re-zeroed by the last CTA.
__device__ void grid_sum_into(float v, float* partials, uint32_t* ticket, float* out) {
  __shared__ float red[32];
  __shared__ uint32_t s_t;
  v = warp_sum(v);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
  __syncthreads();
  if (threadIdx.x < 32) {
    float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
    t = warp_sum(t);
    if (threadIdx.x == 0) {
      partials[blockIdx.x] = t;
      __threadfence();
      s_t = atomicAdd(ticket, 1u);
    }
  }
  __syncthreads();
  if (s_t == gridDim.x - 1 && threadIdx.x == 0) {
    __threadfence();
    float tot = 0.f;
    for (unsigned b = 0; b < gridDim.x; ++b) tot += __ldcg(partials + b);
    *out += tot;
    *ticket = 0u;
  }
}

// Reduce-scatter by pushes, taking the local fp32 gradient directly (the bf16
// cast is fused): push slices, one barrier, reduce the local inbox into the
// fp32 shard (overwrite or accumulate), a trailing barrier so the inbox may be
// reused by the next launch. With sumsq_out, the shard's sum of squares (of the
// reduced, scaled values) is added into *sumsq_out: the first phase of the
// global gradient-norm clip, so the optimizer needs no separate pass.
__global__ void __launch_bounds__(512) rs_push_kernel(ArArgs a, int accumulate, float* sumsq_partials,
                                                      uint32_t* ticket, float* sumsq_out) {
  const int64_t slice_vecs = a.n / 8 / a.world;
  const int64_t per_cta = (slice_vecs + gridDim.x - 1) / gridDim.x;
  const int64_t v0 = (int64_t)blockIdx.x * per_cta;
  const int64_t v1 = v0 + per_cta < slice_vecs ? v0 + per_cta : slice_vecs;
  push_slices(a, slice_vecs, v0, v1);
  if (!cta_barrier(a.peers, a.rank, a.world, a.flag_off, a.slot, 2u * a.epoch + 1u, a.timeout_ns, a.status, 11)) return;
  float ss = 0.f;
  for (int64_t v = v0 + threadIdx.x; v < v1; v += (int64_t)blockDim.x * kU) {
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int64_t w = v + (int64_t)u * blockDim.x;
      if (w < v1) {
        float acc[8];
        reduce_inbox(a, slice_vecs, w, acc);
#pragma unroll
        for (int j = 0; j < 8; ++j) ss += acc[j] * acc[j];
        store_f32x8(a.dst + w * 8, acc, accumulate != 0);
      }
    }
  }
  if (sumsq_out) grid_sum_into(ss, sumsq_partials, ticket, sumsq_out);
  cta_barrier(a.peers, a.rank, a.world, a.flag_off, a.slot, 2u * a.epoch + 2u, a.timeout_ns, a.status, 12);
}

// ---------------------------------------------------------------------------
// FSDP reduce-scatter (+ fused AdamW)
// ---------------------------------------------------------------------------
struct RsArgs {
  Peers peers;
  int64_t shard;             // elements per rank (multiple of 8)
  int64_t send_off;          // byte offset of the unit's full bf16 gradient [world * shard]
  int64_t flag_off;
  int rank, world, slot;
  float scale;
  uint32_t epoch;
  uint64_t timeout_ns;
  uint32_t* status;
  // reduce-scatter output
  float* out;                // fp32 shard gradient (nullable in the AdamW variant)
  float* sumsq_partials;     // [gridDim] (nullable)
  uint32_t* ticket;          // zeroed ticket for the last-CTA sum (nullable)
  float* sumsq_out;          // accumulated norm^2 (nullable)
  // AdamW (nfb_rs_adamw only)
  float* param; float* m; float* v;
  int64_t param_off;         // byte offset of this rank's bf16 parameter shard in its symmetric buffer (-1: none)
  float lr, beta1, beta2, eps, wd, bc1, bc2_sqrt, clip;
  int trailing_barrier;
  int accumulate;            // nfb_rs_f32: out += reduced instead of out = reduced
};

template <bool ADAM>
__global__ void __launch_bounds__(512) rs_kernel(RsArgs a) {
  __shared__ float red[32];
  __shared__ uint32_t s_t;
  if (!cta_barrier(a.peers, a.rank, a.world, a.flag_off, a.slot, 2u * a.epoch + 1u, a.timeout_ns, a.status, 3)) return;
  const int64_t nvec = a.shard / 8;
  const int64_t base = (int64_t)a.rank * nvec;
  float ss = 0.f;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += (int64_t)gridDim.x * blockDim.x) {
    uint4 in[kMaxWorld];
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < a.world) in[q] = __ldcg(reinterpret_cast<const uint4*>(a.peers.base[q] + a.send_off) + base + v);
    float g[8];
#pragma unroll
    for (int j = 0; j < 8; ++j) g[j] = 0.f;
#pragma unroll
    for (int q = 0; q < kMaxWorld; ++q)
      if (q < a.world) bf16x8_add(in[q], g);
#pragma unroll
    for (int j = 0; j < 8; ++j) { g[j] *= a.scale; ss += g[j] * g[j]; }
    if (!ADAM) {
      float4* d = reinterpret_cast<float4*>(a.out + v * 8);
      if (a.accumulate) {
        float4 o0 = d[0], o1 = d[1];
        d[0] = make_float4(o0.x + g[0], o0.y + g[1], o0.z + g[2], o0.w + g[3]);
        d[1] = make_float4(o1.x + g[4], o1.y + g[5], o1.z + g[6], o1.w + g[7]);
      } else {
        d[0] = make_float4(g[0], g[1], g[2], g[3]);
        d[1] = make_float4(g[4], g[5], g[6], g[7]);
      }
    } else {
      float p[8], m[8], w[8];
      float4* pp = reinterpret_cast<float4*>(a.param + v * 8);
      float4* mp = reinterpret_cast<float4*>(a.m + v * 8);
      float4* vp = reinterpret_cast<float4*>(a.v + v * 8);
      float4 t0 = pp[0], t1 = pp[1];
      p[0] = t0.x; p[1] = t0.y; p[2] = t0.z; p[3] = t0.w; p[4] = t1.x; p[5] = t1.y; p[6] = t1.z; p[7] = t1.w;
      t0 = mp[0]; t1 = mp[1];
      m[0] = t0.x; m[1] = t0.y; m[2] = t0.z; m[3] = t0.w; m[4] = t1.x; m[5] = t1.y; m[6] = t1.z; m[7] = t1.w;
      t0 = vp[0]; t1 = vp[1];
      w[0] = t0.x; w[1] = t0.y; w[2] = t0.z; w[3] = t0.w; w[4] = t1.x; w[5] = t1.y; w[6] = t1.z; w[7] = t1.w;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const float gj = g[j] * a.clip;
        p[j] = p[j] * (1.f - a.lr * a.wd);
        m[j] = a.beta1 * m[j] + (1.f - a.beta1) * gj;
        w[j] = a.beta2 * w[j] + (1.f - a.beta2) * gj * gj;
        p[j] = p[j] - (a.lr / a.bc1) * (m[j] / (sqrtf(w[j]) / a.bc2_sqrt + a.eps));
      }
      pp[0] = make_float4(p[0], p[1], p[2], p[3]); pp[1] = make_float4(p[4], p[5], p[6], p[7]);
      mp[0] = make_float4(m[0], m[1], m[2], m[3]); mp[1] = make_float4(m[4], m[5], m[6], m[7]);
      vp[0] = make_float4(w[0], w[1], w[2], w[3]); vp[1] = make_float4(w[4], w[5], w[6], w[7]);
      if (a.param_off >= 0) {
        uint4 u;
        f32x8_to_bf16(p, u);
        reinterpret_cast<uint4*>(a.peers.base[a.rank] + a.param_off)[v] = u;
      }
    }
  }
  if (a.sumsq_partials) {
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    if (threadIdx.x < 32) {
      float t = threadIdx.x < (blockDim.x >> 5) ? red[threadIdx.x] : 0.f;
      t = warp_sum(t);
      if (threadIdx.x == 0) {
        a.sumsq_partials[blockIdx.x] = t;
        __threadfence();
        s_t = atomicAdd(a.ticket, 1u);
      }
    }
    __syncthreads();
    if (s_t == gridDim.x - 1 && threadIdx.x == 0) {
      __threadfence();
      float tot = 0.f;
      for (unsigned b = 0; b < gridDim.x; ++b) tot += __ldcg(a.sumsq_partials + b);
      *a.sumsq_out += tot;
      *a.ticket = 0u;
    }
  }
  if (a.trailing_barrier)
    cta_barrier(a.peers, a.rank, a.world, a.flag_off, a.slot, 2u * a.epoch + 2u, a.timeout_ns, a.status, 4);
}

// ---------------------------------------------------------------------------
// All-gather (pull) and scalar all-reduce
// ---------------------------------------------------------------------------
struct AgArgs {
  Peers peers;
  int64_t shard;        // elements per rank (bf16, multiple of 8)
  int64_t shard_off;    // byte offset of each rank's shard in its symmetric buffer
  void* out;            // local [world * shard] bf16
  int64_t flag_off;
  int rank, world, slot;
  uint32_t epoch;
  uint64_t timeout_ns;
  uint32_t* status;
};

__global__ void __launch_bounds__(512) allgather_kernel(AgArgs a) {
  if (!cta_barrier(a.peers, a.rank, a.world, a.flag_off, a.slot, 2u * a.epoch + 1u, a.timeout_ns, a.status, 5)) return;
  const int64_t nvec = a.shard / 8;
  for (int64_t v = (int64_t)blockIdx.x * blockDim.x + threadIdx.x; v < nvec; v += (int64_t)gridDim.x * blockDim.x) {
    uint4 in[kMaxWorld];
#pragma unroll
    for (int i = 0; i < kMaxWorld; ++i) {
      const int q = (a.rank + i) % a.world;  // start with the local shard
      if (i < a.world) in[i] = __ldcg(reinterpret_cast<const uint4*>(a.peers.base[q] + a.shard_off) + v);
    }
#pragma unroll
    for (int i = 0; i < kMaxWorld; ++i) {
      const int q = (a.rank + i) % a.world;
      if (i < a.world) reinterpret_cast<uint4*>(a.out)[q * nvec + v] = in[i];
    }
  }
  // Peers may overwrite their shard (next optimizer step) only after every
  // rank has finished reading it.
  cta_barrier(a.peers, a.rank, a.world, a.flag_off, a.slot, 2u * a.epoch + 2u, a.timeout_ns, a.status, 6);
}

struct ScalarArgs {
  Peers peers;
  int64_t val_off;      // byte offset of a float[kMaxWorld] exchange area
  float* inout;         // local scalar (device)
  int64_t flag_off;
  int rank, world, slot;
  uint32_t epoch;
  uint64_t timeout_ns;
  uint32_t* status;
};

__global__ void allreduce_scalar_kernel(ScalarArgs a) {
  // write my value into every peer's exchange slot [rank]
  if ((int)threadIdx.x < a.world) {
    float* dst = reinterpret_cast<float*>(a.peers.base[threadIdx.x] + a.val_off) + a.rank;
    *dst = *a.inout;
  }
  if (!cta_barrier(a.peers, a.rank, a.world, a.flag_off, a.slot, 2u * a.epoch + 1u, a.timeout_ns, a.status, 7)) return;
  if (threadIdx.x == 0) {
    const float* src = reinterpret_cast<const float*>(a.peers.base[a.rank] + a.val_off);
    float s = 0.f;
    for (int q = 0; q < a.world; ++q) s += __ldcg(src + q);
    *a.inout = s;
  }
  cta_barrier(a.peers, a.rank, a.world, a.flag_off, a.slot, 2u * a.epoch + 2u, a.timeout_ns, a.status, 8);
}

// Bounded wait on one flag; used by the failure-detection tests (a flag that
// nothing sets must make the kernel give up, report, and return).
__global__ void wait_flag_kernel(const uint32_t* flag, uint32_t target, uint64_t timeout_ns, uint32_t* status) {
  if (threadIdx.x == 0 && !wait_flag_geq(flag, target, timeout_ns)) set_status(status, kTimeoutFlag, 9);
}

static Peers make_peers(const uint64_t* bases, int world) {
  Peers p;
  for (int i = 0; i < kMaxWorld; ++i) p.base[i] = i < world ? bases[i] : 0;
  return p;
}

}  // namespace nfb

using namespace nfb;

NFB_API int nfb_comm_flag_bytes() { return kSlots * kMaxCtas * kMaxWorld * 4; }

NFB_API int nfb_ar_twoshot(const uint64_t* bases, int rank, int world, const float* src, float* dst, int64_t n,
                           int64_t send_off, int64_t recv_off, int64_t flag_off, int slot, float scale,
                           uint32_t epoch, uint64_t timeout_ns, uint32_t* status, int ctas, void* stream) {
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || slot < 0 || slot >= kSlots) return (int)cudaErrorInvalidValue;
  if (n % (8 * world) || ctas < 1 || ctas > kMaxCtas) return (int)cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) return (int)cudaErrorInvalidValue;
  if (n == 0) return 0;
  ArArgs a;
  a.peers = make_peers(bases, world);
  a.src = src; a.dst = dst; a.n = n; a.send_off = send_off; a.recv_off = recv_off; a.flag_off = flag_off;
  a.rank = rank; a.world = world; a.slot = slot; a.scale = scale; a.epoch = epoch; a.timeout_ns = timeout_ns;
  a.status = status;
  ar_twoshot_kernel<<<ctas, 512, 0, (cudaStream_t)stream>>>(a);
  return (int)cudaGetLastError();
}

// Chunk-pipelined two-shot all-reduce (same buffers and result as nfb_ar_twoshot); progress flags
// on slot (pushes) and slot_b (reduced results); chunk = vectors of 8 elements per slice per step.
NFB_API int nfb_ar_pipelined(const uint64_t* bases, int rank, int world, const float* src, float* dst, int64_t n,
                             int64_t send_off, int64_t recv_off, int64_t flag_off, int slot, int slot_b, float scale,
                             uint32_t epoch, uint64_t timeout_ns, uint32_t* status, int64_t chunk, int ctas,
                             void* stream) {
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || slot < 0 || slot >= kSlots || slot_b < 0 ||
      slot_b >= kSlots || slot_b == slot)
    return (int)cudaErrorInvalidValue;
  if (n % (8 * world) || ctas < 1 || ctas > kMaxCtas || chunk < 1) return (int)cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) return (int)cudaErrorInvalidValue;
  if (n == 0) return 0;
  const int64_t slice_vecs = n / 8 / world;
  const int64_t per_cta = (slice_vecs + ctas - 1) / ctas;
  if ((per_cta + chunk - 1) / chunk >= 4096) return (int)cudaErrorInvalidValue;   // progress counter range
  ArArgs a;
  a.peers = make_peers(bases, world);
  a.src = src; a.dst = dst; a.n = n; a.send_off = send_off; a.recv_off = recv_off; a.flag_off = flag_off;
  a.rank = rank; a.world = world; a.slot = slot; a.scale = scale; a.epoch = epoch; a.timeout_ns = timeout_ns;
  a.status = status;
  ar_pipe_kernel<<<ctas, 512, 0, (cudaStream_t)stream>>>(a, slot_b, chunk);
  return (int)cudaGetLastError();
}

// Small-buffer all-reduce; box_off: region of 2 * world * cap_elems bf16 on every rank.
NFB_API int nfb_ar_oneshot(const uint64_t* bases, int rank, int world, const float* src, float* dst, int64_t n,
                           int64_t box_off, int64_t cap_elems, int64_t flag_off, int slot, float scale,
                           uint32_t epoch, uint64_t timeout_ns, uint32_t* status, int ctas, void* stream) {
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || slot < 0 || slot >= kSlots) return (int)cudaErrorInvalidValue;
  if (n % 8 || n > cap_elems || cap_elems % 8 || ctas < 1 || ctas > kMaxCtas) return (int)cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(dst)) & 15) return (int)cudaErrorInvalidValue;
  if (n == 0) return 0;
  ArArgs a;
  a.peers = make_peers(bases, world);
  a.src = src; a.dst = dst; a.n = n; a.send_off = box_off; a.recv_off = 0; a.flag_off = flag_off;
  a.rank = rank; a.world = world; a.slot = slot; a.scale = scale; a.epoch = epoch; a.timeout_ns = timeout_ns;
  a.status = status;
  ar_oneshot_kernel<<<ctas, 512, 0, (cudaStream_t)stream>>>(a, cap_elems / 8);
  return (int)cudaGetLastError();
}

// Reduce-scatter of a local fp32 [n] buffer (bf16 on the wire) into this rank's fp32 shard [n / world];
// inbox_off: region of n bf16 on every rank.
NFB_API int nfb_rs_push(const uint64_t* bases, int rank, int world, const float* src, int64_t n, int64_t inbox_off,
                        int64_t flag_off, int slot, float scale, uint32_t epoch, uint64_t timeout_ns, uint32_t* status,
                        float* out, int accumulate, int ctas, void* stream) {
  return nfb_rs_push_sumsq(bases, rank, world, src, n, inbox_off, flag_off, slot, scale, epoch, timeout_ns, status,
                           out, accumulate, nullptr, nullptr, nullptr, ctas, stream);
}

// nfb_rs_push that also adds the shard's sum of squares into *sumsq_out (overwrite mode only):
// sumsq_partials [>= ctas] fp32, ticket a zeroed uint32 (left zeroed).
NFB_API int nfb_rs_push_sumsq(const uint64_t* bases, int rank, int world, const float* src, int64_t n,
                              int64_t inbox_off, int64_t flag_off, int slot, float scale, uint32_t epoch,
                              uint64_t timeout_ns, uint32_t* status, float* out, int accumulate,
                              float* sumsq_partials, uint32_t* ticket, float* sumsq_out, int ctas, void* stream) {
  if (sumsq_out && (accumulate || !sumsq_partials || !ticket)) return (int)cudaErrorInvalidValue;
  if (world < 1 || world > kMaxWorld || rank < 0 || rank >= world || slot < 0 || slot >= kSlots) return (int)cudaErrorInvalidValue;
  if (n % (8 * world) || ctas < 1 || ctas > kMaxCtas) return (int)cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(src) | reinterpret_cast<uintptr_t>(out)) & 15) return (int)cudaErrorInvalidValue;
  if (n == 0) return 0;
  ArArgs a;
  a.peers = make_peers(bases, world);
  a.src = src; a.dst = out; a.n = n; a.send_off = inbox_off; a.recv_off = 0; a.flag_off = flag_off;
  a.rank = rank; a.world = world; a.slot = slot; a.scale = scale; a.epoch = epoch; a.timeout_ns = timeout_ns;
  a.status = status;
  rs_push_kernel<<<ctas, 512, 0, (cudaStream_t)stream>>>(a, accumulate, sumsq_partials, ticket, sumsq_out);
  return (int)cudaGetLastError();
}

NFB_API int nfb_rs_f32(const uint64_t* bases, int rank, int world, int64_t shard, int64_t send_off, int64_t flag_off,
                       int slot, float scale, uint32_t epoch, uint64_t timeout_ns, uint32_t* status, float* out,
                       float* sumsq_partials, uint32_t* ticket, float* sumsq_out, int trailing_barrier,
                       int accumulate, int ctas, void* stream) {
  if (world < 1 || world > kMaxWorld || shard % 8 || ctas < 1 || ctas > kMaxCtas) return (int)cudaErrorInvalidValue;
  RsArgs a{};
  a.peers = make_peers(bases, world);
  a.shard = shard; a.send_off = send_off; a.flag_off = flag_off; a.rank = rank; a.world = world; a.slot = slot;
  a.scale = scale; a.epoch = epoch; a.timeout_ns = timeout_ns; a.status = status; a.out = out;
  a.sumsq_partials = sumsq_partials; a.ticket = ticket; a.sumsq_out = sumsq_out; a.param_off = -1;
  a.trailing_barrier = trailing_barrier; a.accumulate = accumulate;
  rs_kernel<false><<<ctas, 512, 0, (cudaStream_t)stream>>>(a);
  return (int)cudaGetLastError();
}

NFB_API int nfb_rs_adamw(const uint64_t* bases, int rank, int world, int64_t shard, int64_t send_off, int64_t flag_off,
                         int slot, float scale, uint32_t epoch, uint64_t timeout_ns, uint32_t* status,
                         float* param, float* m, float* v, int64_t param_off, float lr, float beta1, float beta2,
                         float eps, float wd, int64_t step, float clip, int trailing_barrier, int ctas, void* stream) {
  if (world < 1 || world > kMaxWorld || shard % 8 || ctas < 1 || ctas > kMaxCtas) return (int)cudaErrorInvalidValue;
  RsArgs a{};
  a.peers = make_peers(bases, world);
  a.shard = shard; a.send_off = send_off; a.flag_off = flag_off; a.rank = rank; a.world = world; a.slot = slot;
  a.scale = scale; a.epoch = epoch; a.timeout_ns = timeout_ns; a.status = status;
  a.param = param; a.m = m; a.v = v; a.param_off = param_off;
  a.lr = lr; a.beta1 = beta1; a.beta2 = beta2; a.eps = eps; a.wd = wd;
  a.bc1 = 1.f - powf(beta1, (float)step);
  a.bc2_sqrt = sqrtf(1.f - powf(beta2, (float)step));
  a.clip = clip; a.trailing_barrier = trailing_barrier;
  rs_kernel<true><<<ctas, 512, 0, (cudaStream_t)stream>>>(a);
  return (int)cudaGetLastError();
}

NFB_API int nfb_allgather(const uint64_t* bases, int rank, int world, int64_t shard, int64_t shard_off, void* out,
                          int64_t flag_off, int slot, uint32_t epoch, uint64_t timeout_ns, uint32_t* status, int ctas,
                          void* stream) {
  if (world < 1 || world > kMaxWorld || shard % 8 || ctas < 1 || ctas > kMaxCtas) return (int)cudaErrorInvalidValue;
  AgArgs a{};
  a.peers = make_peers(bases, world);
  a.shard = shard; a.shard_off = shard_off; a.out = out; a.flag_off = flag_off; a.rank = rank; a.world = world;
  a.slot = slot; a.epoch = epoch; a.timeout_ns = timeout_ns; a.status = status;
  allgather_kernel<<<ctas, 512, 0, (cudaStream_t)stream>>>(a);
  return (int)cudaGetLastError();
}

NFB_API int nfb_allreduce_scalar(const uint64_t* bases, int rank, int world, int64_t val_off, float* inout,
                                 int64_t flag_off, int slot, uint32_t epoch, uint64_t timeout_ns, uint32_t* status,
                                 void* stream) {
  if (world < 1 || world > kMaxWorld) return (int)cudaErrorInvalidValue;
  ScalarArgs a{};
  a.peers = make_peers(bases, world);
  a.val_off = val_off; a.inout = inout; a.flag_off = flag_off; a.rank = rank; a.world = world; a.slot = slot;
  a.epoch = epoch; a.timeout_ns = timeout_ns; a.status = status;
  allreduce_scalar_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(a);
  return (int)cudaGetLastError();
}

NFB_API int nfb_wait_flag(const uint32_t* flag, uint32_t target, uint64_t timeout_ns, uint32_t* status, void* stream) {
  wait_flag_kernel<<<1, 32, 0, (cudaStream_t)stream>>>(flag, target, timeout_ns, status);
  return (int)cudaGetLastError();
}
