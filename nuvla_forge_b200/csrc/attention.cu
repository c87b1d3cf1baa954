// Flash attention forward on the 5th-generation tensor cores (sm_100a).
//
//   O[b, q, h, :] = softmax(scale * Q[b, q, h, :] . K[b, :, g(h), :]^T) V[b, :, g(h), :]
//   g(h) = h / (Hq / Hkv)  (grouped-query attention), optional causal mask (kv <= q)
//
// Q, K, V and O are in the projection-native [B, S, H, D] layout (any token and
// batch strides, rows of D contiguous), D = 64 or 128, bf16; the kernel also
// writes the row log-sum-exp (natural log) [B, H, Sq] for the backward pass.
//
// One CTA per (128-query tile, head, batch); 6 warps with fixed roles:
//   warp 0      TMA producer: the Q tile once, then K and V tiles of 128 keys
//               into a two-stage ring (4-D tensor maps over [B, S, H, D]).
//   warp 1      MMA issuer (one elected lane): S_j = Q K_j^T into one of two
//               128-column TMEM buffers, then O += P_{j-1} V_{j-1} into a
//               D-column TMEM accumulator (P from shared memory, K-major; V
//               read MN-major straight from its TMA tile), so the tensor core
//               computes S_j while the softmax warps work on S_{j-1}.
//   warps 2-9   softmax: query row r (TMEM lane r) belongs to two threads, one
//               in warps 2-5 (key columns 0-63 of each tile, O columns
//               [0, D/2)) and one in warps 6-9 (the other halves). They read
//               their scores with tcgen05.ld, exchange the tile maximum through
//               shared memory, keep the running max / sums in registers (online
//               softmax in base 2, SFU exp2), rescale their part of the O row in
//               TMEM (tcgen05.ld/st) only when the max grows by more than 2^8,
//               and write their bf16 probabilities -- one 64-key block each --
//               into the 128-byte-swizzled P tile. At the end they normalise
//               their O columns and store them with the log-sum-exp.
// Every mbarrier wait is bounded by %globaltimer and reports a status; no
// cluster, no multicast. Parity: the reference calls
// F.scaled_dot_product_attention (nuvla_forge/model/dit.py:92).
#include "tc_gemm.cuh"
#include "tc_host.cuh"

namespace nfb {
namespace attn {

using namespace nfb::tc;

constexpr int BQ = 128;          // queries per CTA (TMEM lanes)
constexpr int BKV = 128;         // keys per tile
constexpr int kThreadsA = 320;        // producer, MMA, 8 softmax warps
constexpr uint32_t kTmemColsA = 512;   // S0 | S1 | O

struct AttnArgs {
  int B, Sq, Sk, Hq, Hkv, D;
  int causal;
  float scale_log2;             // softmax scale * log2(e)
  __nv_bfloat16* o;
  int64_t so_b, so_s, so_h;     // element strides of O
  float* lse;                   // [B, Hq, Sq] (nullable)
  uint32_t* status;
};

struct alignas(8) AttnShared {
  uint64_t q_full;
  uint64_t kv_full[2];
  uint64_t kv_empty[2];
  uint64_t s_full[2];
  uint64_t p_full;
  uint64_t pv_done;
  uint64_t o_full;
  uint64_t drain;
  uint32_t tmem_base;
  int abort;
};

__device__ __forceinline__ void tma_load_4d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1, int c2,
                                            int c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3, %4, %5}], [%6];"
      ::"r"(smem_u32(dst)), "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3),
        "r"(smem_u32(bar))
      : "memory");
}

__device__ __forceinline__ void tmem_st32(uint32_t taddr, const float* v) {
  asm volatile(
      "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
      "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
      "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};\n\t"
      "tcgen05.wait::st.sync.aligned;"
      ::"r"(taddr), "r"(__float_as_uint(v[0])), "r"(__float_as_uint(v[1])), "r"(__float_as_uint(v[2])),
        "r"(__float_as_uint(v[3])), "r"(__float_as_uint(v[4])), "r"(__float_as_uint(v[5])),
        "r"(__float_as_uint(v[6])), "r"(__float_as_uint(v[7])), "r"(__float_as_uint(v[8])),
        "r"(__float_as_uint(v[9])), "r"(__float_as_uint(v[10])), "r"(__float_as_uint(v[11])),
        "r"(__float_as_uint(v[12])), "r"(__float_as_uint(v[13])), "r"(__float_as_uint(v[14])),
        "r"(__float_as_uint(v[15])), "r"(__float_as_uint(v[16])), "r"(__float_as_uint(v[17])),
        "r"(__float_as_uint(v[18])), "r"(__float_as_uint(v[19])), "r"(__float_as_uint(v[20])),
        "r"(__float_as_uint(v[21])), "r"(__float_as_uint(v[22])), "r"(__float_as_uint(v[23])),
        "r"(__float_as_uint(v[24])), "r"(__float_as_uint(v[25])), "r"(__float_as_uint(v[26])),
        "r"(__float_as_uint(v[27])), "r"(__float_as_uint(v[28])), "r"(__float_as_uint(v[29])),
        "r"(__float_as_uint(v[30])), "r"(__float_as_uint(v[31]))
      : "memory");
}

// Named barrier over the 64 threads of one row pair that also ANDs a flag across them, so both
// warps of a pair always take the same branch (a warp that left alone would strand its partner).
__device__ __forceinline__ bool pair_all(int id, bool v) {
  int r;
  asm volatile(
      "{\n\t.reg .pred p, q;\n\t"
      "setp.ne.b32 p, %1, 0;\n\t"
      "bar.red.and.pred q, %2, 64, p;\n\t"
      "selp.b32 %0, 1, 0, q;\n\t}"
      : "=r"(r)
      : "r"((int)v), "r"(id)
      : "memory");
  return r != 0;
}

// 2^x with the SFU's approximate base-2 exponential (flushes denormal results to zero).
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

__device__ __forceinline__ uint32_t pack_bf16(float a, float b) {
  __nv_bfloat162 h = __floats2bfloat162_rn(a, b);
  return *reinterpret_cast<uint32_t*>(&h);
}

// Shared memory: [Q: D/64 x 16 KB][K: 2 stages x D/64 x 16 KB][V: 2 stages x 2 x D/64 x 8 KB][P: 2 x 16 KB][AttnShared]
template <int D>
struct Layout {
  static constexpr int kDB = D / 64;                        // 64-column blocks of the head dim
  static constexpr int kQBytes = BQ * D * 2;
  static constexpr int kKBytes = BKV * D * 2;
  static constexpr int kVBytes = BKV * D * 2;
  static constexpr int kPBytes = BQ * BKV * 2;
  static constexpr int kQ = 0;
  static constexpr int kK = kQ + kQBytes;
  static constexpr int kV = kK + 2 * kKBytes;
  static constexpr int kP = kV + 2 * kVBytes;
  static constexpr int kS = kP + kPBytes;
  // + AttnShared slot + alignment; at least 116 KB so that one CTA (and its 512 TMEM columns) owns an SM
  static constexpr size_t kRaw = (size_t)kS + 128 + 2048 + 1024;   // AttnShared, [2][2][128] fp32 exchange, alignment
  static constexpr size_t kBytes = kRaw > 116 * 1024 ? kRaw : 116 * 1024;
};

template <int D>
__global__ void __launch_bounds__(kThreadsA, 1)
    attn_fwd_kernel(const __grid_constant__ CUtensorMap tq, const __grid_constant__ CUtensorMap tk,
                    const __grid_constant__ CUtensorMap tv, AttnArgs a) {
  using L = Layout<D>;
  extern __shared__ __align__(1024) uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  AttnShared* S = reinterpret_cast<AttnShared*>(smem + L::kS);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  volatile int* abort_flag = &S->abort;
  const int q0 = blockIdx.x * BQ, h = blockIdx.y, b = blockIdx.z;
  const int hk = h / (a.Hq / a.Hkv);
  // key tiles this query tile needs
  int kv_end = a.Sk;
  if (a.causal) {
    const int lim = q0 + BQ + (a.Sk - a.Sq);   // keys kv <= q + (Sk - Sq)
    kv_end = lim < kv_end ? lim : kv_end;
  }
  const int n_kv = kv_end > 0 ? (kv_end + BKV - 1) / BKV : 0;

  if (threadIdx.x == 0) {
    mbar_init(&S->q_full, 1);
    for (int s = 0; s < 2; ++s) {
      mbar_init(&S->kv_full[s], 1);
      mbar_init(&S->kv_empty[s], 1);
      mbar_init(&S->s_full[s], 1);
    }
    mbar_init(&S->p_full, 256);
    mbar_init(&S->pv_done, 1);
    mbar_init(&S->o_full, 1);
    mbar_init(&S->drain, 1);
    S->abort = 0;
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
  }
  if (warp == 1) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                 ::"r"(smem_u32(&S->tmem_base)), "r"(kTmemColsA) : "memory");
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
  }
  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  const uint32_t tmem_base = S->tmem_base;

  if (warp == 0) {
    // ---------------- TMA producer ----------------
    if (lane == 0 && n_kv > 0) {
      prefetch_tmap(&tq);
      prefetch_tmap(&tk);
      prefetch_tmap(&tv);
      mbar_arrive_expect_tx(&S->q_full, L::kQBytes);
      for (int db = 0; db < L::kDB; ++db) tma_load_4d(smem + L::kQ + db * 16384, &tq, &S->q_full, db * 64, h, q0, b);
      int issued = 0;
      bool ok = true;
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j & 1;
        if (j >= 2 && !mbar_wait(&S->kv_empty[st], ((j >> 1) - 1) & 1, abort_flag)) { ok = false; break; }
        mbar_arrive_expect_tx(&S->kv_full[st], L::kKBytes + L::kVBytes);
        uint8_t* ks = smem + L::kK + st * L::kKBytes;
        uint8_t* vs = smem + L::kV + st * L::kVBytes;
        const int kv0 = j * BKV;
        for (int db = 0; db < L::kDB; ++db) tma_load_4d(ks + db * 16384, &tk, &S->kv_full[st], db * 64, hk, kv0, b);
        for (int kb = 0; kb < 2; ++kb)
          for (int db = 0; db < L::kDB; ++db)
            tma_load_4d(vs + (kb * L::kDB + db) * 8192, &tv, &S->kv_full[st], db * 64, hk, kv0 + kb * 64, b);
        ++issued;
      }
      if (!ok) {
        set_status(a.status, kTimeoutFlag, 120);
        S->abort = 1;
      }
      // the Q load and the last two K/V loads must land before the CTA exits (bounded)
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&S->q_full, 0u) && globaltimer_ns() - t0 < kWaitNs) {}
      for (int j = issued > 2 ? issued - 2 : 0; j < issued; ++j) {
        const uint64_t t1 = globaltimer_ns();
        while (!mbar_try_wait(&S->kv_full[j & 1], (j >> 1) & 1) && globaltimer_ns() - t1 < kWaitNs) {}
      }
    }
  } else if (warp == 1) {
    // ---------------- MMA issuer ----------------
    if (lane == 0 && n_kv > 0) {
      const uint32_t id_s = idesc_bf16(BQ, BKV, false, false);
      const uint32_t id_o = idesc_bf16(BQ, D, false, true);
      const uint32_t sq = smem_u32(smem + L::kQ);
      const uint32_t sp = smem_u32(smem + L::kP);
      const uint32_t t_o = tmem_base + 256;
      bool ok = mbar_wait(&S->q_full, 0u, abort_flag);
      auto issue_pv = [&](int jj) {
        const uint32_t sv = smem_u32(smem + L::kV + (jj & 1) * L::kVBytes);
#pragma unroll
        for (int kb = 0; kb < 2; ++kb)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(t_o, sw128_desc(sp + kb * 16384 + kk * 32),
                      sw128_mn_desc(sv + kb * L::kDB * 8192 + kk * 16 * 128), id_o,
                      (jj > 0 || kb > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&S->pv_done);
        umma_commit(&S->kv_empty[jj & 1]);
      };
      for (int j = 0; j < n_kv && ok; ++j) {
        const int st = j & 1;
        if (!mbar_wait(&S->kv_full[st], (j >> 1) & 1, abort_flag)) { ok = false; break; }
        tmem_fence_after();
        const uint32_t sk = smem_u32(smem + L::kK + st * L::kKBytes);
        const uint32_t t_s = tmem_base + (uint32_t)(st * BKV);
#pragma unroll
        for (int db = 0; db < L::kDB; ++db)
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16(t_s, sw128_desc(sq + db * 16384 + kk * 32), sw128_desc(sk + db * 16384 + kk * 32), id_s,
                      (db > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&S->s_full[st]);
        if (j >= 1) {
          if (!mbar_wait(&S->p_full, (j - 1) & 1, abort_flag)) { ok = false; break; }
          tmem_fence_after();
          issue_pv(j - 1);
        }
      }
      if (ok) {
        ok = mbar_wait(&S->p_full, (n_kv - 1) & 1, abort_flag);
        if (ok) {
          tmem_fence_after();
          issue_pv(n_kv - 1);
          umma_commit(&S->o_full);
        }
      }
      if (!ok) {
        set_status(a.status, kTimeoutFlag, 121);
        S->abort = 1;
      }
      umma_commit(&S->drain);
      const uint64_t t0 = globaltimer_ns();
      while (!mbar_try_wait(&S->drain, 0u) && globaltimer_ns() - t0 < kWaitNs) {}
    }
  } else {
    // ---------------- softmax + epilogue (warps 2..9) ----------------
    // Two warps share each TMEM lane quarter: warps 2-5 take key columns 0-63 of
    // every tile (and O columns [0, D/2)), warps 6-9 key columns 64-127 (and O
    // columns [D/2, D)). The two threads of a row exchange their tile maxima
    // through shared memory behind a 64-thread named barrier.
    const int quarter = warp & 3;
    const int half = (warp - 2) >> 2;
    const int r = quarter * 32 + lane;           // query row in the tile = TMEM lane
    const int q = q0 + r;
    const uint32_t lane_off = (uint32_t)(quarter * 32) << 16;
    const int bar_id = 1 + quarter;
    float* xmax = reinterpret_cast<float*>(smem + L::kS + 128);   // [2][128] partial maxima, then [2][128] sums
    uint8_t* prow = smem + L::kP + half * 16384 + (r >> 3) * 1024 + (r & 7) * 128;
    const int lim = a.causal ? q + (a.Sk - a.Sq) : a.Sk - 1;
    const int last = lim < a.Sk - 1 ? lim : a.Sk - 1;      // last key this row may see
    constexpr int HC = BKV / 2;                            // key columns per thread
    float m = -INFINITY, l = 0.f;                          // running max (log2 units), this half's sum
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int st = j & 1;
      // (this barrier also orders the previous tile's reads of the exchange buffer before its reuse)
      if (!pair_all(bar_id, mbar_wait(&S->s_full[st], (j >> 1) & 1, abort_flag))) { ok = false; break; }
      tmem_fence_after();
      float s[HC];
#pragma unroll
      for (int c = 0; c < HC; c += 32)
        tmem_ld32(tmem_base + lane_off + (uint32_t)(st * BKV + half * HC + c), s + c);
      const int kv0 = j * BKV + half * HC;
      if (kv0 + HC - 1 > last) {
#pragma unroll
        for (int c = 0; c < HC; ++c) s[c] = (kv0 + c <= last) ? s[c] : -INFINITY;
      }
      float mt = s[0];
#pragma unroll
      for (int c = 1; c < HC; ++c) mt = fmaxf(mt, s[c]);
      xmax[half * 128 + r] = mt;
      asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");
      mt = fmaxf(mt, xmax[(half ^ 1) * 128 + r]) * a.scale_log2;
      // lazy rescaling: keep the old reference max unless the new one exceeds it by more than 8 (2^8
      // headroom in fp32), so O is rescaled only on large jumps
      float m_ref = m, alpha = 1.f;
      if (mt > m + 8.f) {
        m_ref = mt;
        alpha = m == -INFINITY ? 0.f : ex2_approx(m - mt);
      }
      const float m_use = m_ref == -INFINITY ? 0.f : m_ref;
      float sum = 0.f;
#pragma unroll
      for (int c = 0; c < HC; ++c) {
        s[c] = ex2_approx(fmaf(s[c], a.scale_log2, -m_use));
        sum += s[c];
      }
      l = l * alpha + sum;
      m = m_ref;
      if (j >= 1) {
        // O may be rescaled (and P overwritten) only after the previous P V finished
        if (!pair_all(bar_id, mbar_wait(&S->pv_done, (j - 1) & 1, abort_flag))) { ok = false; break; }
        tmem_fence_after();
        if (__any_sync(0xffffffffu, alpha != 1.f)) {
#pragma unroll 1
          for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 32) {
            float o[32];
            tmem_ld32(tmem_base + lane_off + 256u + (uint32_t)c, o);
#pragma unroll
            for (int i = 0; i < 32; ++i) o[i] *= alpha;
            tmem_st32(tmem_base + lane_off + 256u + (uint32_t)c, o);
          }
        }
      }
      // this half's 64 bf16 probabilities = one 64-key block of the 128-byte-swizzled K-major P tile
#pragma unroll
      for (int c = 0; c < 8; ++c) {
        const float* p = s + c * 8;
        uint4 v;
        v.x = pack_bf16(p[0], p[1]);
        v.y = pack_bf16(p[2], p[3]);
        v.z = pack_bf16(p[4], p[5]);
        v.w = pack_bf16(p[6], p[7]);
        *reinterpret_cast<uint4*>(prow + ((c ^ (r & 7)) << 4)) = v;
      }
      asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
      tmem_fence_before();
      mbar_arrive(&S->p_full);
    }
    // the row's total sum: this half's plus the partner's
    float* xsum = xmax + 256;
    xsum[half * 128 + r] = l;
    asm volatile("bar.sync %0, 64;" ::"r"(bar_id) : "memory");
    const float l_row = l + xsum[(half ^ 1) * 128 + r];
    if (!ok) {
      if (lane == 0) {
        set_status(a.status, kTimeoutFlag, 122);
        S->abort = 1;
      }
    } else if (n_kv == 0) {
      // no key is visible to any row of this tile (causal with Sq > Sk): zero rows
      if (q < a.Sq) {
        __nv_bfloat16* orow = a.o + (int64_t)b * a.so_b + (int64_t)q * a.so_s + (int64_t)h * a.so_h;
        for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 8)
          *reinterpret_cast<uint4*>(orow + c) = make_uint4(0u, 0u, 0u, 0u);
        if (a.lse && half == 0) a.lse[((int64_t)b * a.Hq + h) * a.Sq + q] = -INFINITY;
      }
    } else {
      const bool w = mbar_wait(&S->o_full, 0u, abort_flag);
      if (__all_sync(0xffffffffu, w)) {
        tmem_fence_after();
        const float inv = l_row > 0.f ? 1.f / l_row : 0.f;
        __nv_bfloat16* orow = a.o + (int64_t)b * a.so_b + (int64_t)q * a.so_s + (int64_t)h * a.so_h;
#pragma unroll 1
        for (int c = half * (D / 2); c < (half + 1) * (D / 2); c += 32) {
          float o[32];
          tmem_ld32(tmem_base + lane_off + 256u + (uint32_t)c, o);
          if (q < a.Sq) {
#pragma unroll
            for (int i = 0; i < 32; i += 8) {
              uint4 v;
              v.x = pack_bf16(o[i] * inv, o[i + 1] * inv);
              v.y = pack_bf16(o[i + 2] * inv, o[i + 3] * inv);
              v.z = pack_bf16(o[i + 4] * inv, o[i + 5] * inv);
              v.w = pack_bf16(o[i + 6] * inv, o[i + 7] * inv);
              *reinterpret_cast<uint4*>(orow + c + i) = v;
            }
          }
        }
        if (q < a.Sq && a.lse && half == 0)
          a.lse[((int64_t)b * a.Hq + h) * a.Sq + q] =
              l_row > 0.f ? m * 0.69314718055994531f + logf(l_row) : -INFINITY;
      } else if (lane == 0) {
        set_status(a.status, kTimeoutFlag, 123);
        S->abort = 1;
      }
    }
  }

  tmem_fence_before();
  __syncthreads();
  tmem_fence_after();
  if (warp == 1) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem_base), "r"(kTmemColsA)
                 : "memory");
  }
}

// 4-D bf16 tensor map over [B, S, H, D] (dims innermost first: D, H, S, B) with a box of
// 64 head-dim columns x 1 head x box_rows tokens x 1 batch, 128-byte swizzle.
static int make_tmap_bshd(CUtensorMap* m, const void* base, int Bn, int Sn, int Hn, int Dn, int64_t sb, int64_t ss,
                          int64_t sh, int box_rows) {
  int rc = get_encode();
  if (rc) return rc;
  rc = bind_device_of(base);
  if (rc) return rc;
  if ((reinterpret_cast<uintptr_t>(base) & 15) || (sb * 2) % 16 || (ss * 2) % 16 || (sh * 2) % 16)
    return (int)cudaErrorInvalidValue;
  cuuint64_t dims[4] = {(cuuint64_t)Dn, (cuuint64_t)Hn, (cuuint64_t)Sn, (cuuint64_t)Bn};
  cuuint64_t strides[3] = {(cuuint64_t)(sh * 2), (cuuint64_t)(ss * 2), (cuuint64_t)(sb * 2)};
  cuuint32_t box[4] = {64, 1, (cuuint32_t)box_rows, 1};
  cuuint32_t estr[4] = {1, 1, 1, 1};
  CUresult r = g_encode(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 4, const_cast<void*>(base), dims, strides, box, estr,
                        CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  return r == CUDA_SUCCESS ? 0 : (int)cudaErrorInvalidValue;
}

template <int D>
static int launch_fwd(const CUtensorMap& tq, const CUtensorMap& tk, const CUtensorMap& tv, const AttnArgs& a,
                      cudaStream_t st) {
  const size_t smem = Layout<D>::kBytes;
  cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel<D>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
  if (e != cudaSuccess) return (int)e;
  dim3 grid((a.Sq + BQ - 1) / BQ, a.Hq, a.B);
  attn_fwd_kernel<D><<<grid, kThreadsA, smem, st>>>(tq, tk, tv, a);
  return (int)cudaGetLastError();
}

}  // namespace attn
}  // namespace nfb

using namespace nfb::attn;

// q [B, Sq, Hq, D], k / v [B, Sk, Hkv, D] (element strides per batch / token / head; D contiguous),
// o [B, Sq, Hq, D] bf16; lse [B, Hq, Sq] fp32 (nullable). D in {64, 128}; Hkv divides Hq.
NFB_API int nfb_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Sq, int Sk,
                         int Hq, int Hkv, int D, int64_t sq_b, int64_t sq_s, int64_t sq_h, int64_t sk_b, int64_t sk_s,
                         int64_t sk_h, int64_t sv_b, int64_t sv_s, int64_t sv_h, int64_t so_b, int64_t so_s,
                         int64_t so_h, int causal, float scale, uint32_t* status, void* stream) {
  if ((D != 64 && D != 128) || B < 1 || Sq < 1 || Sk < 1 || Hkv < 1 || Hq % Hkv) return (int)cudaErrorInvalidValue;
  if ((reinterpret_cast<uintptr_t>(o) & 15) || (so_s * 2) % 16 || (so_h * 2) % 16 || (so_b * 2) % 16)
    return (int)cudaErrorInvalidValue;
  CUtensorMap tq, tk, tv;
  int rc = make_tmap_bshd(&tq, q, B, Sq, Hq, D, sq_b, sq_s, sq_h, BQ);
  if (rc) return rc;
  rc = make_tmap_bshd(&tk, k, B, Sk, Hkv, D, sk_b, sk_s, sk_h, BKV);
  if (rc) return rc;
  rc = make_tmap_bshd(&tv, v, B, Sk, Hkv, D, sv_b, sv_s, sv_h, 64);
  if (rc) return rc;
  AttnArgs a;
  a.B = B; a.Sq = Sq; a.Sk = Sk; a.Hq = Hq; a.Hkv = Hkv; a.D = D; a.causal = causal;
  a.scale_log2 = scale * 1.4426950408889634f;
  a.o = reinterpret_cast<__nv_bfloat16*>(o);
  a.so_b = so_b; a.so_s = so_s; a.so_h = so_h;
  a.lse = lse;
  a.status = status;
  cudaStream_t st = (cudaStream_t)stream;
  return D == 64 ? launch_fwd<64>(tq, tk, tv, a, st) : launch_fwd<128>(tq, tk, tv, a, st);
}
