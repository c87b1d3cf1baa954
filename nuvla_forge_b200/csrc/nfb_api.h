/* C interface of libnfb200.so, the native library of nuvla_forge_b200 (sm_100a only).
 *
 * Every kernel entry point takes raw device pointers, sizes and strides in elements, and the
 * cudaStream_t to launch on (passed as void*); it returns a cudaError_t as int (0 = success).
 * Apart from nfb_ipc_alloc / nfb_ipc_free, no entry point allocates device memory: scratch and
 * status words are passed in by the caller. Status words are device uint32 values that a bounded
 * wait sets to (code << 24 | site) when it gives up (code 1: peer barrier, 2: flag or pipeline
 * wait, 3: bad argument); the caller reads them after the step.
 *
 * dtype codes: 0 = fp32, 1 = bf16, 2 = fp16.
 *
 * The library's own sources include this header, so the compiler checks every definition
 * against the declaration here.
 */
#ifndef NFB_API_H_
#define NFB_API_H_

#include <stdint.h>

#if defined(__GNUC__) || defined(__clang__)
#define NFB_EXPORT __attribute__((visibility("default")))
#else
#define NFB_EXPORT
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- device info ------------------------------------------------------------------------ */
NFB_EXPORT int nfb_num_sms(void);
NFB_EXPORT int nfb_device_synchronize(void);

/* ---- debug build (libnfb200_debug.so, compiled with -DNFB_DEBUG) ------------------------- */
/* Device-side bounds checks record the first failure as (4 << 24 | site) instead of faulting. */
NFB_EXPORT uint32_t nfb_debug_status(void);
NFB_EXPORT void nfb_debug_reset(void);
NFB_EXPORT int nfb_is_debug_build(void);

/* ---- gated residual + RMSNorm + adaLN modulate (norm.cu) -------------------------------- */
/* gate_mode: 0 no gate / residual, 1 residual add, 2 per-sample gate [B, N]; mod: 1 applies
 * (1 + scale) and shift per sample. T = tokens per sample. */
NFB_EXPORT int nfb_norm_fwd(int dtype, int gate_mode, int mod, const void* x, const void* y, const void* gate,
                            const void* weight, const void* scale, const void* shift, void* h, void* out,
                            float* rstd, int64_t M, int64_t N, int64_t T, int64_t sx, int64_t sy, int64_t sh,
                            int64_t so, int64_t sg, int64_t ss, int64_t ssh, float eps, int w_f32, void* stream);
NFB_EXPORT int64_t nfb_norm_bwd_P(int64_t M, int64_t N, int64_t B);
NFB_EXPORT int nfb_norm_bwd(int dtype, int gate_mode, int mod, const void* dh_up, const void* dout, const void* h,
                            const void* y, const void* gate, const void* weight, const void* scale,
                            const float* rstd, void* dx, void* dy, void* dgate, void* dscale, void* dshift,
                            void* dweight, float* partials, float* dwb, uint32_t* tickets, int64_t M, int64_t N,
                            int64_t T, int64_t P, int64_t s_dhup, int64_t s_dout, int64_t s_h, int64_t s_y,
                            int64_t s_dx, int64_t s_dy, int64_t sg, int64_t ss, int w_f32, void* stream);
NFB_EXPORT void nfb_norm_set_status(uint32_t* status);
NFB_EXPORT void nfb_norm_set_impl(int impl);
NFB_EXPORT int nfb_norm_get_impl(void);

/* Allocation-free variant of nfb_norm_bwd: same outputs, with its scratch in a fixed-size
 * device array inside the library (nfb_noalloc_scratch_floats() fp32 elements, at most 1023
 * samples). It exists for callers that may not allocate device memory while they run. Calls
 * that overlap on the GPU share the scratch and race. A rejected call returns
 * cudaErrorInvalidValue and nfb_noalloc_last_error() says why. It has no counterpart in the
 * reference implementation. */
NFB_EXPORT int nfb_norm_bwd_noalloc(int dtype, int gate_mode, int mod, const void* dh_up, const void* dout,
                                    const void* h, const void* y, const void* gate, const void* weight,
                                    const void* scale, const float* rstd, void* dx, void* dy, void* dgate,
                                    void* dscale, void* dshift, void* dweight, int64_t M, int64_t N, int64_t T,
                                    int64_t s_dhup, int64_t s_dout, int64_t s_h, int64_t s_y, int64_t s_dx,
                                    int64_t s_dy, int64_t sg, int64_t ss, int w_f32, void* stream);
NFB_EXPORT const char* nfb_noalloc_last_error(void);
NFB_EXPORT int64_t nfb_noalloc_scratch_floats(void);

/* ---- SwiGLU (swiglu.cu) ----------------------------------------------------------------- */
NFB_EXPORT int nfb_swiglu_fwd(int dtype, const void* a, const void* b, void* out, int64_t M, int64_t N, int64_t sa,
                              int64_t sb, int64_t so, void* stream);
NFB_EXPORT int nfb_swiglu_bwd(int dtype, const void* dout, const void* a, const void* b, void* da, void* db,
                              int64_t M, int64_t N, int64_t sdo, int64_t sa, int64_t sb, int64_t sda, int64_t sdb,
                              void* stream);

/* ---- images (image.cu) ------------------------------------------------------------------ */
NFB_EXPORT int nfb_image_normalize(int out_dtype, const void* in, void* out, int64_t n, int64_t hw,
                                   const float* mean, const float* std, void* stream);
NFB_EXPORT int nfb_image_patchify(int out_dtype, const void* in, void* out, int64_t n_img, int H, int W, int p,
                                  int kpad, const float* mean, const float* std, void* stream);

/* ---- optimizer and reductions (optim.cu) ------------------------------------------------ */
NFB_EXPORT int nfb_adamw_flat(float* param, const float* grad, float* m, float* v, void* param_bf16, int64_t n,
                              float lr, float beta1, float beta2, float eps, float wd, int64_t step,
                              float grad_scale, const float* norm2, float max_norm, void* stream);
NFB_EXPORT int nfb_sumsq_slots(void);
NFB_EXPORT int nfb_sumsq(int dtype, const void* x, int64_t n, float scale, float* partials, uint32_t* ticket,
                         float* out, int accumulate, void* stream);
NFB_EXPORT int nfb_accum(int src_dtype, float* dst, const void* src, int64_t n, float scale, int overwrite,
                         void* stream);
NFB_EXPORT int nfb_cast(int src_dtype, int dst_dtype, void* dst, const void* src, int64_t n, float scale,
                        void* stream);

/* ---- cross entropy (ce_rows.cu, ce_tc.cu) ----------------------------------------------- */
NFB_EXPORT int nfb_ce_rows(int dtype, void* logits, int64_t ld, const int64_t* targets, int64_t rows, int64_t V,
                           int64_t ignore_index, const float* count, float* loss_rows, void* stream);
NFB_EXPORT int nfb_count_valid(const int64_t* targets, int64_t n, int64_t ignore_index, float* out, void* stream);
NFB_EXPORT int nfb_ce_tc_tiles(int V);
NFB_EXPORT int nfb_ce_tc_stats(const void* hidden, int64_t ldh, const void* weight, int64_t ldw,
                               const int64_t* targets, int M, int V, int H, float* pmax, float* psum, float* tlogit,
                               uint32_t* status, void* stream);
NFB_EXPORT int nfb_ce_tc_merge(const float* pmax, const float* psum, const float* tlogit, const int64_t* targets,
                               const float* count, int M, int V, int64_t ignore_index, float* lse,
                               float* loss_rows, void* stream);
NFB_EXPORT int nfb_ce_tc_grad(const void* hidden, int64_t ldh, const void* weight, int64_t ldw,
                              const int64_t* targets, const float* lse, const float* count, int64_t ignore_index,
                              int M, int V, int H, void* dl, int64_t ldd, uint32_t* status, void* stream);

/* ---- single-CTA tcgen05 GEMM core (ce_tc.cu) -------------------------------------------- */
NFB_EXPORT int nfb_tc_gemm_ex(const void* A, const void* B, void* C, int M, int N, int K, int64_t lda, int64_t ldb,
                              int64_t ldc, int out_f32, int a_mn, int b_mn, int accumulate, uint32_t* status,
                              void* stream);
NFB_EXPORT int nfb_tc_gemm_bf16(const void* A, const void* B, void* C, int M, int N, int K, int64_t lda,
                                int64_t ldb, int64_t ldc, int out_f32, uint32_t* status, void* stream);

/* ---- CTA-pair tcgen05 GEMM for the linear layers (gemm.cu) ------------------------------ */
/* C[M, N] = A B^T (+ bias[N]) (+ R[M, N]); A K-major [M, K] (a_mn = 0) or MN-major [K, M];
 * B K-major [N, K] or MN-major [K, N]; bf16 operands, bias and R; C bf16 or fp32 (out_f32). */
NFB_EXPORT int nfb_gemm(const void* A, const void* B, void* C, int M, int N, int K, int64_t lda, int64_t ldb,
                        int64_t ldc, int a_mn, int b_mn, int out_f32, const void* bias, const void* R, int64_t ldr,
                        uint32_t* status, void* stream);
/* fp32 C = A B^T (accumulate = 0) or C += A B^T, split over K into `splits` slices (0: chosen
 * for the shape) that are added in a fixed order. flags: flag_words >= 8 * (tiles of 256 x 256)
 * uint32 words, any initial content; epoch must differ from the previous call that used them. */
NFB_EXPORT int nfb_gemm_acc(const void* A, const void* B, float* C, int M, int N, int K, int64_t lda, int64_t ldb,
                            int64_t ldc, int a_mn, int b_mn, int accumulate, int splits, uint32_t* flags,
                            int64_t flag_words, uint32_t epoch, uint32_t* status, void* stream);
NFB_EXPORT int nfb_gemm_acc_splits(int M, int N, int K);
/* SwiGLU fused into the gate/up projection: W [2F, K] with gate and up rows interleaved in 128-row
 * blocks; writes the pre-activations ab [M, 2F] (same interleaving) and act = silu(gate) * up [M, F]. */
NFB_EXPORT int nfb_gemm_swiglu_fwd(const void* X, const void* W, void* ab, void* act, int M, int F, int K,
                                   int64_t ldx, int64_t ldw, int64_t ldab, int64_t ldact, uint32_t* status,
                                   void* stream);
/* SwiGLU backward fused into the down projection's input gradient: d_ab [M, 2F] (interleaved) from
 * dY [M, D], W_down [D, F] and the forward's ab. */
NFB_EXPORT int nfb_gemm_swiglu_bwd(const void* dY, const void* Wd, const void* ab, void* dab, int M, int F, int D,
                                   int64_t ldy, int64_t ldw, int64_t ldab, int64_t lddab, uint32_t* status,
                                   void* stream);
/* Why the last failing nfb_gemm / nfb_gemm_acc call of this host thread failed ("" if none). */
NFB_EXPORT const char* nfb_gemm_last_error(void);
/* CUDA-core GEMM for widths the tensor-core kernel cannot tile: C[m, n] (+)= sum_k A[m, k] B[n, k]
 * (+ bias[n]) with every operand given by (row, column) element strides; dtype of A, B and bias
 * is fp32 or bf16 (dtype code), C is fp32 (out_f32) or that dtype. */
NFB_EXPORT int nfb_gemm_small(int dtype, int out_f32, const void* A, int64_t sam, int64_t sak, const void* B,
                              int64_t sbn, int64_t sbk, void* C, int64_t scm, int64_t scn, const void* bias, int M,
                              int N, int K, int accumulate, void* stream);
NFB_EXPORT int nfb_gemm_max_clusters(void);

/* ---- attention (attention.cu) ----------------------------------------------------------- */
NFB_EXPORT int nfb_attn_fwd(const void* q, const void* k, const void* v, void* o, float* lse, int B, int Sq, int Sk,
                            int Hq, int Hkv, int D, int64_t sq_b, int64_t sq_s, int64_t sq_h, int64_t sk_b,
                            int64_t sk_s, int64_t sk_h, int64_t sv_b, int64_t sv_s, int64_t sv_h, int64_t so_b,
                            int64_t so_s, int64_t so_h, int causal, float scale, uint32_t* status, void* stream);

/* Backward of nfb_attn_fwd: dq, dk, dv ([B, S, H, D], any 16-byte-aligned strides) from q, k, v, o, do and
 * the forward's lse. strides: 24 element strides, (batch, token, head) of q, k, v, o, do, dq, dk, dv.
 * scratch: nfb_attn_bwd_scratch_bytes(B, Sq, Hq, D) bytes (16-byte aligned). Three launches. */
NFB_EXPORT int64_t nfb_attn_bwd_scratch_bytes(int B, int Sq, int Hq, int D);
/* Profiling aid: 1024 uint64 device counters that later forward / backward launches add per-phase SM
 * cycles to (slots 0-31), with an event timeline of the first CTA from slot 64 (nullptr: off, the
 * default). */
NFB_EXPORT void nfb_attn_fwd_trace(void* counters);
/* Hardware characterisation: SM cycles of `iters` back-to-back M128 x n x K16 bf16 tcgen05.mma on
 * every SM (mode 0: operands K-major in shared memory; 1: B MN-major; 2: A from TMEM, B MN-major). */
NFB_EXPORT int nfb_mma_rate(int mode, int n, int iters, unsigned long long* out, int sms, void* stream);
NFB_EXPORT void nfb_attn_bwd_trace(void* counters);
NFB_EXPORT int nfb_attn_bwd(const void* q, const void* k, const void* v, const void* o, const void* dout,
                            const float* lse, void* dq, void* dk, void* dv, void* scratch, int B, int Sq, int Sk,
                            int Hq, int Hkv, int D, const int64_t* strides, int causal, float scale,
                            uint32_t* status, void* stream);

/* ---- peer memory (ipc.cu) --------------------------------------------------------------- */
NFB_EXPORT int nfb_ipc_handle_bytes(void);
NFB_EXPORT int nfb_ipc_alloc(uint64_t bytes, void** ptr, void* handle_out);
NFB_EXPORT int nfb_ipc_open(const void* handle, void** ptr);
NFB_EXPORT int nfb_ipc_close(void* ptr);
NFB_EXPORT int nfb_ipc_free(void* ptr);
NFB_EXPORT int nfb_copy_async(void* dst, const void* src, int64_t bytes, void* stream);

/* ---- collectives over NVLink peer memory (comm.cu) -------------------------------------- */
/* bases: device array of the world's workspace base addresses (this rank's mapping of each). */
NFB_EXPORT int nfb_comm_flag_bytes(void);
NFB_EXPORT int nfb_ar_twoshot(const uint64_t* bases, int rank, int world, const float* src, float* dst, int64_t n,
                              int64_t send_off, int64_t recv_off, int64_t flag_off, int slot, float scale,
                              uint32_t epoch, uint64_t timeout_ns, uint32_t* status, int ctas, void* stream);
/* Chunk-pipelined two-shot all-reduce: same buffers and result as nfb_ar_twoshot; progress flags on
 * slot and slot_b; chunk = 8-element vectors per slice per pipeline step. */
NFB_EXPORT int nfb_ar_pipelined(const uint64_t* bases, int rank, int world, const float* src, float* dst, int64_t n,
                                int64_t send_off, int64_t recv_off, int64_t flag_off, int slot, int slot_b,
                                float scale, uint32_t epoch, uint64_t timeout_ns, uint32_t* status, int64_t chunk,
                                int ctas, void* stream);
NFB_EXPORT int nfb_ar_oneshot(const uint64_t* bases, int rank, int world, const float* src, float* dst, int64_t n,
                              int64_t box_off, int64_t cap_elems, int64_t flag_off, int slot, float scale,
                              uint32_t epoch, uint64_t timeout_ns, uint32_t* status, int ctas, void* stream);
NFB_EXPORT int nfb_rs_push(const uint64_t* bases, int rank, int world, const float* src, int64_t n,
                           int64_t inbox_off, int64_t flag_off, int slot, float scale, uint32_t epoch,
                           uint64_t timeout_ns, uint32_t* status, float* out, int accumulate, int ctas, void* stream);
/* nfb_rs_push that also adds the shard's sum of squares into *sumsq_out (first phase of the global
 * gradient-norm clip; overwrite mode only). sumsq_partials >= ctas floats, ticket a zeroed word. */
NFB_EXPORT int nfb_rs_push_sumsq(const uint64_t* bases, int rank, int world, const float* src, int64_t n,
                                 int64_t inbox_off, int64_t flag_off, int slot, float scale, uint32_t epoch,
                                 uint64_t timeout_ns, uint32_t* status, float* out, int accumulate,
                                 float* sumsq_partials, uint32_t* ticket, float* sumsq_out, int ctas, void* stream);
NFB_EXPORT int nfb_rs_f32(const uint64_t* bases, int rank, int world, int64_t shard, int64_t send_off,
                          int64_t flag_off, int slot, float scale, uint32_t epoch, uint64_t timeout_ns,
                          uint32_t* status, float* out, float* sumsq_partials, uint32_t* ticket, float* sumsq_out,
                          int trailing_barrier, int accumulate, int ctas, void* stream);
NFB_EXPORT int nfb_rs_adamw(const uint64_t* bases, int rank, int world, int64_t shard, int64_t send_off,
                            int64_t flag_off, int slot, float scale, uint32_t epoch, uint64_t timeout_ns,
                            uint32_t* status, float* param, float* m, float* v, int64_t param_off, float lr,
                            float beta1, float beta2, float eps, float wd, int64_t step, float clip,
                            int trailing_barrier, int ctas, void* stream);
NFB_EXPORT int nfb_allgather(const uint64_t* bases, int rank, int world, int64_t shard, int64_t shard_off, void* out,
                             int64_t flag_off, int slot, uint32_t epoch, uint64_t timeout_ns, uint32_t* status,
                             int ctas, void* stream);
NFB_EXPORT int nfb_allreduce_scalar(const uint64_t* bases, int rank, int world, int64_t val_off, float* inout,
                                    int64_t flag_off, int slot, uint32_t epoch, uint64_t timeout_ns,
                                    uint32_t* status, void* stream);
NFB_EXPORT int nfb_wait_flag(const uint32_t* flag, uint32_t target, uint64_t timeout_ns, uint32_t* status,
                             void* stream);

/* ---- FSDP all-gather fused into the first consuming GEMM (ag_gemm.cu) ------------------- */
NFB_EXPORT int nfb_ag_gemm(const uint64_t* bases, int rank, int world, int64_t shard_off, int64_t shard_bytes,
                           void* full, int64_t lo, int64_t hi, int64_t w_off, int N, int K, const void* X,
                           int64_t ldx, int M, void* Y, int64_t ldy, uint32_t* ready, uint32_t* status,
                           void* stream);
NFB_EXPORT int nfb_ag_gemm_max_nblocks(void);

/* ---- host-side synthetic data (synth.cpp) ----------------------------------------------- */
/* Fills n bytes with a counter-based pseudo-random stream of (seed, index) using `threads`
 * host threads (the same bytes for any thread count). */
NFB_EXPORT int nfb_synth_fill_u8(uint8_t* dst, int64_t n, uint64_t seed, uint64_t index, int threads);

#ifdef __cplusplus
}
#endif

#endif /* NFB_API_H_ */
