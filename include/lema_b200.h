/*
 * lema_b200.h — C ABI of the B200 (sm_100a) W8A8 streamed-layer hot path.
 *
 * Every entry point takes plain pointers, sizes and leading dimensions (in
 * elements), plus a CUDA stream handle passed as `void*` (a `cudaStream_t`;
 * NULL means the legacy default stream). No torch types cross this boundary.
 *
 * Status convention: 0 = success; a nonzero `lema_status` otherwise, with a
 * human-readable message in `lema_last_error()` (thread-local). Nothing
 * aborts or traps. Device-side failures (a bounded wait that ran out) are
 * recorded in a per-device error word read by `lema_device_error()`.
 *
 * Arithmetic contract (the W8A8 operator; the reference has no quantised
 * linear, so this library defines it and the CPU oracle restates it):
 *   quantise rows:  amax[r] = max_k |x[r,k]| (fp32, exact from bf16)
 *                   s[r]    = amax[r] / 127 (IEEE fp32 division), 1 if amax == 0
 *                   q[r,k]  = clamp(rint_half_even(x[r,k] / s[r]), -127, 127)
 *   int8 GEMM:      acc[m,n] = sum_k xq[m,k] * wq[n,k]   (exact s32)
 *   epilogue:       y[m,n] = bf16_rne((float(acc) * sx[m]) * sw[n] + bias[n])
 *                   (fp32, in this order, no fused multiply-add)
 *   dgrad (STE):    wdeq[n,k] = bf16_rne(float(wq[n,k]) * sw[n])
 *                   dx[m,k]   = bf16_rne(sum_n dy[m,n] * wdeq[n,k])  (fp32 acc)
 */
#ifndef LEMA_B200_H
#define LEMA_B200_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define LEMA_API __attribute__((visibility("default")))
#else
#define LEMA_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

typedef enum lema_status {
  LEMA_OK = 0,
  LEMA_ERR_INVALID_ARGUMENT = 1, /* null pointer, negative size, bad stride */
  LEMA_ERR_MISALIGNED = 2,       /* pointer or leading dimension breaks a TMA/vector rule */
  LEMA_ERR_UNSUPPORTED = 3,      /* shape outside what the kernels implement */
  LEMA_ERR_CUDA = 4,             /* a CUDA runtime/driver call failed */
  LEMA_ERR_NOT_REGISTERED = 5,   /* memory manager: unknown buffer / slot id */
  LEMA_ERR_OVERFLOW = 6,         /* memory manager: pack larger than the buffer */
  LEMA_ERR_TIMEOUT = 7,          /* a bounded wait ran out */
  LEMA_ERR_DEVICE = 8            /* a kernel recorded a device-side failure */
} lema_status;

/* ---- errors / introspection ------------------------------------------- */

/* Message of the last failing call on this thread ("" if none). */
LEMA_API const char* lema_last_error(void);

/* Library version string, e.g. "lema_b200 0.1.0 sm_100a". */
LEMA_API const char* lema_version(void);

/* Synchronises the current device, then reads and clears its device-side
 * error word (0 = no kernel recorded a failure). */
LEMA_API int lema_device_error(int32_t* code_out);

/* Enqueues on `stream` a one-thread kernel that moves the current device's
 * error word into *host_word when it is nonzero, and clears it. host_word must
 * be page-locked host memory mapped into the device (cudaHostAlloc, torch's
 * pin_memory()). The host reads *host_word whenever it likes, with no sync: a
 * trainer enqueues this at the end of each step and checks the word before
 * each step, so a bounded wait that ran out stops training at the first step
 * that starts after the failing step's kernels have run. (Replaces no
 * reference interface: the reference has no device code.) */
LEMA_API int lema_device_error_async(int32_t* host_word, void* stream);

/* Number of SMs the kernels size their persistent grids for (current device). */
LEMA_API int lema_num_sms(int32_t* out);

/* ---- K1: per-row dynamic symmetric int8 quantisation ------------------- */
/* Replaces the activation side of the F.linear call inside the nn.Linear
 * projections that adapters/_llama.py:245-250 runs (wrapped by
 * _lora.py:23-26). rows x cols bf16 (row stride ldx) -> int8 (row stride ldq)
 * plus one fp32 scale per row. Per-token for activations (rows = tokens),
 * per-output-channel for weights (rows = out_features of an nn.Linear weight
 * [N,K]). Requires 16-byte aligned rows when cols >= 8 (ldx % 8 == 0, ldq % 16 == 0
 * and aligned base pointers); smaller or ragged rows take a scalar path. */
LEMA_API int lema_quantize_rows(const void* x_bf16, int64_t rows, int64_t cols, int64_t ldx,
                       int8_t* q, int64_t ldq, float* scale, void* stream);

/* The same rule applied to fp32 rows (the true weights of a trainable
 * projection, re-quantised after each optimizer step). */
LEMA_API int lema_quantize_rows_f32(const float* x, int64_t rows, int64_t cols, int64_t ldx,
                           int8_t* q, int64_t ldq, float* scale, void* stream);

/* Per-token activation quantisation (alias of lema_quantize_rows). */
LEMA_API int lema_quantize_per_token(const void* x_bf16, int64_t M, int64_t K, int64_t ldx,
                            int8_t* xq, int64_t ldq, float* sx, void* stream);

/* ---- K2+K3: int8 tcgen05 GEMM with fused dequant/bias/bf16 epilogue ----- */
/* y[M,N] (bf16, row stride ldy) from xq[M,K] (ld ldx), wq[N,K] (ld ldw),
 * sx[M], sw[N] (may be NULL = all ones), bias[N] (bf16, may be NULL = zero). acc_dbg (may be NULL)
 * receives the raw s32 accumulators [M,N] (row stride ldacc) for bit-exact
 * checks; y may be NULL when only acc_dbg is wanted.
 * Constraints: ldx % 16 == 0, ldw % 16 == 0, xq/wq 16-byte aligned,
 * K >= 0 (K == 0 gives y = bias). */
LEMA_API int lema_w8a8_gemm(const int8_t* xq, int64_t ldx, const float* sx,
                   const int8_t* wq, int64_t ldw, const float* sw,
                   const void* bias_bf16, void* y_bf16, int64_t ldy,
                   int32_t* acc_dbg, int64_t ldacc,
                   int64_t M, int64_t N, int64_t K, void* stream);

/* Forward of one W8A8 linear: K1 on x then K2+K3. xq_ws [M, ldq] int8 and
 * sx_ws [M] fp32 are caller-provided workspaces (they hold the quantised
 * activations afterwards). Replaces nn.Linear.forward at the A0 call sites. */
LEMA_API int lema_w8a8_linear_fwd(const void* x_bf16, int64_t ldx,
                         const int8_t* wq, int64_t ldw, const float* sw,
                         const void* bias_bf16, void* y_bf16, int64_t ldy,
                         int8_t* xq_ws, int64_t ldq, float* sx_ws,
                         int64_t M, int64_t N, int64_t K, void* stream);

/* Allocation-free variant of lema_w8a8_linear_fwd. It has no counterpart in
 * the reference. For callers that cannot allocate device memory (a host that
 * binds this ABI from a runtime without a CUDA allocator, or a process whose
 * device memory is owned by a framework's caching allocator under a fixed
 * VRAM budget): the quantised-activation workspace lives in fixed device
 * arrays inside this library (16 MiB of int8 + 65536 fp32 row scales, held
 * by every GPU that loads the library until exit). Requires
 * M * round_up(K, 16) <= 16 MiB and M <= 65536, else LEMA_ERR_UNSUPPORTED.
 * The first call on a device looks up the arrays' device addresses; make it
 * before any stream capture. All calls on a device share the arrays, so calls
 * that overlap on the GPU race and must be serialised by the caller. Calls no
 * cudaMalloc/cudaFree. */
LEMA_API int lema_w8a8_linear_fwd_noalloc(const void* x_bf16, int64_t ldx,
                                          const int8_t* wq, int64_t ldw, const float* sw,
                                          const void* bias_bf16, void* y_bf16, int64_t ldy,
                                          int64_t M, int64_t N, int64_t K, void* stream);

/* ---- K4: backward of the frozen base (straight-through estimator) ------- */
/* wdT[K,N] (bf16, row stride ldt) = bf16_rne(float(wq[n,k]) * sw[n]),
 * transposed so the dgrad GEMM reads it K-major. */
LEMA_API int lema_dequant_transpose(const int8_t* wq, int64_t ldw, const float* sw,
                           int64_t N, int64_t K, void* wdT_bf16, int64_t ldt,
                           void* stream);

/* y[M,N] = bf16_rne(a[M,K] . b[N,K]^T), bf16 operands, fp32 accumulation in
 * TMEM (tcgen05 kind::f16). lda % 8 == 0, ldb % 8 == 0, 16-byte aligned. */
LEMA_API int lema_bf16_gemm_tn(const void* a_bf16, int64_t lda, const void* b_bf16, int64_t ldb,
                      void* y_bf16, int64_t ldy, int64_t M, int64_t N, int64_t K,
                      void* stream);

/* The same bf16 GEMM with the fp32 accumulators as output (y_f32[M,N], row
 * stride ldy): the weight gradient dW = dy^T . x of a trainable projection
 * (selective full fine-tuning), fed transposed operands. Replaces the
 * autograd weight gradient whose fp32 accumulation _full_ft.py:186-192 keeps. */
LEMA_API int lema_bf16_gemm_tn_f32(const void* a_bf16, int64_t lda, const void* b_bf16,
                                   int64_t ldb, float* y_f32, int64_t ldy, int64_t M, int64_t N,
                                   int64_t K, void* stream);

/* dx[M,K] = dy[M,N] . wdeq[N,K]. wdT_ws is a caller-provided bf16 workspace
 * of at least K * ldt elements, ldt = N rounded up to a multiple of 8.
 * Replaces the autograd dgrad of F.linear reached from _trainer.py:161,166. */
LEMA_API int lema_w8a8_dgrad(const void* dy_bf16, int64_t lddy,
                    const int8_t* wq, int64_t ldw, const float* sw,
                    void* dx_bf16, int64_t lddx, void* wdT_ws, int64_t ldt,
                    int64_t M, int64_t N, int64_t K, void* stream);

/* Per-row int8 quantisation of x[r,c] * cs[c] (bf16 x, fp32 column scales cs,
 * the product rounded to fp32), same contract as lema_quantize_rows on the
 * products: the activation side of the int8-dy backward. */
LEMA_API int lema_quantize_rows_colscaled(const void* x_bf16, const float* cs, int64_t rows,
                                          int64_t cols, int64_t ldx, int8_t* q, int64_t ldq,
                                          float* scale, void* stream);

/* wqT[k,n] = wq[n,k] (int8 transpose; ldt >= N, ldt % 16 == 0). */
LEMA_API int lema_transpose_i8(const int8_t* wq, int64_t ldw, int64_t N, int64_t K,
                               int8_t* wqT, int64_t ldt, void* stream);

/* The int8-dy variant of the straight-through dgrad (opt-in; it has no
 * counterpart in the reference and a looser tolerance than lema_w8a8_dgrad):
 * dq, sd = quantise_rows(dy * sw), wqT = wq^T, dx = bf16(sd[m] * (dq . wqT^T)),
 * i.e. dx ~ dy . (wq * sw) with dy carried as int8 per row. Workspaces:
 * wqT_ws int8 [K, ldt] (ldt >= N, multiple of 16), dq_ws int8 [M, ldq]
 * (ldq >= N, multiple of 16), sd_ws fp32 [M]. */
LEMA_API int lema_w8a8_dgrad_int8(const void* dy_bf16, int64_t lddy, const int8_t* wq,
                                  int64_t ldw, const float* sw, void* dx_bf16, int64_t lddx,
                                  int8_t* wqT_ws, int64_t ldt, int8_t* dq_ws, int64_t ldq,
                                  float* sd_ws, int64_t M, int64_t N, int64_t K, void* stream);

/* ---- Selective full fine-tuning: fused optimizer step + re-quantisation ---- */
/* One AdamW step of a trainable projection, in place (the reference's per-layer
 * step, src/lema/_full_ft.py:204-229, each fp32 operation rounded once):
 *   w = f32(w) * decay;  m = m * beta1 + g * c1;  v = v * beta2 + (g * g) * c2;
 *   w = bf16_rne(w + step_size * (m / (sqrt(v) / sqrt_bc2 + eps)))
 * with decay = 1 - lr*wd, c1 = 1 - beta1, c2 = 1 - beta2, sqrt_bc2 =
 * sqrt(1 - beta2^t), step_size = -lr / (1 - beta1^t) (fp32 of the double
 * values); then each row of the new bf16 weight is quantised by the
 * lema_quantize_rows rule into q [rows, ldq] / scale [rows]; g is cleared when
 * zero_grad. w bf16 [rows, ldw], g fp32 [rows, ldg], m and v fp32 [rows, ldmv]. */
LEMA_API int lema_adamw_requant_rows(void* w_bf16, int64_t ldw, float* g, int64_t ldg, float* m,
                                     float* v, int64_t ldmv, int64_t rows, int64_t cols,
                                     float decay, float beta1, float c1, float beta2, float c2,
                                     float sqrt_bc2, float step_size, float eps,
                                     int32_t zero_grad, int8_t* q, int64_t ldq, float* scale,
                                     void* stream);

/* ---- Timing of the int8 GEMM launches ---------------------------------- */
/* Starts recording a CUDA event pair around every int8 GEMM launch (dense and
 * grouped, on the current device, streams not being captured) up to
 * max_records launches; events are created here, not in the timed region. */
LEMA_API int lema_gemm_timer_start(int64_t max_records);
/* Stops recording, waits for the recorded launches and returns the summed
 * 2*M*N*K ops, the summed launch durations in ms, the launches recorded and
 * the launches not recorded (pool full, capturing stream, other device). */
LEMA_API int lema_gemm_timer_stop(double* total_ops, double* total_ms, int64_t* launches,
                                  int64_t* dropped);

/* ---- Stream-K workspace and test hooks --------------------------------- */
/* Number of (device, stream) stream-K workspaces the library holds (each is
 * one cudaMalloc of partial-accumulator slots and flags, made on the first
 * GEMM on that stream whose plan splits a tile). */
LEMA_API int lema_gemm_workspace_count(int64_t* count);
/* Test hooks of the GEMMs' bounded waits; the defaults are what every other
 * caller runs with. skip_publish != 0: split tiles' partial ranges are not
 * published, so the owners' waits for them run out and record 0x104 in the
 * device error word. wait_budget_cycles: clock64 cycles each bounded wait in
 * the GEMM kernels may spin before it records its error and the kernel drains
 * and returns; 0 restores the default (about 2 s). Applies to launches issued
 * after the call, from any thread. */
LEMA_API int lema_gemm_set_test_hooks(int32_t skip_publish, int64_t wait_budget_cycles);

/* ---- Fused producers of the W8A8 GEMM inputs (and their backward) ------ */
/* RMSNorm of HF LlamaRMSNorm as adapters/_llama.py:238,248 apply it, in bf16:
 * hn = bf16(g * bf16(x * rsqrt(mean(x^2) + eps))) per row; rstd[r] (fp32) for
 * the backward; when q is not NULL also the per-row int8 quantisation of hn
 * (the lema_quantize_rows rule) for the projections that read it. cols % 8 == 0,
 * cols <= 16384, 16-byte aligned rows. */
LEMA_API int lema_rmsnorm_quant(const void* x_bf16, int64_t ldx, const void* g_bf16,
                                int64_t rows, int64_t cols, float eps, void* hn_bf16,
                                int64_t ldh, int8_t* q, int64_t ldq, float* scale, float* rstd,
                                void* stream);

/* dx = rstd * (g*dhn - xhat * mean(g*dhn*xhat)), xhat = x * rstd (fp32, bf16 out). */
LEMA_API int lema_rmsnorm_bwd(const void* x_bf16, int64_t ldx, const void* g_bf16,
                              const float* rstd, const void* dhn_bf16, int64_t ldd,
                              int64_t rows, int64_t cols, void* dx_bf16, int64_t lddx,
                              void* stream);

/* Rotary embedding of q and k rows (token t = b*seq + s uses cos/sin row s,
 * [seq, head_dim] bf16): mode 0 = forward with the bf16 roundings of
 * q*cos + rotate_half(q)*sin (HF apply_rotary_pos_emb, reached from
 * adapters/_llama.py:242); mode 1 = backward (transposed rotation). Inputs may
 * be strided rows (ld in elements); outputs are contiguous [tokens, heads*dim]. */
LEMA_API int lema_rope(const void* q_in, int64_t ldq_in, const void* k_in, int64_t ldk_in,
                       const void* cos_bf16, const void* sin_bf16, int64_t tokens, int32_t seq,
                       int32_t heads_q, int32_t heads_k, int32_t head_dim, void* q_out,
                       void* k_out, int32_t mode, void* stream);

/* lema_rope for the three outputs of a stacked q/k/v projection: v_in (may be
 * NULL) is copied, not rotated, into contiguous v_out; q_add / k_add / v_add
 * (may be NULL; contiguous [tokens, heads*dim]) are added first with bf16
 * rounding (LoRA outputs, _lora.py:23-26). Backward (mode 1) ignores v and the
 * addends. */
LEMA_API int lema_rope_qkv(const void* q_in, int64_t ldq, const void* k_in, int64_t ldk,
                           const void* v_in, int64_t ldv, const void* q_add, const void* k_add,
                           const void* v_add, const void* cos_bf16, const void* sin_bf16,
                           int64_t tokens, int32_t seq, int32_t heads_q, int32_t heads_k,
                           int32_t head_dim, void* q_out, void* k_out, void* v_out,
                           int32_t mode, void* stream);

/* SwiGLU of HF LlamaMLP (act(gate) * up) on rows of [gate | up] ([rows, 2*inter],
 * row stride ldgu), quantised per row (lema_quantize_rows rule) for the down
 * projection; m_bf16 (may be NULL) receives the bf16 product. */
LEMA_API int lema_swiglu_quant(const void* gu_bf16, int64_t ldgu, int64_t rows, int64_t inter,
                               int8_t* q, int64_t ldq, float* scale, void* m_bf16, int64_t ldm,
                               void* stream);

/* d[gate | up] from dm and the saved [gate | up] (fp32 math, bf16 out). */
LEMA_API int lema_swiglu_bwd(const void* gu_bf16, int64_t ldgu, const void* dm_bf16,
                             int64_t lddm, int64_t rows, int64_t inter, void* dgu_bf16,
                             int64_t lddgu, void* stream);

/* ---- causal attention (head_dim 128, GQA) on tcgen05 ----------------------- */
/* Replaces the block's torch scaled_dot_product_attention(q, k, v,
 * is_causal=True, scale=scale, enable_gqa=H != Hkv) that the reference's Llama
 * adapter reaches through HF attention (src/lema/adapters/_llama.py:236-252).
 * q [B*S, H*128] (row stride ldq), k / v [B*S, Hkv*128], o [B*S, H*128], all
 * bf16 token-major with 16-byte aligned bases and strides a multiple of 8;
 * query head h reads kv head h / (H / Hkv). lse [B, H, S] fp32 receives each
 * row's log2-domain log-sum-exp of the scaled scores (the backward's input). */
LEMA_API int lema_attn_fwd(const void* q, int64_t ldq, const void* k, int64_t ldk,
                           const void* v, int64_t ldv, void* o, int64_t ldo, float* lse,
                           int64_t B, int64_t S, int64_t H, int64_t Hkv, int64_t head_dim,
                           float scale, void* stream);

/* Gradients of lema_attn_fwd: dq [B*S, H*128], dk / dv [B*S, Hkv*128] (bf16,
 * written whole; dk / dv of a kv head sum over its query heads) from q, k, v,
 * the forward's o and lse, and dout. Caller-provided scratch: delta [B, H, S]
 * fp32 (receives rowsum(dout * o)) and, optionally, dkv_ws of 2*B*S*H*128 fp32
 * (16-byte aligned): with GQA and fewer (b, kv head, key tile) units than SMs,
 * each query head's dK / dV share goes there and a fourth kernel sums
 * them in head order; NULL keeps one CTA per kv head. Three or four kernels on
 * `stream`. */
LEMA_API int lema_attn_bwd(const void* q, int64_t ldq, const void* k, int64_t ldk,
                           const void* v, int64_t ldv, const void* o, int64_t ldo,
                           const void* dout, int64_t lddo, const float* lse, float* delta,
                           float* dkv_ws, void* dq, int64_t lddq, void* dk, int64_t lddk,
                           void* dv, int64_t lddv, int64_t B, int64_t S, int64_t H,
                           int64_t Hkv, int64_t head_dim, float scale, void* stream);

/* Wait budget (clock cycles) of the attention kernels' bounded waits; 0
 * restores the default. A wait that runs out records device error 0x105. */
LEMA_API int lema_attn_set_wait_budget(int64_t cycles);

/* ---- K6: grouped W8A8 GEMM (MoE experts) -------------------------------- */
/* Tokens are pre-sorted by expert: rows [offsets[e], offsets[e+1]) of xq/sx/y
 * belong to expert e, whose weights are wq + e*N*ldw, sw + e*N and
 * bias + e*N (bias may be NULL). offsets is a HOST array of E+1 entries.
 * Replaces the per-expert matmuls of the grouped_mm experts implementation
 * selected at adapters/_mixtral.py:21-22 and run at :266-268. */
LEMA_API int lema_grouped_w8a8_gemm(const int8_t* xq, int64_t ldx, const float* sx,
                           const int8_t* wq, int64_t ldw, const float* sw,
                           const void* bias_bf16, void* y_bf16, int64_t ldy,
                           const int64_t* offsets_host, int32_t E,
                           int64_t N, int64_t K, void* stream);

/* Grouped bf16 GEMM: rows [offsets[e], offsets[e+1]) of a times b_e^T, with
 * b_e = b + e*N*ldb ([N, K] per group), fp32 accumulation, bf16 out. offsets
 * is a HOST array of E+1 entries. */
LEMA_API int lema_grouped_bf16_gemm_tn(const void* a_bf16, int64_t lda, const void* b_bf16,
                                       int64_t ldb, void* y_bf16, int64_t ldy,
                                       const int64_t* offsets_host, int32_t E, int64_t N,
                                       int64_t K, void* stream);

/* Grouped straight-through dgrad of the MoE experts: rows of expert e get
 * dx = dy . bf16(wq_e * sw_e) (wq_e = wq + e*N*ldw, [N, K]). wdT_ws holds at
 * least E * K * ldt bf16 (ldt >= N, multiple of 8). Replaces the autograd
 * dgrad of the per-expert F.linear calls of the grouped_mm experts
 * implementation (adapters/_mixtral.py:21-22, 266-268). */
LEMA_API int lema_grouped_w8a8_dgrad(const void* dy_bf16, int64_t lddy, const int8_t* wq,
                                     int64_t ldw, const float* sw, void* dx_bf16,
                                     int64_t lddx, void* wdT_ws, int64_t ldt,
                                     const int64_t* offsets_host, int32_t E, int64_t N,
                                     int64_t K, void* stream);

/* ---- K5: boundary-activation checkpoint offload -------------------------- */
/* Copies `bytes` from device memory `src` into pinned host memory `dst`
 * (allocated with cudaHostAlloc / torch pin_memory) on `copy_stream`, after
 * `after_event` (may be NULL) has completed; records `done_event` (may be
 * NULL) on copy_stream when the copy is issued. mode 0 = copy engine
 * (cudaMemcpyAsync), mode 1 = SM kernel storing through the mapped host
 * pointer with 16-byte stores. Replaces the VRAM-resident
 * boundary_activations list of _trainer.py:109-111. */
LEMA_API int lema_ckpt_save(const void* src, void* pinned_dst, size_t bytes, int32_t mode,
                   void* copy_stream, void* after_event, void* done_event);

/* Host pinned -> device restore of a saved boundary activation
 * (_trainer.py:146-148), same event protocol, copy engine only. */
LEMA_API int lema_ckpt_restore(const void* pinned_src, void* dst, size_t bytes,
                      void* copy_stream, void* after_event, void* done_event);

/* ---- Native memory manager (drop-in for _csrc/memory_manager.{h,cpp}) ---- */
/* Mirrors LemaMemoryManager (memory_manager.h:25-92, pybind names at
 * memory_manager.cpp:204-217): RAM buffers and VRAM slots are registered by
 * pointer + byte size (the caller keeps ownership), transfers run on one
 * H2D copy stream with a ring of events, prefetch jobs run on 2 worker
 * threads. Errors return a status instead of throwing. */
typedef struct lema_mm lema_mm;
typedef void (*lema_job_fn)(void* user);

LEMA_API int lema_mm_create(int64_t num_layers_hint, int64_t max_layer_size, int32_t device,
                   lema_mm** out);
LEMA_API int lema_mm_destroy(lema_mm* mm);
LEMA_API int lema_mm_register_ram_buffer(lema_mm* mm, int64_t layer_id, void* host_ptr, size_t bytes);
LEMA_API int lema_mm_register_vram_slot(lema_mm* mm, int64_t slot, void* dev_ptr, size_t bytes);
/* Packs n host tensors (pointer + bytes) back to back into RAM buffer layer_id. */
LEMA_API int lema_mm_pack_layer_to_ram(lema_mm* mm, int64_t layer_id, const void* const* srcs,
                              const size_t* sizes, int64_t n);
/* Same, but each tensor starts on a multiple of `align` bytes (int8 segments). */
LEMA_API int lema_mm_pack_layer_to_ram_aligned(lema_mm* mm, int64_t layer_id, const void* const* srcs,
                                      const size_t* sizes, int64_t n, size_t align,
                                      size_t* offsets_out);
/* H2D of the whole registered RAM buffer (or its first `bytes`, 0 = all) into
 * a VRAM slot; returns an event id. The copy stream first waits for the
 * slot's "free" event so a slot is never overwritten while compute still
 * reads it. */
LEMA_API int lema_mm_async_transfer_to_vram(lema_mm* mm, int64_t layer_id, int64_t vram_slot,
                                   size_t bytes, int64_t* event_id_out);
/* Makes `stream` wait (on the device, no host block) for a transfer event. */
LEMA_API int lema_mm_stream_wait_transfer(lema_mm* mm, int64_t event_id, void* stream);
/* Records on `stream` that compute is done reading `vram_slot`. */
LEMA_API int lema_mm_release_vram_slot(lema_mm* mm, int64_t vram_slot, void* stream);
LEMA_API int lema_mm_wait_vram_transfer(lema_mm* mm, int64_t event_id);
/* Bounded variant: LEMA_ERR_TIMEOUT after timeout_ms. */
LEMA_API int lema_mm_wait_vram_transfer_timeout(lema_mm* mm, int64_t event_id, int64_t timeout_ms);
LEMA_API int lema_mm_is_transfer_complete(lema_mm* mm, int64_t event_id, int32_t* done_out);
LEMA_API int lema_mm_synchronize_all(lema_mm* mm);
LEMA_API int lema_mm_submit_prefetch_job(lema_mm* mm, lema_job_fn fn, void* user, int64_t* job_id_out);
LEMA_API int lema_mm_is_prefetch_complete(lema_mm* mm, int64_t job_id, int32_t* done_out);
LEMA_API int lema_mm_wait_for_prefetch(lema_mm* mm, int64_t job_id);
LEMA_API int lema_mm_wait_for_prefetch_timeout(lema_mm* mm, int64_t job_id, int64_t timeout_ms);
LEMA_API int lema_mm_is_layer_in_ram(lema_mm* mm, int64_t layer_id, int32_t* out);
/* The manager's H2D copy stream (a cudaStream_t). */
LEMA_API int lema_mm_copy_stream(lema_mm* mm, void** stream_out);

#ifdef __cplusplus
}
#endif

#endif /* LEMA_B200_H */
