/*
 * gollama_cuda.h — C ABI of libgollama_cuda.so, the sm_100a (B200) backend for
 * the training hot path of gollama (pkg/train + pkg/tensor/grad.go).
 *
 * Conventions (modelled on the reference's only device boundary, the Metal
 * plugin pkg/metal/metal.go:183-246, whose C functions return an int that the
 * Go wrapper turns into an error):
 *   - every function returns int: 0 = success, negative = error (GLC_ERR_*);
 *     the message of the last error is available from glc_last_error();
 *   - no function aborts the process, and there is no CPU fallback: if the
 *     CUDA path cannot run, the call fails;
 *   - tensors are row-major fp32 device buffers, weights are [out, in]
 *     (pkg/train/trainer.go:226-234); token ids are int64 (Go `int`);
 *   - op functions only enqueue work on the context's stream; errors raised
 *     on the device (a bounded wait that ran out) are reported by the next
 *     glc_sync();
 *   - a context is used by one host thread at a time (the reference tape runs
 *     its GradFns sequentially on one goroutine, pkg/tensor/grad.go:70-75).
 */
#ifndef GOLLAMA_CUDA_H
#define GOLLAMA_CUDA_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define GLC_API __attribute__((visibility("default")))
#else
#define GLC_API
#endif

#define GLC_OK 0
#define GLC_ERR_INVALID (-1)     /* bad argument (size, alignment, null pointer) */
#define GLC_ERR_CUDA (-2)        /* CUDA runtime/driver error */
#define GLC_ERR_DEVICE (-3)      /* device-side error word set (bounded wait ran out) */
#define GLC_ERR_NOMEM (-4)       /* device allocation failed */
#define GLC_ERR_NCCL (-5)        /* NCCL error or timeout */
#define GLC_ERR_UNSUPPORTED (-6) /* not available in this build / device */
#define GLC_ERR_IO (-7)          /* a file cannot be opened, read or written, or is malformed or corrupt */

typedef struct glc_ctx glc_ctx;

/* ------------------------------------------------------------------ context
 * Replaces metal.Init / metal_init (pkg/metal/metal.go:184-190, :5-60): opens
 * the device, creates the compute stream, the device error word and resolves
 * cuTensorMapEncodeTiled.  Fails with GLC_ERR_UNSUPPORTED on anything but an
 * sm_100 device. */
GLC_API int glc_init(int device, glc_ctx** out);
/* Replaces metal.Cleanup (pkg/metal/metal.go:193-196).  Trainers and models
 * created on the context must be destroyed before it (they use its stream). */
GLC_API int glc_destroy(glc_ctx* ctx);
/* Copies the last error message (NUL-terminated, truncated to n): the text a
 * Go wrapper puts in its error, as the Metal wrappers format a failing status
 * (pkg/metal/metal.go:185-187).  With ctx == NULL: the message of the calling
 * thread's last failed call that takes no context (the checkpoint file
 * functions). */
GLC_API int glc_last_error(glc_ctx* ctx, char* buf, size_t n);
/* Replaces metal.DeviceName (pkg/metal/metal.go:204-206). */
GLC_API int glc_device_name(glc_ctx* ctx, char* buf, size_t n);
/* Waits for all enqueued work and reports device-side errors.  No reference
 * counterpart: the Metal calls return when their work is done
 * (pkg/metal/metal.go:210-226); this library's calls are enqueued. */
GLC_API int glc_sync(glc_ctx* ctx);
/* Number of kernels this library has launched on the context (diagnostics;
 * no reference counterpart). */
GLC_API int glc_launch_count(glc_ctx* ctx, uint64_t* out);

/* ------------------------------------------------------------------ memory
 * Device-resident storage behind pkg/tensor.Tensor.Data (pkg/tensor/tensor.go:10-14). */
GLC_API int glc_malloc(glc_ctx* ctx, size_t bytes, void** dptr);
GLC_API int glc_free(glc_ctx* ctx, void* dptr);
GLC_API int glc_memcpy_h2d(glc_ctx* ctx, void* dst, const void* src, size_t bytes);
GLC_API int glc_memcpy_d2h(glc_ctx* ctx, void* dst, const void* src, size_t bytes);
GLC_API int glc_memcpy_d2d(glc_ctx* ctx, void* dst, const void* src, size_t bytes);
GLC_API int glc_memset(glc_ctx* ctx, void* dptr, int value, size_t bytes);
/* Page-locked host memory for the asynchronous copies below (no reference
 * counterpart: the Go trainer's host slices are ordinary memory). */
GLC_API int glc_host_alloc(glc_ctx* ctx, size_t bytes, void** hptr);
GLC_API int glc_host_free(glc_ctx* ctx, void* hptr);
GLC_API int glc_memcpy_h2d_async(glc_ctx* ctx, void* dst, const void* src, size_t bytes);
GLC_API int glc_memcpy_d2h_async(glc_ctx* ctx, void* dst, const void* src, size_t bytes);

/* ------------------------------------------------------------------ timing
 * CUDA events on the context's compute stream (no reference counterpart). */
GLC_API int glc_timer_start(glc_ctx* ctx);
GLC_API int glc_timer_stop(glc_ctx* ctx, float* ms); /* synchronises on the stop event */

/* ------------------------------------------------------------------ profiling
 * While enabled, every kernel launch of this library is bracketed by a CUDA
 * event pair on its stream.  glc_profile_end synchronises and returns, per
 * kernel class (GLC_PROF_*), the launch count, the summed device time and the
 * summed algorithmic work (FLOPs for GEMM and attention, bytes otherwise).
 * No reference counterpart. */
#define GLC_PROF_GEMM 0
#define GLC_PROF_ATTN_FWD 1
#define GLC_PROF_ATTN_BWD 2
#define GLC_PROF_RMSNORM 3
#define GLC_PROF_SWIGLU 4
#define GLC_PROF_CE 5
#define GLC_PROF_ADAMW 6
#define GLC_PROF_OTHER 7
#define GLC_PROF_CLASSES 8
GLC_API int glc_profile_begin(glc_ctx* ctx);
GLC_API int glc_profile_end(glc_ctx* ctx, int n_classes, uint64_t* counts, double* total_ms, double* total_work);

/* ------------------------------------------------------------------ linear layers
 * All three run the tcgen05 TF32 tensor-core GEMM with fp32 accumulation.
 * X: [M,K], W: [N,K], Y/dY: [M,N].  Leading dimensions equal the row lengths;
 * every row length must be a multiple of 4 and every pointer 16-byte aligned.
 *
 * Y = X . W^T (+ residual[M,N] when residual != NULL).
 * Replaces MatMulTransposeB (pkg/tensor/matmul.go:145-234) as called by the
 * forward of MatMulGrad (pkg/tensor/grad.go:81-91), with the residual add of
 * AddGrad's forward (pkg/tensor/ops.go:6-17) fused into the epilogue. */
GLC_API int glc_linear_fwd(glc_ctx* ctx, const float* X, const float* W, float* Y, int M, int K, int N,
                   const float* residual);
/* dX (+)= dY . W.  Replaces the dA loop of MatMulGrad (pkg/tensor/grad.go:102-116);
 * accumulate=1 gives the reference's `+=`, accumulate=0 overwrites. */
GLC_API int glc_linear_bwd_dx(glc_ctx* ctx, const float* dY, const float* W, float* dX, int M, int K, int N,
                      int accumulate);
/* dW (+)= dY^T . X.  Replaces the dB loop of MatMulGrad (pkg/tensor/grad.go:118-152). */
GLC_API int glc_linear_bwd_dw(glc_ctx* ctx, const float* dY, const float* X, float* dW, int M, int K, int N,
                      int accumulate);
/* The whole GradFn of MatMulGrad (pkg/tensor/grad.go:94-152) in one launch:
 * dX (+)= dY . W and dW (+)= dY^T . X share one persistent tile queue.
 * dX or dW may be NULL when that gradient is not required. */
GLC_API int glc_linear_bwd(glc_ctx* ctx, const float* dY, const float* X, const float* W, float* dX, float* dW, int M,
                           int K, int N, int accumulate_dx, int accumulate_dw);
/* Gate and up projections with the SwiGLU product in one launch:
 * GU[M][2F] = X[M][K] . Wgu^T (Wgu = [WGate rows F | WUp rows F], each
 * MatMulTransposeB, pkg/tensor/matmul.go:145-234) and H[M][F] = silu(gate) *
 * up (SiLUGrad's forward, pkg/tensor/grad.go:426-427, then the product node,
 * pkg/train/trainer.go:400-422, with the reference's exp32), H TF32-rounded
 * when round_h.  GU and H equal glc_linear_fwd followed by glc_swiglu_fwd bit
 * for bit.  The SwiGLU runs in the GEMM epilogue on CTA pairs; with the
 * reference's float64 exp32 that epilogue does not hide under the MMAs at
 * 4096 x 2048 x 2*5632 (0.47 ms against 0.30 + 0.13 ms for the two calls), so
 * glc_train_step keeps the two launches. */
GLC_API int glc_linear_fwd_swiglu(glc_ctx* ctx, const float* X, const float* Wgu, float* GU, float* H, int M, int K,
                                  int F, int round_h);
/* Frozen quantized weights (pkg/quant/dequant.go).  Type codes are GGUF's
 * (pkg/gguf/format.go:40-58). */
#define GLC_QTYPE_F32 0
#define GLC_QTYPE_F16 1
#define GLC_QTYPE_Q4_0 2
#define GLC_QTYPE_Q4_1 3
#define GLC_QTYPE_Q5_0 6
#define GLC_QTYPE_Q5_1 7
#define GLC_QTYPE_Q8_0 8
#define GLC_QTYPE_Q4_K 12
#define GLC_QTYPE_Q6_K 14
/* Dequantize (pkg/quant/dequant.go:367-393) of n elements on the device, exact
 * fp32 results for every type the reference's Dequantize accepts: F16 via
 * fp16ToFp32 (:9-41), Q8_0 (:68-85), Q4_0 (:99-119; low nibble first), Q4_1
 * (:141-163), Q5_0 (:167-199), Q5_1 (:203-233), Q4_K (:237-300) and Q6_K
 * (:304-344), in the reference's layouts.  src 2-byte aligned, dst 16-byte
 * aligned; n a multiple of 4 and of the block (32, or 256 for the K types). */
GLC_API int glc_dequantize(glc_ctx* ctx, int type, const void* src, float* dst, size_t n);
/* dX (+)= dY . deq(W) for a linear layer whose weight W [N out][K in] is stored
 * quantized row by row: the dA loop of MatMulGrad (pkg/tensor/grad.go:102-116)
 * applied to the weight the reference dequantizes at load
 * (pkg/model/transformer.go:285-303).  Uses the context workspace for one
 * TF32-rounded fp32 copy of W, or none on the fused path (glc_set_quant_path). */
GLC_API int glc_linear_bwd_dx_q(glc_ctx* ctx, const float* dY, const void* Wq, int type, float* dX, int M, int K,
                                int N, int accumulate);
/* General strided form of the three above (the products of MatMulGrad,
 * pkg/tensor/grad.go:81-152, on any operand storage): C[M,N] (+)= A . B^T (+ R) where
 * a_mn/b_mn select MN-major storage (element (i,k) at ptr[k*ld+i]) instead of
 * K-major (ptr[i*ld+k]).  round_out rounds the stored values to TF32. */
GLC_API int glc_gemm_tf32(glc_ctx* ctx, const float* A, int lda, int a_mn, const float* B, int ldb, int b_mn, float* C,
                  int ldc, int M, int N, int K, int accumulate, const float* R, int ldr, int round_out);
/* Selects the GEMM tile shape for later calls on this context (tuning and
 * diagnostics; no reference counterpart): 0 automatic (CTA-pair 256x256 tiles
 * on tcgen05.mma.cta_group::2 unless a problem has at most 128 rows),
 * 1 single-CTA 128x256 tiles, 2 CTA-pair tiles always.  Results agree to fp32
 * rounding across variants. */
GLC_API int glc_set_gemm_variant(glc_ctx* ctx, int variant);
/* Selects how many CTAs share one KV head's query-head group in the attention
 * backward's dK/dV kernel (tuning and diagnostics; no reference counterpart):
 * 0 automatic, else a divisor of H / Hkv (other values fall back to automatic).
 * Each CTA accumulates its heads in TMEM; more than one writes partials that a
 * deterministic group sum adds.  Results agree to fp32 rounding across splits. */
GLC_API int glc_set_attention_split(glc_ctx* ctx, int nsplit);
/* RMSNorm backward kernel (tuning; no reference counterpart): 1 process a
 * block's rows one after another; 2 stage the next rows' x, dy and dx in
 * shared memory with cp.async while the current row is reduced (bit-identical
 * to 1); 3 (the exact gradient only) stream whole rows through a ring of four
 * bulk-copy stages and apply 1/rms as a product (within fp32 rounding of 1);
 * 0 automatic: 3 for the exact gradient, 1 for the reference's simplified one.
 * Variants 2 and 3 take rows of up to 2048 columns; wider rows use 1. */
GLC_API int glc_set_rmsnorm_variant(glc_ctx* ctx, int variant);
/* Softmax cross-entropy kernel for vocabularies above 8192 (tuning; no
 * reference counterpart): 1 one-shot clusters of four CTAs, each row split in
 * quarters held in registers; 2 (V <= 32768) one persistent CTA per SM that
 * streams its rows through a ring of bulk-copied chunks and holds the current
 * row in registers; 0 automatic: 2 for glc_softmax_ce_llama (and the
 * Llama-mode step) up to V = 32768, else 1.  Both sum each row in a fixed
 * order of their own, and 2 computes the Llama exponential as ex2.approx of
 * one FMA: results agree to fp32 rounding, not bit for bit. */
GLC_API int glc_set_ce_variant(glc_ctx* ctx, int variant);
/* glc_linear_bwd_dx_q's path (tuning; no reference counterpart): 0 automatic
 * and 1 dequantize W into the workspace, then the CTA-pair GEMM; 2 decode the
 * stored blocks inside the GEMM's operand load (no fp32 copy of W; F16 and
 * the block formats with K a whole number of blocks, else path 1).  Both
 * round W to TF32 the same way. */
GLC_API int glc_set_quant_path(glc_ctx* ctx, int path);
/* Tracing (no reference counterpart): 1 marks the phases of each training
 * step (forward, loss + backward, the remaining gradient sums, clip + AdamW,
 * the loss readback) as NVTX ranges for a profiler's timeline; 0 (default)
 * skips them.  Without a profiler attached the ranges cost nothing. */
GLC_API int glc_set_tracing(glc_ctx* ctx, int on);
/* Programmatic dependent launch (tuning; no reference counterpart): 1 lets each
 * of this library's kernels begin launching while the previous kernel on the
 * stream finishes; every kernel first waits for that predecessor to complete
 * and its memory to be visible, so results are bit-identical (the default,
 * 0.5-0.7 ms shorter TinyLlama-shape steps); 0: ordinary launches. */
GLC_API int glc_set_pdl(glc_ctx* ctx, int on);
/* Attention forward kernel (tuning; no reference counterpart): 1 one CTA per
 * (query tile, batch, head); 0 automatic and 2 one persistent CTA per SM
 * walking those items with its pipelines running across them (the next
 * item's loads and score products overlap the current item's last tiles and
 * output).  Results are bit-identical. */
GLC_API int glc_set_attention_fwd_variant(glc_ctx* ctx, int variant);
/* The same choice for the attention backward's dQ kernel (tuning; no
 * reference counterpart): 2 walks its
 * (query tile, batch, head) items persistently, moving the next item's Q and
 * dO into TMEM while the current item's dQ is written; 0 automatic and 3 the
 * same with sixteen softmax warps in two groups taking alternate steps; 1 one
 * CTA per item.  Bit-identical. */
GLC_API int glc_set_attention_dq_variant(glc_ctx* ctx, int variant);
/* The attention backward's dK/dV kernel (tuning; no reference counterpart):
 * 1 eight softmax warps that take
 * every 64-query step in turn; 0 automatic and 2 sixteen softmax warps in two
 * groups taking alternate steps, so one group's arithmetic overlaps the
 * other's.  Bit-identical. */
GLC_API int glc_set_attention_dkdv_variant(glc_ctx* ctx, int variant);
/* Tile order of the CTA-pair GEMM (tuning; no reference counterpart): 1 a
 * fixed order per pair (a rotation, or host-built lists for a grouped dX + dW
 * launch); 2 dynamic: every pair takes the next tile from a counter when it
 * is ready, so pairs that start late (their SMs held by another kernel, e.g.
 * the gradient allreduce) take fewer tiles; 0 automatic: 2 once data
 * parallelism is initialised, 1 otherwise.  Each tile is computed the same
 * way in every order: results are bit-identical. */
GLC_API int glc_set_gemm_schedule(glc_ctx* ctx, int mode);
/* Trainer (Llama semantics): 1 computes the SwiGLU forward in the gate/up
 * GEMM's epilogue, 0 (default, faster on B200 at the TinyLlama shape) runs it
 * as its own kernel after the GEMM (diagnostics; no reference counterpart).
 * Results are bit-identical. */
GLC_API int glc_set_fused_swiglu(glc_ctx* ctx, int on);

/* ------------------------------------------------------------------ fused / elementwise ops
 * Building blocks of the tape's GradFns; each mirrors one reference node.
 * round_out != 0 writes TF32-rounded values (round to nearest) for tensors
 * whose consumers are tensor-core GEMMs. */

/* RMSNormTrainable.Forward (pkg/train/trainer.go:141-168): y = (x/rms)*w with
 * rms = float32(sqrt(float64(sum x^2)/cols + float64(eps))); rms[rows] saved. */
GLC_API int glc_rmsnorm_fwd(glc_ctx* ctx, const float* x, const float* w, float* y, float* rms, int rows, int cols,
                            float eps, int round_out);
/* Its GradFn (trainer.go:170-200).  full=0: the reference's simplified
 * gradient; full=1: the exact RMSNorm gradient.  dx (+)= ..., dw (+)= ...;
 * dx_round (nullable) receives dx rounded to TF32. */
GLC_API int glc_rmsnorm_bwd(glc_ctx* ctx, const float* x, const float* w, const float* rms, const float* dy,
                            float* dx, float* dx_round, float* dw, int rows, int cols, int full, int dx_accumulate,
                            int dw_accumulate);
/* SiLUGrad + product node of forwardFFN (pkg/tensor/grad.go:417-449,
 * pkg/train/trainer.go:396-422) fused: h = silu(gate) * up, with the
 * reference's exp32. n = number of elements (multiple of 4). */
GLC_API int glc_swiglu_fwd(glc_ctx* ctx, const float* gate, const float* up, float* h, size_t n, int round_out);
GLC_API int glc_swiglu_bwd(glc_ctx* ctx, const float* gate, const float* up, const float* dh, float* dgate,
                           float* dup, size_t n, int accumulate, int round_out);
/* RoPE (pkg/model/rope.go:96-126, consecutive pairs) in place on x[T, nh*hd],
 * position t % S; inverse=1 is the backward rotation.  cos_t/sin_t are the
 * [max_seq][hd/2] tables of glc_rope_table (device pointers). */
GLC_API int glc_rope(glc_ctx* ctx, float* x, int T, int S, int nh, int hd, const float* cos_t, const float* sin_t,
                     int inverse, int round_out);
/* Host-side RoPE tables (precomputeFreqs, pkg/model/rope.go:33-48). */
GLC_API int glc_rope_table(int hd, int max_seq, float theta, float* cos_host, float* sin_host);
/* Causal attention (forwardAttention, pkg/train/trainer.go:323-389) with
 * grouped KV heads (pkg/model/attention.go:118,149).  q,o: [B*S, H*hd];
 * k,v: [B*S, Hkv*hd]; lse: [B, H, S]. */
GLC_API int glc_attention_fwd(glc_ctx* ctx, const float* q, const float* k, const float* v, float* o, float* lse,
                              int B, int S, int H, int Hkv, int hd, int round_out);
/* Its backward (dq, dk, dv overwritten).  The reference attaches no GradFn to
 * its attention (trainer.go:335-337): this is the Llama semantics' gradient of
 * the same causal attention (pkg/model/attention.go:113-206).  Uses the
 * context workspace. */
GLC_API int glc_attention_bwd(glc_ctx* ctx, const float* q, const float* k, const float* v, const float* o,
                              const float* lse, const float* dO, float* dq, float* dk, float* dv, int B, int S, int H,
                              int Hkv, int hd, int round_dv);
/* The same attention backward for callers that cannot allocate device memory
 * during a call (no counterpart in the reference): programs whose device
 * memory is wholly reserved by their own allocator or budget, and programs
 * that must not let a call synchronise the device (glc_attention_bwd's
 * workspace is cudaMalloc'ed on first use and regrown after a device sync).
 * Its scratch is a fixed 4 MiB file-scope device array, so B*H*S may not
 * exceed 1,048,576; larger calls fail with GLC_ERR_INVALID.  It calls no
 * cudaMalloc, cudaFree or allocating library routine.  glc_init places the
 * array on its device and looks up its address (cudaGetSymbolAddress) when
 * it creates a context, so every device with a context holds the array from
 * then until the process exits, and this call only reads the cached address.
 * All calls share the array, which keeps the last call's
 * contents (it is fully rewritten before use), so calls that overlap on the
 * GPU — on different streams or contexts of one device — race. */
GLC_API int glc_attention_bwd_noalloc(glc_ctx* ctx, const float* q, const float* k, const float* v, const float* o,
                                      const float* lse, const float* dO, float* dq, float* dk, float* dv, int B,
                                      int S, int H, int Hkv, int hd, int round_dv);
/* SoftmaxCrossEntropyGrad (pkg/tensor/grad.go:210-280): loss (device float)
 * = mean over rows of -log32(p_target + 1e-10); write_grad=1 overwrites the
 * logits with the gradient (p - onehot) * scale. row_logp: [rows] scratch. */
GLC_API int glc_softmax_ce(glc_ctx* ctx, float* logits, const int64_t* targets, int rows, int V, float scale,
                           float* row_logp, float* loss, int write_grad, int round_out);
/* The same loss and gradient in the Llama semantics of the training step
 * (glc_trainer_step on a Llama-mode model, which calls this kernel): expf and
 * logf in place of exp32/log32, p = e * (1 / sum) in place of the division;
 * round_out=1 also rounds the gradient to TF32 for the GEMM that reads it.
 * No reference counterpart (the reference trains with exp32). */
GLC_API int glc_softmax_ce_llama(glc_ctx* ctx, float* logits, const int64_t* targets, int rows, int V, float scale,
                                 float* row_logp, float* loss, int write_grad, int round_out);
/* Embedding lookup of TrainableModel.Forward (trainer.go:275-291):
 * out[t] = E[tok[t]] (+ P[t % S] when P != NULL); ids outside [0,V) read row 0. */
GLC_API int glc_embed_fwd(glc_ctx* ctx, const int64_t* tokens, const float* E, const float* P, float* out, int T,
                          int S, int d, int V);
/* Embedding gradient dE[tok[t]] += dh[t] (t ascending, deterministic);
 * tokens_host are the same ids on the host.  The reference's lookup has no
 * GradFn (trainer.go:290-291): this is the Llama semantics' gradient of it. */
GLC_API int glc_embed_bwd(glc_ctx* ctx, const int64_t* tokens_host, int T, const float* dh, float* dE, int d, int V);
/* The same scatter (the gradient of the lookup at trainer.go:275-291) with the
 * ids in device memory: the positions are sorted
 * by id on the device (stable, so the sums run in ascending t and the result
 * is bit-identical to glc_embed_bwd).  Uses the context workspace. */
GLC_API int glc_embed_bwd_device(glc_ctx* ctx, const int64_t* tokens_dev, int T, const float* dh, float* dE, int d,
                                 int V);
/* GradientClipping (pkg/train/optimizer.go:169-196) over the parameters that
 * have a gradient, given as a host table of nseg {start, len} int64 pairs
 * into the gradient arena (multiples of 4 floats): norm_dev (double) receives
 * the global L2 norm, scale_dev (float) the clip factor (1 when not clipped),
 * both in device memory so AdamW can apply it without a host round trip. */
GLC_API int glc_grad_clip_norm(glc_ctx* ctx, const float* grads, const int64_t* segs_host, int nseg, float max_norm,
                               double* norm_dev, float* scale_dev);
/* AdamW.Step (pkg/train/optimizer.go:37-76) over the same segments: grads are
 * scaled by *clip_scale_dev (when given; the clipped values are written back
 * as the reference's in-place clipping leaves them), moments in float32, the
 * bias-corrected update in float64 rounded to float32, decoupled weight decay;
 * `step` is the optimizer's step count after incrementing.  shadow (nullable)
 * receives the new parameters rounded to TF32 for the GEMMs. */
GLC_API int glc_adamw_step(glc_ctx* ctx, float* params, float* grads, float* m, float* v, float* shadow,
                           const int64_t* segs_host, int nseg, const float* clip_scale_dev, float lr, float beta1,
                           float beta2, float eps, float weight_decay, int step);
GLC_API int glc_fill(glc_ctx* ctx, float* p, float value, size_t n);
GLC_API int glc_round_tf32(glc_ctx* ctx, const float* src, float* dst, size_t n);
/* exp32 (pkg/tensor/grad.go:283-293) elementwise: y[i] = float32(_exp(x[i])),
 * the exact value the reference's softmax cross-entropy and SiLU use, through
 * the same device function those kernels call. */
GLC_API int glc_exp32(glc_ctx* ctx, const float* x, float* y, size_t n);
/* addInplace (pkg/tensor/grad.go:200-204): dst += src. */
GLC_API int glc_add_inplace(glc_ctx* ctx, float* dst, const float* src, size_t n);

/* ------------------------------------------------------------------ model / trainer */
#define GLC_SEMANTICS_REFERENCE 0 /* pkg/train exactly, quirks included */
#define GLC_SEMANTICS_LLAMA 1     /* RoPE, GQA, attention backward, full RMSNorm backward, CE-seeded backward */

typedef struct glc_train_config {
  /* TrainConfig (pkg/train/trainer.go:15-40) */
  int vocab_size;
  int hidden_size;
  int num_layers;
  int num_heads;
  int intermediate_size;
  int max_seq_len;
  int batch_size;
  int block_size;
  float learning_rate;
  float weight_decay;
  int warmup_steps;
  int max_steps;
  float grad_clip_norm;
  /* AdamW hyper-parameters (NewAdamW defaults, pkg/train/optimizer.go:24-34) */
  float beta1;
  float beta2;
  float epsilon;
  /* extensions */
  int num_kv_heads; /* Llama semantics; 0 means num_heads */
  int semantics;    /* GLC_SEMANTICS_* */
  float norm_eps;   /* RMSNormTrainable.Eps, 1e-5 */
  float rope_theta; /* 10000 */
  float init_std;   /* std of the seeded normal weight init */
  uint64_t seed;
  int world_size;   /* data-parallel ranks (1 = single GPU) */
} glc_train_config;

typedef struct glc_model glc_model;
typedef struct glc_trainer glc_trainer;

/* DefaultTrainConfig (pkg/train/trainer.go:43-69) plus the extension defaults. */
GLC_API int glc_default_train_config(glc_train_config* cfg);
/* NewTrainableModel (pkg/train/trainer.go:206-256): parameters in one device
 * arena in Params() order; matrices N(0, init_std) from `seed` (the Go
 * math/rand Xavier init is not reproducible without Go), RMSNorm weights 1. */
GLC_API int glc_model_create(glc_ctx* ctx, const glc_train_config* cfg, glc_model** out);
/* Before its context, and after every trainer created on it (no reference
 * counterpart: Go's collector frees the model). */
GLC_API int glc_model_destroy(glc_model* m);
/* Params() (trainer.go:429-431): count, and per parameter its offset/shape in
 * the flat arena and whether it currently has a gradient (Grad != nil). */
GLC_API int glc_model_num_params(glc_model* m, int* n, int64_t* total_floats);
GLC_API int glc_model_param_info(glc_model* m, int idx, int64_t* offset, int64_t* rows, int64_t* cols,
                                 int* has_grad);
/* Host <-> device copies of the whole arena: the Data slices of Params()
 * (trainer.go:429-431) in order; below, their Grad slices and AdamW's m and v
 * (pkg/train/optimizer.go:37-76). */
GLC_API int glc_model_set_params(glc_model* m, const float* host, int64_t n);
GLC_API int glc_model_get_params(glc_model* m, float* host, int64_t n);
/* After a TrainStep the gradients are returned as GradientClipping
 * (pkg/train/optimizer.go:169-196) leaves them
 * (scaled by the clip factor); the step itself keeps them unscaled on the
 * device and applies the factor here, in place, on the first read. */
GLC_API int glc_model_get_grads(glc_model* m, float* host, int64_t n);
GLC_API int glc_model_get_moments(glc_model* m, float* m_host, float* v_host, int64_t n);
/* NewTrainer (trainer.go:447-459): AdamW with the configured hyper-parameters
 * and the warmup + cosine LRScheduler. */
GLC_API int glc_trainer_create(glc_model* m, glc_trainer** out);
/* Before its model and context (no reference counterpart). */
GLC_API int glc_trainer_destroy(glc_trainer* t);
/* Trainer.TrainStep (trainer.go:462-505): LR, ZeroGrad, forward, loss,
 * backward, (data-parallel gradient allreduce), gradient clipping, AdamW.
 * inputs/targets: host int64 [B*S] (row b = sequence b).  Returns the loss. */
GLC_API int glc_train_step(glc_trainer* t, const int64_t* inputs, const int64_t* targets, int B, int S, float* loss);
/* The same step with token ids already in device memory (no host copies; the
 * embedding gradient's token order is sorted on the device).  The only host
 * synchronisation of a step is the loss readback at its end (trainer.go:488). */
GLC_API int glc_train_step_device(glc_trainer* t, const int64_t* inputs_dev, const int64_t* targets_dev, int B, int S,
                                  float* loss);
/* Global gradient norm before clipping (GradientClipping,
 * pkg/train/optimizer.go:169-196) and the learning rate (LRScheduler.GetLR,
 * :157-166) of the last step. */
GLC_API int glc_trainer_last_stats(glc_trainer* t, double* grad_norm, float* lr, int* step);
/* Kernels launched by the last step (all of them this library's;
 * diagnostics, no reference counterpart). */
GLC_API int glc_trainer_last_launches(glc_trainer* t, uint64_t* n);

/* ------------------------------------------------------------------ checkpoints
 * Trainer.SaveCheckpoint (pkg/train/trainer.go:554-584) writes a text file:
 *   GOLLAMA_CKPT\n step=<step>\n vocab_size=..\n hidden_size=..\n
 *   num_layers=..\n num_heads=..\n intermediate_size=..\n WEIGHTS\n
 * then per parameter in Params() order one line of its float32 values, each
 * printed as Go's fmt %v prints it and followed by one space.  The functions
 * below write that format byte for byte; the reference has no reader, and
 * glc_checkpoint_read reads it back bit for bit (any other plain decimal
 * spelling of a value is read as its nearest float32; dimensions and
 * per-parameter counts are checked against cfg).
 *
 * The text format holds no optimizer state.  glc_state_write/read keep a
 * binary resume file with the parameters, AdamW's m and v, AdamW's step and
 * the LRScheduler's step, the model dimensions and a hash of all of them;
 * reading checks all of them before anything is written to the model.
 *
 * Host buffers only, no context, no device (errors: glc_last_error(NULL)).
 * n = the model's parameter count (glc_model_num_params). */
GLC_API int glc_checkpoint_write(const char* path, int step, const glc_train_config* cfg, const float* params,
                                 int64_t n);
GLC_API int glc_checkpoint_read(const char* path, const glc_train_config* cfg, int* step, float* params, int64_t n);
GLC_API int glc_state_write(const char* path, const glc_train_config* cfg, int step, int adam_step,
                            const float* params, const float* m, const float* v, int64_t n);
GLC_API int glc_state_read(const char* path, const glc_train_config* cfg, int* step, int* adam_step, float* params,
                           float* m, float* v, int64_t n);
/* Trainer.SaveCheckpoint on the device-resident parameters: writes
 * <dir>/checkpoint_<step>.bin (trainer.go:555) in the text format, the path
 * is copied to path_out when it is not NULL.  Waits for the queued steps.
 * With data parallelism every rank holds the same parameters and state: call
 * the save functions on one rank; every rank may load the same state file. */
GLC_API int glc_trainer_save_checkpoint(glc_trainer* t, const char* dir, char* path_out, size_t path_cap);
/* Binary resume of a trainer: parameters, m, v and both step counters (no
 * reference counterpart: the reference reloads no optimizer state). */
GLC_API int glc_trainer_save_state(glc_trainer* t, const char* path);
GLC_API int glc_trainer_load_state(glc_trainer* t, const char* path);

/* ------------------------------------------------------------------ GGUF files
 * gguf.Reader (pkg/gguf/reader.go).  glc_gguf_open maps the file read-only and
 * parses it like Reader.parse (:63-123): magic "GGUF", version 2 or 3, every
 * metadata key/value, every tensor info, and the tensor data start rounded up
 * to `general.alignment` (a uint32 key; 32 otherwise).  Every field read is
 * bounds-checked: a truncated or inconsistent file fails with GLC_ERR_IO.
 * Lookups by name return index -1 when absent (a later duplicate wins, like
 * the reference's maps).  Host-only calls report errors through
 * glc_last_error(NULL). */
typedef struct glc_gguf glc_gguf;
/* Open (reader.go:22-49) and Close (:52-61). */
GLC_API int glc_gguf_open(const char* path, glc_gguf** out);
GLC_API int glc_gguf_close(glc_gguf* g);
/* Header (reader.go:299-301) and the data section's offset. */
GLC_API int glc_gguf_header(glc_gguf* g, uint32_t* version, uint64_t* n_tensors, uint64_t* n_kv,
                            uint64_t* data_offset);
/* Metadata entry i (file order): key, value type (GGUF metadata type codes,
 * pkg/gguf/format.go:20-34), element type and count of an array (-1 and 1
 * otherwise).  Values: element `elem` of an array, or the scalar (elem 0);
 * integers through as_int (signed types) / as_uint (unsigned and bool),
 * floats through as_double (float32 exactly).  Nested arrays expose their
 * type and count only. */
GLC_API int glc_gguf_meta_find(glc_gguf* g, const char* key, int64_t* index);
GLC_API int glc_gguf_meta_key(glc_gguf* g, int64_t i, char* buf, size_t cap, size_t* len);
GLC_API int glc_gguf_meta_type(glc_gguf* g, int64_t i, int* type, int* elem_type, uint64_t* count);
GLC_API int glc_gguf_meta_number(glc_gguf* g, int64_t i, uint64_t elem, int64_t* as_int, uint64_t* as_uint,
                                 double* as_double);
GLC_API int glc_gguf_meta_string(glc_gguf* g, int64_t i, uint64_t elem, char* buf, size_t cap, size_t* len);
/* TensorInfo (format.go:152-186): name, GGML type, dimensions in GGUF order
 * (innermost first; up to dims_cap written), offset inside the data section
 * and SizeBytes (whole blocks of GetTypeInfo, format.go:117-149). */
GLC_API int glc_gguf_tensor_find(glc_gguf* g, const char* name, int64_t* index);
GLC_API int glc_gguf_tensor_info(glc_gguf* g, int64_t i, char* name, size_t name_cap, size_t* name_len, int* type,
                                 int* ndims, uint64_t* dims, int dims_cap, uint64_t* offset, uint64_t* nbytes);
/* GetTensorData (reader.go:407-424): a pointer into the mapping, valid until
 * glc_gguf_close; GLC_ERR_IO if the data extends beyond the file. */
GLC_API int glc_gguf_tensor_data(glc_gguf* g, int64_t i, const void** data, uint64_t* nbytes);
/* The tensor's stored bytes (quantized blocks as they are) to device memory
 * of at least `cap` bytes: the operand glc_linear_bwd_dx_q takes.  No
 * reference counterpart: the reference dequantizes every tensor at load. */
GLC_API int glc_gguf_tensor_upload(glc_ctx* ctx, glc_gguf* g, int64_t i, void* dev, uint64_t cap);
/* loadTensor (pkg/model/transformer.go:285-303) on the device: the stored
 * bytes to the device, then glc_dequantize into dev (n = element count). */
GLC_API int glc_gguf_tensor_load(glc_ctx* ctx, glc_gguf* g, int64_t i, float* dev, int64_t n);

/* ------------------------------------------------------------------ data parallel (NCCL)
 * One process per GPU.  Rank 0 creates the id and shares it (file, store, ...);
 * every rank then calls glc_dp_init.  Gradients are summed with ncclAllReduce
 * (fp32) over NVLink during glc_train_step.  No reference counterpart: the
 * reference trains on one device. */
GLC_API int glc_dp_unique_id(unsigned char id[128]);
GLC_API int glc_dp_init(glc_ctx* ctx, int rank, int world, const unsigned char id[128], int timeout_ms);
GLC_API int glc_dp_allreduce_sum(glc_ctx* ctx, float* buf, size_t n);
GLC_API int glc_dp_allreduce_max_host(glc_ctx* ctx, double* value);
GLC_API int glc_dp_barrier(glc_ctx* ctx);
GLC_API int glc_dp_destroy(glc_ctx* ctx);
/* Gradient buckets of the data-parallel sum for a configuration (host only,
 * no device needed; no reference counterpart): [begin[i], end[i]) in floats
 * of the gradient arena, contiguous and covering it: the front parameters
 * (embedding, plus positions in reference mode), one bucket per layer, and
 * the output norm.  During glc_train_step with world_size > 1, a bucket is
 * summed over the ranks on the context's communication stream as soon as the
 * last GradFn writing it has been enqueued, overlapping the rest of the
 * backward.  *count receives the number of buckets; at most `capacity` are
 * written. */
GLC_API int glc_dp_bucket_plan(const glc_train_config* cfg, int64_t* begin, int64_t* end, int capacity, int* count);
/* Host only (no device; diagnostics, no reference counterpart): the tile
 * lists a grouped CTA-pair GEMM launch of two problems (tiles0 tiles of kb0
 * k-blocks, then tiles1 of kb1) walks on `clusters` SM pairs.  On return
 * *used is 1 and out (capacity >= clusters + 1 + tiles0 + tiles1) holds
 * clusters + 1 list offsets followed by the tile ids, or *used is 0 when the
 * fixed rotation tile = cluster + i * clusters is kept. */
GLC_API int glc_gemm_tile_lists(int tiles0, int kb0, int tiles1, int kb1, int clusters, int* out, int capacity,
                                int* used);

#ifdef __cplusplus
}
#endif

#endif /* GOLLAMA_CUDA_H */
