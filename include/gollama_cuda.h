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

typedef struct glc_ctx glc_ctx;

/* ------------------------------------------------------------------ context
 * Replaces metal.Init / metal_init (pkg/metal/metal.go:184-190, :5-60): opens
 * the device, creates the compute stream, the device error word and resolves
 * cuTensorMapEncodeTiled.  Fails with GLC_ERR_UNSUPPORTED on anything but an
 * sm_100 device. */
GLC_API int glc_init(int device, glc_ctx** out);
/* Replaces metal.Cleanup (pkg/metal/metal.go:193-196). */
GLC_API int glc_destroy(glc_ctx* ctx);
/* Copies the last error message (NUL-terminated, truncated to n). */
GLC_API int glc_last_error(glc_ctx* ctx, char* buf, size_t n);
/* Replaces metal.DeviceName (pkg/metal/metal.go:204-206). */
GLC_API int glc_device_name(glc_ctx* ctx, char* buf, size_t n);
/* Waits for all enqueued work and reports device-side errors. */
GLC_API int glc_sync(glc_ctx* ctx);
/* Number of kernels this library has launched on the context. */
GLC_API int glc_launch_count(glc_ctx* ctx, uint64_t* out);

/* ------------------------------------------------------------------ memory
 * Device-resident storage behind pkg/tensor.Tensor.Data (pkg/tensor/tensor.go:10-14). */
GLC_API int glc_malloc(glc_ctx* ctx, size_t bytes, void** dptr);
GLC_API int glc_free(glc_ctx* ctx, void* dptr);
GLC_API int glc_memcpy_h2d(glc_ctx* ctx, void* dst, const void* src, size_t bytes);
GLC_API int glc_memcpy_d2h(glc_ctx* ctx, void* dst, const void* src, size_t bytes);
GLC_API int glc_memcpy_d2d(glc_ctx* ctx, void* dst, const void* src, size_t bytes);
GLC_API int glc_memset(glc_ctx* ctx, void* dptr, int value, size_t bytes);
/* Page-locked host memory for the asynchronous copies below. */
GLC_API int glc_host_alloc(glc_ctx* ctx, size_t bytes, void** hptr);
GLC_API int glc_host_free(glc_ctx* ctx, void* hptr);
GLC_API int glc_memcpy_h2d_async(glc_ctx* ctx, void* dst, const void* src, size_t bytes);
GLC_API int glc_memcpy_d2h_async(glc_ctx* ctx, void* dst, const void* src, size_t bytes);

/* ------------------------------------------------------------------ timing
 * CUDA events on the context's compute stream. */
GLC_API int glc_timer_start(glc_ctx* ctx);
GLC_API int glc_timer_stop(glc_ctx* ctx, float* ms); /* synchronises on the stop event */

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
/* General strided form of the three above: C[M,N] (+)= A . B^T (+ R) where
 * a_mn/b_mn select MN-major storage (element (i,k) at ptr[k*ld+i]) instead of
 * K-major (ptr[i*ld+k]).  round_out rounds the stored values to TF32. */
GLC_API int glc_gemm_tf32(glc_ctx* ctx, const float* A, int lda, int a_mn, const float* B, int ldb, int b_mn, float* C,
                  int ldc, int M, int N, int K, int accumulate, const float* R, int ldr, int round_out);

#ifdef __cplusplus
}
#endif

#endif /* GOLLAMA_CUDA_H */
