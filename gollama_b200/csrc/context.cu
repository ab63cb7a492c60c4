// Context, memory, timing and the linear-layer entry points of the C ABI.
#include <cstdio>
#include <cstring>

#include "glc_internal.h"

using glc::Context;

static inline Context* C_(glc_ctx* c) { return reinterpret_cast<Context*>(c); }

namespace glc {

int Context::workspace(size_t bytes, void** out) {
  if (bytes > ws_bytes) {
    if (ws) {
      cudaError_t e = cudaStreamSynchronize(stream);
      if (e != cudaSuccess) return fail_cuda(e, "workspace: sync");
      cudaFree(ws);
      ws = nullptr;
      ws_bytes = 0;
    }
    size_t want = bytes < (size_t(1) << 20) ? (size_t(1) << 20) : bytes;
    cudaError_t e = cudaMalloc(&ws, want);
    if (e != cudaSuccess) {
      ws = nullptr;
      return fail(GLC_ERR_NOMEM, std::string("workspace: cudaMalloc failed: ") + cudaGetErrorString(e));
    }
    ws_bytes = want;
  }
  *out = ws;
  return 0;
}

namespace {
__global__ void empty_k_kernel(float* C, int ldc, int M, int N, int accumulate, const float* R, int ldr) {
  GLC_PDL_ENTRY();
  const size_t total = static_cast<size_t>(M) * N;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
    const int r = static_cast<int>(i / N), c = static_cast<int>(i % N);
    float v = accumulate ? C[size_t(r) * ldc + c] : 0.f;
    if (R) v += R[size_t(r) * ldr + c];
    C[size_t(r) * ldc + c] = v;
  }
}
}  // namespace

int gemm_empty_k(Context* ctx, float* C, int ldc, int M, int N, bool accumulate, const float* R, int ldr,
                 cudaStream_t stream) {
  const size_t total = static_cast<size_t>(M) * N;
  glc::launch_pdl(ctx, empty_k_kernel, grid_for(total, 256, ctx->num_sms), 256, 0, stream, C, ldc, M, N, accumulate ? 1 : 0, R, ldr);
  GLC_LAUNCH_CHECK(ctx, "gemm_empty_k");
  return 0;
}

}  // namespace glc

extern "C" {

int glc_init(int device, glc_ctx** out) {
  if (!out) return GLC_ERR_INVALID;
  *out = nullptr;
  int count = 0;
  if (cudaGetDeviceCount(&count) != cudaSuccess || count == 0) return GLC_ERR_UNSUPPORTED;
  if (device < 0 || device >= count) return GLC_ERR_INVALID;
  if (cudaSetDevice(device) != cudaSuccess) return GLC_ERR_CUDA;
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, device) != cudaSuccess) return GLC_ERR_CUDA;
  if (p.major != 10) return GLC_ERR_UNSUPPORTED;  // sm_100a only
  auto* c = new Context();
  c->device = device;
  c->num_sms = p.multiProcessorCount;
  if (cudaStreamCreateWithFlags(&c->stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaStreamCreateWithFlags(&c->comm_stream, cudaStreamNonBlocking) != cudaSuccess ||
      cudaMalloc(&c->d_err, sizeof(int)) != cudaSuccess || cudaMemset(c->d_err, 0, sizeof(int)) != cudaSuccess ||
      cudaMalloc(&c->dyn_ctr, sizeof(int) * Context::kDynCounters) != cudaSuccess ||
      cudaMemset(c->dyn_ctr, 0, sizeof(int) * Context::kDynCounters) != cudaSuccess ||
      cudaEventCreate(&c->timer_start) != cudaSuccess || cudaEventCreate(&c->timer_stop) != cudaSuccess) {
    delete c;
    return GLC_ERR_CUDA;
  }
  void* fn = nullptr;
  cudaDriverEntryPointQueryResult q;
  if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) != cudaSuccess ||
      q != cudaDriverEntryPointSuccess || !fn) {
    delete c;
    return GLC_ERR_UNSUPPORTED;
  }
  c->encode_fn = reinterpret_cast<glc::EncodeTiledFn>(fn);
  if (glc::noalloc_scratch_setup(c) != 0) {
    glc_destroy(reinterpret_cast<glc_ctx*>(c));
    return GLC_ERR_CUDA;
  }
  *out = reinterpret_cast<glc_ctx*>(c);
  return GLC_OK;
}

int glc_destroy(glc_ctx* ctx) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  cudaSetDevice(c->device);
  cudaStreamSynchronize(c->stream);
  cudaStreamSynchronize(c->comm_stream);
  if (c->ws) cudaFree(c->ws);
  if (c->d_err) cudaFree(c->d_err);
  if (c->dyn_ctr) cudaFree(c->dyn_ctr);
  if (c->timer_start) cudaEventDestroy(c->timer_start);
  if (c->timer_stop) cudaEventDestroy(c->timer_stop);
  for (auto& r : c->prof) {
    cudaEventDestroy(r.a);
    cudaEventDestroy(r.b);
  }
  for (auto e : c->event_pool) cudaEventDestroy(e);
  for (auto& s : c->gemm_sched) cudaFree(s.second);
  cudaStreamDestroy(c->stream);
  cudaStreamDestroy(c->comm_stream);
  delete c;
  return GLC_OK;
}

int glc_last_error(glc_ctx* ctx, char* buf, size_t n) {
  if (!buf || n == 0) return GLC_ERR_INVALID;
  const std::string& s = ctx ? C_(ctx)->last_error : glc::host_error();
  size_t k = s.size() < n - 1 ? s.size() : n - 1;
  std::memcpy(buf, s.data(), k);
  buf[k] = 0;
  return GLC_OK;
}

int glc_device_name(glc_ctx* ctx, char* buf, size_t n) {
  if (!ctx || !buf || n == 0) return GLC_ERR_INVALID;
  cudaDeviceProp p;
  if (cudaGetDeviceProperties(&p, C_(ctx)->device) != cudaSuccess) return GLC_ERR_CUDA;
  std::snprintf(buf, n, "%s", p.name);
  return GLC_OK;
}

int glc_sync(glc_ctx* ctx) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return c->fail_cuda(e, "glc_sync(stream)");
  e = cudaStreamSynchronize(c->comm_stream);
  if (e != cudaSuccess) return c->fail_cuda(e, "glc_sync(comm_stream)");
  int err = 0;
  e = cudaMemcpy(&err, c->d_err, sizeof(int), cudaMemcpyDeviceToHost);
  if (e != cudaSuccess) return c->fail_cuda(e, "glc_sync(read error word)");
  if (err != 0) {
    cudaMemset(c->d_err, 0, sizeof(int));
    char msg[128];
    std::snprintf(msg, sizeof msg, "device error %d (a bounded wait in a kernel ran out)", err);
    return c->fail(GLC_ERR_DEVICE, msg);
  }
  return GLC_OK;
}

int glc_launch_count(glc_ctx* ctx, uint64_t* out) {
  if (!ctx || !out) return GLC_ERR_INVALID;
  *out = C_(ctx)->launches;
  return GLC_OK;
}

int glc_malloc(glc_ctx* ctx, size_t bytes, void** dptr) {
  if (!ctx || !dptr) return GLC_ERR_INVALID;
  *dptr = nullptr;
  if (bytes == 0) return GLC_OK;
  cudaError_t e = cudaMalloc(dptr, bytes);
  if (e != cudaSuccess) {
    *dptr = nullptr;
    return C_(ctx)->fail(GLC_ERR_NOMEM, std::string("cudaMalloc: ") + cudaGetErrorString(e));
  }
  return GLC_OK;
}

int glc_free(glc_ctx* ctx, void* dptr) {
  if (!ctx) return GLC_ERR_INVALID;
  if (!dptr) return GLC_OK;
  cudaError_t e = cudaFree(dptr);
  return e == cudaSuccess ? GLC_OK : C_(ctx)->fail_cuda(e, "cudaFree");
}

static int copy_sync(glc_ctx* ctx, void* dst, const void* src, size_t bytes, cudaMemcpyKind k, const char* what) {
  if (!ctx || (bytes && (!dst || !src))) return GLC_ERR_INVALID;
  if (bytes == 0) return GLC_OK;
  Context* c = C_(ctx);
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, k, c->stream);
  if (e == cudaSuccess) e = cudaStreamSynchronize(c->stream);
  return e == cudaSuccess ? GLC_OK : c->fail_cuda(e, what);
}

int glc_memcpy_h2d(glc_ctx* ctx, void* dst, const void* src, size_t bytes) {
  return copy_sync(ctx, dst, src, bytes, cudaMemcpyHostToDevice, "memcpy h2d");
}
int glc_memcpy_d2h(glc_ctx* ctx, void* dst, const void* src, size_t bytes) {
  return copy_sync(ctx, dst, src, bytes, cudaMemcpyDeviceToHost, "memcpy d2h");
}
int glc_memcpy_d2d(glc_ctx* ctx, void* dst, const void* src, size_t bytes) {
  if (!ctx || (bytes && (!dst || !src))) return GLC_ERR_INVALID;
  if (bytes == 0) return GLC_OK;
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, C_(ctx)->stream);
  return e == cudaSuccess ? GLC_OK : C_(ctx)->fail_cuda(e, "memcpy d2d");
}
int glc_memset(glc_ctx* ctx, void* dptr, int value, size_t bytes) {
  if (!ctx || (bytes && !dptr)) return GLC_ERR_INVALID;
  if (bytes == 0) return GLC_OK;
  cudaError_t e = cudaMemsetAsync(dptr, value, bytes, C_(ctx)->stream);
  return e == cudaSuccess ? GLC_OK : C_(ctx)->fail_cuda(e, "memset");
}
int glc_host_alloc(glc_ctx* ctx, size_t bytes, void** hptr) {
  if (!ctx || !hptr) return GLC_ERR_INVALID;
  cudaError_t e = cudaMallocHost(hptr, bytes ? bytes : 1);
  return e == cudaSuccess ? GLC_OK : C_(ctx)->fail_cuda(e, "cudaMallocHost");
}
int glc_host_free(glc_ctx* ctx, void* hptr) {
  if (!ctx) return GLC_ERR_INVALID;
  cudaError_t e = cudaFreeHost(hptr);
  return e == cudaSuccess ? GLC_OK : C_(ctx)->fail_cuda(e, "cudaFreeHost");
}
int glc_memcpy_h2d_async(glc_ctx* ctx, void* dst, const void* src, size_t bytes) {
  if (!ctx || (bytes && (!dst || !src))) return GLC_ERR_INVALID;
  if (bytes == 0) return GLC_OK;
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, C_(ctx)->stream);
  return e == cudaSuccess ? GLC_OK : C_(ctx)->fail_cuda(e, "memcpy h2d async");
}
int glc_memcpy_d2h_async(glc_ctx* ctx, void* dst, const void* src, size_t bytes) {
  if (!ctx || (bytes && (!dst || !src))) return GLC_ERR_INVALID;
  if (bytes == 0) return GLC_OK;
  cudaError_t e = cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, C_(ctx)->stream);
  return e == cudaSuccess ? GLC_OK : C_(ctx)->fail_cuda(e, "memcpy d2h async");
}

int glc_timer_start(glc_ctx* ctx) {
  if (!ctx) return GLC_ERR_INVALID;
  cudaError_t e = cudaEventRecord(C_(ctx)->timer_start, C_(ctx)->stream);
  return e == cudaSuccess ? GLC_OK : C_(ctx)->fail_cuda(e, "timer start");
}
int glc_timer_stop(glc_ctx* ctx, float* ms) {
  if (!ctx || !ms) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  cudaError_t e = cudaEventRecord(c->timer_stop, c->stream);
  if (e == cudaSuccess) e = cudaEventSynchronize(c->timer_stop);
  if (e == cudaSuccess) e = cudaEventElapsedTime(ms, c->timer_start, c->timer_stop);
  return e == cudaSuccess ? GLC_OK : c->fail_cuda(e, "timer stop");
}

int glc_profile_begin(glc_ctx* ctx) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  c->profiling = true;
  return GLC_OK;
}

int glc_profile_end(glc_ctx* ctx, int n_classes, uint64_t* counts, double* total_ms, double* total_work) {
  if (!ctx || n_classes <= 0 || !counts || !total_ms || !total_work) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  c->profiling = false;
  cudaError_t e = cudaStreamSynchronize(c->stream);
  if (e != cudaSuccess) return c->fail_cuda(e, "glc_profile_end");
  for (int i = 0; i < n_classes; ++i) {
    counts[i] = 0;
    total_ms[i] = 0.0;
    total_work[i] = 0.0;
  }
  for (auto& r : c->prof) {
    float ms = 0.f;
    if (cudaEventElapsedTime(&ms, r.a, r.b) == cudaSuccess && r.cls >= 0 && r.cls < n_classes) {
      counts[r.cls] += 1;
      total_ms[r.cls] += ms;
      total_work[r.cls] += r.work;
    }
    c->event_pool.push_back(r.a);
    c->event_pool.push_back(r.b);
  }
  c->prof.clear();
  return GLC_OK;
}

int glc_gemm_tf32(glc_ctx* ctx, const float* A, int lda, int a_mn, const float* B, int ldb, int b_mn, float* C,
                  int ldc, int M, int N, int K, int accumulate, const float* R, int ldr, int round_out) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  return glc::gemm_tf32(c, {A, lda, a_mn != 0}, {B, ldb, b_mn != 0}, C, ldc, M, N, K, accumulate != 0, R, ldr,
                        round_out != 0, c->stream);
}

int glc_set_gemm_variant(glc_ctx* ctx, int variant) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  if (variant < 0 || variant > 2) return c->fail(GLC_ERR_INVALID, "set_gemm_variant: variant must be 0, 1 or 2");
  c->gemm_variant = variant;
  return GLC_OK;
}

int glc_set_fused_swiglu(glc_ctx* ctx, int on) {
  if (!ctx) return GLC_ERR_INVALID;
  C_(ctx)->fuse_swiglu = on != 0;
  return GLC_OK;
}

int glc_set_attention_fwd_variant(glc_ctx* ctx, int variant) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  if (variant < 0 || variant > 2) return c->fail(GLC_ERR_INVALID, "set_attention_fwd_variant: variant must be 0, 1 or 2");
  c->attn_fwd_variant = variant;
  return GLC_OK;
}

int glc_set_gemm_schedule(glc_ctx* ctx, int mode) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  if (mode < 0 || mode > 2) return c->fail(GLC_ERR_INVALID, "set_gemm_schedule: mode must be 0, 1 or 2");
  c->gemm_order = mode;
  return GLC_OK;
}

int glc_set_attention_dq_variant(glc_ctx* ctx, int variant) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  if (variant < 0 || variant > 3) return c->fail(GLC_ERR_INVALID, "set_attention_dq_variant: variant must be 0 to 3");
  c->attn_dq_variant = variant;
  return GLC_OK;
}

int glc_set_attention_dkdv_variant(glc_ctx* ctx, int variant) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  if (variant < 0 || variant > 2) return c->fail(GLC_ERR_INVALID, "set_attention_dkdv_variant: variant must be 0, 1 or 2");
  c->attn_dkdv_variant = variant;
  return GLC_OK;
}

int glc_set_pdl(glc_ctx* ctx, int on) {
  if (!ctx) return GLC_ERR_INVALID;
  C_(ctx)->pdl = on != 0;
  return GLC_OK;
}

int glc_set_tracing(glc_ctx* ctx, int on) {
  if (!ctx) return GLC_ERR_INVALID;
  C_(ctx)->tracing = on != 0;
  return GLC_OK;
}

int glc_set_quant_path(glc_ctx* ctx, int path) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  if (path < 0 || path > 2) return c->fail(GLC_ERR_INVALID, "set_quant_path: path must be 0, 1 or 2");
  c->quant_path = path;
  return GLC_OK;
}

int glc_set_rmsnorm_variant(glc_ctx* ctx, int variant) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  if (variant < 0 || variant > 3) return c->fail(GLC_ERR_INVALID, "set_rmsnorm_variant: variant must be 0 to 3");
  c->rmsnorm_variant = variant;
  return GLC_OK;
}

int glc_set_ce_variant(glc_ctx* ctx, int variant) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  if (variant < 0 || variant > 2) return c->fail(GLC_ERR_INVALID, "set_ce_variant: variant must be 0, 1 or 2");
  c->ce_variant = variant;
  return GLC_OK;
}

int glc_set_attention_split(glc_ctx* ctx, int nsplit) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  if (nsplit < 0 || nsplit > 1024) return c->fail(GLC_ERR_INVALID, "set_attention_split: nsplit must be 0..1024");
  c->attn_split = nsplit;
  return GLC_OK;
}

int glc_linear_fwd(glc_ctx* ctx, const float* X, const float* W, float* Y, int M, int K, int N,
                   const float* residual) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  return glc::gemm_tf32(c, {X, K, false}, {W, K, false}, Y, N, M, N, K, false, residual, N, false, c->stream);
}

int glc_linear_fwd_swiglu(glc_ctx* ctx, const float* X, const float* Wgu, float* GU, float* H, int M, int K, int F,
                          int round_h) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  if (F <= 0) return c->fail(GLC_ERR_INVALID, "linear_fwd_swiglu: F must be positive");
  glc::GemmSpec g{{X, K, false}, {Wgu, K, false}, GU, 2 * F, M, 2 * F, K, false, nullptr, 0, false};
  g.glu = F;
  g.glu_h = H;
  g.ld_glu = F;
  g.glu_round = round_h != 0;
  return glc::gemm_tf32_group(c, &g, 1, c->stream);
}

int glc_linear_bwd_dx(glc_ctx* ctx, const float* dY, const float* W, float* dX, int M, int K, int N,
                      int accumulate) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  // dX[M,K] = dY[M,N] . W[N,K]: GEMM (M, K, reduce N); B(k, n) = W[n*K + k] is MN-major
  return glc::gemm_tf32(c, {dY, N, false}, {W, K, true}, dX, K, M, K, N, accumulate != 0, nullptr, 0, false,
                        c->stream);
}

int glc_linear_bwd(glc_ctx* ctx, const float* dY, const float* X, const float* W, float* dX, float* dW, int M, int K,
                   int N, int accumulate_dx, int accumulate_dw) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  glc::GemmSpec g[2];
  int n = 0;
  if (dX) g[n++] = glc::GemmSpec{{dY, N, false}, {W, K, true}, dX, K, M, K, N, accumulate_dx != 0, nullptr, 0, false};
  if (dW) g[n++] = glc::GemmSpec{{dY, N, true}, {X, K, true}, dW, K, N, K, M, accumulate_dw != 0, nullptr, 0, false};
  if (n == 0) return GLC_OK;
  return glc::gemm_tf32_group(c, g, n, c->stream);
}

int glc_linear_bwd_dw(glc_ctx* ctx, const float* dY, const float* X, float* dW, int M, int K, int N,
                      int accumulate) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = C_(ctx);
  // dW[N,K] = dY[M,N]^T . X[M,K]: GEMM (N, K, reduce M); A(n, m) = dY[m*N + n], B(k, m) = X[m*K + k]
  return glc::gemm_tf32(c, {dY, N, true}, {X, K, true}, dW, K, N, K, M, accumulate != 0, nullptr, 0, false,
                        c->stream);
}

}  // extern "C"
