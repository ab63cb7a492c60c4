// Frozen quantized weights (pkg/quant/dequant.go): dequantization and the
// input gradient of a linear layer whose weight is stored quantized.
//
// Every format the reference's Dequantize accepts (dequant.go:367-393): F32,
// F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K and Q6_K, decoded by
// quant_formats.cuh four elements per thread with the reference's float32
// arithmetic (bit-exact).  Weights W [out][in] are stored as the flat
// sequence of blocks the GGUF file holds (pkg/model/transformer.go:285-303).
//
// glc_linear_bwd_dx_q computes dX (+)= dY . deq(W) (MatMulGrad's dA,
// pkg/tensor/grad.go:102-116, on the dequantized weight): one pass writes the
// TF32-rounded weight into the context workspace (the quantized bytes are
// read once, 0.53 to 1.06 B per element), then the tcgen05 GEMM runs with
// the weight as its MN-major B operand; with glc_set_quant_path(ctx, 2) the
// GEMM decodes the stored blocks itself (gemm_quant_fused.cu).
#include "glc_internal.h"
#include "quant_formats.cuh"
#include "sm100.cuh"

namespace glc {
namespace {

// One thread per 4 consecutive outputs (n4 = n / 4 groups); round: TF32 RN.
__global__ void dequant_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst, size_t n4, int type,
                               int round) {
  GLC_PDL_ENTRY();
  for (size_t g = blockIdx.x * size_t(blockDim.x) + threadIdx.x; g < n4; g += size_t(gridDim.x) * blockDim.x) {
    float v[4];
    qf::dequant4(src, type, g, v);
    if (round) {
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = round_tf32(v[i]);
    }
    reinterpret_cast<float4*>(dst)[g] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

size_t quant_bytes(int type, size_t n) {
  const int be = qf::block_elems(type);
  return be ? n / static_cast<size_t>(be) * static_cast<size_t>(qf::block_bytes(type)) : 0;
}

int check_type(Context* ctx, int type, size_t n, const char* what) {
  const int be = qf::block_elems(type);
  if (be == 0)
    return ctx->fail(GLC_ERR_UNSUPPORTED,
                     std::string(what) + ": weight type must be F32, F16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0, Q4_K or Q6_K");
  if (n % static_cast<size_t>(be))
    return ctx->fail(GLC_ERR_INVALID, std::string(what) + ": the element count must be a whole number of blocks (" +
                                          std::to_string(be) + " elements)");
  if (n % 4) return ctx->fail(GLC_ERR_INVALID, std::string(what) + ": element count must be a multiple of 4");
  return 0;
}

int dequant(Context* ctx, int type, const void* src, float* dst, size_t n, bool round, cudaStream_t s) {
  if (n == 0) return 0;
  int rc = check_type(ctx, type, n, "dequantize");
  if (rc) return rc;
  if (!src || !dst || (reinterpret_cast<uintptr_t>(src) & 1) || (reinterpret_cast<uintptr_t>(dst) & 15))
    return ctx->fail(GLC_ERR_INVALID, "dequantize: source must be 2-byte and destination 16-byte aligned");
  ProfScope prof(ctx, PROF_OTHER, static_cast<double>(quant_bytes(type, n) + 4 * n), s);
  glc::launch_pdl(ctx, dequant_kernel, grid_for(n / 4, 256, ctx->num_sms), 256, 0, s, static_cast<const uint8_t*>(src), dst, n / 4,
                  type, round ? 1 : 0);
  GLC_LAUNCH_CHECK(ctx, "dequantize");
  return 0;
}

}  // namespace
}  // namespace glc

using glc::Context;

extern "C" {

int glc_dequantize(glc_ctx* ctx, int type, const void* src, float* dst, size_t n) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = reinterpret_cast<Context*>(ctx);
  return glc::dequant(c, type, src, dst, n, false, c->stream);
}

int glc_linear_bwd_dx_q(glc_ctx* ctx, const float* dY, const void* Wq, int type, float* dX, int M, int K, int N,
                        int accumulate) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = reinterpret_cast<Context*>(ctx);
  if (M < 0 || K <= 0 || N < 0) return c->fail(GLC_ERR_INVALID, "linear_bwd_dx_q: bad size");
  if (M == 0 || N == 0) return glc::gemm_tf32(c, {dY, N, false}, {nullptr, K, true}, dX, K, M, K, N, accumulate != 0,
                                              nullptr, 0, false, c->stream);
  if (c->quant_path == 2 && type != GLC_QTYPE_F32 && glc::quant_fused_supported(type, K))
    return glc::gemm_quant_fused(c, dY, N, Wq, type, dX, K, M, K, N, accumulate != 0, c->stream);
  const size_t n = static_cast<size_t>(N) * K;
  void* ws = nullptr;
  int rc = c->workspace(n * sizeof(float), &ws);
  if (rc) return rc;
  float* w = static_cast<float*>(ws);
  rc = glc::dequant(c, type, Wq, w, n, true, c->stream);
  if (rc) return rc;
  // dX[M,K] = dY[M,N] . W[N,K]: GEMM (M, K, reduce N); B(k, n) = W[n*K + k] is MN-major
  return glc::gemm_tf32(c, {dY, N, false}, {w, K, true}, dX, K, M, K, N, accumulate != 0, nullptr, 0, false,
                        c->stream);
}

}  // extern "C"
