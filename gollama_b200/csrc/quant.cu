// Frozen quantized weights (pkg/quant/dequant.go): dequantization and the
// input gradient of a linear layer whose weight is stored quantized.
//
// Formats (GGUF type codes, pkg/gguf/format.go:40-46), rows of W [out][in]
// stored as consecutive quantized rows of `in` elements:
//   F32  (0)  4 bytes per element
//   F16  (1)  2 bytes per element, widened exactly (fp16ToFp32, dequant.go:9-41)
//   Q4_0 (2)  blocks of 32 elements, 18 bytes: fp16 scale, then 16 bytes whose
//             low nibble is element 2i and high nibble element 2i+1, each
//             minus 8 (dequant.go:99-119)
//   Q8_0 (8)  blocks of 32 elements, 34 bytes: fp16 scale, then 32 int8 codes
//             (dequant.go:68-85)
// w = float32(scale) * float32(code), exact in fp32 like the reference.
//
// glc_linear_bwd_dx_q computes dX (+)= dY . deq(W) (MatMulGrad's dA,
// pkg/tensor/grad.go:102-116, on the dequantized weight): one pass writes the
// TF32-rounded weight into the context workspace (the quantized bytes are
// read once, 0.53 or 1.06 B per element), then the tcgen05 GEMM runs with
// the weight as its MN-major B operand.
#include "glc_internal.h"
#include "sm100.cuh"

namespace glc {
namespace {

// fp16ToFp32 in integer operations: subnormal halves are normalised exactly
// like the reference's shift loop; NaN payloads are kept (mantissa << 13).
__device__ __forceinline__ float half_bits_to_float(uint32_t h) {
  const uint32_t sign = (h >> 15) & 1u, e = (h >> 10) & 0x1fu;
  uint32_t m = h & 0x3ffu, bits;
  if (e == 0) {
    if (m == 0) {
      bits = sign << 31;
    } else {
      const int s = __clz(m) - 21;  // shifts until bit 10 is set
      m = (m << s) & 0x3ffu;
      bits = (sign << 31) | (static_cast<uint32_t>(1 - s + 127 - 15) << 23) | (m << 13);
    }
  } else if (e == 31) {
    bits = (sign << 31) | 0x7f800000u | (m << 13);
  } else {
    bits = (sign << 31) | ((e + 127 - 15) << 23) | (m << 13);
  }
  return __uint_as_float(bits);
}

__device__ __forceinline__ uint32_t ld_u16(const uint8_t* p) {
  return static_cast<uint32_t>(*reinterpret_cast<const uint16_t*>(p));  // 2-byte aligned in every format
}

// One thread per 4 consecutive outputs (n4 = n / 4 groups); round: TF32 RN.
__global__ void dequant_kernel(const uint8_t* __restrict__ src, float* __restrict__ dst, size_t n4, int type,
                               int round) {
  for (size_t g = blockIdx.x * size_t(blockDim.x) + threadIdx.x; g < n4; g += size_t(gridDim.x) * blockDim.x) {
    float v[4];
    if (type == GLC_QTYPE_F32) {
      const uint8_t* p = src + 16 * g;
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = __uint_as_float(ld_u16(p + 4 * i) | (ld_u16(p + 4 * i + 2) << 16));
    } else if (type == GLC_QTYPE_F16) {
      const uint8_t* p = src + 8 * g;
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = half_bits_to_float(ld_u16(p + 2 * i));
    } else if (type == GLC_QTYPE_Q8_0) {
      const size_t blk = g >> 3;  // 8 groups of 4 per 32-element block
      const int j = static_cast<int>(g & 7) * 4;
      const uint8_t* b = src + 34 * blk;
      const float scale = half_bits_to_float(ld_u16(b));
      const uint32_t lo = ld_u16(b + 2 + j), hi = ld_u16(b + 4 + j);
      const uint32_t q = lo | (hi << 16);
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = scale * static_cast<float>(static_cast<int8_t>((q >> (8 * i)) & 0xffu));
    } else {  // Q4_0
      const size_t blk = g >> 3;
      const int j = static_cast<int>(g & 7) * 4;  // elements j..j+3 = bytes j/2, j/2+1
      const uint8_t* b = src + 18 * blk;
      const float scale = half_bits_to_float(ld_u16(b));
      const uint32_t q = ld_u16(b + 2 + j / 2);
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const uint32_t byte = (q >> (8 * (i >> 1))) & 0xffu;
        const int code = static_cast<int>((i & 1) ? (byte >> 4) : (byte & 0x0fu)) - 8;
        v[i] = scale * static_cast<float>(code);
      }
    }
    if (round) {
#pragma unroll
      for (int i = 0; i < 4; ++i) v[i] = round_tf32(v[i]);
    }
    reinterpret_cast<float4*>(dst)[g] = make_float4(v[0], v[1], v[2], v[3]);
  }
}

size_t quant_bytes(int type, size_t n) {
  switch (type) {
    case GLC_QTYPE_F32: return 4 * n;
    case GLC_QTYPE_F16: return 2 * n;
    case GLC_QTYPE_Q4_0: return n / 32 * 18;
    case GLC_QTYPE_Q8_0: return n / 32 * 34;
    default: return 0;
  }
}

int check_type(Context* ctx, int type, size_t n, const char* what) {
  if (type != GLC_QTYPE_F32 && type != GLC_QTYPE_F16 && type != GLC_QTYPE_Q4_0 && type != GLC_QTYPE_Q8_0)
    return ctx->fail(GLC_ERR_UNSUPPORTED, std::string(what) + ": weight type must be F32, F16, Q4_0 or Q8_0");
  if ((type == GLC_QTYPE_Q4_0 || type == GLC_QTYPE_Q8_0) && (n % 32))
    return ctx->fail(GLC_ERR_INVALID, std::string(what) + ": block formats need a multiple of 32 elements");
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
  dequant_kernel<<<grid_for(n / 4, 256, ctx->num_sms), 256, 0, s>>>(static_cast<const uint8_t*>(src), dst, n / 4,
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
