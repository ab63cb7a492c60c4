// The reference's own float32 exp/log (pkg/tensor/grad.go:283-381), evaluated
// on the device with the same float64 operation sequence.  Explicit _rn
// intrinsics keep nvcc from contracting multiply-adds into FMAs, so results
// match the Go code (which does not fuse on amd64) bit for bit.
#pragma once
#include <cuda_runtime.h>

namespace glc {

// _exp (grad.go:310-352).  The repeated doubling/halving by 2^k is exact for
// every argument exp32 passes in (|x| <= 88 gives |k| <= 127), so ldexp gives
// the identical value.
__device__ __forceinline__ double go_exp(double x) {
  const double Ln2Hi = 6.93147180369123816490e-01;
  const double Ln2Lo = 1.90821492927058770002e-10;
  const double Log2e = 1.44269504088896338700e+00;
  if (x > 7.09782712893383973096e+02) return 1.7976931348623157e+308;
  if (x < -7.45133219101941108420e+02) return 0.0;
  int k = static_cast<int>(__dadd_rn(__dmul_rn(x, Log2e), 0.5));
  if (x < 0) k = static_cast<int>(__dsub_rn(__dmul_rn(x, Log2e), 0.5));
  const double dk = static_cast<double>(k);
  const double r = __dsub_rn(__dsub_rn(x, __dmul_rn(dk, Ln2Hi)), __dmul_rn(dk, Ln2Lo));
  const double r2 = __dmul_rn(r, r);
  double t = __dadd_rn(0.0027777777777015593, __dmul_rn(r2, 6.613756321437934e-05));
  t = __dadd_rn(0.16666666666666602, __dmul_rn(r2, t));
  const double p = __dsub_rn(r, __dmul_rn(r2, t));
  const double q = __ddiv_rn(__dmul_rn(r, p), __dsub_rn(p, 2.0));
  const double result = __dsub_rn(1.0, __dsub_rn(q, r));
  return ldexp(result, k);
}

// exp32 (grad.go:283-293)
__device__ __forceinline__ float go_exp32(float x) {
  if (x < -88.f) return 0.f;
  if (x > 88.f) return 3.4e38f;
  return __double2float_rn(go_exp(static_cast<double>(x)));
}

// exp32 with the identical float result at lower cost.  The reference's
// _exp above divides once in double (q = r*p / (p - 2)); here the quotient
// uses the hardware reciprocal estimate refined by two Newton-Raphson steps
// (relative error near the double rounding unit), every other operation is
// the reference's, so the double result differs from _exp's by a few units
// in the last place (q is under 0.06 of the result).  Both round to the same
// float unless the value lies within 2^-40 (relative) of a float rounding
// midpoint; that case, and arguments outside [-87, 88] (subnormal or
// saturated results, NaN), take the exact restatement.
__device__ __forceinline__ float go_exp32_fast(float xf) {
  if (!(xf >= -87.f && xf <= 88.f)) return go_exp32(xf);
  const double Ln2Hi = 6.93147180369123816490e-01;
  const double Ln2Lo = 1.90821492927058770002e-10;
  const double Log2e = 1.44269504088896338700e+00;
  const double x = static_cast<double>(xf);
  int k = static_cast<int>(__dadd_rn(__dmul_rn(x, Log2e), 0.5));
  if (x < 0) k = static_cast<int>(__dsub_rn(__dmul_rn(x, Log2e), 0.5));
  const double dk = static_cast<double>(k);
  const double r = __dsub_rn(__dsub_rn(x, __dmul_rn(dk, Ln2Hi)), __dmul_rn(dk, Ln2Lo));
  const double r2 = __dmul_rn(r, r);
  double t = __dadd_rn(0.0027777777777015593, __dmul_rn(r2, 6.613756321437934e-05));
  t = __dadd_rn(0.16666666666666602, __dmul_rn(r2, t));
  const double p = __dsub_rn(r, __dmul_rn(r2, t));
  const double den = __dsub_rn(p, 2.0);
  double y;
  asm("rcp.approx.ftz.f64 %0, %1;" : "=d"(y) : "d"(den));
  y = fma(y, fma(-den, y, 1.0), y);  // Newton-Raphson for 1/den
  y = fma(y, fma(-den, y, 1.0), y);
  const double q = __dmul_rn(r, p) * y;
  const double res = __dsub_rn(1.0, __dsub_rn(q, r));
  const double v = res * __longlong_as_double(static_cast<long long>(k + 1023) << 52);  // k in [-126, 127]
  const float vf = __double2float_rn(v);
  const uint32_t bits = __float_as_uint(vf);
  const int e = static_cast<int>((bits >> 23) & 0xFFu) - 127;
  if (e < -126) return go_exp32(xf);  // not a normal float: exact path
  const double half_up = __longlong_as_double(static_cast<long long>(e - 24 + 1023) << 52);
  const double half_dn = (bits & 0x7FFFFFu) ? half_up : 0.5 * half_up;  // below a power of two the spacing halves
  const double d = v - static_cast<double>(vf);  // exact (Sterbenz)
  const double tol = v * 9.094947017729282e-13;  // 2^-40 relative
  if (d > half_up - tol || -d > half_dn - tol) return go_exp32(xf);
  return vf;
}

// _log (grad.go:354-381).  The halving/doubling loops that bring x into
// [1, 2) are exact, so frexp gives the same mantissa and exponent.
__device__ __forceinline__ double go_log(double x) {
  if (x <= 0) return -1e100;
  int e;
  double m = frexp(x, &e);  // x = m * 2^e, m in [0.5, 1)
  m = __dmul_rn(m, 2.0);    // [1, 2)
  const int k = e - 1;
  const double f = __dsub_rn(m, 1.0);
  const double s = __ddiv_rn(f, __dadd_rn(2.0, f));
  const double s2 = __dmul_rn(s, s);
  const double s4 = __dmul_rn(s2, s2);
  const double t1 =
      __dmul_rn(s2, __dadd_rn(0.6666666666666735,
                              __dmul_rn(s4, __dadd_rn(0.2857142874366239, __dmul_rn(s4, 0.1818357216161805)))));
  const double t2 = __dmul_rn(s4, __dadd_rn(0.3999999999940942, __dmul_rn(s4, 0.22222198432149784)));
  const double R = __dadd_rn(t1, t2);
  return __dsub_rn(__dadd_rn(__dmul_rn(static_cast<double>(k), 0.6931471805599453), f), __dmul_rn(s, __dsub_rn(f, R)));
}

__device__ __forceinline__ float go_log32(float x) { return __double2float_rn(go_log(static_cast<double>(x))); }

// Sigmoid of SiLUGrad (grad.go:426): 1 / (1 + exp32(-v)) in float32.
__device__ __forceinline__ float go_sigmoid(float v) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, go_exp32_fast(-v))); }

// SwiGLU product h = silu(g) * u: SiLUGrad's forward (grad.go:426-427, x*s)
// then the product node (trainer.go:400-422), float32 operations in order.
__device__ __forceinline__ float go_swiglu(float g, float u) {
  const float s = go_sigmoid(g);
  return __fmul_rn(__fmul_rn(g, s), u);
}

// FAST: Llama semantics, the sigmoid with float expf instead of the
// reference's float64 exp32 (the decoder package takes math.Exp); the same
// float32 operation order otherwise.  Shared by the SwiGLU kernels and the
// GEMM's SwiGLU epilogue, which must agree bit for bit.
template <bool FAST>
__device__ __forceinline__ float sigmoid_f(float g) {
  return FAST ? __fdiv_rn(1.0f, __fadd_rn(1.0f, expf(-g))) : go_sigmoid(g);
}
template <bool FAST>
__device__ __forceinline__ float swiglu_f(float g, float u) {
  return FAST ? __fmul_rn(__fmul_rn(g, sigmoid_f<true>(g)), u) : go_swiglu(g, u);
}

}  // namespace glc
