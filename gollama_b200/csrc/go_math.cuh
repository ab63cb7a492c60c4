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
__device__ __forceinline__ float go_sigmoid(float v) { return __fdiv_rn(1.0f, __fadd_rn(1.0f, go_exp32(-v))); }

}  // namespace glc
