// GradientClipping (pkg/train/optimizer.go:169-196) and AdamW.Step
// (optimizer.go:37-76) over the flat parameter arena.
//
// Parameters, gradients and the AdamW moments live in four arenas with the
// same layout (Params() order), so a "multi-tensor" kernel is a loop over a
// table of contiguous segments: the parameters that have a gradient.
//
// grad_norm: sum of g*g in float64 per block (grid = blocks x segments), then
// one block adds the partials in a fixed order and derives, on the device,
// norm = sqrt(total) and the clip scale float32(max/norm) when
// float32(norm) > max (else 1).
//
// adamw: g *= scale (written back: the reference leaves clipped gradients in
// Grad), m = b1*m + (1-b1)*g, v = b2*v + ((1-b2)*g)*g in float32, the
// bias-corrected update in float64 rounded to float32, p -= lr*(update +
// wd*p) in float32 — the same operation sequence as the reference, without
// FMA contraction — and a TF32-rounded copy of p for the GEMMs.
#include <cmath>

#include "glc_internal.h"
#include "sm100.cuh"

namespace glc {
namespace {

struct Seg {
  int64_t start;
  int64_t len;
};

__global__ void sumsq_kernel(const float* __restrict__ g, const Seg* __restrict__ segs, double* __restrict__ partial) {
  const Seg sg = segs[blockIdx.y];
  double acc = 0.0;
  const float* base = g + sg.start;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < sg.len; i += int64_t(gridDim.x) * blockDim.x) {
    const double v = static_cast<double>(base[i]);
    acc = __dadd_rn(acc, __dmul_rn(v, v));
  }
  __shared__ double red[32];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (blockDim.x >> 5); ++w) t += red[w];
    partial[blockIdx.y * gridDim.x + blockIdx.x] = t;
  }
}

__global__ void norm_finish_kernel(const double* __restrict__ partial, int n, float max_norm, double* __restrict__ norm,
                                   float* __restrict__ scale) {
  __shared__ double red[32];
  double acc = 0.0;
  for (int i = threadIdx.x; i < n; i += blockDim.x) acc += partial[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (blockDim.x >> 5); ++w) t += red[w];
    const double nrm = sqrt(t);
    *norm = nrm;
    float sc = 1.0f;
    if (max_norm > 0.f && __double2float_rn(nrm) > max_norm) sc = __double2float_rn(static_cast<double>(max_norm) / nrm);
    *scale = sc;
  }
}

struct AdamArgs {
  float lr, b1, omb1, b2, omb2, wd;
  double bc1, bc2, eps;
};

__global__ void adamw_kernel(float* __restrict__ p, float* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
                             float* __restrict__ shadow, const Seg* __restrict__ segs,
                             const float* __restrict__ clip_scale, AdamArgs a) {
  const Seg sg = segs[blockIdx.y];
  const float scale = clip_scale ? *clip_scale : 1.0f;
  const bool scaled = scale != 1.0f;
  for (int64_t i = sg.start + blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < sg.start + sg.len;
       i += int64_t(gridDim.x) * blockDim.x) {
    float gi = g[i];
    if (scaled) {
      gi = __fmul_rn(gi, scale);
      g[i] = gi;
    }
    const float mi = __fadd_rn(__fmul_rn(a.b1, m[i]), __fmul_rn(a.omb1, gi));
    const float vi = __fadd_rn(__fmul_rn(a.b2, v[i]), __fmul_rn(__fmul_rn(a.omb2, gi), gi));
    m[i] = mi;
    v[i] = vi;
    const double mhat = __ddiv_rn(static_cast<double>(mi), a.bc1);
    const double vhat = __ddiv_rn(static_cast<double>(vi), a.bc2);
    const float upd = __double2float_rn(__ddiv_rn(mhat, __dadd_rn(__dsqrt_rn(vhat), a.eps)));
    const float pi = p[i];
    const float np = __fsub_rn(pi, __fmul_rn(a.lr, __fadd_rn(upd, __fmul_rn(a.wd, pi))));
    p[i] = np;
    if (shadow) shadow[i] = round_tf32(np);
  }
}

}  // namespace

// segs: device array of {start, len} pairs (int64), nseg entries.
int grad_norm(Context* ctx, const float* grads, const int64_t* segs, int nseg, float max_norm, double* norm_out,
              float* scale_out, double* scratch, int scratch_count, double elems, cudaStream_t s) {
  if (nseg <= 0 || !grads || !segs || !norm_out || !scale_out)
    return ctx->fail(GLC_ERR_INVALID, "grad_norm: bad arguments");
  int bx = (2 * ctx->num_sms + nseg - 1) / nseg;
  if (bx < 1) bx = 1;
  if (bx > 64) bx = 64;
  const int n = bx * nseg;
  double* partial = scratch;
  if (!partial) {
    void* ws = nullptr;
    int rc = ctx->workspace(sizeof(double) * n, &ws);
    if (rc) return rc;
    partial = static_cast<double*>(ws);
  } else if (scratch_count < n) {
    return ctx->fail(GLC_ERR_INVALID, "grad_norm: scratch buffer too small");
  }
  ProfScope prof(ctx, PROF_ADAMW, 4.0 * elems, s);
  sumsq_kernel<<<dim3(bx, nseg), 256, 0, s>>>(grads, reinterpret_cast<const Seg*>(segs), partial);
  GLC_LAUNCH_CHECK(ctx, "grad_norm partial");
  norm_finish_kernel<<<1, 256, 0, s>>>(partial, n, max_norm, norm_out, scale_out);
  GLC_LAUNCH_CHECK(ctx, "grad_norm finish");
  return 0;
}

int adamw(Context* ctx, float* p, float* g, float* m, float* v, float* shadow, const int64_t* segs, int nseg,
          const float* clip_scale, float lr, float beta1, float beta2, float eps, float wd, int step, double elems,
          cudaStream_t s) {
  if (nseg <= 0) return 0;
  if (!p || !g || !m || !v || !segs || step <= 0) return ctx->fail(GLC_ERR_INVALID, "adamw: bad arguments");
  AdamArgs a;
  a.lr = lr;
  a.b1 = beta1;
  a.omb1 = 1.0f - beta1;
  a.b2 = beta2;
  a.omb2 = 1.0f - beta2;
  a.wd = wd;
  a.bc1 = 1.0 - std::pow(static_cast<double>(beta1), static_cast<double>(step));
  a.bc2 = 1.0 - std::pow(static_cast<double>(beta2), static_cast<double>(step));
  a.eps = static_cast<double>(eps);
  int bx = (8 * ctx->num_sms + nseg - 1) / nseg;
  if (bx < 1) bx = 1;
  if (bx > 1024) bx = 1024;
  // p, g, m, v read; p, m, v and the TF32 shadow written
  ProfScope prof(ctx, PROF_ADAMW, (shadow ? 32.0 : 28.0) * elems, s);
  adamw_kernel<<<dim3(bx, nseg), 256, 0, s>>>(p, g, m, v, shadow, reinterpret_cast<const Seg*>(segs), clip_scale, a);
  GLC_LAUNCH_CHECK(ctx, "adamw");
  return 0;
}

}  // namespace glc
