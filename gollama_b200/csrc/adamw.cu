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

#include <math_constants.h>

#include "glc_internal.h"
#include "sm100.cuh"

namespace glc {
namespace {

struct Seg {
  int64_t start;
  int64_t len;
};

__global__ void sumsq_kernel(const float* __restrict__ g, const Seg* __restrict__ segs, double* __restrict__ partial) {
  GLC_PDL_ENTRY();
  const Seg sg = segs[blockIdx.y];
  double acc = 0.0;
  const float4* base = reinterpret_cast<const float4*>(g + sg.start);
  const int64_t n4 = sg.len >> 2;
  for (int64_t i = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i < n4; i += int64_t(gridDim.x) * blockDim.x) {
    const float4 v = base[i];
    const double x = v.x, y = v.y, z = v.z, w = v.w;
    acc = __dadd_rn(acc, __dadd_rn(__dadd_rn(__dmul_rn(x, x), __dmul_rn(y, y)), __dadd_rn(__dmul_rn(z, z), __dmul_rn(w, w))));
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

// Sums of squares of `nchunks` chunks {start, len}, one block per chunk at a
// time (blocks stride over the chunks): out[c] is chunk c's float64 sum, the
// same bits whichever block computes it.  A small grid keeps the pass beside
// other work (the gradient allreduce's stream) from taking the whole GPU.
__global__ void sumsq_chunks_kernel(const float* __restrict__ g, const Seg* __restrict__ chunks, int nchunks,
                                    double* __restrict__ out) {
  GLC_PDL_ENTRY();
  __shared__ double red[32];
  // Few blocks run this beside the backward, so each thread keeps eight
  // independent float4 loads in flight (one at a time left a block at a few
  // GB/s, far below what one SM can pull).
  constexpr int U = 8;
  auto sq4 = [](const float4 v) {
    const double x = v.x, y = v.y, z = v.z, w = v.w;
    return __dadd_rn(__dadd_rn(__dmul_rn(x, x), __dmul_rn(y, y)), __dadd_rn(__dmul_rn(z, z), __dmul_rn(w, w)));
  };
  for (int c = blockIdx.x; c < nchunks; c += gridDim.x) {
    const Seg sg = chunks[c];
    double acc = 0.0, acc2 = 0.0;
    const float4* base = reinterpret_cast<const float4*>(g + sg.start);
    const int64_t n4 = sg.len >> 2;
    const int64_t step = static_cast<int64_t>(blockDim.x) * U;
    int64_t i = threadIdx.x;
    for (; i + (U - 1) * static_cast<int64_t>(blockDim.x) < n4; i += step) {
      float4 v[U];
#pragma unroll
      for (int u = 0; u < U; ++u) v[u] = base[i + u * static_cast<int64_t>(blockDim.x)];
#pragma unroll
      for (int u = 0; u < U; u += 2) {
        acc = __dadd_rn(acc, sq4(v[u]));
        acc2 = __dadd_rn(acc2, sq4(v[u + 1]));
      }
    }
    for (; i < n4; i += blockDim.x) acc = __dadd_rn(acc, sq4(base[i]));
    acc = __dadd_rn(acc, acc2);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
    __syncthreads();
    if (threadIdx.x == 0) {
      double t = 0.0;
      for (int w = 0; w < (blockDim.x >> 5); ++w) t += red[w];
      out[c] = t;
    }
    __syncthreads();
  }
}

__global__ void norm_finish_kernel(const double* __restrict__ partial, int n, float max_norm, double* __restrict__ norm,
                                   float* __restrict__ scale) {
  GLC_PDL_ENTRY();
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

// First level of the finishing sum when the partials are many: block b adds
// partial[b*chunk, min(n, (b+1)*chunk)) in a fixed order into out[b].
__global__ void slot_sum_kernel(const double* __restrict__ partial, long long n, long long chunk,
                                double* __restrict__ out) {
  GLC_PDL_ENTRY();
  __shared__ double red[32];
  const long long b0 = static_cast<long long>(blockIdx.x) * chunk;
  const long long b1 = min(n, b0 + chunk);
  double acc = 0.0;
  for (long long i = b0 + threadIdx.x; i < b1; i += blockDim.x) acc += partial[i];
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) acc += __shfl_xor_sync(0xffffffffu, acc, o);
  if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = acc;
  __syncthreads();
  if (threadIdx.x == 0) {
    double t = 0.0;
    for (int w = 0; w < (blockDim.x >> 5); ++w) t += red[w];
    out[blockIdx.x] = t;
  }
}

struct AdamArgs {
  float lr, b1, omb1, b2, omb2, wd;
  double bc1, bc2, rbc1, rbc2, eps;
};

// float32(mhat / (sqrt(vhat) + eps)) with mhat = m/bc1, vhat = v/bc2 in
// float64 (optimizer.go:68-72).  Fast path: the two bias corrections as
// multiplications by precomputed reciprocals, within a few float64 ulps of
// the reference's quotient; its float32 rounding equals the reference's
// unless the quotient lies within 32 ulps of a float32 rounding midpoint, in
// which case the reference's exact division chain is evaluated instead.
__device__ __forceinline__ float adam_update(float mi, float vi, const AdamArgs& a) {
  const double mh = __dmul_rn(static_cast<double>(mi), a.rbc1);
  const double vh = __dmul_rn(static_cast<double>(vi), a.rbc2);
  const double q = __ddiv_rn(mh, __dadd_rn(__dsqrt_rn(vh), a.eps));
  const float f = __double2float_rn(q);
  const double fd = static_cast<double>(f);
  const double mid_up = 0.5 * (fd + static_cast<double>(nextafterf(f, INFINITY)));
  const double mid_dn = 0.5 * (fd + static_cast<double>(nextafterf(f, -INFINITY)));
  const double tol = 32.0 * 1.1102230246251565e-16 * fabs(q);
  if (fabs(q - mid_up) > tol && fabs(q - mid_dn) > tol) return f;
  const double mhat = __ddiv_rn(static_cast<double>(mi), a.bc1);
  const double vhat = __ddiv_rn(static_cast<double>(vi), a.bc2);
  return __double2float_rn(__ddiv_rn(mhat, __dadd_rn(__dsqrt_rn(vhat), a.eps)));
}

__device__ __forceinline__ void adam_elem(float& p, float& g, float& m, float& v, float scale, bool scaled,
                                          const AdamArgs& a) {
  if (scaled) g = __fmul_rn(g, scale);
  m = __fadd_rn(__fmul_rn(a.b1, m), __fmul_rn(a.omb1, g));
  v = __fadd_rn(__fmul_rn(a.b2, v), __fmul_rn(__fmul_rn(a.omb2, g), g));
  const float upd = adam_update(m, v, a);
  p = __fsub_rn(p, __fmul_rn(a.lr, __fadd_rn(upd, __fmul_rn(a.wd, p))));
}

// Segments start and end on multiples of 4 floats (every parameter's size is
// a multiple of the hidden size, itself a multiple of 4): float4 throughout.
// Each thread takes U float4 groups per iteration (U strides apart) and
// issues all their loads before any arithmetic, so more bytes are in flight
// per thread; the per-element arithmetic is unchanged.
template <int U>
__global__ void adamw_kernel(float* __restrict__ p, float* __restrict__ g, float* __restrict__ m, float* __restrict__ v,
                             float* __restrict__ shadow, const Seg* __restrict__ segs,
                             const float* __restrict__ clip_scale, AdamArgs a, int write_g) {
  GLC_PDL_ENTRY();
  const Seg sg = segs[blockIdx.y];
  const float scale = clip_scale ? *clip_scale : 1.0f;
  const bool scaled = scale != 1.0f;
  float4* p4 = reinterpret_cast<float4*>(p + sg.start);
  float4* g4 = reinterpret_cast<float4*>(g + sg.start);
  float4* m4 = reinterpret_cast<float4*>(m + sg.start);
  float4* v4 = reinterpret_cast<float4*>(v + sg.start);
  float4* s4 = shadow ? reinterpret_cast<float4*>(shadow + sg.start) : nullptr;
  const int64_t n4 = sg.len >> 2;
  const int64_t stride = int64_t(gridDim.x) * blockDim.x;
  for (int64_t i0 = blockIdx.x * int64_t(blockDim.x) + threadIdx.x; i0 < n4; i0 += U * stride) {
    float4 P[U], G[U], M[U], V[U];
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i < n4) {  // each value is read and written once per step: evict-first
        P[u] = __ldcs(p4 + i);
        G[u] = __ldcs(g4 + i);
        M[u] = __ldcs(m4 + i);
        V[u] = __ldcs(v4 + i);
      }
    }
#pragma unroll
    for (int u = 0; u < U; ++u) {
      const int64_t i = i0 + u * stride;
      if (i >= n4) continue;
      adam_elem(P[u].x, G[u].x, M[u].x, V[u].x, scale, scaled, a);
      adam_elem(P[u].y, G[u].y, M[u].y, V[u].y, scale, scaled, a);
      adam_elem(P[u].z, G[u].z, M[u].z, V[u].z, scale, scaled, a);
      adam_elem(P[u].w, G[u].w, M[u].w, V[u].w, scale, scaled, a);
      if (scaled && write_g) __stcs(g4 + i, G[u]);
      __stcs(m4 + i, M[u]);
      __stcs(v4 + i, V[u]);
      __stcs(p4 + i, P[u]);
      if (s4) __stcs(s4 + i, make_float4(round_tf32(P[u].x), round_tf32(P[u].y), round_tf32(P[u].z), round_tf32(P[u].w)));
    }
  }
}

}  // namespace

// segs: device array of {start, len} pairs (int64), nseg entries; every start
// and len a multiple of 4.
int grad_norm_blocks(const Context* ctx, int nseg) {
  if (nseg <= 0) return 0;
  const int bx = (8 * ctx->num_sms + nseg - 1) / nseg;
  return bx < 4 ? 4 : bx;
}

int grad_sumsq(Context* ctx, const float* grads, const int64_t* segs, int nseg, int bx, double* partial, double elems,
               cudaStream_t s) {
  if (nseg <= 0) return 0;
  if (!grads || !segs || !partial || bx <= 0) return ctx->fail(GLC_ERR_INVALID, "grad_sumsq: bad arguments");
  ProfScope prof(ctx, PROF_ADAMW, 4.0 * elems, s);
  glc::launch_pdl(ctx, sumsq_kernel, dim3(bx, nseg), 256, 0, s, grads, reinterpret_cast<const Seg*>(segs), partial);
  GLC_LAUNCH_CHECK(ctx, "grad_norm partial");
  return 0;
}

int grad_sumsq_chunks(Context* ctx, const float* grads, const int64_t* chunks, int nchunks, int blocks, double* out,
                      double elems, cudaStream_t s) {
  if (nchunks <= 0) return 0;
  if (!grads || !chunks || !out || blocks <= 0) return ctx->fail(GLC_ERR_INVALID, "grad_sumsq_chunks: bad arguments");
  ProfScope prof(ctx, PROF_ADAMW, 4.0 * elems, s);
  glc::launch_pdl(ctx, sumsq_chunks_kernel, blocks < nchunks ? blocks : nchunks, 256, 0, s, grads,
                  reinterpret_cast<const Seg*>(chunks), nchunks, out);
  GLC_LAUNCH_CHECK(ctx, "grad_sumsq_chunks");
  return 0;
}

int grad_norm_finish(Context* ctx, const double* partial, long long n, float max_norm, double* norm_out,
                     float* scale_out, cudaStream_t s, double* lvl, long long lvl_cap) {
  if (n <= 0 || n > 0x7fffffffLL || !partial || !norm_out || !scale_out)
    return ctx->fail(GLC_ERR_INVALID, "grad_norm_finish: bad arguments");
  ProfScope prof(ctx, PROF_ADAMW, 8.0 * static_cast<double>(n), s);
  const long long chunk = 1024;
  const long long nb = (n + chunk - 1) / chunk;
  if (n > 8192 && lvl && lvl_cap >= nb) {
    // many partials (the GEMM epilogues' slots): blocks of 1024 first
    glc::launch_pdl(ctx, slot_sum_kernel, static_cast<unsigned>(nb), 256, 0, s, partial, n, chunk, lvl);
    GLC_LAUNCH_CHECK(ctx, "grad_norm slot sum");
    partial = lvl;
    n = nb;
  }
  glc::launch_pdl(ctx, norm_finish_kernel, 1, 256, 0, s, partial, static_cast<int>(n), max_norm, norm_out, scale_out);
  GLC_LAUNCH_CHECK(ctx, "grad_norm finish");
  return 0;
}

int grad_norm(Context* ctx, const float* grads, const int64_t* segs, int nseg, float max_norm, double* norm_out,
              float* scale_out, double* scratch, int scratch_count, double elems, cudaStream_t s) {
  if (nseg <= 0 || !grads || !segs || !norm_out || !scale_out)
    return ctx->fail(GLC_ERR_INVALID, "grad_norm: bad arguments");
  const int bx = grad_norm_blocks(ctx, nseg);
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
  int rc = grad_sumsq(ctx, grads, segs, nseg, bx, partial, elems, s);
  if (!rc) rc = grad_norm_finish(ctx, partial, n, max_norm, norm_out, scale_out, s, nullptr, 0);
  return rc;
}

int adamw(Context* ctx, float* p, float* g, float* m, float* v, float* shadow, const int64_t* segs, int nseg,
          const float* clip_scale, float lr, float beta1, float beta2, float eps, float wd, int step, double elems,
          cudaStream_t s, bool write_grad) {
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
  a.rbc1 = 1.0 / a.bc1;
  a.rbc2 = 1.0 / a.bc2;
  a.eps = static_cast<double>(eps);
  int bx = (8 * ctx->num_sms + nseg - 1) / nseg;
  if (bx < 4) bx = 4;
  // p, g, m, v read; p, m, v and the TF32 shadow written
  ProfScope prof(ctx, PROF_ADAMW, (shadow ? 32.0 : 28.0) * elems, s);
  glc::launch_pdl(ctx, adamw_kernel<2>, dim3(bx, nseg), 256, 0, s, p, g, m, v, shadow, reinterpret_cast<const Seg*>(segs),
                  clip_scale, a, write_grad ? 1 : 0);
  GLC_LAUNCH_CHECK(ctx, "adamw");
  return 0;
}

namespace {
// g = g * scale (float32, as the clipping in the AdamW kernel), unless scale is 1
__global__ void scale_in_place_kernel(float* __restrict__ g, size_t n, const float* __restrict__ scale) {
  GLC_PDL_ENTRY();
  const float sc = *scale;
  if (sc == 1.0f) return;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    g[i] = __fmul_rn(g[i], sc);
}
}  // namespace

int scale_in_place(Context* ctx, float* g, size_t n, const float* scale, cudaStream_t s) {
  if (n == 0) return 0;
  if (!g || !scale) return ctx->fail(GLC_ERR_INVALID, "scale_in_place: null pointer");
  glc::launch_pdl(ctx, scale_in_place_kernel, grid_for(n, 256, ctx->num_sms), 256, 0, s, g, n, scale);
  GLC_LAUNCH_CHECK(ctx, "scale_in_place");
  return 0;
}

}  // namespace glc
