// Fused softmax cross-entropy forward + backward (SoftmaxCrossEntropyGrad,
// pkg/tensor/grad.go:210-280).
//
// One CTA of up to 512 threads per row; the row lives in registers (V <= 65536).  Per row:
//   max (grad.go:220-225), e_v = exp32(l_v - max) and their float32 sum
//   (:228-232), p_v = e_v / sum (:235-237), the target's log32(p_t + 1e-10)
//   (:240-243; targets outside [0, V) contribute nothing), and, when the
//   gradient is wanted, dlogits_v = p_v*scale - [v == t]*scale (:266-276),
//   written in place over the logits (the row is fully in registers first).
// The loss (:246) is summed by a second, single-thread kernel in row order,
// exactly as the reference's running float32 total.
//
// Large vocabularies (V > 8192) split each row over a cluster of CE_CL CTAs
// (ce_cluster_kernel): each holds a quarter of the row in registers, and the
// row max and sum are exchanged through distributed shared memory, added in
// rank order so every CTA of the row derives the same values.  A quarter row
// needs ~64 registers per thread, so several rows share an SM and one row's
// loads overlap another's arithmetic (one CTA per row holds a whole row per
// SM at a time and serialises them).
#include <cfloat>

#include "glc_internal.h"
#include "go_math.cuh"
#include "sm100.cuh"

namespace glc {
namespace {

template <bool IS_MAX>
__device__ __forceinline__ float block_reduce(float v, float* red) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) {
    const float w = __shfl_xor_sync(0xffffffffu, v, o);
    v = IS_MAX ? fmaxf(v, w) : v + w;
  }
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, nw = blockDim.x >> 5;
  __syncthreads();
  if (lane == 0) red[warp] = v;
  __syncthreads();
  if (warp == 0) {
    float t = lane < nw ? red[lane] : (IS_MAX ? -FLT_MAX : 0.f);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
      const float w = __shfl_xor_sync(0xffffffffu, t, o);
      t = IS_MAX ? fmaxf(t, w) : t + w;
    }
    if (lane == 0) red[32] = t;
  }
  __syncthreads();
  return red[32];
}

template <int VPT, bool FAST>
__global__ void __launch_bounds__(512) ce_kernel(float* __restrict__ logits, const int64_t* __restrict__ targets,
                                                  int rows, int V, float scale, float* __restrict__ row_logp,
                                                  int write_grad, int round_out) {
  GLC_PDL_ENTRY();
  __shared__ float red[33];
  const int nc = V >> 2;
  for (int row = blockIdx.x; row < rows; row += gridDim.x) {
    float4* lr = reinterpret_cast<float4*>(logits + static_cast<size_t>(row) * V);
    float4 v[VPT];
    float m = -FLT_MAX;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nc) {
        v[i] = lr[c];
        m = fmaxf(m, fmaxf(fmaxf(v[i].x, v[i].y), fmaxf(v[i].z, v[i].w)));
      }
    }
    m = block_reduce<true>(m, red);
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nc) {
        v[i].x = FAST ? expf(__fsub_rn(v[i].x, m)) : go_exp32_fast(__fsub_rn(v[i].x, m));
        v[i].y = FAST ? expf(__fsub_rn(v[i].y, m)) : go_exp32_fast(__fsub_rn(v[i].y, m));
        v[i].z = FAST ? expf(__fsub_rn(v[i].z, m)) : go_exp32_fast(__fsub_rn(v[i].z, m));
        v[i].w = FAST ? expf(__fsub_rn(v[i].w, m)) : go_exp32_fast(__fsub_rn(v[i].w, m));
        s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
      }
    }
    s = block_reduce<false>(s, red);
    const float inv = FAST ? 1.0f / s : 0.f;
    const int64_t t = targets[row];
#pragma unroll
    for (int i = 0; i < VPT; ++i) {
      const int c = threadIdx.x + i * blockDim.x;
      if (c < nc) {
        // p_v = e_v / sum: the reference's division, bit for bit, where its
        // bits are matched (exp32 path); the Llama path (no reference bits)
        // multiplies by the row's reciprocal.  Without the gradient only the
        // target's p is needed.
        const bool has_t = t >= 4 * c && t < 4 * c + 4;
        float p[4] = {0.f, 0.f, 0.f, 0.f};
        if (FAST) {
          p[0] = v[i].x * inv; p[1] = v[i].y * inv; p[2] = v[i].z * inv; p[3] = v[i].w * inv;
        } else if (write_grad || has_t) {
          p[0] = __fdiv_rn(v[i].x, s); p[1] = __fdiv_rn(v[i].y, s); p[2] = __fdiv_rn(v[i].z, s); p[3] = __fdiv_rn(v[i].w, s);
        }
        if (has_t) {
          const int j = static_cast<int>(t - 4 * c);
          const float pt = j == 0 ? p[0] : j == 1 ? p[1] : j == 2 ? p[2] : p[3];
          row_logp[row] = FAST ? logf(__fadd_rn(pt, 1e-10f)) : go_log32(__fadd_rn(pt, 1e-10f));
        }
        if (write_grad) {
          float g[4];
#pragma unroll
          for (int j = 0; j < 4; ++j) {
            g[j] = __fmul_rn(p[j], scale);
            if (4 * c + j == t) g[j] = __fsub_rn(g[j], scale);
            if (round_out) g[j] = round_tf32(g[j]);
          }
          lr[c] = make_float4(g[0], g[1], g[2], g[3]);
        }
      }
    }
    if ((t < 0 || t >= V) && threadIdx.x == 0) row_logp[row] = 0.f;
    __syncthreads();
  }
}

constexpr int CE_CL = 4;        // CTAs per row
constexpr int CE_CL_THREADS = 256;

// Row max (IS_MAX) or sum over the cluster: block reduce, publish in slot,
// cluster barrier, then every thread combines the CE_CL published values in
// rank order.
template <bool IS_MAX>
__device__ __forceinline__ float cluster_reduce(float v, float* red, float* slot) {
  v = block_reduce<IS_MAX>(v, red);
  if (threadIdx.x == 0) *slot = v;
  cluster_sync_all();
  float t = ld_shared_cluster_f32(mapa_cluster(slot, 0));
#pragma unroll
  for (int r = 1; r < CE_CL; ++r) {
    const float w = ld_shared_cluster_f32(mapa_cluster(slot, r));
    t = IS_MAX ? fmaxf(t, w) : t + w;
  }
  return t;
}

// Grid: rows * CE_CL CTAs, cluster (CE_CL, 1, 1) per row; CTA rank r covers
// float4 columns [r * chunk, (r + 1) * chunk) of the row.
template <int VPT, bool FAST>
__global__ void __cluster_dims__(CE_CL, 1, 1) __launch_bounds__(CE_CL_THREADS, VPT <= 8 ? 4 : 2)
    ce_cluster_kernel(float* __restrict__ logits, const int64_t* __restrict__ targets, int V, int chunk, float scale,
                      float* __restrict__ row_logp, int write_grad, int round_out) {
  GLC_PDL_ENTRY();
  __shared__ float red[33];
  __shared__ float slots[2];
  const int nc = V >> 2;
  const int row = static_cast<int>(blockIdx.x) / CE_CL;
  const int rank = static_cast<int>(cluster_ctarank());
  const int c0 = rank * chunk, c1 = min(nc, c0 + chunk);
  float4* lr = reinterpret_cast<float4*>(logits + static_cast<size_t>(row) * V);
  float4 v[VPT];
  float m = -FLT_MAX;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = c0 + threadIdx.x + i * CE_CL_THREADS;
    if (c < c1) {
      v[i] = lr[c];
      m = fmaxf(m, fmaxf(fmaxf(v[i].x, v[i].y), fmaxf(v[i].z, v[i].w)));
    }
  }
  m = cluster_reduce<true>(m, red, &slots[0]);
  float s = 0.f;
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = c0 + threadIdx.x + i * CE_CL_THREADS;
    if (c < c1) {
      v[i].x = FAST ? expf(__fsub_rn(v[i].x, m)) : go_exp32_fast(__fsub_rn(v[i].x, m));
      v[i].y = FAST ? expf(__fsub_rn(v[i].y, m)) : go_exp32_fast(__fsub_rn(v[i].y, m));
      v[i].z = FAST ? expf(__fsub_rn(v[i].z, m)) : go_exp32_fast(__fsub_rn(v[i].z, m));
      v[i].w = FAST ? expf(__fsub_rn(v[i].w, m)) : go_exp32_fast(__fsub_rn(v[i].w, m));
      s += (v[i].x + v[i].y) + (v[i].z + v[i].w);
    }
  }
  s = cluster_reduce<false>(s, red, &slots[1]);
  const float inv = FAST ? 1.0f / s : 0.f;
  const int64_t t = targets[row];
#pragma unroll
  for (int i = 0; i < VPT; ++i) {
    const int c = c0 + threadIdx.x + i * CE_CL_THREADS;
    if (c < c1) {
      const bool has_t = t >= 4 * c && t < 4 * c + 4;
      float p[4] = {0.f, 0.f, 0.f, 0.f};
      if (FAST) {
        p[0] = v[i].x * inv; p[1] = v[i].y * inv; p[2] = v[i].z * inv; p[3] = v[i].w * inv;
      } else if (write_grad || has_t) {
        p[0] = __fdiv_rn(v[i].x, s); p[1] = __fdiv_rn(v[i].y, s); p[2] = __fdiv_rn(v[i].z, s); p[3] = __fdiv_rn(v[i].w, s);
      }
      if (has_t) {
        const int j = static_cast<int>(t - 4 * c);
        const float pt = j == 0 ? p[0] : j == 1 ? p[1] : j == 2 ? p[2] : p[3];
        row_logp[row] = FAST ? logf(__fadd_rn(pt, 1e-10f)) : go_log32(__fadd_rn(pt, 1e-10f));
      }
      if (write_grad) {
        float g[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) {
          g[j] = __fmul_rn(p[j], scale);
          if (4 * c + j == t) g[j] = __fsub_rn(g[j], scale);
          if (round_out) g[j] = round_tf32(g[j]);
        }
        lr[c] = make_float4(g[0], g[1], g[2], g[3]);
      }
    }
  }
  if ((t < 0 || t >= V) && rank == 0 && threadIdx.x == 0) row_logp[row] = 0.f;
  // no CTA leaves while a peer may still read its slots
  cluster_sync_all();
}

// loss = (0 - logp_0 - logp_1 - ...) / rows over valid targets (grad.go:239-246).
// One block: the threads stage chunks of row_logp in shared memory, thread 0
// subtracts them in row order (the reference's running float32 total).
__global__ void ce_loss_sum_kernel(const float* __restrict__ row_logp, const int64_t* __restrict__ targets, int rows,
                                   int V, float* __restrict__ loss) {
  GLC_PDL_ENTRY();
  constexpr int CHUNK = 2048;
  __shared__ float buf[CHUNK];
  float total = 0.f;
  for (int base = 0; base < rows; base += CHUNK) {
    const int n = min(CHUNK, rows - base);
    for (int i = threadIdx.x; i < n; i += blockDim.x) {
      const int64_t t = targets[base + i];
      buf[i] = (t >= 0 && t < V) ? row_logp[base + i] : 0.f;  // x - 0 == x: invalid rows add nothing
    }
    __syncthreads();
    if (threadIdx.x == 0)
      for (int i = 0; i < n; ++i) total = __fsub_rn(total, buf[i]);
    __syncthreads();
  }
  if (threadIdx.x == 0) *loss = __fdiv_rn(total, static_cast<float>(rows));
}

__global__ void exp32_kernel(const float* __restrict__ x, float* __restrict__ y, size_t n) {
  GLC_PDL_ENTRY();
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    y[i] = go_exp32_fast(x[i]);
}

}  // namespace

int exp32(Context* ctx, const float* x, float* y, size_t n, cudaStream_t s) {
  if (n == 0) return 0;
  if (!x || !y) return ctx->fail(GLC_ERR_INVALID, "exp32: null pointer");
  ProfScope prof(ctx, PROF_OTHER, 8.0 * n, s);
  glc::launch_pdl(ctx, exp32_kernel, grid_for(n, 256, ctx->num_sms), 256, 0, s, x, y, n);
  GLC_LAUNCH_CHECK(ctx, "exp32");
  return 0;
}

int softmax_ce(Context* ctx, float* logits, const int64_t* targets, int rows, int V, float scale, float* row_logp,
               float* loss, bool write_grad, bool round_out, cudaStream_t s, bool fast_exp) {
  if (rows <= 0 || V <= 0) return ctx->fail(GLC_ERR_INVALID, "softmax_ce: empty logits");
  if ((V & 3) || (reinterpret_cast<uintptr_t>(logits) & 15))
    return ctx->fail(GLC_ERR_INVALID, "softmax_ce: vocab must be a multiple of 4, logits 16-byte aligned");
  if (!targets || !row_logp || !loss) return ctx->fail(GLC_ERR_INVALID, "softmax_ce: null pointer");
  const int nc = V / 4;
  const int wg = write_grad ? 1 : 0, ro = round_out ? 1 : 0;
  if (nc > 2048) {
    // V > 8192: a cluster of CE_CL CTAs per row
    const int chunk = (nc + CE_CL - 1) / CE_CL;
    const int vpt = (chunk + CE_CL_THREADS - 1) / CE_CL_THREADS;
    if (static_cast<long long>(rows) * CE_CL > 0x7fffffffLL) return ctx->fail(GLC_ERR_INVALID, "softmax_ce: too many rows");
    const unsigned grid = static_cast<unsigned>(rows) * CE_CL;
    ProfScope prof(ctx, PROF_CE, 4.0 * static_cast<double>(rows) * V * (write_grad ? 2 : 1), s);
    if (vpt <= 4)
      glc::launch_pdl(ctx, (fast_exp ? ce_cluster_kernel<4, true> : ce_cluster_kernel<4, false>), grid, CE_CL_THREADS, 0, s,
                      logits, targets, V, chunk, scale, row_logp, wg, ro);
    else if (vpt <= 8)
      glc::launch_pdl(ctx, (fast_exp ? ce_cluster_kernel<8, true> : ce_cluster_kernel<8, false>), grid, CE_CL_THREADS, 0, s,
                      logits, targets, V, chunk, scale, row_logp, wg, ro);
    else if (vpt <= 16)
      glc::launch_pdl(ctx, (fast_exp ? ce_cluster_kernel<16, true> : ce_cluster_kernel<16, false>), grid, CE_CL_THREADS, 0, s,
                      logits, targets, V, chunk, scale, row_logp, wg, ro);
    else
      return ctx->fail(GLC_ERR_UNSUPPORTED, "softmax_ce: vocab above 65536 is not supported");
    GLC_LAUNCH_CHECK(ctx, "softmax_ce (cluster)");
    glc::launch_pdl(ctx, ce_loss_sum_kernel, 1, 256, 0, s, row_logp, targets, rows, V, loss);
    GLC_LAUNCH_CHECK(ctx, "softmax_ce loss");
    return 0;
  }
  int threads = ((nc + 31) / 32) * 32;
  if (threads > 512) threads = 512;
  const int vpt = (nc + threads - 1) / threads;
  const unsigned grid = static_cast<unsigned>(rows);
  ProfScope prof(ctx, PROF_CE, 4.0 * static_cast<double>(rows) * V * (write_grad ? 2 : 1), s);
  if (vpt <= 1)
    glc::launch_pdl(ctx, (fast_exp ? ce_kernel<1, true> : ce_kernel<1, false>), grid, threads, 0, s, logits, targets, rows, V, scale, row_logp, wg, ro);
  else if (vpt <= 2)
    glc::launch_pdl(ctx, (fast_exp ? ce_kernel<2, true> : ce_kernel<2, false>), grid, threads, 0, s, logits, targets, rows, V, scale, row_logp, wg, ro);
  else if (vpt <= 4)
    glc::launch_pdl(ctx, (fast_exp ? ce_kernel<4, true> : ce_kernel<4, false>), grid, threads, 0, s, logits, targets, rows, V, scale, row_logp, wg, ro);
  else if (vpt <= 8)
    glc::launch_pdl(ctx, (fast_exp ? ce_kernel<8, true> : ce_kernel<8, false>), grid, threads, 0, s, logits, targets, rows, V, scale, row_logp, wg, ro);
  else if (vpt <= 16)
    glc::launch_pdl(ctx, (fast_exp ? ce_kernel<16, true> : ce_kernel<16, false>), grid, threads, 0, s, logits, targets, rows, V, scale, row_logp, wg, ro);
  else if (vpt <= 32)
    glc::launch_pdl(ctx, (fast_exp ? ce_kernel<32, true> : ce_kernel<32, false>), grid, threads, 0, s, logits, targets, rows, V, scale, row_logp, wg, ro);
  else
    return ctx->fail(GLC_ERR_UNSUPPORTED, "softmax_ce: vocab above 65536 is not supported");
  GLC_LAUNCH_CHECK(ctx, "softmax_ce");
  glc::launch_pdl(ctx, ce_loss_sum_kernel, 1, 256, 0, s, row_logp, targets, rows, V, loss);
  GLC_LAUNCH_CHECK(ctx, "softmax_ce loss");
  return 0;
}

}  // namespace glc
