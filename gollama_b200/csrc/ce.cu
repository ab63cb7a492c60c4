// Fused softmax cross-entropy forward + backward (SoftmaxCrossEntropyGrad,
// pkg/tensor/grad.go:210-280).
//
// Up to V = 8192, one CTA of up to 512 threads per row (ce_kernel); in every
// kernel the row lives in registers (V <= 65536).  Per row:
//   max (grad.go:220-225), e_v = exp32(l_v - max) and their float32 sum
//   (:228-232), p_v = e_v / sum (:235-237), the target's log32(p_t + 1e-10)
//   (:240-243; targets outside [0, V) contribute nothing), and, when the
//   gradient is wanted, dlogits_v = p_v*scale - [v == t]*scale (:266-276),
//   written in place over the logits (the row is fully in registers first).
// The loss (:246) is summed by a second kernel whose thread 0 subtracts the
// rows' terms in row order, exactly as the reference's running float32 total.
//
// Large vocabularies in the Llama arithmetic (8192 < V <= 32768) stream their
// rows through persistent CTAs (ce_stream_kernel, below): bulk copies fill a
// shared-memory ring of row chunks ahead of the row in registers.  The others
// split each row over a cluster of CE_CL CTAs (ce_cluster_kernel): each holds
// a quarter of the row in registers, and the row max and sum are exchanged
// through distributed shared memory, added in rank order so every CTA of the
// row derives the same values.
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

// Streamed rows (8192 < V <= 32768): one persistent CTA of CE_ST_THREADS per
// SM walks the rows blockIdx.x, blockIdx.x + gridDim.x, ...  A row is cut
// into CE_ST_CHUNKS chunks of cf4 float4 (the last one shorter).  Thread 0
// keeps a ring of `nslots` shared-memory chunk slots filled with bulk copies
// (one mbarrier per slot), up to nslots chunks ahead of the row in hand.  The
// threads move the current row from its slots into registers (thread t holds
// float4 t + 512 u of every chunk); once every thread has done so the slots
// are refilled with the next chunks, while the row's max, exponentials, sum
// and gradient are computed from registers and the gradient is stored
// straight to global memory.  Loads keep streaming through the reductions
// and stores of the row before (the one-shot clusters load, reduce and store
// in step), and a row never leaves its CTA: two block reductions, no cluster
// barrier.  With the reference's exp32 and division the per-element
// arithmetic is the cluster kernel's (and its float64 exponential makes the
// kernel compute-bound on 16 warps per SM: the clusters' 32 run it faster);
// with the Llama arithmetic e^(x - max) is ex2.approx of one FMA and the
// gradient one product, few enough instructions for the copies to set the
// pace.  The row sum adds each thread's partial, then warp and block partials
// in a fixed order.
constexpr float kLog2e = 1.4426950408889634f;
__device__ __forceinline__ float ex2_approx(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}

constexpr int CE_ST_THREADS = 512;
constexpr int CE_ST_WARPS = CE_ST_THREADS / 32;
constexpr int CE_ST_CHUNKS = 8;
constexpr int CE_ST_MAX_SLOTS = 32;
constexpr size_t CE_ST_SMEM_BYTES = 224 * 1024;  // ring; the static barriers and partials fit beside it

template <int U, bool FAST>
__global__ void __launch_bounds__(CE_ST_THREADS, 1)
    ce_stream_kernel(float* __restrict__ logits, const int64_t* __restrict__ targets, int rows, int V, int cf4,
                     int nslots, float scale, float* __restrict__ row_logp, int write_grad, int round_out, int* err) {
  GLC_PDL_ENTRY();
  extern __shared__ __align__(16) float4 ring[];  // [nslots][cf4]
  __shared__ uint64_t full[CE_ST_MAX_SLOTS];
  __shared__ float red_m[CE_ST_WARPS];
  __shared__ float red_s[CE_ST_WARPS];
  __shared__ int abort_flag;
  const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
  const int nc = V >> 2;
  const int cta = static_cast<int>(blockIdx.x), ncta = static_cast<int>(gridDim.x);
  const int nrows = cta < rows ? (rows - 1 - cta) / ncta + 1 : 0;
  const int nq = nrows * CE_ST_CHUNKS;  // chunks this CTA loads
  // thread 0 only: chunk q is chunk q % CE_ST_CHUNKS of the CTA's row q / CE_ST_CHUNKS, into slot q % nslots
  auto issue = [&](int q) {
    const int j = q % CE_ST_CHUNKS;
    const size_t row = static_cast<size_t>(cta) + static_cast<size_t>(q / CE_ST_CHUNKS) * ncta;
    const uint32_t bytes = static_cast<uint32_t>(min(cf4, nc - j * cf4)) * 16u;
    const int slot = q % nslots;
    mbar_arrive_expect_tx(&full[slot], bytes);
    bulk_load(ring + static_cast<size_t>(slot) * cf4, logits + row * V + static_cast<size_t>(j) * cf4 * 4, bytes,
              &full[slot]);
  };
  if (tid == 0) {
    for (int i = 0; i < nslots; ++i) mbar_init(&full[i], 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  int issued = 0;  // chunks whose copies thread 0 has issued
  if (tid == 0)
    for (; issued < nq && issued < nslots; ++issued) issue(issued);
  int slot = 0;       // slot of the next chunk to consume
  uint32_t ph = 0;    // its phase parity
  bool ok = true, aborted = false;
  int k = 0;
  for (; k < nrows; ++k) {
    const int row = cta + k * ncta;
    const int64_t t64 = targets[row];
    const int t = t64 >= 0 && t64 < V ? static_cast<int>(t64) : -1;  // -1 (no target) matches no column
    const int t4 = t >= 0 ? t >> 2 : -1;                               // the target's float4 column
    float4 v[CE_ST_CHUNKS][U];
    float m = -FLT_MAX;
#pragma unroll
    for (int j = 0; j < CE_ST_CHUNKS; ++j) {
      ok = ok && mbar_wait(&full[slot], ph, &abort_flag, err, GLC_DEV_TIMEOUT_EPILOGUE);
      const int cnt = j + 1 < CE_ST_CHUNKS ? cf4 : nc - j * cf4;
      const float4* src = ring + static_cast<size_t>(slot) * cf4;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int e = tid + u * CE_ST_THREADS;
        if (e < cnt) {
          v[j][u] = src[e];
          m = fmaxf(m, fmaxf(fmaxf(v[j][u].x, v[j][u].y), fmaxf(v[j][u].z, v[j][u].w)));
        }
      }
      if (++slot == nslots) {
        slot = 0;
        ph ^= 1u;
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) m = fmaxf(m, __shfl_xor_sync(0xffffffffu, m, o));
    if (lane == 0) red_m[warp] = m;
    // every thread holds its part of the row (or a wait gave up): the row's slots may be refilled
    if (!__syncthreads_and(ok)) {
      aborted = true;
      break;
    }
    if (tid == 0) {
      const int lim = min(nq, (k + 1) * CE_ST_CHUNKS + nslots);
      for (; issued < lim; ++issued) issue(issued);
    }
    float mx = red_m[0];
#pragma unroll
    for (int w = 1; w < CE_ST_WARPS; ++w) mx = fmaxf(mx, red_m[w]);
    // Llama arithmetic: e^(x - max) = 2^(x log2 e - max log2 e), one FMA and
    // ex2.approx (relative error ~1e-6 against expf, far inside the fp32
    // tolerance of this path and the TF32 rounding its gradient gets)
    const float mlog2 = mx * kLog2e;
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < CE_ST_CHUNKS; ++j) {
      const int cnt = j + 1 < CE_ST_CHUNKS ? cf4 : nc - j * cf4;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        if (tid + u * CE_ST_THREADS < cnt) {
          float4& x = v[j][u];
          if (FAST) {
            x.x = ex2_approx(fmaf(x.x, kLog2e, -mlog2));
            x.y = ex2_approx(fmaf(x.y, kLog2e, -mlog2));
            x.z = ex2_approx(fmaf(x.z, kLog2e, -mlog2));
            x.w = ex2_approx(fmaf(x.w, kLog2e, -mlog2));
          } else {
            x.x = go_exp32_fast(__fsub_rn(x.x, mx));
            x.y = go_exp32_fast(__fsub_rn(x.y, mx));
            x.z = go_exp32_fast(__fsub_rn(x.z, mx));
            x.w = go_exp32_fast(__fsub_rn(x.w, mx));
          }
          s += (x.x + x.y) + (x.z + x.w);
        }
      }
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    if (lane == 0) red_s[warp] = s;
    // red_m is rewritten only after the next row's loads, past this barrier; red_s after the next one's first
    __syncthreads();
    float sum = red_s[0];
#pragma unroll
    for (int w = 1; w < CE_ST_WARPS; ++w) sum += red_s[w];
    float4* lr = reinterpret_cast<float4*>(logits + static_cast<size_t>(row) * V);
    if (FAST) {
      // p = e * (1 / sum), the gradient p * scale as one product; the target's
      // column (one float4 of the row) takes p_t * scale - scale and its log
      const float inv = 1.0f / sum;
      const float ks = inv * scale;
#pragma unroll
      for (int j = 0; j < CE_ST_CHUNKS; ++j) {
        const int cnt = j + 1 < CE_ST_CHUNKS ? cf4 : nc - j * cf4;
#pragma unroll
        for (int u = 0; u < U; ++u) {
          const int e = tid + u * CE_ST_THREADS;
          if (e < cnt) {
            const int c = j * cf4 + e;
            const float4 x = v[j][u];
            float g[4] = {x.x * ks, x.y * ks, x.z * ks, x.w * ks};
            if (c == t4) {
              const int jj = t & 3;
              const float pt = (jj == 0 ? x.x : jj == 1 ? x.y : jj == 2 ? x.z : x.w) * inv;
              row_logp[row] = logf(__fadd_rn(pt, 1e-10f));
              const float gt = __fsub_rn(__fmul_rn(pt, scale), scale);
              g[0] = jj == 0 ? gt : g[0];
              g[1] = jj == 1 ? gt : g[1];
              g[2] = jj == 2 ? gt : g[2];
              g[3] = jj == 3 ? gt : g[3];
            }
            if (write_grad) {
              if (round_out) {
#pragma unroll
                for (int q = 0; q < 4; ++q) g[q] = round_tf32(g[q]);
              }
              lr[c] = make_float4(g[0], g[1], g[2], g[3]);
            }
          }
        }
      }
      if (t < 0 && tid == 0) row_logp[row] = 0.f;
      continue;
    }
#pragma unroll
    for (int j = 0; j < CE_ST_CHUNKS; ++j) {
      const int cnt = j + 1 < CE_ST_CHUNKS ? cf4 : nc - j * cf4;
#pragma unroll
      for (int u = 0; u < U; ++u) {
        const int e = tid + u * CE_ST_THREADS;
        if (e < cnt) {
          const int c = j * cf4 + e;
          const float4 x = v[j][u];
          const bool has_t = static_cast<unsigned>(t - 4 * c) < 4u;
          float p[4] = {0.f, 0.f, 0.f, 0.f};
          if (write_grad || has_t) {
            p[0] = __fdiv_rn(x.x, sum); p[1] = __fdiv_rn(x.y, sum); p[2] = __fdiv_rn(x.z, sum); p[3] = __fdiv_rn(x.w, sum);
          }
          if (has_t) {
            const int jj = t - 4 * c;
            const float pt = jj == 0 ? p[0] : jj == 1 ? p[1] : jj == 2 ? p[2] : p[3];
            row_logp[row] = go_log32(__fadd_rn(pt, 1e-10f));
          }
          if (write_grad) {
            float g[4];
#pragma unroll
            for (int q = 0; q < 4; ++q) {
              g[q] = __fmul_rn(p[q], scale);
              if (q == t - 4 * c) g[q] = __fsub_rn(g[q], scale);
              if (round_out) g[q] = round_tf32(g[q]);
            }
            lr[c] = make_float4(g[0], g[1], g[2], g[3]);
          }
        }
      }
    }
    if (t < 0 && tid == 0) row_logp[row] = 0.f;
  }
  if (aborted && tid == 0) {
    // no copy may land after the CTA exits: wait (bounded) for those in flight
    for (int q = k * CE_ST_CHUNKS; q < issued; ++q) mbar_drain(&full[q % nslots], (q / nslots) & 1, err);
  }
}

// loss = (0 - logp_0 - logp_1 - ...) / rows over valid targets (grad.go:239-246).
// One block: the threads stage chunks of row_logp in shared memory (every
// thread's loads issued together), thread 0 subtracts them in row order (the
// reference's running float32 total).  The chunk is padded with +0 (x - 0 ==
// x exactly, -0 included), so thread 0 reads eight float4 ahead and only the
// chain of subtractions is serial.
constexpr int CE_LS_THREADS = 1024;
__global__ void __launch_bounds__(CE_LS_THREADS) ce_loss_sum_kernel(const float* __restrict__ row_logp,
                                                                  const int64_t* __restrict__ targets, int rows,
                                                                  int V, float* __restrict__ loss) {
  GLC_PDL_ENTRY();
  constexpr int CHUNK = 4096, PER = CHUNK / CE_LS_THREADS;
  __shared__ __align__(16) float buf[CHUNK];
  float total = 0.f;
  for (int base = 0; base < rows; base += CHUNK) {
    const int n = min(CHUNK, rows - base);
    int64_t tt[PER];
    float lp[PER];
#pragma unroll
    for (int u = 0; u < PER; ++u) {
      const int i = static_cast<int>(threadIdx.x) + u * CE_LS_THREADS;
      tt[u] = i < n ? targets[base + i] : -1;
      lp[u] = i < n ? row_logp[base + i] : 0.f;
    }
#pragma unroll
    for (int u = 0; u < PER; ++u)  // invalid rows and the padding add nothing
      buf[threadIdx.x + u * CE_LS_THREADS] = (tt[u] >= 0 && tt[u] < V) ? lp[u] : 0.f;
    __syncthreads();
    if (threadIdx.x == 0) {
      const float4* b4 = reinterpret_cast<const float4*>(buf);
      const int n4 = (n + 3) >> 2;
      for (int i = 0; i < n4; i += 8) {
        float4 q[8];
#pragma unroll
        for (int u = 0; u < 8; ++u) q[u] = b4[i + u];  // i + 8 <= CHUNK / 4: the padding covers the tail
#pragma unroll
        for (int u = 0; u < 8; ++u) {
          total = __fsub_rn(total, q[u].x);
          total = __fsub_rn(total, q[u].y);
          total = __fsub_rn(total, q[u].z);
          total = __fsub_rn(total, q[u].w);
        }
      }
    }
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
  if (nc > 2048 && nc <= CE_ST_CHUNKS * 2 * CE_ST_THREADS &&
      (ctx->ce_variant == 2 || (ctx->ce_variant == 0 && fast_exp))) {
    // 8192 < V <= 32768 (automatic: the Llama arithmetic only): persistent CTAs
    // streaming their rows through bulk-copied chunks
    const int cf4 = (nc + CE_ST_CHUNKS - 1) / CE_ST_CHUNKS;  // <= 1024 float4: a chunk is at most 16 KiB
    const size_t slot_bytes = static_cast<size_t>(cf4) * sizeof(float4);
    int nslots = static_cast<int>(CE_ST_SMEM_BYTES / slot_bytes);  // >= 14 >= CE_ST_CHUNKS: a whole row fits
    if (nslots > CE_ST_MAX_SLOTS) nslots = CE_ST_MAX_SLOTS;
    const size_t smem = static_cast<size_t>(nslots) * slot_bytes;
    const int grid = rows < ctx->num_sms ? rows : ctx->num_sms;
    auto kern = cf4 <= CE_ST_THREADS ? (fast_exp ? ce_stream_kernel<1, true> : ce_stream_kernel<1, false>)
                                     : (fast_exp ? ce_stream_kernel<2, true> : ce_stream_kernel<2, false>);
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return ctx->fail_cuda(e, "softmax_ce: shared memory attribute");
    ProfScope prof(ctx, PROF_CE, 4.0 * static_cast<double>(rows) * V * (write_grad ? 2 : 1), s);
    glc::launch_pdl(ctx, kern, grid, CE_ST_THREADS, smem, s, logits, targets, rows, V, cf4, nslots, scale, row_logp, wg,
                    ro, ctx->d_err);
    GLC_LAUNCH_CHECK(ctx, "softmax_ce (streamed rows)");
    glc::launch_pdl(ctx, ce_loss_sum_kernel, 1, CE_LS_THREADS, 0, s, row_logp, targets, rows, V, loss);
    GLC_LAUNCH_CHECK(ctx, "softmax_ce loss");
    return 0;
  }
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
    glc::launch_pdl(ctx, ce_loss_sum_kernel, 1, CE_LS_THREADS, 0, s, row_logp, targets, rows, V, loss);
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
  glc::launch_pdl(ctx, ce_loss_sum_kernel, 1, CE_LS_THREADS, 0, s, row_logp, targets, rows, V, loss);
  GLC_LAUNCH_CHECK(ctx, "softmax_ce loss");
  return 0;
}

}  // namespace glc
