// RMSNorm forward and backward (RMSNormTrainable, pkg/train/trainer.go:141-203).
//
// Forward: rms = float32(sqrt(float64(sum x^2)/cols + float64(eps))) per row
// (trainer.go:158-163), y = (x / rms) * w.  One warp per row, float4 loads.
// The per-row rms is saved for the backward.
//
// Backward, two variants:
//   simplified (the reference, trainer.go:182-199): dx += dy*w/rms, dw += dy*x/rms
//   full (Llama mode): dx += dy*w/rms - x * sum_j(dy_j w_j x_j) / (cols*rms^3)
// One block per contiguous chunk of rows; each thread owns a fixed set of
// float4 column chunks so its share of dw accumulates in registers.  Per-block
// dw partials go to scratch memory and a second kernel adds them up in block
// order (deterministic).  The residual-stream gradient dx may also be written
// rounded to TF32 for the tensor-core GEMMs that consume it.
#include "glc_internal.h"
#include "sm100.cuh"

namespace glc {
namespace {

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
  for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
  return v;
}

__global__ void rmsnorm_fwd_kernel(const float* __restrict__ x, const float* __restrict__ w, float* __restrict__ y,
                                   float* __restrict__ rms, int rows, int cols, float eps, int round_out) {
  GLC_PDL_ENTRY();
  const int wpb = blockDim.x >> 5;
  const int lane = threadIdx.x & 31;
  const int nc = cols >> 2;
  const float4* w4 = reinterpret_cast<const float4*>(w);
  for (int row = blockIdx.x * wpb + (threadIdx.x >> 5); row < rows; row += gridDim.x * wpb) {
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * cols);
    float ss = 0.f;
    for (int j = lane; j < nc; j += 32) {
      const float4 v = xr[j];
      ss += v.x * v.x + v.y * v.y + v.z * v.z + v.w * v.w;
    }
    ss = warp_sum(ss);
    const float r = __double2float_rn(sqrt(static_cast<double>(ss) / static_cast<double>(cols) +
                                           static_cast<double>(eps)));
    if (lane == 0) rms[row] = r;
    float4* yr = reinterpret_cast<float4*>(y + static_cast<size_t>(row) * cols);
    for (int j = lane; j < nc; j += 32) {
      const float4 v = xr[j], g = w4[j];
      float4 o;
      o.x = __fmul_rn(__fdiv_rn(v.x, r), g.x);
      o.y = __fmul_rn(__fdiv_rn(v.y, r), g.y);
      o.z = __fmul_rn(__fdiv_rn(v.z, r), g.z);
      o.w = __fmul_rn(__fdiv_rn(v.w, r), g.w);
      if (round_out) {
        o.x = round_tf32(o.x); o.y = round_tf32(o.y); o.z = round_tf32(o.z); o.w = round_tf32(o.w);
      }
      yr[j] = o;
    }
  }
}

template <int MAXC>
__global__ void __launch_bounds__(256) rmsnorm_bwd_kernel(const float* __restrict__ x, const float* __restrict__ w,
                                                          const float* __restrict__ rms, const float* __restrict__ dy,
                                                          float* __restrict__ dx, float* __restrict__ dx_round,
                                                          float* __restrict__ dw_partial, int rows, int cols,
                                                          int rows_per_block, int full, int dx_accumulate) {
  GLC_PDL_ENTRY();
  __shared__ float red[32];
  const int nc = cols >> 2;
  const int tid = threadIdx.x;
  const int row0 = blockIdx.x * rows_per_block;
  const int row1 = min(rows, row0 + rows_per_block);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4 wv[MAXC], acc[MAXC];
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * 256;
    wv[i] = c < nc ? w4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  for (int row = row0; row < row1; ++row) {
    const float r = rms[row];
    const float4* xr = reinterpret_cast<const float4*>(x + static_cast<size_t>(row) * cols);
    const float4* dyr = reinterpret_cast<const float4*>(dy + static_cast<size_t>(row) * cols);
    float4* dxr = reinterpret_cast<float4*>(dx + static_cast<size_t>(row) * cols);
    // the accumulated dx is loaded with x and dy, before the row reduction
    float4 xv[MAXC], dv[MAXC], ov[MAXC];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = tid + i * 256;
      if (c < nc) {
        xv[i] = xr[c];
        dv[i] = dyr[c];
        if (dx_accumulate) ov[i] = dxr[c];
        if (full)
          s += dv[i].x * wv[i].x * xv[i].x + dv[i].y * wv[i].y * xv[i].y + dv[i].z * wv[i].z * xv[i].z +
               dv[i].w * wv[i].w * xv[i].w;
      }
    }
    float coef = 0.f;
    if (full) {
      s = warp_sum(s);
      if ((tid & 31) == 0) red[tid >> 5] = s;
      __syncthreads();
      if (tid < 32) {
        float t = tid < (blockDim.x >> 5) ? red[tid] : 0.f;
        t = warp_sum(t);
        if (tid == 0) red[0] = t;
      }
      __syncthreads();
      const float tot = red[0];
      __syncthreads();
      coef = tot / (static_cast<float>(cols) * r * r * r);
    }
    float4* dxq = dx_round ? reinterpret_cast<float4*>(dx_round + static_cast<size_t>(row) * cols) : nullptr;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = tid + i * 256;
      if (c < nc) {
        float4 g;
        g.x = __fdiv_rn(__fmul_rn(dv[i].x, wv[i].x), r);
        g.y = __fdiv_rn(__fmul_rn(dv[i].y, wv[i].y), r);
        g.z = __fdiv_rn(__fmul_rn(dv[i].z, wv[i].z), r);
        g.w = __fdiv_rn(__fmul_rn(dv[i].w, wv[i].w), r);
        if (full) {
          g.x = __fsub_rn(g.x, __fmul_rn(xv[i].x, coef));
          g.y = __fsub_rn(g.y, __fmul_rn(xv[i].y, coef));
          g.z = __fsub_rn(g.z, __fmul_rn(xv[i].z, coef));
          g.w = __fsub_rn(g.w, __fmul_rn(xv[i].w, coef));
        }
        if (dx_accumulate) {
          const float4 o = ov[i];
          g.x = __fadd_rn(o.x, g.x); g.y = __fadd_rn(o.y, g.y); g.z = __fadd_rn(o.z, g.z); g.w = __fadd_rn(o.w, g.w);
        }
        dxr[c] = g;
        if (dxq) dxq[c] = make_float4(round_tf32(g.x), round_tf32(g.y), round_tf32(g.z), round_tf32(g.w));
        acc[i].x += __fdiv_rn(__fmul_rn(dv[i].x, xv[i].x), r);
        acc[i].y += __fdiv_rn(__fmul_rn(dv[i].y, xv[i].y), r);
        acc[i].z += __fdiv_rn(__fmul_rn(dv[i].z, xv[i].z), r);
        acc[i].w += __fdiv_rn(__fmul_rn(dv[i].w, xv[i].w), r);
      }
    }
  }
  float4* part = reinterpret_cast<float4*>(dw_partial + static_cast<size_t>(blockIdx.x) * cols);
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * 256;
    if (c < nc) part[c] = acc[i];
  }
}

// The same backward with the row loads pipelined: each thread copies its own
// float4 chunks of x, dy (and the accumulated dx) for the next PIPE_STAGES - 1
// rows into shared memory with cp.async while it computes the current row, so
// the rows' load latency overlaps the block reduction instead of following
// it.  A thread reads back only the chunks it copied itself, so the pipeline
// needs no barrier beyond the per-thread cp.async.wait_group; a stage is
// refilled only after the values read from it were used (data dependence
// orders the reads before the copy that overwrites them).  The arithmetic and
// its order are the kernel above's: results are bit-identical.
// Shared layout: [stage][array x/dy/dx][MAXC][256 threads] float4, so a warp's
// 16-byte accesses are contiguous.
constexpr int PIPE_STAGES = 3;

__device__ __forceinline__ void cp_async16(void* smem_dst, const void* gsrc) {
  asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(smem_dst)), "l"(gsrc) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
  asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

template <int MAXC>
__global__ void __launch_bounds__(256) rmsnorm_bwd_pipe_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ rms,
    const float* __restrict__ dy, float* __restrict__ dx, float* __restrict__ dx_round,
    float* __restrict__ dw_partial, int rows, int cols, int rows_per_block, int full, int dx_accumulate) {
  GLC_PDL_ENTRY();
  extern __shared__ float4 stage_buf[];  // PIPE_STAGES * 3 * MAXC * 256
  __shared__ float red[32];
  const int nc = cols >> 2;
  const int tid = threadIdx.x;
  const int row0 = blockIdx.x * rows_per_block;
  const int row1 = min(rows, row0 + rows_per_block);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  auto slot = [&](int st, int arr, int i) -> float4* { return stage_buf + ((st * 3 + arr) * MAXC + i) * 256 + tid; };
  // copies of row `row` into stage `st` (this thread's chunks only)
  auto issue = [&](int row, int st) {
    if (row < row1) {
      const size_t base = static_cast<size_t>(row) * cols;
#pragma unroll
      for (int i = 0; i < MAXC; ++i) {
        const int c = tid + i * 256;
        if (c < nc) {
          cp_async16(slot(st, 0, i), x + base + 4 * c);
          cp_async16(slot(st, 1, i), dy + base + 4 * c);
          if (dx_accumulate) cp_async16(slot(st, 2, i), dx + base + 4 * c);
        }
      }
    }
    cp_async_commit();  // one group per row slot, empty past the block's rows
  };
  float4 wv[MAXC], acc[MAXC];
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * 256;
    wv[i] = c < nc ? w4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
#pragma unroll
  for (int s = 0; s < PIPE_STAGES - 1; ++s) issue(row0 + s, s);
  int st = 0;
  for (int row = row0; row < row1; ++row) {
    // refill the stage the previous row used, then wait for this row's group
    issue(row + PIPE_STAGES - 1, (st + PIPE_STAGES - 1) % PIPE_STAGES);
    cp_async_wait<PIPE_STAGES - 1>();
    const float r = rms[row];
    float4* dxr = reinterpret_cast<float4*>(dx + static_cast<size_t>(row) * cols);
    float4 xv[MAXC], dv[MAXC], ov[MAXC];
    float s = 0.f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = tid + i * 256;
      if (c < nc) {
        xv[i] = *slot(st, 0, i);
        dv[i] = *slot(st, 1, i);
        if (dx_accumulate) ov[i] = *slot(st, 2, i);
        if (full)
          s += dv[i].x * wv[i].x * xv[i].x + dv[i].y * wv[i].y * xv[i].y + dv[i].z * wv[i].z * xv[i].z +
               dv[i].w * wv[i].w * xv[i].w;
      }
    }
    float coef = 0.f;
    if (full) {
      s = warp_sum(s);
      if ((tid & 31) == 0) red[tid >> 5] = s;
      __syncthreads();
      if (tid < 32) {
        float t = tid < (blockDim.x >> 5) ? red[tid] : 0.f;
        t = warp_sum(t);
        if (tid == 0) red[0] = t;
      }
      __syncthreads();
      const float tot = red[0];
      __syncthreads();
      coef = tot / (static_cast<float>(cols) * r * r * r);
    }
    float4* dxq = dx_round ? reinterpret_cast<float4*>(dx_round + static_cast<size_t>(row) * cols) : nullptr;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = tid + i * 256;
      if (c < nc) {
        float4 g;
        g.x = __fdiv_rn(__fmul_rn(dv[i].x, wv[i].x), r);
        g.y = __fdiv_rn(__fmul_rn(dv[i].y, wv[i].y), r);
        g.z = __fdiv_rn(__fmul_rn(dv[i].z, wv[i].z), r);
        g.w = __fdiv_rn(__fmul_rn(dv[i].w, wv[i].w), r);
        if (full) {
          g.x = __fsub_rn(g.x, __fmul_rn(xv[i].x, coef));
          g.y = __fsub_rn(g.y, __fmul_rn(xv[i].y, coef));
          g.z = __fsub_rn(g.z, __fmul_rn(xv[i].z, coef));
          g.w = __fsub_rn(g.w, __fmul_rn(xv[i].w, coef));
        }
        if (dx_accumulate) {
          const float4 o = ov[i];
          g.x = __fadd_rn(o.x, g.x); g.y = __fadd_rn(o.y, g.y); g.z = __fadd_rn(o.z, g.z); g.w = __fadd_rn(o.w, g.w);
        }
        dxr[c] = g;
        if (dxq) dxq[c] = make_float4(round_tf32(g.x), round_tf32(g.y), round_tf32(g.z), round_tf32(g.w));
        acc[i].x += __fdiv_rn(__fmul_rn(dv[i].x, xv[i].x), r);
        acc[i].y += __fdiv_rn(__fmul_rn(dv[i].y, xv[i].y), r);
        acc[i].z += __fdiv_rn(__fmul_rn(dv[i].z, xv[i].z), r);
        acc[i].w += __fdiv_rn(__fmul_rn(dv[i].w, xv[i].w), r);
      }
    }
    st = st + 1 == PIPE_STAGES ? 0 : st + 1;
  }
  cp_async_wait<0>();  // no copy outlives the block (groups past the last row are empty)
  float4* part = reinterpret_cast<float4*>(dw_partial + static_cast<size_t>(blockIdx.x) * cols);
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * 256;
    if (c < nc) part[c] = acc[i];
  }
}

// The exact (Llama) backward with whole rows staged by bulk copies: one
// thread streams the rows of x, dy (and the accumulated dx) of a block's
// chunk into a ring of TMA_STAGES shared-memory stages (cp.async.bulk, one
// mbarrier per stage), so several rows per block are in flight while the
// current one is reduced; two 96 KB blocks fit an SM, eight rows in flight.
// The row's 1/rms is applied as a product (the reference-semantics kernel
// above divides, bit for bit with the reference; the exact gradient has no
// reference bits to match), dw partials per block as above.
constexpr int TMA_STAGES = 4;

template <int MAXC>
__global__ void __launch_bounds__(256) rmsnorm_bwd_full_tma_kernel(
    const float* __restrict__ x, const float* __restrict__ w, const float* __restrict__ rms,
    const float* __restrict__ dy, float* __restrict__ dx, float* __restrict__ dx_round,
    float* __restrict__ dw_partial, int rows, int cols, int rows_per_block, int dx_accumulate, int* err) {
  GLC_PDL_ENTRY();
  extern __shared__ __align__(16) float stage_rows[];  // [TMA_STAGES][3][cols], then the barriers
  __shared__ float red[32];
  __shared__ int abort_flag;
  uint64_t* full = reinterpret_cast<uint64_t*>(stage_rows + static_cast<size_t>(TMA_STAGES) * 3 * cols);
  const int nc = cols >> 2;
  const int tid = threadIdx.x;
  const int row0 = blockIdx.x * rows_per_block;
  const int row1 = min(rows, row0 + rows_per_block);
  const uint32_t row_bytes = static_cast<uint32_t>(cols) * 4u;
  const uint32_t stage_bytes = (dx_accumulate ? 3u : 2u) * row_bytes;
  auto stage = [&](int st, int arr) { return stage_rows + (static_cast<size_t>(st) * 3 + arr) * cols; };
  auto issue = [&](int row, int st) {  // thread 0 only
    const size_t base = static_cast<size_t>(row) * cols;
    mbar_arrive_expect_tx(&full[st], stage_bytes);
    bulk_load(stage(st, 0), x + base, row_bytes, &full[st]);
    bulk_load(stage(st, 1), dy + base, row_bytes, &full[st]);
    if (dx_accumulate) bulk_load(stage(st, 2), dx + base, row_bytes, &full[st]);
  };
  if (tid == 0) {
    for (int i = 0; i < TMA_STAGES; ++i) mbar_init(&full[i], 1);
    abort_flag = 0;
    fence_mbar_init();
  }
  __syncthreads();
  int issued = 0;  // rows whose copies thread 0 has issued
  if (tid == 0)
    for (; issued < TMA_STAGES && row0 + issued < row1; ++issued) issue(row0 + issued, issued);
  const float4* w4 = reinterpret_cast<const float4*>(w);
  float4 wv[MAXC], acc[MAXC];
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * 256;
    wv[i] = c < nc ? w4[c] : make_float4(0.f, 0.f, 0.f, 0.f);
    acc[i] = make_float4(0.f, 0.f, 0.f, 0.f);
  }
  const float inv_cols = 1.0f / static_cast<float>(cols);
  bool ok = true;
  int row = row0;  // on abort: the row whose copies the wait gave up on
  for (; row < row1; ++row) {
    const int k = row - row0, st = k % TMA_STAGES;
    if (!__syncthreads_and(mbar_wait(&full[st], (k / TMA_STAGES) & 1, &abort_flag, err, GLC_DEV_TIMEOUT_EPILOGUE))) {
      ok = false;
      break;
    }
    const float rinv = 1.0f / rms[row];
    const float4* xs = reinterpret_cast<const float4*>(stage(st, 0));
    const float4* ds = reinterpret_cast<const float4*>(stage(st, 1));
    const float4* os = reinterpret_cast<const float4*>(stage(st, 2));
    float4 xv[MAXC], dv[MAXC], ov[MAXC];
    float sdot = 0.f;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = tid + i * 256;
      if (c < nc) {
        xv[i] = xs[c];
        dv[i] = ds[c];
        if (dx_accumulate) ov[i] = os[c];
        sdot += dv[i].x * wv[i].x * xv[i].x + dv[i].y * wv[i].y * xv[i].y + dv[i].z * wv[i].z * xv[i].z +
                dv[i].w * wv[i].w * xv[i].w;
      }
    }
    sdot = warp_sum(sdot);
    if ((tid & 31) == 0) red[tid >> 5] = sdot;
    __syncthreads();  // also: every thread holds this row's values, the stage may be refilled
    if (tid == 0 && issued < row1 - row0) {
      issue(row0 + issued, issued % TMA_STAGES);
      ++issued;
    }
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float coef = tot * inv_cols * rinv * rinv * rinv;
    float4* dxr = reinterpret_cast<float4*>(dx + static_cast<size_t>(row) * cols);
    float4* dxq = dx_round ? reinterpret_cast<float4*>(dx_round + static_cast<size_t>(row) * cols) : nullptr;
#pragma unroll
    for (int i = 0; i < MAXC; ++i) {
      const int c = tid + i * 256;
      if (c < nc) {
        float4 g;
        g.x = dv[i].x * wv[i].x * rinv - xv[i].x * coef;
        g.y = dv[i].y * wv[i].y * rinv - xv[i].y * coef;
        g.z = dv[i].z * wv[i].z * rinv - xv[i].z * coef;
        g.w = dv[i].w * wv[i].w * rinv - xv[i].w * coef;
        if (dx_accumulate) {
          g.x += ov[i].x; g.y += ov[i].y; g.z += ov[i].z; g.w += ov[i].w;
        }
        dxr[c] = g;
        if (dxq) dxq[c] = make_float4(round_tf32(g.x), round_tf32(g.y), round_tf32(g.z), round_tf32(g.w));
        acc[i].x += dv[i].x * xv[i].x * rinv;
        acc[i].y += dv[i].y * xv[i].y * rinv;
        acc[i].z += dv[i].z * xv[i].z * rinv;
        acc[i].w += dv[i].w * xv[i].w * rinv;
      }
    }
    __syncthreads();  // red is rewritten by the next row
  }
  if (!ok && tid == 0) {
    // No copy may land after the block exits: wait (bounded) for those in
    // flight, the rows from the one whose wait gave up to the last issued,
    // each in its own stage.  The rows before it were read, and their stages
    // may since have completed a later phase: a parity wait on them would
    // name the wrong phase and spin to its limit.
    for (int r = row; r < row0 + issued; ++r) {
      const int k = r - row0;
      mbar_drain(&full[k % TMA_STAGES], (k / TMA_STAGES) & 1, err);
    }
  }
  float4* part = reinterpret_cast<float4*>(dw_partial + static_cast<size_t>(blockIdx.x) * cols);
#pragma unroll
  for (int i = 0; i < MAXC; ++i) {
    const int c = tid + i * 256;
    if (c < nc) part[c] = acc[i];
  }
}

// dw[j] (+)= sum over blocks b of partial[b][j].  A cluster of CS_CL CTAs
// per 32 columns: CTA rank r adds the partial rows of its quarter
// [r*q, (r+1)*q), each of its 16 warps keeping four running sums (rows
// w + 16*(4i + c), added in order c = 0..3), the warps' sums added in warp
// order; rank 0 then adds the CS_CL quarter sums in rank order through
// distributed shared memory (deterministic).
constexpr int CS_CL = 4;
constexpr int CS_WARPS = 16;
__global__ void __cluster_dims__(CS_CL, 1, 1) __launch_bounds__(CS_WARPS * 32)
    column_sum_kernel(const float* __restrict__ partial, int nblocks, int cols, float* __restrict__ out,
                      int accumulate) {
  GLC_PDL_ENTRY();
  __shared__ float red[CS_WARPS][33];
  __shared__ float quarter[32];
  const int lane = threadIdx.x & 31, w = threadIdx.x >> 5;
  const int rank = static_cast<int>(cluster_ctarank());
  const int j = static_cast<int>(blockIdx.x / CS_CL) * 32 + lane;
  const int q = (nblocks + CS_CL - 1) / CS_CL;
  const int b0 = rank * q, b1 = min(nblocks, b0 + q);
  float s = 0.f;
  if (j < cols) {
    float c4[4] = {0.f, 0.f, 0.f, 0.f};
    int b = b0 + w;
    for (; b + 3 * CS_WARPS < b1; b += 4 * CS_WARPS) {
#pragma unroll
      for (int c = 0; c < 4; ++c) c4[c] += partial[static_cast<size_t>(b + CS_WARPS * c) * cols + j];
    }
#pragma unroll
    for (int c = 0; c < 4; ++c)
      if (b + CS_WARPS * c < b1) c4[c] += partial[static_cast<size_t>(b + CS_WARPS * c) * cols + j];
    s = ((c4[0] + c4[1]) + c4[2]) + c4[3];
  }
  red[w][lane] = s;
  __syncthreads();
  if (w == 0) {
    float t = 0.f;
#pragma unroll
    for (int k = 0; k < CS_WARPS; ++k) t += red[k][lane];
    quarter[lane] = t;
  }
  cluster_sync_all();
  if (rank == 0 && w == 0 && j < cols) {
    float t = ld_shared_cluster_f32(mapa_cluster(&quarter[lane], 0));
#pragma unroll
    for (int r = 1; r < CS_CL; ++r) t += ld_shared_cluster_f32(mapa_cluster(&quarter[lane], r));
    out[j] = accumulate ? __fadd_rn(out[j], t) : t;
  }
  // the peers' quarter sums stay in place until rank 0 has read them
  cluster_sync_all();
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

}  // namespace

int rmsnorm_fwd(Context* ctx, const float* x, const float* w, float* y, float* rms, int rows, int cols, float eps,
                bool round_out, cudaStream_t s) {
  if (rows < 0 || cols <= 0 || (cols & 3)) return ctx->fail(GLC_ERR_INVALID, "rmsnorm_fwd: cols must be a positive multiple of 4");
  if (rows == 0) return 0;
  if (!x || !w || !y || !rms || !aligned16(x) || !aligned16(w) || !aligned16(y))
    return ctx->fail(GLC_ERR_INVALID, "rmsnorm_fwd: null or misaligned pointer");
  const int wpb = 8;
  unsigned grid = static_cast<unsigned>((rows + wpb - 1) / wpb);
  ProfScope prof(ctx, PROF_RMSNORM, 4.0 * (2.0 * rows * cols + rows + cols), s);
  glc::launch_pdl(ctx, rmsnorm_fwd_kernel, grid, wpb * 32, 0, s, x, w, y, rms, rows, cols, eps, round_out ? 1 : 0);
  GLC_LAUNCH_CHECK(ctx, "rmsnorm_fwd");
  return 0;
}

int rmsnorm_bwd(Context* ctx, const float* x, const float* w, const float* rms, const float* dy, float* dx,
                float* dx_round, float* dw, int rows, int cols, bool full, bool dx_accumulate, bool dw_accumulate,
                float* scratch, size_t scratch_bytes, cudaStream_t s) {
  if (rows < 0 || cols <= 0 || (cols & 3)) return ctx->fail(GLC_ERR_INVALID, "rmsnorm_bwd: cols must be a positive multiple of 4");
  const int nc = cols / 4;
  if (nc > 8 * 256) return ctx->fail(GLC_ERR_INVALID, "rmsnorm_bwd: cols above 8192 are not supported");
  if (rows == 0) {
    if (dw && !dw_accumulate) {
      cudaError_t e = cudaMemsetAsync(dw, 0, sizeof(float) * cols, s);
      if (e != cudaSuccess) return ctx->fail_cuda(e, "rmsnorm_bwd: memset");
    }
    return 0;
  }
  if (!x || !w || !rms || !dy || !dx || !dw || !aligned16(x) || !aligned16(w) || !aligned16(dy) || !aligned16(dx) ||
      (dx_round && !aligned16(dx_round)))
    return ctx->fail(GLC_ERR_INVALID, "rmsnorm_bwd: null or misaligned pointer");
  // pipelined variant (opt-in): rows up to 2048 columns.  Both variants split
  // the rows over the same blocks, so the per-block dw partials (and their
  // sum) are the same bits; the pipelined kernel fits three blocks per SM.
  const bool pipe = ctx->rmsnorm_variant == 2 && nc <= 512;
  // the exact gradient streams whole rows through bulk copies (automatic, or
  // variant 3): rows of up to 2048 columns, two blocks per SM
  const bool tma = full && nc <= 512 && (ctx->rmsnorm_variant == 0 || ctx->rmsnorm_variant == 3);
  int nblocks = (tma ? 2 : 4) * ctx->num_sms;
  if (nblocks > rows) nblocks = rows;
  const int rpb = (rows + nblocks - 1) / nblocks;
  nblocks = (rows + rpb - 1) / rpb;
  const size_t need = static_cast<size_t>(nblocks) * cols * sizeof(float);
  float* partial = scratch;
  if (partial == nullptr) {
    void* ws = nullptr;
    int rc = ctx->workspace(need, &ws);
    if (rc) return rc;
    partial = static_cast<float*>(ws);
  } else if (scratch_bytes < need) {
    return ctx->fail(GLC_ERR_INVALID, "rmsnorm_bwd: scratch buffer too small");
  }
  const int fl = full ? 1 : 0, acc = dx_accumulate ? 1 : 0;
  ProfScope prof(ctx, PROF_RMSNORM,
                 4.0 * static_cast<double>(rows) * cols * (3 + (dx_accumulate ? 1 : 0) + (dx_round ? 1 : 0)) + 4.0 * rows,
                 s);
  if (tma) {
    const int maxc = nc <= 256 ? 1 : 2;
    const size_t smem = sizeof(float) * TMA_STAGES * 3 * static_cast<size_t>(cols) + 8 * TMA_STAGES;
    auto kern = maxc == 1 ? rmsnorm_bwd_full_tma_kernel<1> : rmsnorm_bwd_full_tma_kernel<2>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return ctx->fail_cuda(e, "rmsnorm_bwd: shared memory attribute");
    glc::launch_pdl(ctx, kern, nblocks, 256, smem, s, x, w, rms, dy, dx, dx_round, partial, rows, cols, rpb, acc,
                    ctx->d_err);
  } else if (pipe) {
    const int maxc = nc <= 256 ? 1 : 2;
    const size_t smem = sizeof(float4) * PIPE_STAGES * 3 * maxc * 256;
    auto kern = maxc == 1 ? rmsnorm_bwd_pipe_kernel<1> : rmsnorm_bwd_pipe_kernel<2>;
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(smem));
    if (e != cudaSuccess) return ctx->fail_cuda(e, "rmsnorm_bwd: shared memory attribute");
    glc::launch_pdl(ctx, kern, nblocks, 256, smem, s, x, w, rms, dy, dx, dx_round, partial, rows, cols, rpb, fl, acc);
  } else if (nc <= 256)
    glc::launch_pdl(ctx, rmsnorm_bwd_kernel<1>, nblocks, 256, 0, s, x, w, rms, dy, dx, dx_round, partial, rows, cols, rpb, fl, acc);
  else if (nc <= 512)
    glc::launch_pdl(ctx, rmsnorm_bwd_kernel<2>, nblocks, 256, 0, s, x, w, rms, dy, dx, dx_round, partial, rows, cols, rpb, fl, acc);
  else if (nc <= 1024)
    glc::launch_pdl(ctx, rmsnorm_bwd_kernel<4>, nblocks, 256, 0, s, x, w, rms, dy, dx, dx_round, partial, rows, cols, rpb, fl, acc);
  else
    glc::launch_pdl(ctx, rmsnorm_bwd_kernel<8>, nblocks, 256, 0, s, x, w, rms, dy, dx, dx_round, partial, rows, cols, rpb, fl, acc);
  GLC_LAUNCH_CHECK(ctx, "rmsnorm_bwd");
  glc::launch_pdl(ctx, column_sum_kernel, ((cols + 31) / 32) * CS_CL, CS_WARPS * 32, 0, s, partial, nblocks, cols, dw,
                  dw_accumulate ? 1 : 0);
  GLC_LAUNCH_CHECK(ctx, "rmsnorm_bwd column sum");
  return 0;
}

}  // namespace glc
