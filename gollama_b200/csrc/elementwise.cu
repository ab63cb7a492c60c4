// Bandwidth-bound elementwise kernels: SwiGLU forward/backward, RoPE,
// embedding gather / gradient scatter, fills and TF32 rounding copies.
#include "glc_internal.h"
#include "go_math.cuh"
#include "sm100.cuh"

namespace glc {
namespace {

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; }

// ---------------------------------------------------------------- SwiGLU
// Forward of forwardFFN's SiLU and product nodes (trainer.go:397-407 with
// SiLUGrad, grad.go:424-428): s = 1/(1+exp32(-g)), h = (g*s)*u.
// FAST: llama semantics (sigmoid_f / swiglu_f in go_math.cuh).

// 2-D launch: blockIdx.x/threadIdx.x pick a float4 column, blockIdx.y strides
// over rows (32-bit index arithmetic, no per-element division).
template <bool FAST>
__global__ void swiglu_fwd_kernel(const float* __restrict__ g, const float* __restrict__ u, size_t ld_in,
                                  float* __restrict__ h, size_t ld_h, unsigned rows, unsigned cols4, int round_out) {
  GLC_PDL_ENTRY();
  const unsigned c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols4) return;
  for (unsigned r = blockIdx.y; r < rows; r += gridDim.y) {
    const float4 a = reinterpret_cast<const float4*>(g + r * ld_in)[c];
    const float4 b = reinterpret_cast<const float4*>(u + r * ld_in)[c];
    float4 o = make_float4(swiglu_f<FAST>(a.x, b.x), swiglu_f<FAST>(a.y, b.y), swiglu_f<FAST>(a.z, b.z),
                           swiglu_f<FAST>(a.w, b.w));
    if (round_out) o = make_float4(round_tf32(o.x), round_tf32(o.y), round_tf32(o.z), round_tf32(o.w));
    reinterpret_cast<float4*>(h + r * ld_h)[c] = o;
  }
}

// Backward of the product node (trainer.go:418-421) then SiLU (grad.go:441-445):
//   dgs = dh*u, du = dh*(g*s), dg = dgs * (s*(1 + g*(1-s)))
template <bool FAST>
__device__ __forceinline__ void swiglu_b(float g, float u, float dh, float& dg, float& du) {
  const float s = sigmoid_f<FAST>(g);
  const float gs = __fmul_rn(g, s);
  const float dgs = __fmul_rn(dh, u);
  du = __fmul_rn(dh, gs);
  const float grad = __fmul_rn(s, __fadd_rn(1.0f, __fmul_rn(g, __fsub_rn(1.0f, s))));
  dg = __fmul_rn(dgs, grad);
}

template <bool FAST>
__global__ void swiglu_bwd_kernel(const float* __restrict__ g, const float* __restrict__ u, size_t ld_in,
                                  const float* __restrict__ dh, size_t ld_dh, float* __restrict__ dg,
                                  float* __restrict__ du, size_t ld_out, unsigned rows, unsigned cols4, int accumulate,
                                  int round_out) {
  GLC_PDL_ENTRY();
  const unsigned c = blockIdx.x * blockDim.x + threadIdx.x;
  if (c >= cols4) return;
  for (unsigned r = blockIdx.y; r < rows; r += gridDim.y) {
    const float4 a = reinterpret_cast<const float4*>(g + r * ld_in)[c];
    const float4 b = reinterpret_cast<const float4*>(u + r * ld_in)[c];
    const float4 d = reinterpret_cast<const float4*>(dh + r * ld_dh)[c];
    float4 rg, ru;
    swiglu_b<FAST>(a.x, b.x, d.x, rg.x, ru.x);
    swiglu_b<FAST>(a.y, b.y, d.y, rg.y, ru.y);
    swiglu_b<FAST>(a.z, b.z, d.z, rg.z, ru.z);
    swiglu_b<FAST>(a.w, b.w, d.w, rg.w, ru.w);
    float4* pg = reinterpret_cast<float4*>(dg + r * ld_out) + c;
    float4* pu = reinterpret_cast<float4*>(du + r * ld_out) + c;
    if (accumulate) {
      const float4 og = *pg, ou = *pu;
      rg = make_float4(__fadd_rn(og.x, rg.x), __fadd_rn(og.y, rg.y), __fadd_rn(og.z, rg.z), __fadd_rn(og.w, rg.w));
      ru = make_float4(__fadd_rn(ou.x, ru.x), __fadd_rn(ou.y, ru.y), __fadd_rn(ou.z, ru.z), __fadd_rn(ou.w, ru.w));
    }
    if (round_out) {
      rg = make_float4(round_tf32(rg.x), round_tf32(rg.y), round_tf32(rg.z), round_tf32(rg.w));
      ru = make_float4(round_tf32(ru.x), round_tf32(ru.y), round_tf32(ru.z), round_tf32(ru.w));
    }
    *pg = rg;
    *pu = ru;
  }
}

// Grid of a row-strided 2-D elementwise launch: enough column blocks to
// cover cols4 float4s, rows spread so the whole launch has ~16 blocks per SM.
inline dim3 grid_2d(size_t rows, size_t cols4, int block, int num_sms) {
  const unsigned bx = static_cast<unsigned>((cols4 + block - 1) / block);
  size_t by = (static_cast<size_t>(num_sms) * 16 + bx - 1) / bx;
  if (by > rows) by = rows;
  if (by > 65535) by = 65535;
  if (by < 1) by = 1;
  return dim3(bx, static_cast<unsigned>(by));
}

// ---------------------------------------------------------------- fills / copies
__global__ void fill_kernel(float* __restrict__ p, float v, size_t n) {
  GLC_PDL_ENTRY();
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x) p[i] = v;
}

__global__ void add_inplace_kernel(float* __restrict__ dst, const float* __restrict__ src, size_t n) {
  GLC_PDL_ENTRY();
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    dst[i] = __fadd_rn(dst[i], src[i]);
}

__global__ void round_copy_kernel(const float* __restrict__ src, float* __restrict__ dst, size_t n) {
  GLC_PDL_ENTRY();
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < n; i += size_t(gridDim.x) * blockDim.x)
    dst[i] = round_tf32(src[i]);
}

// ---------------------------------------------------------------- RoPE
// apply3D (pkg/model/rope.go:96-126) on rows of nh heads x hd, consecutive
// pairs, position t % S; inverse = 1 applies the transposed rotation (the
// backward).  In place; optional TF32 rounding of the result.
// Launch: blockIdx.y strides over tokens; the threads of a block cover the
// row's nh*hd/2 pairs (blockDim.x * gridDim.x >= pairs per row).
__global__ void rope_kernel(float* __restrict__ x, size_t ld, int T, int S, int nh, int hd,
                            const float* __restrict__ cos_t, const float* __restrict__ sin_t, int inverse,
                            int round_out) {
  GLC_PDL_ENTRY();
  const int half = hd >> 1;
  const int q = blockIdx.x * blockDim.x + threadIdx.x;  // pair index inside the row: head * half + i
  if (q >= nh * half) return;
  const int hh = q / half, i = q - hh * half;
  for (int t = blockIdx.y; t < T; t += gridDim.y) {
    const int pos = t % S;
    const float c = cos_t[pos * half + i], s = sin_t[pos * half + i];
    float2* xp = reinterpret_cast<float2*>(x + static_cast<size_t>(t) * ld + static_cast<size_t>(hh) * hd) + i;
    const float2 v = *xp;
    float2 o;
    if (!inverse) {
      o.x = __fsub_rn(__fmul_rn(v.x, c), __fmul_rn(v.y, s));
      o.y = __fadd_rn(__fmul_rn(v.x, s), __fmul_rn(v.y, c));
    } else {
      o.x = __fadd_rn(__fmul_rn(v.x, c), __fmul_rn(v.y, s));
      o.y = __fadd_rn(__fmul_rn(-v.x, s), __fmul_rn(v.y, c));
    }
    if (round_out) {
      o.x = round_tf32(o.x);
      o.y = round_tf32(o.y);
    }
    *xp = o;
  }
}

// The same two pairs at a time (float4 of x, float2 of the tables) when the
// head size and row stride are multiples of 4 floats and x is 16-byte
// aligned; identical operations per pair.
__device__ __forceinline__ float2 rope_pair(float a, float b, float c, float s, int inverse, int round_out) {
  float2 o;
  if (!inverse) {
    o.x = __fsub_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    o.y = __fadd_rn(__fmul_rn(a, s), __fmul_rn(b, c));
  } else {
    o.x = __fadd_rn(__fmul_rn(a, c), __fmul_rn(b, s));
    o.y = __fadd_rn(__fmul_rn(-a, s), __fmul_rn(b, c));
  }
  if (round_out) {
    o.x = round_tf32(o.x);
    o.y = round_tf32(o.y);
  }
  return o;
}
__global__ void rope4_kernel(float* __restrict__ x, size_t ld, int T, int S, int nh, int hd,
                             const float* __restrict__ cos_t, const float* __restrict__ sin_t, int inverse,
                             int round_out) {
  GLC_PDL_ENTRY();
  const int half = hd >> 1, quads = hd >> 2;
  const int qq = blockIdx.x * blockDim.x + threadIdx.x;  // head * quads + j: pairs 2j and 2j+1 of the head
  if (qq >= nh * quads) return;
  const int hh = qq / quads, j = qq - hh * quads;
  for (int t = blockIdx.y; t < T; t += gridDim.y) {
    const int pos = t % S;
    const float2 c = reinterpret_cast<const float2*>(cos_t + pos * half)[j];
    const float2 s = reinterpret_cast<const float2*>(sin_t + pos * half)[j];
    float4* xp = reinterpret_cast<float4*>(x + static_cast<size_t>(t) * ld + static_cast<size_t>(hh) * hd) + j;
    const float4 v = *xp;
    const float2 o0 = rope_pair(v.x, v.y, c.x, s.x, inverse, round_out);
    const float2 o1 = rope_pair(v.z, v.w, c.y, s.y, inverse, round_out);
    *xp = make_float4(o0.x, o0.y, o1.x, o1.y);
  }
}

// ---------------------------------------------------------------- embedding
// Forward (trainer.go:276-289): h[t] = E[tok] (+ P[t % S]); ids outside
// [0, V) read row 0.
__global__ void embed_fwd_kernel(const int64_t* __restrict__ tok, const float* __restrict__ E,
                                 const float* __restrict__ P, float* __restrict__ out, int T, int S, int d, int V) {
  GLC_PDL_ENTRY();
  const int nc = d >> 2;
  const size_t total = static_cast<size_t>(T) * nc;
  for (size_t i = blockIdx.x * size_t(blockDim.x) + threadIdx.x; i < total; i += size_t(gridDim.x) * blockDim.x) {
    const int t = static_cast<int>(i / nc), c = static_cast<int>(i % nc);
    int64_t id = tok[t];
    if (id < 0 || id >= V) id = 0;
    float4 v = reinterpret_cast<const float4*>(E + id * d)[c];
    if (P) {
      const float4 p = reinterpret_cast<const float4*>(P + static_cast<size_t>(t % S) * d)[c];
      v = make_float4(__fadd_rn(v.x, p.x), __fadd_rn(v.y, p.y), __fadd_rn(v.z, p.z), __fadd_rn(v.w, p.w));
    }
    reinterpret_cast<float4*>(out + static_cast<size_t>(t) * d)[c] = v;
  }
}

// The segments of the gradient scatter, built on the device: the token
// positions t stably sorted by their (clamped) id, the distinct ids in
// ascending order and where each one's run starts, as the host's
// std::stable_sort would give them.  One CTA of 1024 threads: a least-
// significant-digit radix sort over 8-bit digits of the id (as many passes as
// V - 1 has bytes), each pass stable (tiles of 1024 positions in order; in a
// tile, warps in order, and lanes in order through __match_any_sync), then a
// block-wide scan of the run heads.  Scratch: 4 * T ints (two key/position
// buffers).  Outputs: seg_tok[nseg], seg_start[nseg + 1], order[T], *nseg_out.
constexpr int SEG_THREADS = 1024, SEG_RADIX = 256, SEG_WARPS = SEG_THREADS / 32;

__global__ void __launch_bounds__(SEG_THREADS, 1)
    embed_segments_kernel(const int64_t* __restrict__ tok, int T, int V, int passes, int* __restrict__ scratch,
                          int* __restrict__ seg_tok, int* __restrict__ seg_start, int* __restrict__ order,
                          int* __restrict__ nseg_out) {
  GLC_PDL_ENTRY();
  __shared__ int base[SEG_RADIX], tile_total[SEG_RADIX];
  __shared__ int warp_cnt[SEG_WARPS][SEG_RADIX + 1];  // +1: the idle lanes' digit of a partial tile
  __shared__ int warp_heads[SEG_WARPS];
  const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
  const unsigned lt_mask = (1u << lane) - 1u;
  int* keys[2] = {scratch, scratch + 2 * static_cast<size_t>(T)};
  int* vals[2] = {scratch + T, scratch + 3 * static_cast<size_t>(T)};
  for (int i = tid; i < T; i += SEG_THREADS) {
    const int64_t v = tok[i];
    keys[0][i] = (v < 0 || v >= V) ? 0 : static_cast<int>(v);
    vals[0][i] = i;
  }
  __syncthreads();
  for (int p = 0; p < passes; ++p) {
    const int* sk = keys[p & 1];
    const int* sv = vals[p & 1];
    int* dk = keys[(p + 1) & 1];
    int* dv = vals[(p + 1) & 1];
    const int shift = 8 * p;
    if (tid < SEG_RADIX) tile_total[tid] = 0;
    __syncthreads();
    for (int i = tid; i < T; i += SEG_THREADS) atomicAdd(&tile_total[(sk[i] >> shift) & 255], 1);
    __syncthreads();
    if (warp == 0) {
      // exclusive scan of the 256 digit counts: 8 per lane, then across lanes
      int c[8], run = 0;
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        c[j] = run;
        run += tile_total[8 * lane + j];
      }
      int incl = run;
#pragma unroll
      for (int o = 1; o < 32; o <<= 1) {
        const int x = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += x;
      }
      const int excl = incl - run;
#pragma unroll
      for (int j = 0; j < 8; ++j) base[8 * lane + j] = excl + c[j];
    }
    for (int t0 = 0; t0 < T; t0 += SEG_THREADS) {
      __syncthreads();  // base is final; the previous tile's readers of warp_cnt are done
      for (int j = lane; j <= SEG_RADIX; j += 32) warp_cnt[warp][j] = 0;
      const int i = t0 + tid;
      const bool active = i < T;
      const int key = active ? sk[i] : 0;
      const int val = active ? sv[i] : 0;
      const int dgt = active ? ((key >> shift) & 255) : SEG_RADIX;
      const unsigned peers = __match_any_sync(0xffffffffu, dgt);
      const int rank = __popc(peers & lt_mask);
      __syncwarp();
      if (rank == 0) warp_cnt[warp][dgt] = __popc(peers);
      __syncthreads();
      if (tid < SEG_RADIX) {
        int c[SEG_WARPS];
#pragma unroll
        for (int w = 0; w < SEG_WARPS; ++w) c[w] = warp_cnt[w][tid];
        int run = 0;
#pragma unroll
        for (int w = 0; w < SEG_WARPS; ++w) {
          warp_cnt[w][tid] = run;
          run += c[w];
        }
        tile_total[tid] = run;
      }
      __syncthreads();
      if (active) {
        const int pos = base[dgt] + warp_cnt[warp][dgt] + rank;
        dk[pos] = key;
        dv[pos] = val;
      }
      __syncthreads();
      if (tid < SEG_RADIX) base[tid] += tile_total[tid];
    }
    __syncthreads();  // this pass's writes are visible to the whole block
  }
  const int* sk = keys[passes & 1];
  const int* sv = vals[passes & 1];
  int nseg = 0;  // runs before the current tile (the same in every thread)
  for (int t0 = 0; t0 < T; t0 += SEG_THREADS) {
    const int i = t0 + tid;
    const bool active = i < T;
    const int key = active ? sk[i] : 0;
    const bool head = active && (i == 0 || sk[i - 1] != key);
    const unsigned hb = __ballot_sync(0xffffffffu, head);
    if (lane == 0) warp_heads[warp] = __popc(hb);
    __syncthreads();
    int before = 0, total = 0;
    for (int w = 0; w < SEG_WARPS; ++w) {
      const int c = warp_heads[w];
      before += w < warp ? c : 0;
      total += c;
    }
    if (active) {
      order[i] = sv[i];
      if (head) {
        const int u = nseg + before + __popc(hb & lt_mask);
        seg_tok[u] = key;
        seg_start[u] = i;
      }
    }
    nseg += total;
    __syncthreads();  // warp_heads is rewritten by the next tile
  }
  if (tid == 0) {
    seg_start[nseg] = T;
    *nseg_out = nseg;
  }
}

// Gradient scatter dE[tok] += dh[t], t ascending, as one sequential sum per
// distinct id (deterministic; no atomics).  seg_tok[u] is the u-th distinct
// (clamped) id, rows order[seg_start[u] .. seg_start[u+1]) are its tokens in
// ascending t.
// Launch: blockIdx.x strides over segments, blockIdx.y picks a chunk of
// blockDim.x float4 columns, so a frequent id's long segment is spread over
// several blocks; each thread owns one float4 column.  The sum itself is
// sequential (ascending t: the order, and so the bits, of the reference's
// accumulation), so the time of a frequent id's segment (hundreds of rows
// with Zipf-distributed ids) is its load latency: rows come in chunks of 16,
// the next chunk's rows loaded while the current chunk is added and the
// token indices of the chunk after that loaded a chunk earlier still.
// The segment count comes from nseg_dev when it is given (segments built on
// the device), else from nseg.
__global__ void embed_bwd_kernel(const int* __restrict__ seg_tok, const int* __restrict__ seg_start,
                                 const int* __restrict__ order, const float* __restrict__ dh, float* __restrict__ dE,
                                 int nseg, const int* __restrict__ nseg_dev, int d) {
  GLC_PDL_ENTRY();
  const int nc = d >> 2;
  const int c = blockIdx.y * blockDim.x + threadIdx.x;
  if (c >= nc) return;
  if (nseg_dev) nseg = *nseg_dev;
  constexpr int CH = 16;
  const float4* col = reinterpret_cast<const float4*>(dh) + c;
  const size_t rs = static_cast<size_t>(nc);  // float4s per row of dh
  for (int u = blockIdx.x; u < nseg; u += gridDim.x) {
    float4* row = reinterpret_cast<float4*>(dE + static_cast<size_t>(seg_tok[u]) * d);
    const int b = seg_start[u], e = seg_start[u + 1];
    float4 acc = row[c];
    // token indices of chunks 0 and 1, rows of chunk 0
    int ix[CH], ixn[CH];
    float4 cur[CH], nxt[CH];
#pragma unroll
    for (int i = 0; i < CH; ++i) {
      ix[i] = b + i < e ? order[b + i] : 0;
      ixn[i] = b + CH + i < e ? order[b + CH + i] : 0;
    }
#pragma unroll
    for (int i = 0; i < CH; ++i)
      if (b + i < e) cur[i] = col[static_cast<size_t>(ix[i]) * rs];
    for (int k = b; k < e; k += CH) {
      // rows of the next chunk, indices of the one after
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        if (k + CH + i < e) nxt[i] = col[static_cast<size_t>(ixn[i]) * rs];
        ix[i] = k + 2 * CH + i < e ? order[k + 2 * CH + i] : 0;
      }
#pragma unroll
      for (int i = 0; i < CH; ++i)
        if (k + i < e)
          acc = make_float4(__fadd_rn(acc.x, cur[i].x), __fadd_rn(acc.y, cur[i].y), __fadd_rn(acc.z, cur[i].z),
                            __fadd_rn(acc.w, cur[i].w));
#pragma unroll
      for (int i = 0; i < CH; ++i) {
        cur[i] = nxt[i];
        ixn[i] = ix[i];
      }
    }
    row[c] = acc;
  }
}

}  // namespace

int swiglu_fwd(Context* ctx, const float* g, const float* u, size_t ld_in, float* h, size_t ld_h, size_t rows,
               size_t cols, bool round_out, cudaStream_t s, bool fast_exp) {
  if (rows == 0 || cols == 0) return 0;
  if ((cols & 3) || (ld_in & 3) || (ld_h & 3) || !aligned16(g) || !aligned16(u) || !aligned16(h))
    return ctx->fail(GLC_ERR_INVALID, "swiglu_fwd: sizes and strides must be multiples of 4, pointers 16-byte aligned");
  const size_t n = rows * cols;
  ProfScope prof(ctx, PROF_SWIGLU, 12.0 * n, s);
  if (rows > 0xFFFFFFFFu || cols / 4 > 0xFFFFFFFFu) return ctx->fail(GLC_ERR_INVALID, "swiglu_fwd: too large");
  auto kern = fast_exp ? swiglu_fwd_kernel<true> : swiglu_fwd_kernel<false>;
  glc::launch_pdl(ctx, kern, grid_2d(rows, cols / 4, 256, ctx->num_sms), 256, 0, s,
                  g, u, ld_in, h, ld_h, static_cast<unsigned>(rows), static_cast<unsigned>(cols / 4), round_out ? 1 : 0);
  GLC_LAUNCH_CHECK(ctx, "swiglu_fwd");
  return 0;
}

int swiglu_bwd(Context* ctx, const float* g, const float* u, size_t ld_in, const float* dh, size_t ld_dh, float* dg,
               float* du, size_t ld_out, size_t rows, size_t cols, bool accumulate, bool round_out, cudaStream_t s,
               bool fast_exp) {
  if (rows == 0 || cols == 0) return 0;
  if ((cols & 3) || (ld_in & 3) || (ld_dh & 3) || (ld_out & 3) || !aligned16(g) || !aligned16(u) || !aligned16(dh) ||
      !aligned16(dg) || !aligned16(du))
    return ctx->fail(GLC_ERR_INVALID, "swiglu_bwd: sizes and strides must be multiples of 4, pointers 16-byte aligned");
  const size_t n = rows * cols;
  ProfScope prof(ctx, PROF_SWIGLU, (accumulate ? 28.0 : 20.0) * n, s);
  if (rows > 0xFFFFFFFFu || cols / 4 > 0xFFFFFFFFu) return ctx->fail(GLC_ERR_INVALID, "swiglu_bwd: too large");
  auto kern = fast_exp ? swiglu_bwd_kernel<true> : swiglu_bwd_kernel<false>;
  glc::launch_pdl(ctx, kern, grid_2d(rows, cols / 4, 256, ctx->num_sms), 256, 0, s,
                  g, u, ld_in, dh, ld_dh, dg, du, ld_out, static_cast<unsigned>(rows), static_cast<unsigned>(cols / 4),
                  accumulate ? 1 : 0, round_out ? 1 : 0);
  GLC_LAUNCH_CHECK(ctx, "swiglu_bwd");
  return 0;
}

int fill(Context* ctx, float* p, float v, size_t n, cudaStream_t s) {
  if (n == 0) return 0;
  if (!p) return ctx->fail(GLC_ERR_INVALID, "fill: null pointer");
  ProfScope prof(ctx, PROF_OTHER, 4.0 * n, s);
  glc::launch_pdl(ctx, fill_kernel, grid_for(n, 256, ctx->num_sms), 256, 0, s, p, v, n);
  GLC_LAUNCH_CHECK(ctx, "fill");
  return 0;
}

int add_inplace(Context* ctx, float* dst, const float* src, size_t n, cudaStream_t s) {
  if (n == 0) return 0;
  if (!dst || !src) return ctx->fail(GLC_ERR_INVALID, "add_inplace: null pointer");
  ProfScope prof(ctx, PROF_OTHER, 12.0 * n, s);
  glc::launch_pdl(ctx, add_inplace_kernel, grid_for(n, 256, ctx->num_sms), 256, 0, s, dst, src, n);
  GLC_LAUNCH_CHECK(ctx, "add_inplace");
  return 0;
}

int round_copy(Context* ctx, const float* src, float* dst, size_t n, cudaStream_t s) {
  if (n == 0) return 0;
  if (!src || !dst) return ctx->fail(GLC_ERR_INVALID, "round_copy: null pointer");
  ProfScope prof(ctx, PROF_OTHER, 8.0 * n, s);
  glc::launch_pdl(ctx, round_copy_kernel, grid_for(n, 256, ctx->num_sms), 256, 0, s, src, dst, n);
  GLC_LAUNCH_CHECK(ctx, "round_copy");
  return 0;
}

int rope(Context* ctx, float* x, int ld, int T, int S, int nh, int hd, const float* cos_t, const float* sin_t,
         bool inverse, bool round_out, cudaStream_t s) {
  if (T == 0) return 0;
  if (T < 0 || S <= 0 || nh <= 0 || hd <= 0 || (hd & 1) || (ld & 1) || ld < nh * hd || !x || !cos_t || !sin_t ||
      (reinterpret_cast<uintptr_t>(x) & 7))
    return ctx->fail(GLC_ERR_INVALID, "rope: bad arguments");
  const size_t pairs = static_cast<size_t>(T) * nh * (hd / 2);
  ProfScope prof(ctx, PROF_OTHER, 16.0 * pairs, s);
  if ((hd & 3) == 0 && (ld & 3) == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0 &&
      ((reinterpret_cast<uintptr_t>(cos_t) | reinterpret_cast<uintptr_t>(sin_t)) & 7) == 0) {
    const int row_quads = nh * (hd / 4);
    const int bx = (row_quads + 255) / 256;
    int by = (ctx->num_sms * 16 + bx - 1) / bx;
    if (by > T) by = T;
    if (by > 65535) by = 65535;
    glc::launch_pdl(ctx, rope4_kernel, dim3(bx, by), 256, 0, s, x, static_cast<size_t>(ld), T, S, nh, hd, cos_t, sin_t,
                    inverse ? 1 : 0, round_out ? 1 : 0);
    GLC_LAUNCH_CHECK(ctx, "rope");
    return 0;
  }
  const int row_pairs = nh * (hd / 2);
  const int bx = (row_pairs + 255) / 256;
  int by = (ctx->num_sms * 16 + bx - 1) / bx;
  if (by > T) by = T;
  if (by > 65535) by = 65535;
  glc::launch_pdl(ctx, rope_kernel, dim3(bx, by), 256, 0, s, x, static_cast<size_t>(ld), T, S, nh, hd, cos_t, sin_t, inverse ? 1 : 0,
                  round_out ? 1 : 0);
  GLC_LAUNCH_CHECK(ctx, "rope");
  return 0;
}

int embed_fwd(Context* ctx, const int64_t* tok, const float* E, const float* P, float* out, int T, int S, int d, int V,
              cudaStream_t s) {
  if (T == 0) return 0;
  if (T < 0 || S <= 0 || d <= 0 || (d & 3) || V <= 0 || !tok || !E || !out || !aligned16(E) || !aligned16(out) ||
      (P && !aligned16(P)))
    return ctx->fail(GLC_ERR_INVALID, "embed_fwd: bad arguments (hidden size must be a multiple of 4)");
  const size_t total = static_cast<size_t>(T) * (d / 4);
  ProfScope prof(ctx, PROF_OTHER, (P ? 12.0 : 8.0) * T * d, s);
  glc::launch_pdl(ctx, embed_fwd_kernel, grid_for(total, 256, ctx->num_sms), 256, 0, s, tok, E, P, out, T, S, d, V);
  GLC_LAUNCH_CHECK(ctx, "embed_fwd");
  return 0;
}

int embed_bwd(Context* ctx, const int* seg_tok, const int* seg_start, const int* order, int nseg, const float* dh,
              float* dE, int d, cudaStream_t s, const int* nseg_dev) {
  // with nseg_dev, nseg is only an upper bound (the token count) for the grid
  if (nseg == 0) return 0;
  if (nseg < 0 || d <= 0 || (d & 3) || !seg_tok || !seg_start || !order || !dh || !dE)
    return ctx->fail(GLC_ERR_INVALID, "embed_bwd: bad arguments");
  const int nc = d / 4;
  const unsigned gy = static_cast<unsigned>((nc + 127) / 128);
  unsigned gx = static_cast<unsigned>((8 * ctx->num_sms + gy - 1) / gy);
  if (gx > static_cast<unsigned>(nseg)) gx = static_cast<unsigned>(nseg);
  ProfScope prof(ctx, PROF_OTHER, 8.0 * 0, s);
  glc::launch_pdl(ctx, embed_bwd_kernel, dim3(gx, gy), 128, 0, s, seg_tok, seg_start, order, dh, dE, nseg, nseg_dev, d);
  GLC_LAUNCH_CHECK(ctx, "embed_bwd");
  return 0;
}

int embed_segments_device(Context* ctx, const int64_t* tok, int T, int V, int* out, cudaStream_t s) {
  if (T <= 0 || V <= 0 || !tok || !out) return ctx->fail(GLC_ERR_INVALID, "embed_segments: bad arguments");
  int passes = 1;
  while (passes < 4 && (static_cast<int64_t>(V) - 1) >> (8 * passes)) ++passes;
  const EmbedSegLayout L(T);
  ProfScope prof(ctx, PROF_OTHER, 0.0, s);
  glc::launch_pdl(ctx, embed_segments_kernel, dim3(1), SEG_THREADS, 0, s, tok, T, V, passes, out + L.scratch,
                  out + L.seg_tok, out + L.seg_start, out + L.order, out + L.nseg);
  GLC_LAUNCH_CHECK(ctx, "embed_segments");
  return 0;
}

}  // namespace glc
