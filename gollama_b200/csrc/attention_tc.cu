// Causal attention forward and backward on the tcgen05 tensor cores (TF32
// operands, fp32 accumulation in TMEM), flash-style: no S x S matrix in
// global memory.
//
// Semantics follow forwardAttention (pkg/train/trainer.go:331-386): query t of
// sequence b attends to keys j <= t of the same sequence, scores (q.k)*scale
// with scale = float32(1/sqrt(hd)), softmax over them, weighted sum of v; heads
// map to KV heads as in pkg/model/attention.go:118,149.  q/o rows hold H*hd
// floats, k/v rows Hkv*hd; row t = b*S + s.  Inputs are expected TF32-rounded
// (the producing kernels round them); P and dS are rounded when written.
//
// The forward and the one-group backward kernels: 352 threads — warp 0 issues
// TMA loads, warp 1 owns TMEM and issues the score MMAs (S, dP), warp 10 issues
// the accumulating MMAs (O += P V, dV/dK, dQ), warps 2..9 do the softmax
// arithmetic: warp w reads TMEM lane quarter w % 4 (one thread per row) and
// column half (w - 2) / 4 of each tile, so two warps share every row.  Values
// the two halves of a row must agree on pass through shared memory behind an
// mbarrier.  The backward kernels used by default have 608 threads: sixteen
// softmax warps in two groups that take alternate steps (see "two math
// groups" below).  All waits are bounded.
//
// forward   CTA = (128 queries, head).  S_j = Q K_j^T into one of three TMEM
//           buffers (the next S overlaps this softmax); P_j replaces S_j in
//           TMEM; O (TMEM) is rescaled when the row max grows; O += P_j V_j
//           with V as an MN-major operand.
// dK/dV     CTA = (128 keys, KV head, share of its query-head group): loops
//           over its query heads.  S^T = K Q^T, dP^T = V dO^T (64 queries per
//           step), P^T = exp(S^T - lse), dS^T = P^T (dP^T - D) scale,
//           dV += P^T dO, dK += dS^T Q accumulated in TMEM over the heads.
//           With more than one CTA per KV head their partials are summed by a
//           separate deterministic kernel.
// dQ        CTA = (128 queries, head): S = Q K^T, dP = dO V^T (64 keys per
//           step), dS as above, dQ += dS K.
// P, P^T, dS^T and dS never touch shared memory: the math warps write them
// back into TMEM over S (tcgen05.st) and the next MMA reads its A operand from
// TMEM.
#include <cfloat>
#include <atomic>
#include <cmath>

#include "glc_internal.h"
#include "sm100.cuh"

namespace glc {
namespace {

// Warps: 0 TMA producer, 1 MMA issuer for the score products (S, and dP in
// the backward), 2..9 math, 10 MMA issuer for the accumulating products
// (O += P V; dV/dK; dQ).  A warp issues an N = 64 TF32 MMA (A in TMEM) about
// every 52 cycles when the whole warp runs the loop and elect.sync picks the
// issuing lane (about every 80 from a lane-0-only branch); the tensor core
// needs 32: two issuing warps keep it busy, one cannot.
constexpr int NT = 352;
constexpr int MATH_THREADS = 256;  // warps 2..9
constexpr int ACC_WARP = 10;
constexpr float LOG2E = 1.4426950408889634f;
constexpr float LN2 = 0.6931471805599453f;

struct Roles {
  int warp, lane;
  __device__ Roles() : warp(threadIdx.x >> 5), lane(threadIdx.x & 31) {}
  __device__ int quarter() const { return warp & 3; }       // TMEM lanes this warp may access
  __device__ int half() const { return (warp - 2) >> 2; }   // column half of a tile (math warps)
};

// K-major tile of R rows x HD fp32 (HD/32 blocks of [R][128 B], 128B swizzle):
// UMMA descriptor of k-step kk (8 elements of K per step).
template <int R>
__device__ __forceinline__ uint64_t kdesc(uint32_t base, int kk) {
  return umma_sdesc(base + (kk >> 2) * (R * 128) + (kk & 3) * 32, 16, 1024, UMMA_LAYOUT_SW128);
}
// MN-major tile: chunks of 32 MN-elements x R K-rows ([R][128 B], 32-byte-atom
// swizzle), chunk stride R*128 bytes; k-step kk advances 8 K-rows.
template <int R>
__device__ __forceinline__ uint64_t mdesc(uint32_t base, int kk) {
  return umma_sdesc(base + kk * 1024, R * 128, 512, UMMA_LAYOUT_SW128_BASE32B);
}

// Loads R rows x HD columns (starting at column col0, row row0) as HD/32
// boxes of {32, R}; the tensor map fixes the swizzle (K- or MN-major).
template <int HD, int R>
__device__ __forceinline__ void tma_tile(uint8_t* dst, const CUtensorMap* tm, uint64_t* bar, int col0, int row0) {
#pragma unroll
  for (int c = 0; c < HD / 32; ++c) tma_load_2d(dst + c * R * 128, tm, bar, col0 + 32 * c, row0);
}

// tma_tile issued by a whole warp (one elected lane).
template <int HD, int R>
__device__ __forceinline__ void tma_tile_warp(uint8_t* dst, const CUtensorMap* tm, uint64_t* bar, int col0, int row0) {
#pragma unroll
  for (int c = 0; c < HD / 32; ++c) tma_load_2d_warp(dst + c * R * 128, tm, bar, col0 + 32 * c, row0);
}

// 2^x by the MUFU approximation (relative error ~2^-22): P and dS are rounded
// to TF32 (2^-11) right after, so the approximation is invisible.
__device__ __forceinline__ float fast_exp2(float x) {
  float y;
  asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
  return y;
}
// Round-to-nearest TF32 (ties away from zero) of a finite value with integer
// ops on the full-rate ALU; equal to cvt.rna.tf32.f32 for finite inputs.
__device__ __forceinline__ uint32_t tf32_bits(float x) { return (__float_as_uint(x) + 0x1000u) & 0xFFFFE000u; }
// The same rounding for a value that only ever feeds a kind::tf32 MMA, which
// reads the upper 19 bits of each 32-bit operand and ignores the rest: the
// carry of the add does the rounding, the mask is not needed.
__device__ __forceinline__ uint32_t tf32_operand_bits(float x) { return __float_as_uint(x) + 0x1000u; }

// Two fp32 FMAs / products in one sm_100 f32x2 instruction (each element
// rounded as fmaf / __fmul_rn would): halves the FP instructions of the
// softmax and dS arithmetic.
__device__ __forceinline__ float2 fma2(float2 a, float2 b, float2 c) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rc, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\tmov.b64 rc, {%6, %7};\n\t"
      "fma.rn.f32x2 rd, ra, rb, rc;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y), "f"(c.x), "f"(c.y));
  return d;
}
__device__ __forceinline__ float2 mul2(float2 a, float2 b) {
  float2 d;
  asm("{\n\t.reg .b64 ra, rb, rd;\n\t"
      "mov.b64 ra, {%2, %3};\n\tmov.b64 rb, {%4, %5};\n\t"
      "mul.rn.f32x2 rd, ra, rb;\n\t"
      "mov.b64 {%0, %1}, rd;\n\t}"
      : "=f"(d.x), "=f"(d.y)
      : "f"(a.x), "f"(a.y), "f"(b.x), "f"(b.y));
  return d;
}

__device__ __forceinline__ void st_shared_v4(uint32_t addr, float a, float b, float c, float d) {
  asm volatile("st.shared.v4.f32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "f"(a), "f"(b), "f"(c), "f"(d) : "memory");
}

// Bounded wait used by the math warps: every lane polls and the outcome is
// made warp-uniform, so a warp never reaches a warp-collective tcgen05.ld/st
// with some lanes gone.
#define WAIT_OR_BREAK(bar, parity, code)                                                 \
  if (!__all_sync(0xffffffffu, mbar_wait((bar), (parity), abort_flag, err, (code)))) {   \
    ok = false;                                                                           \
    break;                                                                                \
  }

// ===================================================================== forward
// TMEM: three S/P buffers (cols 0, 128, 256) and O (cols 384..384+HD).  The
// softmax threads overwrite S_j with P_j in place; O += P_j V_j reads P as an
// A operand straight from TMEM.  With three buffers, S_{j+2} is computed while
// the softmax works on S_{j+1} and PV_j runs.
template <int HD>
struct FwdLayout {
  static constexpr int Q = 128 * HD * 4, K = 128 * HD * 4, V = 128 * HD * 4;
  static constexpr int OFF_K = Q, OFF_V = OFF_K + 2 * K, OFF_X = OFF_V + 2 * V;
  static constexpr int OFF_BAR = OFF_X + 2 * 2 * 128 * 4;  // [parity][half][row] row maxima
  static constexpr int BYTES = OFF_BAR + 256 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int O_COL = 384;
};

template <int HD>
__global__ void __launch_bounds__(NT, 1)
    attn_fwd_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                       const __grid_constant__ CUtensorMap tmV, float* __restrict__ out, float* __restrict__ lse,
                       int S, int H, int Hkv, int n_qt, float scale_log2, int round_out, int* err) {
  GLC_PDL_ENTRY();
  using L = FwdLayout<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t *q_full = bars, *k_full = bars + 1, *k_empty = bars + 3, *v_full = bars + 5, *v_empty = bars + 7,
           *s_full = bars + 9, *p_full = bars + 12, *pv_done = bars + 15, *drain = bars + 18, *xchg = bars + 19;
  uint64_t* drain_acc = bars + 21;  // abort path of the P V issuer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const Roles ro;
  // grid (H, B, query tiles): query tiles vary slowest and the longest rows
  // (last tile, most keys) are dispatched first
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.z);
  const int h = blockIdx.x, b = blockIdx.y, kh = h / (H / Hkv);
  const int q0 = qt * 128, row_base = b * S;
  const int n_kv = qt + 1;

  if (threadIdx.x == 0) {
    mbar_init(q_full, 1);
    for (int i = 0; i < 2; ++i) {
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
    }
    for (int i = 0; i < 3; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], MATH_THREADS);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(&xchg[0], MATH_THREADS);
    mbar_init(&xchg[1], MATH_THREADS);
    mbar_init(drain, 1);
    mbar_init(drain_acc, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (ro.warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sQ = smem_u32(sm), sK = sQ + L::OFF_K, sV = sQ + L::OFF_V;

  if (ro.warp == 0) {
    if (ro.lane == 0) {
      bool ok = true;
      int armed_k[2] = {-1, -1}, armed_v[2] = {-1, -1};
      mbar_arrive_expect_tx(q_full, L::Q);
      tma_tile<HD, 128>(sm, &tmQ, q_full, h * HD, row_base + q0);
      for (int j = 0; j < n_kv; ++j) {
        const int st = j & 1;
        const uint32_t ph = (j >> 1) & 1;
        if (!mbar_wait(&k_empty[st], ph ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
        mbar_arrive_expect_tx(&k_full[st], L::K);
        tma_tile<HD, 128>(sm + L::OFF_K + st * L::K, &tmK, &k_full[st], kh * HD, row_base + j * 128);
        armed_k[st] = static_cast<int>(ph);
        if (!mbar_wait(&v_empty[st], ph ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
        mbar_arrive_expect_tx(&v_full[st], L::V);
        tma_tile<HD, 128>(sm + L::OFF_V + st * L::V, &tmV, &v_full[st], kh * HD, row_base + j * 128);
        armed_v[st] = static_cast<int>(ph);
      }
      if (!ok) {
        mbar_drain(q_full, 0, err);
        for (int st = 0; st < 2; ++st) {
          if (armed_k[st] >= 0) mbar_drain(&k_full[st], static_cast<uint32_t>(armed_k[st]), err);
          if (armed_v[st] >= 0) mbar_drain(&v_full[st], static_cast<uint32_t>(armed_v[st]), err);
        }
      }
    }
  } else if (ro.warp == 1) {
    if (ro.lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_tf32(128, 128, false, false);
      bool ok = mbar_wait(q_full, 0, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL);
      bool issued = false;
      // S_j = Q K_j^T into buffer j % 3, whose previous P (tile j-3) must be consumed
      for (int j = 0; ok && j < n_kv; ++j) {
        const int sb = j % 3, st = j & 1;
        if (j >= 3 && !mbar_wait(&pv_done[sb], ((j - 3) / 3) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_TMEM)) {
          ok = false;
          break;
        }
        if (!mbar_wait(&k_full[st], (j >> 1) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk)
          umma_tf32(tmem + sb * 128, kdesc<128>(sQ, kk), kdesc<128>(sK + st * L::K, kk), idesc_s, kk > 0 ? 1u : 0u);
        issued = true;
        umma_commit(&k_empty[st]);
        umma_commit(&s_full[sb]);
      }
      if (!ok && issued) {
        umma_commit(drain);
        mbar_drain(drain, 0, err);
      }
    }
  } else if (ro.warp == ACC_WARP) {
    // O += P_j V_j once the softmax has written P_j; pv_done[j % 3] frees the
    // S/P buffer for S_{j+3} and lets the softmax rescale O
    if (ro.lane == 0) {
      constexpr uint32_t idesc_o = umma_idesc_tf32(128, HD, false, true);
      bool ok = true, issued = false;
      for (int j = 0; ok && j < n_kv; ++j) {
        const int sb = j % 3, st = j & 1;
        if (!mbar_wait(&p_full[sb], (j / 3) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        if (!mbar_wait(&v_full[st], (j >> 1) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 16; ++kk)
          umma_tf32_ts(tmem + L::O_COL, tmem + sb * 128 + kk * 8, mdesc<128>(sV + st * L::V, kk), idesc_o,
                       (j > 0 || kk > 0) ? 1u : 0u);
        issued = true;
        umma_commit(&v_empty[st]);
        umma_commit(&pv_done[sb]);
      }
      if (!ok && issued) {
        umma_commit(drain_acc);
        mbar_drain(drain_acc, 0, err);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax
    const int q = ro.quarter(), hf = ro.half();
    const int r = q * 32 + ro.lane;
    const int row_abs = q0 + r;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    float* xmax = reinterpret_cast<float*>(sm + L::OFF_X);
    // Lazy running max (log2 domain): P_j = 2^(s - m_used) with m_used raised
    // only when the tile max exceeds it by more than 8, so P <= 256 and O is
    // rescaled on few tiles; the final O / l is unchanged.  Both warps of a
    // row take the same decisions (they exchange their half-row maxima), and
    // each keeps the partial sum l of its own columns.
    float m_used = -INFINITY, l = 0.f;
    bool ok = true;
    for (int j = 0; j < n_kv; ++j) {
      const int sb = j % 3;
      WAIT_OR_BREAK(&s_full[sb], (j / 3) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
      tc_fence_after();
      const int k0 = j * 128 + hf * 64;
      const uint32_t sa = lane_addr + sb * 128 + hf * 64;
      uint32_t v[64];
      tmem_ld_32x32b_x32(sa + 0, *reinterpret_cast<uint32_t(*)[32]>(v + 0));
      tmem_ld_32x32b_x32(sa + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
      tmem_ld_wait();
      // Masking is needed only on the diagonal tile and past the sequence end
      // (warp-uniform); elsewhere every score is live.
      if (j == qt || k0 + 64 > S) {
#pragma unroll
        for (int e = 0; e < 64; ++e) {
          const int key = k0 + e;
          if (!(key < S && key <= row_abs)) v[e] = __float_as_uint(-INFINITY);
        }
      }
      // max over raw scores (scale > 0); scores enter the exponent scaled by
      // scale*log2(e) in one FMA below
      float mx[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
#pragma unroll
      for (int e = 0; e < 64; ++e) mx[e & 7] = fmaxf(mx[e & 7], __uint_as_float(v[e]));
      const float m_half = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                 fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * scale_log2;
      float* xs = xmax + (j & 1) * 256;
      xs[hf * 128 + r] = m_half;
      mbar_arrive(&xchg[j & 1]);
      WAIT_OR_BREAK(&xchg[j & 1], (j >> 1) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
      const float m_tile = fmaxf(m_half, xs[(hf ^ 1) * 128 + r]);
      const float m_new = (m_tile > m_used + 8.0f) ? m_tile : m_used;
      const float alpha = exp2f(m_used - m_new);  // 1 unless the max was raised; 0 on the first tile
      float sum[8];
#pragma unroll
      for (int i = 0; i < 8; ++i) sum[i] = 0.f;
      // a fully masked row half has m_new = -inf until a live key arrives:
      // its scores are -inf too, and 2^(-inf) = 0 must not become NaN
      const float m_sub = m_new == -INFINITY ? 0.f : m_new;
#pragma unroll
      for (int e = 0; e < 64; ++e) {
        const uint32_t pb = tf32_bits(fast_exp2(fmaf(__uint_as_float(v[e]), scale_log2, -m_sub)));
        sum[e & 7] += __uint_as_float(pb);
        v[e] = pb;
      }
      tmem_st_32x32b_x32(sa + 0, *reinterpret_cast<uint32_t(*)[32]>(v + 0));
      tmem_st_32x32b_x32(sa + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
      tmem_st_wait();
      // both warps of a row see the same alphas, so they agree on this branch
      if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
        // O may only be rescaled once PV_{j-1} has finished accumulating into it
        WAIT_OR_BREAK(&pv_done[(j - 1) % 3], ((j - 1) / 3) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
        tc_fence_after();
#pragma unroll 1
        for (int c = hf; c < HD / 32; c += 2) {
          uint32_t o[32];
          tmem_ld_32x32b_x32(lane_addr + L::O_COL + c * 32, o);
          tmem_ld_wait();
#pragma unroll
          for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
          tmem_st_32x32b_x32(lane_addr + L::O_COL + c * 32, o);
        }
        tmem_st_wait();
      }
      tc_fence_before();
      mbar_arrive(&p_full[sb]);
      l = l * alpha + (((sum[0] + sum[1]) + (sum[2] + sum[3])) + ((sum[4] + sum[5]) + (sum[6] + sum[7])));
      m_used = m_new;
    }
    // total l of the row = sum of the two halves' partial sums (exchange slot
    // and barrier of the next tile parity)
    {
      const int j = n_kv;
      float* xs = xmax + (j & 1) * 256;
      if (ok) {
        xs[hf * 128 + r] = l;
        mbar_arrive(&xchg[j & 1]);
      }
      if (__all_sync(0xffffffffu, ok && mbar_wait(&xchg[j & 1], (j >> 1) & 1, abort_flag, err, GLC_DEV_TIMEOUT_EPILOGUE)))
        l = hf == 0 ? l + xs[128 + r] : xs[r] + l;
      else
        ok = false;
    }
    const int last = n_kv - 1;
    if (__all_sync(0xffffffffu, ok && mbar_wait(&pv_done[last % 3], (last / 3) & 1, abort_flag, err,
                                                   GLC_DEV_TIMEOUT_EPILOGUE))) {
      tc_fence_after();
      const float inv = 1.0f / l;
      float* orow = out + (static_cast<size_t>(row_base) + row_abs) * (static_cast<size_t>(H) * HD) + h * HD;
#pragma unroll 1
      for (int c = hf; c < HD / 32; c += 2) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(lane_addr + L::O_COL + c * 32, v);
        tmem_ld_wait();
        if (row_abs < S) {
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            float4 o4;
            o4.x = __uint_as_float(v[4 * g + 0]) * inv;
            o4.y = __uint_as_float(v[4 * g + 1]) * inv;
            o4.z = __uint_as_float(v[4 * g + 2]) * inv;
            o4.w = __uint_as_float(v[4 * g + 3]) * inv;
            if (round_out) o4 = make_float4(round_tf32(o4.x), round_tf32(o4.y), round_tf32(o4.z), round_tf32(o4.w));
            reinterpret_cast<float4*>(orow + c * 32)[g] = o4;
          }
        }
      }
      if (hf == 0 && row_abs < S) lse[(static_cast<size_t>(b) * H + h) * S + row_abs] = (m_used + log2f(l)) * LN2;
    }
  }
  tc_fence_before();
  __syncthreads();
  if (ro.warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// ============================================================ forward, persistent
// The same per-row arithmetic as attn_fwd_tc_kernel, with one CTA per SM
// walking work items (query tile, batch, head) in the grid kernel's order
// (longest rows first), items it = blockIdx.x + k * gridDim.x.  Every role
// counts K/V tiles, S buffers and max exchanges across items, so the
// pipelines never drain between items: the TMA warp fetches the next item's
// Q (two Q buffers, released by q_empty once an item's score MMAs are done)
// and K/V while the current item finishes, the score MMAs of the next item
// start as soon as S buffers free up, and its P V accumulates into the other
// of two O accumulators (o_full: an item's last P V finished; o_empty: the
// math warps read O out) while the math warps write the current item's
// output.  TMEM: S/P buffers at 0, 128, 256 and O at 384 + {0, HD}
// (HD <= 64).  Results are bit-identical to the grid kernel.
template <int HD>
struct PFwdLayout {
  static constexpr int Q = 128 * HD * 4, K = 128 * HD * 4, V = 128 * HD * 4;
  static constexpr int OFF_K = 2 * Q, OFF_V = OFF_K + 2 * K, OFF_X = OFF_V + 2 * V;
  static constexpr int OFF_BAR = OFF_X + 2 * 2 * 128 * 4;
  static constexpr int BYTES = OFF_BAR + 512 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int O_COL = 384;
  static_assert(O_COL + 2 * HD <= TMEM_COLS, "two O accumulators must fit beside three S buffers");
};

struct FwdItem {
  int h, b, qt;
};
__device__ __forceinline__ FwdItem fwd_item(int it, int H, int B, int n_qt) {
  const int hb = H * B;
  const int z = it / hb, rem = it - z * hb;
  FwdItem w;
  w.qt = n_qt - 1 - z;
  w.b = rem / H;
  w.h = rem - w.b * H;
  return w;
}

template <int HD>
__global__ void __launch_bounds__(NT, 1)
    attn_fwd_persist_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmK,
                            const __grid_constant__ CUtensorMap tmV, float* __restrict__ out, float* __restrict__ lse,
                            int S, int B, int H, int Hkv, int n_qt, float scale_log2, int round_out, int* err) {
  GLC_PDL_ENTRY();
  using L = PFwdLayout<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t *q_full = bars, *q_empty = bars + 2, *k_full = bars + 4, *k_empty = bars + 6, *v_full = bars + 8,
           *v_empty = bars + 10, *s_full = bars + 12, *p_full = bars + 15, *pv_done = bars + 18, *o_full = bars + 21,
           *o_empty = bars + 23, *xchg = bars + 25, *drain = bars + 27, *drain_acc = bars + 28;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 29);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const Roles ro;
  const int n_items = H * B * n_qt;
  const int G = H / Hkv;

  if (threadIdx.x == 0) {
    for (int i = 0; i < 2; ++i) {
      mbar_init(&q_full[i], 1);
      mbar_init(&q_empty[i], 1);
      mbar_init(&k_full[i], 1);
      mbar_init(&k_empty[i], 1);
      mbar_init(&v_full[i], 1);
      mbar_init(&v_empty[i], 1);
      mbar_init(&o_full[i], 1);
      mbar_init(&o_empty[i], MATH_THREADS);
      mbar_init(&xchg[i], MATH_THREADS);
    }
    for (int i = 0; i < 3; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], MATH_THREADS);
      mbar_init(&pv_done[i], 1);
    }
    mbar_init(drain, 1);
    mbar_init(drain_acc, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (ro.warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t sQ = smem_u32(sm), sK = sQ + L::OFF_K, sV = sQ + L::OFF_V;

  if (ro.warp == 0) {
    {  // whole warp: elect.sync issues
      bool ok = true;
      int armed_q[2] = {-1, -1}, armed_k[2] = {-1, -1}, armed_v[2] = {-1, -1};
      int kv = 0, local = 0;
      for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++local) {
        const FwdItem w = fwd_item(it, H, B, n_qt);
        const int kh = w.h / G, row_base = w.b * S;
        const int qb = local & 1;
        const uint32_t qph = (local >> 1) & 1;
        if (!mbar_wait_warp(&q_empty[qb], qph ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
        mbar_arrive_expect_tx_warp(&q_full[qb], L::Q);
        tma_tile_warp<HD, 128>(sm + qb * L::Q, &tmQ, &q_full[qb], w.h * HD, row_base + w.qt * 128);
        armed_q[qb] = static_cast<int>(qph);
        for (int j = 0; j <= w.qt; ++j, ++kv) {
          const int st = kv & 1;
          const uint32_t ph = (kv >> 1) & 1;
          if (!mbar_wait_warp(&k_empty[st], ph ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
          mbar_arrive_expect_tx_warp(&k_full[st], L::K);
          tma_tile_warp<HD, 128>(sm + L::OFF_K + st * L::K, &tmK, &k_full[st], kh * HD, row_base + j * 128);
          armed_k[st] = static_cast<int>(ph);
          if (!mbar_wait_warp(&v_empty[st], ph ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
          mbar_arrive_expect_tx_warp(&v_full[st], L::V);
          tma_tile_warp<HD, 128>(sm + L::OFF_V + st * L::V, &tmV, &v_full[st], kh * HD, row_base + j * 128);
          armed_v[st] = static_cast<int>(ph);
        }
      }
      if (!ok) {
        for (int st = 0; st < 2; ++st) {
          if (armed_q[st] >= 0) mbar_drain(&q_full[st], static_cast<uint32_t>(armed_q[st]), err);
          if (armed_k[st] >= 0) mbar_drain(&k_full[st], static_cast<uint32_t>(armed_k[st]), err);
          if (armed_v[st] >= 0) mbar_drain(&v_full[st], static_cast<uint32_t>(armed_v[st]), err);
        }
      }
    }
  } else if (ro.warp == 1) {
    {  // whole warp: elect.sync issues
      constexpr uint32_t idesc_s = umma_idesc_tf32(128, 128, false, false);
      bool ok = true, issued = false;
      int sq = 0, local = 0;
      for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++local) {
        const FwdItem w = fwd_item(it, H, B, n_qt);
        const int qb = local & 1;
        if (!mbar_wait_warp(&q_full[qb], (local >> 1) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        for (int j = 0; j <= w.qt; ++j, ++sq) {
          const int sb = sq % 3, st = sq & 1;
          if (sq >= 3 && !mbar_wait_warp(&pv_done[sb], ((sq - 3) / 3) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_TMEM)) {
            ok = false;
            break;
          }
          if (!mbar_wait_warp(&k_full[st], (sq >> 1) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < HD / 8; ++kk)
            umma_tf32_warp(tmem + sb * 128, kdesc<128>(sQ + qb * L::Q, kk), kdesc<128>(sK + st * L::K, kk), idesc_s,
                      kk > 0 ? 1u : 0u);
          issued = true;
          umma_commit_warp(&k_empty[st]);
          umma_commit_warp(&s_full[sb]);
        }
        if (!ok) break;
        umma_commit_warp(&q_empty[qb]);  // this item's score MMAs no longer read Q[qb]
      }
      if (!ok && issued) {
        umma_commit_warp(drain);
        mbar_drain(drain, 0, err);
      }
    }
  } else if (ro.warp == ACC_WARP) {
    {  // whole warp: elect.sync issues
      constexpr uint32_t idesc_o = umma_idesc_tf32(128, HD, false, true);
      bool ok = true, issued = false;
      int sq = 0, local = 0;
      for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++local) {
        const FwdItem w = fwd_item(it, H, B, n_qt);
        const int ob = local & 1;
        // O[ob] was read out by the math warps for item local - 2
        if (!mbar_wait_warp(&o_empty[ob], ((local >> 1) & 1) ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_TMEM)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int j = 0; j <= w.qt; ++j, ++sq) {
          const int sb = sq % 3, st = sq & 1;
          if (!mbar_wait_warp(&p_full[sb], (sq / 3) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
          if (!mbar_wait_warp(&v_full[st], (sq >> 1) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 16; ++kk)
            umma_tf32_ts_warp(tmem + L::O_COL + ob * HD, tmem + sb * 128 + kk * 8, mdesc<128>(sV + st * L::V, kk), idesc_o,
                         (j > 0 || kk > 0) ? 1u : 0u);
          issued = true;
          umma_commit_warp(&v_empty[st]);
          umma_commit_warp(&pv_done[sb]);
        }
        if (!ok) break;
        umma_commit_warp(&o_full[ob]);
      }
      if (!ok && issued) {
        umma_commit_warp(drain_acc);
        mbar_drain(drain_acc, 0, err);
      }
    }
  } else {
    // ---------------------------------------------------------------- softmax
    const int q = ro.quarter(), hf = ro.half();
    const int r = q * 32 + ro.lane;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    float* xmax = reinterpret_cast<float*>(sm + L::OFF_X);
    bool ok = true;
    int sq = 0, xc = 0, local = 0;
    for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++local) {
      const FwdItem w = fwd_item(it, H, B, n_qt);
      const int ob = local & 1;
      const uint32_t o_col = L::O_COL + ob * HD;
      const int q0 = w.qt * 128, row_base = w.b * S, row_abs = q0 + r;
      const int n_kv = w.qt + 1;
      float m_used = -INFINITY, l = 0.f;
      for (int j = 0; j < n_kv; ++j, ++sq) {
        const int sb = sq % 3;
        WAIT_OR_BREAK(&s_full[sb], (sq / 3) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
        tc_fence_after();
        const int k0 = j * 128 + hf * 64;
        const uint32_t sa = lane_addr + sb * 128 + hf * 64;
        uint32_t v[64];
        tmem_ld_32x32b_x32(sa + 0, *reinterpret_cast<uint32_t(*)[32]>(v + 0));
        tmem_ld_32x32b_x32(sa + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
        tmem_ld_wait();
        if (j == w.qt || k0 + 64 > S) {
#pragma unroll
          for (int e = 0; e < 64; ++e) {
            const int key = k0 + e;
            if (!(key < S && key <= row_abs)) v[e] = __float_as_uint(-INFINITY);
          }
        }
        float mx[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) mx[i] = -INFINITY;
#pragma unroll
        for (int e = 0; e < 64; ++e) mx[e & 7] = fmaxf(mx[e & 7], __uint_as_float(v[e]));
        const float m_half = fmaxf(fmaxf(fmaxf(mx[0], mx[1]), fmaxf(mx[2], mx[3])),
                                   fmaxf(fmaxf(mx[4], mx[5]), fmaxf(mx[6], mx[7]))) * scale_log2;
        float* xs = xmax + (xc & 1) * 256;
        xs[hf * 128 + r] = m_half;
        mbar_arrive(&xchg[xc & 1]);
        WAIT_OR_BREAK(&xchg[xc & 1], (xc >> 1) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
        const float m_tile = fmaxf(m_half, xs[(hf ^ 1) * 128 + r]);
        ++xc;
        const float m_new = (m_tile > m_used + 8.0f) ? m_tile : m_used;
        const float alpha = exp2f(m_used - m_new);
        float sum[8];
#pragma unroll
        for (int i = 0; i < 8; ++i) sum[i] = 0.f;
        const float m_sub = m_new == -INFINITY ? 0.f : m_new;
#pragma unroll
        for (int e = 0; e < 64; ++e) {
          const uint32_t pb = tf32_bits(fast_exp2(fmaf(__uint_as_float(v[e]), scale_log2, -m_sub)));
          sum[e & 7] += __uint_as_float(pb);
          v[e] = pb;
        }
        tmem_st_32x32b_x32(sa + 0, *reinterpret_cast<uint32_t(*)[32]>(v + 0));
        tmem_st_32x32b_x32(sa + 32, *reinterpret_cast<uint32_t(*)[32]>(v + 32));
        tmem_st_wait();
        if (j > 0 && __any_sync(0xffffffffu, alpha != 1.0f)) {
          // O may only be rescaled once this item's previous P V has finished
          WAIT_OR_BREAK(&pv_done[(sq - 1) % 3], ((sq - 1) / 3) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
          tc_fence_after();
#pragma unroll 1
          for (int c = hf; c < HD / 32; c += 2) {
            uint32_t o[32];
            tmem_ld_32x32b_x32(lane_addr + o_col + c * 32, o);
            tmem_ld_wait();
#pragma unroll
            for (int e = 0; e < 32; ++e) o[e] = __float_as_uint(__uint_as_float(o[e]) * alpha);
            tmem_st_32x32b_x32(lane_addr + o_col + c * 32, o);
          }
          tmem_st_wait();
        }
        tc_fence_before();
        mbar_arrive(&p_full[sb]);
        l = l * alpha + (((sum[0] + sum[1]) + (sum[2] + sum[3])) + ((sum[4] + sum[5]) + (sum[6] + sum[7])));
        m_used = m_new;
      }
      if (!ok) break;
      // total l of the row: the two halves' partial sums through the exchange
      {
        float* xs = xmax + (xc & 1) * 256;
        xs[hf * 128 + r] = l;
        mbar_arrive(&xchg[xc & 1]);
        WAIT_OR_BREAK(&xchg[xc & 1], (xc >> 1) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
        l = hf == 0 ? l + xs[128 + r] : xs[r] + l;
        ++xc;
      }
      WAIT_OR_BREAK(&o_full[ob], (local >> 1) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
      tc_fence_after();
      const float inv = 1.0f / l;
      float* orow = out + (static_cast<size_t>(row_base) + row_abs) * (static_cast<size_t>(H) * HD) + w.h * HD;
#pragma unroll 1
      for (int c = hf; c < HD / 32; c += 2) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(lane_addr + o_col + c * 32, v);
        tmem_ld_wait();
        if (row_abs < S) {
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            float4 o4;
            o4.x = __uint_as_float(v[4 * g + 0]) * inv;
            o4.y = __uint_as_float(v[4 * g + 1]) * inv;
            o4.z = __uint_as_float(v[4 * g + 2]) * inv;
            o4.w = __uint_as_float(v[4 * g + 3]) * inv;
            if (round_out) o4 = make_float4(round_tf32(o4.x), round_tf32(o4.y), round_tf32(o4.z), round_tf32(o4.w));
            reinterpret_cast<float4*>(orow + c * 32)[g] = o4;
          }
        }
      }
      if (hf == 0 && row_abs < S) lse[(static_cast<size_t>(w.b) * H + w.h) * S + row_abs] = (m_used + log2f(l)) * LN2;
      tc_fence_before();
      mbar_arrive(&o_empty[ob]);  // O[ob] read out: the item after next may accumulate into it
    }
  }
  tc_fence_before();
  __syncthreads();
  if (ro.warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// ===================================================================== dK / dV
// TMEM: two sets of {S^T [0,64), dP^T [64,128)} at cols 0 and 128, then K, V
// (the A operands of S^T = K Q^T and dP^T = V dO^T), dV and dK, HD columns
// each.  The math warps overwrite S^T with P^T and dP^T with dS^T in place;
// dV += P^T dO and dK += dS^T Q read them as A operands from TMEM.  With K
// and V out of shared memory, three 64-query Q/dO stages fit: K and V are
// first loaded into the third stage's space, copied row by row into TMEM by
// the math warps, and the space is then released to the producer.
template <int HD>
struct DkdvLayout {
  static constexpr int K = 128 * HD * 4, V = 128 * HD * 4;
  static constexpr int QT = 64 * HD * 4;    // one 64-query operand tile
  static constexpr int STAGE = 4 * QT;      // Q (K-major), Q (MN-major), dO (K-major), dO (MN-major)
  static constexpr int NST = 3, NSET = 2;
  static constexpr int OFF_KV = 2 * STAGE;  // K and V land in stage 2 (K + V == STAGE)
  static constexpr int OFF_LD = NST * STAGE, OFF_BAR = OFF_LD + 1024;
  static constexpr int BYTES = OFF_BAR + 256 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int K_COL = 256, V_COL = 256 + HD, DV_COL = 256 + 2 * HD, DK_COL = 256 + 3 * HD;
  static_assert(K + V == STAGE, "K and V fill exactly one stage");
};

// Copies row `row` of a K-major SW128 tile of 128 rows x HD fp32 (HD/32 blocks
// of [128][128 B]) into TMEM columns [col, col + HD) of the thread's lane: the
// column blocks are shared between the two warps of the lane quarter.
// With NP warps per lane quarter, block b goes to the warp with (b % NP) == part.
template <int HD, int NP = 2>
__device__ __forceinline__ void tile_rows_to_tmem(const uint8_t* tile, int row, uint32_t lane_addr, int col,
                                                  int first_block, int part) {
#pragma unroll
  for (int cb = 0; cb < HD / 32; ++cb) {
    if (((first_block + cb) % NP) != part) continue;
    const uint8_t* rp = tile + cb * (128 * 128) + row * 128;
    uint32_t v[32];
#pragma unroll
    for (int c = 0; c < 8; ++c) {
      const float4 f = *reinterpret_cast<const float4*>(rp + ((c ^ (row & 7)) << 4));
      v[4 * c] = __float_as_uint(f.x);
      v[4 * c + 1] = __float_as_uint(f.y);
      v[4 * c + 2] = __float_as_uint(f.z);
      v[4 * c + 3] = __float_as_uint(f.w);
    }
    tmem_st_32x32b_x32(lane_addr + col + cb * 32, v);
  }
}

// Grid (Hkv * nsplit, B, key tiles): the G query heads of a KV head are
// split over nsplit CTAs, each looping over its G / nsplit heads with dK/dV
// accumulated in TMEM; key tiles vary slowest, so the longest CTAs (key
// tile 0 meets every query) are dispatched first.  nsplit == 1 writes the
// final dk/dv; otherwise partial [T][Hkv * nsplit][hd] for the group sum.
template <int HD>
__global__ void __launch_bounds__(NT, 1)
    attn_bwd_dkdv_tc_kernel(const __grid_constant__ CUtensorMap tmQk, const __grid_constant__ CUtensorMap tmQm,
                            const __grid_constant__ CUtensorMap tmOk, const __grid_constant__ CUtensorMap tmOm,
                            const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                            const float* __restrict__ lse, const float* __restrict__ Dv, float* __restrict__ dk_out,
                            float* __restrict__ dv_out, int dk_ld, int dv_ld, int nsplit, int S, int H, int Hkv,
                            float scale, float scale_log2, int round_dv, int* err) {
  GLC_PDL_ENTRY();
  using L = DkdvLayout<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  // Each step's products are committed in two halves so the math warps and
  // the accumulate issuer start on the first before the second is done:
  // s_full (S^T written) / dp_full (dP^T written) from the score issuer,
  // p_full (P^T written: dV may start) / ds_full (dS^T written: dK) from
  // the math warps.
  uint64_t *kv_full = bars, *qo_full = bars + 1, *qo_empty = bars + 4, *s_full = bars + 7, *p_full = bars + 9,
           *set_free = bars + 11, *acc_done = bars + 13, *drain = bars + 14, *ld_ready = bars + 15,
           *kv_moved = bars + 17;
  uint64_t* drain_acc = bars + 18;  // abort path of the accumulate issuer
  uint64_t *dp_full = bars + 19, *ds_full = bars + 21;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 23);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  float* stage_ld = reinterpret_cast<float*>(sm + L::OFF_LD);  // [2][lse 64 | D 64]
  const Roles ro;
  const int G = H / Hkv;
  const int kt = blockIdx.z, b = blockIdx.y;
  const int kh = static_cast<int>(blockIdx.x) / nsplit, split = static_cast<int>(blockIdx.x) - kh * nsplit;
  const int n_heads = G / nsplit;
  const int h_first = kh * G + split * n_heads;
  const int k0 = kt * 128, row_base = b * S;
  const int qi0 = k0 / 64, n_q64 = (S + 63) / 64;
  const int nq = n_q64 - qi0;
  const int n_it = n_heads * nq;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_moved, MATH_THREADS);
    for (int i = 0; i < L::NST; ++i) {
      mbar_init(&qo_full[i], 1);
      mbar_init(&qo_empty[i], 1);
    }
    for (int i = 0; i < L::NSET; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&dp_full[i], 1);
      mbar_init(&p_full[i], MATH_THREADS);
      mbar_init(&ds_full[i], MATH_THREADS);
      mbar_init(&set_free[i], 1);
      mbar_init(&ld_ready[i], MATH_THREADS);
    }
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    mbar_init(drain_acc, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (ro.warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t s0 = smem_u32(sm);

  if (ro.warp == 0) {
    if (ro.lane == 0) {
      mbar_arrive_expect_tx(kv_full, L::K + L::V);
      tma_tile<HD, 128>(sm + L::OFF_KV, &tmK, kv_full, kh * HD, row_base + k0);
      tma_tile<HD, 128>(sm + L::OFF_KV + L::K, &tmV, kv_full, kh * HD, row_base + k0);
      int armed[L::NST] = {-1, -1, -1};
      bool ok = true;
      for (int it = 0; it < n_it; ++it) {
        const int st = it % L::NST;
        const uint32_t ph = (it / L::NST) & 1;
        const int hq = h_first + it / nq, qr = row_base + (qi0 + it % nq) * 64;
        // stage 2 holds K and V until the math warps have moved them to TMEM
        if (it == 2 && !mbar_wait(kv_moved, 0, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
        if (!mbar_wait(&qo_empty[st], ph ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
        mbar_arrive_expect_tx(&qo_full[st], L::STAGE);
        uint8_t* base = sm + st * L::STAGE;
        tma_tile<HD, 64>(base, &tmQk, &qo_full[st], hq * HD, qr);
        tma_tile<HD, 64>(base + L::QT, &tmQm, &qo_full[st], hq * HD, qr);
        tma_tile<HD, 64>(base + 2 * L::QT, &tmOk, &qo_full[st], hq * HD, qr);
        tma_tile<HD, 64>(base + 3 * L::QT, &tmOm, &qo_full[st], hq * HD, qr);
        armed[st] = static_cast<int>(ph);
      }
      if (!ok) {
        mbar_drain(kv_full, 0, err);
        for (int st = 0; st < L::NST; ++st)
          if (armed[st] >= 0) mbar_drain(&qo_full[st], static_cast<uint32_t>(armed[st]), err);
      }
    }
  } else if (ro.warp == 1) {
    if (ro.lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_tf32(128, 64, false, false);
      // K and V are A operands in TMEM once the math warps have copied them
      bool ok = mbar_wait(kv_moved, 0, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL);
      bool issued = false;
      tc_fence_after();
      for (int it = 0; ok && it < n_it; ++it) {
        const int st = it % L::NST, ts = it % L::NSET;
        const uint32_t base = s0 + st * L::STAGE;
        if (!mbar_wait(&qo_full[st], (it / L::NST) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        if (!mbar_wait(&set_free[ts], ((it / L::NSET) & 1) ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_TMEM)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk)
          umma_tf32_ts(tmem + ts * 128, tmem + L::K_COL + kk * 8, kdesc<64>(base, kk), idesc_s, kk > 0 ? 1u : 0u);
        issued = true;
        umma_commit(&s_full[ts]);
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk)
          umma_tf32_ts(tmem + ts * 128 + 64, tmem + L::V_COL + kk * 8, kdesc<64>(base + 2 * L::QT, kk), idesc_s,
                       kk > 0 ? 1u : 0u);
        umma_commit(&dp_full[ts]);
      }
      if (!ok && issued) {
        umma_commit(drain);
        mbar_drain(drain, 0, err);
      }
    }
  } else if (ro.warp == ACC_WARP) {
    // dV += P^T dO and dK += dS^T Q of each step once the math warps have
    // written P and dS.  Its commits also cover the S/dP MMAs of the same
    // step (they completed before the math warps could read S).
    if (ro.lane == 0) {
      constexpr uint32_t idesc_a = umma_idesc_tf32(128, HD, false, true);
      bool ok = true, issued = false;
      for (int pit = 0; ok && pit < n_it; ++pit) {
        const int ps = pit % L::NST, pts = pit % L::NSET;
        const uint32_t base = s0 + ps * L::STAGE;
        if (!mbar_wait(&p_full[pts], (pit / L::NSET) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_tf32_ts(tmem + L::DV_COL, tmem + pts * 128 + kk * 8, mdesc<64>(base + 3 * L::QT, kk), idesc_a,
                       (pit > 0 || kk > 0) ? 1u : 0u);
        issued = true;
        if (!mbar_wait(&ds_full[pts], (pit / L::NSET) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_tf32_ts(tmem + L::DK_COL, tmem + pts * 128 + 64 + kk * 8, mdesc<64>(base + L::QT, kk), idesc_a,
                       (pit > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&set_free[pts]);
        umma_commit(&qo_empty[ps]);
      }
      if (ok) umma_commit(acc_done);
      if (!ok && issued) {
        umma_commit(drain_acc);
        mbar_drain(drain_acc, 0, err);
      }
    }
  } else {
    const int q = ro.quarter(), hf = ro.half();
    const int c = q * 32 + ro.lane;         // key row within the tile
    const int t = threadIdx.x - 64;         // 0..255 among the math threads
    const int key = k0 + c;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    bool ok = true;
    // K and V rows -> TMEM, then release stage 2 and start the MMA thread
    if (__all_sync(0xffffffffu, mbar_wait(kv_full, 0, abort_flag, err, GLC_DEV_TIMEOUT_EPILOGUE))) {
      tile_rows_to_tmem<HD>(sm + L::OFF_KV, c, lane_addr, L::K_COL, 0, hf);
      tile_rows_to_tmem<HD>(sm + L::OFF_KV + L::K, c, lane_addr, L::V_COL, HD / 32, hf);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(kv_moved);
    } else {
      ok = false;
    }
    // lse (scaled to log2) or D of one of the step's 64 queries: thread t < 128
    // fetches entry t of the step's [lse 64 | D 64] staging slot
    auto fetch = [&](int i) -> float {
      const int hq = h_first + i / nq, qa = (qi0 + i % nq) * 64 + (t & 63);
      const size_t ix = (static_cast<size_t>(b) * H + hq) * S + qa;
      return qa < S ? (t < 64 ? lse[ix] * LOG2E : Dv[ix]) : 0.f;
    };
    float pre = (t < 128 && n_it > 0) ? fetch(0) : 0.f;
    for (int it = 0; ok && it < n_it; ++it) {
      const int st = it & 1, ts = it % L::NSET;
      const int qbase = (qi0 + it % nq) * 64;
      // stage this step's lse and D (double-buffered by step parity; slot st is
      // rewritten two steps later, after every reader has arrived on the other
      // slot's barrier), then fetch the next step's while this one computes
      float* slot = stage_ld + st * 128;
      if (t < 128) slot[t] = pre;
      mbar_arrive(&ld_ready[st]);
      if (t < 128 && it + 1 < n_it) pre = fetch(it + 1);
      WAIT_OR_BREAK(&ld_ready[st], (it >> 1) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
      WAIT_OR_BREAK(&s_full[ts], (it / L::NSET) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
      tc_fence_after();
      // this warp's 32 queries: S^T columns [hf*32, +32), dP^T columns 64 + [hf*32, +32)
      float lse2[32], dqs[32];
      {
        const float4* l4 = reinterpret_cast<const float4*>(slot + hf * 32);
        const float4* d4 = reinterpret_cast<const float4*>(slot + 64 + hf * 32);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 a = l4[i], d = d4[i];
          lse2[4 * i] = a.x; lse2[4 * i + 1] = a.y; lse2[4 * i + 2] = a.z; lse2[4 * i + 3] = a.w;
          dqs[4 * i] = d.x * scale; dqs[4 * i + 1] = d.y * scale; dqs[4 * i + 2] = d.z * scale; dqs[4 * i + 3] = d.w * scale;
        }
      }
      const uint32_t sa = lane_addr + ts * 128 + hf * 32;
      uint32_t sv[32], dpv[32];
      float pf[32];
      tmem_ld_32x32b_x32(sa, sv);
      tmem_ld_wait();
      // every query of this half is past every key of the tile and inside
      // the sequence: no mask (warp-uniform test)
      const int q_lo = qbase + hf * 32;
      const bool nomask = q_lo >= k0 + 127 && q_lo + 32 <= S && k0 + 128 <= S;
      if (nomask) {
#pragma unroll
        for (int e = 0; e < 32; ++e) pf[e] = fast_exp2(fmaf(__uint_as_float(sv[e]), scale_log2, -lse2[e]));
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int qa = q_lo + e;
          const bool valid = qa < S && key < S && key <= qa;
          pf[e] = valid ? fast_exp2(fmaf(__uint_as_float(sv[e]), scale_log2, -lse2[e])) : 0.f;
        }
      }
      // P^T to TMEM: dV += P^T dO may start while dS is computed
#pragma unroll
      for (int e = 0; e < 32; ++e) sv[e] = tf32_bits(pf[e]);
      tmem_st_32x32b_x32(sa, sv);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[ts]);
      WAIT_OR_BREAK(&dp_full[ts], (it / L::NSET) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
      tc_fence_after();
      tmem_ld_32x32b_x32(sa + 64, dpv);
      tmem_ld_wait();
#pragma unroll
      for (int e = 0; e < 32; ++e) dpv[e] = tf32_bits(pf[e] * fmaf(__uint_as_float(dpv[e]), scale, -dqs[e]));
      tmem_st_32x32b_x32(sa + 64, dpv);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&ds_full[ts]);
    }
    if (__all_sync(0xffffffffu, ok && mbar_wait(acc_done, 0, abort_flag, err, GLC_DEV_TIMEOUT_EPILOGUE))) {
      tc_fence_after();
      // final dk/dv at the KV head's columns, or this CTA's partial;
      // column half 0 writes dV, half 1 writes dK
      const int oh = static_cast<int>(blockIdx.x);
      const size_t trow = static_cast<size_t>(row_base) + key;
      const int part = hf;
#pragma unroll 1
      for (int cc = 0; cc < HD / 32; ++cc) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(lane_addr + (part == 0 ? L::DV_COL : L::DK_COL) + cc * 32, v);
        tmem_ld_wait();
        if (key < S) {
          float* dst = (part == 0 ? dv_out + trow * dv_ld : dk_out + trow * dk_ld) + oh * HD + cc * 32;
          const bool rnd = part == 0 && round_dv && nsplit == 1;
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            float4 o4 = make_float4(__uint_as_float(v[4 * g]), __uint_as_float(v[4 * g + 1]),
                                    __uint_as_float(v[4 * g + 2]), __uint_as_float(v[4 * g + 3]));
            if (rnd) o4 = make_float4(round_tf32(o4.x), round_tf32(o4.y), round_tf32(o4.z), round_tf32(o4.w));
            reinterpret_cast<float4*>(dst)[g] = o4;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (ro.warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// ====================================================== backward, two math groups
// 608 threads: warp 0 TMA, warp 1 score MMAs, warps 2..17 math in two groups
// of eight, warp 18 accumulating MMAs.  Group g (warps 2 + 8g .. 9 + 8g) takes
// the steps with step % 2 == g and owns TMEM S/dP set g, so the softmax of one
// step overlaps the other group's: with one group of eight warps the math of
// consecutive steps ran back to back and bounded the kernel.  Each warp
// stages the lse / D of its own 32 queries in a private shared-memory slot
// (no block-wide barrier per step).  Same arithmetic as the one-group
// kernels, bit for bit.
constexpr int NT2 = 608;
constexpr int GROUP_THREADS = 256;
constexpr int ACC_WARP2 = 18;

struct Roles2 {
  int warp, lane;
  __device__ Roles2() : warp(threadIdx.x >> 5), lane(threadIdx.x & 31) {}
  __device__ int quarter() const { return warp & 3; }               // TMEM lanes this warp may access
  __device__ int group() const { return (warp - 2) >> 3; }          // math group (math warps)
  __device__ int half() const { return ((warp - 2) >> 2) & 1; }     // column half of a tile within the group
  __device__ int part() const { return (warp - 2) >> 2; }           // 0..3: the warp among the four of its quarter
};

template <int HD>
struct Dkdv2Layout : DkdvLayout<HD> {
  // per math warp: [lse * log2(e) of its 32 queries | D * scale of them]
  static constexpr int OFF_STG = DkdvLayout<HD>::OFF_LD, STG_BYTES = 16 * 64 * 4;
  static constexpr int OFF_BAR = OFF_STG + STG_BYTES;
  static constexpr int BYTES = OFF_BAR + 256 + 1024;
};

template <int HD>
__global__ void __launch_bounds__(NT2, 1)
    attn_bwd_dkdv2_kernel(const __grid_constant__ CUtensorMap tmQk, const __grid_constant__ CUtensorMap tmQm,
                          const __grid_constant__ CUtensorMap tmOk, const __grid_constant__ CUtensorMap tmOm,
                          const __grid_constant__ CUtensorMap tmK, const __grid_constant__ CUtensorMap tmV,
                          const float* __restrict__ lse, const float* __restrict__ Dv, float* __restrict__ dk_out,
                          float* __restrict__ dv_out, int dk_ld, int dv_ld, int nsplit, int S, int H, int Hkv,
                          float scale, float scale_log2, int round_dv, int* err) {
  GLC_PDL_ENTRY();
  using L = Dkdv2Layout<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  // The two halves of a TMEM set are released separately: s_free once dV
  // has read P^T (S^T of the step after next may then be written),
  // dp_free once dK has read dS^T.
  uint64_t *kv_full = bars, *qo_full = bars + 1, *qo_empty = bars + 4, *s_full = bars + 7, *p_full = bars + 9,
           *dp_free = bars + 11, *acc_done = bars + 13, *drain = bars + 14, *kv_moved = bars + 15,
           *drain_acc = bars + 16, *dp_full = bars + 17, *ds_full = bars + 19, *s_free = bars + 21;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 23);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const Roles2 ro;
  const int G = H / Hkv;
  const int kt = blockIdx.z, b = blockIdx.y;
  const int kh = static_cast<int>(blockIdx.x) / nsplit, split = static_cast<int>(blockIdx.x) - kh * nsplit;
  const int n_heads = G / nsplit;
  const int h_first = kh * G + split * n_heads;
  const int k0 = kt * 128, row_base = b * S;
  const int qi0 = k0 / 64, n_q64 = (S + 63) / 64;
  const int nq = n_q64 - qi0;
  const int n_it = n_heads * nq;

  if (threadIdx.x == 0) {
    mbar_init(kv_full, 1);
    mbar_init(kv_moved, 2 * GROUP_THREADS);
    for (int i = 0; i < L::NST; ++i) {
      mbar_init(&qo_full[i], 1);
      mbar_init(&qo_empty[i], 1);
    }
    for (int i = 0; i < L::NSET; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&dp_full[i], 1);
      mbar_init(&p_full[i], GROUP_THREADS);
      mbar_init(&ds_full[i], GROUP_THREADS);
      mbar_init(&s_free[i], 1);
      mbar_init(&dp_free[i], 1);
    }
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    mbar_init(drain_acc, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (ro.warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t s0 = smem_u32(sm);

  if (ro.warp == 0) {
    {  // whole warp: elect.sync issues
      mbar_arrive_expect_tx_warp(kv_full, L::K + L::V);
      tma_tile_warp<HD, 128>(sm + L::OFF_KV, &tmK, kv_full, kh * HD, row_base + k0);
      tma_tile_warp<HD, 128>(sm + L::OFF_KV + L::K, &tmV, kv_full, kh * HD, row_base + k0);
      int armed[L::NST] = {-1, -1, -1};
      bool ok = true;
      for (int it = 0; it < n_it; ++it) {
        const int st = it % L::NST;
        const uint32_t ph = (it / L::NST) & 1;
        const int hq = h_first + it / nq, qr = row_base + (qi0 + it % nq) * 64;
        // stage 2 holds K and V until the math warps have moved them to TMEM
        if (it == 2 && !mbar_wait_warp(kv_moved, 0, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
        if (!mbar_wait_warp(&qo_empty[st], ph ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
        mbar_arrive_expect_tx_warp(&qo_full[st], L::STAGE);
        uint8_t* base = sm + st * L::STAGE;
        tma_tile_warp<HD, 64>(base, &tmQk, &qo_full[st], hq * HD, qr);
        tma_tile_warp<HD, 64>(base + L::QT, &tmQm, &qo_full[st], hq * HD, qr);
        tma_tile_warp<HD, 64>(base + 2 * L::QT, &tmOk, &qo_full[st], hq * HD, qr);
        tma_tile_warp<HD, 64>(base + 3 * L::QT, &tmOm, &qo_full[st], hq * HD, qr);
        armed[st] = static_cast<int>(ph);
      }
      if (!ok) {
        mbar_drain(kv_full, 0, err);
        for (int st = 0; st < L::NST; ++st)
          if (armed[st] >= 0) mbar_drain(&qo_full[st], static_cast<uint32_t>(armed[st]), err);
      }
    }
  } else if (ro.warp == 1) {
    {  // whole warp: elect.sync issues
      constexpr uint32_t idesc_s = umma_idesc_tf32(128, 64, false, false);
      bool ok = mbar_wait_warp(kv_moved, 0, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL);
      bool issued = false;
      tc_fence_after();
      for (int it = 0; ok && it < n_it; ++it) {
        const int st = it % L::NST, ts = it % L::NSET;
        const uint32_t base = s0 + st * L::STAGE;
        if (!mbar_wait_warp(&qo_full[st], (it / L::NST) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        if (!mbar_wait_warp(&s_free[ts], ((it / L::NSET) & 1) ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_TMEM)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk)
          umma_tf32_ts_warp(tmem + ts * 128, tmem + L::K_COL + kk * 8, kdesc<64>(base, kk), idesc_s, kk > 0 ? 1u : 0u);
        issued = true;
        umma_commit_warp(&s_full[ts]);
        if (!mbar_wait_warp(&dp_free[ts], ((it / L::NSET) & 1) ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_TMEM)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk)
          umma_tf32_ts_warp(tmem + ts * 128 + 64, tmem + L::V_COL + kk * 8, kdesc<64>(base + 2 * L::QT, kk), idesc_s,
                       kk > 0 ? 1u : 0u);
        umma_commit_warp(&dp_full[ts]);
      }
      if (!ok && issued) {
        umma_commit_warp(drain);
        mbar_drain(drain, 0, err);
      }
    }
  } else if (ro.warp == ACC_WARP2) {
    {  // whole warp: elect.sync issues
      constexpr uint32_t idesc_a = umma_idesc_tf32(128, HD, false, true);
      bool ok = true, issued = false;
      for (int pit = 0; ok && pit < n_it; ++pit) {
        const int ps = pit % L::NST, pts = pit % L::NSET;
        const uint32_t base = s0 + ps * L::STAGE;
        if (!mbar_wait_warp(&p_full[pts], (pit / L::NSET) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_tf32_ts_warp(tmem + L::DV_COL, tmem + pts * 128 + kk * 8, mdesc<64>(base + 3 * L::QT, kk), idesc_a,
                       (pit > 0 || kk > 0) ? 1u : 0u);
        issued = true;
        umma_commit_warp(&s_free[pts]);
        if (!mbar_wait_warp(&ds_full[pts], (pit / L::NSET) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_tf32_ts_warp(tmem + L::DK_COL, tmem + pts * 128 + 64 + kk * 8, mdesc<64>(base + L::QT, kk), idesc_a,
                       (pit > 0 || kk > 0) ? 1u : 0u);
        umma_commit_warp(&dp_free[pts]);
        umma_commit_warp(&qo_empty[ps]);
      }
      if (ok) umma_commit_warp(acc_done);
      if (!ok && issued) {
        umma_commit_warp(drain_acc);
        mbar_drain(drain_acc, 0, err);
      }
    }
  } else {
    const int q = ro.quarter(), hf = ro.half(), grp = ro.group();
    const int c = q * 32 + ro.lane;  // key row within the tile
    const int key = k0 + c;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    // [-lse * log2(e) | -D * scale] of this warp's 32 queries (negated: the
    // addends of the FMAs below)
    float* stg = reinterpret_cast<float*>(sm + L::OFF_STG) + (ro.warp - 2) * 64;
    bool ok = true;
    // K and V rows -> TMEM (the 2 HD/32 column blocks dealt over the quarter's
    // four warps), then release stage 2 and start the score issuer
    if (__all_sync(0xffffffffu, mbar_wait(kv_full, 0, abort_flag, err, GLC_DEV_TIMEOUT_EPILOGUE))) {
      tile_rows_to_tmem<HD, 4>(sm + L::OFF_KV, c, lane_addr, L::K_COL, 0, ro.part());
      tile_rows_to_tmem<HD, 4>(sm + L::OFF_KV + L::K, c, lane_addr, L::V_COL, HD / 32, ro.part());
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(kv_moved);
    } else {
      ok = false;
    }
    // lse * log2(e) and D * scale of query (lane) of this warp's half of a
    // step.  Step i is query tile qi0 + i % nq of head h_first + i / nq: the
    // group walks every second step, so (head, tile) advance by two tiles per
    // step without a division.
    float pre_l = 0.f, pre_d = 0.f;
    int cur_h = grp / nq, cur_t = grp % nq;  // the step being computed
    int nxt_h = cur_h, nxt_t = cur_t;        // the step being fetched
    auto advance = [&](int& hh, int& tt) {
      tt += 2;
      while (tt >= nq) {
        tt -= nq;
        ++hh;
      }
    };
    auto fetch = [&]() {
      const int hq = h_first + nxt_h, qa = (qi0 + nxt_t) * 64 + hf * 32 + ro.lane;
      const size_t ix = (static_cast<size_t>(b) * H + hq) * S + qa;
      pre_l = qa < S ? lse[ix] * LOG2E : 0.f;
      pre_d = qa < S ? Dv[ix] * scale : 0.f;
    };
    if (grp < n_it) fetch();
    for (int it = grp; ok && it < n_it; it += 2, advance(cur_h, cur_t)) {
      const uint32_t ph = (it >> 1) & 1;
      const int qbase = (qi0 + cur_t) * 64;
      __syncwarp();
      stg[ro.lane] = -pre_l;
      stg[32 + ro.lane] = -pre_d;
      __syncwarp();
      if (it + 2 < n_it) {
        advance(nxt_h, nxt_t);
        fetch();
      }
      WAIT_OR_BREAK(&s_full[grp], ph, GLC_DEV_TIMEOUT_EPILOGUE);
      tc_fence_after();
      // this warp's 32 queries: S^T columns [hf*32, +32), dP^T columns 64 + [hf*32, +32)
      const uint32_t sa = lane_addr + grp * 128 + hf * 32;
      uint32_t sv[32];
      float pf[32];
      tmem_ld_32x32b_x32(sa, sv);
      tmem_ld_wait();
      const int q_lo = qbase + hf * 32;
      const bool nomask = q_lo >= k0 + 127 && q_lo + 32 <= S && k0 + 128 <= S;
      const float4* l4 = reinterpret_cast<const float4*>(stg);
      if (nomask) {
        const float2 k2 = make_float2(scale_log2, scale_log2);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 l = l4[i];
          const float2 x0 = fma2(make_float2(__uint_as_float(sv[4 * i]), __uint_as_float(sv[4 * i + 1])), k2,
                                 make_float2(l.x, l.y));
          const float2 x1 = fma2(make_float2(__uint_as_float(sv[4 * i + 2]), __uint_as_float(sv[4 * i + 3])), k2,
                                 make_float2(l.z, l.w));
          pf[4 * i] = fast_exp2(x0.x);
          pf[4 * i + 1] = fast_exp2(x0.y);
          pf[4 * i + 2] = fast_exp2(x1.x);
          pf[4 * i + 3] = fast_exp2(x1.y);
        }
      } else {
#pragma unroll
        for (int i = 0; i < 8; ++i) {
          const float4 l = l4[i];
          const float lv[4] = {l.x, l.y, l.z, l.w};
#pragma unroll
          for (int e4 = 0; e4 < 4; ++e4) {
            const int e = 4 * i + e4, qa = q_lo + e;
            const bool valid = qa < S && key < S && key <= qa;
            pf[e] = valid ? fast_exp2(fmaf(__uint_as_float(sv[e]), scale_log2, lv[e4])) : 0.f;
          }
        }
      }
      // P^T to TMEM: dV += P^T dO may start while dS is computed
#pragma unroll
      for (int e = 0; e < 32; ++e) sv[e] = tf32_operand_bits(pf[e]);
      tmem_st_32x32b_x32(sa, sv);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[grp]);
      WAIT_OR_BREAK(&dp_full[grp], ph, GLC_DEV_TIMEOUT_EPILOGUE);
      tc_fence_after();
      tmem_ld_32x32b_x32(sa + 64, sv);
      tmem_ld_wait();
      const float4* d4 = reinterpret_cast<const float4*>(stg + 32);
      const float2 sc2 = make_float2(scale, scale);
#pragma unroll
      for (int i = 0; i < 8; ++i) {
        const float4 d = d4[i];
        const float2 t0 = fma2(make_float2(__uint_as_float(sv[4 * i]), __uint_as_float(sv[4 * i + 1])), sc2,
                               make_float2(d.x, d.y));
        const float2 t1 = fma2(make_float2(__uint_as_float(sv[4 * i + 2]), __uint_as_float(sv[4 * i + 3])), sc2,
                               make_float2(d.z, d.w));
        const float2 g0 = mul2(make_float2(pf[4 * i], pf[4 * i + 1]), t0);
        const float2 g1 = mul2(make_float2(pf[4 * i + 2], pf[4 * i + 3]), t1);
        sv[4 * i] = tf32_operand_bits(g0.x);
        sv[4 * i + 1] = tf32_operand_bits(g0.y);
        sv[4 * i + 2] = tf32_operand_bits(g1.x);
        sv[4 * i + 3] = tf32_operand_bits(g1.y);
      }
      tmem_st_32x32b_x32(sa + 64, sv);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&ds_full[grp]);
    }
    if (__all_sync(0xffffffffu, ok && mbar_wait(acc_done, 0, abort_flag, err, GLC_DEV_TIMEOUT_EPILOGUE))) {
      tc_fence_after();
      // final dk/dv at the KV head's columns, or this CTA's partial: the
      // quarter's four warps take the 2 HD/32 column blocks of dV then dK
      const int oh = static_cast<int>(blockIdx.x);
      const size_t trow = static_cast<size_t>(row_base) + key;
#pragma unroll 1
      for (int blk = ro.part(); blk < 2 * (HD / 32); blk += 4) {
        const int part = blk / (HD / 32), cc = blk % (HD / 32);
        uint32_t v[32];
        tmem_ld_32x32b_x32(lane_addr + (part == 0 ? L::DV_COL : L::DK_COL) + cc * 32, v);
        tmem_ld_wait();
        if (key < S) {
          float* dst = (part == 0 ? dv_out + trow * dv_ld : dk_out + trow * dk_ld) + oh * HD + cc * 32;
          const bool rnd = part == 0 && round_dv && nsplit == 1;
#pragma unroll
          for (int g = 0; g < 8; ++g) {
            float4 o4 = make_float4(__uint_as_float(v[4 * g]), __uint_as_float(v[4 * g + 1]),
                                    __uint_as_float(v[4 * g + 2]), __uint_as_float(v[4 * g + 3]));
            if (rnd) o4 = make_float4(round_tf32(o4.x), round_tf32(o4.y), round_tf32(o4.z), round_tf32(o4.w));
            reinterpret_cast<float4*>(dst)[g] = o4;
          }
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (ro.warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// dk[t][kh] = sum over the nsplit partials of the KV head, partial[t][kh *
// nsplit + g] (g ascending: deterministic); dv the same, optionally
// TF32-rounded.
// With RoPE tables, dk gets the transposed rotation at position t % S and is
// TF32-rounded (what a separate backward RoPE pass would write).
__global__ void group_sum_kernel(const float* __restrict__ pk, const float* __restrict__ pv, float* __restrict__ dk,
                                 float* __restrict__ dv, int dk_ld, int dv_ld, int T, int S, int nsplit, int Hkv, int hd,
                                 int round_dv, const float* __restrict__ rope_cos, const float* __restrict__ rope_sin) {
  GLC_PDL_ENTRY();
  // 32-bit index math: the host checks T * Hkv * hd / 4 < 2^31
  const int n4 = hd / 4, per_t = Hkv * n4;
  const int total = T * per_t;
  for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
    const size_t t = static_cast<unsigned>(i) / static_cast<unsigned>(per_t);
    const int rem = i - static_cast<int>(t) * per_t;
    const int kh = rem / n4, d4 = rem - kh * n4;
    float4 sk = make_float4(0.f, 0.f, 0.f, 0.f), sv = sk;
    for (int g = 0; g < nsplit; ++g) {
      const size_t src = (t * Hkv * nsplit + kh * nsplit + g) * hd / 4 + d4;
      const float4 a = reinterpret_cast<const float4*>(pk)[src];
      const float4 c = reinterpret_cast<const float4*>(pv)[src];
      sk.x += a.x; sk.y += a.y; sk.z += a.z; sk.w += a.w;
      sv.x += c.x; sv.y += c.y; sv.z += c.z; sv.w += c.w;
    }
    if (round_dv) sv = make_float4(round_tf32(sv.x), round_tf32(sv.y), round_tf32(sv.z), round_tf32(sv.w));
    if (rope_cos) {
      // columns 4*d4 .. 4*d4+3 are the pairs 2*d4 and 2*d4+1 of head kh
      const size_t trow = (t % static_cast<unsigned>(S)) * static_cast<size_t>(hd / 2);
      const float2 c = reinterpret_cast<const float2*>(rope_cos + trow)[d4];
      const float2 sn = reinterpret_cast<const float2*>(rope_sin + trow)[d4];
      sk = make_float4(round_tf32(__fadd_rn(__fmul_rn(sk.x, c.x), __fmul_rn(sk.y, sn.x))),
                       round_tf32(__fadd_rn(__fmul_rn(-sk.x, sn.x), __fmul_rn(sk.y, c.x))),
                       round_tf32(__fadd_rn(__fmul_rn(sk.z, c.y), __fmul_rn(sk.w, sn.y))),
                       round_tf32(__fadd_rn(__fmul_rn(-sk.z, sn.y), __fmul_rn(sk.w, c.y))));
    }
    reinterpret_cast<float4*>(dk + t * dk_ld + kh * hd)[d4] = sk;
    reinterpret_cast<float4*>(dv + t * dv_ld + kh * hd)[d4] = sv;
  }
}

// ===================================================================== dQ
// TMEM: two sets of {S [0,64), dP [64,128)} at cols 0 and 128, then Q and dO
// (the A operands of S = Q K^T and dP = dO V^T) and dQ, HD columns each.  The
// math warps overwrite S with dS in place; dQ += dS K reads it from TMEM.
// With Q and dO out of shared memory, four 64-key K/V stages fit: Q and dO
// first land in the space of stages 2 and 3, are copied row by row into TMEM
// by the math warps, and the space is then released to the producer.  The
// MMA thread issues S/dP of step j before dQ of step j-1.
template <int HD>
struct DqLayout {
  static constexpr int Q = 128 * HD * 4, O = 128 * HD * 4;
  static constexpr int KT = 64 * HD * 4;              // one 64-key operand tile
  static constexpr int STAGE = 3 * KT;                // K (K-major), K (MN-major), V (K-major)
  static constexpr int NST = 4, NSET = 2;             // smem K/V stages, TMEM S/dP sets
  static constexpr int OFF_QO = 2 * STAGE;            // Q and dO land in stages 2..3
  static constexpr int OFF_BAR = NST * STAGE;
  static constexpr int BYTES = OFF_BAR + 256 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int Q_COL = 256, O_COL = 256 + HD, DQ_COL = 256 + 2 * HD;
  static_assert(Q + O <= 2 * STAGE, "Q and dO fit in two stages");
};

template <int HD>
__global__ void __launch_bounds__(NT, 1)
    attn_bwd_dq_tc_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmO,
                          const __grid_constant__ CUtensorMap tmKk, const __grid_constant__ CUtensorMap tmKm,
                          const __grid_constant__ CUtensorMap tmVk, const float* __restrict__ lse,
                          const float* __restrict__ Dv, float* __restrict__ dq, int dq_ld, int S, int H, int Hkv,
                          int n_qt, float scale, float scale_log2, const float* __restrict__ rope_cos,
                          const float* __restrict__ rope_sin, int* err) {
  GLC_PDL_ENTRY();
  using L = DqLayout<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t *qo_full = bars, *kv_full = bars + 1, *kv_empty = bars + 5, *s_full = bars + 9, *p_full = bars + 11,
           *set_free = bars + 13, *acc_done = bars + 15, *drain = bars + 16, *qo_moved = bars + 17;
  uint64_t* drain_acc = bars + 18;  // abort path of the accumulate issuer
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 19);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const Roles ro;
  // grid (H, B, query tiles), longest CTAs (last query tile) dispatched first
  const int qt = n_qt - 1 - static_cast<int>(blockIdx.z);
  const int h = blockIdx.x, b = blockIdx.y, kh = h / (H / Hkv);
  const int q0 = qt * 128, row_base = b * S;
  const int n_k64 = (S + 63) / 64;
  const int nk = min(n_k64, (q0 + 128) / 64);

  if (threadIdx.x == 0) {
    mbar_init(qo_full, 1);
    mbar_init(qo_moved, MATH_THREADS);
    for (int i = 0; i < L::NST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < L::NSET; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&p_full[i], MATH_THREADS);
      mbar_init(&set_free[i], 1);
    }
    mbar_init(acc_done, 1);
    mbar_init(drain, 1);
    mbar_init(drain_acc, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (ro.warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t s0 = smem_u32(sm);

  if (ro.warp == 0) {
    if (ro.lane == 0) {
      mbar_arrive_expect_tx(qo_full, L::Q + L::O);
      tma_tile<HD, 128>(sm + L::OFF_QO, &tmQ, qo_full, h * HD, row_base + q0);
      tma_tile<HD, 128>(sm + L::OFF_QO + L::Q, &tmO, qo_full, h * HD, row_base + q0);
      int armed[L::NST] = {-1, -1, -1, -1};
      bool ok = true;
      for (int j = 0; j < nk; ++j) {
        const int st = j % L::NST;
        const uint32_t ph = (j / L::NST) & 1;
        // stages 2 and 3 hold Q and dO until the math warps have moved them to TMEM
        if (j == 2 && !mbar_wait(qo_moved, 0, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
        if (!mbar_wait(&kv_empty[st], ph ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
        mbar_arrive_expect_tx(&kv_full[st], L::STAGE);
        uint8_t* base = sm + st * L::STAGE;
        tma_tile<HD, 64>(base, &tmKk, &kv_full[st], kh * HD, row_base + j * 64);
        tma_tile<HD, 64>(base + L::KT, &tmKm, &kv_full[st], kh * HD, row_base + j * 64);
        tma_tile<HD, 64>(base + 2 * L::KT, &tmVk, &kv_full[st], kh * HD, row_base + j * 64);
        armed[st] = static_cast<int>(ph);
      }
      if (!ok) {
        mbar_drain(qo_full, 0, err);
        for (int st = 0; st < L::NST; ++st)
          if (armed[st] >= 0) mbar_drain(&kv_full[st], static_cast<uint32_t>(armed[st]), err);
      }
    }
  } else if (ro.warp == 1) {
    if (ro.lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_tf32(128, 64, false, false);
      // Q and dO are A operands in TMEM once the math warps have copied them
      bool ok = mbar_wait(qo_moved, 0, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL);
      bool issued = false;
      tc_fence_after();
      for (int j = 0; ok && j < nk; ++j) {
        const int st = j % L::NST, ts = j % L::NSET;
        const uint32_t base = s0 + st * L::STAGE;
        if (!mbar_wait(&kv_full[st], (j / L::NST) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        if (!mbar_wait(&set_free[ts], ((j / L::NSET) & 1) ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_TMEM)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < HD / 8; ++kk) {
          umma_tf32_ts(tmem + ts * 128, tmem + L::Q_COL + kk * 8, kdesc<64>(base, kk), idesc_s, kk > 0 ? 1u : 0u);
          umma_tf32_ts(tmem + ts * 128 + 64, tmem + L::O_COL + kk * 8, kdesc<64>(base + 2 * L::KT, kk), idesc_s,
                       kk > 0 ? 1u : 0u);
        }
        issued = true;
        umma_commit(&s_full[ts]);
      }
      if (!ok && issued) {
        umma_commit(drain);
        mbar_drain(drain, 0, err);
      }
    }
  } else if (ro.warp == ACC_WARP) {
    // dQ += dS K of each step once the math warps have written dS; its
    // commits also cover the step's S/dP MMAs (complete before dS exists)
    if (ro.lane == 0) {
      constexpr uint32_t idesc_q = umma_idesc_tf32(128, HD, false, true);
      bool ok = true, issued = false;
      for (int pj = 0; ok && pj < nk; ++pj) {
        const int ps = pj % L::NST, pts = pj % L::NSET;
        const uint32_t base = s0 + ps * L::STAGE;
        if (!mbar_wait(&p_full[pts], (pj / L::NSET) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        tc_fence_after();
#pragma unroll
        for (int kk = 0; kk < 8; ++kk)
          umma_tf32_ts(tmem + L::DQ_COL, tmem + pts * 128 + kk * 8, mdesc<64>(base + L::KT, kk), idesc_q,
                       (pj > 0 || kk > 0) ? 1u : 0u);
        issued = true;
        umma_commit(&set_free[pts]);
        umma_commit(&kv_empty[ps]);
      }
      if (ok) umma_commit(acc_done);
      if (!ok && issued) {
        umma_commit(drain_acc);
        mbar_drain(drain_acc, 0, err);
      }
    }
  } else {
    const int q = ro.quarter(), hf = ro.half();
    const int r = q * 32 + ro.lane;
    const int qa = q0 + r;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    const size_t lrow = (static_cast<size_t>(b) * H + h) * S + (qa < S ? qa : 0);
    const float lse2 = lse[lrow] * LOG2E, Dq = Dv[lrow];
    bool ok = true;
    // Q and dO rows -> TMEM, then release stages 2..3 and start the MMA thread
    if (__all_sync(0xffffffffu, mbar_wait(qo_full, 0, abort_flag, err, GLC_DEV_TIMEOUT_EPILOGUE))) {
      tile_rows_to_tmem<HD>(sm + L::OFF_QO, r, lane_addr, L::Q_COL, 0, hf);
      tile_rows_to_tmem<HD>(sm + L::OFF_QO + L::Q, r, lane_addr, L::O_COL, HD / 32, hf);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(qo_moved);
    } else {
      ok = false;
    }
    for (int j = 0; ok && j < nk; ++j) {
      const int ts = j % L::NSET;
      WAIT_OR_BREAK(&s_full[ts], (j / L::NSET) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
      tc_fence_after();
      // this warp's 32 keys: S columns [hf*32, +32), dP columns 64 + [hf*32, +32)
      const uint32_t sa = lane_addr + ts * 128 + hf * 32;
      uint32_t sv[32], dpv[32];
      tmem_ld_32x32b_x32(sa, sv);
      tmem_ld_32x32b_x32(sa + 64, dpv);
      tmem_ld_wait();
      const int k_lo = j * 64 + hf * 32;
      const float nDs = -Dq * scale;
      // every key of this half precedes every row of the tile: no mask
      // (warp-uniform test)
      if (k_lo + 32 <= q0 + 1 && q0 + 128 <= S) {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const float p = fast_exp2(fmaf(__uint_as_float(sv[e]), scale_log2, -lse2));
          sv[e] = tf32_bits(p * fmaf(__uint_as_float(dpv[e]), scale, nDs));
        }
      } else {
#pragma unroll
        for (int e = 0; e < 32; ++e) {
          const int key = k_lo + e;
          const bool valid = qa < S && key < S && key <= qa;
          const float p = valid ? fast_exp2(fmaf(__uint_as_float(sv[e]), scale_log2, -lse2)) : 0.f;
          sv[e] = tf32_bits(p * fmaf(__uint_as_float(dpv[e]), scale, nDs));
        }
      }
      tmem_st_32x32b_x32(sa, sv);
      tmem_st_wait();
      tc_fence_before();
      mbar_arrive(&p_full[ts]);
    }
    if (__all_sync(0xffffffffu, ok && mbar_wait(acc_done, 0, abort_flag, err, GLC_DEV_TIMEOUT_EPILOGUE))) {
      tc_fence_after();
      float* drow = dq + (static_cast<size_t>(row_base) + qa) * static_cast<size_t>(dq_ld) + h * HD;
#pragma unroll 1
      for (int cc = hf; cc < HD / 32; cc += 2) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(lane_addr + L::DQ_COL + cc * 32, v);
        tmem_ld_wait();
        if (qa < S && rope_cos) {
          // transposed RoPE rotation of the row's pairs cc*16 .. cc*16+15 at
          // position qa, then TF32 rounding
          const float4* cr = reinterpret_cast<const float4*>(rope_cos + static_cast<size_t>(qa) * (HD / 2) + cc * 16);
          const float4* sr = reinterpret_cast<const float4*>(rope_sin + static_cast<size_t>(qa) * (HD / 2) + cc * 16);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const float4 c4 = cr[g], s4 = sr[g];
            const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int p = 4 * g + e;
              const float x0 = __uint_as_float(v[2 * p]), x1 = __uint_as_float(v[2 * p + 1]);
              v[2 * p] = __float_as_uint(round_tf32(__fadd_rn(__fmul_rn(x0, cs[e]), __fmul_rn(x1, sn[e]))));
              v[2 * p + 1] = __float_as_uint(round_tf32(__fadd_rn(__fmul_rn(-x0, sn[e]), __fmul_rn(x1, cs[e]))));
            }
          }
        }
        if (qa < S) {
#pragma unroll
          for (int g = 0; g < 8; ++g)
            reinterpret_cast<float4*>(drow + cc * 32)[g] =
                make_float4(__uint_as_float(v[4 * g]), __uint_as_float(v[4 * g + 1]), __uint_as_float(v[4 * g + 2]),
                            __uint_as_float(v[4 * g + 3]));
        }
      }
    }
  }
  tc_fence_before();
  __syncthreads();
  if (ro.warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// ================================================================ dQ, persistent
// attn_bwd_dq_tc_kernel's arithmetic with one CTA per SM walking work items
// (query tile, batch, head) in the grid kernel's order, counting K/V stages
// and S/dP sets across items.  Q and dO get their own staging area (three
// K/V stages instead of four), and the math warps move the next item's Q and
// dO into TMEM as soon as they have finished the current item's last step
// (whose S/dP products, the only readers of Q and dO in TMEM, have completed
// by then), before writing the current item's dQ: the next item's products
// overlap that output.  dQ alternates between two accumulators (dq_full: an
// item's last dQ product finished; dq_empty: the math warps read it out).
// TMEM: S/dP sets at 0 and 128, Q at 256, dO at 256 + HD, dQ at 256 + 2 HD
// + {0, HD}.  Results are bit-identical to the grid kernel.
template <int HD>
struct PDqLayout {
  static constexpr int Q = 128 * HD * 4, O = 128 * HD * 4;
  static constexpr int KT = 64 * HD * 4;
  static constexpr int STAGE = 3 * KT;  // K (K-major), K (MN-major), V (K-major)
  static constexpr int NST = 3, NSET = 2;
  static constexpr int OFF_QO = NST * STAGE;
  static constexpr int OFF_BAR = OFF_QO + Q + O;
  static constexpr int BYTES = OFF_BAR + 512 + 1024;
  static constexpr int TMEM_COLS = 512;
  static constexpr int Q_COL = 256, O_COL = 256 + HD, DQ_COL = 256 + 2 * HD;
  static_assert(DQ_COL + 2 * HD <= TMEM_COLS, "two dQ accumulators must fit");
};

template <int HD>
__global__ void __launch_bounds__(NT, 1)
    attn_bwd_dq_persist_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmO,
                               const __grid_constant__ CUtensorMap tmKk, const __grid_constant__ CUtensorMap tmKm,
                               const __grid_constant__ CUtensorMap tmVk, const float* __restrict__ lse,
                               const float* __restrict__ Dv, float* __restrict__ dq, int dq_ld, int S, int B, int H,
                               int Hkv, int n_qt, float scale, float scale_log2, const float* __restrict__ rope_cos,
                               const float* __restrict__ rope_sin, int* err) {
  GLC_PDL_ENTRY();
  using L = PDqLayout<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t *qo_full = bars, *qo_moved = bars + 1, *kv_full = bars + 2, *kv_empty = bars + 5, *s_full = bars + 8,
           *p_full = bars + 10, *set_free = bars + 12, *dq_full = bars + 14, *dq_empty = bars + 16, *drain = bars + 18,
           *drain_acc = bars + 19;
  // S and dP are committed separately (s_full, dp_full): the math warps
  // compute P while the dP products run
  uint64_t* dp_full = bars + 20;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const Roles ro;
  const int n_items = H * B * n_qt;
  const int G = H / Hkv;
  const int n_k64 = (S + 63) / 64;

  if (threadIdx.x == 0) {
    mbar_init(qo_full, 1);
    mbar_init(qo_moved, MATH_THREADS);
    for (int i = 0; i < L::NST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < L::NSET; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&dp_full[i], 1);
      mbar_init(&p_full[i], MATH_THREADS);
      mbar_init(&set_free[i], 1);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_empty[i], MATH_THREADS);
    }
    mbar_init(drain, 1);
    mbar_init(drain_acc, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (ro.warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t s0 = smem_u32(sm);

  if (ro.warp == 0) {
    if (ro.lane == 0) {
      int armed[L::NST] = {-1, -1, -1};
      int armed_qo = -1;
      bool ok = true;
      int kv = 0, local = 0;
      for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++local) {
        const FwdItem w = fwd_item(it, H, B, n_qt);
        const int kh = w.h / G, q0 = w.qt * 128, row_base = w.b * S;
        const int nk = min(n_k64, (q0 + 128) / 64);
        // the staging area is free once the previous item's Q and dO are in TMEM
        if (local > 0 && !mbar_wait(qo_moved, (local - 1) & 1, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx(qo_full, L::Q + L::O);
        tma_tile<HD, 128>(sm + L::OFF_QO, &tmQ, qo_full, w.h * HD, row_base + q0);
        tma_tile<HD, 128>(sm + L::OFF_QO + L::Q, &tmO, qo_full, w.h * HD, row_base + q0);
        armed_qo = local & 1;
        for (int j = 0; j < nk; ++j, ++kv) {
          const int st = kv % L::NST;
          const uint32_t ph = (kv / L::NST) & 1;
          if (!mbar_wait(&kv_empty[st], ph ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
          mbar_arrive_expect_tx(&kv_full[st], L::STAGE);
          uint8_t* base = sm + st * L::STAGE;
          tma_tile<HD, 64>(base, &tmKk, &kv_full[st], kh * HD, row_base + j * 64);
          tma_tile<HD, 64>(base + L::KT, &tmKm, &kv_full[st], kh * HD, row_base + j * 64);
          tma_tile<HD, 64>(base + 2 * L::KT, &tmVk, &kv_full[st], kh * HD, row_base + j * 64);
          armed[st] = static_cast<int>(ph);
        }
      }
      if (!ok) {
        if (armed_qo >= 0) mbar_drain(qo_full, static_cast<uint32_t>(armed_qo), err);
        for (int st = 0; st < L::NST; ++st)
          if (armed[st] >= 0) mbar_drain(&kv_full[st], static_cast<uint32_t>(armed[st]), err);
      }
    }
  } else if (ro.warp == 1) {
    if (ro.lane == 0) {
      constexpr uint32_t idesc_s = umma_idesc_tf32(128, 64, false, false);
      bool ok = true, issued = false;
      int kv = 0, local = 0;
      for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++local) {
        const FwdItem w = fwd_item(it, H, B, n_qt);
        const int nk = min(n_k64, (w.qt * 128 + 128) / 64);
        // this item's Q and dO are in TMEM
        if (!mbar_wait(qo_moved, local & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        tc_fence_after();
        for (int j = 0; j < nk; ++j, ++kv) {
          const int st = kv % L::NST, ts = kv % L::NSET;
          const uint32_t base = s0 + st * L::STAGE;
          if (!mbar_wait(&kv_full[st], (kv / L::NST) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
          if (!mbar_wait(&set_free[ts], ((kv / L::NSET) & 1) ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_TMEM)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < HD / 8; ++kk)
            umma_tf32_ts(tmem + ts * 128, tmem + L::Q_COL + kk * 8, kdesc<64>(base, kk), idesc_s, kk > 0 ? 1u : 0u);
          issued = true;
          umma_commit(&s_full[ts]);
#pragma unroll
          for (int kk = 0; kk < HD / 8; ++kk)
            umma_tf32_ts(tmem + ts * 128 + 64, tmem + L::O_COL + kk * 8, kdesc<64>(base + 2 * L::KT, kk), idesc_s,
                         kk > 0 ? 1u : 0u);
          umma_commit(&dp_full[ts]);
        }
      }
      if (!ok && issued) {
        umma_commit(drain);
        mbar_drain(drain, 0, err);
      }
    }
  } else if (ro.warp == ACC_WARP) {
    if (ro.lane == 0) {
      constexpr uint32_t idesc_q = umma_idesc_tf32(128, HD, false, true);
      bool ok = true, issued = false;
      int kv = 0, local = 0;
      for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++local) {
        const FwdItem w = fwd_item(it, H, B, n_qt);
        const int nk = min(n_k64, (w.qt * 128 + 128) / 64);
        const int ob = local & 1;
        // dQ[ob] was read out by the math warps for item local - 2
        if (!mbar_wait(&dq_empty[ob], ((local >> 1) & 1) ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_TMEM)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int j = 0; j < nk; ++j, ++kv) {
          const int ps = kv % L::NST, pts = kv % L::NSET;
          const uint32_t base = s0 + ps * L::STAGE;
          if (!mbar_wait(&p_full[pts], (kv / L::NSET) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_tf32_ts(tmem + L::DQ_COL + ob * HD, tmem + pts * 128 + kk * 8, mdesc<64>(base + L::KT, kk), idesc_q,
                         (j > 0 || kk > 0) ? 1u : 0u);
          issued = true;
          umma_commit(&set_free[pts]);
          umma_commit(&kv_empty[ps]);
        }
        if (!ok) break;
        umma_commit(&dq_full[ob]);
      }
      if (!ok && issued) {
        umma_commit(drain_acc);
        mbar_drain(drain_acc, 0, err);
      }
    }
  } else {
    const int q = ro.quarter(), hf = ro.half();
    const int r = q * 32 + ro.lane;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    bool ok = true;
    int kv = 0, local = 0;
    // the first item's Q and dO rows -> TMEM
    if (static_cast<int>(blockIdx.x) < n_items) {
      if (__all_sync(0xffffffffu, mbar_wait(qo_full, 0, abort_flag, err, GLC_DEV_TIMEOUT_EPILOGUE))) {
        tile_rows_to_tmem<HD>(sm + L::OFF_QO, r, lane_addr, L::Q_COL, 0, hf);
        tile_rows_to_tmem<HD>(sm + L::OFF_QO + L::Q, r, lane_addr, L::O_COL, HD / 32, hf);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(qo_moved);
      } else {
        ok = false;
      }
    }
    for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++local) {
      const FwdItem w = fwd_item(it, H, B, n_qt);
      const int q0 = w.qt * 128, row_base = w.b * S, qa = q0 + r;
      const int nk = min(n_k64, (q0 + 128) / 64);
      const size_t lrow = (static_cast<size_t>(w.b) * H + w.h) * S + (qa < S ? qa : 0);
      const float lse2 = lse[lrow] * LOG2E, Dq = Dv[lrow];
      for (int j = 0; j < nk; ++j, ++kv) {
        const int ts = kv % L::NSET;
        WAIT_OR_BREAK(&s_full[ts], (kv / L::NSET) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
        tc_fence_after();
        const uint32_t sa = lane_addr + ts * 128 + hf * 32;
        uint32_t sv[32], dpv[32];
        float pf[32];
        tmem_ld_32x32b_x32(sa, sv);
        tmem_ld_wait();
        const int k_lo = j * 64 + hf * 32;
        const float nDs = -Dq * scale;
        if (k_lo + 32 <= q0 + 1 && q0 + 128 <= S) {
#pragma unroll
          for (int e = 0; e < 32; ++e) pf[e] = fast_exp2(fmaf(__uint_as_float(sv[e]), scale_log2, -lse2));
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int key = k_lo + e;
            const bool valid = qa < S && key < S && key <= qa;
            pf[e] = valid ? fast_exp2(fmaf(__uint_as_float(sv[e]), scale_log2, -lse2)) : 0.f;
          }
        }
        WAIT_OR_BREAK(&dp_full[ts], (kv / L::NSET) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
        tc_fence_after();
        tmem_ld_32x32b_x32(sa + 64, dpv);
        tmem_ld_wait();
#pragma unroll
        for (int e = 0; e < 32; ++e) sv[e] = tf32_bits(pf[e] * fmaf(__uint_as_float(dpv[e]), scale, nDs));
        tmem_st_32x32b_x32(sa, sv);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[ts]);
      }
      if (!ok) break;
      // the next item's Q and dO rows -> TMEM: every product of this item that
      // reads them (S reads Q, dP reads dO) completed before its last s_full
      // and dp_full, both waited for above
      if (it + static_cast<int>(gridDim.x) < n_items) {
        WAIT_OR_BREAK(qo_full, (local + 1) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
        tile_rows_to_tmem<HD>(sm + L::OFF_QO, r, lane_addr, L::Q_COL, 0, hf);
        tile_rows_to_tmem<HD>(sm + L::OFF_QO + L::Q, r, lane_addr, L::O_COL, HD / 32, hf);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(qo_moved);
      }
      const int ob = local & 1;
      WAIT_OR_BREAK(&dq_full[ob], (local >> 1) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
      tc_fence_after();
      float* drow = dq + (static_cast<size_t>(row_base) + qa) * static_cast<size_t>(dq_ld) + w.h * HD;
#pragma unroll 1
      for (int cc = hf; cc < HD / 32; cc += 2) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(lane_addr + L::DQ_COL + ob * HD + cc * 32, v);
        tmem_ld_wait();
        if (qa < S && rope_cos) {
          const float4* cr = reinterpret_cast<const float4*>(rope_cos + static_cast<size_t>(qa) * (HD / 2) + cc * 16);
          const float4* sr = reinterpret_cast<const float4*>(rope_sin + static_cast<size_t>(qa) * (HD / 2) + cc * 16);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const float4 c4 = cr[g], s4 = sr[g];
            const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int p = 4 * g + e;
              const float x0 = __uint_as_float(v[2 * p]), x1 = __uint_as_float(v[2 * p + 1]);
              v[2 * p] = __float_as_uint(round_tf32(__fadd_rn(__fmul_rn(x0, cs[e]), __fmul_rn(x1, sn[e]))));
              v[2 * p + 1] = __float_as_uint(round_tf32(__fadd_rn(__fmul_rn(-x0, sn[e]), __fmul_rn(x1, cs[e]))));
            }
          }
        }
        if (qa < S) {
#pragma unroll
          for (int g = 0; g < 8; ++g)
            reinterpret_cast<float4*>(drow + cc * 32)[g] =
                make_float4(__uint_as_float(v[4 * g]), __uint_as_float(v[4 * g + 1]), __uint_as_float(v[4 * g + 2]),
                            __uint_as_float(v[4 * g + 3]));
        }
      }
      tc_fence_before();
      mbar_arrive(&dq_empty[ob]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (ro.warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// ====================================================== dQ, persistent, two math groups
// attn_bwd_dq_persist_kernel with the 608-thread layout of
// attn_bwd_dkdv2_kernel: math group g takes the K/V steps with (running step
// count) % 2 == g and owns TMEM S/dP set g.  The group that ran an item's
// last step moves the next item's Q and dO into TMEM and writes the item's
// dQ while the other group starts on the next item.  Bit-identical to the
// one-group kernels.
template <int HD>
__global__ void __launch_bounds__(NT2, 1)
    attn_bwd_dq2_persist_kernel(const __grid_constant__ CUtensorMap tmQ, const __grid_constant__ CUtensorMap tmO,
                                const __grid_constant__ CUtensorMap tmKk, const __grid_constant__ CUtensorMap tmKm,
                                const __grid_constant__ CUtensorMap tmVk, const float* __restrict__ lse,
                                const float* __restrict__ Dv, float* __restrict__ dq, int dq_ld, int S, int B, int H,
                                int Hkv, int n_qt, float scale, float scale_log2, const float* __restrict__ rope_cos,
                                const float* __restrict__ rope_sin, int* err) {
  GLC_PDL_ENTRY();
  using L = PDqLayout<HD>;
  extern __shared__ uint8_t smem_raw[];
  uint8_t* sm = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* bars = reinterpret_cast<uint64_t*>(sm + L::OFF_BAR);
  uint64_t *qo_full = bars, *qo_moved = bars + 1, *kv_full = bars + 2, *kv_empty = bars + 5, *s_full = bars + 8,
           *p_full = bars + 10, *set_free = bars + 12, *dq_full = bars + 14, *dq_empty = bars + 16, *drain = bars + 18,
           *drain_acc = bars + 19, *dp_full = bars + 20;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(bars + 22);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  const Roles2 ro;
  const int n_items = H * B * n_qt;
  const int G = H / Hkv;
  const int n_k64 = (S + 63) / 64;

  if (threadIdx.x == 0) {
    mbar_init(qo_full, 1);
    mbar_init(qo_moved, GROUP_THREADS);
    for (int i = 0; i < L::NST; ++i) {
      mbar_init(&kv_full[i], 1);
      mbar_init(&kv_empty[i], 1);
    }
    for (int i = 0; i < L::NSET; ++i) {
      mbar_init(&s_full[i], 1);
      mbar_init(&dp_full[i], 1);
      mbar_init(&p_full[i], GROUP_THREADS);
      mbar_init(&set_free[i], 1);
      mbar_init(&dq_full[i], 1);
      mbar_init(&dq_empty[i], GROUP_THREADS);
    }
    mbar_init(drain, 1);
    mbar_init(drain_acc, 1);
    *abort_flag = 0;
    fence_mbar_init();
  }
  if (ro.warp == 1) tmem_alloc(tmem_slot, L::TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  const uint32_t s0 = smem_u32(sm);

  if (ro.warp == 0) {
    {  // whole warp: elect.sync issues
      int armed[L::NST] = {-1, -1, -1};
      int armed_qo = -1;
      bool ok = true;
      int kv = 0, local = 0;
      for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++local) {
        const FwdItem w = fwd_item(it, H, B, n_qt);
        const int kh = w.h / G, q0 = w.qt * 128, row_base = w.b * S;
        const int nk = min(n_k64, (q0 + 128) / 64);
        if (local > 0 && !mbar_wait_warp(qo_moved, (local - 1) & 1, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) {
          ok = false;
          break;
        }
        mbar_arrive_expect_tx_warp(qo_full, L::Q + L::O);
        tma_tile_warp<HD, 128>(sm + L::OFF_QO, &tmQ, qo_full, w.h * HD, row_base + q0);
        tma_tile_warp<HD, 128>(sm + L::OFF_QO + L::Q, &tmO, qo_full, w.h * HD, row_base + q0);
        armed_qo = local & 1;
        for (int j = 0; j < nk; ++j, ++kv) {
          const int st = kv % L::NST;
          const uint32_t ph = (kv / L::NST) & 1;
          if (!mbar_wait_warp(&kv_empty[st], ph ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_PRODUCER)) { ok = false; break; }
          mbar_arrive_expect_tx_warp(&kv_full[st], L::STAGE);
          uint8_t* base = sm + st * L::STAGE;
          tma_tile_warp<HD, 64>(base, &tmKk, &kv_full[st], kh * HD, row_base + j * 64);
          tma_tile_warp<HD, 64>(base + L::KT, &tmKm, &kv_full[st], kh * HD, row_base + j * 64);
          tma_tile_warp<HD, 64>(base + 2 * L::KT, &tmVk, &kv_full[st], kh * HD, row_base + j * 64);
          armed[st] = static_cast<int>(ph);
        }
      }
      if (!ok) {
        if (armed_qo >= 0) mbar_drain(qo_full, static_cast<uint32_t>(armed_qo), err);
        for (int st = 0; st < L::NST; ++st)
          if (armed[st] >= 0) mbar_drain(&kv_full[st], static_cast<uint32_t>(armed[st]), err);
      }
    }
  } else if (ro.warp == 1) {
    {  // whole warp: elect.sync issues
      constexpr uint32_t idesc_s = umma_idesc_tf32(128, 64, false, false);
      bool ok = true, issued = false;
      int kv = 0, local = 0;
      for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++local) {
        const FwdItem w = fwd_item(it, H, B, n_qt);
        const int nk = min(n_k64, (w.qt * 128 + 128) / 64);
        if (!mbar_wait_warp(qo_moved, local & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
        tc_fence_after();
        for (int j = 0; j < nk; ++j, ++kv) {
          const int st = kv % L::NST, ts = kv % L::NSET;
          const uint32_t base = s0 + st * L::STAGE;
          if (!mbar_wait_warp(&kv_full[st], (kv / L::NST) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
          if (!mbar_wait_warp(&set_free[ts], ((kv / L::NSET) & 1) ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_TMEM)) {
            ok = false;
            break;
          }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < HD / 8; ++kk)
            umma_tf32_ts_warp(tmem + ts * 128, tmem + L::Q_COL + kk * 8, kdesc<64>(base, kk), idesc_s, kk > 0 ? 1u : 0u);
          issued = true;
          umma_commit_warp(&s_full[ts]);
#pragma unroll
          for (int kk = 0; kk < HD / 8; ++kk)
            umma_tf32_ts_warp(tmem + ts * 128 + 64, tmem + L::O_COL + kk * 8, kdesc<64>(base + 2 * L::KT, kk), idesc_s,
                         kk > 0 ? 1u : 0u);
          umma_commit_warp(&dp_full[ts]);
        }
      }
      if (!ok && issued) {
        umma_commit_warp(drain);
        mbar_drain(drain, 0, err);
      }
    }
  } else if (ro.warp == ACC_WARP2) {
    {  // whole warp: elect.sync issues
      constexpr uint32_t idesc_q = umma_idesc_tf32(128, HD, false, true);
      bool ok = true, issued = false;
      int kv = 0, local = 0;
      for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++local) {
        const FwdItem w = fwd_item(it, H, B, n_qt);
        const int nk = min(n_k64, (w.qt * 128 + 128) / 64);
        const int ob = local & 1;
        if (!mbar_wait_warp(&dq_empty[ob], ((local >> 1) & 1) ^ 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_TMEM)) {
          ok = false;
          break;
        }
        tc_fence_after();
        for (int j = 0; j < nk; ++j, ++kv) {
          const int ps = kv % L::NST, pts = kv % L::NSET;
          const uint32_t base = s0 + ps * L::STAGE;
          if (!mbar_wait_warp(&p_full[pts], (kv / L::NSET) & 1, abort_flag, err, GLC_DEV_TIMEOUT_MMA_FULL)) { ok = false; break; }
          tc_fence_after();
#pragma unroll
          for (int kk = 0; kk < 8; ++kk)
            umma_tf32_ts_warp(tmem + L::DQ_COL + ob * HD, tmem + pts * 128 + kk * 8, mdesc<64>(base + L::KT, kk), idesc_q,
                         (j > 0 || kk > 0) ? 1u : 0u);
          issued = true;
          umma_commit_warp(&set_free[pts]);
          umma_commit_warp(&kv_empty[ps]);
        }
        if (!ok) break;
        umma_commit_warp(&dq_full[ob]);
      }
      if (!ok && issued) {
        umma_commit_warp(drain_acc);
        mbar_drain(drain_acc, 0, err);
      }
    }
  } else {
    const int q = ro.quarter(), hf = ro.half(), grp = ro.group();
    const int r = q * 32 + ro.lane;
    const uint32_t lane_addr = tmem + (static_cast<uint32_t>(q * 32) << 16);
    bool ok = true;
    int kv = 0, local = 0;
    // the first item's Q and dO rows -> TMEM (group 0)
    if (grp == 0 && static_cast<int>(blockIdx.x) < n_items) {
      if (__all_sync(0xffffffffu, mbar_wait(qo_full, 0, abort_flag, err, GLC_DEV_TIMEOUT_EPILOGUE))) {
        tile_rows_to_tmem<HD>(sm + L::OFF_QO, r, lane_addr, L::Q_COL, 0, hf);
        tile_rows_to_tmem<HD>(sm + L::OFF_QO + L::Q, r, lane_addr, L::O_COL, HD / 32, hf);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(qo_moved);
      } else {
        ok = false;
      }
    }
    for (int it = blockIdx.x; ok && it < n_items; it += gridDim.x, ++local) {
      const FwdItem w = fwd_item(it, H, B, n_qt);
      const int q0 = w.qt * 128, row_base = w.b * S, qa = q0 + r;
      const int nk = min(n_k64, (q0 + 128) / 64);
      const size_t lrow = (static_cast<size_t>(w.b) * H + w.h) * S + (qa < S ? qa : 0);
      const float lse2 = lse[lrow] * LOG2E, Dq = Dv[lrow];
      const float nDs = -Dq * scale;
      const int kv_first = kv;
      kv += nk;
      for (int j = (grp ^ (kv_first & 1)); j < nk; j += 2) {
        const int kvj = kv_first + j;
        const uint32_t ph = (kvj >> 1) & 1;
        WAIT_OR_BREAK(&s_full[grp], ph, GLC_DEV_TIMEOUT_EPILOGUE);
        tc_fence_after();
        const uint32_t sa = lane_addr + grp * 128 + hf * 32;
        uint32_t sv[32];
        float pf[32];
        tmem_ld_32x32b_x32(sa, sv);
        tmem_ld_wait();
        const int k_lo = j * 64 + hf * 32;
        if (k_lo + 32 <= q0 + 1 && q0 + 128 <= S) {
          const float2 k2 = make_float2(scale_log2, scale_log2), nl2 = make_float2(-lse2, -lse2);
#pragma unroll
          for (int e = 0; e < 32; e += 2) {
            const float2 x = fma2(make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), k2, nl2);
            pf[e] = fast_exp2(x.x);
            pf[e + 1] = fast_exp2(x.y);
          }
        } else {
#pragma unroll
          for (int e = 0; e < 32; ++e) {
            const int key = k_lo + e;
            const bool valid = qa < S && key < S && key <= qa;
            pf[e] = valid ? fast_exp2(fmaf(__uint_as_float(sv[e]), scale_log2, -lse2)) : 0.f;
          }
        }
        WAIT_OR_BREAK(&dp_full[grp], ph, GLC_DEV_TIMEOUT_EPILOGUE);
        tc_fence_after();
        tmem_ld_32x32b_x32(sa + 64, sv);
        tmem_ld_wait();
        const float2 sc2 = make_float2(scale, scale), nd2 = make_float2(nDs, nDs);
#pragma unroll
        for (int e = 0; e < 32; e += 2) {
          const float2 t = fma2(make_float2(__uint_as_float(sv[e]), __uint_as_float(sv[e + 1])), sc2, nd2);
          const float2 g = mul2(make_float2(pf[e], pf[e + 1]), t);
          sv[e] = tf32_operand_bits(g.x);
          sv[e + 1] = tf32_operand_bits(g.y);
        }
        tmem_st_32x32b_x32(sa, sv);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(&p_full[grp]);
      }
      if (!ok) break;
      // the group that ran the item's last step (so waited for its S and dP
      // products, which complete after every earlier product of the item)
      // moves the next item's Q and dO and writes this item's dQ
      if (((kv - 1) & 1) != grp) continue;
      if (it + static_cast<int>(gridDim.x) < n_items) {
        WAIT_OR_BREAK(qo_full, (local + 1) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
        tile_rows_to_tmem<HD>(sm + L::OFF_QO, r, lane_addr, L::Q_COL, 0, hf);
        tile_rows_to_tmem<HD>(sm + L::OFF_QO + L::Q, r, lane_addr, L::O_COL, HD / 32, hf);
        tmem_st_wait();
        tc_fence_before();
        mbar_arrive(qo_moved);
      }
      const int ob = local & 1;
      WAIT_OR_BREAK(&dq_full[ob], (local >> 1) & 1, GLC_DEV_TIMEOUT_EPILOGUE);
      tc_fence_after();
      float* drow = dq + (static_cast<size_t>(row_base) + qa) * static_cast<size_t>(dq_ld) + w.h * HD;
#pragma unroll 1
      for (int cc = hf; cc < HD / 32; cc += 2) {
        uint32_t v[32];
        tmem_ld_32x32b_x32(lane_addr + L::DQ_COL + ob * HD + cc * 32, v);
        tmem_ld_wait();
        if (qa < S && rope_cos) {
          const float4* cr = reinterpret_cast<const float4*>(rope_cos + static_cast<size_t>(qa) * (HD / 2) + cc * 16);
          const float4* sr = reinterpret_cast<const float4*>(rope_sin + static_cast<size_t>(qa) * (HD / 2) + cc * 16);
#pragma unroll
          for (int g = 0; g < 4; ++g) {
            const float4 c4 = cr[g], s4 = sr[g];
            const float cs[4] = {c4.x, c4.y, c4.z, c4.w}, sn[4] = {s4.x, s4.y, s4.z, s4.w};
#pragma unroll
            for (int e = 0; e < 4; ++e) {
              const int p = 4 * g + e;
              const float x0 = __uint_as_float(v[2 * p]), x1 = __uint_as_float(v[2 * p + 1]);
              v[2 * p] = __float_as_uint(round_tf32(__fadd_rn(__fmul_rn(x0, cs[e]), __fmul_rn(x1, sn[e]))));
              v[2 * p + 1] = __float_as_uint(round_tf32(__fadd_rn(__fmul_rn(-x0, sn[e]), __fmul_rn(x1, cs[e]))));
            }
          }
        }
        if (qa < S) {
#pragma unroll
          for (int g = 0; g < 8; ++g)
            reinterpret_cast<float4*>(drow + cc * 32)[g] =
                make_float4(__uint_as_float(v[4 * g]), __uint_as_float(v[4 * g + 1]), __uint_as_float(v[4 * g + 2]),
                            __uint_as_float(v[4 * g + 3]));
        }
      }
      tc_fence_before();
      mbar_arrive(&dq_empty[ob]);
    }
  }
  tc_fence_before();
  __syncthreads();
  if (ro.warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, L::TMEM_COLS);
  }
}

// D[b,h,s] = sum_d dO * O.  HD/4 lanes per (token, head) row, one float4 of
// each operand per lane, 32/(HD/4) rows per warp, one row group per warp.
template <int HD>
__global__ void attn_bwd_prep_tc_kernel(const float* __restrict__ o, const float* __restrict__ dO,
                                        float* __restrict__ D, int T, int S, int H) {
  GLC_PDL_ENTRY();
  constexpr int LPR = HD / 4, RPW = 32 / LPR;
  const int lane = threadIdx.x & 31, sub = lane / LPR, li = lane % LPR;
  const int nrow = T * H;
  const int row = (blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5)) * RPW + sub;
  float s = 0.f;
  if (row < nrow) {
    const float4 a = reinterpret_cast<const float4*>(o + static_cast<size_t>(row) * HD)[li];
    const float4 b = reinterpret_cast<const float4*>(dO + static_cast<size_t>(row) * HD)[li];
    s = (a.x * b.x + a.y * b.y) + (a.z * b.z + a.w * b.w);
  }
#pragma unroll
  for (int off = LPR / 2; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
  if (li == 0 && row < nrow) {
    const int t = row / H, h = row - t * H;
    D[(static_cast<size_t>(t / S) * H + h) * S + (t % S)] = s;
  }
}

// ---------------------------------------------------------------- host side
// rows x cols sub-matrix with row stride ld (elements), boxes {32, box_rows}
int encode(Context* ctx, CUtensorMap* tm, const float* ptr, int cols, int ld, int rows, int box_rows, bool mn) {
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
  cuuint32_t box[2] = {32, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1, 1};
  if (ctx->encode_tiled(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box, estr,
                        mn ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                        CU_TENSOR_MAP_L2_PROMOTION_L2_256B) != 0)
    return ctx->fail(GLC_ERR_INVALID, "attention: cuTensorMapEncodeTiled failed");
  return 0;
}

// The dynamic shared-memory limit of a kernel is a per-device attribute: set
// once per device (flags indexed by device; a second setting from a racing
// host thread is harmless, the flag itself is atomic).
constexpr int kMaxDevices = 64;
using SmemFlags = std::atomic<bool>[kMaxDevices];

template <typename K>
int set_smem(Context* ctx, K kern, int bytes, SmemFlags& done) {
  if (ctx->device < 0 || ctx->device >= kMaxDevices) return ctx->fail(GLC_ERR_UNSUPPORTED, "attention: device index too large");
  if (done[ctx->device].load(std::memory_order_acquire)) return 0;
  cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes);
  if (e != cudaSuccess) return ctx->fail_cuda(e, "attention: cudaFuncSetAttribute");
  done[ctx->device].store(true, std::memory_order_release);
  return 0;
}

int check(Context* ctx, const float* q, const float* k, const float* v, int B, int S, int H, int Hkv, int hd) {
  if (B <= 0 || S <= 0 || H <= 0 || Hkv <= 0 || H % Hkv) return ctx->fail(GLC_ERR_INVALID, "attention: bad B/S/H/Hkv");
  if (hd != 32 && hd != 64) return ctx->fail(GLC_ERR_UNSUPPORTED, "attention: head_dim must be 32 or 64");
  // the kernels index rows (B*S*H) and elements of a head slice in 32 bits and
  // put B and the 128-row tiles in grid dimensions (at most 65535 each)
  if (static_cast<long long>(B) * S * H * hd >= (1LL << 31) || B > 65535 || (S + 127) / 128 > 65535)
    return ctx->fail(GLC_ERR_INVALID, "attention: B*S*H*hd must stay below 2^31 and B at most 65535");
  if (!q || !k || !v || ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15))
    return ctx->fail(GLC_ERR_INVALID, "attention: null or misaligned pointer");
  return 0;
}

template <int HD>
int fwd_impl(Context* ctx, const float* q, int q_ld, const float* k, int k_ld, const float* v, int v_ld, float* o,
             float* lse, int B, int S, int H, int Hkv, bool round_out, cudaStream_t s) {
  using L = FwdLayout<HD>;
  static SmemFlags done, done_p;
  const bool persist = ctx->attn_fwd_variant != 1;  // automatic: persistent
  int rc = persist ? set_smem(ctx, attn_fwd_persist_kernel<HD>, PFwdLayout<HD>::BYTES, done_p)
                   : set_smem(ctx, attn_fwd_tc_kernel<HD>, L::BYTES, done);
  if (rc) return rc;
  const int T = B * S;
  CUtensorMap tq, tk, tv;
  if ((rc = encode(ctx, &tq, q, H * HD, q_ld, T, 128, false)) || (rc = encode(ctx, &tk, k, Hkv * HD, k_ld, T, 128, false)) ||
      (rc = encode(ctx, &tv, v, Hkv * HD, v_ld, T, 128, true)))
    return rc;
  const int n_qt = (S + 127) / 128;
  const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(HD)));
  const double causal = 0.5 * static_cast<double>(S) * (S + 1);
  ProfScope prof(ctx, PROF_ATTN_FWD, 2.0 * 2.0 * B * H * causal * HD, s);
  if (persist) {
    const long long items = static_cast<long long>(H) * B * n_qt;
    if (items >= (1LL << 31)) return ctx->fail(GLC_ERR_INVALID, "attention_fwd: too many work items");
    const int grid = static_cast<int>(items < ctx->num_sms ? items : ctx->num_sms);
    glc::launch_pdl(ctx, attn_fwd_persist_kernel<HD>, grid, NT, PFwdLayout<HD>::BYTES, s, tq, tk, tv, o, lse, S, B, H, Hkv, n_qt,
                    scale * LOG2E, round_out ? 1 : 0, ctx->d_err);
  } else {
    glc::launch_pdl(ctx, attn_fwd_tc_kernel<HD>, dim3(H, B, n_qt), NT, L::BYTES, s, tq, tk, tv, o, lse, S, H, Hkv, n_qt, scale * LOG2E,
                    round_out ? 1 : 0, ctx->d_err);
  }
  GLC_LAUNCH_CHECK(ctx, "attention_fwd (tcgen05)");
  return 0;
}

template <int HD>
int bwd_impl(Context* ctx, const AttnIO& io, const float* o, const float* lse, const float* dO, float* D,
             float* partial, int B, int S, int H, int Hkv, bool round_dv, const float* rope_cos,
             const float* rope_sin, cudaStream_t s) {
  const float *q = io.q, *k = io.k, *v = io.v;
  static SmemFlags done_g, done_g2, done_q, done_pq, done_pq2;
  // automatic: the persistent dQ kernel and the dK/dV kernel, both with two
  // groups of softmax warps
  const bool dq_persist = ctx->attn_dq_variant != 1;
  const bool dq2 = ctx->attn_dq_variant == 0 || ctx->attn_dq_variant == 3;
  const bool dkdv2 = ctx->attn_dkdv_variant != 1;
  int rc = dkdv2 ? set_smem(ctx, attn_bwd_dkdv2_kernel<HD>, Dkdv2Layout<HD>::BYTES, done_g2)
                 : set_smem(ctx, attn_bwd_dkdv_tc_kernel<HD>, DkdvLayout<HD>::BYTES, done_g);
  if (!rc)
    rc = dq2          ? set_smem(ctx, attn_bwd_dq2_persist_kernel<HD>, PDqLayout<HD>::BYTES, done_pq2)
         : dq_persist ? set_smem(ctx, attn_bwd_dq_persist_kernel<HD>, PDqLayout<HD>::BYTES, done_pq)
                      : set_smem(ctx, attn_bwd_dq_tc_kernel<HD>, DqLayout<HD>::BYTES, done_q);
  if (rc) return rc;
  const int T = B * S, G = H / Hkv;
  CUtensorMap tQk64, tQm64, tOk64, tOm64, tK128, tV128, tQ128, tO128, tKk64, tKm64, tVk64;
  const int qw = H * HD, kw = Hkv * HD;
  if ((rc = encode(ctx, &tQk64, q, qw, io.q_ld, T, 64, false)) || (rc = encode(ctx, &tQm64, q, qw, io.q_ld, T, 64, true)) ||
      (rc = encode(ctx, &tOk64, dO, qw, qw, T, 64, false)) || (rc = encode(ctx, &tOm64, dO, qw, qw, T, 64, true)) ||
      (rc = encode(ctx, &tK128, k, kw, io.k_ld, T, 128, false)) || (rc = encode(ctx, &tV128, v, kw, io.v_ld, T, 128, false)) ||
      (rc = encode(ctx, &tQ128, q, qw, io.q_ld, T, 128, false)) || (rc = encode(ctx, &tO128, dO, qw, qw, T, 128, false)) ||
      (rc = encode(ctx, &tKk64, k, kw, io.k_ld, T, 64, false)) || (rc = encode(ctx, &tKm64, k, kw, io.k_ld, T, 64, true)) ||
      (rc = encode(ctx, &tVk64, v, kw, io.v_ld, T, 64, false)))
    return rc;
  const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(HD)));
  const double causal = 0.5 * static_cast<double>(S) * (S + 1);
  ProfScope prof(ctx, PROF_ATTN_BWD, 4.0 * 2.0 * B * H * causal * HD, s);
  {
    const long long nrow = static_cast<long long>(T) * H;
    const long long warps = (nrow + (32 / (HD / 4)) - 1) / (32 / (HD / 4));
    glc::launch_pdl(ctx, attn_bwd_prep_tc_kernel<HD>, static_cast<unsigned>((warps + 7) / 8), 256, 0, s, o, dO, D, T, S, H);
  }
  GLC_LAUNCH_CHECK(ctx, "attention_bwd prep");
  const int n_kt = (S + 127) / 128;
  // CTAs per KV head: the fewest that still give 1.5 waves (each CTA loads
  // its K/V tile once and pays one prologue; fewer partials to sum), or the
  // context's override; 1 without scratch or without grouping
  int nsplit = 1;
  if (G > 1 && partial != nullptr) {
    const long long per = static_cast<long long>(n_kt) * B * Hkv;
    nsplit = G;
    for (int d = 1; d <= G; ++d)
      if (G % d == 0 && 2 * per * d >= 3LL * ctx->num_sms) {
        nsplit = d;
        break;
      }
    if (ctx->attn_split > 0 && G % ctx->attn_split == 0) nsplit = ctx->attn_split;
  }
  auto launch_dkdv = [&](int ns, float* dk_out, float* dv_out, int dk_ld, int dv_ld, int rnd) {
    if (dkdv2)
      glc::launch_pdl(ctx, attn_bwd_dkdv2_kernel<HD>, dim3(Hkv * ns, B, n_kt), NT2, Dkdv2Layout<HD>::BYTES, s,
                      tQk64, tQm64, tOk64, tOm64, tK128, tV128, lse, D, dk_out, dv_out, dk_ld, dv_ld, ns, S, H, Hkv,
                      scale, scale * LOG2E, rnd, ctx->d_err);
    else
      glc::launch_pdl(ctx, attn_bwd_dkdv_tc_kernel<HD>, dim3(Hkv * ns, B, n_kt), NT, DkdvLayout<HD>::BYTES, s,
                      tQk64, tQm64, tOk64, tOm64, tK128, tV128, lse, D, dk_out, dv_out, dk_ld, dv_ld, ns, S, H, Hkv,
                      scale, scale * LOG2E, rnd, ctx->d_err);
  };
  if (nsplit == 1) {
    launch_dkdv(1, io.dk, io.dv, io.dk_ld, io.dv_ld, round_dv ? 1 : 0);
    GLC_LAUNCH_CHECK(ctx, "attention_bwd dkdv (tcgen05)");
    if (rope_cos && (rc = rope(ctx, io.dk, io.dk_ld, T, S, Hkv, HD, rope_cos, rope_sin, true, true, s))) return rc;
  } else {
    // partials [T][Hkv * nsplit][hd] for dK and dV, summed by the group sum
    const int pw = Hkv * nsplit * HD;
    float* pk = partial;
    float* pv = partial + static_cast<size_t>(T) * pw;
    launch_dkdv(nsplit, pk, pv, pw, pw, 0);
    GLC_LAUNCH_CHECK(ctx, "attention_bwd dkdv (tcgen05)");
    if (static_cast<long long>(T) * Hkv * HD / 4 >= (1LL << 31))
      return ctx->fail(GLC_ERR_INVALID, "attention_bwd: B*S*Hkv*hd too large");
    glc::launch_pdl(ctx, group_sum_kernel, grid_for(static_cast<size_t>(T) * Hkv * HD / 4, 256, ctx->num_sms), 256, 0, s,
                    pk, pv, io.dk, io.dv, io.dk_ld, io.dv_ld, T, S, nsplit, Hkv, HD, round_dv ? 1 : 0, rope_cos, rope_sin);
    GLC_LAUNCH_CHECK(ctx, "attention_bwd group sum");
  }
  const int n_qt = (S + 127) / 128;
  if (dq_persist) {
    const long long items = static_cast<long long>(H) * B * n_qt;
    if (items >= (1LL << 31)) return ctx->fail(GLC_ERR_INVALID, "attention_bwd: too many work items");
    const int grid = static_cast<int>(items < ctx->num_sms ? items : ctx->num_sms);
    if (dq2)
      glc::launch_pdl(ctx, attn_bwd_dq2_persist_kernel<HD>, grid, NT2, PDqLayout<HD>::BYTES, s,
                      tQ128, tO128, tKk64, tKm64, tVk64, lse, D, io.dq, io.dq_ld, S, B, H, Hkv, n_qt, scale, scale * LOG2E,
                      rope_cos, rope_sin, ctx->d_err);
    else
      glc::launch_pdl(ctx, attn_bwd_dq_persist_kernel<HD>, grid, NT, PDqLayout<HD>::BYTES, s,
                      tQ128, tO128, tKk64, tKm64, tVk64, lse, D, io.dq, io.dq_ld, S, B, H, Hkv, n_qt, scale, scale * LOG2E,
                      rope_cos, rope_sin, ctx->d_err);
  } else {
    glc::launch_pdl(ctx, attn_bwd_dq_tc_kernel<HD>, dim3(H, B, n_qt), NT, DqLayout<HD>::BYTES, s,
                    tQ128, tO128, tKk64, tKm64, tVk64, lse, D, io.dq, io.dq_ld, S, H, Hkv, n_qt, scale, scale * LOG2E, rope_cos,
                    rope_sin, ctx->d_err);
  }
  GLC_LAUNCH_CHECK(ctx, "attention_bwd dq (tcgen05)");
  return 0;
}

}  // namespace

size_t attention_bwd_partial_floats(int B, int S, int H, int Hkv, int hd) {
  if (H == Hkv) return 0;
  return 2 * static_cast<size_t>(B) * S * H * hd;
}

int attention_fwd(Context* ctx, const AttnIO& io, float* o, float* lse, int B, int S, int H, int Hkv, int hd,
                  bool round_out, cudaStream_t s) {
  int rc = check(ctx, io.q, io.k, io.v, B, S, H, Hkv, hd);
  if (rc) return rc;
  if (((io.q_ld | io.k_ld | io.v_ld) & 3) || io.q_ld < H * hd || io.k_ld < Hkv * hd || io.v_ld < Hkv * hd)
    return ctx->fail(GLC_ERR_INVALID, "attention_fwd: bad row strides");
  if (!o || !lse || (reinterpret_cast<uintptr_t>(o) & 15)) return ctx->fail(GLC_ERR_INVALID, "attention_fwd: bad output");
  return hd == 64 ? fwd_impl<64>(ctx, io.q, io.q_ld, io.k, io.k_ld, io.v, io.v_ld, o, lse, B, S, H, Hkv, round_out, s)
                  : fwd_impl<32>(ctx, io.q, io.q_ld, io.k, io.k_ld, io.v, io.v_ld, o, lse, B, S, H, Hkv, round_out, s);
}

int attention_bwd(Context* ctx, const AttnIO& io, const float* o, const float* lse, const float* dO, float* D,
                  float* partial, int B, int S, int H, int Hkv, int hd, bool round_dv, cudaStream_t s,
                  const float* rope_cos, const float* rope_sin) {
  int rc = check(ctx, io.q, io.k, io.v, B, S, H, Hkv, hd);
  if (rc) return rc;
  if (!o || !lse || !dO || !io.dq || !io.dk || !io.dv || !D ||
      ((reinterpret_cast<uintptr_t>(o) | reinterpret_cast<uintptr_t>(dO) | reinterpret_cast<uintptr_t>(io.dq) |
        reinterpret_cast<uintptr_t>(io.dk) |
        reinterpret_cast<uintptr_t>(io.dv)) & 15))
    return ctx->fail(GLC_ERR_INVALID, "attention_bwd: null or misaligned pointer");
  if (((io.q_ld | io.k_ld | io.v_ld | io.dq_ld | io.dk_ld | io.dv_ld) & 3) || io.q_ld < H * hd || io.dq_ld < H * hd ||
      io.k_ld < Hkv * hd || io.v_ld < Hkv * hd || io.dk_ld < Hkv * hd || io.dv_ld < Hkv * hd)
    return ctx->fail(GLC_ERR_INVALID, "attention_bwd: bad row strides");
  if ((rope_cos == nullptr) != (rope_sin == nullptr) ||
      ((reinterpret_cast<uintptr_t>(rope_cos) | reinterpret_cast<uintptr_t>(rope_sin)) & 15))
    return ctx->fail(GLC_ERR_INVALID, "attention_bwd: bad RoPE tables");
  return hd == 64 ? bwd_impl<64>(ctx, io, o, lse, dO, D, partial, B, S, H, Hkv, round_dv, rope_cos, rope_sin, s)
                  : bwd_impl<32>(ctx, io, o, lse, dO, D, partial, B, S, H, Hkv, round_dv, rope_cos, rope_sin, s);
}

}  // namespace glc
