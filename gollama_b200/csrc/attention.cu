// Causal self-attention forward and backward, fp32 on the CUDA cores
// (flash-style: 64x64 tiles in shared memory, online softmax, no S x S
// matrix in global memory).
//
// Semantics follow forwardAttention (pkg/train/trainer.go:331-386): token i of
// sequence b attends to positions j <= i of the same sequence, scores are
// (q.k)*float32(1/sqrt(hd)), softmax over them, weighted sum of v.  Heads map
// to KV heads as in pkg/model/attention.go:118,149 (kvHead = h / (H/Hkv)).
// q/o rows have H*hd floats, k/v rows Hkv*hd; token t = b*S + s.
//
// Backward (Llama mode; the reference attaches no GradFn, trainer.go:335-337):
//   P = exp(S - lse), D_i = sum_d dO_i*O_i, dS = P*(dP - D)*scale,
//   dV_j = sum_i P_ij dO_i, dK_j = sum_i dS_ij q_i, dQ_i = sum_j dS_ij k_j.
// Two kernels keep it deterministic without atomics: one CTA per (KV tile,
// KV head) sums dK/dV over every query head of its group and every query
// tile; one CTA per (query tile, head) computes dQ.
#include <cfloat>
#include <cmath>

#include "glc_internal.h"
#include "sm100.cuh"

namespace glc {
namespace {

constexpr int BT = 64;       // rows per tile (queries and keys)
constexpr int PT = BT + 4;   // padded pitch of [*][64] tiles

template <int HD>
struct AttnCfg {
  static constexpr int DPT = HD / 16;  // output columns per thread
  static constexpr int PHD = HD + 4;   // padded pitch of [*][HD] tiles
};

// Loads rows [r0, r0+64) x [0, HD) of a [*, stride] matrix, zero beyond `limit`.
// trans = true stores dst[d*PT + r]; false stores dst[r*PHD + d].
template <int HD, bool TRANS>
__device__ __forceinline__ void load_tile(float* dst, const float* src, size_t stride, int r0, int limit) {
  constexpr int PHD = AttnCfg<HD>::PHD;
  for (int idx = threadIdx.x; idx < BT * HD / 4; idx += blockDim.x) {
    const int r = idx / (HD / 4), d = (idx % (HD / 4)) * 4;
    float4 v = make_float4(0.f, 0.f, 0.f, 0.f);
    if (r0 + r < limit) v = *reinterpret_cast<const float4*>(src + static_cast<size_t>(r0 + r) * stride + d);
    if (TRANS) {
      dst[(d + 0) * PT + r] = v.x;
      dst[(d + 1) * PT + r] = v.y;
      dst[(d + 2) * PT + r] = v.z;
      dst[(d + 3) * PT + r] = v.w;
    } else {
      *reinterpret_cast<float4*>(dst + r * PHD + d) = v;
    }
  }
}

__device__ __forceinline__ float4 ld4(const float* p) { return *reinterpret_cast<const float4*>(p); }
__device__ __forceinline__ float f4(const float4& v, int i) { return i == 0 ? v.x : i == 1 ? v.y : i == 2 ? v.z : v.w; }

// s[i][j] += sum_d A[d][ra+i] * B[d][cb+j] over transposed tiles
template <int HD>
__device__ __forceinline__ void tile_dot(float (&s)[4][4], const float* At, const float* Bt, int ra, int cb) {
#pragma unroll 8
  for (int d = 0; d < HD; ++d) {
    const float4 a = ld4(At + d * PT + ra), b = ld4(Bt + d * PT + cb);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int j = 0; j < 4; ++j) s[i][j] += f4(a, i) * f4(b, j);
  }
}

template <int HD>
__global__ void __launch_bounds__(256) attn_fwd_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                       const float* __restrict__ v, float* __restrict__ o,
                                                       float* __restrict__ lse, int S, int H, int Hkv, float scale,
                                                       int round_out) {
  constexpr int DPT = AttnCfg<HD>::DPT, PHD = AttnCfg<HD>::PHD;
  extern __shared__ float sm[];
  float* Qt = sm;               // [HD][PT]
  float* Kt = Qt + HD * PT;     // [HD][PT]
  float* Vs = Kt + HD * PT;     // [BT][PHD]
  float* Pt = Vs + BT * PHD;    // [BT][PT]  Pt[c][r]
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (H / Hkv);
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int q0 = qt * BT;
  const size_t qs = static_cast<size_t>(H) * HD, ks = static_cast<size_t>(Hkv) * HD;
  const float* qb = q + static_cast<size_t>(b) * S * qs + h * HD;
  const float* kb = k + static_cast<size_t>(b) * S * ks + kh * HD;
  const float* vb = v + static_cast<size_t>(b) * S * ks + kh * HD;

  load_tile<HD, true>(Qt, qb, qs, q0, S);
  float m[4], l[4], acc[4][DPT];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    m[i] = -FLT_MAX;
    l[i] = 0.f;
#pragma unroll
    for (int d = 0; d < DPT; ++d) acc[i][d] = 0.f;
  }
  for (int j = 0; j <= qt; ++j) {
    const int k0 = j * BT;
    __syncthreads();
    load_tile<HD, true>(Kt, kb, ks, k0, S);
    load_tile<HD, false>(Vs, vb, ks, k0, S);
    __syncthreads();
    float s[4][4] = {};
    tile_dot<HD>(s, Qt, Kt, ty * 4, tx * 4);
#pragma unroll
    for (int i = 0; i < 4; ++i) {
      const int ra = q0 + ty * 4 + i;
      float mx = -FLT_MAX;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const int ca = k0 + tx * 4 + jj;
        s[i][jj] = (ca > ra || ca >= S) ? -FLT_MAX : s[i][jj] * scale;
        mx = fmaxf(mx, s[i][jj]);
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, off));
      const float mnew = fmaxf(m[i], mx);
      const float corr = expf(m[i] - mnew);
      float rs = 0.f;
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) {
        const float p = s[i][jj] == -FLT_MAX ? 0.f : expf(s[i][jj] - mnew);
        Pt[(tx * 4 + jj) * PT + ty * 4 + i] = p;
        rs += p;
      }
#pragma unroll
      for (int off = 1; off < 16; off <<= 1) rs += __shfl_xor_sync(0xffffffffu, rs, off);
      l[i] = l[i] * corr + rs;
      m[i] = mnew;
#pragma unroll
      for (int d = 0; d < DPT; ++d) acc[i][d] *= corr;
    }
    __syncthreads();
#pragma unroll 4
    for (int c = 0; c < BT; ++c) {
      const float4 pa = ld4(Pt + c * PT + ty * 4);
#pragma unroll
      for (int d = 0; d < DPT; ++d) {
        const float vv = Vs[c * PHD + tx * DPT + d];
#pragma unroll
        for (int i = 0; i < 4; ++i) acc[i][d] += f4(pa, i) * vv;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ra = q0 + ty * 4 + i;
    if (ra >= S) continue;
    float* orow = o + (static_cast<size_t>(b) * S + ra) * qs + h * HD + tx * DPT;
#pragma unroll
    for (int d = 0; d < DPT; ++d) {
      float val = acc[i][d] / l[i];
      if (round_out) val = round_tf32(val);
      orow[d] = val;
    }
    if (tx == 0) lse[(static_cast<size_t>(b) * H + h) * S + ra] = m[i] + logf(l[i]);
  }
}

// D[b,h,s] = sum_d dO*O
__global__ void attn_bwd_prep_kernel(const float* __restrict__ o, const float* __restrict__ dO, float* __restrict__ D,
                                     int T, int S, int H, int hd) {
  const int lane = threadIdx.x & 31;
  const int nrow = T * H;
  for (int row = blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5); row < nrow; row += gridDim.x * (blockDim.x >> 5)) {
    const int t = row / H, h = row % H;
    const float* op = o + (static_cast<size_t>(t) * H + h) * hd;
    const float* dp = dO + (static_cast<size_t>(t) * H + h) * hd;
    float s = 0.f;
    for (int d = lane; d < hd; d += 32) s += op[d] * dp[d];
#pragma unroll
    for (int off = 16; off > 0; off >>= 1) s += __shfl_xor_sync(0xffffffffu, s, off);
    if (lane == 0) {
      const int b = t / S, ss = t % S;
      D[(static_cast<size_t>(b) * H + h) * S + ss] = s;
    }
  }
}

// S-block (rows ra.., cols cb..) of P and dS*1 (scale folded in) for one tile pair.
template <int HD>
__device__ __forceinline__ void p_and_ds(float (&P)[4][4], float (&dS)[4][4], const float* Qt, const float* Kt,
                                         const float* dOt, const float* Vt, const float (&lse_r)[4],
                                         const float (&D_r)[4], int q0, int k0, int S, float scale) {
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  float s[4][4] = {}, dp[4][4] = {};
  tile_dot<HD>(s, Qt, Kt, ty * 4, tx * 4);
  tile_dot<HD>(dp, dOt, Vt, ty * 4, tx * 4);
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ra = q0 + ty * 4 + i;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
      const int ca = k0 + tx * 4 + jj;
      const bool valid = ca <= ra && ca < S && ra < S;
      const float p = valid ? expf(s[i][jj] * scale - lse_r[i]) : 0.f;
      P[i][jj] = p;
      dS[i][jj] = p * (dp[i][jj] - D_r[i]) * scale;
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(256) attn_bwd_dkdv_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                            const float* __restrict__ v, const float* __restrict__ dO,
                                                            const float* __restrict__ lse, const float* __restrict__ D,
                                                            float* __restrict__ dk, float* __restrict__ dv, int S,
                                                            int H, int Hkv, float scale, int round_dv) {
  constexpr int DPT = AttnCfg<HD>::DPT, PHD = AttnCfg<HD>::PHD;
  extern __shared__ float sm[];
  float* Kt = sm;                // [HD][PT]
  float* Vt = Kt + HD * PT;      // [HD][PT]
  float* Qt = Vt + HD * PT;      // [HD][PT]
  float* dOt = Qt + HD * PT;     // [HD][PT]
  float* Qs = dOt + HD * PT;     // [BT][PHD]
  float* dOs = Qs + BT * PHD;    // [BT][PHD]
  float* Ps = dOs + BT * PHD;    // [BT][PT]  Ps[r][c]
  float* dSs = Ps + BT * PT;     // [BT][PT]
  const int kt = blockIdx.x, kh = blockIdx.y, b = blockIdx.z;
  const int G = H / Hkv;
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int k0 = kt * BT;
  const size_t qs = static_cast<size_t>(H) * HD, ks = static_cast<size_t>(Hkv) * HD;
  load_tile<HD, true>(Kt, k + static_cast<size_t>(b) * S * ks + kh * HD, ks, k0, S);
  load_tile<HD, true>(Vt, v + static_cast<size_t>(b) * S * ks + kh * HD, ks, k0, S);
  float dka[4][DPT] = {}, dva[4][DPT] = {};
  const int nqt = (S + BT - 1) / BT;
  for (int hh = 0; hh < G; ++hh) {
    const int h = kh * G + hh;
    const float* qb = q + static_cast<size_t>(b) * S * qs + h * HD;
    const float* db = dO + static_cast<size_t>(b) * S * qs + h * HD;
    for (int qt = kt; qt < nqt; ++qt) {
      const int q0 = qt * BT;
      __syncthreads();
      load_tile<HD, true>(Qt, qb, qs, q0, S);
      load_tile<HD, true>(dOt, db, qs, q0, S);
      load_tile<HD, false>(Qs, qb, qs, q0, S);
      load_tile<HD, false>(dOs, db, qs, q0, S);
      float lse_r[4], D_r[4];
#pragma unroll
      for (int i = 0; i < 4; ++i) {
        const int ra = q0 + ty * 4 + i;
        const size_t ix = (static_cast<size_t>(b) * H + h) * S + (ra < S ? ra : 0);
        lse_r[i] = lse[ix];
        D_r[i] = D[ix];
      }
      __syncthreads();
      float P[4][4], dS[4][4];
      p_and_ds<HD>(P, dS, Qt, Kt, dOt, Vt, lse_r, D_r, q0, k0, S, scale);
#pragma unroll
      for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int jj = 0; jj < 4; ++jj) {
          Ps[(ty * 4 + i) * PT + tx * 4 + jj] = P[i][jj];
          dSs[(ty * 4 + i) * PT + tx * 4 + jj] = dS[i][jj];
        }
      __syncthreads();
#pragma unroll 4
      for (int r = 0; r < BT; ++r) {
        const float4 pa = ld4(Ps + r * PT + ty * 4), sa = ld4(dSs + r * PT + ty * 4);
#pragma unroll
        for (int d = 0; d < DPT; ++d) {
          const float dov = dOs[r * PHD + tx * DPT + d], qv = Qs[r * PHD + tx * DPT + d];
#pragma unroll
          for (int i = 0; i < 4; ++i) {
            dva[i][d] += f4(pa, i) * dov;
            dka[i][d] += f4(sa, i) * qv;
          }
        }
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ca = k0 + ty * 4 + i;
    if (ca >= S) continue;
    const size_t base = (static_cast<size_t>(b) * S + ca) * ks + kh * HD + tx * DPT;
#pragma unroll
    for (int d = 0; d < DPT; ++d) {
      dk[base + d] = dka[i][d];
      dv[base + d] = round_dv ? round_tf32(dva[i][d]) : dva[i][d];
    }
  }
}

template <int HD>
__global__ void __launch_bounds__(256) attn_bwd_dq_kernel(const float* __restrict__ q, const float* __restrict__ k,
                                                          const float* __restrict__ v, const float* __restrict__ dO,
                                                          const float* __restrict__ lse, const float* __restrict__ D,
                                                          float* __restrict__ dq, int S, int H, int Hkv, float scale) {
  constexpr int DPT = AttnCfg<HD>::DPT, PHD = AttnCfg<HD>::PHD;
  extern __shared__ float sm[];
  float* Qt = sm;                // [HD][PT]
  float* dOt = Qt + HD * PT;     // [HD][PT]
  float* Kt = dOt + HD * PT;     // [HD][PT]
  float* Vt = Kt + HD * PT;      // [HD][PT]
  float* Ks = Vt + HD * PT;      // [BT][PHD]
  float* dSt = Ks + BT * PHD;    // [BT][PT]  dSt[c][r]
  const int qt = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
  const int kh = h / (H / Hkv);
  const int tid = threadIdx.x, ty = tid >> 4, tx = tid & 15;
  const int q0 = qt * BT;
  const size_t qs = static_cast<size_t>(H) * HD, ks = static_cast<size_t>(Hkv) * HD;
  load_tile<HD, true>(Qt, q + static_cast<size_t>(b) * S * qs + h * HD, qs, q0, S);
  load_tile<HD, true>(dOt, dO + static_cast<size_t>(b) * S * qs + h * HD, qs, q0, S);
  float lse_r[4], D_r[4];
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ra = q0 + ty * 4 + i;
    const size_t ix = (static_cast<size_t>(b) * H + h) * S + (ra < S ? ra : 0);
    lse_r[i] = lse[ix];
    D_r[i] = D[ix];
  }
  const float* kb = k + static_cast<size_t>(b) * S * ks + kh * HD;
  const float* vb = v + static_cast<size_t>(b) * S * ks + kh * HD;
  float dqa[4][DPT] = {};
  for (int j = 0; j <= qt; ++j) {
    const int k0 = j * BT;
    __syncthreads();
    load_tile<HD, true>(Kt, kb, ks, k0, S);
    load_tile<HD, true>(Vt, vb, ks, k0, S);
    load_tile<HD, false>(Ks, kb, ks, k0, S);
    __syncthreads();
    float P[4][4], dS[4][4];
    p_and_ds<HD>(P, dS, Qt, Kt, dOt, Vt, lse_r, D_r, q0, k0, S, scale);
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
      for (int jj = 0; jj < 4; ++jj) dSt[(tx * 4 + jj) * PT + ty * 4 + i] = dS[i][jj];
    __syncthreads();
#pragma unroll 4
    for (int c = 0; c < BT; ++c) {
      const float4 sa = ld4(dSt + c * PT + ty * 4);
#pragma unroll
      for (int d = 0; d < DPT; ++d) {
        const float kv = Ks[c * PHD + tx * DPT + d];
#pragma unroll
        for (int i = 0; i < 4; ++i) dqa[i][d] += f4(sa, i) * kv;
      }
    }
  }
#pragma unroll
  for (int i = 0; i < 4; ++i) {
    const int ra = q0 + ty * 4 + i;
    if (ra >= S) continue;
    float* row = dq + (static_cast<size_t>(b) * S + ra) * qs + h * HD + tx * DPT;
#pragma unroll
    for (int d = 0; d < DPT; ++d) row[d] = dqa[i][d];
  }
}

template <int HD>
constexpr size_t fwd_smem() { return sizeof(float) * (2 * HD * PT + BT * AttnCfg<HD>::PHD + BT * PT); }
template <int HD>
constexpr size_t dkdv_smem() { return sizeof(float) * (4 * HD * PT + 2 * BT * AttnCfg<HD>::PHD + 2 * BT * PT); }
template <int HD>
constexpr size_t dq_smem() { return sizeof(float) * (4 * HD * PT + BT * AttnCfg<HD>::PHD + BT * PT); }

template <int HD>
int set_attrs(Context* ctx) {
  static bool done[8] = {false};
  if (done[ctx->device & 7]) return 0;
  cudaError_t e = cudaFuncSetAttribute(attn_fwd_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)fwd_smem<HD>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_bwd_dkdv_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dkdv_smem<HD>());
  if (e == cudaSuccess)
    e = cudaFuncSetAttribute(attn_bwd_dq_kernel<HD>, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dq_smem<HD>());
  if (e != cudaSuccess) return ctx->fail_cuda(e, "attention: cudaFuncSetAttribute");
  done[ctx->device & 7] = true;
  return 0;
}

int check_args(Context* ctx, const float* q, const float* k, const float* v, int B, int S, int H, int Hkv, int hd) {
  if (B <= 0 || S <= 0 || H <= 0 || Hkv <= 0 || H % Hkv) return ctx->fail(GLC_ERR_INVALID, "attention: bad B/S/H/Hkv");
  if (hd != 32 && hd != 64) return ctx->fail(GLC_ERR_UNSUPPORTED, "attention: head_dim must be 32 or 64");
  if (!q || !k || !v || ((reinterpret_cast<uintptr_t>(q) | reinterpret_cast<uintptr_t>(k) | reinterpret_cast<uintptr_t>(v)) & 15))
    return ctx->fail(GLC_ERR_INVALID, "attention: null or misaligned pointer");
  return 0;
}

}  // namespace

int attention_fwd(Context* ctx, const float* q, const float* k, const float* v, float* o, float* lse, int B, int S,
                  int H, int Hkv, int hd, bool round_out, cudaStream_t s) {
  int rc = check_args(ctx, q, k, v, B, S, H, Hkv, hd);
  if (rc) return rc;
  if (!o || !lse) return ctx->fail(GLC_ERR_INVALID, "attention_fwd: null output");
  const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(hd)));
  dim3 grid((S + BT - 1) / BT, H, B);
  const double causal = 0.5 * static_cast<double>(S) * (S + 1);
  ProfScope prof(ctx, PROF_ATTN_FWD, 2.0 * 2.0 * B * H * causal * hd, s);
  if (hd == 64) {
    if ((rc = set_attrs<64>(ctx))) return rc;
    attn_fwd_kernel<64><<<grid, 256, fwd_smem<64>(), s>>>(q, k, v, o, lse, S, H, Hkv, scale, round_out ? 1 : 0);
  } else {
    if ((rc = set_attrs<32>(ctx))) return rc;
    attn_fwd_kernel<32><<<grid, 256, fwd_smem<32>(), s>>>(q, k, v, o, lse, S, H, Hkv, scale, round_out ? 1 : 0);
  }
  GLC_LAUNCH_CHECK(ctx, "attention_fwd");
  return 0;
}

int attention_bwd(Context* ctx, const float* q, const float* k, const float* v, const float* o, const float* lse,
                  const float* dO, float* dq, float* dk, float* dv, float* D, int B, int S, int H, int Hkv, int hd,
                  bool round_dv, cudaStream_t s) {
  int rc = check_args(ctx, q, k, v, B, S, H, Hkv, hd);
  if (rc) return rc;
  if (!o || !lse || !dO || !dq || !dk || !dv || !D) return ctx->fail(GLC_ERR_INVALID, "attention_bwd: null pointer");
  const float scale = static_cast<float>(1.0 / std::sqrt(static_cast<double>(hd)));
  const int T = B * S;
  const double causal = 0.5 * static_cast<double>(S) * (S + 1);
  ProfScope prof(ctx, PROF_ATTN_BWD, 4.0 * 2.0 * B * H * causal * hd, s);
  attn_bwd_prep_kernel<<<grid_for(static_cast<size_t>(T) * H, 8, ctx->num_sms, 16), 256, 0, s>>>(o, dO, D, T, S, H, hd);
  GLC_LAUNCH_CHECK(ctx, "attention_bwd prep");
  dim3 gkv((S + BT - 1) / BT, Hkv, B), gq((S + BT - 1) / BT, H, B);
  if (hd == 64) {
    if ((rc = set_attrs<64>(ctx))) return rc;
    attn_bwd_dkdv_kernel<64><<<gkv, 256, dkdv_smem<64>(), s>>>(q, k, v, dO, lse, D, dk, dv, S, H, Hkv, scale, round_dv ? 1 : 0);
    GLC_LAUNCH_CHECK(ctx, "attention_bwd dkdv");
    attn_bwd_dq_kernel<64><<<gq, 256, dq_smem<64>(), s>>>(q, k, v, dO, lse, D, dq, S, H, Hkv, scale);
  } else {
    if ((rc = set_attrs<32>(ctx))) return rc;
    attn_bwd_dkdv_kernel<32><<<gkv, 256, dkdv_smem<32>(), s>>>(q, k, v, dO, lse, D, dk, dv, S, H, Hkv, scale, round_dv ? 1 : 0);
    GLC_LAUNCH_CHECK(ctx, "attention_bwd dkdv");
    attn_bwd_dq_kernel<32><<<gq, 256, dq_smem<32>(), s>>>(q, k, v, dO, lse, D, dq, S, H, Hkv, scale);
  }
  GLC_LAUNCH_CHECK(ctx, "attention_bwd dq");
  return 0;
}

}  // namespace glc
