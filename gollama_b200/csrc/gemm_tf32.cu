// TF32 tensor-core GEMM for sm_100a: TMA -> shared memory (128B swizzle) ->
// tcgen05.mma (kind::tf32, fp32 accumulate in TMEM) -> tcgen05.ld epilogue.
//
// C[M,N] = A[M,K] . B[N,K]^T  (+ C if accumulate) (+ R if residual)
//
// The reference computes every linear layer through MatMulGrad
// (pkg/tensor/grad.go:81-155): the forward C = A.B^T via MatMulTransposeB
// (pkg/tensor/matmul.go:145-234), dA += dC.B (grad.go:102-116) and
// dB += dC^T.A (grad.go:118-152).  All three are this one kernel with
// different operand majors:
//   forward  Y  = X . W^T   A = X  (K-major)  B = W (K-major)
//   dX      dX += dY . W    A = dY (K-major)  B = W (MN-major: W is [N_out, K_in])
//   dW      dW += dY^T . X  A = dY (MN-major) B = X (MN-major)
//
// Structure: one persistent CTA per SM, 192 threads:
//   warp 0      TMA producer (one thread), STAGES-deep smem ring
//   warp 1      TMEM allocator + UMMA issuer (one thread)
//   warps 2..5  epilogue: TMEM -> registers -> global (fp32), 1 row per thread
// Two TMEM accumulators (2 x BN columns) let the epilogue of tile i overlap
// the main loop of tile i+1.
//
// Two kernels share this structure:
//   gemm_tf32_kernel       one CTA per 128x256 tile (tcgen05.mma.cta_group::1)
//   gemm_tf32_pair_kernel  a (2,1,1) cluster per 256x256 tile
//                          (tcgen05.mma.cta_group::2): each CTA loads 128 rows
//                          of A and 128 rows of B, so an SM streams 32 KB of
//                          operands per 32-deep k-block instead of 48 KB for
//                          the same MMA work.  At full tensor rate the
//                          single-CTA tile needs ~96 B/clk/SM from L2, near the
//                          L2->SM limit; the pair tile needs ~64.
// The pair kernel serves problems with M > 128; tiny ones keep the
// single-CTA tile.
//
// Up to two problems (the dA and dB of one MatMulGrad) share a launch; on CTA
// pairs they walk host-built tile lists when those balance the pairs better
// than the fixed rotation (pair_schedule).  The epilogue can also add the
// squares of the values it stores into float64 slots (a gradient's share of
// the clip norm, Problem::sumsq).
#include <algorithm>
#include <atomic>
#include <functional>
#include <queue>
#include <utility>

#include "glc_internal.h"
#include "go_math.cuh"
#include "sm100.cuh"

namespace glc {

namespace {

constexpr int BM = 128;         // UMMA M (one CTA, cta_group::1)
constexpr int BN = 256;         // UMMA N
constexpr int BK = 32;          // fp32 elements per k-block = 128 bytes = one swizzle row
constexpr int UMMA_K = 8;       // K per tcgen05.mma for tf32
constexpr int STAGES = 4;
constexpr int A_BYTES = BM * BK * 4;            // 16 KB
constexpr int B_BYTES = BN * BK * 4;            // 32 KB
constexpr int STAGE_BYTES = A_BYTES + B_BYTES;  // 48 KB
constexpr int TMEM_COLS = 2 * BN;               // two accumulators
constexpr int NUM_THREADS = 192;
// CTA-pair kernel: P_EPI_WARPS epilogue warps, P_EPI_WARPS / 4 per TMEM lane
// quarter, each draining an equal share of the accumulator's columns.  Four
// keep pace with the MMAs for the plain epilogue; eight made the SwiGLU
// epilogue 27 % faster but plain GEMMs ~5 % slower.
constexpr int P_EPI_WARPS = 4;
constexpr int P_NUM_THREADS = 64 + 32 * P_EPI_WARPS;
constexpr int P_SPLIT = P_EPI_WARPS / 4;  // warps per lane quarter
constexpr int SMEM_BYTES = STAGES * STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers*/;

// One GEMM problem of a (possibly grouped) launch.
struct Problem {
  float* C;
  const float* R;
  int M, N, K;
  int ldc, ldr;
  int accumulate;  // C += acc
  int round_out;   // round stored values to TF32 (RN)
  // Sum of squares of the stored values (a gradient's share of the clip
  // norm): each epilogue warp writes its float64 sum of a tile to
  // sumsq[tile * slots_per_tile + warp slot]; nullptr: none.
  double* sumsq;
  int a_mn, b_mn;  // operand majors
  int a_3d, b_3d;  // MN-major operand described as [MN/32 chunks][K][32]: one TMA per k-block
  // SwiGLU epilogue (CTA-pair kernel only): glu = F; a tile covers 128 h
  // columns, CTA 0 loading gate rows [n0, n0+128) of B and CTA 1 the up rows
  // [F + n0, ...), so each CTA's accumulator holds gate in columns 0..127 and
  // up in 128..255 for the same outputs.
  int glu;
  float* h;
  int ldh;
  int round_h;
  int glu_fast;    // h with expf (Llama semantics) instead of the reference's exp32
  int m_tiles, n_tiles, k_blocks, tiles;
  // Tile order.  Concurrent tiles share the operand of the slow-moving index
  // through L2 and stream the other; the operand of the fast-moving index is
  // re-read once per sweep unless it stays in L2.  n_fast walks N fastest
  // (A tiles stay hot), chosen when A is the larger operand.
  int n_fast;
};

// Up to two independent problems share one persistent launch: their tiles
// form one index space (problem 0 first), so the two GEMMs of a MatMulGrad
// GradFn (dA and dB) fill the machine together instead of each leaving a
// partial last wave.
struct GroupArgs {
  Problem p[2];
  int nprob;
  int total_tiles;
  int* err;
  // Tile order of the CTA-pair kernel: nullptr walks tile = cluster,
  // cluster + clusters, ...; otherwise sched[c] .. sched[c + 1] index into
  // the tile list sched[clusters + 1 ..] the clusters of cluster c.
  const int* sched;
  // Dynamic order (CTA-pair kernel, when not null): a zeroed counter in
  // device memory; each pair takes the next tile index when it is ready for
  // one, so pairs that start late (their SMs busy with another kernel, such
  // as a collective on the communication stream) simply take fewer tiles.
  int* dyn;
};

// The range of list positions of cluster c and the tile at position it.
__device__ __forceinline__ void sched_range(const GroupArgs& a, int c, int nclusters, int& it0, int& it1, int& step) {
  if (a.sched) {
    it0 = a.sched[c];
    it1 = a.sched[c + 1];
    step = 1;
  } else {
    it0 = c;
    it1 = a.total_tiles;
    step = nclusters;
  }
}
__device__ __forceinline__ int sched_tile(const GroupArgs& a, int nclusters, int it) {
  return a.sched ? a.sched[nclusters + 1 + it] : it;
}

// UMMA descriptor of the operand for k-step kk inside one stage's tile.
//   K-major : rows of 128 B (16-byte-chunk swizzle), 8-row groups 1 KB apart;
//             a k-step advances 32 B inside the swizzle row.
//   MN-major: 4 KB chunks of 32 K-rows x 32 MN-elements (32-byte-chunk
//             swizzle), 4-row K groups 512 B apart, chunks 4 KB apart (LBO);
//             a k-step (8 K-rows) advances 1 KB.
__device__ __forceinline__ uint64_t operand_desc(bool mn, uint32_t tile_saddr, int kk) {
  return mn ? umma_sdesc(tile_saddr + kk * 1024, /*LBO: MN chunk stride*/ BK * 128, /*SBO*/ 512,
                         UMMA_LAYOUT_SW128_BASE32B)
            : umma_sdesc(tile_saddr + kk * 32, /*LBO unused*/ 16, /*SBO: 8 rows*/ 1024, UMMA_LAYOUT_SW128);
}

__device__ __forceinline__ void load_operand(bool mn, bool mn3d, int rows, void* sdst, const CUtensorMap* tm,
                                             uint64_t* bar, int mn0, int k0) {
  if (mn3d) {
    // all rows/32 chunks of 32 MN-elements x BK K-rows in one copy (same smem layout)
    tma_load_3d(sdst, tm, bar, 0, k0, mn0 / 32);
  } else if (mn) {
    // tensor map dims {MN, K}, box {32, BK}: one 4 KB chunk per 32 MN-elements
    for (int c = 0; c < rows / 32; ++c)
      tma_load_2d(static_cast<uint8_t*>(sdst) + c * (BK * 128), tm, bar, mn0 + 32 * c, k0);
  } else {
    // tensor map dims {K, MN}, box {BK, rows}
    tma_load_2d(sdst, tm, bar, k0, mn0);
  }
}

struct TileRef {
  int prob, m0, n0;
};
template <int TILE_M>
__device__ __forceinline__ TileRef locate(const GroupArgs& a, int tile) {
  TileRef t;
  t.prob = (tile < a.p[0].tiles) ? 0 : 1;
  const int lt = t.prob ? tile - a.p[0].tiles : tile;
  const Problem& p = a.p[t.prob];
  const int tn = p.glu ? 128 : BN;  // output columns per tile
  if (p.n_fast) {
    t.n0 = (lt % p.n_tiles) * tn;
    t.m0 = (lt / p.n_tiles) * TILE_M;
  } else {
    t.m0 = (lt % p.m_tiles) * TILE_M;
    t.n0 = (lt / p.m_tiles) * tn;
  }
  return t;
}

__global__ void __launch_bounds__(NUM_THREADS, 1)
    gemm_tf32_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmB0,
                     const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmB1,
                     const GroupArgs args) {
  GLC_PDL_ENTRY();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + STAGES * STAGE_BYTES);
  uint64_t* empty_bar = full_bar + STAGES;
  uint64_t* tfull_bar = empty_bar + STAGES;   // [2]
  uint64_t* tempty_bar = tfull_bar + 2;       // [2]
  uint64_t* drain_bar = tempty_bar + 2;       // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 4 * 32);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA0);
    tma_prefetch_desc(&tmB0);
    if (args.nprob > 1) {
      tma_prefetch_desc(&tmA1);
      tma_prefetch_desc(&tmB1);
    }
  }
  if (warp == 1) tmem_alloc(tmem_slot, TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int in_flight = 0;  // stages issued (capped at STAGES) for the abort drain
      bool ok = true;
      for (int tile = blockIdx.x; tile < args.total_tiles && ok; tile += gridDim.x) {
        const TileRef t = locate<BM>(args, tile);
        const Problem& p = args.p[t.prob];
        const CUtensorMap* tmA = t.prob ? &tmA1 : &tmA0;
        const CUtensorMap* tmB = t.prob ? &tmB1 : &tmB0;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, args.err, GLC_DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + stage * STAGE_BYTES;
          uint8_t* sB = sA + A_BYTES;
          mbar_arrive_expect_tx(&full_bar[stage], STAGE_BYTES);
          load_operand(p.a_mn, p.a_3d, BM, sA, tmA, &full_bar[stage], t.m0, kb * BK);
          load_operand(p.b_mn, p.b_3d, BN, sB, tmB, &full_bar[stage], t.n0, kb * BK);
          in_flight = in_flight < STAGES ? in_flight + 1 : STAGES;
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Abort path: wait (bounded) for the copies this thread issued to land
        // before the CTA releases its shared memory.
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < in_flight; ++i) {
          if (--s < 0) {
            s = STAGES - 1;
            ph ^= 1;
          }
          mbar_drain(&full_bar[s], ph, args.err);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      bool issued_any = false;
      for (int tile = blockIdx.x; tile < args.total_tiles && ok; tile += gridDim.x, ++local) {
        const TileRef t = locate<BM>(args, tile);
        const Problem& p = args.p[t.prob];
        const uint32_t idesc = umma_idesc_tf32(BM, BN, p.a_mn != 0, p.b_mn != 0);
        const int buf = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1);
        if (!mbar_wait(&tempty_bar[buf], (use & 1) ^ 1, abort_flag, args.err, GLC_DEV_TIMEOUT_MMA_TMEM)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + buf * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&full_bar[stage], phase, abort_flag, args.err, GLC_DEV_TIMEOUT_MMA_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sA = smem_u32(smem + stage * STAGE_BYTES);
          const uint32_t sB = sA + A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            umma_tf32(tmem_d, operand_desc(p.a_mn, sA, kk), operand_desc(p.b_mn, sB, kk), idesc,
                      (kb > 0 || kk > 0) ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&empty_bar[stage]);  // frees the smem stage when these MMAs finish
          if (++stage == STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[buf]);  // accumulator ready for the epilogue
      }
      if (!ok && issued_any) {
        // Abort path: make sure no MMA is still writing TMEM before dealloc.
        umma_commit(drain_bar);
        mbar_drain(drain_bar, 0, args.err);
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;  // TMEM lane quarter this warp may access
    const int row_in_tile = q * 32 + lane;
    int local = 0;
    for (int tile = blockIdx.x; tile < args.total_tiles; tile += gridDim.x, ++local) {
      const TileRef t = locate<BM>(args, tile);
      const Problem& p = args.p[t.prob];
      const bool vec_ok = ((p.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
                          (p.R == nullptr || (((p.ldr & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.R) & 15) == 0)));
      const int buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      // warp-uniform outcome: the TMEM loads below are warp-collective
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull_bar[buf], use & 1, abort_flag, args.err, GLC_DEV_TIMEOUT_EPILOGUE)))
        break;
      tc_fence_after();
      const int row = t.m0 + row_in_tile;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
      double sq = 0.0;
#pragma unroll 1
      for (int chunk = 0; chunk < BN / 32; ++chunk) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + chunk * 32, r);
        tmem_ld_wait();
        if (chunk == BN / 32 - 1) {
          // all TMEM reads of this accumulator are done: hand it back
          tc_fence_before();
          mbar_arrive(&tempty_bar[buf]);
        }
        const int col0 = t.n0 + chunk * 32;
        if (row >= p.M || col0 >= p.N) continue;
        float* crow = p.C + static_cast<size_t>(row) * p.ldc + col0;
        const float* rrow = p.R ? p.R + static_cast<size_t>(row) * p.ldr + col0 : nullptr;
        if (vec_ok && col0 + 32 <= p.N) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float4 v = make_float4(__uint_as_float(r[4 * j + 0]), __uint_as_float(r[4 * j + 1]),
                                   __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
            if (p.accumulate) {
              const float4 c = reinterpret_cast<const float4*>(crow)[j];
              v.x += c.x; v.y += c.y; v.z += c.z; v.w += c.w;
            }
            if (rrow) {
              const float4 c = reinterpret_cast<const float4*>(rrow)[j];
              v.x += c.x; v.y += c.y; v.z += c.z; v.w += c.w;
            }
            if (p.round_out) {
              v.x = round_tf32(v.x); v.y = round_tf32(v.y); v.z = round_tf32(v.z); v.w = round_tf32(v.w);
            }
            if (p.sumsq) {
              sq = fma(static_cast<double>(v.x), static_cast<double>(v.x), sq);
              sq = fma(static_cast<double>(v.y), static_cast<double>(v.y), sq);
              sq = fma(static_cast<double>(v.z), static_cast<double>(v.z), sq);
              sq = fma(static_cast<double>(v.w), static_cast<double>(v.w), sq);
            }
            reinterpret_cast<float4*>(crow)[j] = v;
          }
        } else {
          const int lim = min(32, p.N - col0);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j < lim) {
              float v = __uint_as_float(r[j]);
              if (p.accumulate) v += crow[j];
              if (rrow) v += rrow[j];
              if (p.round_out) v = round_tf32(v);
              if (p.sumsq) sq = fma(static_cast<double>(v), static_cast<double>(v), sq);
              crow[j] = v;
            }
          }
        }
      }
      if (p.sumsq) {
        // 4 epilogue warps per 128x256 tile, slot = warp - 2
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        const int tid = (t.m0 / BM) * p.n_tiles + t.n0 / BN;
        if (lane == 0) p.sumsq[tid * 4 + (warp - 2)] = sq;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, TMEM_COLS);
  }
}

// ------------------------------------------------------------ CTA-pair kernel
constexpr int PAIR_BM = 256;                         // cluster tile rows (128 per CTA)
constexpr int HALF_ROWS = 128;                       // rows of A and of B each CTA loads
constexpr int P_STAGES = 6;
constexpr int P_A_BYTES = HALF_ROWS * BK * 4;        // 16 KB
constexpr int P_B_BYTES = HALF_ROWS * BK * 4;        // 16 KB
constexpr int P_STAGE_BYTES = P_A_BYTES + P_B_BYTES; // 32 KB per CTA, 64 KB per pair
constexpr int P_TILE_RING = 8;                       // dynamic order: tile indices published ahead
constexpr int P_RING_CONSUMERS = 2 + 2 * P_EPI_WARPS; // peer producer, MMA issuer, epilogue warps of both CTAs
constexpr int P_SMEM_BYTES = P_STAGES * P_STAGE_BYTES + 1024 + 512;

__device__ __forceinline__ void load_operand_pair(bool mn, bool mn3d, void* sdst, const CUtensorMap* tm,
                                                  uint32_t bar_cluster, int mn0, int k0) {
  if (mn3d) {
    tma_load_3d_pair(sdst, tm, bar_cluster, 0, k0, mn0 / 32);
  } else if (mn) {
#pragma unroll
    for (int c = 0; c < HALF_ROWS / 32; ++c)
      tma_load_2d_pair(static_cast<uint8_t*>(sdst) + c * (BK * 128), tm, bar_cluster, mn0 + 32 * c, k0);
  } else {
    tma_load_2d_pair(sdst, tm, bar_cluster, k0, mn0);
  }
}

// Barriers (same offsets in both CTAs):
//   full[s]    leader only: the leader's producer arrives with expect_tx of
//              the pair's 64 KB; both CTAs' copies complete_tx on it.  The
//              peer's copies may land before that arrival (the transaction
//              count goes negative meanwhile), never into an earlier phase:
//              the peer refills stage s only after the MMA consumed it.
//   empty[s]   both CTAs: the leader's MMA commit frees stage s in each CTA
//   tfull[b]   both CTAs: accumulator b finished (leader's commit to each)
//   tempty[b]  leader only: the 4 epilogue warps of each CTA released b
//   drain      leader only: abort path, all issued MMAs finished
__global__ void __cluster_dims__(2, 1, 1) __launch_bounds__(P_NUM_THREADS, 1)
    gemm_tf32_pair_kernel(const __grid_constant__ CUtensorMap tmA0, const __grid_constant__ CUtensorMap tmB0,
                          const __grid_constant__ CUtensorMap tmA1, const __grid_constant__ CUtensorMap tmB1,
                          const GroupArgs args) {
  GLC_PDL_ENTRY();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint64_t* full_bar = reinterpret_cast<uint64_t*>(smem + P_STAGES * P_STAGE_BYTES);
  uint64_t* empty_bar = full_bar + P_STAGES;
  uint64_t* tfull_bar = empty_bar + P_STAGES;  // [2]
  uint64_t* tempty_bar = tfull_bar + 2;        // [2]
  uint64_t* drain_bar = tempty_bar + 2;        // [1]
  uint64_t* ring_full = drain_bar + 1;         // [P_TILE_RING] each CTA: tile index published
  uint64_t* ring_empty = ring_full + P_TILE_RING;  // [P_TILE_RING] leader: every consumer read it
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(ring_empty + P_TILE_RING);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);
  int* ring = reinterpret_cast<int*>(tmem_slot + 2);  // [P_TILE_RING]

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const int cluster = static_cast<int>(blockIdx.x >> 1);
  const int nclusters = static_cast<int>(gridDim.x >> 1);
  // Dynamic order: the leader's producer takes tile indices from the counter
  // and publishes each in slot i % P_TILE_RING of both CTAs' rings; every
  // other role of the pair reads the slots in order and releases them on the
  // leader's ring_empty.  A -1 ends the sequence; -2 means a wait gave up.
  auto consume = [&](int i, bool warp_wide) -> int {
    const int slot = i % P_TILE_RING;
    const uint32_t ph = static_cast<uint32_t>(i / P_TILE_RING) & 1u;
    const bool got = mbar_wait_cluster(&ring_full[slot], ph, abort_flag, args.err, GLC_DEV_TIMEOUT_MMA_FULL);
    if (warp_wide ? !__all_sync(0xffffffffu, got) : !got) return -2;
    const int t = ring[slot];
    if (warp_wide) __syncwarp();
    if (!warp_wide || lane == 0) mbar_arrive_cluster(mapa_cluster(&ring_empty[slot], 0));
    return t;
  };

  if (threadIdx.x == 0) {
    for (int s = 0; s < P_STAGES; ++s) {
      mbar_init(&full_bar[s], 1);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 2 * P_EPI_WARPS);
    }
    mbar_init(drain_bar, 1);
    for (int i = 0; i < P_TILE_RING; ++i) {
      mbar_init(&ring_full[i], 1);
      mbar_init(&ring_empty[i], P_RING_CONSUMERS);
    }
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA0);
    tma_prefetch_desc(&tmB0);
    if (args.nprob > 1) {
      tma_prefetch_desc(&tmA1);
      tma_prefetch_desc(&tmB1);
    }
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, TMEM_COLS);
  tc_fence_before();
  // both CTAs' barriers exist before either CTA arrives on the other's
  cluster_sync_all();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ producers (both CTAs)
    if (lane == 0) {
      const uint32_t full_leader = mapa_cluster(full_bar, 0);
      int stage = 0;
      uint32_t phase = 0;
      bool ok = true;
      int it0, it1, istep;
      sched_range(args, cluster, nclusters, it0, it1, istep);
      for (int it = it0, i = 0; ok; it += istep, ++i) {
        int tile;
        if (!args.dyn) {
          if (it >= it1) break;
          tile = sched_tile(args, nclusters, it);
        } else if (rank == 0) {
          // the pair's scheduler: take the next index, publish it to both CTAs
          const int slot = i % P_TILE_RING;
          if (!mbar_wait(&ring_empty[slot], (static_cast<uint32_t>(i / P_TILE_RING) & 1u) ^ 1u, abort_flag, args.err,
                         GLC_DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          tile = atomicAdd(args.dyn, 1);
          if (tile >= args.total_tiles) tile = -1;
          ring[slot] = tile;
          st_shared_cluster_u32(mapa_cluster(&ring[slot], 1), tile);
          mbar_arrive(&ring_full[slot]);
          mbar_arrive_cluster(mapa_cluster(&ring_full[slot], 1));
        } else {
          tile = consume(i, false);
          if (tile == -2) {
            ok = false;
            break;
          }
        }
        if (tile < 0) break;
        const TileRef t = locate<PAIR_BM>(args, tile);
        const Problem& p = args.p[t.prob];
        const CUtensorMap* tmA = t.prob ? &tmA1 : &tmA0;
        const CUtensorMap* tmB = t.prob ? &tmB1 : &tmB0;
        const int a_row = t.m0 + static_cast<int>(rank) * HALF_ROWS;
        const int b_row = p.glu ? (rank ? p.glu + t.n0 : t.n0) : t.n0 + static_cast<int>(rank) * HALF_ROWS;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, args.err, GLC_DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          uint8_t* sA = smem + stage * P_STAGE_BYTES;
          uint8_t* sB = sA + P_A_BYTES;
          const uint32_t fb = full_leader + stage * 8;
          if (rank == 0) mbar_arrive_expect_tx(&full_bar[stage], 2 * P_STAGE_BYTES);
          load_operand_pair(p.a_mn, p.a_3d, sA, tmA, fb, a_row, kb * BK);
          load_operand_pair(p.b_mn, p.b_3d, sB, tmB, fb, b_row, kb * BK);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      // Copies signal the leader's barriers; on abort the leader waits for
      // the stages in flight before the pair leaves (see the MMA issuer).
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer (leader)
    if (rank == 0) {  // the leader's whole warp; elect.sync issues
      const uint32_t empty_own = mapa_cluster(empty_bar, 0), empty_peer = mapa_cluster(empty_bar, 1);
      const uint32_t tfull_own = mapa_cluster(tfull_bar, 0), tfull_peer = mapa_cluster(tfull_bar, 1);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      bool issued_any = false;
      int it0, it1, istep;
      sched_range(args, cluster, nclusters, it0, it1, istep);
      for (int it = it0; ok; it += istep, ++local) {
        int tile;
        if (!args.dyn) {
          if (it >= it1) break;
          tile = sched_tile(args, nclusters, it);
        } else {
          tile = consume(local, true);
          if (tile == -2) {
            ok = false;
            break;
          }
        }
        if (tile < 0) break;
        const TileRef t = locate<PAIR_BM>(args, tile);
        const Problem& p = args.p[t.prob];
        const uint32_t idesc = umma_idesc_tf32(PAIR_BM, BN, p.a_mn != 0, p.b_mn != 0);
        const int buf = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1);
        if (!mbar_wait_warp(&tempty_bar[buf], (use & 1) ^ 1, abort_flag, args.err, GLC_DEV_TIMEOUT_MMA_TMEM)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + buf * BN;
        for (int kb = 0; kb < p.k_blocks; ++kb) {
          if (!mbar_wait_warp(&full_bar[stage], phase, abort_flag, args.err, GLC_DEV_TIMEOUT_MMA_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sA = smem_u32(smem + stage * P_STAGE_BYTES);
          const uint32_t sB = sA + P_A_BYTES;
#pragma unroll
          for (int kk = 0; kk < BK / UMMA_K; ++kk) {
            umma_tf32_pair_warp(tmem_d, operand_desc(p.a_mn, sA, kk), operand_desc(p.b_mn, sB, kk), idesc,
                           (kb > 0 || kk > 0) ? 1u : 0u);
          }
          issued_any = true;
          // stage s is free in both CTAs once these MMAs have read it
          umma_commit_pair_warp(empty_own + stage * 8);
          umma_commit_pair_warp(empty_peer + stage * 8);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit_pair_warp(tfull_own + buf * 8);
        umma_commit_pair_warp(tfull_peer + buf * 8);
      }
      if (!ok) {
        // Abort path.  (1) No MMA may still read shared memory or write TMEM
        // of either CTA when the pair leaves.  (2) Copies the producers issued
        // for stages not yet consumed signal this CTA's full barriers: wait
        // for them (each wait bounded) so none lands after exit.
        if (issued_any) {
          umma_commit_pair_warp(mapa_cluster(drain_bar, 0));
          mbar_drain(drain_bar, 0, args.err);
        }
        for (int i = 0; i < P_STAGES; ++i) {
          mbar_drain(&full_bar[stage], phase, args.err);
          if (++stage == P_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ epilogue (both CTAs)
    const int q = warp & 3;
    const int ch = (warp - 2) >> 2;  // share of the accumulator's columns this warp drains
    const int row_in_half = q * 32 + lane;
    const uint32_t tempty_leader = mapa_cluster(tempty_bar, 0);
    int local = 0;
    int it0, it1, istep;
    sched_range(args, cluster, nclusters, it0, it1, istep);
    for (int it = it0;; it += istep, ++local) {
      int tile;
      if (!args.dyn) {
        if (it >= it1) break;
        tile = sched_tile(args, nclusters, it);
      } else {
        tile = consume(local, true);
      }
      if (tile < 0) break;
      const TileRef t = locate<PAIR_BM>(args, tile);
      const Problem& p = args.p[t.prob];
      const bool vec_ok = ((p.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.C) & 15) == 0) &&
                          (p.R == nullptr || (((p.ldr & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.R) & 15) == 0)));
      const int buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull_bar[buf], use & 1, abort_flag, args.err, GLC_DEV_TIMEOUT_EPILOGUE)))
        break;
      tc_fence_after();
      const int row = t.m0 + static_cast<int>(rank) * HALF_ROWS + row_in_half;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * BN;
      if (p.glu) {
        // gate in accumulator columns 0..127, up in 128..255, same outputs
        const int F = p.glu;
        const bool hvec = vec_ok && ((p.ldh & 3) == 0) && ((reinterpret_cast<uintptr_t>(p.h) & 15) == 0) &&
                          ((F & 3) == 0);
#pragma unroll 1
        for (int chunk = ch * (4 / P_SPLIT); chunk < (ch + 1) * (4 / P_SPLIT); ++chunk) {
          uint32_t g[32], u[32];
          tmem_ld_32x32b_x32(taddr + chunk * 32, g);
          tmem_ld_32x32b_x32(taddr + 128 + chunk * 32, u);
          tmem_ld_wait();
          if (chunk == (ch + 1) * (4 / P_SPLIT) - 1) {
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_cluster(tempty_leader + buf * 8);
          }
          const int col0 = t.n0 + chunk * 32;
          if (row >= p.M || col0 >= F) continue;
          float* grow = p.C + static_cast<size_t>(row) * p.ldc + col0;
          float* urow = grow + F;
          float* hrow = p.h + static_cast<size_t>(row) * p.ldh + col0;
          if (hvec && col0 + 32 <= F) {
#pragma unroll
            for (int j = 0; j < 8; ++j) {
              const float4 gv = make_float4(__uint_as_float(g[4 * j]), __uint_as_float(g[4 * j + 1]),
                                            __uint_as_float(g[4 * j + 2]), __uint_as_float(g[4 * j + 3]));
              const float4 uv = make_float4(__uint_as_float(u[4 * j]), __uint_as_float(u[4 * j + 1]),
                                            __uint_as_float(u[4 * j + 2]), __uint_as_float(u[4 * j + 3]));
              float4 hv = p.glu_fast ? make_float4(swiglu_f<true>(gv.x, uv.x), swiglu_f<true>(gv.y, uv.y),
                                                   swiglu_f<true>(gv.z, uv.z), swiglu_f<true>(gv.w, uv.w))
                                     : make_float4(go_swiglu(gv.x, uv.x), go_swiglu(gv.y, uv.y),
                                                   go_swiglu(gv.z, uv.z), go_swiglu(gv.w, uv.w));
              if (p.round_h) hv = make_float4(round_tf32(hv.x), round_tf32(hv.y), round_tf32(hv.z), round_tf32(hv.w));
              reinterpret_cast<float4*>(grow)[j] = gv;
              reinterpret_cast<float4*>(urow)[j] = uv;
              reinterpret_cast<float4*>(hrow)[j] = hv;
            }
          } else {
            const int lim = min(32, F - col0);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
              if (j < lim) {
                const float gv = __uint_as_float(g[j]), uv = __uint_as_float(u[j]);
                float hv = p.glu_fast ? swiglu_f<true>(gv, uv) : go_swiglu(gv, uv);
                if (p.round_h) hv = round_tf32(hv);
                grow[j] = gv;
                urow[j] = uv;
                hrow[j] = hv;
              }
            }
          }
        }
        continue;
      }
      double sq = 0.0;
#pragma unroll 1
      for (int chunk = ch * (BN / 32 / P_SPLIT); chunk < (ch + 1) * (BN / 32 / P_SPLIT); ++chunk) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + chunk * 32, r);
        tmem_ld_wait();
        if (chunk == (ch + 1) * (BN / 32 / P_SPLIT) - 1) {
          // this warp's reads of accumulator buf are done: one arrival per warp
          tc_fence_before();
          __syncwarp();
          if (lane == 0) mbar_arrive_cluster(tempty_leader + buf * 8);
        }
        const int col0 = t.n0 + chunk * 32;
        if (row >= p.M || col0 >= p.N) continue;
        float* crow = p.C + static_cast<size_t>(row) * p.ldc + col0;
        const float* rrow = p.R ? p.R + static_cast<size_t>(row) * p.ldr + col0 : nullptr;
        if (vec_ok && col0 + 32 <= p.N) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float4 v = make_float4(__uint_as_float(r[4 * j + 0]), __uint_as_float(r[4 * j + 1]),
                                   __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
            if (p.accumulate) {
              const float4 c = reinterpret_cast<const float4*>(crow)[j];
              v.x += c.x; v.y += c.y; v.z += c.z; v.w += c.w;
            }
            if (rrow) {
              const float4 c = reinterpret_cast<const float4*>(rrow)[j];
              v.x += c.x; v.y += c.y; v.z += c.z; v.w += c.w;
            }
            if (p.round_out) {
              v.x = round_tf32(v.x); v.y = round_tf32(v.y); v.z = round_tf32(v.z); v.w = round_tf32(v.w);
            }
            if (p.sumsq) {
              sq = fma(static_cast<double>(v.x), static_cast<double>(v.x), sq);
              sq = fma(static_cast<double>(v.y), static_cast<double>(v.y), sq);
              sq = fma(static_cast<double>(v.z), static_cast<double>(v.z), sq);
              sq = fma(static_cast<double>(v.w), static_cast<double>(v.w), sq);
            }
            reinterpret_cast<float4*>(crow)[j] = v;
          }
        } else {
          const int lim = min(32, p.N - col0);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j < lim) {
              float v = __uint_as_float(r[j]);
              if (p.accumulate) v += crow[j];
              if (rrow) v += rrow[j];
              if (p.round_out) v = round_tf32(v);
              if (p.sumsq) sq = fma(static_cast<double>(v), static_cast<double>(v), sq);
              crow[j] = v;
            }
          }
        }
      }
      if (p.sumsq) {
        // 2 * P_EPI_WARPS epilogue warps per 256x256 tile, slot = rank * P_EPI_WARPS + warp - 2
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        const int tid = (t.m0 / PAIR_BM) * p.n_tiles + t.n0 / BN;
        if (lane == 0) p.sumsq[tid * (2 * P_EPI_WARPS) + static_cast<int>(rank) * P_EPI_WARPS + (warp - 2)] = sq;
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  // neither CTA leaves (or frees TMEM) while the other may still touch its
  // shared memory, barriers or TMEM
  cluster_sync_all();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem_base, TMEM_COLS);
  }
}

// ---------------------------------------------------------------- host side

// Global tensor: a K-major operand is [rows_mn][k] with row stride ld; an
// MN-major one [k][rows_mn].  An MN-major operand whose MN extent is a
// multiple of 32 is described in three dimensions, {32, k, rows_mn/32} with
// strides {ld, 32} elements, so one box brings all of a tile's 32-element
// chunks; otherwise 2-D boxes of 32 MN-elements (the partial chunk is
// zero-filled).  *three_d reports which.
int encode_operand(Context* ctx, CUtensorMap* tm, const float* ptr, int ld, bool mn, int rows_mn, int k, int box_mn,
                   int* three_d) {
  cuuint32_t estr[3] = {1, 1, 1};
  *three_d = 0;
  if (mn && rows_mn % 32 == 0 && box_mn % 32 == 0) {
    cuuint64_t dims[3] = {32, static_cast<cuuint64_t>(k), static_cast<cuuint64_t>(rows_mn / 32)};
    cuuint64_t strides[2] = {static_cast<cuuint64_t>(ld) * 4, 128};
    cuuint32_t box[3] = {32, BK, static_cast<cuuint32_t>(box_mn / 32)};
    *three_d = 1;
    return ctx->encode_tiled(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 3, const_cast<float*>(ptr), dims, strides, box,
                             estr, CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
  }
  cuuint64_t dims[2];
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ld) * 4};
  cuuint32_t box[2];
  if (mn) {
    dims[0] = static_cast<cuuint64_t>(rows_mn);
    dims[1] = static_cast<cuuint64_t>(k);
    box[0] = 32;
    box[1] = BK;
  } else {
    dims[0] = static_cast<cuuint64_t>(k);
    dims[1] = static_cast<cuuint64_t>(rows_mn);
    box[0] = BK;
    box[1] = static_cast<cuuint32_t>(box_mn);
  }
  return ctx->encode_tiled(tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(ptr), dims, strides, box,
                           estr, mn ? CU_TENSOR_MAP_SWIZZLE_128B_ATOM_32B : CU_TENSOR_MAP_SWIZZLE_128B,
                           CU_TENSOR_MAP_L2_PROMOTION_L2_256B);
}

// tile_m: rows of C per tile (BM, or PAIR_BM for the CTA pair); box_a/box_b:
// rows of A/B one CTA loads per k-block.
int prepare(Context* ctx, const GemmSpec& g, Problem* p, CUtensorMap* ta, CUtensorMap* tb, int tile_m, int box_a,
            int box_b) {
  if (g.M < 0 || g.N < 0 || g.K <= 0) return ctx->fail(GLC_ERR_INVALID, "gemm: bad size");
  if (!g.A.ptr || !g.B.ptr || !g.C) return ctx->fail(GLC_ERR_INVALID, "gemm: null pointer");
  if ((g.A.ld & 3) || (g.B.ld & 3) || (reinterpret_cast<uintptr_t>(g.A.ptr) & 15) ||
      (reinterpret_cast<uintptr_t>(g.B.ptr) & 15))
    return ctx->fail(GLC_ERR_INVALID, "gemm: operand leading dimensions must be multiples of 4 floats and 16-byte aligned");
  if (encode_operand(ctx, ta, g.A.ptr, g.A.ld, g.A.mn_major, g.M, g.K, box_a, &p->a_3d) != 0)
    return ctx->fail(GLC_ERR_INVALID, "gemm: cuTensorMapEncodeTiled failed for A");
  if (encode_operand(ctx, tb, g.B.ptr, g.B.ld, g.B.mn_major, g.N, g.K, box_b, &p->b_3d) != 0)
    return ctx->fail(GLC_ERR_INVALID, "gemm: cuTensorMapEncodeTiled failed for B");
  p->C = g.C;
  p->R = g.R;
  p->M = g.M;
  p->N = g.N;
  p->K = g.K;
  p->ldc = g.ldc;
  p->ldr = g.ldr;
  p->accumulate = g.accumulate ? 1 : 0;
  p->round_out = g.round_out ? 1 : 0;
  p->sumsq = g.sumsq;
  p->a_mn = g.A.mn_major ? 1 : 0;
  p->b_mn = g.B.mn_major ? 1 : 0;
  p->m_tiles = (g.M + tile_m - 1) / tile_m;
  p->n_tiles = (g.N + BN - 1) / BN;
  p->k_blocks = (g.K + BK - 1) / BK;
  p->tiles = p->m_tiles * p->n_tiles;
  p->n_fast = static_cast<double>(g.M) > static_cast<double>(g.N) ? 1 : 0;  // A (M x K) larger than B (N x K)
  p->glu = g.glu;
  p->h = g.glu_h;
  p->ldh = g.ld_glu;
  p->round_h = g.glu_round ? 1 : 0;
  p->glu_fast = g.glu_fast ? 1 : 0;
  if (g.glu) p->n_tiles = (g.glu + 127) / 128;
  p->tiles = p->m_tiles * p->n_tiles;
  if (g.sumsq) {
    const long long per_tile = tile_m == PAIR_BM ? 2 * P_EPI_WARPS : 4;
    if (g.glu || static_cast<long long>(p->tiles) * per_tile > g.sumsq_cap)
      return ctx->fail(GLC_ERR_INVALID, "gemm: sum-of-squares slots too few, or with the SwiGLU epilogue");
  }
  return 0;
}

// Tile lists for a grouped CTA-pair launch.  The two problems' tiles cost
// different times (their k-block counts differ: dX and dW of one layer), so
// the fixed rotation tile = cluster + i * clusters can leave some clusters a
// long tile more than others.  Here tiles are handed out in index order to
// the cluster that frees first, with a tile's time estimated as its k-blocks
// plus 2 (pipeline turn-around): the order a dynamic queue would produce,
// fixed on the host so every role of both CTAs walks the same list.  Cached
// per shape on the device; nullptr (the rotation) when the estimate is not
// at least 1 % shorter than the rotation's (the rotation keeps concurrent
// tiles adjacent) or if memory is short.
const int* pair_schedule(Context* ctx, const GroupArgs& a, int clusters) {
  const std::array<long long, 5> key{a.p[0].tiles, a.p[0].k_blocks, a.p[1].tiles, a.p[1].k_blocks, clusters};
  for (auto& e : ctx->gemm_sched)
    if (e.first == key) return e.second;
  std::vector<int> h;
  if (!gemm_tile_lists(a.p[0].tiles, a.p[0].k_blocks, a.p[1].tiles, a.p[1].k_blocks, clusters, &h)) {
    ctx->gemm_sched.push_back({key, nullptr});
    return nullptr;
  }
  int* d = nullptr;
  if (cudaMalloc(&d, h.size() * sizeof(int)) != cudaSuccess) {
    cudaGetLastError();
    return nullptr;
  }
  if (cudaMemcpy(d, h.data(), h.size() * sizeof(int), cudaMemcpyHostToDevice) != cudaSuccess) {
    cudaFree(d);
    cudaGetLastError();
    return nullptr;
  }
  ctx->gemm_sched.push_back({key, d});
  return d;
}

}  // namespace

bool gemm_tile_lists(int tiles0, int kb0, int tiles1, int kb1, int clusters, std::vector<int>* out) {
  const int total = tiles0 + tiles1;
  if (clusters <= 0 || total <= 0) return false;
  std::vector<std::vector<int>> lists(clusters);
  using Slot = std::pair<long long, int>;  // (estimated finish, cluster): ties go to the lower cluster
  std::priority_queue<Slot, std::vector<Slot>, std::greater<Slot>> q;
  for (int c = 0; c < clusters; ++c) q.push({0, c});
  std::vector<long long> rot(clusters, 0);
  long long greedy_end = 0;
  for (int t = 0; t < total; ++t) {
    const Slot s = q.top();
    q.pop();
    lists[s.second].push_back(t);
    const int kb = t < tiles0 ? kb0 : kb1;
    q.push({s.first + kb + 2, s.second});
    greedy_end = std::max(greedy_end, s.first + kb + 2);
    rot[t % clusters] += kb + 2;
  }
  if (100 * greedy_end > 99 * *std::max_element(rot.begin(), rot.end())) return false;
  out->assign(static_cast<size_t>(clusters) + 1 + total, 0);
  int pos = 0;
  for (int c = 0; c < clusters; ++c) {
    (*out)[c] = pos;
    for (int t : lists[c]) (*out)[clusters + 1 + pos++] = t;
  }
  (*out)[clusters] = pos;
  return true;
}

long long gemm_sumsq_slots(long long M, long long N) {
  static_assert(2 * P_EPI_WARPS <= 8, "pair tiles: at most 8 slots per 256-row tile");
  return ((M + BM - 1) / BM) * ((N + BN - 1) / BN) * 8;
}

int gemm_tf32_group(Context* ctx, const GemmSpec* specs, int n, cudaStream_t stream) {
  if (n < 1 || n > 2) return ctx->fail(GLC_ERR_INVALID, "gemm: 1 or 2 problems per launch");
  // empty problems are finished here; K == 0 needs no tensor core
  GemmSpec live[2];
  int nl = 0;
  for (int i = 0; i < n; ++i) {
    const GemmSpec& g = specs[i];
    if (g.M < 0 || g.N < 0 || g.K < 0) return ctx->fail(GLC_ERR_INVALID, "gemm: negative size");
    if (g.M == 0 || g.N == 0) continue;
    if (!g.C) return ctx->fail(GLC_ERR_INVALID, "gemm: null pointer");
    if (g.K == 0) {
      int rc = gemm_empty_k(ctx, g.C, g.ldc, g.M, g.N, g.accumulate, g.R, g.ldr, stream);
      if (rc) return rc;
      continue;
    }
    live[nl++] = g;
  }
  if (nl == 0) return 0;
  // longer reductions first: their tiles take longest, so they start first
  if (nl == 2 && live[1].K > live[0].K) std::swap(live[0], live[1]);
  // CTA pairs unless a problem has at most 128 rows (a pair tile would be
  // half empty) or the context pins a variant.
  bool pair = true;
  for (int i = 0; i < nl; ++i) pair = pair && live[i].M > BM;
  if (ctx->gemm_variant == 1) pair = false;
  if (ctx->gemm_variant == 2) pair = true;
  bool any_glu = false;
  for (int i = 0; i < nl; ++i) {
    const GemmSpec& g = live[i];
    if (!g.glu) continue;
    any_glu = true;
    if (g.N != 2 * g.glu || g.accumulate || g.R || !g.glu_h || g.ld_glu < g.glu)
      return ctx->fail(GLC_ERR_INVALID, "gemm: SwiGLU epilogue needs N = 2F, no accumulate or residual, an output h");
  }
  if (any_glu && !pair) {
    // the fused epilogue exists on CTA pairs only: GEMM, then the SwiGLU kernel
    GemmSpec plain[2];
    for (int i = 0; i < nl; ++i) {
      plain[i] = live[i];
      plain[i].glu = 0;
    }
    int rc = gemm_tf32_group(ctx, plain, nl, stream);
    for (int i = 0; i < nl && !rc; ++i) {
      const GemmSpec& g = live[i];
      if (g.glu)
        rc = swiglu_fwd(ctx, g.C, g.C + g.glu, static_cast<size_t>(g.ldc), g.glu_h, static_cast<size_t>(g.ld_glu),
                        static_cast<size_t>(g.M), static_cast<size_t>(g.glu), g.glu_round, stream, g.glu_fast);
    }
    return rc;
  }
  GroupArgs a{};
  CUtensorMap tm[4];
  for (int i = 0; i < nl; ++i) {
    int rc = pair ? prepare(ctx, live[i], &a.p[i], &tm[2 * i], &tm[2 * i + 1], PAIR_BM, HALF_ROWS, HALF_ROWS)
                  : prepare(ctx, live[i], &a.p[i], &tm[2 * i], &tm[2 * i + 1], BM, BM, BN);
    if (rc) return rc;
  }
  if (nl == 1) {
    tm[2] = tm[0];
    tm[3] = tm[1];
    a.p[1] = a.p[0];
    a.p[1].tiles = 0;
  }
  a.nprob = nl;
  a.total_tiles = a.p[0].tiles + (nl > 1 ? a.p[1].tiles : 0);
  a.err = ctx->d_err;
  // the shared-memory limit is a per-device attribute of each kernel: set
  // once per device (atomic flags; a repeated setting from a racing host
  // thread is harmless)
  constexpr int kMaxDevices = 64;
  static std::atomic<bool> attr_set[2][kMaxDevices];
  if (ctx->device < 0 || ctx->device >= kMaxDevices) return ctx->fail(GLC_ERR_UNSUPPORTED, "gemm: device index too large");
  if (!attr_set[pair][ctx->device].load(std::memory_order_acquire)) {
    cudaError_t e = pair ? cudaFuncSetAttribute(gemm_tf32_pair_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                P_SMEM_BYTES)
                         : cudaFuncSetAttribute(gemm_tf32_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                                SMEM_BYTES);
    if (e != cudaSuccess) return ctx->fail_cuda(e, "cudaFuncSetAttribute(gemm_tf32)");
    attr_set[pair][ctx->device].store(true, std::memory_order_release);
  }
  double flops = 0;
  for (int i = 0; i < nl; ++i) flops += 2.0 * a.p[i].M * a.p[i].N * static_cast<double>(a.p[i].K);
  ProfScope prof(ctx, PROF_GEMM, flops, stream);
  if (pair) {
    // one cluster per SM pair; clusters loop over the tiles
    const int pairs = ctx->num_sms / 2;
    const int clusters = a.total_tiles < pairs ? a.total_tiles : pairs;
    // automatic: the dynamic order under data parallelism, where the
    // gradient allreduce holds SMs during the backward (2 GPUs, dynamic vs
    // fixed: 87.2 vs 90.2 ms per step), the fixed order on one GPU
    if (ctx->gemm_order == 2 || (ctx->gemm_order == 0 && ctx->world > 1)) {
      // dynamic order: a fresh zero counter per launch from the context's
      // ring of counters, cleared on the stream whenever the ring wraps
      const unsigned idx = static_cast<unsigned>(ctx->dyn_next++ % Context::kDynCounters);
      if (idx == 0 && ctx->dyn_next > 1) {
        cudaError_t e = cudaMemsetAsync(ctx->dyn_ctr, 0, sizeof(int) * Context::kDynCounters, stream);
        if (e != cudaSuccess) return ctx->fail_cuda(e, "gemm: clearing the tile counters");
      }
      a.dyn = ctx->dyn_ctr + idx;
    } else if (nl == 2) {
      a.sched = pair_schedule(ctx, a, clusters);
    }
    glc::launch_pdl(ctx, gemm_tf32_pair_kernel, 2 * clusters, P_NUM_THREADS, P_SMEM_BYTES, stream, tm[0], tm[1], tm[2], tm[3], a);
  } else {
    const int grid = a.total_tiles < ctx->num_sms ? a.total_tiles : ctx->num_sms;
    glc::launch_pdl(ctx, gemm_tf32_kernel, grid, NUM_THREADS, SMEM_BYTES, stream, tm[0], tm[1], tm[2], tm[3], a);
  }
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return ctx->fail_cuda(e, "launch gemm_tf32");
  ctx->count_launch();
  return 0;
}

int gemm_tf32(Context* ctx, const GemmOperand& A, const GemmOperand& B, float* C, int ldc, int M, int N, int K,
              bool accumulate, const float* R, int ldr, bool round_out, cudaStream_t stream) {
  GemmSpec g{A, B, C, ldc, M, N, K, accumulate, R, ldr, round_out};
  return gemm_tf32_group(ctx, &g, 1, stream);
}

}  // namespace glc
