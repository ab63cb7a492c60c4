// dX (+)= dY . deq(W) with the dequantization inside the GEMM's operand load.
//
// W [Nout][Kin] is a frozen weight stored in a GGUF format (F16 or a block
// format of pkg/quant/dequant.go) as consecutive rows of Kin elements.  In
// the GEMM C[M, Kin] = dY[M, Nout] . W the weight is the MN-major B operand
// (B(kin, nout) = W[nout][kin]): a k-block of the tile holds 32 reduction
// rows (nout) of 256 output columns (kin), stored as eight 4 KB chunks of 32
// columns, one 128-byte row per reduction index, the 32-byte atoms of a row
// XOR-ed with (row % 4) (the UMMA layout SW128_BASE32B that TMA writes with
// SWIZZLE_128B_ATOM_32B).  One chunk row is exactly one 32-element block of
// the 32-block formats, and a tile's 256 columns of one row are exactly one
// K-format super-block, so no block straddles a tile.
//
// Instead of a TMA load of an fp32 copy, eight producer warps read the
// stored blocks (0.56 to 2 bytes per element), decode them with the
// reference's arithmetic (quant_formats.cuh, bit-exact), round to TF32 and
// store the values into the swizzled tile; the tensor core reads them as
// usual.  No dequantized copy of W exists in global memory, and each CTA
// streams ~25 KB per k-block (16 KB of dY, the rest quantized W) instead of
// 48 KB, so the single-CTA 128x256 tile (cta_group::1) needs no CTA pair.
//
// One persistent CTA per SM, 448 threads:
//   warp 0       TMA producer of dY tiles (one thread)
//   warp 1       TMEM allocator + MMA issuer (one thread)
//   warps 2..5   epilogue: TMEM -> registers -> global
//   warps 6..13  W producers: warps 6+2s and 7+2s fill ring slot s, each
//                half of its 32 reduction rows
// Every wait is bounded (mbar_wait); on a timeout every role leaves its loop,
// the TMA thread drains its copies, the MMA thread its MMAs, and TMEM is
// freed before the CTA exits.
#include "glc_internal.h"
#include "quant_formats.cuh"
#include "sm100.cuh"

namespace glc {
namespace {

constexpr int QF_BM = 128;
constexpr int QF_BN = 256;
constexpr int QF_BK = 32;
constexpr int QF_UMMA_K = 8;
constexpr int QF_STAGES = 4;
constexpr int QF_A_BYTES = QF_BM * QF_BK * 4;            // 16 KB
constexpr int QF_B_BYTES = QF_BN * QF_BK * 4;            // 32 KB
constexpr int QF_STAGE_BYTES = QF_A_BYTES + QF_B_BYTES;  // 48 KB
constexpr int QF_TMEM_COLS = 2 * QF_BN;
constexpr int QF_PRODUCER_WARPS = 2 * QF_STAGES;
constexpr int QF_THREADS = 32 * (6 + QF_PRODUCER_WARPS);
constexpr int QF_SMEM_BYTES = QF_STAGES * QF_STAGE_BYTES + 1024 /*align slack*/ + 256 /*barriers: 17 x 8 B + 8*/;
constexpr int QF_BATCH = 8;  // items a producer lane decodes between stores (loads in flight)

struct QuantGemmArgs {
  const uint8_t* w;  // stored W
  int type;
  float* C;
  int ldc;
  int M, Kin, Nout;
  int accumulate;
  int m_tiles, n_tiles, k_blocks, tiles;
  int* err;
};

// Byte offset of element (kin within the tile, k-row r) in the MN-major B
// tile: chunk kin/32 (4 KB apart), row r (128 B), 32-byte atom ((kin/8) % 4)
// XOR (r % 4), then (kin % 8) * 4.  For the float4 of elements 4j..4j+3 of a
// chunk: atom j/2, 16-byte half j%2.
__device__ __forceinline__ uint32_t b_tile_offset(int chunk, int r, int j) {
  return static_cast<uint32_t>(chunk) * 4096u + static_cast<uint32_t>(r) * 128u +
         ((static_cast<uint32_t>(j >> 1) ^ (static_cast<uint32_t>(r) & 3u)) << 5) + static_cast<uint32_t>(j & 1) * 16u;
}

__global__ void __launch_bounds__(QF_THREADS, 1)
    gemm_quant_fused_kernel(const __grid_constant__ CUtensorMap tmA, const QuantGemmArgs args) {
  GLC_PDL_ENTRY();
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  // afull[s]: the dY copy of stage s landed (TMA complete_tx); bfull[s]: the
  // slot's two producer warps stored their W halves; empty[s]: the MMAs that
  // read stage s finished (tcgen05.commit)
  uint64_t* afull_bar = reinterpret_cast<uint64_t*>(smem + QF_STAGES * QF_STAGE_BYTES);
  uint64_t* bfull_bar = afull_bar + QF_STAGES;
  uint64_t* empty_bar = bfull_bar + QF_STAGES;
  uint64_t* tfull_bar = empty_bar + QF_STAGES;  // [2]
  uint64_t* tempty_bar = tfull_bar + 2;         // [2]
  uint64_t* drain_bar = tempty_bar + 2;         // [1]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain_bar + 1);
  volatile int* abort_flag = reinterpret_cast<volatile int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < QF_STAGES; ++s) {
      mbar_init(&afull_bar[s], 1);
      mbar_init(&bfull_bar[s], 2);
      mbar_init(&empty_bar[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&tfull_bar[b], 1);
      mbar_init(&tempty_bar[b], 4 * 32);
    }
    mbar_init(drain_bar, 1);
    *abort_flag = 0;
    fence_mbar_init();
    tma_prefetch_desc(&tmA);
  }
  if (warp == 1) tmem_alloc(tmem_slot, QF_TMEM_COLS);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem_base = *tmem_slot;

  if (warp == 0) {
    // ------------------------------------------------------------ dY tiles
    if (lane == 0) {
      int stage = 0;
      uint32_t phase = 0;
      int in_flight = 0;
      bool ok = true;
      for (int tile = blockIdx.x; tile < args.tiles && ok; tile += gridDim.x) {
        const int m0 = (tile / args.n_tiles) * QF_BM;
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait(&empty_bar[stage], phase ^ 1, abort_flag, args.err, GLC_DEV_TIMEOUT_PRODUCER)) {
            ok = false;
            break;
          }
          mbar_arrive_expect_tx(&afull_bar[stage], QF_A_BYTES);
          tma_load_2d(smem + stage * QF_STAGE_BYTES, &tmA, &afull_bar[stage], kb * QF_BK, m0);
          in_flight = in_flight < QF_STAGES ? in_flight + 1 : QF_STAGES;
          if (++stage == QF_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
      }
      if (!ok) {
        // Abort path: wait (bounded) for this thread's copies before the CTA
        // releases its shared memory.
        int s = stage;
        uint32_t ph = phase;
        for (int i = 0; i < in_flight; ++i) {
          if (--s < 0) {
            s = QF_STAGES - 1;
            ph ^= 1;
          }
          mbar_drain(&afull_bar[s], ph, args.err);
        }
      }
    }
  } else if (warp == 1) {
    // ------------------------------------------------------------ MMA issuer
    if (lane == 0) {
      const uint32_t idesc = umma_idesc_tf32(QF_BM, QF_BN, false, true);
      int stage = 0;
      uint32_t phase = 0;
      int local = 0;
      bool ok = true;
      bool issued_any = false;
      for (int tile = blockIdx.x; tile < args.tiles && ok; tile += gridDim.x, ++local) {
        const int buf = local & 1;
        const uint32_t use = static_cast<uint32_t>(local >> 1);
        if (!mbar_wait(&tempty_bar[buf], (use & 1) ^ 1, abort_flag, args.err, GLC_DEV_TIMEOUT_MMA_TMEM)) {
          ok = false;
          break;
        }
        tc_fence_after();
        const uint32_t tmem_d = tmem_base + buf * QF_BN;
        for (int kb = 0; kb < args.k_blocks; ++kb) {
          if (!mbar_wait(&afull_bar[stage], phase, abort_flag, args.err, GLC_DEV_TIMEOUT_MMA_FULL) ||
              !mbar_wait(&bfull_bar[stage], phase, abort_flag, args.err, GLC_DEV_TIMEOUT_MMA_FULL)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint32_t sA = smem_u32(smem + stage * QF_STAGE_BYTES);
          const uint32_t sB = sA + QF_A_BYTES;
#pragma unroll
          for (int kk = 0; kk < QF_BK / QF_UMMA_K; ++kk) {
            // A: K-major, 128-byte rows, 8-row groups 1 KB apart; B: MN-major
            // chunks 4 KB apart (LBO), 4-row groups 512 B apart (SBO)
            umma_tf32(tmem_d, umma_sdesc(sA + kk * 32, 16, 1024, UMMA_LAYOUT_SW128),
                      umma_sdesc(sB + kk * 1024, QF_BK * 128, 512, UMMA_LAYOUT_SW128_BASE32B), idesc,
                      (kb > 0 || kk > 0) ? 1u : 0u);
          }
          issued_any = true;
          umma_commit(&empty_bar[stage]);
          if (++stage == QF_STAGES) {
            stage = 0;
            phase ^= 1;
          }
        }
        if (!ok) break;
        umma_commit(&tfull_bar[buf]);
      }
      if (!ok && issued_any) {
        umma_commit(drain_bar);
        mbar_drain(drain_bar, 0, args.err);
      }
    }
  } else if (warp < 6) {
    // ------------------------------------------------------------ epilogue
    const int q = warp & 3;
    const int row_in_tile = q * 32 + lane;
    int local = 0;
    const bool vec_ok = ((args.ldc & 3) == 0) && ((reinterpret_cast<uintptr_t>(args.C) & 15) == 0);
    for (int tile = blockIdx.x; tile < args.tiles; tile += gridDim.x, ++local) {
      const int m0 = (tile / args.n_tiles) * QF_BM, n0 = (tile % args.n_tiles) * QF_BN;
      const int buf = local & 1;
      const uint32_t use = static_cast<uint32_t>(local >> 1);
      if (!__all_sync(0xffffffffu, mbar_wait(&tfull_bar[buf], use & 1, abort_flag, args.err, GLC_DEV_TIMEOUT_EPILOGUE)))
        break;
      tc_fence_after();
      const int row = m0 + row_in_tile;
      const uint32_t taddr = tmem_base + (static_cast<uint32_t>(q * 32) << 16) + buf * QF_BN;
#pragma unroll 1
      for (int chunk = 0; chunk < QF_BN / 32; ++chunk) {
        uint32_t r[32];
        tmem_ld_32x32b_x32(taddr + chunk * 32, r);
        tmem_ld_wait();
        if (chunk == QF_BN / 32 - 1) {
          tc_fence_before();
          mbar_arrive(&tempty_bar[buf]);
        }
        const int col0 = n0 + chunk * 32;
        if (row >= args.M || col0 >= args.Kin) continue;
        float* crow = args.C + static_cast<size_t>(row) * args.ldc + col0;
        if (vec_ok && col0 + 32 <= args.Kin) {
#pragma unroll
          for (int j = 0; j < 8; ++j) {
            float4 v = make_float4(__uint_as_float(r[4 * j + 0]), __uint_as_float(r[4 * j + 1]),
                                   __uint_as_float(r[4 * j + 2]), __uint_as_float(r[4 * j + 3]));
            if (args.accumulate) {
              const float4 c = reinterpret_cast<const float4*>(crow)[j];
              v.x += c.x; v.y += c.y; v.z += c.z; v.w += c.w;
            }
            reinterpret_cast<float4*>(crow)[j] = v;
          }
        } else {
          const int lim = min(32, args.Kin - col0);
#pragma unroll
          for (int j = 0; j < 32; ++j) {
            if (j < lim) {
              float v = __uint_as_float(r[j]);
              if (args.accumulate) v += crow[j];
              crow[j] = v;
            }
          }
        }
      }
    }
  } else {
    // ------------------------------------------------------------ W producers
    // Warp pair (6+2s, 7+2s) fills ring slot s: k-blocks seq with seq % 4 == s.
    // Warp half h takes rows 16h..16h+15 of the 32; lane (cq = lane/8,
    // j = lane%8) decodes elements 4j..4j+3 of chunks cq and cq+4 of each row.
    const int pw = warp - 6;
    const int slot = pw >> 1, half = pw & 1;
    const int cq = lane >> 3, j = lane & 7;
    const int groups_per_row = args.Kin >> 2;
    int seq = 0;
    bool ok = true;
    for (int tile = blockIdx.x; tile < args.tiles && ok; tile += gridDim.x) {
      const int n0 = (tile % args.n_tiles) * QF_BN;
      for (int kb = 0; kb < args.k_blocks; ++kb, ++seq) {
        if ((seq % QF_STAGES) != slot) continue;
        const uint32_t phase = static_cast<uint32_t>(seq / QF_STAGES) & 1u;
        if (!__all_sync(0xffffffffu,
                        mbar_wait(&empty_bar[slot], phase ^ 1, abort_flag, args.err, GLC_DEV_TIMEOUT_PRODUCER))) {
          ok = false;
          break;
        }
        uint8_t* sB = smem + slot * QF_STAGE_BYTES + QF_A_BYTES;
#pragma unroll 1
        for (int b0 = 0; b0 < 32; b0 += QF_BATCH) {
          // items t: row 16*half + (b0 + t) / 2, chunk cq + 4 * ((b0 + t) % 2)
          float v[QF_BATCH][4];
#pragma unroll
          for (int t = 0; t < QF_BATCH; ++t) {
            const int it = b0 + t;
            const int r = 16 * half + (it >> 1), chunk = cq + 4 * (it & 1);
            const int nout = kb * QF_BK + r, kin = n0 + 32 * chunk + 4 * j;
            if (nout < args.Nout && kin < args.Kin) {
              const size_t g = static_cast<size_t>(nout) * static_cast<size_t>(groups_per_row) + (kin >> 2);
              qf::dequant4(args.w, args.type, g, v[t]);
            } else {
              v[t][0] = v[t][1] = v[t][2] = v[t][3] = 0.f;  // rows past Nout must not add to the sums
            }
          }
#pragma unroll
          for (int t = 0; t < QF_BATCH; ++t) {
            const int it = b0 + t;
            const int r = 16 * half + (it >> 1), chunk = cq + 4 * (it & 1);
            *reinterpret_cast<float4*>(sB + b_tile_offset(chunk, r, j)) =
                make_float4(round_tf32(v[t][0]), round_tf32(v[t][1]), round_tf32(v[t][2]), round_tf32(v[t][3]));
          }
        }
        fence_proxy_async_smem();  // these generic stores are read by the tensor core (async proxy)
        __syncwarp();
        if (lane == 0) mbar_arrive(&bfull_bar[slot]);
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem_base, QF_TMEM_COLS);
  }
}

}  // namespace

// Whether the fused kernel takes this weight: a decodable stored format whose
// blocks never straddle a row or a 256-column tile.
bool quant_fused_supported(int type, int Kin) {
  const int be = qf::block_elems(type);
  if (be == 0 || type == qf::F32) return false;
  return Kin % (be > 4 ? be : 4) == 0;
}

int gemm_quant_fused(Context* ctx, const float* dY, int ldy, const void* Wq, int type, float* dX, int ldx, int M,
                     int Kin, int Nout, bool accumulate, cudaStream_t s) {
  if (M < 0 || Kin <= 0 || Nout <= 0) return ctx->fail(GLC_ERR_INVALID, "quant gemm: bad size");
  if (!quant_fused_supported(type, Kin))
    return ctx->fail(GLC_ERR_INVALID, "quant gemm: format not decodable in the GEMM for this row length");
  if (!dY || !Wq || !dX || (ldy & 3) || (reinterpret_cast<uintptr_t>(dY) & 15) ||
      (reinterpret_cast<uintptr_t>(Wq) & 1) || ldy < Nout || ldx < Kin)
    return ctx->fail(GLC_ERR_INVALID, "quant gemm: dY must be 16-byte aligned with ld a multiple of 4, W 2-byte aligned");
  if (M == 0) return 0;
  CUtensorMap tm;
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(Nout), static_cast<cuuint64_t>(M)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(ldy) * 4};
  cuuint32_t box[2] = {QF_BK, QF_BM};
  cuuint32_t estr[2] = {1, 1};
  if (ctx->encode_tiled(&tm, CU_TENSOR_MAP_DATA_TYPE_FLOAT32, 2, const_cast<float*>(dY), dims, strides, box, estr,
                        CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B) != 0)
    return ctx->fail(GLC_ERR_INVALID, "quant gemm: cuTensorMapEncodeTiled failed for dY");
  QuantGemmArgs a;
  a.w = static_cast<const uint8_t*>(Wq);
  a.type = type;
  a.C = dX;
  a.ldc = ldx;
  a.M = M;
  a.Kin = Kin;
  a.Nout = Nout;
  a.accumulate = accumulate ? 1 : 0;
  a.m_tiles = (M + QF_BM - 1) / QF_BM;
  a.n_tiles = (Kin + QF_BN - 1) / QF_BN;
  a.k_blocks = (Nout + QF_BK - 1) / QF_BK;
  a.tiles = a.m_tiles * a.n_tiles;
  a.err = ctx->d_err;
  cudaError_t e = cudaFuncSetAttribute(gemm_quant_fused_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                       QF_SMEM_BYTES);
  if (e != cudaSuccess) return ctx->fail_cuda(e, "quant gemm: shared memory attribute");
  const int grid = a.tiles < ctx->num_sms ? a.tiles : ctx->num_sms;
  ProfScope prof(ctx, PROF_GEMM, 2.0 * M * static_cast<double>(Kin) * Nout, s);
  glc::launch_pdl(ctx, gemm_quant_fused_kernel, grid, QF_THREADS, QF_SMEM_BYTES, s, tm, a);
  GLC_LAUNCH_CHECK(ctx, "quant gemm");
  return 0;
}

}  // namespace glc
