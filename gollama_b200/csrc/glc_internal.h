// Internal host-side declarations shared by the library's translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <array>
#include <cstddef>
#include <cstdint>
#include <functional>
#include <mutex>
#include <string>
#include <utility>
#include <vector>

#include <nvtx3/nvToolsExt.h>

#include "../../include/gollama_cuda.h"

#if defined(__CUDACC__)
// First statement of every kernel: wait for the grid this launch depends on
// (a no-op unless launched with programmatic serialization), then let the
// next kernel's launch begin while this one runs.
#define GLC_PDL_ENTRY()                                      \
  do {                                                       \
    asm volatile("griddepcontrol.wait;" ::: "memory");       \
    asm volatile("griddepcontrol.launch_dependents;" :::);   \
  } while (0)
#endif

namespace glc {

using EncodeTiledFn = CUresult (*)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                   const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

struct Context {
  int device = 0;
  int num_sms = 0;
  cudaStream_t stream = nullptr;       // compute stream: every op is enqueued here
  cudaStream_t comm_stream = nullptr;  // data-parallel gradient allreduce
  int* d_err = nullptr;                // device error word written by bounded waits
  std::string last_error;
  uint64_t launches = 0;               // kernels this library launched
  int gemm_variant = 0;                // 0 automatic, 1 single-CTA tiles, 2 CTA-pair tiles
  int gemm_order = 0;                  // CTA-pair tile order: 0 automatic (= 1), 1 host lists / rotation, 2 dynamic
  // dynamic tile order: one zeroed counter per launch, from a ring cleared
  // on the stream when it wraps
  static constexpr int kDynCounters = 1024;
  int* dyn_ctr = nullptr;
  unsigned long long dyn_next = 0;
  // device tile lists of grouped CTA-pair GEMM launches, by (tiles and
  // k-blocks of each problem, clusters); built once per shape
  std::vector<std::pair<std::array<long long, 5>, int*>> gemm_sched;
  bool fuse_swiglu = false;            // trainer: SwiGLU forward in the gate/up GEMM epilogue (Llama semantics)
  int attn_split = 0;                  // dK/dV CTAs per KV head: 0 automatic, else a divisor of the group
  int rmsnorm_variant = 0;             // RMSNorm backward: 0 automatic (3 for the exact gradient, else 1), 1 row per iteration, 2 cp.async rows, 3 bulk-copied rows
  int attn_dq_variant = 0;             // attention backward dQ: 0 automatic (= 3), 1 a CTA per query tile, 2 persistent,
                                       // 3 persistent with two math groups
  int attn_dkdv_variant = 0;           // attention backward dK/dV: 0 automatic (= 2), 1 one math group, 2 two math groups
  int ce_variant = 0;                  // softmax-CE above V = 8192: 0 automatic (2 for the Llama arithmetic up to V = 32768, else 1), 1 one-shot 4-CTA clusters, 2 streamed rows
  int attn_fwd_variant = 0;            // attention forward: 0 automatic (= 2), 1 a CTA per query tile, 2 persistent
  int quant_path = 0;                  // dX through a stored weight: 0 automatic (= 1), 1 dequantize + GEMM, 2 fused
  bool tracing = false;                // NVTX ranges around the phases of a training step
  bool pdl = true;                     // programmatic dependent launch between this library's kernels
  EncodeTiledFn encode_fn = nullptr;
  // scratch workspace owned by the context (grown on demand, never shrunk)
  void* ws = nullptr;
  size_t ws_bytes = 0;
  // data parallel
  void* nccl_comm = nullptr;
  int rank = 0;
  int world = 1;
  cudaEvent_t timer_start = nullptr, timer_stop = nullptr;
  // per-kernel-class timing (glc_profile_begin/end): event pairs recorded on
  // the launching stream around each launch
  struct ProfRecord {
    cudaEvent_t a, b;
    int cls;
    double work;
  };
  bool profiling = false;
  std::vector<ProfRecord> prof;
  std::vector<cudaEvent_t> event_pool;
  cudaEvent_t get_event() {
    if (!event_pool.empty()) {
      cudaEvent_t e = event_pool.back();
      event_pool.pop_back();
      return e;
    }
    cudaEvent_t e = nullptr;
    cudaEventCreate(&e);
    return e;
  }

  int fail(int code, const std::string& msg) {
    last_error = msg;
    return code;
  }
  int fail_cuda(cudaError_t e, const char* what) {
    last_error = std::string(what) + ": " + cudaGetErrorString(e);
    return GLC_ERR_CUDA;
  }
  void count_launch() { ++launches; }
  int encode_tiled(CUtensorMap* tm, CUtensorMapDataType dt, cuuint32_t rank, void* ptr, const cuuint64_t* dims,
                   const cuuint64_t* strides, const cuuint32_t* box, const cuuint32_t* estr, CUtensorMapSwizzle sw,
                   CUtensorMapL2promotion l2) {
    if (!encode_fn) return -1;
    CUresult r = encode_fn(tm, dt, rank, ptr, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, sw, l2,
                           CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS ? 0 : -1;
  }
  // Returns a device scratch buffer of at least `bytes` (stream-ordered use only).
  int workspace(size_t bytes, void** out);
};

// An NVTX range for the lifetime of the object when the context traces
// (NVTX v3 is header-only: without a tool attached the calls return at once).
struct TraceRange {
  bool on;
  TraceRange(const Context* c, const char* name) : on(c->tracing) {
    if (on) nvtxRangePushA(name);
  }
  ~TraceRange() {
    if (on) nvtxRangePop();
  }
  TraceRange(const TraceRange&) = delete;
  TraceRange& operator=(const TraceRange&) = delete;
};

// Kernel classes of the profiler; work is FLOPs (GEMM, attention) or bytes.
enum ProfClass : int {
  PROF_GEMM = 0,      // tcgen05 TF32 GEMM, 2*M*N*K FLOPs
  PROF_ATTN_FWD = 1,  // 2 matmuls over the causal half, FLOPs
  PROF_ATTN_BWD = 2,  // dV, dP, dQ, dK matmuls over the causal half, FLOPs
  PROF_RMSNORM = 3,   // bytes
  PROF_SWIGLU = 4,    // bytes
  PROF_CE = 5,        // bytes
  PROF_ADAMW = 6,     // bytes (grad norm + AdamW)
  PROF_OTHER = 7,     // bytes (embedding, RoPE, fills, copies)
  PROF_CLASSES = 8
};

// Records an event pair around the launches in its scope when profiling.
struct ProfScope {
  Context* c;
  int cls;
  double work;
  cudaStream_t s;
  cudaEvent_t a = nullptr;
  ProfScope(Context* ctx, int k, double w, cudaStream_t st) : c(ctx), cls(k), work(w), s(st) {
    if (c->profiling) {
      a = c->get_event();
      cudaEventRecord(a, s);
    }
  }
  ~ProfScope() {
    if (a) {
      cudaEvent_t b = c->get_event();
      cudaEventRecord(b, s);
      c->prof.push_back({a, b, cls, work});
    }
  }
};

// A GEMM operand.  K-major: element (i, k) at ptr[i*ld + k].
// MN-major: element (i, k) at ptr[k*ld + i].
struct GemmOperand {
  const float* ptr;
  int ld;
  bool mn_major;
};

int gemm_tf32(Context* ctx, const GemmOperand& A, const GemmOperand& B, float* C, int ldc, int M, int N, int K,
              bool accumulate, const float* R, int ldr, bool round_out, cudaStream_t stream);
// One GEMM C[M,N] (+)= A . B^T (+ R) of a grouped launch.
struct GemmSpec {
  GemmOperand A, B;
  float* C;
  int ldc, M, N, K;
  bool accumulate;
  const float* R;
  int ldr;
  bool round_out;
  // SwiGLU epilogue: glu = F > 0 means B's rows are [gate F | up F] (N = 2F);
  // C receives both halves and glu_h [M][F] (row stride ld_glu) receives
  // h = silu(gate) * up, TF32-rounded when glu_round.
  int glu = 0;
  float* glu_h = nullptr;
  int ld_glu = 0;
  bool glu_round = false;
  bool glu_fast = false;  // Llama semantics: expf in the sigmoid
  // Sum of squares of the stored C (float64 partials, one per epilogue warp
  // and tile, at most gemm_sumsq_slots(M, N) of them, added in any fixed
  // order by the caller); nullptr: none.  Not with the SwiGLU epilogue.
  double* sumsq = nullptr;
  long long sumsq_cap = 0;
};
// Upper bound of the partial slots a GEMM with sumsq writes (either tile
// shape): ceil(M/128) * ceil(N/256) * 8.
long long gemm_sumsq_slots(long long M, long long N);
// Tile lists of a grouped CTA-pair launch: tiles 0..tiles0-1 of problem 0
// (kb0 k-blocks each) then tiles1 of problem 1, handed out in order to the
// cluster that frees first (cost k-blocks + 2).  Writes [clusters + 1 offsets
// | tile ids] and returns true when that estimate beats the rotation
// tile = cluster + i * clusters by at least 1 %; false: keep the rotation.
bool gemm_tile_lists(int tiles0, int kb0, int tiles1, int kb1, int clusters, std::vector<int>* out);
// dX[M, Kin] (+)= dY[M, Nout] . deq(W) with W [Nout][Kin] stored in a GGUF
// format, decoded inside the GEMM's operand load (gemm_quant_fused.cu).
bool quant_fused_supported(int type, int Kin);
// Shared-memory image (1024 floats) of one MN-major 32 x 32 TMA box loaded
// with SWIZZLE_128B_ATOM_32B from src (element (mn, k) at src[k * 32 + mn]).
int gemm_quant_fused(Context* ctx, const float* dY, int ldy, const void* Wq, int type, float* dX, int ldx, int M,
                     int Kin, int Nout, bool accumulate, cudaStream_t s);
// Runs up to two independent GEMMs in one persistent launch (shared tile queue).
int gemm_tf32_group(Context* ctx, const GemmSpec* specs, int n, cudaStream_t stream);
int gemm_empty_k(Context* ctx, float* C, int ldc, int M, int N, bool accumulate, const float* R, int ldr,
                 cudaStream_t stream);

// ---- kernels (each enqueues on stream `s`; returns 0 or a GLC_ERR_* code)
int rmsnorm_fwd(Context* ctx, const float* x, const float* w, float* y, float* rms, int rows, int cols, float eps,
                bool round_out, cudaStream_t s);
// scratch == nullptr: per-block dw partials go to the context workspace.
int rmsnorm_bwd(Context* ctx, const float* x, const float* w, const float* rms, const float* dy, float* dx,
                float* dx_round, float* dw, int rows, int cols, bool full, bool dx_accumulate, bool dw_accumulate,
                float* scratch, size_t scratch_bytes, cudaStream_t s);
// rows x cols, each operand with its own row stride (elements; multiples of 4).
// fast_exp: llama semantics, expf/logf instead of the reference's exp32/log32
int swiglu_fwd(Context* ctx, const float* g, const float* u, size_t ld_in, float* h, size_t ld_h, size_t rows,
               size_t cols, bool round_out, cudaStream_t s, bool fast_exp = false);
int swiglu_bwd(Context* ctx, const float* g, const float* u, size_t ld_in, const float* dh, size_t ld_dh, float* dg,
               float* du, size_t ld_out, size_t rows, size_t cols, bool accumulate, bool round_out, cudaStream_t s,
               bool fast_exp = false);
int fill(Context* ctx, float* p, float v, size_t n, cudaStream_t s);
int round_copy(Context* ctx, const float* src, float* dst, size_t n, cudaStream_t s);
// data parallel (dp.cu): in-place fp32 sum over the ranks
int dp_allreduce_grads(Context* c, float* buf, size_t n);
int dp_allreduce_on(Context* c, float* buf, size_t n, cudaStream_t stream);
int exp32(Context* ctx, const float* x, float* y, size_t n, cudaStream_t s);
int add_inplace(Context* ctx, float* dst, const float* src, size_t n, cudaStream_t s);
// x: T rows of row stride ld (elements); the first nh*hd columns are rotated.
int rope(Context* ctx, float* x, int ld, int T, int S, int nh, int hd, const float* cos_t, const float* sin_t,
         bool inverse, bool round_out, cudaStream_t s);
int embed_fwd(Context* ctx, const int64_t* tok, const float* E, const float* P, float* out, int T, int S, int d, int V,
              cudaStream_t s);
int embed_bwd(Context* ctx, const int* seg_tok, const int* seg_start, const int* order, int nseg, const float* dh,
              float* dE, int d, cudaStream_t s, const int* nseg_dev = nullptr);
// Offsets (ints) of the device-built scatter segments of T tokens in one
// buffer of `total` ints: seg_tok[T], seg_start[T + 1], order[T], nseg[1],
// then 4*T ints of sort scratch.
struct EmbedSegLayout {
  int64_t seg_tok, seg_start, order, nseg, scratch, total;
  explicit EmbedSegLayout(int64_t T)
      : seg_tok(0), seg_start(T), order(2 * T + 1), nseg(3 * T + 1), scratch(3 * T + 2), total(7 * T + 2) {}
};
// Builds the segments of embed_bwd for tok[T] (device ids) into out
// (EmbedSegLayout(T).total ints), on the device, with no host round trip.
int embed_segments_device(Context* ctx, const int64_t* tok, int T, int V, int* out, cudaStream_t s);
int softmax_ce(Context* ctx, float* logits, const int64_t* targets, int rows, int V, float scale, float* row_logp,
               float* loss, bool write_grad, bool round_out, cudaStream_t s, bool fast_exp = false);
// q/k/v (and their gradients) may be column slices of one fused projection
// output: each has its own row stride in elements.
struct AttnIO {
  const float* q;
  int q_ld;
  const float* k;
  int k_ld;
  const float* v;
  int v_ld;
  float* dq;
  int dq_ld;
  float* dk;
  int dk_ld;
  float* dv;
  int dv_ld;
};
// o: [B*S, H*hd] contiguous; lse: [B, H, S].
int attention_fwd(Context* ctx, const AttnIO& io, float* o, float* lse, int B, int S, int H, int Hkv, int hd,
                  bool round_out, cudaStream_t s);
// partial: 2*B*S*H*hd floats of scratch for per-query-head dK/dV partials
// (attention_bwd_partial_floats); nullptr makes each CTA loop over its KV
// head's query-head group instead (no scratch beyond D).  dO: contiguous.
// rope_cos/rope_sin ([>= S][hd/2], 16-byte aligned): when given, dq and dk
// leave with the transposed RoPE rotation applied and TF32-rounded, as the
// separate backward RoPE pass would leave them.
// Looks up, with ctx->device current, the device address of the fixed scratch
// array of glc_attention_bwd_noalloc and caches it (once per device); called
// by glc_init.
int noalloc_scratch_setup(Context* ctx);
int attention_bwd(Context* ctx, const AttnIO& io, const float* o, const float* lse, const float* dO, float* D,
                  float* partial, int B, int S, int H, int Hkv, int hd, bool round_dv, cudaStream_t s,
                  const float* rope_cos = nullptr, const float* rope_sin = nullptr);
size_t attention_bwd_partial_floats(int B, int S, int H, int Hkv, int hd);
// elems: number of gradient elements the segments cover (for the profiler).
int grad_norm(Context* ctx, const float* grads, const int64_t* segs, int nseg, float max_norm, double* norm_out,
              float* scale_out, double* scratch, int scratch_count, double elems, cudaStream_t s);
// The two halves of grad_norm: grad_sumsq writes bx * nseg float64 partial
// sums of squares (bx = grad_norm_blocks(nseg) blocks per segment);
// grad_norm_finish adds n partials in a fixed order and derives the norm and
// the clip scale (GradientClipping, optimizer.go:169-196); with more than
// 8192 partials and lvl (room for ceil(n/1024) doubles) it adds them in
// blocks of 1024 first.
int grad_norm_blocks(const Context* ctx, int nseg);
int grad_sumsq(Context* ctx, const float* grads, const int64_t* segs, int nseg, int bx, double* partial, double elems,
               cudaStream_t s);
// Per-chunk float64 sums of squares of chunks {start, len} (multiples of 4
// floats) into out[nchunks], `blocks` blocks striding over the chunks.
int grad_sumsq_chunks(Context* ctx, const float* grads, const int64_t* chunks, int nchunks, int blocks, double* out,
                      double elems, cudaStream_t s);
int grad_norm_finish(Context* ctx, const double* partial, long long n, float max_norm, double* norm_out,
                     float* scale_out, cudaStream_t s, double* lvl = nullptr, long long lvl_cap = 0);
int adamw(Context* ctx, float* p, float* g, float* m, float* v, float* shadow, const int64_t* segs, int nseg,
          const float* clip_scale, float lr, float beta1, float beta2, float eps, float wd, int step, double elems,
          cudaStream_t s, bool write_grad = true);
// write_grad = false leaves the unclipped gradient in g (the caller applies the
// clip scale later, scale_in_place); otherwise g receives the clipped gradient
// as GradientClipping (optimizer.go:169-196) leaves it.
int scale_in_place(Context* ctx, float* g, size_t n, const float* scale, cudaStream_t s);

// RoPE tables (pkg/model/rope.go:33-48) computed on the host in float64 and
// rounded to float32: cos_t/sin_t are [max_seq][dim/2].
void rope_table_host(int dim, int max_seq, float theta, float* cos_t, float* sin_t);

// Deterministic embedding-gradient segments from host token ids (clamped to
// [0, V)): distinct ids ascending, their tokens in ascending position.
void embed_segments_host(const int64_t* tok, int T, int V, std::vector<int>& seg_tok, std::vector<int>& seg_start,
                         std::vector<int>& order);

// ---------------------------------------------------------------- checkpoints (checkpoint.cpp)
// Message of the calling thread's last failed host-only call (no context).
std::string& host_error();
// Element counts of the parameters in Params() order (trainer.cu; host only).
bool param_sizes(const glc_train_config& cfg, std::vector<int64_t>* sizes);
// Go's fmt %v of a float32 into out (at most 16 bytes); returns the length.
int format_go_float32(float v, char* out);
bool parse_go_float32(const char* s, const char* e, float* v);
// Callbacks that move floats [off, off + n) of the parameter arena (text) or
// of arena a = 0 parameters, 1 m, 2 v (state) between the model and a host
// chunk; they return false on a failed copy.
using CkptFetch = std::function<bool(int64_t off, int64_t n, float* dst)>;
using CkptStore = std::function<bool(int64_t off, int64_t n, const float* src)>;
using StateFetch = std::function<bool(int a, int64_t off, int64_t n, float* dst)>;
using StateStore = std::function<bool(int a, int64_t off, int64_t n, const float* src)>;
struct StateInfo {
  int step;       // LRScheduler step (Trainer.step)
  int adam_step;  // AdamW.t
};
int ckpt_text_write(const char* path, int step, const glc_train_config& cfg, const std::vector<int64_t>& sizes,
                    const CkptFetch& fetch);
int ckpt_text_read(const char* path, const glc_train_config& cfg, const std::vector<int64_t>& sizes, int* step,
                   const CkptStore& store);
int state_write(const char* path, const StateInfo& info, const glc_train_config& cfg, int64_t n,
                const StateFetch& fetch);
int state_read(const char* path, const glc_train_config& cfg, int64_t n, StateInfo* info, const StateStore& store);

// Kernel launch through cudaLaunchKernelEx.  With the context's pdl switch on,
// the launch may begin while the previous kernel on the stream finishes
// (programmatic dependent launch); every kernel launched this way starts with
// GLC_PDL_ENTRY, which waits for that predecessor to complete and its memory
// to be visible before touching global memory.  Off (default), it is an
// ordinary launch.
template <typename... KArgs, typename... Args>
inline void launch_pdl(const Context* ctx, void (*kernel)(KArgs...), dim3 grid, dim3 block, size_t smem,
                       cudaStream_t s, Args&&... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = grid;
  cfg.blockDim = block;
  cfg.dynamicSmemBytes = smem;
  cfg.stream = s;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = ctx->pdl ? 1 : 0;
  cudaLaunchKernelEx(&cfg, kernel, std::forward<Args>(args)...);
}

inline unsigned grid_for(size_t n, int block, int num_sms, int per_sm = 8) {
  size_t g = (n + block - 1) / block;
  size_t cap = static_cast<size_t>(num_sms) * per_sm;
  if (g > cap) g = cap;
  if (g == 0) g = 1;
  return static_cast<unsigned>(g);
}

}  // namespace glc

#define GLC_LAUNCH_CHECK(ctx, what)                              \
  do {                                                           \
    cudaError_t e__ = cudaGetLastError();                        \
    if (e__ != cudaSuccess) return (ctx)->fail_cuda(e__, what); \
    (ctx)->count_launch();                                       \
  } while (0)
