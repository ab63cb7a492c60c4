// Attention backward without any device allocation.
//
// glc_attention_bwd takes its scratch (the per-row D = sum(dO * O) vector,
// B*H*S floats) from the context workspace, which is cudaMalloc'ed on first
// use and re-allocated, after a device synchronisation, when a larger call
// arrives.  Some callers cannot allow either: a host program whose device
// memory is entirely reserved by its own allocator or budget (a cudaMalloc
// there fails or fragments the pool), and a program that must never make the
// device synchronise in the middle of its work (growing the workspace waits
// for all queued kernels, stalling other streams such as a gradient allreduce
// in flight).  glc_attention_bwd_noalloc serves them: the scratch is a
// file-scope __device__ array of fixed size, and the call performs no
// cudaMalloc, no cudaFree and no allocating library call.
//
// The library is built without relocatable device code, so this file is a
// module of its own, and CUDA loads modules lazily by default: the array is
// placed in device memory when its module is first touched on a device.  That
// happens in glc_init (noalloc_scratch_setup below), which looks up the
// array's device address with the device current and caches it, so a device
// holds the array from the first context created on it until the process
// exits, and the entry point itself only reads the cached address.
#include <mutex>
#include <string>

#include "glc_internal.h"

// Maximum B*H*S (rows of D) a call may need: 1,048,576 floats = 4 MiB.
#define GLC_ATTN_NOALLOC_MAX_ROWS (1 << 20)

namespace {

static __device__ __align__(256) float g_attn_bwd_scratch[GLC_ATTN_NOALLOC_MAX_ROWS];

// In host code the array name is only a host-side stand-in, not a device
// address: the device address is looked up once per device with
// cudaGetSymbolAddress and cached here.
constexpr int kMaxDevices = 64;
std::mutex g_mu;
float* g_scratch_ptr[kMaxDevices] = {nullptr};

}  // namespace

namespace glc {

int noalloc_scratch_setup(Context* c) {
  if (c->device < 0 || c->device >= kMaxDevices) return 0;  // the entry point reports it
  std::lock_guard<std::mutex> lock(g_mu);
  if (g_scratch_ptr[c->device]) return 0;
  // glc_init made c->device current; the lookup loads this file's module on
  // that device if lazy loading has not done so yet.
  void* p = nullptr;
  cudaError_t e = cudaGetSymbolAddress(&p, g_attn_bwd_scratch);
  if (e != cudaSuccess || !p) return c->fail_cuda(e, "attention_bwd_noalloc set-up: cudaGetSymbolAddress");
  g_scratch_ptr[c->device] = static_cast<float*>(p);
  return 0;
}

}  // namespace glc

namespace {

int scratch_for_device(glc::Context* c, float** out) {
  if (c->device < 0 || c->device >= kMaxDevices) return c->fail(GLC_ERR_UNSUPPORTED, "attention_bwd_noalloc: device index too large");
  std::lock_guard<std::mutex> lock(g_mu);
  if (!g_scratch_ptr[c->device])
    return c->fail(GLC_ERR_INVALID, "attention_bwd_noalloc: the scratch address was not set up by glc_init");
  *out = g_scratch_ptr[c->device];
  return 0;
}

}  // namespace

extern "C" int glc_attention_bwd_noalloc(glc_ctx* ctx, const float* q, const float* k, const float* v,
                                         const float* o, const float* lse, const float* dO, float* dq, float* dk,
                                         float* dv, int B, int S, int H, int Hkv, int hd, int round_dv) {
  if (!ctx) return GLC_ERR_INVALID;
  glc::Context* c = reinterpret_cast<glc::Context*>(ctx);
  if (B <= 0 || S <= 0 || H <= 0) return c->fail(GLC_ERR_INVALID, "attention_bwd_noalloc: empty problem");
  const long long rows = static_cast<long long>(B) * H * S;
  if (rows > GLC_ATTN_NOALLOC_MAX_ROWS)
    return c->fail(GLC_ERR_INVALID, "attention_bwd_noalloc: B*H*S = " + std::to_string(rows) +
                                        " exceeds the fixed scratch of " + std::to_string(GLC_ATTN_NOALLOC_MAX_ROWS) +
                                        " rows; use glc_attention_bwd");
  float* D = nullptr;
  int rc = scratch_for_device(c, &D);
  if (rc) return rc;
  // D is fully written by the first kernel of the backward before it is
  // read, so the previous call's contents need no clearing.
  // No partial buffer: each CTA sums its KV head's query-head group itself.
  const glc::AttnIO io{q, H * hd, k, Hkv * hd, v, Hkv * hd, dq, H * hd, dk, Hkv * hd, dv, Hkv * hd};
  return glc::attention_bwd(c, io, o, lse, dO, D, nullptr, B, S, H, Hkv, hd, round_dv != 0, c->stream);
}
