// Data parallelism: one process per GPU, fp32 gradient sum with NCCL over
// NVLink.  The reference has no distributed backend; this is the one exchange
// step data-parallel training needs (every rank holds a replica, trains on its
// share of the batch, and the gradients are summed before clipping and AdamW).
//
// Communicators are created non-blocking and every NCCL call is polled with a
// deadline, so a rank that never joins or dies turns into an error return
// (GLC_ERR_NCCL) after ncclCommAbort instead of a hang.
#include <dlfcn.h>
#include <nccl.h>

#include <chrono>
#include <cstdlib>
#include <cstring>
#include <thread>

#include "glc_internal.h"

namespace glc {
namespace {

// NCCL is resolved at run time (dlopen) rather than linked: a process may
// already hold another NCCL build under the same soname (PyTorch bundles
// one), and two copies must not meet.  Search order: $GLC_NCCL_LIB, a
// libnccl.so.2 already loaded in the process, then the system one.
struct NcclApi {
  decltype(&::ncclGetUniqueId) GetUniqueId = nullptr;
  decltype(&::ncclCommInitRankConfig) CommInitRankConfig = nullptr;
  decltype(&::ncclCommGetAsyncError) CommGetAsyncError = nullptr;
  decltype(&::ncclCommAbort) CommAbort = nullptr;
  decltype(&::ncclCommFinalize) CommFinalize = nullptr;
  decltype(&::ncclCommDestroy) CommDestroy = nullptr;
  decltype(&::ncclAllReduce) AllReduce = nullptr;
  decltype(&::ncclGetErrorString) GetErrorString = nullptr;
  bool ok = false;
};

const NcclApi& nccl() {
  static NcclApi api = [] {
    NcclApi a;
    void* h = nullptr;
    if (const char* env = std::getenv("GLC_NCCL_LIB")) h = dlopen(env, RTLD_NOW | RTLD_GLOBAL);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL | RTLD_NOLOAD);
    if (!h) h = dlopen("libnccl.so.2", RTLD_NOW | RTLD_GLOBAL);
    if (!h) return a;
    a.GetUniqueId = reinterpret_cast<decltype(a.GetUniqueId)>(dlsym(h, "ncclGetUniqueId"));
    a.CommInitRankConfig = reinterpret_cast<decltype(a.CommInitRankConfig)>(dlsym(h, "ncclCommInitRankConfig"));
    a.CommGetAsyncError = reinterpret_cast<decltype(a.CommGetAsyncError)>(dlsym(h, "ncclCommGetAsyncError"));
    a.CommAbort = reinterpret_cast<decltype(a.CommAbort)>(dlsym(h, "ncclCommAbort"));
    a.CommFinalize = reinterpret_cast<decltype(a.CommFinalize)>(dlsym(h, "ncclCommFinalize"));
    a.CommDestroy = reinterpret_cast<decltype(a.CommDestroy)>(dlsym(h, "ncclCommDestroy"));
    a.AllReduce = reinterpret_cast<decltype(a.AllReduce)>(dlsym(h, "ncclAllReduce"));
    a.GetErrorString = reinterpret_cast<decltype(a.GetErrorString)>(dlsym(h, "ncclGetErrorString"));
    a.ok = a.GetUniqueId && a.CommInitRankConfig && a.CommGetAsyncError && a.CommAbort && a.CommFinalize &&
           a.CommDestroy && a.AllReduce && a.GetErrorString;
    return a;
  }();
  return api;
}

struct Comm {
  ncclComm_t comm = nullptr;
  int timeout_ms = 600000;
  double* scratch = nullptr;
};

Comm* comm_of(Context* c) { return static_cast<Comm*>(c->nccl_comm); }

// Waits until the communicator has no operation in progress; aborts it on error or timeout.
int nccl_wait(Context* c, ncclResult_t r, const char* what) {
  Comm* cm = comm_of(c);
  auto t0 = std::chrono::steady_clock::now();
  while (true) {
    if (r != ncclSuccess && r != ncclInProgress) break;
    ncclResult_t st = ncclSuccess;
    ncclResult_t q = nccl().CommGetAsyncError(cm->comm, &st);
    if (q != ncclSuccess) {
      r = q;
      break;
    }
    if (st == ncclSuccess) return 0;
    if (st != ncclInProgress) {
      r = st;
      break;
    }
    if (std::chrono::duration_cast<std::chrono::milliseconds>(std::chrono::steady_clock::now() - t0).count() >
        cm->timeout_ms) {
      nccl().CommAbort(cm->comm);
      cm->comm = nullptr;
      return c->fail(GLC_ERR_NCCL, std::string(what) + ": timed out (communicator aborted)");
    }
    std::this_thread::sleep_for(std::chrono::microseconds(50));
  }
  std::string msg = std::string(what) + ": " + nccl().GetErrorString(r);
  if (cm->comm) {
    nccl().CommAbort(cm->comm);
    cm->comm = nullptr;
  }
  return c->fail(GLC_ERR_NCCL, msg);
}

}  // namespace

int dp_allreduce_grads(Context* c, float* buf, size_t n) { return dp_allreduce_on(c, buf, n, c->stream); }

// Enqueues an in-place fp32 sum over the ranks on `stream` and returns once
// NCCL has accepted it (the reduction itself runs asynchronously).
int dp_allreduce_on(Context* c, float* buf, size_t n, cudaStream_t stream) {
  Comm* cm = comm_of(c);
  if (!cm || !cm->comm) return c->fail(GLC_ERR_NCCL, "allreduce: data parallelism not initialised (glc_dp_init)");
  if (n == 0) return 0;
  ncclResult_t r = nccl().AllReduce(buf, buf, n, ncclFloat, ncclSum, cm->comm, stream);
  return nccl_wait(c, r, "ncclAllReduce");
}

}  // namespace glc

using glc::Context;

extern "C" {

int glc_dp_unique_id(unsigned char id[128]) {
  static_assert(sizeof(ncclUniqueId) == 128, "ncclUniqueId size");
  if (!id) return GLC_ERR_INVALID;
  if (!glc::nccl().ok) return GLC_ERR_NCCL;  // no usable libnccl.so.2
  ncclUniqueId u;
  if (glc::nccl().GetUniqueId(&u) != ncclSuccess) return GLC_ERR_NCCL;
  std::memcpy(id, &u, sizeof(u));
  return GLC_OK;
}

int glc_dp_init(glc_ctx* ctx, int rank, int world, const unsigned char id[128], int timeout_ms) {
  if (!ctx || !id || world < 1 || rank < 0 || rank >= world) return GLC_ERR_INVALID;
  Context* c = reinterpret_cast<Context*>(ctx);
  if (c->nccl_comm) return c->fail(GLC_ERR_INVALID, "glc_dp_init: already initialised");
  if (!glc::nccl().ok) return c->fail(GLC_ERR_NCCL, "glc_dp_init: libnccl.so.2 not found (set GLC_NCCL_LIB)");
  cudaSetDevice(c->device);
  auto* cm = new glc::Comm();
  cm->timeout_ms = timeout_ms > 0 ? timeout_ms : 600000;
  c->nccl_comm = cm;
  ncclUniqueId u;
  std::memcpy(&u, id, sizeof(u));
  ncclConfig_t cfg = NCCL_CONFIG_INITIALIZER;
  cfg.blocking = 0;
  // tuning: how many CTAs NCCL's kernels may take (SMs the gradient sums
  // hold while the backward's GEMMs run beside them); NCCL's default if unset
  if (const char* v = std::getenv("GLC_NCCL_MAX_CTAS")) cfg.maxCTAs = std::atoi(v);
  if (const char* v = std::getenv("GLC_NCCL_MIN_CTAS")) cfg.minCTAs = std::atoi(v);
  ncclResult_t r = glc::nccl().CommInitRankConfig(&cm->comm, world, u, rank, &cfg);
  int rc = glc::nccl_wait(c, r, "ncclCommInitRankConfig");
  if (rc) {
    delete cm;
    c->nccl_comm = nullptr;
    return rc;
  }
  if (cudaMalloc(&cm->scratch, 64) != cudaSuccess) return c->fail(GLC_ERR_NOMEM, "glc_dp_init: scratch");
  c->rank = rank;
  c->world = world;
  return GLC_OK;
}

int glc_dp_allreduce_sum(glc_ctx* ctx, float* buf, size_t n) {
  if (!ctx || (n && !buf)) return GLC_ERR_INVALID;
  return glc::dp_allreduce_grads(reinterpret_cast<Context*>(ctx), buf, n);
}

int glc_dp_allreduce_max_host(glc_ctx* ctx, double* value) {
  if (!ctx || !value) return GLC_ERR_INVALID;
  Context* c = reinterpret_cast<Context*>(ctx);
  glc::Comm* cm = glc::comm_of(c);
  if (!cm || !cm->comm) return c->fail(GLC_ERR_NCCL, "allreduce: data parallelism not initialised");
  if (cudaMemcpyAsync(cm->scratch, value, sizeof(double), cudaMemcpyHostToDevice, c->stream) != cudaSuccess)
    return GLC_ERR_CUDA;
  int rc = glc::nccl_wait(c, glc::nccl().AllReduce(cm->scratch, cm->scratch, 1, ncclDouble, ncclMax, cm->comm, c->stream),
                          "ncclAllReduce(max)");
  if (rc) return rc;
  if (cudaMemcpyAsync(value, cm->scratch, sizeof(double), cudaMemcpyDeviceToHost, c->stream) != cudaSuccess ||
      cudaStreamSynchronize(c->stream) != cudaSuccess)
    return GLC_ERR_CUDA;
  return GLC_OK;
}

int glc_dp_barrier(glc_ctx* ctx) {
  double v = 0.0;
  int rc = glc_dp_allreduce_max_host(ctx, &v);
  return rc;
}

int glc_dp_destroy(glc_ctx* ctx) {
  if (!ctx) return GLC_ERR_INVALID;
  Context* c = reinterpret_cast<Context*>(ctx);
  glc::Comm* cm = glc::comm_of(c);
  if (!cm) return GLC_OK;
  cudaStreamSynchronize(c->stream);
  if (cm->comm) {
    glc::nccl().CommFinalize(cm->comm);
    glc::nccl_wait(c, ncclSuccess, "ncclCommFinalize");
    if (cm->comm) glc::nccl().CommDestroy(cm->comm);
  }
  cudaFree(cm->scratch);
  delete cm;
  c->nccl_comm = nullptr;
  c->world = 1;
  c->rank = 0;
  return GLC_OK;
}

}  // extern "C"
