// Internal host-side declarations shared by the library's translation units.
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>

#include <cstddef>
#include <cstdint>
#include <mutex>
#include <string>
#include <vector>

#include "../../include/gollama_cuda.h"

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
  EncodeTiledFn encode_fn = nullptr;
  // scratch workspace owned by the context (grown on demand, never shrunk)
  void* ws = nullptr;
  size_t ws_bytes = 0;
  // data parallel
  void* nccl_comm = nullptr;
  int rank = 0;
  int world = 1;
  cudaEvent_t timer_start = nullptr, timer_stop = nullptr;

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

// A GEMM operand.  K-major: element (i, k) at ptr[i*ld + k].
// MN-major: element (i, k) at ptr[k*ld + i].
struct GemmOperand {
  const float* ptr;
  int ld;
  bool mn_major;
};

int gemm_tf32(Context* ctx, const GemmOperand& A, const GemmOperand& B, float* C, int ldc, int M, int N, int K,
              bool accumulate, const float* R, int ldr, bool round_out, cudaStream_t stream);
int gemm_empty_k(Context* ctx, float* C, int ldc, int M, int N, bool accumulate, const float* R, int ldr,
                 cudaStream_t stream);

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
