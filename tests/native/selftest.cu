// Test-only native code (not part of libgollama_cuda.so): checks of the
// library's device-side primitives that need a kernel of their own.
//
// glc_selftest_bounded_wait: the library's bounded mbarrier wait (mbar_wait,
// gollama_b200/csrc/sm100.cuh) compiled with a short limit, on a barrier that
// nothing ever arrives on.  Every thread of the block must give up after the
// limit, record the error code in *err and return; the kernel then exits
// normally, so the context stays usable.  No TMA copy or MMA is in flight.
#define GLC_WAIT_TIMEOUT_NS 200000000ull  // 200 ms
#include "sm100.cuh"

namespace {

__global__ void bounded_wait_kernel(int* err, int* gave_up, unsigned long long* elapsed_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  if (threadIdx.x == 0) {
    glc::mbar_init(&bar, 1);
    abort_flag = 0;
    glc::fence_mbar_init();
  }
  __syncthreads();
  const uint64_t t0 = glc::globaltimer_ns();
  // phase 0 never completes: no thread arrives
  const bool ok = glc::mbar_wait(&bar, 0, &abort_flag, err, GLC_DEV_TIMEOUT_EPILOGUE);
  if (!ok) atomicAdd(gave_up, 1);
  __syncthreads();
  if (threadIdx.x == 0) *elapsed_ns = glc::globaltimer_ns() - t0;
}

}  // namespace

// out[0] = error code recorded, out[1] = threads that gave up, out[2..3] =
// elapsed ns (uint64).  Returns 0, or the CUDA error of the launch or copy.
extern "C" __attribute__((visibility("default"))) int glc_selftest_bounded_wait(int threads, long long* out) {
  int* d = nullptr;
  cudaError_t e = cudaMalloc(&d, 4 * sizeof(int) + sizeof(unsigned long long));
  if (e != cudaSuccess) return static_cast<int>(e);
  cudaMemset(d, 0, 4 * sizeof(int) + sizeof(unsigned long long));
  unsigned long long* el = reinterpret_cast<unsigned long long*>(d + 2);
  bounded_wait_kernel<<<1, threads>>>(d, d + 1, el);
  e = cudaDeviceSynchronize();
  int h[2] = {0, 0};
  unsigned long long ns = 0;
  if (e == cudaSuccess) e = cudaMemcpy(h, d, sizeof(h), cudaMemcpyDeviceToHost);
  if (e == cudaSuccess) e = cudaMemcpy(&ns, el, sizeof(ns), cudaMemcpyDeviceToHost);
  cudaFree(d);
  out[0] = h[0];
  out[1] = h[1];
  out[2] = static_cast<long long>(ns);
  return static_cast<int>(e);
}
