// selftest.cu -- failure-detection self-test: the bounded waits of the GEMM kernels, made
// to run out on purpose, without faulting or hanging anything.
//
// Every wait in the operator's kernels is bounded (sm100.cuh): an mbarrier wait, or a wait
// for another CTA's flag in global memory, gives up after a time limit, and the kernel
// records an error bit and returns instead of spinning. fmoe_selftest_wait_timeout() runs
// one small kernel whose two waits can never complete -- an mbarrier nobody arrives on,
// and a global flag nobody sets -- with a short limit, and reports what the kernel saw:
// which waits expired and how long each one waited. The CUDA context stays usable; the
// caller can run the operator right after. No GPU fault, trap or endless loop is involved.
#include <cuda_runtime.h>

#include <string>

#include "fmoe.h"
#include "fmoe_common.cuh"
#include "fmoe_kernels.cuh"
#include "sm100.cuh"

namespace fmoe {
namespace {

using namespace sm100;

// [0] bit 0: the mbarrier wait expired, bit 1: the flag wait expired;
// [1], [2] nanoseconds each wait took. g_never_set is zero-initialised and never written.
__device__ unsigned long long g_selftest_result[3];
__device__ int g_never_set;

__global__ void __launch_bounds__(64) wait_timeout_selftest_kernel(uint64_t timeout_ns) {
  __shared__ uint64_t bar;
  __shared__ int abort_flag;
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  if (threadIdx.x == 0) {
    mbar_init(&bar, 1);
    abort_flag = 0;
    fence_mbar_init();
    g_selftest_result[0] = 0;
  }
  __syncthreads();
  if (lane == 0) {
    const uint64_t t0 = globaltimer();
    bool done;
    if (warp == 0)
      done = mbar_wait(&bar, 0, &abort_flag, timeout_ns);  // nobody arrives
    else
      done = wait_nonzero(&g_never_set, &abort_flag, timeout_ns);  // nobody writes
    const uint64_t dt = globaltimer() - t0;
    g_selftest_result[1 + warp] = dt;
    if (!done) atomicOr(&g_selftest_result[0], 1ull << warp);
  }
  __syncthreads();
}

}  // namespace
}  // namespace fmoe

using namespace fmoe;

extern "C" int fmoe_selftest_wait_timeout(uint64_t timeout_ns, uint64_t* result,
                                          void* stream_ptr) {
  if (!result) {
    set_last_error("result must not be NULL");
    return FMOE_ERR_VALUE;
  }
  if (timeout_ns == 0 || timeout_ns > 100000000ull) {
    set_last_error("timeout_ns must be in (0, 1e8]");
    return FMOE_ERR_VALUE;
  }
  cudaStream_t stream = static_cast<cudaStream_t>(stream_ptr);
  wait_timeout_selftest_kernel<<<1, 64, 0, stream>>>(timeout_ns);
  cudaError_t e = cudaGetLastError();
  if (e == cudaSuccess) e = cudaStreamSynchronize(stream);
  if (e == cudaSuccess)
    e = cudaMemcpyFromSymbol(result, g_selftest_result, sizeof(unsigned long long) * 3);
  if (e != cudaSuccess) {
    set_last_error(std::string("self-test: ") + cudaGetErrorString(e));
    return FMOE_ERR_RUNTIME;
  }
  return FMOE_OK;
}
