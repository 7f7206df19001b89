// Failure-detection self-test: the library's bounded mbarrier wait run against a barrier that nothing ever completes.
// Every wait in the pipelined kernels (producer ring slots, consumer data, tensor-memory hand-offs) is this wait with a
// 2 s limit: on expiry the kernel records a bit in the workspace error word, leaves its loops, drains its own copies
// and returns, so a stalled pipeline surfaces as GLMX_E_DEVICE from glmx_check instead of a hung GPU. The probe below
// exercises exactly that path with a short limit, without any fault.
#include <cuda_runtime.h>

#include "glmx.h"
#include "glmx_common.cuh"
#include "glmx_internal.h"

namespace glmx {

namespace {

__global__ void bounded_wait_probe(uint64_t timeout_ns, int* flag)
{
    __shared__ uint64_t bar;
    if (threadIdx.x == 0)
    {
        mbar_init(&bar, 1);
        fence_barrier_init();
    }
    __syncthreads();
    // one arrival is expected and none comes: phase 0 never completes
    const bool ok = mbar_wait_bounded_ns(&bar, 0, timeout_ns);
    if (!ok && threadIdx.x == 0) atomicOr(flag, ERR_TIMEOUT_FULL);
}

}  // namespace

}  // namespace glmx

extern "C" int glmx_selftest_bounded_wait(int timeout_us, int* flag, void* stream)
{
    if (timeout_us < 1 || timeout_us > 10000000 || !flag)
    {
        glmx::set_error("glmx_selftest_bounded_wait: timeout_us in [1, 1e7] and a device flag are required");
        return GLMX_E_ARG;
    }
    glmx::bounded_wait_probe<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>((uint64_t) timeout_us * 1000u, flag);
    const cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess)
    {
        glmx::set_error(std::string("glmx_selftest_bounded_wait: launch: ") + cudaGetErrorString(e));
        return GLMX_E_CUDA;
    }
    return GLMX_OK;
}
