// selftest.cu - failure detection without a GPU fault.
//
// Every wait inside the library's kernels is bounded: if the awaited phase never
// completes (a lost TMA transaction, a producer that died), the waiting thread
// records SV_DEVERR_TIMEOUT in the error word and the kernel unwinds instead of
// hanging the GPU.  sv_selftest_wait_timeout runs that path on purpose: its
// kernel waits on an mbarrier nothing will ever complete, with a short limit,
// so a test can check that the wait expires, the error bit reaches the host and
// the context stays usable.
#include "common.cuh"
#include "internal.hpp"

namespace svkv {
namespace {

__global__ void selftest_wait_kernel(int* err, uint64_t limit_ns, int* reached_end) {
    __shared__ uint64_t bar;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);             // expects one arrival that never comes
        fence_barrier_init();
    }
    __syncthreads();
    const bool ok = mbar_wait_limit(&bar, 0, err, limit_ns);
    __syncthreads();
    if (threadIdx.x == 0 && reached_end) *reached_end = ok ? 2 : 1;
}

}  // namespace
}  // namespace svkv

extern "C" int sv_selftest_wait_timeout(int* err_dev, int* reached_end_dev, unsigned limit_us, void* stream) {
    if (!err_dev || limit_us == 0 || limit_us > 1000000u) return SV_ERR_INVALID;
    svkv::selftest_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(
        err_dev, (uint64_t)limit_us * 1000ull, reached_end_dev);
    return cudaGetLastError() == cudaSuccess ? SV_OK : SV_ERR_CUDA;
}
