// selftest.cu -- exercises the kernels' failure path on a GPU without a fault: a wait that
// nothing will satisfy gives up after a short limit, records the timeout in the backend's
// device error word and returns, exactly as a stuck pipeline stage of the GEMM would; the
// host then reports QLINEAR_ERR_TIMEOUT and the context stays usable.
#include "../../include/qlinear.h"
#include "common.cuh"
#include "kernels.h"

namespace ql {

namespace {

// One warp waits on an mbarrier (one expected arrival) that nobody arrives on.
__global__ void wait_selftest_kernel(unsigned *err, unsigned long long limit_ns) {
    __shared__ __align__(8) uint64_t bar;
    __shared__ int abort_flag_s;
    if (threadIdx.x == 0) {
        mbar_init(&bar, 1);
        abort_flag_s = 0;
        mbar_fence_init();
    }
    __syncwarp();
    volatile int *abort_flag = &abort_flag_s;
    mbar_wait(&bar, 0, err, abort_flag, limit_ns);
}

}  // namespace

cudaError_t launch_wait_selftest(unsigned *err, unsigned long long limit_ns, cudaStream_t stream) {
    wait_selftest_kernel<<<1, 32, 0, stream>>>(err, limit_ns);
    return cudaGetLastError();
}

}  // namespace ql
