// peer_sync.cu -- completion signal of the split-N output exchange.
//
// After a rank's scatter kernels have stored its output columns into every rank's buffer
// (and made them visible system-wide: each storing thread ends with a system-scope fence),
// one warp of this kernel, stream-ordered after them, raises this rank's flag in every
// rank's signal array to the call's epoch (release stores at system scope over NVLink) and
// waits until every rank's flag in this GPU's array has reached the epoch (acquire loads),
// so the kernels that follow on this rank's stream see the whole [M][N] output.  Flags are
// 64-bit and only grow, so arrays never need re-zeroing; every rank passes the same epoch
// sequence.  The wait is bounded by %globaltimer: a rank that never signals makes the others
// record QL_DEVERR_TIMEOUT in the backend's error word and return (the host then reports
// QLINEAR_ERR_TIMEOUT); no GPU waits on another kernel of its own.
#include "common.cuh"
#include "kernels.h"

namespace ql {

namespace {

__global__ void peer_signal_wait_kernel(PeerSignals s, unsigned long long epoch, unsigned *err,
                                        unsigned long long limit_ns) {
    const int lane = threadIdx.x;
    if (lane < s.world) {
        unsigned long long *flag = static_cast<unsigned long long *>(s.sig[lane]) + s.rank;
        asm volatile("st.release.sys.global.u64 [%0], %1;" ::"l"(flag), "l"(epoch) : "memory");
    }
    if (lane < s.world) {
        const unsigned long long *flag =
            static_cast<const unsigned long long *>(s.sig[s.rank]) + lane;
        const unsigned long long t0 = global_ns();
        while (true) {
            unsigned long long v;
            asm volatile("ld.acquire.sys.global.u64 %0, [%1];" : "=l"(v) : "l"(flag) : "memory");
            if (v >= epoch) break;
            if (global_ns() - t0 > limit_ns) {
                atomicOr(err, QL_DEVERR_TIMEOUT);
                break;
            }
            __nanosleep(64);
        }
    }
}

}  // namespace

cudaError_t launch_peer_signal_wait(const PeerSignals &s, unsigned long long epoch, unsigned *err,
                                    unsigned long long limit_ns, cudaStream_t stream) {
    if (s.world < 1 || s.world > kMaxOutputs || s.rank < 0 || s.rank >= s.world)
        return cudaErrorInvalidValue;
    peer_signal_wait_kernel<<<1, 32, 0, stream>>>(s, epoch, err, limit_ns);
    return cudaGetLastError();
}

}  // namespace ql
