// gemv_scatter.cu -- the decode GEMV of the split-N exchange: every output element is stored
// to this GPU's buffer and to the peers' (CUDA IPC mappings), then made visible system-wide
// at the kernel's end.  The kernel is in gemv_impl.cuh.
#include "gemv_impl.cuh"

namespace ql {

cudaError_t launch_gemv_scatter(const WeightView &w, const GemvInput &in, int rows,
                                const OutputSet &out, int out_type, long long ldc, bool swiglu,
                                int num_sms, cudaStream_t stream) {
    return launch_checked<true>(w, in, rows, out, out_type, ldc, swiglu, num_sms, stream);
}

}  // namespace ql
