// gemv.cu -- decode path (rows <= 8), one output buffer; the kernel is in gemv_impl.cuh.
#include "gemv_impl.cuh"

namespace ql {

bool gemv_fits(int rows, int Kp, int N, int bits, bool swiglu, int num_sms) {
    Plan pl;
    return plan(rows, Kp, N, bits, swiglu, num_sms, &pl);
}

bool gemv_can_fuse(const void *x, int type, long long ldx, int K) {
    const int vec = type == kF16 ? 8 : type == kF32 ? 4 : 0;
    return vec && K % vec == 0 && ldx % vec == 0 && (reinterpret_cast<uintptr_t>(x) & 15) == 0;
}

cudaError_t launch_gemv(const WeightView &w, const GemvInput &in, int rows, const OutputSet &out,
                        int out_type, long long ldc, bool swiglu, int num_sms, cudaStream_t stream) {
    if (out.count > 1)
        return launch_gemv_scatter(w, in, rows, out, out_type, ldc, swiglu, num_sms, stream);
    return launch_checked<false>(w, in, rows, out, out_type, ldc, swiglu, num_sms, stream);
}

}  // namespace ql
