// swiglu.cu -- SiLU-gated product over a gate/up projection output.
//
// out[m][j] = silu(y[m][j]) * y[m][N/2 + j], silu(g) = g / (1 + exp(-g)), computed in f32
// from the exact f32 dequantised values (the expectation of src/npu.rs:1202-1208; the
// reference's production CPU path, src/model/cpu.rs:119-152, evaluates exp in f64 for
// |g| <= 80 -- the difference is within the reference's own 3e-5 tolerance).  Used after
// the tensor-core GEMM; the decode GEMV fuses the same arithmetic into its epilogue.
#include "common.cuh"
#include "kernels.h"

namespace ql {

namespace {

template <typename OutT>
__global__ void swiglu_kernel(const float *__restrict__ y, int rows, int N,
                              OutT *__restrict__ out, long long ldc) {
    const int h = N / 2;
    const long long total = (long long)rows * h;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long m = i / h;
        const int j = (int)(i % h);
        const float g = y[m * N + j];
        const float u = y[m * N + h + j];
        const float v = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
        out[m * ldc + j] = OutCvt<OutT>::from(v);
    }
}

}  // namespace

cudaError_t launch_swiglu(const float *y, int rows, int N, void *out, int out_type, long long ldc,
                          cudaStream_t stream) {
    const long long total = (long long)rows * (N / 2);
    int grid = (int)((total + 255) / 256);
    if (grid > 148 * 16) grid = 148 * 16;
    if (grid < 1) grid = 1;
    if (out_type == kF16)
        swiglu_kernel<__half><<<grid, 256, 0, stream>>>(y, rows, N, static_cast<__half *>(out), ldc);
    else if (out_type == kF32)
        swiglu_kernel<float><<<grid, 256, 0, stream>>>(y, rows, N, static_cast<float *>(out), ldc);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace ql
