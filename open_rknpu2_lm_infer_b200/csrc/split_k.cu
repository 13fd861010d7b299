// split_k.cu -- the pieces a K-split (row-parallel) linear needs around the usual kernels.
//
// When the K dimension of a linear is split over ranks (each holds the weight rows of its
// K slice and the matching slice of every activation row), the reference's arithmetic
// (src/npu.rs:1099-1117) is kept exactly by: the row max |x| of each slice (row_amax), the
// max over the slices (a collective of the caller's), every slice quantised with the scale
// of that whole-row max (act_quant with amax_in: the codes of the whole row), the int32
// partial accumulators of the slices summed (exact), and one dequant with the whole-row
// scale (dequant below).  The result equals the unsplit linear bit for bit.
#include "common.cuh"
#include "kernels.h"

namespace ql {

namespace {

constexpr int kThreads = 256;

template <typename T>
__device__ __forceinline__ float as_f32(T v) { return static_cast<float>(v); }
template <>
__device__ __forceinline__ float as_f32<__half>(__half v) { return __half2float(v); }

// One CTA per row; fmaxf ignores NaN (Rust f32::max), max is order independent: exact.
template <typename T>
__global__ void __launch_bounds__(kThreads)
    row_amax_kernel(const T *__restrict__ x, long long ldx, int K, float *__restrict__ amax) {
    __shared__ float red[kThreads / 32];
    const T *xr = x + (long long)blockIdx.x * ldx;
    float v = 0.0f;
    for (int k = threadIdx.x; k < K; k += kThreads) v = fmaxf(v, fabsf(as_f32(xr[k])));
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = v;
    __syncthreads();
    if (threadIdx.x == 0) {
        float a = 0.0f;
        for (int w = 0; w < kThreads / 32; w++) a = fmaxf(a, red[w]);
        amax[blockIdx.x] = a;
    }
}

template <typename OutT>
__global__ void dequant_kernel(const int32_t *__restrict__ acc, long long lda,
                               const float *__restrict__ amax, const float *__restrict__ wscale,
                               int rows, int N, OutT *__restrict__ out, long long ldc) {
    const long long total = (long long)rows * N;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const long long m = i / N;
        const int n = (int)(i - m * N);
        float sa, inv;
        a8_row_scale(amax[m], sa, inv);
        const float y = __fmul_rn(__fmul_rn(__int2float_rn(acc[m * lda + n]), sa), wscale[n]);
        out[m * ldc + n] = OutCvt<OutT>::from(y);
    }
}

}  // namespace

cudaError_t launch_row_amax(const void *x, int x_type, long long ldx, int rows, int K, float *amax,
                            cudaStream_t stream) {
    if (rows < 1 || K < 1 || !x || !amax) return cudaErrorInvalidValue;
    if (x_type == kF16)
        row_amax_kernel<__half><<<rows, kThreads, 0, stream>>>(static_cast<const __half *>(x), ldx,
                                                                K, amax);
    else if (x_type == kF32)
        row_amax_kernel<float><<<rows, kThreads, 0, stream>>>(static_cast<const float *>(x), ldx,
                                                               K, amax);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

cudaError_t launch_dequant(const int32_t *acc, long long lda, const float *amax,
                           const float *wscale, int rows, int N, void *out, int out_type,
                           long long ldc, int num_sms, cudaStream_t stream) {
    if (rows < 1 || N < 1 || !acc || !amax || !wscale || !out || lda < N || ldc < N)
        return cudaErrorInvalidValue;
    const long long total = (long long)rows * N;
    long long grid = (total + kThreads - 1) / kThreads;
    if (grid > (long long)num_sms * 8) grid = (long long)num_sms * 8;
    if (out_type == kF16)
        dequant_kernel<__half><<<(int)grid, kThreads, 0, stream>>>(
            acc, lda, amax, wscale, rows, N, static_cast<__half *>(out), ldc);
    else if (out_type == kF32)
        dequant_kernel<float><<<(int)grid, kThreads, 0, stream>>>(
            acc, lda, amax, wscale, rows, N, static_cast<float *>(out), ldc);
    else
        return cudaErrorInvalidValue;
    return cudaGetLastError();
}

}  // namespace ql
