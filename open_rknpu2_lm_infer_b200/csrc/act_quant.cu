// act_quant.cu -- dynamic per-token symmetric int8 activation quantisation.
//
// Restates, per row m of x [rows][K] (f32 or fp16 widened exactly to f32), the
// reference's quantiser (src/npu.rs:1099-1110, rk_npu_w4a8_quant in the un-vendored
// operator library):
//   amax  = max_k |x|          fmaxf ignores NaN like Rust's f32::max
//   scale = amax == 0 ? 1 : max(amax / 127, FLT_MIN)       IEEE division
//   inv   = 1 / scale                                        IEEE division
//   q     = clamp(round(x * inv), -127, 127)                 roundf: ties away from zero
//                                                            (rintf with QLINEAR_ROUND_EVEN)
//   NaN -> 0 (Rust `NaN as i32`), +-inf -> +-127.
// Writes int8 codes into a [rows][Kp] buffer (Kp = K rounded up to the 128-element
// k-block, the pad zeroed), the f32 scale per row and the i32 sum of the row's codes
// (used by the W4 epilogue, whose weights are stored offset by +8).
//
// Launched with programmatic stream serialization and a griddepcontrol.wait before any memory
// access, so its launch overlaps the tail of the preceding kernel (measured on B200: cfg0
// 26.8 -> 24.5 us per act-quant + GEMM call, the 36-layer prefill pass 4995 -> 4743 us).
// One CTA per row; the row is read once with 16-byte loads and held in registers (up to
// kCache chunks per thread; longer rows are re-read from L1/L2), the max is reduced with
// warp shuffles (max is order independent, so the result is exact), codes are written
// with 8-byte (fp16 input) or 4-byte (f32 input) stores.  HBM-bound: 2 or 4 bytes read
// and 1 byte written per element.
#include "common.cuh"
#include "kernels.h"


namespace ql {

namespace {

constexpr int kThreads = 256;
constexpr int kCache = 6;

// 16-byte vector of the input type; kept raw (4 registers) in the row cache and widened
// to f32 on use.
template <typename T>
struct Vec;
template <>
struct Vec<__half> {
    static constexpr int N = 8;
    __device__ static __forceinline__ void widen(const uint4 &raw, float (&v)[8]) {
        const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
        for (int i = 0; i < 4; i++) {
            float2 f = __half22float2(h[i]);
            v[2 * i] = f.x;
            v[2 * i + 1] = f.y;
        }
    }
};
template <>
struct Vec<float> {
    static constexpr int N = 4;
    __device__ static __forceinline__ void widen(const uint4 &raw, float (&v)[4]) {
        v[0] = __uint_as_float(raw.x); v[1] = __uint_as_float(raw.y);
        v[2] = __uint_as_float(raw.z); v[3] = __uint_as_float(raw.w);
    }
};

__device__ __forceinline__ float to_f32(float v) { return v; }
__device__ __forceinline__ float to_f32(__half v) { return __half2float(v); }

__device__ __forceinline__ float block_max(float v, float *red) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        v = l < (int)(blockDim.x >> 5) ? red[l] : 0.0f;
#pragma unroll
        for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
        if (l == 0) red[0] = v;
    }
    __syncthreads();
    return red[0];
}

__device__ __forceinline__ int block_sum(int v, int *red) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = v;
    __syncthreads();
    if (w == 0) {
        v = l < (int)(blockDim.x >> 5) ? red[l] : 0;
#pragma unroll
        for (int o = 16; o; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
        if (l == 0) red[0] = v;
    }
    __syncthreads();
    return red[0];
}

// Vectorised path: K % VEC == 0 and every row 16-byte aligned.
template <typename T>
__global__ void __launch_bounds__(kThreads) act_quant_vec_kernel(
    const T *__restrict__ x, long long ldx, int K, int Kp, int round_mode,
    int8_t *__restrict__ codes, float *__restrict__ scales, int32_t *__restrict__ rowsums,
    const float *__restrict__ amax_in, int early) {
    // launched with programmatic stream serialization: nothing is read or written before
    // the preceding kernel has completed
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (early) asm volatile("griddepcontrol.launch_dependents;");
    constexpr int V = Vec<T>::N;
    __shared__ float redf[32];
    __shared__ int redi[32];
    const long long m = blockIdx.x;
    const T *xr = x + m * ldx;
    int8_t *cr = codes + m * (long long)Kp;
    const int nchunks = K / V;

    const uint4 *xv = reinterpret_cast<const uint4 *>(xr);
    uint4 raw[kCache];
    float amax = 0.0f;
#pragma unroll
    for (int i = 0; i < kCache; i++) {
        const int c = threadIdx.x + i * kThreads;
        if (c < nchunks) {
            raw[i] = __ldg(xv + c);
            float t[V];
            Vec<T>::widen(raw[i], t);
#pragma unroll
            for (int e = 0; e < V; e++) amax = fmaxf(amax, fabsf(t[e]));
        }
    }
    for (int c = threadIdx.x + kCache * kThreads; c < nchunks; c += kThreads) {
        float t[V];
        Vec<T>::widen(__ldg(xv + c), t);
#pragma unroll
        for (int e = 0; e < V; e++) amax = fmaxf(amax, fabsf(t[e]));
    }
    // amax_in: the row's max |x| given by the caller (the max over every rank's slice of a
    // K-split row), so the codes are those of the whole row
    amax = amax_in ? amax_in[m] : block_max(amax, redf);
    float scale, inv;
    a8_row_scale(amax, scale, inv);

    int sum = 0;
    auto emit = [&](int c, const uint4 &rv) {
        float t[V];
        Vec<T>::widen(rv, t);
        uint32_t w[V / 4];
#pragma unroll
        for (int g = 0; g < V / 4; g++) {
            uint32_t packed = 0;
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int q = a8_code(t[4 * g + e], inv, round_mode);
                sum += q;
                packed |= (uint32_t)(q & 0xff) << (8 * e);
            }
            w[g] = packed;
        }
        if constexpr (V == 8)
            *reinterpret_cast<uint2 *>(cr + (long long)c * 8) = make_uint2(w[0], w[1]);
        else
            *reinterpret_cast<uint32_t *>(cr + (long long)c * 4) = w[0];
    };
#pragma unroll
    for (int i = 0; i < kCache; i++) {
        const int c = threadIdx.x + i * kThreads;
        if (c < nchunks) emit(c, raw[i]);
    }
    for (int c = threadIdx.x + kCache * kThreads; c < nchunks; c += kThreads) emit(c, __ldg(xv + c));
    for (int k = K + threadIdx.x; k < Kp; k += kThreads) cr[k] = 0;
    sum = block_sum(sum, redi);
    if (threadIdx.x == 0) {
        scales[m] = scale;
        if (rowsums) rowsums[m] = sum;
    }
    // Let a dependent kernel launched with programmatic stream serialization (the GEMM /
    // GEMV) launch; it waits (griddepcontrol.wait) for this grid's completion and memory
    // before reading what this kernel wrote.  The dependent launches only once every CTA of
    // this grid has issued the instruction or exited, so no dependent CTA can take an SM a
    // row still waiting to be scheduled needs.  With `early` (the whole grid resident at
    // once) it was issued at the start, so the dependent's launch, prologue and first weight
    // loads overlap the quantisation; larger grids keep it here, at the end.
    if (!early) asm volatile("griddepcontrol.launch_dependents;");
}

// Scalar path for any K / alignment (re-reads the row for the second pass).
template <typename T>
__global__ void __launch_bounds__(kThreads) act_quant_scalar_kernel(
    const T *__restrict__ x, long long ldx, int K, int Kp, int round_mode,
    int8_t *__restrict__ codes, float *__restrict__ scales, int32_t *__restrict__ rowsums,
    const float *__restrict__ amax_in, int early) {
    asm volatile("griddepcontrol.wait;" ::: "memory");
    if (early) asm volatile("griddepcontrol.launch_dependents;");
    __shared__ float redf[32];
    __shared__ int redi[32];
    const long long m = blockIdx.x;
    const T *xr = x + m * ldx;
    int8_t *cr = codes + m * (long long)Kp;
    float amax = 0.0f;
    if (amax_in) {
        amax = amax_in[m];
    } else {
        for (int k = threadIdx.x; k < K; k += kThreads) amax = fmaxf(amax, fabsf(to_f32(xr[k])));
        amax = block_max(amax, redf);
    }
    float scale, inv;
    a8_row_scale(amax, scale, inv);
    int sum = 0;
    for (int k = threadIdx.x; k < K; k += kThreads) {
        const int q = a8_code(to_f32(xr[k]), inv, round_mode);
        sum += q;
        cr[k] = (int8_t)q;
    }
    for (int k = K + threadIdx.x; k < Kp; k += kThreads) cr[k] = 0;
    sum = block_sum(sum, redi);
    if (threadIdx.x == 0) {
        scales[m] = scale;
        if (rowsums) rowsums[m] = sum;
    }
    if (!early) asm volatile("griddepcontrol.launch_dependents;");
}

// CTAs of `kern` the current device holds at once (0 if unknown); cached per device.
template <typename K>
int resident_ctas(K kern, int (&cache)[64]) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    if (cache[dev] == 0) {
        int per_sm = 0, sms = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, kThreads, 0) !=
                cudaSuccess ||
            cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess)
            return 0;
        cache[dev] = per_sm * sms > 0 ? per_sm * sms : -1;
    }
    return cache[dev] > 0 ? cache[dev] : 0;
}

// A launch with programmatic stream serialization (the kernel waits with griddepcontrol.wait
// before it touches memory): its launch overlaps the tail of the preceding kernel.
template <typename Kern, typename... Args>
cudaError_t launch_pdl(Kern kern, int rows, cudaStream_t stream, Args... args) {
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(rows);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = 0;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, args...);
}

template <typename T>
cudaError_t launch_typed(const T *x, long long ldx, int rows, int K, int Kp, int round_mode,
                         int8_t *codes, float *scales, int32_t *rowsums, cudaStream_t stream,
                         const float *amax_in) {
    constexpr int V = Vec<T>::N;
    const bool vec = (K % V == 0) && (ldx % V == 0) &&
                     ((reinterpret_cast<uintptr_t>(x) & 15) == 0);
    // A grid no larger than the resident capacity triggers the dependent launch at its start
    // (see the kernels).
    static int cap_vec[64] = {0}, cap_scalar[64] = {0};
    if (vec) {
        const int early = rows <= resident_ctas(act_quant_vec_kernel<T>, cap_vec) ? 1 : 0;
        return launch_pdl(act_quant_vec_kernel<T>, rows, stream, x, ldx, K, Kp, round_mode,
                          codes, scales, rowsums, amax_in, early);
    } else {
        const int early = rows <= resident_ctas(act_quant_scalar_kernel<T>, cap_scalar) ? 1 : 0;
        return launch_pdl(act_quant_scalar_kernel<T>, rows, stream, x, ldx, K, Kp, round_mode,
                          codes, scales, rowsums, amax_in, early);
    }
    return cudaGetLastError();
}

}  // namespace

cudaError_t launch_act_quant(const void *x, int x_type, long long ldx, int rows, int K, int Kp,
                             int round_mode, int8_t *codes, float *scales, int32_t *rowsums,
                             cudaStream_t stream, const float *amax_in) {
    if (rows <= 0) return cudaSuccess;
    if (x_type == kF16)
        return launch_typed(static_cast<const __half *>(x), ldx, rows, K, Kp, round_mode, codes,
                            scales, rowsums, stream, amax_in);
    return launch_typed(static_cast<const float *>(x), ldx, rows, K, Kp, round_mode, codes, scales,
                        rowsums, stream, amax_in);
}

}  // namespace ql
