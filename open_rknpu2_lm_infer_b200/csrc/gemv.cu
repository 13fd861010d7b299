// gemv.cu -- decode path (rows <= 8): stream the packed weights from HBM once.
//
// acc[m][n] = sum_k q[m][k] * w[k][n] exactly in int32 (src/npu.rs:1111-1116), then
// y = (f32(acc) * s_a[m]) * s_w[n] (src/npu.rs:1117), written as f32 / fp16 / raw i32;
// with swiglu, out[m][j] = silu(y[m][j]) * y[m][N/2 + j] (src/npu.rs:1202-1208).
//
// Work split: one warp owns ROWS weight rows (output channels) at a time; its 32 lanes
// walk K in 16-byte chunks (16 W8 codes or 32 W4 codes per chunk), so every warp-wide
// load is 512 contiguous bytes of one weight row.  Two chunks per row are loaded before
// any is consumed (ROWS*2 16-byte loads in flight per lane).  The activation codes of the
// call (rows x Kp int8) are staged once per CTA in shared memory.  Products use dp4a
// (s8 x s8 for W8, u8 x s8 for W4's offset-binary nibbles, corrected by 8*sum(q) in the
// epilogue).  The ROWS x MT partial sums of a lane are reduced across the warp with a
// halving butterfly (ROWS*MT - 1 + 5 - log2(ROWS*MT) shuffles instead of 5 per value).
#include "common.cuh"
#include "kernels.h"

namespace ql {

namespace {

constexpr int kWarps = 8;
constexpr int kThreads = kWarps * 32;

// Reduce V = 2^p values per lane across the warp; afterwards lane l holds the full sum of
// value index l / (32 / V) in v[0].
template <int V>
__device__ __forceinline__ void warp_reduce_spread(int (&v)[V], int lane) {
    int off = 16;
#pragma unroll
    for (int n = V; n > 1; n >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; i++) {
            const int send = upper ? v[i] : v[i + n / 2];
            const int keep = upper ? v[i + n / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
        off >>= 1;
    }
    for (; off >= 1; off >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
}

template <typename OutT>
__device__ __forceinline__ void store_out(OutT *p, float y) { *p = OutCvt<OutT>::from(y); }

// BITS: 4/8.  MT: activation rows held (>= rows of the call).  ROWS: weight rows per warp
// task (with SWIGLU the first ROWS/2 are gate rows n, the rest their up rows N/2 + n).
template <int BITS, int MT, int ROWS, bool SWIGLU, typename OutT>
__global__ void __launch_bounds__(kThreads) gemv_kernel(
    const uint8_t *__restrict__ wq, const float *__restrict__ wscale, int N, int Np, int Kp,
    const int8_t *__restrict__ codes, const float *__restrict__ ascale,
    const int32_t *__restrict__ rowsum, int M, OutT *__restrict__ out, long long ldc) {
    extern __shared__ __align__(16) uint8_t xs[];  // [MT][Kp] activation codes
    constexpr int V = ROWS * MT;
    static_assert(V <= 32 && (V & (V - 1)) == 0, "ROWS*MT must be a power of two <= 32");
    constexpr int CH = SWIGLU ? ROWS / 2 : ROWS;  // output channels per task

    // Stage the activation codes (rows >= M are zero).
    {
        const int n16 = MT * Kp / 16;
        for (int i = threadIdx.x; i < n16; i += kThreads) {
            const int m = (i * 16) / Kp;
            uint4 v = make_uint4(0, 0, 0, 0);
            if (m < M) v = *reinterpret_cast<const uint4 *>(codes + (long long)i * 16);
            reinterpret_cast<uint4 *>(xs)[i] = v;
        }
    }
    __syncthreads();

    const int lane = threadIdx.x & 31;
    const int warp = threadIdx.x >> 5;
    const int out_width = SWIGLU ? N / 2 : N;
    const int tasks = (out_width + CH - 1) / CH;
    const long long row_bytes = BITS == 8 ? Kp : Kp / 2;
    const int nchunks = (int)(row_bytes / 16);

    for (int task = blockIdx.x * kWarps + warp; task < tasks; task += gridDim.x * kWarps) {
        const int c0 = task * CH;
        const uint8_t *wrow[ROWS];
        int nrow[ROWS];
#pragma unroll
        for (int r = 0; r < ROWS; r++) {
            int n = SWIGLU ? (r < CH ? c0 + r : N / 2 + c0 + (r - CH)) : c0 + r;
            nrow[r] = n;
            if (n >= Np) n = 0;  // keep the load in bounds; the result is discarded
            wrow[r] = wq + (long long)n * row_bytes;
        }
        int acc[V];
#pragma unroll
        for (int i = 0; i < V; i++) acc[i] = 0;

        for (int j0 = lane; j0 < nchunks; j0 += 64) {
            uint4 w[2][ROWS];
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int j = j0 + 32 * u;
#pragma unroll
                for (int r = 0; r < ROWS; r++)
                    w[u][r] = j < nchunks ? ldg_stream(wrow[r] + (long long)j * 16)
                                          : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int j = j0 + 32 * u;
                if (j >= nchunks) break;
                if constexpr (BITS == 8) {
#pragma unroll
                    for (int m = 0; m < MT; m++) {
                        const uint4 x = *reinterpret_cast<const uint4 *>(xs + m * Kp + j * 16);
#pragma unroll
                        for (int r = 0; r < ROWS; r++) {
                            int a = acc[r * MT + m];
                            a = dp4a_ss(w[u][r].x, x.x, a);
                            a = dp4a_ss(w[u][r].y, x.y, a);
                            a = dp4a_ss(w[u][r].z, x.z, a);
                            a = dp4a_ss(w[u][r].w, x.w, a);
                            acc[r * MT + m] = a;
                        }
                    }
                } else {
                    // 16 packed bytes = 32 codes k = 32j .. 32j+31; word p covers 8 codes:
                    // low nibbles -> k 8p..8p+3, high nibbles -> k 8p+4..8p+7.
                    uint32_t lo[ROWS][4], hi[ROWS][4];
#pragma unroll
                    for (int r = 0; r < ROWS; r++) {
                        const uint32_t p4[4] = {w[u][r].x, w[u][r].y, w[u][r].z, w[u][r].w};
#pragma unroll
                        for (int p = 0; p < 4; p++) {
                            lo[r][p] = p4[p] & 0x0F0F0F0Fu;
                            hi[r][p] = (p4[p] >> 4) & 0x0F0F0F0Fu;
                        }
                    }
#pragma unroll
                    for (int m = 0; m < MT; m++) {
                        const uint4 xa = *reinterpret_cast<const uint4 *>(xs + m * Kp + j * 32);
                        const uint4 xb = *reinterpret_cast<const uint4 *>(xs + m * Kp + j * 32 + 16);
                        const uint32_t x8[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
#pragma unroll
                        for (int r = 0; r < ROWS; r++) {
                            int a = acc[r * MT + m];
#pragma unroll
                            for (int p = 0; p < 4; p++) {
                                a = dp4a_us(lo[r][p], x8[2 * p], a);
                                a = dp4a_us(hi[r][p], x8[2 * p + 1], a);
                            }
                            acc[r * MT + m] = a;
                        }
                    }
                }
            }
        }

        warp_reduce_spread<V>(acc, lane);
        const int idx = lane / (32 / V);  // value index held by this lane
        const int r = idx / MT, m = idx % MT;
        int total = acc[0];
        if (BITS == 4) total -= 8 * (m < M ? rowsum[m] : 0);
        const bool leader = (lane % (32 / V)) == 0;
        if constexpr (SWIGLU) {
            // gate value (r < CH) pairs with the up value at index idx + CH*MT
            const int partner = (idx + CH * MT) * (32 / V);
            const int up_total = __shfl_sync(0xffffffffu, total, partner & 31);
            if (leader && r < CH && m < M) {
                const int n = nrow[0] + r;  // gate channel c0 + r
                if (n < N / 2) {
                    const float sa = ascale[m];
                    const float g = __fmul_rn(__fmul_rn(__int2float_rn(total), sa), wscale[n]);
                    const float up = __fmul_rn(__fmul_rn(__int2float_rn(up_total), sa),
                                               wscale[N / 2 + n]);
                    const float y = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), up);
                    store_out(out + (long long)m * ldc + n, y);
                }
            }
        } else {
            if (leader && m < M) {
                const int n = c0 + r;
                if (n < N) {
                    if constexpr (sizeof(OutT) == 4 && !std::is_same<OutT, float>::value) {
                        out[(long long)m * ldc + n] = total;
                    } else {
                        const float y = __fmul_rn(__fmul_rn(__int2float_rn(total), ascale[m]),
                                                  wscale[n]);
                        store_out(out + (long long)m * ldc + n, y);
                    }
                }
            }
        }
    }
}

template <int BITS, int MT, int ROWS, bool SWIGLU, typename OutT>
cudaError_t launch_t(const WeightView &w, const ActView &a, int rows, OutT *out, long long ldc,
                     int num_sms, cudaStream_t stream) {
    constexpr int CH = SWIGLU ? ROWS / 2 : ROWS;
    const int out_width = SWIGLU ? w.N / 2 : w.N;
    const int tasks = (out_width + CH - 1) / CH;
    int grid = (tasks + kWarps - 1) / kWarps;
    const int cap = num_sms * 4;
    if (grid > cap) grid = cap;
    if (grid < 1) grid = 1;
    const size_t smem = (size_t)MT * w.Kp;
    auto kern = gemv_kernel<BITS, MT, ROWS, SWIGLU, OutT>;
    static int configured[64] = {0};  // per device: raise the opt-in limit once
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        cudaError_t e =
            cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    kern<<<grid, kThreads, smem, stream>>>(w.w, w.scales, w.N, w.Np, w.Kp, a.codes, a.scales,
                                           a.rowsums, rows, out, ldc);
    return cudaGetLastError();
}

template <int BITS, bool SWIGLU, typename OutT>
cudaError_t launch_mt(const WeightView &w, const ActView &a, int rows, OutT *out, long long ldc,
                      int num_sms, cudaStream_t stream) {
    if (rows <= 1) return launch_t<BITS, 1, 8, SWIGLU, OutT>(w, a, rows, out, ldc, num_sms, stream);
    if (rows <= 2) return launch_t<BITS, 2, 8, SWIGLU, OutT>(w, a, rows, out, ldc, num_sms, stream);
    if (rows <= 4) return launch_t<BITS, 4, 8, SWIGLU, OutT>(w, a, rows, out, ldc, num_sms, stream);
    return launch_t<BITS, 8, 4, SWIGLU, OutT>(w, a, rows, out, ldc, num_sms, stream);
}

template <int BITS>
cudaError_t launch_bits(const WeightView &w, const ActView &a, int rows, void *out, int out_type,
                        long long ldc, bool swiglu, int num_sms, cudaStream_t stream) {
    if (swiglu) {
        if (out_type == kF16)
            return launch_mt<BITS, true, __half>(w, a, rows, static_cast<__half *>(out), ldc,
                                                 num_sms, stream);
        if (out_type == kF32)
            return launch_mt<BITS, true, float>(w, a, rows, static_cast<float *>(out), ldc,
                                                num_sms, stream);
        return cudaErrorInvalidValue;
    }
    if (out_type == kF16)
        return launch_mt<BITS, false, __half>(w, a, rows, static_cast<__half *>(out), ldc, num_sms,
                                              stream);
    if (out_type == kF32)
        return launch_mt<BITS, false, float>(w, a, rows, static_cast<float *>(out), ldc, num_sms,
                                             stream);
    return launch_mt<BITS, false, int32_t>(w, a, rows, static_cast<int32_t *>(out), ldc, num_sms,
                                           stream);
}

}  // namespace

cudaError_t launch_gemv(const WeightView &w, const ActView &a, int rows, void *out, int out_type,
                        long long ldc, bool swiglu, int num_sms, cudaStream_t stream) {
    if (rows < 1 || rows > 8) return cudaErrorInvalidValue;
    if (w.bits == 8) return launch_bits<8>(w, a, rows, out, out_type, ldc, swiglu, num_sms, stream);
    return launch_bits<4>(w, a, rows, out, out_type, ldc, swiglu, num_sms, stream);
}

}  // namespace ql
