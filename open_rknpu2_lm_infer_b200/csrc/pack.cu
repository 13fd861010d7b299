// pack.cu -- weight upload: QuantMatrix / checkpoint layouts -> the device layout.
//
// The reference hands its operator library the QuantMatrix codes int8 [K][N]
// (src/npu.rs:112-118, :1115), produced from the checkpoint by transposing
// compressed-tensors storage [N][K] (src/model/checkpoint.rs:237-251, :352-378).  The GPU
// kernels want K contiguous per output channel, so both entry points end in the same
// device layout (kernels.h):
//   W8: int8 [Np][Kp];
//   W4: [Np][Kp/2] bytes, word w of row n = 8 codes k = 8w..8w+7, byte j = u(8w+j) |
//       u(8w+j+4) << 4, u = code + 8 (the checkpoint's own offset-binary nibble, so the
//       unpack is two masks and no sign extension; the GEMM epilogue subtracts
//       8 * sum_k q[m,k]).
// Padding (k >= K, n >= N) holds code 0.
#include "common.cuh"
#include "kernels.h"

namespace ql {

namespace {

constexpr int T = 64;  // tile edge (k and n)

__device__ __forceinline__ uint32_t u4(int8_t c) { return (uint32_t)(c + 8) & 0xFu; }

// One CTA transposes a 64(k) x 64(n) tile of codes [K][n_total] (columns n_begin + ...).
template <int BITS>
__global__ void __launch_bounds__(256) pack_kn_kernel(const int8_t *__restrict__ src, int K,
                                                      int n_total, int n_begin, int N, int Kp,
                                                      uint8_t *__restrict__ dst) {
    __shared__ int8_t tile[T][T + 4];
    const int k0 = blockIdx.x * T, n0 = blockIdx.y * T;
    for (int i = threadIdx.x; i < T * T; i += blockDim.x) {
        const int kk = i / T, nn = i % T;
        const int k = k0 + kk, n = n0 + nn;
        tile[kk][nn] = (k < K && n < N) ? src[(long long)k * n_total + n_begin + n] : (int8_t)0;
    }
    __syncthreads();
    const int t = threadIdx.x;
    const int nn = t >> 2, part = t & 3;
    const long long n = n0 + nn;
    if constexpr (BITS == 8) {
        uint32_t w[4];
#pragma unroll
        for (int q = 0; q < 4; q++) {
            uint32_t v = 0;
#pragma unroll
            for (int b = 0; b < 4; b++)
                v |= (uint32_t)(uint8_t)tile[part * 16 + q * 4 + b][nn] << (8 * b);
            w[q] = v;
        }
        *reinterpret_cast<uint4 *>(dst + n * Kp + k0 + part * 16) = make_uint4(w[0], w[1], w[2], w[3]);
    } else {
        uint32_t w[2];
#pragma unroll
        for (int q = 0; q < 2; q++) {
            const int kb = part * 16 + q * 8;  // first k of this word within the tile
            uint32_t v = 0;
#pragma unroll
            for (int j = 0; j < 4; j++) {
                const uint32_t lo = u4(tile[kb + j][nn]), hi = u4(tile[kb + j + 4][nn]);
                v |= (lo | (hi << 4)) << (8 * j);
            }
            w[q] = v;
        }
        *reinterpret_cast<uint2 *>(dst + n * (Kp / 2) + k0 / 2 + part * 8) = make_uint2(w[0], w[1]);
    }
}

// W4 from compressed-tensors weight_packed: int32 [N][ceil(K/8)], nibble j of word w is
// k = 8w + j stored as code + 8 (src/model/checkpoint.rs:352-371).
__global__ void pack_ckpt_w4_kernel(const uint32_t *__restrict__ src, int K, int N, int Kp, int Np,
                                    uint32_t *__restrict__ dst) {
    const int words = Kp / 8;
    const long long total = (long long)Np * words;
    const int kw = (K + 7) / 8;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int n = (int)(i / words), w = (int)(i % words);
        uint32_t u[8];
        const uint32_t cw = (n < N && w < kw) ? src[(long long)n * kw + w] : 0u;
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const int k = 8 * w + j;
            u[j] = (n < N && k < K) ? ((cw >> (4 * j)) & 0xFu) : 8u;
        }
        uint32_t v = 0;
#pragma unroll
        for (int j = 0; j < 4; j++) v |= (u[j] | (u[j + 4] << 4)) << (8 * j);
        dst[i] = v;
    }
}

// W8 from compressed-tensors int-quantized weight: int8 [N][K] (src/model/checkpoint.rs:372-378).
__global__ void pack_ckpt_w8_kernel(const int8_t *__restrict__ src, int K, int N, int Kp, int Np,
                                    int8_t *__restrict__ dst) {
    const long long total = (long long)Np * Kp;
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < total;
         i += (long long)gridDim.x * blockDim.x) {
        const int n = (int)(i / Kp), k = (int)(i % Kp);
        dst[i] = (n < N && k < K) ? src[(long long)n * K + k] : (int8_t)0;
    }
}

// int8 expansion of the device W4 layout: out [Np][Kp] int8 from packed [Np][Kp/2]
// (word w byte j = u(8w+j) | u(8w+j+4) << 4, code = u - 8).  One thread per packed word.
__global__ void expand_w4_kernel(const uint32_t *__restrict__ packed, long long words,
                                 uint32_t *__restrict__ out) {
    for (long long i = blockIdx.x * (long long)blockDim.x + threadIdx.x; i < words;
         i += (long long)gridDim.x * blockDim.x) {
        const uint32_t w = packed[i];
        // bytes of lo: codes 8w..8w+3 (u), hi: 8w+4..8w+7; u - 8 per byte without borrows
        const uint32_t lo = ((w & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
        const uint32_t hi = (((w >> 4) & 0x0F0F0F0Fu) + 0x78787878u) ^ 0x80808080u;
        out[2 * i] = lo;
        out[2 * i + 1] = hi;
    }
}

}  // namespace

cudaError_t launch_expand_w4(const WeightView &w4, uint8_t *dst, cudaStream_t stream) {
    const long long words = (long long)w4.Np * (w4.Kp / 8);
    expand_w4_kernel<<<1024, 256, 0, stream>>>(reinterpret_cast<const uint32_t *>(w4.w), words,
                                              reinterpret_cast<uint32_t *>(dst));
    return cudaGetLastError();
}

cudaError_t launch_pack_from_kn(const int8_t *codes_kn, int K, int n_total, int n_begin,
                                const WeightView &w, uint8_t *dst, cudaStream_t stream) {
    dim3 grid(w.Kp / T, w.Np / T);
    if (w.bits == 8)
        pack_kn_kernel<8><<<grid, 256, 0, stream>>>(codes_kn, K, n_total, n_begin, w.N, w.Kp, dst);
    else
        pack_kn_kernel<4><<<grid, 256, 0, stream>>>(codes_kn, K, n_total, n_begin, w.N, w.Kp, dst);
    return cudaGetLastError();
}

cudaError_t launch_pack_from_checkpoint(const void *storage, const WeightView &w, uint8_t *dst,
                                        cudaStream_t stream) {
    if (w.bits == 4)
        pack_ckpt_w4_kernel<<<1024, 256, 0, stream>>>(static_cast<const uint32_t *>(storage), w.K,
                                                      w.N, w.Kp, w.Np,
                                                      reinterpret_cast<uint32_t *>(dst));
    else
        pack_ckpt_w8_kernel<<<1024, 256, 0, stream>>>(static_cast<const int8_t *>(storage), w.K,
                                                      w.N, w.Kp, w.Np,
                                                      reinterpret_cast<int8_t *>(dst));
    return cudaGetLastError();
}

}  // namespace ql
