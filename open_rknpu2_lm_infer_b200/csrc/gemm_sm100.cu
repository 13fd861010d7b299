// gemm_sm100.cu -- prefill path: int8 x (int4|int8) -> int32 on the 5th-generation tensor
// core (tcgen05.mma kind::i8, accumulators in tensor memory), fed by TMA.
//
// Computes acc[m][n] = sum_k q[m][k] * w[k][n] exactly (src/npu.rs:1111-1116) and the
// epilogue y = (f32(acc) * s_a[m]) * s_w[n] (src/npu.rs:1117) in registers.
//
// Orientation: the MMA's M dimension (128) is 128 weight channels, its N dimension
// (`tok`, 16..256) is a tile of tokens, so decode-ish and prefill token counts both map
// onto one instruction shape:  D[ch][tok] = W[ch][:] . X[tok][:].
//
// Tiles and roles (one persistent CTA per SM, tiles strided over the grid, the token
// tile index fastest so CTAs running side by side share a weight tile through L2):
//   warp 0      TMA producer: activation tile [tok][128] (128-byte swizzle) and, for W8,
//               the weight tile [128][128] (128-byte swizzle); for W4 the packed tile
//               [128][64 bytes] (no swizzle) into a staging ring.
//   warp 1      TMEM allocator and MMA issuer (one thread): 4 x tcgen05.mma (K = 32 each)
//               per 128-deep k-block, tcgen05.commit frees the smem stage.
//   warps 2..5  epilogue: tcgen05.ld 32 lanes x 16 columns, dequant, store.  Two TMEM
//               accumulators (2 x tok columns) let the epilogue of tile i overlap the
//               main loop of tile i+1.
//   warps 6..9  (W4 only) converter: packed nibbles -> 8-bit codes written straight into
//               the 128-byte-swizzled K-major layout the MMA reads.  The nibbles stay
//               offset-binary (u = code + 8, A is declared unsigned) so the unpack is two
//               masks per word; the epilogue subtracts 8 * sum_k q[m][k].
// Every mbarrier wait is bounded (common.cuh); on a timeout the CTA unwinds, drains its
// in-flight copies and MMAs and frees its tensor memory.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <type_traits>

namespace ql {

namespace {

constexpr int A_TILE_BYTES = CH_TILE * KBLK;       // 16 KB: 128 channels x 128 codes
constexpr int P_TILE_BYTES = CH_TILE * KBLK / 2;   // 8 KB: packed W4
constexpr int MAX_DYN_SMEM = 232448;               // 227 KB opt-in per block on sm_100
constexpr int SMEM_RESERVE = 1024 + 512;           // alignment slack + barriers

struct GemmArgs {
    const float *wscale;
    const float *ascale;
    const int32_t *rowsum;
    void *out;
    long long ldc;
    int M, N, nkb;
    int tok, stages, n_tok_tiles, num_tiles;
    uint32_t tmem_cols;
    unsigned *err;
};

template <int BITS>
constexpr int gemm_threads() { return BITS == 4 ? 320 : 192; }

template <int BITS, typename OutT>
__global__ void __launch_bounds__(gemm_threads<BITS>(), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap amap,
                const GemmArgs p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    const int S = p.stages;
    const int tok = p.tok;
    const int b_tile_bytes = tok * KBLK;
    uint8_t *sA = smem;
    uint8_t *sB = sA + S * A_TILE_BYTES;
    uint8_t *sP = sB + S * b_tile_bytes;
    uint64_t *bars = reinterpret_cast<uint64_t *>(sP + (BITS == 4 ? S * P_TILE_BYTES : 0));
    uint64_t *full = bars;            // [S] TMA bytes landed (B, and A for W8)
    uint64_t *empty = full + S;       // [S] MMA done with stage s
    uint64_t *afull = empty + S;      // [S] W4: converter wrote A[s]
    uint64_t *pfull = afull + S;      // [S] W4: packed tile landed
    uint64_t *pempty = pfull + S;     // [S] W4: converter done with packed tile
    uint64_t *accf = pempty + S;      // [2] accumulator ready for the epilogue
    uint64_t *acce = accf + 2;        // [2] epilogue drained the accumulator
    uint64_t *drain = acce + 2;       // [1] MMA drain on abort
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&afull[s], 128);
            mbar_init(&pfull[s], 1);
            mbar_init(&pempty[s], 128);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&accf[b], 1);
            mbar_init(&acce[b], 128);
        }
        mbar_init(drain, 1);
        *abort_flag = 0;
        mbar_fence_init();
    }
    if (warp == 0 && lane == 0) {
        tma_prefetch_desc(&wmap);
        tma_prefetch_desc(&amap);
    }
    if (warp == 1) {
        tmem_alloc(tmem_slot, p.tmem_cols);
        tmem_relinquish();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    unsigned *err = p.err;

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                const int tc = t / p.n_tok_tiles, tt = t % p.n_tok_tiles;
                for (int kb = 0; kb < p.nkb; kb++, it++) {
                    const int s = it % S;
                    const uint32_t ph = (it / S) & 1;
                    if (!(ok = mbar_wait(&empty[s], ph ^ 1, err, abort_flag))) break;
                    if (BITS == 4 && !(ok = mbar_wait(&pempty[s], ph ^ 1, err, abort_flag))) break;
                    if (BITS == 8) {
                        mbar_arrive_expect_tx(&full[s], A_TILE_BYTES + b_tile_bytes);
                        tma_load_2d(sA + s * A_TILE_BYTES, &wmap, &full[s], kb * KBLK, tc * CH_TILE);
                    } else {
                        mbar_arrive_expect_tx(&full[s], b_tile_bytes);
                    }
                    tma_load_2d(sB + s * b_tile_bytes, &amap, &full[s], kb * KBLK, tt * tok);
                    if (BITS == 4) {
                        mbar_arrive_expect_tx(&pfull[s], P_TILE_BYTES);
                        tma_load_2d(sP + s * P_TILE_BYTES, &wmap, &pfull[s], kb * (KBLK / 2),
                                    tc * CH_TILE);
                    }
                }
            }
            if (!ok) {
                // Let every copy already issued land before the CTA exits: wait (bounded,
                // ignoring the abort flag) on the last S stages' barriers.
                volatile int never = 0;
                const uint32_t first = it > (uint32_t)S ? it - S : 0;
                for (uint32_t j = first; j < it; j++) {
                    const int s = j % S;
                    const uint32_t ph = (j / S) & 1;
                    mbar_wait(&full[s], ph, nullptr, &never);
                    if (BITS == 4) mbar_wait(&pfull[s], ph, nullptr, &never);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_i8(CH_TILE, tok, BITS == 8, true);
            uint32_t it = 0, local = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, local++) {
                const int ab = local & 1;
                const uint32_t aph = (local >> 1) & 1;
                if (!(ok = mbar_wait(&acce[ab], aph ^ 1, err, abort_flag))) break;
                tc_fence_after();
                const uint32_t d_tmem = tmem_base + (uint32_t)(ab * tok);
                for (int kb = 0; kb < p.nkb; kb++, it++) {
                    const int s = it % S;
                    const uint32_t ph = (it / S) & 1;
                    if (!(ok = mbar_wait(&full[s], ph, err, abort_flag))) break;
                    if (BITS == 4 && !(ok = mbar_wait(&afull[s], ph, err, abort_flag))) break;
                    tc_fence_after();
                    const uint64_t adesc = smem_desc_sw128(sA + s * A_TILE_BYTES);
                    const uint64_t bdesc = smem_desc_sw128(sB + s * b_tile_bytes);
#pragma unroll
                    for (int k = 0; k < KBLK / 32; k++)
                        mma_i8_ss(d_tmem, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0);
                    mma_commit(&empty[s]);
                }
                if (ok) mma_commit(&accf[ab]);
            }
            if (!ok) {
                volatile int never = 0;
                mma_commit(drain);
                mbar_wait(drain, 0, nullptr, &never);
            }
        }
    } else if (warp < 6) {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;  // TMEM lane quadrant this warp may access
        uint32_t local = 0;
        for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, local++) {
            const int tc = t / p.n_tok_tiles, tt = t % p.n_tok_tiles;
            const int ab = local & 1;
            const uint32_t aph = (local >> 1) & 1;
            // every lane waits (bounded); the warp leaves together if any lane gave up,
            // so the warp-collective tcgen05.ld / shuffles below stay converged
            const bool ok = mbar_wait(&accf[ab], aph, err, abort_flag);
            if (!__all_sync(0xffffffffu, ok)) break;
            tc_fence_after();
            const int ch = tc * CH_TILE + q * 32 + lane;
            const bool chv = ch < p.N;
            const float sw = chv ? p.wscale[ch] : 0.0f;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) + (uint32_t)(ab * tok);
            OutT *out = static_cast<OutT *>(p.out);
            for (int c = 0; c < tok / 16; c++) {
                uint32_t r[16];
                tmem_ld16(taddr + c * 16, r);
                tmem_ld_wait();
                const int tok0 = tt * tok + c * 16;
                const bool lv = lane < 16 && tok0 + lane < p.M;
                const float sa_l = lv ? p.ascale[tok0 + lane] : 0.0f;
                const int rs_l = (BITS == 4 && lv) ? p.rowsum[tok0 + lane] : 0;
#pragma unroll
                for (int j = 0; j < 16; j++) {
                    const float sa = __shfl_sync(0xffffffffu, sa_l, j);
                    const int rs = __shfl_sync(0xffffffffu, rs_l, j);
                    const int m = tok0 + j;
                    if (chv && m < p.M) {
                        int acc = (int)r[j];
                        if (BITS == 4) acc -= 8 * rs;
                        if constexpr (std::is_same<OutT, int32_t>::value) {
                            out[(long long)m * p.ldc + ch] = acc;
                        } else {
                            const float y = __fmul_rn(__fmul_rn(__int2float_rn(acc), sa), sw);
                            out[(long long)m * p.ldc + ch] = OutCvt<OutT>::from(y);
                        }
                    }
                }
            }
            tc_fence_before();
            mbar_arrive(&acce[ab]);
        }
    } else {
        // ------------------------------------------------------------ W4 converter
        if constexpr (BITS == 4) {
            const int ct = threadIdx.x - 192;  // 0..127
            const int cp = ct & 3;             // packed 16-byte chunk of the row (32 codes)
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                for (int kb = 0; kb < p.nkb; kb++, it++) {
                    const int s = it % S;
                    const uint32_t ph = (it / S) & 1;
                    if (!(ok = mbar_wait(&pfull[s], ph, err, abort_flag))) break;
                    if (!(ok = mbar_wait(&empty[s], ph ^ 1, err, abort_flag))) break;
                    const uint8_t *P = sP + s * P_TILE_BYTES;
                    uint8_t *A = sA + s * A_TILE_BYTES;
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        const int row = (ct >> 2) + 32 * j;
                        const uint4 v = *reinterpret_cast<const uint4 *>(P + row * 64 + cp * 16);
                        const uint4 c0 = make_uint4(v.x & 0x0F0F0F0Fu, (v.x >> 4) & 0x0F0F0F0Fu,
                                                    v.y & 0x0F0F0F0Fu, (v.y >> 4) & 0x0F0F0F0Fu);
                        const uint4 c1 = make_uint4(v.z & 0x0F0F0F0Fu, (v.z >> 4) & 0x0F0F0F0Fu,
                                                    v.w & 0x0F0F0F0Fu, (v.w >> 4) & 0x0F0F0F0Fu);
                        const int sw = row & 7;
                        *reinterpret_cast<uint4 *>(A + row * 128 + (((2 * cp) ^ sw) << 4)) = c0;
                        *reinterpret_cast<uint4 *>(A + row * 128 + (((2 * cp + 1) ^ sw) << 4)) = c1;
                    }
                    fence_proxy_async_smem();
                    mbar_arrive(&afull[s]);
                    mbar_arrive(&pempty[s]);
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc(tmem_base, p.tmem_cols);
    }
}

template <int BITS, typename OutT>
cudaError_t launch_t(const CUtensorMap &wmap, const CUtensorMap &amap, const GemmArgs &args,
                     const GemmPlan &plan, cudaStream_t stream) {
    auto kern = gemm_kernel<BITS, OutT>;
    // The opt-in shared-memory limit is a per-device, per-kernel attribute: set it to the
    // maximum once per device (an attribute call per launch costs host time).
    static int configured[64] = {0};
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             MAX_DYN_SMEM);
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    kern<<<plan.grid, gemm_threads<BITS>(), plan.smem_bytes, stream>>>(wmap, amap, args);
    return cudaGetLastError();
}

}  // namespace

GemmPlan plan_gemm(const WeightView &w, int rows, int num_sms) {
    GemmPlan plan{};
    const int tiles_m = std::max(1, (rows + 255) / 256);
    int tok = (rows + tiles_m - 1) / tiles_m;
    tok = std::max(16, (tok + 15) / 16 * 16);
    plan.tok = tok;
    const int stage_bytes = A_TILE_BYTES + tok * KBLK + (w.bits == 4 ? P_TILE_BYTES : 0);
    int stages = (MAX_DYN_SMEM - SMEM_RESERVE) / stage_bytes;
    stages = std::min(stages, 8);
    plan.stages = stages;
    int smem = stages * stage_bytes + SMEM_RESERVE;
    // One CTA per SM: the kernel allocates up to 512 TMEM columns.
    smem = std::max(smem, 120 * 1024);
    plan.smem_bytes = smem;
    const int n_tok_tiles = (rows + tok - 1) / tok;
    plan.tiles = (w.Np / CH_TILE) * n_tok_tiles;
    plan.grid = std::min(plan.tiles, num_sms);
    return plan;
}

cudaError_t launch_gemm(const WeightView &w, const CUtensorMap &wmap, const ActView &a,
                        const CUtensorMap &amap, const GemmPlan &plan, int rows, void *out,
                        int out_type, long long ldc, unsigned *err, cudaStream_t stream) {
    GemmArgs args{};
    args.wscale = w.scales;
    args.ascale = a.scales;
    args.rowsum = a.rowsums;
    args.out = out;
    args.ldc = ldc;
    args.M = rows;
    args.N = w.N;
    args.nkb = w.Kp / KBLK;
    args.tok = plan.tok;
    args.stages = plan.stages;
    args.n_tok_tiles = (rows + plan.tok - 1) / plan.tok;
    args.num_tiles = plan.tiles;
    uint32_t cols = 32;
    while (cols < (uint32_t)(2 * plan.tok)) cols <<= 1;
    args.tmem_cols = cols;
    args.err = err;
    if (w.bits == 8) {
        if (out_type == kF16) return launch_t<8, __half>(wmap, amap, args, plan, stream);
        if (out_type == kF32) return launch_t<8, float>(wmap, amap, args, plan, stream);
        return launch_t<8, int32_t>(wmap, amap, args, plan, stream);
    }
    if (out_type == kF16) return launch_t<4, __half>(wmap, amap, args, plan, stream);
    if (out_type == kF32) return launch_t<4, float>(wmap, amap, args, plan, stream);
    return launch_t<4, int32_t>(wmap, amap, args, plan, stream);
}

}  // namespace ql
