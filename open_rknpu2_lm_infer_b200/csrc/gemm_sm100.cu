// gemm_sm100.cu -- prefill path: int8 x (int4|int8) -> int32 on the 5th-generation tensor
// core (tcgen05.mma kind::i8, accumulators in tensor memory), fed by TMA.
//
// Computes acc[m][n] = sum_k q[m][k] * w[k][n] exactly (src/npu.rs:1111-1116) and the
// epilogue y = (f32(acc) * s_a[m]) * s_w[n] (src/npu.rs:1117) in registers.
//
// Orientation: the MMA's M dimension (128) is weight channels, its N dimension (`tok`,
// 16..256) is tokens:  D[ch][tok] = W[ch][:] . X[tok][:].  One CTA tile is 256 channels x
// tok tokens, computed as two M=128 MMAs that share every activation tile, which halves
// the bytes each SM must pull per multiply-accumulate compared with a 128 x 256 tile (the
// SM's ingress bandwidth, not the tensor core, bounds a 128-channel tile on B200).
//
// Pipeline (one persistent CTA per SM; tiles strided over the grid, token tile fastest so
// CTAs running side by side share a weight tile through L2); k-blocks are 64 deep and use
// the 64-byte swizzle so the load ring is 6 stages deep:
//   warp 0        TMA producer.  Per k-block: the activation tile [tok][64] (SW64) and
//                 either the W8 weight tile [256][64] (SW64) or the packed W4 tile
//                 [256][32 bytes].  Weight loads of the first stages are issued before
//                 griddepcontrol.wait, so with programmatic dependent launch they overlap
//                 the activation-quantisation kernel.
//   warp 1        TMEM allocator and MMA issuer (one thread): 2 halves x 2 K-steps of
//                 tcgen05.mma (M128 x N tok x K32) per k-block; tcgen05.commit releases the
//                 smem slots and, per tile, hands the accumulators to the epilogue.
//   warps 2..9    epilogue: warp (quadrant q, half h) drains TMEM lanes 32q.. of the half-h
//                 accumulator with tcgen05.ld (32 lanes x 16 columns), dequantises and
//                 stores.  When 4*tok <= 512 columns the accumulators are double-buffered
//                 so the epilogue of one tile overlaps the main loop of the next.
//   warps 10..13  (W4 only) converter: packed nibbles -> 8-bit codes in the SW64 K-major
//                 layout of a separate 3-slot ring.  The nibbles stay offset-binary
//                 (u = code + 8; A is declared unsigned) so the unpack is two masks per
//                 word; the epilogue subtracts 8 * sum_k q[m][k].
// Every mbarrier wait is bounded (common.cuh); on a timeout the CTA unwinds, drains its
// in-flight copies and MMAs and frees its tensor memory.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <type_traits>

namespace ql {

namespace {

constexpr int KB = 64;                    // k-block depth (int8 codes per row per stage)
constexpr int CHT = 2 * CH_TILE;          // 256 channels per CTA tile
constexpr int A_SLOT = CHT * KB;          // 16 KB unpacked weights
constexpr int P_SLOT = CHT * KB / 2;      // 8 KB packed W4
constexpr int A_SLOTS_W4 = 3;             // converter ring depth
constexpr int MAX_DYN_SMEM = 232448;      // 227 KB opt-in per block on sm_100
constexpr int SMEM_RESERVE = 1024 + 512;  // alignment slack + barriers
constexpr int MAX_STAGES = 8;

struct GemmArgs {
    const float *wscale;
    const float *ascale;
    const int32_t *rowsum;
    void *out;
    long long ldc;
    int M, N, nkb;
    int tok, stages, n_tok_tiles, num_tiles, acc_bufs;
    uint32_t tmem_cols;
    unsigned *err;
};

template <int BITS>
constexpr int gemm_threads() { return BITS == 4 ? 448 : 320; }

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Shared-memory descriptor, K-major, 64-byte swizzle: rows of 64 bytes, 8-row groups 512
// bytes apart (stride byte offset), leading byte offset 16 (unused for swizzled K-major),
// version 1, layout type 4 (SWIZZLE_64B).
__device__ __forceinline__ uint64_t smem_desc_sw64(const void *tile) {
    const uint64_t addr = smem_u32(tile);
    return ((addr >> 4) & 0x3FFFull) | ((uint64_t)1 << 16) | ((uint64_t)(512 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)4 << 61);
}

template <int BITS, typename OutT>
__global__ void __launch_bounds__(gemm_threads<BITS>(), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap amap,
                const GemmArgs p) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    const int S = p.stages;
    const int tok = p.tok;
    const int b_slot = tok * KB;
    constexpr int w_slot = BITS == 8 ? A_SLOT : P_SLOT;   // what TMA brings per k-block
    uint8_t *sB = smem;                                    // [S][tok][64]
    uint8_t *sW = sB + S * b_slot;                         // [S][256][64] or [S][256][32]
    uint8_t *sA = sW + S * w_slot;                         // W4: [3][256][64] unpacked
    uint64_t *bars =
        reinterpret_cast<uint64_t *>(sA + (BITS == 4 ? A_SLOTS_W4 * A_SLOT : 0));
    uint64_t *full = bars;                  // [S]  TMA bytes landed
    uint64_t *empty = full + S;             // [S]  slot consumed (MMA, and converter for W4)
    uint64_t *afull = empty + S;            // [3]  W4: converter wrote A slot
    uint64_t *aempty = afull + A_SLOTS_W4;  // [3]  W4: MMA done with A slot
    uint64_t *accf = aempty + A_SLOTS_W4;   // [2]  accumulators ready for the epilogue
    uint64_t *acce = accf + 2;              // [2]  epilogue drained the accumulators
    uint64_t *drain = acce + 2;             // [1]  MMA drain on abort
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], BITS == 4 ? 1 + 128 : 1);
        }
        for (int a = 0; a < A_SLOTS_W4; a++) {
            mbar_init(&afull[a], 128);
            mbar_init(&aempty[a], 1);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&accf[b], 1);
            mbar_init(&acce[b], 256);
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
    const uint32_t tx_bytes = (uint32_t)(b_slot + w_slot);

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            // Weight tiles of the first stages do not depend on the preceding kernel:
            // issue them before waiting for it.
            const int pre = ((int)blockIdx.x < p.num_tiles) ? std::min(S, p.nkb) : 0;
            {
                const int tc = blockIdx.x / p.n_tok_tiles;
                for (int j = 0; j < pre; j++) {
                    mbar_arrive_expect_tx(&full[j], tx_bytes);
                    tma_load_2d(sW + j * w_slot, &wmap, &full[j], j * (BITS == 8 ? KB : KB / 2),
                                tc * CHT);
                }
            }
            grid_dep_wait();
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                const int tc = t / p.n_tok_tiles, tt = t % p.n_tok_tiles;
                for (int kb = 0; kb < p.nkb; kb++, it++) {
                    const int s = it % S;
                    const uint32_t ph = (it / S) & 1;
                    if (it >= (uint32_t)pre) {
                        if (!(ok = mbar_wait(&empty[s], ph ^ 1, err, abort_flag))) break;
                        mbar_arrive_expect_tx(&full[s], tx_bytes);
                        tma_load_2d(sW + s * w_slot, &wmap, &full[s],
                                    kb * (BITS == 8 ? KB : KB / 2), tc * CHT);
                    }
                    tma_load_2d(sB + s * b_slot, &amap, &full[s], kb * KB, tt * tok);
                }
            }
            if (!ok) {
                // Let every copy already issued land before the CTA exits.
                volatile int never = 0;
                const uint32_t issued = std::max(it, (uint32_t)pre);
                const uint32_t first = issued > (uint32_t)S ? issued - S : 0;
                for (uint32_t j = first; j < issued; j++)
                    mbar_wait(&full[j % S], (j / S) & 1, nullptr, &never);
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer
        if (lane == 0) {
            const uint32_t idesc = idesc_i8(CH_TILE, tok, BITS == 8, true);
            uint32_t it = 0, local = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x, local++) {
                const int ab = local % p.acc_bufs;
                const uint32_t aph = (local / p.acc_bufs) & 1;
                if (!(ok = mbar_wait(&acce[ab], aph ^ 1, err, abort_flag))) break;
                tc_fence_after();
                const uint32_t d0 = tmem_base + (uint32_t)(ab * 2 * tok);
                for (int kb = 0; kb < p.nkb; kb++, it++) {
                    const int s = it % S;
                    const uint32_t ph = (it / S) & 1;
                    const int a = it % A_SLOTS_W4;
                    if (!(ok = mbar_wait(&full[s], ph, err, abort_flag))) break;
                    if (BITS == 4 &&
                        !(ok = mbar_wait(&afull[a], (it / A_SLOTS_W4) & 1, err, abort_flag)))
                        break;
                    tc_fence_after();
                    const uint8_t *At = BITS == 8 ? sW + s * w_slot : sA + a * A_SLOT;
                    const uint64_t bdesc = smem_desc_sw64(sB + s * b_slot);
#pragma unroll
                    for (int h = 0; h < 2; h++) {
                        const uint64_t adesc = smem_desc_sw64(At + h * (CH_TILE * KB));
#pragma unroll
                        for (int k = 0; k < KB / 32; k++)
                            mma_i8_ss(d0 + (uint32_t)(h * tok), adesc + 2 * k, bdesc + 2 * k,
                                      idesc, (kb | k) != 0);
                    }
                    mma_commit(&empty[s]);
                    if (BITS == 4) mma_commit(&aempty[a]);
                }
                if (ok) mma_commit(&accf[ab]);
            }
            if (!ok) {
                volatile int never = 0;
                mma_commit(drain);
                mbar_wait(drain, 0, nullptr, &never);
            }
        }
    } else if (warp < 10) {
        // ------------------------------------------------------------ epilogue
        grid_dep_wait();  // the activation scales/rowsums come from the previous kernel
        const int q = warp & 3;            // TMEM lane quadrant this warp may access
        const int h = (warp - 2) >> 2;     // accumulator half (channels h*128 ..)
        uint32_t local = 0;
        OutT *out = static_cast<OutT *>(p.out);
        for (int t = blockIdx.x; t < p.num_tiles; t += gridDim.x, local++) {
            const int tc = t / p.n_tok_tiles, tt = t % p.n_tok_tiles;
            const int ab = local % p.acc_bufs;
            const uint32_t aph = (local / p.acc_bufs) & 1;
            // every lane waits (bounded); the warp leaves together if any lane gave up,
            // so the warp-collective tcgen05.ld / shuffles below stay converged
            const bool okw = mbar_wait(&accf[ab], aph, err, abort_flag);
            if (!__all_sync(0xffffffffu, okw)) break;
            tc_fence_after();
            const int ch = tc * CHT + h * CH_TILE + q * 32 + lane;
            const bool chv = ch < p.N;
            const float sw = chv ? p.wscale[ch] : 0.0f;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) +
                                   (uint32_t)(ab * 2 * tok + h * tok);
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
            const int ct = threadIdx.x - 320;  // 0..127
            const int half = ct & 1;           // which 16-byte half of a 32-byte packed row
            uint32_t it = 0;
            bool ok = true;
            for (int t = blockIdx.x; t < p.num_tiles && ok; t += gridDim.x) {
                for (int kb = 0; kb < p.nkb; kb++, it++) {
                    const int s = it % S;
                    const int a = it % A_SLOTS_W4;
                    if (!(ok = mbar_wait(&full[s], (it / S) & 1, err, abort_flag))) break;
                    if (!(ok = mbar_wait(&aempty[a], ((it / A_SLOTS_W4) & 1) ^ 1, err, abort_flag)))
                        break;
                    const uint8_t *P = sW + s * w_slot;
                    uint8_t *A = sA + a * A_SLOT;
#pragma unroll
                    for (int j = 0; j < 4; j++) {
                        // a thread pair per row; 64 rows per pass
                        const int row = (ct >> 1) + 64 * j;
                        const uint4 v = *reinterpret_cast<const uint4 *>(P + row * 32 + half * 16);
                        // 16 packed bytes = codes k = 32*half .. 32*half+31 of this k-block:
                        // word p covers 8 codes, low nibbles k 8p..8p+3, high 8p+4..8p+7.
                        const uint4 c0 = make_uint4(v.x & 0x0F0F0F0Fu, (v.x >> 4) & 0x0F0F0F0Fu,
                                                    v.y & 0x0F0F0F0Fu, (v.y >> 4) & 0x0F0F0F0Fu);
                        const uint4 c1 = make_uint4(v.z & 0x0F0F0F0Fu, (v.z >> 4) & 0x0F0F0F0Fu,
                                                    v.w & 0x0F0F0F0Fu, (v.w >> 4) & 0x0F0F0F0Fu);
                        const int sw = (row >> 1) & 3;  // 64-byte swizzle of this row
                        *reinterpret_cast<uint4 *>(A + row * 64 + (((2 * half) ^ sw) << 4)) = c0;
                        *reinterpret_cast<uint4 *>(A + row * 64 + (((2 * half + 1) ^ sw) << 4)) = c1;
                    }
                    fence_proxy_async_smem();
                    mbar_arrive(&afull[a]);
                    mbar_arrive(&empty[s]);
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
                     const GemmPlan &plan, bool pdl, cudaStream_t stream) {
    auto kern = gemm_kernel<BITS, OutT>;
    // The opt-in shared-memory limit is a per-device, per-kernel attribute: set it once per
    // device (an attribute call per launch costs host time).
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
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(plan.grid);
    cfg.blockDim = dim3(gemm_threads<BITS>());
    cfg.dynamicSmemBytes = plan.smem_bytes;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    return cudaLaunchKernelEx(&cfg, kern, wmap, amap, args);
}

}  // namespace

GemmPlan plan_gemm(const WeightView &w, int rows, int num_sms) {
    GemmPlan plan{};
    const int tiles_m = std::max(1, (rows + 255) / 256);
    int tok = (rows + tiles_m - 1) / tiles_m;
    tok = std::max(16, (tok + 15) / 16 * 16);
    plan.tok = tok;
    const int stage_bytes = tok * KB + (w.bits == 8 ? A_SLOT : P_SLOT);
    const int fixed = SMEM_RESERVE + (w.bits == 4 ? A_SLOTS_W4 * A_SLOT : 0);
    const int stages = std::min(MAX_STAGES, (MAX_DYN_SMEM - fixed) / stage_bytes);
    plan.stages = stages;
    // One CTA per SM: the kernel allocates up to 512 TMEM columns.
    plan.smem_bytes = std::max(stages * stage_bytes + fixed, 120 * 1024);
    const int n_tok_tiles = (rows + tok - 1) / tok;
    plan.tiles = ((w.Np + CHT - 1) / CHT) * n_tok_tiles;
    plan.grid = std::min(plan.tiles, num_sms);
    return plan;
}

cudaError_t launch_gemm(const WeightView &w, const CUtensorMap &wmap, const ActView &a,
                        const CUtensorMap &amap, const GemmPlan &plan, int rows, void *out,
                        int out_type, long long ldc, unsigned *err, bool pdl,
                        cudaStream_t stream) {
    GemmArgs args{};
    args.wscale = w.scales;
    args.ascale = a.scales;
    args.rowsum = a.rowsums;
    args.out = out;
    args.ldc = ldc;
    args.M = rows;
    args.N = w.N;
    args.nkb = w.Kp / KB;
    args.tok = plan.tok;
    args.stages = plan.stages;
    args.n_tok_tiles = (rows + plan.tok - 1) / plan.tok;
    args.num_tiles = plan.tiles;
    args.acc_bufs = (4 * plan.tok <= 512) ? 2 : 1;
    uint32_t cols = 32;
    while (cols < (uint32_t)(2 * plan.tok * args.acc_bufs)) cols <<= 1;
    args.tmem_cols = cols;
    args.err = err;
    if (w.bits == 8) {
        if (out_type == kF16) return launch_t<8, __half>(wmap, amap, args, plan, pdl, stream);
        if (out_type == kF32) return launch_t<8, float>(wmap, amap, args, plan, pdl, stream);
        return launch_t<8, int32_t>(wmap, amap, args, plan, pdl, stream);
    }
    if (out_type == kF16) return launch_t<4, __half>(wmap, amap, args, plan, pdl, stream);
    if (out_type == kF32) return launch_t<4, float>(wmap, amap, args, plan, pdl, stream);
    return launch_t<4, int32_t>(wmap, amap, args, plan, pdl, stream);
}

}  // namespace ql
