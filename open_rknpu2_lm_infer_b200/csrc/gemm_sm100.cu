// gemm_sm100.cu -- prefill path: int8 x (int4|int8) -> int32 on the 5th-generation tensor
// core (tcgen05.mma kind::i8, accumulators in tensor memory), fed by TMA, run by CTA pairs.
//
// Computes acc[m][n] = sum_k q[m][k] * w[k][n] exactly (src/npu.rs:1111-1116) and the
// epilogue y = (f32(acc) * s_a[m]) * s_w[n] (src/npu.rs:1117) in registers.
//
// Orientation: the MMA's M dimension is weight channels, its N dimension (`tok`, 32..256)
// tokens:  D[ch][tok] = W[ch][:] . X[tok][:].  A cluster of two CTAs on the two SMs of a
// TPC computes a 256-channel x tok tile with tcgen05.mma.cta_group::2 (M = 256): each CTA
// stages its own 128 weight channels and half of the tok activation rows, the tensor core
// reads both halves of B across the pair, and each CTA's tensor memory receives the
// accumulators of its 128 channels for all tok tokens.  Measured on B200, a one-CTA M=128
// MMA is bounded by the tensor core's shared-memory operand bandwidth (~2.9 POPS at
// N=256); the pair halves each SM's operand traffic, and the 256-wide tile halves the
// bytes each SM pulls from L2 per multiply-accumulate.
//
// Roles (one persistent CTA pair per TPC; tiles strided over the clusters, the token tile
// fastest so neighbouring pairs share a weight tile through L2); 128-deep k-blocks in the
// 128-byte swizzle (4 MMAs per hand-off: measured on B200, one producer -> MMA -> commit
// round costs ~400 cycles, so a hand-off must carry at least that much tensor work), a ring
// of up to 8 stages:
//   warp 0        TMA producer (both CTAs).  Activation half-tile [tok/2][128] and, for W8,
//                 the weight tile [128][128], both counted on the leader CTA's `full`
//                 barrier (cta_group::2 copies).  W8 weight loads of the first stages are
//                 issued before griddepcontrol.wait, overlapping the activation-quantisation
//                 kernel under programmatic dependent launch.
//   warp 1        tensor-memory allocation (both CTAs, pair-wide); in the leader CTA one
//                 thread issues 4 MMAs (K=32 each) per k-block and commits them to the
//                 barriers of both CTAs (multicast commit), freeing the smem slots and, per
//                 tile, handing the accumulators to the epilogues.
//   warps 2..9    epilogue (both CTAs): warp (lane quadrant q, column half) drains its
//                 part of the tensor-memory accumulator with tcgen05.ld, dequantises and
//                 stores.  Accumulators are double-buffered (2 x tok <= 512 columns) so the
//                 epilogue of one tile overlaps the main loop of the next.
//   warps 10..13  (W4 only, both CTAs) converter: streams the packed weights of its 128
//                 channels from global memory into a 4-deep register prefetch ring (no
//                 shared-memory staging: every shared-memory byte saved shortens the stage
//                 round trip), unpacks them into the stage's SW128 K-major A buffer once the
//                 MMA has released the stage, and announces it to the leader.
//                 The nibbles stay offset-binary (u = code + 8; A is declared unsigned) so
//                 the unpack is two masks per word; the epilogue subtracts 8 * sum_k q[m][k].
// Every mbarrier wait is bounded (common.cuh); on a timeout the pair unwinds, drains its
// in-flight copies and MMAs and frees its tensor memory.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <type_traits>

namespace ql {

namespace {

constexpr int KB = GEMM_KB;                 // k-block depth (int8 codes per row per stage)
static_assert(KB == 128, "one 128-byte swizzle atom per row per stage");
constexpr int CH_CTA = CH_TILE;             // 128 channels per CTA
constexpr int CHT = 2 * CH_CTA;             // 256 channels per pair tile
constexpr int A_SLOT = CH_CTA * KB;         // 16 KB unpacked weights per CTA
constexpr int W4_PREFETCH = 4;              // converter register ring depth (k-blocks)
constexpr int EPI_WARPS = 8;
constexpr int MAX_DYN_SMEM = 232448;        // 227 KB opt-in per block on sm_100
constexpr int SMEM_RESERVE = 1024 + 1024;   // alignment slack + barriers
constexpr int MAX_STAGES = 8;

struct GemmArgs {
    const uint8_t *wq;     // W4 packed weights [Np][Kp/2] (read by the converter)
    int Np;
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
constexpr int gemm_threads() { return (2 + EPI_WARPS + (BITS == 4 ? 4 : 0)) * 32; }

__device__ __forceinline__ void grid_dep_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

__device__ __forceinline__ uint32_t cluster_id_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%clusterid.x;" : "=r"(r));
    return r;
}
__device__ __forceinline__ uint32_t num_clusters_x() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%nclusterid.x;" : "=r"(r));
    return r;
}

// Shared-memory descriptor, K-major, 128-byte swizzle: rows of 128 bytes, 8-row groups 1024
// bytes apart (stride byte offset), leading byte offset 16 (unused for swizzled K-major),
// version 1, layout type 2 (SWIZZLE_128B).  Advancing the start address by 32 bytes steps
// one MMA (K = 32) along the row; the swizzle is applied to absolute address bits.
__device__ __forceinline__ uint64_t smem_desc_sw128_k(const void *tile) {
    const uint64_t addr = smem_u32(tile);
    return ((addr >> 4) & 0x3FFFull) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
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
    const int b_half = (tok / 2) * KB;                    // this CTA's activation rows
    constexpr int w_slot = A_SLOT;   // 8-bit weights per stage (TMA for W8, converter for W4)
    uint8_t *sB = smem;              // [S][tok/2][128]
    uint8_t *sW = sB + S * b_half;   // [S][128][128]
    uint64_t *bars = reinterpret_cast<uint64_t *>(sW + S * w_slot);
    uint64_t *full = bars;              // [S] leader: both CTAs' TMA bytes landed
    uint64_t *empty = full + S;         // [S] the MMA is done with the stage
    uint64_t *afull = empty + S;        // [S] leader: both converters unpacked the stage
    uint64_t *cdone = afull + S;        // [S] W4: this CTA's 128 converter threads wrote it
    uint64_t *accf = cdone + S;         // [2] accumulators ready for the epilogue
    uint64_t *acce = accf + 2;          // [2] leader: both epilogues drained them
    uint64_t *drain = acce + 2;         // [1] leader: MMA drain on abort
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(drain + 1);
    volatile int *abort_flag = reinterpret_cast<volatile int *>(tmem_slot + 1);

    const int warp = threadIdx.x >> 5;
    const int lane = threadIdx.x & 31;
    const uint32_t rank = cluster_ctarank();  // 0 = leader
    const uint32_t cid = cluster_id_x(), ncl = num_clusters_x();

    if (threadIdx.x == 0) {
        for (int s = 0; s < S; s++) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
            mbar_init(&afull[s], 2);
            mbar_init(&cdone[s], 128);
        }
        for (int b = 0; b < 2; b++) {
            mbar_init(&accf[b], 1);
            mbar_init(&acce[b], 2 * EPI_WARPS);
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
        tmem_alloc_pair(tmem_slot, p.tmem_cols);
        tmem_relinquish_pair();
    }
    tc_fence_before();
    __syncthreads();
    cluster_sync();  // the peer's barriers are initialised before anyone signals them
    tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;
    unsigned *err = p.err;
    const uint32_t full0 = map_to_rank(&full[0], 0);  // leader's barriers (cluster addresses)
    const uint32_t afull0 = map_to_rank(&afull[0], 0);
    const uint32_t acce0 = map_to_rank(&acce[0], 0);
    // bytes the leader's `full` barrier receives per stage from both CTAs
    const uint32_t tx_pair = 2u * (uint32_t)(b_half + (BITS == 8 ? A_SLOT : 0));

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            auto load_weights = [&](int s, int kb, int tc) {
                if (BITS == 8)
                    tma_load_2d_pair(sW + s * w_slot, &wmap, full0 + 8u * s, kb * KB,
                                     tc * CHT + (int)rank * CH_CTA);
                if (rank == 0) mbar_arrive_expect_tx(&full[s], tx_pair);
            };
            // Weight tiles of the first stages do not depend on the preceding kernel:
            // issue them before waiting for it.
            const int pre = ((int)cid < p.num_tiles) ? std::min(S, p.nkb) : 0;
            for (int j = 0; j < pre; j++) load_weights(j, j, (int)cid / p.n_tok_tiles);
            grid_dep_wait();
            uint32_t it = 0, s = 0, ph = 0;  // iteration, stage, stage phase
            bool ok = true;
            for (int t = (int)cid; t < p.num_tiles && ok; t += (int)ncl) {
                const int tc = t / p.n_tok_tiles, tt = t % p.n_tok_tiles;
                for (int kb = 0; kb < p.nkb; kb++, it++) {
                    if (it >= (uint32_t)pre) {
                        if (!(ok = mbar_wait(&empty[s], ph ^ 1, err, abort_flag))) break;
                        load_weights(s, kb, tc);
                    }
                    tma_load_2d_pair(sB + s * b_half, &amap, full0 + 8u * s, kb * KB,
                                     tt * tok + (int)rank * (tok / 2));
                    if (++s == (uint32_t)S) { s = 0; ph ^= 1; }
                }
            }
            if (!ok) {
                // Let the copies already issued land before the pair exits.
                volatile int never = 0;
                const uint32_t issued = std::max(it, (uint32_t)pre);
                const uint32_t first = issued > (uint32_t)S ? issued - S : 0;
                for (uint32_t j = first; j < issued; j++) {
                    if (rank == 0) mbar_wait(&full[j % S], (j / S) & 1, nullptr, &never);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader)
        if (lane == 0 && rank == 0) {
            const uint32_t idesc = idesc_i8(2 * CH_CTA, tok, BITS == 8, true);
            uint32_t s = 0, ph = 0, local = 0;
            bool ok = true;
            for (int t = (int)cid; t < p.num_tiles && ok; t += (int)ncl, local++) {
                const int ab = local & 1;
                if (!(ok = mbar_wait(&acce[ab], ((local >> 1) & 1) ^ 1, err, abort_flag))) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(ab * tok);
                for (int kb = 0; kb < p.nkb; kb++) {
                    if (!(ok = mbar_wait(&full[s], ph, err, abort_flag))) break;
                    if (BITS == 4 && !(ok = mbar_wait(&afull[s], ph, err, abort_flag))) break;
                    tc_fence_after();
                    const uint64_t adesc = smem_desc_sw128_k(sW + s * w_slot);
                    const uint64_t bdesc = smem_desc_sw128_k(sB + s * b_half);
#pragma unroll
                    for (int k = 0; k < KB / 32; k++)
                        mma_i8_ss_pair(d, adesc + 2 * k, bdesc + 2 * k, idesc, (kb | k) != 0);
                    mma_commit_pair(&empty[s], 0x3);
                    if (++s == (uint32_t)S) { s = 0; ph ^= 1; }
                }
                if (ok) mma_commit_pair(&accf[ab], 0x3);
            }
            if (!ok) {
                volatile int never = 0;
                mma_commit_pair(drain, 0x1);  // leader's drain barrier only
                mbar_wait(drain, 0, nullptr, &never);
            }
        }
    } else if (warp < 2 + EPI_WARPS) {
        // ------------------------------------------------------------ epilogue
        grid_dep_wait();  // the activation scales / row sums come from the previous kernel
        const int q = warp & 3;                 // TMEM lane quadrant this warp may access
        const int colh = (warp - 2) >> 2;       // which half of the tok columns
        const int cols = tok / 2;
        uint32_t local = 0;
        OutT *out = static_cast<OutT *>(p.out);
        for (int t = (int)cid; t < p.num_tiles; t += (int)ncl, local++) {
            const int tc = t / p.n_tok_tiles, tt = t % p.n_tok_tiles;
            const int ab = local & 1;
            // every lane waits (bounded); the warp leaves together if any lane gave up,
            // so the warp-collective tcgen05.ld / shuffles below stay converged
            const bool okw = mbar_wait(&accf[ab], (local >> 1) & 1, err, abort_flag);
            if (!__all_sync(0xffffffffu, okw)) break;
            tc_fence_after();
            const int ch = tc * CHT + (int)rank * CH_CTA + q * 32 + lane;
            const bool chv = ch < p.N;
            const float sw = chv ? p.wscale[ch] : 0.0f;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) +
                                   (uint32_t)(ab * tok + colh * cols);
            for (int c = 0; c < cols / 16; c++) {
                uint32_t r[16];
                tmem_ld16(taddr + c * 16, r);
                tmem_ld_wait();
                const int tok0 = tt * tok + colh * cols + c * 16;
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
            __syncwarp();
            if (lane == 0) mbar_arrive_remote(acce0 + 8u * ab);
        }
    } else {
        // ------------------------------------------------------------ W4 converter
        if constexpr (BITS == 4) {
            const int ct = threadIdx.x - (2 + EPI_WARPS) * 32;  // 0..127
            const int cp = ct & 3;      // 16-byte quarter of a row's 64 packed bytes (32 codes)
            const int r0 = ct >> 2;     // rows r0 + 32 j, j = 0..3
            const long long row_bytes = (long long)p.nkb * (KB / 2);
            // Packed codes of iteration (tile t, k-block kb) for this thread's 4 rows.
            auto fetch = [&](uint4 (&b)[4], int t, int kb) {
                const int n0 = (t / p.n_tok_tiles) * CHT + (int)rank * CH_CTA;
#pragma unroll
                for (int j = 0; j < 4; j++) {
                    const int n = n0 + r0 + 32 * j;
                    b[j] = n < p.Np ? ldg_stream(p.wq + (long long)n * row_bytes + kb * (KB / 2) +
                                                 cp * 16)
                                    : make_uint4(0, 0, 0, 0);
                }
            };
            uint4 buf[W4_PREFETCH][4];
            int ft = (int)cid, fkb = 0;  // prefetch stream position
#pragma unroll
            for (int u = 0; u < W4_PREFETCH; u++) {
                if (ft < p.num_tiles) {
                    fetch(buf[u], ft, fkb);
                    if (++fkb == p.nkb) { fkb = 0; ft += (int)ncl; }
                }
            }
            uint32_t s = 0, ph = 0;
            int t = (int)cid, kb = 0;
            bool live = t < p.num_tiles;
            while (live) {
#pragma unroll
                for (int u = 0; u < W4_PREFETCH; u++) {
                    if (live) {
                        // the MMA released the stage (its A buffer) of iteration it - S
                        if (!mbar_wait(&empty[s], ph ^ 1, err, abort_flag)) { live = false; break; }
                        uint8_t *A = sW + s * w_slot;
#pragma unroll
                        for (int j = 0; j < 4; j++) {
                            const int row = r0 + 32 * j;
                            const uint4 v = buf[u][j];
                            // word p of the 16 packed bytes covers 8 codes: low nibbles
                            // k 8p..8p+3, high nibbles 8p+4..8p+7 (k relative to 32*cp).
                            const uint4 c0 = make_uint4(v.x & 0x0F0F0F0Fu, (v.x >> 4) & 0x0F0F0F0Fu,
                                                        v.y & 0x0F0F0F0Fu, (v.y >> 4) & 0x0F0F0F0Fu);
                            const uint4 c1 = make_uint4(v.z & 0x0F0F0F0Fu, (v.z >> 4) & 0x0F0F0F0Fu,
                                                        v.w & 0x0F0F0F0Fu, (v.w >> 4) & 0x0F0F0F0Fu);
                            const int sw = row & 7;  // 128-byte swizzle of this row
                            *reinterpret_cast<uint4 *>(A + row * 128 + (((2 * cp) ^ sw) << 4)) = c0;
                            *reinterpret_cast<uint4 *>(A + row * 128 + (((2 * cp + 1) ^ sw) << 4)) = c1;
                        }
                        // refill this register slot with the iteration W4_PREFETCH ahead
                        if (ft < p.num_tiles) {
                            fetch(buf[u], ft, fkb);
                            if (++fkb == p.nkb) { fkb = 0; ft += (int)ncl; }
                        }
                        // every writer makes its stores visible to the async proxy and
                        // arrives locally; one thread collects the 128 arrivals (bounded) and
                        // announces the stage to the leader with one cluster-scope arrive
                        fence_proxy_async_smem();
                        mbar_arrive(&cdone[s]);
                        if (ct == 0) {
                            if (!mbar_wait(&cdone[s], ph, err, abort_flag)) live = false;
                            else mbar_arrive_remote(afull0 + 8u * s);
                        }
                        if (++s == (uint32_t)S) { s = 0; ph ^= 1; }
                        if (++kb == p.nkb) {
                            kb = 0;
                            t += (int)ncl;
                            live = t < p.num_tiles;
                        }
                    }
                }
            }
        }
    }

    tc_fence_before();
    __syncthreads();
    cluster_sync();  // neither CTA leaves while the pair may still touch its shared memory
    if (warp == 1) {
        tc_fence_after();
        tmem_dealloc_pair(tmem_base, p.tmem_cols);
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
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    return cudaLaunchKernelEx(&cfg, kern, wmap, amap, args);
}

template <int BITS>
int pair_capacity_t() {
    cudaLaunchConfig_t q{};
    q.gridDim = dim3(2);
    q.blockDim = dim3(gemm_threads<BITS>());
    q.dynamicSmemBytes = MAX_DYN_SMEM - 1024;
    cudaLaunchAttribute qa[1];
    qa[0].id = cudaLaunchAttributeClusterDimension;
    qa[0].val.clusterDim.x = 2;
    qa[0].val.clusterDim.y = 1;
    qa[0].val.clusterDim.z = 1;
    q.attrs = qa;
    q.numAttrs = 1;
    auto kern = gemm_kernel<BITS, __half>;
    if (cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, MAX_DYN_SMEM) !=
        cudaSuccess)
        return 0;
    int n = 0;
    if (cudaOccupancyMaxActiveClusters(&n, kern, &q) != cudaSuccess) return 0;
    return n;
}

}  // namespace

// How many CTA pairs of the GEMM the current device holds at once (TPCs whose two SMs are
// both available); the persistent grid is sized to it so every pair is resident.
int gemm_pair_capacity(int bits) { return bits == 8 ? pair_capacity_t<8>() : pair_capacity_t<4>(); }

GemmPlan plan_gemm(const WeightView &w, int rows, int max_pairs) {
    GemmPlan plan{};
    const int tiles_m = std::max(1, (rows + 255) / 256);
    int tok = (rows + tiles_m - 1) / tiles_m;
    tok = std::max(32, (tok + 31) / 32 * 32);  // 2-CTA MMA: N multiple of 32
    plan.tok = tok;
    const int stage_bytes = (tok / 2) * KB + A_SLOT;
    const int fixed = SMEM_RESERVE;
    const int stages = std::min(MAX_STAGES, (MAX_DYN_SMEM - fixed) / stage_bytes);
    plan.stages = stages;
    // One CTA per SM: each CTA of the pair allocates up to 512 TMEM columns.
    plan.smem_bytes = std::max(stages * stage_bytes + fixed, 120 * 1024);
    const int n_tok_tiles = (rows + tok - 1) / tok;
    plan.tiles = ((w.Np + CHT - 1) / CHT) * n_tok_tiles;
    plan.grid = 2 * std::min(plan.tiles, std::max(1, max_pairs));
    return plan;
}

cudaError_t launch_gemm(const WeightView &w, const CUtensorMap &wmap, const ActView &a,
                        const CUtensorMap &amap, const GemmPlan &plan, int rows, void *out,
                        int out_type, long long ldc, unsigned *err, bool pdl,
                        cudaStream_t stream) {
    GemmArgs args{};
    args.wq = w.w;
    args.Np = w.Np;
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
    uint32_t cols = 32;
    while (cols < (uint32_t)(2 * plan.tok)) cols <<= 1;
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
