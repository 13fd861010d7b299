// gemm_impl.cuh -- prefill path: int8 x (int4|int8) -> int32 on the 5th-generation tensor
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
//
// The kernel is instantiated for one output buffer in gemm_sm100.cu and for the split-N
// exchange (2, 4 or 8 destinations) in gemm_scatter.cu, so the two sets compile in parallel.
#pragma once
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
constexpr int A_SLOT = CH_CTA * KB;         // 16 KB 8-bit weights per CTA per stage
constexpr int P_SLOT = CH_CTA * KB / 2;     // 8 KB packed W4 weights per CTA per stage
// W4: the unpacked weights live in tensor memory, a ring of A_SLOTS 32-column slots (128 codes
// of each of the CTA's 128 channels per k-block) after the two accumulator buffers; so the
// token tile is at most 128 (2 x 128 accumulator columns).  The shared-memory ring of
// activation and packed-weight tiles is deeper (up to MAX_STAGES_W4), so the copies run
// further ahead of the unpacking.
constexpr uint32_t A_TMEM_COL = 256;
constexpr int W4_MAX_TOK = 128;
#ifndef QL_W4_CONV_BATCH
#define QL_W4_CONV_BATCH 1
#endif
constexpr int W4_CONV_BATCH = QL_W4_CONV_BATCH;  // stages a converter warp unpacks per wait
#ifndef QL_W4_CONV_GROUPS
#define QL_W4_CONV_GROUPS 1
#endif
// groups of 4 converter warps (one per tensor-memory lane quadrant); group g unpacks the
// k-block iterations it with it % W4_CONV_GROUPS == g
constexpr int W4_CONV_GROUPS = QL_W4_CONV_GROUPS;
constexpr int EPI_WARPS = 8;
constexpr int MAX_DYN_SMEM = 232448;        // 227 KB opt-in per block on sm_100
constexpr int SMEM_RESERVE = 1024 + 1024;   // alignment slack + barriers
constexpr int MAX_STAGES = 8;
constexpr int MAX_STAGES_W4 = 12;           // W4: a 16 KB stage (activations + packed weights)
constexpr int A_SLOTS = 8;                  // W4: unpacked-weight slots in tensor memory
// Stream-K workspace: the contribution counters first, at a fixed place for every plan (they
// must be zero before each launch, and the partial-sum buffers after them are overwritten
// with plan-dependent layouts), room for SK_MAX_PAIRS pairs x 2 * EPI_WARPS sub-blocks.
constexpr int SK_MAX_PAIRS = 256;
constexpr size_t SK_CNT_BYTES = (size_t)SK_MAX_PAIRS * 2 * EPI_WARPS * sizeof(int);

struct GemmArgs {
    const uint8_t *wq;     // W4 packed weights [Np][Kp/2] (read by the converter)
    int Np;
    const float *wscale;
    const float *ascale;
    const int32_t *rowsum;
    void *out;             // the output, when one buffer takes it (otherwise the OutputSet
                           // parameter of a SCATTER kernel)
    long long ldc;
    int M, N, nkb;
    int tok, stages, n_tok_tiles, num_tiles;
    uint32_t tmem_cols;
    unsigned *err;
    int sk;              // 1: stream-K; 2: tail split; 0: whole tiles strided over the pairs
    int sk_tiles;        // stream-K / tail split: the last sk_tiles tiles are split, the
                         // others whole
    long long units;     // stream-K: (channel tile, k-block) iterations of one token tile
                         // in the split region; tail split: sub-tiles per split tile
    int32_t *sk_ws;      // stream-K partial sums [pairs][left | right][tok][256]
    int *sk_cnt;         // contributions per (slot, epilogue sub-block) [256][16], zero
                         // between launches
};

// The work of one CTA pair, as a sequence of segments (tile t, k-blocks [kb0, kb1)).
// Data-parallel: whole tiles cid, cid + ncl, ...  Stream-K: whole tiles first, then a share
// of the split region.  The whole tiles are [0, T - sk_tiles), a whole number of waves,
// strided over the pairs.  The split region is the last sk_tiles tiles: the pairs form one
// group per token tile (pair cid serves token tile g = cid % G, G = n_tok_tiles, as the
// i = cid / G-th of the group's Pg = ncl / G pairs); each group walks the U = (sk_tiles /
// G) * nkb (channel tile, k-block) iterations of its token tile, pair i taking the
// contiguous range [i U / Pg, (i + 1) U / Pg) cut at tile boundaries, so every pair gets
// the same number of k-blocks (+-1) and the i-th pairs of all groups read the same weight
// tiles at the same time (one DRAM read, the other groups hit L2).  The split region is
// sized to absorb the imbalance of the last wave.  A split tile's segments are summed in a
// global workspace (int32 sums are exact in any order, so the result does not depend on
// which pair finishes first).  The split region comes last on purpose: measured on B200,
// the loads that sum a split tile wait behind the TMA weight stream for tens of
// microseconds while the main loops run, and are quick once it has ended.
//
// Tail split (sk == 2): the whole tiles are the first num_tiles - sk_tiles, a whole number of
// waves; each of the last sk_tiles tiles is cut along its tokens into `units` sub-tiles of
// tok / units tokens (whole k-loop each), sub-tile j going to pair j, so the last partial
// wave of big tiles becomes one short wave of small ones on otherwise idle pairs.  Sub-tile
// j is reported as t = num_tiles + j (tile_geom gives its coordinates).
struct Sched {
    long long u, end;  // split-region iterations still to walk
    int t_dp, dp_end, step, nkb, ntt, g, base, tail;
    __device__ Sched(const GemmArgs &p, int cid, int ncl)
        : t_dp(cid), step(ncl), nkb(p.nkb), ntt(p.n_tok_tiles), tail(-1) {
        if (p.sk == 1) {
            const int pg = ncl / ntt, i = cid / ntt;
            g = cid % ntt;
            u = p.units * i / pg;
            end = p.units * (i + 1) / pg;
            base = dp_end = p.num_tiles - p.sk_tiles;
        } else {
            g = base = 0;
            u = end = 0;
            dp_end = p.num_tiles;
            if (p.sk == 2) {
                dp_end = p.num_tiles - p.sk_tiles;
                if ((long long)cid < (long long)p.sk_tiles * p.units) tail = p.num_tiles + cid;
            }
        }
    }
    __device__ bool next(int &t, int &kb0, int &kb1) {
        if (t_dp < dp_end) {
            t = t_dp;
            kb0 = 0;
            kb1 = nkb;
            t_dp += step;
            return true;
        }
        if (tail >= 0) {
            t = tail;
            kb0 = 0;
            kb1 = nkb;
            tail = -1;
            return true;
        }
        if (u >= end) return false;
        const int tc = (int)(u / nkb);
        t = base + tc * ntt + g;
        kb0 = (int)(u - (long long)tc * nkb);
        const long long rem = end - u;
        kb1 = rem < (long long)(nkb - kb0) ? kb0 + (int)rem : nkb;
        u += kb1 - kb0;
        return true;
    }
};

// Coordinates of work item t (Sched::next): channel tile tc, first token tok0, tokens ntok
// (the MMA's N).
__device__ __forceinline__ void tile_geom(const GemmArgs &p, int t, int &tc, int &tok0, int &ntok) {
    if (t < p.num_tiles) {
        tc = t / p.n_tok_tiles;
        tok0 = (t - tc * p.n_tok_tiles) * p.tok;
        ntok = p.tok;
    } else {  // tail sub-tile j of split tile num_tiles - sk_tiles + j / units
        const int j = t - p.num_tiles, split = (int)p.units;
        const int tile = p.num_tiles - p.sk_tiles + j / split;
        tc = tile / p.n_tok_tiles;
        ntok = p.tok / split;
        tok0 = (tile - tc * p.n_tok_tiles) * p.tok + (j % split) * ntok;
    }
}

// The same sequence one k-block at a time.
struct Units {
    Sched s;
    int t = 0, kb = 0, k1 = 0;
    bool live;
    __device__ Units(const GemmArgs &p, int cid, int ncl) : s(p, cid, ncl) { live = s.next(t, kb, k1); }
    __device__ void advance() {
        if (++kb >= k1) live = s.next(t, kb, k1);
    }
};

// Stream-K: the workspace slot of split tile t and how many segments it is cut into.  In
// its token tile's group (Pg pairs, boundaries w_b = floor(b U / Pg)), the tile's range
// [s0, e0) is cut by the boundaries b in [1, Pg) with s0 < w_b < e0; the slot is
// g * Pg + (the first of them), distinct for every split tile.
__device__ __forceinline__ void sk_split(const GemmArgs &p, int ncl, int t, int &slot, int &nseg) {
    const int ntt = p.n_tok_tiles, tl = t - (p.num_tiles - p.sk_tiles);  // within the region
    const int g = tl % ntt, tc = tl / ntt;
    const long long pg = ncl / ntt;
    const long long s0 = (long long)tc * p.nkb, e0 = s0 + p.nkb, U = p.units;
    const long long bf = ((s0 + 1) * pg + U - 1) / U;  // first boundary with w_b > s0
    long long bl = (e0 * pg + U - 1) / U - 1;          // last boundary with w_b < e0
    if (bl > pg - 1) bl = pg - 1;
    slot = g * (int)pg + (int)bf;
    nseg = (int)(bl >= bf ? bl - bf + 1 : 0) + 1;
}

template <int BITS>
constexpr int gemm_threads() { return (2 + EPI_WARPS + (BITS == 4 ? 4 * W4_CONV_GROUPS : 0)) * 32; }

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

// NDST > 1: the epilogue stores every element to each of outs' NDST destinations (the
// split-N exchange); NDST == 1: to p.out alone, and outs is unused.  The destinations are a
// separate trailing parameter, not a GemmArgs field: growing GemmArgs changed the register
// allocation of the single-output kernel (168 -> 150 registers) and measured 2.2x slower on
// B200.
//
// GLU (8-bit weights, one output): the SiLU-gated product of a gate/up matrix (gate columns
// [0, N/2), up columns [N/2, N), the order src/model/checkpoint.rs:392-423 concatenates
// them) in the epilogue.  Channel tile tc covers the 128 output channels [128 tc, 128 tc +
// 128): CTA `rank` stages, per 32-row quadrant q of its weight slot, 16 gate rows
// c0 .. c0 + 15 and then the 16 up rows N/2 + c0 .. with c0 = 128 tc + 64 rank + 16 q (two
// boxes of 16 rows through `wmap`, whose box is 16 rows high).  So lane l < 16 of the
// epilogue warp of quadrant q holds gate channel c0 + l and lane l + 16 its up channel: one
// shuffle per token pair hands each lane the other half, and each lane stores
// silu(g) * u (src/npu.rs:1202-1208) for every other token.  No [M][N] intermediate.
template <int BITS, typename OutT, int NDST, bool GLU = false>
__global__ void __launch_bounds__(gemm_threads<BITS>(), 1)
    gemm_kernel(const __grid_constant__ CUtensorMap wmap, const __grid_constant__ CUtensorMap amap,
                const GemmArgs p, const OutputSet outs,
                const __grid_constant__ CUtensorMap amap_sub) {
    // NDST == 0: one destination, the NVSwitch multicast address of every rank's buffer
    // (multimem stores: the switch writes each element into every GPU's copy)
    constexpr bool MCAST = NDST == 0;
    constexpr bool SCATTER = NDST > 1 || MCAST;
    constexpr int NPTR = MCAST ? 1 : NDST;
    extern __shared__ uint8_t smem_raw[];
    uint8_t *smem = reinterpret_cast<uint8_t *>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                                ~uintptr_t(1023));
    const int S = p.stages;
    const int tok = p.tok;
    const int b_half = (tok / 2) * KB;                    // this CTA's activation rows
    // weights per stage: W8 the [128][128] tile (128-byte swizzle), W4 the packed [128][64]
    // tile (64-byte swizzle) that the converter unpacks into tensor memory
    constexpr int w_slot = BITS == 8 ? A_SLOT : P_SLOT;
    uint8_t *sB = smem;              // [S][tok/2][128]
    uint8_t *sW = sB + S * b_half;   // [S][w_slot]
    uint64_t *bars = reinterpret_cast<uint64_t *>(sW + S * w_slot);
    uint64_t *full = bars;              // [S] leader: both CTAs' activation (W8: + weight) bytes
    uint64_t *empty = full + S;         // [S] the MMA is done with the stage
    uint64_t *wfull = empty + S;        // [S] W4: this CTA's packed weight tile landed
    uint64_t *afull = wfull + S;        // [A_SLOTS] W4, leader: both converters filled the slot
    uint64_t *cdone = afull + A_SLOTS;  // [A_SLOTS] W4: this CTA's 128 converter threads did
    uint64_t *aempty = cdone + A_SLOTS; // [A_SLOTS] W4: the MMA is done with the slot
    uint64_t *accf = aempty + A_SLOTS;  // [2] accumulators ready for the epilogue
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
            mbar_init(&wfull[s], 1);
        }
        for (int a = 0; a < A_SLOTS; a++) {
            mbar_init(&afull[a], 2);
            mbar_init(&cdone[a], 128);
            mbar_init(&aempty[a], 1);
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
        if (p.sk == 2) tma_prefetch_desc(&amap_sub);
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

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            // tx: the bytes the leader's `full` barrier receives for the stage from both CTAs
            auto load_weights = [&](int s, int kb, int tc, uint32_t tx) {
                if constexpr (BITS == 4) {
                    // this CTA's packed tile, counted on its own barrier (the converter's)
                    if constexpr (GLU) {
#pragma unroll
                        for (int b = 0; b < 8; b++)
                            tma_load_2d(sW + s * w_slot + b * 16 * (KB / 2), &wmap, &wfull[s],
                                        kb * (KB / 2),
                                        (b & 1) * (p.N / 2) + tc * CH_CTA + (int)rank * 64 +
                                            (b >> 1) * 16);
                    } else {
                        tma_load_2d(sW + s * w_slot, &wmap, &wfull[s], kb * (KB / 2),
                                    tc * CHT + (int)rank * CH_CTA);
                    }
                    mbar_arrive_expect_tx(&wfull[s], (uint32_t)P_SLOT);
                } else if constexpr (GLU) {
                    // quadrant q: gate rows c0 .. c0 + 15, then up rows N/2 + c0 ..
#pragma unroll
                    for (int b = 0; b < 8; b++)
                        tma_load_2d_pair(sW + s * w_slot + b * 16 * KB, &wmap, full0 + 8u * s,
                                         kb * KB,
                                         (b & 1) * (p.N / 2) + tc * CH_CTA + (int)rank * 64 +
                                             (b >> 1) * 16);
                } else if (BITS == 8) {
                    tma_load_2d_pair(sW + s * w_slot, &wmap, full0 + 8u * s, kb * KB,
                                     tc * CHT + (int)rank * CH_CTA);
                }
                if (rank == 0) mbar_arrive_expect_tx(&full[s], tx);
            };
            // Weight tiles of the first stages do not depend on the preceding kernel:
            // issue them before waiting for it.
            int pre = 0;
            {
                Sched sp(p, (int)cid, (int)ncl);
                int t, kb0, kb1;
                while (pre < S && sp.next(t, kb0, kb1)) {
                    int tc, tok0, ntok;
                    tile_geom(p, t, tc, tok0, ntok);
                    const uint32_t tx = 2u * (uint32_t)((ntok / 2) * KB + (BITS == 8 ? A_SLOT : 0));
                    for (int kb = kb0; kb < kb1 && pre < S; kb++) load_weights(pre++, kb, tc, tx);
                }
            }
            grid_dep_wait();
            uint32_t it = 0, s = 0, ph = 0;  // iteration, stage, stage phase
            bool ok = true;
            Sched sp(p, (int)cid, (int)ncl);
            int t, kb0, kb1;
            while (ok && sp.next(t, kb0, kb1)) {
                int tc, tok0, ntok;
                tile_geom(p, t, tc, tok0, ntok);
                // a tail sub-tile loads only its own activation rows (a box of ntok/2 rows)
                const CUtensorMap *am = ntok == tok ? &amap : &amap_sub;
                const uint32_t tx = 2u * (uint32_t)((ntok / 2) * KB + (BITS == 8 ? A_SLOT : 0));
                for (int kb = kb0; kb < kb1; kb++, it++) {
                    if (it >= (uint32_t)pre) {
                        if (!(ok = mbar_wait(&empty[s], ph ^ 1, err, abort_flag))) break;
                        load_weights(s, kb, tc, tx);
                    }
                    tma_load_2d_pair(sB + s * b_half, am, full0 + 8u * s, kb * KB,
                                     tok0 + (int)rank * (ntok / 2));
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
                    if (BITS == 4) mbar_wait(&wfull[j % S], (j / S) & 1, nullptr, &never);
                }
            }
        }
    } else if (warp == 1) {
        // ------------------------------------------------------------ MMA issuer (leader)
        if (lane == 0 && rank == 0) {
            uint32_t s = 0, ph = 0, local = 0;
            uint32_t as = 0, aph = 0;  // W4: tensor-memory slot of the unpacked weights
            bool ok = true;
            Sched sm(p, (int)cid, (int)ncl);
            int t, kb0, kb1;
            for (; ok && sm.next(t, kb0, kb1); local++) {
                const int ab = local & 1;
                if (!(ok = mbar_wait(&acce[ab], ((local >> 1) & 1) ^ 1, err, abort_flag))) break;
                tc_fence_after();
                const uint32_t d = tmem_base + (uint32_t)(ab * tok);
                int tc, tok0, ntok;
                tile_geom(p, t, tc, tok0, ntok);
                const uint32_t idesc = idesc_i8(2 * CH_CTA, ntok, BITS == 8, true);
                for (int kb = kb0; kb < kb1; kb++) {
                    if (!(ok = mbar_wait(&full[s], ph, err, abort_flag))) break;
                    if (BITS == 4 && !(ok = mbar_wait(&afull[as], aph, err, abort_flag))) break;
                    tc_fence_after();
                    const uint64_t bdesc = smem_desc_sw128_k(sB + s * b_half);
                    if constexpr (BITS == 4) {
                        // A: the stage's unpacked weights in tensor memory, 8 columns per MMA
                        const uint32_t at = tmem_base + A_TMEM_COL + 32u * as;
#pragma unroll
                        for (int k = 0; k < KB / 32; k++)
                            mma_i8_ts_pair(d, at + 8 * k, bdesc + 2 * k, idesc, kb != kb0 || k != 0);
                    } else {
                        const uint64_t adesc = smem_desc_sw128_k(sW + s * w_slot);
#pragma unroll
                        for (int k = 0; k < KB / 32; k++)
                            mma_i8_ss_pair(d, adesc + 2 * k, bdesc + 2 * k, idesc, kb != kb0 || k != 0);
                    }
                    mma_commit_pair(&empty[s], 0x3);
                    if (++s == (uint32_t)S) { s = 0; ph ^= 1; }
                    if constexpr (BITS == 4) {
                        mma_commit_pair(&aempty[as], 0x3);
                        if (++as == (uint32_t)A_SLOTS) { as = 0; aph ^= 1; }
                    }
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
        const int sub = (int)rank * EPI_WARPS + (warp - 2);  // this warp's part of a tile
        const int tl = (int)rank * CH_CTA + q * 32 + lane;  // tensor-memory lane in the tile
        const int chl = GLU ? (int)rank * 64 + q * 16 + (lane & 15)  // output channel
                            : tl;                                    // channel within the tile
        uint32_t local = 0;
        // Activation scales (and W4 row sums) of this warp's columns, loaded once per tile:
        // column c of the warp's range sits in lane c % 32 of register c / 32.
        float sa_r[4];
        int rs_r[4];
        auto load_scales = [&](int tok_base, int cols) {
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const int m = tok_base + i * 32 + lane;
                const bool v = i * 32 + lane < cols && m < p.M;
                sa_r[i] = v ? p.ascale[m] : 0.0f;
                rs_r[i] = (BITS == 4 && v) ? p.rowsum[m] : 0;
            }
        };
        OutT *out = static_cast<OutT *>(p.out);
        // The exchange's destinations, held in registers.  (Measured on B200: a predicated
        // store per slot of the parameter array made a 16-token chunk's stores ~5x slower
        // than these unconditional ones.)
        OutT *od[NPTR];
        if constexpr (SCATTER) {
#pragma unroll
            for (int d = 0; d < NPTR; d++) od[d] = static_cast<OutT *>(outs.dst[d]) + outs.col0;
        }
        // Multicast stores of chunk cc: multimem stores are at least 32 bits wide, so for fp16
        // the lanes of a pair (channels 2i, 2i + 1) swap one value per token pair and each
        // stores one channel pair: the even lane token 2t, the odd lane token 2t + 1.  (The
        // output's column offset and row stride are even, so the pair is 4-byte aligned.)
        auto emit16_mc = [&](const uint32_t (&r)[16], int cc, int tok_base, int ch, bool chv,
                             float sw) {
            uint32_t v[16];
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int src = (cc & 1) * 16 + j;
                const float sa = __shfl_sync(0xffffffffu, sa_r[cc >> 1], src);
                const int rs = __shfl_sync(0xffffffffu, rs_r[cc >> 1], src);
                int acc = (int)r[j];
                if (BITS == 4) acc -= 8 * rs;
                if constexpr (std::is_same<OutT, int32_t>::value)
                    v[j] = (uint32_t)acc;
                else if constexpr (std::is_same<OutT, float>::value)
                    v[j] = __float_as_uint(__fmul_rn(__fmul_rn(__int2float_rn(acc), sa), sw));
                else
                    v[j] = (uint32_t)__half_as_ushort(
                        __float2half_rn(__fmul_rn(__fmul_rn(__int2float_rn(acc), sa), sw)));
            }
            const int m0 = tok_base + cc * 16;
            if constexpr (std::is_same<OutT, __half>::value) {
                const bool odd = (lane & 1) != 0;
#pragma unroll
                for (int t = 0; t < 8; t++) {
                    const uint32_t other =
                        __shfl_xor_sync(0xffffffffu, odd ? v[2 * t] : v[2 * t + 1], 1);
                    const int m = m0 + 2 * t + (odd ? 1 : 0);
                    if (chv && m < p.M) {
                        const uint32_t pair = odd ? (other | (v[2 * t + 1] << 16))
                                                  : (v[2 * t] | (other << 16));
                        multimem_st_b32(od[0] + (long long)m * p.ldc + (ch & ~1), pair);
                    }
                }
            } else {
#pragma unroll
                for (int j = 0; j < 16; j++)
                    if (chv && m0 + j < p.M)
                        multimem_st_b32(od[0] + (long long)(m0 + j) * p.ldc + ch, v[j]);
            }
        };
        // dequantise and store chunk cc (columns 16 cc .. 16 cc + 15 of the warp's range)
        auto emit16 = [&](const uint32_t (&r)[16], int cc, int tok_base, int ch, bool chv,
                          float sw) {
            if constexpr (MCAST) {
                emit16_mc(r, cc, tok_base, ch, chv, sw);
                return;
            }
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int src = (cc & 1) * 16 + j;
                const float sa = __shfl_sync(0xffffffffu, sa_r[cc >> 1], src);
                const int rs = __shfl_sync(0xffffffffu, rs_r[cc >> 1], src);
                const int m = tok_base + cc * 16 + j;
                if (chv && m < p.M) {
                    int acc = (int)r[j];
                    if (BITS == 4) acc -= 8 * rs;
                    if constexpr (!SCATTER) {
                        if constexpr (std::is_same<OutT, int32_t>::value) {
                            out[(long long)m * p.ldc + ch] = acc;
                        } else {
                            const float y = __fmul_rn(__fmul_rn(__int2float_rn(acc), sa), sw);
                            out[(long long)m * p.ldc + ch] = OutCvt<OutT>::from(y);
                        }
                    } else {
                        OutT v;
                        if constexpr (std::is_same<OutT, int32_t>::value)
                            v = acc;
                        else
                            v = OutCvt<OutT>::from(
                                __fmul_rn(__fmul_rn(__int2float_rn(acc), sa), sw));
                        const long long idx = (long long)m * p.ldc + ch;
#pragma unroll
                        for (int d = 0; d < NPTR; d++) od[d][idx] = v;
                    }
                }
            }
        };
        // GLU: dequantise chunk cc, swap halves with the partner lane (l ^ 16), and store
        // silu(g) * u: gate lanes the chunk's even tokens, up lanes the odd ones.
        auto emit16_glu = [&](const uint32_t (&r)[16], int cc, int tok_base, int ch, bool chv,
                              float sw) {
            const bool up = lane >= 16;
            float y[16];
#pragma unroll
            for (int j = 0; j < 16; j++) {
                const int src = (cc & 1) * 16 + j;
                const float sa = __shfl_sync(0xffffffffu, sa_r[cc >> 1], src);
                const int rs = __shfl_sync(0xffffffffu, rs_r[cc >> 1], src);
                int acc = (int)r[j];
                if (BITS == 4) acc -= 8 * rs;
                y[j] = __fmul_rn(__fmul_rn(__int2float_rn(acc), sa), sw);
            }
#pragma unroll
            for (int i = 0; i < 8; i++) {
                const float other = __shfl_xor_sync(0xffffffffu, up ? y[2 * i] : y[2 * i + 1], 16);
                const float g = up ? other : y[2 * i];
                const float u = up ? y[2 * i + 1] : other;
                const int m = tok_base + cc * 16 + 2 * i + (up ? 1 : 0);
                if constexpr (!std::is_same<OutT, int32_t>::value) {
                    if (chv && m < p.M) {
                        const float v = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), u);
                        out[(long long)m * p.ldc + ch] = OutCvt<OutT>::from(v);
                    }
                }
            }
        };
        const int pg = p.sk == 1 ? (int)ncl / p.n_tok_tiles : 1;  // stream-K pairs per group
        Sched se(p, (int)cid, (int)ncl);
        int t, kb0, kb1;
        for (; se.next(t, kb0, kb1); local++) {
            int tc, tok0, ntok;
            tile_geom(p, t, tc, tok0, ntok);
            const int cols = ntok / 2;  // this warp's columns: <= 128, at most 8 chunks of 16
            const int ab = local & 1;
            // every lane waits (bounded); the warp leaves together if any lane gave up,
            // so the warp-collective tcgen05.ld / shuffles below stay converged
            const bool okw = mbar_wait(&accf[ab], (local >> 1) & 1, err, abort_flag);
            if (!__all_sync(0xffffffffu, okw)) break;
            tc_fence_after();
            const int ch = GLU ? tc * CH_CTA + chl : tc * CHT + chl;
            const bool chv = ch < (GLU ? p.N / 2 : p.N);
            const int tok_base = tok0 + colh * cols;
            const uint32_t taddr = tmem_base + ((uint32_t)(q * 32) << 16) +
                                   (uint32_t)(ab * tok + colh * cols);
            if (kb0 == 0 && kb1 == p.nkb) {
                // the whole tile: dequantise from tensor memory
                const float sw =
                    chv ? p.wscale[(GLU && lane >= 16 ? p.N / 2 : 0) + ch] : 0.0f;
                load_scales(tok_base, cols);
#pragma unroll
                for (int cc = 0; cc < 8; cc++) {
                    if (cc * 16 >= cols) break;
                    uint32_t r[16];
                    tmem_ld16(taddr + cc * 16, r);
                    tmem_ld_wait();
                    if constexpr (GLU)
                        emit16_glu(r, cc, tok_base, ch, chv, sw);
                    else
                        emit16(r, cc, tok_base, ch, chv, sw);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive_remote_tc(acce0 + 8u * ab);
                continue;
            }
            // A segment of a split tile.  Its partial sums go to its own workspace buffer
            // ([tok][256] int32, lanes = consecutive channels): the tile's first segment
            // (it ends at the tile's first boundary b_f) to "left" of b_f, every other one
            // to "right" of the pair boundary it starts at.  Then the contribution is
            // counted; the warp that completes the count for its sub-block adds the tile's
            // nseg buffers and finishes the sub-block.
            int slot, nseg;
            sk_split(p, (int)ncl, t, slot, nseg);  // slot = g * pg + b_f
            const int g = (t - (p.num_tiles - p.sk_tiles)) % p.n_tok_tiles;
            const int bstart = kb0 == 0 ? slot : g * pg + (int)cid / p.n_tok_tiles;
            int32_t *mine = p.sk_ws + ((long long)(2 * bstart + (kb0 == 0 ? 0 : 1)) * tok) * CHT;
            // the partial sums stay in L2 until the finishing warp reads them (the weight
            // stream would otherwise push them out to DRAM, where their reads queue behind it)
            const uint64_t keep = l2_policy_evict_last();
#pragma unroll
            for (int cc = 0; cc < 8; cc++) {
                if (cc * 16 >= cols) break;
                uint32_t r[16];
                tmem_ld16(taddr + cc * 16, r);
                tmem_ld_wait();
                const int col0 = colh * cols + cc * 16;
#pragma unroll
                for (int j = 0; j < 16; j++)
                    st_l2_hint(mine + (long long)(col0 + j) * CHT + tl, (int)r[j], keep);
            }
            tc_fence_before();
            __syncwarp();
            if (lane == 0) mbar_arrive_remote_tc(acce0 + 8u * ab);  // tensor memory is free
            __threadfence();
            __syncwarp();
            int last = 0;
            if (lane == 0) last = atomicAdd(p.sk_cnt + slot * (2 * EPI_WARPS) + sub, 1) == nseg - 1;
            last = __shfl_sync(0xffffffffu, last, 0);
            if (!last) continue;
            __threadfence();
            const float sw =
                chv ? p.wscale[(GLU && lane >= 16 ? p.N / 2 : 0) + ch] : 0.0f;
            load_scales(tok_base, cols);
            // the tile's buffers: left of b_f, right of b_f .. b_f + nseg - 2.  Two chunks at
            // a time, the loads of both first buffers issued together: under the main loops'
            // traffic an L2 round trip costs microseconds, so the number of dependent
            // round trips, not the bytes, sets the time of this pass.
            const uint64_t drop = l2_policy_evict_first();
            const int32_t *left = p.sk_ws + ((long long)(2 * slot) * tok) * CHT;
            const int32_t *right0 = p.sk_ws + ((long long)(2 * slot + 1) * tok) * CHT;
#pragma unroll
            for (int cc = 0; cc < 8; cc += 2) {
                if (cc * 16 >= cols) break;
                const bool two = (cc + 1) * 16 < cols;
                const int col0 = colh * cols + cc * 16;
                uint32_t r[2][16], q2[2][16];
#pragma unroll
                for (int h = 0; h < 2; h++)
#pragma unroll
                    for (int j = 0; j < 16; j++) {
                        const long long off = (long long)(col0 + h * 16 + j) * CHT + tl;
                        r[h][j] = (h == 0 || two) ? (uint32_t)ld_l2_hint(left + off, drop) : 0u;
                        q2[h][j] = (h == 0 || two) ? (uint32_t)ld_l2_hint(right0 + off, drop) : 0u;
                    }
#pragma unroll
                for (int h = 0; h < 2; h++)
#pragma unroll
                    for (int j = 0; j < 16; j++) r[h][j] += q2[h][j];
                for (int sgi = 1; sgi < nseg - 1; sgi++) {  // tiles cut into three or more
                    const int32_t *right = p.sk_ws + ((long long)(2 * (slot + sgi) + 1) * tok) * CHT;
#pragma unroll
                    for (int h = 0; h < 2; h++)
#pragma unroll
                        for (int j = 0; j < 16; j++)
                            if (h == 0 || two)
                                r[h][j] += (uint32_t)ld_l2_hint(
                                    right + (long long)(col0 + h * 16 + j) * CHT + tl, drop);
                }
                if constexpr (GLU) {
                    emit16_glu(r[0], cc, tok_base, ch, chv, sw);
                    if (two) emit16_glu(r[1], cc + 1, tok_base, ch, chv, sw);
                } else {
                    emit16(r[0], cc, tok_base, ch, chv, sw);
                    if (two) emit16(r[1], cc + 1, tok_base, ch, chv, sw);
                }
            }
            if (lane == 0) p.sk_cnt[slot * (2 * EPI_WARPS) + sub] = 0;
        }
        // peers' copies of the output: visible system-wide before the next work on this
        // stream (the collective that tells the peers the output is complete)
        if constexpr (SCATTER) __threadfence_system();
    } else {
        // ------------------------------------------------------------ W4 converter
        // Thread (warp w, lane l) owns tensor-memory lane 32 (w % 4) + l, i.e. row 32 (w % 4) + l
        // of the CTA's weight slot (a warp may only access its own lane quadrant).  Per stage
        // it reads its row's 64 packed bytes from shared memory (64-byte swizzle: 16-byte
        // chunk c of row r sits at chunk c ^ ((r >> 1) & 3), so the warp's reads are
        // conflict-free), unpacks them and writes the 128 codes to the stage's 32 columns
        // of tensor memory.  Nibbles stay offset-binary (u = code + 8; A is declared
        // unsigned), so the unpack is two masks per word and the epilogue subtracts
        // 8 * sum_k q[m][k].  Word i of a row's 16 covers k = 8i .. 8i + 7: its low nibbles
        // k 8i .. 8i + 3 (column 2i), its high nibbles 8i + 4 .. 8i + 7 (column 2i + 1).
        if constexpr (BITS == 4) {
            const int ct = threadIdx.x - (2 + EPI_WARPS) * 32;  // 0 .. 128 groups - 1
            const int grp = ct >> 7;
            const int q = warp & 3;
            const int row = q * 32 + lane;
            const int swz = (row >> 1) & 3;
            const uint32_t tcol = tmem_base + ((uint32_t)(q * 32) << 16) + A_TMEM_COL;
            uint32_t s = 0, ph = 0;    // shared-memory stage of the packed tile
            uint32_t as = 0, aph = 0;  // tensor-memory slot it is unpacked into
            Units cu(p, (int)cid, (int)ncl);
            bool okw = true;
            uint32_t it = 0;
            while (cu.live && okw) {
                // W4_CONV_BATCH stages per round: their tensor-memory writes complete under
                // one tcgen05.wait::st before the stages are announced
                uint32_t bs[W4_CONV_BATCH], bp[W4_CONV_BATCH];
                int nb = 0;
#pragma unroll
                for (int b = 0; b < W4_CONV_BATCH; b++) {
                    // the other groups' iterations
                    while (W4_CONV_GROUPS > 1 && cu.live && (int)(it % W4_CONV_GROUPS) != grp) {
                        if (++s == (uint32_t)S) { s = 0; ph ^= 1; }
                        if (++as == (uint32_t)A_SLOTS) { as = 0; aph ^= 1; }
                        cu.advance();
                        it++;
                    }
                    if (!cu.live) break;
                    // the MMA released the tensor-memory slot (iteration it - A_SLOTS) and this
                    // iteration's packed tile landed; the warp stays converged
                    okw = mbar_wait(&aempty[as], aph ^ 1, err, abort_flag) &&
                          mbar_wait(&wfull[s], ph, err, abort_flag);
                    if (!__all_sync(0xffffffffu, okw)) { okw = false; break; }
                    const uint8_t *P = sW + s * w_slot + row * (KB / 2);
                    uint32_t u[32];
#pragma unroll
                    for (int c = 0; c < 4; c++) {
                        const uint4 v = *reinterpret_cast<const uint4 *>(P + 16 * (c ^ swz));
                        const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                        for (int i = 0; i < 4; i++) {
                            u[8 * c + 2 * i] = w4[i] & 0x0F0F0F0Fu;
                            u[8 * c + 2 * i + 1] = (w4[i] >> 4) & 0x0F0F0F0Fu;
                        }
                    }
                    tmem_st32(tcol + 32u * as, u);
                    bs[nb] = as;
                    bp[nb] = aph;
                    nb++;
                    if (++s == (uint32_t)S) { s = 0; ph ^= 1; }
                    if (++as == (uint32_t)A_SLOTS) { as = 0; aph ^= 1; }
                    cu.advance();
                    it++;
                }
                if (!okw) break;
                if (nb == 0) break;
                tmem_st_wait();
                // the writes before the arrivals, ordered for the MMAs issued after the wait
                tc_fence_before();
#pragma unroll
                for (int b = 0; b < W4_CONV_BATCH; b++)
                    if (b < nb) mbar_arrive(&cdone[bs[b]]);
                if ((ct & 127) == 0) {
#pragma unroll
                    for (int b = 0; b < W4_CONV_BATCH; b++) {
                        if (b >= nb || !okw) break;
                        if (!mbar_wait(&cdone[bs[b]], bp[b], err, abort_flag)) okw = false;
                        else mbar_arrive_remote_tc(afull0 + 8u * bs[b]);
                    }
                }
                okw = __all_sync(0xffffffffu, okw);
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

template <int BITS, typename OutT, int NDST, bool GLU = false>
cudaError_t launch_s(const CUtensorMap &wmap, const CUtensorMap &amap,
                     const CUtensorMap &amap_sub, const GemmArgs &args,
                     const OutputSet &outs, const GemmPlan &plan, bool pdl,
                     cudaStream_t stream) {
    auto kern = gemm_kernel<BITS, OutT, NDST, GLU>;
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
    return cudaLaunchKernelEx(&cfg, kern, wmap, amap, args, outs, amap_sub);
}

// The kernel's arguments for a launch (the output pointer is set by the caller).
inline GemmArgs make_args(const WeightView &w, const ActView &a, const GemmPlan &plan, int rows,
                          long long ldc, unsigned *err, void *sk_ws) {
    GemmArgs args{};
    args.wq = w.w;
    args.Np = w.Np;
    args.wscale = w.scales;
    args.ascale = a.scales;
    args.rowsum = a.rowsums;
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
    // W4: the accumulators and the ring of unpacked weights (A_TMEM_COL + 8 x 32 columns)
    args.tmem_cols = w.bits == 4 ? 512u : cols;
    args.err = err;
    args.sk_tiles = plan.sk_tiles;
    if (plan.sk == 2) {  // tail split: sub-tiles per split tile, no workspace
        args.sk = 2;
        args.units = plan.split;
        return args;
    }
    args.units = (long long)(plan.sk_tiles / args.n_tok_tiles) * args.nkb;
    args.sk = plan.sk == 1 && sk_ws && plan.grid / 2 <= SK_MAX_PAIRS ? 1 : 0;
    if (args.sk) {
        args.sk_cnt = static_cast<int *>(sk_ws);
        args.sk_ws = reinterpret_cast<int32_t *>(static_cast<char *>(sk_ws) + SK_CNT_BYTES);
    }
    return args;
}

// Launches the NDST-destination kernel for the weights' bits and the output type.
template <int NDST>
cudaError_t launch_n(const CUtensorMap &wmap, const CUtensorMap &amap,
                     const CUtensorMap &amap_sub, const GemmArgs &args,
                     const OutputSet &outs, const GemmPlan &plan, int bits, int out_type, bool pdl,
                     cudaStream_t stream) {
    if (bits == 8) {
        if (out_type == kF16) return launch_s<8, __half, NDST>(wmap, amap, amap_sub, args, outs, plan, pdl, stream);
        if (out_type == kF32) return launch_s<8, float, NDST>(wmap, amap, amap_sub, args, outs, plan, pdl, stream);
        return launch_s<8, int32_t, NDST>(wmap, amap, amap_sub, args, outs, plan, pdl, stream);
    }
    if (out_type == kF16) return launch_s<4, __half, NDST>(wmap, amap, amap_sub, args, outs, plan, pdl, stream);
    if (out_type == kF32) return launch_s<4, float, NDST>(wmap, amap, amap_sub, args, outs, plan, pdl, stream);
    return launch_s<4, int32_t, NDST>(wmap, amap, amap_sub, args, outs, plan, pdl, stream);
}

}  // namespace

}  // namespace ql
