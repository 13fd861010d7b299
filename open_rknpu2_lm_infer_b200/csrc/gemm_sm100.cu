// gemm_sm100.cu -- prefill path, one output buffer: plan, pair capacity and launch; the
// tcgen05 kernel itself is in gemm_impl.cuh.
#include "gemm_impl.cuh"

namespace ql {

namespace {

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
    auto kern = gemm_kernel<BITS, __half, 1>;
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

GemmPlan plan_gemm(const WeightView &w, int rows, int max_pairs, bool allow_sk) {
    GemmPlan plan{};
    // W4 keeps its unpacked weights in tensor memory beside the accumulators: token tiles
    // of at most 128
#ifndef QL_W8_MAX_TOK
#define QL_W8_MAX_TOK 256
#endif
    const int tok_max = w.bits == 4 ? W4_MAX_TOK : QL_W8_MAX_TOK;
    const int tiles_m = std::max(1, (rows + tok_max - 1) / tok_max);
    int tok = (rows + tiles_m - 1) / tiles_m;
    tok = std::max(32, (tok + 31) / 32 * 32);  // 2-CTA MMA: N multiple of 32
    // A narrow weight shard (split-N over many GPUs) leaves pairs idle: halve the token tile
    // while twice the tiles still run in one wave on the pairs (not below 64 tokens, where
    // the weight operand's shared-memory traffic per multiply-accumulate starts to bound the
    // MMA).  cfg4 at M=512 on 8 GPUs: 28 tiles of 256 tokens -> 56 of 128 on 74 pairs.
    {
        const long long ch_tiles = (w.Np + CHT - 1) / CHT;
        while (tok >= 128 && tok % 64 == 0 &&
               ch_tiles * ((rows + tok / 2 - 1) / (tok / 2)) <= std::max(1, max_pairs))
            tok /= 2;
    }
    plan.tok = tok;
    const int stage_bytes = (tok / 2) * KB + (w.bits == 8 ? A_SLOT : P_SLOT);
    const int fixed = SMEM_RESERVE;
    const int stages = std::min(w.bits == 4 ? MAX_STAGES_W4 : MAX_STAGES,
                                (MAX_DYN_SMEM - fixed) / stage_bytes);
    plan.stages = stages;
    // One CTA per SM: each CTA of the pair allocates up to 512 TMEM columns.
    plan.smem_bytes = std::max(stages * stage_bytes + fixed, 120 * 1024);
    const int n_tok_tiles = (rows + tok - 1) / tok;
    plan.tiles = ((w.Np + CHT - 1) / CHT) * n_tok_tiles;
    // Whole tiles strided over the pairs.  With allow_sk, stream-K where that leaves much of
    // the GPU idle (fewer tiles than pairs, or a mostly empty last wave: cfg4 at M=512 runs
    // 224 tiles on 74 pairs in 4 waves for 3.03 waves of work), on (nearly) every resident
    // pair -- a multiple of the token tiles, one group per token tile -- provided the k-loop
    // is long enough that cutting it costs little.  Measured on B200 it balances the main
    // loops as intended (every pair's last MMA within ~1 us of the others) but the pass
    // that finishes split tiles is bound by the epilogue's output stores (one 16-token
    // chunk of a warp's fp16 stores takes ~1.3 us while the main loops run, ~3.5 us when
    // every pair finishes at once), so it loses to whole tiles on every shape tried
    // (cfg4 M=512: 122 vs 108 us per call) and is off unless asked for.
    const int maxp = std::max(1, max_pairs);
    const int dp_pairs = std::min(plan.tiles, maxp);
    const long long waves = (plan.tiles + dp_pairs - 1) / dp_pairs;
    const int nkb = w.Kp / KB;
    const long long ch_tiles = (w.Np + CHT - 1) / CHT;
    const long long group = std::min<long long>(maxp / n_tok_tiles, ch_tiles * nkb);
    plan.sk = 0;
    plan.sk_tiles = 0;
    if (allow_sk && group >= 1 && nkb >= 8) {
        const long long sk_pairs = group * n_tok_tiles;
        // stream-K's balanced work vs the data-parallel waves, both on the whole GPU
        const double dp_eff = (double)plan.tiles / ((double)waves * maxp);
        const double sk_eff = (double)sk_pairs / maxp;
        if (dp_eff < 0.9 && sk_eff > dp_eff + 0.05) {
            plan.sk = 1;
            // whole waves of whole tiles after the split region (keep at least one wave's
            // worth of tiles, and the last partial wave, split)
            const long long whole = std::max<long long>(0, plan.tiles / sk_pairs - 1);
            plan.sk_tiles = (int)(plan.tiles - whole * sk_pairs);
        }
    }
    // Tail split: R tiles left for a last partial wave of whole tiles (at most half the
    // pairs busy) are each cut along their tokens into S sub-tiles (S a power of two, S*R
    // pairs, >= 32 tokens each) that run at once on otherwise idle pairs.  Each sub-tile
    // still streams its tile's whole weight block, but from L2 after the first.  cfg4 at
    // M=512: 224 tiles on 74 pairs = 3 waves + 2 tiles; the 2 tiles become 16 sub-tiles of
    // 32 tokens.
    plan.split = 1;
    if (!plan.sk && plan.tiles > maxp) {
        const int R = plan.tiles % maxp;
        int S = 1;
        while (R > 0 && 2 * S * R <= maxp && tok / (2 * S) >= 32 && (tok / (2 * S)) % 32 == 0)
            S *= 2;
        if (S > 1) {
            plan.sk = 2;
            plan.sk_tiles = R;
            plan.split = S;
        }
    }
    const int pairs = plan.sk == 1 ? (int)(group * n_tok_tiles) : dp_pairs;
    plan.grid = 2 * pairs;
    return plan;
}

size_t gemm_sk_bytes(const GemmPlan &plan) {
    if (plan.sk != 1) return 0;
    const size_t pairs = (size_t)plan.grid / 2;
    return SK_CNT_BYTES + 2 * pairs * (size_t)plan.tok * CHT * sizeof(int32_t);
}

cudaError_t launch_gemm(const WeightView &w, const CUtensorMap &wmap, const ActView &a,
                        const CUtensorMap &amap, const CUtensorMap &amap_sub,
                        const GemmPlan &plan, int rows,
                        const OutputSet &out, int out_type, long long ldc, unsigned *err,
                        void *sk_ws, bool pdl, cudaStream_t stream) {
    if (out.count < 1 || out.count > kMaxOutputs) return cudaErrorInvalidValue;
    if (out.count > 1)
        return launch_gemm_scatter(w, wmap, a, amap, amap_sub, plan, rows, out, out_type, ldc,
                                   err, sk_ws,
                                   pdl, stream);
    GemmArgs args = make_args(w, a, plan, rows, ldc, err, sk_ws);
    // one destination: p.out, offset by the column offset
    args.out = static_cast<char *>(out.dst[0]) + out.col0 * (out_type == kF16 ? 2 : 4);
    return launch_n<1>(wmap, amap, amap_sub, args, out, plan, w.bits, out_type, pdl, stream);
}

}  // namespace ql
