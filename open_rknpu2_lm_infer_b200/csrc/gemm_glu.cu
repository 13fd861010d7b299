// gemm_glu.cu -- prefill path for Linear::run_swiglu (src/npu.rs:1009-1024): the tcgen05
// GEMM of a gate/up matrix with the SiLU-gated product in its epilogue, so the [rows][N]
// projection output is never written.  The kernel is gemm_kernel<BITS, OutT, 1, true> in
// gemm_impl.cuh (BITS 8: an 8-bit copy of the weights; 4: the packed weights).
#include "gemm_impl.cuh"

namespace ql {

cudaError_t launch_gemm_glu(const WeightView &w, const CUtensorMap &wmap_glu, const ActView &a,
                            const CUtensorMap &amap, const CUtensorMap &amap_sub,
                            const GemmPlan &plan, int rows, void *out, int out_type,
                            long long ldc, unsigned *err, void *sk_ws, bool pdl,
                            cudaStream_t stream) {
    // 8-bit weights, an even N, a floating-point output; sk_ws: the stream-K workspace of
    // gemm_sk_bytes(plan) bytes when the plan chose stream-K
    if (w.N % 2 != 0 || !out || ldc < w.N / 2 || (plan.sk == 1 && !sk_ws))
        return cudaErrorInvalidValue;
    GemmArgs args = make_args(w, a, plan, rows, ldc, err, sk_ws);
    args.out = out;
    const OutputSet none{};
    if (w.bits == 8) {
        if (out_type == kF16)
            return launch_s<8, __half, 1, true>(wmap_glu, amap, amap_sub, args, none, plan, pdl, stream);
        if (out_type == kF32)
            return launch_s<8, float, 1, true>(wmap_glu, amap, amap_sub, args, none, plan, pdl, stream);
    } else {
        if (out_type == kF16)
            return launch_s<4, __half, 1, true>(wmap_glu, amap, amap_sub, args, none, plan, pdl, stream);
        if (out_type == kF32)
            return launch_s<4, float, 1, true>(wmap_glu, amap, amap_sub, args, none, plan, pdl, stream);
    }
    return cudaErrorInvalidValue;
}

}  // namespace ql
