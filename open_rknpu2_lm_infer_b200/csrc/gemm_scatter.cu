// gemm_scatter.cu -- the prefill GEMM of the split-N exchange: every output element is
// stored to this GPU's buffer and to the peers' (CUDA IPC mappings), then made visible
// system-wide at the end of the epilogue.  The kernel is in gemm_impl.cuh.
#include "gemm_impl.cuh"

namespace ql {

cudaError_t launch_gemm_scatter(const WeightView &w, const CUtensorMap &wmap, const ActView &a,
                                const CUtensorMap &amap, const CUtensorMap &amap_sub,
                                const GemmPlan &plan, int rows,
                                const OutputSet &out, int out_type, long long ldc, unsigned *err,
                                void *sk_ws, bool pdl, cudaStream_t stream) {
    if (out.count < 2 || out.count > kMaxOutputs) return cudaErrorInvalidValue;
    const GemmArgs args = make_args(w, a, plan, rows, ldc, err, sk_ws);
    // kernels for 2, 4 and 8 destinations; the padding slots repeat this GPU's buffer (the
    // same value stored twice)
    const int n = out.count <= 2 ? 2 : out.count <= 4 ? 4 : 8;
    OutputSet o = out;
    for (int d = out.count; d < n; d++) o.dst[d] = out.dst[0];
    o.count = n;
    if (n == 2) return launch_n<2>(wmap, amap, amap_sub, args, o, plan, w.bits, out_type, pdl, stream);
    if (n == 4) return launch_n<4>(wmap, amap, amap_sub, args, o, plan, w.bits, out_type, pdl, stream);
    return launch_n<8>(wmap, amap, amap_sub, args, o, plan, w.bits, out_type, pdl, stream);
}

// The same GEMM storing through one NVSwitch multicast address (out.dst[0], out.count 1):
// each element is stored once and the switch writes it into every rank's buffer.
cudaError_t launch_gemm_multicast(const WeightView &w, const CUtensorMap &wmap, const ActView &a,
                                  const CUtensorMap &amap, const CUtensorMap &amap_sub,
                                  const GemmPlan &plan, int rows, const OutputSet &out,
                                  int out_type, long long ldc, unsigned *err, void *sk_ws,
                                  bool pdl, cudaStream_t stream) {
    // multimem stores are 32-bit: fp16 pairs need an even column offset and row stride
    if (out.count != 1 || !out.dst[0] || (out_type == kF16 && ((out.col0 | ldc) & 1)))
        return cudaErrorInvalidValue;
    const GemmArgs args = make_args(w, a, plan, rows, ldc, err, sk_ws);
    return launch_n<0>(wmap, amap, amap_sub, args, out, plan, w.bits, out_type, pdl, stream);
}

}  // namespace ql
