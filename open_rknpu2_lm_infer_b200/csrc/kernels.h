// kernels.h -- host-side launchers of the library's kernels (internal; not the C ABI).
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace ql {

enum ElemType { kF32 = 0, kF16 = 1, kI32 = 2, kI8Codes = 3 };

// Device weight layout (see pack.cu):
//   W8: int8 [Np][Kp], row n holds codes w[k][n] for k < K, zero padding.
//   W4: uint8 [Np][Kp/2]; each 4-byte word w of row n covers k = 8w .. 8w+7 and its
//       byte j holds u(8w+j) | u(8w+j+4) << 4 with u = code + 8 (padding: code 0).
struct WeightView {
    int bits, K, N, Kp, Np;
    const uint8_t *w;      // device
    const float *scales;   // device, [Np], zero padded
};

// Where a kernel writes its output: dst[0] (this GPU's buffer) and, for the split-N
// exchange, up to kMaxOutputs - 1 peers' buffers mapped into this process (CUDA IPC); the
// element (m, n) goes to column col0 + n of row m (row stride ldc) of every destination.
constexpr int kMaxOutputs = 8;
struct OutputSet {
    void *dst[kMaxOutputs];
    int count;
    long long col0;
};
inline OutputSet single_output(void *p) {
    OutputSet o{};
    o.dst[0] = p;
    o.count = 1;
    o.col0 = 0;
    return o;
}

// Activation workspace: codes int8 [rows_cap][Kp], scales f32 [rows_cap], rowsums i32.
struct ActView {
    const int8_t *codes;
    const float *scales;
    const int32_t *rowsums;
    int rows_cap;          // rows the codes buffer holds (>= rows of the call)
};

// amax_in (optional, [rows]): the rows' max |x| given by the caller instead of computed here.
cudaError_t launch_act_quant(const void *x, int x_type, long long ldx, int rows, int K, int Kp,
                             int round_mode, int8_t *codes, float *scales, int32_t *rowsums,
                             cudaStream_t stream, const float *amax_in = nullptr);

// Split-K helpers (split_k.cu).  Row max |x| of x [rows][K] (NaN ignored, like act_quant), and
// the dequant of int32 accumulators acc [rows][lda] (summed over the K slices):
// out[m][n] = (f32(acc[m][n]) * s_a[m]) * s_w[n] with s_a the act_quant scale of amax[m].
cudaError_t launch_row_amax(const void *x, int x_type, long long ldx, int rows, int K, float *amax,
                            cudaStream_t stream);
cudaError_t launch_dequant(const int32_t *acc, long long lda, const float *amax,
                           const float *wscale, int rows, int N, void *out, int out_type,
                           long long ldc, int num_sms, cudaStream_t stream);

// Weight packing from the QuantMatrix layout int8 [K][N] (device copy) into the device
// layout above; only columns [n_begin, n_begin + N) of a matrix with n_total columns.
cudaError_t launch_pack_from_kn(const int8_t *codes_kn, int K, int n_total, int n_begin,
                                const WeightView &w, uint8_t *dst, cudaStream_t stream);
// From the checkpoint storage (W4: int32 words [N][ceil(K/8)], W8: int8 [N][K]).
cudaError_t launch_pack_from_checkpoint(const void *storage, const WeightView &w, uint8_t *dst,
                                        cudaStream_t stream);

// int8 expansion [Np][Kp] of a packed W4 device layout (the prefill GEMM's operand).
cudaError_t launch_expand_w4(const WeightView &w4, uint8_t *dst, cudaStream_t stream);

// Decode GEMV (rows <= 8).  Input either activation codes from the quantisation kernel
// (type kI8Codes: x = codes [rows][Kp], ascale / rowsum set) or raw activations (kF16 /
// kF32: x = [rows][ldx], K % (16 / elem) == 0, ldx likewise, x 16-byte aligned), which the
// GEMV quantises itself.  out [rows][ldc] of out_type; swiglu: width N/2.
struct GemvInput {
    const void *x;
    int type;
    long long ldx;
    int round_mode;
    const float *ascale;
    const int32_t *rowsum;
    unsigned *err;  // device error word (bounded waits)
};
// rows <= 8 and the activation codes and the CTA's weight scales fit the GEMV's shared memory
bool gemv_fits(int rows, int Kp, int N, int bits, bool swiglu, int num_sms);
bool gemv_can_fuse(const void *x, int type, long long ldx, int K);
cudaError_t launch_gemv(const WeightView &w, const GemvInput &in, int rows, const OutputSet &out,
                        int out_type, long long ldc, bool swiglu, int num_sms, cudaStream_t stream);
// The same with out.count > 1 (launch_gemv forwards to it): the split-N exchange's GEMV.
cudaError_t launch_gemv_scatter(const WeightView &w, const GemvInput &in, int rows,
                                const OutputSet &out, int out_type, long long ldc, bool swiglu,
                                int num_sms, cudaStream_t stream);

// tcgen05 GEMM (any rows).  wmap / amap are the TMA descriptors of the weights and the
// activation codes (see encode_* below).  out [rows][ldc] of out_type.
struct GemmPlan {
    int tok;        // token tile (the MMA's N): multiple of 16, <= 256
    int stages;     // pipeline depth
    int smem_bytes; // dynamic shared memory
    int grid;       // persistent CTAs
    int tiles;
    int sk;         // 1: stream-K (every pair the same number of k-blocks, split tiles
                    //    summed in a workspace); 2: tail split (the last partial wave's
                    //    tiles cut along their tokens into `split` sub-tiles on idle
                    //    pairs); 0: whole tiles strided over the pairs
    int sk_tiles;   // stream-K / tail split: the last sk_tiles tiles
    int split;      // tail split: sub-tiles per split tile
};
// max_pairs: gemm_pair_capacity() of the device (CTA pairs resident at once); allow_sk: the
// plan may choose the stream-K schedule (QLINEAR_BACKEND_GEMM_STREAM_K).
GemmPlan plan_gemm(const WeightView &w, int rows, int max_pairs, bool allow_sk);
int gemm_pair_capacity(int bits);
// Bytes of the stream-K workspace a plan needs (0 without stream-K): partial-sum buffers
// (no initial value needed) and per-tile contribution counters, which must be zero before a
// launch.  The caller zero-fills it once; every launch leaves the counters zero again
// (unless a launch gave up on a timeout).
size_t gemm_sk_bytes(const GemmPlan &plan);
// pdl: launch with programmatic stream serialization (the kernel waits with
// griddepcontrol.wait before reading the activation codes / scales).  sk_ws: the zeroed
// stream-K workspace of gemm_sk_bytes(plan) bytes (ignored without stream-K).
cudaError_t launch_gemm(const WeightView &w, const CUtensorMap &wmap, const ActView &a,
                        const CUtensorMap &amap, const CUtensorMap &amap_sub,
                        const GemmPlan &plan, int rows,
                        const OutputSet &out,
                        int out_type, long long ldc, unsigned *err, void *sk_ws, bool pdl,
                        cudaStream_t stream);
// SwiGLU in the GEMM's epilogue (gemm_glu.cu): w is an 8-bit gate/up matrix (N even, gate
// columns first), wmap_glu its map from encode_glu_map (16-row boxes), plan from plan_gemm
// (sk_ws as for launch_gemm); out [rows][ldc] (ldc >= N/2) of kF16 or kF32 receives
// silu(y[m][j]) * y[m][N/2 + j].
cudaError_t launch_gemm_glu(const WeightView &w, const CUtensorMap &wmap_glu, const ActView &a,
                            const CUtensorMap &amap, const CUtensorMap &amap_sub,
                            const GemmPlan &plan, int rows, void *out, int out_type,
                            long long ldc, unsigned *err, void *sk_ws, bool pdl,
                            cudaStream_t stream);
// The same with out.count > 1 (launch_gemm forwards to it): the split-N exchange's GEMM.
cudaError_t launch_gemm_scatter(const WeightView &w, const CUtensorMap &wmap, const ActView &a,
                                const CUtensorMap &amap, const CUtensorMap &amap_sub,
                                const GemmPlan &plan, int rows,
                                const OutputSet &out, int out_type, long long ldc, unsigned *err,
                                void *sk_ws, bool pdl, cudaStream_t stream);

// The split-N exchange's GEMM through an NVSwitch multicast address (out.dst[0]; fp16 needs
// an even out.col0 and ldc).
cudaError_t launch_gemm_multicast(const WeightView &w, const CUtensorMap &wmap, const ActView &a,
                                  const CUtensorMap &amap, const CUtensorMap &amap_sub,
                                  const GemmPlan &plan, int rows, const OutputSet &out,
                                  int out_type, long long ldc, unsigned *err, void *sk_ws,
                                  bool pdl, cudaStream_t stream);

// Signal arrays of the split-N exchange's ranks (peer_sync.cu): sig[r] = rank r's, mapped here.
struct PeerSignals {
    void *sig[kMaxOutputs];
    int world, rank;
};
cudaError_t launch_peer_signal_wait(const PeerSignals &s, unsigned long long epoch, unsigned *err,
                                    unsigned long long limit_ns, cudaStream_t stream);

// Failure-path self-test: one warp waits limit_ns on an mbarrier nobody arrives on, then
// records QL_DEVERR_TIMEOUT in *err and returns.
cudaError_t launch_wait_selftest(unsigned *err, unsigned long long limit_ns, cudaStream_t stream);

// SwiGLU over an f32 [rows][N] buffer: out[m][j] = silu(y[m][j]) * y[m][N/2 + j].
cudaError_t launch_swiglu(const float *y, int rows, int N, void *out, int out_type,
                          long long ldc, cudaStream_t stream);

// dst[m][s*shard_cols + j] = src[s][m][j] (split-N output assembly).
cudaError_t launch_interleave(const void *src, void *dst, int shards, int rows, int shard_cols,
                              int elem_bytes, int num_sms, cudaStream_t stream);

// Weights view, device and backend settings of a weights object (qlinear_api.cu), for the
// allocation-free decode call (noalloc.cu).
}  // namespace ql
struct qlinear_weights;
namespace ql {
bool weights_for_noalloc(const qlinear_weights *w, WeightView *view, int *device, int *round_mode,
                         int *num_sms);

// TMA descriptor encoding through the driver entry point (no -lcuda link needed).
bool tma_available();
bool encode_weight_map(const WeightView &w, CUtensorMap *map);
// 8-bit weights [Np][Kp] in boxes of 128 k x 16 channels (the SwiGLU GEMM's gate/up boxes).
bool encode_glu_map(const WeightView &w, CUtensorMap *map);
bool encode_act_map(const int8_t *codes, int rows_cap, int Kp, int tok, CUtensorMap *map);

}  // namespace ql
