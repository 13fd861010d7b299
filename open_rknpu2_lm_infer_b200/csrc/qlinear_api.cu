// qlinear_api.cu -- the C ABI of include/qlinear.h: backend and weight objects, workspace
// management, dispatch between the decode GEMV (rows <= 8) and the tcgen05 GEMM, and the
// synchronous host-f32 path that replaces the reference's rk_npu_*_run calls.
//
// Reference behaviour kept (src/npu.rs):
//   - Backend::load validates bits (4|8), K/N > 0 and the code/scale lengths (:368-384);
//   - Linear::run takes f32 rows [rows][K] and returns f32 [rows][N], synchronously
//     (:1006, :1025-1071); Linear::run_swiglu returns [rows][N/2] (:1009-1024);
//   - errors are int status codes with a message (:138-144), never an abort.
// Deliberately different: no 256-row cap and no M-bucket padding (the GPU kernels mask
// ragged tiles), no tuning (one static dispatch), run_swiglu supported for W4 and W8.
#include "../../include/qlinear.h"
#include "common.cuh"
#include "host_pool.h"
#include "kernels.h"

#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdio>
#include <cstring>
#include <map>
#include <memory>
#include <mutex>
#include <new>
#include <thread>
#include <string>
#include <tuple>
#include <vector>
#include <array>

using namespace ql;

struct qlinear_backend {
    // the caller's handle plus one per live weights object: weights keep their backend alive,
    // like the reference's Linear holding a Backend clone (src/npu.rs:252-260), so weights
    // freed after the backend handle still find it
    int refs = 1;
    int device = 0;
    int round_mode = QLINEAR_ROUND_AWAY;
    unsigned flags = 0;
    int num_sms = 148;
    int gemm_pairs[2] = {0, 0};  // resident CTA pairs of the W4 / W8 GEMM
    cudaStream_t stream = nullptr;  // host-path calls and uploads
    cudaStream_t stream_in = nullptr;  // host path, page-locked input: row pieces sent ahead
    unsigned *d_err = nullptr;
    unsigned *h_err = nullptr;      // pinned
    // activation workspace
    uint8_t *d_ws = nullptr;        // codes
    size_t ws_bytes = 0;
    float *d_ascale = nullptr;
    int32_t *d_rowsum = nullptr;
    size_t ws_rows = 0;
    // f32 gate/up scratch for SwiGLU through the GEMM
    float *d_y = nullptr;
    size_t y_elems = 0;
    // the MLP block's f32 intermediate [rows][N/2] (qlinear_run_mlp_device)
    float *d_mid = nullptr;
    size_t mid_bytes = 0;
    unsigned long long mlp_calls = 0;
    // stream-K partial sums and contribution counters of the GEMM (counters zero between
    // launches)
    void *d_sk = nullptr;
    size_t sk_bytes = 0;
    // host path staging
    void *d_in = nullptr, *d_out = nullptr;
    size_t d_in_bytes = 0, d_out_bytes = 0;
    void *h_in = nullptr, *h_out = nullptr;
    size_t h_in_bytes = 0, h_out_bytes = 0;
    std::unique_ptr<HostPool> pool;         // host copies of the f32 host path
    std::vector<cudaEvent_t> chunk_events;  // one per output chunk in flight
    // bookkeeping (Backend::stats)
    int loaded_w4 = 0, loaded_w8 = 0;
    uint64_t weight_bytes = 0;
    int max_kp = 0, max_n = 0;
    int prepared_rows = 0;
    unsigned long long launches = 0;
    unsigned long long gemv_calls = 0, gemm_calls = 0, gemm_stream_k_calls = 0,
                       gemm_glu_calls = 0;
    std::map<std::tuple<const void *, int, int, size_t>, CUtensorMap> amaps;
    // per-kernel device timing (qlinear_backend_profile)
    bool profiling = false;
    std::vector<std::array<cudaEvent_t, 3>> prof_events;
    size_t prof_used = 0;
};

struct qlinear_weights {
    qlinear_backend *backend = nullptr;
    WeightView view{};         // as loaded (W4 packed or W8)
    uint8_t *d_w = nullptr;
    float *d_s = nullptr;
    uint64_t bytes = 0;
    CUtensorMap wmap{};
    // W4 only: int8 expansion read by the prefill GEMM (absent with
    // QLINEAR_BACKEND_W4_PACKED_ONLY)
    WeightView view8{};
    uint8_t *d_w8 = nullptr;
    CUtensorMap wmap8{};
    // even N with an 8-bit prefill copy: that copy in 16-channel boxes for the GEMM with
    // the SwiGLU epilogue (gate and up rows of a channel staged side by side)
    bool has_glu = false;
    CUtensorMap wmap_glu{};
};

namespace {

thread_local int g_last_status = QLINEAR_OK;

// K * 127 * 127 must fit in int32 for the exact accumulator (W8; W4 is far looser).
constexpr long long kMaxK = 133143;

int fail(int status) {
    g_last_status = status;
    return status;
}

int cuda_status(cudaError_t e) {
    if (e == cudaSuccess) return QLINEAR_OK;
    if (e == cudaErrorMemoryAllocation) return QLINEAR_ERR_ALLOC;
    return QLINEAR_ERR_CUDA;
}

#define QL_TRY(expr)                              \
    do {                                          \
        cudaError_t _e = (expr);                  \
        if (_e != cudaSuccess) return cuda_status(_e); \
    } while (0)

struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        if (cudaGetDevice(&prev) != cudaSuccess) prev = -1;
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        if (prev >= 0 && cudaGetDevice(&cur) == cudaSuccess && cur != prev) cudaSetDevice(prev);
    }
};

// ---------------------------------------------------------------- TMA descriptors
PFN_cuTensorMapEncodeTiled_v12000 g_encode = nullptr;
std::once_flag g_encode_once;

void load_encode() {
    std::call_once(g_encode_once, [] {
        void *fn = nullptr;
        cudaDriverEntryPointQueryResult q{};
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &fn, cudaEnableDefault, &q) ==
                cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            g_encode = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(fn);
    });
}

bool encode_2d(CUtensorMap *map, const void *base, uint64_t inner, uint64_t outer,
               uint64_t row_bytes, uint32_t box_inner, uint32_t box_outer,
               CUtensorMapSwizzle swz) {
    load_encode();
    if (!g_encode) return false;
    cuuint64_t dims[2] = {inner, outer};
    cuuint64_t strides[1] = {row_bytes};
    cuuint32_t box[2] = {box_inner, box_outer};
    cuuint32_t estr[2] = {1, 1};
    CUresult r = g_encode(map, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void *>(base), dims,
                          strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, swz,
                          CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    return r == CUDA_SUCCESS;
}

}  // namespace

namespace ql {
bool tma_available() {
    load_encode();
    return g_encode != nullptr;
}
// The GEMM runs on CTA pairs: each CTA streams 128-deep k-blocks of its 128 weight channels
// (128-byte swizzle for 8-bit operands; packed W4 rows of 64 bytes, unpacked in the kernel)
// and of half of the token tile.
bool encode_weight_map(const WeightView &w, CUtensorMap *map) {
    if (w.bits == 8)
        return encode_2d(map, w.w, w.Kp, w.Np, w.Kp, GEMM_KB, CH_TILE, CU_TENSOR_MAP_SWIZZLE_128B);
    // packed W4 rows of 64 bytes per k-block; the 64-byte swizzle lets the converter's
    // 128 threads (one row each) read the tile without bank conflicts
    return encode_2d(map, w.w, w.Kp / 2, w.Np, w.Kp / 2, GEMM_KB / 2, CH_TILE,
                     CU_TENSOR_MAP_SWIZZLE_64B);
}
bool encode_glu_map(const WeightView &w, CUtensorMap *map) {
    if (w.bits == 8)
        return encode_2d(map, w.w, w.Kp, w.Np, w.Kp, GEMM_KB, 16, CU_TENSOR_MAP_SWIZZLE_128B);
    return encode_2d(map, w.w, w.Kp / 2, w.Np, w.Kp / 2, GEMM_KB / 2, 16,
                     CU_TENSOR_MAP_SWIZZLE_64B);
}
bool encode_act_map(const int8_t *codes, int rows_cap, int Kp, int tok, CUtensorMap *map) {
    return encode_2d(map, codes, Kp, rows_cap, Kp, GEMM_KB, tok / 2, CU_TENSOR_MAP_SWIZZLE_128B);
}
}  // namespace ql

namespace {

// ---------------------------------------------------------------- workspaces
int ensure_act_ws(qlinear_backend *b, int rows, int Kp) {
    const size_t need = (size_t)rows * Kp;
    if (need <= b->ws_bytes && (size_t)rows <= b->ws_rows) return QLINEAR_OK;
    size_t bytes = std::max(need, b->ws_bytes);
    size_t nrows = std::max((size_t)rows, b->ws_rows);
    nrows = (nrows + 255) / 256 * 256;
    bytes = std::max(bytes, nrows * (size_t)std::max(Kp, b->max_kp));
    bytes = (bytes + 4095) / 4096 * 4096;
    cudaFree(b->d_ws);
    cudaFree(b->d_ascale);
    cudaFree(b->d_rowsum);
    b->d_ws = nullptr;
    b->d_ascale = nullptr;
    b->d_rowsum = nullptr;
    b->ws_bytes = 0;
    b->ws_rows = 0;
    b->amaps.clear();
    QL_TRY(cudaMalloc(&b->d_ws, bytes));
    QL_TRY(cudaMalloc(&b->d_ascale, nrows * sizeof(float)));
    QL_TRY(cudaMalloc(&b->d_rowsum, nrows * sizeof(int32_t)));
    b->ws_bytes = bytes;
    b->ws_rows = nrows;
    return QLINEAR_OK;
}

int ensure_dev(void **p, size_t *cap, size_t need) {
    if (need <= *cap) return QLINEAR_OK;
    cudaFree(*p);
    *p = nullptr;
    *cap = 0;
    need = (need + 4095) / 4096 * 4096;
    QL_TRY(cudaMalloc(p, need));
    *cap = need;
    return QLINEAR_OK;
}

// The stream-K workspace: grown on demand, zero-filled when (re)allocated; the GEMM leaves
// its counters zero after every launch that completes.
int ensure_sk(qlinear_backend *b, size_t need) {
    if (need <= b->sk_bytes) return QLINEAR_OK;
    cudaFree(b->d_sk);
    b->d_sk = nullptr;
    b->sk_bytes = 0;
    need = (need + 4095) / 4096 * 4096;
    QL_TRY(cudaMalloc(&b->d_sk, need));
    QL_TRY(cudaMemset(b->d_sk, 0, need));
    b->sk_bytes = need;
    return QLINEAR_OK;
}

// After a device-side timeout a GEMM may have left contribution counters behind.
void reset_after_timeout(qlinear_backend *b) {
    if (b->d_sk) cudaMemset(b->d_sk, 0, b->sk_bytes);
}

int ensure_host(void **p, size_t *cap, size_t need) {
    if (need <= *cap) return QLINEAR_OK;
    cudaFreeHost(*p);
    *p = nullptr;
    *cap = 0;
    need = (need + 4095) / 4096 * 4096;
    QL_TRY(cudaMallocHost(p, need));
    *cap = need;
    return QLINEAR_OK;
}

int get_amap(qlinear_backend *b, int Kp, int tok, const CUtensorMap **out) {
    const int rows_cap = (int)std::min<size_t>(b->ws_bytes / Kp, 1u << 30);
    auto key = std::make_tuple((const void *)b->d_ws, Kp, tok, (size_t)rows_cap);
    auto it = b->amaps.find(key);
    if (it == b->amaps.end()) {
        CUtensorMap m;
        if (!encode_act_map(reinterpret_cast<const int8_t *>(b->d_ws), rows_cap, Kp, tok, &m))
            return QLINEAR_ERR_CUDA;
        it = b->amaps.emplace(key, m).first;
    }
    *out = &it->second;
    return QLINEAR_OK;
}

bool valid_io_type(int t) { return t == QLINEAR_F32 || t == QLINEAR_F16; }

int next_prof_events(qlinear_backend *b, const std::array<cudaEvent_t, 3> **out) {
    if (b->prof_used == b->prof_events.size()) {
        if (b->prof_events.size() >= 65536) return QLINEAR_ERR_STATE;  // collect first
        std::array<cudaEvent_t, 3> e{};
        for (auto &x : e) QL_TRY(cudaEventCreate(&x));
        b->prof_events.push_back(e);
    }
    *out = &b->prof_events[b->prof_used++];
    return QLINEAR_OK;
}

// outs: where the output goes (this GPU's buffer, plus peers' for the split-N exchange);
// c_dev = outs.dst[0].
// amax_in (optional, device [rows]): quantise with these row maxima (a K-split row's max over
// every rank's slice) instead of each row's own.
// mc (optional): the NVSwitch multicast address of the exchange buffers; the tensor-core GEMM
// then stores through it once instead of to each of outs' destinations (the decode GEMV
// still stores to outs).
int run_device_impl(qlinear_backend *b, const qlinear_weights *w, const void *a_dev, int a_type,
                    const OutputSet &outs, int c_type, long long ldc, int rows, unsigned flags,
                    cudaStream_t stream, const float *amax_in = nullptr, void *mc = nullptr) {
    const WeightView &v = w->view;
    const bool swiglu = (flags & QLINEAR_RUN_SWIGLU) != 0;
    const int width = swiglu ? v.N / 2 : v.N;
    void *c_dev = outs.dst[0];
    if (rows < 1 || !a_dev || !valid_io_type(a_type) || outs.count < 1 || outs.count > kMaxOutputs)
        return QLINEAR_ERR_PARAM;
    for (int d = 0; d < outs.count; d++)
        if (!outs.dst[d]) return QLINEAR_ERR_PARAM;
    if (c_type != QLINEAR_F32 && c_type != QLINEAR_F16 && c_type != QLINEAR_I32)
        return QLINEAR_ERR_PARAM;
    if (swiglu && (v.N % 2 != 0 || c_type == QLINEAR_I32)) return QLINEAR_ERR_PARAM;
    if (ldc < width) return QLINEAR_ERR_PARAM;
    if ((flags & ~QLINEAR_RUN_SWIGLU) != 0) return QLINEAR_ERR_PARAM;

    int st;
    const std::array<cudaEvent_t, 3> *ev = nullptr;
    if (!amax_in && gemv_fits(rows, v.Kp, v.N, v.bits, swiglu, b->num_sms) &&
        gemv_can_fuse(a_dev, a_type, v.K, v.K)) {
        // decode: one kernel that quantises the rows itself and streams the weights
        if (b->profiling) {
            if ((st = next_prof_events(b, &ev))) return st;
            QL_TRY(cudaEventRecord((*ev)[0], stream));
            QL_TRY(cudaEventRecord((*ev)[1], stream));
        }
        GemvInput in{a_dev, a_type, v.K, b->round_mode, nullptr, nullptr, b->d_err};
        const cudaError_t e = launch_gemv(v, in, rows, outs, c_type, ldc, swiglu, b->num_sms, stream);
        if (ev) cudaEventRecord((*ev)[2], stream);
        QL_TRY(e);
        b->launches++;
        b->gemv_calls++;
        return QLINEAR_OK;
    }
    if ((st = ensure_act_ws(b, rows, v.Kp))) return st;
    if (b->profiling) {
        if ((st = next_prof_events(b, &ev))) return st;
        QL_TRY(cudaEventRecord((*ev)[0], stream));
    }
    int8_t *codes = reinterpret_cast<int8_t *>(b->d_ws);
    QL_TRY(launch_act_quant(a_dev, a_type, v.K, rows, v.K, v.Kp, b->round_mode, codes, b->d_ascale,
                            b->d_rowsum, stream, amax_in));
    b->launches++;
    if (ev) QL_TRY(cudaEventRecord((*ev)[1], stream));
    struct Stop {  // records the third event on every exit path below
        const std::array<cudaEvent_t, 3> *ev;
        cudaStream_t s;
        ~Stop() {
            if (ev) cudaEventRecord((*ev)[2], s);
        }
    } stop{ev, stream};
    ActView av{codes, b->d_ascale, b->d_rowsum, (int)(b->ws_bytes / v.Kp)};

    if (gemv_fits(rows, v.Kp, v.N, v.bits, swiglu, b->num_sms)) {
        GemvInput in{codes, kI8Codes, v.Kp, b->round_mode, b->d_ascale, b->d_rowsum, b->d_err};
        QL_TRY(launch_gemv(v, in, rows, outs, c_type, ldc, swiglu, b->num_sms, stream));
        b->launches++;
        b->gemv_calls++;
        return QLINEAR_OK;
    }
    const int gbits = (v.bits == 8 || w->d_w8) ? 8 : 4;
    int &pairs = b->gemm_pairs[gbits == 8 ? 1 : 0];
    if (!pairs) {
        pairs = gemm_pair_capacity(gbits);
        if (!pairs) return QLINEAR_ERR_CUDA;
    }
    // W4 prefill reads the int8 expansion when the weights carry one
    const bool use8 = w->d_w8 != nullptr;
    const WeightView &gv = use8 ? w->view8 : v;
    const CUtensorMap &gmap = use8 ? w->wmap8 : w->wmap;
    // SwiGLU in the GEMM's epilogue: one output buffer, 8-bit prefill weights
    const bool glu = swiglu && w->has_glu && outs.count == 1 &&
                     !(b->flags & QLINEAR_BACKEND_SWIGLU_UNFUSED);
    const GemmPlan plan = plan_gemm(gv, rows, pairs, (b->flags & QLINEAR_BACKEND_GEMM_STREAM_K) != 0);
    if ((st = ensure_sk(b, gemm_sk_bytes(plan)))) return st;
    if (plan.sk == 1) b->gemm_stream_k_calls++;
    const CUtensorMap *amap = nullptr;
    st = get_amap(b, v.Kp, plan.tok, &amap);
    if (st) return st;
    // the tail split's sub-tiles load a box of their own rows
    const CUtensorMap *amap_sub = amap;
    if (plan.sk == 2) {
        st = get_amap(b, v.Kp, plan.tok / plan.split, &amap_sub);
        if (st) return st;
    }
    if (!swiglu && mc) {
        OutputSet mo{};
        mo.dst[0] = mc;
        mo.count = 1;
        mo.col0 = outs.col0;
        QL_TRY(launch_gemm_multicast(gv, gmap, av, *amap, *amap_sub, plan, rows, mo, c_type, ldc,
                                     b->d_err, b->d_sk, true, stream));
        b->launches++;
    } else if (!swiglu) {
        QL_TRY(launch_gemm(gv, gmap, av, *amap, *amap_sub, plan, rows, outs, c_type, ldc,
                           b->d_err, b->d_sk, true, stream));
        b->launches++;
    } else if (glu) {
        QL_TRY(launch_gemm_glu(gv, w->wmap_glu, av, *amap, *amap_sub, plan, rows, c_dev, c_type,
                               ldc, b->d_err, b->d_sk, true, stream));
        b->launches++;
        b->gemm_glu_calls++;
    } else {
        st = ensure_dev(reinterpret_cast<void **>(&b->d_y), &b->y_elems,
                        (size_t)rows * v.N * sizeof(float));
        if (st) return st;
        if (outs.count != 1) return QLINEAR_ERR_UNSUPPORTED;  // the SwiGLU pass writes one buffer
        QL_TRY(launch_gemm(gv, gmap, av, *amap, *amap_sub, plan, rows, single_output(b->d_y), kF32,
                           v.N, b->d_err, b->d_sk, true, stream));
        QL_TRY(launch_swiglu(b->d_y, rows, v.N, c_dev, c_type, ldc, stream));
        b->launches += 2;
    }
    b->gemm_calls++;
    return QLINEAR_OK;
}

qlinear_weights *weights_create_common(qlinear_backend *b, const qlinear_weight_config *cfg,
                                       const void *src, size_t src_bytes, const float *scales,
                                       int n_total, int n_begin, int n_end, bool checkpoint) {
    if (!b || !cfg || !src || !scales) return fail(QLINEAR_ERR_PARAM), nullptr;
    if ((cfg->bits != 4 && cfg->bits != 8) || cfg->K <= 0 || cfg->N <= 0 || cfg->K > kMaxK)
        return fail(QLINEAR_ERR_PARAM), nullptr;
    if (n_begin < 0 || n_end > n_total || n_begin >= n_end) return fail(QLINEAR_ERR_PARAM), nullptr;
    const int N = n_end - n_begin;
    for (int n = n_begin; n < n_end; n++)
        if (!(scales[n] > 0.0f) || !(scales[n] < INFINITY))  // src/model/checkpoint.rs:334-337
            return fail(QLINEAR_ERR_PARAM), nullptr;
    DeviceGuard guard(b->device);
    auto *w = new (std::nothrow) qlinear_weights();
    if (!w) return fail(QLINEAR_ERR_ALLOC), nullptr;
    w->backend = b;
    WeightView &v = w->view;
    v.bits = cfg->bits;
    v.K = cfg->K;
    v.N = N;
    v.Kp = (int)round_up(cfg->K, KBLK);
    v.Np = (int)round_up(N, CH_TILE);
    const size_t wbytes = (size_t)v.Np * (v.bits == 8 ? v.Kp : v.Kp / 2);
    void *tmp = nullptr;
    auto cleanup = [&](int status) -> qlinear_weights * {
        cudaFree(tmp);
        cudaFree(w->d_w8);
        cudaFree(w->d_w);
        cudaFree(w->d_s);
        delete w;
        fail(status);
        return nullptr;
    };
    cudaError_t e;
    if ((e = cudaMalloc(&w->d_w, wbytes)) != cudaSuccess) return cleanup(cuda_status(e));
    if ((e = cudaMalloc(&w->d_s, (size_t)v.Np * sizeof(float))) != cudaSuccess)
        return cleanup(cuda_status(e));
    if ((e = cudaMemsetAsync(w->d_s, 0, (size_t)v.Np * sizeof(float), b->stream)) != cudaSuccess)
        return cleanup(cuda_status(e));
    if ((e = cudaMemcpyAsync(w->d_s, scales + n_begin, (size_t)N * sizeof(float),
                             cudaMemcpyHostToDevice, b->stream)) != cudaSuccess)
        return cleanup(cuda_status(e));
    if ((e = cudaMalloc(&tmp, src_bytes)) != cudaSuccess) return cleanup(cuda_status(e));
    if ((e = cudaMemcpyAsync(tmp, src, src_bytes, cudaMemcpyHostToDevice, b->stream)) != cudaSuccess)
        return cleanup(cuda_status(e));
    v.w = w->d_w;
    v.scales = w->d_s;
    if (checkpoint)
        e = launch_pack_from_checkpoint(tmp, v, w->d_w, b->stream);
    else
        e = launch_pack_from_kn(static_cast<const int8_t *>(tmp), cfg->K, n_total, n_begin, v,
                                w->d_w, b->stream);
    if (e != cudaSuccess) return cleanup(cuda_status(e));
    b->launches++;
    if ((e = cudaStreamSynchronize(b->stream)) != cudaSuccess) return cleanup(cuda_status(e));
    cudaFree(tmp);
    tmp = nullptr;
    if (!encode_weight_map(v, &w->wmap)) return cleanup(QLINEAR_ERR_CUDA);
    w->bytes = wbytes + (uint64_t)v.Np * sizeof(float);
    if (v.bits == 4 && !(b->flags & QLINEAR_BACKEND_W4_PACKED_ONLY)) {
        const size_t bytes8 = (size_t)v.Np * v.Kp;
        if ((e = cudaMalloc(&w->d_w8, bytes8)) != cudaSuccess) return cleanup(cuda_status(e));
        w->view8 = v;
        w->view8.bits = 8;
        w->view8.w = w->d_w8;
        if ((e = launch_expand_w4(v, w->d_w8, b->stream)) != cudaSuccess ||
            (e = cudaStreamSynchronize(b->stream)) != cudaSuccess)
            return cleanup(cuda_status(e));
        b->launches++;
        if (!encode_weight_map(w->view8, &w->wmap8)) return cleanup(QLINEAR_ERR_CUDA);
        w->bytes += bytes8;
    }
    if (N % 2 == 0) {
        // the prefill weights' map in 16-row boxes: the 8-bit copy when there is one, else
        // the packed W4 rows
        if (!encode_glu_map(w->d_w8 ? w->view8 : v, &w->wmap_glu))
            return cleanup(QLINEAR_ERR_CUDA);
        w->has_glu = true;
    }
    b->weight_bytes += w->bytes;
    (v.bits == 4 ? b->loaded_w4 : b->loaded_w8)++;
    b->refs++;
    b->max_kp = std::max(b->max_kp, v.Kp);
    b->max_n = std::max(b->max_n, v.N);
    return w;
}

}  // namespace

// What the allocation-free decode call (noalloc.cu) needs from a weights object.
namespace ql {
bool weights_for_noalloc(const qlinear_weights *w, WeightView *view, int *device, int *round_mode,
                         int *num_sms) {
    if (!w || !w->backend) return false;
    *view = w->view;
    *device = w->backend->device;
    *round_mode = w->backend->round_mode;
    *num_sms = w->backend->num_sms;
    return true;
}
}  // namespace ql

// ====================================================================== C ABI
extern "C" {

void qlinear_backend_config_init(qlinear_backend_config *cfg) {
    if (!cfg) return;
    std::memset(cfg, 0, sizeof(*cfg));
    cfg->device = 0;
    cfg->round_mode = QLINEAR_ROUND_AWAY;
    cfg->max_rows = 256;
}

qlinear_backend *qlinear_backend_create(const qlinear_backend_config *cfg) {
    qlinear_backend_config def;
    qlinear_backend_config_init(&def);
    if (!cfg) cfg = &def;
    if (cfg->round_mode != QLINEAR_ROUND_AWAY && cfg->round_mode != QLINEAR_ROUND_EVEN)
        return fail(QLINEAR_ERR_PARAM), nullptr;
    if (cfg->max_rows < 0 ||
        (cfg->flags & ~(QLINEAR_BACKEND_W4_PACKED_ONLY | QLINEAR_BACKEND_GEMM_STREAM_K |
                        QLINEAR_BACKEND_SWIGLU_UNFUSED)))
        return fail(QLINEAR_ERR_PARAM), nullptr;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || cfg->device < 0 || cfg->device >= ndev)
        return fail(ndev == 0 ? QLINEAR_ERR_CUDA : QLINEAR_ERR_PARAM), nullptr;
    cudaDeviceProp prop;
    if (cudaGetDeviceProperties(&prop, cfg->device) != cudaSuccess)
        return fail(QLINEAR_ERR_CUDA), nullptr;
    if (prop.major != 10 || prop.minor != 0) return fail(QLINEAR_ERR_UNSUPPORTED), nullptr;
    if (!tma_available()) return fail(QLINEAR_ERR_UNSUPPORTED), nullptr;
    DeviceGuard guard(cfg->device);
    auto *b = new (std::nothrow) qlinear_backend();
    if (!b) return fail(QLINEAR_ERR_ALLOC), nullptr;
    b->device = cfg->device;
    b->round_mode = cfg->round_mode;
    b->flags = cfg->flags;
    b->num_sms = prop.multiProcessorCount;
    b->prepared_rows = cfg->max_rows ? cfg->max_rows : 256;
    if (cudaStreamCreateWithFlags(&b->stream, cudaStreamNonBlocking) != cudaSuccess ||
        cudaMalloc(&b->d_err, sizeof(unsigned)) != cudaSuccess ||
        cudaMallocHost(&b->h_err, sizeof(unsigned)) != cudaSuccess ||
        cudaMemset(b->d_err, 0, sizeof(unsigned)) != cudaSuccess) {
        qlinear_backend_free(b);
        return fail(QLINEAR_ERR_CUDA), nullptr;
    }
    return b;
}

namespace {
void destroy_backend(qlinear_backend *b) {
    DeviceGuard guard(b->device);
    if (b->stream) cudaStreamSynchronize(b->stream);
    cudaFree(b->d_ws);
    cudaFree(b->d_ascale);
    cudaFree(b->d_rowsum);
    cudaFree(b->d_y);
    cudaFree(b->d_mid);
    cudaFree(b->d_sk);
    cudaFree(b->d_in);
    cudaFree(b->d_out);
    cudaFree(b->d_err);
    cudaFreeHost(b->h_in);
    cudaFreeHost(b->h_out);
    cudaFreeHost(b->h_err);
    for (auto e : b->chunk_events) cudaEventDestroy(e);
    b->pool.reset();
    for (auto &e : b->prof_events)
        for (auto x : e) cudaEventDestroy(x);
    if (b->stream_in) cudaStreamDestroy(b->stream_in);
    if (b->stream) cudaStreamDestroy(b->stream);
    delete b;
}
}  // namespace

void qlinear_backend_free(qlinear_backend *b) {
    if (b && --b->refs == 0) destroy_backend(b);
}

qlinear_weights *qlinear_weights_create(qlinear_backend *b, const qlinear_weight_config *cfg,
                                        const int8_t *codes_kn, const float *scales) {
    if (!cfg) return fail(QLINEAR_ERR_PARAM), nullptr;
    return weights_create_common(b, cfg, codes_kn, (size_t)cfg->K * cfg->N, scales, cfg->N, 0,
                                 cfg->N, false);
}

qlinear_weights *qlinear_weights_create_shard(qlinear_backend *b, const qlinear_weight_config *cfg,
                                              const int8_t *codes_kn, const float *scales,
                                              int n_begin, int n_end) {
    if (!cfg) return fail(QLINEAR_ERR_PARAM), nullptr;
    return weights_create_common(b, cfg, codes_kn, (size_t)cfg->K * cfg->N, scales, cfg->N, n_begin,
                                 n_end, false);
}

qlinear_weights *qlinear_weights_create_checkpoint(qlinear_backend *b,
                                                   const qlinear_weight_config *cfg,
                                                   const void *storage, const float *scales) {
    if (!cfg || cfg->K <= 0 || cfg->N <= 0) return fail(QLINEAR_ERR_PARAM), nullptr;
    const size_t bytes = cfg->bits == 4 ? (size_t)cfg->N * ((cfg->K + 7) / 8) * 4
                                        : (size_t)cfg->N * cfg->K;
    return weights_create_common(b, cfg, storage, bytes, scales, cfg->N, 0, cfg->N, true);
}

int qlinear_weights_query(const qlinear_weights *w, qlinear_weight_info *info) {
    if (!w || !info) return QLINEAR_ERR_PARAM;
    info->bits = w->view.bits;
    info->K = w->view.K;
    info->N = w->view.N;
    info->K_padded = w->view.Kp;
    info->N_padded = w->view.Np;
    info->device_bytes = w->bytes;
    return QLINEAR_OK;
}

void qlinear_weights_free(qlinear_weights *w) {
    if (!w) return;
    qlinear_backend *b = w->backend;
    DeviceGuard guard(b->device);
    cudaStreamSynchronize(b->stream);
    cudaFree(w->d_w);
    cudaFree(w->d_w8);
    cudaFree(w->d_s);
    b->weight_bytes -= w->bytes;
    (w->view.bits == 4 ? b->loaded_w4 : b->loaded_w8)--;
    delete w;
    if (--b->refs == 0) destroy_backend(b);  // the backend handle was freed before
}

int qlinear_backend_prepare(qlinear_backend *b, int rows) {
    if (!b || rows < 1) return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    b->prepared_rows = std::max(b->prepared_rows, rows);
    if (b->max_kp == 0) return QLINEAR_OK;
    int st = ensure_act_ws(b, rows, b->max_kp);
    if (st) return st;
    if (rows > 8)
        st = ensure_dev(reinterpret_cast<void **>(&b->d_y), &b->y_elems,
                        (size_t)rows * b->max_n * sizeof(float));
    return st;
}

int qlinear_run_device(qlinear_backend *b, const qlinear_weights *w, const void *a_dev, int a_type,
                       void *c_dev, int c_type, long long ldc, int rows, unsigned flags,
                       void *stream) {
    if (!b || !w || w->backend != b) return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    return run_device_impl(b, w, a_dev, a_type, single_output(c_dev), c_type, ldc, rows, flags,
                           static_cast<cudaStream_t>(stream));
}

int qlinear_run_mlp_device(qlinear_backend *b, const qlinear_weights *gate_up,
                           const qlinear_weights *down, const void *a_dev, int a_type, void *c_dev,
                           int c_type, long long ldc, int rows, void *stream) {
    if (!b || !gate_up || !down || gate_up->backend != b || down->backend != b)
        return QLINEAR_ERR_PARAM;
    const WeightView &gu = gate_up->view, &dn = down->view;
    if (gu.N % 2 != 0 || dn.K != gu.N / 2 || rows < 1 || !a_dev || !c_dev ||
        !valid_io_type(a_type) || !valid_io_type(c_type) || ldc < dn.N)
        return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const int h = gu.N / 2;
    int st = ensure_dev(reinterpret_cast<void **>(&b->d_mid), &b->mid_bytes,
                        (size_t)rows * h * sizeof(float));
    if (st) return st;
    b->mlp_calls++;
    // gate/up with the SiLU-gated product into the f32 intermediate, then down (each call
    // launched with programmatic stream serialization, so the down call's weight stream
    // starts while the gate/up call drains)
    st = run_device_impl(b, gate_up, a_dev, a_type, single_output(b->d_mid), QLINEAR_F32, h, rows,
                         QLINEAR_RUN_SWIGLU, s);
    if (st) return st;
    return run_device_impl(b, down, b->d_mid, QLINEAR_F32, single_output(c_dev), c_type, ldc, rows,
                           0, s);
}

int qlinear_run_device_multicast(qlinear_backend *b, const qlinear_weights *w, const void *a_dev,
                                 int a_type, void *const *c_devs, int ndev, void *mc_dev,
                                 int c_type, long long ldc, long long col_offset, int rows,
                                 void *stream) {
    if (!b || !w || w->backend != b || !c_devs || !mc_dev || ndev < 1 || ndev > kMaxOutputs ||
        col_offset < 0 || ldc < col_offset + w->view.N)
        return QLINEAR_ERR_PARAM;
    if (c_type == QLINEAR_F16 && ((col_offset | ldc | w->view.N) & 1)) return QLINEAR_ERR_PARAM;
    OutputSet o{};
    for (int d = 0; d < ndev; d++) o.dst[d] = c_devs[d];
    o.count = ndev;
    o.col0 = col_offset;
    DeviceGuard guard(b->device);
    return run_device_impl(b, w, a_dev, a_type, o, c_type, ldc, rows, 0,
                           static_cast<cudaStream_t>(stream), nullptr, mc_dev);
}

int qlinear_run_device_scatter(qlinear_backend *b, const qlinear_weights *w, const void *a_dev,
                               int a_type, void *const *c_devs, int ndev, int c_type,
                               long long ldc, long long col_offset, int rows, unsigned flags,
                               void *stream) {
    if (!b || !w || w->backend != b || !c_devs || ndev < 1 || ndev > kMaxOutputs || col_offset < 0)
        return QLINEAR_ERR_PARAM;
    const int width = (flags & QLINEAR_RUN_SWIGLU) ? w->view.N / 2 : w->view.N;
    if (ldc < col_offset + width) return QLINEAR_ERR_PARAM;
    OutputSet o{};
    for (int d = 0; d < ndev; d++) o.dst[d] = c_devs[d];
    o.count = ndev;
    o.col0 = col_offset;
    DeviceGuard guard(b->device);
    return run_device_impl(b, w, a_dev, a_type, o, c_type, ldc, rows, flags,
                           static_cast<cudaStream_t>(stream));
}

int qlinear_peer_buffer_create(qlinear_backend *b, size_t bytes, void **dev_ptr,
                               unsigned char *ipc_handle) {
    if (!b || !dev_ptr || !ipc_handle || bytes == 0) return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    void *p = nullptr;
    QL_TRY(cudaMalloc(&p, bytes));
    cudaIpcMemHandle_t h;
    const cudaError_t e = cudaIpcGetMemHandle(&h, p);
    if (e != cudaSuccess) {
        cudaFree(p);
        return cuda_status(e);
    }
    static_assert(sizeof(h) == QLINEAR_IPC_HANDLE_BYTES, "CUDA IPC handle size");
    const cudaError_t z = cudaMemset(p, 0, bytes);  // signal arrays start at epoch 0
    if (z != cudaSuccess) {
        cudaFree(p);
        return cuda_status(z);
    }
    std::memcpy(ipc_handle, &h, sizeof(h));
    *dev_ptr = p;
    return QLINEAR_OK;
}

int qlinear_peer_buffer_open(qlinear_backend *b, const unsigned char *ipc_handle, void **dev_ptr) {
    if (!b || !dev_ptr || !ipc_handle) return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    cudaIpcMemHandle_t h;
    std::memcpy(&h, ipc_handle, sizeof(h));
    void *p = nullptr;
    QL_TRY(cudaIpcOpenMemHandle(&p, h, cudaIpcMemLazyEnablePeerAccess));
    *dev_ptr = p;
    return QLINEAR_OK;
}

int qlinear_peer_buffer_free(qlinear_backend *b, void *dev_ptr, int opened) {
    if (!b || !dev_ptr) return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    QL_TRY(opened ? cudaIpcCloseMemHandle(dev_ptr) : cudaFree(dev_ptr));
    return QLINEAR_OK;
}

// Whether [p, p + bytes) is page-locked host memory the GPU can copy from or to directly
// (cudaHostAlloc'd or cudaHostRegister'ed): both ends are checked.
static bool host_pinned(const void *p, size_t bytes) {
    for (const char *q : {static_cast<const char *>(p), static_cast<const char *>(p) + bytes - 1}) {
        cudaPointerAttributes at{};
        if (cudaPointerGetAttributes(&at, q) != cudaSuccess) {
            cudaGetLastError();  // not a CUDA pointer: clear the error, use the staging path
            return false;
        }
        if (at.type != cudaMemoryTypeHost) return false;
    }
    return true;
}

static int run_host(qlinear_backend *b, const qlinear_weights *w, const float *a_host,
                    float *c_host, long long ldc, int rows, unsigned flags) {
    if (!b || !w || w->backend != b || !a_host || !c_host || rows < 1) return QLINEAR_ERR_PARAM;
    if ((flags & ~QLINEAR_RUN_SWIGLU) != 0) return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    const WeightView &v = w->view;
    const bool swiglu = (flags & QLINEAR_RUN_SWIGLU) != 0;
    if (swiglu && v.N % 2) return QLINEAR_ERR_PARAM;
    const int width = swiglu ? v.N / 2 : v.N;
    if (ldc < width) return QLINEAR_ERR_PARAM;
    const size_t in_bytes = (size_t)rows * v.K * sizeof(float);
    const size_t out_bytes = (size_t)rows * width * sizeof(float);
    int st;
    // Caller buffers in page-locked memory: copied by DMA directly, no staging and no host
    // copies.  Large calls go in pieces of 128 rows: the input pieces are sent on a second
    // stream, and each piece is computed and its output rows (stride ldc, one 2-D transfer)
    // sent back as soon as its input has landed, so the output of one piece travels back
    // while the next piece's input travels in (the link is full duplex).
    if (host_pinned(a_host, in_bytes) &&
        host_pinned(c_host, ((size_t)(rows - 1) * ldc + width) * sizeof(float))) {
        if ((st = ensure_dev(&b->d_in, &b->d_in_bytes, in_bytes)) ||
            (st = ensure_dev(&b->d_out, &b->d_out_bytes, out_bytes)))
            return st;
        if (!b->stream_in)
            QL_TRY(cudaStreamCreateWithFlags(&b->stream_in, cudaStreamNonBlocking));
        const int piece = rows >= 256 ? 128 : rows;
        const int npieces = (rows + piece - 1) / piece;
        while ((int)b->chunk_events.size() < npieces) {
            cudaEvent_t e;
            QL_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
            b->chunk_events.push_back(e);
        }
        const char *a_bytes = reinterpret_cast<const char *>(a_host);
        char *d_in = static_cast<char *>(b->d_in);
        const size_t in_row = (size_t)v.K * sizeof(float), out_row = (size_t)width * sizeof(float);
        for (int i = 0; i < npieces; i++) {
            const int r0 = i * piece, n = std::min(piece, rows - r0);
            QL_TRY(cudaMemcpyAsync(d_in + r0 * in_row, a_bytes + r0 * in_row, n * in_row,
                                   cudaMemcpyHostToDevice, b->stream_in));
            QL_TRY(cudaEventRecord(b->chunk_events[i], b->stream_in));
        }
        char *d_out = static_cast<char *>(b->d_out);
        for (int i = 0; i < npieces; i++) {
            const int r0 = i * piece, n = std::min(piece, rows - r0);
            QL_TRY(cudaStreamWaitEvent(b->stream, b->chunk_events[i], 0));
            st = run_device_impl(b, w, d_in + r0 * in_row, QLINEAR_F32,
                                 single_output(d_out + r0 * out_row), QLINEAR_F32, width, n,
                                 flags, b->stream);
            if (st) {
                cudaStreamSynchronize(b->stream_in);
                return st;
            }
            QL_TRY(cudaMemcpy2DAsync(c_host + (size_t)r0 * ldc, (size_t)ldc * sizeof(float),
                                     d_out + r0 * out_row, out_row, out_row, n,
                                     cudaMemcpyDeviceToHost, b->stream));
        }
        QL_TRY(cudaMemcpyAsync(b->h_err, b->d_err, sizeof(unsigned), cudaMemcpyDeviceToHost,
                               b->stream));
        QL_TRY(cudaStreamSynchronize(b->stream));
        if (*b->h_err) {
            cudaMemsetAsync(b->d_err, 0, sizeof(unsigned), b->stream);
            cudaStreamSynchronize(b->stream);
            reset_after_timeout(b);
            return QLINEAR_ERR_TIMEOUT;
        }
        return QLINEAR_OK;
    }
    if ((st = ensure_host(&b->h_in, &b->h_in_bytes, in_bytes)) ||
        (st = ensure_host(&b->h_out, &b->h_out_bytes, out_bytes)) ||
        (st = ensure_dev(&b->d_in, &b->d_in_bytes, in_bytes)) ||
        (st = ensure_dev(&b->d_out, &b->d_out_bytes, out_bytes)))
        return st;
    if (!b->pool) {
        const unsigned hw = std::thread::hardware_concurrency();
        b->pool.reset(new (std::nothrow) HostPool((int)std::min(16u, std::max(1u, hw)) - 1));
        if (!b->pool) return QLINEAR_ERR_ALLOC;
    }
    HostPool &pool = *b->pool;
    // Input: row chunks of ~2 MB copied into pinned staging by the pool, each sent as soon
    // as it is staged, so the next chunk's copy overlaps the previous chunk's transfer.
    const size_t in_row = (size_t)v.K * sizeof(float), out_row = (size_t)width * sizeof(float);
    char *h_in = static_cast<char *>(b->h_in), *d_in = static_cast<char *>(b->d_in);
    const int in_chunk = (int)std::max<size_t>(1, (2u << 20) / in_row);
    for (int r0 = 0; r0 < rows; r0 += in_chunk) {
        const int n = std::min(in_chunk, rows - r0);
        pool.copy_rows(h_in + r0 * in_row, in_row, a_host + (size_t)r0 * v.K, in_row, n, in_row);
        QL_TRY(cudaMemcpyAsync(d_in + r0 * in_row, h_in + r0 * in_row, n * in_row,
                               cudaMemcpyHostToDevice, b->stream));
    }
    st = run_device_impl(b, w, b->d_in, QLINEAR_F32, single_output(b->d_out), QLINEAR_F32, width,
                         rows, flags, b->stream);
    if (st) return st;
    // Output: row chunks of ~4 MB, each transfer followed by an event; each chunk is copied
    // to the caller's rows (stride ldc) while the next ones are still in transit.
    int out_chunk = (int)std::max<size_t>(1, (4u << 20) / out_row);
    const int kMaxChunks = 64;
    out_chunk = std::max(out_chunk, (rows + kMaxChunks - 1) / kMaxChunks);
    const int nchunks = (rows + out_chunk - 1) / out_chunk;
    while ((int)b->chunk_events.size() < nchunks) {
        cudaEvent_t e;
        QL_TRY(cudaEventCreateWithFlags(&e, cudaEventDisableTiming));
        b->chunk_events.push_back(e);
    }
    char *h_out = static_cast<char *>(b->h_out), *d_out = static_cast<char *>(b->d_out);
    for (int i = 0; i < nchunks; i++) {
        const int r0 = i * out_chunk, n = std::min(out_chunk, rows - r0);
        QL_TRY(cudaMemcpyAsync(h_out + r0 * out_row, d_out + r0 * out_row, n * out_row,
                               cudaMemcpyDeviceToHost, b->stream));
        QL_TRY(cudaEventRecord(b->chunk_events[i], b->stream));
    }
    QL_TRY(cudaMemcpyAsync(b->h_err, b->d_err, sizeof(unsigned), cudaMemcpyDeviceToHost, b->stream));
    for (int i = 0; i < nchunks; i++) {
        const int r0 = i * out_chunk, n = std::min(out_chunk, rows - r0);
        QL_TRY(cudaEventSynchronize(b->chunk_events[i]));
        pool.copy_rows(c_host + (size_t)r0 * ldc, (size_t)ldc * sizeof(float), h_out + r0 * out_row,
                       out_row, n, out_row);
    }
    QL_TRY(cudaStreamSynchronize(b->stream));
    if (*b->h_err) {
        cudaMemsetAsync(b->d_err, 0, sizeof(unsigned), b->stream);
        cudaStreamSynchronize(b->stream);
        reset_after_timeout(b);
        return QLINEAR_ERR_TIMEOUT;
    }
    return QLINEAR_OK;
}

int qlinear_run_f32(qlinear_backend *b, const qlinear_weights *w, const float *a_host,
                    float *c_host, int rows) {
    const long long width = w ? w->view.N : 0;
    return run_host(b, w, a_host, c_host, width, rows, 0);
}

int qlinear_run_swiglu_f32(qlinear_backend *b, const qlinear_weights *w, const float *a_host,
                           float *c_host, int rows) {
    const long long width = w ? w->view.N / 2 : 0;
    return run_host(b, w, a_host, c_host, width, rows, QLINEAR_RUN_SWIGLU);
}

int qlinear_run_f32_ex(qlinear_backend *b, const qlinear_weights *w, const float *a_host,
                       float *c_host, long long ldc, int rows, unsigned flags) {
    return run_host(b, w, a_host, c_host, ldc, rows, flags);
}

int qlinear_act_quant_device(qlinear_backend *b, const void *a_dev, int a_type, int rows, int K,
                             int8_t *codes_dev, float *scales_dev, int32_t *rowsums_dev,
                             void *stream) {
    if (!b || !a_dev || !codes_dev || !scales_dev || rows < 1 || K < 1 || !valid_io_type(a_type))
        return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    QL_TRY(launch_act_quant(a_dev, a_type, K, rows, K, K, b->round_mode, codes_dev, scales_dev,
                            rowsums_dev, static_cast<cudaStream_t>(stream)));
    b->launches++;
    return QLINEAR_OK;
}

int qlinear_row_amax_device(qlinear_backend *b, const void *a_dev, int a_type, int rows, int K,
                            float *amax_dev, void *stream) {
    if (!b || !a_dev || !amax_dev || rows < 1 || K < 1 || !valid_io_type(a_type))
        return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    QL_TRY(launch_row_amax(a_dev, a_type, K, rows, K, amax_dev, static_cast<cudaStream_t>(stream)));
    b->launches++;
    return QLINEAR_OK;
}

int qlinear_run_device_amax(qlinear_backend *b, const qlinear_weights *w, const void *a_dev,
                            int a_type, const float *row_amax_dev, void *c_dev, int c_type,
                            long long ldc, int rows, void *stream) {
    if (!b || !w || w->backend != b || !row_amax_dev) return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    return run_device_impl(b, w, a_dev, a_type, single_output(c_dev), c_type, ldc, rows, 0,
                           static_cast<cudaStream_t>(stream), row_amax_dev);
}

int qlinear_dequant_device(qlinear_backend *b, const qlinear_weights *w, const int32_t *acc_dev,
                           long long lda, const float *row_amax_dev, void *c_dev, int c_type,
                           long long ldc, int rows, void *stream) {
    if (!b || !w || w->backend != b || !acc_dev || !row_amax_dev || !c_dev || rows < 1 ||
        !valid_io_type(c_type) || lda < w->view.N || ldc < w->view.N)
        return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    QL_TRY(launch_dequant(acc_dev, lda, row_amax_dev, w->view.scales, rows, w->view.N, c_dev,
                          c_type, ldc, b->num_sms, static_cast<cudaStream_t>(stream)));
    b->launches++;
    return QLINEAR_OK;
}

int qlinear_swiglu_device(qlinear_backend *b, const float *y_dev, int rows, int N, void *c_dev,
                          int c_type, long long ldc, void *stream) {
    if (!b || !y_dev || !c_dev || rows < 1 || N < 2 || N % 2 || ldc < N / 2 ||
        (c_type != QLINEAR_F16 && c_type != QLINEAR_F32))
        return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    QL_TRY(launch_swiglu(y_dev, rows, N, c_dev, c_type == QLINEAR_F16 ? kF16 : kF32, ldc,
                         static_cast<cudaStream_t>(stream)));
    b->launches++;
    return QLINEAR_OK;
}

int qlinear_interleave_columns(qlinear_backend *b, const void *src, void *dst, int shards,
                               int rows, int shard_cols, int elem_bytes, void *stream) {
    if (!b || !src || !dst || shards < 1 || rows < 1 || shard_cols < 1 ||
        (elem_bytes != 2 && elem_bytes != 4))
        return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    QL_TRY(launch_interleave(src, dst, shards, rows, shard_cols, elem_bytes, b->num_sms,
                             static_cast<cudaStream_t>(stream)));
    b->launches++;
    return QLINEAR_OK;
}

int qlinear_backend_profile(qlinear_backend *b, int enable) {
    if (!b) return QLINEAR_ERR_PARAM;
    b->profiling = enable != 0;
    return QLINEAR_OK;
}

int qlinear_backend_profile_collect(qlinear_backend *b, double *quant_ms, double *main_ms,
                                    int *calls) {
    if (!b) return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    double q = 0, m = 0;
    for (size_t i = 0; i < b->prof_used; i++) {
        auto &e = b->prof_events[i];
        QL_TRY(cudaEventSynchronize(e[2]));
        float a = 0, c = 0;
        QL_TRY(cudaEventElapsedTime(&a, e[0], e[1]));
        QL_TRY(cudaEventElapsedTime(&c, e[1], e[2]));
        q += a;
        m += c;
    }
    if (quant_ms) *quant_ms = q;
    if (main_ms) *main_ms = m;
    if (calls) *calls = (int)b->prof_used;
    b->prof_used = 0;
    return QLINEAR_OK;
}

int qlinear_backend_check(qlinear_backend *b, void *stream) {
    if (!b) return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    QL_TRY(cudaStreamSynchronize(s));
    QL_TRY(cudaMemcpy(b->h_err, b->d_err, sizeof(unsigned), cudaMemcpyDeviceToHost));
    if (*b->h_err) {
        QL_TRY(cudaMemset(b->d_err, 0, sizeof(unsigned)));
        reset_after_timeout(b);
        return QLINEAR_ERR_TIMEOUT;
    }
    return QLINEAR_OK;
}

int qlinear_peer_signal_wait(qlinear_backend *b, void *const *sig, int world, int rank,
                             unsigned long long epoch, unsigned long long limit_ns,
                             void *stream) {
    if (!b || !sig || world < 1 || world > kMaxOutputs || rank < 0 || rank >= world)
        return QLINEAR_ERR_PARAM;
    PeerSignals s{};
    for (int r = 0; r < world; r++) {
        if (!sig[r]) return QLINEAR_ERR_PARAM;
        s.sig[r] = sig[r];
    }
    s.world = world;
    s.rank = rank;
    DeviceGuard guard(b->device);
    QL_TRY(launch_peer_signal_wait(s, epoch, b->d_err, limit_ns ? limit_ns : QL_WAIT_NS,
                                   static_cast<cudaStream_t>(stream)));
    b->launches++;
    return QLINEAR_OK;
}

int qlinear_selftest_wait_timeout(qlinear_backend *b, unsigned long long limit_ns) {
    if (!b || limit_ns < 1000000ull || limit_ns > 2000000000ull) return QLINEAR_ERR_PARAM;
    DeviceGuard guard(b->device);
    QL_TRY(launch_wait_selftest(b->d_err, limit_ns, b->stream));
    b->launches++;
    return qlinear_backend_check(b, b->stream);
}

int qlinear_backend_stats(const qlinear_backend *b, char *buf, size_t len) {
    if (!b) return QLINEAR_ERR_PARAM;
    const size_t ws = b->ws_bytes + b->ws_rows * 8 + b->y_elems + b->d_in_bytes + b->d_out_bytes;
    char tmp[2048];
    const int n = std::snprintf(
        tmp, sizeof(tmp),
        "{\"backend\": \"cuda-sm100a\", \"device\": %d, \"sm_count\": %d, \"loaded_w4\": %d, "
        "\"loaded_w8\": %d, \"weight_payload_bytes\": %llu, \"workspace_payload_bytes\": %llu, "
        "\"workspace_count\": %d, \"host_staging_bytes\": %llu, \"tune_cache_hits\": 0, "
        "\"tune_cache_misses\": 0, \"tune_calls\": 0, \"strategy_fallbacks\": 0, "
        "\"strategy_fallback_calls\": 0, \"weight_reload_calls\": 0, \"round_mode\": \"%s\", "
        "\"prepared_rows\": %d, \"kernel_launches\": %llu, \"gemv_calls\": %llu, "
        "\"gemm_calls\": %llu, \"gemm_stream_k_calls\": %llu, \"gemm_swiglu_fused_calls\": %llu, "
        "\"mlp_calls\": %llu, \"w4_prefill\": \"%s\", "
        "\"gemm_pairs_resident\": [%d, %d]}",
        b->device, b->num_sms, b->loaded_w4, b->loaded_w8, (unsigned long long)b->weight_bytes,
        (unsigned long long)ws, b->ws_bytes ? 1 : 0,
        (unsigned long long)(b->h_in_bytes + b->h_out_bytes),
        b->round_mode == QLINEAR_ROUND_AWAY ? "away" : "even", b->prepared_rows, b->launches,
        b->gemv_calls, b->gemm_calls, b->gemm_stream_k_calls, b->gemm_glu_calls, b->mlp_calls,
        (b->flags & QLINEAR_BACKEND_W4_PACKED_ONLY) ? "packed" : "int8 copy",
        b->gemm_pairs[0], b->gemm_pairs[1]);
    if (n < 0) return QLINEAR_ERR_PARAM;
    if (buf && len) {
        std::strncpy(buf, tmp, len - 1);
        buf[len - 1] = 0;
    }
    return n;
}

unsigned long long qlinear_backend_launches(const qlinear_backend *b) { return b ? b->launches : 0; }

const char *qlinear_strerror(int status) {
    switch (status) {
    case QLINEAR_OK: return "ok";
    case QLINEAR_ERR_PARAM: return "invalid argument";
    case QLINEAR_ERR_ALLOC: return "allocation failed";
    case QLINEAR_ERR_CUDA: return "CUDA error";
    case QLINEAR_ERR_UNSUPPORTED: return "unsupported";
    case QLINEAR_ERR_TIMEOUT: return "device wait timed out";
    case QLINEAR_ERR_NCCL: return "NCCL error";
    case QLINEAR_ERR_STATE: return "invalid state";
    case QLINEAR_ERR_LIMIT: return "request exceeds a fixed limit of this call";
    default: return "unknown status";
    }
}

int qlinear_last_status(void) { return g_last_status; }

const char *qlinear_version(void) { return "qlinear-b200 0.1.0 (sm_100a)"; }

}  // extern "C"
