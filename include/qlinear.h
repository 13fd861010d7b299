/*
 * qlinear.h -- C ABI of the B200 (sm_100a) quantized-linear library.
 *
 * Drop-in replacement for the subset of the rk_npu_* C ABI that open_rknpu2_lm_infer's
 * quantized-linear backend binds through bindgen (build.rs:49-68, allowlist rk_npu_.*)
 * and calls from src/npu.rs.  The mapping, function by function, is given beside each
 * declaration as "replaces <reference call> (file:line)".
 *
 * Path: dynamic per-token symmetric int8 activation quantisation -> W4/W8 x int8
 * GEMM/GEMV with exact int32 accumulation -> (f32(acc) * s_a) * s_w epilogue, written as
 * f32 (host API, bit-exact with the reference's CPU oracle src/npu.rs:1097-1121) or fp16
 * (device API, the same f32 value rounded once to nearest-even).
 *
 * Conventions (mirroring the reference's):
 *   - object handles are opaque; *_create returns NULL on failure (src/npu.rs:123-131)
 *     and qlinear_last_status() then gives the reason;
 *   - every other call returns an int status, 0 = QLINEAR_OK; qlinear_strerror()
 *     gives its text (src/npu.rs:138-144);
 *   - weight codes are passed in the reference's QuantMatrix layout: int8 [K][N]
 *     row-major, element (k, n) at codes[k*N + n] (src/npu.rs:112-118, :1115), W4 codes
 *     in [-8, 7] one per byte, W8 codes in [-127, 127]; scales f32 [N], > 0;
 *   - a backend and everything created from it are used from one host thread at a time
 *     (the reference's Backend is Rc<RefCell<..>>, src/npu.rs:252-254);
 *   - nothing aborts or traps; device-side waits are bounded and report
 *     QLINEAR_ERR_TIMEOUT.
 *
 * No symbol here uses torch or CUDA runtime types: streams are passed as void*
 * (a cudaStream_t), device buffers as plain pointers.
 */
#ifndef QLINEAR_H
#define QLINEAR_H

#include <stddef.h>
#include <stdint.h>

#if defined(__GNUC__)
#define QLINEAR_API __attribute__((visibility("default")))
#else
#define QLINEAR_API
#endif

#ifdef __cplusplus
extern "C" {
#endif

/* ---- status codes (replace RK_NPU_ERR_*, src/npu.rs:138-151) ---------------------- */
#define QLINEAR_OK 0
#define QLINEAR_ERR_PARAM (-1)       /* invalid argument or shape (RK_NPU_ERR_PARAM) */
#define QLINEAR_ERR_ALLOC (-2)       /* device or pinned allocation failed */
#define QLINEAR_ERR_CUDA (-3)        /* a CUDA runtime/driver call failed */
#define QLINEAR_ERR_UNSUPPORTED (-4) /* valid request this build does not implement */
#define QLINEAR_ERR_TIMEOUT (-5)     /* a bounded device-side wait gave up */
#define QLINEAR_ERR_NCCL (-6)        /* an NCCL call failed */
#define QLINEAR_ERR_STATE (-7)       /* object used in the wrong state */
#define QLINEAR_ERR_LIMIT (-8)       /* request exceeds a fixed maximum (see the call's limits) */

/* ---- rounding of the activation quantiser ------------------------------------------ */
#define QLINEAR_ROUND_AWAY 0 /* f32::round, ties away from zero: the reference (src/npu.rs:1109) */
#define QLINEAR_ROUND_EVEN 1 /* round half to even (opt-in; not the reference's) */

/* ---- element types of device buffers ----------------------------------------------- */
#define QLINEAR_F32 0
#define QLINEAR_F16 1
#define QLINEAR_I32 2 /* output only: raw int32 accumulators (parity export) */

/* ---- run flags ----------------------------------------------------------------------- */
#define QLINEAR_RUN_SWIGLU 1u /* out[m][j] = silu(y[m][j]) * y[m][N/2 + j], width N/2 */

typedef struct qlinear_backend qlinear_backend;
typedef struct qlinear_weights qlinear_weights;

/* ---- backend flags ------------------------------------------------------------------- */
/* W4 weights normally keep two device copies: the packed nibbles (read by the HBM-bound
 * decode GEMV) and an int8 expansion (read by the tensor-core prefill GEMM, which is
 * compute-bound, so the doubled bytes cost little time).  With this flag only the packed
 * copy is kept and the prefill GEMM unpacks the nibbles in shared memory instead
 * (0.5 byte per weight instead of 1.5, at a lower prefill throughput). */
#define QLINEAR_BACKEND_W4_PACKED_ONLY 1u
/* Let the prefill GEMM use its stream-K schedule where whole tiles would leave CTA pairs
 * idle (every pair then takes the same number of k-blocks; split tiles are summed exactly
 * in an int32 workspace, so results are bit-identical).  Off by default: on B200 the pass
 * that finishes split tiles is bound by the epilogue's output stores and loses to the
 * whole-tile schedule on every shape measured so far. */
#define QLINEAR_BACKEND_GEMM_STREAM_K 2u
/* Run the prefill SwiGLU (QLINEAR_RUN_SWIGLU above the decode row count) as the GEMM into
 * an f32 [rows][N] workspace followed by a separate SiLU-gated-product pass, instead of the
 * GEMM whose epilogue computes the product (the default for weights with an 8-bit prefill
 * copy).  Both give bit-identical results; this is for comparison and testing. */
#define QLINEAR_BACKEND_SWIGLU_UNFUSED 4u

typedef struct qlinear_backend_config {
    int device;     /* CUDA device ordinal (replaces the IOMMU domain id, src/npu.rs:310) */
    int round_mode; /* QLINEAR_ROUND_AWAY (default) or QLINEAR_ROUND_EVEN */
    int max_rows;   /* rows one host call may stage without reallocating; 0 = 256 */
    unsigned flags; /* QLINEAR_BACKEND_* */
} qlinear_backend_config;

typedef struct qlinear_weight_config {
    int bits; /* 4 or 8 */
    int K;    /* input features  (> 0) */
    int N;    /* output features (> 0) */
    int reserved;
} qlinear_weight_config;

typedef struct qlinear_weight_info {
    int bits, K, N;
    int K_padded;          /* K rounded up to the GEMM's 128-element k-block */
    int N_padded;          /* N rounded up to the 128-channel tile */
    uint64_t device_bytes; /* bytes of device memory the weights (all copies) and scales hold */
} qlinear_weight_info;

/* Fills cfg with defaults (device 0, ties-away, 256 rows). */
QLINEAR_API void qlinear_backend_config_init(qlinear_backend_config *cfg);

/* Replaces rk_npu_open + rk_npu_iommu_domain_create (src/npu.rs:310-366). */
QLINEAR_API qlinear_backend *qlinear_backend_create(const qlinear_backend_config *cfg);
/* Replaces rk_npu_iommu_domain_free + rk_npu_close (Handle drop, src/npu.rs:133-137).
 * Releases the caller's handle; every weights object holds its backend (as the reference's
 * Linear holds a Backend clone, src/npu.rs:252-260), so the device resources go when the
 * handle and the last weights object of the backend have both been freed, in either order. */
QLINEAR_API void qlinear_backend_free(qlinear_backend *backend);

/* Replaces rk_npu_w4a8_weights_create (src/npu.rs:395-402) for bits == 4 and
 * rk_npu_f32i8f32_weights_create (src/npu.rs:438-445) for bits == 8: copies codes
 * [K][N] and scales [N] (host memory) into the device layout. */
QLINEAR_API qlinear_weights *qlinear_weights_create(qlinear_backend *backend, const qlinear_weight_config *cfg,
                                        const int8_t *codes_kn, const float *scales);
/* Same, keeping only output columns [n_begin, n_end) of the matrix: the column-parallel
 * (split-N) shard of one rank.  No reference counterpart (the reference is single-device). */
QLINEAR_API qlinear_weights *qlinear_weights_create_shard(qlinear_backend *backend,
                                              const qlinear_weight_config *cfg,
                                              const int8_t *codes_kn, const float *scales,
                                              int n_begin, int n_end);
/* Same, from the checkpoint's compressed-tensors storage without the [K][N] transpose:
 * bits == 4: weight_packed int32 [N][ceil(K/8)], nibble j of word w is k = 8w + j,
 * stored as code + 8 (src/model/checkpoint.rs:352-371); bits == 8: weight int8 [N][K]
 * (src/model/checkpoint.rs:372-378). */
QLINEAR_API qlinear_weights *qlinear_weights_create_checkpoint(qlinear_backend *backend,
                                                   const qlinear_weight_config *cfg,
                                                   const void *storage, const float *scales);
/* Replaces rk_npu_w4a8_weights_query / rk_npu_i4_weights_memory_query /
 * rk_npu_f32i8f32_weights_memory_query (src/npu.rs:404-426, :447-453). */
QLINEAR_API int qlinear_weights_query(const qlinear_weights *weights, qlinear_weight_info *info);
/* Replaces rk_npu_w4a8_weights_free / rk_npu_f32i8f32_weights_free. */
QLINEAR_API void qlinear_weights_free(qlinear_weights *weights);

/* Replaces the workspace creation of Backend::prepare/get_work (src/npu.rs:595-615,
 * :941-996): makes the per-call workspaces large enough for `rows` rows of every K/N
 * loaded so far.  Optional: run calls grow the workspace on demand. */
QLINEAR_API int qlinear_backend_prepare(qlinear_backend *backend, int rows);

/* Replaces rk_npu_w4a8_run_f32 (src/npu.rs:1047) and rk_npu_f32i8f32_run_dynamic
 * (src/npu.rs:1054): a_host f32 [rows][K] -> c_host f32 [rows][N], synchronous.
 * Unlike the reference (rows <= 256, src/npu.rs:152-156) any rows >= 1 is accepted.
 * Host buffers in ordinary (pageable) memory go through the backend's pinned staging;
 * page-locked buffers (cudaHostAlloc / cudaHostRegister) are copied by DMA directly. */
QLINEAR_API int qlinear_run_f32(qlinear_backend *backend, const qlinear_weights *weights, const float *a_host,
                    float *c_host, int rows);
/* Replaces rk_npu_w4a8_run_swiglu_f32 (src/npu.rs:1045): c_host f32 [rows][N/2] with
 * c[m][j] = silu(y[m][j]) * y[m][N/2 + j].  N must be even.  Works for W4 and W8. */
QLINEAR_API int qlinear_run_swiglu_f32(qlinear_backend *backend, const qlinear_weights *weights,
                           const float *a_host, float *c_host, int rows);

/* The host path writing into a wider output: c_host f32 rows of stride ldc >= the output
 * width (N, or N/2 with QLINEAR_RUN_SWIGLU in flags), columns [0, width) of each row;
 * the rest of each row is left untouched.  This is what Projection::run_from
 * (src/model/projection.rs:200-232) does with a scratch buffer and a row-by-row copy when a
 * fused projection is stored as several linears (mixed bit widths): each part writes its
 * column range of the fused [rows][width] output directly (pass c_host + column offset). */
QLINEAR_API int qlinear_run_f32_ex(qlinear_backend *backend, const qlinear_weights *weights,
                                   const float *a_host, float *c_host, long long ldc, int rows,
                                   unsigned flags);

/* Device-resident path (no reference counterpart; the benchmark and multi-GPU path):
 * a_dev [rows][K] of a_type (QLINEAR_F16 or QLINEAR_F32), c_dev [rows][ldc] of c_type
 * (QLINEAR_F16, QLINEAR_F32 or QLINEAR_I32 raw accumulators), ldc >= output width
 * (N, or N/2 with QLINEAR_RUN_SWIGLU).  Asynchronous on `stream` (a cudaStream_t; NULL =
 * the legacy default stream).  Uses the backend's device workspace, so calls on one
 * backend must be ordered on one stream. */
QLINEAR_API int qlinear_run_device(qlinear_backend *backend, const qlinear_weights *weights,
                       const void *a_dev, int a_type, void *c_dev, int c_type, long long ldc,
                       int rows, unsigned flags, void *stream);

/* The MLP block of a decoder layer, replacing the two calls of src/model/dense.rs:499-530
 * (gate_up.run_swiglu(normalized -> middle), then down.run(middle -> projected)):
 * c_dev [rows][ldc] (ldc >= N of down) = down(silu(g) * u) with [g | u] = gate_up(a_dev), the
 * [rows][N/2] middle kept in f32 as in the reference (so the result is that of the two calls
 * with an f32 middle, bit for bit).  gate_up: N even, gate columns first; down: K = N/2 of
 * gate_up.  a_type / c_type: QLINEAR_F16 or QLINEAR_F32.  The middle lives in a backend
 * scratch buffer; the two GEMV/GEMM calls run back to back, the second one's weight stream
 * starting while the first drains.  Asynchronous on `stream`; the same ordering rule as
 * qlinear_run_device. */
QLINEAR_API int qlinear_run_mlp_device(qlinear_backend *backend, const qlinear_weights *gate_up,
                                       const qlinear_weights *down, const void *a_dev,
                                       int a_type, void *c_dev, int c_type, long long ldc,
                                       int rows, void *stream);

/* Split-N output exchange fused into the kernels (no reference counterpart; one process per
 * GPU, the layer's output columns sharded over the GPUs of one node): like
 * qlinear_run_device, but the kernels' epilogues store every output element into each of
 * the ndev (1..8) buffers c_devs[] -- this GPU's own and the peers' (opened with
 * qlinear_peer_buffer_open) -- at row m, column col_offset + n, row stride ldc.  The stores
 * to peers cross NVLink while the kernel computes; the kernels end with a system-scope
 * fence, so a signal issued on the same stream afterwards (qlinear_peer_signal_wait, or a
 * collective such as a one-element NCCL all-reduce) tells every peer that this rank's
 * columns are in place.  The caller must keep
 * peers from reading the destination rows until then, and from being written by a later
 * call while they still read them.  SwiGLU through the tensor-core path (rows > 8) is not
 * supported here (QLINEAR_ERR_UNSUPPORTED). */
QLINEAR_API int qlinear_run_device_scatter(qlinear_backend *backend, const qlinear_weights *weights,
                                           const void *a_dev, int a_type, void *const *c_devs,
                                           int ndev, int c_type, long long ldc, long long col_offset,
                                           int rows, unsigned flags, void *stream);

/* The split-N exchange through NVSwitch multicast (no reference counterpart): as
 * qlinear_run_device_scatter without SwiGLU, with mc_dev the multicast address (NVLS) bound to
 * every rank's exchange buffer (the same layout as c_devs[], whose first entry is this GPU's
 * own).  The tensor-core GEMM (rows above the decode path's 8) stores each output element
 * once through mc_dev and the switch writes it into every rank's buffer, so each GPU sends
 * its columns over NVLink once instead of once per peer; the decode GEMV stores to c_devs[]
 * as qlinear_run_device_scatter does.  fp16 output: col_offset, ldc and N must be even
 * (multimem stores are 32 bits wide).  The kernels end with a system-scope fence, as for
 * qlinear_run_device_scatter. */
QLINEAR_API int qlinear_run_device_multicast(qlinear_backend *backend,
                                             const qlinear_weights *weights, const void *a_dev,
                                             int a_type, void *const *c_devs, int ndev,
                                             void *mc_dev, int c_type, long long ldc,
                                             long long col_offset, int rows, void *stream);

/* Exchange buffers for qlinear_run_device_scatter: qlinear_peer_buffer_create allocates
 * `bytes` of device memory on the backend's GPU and writes its CUDA IPC handle
 * (QLINEAR_IPC_HANDLE_BYTES bytes) to ipc_handle; another process opens that handle with
 * qlinear_peer_buffer_open and gets a pointer its kernels can store to over NVLink;
 * qlinear_peer_buffer_free releases either kind (opened = 1 for a pointer from
 * qlinear_peer_buffer_open).  New buffers are zero-filled. */
#define QLINEAR_IPC_HANDLE_BYTES 64
QLINEAR_API int qlinear_peer_buffer_create(qlinear_backend *backend, size_t bytes, void **dev_ptr,
                                           unsigned char *ipc_handle);
QLINEAR_API int qlinear_peer_buffer_open(qlinear_backend *backend, const unsigned char *ipc_handle,
                                         void **dev_ptr);
QLINEAR_API int qlinear_peer_buffer_free(qlinear_backend *backend, void *dev_ptr, int opened);

/* Completion signal of the split-N exchange, on `stream` after this rank's
 * qlinear_run_device_scatter: raises this rank's flag to `epoch` in every rank's signal
 * array, then waits until all `world` flags in this GPU's array have reached `epoch`, so
 * work queued on `stream` afterwards sees every rank's columns.  sig[r]: rank r's signal
 * array as mapped in this process (sig[rank] = this GPU's own), a peer buffer of at least
 * 8 * world bytes, zero at creation.  epoch: 1, 2, 3, ... -- the same sequence on every
 * rank.  limit_ns: how long the wait may take (0: 2 s); past it the kernel records a timeout
 * that qlinear_backend_check reports as QLINEAR_ERR_TIMEOUT, and returns.  Asynchronous;
 * QLINEAR_ERR_PARAM for world outside 1..8 or rank outside [0, world). */
QLINEAR_API int qlinear_peer_signal_wait(qlinear_backend *backend, void *const *sig, int world,
                                         int rank, unsigned long long epoch,
                                         unsigned long long limit_ns, void *stream);

/* Activation quantisation alone (parity export of the int8 codes): a_dev [rows][K] ->
 * codes_dev int8 [rows][K], scales_dev f32 [rows], rowsums_dev int32 [rows] (may be NULL;
 * sum of the row's codes).  Asynchronous on `stream`. */
QLINEAR_API int qlinear_act_quant_device(qlinear_backend *backend, const void *a_dev, int a_type, int rows,
                             int K, int8_t *codes_dev, float *scales_dev, int32_t *rowsums_dev,
                             void *stream);

/* Row-parallel (split-K) linear over ranks (no reference counterpart; the reference is
 * single-device).  A rank holds the weight rows of its K slice (a weights object of K_slice
 * inputs) and the matching slice of every activation row.  The reference's arithmetic
 * (src/npu.rs:1099-1117) is kept exactly:
 *   qlinear_row_amax_device: amax_dev[m] = max |a[m][:]| of this slice (NaN ignored);
 *   (the caller takes the max over the ranks, e.g. an all-reduce MAX)
 *   qlinear_run_device_amax: the slice quantised with the scale of the given whole-row max
 *     (so the codes are those of the whole row), c_type QLINEAR_I32 gives this slice's exact
 *     int32 partial accumulators (the W4 offset already removed);
 *   (the caller sums the partial accumulators over the ranks, e.g. an int32 all-reduce SUM)
 *   qlinear_dequant_device: c[m][n] = (f32(acc[m][n]) * s_a[m]) * s_w[n], s_a the scale of
 *     row_amax[m], s_w the weights' scales (every rank's slice has the same N and scales).
 * The result equals the unsplit linear bit for bit.  Asynchronous on `stream`. */
QLINEAR_API int qlinear_row_amax_device(qlinear_backend *backend, const void *a_dev, int a_type,
                                        int rows, int K, float *amax_dev, void *stream);
QLINEAR_API int qlinear_run_device_amax(qlinear_backend *backend, const qlinear_weights *weights,
                                        const void *a_dev, int a_type, const float *row_amax_dev,
                                        void *c_dev, int c_type, long long ldc, int rows,
                                        void *stream);
QLINEAR_API int qlinear_dequant_device(qlinear_backend *backend, const qlinear_weights *weights,
                                       const int32_t *acc_dev, long long lda,
                                       const float *row_amax_dev, void *c_dev, int c_type,
                                       long long ldc, int rows, void *stream);

/* SiLU-gated product of a gate/up projection output held on the device, replacing the CPU
 * fallback of src/model/dense.rs:509-523 (`gate_up.run` into [rows][2f], then `Cpu::swiglu`,
 * src/model/cpu.rs:327-351), which the reference takes when gate and up have different bit
 * widths and so are two matrices: y_dev f32 [rows][N] (gate columns [0, N/2), up [N/2, N)),
 * c_dev [rows][ldc] of c_type (QLINEAR_F16 or QLINEAR_F32), ldc >= N/2,
 * c[m][j] = silu(y[m][j]) * y[m][N/2 + j] with the same f32 arithmetic as the fused SwiGLU
 * epilogues.  Asynchronous on `stream`. */
QLINEAR_API int qlinear_swiglu_device(qlinear_backend *backend, const float *y_dev, int rows,
                                      int N, void *c_dev, int c_type, long long ldc,
                                      void *stream);

/* Column-parallel (split-N) output assembly: src holds `shards` slabs [rows][shard_cols]
 * back to back (the layout an all-gather of per-rank outputs produces), dst is
 * [rows][shards * shard_cols] with dst[m][s * shard_cols + j] = src[s][m][j].  elem_bytes
 * is 2 (fp16) or 4 (f32).  Asynchronous on `stream`.  No reference counterpart. */
QLINEAR_API int qlinear_interleave_columns(qlinear_backend *backend, const void *src, void *dst,
                                           int shards, int rows, int shard_cols, int elem_bytes,
                                           void *stream);

/* Per-kernel device timing (the role of the `timings` argument of rk_npu_w4a8_run_f32,
 * src/npu.rs:1047): while enabled, every run records CUDA events around its activation
 * quantisation and around its main kernel (GEMM or GEMV) on the call's stream.
 * qlinear_backend_profile_collect synchronizes those events, returns the summed
 * milliseconds and the number of calls, and clears the record. */
QLINEAR_API int qlinear_backend_profile(qlinear_backend *backend, int enable);
QLINEAR_API int qlinear_backend_profile_collect(qlinear_backend *backend, double *quant_ms,
                                                double *main_ms, int *calls);

/* Allocation-free decode call.  No counterpart in the reference.  For callers that cannot
 * allocate device memory while they run a layer: a process whose device memory is
 * entirely reserved up front by its own pool allocator, or a latency-critical decode loop
 * that must not call cudaMalloc/cudaFree (which can synchronise the device and stall every
 * stream).  Same arithmetic and results as qlinear_run_device (plain output, no SwiGLU),
 * but the activation codes, scales and row sums live in a fixed scratch array compiled
 * into the library (a file-scope __device__ array of QLINEAR_NOALLOC_SCRATCH_BYTES, held by
 * every GPU that loads the library until the process exits) instead of the backend's
 * workspace.  The call allocates nothing, on the device or the host.
 *   Limits: rows <= QLINEAR_NOALLOC_MAX_ROWS and K (rounded up to 128) <= QLINEAR_NOALLOC_MAX_K;
 *   larger requests return QLINEAR_ERR_LIMIT without launching anything.
 *   The first call on a device looks the scratch up (cudaGetSymbolAddress, which may load
 *   the library's device code on that device) and keeps its address for the life of the
 *   process; make that first call before any stream capture, and do not reset the device
 *   (cudaDeviceReset) while using this call.
 *   All calls on a device share the one scratch array: calls whose kernels can overlap on
 *   the GPU (different streams, or different host threads) race and corrupt each other's
 *   codes.  Order them on one stream.  Each call rewrites everything it reads back. */
#define QLINEAR_NOALLOC_MAX_ROWS 8
#define QLINEAR_NOALLOC_MAX_K 16384
#define QLINEAR_NOALLOC_SCRATCH_BYTES \
    (QLINEAR_NOALLOC_MAX_ROWS * QLINEAR_NOALLOC_MAX_K + 8 * QLINEAR_NOALLOC_MAX_ROWS)
QLINEAR_API int qlinear_run_device_noalloc(const qlinear_weights *weights, const void *a_dev,
                                           int a_type, void *c_dev, int c_type, long long ldc,
                                           int rows, void *stream);

/* Reads and clears the backend's device error word (bounded waits that gave up);
 * synchronizes `stream` first.  Returns QLINEAR_OK or QLINEAR_ERR_TIMEOUT. */
QLINEAR_API int qlinear_backend_check(qlinear_backend *backend, void *stream);

/* Failure-path self-test (no reference counterpart): launches one warp that waits on an
 * mbarrier nothing arrives on.  After limit_ns (1 ms .. 2 s) the wait gives up, records the
 * timeout in the backend's device error word and the kernel returns, as a stuck pipeline
 * stage of the GEMM would.  Returns QLINEAR_ERR_TIMEOUT, the expected result (the error word
 * is cleared and the backend stays usable); QLINEAR_ERR_PARAM for a limit out of range. */
QLINEAR_API int qlinear_selftest_wait_timeout(qlinear_backend *backend, unsigned long long limit_ns);

/* Replaces Backend::stats (src/npu.rs:631-661): JSON text into buf (NUL-terminated).
 * Returns the length needed (excluding NUL) or a negative status. */
QLINEAR_API int qlinear_backend_stats(const qlinear_backend *backend, char *buf, size_t len);

/* Number of kernels this backend has launched since creation (instrumentation). */
QLINEAR_API unsigned long long qlinear_backend_launches(const qlinear_backend *backend);

/* Replaces rk_npu_strerror (src/npu.rs:138-144). */
QLINEAR_API const char *qlinear_strerror(int status);
/* Status of the last failed *_create on this thread. */
QLINEAR_API int qlinear_last_status(void);
/* Library version string. */
QLINEAR_API const char *qlinear_version(void);

#ifdef __cplusplus
}
#endif

#endif /* QLINEAR_H */
