// noalloc.cu -- the allocation-free decode call (qlinear_run_device_noalloc).
//
// Some callers cannot allocate device memory while they run a layer: a process whose
// device memory is reserved up front by its own pool allocator, or a latency-critical decode
// loop that must not call cudaMalloc/cudaFree (they can synchronise the device).  The
// regular call keeps its activation codes in a workspace the backend allocates on demand;
// this variant keeps them in a fixed scratch array compiled into the library instead, so
// the call itself allocates nothing.  It runs the same two kernels as the regular decode
// path (act-quant, then the GEMV) and produces identical results.
//
// The scratch is one file-scope __device__ array of QLINEAR_NOALLOC_SCRATCH_BYTES (128 KiB
// of codes plus scales and row sums): every GPU that loads the library holds it until the
// process exits.  Host code cannot pass the array's name to a kernel (on the host it is a
// stand-in, not a device address), so the first call on each device, with that device
// current, looks its address up with cudaGetSymbolAddress and keeps it for the life of the
// process (a cudaDeviceReset, which unloads the library's device code, is not supported
// while this call is in use: the kept address would be stale).  All calls on a
// device share the array; calls that overlap on the GPU race.  Nothing in it needs to start
// at zero: act-quant rewrites the codes (and their K padding), scales and row sums of every
// row the GEMV then reads.
#include "../../include/qlinear.h"
#include "common.cuh"
#include "kernels.h"

#include <atomic>

using namespace ql;

namespace {

constexpr int kMaxRows = QLINEAR_NOALLOC_MAX_ROWS;
constexpr int kMaxK = QLINEAR_NOALLOC_MAX_K;
constexpr size_t kCodesBytes = (size_t)kMaxRows * kMaxK;
constexpr size_t kScratchBytes = QLINEAR_NOALLOC_SCRATCH_BYTES;
static_assert(kScratchBytes == kCodesBytes + 4 * kMaxRows + 4 * kMaxRows, "scratch layout");

// codes int8 [kMaxRows][Kp] (Kp <= kMaxK), then scales f32 [kMaxRows], row sums int32 [kMaxRows]
static __device__ __align__(256) unsigned char g_noalloc_scratch[kScratchBytes];

constexpr int kMaxDevices = 64;
std::atomic<unsigned char *> g_scratch_addr[kMaxDevices];

}  // namespace

extern "C" int qlinear_run_device_noalloc(const qlinear_weights *weights, const void *a_dev,
                                          int a_type, void *c_dev, int c_type, long long ldc,
                                          int rows, void *stream) {
    WeightView v;
    int device = 0, round_mode = 0, num_sms = 0;
    if (!weights_for_noalloc(weights, &v, &device, &round_mode, &num_sms)) return QLINEAR_ERR_PARAM;
    if (!a_dev || !c_dev || rows < 1 || (a_type != QLINEAR_F32 && a_type != QLINEAR_F16) ||
        (c_type != QLINEAR_F32 && c_type != QLINEAR_F16 && c_type != QLINEAR_I32) || ldc < v.N)
        return QLINEAR_ERR_PARAM;
    if (rows > kMaxRows || v.Kp > kMaxK) return QLINEAR_ERR_LIMIT;
    // the GEMV's own shared-memory plan (very wide layers stage more scales per CTA than it
    // holds): refused here, before anything is launched
    if (!gemv_fits(rows, v.Kp, v.N, v.bits, false, num_sms)) return QLINEAR_ERR_LIMIT;
    if (device < 0 || device >= kMaxDevices) return QLINEAR_ERR_PARAM;

    int prev = -1;
    if (cudaGetDevice(&prev) != cudaSuccess) return QLINEAR_ERR_CUDA;
    if (prev != device && cudaSetDevice(device) != cudaSuccess) return QLINEAR_ERR_CUDA;
    int status = QLINEAR_OK;
    unsigned char *base = g_scratch_addr[device].load(std::memory_order_acquire);
    if (!base) {
        // once per device, with the device current: the array's device address
        void *addr = nullptr;
        if (cudaGetSymbolAddress(&addr, g_noalloc_scratch) != cudaSuccess || !addr)
            status = QLINEAR_ERR_CUDA;
        else {
            base = static_cast<unsigned char *>(addr);
            g_scratch_addr[device].store(base, std::memory_order_release);
        }
    }
    if (status == QLINEAR_OK) {
        int8_t *codes = reinterpret_cast<int8_t *>(base);
        float *scales = reinterpret_cast<float *>(base + kCodesBytes);
        int32_t *rowsums = reinterpret_cast<int32_t *>(base + kCodesBytes + 4 * kMaxRows);
        cudaStream_t s = static_cast<cudaStream_t>(stream);
        if (launch_act_quant(a_dev, a_type, v.K, rows, v.K, v.Kp, round_mode, codes, scales,
                             rowsums, s) != cudaSuccess)
            status = QLINEAR_ERR_CUDA;
        else {
            GemvInput in{codes, kI8Codes, v.Kp, round_mode, scales, rowsums, nullptr};
            if (launch_gemv(v, in, rows, single_output(c_dev), c_type, ldc, false, num_sms, s) != cudaSuccess)
                status = QLINEAR_ERR_CUDA;
        }
    }
    if (prev >= 0 && prev != device) cudaSetDevice(prev);
    return status;
}
