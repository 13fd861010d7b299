// gemv_impl.cuh -- decode path (rows <= 8): stream the packed weights from HBM once.
//
// The kernel and its launch templates, instantiated in two translation units: gemv.cu (one
// output buffer) and gemv_scatter.cu (the split-N exchange: every output element stored to
// this GPU's buffer and to the peers').  Two units so the two sets compile in parallel.
//
// acc[m][n] = sum_k q[m][k] * w[k][n] exactly in int32 (src/npu.rs:1111-1116), then
// y = (f32(acc) * s_a[m]) * s_w[n] (src/npu.rs:1117), written as f32 / fp16 / raw i32;
// with swiglu, out[m][j] = silu(y[m][j]) * y[m][N/2 + j] (src/npu.rs:1202-1208).
//
// Work split: CTA c (one per SM, 16 warps) owns the contiguous output rows [r0, r1) (an even
// split, or for small layers a ramp from more rows at the first CTA to fewer at the last:
// gemv_row_start); warp w owns the CTA's rows w, w + 16, ...  A task is one chunk of one row (with swiglu: the gate
// row n and its up row N/2 + n together): U 16-byte units per lane, i.e. 512*U contiguous
// bytes per segment, read with ld.global.nc.L1::no_allocate straight into registers.  A warp
// keeps D tasks in flight in a register ring (D*U*16 bytes per lane, about 192 KB per SM in
// all), issuing task t + D as soon as task t's registers are consumed, and it issues its
// first D tasks before the activation prologue, so the weight stream starts at the first
// instruction of the kernel.  There is no shared-memory staging and no barrier on the
// stream path: measured against a bulk-copy ring with producer/consumer mbarriers, this
// streams the same bytes in about two thirds of the time on B200 (the ring's hand-offs
// between warps, not HBM, limited it).
//
// Products use dp4a (s8 x s8 for W8, u8 x s8 for W4's offset-binary nibbles, corrected by
// 8*sum(q) in the epilogue); a row's MT sums are reduced across the warp once with a halving
// butterfly and its outputs written by the lanes that hold them.  The CTA's weight scales are
// staged in shared memory at the start, so the per-row epilogue touches no global memory
// but its store.
//
// Activations: either codes from the quantisation kernel (int8 [M][Kp] plus scales and row
// sums) or -- the fused decode path -- the raw fp16 / f32 rows, which the CTA quantises in
// the prologue while its first tasks are in flight (a8_row_scale / a8_code: the same
// arithmetic as act_quant.cu, so the codes are identical).
#pragma once
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <type_traits>

namespace ql {

namespace {

constexpr int kWarps = 16;
constexpr int kThreads = kWarps * 32;
constexpr int kSmemBudget = 220 * 1024;
constexpr int kMaxUnits = 16;        // units per lane per task (longer rows are split in chunks)
constexpr int kMaxUnitsSwiglu = 8;   // swiglu and paired tasks carry two rows

// Tasks of two weight rows where the activation reads from shared memory would otherwise
// bound the kernel: per weight byte and activation row, W4 reads two bytes of codes and W8
// one, and an SM reads 128 bytes of shared memory per clock.  A task of two rows (the first
// and second half of the CTA's rows) reads each activation chunk once for both.
__host__ __device__ constexpr bool gemv_paired(int bits, int mt, bool swiglu) {
    return !swiglu && (bits == 4 ? mt >= 4 : mt >= 8);
}

// Balanced mode (BAL, one or two activation rows, one output buffer): a CTA's rows are cut
// into nch chunks and each of its 16 warps takes a contiguous range of the row-major
// (row, chunk) task list, instead of whole rows (66 rows per CTA for N = 9728 left 2 warps
// streaming a fifth row while 14 waited).  A warp reduces its sums only where a row ends or
// its range ends (a row split between two warps), and adds them into shared memory (int32
// atomics: exact in any order); a pass after a CTA barrier forms the outputs.  (Dealing the
// tasks round-robin instead measured 2x slower: a warp's consecutive tasks then belong to
// different rows, and the shuffle reduction after every 512-byte task stalled it.)
// Smaller tasks, so the ring is deeper: about 20 units per lane in flight, as in the
// whole-row mode.  plan() chooses it only where whole rows are badly uneven.
__host__ __device__ constexpr int bal_depth(int units) { return 20 / units < 1 ? 1 : 20 / units; }

// Register ring depth for NSEG*U units per lane per task: about 96 data registers per thread
// with one or two activation rows, less with more (their partial sums need registers too).
__host__ __device__ constexpr int ring_depth(int units, int mt) {
    return (mt <= 2 ? 24 : mt == 4 ? 16 : 12) / units < 1 ? 1
         : (mt <= 2 ? 24 : mt == 4 ? 16 : 12) / units > 8 ? 8
         : (mt <= 2 ? 24 : mt == 4 ? 16 : 12) / units;
}

// The per-lane unit counts the kernel is built for.
__host__ __device__ constexpr int round_units(int u) {
    return u <= 1 ? 1 : u <= 2 ? 2 : u <= 3 ? 3 : u <= 4 ? 4 : u <= 5 ? 5 : u <= 6 ? 6
         : u <= 8 ? 8 : u <= 10 ? 10 : u <= 12 ? 12 : 16;
}

// Reduce V = 2^p values per lane across the warp; afterwards lane l holds the full sum of
// value index l / (32 / V) in v[0] (V - 1 + 5 - log2 V shuffles instead of 5 per value).
template <int V>
__device__ __forceinline__ void warp_reduce_spread(int (&v)[V], int lane) {
    int off = 16;
#pragma unroll
    for (int n = V; n > 1; n >>= 1) {
        const bool upper = (lane & off) != 0;
#pragma unroll
        for (int i = 0; i < n / 2; i++) {
            const int send = upper ? v[i] : v[i + n / 2];
            const int keep = upper ? v[i + n / 2] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, off);
        }
        off >>= 1;
    }
    for (; off >= 1; off >>= 1) v[0] += __shfl_xor_sync(0xffffffffu, v[0], off);
}

__device__ __forceinline__ void store_typed(void *out, int type, long long idx, float y, int raw) {
    if (type == kF16)
        static_cast<__half *>(out)[idx] = __float2half_rn(y);
    else if (type == kF32)
        static_cast<float *>(out)[idx] = y;
    else
        static_cast<int32_t *>(out)[idx] = raw;
}

// Store one output element into every destination of the set (this GPU's buffer and, for
// the split-N exchange, the peers').
__device__ __forceinline__ void store_all(const OutputSet &o, int type, long long idx, float y,
                                          int raw) {
#pragma unroll  // compile-time indices into the parameter array (no local-memory copy)
    for (int d = 0; d < kMaxOutputs; d++)
        if (d < o.count) store_typed(o.dst[d], type, idx + o.col0, y, raw);
}

// Where code k of an activation row sits in shared memory.  W8: at k (lane l reads the 16
// codes of unit j = 32 c + l at 16 j, 16-byte strides: conflict-free).  W4: a unit covers 32
// codes, read as two 16-byte halves; with a plain layout the lanes' reads would be 32 bytes
// apart (two-way bank conflicts on both reads).  So the 16-byte chunks are interleaved per
// block of 32 units: half h of unit j = 32 b + l goes to chunk 64 b + h * nb + l (nb = the
// block's unit count, 32 except in a row's last block), and a warp's read of one half is 32
// consecutive chunks.
template <int BITS>
__host__ __device__ __forceinline__ int xs_chunk(int j, int h, int upr) {
    if constexpr (BITS == 8) {
        return j;
    } else {
        const int b = j >> 5;
        const int nb = min(32, upr - 32 * b);
        return 64 * b + h * nb + (j & 31);
    }
}
template <int BITS>
__host__ __device__ __forceinline__ int xs_byte(int k, int upr) {
    if constexpr (BITS == 8)
        return k;
    else
        return xs_chunk<BITS>(k >> 5, (k >> 4) & 1, upr) * 16 + (k & 15);
}

struct GemvArgs {
    const uint8_t *wq;
    const float *wscale;
    int N, Kp, K;
    int skew_q10;      // 0: rows_per_cta rows per CTA; else the ramp gemv_row_start draws
    const void *xin;
    int in_type;
    long long ldx;
    int round_mode;
    const float *ascale;
    const int32_t *rowsum;
    int M;
    void *out;  // the output when one buffer takes it; several: the kernel's OutputSet
    int out_type;
    long long ldc;
    int rows_per_cta;  // output rows (channels, or gate rows with swiglu) per CTA (the most)
    int nch;           // chunks per row
    unsigned *err;
};
// 128 bytes: one more field past that (the skew once sat there) measured the W4 layer at
// eight rows 52.3 -> 57.5 us per call, so new fields go into the padding above
static_assert(sizeof(GemvArgs) == 128, "GemvArgs grew past 128 bytes");

// Skewed row split (single-output kernel, one or two activation rows): CTA j of G owns rows
// [R(j), R(j+1)) with R(j) = n ((1 + s) j G - s j^2) / G^2, s = q / 1024 -- a linear ramp from
// (1 + s) n / G rows at the first CTA to (1 - s) n / G at the last.  Why: with the early
// dependent launch, call i+1's CTAs take the SMs in blockIdx order as call i's CTAs exit, so
// its last CTAs land when call i completes and, with an even split, then stream a whole
// share; the ramp gives the early CTAs (which stream while call i drains) more rows and the
// late ones fewer.  Sized in bytes, not as a fraction: about 68 KB above and below the mean
// share, so large layers (the lm_head: 2.6 MB per CTA) stay nearly even (a fixed 20-40% ramp
// slowed the lm_head and the 117 MB W4 layer by 13-28%).  Measured on B200, same box,
// alternating runs: cfg2's block at M=1 21.9 -> 19.6 us, the 36-layer decode pass 1157 ->
// 1100 us per token (1118 -> 1072 us replayed as a CUDA graph), cfg1 W8 M=1 7.9 -> 7.8 us,
// cfg4 W4 M=1 27.9 -> 27.6 us, the lm_head unchanged.
__host__ __device__ inline int gemv_row_start(long long j, long long G, long long n, int q) {
    return (int)(n * ((1024 + q) * j * G - q * j * j) / (1024 * G * G));
}

// Quantise the call's rows into xs (codes [MT][Kp], zero beyond M and K) and set s_scale /
// s_rowsum.  TIn: __half or float; K and ldx are multiples of 16 / sizeof(TIn) and the rows
// 16-byte aligned (gemv_can_fuse).
template <int BITS, int MT, typename TIn>
__device__ __forceinline__ void quantise_rows(const GemvArgs &p, uint8_t *xs, float *s_scale,
                                              int *s_rowsum, float (*s_red)[MT],
                                              int (*s_redi)[MT]) {
    constexpr int VEC = 16 / sizeof(TIn);
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int upr = (BITS == 8 ? p.Kp : p.Kp / 2) / 16;  // 16-byte weight units per row
    const TIn *x = static_cast<const TIn *>(p.xin);
    const int nvec = p.K / VEC;
    auto widen = [](const uint4 &raw, float (&f)[VEC]) {
        if constexpr (VEC == 8) {
            const __half2 *h = reinterpret_cast<const __half2 *>(&raw);
#pragma unroll
            for (int i = 0; i < 4; i++) {
                const float2 t = __half22float2(h[i]);
                f[2 * i] = t.x;
                f[2 * i + 1] = t.y;
            }
        } else {
            f[0] = __uint_as_float(raw.x); f[1] = __uint_as_float(raw.y);
            f[2] = __uint_as_float(raw.z); f[3] = __uint_as_float(raw.w);
        }
    };
    // pass 1: per-row max |x| (fmaxf ignores NaN, like Rust's f32::max)
    float am[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) am[m] = 0.0f;
    for (int v = tid; v < nvec; v += kThreads) {
#pragma unroll
        for (int m = 0; m < MT; m++) {
            if (m < p.M) {
                float f[VEC];
                widen(__ldg(reinterpret_cast<const uint4 *>(x + (long long)m * p.ldx) + v), f);
#pragma unroll
                for (int e = 0; e < VEC; e++) am[m] = fmaxf(am[m], fabsf(f[e]));
            }
        }
    }
#pragma unroll
    for (int m = 0; m < MT; m++) {
#pragma unroll
        for (int o = 16; o; o >>= 1) am[m] = fmaxf(am[m], __shfl_xor_sync(0xffffffffu, am[m], o));
        if (lane == 0) s_red[warp][m] = am[m];
    }
    __syncthreads();
    __shared__ float s_inv[MT];
    if (tid < MT) {
        float a = 0.0f;
        for (int w = 0; w < kWarps; w++) a = fmaxf(a, s_red[w][tid]);
        float sc, inv;
        a8_row_scale(a, sc, inv);
        s_scale[tid] = sc;
        s_inv[tid] = inv;
    }
    __syncthreads();
    float inv[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) inv[m] = s_inv[m];
    // pass 2: codes (rows >= M and the K padding are zero)
    int sum[MT];
#pragma unroll
    for (int m = 0; m < MT; m++) sum[m] = 0;
    for (int v = tid; v < nvec; v += kThreads) {
#pragma unroll
        for (int m = 0; m < MT; m++) {
            uint32_t w[VEC / 4];
#pragma unroll
            for (int g = 0; g < VEC / 4; g++) w[g] = 0;
            if (m < p.M) {
                float f[VEC];
                widen(__ldg(reinterpret_cast<const uint4 *>(x + (long long)m * p.ldx) + v), f);
#pragma unroll
                for (int g = 0; g < VEC / 4; g++) {
#pragma unroll
                    for (int e = 0; e < 4; e++) {
                        const int q = a8_code(f[4 * g + e], inv[m], p.round_mode);
                        sum[m] += q;
                        w[g] |= (uint32_t)(q & 0xff) << (8 * e);
                    }
                }
            }
            // VEC codes at k = v * VEC stay inside one 16-byte chunk of the layout
            const int at = m * p.Kp + xs_byte<BITS>(v * VEC, upr);
            if constexpr (VEC == 8)
                *reinterpret_cast<uint2 *>(xs + at) = make_uint2(w[0], w[1]);
            else
                *reinterpret_cast<uint32_t *>(xs + at) = w[0];
        }
    }
    for (int i = p.K + tid; i < p.Kp; i += kThreads) {
#pragma unroll
        for (int m = 0; m < MT; m++) xs[m * p.Kp + xs_byte<BITS>(i, upr)] = 0;
    }
#pragma unroll
    for (int m = 0; m < MT; m++) {
#pragma unroll
        for (int o = 16; o; o >>= 1) sum[m] += __shfl_xor_sync(0xffffffffu, sum[m], o);
        if (lane == 0) s_redi[warp][m] = sum[m];
    }
    __syncthreads();
    if (tid < MT) {
        int t = 0;
        for (int w = 0; w < kWarps; w++) t += s_redi[w][tid];
        s_rowsum[tid] = t;
    }
}

// The scatter kernel's destinations; the single-output kernel takes an empty parameter in
// their place and stores to p.out alone.  (Measured on B200: a run-time choice between the
// two in one kernel cost the M=1 decode call 0.4 us of its 9 us.)
struct NoOutputs {};
template <bool SCATTER> struct OutsParam { using type = NoOutputs; };
template <> struct OutsParam<true> { using type = OutputSet; };

// The GEMV of one call, run by every CTA of the grid.  BITS: 4/8.  MT: activation rows held
// (>= M).  U: 16-byte units per lane per task segment.  SCATTER: store every output element
// to each of outs' destinations.  smem: this call's dynamic shared memory (codes [MT][Kp],
// then the weight scales).  wait(): called by every thread after the first weight loads are
// issued and before the activations are read; returns false to abandon the call (the
// loads in flight are plain loads into registers and need no draining).
template <int BITS, int MT, bool SWIGLU, int U, bool SCATTER, bool BAL, typename Wait>
__device__ __forceinline__ void gemv_body(const GemvArgs &p,
                                          const typename OutsParam<SCATTER>::type &outs,
                                          uint8_t *smem, Wait &&wait) {
    constexpr bool PAIR = gemv_paired(BITS, MT, SWIGLU);
    constexpr int NSEG = SWIGLU || PAIR ? 2 : 1;
    constexpr int D = BAL ? bal_depth(NSEG * U) : ring_depth(NSEG * U, MT);
    constexpr int V = MT;  // sums a warp reduces per row and segment
    __shared__ float s_scale[MT];
    __shared__ int s_rowsum[MT];
    __shared__ float s_red[kWarps][MT];
    __shared__ int s_redi[kWarps][MT];

    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int row_bytes = BITS == 8 ? p.Kp : p.Kp / 2;
    const int upr = row_bytes / 16;  // 16-byte units per row
    const int nrows_out = SWIGLU ? p.N / 2 : p.N;
    // plan() skews only at one or two rows; the clamp never bites (rows_per_cta is sized
    // for the ramp)
    constexpr bool SKEW = MT <= 2;
    const bool skew = SKEW && p.skew_q10 != 0;
    const int r0 = skew ? gemv_row_start(blockIdx.x, gridDim.x, nrows_out, p.skew_q10)
                        : blockIdx.x * p.rows_per_cta;
    const int nr = skew ? min(gemv_row_start(blockIdx.x + 1, gridDim.x, nrows_out, p.skew_q10) - r0,
                              p.rows_per_cta)
                        : max(0, min(nrows_out, r0 + p.rows_per_cta) - r0);
    // PAIR: the CTA's rows in two halves, [0, h1) and [h1, nr); a task covers local row lr
    // of both (the second half may be one row shorter)
    const int h1 = PAIR ? (nr + 1) / 2 : nr;
    const int my_rows = h1 > warp ? (h1 - warp + kWarps - 1) / kWarps : 0;
    // Task t of this warp: whole-row mode, local row warp + (t / nch) * kWarps and chunk
    // t % nch; balanced mode, CTA task T = tb + t = row * nch + chunk, [tb, te) this warp's
    // share of the h1 * nch tasks.
    const int tb = BAL ? (int)((long long)warp * h1 * p.nch / kWarps) : 0;
    const int te = BAL ? (int)((long long)(warp + 1) * h1 * p.nch / kWarps) : 0;
    const int ntask = BAL ? te - tb : my_rows * p.nch;
    auto task_of = [&](int t, int &lr, int &c) {
        if constexpr (BAL) {
            const int T = tb + t;
            lr = T / p.nch;
            c = T - lr * p.nch;
        } else {
            const int i = t / p.nch;
            c = t - i * p.nch;
            lr = warp + i * kWarps;
        }
    };
    const uint8_t *seg0 = p.wq + (long long)r0 * row_bytes;  // gate / only / first-half rows
    const uint8_t *seg1 = p.wq + (PAIR ? (long long)(r0 + h1)        // second-half rows
                                       : (long long)p.N / 2 + r0)    // up rows (swiglu)
                                     * row_bytes;

    uint8_t *xs = smem;                                         // [MT][Kp] codes
    float *ws = reinterpret_cast<float *>(xs + (size_t)MT * p.Kp);  // [NSEG][rows_per_cta]
    // balanced mode: the rows' sums [NSEG][rows_per_cta][MT]
    int *s_acc = reinterpret_cast<int *>(ws + (SWIGLU ? 2 : 1) * p.rows_per_cta);

    uint4 ring[D][NSEG * U];
    auto issue = [&](int t, uint4 (&dst)[NSEG * U]) {
        int lr, c;
        task_of(t, lr, c);
        const long long off = (long long)lr * row_bytes;
        const int j0 = c * 32 * U + lane;
#pragma unroll
        for (int s = 0; s < NSEG; s++) {
            const uint8_t *row = (s == 0 ? seg0 : seg1) + off;
            const bool live = !PAIR || s == 0 || h1 + lr < nr;
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int j = j0 + u * 32;
                dst[s * U + u] = live && j < upr ? ldg_stream(row + j * 16) : make_uint4(0, 0, 0, 0);
            }
        }
    };
#pragma unroll
    for (int d = 0; d < D; d++)
        if (d < ntask) issue(d, ring[d]);

    // Scales of the CTA's rows (plain loads, consumed after the prologue's barriers).
    for (int i = tid; i < nr; i += kThreads) {
        ws[i] = p.wscale[r0 + i];
        if (SWIGLU) ws[p.rows_per_cta + i] = p.wscale[p.N / 2 + r0 + i];
    }

    if constexpr (BAL) {  // zeroed before the prologue's barriers
        for (int i = tid; i < NSEG * p.rows_per_cta * MT; i += kThreads) s_acc[i] = 0;
    }

    // ---------------------------------------------------------------- activation codes
    if (!wait()) return;
    if (p.in_type == kF16) {
        quantise_rows<BITS, MT, __half>(p, xs, s_scale, s_rowsum, s_red, s_redi);
    } else if (p.in_type == kF32) {
        quantise_rows<BITS, MT, float>(p, xs, s_scale, s_rowsum, s_red, s_redi);
    } else {
        const int8_t *codes = static_cast<const int8_t *>(p.xin);
        const int n16 = MT * p.Kp / 16;
        const int row16 = p.Kp / 16;  // 16-byte chunks per row
        for (int i = tid; i < n16; i += kThreads) {
            const int m = i / row16, c = i - m * row16;  // chunk c holds codes 16c .. 16c+15
            uint4 v = make_uint4(0, 0, 0, 0);
            if (m < p.M) v = *reinterpret_cast<const uint4 *>(codes + (long long)i * 16);
            *reinterpret_cast<uint4 *>(xs + m * p.Kp + 16 * xs_chunk<BITS>(c >> (BITS == 8 ? 0 : 1),
                                                                          c & 1, upr)) = v;
        }
        if (tid < MT) {
            s_scale[tid] = tid < p.M ? p.ascale[tid] : 0.0f;
            s_rowsum[tid] = tid < p.M ? p.rowsum[tid] : 0;
        }
    }
    __syncthreads();

    // Row lr's outputs for activation row m from its int32 totals (W4: minus 8 * sum(q)).
    auto emit_row = [&](int (&tot)[NSEG], int m, int lr) {
        if (BITS == 4) {
#pragma unroll
            for (int s = 0; s < NSEG; s++) tot[s] -= 8 * s_rowsum[m];
        }
        const int n = r0 + lr;
        const float sa = s_scale[m];
        if constexpr (SWIGLU) {
            const float g = __fmul_rn(__fmul_rn(__int2float_rn(tot[0]), sa), ws[lr]);
            const float up = __fmul_rn(__fmul_rn(__int2float_rn(tot[NSEG - 1]), sa),
                                       ws[p.rows_per_cta + lr]);
            const float y = __fmul_rn(__fdiv_rn(g, __fadd_rn(1.0f, expf(-g))), up);
            if constexpr (SCATTER)
                store_all(outs, p.out_type, (long long)m * p.ldc + n, y, 0);
            else
                store_typed(p.out, p.out_type, (long long)m * p.ldc + n, y, 0);
        } else {
#pragma unroll
            for (int s = 0; s < NSEG; s++) {
                const int l = s * h1 + lr;  // the CTA-local row of segment s
                if (s > 0 && l >= nr) break;
                const float y = __fmul_rn(__fmul_rn(__int2float_rn(tot[s]), sa), ws[l]);
                if constexpr (SCATTER)
                    store_all(outs, p.out_type, (long long)m * p.ldc + n + s * h1, y, tot[s]);
                else
                    store_typed(p.out, p.out_type, (long long)m * p.ldc + n + s * h1, y, tot[s]);
            }
        }
    };

    // ---------------------------------------------------------------- stream the weights
    int acc[NSEG][V];
#pragma unroll
    for (int s = 0; s < NSEG; s++)
#pragma unroll
        for (int m = 0; m < V; m++) acc[s][m] = 0;
    for (int t0 = 0; t0 < ntask; t0 += D) {
#pragma unroll
        for (int d = 0; d < D; d++) {
            const int t = t0 + d;
            if (t >= ntask) break;
            int lr, c;
            task_of(t, lr, c);
            const int j0 = c * 32 * U + lane;
#pragma unroll
            for (int u = 0; u < U; u++) {
                const int j = j0 + u * 32;
                if (j < upr) {
#pragma unroll
                    for (int s = 0; s < NSEG; s++) {
                        const uint4 wv = ring[d][s * U + u];
                        if constexpr (BITS == 8) {
#pragma unroll
                            for (int m = 0; m < MT; m++) {
                                const uint4 xv = *reinterpret_cast<const uint4 *>(xs + m * p.Kp + j * 16);
                                int a = dp4a_ss(wv.x, xv.x, acc[s][m]);
                                a = dp4a_ss(wv.y, xv.y, a);
                                a = dp4a_ss(wv.z, xv.z, a);
                                acc[s][m] = dp4a_ss(wv.w, xv.w, a);
                            }
                        } else {
                            // 16 packed bytes = 32 codes k = 32j .. 32j+31; word q covers 8
                            // codes: low nibbles k 8q..8q+3, high nibbles k 8q+4..8q+7.
                            const uint32_t w4[4] = {wv.x, wv.y, wv.z, wv.w};
                            const int ca = 16 * xs_chunk<4>(j, 0, upr);
                            const int cb = 16 * xs_chunk<4>(j, 1, upr);
#pragma unroll
                            for (int m = 0; m < MT; m++) {
                                const uint4 xa = *reinterpret_cast<const uint4 *>(xs + m * p.Kp + ca);
                                const uint4 xb = *reinterpret_cast<const uint4 *>(xs + m * p.Kp + cb);
                                const uint32_t x8[8] = {xa.x, xa.y, xa.z, xa.w,
                                                        xb.x, xb.y, xb.z, xb.w};
                                int a = acc[s][m];
#pragma unroll
                                for (int q = 0; q < 4; q++) {
                                    a = dp4a_us(w4[q] & 0x0F0F0F0Fu, x8[2 * q], a);
                                    a = dp4a_us((w4[q] >> 4) & 0x0F0F0F0Fu, x8[2 * q + 1], a);
                                }
                                acc[s][m] = a;
                            }
                        }
                    }
                }
            }
            if (t + D < ntask) issue(t + D, ring[d]);  // refill the slot just consumed
            // the row has more chunks (balanced mode: in this warp's range)
            if (c != p.nch - 1 && (!BAL || t != ntask - 1)) continue;

            // ---------------------------------------------------------- row epilogue
            int tot[NSEG];
#pragma unroll
            for (int s = 0; s < NSEG; s++) {
                warp_reduce_spread<V>(acc[s], lane);
                tot[s] = acc[s][0];
#pragma unroll
                for (int m = 0; m < V; m++) acc[s][m] = 0;
            }
            const int m = lane / (32 / V);  // activation row whose totals this lane holds
            if ((lane % (32 / V)) == 0 && m < p.M) {
                if constexpr (BAL) {
#pragma unroll
                    for (int s = 0; s < NSEG; s++)
                        atomicAdd(&s_acc[(s * p.rows_per_cta + lr) * MT + m], tot[s]);
                } else {
                    emit_row(tot, m, lr);
                }
            }
        }
    }
    if constexpr (BAL) {  // every task's sums are in s_acc: form the outputs
        __syncthreads();
        for (int e = tid; e < h1 * MT; e += kThreads) {
            const int lr = e / MT, m = e - lr * MT;
            if (m >= p.M) continue;
            int tot[NSEG];
#pragma unroll
            for (int s = 0; s < NSEG; s++) tot[s] = s_acc[(s * p.rows_per_cta + lr) * MT + m];
            emit_row(tot, m, lr);
        }
    }
    // peers' copies of the output: visible system-wide before the next work on this stream
    if constexpr (SCATTER) __threadfence_system();
}

template <int BITS, int MT, bool SWIGLU, int U, bool SCATTER, bool BAL>
__global__ void __launch_bounds__(kThreads, 1)
    gemv_kernel(const GemvArgs p, const typename OutsParam<SCATTER>::type outs) {
    extern __shared__ __align__(16) uint8_t smem[];
    // Let the next call on the stream launch now: its CTAs take the SMs this grid frees one
    // by one and stream their own weights while this grid drains.  Safe for any dependent
    // this library launches with programmatic serialization (the GEMV and the GEMM): before
    // their griddepcontrol.wait they only read their own weights and weight scales, which
    // nothing writes while calls run, and they read activations and store outputs only
    // after it (this grid complete, its stores visible).  Every other kernel is launched
    // without programmatic serialization and starts after this grid completes.  The
    // exchange kernels keep the implicit trigger at exit.
    if constexpr (!SCATTER) asm volatile("griddepcontrol.launch_dependents;");
    gemv_body<BITS, MT, SWIGLU, U, SCATTER, BAL>(p, outs, smem, [] {
        asm volatile("griddepcontrol.wait;" ::: "memory");
        return true;
    });
}

inline int mt_of(int rows) { return rows <= 1 ? 1 : rows <= 2 ? 2 : rows <= 4 ? 4 : 8; }

struct Plan {
    int rows_per_cta, grid, nch, units;
    size_t smem;
    bool bal;  // balanced (row, chunk) tasks; units then 1, 2 or 4
    int skew_q10;  // skewed row split (gemv_row_start), 0: even
};

// The ramp of the skewed row split for a layer of `nrows` rows of `row_bytes` (x2 with
// SwiGLU: gate and up rows) over `grid` CTAs at `mt` activation rows: q / 1024 = about 68 KB
// over the mean bytes per CTA, at most 0.4, none below 1/64 or at four or more rows (there
// the dot products take longer per byte and the ramp measured no gain: cfg1 at M=4 10.3 ->
// 10.4 us with a 20% ramp, the W4 layer at M=8 slower).
inline int gemv_skew_q10(long long nrows, long long row_bytes, int nseg, int grid, int mt) {
    if (mt > 2 || grid < 2) return 0;
    const long long ramp = 68 * 1024;
    const long long cta_bytes = nrows * row_bytes * nseg / grid;
    if (cta_bytes <= 0) return 0;
    const long long q = std::min<long long>(410, ramp * 1024 / cta_bytes);
    return q >= 16 ? (int)q : 0;
}

// Rows per CTA (one CTA per SM), chunks per row and units per lane, shared memory.
// allow_bal: the caller launches the single-output kernel (the balanced mode is built only
// for that, at one or two activation rows).
inline bool plan(int rows, int Kp, int N, int bits, bool swiglu, int num_sms, Plan *pl,
                 bool allow_bal = false) {
    if (rows < 1 || rows > 8 || num_sms < 1) return false;
    const int nrows = swiglu ? N / 2 : N;
    if (nrows < 1) return false;
    const int per = (nrows + num_sms - 1) / num_sms;
    const int upr = (bits == 8 ? Kp : Kp / 2) / 16;
    const int lane_units = (upr + 31) / 32;
    const int maxu = swiglu || gemv_paired(bits, mt_of(rows), swiglu) ? kMaxUnitsSwiglu : kMaxUnits;
    const int nch = (lane_units + maxu - 1) / maxu;
    const size_t smem = (size_t)mt_of(rows) * Kp + (size_t)(swiglu ? 2 : 1) * per * 4;
    if (smem > (size_t)kSmemBudget) return false;
    pl->rows_per_cta = per;
    pl->grid = (nrows + per - 1) / per;
    pl->nch = nch;
    pl->units = round_units((lane_units + nch - 1) / nch);
    pl->smem = smem;
    pl->bal = false;
    pl->skew_q10 = 0;
    const int row_bytes = bits == 8 ? Kp : Kp / 2;
    if (allow_bal) {
        // the skewed split where it fits the shared-memory budget (else the even one, so a
        // request that fits the even split never fails here)
        const int g = std::min(num_sms, nrows);
        const int q = gemv_skew_q10(nrows, row_bytes, swiglu ? 2 : 1, g, mt_of(rows));
        if (q) {
            const int pmax = (int)(((long long)nrows * (1024 + q) + 1024LL * g - 1) / (1024LL * g)) + 2;
            const size_t smem_s = (size_t)mt_of(rows) * Kp + (size_t)(swiglu ? 2 : 1) * pmax * 4;
            if (smem_s <= (size_t)kSmemBudget) {
                pl->rows_per_cta = pmax;
                pl->grid = g;
                pl->smem = smem_s;
                pl->skew_q10 = q;
            }
        }
    }
    if (allow_bal && mt_of(rows) <= 2) {
        const int per = pl->rows_per_cta;  // the busiest CTA's rows
        const size_t smem = pl->smem;
        // time ~ the busiest warp's units per lane: whole rows, ceil(per / 16) rows of nch
        // chunks of `units`; balanced, ceil(per * nchb / 16) tasks of u units
        const long long whole = (long long)((per + kWarps - 1) / kWarps) * nch * pl->units;
        long long best = whole;
        int bu = 0;
        for (int u : {4, 2, 1}) {
            const int nchb = (lane_units + u - 1) / u;
            const long long cost = (long long)(((long long)per * nchb + kWarps - 1) / kWarps) * u;
            if (cost < best) { best = cost; bu = u; }
        }
        // Only where whole rows leave the warps badly uneven (a busiest warp with >= 1.4x
        // the units of the balanced split: the 2560-wide projections' 18 rows per CTA).
        // Measured on B200, the balanced mode's small tasks cost more issue slots per byte:
        // cfg1 (66 rows per CTA, predicted 25 -> 21) ran 9.1 -> 10.9 us per call, cfg4 W4
        // M=1 (194 rows, 104 -> 97) 30.1 -> 58.5 us.
        if (bu && 10 * best * 14 <= 100 * whole) {
            const int nseg = swiglu ? 2 : 1;
            const size_t smem_b = smem + (size_t)nseg * per * mt_of(rows) * 4;
            if (smem_b <= (size_t)kSmemBudget) {
                pl->bal = true;
                pl->units = bu;
                pl->nch = (lane_units + bu - 1) / bu;
                pl->smem = smem_b;
            }
        }
    }
    return true;
}

template <int BITS, int MT, bool SWIGLU, int U, bool SCATTER, bool BAL = false>
cudaError_t launch_t(const WeightView &w, const GemvInput &in, int rows, const OutputSet &out, int out_type,
                     long long ldc, const Plan &pl, cudaStream_t stream) {
    GemvArgs a{};
    a.wq = w.w;
    a.wscale = w.scales;
    a.N = w.N;
    a.Kp = w.Kp;
    a.K = w.K;
    a.xin = in.x;
    a.in_type = in.type;
    a.ldx = in.ldx;
    a.round_mode = in.round_mode;
    a.ascale = in.ascale;
    a.rowsum = in.rowsum;
    a.M = rows;
    // one destination: offset by the column offset here; scatter: the kernel adds it
    a.out = SCATTER ? nullptr
                    : static_cast<char *>(out.dst[0]) + out.col0 * (out_type == kF16 ? 2 : 4);
    a.out_type = out_type;
    a.ldc = ldc;
    a.rows_per_cta = pl.rows_per_cta;
    a.nch = pl.nch;
    a.skew_q10 = pl.skew_q10;
    a.err = in.err;
    auto kern = gemv_kernel<BITS, MT, SWIGLU, U, SCATTER, BAL>;
    static int configured[64] = {0};  // per device: raise the opt-in limit once
    int dev = 0;
    cudaGetDevice(&dev);
    if (dev < 0 || dev >= 64) return cudaErrorInvalidDevice;
    if (!configured[dev]) {
        cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                             kSmemBudget);
        if (e != cudaSuccess) return e;
        configured[dev] = 1;
    }
    cudaLaunchConfig_t cfg{};
    cfg.gridDim = dim3(pl.grid);
    cfg.blockDim = dim3(kThreads);
    cfg.dynamicSmemBytes = pl.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    if constexpr (SCATTER)
        return cudaLaunchKernelEx(&cfg, kern, a, out);
    else
        return cudaLaunchKernelEx(&cfg, kern, a, NoOutputs{});
}

template <int BITS, int MT, bool SWIGLU, bool SCATTER>
cudaError_t launch_u(const WeightView &w, const GemvInput &in, int rows, const OutputSet &out, int out_type,
                     long long ldc, const Plan &pl, cudaStream_t stream) {
#define QL_GEMV_U(u)                                                                      \
    case u:                                                                               \
        if constexpr (!(SWIGLU || gemv_paired(BITS, MT, SWIGLU)) || u <= kMaxUnitsSwiglu) \
            return launch_t<BITS, MT, SWIGLU, u, SCATTER>(w, in, rows, out, out_type, ldc, pl, \
                                                             stream);                    \
        return cudaErrorInvalidValue;
    if constexpr (MT <= 2 && !SCATTER) {
        if (pl.bal) {
            switch (pl.units) {
            case 1: return launch_t<BITS, MT, SWIGLU, 1, false, true>(w, in, rows, out, out_type, ldc, pl, stream);
            case 2: return launch_t<BITS, MT, SWIGLU, 2, false, true>(w, in, rows, out, out_type, ldc, pl, stream);
            case 4: return launch_t<BITS, MT, SWIGLU, 4, false, true>(w, in, rows, out, out_type, ldc, pl, stream);
            default: return cudaErrorInvalidValue;
            }
        }
    }
    if (pl.bal) return cudaErrorInvalidValue;
    switch (pl.units) {
        QL_GEMV_U(1) QL_GEMV_U(2) QL_GEMV_U(3) QL_GEMV_U(4) QL_GEMV_U(5)
        QL_GEMV_U(6) QL_GEMV_U(8) QL_GEMV_U(10) QL_GEMV_U(12) QL_GEMV_U(16)
    default: return cudaErrorInvalidValue;
    }
#undef QL_GEMV_U
}

template <int BITS, bool SWIGLU, bool SCATTER>
cudaError_t launch_mt(const WeightView &w, const GemvInput &in, int rows, const OutputSet &out, int out_type,
                      long long ldc, const Plan &pl, cudaStream_t stream) {
    switch (mt_of(rows)) {
    case 1: return launch_u<BITS, 1, SWIGLU, SCATTER>(w, in, rows, out, out_type, ldc, pl, stream);
    case 2: return launch_u<BITS, 2, SWIGLU, SCATTER>(w, in, rows, out, out_type, ldc, pl, stream);
    case 4: return launch_u<BITS, 4, SWIGLU, SCATTER>(w, in, rows, out, out_type, ldc, pl, stream);
    default: return launch_u<BITS, 8, SWIGLU, SCATTER>(w, in, rows, out, out_type, ldc, pl, stream);
    }
}

// Checks the request and launches the kernel built for it.
template <bool SCATTER>
cudaError_t launch_checked(const WeightView &w, const GemvInput &in, int rows, const OutputSet &out,
                           int out_type, long long ldc, bool swiglu, int num_sms,
                           cudaStream_t stream) {
    Plan pl;
    if (!plan(rows, w.Kp, w.N, w.bits, swiglu, num_sms, &pl, !SCATTER)) return cudaErrorInvalidValue;
    if (in.type != kI8Codes && !gemv_can_fuse(in.x, in.type, in.ldx, w.K)) return cudaErrorInvalidValue;
    if (out_type != kF16 && out_type != kF32 && (out_type != kI32 || swiglu))
        return cudaErrorInvalidValue;
    if (out.count < 1 || out.count > kMaxOutputs) return cudaErrorInvalidValue;
    if (w.bits == 8)
        return swiglu ? launch_mt<8, true, SCATTER>(w, in, rows, out, out_type, ldc, pl, stream)
                      : launch_mt<8, false, SCATTER>(w, in, rows, out, out_type, ldc, pl, stream);
    return swiglu ? launch_mt<4, true, SCATTER>(w, in, rows, out, out_type, ldc, pl, stream)
                  : launch_mt<4, false, SCATTER>(w, in, rows, out, out_type, ldc, pl, stream);
}

}  // namespace

}  // namespace ql
