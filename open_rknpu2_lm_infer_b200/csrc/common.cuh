// common.cuh -- device helpers shared by the quantized-linear kernels (sm_100a only).
//
// Inline PTX for mbarriers, TMA tensor loads (every one into this CTA's own shared memory),
// the 5th-generation tensor core (tcgen05.*) and bounded waits.  Every wait in these
// kernels gives up after QL_WAIT_NS nanoseconds of %globaltimer, records
// QL_DEVERR_TIMEOUT in the backend's device error word and lets the kernel unwind, so a
// logic error shows up as QLINEAR_ERR_TIMEOUT on the host instead of a hung GPU.
#pragma once

#include <cuda.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#if defined(__CUDA_ARCH__) && (__CUDA_ARCH__ < 1000)
#error "this library targets sm_100a only"
#endif

namespace ql {

// Device error word bits (the backend's error word is an unsigned int in device memory).
constexpr unsigned QL_DEVERR_TIMEOUT = 1u;   // a bounded wait gave up
constexpr unsigned QL_DEVERR_BOUNDS = 2u;    // a checked index fell outside its buffer

constexpr unsigned long long QL_WAIT_NS = 2000000000ull;  // 2 s per wait

// GEMM geometry shared by the weight packer and the kernels.
constexpr int KBLK = 128;       // k-block: one 128-byte swizzle atom of int8 codes
constexpr int CH_TILE = 128;    // weight channels per MMA (the MMA's M)
constexpr int GEMM_KB = 128;    // k-block depth of the tensor-core GEMM's TMA tiles

__host__ __device__ inline long long round_up(long long v, long long m) { return (v + m - 1) / m * m; }

__device__ __forceinline__ unsigned long long global_ns() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_u32(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ------------------------------------------------------------------ mbarrier
__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count));
}
__device__ __forceinline__ void mbar_fence_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)),
                 "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity), "r"(1000000u)
        : "memory");
    return ok != 0;
}

// Bounded wait for the phase with the given parity to complete.  Returns false (after
// recording the timeout in *err and in the CTA-wide abort flag) if it gave up, or if
// another role of the CTA already gave up.
__device__ __forceinline__ bool mbar_wait(uint64_t *bar, uint32_t parity, unsigned *err,
                                          volatile int *abort_flag,
                                          unsigned long long limit_ns = QL_WAIT_NS) {
    if (mbar_try_wait(bar, parity)) return true;
    unsigned long long t0 = global_ns();
    while (true) {
        if (mbar_try_wait(bar, parity)) return true;
        if (*abort_flag) return false;
        if (global_ns() - t0 > limit_ns) {
            *abort_flag = 1;
            if (err) atomicOr(err, QL_DEVERR_TIMEOUT);
            return false;
        }
    }
}

// ------------------------------------------------------------------ TMA
__device__ __forceinline__ void tma_prefetch_desc(const CUtensorMap *map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}
// 2-D tiled load into this CTA's shared memory; completion is signalled on `bar` as
// transaction bytes.  No multicast.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, uint64_t *bar,
                                            int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(x), "r"(y)
        : "memory");
}
// Untiled bulk copy global -> this CTA's shared memory, completion counted on `bar`
// (both addresses 16-byte aligned, size a multiple of 16).  No multicast.
__device__ __forceinline__ void bulk_load(void *dst, const void *src, uint32_t bytes,
                                          uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::
            "r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(src)), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// Generic-proxy shared-memory writes -> visible to the async proxy (tensor core, TMA).
__device__ __forceinline__ void fence_proxy_async_smem() {
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// ------------------------------------------------------------------ tcgen05
__device__ __forceinline__ void tmem_alloc(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tc_fence_before() {
    asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}
__device__ __forceinline__ void tc_fence_after() {
    asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}
// D[tmem] (+)= A[smem desc] * B[smem desc]^T, int8 x int8 -> int32.
__device__ __forceinline__ void mma_i8_ss(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                          uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive on `bar` once every tcgen05.mma issued so far by this thread has completed.
__device__ __forceinline__ void mma_commit(uint64_t *bar) {
    asm volatile(
        "tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
            smem_u32(bar))
        : "memory");
}
// 32 lanes x 32 bit, 16 consecutive columns per thread.
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, uint32_t (&r)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 "
        "{%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]),
          "=r"(r[7]), "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]),
          "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr)
        : "memory");
}
__device__ __forceinline__ void tmem_ld_wait() {
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}
// 32 lanes x 32 bit, 32 consecutive columns per thread (the warp's own lane quadrant).
__device__ __forceinline__ void tmem_st32(uint32_t taddr, const uint32_t (&r)[32]) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], "
        "{%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,"
        "%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]),
        "r"(r[8]), "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]),
        "r"(r[15]), "r"(r[16]), "r"(r[17]), "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]),
        "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]), "r"(r[27]), "r"(r[28]),
        "r"(r[29]), "r"(r[30]), "r"(r[31])
        : "memory");
}
// Wait until this thread's tcgen05.st writes have completed.
__device__ __forceinline__ void tmem_st_wait() {
    asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
}


// ------------------------------------------------------------------ clusters (CTA pairs)
__device__ __forceinline__ uint32_t cluster_ctarank() {
    uint32_t r;
    asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
    return r;
}
// shared::cluster address of the same shared-memory offset in CTA `rank` of the cluster.
__device__ __forceinline__ uint32_t map_to_rank(const void *p, uint32_t rank) {
    uint32_t out;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(out) : "r"(smem_u32(p)), "r"(rank));
    return out;
}
__device__ __forceinline__ void cluster_sync() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// Arrive on an mbarrier of another CTA of the cluster (release at cluster scope).
__device__ __forceinline__ void mbar_arrive_remote(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr)
                 : "memory");
}
// Arrive on a peer CTA's mbarrier to announce tensor-memory work (tcgen05.st or tcgen05.ld)
// that the arriving thread has waited for (tcgen05.wait) and fenced
// (tcgen05.fence::before_thread_sync): release at CTA scope, the default of the instruction.
// The cluster-scope release above also orders the thread's generic memory accesses for the
// peer, which this hand-off does not need; measured on B200 it held the packed-W4 GEMM (whose
// converter warps hand every stage to the pair's MMA thread this way) at 0.66 POPS against
// 1.1 POPS with this form (cfg4, M=512).
__device__ __forceinline__ void mbar_arrive_remote_tc(uint32_t cluster_addr) {
    asm volatile("mbarrier.arrive.shared::cluster.b64 _, [%0];" ::"r"(cluster_addr) : "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx_remote(uint32_t cluster_addr, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.release.cluster.shared::cluster.b64 _, [%0], %1;" ::"r"(
                     cluster_addr),
                 "r"(bytes)
                 : "memory");
}
// 2-D tiled TMA load into this CTA's shared memory whose completion is counted on an
// mbarrier of either CTA of the pair (cta_group::2).  No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void *dst, const CUtensorMap *map,
                                                 uint32_t bar_cluster_addr, int x, int y) {
    asm volatile(
        "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%3, %4}], [%2];" ::"r"(smem_u32(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster_addr), "r"(x), "r"(y)
        : "memory");
}
// Pair-wide tensor-memory allocation (both CTAs' same warp, same shared-memory slot).
__device__ __forceinline__ void tmem_alloc_pair(uint32_t *dst_smem, uint32_t ncols) {
    asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                     smem_u32(dst_smem)),
                 "r"(ncols)
                 : "memory");
}
__device__ __forceinline__ void tmem_relinquish_pair() {
    asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}
__device__ __forceinline__ void tmem_dealloc_pair(uint32_t taddr, uint32_t ncols) {
    asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(taddr), "r"(ncols)
                 : "memory");
}
// D[tmem of both CTAs] (+)= A x B^T for a CTA pair: M = 256 rows (128 per CTA, each from
// its own shared memory), B's N columns split half per CTA.  Issued by the leader CTA.
__device__ __forceinline__ void mma_i8_ss_pair(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], %1, %2, %3, p;\n\t}" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// The same with A read from tensor memory: each CTA's 128 rows of A sit in its own tensor
// memory at a_tmem (lane = row, four 8-bit codes per 32-bit column, 8 columns per K = 32),
// B from shared memory as above.  Issued by the leader CTA.
__device__ __forceinline__ void mma_i8_ts_pair(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc,
                                               uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::2.kind::i8 [%0], [%1], %2, %3, p;\n\t}" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}
// Arrive once on the same mbarrier offset in every CTA of `mask` when all prior
// tcgen05.mma of this thread have completed.
__device__ __forceinline__ void mma_commit_pair(uint64_t *bar, uint16_t mask) {
    asm volatile(
        "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64"
        " [%0], %1;" ::"r"(smem_u32(bar)),
        "h"(mask)
        : "memory");
}

// Shared-memory matrix descriptor for a K-major operand tile stored with the 128-byte
// swizzle (rows of 128 bytes, 8-row groups 1024 bytes apart).  Layout (tcgen05):
// [0,14) start>>4, [16,30) leading byte offset>>4 (unused for swizzled K-major),
// [32,46) stride byte offset>>4, [46,48) version = 1, [49,52) base offset, [61,64) swizzle
// mode (2 = 128B).
__device__ __forceinline__ uint64_t smem_desc_sw128(const void *tile) {
    uint64_t addr = smem_u32(tile);
    uint64_t d = 0;
    d |= (addr >> 4) & 0x3FFFull;
    d |= (uint64_t)1 << 16;            // LBO (ignored)
    d |= (uint64_t)(1024 >> 4) << 32;  // SBO: 8 rows x 128 B
    d |= (uint64_t)1 << 46;            // descriptor version for tcgen05
    d |= (uint64_t)2 << 61;            // SWIZZLE_128B
    return d;
}

// Instruction descriptor, kind::i8, D = S32, K-major A and B.
// [4,6) D format (2 = S32), [7,10) A format (0 unsigned / 1 signed), [10,13) B format,
// [15] A major, [16] B major, [17,23) N>>3, [24,29) M>>4.
__host__ __device__ constexpr uint32_t idesc_i8(int m, int n, bool a_signed, bool b_signed) {
    return (2u << 4) | ((a_signed ? 1u : 0u) << 7) | ((b_signed ? 1u : 0u) << 10) |
           ((uint32_t)(n >> 3) << 17) | ((uint32_t)(m >> 4) << 24);
}

// u32 x s32 4-way byte dot product: sum_i u8(a_i) * s8(b_i) + c.
__device__ __forceinline__ int dp4a_us(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.u32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
__device__ __forceinline__ int dp4a_ss(uint32_t a, uint32_t b, int c) {
    int d;
    asm("dp4a.s32.s32 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}

// 16-byte streaming load that does not allocate in L1 (weights are read once).
// L2 eviction-priority policies (createpolicy) and the loads / stores that carry them.
__device__ __forceinline__ uint64_t l2_policy_evict_last() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
__device__ __forceinline__ void st_l2_hint(int32_t *p, int32_t v, uint64_t pol) {
    asm volatile("st.global.L2::cache_hint.b32 [%0], %1, %2;" ::"l"(p), "r"(v), "l"(pol) : "memory");
}
__device__ __forceinline__ int32_t ld_l2_hint(const int32_t *p, uint64_t pol) {
    int32_t v;
    asm volatile("ld.global.cg.L2::cache_hint.b32 %0, [%1], %2;" : "=r"(v) : "l"(p), "l"(pol) : "memory");
    return v;
}

__device__ __forceinline__ uint4 ldg_stream(const void *p) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p));
    return v;
}


// ------------------------------------------------------------------ the A8 quantiser
// (src/npu.rs:1099-1110): scale = amax == 0 ? 1 : max(amax / 127, FLT_MIN) and inv = 1 / scale
// (IEEE divisions); q = clamp(round(x * inv), -127, 127) with round = roundf (ties away from
// zero; rintf for QLINEAR_ROUND_EVEN), NaN -> 0 like Rust's `NaN as i32`.  Shared by the
// stand-alone quantisation kernel and the fused decode GEMV so both give identical codes.
__device__ __forceinline__ void a8_row_scale(float amax, float &scale, float &inv) {
    scale = amax == 0.0f ? 1.0f : fmaxf(__fdiv_rn(amax, 127.0f), 1.17549435e-38f);
    inv = __fdiv_rn(1.0f, scale);
}
__device__ __forceinline__ int a8_code(float v, float inv, int round_mode) {
    const float s = __fmul_rn(v, inv);
    const float r = round_mode ? rintf(s) : roundf(s);
    const int q = (r != r) ? 0 : __float2int_rz(r);
    return max(-127, min(127, q));
}

// 32-bit store through an NVSwitch multicast address (the NVLS mapping of every rank's
// buffer): one store, written by the switch into every GPU's copy.  Multimem stores are at
// least 32 bits wide.
__device__ __forceinline__ void multimem_st_b32(const void *mc_addr, uint32_t v) {
    asm volatile("multimem.st.global.b32 [%0], %1;" ::"l"(mc_addr), "r"(v) : "memory");
}

// Output element store helpers (f32 / f16 / raw i32).
template <typename T>
struct OutCvt;
template <>
struct OutCvt<float> {
    __device__ static __forceinline__ float from(float v) { return v; }
};
template <>
struct OutCvt<__half> {
    __device__ static __forceinline__ __half from(float v) { return __float2half_rn(v); }
};

}  // namespace ql
