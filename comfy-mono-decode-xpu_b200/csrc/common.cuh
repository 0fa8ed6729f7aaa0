// Shared device helpers for the sm_100a decode kernels: PTX wrappers for mbarriers, bulk (TMA 1-D)
// copies, cp.async, int8 mma.sync, exact bf16 conversions, and the device error word.
#pragma once
#include <cstdint>
#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>

namespace mono {

// ---- device error word ---------------------------------------------------------------------------
// Every bounded wait that gives up records a code here instead of trapping; the host reads it with
// mono_device_status(). 0 = no error.
enum DeviceError : int {
    DEV_OK = 0,
    DEV_MBAR_TIMEOUT = 1,   // an mbarrier wait ran past its iteration limit
    DEV_GRID_TIMEOUT = 2,   // a grid-wide barrier ran past its iteration limit
    DEV_FLAG_TIMEOUT = 3,   // a flag wait (peer / producer) ran past its iteration limit
    DEV_BAD_POSITION = 4,   // a KV-cache position outside [0, capacity): the write was skipped
    DEV_BAD_TREE = 5,       // a children table entry not after its parent or not below rows: the accept walk stopped
    DEV_PEER_TIMEOUT = 6,   // a wait for the peer GPU's arrival (two-GPU all-reduce) gave up
    DEV_BAD_TOKEN = 7,      // a token id outside [0, vocabulary): embedding row 0 was read instead
};
extern __device__ int g_device_error;

__device__ __forceinline__ void set_device_error(int code) { atomicCAS(&g_device_error, 0, code); }

// ---- phase trace ------------------------------------------------------------------------------------
// Off unless mono_trace_enable() set a buffer: thread 0 of every CTA of the traced kernels stores
// %globaltimer (ns) at each phase boundary into slot [blockIdx.x][phase] of a [kTraceCtas][kTracePhases]
// table. One global load per stamp when off.
constexpr int kTracePhases = 16;
constexpr int kTraceCtas = 1024;
extern __device__ unsigned long long* g_trace;

__device__ __forceinline__ unsigned long long globaltimer() {
    unsigned long long t;
    asm volatile("mov.u64 %0, %globaltimer;" : "=l"(t));
    return t;
}
__device__ __forceinline__ void trace_stamp(int phase) {
    unsigned long long* tr = g_trace;
    if (tr != nullptr && threadIdx.x == 0 && blockIdx.x < kTraceCtas && phase < kTracePhases)
        tr[blockIdx.x * kTracePhases + phase] = globaltimer();
}
// the same for a two-dimensional grid: slot = blockIdx.y * gridDim.x + blockIdx.x
__device__ __forceinline__ void trace_stamp_2d(int phase) {
    unsigned long long* tr = g_trace;
    const unsigned slot = blockIdx.y * gridDim.x + blockIdx.x;
    if (tr != nullptr && threadIdx.x == 0 && slot < kTraceCtas && phase < kTracePhases)
        tr[slot * kTracePhases + phase] = globaltimer();
}

// ---- shared-memory addresses ---------------------------------------------------------------------
__device__ __forceinline__ uint32_t smem_u32(const void* p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier -----------------------------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}
__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
__device__ __forceinline__ bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
// Bounded wait: returns false (and records DEV_MBAR_TIMEOUT) if the phase has not completed after
// kWaitLimitNs of %globaltimer time (checked every 256 polls) or kMbarSpinLimit polls. Plain try_wait
// polls (try_wait itself parks the warp for a short, hardware-chosen time): measured on B200, a suspend-time
// hint or __nanosleep back-off between polls delayed the wake-up of a producer warp waiting for a freed
// ring slot by a microsecond or more, which serialized the refills.
constexpr uint32_t kMbarSpinLimit = 1u << 26;
constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // 1 s
__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t0 = globaltimer();
    for (uint32_t i = 1; i < kMbarSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255) == 0 && globaltimer() - t0 > kWaitLimitNs) break;
    }
    set_device_error(DEV_MBAR_TIMEOUT);
    return false;
}

// ---- bulk copies (the TMA unit's 1-D mode) ---------------------------------------------------------
// Both addresses 16-byte aligned, size a multiple of 16 bytes (checked by the callers' layouts).
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar))
        : "memory");
}
// L2 policy for data read once per step (the streamed weights, ~6.6 GB a step, far above the L2): first to be
// evicted, so the activations, states, caches and kernel code that the next launches reuse stay in L2.
__device__ __forceinline__ uint64_t l2_evict_first_policy() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// bulk_g2s with an L2 cache policy (l2_evict_first_policy for the weight stream).
__device__ __forceinline__ void bulk_g2s_hint(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
            smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// ---- cp.async (16 B, global -> shared) --------------------------------------------------------------
__device__ __forceinline__ void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// ---- programmatic dependent launch ------------------------------------------------------------------
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void pdl_launch_dependents() {
    asm volatile("griddepcontrol.launch_dependents;" ::: "memory");
}

// ---- loads ------------------------------------------------------------------------------------------
__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "l"(p));
    return r;
}
__device__ __forceinline__ uint4 lds_v4(const void* p) {
    uint4 r;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w)
                 : "r"(smem_u32(p)));
    return r;
}

// ---- int8 tensor-core dot: D(16x8, s32) += A(16x32, s8, row) * B(32x8, s8, col) -----------------------
// Fragment ownership (lane = 4 * g + t): a0 = A[g][4t..4t+3], a1 = A[g+8][4t..], a2 = A[g][16+4t..],
// a3 = A[g+8][16+4t..]; b0 = B[4t..4t+3][g], b1 = B[16+4t..][g]; c0,c1 = D[g][2t, 2t+1],
// c2,c3 = D[g+8][2t, 2t+1].
__device__ __forceinline__ void mma_s8_16832(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+r"(d[0]), "+r"(d[1]), "+r"(d[2]), "+r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// D = A * B (+ 0): the zero accumulator comes from registers the caller keeps zero for the whole kernel
__device__ __forceinline__ void mma_s8_16832_z(int (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                                               uint32_t b0, uint32_t b1, uint32_t z) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%10,%10,%10,%10};"
        : "=r"(d[0]), "=r"(d[1]), "=r"(d[2]), "=r"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(z));
}

__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// ---- exact conversions ------------------------------------------------------------------------------
__device__ __forceinline__ float bf16_bits_to_f32(uint16_t b) { return __uint_as_float(uint32_t(b) << 16); }
__device__ __forceinline__ uint16_t f32_to_bf16_bits(float f) {
    return __bfloat16_as_ushort(__float2bfloat16_rn(f));
}
__device__ __forceinline__ float bf16_round(float f) { return bf16_bits_to_f32(f32_to_bf16_bits(f)); }
__device__ __forceinline__ float fp8e4m3_to_f32(uint8_t b) {
    // e4m3fn: 1 sign, 4 exponent (bias 7), 3 mantissa; 0x7F / 0xFF are NaN, no infinities.
    const uint32_t s = uint32_t(b & 0x80) << 24;
    const uint32_t e = (b >> 3) & 0xF, m = b & 7;
    if (e == 0xF && m == 7) return __uint_as_float(0x7FC00000u | s);
    if (e == 0) return __uint_as_float(s) + (s ? -1.f : 1.f) * float(m) * 0.001953125f;  // m * 2^-9
    return __uint_as_float(s | ((e + 120) << 23) | (m << 20));
}

__host__ __device__ constexpr int ceil_div(int a, int b) { return (a + b - 1) / b; }

}  // namespace mono
