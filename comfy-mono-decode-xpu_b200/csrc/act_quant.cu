// Per-token int8 activation quantization.
//
// GPTQ mode: s = amax / 127 (IEEE fp32 division), q = clamp(rint(x / s), -127, 127)
// with RNE, per row; a row of zeros gives s = 0 and q = 0.
//
// REF mode, rot_quant (the reference's ConvRot rotate + quantize, csrc/act_prep.sycl:4-10, :71-91):
//   x_rot = bf16(x_grouped @ H)                       per 256-group; here the fp64 sum of the exact
//                                                      bf16 x bf16 products, rounded once to bf16
//   s     = max(float(amax) / 127, 1e-30)              (fp32, returned)
//   s_bf  = bf16(s), zero -> bf16 tiny (0x0080)
//   q     = int8(clamp(rint(bf16(float(x_rot) / float(s_bf))), -128, 127))
// The reference accumulates the rotation in fp32 on its matrix engine; wherever those fp32 partial sums
// are exact (bounded exponent spread inside a group, the normal case) both give the correctly rounded
// value, which the fp64 sum here gives for every input whose group spans at most 2^37 in magnitude.
#include <mutex>

#include "launch.h"
#include "rowops.cuh"

namespace mono {

namespace {

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// block-wide max of non-negative values (order-independent: exact)
template <int THREADS>
__device__ __forceinline__ float block_max(float v, float* red) {
    v = warp_max(v);
    const int w = threadIdx.x >> 5, l = threadIdx.x & 31;
    if (l == 0) red[w] = v;
    __syncthreads();
    float r = 0.f;
#pragma unroll
    for (int i = 0; i < THREADS / 32; ++i) r = fmaxf(r, red[i]);
    __syncthreads();
    return r;
}

constexpr int kAqThreads = 256;

// one CTA per row; bf16 x -> int8 q, fp32 scale
__global__ void __launch_bounds__(kAqThreads) act_quant_kernel(const uint16_t* __restrict__ x, int K,
                                                               int8_t* __restrict__ q, float* __restrict__ xs) {
    __shared__ float red[kAqThreads / 32];
    // The next kernel may launch right away (its weight prefetch overlaps this one); its own dependency
    // wait covers this kernel's output. This kernel's wait makes its completion imply the predecessor's.
    pdl_launch_dependents();
    pdl_wait();
    const int r = blockIdx.x;
    const uint16_t* xr = x + size_t(r) * K;
    float amax = 0.f;
    for (int i = threadIdx.x * 8; i < K; i += kAqThreads * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            amax = fmaxf(amax, fabsf(__uint_as_float(w[j] << 16)));
            amax = fmaxf(amax, fabsf(__uint_as_float(w[j] & 0xFFFF0000u)));
        }
    }
    amax = block_max<kAqThreads>(amax, red);
    const float s = __fdiv_rn(amax, 127.f);
    if (threadIdx.x == 0) xs[r] = s;
    int8_t* qr = q + size_t(r) * K;
    for (int i = threadIdx.x * 8; i < K; i += kAqThreads * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + i);
        const uint32_t w[4] = {v.x, v.y, v.z, v.w};
        float f[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) f[j] = __uint_as_float((j & 1) ? (w[j >> 1] & 0xFFFF0000u) : (w[j >> 1] << 16));
        *reinterpret_cast<uint2*>(qr + i) = quant8(f, s);  // rowops.cuh: the quotient's rounding without dividing
    }
}

// ---- REF rot_quant ----------------------------------------------------------------------------------
// Exactly rounded fp64 -> bf16 (RNE, subnormals included): quantum 2^(max(e, -126) - 7).
__device__ __forceinline__ uint16_t f64_to_bf16_bits(double v) {
    if (isnan(v)) return 0x7FC0;
    const int e = ilogb(fabs(v));  // ilogb(0) = INT_MIN
    const int qe = (e > -126 ? e : -126) - 7;
    const double r = rint(scalbn(v, -qe)) * scalbn(1.0, qe);
    const float f = float(r);  // exact: r has at most 8 significant bits (or is +-inf after overflow)
    return uint16_t(__float_as_uint(f) >> 16);
}

// Phase 1: block (group, row): x_rot of one 256-group; thread j owns output column j.
__global__ void __launch_bounds__(256) rot_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ h,
                                                  int K, uint16_t* __restrict__ xr, unsigned* __restrict__ amax_bits) {
    __shared__ double xg[256];
    pdl_wait();
    const int grp = blockIdx.x, r = blockIdx.y, j = threadIdx.x;
    const uint16_t* src = x + size_t(r) * K + grp * 256;
    xg[j] = double(bf16_bits_to_f32(src[j]));
    __syncthreads();
    double acc = 0.0;
#pragma unroll 8
    for (int k = 0; k < 256; ++k) acc = fma(xg[k], double(bf16_bits_to_f32(__ldg(h + k * 256 + j))), acc);
    const uint16_t b = f64_to_bf16_bits(acc);
    xr[size_t(r) * K + grp * 256 + j] = b;
    __shared__ float red[8];
    const float m = block_max<256>(fabsf(bf16_bits_to_f32(b)), red);
    if (j == 0) atomicMax(amax_bits + r, __float_as_uint(m));  // non-negative floats order as integers
}

// Phase 2: one block per (group, row): scale and quantize; the last group of a row resets its amax word.
__global__ void __launch_bounds__(256) rot_quant_kernel(const uint16_t* __restrict__ xr, int K,
                                                        unsigned* __restrict__ amax_bits, unsigned* __restrict__ done,
                                                        int8_t* __restrict__ q, float* __restrict__ scale) {
    const int grp = blockIdx.x, r = blockIdx.y, j = threadIdx.x;
    const float amax = __uint_as_float(__ldcg(amax_bits + r));
    const float s = fmaxf(__fdiv_rn(amax, 127.f), 1e-30f);
    uint16_t sb = f32_to_bf16_bits(s);
    if ((sb & 0x7FFF) == 0) sb = 0x0080;  // torch.finfo(bfloat16).tiny
    const float sbf = bf16_bits_to_f32(sb);
    const float d = bf16_round(__fdiv_rn(bf16_bits_to_f32(xr[size_t(r) * K + grp * 256 + j]), sbf));
    const float c = fminf(fmaxf(rintf(d), -128.f), 127.f);
    q[size_t(r) * K + grp * 256 + j] = int8_t(int(c));
    if (grp == 0 && j == 0) scale[r] = s;
    __syncthreads();
    if (j == 0) {
        __threadfence();
        if (atomicAdd(done + r, 1u) == unsigned(gridDim.x) - 1) {
            amax_bits[r] = 0u;
            done[r] = 0u;
        }
    }
    pdl_launch_dependents();
}

}  // namespace

int launch_act_quant(const void* x, int M, int K, int8_t* q, float* xs, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(M);
    cfg.blockDim = dim3(kAqThreads);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, act_quant_kernel, static_cast<const uint16_t*>(x), K, q, xs));
    return MONO_OK;
}

// workspace: amax words [kRotMaxRows] and done counters [kRotMaxRows] at fixed offsets (zero on first use;
// the kernels leave them zero again), then xr bf16 [M][K]. The fixed offsets keep the counters clear of
// the rotated rows of any earlier call with another shape.
constexpr int kRotMaxRows = 256;
size_t rot_quant_workspace(int M, int K) { return size_t(kRotMaxRows) * 8 + size_t(M) * K * 2; }

int launch_rot_quant(const void* x, const void* h, int M, int K, int8_t* q, float* s, void* ws, cudaStream_t stream) {
    if (M > kRotMaxRows) return fail(MONO_EINVAL, "rot_quant: at most %d rows (got %d)", kRotMaxRows, M);
    auto* amax = static_cast<unsigned*>(ws);
    auto* done = amax + kRotMaxRows;
    auto* xr = reinterpret_cast<uint16_t*>(static_cast<uint8_t*>(ws) + size_t(kRotMaxRows) * 8);
    rot_kernel<<<dim3(K / 256, M), 256, 0, stream>>>(static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(h),
                                                      K, xr, amax);
    CUDA_TRY(cudaGetLastError());
    rot_quant_kernel<<<dim3(K / 256, M), 256, 0, stream>>>(xr, K, amax, done, q, s);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

// ---- rot_quant without allocation ------------------------------------------------------------------
// Scratch of mono_rot_quant_noalloc: the same layout as the caller-provided workspace of mono_rot_quant
// (kRotMaxRows amax words and done counters, then the rotated rows), sized for at most
// kNoAllocRows x kNoAllocK. Every GPU that loads the library holds these ~386 KB until the process exits.
constexpr int kNoAllocRows = 16;
constexpr int kNoAllocK = 12288;
constexpr size_t kNoAllocBytes = size_t(kRotMaxRows) * 8 + size_t(kNoAllocRows) * kNoAllocK * 2;
static __device__ __align__(256) uint8_t g_rot_scratch[kNoAllocBytes];

// Device address of g_rot_scratch in the current context, looked up once per (device, context). In host code
// the symbol names a host-side stand-in, never the device memory: only this address may reach a kernel. The
// cache remembers which context the address belongs to (the driver's cuCtxGetCurrent, reached through the
// runtime's entry-point query so no driver library is linked): after cudaDeviceReset, or with another context
// made current on the same device, the address is looked up again instead of reusing a stale one.
typedef int (*CtxGetCurrentFn)(void**);
static CtxGetCurrentFn ctx_get_current() {
    static CtxGetCurrentFn fn = [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        if (cudaGetDriverEntryPoint("cuCtxGetCurrent", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            p = nullptr;
        return reinterpret_cast<CtxGetCurrentFn>(p);
    }();
    return fn;
}

static int rot_scratch_address(void** out) {
    static std::mutex mu;
    static void* addr[64] = {};
    static void* owner[64] = {};
    int dev = 0;
    CUDA_TRY(cudaGetDevice(&dev));
    if (dev < 0 || dev >= 64) return fail(MONO_EINVAL, "rot_quant_noalloc: device ordinal %d out of range", dev);
    const CtxGetCurrentFn get = ctx_get_current();
    if (get == nullptr) return fail(MONO_ECUDA, "rot_quant_noalloc: cuCtxGetCurrent is not available");
    void* ctx = nullptr;
    if (get(&ctx) != 0) return fail(MONO_ECUDA, "rot_quant_noalloc: cuCtxGetCurrent failed");
    std::lock_guard<std::mutex> lock(mu);
    if (ctx == nullptr || addr[dev] == nullptr || owner[dev] != ctx) {
        void* p = nullptr;
        CUDA_TRY(cudaGetSymbolAddress(&p, g_rot_scratch));  // (initializes the device's context if none was current)
        if (ctx == nullptr && (get(&ctx) != 0 || ctx == nullptr))
            return fail(MONO_ECUDA, "rot_quant_noalloc: no current CUDA context");
        addr[dev] = p;
        owner[dev] = ctx;
    }
    *out = addr[dev];
    return MONO_OK;
}

int launch_rot_quant_noalloc(const void* x, const void* h, int M, int K, int8_t* q, float* s, cudaStream_t stream) {
    if (M < 1 || M > kNoAllocRows || K < 256 || K > kNoAllocK || K % 256)
        return fail(MONO_EINVAL,
                    "rot_quant_noalloc: shape [%d, %d] exceeds the fixed scratch (1 <= M <= %d rows, K <= %d, K %% 256 "
                    "== 0); use mono_rot_quant with a workspace",
                    M, K, kNoAllocRows, kNoAllocK);
    void* ws = nullptr;
    const int rc = rot_scratch_address(&ws);
    if (rc) return rc;
    // the amax words and done counters must start at zero: clear them (the rows need no clearing)
    CUDA_TRY(cudaMemsetAsync(ws, 0, size_t(kRotMaxRows) * 8, stream));
    return launch_rot_quant(x, h, M, K, q, s, ws, stream);
}

}  // namespace mono
