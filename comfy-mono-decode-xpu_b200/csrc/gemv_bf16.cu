// bf16 GEMV of the MTP draft head's projections (fc, qkv, o, gate | up, down: the reference's F.linear calls on
// one draft row, comfy_mono_decode_xpu/draft_head.py:198-210): out[m][n] = bf16(sum_k x[m][k] * w[n][k]) with
// fp32 accumulation, for a few rows (M <= 8) of x against a bf16 weight [N][K] far larger than L2.
//
// HBM-bound: the algorithmic bytes are the weight (N * K * 2) plus M * (K + N) * 2. For K a multiple of 512 (all
// of the draft head's projections) the call runs the lm_head's ring kernel without its pick (lmhead.cu: tensor-core
// MMAs, kilobyte bulk copies). Otherwise, this file's kernel: one warp per output column
// n: lane l reads the 16-byte pieces l, l + 32, ... of weight row n (each warp load is 512 contiguous bytes),
// 4 pieces in flight per lane (measured faster than 8 at M = 1: more resident warps), read past L1 and marked evict-first in L2 (the weight is streamed once per
// draft; the KV cache and activations keep L2). The x rows come through the read-only path (L1 hits after the
// first warp). Each lane accumulates its pieces in order with fmaf, the warp reduces by a butterfly and lane 0
// rounds to bf16.
#include "launch.h"

namespace mono {

constexpr int kGvWarps = 8, kGvBatch = 4, kGvMaxM = 8;

__device__ __forceinline__ uint4 gv_ld_stream(const uint4* p, uint64_t pol) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}

__device__ __forceinline__ float gv_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float gv_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

template <int M>
__device__ __forceinline__ void gv_piece(const uint4& wv, const uint16_t* x, int64_t x_stride, int64_t piece,
                                         float (&acc)[M]) {
#pragma unroll
    for (int m = 0; m < M; ++m) {
        const uint4 xv = __ldg(reinterpret_cast<const uint4*>(x + m * x_stride) + piece);
        float a = acc[m];
        a = fmaf(gv_lo(wv.x), gv_lo(xv.x), a);
        a = fmaf(gv_hi(wv.x), gv_hi(xv.x), a);
        a = fmaf(gv_lo(wv.y), gv_lo(xv.y), a);
        a = fmaf(gv_hi(wv.y), gv_hi(xv.y), a);
        a = fmaf(gv_lo(wv.z), gv_lo(xv.z), a);
        a = fmaf(gv_hi(wv.z), gv_hi(xv.z), a);
        a = fmaf(gv_lo(wv.w), gv_lo(xv.w), a);
        a = fmaf(gv_hi(wv.w), gv_hi(xv.w), a);
        acc[m] = a;
    }
}

// grid: ceil(N / 8) CTAs of 8 warps; warp w of CTA b computes column n = 8 b + w for all M rows. At M <= 2,
// 4 CTAs fit an SM (592 resident), so the 4096-column projections run in one wave.
template <int M>
__global__ void __launch_bounds__(kGvWarps * 32, M <= 2 ? 4 : 2)
    gemv_bf16_kernel(const uint16_t* __restrict__ x, int64_t x_stride, const uint16_t* __restrict__ w, int K, int N,
                     uint16_t* __restrict__ out, int64_t out_stride) {
    const int lane = threadIdx.x & 31;
    const int n = blockIdx.x * kGvWarps + (threadIdx.x >> 5);
    if (n >= N) return;
    const uint64_t pol = l2_evict_first_policy();
    const uint4* wrow = reinterpret_cast<const uint4*>(w + int64_t(n) * K);
    const int per_lane = K / 256;  // pieces of 8 per lane
    float acc[M];
#pragma unroll
    for (int m = 0; m < M; ++m) acc[m] = 0.f;
    for (int j0 = 0; j0 < per_lane; j0 += kGvBatch) {
        uint4 wv[kGvBatch];
#pragma unroll
        for (int u = 0; u < kGvBatch; ++u)
            if (j0 + u < per_lane) wv[u] = gv_ld_stream(wrow + (j0 + u) * 32 + lane, pol);
#pragma unroll
        for (int u = 0; u < kGvBatch; ++u)
            if (j0 + u < per_lane) gv_piece<M>(wv[u], x, x_stride, int64_t(j0 + u) * 32 + lane, acc);
    }
#pragma unroll
    for (int m = 0; m < M; ++m) {
        float a = acc[m];
#pragma unroll
        for (int d = 16; d > 0; d >>= 1) a += __shfl_xor_sync(0xffffffffu, a, d);
        if (lane == 0) out[m * out_stride + n] = __bfloat16_as_ushort(__float2bfloat16_rn(a));
    }
}

template <int M>
static void gemv_bf16_launch(const uint16_t* x, int64_t x_stride, const uint16_t* w, int K, int N, uint16_t* out,
                             int64_t out_stride, cudaStream_t s) {
    gemv_bf16_kernel<M><<<unsigned((N + kGvWarps - 1) / kGvWarps), kGvWarps * 32, 0, s>>>(x, x_stride, w, K, N, out,
                                                                                         out_stride);
}

}  // namespace mono

using namespace mono;

extern "C" int mono_gemv_bf16(const void* x, int64_t x_stride, const void* w, int64_t M, int64_t N, int64_t K,
                              void* out, int64_t out_stride, mono_stream_t stream) {
    MONO_CHECK(x && w && out, "null operand");
    MONO_CHECK(M >= 1 && M <= kGvMaxM, "1 <= M <= %d rows", kGvMaxM);
    MONO_CHECK(K >= 256 && K % 256 == 0 && K <= (1 << 20), "K a multiple of 256 up to 2^20");
    MONO_CHECK(N >= 1 && N < (int64_t(1) << 31) && N * K < (int64_t(1) << 40), "1 <= N < 2^31");
    MONO_CHECK(x_stride >= K && x_stride % 8 == 0 && aligned(x, 16) && aligned(w, 16),
               "x rows and w 16-byte aligned, x_stride a multiple of 8 elements");
    MONO_CHECK(out_stride >= N && aligned(out, 2), "out rows of out_stride >= N elements");
    const auto* xs = static_cast<const uint16_t*>(x);
    const auto* ws = static_cast<const uint16_t*>(w);
    auto* o = static_cast<uint16_t*>(out);
    const cudaStream_t s = reinterpret_cast<cudaStream_t>(stream);
    const int k = int(K), n = int(N);
    // K a multiple of 512 (every projection of the draft head): the tensor-core ring kernel of the lm_head, which
    // keeps S kilobyte requests per warp in flight; other K: the warp-per-column kernel below
    if (aligned(out, 16) && out_stride % 8 == 0 && bf16_rows_fit(int(M), k))
        return launch_bf16_rows(xs, x_stride, ws, int(M), n, k, o, out_stride, s);
    switch (M) {
        case 1: gemv_bf16_launch<1>(xs, x_stride, ws, k, n, o, out_stride, s); break;
        case 2: gemv_bf16_launch<2>(xs, x_stride, ws, k, n, o, out_stride, s); break;
        case 3: gemv_bf16_launch<3>(xs, x_stride, ws, k, n, o, out_stride, s); break;
        case 4: gemv_bf16_launch<4>(xs, x_stride, ws, k, n, o, out_stride, s); break;
        case 5: gemv_bf16_launch<5>(xs, x_stride, ws, k, n, o, out_stride, s); break;
        case 6: gemv_bf16_launch<6>(xs, x_stride, ws, k, n, o, out_stride, s); break;
        case 7: gemv_bf16_launch<7>(xs, x_stride, ws, k, n, o, out_stride, s); break;
        default: gemv_bf16_launch<8>(xs, x_stride, ws, k, n, o, out_stride, s); break;
    }
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}
