// Row-local device operations of the fused kernels, run by one warp-group (128 threads, named barrier),
// with a pinned reduction order so the CPU oracle reproduces every bit.
//
// RMSNorm of one row of H bf16 values (the role of csrc/mono_common.hpp:452-505 rms_norm_row; the order is
// this build's own, every op IEEE fp32 RNE, no fused multiply-add):
//   sq[i]   = x[i] * x[i]
//   P[v]    = sum_j sq[v + 256 j]              v = 0..255, sequential in j from +0
//   W[w]    = butterfly sum of P[32 w .. 32 w + 31] (lanes l and l ^ 16, then ^ 8, ^ 4, ^ 2, ^ 1)
//   total   = sum_{w=0..7} W[w]                 sequential from +0
//   r       = 1 / sqrt(total / H + eps)         (IEEE division and square root)
//   out[i]  = bf16((x[i] * r) * w[i])
// Per-token GPTQ quantization of a bf16 row: s = amax / 127, q = clamp(rint(x / s), -127, 127), s = 0 -> q = 0.
#pragma once
#include "common.cuh"

namespace mono {

__device__ __forceinline__ void wg_sync(int wg) {
    asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory");
}

// red: >= 16 floats of shared memory owned by the warp-group. H % 256 == 0.
__device__ __forceinline__ void rmsnorm_row(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                            uint16_t* __restrict__ out, int H, float eps, float* red, int tig, int wg) {
    const int lane = tig & 31, warp = tig >> 5;
    float pa = 0.f, pb = 0.f;  // virtual threads tig and tig + 128
    for (int j = 0; j * 256 < H; ++j) {
        const float a = bf16_bits_to_f32(x[tig + 256 * j]);
        const float b = bf16_bits_to_f32(x[tig + 128 + 256 * j]);
        pa = __fadd_rn(pa, __fmul_rn(a, a));
        pb = __fadd_rn(pb, __fmul_rn(b, b));
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        pa = __fadd_rn(pa, __shfl_xor_sync(0xffffffffu, pa, o));
        pb = __fadd_rn(pb, __shfl_xor_sync(0xffffffffu, pb, o));
    }
    if (lane == 0) {
        red[warp] = pa;
        red[4 + warp] = pb;
    }
    wg_sync(wg);
    if (tig == 0) {
        float tot = 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) tot = __fadd_rn(tot, red[i]);
        const float v = __fadd_rn(__fdiv_rn(tot, float(H)), eps);
        red[8] = __fdiv_rn(1.f, __fsqrt_rn(v));
    }
    wg_sync(wg);
    const float r = red[8];
    for (int i = tig; i < H; i += 128)
        out[i] = f32_to_bf16_bits(__fmul_rn(__fmul_rn(bf16_bits_to_f32(x[i]), r), bf16_bits_to_f32(w[i])));
    wg_sync(wg);
}

__device__ __forceinline__ int8_t quant_one(float v, float s) {
    if (!(s > 0.f)) return 0;
    int q = __float2int_rn(__fdiv_rn(v, s));
    q = q > 127 ? 127 : (q < -127 ? -127 : q);
    return int8_t(q);
}

// red: >= 8 floats of the warp-group's shared memory.
__device__ __forceinline__ void quant_row(const uint16_t* __restrict__ x, int K, int8_t* __restrict__ q,
                                          float* __restrict__ s_out, float* red, int tig, int wg) {
    float amax = 0.f;
    for (int i = tig; i < K; i += 128) amax = fmaxf(amax, fabsf(bf16_bits_to_f32(x[i])));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if ((tig & 31) == 0) red[tig >> 5] = amax;
    wg_sync(wg);
    const float m = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
    const float s = __fdiv_rn(m, 127.f);
    if (tig == 0) *s_out = s;
    for (int i = tig; i < K; i += 128) q[i] = quant_one(bf16_bits_to_f32(x[i]), s);
    wg_sync(wg);
}

}  // namespace mono
