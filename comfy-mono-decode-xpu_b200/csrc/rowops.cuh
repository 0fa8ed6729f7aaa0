// Row-local device operations of the fused kernels, run by one warp-group (128 threads, named barrier),
// with a pinned reduction order so the CPU oracle reproduces every bit.
//
// A row of H bf16 values (H % 1024 == 0, H <= 4096) is held in registers: thread t owns the 8-element
// pieces c = t + 128 j (j = 0 .. H/1024 - 1), loaded with all requests in flight.
//
// RMSNorm (the role of csrc/mono_common.hpp:452-505 rms_norm_row; this order is this build's own, every op
// IEEE fp32 RNE, no fused multiply-add):
//   P[t]   = sum over j, then over e = 0..7, of x[8 (t + 128 j) + e]^2      sequential from +0
//   W[w]   = butterfly sum of P[32 w .. 32 w + 31] (lanes l and l ^ 16, then ^ 8, ^ 4, ^ 2, ^ 1)
//   total  = W[0] + W[1] + W[2] + W[3]                                        sequential from +0
//   r      = 1 / sqrt(total / H + eps)                                        (IEEE division, square root)
//   out[i] = bf16((x[i] * r) * w[i])
// Per-token GPTQ quantization: s = amax / 127, q = clamp(rint(x / s), -127, 127) (x / s the IEEE quotient; see
// quant_i), s = 0 -> q = 0; q is written in the engine's permuted activation layout (bytes 0 2 4 6 1 3 5 7 of
// every 8).
#pragma once
#include "common.cuh"

namespace mono {

constexpr int kRowMaxPieces = 4;  // H <= 4096

__device__ __forceinline__ void wg_sync(int wg) {
    asm volatile("bar.sync %0, 128;" ::"r"(1 + wg) : "memory");
}

// Per-token quantization of one value: q = clamp(rint(RN32(v / s)), -127, 127), RN32(v / s) the IEEE fp32 quotient
// (round to nearest even), rint ties to even; s <= 0 (or NaN) gives 0. Division-free, with the same results:
//   a = RN(v * inv), inv = RN(1 / s), with s in [2^-120, 2^120] (inv normal): |a - v / s| <= |v / s| 2^-23 and
//   |RN32(v / s) - v / s| <= |v / s| 2^-24, so for |a| < 200 both lie within 2^-14 of each other. rint(a) is formed
//   by the magic-number addition t = a + 1.5 * 2^23 (exact integer rounding, ties to even, for |a| < 2^22).
//   When a is farther than 2^-14 from the half-integer between the two candidate integers, rint(a) is the
//   answer (about 2^13 values in 2^14). Otherwise quant_near_half decides exactly.
// quant_near_half: with h the half-integer, X = v - h s is exact in fp64 (h has <= 9 significant bits, s 24, and
//   v - h s is a small multiple of their common quantum); RN32(v / s) = h exactly when X lies in
//   [-gap_below s, gap_above s], the gaps being half the fp32 spacing on each side of h (a quarter below |h| =
//   0.5, the one power of two among half-integers; the ties at the ends go to h, whose significand is even),
//   and rint(h) is the even neighbour; otherwise RN32(v / s) lies on the side given by the sign of X.
static __device__ __noinline__ int quant_near_half(float v, float s, float a) {
    if (!(a == a)) return 0;                                  // NaN (the quotient converts to 0)
    if (!(fabsf(a) < 200.f)) return a > 0.f ? 127 : -127;     // clamps either way
    const float h = floorf(a) + 0.5f;
    const double X = double(v) - double(h) * double(s);
    const int eb = (__float_as_int(h) >> 23) & 0xFF;
    const double half_u = ldexp(1.0, eb - 151);               // half the fp32 spacing at |h|: 2^(e - 24)
    const bool pow2 = (__float_as_int(h) & 0x7FFFFF) == 0;    // |h| = 0.5
    const double away = half_u * double(s), toward = (pow2 ? 0.5 * half_u : half_u) * double(s);
    const double above = h > 0.f ? away : toward, below = h > 0.f ? toward : away;
    const int k = int(h - 0.5f);                              // the integer below h
    if (X > above) return k + 1;
    if (X < -below) return k;
    return (k & 1) ? k + 1 : k;
}
// the IEEE quotient itself, for scales outside [2^-120, 2^120]
static __device__ __noinline__ int quant_by_division(float v, float s) { return __float2int_rn(__fdiv_rn(v, s)); }

__device__ __forceinline__ bool quant_scale_fast(float s) { return s >= 0x1p-120f && s <= 0x1p120f; }

__device__ __forceinline__ int quant_i(float v, float s, float inv) {
    const float a = __fmul_rn(v, inv);
    const float t = __fadd_rn(a, 12582912.f);
    const float d = __fsub_rn(a, __fsub_rn(t, 12582912.f));
    int q = __float_as_int(t) - 0x4B400000;
    if (!(fabsf(a) < 200.f && fabsf(d) < 0.5f - 0x1p-14f)) q = quant_near_half(v, s, a);
    return max(-127, min(127, q));
}

// 8 values -> 8 int8 (as int) with the scale's checks done once
__device__ __forceinline__ void quant8_ints(const float (&v)[8], float s, int (&q)[8]) {
    if (!(s > 0.f)) {
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] = 0;
    } else if (quant_scale_fast(s)) {
        const float inv = __frcp_rn(s);
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] = quant_i(v[e], s, inv);
    } else {
#pragma unroll
        for (int e = 0; e < 8; ++e) q[e] = max(-127, min(127, quant_by_division(v[e], s)));
    }
}

// 8 quantized values in natural byte order (bytes 0..7)
__device__ __forceinline__ uint2 quant8(const float (&v)[8], float s) {
    int q[8];
    quant8_ints(v, s, q);
    uint32_t b[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) b[e] = uint32_t(q[e]) & 0xFFu;
    return make_uint2(b[0] | b[1] << 8 | b[2] << 16 | b[3] << 24, b[4] | b[5] << 8 | b[6] << 16 | b[7] << 24);
}

// Position of byte i in the engine's permuted activation layout (bytes 0 2 4 6 1 3 5 7 of every 8).
__device__ __forceinline__ int perm8(int i) { return (i & ~7) | ((i & 1) ? 4 + ((i & 7) >> 1) : ((i & 7) >> 1)); }

// 8 quantized values -> the permuted 8-byte word (bytes 0 2 4 6 | 1 3 5 7)
__device__ __forceinline__ uint2 quant8_perm(const float (&v)[8], float s) {
    int q[8];
    quant8_ints(v, s, q);
    uint32_t b[8];
#pragma unroll
    for (int e = 0; e < 8; ++e) b[e] = uint32_t(q[e]) & 0xFFu;
    return make_uint2(b[0] | b[2] << 8 | b[4] << 16 | b[6] << 24, b[1] | b[3] << 8 | b[5] << 16 | b[7] << 24);
}

// Optional RMSNorm (w != null) and per-token quantization of one row. xn_out (optional): the normalized
// bf16 row. q: int8 [H] permuted; s_out: the row scale. red: >= 16 floats of the warp-group's shared memory.
__device__ __forceinline__ void norm_quant_row(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w, float eps,
                                               int H, uint16_t* __restrict__ xn_out, int8_t* __restrict__ q,
                                               float* __restrict__ s_out, float* red, int tig, int wg) {
    const int lane = tig & 31, warp = tig >> 5, J = H >> 10;
    uint4 xv[kRowMaxPieces], wv[kRowMaxPieces];
#pragma unroll
    for (int j = 0; j < kRowMaxPieces; ++j)
        if (j < J) {
            xv[j] = __ldcg(reinterpret_cast<const uint4*>(x) + tig + 128 * j);
            if (w) wv[j] = __ldg(reinterpret_cast<const uint4*>(w) + tig + 128 * j);
        }
    float vals[kRowMaxPieces][8];
#pragma unroll
    for (int j = 0; j < kRowMaxPieces; ++j)
        if (j < J) {
            const uint32_t u[4] = {xv[j].x, xv[j].y, xv[j].z, xv[j].w};
#pragma unroll
            for (int e = 0; e < 8; ++e) vals[j][e] = __uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16));
        }
    if (w) {
        float p = 0.f;
#pragma unroll
        for (int j = 0; j < kRowMaxPieces; ++j)
            if (j < J)
#pragma unroll
                for (int e = 0; e < 8; ++e) p = __fadd_rn(p, __fmul_rn(vals[j][e], vals[j][e]));
#pragma unroll
        for (int o = 16; o; o >>= 1) p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, o));
        if (lane == 0) red[warp] = p;
        wg_sync(wg);
        const float tot = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.f, red[0]), red[1]), red[2]), red[3]);
        const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, float(H)), eps)));
#pragma unroll
        for (int j = 0; j < kRowMaxPieces; ++j)
            if (j < J) {
                const uint32_t u[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
                uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float wf = __uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16));
                    const uint16_t b = f32_to_bf16_bits(__fmul_rn(__fmul_rn(vals[j][e], r), wf));
                    vals[j][e] = bf16_bits_to_f32(b);
                    o[e >> 1] |= uint32_t(b) << (16 * (e & 1));
                }
                if (xn_out) reinterpret_cast<uint4*>(xn_out)[tig + 128 * j] = make_uint4(o[0], o[1], o[2], o[3]);
            }
    }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < kRowMaxPieces; ++j)
        if (j < J)
#pragma unroll
            for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(vals[j][e]));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red[8 + warp] = amax;
    wg_sync(wg);
    const float m = fmaxf(fmaxf(red[8], red[9]), fmaxf(red[10], red[11]));
    const float s = __fdiv_rn(m, 127.f);
    if (tig == 0) *s_out = s;
#pragma unroll
    for (int j = 0; j < kRowMaxPieces; ++j)
        if (j < J) reinterpret_cast<uint2*>(q)[tig + 128 * j] = quant8_perm(vals[j], s);
    wg_sync(wg);
}

// Sigmoid gate and per-token quantization of one row by a warp-group (H = 128 t + 1024 j pieces as in
// norm_quant_row; H <= 4096).
__device__ __forceinline__ void gate_quant_row(const uint16_t* __restrict__ x, const uint16_t* __restrict__ gate,
                                               int64_t gate_head_stride, const uint16_t* __restrict__ lut, int H,
                                               int8_t* __restrict__ q, float* __restrict__ s_out, float* red, int tig,
                                               int wg) {
    const int lane = tig & 31, warp = tig >> 5, J = H >> 10;
    float vals[kRowMaxPieces][8];
#pragma unroll
    for (int j = 0; j < kRowMaxPieces; ++j)
        if (j < J) {
            const int c0 = (tig + 128 * j) * 8;  // 8 columns inside one 256-wide head
            const uint4 xv = __ldcg(reinterpret_cast<const uint4*>(x + c0));
            const uint4 gv = __ldcg(reinterpret_cast<const uint4*>(gate + (c0 >> 8) * gate_head_stride + (c0 & 255)));
            const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w}, gu[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const uint32_t xb = (e & 1) ? (xu[e >> 1] >> 16) : (xu[e >> 1] & 0xFFFFu);
                const uint32_t gb = (e & 1) ? (gu[e >> 1] >> 16) : (gu[e >> 1] & 0xFFFFu);
                vals[j][e] = bf16_round(__fmul_rn(bf16_bits_to_f32(uint16_t(xb)), bf16_bits_to_f32(__ldg(lut + gb))));
            }
        }
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < kRowMaxPieces; ++j)
        if (j < J)
#pragma unroll
            for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(vals[j][e]));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red[8 + warp] = amax;
    wg_sync(wg);
    const float m = fmaxf(fmaxf(red[8], red[9]), fmaxf(red[10], red[11]));
    const float s = __fdiv_rn(m, 127.f);
    if (tig == 0) *s_out = s;
#pragma unroll
    for (int j = 0; j < kRowMaxPieces; ++j)
        if (j < J) reinterpret_cast<uint2*>(q)[tig + 128 * j] = quant8_perm(vals[j], s);
    wg_sync(wg);
}

// ---- the same row operations spread over NT threads of one CTA (named barrier BAR of those NT threads) ----
// Same bits as the warp-group forms above: the RMSNorm sum of squares is still formed by threads t < 128 over
// pieces t + 128 j (the pinned order); everything per element (normalize, gate, quantize) and the row maximum
// (order-free) is spread over all NT threads, piece c on thread c % NT. red: >= 64 floats of shared memory.
template <int NT>
struct RowPieces {
    static constexpr int kMax = (512 + NT - 1) / NT;  // 8-element pieces per thread (rows up to 4096)
};

template <int NT, int BAR>
__device__ __forceinline__ void row_sync() {
    asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(NT) : "memory");
}

// Row maximum of |vals| over the NT threads and the quantization of the thread's pieces.
template <int NT, int BAR>
__device__ __forceinline__ void row_quant_pieces(const float (&vals)[RowPieces<NT>::kMax][8], int np, int8_t* q,
                                                 float* s_out, float* red) {
    constexpr int KP = RowPieces<NT>::kMax;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    float amax = 0.f;
#pragma unroll
    for (int i = 0; i < KP; ++i)
        if (tid + NT * i < np)
#pragma unroll
            for (int e = 0; e < 8; ++e) amax = fmaxf(amax, fabsf(vals[i][e]));
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red[16 + warp] = amax;
    row_sync<NT, BAR>();
    float m = 0.f;
#pragma unroll
    for (int w = 0; w < NT / 32; ++w) m = fmaxf(m, red[16 + w]);
    const float s = __fdiv_rn(m, 127.f);
    if (tid == 0) *s_out = s;
#pragma unroll
    for (int i = 0; i < KP; ++i)
        if (tid + NT * i < np) reinterpret_cast<uint2*>(q)[tid + NT * i] = quant8_perm(vals[i], s);
    row_sync<NT, BAR>();
}

// Optional RMSNorm (w != null) and per-token quantization of one row (norm_quant_row's arithmetic).
template <int NT, int BAR>
__device__ __forceinline__ void norm_quant_row_cta(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                                   float eps, int H, uint16_t* __restrict__ xn_out, int8_t* __restrict__ q,
                                                   float* __restrict__ s_out, float* red) {
    constexpr int KP = RowPieces<NT>::kMax;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, np = H >> 3, J = H >> 10;
    float vals[KP][8];
    uint4 wv[KP], xv[KP];
    // every load of the row in flight at once: the pieces of the sum of squares (threads t < 128: pieces
    // t + 128 j, the pinned order), then the thread's own pieces and norm weights
    uint4 sv[kRowMaxPieces];
    if (w && tid < 128)
#pragma unroll
        for (int j = 0; j < kRowMaxPieces; ++j)
            if (j < J) sv[j] = __ldcg(reinterpret_cast<const uint4*>(x) + tid + 128 * j);
#pragma unroll
    for (int i = 0; i < KP; ++i)
        if (tid + NT * i < np) {
            xv[i] = __ldcg(reinterpret_cast<const uint4*>(x) + tid + NT * i);
            if (w) wv[i] = __ldg(reinterpret_cast<const uint4*>(w) + tid + NT * i);
        }
#pragma unroll
    for (int i = 0; i < KP; ++i)
        if (tid + NT * i < np) {
            const uint32_t u[4] = {xv[i].x, xv[i].y, xv[i].z, xv[i].w};
#pragma unroll
            for (int e = 0; e < 8; ++e) vals[i][e] = __uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16));
        }
    if (w) {
        if (tid < 128) {  // the pinned sum of squares: thread t over pieces t + 128 j
            float p = 0.f;
#pragma unroll
            for (int j = 0; j < kRowMaxPieces; ++j)
                if (j < J) {
                    const uint32_t u[4] = {sv[j].x, sv[j].y, sv[j].z, sv[j].w};
#pragma unroll
                    for (int e = 0; e < 8; ++e) {
                        const float f = __uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16));
                        p = __fadd_rn(p, __fmul_rn(f, f));
                    }
                }
#pragma unroll
            for (int o = 16; o; o >>= 1) p = __fadd_rn(p, __shfl_xor_sync(0xffffffffu, p, o));
            if (lane == 0) red[warp] = p;
        }
        row_sync<NT, BAR>();
        const float tot = __fadd_rn(__fadd_rn(__fadd_rn(__fadd_rn(0.f, red[0]), red[1]), red[2]), red[3]);
        const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, float(H)), eps)));
#pragma unroll
        for (int i = 0; i < KP; ++i)
            if (tid + NT * i < np) {
                const uint32_t u[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
                uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float wf = __uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16));
                    const uint16_t b = f32_to_bf16_bits(__fmul_rn(__fmul_rn(vals[i][e], r), wf));
                    vals[i][e] = bf16_bits_to_f32(b);
                    o[e >> 1] |= uint32_t(b) << (16 * (e & 1));
                }
                if (xn_out) reinterpret_cast<uint4*>(xn_out)[tid + NT * i] = make_uint4(o[0], o[1], o[2], o[3]);
            }
    }
    row_quant_pieces<NT, BAR>(vals, np, q, s_out, red);
}

// Sigmoid gate and quantization of one row (gate_quant_row's arithmetic).
template <int NT, int BAR>
__device__ __forceinline__ void gate_quant_row_cta(const uint16_t* __restrict__ x, const uint16_t* __restrict__ gate,
                                                   int64_t gate_head_stride, const uint16_t* __restrict__ lut, int H,
                                                   int8_t* __restrict__ q, float* __restrict__ s_out, float* red) {
    constexpr int KP = RowPieces<NT>::kMax;
    const int tid = threadIdx.x, np = H >> 3;
    float vals[KP][8];
#pragma unroll
    for (int i = 0; i < KP; ++i)
        if (tid + NT * i < np) {
            const int c0 = (tid + NT * i) * 8;
            const uint4 xv = __ldcg(reinterpret_cast<const uint4*>(x + c0));
            const uint4 gv = __ldcg(reinterpret_cast<const uint4*>(gate + (c0 >> 8) * gate_head_stride + (c0 & 255)));
            const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w}, gu[4] = {gv.x, gv.y, gv.z, gv.w};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const uint32_t xb = (e & 1) ? (xu[e >> 1] >> 16) : (xu[e >> 1] & 0xFFFFu);
                const uint32_t gb = (e & 1) ? (gu[e >> 1] >> 16) : (gu[e >> 1] & 0xFFFFu);
                vals[i][e] = bf16_round(__fmul_rn(bf16_bits_to_f32(uint16_t(xb)), bf16_bits_to_f32(__ldg(lut + gb))));
            }
        }
    row_quant_pieces<NT, BAR>(vals, np, q, s_out, red);
}

// Per-token quantization of a whole activation block x [M][K] bf16 by the first T threads of the CTA
// (named barrier BAR), into the permuted int8 rows of a shared buffer (row pitch `pitch`) and the row
// scales xs[M]. Rows are taken in batches whose 16-byte pieces fit 8 per thread, so a batch costs one round
// trip to L2: every load of a batch is issued before any is used. Row maxima meet in shared memory
// (rowmax[16], float bits: the values are non-negative, so integer order is float order; zeroed here).
// Same results as the per-token quantization above (amax is order-free).
template <int T, int BAR>
__device__ __forceinline__ void quant_block(const uint16_t* __restrict__ x, int M, int K, int8_t* __restrict__ xsm,
                                            int pitch, float* __restrict__ xs, unsigned* rowmax) {
    auto sync = [] { asm volatile("bar.sync %0, %1;" ::"n"(BAR), "n"(T) : "memory"); };
    const int tid = threadIdx.x, lane = tid & 31, P = K >> 3;  // P % 128 == 0
    if (tid < 16) rowmax[tid] = 0u;
    sync();
    const int RB = (8 * T) / P > 0 ? ((8 * T) / P < M ? (8 * T) / P : M) : 1;
    for (int r0 = 0; r0 < M; r0 += RB) {
        const int rb = M - r0 < RB ? M - r0 : RB;
        const int n = rb * P;
        const uint4* src = reinterpret_cast<const uint4*>(x + size_t(r0) * K);
        uint4 v[8];
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = tid + T * j;
            if (i < n) v[j] = __ldcg(src + i);
        }
        if (RB == 1 && P > 8 * T) {
            // one row longer than the threads hold in registers: fold the rest of it in a second loop (the
            // quantization pass below re-reads those pieces)
            float am = 0.f;
            for (int i = tid + 8 * T; i < P; i += T) {
                const uint4 w = __ldcg(src + i);
                const uint32_t u[4] = {w.x, w.y, w.z, w.w};
#pragma unroll
                for (int e = 0; e < 8; ++e)
                    am = fmaxf(am, fabsf(__uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16))));
            }
#pragma unroll
            for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
            if (lane == 0) atomicMax(rowmax + r0, __float_as_uint(am));
        }
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = tid + T * j;
            if (T * j < n) {  // warp-uniform: n and T are multiples of 32
                float am = 0.f;
                if (i < n) {
                    const uint32_t u[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        am = fmaxf(am, fabsf(__uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16))));
                }
#pragma unroll
                for (int o = 16; o; o >>= 1) am = fmaxf(am, __shfl_xor_sync(0xffffffffu, am, o));
                // the 32 pieces of a warp lie in one row (P % 32 == 0)
                if (lane == 0 && i < n) atomicMax(rowmax + r0 + i / P, __float_as_uint(am));
            }
        }
        sync();
#pragma unroll
        for (int j = 0; j < 8; ++j) {
            const int i = tid + T * j;
            if (i < n) {
                const int r = i / P, c = i - r * P;
                const float s = __fdiv_rn(__uint_as_float(rowmax[r0 + r]), 127.f);
                const uint32_t u[4] = {v[j].x, v[j].y, v[j].z, v[j].w};
                float vals[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) vals[e] = __uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16));
                reinterpret_cast<uint2*>(xsm + size_t(r0 + r) * pitch)[c] = quant8_perm(vals, s);
            }
        }
        if (RB == 1 && P > 8 * T) {
            const float s = __fdiv_rn(__uint_as_float(rowmax[r0]), 127.f);
            for (int i = tid + 8 * T; i < P; i += T) {
                const uint4 w = __ldcg(src + i);
                const uint32_t u[4] = {w.x, w.y, w.z, w.w};
                float vals[8];
#pragma unroll
                for (int e = 0; e < 8; ++e) vals[e] = __uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16));
                reinterpret_cast<uint2*>(xsm + size_t(r0) * pitch)[i] = quant8_perm(vals, s);
            }
        }
    }
    sync();
    if (tid < M) xs[tid] = __fdiv_rn(__uint_as_float(rowmax[tid]), 127.f);
    sync();
}

}  // namespace mono
