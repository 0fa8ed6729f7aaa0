// Small row kernels of the bf16 parts of the decode step (the MTP draft head, the final norm): each replaces
// a handful of framework elementwise launches.
//   rmsnorm_add  s = add ? bf16(x + add) : x;  out = bf16((s * r) * w), r = 1 / sqrt(mean(s^2) + eps)
//                (sum_out receives s). One CTA of 256 threads per row; thread t owns the 8-element pieces
//                t + 256 j; squares summed per thread (j outer, element inner), xor butterfly per warp, the
//                8 warp sums in order; IEEE division and square root.
//   lut_mul      out[m][c] = bf16(a[m][c] * lut[b[m][(c / 256) * b_head_stride + c % 256]]) with lut the SiLU
//                or sigmoid of every bf16 pattern: SiLU(gate) * up, or attention * sigmoid(gate).
#include "launch.h"

namespace mono {

// One row by the 256 threads of a CTA: s = add ? bf16(xr + addr) : xr (sum_r receives s), out_r = bf16((s * r) * w).
__device__ __forceinline__ void rmsnorm_row(const uint16_t* __restrict__ xr, const uint16_t* __restrict__ addr,
                                            const uint16_t* __restrict__ w, float eps, int H, uint16_t* __restrict__ out_r,
                                            uint16_t* __restrict__ sum_r, float* red) {
    const int t = threadIdx.x, lane = t & 31, warp = t >> 5, P = H >> 3;
    const uint16_t* add = addr;
    uint16_t* sum_out = sum_r;
    float ss = 0.f;
    for (int c = t; c < P; c += 256) {
        const uint4 v = __ldg(reinterpret_cast<const uint4*>(xr) + c);
        uint4 a = make_uint4(0, 0, 0, 0);
        if (add) a = __ldg(reinterpret_cast<const uint4*>(add) + c);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w}, au[4] = {a.x, a.y, a.z, a.w};
        uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            float f = __uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16));
            if (add) f = bf16_round(__fadd_rn(f, __uint_as_float((e & 1) ? (au[e >> 1] & 0xFFFF0000u) : (au[e >> 1] << 16))));
            ss = __fadd_rn(ss, __fmul_rn(f, f));
            o[e >> 1] |= uint32_t(f32_to_bf16_bits(f)) << (16 * (e & 1));
        }
        if (sum_out) reinterpret_cast<uint4*>(sum_out)[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) ss = __fadd_rn(ss, __shfl_xor_sync(0xffffffffu, ss, o));
    if (lane == 0) red[warp] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot = __fadd_rn(tot, red[i]);
    const float r = __fdiv_rn(1.f, __fsqrt_rn(__fadd_rn(__fdiv_rn(tot, float(H)), eps)));
    for (int c = t; c < P; c += 256) {
        const uint4 v = sum_out ? reinterpret_cast<const uint4*>(sum_out)[c] : __ldg(reinterpret_cast<const uint4*>(xr) + c);
        const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w) + c);
        const uint32_t u[4] = {v.x, v.y, v.z, v.w}, wu[4] = {wv.x, wv.y, wv.z, wv.w};
        uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
        for (int e = 0; e < 8; ++e) {
            const float f = __uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16));
            const float wf = __uint_as_float((e & 1) ? (wu[e >> 1] & 0xFFFF0000u) : (wu[e >> 1] << 16));
            o[e >> 1] |= uint32_t(f32_to_bf16_bits(__fmul_rn(__fmul_rn(f, r), wf))) << (16 * (e & 1));
        }
        reinterpret_cast<uint4*>(out_r)[c] = make_uint4(o[0], o[1], o[2], o[3]);
    }
}

__global__ void __launch_bounds__(256) rmsnorm_add_kernel(const uint16_t* __restrict__ x, const uint16_t* __restrict__ add,
                                                          const uint16_t* __restrict__ w, float eps, int H, int64_t x_stride,
                                                          int64_t add_stride, int64_t out_stride, uint16_t* __restrict__ out,
                                                          uint16_t* __restrict__ sum_out) {
    pdl_launch_dependents();  // an ordinary launch: its inputs are complete; the next kernel may start
    __shared__ float red[8];
    const size_t m = blockIdx.x;
    rmsnorm_row(x + m * x_stride, add ? add + m * add_stride : nullptr, w, eps, H, out + m * out_stride,
                sum_out ? sum_out + m * out_stride : nullptr, red);
}

// The MTP draft head's front for row b (one per stream): CTA (0, b) normalizes the embedding row of token
// tokens[b * tok_stride + index] with enorm into out[b][0, H), CTA (1, b) the hidden row with hnorm into
// out[b][H, 2H) (rmsnorm_row: the bits of two mono_rmsnorm_add calls on the gathered rows).
__global__ void __launch_bounds__(256) draft_embed_norm_cat_kernel(
    const uint16_t* __restrict__ embed, int64_t V, int H, const int64_t* __restrict__ tokens, int64_t tok_stride,
    int64_t index, const uint16_t* __restrict__ enorm, const uint16_t* __restrict__ hidden, int64_t hidden_stride,
    const uint16_t* __restrict__ hnorm, float eps, uint16_t* __restrict__ out, int64_t out_stride) {
    pdl_launch_dependents();
    __shared__ float red[8];
    const size_t b = blockIdx.y;
    uint16_t* o = out + b * out_stride;
    if (blockIdx.x == 0) {
        int64_t tok = tokens[b * tok_stride + index];
        if (tok < 0 || tok >= V) {
            if (threadIdx.x == 0) set_device_error(DEV_BAD_TOKEN);
            tok = 0;
        }
        rmsnorm_row(embed + size_t(tok) * H, nullptr, enorm, eps, H, o, nullptr, red);
    } else {
        rmsnorm_row(hidden + b * hidden_stride, nullptr, hnorm, eps, H, o + H, nullptr, red);
    }
}

__global__ void __launch_bounds__(256) lut_mul_kernel(const uint16_t* __restrict__ a, int64_t a_stride,
                                                      const uint16_t* __restrict__ b, int64_t b_stride,
                                                      int64_t b_head_stride, const uint16_t* __restrict__ lut, int K,
                                                      uint16_t* __restrict__ out, int64_t out_stride) {
    pdl_launch_dependents();  // an ordinary launch: its inputs are complete; the next kernel may start
    const int m = blockIdx.y;
    const int c0 = (blockIdx.x * 256 + threadIdx.x) * 8;
    if (c0 >= K) return;
    const uint4 av = __ldg(reinterpret_cast<const uint4*>(a + size_t(m) * a_stride + c0));
    const uint4 bv = __ldg(reinterpret_cast<const uint4*>(b + size_t(m) * b_stride + (c0 >> 8) * b_head_stride + (c0 & 255)));
    const uint32_t au[4] = {av.x, av.y, av.z, av.w}, bu[4] = {bv.x, bv.y, bv.z, bv.w};
    uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
    for (int e = 0; e < 8; ++e) {
        const uint32_t ab = (e & 1) ? (au[e >> 1] >> 16) : (au[e >> 1] & 0xFFFFu);
        const uint32_t bb = (e & 1) ? (bu[e >> 1] >> 16) : (bu[e >> 1] & 0xFFFFu);
        const float f = __fmul_rn(bf16_bits_to_f32(uint16_t(ab)), bf16_bits_to_f32(__ldg(lut + bb)));
        o[e >> 1] |= uint32_t(f32_to_bf16_bits(f)) << (16 * (e & 1));
    }
    reinterpret_cast<uint4*>(out + size_t(m) * out_stride + c0)[0] = make_uint4(o[0], o[1], o[2], o[3]);
}

}  // namespace mono

using namespace mono;

extern "C" {

int mono_rmsnorm_add(const void* x, int64_t x_stride, const void* add, int64_t add_stride, const void* w, float eps,
                     int64_t M, int64_t H, void* out, void* sum_out, int64_t out_stride, mono_stream_t stream) {
    MONO_CHECK(x && w && out && (sum_out || !add) && (!sum_out || add), "null operand (sum_out goes with add)");
    MONO_CHECK(M >= 1 && M <= 65535 && H >= 8 && H % 8 == 0 && eps > 0.f, "1 <= M <= 65535, H a multiple of 8");
    MONO_CHECK(x_stride % 8 == 0 && add_stride % 8 == 0 && out_stride % 8 == 0 && x_stride >= H && out_stride >= H,
               "row strides: multiples of 8 elements covering H");
    const void* ptrs[] = {x, w, out};
    for (const void* p : ptrs) MONO_CHECK(aligned(p, 16), "16-byte aligned rows");
    MONO_CHECK((!add || aligned(add, 16)) && (!sum_out || aligned(sum_out, 16)), "16-byte aligned rows");
    rmsnorm_add_kernel<<<int(M), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(add), static_cast<const uint16_t*>(w), eps, int(H),
        x_stride, add_stride, out_stride, static_cast<uint16_t*>(out), static_cast<uint16_t*>(sum_out));
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

int mono_draft_embed_norm_cat(const void* embed, int64_t V, int64_t H, const int64_t* tokens, int64_t tok_stride,
                              int64_t index, const void* enorm_w, const void* hidden, int64_t hidden_stride,
                              const void* hnorm_w, float eps, int64_t B, void* out, int64_t out_stride,
                              mono_stream_t stream) {
    MONO_CHECK(embed && tokens && enorm_w && hidden && hnorm_w && out, "null operand");
    MONO_CHECK(B >= 1 && B <= 65535 && V >= 1 && H >= 8 && H % 8 == 0 && eps > 0.f, "1 <= B, V >= 1, H a multiple of 8");
    MONO_CHECK(index >= 0 && tok_stride >= 0 && hidden_stride % 8 == 0 && hidden_stride >= H && out_stride % 8 == 0 &&
                   out_stride >= 2 * H,
               "index >= 0; row strides multiples of 8 covering H (hidden) and 2 H (out)");
    const void* ptrs[] = {embed, enorm_w, hidden, hnorm_w, out};
    for (const void* p : ptrs) MONO_CHECK(aligned(p, 16), "16-byte aligned rows");
    MONO_CHECK(aligned(tokens, 8), "aligned token ids");
    draft_embed_norm_cat_kernel<<<dim3(2, unsigned(B)), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(embed), V, int(H), tokens, tok_stride, index, static_cast<const uint16_t*>(enorm_w),
        static_cast<const uint16_t*>(hidden), hidden_stride, static_cast<const uint16_t*>(hnorm_w), eps,
        static_cast<uint16_t*>(out), out_stride);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

int mono_lut_mul(const void* a, int64_t a_stride, const void* b, int64_t b_stride, int64_t b_head_stride, const void* lut,
                 int64_t M, int64_t K, void* out, int64_t out_stride, mono_stream_t stream) {
    MONO_CHECK(a && b && lut && out, "null operand");
    MONO_CHECK(M >= 1 && M <= 65535 && K >= 8 && K % 8 == 0, "1 <= M <= 65535, K a multiple of 8");
    MONO_CHECK(a_stride % 8 == 0 && b_stride % 8 == 0 && b_head_stride % 8 == 0 && out_stride % 8 == 0 &&
                   b_head_stride >= 256 && a_stride >= K && out_stride >= K,
               "strides: multiples of 8 elements, head stride >= 256");
    MONO_CHECK(aligned(a, 16) && aligned(b, 16) && aligned(out, 16), "16-byte aligned rows");
    lut_mul_kernel<<<dim3(unsigned((K / 8 + 255) / 256), unsigned(M)), 256, 0, reinterpret_cast<cudaStream_t>(stream)>>>(
        static_cast<const uint16_t*>(a), a_stride, static_cast<const uint16_t*>(b), b_stride, b_head_stride,
        static_cast<const uint16_t*>(lut), int(K), static_cast<uint16_t*>(out), out_stride);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

}  // extern "C"
