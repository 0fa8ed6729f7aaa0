// Gated-DeltaNet decode step (the core of the reference's layer_gdn P3-P5, csrc/mono_gdn.sycl:313-611).
//
// Two forms. Committing (ctl == null): M sequential rows, each advancing the recurrent and conv state, which
// are written back. Deferred (ctl != null; the reference's replay + verify, :385-567): the n = ctl[0] rows
// accepted at the previous step (slots ctl[2 + i], inputs saved by that step) are replayed first and their
// states persisted; then the M verify rows of this step run as a chain on a register copy (outputs only,
// nothing persisted); their inputs are saved for the next step's replay. The conv state advances by the
// replayed rows only.
//
// Kernel 1 (one thread per qkv channel): the depthwise causal conv of width 4, y = bf16(fma chain x[t] w[3],
// x[t-1] w[2], .. from 0), out = bf16(y / (1 + exp(-y))), over the conv state (3 newest inputs, oldest
// first) and the replayed then the verify rows. Threads < (n + M) * HV make the gates:
// decay = exp(g_decay * softplus(a + dt_bias)) (softplus(v) = v above 20), beta = bf16(sigmoid(b)).
// Kernel 2 (one CTA per value head, 512 threads = 4 row groups x 128 value columns; thread (rg, col) keeps
// state rows rg * 32 .. rg * 32 + 31 of column col in registers): L2 norms of q and k of the key head
// (qi = 1 / max(sqrt(sum), 1e-12), q <- (q * scale) * qi, k <- k * ki), then per row in order
//   S <- S * decay;  mem = S^T k;  delta = (v - mem) * beta;  S <- S + k delta^T;  o = S^T q
// (fma chains over each row group's 32 rows, the 4 group partials summed in order), raw = bf16(o); the
// gated RMSNorm core = bf16(bf16(raw * w * rsqrt(mean(raw^2) + eps)) * bf16(silu(z))). fp32 throughout;
// results are checked against an fp64 reference with a stated tolerance.
#include <cmath>

#include "launch.h"

namespace mono {

constexpr int kDH = 128, kRG = 4, kRPG = kDH / kRG, kGdnMaxRows = 8, kGdnMaxAll = 2 * kGdnMaxRows;

__device__ __forceinline__ int gdn_pending(const GdnArgs& A) {
    if (A.ctl == nullptr) return 0;
    const int n = A.ctl[0];
    return n < 0 ? 0 : (n > kGdnMaxRows ? kGdnMaxRows : n);
}
__device__ __forceinline__ int gdn_slot(const GdnArgs& A, int i) {
    const int s = A.ctl[2 + i];
    return s < 0 ? 0 : (s >= kGdnMaxRows ? kGdnMaxRows - 1 : s);
}

__global__ void __launch_bounds__(256) gdn_conv_kernel(const GdnArgs A) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    const int n = gdn_pending(A), R = n + A.M;
    if (i < R * A.HV) {  // gates of every row (replayed rows: from the saved a / b)
        const int t = i / A.HV, h = i % A.HV;
        const uint16_t ab = t < n ? A.prev_a[size_t(gdn_slot(A, t)) * A.HV + h] : A.a[size_t(t - n) * A.ab_stride + h];
        const uint16_t bb = t < n ? A.prev_b[size_t(gdn_slot(A, t)) * A.HV + h] : A.b[size_t(t - n) * A.ab_stride + h];
        const float av = bf16_bits_to_f32(ab) + A.dt_bias[h];
        const float sp = av > 20.f ? av : logf(1.f + expf(av));
        A.gates[i * 2] = expf(A.g_decay[h] * sp);
        A.gates[i * 2 + 1] = bf16_round(1.f / (1.f + expf(-bf16_bits_to_f32(bb))));
    }
    if (A.save_a != nullptr && i < A.M * A.HV) {
        const int t = i / A.HV, h = i % A.HV;
        A.save_a[i] = A.a[size_t(t) * A.ab_stride + h];
        A.save_b[i] = A.b[size_t(t) * A.ab_stride + h];
    }
    if (i >= A.C) return;
    float w[4], hist[3 + kGdnMaxAll];
#pragma unroll
    for (int d = 0; d < 4; ++d) w[d] = bf16_bits_to_f32(A.conv_w[size_t(i) * 4 + d]);
#pragma unroll
    for (int r = 0; r < 3; ++r) hist[r] = bf16_bits_to_f32(A.conv_state[size_t(i) * 3 + r]);
#pragma unroll
    for (int t = 0; t < kGdnMaxAll; ++t) {
        if (t < n) hist[3 + t] = bf16_bits_to_f32(A.prev_qkv[size_t(gdn_slot(A, t)) * A.C + i]);
        else if (t < R) {
            const uint16_t v = A.qkv[size_t(t - n) * A.qkv_stride + i];
            hist[3 + t] = bf16_bits_to_f32(v);
            if (A.save_qkv != nullptr) A.save_qkv[size_t(t - n) * A.C + i] = v;
        }
    }
#pragma unroll
    for (int t = 0; t < kGdnMaxAll; ++t) {
        if (t >= R) break;
        float sum = 0.f;
#pragma unroll
        for (int d = 0; d < 4; ++d) sum = fmaf(hist[3 + t - d], w[3 - d], sum);
        const float y = bf16_round(sum);
        A.conv_out[size_t(t) * A.C + i] = f32_to_bf16_bits(y / (1.f + expf(-y)));
    }
    // the state becomes the three newest committed inputs (oldest first): the replayed rows in the deferred
    // form, all rows in the committing form
    const int keep = A.ctl != nullptr ? n : R;
#pragma unroll
    for (int r = 0; r < 3; ++r) {
        float v = hist[r];
#pragma unroll
        for (int t = 0; t < kGdnMaxAll + 3; ++t)
            if (t == keep + r) v = hist[t];
        A.conv_state[size_t(i) * 3 + r] = f32_to_bf16_bits(v);
    }
}

__global__ void __launch_bounds__(kRG * kDH) gdn_delta_kernel(const GdnArgs A) {
    __shared__ float qn[kGdnMaxAll][kDH], kn[kGdnMaxAll][kDH];
    __shared__ float part[2][kRG][kDH];
    __shared__ float raw[kGdnMaxRows][kDH];
    __shared__ float sums[2 * kGdnMaxAll];
    const int h = blockIdx.x, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rg = tid / kDH, col = tid % kDH;
    const int kh = h / (A.HV / A.HK), KD = A.HK * kDH, M = A.M;
    const int n = gdn_pending(A), R = n + M;
    // sums of squares of q and k of the key head per row: (row, q or k) pairs over the 16 warps
    for (int pr = warp; pr < 2 * R; pr += 16) {
        const int t = pr >> 1, which = pr & 1;
        const uint16_t* src = A.conv_out + size_t(t) * A.C + which * KD + kh * kDH;
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const float v = bf16_bits_to_f32(src[lane + 32 * j]);
            s = fmaf(v, v, s);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) sums[pr] = s;
    }
    __syncthreads();
    for (int e = tid; e < R * kDH; e += blockDim.x) {
        const int t = e / kDH, d = e % kDH;
        const float qi = 1.f / fmaxf(sqrtf(sums[2 * t]), 1e-12f), ki = 1.f / fmaxf(sqrtf(sums[2 * t + 1]), 1e-12f);
        qn[t][d] = (bf16_bits_to_f32(A.conv_out[size_t(t) * A.C + kh * kDH + d]) * A.qscale) * qi;
        kn[t][d] = bf16_bits_to_f32(A.conv_out[size_t(t) * A.C + KD + kh * kDH + d]) * ki;
    }
    float st[kRPG];
    float* S = A.state + (size_t(h) * kDH + rg * kRPG) * kDH + col;
#pragma unroll
    for (int r = 0; r < kRPG; ++r) st[r] = S[size_t(r) * kDH];
    __syncthreads();
    for (int t = 0; t < R; ++t) {
        const float decay = A.gates[(t * A.HV + h) * 2], beta = A.gates[(t * A.HV + h) * 2 + 1];
        const float v = bf16_bits_to_f32(A.conv_out[size_t(t) * A.C + 2 * KD + h * kDH + col]);
        float mem = 0.f;
#pragma unroll
        for (int r = 0; r < kRPG; ++r) {
            st[r] *= decay;
            mem = fmaf(st[r], kn[t][rg * kRPG + r], mem);
        }
        part[0][rg][col] = mem;
        __syncthreads();
        const float kv = part[0][0][col] + part[0][1][col] + part[0][2][col] + part[0][3][col];
        const float delta = (v - kv) * beta;
        float o = 0.f;
#pragma unroll
        for (int r = 0; r < kRPG; ++r) {
            st[r] = fmaf(kn[t][rg * kRPG + r], delta, st[r]);
            o = fmaf(st[r], qn[t][rg * kRPG + r], o);
        }
        part[1][rg][col] = o;
        __syncthreads();
        if (rg == 0 && t >= n) raw[t - n][col] = bf16_round(part[1][0][col] + part[1][1][col] + part[1][2][col] + part[1][3][col]);
        if (A.ctl != nullptr && t == n - 1)  // the committed state after the replay
#pragma unroll
            for (int r = 0; r < kRPG; ++r) S[size_t(r) * kDH] = st[r];
    }
    if (A.ctl == nullptr)
#pragma unroll
        for (int r = 0; r < kRPG; ++r) S[size_t(r) * kDH] = st[r];
    __syncthreads();
    // gated RMSNorm of every output row: warp w < M sums row w's squares
    if (warp < M) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) s += raw[warp][lane + 32 * j] * raw[warp][lane + 32 * j];
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) sums[warp] = s;
    }
    __syncthreads();
    for (int e = tid; e < M * kDH; e += blockDim.x) {
        const int t = e / kDH, d = e % kDH;
        const float rs = 1.f / sqrtf(sums[t] / float(kDH) + A.gnorm_eps);
        const float normed = bf16_round((raw[t][d] * bf16_bits_to_f32(A.gnorm_w[d])) * rs);
        const float z = bf16_bits_to_f32(A.z[size_t(t) * A.z_stride + h * kDH + d]);
        const float gz = bf16_round(z / (1.f + expf(-z)));
        A.core[size_t(t) * A.HV * kDH + h * kDH + d] = f32_to_bf16_bits(normed * gz);
    }
}

size_t gdn_workspace_bytes(int M, int C, int HV) {
    // conv outputs and gates of up to 8 replayed rows + the M verify rows
    const size_t rows = size_t(M) + kGdnMaxRows;
    return (rows * C * 2 + 255) / 256 * 256 + rows * HV * 2 * 4;
}

int launch_gdn_step(GdnArgs A, void* ws, cudaStream_t stream) {
    const size_t rows = size_t(A.M) + kGdnMaxRows;
    A.conv_out = static_cast<uint16_t*>(ws);
    A.gates = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + (rows * A.C * 2 + 255) / 256 * 256);
    const int rmax = int(rows);
    const int nthreads = A.C > rmax * A.HV ? A.C : rmax * A.HV;
    gdn_conv_kernel<<<(nthreads + 255) / 256, 256, 0, stream>>>(A);
    CUDA_TRY(cudaGetLastError());
    gdn_delta_kernel<<<A.HV, kRG * kDH, 0, stream>>>(A);
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

}  // namespace mono
