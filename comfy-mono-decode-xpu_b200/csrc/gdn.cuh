// Gated-DeltaNet pieces shared by the standalone GDN kernels (gdn.cu) and the layer programs (program.cu), so
// both run the same floating-point operations in the same order (results agree bit for bit).
// Reference: csrc/mono_gdn.sycl:313-611 (deferred conv, gates, sums, replay + verify delta, gated RMSNorm).
#pragma once
#include "launch.h"
#include "rowops.cuh"

namespace mono {

// kRG row groups of the 128 key rows (kRPG rows each): a delta-rule thread keeps kRPG state rows of one value column
// in registers; S^T k and S^T q are fma chains over a group's rows, the kRG group partials summed in group order.
constexpr int kDH = 128, kRG = 8, kRPG = kDH / kRG, kGdnMaxRows = 8, kGdnMaxAll = 2 * kGdnMaxRows;

// The conv and gated-norm SiLU: bf16(y / (1 + exp(-y))) of a bf16 value y, fp32 arithmetic, evaluated in place
// (a table lookup would put a dependent global load behind every output).
__device__ __forceinline__ float gdn_silu_formula(float y) { return y / (1.f + expf(-y)); }
__device__ __forceinline__ uint16_t gdn_silu_bits(float y_bf16) { return f32_to_bf16_bits(gdn_silu_formula(y_bf16)); }
__device__ __forceinline__ float gdn_silu(float y_bf16) { return bf16_bits_to_f32(gdn_silu_bits(y_bf16)); }

// ctl (deferred form) = [pending, parity, accepted slots[8], parents[8], program[8]] (csrc/mono_gdn.sycl:38-40).
// parent(t) of verify row t: a row before it, or -1 (the root's parent; anything else reads as -1). Without ctl (the
// committing form) the rows are a chain.
__device__ __forceinline__ int gdn_parent(const GdnArgs& A, int t) {
    if (A.ctl == nullptr) return t - 1;
    const int p = __ldcg(A.ctl + 2 + kGdnMaxRows + t);
    return p >= 0 && p < t ? p : -1;
}
// Verify entries of the step: the program's words p = slot | 32 * commit, up to the first one whose slot is outside
// [0, M) (the committing form: every row in order, each committing).
__device__ __forceinline__ int gdn_verify_entries(const GdnArgs& A) {
    if (A.ctl == nullptr) return A.M;
    int e = 0;
    while (e < kGdnMaxRows) {
        const int p = __ldcg(A.ctl + 2 + 2 * kGdnMaxRows + e);
        if (p < 0 || (p & 15) >= A.M) break;
        ++e;
    }
    return e;
}
// Entry e of the step's list (replayed rows first: e < n): its conv-output row, its output slot (-1: none) and
// whether it advances the running state.
struct GdnEntry {
    int row, out;
    bool commit;
};
__device__ __forceinline__ GdnEntry gdn_entry(const GdnArgs& A, int n, int e) {
    if (e < n) return GdnEntry{e, -1, true};
    if (A.ctl == nullptr) return GdnEntry{e, e, true};
    const int p = __ldcg(A.ctl + 2 + 2 * kGdnMaxRows + (e - n));
    return GdnEntry{n + (p & 15), p & 15, (p & 32) != 0};
}

// The same accessors over a shared-memory copy of the ctl words (gdn_ctl_stage, then a barrier): for kernels that
// walk the entries one after another, so that no entry waits for a global load.
constexpr int kGdnCtlWords = 2 + 3 * kGdnMaxRows;
__device__ __forceinline__ void gdn_ctl_stage(const GdnArgs& A, int* cs) {
    if (A.ctl != nullptr && threadIdx.x < kGdnCtlWords) cs[threadIdx.x] = __ldcg(A.ctl + threadIdx.x);
}
__device__ __forceinline__ int gdn_pending_s(const GdnArgs& A, const int* cs) {
    if (A.ctl == nullptr) return 0;
    const int n = cs[0];
    return n < 0 ? 0 : (n > kGdnMaxRows ? kGdnMaxRows : n);
}
__device__ __forceinline__ int gdn_verify_entries_s(const GdnArgs& A, const int* cs) {
    if (A.ctl == nullptr) return A.M;
    int e = 0;
    while (e < kGdnMaxRows) {
        const int p = cs[2 + 2 * kGdnMaxRows + e];
        if (p < 0 || (p & 15) >= A.M) break;
        ++e;
    }
    return e;
}
__device__ __forceinline__ GdnEntry gdn_entry_s(const GdnArgs& A, const int* cs, int n, int e) {
    if (e < n) return GdnEntry{e, -1, true};
    if (A.ctl == nullptr) return GdnEntry{e, e, true};
    const int p = cs[2 + 2 * kGdnMaxRows + (e - n)];
    return GdnEntry{n + (p & 15), p & 15, (p & 32) != 0};
}

__device__ __forceinline__ int gdn_pending(const GdnArgs& A) {
    if (A.ctl == nullptr) return 0;
    const int n = __ldcg(A.ctl);
    return n < 0 ? 0 : (n > kGdnMaxRows ? kGdnMaxRows : n);
}
__device__ __forceinline__ int gdn_slot(const GdnArgs& A, int i) {
    const int s = __ldcg(A.ctl + 2 + i);
    return s < 0 ? 0 : (s >= kGdnMaxRows ? kGdnMaxRows - 1 : s);
}

// a[i] of a small register array at a run-time index, as a select chain (no local-memory indexing)
template <int N>
__device__ __forceinline__ float pick(const float (&a)[N], int i) {
    float v = a[0];
#pragma unroll
    for (int k = 1; k < N; ++k) v = i == k ? a[k] : v;
    return v;
}

// Work item i of the conv step (one thread each, i < max(C, (n + M) * HV)): the gates of (row, head) i, the
// saved a / b of this step's rows, and the depthwise causal conv of channel i:
//   gates: decay = exp(g_decay * softplus(a + dt_bias)) (softplus(v) = v above 20), beta = bf16(sigmoid(b))
//   conv:  y = bf16(fma chain x[t] w[3], x[t-1] w[2], .. from 0), out = bf16(y / (1 + exp(-y)))
// The replayed rows run as a chain over the conv state (an accepted path: each row's predecessors are the rows
// before it); verify row t reads its own input, then its ancestors' (gdn_parent), then the committed history (the
// conv state after the replay), newest first (csrc/mono_gdn.sycl:313-375). The conv state becomes the three
// newest committed inputs (the replayed rows in the deferred form, all rows in the committing form). All
// activations are read through L2 (they may have been written by this launch).
// PDL (a launch with programmatic dependency): the inputs no recent kernel writes (ctl words, the replay rows
// saved by the previous step, conv weights and state, gate parameters) are loaded before griddepcontrol.wait,
// this step's rows (qkv, a, b) after it.
template <bool PDL = false>
__device__ __forceinline__ void gdn_conv_item(const GdnArgs& A, int i) {
    // Loads in two round trips: the ctl words (pending count, slots, parents), then every input this item reads;
    // no store before the last load (a load after a store the compiler cannot prove disjoint waits for it).
    int n = 0, slot[kGdnMaxRows], par[kGdnMaxRows];
    if (A.ctl != nullptr) {
        int raw_n = __ldcg(A.ctl), raw_s[kGdnMaxRows], raw_p[kGdnMaxRows];
#pragma unroll
        for (int t = 0; t < kGdnMaxRows; ++t) {
            raw_s[t] = __ldcg(A.ctl + 2 + t);
            raw_p[t] = __ldcg(A.ctl + 2 + kGdnMaxRows + t);
        }
        n = raw_n < 0 ? 0 : (raw_n > kGdnMaxRows ? kGdnMaxRows : raw_n);
#pragma unroll
        for (int t = 0; t < kGdnMaxRows; ++t) {
            slot[t] = raw_s[t] < 0 ? 0 : (raw_s[t] >= kGdnMaxRows ? kGdnMaxRows - 1 : raw_s[t]);
            par[t] = t < A.M && raw_p[t] >= 0 && raw_p[t] < t ? raw_p[t] : -1;  // gdn_parent
        }
    } else {
#pragma unroll
        for (int t = 0; t < kGdnMaxRows; ++t) {
            slot[t] = 0;
            par[t] = t < A.M ? t - 1 : -1;
        }
    }
    const int R = n + A.M;
    const bool saving = A.save_a != nullptr && i < A.M * A.HV;
    const bool gating = i < R * A.HV;
    const bool conv = i < A.C;
    uint16_t sa = 0, sb = 0, ab = 0, bb = 0;
    float dtb = 0.f, gdec = 0.f;
    const int gt = i / A.HV, gh = i % A.HV;  // gating / saving: row gt, value head gh
    if (gating) {
        int st = 0;
#pragma unroll
        for (int u = 0; u < kGdnMaxRows; ++u)
            if (u == gt) st = slot[u];
        if (gt < n) {
            ab = __ldcg(A.prev_a + size_t(st) * A.HV + gh);
            bb = __ldcg(A.prev_b + size_t(st) * A.HV + gh);
        }
        dtb = A.dt_bias[gh];
        gdec = A.g_decay[gh];
    }
    uint16_t rp[kGdnMaxRows], rv[kGdnMaxRows];  // raw inputs of the replayed rows / of the verify rows
    float w[4], hist[3 + kGdnMaxRows], vr[kGdnMaxRows];
    if (conv) {
#pragma unroll
        for (int t = 0; t < kGdnMaxRows; ++t) rp[t] = t < n ? __ldcg(A.prev_qkv + size_t(slot[t]) * A.C + i) : uint16_t(0);
#pragma unroll
        for (int d = 0; d < 4; ++d) w[d] = bf16_bits_to_f32(A.conv_w[size_t(i) * 4 + d]);
#pragma unroll
        for (int r = 0; r < 3; ++r) hist[r] = bf16_bits_to_f32(A.conv_state[size_t(i) * 3 + r]);
    }
    if constexpr (PDL) {
        pdl_wait();  // this step's rows: written by the preceding kernels
        pdl_launch_dependents();  // after the wait: a dependent's early reads never see this kernel's inputs change
    }
    if (saving) {
        sa = __ldcg(A.a + size_t(gt) * A.ab_stride + gh);
        sb = __ldcg(A.b + size_t(gt) * A.ab_stride + gh);
    }
    if (gating && gt >= n) {
        ab = __ldcg(A.a + size_t(gt - n) * A.ab_stride + gh);
        bb = __ldcg(A.b + size_t(gt - n) * A.ab_stride + gh);
    }
    if (conv)
#pragma unroll
        for (int t = 0; t < kGdnMaxRows; ++t) rv[t] = t < A.M ? __ldcg(A.qkv + size_t(t) * A.qkv_stride + i) : uint16_t(0);
    if (gating) {
        const float av = bf16_bits_to_f32(ab) + dtb;
        const float sp = av > 20.f ? av : logf(1.f + expf(av));
        A.gates[i * 2] = expf(gdec * sp);
        A.gates[i * 2 + 1] = bf16_round(1.f / (1.f + expf(-bf16_bits_to_f32(bb))));
    }
    if (saving) {
        A.save_a[i] = sa;
        A.save_b[i] = sb;
    }
    if (!conv) return;
    if (A.save_qkv != nullptr)
#pragma unroll
        for (int t = 0; t < kGdnMaxRows; ++t)
            if (t < A.M) A.save_qkv[size_t(t) * A.C + i] = rv[t];
    // replayed rows: a chain over the conv state; hist[3 + t] = input of replayed row t
#pragma unroll
    for (int t = 0; t < kGdnMaxRows; ++t) {
        hist[3 + t] = bf16_bits_to_f32(rp[t]);
        if (t < n) {
            float sum = 0.f;
#pragma unroll
            for (int d = 0; d < 4; ++d) sum = fmaf(hist[3 + t - d], w[3 - d], sum);
            const float y = bf16_round(sum);
            A.conv_out[size_t(t) * A.C + i] = gdn_silu_bits(y);
        }
    }
    // the committed window after the replay: the three newest of (conv state, replayed inputs), oldest first
    float win[3];
#pragma unroll
    for (int r = 0; r < 3; ++r) {
        float v = hist[r];
#pragma unroll
        for (int t = 1; t < 3 + kGdnMaxRows; ++t)
            if (t == n + r) v = hist[t];
        win[r] = v;
    }
    // verify rows: own input, then the ancestors' inputs, then the committed window (newest first)
#pragma unroll
    for (int t = 0; t < kGdnMaxRows; ++t) vr[t] = bf16_bits_to_f32(rv[t]);
#pragma unroll
    for (int t = 0; t < kGdnMaxRows; ++t) {
        if (t >= A.M) break;
        float sum = fmaf(vr[t], w[3], 0.f);
        int anc = t, miss = 0;
#pragma unroll
        for (int d = 1; d < 4; ++d) {
            int pa = -1;
#pragma unroll
            for (int u = 0; u < kGdnMaxRows; ++u)
                if (u == anc) pa = par[u];
            anc = anc >= 0 ? pa : -1;
            miss += anc < 0;
            const float v = anc >= 0 ? pick(vr, anc) : (miss == 1 ? win[2] : (miss == 2 ? win[1] : win[0]));
            sum = fmaf(v, w[3 - d], sum);
        }
        const float y = bf16_round(sum);
        A.conv_out[size_t(n + t) * A.C + i] = gdn_silu_bits(y);
    }
    // the new conv state: the committed window (deferred form), or the three newest of (conv state, all M rows)
    // (committing form, n = 0: sequence position M + r, oldest first)
#pragma unroll
    for (int r = 0; r < 3; ++r) {
        float v = win[r];
        if (A.ctl == nullptr) {
            v = hist[r];
#pragma unroll
            for (int k = 1; k < 3; ++k)
                if (A.M + r == k) v = hist[k];
#pragma unroll
            for (int t = 0; t < kGdnMaxRows; ++t)
                if (A.M + r == t + 3) v = vr[t];
        }
        A.conv_state[size_t(i) * 3 + r] = f32_to_bf16_bits(v);
    }
}

// Sum of squares of 128 bf16 values by one warp: lane l takes elements l + 32 j (j = 0..3) in order (fma chain
// from 0), then the xor butterfly (16, 8, 4, 2, 1).
__device__ __forceinline__ float gdn_sumsq128(const uint16_t* src, int lane) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < 4; ++j) {
        const float v = bf16_bits_to_f32(__ldcg(src + lane + 32 * j));
        s = fmaf(v, v, s);
    }
#pragma unroll
    for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
    return s;
}
__device__ __forceinline__ float gdn_l2_inv(float sumsq) { return 1.f / fmaxf(sqrtf(sumsq), 1e-12f); }

// Gated RMSNorm of one head of a raw output row: r = 1 / sqrt(sum(raw^2) / 128 + eps) (sum as gdn_sumsq128 over
// the bf16 raw values), core = bf16(bf16((raw * w) * r) * bf16(silu(z))).
__device__ __forceinline__ float gdn_norm_inv(float sumsq, float eps) { return 1.f / sqrtf(sumsq / float(kDH) + eps); }
__device__ __forceinline__ uint16_t gdn_core(float raw, float w, float r, float z) {
    const float normed = bf16_round((raw * w) * r);
    return f32_to_bf16_bits(normed * gdn_silu(z));  // z is a bf16 value
}

// a | b projection (the role of the reference's in_proj_a / in_proj_b BF16 linear, csrc/mono_gdn.sycl:10-11), in
// this build's pinned fp32 order, every product and sum rounded on its own (no fma):
//   column n's K range is cut into 4 quarters of K / 1024 slices of 256; for quarter q, lane l of 32 sums
//   x[m][k] * w[n][k] over its 8-element pieces l + 32 j (j ascending over the quarter's slices, elements in
//   order) from +0, then the xor butterfly (16, 8, 4, 2, 1) gives Q_q;  out[m][n] = bf16(((Q_0 + Q_1) + Q_2) + Q_3).
// One warp per (column, quarter): its weight pieces (<= 4 per lane) are all in flight at once; x [M][K] is read
// from shared memory. K % 1024 == 0, K <= 4096, M <= 16.
// The quarter's weight pieces of column n (issued before anything waits on them).
__device__ __forceinline__ void gdn_ab_load_w(const uint16_t* __restrict__ w, int K, int n, int q, int lane, uint4 (&wv)[4]) {
    const int J4 = K >> 10;
    const uint4* wr = reinterpret_cast<const uint4*>(w + size_t(n) * K) + 32 * (q * J4) + lane;
#pragma unroll
    for (int j = 0; j < 4; ++j)
        if (j < J4) wv[j] = __ldg(wr + 32 * j);
}
// Rows m0, m0 + mstep, .. < M of xs (row stride K); qsum[m] = the quarter sum of row m.
__device__ __forceinline__ void gdn_ab_quarter(const uint16_t* __restrict__ xs, const uint4 (&wv)[4], int K, int M, int q,
                                               int lane, float* qsum, int m0 = 0, int mstep = 1) {
    const int J4 = K >> 10;
#pragma unroll 1
    for (int m = m0; m < M; m += mstep) {
        const uint4* xr = reinterpret_cast<const uint4*>(xs + size_t(m) * K) + 32 * (q * J4) + lane;
        float acc = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j)
            if (j < J4) {
                const uint4 xv = xr[32 * j];
                const uint32_t xu[4] = {xv.x, xv.y, xv.z, xv.w}, wu[4] = {wv[j].x, wv[j].y, wv[j].z, wv[j].w};
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    const float a = __uint_as_float((e & 1) ? (xu[e >> 1] & 0xFFFF0000u) : (xu[e >> 1] << 16));
                    const float b = __uint_as_float((e & 1) ? (wu[e >> 1] & 0xFFFF0000u) : (wu[e >> 1] << 16));
                    acc = __fadd_rn(acc, __fmul_rn(a, b));
                }
            }
#pragma unroll
        for (int o = 16; o; o >>= 1) acc = __fadd_rn(acc, __shfl_xor_sync(0xffffffffu, acc, o));
        if (lane == 0) qsum[m] = acc;
    }
}
// out[m][n] from the four quarter sums of one column (qs[q * stride + m]).
__device__ __forceinline__ uint16_t gdn_ab_combine(const float* qs, int stride, int m) {
    return f32_to_bf16_bits(
        __fadd_rn(__fadd_rn(__fadd_rn(qs[m], qs[stride + m]), qs[2 * stride + m]), qs[3 * stride + m]));
}

// Gated RMSNorm of every head of one raw row (K = heads * 128 <= 4096) and the row's per-token quantization, by
// one warp-group: warp w takes heads w, w + 4, .. for the norm factors (gdn_sumsq128, gdn_norm_inv); thread t
// then forms core = gdn_core(..) for its 8-element pieces t + 128 j and quantizes them (rowops.cuh order).
// core_out (optional): the core row. hs: >= 32 floats of the warp-group's shared memory.
__device__ __forceinline__ void gdn_norm_quant_row(const uint16_t* __restrict__ raw, const uint16_t* __restrict__ z,
                                                   const uint16_t* __restrict__ w, float eps, int K,
                                                   uint16_t* __restrict__ core_out, int8_t* __restrict__ q,
                                                   float* __restrict__ s_out, float* red, float* hs, int tig, int wg) {
    const int lane = tig & 31, warp = tig >> 5, J = K >> 10, nh = K >> 7;
    {
        // every head's values loaded before any sum (8 heads per warp at most)
        float v[8][4];
#pragma unroll
        for (int i = 0; i < 8; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                v[i][j] = warp + 4 * i < nh ? bf16_bits_to_f32(__ldcg(raw + (warp + 4 * i) * kDH + lane + 32 * j)) : 0.f;
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) ss = fmaf(v[i][j], v[i][j], ss);
#pragma unroll
            for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0 && warp + 4 * i < nh) hs[warp + 4 * i] = gdn_norm_inv(ss, eps);
        }
    }
    wg_sync(wg);
    uint32_t cw[kRowMaxPieces][4];  // the core values, bf16 pairs
    float amax = 0.f;
#pragma unroll
    for (int j = 0; j < kRowMaxPieces; ++j)
        if (j < J) {
            const int c0 = (tig + 128 * j) * 8, h = c0 / kDH, d0 = c0 % kDH;
            const uint4 rv = __ldcg(reinterpret_cast<const uint4*>(raw + c0));
            const uint4 zv = __ldcg(reinterpret_cast<const uint4*>(z + c0));
            const uint4 wv = __ldg(reinterpret_cast<const uint4*>(w + d0));
            const uint32_t ru[4] = {rv.x, rv.y, rv.z, rv.w}, zu[4] = {zv.x, zv.y, zv.z, zv.w}, wu[4] = {wv.x, wv.y, wv.z, wv.w};
            const float r = hs[h];
#pragma unroll
            for (int p = 0; p < 4; ++p) {
                const uint16_t lo = gdn_core(__uint_as_float(ru[p] << 16), __uint_as_float(wu[p] << 16), r,
                                             __uint_as_float(zu[p] << 16));
                const uint16_t hi = gdn_core(__uint_as_float(ru[p] & 0xFFFF0000u), __uint_as_float(wu[p] & 0xFFFF0000u), r,
                                             __uint_as_float(zu[p] & 0xFFFF0000u));
                cw[j][p] = uint32_t(lo) | (uint32_t(hi) << 16);
                amax = fmaxf(amax, fmaxf(fabsf(bf16_bits_to_f32(lo)), fabsf(bf16_bits_to_f32(hi))));
            }
            if (core_out) reinterpret_cast<uint4*>(core_out)[tig + 128 * j] = make_uint4(cw[j][0], cw[j][1], cw[j][2], cw[j][3]);
        }
#pragma unroll
    for (int o = 16; o; o >>= 1) amax = fmaxf(amax, __shfl_xor_sync(0xffffffffu, amax, o));
    if (lane == 0) red[8 + warp] = amax;
    wg_sync(wg);
    const float m = fmaxf(fmaxf(red[8], red[9]), fmaxf(red[10], red[11]));
    const float s = __fdiv_rn(m, 127.f);
    if (tig == 0) *s_out = s;
#pragma unroll
    for (int j = 0; j < kRowMaxPieces; ++j)
        if (j < J) {
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = __uint_as_float((e & 1) ? (cw[j][e >> 1] & 0xFFFF0000u) : (cw[j][e >> 1] << 16));
            reinterpret_cast<uint2*>(q)[tig + 128 * j] = quant8_perm(v, s);
        }
    wg_sync(wg);
}

// The gated norm + quantization of one raw row over NT threads of one CTA (gdn_norm_quant_row's arithmetic):
// head h's norm factor by warp h % (NT / 32) (gdn_sumsq128 order), then the elements spread as the _cta row ops.
// hs: >= 32 floats of shared memory.
template <int NT, int BAR>
__device__ __forceinline__ void gdn_norm_quant_row_cta(const uint16_t* __restrict__ raw, const uint16_t* __restrict__ z,
                                                       const uint16_t* __restrict__ w, float eps, int K,
                                                       uint16_t* __restrict__ core_out, int8_t* __restrict__ q,
                                                       float* __restrict__ s_out, float* red, float* hs) {
    constexpr int KP = RowPieces<NT>::kMax, NW = NT / 32, HPW = (32 + NW - 1) / NW;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5, np = K >> 3, nh = K >> 7;
    {
        float v[HPW][4];
#pragma unroll
        for (int i = 0; i < HPW; ++i)
#pragma unroll
            for (int j = 0; j < 4; ++j)
                v[i][j] = warp + NW * i < nh ? bf16_bits_to_f32(__ldcg(raw + (warp + NW * i) * kDH + lane + 32 * j)) : 0.f;
#pragma unroll
        for (int i = 0; i < HPW; ++i) {
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < 4; ++j) ss = fmaf(v[i][j], v[i][j], ss);
#pragma unroll
            for (int o = 16; o; o >>= 1) ss += __shfl_xor_sync(0xffffffffu, ss, o);
            if (lane == 0 && warp + NW * i < nh) hs[warp + NW * i] = gdn_norm_inv(ss, eps);
        }
    }
    float vals[KP][8];
    uint4 rv[KP], zv[KP], wv[KP];
#pragma unroll
    for (int i = 0; i < KP; ++i)
        if (tid + NT * i < np) {
            const int c0 = (tid + NT * i) * 8;
            rv[i] = __ldcg(reinterpret_cast<const uint4*>(raw + c0));
            zv[i] = __ldcg(reinterpret_cast<const uint4*>(z + c0));
            wv[i] = __ldg(reinterpret_cast<const uint4*>(w + c0 % kDH));
        }
    row_sync<NT, BAR>();
#pragma unroll
    for (int i = 0; i < KP; ++i)
        if (tid + NT * i < np) {
            const int c0 = (tid + NT * i) * 8;
            const float r = hs[c0 / kDH];
            const uint32_t ru[4] = {rv[i].x, rv[i].y, rv[i].z, rv[i].w}, zu[4] = {zv[i].x, zv[i].y, zv[i].z, zv[i].w},
                           wu[4] = {wv[i].x, wv[i].y, wv[i].z, wv[i].w};
            uint32_t o[4] = {0, 0, 0, 0};
#pragma unroll
            for (int e = 0; e < 8; ++e) {
                const auto f = [](uint32_t u, int e) { return __uint_as_float((e & 1) ? (u & 0xFFFF0000u) : (u << 16)); };
                const uint16_t c = gdn_core(f(ru[e >> 1], e), f(wu[e >> 1], e), r, f(zu[e >> 1], e));
                vals[i][e] = bf16_bits_to_f32(c);
                o[e >> 1] |= uint32_t(c) << (16 * (e & 1));
            }
            if (core_out) reinterpret_cast<uint4*>(core_out)[tid + NT * i] = make_uint4(o[0], o[1], o[2], o[3]);
        }
    row_quant_pieces<NT, BAR>(vals, np, q, s_out, red);
}

}  // namespace mono
