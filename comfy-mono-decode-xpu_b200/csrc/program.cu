// Layer programs (program.h): one persistent cooperative launch runs a list of ops, the W4 weights of all its
// GEMV ops streaming through the producer warps' ring from the first instruction to the last.
//
// CTA = CW consumer warps + PW producer warps (stream.cuh), one per SM. The producers walk the CTA's items of
// every GEMV op in program order and, `prefetch` items ahead of the copies, ask the L2 to fetch the items they
// will copy next (cp.async.bulk.prefetch.L2), so HBM keeps streaming while the consumers are in a row phase, a
// Gated-DeltaNet phase or a grid barrier: the ring holds only S items per SM, the L2 a whole layer.
// The consumers run the ops in order:
//   OP_ROWS   rows m = wg * G + b (warp-group wg of CTA b): RMSNorm / sigmoid gate / plain / GDN gated norm,
//             then per-token quantization (rowops.cuh, gdn.cuh)
//   OP_GEMV   the CTA's tiles of the op (tile T = b + k G), partials in shared memory, epilogue per output:
//             out = bf16(total * xs[m]) (+ residual), or for a gate | up pair h = bf16(silu(g) * u) and the row
//             maxima of |h| (the reference's mono_mlp / layer_post arithmetic, mono_layer.sycl:272-313)
//   OP_QUANT  q = quant(h) with the row maxima of the paired GEMV
//   OP_AB     the bf16 a | b projection, one warp per output column on the last CTAs
//   OP_GDN_*  the Gated-DeltaNet conv + gates (gdn_conv_item over the channels) and delta rule (value columns
//             spread over the CTAs: CTA b holds columns [b CW 4, (b + 1) CW 4) as 8 row groups of 16 state rows)
// Every activation that an earlier op of the launch wrote is read through L2 (ld.global.cg).
#include <cstring>
#include <mutex>

#include "gdn.cuh"
#include "grid.cuh"
#include "program.h"
#include "rowops.cuh"
#include "stream.cuh"

namespace mono {

struct ProgParam {
    Op op[kProgParamOps];  // the ops when by_value
    const Op* ext;         // else: nops ops in device memory
    unsigned* bar;
    int nops, M, prefetch, by_value;
};

// Walk over a CTA's GEMV items across the ops (no divisions per step).
struct OpWalk {
    const Op* ops;
    int nops, op, k, sub, c, ntk, subs, C;
    bool done;
    __device__ void seek(int from) {
        for (op = from; op < nops; ++op) {
            if (ops[op].kind != OP_GEMV) continue;
            const PhaseDesc& p = ops[op].g.ph;
            ntk = cta_tiles(p);
            if (ntk == 0) continue;
            subs = phase_subs(p);
            C = p.K >> 10;
            k = sub = c = 0;
            done = false;
            return;
        }
        done = true;
    }
    __device__ void step() {
        if (++c < C) return;
        c = 0;
        if (++sub < subs) return;
        sub = 0;
        if (++k < ntk) return;
        seek(op + 1);
    }
    __device__ void skip(int n) {
        for (int i = 0; i < n && !done; ++i) step();
    }
};

// Producer warp p (of PW): items p, p + PW, ... into slot i % S; L2 prefetch of item i + prefetch first. Waits
// (bounded) for the last copy of each of its slots before returning.
template <int PW>
__device__ __forceinline__ void program_produce(const Op* ops, int nops, int prefetch, uint8_t* ring, uint64_t* full,
                                                uint64_t* empty, int S, int p, int lane) {
    constexpr int SB = stage_bytes<FMT_GPTQ>();
    OpWalk w{ops, nops};
    w.seek(0);
    w.skip(p);
    OpWalk f{ops, nops};
    f.done = true;
    if (prefetch > 0) {
        f.seek(0);
        f.skip(p + prefetch);
    }
    bool ok = true;
    int i = p;
    for (; !w.done && ok; i += PW) {
        const int s = i % S;
        if (!f.done) {
            if (lane == 0) prefetch_item_l2<FMT_GPTQ>(ops[f.op].g.ph, f.k, f.sub, f.c);
            f.skip(PW);
        }
        if (i >= S) ok = __all_sync(0xffffffffu, mbar_wait(&empty[s], ((i / S) - 1) & 1));
        if (!ok) break;
        issue_item<FMT_GPTQ, LAYOUT_TILED>(ops[w.op].g.ph, w.k, w.sub, w.c, ring + size_t(s) * SB, &full[s], lane);
        w.skip(PW);
    }
    const int issued = (i - p) / PW, keep = S / PW < issued ? S / PW : issued;
    for (int j = 0; j < keep; ++j) {
        const int it = i - PW * (j + 1);
        mbar_wait(&full[it % S], (it / S) & 1);
    }
}

// Cold ops (rows, quantization, a | b, GDN) are separate functions, so their registers are not added to those
// the GEMV path keeps live; each row mode is its own function for the same reason.
template <int MODE, int CW>
static __device__ __noinline__ void prog_rows_mode(const OpRows& r, int M, float* red, float* hs) {
    constexpr int NT = CW * 32;
    for (int m = int(blockIdx.x); m < M; m += int(gridDim.x)) {
        const uint16_t* xr = r.x + size_t(m) * r.x_stride;
        int8_t* q = r.q + size_t(m) * r.K;
        uint16_t* xn = r.xn_out ? r.xn_out + size_t(m) * r.K : nullptr;
        if constexpr (MODE == ROWS_GATE)
            gate_quant_row_cta<NT, kConsumerBar>(xr, r.gate + size_t(m) * r.gate_row_stride, r.gate_head_stride, r.lut,
                                                 r.K, q, r.s + m, red);
        else if constexpr (MODE == ROWS_GDN)
            gdn_norm_quant_row_cta<NT, kConsumerBar>(xr, r.gate + size_t(m) * r.gate_row_stride, r.norm_w, r.eps, r.K,
                                                     xn, q, r.s + m, red, hs);
        else
            norm_quant_row_cta<NT, kConsumerBar>(xr, MODE == ROWS_NORM ? r.norm_w : nullptr, r.eps, r.K, xn, q,
                                                 r.s + m, red);
    }
}

// One row per CTA (all consumer threads of CTA m take row m).
template <int CW>
__device__ __forceinline__ void prog_rows(const OpRows& r, int M, float* red, float* hs) {
    if (r.zero != nullptr && blockIdx.x == 0 && threadIdx.x < 16) r.zero[threadIdx.x] = 0u;
    if (int(blockIdx.x) >= M) return;
    if (r.mode == ROWS_GATE) prog_rows_mode<ROWS_GATE, CW>(r, M, red, hs);
    else if (r.mode == ROWS_GDN) prog_rows_mode<ROWS_GDN, CW>(r, M, red, hs);
    else if (r.mode == ROWS_NORM) prog_rows_mode<ROWS_NORM, CW>(r, M, red, hs);
    else prog_rows_mode<ROWS_QUANT, CW>(r, M, red, hs);
}

template <int MT, int CW>
__device__ __forceinline__ bool prog_gemv(const OpGemv& g, int base, int M, uint8_t* ring, uint64_t* full,
                                          uint64_t* empty, int S, uint32_t* part, int8_t* xsm, unsigned* rowmax) {
    constexpr int NT = CW * 32;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const PhaseDesc& ph = g.ph;
    const int K = ph.K, C = K >> 10, ntl = cta_tiles(ph), paired = ph.paired;
    XSrc xs{ph.x, K, false, true, true};
    if (ph.xsmem) {
        stage_x_consumers<CW>(ph.x, M, K, true, xsm);
        xs = XSrc{xsm, K + 16, true, true};
    }
    if (paired && threadIdx.x < 16) rowmax[threadIdx.x] = 0u;
    bool ok = consume_items<FMT_GPTQ, LAYOUT_TILED, MT, CW>(ph, base, nullptr, M, xs, ring, full, empty, S, part, warp,
                                                             lane);
    ok = consumer_sync_and<CW>(ok);
    if (!paired) {
        for (int e = threadIdx.x; e < ntl * M * 16 && ok; e += NT) {
            const int k = e / (M * 16), r = e - k * (M * 16), m = r >> 4, nl = r & 15;
            const int n = (int(blockIdx.x) + k * int(gridDim.x)) * 16 + nl;  // concatenated output column
            const float tot = __uint_as_float(tile_total<FMT_GPTQ, MT>(part + size_t(k) * C * MT * 128, C, 0, m, nl));
            uint16_t rr = f32_to_bf16_bits(__fmul_rn(tot, __ldcg(g.xs + m)));
            if (g.residual)
                rr = f32_to_bf16_bits(
                    __fadd_rn(bf16_bits_to_f32(__ldcg(g.residual + size_t(m) * g.res_stride + n)), bf16_bits_to_f32(rr)));
            g.out[size_t(m) * g.out_stride + n] = rr;
        }
    } else {
        for (int e = threadIdx.x; e < ntl * M * 16 && ok; e += NT) {
            const int k = e / (M * 16), r = e - k * (M * 16), m = r >> 4, nl = r & 15;
            const int n = (int(blockIdx.x) + k * int(gridDim.x)) * 16 + nl;
            const uint32_t* pk = part + size_t(k) * 2 * C * MT * 128;
            const float s = __ldcg(g.xs + m);
            const float tg = __uint_as_float(tile_total<FMT_GPTQ, MT>(pk, C, 0, m, nl));
            const float tu = __uint_as_float(tile_total<FMT_GPTQ, MT>(pk, C, 1, m, nl));
            const uint16_t gb = f32_to_bf16_bits(__fmul_rn(tg, s));
            const float u = bf16_round(__fmul_rn(tu, s));
            const uint16_t hb = f32_to_bf16_bits(__fmul_rn(bf16_bits_to_f32(__ldg(g.lut + gb)), u));
            g.out[size_t(m) * g.out_stride + n] = hb;
            atomicMax(&rowmax[m], __float_as_uint(fabsf(bf16_bits_to_f32(hb))));
        }
        consumer_sync<CW>();
        if (threadIdx.x < M) atomicMax(g.amax + threadIdx.x, rowmax[threadIdx.x]);
    }
    return ok;
}

template <int CW>
static __device__ __noinline__ void prog_quant(const OpQuant& o, int M) {
    constexpr int NT = CW * 32;
    const int ppr = o.K >> 3, pieces = M * ppr, stride = int(gridDim.x) * NT;
    for (int i = int(blockIdx.x) * NT + int(threadIdx.x); i < pieces; i += stride) {
        const int m = i / ppr;
        const float s = __fdiv_rn(__uint_as_float(__ldcg(o.amax + m)), 127.f);
        const uint4 hv = __ldcg(reinterpret_cast<const uint4*>(o.h) + i);
        const uint32_t u[4] = {hv.x, hv.y, hv.z, hv.w};
        float v[8];
#pragma unroll
        for (int e = 0; e < 8; ++e) v[e] = __uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16));
        reinterpret_cast<uint2*>(o.q)[i] = quant8_perm(v, s);
    }
    if (blockIdx.x == 0 && threadIdx.x < M) o.s[threadIdx.x] = __fdiv_rn(__uint_as_float(__ldcg(o.amax + threadIdx.x)), 127.f);
}

template <int CW>
static __device__ __noinline__ void prog_ab(const OpAb& a, int M, uint16_t* xsm) {
    // the last CTAs take CW / 4 columns each (the 4 quarters of a column on 4 warps, gdn.cuh gdn_ab_quarter): they
    // hold the fewest GEMV tiles. Such a CTA first copies the M normalized rows into shared memory.
    constexpr int NT = CW * 32, CPA = CW / 4;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int first = (int(gridDim.x) - 1 - int(blockIdx.x)) * CPA;
    if (first >= a.N) return;
    float* qs = reinterpret_cast<float*>(xsm + size_t(M) * a.K);  // [CPA][4][16]
    const int cl = warp >> 2, q = warp & 3;
    uint4 wv[4];
    if (cl < CPA && first + cl < a.N) gdn_ab_load_w(a.w, a.K, first + cl, q, lane, wv);  // in flight during the copy
    const int per = a.K >> 3;  // 16-byte pieces per row
    for (int i = threadIdx.x; i < M * per; i += NT) {
        const int m = i / per, c = i - m * per;
        reinterpret_cast<uint4*>(xsm + size_t(m) * a.K)[c] = __ldcg(reinterpret_cast<const uint4*>(a.x + size_t(m) * a.x_stride) + c);
    }
    consumer_sync<CW>();
    if (cl < CPA && first + cl < a.N) gdn_ab_quarter(xsm, wv, a.K, M, q, lane, qs + (cl * 4 + q) * 16);
    consumer_sync<CW>();
    if (int(threadIdx.x) < CPA * M) {
        const int c = threadIdx.x / M, m = threadIdx.x % M;
        if (first + c < a.N) a.out[size_t(m) * a.N + first + c] = gdn_ab_combine(qs + c * 64, 16, m);
    }
    consumer_sync<CW>();
}

template <int CW>
static __device__ __noinline__ void prog_gdn_conv(const GdnArgs& A) {
    constexpr int NT = CW * 32;
    const int n = A.C > (kGdnMaxRows + A.M) * A.HV ? A.C : (kGdnMaxRows + A.M) * A.HV;
    for (int i = int(blockIdx.x) * NT + int(threadIdx.x); i < n; i += int(gridDim.x) * NT) gdn_conv_item(A, i);
}

// Shared scratch of the delta op: q / k rows of up to two heads, the row-group partials, the sums of squares.
template <int CW>
__host__ __device__ constexpr size_t delta_scratch_bytes() {
    return (2 * 2 * kGdnMaxAll * kDH + 2 * kRG * (CW * 32 / kRG) + 2 * 2 * kGdnMaxAll + kGdnMaxAll * (CW * 32 / kRG) +
            kGdnMaxAll * 2 * 2) * sizeof(float);
}

// The delta rule of CTA b's value columns (gdn_delta_kernel's arithmetic, value columns spread over CTAs): raw
// outputs bf16(o) of the verify rows to A.core [M][HV * 128]; committed states persisted as the standalone form.
template <int CW>
static __device__ __noinline__ void prog_gdn_delta(const GdnArgs& A, float* scratch) {
    constexpr int NT = CW * 32, CPC = NT / kRG;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31, rg = tid / CPC, cl = tid % CPC;
    const int total = A.HV * kDH, c0 = int(blockIdx.x) * CPC;
    if (c0 >= total) return;  // the whole CTA
    const int gc = c0 + cl;
    const bool active = gc < total;
    const int h0 = c0 / kDH, h1 = ((c0 + CPC < total ? c0 + CPC : total) - 1) / kDH, nhl = h1 - h0 + 1;
    __shared__ int cs[kGdnCtlWords];  // the ctl words, read once (the entry walk below reads them many times)
    gdn_ctl_stage(A, cs);
    consumer_sync<CW>();
    const int n = gdn_pending_s(A, cs), R = n + A.M, KD = A.HK * kDH, grp = A.HV / A.HK;
    float* qn = scratch;                         // [2][kGdnMaxAll][kDH]
    float* kn = qn + 2 * kGdnMaxAll * kDH;       // [2][kGdnMaxAll][kDH]
    float* part = kn + 2 * kGdnMaxAll * kDH;     // [2][kRG][CPC]
    float* sums = part + 2 * kRG * CPC;          // [2 heads][q, k][kGdnMaxAll]
    float* vsm = sums + 2 * 2 * kGdnMaxAll;      // [kGdnMaxAll][CPC]: v of the CTA's columns
    float* gsm = vsm + kGdnMaxAll * CPC;         // [kGdnMaxAll][2 heads][decay, beta]
    for (int pr = warp; pr < nhl * 2 * R; pr += CW) {
        const int hl = pr / (2 * R), rem = pr - hl * 2 * R, t = rem >> 1, which = rem & 1;
        const int kh = (h0 + hl) / grp;
        const float s = gdn_sumsq128(A.conv_out + size_t(t) * A.C + which * KD + kh * kDH, lane);
        if (lane == 0) sums[(hl * 2 + which) * kGdnMaxAll + t] = s;
    }
    consumer_sync<CW>();
    for (int e = tid; e < nhl * R * kDH; e += NT) {
        const int hl = e / (R * kDH), rem = e - hl * R * kDH, t = rem / kDH, d = rem % kDH;
        const int kh = (h0 + hl) / grp;
        const float qi = gdn_l2_inv(sums[(hl * 2) * kGdnMaxAll + t]), ki = gdn_l2_inv(sums[(hl * 2 + 1) * kGdnMaxAll + t]);
        qn[(hl * kGdnMaxAll + t) * kDH + d] =
            (bf16_bits_to_f32(__ldcg(A.conv_out + size_t(t) * A.C + kh * kDH + d)) * A.qscale) * qi;
        kn[(hl * kGdnMaxAll + t) * kDH + d] = bf16_bits_to_f32(__ldcg(A.conv_out + size_t(t) * A.C + KD + kh * kDH + d)) * ki;
    }
    for (int e = tid; e < R * CPC; e += NT) {
        const int t = e / CPC, c = e % CPC;
        vsm[e] = c0 + c < total ? bf16_bits_to_f32(__ldcg(A.conv_out + size_t(t) * A.C + 2 * KD + c0 + c)) : 0.f;
    }
    if (tid < R * nhl * 2) {
        const int t = tid / (nhl * 2), hl = (tid >> 1) % nhl, which = tid & 1;
        gsm[(t * 2 + hl) * 2 + which] = __ldcg(A.gates + (t * A.HV + h0 + hl) * 2 + which);
    }
    const int h = active ? gc / kDH : h0, col = gc % kDH, hl = h - h0;
    float st[kRPG];
    float* Sp = A.state + (size_t(h) * kDH + rg * kRPG) * kDH + col;
    if (active) {
#pragma unroll
        for (int r = 0; r < kRPG; ++r) st[r] = __ldcg(Sp + size_t(r) * kDH);
    } else {
#pragma unroll
        for (int r = 0; r < kRPG; ++r) st[r] = 0.f;
    }
    consumer_sync<CW>();
    const float* qh = qn + hl * kGdnMaxAll * kDH + rg * kRPG;
    const float* kh_ = kn + hl * kGdnMaxAll * kDH + rg * kRPG;
    float* p0 = part;
    float* p1 = part + kRG * CPC;
    if (active && rg == 0)  // rows no entry names read as zero (the entries below overwrite the others)
        for (int m = 0; m < A.M; ++m) A.core[size_t(m) * total + gc] = 0;
    const int E = n + gdn_verify_entries_s(A, cs);
    for (int e = 0; e < E; ++e) {
        const GdnEntry en = gdn_entry_s(A, cs, n, e);
        const int t = en.row;
        float mem = 0.f, decay = 1.f, beta = 0.f, v = 0.f;
        if (active) {
            decay = gsm[(t * 2 + hl) * 2];
            beta = gsm[(t * 2 + hl) * 2 + 1];
            v = vsm[t * CPC + cl];
            if (en.commit) {
#pragma unroll
                for (int r = 0; r < kRPG; ++r) {
                    st[r] *= decay;
                    mem = fmaf(st[r], kh_[t * kDH + r], mem);
                }
            } else {
#pragma unroll
                for (int r = 0; r < kRPG; ++r) mem = fmaf(st[r] * decay, kh_[t * kDH + r], mem);
            }
        }
        p0[rg * CPC + cl] = mem;
        consumer_sync<CW>();
        float o = 0.f;
        if (active) {
            float kv = p0[cl];  // the group partials in group order (gdn_delta_kernel's)
#pragma unroll
            for (int j = 1; j < kRG; ++j) kv += p0[j * CPC + cl];
            const float delta = (v - kv) * beta;
            if (en.commit) {
#pragma unroll
                for (int r = 0; r < kRPG; ++r) {
                    st[r] = fmaf(kh_[t * kDH + r], delta, st[r]);
                    o = fmaf(st[r], qh[t * kDH + r], o);
                }
            } else {
#pragma unroll
                for (int r = 0; r < kRPG; ++r) o = fmaf(fmaf(kh_[t * kDH + r], delta, st[r] * decay), qh[t * kDH + r], o);
            }
        }
        p1[rg * CPC + cl] = o;
        consumer_sync<CW>();
        if (active && rg == 0 && en.out >= 0) {
            float os = p1[cl];
#pragma unroll
            for (int j = 1; j < kRG; ++j) os += p1[j * CPC + cl];
            A.core[size_t(en.out) * total + gc] = f32_to_bf16_bits(bf16_round(os));
        }
        if (active && A.ctl != nullptr && e == n - 1)
#pragma unroll
            for (int r = 0; r < kRPG; ++r) Sp[size_t(r) * kDH] = st[r];
    }
    if (active && A.ctl == nullptr)
#pragma unroll
        for (int r = 0; r < kRPG; ++r) Sp[size_t(r) * kDH] = st[r];
}

template <int MT, int CW, int PW>
__global__ void __launch_bounds__((CW + PW) * 32, 1) program_kernel(const __grid_constant__ ProgParam G, const MlpShape Z) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[64];
    __shared__ float hs[32];
    __shared__ unsigned rowmax[16];
    __shared__ int flag;
    const Op* ops = G.by_value ? G.op : G.ext;
    const int nops = G.nops, M = G.M, S = Z.S;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const StreamPlan plan(stage_bytes<FMT_GPTQ>(), S, Z.part_bytes, Z.x_bytes, 0);
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + plan.ring);
    uint64_t* empty = full + S;
    uint32_t* part = reinterpret_cast<uint32_t*>(smem + plan.ring + plan.bars);
    int8_t* xsm = reinterpret_cast<int8_t*>(smem + plan.ring + plan.bars + plan.part);
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    trace_stamp(0);
    pdl_launch_dependents();
    if (warp >= CW) {
        // weights do not depend on the preceding kernel: stream them before (without) the dependency wait
        program_produce<PW>(ops, nops, G.prefetch, ring, full, empty, S, warp - CW, lane);
        return;
    }
    constexpr int NT = CW * 32;
    pdl_wait();
    unsigned epoch = 0;
    bool ok = true;
    int base = 0;  // the CTA's request index of the current GEMV op's first item
    for (int j = 0; j < nops; ++j) {
        const Op& op = ops[j];
        const int kind = op.kind;
        if (kind == OP_ROWS) {
            prog_rows<CW>(op.r, M, red, hs);
        } else if (kind == OP_GEMV) {
            ok = prog_gemv<MT, CW>(op.g, base, M, ring, full, empty, S, part, xsm, rowmax) && ok;
            base += cta_items(op.g.ph);
        } else if (kind == OP_QUANT) {
            prog_quant<CW>(op.q, M);
        } else if (kind == OP_AB) {
            prog_ab<CW>(op.ab, M, reinterpret_cast<uint16_t*>(xsm));
        } else if (kind == OP_GDN_CONV) {
            prog_gdn_conv<CW>(op.gdn);
        } else if (kind == OP_GDN_DELTA) {
            prog_gdn_delta<CW>(op.gdn, reinterpret_cast<float*>(xsm));
        }
        if (j < kTracePhases - 1) trace_stamp(1 + j);
        if (op.barrier) ok = grid_barrier_named<kConsumerBar, NT>(G.bar, epoch, &flag) && ok;
    }
    grid_exit_named<kConsumerBar, NT>(G.bar);
}

// ---- host side ----

static int op_tiles_per_cta(const PhaseDesc& p, int G) { return (phase_tiles(p) + G - 1) / G; }

static size_t op_part_bytes(const Op& op, int G, int MT) {
    if (op.kind != OP_GEMV) return 0;
    const PhaseDesc& p = op.g.ph;
    return size_t(op_tiles_per_cta(p, G)) * (p.paired ? 2 : 1) * phase_chunks(p) * MT * 128 * 4;
}

// Shared shape for the current staging flags: the first stream configuration that fits, or -1.
static int program_shape(const Op* ops, int nops, int M, MlpShape& Z) {
    const int G = sm_count(), MT = M > 8 ? 2 : 1;
    size_t part = 0, xb = 0, scratch = 0;
    for (int i = 0; i < nops; ++i) {
        const size_t pb = op_part_bytes(ops[i], G, MT);
        part = pb > part ? pb : part;
        if (ops[i].kind == OP_GEMV && ops[i].g.ph.xsmem) {
            const size_t b = size_t(M) * (ops[i].g.ph.K + 16);
            xb = b > xb ? b : xb;
        }
        if (ops[i].kind == OP_GDN_DELTA) scratch = scratch > delta_scratch_bytes<12>() ? scratch : delta_scratch_bytes<12>();
        if (ops[i].kind == OP_AB) {
            const size_t b = size_t(M) * ops[i].ab.K * 2 + 12 / 4 * 4 * 16 * 4;  // staged rows + quarter sums
            scratch = b > scratch ? b : scratch;
        }
    }
    xb = scratch > xb ? scratch : xb;
    for (int c = 0; c < kStreamConfigs; ++c) {
        const StreamConfig sc = kStreamConfig[c];
        const StreamPlan plan(stage_bytes<FMT_GPTQ>(), sc.S, part, xb, 0);
        if (plan.total > kStreamSmemLimit) continue;
        Z = MlpShape{sc.S, int(part), int(xb)};
        return c;
    }
    return -1;
}

static int check_op(const Op& op, int M) {
    switch (op.kind) {
    case OP_ROWS: {
        const OpRows& r = op.r;
        MONO_CHECK(r.x && r.q && r.s, "rows op: null operand");
        MONO_CHECK(r.K >= 1024 && r.K % 1024 == 0 && r.K <= 4096, "rows op: K a multiple of 1024 up to 4096");
        MONO_CHECK(r.mode >= ROWS_NORM && r.mode <= ROWS_GDN, "rows op: mode");
        MONO_CHECK(r.mode != ROWS_NORM || r.norm_w, "rows op: norm weight");
        MONO_CHECK(r.mode != ROWS_GATE || (r.gate && r.lut), "rows op: gate and LUT");
        MONO_CHECK(r.mode != ROWS_GDN || (r.gate && r.norm_w && r.K <= 32 * 128), "rows op: z and gated-norm weight");
        MONO_CHECK(aligned(r.x, 16) && r.x_stride % 8 == 0 && aligned(r.q, 8), "rows op: 16-byte aligned rows");
        return MONO_OK;
    }
    case OP_GEMV: {
        const PhaseDesc& p = op.g.ph;
        MONO_CHECK(p.nm >= 1 && p.nm <= 3 && (!p.paired || p.nm == 2), "gemv op: 1 to 3 matrices or a pair");
        MONO_CHECK(p.K >= 1024 && p.K % 1024 == 0 && p.K <= kChunkK * kMaxChunks, "gemv op: K");
        for (int i = 0; i < p.nm; ++i) MONO_CHECK(p.m[i].q && p.m[i].n >= 16 && p.m[i].n % 16 == 0 && aligned(p.m[i].q, 16), "gemv op: matrix");
        MONO_CHECK(!p.paired || p.m[0].n == p.m[1].n, "gemv op: pair shapes");
        MONO_CHECK(p.x && aligned(p.x, 16) && op.g.xs && op.g.out, "gemv op: null operand");
        MONO_CHECK(!p.paired || (op.g.lut && op.g.amax && !op.g.residual), "gemv op: pair needs LUT and row maxima");
        return MONO_OK;
    }
    case OP_QUANT:
        MONO_CHECK(op.q.h && op.q.amax && op.q.q && op.q.s && op.q.K % 8 == 0 && aligned(op.q.h, 16), "quant op");
        return MONO_OK;
    case OP_AB:
        MONO_CHECK(op.ab.x && op.ab.w && op.ab.out && op.ab.K % 1024 == 0 && op.ab.K <= 4096 && op.ab.x_stride % 8 == 0 && aligned(op.ab.x, 16) &&
                       aligned(op.ab.w, 16),
                   "a|b op");
        return MONO_OK;
    case OP_GDN_CONV:
    case OP_GDN_DELTA:
        MONO_CHECK(op.gdn.M == M && op.gdn.conv_out && op.gdn.gates && op.gdn.core, "gdn op: rows / workspace");
        MONO_CHECK(op.gdn.HV * 128 <= 4096, "gdn op: HV <= 32");
        return MONO_OK;
    }
    return fail(MONO_EINVAL, "unknown op kind %d", op.kind);
}

int plan_program(Op* ops, int nops, int M) {
    MONO_CHECK(ops && nops >= 1, "empty program");
    MONO_CHECK(M >= 1 && M <= 16, "1 <= M <= 16 rows");
    for (int i = 0; i < nops; ++i) {
        const int rc = check_op(ops[i], M);
        if (rc != MONO_OK) return rc;
    }
    for (int i = 0; i < nops; ++i)
        if (ops[i].kind == OP_GEMV) ops[i].g.ph.xsmem = 1;
    for (;;) {
        MlpShape Z;
        if (program_shape(ops, nops, M, Z) >= 0) return MONO_OK;
        int big = -1;
        for (int i = 0; i < nops; ++i)
            if (ops[i].kind == OP_GEMV && ops[i].g.ph.xsmem && (big < 0 || ops[i].g.ph.K > ops[big].g.ph.K)) big = i;
        if (big < 0) break;
        ops[big].g.ph.xsmem = 0;
    }
    return fail(MONO_EINVAL, "program: no shared-memory plan fits (M=%d)", M);
}

template <int MT, int CW, int PW>
static int launch_program_t(const ProgParam& G, const MlpShape& Z, size_t smem, cudaStream_t stream) {
    auto kern = program_kernel<MT, CW, PW>;
    static std::mutex mu;
    static size_t opt_in = 0;
    static int per_sm = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (smem > opt_in) {
            CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
            opt_in = smem;
            CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, (CW + PW) * 32, smem));
        }
    }
    if (per_sm < 1) return fail(MONO_EINVAL, "program: one CTA does not fit an SM (%zu B shared)", smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sm_count());
    cfg.blockDim = dim3((CW + PW) * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, G, Z));
    return MONO_OK;
}

int launch_program(const Op* ops_host, const Op* ops_dev, int nops, int M, unsigned* bar, int prefetch,
                   cudaStream_t stream) {
    MONO_CHECK(ops_host && nops >= 1 && bar, "program: ops and barrier words");
    MONO_CHECK(ops_dev || nops <= kProgParamOps, "program: more than %d ops need a device copy", kProgParamOps);
    MONO_CHECK(M >= 1 && M <= 16, "1 <= M <= 16 rows");
    MONO_CHECK(prefetch >= 0 && prefetch <= 4096, "prefetch distance");
    MlpShape Z;
    const int c = program_shape(ops_host, nops, M, Z);
    MONO_CHECK(c >= 0, "program: not planned (mono_program_plan)");
    static_assert(sizeof(ProgParam) < 32000, "kernel parameter space");
    ProgParam G;
    std::memset(&G, 0, sizeof(G));
    if (ops_dev) {
        G.ext = ops_dev;
        G.by_value = 0;
    } else {
        std::memcpy(G.op, ops_host, sizeof(Op) * nops);
        G.by_value = 1;
    }
    G.bar = bar;
    G.nops = nops;
    G.M = M;
    G.prefetch = prefetch;
    const StreamPlan plan(stage_bytes<FMT_GPTQ>(), Z.S, Z.part_bytes, Z.x_bytes, 0);
    const bool two = M > 8;
#define MONO_PG(MTV, CWV, PWV) return launch_program_t<MTV, CWV, PWV>(G, Z, plan.total, stream)
    if (!two) {
        if (c == 0) MONO_PG(1, 10, 2);
        if (c == 1 || c == 3) MONO_PG(1, 8, 4);
        MONO_PG(1, 12, 4);
    } else {
        if (c == 0) MONO_PG(2, 10, 2);
        if (c == 1 || c == 3) MONO_PG(2, 8, 4);
        MONO_PG(2, 12, 4);
    }
#undef MONO_PG
}

}  // namespace mono
