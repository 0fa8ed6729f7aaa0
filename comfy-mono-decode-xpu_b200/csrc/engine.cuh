// The W4A8 stream engine: every W4A8 GEMV of the decode step, standalone or inside a fused kernel.
//
// Arithmetic (two weight formats sharing one int4 unpack and one int8 tensor-core dot):
//   GPTQ  int4 v in [-8, 7] stored as nibble v + 8, fp16 scale per (row, 128-group):
//           acc_g = int32 dot over group g;  F_c = fp32 sum over the 8 groups of 1024-chunk c of
//           float(acc_g) * float(s[n, g]);   total = fp32 sum of F_c over c   (sums in order, from +0,
//           every op IEEE RNE, never fused)
//   REF   the reference's packed W4A8 (csrc/w4a8_decode.sycl:4-11, :35-45): codes into an fp32 codebook
//         at FP8 e4m3 G16 relative scales, decoded onto the int8 grid through a pair table;
//           total = int32 (mod 2^32) dot over all of K.
//
// Work: a program of GEMV phases. A phase multiplies the activation rows x [M][K] by up to three
// matrices that share K, with tiles concatenated (q | k | v), or by a gate/up pair whose tiles are
// processed together. Tile = 16 output rows; its K is cut into 1024-wide chunks (items). A CTA holds
// warp-groups of 4 warps; each warp-group is a virtual CTA (interleaved over the SMs) that takes tiles
// round-robin, its warps take a tile's items round-robin, and the chunk partials meet in shared memory
// where one thread per output sums them in chunk order.
//
// Streaming: one item = 8 KB of weights + its scales, one TMA bulk copy from the tile-major layout
// (mono_w4_repack: per (tile, chunk) the weights then the scales, contiguous), or 16-byte cp.async
// pieces from the checkpoint's row-major layout. Every warp owns a 2-deep ring of item stages; its
// producer cursor walks the warp's items across all phases of the program, so the next phase's weights
// are in flight while the CTA waits at a grid barrier. (Measured on B200: 8 KB copies, 2 stages, 8 warps
// per SM stream at ~6.3 TB/s; 2 KB copies plus separate scale copies were capped by the per-copy cost of
// the TMA unit.) Activations of a phase are staged once per CTA in shared memory by vector loads (pitch
// K + 16: conflict-free fragment reads) when they fit, else read through L1.
//
// mma fragment mapping (swap-AB: weights are the 16-row A operand, activations the 8-column B operand).
// Inside a 128-group lane (g, t) owns bytes [16t, 16t + 16) of rows g and g + 8, i.e. packed words
// 4t + s (s = 0..3). At k-step s its word's even nibbles are A columns 4t..4t+3 and its odd nibbles A
// columns 16 + 4t..; the activation bytes of those columns are x[8(4t + s) + {0,2,4,6}] and
// x[8(4t + s) + {1,3,5,7}] of the group: 32 contiguous bytes per lane and group, stored permuted
// (bytes 0 2 4 6 1 3 5 7 of every 8) so each B register is one 32-bit word.
#pragma once
#include "common.cuh"

namespace mono {

enum W4Format : int { FMT_GPTQ = 0, FMT_REF = 1 };
enum W4Layout : int { LAYOUT_ROW = 0, LAYOUT_TILED = 1 };

constexpr int kGroupWarps = 4;     // warps per warp-group
constexpr int kMaxStages = 2;      // deepest ring per warp (item stages)
constexpr int kStageW = 8192;      // weight bytes per item (8 groups x 16 rows x 64 B)
constexpr int kChunkK = 1024;      // K per item
constexpr int kMaxChunks = 16;     // K <= 16384
constexpr int kMaxPhases = 4;

template <int FMT>
struct Fmt;
template <>
struct Fmt<FMT_GPTQ> {
    static constexpr int SB = 256;  // item scales: [16 rows][8 groups] fp16
};
template <>
struct Fmt<FMT_REF> {
    static constexpr int SB = 1024;  // item scales: [16 rows][8 groups x 8 G16] fp8
};
template <int FMT>
__host__ __device__ constexpr int stage_bytes() { return kStageW + Fmt<FMT>::SB; }

struct MatDesc {
    const uint8_t* q;  // TILED: [N/16][K/1024][8 KB weights | scales]; ROW: [N][K/2] bytes (low nibble = even k)
    const uint8_t* s;  // ROW only: GPTQ fp16 [N][K/128] / REF fp8 [N][K/16]
    int n;
};

struct PhaseDesc {
    MatDesc m[3];
    int nm, paired, K;
    const int8_t* x;  // activation rows [M][K] (row stride K)
    int xsmem;        // 1: staged in shared memory
    int xperm;        // 1: x is already in the permuted byte order
    int rev;          // 1: tiles dealt to the CTAs in reverse order (stream.cuh cta_slot)
};

struct Program {
    PhaseDesc ph[kMaxPhases];
    int nph, M;
    const uint16_t* pair_tab;  // REF decode table (mono_w4_pair_table)
};

__host__ __device__ inline int phase_tiles(const PhaseDesc& p) {
    if (p.paired) return p.m[0].n >> 4;
    int t = 0;
    for (int i = 0; i < p.nm; ++i) t += p.m[i].n >> 4;
    return t;
}
__host__ __device__ inline int phase_chunks(const PhaseDesc& p) { return p.K / kChunkK; }
__host__ __device__ inline int phase_items(const PhaseDesc& p) { return (p.paired ? 2 : 1) * phase_chunks(p); }

// (phase tile T, subtile) -> (matrix, local 16-row tile)
__host__ __device__ inline void resolve(const PhaseDesc& p, int T, int sub, int& mat, int& lt) {
    if (p.paired) {
        mat = sub;
        lt = T;
        return;
    }
    mat = 0;
    lt = T;
    if (p.nm > 1 && lt >= (p.m[0].n >> 4)) {
        lt -= p.m[0].n >> 4;
        mat = 1;
        if (p.nm > 2 && lt >= (p.m[1].n >> 4)) {
            lt -= p.m[1].n >> 4;
            mat = 2;
        }
    }
}

struct Cursor {
    int ph, ti, it;  // phase, k-th own tile, k-th own item of the tile
    int sub, chunk;  // item = warp + 4 it -> (subtile, chunk)
    bool done;
};

// The item sequence of one warp: virtual CTA vc of nvc, warp `warp` of its group. Per-phase counts are
// computed from the kernel parameters when needed (no per-phase arrays: those would live in local memory).
struct Seq {
    int warp, vc, nvc;
    const Program* prog;
    __device__ void init(const Program& P, int warp_, int vc_, int nvc_) {
        warp = warp_;
        vc = vc_;
        nvc = nvc_;
        prog = &P;
    }
    __device__ int my_tiles(int ph) const {
        const int t = phase_tiles(prog->ph[ph]);
        return vc < t ? (t - 1 - vc) / nvc + 1 : 0;
    }
    __device__ int my_items(int ph) const {
        const int it = phase_items(prog->ph[ph]);
        return warp < it ? ((it - 1 - warp) >> 2) + 1 : 0;
    }
    __device__ int chunks(int ph) const { return prog->ph[ph].K >> 10; }
    __device__ void first_item(Cursor& c) const {
        const int C = chunks(c.ph);
        c.chunk = warp;
        c.sub = 0;
        while (c.chunk >= C) {
            c.chunk -= C;
            ++c.sub;
        }
    }
    __device__ Cursor start(const Program& P, int ph) const {
        Cursor c{ph, 0, 0, 0, 0, false};
        while (c.ph < P.nph && (my_tiles(c.ph) == 0 || my_items(c.ph) == 0)) ++c.ph;
        c.done = c.ph >= P.nph;
        if (!c.done) first_item(c);
        return c;
    }
    __device__ void advance(const Program& P, Cursor& c) const {
        if (++c.it < my_items(c.ph)) {
            const int C = chunks(c.ph);
            c.chunk += kGroupWarps;
            while (c.chunk >= C) {
                c.chunk -= C;
                ++c.sub;
            }
            return;
        }
        c.it = 0;
        if (++c.ti < my_tiles(c.ph)) {
            first_item(c);
            return;
        }
        c = start(P, c.ph + 1);
    }
};

// The tile-major source of an item (weights followed by scales, stage_bytes<FMT>() contiguous bytes).
template <int FMT>
__device__ __forceinline__ const uint8_t* item_src(const Program& P, const Seq& sq, const Cursor& c) {
    const PhaseDesc& p = P.ph[c.ph];
    const int T = sq.vc + c.ti * sq.nvc;
    int mat, lt;
    resolve(p, T, c.sub, mat, lt);
    return p.m[mat].q + (size_t(lt) * (p.K >> 10) + c.chunk) * stage_bytes<FMT>();
}

template <int FMT, int LAYOUT>
__device__ __forceinline__ void issue_item(const Program& P, const Seq& sq, const Cursor& c, uint8_t* stage,
                                           uint64_t* bar, int lane) {
    constexpr int SB = Fmt<FMT>::SB;
    const PhaseDesc& p = P.ph[c.ph];
    const int T = sq.vc + c.ti * sq.nvc;
    int mat, lt;
    resolve(p, T, c.sub, mat, lt);
    const MatDesc& w = p.m[mat];
    const int C = p.K >> 10;
    if constexpr (LAYOUT == LAYOUT_TILED) {
        if (lane == 0) {
            // The slot's previous contents were consumed into registers before the warp's __syncwarp in
            // Ring::release: the bulk copy may overwrite it without a proxy fence.
            mbar_arrive_expect_tx(bar, kStageW + SB);
            bulk_g2s(stage, w.q + (size_t(lt) * C + c.chunk) * (kStageW + SB), kStageW + SB, bar);
        }
    } else {
        const int g = lane >> 2, t = lane & 3;
        const size_t rowb = size_t(p.K) >> 1;
        const uint8_t* r0 = w.q + size_t(lt * 16 + g) * rowb + size_t(c.chunk) * 512 + t * 16;
        const uint8_t* r1 = r0 + 8 * rowb;
#pragma unroll
        for (int gi = 0; gi < 8; ++gi) {
            cp_async16(stage + gi * 1024 + lane * 16, r0 + gi * 64);
            cp_async16(stage + gi * 1024 + 512 + lane * 16, r1 + gi * 64);
        }
        if constexpr (FMT == FMT_GPTQ) {
            // [16 rows][8 groups] fp16: 16 bytes per row
            if (lane < 16) cp_async16(stage + kStageW + lane * 16, w.s + (size_t(lt * 16 + lane) * (p.K >> 7) + c.chunk * 8) * 2);
        } else {
            // [16 rows][64 bytes]: 4 pieces per row, 2 per lane
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int piece = lane + 32 * h, row = piece >> 2, part = piece & 3;
                cp_async16(stage + kStageW + row * 64 + part * 16, w.s + size_t(lt * 16 + row) * (p.K >> 4) + c.chunk * 64 + part * 16);
            }
        }
        cp_async_commit();
    }
}

template <int FMT, int LAYOUT, int kStages>
struct Ring {
    uint8_t* buf;
    uint64_t* bars;
    Cursor prod;  // next item to copy into the ring
    Cursor pfc;   // next item to request into L2 (tiled layouts): pf_dist items ahead of prod
    int issued, consumed;
    bool ok;

    // Issue the first kStages copies and L2 prefetches of the pf_dist items after them. The copies go
    // through this SM's TMA unit in order: callers issue them after any urgent activation loads.
    __device__ void init(const Program& P, const Seq& sq, int lane, int pf_dist) {
        if (LAYOUT == LAYOUT_TILED && lane == 0) {
            for (int i = 0; i < kStages; ++i) mbar_init(&bars[i], 1);
            fence_mbar_init();
        }
        __syncwarp();
        prod = sq.start(P, 0);
        issued = consumed = 0;
        ok = true;
        for (int i = 0; i < kStages; ++i) {
            if (!prod.done) {
                issue_item<FMT, LAYOUT>(P, sq, prod, buf + (issued % kStages) * stage_bytes<FMT>(), &bars[issued % kStages],
                                        lane);
                ++issued;
                sq.advance(P, prod);
            } else if (LAYOUT == LAYOUT_ROW) {
                cp_async_commit();
            }
        }
        pfc = prod;
        if constexpr (LAYOUT == LAYOUT_TILED)
            for (int i = 0; i < pf_dist && !pfc.done; ++i) prefetch_next(P, sq, lane);
    }
    __device__ void prefetch_next(const Program& P, const Seq& sq, int lane) {
        if (lane == 0) bulk_prefetch_l2(item_src<FMT>(P, sq, pfc), stage_bytes<FMT>());
        sq.advance(P, pfc);
    }
    __device__ uint8_t* wait() {
        const int slot = consumed % kStages;
        if constexpr (LAYOUT == LAYOUT_TILED) {
            if (ok) ok = mbar_wait(&bars[slot], (consumed / kStages) & 1);
        } else {
            cp_async_wait<kStages - 1>();
            __syncwarp();
        }
        return buf + slot * stage_bytes<FMT>();
    }
    __device__ void release(const Program& P, const Seq& sq, int lane) {
        __syncwarp();
        const int slot = consumed % kStages;
        ++consumed;
        if (!prod.done && ok) {
            issue_item<FMT, LAYOUT>(P, sq, prod, buf + slot * stage_bytes<FMT>(), &bars[slot], lane);
            ++issued;
            sq.advance(P, prod);
            if constexpr (LAYOUT == LAYOUT_TILED)
                if (!pfc.done) prefetch_next(P, sq, lane);
        } else if (LAYOUT == LAYOUT_ROW) {
            cp_async_commit();
        }
    }
    // Before exit: wait (bounded) for copies still in flight (none on the normal path, where every
    // issued stage was consumed).
    __device__ void drain(int lane) {
        if constexpr (LAYOUT == LAYOUT_ROW) {
            cp_async_wait<0>();
        } else if (lane == 0) {
            for (int k = consumed; k < issued; ++k) mbar_wait(&bars[k % kStages], (k / kStages) & 1);
        }
    }
};

// REF decode of one packed word (8 codes sharing one fp8 scale byte) into the even / odd A registers.
__device__ __forceinline__ void ref_decode(const uint16_t* __restrict__ tab, uint32_t word, uint32_t sb,
                                           uint32_t& even, uint32_t& odd) {
    const uint16_t* row = tab + (sb << 8);
    const uint32_t e0 = __ldg(row + (word & 0xFF)), e1 = __ldg(row + ((word >> 8) & 0xFF));
    const uint32_t e2 = __ldg(row + ((word >> 16) & 0xFF)), e3 = __ldg(row + (word >> 24));
    const uint32_t r01 = e0 | (e1 << 16), r23 = e2 | (e3 << 16);
    even = prmt(r01, r23, 0x6420);
    odd = prmt(r01, r23, 0x7531);
}

// Activation source of a phase: shared (pitch K + 16) or global through L1 (pitch K); perm: permuted bytes.
struct XSrc {
    const int8_t* p;
    int pitch;
    bool smem, perm;
    bool cg = false;  // global rows written earlier in the same launch: read through L2 only (ld.global.cg)
};

// Consume one item (8 groups). R = the chunk partial per fragment element: fp32 bits (GPTQ, carrying a
// factor 16, see below) or the int32 dot (REF). Fragment element i of m-tile mt: (row g + 8 (i >> 1),
// activation 2t + (i & 1)).
// XMODE: 0 = global, natural byte order; 1 = global, permuted; 2 = shared (pitch K + 16), permuted;
// 3 = global, permuted, read through L2 only (rows written by other CTAs of the same launch).
template <int FMT, int LAYOUT, int MT, int XMODE>
__device__ __forceinline__ void compute_item(const uint8_t* __restrict__ stage, const uint16_t* __restrict__ pair_tab,
                                             const XSrc& xs, int M, int chunk, int lane, uint32_t (&R)[MT][4]) {
    const int g = lane >> 2, t = lane & 3;
    float F[MT][4];
    int A[MT][4];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            F[mt][i] = 0.f;
            A[mt][i] = 0;
        }
    // GPTQ item scales: [16 rows][8 groups] fp16
    const __half* sc16 = reinterpret_cast<const __half*>(stage + kStageW);
    const uint32_t zero = 0;
    const int8_t* xrow[MT];
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) xrow[mt] = xs.p + size_t(g + 8 * mt) * xs.pitch + chunk * kChunkK + 32 * t;
#pragma unroll 2
    for (int gi = 0; gi < 8; ++gi) {
        const uint4 wa = lds_v4(stage + gi * 1024 + lane * 16);
        const uint4 wb = lds_v4(stage + gi * 1024 + 512 + lane * 16);
        const uint32_t wA[4] = {wa.x, wa.y, wa.z, wa.w}, wB[4] = {wb.x, wb.y, wb.z, wb.w};
        uint4 xv[MT][2];
#pragma unroll
        for (int mt = 0; mt < MT; ++mt) {
            if (g + 8 * mt < M) {
                const int8_t* xr = xrow[mt] + gi * 128;
                if (XMODE == 2) {
                    xv[mt][0] = lds_v4(xr);
                    xv[mt][1] = lds_v4(xr + 16);
                } else if (XMODE == 3) {
                    xv[mt][0] = __ldcg(reinterpret_cast<const uint4*>(xr));
                    xv[mt][1] = __ldcg(reinterpret_cast<const uint4*>(xr + 16));
                } else {
                    xv[mt][0] = __ldg(reinterpret_cast<const uint4*>(xr));
                    xv[mt][1] = __ldg(reinterpret_cast<const uint4*>(xr + 16));
                }
            } else {
                xv[mt][0] = make_uint4(0, 0, 0, 0);
                xv[mt][1] = make_uint4(0, 0, 0, 0);
            }
        }
        uint32_t sbA = 0, sbB = 0;
        if constexpr (FMT == FMT_REF) {
            const uint8_t* sc = stage + kStageW;
            sbA = *reinterpret_cast<const uint16_t*>(sc + g * 64 + gi * 8 + 2 * t);
            sbB = *reinterpret_cast<const uint16_t*>(sc + (g + 8) * 64 + gi * 8 + 2 * t);
        }
        // two mma chains of depth 2 (k-steps 0,1 and 2,3), each started from the zero register
        int c0[MT][4], c1[MT][4];
#pragma unroll
        for (int s = 0; s < 4; ++s) {
            uint32_t a0, a1, a2, a3;
            if constexpr (FMT == FMT_GPTQ) {
                // two's complement nibbles (tile-major copies are re-coded by the repack; row-major
                // nibbles v + 8 are re-coded here) moved into the high half of each byte: 16 * v
                const uint32_t xa = LAYOUT == LAYOUT_ROW ? (wA[s] ^ 0x88888888u) : wA[s];
                const uint32_t xb = LAYOUT == LAYOUT_ROW ? (wB[s] ^ 0x88888888u) : wB[s];
                a0 = (xa << 4) & 0xF0F0F0F0u;
                a1 = (xb << 4) & 0xF0F0F0F0u;
                a2 = xa & 0xF0F0F0F0u;
                a3 = xb & 0xF0F0F0F0u;
            } else {
                ref_decode(pair_tab, wA[s], (sbA >> (8 * (s >> 1))) & 0xFF, a0, a2);
                ref_decode(pair_tab, wB[s], (sbB >> (8 * (s >> 1))) & 0xFF, a1, a3);
            }
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                uint32_t b0 = (s < 2) ? (s == 0 ? xv[mt][0].x : xv[mt][0].z) : (s == 2 ? xv[mt][1].x : xv[mt][1].z);
                uint32_t b1 = (s < 2) ? (s == 0 ? xv[mt][0].y : xv[mt][0].w) : (s == 2 ? xv[mt][1].y : xv[mt][1].w);
                if (XMODE == 0) {
                    const uint32_t lo = b0, hi = b1;
                    b0 = prmt(lo, hi, 0x6420);
                    b1 = prmt(lo, hi, 0x7531);
                }
                int(&c)[4] = (s < 2) ? c0[mt] : c1[mt];
                if ((s & 1) == 0)
                    mma_s8_16832_z(c, a0, a1, a2, a3, b0, b1, zero);
                else
                    mma_s8_16832(c, a0, a1, a2, a3, b0, b1);
            }
        }
        if constexpr (FMT == FMT_GPTQ) {
            const float sa = __half2float(sc16[g * 8 + gi]), sb = __half2float(sc16[(g + 8) * 8 + gi]);
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                // The dots carry the factor 16 of the shifted nibbles, and so do these products and sums:
                // scaling by 16 is exact in every step (|acc| < 2^21, no overflow, no subnormal), so the
                // partial is 16 * F bit for bit; tile_total() removes the factor.
#pragma unroll
                for (int i = 0; i < 4; ++i)
                    F[mt][i] = __fadd_rn(F[mt][i], __fmul_rn(__int2float_rn(c0[mt][i] + c1[mt][i]), i < 2 ? sa : sb));
            }
        } else {
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) A[mt][i] += c0[mt][i] + c1[mt][i];
        }
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) R[mt][i] = FMT == FMT_GPTQ ? __float_as_uint(F[mt][i]) : uint32_t(A[mt][i]);
}

template <int FMT, int LAYOUT, int MT, int ST, int XMODE>
__device__ __forceinline__ void consume_item_x(Ring<FMT, LAYOUT, ST>& r, const Program& P, const Seq& sq, const XSrc& xs,
                                               int M, int chunk, int lane, uint32_t (&R)[MT][4]) {
    const uint8_t* stage = r.wait();
    compute_item<FMT, LAYOUT, MT, XMODE>(stage, P.pair_tab, xs, M, chunk, lane, R);
    r.release(P, sq, lane);
}

template <int FMT, int LAYOUT, int MT, int ST>
__device__ __forceinline__ void consume_item(Ring<FMT, LAYOUT, ST>& r, const Program& P, const Seq& sq, const XSrc& xs,
                                             int M, int chunk, int lane, uint32_t (&R)[MT][4]) {
    // one warp-uniform branch per item; each body has only its own activation path
    if (xs.smem)
        consume_item_x<FMT, LAYOUT, MT, ST, 2>(r, P, sq, xs, M, chunk, lane, R);
    else if (xs.perm)
        consume_item_x<FMT, LAYOUT, MT, ST, 1>(r, P, sq, xs, M, chunk, lane, R);
    else
        consume_item_x<FMT, LAYOUT, MT, ST, 0>(r, P, sq, xs, M, chunk, lane, R);
}

// Partials of one warp-group tile: [item][MT * 8 rows][16 columns] 32-bit words.
template <int MT>
__device__ __forceinline__ void store_partial(uint32_t* part, int item, int lane, const uint32_t (&R)[MT][4]) {
    const int g = lane >> 2, t = lane & 3;
    uint32_t* pc = part + item * (MT * 8 * 16);
#pragma unroll
    for (int mt = 0; mt < MT; ++mt) {
        const int m0 = 2 * t + 8 * mt;
        pc[m0 * 16 + g] = R[mt][0];
        pc[(m0 + 1) * 16 + g] = R[mt][1];
        pc[m0 * 16 + g + 8] = R[mt][2];
        pc[(m0 + 1) * 16 + g + 8] = R[mt][3];
    }
}

// Total of subtile `sub` at (m, nl) over the C chunk partials, in chunk order (GPTQ: the factor 16 of the
// partials is removed exactly at the end).
template <int FMT, int MT>
__device__ __forceinline__ uint32_t tile_total(const uint32_t* part, int C, int sub, int m, int nl) {
    if constexpr (FMT == FMT_GPTQ) {
        float tot = 0.f;
        for (int c = 0; c < C; ++c) tot = __fadd_rn(tot, __uint_as_float(part[(sub * C + c) * (MT * 128) + m * 16 + nl]));
        return __float_as_uint(__fmul_rn(tot, 0.0625f));
    } else {
        uint32_t tot = 0;
        for (int c = 0; c < C; ++c) tot += part[(sub * C + c) * (MT * 128) + m * 16 + nl];
        return tot;
    }
}

__device__ __forceinline__ void group_sync(int wg) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + wg), "r"(kGroupWarps * 32) : "memory");
}

// Stage the activation block x [M][K] of a phase into shared memory (pitch K + 16), permuting the bytes
// unless x is permuted already. Two paths:
//  * vector loads by all threads (L2, every load of a batch in flight before any store) when the block is at
//    most 16 pieces of 16 bytes per thread: these bypass the TMA unit, whose queue is full of weight copies
//    while a phase starts (measured on B200: row copies queued behind the rings' and the L2 prefetches'
//    requests landed 1.5-2.5 us after issue; vector loads take one L2 round trip);
//  * otherwise one TMA bulk copy per row by thread 0, waited on (bounded) through xbar with `parity` (flipped
//    for the barrier's next phase), and the permutation in place.
// Returns false if a wait gave up. CTA-uniform result (the callers' tile loops hold warp-group barriers).
__device__ __forceinline__ uint4 perm16(uint4 v) {
    return make_uint4(prmt(v.x, v.y, 0x6420), prmt(v.x, v.y, 0x7531), prmt(v.z, v.w, 0x6420), prmt(v.z, v.w, 0x7531));
}

// One-batch vector staging split in two, so that other requests (the weight rings) can be issued while the
// activation loads are in flight: fits when the block is at most 8 pieces of 16 bytes per thread.
__device__ __forceinline__ bool stage_x_lsu_fits(const PhaseDesc& p, int M) { return M * (p.K >> 4) <= 8 * int(blockDim.x); }
__device__ __forceinline__ void stage_x_lsu_load(const PhaseDesc& p, int M, uint4 (&v)[8]) {
    const int T = blockDim.x, total = M * (p.K >> 4);
    const uint4* src = reinterpret_cast<const uint4*>(p.x);
#pragma unroll
    for (int j = 0; j < 8; ++j)
        if (int(threadIdx.x) + j * T < total) v[j] = __ldcg(src + threadIdx.x + j * T);
}
__device__ __forceinline__ void stage_x_lsu_store(const PhaseDesc& p, int M, int8_t* xsm, const uint4 (&v)[8]) {
    const int T = blockDim.x, words = p.K >> 4, total = M * words;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int i = threadIdx.x + j * T;
        if (i < total) {
            const int m = i / words, c = i - m * words;
            reinterpret_cast<uint4*>(xsm + size_t(m) * (p.K + 16))[c] = p.xperm ? v[j] : perm16(v[j]);
        }
    }
    __syncthreads();
}

__device__ __forceinline__ bool stage_x(const PhaseDesc& p, int M, int8_t* xsm, uint64_t* xbar, int& parity) {
    const int T = blockDim.x, words = p.K >> 4, total = M * words;
    if (total <= 16 * T) {
        const uint4* src = reinterpret_cast<const uint4*>(p.x);  // rows contiguous: piece i = (i / words, i % words)
        for (int base = threadIdx.x; base < total; base += 8 * T) {
            uint4 v[8];
#pragma unroll
            for (int j = 0; j < 8; ++j)
                if (base + j * T < total) v[j] = __ldcg(src + base + j * T);
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                const int i = base + j * T;
                if (i < total) {
                    const int m = i / words, c = i - m * words;
                    reinterpret_cast<uint4*>(xsm + size_t(m) * (p.K + 16))[c] = p.xperm ? v[j] : perm16(v[j]);
                }
            }
        }
        __syncthreads();
        return true;
    }
    if (threadIdx.x == 0) {
        // earlier generic accesses of the buffer (fragment reads, the permutation) before the async writes
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        asm volatile("fence.proxy.async.global;" ::: "memory");
        mbar_arrive_expect_tx(xbar, uint32_t(M) * p.K);
        for (int i = 0; i < M; ++i) {
            const int m = (i + int(blockIdx.x)) % M;  // CTAs start at different rows
            bulk_g2s(xsm + size_t(m) * (p.K + 16), p.x + size_t(m) * p.K, p.K, xbar);
        }
    }
    const bool ok = __syncthreads_and(mbar_wait(xbar, parity));
    parity ^= 1;
    if (!p.xperm) {
        for (int m = 0; m < M; ++m) {
            uint4* row = reinterpret_cast<uint4*>(xsm + size_t(m) * (p.K + 16));
            for (int c = threadIdx.x; c < words; c += T) row[c] = perm16(row[c]);
        }
        __syncthreads();
    }
    return ok;
}

// Shared-memory plan of an engine kernel (bytes): rings, ring barriers, partials, staged activations.
template <int FMT, int MT>
struct SmemPlan {
    size_t rings, bars, part, x, total;
    __host__ __device__ SmemPlan(int groups, int stages, int max_items, int x_bytes) {
        rings = size_t(groups) * kGroupWarps * stages * stage_bytes<FMT>();
        bars = (size_t(groups) * kGroupWarps * stages * 8 + 8 + 127) / 128 * 128;  // ring barriers + xbar
        part = size_t(groups) * 2 * max_items * MT * 128 * 4;
        x = size_t(x_bytes + 127) / 128 * 128;
        total = rings + bars + part + x;
    }
};

}  // namespace mono
