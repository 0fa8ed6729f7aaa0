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
// kGroups warp-groups of 4 warps; each warp-group is a virtual CTA that takes tiles round-robin, its
// warps take a tile's items round-robin, and the chunk partials meet in shared memory where one thread
// per output sums them in chunk order. Every warp streams its items through a private ring of 2-group
// stages (2 KB of weights + scales): TMA bulk copies for tile-major weights, cp.async for the
// checkpoint's row-major weights. The producer cursor walks the warp's stages across all phases, so the
// next phase's weights are in flight while the CTA waits at a grid barrier. Activations of a phase are
// staged once per CTA in shared memory (pitch K + 16 bytes: the fragment reads are conflict-free) when
// they fit, otherwise read from L2.
//
// mma fragment mapping (swap-AB: weights are the 16-row A operand, activations the 8-column B operand).
// Inside a 128-group lane (g, t) owns bytes [16t, 16t + 16) of rows g and g + 8, i.e. packed words
// 4t + s (s = 0..3). At k-step s its word's even nibbles are A columns 4t..4t+3 and its odd nibbles A
// columns 16 + 4t..; the activation bytes of those columns are x[8(4t + s) + {0,2,4,6}] and
// x[8(4t + s) + {1,3,5,7}] of the group: 32 contiguous bytes per lane and group.
#pragma once
#include "common.cuh"

namespace mono {

enum W4Format : int { FMT_GPTQ = 0, FMT_REF = 1 };
enum W4Layout : int { LAYOUT_ROW = 0, LAYOUT_TILED = 1 };

constexpr int kGroupWarps = 4;   // warps per warp-group
constexpr int kStages = 4;       // ring depth per warp
constexpr int kStageW = 2048;    // weight bytes per stage (2 groups x 16 rows x 64 B)
constexpr int kChunkK = 1024;    // K per item
constexpr int kMaxChunks = 16;   // K <= 16384
constexpr int kMaxPhases = 4;
constexpr int kXStageMax = 98304;  // largest activation block staged in shared memory (M * K bytes)

template <int FMT>
struct Fmt;
template <>
struct Fmt<FMT_GPTQ> {
    static constexpr int SB = 64;  // scale bytes per stage: [16 rows][2 groups] fp16
};
template <>
struct Fmt<FMT_REF> {
    static constexpr int SB = 256;  // [16 rows][16 fp8] (2 groups x 8 G16 scales)
};
template <int FMT>
__host__ __device__ constexpr int stage_bytes() { return kStageW + Fmt<FMT>::SB; }

struct MatDesc {
    const uint8_t* q;  // TILED: [N/16][K/128][2][32][16]; ROW: [N][K/2] bytes (low nibble = even k)
    const uint8_t* s;  // GPTQ fp16 / REF fp8 scales, TILED [N/16][K/256][16][SB/16] or ROW [N][K/g]
    int n;
};

struct PhaseDesc {
    MatDesc m[3];
    int nm, paired, K;
    const int8_t* x;  // activation rows [M][K] (row stride K)
    int xsmem;        // 1: staged in shared memory
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
    int ph, ti, it, pair;
    bool done;
};

// The stage sequence of one warp: virtual CTA vc of nvc, warp `warp` of its group.
struct Seq {
    int warp, vc, nvc;
    __device__ int my_tiles(const Program& P, int ph) const {
        const int t = phase_tiles(P.ph[ph]);
        return vc < t ? (t - 1 - vc) / nvc + 1 : 0;
    }
    __device__ int my_items(const Program& P, int ph) const {
        const int it = phase_items(P.ph[ph]);
        return warp < it ? (it - 1 - warp) / kGroupWarps + 1 : 0;
    }
    __device__ Cursor start(const Program& P, int ph) const {
        Cursor c{ph, 0, 0, 0, false};
        while (c.ph < P.nph && (my_tiles(P, c.ph) == 0 || my_items(P, c.ph) == 0)) ++c.ph;
        c.done = c.ph >= P.nph;
        return c;
    }
    __device__ void advance(const Program& P, Cursor& c) const {
        if (++c.pair < 4) return;
        c.pair = 0;
        if (++c.it < my_items(P, c.ph)) return;
        c.it = 0;
        if (++c.ti < my_tiles(P, c.ph)) return;
        c = start(P, c.ph + 1);
    }
};

template <int FMT, int LAYOUT>
__device__ __forceinline__ void issue_stage(const Program& P, const Seq& sq, const Cursor& c, uint8_t* stage,
                                            uint64_t* bar, int lane) {
    constexpr int SB = Fmt<FMT>::SB;
    const PhaseDesc& p = P.ph[c.ph];
    const int T = sq.vc + c.ti * sq.nvc;
    const int item = sq.warp + c.it * kGroupWarps;
    const int C = phase_chunks(p);
    const int sub = item / C, chunk = item - sub * C;
    int mat, lt;
    resolve(p, T, sub, mat, lt);
    const MatDesc& w = p.m[mat];
    const int G = p.K >> 7;
    const int g0 = chunk * 8 + c.pair * 2;
    if constexpr (LAYOUT == LAYOUT_TILED) {
        if (lane == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive_expect_tx(bar, kStageW + SB);
            bulk_g2s(stage, w.q + (size_t(lt) * G + g0) * 1024, kStageW, bar);
            bulk_g2s(stage + kStageW, w.s + (size_t(lt) * (G >> 1) + (g0 >> 1)) * SB, SB, bar);
        }
    } else {
        const int g = lane >> 2, t = lane & 3;
        const size_t rowb = size_t(p.K) >> 1;
        const uint8_t* r0 = w.q + size_t(lt * 16 + g) * rowb + size_t(g0) * 64 + t * 16;
        const uint8_t* r1 = r0 + 8 * rowb;
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
            cp_async16(stage + gi * 1024 + lane * 16, r0 + gi * 64);
            cp_async16(stage + gi * 1024 + 512 + lane * 16, r1 + gi * 64);
        }
        if (lane < 16) {
            const int row = lt * 16 + lane;
            if constexpr (FMT == FMT_GPTQ) {
                const uint8_t* s = w.s + (size_t(row) * G + g0) * 2;
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(stage + kStageW + lane * 4)),
                             "l"(s)
                             : "memory");
            } else {
                cp_async16(stage + kStageW + lane * 16, w.s + size_t(row) * (p.K >> 4) + g0 * 8);
            }
        }
        cp_async_commit();
    }
}

template <int FMT, int LAYOUT>
struct Ring {
    uint8_t* buf;
    uint64_t* bars;
    Cursor prod;
    int issued, consumed;
    bool ok;

    __device__ void init(const Program& P, const Seq& sq, int lane) {
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
                issue_stage<FMT, LAYOUT>(P, sq, prod, buf + (issued % kStages) * stage_bytes<FMT>(),
                                         &bars[issued % kStages], lane);
                ++issued;
                sq.advance(P, prod);
            } else if (LAYOUT == LAYOUT_ROW) {
                cp_async_commit();
            }
        }
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
            issue_stage<FMT, LAYOUT>(P, sq, prod, buf + slot * stage_bytes<FMT>(), &bars[slot], lane);
            ++issued;
            sq.advance(P, prod);
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

// Activation source of a phase: shared (pitch K + 16) or global (pitch K).
struct XSrc {
    const int8_t* p;
    int pitch;
    bool smem;
};

// Consume one item (4 stages = 8 groups). R = the chunk partial per fragment element: fp32 bits (GPTQ)
// or the int32 dot (REF). Fragment element i of m-tile mt: (row g + 8 (i >> 1), activation 2t + (i & 1)).
template <int FMT, int LAYOUT, int MT>
__device__ __forceinline__ void consume_item(Ring<FMT, LAYOUT>& r, const Program& P, const Seq& sq, const XSrc& xs,
                                             int M, int chunk, int lane, uint32_t (&R)[MT][4]) {
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
    for (int pair = 0; pair < 4; ++pair) {
        uint8_t* stage = r.wait();
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
            const int grp = chunk * 8 + pair * 2 + gi;
            const uint4 wa = lds_v4(stage + gi * 1024 + lane * 16);
            const uint4 wb = lds_v4(stage + gi * 1024 + 512 + lane * 16);
            const uint32_t wA[4] = {wa.x, wa.y, wa.z, wa.w}, wB[4] = {wb.x, wb.y, wb.z, wb.w};
            uint4 xv[MT][2];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int m = g + 8 * mt;
                if (m < M) {
                    const int8_t* xr = xs.p + size_t(m) * xs.pitch + grp * 128 + 32 * t;
                    if (xs.smem) {
                        xv[mt][0] = lds_v4(xr);
                        xv[mt][1] = lds_v4(xr + 16);
                    } else {
                        xv[mt][0] = __ldcg(reinterpret_cast<const uint4*>(xr));
                        xv[mt][1] = __ldcg(reinterpret_cast<const uint4*>(xr + 16));
                    }
                } else {
                    xv[mt][0] = make_uint4(0, 0, 0, 0);
                    xv[mt][1] = make_uint4(0, 0, 0, 0);
                }
            }
            int acc[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) acc[mt][i] = 0;
            uint32_t sbA = 0, sbB = 0;
            if constexpr (FMT == FMT_REF) {
                const uint8_t* sc = stage + kStageW;
                sbA = *reinterpret_cast<const uint16_t*>(sc + g * 16 + gi * 8 + 2 * t);
                sbB = *reinterpret_cast<const uint16_t*>(sc + (g + 8) * 16 + gi * 8 + 2 * t);
            }
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
                    ref_decode(P.pair_tab, wA[s], (sbA >> (8 * (s >> 1))) & 0xFF, a0, a2);
                    ref_decode(P.pair_tab, wB[s], (sbB >> (8 * (s >> 1))) & 0xFF, a1, a3);
                }
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    const uint32_t lo = (s < 2) ? (s == 0 ? xv[mt][0].x : xv[mt][0].z) : (s == 2 ? xv[mt][1].x : xv[mt][1].z);
                    const uint32_t hi = (s < 2) ? (s == 0 ? xv[mt][0].y : xv[mt][0].w) : (s == 2 ? xv[mt][1].y : xv[mt][1].w);
                    if constexpr (FMT == FMT_GPTQ)
                        mma_s8_16832(acc[mt], a0, a1, a2, a3, prmt(lo, hi, 0x6420), prmt(lo, hi, 0x7531));
                    else
                        mma_s8_16832(A[mt], a0, a1, a2, a3, prmt(lo, hi, 0x6420), prmt(lo, hi, 0x7531));
                }
            }
            if constexpr (FMT == FMT_GPTQ) {
                const __half* sc = reinterpret_cast<const __half*>(stage + kStageW);
                const float sa = __half2float(sc[g * 2 + gi]), sb = __half2float(sc[(g + 8) * 2 + gi]);
#pragma unroll
                for (int mt = 0; mt < MT; ++mt) {
                    // the int32 dots carry the factor 16 of the shifted nibbles: exact >> 4
                    F[mt][0] = __fadd_rn(F[mt][0], __fmul_rn(__int2float_rn(acc[mt][0] >> 4), sa));
                    F[mt][1] = __fadd_rn(F[mt][1], __fmul_rn(__int2float_rn(acc[mt][1] >> 4), sa));
                    F[mt][2] = __fadd_rn(F[mt][2], __fmul_rn(__int2float_rn(acc[mt][2] >> 4), sb));
                    F[mt][3] = __fadd_rn(F[mt][3], __fmul_rn(__int2float_rn(acc[mt][3] >> 4), sb));
                }
            }
        }
        r.release(P, sq, lane);
    }
#pragma unroll
    for (int mt = 0; mt < MT; ++mt)
#pragma unroll
        for (int i = 0; i < 4; ++i) R[mt][i] = FMT == FMT_GPTQ ? __float_as_uint(F[mt][i]) : uint32_t(A[mt][i]);
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

// Total of subtile `sub` at (m, nl) over the C chunk partials, in chunk order.
template <int FMT, int MT>
__device__ __forceinline__ uint32_t tile_total(const uint32_t* part, int C, int sub, int m, int nl) {
    if constexpr (FMT == FMT_GPTQ) {
        float tot = 0.f;
        for (int c = 0; c < C; ++c) tot = __fadd_rn(tot, __uint_as_float(part[(sub * C + c) * (MT * 128) + m * 16 + nl]));
        return __float_as_uint(tot);
    } else {
        uint32_t tot = 0;
        for (int c = 0; c < C; ++c) tot += part[(sub * C + c) * (MT * 128) + m * 16 + nl];
        return tot;
    }
}

__device__ __forceinline__ void group_sync(int wg) {
    asm volatile("bar.sync %0, %1;" ::"r"(1 + wg), "r"(kGroupWarps * 32) : "memory");
}

// Stage the activation block x [M][K] of a phase into shared memory (pitch K + 16): one bulk copy per row.
__device__ __forceinline__ void stage_x(const PhaseDesc& p, int M, int8_t* xsm, uint64_t* xbar) {
    if (threadIdx.x == 0) {
        asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
        mbar_arrive_expect_tx(xbar, uint32_t(M) * p.K);
        for (int m = 0; m < M; ++m) bulk_g2s(xsm + size_t(m) * (p.K + 16), p.x + size_t(m) * p.K, p.K, xbar);
    }
}

// Shared-memory plan of an engine kernel (bytes): rings, ring barriers, the x barrier, partials, x.
template <int FMT, int MT>
struct SmemPlan {
    size_t rings, bars, part, x, total;
    __host__ __device__ SmemPlan(int groups, int max_items, int x_bytes) {
        rings = size_t(groups) * kGroupWarps * kStages * stage_bytes<FMT>();
        bars = size_t(groups) * kGroupWarps * kStages * 8 + 16;
        part = size_t(groups) * 2 * max_items * MT * 128 * 4;
        x = size_t(x_bytes + 127) / 128 * 128;
        total = rings + bars + part + x;
    }
};

}  // namespace mono
