// W4A8 decode GEMV for 1..16 activation rows (the tree-verify rows of a decode step).
//
// out[m, n] for two weight formats that share one int4 unpack / int8 tensor-core dot:
//   GPTQ  int4 symmetric v in [-8, 7] stored as nibble v + 8, fp16 scale per (row, 128-group):
//           acc_g  = int32 sum_{k in group g} xq[m, k] * v[n, k]
//           F_c    = fp32 sequential sum over the 8 groups of 1024-chunk c of float(acc_g) * float(s[n, g])
//           total  = fp32 sequential sum over chunks c of F_c,     out = bf16(total * xs[m])
//         (every sum starts from +0, each product and sum is one IEEE RNE op, never fused)
//   REF   the reference's packed W4A8 (csrc/w4a8_decode.sycl:4-11, :35-45, :150-163): 4-bit codes into an
//         fp32 codebook, FP8 e4m3 relative scale per (row, 16-group), fp32 channel scale:
//           w_i8   = isnan(r) ? 0 : clamp(r, -127, 127),  r = rint(codebook[code] * s_rel)
//           acc    = int32 (mod 2^32) sum over all of K of xq * w_i8
//           out    = cast(float(acc) * xs[m] * s_channel[n])  (two fp32 multiplies, then one cast)
//         optional residual: out = cast(float(residual) + float(cast(f)))  (w4a8_decode.sycl:155-160)
//
// Work split: a 16-row output tile is one CTA work item; its K is cut into 1024-wide chunks that the
// CTA's warps take round-robin. A warp streams its chunk as 2-group (2 KB) stages through a private ring
// in shared memory, filled either by the TMA bulk-copy unit (tile-major weights) or by cp.async
// (row-major weights). Chunk partials meet in shared memory and one thread per output sums them in
// chunk order. CTAs are persistent over tiles; the next tile's stages are in flight while a tile's
// epilogue runs.
//
// mma fragment mapping (swap-AB: weights are the 16-row A operand, activations the 8-column B operand).
// Inside a 128-group, lane (g, t) owns bytes [16t, 16t + 16) of rows g and g + 8, i.e. packed words
// 4t + s (s = 0..3). At k-step s its word's even nibbles are A columns 4t..4t+3 and its odd nibbles A
// columns 16 + 4t..; the activation bytes for those columns are x[8(4t + s) + {0,2,4,6}] and
// x[8(4t + s) + {1,3,5,7}] of the group, which the same lane reads as 32 contiguous bytes. Every group's
// int32 dot is therefore complete inside one warp's 4 k-steps.
#pragma once
#include "common.cuh"

namespace mono {

enum W4Format : int { FMT_GPTQ = 0, FMT_REF = 1 };
enum W4Layout : int { LAYOUT_ROW = 0, LAYOUT_TILED = 1 };

constexpr int kGemvWarps = 4;          // warps per CTA
constexpr int kGemvStages = 4;         // ring depth per warp (2 groups = 2 KB of weights per stage)
constexpr int kStageW = 2048;          // weight bytes per stage
constexpr int kChunkK = 1024;          // K per chunk (8 groups)
constexpr int kMaxChunks = 16;         // K <= 16384

template <int FMT>
struct ScaleBytes;  // scale bytes per stage: [16 rows][2 groups]
template <>
struct ScaleBytes<FMT_GPTQ> { static constexpr int value = 16 * 2 * 2; };   // fp16
template <>
struct ScaleBytes<FMT_REF> { static constexpr int value = 16 * 16; };      // 8 fp8 per group

struct GemvParams {
    const uint8_t* q;          // ROW: [N][K/2] bytes (low nibble = even k); TILED: [N/16][K/128][2][32][16]
    const uint8_t* scales;     // GPTQ fp16 [N][K/128] (ROW) / [N/16][K/256][16][2] (TILED);
                               // REF fp8 [N][K/16] (ROW) / [N/16][K/256][16][16] (TILED)
    const float* s_channel;    // REF: [N]
    const uint16_t* pair_tab;  // REF: [256 scale bytes][256 code bytes] -> int8 (low code) | int8 (high) << 8
    const int8_t* x;           // [M][K]
    const float* xs;           // [M]
    const void* residual;      // [M][N] in the output dtype, or null
    void* out;                 // [M][N]
    int M, N, K;
    int out_bf16;              // 1: bf16 output, 0: fp32 output
};

template <int FMT>
__host__ __device__ constexpr int stage_bytes() { return kStageW + ScaleBytes<FMT>::value; }

template <int FMT>
inline size_t gemv_smem_bytes(int chunks) {
    // rings + mbarriers + double-buffered chunk partials [2][chunks][16 m][16 n] (4 B each)
    return size_t(kGemvWarps) * kGemvStages * stage_bytes<FMT>() + kGemvWarps * kGemvStages * 8 +
           size_t(2) * chunks * 16 * 16 * 4;
}

// ---- per-stage producers ----------------------------------------------------------------------------
// Stage j of a warp's sequence covers groups 2 * pair .. 2 * pair + 1 of chunk `chunk` of tile `tile`.
template <int FMT, int LAYOUT>
__device__ __forceinline__ void issue_stage(const GemvParams& p, uint8_t* stage, uint64_t* bar, int tile,
                                            int chunk, int pair, int lane) {
    const int G = p.K >> 7;                   // groups per row
    const int g0 = chunk * 8 + pair * 2;      // first group of the stage
    constexpr int SB = ScaleBytes<FMT>::value;
    if constexpr (LAYOUT == LAYOUT_TILED) {
        if (lane == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            mbar_arrive_expect_tx(bar, kStageW + SB);
            bulk_g2s(stage, p.q + (size_t(tile) * G + g0) * 1024, kStageW, bar);
            bulk_g2s(stage + kStageW, p.scales + (size_t(tile) * (G >> 1) + (g0 >> 1)) * SB, SB, bar);
        }
    } else {
        const int g = lane >> 2, t = lane & 3;
        const size_t rowb = size_t(p.K) >> 1;
        const uint8_t* r0 = p.q + size_t(tile * 16 + g) * rowb + size_t(g0) * 64 + t * 16;
        const uint8_t* r1 = r0 + 8 * rowb;
#pragma unroll
        for (int gi = 0; gi < 2; ++gi) {
            cp_async16(stage + gi * 1024 + lane * 16, r0 + gi * 64);
            cp_async16(stage + gi * 1024 + 512 + lane * 16, r1 + gi * 64);
        }
        // scales of the 16 rows for the stage's 2 groups: [16 rows][SB / 16 bytes]
        if (lane < 16) {
            const int row = tile * 16 + lane;
            if constexpr (FMT == FMT_GPTQ) {
                const uint8_t* s = p.scales + (size_t(row) * G + g0) * 2;  // 2 fp16 = 4 B, 4 B aligned
                asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_u32(stage + kStageW + lane * 4)),
                             "l"(s)
                             : "memory");
            } else {
                const uint8_t* s = p.scales + size_t(row) * (p.K >> 4) + g0 * 8;  // 16 fp8 = 16 B
                cp_async16(stage + kStageW + lane * 16, s);
            }
        }
        cp_async_commit();
    }
}

// ---- REF decode of one packed word (8 codes sharing one fp8 scale byte) -------------------------------
__device__ __forceinline__ void ref_decode(const uint16_t* __restrict__ tab, uint32_t word, uint32_t sb,
                                           uint32_t& even, uint32_t& odd) {
    const uint16_t* row = tab + (sb << 8);
    const uint32_t e0 = __ldg(row + (word & 0xFF)), e1 = __ldg(row + ((word >> 8) & 0xFF));
    const uint32_t e2 = __ldg(row + ((word >> 16) & 0xFF)), e3 = __ldg(row + (word >> 24));
    const uint32_t r01 = e0 | (e1 << 16), r23 = e2 | (e3 << 16);
    even = prmt(r01, r23, 0x6420);
    odd = prmt(r01, r23, 0x7531);
}

// ---- the kernel ---------------------------------------------------------------------------------------
// MT = activation m-tiles of 8 rows (1: M <= 8, 2: M <= 16).
template <int FMT, int LAYOUT, int MT>
__global__ void __launch_bounds__(kGemvWarps * 32) w4a8_gemv_kernel(const GemvParams p) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int SBYTES = stage_bytes<FMT>();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, t = lane & 3;
    uint8_t* ring = smem + size_t(warp) * kGemvStages * SBYTES;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + size_t(kGemvWarps) * kGemvStages * SBYTES) +
                     warp * kGemvStages;
    float* partials = reinterpret_cast<float*>(smem + size_t(kGemvWarps) * kGemvStages * SBYTES +
                                               kGemvWarps * kGemvStages * 8);

    const int ntiles = p.N >> 4, C = p.K / kChunkK;
    const int my_chunks = C > warp ? (C - 1 - warp) / kGemvWarps + 1 : 0;
    const int my_tiles = blockIdx.x < ntiles ? (ntiles - 1 - blockIdx.x) / gridDim.x + 1 : 0;
    const int total = my_tiles * my_chunks * 4;  // stages in this warp's sequence

    if (LAYOUT == LAYOUT_TILED && lane == 0) {
        for (int i = 0; i < kGemvStages; ++i) mbar_init(&bars[i], 1);
        fence_mbar_init();
    }
    __syncwarp();
    auto coords = [&](int j, int& tile, int& chunk, int& pair) {
        const int per_tile = my_chunks * 4;
        const int ti = j / per_tile, r = j - ti * per_tile;
        tile = blockIdx.x + ti * gridDim.x;
        chunk = warp + (r >> 2) * kGemvWarps;
        pair = r & 3;
    };
    // The weights do not depend on the previous kernel in the stream: start streaming them before the
    // dependency wait (programmatic dependent launch), then wait before reading activations.
    for (int j = 0; j < kGemvStages; ++j) {
        if (j < total) {
            int tile, chunk, pair;
            coords(j, tile, chunk, pair);
            issue_stage<FMT, LAYOUT>(p, ring + j * SBYTES, &bars[j], tile, chunk, pair, lane);
        } else if (LAYOUT == LAYOUT_ROW) {
            cp_async_commit();  // keep the group count uniform
        }
    }
    pdl_wait();

    bool ok = true;
    int j = 0;
    for (int ti = 0; ti < my_tiles; ++ti) {
        const int tile = blockIdx.x + ti * gridDim.x;
        float* part = partials + (ti & 1) * (C * 256);
        for (int ci = 0; ci < my_chunks; ++ci) {
            const int chunk = warp + ci * kGemvWarps;
            float F[MT][4];
            int A[MT][4];
#pragma unroll
            for (int mt = 0; mt < MT; ++mt)
#pragma unroll
                for (int i = 0; i < 4; ++i) { F[mt][i] = 0.f; A[mt][i] = 0; }
            for (int pair = 0; pair < 4; ++pair, ++j) {
                const int slot = j % kGemvStages;
                uint8_t* stage = ring + slot * SBYTES;
                if constexpr (LAYOUT == LAYOUT_TILED) {
                    if (ok) ok = mbar_wait(&bars[slot], (j / kGemvStages) & 1);
                } else {
                    cp_async_wait<kGemvStages - 1>();
                    __syncwarp();
                }
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
                        if (m < p.M) {
                            const int8_t* xr = p.x + size_t(m) * p.K + grp * 128 + 32 * t;
                            xv[mt][0] = ldg_nc_v4(xr);
                            xv[mt][1] = ldg_nc_v4(xr + 16);
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
                        // fp8 scale bytes of words s = 0,1 (G16 index 2t) and s = 2,3 (2t + 1), rows g, g + 8
                        const uint8_t* sc = stage + kStageW;
                        sbA = *reinterpret_cast<const uint16_t*>(sc + g * 16 + gi * 8 + 2 * t);
                        sbB = *reinterpret_cast<const uint16_t*>(sc + (g + 8) * 16 + gi * 8 + 2 * t);
                    }
#pragma unroll
                    for (int s = 0; s < 4; ++s) {
                        uint32_t a0, a1, a2, a3;
                        if constexpr (FMT == FMT_GPTQ) {
                            // nibbles are stored as two's complement (tile-major: XORed by the repack;
                            // row-major: XORed here) and shifted into the high half of each byte: 16 * v
                            const uint32_t xa = LAYOUT == LAYOUT_ROW ? (wA[s] ^ 0x88888888u) : wA[s];
                            const uint32_t xb = LAYOUT == LAYOUT_ROW ? (wB[s] ^ 0x88888888u) : wB[s];
                            a0 = (xa << 4) & 0xF0F0F0F0u;
                            a1 = (xb << 4) & 0xF0F0F0F0u;
                            a2 = xa & 0xF0F0F0F0u;
                            a3 = xb & 0xF0F0F0F0u;
                        } else {
                            ref_decode(p.pair_tab, wA[s], (sbA >> (8 * (s >> 1))) & 0xFF, a0, a2);
                            ref_decode(p.pair_tab, wB[s], (sbB >> (8 * (s >> 1))) & 0xFF, a1, a3);
                        }
#pragma unroll
                        for (int mt = 0; mt < MT; ++mt) {
                            const uint32_t lo = (s < 2) ? (s == 0 ? xv[mt][0].x : xv[mt][0].z)
                                                        : (s == 2 ? xv[mt][1].x : xv[mt][1].z);
                            const uint32_t hi = (s < 2) ? (s == 0 ? xv[mt][0].y : xv[mt][0].w)
                                                        : (s == 2 ? xv[mt][1].y : xv[mt][1].w);
                            const uint32_t b0 = prmt(lo, hi, 0x6420), b1 = prmt(lo, hi, 0x7531);
                            if constexpr (FMT == FMT_GPTQ)
                                mma_s8_16832(acc[mt], a0, a1, a2, a3, b0, b1);
                            else
                                mma_s8_16832(A[mt], a0, a1, a2, a3, b0, b1);
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
                // the slot is consumed: refill it with stage j + kGemvStages
                __syncwarp();
                const int jn = j + kGemvStages;
                if (jn < total && ok) {
                    int tn, cn, pn;
                    coords(jn, tn, cn, pn);
                    issue_stage<FMT, LAYOUT>(p, stage, &bars[slot], tn, cn, pn, lane);
                } else if (LAYOUT == LAYOUT_ROW) {
                    cp_async_commit();
                }
            }
            // chunk partial -> shared [chunk][m][n]
#pragma unroll
            for (int mt = 0; mt < MT; ++mt) {
                const int m0 = 2 * t + 8 * mt;
                float* pc = part + chunk * 256;
                if constexpr (FMT == FMT_GPTQ) {
                    pc[m0 * 16 + g] = F[mt][0];
                    pc[(m0 + 1) * 16 + g] = F[mt][1];
                    pc[m0 * 16 + g + 8] = F[mt][2];
                    pc[(m0 + 1) * 16 + g + 8] = F[mt][3];
                } else {
                    int* pi = reinterpret_cast<int*>(pc);
                    pi[m0 * 16 + g] = A[mt][0];
                    pi[(m0 + 1) * 16 + g] = A[mt][1];
                    pi[m0 * 16 + g + 8] = A[mt][2];
                    pi[(m0 + 1) * 16 + g + 8] = A[mt][3];
                }
            }
        }
        __syncthreads();
        // epilogue: one thread per (m, n) of the tile sums the chunk partials in chunk order
        for (int e = threadIdx.x; e < p.M * 16; e += blockDim.x) {
            const int m = e >> 4, nl = e & 15, n = tile * 16 + nl;
            float f;
            if constexpr (FMT == FMT_GPTQ) {
                float total_ = 0.f;
                for (int c = 0; c < C; ++c) total_ = __fadd_rn(total_, part[c * 256 + m * 16 + nl]);
                f = __fmul_rn(total_, p.xs[m]);
            } else {
                const int* pi = reinterpret_cast<const int*>(part);
                uint32_t acc = 0;
                for (int c = 0; c < C; ++c) acc += uint32_t(pi[c * 256 + m * 16 + nl]);
                f = __fmul_rn(__int2float_rn(int(acc)), p.xs[m]);
                f = __fmul_rn(f, p.s_channel[n]);
            }
            const size_t o = size_t(m) * p.N + n;
            if (p.out_bf16) {
                uint16_t r = f32_to_bf16_bits(f);
                if (p.residual)
                    r = f32_to_bf16_bits(
                        __fadd_rn(bf16_bits_to_f32(static_cast<const uint16_t*>(p.residual)[o]), bf16_bits_to_f32(r)));
                static_cast<uint16_t*>(p.out)[o] = r;
            } else {
                if (p.residual) f = __fadd_rn(static_cast<const float*>(p.residual)[o], f);
                static_cast<float*>(p.out)[o] = f;
            }
        }
    }
    if (LAYOUT == LAYOUT_ROW) cp_async_wait<0>();
    if (LAYOUT == LAYOUT_TILED && !ok && lane == 0) {
        // a wait gave up (error recorded): wait, again bounded, for the copies this warp still has in
        // flight before the CTA's shared memory is released
        for (int k = j; k < total && k < j + kGemvStages; ++k) mbar_wait(&bars[k % kGemvStages], (k / kGemvStages) & 1);
    }
    // allow the next kernel in the stream to start its prologue
    pdl_launch_dependents();
}

}  // namespace mono
