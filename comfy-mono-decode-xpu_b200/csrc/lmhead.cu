// bf16 lm_head with the greedy / draft pick fused (the role of the reference's verify logits + argmax, and of its
// draft pick, csrc/draft_lmhead.sycl:87-292): for M <= 16 rows of x [M][K] against W [V][K] (bf16, far larger than
// L2), logits = bf16(x W^T) on the tensor cores, and per row the argmax (argmax rank: smallest index on ties) and
// the top-k (k <= 8, top-k rank), without writing the logits (optional).
//
// Work: a persistent grid of one CTA per SM, 8 warps each; warp j of CTA b takes the tiles of 8 vocabulary rows
// b * 8 + j, + G * 8, ... For each tile it streams the rows in chunks of 512 k: lanes 0..7 each copy one row's 1 KB
// (a bulk copy, evict-first, completion on the stage's mbarrier) into the warp's own ring of S stages (rows 16-byte
// skewed: conflict-free ldmatrix), so every request is a contiguous kilobyte and the ring keeps S chunks per warp
// in flight. The MMA is m16n8k16 with A = the x rows (rows past M zero) and B = the 8 weight rows, both read with
// ldmatrix; two accumulators take alternate k-steps of the tile and are added at its end (one fixed partition and
// order: the same bits on every launch), then rounded once to bf16.
//
// Pick: thread (g, t) of a warp holds rows g and g + 8's logits at columns 2t, 2t + 1 of each tile and keeps those
// rows' running top-k lists and argmaxes in registers; at the end the CTA merges its 32 lists per row and writes them to the
// workspace; the last CTA to finish (an arrival counter) merges the CTAs' lists - ranks are distinct, so the merge
// order does not matter - and writes the indices. The pick form then scatters the draft's tokens into the verify-token row: dst[children[0]] =
// argmax, dst[children[j]] = top-k[j] (j >= 1), the reference's draft pick (csrc/draft_lmhead.sycl:4-17).
#include <algorithm>
#include <mutex>

#include "launch.h"
#include "ranks.cuh"

namespace mono {

constexpr int kLhWarps = 8, kLhMaxM = 16, kLhRows = 8, kLhChunk = 512;
constexpr int kLhRowPitch = kLhChunk * 2 + 16;   // bytes per staged weight row (16-byte skew: conflict-free ldmatrix)
constexpr int kLhStage = kLhRows * kLhRowPitch;  // one ring stage: 8 rows x 512 k
constexpr size_t kLhSmemLimit = 227 * 1024 - 8 * 1024;  // dynamic bytes: the opt-in maximum less the static ones

// A rows 0..7 (a0, a2) and 8..15 (a1, a3: zero registers when M <= 8) are x rows
__device__ __forceinline__ void lh_mma(float (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                       uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0, %1, %2, %3}, {%4, %5, %6, %7}, {%8, %9}, "
        "{%0, %1, %2, %3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}
__device__ __forceinline__ void lh_ldsm_x4(uint32_t (&r)[4], const void* p) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0, %1, %2, %3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(smem_u32(p)));
}

struct LmHeadArgs {
    const uint16_t* x;        // [M][x_stride] bf16
    const uint16_t* w;        // [V][K] bf16
    uint16_t* logits;         // [M][V] bf16 or null
    int64_t* argmax;          // [M] or null
    int64_t* topk;            // [M][k] or null (k = 0: none)
    const int32_t* children;  // pick form: up to 8 slots of a dst row, -1 ends, or null
    int64_t* dst;             // pick form: the verify-token rows, row m's at dst + m * dst_stride
    int64_t dst_stride;
    uint64_t* ws;             // the arrival counter (first 256 bytes), then [G][kLhMaxM][kTkK + 1] CTA lists
    int64_t x_stride, out_stride;  // out_stride: the logits' row stride (V for the pick)
    int64_t index_base;            // the pick's index of row 0 of w (a vocabulary shard's offset; 0 otherwise)
    int K, V, M, k;
    int ks;  // K slices per tile (1, 2, 4 or 8; lmhead_split)
};

size_t lmhead_workspace_bytes(int grid) { return size_t(grid) * kLhMaxM * (kTkK + 1) * 8 + 256; }

// Shared memory of one CTA: the warps' rings [warp][S][stage], their barriers, then x [M][K + 8] and a 16-byte zero
// row (the ldmatrix rows of x past M). The pick's lists reuse the ring area after the last chunk.
struct LhPlan {
    size_t rings, bars, x, total;
    __host__ __device__ LhPlan(int M, int K, int S) {
        rings = size_t(kLhWarps) * S * kLhStage;
        bars = (size_t(kLhWarps) * S * 8 + 127) / 128 * 128;
        x = size_t(M) * (K + 8) * 2 + 16;
        total = rings + bars + x;
    }
};

// PICK = false: the plain bf16 GEMV (the draft head's projections): logits = out [M][out_stride], no pick.
template <int S, bool PICK>
__global__ void __launch_bounds__(kLhWarps * 32, 1) lmhead_pick_kernel(const LmHeadArgs A) {
    constexpr int NT = kLhWarps * 32;
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float2 part[2][kLhWarps][32];  // the K slices' sums of a round (ks > 1), double-buffered
    __shared__ uint64_t finb[kLhWarps];
    __shared__ int last;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const int g = lane >> 2, t = lane & 3;
    const LhPlan plan(A.M, A.K, S);
    uint8_t* ring = smem + size_t(warp) * S * kLhStage;
    uint64_t* bars = reinterpret_cast<uint64_t*>(smem + plan.rings) + warp * S;
    uint16_t* xs = reinterpret_cast<uint16_t*>(smem + plan.rings + plan.bars);
    const int pitch = A.K + 8;
    const uint16_t* zero16 = xs + size_t(A.M) * pitch;
    if (lane < S) mbar_init(&bars[lane], 1);
    fence_mbar_init();
    __syncwarp();
    pdl_launch_dependents();
    // this warp's tiles of 8 vocabulary rows: wg, wg + NW, ...; chunk q = (tile q / CPT, k chunk q % CPT)
    // K split: warp w takes slice w % ks of tile w / ks of the CTA's round (8 / ks tiles a round); ks = 1 when the
    // tiles outnumber the warps enough for an even load (lmhead_split)
    const int ks = A.ks, TPR = kLhWarps / ks, CPT = A.K / kLhChunk, CPU = CPT / ks;
    const int lt = warp / ks, sl = warp % ks;
    const int tiles = (A.V + kLhRows - 1) / kLhRows;
    const int G = int(gridDim.x), b = int(blockIdx.x), stride = G * TPR;
    const int first = b * TPR + lt;  // this warp's tile in round 0
    const int Rc = b * TPR < tiles ? (tiles - b * TPR + stride - 1) / stride : 0;  // the CTA's rounds
    const int Rw = first < tiles ? (tiles - first + stride - 1) / stride : 0;      // rounds with a tile for this warp
    const int Q = Rw * CPU;
    const uint64_t pol = l2_evict_first_policy();
    auto issue = [&](int q) {  // lane r < 8 copies row r of chunk q (1 KB) into stage q % S
        const int r = q / CPU, c = sl * CPU + (q - r * CPU);
        const int n0 = (first + r * stride) * kLhRows, rows = min(kLhRows, A.V - n0);
        uint64_t* bar = &bars[q % S];
        if (lane == 0) {
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");  // the stage's earlier reads first
            mbar_arrive_expect_tx(bar, uint32_t(rows) * (kLhChunk * 2));
        }
        __syncwarp();
        if (lane < rows)
            bulk_g2s_hint(ring + (q % S) * kLhStage + lane * kLhRowPitch,
                          A.w + int64_t(n0 + lane) * A.K + int64_t(c) * kLhChunk, kLhChunk * 2, bar, pol);
    };
    // the weights do not depend on the preceding kernel: start the rings before waiting for it
    for (int q = 0; q < S && q < Q; ++q) issue(q);
    pdl_wait();
    {
        // the x rows in batches of 16 pieces per thread, every load of a batch issued before its stores (one L2
        // round trip per batch, not one per piece)
        const int per_row = A.K >> 3, total = A.M * per_row;
        for (int base = threadIdx.x; base < total; base += 16 * NT) {
            uint4 v[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int i = base + j * NT;
                if (i < total) {
                    const int m = i / per_row, c = i - m * per_row;
                    v[j] = __ldg(reinterpret_cast<const uint4*>(A.x + m * A.x_stride) + c);
                }
            }
#pragma unroll
            for (int j = 0; j < 16; ++j) {
                const int i = base + j * NT;
                if (i < total) {
                    const int m = i / per_row, c = i - m * per_row;
                    *reinterpret_cast<uint4*>(xs + size_t(m) * pitch + 8 * c) = v[j];
                }
            }
        }
        if (threadIdx.x == 0) *reinterpret_cast<uint4*>(const_cast<uint16_t*>(zero16)) = make_uint4(0, 0, 0, 0);
    }
    __syncthreads();
    uint64_t top[2][kTkK], best[2] = {0, 0};  // rows g and g + 8
#pragma unroll
    for (int j = 0; j < kTkK; ++j) top[0][j] = top[1][j] = 0;
    // ldmatrix row addresses: W rows lane & 7 at k + 8 (lane >> 3); x rows likewise, and rows 8 + (lane & 7) when
    // M > 8 (past M: the zero row)
    const int lr = lane & 7, lk = 8 * (lane >> 3);
    const uint16_t* xrow = lr < A.M ? xs + size_t(lr) * pitch + lk : nullptr;
    const uint16_t* xrow2 = 8 + lr < A.M ? xs + size_t(8 + lr) * pitch + lk : nullptr;
    const bool hi = A.M > 8;
    int q = 0;
    bool bad = false;
    for (int r = 0; r < Rc; ++r) {
        float c0[4] = {0.f, 0.f, 0.f, 0.f}, c1[4] = {0.f, 0.f, 0.f, 0.f};
        if (r < Rw && !bad) {
            for (int cc = 0; cc < CPU; ++cc, ++q) {
                if (!mbar_wait(&bars[q % S], uint32_t(q / S) & 1u)) {
                    bad = true;
                    break;
                }
                const uint8_t* st = ring + (q % S) * kLhStage + lr * kLhRowPitch + lk * 2;
                const int kx = (sl * CPU + cc) * kLhChunk;
#pragma unroll 4
                for (int kk = 0; kk < kLhChunk; kk += 32) {
                    uint32_t bw[4], a[4], a8[4] = {0u, 0u, 0u, 0u};
                    lh_ldsm_x4(bw, st + kk * 2);
                    lh_ldsm_x4(a, xrow ? xrow + kx + kk : zero16);
                    if (hi) lh_ldsm_x4(a8, xrow2 ? xrow2 + kx + kk : zero16);
                    lh_mma(c0, a[0], a8[0], a[1], a8[1], bw[0], bw[1]);
                    lh_mma(c1, a[2], a8[2], a[3], a8[3], bw[2], bw[3]);
                }
                __syncwarp();
                if (q + S < Q) issue(q + S);
            }
        }
        // the slice's sums (the two k-step chains added in order), then the ks slices of the tile in slice order
        // (ks > 1 only for M <= 8: rows g + 8 are empty there)
        float v0 = c0[0] + c1[0], v1 = c0[1] + c1[1], v2 = c0[2] + c1[2], v3 = c0[3] + c1[3];
        if (ks > 1) {
            part[r & 1][warp][lane] = make_float2(v0, v1);
            __syncthreads();  // (the other buffer is read before the next round's barrier: no second one needed)
            if (sl == 0)
                for (int j = 1; j < ks; ++j) {
                    const float2 o = part[r & 1][warp + j][lane];
                    v0 += o.x;
                    v1 += o.y;
                }
        }
        if (sl == 0 && r < Rw && g < A.M) {
            // the tile's outputs: rows g and g + 8 (< M) at columns n0 + 2t, n0 + 2t + 1
            const int n0 = (first + r * stride) * kLhRows;
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int row = g + 8 * h;
                if (h == 1 && row >= A.M) break;
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int n = n0 + 2 * t + e;
                    if (n < A.V) {
                        const float v = h ? (e ? v3 : v2) : (e ? v1 : v0);
                        const uint16_t bits = __bfloat16_as_ushort(__float2bfloat16_rn(v));
                        if (!PICK || A.logits) A.logits[int64_t(row) * A.out_stride + n] = bits;
                        if constexpr (PICK) {
                            const uint32_t gi = uint32_t(A.index_base + n);  // ranked by the global index
                            if (A.k > 0) insert_rank(top[h], rank_topk(bits, gi), A.k);
                            best[h] = max(best[h], rank_argmax(bits, gi));
                        }
                    }
                }
            }
        }
    }
    if (bad) {
        // a wait gave up (the error word is set): wait, bounded, for this warp's copies still in flight
        for (int r2 = q + 1; r2 < Q && r2 < q + S; ++r2) mbar_wait(&bars[r2 % S], uint32_t(r2 / S) & 1u);
    }
    if constexpr (!PICK) return;
    __syncthreads();  // every ring is idle: its memory now holds the pick's lists
    uint64_t* lst = reinterpret_cast<uint64_t*>(smem);      // [warp * 4 + t][kLhMaxM][kTkK + 1]
    uint64_t* fin = lst + kLhWarps * 4 * kLhMaxM * (kTkK + 1);  // [NT][kTkK]
#pragma unroll
    for (int h = 0; h < 2; ++h)
        if (g + 8 * h < A.M) {
            uint64_t* l = lst + ((warp * 4 + t) * kLhMaxM + g + 8 * h) * (kTkK + 1);
#pragma unroll
            for (int j = 0; j < kTkK; ++j) l[j] = top[h][j];
            l[kTkK] = best[h];
        }
    __syncthreads();
    unsigned* counter = reinterpret_cast<unsigned*>(A.ws);  // fixed offset: calls of any grid share a workspace
    uint64_t* ws = A.ws + 32;
    if (threadIdx.x < A.M) {
        const int m = threadIdx.x;
        uint64_t t2[kTkK], b2 = 0;
#pragma unroll
        for (int j = 0; j < kTkK; ++j) t2[j] = 0;
        for (int r = 0; r < kLhWarps * 4; ++r) {
            const uint64_t* l = lst + (r * kLhMaxM + m) * (kTkK + 1);
            for (int j = 0; j < A.k; ++j) insert_rank(t2, l[j], A.k);
            b2 = max(b2, l[kTkK]);
        }
        uint64_t* out = ws + (size_t(blockIdx.x) * kLhMaxM + m) * (kTkK + 1);
#pragma unroll
        for (int j = 0; j < kTkK; ++j) __stcg(out + j, t2[j]);
        __stcg(out + kTkK, b2);
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence();
        last = atomicAdd(counter, 1u) == unsigned(G - 1);
        if (last) __threadfence();
    }
    __syncthreads();
    if (!last) return;
    // the last CTA, per row: thread t merges the lists of CTAs t, t + 256, ..., then a pairwise merge tree in
    // shared memory (merge_lists) and one thread writes the indices
    for (int m = 0; m < A.M; ++m) {
        uint64_t t2[kTkK], b2 = 0;
#pragma unroll
        for (int j = 0; j < kTkK; ++j) t2[j] = 0;
        for (int cta = threadIdx.x; cta < G; cta += NT) {
            const uint64_t* src = ws + (size_t(cta) * kLhMaxM + m) * (kTkK + 1);
            for (int j = 0; j < A.k; ++j) insert_rank(t2, __ldcg(src + j), A.k);
            b2 = max(b2, __ldcg(src + kTkK));
        }
#pragma unroll
        for (int j = 0; j < kTkK; ++j) fin[threadIdx.x * kTkK + j] = t2[j];
#pragma unroll
        for (int o = 16; o; o >>= 1) b2 = max(b2, __shfl_xor_sync(0xffffffffu, b2, o));
        if (lane == 0) finb[warp] = b2;
        __syncthreads();
        for (int n = NT / 2; n >= 1; n >>= 1) {
            if (int(threadIdx.x) < n) merge_lists(fin, threadIdx.x * kTkK, (threadIdx.x + n) * kTkK, A.k);
            __syncthreads();
        }
        if (threadIdx.x == 0) {
            uint64_t bb = 0;
            for (int w = 0; w < kLhWarps; ++w) bb = max(bb, finb[w]);
            const int64_t am = int64_t(0xFFFFFFFFu - uint32_t(bb));
            if (A.argmax) A.argmax[m] = am;
            if (A.topk)
                for (int j = 0; j < A.k; ++j) A.topk[m * A.k + j] = int64_t(topk_index(fin[j]));
            if (A.children != nullptr)
                for (int j = 0; j < 8; ++j) {
                    const int c = A.children[j];
                    if (c < 0) break;
                    A.dst[m * A.dst_stride + c] = (j == 0 || j >= A.k) ? am : int64_t(topk_index(fin[j]));
                }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) atomicExch(counter, 0u);  // reusable by the next launch
}

int lmhead_grid() { return sm_count(); }

// the deepest ring (stages per warp) whose plan fits the shared memory, or 0
int lmhead_stages(int M, int K) {
    for (int S = 4; S >= 1; --S)
        if (LhPlan(M, K, S).total <= kLhSmemLimit) return S;
    return 0;
}

template <int S, bool PICK>
static int launch_lh(const LmHeadArgs& A, cudaStream_t stream) {
    auto kern = lmhead_pick_kernel<S, PICK>;
    const size_t smem = LhPlan(A.M, A.K, S).total;
    static std::mutex mu;
    static size_t opt_in = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (smem > opt_in) {
            CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
            opt_in = smem;
        }
    }
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(lmhead_grid());
    cfg.blockDim = dim3(kLhWarps * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, A));
    return MONO_OK;
}

// K slices per tile: the fewest (1, 2, 4, 8 dividing the K chunks) whose rounds keep the warps busy within 2 % of
// the best split; the matrices of the draft head have fewer 8-row tiles than the grid has warps, the lm_head many
int lmhead_split(int V, int K) {
    const int64_t tiles = (int64_t(V) + kLhRows - 1) / kLhRows, cpt = K / kLhChunk, G = sm_count();
    int best = 1;
    double best_eff = 0.0;
    for (int ks = 1; ks <= kLhWarps; ks *= 2) {
        if (cpt % ks) break;
        const int64_t per_round = G * (kLhWarps / ks), rounds = (tiles + per_round - 1) / per_round;
        const double eff = double(tiles) / double(rounds * per_round);
        if (eff > best_eff + 0.02) {
            best_eff = eff;
            best = ks;
        }
    }
    return best;
}

template <bool PICK>
static int launch_lmhead_t(LmHeadArgs A, cudaStream_t stream) {
    // the pick over a vocabulary has tiles enough for every warp: no split (a split's per-round barrier measured
    // slower there: 235 against 197 us)
    A.ks = (PICK || A.M > 8) ? 1 : lmhead_split(A.V, A.K);
    switch (lmhead_stages(A.M, A.K)) {
        case 4: return launch_lh<4, PICK>(A, stream);
        case 3: return launch_lh<3, PICK>(A, stream);
        case 2: return launch_lh<2, PICK>(A, stream);
        case 1: return launch_lh<1, PICK>(A, stream);
        default: return fail(MONO_EINVAL, "lm_head: x rows of K = %d do not fit next to the rings", A.K);
    }
}

int launch_lmhead(const LmHeadArgs& A, cudaStream_t stream) { return launch_lmhead_t<true>(A, stream); }

bool bf16_rows_fit(int M, int K) { return K >= kLhChunk && K % kLhChunk == 0 && M <= kLhMaxM && lmhead_stages(M, K) > 0; }

int launch_bf16_rows(const uint16_t* x, int64_t x_stride, const uint16_t* w, int M, int N, int K, uint16_t* out,
                     int64_t out_stride, cudaStream_t stream) {
    LmHeadArgs A{};
    A.x = x;
    A.w = w;
    A.logits = out;
    A.x_stride = x_stride;
    A.out_stride = out_stride;
    A.K = K;
    A.V = N;
    A.M = M;
    return launch_lmhead_t<false>(A, stream);
}

}  // namespace mono

using namespace mono;

extern "C" size_t mono_lmhead_workspace(void) { return lmhead_workspace_bytes(lmhead_grid()); }

extern "C" int mono_lmhead_pick(const void* x, int64_t x_stride, const void* w, int64_t M, int64_t V, int64_t K, int64_t k,
                                int64_t index_base, void* logits, int64_t* argmax, int64_t* topk,
                                const int32_t* children, int64_t* dst, int64_t dst_stride, void* workspace,
                                size_t workspace_bytes, mono_stream_t stream) {
    MONO_CHECK(x && w && workspace, "null operand");
    MONO_CHECK(M >= 1 && M <= kLhMaxM, "1 <= M <= %d rows", kLhMaxM);
    MONO_CHECK(k >= 0 && k <= kTkK, "0 <= k <= %d", kTkK);
    MONO_CHECK(K >= kLhChunk && K % kLhChunk == 0 && lmhead_stages(int(M), int(std::min<int64_t>(K, 1 << 20))) > 0,
               "K a multiple of 512 whose M x rows fit in shared memory beside the rings (K <= 4096 at M = 16)");
    MONO_CHECK(V >= 1 && V < (int64_t(1) << 31) && V * K < (int64_t(1) << 40), "1 <= V < 2^31");
    MONO_CHECK(index_base >= 0 && index_base + V < (int64_t(1) << 31), "0 <= index_base, index_base + V < 2^31");
    MONO_CHECK(x_stride >= K && x_stride % 8 == 0 && aligned(x, 16) && aligned(w, 16),
               "x rows and w 16-byte aligned, x_stride a multiple of 8 elements");
    MONO_CHECK(argmax || (topk && k > 0) || logits || children, "no output requested");
    MONO_CHECK(k == 0 || topk || children, "top-k wanted but no top-k output");
    MONO_CHECK(!children || (dst && (M == 1 || dst_stride >= 8)), "the pick form: a destination, rows 8 slots apart");
    MONO_CHECK(aligned(workspace, 256) && workspace_bytes >= lmhead_workspace_bytes(lmhead_grid()),
               "workspace: mono_lmhead_workspace() bytes, 256-byte aligned, zero-filled before its first use");
    LmHeadArgs A{};
    A.x = static_cast<const uint16_t*>(x);
    A.w = static_cast<const uint16_t*>(w);
    A.logits = static_cast<uint16_t*>(logits);
    A.argmax = argmax;
    A.topk = topk;
    A.children = children;
    A.dst = dst;
    A.dst_stride = dst_stride;
    A.ws = static_cast<uint64_t*>(workspace);
    A.x_stride = x_stride;
    A.out_stride = V;
    A.index_base = index_base;
    A.K = int(K);
    A.V = int(V);
    A.M = int(M);
    A.k = int(k);
    return launch_lmhead(A, reinterpret_cast<cudaStream_t>(stream));
}
