// bf16 lm_head with the greedy / draft pick fused (the role of the reference's verify logits + argmax, and of its
// draft pick, csrc/draft_lmhead.sycl:87-292): for M <= 8 rows of x [M][K] against W [V][K] (bf16, far larger than
// L2), logits = bf16(x W^T) in the bf16 GEMV's pinned order (gemv_bf16.cu: lane l accumulates its 16-byte pieces
// l, l + 32, ... with fmaf, element by element, then the xor butterfly 16, 8, 4, 2, 1; bf16 x bf16 products are
// exact in fp32, so the oracle reproduces every bit), and per row the argmax (argmax rank: smallest index on ties)
// and the top-k (k <= 8, top-k rank), without writing the logits (optional).
//
// Work: a persistent grid; warp w of CTA b takes column groups of NC columns g = b * 8 + w, + G * 8, ... (NC > 1
// at several rows: one load of each x piece serves NC columns; the per-column arithmetic is unchanged; two rows
// share each paired fma, __ffma2_rn, whose halves round exactly as fmaf). Lane m < M
// keeps row m's running top-k list and argmax in registers. At the end the CTA merges its warps' lists in shared
// memory and writes them to the workspace; the last CTA to finish (an arrival counter) merges the CTAs' lists -
// ranks are distinct, so the merge order does not matter - and writes the indices. The pick form then scatters the
// draft's tokens into the verify-token row: dst[children[0]] = argmax, dst[children[j]] = top-k[j] (j >= 1), the
// reference's draft pick (csrc/draft_lmhead.sycl:4-17).
#include "launch.h"
#include "ranks.cuh"

namespace mono {

constexpr int kLhWarps = 8, kLhMaxM = 8, kLhCtasPerSm = 2;

__device__ __forceinline__ uint4 lh_ld_stream(const uint4* p, uint64_t pol) {
    uint4 v;
    asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "l"(p), "l"(pol));
    return v;
}
__device__ __forceinline__ float lh_lo(uint32_t u) { return __uint_as_float(u << 16); }
__device__ __forceinline__ float lh_hi(uint32_t u) { return __uint_as_float(u & 0xFFFF0000u); }

struct LmHeadArgs {
    const uint16_t* x;        // [M][x_stride] bf16
    const uint16_t* w;        // [V][K] bf16
    uint16_t* logits;         // [M][V] bf16 or null
    int64_t* argmax;          // [M] or null
    int64_t* topk;            // [M][k] or null (k = 0: none)
    const int32_t* children;  // pick form: up to 8 slots of dst, -1 ends (row 0's tokens), or null
    int64_t* dst;             // pick form: the verify-token row
    uint64_t* ws;             // the arrival counter (first 256 bytes), then [G][kLhMaxM][kTkK + 1] CTA lists
    int64_t x_stride;
    int K, V, M, k;
};

size_t lmhead_workspace_bytes(int grid) { return size_t(grid) * kLhMaxM * (kTkK + 1) * 8 + 256; }

template <int M, int NC, int CPS>
__global__ void __launch_bounds__(kLhWarps * 32, CPS) lmhead_pick_kernel(const LmHeadArgs A) {
    constexpr int NT = kLhWarps * 32;
    __shared__ uint64_t lst[kLhWarps][M][kTkK + 1];
    __shared__ uint64_t fin[NT * kTkK];
    __shared__ uint64_t finb[kLhWarps];
    __shared__ int last;
    pdl_launch_dependents();
    pdl_wait();
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    const uint64_t pol = l2_evict_first_policy();
    const int per_lane = A.K / 256;  // 8-element pieces per lane
    const int groups = (A.V + NC - 1) / NC, G = int(gridDim.x);
    uint64_t top[kTkK], best = 0;
#pragma unroll
    for (int j = 0; j < kTkK; ++j) top[j] = 0;
    constexpr int MP = (M + 1) / 2;  // row pairs (an odd M pads its last pair with a zero row)
    for (int grp = int(blockIdx.x) * kLhWarps + warp; grp < groups; grp += G * kLhWarps) {
        const int n0 = grp * NC;
        float acc[NC][M];
        if constexpr (M == 1) {
#pragma unroll
            for (int c = 0; c < NC; ++c) acc[c][0] = 0.f;
            for (int j = 0; j < per_lane; ++j) {
                const int64_t piece = int64_t(j) * 32 + lane;
                uint4 wv[NC];
#pragma unroll
                for (int c = 0; c < NC; ++c)
                    wv[c] = n0 + c < A.V ? lh_ld_stream(reinterpret_cast<const uint4*>(A.w + int64_t(n0 + c) * A.K) + piece, pol)
                                         : make_uint4(0, 0, 0, 0);
                const uint4 xv = __ldg(reinterpret_cast<const uint4*>(A.x) + piece);
                const float xf[8] = {lh_lo(xv.x), lh_hi(xv.x), lh_lo(xv.y), lh_hi(xv.y),
                                     lh_lo(xv.z), lh_hi(xv.z), lh_lo(xv.w), lh_hi(xv.w)};
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    float a = acc[c][0];
                    a = fmaf(lh_lo(wv[c].x), xf[0], a);
                    a = fmaf(lh_hi(wv[c].x), xf[1], a);
                    a = fmaf(lh_lo(wv[c].y), xf[2], a);
                    a = fmaf(lh_hi(wv[c].y), xf[3], a);
                    a = fmaf(lh_lo(wv[c].z), xf[4], a);
                    a = fmaf(lh_hi(wv[c].z), xf[5], a);
                    a = fmaf(lh_lo(wv[c].w), xf[6], a);
                    a = fmaf(lh_hi(wv[c].w), xf[7], a);
                    acc[c][0] = a;
                }
            }
        } else {
            // two rows per paired fma (__ffma2_rn: each half rounds as fmaf, so the bits are the scalar order's)
            float2 acc2[NC][MP];
#pragma unroll
            for (int c = 0; c < NC; ++c)
#pragma unroll
                for (int p = 0; p < MP; ++p) acc2[c][p] = make_float2(0.f, 0.f);
            // the weight pieces of step j + 1 are requested before step j's arithmetic (one step of look-ahead)
            uint4 wn[NC];
#pragma unroll
            for (int c = 0; c < NC; ++c)
                wn[c] = n0 + c < A.V ? lh_ld_stream(reinterpret_cast<const uint4*>(A.w + int64_t(n0 + c) * A.K) + lane, pol)
                                     : make_uint4(0, 0, 0, 0);
            for (int j = 0; j < per_lane; ++j) {
                const int64_t piece = int64_t(j) * 32 + lane;
                uint4 wv[NC];
#pragma unroll
                for (int c = 0; c < NC; ++c) {
                    wv[c] = wn[c];
                    if (j + 1 < per_lane && n0 + c < A.V)
                        wn[c] = lh_ld_stream(reinterpret_cast<const uint4*>(A.w + int64_t(n0 + c) * A.K) + piece + 32, pol);
                }
                uint4 xv[2 * MP];
#pragma unroll
                for (int m = 0; m < 2 * MP; ++m)
                    xv[m] = m < M ? __ldg(reinterpret_cast<const uint4*>(A.x + m * A.x_stride) + piece) : make_uint4(0, 0, 0, 0);
#pragma unroll
                for (int e = 0; e < 8; ++e) {
                    float2 xp[MP];
#pragma unroll
                    for (int p = 0; p < MP; ++p) {
                        const uint32_t ua = (&xv[2 * p].x)[e >> 1], ub = (&xv[2 * p + 1].x)[e >> 1];
                        xp[p] = make_float2((e & 1) ? lh_hi(ua) : lh_lo(ua), (e & 1) ? lh_hi(ub) : lh_lo(ub));
                    }
#pragma unroll
                    for (int c = 0; c < NC; ++c) {
                        const uint32_t uw = (&wv[c].x)[e >> 1];
                        const float wf = (e & 1) ? lh_hi(uw) : lh_lo(uw);
                        const float2 w2 = make_float2(wf, wf);
#pragma unroll
                        for (int p = 0; p < MP; ++p) acc2[c][p] = __ffma2_rn(w2, xp[p], acc2[c][p]);
                    }
                }
            }
#pragma unroll
            for (int c = 0; c < NC; ++c)
#pragma unroll
                for (int m = 0; m < M; ++m) acc[c][m] = (m & 1) ? acc2[c][m >> 1].y : acc2[c][m >> 1].x;
        }
#pragma unroll
        for (int c = 0; c < NC; ++c) {
            const int n = n0 + c;
#pragma unroll
            for (int m = 0; m < M; ++m) {
                float a = acc[c][m];
#pragma unroll
                for (int d = 16; d > 0; d >>= 1) a += __shfl_xor_sync(0xffffffffu, a, d);
                acc[c][m] = a;  // every lane holds the same sum
            }
            if (n < A.V) {
                // lane m takes row m: rank the logit into its running lists
#pragma unroll
                for (int m = 0; m < M; ++m)
                    if (lane == m) {
                        const uint16_t b = __bfloat16_as_ushort(__float2bfloat16_rn(acc[c][m]));
                        if (A.logits) A.logits[int64_t(m) * A.V + n] = b;
                        if (A.k > 0) insert_rank(top, rank_topk(b, uint32_t(n)), A.k);
                        best = max(best, rank_argmax(b, uint32_t(n)));
                    }
            }
        }
    }
    // the CTA's lists: per row, the warps' lists merged by warp 0's lane m
    if (lane < M) {
#pragma unroll
        for (int j = 0; j < kTkK; ++j) lst[warp][lane][j] = top[j];
        lst[warp][lane][kTkK] = best;
    }
    __syncthreads();
    // the counter sits at a fixed offset, so calls of any grid size share a workspace safely
    unsigned* counter = reinterpret_cast<unsigned*>(A.ws);
    uint64_t* ws = A.ws + 32;
    if (warp == 0 && lane < M) {
        for (int w = 1; w < kLhWarps; ++w) {
            for (int j = 0; j < A.k; ++j) insert_rank(top, lst[w][lane][j], A.k);
            best = max(best, lst[w][lane][kTkK]);
        }
        uint64_t* mine = ws + (size_t(blockIdx.x) * kLhMaxM + lane) * (kTkK + 1);
#pragma unroll
        for (int j = 0; j < kTkK; ++j) __stcg(mine + j, top[j]);
        __stcg(mine + kTkK, best);
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
    for (int m = 0; m < M; ++m) {
        uint64_t t2[kTkK], b2 = 0;
#pragma unroll
        for (int j = 0; j < kTkK; ++j) t2[j] = 0;
        for (int c = threadIdx.x; c < G; c += NT) {
            const uint64_t* src = ws + (size_t(c) * kLhMaxM + m) * (kTkK + 1);
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
            if (m == 0 && A.children != nullptr)
                for (int j = 0; j < 8; ++j) {
                    const int c = A.children[j];
                    if (c < 0) break;
                    A.dst[c] = (j == 0 || j >= A.k) ? am : int64_t(topk_index(fin[j]));
                }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) atomicExch(counter, 0u);  // reusable by the next launch
}

int lmhead_grid() { return sm_count() * kLhCtasPerSm; }

template <int M, int NC>
static int launch_lh(const LmHeadArgs& A, cudaStream_t stream) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(lmhead_grid());
    cfg.blockDim = dim3(kLhWarps * 32);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, lmhead_pick_kernel<M, NC, kLhCtasPerSm>, A));
    return MONO_OK;
}

// (measured at 8 rows: 4 columns per warp at 2 CTAs per SM, 460 us; 2 columns at 3 CTAs per SM, 599 us; 8 columns
// at 1 CTA per SM, 575 us)
int launch_lmhead(const LmHeadArgs& A, cudaStream_t stream) {
    switch (A.M) {
        case 1: return launch_lh<1, 1>(A, stream);
        case 2: return launch_lh<2, 2>(A, stream);
        case 3: return launch_lh<3, 2>(A, stream);
        case 4: return launch_lh<4, 4>(A, stream);
        case 5: return launch_lh<5, 4>(A, stream);
        case 6: return launch_lh<6, 4>(A, stream);
        case 7: return launch_lh<7, 4>(A, stream);
        default: return launch_lh<8, 4>(A, stream);
    }
}

}  // namespace mono

using namespace mono;

extern "C" size_t mono_lmhead_workspace(void) { return lmhead_workspace_bytes(lmhead_grid()); }

extern "C" int mono_lmhead_pick(const void* x, int64_t x_stride, const void* w, int64_t M, int64_t V, int64_t K, int64_t k,
                                void* logits, int64_t* argmax, int64_t* topk, const int32_t* children, int64_t* dst,
                                void* workspace, size_t workspace_bytes, mono_stream_t stream) {
    MONO_CHECK(x && w && workspace, "null operand");
    MONO_CHECK(M >= 1 && M <= kLhMaxM, "1 <= M <= %d rows", kLhMaxM);
    MONO_CHECK(k >= 0 && k <= kTkK, "0 <= k <= %d", kTkK);
    MONO_CHECK(K >= 256 && K % 256 == 0 && K <= (1 << 20), "K a multiple of 256 up to 2^20");
    MONO_CHECK(V >= 1 && V < (int64_t(1) << 31) && V * K < (int64_t(1) << 40), "1 <= V < 2^31");
    MONO_CHECK(x_stride >= K && x_stride % 8 == 0 && aligned(x, 16) && aligned(w, 16),
               "x rows and w 16-byte aligned, x_stride a multiple of 8 elements");
    MONO_CHECK(argmax || (topk && k > 0) || logits || children, "no output requested");
    MONO_CHECK(k == 0 || topk || children, "top-k wanted but no top-k output");
    MONO_CHECK(!children || (dst && M == 1), "the pick form takes one row and a destination");
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
    A.ws = static_cast<uint64_t*>(workspace);
    A.x_stride = x_stride;
    A.K = int(K);
    A.V = int(V);
    A.M = int(M);
    A.k = int(k);
    return launch_lmhead(A, reinterpret_cast<cudaStream_t>(stream));
}
