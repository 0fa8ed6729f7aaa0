// Fused decode MLP block in one cooperative launch (the role of csrc/mono_mlp.sycl:34-180 and of the MLP
// phases 3-6 of layer_post, csrc/mono_layer.sycl:272-313), GPTQ W4A8:
//
//   P1 rows  xn = RMSNorm(x) (or x when no norm weight); q1, s1 = quant(xn)
//   P2 all   g, u = W4A8 gate / up (q1);  h = bf16(silu_lut[bf16 g] * bf16 u);  row amax of h
//   P3 all   q2, s2 = quant(h)
//   P4 all   out = bf16(x + bf16(W4A8 down (q2)))  (or bf16(W4A8 down (q2)) without the residual)
//
// Phases are separated by bounded grid barriers; the weight rings run across them (engine.cuh), so
// gate/up and down weights stream while rows are normalized and quantized.
#include <mutex>

#include "launch.h"
#include "grid.cuh"
#include "rowops.cuh"

namespace mono {

// Items each warp keeps requested into L2 beyond its ring: the weight stream runs on through the row
// phases and grid barriers (the role of the reference's prefetch_stream, csrc/mono_common.hpp:318-340).
constexpr int kMlpPrefetch = 6;

template <int MT, int GROUPS, int ST>
__global__ void __launch_bounds__(GROUPS * 128) mlp_kernel(const Program P, const MlpArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[GROUPS][16];
    __shared__ int flag;
    const int wg = threadIdx.x >> 7, tig = threadIdx.x & 127, warp = tig >> 5, lane = threadIdx.x & 31;
    const int M = P.M;
    int xbytes = 0;
    for (int i = 0; i < P.nph; ++i)
        if (P.ph[i].xsmem && M * (P.ph[i].K + 16) > xbytes) xbytes = M * (P.ph[i].K + 16);
    const SmemPlan<FMT_GPTQ, MT> plan(GROUPS, ST, A.max_items, xbytes);
    constexpr int SBY = stage_bytes<FMT_GPTQ>();
    const int wid = wg * kGroupWarps + warp;
    uint64_t* bar_base = reinterpret_cast<uint64_t*>(smem + plan.rings);
    uint64_t* xbar = bar_base + GROUPS * kGroupWarps * ST;
    uint32_t* part = reinterpret_cast<uint32_t*>(smem + plan.rings + plan.bars) + wg * 2 * A.max_items * MT * 128;
    int8_t* xsm = reinterpret_cast<int8_t*>(smem + plan.rings + plan.bars + plan.part);

    Ring<FMT_GPTQ, LAYOUT_TILED, ST> ring;
    ring.buf = smem + size_t(wid) * ST * SBY;
    ring.bars = bar_base + wid * ST;
    Seq sq;
    sq.init(P, warp, wg * int(gridDim.x) + int(blockIdx.x), int(gridDim.x) * GROUPS);
    if (threadIdx.x == 0) {
        mbar_init(xbar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    trace_stamp(0);
    pdl_launch_dependents();  // the next kernel may launch and stream its weights as our CTAs exit
    // Warp-groups without a P1 row start their weight streams before the dependency wait; those with a
    // row load it first (vector loads), so its requests are not queued behind weight copies in this SM's
    // TMA unit, and start their streams right after.
    const bool has_row = sq.vc < M;
    if (!has_row) ring.init(P, sq, lane, kMlpPrefetch);
    pdl_wait();
    trace_stamp(1);
    unsigned epoch = 0;
    bool ok = true;

    // ---- P1: norm + quant of the rows (one warp-group per row) ----
    if (blockIdx.x == 0 && threadIdx.x < 16) A.amax2[threadIdx.x] = 0u;
    for (int m = sq.vc; m < M; m += sq.nvc)
        norm_quant_row(A.x + size_t(m) * A.H, A.norm_w, A.eps, A.H, nullptr, A.q1 + size_t(m) * A.H, A.s1 + m, red[wg],
                       tig, wg);
    if (has_row) ring.init(P, sq, lane, kMlpPrefetch);
    trace_stamp(2);
    ok = grid_barrier(A.bar, epoch, &flag);
    trace_stamp(3);

    int xpar = 0;
    auto phase_x = [&](int ph) {
        const PhaseDesc& p = P.ph[ph];
        if (!p.xsmem) return XSrc{p.x, p.K, false, true};
        ok = stage_x(p, M, xsm, xbar, xpar) && ok;
        return XSrc{xsm, p.K + 16, true, true};
    };

    // ---- P2: gate / up, h = silu(g) * u ----
    {
        const XSrc xs = phase_x(0);
        trace_stamp(4);
        const PhaseDesc& ph = P.ph[0];
        const int C = phase_chunks(ph), items = phase_items(ph);
        float rmax0 = 0.f, rmax1 = 0.f;  // running |h| max of rows tig >> 4 and (tig >> 4) + 8
        const int ntiles = sq.my_tiles(0);
        for (int ti = 0; ti < ntiles && ok; ++ti) {
            const int T = sq.vc + ti * sq.nvc;
            uint32_t* pt = part + (ti & 1) * A.max_items * MT * 128;
            for (int item = warp; item < items; item += kGroupWarps) {
                uint32_t R[MT][4];
                consume_item<FMT_GPTQ, LAYOUT_TILED, MT, ST>(ring, P, sq, xs, M, item % C, lane, R);
                store_partial<MT>(pt, item, lane, R);
            }
            group_sync(wg);
            for (int e = tig; e < M * 16; e += 128) {
                const int m = e >> 4, n = T * 16 + (e & 15);
                const float s = __ldcg(A.s1 + m);
                const float tg = __uint_as_float(tile_total<FMT_GPTQ, MT>(pt, C, 0, m, e & 15));
                const float tu = __uint_as_float(tile_total<FMT_GPTQ, MT>(pt, C, 1, m, e & 15));
                const uint16_t gb = f32_to_bf16_bits(__fmul_rn(tg, s));
                const float u = bf16_round(__fmul_rn(tu, s));
                const uint16_t hb = f32_to_bf16_bits(__fmul_rn(bf16_bits_to_f32(A.lut[gb]), u));
                A.h[size_t(m) * A.I + n] = hb;
                const float a = fabsf(bf16_bits_to_f32(hb));
                if (e < 128) rmax0 = fmaxf(rmax0, a); else rmax1 = fmaxf(rmax1, a);
            }
        }
        // row maxima: the 16 threads of a row are one half-warp
#pragma unroll
        for (int o = 8; o; o >>= 1) {
            rmax0 = fmaxf(rmax0, __shfl_xor_sync(0xffffffffu, rmax0, o));
            rmax1 = fmaxf(rmax1, __shfl_xor_sync(0xffffffffu, rmax1, o));
        }
        if ((tig & 15) == 0) {
            const int m = tig >> 4;
            if (m < M) atomicMax(A.amax2 + m, __float_as_uint(rmax0));
            if (m + 8 < M) atomicMax(A.amax2 + m + 8, __float_as_uint(rmax1));
        }
    }
    trace_stamp(5);
    ok = grid_barrier(A.bar, epoch, &flag) && ok;
    trace_stamp(6);

    // ---- P3: q2 = quant(h) ----
    {
        // 8-element pieces: one 16-byte load of h, one 8-byte store of permuted q2
        const int ppr = A.I >> 3, pieces = M * ppr;
        const int stride = int(gridDim.x * blockDim.x);
        for (int i = int(blockIdx.x * blockDim.x + threadIdx.x); i < pieces; i += stride) {
            const int m = i / ppr;
            const float s = __fdiv_rn(__uint_as_float(__ldcg(A.amax2 + m)), 127.f);
            const uint4 hv = __ldcg(reinterpret_cast<const uint4*>(A.h) + i);
            const uint32_t u[4] = {hv.x, hv.y, hv.z, hv.w};
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = __uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16));
            reinterpret_cast<uint2*>(A.q2)[i] = quant8_perm(v, s);
        }
        if (blockIdx.x == 0 && threadIdx.x < M) A.s2[threadIdx.x] = __fdiv_rn(__uint_as_float(__ldcg(A.amax2 + threadIdx.x)), 127.f);
    }
    trace_stamp(7);
    ok = grid_barrier(A.bar, epoch, &flag) && ok;
    trace_stamp(8);

    // ---- P4: down (+ residual) ----
    {
        const XSrc xs = phase_x(1);
        trace_stamp(9);
        const PhaseDesc& ph = P.ph[1];
        const int C = phase_chunks(ph), items = phase_items(ph);
        const int ntiles = sq.my_tiles(1);
        for (int ti = 0; ti < ntiles && ok; ++ti) {
            const int T = sq.vc + ti * sq.nvc;
            uint32_t* pt = part + (ti & 1) * A.max_items * MT * 128;
            for (int item = warp; item < items; item += kGroupWarps) {
                uint32_t R[MT][4];
                consume_item<FMT_GPTQ, LAYOUT_TILED, MT, ST>(ring, P, sq, xs, M, item % C, lane, R);
                store_partial<MT>(pt, item, lane, R);
            }
            group_sync(wg);
            for (int e = tig; e < M * 16; e += 128) {
                const int m = e >> 4, n = T * 16 + (e & 15);
                const float s = __fdiv_rn(__uint_as_float(__ldcg(A.amax2 + m)), 127.f);
                const float tot = __uint_as_float(tile_total<FMT_GPTQ, MT>(pt, C, 0, m, e & 15));
                uint16_t r = f32_to_bf16_bits(__fmul_rn(tot, s));
                const size_t o = size_t(m) * A.H + n;
                if (A.residual) r = f32_to_bf16_bits(__fadd_rn(bf16_bits_to_f32(A.x[o]), bf16_bits_to_f32(r)));
                A.out[o] = r;
            }
        }
    }
    trace_stamp(10);
    ring.drain(lane);
    grid_exit(A.bar);
}

size_t mlp_workspace_bytes(int H, int I) {
    // xn, q1, h, q2 (16 rows each), s1, s2, amax2, barrier words; every piece 256-byte aligned
    auto al = [](size_t b) { return (b + 255) / 256 * 256; };
    return al(16 * size_t(H) * 2) + al(16 * size_t(H)) + al(16 * size_t(I) * 2) + al(16 * size_t(I)) + 4 * 256;
}

template <int MT, int GROUPS, int ST>
static int launch_mlp_t(const Program& P, const MlpArgs& A, size_t smem, cudaStream_t stream) {
    auto kern = mlp_kernel<MT, GROUPS, ST>;
    static std::mutex mu;
    static size_t opt_in = 0;
    static int per_sm = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (smem > opt_in) {
            CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
            opt_in = smem;
            CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, GROUPS * 128, smem));
        }
    }
    if (per_sm < 1) return fail(MONO_EINVAL, "mlp: one CTA does not fit an SM (%zu B shared)", smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sm_count());
    cfg.blockDim = dim3(GROUPS * 128);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, P, A));
    return MONO_OK;
}

constexpr size_t kMlpSmemLimit = 227 * 1024 - 1024;  // leave room for the static shared memory

int launch_mlp(Program& P, MlpArgs& A, cudaStream_t stream) {
    const int M = P.M;
    A.max_items = 0;
    for (int i = 0; i < P.nph; ++i) A.max_items = phase_items(P.ph[i]) > A.max_items ? phase_items(P.ph[i]) : A.max_items;
    // stage each phase's activations when they fit next to the rings (largest phase first)
    for (int i = 0; i < P.nph; ++i) P.ph[i].xsmem = 1;
    const bool two = M > 8;
    // plans in order: 16 warps x 1 stage, 8 warps x 2 stages, 4 warps x 2 stages, with every activation
    // block staged; then the same with the largest block read through L1
    for (int attempt = 0; attempt < 3; ++attempt) {
        int xb = 0;
        for (int i = 0; i < P.nph; ++i)
            if (P.ph[i].xsmem) xb = M * (P.ph[i].K + 16) > xb ? M * (P.ph[i].K + 16) : xb;
#define MONO_MLP_TRY(MTV)                                                                              \
    {                                                                                                  \
        const SmemPlan<FMT_GPTQ, MTV> a(4, 1, A.max_items, xb), b(2, 2, A.max_items, xb), c(1, 2, A.max_items, xb); \
        if (MTV == 1 && a.total <= kMlpSmemLimit) return launch_mlp_t<1, 4, 1>(P, A, a.total, stream); \
        if (b.total <= kMlpSmemLimit) return launch_mlp_t<MTV, 2, 2>(P, A, b.total, stream);          \
        if (c.total <= kMlpSmemLimit) return launch_mlp_t<MTV, 1, 2>(P, A, c.total, stream);          \
    }
        if (two) MONO_MLP_TRY(2) else MONO_MLP_TRY(1)
#undef MONO_MLP_TRY
        int big = -1;
        for (int i = 0; i < P.nph; ++i)
            if (P.ph[i].xsmem && (big < 0 || P.ph[i].K > P.ph[big].K)) big = i;
        if (big < 0) break;
        P.ph[big].xsmem = 0;
    }
    return fail(MONO_EINVAL, "mlp: no shared-memory plan fits (M=%d)", M);
}

}  // namespace mono
