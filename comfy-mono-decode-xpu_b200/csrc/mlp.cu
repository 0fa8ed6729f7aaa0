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

#include "abi_internal.h"
#include "engine.cuh"
#include "grid.cuh"
#include "rowops.cuh"

namespace mono {

struct MlpArgs {
    const uint16_t* x;       // [M][H] bf16
    const uint16_t* norm_w;  // [H] bf16 or null
    const uint16_t* lut;     // [65536] bf16: silu of every bf16 pattern
    uint16_t* out;           // [M][H] bf16
    float eps;
    int H, I, residual, max_items;
    // workspace
    uint16_t* xn;     // [M][H]
    int8_t* q1;       // [M][H]
    float* s1;        // [16]
    uint16_t* h;      // [M][I]
    unsigned* amax2;  // [16] (float bits of non-negative values)
    int8_t* q2;       // [M][I]
    float* s2;        // [16]
    unsigned* bar;    // [2] grid barrier words (zero between launches)
};

template <int MT, int GROUPS>
__global__ void __launch_bounds__(GROUPS * 128) mlp_kernel(const Program P, const MlpArgs A) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[GROUPS][16];
    __shared__ int flag;
    const int wg = threadIdx.x >> 7, tig = threadIdx.x & 127, warp = tig >> 5, lane = threadIdx.x & 31;
    const int M = P.M;
    int xbytes = 0;
    for (int i = 0; i < P.nph; ++i)
        if (P.ph[i].xsmem && M * (P.ph[i].K + 16) > xbytes) xbytes = M * (P.ph[i].K + 16);
    const SmemPlan<FMT_GPTQ, MT> plan(GROUPS, A.max_items, xbytes);
    constexpr int SBY = stage_bytes<FMT_GPTQ>();
    const int wid = wg * kGroupWarps + warp;
    uint64_t* bar_base = reinterpret_cast<uint64_t*>(smem + plan.rings);
    uint64_t* xbar = bar_base + GROUPS * kGroupWarps * kStages;
    uint32_t* part = reinterpret_cast<uint32_t*>(smem + plan.rings + plan.bars) + wg * 2 * A.max_items * MT * 128;
    int8_t* xsm = reinterpret_cast<int8_t*>(smem + plan.rings + plan.bars + plan.part);

    Ring<FMT_GPTQ, LAYOUT_TILED> ring;
    ring.buf = smem + size_t(wid) * kStages * SBY;
    ring.bars = bar_base + wid * kStages;
    const Seq sq{warp, int(blockIdx.x) * GROUPS + wg, int(gridDim.x) * GROUPS};
    if (threadIdx.x == 0) {
        mbar_init(xbar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    ring.init(P, sq, lane);
    pdl_wait();
    unsigned epoch = 0;
    bool ok = true;

    // ---- P1: norm + quant of the rows (one warp-group per row) ----
    if (blockIdx.x == 0 && threadIdx.x < 16) A.amax2[threadIdx.x] = 0u;
    for (int m = sq.vc; m < M; m += sq.nvc) {
        const uint16_t* src = A.x + size_t(m) * A.H;
        if (A.norm_w) {
            rmsnorm_row(src, A.norm_w, A.xn + size_t(m) * A.H, A.H, A.eps, red[wg], tig, wg);
            src = A.xn + size_t(m) * A.H;
        }
        quant_row(src, A.H, A.q1 + size_t(m) * A.H, A.s1 + m, red[wg], tig, wg);
    }
    ok = grid_barrier(A.bar, epoch, &flag);

    // ---- P2: gate / up, h = silu(g) * u ----
    int xpar = 0;
    auto phase_x = [&](int ph) {
        const PhaseDesc& p = P.ph[ph];
        if (!p.xsmem) return XSrc{p.x, p.K, false};
        if (threadIdx.x == 0) asm volatile("fence.proxy.async.global;" ::: "memory");
        stage_x(p, M, xsm, xbar);
        // uniform over the CTA: the tile loops hold warp-group barriers
        ok = __syncthreads_and(mbar_wait(xbar, xpar) && ok);
        xpar ^= 1;
        return XSrc{xsm, p.K + 16, true};
    };
    {
        const XSrc xs = phase_x(0);
        const PhaseDesc& ph = P.ph[0];
        const int C = phase_chunks(ph), items = phase_items(ph);
        float rmax0 = 0.f, rmax1 = 0.f;  // running |h| max of rows tig >> 4 and (tig >> 4) + 8
        const int ntiles = sq.my_tiles(P, 0);
        for (int ti = 0; ti < ntiles && ok; ++ti) {
            const int T = sq.vc + ti * sq.nvc;
            uint32_t* pt = part + (ti & 1) * A.max_items * MT * 128;
            for (int item = warp; item < items; item += kGroupWarps) {
                uint32_t R[MT][4];
                consume_item<FMT_GPTQ, LAYOUT_TILED, MT>(ring, P, sq, xs, M, item % C, lane, R);
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
    ok = grid_barrier(A.bar, epoch, &flag) && ok;

    // ---- P3: q2 = quant(h) ----
    {
        const size_t total = size_t(M) * A.I;
        const size_t stride = size_t(gridDim.x) * blockDim.x;
        for (size_t i = size_t(blockIdx.x) * blockDim.x + threadIdx.x; i < total; i += stride) {
            const int m = int(i / A.I);
            const float s = __fdiv_rn(__uint_as_float(__ldcg(A.amax2 + m)), 127.f);
            A.q2[i] = quant_one(bf16_bits_to_f32(__ldcg(A.h + i)), s);
        }
        if (blockIdx.x == 0 && threadIdx.x < M) A.s2[threadIdx.x] = __fdiv_rn(__uint_as_float(__ldcg(A.amax2 + threadIdx.x)), 127.f);
    }
    ok = grid_barrier(A.bar, epoch, &flag) && ok;

    // ---- P4: down (+ residual) ----
    {
        const XSrc xs = phase_x(1);
        const PhaseDesc& ph = P.ph[1];
        const int C = phase_chunks(ph), items = phase_items(ph);
        const int ntiles = sq.my_tiles(P, 1);
        for (int ti = 0; ti < ntiles && ok; ++ti) {
            const int T = sq.vc + ti * sq.nvc;
            uint32_t* pt = part + (ti & 1) * A.max_items * MT * 128;
            for (int item = warp; item < items; item += kGroupWarps) {
                uint32_t R[MT][4];
                consume_item<FMT_GPTQ, LAYOUT_TILED, MT>(ring, P, sq, xs, M, item % C, lane, R);
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
    ring.drain(lane);
    grid_exit(A.bar);
}

size_t mlp_workspace_bytes(int H, int I) {
    // xn, q1, h, q2 (16 rows each), s1, s2, amax2, barrier words; every piece 256-byte aligned
    auto al = [](size_t b) { return (b + 255) / 256 * 256; };
    return al(16 * size_t(H) * 2) + al(16 * size_t(H)) + al(16 * size_t(I) * 2) + al(16 * size_t(I)) + 4 * 256;
}

template <int MT, int GROUPS>
static int launch_mlp_t(const Program& P, const MlpArgs& A, size_t smem, cudaStream_t stream) {
    auto kern = mlp_kernel<MT, GROUPS>;
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
    for (int attempt = 0; attempt < 3; ++attempt) {
        int xb = 0;
        for (int i = 0; i < P.nph; ++i)
            if (P.ph[i].xsmem) xb = M * (P.ph[i].K + 16) > xb ? M * (P.ph[i].K + 16) : xb;
        if (two) {
            const SmemPlan<FMT_GPTQ, 2> p2(2, A.max_items, xb);
            if (p2.total <= kMlpSmemLimit) return launch_mlp_t<2, 2>(P, A, p2.total, stream);
        } else {
            const SmemPlan<FMT_GPTQ, 1> p2(2, A.max_items, xb);
            if (p2.total <= kMlpSmemLimit) return launch_mlp_t<1, 2>(P, A, p2.total, stream);
        }
        // drop the staging of the phase with the largest activation block
        int big = -1;
        for (int i = 0; i < P.nph; ++i)
            if (P.ph[i].xsmem && (big < 0 || P.ph[i].K > P.ph[big].K)) big = i;
        if (big < 0) break;
        P.ph[big].xsmem = 0;
    }
    return fail(MONO_EINVAL, "mlp: no shared-memory plan fits (M=%d)", M);
}

}  // namespace mono
