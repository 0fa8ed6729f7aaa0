// Standalone W4A8 linear (GPTQ or REF, row-major or tile-major weights) on the stream engine.
//   GPTQ: out = cast(total * x_scale[m]);   REF: out = cast(float(acc) * x_scale[m] * s_channel[n])
//   residual: out = cast(float(residual) + float(cast(f)))  (csrc/w4a8_decode.sycl:155-160)
#include <mutex>

#include "abi_internal.h"
#include "engine.cuh"

namespace mono {

struct LinearEpi {
    const float* xs;         // [M]
    const float* s_channel;  // REF: [N]
    const void* residual;    // [M][N] output dtype, or null
    void* out;               // [M][N]
    int out_bf16;
    int max_items;
};

template <int FMT, int LAYOUT, int MT, int GROUPS>
__global__ void __launch_bounds__(GROUPS * 128) linear_kernel(const Program P, const LinearEpi E) {
    extern __shared__ __align__(128) uint8_t smem[];
    const PhaseDesc& ph = P.ph[0];
    const int wg = threadIdx.x >> 7, tig = threadIdx.x & 127, warp = tig >> 5, lane = threadIdx.x & 31;
    const int M = P.M, K = ph.K, C = phase_chunks(ph), items = phase_items(ph);
    const SmemPlan<FMT, MT> plan(GROUPS, E.max_items, ph.xsmem ? M * (K + 16) : 0);
    constexpr int SBY = stage_bytes<FMT>();
    const int wid = wg * kGroupWarps + warp;
    uint64_t* bar_base = reinterpret_cast<uint64_t*>(smem + plan.rings);
    uint64_t* xbar = bar_base + GROUPS * kGroupWarps * kStages;
    uint32_t* part = reinterpret_cast<uint32_t*>(smem + plan.rings + plan.bars) + wg * 2 * E.max_items * MT * 128;
    int8_t* xsm = reinterpret_cast<int8_t*>(smem + plan.rings + plan.bars + plan.part);

    Ring<FMT, LAYOUT> ring;
    ring.buf = smem + size_t(wid) * kStages * SBY;
    ring.bars = bar_base + wid * kStages;
    const Seq sq{warp, int(blockIdx.x) * GROUPS + wg, int(gridDim.x) * GROUPS};
    if (threadIdx.x == 0 && ph.xsmem) {
        mbar_init(xbar, 1);
        fence_mbar_init();
    }
    __syncthreads();
    // weights do not depend on the preceding kernel: stream them before the dependency wait
    ring.init(P, sq, lane);
    pdl_wait();
    XSrc xs{ph.x, K, false};
    bool ok = true;
    if (ph.xsmem) {
        stage_x(ph, M, xsm, xbar);
        ok = __syncthreads_and(mbar_wait(xbar, 0));  // uniform: the tile loop holds warp-group barriers
        xs = XSrc{xsm, K + 16, true};
    }
    const int ntiles = sq.my_tiles(P, 0);
    for (int ti = 0; ti < ntiles && ok; ++ti) {
        const int T = sq.vc + ti * sq.nvc;
        uint32_t* pt = part + (ti & 1) * E.max_items * MT * 128;
        for (int item = warp; item < items; item += kGroupWarps) {
            uint32_t R[MT][4];
            consume_item<FMT, LAYOUT, MT>(ring, P, sq, xs, M, item % C, lane, R);
            store_partial<MT>(pt, item, lane, R);
        }
        group_sync(wg);
        const int N = ph.m[0].n;
        for (int e = tig; e < M * 16; e += 128) {
            const int m = e >> 4, nl = e & 15, n = T * 16 + nl;
            const uint32_t tot = tile_total<FMT, MT>(pt, C, 0, m, nl);
            float f;
            if constexpr (FMT == FMT_GPTQ) {
                f = __fmul_rn(__uint_as_float(tot), E.xs[m]);
            } else {
                f = __fmul_rn(__int2float_rn(int(tot)), E.xs[m]);
                f = __fmul_rn(f, E.s_channel[n]);
            }
            const size_t o = size_t(m) * N + n;
            if (E.out_bf16) {
                uint16_t rb = f32_to_bf16_bits(f);
                if (E.residual)
                    rb = f32_to_bf16_bits(__fadd_rn(bf16_bits_to_f32(static_cast<const uint16_t*>(E.residual)[o]),
                                                    bf16_bits_to_f32(rb)));
                static_cast<uint16_t*>(E.out)[o] = rb;
            } else {
                if (E.residual) f = __fadd_rn(static_cast<const float*>(E.residual)[o], f);
                static_cast<float*>(E.out)[o] = f;
            }
        }
    }
    ring.drain(lane);
    pdl_launch_dependents();
}

template <int FMT, int LAYOUT, int MT, int GROUPS>
static int launch_linear_t(const Program& P, const LinearEpi& E, size_t smem, cudaStream_t stream) {
    auto kern = linear_kernel<FMT, LAYOUT, MT, GROUPS>;
    static std::mutex mu;
    static size_t opt_in = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (smem > opt_in) {
            CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
            opt_in = smem;
        }
    }
    const int tiles = phase_tiles(P.ph[0]);
    const int vctas = (tiles + GROUPS - 1) / GROUPS;
    const int grid = vctas < sm_count() ? vctas : sm_count();
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
    cfg.blockDim = dim3(GROUPS * 128);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, P, E));
    return MONO_OK;
}

constexpr size_t kSmemLimit = 227 * 1024;

template <int FMT, int LAYOUT, int MT>
static int launch_linear_mt(Program& P, LinearEpi& E, cudaStream_t stream) {
    PhaseDesc& ph = P.ph[0];
    E.max_items = phase_items(ph);
    ph.xsmem = P.M * ph.K <= kXStageMax;
    for (int attempt = 0; attempt < 2; ++attempt) {
        const int xb = ph.xsmem ? P.M * (ph.K + 16) : 0;
        const SmemPlan<FMT, MT> p4(4, E.max_items, xb), p2(2, E.max_items, xb);
        if (p4.total <= kSmemLimit) return launch_linear_t<FMT, LAYOUT, MT, 4>(P, E, p4.total, stream);
        if (p2.total <= kSmemLimit) return launch_linear_t<FMT, LAYOUT, MT, 2>(P, E, p2.total, stream);
        ph.xsmem = 0;  // activations too large to stage next to the rings: read them from L2
    }
    return fail(MONO_EINVAL, "w4a8 linear: no shared-memory plan fits (M=%d K=%d)", P.M, ph.K);
}

int launch_linear(int fmt, int layout, Program& P, LinearEpi& E, cudaStream_t stream) {
    const bool two = P.M > 8;
#define MONO_LIN_CASE(F, L)                                                                      \
    if (fmt == F && layout == L)                                                                 \
        return two ? launch_linear_mt<F, L, 2>(P, E, stream) : launch_linear_mt<F, L, 1>(P, E, stream);
    MONO_LIN_CASE(FMT_GPTQ, LAYOUT_ROW)
    MONO_LIN_CASE(FMT_GPTQ, LAYOUT_TILED)
    MONO_LIN_CASE(FMT_REF, LAYOUT_ROW)
    MONO_LIN_CASE(FMT_REF, LAYOUT_TILED)
#undef MONO_LIN_CASE
    return fail(MONO_EINVAL, "w4a8 linear: unknown format %d / layout %d", fmt, layout);
}

}  // namespace mono
