// Standalone W4A8 linear (GPTQ or REF, row-major or tile-major weights) on the stream engine.
//   GPTQ: out = cast(total * x_scale[m]);   REF: out = cast(float(acc) * x_scale[m] * s_channel[n])
//   residual: out = cast(float(residual) + float(cast(f)))  (csrc/w4a8_decode.sycl:155-160)
#include <cstdlib>
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

template <int FMT, int LAYOUT, int MT, int GROUPS, int ST>
__global__ void __launch_bounds__(GROUPS * 128, GROUPS == 1 ? 2 : 1) linear_kernel(const Program P, const LinearEpi E) {
    extern __shared__ __align__(128) uint8_t smem[];
    const PhaseDesc& ph = P.ph[0];
    const int wg = threadIdx.x >> 7, tig = threadIdx.x & 127, warp = tig >> 5, lane = threadIdx.x & 31;
    const int M = P.M, K = ph.K, C = phase_chunks(ph), items = phase_items(ph);
    const SmemPlan<FMT, MT> plan(GROUPS, ST, E.max_items, ph.xsmem ? M * (K + 16) : 0);
    constexpr int SBY = stage_bytes<FMT>();
    const int wid = wg * kGroupWarps + warp;
    uint64_t* bar_base = reinterpret_cast<uint64_t*>(smem + plan.rings);
    uint64_t* xbar = bar_base + GROUPS * kGroupWarps * ST;
    uint32_t* part = reinterpret_cast<uint32_t*>(smem + plan.rings + plan.bars) + wg * 2 * E.max_items * MT * 128;
    int8_t* xsm = reinterpret_cast<int8_t*>(smem + plan.rings + plan.bars + plan.part);

    Ring<FMT, LAYOUT, ST> ring;
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
    // weights do not depend on the preceding kernel: stream them before the dependency wait
    TileCursor pf = tile_start(P, sq, 0);
    const bool pf_lane = LAYOUT == LAYOUT_TILED && tig == 0;
    if (pf_lane) {
        tile_advance(P, sq, pf);  // the first tile is in the rings
        prefetch_ahead<FMT>(P, sq, pf, true);
    }
    ring.init(P, sq, lane);
    // let the next kernel in the stream launch now: its CTAs take SMs as ours exit and start streaming
    // their weights; its dependency wait still covers all of this kernel's memory effects
    pdl_launch_dependents();
    pdl_wait();
    XSrc xs{ph.x, K, false, ph.xperm != 0};
    bool ok = true;
    if (ph.xsmem) {
        ok = stage_x(ph, M, xsm, xbar, 0);
        xs = XSrc{xsm, K + 16, true, true};
    }
    trace_stamp(1);
    const int ntiles = sq.my_tiles(0);
    for (int ti = 0; ti < ntiles && ok; ++ti) {
        const int T = sq.vc + ti * sq.nvc;
        uint32_t* pt = part + (ti & 1) * E.max_items * MT * 128;
        if (pf_lane) prefetch_ahead<FMT>(P, sq, pf, false);
        for (int item = warp; item < items; item += kGroupWarps) {
            uint32_t R[MT][4];
            consume_item<FMT, LAYOUT, MT, ST>(ring, P, sq, xs, M, item % C, lane, R);
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
    trace_stamp(2);
    ring.drain(lane);
}

template <int FMT, int LAYOUT, int MT, int GROUPS, int ST>
static int launch_linear_t(const Program& P, const LinearEpi& E, size_t smem, int ctas_per_sm, cudaStream_t stream) {
    auto kern = linear_kernel<FMT, LAYOUT, MT, GROUPS, ST>;
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
    const int slots = sm_count() * ctas_per_sm;
    const int grid = vctas < slots ? vctas : slots;
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

constexpr size_t kSmemLimit = 227 * 1024;     // one CTA per SM
constexpr size_t kSmemHalf = 113 * 1024;      // two CTAs per SM (the next kernel's CTAs can co-reside)

// Launch plans (warp-groups x ring depth per warp): 16 warps with single-stage rings (the most compute
// in flight), 8 warps with 2-stage rings, or 2 CTAs of 4 warps per SM (the next kernel's CTAs can then
// co-reside). MONO_B200_PLAN=a|b|c forces one (for measurements); the default takes the first that fits.
static char plan_override() {
    static char c = [] {
        const char* v = getenv("MONO_B200_PLAN");
        return (v && (v[0] == 'a' || v[0] == 'b' || v[0] == 'c')) ? v[0] : '0';
    }();
    return c;
}

template <int FMT, int LAYOUT, int MT>
static int launch_linear_mt(Program& P, LinearEpi& E, cudaStream_t stream) {
    PhaseDesc& ph = P.ph[0];
    E.max_items = phase_items(ph);
    const char force = plan_override();
    for (int staged = 1; staged >= 0; --staged) {
        ph.xsmem = staged;
        const int xb = staged ? P.M * (ph.K + 16) : 0;
        const SmemPlan<FMT, MT> pa(4, 1, E.max_items, xb), pb(2, 2, E.max_items, xb), pc(1, 2, E.max_items, xb);
        if constexpr (MT == 1)  // (two m-tiles need more than the 128 registers a 16-warp CTA allows)
            if ((force == '0' || force == 'a') && pa.total <= kSmemLimit)
                return launch_linear_t<FMT, LAYOUT, MT, 4, 1>(P, E, pa.total, 1, stream);
        if ((force == '0' || force == 'b') && pb.total <= kSmemLimit)
            return launch_linear_t<FMT, LAYOUT, MT, 2, 2>(P, E, pb.total, 1, stream);
        if ((force == '0' || force == 'c') && pc.total <= kSmemHalf)
            return launch_linear_t<FMT, LAYOUT, MT, 1, 2>(P, E, pc.total, 2, stream);
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
