// Standalone W4A8 linear (GPTQ or REF, row-major or tile-major weights) on the stream engine (stream.cuh).
//   GPTQ: out = cast(total * x_scale[m]);   REF: out = cast(float(acc) * x_scale[m] * s_channel[n])
//   residual: out = cast(float(residual) + float(cast(f)))  (csrc/w4a8_decode.sycl:155-160)
#include <cstdlib>
#include <mutex>

#include "launch.h"
#include "rowops.cuh"
#include "stream.cuh"

namespace mono {

// One CTA per SM: 12 consumer warps + 4 producer warps (stream.cuh), S = 12 ring stages (one per consumer
// warp, three per producer: 101 KB of weights in flight per SM).
constexpr int kLinCW = 12, kLinPW = 4, kLinThreads = (kLinCW + kLinPW) * 32;

template <int FMT, int LAYOUT, int MT>
__global__ void __launch_bounds__(kLinThreads, 1) linear_kernel(const Program P, const LinearEpi E, const int S) {
    extern __shared__ __align__(128) uint8_t smem[];
    const PhaseDesc& ph = P.ph[0];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int M = P.M, K = ph.K, C = phase_chunks(ph);
    const size_t part_bytes = size_t(E.max_items) * MT * 128 * 4;
    const StreamPlan plan(stage_bytes<FMT>(), S, part_bytes, ph.xsmem ? size_t(M) * (K + 16) : 0, 128);
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + plan.ring);
    uint64_t* empty = full + S;
    uint32_t* part = reinterpret_cast<uint32_t*>(smem + plan.ring + plan.bars);
    int8_t* xsm = reinterpret_cast<int8_t*>(smem + plan.ring + plan.bars + plan.part);
    float* xs_sm = reinterpret_cast<float*>(smem + plan.ring + plan.bars + plan.part + plan.x);  // [16] row scales
    unsigned* rowmax = reinterpret_cast<unsigned*>(xs_sm + 16);                                 // [16]
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], LAYOUT == LAYOUT_TILED ? 1 : 32);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    trace_stamp(0);
    // let the next kernel in the stream launch now: its CTAs take SMs as ours exit and start streaming
    // their weights; its dependency wait still covers all of this kernel's memory effects
    pdl_launch_dependents();
    if (warp >= kLinCW) {
        // weights do not depend on the preceding kernel: stream them before (without) the dependency wait
        produce_all<FMT, LAYOUT, kLinPW>(P, ring, full, empty, S, warp - kLinCW, lane);
        return;
    }
    pdl_wait();
    XSrc xs{ph.x, K, false, ph.xperm != 0};
    if (E.xb) {
        // every CTA quantizes all M rows itself straight into shared memory
        quant_block<kLinCW * 32, kConsumerBar>(E.xb, M, K, xsm, K + 16, xs_sm, rowmax);
        xs = XSrc{xsm, K + 16, true, true};
    } else if (ph.xsmem) {
        stage_x_consumers<kLinCW>(ph.x, M, K, ph.xperm != 0, xsm);
        xs = XSrc{xsm, K + 16, true, true};
    }
    trace_stamp(1);
    // tiles in batches of E.max_items / C (the partials of one batch fit the shared buffer), epilogue per batch
    const int N = ph.m[0].n, ntl = cta_tiles(ph), TB = E.max_items / C;
    bool all_ok = true;
    for (int k0 = 0; k0 < ntl && all_ok; k0 += TB) {
        const int kb = ntl - k0 < TB ? ntl - k0 : TB;
        const bool ok = consume_phase<FMT, LAYOUT, MT, kLinCW>(P, 0, xs, ring, full, empty, S, part, warp, lane, k0 * C,
                                                               kb * C);
        all_ok = consumer_sync_and<kLinCW>(ok);
        if (k0 == 0) trace_stamp(2);
        if (!all_ok) break;
        for (int e = threadIdx.x; e < kb * M * 16; e += kLinCW * 32) {
            const int kk = e / (M * 16), r = e - kk * (M * 16), m = r >> 4, nl = r & 15;
            const int n = (int(blockIdx.x) + (k0 + kk) * int(gridDim.x)) * 16 + nl;
            const uint32_t tot = tile_total<FMT, MT>(part + size_t(kk) * C * MT * 128, C, 0, m, nl);
            float f;
            const float xsv = E.xb ? xs_sm[m] : E.xs[m];
            if constexpr (FMT == FMT_GPTQ) {
                f = __fmul_rn(__uint_as_float(tot), xsv);
            } else {
                f = __fmul_rn(__int2float_rn(int(tot)), xsv);
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
        consumer_sync<kLinCW>();  // the batch's partials are read before the next batch writes them
    }
    trace_stamp(3);
}

constexpr size_t kSmemLimit = 227 * 1024;

template <int FMT, int LAYOUT, int MT>
static int launch_linear_mt(Program& P, LinearEpi& E, cudaStream_t stream) {
    PhaseDesc& ph = P.ph[0];
    const int tiles = phase_tiles(ph), grid = tiles < sm_count() ? tiles : sm_count();
    const int tiles_cta = (tiles + grid - 1) / grid, C = phase_chunks(ph);
    // partial slots: the CTA's tiles in batches of at most 16 (for very wide matrices such as an lm_head)
    E.max_items = (tiles_cta < 16 ? tiles_cta : 16) * C;
    const size_t part_bytes = size_t(E.max_items) * MT * 128 * 4;
    // stage the activations when they fit next to the partials and the ring
    for (int staged = 1; staged >= (E.xb ? 1 : 0); --staged) {
        ph.xsmem = staged;
        const size_t xb = staged ? size_t(P.M) * (ph.K + 16) : 0;
        const StreamPlan plan(stage_bytes<FMT>(), kLinCW, part_bytes, xb, 128);
        if (plan.total > kSmemLimit) continue;
        auto kern = linear_kernel<FMT, LAYOUT, MT>;
        static std::mutex mu;
        static size_t opt_in = 0;
        {
            std::lock_guard<std::mutex> lock(mu);
            if (plan.total > opt_in) {
                CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(plan.total)));
                opt_in = plan.total;
            }
        }
        cudaLaunchConfig_t cfg = {};
        cfg.gridDim = dim3(grid);
        cfg.blockDim = dim3(kLinThreads);
        cfg.dynamicSmemBytes = plan.total;
        cfg.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
        attr[0].val.programmaticStreamSerializationAllowed = 1;
        cfg.attrs = attr;
        cfg.numAttrs = 1;
        CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, P, E, plan.S));
        return MONO_OK;
    }
    return fail(MONO_EINVAL, "w4a8 linear: no shared-memory plan fits (M=%d K=%d N=%d%s)", P.M, ph.K, ph.m[0].n,
                E.xb ? ", bf16 input quantized in shared memory" : "");
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
