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
#include "stream.cuh"

namespace mono {

// One CTA per SM (cooperative): 12 consumer warps + 4 producer warps (stream.cuh), S = 12 ring stages. The
// producers stream gate/up and then down weights straight through the row phases and the grid barriers.
// Warp configurations (consumer warps CW, producer warps PW, ring stages S = a common multiple): the deepest
// ring that fits next to the partials and the staged activations is taken (stream_config in stream.cuh).

template <int MT, int CW, int PW>
__global__ void __launch_bounds__((CW + PW) * 32, 1) mlp_kernel(const Program P, const MlpArgs A, const MlpShape Z) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[64];
    __shared__ unsigned rowmax[16];
    __shared__ int flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int M = P.M, S = Z.S;
    const StreamPlan plan(stage_bytes<FMT_GPTQ>(), S, Z.part_bytes, Z.x_bytes, 0);
    uint8_t* ring = smem;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + plan.ring);
    uint64_t* empty = full + S;
    uint32_t* part = reinterpret_cast<uint32_t*>(smem + plan.ring + plan.bars);
    int8_t* xsm = reinterpret_cast<int8_t*>(smem + plan.ring + plan.bars + plan.part);
    if (threadIdx.x == 0) {
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], 1);
        }
        fence_mbar_init();
    }
    __syncthreads();
    trace_stamp(0);
    pdl_launch_dependents();  // the next kernel may launch and stream its weights as our CTAs exit
    if (warp >= CW) {
        // weights do not depend on the preceding kernel: stream them before (without) the dependency wait
        produce_all<FMT_GPTQ, LAYOUT_TILED, PW>(P, ring, full, empty, S, warp - CW, lane);
        return;
    }
    constexpr int NT = CW * 32;
    pdl_wait();
    trace_stamp(1);
    unsigned epoch = 0;
    bool ok = true;

    // ---- P1: norm + quant of the rows (one warp-group of consumers per row) ----
    if (blockIdx.x == 0 && threadIdx.x < 16) A.amax2[threadIdx.x] = 0u;
    // row m on CTA m, all consumer threads (rowops.cuh: the pinned order of the warp-group form)
    for (int m = int(blockIdx.x); m < M; m += int(gridDim.x))
        norm_quant_row_cta<NT, kConsumerBar>(A.x + size_t(m) * A.H, A.norm_w, A.eps, A.H, nullptr, A.q1 + size_t(m) * A.H,
                                             A.s1 + m, red);
    trace_stamp(2);
    ok = grid_barrier_named<kConsumerBar, NT>(A.bar, epoch, &flag);
    trace_stamp(3);

    auto phase_x = [&](int ph) {
        const PhaseDesc& p = P.ph[ph];
        if (!p.xsmem) return XSrc{p.x, p.K, false, true, true};  // written by this launch: L2 reads
        stage_x_consumers<CW>(p.x, M, p.K, true, xsm);
        return XSrc{xsm, p.K + 16, true, true};
    };

    // ---- P2: gate / up, h = silu(g) * u, row maxima of |h| ----
    {
        const XSrc xs = phase_x(0);
        trace_stamp(4);
        const PhaseDesc& ph = P.ph[0];
        const int C = phase_chunks(ph), ntl = cta_tiles(ph);
        if (threadIdx.x < 16) rowmax[threadIdx.x] = 0u;
        ok = consume_phase<FMT_GPTQ, LAYOUT_TILED, MT, CW>(P, 0, xs, ring, full, empty, S, part, warp, lane) && ok;
        ok = consumer_sync_and<CW>(ok);
        for (int e = threadIdx.x; e < ntl * M * 16 && ok; e += NT) {
            const int k = e / (M * 16), r = e - k * (M * 16), m = r >> 4, nl = r & 15;
            const int n = (int(blockIdx.x) + k * int(gridDim.x)) * 16 + nl;
            const uint32_t* pk = part + size_t(k) * 2 * C * MT * 128;
            const float s = __ldcg(A.s1 + m);
            const float tg = __uint_as_float(tile_total<FMT_GPTQ, MT>(pk, C, 0, m, nl));
            const float tu = __uint_as_float(tile_total<FMT_GPTQ, MT>(pk, C, 1, m, nl));
            const uint16_t gb = f32_to_bf16_bits(__fmul_rn(tg, s));
            const float u = bf16_round(__fmul_rn(tu, s));
            const uint16_t hb = f32_to_bf16_bits(__fmul_rn(bf16_bits_to_f32(A.lut[gb]), u));
            A.h[size_t(m) * A.I + n] = hb;
            atomicMax(&rowmax[m], __float_as_uint(fabsf(bf16_bits_to_f32(hb))));
        }
        consumer_sync<CW>();
        if (threadIdx.x < M) atomicMax(A.amax2 + threadIdx.x, rowmax[threadIdx.x]);
    }
    trace_stamp(5);
    ok = grid_barrier_named<kConsumerBar, NT>(A.bar, epoch, &flag) && ok;
    trace_stamp(6);

    // ---- P3: q2 = quant(h) ----
    {
        // 8-element pieces: one 16-byte load of h, one 8-byte store of permuted q2
        const int ppr = A.I >> 3, pieces = M * ppr;
        const int stride = int(gridDim.x) * NT;
        for (int i = int(blockIdx.x) * NT + int(threadIdx.x); i < pieces; i += stride) {
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
    ok = grid_barrier_named<kConsumerBar, NT>(A.bar, epoch, &flag) && ok;
    trace_stamp(8);

    // ---- P4: down (+ residual) ----
    {
        const XSrc xs = phase_x(1);
        trace_stamp(9);
        const PhaseDesc& ph = P.ph[1];
        const int C = phase_chunks(ph), ntl = cta_tiles(ph);
        ok = consume_phase<FMT_GPTQ, LAYOUT_TILED, MT, CW>(P, 1, xs, ring, full, empty, S, part, warp, lane) && ok;
        ok = consumer_sync_and<CW>(ok);
        for (int e = threadIdx.x; e < ntl * M * 16 && ok; e += NT) {
            const int k = e / (M * 16), r = e - k * (M * 16), m = r >> 4, nl = r & 15;
            const int n = (int(blockIdx.x) + k * int(gridDim.x)) * 16 + nl;
            const float s = __fdiv_rn(__uint_as_float(__ldcg(A.amax2 + m)), 127.f);
            const float tot = __uint_as_float(tile_total<FMT_GPTQ, MT>(part + size_t(k) * C * MT * 128, C, 0, m, nl));
            uint16_t rr = f32_to_bf16_bits(__fmul_rn(tot, s));
            const size_t o = size_t(m) * A.H + n;
            if (A.residual) rr = f32_to_bf16_bits(__fadd_rn(bf16_bits_to_f32(A.x[o]), bf16_bits_to_f32(rr)));
            A.out[o] = rr;
        }
    }
    trace_stamp(10);
    grid_exit_named<kConsumerBar, NT>(A.bar);
}

size_t mlp_workspace_bytes(int H, int I) {
    // xn, q1, h, q2 (16 rows each), s1, s2, amax2, barrier words; every piece 256-byte aligned
    auto al = [](size_t b) { return (b + 255) / 256 * 256; };
    return al(16 * size_t(H) * 2) + al(16 * size_t(H)) + al(16 * size_t(I) * 2) + al(16 * size_t(I)) + 4 * 256;
}

template <int MT, int CW, int PW>
static int launch_mlp_t(const Program& P, const MlpArgs& A, const MlpShape& Z, size_t smem, cudaStream_t stream) {
    auto kern = mlp_kernel<MT, CW, PW>;
    static std::mutex mu;
    static size_t opt_in = 0;
    static int per_sm = 0;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (smem > opt_in) {
            CUDA_TRY(cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
            opt_in = smem;
            CUDA_TRY(cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, kern, (CW + PW) * 32, smem));
        }
    }
    if (per_sm < 1) return fail(MONO_EINVAL, "mlp: one CTA does not fit an SM (%zu B shared)", smem);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(sm_count());
    cfg.blockDim = dim3((CW + PW) * 32);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeCooperative;
    attr[0].val.cooperative = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 2;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, kern, P, A, Z));
    return MONO_OK;
}


int launch_mlp(Program& P, MlpArgs& A, cudaStream_t stream) {
    const int M = P.M, G = sm_count();
    const bool two = M > 8;
    const int MT = two ? 2 : 1;
    // partials: the larger phase's items of one CTA
    size_t part = 0;
    for (int i = 0; i < P.nph; ++i) {
        const int nt = phase_tiles(P.ph[i]), per_cta = (nt + G - 1) / G;
        const size_t b = size_t(per_cta) * (P.ph[i].paired ? 2 : 1) * phase_chunks(P.ph[i]) * MT * 128 * 4;
        part = b > part ? b : part;
    }
    A.max_items = 0;
    // stage every phase's activations when they fit next to the ring; else drop the largest block
    for (int i = 0; i < P.nph; ++i) P.ph[i].xsmem = 1;
    for (int attempt = 0; attempt <= P.nph; ++attempt) {
        size_t xb = 0;
        for (int i = 0; i < P.nph; ++i)
            if (P.ph[i].xsmem) xb = size_t(M) * (P.ph[i].K + 16) > xb ? size_t(M) * (P.ph[i].K + 16) : xb;
        for (int c = 0; c < kStreamConfigs; ++c) {
            const StreamConfig sc = kStreamConfig[c];
            const StreamPlan plan(stage_bytes<FMT_GPTQ>(), sc.S, part, xb, 0);
            if (plan.total > kStreamSmemLimit) continue;
            const MlpShape Z{sc.S, int(part), int(xb)};
#define MONO_MLP(MTV, CWV, PWV) return launch_mlp_t<MTV, CWV, PWV>(P, A, Z, plan.total, stream)
            if (!two) {
                if (c == 0) MONO_MLP(1, 10, 2);
                if (c == 1) MONO_MLP(1, 8, 4);
                MONO_MLP(1, 12, 4);
            } else {
                if (c == 0) MONO_MLP(2, 10, 2);
                if (c == 1) MONO_MLP(2, 8, 4);
                MONO_MLP(2, 12, 4);
            }
#undef MONO_MLP
        }
        int big = -1;
        for (int i = 0; i < P.nph; ++i)
            if (P.ph[i].xsmem && (big < 0 || P.ph[i].K > P.ph[big].K)) big = i;
        if (big < 0) break;
        P.ph[big].xsmem = 0;
    }
    return fail(MONO_EINVAL, "mlp: no shared-memory plan fits (M=%d)", M);
}

}  // namespace mono
