// Fused decode MLP block in one cooperative launch (the role of csrc/mono_mlp.sycl:34-180 and of the MLP
// phases 3-6 of layer_post, csrc/mono_layer.sycl:272-313), GPTQ W4A8:
//
//   xn = RMSNorm(x) (or x when no norm weight); q1, s1 = quant(xn)
//   g, u = W4A8 gate / up (q1);  h = bf16(silu_lut[bf16 g] * bf16 u);  q2, s2 = quant(h)
//   out = bf16(x + bf16(W4A8 down (q2)))  (or bf16(W4A8 down (q2)) without the residual)
//
// Phases are separated by bounded grid barriers; the weight rings run across them, so gate / up and down
// weights stream while rows are normalized and quantized.
#include <algorithm>
#include <mutex>

#include "launch.h"
#include "grid.cuh"
#include "rowops.cuh"
#include "stream.cuh"

namespace mono {

// One CTA per SM (cooperative): CW consumer + PW producer warps (stream.cuh) and a ring of S stages; the
// producers stream the gate / up and then the down weights from the first instruction, straight through the
// row phases and the grid barriers. The down tiles are dealt in reverse CTA order (PhaseDesc::rev): the CTAs with
// an extra gate / up tile get fewer down tiles, and their rings carry the difference across the barriers.
//
//   P1  rows: row m on CTA m (norm_quant_row_cta, the pinned order) -> q1, s1;  barrier;  every CTA stages q1
//   P2  gate / up tiles: h = bf16(silu_lut[bf16 g] * bf16 u) to the workspace, row maxima of |h| (atomic max,
//       order-free);  barrier
//   P3  q2 = quant(h), spread over all CTAs;  barrier;  every CTA stages q2 (when it fits next to the ring; else
//       the down items read it through L2)
//   P4  down tiles: out = bf16(x + bf16(total * s2)) (or without the residual)
// The last CTA to leave clears the row maxima for the next launch (every CTA has read them by then).
// Measured alternatives (not kept): every CTA preparing all rows itself, or quantizing all of h itself, to drop
// a barrier: the per-element work of M full rows on one SM outweighs a barrier (12 us against 6 us for P1 at
// M = 5; every CTA quantizing all 8 x 12288 values of h while staging them, with 16 loads in flight per thread:
// P3 28 us against 6 us, about 17 instructions per value, i.e. ~15k issue cycles per SM); and tiles split across
// CTAs for an even item count: the exchange of the cut tiles' partials costs three L2 round trips per phase.
template <int MT, int CW, int PW>
__global__ void __launch_bounds__((CW + PW) * 32, 1) mlp_kernel(const Program P, const MlpArgs A, const MlpShape Z) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[64];
    __shared__ float s1s[kStreamMaxRows], s2s[kStreamMaxRows];
    __shared__ unsigned rowmax[kStreamMaxRows];
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
    constexpr int NT = CW * 32, NWG = CW / 4;
    pdl_wait();
    trace_stamp(1);
    unsigned epoch = 0;
    bool ok = true;

    // ---- P1: RMSNorm + quant of the rows: row m on CTA m (all consumer threads) to the workspace, a grid
    // barrier, then every CTA stages them ----
    for (int m = int(blockIdx.x); m < M; m += int(gridDim.x))
        norm_quant_row_cta<NT, kConsumerBar>(A.x + size_t(m) * A.H, A.norm_w, A.eps, A.H, nullptr, A.q1 + size_t(m) * A.H,
                                             A.s1 + m, red);
    if (threadIdx.x < kStreamMaxRows) rowmax[threadIdx.x] = 0u;
    trace_stamp(12);
    ok = grid_barrier_named<kConsumerBar, NT>(A.bar, epoch, &flag) && ok;
    trace_stamp(13);
    stage_x_consumers<CW>(A.q1, M, A.H, true, xsm, A.s1, s1s);  // the rows and their scales in one round trip
    trace_stamp(2);

    // ---- P2: gate / up, h = silu(g) * u, row maxima of |h| (tiles in batches of Z.tb0: the partials of a batch
    // fit the shared buffer; one batch unless the rows are many) ----
    {
        const PhaseDesc& ph = P.ph[0];
        const XSrc xs{xsm, A.H + 16, true, true};
        const int C = phase_chunks(ph), ntl = cta_tiles(ph), TB = Z.tb0;
        for (int k0 = 0; k0 < ntl && ok; k0 += TB) {
        const int kb = ntl - k0 < TB ? ntl - k0 : TB;
        ok = consume_phase<FMT_GPTQ, LAYOUT_TILED, MT, CW>(P, 0, xs, ring, full, empty, S, part, warp, lane, k0 * 2 * C,
                                                           kb * 2 * C) && ok;
        ok = consumer_sync_and<CW>(ok);
        if (k0 + kb >= ntl) trace_stamp(3);
        for (int e = threadIdx.x; e < kb * M * 16 && ok; e += NT) {
            const int k = e / (M * 16), r = e - k * (M * 16), m = r >> 4, nl = r & 15;
            const int n = cta_tile(ph, k0 + k) * 16 + nl;
            const uint32_t* pk = part + size_t(k) * 2 * C * MT * 128;
            const float s = s1s[m];
            const float tg = __uint_as_float(tile_total<FMT_GPTQ, MT>(pk, C, 0, m, nl));
            const float tu = __uint_as_float(tile_total<FMT_GPTQ, MT>(pk, C, 1, m, nl));
            const uint16_t gb = f32_to_bf16_bits(__fmul_rn(tg, s));
            const float u = bf16_round(__fmul_rn(tu, s));
            const uint16_t hb = f32_to_bf16_bits(__fmul_rn(bf16_bits_to_f32(A.lut[gb]), u));
            A.h[size_t(m) * A.I + n] = hb;
            atomicMax(&rowmax[m], __float_as_uint(fabsf(bf16_bits_to_f32(hb))));
        }
        consumer_sync<CW>();  // the batch's partials are read before the next batch writes them
        }
        if (threadIdx.x < M) atomicMax(A.amax2 + threadIdx.x, rowmax[threadIdx.x]);
    }
    trace_stamp(4);
    ok = grid_barrier_named<kConsumerBar, NT>(A.bar, epoch, &flag) && ok;
    trace_stamp(5);

    // ---- P3: q2 = quant(h) ----
    XSrc xs1{A.q2, A.I, false, true, true};
    {
        // 8-element pieces: one 16-byte load of h, one 8-byte store of permuted q2, spread over all CTAs; the
        // thread's first piece is loaded before the row maxima, so both loads are in flight together
        const int ppr = A.I >> 3, pieces = M * ppr;
        const int stride = int(gridDim.x) * NT, i0 = int(blockIdx.x) * NT + int(threadIdx.x);
        uint4 h0 = make_uint4(0, 0, 0, 0);
        if (i0 < pieces) h0 = __ldcg(reinterpret_cast<const uint4*>(A.h) + i0);
        if (threadIdx.x < M) s2s[threadIdx.x] = __fdiv_rn(__uint_as_float(__ldcg(A.amax2 + threadIdx.x)), 127.f);
        consumer_sync<CW>();
        trace_stamp(9);
        for (int i = i0; i < pieces; i += stride) {
            const int m = i / ppr;
            const uint4 hv = i == i0 ? h0 : __ldcg(reinterpret_cast<const uint4*>(A.h) + i);
            const uint32_t u[4] = {hv.x, hv.y, hv.z, hv.w};
            float v[8];
#pragma unroll
            for (int e = 0; e < 8; ++e) v[e] = __uint_as_float((e & 1) ? (u[e >> 1] & 0xFFFF0000u) : (u[e >> 1] << 16));
            reinterpret_cast<uint2*>(A.q2)[i] = quant8_perm(v, s2s[m]);
        }
        trace_stamp(10);
        ok = grid_barrier_named<kConsumerBar, NT>(A.bar, epoch, &flag) && ok;
        trace_stamp(11);
        if (P.ph[1].xsmem) {
            stage_x_consumers<CW, 16>(A.q2, M, A.I, true, xsm);  // 16 loads in flight: one round trip at 8 rows
            xs1 = XSrc{xsm, A.I + 16, true, true};
        }
    }
    trace_stamp(6);

    // ---- P4: down (+ residual), tiles in batches of Z.tb1 ----
    {
        const PhaseDesc& ph = P.ph[1];
        const int C = phase_chunks(ph), ntl = cta_tiles(ph), TB = Z.tb1;
        for (int k0 = 0; k0 < ntl && ok; k0 += TB) {
            const int kb = ntl - k0 < TB ? ntl - k0 : TB;
            ok = consume_phase<FMT_GPTQ, LAYOUT_TILED, MT, CW>(P, 1, xs1, ring, full, empty, S, part, warp, lane, k0 * C,
                                                               kb * C) && ok;
            ok = consumer_sync_and<CW>(ok);
            if (k0 + kb >= ntl) trace_stamp(7);
            for (int e = threadIdx.x; e < kb * M * 16 && ok; e += NT) {
                const int k = e / (M * 16), r = e - k * (M * 16), m = r >> 4, nl = r & 15;
                const int n = cta_tile(ph, k0 + k) * 16 + nl;
                const float tot = __uint_as_float(tile_total<FMT_GPTQ, MT>(part + size_t(k) * C * MT * 128, C, 0, m, nl));
                uint16_t rr = f32_to_bf16_bits(__fmul_rn(tot, s2s[m]));
                const size_t o = size_t(m) * A.H + n;
                if (A.residual) rr = f32_to_bf16_bits(__fadd_rn(bf16_bits_to_f32(A.x[o]), bf16_bits_to_f32(rr)));
                A.out[o] = rr;
            }
            consumer_sync<CW>();
        }
    }
    trace_stamp(8);
    // exit: the last CTA resets the barrier words and clears the row maxima
    asm volatile("bar.sync %0, %1;" ::"n"(kConsumerBar), "n"(NT) : "memory");
    if (threadIdx.x == 0) {
        __threadfence();
        if (atomicAdd(A.bar + 1, 1u) == gridDim.x - 1) {
            for (int m = 0; m < kStreamMaxRows; ++m) atomicExch(A.amax2 + m, 0u);
            atomicExch(A.bar, 0u);
            atomicExch(A.bar + 1, 0u);
        }
    }
}

size_t mlp_workspace_bytes(int H, int I) {
    // q1, h, q2 (kStreamMaxRows rows each), s1, amax2, barrier words; every piece 256-byte aligned
    auto al = [](size_t b) { return (b + 255) / 256 * 256; };
    const size_t R = kStreamMaxRows;
    return al(R * size_t(H)) + al(R * size_t(I) * 2) + al(R * size_t(I)) + 4 * 256;
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


// Stream configuration c of kStreamConfig (consumer and producer warps; the ring depth is the plan's).
template <int MT>
static int dispatch_mlp(int c, Program& P, MlpArgs& A, const MlpShape& Z, size_t smem, cudaStream_t stream) {
    switch (c) {
        case 0: return launch_mlp_t<MT, 10, 2>(P, A, Z, smem, stream);
        case 2: return launch_mlp_t<MT, 12, 4>(P, A, Z, smem, stream);
        default: return launch_mlp_t<MT, 8, 4>(P, A, Z, smem, stream);  // configs 1 and 3
    }
}

int launch_mlp(Program& P, MlpArgs& A, cudaStream_t stream) {
    const int M = P.M, G = sm_count();
    const int MT = M > 16 ? 4 : (M > 8 ? 2 : 1);
    // partials per tile (items x MT 8-row tiles x 128 words) and the CTA's tiles of each phase
    int per_cta[2];
    size_t tile_bytes[2];
    for (int i = 0; i < 2; ++i) {
        const int nt = phase_tiles(P.ph[i]);
        per_cta[i] = (nt + G - 1) / G;
        tile_bytes[i] = size_t(P.ph[i].paired ? 2 : 1) * phase_chunks(P.ph[i]) * MT * 128 * 4;
    }
    P.ph[0].rev = 0;
    P.ph[1].rev = 1;
    A.max_items = 0;
    // the first phase's block is always staged (P1 writes it); the down phase's when it fits next to the ring.
    // Pass 0: every tile's partials at once (one batch per phase); pass 1 (many rows): tiles in batches.
    P.ph[0].xsmem = 1;
    for (int pass = 0; pass < 2; ++pass)
        for (int staged = 1; staged >= 0; --staged) {
            P.ph[1].xsmem = staged;
            size_t xb = size_t(M) * (P.ph[0].K + 16);
            if (staged) xb = std::max(xb, size_t(M) * (P.ph[1].K + 16));
            for (int c = 0; c < kStreamConfigs; ++c) {
                const StreamConfig sc = kStreamConfig[c];
                int tb0 = per_cta[0], tb1 = per_cta[1];
                if (pass == 1) {
                    const StreamPlan bare(stage_bytes<FMT_GPTQ>(), sc.S, 0, xb, 0);
                    if (bare.total >= kStreamSmemLimit) continue;
                    const size_t budget = (kStreamSmemLimit - bare.total) / 128 * 128;
                    tb0 = std::min<int>(tb0, int(budget / tile_bytes[0]));
                    tb1 = std::min<int>(tb1, int(budget / tile_bytes[1]));
                    if (tb0 < 1 || tb1 < 1) continue;
                }
                const size_t part = std::max(size_t(tb0) * tile_bytes[0], size_t(tb1) * tile_bytes[1]);
                const StreamPlan plan(stage_bytes<FMT_GPTQ>(), sc.S, part, xb, 0);
                if (plan.total > kStreamSmemLimit) continue;
                const MlpShape Z{sc.S, int(part), int(xb), tb0, tb1};
                if (MT == 1) return dispatch_mlp<1>(c, P, A, Z, plan.total, stream);
                if (MT == 2) return dispatch_mlp<2>(c, P, A, Z, plan.total, stream);
                return dispatch_mlp<4>(c, P, A, Z, plan.total, stream);
            }
        }
    return fail(MONO_EINVAL, "mlp: no shared-memory plan fits (M=%d)", M);
}

}  // namespace mono
