// Row preparation + W4A8 GPTQ linear in one cooperative launch: the reference's layer_pre (input RMSNorm ->
// quantization -> q / k / v projections, csrc/mono_layer.sycl:69-155) and the front of layer_post (sigmoid gate
// -> quantization -> out projection + residual, csrc/mono_layer.sycl:243-270), on the stream engine.
//
//   P1 rows  mode NORM:  xn = RMSNorm(x; w) (pinned order, rowops.cuh), q, s = quant(xn)   (xn_out optional)
//            mode GATE:  y = bf16(x * sigmoid_lut[gate]), q, s = quant(y)   (gate element (m, c) at
//                        gate[m * gate_row_stride + (c / 256) * gate_head_stride + c % 256])
//            mode QUANT: q, s = quant(x)
//   P2 all   out[m][n] = bf16(total[m][n] * s[m]) (+ residual: bf16(residual + that)) for the up to three
//            matrices of the phase, outputs concatenated along n (row stride = the sum of their rows)
// The producer warps stream the weights from the start, across the row phase and the grid barrier.
#include <algorithm>
#include <mutex>

#include "launch.h"
#include "gdn.cuh"
#include "grid.cuh"
#include "rowops.cuh"
#include "stream.cuh"

namespace mono {

// Warp configurations (consumer warps CW, producer warps PW, ring stages S = a common multiple): the deepest
// ring that fits next to the partials and the staged activations is taken (stream_config in stream.cuh).

template <int MT, int CW, int PW>
__global__ void __launch_bounds__((CW + PW) * 32, 1) rowlin_kernel(const Program P, const RowLinArgs A, const MlpShape Z) {
    extern __shared__ __align__(128) uint8_t smem[];
    __shared__ float red[64];
    __shared__ float ss[kStreamMaxRows];  // the row scales, staged with the rows
    __shared__ int flag;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int M = P.M, S = Z.S, K = P.ph[0].K;
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
    pdl_launch_dependents();
    if (warp >= CW) {
        produce_all<FMT_GPTQ, LAYOUT_TILED, PW>(P, ring, full, empty, S, warp - CW, lane);
        return;
    }
    constexpr int NT = CW * 32;
    const int ab_col = int(gridDim.x) - 1 - int(blockIdx.x);
    const bool ab = A.ab_out != nullptr && ab_col < A.ab_n;
    if (ab && threadIdx.x == 0)  // the a | b column's weights (constant) into L2 for the tail phase
        asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(A.ab_w + size_t(ab_col) * K), "r"(K * 2)
                     : "memory");
    pdl_wait();
    trace_stamp(1);
    unsigned epoch = 0;
    bool ok = true;
    // row m on CTA m, all consumer threads (rowops.cuh: the pinned order of the warp-group forms)
    for (int m = int(blockIdx.x); m < M; m += int(gridDim.x)) {
        const uint16_t* xr = A.x + size_t(m) * K;
        if (A.mode == ROWLIN_GATE)
            gate_quant_row_cta<NT, kConsumerBar>(xr, A.gate + size_t(m) * A.gate_row_stride, A.gate_head_stride, A.lut, K,
                                                 A.q + size_t(m) * K, A.s + m, red);
        else
            norm_quant_row_cta<NT, kConsumerBar>(xr, A.mode == ROWLIN_NORM ? A.norm_w : nullptr, A.eps, K,
                                                 A.xn_out ? A.xn_out + size_t(m) * K : nullptr, A.q + size_t(m) * K,
                                                 A.s + m, red);
    }
    trace_stamp(2);
    ok = grid_barrier_named<kConsumerBar, NT>(A.bar, epoch, &flag);
    trace_stamp(3);
    const PhaseDesc& ph = P.ph[0];
    XSrc xs{ph.x, K, false, true, true};  // written by this launch: L2 reads
    if (ph.xsmem) {
        stage_x_consumers<CW>(ph.x, M, K, true, xsm, A.s, ss);  // the rows and their scales in one round trip
        xs = XSrc{xsm, K + 16, true, true};
    } else {
        if (int(threadIdx.x) < M) ss[threadIdx.x] = __ldcg(A.s + threadIdx.x);
        consumer_sync<CW>();
    }
    trace_stamp(4);
    // tiles in batches of Z.tb0 (the partials of a batch fit the shared buffer; one batch unless the rows are many)
    const int C = phase_chunks(ph), ntl = cta_tiles(ph), TB = Z.tb0;
    for (int k0 = 0; k0 < ntl && ok; k0 += TB) {
        const int kb = ntl - k0 < TB ? ntl - k0 : TB;
        ok = consume_phase<FMT_GPTQ, LAYOUT_TILED, MT, CW>(P, 0, xs, ring, full, empty, S, part, warp, lane, k0 * C,
                                                           kb * C) && ok;
        ok = consumer_sync_and<CW>(ok);
        for (int e = threadIdx.x; e < kb * M * 16 && ok; e += NT) {
            const int k = e / (M * 16), r = e - k * (M * 16), m = r >> 4, nl = r & 15;
            const int n = (int(blockIdx.x) + (k0 + k) * int(gridDim.x)) * 16 + nl;  // concatenated output column
            const float tot = __uint_as_float(tile_total<FMT_GPTQ, MT>(part + size_t(k) * C * MT * 128, C, 0, m, nl));
            uint16_t rr = f32_to_bf16_bits(__fmul_rn(tot, ss[m]));
            const size_t o = size_t(m) * A.N + n;
            if (A.residual) rr = f32_to_bf16_bits(__fadd_rn(bf16_bits_to_f32(A.residual[o]), bf16_bits_to_f32(rr)));
            A.out[o] = rr;
        }
        consumer_sync<CW>();  // the batch's partials are read before the next batch writes them
    }
    trace_stamp(5);
    if (ab && ok) {
        // GDN a | b column ab_col on a CTA with the fewest GEMV tiles: warp w takes quarter w & 3 of the rows
        // w / 4, w / 4 + RG, .. (gdn.cuh gdn_ab_quarter: the order of mono_gdn_ab); the normalized rows (written
        // in P1, before the grid barrier) are copied in blocks into the ring, idle once every item is consumed.
        constexpr int RG = CW / 4;
        const int q = warp & 3, rg = warp >> 2, per = K >> 3;
        const int R = int(plan.ring / (size_t(K) * 2));
        float* abq = reinterpret_cast<float*>(part);  // [4][kStreamMaxRows]; the partials are summed already
        uint16_t* xs = reinterpret_cast<uint16_t*>(ring);
        uint4 wv[4];
        if (rg < RG) gdn_ab_load_w(A.ab_w, K, ab_col, q, lane, wv);
        for (int r0 = 0; r0 < M; r0 += R) {
            const int rb = M - r0 < R ? M - r0 : R;
            const uint4* src = reinterpret_cast<const uint4*>(A.xn_out + size_t(r0) * K);
            for (int base = threadIdx.x; base < rb * per; base += 16 * NT) {
                uint4 v[16];
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (base + j * NT < rb * per) v[j] = __ldcg(src + base + j * NT);
#pragma unroll
                for (int j = 0; j < 16; ++j)
                    if (base + j * NT < rb * per) reinterpret_cast<uint4*>(xs)[base + j * NT] = v[j];
            }
            consumer_sync<CW>();
            if (rg < RG) gdn_ab_quarter(xs, wv, K, rb, q, lane, abq + q * kStreamMaxRows + r0, rg, RG);
            consumer_sync<CW>();
        }
        if (int(threadIdx.x) < M)
            A.ab_out[size_t(threadIdx.x) * A.ab_stride + ab_col] = gdn_ab_combine(abq, kStreamMaxRows, threadIdx.x);
        trace_stamp(6);
    }
    grid_exit_named<kConsumerBar, NT>(A.bar);
}

size_t rowlin_workspace_bytes(int K) { return (size_t(kStreamMaxRows) * K + 255) / 256 * 256 + 3 * 256; }

template <int MT, int CW, int PW>
static int launch_rowlin_t(const Program& P, const RowLinArgs& A, const MlpShape& Z, size_t smem, cudaStream_t stream) {
    auto kern = rowlin_kernel<MT, CW, PW>;
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
    if (per_sm < 1) return fail(MONO_EINVAL, "rowlin: one CTA does not fit an SM (%zu B shared)", smem);
    const int tiles = phase_tiles(P.ph[0]);
    const int grid = tiles < sm_count() ? tiles : sm_count();
    if (A.ab_out && A.ab_n > grid) return fail(MONO_EINVAL, "rowlin: %d a|b columns on %d CTAs", A.ab_n, grid);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(grid);
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

template <int MT>
static int dispatch_rowlin(int c, const Program& P, const RowLinArgs& A, const MlpShape& Z, size_t smem,
                           cudaStream_t stream) {
    switch (c) {
        case 0: return launch_rowlin_t<MT, 10, 2>(P, A, Z, smem, stream);
        case 2: return launch_rowlin_t<MT, 12, 4>(P, A, Z, smem, stream);
        default: return launch_rowlin_t<MT, 8, 4>(P, A, Z, smem, stream);  // configs 1 and 3
    }
}

int launch_rowlin(Program& P, RowLinArgs& A, cudaStream_t stream) {
    const int M = P.M, G = sm_count();
    const int MT = M > 16 ? 4 : (M > 8 ? 2 : 1);
    const int nt = phase_tiles(P.ph[0]), grid = nt < G ? nt : G, per_cta = (nt + grid - 1) / grid;
    const size_t tile_bytes = size_t(phase_chunks(P.ph[0])) * MT * 128 * 4;
    // pass 0: every tile's partials at once; pass 1 (many rows): tiles in batches
    for (int pass = 0; pass < 2; ++pass)
        for (int staged = 1; staged >= 0; --staged) {
            P.ph[0].xsmem = staged;
            const size_t xb = staged ? size_t(M) * (P.ph[0].K + 16) : 0;
            for (int c = 0; c < kStreamConfigs; ++c) {
                const StreamConfig sc = kStreamConfig[c];
                int tb = per_cta;
                if (pass == 1) {
                    const StreamPlan bare(stage_bytes<FMT_GPTQ>(), sc.S, 0, xb, 0);
                    if (bare.total >= kStreamSmemLimit) continue;
                    tb = std::min<int>(tb, int((kStreamSmemLimit - bare.total) / 128 * 128 / tile_bytes));
                    if (tb < 1) continue;
                }
                const size_t part = size_t(tb) * tile_bytes;
                const StreamPlan plan(stage_bytes<FMT_GPTQ>(), sc.S, part, xb, 0);
                if (plan.total > kStreamSmemLimit) continue;
                const MlpShape Z{sc.S, int(part), int(xb), tb, 0};
                if (MT == 1) return dispatch_rowlin<1>(c, P, A, Z, plan.total, stream);
                if (MT == 2) return dispatch_rowlin<2>(c, P, A, Z, plan.total, stream);
                return dispatch_rowlin<4>(c, P, A, Z, plan.total, stream);
            }
        }
    return fail(MONO_EINVAL, "rowlin: no shared-memory plan fits (M=%d K=%d)", M, P.ph[0].K);
}

}  // namespace mono
