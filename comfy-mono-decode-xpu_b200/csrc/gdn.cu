// Gated-DeltaNet decode step (the core of the reference's layer_gdn P3-P5, csrc/mono_gdn.sycl:313-611).
//
// Two forms. Committing (ctl == null): M sequential rows, each advancing the recurrent and conv state, which
// are written back. Deferred (ctl != null; the reference's replay + verify, :385-567): the n = ctl[0] rows
// accepted at the previous step (slots ctl[2 + i], inputs saved by that step) are replayed first and their
// states persisted; then this step's verify tree runs on a register copy (outputs only, nothing persisted): each
// verify row's conv reads its ancestors (parents ctl[10 + t]), and the program ctl[18 + e] (slot | 32 * commit)
// orders the rows so that every row sees the state after its parent (committing entries advance the copy,
// the others use temporaries). The verify inputs are saved for the next step's replay. The conv state advances
// by the replayed rows only.
//
// Kernel 1 (one thread per qkv channel): the depthwise causal conv of width 4, y = bf16(fma chain x[t] w[3],
// x[t-1] w[2], .. from 0), out = bf16(y / (1 + exp(-y))), over the conv state (3 newest inputs, oldest
// first) and the replayed then the verify rows. Threads < (n + M) * HV make the gates:
// decay = exp(g_decay * softplus(a + dt_bias)) (softplus(v) = v above 20), beta = bf16(sigmoid(b)).
// Kernel 2 (per value head 8 row groups x 128 value columns, spread over a cluster of 4 CTAs below; thread
// (rg, col) keeps state rows rg * 16 .. rg * 16 + 15 of column col in registers): L2 norms of q and k of the key head
// (qi = 1 / max(sqrt(sum), 1e-12), q <- (q * scale) * qi, k <- k * ki), then per row in order
//   S <- S * decay;  mem = S^T k;  delta = (v - mem) * beta;  S <- S + k delta^T;  o = S^T q
// (fma chains over each row group's 16 rows, the 8 group partials summed in order), raw = bf16(o); the
// gated RMSNorm core = bf16(bf16(raw * w * rsqrt(mean(raw^2) + eps)) * bf16(silu(z))). fp32 throughout;
// results are checked against an fp64 reference with a stated tolerance.
#include <cmath>
#include <mutex>
#include <utility>

#include <cooperative_groups.h>

#include "gdn.cuh"

namespace mono {

namespace cg = cooperative_groups;

constexpr int kConvThreads = 64;  // 128 CTAs over the 8192 channels of the 9B model: one per SM, not 32

// Stream b's view of a batched call's operands (the layout of GdnArgs::streams).
__device__ __forceinline__ GdnArgs gdn_stream(const GdnArgs& A0, int b) {
    GdnArgs A = A0;
    const size_t rows = size_t(b) * A.M, wrows = size_t(b) * (A.M + kGdnMaxRows);
    A.qkv += rows * A.qkv_stride;
    A.z += rows * A.z_stride;
    A.a += rows * A.ab_stride;
    A.b += rows * A.ab_stride;
    A.core += rows * A.HV * kDH;
    A.conv_state += size_t(b) * A.C * 3;
    A.state += size_t(b) * A.HV * kDH * kDH;
    A.conv_out += wrows * A.C;
    A.gates += wrows * A.HV * 2;
    // (null pointers stay null: the offsets are zero for stream 0, and batched calls are deferred ones)
    A.ctl += size_t(b) * A.ctl_stride;
    A.prev_qkv += size_t(b) * kGdnMaxRows * A.C;
    A.prev_a += size_t(b) * kGdnMaxRows * A.HV;
    A.prev_b += size_t(b) * kGdnMaxRows * A.HV;
    A.save_qkv += size_t(b) * kGdnMaxRows * A.C;
    A.save_a += size_t(b) * kGdnMaxRows * A.HV;
    A.save_b += size_t(b) * kGdnMaxRows * A.HV;
    return A;
}

__global__ void __launch_bounds__(kConvThreads) gdn_conv_kernel(const GdnArgs A0) {
    const GdnArgs A = gdn_stream(A0, blockIdx.y);
    gdn_conv_item<true>(A, blockIdx.x * blockDim.x + threadIdx.x);
}

// Kernel 2 runs as a cluster of 4 CTAs per value head (128 CTAs at 32 heads): CTA c of the cluster keeps value
// columns 32c .. 32c + 31, thread (row group = warp, lane) column 32c + lane, state rows rg * kRPG .. + kRPG - 1 -
// the partition and every sum order of a one-CTA head, so the bits are the same. The gated RMSNorm of a row needs
// all 128 columns: after a cluster barrier each CTA reads the others' raw rows from their shared memory.
constexpr int kDcCols = 32, kDcCtas = kDH / kDcCols;
static_assert(kRG == 8 && kDcCols == 32, "one warp per row group, one lane per column");

__global__ void __cluster_dims__(kDcCtas, 1, 1) __launch_bounds__(kRG * kDcCols) gdn_delta_kernel(const GdnArgs A0) {
    const GdnArgs A = gdn_stream(A0, blockIdx.y);
    __shared__ __align__(16) float qn[kGdnMaxAll][kDH];
    __shared__ __align__(16) float kn[kGdnMaxAll][kDH];
    __shared__ float part[2][kRG][kDcCols];           // the entries' S^T k partials, by entry parity
    __shared__ float opart[kGdnMaxAll][kRG][kDcCols];  // every entry's output partials (summed after the entries)
    __shared__ int eout[kGdnMaxAll];
    __shared__ float raw[kGdnMaxRows][kDcCols];
    __shared__ float sums[2 * kGdnMaxAll];
    __shared__ float nsum[kGdnMaxRows];
    __shared__ float vsm[kGdnMaxAll][kDcCols];  // v of the CTA's columns, every row
    __shared__ float gsm[kGdnMaxAll][2];        // decay, beta of every row
    __shared__ int cs[kGdnCtlWords];
    trace_stamp_2d(0);
    gdn_ctl_stage(A, cs);
    __syncthreads();
    cg::cluster_group cluster = cg::this_cluster();
    const int cr = int(cluster.block_rank());
    const int h = int(blockIdx.x) / kDcCtas, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int rg = warp, col = cr * kDcCols + lane;
    const int kh = h / (A.HV / A.HK), KD = A.HK * kDH, M = A.M;
    const int n = gdn_pending_s(A, cs), R = n + M;
    // The recurrent state (written by this kernel's previous launch for the layer) before the dependency wait;
    // then the rows' q, k (key head kh, element tid) and v (this CTA's 32 columns) with every load issued before
    // the first store: one L2 round trip, not one per row.
    float st[kRPG];
    float* S = A.state + (size_t(h) * kDH + rg * kRPG) * kDH + col;
#pragma unroll
    for (int r = 0; r < kRPG; ++r) st[r] = S[size_t(r) * kDH];
    pdl_wait();
    pdl_launch_dependents();
    trace_stamp_2d(1);
    // the gated norm's z and weight for this thread's output elements e = tid + 128 j (rows t = e / 32), loaded
    // now: their latency hides behind the recurrence
    constexpr int kZPer = kGdnMaxRows * kDcCols / (kRG * kDcCols);
    float zv[kZPer], gw[kZPer];
#pragma unroll
    for (int j = 0; j < kZPer; ++j) {
        const int e = tid + j * kRG * kDcCols;
        zv[j] = gw[j] = 0.f;
        if (e < M * kDcCols) {
            const int t = e / kDcCols, d = cr * kDcCols + e % kDcCols;
            zv[j] = bf16_bits_to_f32(__ldcg(A.z + size_t(t) * A.z_stride + h * kDH + d));
            gw[j] = bf16_bits_to_f32(A.gnorm_w[d]);
        }
    }
    static_assert(kRG * kDcCols == 2 * kDH, "one thread per q or k element");
    const int qe = tid & (kDH - 1);
    const bool isk = tid >= kDH;  // threads [0, 128): q element qe of every row; [128, 256): k element qe
    float qk[kGdnMaxAll], vr[kGdnMaxAll / kRG];
#pragma unroll
    for (int t = 0; t < kGdnMaxAll; ++t)
        if (t < R) qk[t] = bf16_bits_to_f32(__ldcg(A.conv_out + size_t(t) * A.C + (isk ? KD : 0) + kh * kDH + qe));
#pragma unroll
    for (int j = 0; j < kGdnMaxAll / kRG; ++j) {
        const int t = warp + kRG * j;  // v rows of this warp: warp, warp + kRG, ...
        if (t < R) vr[j] = bf16_bits_to_f32(__ldcg(A.conv_out + size_t(t) * A.C + 2 * KD + h * kDH + cr * kDcCols + lane));
    }
    const float g0 = tid < 2 * R ? __ldcg(A.gates + ((tid >> 1) * A.HV + h) * 2 + (tid & 1)) : 0.f;
#pragma unroll
    for (int t = 0; t < kGdnMaxAll; ++t)
        if (t < R) (isk ? kn : qn)[t][qe] = qk[t];
#pragma unroll
    for (int j = 0; j < kGdnMaxAll / kRG; ++j)
        if (warp + kRG * j < R) vsm[warp + kRG * j][lane] = vr[j];
    if (tid < 2 * R) gsm[tid >> 1][tid & 1] = g0;
    __syncthreads();
    trace_stamp_2d(2);
    // sums of squares of q and k per row in gdn_sumsq128's order (lane l: elements l, l + 32, l + 64, l + 96, then
    // the xor butterfly), (row, q or k) pairs over the warps, read back from shared memory
    for (int pr = warp; pr < 2 * R; pr += kRG) {
        const float* src = (pr & 1) ? &kn[pr >> 1][0] : &qn[pr >> 1][0];
        float sq = 0.f;
#pragma unroll
        for (int j = 0; j < 4; ++j) sq = fmaf(src[lane + 32 * j], src[lane + 32 * j], sq);
#pragma unroll
        for (int o = 16; o; o >>= 1) sq += __shfl_xor_sync(0xffffffffu, sq, o);
        if (lane == 0) sums[pr] = gdn_l2_inv(sq);  // the row's inverse norm, once (not once per thread)
    }
    __syncthreads();
#pragma unroll
    for (int t = 0; t < kGdnMaxAll; ++t)
        if (t < R) {
            if (isk)
                kn[t][qe] = qk[t] * sums[2 * t + 1];
            else
                qn[t][qe] = (qk[t] * A.qscale) * sums[2 * t];
        }
    for (int e = tid; e < M * kDcCols; e += blockDim.x) raw[e / kDcCols][e % kDcCols] = 0.f;  // rows no entry names
    __syncthreads();
    trace_stamp_2d(3);
    // the entries: the replayed rows (committing), then the verify program (gdn_entry)
    const int E = n + gdn_verify_entries_s(A, cs);
    for (int e = 0; e < E; ++e) {
        const GdnEntry en = gdn_entry_s(A, cs, n, e);
        const int t = en.row;
        const float decay = gsm[t][0], beta = gsm[t][1];
        const float v = vsm[t][lane];
        // the row group's kRPG k and q values as 16-byte shared loads (a warp's lanes share the row group: broadcast)
        float kr[kRPG], qr[kRPG];
#pragma unroll
        for (int r4 = 0; r4 < kRPG / 4; ++r4) {
            const float4 k4 = reinterpret_cast<const float4*>(&kn[t][rg * kRPG])[r4];
            const float4 q4 = reinterpret_cast<const float4*>(&qn[t][rg * kRPG])[r4];
            kr[4 * r4] = k4.x, kr[4 * r4 + 1] = k4.y, kr[4 * r4 + 2] = k4.z, kr[4 * r4 + 3] = k4.w;
            qr[4 * r4] = q4.x, qr[4 * r4 + 1] = q4.y, qr[4 * r4 + 2] = q4.z, qr[4 * r4 + 3] = q4.w;
        }
        // a committing entry advances the state; another computes its row from temporaries (the same operations)
        float mem = 0.f;
        if (en.commit) {
#pragma unroll
            for (int r = 0; r < kRPG; ++r) {
                st[r] *= decay;
                mem = fmaf(st[r], kr[r], mem);
            }
        } else {
#pragma unroll
            for (int r = 0; r < kRPG; ++r) mem = fmaf(st[r] * decay, kr[r], mem);
        }
        float (&pe)[kRG][kDcCols] = part[e & 1];  // the other buffer is still being read by the previous entry
        pe[rg][lane] = mem;
        __syncthreads();
        float kv = pe[0][lane];  // the group partials in group order
#pragma unroll
        for (int j = 1; j < kRG; ++j) kv += pe[j][lane];
        const float delta = (v - kv) * beta;
        float o = 0.f;
        if (en.commit) {
#pragma unroll
            for (int r = 0; r < kRPG; ++r) {
                st[r] = fmaf(kr[r], delta, st[r]);
                o = fmaf(st[r], qr[r], o);
            }
        } else {
#pragma unroll
            for (int r = 0; r < kRPG; ++r) o = fmaf(fmaf(kr[r], delta, st[r] * decay), qr[r], o);
        }
        opart[e][rg][lane] = o;
        if (tid == 0) eout[e] = en.out;
        if (A.ctl != nullptr && e == n - 1)  // the committed state after the replay
#pragma unroll
            for (int r = 0; r < kRPG; ++r) S[size_t(r) * kDH] = st[r];
    }
    if (A.ctl == nullptr)
#pragma unroll
        for (int r = 0; r < kRPG; ++r) S[size_t(r) * kDH] = st[r];
    __syncthreads();  // every entry's output partials are written
    trace_stamp_2d(4);
    if (rg == 0)  // the entries' outputs in entry order (a later entry naming the same row wins, as it did in turn)
        for (int e = 0; e < E; ++e)
            if (eout[e] >= 0) {
                float o = opart[e][0][lane];
#pragma unroll
                for (int j = 1; j < kRG; ++j) o += opart[e][j][lane];
                raw[eout[e]][lane] = bf16_round(o);
            }
    cluster.sync();  // every CTA's raw rows are written (a cluster barrier orders its shared-memory writes)
    trace_stamp_2d(5);
    // gated RMSNorm of every output row: row t's squares in gdn_sumsq128's order (lane l: columns l, l + 32, l + 64,
    // l + 96 in order, i.e. CTA 0 .. 3's column l, then the xor butterfly)
    for (int t = warp; t < M; t += kRG) {
        float s = 0.f;
#pragma unroll
        for (int j = 0; j < kDcCtas; ++j) {
            const float* rj = cluster.map_shared_rank(&raw[0][0], j);
            const float v = rj[t * kDcCols + lane];
            s = fmaf(v, v, s);
        }
#pragma unroll
        for (int o = 16; o; o >>= 1) s += __shfl_xor_sync(0xffffffffu, s, o);
        if (lane == 0) nsum[t] = gdn_norm_inv(s, A.gnorm_eps);  // the row's norm factor, once
    }
    // this CTA's reads of the others' raw rows are done: arrive now, wait only before leaving (no CTA may leave
    // while another still reads its raw rows), so the stores below need not wait for the slowest reader
    auto done_reading = cluster.barrier_arrive();
    __syncthreads();  // nsum is visible to the CTA
    trace_stamp_2d(6);
    for (int j = 0; j < kZPer; ++j) {
        const int e = tid + j * kRG * kDcCols;
        if (e < M * kDcCols) {
            const int t = e / kDcCols, c = e % kDcCols, d = cr * kDcCols + c;
            A.core[size_t(t) * A.HV * kDH + h * kDH + d] = gdn_core(raw[t][c], gw[j], nsum[t], zv[j]);
        }
    }
    trace_stamp_2d(7);
    cluster.barrier_wait(std::move(done_reading));
}

// a | b projection: CTA (x, y) copies rows [16 y, 16 y + 16) of the M rows into shared memory; its 8 warps take
// the 4 quarters of columns 2x, 2x + 1. Launched with a programmatic dependency: the weights load before
// griddepcontrol.wait, the rows after it.
constexpr int kAbRows = 16;
__global__ void __launch_bounds__(256) gdn_ab_kernel(const uint16_t* x, int64_t x_stride, const uint16_t* w, int K,
                                                      int M, int N, uint16_t* out, int64_t out_stride) {
    extern __shared__ __align__(16) uint16_t xs[];
    {  // this CTA's block of rows
        const int r0 = int(blockIdx.y) * kAbRows;
        x += size_t(r0) * x_stride;
        out += size_t(r0) * out_stride;
        M = M - r0 < kAbRows ? M - r0 : kAbRows;
    }
    __shared__ float qs[2][4][kAbRows];
    const int per = K >> 3, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cl = warp >> 2, q = warp & 3, n = blockIdx.x * 2 + cl;
    uint4 wv[4];
    if (n < N) gdn_ab_load_w(w, K, n, q, lane, wv);  // in flight while the rows are copied
    pdl_wait();
    pdl_launch_dependents();  // after the wait: a dependent's early loads never see this kernel's inputs change
    // the rows in batches of 16 pieces per thread, every load of a batch issued before its stores (one L2 round
    // trip per batch instead of one per piece)
    for (int base = 0; base < M * per; base += 16 * 256) {
        uint4 v[16];
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int i = base + j * 256 + int(threadIdx.x);
            if (i < M * per) {
                const int m = i / per, c = i - m * per;
                v[j] = __ldcg(reinterpret_cast<const uint4*>(x + size_t(m) * x_stride) + c);
            }
        }
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            const int i = base + j * 256 + int(threadIdx.x);
            if (i < M * per) {
                const int m = i / per, c = i - m * per;
                reinterpret_cast<uint4*>(xs + size_t(m) * K)[c] = v[j];
            }
        }
    }
    __syncthreads();
    if (n < N) gdn_ab_quarter(xs, wv, K, M, q, lane, &qs[cl][q][0]);
    __syncthreads();
    if (threadIdx.x < 2 * M) {
        const int c = threadIdx.x / M, m = threadIdx.x % M, nn = blockIdx.x * 2 + c;
        if (nn < N) out[size_t(m) * out_stride + nn] = gdn_ab_combine(&qs[c][0][0], kAbRows, m);
    }
}

int launch_gdn_ab(const uint16_t* x, int64_t x_stride, const uint16_t* w, int K, int M, int N, uint16_t* out,
                  int64_t out_stride, cudaStream_t stream) {
    const size_t smem = size_t(M < kAbRows ? M : kAbRows) * K * 2;
    static std::mutex mu;
    static size_t opt_in = 48 * 1024;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (smem > opt_in) {
            CUDA_TRY(cudaFuncSetAttribute(gdn_ab_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, int(smem)));
            opt_in = smem;
        }
    }
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((N + 1) / 2, (M + kAbRows - 1) / kAbRows);
    cfg.blockDim = dim3(256);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, gdn_ab_kernel, x, x_stride, w, K, M, N, out, out_stride));
    return MONO_OK;
}

size_t gdn_workspace_bytes(int M, int C, int HV, int streams) {
    // per stream: conv outputs and gates of up to 8 replayed rows + the M verify rows
    const size_t rows = (size_t(M) + kGdnMaxRows) * streams;
    return (rows * C * 2 + 255) / 256 * 256 + rows * HV * 2 * 4;
}

int launch_gdn_step(GdnArgs A, void* ws, cudaStream_t stream) {
    const size_t rows = size_t(A.M) + kGdnMaxRows;
    A.conv_out = static_cast<uint16_t*>(ws);
    A.gates = reinterpret_cast<float*>(static_cast<uint8_t*>(ws) + (rows * A.streams * A.C * 2 + 255) / 256 * 256);
    const int rmax = int(rows);
    const int nthreads = A.C > rmax * A.HV ? A.C : rmax * A.HV;
    // both with a programmatic dependency on their predecessor (griddepcontrol.wait inside, after the loads that
    // no recent kernel writes)
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3((nthreads + kConvThreads - 1) / kConvThreads, A.streams);
    cfg.blockDim = dim3(kConvThreads);
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    CUDA_TRY(cudaLaunchKernelEx(&cfg, gdn_conv_kernel, A));
    cfg.gridDim = dim3(A.HV * kDcCtas, A.streams);
    cfg.blockDim = dim3(kRG * kDcCols);
    CUDA_TRY(cudaLaunchKernelEx(&cfg, gdn_delta_kernel, A));
    CUDA_TRY(cudaGetLastError());
    return MONO_OK;
}

}  // namespace mono
