// extern "C" entry points: host-side validation, then the launchers.
#include <cstring>
#include <mutex>
#include <string>

#include "gdn.cuh"
#include "launch.h"

namespace mono {

namespace {
thread_local std::string g_last_error;
}

int fail(int code, const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof(buf), fmt, ap);
    va_end(ap);
    g_last_error = buf;
    return code;
}

int sm_count() {
    static int counts[64] = {};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    if (counts[dev] == 0) {
        int n = 0;
        if (cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess || n <= 0) n = 148;
        counts[dev] = n;
    }
    return counts[dev];
}

static int check_linear_common(const int8_t* x, const float* xs, const void* packed, const void* scales,
                               const void* out, int64_t M, int64_t N, int64_t K, int out_dtype_code, int layout) {
    MONO_CHECK(x && xs && packed && out && (scales || layout == MONO_LAYOUT_TILED), "null operand");
    MONO_CHECK(M >= 1 && M <= 16, "1 <= M <= 16 (got %lld)", (long long)M);
    MONO_CHECK(K >= kChunkK && K % kChunkK == 0 && K <= kChunkK * kMaxChunks, "K must be a multiple of 1024 in [1024, 16384] (got %lld)",
               (long long)K);
    MONO_CHECK(N >= 16 && N % 16 == 0 && N <= (1 << 24), "N must be a positive multiple of 16 (got %lld)", (long long)N);
    MONO_CHECK(out_dtype_code == MONO_OUT_F32 || out_dtype_code == MONO_OUT_BF16, "out dtype fp32 (0) or bf16 (2)");
    MONO_CHECK(layout == MONO_LAYOUT_ROW || layout == MONO_LAYOUT_TILED, "layout ROW (0) or TILED (1)");
    MONO_CHECK(aligned(x, 16), "x must be 16-byte aligned");
    MONO_CHECK(aligned(packed, 16), "packed weights must be 16-byte aligned");
    MONO_CHECK(layout == MONO_LAYOUT_TILED || aligned(scales, 16), "scales must be 16-byte aligned");
    return MONO_OK;
}

int fill_gdn_args(GdnArgs& A, const void* qkv, const void* z, const void* a, const void* b, const void* conv_w,
                         void* conv_state, const float* dt_bias, const float* g_decay, float* state, const void* gnorm_w,
                         float gnorm_eps, float qscale, int64_t M, int64_t HK, int64_t HV, void* core, void* workspace,
                         size_t workspace_bytes, const int32_t* ctl, const void* prev_qkv, const void* prev_a,
                         const void* prev_b, void* save_qkv, void* save_a, void* save_b, int64_t qkv_stride,
                         int64_t z_stride, int64_t ab_stride) {
    MONO_CHECK(qkv && z && a && b && conv_w && conv_state && dt_bias && g_decay && state && gnorm_w && core && workspace,
               "null operand");
    MONO_CHECK(M >= 1 && M <= 8, "1 <= M <= 8 rows (got %lld)", (long long)M);
    MONO_CHECK(HK >= 1 && HV >= HK && HV % HK == 0 && HV <= 1024, "value heads a multiple of key heads");
    MONO_CHECK(gnorm_eps > 0.f, "positive eps");
    const int64_t C = (2 * HK + HV) * 128;
    MONO_CHECK(workspace_bytes >= mono_gdn_step_workspace(M, C, HV), "workspace too small (mono_gdn_step_workspace)");
    MONO_CHECK(aligned(workspace, 256) && aligned(state, 16), "aligned workspace / state");
    A = GdnArgs{};
    A.qkv = static_cast<const uint16_t*>(qkv);
    A.z = static_cast<const uint16_t*>(z);
    A.a = static_cast<const uint16_t*>(a);
    A.b = static_cast<const uint16_t*>(b);
    A.conv_w = static_cast<const uint16_t*>(conv_w);
    A.conv_state = static_cast<uint16_t*>(conv_state);
    A.dt_bias = dt_bias;
    A.g_decay = g_decay;
    A.state = state;
    A.gnorm_w = static_cast<const uint16_t*>(gnorm_w);
    A.gnorm_eps = gnorm_eps;
    A.qscale = qscale;
    A.core = static_cast<uint16_t*>(core);
    MONO_CHECK(qkv_stride >= C && z_stride >= HV * 128 && ab_stride >= HV, "row strides cover the rows");
    A.qkv_stride = qkv_stride;
    A.z_stride = z_stride;
    A.ab_stride = ab_stride;
    A.ctl = ctl;
    A.prev_qkv = static_cast<const uint16_t*>(prev_qkv);
    A.prev_a = static_cast<const uint16_t*>(prev_a);
    A.prev_b = static_cast<const uint16_t*>(prev_b);
    A.save_qkv = static_cast<uint16_t*>(save_qkv);
    A.save_a = static_cast<uint16_t*>(save_a);
    A.save_b = static_cast<uint16_t*>(save_b);
    A.M = int(M);
    A.C = int(C);
    A.HK = int(HK);
    A.HV = int(HV);
    A.streams = 1;
    A.ctl_stride = 0;
    const size_t rows = size_t(M) + 8;
    A.conv_out = static_cast<uint16_t*>(workspace);
    A.gates = reinterpret_cast<float*>(static_cast<uint8_t*>(workspace) + (rows * C * 2 + 255) / 256 * 256);
    return MONO_OK;
}

}  // namespace mono

using namespace mono;

extern "C" {

const char* mono_last_error(void) { return g_last_error.c_str(); }

int mono_abi_version(void) { return 1; }

int mono_device_status(int* code, int reset) {
    int v = 0;
    CUDA_TRY(cudaMemcpyFromSymbol(&v, g_device_error, sizeof(int)));
    if (code) *code = v;
    if (reset && v) {
        const int zero = 0;
        CUDA_TRY(cudaMemcpyToSymbol(g_device_error, &zero, sizeof(int)));
    }
    return v ? fail(MONO_EDEVICE, "device error word = %d", v) : MONO_OK;
}

size_t mono_trace_bytes(void) { return size_t(kTraceCtas) * kTracePhases * 8; }

int mono_trace_enable(void* buffer, size_t bytes) {
    MONO_CHECK(buffer == nullptr || bytes >= size_t(kTraceCtas) * kTracePhases * 8, "trace buffer too small");
    unsigned long long* p = static_cast<unsigned long long*>(buffer);
    CUDA_TRY(cudaMemcpyToSymbol(g_trace, &p, sizeof(p)));
    return MONO_OK;
}

int mono_w4a8_decode_linear(const int8_t* x, const float* x_scale, const void* packed, const void* s_rel,
                            int s_rel_dtype, const float* s_channel, const uint16_t* pair_table,
                            const void* residual, int64_t M, int64_t N, int64_t K, int64_t group_size,
                            int out_dtype_code, int layout, void* out, mono_stream_t stream) {
    int rc = check_linear_common(x, x_scale, packed, s_rel, out, M, N, K, out_dtype_code, layout);
    if (rc) return rc;
    MONO_CHECK(group_size == 16, "group_size must be 16 (G16 FP8 relative scales)");
    MONO_CHECK(s_rel_dtype == MONO_SCALE_FP8_E4M3, "s_rel must be FP8 e4m3");
    MONO_CHECK(s_channel && pair_table, "s_channel and pair_table are required");
    Program P{};
    P.nph = 1;
    P.M = int(M);
    P.pair_tab = pair_table;
    P.ph[0].m[0] = MatDesc{static_cast<const uint8_t*>(packed), static_cast<const uint8_t*>(s_rel), int(N)};
    P.ph[0].nm = 1;
    P.ph[0].K = int(K);
    P.ph[0].x = x;
    LinearEpi E{nullptr, x_scale, s_channel, residual, out, out_dtype_code == MONO_OUT_BF16, 0};
    return launch_linear(FMT_REF, layout, P, E, reinterpret_cast<cudaStream_t>(stream));
}

int mono_w4_pair_table(const float* codebook, uint16_t* table, mono_stream_t stream) {
    MONO_CHECK(table, "null table");
    return launch_pair_table(codebook, table, reinterpret_cast<cudaStream_t>(stream));
}

int mono_w4a8_gptq_linear(const int8_t* x, const float* x_scale, const void* packed, const void* scales,
                          const void* residual, int64_t M, int64_t N, int64_t K, int out_dtype_code, int layout,
                          void* out, mono_stream_t stream) {
    int rc = check_linear_common(x, x_scale, packed, scales, out, M, N, K, out_dtype_code, layout);
    if (rc) return rc;
    Program P{};
    P.nph = 1;
    P.M = int(M);
    P.ph[0].m[0] = MatDesc{static_cast<const uint8_t*>(packed), static_cast<const uint8_t*>(scales), int(N)};
    P.ph[0].nm = 1;
    P.ph[0].K = int(K);
    P.ph[0].x = x;
    LinearEpi E{nullptr, x_scale, nullptr, residual, out, out_dtype_code == MONO_OUT_BF16, 0};
    return launch_linear(FMT_GPTQ, layout, P, E, reinterpret_cast<cudaStream_t>(stream));
}

int mono_w4a8_gptq_linear_bf16(const void* x, const void* packed, const void* scales, const void* residual, int64_t M,
                               int64_t N, int64_t K, int out_dtype_code, int layout, void* out, mono_stream_t stream) {
    // the int8 checks with x standing in for both activation operands (x_scale is produced in the kernel)
    int rc = check_linear_common(static_cast<const int8_t*>(x), static_cast<const float*>(x), packed, scales, out, M, N,
                                 K, out_dtype_code, layout);
    if (rc) return rc;
    Program P{};
    P.nph = 1;
    P.M = int(M);
    P.ph[0].m[0] = MatDesc{static_cast<const uint8_t*>(packed), static_cast<const uint8_t*>(scales), int(N)};
    P.ph[0].nm = 1;
    P.ph[0].K = int(K);
    P.ph[0].x = nullptr;
    P.ph[0].xperm = 1;
    LinearEpi E{static_cast<const uint16_t*>(x), nullptr, nullptr, residual, out, out_dtype_code == MONO_OUT_BF16, 0};
    return launch_linear(FMT_GPTQ, layout, P, E, reinterpret_cast<cudaStream_t>(stream));
}

size_t mono_w4_tiled_bytes(int fmt, int64_t N, int64_t K) { return tiled_bytes(fmt, N, K); }

int mono_w4_repack(int fmt, const void* packed, const void* scales, int64_t N, int64_t K, void* tiled,
                   mono_stream_t stream) {
    MONO_CHECK(fmt == MONO_FMT_GPTQ || fmt == MONO_FMT_REF, "fmt GPTQ (0) or REF (1)");
    MONO_CHECK(packed && scales && tiled, "null operand");
    MONO_CHECK(N >= 16 && N % 16 == 0 && K >= kChunkK && K % kChunkK == 0, "N % 16 == 0 and K % 1024 == 0");
    MONO_CHECK(aligned(packed, 16) && aligned(scales, 16) && aligned(tiled, 16), "operands must be 16-byte aligned");
    return launch_repack(fmt, packed, scales, int(N), int(K), tiled, reinterpret_cast<cudaStream_t>(stream));
}

int mono_act_quant(const void* x_bf16, int64_t M, int64_t K, int8_t* q, float* scale, mono_stream_t stream) {
    MONO_CHECK(x_bf16 && q && scale, "null operand");
    MONO_CHECK(M >= 1 && M <= 65535 && K >= 8 && K % 8 == 0, "M in [1, 65535], K % 8 == 0");
    MONO_CHECK(aligned(x_bf16, 16) && aligned(q, 8), "x must be 16-byte and q 8-byte aligned");
    return launch_act_quant(x_bf16, int(M), int(K), q, scale, reinterpret_cast<cudaStream_t>(stream));
}

size_t mono_rot_quant_workspace(int64_t M, int64_t K) { return rot_quant_workspace(int(M), int(K)); }

int mono_rot_quant(const void* x_bf16, const void* h_bf16, int64_t M, int64_t K, int8_t* q, float* scale,
                   void* workspace, mono_stream_t stream) {
    MONO_CHECK(x_bf16 && h_bf16 && q && scale && workspace, "null operand");
    MONO_CHECK(M >= 1 && M <= 65535 && K >= 256 && K % 256 == 0, "M in [1, 65535], K % 256 == 0");
    MONO_CHECK(aligned(workspace, 16), "workspace must be 16-byte aligned");
    return launch_rot_quant(x_bf16, h_bf16, int(M), int(K), q, scale, workspace, reinterpret_cast<cudaStream_t>(stream));
}

int mono_rot_quant_noalloc(const void* x_bf16, const void* h_bf16, int64_t M, int64_t K, int8_t* q, float* scale,
                           mono_stream_t stream) {
    MONO_CHECK(x_bf16 && h_bf16 && q && scale, "null operand");
    MONO_CHECK(M >= 1 && M <= 65535 && K >= 256 && K <= (1 << 20), "M in [1, 65535], K in [256, 2^20]");
    return launch_rot_quant_noalloc(x_bf16, h_bf16, int(M), int(K), q, scale, reinterpret_cast<cudaStream_t>(stream));
}

size_t mono_mlp_gptq_workspace(int64_t H, int64_t I) { return mlp_workspace_bytes(int(H), int(I)); }

int mono_mlp_gptq(const void* x, const void* norm_w, float eps, const void* gate_q, const void* up_q,
                  const void* down_q, const void* silu_lut,
                  int64_t M, int64_t H, int64_t I, int residual, void* out, void* workspace, size_t workspace_bytes,
                  mono_stream_t stream) {
    MONO_CHECK(x && gate_q && up_q && down_q && silu_lut && out && workspace, "null operand");
    MONO_CHECK(M >= 1 && M <= kStreamMaxRows, "1 <= M <= %d (got %lld)", kStreamMaxRows, (long long)M);
    MONO_CHECK(H >= kChunkK && H % kChunkK == 0 && H <= 4096, "H must be a multiple of 1024 up to 4096");
    MONO_CHECK(I >= kChunkK && I % kChunkK == 0 && I <= kChunkK * kMaxChunks, "I must be a multiple of 1024 up to 16384");
    MONO_CHECK(workspace_bytes >= mlp_workspace_bytes(int(H), int(I)), "workspace too small (%zu < %zu)", workspace_bytes,
               mlp_workspace_bytes(int(H), int(I)));
    MONO_CHECK(aligned(x, 16) && aligned(out, 16) && aligned(workspace, 256), "x/out 16-byte, workspace 256-byte aligned");
    for (const void* p : {gate_q, up_q, down_q}) MONO_CHECK(aligned(p, 16), "weights 16-byte aligned");
    auto al = [](size_t b) { return (b + 255) / 256 * 256; };
    uint8_t* w = static_cast<uint8_t*>(workspace);
    MlpArgs A{};
    A.x = static_cast<const uint16_t*>(x);
    A.norm_w = static_cast<const uint16_t*>(norm_w);
    A.lut = static_cast<const uint16_t*>(silu_lut);
    A.out = static_cast<uint16_t*>(out);
    A.eps = eps;
    A.H = int(H);
    A.I = int(I);
    A.residual = residual != 0;
    const size_t R = kStreamMaxRows;
    A.q1 = reinterpret_cast<int8_t*>(w);
    w += al(R * size_t(H));
    A.h = reinterpret_cast<uint16_t*>(w);
    w += al(R * size_t(I) * 2);
    A.q2 = reinterpret_cast<int8_t*>(w);
    w += al(R * size_t(I));
    A.s1 = reinterpret_cast<float*>(w + 256);
    A.amax2 = reinterpret_cast<unsigned*>(w + 512);
    A.bar = reinterpret_cast<unsigned*>(w + 768);
    Program P{};
    P.nph = 2;
    P.M = int(M);
    P.ph[0].m[0] = MatDesc{static_cast<const uint8_t*>(gate_q), nullptr, int(I)};
    P.ph[0].m[1] = MatDesc{static_cast<const uint8_t*>(up_q), nullptr, int(I)};
    P.ph[0].nm = 2;
    P.ph[0].paired = 1;
    P.ph[0].K = int(H);
    P.ph[0].x = nullptr;  // (staged by the kernel itself)
    P.ph[0].xperm = 1;
    P.ph[1].m[0] = MatDesc{static_cast<const uint8_t*>(down_q), nullptr, int(H)};
    P.ph[1].nm = 1;
    P.ph[1].K = int(I);
    P.ph[1].x = A.q2;
    P.ph[1].xperm = 1;
    return launch_mlp(P, A, reinterpret_cast<cudaStream_t>(stream));
}


int mono_qk_norm_rope_kv(const void* rawq, int64_t q_row_stride, int64_t q_head_stride, const void* rawk,
                         int64_t k_row_stride, const void* v, int64_t v_row_stride, const void* wq, const void* wk,
                         const float* freqs, void* key_cache, void* value_cache, int64_t cap, const int64_t* position,
                         int64_t S, int64_t Hq, int64_t Hk, float epsq, float epsk, int64_t rd, void* out_q,
                         void* out_k, mono_stream_t stream) {
    return mono_qk_norm_rope_kv_streams(rawq, q_row_stride, q_head_stride, rawk, k_row_stride, v, v_row_stride, wq, wk,
                                        freqs, key_cache, value_cache, cap, position, S, 1, Hq, Hk, epsq, epsk, rd,
                                        out_q, out_k, stream);
}

int mono_qk_norm_rope_kv_streams(const void* rawq, int64_t q_row_stride, int64_t q_head_stride, const void* rawk,
                                 int64_t k_row_stride, const void* v, int64_t v_row_stride, const void* wq,
                                 const void* wk, const float* freqs, void* key_cache, void* value_cache, int64_t cap,
                                 const int64_t* position, int64_t S, int64_t streams, int64_t Hq, int64_t Hk,
                                 float epsq, float epsk, int64_t rd, void* out_q, void* out_k, mono_stream_t stream) {
    MONO_CHECK(rawq && rawk && v && wq && wk && freqs && key_cache && value_cache && position && out_q && out_k,
               "null operand");
    MONO_CHECK(streams >= 1 && streams <= 8 && S % streams == 0 && S / streams >= 1 && S / streams <= 8,
               "1 <= streams <= 8 of 1 <= S / streams <= 8 decode rows each (S = %lld)", (long long)S);
    MONO_CHECK(Hq >= 1 && Hk >= 1 && Hq <= 1024 && Hk <= 1024, "head counts");
    MONO_CHECK(rd >= 2 && rd <= 256 && rd % 2 == 0, "even rotary dimension in [2, 256] (got %lld)", (long long)rd);
    MONO_CHECK(cap >= 1 && epsq > 0.f && epsk > 0.f, "positive capacity and eps");
    MONO_CHECK(q_head_stride >= 256 && q_row_stride >= Hq * q_head_stride && k_row_stride >= Hk * 256 &&
                   v_row_stride >= Hk * 256 && q_head_stride % 8 == 0 && q_row_stride % 8 == 0 &&
                   k_row_stride % 8 == 0 && v_row_stride % 8 == 0,
               "strides (elements): q head >= 256, rows cover their heads, multiples of 8");
    const void* ptrs[] = {rawq, rawk, v, wq, wk, key_cache, value_cache, out_q, out_k};
    for (const void* ptr : ptrs) MONO_CHECK(aligned(ptr, 16), "16-byte aligned operands");
    MONO_CHECK(aligned(freqs, 4) && aligned(position, 8), "aligned freqs / positions");
    NormRopeArgs A{};
    A.q = static_cast<const uint16_t*>(rawq);
    A.k = static_cast<const uint16_t*>(rawk);
    A.v = static_cast<const uint16_t*>(v);
    A.wq = static_cast<const uint16_t*>(wq);
    A.wk = static_cast<const uint16_t*>(wk);
    A.freqs = freqs;
    A.kc = static_cast<uint16_t*>(key_cache);
    A.vc = static_cast<uint16_t*>(value_cache);
    A.pos = position;
    A.oq = static_cast<uint16_t*>(out_q);
    A.ok = static_cast<uint16_t*>(out_k);
    A.qs = q_row_stride;
    A.qh = q_head_stride;
    A.ks = k_row_stride;
    A.vs = v_row_stride;
    A.cap = cap;
    A.S = int(S);
    A.Hq = int(Hq);
    A.Hk = int(Hk);
    A.rd = int(rd);
    A.epsq = epsq;
    A.epsk = epsk;
    A.streams = int(streams);
    return launch_qk_norm_rope_kv(A, reinterpret_cast<cudaStream_t>(stream));
}

size_t mono_tree_attention_workspace(int64_t Hk, int64_t cap) { return mono_tree_attention_streams_workspace(Hk, 1, cap); }

size_t mono_tree_attention_streams_workspace(int64_t Hk, int64_t streams, int64_t cap) {
    if (Hk < 1 || cap < 1 || streams < 1 || streams > 8) return 0;
    return attn_workspace_bytes(int(Hk * streams), int(streams), int(cap), sm_count());
}

int mono_tree_attention(const void* q, const void* key_cache, const void* value_cache, const int32_t* seqlen,
                        const void* xk, const void* xv, const int32_t* mask, int64_t H, int64_t Hk, int64_t S,
                        int64_t cap, void* out, void* workspace, size_t workspace_bytes, mono_stream_t stream) {
    return mono_tree_attention_streams(q, key_cache, value_cache, seqlen, xk, xv, mask, H, Hk, S, 1, cap, Hk * S * 256,
                                       S * 256, 256, out, workspace, workspace_bytes, stream);
}

int mono_tree_attention_streams(const void* q, const void* key_cache, const void* value_cache, const int32_t* seqlen,
                                const void* xk, const void* xv, const int32_t* mask, int64_t H, int64_t Hk, int64_t S,
                                int64_t streams, int64_t cap, int64_t xv_stream_stride, int64_t xv_head_stride,
                                int64_t xv_row_stride, void* out, void* workspace, size_t workspace_bytes,
                                mono_stream_t stream) {
    MONO_CHECK(q && key_cache && value_cache && seqlen && out && workspace, "null operand");
    MONO_CHECK(streams >= 1 && streams <= 8, "1 <= streams <= 8");
    MONO_CHECK(xv_stream_stride >= 0 && xv_head_stride >= 0 && xv_row_stride >= 0 && xv_stream_stride % 8 == 0 &&
                   xv_head_stride % 8 == 0 && xv_row_stride % 8 == 0,
               "tree value strides: non-negative multiples of 8 elements");
    MONO_CHECK(S >= 1 && S <= 8 && Hk >= 1 && H % Hk == 0 && (H / Hk) * S <= 32,
               "1..8 rows, H a multiple of Hk, (H / Hk) * S <= 32 query rows per kv head");
    MONO_CHECK(mask != nullptr || S == 1, "a tree mask for S > 1 rows (S = 1 without a mask: the draft row)");
    MONO_CHECK(mask == nullptr || (xk && xv && aligned(xk, 16) && aligned(xv, 16)), "tree rows need 16-byte aligned xk / xv");
    MONO_CHECK(cap >= 1 && cap <= (int64_t(1) << 30), "cache capacity");
    MONO_CHECK(workspace_bytes >= mono_tree_attention_streams_workspace(Hk, streams, cap),
               "workspace too small (mono_tree_attention_streams_workspace)");
    const void* ptrs[] = {q, key_cache, value_cache, out, workspace};
    for (const void* ptr : ptrs) MONO_CHECK(aligned(ptr, 16), "16-byte aligned operands");
    AttnArgs A{};
    A.q = static_cast<const uint16_t*>(q);
    A.kc = static_cast<const uint16_t*>(key_cache);
    A.vc = static_cast<const uint16_t*>(value_cache);
    A.seqlen = seqlen;
    A.xk = static_cast<const uint16_t*>(xk);
    A.xv = static_cast<const uint16_t*>(xv);
    A.mask = mask;
    A.xv_bs = xv_stream_stride;
    A.xv_hs = xv_head_stride;
    A.xv_rs = xv_row_stride;
    A.out = static_cast<uint16_t*>(out);
    A.H = int(H * streams);
    A.Hk = int(Hk * streams);
    A.S = int(S);
    A.cap = int(cap);
    A.streams = int(streams);
    return launch_tree_attention(A, workspace, reinterpret_cast<cudaStream_t>(stream));
}

size_t mono_gdn_step_workspace(int64_t M, int64_t C, int64_t HV) {
    if (M < 1 || C < 1 || HV < 1) return 0;
    return gdn_workspace_bytes(int(M), int(C), int(HV), 1);
}

size_t mono_gdn_step_streams_workspace(int64_t M, int64_t C, int64_t HV, int64_t streams) {
    if (M < 1 || C < 1 || HV < 1 || streams < 1 || streams > 8) return 0;
    return gdn_workspace_bytes(int(M), int(C), int(HV), int(streams));
}

static int gdn_step_impl(const void* qkv, const void* z, const void* a, const void* b, const void* conv_w,
                         void* conv_state, const float* dt_bias, const float* g_decay, float* state, const void* gnorm_w,
                         float gnorm_eps, float qscale, int64_t M, int64_t HK, int64_t HV, void* core, void* workspace,
                         size_t workspace_bytes, const int32_t* ctl, const void* prev_qkv, const void* prev_a,
                         const void* prev_b, void* save_qkv, void* save_a, void* save_b, int64_t qkv_stride,
                         int64_t z_stride, int64_t ab_stride, mono_stream_t stream, int64_t streams = 1,
                         int64_t ctl_stride = 0) {
    MONO_CHECK(streams >= 1 && streams <= 8, "1 <= streams <= 8");
    MONO_CHECK(streams == 1 || ctl == nullptr || ctl_stride >= kGdnCtlWords, "ctl rows of %d words", kGdnCtlWords);
    MONO_CHECK(workspace_bytes >= mono_gdn_step_streams_workspace(M, (2 * HK + HV) * 128, HV, streams),
               "workspace too small (mono_gdn_step_streams_workspace)");
    GdnArgs A;
    const int rc = fill_gdn_args(A, qkv, z, a, b, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, gnorm_eps, qscale,
                                 M, HK, HV, core, workspace, workspace_bytes, ctl, prev_qkv, prev_a, prev_b, save_qkv,
                                 save_a, save_b, qkv_stride, z_stride, ab_stride);
    if (rc != MONO_OK) return rc;
    A.streams = int(streams);
    A.ctl_stride = int(ctl_stride);
    return launch_gdn_step(A, workspace, reinterpret_cast<cudaStream_t>(stream));
}

int mono_gdn_step(const void* qkv, const void* z, const void* a, const void* b, const void* conv_w, void* conv_state,
                  const float* dt_bias, const float* g_decay, float* state, const void* gnorm_w, float gnorm_eps,
                  float qscale, int64_t M, int64_t HK, int64_t HV, void* core, void* workspace, size_t workspace_bytes,
                  mono_stream_t stream) {
    return gdn_step_impl(qkv, z, a, b, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, gnorm_eps, qscale, M, HK,
                         HV, core, workspace, workspace_bytes, nullptr, nullptr, nullptr, nullptr, nullptr, nullptr,
                         nullptr, (2 * HK + HV) * 128, HV * 128, HV, stream);
}

int mono_gdn_step_deferred(const void* qkv, const void* z, const void* a, const void* b, const void* conv_w,
                           void* conv_state, const float* dt_bias, const float* g_decay, float* state,
                           const void* gnorm_w, float gnorm_eps, float qscale, int64_t M, int64_t HK, int64_t HV,
                           void* core, const int32_t* ctl, const void* prev_qkv, const void* prev_a, const void* prev_b,
                           void* save_qkv, void* save_a, void* save_b, int64_t qkv_stride, int64_t z_stride,
                           int64_t ab_stride, void* workspace, size_t workspace_bytes, mono_stream_t stream) {
    MONO_CHECK(ctl && prev_qkv && prev_a && prev_b && save_qkv && save_a && save_b, "deferred form: ctl, prev and save buffers");
    MONO_CHECK(prev_qkv != save_qkv && prev_a != save_a && prev_b != save_b, "save buffers must not alias the replayed ones");
    return gdn_step_impl(qkv, z, a, b, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, gnorm_eps, qscale, M, HK,
                         HV, core, workspace, workspace_bytes, ctl, prev_qkv, prev_a, prev_b, save_qkv, save_a, save_b,
                         qkv_stride, z_stride, ab_stride, stream);
}

int mono_gdn_step_deferred_streams(const void* qkv, const void* z, const void* a, const void* b, const void* conv_w,
                                   void* conv_state, const float* dt_bias, const float* g_decay, float* state,
                                   const void* gnorm_w, float gnorm_eps, float qscale, int64_t M, int64_t HK,
                                   int64_t HV, int64_t streams, void* core, const int32_t* ctl, int64_t ctl_stride,
                                   const void* prev_qkv, const void* prev_a, const void* prev_b, void* save_qkv,
                                   void* save_a, void* save_b, int64_t qkv_stride, int64_t z_stride, int64_t ab_stride,
                                   void* workspace, size_t workspace_bytes, mono_stream_t stream) {
    MONO_CHECK(ctl && prev_qkv && prev_a && prev_b && save_qkv && save_a && save_b, "deferred form: ctl, prev and save buffers");
    MONO_CHECK(prev_qkv != save_qkv && prev_a != save_a && prev_b != save_b, "save buffers must not alias the replayed ones");
    return gdn_step_impl(qkv, z, a, b, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, gnorm_eps, qscale, M, HK,
                         HV, core, workspace, workspace_bytes, ctl, prev_qkv, prev_a, prev_b, save_qkv, save_a, save_b,
                         qkv_stride, z_stride, ab_stride, stream, streams, ctl_stride);
}

size_t mono_topk_workspace(int64_t rows) { return rows < 1 ? 0 : topk_workspace_bytes(rows); }

int mono_fast_topk(const void* x, int64_t rows, int64_t V, int64_t k, int argmax_order, int with_argmax, void* values,
                   int64_t* indices, int64_t* argmax, void* workspace, size_t workspace_bytes, mono_stream_t stream) {
    MONO_CHECK(x && values && indices && workspace && (argmax || !with_argmax), "null operand");
    MONO_CHECK(rows >= 1 && rows <= 65535, "1 <= rows <= 65535");
    MONO_CHECK(k >= 1 && k <= 8 && V >= k && V < (int64_t(1) << 31), "1 <= k <= 8, k <= V < 2^31");
    MONO_CHECK(!argmax_order || k == 1, "argmax order ranks k = 1 only");
    MONO_CHECK(workspace_bytes >= mono_topk_workspace(rows) && aligned(workspace, 8), "workspace (mono_topk_workspace)");
    TopkArgs A{};
    A.x = static_cast<const uint16_t*>(x);
    A.values = static_cast<uint16_t*>(values);
    A.indices = indices;
    A.argmax = argmax;
    A.ws = static_cast<uint64_t*>(workspace);
    A.V = V;
    A.rows = int(rows);
    A.k = int(k);
    A.argmax_order = argmax_order != 0;
    A.with_argmax = with_argmax != 0;
    return launch_topk(A, reinterpret_cast<cudaStream_t>(stream));
}

size_t mono_rowlin_gptq_workspace(int64_t K) { return K < 1 ? 0 : rowlin_workspace_bytes(int(K)); }

static int rowlin_entry(const void* x, int mode, const void* norm_w, float eps, const void* gate, int64_t gate_row_stride,
                        int64_t gate_head_stride, const void* lut, const void* const* weights, const int64_t* rows, int nm,
                        int64_t M, int64_t K, const void* residual, void* out, void* xn_out, const void* ab_w,
                        int64_t ab_n, void* ab_out, int64_t ab_stride, void* workspace, size_t workspace_bytes,
                        mono_stream_t stream) {
    MONO_CHECK(x && weights && rows && out && workspace, "null operand");
    MONO_CHECK(mode == ROWLIN_NORM || mode == ROWLIN_GATE || mode == ROWLIN_QUANT, "mode 0 (norm), 1 (gate), 2 (quant)");
    MONO_CHECK(mode != ROWLIN_NORM || norm_w, "norm mode needs norm_w");
    MONO_CHECK(mode != ROWLIN_GATE || (gate && lut && gate_head_stride >= 256 && gate_head_stride % 8 == 0 &&
                                       gate_row_stride % 8 == 0 && aligned(gate, 16)),
               "gate mode: gate (16-byte aligned, strides multiples of 8 elements) and lut");
    MONO_CHECK(nm >= 1 && nm <= 3, "1 to 3 matrices");
    MONO_CHECK(M >= 1 && M <= kStreamMaxRows, "1 <= M <= %d (got %lld)", kStreamMaxRows, (long long)M);
    MONO_CHECK(K >= kChunkK && K % kChunkK == 0 && K <= 4096, "K a multiple of 1024 up to 4096 (got %lld)", (long long)K);
    MONO_CHECK(workspace_bytes >= rowlin_workspace_bytes(int(K)) && aligned(workspace, 256), "workspace (mono_rowlin_gptq_workspace)");
    MONO_CHECK(aligned(x, 16) && aligned(out, 16) && (!xn_out || aligned(xn_out, 16)), "16-byte aligned rows");
    Program P{};
    P.nph = 1;
    P.M = int(M);
    int64_t N = 0;
    for (int i = 0; i < nm; ++i) {
        MONO_CHECK(weights[i] && aligned(weights[i], 16) && rows[i] >= 16 && rows[i] % 16 == 0, "weight %d: tiled, rows a multiple of 16", i);
        P.ph[0].m[i] = MatDesc{static_cast<const uint8_t*>(weights[i]), nullptr, int(rows[i])};
        N += rows[i];
    }
    MONO_CHECK(N < (int64_t(1) << 24), "output rows");
    uint8_t* w = static_cast<uint8_t*>(workspace);
    P.ph[0].nm = nm;
    P.ph[0].K = int(K);
    P.ph[0].x = reinterpret_cast<const int8_t*>(w);
    P.ph[0].xperm = 1;
    RowLinArgs A{};
    A.x = static_cast<const uint16_t*>(x);
    A.norm_w = static_cast<const uint16_t*>(norm_w);
    A.eps = eps;
    A.gate = static_cast<const uint16_t*>(gate);
    A.gate_row_stride = gate_row_stride;
    A.gate_head_stride = gate_head_stride;
    A.lut = static_cast<const uint16_t*>(lut);
    A.residual = static_cast<const uint16_t*>(residual);
    A.out = static_cast<uint16_t*>(out);
    A.xn_out = static_cast<uint16_t*>(xn_out);
    A.q = reinterpret_cast<int8_t*>(w);
    const size_t qb = (size_t(kStreamMaxRows) * K + 255) / 256 * 256;
    A.s = reinterpret_cast<float*>(w + qb);
    A.bar = reinterpret_cast<unsigned*>(w + qb + 256);
    A.mode = mode;
    A.N = int(N);
    if (ab_out) {
        MONO_CHECK(mode == ROWLIN_NORM && xn_out, "a|b projection: norm mode with xn_out");
        MONO_CHECK(ab_w && aligned(ab_w, 16) && ab_n >= 1 && ab_n <= 128 && ab_stride >= ab_n,
                   "a|b: bf16 weights [ab_n][K] (16-byte aligned), 1 <= ab_n <= 128, ab_stride >= ab_n");
        A.ab_w = static_cast<const uint16_t*>(ab_w);
        A.ab_out = static_cast<uint16_t*>(ab_out);
        A.ab_n = int(ab_n);
        A.ab_stride = ab_stride;
    }
    return launch_rowlin(P, A, reinterpret_cast<cudaStream_t>(stream));
}

int mono_rowlin_gptq(const void* x, int mode, const void* norm_w, float eps, const void* gate, int64_t gate_row_stride,
                     int64_t gate_head_stride, const void* lut, const void* const* weights, const int64_t* rows, int nm,
                     int64_t M, int64_t K, const void* residual, void* out, void* xn_out, void* workspace,
                     size_t workspace_bytes, mono_stream_t stream) {
    return rowlin_entry(x, mode, norm_w, eps, gate, gate_row_stride, gate_head_stride, lut, weights, rows, nm, M, K,
                        residual, out, xn_out, nullptr, 0, nullptr, 0, workspace, workspace_bytes, stream);
}

int mono_rowlin_norm_ab_gptq(const void* x, const void* norm_w, float eps, const void* const* weights,
                             const int64_t* rows, int nm, int64_t M, int64_t K, void* out, void* xn_out,
                             const void* ab_w, int64_t ab_n, void* ab_out, int64_t ab_stride, void* workspace,
                             size_t workspace_bytes, mono_stream_t stream) {
    MONO_CHECK(ab_out && xn_out, "null operand");
    return rowlin_entry(x, ROWLIN_NORM, norm_w, eps, nullptr, 0, 0, nullptr, weights, rows, nm, M, K, nullptr, out,
                        xn_out, ab_w, ab_n, ab_out, ab_stride, workspace, workspace_bytes, stream);
}

}  // extern "C"
