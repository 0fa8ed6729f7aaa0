// extern "C" entry points of the layer programs (program.h): the op builders, plan and launch, and the reference's
// one-launch layers built on them (layer_post: csrc/mono_layer.sycl:243-313; layer_gdn: csrc/mono_gdn.sycl:5-20).
#include <cstring>

#include "program.h"

namespace mono {
namespace {

size_t al256(size_t b) { return (b + 255) / 256 * 256; }

Op* op_at(void* ops, int index) { return static_cast<Op*>(ops) + index; }

int set_rows(Op& op, int mode, const void* x, int64_t x_stride, int64_t K, const void* norm_w, float eps,
             const void* gate, int64_t gate_row_stride, int64_t gate_head_stride, const void* lut, void* xn_out, void* q,
             void* s, void* zero, int barrier) {
    MONO_CHECK(x && q && s, "rows op: null operand");
    MONO_CHECK(mode >= ROWS_NORM && mode <= ROWS_GDN, "rows op: mode 0 (norm), 1 (gate), 2 (quant), 3 (GDN gated norm)");
    MONO_CHECK(K >= kChunkK && K % kChunkK == 0 && K <= 4096, "rows op: K a multiple of 1024 up to 4096");
    MONO_CHECK(x_stride >= K && x_stride % 8 == 0 && aligned(x, 16) && aligned(q, 8) && (!xn_out || aligned(xn_out, 16)),
               "rows op: 16-byte aligned rows");
    MONO_CHECK(mode != ROWS_GATE || (gate && lut && gate_head_stride >= 256 && gate_head_stride % 8 == 0 &&
                                     gate_row_stride % 8 == 0 && aligned(gate, 16)),
               "rows op: gate (16-byte aligned, strides multiples of 8) and LUT");
    MONO_CHECK(mode != ROWS_GDN || (gate && norm_w && gate_row_stride % 8 == 0 && aligned(gate, 16) && aligned(norm_w, 16)),
               "rows op: z rows and the gated-norm weight");
    MONO_CHECK(mode != ROWS_NORM || (norm_w && aligned(norm_w, 16)), "rows op: norm weight");
    std::memset(&op, 0, sizeof(op));
    op.kind = OP_ROWS;
    op.barrier = barrier != 0;
    OpRows& r = op.r;
    r.x = static_cast<const uint16_t*>(x);
    r.norm_w = static_cast<const uint16_t*>(norm_w);
    r.gate = static_cast<const uint16_t*>(gate);
    r.lut = static_cast<const uint16_t*>(lut);
    r.xn_out = static_cast<uint16_t*>(xn_out);
    r.q = static_cast<int8_t*>(q);
    r.s = static_cast<float*>(s);
    r.zero = static_cast<unsigned*>(zero);
    r.x_stride = x_stride;
    r.gate_row_stride = gate_row_stride;
    r.gate_head_stride = gate_head_stride;
    r.eps = eps;
    r.mode = mode;
    r.K = int(K);
    return MONO_OK;
}

int set_gemv(Op& op, const void* const* weights, const int64_t* rows, int nm, int paired, int64_t K, const void* q,
             const void* s, void* out, int64_t out_stride, const void* residual, int64_t res_stride, const void* lut,
             void* amax, int barrier) {
    MONO_CHECK(weights && rows && q && s && out, "gemv op: null operand");
    MONO_CHECK(nm >= 1 && nm <= 3 && (!paired || nm == 2), "gemv op: 1 to 3 matrices, or a gate | up pair");
    MONO_CHECK(K >= kChunkK && K % kChunkK == 0 && K <= kChunkK * kMaxChunks, "gemv op: K a multiple of 1024 up to 16384");
    MONO_CHECK(aligned(q, 16), "gemv op: 16-byte aligned rows");
    std::memset(&op, 0, sizeof(op));
    op.kind = OP_GEMV;
    op.barrier = barrier != 0;
    OpGemv& g = op.g;
    int64_t N = 0;
    for (int i = 0; i < nm; ++i) {
        MONO_CHECK(weights[i] && aligned(weights[i], 16) && rows[i] >= 16 && rows[i] % 16 == 0 && rows[i] < (1 << 24),
                   "gemv op: weight %d tiled, rows a multiple of 16", i);
        g.ph.m[i] = MatDesc{static_cast<const uint8_t*>(weights[i]), nullptr, int(rows[i])};
        N += rows[i];
    }
    if (paired) {
        MONO_CHECK(rows[0] == rows[1], "gemv op: gate and up of one shape");
        MONO_CHECK(lut && amax && !residual, "gemv op: a pair needs the SiLU LUT and the row-maxima words, no residual");
        N = rows[0];
    }
    MONO_CHECK(out_stride >= N && (!residual || res_stride >= N), "gemv op: row strides cover the outputs");
    g.ph.nm = nm;
    g.ph.paired = paired != 0;
    g.ph.K = int(K);
    g.ph.x = static_cast<const int8_t*>(q);
    g.ph.xperm = 1;
    g.xs = static_cast<const float*>(s);
    g.out = static_cast<uint16_t*>(out);
    g.residual = static_cast<const uint16_t*>(residual);
    g.lut = static_cast<const uint16_t*>(lut);
    g.amax = static_cast<unsigned*>(amax);
    g.out_stride = out_stride;
    g.res_stride = res_stride;
    return MONO_OK;
}

int set_quant(Op& op, const void* h, int64_t K, const void* amax, void* q, void* s, int barrier) {
    MONO_CHECK(h && amax && q && s && K % 8 == 0 && K > 0 && aligned(h, 16) && aligned(q, 8), "quant op");
    std::memset(&op, 0, sizeof(op));
    op.kind = OP_QUANT;
    op.barrier = barrier != 0;
    op.q = OpQuant{static_cast<const uint16_t*>(h), static_cast<const unsigned*>(amax), static_cast<int8_t*>(q),
                   static_cast<float*>(s), int(K)};
    return MONO_OK;
}

int set_ab(Op& op, const void* x, int64_t x_stride, int64_t K, const void* w, int64_t N, void* out, int barrier) {
    MONO_CHECK(x && w && out && K % 1024 == 0 && K > 0 && K <= 4096 && N >= 1 && x_stride >= K && x_stride % 8 == 0 &&
                   aligned(x, 16) && aligned(w, 16),
               "a|b op: K a multiple of 1024 up to 4096, 16-byte aligned rows");
    std::memset(&op, 0, sizeof(op));
    op.kind = OP_AB;
    op.barrier = barrier != 0;
    op.ab = OpAb{static_cast<const uint16_t*>(x), static_cast<const uint16_t*>(w), static_cast<uint16_t*>(out), x_stride,
                 int(K), int(N)};
    return MONO_OK;
}

// Workspace of a one-launch layer: barrier words, then 256-aligned pieces.
struct Carve {
    uint8_t* p;
    size_t off = 0;
    template <class T>
    T* take(size_t bytes) {
        T* r = reinterpret_cast<T*>(p ? p + off : nullptr);
        off += al256(bytes);
        return r;
    }
};

// The post block shared by both layers: x1 = x + W_o(q_o) -> RMSNorm -> gate | up -> quant -> down + x1.
struct PostBufs {
    unsigned* bar;
    uint16_t* x1;
    int8_t* q1;
    float* s1;
    uint16_t* h;
    int8_t* q2;
    float* s2;
    unsigned* amax;
};
PostBufs carve_post(Carve& c, int64_t H, int64_t I) {
    PostBufs b;
    b.bar = c.take<unsigned>(256);
    b.x1 = c.take<uint16_t>(16 * H * 2);
    b.q1 = c.take<int8_t>(16 * (H > 4096 ? H : 4096));
    b.s1 = c.take<float>(64);
    b.h = c.take<uint16_t>(16 * I * 2);
    b.q2 = c.take<int8_t>(16 * I);
    b.s2 = c.take<float>(64);
    b.amax = c.take<unsigned>(64);
    return b;
}

// ops [n, n + 5): out projection + residual, then the MLP block
int add_post(Op* ops, int& n, const PostBufs& b, const void* q_o, const void* s_o, int64_t K, const void* o_w,
             const void* x, const void* norm_w, float eps, const void* gate_w, const void* up_w, const void* down_w,
             const void* silu_lut, int64_t H, int64_t I, void* out) {
    int rc;
    const void* wo[1] = {o_w};
    const int64_t ro[1] = {H};
    if ((rc = set_gemv(ops[n++], wo, ro, 1, 0, K, q_o, s_o, b.x1, H, x, H, nullptr, nullptr, 1)) != MONO_OK) return rc;
    if ((rc = set_rows(ops[n++], ROWS_NORM, b.x1, H, H, norm_w, eps, nullptr, 0, 0, nullptr, nullptr, b.q1, b.s1, b.amax,
                       1)) != MONO_OK)
        return rc;
    const void* wgu[2] = {gate_w, up_w};
    const int64_t rgu[2] = {I, I};
    if ((rc = set_gemv(ops[n++], wgu, rgu, 2, 1, H, b.q1, b.s1, b.h, I, nullptr, 0, silu_lut, b.amax, 1)) != MONO_OK)
        return rc;
    if ((rc = set_quant(ops[n++], b.h, I, b.amax, b.q2, b.s2, 1)) != MONO_OK) return rc;
    const void* wd[1] = {down_w};
    const int64_t rd[1] = {H};
    return set_gemv(ops[n++], wd, rd, 1, 0, I, b.q2, b.s2, out, H, b.x1, H, nullptr, nullptr, 0);
}

}  // namespace
}  // namespace mono

using namespace mono;

extern "C" {

size_t mono_program_op_bytes(void) { return sizeof(Op); }

size_t mono_program_workspace(void) { return 256; }

int mono_program_rows(void* ops, int index, int mode, const void* x, int64_t x_stride, int64_t K, const void* norm_w,
                      float eps, const void* gate, int64_t gate_row_stride, int64_t gate_head_stride, const void* lut,
                      void* xn_out, void* q, void* s, void* zero, int barrier) {
    MONO_CHECK(ops && index >= 0, "ops array");
    return set_rows(*op_at(ops, index), mode, x, x_stride, K, norm_w, eps, gate, gate_row_stride, gate_head_stride, lut,
                    xn_out, q, s, zero, barrier);
}

int mono_program_gemv(void* ops, int index, const void* const* weights, const int64_t* rows, int nm, int paired,
                      int64_t K, const void* q, const void* s, void* out, int64_t out_stride, const void* residual,
                      int64_t residual_stride, const void* silu_lut, void* amax, int barrier) {
    MONO_CHECK(ops && index >= 0, "ops array");
    return set_gemv(*op_at(ops, index), weights, rows, nm, paired, K, q, s, out, out_stride, residual, residual_stride,
                    silu_lut, amax, barrier);
}

int mono_program_quant(void* ops, int index, const void* h, int64_t K, const void* amax, void* q, void* s, int barrier) {
    MONO_CHECK(ops && index >= 0, "ops array");
    return set_quant(*op_at(ops, index), h, K, amax, q, s, barrier);
}

int mono_program_ab(void* ops, int index, const void* x, int64_t x_stride, int64_t K, const void* w, int64_t N, void* out,
                    int barrier) {
    MONO_CHECK(ops && index >= 0, "ops array");
    return set_ab(*op_at(ops, index), x, x_stride, K, w, N, out, barrier);
}

int mono_program_gdn(void* ops, int index, int delta, const void* qkv, const void* z, const void* a, const void* b,
                     const void* conv_w, void* conv_state, const float* dt_bias, const float* g_decay, float* state,
                     const void* gnorm_w, float gnorm_eps, float qscale, int64_t M, int64_t HK, int64_t HV, void* raw,
                     const int32_t* ctl, const void* prev_qkv, const void* prev_a, const void* prev_b, void* save_qkv,
                     void* save_a, void* save_b, int64_t qkv_stride, int64_t z_stride, int64_t ab_stride,
                     void* workspace, size_t workspace_bytes, int barrier) {
    MONO_CHECK(ops && index >= 0, "ops array");
    MONO_CHECK(!ctl || (prev_qkv && prev_a && prev_b && save_qkv && save_a && save_b), "deferred form: prev and save buffers");
    MONO_CHECK(HV <= 32, "at most 32 value heads");
    Op& op = *op_at(ops, index);
    std::memset(&op, 0, sizeof(op));
    const int rc = fill_gdn_args(op.gdn, qkv, z, a, b, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, gnorm_eps,
                                 qscale, M, HK, HV, raw, workspace, workspace_bytes, ctl, prev_qkv, prev_a, prev_b,
                                 save_qkv, save_a, save_b, qkv_stride, z_stride, ab_stride);
    if (rc != MONO_OK) return rc;
    op.kind = delta ? OP_GDN_DELTA : OP_GDN_CONV;
    op.barrier = barrier != 0;
    return MONO_OK;
}

int mono_program_plan(void* ops, int nops, int64_t M) {
    MONO_CHECK(ops, "ops array");
    return plan_program(static_cast<Op*>(ops), nops, int(M));
}

int mono_program_launch(const void* ops, const void* ops_device, int nops, int64_t M, void* workspace, int prefetch,
                        mono_stream_t stream) {
    MONO_CHECK(workspace && aligned(workspace, 256), "workspace (mono_program_workspace bytes, zero-filled once)");
    MONO_CHECK(!ops_device || aligned(ops_device, 16), "ops in device memory: 16-byte aligned");
    return launch_program(static_cast<const Op*>(ops), static_cast<const Op*>(ops_device), nops, int(M),
                          static_cast<unsigned*>(workspace), prefetch, reinterpret_cast<cudaStream_t>(stream));
}

int mono_gdn_ab(const void* x, int64_t x_stride, const void* w, int64_t K, int64_t M, int64_t N, void* out,
                mono_stream_t stream) {
    MONO_CHECK(x && w && out, "null operand");
    MONO_CHECK(M >= 1 && M <= 32 && N >= 1 && K % 1024 == 0 && K > 0 && K <= 4096 && x_stride >= K && x_stride % 8 == 0,
               "1 <= M <= 32, K a multiple of 1024 up to 4096");
    MONO_CHECK(aligned(x, 16) && aligned(w, 16), "16-byte aligned rows");
    return launch_gdn_ab(static_cast<const uint16_t*>(x), x_stride, static_cast<const uint16_t*>(w), int(K), int(M), int(N),
                         static_cast<uint16_t*>(out), N, reinterpret_cast<cudaStream_t>(stream));
}

size_t mono_layer_post_gptq_workspace(int64_t K, int64_t H, int64_t I) {
    if (K < 1 || H < 1 || I < 1) return 0;
    Carve c{nullptr};
    carve_post(c, H, I);
    c.take<int8_t>(16 * K);  // q of the out projection's input
    c.take<float>(64);
    return c.off;
}

int mono_layer_post_gptq(const void* x, const void* y, int64_t K, const void* gate, int64_t gate_row_stride,
                         int64_t gate_head_stride, const void* sig_lut, const void* o_w, const void* norm_w, float eps,
                         const void* gate_w, const void* up_w, const void* down_w, const void* silu_lut, int64_t M,
                         int64_t H, int64_t I, void* out, void* workspace, size_t workspace_bytes, mono_stream_t stream) {
    MONO_CHECK(x && y && o_w && norm_w && gate_w && up_w && down_w && silu_lut && out && workspace, "null operand");
    MONO_CHECK(M >= 1 && M <= 16, "1 <= M <= 16 (got %lld)", (long long)M);
    MONO_CHECK(H >= 1024 && H % 1024 == 0 && H <= 4096 && I >= 1024 && I % 1024 == 0 && I <= 16384,
               "H a multiple of 1024 up to 4096, I a multiple of 1024 up to 16384");
    MONO_CHECK(workspace_bytes >= mono_layer_post_gptq_workspace(K, H, I) && aligned(workspace, 256),
               "workspace (mono_layer_post_gptq_workspace), zero-filled before its first use");
    MONO_CHECK(aligned(x, 16) && aligned(out, 16), "16-byte aligned rows");
    Carve c{static_cast<uint8_t*>(workspace)};
    const PostBufs b = carve_post(c, H, I);
    int8_t* qo = c.take<int8_t>(16 * K);
    float* so = c.take<float>(64);
    Op ops[kProgParamOps];
    int n = 0, rc;
    if ((rc = set_rows(ops[n++], gate ? ROWS_GATE : ROWS_QUANT, y, K, K, nullptr, 0.f, gate, gate_row_stride,
                       gate_head_stride, sig_lut, nullptr, qo, so, nullptr, 1)) != MONO_OK)
        return rc;
    if ((rc = add_post(ops, n, b, qo, so, K, o_w, x, norm_w, eps, gate_w, up_w, down_w, silu_lut, H, I, out)) != MONO_OK)
        return rc;
    if ((rc = plan_program(ops, n, int(M))) != MONO_OK) return rc;
    return launch_program(ops, nullptr, n, int(M), b.bar, 0, reinterpret_cast<cudaStream_t>(stream));
}

size_t mono_layer_gdn_gptq_workspace(int64_t M, int64_t H, int64_t I, int64_t HK, int64_t HV) {
    if (M < 1 || H < 1 || I < 1 || HK < 1 || HV < 1) return 0;
    const int64_t C = (2 * HK + HV) * 128, Z = HV * 128;
    Carve c{nullptr};
    carve_post(c, H, I);
    c.take<uint16_t>(16 * H * 2);         // xn
    c.take<uint16_t>(16 * (C + Z) * 2);   // proj | z
    c.take<uint16_t>(16 * 2 * HV * 2);    // a | b
    c.take<uint16_t>(16 * Z * 2);         // raw
    c.take<int8_t>(16 * Z);               // q of the core rows
    c.take<float>(64);
    c.take<uint8_t>(mono_gdn_step_workspace(M, C, HV));
    return c.off;
}

int mono_layer_gdn_gptq(const void* x, const void* norm_in, float eps_in, const void* qkv_w, const void* z_w,
                        const void* wab, const void* conv_w, void* conv_state, const float* dt_bias, const float* g_decay,
                        float* state, const void* gnorm_w, float gnorm_eps, float qscale, const int32_t* ctl,
                        const void* prev_qkv, const void* prev_a, const void* prev_b, void* save_qkv, void* save_a,
                        void* save_b, const void* out_w, const void* norm_post, float eps_post, const void* gate_w,
                        const void* up_w, const void* down_w, const void* silu_lut, int64_t M, int64_t H, int64_t I,
                        int64_t HK, int64_t HV, void* out, void* workspace, size_t workspace_bytes, mono_stream_t stream) {
    MONO_CHECK(x && norm_in && qkv_w && z_w && wab && out_w && norm_post && gate_w && up_w && down_w && silu_lut && out &&
                   workspace,
               "null operand");
    MONO_CHECK(M >= 1 && M <= 8, "1 <= M <= 8 rows (got %lld)", (long long)M);
    MONO_CHECK(H >= 1024 && H % 1024 == 0 && H <= 4096 && I >= 1024 && I % 1024 == 0 && I <= 16384,
               "H a multiple of 1024 up to 4096, I a multiple of 1024 up to 16384");
    MONO_CHECK(HK >= 1 && HV % HK == 0 && HV * 128 <= 4096 && (HV * 128) % 1024 == 0, "value heads: 8, 16, 24 or 32");
    MONO_CHECK(workspace_bytes >= mono_layer_gdn_gptq_workspace(M, H, I, HK, HV) && aligned(workspace, 256),
               "workspace (mono_layer_gdn_gptq_workspace), zero-filled before its first use");
    MONO_CHECK(aligned(x, 16) && aligned(out, 16), "16-byte aligned rows");
    const int64_t C = (2 * HK + HV) * 128, Z = HV * 128;
    Carve c{static_cast<uint8_t*>(workspace)};
    const PostBufs b = carve_post(c, H, I);
    uint16_t* xn = c.take<uint16_t>(16 * H * 2);
    uint16_t* proj = c.take<uint16_t>(16 * (C + Z) * 2);
    uint16_t* ab = c.take<uint16_t>(16 * 2 * HV * 2);
    uint16_t* raw = c.take<uint16_t>(16 * Z * 2);
    int8_t* qc = c.take<int8_t>(16 * Z);
    float* sc = c.take<float>(64);
    void* gws = c.take<uint8_t>(mono_gdn_step_workspace(M, C, HV));
    const size_t gws_bytes = mono_gdn_step_workspace(M, C, HV);
    Op ops[kProgParamOps];
    int n = 0, rc;
    // P1 rows: xn = RMSNorm(x), q1 = quant(xn)
    if ((rc = set_rows(ops[n++], ROWS_NORM, x, H, H, norm_in, eps_in, nullptr, 0, 0, nullptr, xn, b.q1, b.s1, nullptr, 1)) !=
        MONO_OK)
        return rc;
    // P2: a | b (bf16, on the last CTAs) and proj | z = W4(q1)
    if ((rc = set_ab(ops[n++], xn, H, H, wab, 2 * HV, ab, 0)) != MONO_OK) return rc;
    const void* wp[2] = {qkv_w, z_w};
    const int64_t rp[2] = {C, Z};
    if ((rc = set_gemv(ops[n++], wp, rp, 2, 0, H, b.q1, b.s1, proj, C + Z, nullptr, 0, nullptr, nullptr, 1)) != MONO_OK)
        return rc;
    // P3 conv + gates, P4-P5 replay + verify delta
    for (int delta = 0; delta < 2; ++delta) {
        Op& op = ops[n++];
        std::memset(&op, 0, sizeof(op));
        if ((rc = fill_gdn_args(op.gdn, proj, proj + C, ab, ab + HV, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w,
                                gnorm_eps, qscale, M, HK, HV, raw, gws, gws_bytes, ctl, prev_qkv, prev_a, prev_b, save_qkv,
                                save_a, save_b, C + Z, C + Z, 2 * HV)) != MONO_OK)
            return rc;
        op.kind = delta ? OP_GDN_DELTA : OP_GDN_CONV;
        op.barrier = 1;
    }
    // gated RMSNorm + quant of the core rows, then the post block
    if ((rc = set_rows(ops[n++], ROWS_GDN, raw, Z, Z, gnorm_w, gnorm_eps, proj + C, C + Z, 0, nullptr, nullptr, qc, sc,
                       nullptr, 1)) != MONO_OK)
        return rc;
    if ((rc = add_post(ops, n, b, qc, sc, Z, out_w, x, norm_post, eps_post, gate_w, up_w, down_w, silu_lut, H, I, out)) !=
        MONO_OK)
        return rc;
    if ((rc = plan_program(ops, n, int(M))) != MONO_OK) return rc;
    return launch_program(ops, nullptr, n, int(M), b.bar, 0, reinterpret_cast<cudaStream_t>(stream));
}

}  // extern "C"
