/* mono_b200: C ABI of the B200 (sm_100a) W4A8 decode-step kernels.
 *
 * One entry point per operation of the reference's native module (comfy-mono-decode-xpu
 * csrc/bindings.cpp), with torch::Tensor arguments replaced by device pointers, sizes and a CUDA stream.
 * Conventions:
 *   - every pointer is device memory owned by the caller (outputs included), unless noted;
 *   - shapes and alignment are validated on the host before any launch; a rejected call launches nothing;
 *   - the return value is a status (MONO_OK = 0); mono_last_error() gives the calling thread's last message;
 *   - work is enqueued on `stream` (NULL = the legacy default stream) and nothing synchronizes;
 *   - bounded device-side waits never trap: they record a code that mono_device_status() reads.
 */
#ifndef MONO_B200_H
#define MONO_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define MONO_API __attribute__((visibility("default")))
#else
#define MONO_API
#endif

typedef struct CUstream_st* mono_stream_t; /* the same handle as cudaStream_t */

enum {
    MONO_OK = 0,
    MONO_EINVAL = 1,   /* argument rejected before launch */
    MONO_ECUDA = 2,    /* a CUDA runtime call failed */
    MONO_ETIMEOUT = 3, /* a device-side bounded wait gave up */
    MONO_EDEVICE = 4   /* the device error word is set */
};

/* output dtype codes, as the reference's out_dtype_code (csrc/w4a8_decode.sycl:360-361) */
enum { MONO_OUT_F32 = 0, MONO_OUT_BF16 = 2 };
/* relative-scale dtypes of the REF weight format */
enum { MONO_SCALE_FP8_E4M3 = 0, MONO_SCALE_F32 = 1 };
/* W4 weight formats: GPTQ = int4 symmetric, fp16 scale per (row, 128-group);
 * REF = the reference's AsymW4A8Int8Layout codes + codebook + FP8 G16 + channel scale */
enum { MONO_FMT_GPTQ = 0, MONO_FMT_REF = 1 };
/* W4 weight layouts: ROW = the checkpoint's [N][K/2] bytes; TILED = mono_w4_repack's B200 tile-major copy */
enum { MONO_LAYOUT_ROW = 0, MONO_LAYOUT_TILED = 1 };

MONO_API const char* mono_last_error(void);
MONO_API int mono_abi_version(void);
/* Reads (and with reset != 0 clears) the device error word of the current device. Synchronizes. */
MONO_API int mono_device_status(int* code, int reset);

/* Phase trace (the role of the reference's per-phase clock stamps, csrc/mono_mlp.sycl:108-169): with a
 * device buffer of mono_trace_bytes() set, thread 0 of every CTA of the fused kernels writes %globaltimer
 * (ns) at each phase boundary to [cta][phase] (uint64, 1024 x 16). NULL turns it off (the default).
 * Synchronous; not for use while kernels run. */
MONO_API size_t mono_trace_bytes(void);
MONO_API int mono_trace_enable(void* buffer, size_t bytes);

/* ---- W4A8 linear ----------------------------------------------------------------------------------- */

/* Replaces _C.w4a8_decode_linear (csrc/bindings.cpp:71-74; csrc/w4a8_decode.sycl:325-370).
 *   out[m, n] = cast(float(int32 sum_k x[m, k] * w_i8[n, k]) * x_scale[m] * s_channel[n]) (+ residual)
 *   w_i8 = isnan(r) ? 0 : clamp(r, -127, 127), r = rint(codebook[code] * s_rel[n, k / 16])
 * x int8 [M, K] (16 B aligned), x_scale f32 [M], packed [N, K/2] bytes (low nibble = even k) with s_rel
 * FP8 e4m3 [N, K/16] (G16), or packed = the TILED copy (s_rel unused), s_channel f32 [N], pair_table from
 * mono_w4_pair_table(codebook), residual [M, N] in the output dtype or NULL, out [M, N].
 * 1 <= M <= 16, K % 1024 == 0, K <= 16384, N % 16 == 0, group_size == 16. */
MONO_API int mono_w4a8_decode_linear(const int8_t* x, const float* x_scale, const void* packed, const void* s_rel,
                            int s_rel_dtype, const float* s_channel, const uint16_t* pair_table,
                            const void* residual, int64_t M, int64_t N, int64_t K, int64_t group_size,
                            int out_dtype_code, int layout, void* out, mono_stream_t stream);

/* The REF decode table of one codebook (NULL = the reference's default float(i - 8)): 65536 uint16
 * entries (scale byte << 8 | code byte) -> int8 value of the low code | int8 value of the high code << 8.
 * Stands in for the per-element decode of csrc/w4a8_decode.sycl:35-45 and the pair table of
 * csrc/mono_common.hpp:94-141 (which covers scale bytes < 0x80 only; this one covers all 256). */
MONO_API int mono_w4_pair_table(const float* codebook, uint16_t* table, mono_stream_t stream);

/* GPTQ W4A8 linear (the reference has no GPTQ entry, its W4A8 linear above is the
 * closest): int4 v in [-8, 7] stored as nibble v + 8 (8 per int32 along K, i.e. [N, K/2] bytes),
 * fp16 scales [N, K/128] (or packed = the TILED copy, scales unused);
 *   acc_g = int32 sum over group g of x * v;  F_c = sum_{g in 1024-chunk c} float(acc_g) * float(s[n, g]);
 *   out = cast((sum_c F_c) * x_scale[m])  (fp32, sequential sums from +0, no fused multiply-add). */
MONO_API int mono_w4a8_gptq_linear(const int8_t* x, const float* x_scale, const void* packed, const void* scales,
                          const void* residual, int64_t M, int64_t N, int64_t K, int out_dtype_code, int layout,
                          void* out, mono_stream_t stream);

/* The same linear from bf16 activations x [M, K]: the per-token int8 quantization (mono_act_quant's
 * arithmetic, bit for bit) runs inside the kernel, so config 0's whole op (bf16 in -> quant -> W4A8 GEMV
 * -> bf16 out) is one launch. The quantized rows are held in shared memory: shapes whose M * (K + 16)
 * bytes do not fit next to the weight rings return MONO_EINVAL (use mono_act_quant + the entry above).
 * No reference counterpart (the reference quantizes inside its fused layer kernels,
 * csrc/mono_layer.sycl:69-155). */
MONO_API int mono_w4a8_gptq_linear_bf16(const void* x, const void* packed, const void* scales, const void* residual,
                                        int64_t M, int64_t N, int64_t K, int out_dtype_code, int layout, void* out,
                                        mono_stream_t stream);

/* Tile-major copy of a W4 weight for the TILED layout (the role of tiles.py tile_major,
 * comfy_mono_decode_xpu/tiles.py:45-48, in this build's own layout): one buffer of
 * mono_w4_tiled_bytes(fmt, N, K) bytes holding, per (16-row tile, 1024-wide chunk), the chunk's weights in
 * mma fragment order (GPTQ nibbles re-coded as two's complement) followed by its scales, so the kernels
 * fetch a whole chunk with one bulk copy. packed [N, K/2], scales GPTQ fp16 [N, K/128] / REF fp8
 * [N, K/16]. N % 16 == 0, K % 1024 == 0. */
MONO_API size_t mono_w4_tiled_bytes(int fmt, int64_t N, int64_t K);
MONO_API int mono_w4_repack(int fmt, const void* packed, const void* scales, int64_t N, int64_t K, void* tiled,
                            mono_stream_t stream);

/* ---- activation quantization ----------------------------------------------------------------------- */

/* GPTQ activation quant: per row s = amax / 127, q = clamp(rint(x / s), -127, 127).
 * x bf16 [M, K] (16 B aligned), q int8 [M, K], scale f32 [M]. K % 8 == 0. */
MONO_API int mono_act_quant(const void* x_bf16, int64_t M, int64_t K, int8_t* q, float* scale, mono_stream_t stream);

/* Replaces _C.rot_quant (csrc/bindings.cpp:104; csrc/act_prep.sycl:97-110): ConvRot rotation by H
 * (bf16 [256, 256]) per 256-group, then row-wise int8 quantization. x bf16 [M, K], q int8 [M, K],
 * scale f32 [M]. 1 <= M <= 256, K % 256 == 0. workspace: mono_rot_quant_workspace(M, K) bytes, zero-filled
 * before its first use (the kernels leave it reusable); one call at a time per workspace. */
MONO_API size_t mono_rot_quant_workspace(int64_t M, int64_t K);
MONO_API int mono_rot_quant(const void* x_bf16, const void* h_bf16, int64_t M, int64_t K, int8_t* q, float* scale,
                   void* workspace, mono_stream_t stream);

/* rot_quant for callers that cannot allocate device memory (no counterpart in the reference): a host
 * framework that owns every device allocation through its own fixed pool and forbids others, or a plugin
 * loaded into a process whose allocator it may not touch, gets the same result as mono_rot_quant without
 * passing a workspace. The scratch is a fixed array inside the library (about 386 KB per GPU that loads
 * it, held until the process exits), so shapes are limited to 1 <= M <= 16 rows and K <= 12288
 * (K % 256 == 0); larger shapes return MONO_EINVAL. The first call in each device context looks up the
 * array's device address (a runtime query, done again if the context changes); make that first call
 * before any stream capture. All calls share the array and it keeps the last call's contents (the
 * counters that must start at zero are cleared by every call): calls that overlap on the GPU (other
 * streams, other threads) race and must be serialized by the caller. Allocates nothing (no cudaMalloc /
 * cudaFree). */
MONO_API int mono_rot_quant_noalloc(const void* x_bf16, const void* h_bf16, int64_t M, int64_t K, int8_t* q,
                                    float* scale, mono_stream_t stream);

/* ---- fused MLP block --------------------------------------------------------------------------------- */

/* GPTQ MLP block in one cooperative launch (the GPTQ counterpart of _C.mono_mlp, csrc/bindings.cpp:75-77;
 * csrc/mono_mlp.sycl:34-180, and of layer_post's MLP phases, csrc/mono_layer.sycl:272-313):
 *   xn = RMSNorm(x; norm_w, eps)  (norm_w NULL: xn = x)        q1, s1 = act_quant(xn)
 *   g, u = GPTQ linear (gate, up)(q1)  h = bf16(silu_lut[g] * u)  q2, s2 = act_quant(h)
 *   out = bf16(x + bf16(GPTQ down(q2)))  (residual != 0)  or  bf16(GPTQ down(q2))
 * RMSNorm order: P[t] = sum over the 8-element pieces t + 128 j (j outer, element inner) of x^2 (t < 128),
 * butterfly within each 32, the 4 partial sums in order, r = 1 / sqrt(total / H + eps),
 * out = bf16((x * r) * w) (IEEE fp32 ops, no fused multiply-add).
 * x, out bf16 [M, H] (out may alias x); gate/up: TILED copies of [I, H/2] weights; down: of [H, I/2];
 * silu_lut bf16 [65536] (SiLU of every bf16 bit pattern). 1 <= M <= 16, H a multiple of 1024 up to
 * 4096, I a multiple of 1024 up to 16384. workspace: mono_mlp_gptq_workspace(H, I) bytes, zero-filled before its first use (the kernel
 * leaves it reusable); one call at a time per workspace. */
MONO_API size_t mono_mlp_gptq_workspace(int64_t H, int64_t I);
MONO_API int mono_mlp_gptq(const void* x, const void* norm_w, float eps, const void* gate, const void* up,
                           const void* down, const void* silu_lut, int64_t M, int64_t H, int64_t I, int residual,
                           void* out, void* workspace, size_t workspace_bytes, mono_stream_t stream);

/* Row preparation + GPTQ W4A8 linear in one cooperative launch (the reference's layer_pre, csrc/mono_layer.sycl:
 * 69-155, and the gate / out-projection front of layer_post, :243-270):
 *   mode 0 (norm):  xn = RMSNorm(x; norm_w, eps) (the order of mono_mlp_gptq), q, s = act_quant(xn)
 *                   (xn_out, if not NULL, receives xn)
 *   mode 1 (gate):  y = bf16(x * lut[gate]) with gate element (m, c) at
 *                   gate[m * gate_row_stride + (c / 256) * gate_head_stride + c % 256] (the gate half of the
 *                   gated query heads: head stride 512) and lut the sigmoid of every bf16 pattern; q, s = act_quant(y)
 *   mode 2 (quant): q, s = act_quant(x)
 *   out[m][n] = bf16(GPTQ linear(q, s)) (+ residual: bf16(residual + that)) for nm (1..3) TILED weights of
 *   rows[i] outputs each, concatenated along n (out row stride = sum of rows).
 * x bf16 [M][K], 1 <= M <= 32, K a multiple of 1024 up to 4096. workspace: mono_rowlin_gptq_workspace(K) bytes,
 * zero-filled before its first use (the kernel leaves it reusable); one call at a time per workspace. */
MONO_API size_t mono_rowlin_gptq_workspace(int64_t K);
MONO_API int mono_rowlin_gptq(const void* x, int mode, const void* norm_w, float eps, const void* gate,
                              int64_t gate_row_stride, int64_t gate_head_stride, const void* lut,
                              const void* const* weights, const int64_t* rows, int nm, int64_t M, int64_t K,
                              const void* residual, void* out, void* xn_out, void* workspace, size_t workspace_bytes,
                              mono_stream_t stream);
/* The GDN layer's front in one launch: mono_rowlin_gptq in mode 0 (RMSNorm -> quant -> qkv | z, the normalized
 * rows to xn_out [M][K], required) and the a | b projection of those rows, ab_out[m * ab_stride + n] =
 * mono_gdn_ab(xn_out, ab_w)[m][n] bit for bit (ab_w bf16 [ab_n][K], 1 <= ab_n <= 128 and at most the launch's
 * CTAs: min(output rows / 16, SMs)). It replaces mono_rowlin_gptq + mono_gdn_ab of the reference's GDN layer_pre
 * (csrc/mono_layer.sycl:69-155 and the in_proj_a / in_proj_b linear, csrc/mono_gdn.sycl:10-11). */
MONO_API int mono_rowlin_norm_ab_gptq(const void* x, const void* norm_w, float eps, const void* const* weights,
                                      const int64_t* rows, int nm, int64_t M, int64_t K, void* out, void* xn_out,
                                      const void* ab_w, int64_t ab_n, void* ab_out, int64_t ab_stride,
                                      void* workspace, size_t workspace_bytes, mono_stream_t stream);

/* ---- full-attention decode layer ------------------------------------------------------------------ */

/* Per-head Q/K RMSNorm + partial split-half RoPE + K/V cache write (the role of the reference's
 * qk_norm_rope_kv, csrc/rope_kv.sycl:120-245; bindings.cpp exposes it as _C.qk_norm_rope_kv).
 * rawq: bf16 query heads [S][Hq] of 256 (row / head strides in elements: the query half of gated heads has
 * head stride 512); rawk, v: bf16 [S][Hk][256] (row strides in elements); wq, wk: bf16 [256] norm weights;
 * freqs: fp32 [S][rd/2][2][2] ([[f00, f01], [f10, f11]] per pair); key/value caches bf16 [Hk][cap][256];
 * position: int64 [S] device positions (outside [0, cap): the write is skipped, mono_device_status reports
 * code 4). Head norm: lane sums of squares over 8-element pieces, xor butterfly, r = 1 / sqrt(sum / 256 + eps),
 * bf16((x * r) * w) (this build's pinned order); RoPE per pair j < rd/2 of the normalized row:
 *   o0 = t[j] * f00 + t[j + rd/2] * f01,  o1 = t[j + rd/2] * f11 + t[j] * f10
 * each product rounded to fp32, the sum once to bf16 (csrc/rope_kv.sycl:7-9). out_q bf16 [Hq][S][256],
 * out_k bf16 [Hk][S][256]. 1 <= S <= 8. */
MONO_API int mono_qk_norm_rope_kv(const void* rawq, int64_t q_row_stride, int64_t q_head_stride, const void* rawk,
                                  int64_t k_row_stride, const void* v, int64_t v_row_stride, const void* wq,
                                  const void* wk, const float* freqs, void* key_cache, void* value_cache, int64_t cap,
                                  const int64_t* position, int64_t S, int64_t Hq, int64_t Hk, float epsq, float epsk,
                                  int64_t rd, void* out_q, void* out_k, mono_stream_t stream);
/* The same for `streams` batched decode streams (1 <= streams <= 8) sharing one launch: rows [b R, (b + 1) R) of
 * the S = streams x R rows (R <= 8) are stream b's; its caches are heads [b Hk, (b + 1) Hk) of key/value caches
 * bf16 [streams][Hk][cap][256]; out_q bf16 [streams][Hq][R][256], out_k bf16 [streams][Hk][R][256]. Each row's
 * result is the one-stream call's (streams = 1 is mono_qk_norm_rope_kv). */
MONO_API int mono_qk_norm_rope_kv_streams(const void* rawq, int64_t q_row_stride, int64_t q_head_stride,
                                          const void* rawk, int64_t k_row_stride, const void* v, int64_t v_row_stride,
                                          const void* wq, const void* wk, const float* freqs, void* key_cache,
                                          void* value_cache, int64_t cap, const int64_t* position, int64_t S,
                                          int64_t streams, int64_t Hq, int64_t Hk, float epsq, float epsk, int64_t rd,
                                          void* out_q, void* out_k, mono_stream_t stream);

/* Tree decode attention (the role of the reference's attn_dpas, csrc/attn_dpas.sycl:269-342): every query row
 * (q head h, row s) attends the committed prefix [0, L) of the cache of kv head h / (H / Hk) and the tree
 * rows t with (mask[s] >> t) & 1 (their keys / values in xk / xv), softmax of (k . q) / 16, P rounded to bf16
 * for P V, fp32 accumulation, bf16 output. L = clamp(seqlen[0], 0, cap) is read on the device (no host sync).
 * q bf16 [H][S][256]; caches bf16 [Hk][cap][256]; xk, xv bf16 [Hk][S][256]; mask int32 [S] (NULL with S = 1:
 * the MTP draft row, prefix only); out bf16 [S][H * 256]. (H / Hk) * S <= 32, 1 <= S <= 8. workspace:
 * mono_tree_attention_workspace(Hk, cap) bytes, zero-filled before its first use (the call leaves its arrival
 * counters at zero again); one call at a time per workspace. Launch order: the kernel carries a programmatic
 * dependency on the preceding kernel and may load K / V tiles of the prefix before waiting for it: the prefix
 * [0, L) (with a mask; [0, L - S) without) must not be written by the two kernels launched just before the call. Not bit-exact with any other implementation: results are within the tolerance of an fp64
 * reference stated by the tests. */
MONO_API size_t mono_tree_attention_workspace(int64_t Hk, int64_t cap);
MONO_API int mono_tree_attention(const void* q, const void* key_cache, const void* value_cache, const int32_t* seqlen,
                                 const void* xk, const void* xv, const int32_t* mask, int64_t H, int64_t Hk, int64_t S,
                                 int64_t cap, void* out, void* workspace, size_t workspace_bytes, mono_stream_t stream);
/* The same for `streams` batched decode streams (1 <= streams <= 8) with one tree shape (mask int32 [S], shared):
 * q bf16 [streams][H][S][256]; caches bf16 [streams][Hk][cap][256]; seqlen int32 [streams] (stream b's committed
 * length); xk bf16 [streams][Hk][S][256]; xv: the tree value row t of stream b's kv head k at element offset
 * b xv_stream_stride + k xv_head_stride + t xv_row_stride (multiples of 8; the projection rows in place, no
 * copy); out bf16 [streams][S][H * 256]. Every stream's context is split as it would be alone, so each stream's
 * output equals its one-stream call's. Workspace: mono_tree_attention_streams_workspace(Hk, streams, cap) bytes,
 * zero-filled before first use. */
MONO_API size_t mono_tree_attention_streams_workspace(int64_t Hk, int64_t streams, int64_t cap);
MONO_API int mono_tree_attention_streams(const void* q, const void* key_cache, const void* value_cache,
                                         const int32_t* seqlen, const void* xk, const void* xv, const int32_t* mask,
                                         int64_t H, int64_t Hk, int64_t S, int64_t streams, int64_t cap,
                                         int64_t xv_stream_stride, int64_t xv_head_stride, int64_t xv_row_stride,
                                         void* out, void* workspace, size_t workspace_bytes, mono_stream_t stream);

/* ---- Gated-DeltaNet ----------------------------------------------------------------------------------- */

/* Gated-DeltaNet decode step for M sequential rows that all commit (the conv / gates / L2 norm / delta rule /
 * gated RMSNorm of the reference's layer_gdn, csrc/mono_gdn.sycl:313-611):
 *   conv   y = bf16(sum_d x[t-d] w[3-d]) over the conv state and the new rows, out = bf16(y / (1 + exp(-y)))
 *   gates  decay = exp(g_decay * softplus(a + dt_bias)), beta = bf16(sigmoid(b))
 *   l2     q <- (q * qscale) / max(|q|, 1e-12), k <- k / max(|k|, 1e-12)   (per key head)
 *   delta  S <- S decay; delta = (v - S^T k) beta; S <- S + k delta^T; o = S^T q   (value head h: key head
 *          h / (HV / HK))
 *   gnorm  core = bf16(bf16(bf16(o) * w * rsqrt(mean(bf16(o)^2) + eps)) * bf16(silu(z)))
 * qkv bf16 [M][C] with C = (2 HK + HV) * 128 (q heads, k heads, v heads); z bf16 [M][HV * 128]; a, b bf16
 * [M][HV]; conv_w bf16 [C][4]; conv_state bf16 [C][3] (oldest first, updated); dt_bias, g_decay fp32 [HV];
 * state fp32 [HV][128][128] ([k][v], updated); gnorm_w bf16 [128]; core bf16 [M][HV * 128]. 1 <= M <= 8.
 * fp32 arithmetic; results within the tolerance of an fp64 reference stated by the tests. workspace:
 * mono_gdn_step_workspace(M, C, HV) bytes (256-byte aligned). */
MONO_API size_t mono_gdn_step_workspace(int64_t M, int64_t C, int64_t HV);  /* covers both forms */
/* Launch order: the step's two kernels carry a programmatic dependency on the preceding kernel (they may start
 * while it runs and wait for it before reading qkv, z, a, b): the ctl words, the replay / save buffers and the
 * conv and recurrent states must not be written by the two kernels launched just before the call. */
MONO_API int mono_gdn_step(const void* qkv, const void* z, const void* a, const void* b, const void* conv_w,
                           void* conv_state, const float* dt_bias, const float* g_decay, float* state,
                           const void* gnorm_w, float gnorm_eps, float qscale, int64_t M, int64_t HK, int64_t HV,
                           void* core, void* workspace, size_t workspace_bytes, mono_stream_t stream);

/* The deferred form used by the device MTP loop (the reference's replay + verify, csrc/mono_gdn.sycl:385-567):
 * first the n = ctl[0] rows accepted at the previous step (slots ctl[2 + i], their inputs in prev_qkv [8][C],
 * prev_a / prev_b [8][HV] as saved by that step) are replayed and the recurrent and conv states persisted;
 * then the M verify rows run as a tree on a register copy of the state (core outputs only, nothing persisted):
 * verify row t's conv reads its own input, then its ancestors' (parents ctl[10 + t], -1 at the root), then the
 * committed history; the program ctl[18 + e] (slot | 32 to advance the copy, up to the first slot outside
 * [0, M)) orders the rows so each sees the state after its parent (rows no entry names give a zero raw output);
 * and their inputs are saved to save_qkv / save_a / save_b (which must not alias the prev buffers: alternate
 * two sets between steps). ctl: int32 [26] as written by mono_mtp_accept. qkv, z and a / b may be column
 * slices of wider rows: their row strides (elements) are given (qkv_stride >= C, z_stride >= HV * 128,
 * ab_stride >= HV). */
MONO_API int mono_gdn_step_deferred(const void* qkv, const void* z, const void* a, const void* b, const void* conv_w,
                                    void* conv_state, const float* dt_bias, const float* g_decay, float* state,
                                    const void* gnorm_w, float gnorm_eps, float qscale, int64_t M, int64_t HK,
                                    int64_t HV, void* core, const int32_t* ctl, const void* prev_qkv,
                                    const void* prev_a, const void* prev_b, void* save_qkv, void* save_a, void* save_b,
                                    int64_t qkv_stride, int64_t z_stride, int64_t ab_stride, void* workspace,
                                    size_t workspace_bytes, mono_stream_t stream);
/* The deferred form for `streams` batched decode streams (1 <= streams <= 8) in one launch pair: M rows per stream;
 * qkv, z, a, b, core hold the streams' rows one after another (stream b's rows [b M, (b + 1) M), the row strides
 * as above); conv_state bf16 [streams][C][3], state fp32 [streams][HV][128][128], ctl int32 [streams][ctl_stride
 * >= 26], prev / save buffers [streams][8][C] and [streams][8][HV]; conv_w, dt_bias, g_decay, gnorm_w shared.
 * Each stream's results are its one-stream call's. Workspace: mono_gdn_step_streams_workspace(M, C, HV, streams)
 * bytes. */
MONO_API size_t mono_gdn_step_streams_workspace(int64_t M, int64_t C, int64_t HV, int64_t streams);
MONO_API int mono_gdn_step_deferred_streams(const void* qkv, const void* z, const void* a, const void* b,
                                           const void* conv_w, void* conv_state, const float* dt_bias,
                                           const float* g_decay, float* state, const void* gnorm_w, float gnorm_eps,
                                           float qscale, int64_t M, int64_t HK, int64_t HV, int64_t streams, void* core,
                                           const int32_t* ctl, int64_t ctl_stride, const void* prev_qkv,
                                           const void* prev_a, const void* prev_b, void* save_qkv, void* save_a,
                                           void* save_b, int64_t qkv_stride, int64_t z_stride, int64_t ab_stride,
                                           void* workspace, size_t workspace_bytes, mono_stream_t stream);

/* ---- small row kernels of the bf16 parts of the step (MTP draft head, final norm) ------------------------- */

/* s = add ? bf16(x + add) : x (sum_out receives s when add is given); out = bf16((s * r) * w),
 * r = 1 / sqrt(mean(s^2) + eps) (fp32, per-thread then butterfly then warp-order sums; IEEE div / sqrt).
 * bf16 rows with strides in elements (multiples of 8), H a multiple of 8. */
MONO_API int mono_rmsnorm_add(const void* x, int64_t x_stride, const void* add, int64_t add_stride, const void* w,
                              float eps, int64_t M, int64_t H, void* out, void* sum_out, int64_t out_stride,
                              mono_stream_t stream);
/* The MTP draft head's front in one launch (the reference's draft_embed_norm_cat with a bf16 embedding,
 * csrc/draft_fused.sycl:4-6): for each of B rows (one per decode stream), out[b][0, H) = RMSNorm(embed row of
 * token tokens[b * tok_stride + index]; enorm_w) and out[b][H, 2 H) = RMSNorm(hidden[b]; hnorm_w), each with
 * mono_rmsnorm_add's arithmetic (the same bits as the gather + two mono_rmsnorm_add calls). embed bf16 [V][H];
 * tokens int64 on the device (a token outside [0, V) reads row 0 and sets device status 7); hidden bf16 rows
 * (hidden_stride elements apart); out bf16 rows of 2 H (out_stride apart). */
MONO_API int mono_draft_embed_norm_cat(const void* embed, int64_t V, int64_t H, const int64_t* tokens,
                                       int64_t tok_stride, int64_t index, const void* enorm_w, const void* hidden,
                                       int64_t hidden_stride, const void* hnorm_w, float eps, int64_t B, void* out,
                                       int64_t out_stride, mono_stream_t stream);

/* out[m][c] = bf16(a[m][c] * lut[b[m][(c / 256) * b_head_stride + c % 256]]) (lut: bf16 [65536], e.g. SiLU or
 * sigmoid of every bf16 pattern): SiLU(gate) * up, or attention * sigmoid(gate of gated heads). */
MONO_API int mono_lut_mul(const void* a, int64_t a_stride, const void* b, int64_t b_stride, int64_t b_head_stride,
                          const void* lut, int64_t M, int64_t K, void* out, int64_t out_stride, mono_stream_t stream);

/* ---- logit picks ----------------------------------------------------------------------------------------- */

/* Exact top-k (k <= 8) of every bf16 row x [rows][V] (the role of the reference's fast_topk / fast_pick,
 * csrc/fast_topk.sycl:22-176, which take one row): ranks = the bf16 radix key (NaN on top, -0 below +0), ties
 * in the XPU topk gather order (i >> 15, then (i & 8191) >> 3, then (i & 32767) >> 13, then i & 7);
 * argmax_order != 0 (k = 1): the float argmax order (NaN first, -0 == +0, smallest index on ties).
 * with_argmax != 0 also writes argmax [rows] (int64) from the same pass. values bf16 [rows][k], indices int64
 * [rows][k], best first. workspace: mono_topk_workspace(rows) bytes. */
MONO_API size_t mono_topk_workspace(int64_t rows);
MONO_API int mono_fast_topk(const void* x, int64_t rows, int64_t V, int64_t k, int argmax_order, int with_argmax,
                            void* values, int64_t* indices, int64_t* argmax, void* workspace, size_t workspace_bytes,
                            mono_stream_t stream);

/* ---- MTP loop bookkeeping on the device (the role of csrc/mtp_loop.sycl:29-196) ------------------------ */
/* st: int64 [4] loop state (st[0] committed length = attention index, st[1] MTP KV length); ctl: int32 [26] =
 * [pending, parity, accepted slots[8], tree parents[8], tree program[8]]. Nothing reads back to the host. */

/* freqs[0 .. row_elems) = ftab[min(st[0] + k, cap - 1)] (fp32 rows of row_elems), mpos[i] = st[1] + k + i
 * (i < np), mseq = st[1] + k + 1 (reference: mtp_prep_draft). */
MONO_API int mono_mtp_prep_draft(const int64_t* st, int64_t k, const float* ftab, int64_t row_elems, int64_t cap,
                                 float* freqs, int64_t* mpos, int64_t np, int32_t* mseq, mono_stream_t stream);
/* The same for `streams` batched decode streams in one launch: stream b's st, freqs, mpos and mseq start b x their
 * strides (elements) after the given pointers; each stream's words are its one-stream call's. */
MONO_API int mono_mtp_prep_draft_streams(const int64_t* st, int64_t st_stride, int64_t k, const float* ftab,
                                         int64_t row_elems, int64_t cap, float* freqs, int64_t freqs_stride,
                                         int64_t* mpos, int64_t mpos_stride, int64_t np, int32_t* mseq,
                                         int64_t mseq_stride, int64_t streams, mono_stream_t stream);

/* apos[i] = st[0] + i (i < np <= 64), aseq = st[0], vpos[r] = tree_pos[r] + st[0] + rope_offset (r < rows <= 8),
 * ctl[1] = parity, ctl[10 .. 26) = tree_ctl[0 .. 16) (reference: mtp_prep_verify). */
MONO_API int mono_mtp_prep_verify(const int64_t* st, int64_t* apos, int64_t np, int32_t* aseq, int64_t* vpos,
                                  const int64_t* tree_pos, int64_t rows, int32_t* ctl, const int32_t* tree_ctl,
                                  int64_t parity, int64_t rope_offset, mono_stream_t stream);
/* The same for `streams` batched decode streams in one launch: stream b's st, apos, aseq, vpos and ctl start b x
 * their strides (elements) after the given pointers (tree_pos and tree_ctl are shared); each stream's words are its
 * one-stream call's. */
MONO_API int mono_mtp_prep_verify_streams(const int64_t* st, int64_t st_stride, int64_t* apos, int64_t apos_stride,
                                          int64_t np, int32_t* aseq, int64_t aseq_stride, int64_t* vpos,
                                          int64_t vpos_stride, const int64_t* tree_pos, int64_t rows, int32_t* ctl,
                                          int64_t ctl_stride, const int32_t* tree_ctl, int64_t parity,
                                          int64_t rope_offset, int64_t streams, mono_stream_t stream);

/* The accept step (reference: mtp_accept; host twin comfy_mono_decode_xpu/mtp_loop.py:117-136): from row 0,
 * continue along the first child c (children int32 [8][8], -1 ends a list) with drafts[c] == toks[current];
 * result int64 [32] = [n, commit[8] (drafts along the path, then toks[last], -1 padded), row, on_chain,
 * nranks, ranks[7] (rank of toks[node] among cand[node][0..7), 7 if absent, for path nodes < depth), pos,
 * kept]; st[0] += n, st[1] += kept (kept = min(on_chain ? n : n - 1, depth)); ctl[0] = n,
 * ctl[2 + i] = path[i] (i < n, else i); next_tok = toks[row]; h_out = x[row] (bf16 [rows][H]); for an
 * off-chain path, in every bf16 KV cache [heads][cap][head_dim] listed in kv_ptrs (device int64 [nkv]),
 * slot (pos + path[k]) % cap moves to (pos + k) % cap for k = 1 .. n - 1. cand NULL: no ranks. A listed child
 * index that is not after its parent or not below rows ends the walk there and sets the device status to 5
 * (mono_device_status). */
MONO_API int mono_mtp_accept(int64_t* st, const int64_t* toks, const int64_t* drafts, const int64_t* cand,
                             const int32_t* children, int64_t rows, int64_t depth, const void* x, int64_t H,
                             int64_t* next_tok, void* h_out, int32_t* ctl, const int64_t* kv_ptrs, int64_t nkv,
                             int64_t heads, int64_t cap, int64_t head_dim, int64_t* result, mono_stream_t stream);

/* bf16 GEMV of the MTP draft head (the reference's F.linear on one draft row, comfy_mono_decode_xpu/draft_head.py:
 * 198-210: fc, qkv, o, gate | up, down): out[m][n] = bf16(sum_k x[m][k] * w[n][k]), fp32 accumulation (torch's
 * bf16 linear contract; the summation order is this kernel's). x bf16 [M][x_stride], w bf16 [N][K] row-major,
 * out bf16 [M][out_stride]. 1 <= M <= 8, K a multiple of 256, x and w 16-byte aligned, x_stride % 8 == 0. */
MONO_API int mono_gemv_bf16(const void* x, int64_t x_stride, const void* w, int64_t M, int64_t N, int64_t K, void* out,
                            int64_t out_stride, mono_stream_t stream);

/* bf16 lm_head with the pick fused: the verify's greedy logits + argmax (the reference's verify_logits then
 * lg.argmax, comfy_mono_decode_xpu/mtp_loop.py:325-327) and the draft pick (csrc/draft_lmhead.sycl:87-292: the
 * draft token, the top-n row and the children's verify tokens in one launch). For M <= 16 rows of x [M][x_stride]
 * against w [V][K]: logits = bf16(sum_k x[m][k] * w[n][k]) on the tensor cores (fp32 accumulation over a fixed
 * partition of K into 8 slices, the slices summed in order: the same bits on every launch), then per row
 *   argmax[m]   the argmax by the rank (float order, NaN largest, -0 == +0, smallest index on ties)
 *   topk[m][j]  j < k <= 8, descending by the top-k rank (the reference's fast_topk tie order)
 *   logits      (optional, NULL: not written) bf16 [M][V]
 * and, with children (device int32, up to 8 slots of a dst row, -1 ends) and dst (device int64), for every row m:
 * d = dst + m * dst_stride (dst_stride >= 8 when M > 1), d[children[0]] = argmax, d[children[j]] = topk[j] for
 * 1 <= j < k (a draft token and its siblings' tokens; one row per batched stream). index_base: the
 * vocabulary index of w's row 0 (a tensor-parallel shard; 0 otherwise): ranks and written indices are
 * index_base + row, so the shards' candidates merge into the whole vocabulary's pick. K % 512 == 0, M x rows of
 * K fitting in shared memory next to the rings (K <= 4096 at M = 16);
 * workspace: mono_lmhead_workspace() bytes, zero-filled before first use (the kernel leaves it reusable); one call
 * at a time per workspace. */
MONO_API size_t mono_lmhead_workspace(void);
MONO_API int mono_lmhead_pick(const void* x, int64_t x_stride, const void* w, int64_t M, int64_t V, int64_t K, int64_t k,
                              int64_t index_base, void* logits, int64_t* argmax, int64_t* topk, const int32_t* children,
                              int64_t* dst, int64_t dst_stride, void* workspace, size_t workspace_bytes,
                              mono_stream_t stream);

/* ---- two-GPU one-shot all-reduce (the tensor-parallel variant's residual sum) ------------------------------
 * Each rank allocates an area of mono_allreduce2_area_bytes(cap) bytes with mono_p2p_area_alloc (its own
 * cudaMalloc, zeroed: an IPC handle names a whole allocation), passes its handle (mono_ipc_handle, 64 bytes) to
 * the peer, and maps the peer's (mono_ipc_open). mono_allreduce2_bf16 then sums the n bf16 values of `in` on both
 * ranks into `out` (may be `in`): the chunk of CTA b is stored into the peer's area over NVLink, a release-add
 * raises the peer's counter b, the CTA waits (acquire, bounded: 1 s, device error 6) for its own counter b, and
 * writes bf16(float(in) + float(received)) — the same bits on both ranks. my_calls: a zeroed device int32 [16]
 * of this rank (the call count per CTA: the kernel takes no host scalar and replays in CUDA graphs). Both ranks
 * must make the same calls in the same order. n % 8 == 0, n <= cap. Plain peer stores and loads only. */
MONO_API size_t mono_allreduce2_area_bytes(int64_t cap);
MONO_API int mono_p2p_area_alloc(size_t bytes, void** ptr_out);
MONO_API int mono_p2p_area_free(void* ptr);
MONO_API int mono_ipc_handle(void* ptr, void* handle_out, size_t handle_bytes);
MONO_API int mono_ipc_open(const void* handle, size_t handle_bytes, void** ptr_out);
MONO_API int mono_ipc_close(void* ptr);
MONO_API int mono_allreduce2_bf16(const void* in, void* out, int64_t n, void* my_area, void* peer_area, int64_t cap,
                                  unsigned* my_calls, mono_stream_t stream);

/* Exact top-k of a few long rows, k <= 64 (the reference's topk_rows, csrc/topk_rows.sycl:2-17: the verify
 * sampling's torch.topk(logits.float(), k)): per row the k largest by the radix key of the fp32 value (sign-flipped
 * bits: -0 below +0; rows holding NaN are not torch's order), sorted descending. Equal values come out in one of two
 * orders, by the 64-bit rank key << 32 | (0xFFFFFFFF - g):
 *   flags without MONO_TOPK_INDEX_ORDER: the reference platform's (torch-XPU) gather order, g = (i >> 15) << 15 |
 *     ((i % 4096) >> 2) << 5 | ((i % 32768) >> 12) << 2 | (i % 4) (csrc/topk_rows.sycl:34-42);
 *   MONO_TOPK_INDEX_ORDER: g = i, ascending index -- torch's CUDA topk order for k >= 33 and k = 1 (measured on
 *     B200; for 2 <= k <= 32 torch's order among equal values is its sorting network's and not reproduced).
 * x: fp32, or bf16 with MONO_TOPK_BF16 in flags, [rows][N]; values fp32 [rows][k], indices int64 [rows][k].
 * 1 <= rows <= 16, 64 <= N < 2^31. workspace: mono_topk_rows_workspace(rows, N) bytes. */
#define MONO_TOPK_BF16 1
#define MONO_TOPK_INDEX_ORDER 2
MONO_API size_t mono_topk_rows_workspace(int64_t rows, int64_t N);
MONO_API int mono_topk_rows(const void* x, int flags, int64_t rows, int64_t N, int64_t k, float* values, int64_t* indices,
                            void* workspace, size_t workspace_bytes, mono_stream_t stream);

/* ---- Layer programs: the reference's single-launch layers (layer_pre / layer_post, csrc/mono_layer.sycl:1-9;
 * layer_gdn, csrc/mono_gdn.sycl:5-20), generalised to any sequence of their phases ----
 * A program is an array of ops of mono_program_op_bytes() bytes each, filled on the host by the builders below
 * (op `index` of the array `ops`), planned once by mono_program_plan (which stores the shared-memory staging
 * choice in the ops) and run by mono_program_launch as ONE persistent cooperative kernel: its producer warps
 * stream the tiled GPTQ weights of every GEMV op in order (and `prefetch` items ahead into L2) while its
 * consumer warps run the ops; `barrier` != 0 puts a grid barrier after an op. M (rows) is the program's.
 * Arithmetic: each op is the same as the standalone entry it mirrors (mono_rowlin_gptq's row modes,
 * mono_w4a8_gptq_linear's GEMV, mono_mlp_gptq's SiLU pair and re-quantization, mono_gdn_step_deferred) and
 * gives the same bits. */
MONO_API size_t mono_program_op_bytes(void);
/* Barrier words of a launch: zero-filled once, left zero by every launch; one launch in flight per workspace. */
MONO_API size_t mono_program_workspace(void);
/* Rows op: for m < M, mode 0: xn = RMSNorm(x[m]; norm_w, eps); 1: y = bf16(x * lut[gate]) (gate element (m, c)
 * at gate[m * gate_row_stride + (c / 256) * gate_head_stride + c % 256]); 2: x; 3 (GDN gated norm): per
 * 128-wide head of the raw row x[m], core = bf16(bf16((raw * norm_w[d]) / sqrt(mean(raw^2) + eps)) *
 * bf16(silu(z))) with z element (m, c) at gate[m * gate_row_stride + c] (norm_w [128]); then q[m], s[m] =
 * act_quant of that row (xn_out, if not NULL: the normalized / core rows [M][K]). zero: 16 words set to 0, or
 * NULL. K a multiple of 1024 up to 4096; x row stride x_stride elements. */
MONO_API int mono_program_rows(void* ops, int index, int mode, const void* x, int64_t x_stride, int64_t K,
                               const void* norm_w, float eps, const void* gate, int64_t gate_row_stride,
                               int64_t gate_head_stride, const void* lut, void* xn_out, void* q, void* s, void* zero,
                               int barrier);
/* GEMV op: out[m][n] = bf16(GPTQ linear(q, s)) (+ residual: bf16(residual + that)) for nm (1..3) tiled
 * weights of rows[i] outputs, concatenated along n (row strides out_stride / residual_stride elements); or,
 * paired (nm = 2: gate, up of one shape), h = bf16(silu_lut[bf16(g s)] * bf16(u s)) to out and the row maxima
 * of |h| (float bits) into amax[m] (zeroed by an earlier rows op). q int8 [M][K] permuted (written by a rows or
 * quant op of the program), s [M]. */
MONO_API int mono_program_gemv(void* ops, int index, const void* const* weights, const int64_t* rows, int nm,
                               int paired, int64_t K, const void* q, const void* s, void* out, int64_t out_stride,
                               const void* residual, int64_t residual_stride, const void* silu_lut, void* amax,
                               int barrier);
/* Quant op: q[m], s[m] = quantization of h [M][K] bf16 with s = amax[m] / 127 (the paired GEMV's maxima). */
MONO_API int mono_program_quant(void* ops, int index, const void* h, int64_t K, const void* amax, void* q, void* s,
                                int barrier);
/* a | b op (the GDN gates' bf16 projection, mono_gdn_ab's arithmetic): out [M][N] = x [M][K] w^T. */
MONO_API int mono_program_ab(void* ops, int index, const void* x, int64_t x_stride, int64_t K, const void* w,
                             int64_t N, void* out, int barrier);
/* GDN op: delta = 0: the conv + gates step; delta = 1: the replay + verify delta rule, raw outputs bf16(o) to
 * raw [M][HV * 128] (the gated norm is a rows op, mode 3). Operands as mono_gdn_step_deferred (ctl NULL: the
 * committing form); the two ops of one step share `workspace` (mono_gdn_step_workspace bytes). HV <= 32. */
MONO_API int mono_program_gdn(void* ops, int index, int delta, const void* qkv, const void* z, const void* a,
                              const void* b, const void* conv_w, void* conv_state, const float* dt_bias,
                              const float* g_decay, float* state, const void* gnorm_w, float gnorm_eps, float qscale,
                              int64_t M, int64_t HK, int64_t HV, void* raw, const int32_t* ctl, const void* prev_qkv,
                              const void* prev_a, const void* prev_b, void* save_qkv, void* save_a, void* save_b,
                              int64_t qkv_stride, int64_t z_stride, int64_t ab_stride, void* workspace,
                              size_t workspace_bytes, int barrier);
/* Checks the ops and plans the launch for M rows (1..16); call before copying the ops to the device. */
MONO_API int mono_program_plan(void* ops, int nops, int64_t M);
/* Runs a planned program. ops: the host array; ops_device: the same bytes in device memory (16-byte aligned),
 * or NULL to pass up to 16 ops by value. prefetch: L2 look-ahead in weight items per producer warp (0 = none).
 * Every buffer an op names must stay valid until the launch completes. */
MONO_API int mono_program_launch(const void* ops, const void* ops_device, int nops, int64_t M, void* workspace,
                                 int prefetch, mono_stream_t stream);

/* The GDN gates' a | b projection (the reference's in_proj_a / in_proj_b BF16 linear, csrc/mono_gdn.sycl:10-11):
 * out[m][n] = bf16(sum_k x[m][k] w[n][k]) in fp32 with every product and sum rounded on its own: K is cut into
 * 4 quarters; for quarter q, lane l of 32 sums its 8-element pieces l + 32 j (j ascending over the quarter's
 * 256-wide slices, elements in order) from +0, then the xor butterfly (16, 8, 4, 2, 1) gives Q_q; out =
 * bf16(((Q_0 + Q_1) + Q_2) + Q_3). x bf16 [M][K] (row stride x_stride), w bf16 [N][K], out bf16 [M][N];
 * K % 1024 == 0, K <= 4096, M <= 32. */
MONO_API int mono_gdn_ab(const void* x, int64_t x_stride, const void* w, int64_t K, int64_t M, int64_t N, void* out,
                         mono_stream_t stream);

/* layer_post (csrc/mono_layer.sycl:243-313) in one launch: y' = gate ? bf16(y * sigmoid_lut[gate]) : y (gate
 * element (m, c) as the rows op, mode 1), x1 = bf16(x + GPTQ linear(act_quant(y'); o_w)), out = bf16(x1 +
 * down(quant(h))), h = silu(gate_w(q1)) * up_w(q1), q1 = act_quant(RMSNorm(x1; norm_w, eps)) — the bits of
 * mono_rowlin_gptq (mode gate / quant, residual x) followed by mono_mlp_gptq (residual). y bf16 [M][K] (K a
 * multiple of 1024 up to 4096), x / out bf16 [M][H] (out may alias x). workspace:
 * mono_layer_post_gptq_workspace(K, H, I) bytes, zero-filled before its first use. */
MONO_API size_t mono_layer_post_gptq_workspace(int64_t K, int64_t H, int64_t I);
MONO_API int mono_layer_post_gptq(const void* x, const void* y, int64_t K, const void* gate, int64_t gate_row_stride,
                                  int64_t gate_head_stride, const void* sig_lut, const void* o_w, const void* norm_w,
                                  float eps, const void* gate_w, const void* up_w, const void* down_w,
                                  const void* silu_lut, int64_t M, int64_t H, int64_t I, void* out, void* workspace,
                                  size_t workspace_bytes, mono_stream_t stream);

/* layer_gdn (csrc/mono_gdn.sycl:5-20) in one launch: xn = RMSNorm(x; norm_in), proj | z = W4(act_quant(xn);
 * qkv_w, z_w), a | b = mono_gdn_ab(xn; wab [2 HV][H]), the deferred GDN step (mono_gdn_step_deferred operands;
 * ctl NULL: committing), core = the gated norm (rows op mode 3), then x1 = x + W4(act_quant(core); out_w) and the
 * MLP block with norm_post (as mono_layer_post_gptq). 1 <= M <= 8; HV * 128 a multiple of 1024 up to 4096.
 * workspace: mono_layer_gdn_gptq_workspace(M, H, I, HK, HV) bytes, zero-filled before its first use. */
MONO_API size_t mono_layer_gdn_gptq_workspace(int64_t M, int64_t H, int64_t I, int64_t HK, int64_t HV);
MONO_API int mono_layer_gdn_gptq(const void* x, const void* norm_in, float eps_in, const void* qkv_w, const void* z_w,
                                 const void* wab, const void* conv_w, void* conv_state, const float* dt_bias,
                                 const float* g_decay, float* state, const void* gnorm_w, float gnorm_eps, float qscale,
                                 const int32_t* ctl, const void* prev_qkv, const void* prev_a, const void* prev_b,
                                 void* save_qkv, void* save_a, void* save_b, const void* out_w, const void* norm_post,
                                 float eps_post, const void* gate_w, const void* up_w, const void* down_w,
                                 const void* silu_lut, int64_t M, int64_t H, int64_t I, int64_t HK, int64_t HV,
                                 void* out, void* workspace, size_t workspace_bytes, mono_stream_t stream);

#ifdef __cplusplus
}
#endif
#endif /* MONO_B200_H */
