// Argument blocks and launchers shared by the C-ABI entry points and the kernel translation units.
#pragma once
#include "abi_internal.h"
#include "engine.cuh"

namespace mono {

// Shared bytes after the staged rows for the fused quantization: 16 row scales + 8 reduction floats per
// warp-group.
constexpr int kQuantExtra = 256;
// Rows of the fused MLP and the row linear (the verify rows of up to 4 batched decode streams); their
// workspaces hold this many rows.
constexpr int kStreamMaxRows = 32;

struct LinearEpi {
    const uint16_t* xb;      // bf16 activations [M][K]: quantized per token inside the kernel (xs unused), or null
    const float* xs;         // [M]
    const float* s_channel;  // REF: [N]
    const void* residual;    // [M][N] output dtype, or null
    void* out;               // [M][N]
    int out_bf16;
    int max_items;
};
int launch_linear(int fmt, int layout, Program& P, LinearEpi& E, cudaStream_t stream);

struct MlpArgs {
    const uint16_t* x;       // [M][H] bf16
    const uint16_t* norm_w;  // [H] bf16 or null
    const uint16_t* lut;     // [65536] bf16: silu of every bf16 pattern
    uint16_t* out;           // [M][H] bf16
    float eps;
    int H, I, residual, max_items;
    // workspace
    int8_t* q1;       // [M][H]
    float* s1;        // [kStreamMaxRows]
    uint16_t* h;      // [M][I]
    unsigned* amax2;  // [kStreamMaxRows] (float bits of non-negative values; zero between launches)
    int8_t* q2;       // [M][I] (only when the down phase's activations are not staged in shared memory)
    unsigned* bar;    // [2] grid barrier words (zero between launches)
};
// Shared-memory shape of a cooperative stream kernel: ring stages, partial bytes, staged-activation bytes.
struct MlpShape {
    int S;
    int part_bytes;  // partials of the larger phase's batch
    int x_bytes;     // staged activations of the larger staged phase
    int tb0, tb1;    // tiles per batch of phase 0 and 1 (the partials of a batch fit part_bytes)
};
int launch_mlp(Program& P, MlpArgs& A, cudaStream_t stream);

enum RowLinMode : int { ROWLIN_NORM = 0, ROWLIN_GATE = 1, ROWLIN_QUANT = 2 };
struct RowLinArgs {
    const uint16_t* x;  // [M][K] bf16
    const uint16_t* norm_w;
    float eps;
    const uint16_t* gate;  // GATE: element (m, c) at gate[m * gate_row_stride + (c / 256) * gate_head_stride + c % 256]
    int64_t gate_row_stride, gate_head_stride;
    const uint16_t* lut;  // GATE: sigmoid of every bf16 pattern
    const uint16_t* residual;  // [M][N] or null
    uint16_t* out;             // [M][N]
    uint16_t* xn_out;          // NORM: normalized rows [M][K], or null
    int8_t* q;                 // workspace [kStreamMaxRows][K]
    float* s;                  // workspace [kStreamMaxRows]
    unsigned* bar;             // workspace [2], zero between launches
    int mode, N;
    // NORM with xn_out: the GDN a | b projection of the normalized rows (gdn.cuh gdn_ab_quarter order), column c
    // by CTA gridDim.x - 1 - c after its GEMV tiles: ab_out[m * ab_stride + c] for c < ab_n (null: none)
    const uint16_t* ab_w;  // [ab_n][K] bf16
    uint16_t* ab_out;
    int ab_n;
    int64_t ab_stride;
};
size_t rowlin_workspace_bytes(int K);
int launch_rowlin(Program& P, RowLinArgs& A, cudaStream_t stream);
size_t mlp_workspace_bytes(int H, int I);

int launch_repack(int fmt, const void* q, const void* s, int N, int K, void* out, cudaStream_t stream);
size_t tiled_bytes(int fmt, int64_t N, int64_t K);
int launch_pair_table(const float* codebook, uint16_t* tab, cudaStream_t stream);
int launch_act_quant(const void* x, int M, int K, int8_t* q, float* xs, cudaStream_t stream);
size_t rot_quant_workspace(int M, int K);
int launch_rot_quant(const void* x, const void* h, int M, int K, int8_t* q, float* s, void* ws, cudaStream_t stream);
int launch_rot_quant_noalloc(const void* x, const void* h, int M, int K, int8_t* q, float* s, cudaStream_t stream);

struct NormRopeArgs {
    const uint16_t* q;  // [S][Hq] heads, row stride qs, head stride qh (elements)
    const uint16_t* k;  // [S][Hk][256], row stride ks
    const uint16_t* v;  // [S][Hk][256], row stride vs
    const uint16_t* wq;
    const uint16_t* wk;
    const float* freqs;  // [S][rd/2][2][2]
    uint16_t* kc;        // [Hk][cap][256]
    uint16_t* vc;
    const int64_t* pos;
    uint16_t* oq;  // [streams][Hq][S / streams][256]
    uint16_t* ok;  // [streams][Hk][S / streams][256]
    int64_t qs, qh, ks, vs, cap;
    int S, Hq, Hk, rd;
    int streams;   // batched streams: S / streams rows each, caches [streams][Hk][cap][256]
    float epsq, epsk;
};
int launch_qk_norm_rope_kv(const NormRopeArgs& A, cudaStream_t stream);

struct AttnArgs {
    const uint16_t* q;    // [H][S][256]
    const uint16_t* kc;   // [Hk][cap][256]
    const uint16_t* vc;
    const int32_t* seqlen;
    const uint16_t* xk;   // [Hk][S][256]
    const uint16_t* xv;   // element (stream b, kv head k of the stream, row t) at b xv_bs + k xv_hs + t xv_rs
    int64_t xv_bs, xv_hs, xv_rs;
    const int32_t* mask;  // [S] or null
    uint16_t* out;        // [streams][S][H / streams * 256]
    float* part;          // workspace: [Hk][chunks / 8][32][256] merged rows of each cluster
    float* ml;            // [Hk][chunks / 8][32][2]
    unsigned* count;      // [Hk][8] arrivals per (kv head, cluster rank); zero between launches
    int H, Hk, S, cap, chunks;  // H, Hk: all streams' heads (stream b: q heads [b H / streams, ...), its kv heads)
    int streams;                // seqlen[b]: stream b's committed length
};
size_t attn_workspace_bytes(int Hk, int streams, int cap, int sms);
int launch_tree_attention(AttnArgs A, void* ws, cudaStream_t stream);

struct GdnArgs {
    const uint16_t* qkv;     // [M][C] projections: q heads | k heads | v heads (bf16)
    const uint16_t* z;       // [M][HV * 128]
    const uint16_t* a;       // [M][HV]
    const uint16_t* b;       // [M][HV]
    const uint16_t* conv_w;  // [C][4]
    uint16_t* conv_state;    // [C][3], updated
    const float* dt_bias;    // [HV]
    const float* g_decay;    // [HV]
    float* state;            // [HV][128][128] ([k][v]), updated
    const uint16_t* gnorm_w; // [128]
    float gnorm_eps, qscale;
    uint16_t* core;          // [M][HV * 128]
    uint16_t* conv_out;      // workspace [8 + M][C]
    float* gates;            // workspace [8 + M][HV][2]
    // deferred form (ctl != null): replay ctl[0] rows of the previous step (slots ctl[2 + i]) from prev_*,
    // save this step's inputs to save_* (which must not alias prev_*)
    const int32_t* ctl;
    const uint16_t* prev_qkv;  // [8][C]
    const uint16_t* prev_a;    // [8][HV]
    const uint16_t* prev_b;
    uint16_t* save_qkv;
    uint16_t* save_a;
    uint16_t* save_b;
    int64_t qkv_stride, z_stride, ab_stride;  // row strides (elements) of qkv, z, a / b
    int M, C, HK, HV;
    // batched streams (grid y): stream b's rows are [b M, (b + 1) M) of qkv / z / a / b / core; its conv state,
    // recurrent state, ctl (ctl_stride words apart), replay / save buffers and workspace rows are the b-th of
    // `streams` consecutive copies (gdn_stream)
    int streams, ctl_stride;
};
size_t gdn_workspace_bytes(int M, int C, int HV, int streams);
// Validates the GDN step's operands and fills A (workspace: gdn_workspace_bytes; conv_out and gates in it).
int fill_gdn_args(GdnArgs& A, const void* qkv, const void* z, const void* a, const void* b, const void* conv_w,
                  void* conv_state, const float* dt_bias, const float* g_decay, float* state, const void* gnorm_w,
                  float gnorm_eps, float qscale, int64_t M, int64_t HK, int64_t HV, void* core, void* workspace,
                  size_t workspace_bytes, const int32_t* ctl, const void* prev_qkv, const void* prev_a,
                  const void* prev_b, void* save_qkv, void* save_a, void* save_b, int64_t qkv_stride,
                  int64_t z_stride, int64_t ab_stride);
int launch_gdn_step(GdnArgs A, void* ws, cudaStream_t stream);
// a | b projection (gdn.cuh gdn_ab_column): out[m][n] for n < N, one warp per column
int launch_gdn_ab(const uint16_t* x, int64_t x_stride, const uint16_t* w, int K, int M, int N, uint16_t* out,
                  int64_t out_stride, cudaStream_t stream);

struct TopkArgs {
    const uint16_t* x;  // [rows][V] bf16
    uint16_t* values;   // [rows][k]
    int64_t* indices;   // [rows][k]
    int64_t* argmax;    // [rows] (with_argmax)
    uint64_t* ws;       // [rows][slices][k + 1]
    int64_t V;
    int rows, k, argmax_order, with_argmax;
};
// the lm_head's bf16 ring kernel without the pick (lmhead.cu): out[m][n] = bf16(x[m] . w[n]) on the tensor cores
bool bf16_rows_fit(int M, int K);
int launch_bf16_rows(const uint16_t* x, int64_t x_stride, const uint16_t* w, int M, int N, int K, uint16_t* out,
                     int64_t out_stride, cudaStream_t stream);

size_t topk_workspace_bytes(int64_t rows);
int launch_topk(const TopkArgs& A, cudaStream_t stream);

}  // namespace mono
