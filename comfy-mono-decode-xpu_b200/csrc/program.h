// Layer programs: a list of ops that one persistent cooperative launch runs in order, with a grid barrier of the
// consumer warps after every op that asks for one. The producer warps stream the W4 weights of every GEMV op of
// the list through the CTA's ring from the start (and, ahead of that, into L2), across the row phases, the
// Gated-DeltaNet phases and the barriers between them. This is the reference's single-launch layer kernels
// (layer_pre / layer_post / layer_gdn, csrc/mono_layer.sycl and csrc/mono_gdn.sycl: phases separated by
// device-wide barriers, every work-group resident), generalised so that one launch may also span several layers.
#pragma once
#include "launch.h"

namespace mono {

enum OpKind : int {
    OP_ROWS = 1,      // per row m < M (one warp-group): norm / gate / plain / GDN gated-norm, then quantization
    OP_GEMV = 2,      // W4A8 GPTQ GEMV of the quantized rows by up to three matrices (or a gate | up pair)
    OP_QUANT = 3,     // quantization of h [M][K] with the row maxima of a paired GEMV
    OP_AB = 4,        // bf16 a | b projection of the normalized rows (GDN gates)
    OP_GDN_CONV = 5,  // GDN conv + gates (gdn_conv_item over every channel)
    OP_GDN_DELTA = 6, // GDN replay + verify delta rule; raw outputs to `core` (the gated norm is an OP_ROWS)
};
enum RowsMode : int { ROWS_NORM = 0, ROWS_GATE = 1, ROWS_QUANT = 2, ROWS_GDN = 3 };

struct OpRows {
    const uint16_t* x;       // [M] rows of K, row stride x_stride (GDN: the raw delta outputs)
    const uint16_t* norm_w;  // NORM: [K]; GDN: [128] gated-norm weight
    const uint16_t* gate;    // GATE: element (m, c) at gate[m * gate_row_stride + (c / 256) * gate_head_stride + c % 256]
                             // GDN: z, element (m, c) at gate[m * gate_row_stride + c]
    const uint16_t* lut;     // GATE: sigmoid of every bf16 pattern
    uint16_t* xn_out;        // NORM / GDN: the normalized (core) rows [M][K], or null
    int8_t* q;               // [M][K] permuted
    float* s;                // [M]
    unsigned* zero;          // 16 words zeroed by this op (row maxima of a later paired GEMV), or null
    int64_t x_stride, gate_row_stride, gate_head_stride;
    float eps;
    int mode, K;
};
struct OpGemv {
    PhaseDesc ph;              // matrices (TILED GPTQ), K, x = the quantized rows [M][K] (permuted), paired
    const float* xs;           // [M] row scales of x
    uint16_t* out;             // bf16 [M][out_stride]; matrices concatenated along n (paired: h = silu(g) * u)
    const uint16_t* residual;  // [M][res_stride] or null (not paired)
    const uint16_t* lut;       // paired: silu of every bf16 pattern
    unsigned* amax;            // paired: row maxima of |h| (zeroed by an earlier op)
    int64_t out_stride, res_stride;
};
struct OpQuant {
    const uint16_t* h;     // [M][K]
    const unsigned* amax;  // [M] float bits
    int8_t* q;             // [M][K] permuted
    float* s;              // [M]
    int K;
};
struct OpAb {
    const uint16_t* x;  // normalized rows [M][K] (stride x_stride)
    const uint16_t* w;  // [N][K] bf16
    uint16_t* out;      // [M][N]
    int64_t x_stride;
    int K, N;
};
struct Op {
    int kind, barrier;  // barrier: a grid barrier of the consumer warps follows the op
    union {
        OpRows r;
        OpGemv g;
        OpQuant q;
        OpAb ab;
        GdnArgs gdn;  // OP_GDN_CONV / OP_GDN_DELTA (DELTA writes the raw bf16 outputs to gdn.core, [M][HV * 128])
    };
};

constexpr int kProgParamOps = 16;  // ops passed by value (the one-layer entry points)

// Plans the launch (shared-memory shape; activation staging per GEMV op, stored in the ops) and checks the ops.
int plan_program(Op* ops, int nops, int M);
// ops_host: the planned ops; ops_dev: the same bytes in device memory, or null to pass them by value
// (nops <= kProgParamOps). bar: two zeroed words (zero again after the launch). prefetch: L2 look-ahead in
// items per producer warp (0: none).
int launch_program(const Op* ops_host, const Op* ops_dev, int nops, int M, unsigned* bar, int prefetch,
                   cudaStream_t stream);

}  // namespace mono
