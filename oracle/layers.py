"""Row operations and the fused blocks on the CPU (test infrastructure only; see oracle/__init__.py)."""
from __future__ import annotations

import numpy as np

from .numerics import bf16_bits_to_f32, f32_to_bf16_bits
from .w4a8 import act_quant, gptq_linear

F32 = np.float32


def _butterfly32(a: np.ndarray) -> np.ndarray:
    """Sum over the last axis (32 lanes) in xor-shuffle order: halves 16, 8, 4, 2, 1."""
    while a.shape[-1] > 1:
        h = a.shape[-1] // 2
        a = (a[..., :h] + a[..., h:]).astype(F32)
    return a[..., 0]


def rmsnorm(x_bits: np.ndarray, w_bits: np.ndarray, eps: float) -> np.ndarray:
    """RMSNorm with the pinned order of the fused kernels (include/mono_b200.h mono_mlp_gptq): thread t of 128
    sums the squares of its 8-element pieces t + 128 j (j outer, element inner, from +0), butterfly within
    each 32, the 4 warp sums in order, r = 1 / sqrt(total / H + eps), out = bf16((x * r) * w).
    The role of csrc/mono_common.hpp:452-505 (whose reduction order is the Intel build's)."""
    x = bf16_bits_to_f32(x_bits).astype(F32)
    M, H = x.shape
    sq = (x * x).astype(F32).reshape(M, H // 1024, 128, 8)  # [m, j, t, e]
    P = np.zeros((M, 128), dtype=F32)
    for j in range(H // 1024):
        for e in range(8):
            P = (P + sq[:, j, :, e]).astype(F32)
    W = _butterfly32(P.reshape(M, 4, 32))  # [M, 4]
    tot = np.zeros(M, dtype=F32)
    for w in range(4):
        tot = (tot + W[:, w]).astype(F32)
    v = ((tot / F32(H)).astype(F32) + F32(eps)).astype(F32)
    r = (F32(1.0) / np.sqrt(v).astype(F32)).astype(F32)
    return f32_to_bf16_bits(((x * r[:, None]).astype(F32) * bf16_bits_to_f32(w_bits)[None, :]).astype(F32))


def silu_mul(g_bits: np.ndarray, u_bits: np.ndarray, lut_bits: np.ndarray) -> np.ndarray:
    """h = bf16(silu_lut[g] * u) (csrc/mono_layer.sycl:289-291, csrc/mono_mlp.sycl:136-138)."""
    return f32_to_bf16_bits((bf16_bits_to_f32(lut_bits[g_bits.astype(np.int64)]) * bf16_bits_to_f32(u_bits)).astype(F32))


def mlp_gptq(x_bits, norm_w_bits, eps, gate, up, down, lut_bits, residual=True):
    """The fused GPTQ MLP block (include/mono_b200.h mono_mlp_gptq); gate/up/down = (packed, scales)."""
    xn = rmsnorm(x_bits, norm_w_bits, eps) if norm_w_bits is not None else x_bits
    q1, s1 = act_quant(xn)
    g = gptq_linear(q1, s1, *gate)
    u = gptq_linear(q1, s1, *up)
    h = silu_mul(g, u, lut_bits)
    q2, s2 = act_quant(h)
    return gptq_linear(q2, s2, *down, residual=x_bits if residual else None)
