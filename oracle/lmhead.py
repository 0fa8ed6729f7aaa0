"""bf16 lm_head logits in the GEMV's pinned order, and the fused pick, on the CPU (test infrastructure only; see
oracle/__init__.py).

The kernel (comfy-mono-decode-xpu_b200/csrc/lmhead.cu, the same order as csrc/gemv_bf16.cu) forms logit (m, n) as:
lane l of 32 takes the 8-element pieces l, l + 32, ... of the K axis in order and accumulates x[m][k] * w[n][k]
element by element from +0 (fmaf: a bf16 x bf16 product is exact in fp32, so fmaf rounds only the sum, as a
float32 addition does here); then the xor butterfly over the lanes (16, 8, 4, 2, 1); then bf16 (round to nearest
even). The pick is the reference's greedy / draft choice (csrc/draft_lmhead.sycl:4-17) on those logits: argmax by
the argmax rank, top-k by the top-k rank (oracle/topk.py: the reference's tie orders)."""
from __future__ import annotations

import numpy as np

from . import topk as otk
from .numerics import bf16_bits_to_f32, f32_to_bf16_bits


def logits(x_bits: np.ndarray, w_bits: np.ndarray, block: int = 8192) -> np.ndarray:
    """x bf16 bits [M, K], w bf16 bits [V, K] (K % 256 == 0). Returns bf16 bits [M, V]."""
    x = bf16_bits_to_f32(np.asarray(x_bits)).astype(np.float32)
    M, K = x.shape
    V = w_bits.shape[0]
    J = K // 256
    xr = x.reshape(M, J, 32, 8)  # [m][piece row j][lane][element]
    out = np.empty((M, V), dtype=np.uint16)
    lanes = np.arange(32)
    for v0 in range(0, V, block):
        w = bf16_bits_to_f32(np.asarray(w_bits[v0:v0 + block])).astype(np.float32)
        wr = w.reshape(-1, J, 32, 8)
        acc = np.zeros((M, wr.shape[0], 32), dtype=np.float32)
        for j in range(J):
            for e in range(8):
                acc = (acc + xr[:, None, j, :, e] * wr[None, :, j, :, e]).astype(np.float32)
        for o in (16, 8, 4, 2, 1):
            acc = (acc + acc[:, :, lanes ^ o]).astype(np.float32)
        out[:, v0:v0 + wr.shape[0]] = f32_to_bf16_bits(acc[:, :, 0])
    return out


def pick(x_bits, w_bits, k: int):
    """(logits bits [M, V], argmax [M] int64, top-k indices [M, k] int64) of the fused lm_head pick."""
    lg = logits(x_bits, w_bits)
    am = otk.argmax(lg)
    top = otk.topk(lg, k)[1] if k > 0 else np.zeros((lg.shape[0], 0), dtype=np.int64)
    return lg, am, top


def draft_scatter(am: int, top, children, dst):
    """The pick form's scatter into the verify-token row: dst[children[0]] = argmax, dst[children[j]] = top[j]."""
    for j, c in enumerate(children):
        if c < 0:
            break
        dst[c] = am if j == 0 or j >= len(top) else top[j]
    return dst
