"""The fused bf16 lm_head pick on the CPU (test infrastructure only; see oracle/__init__.py).

The kernel (comfy-mono-decode-xpu_b200/csrc/lmhead.cu) forms the logits on the tensor cores: fp32 accumulation over
a fixed partition of K, rounded once to bf16. Tensor-core accumulation is not an IEEE sequence of additions, so the
logits are checked against the exact dot products (logits_exact, fp64: bf16 x bf16 products and their sums of 4096
terms are exact there up to a relative 2^-40) within the tolerance `tolerance` states, and the pick is checked bit
for bit on the kernel's own logits: argmax by the argmax rank, top-k by the top-k rank (oracle/topk.py, the
reference's tie orders; csrc/draft_lmhead.sycl:4-17 for the draft pick)."""
from __future__ import annotations

import numpy as np

from . import topk as otk
from .numerics import bf16_bits_to_f32


def logits_exact(x_bits: np.ndarray, w_bits: np.ndarray) -> tuple:
    """(x W^T, |x| |W|^T) in fp64 for x bf16 bits [M, K], w bf16 bits [V, K]."""
    x = bf16_bits_to_f32(np.asarray(x_bits)).astype(np.float64)
    w = bf16_bits_to_f32(np.asarray(w_bits)).astype(np.float64)
    return x @ w.T, np.abs(x) @ np.abs(w).T


def tolerance(exact: np.ndarray, abs_sum: np.ndarray) -> np.ndarray:
    """The bound on |logit - exact|: one bf16 rounding (2^-8 relative, with margin) plus the fp32 accumulation of the
    partition (at most ~600 dependent additions per sum: 2^-12 of the sum of |terms| is 8x that bound)."""
    return 2.0 ** -8 * np.abs(exact) + 2.0 ** -12 * abs_sum + 1e-30


def pick_logits(lg_bits: np.ndarray, k: int):
    """(argmax [M] int64, top-k indices [M, k] int64) of bf16 logits [M, V]: the kernel's pick on its own logits."""
    lg = np.asarray(lg_bits)
    am = otk.argmax(lg)
    top = otk.topk(lg, k)[1] if k > 0 else np.zeros((lg.shape[0], 0), dtype=np.int64)
    return am, top


def draft_scatter(am: int, top, children, dst):
    """The pick form's scatter into the verify-token row: dst[children[0]] = argmax, dst[children[j]] = top[j]."""
    for j, c in enumerate(children):
        if c < 0:
            break
        dst[c] = am if j == 0 or j >= len(top) else top[j]
    return dst
