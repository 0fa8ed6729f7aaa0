"""Full-attention decode layer pieces on the CPU (test infrastructure only; see oracle/__init__.py).

* qk_norm_rope_kv: per-head RMSNorm (head dim 256) with this build's pinned order, then the partial split-half
  RoPE of csrc/rope_kv.sycl:7-9 / :46-52 and tests/test_rope_kv.py:9-23 (each product rounded to fp32 on its
  own, the sum rounded once to bf16), and the K/V cache write at the given positions (csrc/rope_kv.sycl:100-113).
* attention_fp64: decode attention of the tree rows over the prefix [0, L) of the cache plus the tree rows a
  row's mask admits, in fp64 (the reference's own known-answer, tests/test_attn_dpas.py:11-29).
* tree_mask: mask[r] = mask[parent[r]] | 1 << r (tests/test_attn_dpas.py:11-15).
"""
from __future__ import annotations

import numpy as np

from .numerics import bf16_bits_to_f32, f32_to_bf16_bits

F32 = np.float32
HD = 256


def tree_mask(parents):
    """Ancestor bitmask of every tree row (parents[r] < r, -1 for the root)."""
    m = []
    for r, p in enumerate(parents):
        m.append((m[p] if p >= 0 else 0) | (1 << r))
    return m


def head_rmsnorm(x_bits: np.ndarray, w_bits: np.ndarray, eps: float) -> np.ndarray:
    """RMSNorm over the last axis (256) with the pinned order of the kernel: lane l of a warp holds elements
    8l .. 8l + 7 and sums their squares in order from +0 (each product and sum rounded to fp32), the 32 lane
    sums meet in an xor butterfly (16, 8, 4, 2, 1), r = 1 / sqrt(total / 256 + eps) (IEEE division and square
    root), out = bf16((x * r) * w). The role of the reference's q_norm / k_norm (csrc/rope_kv.sycl:188-216,
    whose reduction trees are the Intel build's own)."""
    x = bf16_bits_to_f32(x_bits).astype(F32)
    lead = x.shape[:-1]
    sq = (x * x).astype(F32).reshape(*lead, 32, 8)
    lanes = np.zeros((*lead, 32), dtype=F32)
    for e in range(8):
        lanes = (lanes + sq[..., e]).astype(F32)
    a = lanes
    while a.shape[-1] > 1:
        h = a.shape[-1] // 2
        a = (a[..., :h] + a[..., h:]).astype(F32)
    tot = a[..., 0]
    v = ((tot / F32(HD)).astype(F32) + F32(eps)).astype(F32)
    r = (F32(1.0) / np.sqrt(v).astype(F32)).astype(F32)
    return f32_to_bf16_bits(((x * r[..., None]).astype(F32) * bf16_bits_to_f32(w_bits).astype(F32)).astype(F32))


def rope(t_bits: np.ndarray, freqs: np.ndarray, rd: int) -> np.ndarray:
    """Partial split-half RoPE on the first rd lanes of the last axis. t_bits [S, H, 256] bf16 bits, freqs
    [S, rd/2, 2, 2] fp32 ([[f00, f01], [f10, f11]] per pair):
        o0 = t[j] * f00 + t[j + half] * f01,  o1 = t[j + half] * f11 + t[j] * f10
    products rounded to fp32 separately (no fused multiply-add), sum rounded once to bf16."""
    half = rd // 2
    t = bf16_bits_to_f32(t_bits).astype(F32)
    lo, hi = t[..., :half], t[..., half:rd]
    f = freqs.astype(F32)
    f00, f01 = f[:, None, :, 0, 0], f[:, None, :, 0, 1]
    f10, f11 = f[:, None, :, 1, 0], f[:, None, :, 1, 1]
    o0 = ((lo * f00).astype(F32) + (hi * f01).astype(F32)).astype(F32)
    o1 = ((hi * f11).astype(F32) + (lo * f10).astype(F32)).astype(F32)
    out = t_bits.copy()
    out[..., :half] = f32_to_bf16_bits(o0)
    out[..., half:rd] = f32_to_bf16_bits(o1)
    return out


def qk_norm_rope_kv(rawq, rawk, v, wq, wk, freqs, key, value, pos, epsq, epsk, rd):
    """rawq [S, Hq, 256], rawk / v [S, Hk, 256] bf16 bits; key / value caches [Hk, cap, 256] bf16 bits (updated in
    place); pos [S] int. Returns (q [Hq, S, 256], k [Hk, S, 256]) bf16 bits."""
    q = rope(head_rmsnorm(rawq, wq, epsq), freqs, rd)
    k = rope(head_rmsnorm(rawk, wk, epsk), freqs, rd)
    for s, p in enumerate(pos):
        key[:, p] = k[s]
        value[:, p] = v[s]
    return np.ascontiguousarray(q.transpose(1, 0, 2)), np.ascontiguousarray(k.transpose(1, 0, 2))


def attention_fp64(q, key, value, L, xk, xv, mask):
    """q [H, S, 256], key / value [Hk, cap, 256], xk / xv [Hk, S, 256] (bf16 bits); mask [S] ints or None (the
    single draft row: prefix only). Returns fp64 [S, H * 256]: per q head h (kv head h / (H / Hk)),
    softmax over the prefix [0, L) and the admitted tree rows of (K . q) / 16, times V."""
    qf, kf, vf = (bf16_bits_to_f32(a).astype(np.float64) for a in (q, key, value))
    xkf, xvf = bf16_bits_to_f32(xk).astype(np.float64), bf16_bits_to_f32(xv).astype(np.float64)
    H, S = qf.shape[0], qf.shape[1]
    Hk = kf.shape[0]
    out = np.zeros((S, H * HD), dtype=np.float64)
    for h in range(H):
        kh = h // (H // Hk)
        for s in range(S):
            rows = [t for t in range(S) if mask is not None and (mask[s] >> t) & 1]
            K = np.concatenate([kf[kh, :L], xkf[kh, rows]])
            V = np.concatenate([vf[kh, :L], xvf[kh, rows]])
            if K.shape[0] == 0:
                continue
            sc = K @ qf[h, s] / 16.0
            p = np.exp(sc - sc.max())
            out[s, h * HD:(h + 1) * HD] = (p / p.sum()) @ V
    return out
