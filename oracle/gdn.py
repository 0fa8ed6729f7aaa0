"""Gated-DeltaNet decode step on the CPU in fp64 (test infrastructure only; see oracle/__init__.py).

Follows the reference's arithmetic (csrc/mono_gdn.sycl) for M sequential rows (a chain: every row commits):
  conv   (:313-375)  y = bf16(sum_{d=0..3} x[t-d] * w[3-d]) with x[-1..-3] the conv state (newest last),
                     out = bf16(y / (1 + exp(-y)));  the conv state becomes the last 3 inputs
  gates  (:427-456)  decay = exp(g_decay[h] * softplus(a + dt_bias[h])) (softplus(v) = v for v > 20),
                     beta = bf16(sigmoid(b))
  l2     (:458-498)  qi = 1 / max(sqrt(sum q^2), 1e-12); q <- (q * scale) * qi; k <- k * ki  (per key head)
  delta  (:531-567)  S <- S * decay; mem = S^T k; delta = (v - mem) * beta; S <- S + k delta^T; o = S^T q
                     (S[h] is [k][v]; value head h reads key head h / (HV / HK))
  gnorm  (:574-607)  raw = bf16(o); core = bf16(bf16(raw * w * rsqrt(mean(raw^2) + eps)) * bf16(silu(z)))
Everything in fp64 except the bf16 roundings the reference makes explicit.
"""
from __future__ import annotations

import numpy as np

from .numerics import bf16_bits_to_f32, f64_to_bf16_bits

DH = 128


def _bf(x):
    """Round fp64 values to bf16 (RNE) and back to fp64."""
    return bf16_bits_to_f32(f64_to_bf16_bits(np.asarray(x, dtype=np.float64))).astype(np.float64)


def gdn_step(qkv, z, a, b, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, gnorm_eps, qscale, HK):
    """qkv [M, C] bf16 bits (C = 2 HK 128 + HV 128: q heads | k heads | v heads), z [M, HV 128], a / b [M, HV]
    bf16 bits; conv_w [C, 4] bf16 bits; conv_state [C, 3] bf16 bits; dt_bias / g_decay [HV] fp32; state
    [HV, 128, 128] fp32 ([k][v]); gnorm_w [128] bf16 bits.
    Returns (core [M, HV 128] fp64, conv_state' [C, 3] bf16 bits, state' [HV, 128, 128] fp64)."""
    x = bf16_bits_to_f32(qkv).astype(np.float64)
    M, C = x.shape
    HV = a.shape[1]
    KD = HK * DH
    w = bf16_bits_to_f32(conv_w).astype(np.float64)
    hist = bf16_bits_to_f32(conv_state).astype(np.float64)  # [C, 3], oldest first
    seq = np.concatenate([hist, x.T], axis=1)  # [C, 3 + M]
    conv = np.zeros((M, C))
    for t in range(M):
        win = seq[:, t:t + 4]  # x[t-3] .. x[t]
        s = np.zeros(C)
        for d in range(4):  # d steps back, weight w[3 - d]
            s = s + win[:, 3 - d] * w[:, 3 - d]
        y = _bf(s)
        conv[t] = _bf(y / (1.0 + np.exp(-y)))
    new_hist = seq[:, -3:]
    av = _bf(bf16_bits_to_f32(a).astype(np.float64)) + dt_bias.astype(np.float64)[None, :]
    sp = np.where(av > 20.0, av, np.log1p(np.exp(np.minimum(av, 20.0))))
    decay = np.exp(g_decay.astype(np.float64)[None, :] * sp)
    beta = _bf(1.0 / (1.0 + np.exp(-bf16_bits_to_f32(b).astype(np.float64))))
    q = conv[:, :KD].reshape(M, HK, DH)
    k = conv[:, KD:2 * KD].reshape(M, HK, DH)
    v = conv[:, 2 * KD:].reshape(M, HV, DH)
    qi = 1.0 / np.maximum(np.sqrt((q * q).sum(-1)), 1e-12)
    ki = 1.0 / np.maximum(np.sqrt((k * k).sum(-1)), 1e-12)
    qn = (q * qscale) * qi[..., None]
    kn = k * ki[..., None]
    S = state.astype(np.float64).copy()
    raw = np.zeros((M, HV, DH))
    for t in range(M):
        for h in range(HV):
            kh = h // (HV // HK)
            St = S[h] * decay[t, h]
            mem = St.T @ kn[t, kh]
            delta = (v[t, h] - mem) * beta[t, h]
            St = St + np.outer(kn[t, kh], delta)
            S[h] = St
            raw[t, h] = St.T @ qn[t, kh]
    rawb = _bf(raw)
    gw = bf16_bits_to_f32(gnorm_w).astype(np.float64)
    rs = 1.0 / np.sqrt((rawb * rawb).mean(-1, keepdims=True) + gnorm_eps)
    normed = _bf(rawb * gw * rs)
    zf = bf16_bits_to_f32(z).astype(np.float64).reshape(M, HV, DH)
    gz = _bf(zf / (1.0 + np.exp(-zf)))
    core = (normed * gz).reshape(M, HV * DH)
    return core, f64_to_bf16_bits(new_hist), S


def ab_projection(x_bits, w_bits):
    """The GDN gates' a | b projection in the kernel's pinned fp32 order (mono_gdn_ab; the role of the reference's
    in_proj_a / in_proj_b BF16 linear, csrc/mono_gdn.sycl:10-11): out[m][n] = bf16(sum_k x[m][k] w[n][k]) with every
    product and sum rounded to fp32 on its own. K is cut into 4 quarters of K / 1024 slices of 256; in quarter q,
    lane l of 32 sums its 8-element pieces l + 32 j (j ascending over the quarter's slices, elements in order)
    from +0, then the xor butterfly (16, 8, 4, 2, 1) gives Q_q; out = bf16(((Q_0 + Q_1) + Q_2) + Q_3). x bf16
    bits [M, K], w bf16 bits [N, K] (K % 1024 == 0). Returns bf16 bits [M, N]. Bit-exact by construction (numpy
    float32 rounds each operation to nearest even)."""
    from .numerics import f32_to_bf16_bits
    x = bf16_bits_to_f32(np.asarray(x_bits)).astype(np.float32)
    w = bf16_bits_to_f32(np.asarray(w_bits)).astype(np.float32)
    M, K = x.shape
    N, J = w.shape[0], K // 256
    J4 = J // 4
    xr, wr = x.reshape(M, J, 32, 8), w.reshape(N, J, 32, 8)
    lanes = np.arange(32)
    Q = []
    for q in range(4):
        acc = np.zeros((M, N, 32), dtype=np.float32)
        for j in range(q * J4, (q + 1) * J4):
            for e in range(8):
                acc = (acc + (xr[:, None, j, :, e] * wr[None, :, j, :, e]).astype(np.float32)).astype(np.float32)
        for o in (16, 8, 4, 2, 1):
            acc = (acc + acc[:, :, lanes ^ o]).astype(np.float32)
        Q.append(acc[:, :, 0])
    out = (((Q[0] + Q[1]).astype(np.float32) + Q[2]).astype(np.float32) + Q[3]).astype(np.float32)
    return f32_to_bf16_bits(out)


def gdn_step_tree(qkv, z, a, b, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, gnorm_eps, qscale, HK,
                  parents, prog, replay=None):
    """The deferred (replay + tree verify) form of the step (csrc/mono_gdn.sycl:38-40 ctl, :313-375 conv,
    :398-571 entries), in fp64 with the reference's bf16 roundings:
      replay   `replay` = (qkv, a, b) of the previous step's accepted rows, in path order: they run the committing
               chain (gdn_step) from (conv_state, state); the resulting conv state and recurrent state persist
      conv     verify row t reads its own input, then its ancestors' (parents[t], parents[parents[t]], ..., -1
               ends), then the committed history (the conv state after the replay), newest first
      delta    the program entries in order: entry p = slot | 32 * commit; the running state starts from the
               persisted one; a committing entry advances it, a non-committing one computes its row from
               temporaries (S * decay, then the rank-one update) and leaves it; the list ends at the first entry
               whose slot is negative or >= M
      output   core of the rows the program names; other rows have raw = 0
    Returns (core [M, HV 128], conv_state' [C, 3] bf16 bits, state' [HV, 128, 128] fp64): the persisted states."""
    M, C = np.asarray(qkv).shape
    HV = np.asarray(a).shape[1]
    KD = HK * DH
    if replay is not None and len(replay[0]):
        rq, ra, rb = replay
        rz = np.zeros((len(rq), HV * DH), dtype=np.uint16)
        _, hist_bits, S0 = gdn_step(rq, rz, ra, rb, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, gnorm_eps,
                                    qscale, HK)
    else:
        hist_bits, S0 = np.asarray(conv_state), state.astype(np.float64)
    x = bf16_bits_to_f32(qkv).astype(np.float64)
    w = bf16_bits_to_f32(conv_w).astype(np.float64)
    hist = bf16_bits_to_f32(hist_bits).astype(np.float64)  # [C, 3], oldest first
    conv = np.zeros((M, C))
    for t in range(M):
        taps, anc, miss = [x[t]], t, 0
        for d in range(1, 4):
            anc = parents[anc] if anc >= 0 else -1
            if anc is not None and 0 <= anc < t:
                taps.append(x[anc])
            else:
                anc = -1
                miss += 1
                taps.append(hist[:, 3 - miss])
        s = np.zeros(C)
        for d in range(4):  # newest first, weight w[3 - d]
            s = s + taps[d] * w[:, 3 - d]
        y = _bf(s)
        conv[t] = _bf(y / (1.0 + np.exp(-y)))
    av = _bf(bf16_bits_to_f32(a).astype(np.float64)) + dt_bias.astype(np.float64)[None, :]
    sp = np.where(av > 20.0, av, np.log1p(np.exp(np.minimum(av, 20.0))))
    decay = np.exp(g_decay.astype(np.float64)[None, :] * sp)
    beta = _bf(1.0 / (1.0 + np.exp(-bf16_bits_to_f32(b).astype(np.float64))))
    q = conv[:, :KD].reshape(M, HK, DH)
    k = conv[:, KD:2 * KD].reshape(M, HK, DH)
    v = conv[:, 2 * KD:].reshape(M, HV, DH)
    qi = 1.0 / np.maximum(np.sqrt((q * q).sum(-1)), 1e-12)
    ki = 1.0 / np.maximum(np.sqrt((k * k).sum(-1)), 1e-12)
    qn = (q * qscale) * qi[..., None]
    kn = k * ki[..., None]
    S = S0.copy()
    raw = np.zeros((M, HV, DH))
    for p in prog:
        if p < 0 or (p & 15) >= M:
            break
        t, commit = p & 15, bool(p & 32)
        for h in range(HV):
            kh = h // (HV // HK)
            St = S[h] * decay[t, h]
            mem = St.T @ kn[t, kh]
            delta = (v[t, h] - mem) * beta[t, h]
            St = St + np.outer(kn[t, kh], delta)
            raw[t, h] = St.T @ qn[t, kh]
            if commit:
                S[h] = St
    rawb = _bf(raw)
    gw = bf16_bits_to_f32(gnorm_w).astype(np.float64)
    rs = 1.0 / np.sqrt((rawb * rawb).mean(-1, keepdims=True) + gnorm_eps)
    normed = _bf(rawb * gw * rs)
    zf = bf16_bits_to_f32(z).astype(np.float64).reshape(M, HV, DH)
    gz = _bf(zf / (1.0 + np.exp(-zf)))
    core = (normed * gz).reshape(M, HV * DH)
    return core, np.asarray(hist_bits), S0


def chain_program(rows):
    """parents / program of a chain of `rows` verify rows (every entry commits), padded to 8 with -1."""
    parents = [r - 1 for r in range(rows)] + [-1] * (8 - rows)
    prog = [r | 32 for r in range(rows)] + [-1] * (8 - rows)
    return parents, prog


def tree_program(parents, rows):
    """The verify program of a tree whose branches off the first-child chain are leaves (the shape qwen35's
    tree_spec builds): walk the chain from the root; each chain node commits and is followed by its other
    children (leaves, not committed). Returns prog padded to 8 with -1. Raises ValueError for other shapes."""
    children = [[] for _ in range(rows)]
    for r in range(1, rows):
        p = parents[r]
        if not 0 <= p < r:
            raise ValueError(f"row {r}: parent {p} must precede it")
        children[p].append(r)
    prog, node = [], 0
    while True:
        prog.append(node | 32)
        kids = children[node]
        for leaf in kids[1:]:
            if children[leaf]:
                raise ValueError(f"row {leaf}: an off-chain node with children")
            prog.append(leaf)
        if not kids:
            break
        node = kids[0]
    if sorted(p & 15 for p in prog) != list(range(rows)):
        raise ValueError("the program does not cover every row")
    return prog + [-1] * (8 - len(prog))
