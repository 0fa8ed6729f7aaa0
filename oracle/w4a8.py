"""W4A8 linear and activation quantization on the CPU (test infrastructure only; see oracle/__init__.py).

bf16 tensors are carried as uint16 bit patterns so every rounding is explicit.
"""
from __future__ import annotations

import numpy as np
import torch

from .numerics import bf16_bits_to_f32, f32_to_bf16_bits, f64_to_bf16_bits, fp8e4m3_to_f32

CHUNK_K = 1024  # the GPTQ format's fp32 chunk (8 groups of 128)


def _int_dot(x: np.ndarray, w: np.ndarray) -> np.ndarray:
    """Exact int32-range dot products x [M, K] . w [N, K] -> int64 [M, N] (fp64 matmul of small integers
    is exact: every partial sum stays below 2^53)."""
    xt = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float64))
    wt = torch.from_numpy(np.ascontiguousarray(w, dtype=np.float64))
    return (xt @ wt.T).numpy().astype(np.int64)


def _group_dot(x: np.ndarray, w: np.ndarray, group: int) -> np.ndarray:
    """Per-group exact dots: x [M, K], w [N, K] -> int64 [M, N, K / group]."""
    M, K = x.shape
    N = w.shape[0]
    G = K // group
    xt = torch.from_numpy(np.ascontiguousarray(x, dtype=np.float64).reshape(M, G, group).transpose(1, 0, 2).copy())
    wt = torch.from_numpy(np.ascontiguousarray(w, dtype=np.float64).reshape(N, G, group).transpose(1, 2, 0).copy())
    return torch.bmm(xt, wt).numpy().transpose(1, 2, 0).astype(np.int64)


def _finish(f: np.ndarray, residual, out_bf16: bool):
    """Output cast with the reference's residual rule (csrc/w4a8_decode.sycl:155-163):
    out = cast(float(residual) + float(cast(f)))."""
    f = np.asarray(f, dtype=np.float32)
    if out_bf16:
        r = f32_to_bf16_bits(f)
        if residual is not None:
            r = f32_to_bf16_bits(bf16_bits_to_f32(residual) + bf16_bits_to_f32(r))
        return r
    if residual is not None:
        f = (np.asarray(residual, dtype=np.float32) + f).astype(np.float32)
    return f


# ---- GPTQ format ------------------------------------------------------------

def gen_gptq(N: int, K: int, seed: int):
    """Config 0's weight: int4 v uniform in [-8, 7], packed 8 per int32 along K as nibble v + 8 (low nibble
    first), i.e. bytes [N, K/2]; fp16 scales [N, K/128] = |N(0,1)| * 0.02 / 7 + 1e-4."""
    g = torch.Generator().manual_seed(seed)
    v = torch.randint(-8, 8, (N, K), generator=g, dtype=torch.int16).numpy()
    nib = (v + 8).astype(np.uint8)
    packed = (nib[:, 0::2] | (nib[:, 1::2] << 4)).astype(np.uint8)
    scales = (torch.randn(N, K // 128, generator=g).abs() * 0.02 / 7 + 1e-4).to(torch.float16).numpy()
    return packed, scales


def gptq_unpack(packed: np.ndarray) -> np.ndarray:
    """[N, K/2] bytes (nibble = v + 8, low nibble = even k) -> int8 v [N, K]."""
    N, H = packed.shape
    v = np.empty((N, 2 * H), dtype=np.int8)
    v[:, 0::2] = (packed & 0xF).astype(np.int8) - 8
    v[:, 1::2] = (packed >> 4).astype(np.int8) - 8
    return v


def gptq_linear(xq: np.ndarray, xs: np.ndarray, packed: np.ndarray, scales: np.ndarray, residual=None,
                out_bf16: bool = True):
    """GPTQ W4A8 linear, the order of include/mono_b200.h mono_w4a8_gptq_linear:
    acc_g = int32 dot per 128-group; F_c = fp32 sum over the groups of each 1024-chunk (ascending, from +0)
    of float(acc_g) * float(s[n, g]); total = fp32 sum of F_c (ascending, from +0); out = cast(total * xs[m])."""
    M, K = xq.shape
    v = gptq_unpack(packed)
    acc = _group_dot(xq, v, 128)  # [M, N, G]
    s = scales.astype(np.float32)  # fp16 -> fp32 exact
    G = K // 128
    total = np.zeros((M, v.shape[0]), dtype=np.float32)
    for c in range(K // CHUNK_K):
        F = np.zeros_like(total)
        for g in range(c * 8, c * 8 + 8):
            F = (F + (acc[:, :, g].astype(np.float32) * s[None, :, g]).astype(np.float32)).astype(np.float32)
        total = (total + F).astype(np.float32)
    assert G == (K // CHUNK_K) * 8
    f = (total * np.asarray(xs, dtype=np.float32)[:, None]).astype(np.float32)
    return _finish(f, residual, out_bf16)


def act_quant(x_bits: np.ndarray):
    """GPTQ per-token activation quant: s = amax / 127 (fp32), q = clamp(rint(x / s), -127, 127); zero rows
    give s = 0 and q = 0."""
    x = bf16_bits_to_f32(x_bits)
    amax = np.abs(x).max(axis=1).astype(np.float32)
    s = (amax / np.float32(127.0)).astype(np.float32)
    with np.errstate(divide="ignore", invalid="ignore"):
        d = (x / s[:, None]).astype(np.float32)
    q = np.clip(np.rint(d), -127, 127)
    q = np.where(s[:, None] > 0, q, 0).astype(np.int8)
    return q, s


# ---- REF format (the reference's packed W4A8) ---------------------------------------------------------

def random_w4(N: int, K: int, g: torch.Generator):
    """The reference's test weight generator (tests/test_w4a8_linear.py:9-16): int4 codes as random bytes,
    FP8 group scales (G16, bytes 0x18-0x57), channel scales U * 1e-3 + 1e-4, codebook arange(-8, 8)."""
    q = torch.randint(-128, 128, (N, K // 2), generator=g, dtype=torch.int8)
    s = torch.randint(0x18, 0x58, (N, K // 16), generator=g, dtype=torch.uint8)
    c = torch.rand(N, generator=g) * 1e-3 + 1e-4
    cb = torch.arange(-8, 8, dtype=torch.float32)
    return q.view(torch.uint8).numpy(), s.numpy(), c.numpy(), cb.numpy()


def ref_decode(packed: np.ndarray, s_rel: np.ndarray, codebook) -> np.ndarray:
    """int8 grid of the reference decode (csrc/w4a8_decode.sycl:4-11, :35-45):
    w = isnan(r) ? 0 : clamp(r, -127, 127), r = rint(codebook[code] * s_rel[n, k / 16]) in fp32."""
    N, H = packed.shape
    K = 2 * H
    codes = np.empty((N, K), dtype=np.int64)
    codes[:, 0::2] = packed & 0xF
    codes[:, 1::2] = packed >> 4
    cb = np.arange(-8, 8, dtype=np.float32) if codebook is None else np.asarray(codebook, dtype=np.float32)
    sc = fp8e4m3_to_f32(s_rel)  # [N, K/16]
    prod = (cb[codes] * np.repeat(sc, 16, axis=1)).astype(np.float32)
    r = np.rint(prod)
    w = np.where(np.isnan(r), 0, np.clip(r, -127, 127))
    return w.astype(np.int8)


def ref_linear(xq: np.ndarray, xs: np.ndarray, packed: np.ndarray, s_rel: np.ndarray, s_channel: np.ndarray,
               codebook=None, residual=None, out_bf16: bool = True):
    """The reference's w4a8_decode_linear (csrc/w4a8_decode.sycl:150-163): f = float(acc) * xs[m];
    f = f * s_channel[n]; out = cast(f) (+ residual)."""
    w = ref_decode(packed, s_rel, codebook)
    acc = _int_dot(xq, w)
    acc = ((acc + 2 ** 31) % 2 ** 32 - 2 ** 31).astype(np.int64)  # int32 modular accumulation
    f = (acc.astype(np.float32) * np.asarray(xs, dtype=np.float32)[:, None]).astype(np.float32)
    f = (f * np.asarray(s_channel, dtype=np.float32)[None, :]).astype(np.float32)
    return _finish(f, residual, out_bf16)


def ref_pair_table(codebook=None) -> np.ndarray:
    """The REF decode table of include/mono_b200.h mono_w4_pair_table: entry (s << 8 | byte) = int8 grid value
    of the low code | of the high code << 8, for every FP8 scale byte s."""
    cb = np.arange(-8, 8, dtype=np.float32) if codebook is None else np.asarray(codebook, dtype=np.float32)
    scale = fp8e4m3_to_f32(np.arange(256, dtype=np.uint8))[:, None]  # [256 scale bytes, 1]
    byte = np.arange(256)[None, :]

    def grid(code):
        r = np.rint((cb[code] * scale).astype(np.float32))
        return np.where(np.isnan(r), 0, np.clip(r, -127, 127)).astype(np.int8).astype(np.uint8).astype(np.uint16)

    return (grid(byte & 15) | (grid(byte >> 4) << 8)).reshape(-1).astype(np.uint16)


def rot_quant(x_bits: np.ndarray, h_bits: np.ndarray):
    """ConvRot rotate + row quantize (csrc/act_prep.sycl:4-10, :71-91), with the rotation's 256-term sums
    exact (fp64) and rounded once to bf16:
    x_rot = bf16(x_grouped @ H); s = max(amax / 127, 1e-30); s_bf = bf16(s) (0 -> tiny);
    q = clamp(rint(bf16(x_rot / s_bf)), -128, 127)."""
    M, K = x_bits.shape
    x = bf16_bits_to_f32(x_bits).astype(np.float64).reshape(M, K // 256, 256)
    h = bf16_bits_to_f32(h_bits).astype(np.float64).reshape(256, 256)
    rot = f64_to_bf16_bits(np.einsum("mgk,kj->mgj", x, h).reshape(M, K))
    xr = bf16_bits_to_f32(rot)
    amax = np.abs(xr).max(axis=1).astype(np.float32)
    s = np.maximum((amax / np.float32(127.0)).astype(np.float32), np.float32(1e-30)).astype(np.float32)
    sb = f32_to_bf16_bits(s)
    sb = np.where((sb & 0x7FFF) == 0, np.uint16(0x0080), sb)
    sbf = bf16_bits_to_f32(sb)
    d = bf16_bits_to_f32(f32_to_bf16_bits((xr / sbf[:, None]).astype(np.float32)))
    q = np.clip(np.rint(d), -128, 127).astype(np.int8)
    return q, s


def hadamard_256() -> np.ndarray:
    """The regular Hadamard matrix of order 256 divided by 16, as bf16 bits: kron of four copies of the
    regular H4 (-1 exactly where i ^ j == 3), the matrix comfy_mono_decode_xpu/layer.py:74-90 rebuilds and
    checks against Kitchen's _build_hadamard(256)."""
    h4 = np.where((np.arange(4)[:, None] ^ np.arange(4)[None, :]) == 3, -1.0, 1.0)
    h = h4
    for _ in range(3):
        h = np.kron(h, h4)
    return f32_to_bf16_bits((h / 16.0).astype(np.float32))
