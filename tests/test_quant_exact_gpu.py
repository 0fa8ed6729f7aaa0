"""The per-token quantization's division-free rounding (rowops.cuh quant_i) against the IEEE quotient, over every
bf16 value of a row at several scales: q = clamp(rint(fl32(x / s)), -127, 127), s = fl32(amax / 127).

Every bf16 pattern whose magnitude is at most the row maximum is quantized (rows of 4096: the maximum first, then
the sweep), through mono_act_quant, and compared bit for bit with the numpy oracle (float32 division, rint ties to
even). The scales include s = 1 and powers of two (the quotients are exact, so every half-integer bf16 value is a
tie), scales with full 24-bit significands, and scales far outside [2^-120, 2^120] (the division path)."""
import numpy as np
import pytest
import torch

from oracle import w4a8 as ow

pytestmark = pytest.mark.gpu

AMAX = [127.0, 127.0 * 8, 127.0 / 64, 1.0, 0.7431640625, 3.140625, 250.0, 1.5e-30, 3.0e-38, 1.0e-36, 2.5e38, 6.0e4]


def _bf16_round(x: np.ndarray) -> np.ndarray:
    """float32 -> nearest bf16 bit pattern (ties to even)."""
    u = x.astype(np.float32).view(np.uint32).astype(np.uint64)
    u = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    return u.astype(np.uint16)


def _sweep_rows(amax_bits: int) -> np.ndarray:
    allp = np.arange(65536, dtype=np.uint32).astype(np.uint16)
    vals = ow.bf16_bits_to_f32(allp)
    amax = ow.bf16_bits_to_f32(np.array([amax_bits], dtype=np.uint16))[0]
    ok = np.isfinite(vals) & (np.abs(vals) <= amax)
    pats = allp[ok]
    per = 4095
    nrow = (pats.size + per - 1) // per
    rows = np.zeros((nrow, 4096), dtype=np.uint16)
    rows[:, 0] = amax_bits
    flat = np.zeros(nrow * per, dtype=np.uint16)
    flat[:pats.size] = pats
    rows[:, 1:] = flat.reshape(nrow, per)
    return rows


@pytest.mark.parametrize("amax", AMAX)
def test_quant_matches_ieee_quotient_on_every_bf16_value(cuda, amax):
    from mono_b200 import _C
    amax_bits = int(_bf16_round(np.array([amax], dtype=np.float32))[0])
    rows = _sweep_rows(amax_bits)
    q_ref, s_ref = ow.act_quant(rows)
    x = torch.from_numpy(rows.view(np.int16)).view(torch.bfloat16).to(cuda)
    q, s = _C.act_quant(x)
    torch.cuda.synchronize()
    assert np.array_equal(s.cpu().numpy().reshape(-1).view(np.uint32), s_ref.view(np.uint32))
    got = q.cpu().numpy()
    bad = np.argwhere(got != q_ref)
    assert bad.size == 0, (amax, bad[:5], [(rows[r, c], got[r, c], q_ref[r, c]) for r, c in bad[:5]])


def test_quant_ties_and_signs(cuda):
    """Rows built so that x / s lands exactly on half-integers (s a power of two) and just beside them."""
    from mono_b200 import _C
    g = np.random.default_rng(7)
    rows = []
    for e in (-3, 0, 2):
        s = np.float32(2.0 ** e)
        amax = np.float32(127.0) * s
        half = (np.arange(-127, 127) + np.float32(0.5)) * s
        near = np.concatenate([np.nextafter(half, np.float32(np.inf)), np.nextafter(half, np.float32(-np.inf))])
        vals = np.concatenate([[amax], half, near, g.standard_normal(4096).astype(np.float32) * s * 40])[:4096]
        rows.append(_bf16_round(np.clip(vals, -amax, amax).astype(np.float32)))
    rows = np.stack(rows)
    q_ref, _ = ow.act_quant(rows)
    q, _ = _C.act_quant(torch.from_numpy(rows.view(np.int16)).view(torch.bfloat16).to(cuda))
    assert np.array_equal(q.cpu().numpy(), q_ref)
