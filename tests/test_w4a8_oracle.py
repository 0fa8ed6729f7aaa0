"""The W4A8 oracle against independent restatements (CPU only)."""
import numpy as np
import pytest
import torch

from oracle import numerics as nu
from oracle import w4a8


def test_bf16_rounding_matches_torch():
    g = torch.Generator().manual_seed(0)
    x = torch.randn(100000, generator=g) * torch.exp(torch.randn(100000, generator=g) * 8)
    x[:10] = torch.tensor([0.0, -0.0, float("inf"), float("-inf"), 1e-40, -1e-40, 3.4e38, 1.0, 65504.0, -2.5])
    ours = nu.f32_to_bf16_bits(x.numpy())
    ref = x.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(ours, ref)


def test_f64_to_bf16_single_rounding():
    g = torch.Generator().manual_seed(1)
    v = (torch.randn(50000, generator=g, dtype=torch.float64) * torch.exp(torch.randn(50000, generator=g,
                                                                                        dtype=torch.float64) * 20))
    bits = nu.f64_to_bf16_bits(v.numpy())
    back = nu.bf16_bits_to_f32(bits).astype(np.float64)
    # the result is a bf16 neighbour of v and no other bf16 is closer
    up = nu.bf16_bits_to_f32((bits.astype(np.int32) + 1).astype(np.uint16)).astype(np.float64)
    dn = nu.bf16_bits_to_f32((bits.astype(np.int32) - 1).astype(np.uint16)).astype(np.float64)
    err = np.abs(back - v.numpy())
    fin = np.isfinite(back) & np.isfinite(up) & np.isfinite(dn)
    assert np.all(err[fin] <= np.abs(up - v.numpy())[fin]) and np.all(err[fin] <= np.abs(dn - v.numpy())[fin])
    # exact ties go to the even pattern
    tie = np.array([1.0 + 2.0 ** -8, 1.0 + 3 * 2.0 ** -8], dtype=np.float64)
    assert list(nu.f64_to_bf16_bits(tie)) == [0x3F80, 0x3F82]
    assert nu.f64_to_bf16_bits(np.array([0.0, -0.0])).tolist() == [0, 0x8000]


def test_fp8_decode_matches_torch():
    b = torch.arange(256, dtype=torch.uint8)
    ref = b.view(torch.float8_e4m3fn).float().numpy()
    ours = nu.fp8e4m3_to_f32(b.numpy())
    assert np.array_equal(np.isnan(ours), np.isnan(ref))
    assert np.array_equal(ours[~np.isnan(ref)].view(np.uint32), ref[~np.isnan(ref)].view(np.uint32))


@pytest.mark.parametrize("M", [1, 3, 8, 16])
def test_gptq_linear_near_fp64(M):
    N, K = 256, 2048
    packed, scales = w4a8.gen_gptq(N, K, seed=7)
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    xq, xs = w4a8.act_quant(x.view(torch.int16).numpy().view(np.uint16))
    out = nu.bf16_bits_to_f32(w4a8.gptq_linear(xq, xs, packed, scales))
    v = w4a8.gptq_unpack(packed).astype(np.float64)
    s = np.repeat(scales.astype(np.float64), 128, axis=1)
    exact = (xq.astype(np.float64) @ (v * s).T) * xs.astype(np.float64)[:, None]
    assert np.allclose(out, exact, rtol=2 ** -7, atol=1e-6)


def test_gptq_unpack_roundtrip():
    packed, _ = w4a8.gen_gptq(32, 256, seed=3)
    v = w4a8.gptq_unpack(packed)
    assert v.min() >= -8 and v.max() <= 7
    nib = (v + 8).astype(np.uint8)
    assert np.array_equal(nib[:, 0::2] | (nib[:, 1::2] << 4), packed)


def test_act_quant_properties():
    g = torch.Generator().manual_seed(5)
    x = torch.randn(4, 4096, generator=g).to(torch.bfloat16)
    x[2] = 0
    q, s = w4a8.act_quant(x.view(torch.int16).numpy().view(np.uint16))
    assert s[2] == 0 and not q[2].any()
    for r in (0, 1, 3):
        assert np.abs(q[r]).max() == 127
        deq = q[r].astype(np.float64) * s[r]
        assert np.max(np.abs(deq - x[r].float().numpy())) <= s[r] * 0.5 * (1 + 1e-5)


def test_ref_decode_and_pair_table_agree():
    g = torch.Generator().manual_seed(9)
    packed, s_rel, sch, cb = w4a8.random_w4(64, 512, g)
    w = w4a8.ref_decode(packed, s_rel, cb)
    tab = w4a8.ref_pair_table(cb)
    sb = np.repeat(s_rel, 8, axis=1).astype(np.int64)  # scale byte of each packed byte (16 codes / 8 bytes)
    ent = tab[(sb << 8) | packed.astype(np.int64)]
    lo = (ent & 0xFF).astype(np.uint8).view(np.int8)
    hi = (ent >> 8).astype(np.uint8).view(np.int8)
    assert np.array_equal(lo, w[:, 0::2]) and np.array_equal(hi, w[:, 1::2])


def test_ref_linear_matches_direct_formula():
    g = torch.Generator().manual_seed(11)
    packed, s_rel, sch, cb = w4a8.random_w4(128, 2048, g)
    x = torch.randint(-127, 128, (3, 2048), generator=g, dtype=torch.int8).numpy()
    xs = (torch.rand(3, generator=g) * 0.05 + 1e-3).numpy()
    out = w4a8.ref_linear(x, xs, packed, s_rel, sch, cb)
    w = w4a8.ref_decode(packed, s_rel, cb).astype(np.int64)
    acc = x.astype(np.int64) @ w.T
    f = (acc.astype(np.float32) * xs[:, None]).astype(np.float32)
    f = (f * sch[None, :]).astype(np.float32)
    ref = torch.from_numpy(f).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    assert np.array_equal(out, ref)


def test_rot_quant_regular_hadamard():
    h = w4a8.hadamard_256()
    hf = nu.bf16_bits_to_f32(h).astype(np.float64).reshape(256, 256)
    assert np.allclose(hf @ hf.T, np.eye(256))  # orthonormal
    g = torch.Generator().manual_seed(2)
    x = torch.randn(2, 512, generator=g).to(torch.bfloat16)
    q, s = w4a8.rot_quant(x.view(torch.int16).numpy().view(np.uint16), h)
    assert q.dtype == np.int8 and s.shape == (2,)
    rot = x.double().numpy().reshape(2, 2, 256) @ hf
    deq = q.astype(np.float64).reshape(2, 2, 256) * s[:, None, None]
    assert np.max(np.abs(deq - rot)) < 0.05 * np.abs(rot).max()
