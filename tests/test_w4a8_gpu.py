"""W4A8 linear and activation quantization on the GPU (through the C ABI) against the CPU oracle.

Bit-exact for the int8 quantization, the int32 dots and the pinned fp32 epilogues (no tolerance)."""
import numpy as np
import pytest
import torch

from conftest import bf16_bits, bits_equal
from oracle import w4a8 as ow

pytestmark = pytest.mark.gpu

SHAPES = [(12288, 4096), (4096, 12288), (1024, 4096), (4096, 1024), (48, 3072), (8192 + 2048, 4096)]


def _bf16_t(bits, dev):
    return torch.from_numpy(np.ascontiguousarray(bits).view(np.int16)).view(torch.bfloat16).to(dev)


@pytest.mark.parametrize("N,K", SHAPES)
@pytest.mark.parametrize("tiled", [False, True])
def test_gptq_linear_bit_exact(cuda, N, K, tiled):
    from mono_b200 import _C
    packed, scales = ow.gen_gptq(N, K, seed=0x5EED + N + K)
    pk = torch.from_numpy(packed).to(cuda)
    sc = torch.from_numpy(scales).to(cuda)
    if tiled:
        pk, sc = _C.w4_repack(0, pk, sc, N, K), None
    g = torch.Generator().manual_seed(N * 3 + K)
    for M in (1, 2, 4, 8, 9, 16):
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        xq, xs = ow.act_quant(x.view(torch.int16).numpy().view(np.uint16))
        ref = ow.gptq_linear(xq, xs, packed, scales)
        out = _C.w4a8_gptq_linear(torch.from_numpy(xq).to(cuda), torch.from_numpy(xs).to(cuda), pk, sc, tiled=tiled, N=N)
        assert bits_equal(bf16_bits(out), ref), (M, N, K, tiled)


@pytest.mark.parametrize("N,K", [(12288, 4096), (4096, 12288), (1024, 4096), (48, 3072), (16 * 148 * 10 + 48, 4096)])
@pytest.mark.parametrize("tiled", [False, True])
def test_gptq_linear_bf16_fused_quant(cuda, N, K, tiled):
    """bf16 x with the per-token quantization inside the kernel == act_quant then the int8 linear (oracle),
    including all-zero rows (scale 0) and a row of one large value."""
    from mono_b200 import _C
    packed, scales = ow.gen_gptq(N, K, seed=0x5EED + 7 * N + K)
    pk = torch.from_numpy(packed).to(cuda)
    sc = torch.from_numpy(scales).to(cuda)
    if tiled:
        pk, sc = _C.w4_repack(0, pk, sc, N, K), None
    g = torch.Generator().manual_seed(N + 5 * K)
    for M in (1, 4, 8, 13, 16):
        if K > 4096 and M > 8:  # the staged rows of larger blocks do not fit next to the rings
            continue
        x = torch.randn(M, K, generator=g).to(torch.bfloat16)
        if M >= 4:
            x[1] = 0
            x[2] = 0
            x[2, K // 3] = 300.0
        xb = x.view(torch.int16).numpy().view(np.uint16)
        xq, xs = ow.act_quant(xb)
        ref = ow.gptq_linear(xq, xs, packed, scales)
        out = _C.w4a8_gptq_linear_bf16(x.to(cuda), pk, sc, tiled=tiled, N=N)
        assert bits_equal(bf16_bits(out), ref), (M, N, K, tiled)
        res = torch.randn(M, N, generator=g).to(torch.bfloat16)
        ref_r = ow.gptq_linear(xq, xs, packed, scales, residual=bf16_bits(res))
        out_r = _C.w4a8_gptq_linear_bf16(x.to(cuda), pk, sc, residual=res.to(cuda), tiled=tiled, N=N)
        assert bits_equal(bf16_bits(out_r), ref_r), (M, N, K, tiled, "residual")


def test_gptq_linear_bf16_rejects_oversized_rows(cuda):
    from mono_b200 import _C
    from mono_b200._lib import MonoError
    N, K, M = 64, 16384, 16
    packed, scales = ow.gen_gptq(N, K, seed=1)
    x = torch.zeros(M, K, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(MonoError, match="bf16 input"):
        _C.w4a8_gptq_linear_bf16(x, torch.from_numpy(packed).to(cuda), torch.from_numpy(scales).to(cuda))


def test_gptq_linear_residual_and_fp32(cuda):
    from mono_b200 import _C
    N, K, M = 2048, 4096, 5
    packed, scales = ow.gen_gptq(N, K, seed=3)
    g = torch.Generator().manual_seed(4)
    x = torch.randn(M, K, generator=g).to(torch.bfloat16)
    xq, xs = ow.act_quant(x.view(torch.int16).numpy().view(np.uint16))
    res = torch.randn(M, N, generator=g).to(torch.bfloat16)
    ref = ow.gptq_linear(xq, xs, packed, scales, residual=bf16_bits(res))
    args = (torch.from_numpy(xq).to(cuda), torch.from_numpy(xs).to(cuda), torch.from_numpy(packed).to(cuda),
            torch.from_numpy(scales).to(cuda))
    out = _C.w4a8_gptq_linear(*args, residual=res.to(cuda))
    assert bits_equal(bf16_bits(out), ref)
    ref32 = ow.gptq_linear(xq, xs, packed, scales, out_bf16=False)
    out32 = _C.w4a8_gptq_linear(*args, out_dtype_code=0)
    assert bits_equal(out32.cpu().numpy(), ref32)


@pytest.mark.parametrize("N,K", [(4096, 4096), (12288, 4096), (4096, 12288)])
@pytest.mark.parametrize("tiled", [False, True])
def test_ref_decode_linear_bit_exact(cuda, N, K, tiled):
    """The reference's own test generator (tests/test_w4a8_linear.py:9-29) at its shapes, M in {1,2,3,8}."""
    from mono_b200 import _C
    g = torch.Generator().manual_seed(N + K)
    packed, s_rel, sch, cb = ow.random_w4(N, K, g)
    pk = torch.from_numpy(packed).to(cuda)
    sr = torch.from_numpy(s_rel).to(cuda)
    if tiled:
        pk, sr = _C.w4_repack(1, pk, sr, N, K), None
    else:
        sr = sr.view(torch.float8_e4m3fn)
    for M in (1, 2, 3, 8, 16):
        x = torch.randint(-127, 128, (M, K), generator=g, dtype=torch.int8)
        xs = torch.rand(M, generator=g) * 0.05 + 1e-3
        ref = ow.ref_linear(x.numpy(), xs.numpy(), packed, s_rel, sch, cb)
        out = _C.w4a8_decode_linear(x.to(cuda), xs.to(cuda), pk, sr, torch.from_numpy(sch).to(cuda),
                                    torch.from_numpy(cb).to(cuda), None, 16, 2, 0, False, tiled=tiled)
        assert bits_equal(bf16_bits(out), ref), (M, N, K, tiled)


def test_ref_decode_linear_residual_fp32_and_edge_scales(cuda):
    """Residual, fp32 output, and scale bytes that saturate, are NaN or negative."""
    from mono_b200 import _C
    N, K, M = 256, 2048, 3
    g = torch.Generator().manual_seed(77)
    packed, s_rel, sch, _ = ow.random_w4(N, K, g)
    s_rel = torch.randint(0, 256, s_rel.shape, generator=g, dtype=torch.uint8).numpy()  # every fp8 byte
    cb = (torch.randn(16, generator=g) * 4).numpy().astype(np.float32)
    x = torch.randint(-128, 128, (M, K), generator=g, dtype=torch.int8)
    xs = torch.rand(M, generator=g) * 0.05 + 1e-3
    for out_code in (2, 0):
        dt = torch.bfloat16 if out_code == 2 else torch.float32
        res = torch.randn(M, N, generator=g).to(dt)
        ref = ow.ref_linear(x.numpy(), xs.numpy(), packed, s_rel, sch, cb,
                            residual=bf16_bits(res) if out_code == 2 else res.numpy(), out_bf16=out_code == 2)
        out = _C.w4a8_decode_linear(x.to(cuda), xs.to(cuda), torch.from_numpy(packed).to(cuda),
                                    torch.from_numpy(s_rel).to(cuda).view(torch.float8_e4m3fn),
                                    torch.from_numpy(sch).to(cuda), torch.from_numpy(cb).to(cuda), res.to(cuda),
                                    16, out_code, 0, False)
        got = bf16_bits(out) if out_code == 2 else out.cpu().numpy()
        assert bits_equal(got, ref), out_code


def test_pair_table_matches_oracle(cuda):
    from mono_b200 import _C
    g = torch.Generator().manual_seed(5)
    cb = (torch.randn(16, generator=g) * 30).float()
    for c in (None, cb):
        tab = _C.pair_table(None if c is None else c.to(cuda), cuda)
        ref = ow.ref_pair_table(None if c is None else c.numpy())
        assert np.array_equal(tab.cpu().numpy().view(np.uint16), ref)


@pytest.mark.parametrize("K", [4096, 12288, 8])
def test_act_quant_bit_exact(cuda, K):
    from mono_b200 import _C
    g = torch.Generator().manual_seed(K)
    for kind in ("normal", "outlier", "wide", "tiny", "zero"):
        x = torch.randn(8, K, generator=g)
        if kind == "outlier":
            x[:, torch.randint(0, K, (4,), generator=g)] *= 300
        if kind == "wide":
            x = x * torch.exp(torch.randn(8, K, generator=g) * 3)
        if kind == "tiny":
            x = x * 1e-36
        if kind == "zero":
            x = x * 0
        x = x.to(torch.bfloat16)
        q, s = _C.act_quant(x.to(cuda))
        rq, rs = ow.act_quant(x.view(torch.int16).numpy().view(np.uint16))
        assert np.array_equal(q.cpu().numpy(), rq), kind
        assert bits_equal(s.view(-1).cpu().numpy(), rs), kind


@pytest.mark.parametrize("K", [4096, 12288])
def test_rot_quant_bit_exact(cuda, K):
    """rot_quant over the reference test's input kinds (tests/test_rot_quant.py:7-30)."""
    from mono_b200 import _C
    h = ow.hadamard_256()
    ht = _bf16_t(h, cuda)
    g = torch.Generator().manual_seed(0)
    for M in (1, 3, 8):
        for kind in ("normal", "outlier", "wide", "tiny", "zero"):
            x = torch.randn(M, K, generator=g)
            if kind == "outlier":
                x[:, torch.randint(0, K, (8,), generator=g)] *= 300
            if kind == "wide":
                x = x * torch.exp(torch.randn(M, K, generator=g) * 3)
            if kind == "tiny":
                x = x * 1e-36
            if kind == "zero":
                x = x * 0
            x = x.to(torch.bfloat16)
            q, s = _C.rot_quant(x.to(cuda), ht, 3)
            rq, rs = ow.rot_quant(x.view(torch.int16).numpy().view(np.uint16), h)
            assert np.array_equal(q.cpu().numpy(), rq), (K, M, kind)
            assert bits_equal(s.view(-1).cpu().numpy(), rs), (K, M, kind)


def test_rejects_unsupported(cuda):
    from mono_b200 import _C
    x = torch.zeros(17, 4096, dtype=torch.int8, device=cuda)
    xs = torch.ones(17, device=cuda)
    pk = torch.zeros(256, 2048, dtype=torch.uint8, device=cuda)
    sc = torch.ones(256, 32, dtype=torch.float16, device=cuda)
    with pytest.raises(RuntimeError, match="M"):
        _C.w4a8_gptq_linear(x, xs, pk, sc)
    assert _C.device_status() == 0
