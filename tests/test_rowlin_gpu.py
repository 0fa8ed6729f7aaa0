"""Row preparation + GPTQ W4A8 linear (layer_pre / the gate + out projection of layer_post) on the GPU against the
CPU oracle, bit-exact (pinned RMSNorm order, per-token quant, pinned GPTQ epilogue)."""
import numpy as np
import pytest
import torch

from conftest import bf16_bits
from oracle import layers as ol
from oracle import w4a8 as ow
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def _mats(shapes, K, seed, cuda):
    from mono_b200 import _C
    host, dev = [], []
    for i, N in enumerate(shapes):
        p, s = ow.gen_gptq(N, K, seed + i)
        host.append((p, s))
        dev.append((_C.w4_repack(0, torch.from_numpy(p).to(cuda), torch.from_numpy(s).to(cuda), N, K), N))
    return host, dev


@pytest.mark.parametrize("M", [1, 8, 9, 16, 25, 32])
def test_rowlin_norm_qkv_bit_exact(cuda, M):
    from mono_b200 import _C
    K = 4096
    host, dev = _mats([8192, 1024, 1024], K, 0x5EED + 2, cuda)
    g = torch.Generator().manual_seed(M)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (1 + torch.randn(K, generator=g) * 0.02).bfloat16()
    xn = ol.rmsnorm(bf16_bits(x), bf16_bits(w), 1e-6)
    q, s = ow.act_quant(xn)
    ref = np.concatenate([ow.gptq_linear(q, s, p, sc) for p, sc in host], axis=1)
    xn_out = torch.empty(M, K, dtype=torch.bfloat16, device=cuda)
    out = _C.rowlin_gptq(x.to(cuda), _C.ROWLIN_NORM, dev, norm_w=w.to(cuda), eps=1e-6, xn_out=xn_out)
    assert np.array_equal(bf16_bits(out), ref)
    assert np.array_equal(bf16_bits(xn_out), xn)


@pytest.mark.parametrize("M", [1, 5, 8, 16, 24, 32])
def test_rowlin_norm_ab_bit_exact(cuda, M):
    """The GDN layer_pre in one launch (mono_rowlin_norm_ab_gptq): qkv | z, the normalized rows and the a | b
    projection of those rows (on the launch's last CTAs) equal the oracle and the separate mono_gdn_ab call."""
    from mono_b200 import _C
    from oracle import gdn as og
    K, HV = 4096, 32
    host, dev = _mats([8192, 4096], K, 0x5EED + 7, cuda)
    g = torch.Generator().manual_seed(70 + M)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (1 + torch.randn(K, generator=g) * 0.02).bfloat16()
    wab = (torch.randn(2 * HV, K, generator=g) * 0.02).bfloat16()
    xn = ol.rmsnorm(bf16_bits(x), bf16_bits(w), 1e-6)
    q, s = ow.act_quant(xn)
    ref = np.concatenate([ow.gptq_linear(q, s, p, sc) for p, sc in host], axis=1)
    xn_out = torch.empty(M, K, dtype=torch.bfloat16, device=cuda)
    wide = torch.full((M, 2 * HV + 8), -1.0, dtype=torch.bfloat16, device=cuda)  # a row stride wider than N
    ab = wide[:, 4:4 + 2 * HV]
    out = _C.rowlin_gptq(x.to(cuda), _C.ROWLIN_NORM, dev, norm_w=w.to(cuda), eps=1e-6, xn_out=xn_out,
                         ab=(wab.to(cuda), ab))
    torch.cuda.synchronize()
    assert np.array_equal(bf16_bits(out), ref)
    assert np.array_equal(bf16_bits(xn_out), xn)
    assert np.array_equal(bf16_bits(ab), og.ab_projection(xn, bf16_bits(wab)))
    assert np.array_equal(bf16_bits(ab), bf16_bits(_C.gdn_ab(xn_out, wab.to(cuda))))
    assert bool((wide[:, :4] == -1).all()) and bool((wide[:, 4 + 2 * HV:] == -1).all())  # nothing outside the view
    assert _C.device_status() == 0


@pytest.mark.parametrize("M", [1, 8, 32])
def test_rowlin_gate_oproj_residual_bit_exact(cuda, M):
    from mono_b200 import _C
    K = 4096
    host, dev = _mats([4096], K, 0x5EED + 5, cuda)
    g = torch.Generator().manual_seed(10 + M)
    y = torch.randn(M, K, generator=g).bfloat16()
    qg = torch.randn(M, 16, 512, generator=g).bfloat16()  # gated query heads: [query 256 | gate 256]
    res = torch.randn(M, K, generator=g).bfloat16()
    lut = _C.act_luts(cuda)[1]  # sigmoid of every bf16 pattern
    gate_cols = qg[:, :, 256:].reshape(M, K)
    lut_h = bf16_bits(lut)
    yg = f32_to_bf16_bits((bf16_bits_to_f32(bf16_bits(y)) * bf16_bits_to_f32(lut_h[bf16_bits(gate_cols).astype(np.int64)]))
                          .astype(np.float32))
    q, s = ow.act_quant(yg)
    ref = ow.gptq_linear(q, s, *host[0], residual=bf16_bits(res))
    qgd = qg.to(cuda).reshape(M, 16 * 512)
    out = _C.rowlin_gptq(y.to(cuda), _C.ROWLIN_GATE, dev, gate=qgd[:, 256:], gate_head_stride=512, lut=lut,
                         residual=res.to(cuda))
    assert np.array_equal(bf16_bits(out), ref)


def test_rowlin_quant_residual_bit_exact(cuda):
    from mono_b200 import _C
    K, M = 4096, 8
    host, dev = _mats([4096], K, 0x5EED + 7, cuda)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(M, K, generator=g).bfloat16()
    res = torch.randn(M, K, generator=g).bfloat16()
    q, s = ow.act_quant(bf16_bits(x))
    ref = ow.gptq_linear(q, s, *host[0], residual=bf16_bits(res))
    out = _C.rowlin_gptq(x.to(cuda), _C.ROWLIN_QUANT, dev, residual=res.to(cuda))
    assert np.array_equal(bf16_bits(out), ref)
    out2 = _C.rowlin_gptq(x.to(cuda), _C.ROWLIN_QUANT, dev, residual=res.to(cuda))  # workspace reuse
    assert np.array_equal(bf16_bits(out2), ref)
