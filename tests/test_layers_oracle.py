"""Row operations and the MLP chain of the oracle against fp64 (CPU only)."""
import numpy as np
import torch

from oracle import layers as ol
from oracle import numerics as nu
from oracle import w4a8 as ow


def _bits(t):
    return t.to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)


def test_rmsnorm_near_fp64():
    g = torch.Generator().manual_seed(0)
    for H in (4096, 1024):
        x = torch.randn(5, H, generator=g) * torch.exp(torch.randn(5, 1, generator=g))
        w = 1 + torch.randn(H, generator=g) * 0.02
        out = nu.bf16_bits_to_f32(ol.rmsnorm(_bits(x), _bits(w), 1e-6)).astype(np.float64)
        xb = nu.bf16_bits_to_f32(_bits(x)).astype(np.float64)
        wb = nu.bf16_bits_to_f32(_bits(w)).astype(np.float64)
        ref = xb / np.sqrt((xb ** 2).mean(1, keepdims=True) + 1e-6) * wb
        assert np.max(np.abs(out - ref) / (np.abs(ref) + 1e-30)) <= 2 ** -8 + 1e-6


def test_rmsnorm_zero_row():
    x = np.zeros((1, 4096), dtype=np.uint16)
    w = _bits(torch.ones(4096))
    assert not ol.rmsnorm(x, w, 1e-6).any()


def test_mlp_chain_near_fp64():
    H, I, M = 1024, 2048, 3
    g = torch.Generator().manual_seed(1)
    x = _bits(torch.randn(M, H, generator=g))
    w = _bits(1 + torch.randn(H, generator=g) * 0.02)
    gate, up = ow.gen_gptq(I, H, seed=1), ow.gen_gptq(I, H, seed=2)
    down = ow.gen_gptq(H, I, seed=3)
    allbf = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    lut = torch.nn.functional.silu(allbf.float()).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    out = nu.bf16_bits_to_f32(ol.mlp_gptq(x, w, 1e-6, gate, up, down, lut)).astype(np.float64)

    def deq(pk, sc):
        return ow.gptq_unpack(pk).astype(np.float64) * np.repeat(sc.astype(np.float64), 128, axis=1)

    xf = nu.bf16_bits_to_f32(x).astype(np.float64)
    xn = xf / np.sqrt((xf ** 2).mean(1, keepdims=True) + 1e-6) * nu.bf16_bits_to_f32(w)
    gg, uu = xn @ deq(*gate).T, xn @ deq(*up).T
    h = gg / (1 + np.exp(-gg)) * uu
    ref = xf + h @ deq(*down).T
    err = np.abs(out - ref)
    # int8 activation quantization twice: errors relative to the output scale stay at the percent level
    assert err.max() <= 0.05 * np.abs(ref).max() and err.mean() <= 0.01 * np.abs(ref).mean()
