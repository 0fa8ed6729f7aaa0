"""The fused GPTQ MLP block (one cooperative launch) against the oracle chain, bit for bit."""
import numpy as np
import pytest
import torch

from conftest import bf16_bits, bits_equal
from oracle import layers as ol
from oracle import w4a8 as ow

pytestmark = pytest.mark.gpu


def _weights(cuda, H, I, seed):
    from mono_b200 import _C
    mats = [ow.gen_gptq(I, H, seed), ow.gen_gptq(I, H, seed + 1), ow.gen_gptq(H, I, seed + 2)]
    dev = []
    for (pk, sc), (n, k) in zip(mats, [(I, H), (I, H), (H, I)]):
        dev.append(_C.w4_repack(0, torch.from_numpy(pk).to(cuda), torch.from_numpy(sc).to(cuda), n, k))
    return mats, dev


@pytest.mark.parametrize("H,I", [(4096, 12288), (2048, 4096)])
def test_mlp_gptq_bit_exact(cuda, H, I):
    from mono_b200 import _C
    mats, dev = _weights(cuda, H, I, seed=0x5EED + 1)
    lut = _C.act_luts(cuda)[0]
    lut_np = bf16_bits(lut)
    g = torch.Generator().manual_seed(H + I)
    w = (1 + torch.randn(H, generator=g) * 0.02).to(torch.bfloat16)
    for M in (1, 3, 8, 9, 16, 24, 32):  # (17..32: four 8-row tiles, tiles in batches)
        x = torch.randn(M, H, generator=g).to(torch.bfloat16)
        ref = ol.mlp_gptq(bf16_bits(x), bf16_bits(w), 1e-6, *mats, lut_np)
        for _ in range(2):  # the second call reuses the workspace (barrier words reset by the kernel)
            out = _C.mlp_gptq(x.to(cuda), w.to(cuda), 1e-6, *dev, silu_lut=lut)
            assert bits_equal(bf16_bits(out), ref), (H, I, M)
    assert _C.device_status() == 0


def test_mlp_gptq_variants(cuda):
    """No norm (the reference's mono_mlp takes the normed rows), no residual, and in place."""
    from mono_b200 import _C
    H, I = 2048, 4096
    mats, dev = _weights(cuda, H, I, seed=11)
    lut = _C.act_luts(cuda)[0]
    lut_np = bf16_bits(lut)
    g = torch.Generator().manual_seed(3)
    x = torch.randn(8, H, generator=g).to(torch.bfloat16)
    ref = ol.mlp_gptq(bf16_bits(x), None, 1e-6, *mats, lut_np, residual=False)
    out = _C.mlp_gptq(x.to(cuda), None, 1e-6, *dev, silu_lut=lut, residual=False)
    assert bits_equal(bf16_bits(out), ref)
    w = (1 + torch.randn(H, generator=g) * 0.02).to(torch.bfloat16)
    ref = ol.mlp_gptq(bf16_bits(x), bf16_bits(w), 1e-6, *mats, lut_np)
    xd = x.to(cuda)
    _C.mlp_gptq(xd, w.to(cuda), 1e-6, *dev, silu_lut=lut, out=xd)
    assert bits_equal(bf16_bits(xd), ref)


def test_mlp_gptq_graph_replay(cuda):
    """Captured once in a CUDA graph, replayed: same bits every replay."""
    from mono_b200 import _C
    H, I = 2048, 4096
    mats, dev = _weights(cuda, H, I, seed=21)
    lut = _C.act_luts(cuda)[0]
    g = torch.Generator().manual_seed(4)
    x = torch.randn(8, H, generator=g).to(torch.bfloat16).to(cuda)
    w = (1 + torch.randn(H, generator=g) * 0.02).to(torch.bfloat16).to(cuda)
    out = torch.empty_like(x)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        _C.mlp_gptq(x, w, 1e-6, *dev, silu_lut=lut, out=out)
    s.synchronize()
    first = out.clone()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=s):
        _C.mlp_gptq(x, w, 1e-6, *dev, silu_lut=lut, out=out)
    for _ in range(5):
        out.zero_()
        graph.replay()
        torch.cuda.synchronize()
        assert torch.equal(out.view(torch.int16), first.view(torch.int16))
