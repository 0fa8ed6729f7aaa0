"""The backend install points (mono_b200.patch) on the GPU: a replaced w4a8_linear_prequantized /
quantize_and_rotate_rowwise answers eligible calls with this build's kernels, bit-identical to the oracle of the
original chain, and hands calls the C ABI refuses (17 rows, K not a multiple of 1024, misaligned operands) to the
original under the ABI's own reason, leaving the piece on."""
import types

import numpy as np
import pytest
import torch

from conftest import bf16_bits, bits_equal
from oracle import w4a8 as ow

pytestmark = pytest.mark.gpu


def _module(name, fn_name):
    mod = types.ModuleType(name)
    calls = []

    def stock(*args, **kwargs):
        calls.append(args)
        return "stock"
    setattr(mod, fn_name, stock)
    return mod, calls


def test_patched_linear_serves_eligible_calls_and_refuses_the_rest(cuda):
    from mono_b200 import guard, patch
    guard.reset()
    mod, calls = _module("omni_xpu_kernel.int8", "w4a8_linear_prequantized")
    patch.install(mod)
    N, K = 4096, 4096
    g = torch.Generator().manual_seed(31)
    packed, s_rel, sch, cb = ow.random_w4(N, K, g)
    pk = torch.from_numpy(packed).to(cuda)
    sr = torch.from_numpy(s_rel).to(cuda).view(torch.float8_e4m3fn)
    sc = torch.from_numpy(sch).to(cuda).reshape(N, 1)  # [N, 1] channel scales, as the backend stores them
    cbt = torch.from_numpy(cb).to(cuda)
    served = patch.stats()["fused"]
    for shape in ((1, 1, K), (2, 4, K), (16, K)):
        x = torch.randint(-127, 128, shape, generator=g, dtype=torch.int8)
        xs = (torch.rand(*shape[:-1], 1, generator=g) * 0.05 + 1e-3)
        out = mod.w4a8_linear_prequantized(x.to(cuda), xs.to(cuda), pk, sr, sc, cbt, None, 16, torch.bfloat16)
        assert out.shape == (*shape[:-1], N)
        ref = ow.ref_linear(x.reshape(-1, K).numpy(), xs.reshape(-1).numpy(), packed, s_rel, sch, cb)
        assert bits_equal(bf16_bits(out.reshape(-1, N)), ref), shape
    assert patch.stats()["fused"] == served + 3 and not calls
    before = patch.stats()["reasons"]
    x17 = torch.zeros(17, K, dtype=torch.int8, device=cuda)
    assert mod.w4a8_linear_prequantized(x17, torch.ones(17, 1, device=cuda), pk, sr, sc, cbt) == "stock"
    pk_odd = torch.zeros(N, 500, dtype=torch.int8, device=cuda)
    x_odd = torch.zeros(1, 1000, dtype=torch.int8, device=cuda)
    sr_odd = torch.zeros(N, 1000 // 16, dtype=torch.uint8, device=cuda).view(torch.float8_e4m3fn)
    assert mod.w4a8_linear_prequantized(x_odd, torch.ones(1, 1, device=cuda), pk_odd, sr_odd, sc, cbt) == "stock"
    after = patch.stats()["reasons"]
    assert len(calls) == 2 and not guard.off("w4")
    assert sum(after.values()) == sum(before.values()) + 2
    assert any("1 <= M <= 16" in r for r in after), after


def test_patched_rot_quant_serves_eligible_calls(cuda):
    from mono_b200 import guard, patch
    guard.reset()
    mod, calls = _module("comfy_kitchen.backends.cuda.w4a8_int8", "quantize_and_rotate_rowwise")
    assert patch.install_prep([mod]) == 1
    h = ow.hadamard_256()
    ht = torch.from_numpy(h.view(np.int16)).view(torch.bfloat16).to(cuda)
    g = torch.Generator().manual_seed(8)
    x = torch.randn(1, 3, 4096, generator=g).bfloat16()
    q, s = mod.quantize_and_rotate_rowwise(x.to(cuda), ht, 256)
    rq, rs = ow.rot_quant(x.reshape(3, -1).view(torch.int16).numpy().view(np.uint16), h)
    assert q.shape == (1, 3, 4096) and s.shape == (1, 3, 1)
    assert np.array_equal(q.reshape(3, -1).cpu().numpy(), rq) and bits_equal(s.reshape(-1).cpu().numpy(), rs)
    assert mod.quantize_and_rotate_rowwise(torch.zeros(2, 100, dtype=torch.bfloat16, device=cuda), ht, 256) == "stock"
    assert len(calls) == 1 and not guard.off("prep")
