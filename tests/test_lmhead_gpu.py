"""The fused bf16 lm_head + pick (mono_lmhead_pick, tensor-core logits): logits within the stated tolerance of the
exact fp64 dot products (oracle/lmhead.py tolerance), the same bits on every launch and for equal weight rows, argmax
and top-k indices bit-exact against the oracle's pick on the kernel's own logits (planted ties decide by the tie
orders), and the draft pick's scatter into the verify-token row."""
import numpy as np
import pytest
import torch

from conftest import bf16_bits
from oracle import lmhead as olh
from oracle.numerics import bf16_bits_to_f32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,V,k,K", [(1, 30001, 2, 4096), (5, 16384, 0, 4096), (8, 12289, 8, 4096),
                                     (3, 4099, 1, 4096), (8, 32768, 2, 2048), (2, 151936, 8, 4096),
                                     (16, 20011, 2, 4096), (12, 8192, 8, 4096), (16, 4104, 0, 2048)])
def test_lmhead_pick(cuda, M, V, k, K):
    from mono_b200 import _C
    g = torch.Generator().manual_seed(M * 7 + V)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(V, K, generator=g) * 0.02).bfloat16()
    # plant exact ties: duplicate rows of w give equal logits, so the tie orders decide
    w[V // 3] = w[V // 2]
    w[V - 1] = w[7]
    w[V // 5] = w[V // 2]
    xb, wb = bf16_bits(x), bf16_bits(w)
    runs = []
    for _ in range(2):  # the second call reuses the workspace (the arrival counter is reset by the kernel)
        am, tk, lg = _C.lmhead_pick(x.to(cuda), w.to(cuda), k=k, logits=True)
        torch.cuda.synchronize()
        runs.append((am.cpu().numpy(), None if tk is None else tk.cpu().numpy(), bf16_bits(lg)))
    (am, tk, lg), (am2, tk2, lg2) = runs
    assert np.array_equal(lg, lg2) and np.array_equal(am, am2)  # deterministic
    assert np.array_equal(lg[:, V // 3], lg[:, V // 2]) and np.array_equal(lg[:, V - 1], lg[:, 7])
    exact, abs_sum = olh.logits_exact(xb, wb)
    err = np.abs(bf16_bits_to_f32(lg).astype(np.float64) - exact)
    assert (err <= olh.tolerance(exact, abs_sum)).all(), err.max()
    am_ref, top_ref = olh.pick_logits(lg, k)
    assert np.array_equal(am, am_ref)
    if k:
        assert np.array_equal(tk, top_ref) and np.array_equal(tk2, top_ref)


def test_lmhead_pick_without_logits_matches(cuda):
    """The pick alone (no logits written) equals the pick of the logits the same kernel writes."""
    from mono_b200 import _C
    g = torch.Generator().manual_seed(44)
    x = torch.randn(8, 4096, generator=g).bfloat16().to(cuda)
    w = (torch.randn(65536, 4096, generator=g) * 0.02).bfloat16().to(cuda)
    am, tk, lg = _C.lmhead_pick(x, w, k=4, logits=True)
    am2, tk2 = _C.lmhead_pick(x, w, k=4)[:2]
    assert torch.equal(am, am2) and torch.equal(tk, tk2)
    am_ref, top_ref = olh.pick_logits(bf16_bits(lg), 4)
    assert np.array_equal(am.cpu().numpy(), am_ref) and np.array_equal(tk.cpu().numpy(), top_ref)


def test_lmhead_draft_pick_scatter(cuda):
    from mono_b200 import _C
    K, V = 4096, 20011
    g = torch.Generator().manual_seed(5)
    x = torch.randn(1, K, generator=g).bfloat16().to(cuda)
    w = (torch.randn(V, K, generator=g) * 0.02).bfloat16().to(cuda)
    _, _, lg = _C.lmhead_pick(x, w, k=2, logits=True)
    am_ref, top_ref = olh.pick_logits(bf16_bits(lg), 2)
    children = torch.tensor([2, 6, -1, -1, -1, -1, -1, -1], dtype=torch.int32, device=cuda)
    dst = torch.full((8,), -5, dtype=torch.int64, device=cuda)
    _C.lmhead_pick(x, w, k=2, children=children, dst=dst)
    ref = olh.draft_scatter(int(am_ref[0]), list(top_ref[0]), [2, 6, -1], [-5] * 8)
    assert dst.cpu().tolist() == ref
