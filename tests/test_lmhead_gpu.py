"""The fused bf16 lm_head + pick (mono_lmhead_pick) against the pinned-order oracle (oracle/lmhead.py): logits
bit-exact, argmax and top-k indices bit-exact, and the draft pick's scatter into the verify-token row."""
import numpy as np
import pytest
import torch

from conftest import bf16_bits
from oracle import lmhead as olh

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,V,k", [(1, 30001, 2), (5, 16384, 0), (8, 12289, 8), (3, 4099, 1)])
def test_lmhead_pick_bit_exact(cuda, M, V, k):
    from mono_b200 import _C
    K = 4096
    g = torch.Generator().manual_seed(M * 7 + V)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(V, K, generator=g) * 0.02).bfloat16()
    # plant exact ties: duplicate rows of w give equal logits, so the tie orders decide
    w[V // 3] = w[V // 2]
    w[V - 1] = w[7]
    lg_ref, am_ref, top_ref = olh.pick(bf16_bits(x), bf16_bits(w), k)
    for _ in range(2):  # the second call reuses the workspace (the arrival counter is reset by the kernel)
        am, tk, lg = _C.lmhead_pick(x.to(cuda), w.to(cuda), k=k, logits=True)
        torch.cuda.synchronize()
        assert np.array_equal(bf16_bits(lg), lg_ref)
        assert np.array_equal(am.cpu().numpy(), am_ref)
        if k:
            assert np.array_equal(tk.cpu().numpy(), top_ref)


def test_lmhead_draft_pick_scatter(cuda):
    from mono_b200 import _C
    K, V = 4096, 20011
    g = torch.Generator().manual_seed(5)
    x = torch.randn(1, K, generator=g).bfloat16()
    w = (torch.randn(V, K, generator=g) * 0.02).bfloat16()
    _, am_ref, top_ref = olh.pick(bf16_bits(x), bf16_bits(w), 2)
    children = torch.tensor([2, 6, -1, -1, -1, -1, -1, -1], dtype=torch.int32, device=cuda)
    dst = torch.full((8,), -5, dtype=torch.int64, device=cuda)
    _C.lmhead_pick(x.to(cuda), w.to(cuda), k=2, children=children, dst=dst)
    ref = olh.draft_scatter(int(am_ref[0]), list(top_ref[0]), [2, 6, -1], [-5] * 8)
    assert dst.cpu().tolist() == ref
