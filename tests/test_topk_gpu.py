"""Exact top-k / argmax over bf16 logit rows on the GPU against the oracle (oracle/topk.py, the reference's rank
keys csrc/fast_topk.sycl:22-40): bit-exact indices and values, including ties, +-0, NaN and all-equal rows."""
import numpy as np
import pytest
import torch

from oracle import topk as ot

pytestmark = pytest.mark.gpu


def _rows(V, n, seed):
    g = torch.Generator().manual_seed(seed)
    for trial in range(n):
        x = (torch.randn(3, V, generator=g) * 3).to(torch.bfloat16)
        if trial % 2:
            x = (torch.round(x.float() * 2) / 2).to(torch.bfloat16)  # many ties
        if trial % 3 == 0:
            x[:, torch.randint(0, V, (6,), generator=g)] = x.max()
        if trial % 7 == 0:
            x[:, torch.randint(0, V, (3,), generator=g)] = 0.0
            x[:, 5] = -0.0
        if trial % 5 == 0:
            x[1, torch.randint(0, V, (2,), generator=g)] = float("nan")
        if trial % 11 == 0:
            x = torch.zeros(3, V, dtype=torch.bfloat16)
        yield x


@pytest.mark.parametrize("V", [151936, 248320, 40000])
def test_fast_topk_and_pick_match_oracle(cuda, V):
    from mono_b200 import _C
    for x in _rows(V, 12, V):
        bits = x.view(torch.int16).numpy().view(np.uint16)
        xd = x.to(cuda)
        for k in (1, 2, 3, 7, 8):
            v, i = _C.fast_topk(xd, k, False)
            rv, ri = ot.topk(bits, k)
            assert np.array_equal(i.cpu().numpy(), ri), k
            assert np.array_equal(v.cpu().view(torch.int16).numpy().view(np.uint16), rv), k
        _, ai = _C.fast_topk(xd, 1, True)
        assert np.array_equal(ai.cpu().numpy().reshape(-1), ot.argmax(bits))
        v8, i8, am = _C.fast_pick(xd, 8)
        assert np.array_equal(i8.cpu().numpy(), ot.topk(bits, 8)[1]) and np.array_equal(am.cpu().numpy(), ot.argmax(bits))


def test_fast_topk_rejects_unsupported(cuda):
    from mono_b200 import _C
    with pytest.raises(RuntimeError):
        _C.fast_topk(torch.zeros(1, 1024, dtype=torch.bfloat16, device=cuda), 9, False)
    with pytest.raises(RuntimeError):
        _C.fast_topk(torch.zeros(1, 1024, dtype=torch.bfloat16, device=cuda), 2, True)
