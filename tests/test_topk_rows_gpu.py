"""Exact top-k of a few long rows (include/mono_b200.h mono_topk_rows; the reference's topk_rows) on the GPU
against the oracle (oracle/topk.py topk_rows), bit for bit: fp32 and bf16 rows, random, tie-heavy and signed-zero
rows, k from 1 to 64, 1 to 16 rows, rows from 64 to 248k elements."""
import numpy as np
import pytest
import torch

from oracle.topk import topk_rows as ref_topk_rows

pytestmark = pytest.mark.gpu


def _check(x, k, cuda):
    from mono_b200 import _C
    v, i = _C.topk_rows(x.to(cuda), k)
    rv, ri = ref_topk_rows(x.float().numpy(), k)
    assert np.array_equal(i.cpu().numpy(), ri)
    assert np.array_equal(v.cpu().numpy().view(np.uint32), rv.view(np.uint32))


@pytest.mark.parametrize("R,N,k", [(8, 248320, 64), (1, 151936, 20), (16, 4096, 64), (3, 64, 64), (2, 100, 1)])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_topk_rows_random(cuda, R, N, k, dtype):
    g = torch.Generator().manual_seed(R * 1000 + k)
    _check((torch.randn(R, N, generator=g) * 3).to(dtype), k, cuda)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_topk_rows_ties_and_signed_zeros(cuda, dtype):
    g = torch.Generator().manual_seed(9)
    x = torch.randint(-3, 4, (4, 70000), generator=g).float()  # seven values: ties everywhere
    x[1] = 0.0
    x[2, ::2] = -0.0
    x[3, :] = 1.0
    _check(x.to(dtype), 64, cuda)


def test_topk_rows_rejects_bad_shapes(cuda):
    from mono_b200 import _C, _lib
    with pytest.raises(_lib.MonoError):
        _C.topk_rows(torch.zeros(2, 32, device=cuda), 8)  # N < 64
    with pytest.raises(_lib.MonoError):
        _C.topk_rows(torch.zeros(17, 1000, device=cuda), 8)  # 17 rows
    with pytest.raises(_lib.MonoError):
        _C.topk_rows(torch.zeros(2, 1000, device=cuda), 65)  # k > 64


def test_sampling_mode_serves_torch_topk_on_cuda(cuda):
    """Inside the verify sampling's context, torch.topk on the CUDA verify rows returns topk_rows' result: the
    oracle's indices (bf16 rows hold ties: the torch-XPU tie order) and torch's own values."""
    from mono_b200 import _C, sampling
    g = torch.Generator().manual_seed(12)
    lg0 = (torch.randn(8, 248320, generator=g) * 3).bfloat16().to(cuda)
    before = sampling.stats()["calls"]
    ctx, rows = sampling.verify_rows(_C, lg0)
    with ctx:
        v, i = torch.topk(rows, 64)
    assert sampling.stats()["calls"] == before + 1
    rv, ri = ref_topk_rows(lg0.float().cpu().numpy(), 64)
    assert np.array_equal(i.cpu().numpy(), ri) and torch.equal(v, torch.topk(lg0.float(), 64).values)
