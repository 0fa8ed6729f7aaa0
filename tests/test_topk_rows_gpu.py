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
    """Inside the verify sampling's context, torch.topk on the CUDA verify rows returns topk_rows' result in the
    ascending-index tie order: torch's own values bit for bit, and for k = 64 torch's own CUDA indices too (the rows
    come from bf16 logits: ties everywhere); a call the ABI rejects (k > 64) runs torch's topk, the piece stays on."""
    from mono_b200 import _C, guard, sampling
    g = torch.Generator().manual_seed(12)
    lg0 = (torch.randn(8, 248320, generator=g) * 3).bfloat16().to(cuda)
    before = sampling.stats()
    ctx, rows = sampling.verify_rows(_C, lg0)
    with ctx:
        v, i = torch.topk(rows, 64)
        vb, ib = lg0.topk(20)
        big = torch.topk(rows, 100)
    after = sampling.stats()
    assert after["calls"] == before.get("calls", 0) + 2 and after["rejected"] == before.get("rejected", 0) + 1
    assert not guard.off(sampling.PIECE)
    ref = torch.topk(rows, 64)
    assert torch.equal(v, ref.values) and torch.equal(i, ref.indices)
    rv, ri = ref_topk_rows(lg0.float().cpu().numpy(), 64, index_order=True)
    assert np.array_equal(i.cpu().numpy(), ri)
    assert vb.dtype == torch.bfloat16 and torch.equal(vb, torch.topk(lg0, 20).values)
    assert np.array_equal(ib.cpu().numpy(), ri[:, :20])
    assert torch.equal(big.values, torch.topk(rows, 100).values)


@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16])
def test_index_order_matches_torch_cuda_for_k_above_32(cuda, dtype):
    """MONO_TOPK_INDEX_ORDER on tie-heavy rows against torch's own CUDA topk (k in 33..64) and the oracle."""
    from mono_b200 import _C
    g = torch.Generator().manual_seed(21)
    x = torch.randint(-3, 4, (5, 70000), generator=g).float()
    x[1, ::3] = -0.0
    x[2] = 0.0
    x[2, 1::2] = -0.0
    x = x.to(dtype).to(cuda)
    for k in (33, 40, 64):
        v, i = _C.topk_rows(x, k, index_order=True)
        ref = torch.topk(x.float(), k)
        assert torch.equal(i, ref.indices) and torch.equal(v, ref.values), k
        rv, ri = ref_topk_rows(x.float().cpu().numpy(), k, index_order=True)
        assert np.array_equal(i.cpu().numpy(), ri), k
