"""bf16 GEMV of the draft head's projections on the GPU (include/mono_b200.h mono_gemv_bf16) against an fp64
product of the same bf16 operands. The reference computes these projections with torch's bf16 F.linear (fp32
accumulation, library-chosen order), so the contract is a tolerance, not bits: |out - ref| <= 2^-8 |ref| +
1e-3 max|ref| (the bf16 rounding of the output plus fp32 summation error over K terms)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _within(out, ref):
    ref = ref.double()
    err = (out.double().cpu() - ref).abs()
    bound = ref.abs() * 2.0 ** -8 + 1e-3 * ref.abs().max()
    return bool((err <= bound).all()), float((err / bound).max())


# the draft head's shapes (fc, qkv, o, gate | up, down at H = 4096, I = 12288) and small / ragged ones
@pytest.mark.parametrize("M,N,K", [(1, 4096, 8192), (1, 12288, 4096), (1, 4096, 4096), (1, 24576, 4096),
                                   (1, 4096, 12288), (2, 1003, 256), (5, 777, 2304), (8, 4096, 4096), (3, 64, 768)])
def test_gemv_bf16_within_tolerance_of_fp64(cuda, M, N, K):
    from mono_b200 import _C
    g = torch.Generator().manual_seed(M * 7 + N + K)
    x = torch.randn(M, K, generator=g).bfloat16()
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16()
    ref = x.double() @ w.double().t()
    out = _C.gemv_bf16(x.to(cuda), w.to(cuda))
    ok, worst = _within(out, ref)
    assert ok, worst


def test_gemv_bf16_strided_rows(cuda):
    """x a column window of wider rows, out a column window of a wider buffer (as the draft head writes its
    projections into slices): the columns outside the window stay untouched."""
    from mono_b200 import _C
    g = torch.Generator().manual_seed(11)
    M, N, K = 4, 2048, 4096
    wide = torch.randn(M, K + 512, generator=g).bfloat16().to(cuda)
    w = (torch.randn(N, K, generator=g) * 0.02).bfloat16().to(cuda)
    buf = torch.full((M, N + 128), 7.0, dtype=torch.bfloat16, device=cuda)
    x = wide[:, 256:256 + K]
    _C.gemv_bf16(x, w, out=buf[:, 64:64 + N])
    ok, worst = _within(buf[:, 64:64 + N], x.double().cpu() @ w.double().cpu().t())
    assert ok, worst
    assert bool((buf[:, :64] == 7.0).all()) and bool((buf[:, 64 + N:] == 7.0).all())


def test_gemv_bf16_rejects(cuda):
    from mono_b200 import _C, _lib
    w = torch.zeros(64, 4096, dtype=torch.bfloat16, device=cuda)
    with pytest.raises(_lib.MonoError):
        _C.gemv_bf16(torch.zeros(9, 4096, dtype=torch.bfloat16, device=cuda), w)  # M > 8
    with pytest.raises(_lib.MonoError):
        _C.gemv_bf16(torch.zeros(1, 1000, dtype=torch.bfloat16, device=cuda), torch.zeros(64, 1000, dtype=torch.bfloat16,
                                                                                           device=cuda))  # K % 256
