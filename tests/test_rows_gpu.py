"""Row kernels of the bf16 parts (RMSNorm with residual add, LUT multiply) against fp64 / exact references."""
import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def test_rmsnorm_add_within_one_bf16_rounding_of_fp64(cuda):
    from mono_b200 import _C
    g = torch.Generator().manual_seed(5)
    for M, H in ((1, 4096), (5, 4096), (3, 8192)):
        x = torch.randn(M, H, generator=g).bfloat16()
        a = torch.randn(M, H, generator=g).bfloat16()
        w = (1 + 0.02 * torch.randn(H, generator=g)).bfloat16()
        out, s = _C.rmsnorm_add(x.to(cuda), w.to(cuda), 1e-6, add=a.to(cuda))
        s_ref = (x.float() + a.float()).bfloat16()
        assert torch.equal(s.cpu(), s_ref)  # one bf16 rounding of the sum
        sd = s_ref.double()
        ref = sd / torch.sqrt(sd.pow(2).mean(-1, keepdim=True) + 1e-6) * w.double()
        err = (out.cpu().double() - ref).abs()
        assert (err <= 2 ** -7 * ref.abs() + 1e-6).all()
        only = _C.rmsnorm_add(x.to(cuda), w.to(cuda), 1e-6)
        xd = x.double()
        ref2 = xd / torch.sqrt(xd.pow(2).mean(-1, keepdim=True) + 1e-6) * w.double()
        assert ((only.cpu().double() - ref2).abs() <= 2 ** -7 * ref2.abs() + 1e-6).all()


def test_lut_mul_matches_torch_exactly(cuda):
    from mono_b200 import _C
    silu, sig = _C.act_luts(cuda)
    g = torch.Generator().manual_seed(6)
    gu = torch.randn(3, 2 * 12288, generator=g).bfloat16().to(cuda)
    h = _C.lut_mul(gu[:, 12288:], gu[:, :12288], silu)
    ref = (torch.nn.functional.silu(gu[:, :12288]).float() * gu[:, 12288:].float()).bfloat16()
    assert torch.equal(h, ref)
    y = torch.randn(2, 4096, generator=g).bfloat16().to(cuda)
    qg = torch.randn(2, 16, 512, generator=g).bfloat16().to(cuda).reshape(2, -1)
    out = _C.lut_mul(y, qg[:, 256:], sig, b_head_stride=512)
    ref = (y.float() * torch.sigmoid(qg.view(2, 16, 512)[..., 256:].reshape(2, -1)).float()).bfloat16()
    assert torch.equal(out, ref)


@pytest.mark.parametrize("B", [1, 3])
def test_draft_embed_norm_cat_equals_gather_and_two_norms(cuda, B):
    """mono_draft_embed_norm_cat: the embedding rows of tokens[b, index] and the hidden rows, each RMS-normalized,
    side by side; bit for bit the torch gather + two mono_rmsnorm_add calls. A token outside the vocabulary reads
    row 0 and sets device status 7 (the kernel's own check; no out-of-bounds read)."""
    from mono_b200 import _C
    g = torch.Generator().manual_seed(90 + B)
    V, H = 1000, 4096
    embed = (torch.randn(V, H, generator=g) * 0.02).bfloat16().to(cuda)
    hidden = torch.randn(B, H, generator=g).bfloat16().to(cuda)
    ew = (1 + torch.randn(H, generator=g) * 0.1).bfloat16().to(cuda)
    hw = (1 + torch.randn(H, generator=g) * 0.1).bfloat16().to(cuda)
    tokens = torch.randint(0, V, (B, 9), generator=g).to(cuda)
    for index in (0, 4, 8):
        out = _C.draft_embed_norm_cat(embed, tokens, index, ew, hidden, hw, 1e-6)
        ref_e = _C.rmsnorm_add(embed[tokens[:, index]], ew, 1e-6)
        ref_h = _C.rmsnorm_add(hidden, hw, 1e-6)
        assert torch.equal(out[:, :H], ref_e) and torch.equal(out[:, H:], ref_h), index
    assert _C.device_status() == 0
    bad = tokens.clone()
    bad[0, 2] = V + 5
    out = _C.draft_embed_norm_cat(embed, bad, 2, ew, hidden, hw, 1e-6)
    assert torch.equal(out[0, :H], _C.rmsnorm_add(embed[:1], ew, 1e-6)[0])
    assert _C.device_status() == 7
    assert _C.device_status() == 0  # read and reset
