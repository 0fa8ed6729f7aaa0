"""Full-attention decode pieces on the GPU (through the C ABI) against the CPU oracle.

qk_norm_rope_kv: bit-exact (pinned head-norm order, the reference's RoPE rounding) incl. the cache writes.
Tree attention: within a stated tolerance of the fp64 reference (tests/test_attn_dpas.py:18-29):
    max |out - ref| <= 8e-3 + 2^-7 |ref|   and   mean |out - ref| <= 1e-3
(one bf16 rounding of the output is 2^-9 |ref|; P is rounded to bf16 before P V)."""
import numpy as np
import pytest
import torch

from conftest import bf16_bits
from oracle import attention as oa
from oracle.numerics import bf16_bits_to_f32

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.contiguous().cpu().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("i", range(36))
def test_qk_norm_rope_kv_bit_exact(cuda, i):
    from mono_b200 import _C
    g = torch.Generator().manual_seed(211 + i)
    S = (1, 3, 8)[i % 3]
    Hq, Hk = ((16, 4), (4, 2), (1, 1))[(i // 3) % 3]
    rd = (64, 128, 256)[(i // 9) % 3]
    kind = i // 27 if i < 27 else 1 + (i % 3)
    qg = torch.randn(1, S, Hq, 512, generator=g)
    k = torch.randn(1, S, Hk, 256, generator=g)
    if kind == 1:
        qg *= torch.exp(torch.randn(qg.shape, generator=g) * 2)
        k *= 30
    elif kind == 2:
        qg *= 1e-4
        k *= 1e-4
    elif kind == 3:
        qg.zero_()
        qg[..., ::2] = -0.0
        k.zero_()
        k[..., ::2] = -0.0
    qg, k = qg.bfloat16(), k.bfloat16()
    v = torch.randn(k.shape, generator=g).bfloat16()
    wq = (1 + torch.randn(256, generator=g) * .3).bfloat16()
    wk = (1 + torch.randn(256, generator=g) * .3).bfloat16()
    f = torch.randn(S, rd // 2, 2, 2, generator=g)
    cap = 64
    pos = torch.randperm(cap, generator=g)[:S]
    key = torch.randn(1, Hk, cap, 256, generator=g).bfloat16()
    val = torch.randn(1, Hk, cap, 256, generator=g).bfloat16()
    ek, ev = _bits(key[0]).copy(), _bits(val[0]).copy()
    rq, rk = oa.qk_norm_rope_kv(_bits(qg[0, :, :, :256]), _bits(k[0]), _bits(v[0]), _bits(wq), _bits(wk), f.numpy(),
                                ek, ev, pos.numpy(), 1e-6, 2e-5, rd)
    kd, vd = key.to(cuda), val.to(cuda)
    qgd = qg.to(cuda)
    oq, ok = _C.qk_norm_rope_kv(qgd[..., :256], k.to(cuda), v.to(cuda), wq.to(cuda), wk.to(cuda), f.to(cuda), kd, vd,
                                pos.to(cuda), 1e-6, 2e-5, rd)
    assert np.array_equal(_bits(oq[0]), rq), i
    assert np.array_equal(_bits(ok[0]), rk), i
    assert np.array_equal(_bits(kd[0]), ek) and np.array_equal(_bits(vd[0]), ev), i


def test_qk_norm_rope_kv_skips_bad_positions(cuda):
    from mono_b200 import _C
    S, Hq, Hk, cap = 2, 4, 2, 16
    qg = torch.randn(1, S, Hq, 512).bfloat16().to(cuda)
    k = torch.randn(1, S, Hk, 256).bfloat16().to(cuda)
    key = torch.zeros(1, Hk, cap, 256, dtype=torch.bfloat16, device=cuda)
    val = torch.zeros_like(key)
    w = torch.ones(256, dtype=torch.bfloat16, device=cuda)
    f = torch.randn(S, 32, 2, 2, device=cuda)
    pos = torch.tensor([3, cap + 5], dtype=torch.int64, device=cuda)
    _C.device_status(reset=True)
    _C.qk_norm_rope_kv(qg[..., :256], k, k, w, w, f, key, val, pos, 1e-6, 1e-6, 64)
    assert _C.device_status(reset=True) == 4
    assert key[0, :, 3].abs().sum() > 0 and key[0, :, 4:].abs().sum() == 0


CASES = [
    (0, 512, [-1, 0, 1]),
    (63, 4096, [-1, 0, 1, 2, 3, 4, 5, 6]),
    (777, 4096, [-1, 0, 0, 0, 0, 1, 1, 1]),
    (2048, 4096, [-1, 0, 1, 2, 3, 4, 5, 6]),
    (3500, 11400, [-1, 0, 1, 2, 3, 4, 5, 6]),
    (8192, 8200, [-1, 0, 1, 1, 2, 3, 3, 4]),
    (11400, 11400, [-1, 0, 1, 2, 3, 4, 5, 6]),
    (1000, 4096, None),
    (8000, 11400, None),
    (1, 64, [-1, 0]),
]


@pytest.mark.parametrize("L,cap,parents", CASES)
def test_tree_attention_within_tolerance_of_fp64(cuda, L, cap, parents):
    from mono_b200 import _C
    H, HK, D = 16, 4, 256
    g = torch.Generator().manual_seed(L + cap)
    S = 1 if parents is None else len(parents)
    q = (torch.randn(1, H, S, D, generator=g) * 2).to(torch.bfloat16)
    k = (torch.randn(1, HK, cap, D, generator=g) * 1.5).to(torch.bfloat16)
    v = torch.randn(1, HK, cap, D, generator=g).to(torch.bfloat16)
    xk = (torch.randn(1, HK, S, D, generator=g) * 1.5).to(torch.bfloat16)
    xv = torch.randn(1, HK, S, D, generator=g).to(torch.bfloat16)
    mask = None if parents is None else oa.tree_mask(parents)
    ref = oa.attention_fp64(_bits(q[0]), _bits(k[0]), _bits(v[0]), L, _bits(xk[0]), _bits(xv[0]), mask)
    mt = torch.empty(0, dtype=torch.int32) if mask is None else torch.tensor(mask, dtype=torch.int32)
    sl = torch.tensor([L], dtype=torch.int32)
    out = _C.attn_dpas(q.to(cuda), k.to(cuda), v.to(cuda), sl.to(cuda), xk.to(cuda), xv.to(cuda), mt.to(cuda))
    o = bf16_bits_to_f32(bf16_bits(out[0])).astype(np.float64)
    err = np.abs(o - ref)
    assert np.isfinite(o).all()
    assert (err <= 8e-3 + 2 ** -7 * np.abs(ref)).all(), (err.max(), (err - 2 ** -7 * np.abs(ref)).max())
    assert err.mean() <= 1e-3, err.mean()


@pytest.mark.parametrize("S,lens", [(8, (1030, 517)), (1, (1000, 64)), (8, (0, 300))])
def test_batched_streams_equal_one_stream_calls(cuda, S, lens):
    """qk_norm_rope_kv and tree attention over two batched streams (mono_*_streams: stacked heads, one length per
    stream) give exactly each stream's one-stream results, caches included."""
    from mono_b200 import _C
    H, HK, D, cap, B = 16, 4, 256, 1152, 2
    g = torch.Generator().manual_seed(S + lens[0])
    qg = torch.randn(1, B * S, H, 512, generator=g).bfloat16().to(cuda)
    rk = torch.randn(1, B * S, HK, D, generator=g).bfloat16().to(cuda)
    v = torch.randn(1, B * S, HK, D, generator=g).bfloat16().to(cuda)
    wq = (1 + torch.randn(D, generator=g) * .3).bfloat16().to(cuda)
    wk = (1 + torch.randn(D, generator=g) * .3).bfloat16().to(cuda)
    f = torch.randn(B * S, 32, 2, 2, generator=g).to(cuda)
    kc = torch.randn(1, B * HK, cap, D, generator=g).bfloat16().to(cuda)
    vc = torch.randn(1, B * HK, cap, D, generator=g).bfloat16().to(cuda)
    pos = torch.cat([torch.arange(S) + lens[b] for b in range(B)]).to(cuda)
    mask = torch.tensor(oa.tree_mask([-1, 0, 1, 2, 3, 0, 5, 1][:S]) if S > 1 else [], dtype=torch.int32).to(cuda)
    seq = torch.tensor(lens, dtype=torch.int32).to(cuda)
    kc1, vc1 = kc.clone(), vc.clone()
    q, k = _C.qk_norm_rope_kv(qg[..., :D], rk, v, wq, wk, f, kc, vc, pos, 1e-6, 1e-6, 64, streams=B)
    xv = v.view(B, S, HK, D).permute(0, 2, 1, 3).reshape(1, B * HK, S, D)
    out = _C.attn_dpas(q, kc, vc, seq, k, xv, mask, streams=B)
    for b in range(B):
        rows = slice(b * S, (b + 1) * S)
        heads = slice(b * HK, (b + 1) * HK)
        kcb, vcb = kc1[:, heads].contiguous(), vc1[:, heads].contiguous()
        qb, kb = _C.qk_norm_rope_kv(qg[:, rows, :, :D], rk[:, rows], v[:, rows], wq, wk, f[rows].contiguous(), kcb, vcb,
                                    pos[rows].contiguous(), 1e-6, 1e-6, 64)
        assert torch.equal(qb[0], q[0, b * H:(b + 1) * H]) and torch.equal(kb[0], k[0, heads])
        assert torch.equal(kcb, kc[:, heads]) and torch.equal(vcb, vc[:, heads])
        ob = _C.attn_dpas(qb, kcb, vcb, seq[b:b + 1], kb, v[:, rows].transpose(1, 2), mask)
        assert torch.equal(ob[0], out[0, rows]), b
