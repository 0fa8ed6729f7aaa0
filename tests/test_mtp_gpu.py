"""MTP loop bookkeeping on the GPU against the oracle (oracle/mtp.py, itself pinned to the reference's host walk):
accept walk, result row, counters, ctl, next token / hidden row, KV slot moves (bit-exact); prep kernels."""
import random

import numpy as np
import pytest
import torch

from oracle import mtp as om

pytestmark = pytest.mark.gpu
SLOTS, H, HK, CAP, D = 8, 64, 4, 96, 256


def _tree(widths_or_spec):
    """parent / children / chain depth of a nested child-list spec, padded to 8 rows."""
    parent, children = [], []

    def add(node, p):
        r = len(parent)
        parent.append(p)
        children.append([])
        if p >= 0:
            children[p].append(r)
        for child in node:
            add(child, r)
    add(widths_or_spec, -1)
    chain = 0
    while children[chain]:
        chain = children[chain][0]
    while len(parent) < SLOTS:
        parent.append(-1)
        children.append([])
    return children, chain


def _spec(widths):
    node = []
    for width in reversed(widths):
        node = [node] + [[] for _ in range(width - 1)]
    return node


SPECS = [_spec(w) for w in ((4, 3), (7,), (1, 1, 1, 1, 1, 1, 1), (2, 2, 3), (3, 1, 1, 2))] + \
        [[[[[[]], []], []], []], [[[[[]]]]]]


@pytest.mark.parametrize("spec_index", range(len(SPECS)))
def test_mtp_accept_matches_oracle(cuda, spec_index):
    from mono_b200 import _C
    rng = random.Random(1000 + spec_index)
    children, chain = _tree(SPECS[spec_index])
    ch = np.full((SLOTS, SLOTS), -1, dtype=np.int32)
    for r, cs in enumerate(children):
        ch[r, :len(cs)] = cs
    chd = torch.from_numpy(ch.reshape(-1)).to(cuda)
    for trial in range(20):
        toks = [rng.randrange(50) for _ in range(SLOTS)]
        dr = [rng.randrange(50) for _ in range(SLOTS)]
        for r in range(SLOTS):
            if children[r] and rng.random() < 0.8:
                dr[rng.choice(children[r])] = toks[r]
        cand = [rng.randrange(50) for _ in range(49)]
        for node in range(chain):
            if rng.random() < 0.7:
                cand[7 * node + rng.randrange(7)] = toks[node]
        pos, mtp_pos = rng.randrange(0, 40), rng.randrange(0, 30)
        x = torch.randn(SLOTS, H).to(torch.bfloat16)
        keys = [torch.randn(HK, CAP, D).to(torch.bfloat16) for _ in range(3)]
        host_keys = [k.view(torch.int16).numpy().copy() for k in keys]
        st_h = np.array([pos, mtp_pos, 0, 0], dtype=np.int64)
        ctl_h = np.zeros(26, dtype=np.int32)
        res_h, nt_h, hrow_h = om.mtp_accept(st_h, toks, dr, cand, ch, SLOTS, chain, x.view(torch.int16).numpy(),
                                            ctl_h, host_keys, CAP)
        st = torch.tensor([pos, mtp_pos, 0, 0], dtype=torch.int64, device=cuda)
        kd = [k.to(cuda) for k in keys]
        ptrs = torch.tensor([k.data_ptr() for k in kd], dtype=torch.int64, device=cuda)
        nt = torch.empty(1, 1, dtype=torch.int64, device=cuda)
        hb = torch.empty(1, 1, H, dtype=torch.bfloat16, device=cuda)
        ctl = torch.zeros(26, dtype=torch.int32, device=cuda)
        result = torch.zeros(32, dtype=torch.int64, device=cuda)
        _C.mtp_accept(st, torch.tensor([toks], device=cuda), torch.tensor([dr], device=cuda),
                      torch.tensor(cand, device=cuda).view(7, 7), chd, SLOTS, chain, x.to(cuda), nt, hb, ctl, ptrs,
                      HK, CAP, D, result)
        r = result.cpu().numpy()
        n = int(res_h[0])
        assert np.array_equal(r[:12 + int(res_h[11])], res_h[:12 + int(res_h[11])]), (trial, r, res_h)
        assert r[19] == res_h[19] and r[20] == res_h[20]
        assert np.array_equal(st.cpu().numpy(), st_h) and np.array_equal(ctl.cpu().numpy(), ctl_h)
        assert nt.item() == nt_h and np.array_equal(hb.view(-1).cpu().view(torch.int16).numpy(), hrow_h)
        for kh, k in zip(host_keys, kd):
            assert np.array_equal(k.cpu().view(torch.int16).numpy(), kh), (trial, n)


def test_mtp_prep_match_oracle(cuda):
    from mono_b200 import _C
    st = torch.tensor([37, 11, 0, 0], dtype=torch.int64, device=cuda)
    ftab = torch.randn(1, 1, 64, 32, 2, 2, device=cuda)
    freqs = torch.empty(1, 1, 1, 32, 2, 2, device=cuda)
    mpos = torch.empty(SLOTS, dtype=torch.int64, device=cuda)
    mseq = torch.empty(1, dtype=torch.int32, device=cuda)
    _C.mtp_prep_draft(st, 2, ftab, freqs, mpos, mseq)
    f_h, mpos_h, mseq_h = om.prep_draft(st.cpu().numpy(), 2, ftab.cpu().numpy().reshape(64, -1), SLOTS)
    assert np.array_equal(freqs.cpu().numpy().reshape(-1), f_h)
    assert list(mpos.cpu().numpy()) == list(mpos_h) and mseq.item() == mseq_h
    apos = torch.empty(SLOTS, dtype=torch.int64, device=cuda)
    aseq = torch.empty(1, dtype=torch.int32, device=cuda)
    vpos = torch.empty(1, 8, dtype=torch.int64, device=cuda)
    tpos = torch.tensor([0, 1, 2, 3, 4, 1, 2, 1], dtype=torch.int64, device=cuda)
    ctl = torch.zeros(26, dtype=torch.int32, device=cuda)
    tctl = torch.arange(100, 116, dtype=torch.int32, device=cuda)
    _C.mtp_prep_verify(st, apos, aseq, vpos, tpos, ctl, tctl, 1, 5)
    ctl_h = np.zeros(26, dtype=np.int32)
    apos_h, aseq_h, vpos_h = om.prep_verify(st.cpu().numpy(), SLOTS, tpos.cpu().numpy(), ctl_h, tctl.cpu().numpy(), 1, 5)
    assert list(apos.cpu().numpy()) == list(apos_h) and aseq.item() == aseq_h
    assert list(vpos.view(-1).cpu().numpy()) == list(vpos_h) and np.array_equal(ctl.cpu().numpy(), ctl_h)


def test_mtp_accept_malformed_children_table_stops_with_status(cuda):
    """A children table whose entry points back to an earlier row (a cycle) ends the walk at that node and sets the
    device status (5), instead of repeating rows or moving a KV slot before it is read."""
    from mono_b200 import _C
    _C.device_status()  # clear
    ch = torch.full((SLOTS, SLOTS), -1, dtype=torch.int32)
    ch[0, 0], ch[1, 0] = 1, 0  # 0 -> 1 -> 0
    toks = torch.tensor([[5, 5, 0, 0, 0, 0, 0, 0]], dtype=torch.int64, device=cuda)
    dr = torch.tensor([[5, 5, 0, 0, 0, 0, 0, 0]], dtype=torch.int64, device=cuda)
    st = torch.tensor([10, 10, 0, 0], dtype=torch.int64, device=cuda)
    x = torch.zeros(SLOTS, 64, dtype=torch.bfloat16, device=cuda)
    nt = torch.zeros(1, 1, dtype=torch.int64, device=cuda)
    hb = torch.zeros(1, 1, 64, dtype=torch.bfloat16, device=cuda)
    ctl = torch.zeros(26, dtype=torch.int32, device=cuda)
    result = torch.zeros(32, dtype=torch.int64, device=cuda)
    ptrs = torch.empty(0, dtype=torch.int64, device=cuda)
    _C.mtp_accept(st, toks, dr, None, ch.reshape(-1).to(cuda), SLOTS, 4, x, nt, hb, ctl, ptrs, 1, 32, 64, result)
    torch.cuda.synchronize()
    assert result[0].item() == 2  # rows 0 and 1, then the bad entry (back to 0) ends the walk
    assert _C.device_status() == 5
    assert _C.device_status() == 0  # (reset by the read)


def test_prep_draft_streams_equals_one_stream_calls(cuda):
    """mono_mtp_prep_draft_streams: one launch for B streams writes each stream's rope row, MTP KV positions and
    length exactly as B one-stream calls do (different counters per stream, one past the table's end)."""
    from mono_b200 import _C
    B, cap, rd = 3, 64, 64
    g = torch.Generator().manual_seed(4)
    rope = torch.randn(cap, rd // 2, 2, 2, generator=g).to(cuda)
    st = torch.tensor([[10, 7, 0, 0], [63, 40, 0, 0], [0, 0, 0, 0]], dtype=torch.int64, device=cuda)
    for k in (0, 2):
        freqs = torch.zeros(B, rd // 2, 2, 2, device=cuda)
        mpos = torch.zeros(B, 1, dtype=torch.int64, device=cuda)
        mseq = torch.zeros(B, dtype=torch.int32, device=cuda)
        _C.mtp_prep_draft_streams(st, k, rope, freqs, mpos, mseq)
        for b in range(B):
            f1 = torch.zeros(1, 1, 1, rd // 2, 2, 2, device=cuda)
            p1 = torch.zeros(1, dtype=torch.int64, device=cuda)
            s1 = torch.zeros(1, dtype=torch.int32, device=cuda)
            _C.mtp_prep_draft(st[b], k, rope.view(1, 1, cap, -1, 2, 2), f1, p1, s1)
            assert torch.equal(freqs[b], f1.view(rd // 2, 2, 2)), (k, b)
            assert torch.equal(mpos[b], p1) and torch.equal(mseq[b:b + 1], s1), (k, b)


def test_prep_verify_streams_equals_one_stream_calls(cuda):
    """mono_mtp_prep_verify_streams: one launch for B streams writes each stream's attention positions / length,
    verify RoPE positions and ctl words exactly as B one-stream calls do."""
    from mono_b200 import _C
    B, R = 3, 8
    st = torch.tensor([[10, 7, 0, 0], [500, 40, 0, 0], [0, 0, 0, 0]], dtype=torch.int64, device=cuda)
    tree_pos = torch.tensor([0, 1, 2, 3, 4, 3, 2, 1], dtype=torch.int64, device=cuda)
    tree_ctl = torch.arange(16, dtype=torch.int32, device=cuda) - 3
    outs = [torch.full((B, R), -9, dtype=torch.int64, device=cuda), torch.full((B,), -9, dtype=torch.int32, device=cuda),
            torch.full((B, R), -9, dtype=torch.int64, device=cuda), torch.full((B, 26), -9, dtype=torch.int32, device=cuda)]
    _C.mtp_prep_verify_streams(st, outs[0], outs[1], outs[2], tree_pos, outs[3], tree_ctl, 1, 5)
    for b in range(B):
        one = [torch.full((R,), -9, dtype=torch.int64, device=cuda), torch.full((1,), -9, dtype=torch.int32, device=cuda),
               torch.full((R,), -9, dtype=torch.int64, device=cuda), torch.full((26,), -9, dtype=torch.int32, device=cuda)]
        _C.mtp_prep_verify(st[b], one[0], one[1], one[2], tree_pos, one[3], tree_ctl, 1, 5)
        assert torch.equal(outs[0][b], one[0]) and torch.equal(outs[1][b:b + 1], one[1]), b
        assert torch.equal(outs[2][b], one[2]) and torch.equal(outs[3][b], one[3]), b
