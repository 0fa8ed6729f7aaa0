"""Gated-DeltaNet decode step on the GPU (through the C ABI) against the fp64 oracle (oracle/gdn.py), BASELINE
configs[3] shapes: 16 key heads, 32 value heads, d = 128, state ~ N(0, 0.1), M in {1, 3, 8} sequential rows.
Tolerances (fp32 kernel vs fp64 with the reference's explicit bf16 roundings applied in both):
    core:        max |out - ref| <= 2^-6 |ref| + 2e-3,  mean |out - ref| <= 2e-3 mean |ref|
    state:       |S - S_ref| <= 1e-4 (1 + |S_ref|)
    conv state:  bit-exact (a copy of the newest inputs)"""
import numpy as np
import pytest
import torch

from conftest import bf16_bits
from oracle import gdn as og
from oracle.numerics import bf16_bits_to_f32

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M", [1, 3, 8])
@pytest.mark.parametrize("seed", [0, 1])
def test_gdn_step_within_tolerance_of_fp64(cuda, M, seed):
    from mono_b200 import _C
    HK, HV, D = 16, 32, 128
    C = (2 * HK + HV) * D
    g = torch.Generator().manual_seed(0x5EED + 3 + 10 * M + seed)
    qkv = torch.randn(M, C, generator=g).bfloat16()
    z = torch.randn(M, HV * D, generator=g).bfloat16()
    a = torch.randn(M, HV, generator=g).bfloat16()
    b = torch.randn(M, HV, generator=g).bfloat16()
    conv_w = (torch.randn(C, 4, generator=g) * 0.5).bfloat16()
    conv_state = torch.randn(C, 3, generator=g).bfloat16()
    dt_bias = torch.randn(HV, generator=g) * 0.1 if seed else torch.zeros(HV)
    g_decay = -torch.exp(torch.randn(HV, generator=g) * 0.5) if seed else -torch.ones(HV)
    state = torch.randn(HV, D, D, generator=g) * 0.1
    gw = (1 + torch.randn(D, generator=g) * 0.1).bfloat16()
    qscale = D ** -0.5
    core_ref, hist_ref, state_ref = og.gdn_step(bf16_bits(qkv), bf16_bits(z), bf16_bits(a), bf16_bits(b),
                                                bf16_bits(conv_w), bf16_bits(conv_state), dt_bias.numpy(),
                                                g_decay.numpy(), state.numpy(), bf16_bits(gw), 1e-6, qscale, HK)
    cs, st = conv_state.to(cuda), state.to(cuda)
    core = _C.gdn_step(qkv.to(cuda), z.to(cuda), a.to(cuda), b.to(cuda), conv_w.to(cuda), cs, dt_bias.to(cuda),
                       g_decay.to(cuda), st, gw.to(cuda), 1e-6, qscale, HK)
    o = bf16_bits_to_f32(bf16_bits(core)).astype(np.float64)
    err = np.abs(o - core_ref)
    assert np.isfinite(o).all()
    assert (err <= 2 ** -6 * np.abs(core_ref) + 2e-3).all(), err.max()
    assert err.mean() <= 2e-3 * np.abs(core_ref).mean(), err.mean()
    assert np.array_equal(bf16_bits(cs), hist_ref)
    serr = np.abs(st.cpu().numpy().astype(np.float64) - state_ref)
    assert (serr <= 1e-4 * (1 + np.abs(state_ref))).all(), serr.max()


def test_gdn_deferred_replay_then_verify(cuda):
    """Step 1 verifies 5 rows without persisting; step 2 replays 3 of them (slots 0, 1, 2, as an accept of a
    chain writes them) and verifies 4 new rows. Reference: the committing oracle on the replayed rows, then on the
    verify rows from a copy of that state."""
    from mono_b200 import _C
    HK, HV, D = 16, 32, 128
    C = (2 * HK + HV) * D
    g = torch.Generator().manual_seed(77)
    rnd = lambda *s: torch.randn(*s, generator=g).bfloat16()
    conv_w = (torch.randn(C, 4, generator=g) * 0.5).bfloat16()
    conv_state = rnd(C, 3)
    dt_bias, g_decay = torch.randn(HV, generator=g) * 0.1, -torch.exp(torch.randn(HV, generator=g) * 0.5)
    state = torch.randn(HV, D, D, generator=g) * 0.1
    gw = (1 + torch.randn(D, generator=g) * 0.1).bfloat16()
    qs = D ** -0.5
    rows1 = (rnd(5, C), rnd(5, HV * D), rnd(5, HV), rnd(5, HV))
    rows2 = (rnd(4, C), rnd(4, HV * D), rnd(4, HV), rnd(4, HV))
    bufs = [(torch.zeros(8, C, dtype=torch.bfloat16, device=cuda), torch.zeros(8, HV, dtype=torch.bfloat16, device=cuda),
             torch.zeros(8, HV, dtype=torch.bfloat16, device=cuda)) for _ in range(2)]
    ctl = torch.zeros(26, dtype=torch.int32, device=cuda)
    par, prog = og.chain_program(5)
    ctl[10:26] = torch.tensor(par + prog, dtype=torch.int32)
    cs, st = conv_state.to(cuda), state.to(cuda)
    args = (conv_w.to(cuda), cs, dt_bias.to(cuda), g_decay.to(cuda), st, gw.to(cuda), 1e-6, qs, HK)
    core1 = _C.gdn_step_deferred(*[t.to(cuda) for t in rows1], *args, ctl, bufs[1], bufs[0])
    assert torch.equal(cs.cpu(), conv_state) and torch.equal(st.cpu(), state)  # nothing persisted
    ref1, _, _ = og.gdn_step(*[bf16_bits(t) for t in rows1], bf16_bits(conv_w), bf16_bits(conv_state), dt_bias.numpy(),
                             g_decay.numpy(), state.numpy(), bf16_bits(gw), 1e-6, qs, HK)
    o1 = bf16_bits_to_f32(bf16_bits(core1)).astype(np.float64)
    assert (np.abs(o1 - ref1) <= 2 ** -6 * np.abs(ref1) + 2e-3).all()
    ctl[0] = 3
    ctl[2:10] = torch.arange(8, dtype=torch.int32)
    par, prog = og.chain_program(4)
    ctl[10:26] = torch.tensor(par + prog, dtype=torch.int32)
    core2 = _C.gdn_step_deferred(*[t.to(cuda) for t in rows2], *args, ctl, bufs[0], bufs[1])
    rep = tuple(t[:3] for t in rows1)
    _, hist_r, state_r = og.gdn_step(*[bf16_bits(t) for t in rep], bf16_bits(conv_w), bf16_bits(conv_state),
                                     dt_bias.numpy(), g_decay.numpy(), state.numpy(), bf16_bits(gw), 1e-6, qs, HK)
    ref2, _, _ = og.gdn_step(*[bf16_bits(t) for t in rows2], bf16_bits(conv_w), hist_r, dt_bias.numpy(), g_decay.numpy(),
                             state_r.astype(np.float32), bf16_bits(gw), 1e-6, qs, HK)
    o2 = bf16_bits_to_f32(bf16_bits(core2)).astype(np.float64)
    assert (np.abs(o2 - ref2) <= 2 ** -6 * np.abs(ref2) + 2e-3).all(), np.abs(o2 - ref2).max()
    assert np.array_equal(bf16_bits(cs), hist_r)
    assert (np.abs(st.cpu().numpy() - state_r) <= 1e-4 * (1 + np.abs(state_r))).all()


# tree4s1m8 (the reference test's spec, tests/test_mtp_accept.py:46-47): the chain 0-1-2-3-4 with one leaf beside
# each of rows 1, 2, 3 (rows 7, 6, 5, whose parents are 0, 1, 2)
TREE8_PARENTS = [-1, 0, 1, 2, 3, 2, 1, 0]


@pytest.mark.parametrize("path", [[0, 1, 6], [0, 7], [0, 1, 2, 3, 4], [0]])
def test_gdn_deferred_tree_verify_then_replay_off_chain(cuda, path):
    """Step 1 verifies the 8-node tree (each row's conv over its ancestors, leaves from temporaries); step 2 replays
    an accepted path of step 1 (possibly ending on a leaf) and verifies the tree again. Reference: oracle
    gdn_step_tree (fp64), same tolerances as above; the conv state is bit-exact."""
    from mono_b200 import _C
    HK, HV, D = 16, 32, 128
    C = (2 * HK + HV) * D
    g = torch.Generator().manual_seed(1000 + len(path) + path[-1])
    rnd = lambda *s: torch.randn(*s, generator=g).bfloat16()
    conv_w = (torch.randn(C, 4, generator=g) * 0.5).bfloat16()
    conv_state = rnd(C, 3)
    dt_bias, g_decay = torch.randn(HV, generator=g) * 0.1, -torch.exp(torch.randn(HV, generator=g) * 0.5)
    state = torch.randn(HV, D, D, generator=g) * 0.1
    gw = (1 + torch.randn(D, generator=g) * 0.1).bfloat16()
    qs = D ** -0.5
    prog = og.tree_program(TREE8_PARENTS, 8)
    rows1 = (rnd(8, C), rnd(8, HV * D), rnd(8, HV), rnd(8, HV))
    rows2 = (rnd(8, C), rnd(8, HV * D), rnd(8, HV), rnd(8, HV))
    bufs = [(torch.zeros(8, C, dtype=torch.bfloat16, device=cuda), torch.zeros(8, HV, dtype=torch.bfloat16, device=cuda),
             torch.zeros(8, HV, dtype=torch.bfloat16, device=cuda)) for _ in range(2)]
    ctl = torch.zeros(26, dtype=torch.int32, device=cuda)
    ctl[10:26] = torch.tensor(TREE8_PARENTS + prog, dtype=torch.int32)
    cs, st = conv_state.to(cuda), state.to(cuda)
    args = (conv_w.to(cuda), cs, dt_bias.to(cuda), g_decay.to(cuda), st, gw.to(cuda), 1e-6, qs, HK)
    common = (bf16_bits(conv_w), bf16_bits(conv_state), dt_bias.numpy(), g_decay.numpy(), state.numpy(), bf16_bits(gw),
              1e-6, qs, HK)
    core1 = _C.gdn_step_deferred(*[t.to(cuda) for t in rows1], *args, ctl, bufs[1], bufs[0])
    ref1, _, _ = og.gdn_step_tree(*[bf16_bits(t) for t in rows1], *common, TREE8_PARENTS, prog)
    o1 = bf16_bits_to_f32(bf16_bits(core1)).astype(np.float64)
    assert (np.abs(o1 - ref1) <= 2 ** -6 * np.abs(ref1) + 2e-3).all(), np.abs(o1 - ref1).max()
    assert torch.equal(cs.cpu(), conv_state) and torch.equal(st.cpu(), state)  # nothing persisted
    # step 2: replay the accepted path (slots of step 1), verify the tree again
    ctl[0] = len(path)
    ctl[2:10] = torch.tensor(path + list(range(len(path), 8)), dtype=torch.int32)
    core2 = _C.gdn_step_deferred(*[t.to(cuda) for t in rows2], *args, ctl, bufs[0], bufs[1])
    rep = tuple(bf16_bits(t)[path] for t in (rows1[0], rows1[2], rows1[3]))
    ref2, hist2, state2 = og.gdn_step_tree(*[bf16_bits(t) for t in rows2], *common, TREE8_PARENTS, prog, replay=rep)
    o2 = bf16_bits_to_f32(bf16_bits(core2)).astype(np.float64)
    assert (np.abs(o2 - ref2) <= 2 ** -6 * np.abs(ref2) + 2e-3).all(), np.abs(o2 - ref2).max()
    assert np.abs(o2 - ref2).mean() <= 2e-3 * np.abs(ref2).mean()
    assert np.array_equal(bf16_bits(cs), hist2)
    assert (np.abs(st.cpu().numpy() - state2) <= 1e-4 * (1 + np.abs(state2))).all()


def test_deferred_streams_equal_one_stream_calls(cuda):
    """mono_gdn_step_deferred_streams: two streams in one launch pair give exactly the two one-stream calls'
    outputs, states, conv states and saved rows (different replay counts per stream)."""
    from mono_b200 import _C
    HK, HV, M, B = 4, 8, 8, 2
    C = (2 * HK + HV) * 128
    g = torch.Generator().manual_seed(5)
    r = lambda *s, sc=1.0: (torch.randn(*s, generator=g) * sc)  # noqa: E731
    qkv = r(B * M, C).bfloat16().to(cuda)
    z = r(B * M, HV * 128).bfloat16().to(cuda)
    ab = r(B * M, 2 * HV).bfloat16().to(cuda)
    conv_w = r(C, 4, sc=0.5).bfloat16().to(cuda)
    conv = r(B, C, 3).bfloat16().to(cuda)
    dt = r(HV, sc=0.1).to(cuda)
    gd = -r(HV).abs().to(cuda)
    state = r(B, HV, 128, 128, sc=0.1).to(cuda)
    gw = (1 + r(128, sc=0.1)).bfloat16().to(cuda)
    prev = (r(B, 8, C).bfloat16().to(cuda), r(B, 8, HV).bfloat16().to(cuda), r(B, 8, HV).bfloat16().to(cuda))
    save = tuple(torch.zeros_like(t) for t in prev)
    ctl = torch.zeros(B, 26, dtype=torch.int32)
    prog = og.tree_program(TREE8_PARENTS, 8)
    for b, path in enumerate(([0, 1, 6], [0])):  # accepted paths of the previous step, replayed first
        ctl[b, 0] = len(path)
        ctl[b, 2:10] = torch.tensor(path + list(range(len(path), 8)), dtype=torch.int32)
        ctl[b, 10:26] = torch.tensor(TREE8_PARENTS + prog, dtype=torch.int32)
    ctl = ctl.to(cuda)
    ones = [dict(conv=conv[b].clone(), state=state[b].clone(), save=tuple(torch.zeros_like(t[b]) for t in prev))
            for b in range(B)]
    core = _C.gdn_step_deferred(qkv, z, ab[:, :HV], ab[:, HV:], conv_w, conv, dt, gd, state, gw, 1e-6, 128 ** -0.5, HK,
                                ctl, prev, save, streams=B)
    for b in range(B):
        rows = slice(b * M, (b + 1) * M)
        o = ones[b]
        cb = _C.gdn_step_deferred(qkv[rows], z[rows], ab[rows, :HV], ab[rows, HV:], conv_w, o["conv"], dt, gd,
                                  o["state"], gw, 1e-6, 128 ** -0.5, HK, ctl[b], tuple(t[b] for t in prev), o["save"])
        assert torch.equal(cb, core[rows]), b
        assert torch.equal(o["state"], state[b]) and torch.equal(o["conv"], conv[b])
        for q in range(3):
            assert torch.equal(o["save"][q], save[q][b])
