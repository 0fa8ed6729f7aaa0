"""The MTP accept oracle pinned to the reference's own host walk (golden fixture made by
tests/golden/make_golden.py from comfy_mono_decode_xpu/mtp_loop.py:117-136 on the tree specs of
tests/test_mtp_accept.py)."""
import os

import numpy as np

from oracle import mtp as om

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_accept_walk_matches_reference_fixture():
    d = np.load(os.path.join(GOLDEN, "accept_walk.npz"))
    assert int(d["n"]) >= 80
    for k in range(int(d["n"])):
        ch = d[f"children{k}"]
        children = [[int(c) for c in row if c >= 0] for row in ch]
        got = om.accept_walk(children, list(d[f"toks{k}"]), list(d[f"dr{k}"]), int(d[f"depth{k}"]), list(d[f"cand{k}"]))
        path, commit, ranks, row, on_chain, kept = got
        assert path == list(d[f"path{k}"]) and commit == list(d[f"commit{k}"]), k
        assert ranks == list(d[f"ranks{k}"]) and row == int(d[f"row{k}"]), k
        assert int(on_chain) == int(d[f"on_chain{k}"]) and kept == int(d[f"kept{k}"]), k


def test_prep_models():
    st = np.array([37, 11, 0, 0], dtype=np.int64)
    ftab = np.arange(64 * 4, dtype=np.float32).reshape(64, 4)
    f, mpos, mseq = om.prep_draft(st, 2, ftab, 8)
    assert np.array_equal(f, ftab[39]) and list(mpos) == list(range(13, 21)) and mseq == 14
    ctl = np.zeros(26, dtype=np.int32)
    apos, aseq, vpos = om.prep_verify(st, 8, [0, 1, 2, 3, 4, 1, 2, 1], ctl, np.arange(100, 116), 1, 5)
    assert list(apos) == list(range(37, 45)) and aseq == 37
    assert list(vpos) == [37 + 5 + d for d in [0, 1, 2, 3, 4, 1, 2, 1]]
    assert ctl[1] == 1 and list(ctl[10:]) == list(range(100, 116))
