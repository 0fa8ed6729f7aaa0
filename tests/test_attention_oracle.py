"""The attention oracle pinned to the reference's own CPU functions (golden fixtures made by
tests/golden/make_golden.py from tests/test_rope_kv.py:9-23 and tests/test_attn_dpas.py:11-29)."""
import os

import numpy as np

from oracle import attention as oa

GOLDEN = os.path.join(os.path.dirname(__file__), "golden")


def test_rope_matches_reference_fixture():
    d = np.load(os.path.join(GOLDEN, "rope_kv.npz"))
    for i in range(int(d["n"])):
        y = oa.rope(d[f"x{i}"], d[f"f{i}"], int(d[f"rd{i}"]))
        assert np.array_equal(y, d[f"y{i}"]), i


def test_tree_mask_and_fp64_attention_match_reference_fixture():
    d = np.load(os.path.join(GOLDEN, "attn_fp64.npz"))
    parents = {1: [-1, 0, 1, 2, 3, 4, 5, 6], 2: [-1, 0, 0, 0, 0, 1, 1, 1]}
    for i in range(int(d["n"])):
        mask = [int(m) for m in d[f"mask{i}"]] or None
        if i in parents:
            assert oa.tree_mask(parents[i]) == mask
        out = oa.attention_fp64(d[f"q{i}"], d[f"k{i}"], d[f"v{i}"], int(d[f"L{i}"]), d[f"xk{i}"], d[f"xv{i}"], mask)
        np.testing.assert_allclose(out, d[f"ref{i}"], rtol=1e-12, atol=1e-12)


def test_head_rmsnorm_close_to_fp64():
    g = np.random.default_rng(5)
    x = g.standard_normal((8, 16, 256)).astype(np.float32) * np.exp(g.standard_normal((8, 16, 1)).astype(np.float32))
    from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits
    xb = f32_to_bf16_bits(x)
    w = f32_to_bf16_bits((1 + 0.3 * g.standard_normal(256)).astype(np.float32))
    y = bf16_bits_to_f32(oa.head_rmsnorm(xb, w, 1e-6)).astype(np.float64)
    xf = bf16_bits_to_f32(xb).astype(np.float64)
    ref = xf / np.sqrt((xf * xf).mean(-1, keepdims=True) + 1e-6) * bf16_bits_to_f32(w).astype(np.float64)
    assert np.max(np.abs(y - ref) / (np.abs(ref) + 1e-30)) < 2 ** -7
