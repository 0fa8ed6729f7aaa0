"""The GDN oracle's conv and gates against direct restatements (csrc/mono_gdn.sycl:313-375, :427-456)."""
import numpy as np

from oracle import gdn as og
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits


def test_conv_state_is_the_newest_inputs_and_delta_rule_reduces_to_outer_products():
    rng = np.random.default_rng(3)
    HK, HV, M = 1, 2, 3
    C = (2 * HK + HV) * 128
    bits = lambda a: f32_to_bf16_bits(np.asarray(a, dtype=np.float32))
    qkv = bits(rng.standard_normal((M, C)))
    hist = bits(rng.standard_normal((C, 3)))
    z = bits(rng.standard_normal((M, HV * 128)))
    a = bits(np.full((M, HV), -50.0))  # softplus ~ 0: decay = 1
    b = bits(np.full((M, HV), 50.0))   # beta = 1
    w = bits(np.zeros((C, 4)))
    st = np.zeros((HV, 128, 128), dtype=np.float32)
    core, new_hist, S = og.gdn_step(qkv, z, a, b, w, hist, np.zeros(HV, np.float32), -np.ones(HV, np.float32), st,
                                    bits(np.ones(128)), 1e-6, 128 ** -0.5, HK)
    assert np.array_equal(new_hist, qkv[-3:].T)
    # zero conv weights: every conv output is silu(0) = 0, so k = 0 and the state stays 0
    assert np.abs(S).max() == 0 and np.abs(core).max() == 0


def test_ab_projection_follows_its_pinned_order():
    """The a|b oracle against a direct restatement of its order (one column, scalar loops) and against fp64 within
    one bf16 rounding plus the fp32 accumulation error."""
    import numpy as np

    from oracle.gdn import ab_projection
    from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits
    r = np.random.default_rng(7)
    M, N, K = 2, 3, 2048
    x = f32_to_bf16_bits(r.standard_normal((M, K)).astype(np.float32))
    w = f32_to_bf16_bits((r.standard_normal((N, K)) * 0.05).astype(np.float32))
    got = ab_projection(x, w)
    xf, wf = bf16_bits_to_f32(x).astype(np.float32), bf16_bits_to_f32(w).astype(np.float32)
    J4 = K // 1024
    for m in range(M):
        for n in range(N):
            Q = []
            for q in range(4):
                lanes = []
                for lane in range(32):
                    acc = np.float32(0)
                    for j in range(q * J4, (q + 1) * J4):
                        for e in range(8):
                            k = 256 * j + 8 * lane + e
                            acc = np.float32(acc + np.float32(xf[m, k] * wf[n, k]))
                    lanes.append(acc)
                v = np.array(lanes, dtype=np.float32)
                for o in (16, 8, 4, 2, 1):
                    v = (v + v[np.arange(32) ^ o]).astype(np.float32)
                Q.append(v[0])
            ref = np.float32(np.float32(np.float32(Q[0] + Q[1]) + Q[2]) + Q[3])
            assert got[m, n] == f32_to_bf16_bits(np.array([ref], dtype=np.float32))[0]
    exact = xf.astype(np.float64) @ wf.astype(np.float64).T
    assert np.allclose(bf16_bits_to_f32(got), exact, rtol=2 ** -7, atol=1e-4)


def test_gdn_tree_oracle_reduces_to_the_chain():
    """The tree oracle on a chain program equals the committing oracle (consistency of the restatement)."""
    HK, HV, D = 2, 4, 128
    C = (2 * HK + HV) * D
    rng = np.random.default_rng(3)
    from oracle.numerics import f64_to_bf16_bits
    bits = lambda *s: f64_to_bf16_bits(rng.standard_normal(s))
    qkv, z, a, b = bits(5, C), bits(5, HV * D), bits(5, HV), bits(5, HV)
    conv_w, conv_state = f64_to_bf16_bits(rng.standard_normal((C, 4)) * 0.5), bits(C, 3)
    dt, gd = np.zeros(HV, np.float32), -np.ones(HV, np.float32)
    state = (rng.standard_normal((HV, D, D)) * 0.1).astype(np.float32)
    gw = f64_to_bf16_bits(1 + rng.standard_normal(D) * 0.1)
    ref, _, _ = og.gdn_step(qkv, z, a, b, conv_w, conv_state, dt, gd, state, gw, 1e-6, D ** -0.5, HK)
    par, prog = og.chain_program(5)
    got, _, _ = og.gdn_step_tree(qkv, z, a, b, conv_w, conv_state, dt, gd, state, gw, 1e-6, D ** -0.5, HK, par, prog)
    assert np.allclose(got, ref, rtol=0, atol=0)


def test_tree_program_of_tree4s1m8():
    """tree4s1m8 (parents -1 0 1 2 3 2 1 0): each chain node commits and is followed by its leaf."""
    assert og.tree_program([-1, 0, 1, 2, 3, 2, 1, 0], 8) == [32, 7, 33, 6, 34, 5, 35, 36]
    assert og.chain_program(5) == ([-1, 0, 1, 2, 3, -1, -1, -1], [32, 33, 34, 35, 36, -1, -1, -1])
