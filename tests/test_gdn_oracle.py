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
