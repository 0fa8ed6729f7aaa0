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
