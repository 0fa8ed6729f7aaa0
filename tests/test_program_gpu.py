"""Layer programs on the GPU (include/mono_b200.h mono_program_*, mono_layer_post_gptq, mono_layer_gdn_gptq): one
persistent launch gives the same bits as the standalone entry points it fuses (mono_rowlin_gptq + mono_mlp_gptq;
mono_rowlin_gptq + mono_gdn_ab + mono_gdn_step_deferred + mono_rowlin_gptq + mono_mlp_gptq), with and without the
L2 prefetch; the a | b projection matches the CPU oracle bit for bit; the synthetic decoder gives the same tokens
and hidden rows through 9 layer programs as through its op-by-op path."""
import numpy as np
import pytest
import torch

from conftest import bf16_bits
from oracle import gdn as og

pytestmark = pytest.mark.gpu

H, I = 4096, 12288


def _w4(N, K, g, cuda):
    from mono_b200 import _C
    packed = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, generator=g).to(cuda)
    scales = (torch.randn(N, K // 128, generator=g).abs() * (0.02 / 7) + 1e-4).half().to(cuda)
    return _C.w4_repack(0, packed, scales, N, K)


def _bf(g, *shape, std=1.0, mean=0.0):
    return (torch.randn(*shape, generator=g) * std + mean).bfloat16()


@pytest.mark.parametrize("M", [1, 5, 16])
def test_gdn_ab_matches_oracle(cuda, M):
    from mono_b200 import _C
    g = torch.Generator().manual_seed(40 + M)
    x, w = _bf(g, M, H), _bf(g, 64, H, std=0.02)
    out = _C.gdn_ab(x.to(cuda), w.to(cuda))
    assert np.array_equal(bf16_bits(out), og.ab_projection(bf16_bits(x), bf16_bits(w)))
    # a column slice of wider rows (the decoder's normalized rows live in their own buffer; any row stride works)
    wide = _bf(g, M, H + 1024)
    out2 = _C.gdn_ab(wide.to(cuda)[:, 512:512 + H], w.to(cuda))
    assert np.array_equal(bf16_bits(out2), og.ab_projection(bf16_bits(wide[:, 512:512 + H].contiguous()), bf16_bits(w)))


@pytest.fixture(scope="module")
def mlp_weights(cuda):
    g = torch.Generator().manual_seed(0x5EED + 11)
    return dict(o=_w4(H, 4096, g, cuda), gate=_w4(I, H, g, cuda), up=_w4(I, H, g, cuda), down=_w4(H, I, g, cuda),
                ln2=_bf(g, H, std=0.02, mean=1.0).to(cuda))


@pytest.mark.parametrize("M", [1, 5, 8, 12])
@pytest.mark.parametrize("gated", [True, False])
def test_layer_post_matches_rowlin_then_mlp(cuda, mlp_weights, M, gated):
    from mono_b200 import _C
    W = mlp_weights
    silu, sig = _C.act_luts(cuda)
    g = torch.Generator().manual_seed(M + 100 * gated)
    x = (_bf(g, M, H) * 4).to(cuda)
    y = _bf(g, M, 4096).to(cuda)
    pre = _bf(g, M, 8192).to(cuda)
    gate = pre[:, 256:] if gated else None
    mode = _C.ROWLIN_GATE if gated else _C.ROWLIN_QUANT
    x1 = _C.rowlin_gptq(y, mode, [(W["o"], H)], gate=gate, gate_head_stride=512, lut=sig if gated else None, residual=x)
    ref = _C.mlp_gptq(x1, W["ln2"], 1e-6, W["gate"], W["up"], W["down"], silu_lut=silu, I=I)
    out = _C.layer_post(x, y, W["o"], W["ln2"], 1e-6, W["gate"], W["up"], W["down"], silu, I, gate=gate,
                        sig_lut=sig if gated else None, gate_head_stride=512)
    assert np.array_equal(bf16_bits(out), bf16_bits(ref))
    # in place (out aliases x), as the decoder's residual stream runs
    xi = x.clone()
    _C.layer_post(xi, y, W["o"], W["ln2"], 1e-6, W["gate"], W["up"], W["down"], silu, I, gate=gate,
                  sig_lut=sig if gated else None, gate_head_stride=512, out=xi)
    assert np.array_equal(bf16_bits(xi), bf16_bits(ref))


def _gdn_layer(cuda, seed, HK=16, HV=32):
    g = torch.Generator().manual_seed(seed)
    D = 128
    C = (2 * HK + HV) * D
    L = dict(ln1=_bf(g, H, std=0.02, mean=1.0), qkv=_w4(C, H, g, cuda), z=_w4(HV * D, H, g, cuda),
             wab=_bf(g, 2 * HV, H, std=0.02), conv_w=_bf(g, C, 4, std=0.5), conv_state=_bf(g, C, 3),
             dt_bias=torch.randn(HV, generator=g) * 0.1, g_decay=-torch.exp(torch.randn(HV, generator=g) * 0.5),
             gnorm=_bf(g, D, std=0.1, mean=1.0), state=torch.randn(HV, D, D, generator=g) * 0.1,
             out=_w4(H, HV * D, g, cuda), ln2=_bf(g, H, std=0.02, mean=1.0), gate=_w4(I, H, g, cuda),
             up=_w4(I, H, g, cuda), down=_w4(H, I, g, cuda))
    return {k: v.to(cuda) for k, v in L.items()}, HK, HV, C


def _saved(C, HV, cuda):
    return tuple(torch.zeros(8, n, dtype=torch.bfloat16, device=cuda) for n in (C, HV, HV))


@pytest.mark.parametrize("M", [1, 5, 8])
def test_layer_gdn_matches_op_chain(cuda, M):
    """Two steps of the deferred form (the second replays 3 accepted rows), the whole layer in one launch against
    the op-by-op chain on its own copies of every state; everything bit for bit."""
    from mono_b200 import _C
    L, HK, HV, C = _gdn_layer(cuda, 0x5EED + 12 + M)
    Z = HV * 128
    silu, _ = _C.act_luts(cuda)
    states = {}
    for path in ("chain", "fused"):
        states[path] = dict(cs=L["conv_state"].clone(), st=L["state"].clone(),
                            saved=[_saved(C, HV, cuda), _saved(C, HV, cuda)], ctl=torch.zeros(26, dtype=torch.int32, device=cuda))
    g = torch.Generator().manual_seed(M)
    for step in range(2):
        x = (_bf(g, M, H) * 2).to(cuda)
        outs = {}
        for path, S in states.items():
            ctl = S["ctl"]
            if step == 1:
                ctl.zero_()
                n = min(3, M)
                ctl[0] = n
                ctl[2:2 + n] = torch.arange(n, dtype=torch.int32)
            prev, save = S["saved"][step % 2], S["saved"][1 - step % 2]
            if path == "chain":
                xn = torch.empty_like(x)
                pre = _C.rowlin_gptq(x, _C.ROWLIN_NORM, [(L["qkv"], C), (L["z"], Z)], norm_w=L["ln1"], eps=1e-6, xn_out=xn)
                ab = _C.gdn_ab(xn, L["wab"])
                core = _C.gdn_step_deferred(pre[:, :C], pre[:, C:], ab[:, :HV], ab[:, HV:], L["conv_w"], S["cs"],
                                            L["dt_bias"], L["g_decay"], S["st"], L["gnorm"], 1e-6, 128 ** -0.5, HK, ctl,
                                            prev, save)
                x1 = _C.rowlin_gptq(core, _C.ROWLIN_QUANT, [(L["out"], H)], residual=x)
                outs[path] = _C.mlp_gptq(x1, L["ln2"], 1e-6, L["gate"], L["up"], L["down"], silu_lut=silu, I=I)
            else:
                outs[path] = _C.layer_gdn(x, L["ln1"], 1e-6, L["qkv"], L["z"], L["wab"], L["conv_w"], S["cs"],
                                          L["dt_bias"], L["g_decay"], S["st"], L["gnorm"], 1e-6, 128 ** -0.5, HK, ctl,
                                          prev, save, L["out"], L["ln2"], 1e-6, L["gate"], L["up"], L["down"], silu, I)
        a, b = states["chain"], states["fused"]
        assert np.array_equal(bf16_bits(outs["fused"]), bf16_bits(outs["chain"])), step
        assert np.array_equal(bf16_bits(b["cs"]), bf16_bits(a["cs"]))
        assert torch.equal(b["st"], a["st"])
        for i in range(2):
            for t_a, t_b in zip(a["saved"][i], b["saved"][i]):
                assert torch.equal(t_a, t_b)


def _small_cfg():
    from mono_b200.decoder import Qwen35Config
    return Qwen35Config(hidden=2048, inter=4096, vocab=32768, layers=8, heads=8, kv_heads=2, gdn_k_heads=8,
                        gdn_v_heads=16)


@pytest.mark.parametrize("prefetch", [0, 24])
def test_decoder_programs_match_op_by_op(cuda, prefetch):
    """Three MTP decode steps of an 8-layer synthetic model (2 attention layers): the 3 layer programs per step
    (plus the attention kernels between them) commit the same tokens, hidden rows and counters as the op-by-op
    path, bit for bit."""
    from mono_b200.decoder import Qwen35W4A8
    cfg = _small_cfg()
    ref = Qwen35W4A8(cfg, cuda, prompt_len=96, gen_tokens=64, fused=False)
    fus = Qwen35W4A8(cfg, cuda, prompt_len=96, gen_tokens=64, fused=True, prefetch=prefetch)
    assert len(fus.programs[0]) == 3
    for _ in range(3):
        r_ref = ref.step().clone()
        r_fus = fus.step().clone()
        assert torch.equal(r_ref, r_fus)
        assert np.array_equal(bf16_bits(ref.hidden), bf16_bits(fus.hidden))
        assert torch.equal(ref.st, fus.st) and torch.equal(ref.ctl, fus.ctl)
    for La, Lb in zip(ref.layers, fus.layers):
        if "state" in La:
            assert torch.equal(La["state"], Lb["state"]) and torch.equal(La["conv_state"], Lb["conv_state"])
        else:
            assert torch.equal(La["kc"], Lb["kc"]) and torch.equal(La["vc"], Lb["vc"])


def test_program_rejects_bad_ops(cuda):
    """Host-side checks: unplanned launches, too many by-value ops and malformed ops fail with EINVAL before any
    launch."""
    from mono_b200 import _C, _lib
    P = _C.Program(cuda)
    x = torch.zeros(4, 4096, dtype=torch.bfloat16, device=cuda)
    q = torch.zeros(16, 4096, dtype=torch.int8, device=cuda)
    s = torch.zeros(64, dtype=torch.float32, device=cuda)
    with pytest.raises(_lib.MonoError):
        P.rows(_C.ROWS_NORM, x, 4096, q, s)  # norm without a weight
    with pytest.raises(_lib.MonoError):
        P.rows(_C.ROWS_QUANT, x, 1000, q, s)  # K not a multiple of 1024
    P2 = _C.Program(cuda)
    with pytest.raises(RuntimeError):
        P2.launch()  # not planned
