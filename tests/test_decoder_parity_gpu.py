"""Decoder-level parity: several MTP decode steps of a small Qwen3.5-shaped W4A8 model (4 layers: 3 GDN + 1 full
attention, hidden 2048, the 8-node tree4s1m8 draft tree) through the device loop, every operation of the composed
step checked against the CPU oracle on the GPU's own inputs (what each op received inside the step: views,
strides, the parity-alternating GDN buffers, the ctl handoff from the accept to the next step's replay):

  bit-exact   layer_pre (RMSNorm -> quant -> W4A8 q|k|v or qkv|z), Q/K norm + RoPE + KV-cache rows, the a|b
              projection, the gate / quant -> o_proj / out_proj + residual, the fused MLP, the final norm, the
              verify argmax and every draft's pick into the verify-token row (on the lm_head kernel's own logits),
              the accept walk (result row, counters, ctl, next token, hidden row) and the KV slot moves of an
              off-chain path, the GDN conv state after the replay
  tolerance   tree attention and the GDN core / recurrent state against fp64 (the bounds of
              tests/test_attention_gpu.py and tests/test_gdn_gpu.py); the tensor-core lm_head logits against the exact
              dot products (oracle/lmhead.py tolerance)

The accepted path is steered on some steps (the verify tokens are rewritten before the accept), so the replay of an
off-chain leaf, a full-chain accept and the KV moves run on the device and are checked like the natural steps."""
import numpy as np
import pytest
import torch

from conftest import bf16_bits
from oracle import attention as oa
from oracle import gdn as og
from oracle import layers as ol
from oracle import lmhead as olh
from oracle import mtp as om
from oracle import w4a8 as ow
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits

pytestmark = pytest.mark.gpu


def _gptq(xq, xs, src, residual=None):
    return ow.gptq_linear(xq, xs, *src, residual=residual)


def _row_linear(x_bits, norm_bits, eps, srcs, residual=None):
    xn = ol.rmsnorm(x_bits, norm_bits, eps) if norm_bits is not None else x_bits
    q, s = ow.act_quant(xn)
    return xn, np.concatenate([_gptq(q, s, src, residual) for src in srcs], axis=1)


def _kernel_pick(xf, lm_t, lm, k):
    """The pick of the lm_head kernel's own logits for the normed rows xf (device), after checking those logits
    against the exact dot products."""
    from mono_b200 import _C
    lg = bf16_bits(_C.lmhead_pick(xf, lm_t, k=0, logits=True)[2])
    exact, abs_sum = olh.logits_exact(bf16_bits(xf), lm)
    err = np.abs(bf16_bits_to_f32(lg).astype(np.float64) - exact)
    assert (err <= olh.tolerance(exact, abs_sum)).all(), err.max()
    return olh.pick_logits(lg, k)


def _steer(model, path):
    """Rewrite the verify tokens so that the greedy walk accepts exactly `path` (rows of the tree)."""
    def fn(toks):
        for a, b in zip(path[:-1], path[1:]):
            toks[0, a] = model.drafts[b]
        last = path[-1]
        # make the walk stop at the last row: a token no child of it carries
        kids = [c for c in model.tree["children"][last] if c >= 0]
        if kids:
            toks[0, last] = (model.drafts[kids].max() + 1) % model.cfg.vocab
    return fn


def test_decoder_steps_match_oracle_op_by_op(cuda):
    from mono_b200.decoder import Qwen35Config, Qwen35W4A8
    cfg = Qwen35Config(hidden=2048, inter=4096, vocab=32768, layers=4, heads=8, kv_heads=2, gdn_k_heads=8,
                       gdn_v_heads=16)
    model = Qwen35W4A8(cfg, cuda, prompt_len=64, gen_tokens=64, keep_sources=True)
    W = {k: (v[0].cpu().numpy(), v[1].cpu().numpy()) for k, v in model.w4_src.items()}
    lut_silu, lut_sig = bf16_bits(model.silu_lut), bf16_bits(model.sig_lut)
    lm = bf16_bits(model.lm_head)
    tree = model.tree
    R, hd, eps = tree["rows"], cfg.head_dim, cfg.eps
    HK, HV, D = cfg.gdn_k_heads, cfg.gdn_v_heads, cfg.gdn_dim
    Ck = 2 * HK * D + HV * D
    nq, nkv = 2 * cfg.heads * hd, cfg.kv_heads * hd
    events = []
    model.trace = lambda name, layer, tensors: events.append((name, layer, tensors))
    steers = [None, [0, 7], [0, 1, 2, 3, 4], [0, 1, 2, 5], None]
    checked = {"gdn": 0, "attn": 0, "draft": 0, "offchain": 0}
    for step, path in enumerate(steers):
        gdn_before = {i: (L["state"].clone(), L["conv_state"].clone(), [tuple(b.clone() for b in s) for s in L["saved"]])
                      for i, L in enumerate(model.layers) if "state" in L}
        ctl0, parity, next_tok0 = model.ctl.clone(), model.parity, int(model.next_tok.item())
        events.clear()
        model.step(steer=_steer(model, path) if path else None)
        torch.cuda.synchronize()
        drafts_seen, x_final = None, None
        for name, i, T in events:
            if name == "draft":
                # the pick of draft i: its children's verify tokens, from the GPU's normed hidden row
                am, top = _kernel_pick(T["xf"], model.lm_head, lm, cfg.tree[i])
                d = T["drafts"].cpu().tolist()
                kids = [c for c in tree["children"][i] if c >= 0]
                assert d[kids[0]] == int(am[0]), (step, i)
                for j, c in enumerate(kids[1:], 1):
                    assert d[c] == int(top[0][j]), (step, i, j)
                if i == 0:
                    assert d[0] == next_tok0
                drafts_seen = d
                checked["draft"] += 1
            elif name == "gdn":
                L = model.layers[i]
                x, pre, xn, ab = (bf16_bits(T[k]) for k in ("x", "pre", "xn", "ab"))
                xn_ref, pre_ref = _row_linear(x, bf16_bits(L["ln1"]), eps, [W[(i, "qkv")], W[(i, "z")]])
                assert np.array_equal(xn, xn_ref) and np.array_equal(pre, pre_ref), (step, i)
                assert np.array_equal(ab, og.ab_projection(xn, bf16_bits(L["wab"]))), (step, i)
                st0, cs0, saved0 = gdn_before[i]
                n = int(ctl0[0])
                slots = ctl0[2:2 + n].cpu().numpy()
                replay = tuple(bf16_bits(t)[slots] for t in saved0[parity]) if n else None
                core_ref, cs_ref, st_ref = og.gdn_step_tree(
                    pre[:, :Ck], pre[:, Ck:], ab[:, :HV], ab[:, HV:], bf16_bits(L["conv_w"]), bf16_bits(cs0),
                    L["dt_bias"].cpu().numpy(), L["g_decay"].cpu().numpy(), st0.cpu().numpy(), bf16_bits(L["gnorm"]),
                    eps, D ** -0.5, HK, tree["parents"], tree["program"], replay=replay)
                core = bf16_bits_to_f32(bf16_bits(T["core"])).astype(np.float64)
                err = np.abs(core - core_ref)
                assert (err <= 2 ** -6 * np.abs(core_ref) + 2e-3).all(), (step, i, err.max())
                assert np.array_equal(bf16_bits(T["conv_state"]), cs_ref), (step, i)
                st = T["state"].cpu().numpy().astype(np.float64)
                assert (np.abs(st - st_ref) <= 1e-4 * (1 + np.abs(st_ref))).all(), (step, i)
                q, s = ow.act_quant(bf16_bits(T["core"]))
                x1_ref = _gptq(q, s, W[(i, "out")], residual=x)
                assert np.array_equal(bf16_bits(T["x1"]), x1_ref), (step, i)
                out_ref = ol.mlp_gptq(x1_ref, bf16_bits(L["ln2"]), eps, W[(i, "gate")], W[(i, "up")], W[(i, "down")],
                                      lut_silu)
                assert np.array_equal(bf16_bits(T["out"]), out_ref), (step, i)
                checked["gdn"] += 1
            elif name == "attn":
                L = model.layers[i]
                x, pre = bf16_bits(T["x"]), bf16_bits(T["pre"])
                _, pre_ref = _row_linear(x, bf16_bits(L["ln1"]), eps, [W[(i, "q")], W[(i, "k")], W[(i, "v")]])
                assert np.array_equal(pre, pre_ref), (step, i)
                rawq = pre[:, :nq].reshape(R, cfg.heads, 2 * hd)[:, :, :hd]
                rawk = pre[:, nq:nq + nkv].reshape(R, cfg.kv_heads, hd)
                v = pre[:, nq + nkv:].reshape(R, cfg.kv_heads, hd)
                kc, vc = bf16_bits(T["kc"])[0], bf16_bits(T["vc"])[0]
                key, value = kc.copy(), vc.copy()
                pos = T["apos"].cpu().numpy()[:R]
                q_ref, k_ref = oa.qk_norm_rope_kv(rawq, rawk, v, bf16_bits(L["q_norm"]), bf16_bits(L["k_norm"]),
                                                  T["freqs"].cpu().numpy().reshape(R, -1, 2, 2), key, value, pos, eps,
                                                  eps, cfg.rotary_dim)
                assert np.array_equal(bf16_bits(T["q"])[0], q_ref) and np.array_equal(bf16_bits(T["k"])[0], k_ref)
                assert np.array_equal(kc, key) and np.array_equal(vc, value), (step, i)  # the rows written at pos
                Lctx = int(T["aseq"].item())
                y_ref = oa.attention_fp64(q_ref, kc, vc, Lctx, k_ref, np.ascontiguousarray(v.transpose(1, 0, 2)),
                                          tree["mask"])
                y = bf16_bits_to_f32(bf16_bits(T["y"])[0]).astype(np.float64)
                assert (np.abs(y - y_ref) <= 8e-3 + 2 ** -7 * np.abs(y_ref)).all(), (step, i)
                gate = pre[:, :nq].reshape(R, cfg.heads, 2 * hd)[:, :, hd:].reshape(R, -1)
                yg = f32_to_bf16_bits((bf16_bits_to_f32(bf16_bits(T["y"])[0]) *
                                       bf16_bits_to_f32(lut_sig[gate.astype(np.int64)])).astype(np.float32))
                q, s = ow.act_quant(yg)
                x1_ref = _gptq(q, s, W[(i, "o")], residual=x)
                assert np.array_equal(bf16_bits(T["x1"]), x1_ref), (step, i)
                out_ref = ol.mlp_gptq(x1_ref, bf16_bits(L["ln2"]), eps, W[(i, "gate")], W[(i, "up")], W[(i, "down")],
                                      lut_silu)
                assert np.array_equal(bf16_bits(T["out"]), out_ref), (step, i)
                checked["attn"] += 1
            elif name == "verify":
                assert T["tokens"].cpu().tolist() == drafts_seen
                xf_ref = ol.rmsnorm(bf16_bits(T["x"]), bf16_bits(model.final_norm), eps)
                assert np.array_equal(bf16_bits(T["xf"]), xf_ref)
                am, _ = _kernel_pick(T["xf"], model.lm_head, lm, 0)
                assert T["toks"].view(-1).cpu().tolist() == am.tolist(), step
                x_final = bf16_bits(T["x"])
            elif name == "accept_in":
                st = T["st"].cpu().numpy().copy()
                ctl = T["ctl"].cpu().numpy().copy()
                kv = [a[0] for a in bf16_bits(T["kv"])]
                children = np.array(tree["children"], dtype=np.int64)
                res, nt, hrow = om.mtp_accept(st, T["toks"].view(-1).cpu().tolist(), T["drafts"].cpu().tolist(), None,
                                              children, R, cfg.depth, x_final, ctl, kv, model.cap)
                assert model.result.cpu().numpy().tolist()[:21] == res.tolist()[:21], step
                assert model.st.cpu().numpy().tolist() == st.tolist() and model.ctl.cpu().numpy().tolist() == ctl.tolist()
                assert int(model.next_tok.item()) == nt and np.array_equal(bf16_bits(model.hidden).reshape(-1), hrow)
                after = [bf16_bits(t)[0] for L in model.layers if "kc" in L for t in (L["kc"], L["vc"])]
                assert all(np.array_equal(a, b) for a, b in zip(after, kv)), step
                if path:
                    assert res[0] == len(path) and res[9] == path[-1], (step, res[:12])
                    checked["offchain"] += int(not res[10])
    assert checked["gdn"] == 3 * len(steers) and checked["attn"] == len(steers)
    assert checked["draft"] == cfg.depth * len(steers) and checked["offchain"] == 2
    from mono_b200 import _C
    assert _C.device_status() == 0
