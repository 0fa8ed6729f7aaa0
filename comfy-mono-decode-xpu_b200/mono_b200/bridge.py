"""Generate-time weight bridge: tile-major copies of a Qwen3.5 model's packed W4 linears and the decode plans that
the block route (layer.install) and the MLP route (mono.install) run on them (the role of
comfy_mono_decode_xpu/tiles.py:309-354 and of the block plans of comfy_mono_decode_xpu/layer.py:106-199).

Formats, read from ``lin.weight`` (the INT8 backend's QuantizedTensor: ``_qdata`` and ``_params``) of a linear
module without bias:

  REF   AsymW4A8Int8Layout: _qdata int8 / uint8 [N, K/2] (two 4-bit codes per byte, low nibble = even k),
        _params.scale fp8 e4m3 [N, K/16] (G16 relative scales, sign bits clear), _params.s_channel [N],
        _params.codebook [16]; the stock chain rotates the activations in 256-groups and quantizes each row
        (quantize_and_rotate_rowwise -> mono_rot_quant), then w4a8_linear_prequantized
  GPTQ  _qdata uint8 [N, K/2] (nibbles v + 8), _params.scale fp16 [N, K/128]; rows quantized per token (act_quant)

N must be a multiple of 16 and K a multiple of 1024 (the kernels' tile); any other module is not bridged and keeps
the stock path.

A session spans one generate call (install() wraps Qwen35.generate with begin(model) / end(); both can be called
directly). Inside it, parts(lins) is one tile-major copy (mono_w4_repack) of the rows of `lins` stacked in order
(q|k|v, gate|up) with the operands its epilogue needs, made on first use and checked against the source tensors
on every use (a replaced weight makes a new copy); block_plan(block) and mlp_plan(mlp) are the decode plans, None
for modules that are not bridged. end() drops every copy and plan. Outside a session nothing is bridged.
"""
from __future__ import annotations

import functools
import threading
import weakref

import torch

from . import guard

CLAIM = "__comfy_mono_decode_b200_bridge__"
H_ROT = 256  # the rotation group of the REF chain

_lock = threading.Lock()
_session = {"active": False, "model": None, "parts": {}, "plans": {}, "bytes": 0}
_stats = {"sessions": 0, "copies": 0, "copy_bytes": 0, "plans": 0, "not_bridged": 0}


def stats():
    with _lock:
        return dict(_stats, live_bytes=_session["bytes"], active=_session["active"])


def active():
    return _session["active"]


def begin(model=None):
    with _lock:
        _session.update(active=True, model=None if model is None else weakref.ref(model), parts={}, plans={}, bytes=0)
        _stats["sessions"] += 1


def end():
    with _lock:
        _session.update(active=False, model=None, parts={}, plans={}, bytes=0)


def weight_format(lin):
    """("ref" | "gptq", N, K) for a bridgeable linear module, else None (never raises)."""
    try:
        if getattr(lin, "bias", None) is not None or getattr(lin, "weight_function", None):
            return None
        w = lin.weight
        q, p = getattr(w, "_qdata", None), getattr(w, "_params", None)
        scale = getattr(p, "scale", None)
        if q is None or scale is None or q.dim() != 2 or q.dtype not in (torch.int8, torch.uint8):
            return None
        N, K = q.shape[0], 2 * q.shape[1]
        if N % 16 or K % 1024 or not q.is_contiguous() or not scale.is_contiguous():
            return None
        if scale.dtype == torch.float8_e4m3fn and tuple(scale.shape) == (N, K // 16):
            cb, sc = getattr(p, "codebook", None), getattr(p, "s_channel", None)
            if cb is None or sc is None or cb.numel() != 16 or sc.numel() != N:
                return None
            if getattr(p, "group_size", 16) != 16 or getattr(p, "convrot_groupsize", H_ROT) != H_ROT:
                return None
            return "ref", N, K
        if scale.dtype == torch.float16 and tuple(scale.shape) == (N, K // 128):
            return "gptq", N, K
    except Exception:
        return None
    return None


def _sources(lins):
    return tuple((lin.weight._qdata, lin.weight._params.scale) for lin in lins)


def _same_sources(a, b):
    return len(a) == len(b) and all(x[0] is y[0] and x[1] is y[1] for x, y in zip(a, b))


def _build_parts(lins, fmt, K, device):
    from . import _C
    q = torch.cat([lin.weight._qdata.to(device) for lin in lins]).view(torch.uint8).contiguous()
    N = q.shape[0]
    if fmt == "ref":
        sc = torch.cat([lin.weight._params.scale.to(device).view(torch.uint8) for lin in lins]).contiguous()
        cb = lins[0].weight._params.codebook.to(device=device, dtype=torch.float32).contiguous()
        sch = torch.cat([lin.weight._params.s_channel.to(device).reshape(-1).float() for lin in lins]).contiguous()
        w = _C.w4_repack(1, q, sc, N, K)
        return {"fmt": fmt, "w": w, "N": N, "K": K, "cb": cb, "sch": sch, "rows": [l.weight._qdata.shape[0] for l in lins]}
    sc = torch.cat([lin.weight._params.scale.to(device) for lin in lins]).contiguous()
    w = _C.w4_repack(0, q, sc, N, K)
    return {"fmt": fmt, "w": w, "N": N, "K": K, "rows": [l.weight._qdata.shape[0] for l in lins]}


def parts(lins, device):
    """The session's tile-major copy of `lins` stacked (same format, K and, for REF, codebook), or None."""
    if not _session["active"]:
        return None
    key = (tuple(id(lin) for lin in lins), torch.device(device))
    src = _sources(lins) if all(weight_format(lin) for lin in lins) else None
    hit = _session["parts"].get(key)
    if hit is not None and src is not None and _same_sources(hit[0], src):
        return hit[1]
    fmts = [weight_format(lin) for lin in lins]
    if src is None or len({(f[0], f[2]) for f in fmts}) != 1:
        return None
    fmt, K = fmts[0][0], fmts[0][2]
    if fmt == "ref":
        cb0 = lins[0].weight._params.codebook.cpu()
        if any(not torch.equal(cb0, lin.weight._params.codebook.cpu()) for lin in lins[1:]):
            return None
    p = _build_parts(lins, fmt, K, torch.device(device))
    size = p["w"].numel()
    with _lock:
        old = _session["parts"].get(key)
        if old is not None:
            _session["bytes"] -= old[1]["w"].numel()
        _session["parts"][key] = (src, p)
        _session["bytes"] += size
        _stats["copies"] += 1
        _stats["copy_bytes"] += size
    return p


def _cached_plan(key, lins, build):
    """The session's plan under `key`, rebuilt when a source weight of `lins` was replaced."""
    hit = _session["plans"].get(key)
    if hit is not None:
        plan, src = hit
        if plan is None or _same_sources(src, _sources(lins)):
            return plan
    try:
        plan = build()
    except Exception as e:  # an unexpected module state: that module keeps the stock path (logged once)
        guard.failed("bridge_plan:" + type(e).__name__, e)
        plan = None
    with _lock:
        _stats["plans" if plan is not None else "not_bridged"] += 1
    _session["plans"][key] = (plan, _sources(lins) if plan is not None else None)
    return plan


def _norm_scale(norm):
    """The norm weight the stock RMSNorm multiplies by (RMSNorm(add=True).scale() = weight + 1), bf16."""
    w = norm.scale() if hasattr(norm, "scale") else norm.weight
    return w.to(torch.bfloat16).contiguous()


def mlp_plan(mlp, device):
    """{"fmt", "gu" (REF: gate | up stacked) or "gate" / "up" (GPTQ), "down", "I"} for a llama.MLP, or None."""
    if not _session["active"] or getattr(mlp, "merged_mlp", False):
        return None
    lins = (mlp.gate_proj, mlp.up_proj, mlp.down_proj)

    def build():
        fmts = [weight_format(lin) for lin in lins]
        if any(f is None for f in fmts) or len({f[0] for f in fmts}) != 1:
            return None
        fmt = fmts[0][0]
        if fmt == "ref":
            gu, down = parts(lins[:2], device), parts(lins[2:], device)
            return None if gu is None or down is None else {"fmt": fmt, "gu": gu, "down": down, "I": fmts[0][1]}
        ps = [parts([lin], device) for lin in lins]
        return None if any(p is None for p in ps) else {"fmt": fmt, "gate": ps[0], "up": ps[1], "down": ps[2],
                                                          "I": fmts[0][1]}
    return _cached_plan(("mlp", id(mlp), torch.device(device)), lins, build)


def block_plan(block, device):
    """The decode plan of a Qwen35TransformerBlock: {"run": fn, ...} for a full-attention block whose projections
    are bridged; None otherwise (Gated-DeltaNet blocks keep the stock forward, whose MLP and linears take the MLP
    and W4 routes)."""
    if not _session["active"]:
        return None
    if getattr(block, "layer_type", None) == "linear_attention" or not hasattr(block, "self_attn"):
        return None
    mix = block.self_attn
    lins = (mix.q_proj, mix.k_proj, mix.v_proj, mix.o_proj, block.mlp.gate_proj, block.mlp.up_proj,
            block.mlp.down_proj)

    def build():
        pre = parts(lins[:3], device)
        out = parts(lins[3:4], device)
        mlp = mlp_plan(block.mlp, device)
        if pre is None or out is None or mlp is None or not pre["fmt"] == out["fmt"] == mlp["fmt"]:
            return None
        return {"kind": "attention", "fmt": pre["fmt"], "pre": pre, "out": out, "mlp": mlp,
                "run": _run_attention_block}
    return _cached_plan(("block", id(block), torch.device(device)), lins, build)


# ---- the plans' kernel chains -------------------------------------------------------------------------------

def _linear(parts_, x, residual=None, quant=None):
    """The stacked linear on bf16 rows x [M, K] (quant: the (q, scale) of x when already made): REF rotates +
    quantizes (rot_quant) then runs the REF linear; GPTQ quantizes per token then runs the GPTQ linear."""
    from . import _C, constants
    if parts_["fmt"] == "ref":
        q, s = quant if quant is not None else _C.rot_quant(x, constants.hadamard(x.device))
        return _C.w4a8_decode_linear(q, s.view(-1), parts_["w"], None, parts_["sch"], parts_["cb"], residual, 16, 2,
                                     tiled=True)
    q, s = quant if quant is not None else _C.act_quant(x)
    return _C.w4a8_gptq_linear(q, s.view(-1), parts_["w"], None, residual=residual, tiled=True, N=parts_["N"])


def run_mlp(plan, x, norm_w, eps, residual):
    """The MLP block on bf16 rows x [M, H]: RMSNorm (norm_w None: x is normed already) -> gate / up -> SiLU * up ->
    down (+ x when residual). GPTQ: one fused launch (mono_mlp_gptq); REF: the stock chain's kernels in order."""
    from . import _C, constants
    if plan["fmt"] == "gptq":
        return _C.mlp_gptq(x, norm_w, eps, plan["gate"]["w"], plan["up"]["w"], plan["down"]["w"],
                           silu_lut=_C.act_luts(x.device)[0], residual=residual, I=plan["I"])
    xn = _C.rmsnorm_add(x, norm_w, eps) if norm_w is not None else x
    gu = _linear(plan["gu"], xn)
    I = plan["I"]
    h = _C.lut_mul(gu[:, I:], gu[:, :I], constants.silu_lut(x.device))
    return _linear(plan["down"], h, residual=x if residual else None)


def _run_attention_block(block, x, attention_mask, freqs_cis, kv, state):
    """A full-attention decode block on the plan's kernels: RMSNorm -> q|k|v -> Q/K norm + RoPE + KV write ->
    tree attention -> sigmoid gate -> o_proj + residual -> MLP + residual. Returns (out, kv) like the stock
    forward; raises layer.Ineligible (before any write) when the call is not one the chain serves."""
    from . import _C, constants, layer
    plan = block_plan(block, x.device)
    mix = block.self_attn
    B, S, H = x.shape
    x2 = x.reshape(S, H)
    ln1, ln2 = block.input_layernorm, block.post_attention_layernorm
    xn = _C.rmsnorm_add(x2, _norm_scale(ln1), ln1.eps)
    pre = _linear(plan["pre"], xn)
    nq, nkv = plan["pre"]["rows"][0], plan["pre"]["rows"][1]
    qg, xk, xv = pre[:, :nq].view(1, S, nq), pre[:, nq:nq + nkv].view(1, S, nkv), pre[:, nq + nkv:].view(1, S, nkv)
    state["mutated"] = True  # the KV cache is written from here on (attention_core raises Ineligible before)
    y = layer.attention_core(mix, qg, xk, xv, freqs_cis, kv)
    hd = mix.head_dim  # each head's gate follows its query: column c of the gate at (c / hd) * 2 hd + hd + c % hd
    yg = _C.lut_mul(y.reshape(S, -1), pre[:, hd:nq], constants.sigmoid_lut(x.device), b_head_stride=2 * hd)
    x1 = _linear(plan["out"], yg, residual=x2)
    out = run_mlp(plan["mlp"], x1, _norm_scale(ln2), ln2.eps, residual=True)
    return out.view(B, S, H), kv


def install(q35=None):
    """Wrap Qwen35.generate with a bridge session (begin / end around the call); False when already wrapped."""
    if q35 is None:
        from comfy.text_encoders import qwen35 as q35
    cls = q35.Qwen35
    original = getattr(cls, "generate", None)
    if original is None or getattr(original, CLAIM, False):
        return False

    @functools.wraps(original)
    def generate(self, *args, **kwargs):
        if _session["active"] or guard.off("bridge"):
            return original(self, *args, **kwargs)
        begin(self)
        try:
            return original(self, *args, **kwargs)
        finally:
            end()

    setattr(generate, CLAIM, True)
    generate.__wrapped__ = original
    cls.generate = generate
    return True
