"""MLP install point (the role of comfy_mono_decode_xpu/mono.py:147-201): ``llama.MLP.forward(self, x, norm=None)``
-> the MLP block on this build's kernels for decode rows (bf16 CUDA rows, 1-16 of them) when a plan exists:

  GPTQ  one fused launch (mono_mlp_gptq: RMSNorm -> gate / up -> SiLU * up -> re-quant -> down)
  REF   the stock chain's kernels in order (RMSNorm; rot_quant -> gate | up in one stacked linear; SiLU * up;
        rot_quant -> down), each bit-identical to the stock op

The plan is the generate session's (bridge.mlp_plan: tile-major copies of the module's own packed weights), or one
attached to the projections (``mono_b200_w4`` = (tiled GPTQ tensor, rows) on each of gate / up / down). The
original forward adds no residual, so neither does the route. Calls the kernels' argument checks refuse run the
original; a failure switches the piece off (guard.route).
"""
from __future__ import annotations

import collections
import threading

import torch

from . import guard

CLAIM = "__comfy_mono_decode_b200__"
_lock = threading.Lock()
_stats = collections.Counter()


def stats():
    with _lock:
        return dict(_stats)


def _count(key):
    with _lock:
        _stats[key] += 1


def _attached(mlp):
    """A GPTQ plan from tile-major copies attached to the three projections, or None."""
    parts = [getattr(lin, "mono_b200_w4", None) for lin in (mlp.gate_proj, mlp.up_proj, mlp.down_proj)]
    if not all(isinstance(p, tuple) and len(p) == 2 for p in parts):
        return None
    return {"fmt": "gptq", "gate": {"w": parts[0][0]}, "up": {"w": parts[1][0]}, "down": {"w": parts[2][0]},
            "I": parts[0][1]}


def plan_for(mlp, x):
    plan = _attached(mlp)
    if plan is None and x.device.type == "cuda":
        from . import bridge
        plan = bridge.mlp_plan(mlp, x.device)
    return plan


def install(llama=None):
    if llama is None:
        from comfy.text_encoders import llama
    MLP = llama.MLP
    original = MLP.forward
    if getattr(original, CLAIM, False) or getattr(original, "__comfy_mono_decode_xpu__", False):
        return False

    def forward(self, x, norm=None):
        def stock():
            return original(self, x, norm=norm)

        if (guard.off("mono") or norm is None or x.device.type != "cuda" or x.dtype != torch.bfloat16
                or x.dim() == 0 or not 1 <= x.numel() // max(x.shape[-1], 1) <= 16):
            _count("fallback")
            return stock()
        plan = plan_for(self, x)
        if plan is None:
            _count("fallback_weights")
            return stock()

        def kernel():
            from . import bridge
            w = norm.scale() if hasattr(norm, "scale") else norm.weight
            x2 = x.reshape(-1, x.shape[-1]).contiguous()
            out = bridge.run_mlp(plan, x2, w.to(torch.bfloat16).contiguous(), norm.eps, residual=False)
            _count("mono_" + plan["fmt"])
            return out.reshape(*x.shape[:-1], out.shape[-1])

        return guard.route("mono", kernel, stock, lambda reason: _count("fallback: " + reason))

    setattr(forward, CLAIM, True)
    forward.__wrapped__ = original
    MLP.forward = forward
    return True
