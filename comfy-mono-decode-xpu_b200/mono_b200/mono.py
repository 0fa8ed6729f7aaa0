"""MLP install point (the role of comfy_mono_decode_xpu/mono.py:147-201): ``llama.MLP.forward(self, x, norm=None)``
-> the fused MLP block (mono_mlp_gptq: RMSNorm -> gate / up -> SiLU * up -> re-quant -> down -> residual) for
decode rows (1-16 rows of hidden 4096, CUDA, bf16) whose three projections carry this build's tile-major GPTQ
weights (``mono_b200_w4`` = (tiled uint8 tensor, rows) on the linear modules). Every other call runs the original.
The fused kernel adds the residual itself; the original forward does not, so the route passes residual=False.
"""
from __future__ import annotations

import threading

import torch

from . import guard

CLAIM = "__comfy_mono_decode_b200__"
_stats = {"mono": 0, "fallback": 0}
_lock = threading.Lock()


def stats():
    with _lock:
        return dict(_stats)


def _w4(lin):
    w = getattr(lin, "mono_b200_w4", None)
    return w if isinstance(w, tuple) and len(w) == 2 else None


def install(llama=None):
    if llama is None:
        from comfy.text_encoders import llama
    from . import _C
    MLP = llama.MLP
    original = MLP.forward
    if getattr(original, CLAIM, False) or getattr(original, "__comfy_mono_decode_xpu__", False):
        return False

    def forward(self, x, norm=None):
        lins = (self.gate_proj, self.up_proj, self.down_proj)
        parts = [_w4(l) for l in lins]
        if (guard.off("mono") or norm is None or x.device.type != "cuda" or x.dtype != torch.bfloat16
                or x.shape[-1] != 4096 or not 1 <= x.numel() // x.shape[-1] <= 16 or any(p is None for p in parts)):
            with _lock:
                _stats["fallback"] += 1
            return original(self, x, norm=norm)
        try:
            w = norm.scale() if hasattr(norm, "scale") else norm.weight
            out = _C.mlp_gptq(x.reshape(-1, x.shape[-1]).contiguous(), w.to(torch.bfloat16).contiguous(), norm.eps,
                              parts[0][0], parts[1][0], parts[2][0], residual=False, I=parts[0][1])
        except Exception as e:  # nothing was written: the original forward recomputes from x
            guard.failed("mono", e)
            return original(self, x, norm=norm)
        with _lock:
            _stats["mono"] += 1
        return out.reshape(*x.shape[:-1], out.shape[-1])

    setattr(forward, CLAIM, True)
    forward.__wrapped__ = original
    MLP.forward = forward
    return True
