"""Route small-M packed W4A8 linears and the decode-row rotate + quantize step to the B200 kernels (the install
points of comfy_mono_decode_xpu/patch.py:68-96 and :122-137).

install() wraps ``omni_xpu_kernel.int8.w4a8_linear_prequantized`` (the entry the Kitchen backend looks up on
every call): a call that matches the kernel contract (CUDA tensors, 1-16 rows, K a multiple of 1024 up to 16384,
G16 FP8 relative scales, no bias, bf16 / fp32 output, aligned contiguous operands) runs mono_w4a8_decode_linear,
bit-identical to the original chain; every other call runs the original. install_prep() wraps
``quantize_and_rotate_rowwise`` of the loaded ``*.w4a8_int8`` backend modules the same way (rot_quant).
Both are idempotent (the CLAIM attribute, the original kept as __wrapped__) and switched by the reference's
environment variables (MONO_DECODE_XPU_STATS: a JSON file of the counters written at exit).
"""
from __future__ import annotations

import atexit
import json
import os
import sys
import threading

import torch

from . import guard

CLAIM = "__comfy_mono_decode_b200__"
_stats = {"fused": 0, "fallback": 0, "reasons": {}}
_lock = threading.Lock()


def stats():
    with _lock:
        return dict(_stats, reasons=dict(_stats["reasons"]))


def _reason(r):
    with _lock:
        _stats["fallback"] += 1
        _stats["reasons"][r] = _stats["reasons"].get(r, 0) + 1


def claimed(fn) -> bool:
    return getattr(fn, CLAIM, False) or getattr(fn, "__comfy_mono_decode_xpu__", False)


def contract(x, x_scale, packed, s_rel, s_channel, codebook, bias, group_size, out_dtype):
    """None when the call fits mono_w4a8_decode_linear, else the reason (the reference's _contract, with this
    build's limits)."""
    if bias is not None:
        return "bias"
    if out_dtype not in (torch.bfloat16, torch.float32):
        return "out_dtype"
    if x.device.type != "cuda" or x.dtype != torch.int8 or not x.is_contiguous():
        return "x"
    k = x.shape[-1]
    rows = x.numel() // k if k else 0
    if not 1 <= rows <= 16:
        return "rows"
    if k % 1024 or k > 16384 or group_size != 16:
        return "shape"
    if packed.dtype not in (torch.int8, torch.uint8) or packed.dim() != 2 or not packed.is_contiguous() \
            or packed.shape[1] * 2 != k or packed.shape[0] % 16:
        return "packed"
    if packed.data_ptr() % 16 or x.data_ptr() % 16:
        return "align"
    if s_rel.dtype != torch.float8_e4m3fn or not s_rel.is_contiguous():
        return "s_rel"
    if s_channel.numel() != packed.shape[0]:
        return "s_channel"
    if codebook is not None and (codebook.dtype != torch.float32 or codebook.numel() != 16):
        return "codebook"
    devs = {t.device for t in (x, x_scale, packed, s_rel, s_channel) + ((codebook,) if codebook is not None else ())}
    if len(devs) != 1 or x_scale.numel() != rows:
        return "operands"
    return None


def install(module=None):
    """Wrap omni_xpu_kernel.int8.w4a8_linear_prequantized (or `module`'s, for tests). False if already wrapped
    or the module is missing."""
    if module is None:
        try:
            from omni_xpu_kernel import int8 as module
        except ImportError:
            return False
    original = module.w4a8_linear_prequantized
    if claimed(original):
        return False
    from . import _C

    def w4a8_linear_prequantized(x_int8, x_scale, packed, relative_scale, channel_scale, codebook=None, bias=None,
                                 group_size=16, out_dtype=torch.bfloat16):
        if guard.off("w4") or torch.compiler.is_compiling():
            return original(x_int8, x_scale, packed, relative_scale, channel_scale, codebook, bias, group_size, out_dtype)
        why = contract(x_int8, x_scale, packed, relative_scale, channel_scale, codebook, bias, group_size, out_dtype)
        if why is not None:
            _reason(why)
            return original(x_int8, x_scale, packed, relative_scale, channel_scale, codebook, bias, group_size, out_dtype)
        k = x_int8.shape[-1]
        try:
            out = _C.w4a8_decode_linear(x_int8.reshape(-1, k), x_scale.reshape(-1).to(torch.float32).contiguous(), packed,
                                        relative_scale, channel_scale.reshape(-1).to(torch.float32).contiguous(), codebook,
                                        None, group_size, 0 if out_dtype == torch.float32 else 2, 0, False)
        except Exception as e:  # a pure function of its inputs: the original recomputes it
            guard.failed("w4", e)
            return original(x_int8, x_scale, packed, relative_scale, channel_scale, codebook, bias, group_size, out_dtype)
        with _lock:
            _stats["fused"] += 1
        return out.reshape(*x_int8.shape[:-1], packed.shape[0])

    setattr(w4a8_linear_prequantized, CLAIM, True)
    w4a8_linear_prequantized.__wrapped__ = original
    module.w4a8_linear_prequantized = w4a8_linear_prequantized
    output = os.environ.get("MONO_DECODE_XPU_STATS")
    if output:
        atexit.register(lambda: json.dump(stats(), open(output, "w")))
    return True


def install_prep(modules=None):
    """Wrap quantize_and_rotate_rowwise of every loaded ``*.w4a8_int8`` backend module (or `modules`). Returns the
    number wrapped."""
    from . import _C
    targets = modules if modules is not None else [
        m for n, m in list(sys.modules.items()) if n.endswith(".w4a8_int8") and hasattr(m, "quantize_and_rotate_rowwise")]
    done = 0
    for mod in targets:
        original = mod.quantize_and_rotate_rowwise
        if claimed(original):
            continue

        def quantize_and_rotate_rowwise(x, h, group_size, stochastic_rounding=0, _original=original):
            k = x.shape[-1] if x.dim() else 0
            ok = (not guard.off("prep") and group_size == 256 and not stochastic_rounding and x.device.type == "cuda"
                  and x.dtype == torch.bfloat16 and h.dtype == torch.bfloat16 and h.numel() == 65536 and k
                  and k % 256 == 0 and 1 <= x.numel() // k <= 256)
            if not ok:
                _reason("prep")
                return _original(x, h, group_size, stochastic_rounding)
            try:
                out = _C.rot_quant(x.reshape(-1, k).contiguous(), h.contiguous(), 3)
            except Exception as e:
                guard.failed("prep", e)
                return _original(x, h, group_size, stochastic_rounding)
            with _lock:
                _stats["prep"] = _stats.get("prep", 0) + 1
            return out

        setattr(quantize_and_rotate_rowwise, CLAIM, True)
        quantize_and_rotate_rowwise.__wrapped__ = original
        mod.quantize_and_rotate_rowwise = quantize_and_rotate_rowwise
        done += 1
    return done
