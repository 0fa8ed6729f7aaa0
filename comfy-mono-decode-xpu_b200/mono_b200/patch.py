"""Route the Kitchen INT8 backend's packed W4A8 linears and its rotate + quantize row step to this build's kernels
(the install points of comfy_mono_decode_xpu/patch.py:68-96 and :122-137).

install() replaces ``omni_xpu_kernel.int8.w4a8_linear_prequantized`` (the backend looks it up on every call) and
install_prep() replaces ``quantize_and_rotate_rowwise`` in each loaded ``*.w4a8_int8`` backend module. A replaced
entry hands its call to the mono_b200 binding, and the binding and the C ABI decide whether the kernel takes it
(mono_w4a8_decode_linear: 1-16 rows, K a multiple of 1024 up to 16384, N a multiple of 16, G16 FP8 relative scales,
16-byte aligned operands, one CUDA device; mono_rot_quant: bf16 rows, K a multiple of 256, a 256 x 256 bf16
rotation). A refused call runs the original and is counted under the ABI's reason; a failure switches the piece off
(guard.route). Decided here are only what the C ABI has no parameter for: a bias, an output dtype other than bf16 /
fp32, stochastic rounding, a rotation group other than 256, and torch.compile tracing.

Both entries are pure functions of their inputs, so the original recomputes exactly what a refused call would
have returned; the kernels' results are bit-identical to the original chain's. Replacements are idempotent (the
CLAIM attribute; the original is kept as __wrapped__). MONO_DECODE_XPU_STATS names a JSON file the counters are
written to at exit.
"""
from __future__ import annotations

import atexit
import collections
import json
import os
import sys
import threading

import torch

from . import _lib, guard

CLAIM = "__comfy_mono_decode_b200__"
_OUT_CODES = {torch.bfloat16: _lib.OUT_BF16, torch.float32: _lib.OUT_F32}
_ROTATION = 256  # the rotation block the kernel applies (K is rotated in 256-wide groups)

_lock = threading.Lock()
_served = collections.Counter()  # piece -> calls run by the kernels
_refused = collections.Counter()  # reason -> calls run by the original
_stats_file = []


def stats():
    """{"fused": linear calls served, "prep": rotate + quantize calls served, "fallback": calls sent to the
    original, "reasons": {reason: count}}."""
    with _lock:
        return {"fused": _served["w4"], "prep": _served["prep"], "fallback": sum(_refused.values()),
                "reasons": dict(_refused)}


def _refuse(reason):
    with _lock:
        _refused[reason] += 1


def _serve(piece, kernel, original):
    def counted():
        out = kernel()
        with _lock:
            _served[piece] += 1
        return out
    return guard.route(piece, counted, original, _refuse)


def claimed(fn) -> bool:
    return getattr(fn, CLAIM, False) or getattr(fn, "__comfy_mono_decode_xpu__", False)


def _claim(wrapper, original):
    setattr(wrapper, CLAIM, True)
    wrapper.__wrapped__ = original
    return wrapper


def _write_stats_at_exit():
    path = os.environ.get("MONO_DECODE_XPU_STATS")
    if path and not _stats_file:
        _stats_file.append(path)
        atexit.register(lambda: json.dump(stats(), open(path, "w")))


def install(module=None):
    """Replace omni_xpu_kernel.int8.w4a8_linear_prequantized (or `module`'s, for tests). False when it is already
    replaced or the module is missing."""
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
        def stock():
            return original(x_int8, x_scale, packed, relative_scale, channel_scale, codebook, bias, group_size,
                            out_dtype)

        if torch.compiler.is_compiling():
            return stock()
        if bias is not None or out_dtype not in _OUT_CODES:
            _refuse("bias" if bias is not None else "out_dtype")
            return stock()

        def kernel():
            k = x_int8.shape[-1]
            y = _C.w4a8_decode_linear(x_int8.reshape(-1, k), x_scale.reshape(-1).float(), packed, relative_scale,
                                      channel_scale.reshape(-1).float(), codebook, None, group_size,
                                      _OUT_CODES[out_dtype])
            return y.reshape(*x_int8.shape[:-1], y.shape[-1])

        return _serve("w4", kernel, stock)

    module.w4a8_linear_prequantized = _claim(w4a8_linear_prequantized, original)
    _write_stats_at_exit()
    return True


def install_prep(modules=None):
    """Replace quantize_and_rotate_rowwise in every loaded ``*.w4a8_int8`` backend module (or in `modules`).
    Returns how many were replaced."""
    if modules is None:
        modules = [m for n, m in list(sys.modules.items())
                   if n.endswith(".w4a8_int8") and hasattr(m, "quantize_and_rotate_rowwise")]
    from . import _C
    done = 0
    for mod in modules:
        original = mod.quantize_and_rotate_rowwise
        if claimed(original):
            continue

        def quantize_and_rotate_rowwise(x, h, group_size, stochastic_rounding=0, _original=original):
            def stock():
                return _original(x, h, group_size, stochastic_rounding)

            if torch.compiler.is_compiling():
                return stock()
            if group_size != _ROTATION or stochastic_rounding:
                _refuse("group_size" if group_size != _ROTATION else "stochastic_rounding")
                return stock()
            return _serve("prep", lambda: _C.rot_quant(x.contiguous(), h.contiguous()), stock)

        mod.quantize_and_rotate_rowwise = _claim(quantize_and_rotate_rowwise, original)
        done += 1
    if done:
        _write_stats_at_exit()
    return done
