"""Failure handling shared by every fast path (the role of comfy_mono_decode_xpu/guard.py).

A fast path that raises (an argument check of the C ABI, a CUDA error at launch, an out-of-memory) is logged
once with its traceback and switched off for the rest of the process; the call that hit the error runs the
original code instead. Callers fall back only while no state has been modified; otherwise they re-raise after
switching the path off. A user interrupt (ComfyUI's InterruptProcessingException) is not a failure.
"""
from __future__ import annotations

import logging
import threading

_lock = threading.Lock()
_off = {}  # piece -> reason


def off(piece: str) -> bool:
    return piece in _off


def _is_interrupt(exc) -> bool:
    try:
        import comfy.model_management
        return isinstance(exc, comfy.model_management.InterruptProcessingException)
    except Exception:
        return False


def failed(piece: str, exc: BaseException, *, can_fallback: bool = True):
    """Record a failure of `piece` and switch it off (logged once per piece); re-raise user interrupts."""
    if _is_interrupt(exc):
        raise exc
    with _lock:
        first = piece not in _off
        _off[piece] = f"{type(exc).__name__}: {exc}"
    if first:
        action = "trying the stock path" if can_fallback else "aborting this call without replaying modified state"
        logging.warning("[mono_b200] %s path failed and is now disabled; %s", piece, action,
                        exc_info=(type(exc), exc, exc.__traceback__))


def disabled() -> dict:
    with _lock:
        return dict(_off)


def reset():
    """Re-enable every path (tests)."""
    with _lock:
        _off.clear()
