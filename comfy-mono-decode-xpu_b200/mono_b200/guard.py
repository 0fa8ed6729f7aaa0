"""Failure handling shared by every fast path (the role of comfy_mono_decode_xpu/guard.py).

Two kinds of refusal reach a fast path. An argument rejection (mono_b200._lib.rejected: the binding or the C ABI
found the call outside what the kernels take, before anything was launched) sends that one call to the original
code. A failure (a CUDA error at launch, an out-of-memory, any other exception) is logged once with its traceback
and switches the path off for the rest of the process; the call that hit it runs the original code instead.
Callers fall back only while no state has been modified; otherwise they re-raise after switching the path off.
A user interrupt (ComfyUI's InterruptProcessingException) is neither: it propagates.
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


def route(piece: str, kernel, original, refused=None):
    """kernel() when `piece` is on and the kernel takes the call, else original(); both are zero-argument calls
    that compute the same pure function of the call's inputs. refused(reason), when given, hears why a call ran
    the original: "off", the rejection's reason (the ABI's message), or "failed"."""
    if piece in _off:
        if refused:
            refused("off")
        return original()
    try:
        return kernel()
    except Exception as e:
        from . import _lib
        if _lib.rejected(e):
            reason = e.reason
        else:
            failed(piece, e)
            reason = "failed"
    if refused:
        refused(reason)
    return original()
