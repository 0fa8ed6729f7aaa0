"""One-launch exact top-k for the verify step's sampling filter on CUDA (the role of
comfy_mono_decode_xpu/sampling.py; switch MONO_DECODE_XPU_SAMPLE_TOPK: "1" on (default), "0" off, "check": both
run, torch's answer is returned and disagreements are counted).

Upstream's sampling (ComfyUI's sample_token / processed_probs) starts its top-k filter with torch.topk(rows,
top_k) over the verify rows: up to 16 rows of the ~248k-entry vocabulary. Inside the context that topk_mode /
verify_rows return, every torch.topk / Tensor.topk call is bound to torch.topk's own signature; a call that asks
for the k largest, sorted, along the last dimension, without out=, of a CUDA tensor is handed to C.topk_rows over
its rows (leading dimensions flattened). Whether the kernel answers is decided by the binding and the C ABI (row
count, row length, k, dtype: include/mono_b200.h mono_topk_rows): an argument rejection (_lib.rejected) runs
torch's topk for that call only; any other exception switches the piece off (guard) and runs torch's topk. No
other operation is intercepted: torch.sort, softmax, multinomial and the masked writes stay upstream's.

Values are torch's bit for bit (the same multiset, sorted descending; bf16 rows give bf16 values, which their fp32
results convert to exactly). Equal values come out by ascending index (mono_topk_rows with MONO_TOPK_INDEX_ORDER):
torch's own CUDA topk order for k >= 33 and for k = 1, as measured on B200 over tie-heavy rows, so those calls
return torch's indices exactly. For 2 <= k <= 32 torch orders equal values by its small sorting network, which no
fixed rule reproduces: there "check" mode can count a tie as a disagreement while the value sets agree. (The
reference keeps its platform's torch-XPU order; that order is the kernel's other mode.)
"""
from __future__ import annotations

import collections
import contextlib
import inspect
import operator
import os
import threading

import torch

from . import _lib, guard

MODE = os.environ.get("MONO_DECODE_XPU_SAMPLE_TOPK", "1")
DEVICES = ("cuda",)  # device types whose topk calls are offered to the kernel
PIECE = "sample_topk"

_counts = collections.Counter()
_lock = threading.Lock()


def _topk_parameters(input, k, dim=-1, largest=True, sorted=True, *, out=None):
    """torch.topk's parameters; Tensor.topk binds self as `input`."""


_SIGNATURE = inspect.signature(_topk_parameters)
_TOPK = (torch.topk, torch.Tensor.topk)


def stats():
    """Counters: "calls" (answered by the kernel), "passed" (topk calls of another form), "rejected" and
    "rejected: <reason>" (the ABI refused the arguments), "checked" / "check_mismatch" (check mode)."""
    with _lock:
        return dict(_counts)


def _count(*keys):
    with _lock:
        for key in keys:
            _counts[key] += 1


def _bind(args, kwargs):
    try:
        bound = _SIGNATURE.bind(*args, **kwargs)
    except TypeError:
        return None
    bound.apply_defaults()
    return bound.arguments


def _request(a):
    """(rows [R, N], k) when the bound call asks for the k largest along the last dim, sorted, into fresh tensors,
    of a plain CUDA tensor; None otherwise (the kernel's own limits are not tested here)."""
    x = a["input"]
    if type(x) is not torch.Tensor or x.device.type not in DEVICES or x.dim() == 0:
        return None
    if a["out"] is not None or a["largest"] is not True or a["sorted"] is not True:
        return None
    if isinstance(a["k"], bool) or isinstance(a["dim"], bool):
        return None
    try:
        k, dim = operator.index(a["k"]), operator.index(a["dim"])
    except TypeError:
        return None
    if dim not in (-1, x.dim() - 1):
        return None
    return x.reshape(-1, x.shape[-1]), k


class TopkServer(torch.overrides.TorchFunctionMode):
    """Answers the eligible torch.topk calls made inside it with C.topk_rows (module docstring)."""

    def __init__(self, C):
        super().__init__()
        self.C = C

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        if func not in _TOPK or guard.off(PIECE):
            return func(*args, **kwargs)
        a = _bind(args, kwargs)
        req = None if a is None else _request(a)
        if req is None:
            _count("passed")
            return func(*args, **kwargs)
        rows, k = req
        try:
            values, indices = self.C.topk_rows(rows, k, index_order=True)
        except Exception as e:
            if _lib.rejected(e):
                _count("rejected", "rejected: " + e.reason)
            else:
                guard.failed(PIECE, e)
            return func(*args, **kwargs)
        x = a["input"]
        shape = (*x.shape[:-1], k)
        got = torch.return_types.topk((values.to(x.dtype).reshape(shape), indices.reshape(shape)))
        if MODE != "check":
            _count("calls")
            return got
        ref = func(*args, **kwargs)
        same = (torch.equal(ref.indices, got.indices) and ref.values.dtype == got.values.dtype
                and torch.equal(ref.values.contiguous().view(torch.uint8), got.values.view(torch.uint8)))
        _count("checked", *(() if same else ("check_mismatch",)))
        return ref


def topk_mode(C):
    """The context in which C.topk_rows answers the sampling's top-k (a null context when the switch is "0", the
    piece is off, or C has no topk_rows)."""
    if MODE == "0" or guard.off(PIECE) or not hasattr(C, "topk_rows"):
        return contextlib.nullcontext()
    return TopkServer(C)


def verify_rows(C, lg0):
    """(context, rows) for sampling from the verify logits lg0 [R, N]: rows is the fp32 tensor upstream's sampling
    takes (lg0 itself when already fp32, else its fp32 copy: 6 bytes of traffic per logit, ~2 us for 8 x 248k on
    this device, so no lazy stand-in is kept for it), context is topk_mode(C)."""
    return topk_mode(C), (lg0 if lg0.dtype == torch.float32 else lg0.float())
