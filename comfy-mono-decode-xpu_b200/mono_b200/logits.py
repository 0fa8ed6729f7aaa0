"""Single-launch picks on the generate's logits (the role of comfy_mono_decode_xpu/logits.py; switch
MONO_DECODE_XPU_LOGITS, "0" off).

install() wraps BaseGenerate.logits: for a Qwen3.5 model whose logits come back as a plain CUDA bf16 tensor, the
result is handed out as a PickRows view of it (a torch.Tensor subclass over the same storage). On PickRows:

  argmax / Tensor.argmax, dim = last   mono_fast_topk with the argmax pass: the argmax of every row and, from the
                                       same launch, the top-8 of every row, kept for a topk that follows
  topk / Tensor.topk, k <= 8, largest, sorted, dim = last
                                       the kept top-8's first k columns when the rows are the ones the argmax read
                                       (same base tensor, offset, shape, strides and version counter: an in-place
                                       write in between bumps the version), else mono_fast_topk

The argmax is torch's (the first of equal maxima; NaN counts as the largest). The top-k values are torch's;
among equal values the indices follow mono_fast_topk's documented order (include/mono_b200.h). Whether the
kernel takes a call is the binding's and the C ABI's decision (rows, k, dtype, layout): a refused call runs
torch's op, a failure switches the piece off (guard.route). Indexing keeps the result a PickRows view (so
logits[:, -1] stays eligible); every other op returns plain tensors. Other models are not touched.
"""
from __future__ import annotations

import collections
import inspect
import operator
import os
import threading
import weakref

import torch

from . import guard

CLAIM = "__comfy_mono_decode_b200__"
MODE = os.environ.get("MONO_DECODE_XPU_LOGITS", "1")
PIECE = "logits"
TOP = 8  # columns the argmax pass keeps (mono_fast_topk's largest k)

_lock = threading.Lock()
_counts = collections.Counter()


def stats():
    """Counters: "argmax", "topk" (kernel launches), "topk_kept" (answered from the argmax pass), and the reasons
    of calls sent to torch."""
    with _lock:
        return dict(_counts)


def _count(key):
    with _lock:
        _counts[key] += 1


def _argmax_parameters(input, dim=None, keepdim=False, *, out=None):
    """torch.argmax's parameters."""


def _topk_parameters(input, k, dim=-1, largest=True, sorted=True, *, out=None):
    """torch.topk's parameters."""


_ARGMAX_SIG = inspect.signature(_argmax_parameters)
_TOPK_SIG = inspect.signature(_topk_parameters)
_ARGMAX = (torch.argmax, torch.Tensor.argmax)
_TOPK = (torch.topk, torch.Tensor.topk)
_INDEX = (torch.Tensor.__getitem__,)


def _bind(sig, args, kwargs):
    try:
        b = sig.bind(*args, **kwargs)
    except TypeError:
        return None
    b.apply_defaults()
    return b.arguments


def _last_dim(x, dim):
    if dim is None or isinstance(dim, bool):
        return False
    try:
        d = operator.index(dim)
    except TypeError:
        return False
    return d in (-1, x.dim() - 1)


class _Kept:
    """The top-8 rows of the latest argmax passes, keyed by the rows they read. The key holds a weak reference to
    the base tensor, so a new tensor that reuses a freed one's memory and id never matches."""

    def __init__(self, size=4):
        self.size = size
        self.items = collections.OrderedDict()

    @staticmethod
    def key(x):
        base = x._base if x._base is not None else x
        return id(base), weakref.ref(base), x.storage_offset(), tuple(x.shape), tuple(x.stride()), x._version

    def put(self, x, values, indices):
        k = self.key(x)
        with _lock:
            self.items[(k[0],) + k[2:]] = (k[1], values, indices)
            while len(self.items) > self.size:
                self.items.popitem(last=False)

    def get(self, x):
        k = self.key(x)
        with _lock:
            hit = self.items.get((k[0],) + k[2:])
        if hit is None or hit[0]() is not k[1]():
            return None
        return hit[1], hit[2]


_kept = _Kept()


def _argmax(C, x, keepdim):
    values, indices, am = C.fast_pick(x, TOP)
    _kept.put(x, values, indices)
    _count("argmax")
    return am.reshape(*x.shape[:-1], *((1,) if keepdim else ()))


def _topk(C, x, k):
    hit = _kept.get(x)
    if hit is not None and k <= hit[0].shape[-1]:
        _count("topk_kept")
        return torch.return_types.topk((hit[0][..., :k].clone(), hit[1][..., :k].clone()))
    values, indices = C.fast_topk(x, k, False)
    _count("topk")
    return torch.return_types.topk((values, indices))


def _refused(reason):
    _count("torch: " + reason)


class PickRows(torch.Tensor):
    """Logits rows whose argmax / top-k run on mono_fast_topk (module docstring)."""

    @classmethod
    def __torch_function__(cls, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}

        def plain():
            with torch._C.DisableTorchFunctionSubclass():
                return func(*args, **kwargs)

        if guard.off(PIECE) or func not in _ARGMAX + _TOPK + _INDEX:
            return plain()
        if func in _INDEX:
            out = plain()
            return out.as_subclass(cls) if type(out) is torch.Tensor else out
        from . import _C
        if func in _ARGMAX:
            a = _bind(_ARGMAX_SIG, args, kwargs)
            if a is None or a["out"] is not None or not _last_dim(a["input"], a["dim"]):
                return plain()
            x = a["input"].as_subclass(torch.Tensor)
            return guard.route(PIECE, lambda: _argmax(_C, x, bool(a["keepdim"])), plain, _refused)
        a = _bind(_TOPK_SIG, args, kwargs)
        if (a is None or a["out"] is not None or a["largest"] is not True or a["sorted"] is not True
                or not _last_dim(a["input"], a["dim"]) or isinstance(a["k"], bool)):
            return plain()
        try:
            k = operator.index(a["k"])
        except TypeError:
            return plain()
        x = a["input"].as_subclass(torch.Tensor)
        return guard.route(PIECE, lambda: _topk(_C, x, k), plain, _refused)


def install(llama=None, q35=None):
    """Wrap BaseGenerate.logits (Qwen35 resolves logits there); False when already wrapped or switched off."""
    if MODE == "0":
        return False
    if llama is None:
        from comfy.text_encoders import llama
    if q35 is None:
        from comfy.text_encoders import qwen35 as q35
    cls = llama.BaseGenerate
    original = cls.logits
    if getattr(original, CLAIM, False) or getattr(original, "__comfy_mono_decode_xpu_logits__", False):
        return False

    def logits(self, x):
        out = original(self, x)
        if (isinstance(self, q35.Qwen35) and type(out) is torch.Tensor and out.device.type == "cuda"
                and out.dtype == torch.bfloat16 and not guard.off(PIECE)):
            return out.as_subclass(PickRows)
        return out

    setattr(logits, CLAIM, True)
    logits.__wrapped__ = original
    cls.logits = logits
    return True
