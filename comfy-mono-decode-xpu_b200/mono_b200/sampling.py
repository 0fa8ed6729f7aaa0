"""Exact fast top-k for the verify step's sampling filter (the reference's comfy_mono_decode_xpu/sampling.py,
switch MONO_DECODE_XPU_SAMPLE_TOPK), on CUDA tensors through mono_topk_rows.

ComfyUI's sampling filters start with torch.topk(logits, top_k) over the verify rows (a few rows of ~248k fp32
logits). Inside the verify sampling's context this module answers that call with _C.topk_rows, which returns
the same values and indices in the same order as torch's top-k, ties included (include/mono_b200.h
mono_topk_rows). Every other sampling op (temperature, min-p, top-p, softmax, multinomial) stays upstream's.

verify_rows(C, lg0) hands the sampling the bf16 logits themselves as the stand-in for their fp32 copy: shape
queries pass through, .dtype reads fp32, torch.topk reads the bf16 rows directly (bf16 -> fp32 is exact) and any
other op gets the fp32 copy, made on first use. A later torch.sort(values, descending=True) of values this
context returned gets a copy and the index arange: they are already sorted, ties in order, and a stable sort
would return exactly that.

MODE: "1" (default) on, "0" off, "check": both run, torch's result is returned and mismatches are counted.
"""
from __future__ import annotations

import contextlib
import os
import threading

import torch

from . import guard

MODE = os.environ.get("MONO_DECODE_XPU_SAMPLE_TOPK", "1")
DEVICES = ("cuda",)  # device types served (the reference serves "xpu")
_lock = threading.Lock()
_stats = {"calls": 0, "checked": 0, "check_mismatch": 0, "skipped": 0, "sorted": 0, "lazy_rows": 0}
_aranges = {}


def stats():
    with _lock:
        return dict(_stats)


def _bump(key, n=1):
    with _lock:
        _stats[key] = _stats.get(key, 0) + n


def _topk_request(args, kwargs, want_dtype):
    """(x, k) when torch.topk(*args, **kwargs) is a call topk_rows answers exactly, else None: the last dim,
    largest first, sorted, no out=, a plain contiguous 2-D tensor of want_dtype with 1..16 rows of at least
    32768 elements, 1 <= k <= 64."""
    if len(args) < 2 or kwargs.get("out") is not None:
        return None
    x, k = args[0], args[1]
    dim = args[2] if len(args) > 2 else kwargs.get("dim", -1)
    largest = args[3] if len(args) > 3 else kwargs.get("largest", True)
    srt = args[4] if len(args) > 4 else kwargs.get("sorted", True)
    if type(x) is not torch.Tensor or type(k) is not int or dim not in (-1, 1) or largest is not True or srt is not True:
        return None
    if (x.device.type not in DEVICES or x.dtype != want_dtype or x.dim() != 2 or not x.is_contiguous()
            or not 1 <= x.shape[0] <= 16 or x.shape[1] < 32768 or not 1 <= k <= 64):
        return None
    return x, k


def _index_rows(R, k, device):
    key = (R, k, str(device))
    if key not in _aranges:
        _aranges[key] = torch.arange(k, device=device).expand(R, k).contiguous()
    return _aranges[key]


_SHAPE_QUERIES = (torch.Tensor.size, torch.Tensor.dim, torch.Tensor.numel, torch.Tensor.is_contiguous,
                  torch.Tensor.shape.__get__, torch.Tensor.ndim.__get__, torch.Tensor.device.__get__)
_TOPK = (torch.topk, torch.Tensor.topk)
_SORT = (torch.sort, torch.Tensor.sort)


class TopkRowsMode(torch.overrides.TorchFunctionMode):
    """Serves eligible torch.topk calls with C.topk_rows; `stand_in` (optional) is a bf16 [R, N] tensor that
    stands for stand_in.float() inside the context."""

    def __init__(self, C, stand_in=None):
        super().__init__()
        self.C = C
        self.stand_in = stand_in
        self.fp32 = None
        self.returned = []  # value tensors returned by topk_rows (sorted descending)

    def _dense(self, a):
        if a is self.stand_in:
            if self.fp32 is None:
                self.fp32 = self.stand_in.float()  # torch functions run without this mode inside the handler
            return self.fp32
        if isinstance(a, (list, tuple)):
            return type(a)(self._dense(v) for v in a)
        return a

    def _serve(self, x, k):
        try:
            v, i = self.C.topk_rows(x, k)
        except Exception as e:  # an argument check: torch computes it
            guard.failed("sample_topk", e)
            return None
        return v, i

    def __torch_function__(self, func, types, args=(), kwargs=None):
        kwargs = kwargs or {}
        on_stand_in = self.stand_in is not None and len(args) > 0 and args[0] is self.stand_in
        if on_stand_in:
            if func in _SHAPE_QUERIES:
                return func(*args, **kwargs)
            if func is torch.Tensor.dtype.__get__:
                return torch.float32
            if func in _TOPK and MODE != "check" and not guard.off("sample_topk"):
                req = _topk_request(args, kwargs, torch.bfloat16)
                if req is not None:
                    got = self._serve(*req)
                    if got is not None:
                        _bump("calls")
                        _bump("lazy_rows")
                        self.returned.append(got[0])
                        return torch.return_types.topk(got)
        if func in _SORT and len(args) > 0 and any(args[0] is v for v in self.returned):
            dim = args[1] if len(args) > 1 else kwargs.get("dim", -1)
            desc = args[2] if len(args) > 2 else kwargs.get("descending", False)
            if len(args) <= 3 and set(kwargs) <= {"dim", "descending", "stable"} and dim in (-1, 1) and desc is True:
                x = args[0]
                _bump("sorted")
                return torch.return_types.sort((x.clone(), _index_rows(x.shape[0], x.shape[1], x.device)))
        if self.stand_in is not None:
            args = self._dense(tuple(args))
            kwargs = {key: self._dense(val) for key, val in kwargs.items()}
        if func in _TOPK and not guard.off("sample_topk"):
            req = _topk_request(args, kwargs, torch.float32)
            if req is not None:
                got = self._serve(*req)
                if got is not None:
                    if MODE != "check":
                        _bump("calls")
                        self.returned.append(got[0])
                        return torch.return_types.topk(got)
                    ref = func(*args, **kwargs)
                    same = torch.equal(ref.indices, got[1]) and torch.equal(ref.values.view(torch.int32),
                                                                            got[0].view(torch.int32))
                    _bump("checked")
                    _bump("check_mismatch", int(not same))
                    return ref
            _bump("skipped")
        return func(*args, **kwargs)


def topk_mode(C):
    """The verify sampling's context: C.topk_rows serves its eligible torch.topk calls (a null context when the
    mode is off or C has no topk_rows)."""
    if MODE == "0" or guard.off("sample_topk") or not hasattr(C, "topk_rows"):
        return contextlib.nullcontext()
    return TopkRowsMode(C)


def verify_rows(C, lg0):
    """(context, rows) for sampling from the bf16 logits lg0 [R, N]: rows stands for lg0.float() — the bf16
    tensor itself, served lazily inside the context, or (mode off / check, or lg0 not eligible) the fp32 copy."""
    if (MODE in ("0", "check") or guard.off("sample_topk") or not hasattr(C, "topk_rows")
            or lg0.dtype != torch.bfloat16 or lg0.dim() != 2 or not lg0.is_contiguous()
            or lg0.device.type not in DEVICES):
        return topk_mode(C), lg0.float()
    return TopkRowsMode(C, stand_in=lg0), lg0
