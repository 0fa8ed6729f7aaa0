"""Per-device constant tables of the decode chains: the SiLU / sigmoid tables (torch's own values for every bf16
input, mono_b200._C.act_luts) and the 256 x 256 rotation of the REF activation step.

The rotation is the INT8 backend's own matrix when the backend is importable (comfy_kitchen's _build_hadamard(256),
the matrix its quantize_and_rotate_rowwise applies); otherwise the same matrix built here: the regular Hadamard
matrix of order 256 divided by 16, the Kronecker product of four copies of the regular order-4 matrix (-1 exactly
where i ^ j == 3), every entry +-1/16 (exact in bf16).
"""
from __future__ import annotations

import threading

import torch

_lock = threading.Lock()
_rot = {}


def silu_lut(device):
    from . import _C
    return _C.act_luts(device)[0]


def sigmoid_lut(device):
    from . import _C
    return _C.act_luts(device)[1]


def regular_hadamard_256(device=None):
    """The regular Hadamard matrix of order 256 / 16 as bf16 [256, 256]."""
    i = torch.arange(4)
    h4 = torch.where((i[:, None] ^ i[None, :]) == 3, -1.0, 1.0)
    h = h4
    for _ in range(3):
        h = torch.kron(h, h4)
    return (h / 16.0).to(torch.bfloat16).to(device).contiguous()


def hadamard(device):
    dev = torch.device(device)
    with _lock:
        h = _rot.get(dev)
    if h is None:
        try:
            from comfy_kitchen.tensor.int8_utils import _build_hadamard
            h = _build_hadamard(256, device=dev, dtype=torch.bfloat16).contiguous()
        except Exception:  # no backend here: the same matrix, built from its definition
            h = regular_hadamard_256(dev)
        with _lock:
            _rot[dev] = h
    return h
