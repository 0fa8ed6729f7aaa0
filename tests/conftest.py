"""Test configuration: the `gpu` marker, import paths and shared helpers.

`-m "not gpu"` runs the oracle, host logic and C-ABI load checks (no CUDA device needed);
`-m gpu` runs the parity tests of the CUDA kernels through the C ABI against the CPU oracle.
"""
import os
import sys

import numpy as np
import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
PKG = os.path.join(ROOT, "comfy-mono-decode-xpu_b200")
for p in (ROOT, PKG):
    if p not in sys.path:
        sys.path.insert(0, p)


def pytest_configure(config):
    config.addinivalue_line("markers", "gpu: needs a CUDA device (B200) and the built libmono_b200.so")


@pytest.fixture(scope="session")
def cuda():
    import torch
    if not torch.cuda.is_available():
        pytest.skip("no CUDA device")
    from mono_b200 import _C  # raises ImportError when the library is missing: a failure, not a skip
    _C.pair_table(None, "cuda")
    return torch.device("cuda")


def bits_equal(a, b):
    """Bitwise equality of two arrays/tensors of the same dtype (NaN payloads and signed zeros included)."""
    import torch
    if isinstance(a, torch.Tensor):
        a = a.detach().cpu()
        if a.dtype == torch.bfloat16:
            a = a.view(torch.int16)
        a = a.numpy()
    if isinstance(b, torch.Tensor):
        b = b.detach().cpu()
        if b.dtype == torch.bfloat16:
            b = b.view(torch.int16)
        b = b.numpy()
    a, b = np.asarray(a), np.asarray(b)
    if a.shape != b.shape or a.dtype.itemsize != b.dtype.itemsize:
        return False
    return np.array_equal(a.view(f"u{a.dtype.itemsize}"), b.view(f"u{b.dtype.itemsize}"))


def bf16_bits(t):
    """A torch bf16 tensor -> numpy uint16 bit patterns."""
    return t.detach().cpu().contiguous().view(__import__("torch").int16).numpy().view(np.uint16)
