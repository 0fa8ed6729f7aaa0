"""The two-GPU one-shot all-reduce kernel (include/mono_b200.h mono_allreduce2_bf16) on one GPU:
  * loopback: the "peer" area is this rank's own, so each call stores the input into its own receive buffer,
    raises its own counters and returns bf16(in + in) — the arithmetic and the alternating buffers, bit for bit,
    over several calls of different sizes;
  * a wait that runs out: the peer area is a second local area whose counters nobody raises on the waiting side;
    every CTA gives up after its 1 s limit, the device error word reads 6 (DEV_PEER_TIMEOUT), the output is left
    alone and the context stays usable. (No fault, no trap: the bounded wait is the thing under test.)"""
import ctypes

import numpy as np
import pytest
import torch

pytestmark = pytest.mark.gpu


def _area(lib, _lib, cap):
    p = ctypes.c_void_p()
    _lib.call("mono_p2p_area_alloc", lib.mono_allreduce2_area_bytes(cap), ctypes.byref(p))
    return p.value


def _stream():
    return torch.cuda.current_stream().cuda_stream


def test_loopback_sums_in_with_itself(cuda):
    from mono_b200 import _C, _lib
    lib = _lib.load()
    cap = 8 * 4096
    area = _area(lib, _lib, cap)
    calls = torch.zeros(16, dtype=torch.int32, device=cuda)
    try:
        g = torch.Generator().manual_seed(3)
        for n in (8 * 4096, 4096, 8 * 4096, 64):
            x = (torch.randn(n, generator=g) * 3).bfloat16()
            t = x.to(cuda)
            _lib.call("mono_allreduce2_bf16", t.data_ptr(), t.data_ptr(), n, area, area, cap, calls.data_ptr(), _stream())
            torch.cuda.synchronize()
            ref = (x.float() + x.float()).bfloat16()
            assert torch.equal(t.cpu().view(torch.int16), ref.view(torch.int16)), n
        assert calls.cpu().tolist() == [4] * 16
        assert _C.device_status() == 0
        with pytest.raises(_lib.MonoError):
            _lib.call("mono_allreduce2_bf16", t.data_ptr(), t.data_ptr(), cap + 8, area, area, cap, calls.data_ptr(),
                      _stream())
    finally:
        _lib.call("mono_p2p_area_free", area)


def test_a_wait_nobody_ends_gives_up_with_status_6(cuda):
    from mono_b200 import _C, _lib
    lib = _lib.load()
    cap = 4096
    mine, other = _area(lib, _lib, cap), _area(lib, _lib, cap)
    calls = torch.zeros(16, dtype=torch.int32, device=cuda)
    try:
        t = torch.ones(cap, dtype=torch.bfloat16, device=cuda)
        _lib.call("mono_allreduce2_bf16", t.data_ptr(), t.data_ptr(), cap, mine, other, cap, calls.data_ptr(), _stream())
        torch.cuda.synchronize()
        assert _C.device_status() == 6
        assert torch.equal(t.cpu(), torch.ones(cap, dtype=torch.bfloat16))  # the output is not written
        assert float(torch.ones(4, device=cuda).sum().item()) == 4.0  # the context still works
    finally:
        _lib.call("mono_p2p_area_free", mine)
        _lib.call("mono_p2p_area_free", other)
