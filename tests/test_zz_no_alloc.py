"""mono_rot_quant_noalloc: rot_quant for callers that cannot allocate device memory (a host framework that
owns every device allocation through its own pool, a plugin loaded into a process whose allocator it may
not touch). It uses a fixed scratch array inside the library instead of a caller workspace; its results
must equal those of mono_rot_quant with a workspace. This file is collected last on purpose: if it fails, a run
that stops at the first failure has already run every other test."""
import ctypes

import numpy as np
import pytest
import torch

from oracle import w4a8 as ow

pytestmark = pytest.mark.gpu


def _rot_quant_with_workspace(lib, x, h):
    M, K = x.shape
    q = torch.empty(M, K, dtype=torch.int8, device=x.device)
    s = torch.empty(M, dtype=torch.float32, device=x.device)
    ws = torch.zeros(lib.mono_rot_quant_workspace(M, K), dtype=torch.uint8, device=x.device)
    rc = lib.mono_rot_quant(x.data_ptr(), h.data_ptr(), M, K, q.data_ptr(), s.data_ptr(), ws.data_ptr(),
                            torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.mono_last_error()
    return q, s


def _rot_quant_noalloc(lib, x, h):
    M, K = x.shape
    q = torch.empty(M, K, dtype=torch.int8, device=x.device)
    s = torch.empty(M, dtype=torch.float32, device=x.device)
    rc = lib.mono_rot_quant_noalloc(x.data_ptr(), h.data_ptr(), M, K, q.data_ptr(), s.data_ptr(),
                                    torch.cuda.current_stream().cuda_stream)
    assert rc == 0, lib.mono_last_error()
    return q, s


def test_rot_quant_noalloc_matches_workspace_entry(cuda):
    from mono_b200 import _lib
    lib = _lib.load()
    h = torch.from_numpy(ow.hadamard_256().view(np.int16)).view(torch.bfloat16).to(cuda)
    g = torch.Generator().manual_seed(2024)
    # two calls in a row (different shapes and inputs): the shared scratch keeps the previous call's rows
    for M, K in ((8, 4096), (16, 12288), (3, 12288)):
        x = (torch.randn(M, K, generator=g) * torch.exp(torch.randn(M, K, generator=g))).to(torch.bfloat16).to(cuda)
        q_ref, s_ref = _rot_quant_with_workspace(lib, x, h)
        q, s = _rot_quant_noalloc(lib, x, h)
        torch.cuda.synchronize()
        assert torch.equal(q, q_ref), (M, K)  # same tolerance as the other rot_quant tests: bit-exact
        assert torch.equal(s.view(torch.int32), s_ref.view(torch.int32)), (M, K)


def test_rot_quant_noalloc_rejects_shapes_beyond_its_scratch(cuda):
    from mono_b200 import _lib
    lib = _lib.load()
    dummy = ctypes.c_void_p(256)  # never dereferenced: the shape check comes first
    assert lib.mono_rot_quant_noalloc(dummy, dummy, 17, 4096, dummy, dummy, None) == _lib.MONO_EINVAL
    assert b"fixed scratch" in lib.mono_last_error()
    assert lib.mono_rot_quant_noalloc(dummy, dummy, 8, 16384, dummy, dummy, None) == _lib.MONO_EINVAL


def test_rot_quant_noalloc_in_a_cuda_graph(cuda):
    """The use the header names: after one call in the context, the entry is captured in a CUDA graph (its memset
    node and two kernels, nothing allocated) and replayed with new inputs written into the captured buffers; every
    replay equals the workspace entry bit for bit."""
    from mono_b200 import _lib
    lib = _lib.load()
    h = torch.from_numpy(ow.hadamard_256().view(np.int16)).view(torch.bfloat16).to(cuda)
    g = torch.Generator().manual_seed(7)
    M, K = 8, 4096
    x = torch.zeros(M, K, dtype=torch.bfloat16, device=cuda)
    q = torch.empty(M, K, dtype=torch.int8, device=cuda)
    s = torch.empty(M, dtype=torch.float32, device=cuda)
    _rot_quant_noalloc(lib, x, h)  # the first call in the context (outside any capture)
    torch.cuda.synchronize()
    side = torch.cuda.Stream()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=side):
        rc = lib.mono_rot_quant_noalloc(x.data_ptr(), h.data_ptr(), M, K, q.data_ptr(), s.data_ptr(),
                                        side.cuda_stream)
    assert rc == 0, lib.mono_last_error()
    for _ in range(2):
        x.copy_((torch.randn(M, K, generator=g) * torch.exp(torch.randn(M, K, generator=g))).to(torch.bfloat16))
        graph.replay()
        torch.cuda.synchronize()
        q_ref, s_ref = _rot_quant_with_workspace(lib, x, h)
        torch.cuda.synchronize()
        assert torch.equal(q, q_ref)
        assert torch.equal(s.view(torch.int32), s_ref.view(torch.int32))
    del graph
