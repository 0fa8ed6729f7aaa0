"""The C ABI library loads and exports every entry point include/mono_b200.h declares (no GPU needed)."""
import ctypes
import os
import re

from conftest import ROOT


def _declared():
    src = open(os.path.join(ROOT, "include", "mono_b200.h")).read()
    return sorted(set(re.findall(r"MONO_API\s+[\w\s\*]+?\b(mono_\w+)\s*\(", src)))


def test_header_declares_entry_points():
    names = _declared()
    assert "mono_w4a8_decode_linear" in names and "mono_last_error" in names
    assert len(names) >= 10


def test_library_exports_every_declared_symbol():
    from mono_b200 import _lib
    lib = _lib.load()
    for name in _declared():
        assert hasattr(lib, name), name


def test_binding_covers_header():
    from mono_b200 import _lib
    assert sorted(_lib.SIGNATURES) == _declared()


def test_library_has_no_torch_dependency():
    from mono_b200 import _lib
    deps = open(_lib.LIB_PATH, "rb").read()
    assert b"libtorch" not in deps and b"libc10" not in deps


def test_host_validation_without_gpu():
    """Argument checks run on the host before any CUDA call: bad shapes are rejected with EINVAL."""
    from mono_b200 import _lib
    lib = _lib.load()
    p = ctypes.c_void_p(16)
    # M = 17 rows is outside the kernel contract
    rc = lib.mono_w4a8_gptq_linear(p, p, p, p, None, 17, 4096, 4096, 2, 0, p, None)
    assert rc == _lib.MONO_EINVAL and b"M" in lib.mono_last_error()
    rc = lib.mono_w4a8_gptq_linear(p, p, p, p, None, 1, 4096, 1000, 2, 0, p, None)
    assert rc == _lib.MONO_EINVAL and b"K" in lib.mono_last_error()
    rc = lib.mono_w4a8_gptq_linear(p, p, p, p, None, 1, 4100, 4096, 2, 0, p, None)
    assert rc == _lib.MONO_EINVAL
    rc = lib.mono_w4a8_decode_linear(p, p, p, p, 0, p, p, None, 1, 4096, 4096, 32, 2, 0, p, None)
    assert rc == _lib.MONO_EINVAL and b"group_size" in lib.mono_last_error()
    rc = lib.mono_w4a8_gptq_linear(ctypes.c_void_p(8), p, p, p, None, 1, 4096, 4096, 2, 0, p, None)
    assert rc == _lib.MONO_EINVAL and b"aligned" in lib.mono_last_error()
