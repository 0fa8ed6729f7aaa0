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
    # bf16 GEMV: rows, K granularity, strides and alignment are checked before the launch
    rc = lib.mono_gemv_bf16(p, 4096, p, 9, 4096, 4096, p, 4096, None)
    assert rc == _lib.MONO_EINVAL and b"M" in lib.mono_last_error()
    rc = lib.mono_gemv_bf16(p, 4096, p, 1, 4096, 4000, p, 4096, None)
    assert rc == _lib.MONO_EINVAL and b"K" in lib.mono_last_error()
    rc = lib.mono_gemv_bf16(p, 4100, p, 2, 4096, 4096, p, 4096, None)
    assert rc == _lib.MONO_EINVAL and b"x_stride" in lib.mono_last_error()
    rc = lib.mono_gemv_bf16(p, 4096, ctypes.c_void_p(24), 1, 4096, 4096, p, 4096, None)
    assert rc == _lib.MONO_EINVAL and b"aligned" in lib.mono_last_error()
    rc = lib.mono_gemv_bf16(p, 4096, p, 1, 4096, 4096, p, 4000, None)
    assert rc == _lib.MONO_EINVAL and b"out_stride" in lib.mono_last_error()


def _fake(addr):
    """A 256-aligned fake device address: the builders and the planner only validate and record pointers."""
    import ctypes
    return ctypes.c_void_p(addr * 4096)


def test_layer_program_builds_and_plans_without_gpu():
    """A GDN layer program (rows, a|b, GEMV, conv, delta, gated-norm rows, out projection, MLP) is built and planned
    on the host; malformed ops are rejected with EINVAL before anything could launch."""
    import ctypes

    import numpy as np
    from mono_b200 import _lib
    lib = _lib.load()
    opb = lib.mono_program_op_bytes()
    assert 128 <= opb <= 512
    ops = np.zeros(16 * opb, dtype=np.uint8)
    P = ops.ctypes.data
    H, I, HK, HV, M = 4096, 12288, 16, 32, 5
    C, Z = (2 * HK + HV) * 128, HV * 128
    ptr = iter(range(1, 1000))
    f = lambda: _fake(next(ptr))  # noqa: E731
    W2 = (ctypes.c_void_p * 2)(f().value, f().value)
    R2 = (ctypes.c_int64 * 2)(C, Z)
    W1 = (ctypes.c_void_p * 1)(f().value)
    R1 = (ctypes.c_int64 * 1)(H)
    q, s, xn, proj, ab, raw, x = f(), f(), f(), f(), f(), f(), f()
    ok = _lib.MONO_OK
    assert lib.mono_program_rows(P, 0, 0, x, H, H, f(), ctypes.c_float(1e-6), None, 0, 0, None, xn, q, s, None, 1) == ok
    assert lib.mono_program_ab(P, 1, xn, H, H, f(), 2 * HV, ab, 0) == ok
    assert lib.mono_program_gemv(P, 2, W2, R2, 2, 0, H, q, s, proj, C + Z, None, 0, None, None, 1) == ok
    ws_bytes = lib.mono_gdn_step_workspace(M, C, HV)
    for i, delta in ((3, 0), (4, 1)):
        rc = lib.mono_program_gdn(P, i, delta, proj, f(), ab, f(), f(), f(), f(), f(), f(), f(), ctypes.c_float(1e-6),
                                  ctypes.c_float(128 ** -0.5), M, HK, HV, raw, f(), f(), f(), f(), f(), f(), f(),
                                  C + Z, C + Z, 2 * HV, f(), ws_bytes, 1)
        assert rc == ok, lib.mono_last_error()
    assert lib.mono_program_rows(P, 5, 3, raw, Z, Z, f(), ctypes.c_float(1e-6), f(), C + Z, 0, None, None, q, s, None, 1) == ok
    assert lib.mono_program_gemv(P, 6, W1, R1, 1, 0, Z, q, s, f(), H, x, H, None, None, 1) == ok
    assert lib.mono_program_plan(P, 7, M) == ok, lib.mono_last_error()
    # rejected: rows op K not a multiple of 1024, a pair without its LUT, more rows than the program allows
    assert lib.mono_program_rows(P, 7, 2, x, 1000, 1000, None, ctypes.c_float(0), None, 0, 0, None, None, q, s, None, 1) == _lib.MONO_EINVAL
    assert lib.mono_program_gemv(P, 7, W2, (ctypes.c_int64 * 2)(I, I), 2, 1, H, q, s, f(), I, None, 0, None, None, 1) == _lib.MONO_EINVAL
    assert lib.mono_program_plan(P, 7, 17) == _lib.MONO_EINVAL
    assert lib.mono_program_gdn(P, 7, 0, proj, f(), ab, f(), f(), f(), f(), f(), f(), f(), ctypes.c_float(1e-6),
                                ctypes.c_float(1.0), 9, HK, HV, raw, None, None, None, None, None, None, None,
                                C + Z, C + Z, 2 * HV, f(), ws_bytes, 1) == _lib.MONO_EINVAL  # M = 9 > 8 rows
    # a by-value launch of more than 16 ops is refused before any CUDA call
    big = np.zeros(17 * opb, dtype=np.uint8)
    assert lib.mono_program_launch(big.ctypes.data, None, 17, M, _fake(1), 0, None) == _lib.MONO_EINVAL
