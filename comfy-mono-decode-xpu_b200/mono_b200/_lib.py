"""ctypes binding of libmono_b200.so (the C ABI declared in include/mono_b200.h).

The library is built in-tree (csrc/build.py) and loaded from this directory. A missing or unloadable
library raises ImportError: there is no CPU or eager fallback behind these entry points.
"""
from __future__ import annotations

import ctypes
import os
import re
import threading

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libmono_b200.so")

P = ctypes.c_void_p
I = ctypes.c_int
I64 = ctypes.c_int64
SZ = ctypes.c_size_t

# name -> (restype, argtypes); every int-returning entry returns a MONO_* status
SIGNATURES = {
    "mono_last_error": (ctypes.c_char_p, []),
    "mono_abi_version": (I, []),
    "mono_device_status": (I, [ctypes.POINTER(I), I]),
    "mono_trace_bytes": (SZ, []),
    "mono_trace_enable": (I, [P, SZ]),
    "mono_w4a8_decode_linear": (I, [P, P, P, P, I, P, P, P, I64, I64, I64, I64, I, I, P, P]),
    "mono_w4_pair_table": (I, [P, P, P]),
    "mono_w4a8_gptq_linear": (I, [P, P, P, P, P, I64, I64, I64, I, I, P, P]),
    "mono_w4a8_gptq_linear_bf16": (I, [P, P, P, P, I64, I64, I64, I, I, P, P]),
    "mono_w4_tiled_bytes": (SZ, [I, I64, I64]),
    "mono_w4_repack": (I, [I, P, P, I64, I64, P, P]),
    "mono_act_quant": (I, [P, I64, I64, P, P, P]),
    "mono_rot_quant_workspace": (SZ, [I64, I64]),
    "mono_rot_quant": (I, [P, P, I64, I64, P, P, P, P]),
    "mono_rot_quant_noalloc": (I, [P, P, I64, I64, P, P, P]),
    "mono_mlp_gptq_workspace": (SZ, [I64, I64]),
    "mono_mlp_gptq": (I, [P, P, ctypes.c_float, P, P, P, P, I64, I64, I64, I, P, P, SZ, P]),
    "mono_qk_norm_rope_kv": (I, [P, I64, I64, P, I64, P, I64, P, P, P, P, P, I64, P, I64, I64, I64, ctypes.c_float,
                                 ctypes.c_float, I64, P, P, P]),
    "mono_qk_norm_rope_kv_streams": (I, [P, I64, I64, P, I64, P, I64, P, P, P, P, P, I64, P, I64, I64, I64, I64,
                                         ctypes.c_float, ctypes.c_float, I64, P, P, P]),
    "mono_tree_attention_workspace": (SZ, [I64, I64]),
    "mono_tree_attention_streams_workspace": (SZ, [I64, I64, I64]),
    "mono_tree_attention_streams": (I, [P, P, P, P, P, P, P, I64, I64, I64, I64, I64, I64, I64, I64, P, P, SZ, P]),
    "mono_gdn_step_streams_workspace": (SZ, [I64, I64, I64, I64]),
    "mono_gdn_step_deferred_streams": (I, [P, P, P, P, P, P, P, P, P, P, ctypes.c_float, ctypes.c_float, I64, I64, I64,
                                           I64, P, P, I64, P, P, P, P, P, P, I64, I64, I64, P, SZ, P]),
    "mono_tree_attention": (I, [P, P, P, P, P, P, P, I64, I64, I64, I64, P, P, SZ, P]),
    "mono_gdn_step_workspace": (SZ, [I64, I64, I64]),
    "mono_rowlin_gptq_workspace": (SZ, [I64]),
    "mono_draft_embed_norm_cat": (I, [P, I64, I64, P, I64, I64, P, P, I64, P, ctypes.c_float, I64, P, I64, P]),
    "mono_mtp_prep_draft_streams": (I, [P, I64, I64, P, I64, I64, P, I64, P, I64, I64, P, I64, I64, P]),
    "mono_mtp_prep_verify_streams": (I, [P, I64, P, I64, I64, P, I64, P, I64, P, I64, P, I64, P, I64, I64, I64, P]),
    "mono_rowlin_gptq": (I, [P, I, P, ctypes.c_float, P, I64, I64, P, P, P, I, I64, I64, P, P, P, P, SZ, P]),
    "mono_rowlin_norm_ab_gptq": (I, [P, P, ctypes.c_float, P, P, I, I64, I64, P, P, P, I64, P, I64, P, SZ, P]),
    "mono_rmsnorm_add": (I, [P, I64, P, I64, P, ctypes.c_float, I64, I64, P, P, I64, P]),
    "mono_lut_mul": (I, [P, I64, P, I64, I64, P, I64, I64, P, I64, P]),
    "mono_topk_workspace": (SZ, [I64]),
    "mono_fast_topk": (I, [P, I64, I64, I64, I, I, P, P, P, P, SZ, P]),
    "mono_mtp_prep_draft": (I, [P, I64, P, I64, I64, P, P, I64, P, P]),
    "mono_mtp_prep_verify": (I, [P, P, I64, P, P, P, I64, P, P, I64, I64, P]),
    "mono_mtp_accept": (I, [P, P, P, P, P, I64, I64, P, I64, P, P, P, P, I64, I64, I64, I64, P, P]),
    "mono_gdn_step": (I, [P, P, P, P, P, P, P, P, P, P, ctypes.c_float, ctypes.c_float, I64, I64, I64, P, P, SZ, P]),
    "mono_gdn_step_deferred": (I, [P, P, P, P, P, P, P, P, P, P, ctypes.c_float, ctypes.c_float, I64, I64, I64, P, P, P,
                                   P, P, P, P, P, I64, I64, I64, P, SZ, P]),
    "mono_gemv_bf16": (I, [P, I64, P, I64, I64, I64, P, I64, P]),
    "mono_lmhead_workspace": (SZ, []),
    "mono_lmhead_pick": (I, [P, I64, P, I64, I64, I64, I64, I64, P, P, P, P, P, I64, P, SZ, P]),
    "mono_allreduce2_area_bytes": (SZ, [I64]),
    "mono_p2p_area_alloc": (I, [SZ, P]),
    "mono_p2p_area_free": (I, [P]),
    "mono_ipc_handle": (I, [P, P, SZ]),
    "mono_ipc_open": (I, [P, SZ, P]),
    "mono_ipc_close": (I, [P]),
    "mono_allreduce2_bf16": (I, [P, P, I64, P, P, I64, P, P]),
    "mono_topk_rows_workspace": (SZ, [I64, I64]),
    "mono_topk_rows": (I, [P, I, I64, I64, I64, P, P, P, SZ, P]),
    "mono_program_op_bytes": (SZ, []),
    "mono_program_workspace": (SZ, []),
    "mono_program_rows": (I, [P, I, I, P, I64, I64, P, ctypes.c_float, P, I64, I64, P, P, P, P, P, I]),
    "mono_program_gemv": (I, [P, I, P, P, I, I, I64, P, P, P, I64, P, I64, P, P, I]),
    "mono_program_quant": (I, [P, I, P, I64, P, P, P, I]),
    "mono_program_ab": (I, [P, I, P, I64, I64, P, I64, P, I]),
    "mono_program_gdn": (I, [P, I, I, P, P, P, P, P, P, P, P, P, P, ctypes.c_float, ctypes.c_float, I64, I64, I64, P, P,
                             P, P, P, P, P, P, I64, I64, I64, P, SZ, I]),
    "mono_program_plan": (I, [P, I, I64]),
    "mono_program_launch": (I, [P, P, I, I64, P, I, P]),
    "mono_gdn_ab": (I, [P, I64, P, I64, I64, I64, P, P]),
    "mono_layer_post_gptq_workspace": (SZ, [I64, I64, I64]),
    "mono_layer_post_gptq": (I, [P, P, I64, P, I64, I64, P, P, P, ctypes.c_float, P, P, P, P, I64, I64, I64, P, P, SZ,
                                 P]),
    "mono_layer_gdn_gptq_workspace": (SZ, [I64, I64, I64, I64, I64]),
    "mono_layer_gdn_gptq": (I, [P, P, ctypes.c_float, P, P, P, P, P, P, P, P, P, ctypes.c_float, ctypes.c_float, P, P, P,
                                P, P, P, P, P, P, ctypes.c_float, P, P, P, P, I64, I64, I64, I64, I64, P, P, SZ, P]),
}

MONO_OK, MONO_EINVAL, MONO_ECUDA, MONO_ETIMEOUT, MONO_EDEVICE = 0, 1, 2, 3, 4
OUT_F32, OUT_BF16 = 0, 2
FMT_GPTQ, FMT_REF = 0, 1
LAYOUT_ROW, LAYOUT_TILED = 0, 1
SCALE_FP8, SCALE_F32 = 0, 1
TOPK_BF16, TOPK_INDEX_ORDER = 1, 2

_lock = threading.Lock()
_lib = None


class MonoError(RuntimeError):
    """A C-ABI call returned a non-zero status (message from mono_last_error()), or the Python binding refused an
    argument before the call (status MONO_EINVAL, like the C-side checks)."""

    def __init__(self, name, status, message):
        super().__init__(f"{name}: status {status}: {message}")
        self.status = status
        self.message = message

    @property
    def reason(self):
        """The message without its "(got ...)" detail: one key per kind of rejection."""
        return re.sub(r"\s*\(got [^)]*\)", "", self.message).strip()


def rejected(exc) -> bool:
    """True when `exc` is an argument rejection (status MONO_EINVAL): the call lies outside what the kernels
    accept and nothing was launched; any other exception is a failure."""
    return isinstance(exc, MonoError) and exc.status == MONO_EINVAL


def load():
    """Load the library once and declare every signature of SIGNATURES."""
    global _lib
    with _lock:
        if _lib is None:
            if not os.path.isfile(LIB_PATH):
                raise ImportError(f"{LIB_PATH} is not built: run python csrc/build.py (or __graft_entry__.build())")
            lib = ctypes.CDLL(LIB_PATH)
            for name, (res, args) in SIGNATURES.items():
                fn = getattr(lib, name)
                fn.restype = res
                fn.argtypes = args
            _lib = lib
    return _lib


def call(name, *args):
    """Call an int-status entry point; a non-zero status raises MonoError (a RuntimeError)."""
    lib = load()
    status = getattr(lib, name)(*args)
    if status != MONO_OK:
        msg = lib.mono_last_error()
        raise MonoError(name, status, msg.decode() if msg else "")
    return status


def exported_symbols():
    return list(SIGNATURES)
