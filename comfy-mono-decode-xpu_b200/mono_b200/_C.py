"""The reference's native op surface (comfy_mono_decode_xpu._C, csrc/bindings.cpp:70-104) over torch CUDA
tensors, implemented by the C ABI of libmono_b200.so.

Same op names, argument order and meaning; outputs are allocated here with torch (the C ABI never
allocates) and every call is enqueued on torch's current CUDA stream. Argument errors raise RuntimeError
before anything is launched, as the reference's TORCH_CHECKs do.
"""
from __future__ import annotations

import threading
import weakref

import torch

from . import _lib

_tables = {}
_tables_lock = threading.Lock()


def _check(cond, msg):
    """An argument check of the binding: raises the C ABI's argument rejection (MonoError, MONO_EINVAL)."""
    if not cond:
        raise _lib.MonoError("argument", _lib.MONO_EINVAL, msg)


def _cuda(*ts):
    for t in ts:
        _check(t is not None and t.is_cuda, "operands must be CUDA tensors")
    dev = ts[0].device
    for t in ts:
        _check(t.device == dev, "operands must be on one device")


def _stream(dev):
    return torch.cuda.current_stream(dev).cuda_stream


def _p(t):
    return None if t is None else t.data_ptr()


def pair_table(codebook, device):
    """REF decode table for `codebook` (None = float(i - 8)), cached per (device, codebook tensor, version).
    The entry holds a weak reference to the codebook: a new tensor that reuses a freed codebook's address
    (same data_ptr, version 0) gets its own table."""
    dev = torch.device(device)
    key = (dev, None) if codebook is None else (dev, codebook.data_ptr())
    with _tables_lock:
        hit = _tables.get(key)
    tab = None
    if hit is not None:
        ref, version, cached = hit
        if codebook is None or (ref() is codebook and version == codebook._version):
            tab = cached
    if tab is None:
        if codebook is not None:
            _check(codebook.dtype == torch.float32 and codebook.numel() == 16 and codebook.is_contiguous(),
                   "codebook f32 [16]")
            _cuda(codebook)
        tab = torch.empty(65536, dtype=torch.int16, device=dev)
        with torch.cuda.device(dev):
            _lib.call("mono_w4_pair_table", _p(codebook), tab.data_ptr(), _stream(dev))
        with _tables_lock:
            _tables[key] = (None if codebook is None else weakref.ref(codebook),
                            None if codebook is None else codebook._version, tab)
    return tab


def w4a8_decode_linear(x, x_scale, packed, s_rel, s_channel, codebook=None, residual=None, group_size=16,
                       out_dtype_code=2, cols=0, fast=False, tiled=False, N=None):
    """out[m, n] = cast(float(int32 dot(x[m], decode(w[n]))) * x_scale[m] * s_channel[n]) (+ residual).
    Reference: csrc/w4a8_decode.sycl:325-370. `cols` and `fast` are the reference's tuning knobs and are
    accepted for signature compatibility; `tiled` selects mono_w4_repack's tile-major weights."""
    _cuda(x, x_scale, packed, s_channel)
    _check(x.dtype == torch.int8 and x.dim() == 2 and x.is_contiguous(), "x must be contiguous int8 [M, K]")
    M, K = x.shape
    if tiled:
        N = s_channel.numel()
        _check(packed.numel() == _lib.load().mono_w4_tiled_bytes(1, N, K), "tiled weight size")
    else:
        N = packed.shape[0]
        _check(packed.dtype in (torch.int8, torch.uint8) and packed.is_contiguous() and packed.dim() == 2
               and packed.shape[1] * 2 == K, "packed must be contiguous int8 [N, K/2]")
        _check(s_rel.is_contiguous() and s_rel.numel() == N * (K // group_size), "s_rel must be contiguous [N, K/G]")
        _check(s_rel.dtype == torch.float8_e4m3fn, "s_rel must be fp8 e4m3")
    _check(x_scale.dtype == torch.float32 and x_scale.is_contiguous() and x_scale.numel() == M, "x_scale f32 [M]")
    _check(s_channel.dtype == torch.float32 and s_channel.is_contiguous() and s_channel.numel() == N,
           "s_channel f32 [N]")
    _check(out_dtype_code in (0, 2), "out dtype fp32 or bf16")
    dtype = torch.float32 if out_dtype_code == 0 else torch.bfloat16
    out = torch.empty((M, N), dtype=dtype, device=x.device)
    if residual is not None:
        _check(residual.dtype == dtype and residual.is_contiguous() and residual.numel() == M * N,
               "residual must match output")
    tab = pair_table(codebook, x.device)
    with torch.cuda.device(x.device):
        _lib.call("mono_w4a8_decode_linear", _p(x), _p(x_scale), _p(packed), _p(s_rel), _lib.SCALE_FP8,
                  _p(s_channel), _p(tab), _p(residual), M, N, K, group_size, out_dtype_code,
                  _lib.LAYOUT_TILED if tiled else _lib.LAYOUT_ROW, _p(out), _stream(x.device))
    return out


def w4a8_gptq_linear(x, x_scale, packed, scales, residual=None, out_dtype_code=2, tiled=False, N=None, out=None):
    """GPTQ W4A8 linear (BASELINE configs[0] format): int4 nibbles v + 8 [N, K/2], fp16 scales [N, K/128];
    tiled=True: `packed` is the w4_repack copy (pass N; `scales` is ignored)."""
    _cuda(x, x_scale, packed)
    _check(x.dtype == torch.int8 and x.dim() == 2 and x.is_contiguous(), "x must be contiguous int8 [M, K]")
    M, K = x.shape
    if tiled:
        _check(N is not None and packed.numel() == _lib.load().mono_w4_tiled_bytes(0, N, K), "tiled weight size")
    else:
        N = packed.shape[0]
        _check(packed.dtype in (torch.int8, torch.uint8, torch.int32) and packed.is_contiguous()
               and packed.numel() * packed.element_size() == N * K // 2, "packed must be contiguous [N, K/2] bytes")
        _check(scales.dtype == torch.float16 and scales.is_contiguous() and scales.numel() == N * (K // 128),
               "scales must be contiguous fp16 [N, K/128]")
    _check(x_scale.dtype == torch.float32 and x_scale.numel() == M, "x_scale f32 [M]")
    dtype = torch.float32 if out_dtype_code == 0 else torch.bfloat16
    if out is None:
        out = torch.empty((M, N), dtype=dtype, device=x.device)
    _check(out.dtype == dtype and out.is_contiguous() and out.numel() == M * N, "out must be contiguous [M, N]")
    if residual is not None:
        _check(residual.dtype == dtype and residual.is_contiguous() and residual.numel() == M * N,
               "residual must match output")
    with torch.cuda.device(x.device):
        _lib.call("mono_w4a8_gptq_linear", _p(x), _p(x_scale), _p(packed), _p(scales), _p(residual), M, N, K,
                  out_dtype_code, _lib.LAYOUT_TILED if tiled else _lib.LAYOUT_ROW, _p(out), _stream(x.device))
    return out


def w4a8_gptq_linear_bf16(x, packed, scales, residual=None, out_dtype_code=2, tiled=False, N=None, out=None):
    """Config 0's whole op in one launch: bf16 x [M, K] -> per-token int8 quant (in the kernel) -> GPTQ W4A8
    GEMV -> out. Same results as act_quant followed by w4a8_gptq_linear."""
    _cuda(x, packed)
    _check(x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous(), "x must be contiguous bf16 [M, K]")
    M, K = x.shape
    if tiled:
        _check(N is not None and packed.numel() == _lib.load().mono_w4_tiled_bytes(0, N, K), "tiled weight size")
    else:
        N = packed.shape[0]
        _check(packed.numel() * packed.element_size() == N * K // 2 and packed.is_contiguous(), "packed [N, K/2] bytes")
        _check(scales.dtype == torch.float16 and scales.numel() == N * (K // 128), "scales fp16 [N, K/128]")
    dtype = torch.float32 if out_dtype_code == 0 else torch.bfloat16
    if out is None:
        out = torch.empty((M, N), dtype=dtype, device=x.device)
    _check(out.dtype == dtype and out.is_contiguous() and out.numel() == M * N, "out must be contiguous [M, N]")
    if residual is not None:
        _check(residual.dtype == dtype and residual.is_contiguous() and residual.numel() == M * N,
               "residual must match output")
    with torch.cuda.device(x.device):
        _lib.call("mono_w4a8_gptq_linear_bf16", _p(x), _p(packed), _p(scales), _p(residual), M, N, K, out_dtype_code,
                  _lib.LAYOUT_TILED if tiled else _lib.LAYOUT_ROW, _p(out), _stream(x.device))
    return out


def w4_repack(fmt, packed, scales, N, K):
    """The tile-major copy (one uint8 tensor: weights and scales per chunk item) of a W4 weight."""
    _cuda(packed, scales)
    _check(packed.is_contiguous() and scales.is_contiguous(), "contiguous operands")
    out = torch.empty(_lib.load().mono_w4_tiled_bytes(fmt, N, K), dtype=torch.uint8, device=packed.device)
    with torch.cuda.device(packed.device):
        _lib.call("mono_w4_repack", fmt, _p(packed), _p(scales), N, K, _p(out), _stream(packed.device))
    return out


def act_quant(x):
    """GPTQ per-token int8 quantization of bf16 rows: (q int8 [..., K], scale f32 [..., 1])."""
    _cuda(x)
    _check(x.dtype == torch.bfloat16 and x.is_contiguous(), "x bf16 contiguous")
    K = x.shape[-1]
    M = x.numel() // K
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    s = torch.empty((*x.shape[:-1], 1), dtype=torch.float32, device=x.device)
    if M:
        with torch.cuda.device(x.device):
            _lib.call("mono_act_quant", _p(x), M, K, _p(q), _p(s), _stream(x.device))
    return q, s


_rot_ws = {}


def rot_quant(x, h, order=0):
    """ConvRot rotation + row-wise INT8 quantization (csrc/act_prep.sycl:97-110): (q, scale [..., 1])."""
    _cuda(x, h)
    _check(x.dtype == torch.bfloat16 and x.is_contiguous(), "x bf16 contiguous")
    _check(h.dtype == torch.bfloat16 and h.is_contiguous() and h.numel() == 65536, "H bf16 [256,256]")
    K = x.shape[-1]
    M = x.numel() // K
    _check(K % 256 == 0, "K must be a multiple of 256")
    q = torch.empty(x.shape, dtype=torch.int8, device=x.device)
    s = torch.empty((*x.shape[:-1], 1), dtype=torch.float32, device=x.device)
    if M == 0:
        return q, s
    need = _lib.load().mono_rot_quant_workspace(M, K)
    key = x.device
    ws = _rot_ws.get(key)
    if ws is None or ws.numel() < need:
        ws = torch.zeros(need, dtype=torch.uint8, device=x.device)
        _rot_ws[key] = ws
    with torch.cuda.device(x.device):
        _lib.call("mono_rot_quant", _p(x), _p(h), M, K, _p(q), _p(s), _p(ws), _stream(x.device))
    return q, s


def device_status(reset=True):
    """The device error word (0 = no bounded wait has given up)."""
    import ctypes
    code = ctypes.c_int(0)
    _lib.load().mono_device_status(ctypes.byref(code), 1 if reset else 0)
    return code.value


# ---- constants of the fused kernels -------------------------------------------------------------------

_luts = {}


def act_luts(device):
    """(silu, sigmoid) of every bf16 bit pattern as bf16 [65536], from torch's own F.silu / torch.sigmoid on
    the device (as comfy_mono_decode_xpu/layer.py:100-102 builds them)."""
    dev = torch.device(device)
    c = _luts.get(dev)
    if c is None:
        allbf = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16).to(dev)
        c = _luts[dev] = (torch.nn.functional.silu(allbf).contiguous(), torch.sigmoid(allbf).contiguous())
    return c


_mlp_ws = {}


def _workspace(table, key, nbytes, device):
    ws = table.get(key)
    if ws is None or ws.numel() < nbytes:
        ws = torch.zeros(nbytes, dtype=torch.uint8, device=device)  # zero-filled: barrier words start at 0
        table[key] = ws
    return ws


def mlp_gptq(x, norm_w, eps, gate, up, down, silu_lut=None, residual=True, out=None, I=None):
    """Fused GPTQ MLP block (include/mono_b200.h mono_mlp_gptq). gate/up/down: tile-major copies from
    w4_repack. x bf16 [..., H]; returns bf16 [..., H] (out may be x: in place)."""
    _cuda(x)
    _check(x.dtype == torch.bfloat16 and x.is_contiguous(), "x bf16 contiguous")
    H = x.shape[-1]
    M = x.numel() // H
    if I is None:  # the tiled GPTQ copy holds N * K / 2 weight bytes + N * K / 64 scale bytes
        I = gate.numel() * 64 // (33 * H)
    if silu_lut is None:
        silu_lut = act_luts(x.device)[0]
    if norm_w is not None:
        _check(norm_w.dtype == torch.bfloat16 and norm_w.numel() == H and norm_w.is_contiguous(), "norm_w bf16 [H]")
    if out is None:
        out = torch.empty_like(x)
    need = _lib.load().mono_mlp_gptq_workspace(H, I)
    ws = _workspace(_mlp_ws, (x.device, H, I), need, x.device)
    with torch.cuda.device(x.device):
        _lib.call("mono_mlp_gptq", _p(x), _p(norm_w), float(eps), _p(gate), _p(up), _p(down), _p(silu_lut), M, H, I,
                  1 if residual else 0, _p(out), _p(ws), need, _stream(x.device))
    return out


def qk_norm_rope_kv(rawq, rawk, vn, weightq, weightk, freqs, key, value, position, epsq, epsk, rd, streams=1):
    """Q/K head RMSNorm + partial RoPE + K/V cache write (the reference's _C.qk_norm_rope_kv,
    csrc/rope_kv.sycl:120-245). rawq bf16 [1, S, Hq, 256] (the query half of gated heads: head stride 512, or
    dense), rawk / vn bf16 [1, S, Hk, 256] (dense heads), weights bf16 [256], freqs fp32 [S, rd/2, 2, 2], key /
    value caches bf16 [1, Hk, cap, 256] (written in place at position[s]), position int64 [>= S].
    Returns (q [1, Hq, S, 256], k [1, Hk, S, 256]).
    streams > 1 (batched decode streams, include/mono_b200.h mono_qk_norm_rope_kv_streams): the S rows are
    `streams` groups of S / streams, the caches [1, streams * Hk, cap, 256] (stream b: heads [b Hk, (b + 1) Hk));
    returns q [1, streams * Hq, S / streams, 256] and k [1, streams * Hk, S / streams, 256]."""
    _cuda(rawq, rawk, vn, weightq, weightk, freqs, key, value, position)
    _check(rawq.dtype == torch.bfloat16 and rawq.dim() == 4 and rawq.size(0) == 1 and rawq.size(3) == 256
           and rawq.stride(3) == 1, "Q: bf16 [1, S, Hq, 256]")
    S, Hq, Hk = rawq.size(1), rawq.size(2), rawk.size(2)
    _check(streams >= 1 and S % streams == 0, "rows in equal groups per stream")
    R = S // streams
    _check(rawk.dim() == 4 and rawk.shape == vn.shape and rawk.size(1) == S and rawk.stride(3) == 1 and
           rawk.stride(2) == 256 and vn.stride(3) == 1 and vn.stride(2) == 256, "K/V: bf16 [1, S, Hk, 256], dense heads")
    _check(all(t.dtype == torch.bfloat16 for t in (rawk, vn, key, value, weightq, weightk)), "bf16 K/V, caches, weights")
    _check(key.is_contiguous() and value.is_contiguous() and key.shape == value.shape and key.dim() == 4 and
           key.size(1) == streams * Hk and key.size(3) == 256, "K/V cache: bf16 [1, streams * Hk, cap, 256]")
    _check(freqs.dtype == torch.float32 and freqs.is_contiguous() and freqs.numel() == S * (rd // 2) * 4,
           "frequencies: fp32 [S, rd/2, 2, 2]")
    _check(position.dtype == torch.int64 and position.is_contiguous() and position.numel() >= S, "int64 positions")
    _check(weightq.is_contiguous() and weightk.is_contiguous(), "contiguous norm weights")
    q = torch.empty((1, streams * Hq, R, 256), dtype=torch.bfloat16, device=rawq.device)
    k = torch.empty((1, streams * Hk, R, 256), dtype=torch.bfloat16, device=rawq.device)
    with torch.cuda.device(rawq.device):
        if streams == 1:
            _lib.call("mono_qk_norm_rope_kv", _p(rawq), rawq.stride(1), rawq.stride(2), _p(rawk), rawk.stride(1),
                      _p(vn), vn.stride(1), _p(weightq), _p(weightk), _p(freqs), _p(key), _p(value), key.size(2),
                      _p(position), S, Hq, Hk, float(epsq), float(epsk), int(rd), _p(q), _p(k), _stream(rawq.device))
        else:
            _lib.call("mono_qk_norm_rope_kv_streams", _p(rawq), rawq.stride(1), rawq.stride(2), _p(rawk),
                      rawk.stride(1), _p(vn), vn.stride(1), _p(weightq), _p(weightk), _p(freqs), _p(key), _p(value),
                      key.size(2), _p(position), S, streams, Hq, Hk, float(epsq), float(epsk), int(rd), _p(q), _p(k),
                      _stream(rawq.device))
    return q, k


_attn_ws = {}


def attn_dpas(q, key, value, seqlen, xk, xv, mask, chunks_hint=0, out=None, streams=1):
    """Tree decode attention (the reference's _C.attn_dpas, csrc/attn_dpas.sycl:269-342). q bf16 [1, H, S, 256];
    key / value bf16 [1, Hk, cap, 256]; seqlen int32 [1] on the device (L, no host sync); xk / xv bf16
    [1, Hk, S, 256]; mask int32 [S] (an empty tensor: the single draft row over the prefix only).
    Returns bf16 [1, S, H * 256] (into `out` when given). chunks_hint is accepted for the reference's signature and
    unused. xv may be any strided view with unit last stride (e.g. the projection's value columns transposed): the
    kernel reads it in place. streams > 1 (batched decode streams, include/mono_b200.h mono_tree_attention_streams):
    q, the caches and xk hold `streams` groups of heads (stream b: q heads [b H, (b + 1) H), kv heads
    [b Hk, (b + 1) Hk)), xv is [streams, Hk, S, 256] (any strides, unit last), seqlen int32 [streams], one mask for
    all; returns bf16 [1, streams * S, H * 256] (stream b's rows [b S, ...))."""
    _cuda(q, key, value, seqlen, xk, xv)
    _check(q.dtype == torch.bfloat16 and q.dim() == 4 and q.size(0) == 1 and q.size(3) == 256, "q bf16 [1, H, S, 256]")
    _check(streams >= 1 and q.size(1) % streams == 0 and key.size(1) % streams == 0, "heads in equal groups per stream")
    H, S, Hk, cap = q.size(1) // streams, q.size(2), key.size(1) // streams, key.size(2)
    _check(seqlen.numel() >= streams, "one length per stream")
    _check(key.is_contiguous() and value.is_contiguous() and key.shape == value.shape and key.size(3) == 256,
           "cache bf16 [1, Hk, cap, 256]")
    _check(seqlen.dtype == torch.int32 and mask.dtype == torch.int32, "int32 seqlen / mask")
    tree = mask.numel() > 0
    _check(mask.numel() == S if tree else S == 1, "mask [S] (or empty with one row)")
    q = q.contiguous()
    xk = xk.contiguous()
    if xv.dim() == 4 and xv.size(0) == 1 and xv.size(1) == streams * Hk and streams > 1:
        xv = xv.view(streams, Hk, xv.size(2), xv.size(3)) if xv.is_contiguous() else xv.contiguous().view(
            streams, Hk, xv.size(2), xv.size(3))
    _check(xv.dim() == 4 and tuple(xv.shape[1:]) == (Hk, S, 256) and xv.size(0) in (1, streams) and xv.stride(3) == 1,
           "xv bf16 [streams or 1, Hk, S, 256] with unit last stride")
    if xv.stride(1) % 8 or xv.stride(2) % 8 or (streams > 1 and xv.stride(0) % 8) or xv.data_ptr() % 16:
        xv = xv.contiguous()
    xv_strides = (xv.stride(0) if streams > 1 else 0, xv.stride(1), xv.stride(2))
    nbytes = _lib.load().mono_tree_attention_streams_workspace(Hk, streams, cap)
    ws = _workspace(_attn_ws, (q.device, Hk, streams, cap), nbytes, q.device)
    if out is None:
        out = torch.empty((1, streams * S, H * 256), dtype=torch.bfloat16, device=q.device)
    _check(out.dtype == torch.bfloat16 and out.is_contiguous() and out.numel() == streams * S * H * 256,
           "out bf16 [1, streams * S, H * 256]")
    with torch.cuda.device(q.device):
        _lib.call("mono_tree_attention_streams", _p(q), _p(key), _p(value), _p(seqlen), _p(xk), _p(xv),
                  _p(mask) if tree else None, H, Hk, S, streams, cap, *xv_strides, _p(out), _p(ws), nbytes,
                  _stream(q.device))
    return out


_gdn_ws = {}


def gdn_step(qkv, z, a, b, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, gnorm_eps, qscale, hk):
    """Gated-DeltaNet decode step for M sequential rows (include/mono_b200.h mono_gdn_step). Updates conv_state
    and state in place; returns core bf16 [M, HV * 128]."""
    _cuda(qkv, z, a, b, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w)
    M, C = qkv.shape
    HV = a.shape[1]
    _check(C == (2 * hk + HV) * 128 and z.shape == (M, HV * 128) and b.shape == a.shape, "GDN shapes")
    for t in (qkv, z, a, b, conv_w, conv_state, gnorm_w):
        _check(t.dtype == torch.bfloat16 and t.is_contiguous(), "bf16 contiguous operands")
    _check(state.dtype == torch.float32 and state.is_contiguous() and state.shape == (HV, 128, 128), "fp32 state")
    _check(dt_bias.dtype == torch.float32 and g_decay.dtype == torch.float32, "fp32 dt_bias / g_decay")
    nbytes = _lib.load().mono_gdn_step_workspace(M, C, HV)
    ws = _workspace(_gdn_ws, (qkv.device, M, C, HV), nbytes, qkv.device)
    core = torch.empty((M, HV * 128), dtype=torch.bfloat16, device=qkv.device)
    with torch.cuda.device(qkv.device):
        _lib.call("mono_gdn_step", _p(qkv), _p(z), _p(a), _p(b), _p(conv_w), _p(conv_state), _p(dt_bias), _p(g_decay),
                  _p(state), _p(gnorm_w), float(gnorm_eps), float(qscale), M, hk, HV, _p(core), _p(ws), nbytes,
                  _stream(qkv.device))
    return core


def mtp_prep_draft(st, k, ftab, freqs, mpos, mseq):
    """The reference's _C.mtp_prep_draft (csrc/mtp_loop.sycl:29-55): rope row, MTP KV positions / seqlen of
    draft k from the device counters st."""
    _cuda(st, ftab, freqs, mpos, mseq)
    _check(st.dtype == torch.int64 and mpos.dtype == torch.int64 and mseq.dtype == torch.int32, "int64 st / mpos, int32 mseq")
    _check(ftab.dtype == torch.float32 and ftab.is_contiguous() and freqs.is_contiguous() and freqs.dim() == ftab.dim()
           and freqs.size(2) == 1, "rope table [.., .., cap, ...] / row [.., .., 1, ...] float")
    n, cap = freqs.numel(), ftab.size(2)
    _check(ftab.numel() == cap * n, "rope table row size")
    with torch.cuda.device(st.device):
        _lib.call("mono_mtp_prep_draft", _p(st), int(k), _p(ftab), n, cap, _p(freqs), _p(mpos), mpos.numel(), _p(mseq),
                  _stream(st.device))


def mtp_prep_draft_streams(st, k, ftab, freqs, mpos, mseq):
    """mtp_prep_draft for B batched streams in one launch (mono_mtp_prep_draft_streams): st int64 [B, W], freqs
    float [B, ...] (row b: stream b's rope row), mpos int64 [B, np], mseq int32 [B]."""
    _cuda(st, ftab, freqs, mpos, mseq)
    _check(st.dtype == torch.int64 and mpos.dtype == torch.int64 and mseq.dtype == torch.int32, "int64 st / mpos, int32 mseq")
    B = st.size(0)
    _check(st.dim() == 2 and st.stride(1) == 1 and freqs.size(0) == B and freqs.is_contiguous() and
           mpos.dim() == 2 and mpos.size(0) == B and mpos.stride(1) == 1 and mseq.numel() == B and mseq.dim() == 1,
           "per-stream rows [B, ...]")
    _check(ftab.dtype == torch.float32 and ftab.is_contiguous() and freqs.dtype == torch.float32, "float rope rows")
    n = freqs[0].numel()
    cap = ftab.numel() // n
    _check(cap * n == ftab.numel(), "rope table rows of the row size")
    with torch.cuda.device(st.device):
        _lib.call("mono_mtp_prep_draft_streams", _p(st), st.stride(0), int(k), _p(ftab), n, cap, _p(freqs), n,
                  _p(mpos), mpos.stride(0), mpos.size(1), _p(mseq), mseq.stride(0), B, _stream(st.device))


def mtp_prep_verify(st, apos, aseq, vpos, tree_pos, ctl, tree_ctl, parity, rope_offset):
    """The reference's _C.mtp_prep_verify (csrc/mtp_loop.sycl:57-90)."""
    _cuda(st, apos, aseq, vpos, tree_pos, ctl, tree_ctl)
    _check(ctl.dtype == torch.int32 and ctl.numel() == 26 and tree_ctl.dtype == torch.int32 and tree_ctl.numel() == 16,
           "ctl / tree program")
    _check(tree_pos.numel() == vpos.numel(), "rows")
    with torch.cuda.device(st.device):
        _lib.call("mono_mtp_prep_verify", _p(st), _p(apos), apos.numel(), _p(aseq), _p(vpos), _p(tree_pos), vpos.numel(),
                  _p(ctl), _p(tree_ctl), int(parity), int(rope_offset), _stream(st.device))


def mtp_prep_verify_streams(st, apos, aseq, vpos, tree_pos, ctl, tree_ctl, parity, rope_offset):
    """mtp_prep_verify for B batched streams in one launch (mono_mtp_prep_verify_streams): st int64 [B, W], apos
    int64 [B, np], aseq int32 [B], vpos int64 [B, rows], ctl int32 [B, 26]; tree_pos / tree_ctl shared."""
    _cuda(st, apos, aseq, vpos, tree_pos, ctl, tree_ctl)
    B = st.size(0)
    _check(st.dtype == torch.int64 and st.dim() == 2 and st.stride(1) == 1, "st int64 [B, W]")
    _check(apos.dim() == 2 and apos.size(0) == B and apos.stride(1) == 1 and aseq.dim() == 1 and aseq.numel() == B and
           vpos.dim() == 2 and vpos.size(0) == B and vpos.stride(1) == 1 and ctl.dim() == 2 and ctl.size(0) == B and
           ctl.size(1) == 26 and ctl.stride(1) == 1, "per-stream rows [B, ...]")
    _check(ctl.dtype == torch.int32 and tree_ctl.dtype == torch.int32 and tree_ctl.numel() == 16, "ctl / tree program")
    _check(tree_pos.numel() == vpos.size(1), "rows")
    with torch.cuda.device(st.device):
        _lib.call("mono_mtp_prep_verify_streams", _p(st), st.stride(0), _p(apos), apos.stride(0), apos.size(1),
                  _p(aseq), aseq.stride(0), _p(vpos), vpos.stride(0), _p(tree_pos), vpos.size(1), _p(ctl),
                  ctl.stride(0), _p(tree_ctl), int(parity), int(rope_offset), B, _stream(st.device))


def mtp_accept(st, toks, vtok, cand, children, rows, depth, x, nt_buf, h_buf, ctl, kv_ptrs, kv_heads, kv_cap, head_dim,
               result):
    """The reference's _C.mtp_accept (csrc/mtp_loop.sycl:92-196): accept walk, result row, counters, ctl, next
    token / hidden row and the off-chain KV slot moves, all on the device."""
    _cuda(st, toks, vtok, children, x, nt_buf, h_buf, ctl, kv_ptrs, result)
    _check(st.dtype == torch.int64 and toks.dtype == torch.int64 and vtok.dtype == torch.int64, "int64 tokens / st")
    _check(children.dtype == torch.int32 and children.numel() == 64, "children [8][8]")
    _check(x.dtype == torch.bfloat16 and h_buf.dtype == torch.bfloat16 and x.numel() >= rows * h_buf.numel(), "hidden rows")
    _check(result.numel() >= 32 and result.dtype == torch.int64, "result slot")
    has_cand = cand is not None and cand.numel() > 0
    with torch.cuda.device(st.device):
        _lib.call("mono_mtp_accept", _p(st), _p(toks), _p(vtok), _p(cand) if has_cand else None, _p(children), int(rows),
                  int(depth), _p(x), h_buf.numel(), _p(nt_buf), _p(h_buf), _p(ctl), _p(kv_ptrs), kv_ptrs.numel(),
                  int(kv_heads), int(kv_cap), int(head_dim), _p(result), _stream(st.device))


_topk_ws = {}


def _topk(x, k, argmax_order, with_argmax):
    _cuda(x)
    _check(x.dtype == torch.bfloat16 and x.is_contiguous(), "bf16 contiguous")
    V = x.size(-1)
    rows = x.numel() // V
    values = torch.empty((*x.shape[:-1], k) if x.dim() > 1 else (k,), dtype=torch.bfloat16, device=x.device)
    indices = torch.empty(values.shape, dtype=torch.int64, device=x.device)
    am = torch.empty((rows,) if with_argmax else (0,), dtype=torch.int64, device=x.device)
    nbytes = _lib.load().mono_topk_workspace(rows)
    ws = _workspace(_topk_ws, (x.device, rows), nbytes, x.device)
    with torch.cuda.device(x.device):
        _lib.call("mono_fast_topk", _p(x), rows, V, int(k), int(argmax_order), int(with_argmax), _p(values), _p(indices),
                  _p(am) if with_argmax else None, _p(ws), nbytes, _stream(x.device))
    return values, indices, am


def fast_topk(x, k, argmax_order):
    """The reference's _C.fast_topk (csrc/fast_topk.sycl:164-167) for every row of x: (values, indices)."""
    v, i, _ = _topk(x, k, argmax_order, False)
    return v, i


def fast_pick(x, k):
    """The reference's _C.fast_pick (:169-171): top-k (top-k order) and the argmax of the same rows in one pass."""
    return _topk(x, k, False, True)


ROWLIN_NORM, ROWLIN_GATE, ROWLIN_QUANT = 0, 1, 2
_rowlin_ws = {}


def rowlin_gptq(x, mode, weights, norm_w=None, eps=1e-6, gate=None, gate_head_stride=512, lut=None, residual=None,
                out=None, xn_out=None, ab=None):
    """Row preparation (RMSNorm / sigmoid gate / plain) + per-token quant + GPTQ W4A8 linear of up to three TILED
    matrices in one launch (include/mono_b200.h mono_rowlin_gptq). weights: list of (tiled uint8 tensor, rows).
    gate: bf16 [M, ...] whose row m holds the gate of column c at (c / 256) * gate_head_stride + c % 256.
    ab = (w bf16 [N, K], out bf16 [M, N] with unit column stride): NORM mode with xn_out only; the same launch
    also writes the GDN a | b projection of the normalized rows, gdn_ab(xn_out, w) bit for bit
    (mono_rowlin_norm_ab_gptq). Returns out bf16 [M, sum rows]."""
    import ctypes
    _cuda(x)
    _check(x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous(), "x bf16 [M, K] contiguous")
    M, K = x.shape
    N = sum(int(r) for _, r in weights)
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    _check(out.is_contiguous() and out.numel() == M * N, "out [M, N]")
    if residual is not None:
        _check(residual.dtype == torch.bfloat16 and residual.is_contiguous() and residual.numel() == M * N, "residual")
    for w, r in weights:
        _check(w.is_cuda and w.dtype == torch.uint8 and w.numel() == _lib.load().mono_w4_tiled_bytes(0, int(r), K),
               "tiled GPTQ weights")
    ptrs = (ctypes.c_void_p * len(weights))(*[w.data_ptr() for w, _ in weights])
    rows = (ctypes.c_int64 * len(weights))(*[int(r) for _, r in weights])
    nbytes = _lib.load().mono_rowlin_gptq_workspace(K)
    ws = _workspace(_rowlin_ws, (x.device, K), nbytes, x.device)
    gate_row_stride = gate.stride(0) if gate is not None else 0
    if ab is not None:
        wab, ab_out = ab
        _check(mode == ROWLIN_NORM and xn_out is not None and norm_w is not None and residual is None,
               "a|b projection: norm mode with xn_out, no residual")
        _check(xn_out.dtype == torch.bfloat16 and xn_out.is_contiguous() and xn_out.shape == x.shape, "xn_out [M, K]")
        _check(wab.dtype == torch.bfloat16 and wab.is_contiguous() and wab.dim() == 2 and wab.shape[1] == K,
               "a|b weights bf16 [N, K]")
        _check(ab_out.dtype == torch.bfloat16 and ab_out.dim() == 2 and ab_out.shape == (M, wab.shape[0]) and
               ab_out.stride(1) == 1, "a|b out bf16 [M, N]")
        _cuda(wab, ab_out)
        with torch.cuda.device(x.device):
            _lib.call("mono_rowlin_norm_ab_gptq", _p(x), _p(norm_w), float(eps), ctypes.cast(ptrs, ctypes.c_void_p),
                      ctypes.cast(rows, ctypes.c_void_p), len(weights), M, K, _p(out), _p(xn_out), _p(wab),
                      int(wab.shape[0]), _p(ab_out), ab_out.stride(0), _p(ws), nbytes, _stream(x.device))
        return out
    with torch.cuda.device(x.device):
        _lib.call("mono_rowlin_gptq", _p(x), int(mode), _p(norm_w), float(eps), _p(gate), gate_row_stride,
                  int(gate_head_stride), _p(lut), ctypes.cast(ptrs, ctypes.c_void_p), ctypes.cast(rows, ctypes.c_void_p),
                  len(weights), M, K, _p(residual), _p(out), _p(xn_out), _p(ws), nbytes, _stream(x.device))
    return out


def gdn_step_deferred(qkv, z, a, b, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, gnorm_eps, qscale, hk, ctl,
                      prev, save, streams=1):
    """The deferred GDN step of the device MTP loop (include/mono_b200.h mono_gdn_step_deferred): replays the
    ctl[0] accepted rows of the previous step from prev = (qkv [8, C], a [8, HV], b [8, HV]), persists, then runs
    this step's rows as a chain without persisting and saves their inputs to save (same shapes, not aliasing
    prev). Returns core bf16 [M, HV * 128].
    streams > 1 (batched decode streams, mono_gdn_step_deferred_streams): the rows are `streams` groups of
    M / streams; conv_state [streams, C, 3], state [streams, HV, 128, 128], ctl int32 [streams, 26], prev / save
    [streams, 8, ...]: each stream's slice is its one-stream call's."""
    _cuda(qkv, z, a, b, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, ctl, *prev, *save)
    MT, C = qkv.shape
    HV = a.shape[1]
    _check(streams >= 1 and MT % streams == 0, "rows in equal groups per stream")
    if streams == 1 and prev[0].dim() == 3:  # one stream's slice of the batched layout
        prev, save = tuple(t[0] for t in prev), tuple(t[0] for t in save)
    M = MT // streams
    _check(C == (2 * hk + HV) * 128 and z.shape == (MT, HV * 128) and b.shape == a.shape, "GDN shapes")
    _check(ctl.dtype == torch.int32 and ctl.is_contiguous() and ctl.numel() >= 26 * streams - 16, "ctl int32 [26]")
    if streams > 1:
        _check(ctl.dim() == 2 and ctl.size(0) == streams and conv_state.shape == (streams, C, 3) and
               state.shape == (streams, HV, 128, 128) and prev[0].shape == (streams, 8, C) and
               prev[1].shape == (streams, 8, HV) and save[0].shape == (streams, 8, C), "per-stream state shapes")
    else:
        _check(prev[0].shape == (8, C) and prev[1].shape == (8, HV) and save[0].shape == (8, C), "saved rows [8, ...]")
    for t in (qkv, z, a, b):  # column slices of wider rows are fine
        _check(t.dtype == torch.bfloat16 and t.stride(1) == 1, "bf16 rows with unit column stride")
    _check(a.stride(0) == b.stride(0), "a and b share a row stride")
    for t in (conv_w, conv_state, gnorm_w, *prev, *save):
        _check(t.dtype == torch.bfloat16 and t.is_contiguous(), "bf16 contiguous operands")
    nbytes = _lib.load().mono_gdn_step_streams_workspace(M, C, HV, streams)
    ws = _workspace(_gdn_ws, (qkv.device, M, C, HV, streams), nbytes, qkv.device)
    core = torch.empty((MT, HV * 128), dtype=torch.bfloat16, device=qkv.device)
    with torch.cuda.device(qkv.device):
        if streams == 1:
            _lib.call("mono_gdn_step_deferred", _p(qkv), _p(z), _p(a), _p(b), _p(conv_w), _p(conv_state), _p(dt_bias),
                      _p(g_decay), _p(state), _p(gnorm_w), float(gnorm_eps), float(qscale), M, hk, HV, _p(core),
                      _p(ctl), _p(prev[0]), _p(prev[1]), _p(prev[2]), _p(save[0]), _p(save[1]), _p(save[2]),
                      qkv.stride(0), z.stride(0), a.stride(0), _p(ws), nbytes, _stream(qkv.device))
        else:
            _lib.call("mono_gdn_step_deferred_streams", _p(qkv), _p(z), _p(a), _p(b), _p(conv_w), _p(conv_state),
                      _p(dt_bias), _p(g_decay), _p(state), _p(gnorm_w), float(gnorm_eps), float(qscale), M, hk, HV,
                      streams, _p(core), _p(ctl), ctl.stride(0), _p(prev[0]), _p(prev[1]), _p(prev[2]), _p(save[0]),
                      _p(save[1]), _p(save[2]), qkv.stride(0), z.stride(0), a.stride(0), _p(ws), nbytes,
                      _stream(qkv.device))
    return core


def rmsnorm_add(x, w, eps, add=None, out=None, sum_out=None):
    """out = RMSNorm(x (+ add, rounded to bf16 and written to sum_out)) for bf16 rows [M, H] (column slices of
    wider rows are fine). Returns out (and sum_out when add is given)."""
    _cuda(x, w)
    M, H = x.shape
    if out is None:
        out = torch.empty((M, H), dtype=torch.bfloat16, device=x.device)
    if add is not None and sum_out is None:
        sum_out = torch.empty_like(out)
    _check(out.stride(0) == (sum_out.stride(0) if sum_out is not None else out.stride(0)), "out / sum_out strides")
    with torch.cuda.device(x.device):
        _lib.call("mono_rmsnorm_add", _p(x), x.stride(0), _p(add), add.stride(0) if add is not None else 0, _p(w),
                  float(eps), M, H, _p(out), _p(sum_out), out.stride(0), _stream(x.device))
    return (out, sum_out) if add is not None else out


def draft_embed_norm_cat(embed, tokens, index, enorm_w, hidden, hnorm_w, eps, out=None):
    """The MTP draft head's front (include/mono_b200.h mono_draft_embed_norm_cat): for each row b of hidden
    [B, H], cat(RMSNorm(embed[tokens[b, index]]; enorm_w), RMSNorm(hidden[b]; hnorm_w)) -> bf16 [B, 2 H].
    tokens: int64 [B, n] (or [n] for B = 1) on the device."""
    _cuda(embed, tokens, enorm_w, hidden, hnorm_w)
    B, H = hidden.shape
    V = embed.shape[0]
    _check(embed.dtype == torch.bfloat16 and embed.is_contiguous() and embed.shape[1] == H, "embed bf16 [V, H]")
    _check(tokens.dtype == torch.int64 and tokens.stride(-1) == 1, "int64 token ids")
    tok2 = tokens.view(1, -1) if tokens.dim() == 1 else tokens
    _check(tok2.shape[0] == B and 0 <= index < tok2.shape[1], "tokens [B, n], index < n")
    _check(hidden.dtype == torch.bfloat16 and hidden.stride(1) == 1, "hidden bf16 rows")
    if out is None:
        out = torch.empty((B, 2 * H), dtype=torch.bfloat16, device=hidden.device)
    _check(out.dtype == torch.bfloat16 and out.shape == (B, 2 * H) and out.stride(1) == 1, "out bf16 [B, 2 H]")
    with torch.cuda.device(hidden.device):
        _lib.call("mono_draft_embed_norm_cat", _p(embed), V, H, _p(tok2), tok2.stride(0), int(index), _p(enorm_w),
                  _p(hidden), hidden.stride(0), _p(hnorm_w), float(eps), B, _p(out), out.stride(0),
                  _stream(hidden.device))
    return out


def lut_mul(a, b, lut, b_head_stride=256, out=None):
    """bf16(a * lut[b]) elementwise over rows [M, K]; b's column c at (c / 256) * b_head_stride + c % 256."""
    _cuda(a, b, lut)
    M, K = a.shape
    if out is None:
        out = torch.empty((M, K), dtype=torch.bfloat16, device=a.device)
    with torch.cuda.device(a.device):
        _lib.call("mono_lut_mul", _p(a), a.stride(0), _p(b), b.stride(0), int(b_head_stride), _p(lut), M, K, _p(out),
                  out.stride(0), _stream(a.device))
    return out


# ---- layer programs (include/mono_b200.h mono_program_*) ----------------------------------------------------------

ROWS_NORM, ROWS_GATE, ROWS_QUANT, ROWS_GDN = 0, 1, 2, 3


class Program:
    """A layer program: ops appended in order, planned for M rows, copied to the device once, then launched as
    one persistent cooperative kernel per call (graph-capturable). Every tensor an op names is kept alive by
    the program; the ops hold raw pointers, so those tensors must not be reallocated afterwards."""

    def __init__(self, device, capacity=512):
        import numpy as np
        lib = _lib.load()
        self.device = torch.device(device)
        self.opb = int(lib.mono_program_op_bytes())
        self.host = np.zeros(capacity * self.opb, dtype=np.uint8)
        self.n = 0
        self.keep = []
        self.dev_ops = None
        self.M = None
        self.ws = torch.zeros(int(lib.mono_program_workspace()), dtype=torch.uint8, device=self.device)

    def _ptr(self):
        return self.host.ctypes.data

    def _next(self):
        _check(self.dev_ops is None, "program already planned")
        _check(self.n * self.opb < self.host.size, "program capacity")
        i = self.n
        self.n += 1
        return i

    def _hold(self, *ts):
        self.keep.extend(t for t in ts if t is not None)

    def rows(self, mode, x, K, q, s, norm_w=None, eps=1e-6, gate=None, gate_row_stride=0, gate_head_stride=0, lut=None,
             xn_out=None, zero=None, barrier=True, x_stride=None):
        self._hold(x, q, s, norm_w, gate, lut, xn_out, zero)
        _lib.call("mono_program_rows", self._ptr(), self._next(), int(mode), _p(x), int(x_stride or K), int(K), _p(norm_w),
                  float(eps), _p(gate), int(gate_row_stride), int(gate_head_stride), _p(lut), _p(xn_out), _p(q), _p(s),
                  _p(zero), int(bool(barrier)))

    def gemv(self, weights, K, q, s, out, out_stride, residual=None, residual_stride=0, paired=False, silu_lut=None,
             amax=None, barrier=True):
        import ctypes
        self._hold(q, s, out, residual, silu_lut, amax, *[w for w, _ in weights])
        ptrs = (ctypes.c_void_p * len(weights))(*[w.data_ptr() for w, _ in weights])
        rows = (ctypes.c_int64 * len(weights))(*[int(r) for _, r in weights])
        _lib.call("mono_program_gemv", self._ptr(), self._next(), ctypes.cast(ptrs, ctypes.c_void_p),
                  ctypes.cast(rows, ctypes.c_void_p), len(weights), int(bool(paired)), int(K), _p(q), _p(s), _p(out),
                  int(out_stride), _p(residual), int(residual_stride), _p(silu_lut), _p(amax), int(bool(barrier)))

    def quant(self, h, K, amax, q, s, barrier=True):
        self._hold(h, amax, q, s)
        _lib.call("mono_program_quant", self._ptr(), self._next(), _p(h), int(K), _p(amax), _p(q), _p(s),
                  int(bool(barrier)))

    def ab(self, x, x_stride, K, w, out, barrier=False):
        self._hold(x, w, out)
        _lib.call("mono_program_ab", self._ptr(), self._next(), _p(x), int(x_stride), int(K), _p(w), int(w.shape[0]),
                  _p(out), int(bool(barrier)))

    def gdn(self, delta, qkv, z, a, b, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, gnorm_eps, qscale, M, hk,
            hv, raw, ctl, prev, save, qkv_stride, z_stride, ab_stride, workspace, barrier=True):
        prev = prev if prev is not None else (None, None, None)
        save = save if save is not None else (None, None, None)
        self._hold(qkv, z, a, b, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, raw, ctl, workspace, *prev, *save)
        _lib.call("mono_program_gdn", self._ptr(), self._next(), int(bool(delta)), _p(qkv), _p(z), _p(a), _p(b),
                  _p(conv_w), _p(conv_state), _p(dt_bias), _p(g_decay), _p(state), _p(gnorm_w), float(gnorm_eps),
                  float(qscale), int(M), int(hk), int(hv), _p(raw), _p(ctl), _p(prev[0]), _p(prev[1]), _p(prev[2]),
                  _p(save[0]), _p(save[1]), _p(save[2]), int(qkv_stride), int(z_stride), int(ab_stride),
                  _p(workspace), workspace.numel() * workspace.element_size(), int(bool(barrier)))

    def plan(self, M):
        """Checks and plans the ops for M rows and copies them to the device."""
        _lib.call("mono_program_plan", self._ptr(), self.n, int(M))
        self.M = int(M)
        self.dev_ops = torch.from_numpy(self.host[: self.n * self.opb].copy()).to(self.device)
        return self

    def launch(self, prefetch=0):
        _check(self.dev_ops is not None, "program not planned")
        with torch.cuda.device(self.device):
            _lib.call("mono_program_launch", self._ptr(), _p(self.dev_ops), self.n, self.M, _p(self.ws), int(prefetch),
                      _stream(self.device))


def gdn_ab(x, w, out=None):
    """The GDN gates' a | b projection (include/mono_b200.h mono_gdn_ab): x bf16 [M, K] (unit column stride),
    w bf16 [N, K] -> bf16 [M, N]."""
    _cuda(x, w)
    _check(x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1, "x bf16 [M, K] rows")
    _check(w.dtype == torch.bfloat16 and w.is_contiguous() and w.shape[1] == x.shape[1], "w bf16 [N, K]")
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    _check(out.is_contiguous() and out.numel() == M * N, "out [M, N]")
    with torch.cuda.device(x.device):
        _lib.call("mono_gdn_ab", _p(x), x.stride(0), _p(w), K, M, N, _p(out), _stream(x.device))
    return out


_post_ws = {}
_gdn_layer_ws = {}


def layer_post(x, y, o_w, norm_w, eps, gate_w, up_w, down_w, silu_lut, I, gate=None, sig_lut=None,
               gate_head_stride=512, out=None):
    """The reference's layer_post in one launch (include/mono_b200.h mono_layer_post_gptq): sigmoid gate (if
    gate is given) -> quant -> o projection + residual x -> RMSNorm -> MLP + residual. x, y bf16 [M, H] / [M, K]
    contiguous; weights TILED GPTQ. Returns out bf16 [M, H] (may be x)."""
    _cuda(x, y)
    _check(x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous(), "x bf16 [M, H] contiguous")
    _check(y.dtype == torch.bfloat16 and y.dim() == 2 and y.is_contiguous() and y.shape[0] == x.shape[0], "y bf16 [M, K]")
    M, H = x.shape
    K = y.shape[1]
    if out is None:
        out = torch.empty_like(x)
    nbytes = _lib.load().mono_layer_post_gptq_workspace(K, H, I)
    ws = _workspace(_post_ws, (x.device, K, H, I), nbytes, x.device)
    with torch.cuda.device(x.device):
        _lib.call("mono_layer_post_gptq", _p(x), _p(y), K, _p(gate), gate.stride(0) if gate is not None else 0,
                  int(gate_head_stride), _p(sig_lut), _p(o_w), _p(norm_w), float(eps), _p(gate_w), _p(up_w), _p(down_w),
                  _p(silu_lut), M, H, int(I), _p(out), _p(ws), nbytes, _stream(x.device))
    return out


def layer_gdn(x, norm_in, eps_in, qkv_w, z_w, wab, conv_w, conv_state, dt_bias, g_decay, state, gnorm_w, gnorm_eps,
              qscale, hk, ctl, prev, save, out_w, norm_post, eps_post, gate_w, up_w, down_w, silu_lut, I, out=None):
    """The reference's layer_gdn in one launch (include/mono_b200.h mono_layer_gdn_gptq): the whole Gated-DeltaNet
    decoder layer for x bf16 [M, H] (M <= 8); deferred GDN state handling as gdn_step_deferred (ctl None:
    committing). Returns out bf16 [M, H] (may be x)."""
    _cuda(x)
    _check(x.dtype == torch.bfloat16 and x.dim() == 2 and x.is_contiguous(), "x bf16 [M, H] contiguous")
    M, H = x.shape
    HV = dt_bias.numel()
    if out is None:
        out = torch.empty_like(x)
    prev = prev if prev is not None else (None, None, None)
    save = save if save is not None else (None, None, None)
    nbytes = _lib.load().mono_layer_gdn_gptq_workspace(M, H, I, hk, HV)
    ws = _workspace(_gdn_layer_ws, (x.device, M, H, I, hk, HV), nbytes, x.device)
    with torch.cuda.device(x.device):
        _lib.call("mono_layer_gdn_gptq", _p(x), _p(norm_in), float(eps_in), _p(qkv_w), _p(z_w), _p(wab), _p(conv_w),
                  _p(conv_state), _p(dt_bias), _p(g_decay), _p(state), _p(gnorm_w), float(gnorm_eps), float(qscale),
                  _p(ctl), _p(prev[0]), _p(prev[1]), _p(prev[2]), _p(save[0]), _p(save[1]), _p(save[2]), _p(out_w),
                  _p(norm_post), float(eps_post), _p(gate_w), _p(up_w), _p(down_w), _p(silu_lut), M, H, int(I), int(hk),
                  HV, _p(out), _p(ws), nbytes, _stream(x.device))
    return out


_lmhead_ws = {}


def lmhead_pick(x, w, k=0, logits=False, argmax_out=None, topk_out=None, children=None, dst=None, index_base=0):
    """bf16 lm_head of M <= 16 rows with the greedy / draft pick fused (include/mono_b200.h mono_lmhead_pick):
    x bf16 [M, K] (rows 16-byte aligned), w bf16 [V, K]. Returns (argmax int64 [M], top-k int64 [M, k] or None,
    logits bf16 [M, V] or None). With children (int32 device tensor of up to 8 slots, -1 ends) and dst (int64 device
    tensor: one row, or [M, >= 8] with unit column stride, one row per x row), also writes each row's draft pick
    into its dst row. index_base: the vocabulary index of w's row 0 (a tensor-parallel shard): ranks and returned
    indices are global."""
    _cuda(x, w)
    _check(x.dtype == torch.bfloat16 and w.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1 and
           w.is_contiguous() and w.dim() == 2 and w.size(1) == x.size(1), "x bf16 [M, K], w bf16 [V, K]")
    M, K = x.shape
    V = w.size(0)
    am = argmax_out if argmax_out is not None else torch.empty(M, dtype=torch.int64, device=x.device)
    tk = None
    if k > 0 and children is None:
        tk = topk_out if topk_out is not None else torch.empty(M, k, dtype=torch.int64, device=x.device)
    lg = torch.empty(M, V, dtype=torch.bfloat16, device=x.device) if logits else None
    dst_stride = 0
    if children is not None:
        _check(dst is not None and dst.dtype == torch.int64, "the pick form needs an int64 dst")
        if M > 1:
            _check(dst.dim() == 2 and dst.size(0) == M and dst.size(1) >= 8 and dst.stride(1) == 1,
                   "dst [M, >= 8] rows for M > 1")
            dst_stride = dst.stride(0)
    need = _lib.load().mono_lmhead_workspace()
    ws = _workspace(_lmhead_ws, (x.device,), need, x.device)
    with torch.cuda.device(x.device):
        _lib.call("mono_lmhead_pick", _p(x), x.stride(0), _p(w), M, V, K, k, int(index_base), _p(lg), _p(am), _p(tk),
                  _p(children), _p(dst), dst_stride, _p(ws), need, _stream(x.device))
    return am, tk, lg


def gemv_bf16(x, w, out=None):
    """bf16 GEMV of the draft head's projections (include/mono_b200.h mono_gemv_bf16): x bf16 [M, K] (M <= 8,
    unit column stride), w bf16 [N, K] contiguous -> bf16 [M, N] (out: any [M, N] view with unit column stride),
    fp32 accumulation; what F.linear(x, w) computes for a few rows."""
    _cuda(x, w)
    _check(x.dtype == torch.bfloat16 and x.dim() == 2 and x.stride(1) == 1, "x bf16 [M, K] rows")
    _check(w.dtype == torch.bfloat16 and w.dim() == 2 and w.is_contiguous() and w.shape[1] == x.shape[1],
           "w bf16 [N, K]")
    M, K = x.shape
    N = w.shape[0]
    if out is None:
        out = torch.empty((M, N), dtype=torch.bfloat16, device=x.device)
    _check(out.dtype == torch.bfloat16 and out.dim() == 2 and tuple(out.shape) == (M, N) and out.stride(1) == 1,
           "out bf16 [M, N] rows")
    with torch.cuda.device(x.device):
        _lib.call("mono_gemv_bf16", _p(x), x.stride(0), _p(w), M, N, K, _p(out), out.stride(0), _stream(x.device))
    return out


_topk_rows_ws = {}


def topk_rows(x, k, index_order=False):
    """Exact top-k (k <= 64) of a few long rows (the reference's _C.topk_rows, csrc/topk_rows.sycl): x fp32 or
    bf16 [R, N] (R <= 16) -> (values fp32 [R, k], indices int64 [R, k]) = torch.topk(x.float(), k); equal values in
    the torch-XPU order, or with index_order by ascending index, torch's CUDA order for k >= 33 and k = 1
    (include/mono_b200.h mono_topk_rows)."""
    _cuda(x)
    _check(x.dim() == 2 and x.is_contiguous() and x.dtype in (torch.float32, torch.bfloat16), "x fp32 / bf16 [R, N]")
    R, N = x.shape
    values = torch.empty((R, int(k)), dtype=torch.float32, device=x.device)
    indices = torch.empty((R, int(k)), dtype=torch.int64, device=x.device)
    nbytes = _lib.load().mono_topk_rows_workspace(R, N)
    ws = _workspace(_topk_rows_ws, (x.device, R, N), nbytes, x.device)
    flags = (_lib.TOPK_BF16 if x.dtype == torch.bfloat16 else 0) | (_lib.TOPK_INDEX_ORDER if index_order else 0)
    with torch.cuda.device(x.device):
        _lib.call("mono_topk_rows", _p(x), flags, R, N, int(k), _p(values), _p(indices), _p(ws), nbytes,
                  _stream(x.device))
    return values, indices


class PeerSum:
    """The two-GPU one-shot all-reduce of bf16 rows (include/mono_b200.h mono_allreduce2_bf16) between this rank and
    its peer: an area of this rank's memory (receive buffers + arrival counters) is mapped by the peer through CUDA
    IPC. `exchange(handle: bytes) -> [handle of rank 0, handle of rank 1]` passes the handles (e.g. through
    torch.distributed.all_gather_object); `peer` is the other rank's index. Calls sum in place; both ranks must make
    the same calls in the same order."""

    def __init__(self, device, cap, exchange, peer):
        import ctypes
        lib = _lib.load()
        self.device, self.cap = torch.device(device), int(cap)
        nbytes = lib.mono_allreduce2_area_bytes(self.cap)
        area = ctypes.c_void_p()
        with torch.cuda.device(self.device):
            _lib.call("mono_p2p_area_alloc", nbytes, ctypes.byref(area))
            self.area = area.value
            h = (ctypes.c_char * 64)()
            _lib.call("mono_ipc_handle", self.area, h, 64)
            handles = exchange(bytes(h))
            ph = (ctypes.c_char * 64).from_buffer_copy(handles[peer])
            pp = ctypes.c_void_p()
            _lib.call("mono_ipc_open", ph, 64, ctypes.byref(pp))
            self.peer = pp.value
        self.calls = torch.zeros(16, dtype=torch.int32, device=self.device)

    def __call__(self, t):
        _check(t.is_cuda and t.dtype == torch.bfloat16 and t.is_contiguous() and t.numel() <= self.cap,
               "bf16 contiguous rows within the area's capacity")
        with torch.cuda.device(t.device):
            _lib.call("mono_allreduce2_bf16", _p(t), _p(t), t.numel(), self.area, self.peer, self.cap, _p(self.calls),
                      _stream(t.device))
        return t

    def close(self):
        with torch.cuda.device(self.device):
            if self.peer:
                _lib.call("mono_ipc_close", self.peer)
                self.peer = None
            if self.area:
                _lib.call("mono_p2p_area_free", self.area)
                self.area = None
