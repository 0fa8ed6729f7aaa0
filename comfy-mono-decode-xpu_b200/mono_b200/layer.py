"""Decode-layer install points (the role of comfy_mono_decode_xpu/layer.py:396-617) over ComfyUI's Qwen3.5 text
encoder classes, routed to the B200 kernels.

  FixedKVCache.attend          tree verify rows / the MTP draft row -> mono_tree_attention (the tree mask from the
                               cache's tracker; reads the cache only, so any failure falls back to the original)
  GatedAttention.forward       stock projections, then Q/K RMSNorm + partial RoPE + KV write in one launch
                               (mono_qk_norm_rope_kv) and the attend above; gate and o_proj stock
  Qwen35TransformerBlock.forward
                               the whole layer on the fused kernels (rowlin / attention or GDN / MLP) when its
                               projections carry this build's tile-major GPTQ weights (``mono_b200_w4``); any
                               other block runs the original
  RMSNorm.scale                weight + 1 cached per weight (MONO_DECODE_XPU_NORM_CACHE)

Environment switches (the reference's names): MONO_DECODE_XPU_ATTN, MONO_DECODE_XPU_ATTN_DPAS, MONO_DECODE_XPU_ROPE,
MONO_DECODE_XPU_NORM_CACHE ("0" turns a piece off). Failure contract: a pure op falls back after guard.failed; a
path that has written state (KV, x) re-raises after switching itself off (SubpathError for a sub-route).
"""
from __future__ import annotations

import os
import threading

import torch

from . import guard

CLAIM = "__comfy_mono_decode_b200__"
_lock = threading.Lock()
_stats = {}
_attn = os.environ.get("MONO_DECODE_XPU_ATTN", "1") == "1" and os.environ.get("MONO_DECODE_XPU_ATTN_DPAS", "1") == "1"
_rope = os.environ.get("MONO_DECODE_XPU_ROPE", "1") == "1"


class SubpathError(RuntimeError):
    """A fused sub-route failed after writing state; it is switched off and the block is not replayed."""


class Ineligible(RuntimeError):
    """A fused route cannot serve this call; raised before anything was written (the caller runs the original)."""


def stats():
    with _lock:
        return dict(_stats)


def _count(k):
    with _lock:
        _stats[k] = _stats.get(k, 0) + 1


def _claimed(fn):
    return getattr(fn, CLAIM, False) or getattr(fn, "__comfy_mono_decode_xpu__", False)


def _install_attend(llama=None):
    if llama is None:
        from comfy.text_encoders import llama
    from . import _C
    cls = llama.FixedKVCache
    original = cls.attend
    if _claimed(original):
        return False
    empty = {}

    def attend(self, xq, xk, xv):
        tree = self.tracker.get("tree") if isinstance(getattr(self, "tracker", None), dict) else None
        S = xq.shape[2] if xq.dim() == 4 else 0
        if (_attn and not guard.off("attn") and xq.device.type == "cuda" and xq.dtype == torch.bfloat16
                and xq.shape[0] == 1 and xq.shape[-1] == 256 and self.key.dtype == torch.bfloat16
                and self.key.is_contiguous() and self.value.is_contiguous() and 1 <= S <= 8
                and self.seqlen.dtype == torch.int32 and (xq.shape[1] // self.key.shape[1]) * S <= 32):
            if tree is not None and tree.mask.numel() == S and tree.mask.dtype == torch.int32:
                mask = tree.mask
            elif tree is None and S == 1:
                mask = empty.setdefault(xq.device, torch.empty(0, dtype=torch.int32, device=xq.device))
            else:
                mask = None
            if mask is not None:
                try:
                    out = _C.attn_dpas(xq, self.key, self.value, self.seqlen, xk, xv, mask, 0)
                except Exception as e:  # reads the cache only: the original recomputes it
                    guard.failed("attn", e)
                    return original(self, xq, xk, xv)
                _count("attn")
                return out
        return original(self, xq, xk, xv)

    setattr(attend, CLAIM, True)
    attend.__wrapped__ = original
    cls.attend = attend
    return True


def attention_core(mix, qg, xk, xv, freqs_cis, kv):
    """The attention core of a GatedAttention decode call after its projections: Q/K RMSNorm + partial RoPE + K/V
    cache write in one launch (mono_qk_norm_rope_kv), then kv.attend (the attend route). qg [1, S, heads * 2 *
    head_dim] (query | gate per head), xk / xv [1, S, kv_heads * head_dim]. Returns the attention rows
    [1, S, heads * head_dim] (before the gate). Raises Ineligible before any write when the call is not one the
    kernels serve; a failure after the write switches the piece off and raises SubpathError."""
    from . import _C
    B, S = qg.shape[0], qg.shape[1]
    qgv = qg.view(B, S, mix.num_heads, mix.head_dim * 2)
    rawq = qgv[..., :mix.head_dim]
    rawk = xk.view(B, S, mix.num_kv_heads, mix.head_dim)
    xv4 = xv.view(B, S, mix.num_kv_heads, mix.head_dim)
    if (not _rope or guard.off("norm_rope") or torch.is_grad_enabled() or freqs_cis is None
            or getattr(kv, "position", None) is None or mix.rotary_dim % 2):
        raise Ineligible("norm_rope")
    try:
        f = freqs_cis.reshape(S, mix.rotary_dim // 2, 2, 2).float().contiguous()
        q, k = _C.qk_norm_rope_kv(rawq, rawk, xv4, mix.q_norm.weight, mix.k_norm.weight, f, kv.key, kv.value,
                                  kv.position[:S], mix.q_norm.eps, mix.k_norm.eps, mix.rotary_dim)
    except Exception as e:
        from . import _lib
        if _lib.rejected(e):  # the binding refused the operands before the launch: nothing was written
            raise Ineligible("norm_rope: " + e.reason) from e
        guard.failed("norm_rope", e, can_fallback=False)  # the KV cache may be written: no replay
        raise SubpathError("norm_rope") from e
    _count("norm_rope")
    return kv.attend(q, k, xv4.transpose(1, 2))


def _install_gated_attention(q35=None):
    if q35 is None:
        from comfy.text_encoders import qwen35 as q35
    cls = q35.GatedAttention
    original = cls.forward
    if _claimed(original):
        return False

    def forward(self, x, attention_mask=None, freqs_cis=None, optimized_attention=None, past_key_value=None):
        if (x.dim() != 3 or x.shape[0] != 1 or not 1 <= x.shape[1] <= 8 or past_key_value is None
                or attention_mask is not None or x.device.type != "cuda" or x.dtype != torch.bfloat16):
            return original(self, x, attention_mask, freqs_cis, optimized_attention, past_key_value)
        B, S = x.shape[0], x.shape[1]
        qg, xk, xv = self.q_proj(x), self.k_proj(x), self.v_proj(x)
        try:
            out = attention_core(self, qg, xk, xv, freqs_cis, past_key_value)
        except Ineligible:
            return original(self, x, attention_mask, freqs_cis, optimized_attention, past_key_value)
        gate = qg.view(B, S, self.num_heads, self.head_dim * 2)[..., self.head_dim:].reshape(B, S, -1)
        out = out * gate.sigmoid()
        return self.o_proj(out), past_key_value

    setattr(forward, CLAIM, True)
    forward.__wrapped__ = original
    cls.forward = forward
    return True


def _install_norm_scale(llama=None):
    """RMSNorm(add=True).scale() -> weight + 1 cached per weight (same bf16 values, no launch per call)."""
    if llama is None:
        from comfy.text_encoders import llama
    cls = llama.RMSNorm
    original = getattr(cls, "scale", None)
    if original is None or _claimed(original):
        return False
    cache = {}

    def scale(self):
        if torch.is_grad_enabled():
            return original(self)
        key = (id(self.weight), self.weight._version if hasattr(self.weight, "_version") else 0)
        hit = cache.get(id(self))
        if hit is None or hit[0] != key:
            hit = cache[id(self)] = (key, original(self))
        return hit[1]

    setattr(scale, CLAIM, True)
    scale.__wrapped__ = original
    cls.scale = scale
    return True


def _block_plan(block, x):
    """The block's decode plan: one attached as ``mono_b200_w4`` (a dict with "run"), else the generate session's
    (bridge.block_plan), else None (the original forward)."""
    w = getattr(block, "mono_b200_w4", None)
    if isinstance(w, dict):
        return w
    from . import bridge
    return bridge.block_plan(block, x.device) if x.device.type == "cuda" else None


def install(q35=None, llama=None):
    """Install every layer-level point; True if the block forward was wrapped now."""
    if q35 is None:
        from comfy.text_encoders import qwen35 as q35
    if llama is None:
        from comfy.text_encoders import llama
    _install_attend(llama)
    if _rope:
        _install_gated_attention(q35)
    if os.environ.get("MONO_DECODE_XPU_NORM_CACHE", "1") == "1":
        _install_norm_scale(llama)
    Block = q35.Qwen35TransformerBlock
    original = Block.forward
    if _claimed(original):
        return False

    def forward(self, x, attention_mask=None, freqs_cis=None, optimized_attention=None, past_key_value=None):
        S = x.shape[1] if x.dim() == 3 else 0
        if (guard.off("layer") or past_key_value is None or x.device.type != "cuda" or x.dtype != torch.bfloat16
                or x.shape[0] != 1 or not 1 <= S <= 8 or not x.is_contiguous() or attention_mask is not None):
            return original(self, x, attention_mask, freqs_cis, optimized_attention, past_key_value)
        plan = _block_plan(self, x)
        if plan is None:
            _count("fallback_weights")
            return original(self, x, attention_mask, freqs_cis, optimized_attention, past_key_value)
        state = {"mutated": False}
        try:
            out = plan["run"](self, x, attention_mask, freqs_cis, past_key_value, state)
        except Ineligible:  # nothing was written
            _count("fallback_call")
            return original(self, x, attention_mask, freqs_cis, optimized_attention, past_key_value)
        except SubpathError:
            raise
        except Exception as e:
            guard.failed("layer", e, can_fallback=not state["mutated"])
            if state["mutated"]:
                raise
            return original(self, x, attention_mask, freqs_cis, optimized_attention, past_key_value)
        _count("layer")
        return out

    setattr(forward, CLAIM, True)
    forward.__wrapped__ = original
    Block.forward = forward
    return True
