"""Device-side MTP decode loop install point (the role of comfy_mono_decode_xpu/mtp_loop.py:139-489):
``Qwen35._generate_mtp(self, embeds, max_length, stop_tokens, mtp, sampling=None, position_ids=None,
repetition_penalty=1.0, presence_penalty=0.0)``.

The loop's decisions (accept walk, counters, GDN replay ctl, next token / hidden row, KV slot moves) run on the
device (mono_mtp_accept / mono_mtp_prep_*), so the host queues step after step without reading anything back;
mono_b200.decoder.Qwen35W4A8.step is that step for models built on this build's kernels. A model exposing such a
decoder as ``self.mono_b200_decoder`` is routed to it for greedy generation (sampling None, no penalties); any
other call runs the original. Also the cache hooks of the reference (FixedKV.advance / FixedKVState.prepare /
LinearKV.prepare become no-ops for device-owned caches, marked ``_mono_device``).

Environment: MONO_DECODE_XPU_DEVICE_MTP ("0" off).
"""
from __future__ import annotations

import os

import torch

from . import guard

CLAIM = "__comfy_mono_decode_b200__"
MODE = os.environ.get("MONO_DECODE_XPU_DEVICE_MTP", "1")


def _install_device_kv(classes):
    """FixedKV.advance / FixedKVState.prepare / LinearKV.prepare -> no-ops on device-owned caches."""
    done = 0
    for cls, name in classes:
        original = cls.__dict__.get(name)
        if original is None or getattr(original, CLAIM, False):
            continue

        def make(original=original):
            def method(self, num_tokens):
                if getattr(self, "_mono_device", False):
                    return None
                return original(self, num_tokens)
            setattr(method, CLAIM, True)
            method.__wrapped__ = original
            return method
        setattr(cls, name, make())
        done += 1
    return done


def generate_device(decoder, max_new_tokens, stop_tokens=(), sync_every=8):
    """Greedy MTP generation on a mono_b200 decoder: steps are queued without host reads (replayed from CUDA graphs
    when the decoder offers step_graphed); each step's result row is copied to a device ring, and the committed
    tokens are read back once every `sync_every` steps (one device -> host copy of the ring) to check the stop
    condition (the reference reads each step one step late from a pinned ring, mtp_loop.py:413-441)."""
    out = []
    stop = set(int(t) for t in stop_tokens)
    step = getattr(decoder, "step_graphed", None) or decoder.step
    ring = None
    while len(out) < max_new_tokens:
        for i in range(sync_every):
            r = step()
            if ring is None:
                ring = torch.empty(sync_every, r.numel(), dtype=r.dtype, device=r.device)
            ring[i].copy_(r)
        for r in ring.cpu().tolist():
            n = r[0]
            for t in r[1:1 + n]:
                out.append(t)
                if t in stop or len(out) >= max_new_tokens:
                    return out
    return out


def generate_device_streams(decoder, max_new_tokens, sync_every=8):
    """generate_device for a batch of streams (mono_b200.streams.Qwen35W4A8Streams): each step's result rows [B, 32]
    go to a device ring read back every `sync_every` steps; runs until every stream has max_new_tokens. Returns the
    committed tokens of each stream."""
    step = getattr(decoder, "step_graphed", None) or decoder.step
    B = decoder.streams
    out = [[] for _ in range(B)]
    ring = None
    while min(len(o) for o in out) < max_new_tokens:
        for i in range(sync_every):
            r = step()
            if ring is None:
                ring = torch.empty((sync_every,) + tuple(r.shape), dtype=r.dtype, device=r.device)
            ring[i].copy_(r)
        for rows in ring.cpu().tolist():
            for b, r in enumerate(rows):
                if len(out[b]) < max_new_tokens:
                    out[b].extend(r[1:1 + r[0]][:max_new_tokens - len(out[b])])
    return out


def install(q35=None, llama=None):
    if MODE == "0":
        return False
    if q35 is None:
        from comfy.text_encoders import qwen35 as q35
    if llama is None:
        from comfy.text_encoders import llama
    cls = getattr(q35, "Qwen35", None)
    original = getattr(cls, "_generate_mtp", None)
    if original is None or getattr(original, CLAIM, False) or getattr(original, "__comfy_mono_decode_xpu__", False):
        return False
    kv_classes = [(getattr(llama, n), m) for n, m in (("FixedKV", "advance"), ("FixedKVState", "prepare"))
                  if hasattr(llama, n)]
    if hasattr(q35, "LinearKV"):
        kv_classes.append((q35.LinearKV, "prepare"))
    _install_device_kv(kv_classes)

    def _generate_mtp(self, embeds, max_length, stop_tokens, mtp, sampling=None, position_ids=None,
                      repetition_penalty=1.0, presence_penalty=0.0):
        dec = getattr(self, "mono_b200_decoder", None)
        if (dec is None or guard.off("mtp_loop") or sampling is not None or repetition_penalty != 1.0
                or presence_penalty != 0.0):
            return original(self, embeds, max_length, stop_tokens, mtp, sampling, position_ids, repetition_penalty,
                            presence_penalty)
        try:
            return generate_device(dec, max_length, stop_tokens)
        except Exception as e:
            guard.failed("mtp_loop", e, can_fallback=False)
            raise

    setattr(_generate_mtp, CLAIM, True)
    _generate_mtp.__wrapped__ = original
    cls._generate_mtp = _generate_mtp
    return True
