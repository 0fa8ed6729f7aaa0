"""ComfyUI custom-node entry: this directory, placed under ComfyUI/custom_nodes/, installs mono_b200's decode routes
when ComfyUI loads it, and adds no nodes (the role of the reference node's __init__.py:16-77).

Switches, read when install() runs (at load): MONO_DECODE_XPU is the master ("1" by default, "0" off) and
MONO_DECODE_XPU_W4 / _PREP / _MONO / _LAYER set one piece each, defaulting to the master; a piece set explicitly
overrides the master (MONO_DECODE_XPU=0 MONO_DECODE_XPU_W4=1 installs only the W4 linear route).

  W4     patch.install        packed W4A8 linears of the INT8 backend -> mono_w4a8_decode_linear
  PREP   patch.install_prep   the backend's rotate + quantize row step -> mono_rot_quant
  MONO   mono.install         llama.MLP.forward on decode rows -> the fused MLP block
  LAYER  layer.install        decode blocks, attend, gated attention, RMSNorm scale cache
         logits.install       argmax / top-k of the generate's logits -> mono_fast_topk
         mtp_loop.install     Qwen35._generate_mtp -> the device MTP loop
         bridge.install       generate-time tile-major weight copies and block plans

Every piece installs on its own: one that raises is logged and left on the stock path, the others still load.
Without the built library (mono_b200/libmono_b200.so) nothing is installed and decode runs the stock code.
"""
from __future__ import annotations

import logging
import os
import sys

NODE_CLASS_MAPPINGS = {}
NODE_DISPLAY_NAME_MAPPINGS = {}

_HERE = os.path.dirname(os.path.realpath(__file__))
PIECES = ("W4", "PREP", "MONO", "LAYER")


def switches(env=None):
    """{piece: bool} from the environment (`env`, default os.environ)."""
    env = os.environ if env is None else env
    master = env.get("MONO_DECODE_XPU", "1") == "1"
    out = {}
    for piece in PIECES:
        value = env.get(f"MONO_DECODE_XPU_{piece}")
        out[piece] = master if value is None else value == "1"
    return out


def _installers():
    from mono_b200 import bridge, layer, logits, mono, mtp_loop, patch

    def prep():
        try:
            import comfy_kitchen  # noqa: F401  (loads the backend modules whose row step is replaced)
        except ImportError:
            pass
        return patch.install_prep()

    return {"W4": [("w4a8 linear", patch.install)],
            "PREP": [("rotate + quantize", prep)],
            "MONO": [("mlp block", mono.install)],
            "LAYER": [("decode layer", layer.install), ("logits picks", logits.install),
                      ("device MTP loop", mtp_loop.install), ("weight bridge", bridge.install)]}


def install(env=None):
    """Install the switched-on pieces; returns {label: what its install returned, or None after an error}."""
    on = switches(env)
    if not any(on.values()):
        return {}
    if _HERE not in sys.path:
        sys.path.insert(0, _HERE)  # one module identity: mono_b200 is imported by its own name
    try:
        from mono_b200 import _lib
        _lib.load()
    except (ImportError, OSError) as e:
        logging.warning("[mono_b200] library not available (%s): build it with `python csrc/build.py` in %s; "
                        "decode runs the stock path", e, _HERE)
        return {}
    results = {}
    for piece, entries in _installers().items():
        if not on[piece]:
            continue
        for label, fn in entries:
            try:
                results[label] = fn()
                logging.info("[mono_b200] %s installed=%s", label, results[label])
            except Exception:  # never take ComfyUI down: this piece keeps the stock path
                results[label] = None
                logging.exception("[mono_b200] %s failed to install; it stays on the stock path", label)
    return results


install()
