"""mono_b200: B200 (sm_100a) kernels for the Qwen3.5-9B W4A8 decode step behind the reference's hook surface.

Submodules mirror comfy_mono_decode_xpu: _C (native ops), guard, patch (W4 linear / rot-quant routes),
mono (MLP route), layer (decode block route), tiles (tile-major weight copies).
"""
