"""mono_b200: B200 (sm_100a) kernels for the Qwen3.5-9B W4A8 decode step behind the reference's hook surface.

Submodules mirror comfy_mono_decode_xpu: _C (native ops over the C ABI; _lib loads libmono_b200.so), guard (error
contract), patch (W4 linear / rot-quant routes), mono (MLP route), layer (decode block route), logits (lm_head
route), bridge (a stock model's linears as tile-major copies, block and MLP plans), mtp_loop (device MTP loop),
sampling (verify top-k), constants (activation tables, the Hadamard rotation). Beyond the reference: decoder (the
synthetic Qwen3.5-9B-shaped model on these kernels), streams (several decode streams batched in one step on one
GPU), tp (one stream in 2-way tensor parallel).
"""
