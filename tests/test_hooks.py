"""The host install points (mono_b200.guard / patch / mono / layer / mtp_loop) against stand-ins of the ComfyUI and
omni_xpu_kernel entry types (the approach of the reference's tests/test_runtime.py:24-31): idempotent claims,
__wrapped__, environment switches, contract fallbacks and the failure guard. CPU only."""
import types

import pytest
import torch

from mono_b200 import guard, layer, mono, mtp_loop, patch


@pytest.fixture(autouse=True)
def _clean_guard():
    guard.reset()
    yield
    guard.reset()


def test_guard_disables_a_piece_and_reraises_interrupts(monkeypatch):
    guard.failed("x", RuntimeError("boom"))
    assert guard.off("x") and "boom" in guard.disabled()["x"]
    monkeypatch.setattr(guard, "_is_interrupt", lambda e: True)
    with pytest.raises(KeyboardInterrupt):
        guard.failed("y", KeyboardInterrupt())
    assert not guard.off("y")


def _omni():
    calls = []
    mod = types.ModuleType("omni_xpu_kernel.int8")

    def w4a8_linear_prequantized(x, xs, packed, s_rel, s_ch, codebook=None, bias=None, group_size=16,
                                 out_dtype=torch.bfloat16):
        calls.append("original")
        return "stock"
    mod.w4a8_linear_prequantized = w4a8_linear_prequantized
    return mod, calls


def test_patch_install_is_idempotent_and_falls_back_off_contract():
    mod, calls = _omni()
    original = mod.w4a8_linear_prequantized
    assert patch.install(mod) is True and patch.install(mod) is False
    assert mod.w4a8_linear_prequantized.__wrapped__ is original
    x = torch.zeros(2, 4096, dtype=torch.int8)  # CPU tensors: outside the contract
    before = patch.stats()["reasons"].get("x", 0)
    assert mod.w4a8_linear_prequantized(x, torch.ones(2), torch.zeros(64, 2048, dtype=torch.int8),
                                        torch.zeros(64, 256), torch.ones(64)) == "stock"
    assert calls == ["original"] and patch.stats()["reasons"]["x"] == before + 1
    guard.failed("w4", RuntimeError("off"))
    assert mod.w4a8_linear_prequantized(x, None, None, None, None) == "stock"


def test_patch_contract_reasons():
    c = patch.contract
    x = torch.zeros(2, 4096, dtype=torch.int8)
    assert c(x, None, None, None, None, None, torch.zeros(1), 16, torch.bfloat16) == "bias"
    assert c(x, None, None, None, None, None, None, 16, torch.float16) == "out_dtype"
    assert c(x, None, None, None, None, None, None, 16, torch.bfloat16) == "x"


def test_install_prep_wraps_backend_modules_once():
    mod = types.ModuleType("comfy_kitchen.backends.cuda.w4a8_int8")
    mod.quantize_and_rotate_rowwise = lambda x, h, group_size, stochastic_rounding=0: "stock"
    assert patch.install_prep([mod]) == 1 and patch.install_prep([mod]) == 0
    assert mod.quantize_and_rotate_rowwise(torch.zeros(2, 4096, dtype=torch.bfloat16), torch.zeros(256, 256), 256) == "stock"


def _comfy():
    llama = types.ModuleType("comfy.text_encoders.llama")
    q35 = types.ModuleType("comfy.text_encoders.qwen35")

    class MLP:
        def forward(self, x, norm=None):
            return "stock-mlp"

    class FixedKVCache:
        def attend(self, xq, xk, xv):
            return "stock-attend"

    class RMSNorm:
        def __init__(self):
            self.weight = torch.ones(4)
            self.n = 0

        def scale(self):
            self.n += 1
            return self.weight + 1

    class Block:
        def forward(self, x, attention_mask=None, freqs_cis=None, optimized_attention=None, past_key_value=None):
            return "stock-block"

    class GatedAttention:
        def forward(self, x, attention_mask=None, freqs_cis=None, optimized_attention=None, past_key_value=None):
            return "stock-attn"

    class Qwen35:
        def _generate_mtp(self, embeds, max_length, stop_tokens, mtp, sampling=None, position_ids=None,
                          repetition_penalty=1.0, presence_penalty=0.0):
            return "stock-generate"

    class LinearKV:
        def prepare(self, num_tokens):
            return "stock-prepare"

    llama.MLP, llama.FixedKVCache, llama.RMSNorm, llama.SPEC_ROWS = MLP, FixedKVCache, RMSNorm, 8
    q35.Qwen35TransformerBlock, q35.GatedAttention, q35.Qwen35, q35.LinearKV = Block, GatedAttention, Qwen35, LinearKV
    return llama, q35


def test_mono_install_falls_back_without_tiled_weights():
    llama, _ = _comfy()
    assert mono.install(llama) and not mono.install(llama)
    m = llama.MLP()
    m.gate_proj = m.up_proj = m.down_proj = object()
    assert m.forward(torch.zeros(1, 4096, dtype=torch.bfloat16), norm=object()) == "stock-mlp"
    assert llama.MLP.forward.__wrapped__(m, None) == "stock-mlp"


def test_layer_install_points_and_fallbacks():
    llama, q35 = _comfy()
    assert layer.install(q35, llama) and not layer.install(q35, llama)
    kv = llama.FixedKVCache()
    kv.key = kv.value = torch.zeros(1, 4, 16, 256, dtype=torch.bfloat16)
    kv.seqlen = torch.zeros(1, dtype=torch.int32)
    kv.tracker = {}
    assert kv.attend(torch.zeros(1, 16, 1, 256, dtype=torch.bfloat16), None, None) == "stock-attend"  # CPU
    blk = q35.Qwen35TransformerBlock()
    assert blk.forward(torch.zeros(1, 2, 4096, dtype=torch.bfloat16), past_key_value=object()) == "stock-block"
    assert layer.stats().get("fallback_weights", 0) >= 1
    n = llama.RMSNorm()
    with torch.inference_mode():
        a, b = n.scale(), n.scale()
    assert a is b and n.n == 1  # cached per weight
    ga = q35.GatedAttention()
    assert ga.forward(torch.zeros(1, 2, 4096)) == "stock-attn"  # fp32 / no cache: the original


def test_mtp_loop_install_routes_only_decoder_models(monkeypatch):
    llama, q35 = _comfy()
    assert mtp_loop.install(q35, llama) and not mtp_loop.install(q35, llama)
    model = q35.Qwen35()
    assert model._generate_mtp(None, 4, [], None) == "stock-generate"
    lk = q35.LinearKV()
    assert lk.prepare(1) == "stock-prepare"
    lk._mono_device = True
    assert lk.prepare(1) is None

    class FakeDecoder:
        def __init__(self):
            self.i = 0

        def step(self):
            self.i += 1
            r = torch.zeros(32, dtype=torch.int64)
            r[0], r[1] = 1, 100 + self.i
            return r
    model.mono_b200_decoder = FakeDecoder()
    assert model._generate_mtp(None, 5, [], None) == [101, 102, 103, 104, 105]
    assert model._generate_mtp(None, 5, [], None, sampling=object()) == "stock-generate"
    monkeypatch.setattr(mtp_loop, "MODE", "0")
    llama2, q352 = _comfy()
    assert mtp_loop.install(q352, llama2) is False
