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


def test_patch_install_is_idempotent_and_falls_back_on_the_abi_refusal():
    mod, calls = _omni()
    original = mod.w4a8_linear_prequantized
    assert patch.install(mod) is True and patch.install(mod) is False
    assert mod.w4a8_linear_prequantized.__wrapped__ is original
    x = torch.zeros(2, 4096, dtype=torch.int8)  # CPU tensors: the binding refuses them (MONO_EINVAL)
    reason = "operands must be CUDA tensors"
    before = patch.stats()["reasons"].get(reason, 0)
    assert mod.w4a8_linear_prequantized(x, torch.ones(2), torch.zeros(64, 2048, dtype=torch.int8),
                                        torch.zeros(64, 256), torch.ones(64)) == "stock"
    assert calls == ["original"] and patch.stats()["reasons"][reason] == before + 1
    assert not guard.off("w4")  # a refusal is not a failure
    guard.failed("w4", RuntimeError("off"))
    assert mod.w4a8_linear_prequantized(x, None, None, None, None) == "stock"
    assert patch.stats()["reasons"]["off"] >= 1


def test_patch_refusals_decided_on_the_host_and_failures():
    mod, calls = _omni()
    patch.install(mod)
    x = torch.zeros(2, 4096, dtype=torch.int8)
    before = patch.stats()["reasons"]
    assert mod.w4a8_linear_prequantized(x, None, None, None, None, bias=torch.zeros(1)) == "stock"
    assert mod.w4a8_linear_prequantized(x, None, None, None, None, out_dtype=torch.float16) == "stock"
    after = patch.stats()["reasons"]
    assert after["bias"] == before.get("bias", 0) + 1 and after["out_dtype"] == before.get("out_dtype", 0) + 1
    # an exception that is not an argument rejection switches the piece off
    assert mod.w4a8_linear_prequantized(x, None, None, None, None) == "stock"  # x_scale None: AttributeError
    assert guard.off("w4") and patch.stats()["reasons"]["failed"] == before.get("failed", 0) + 1


def test_install_prep_wraps_backend_modules_once():
    mod = types.ModuleType("comfy_kitchen.backends.cuda.w4a8_int8")
    mod.quantize_and_rotate_rowwise = lambda x, h, group_size, stochastic_rounding=0: "stock"
    assert patch.install_prep([mod]) == 1 and patch.install_prep([mod]) == 0
    before = patch.stats()["reasons"]
    x = torch.zeros(2, 4096, dtype=torch.bfloat16)
    assert mod.quantize_and_rotate_rowwise(x, torch.zeros(256, 256), 256) == "stock"  # CPU: refused by the binding
    assert mod.quantize_and_rotate_rowwise(x, torch.zeros(256, 256), 128) == "stock"
    assert mod.quantize_and_rotate_rowwise(x, torch.zeros(256, 256), 256, 1) == "stock"
    after = patch.stats()["reasons"]
    for key in ("operands must be CUDA tensors", "group_size", "stochastic_rounding"):
        assert after[key] == before.get(key, 0) + 1, key
    assert not guard.off("prep")


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


# ---- node entry, logits picks, weight bridge ---------------------------------------------------------------------

def _load_node(monkeypatch):
    """The custom-node entry module, loaded as ComfyUI loads it (by file), with the master switch off so that
    loading installs nothing."""
    import importlib.util
    import os
    monkeypatch.setenv("MONO_DECODE_XPU", "0")
    for piece in ("W4", "PREP", "MONO", "LAYER"):
        monkeypatch.delenv(f"MONO_DECODE_XPU_{piece}", raising=False)
    root = os.path.join(os.path.dirname(os.path.dirname(os.path.abspath(__file__))), "comfy-mono-decode-xpu_b200")
    spec = importlib.util.spec_from_file_location("mono_node_under_test", os.path.join(root, "__init__.py"),
                                                  submodule_search_locations=[root])
    node = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(node)
    return node


def test_node_entry_switches(monkeypatch):
    node = _load_node(monkeypatch)
    assert node.NODE_CLASS_MAPPINGS == {} and node.install({"MONO_DECODE_XPU": "0"}) == {}
    assert node.switches({}) == {"W4": True, "PREP": True, "MONO": True, "LAYER": True}
    assert node.switches({"MONO_DECODE_XPU": "0"}) == {"W4": False, "PREP": False, "MONO": False, "LAYER": False}
    assert node.switches({"MONO_DECODE_XPU": "0", "MONO_DECODE_XPU_W4": "1"})["W4"] is True
    assert node.switches({"MONO_DECODE_XPU_LAYER": "0"}) == {"W4": True, "PREP": True, "MONO": True, "LAYER": False}


def test_node_entry_installs_each_piece_on_its_own(monkeypatch):
    import sys
    node = _load_node(monkeypatch)
    llama, q35 = _comfy()
    mod, _ = _omni()

    class BaseGenerate:
        def logits(self, x):
            return x

    class Qwen35(BaseGenerate):
        def generate(self):
            return "stock"

        def _generate_mtp(self, *a, **k):
            return "stock-generate"
    llama.BaseGenerate, q35.Qwen35 = BaseGenerate, Qwen35
    comfy = types.ModuleType("comfy")
    te = types.ModuleType("comfy.text_encoders")
    te.llama, te.qwen35 = llama, q35
    omni = types.ModuleType("omni_xpu_kernel")
    omni.int8 = mod
    for name, m in (("comfy", comfy), ("comfy.text_encoders", te), ("comfy.text_encoders.llama", llama),
                    ("comfy.text_encoders.qwen35", q35), ("omni_xpu_kernel", omni), ("omni_xpu_kernel.int8", mod)):
        monkeypatch.setitem(sys.modules, name, m)
    monkeypatch.delattr(q35, "LinearKV")  # the device loop's KV hooks: absent in this stand-in
    got = node.install({"MONO_DECODE_XPU": "1", "MONO_DECODE_XPU_PREP": "0"})
    assert got["w4a8 linear"] is True and got["mlp block"] is True and got["decode layer"] is True
    assert got["logits picks"] is True and got["weight bridge"] is True and "rotate + quantize" not in got
    assert getattr(mod.w4a8_linear_prequantized, patch.CLAIM) and llama.MLP.forward.__wrapped__
    assert Qwen35().generate() == "stock" and not __import__("mono_b200").bridge.active()


def test_logits_picks_serve_argmax_then_reuse_the_top8(monkeypatch):
    from mono_b200 import logits

    class C:
        calls = []

        @classmethod
        def fast_pick(cls, x, k):
            cls.calls.append("pick")
            v, i = torch.topk(x.float(), k)
            return v.to(x.dtype), i, x.float().argmax(-1)

        @classmethod
        def fast_topk(cls, x, k, argmax_order):
            cls.calls.append("topk")
            v, i = torch.topk(x.float(), k)
            return v.to(x.dtype), i

    import sys
    fake = types.ModuleType("mono_b200._C")
    fake.fast_pick, fake.fast_topk = C.fast_pick, C.fast_topk
    monkeypatch.setitem(sys.modules, "mono_b200._C", fake)
    monkeypatch.setattr(__import__("mono_b200"), "_C", fake, raising=False)
    base = torch.randn(2, 3, 5000, generator=torch.Generator().manual_seed(1)).bfloat16()
    lg = base.as_subclass(logits.PickRows)
    row = lg[:, -1]
    assert type(row) is logits.PickRows
    am = row.argmax(dim=-1)
    assert torch.equal(am, base[:, -1].float().argmax(-1)) and C.calls == ["pick"]
    v, i = torch.topk(lg[:, -1], 4)  # another view object of the same rows: the kept top-8
    assert C.calls == ["pick"] and torch.equal(v, torch.topk(base[:, -1], 4).values)
    base[0, -1, 0] = 100.0  # an in-place write bumps the version: the kept rows no longer apply
    v, i = lg[:, -1].topk(2)
    assert C.calls == ["pick", "topk"] and int(i[0, 0]) == 0
    s = lg.sum()  # other ops: plain tensors
    assert type(s) is torch.Tensor
    assert logits.stats()["topk_kept"] >= 1


def test_bridge_formats_and_session():
    from mono_b200 import bridge

    class Params:
        pass

    class W:
        def __init__(self, q, p):
            self._qdata, self._params = q, p

    def lin(N, K, fmt):
        p = Params()
        if fmt == "ref":
            p.scale = torch.zeros(N, K // 16, dtype=torch.uint8).view(torch.float8_e4m3fn)
            p.s_channel, p.codebook, p.group_size, p.convrot_groupsize = torch.ones(N), torch.zeros(16), 16, 256
        else:
            p.scale = torch.zeros(N, K // 128, dtype=torch.float16)
        m = types.SimpleNamespace(weight=W(torch.zeros(N, K // 2, dtype=torch.int8), p), bias=None)
        return m

    assert bridge.weight_format(lin(64, 4096, "ref")) == ("ref", 64, 4096)
    assert bridge.weight_format(lin(64, 4096, "gptq")) == ("gptq", 64, 4096)
    assert bridge.weight_format(lin(64, 1000, "ref")) is None  # K not a multiple of 1024
    odd = lin(64, 4096, "ref")
    odd.weight._params.convrot_groupsize = 128
    assert bridge.weight_format(odd) is None
    biased = lin(64, 4096, "gptq")
    biased.bias = torch.zeros(64)
    assert bridge.weight_format(biased) is None and bridge.weight_format(types.SimpleNamespace(weight=None)) is None
    assert not bridge.active() and bridge.parts([lin(64, 4096, "ref")], "cpu") is None  # no session: nothing
    assert bridge.mlp_plan(types.SimpleNamespace(), "cpu") is None
    bridge.begin()
    assert bridge.active()
    bridge.end()
    assert not bridge.active()
