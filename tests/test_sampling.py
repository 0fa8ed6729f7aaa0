"""The verify sampling's top-k server (mono_b200.sampling; the reference's sampling.py) on CPU tensors, with the
oracle standing in for C.topk_rows and raising the C ABI's argument rejection where mono_topk_rows would:
torch.topk / Tensor.topk calls are bound to torch.topk's signature and served when they ask for the sorted k
largest along the last dim; other forms, rejected arguments, failures and check mode fall through to torch; no
other op is intercepted."""
import numpy as np
import pytest
import torch

from mono_b200 import _lib, guard, sampling
from oracle.topk import topk_rows as ref_topk_rows


class _C:
    calls = 0

    @classmethod
    def topk_rows(cls, x, k, index_order=False):
        """mono_topk_rows's argument checks (include/mono_b200.h), then the oracle."""
        ok = (x.dim() == 2 and x.is_contiguous() and x.dtype in (torch.float32, torch.bfloat16)
              and 1 <= x.shape[0] <= 16 and 64 <= x.shape[1] and 1 <= k <= 64)
        if not ok:
            raise _lib.MonoError("mono_topk_rows", _lib.MONO_EINVAL, f"rows in [1, 16], N >= 64, k in [1, 64] (got {k})")
        cls.calls += 1
        v, i = ref_topk_rows(x.float().numpy(), k, index_order)
        return torch.from_numpy(v), torch.from_numpy(i)


@pytest.fixture(autouse=True)
def _cpu(monkeypatch):
    monkeypatch.setattr(sampling, "DEVICES", ("cpu",))
    monkeypatch.setattr(sampling, "MODE", "1")
    guard.reset()
    _C.calls = 0
    yield
    guard.reset()


def test_every_spelling_of_the_call_is_served_and_matches_torch():
    x = torch.randn(4, 40000, generator=torch.Generator().manual_seed(3))  # fp32 normals: no ties
    ref = torch.topk(x, 50)
    with sampling.topk_mode(_C):
        got = [torch.topk(x, 50), x.topk(50), torch.topk(x, k=50, dim=1, largest=True, sorted=True),
               torch.topk(input=x, k=50, dim=-1), x.topk(np.int64(50), -1)]
    assert _C.calls == len(got)
    for v, i in got:
        assert torch.equal(v, ref.values) and torch.equal(i, ref.indices)


def test_leading_dims_are_flattened_and_bf16_values_stay_bf16():
    x = (torch.randn(2, 3, 40000, generator=torch.Generator().manual_seed(4)) * 3).bfloat16()  # bf16: ties
    with sampling.topk_mode(_C):
        v, i = torch.topk(x, 16)
    assert _C.calls == 1 and v.shape == (2, 3, 16) and v.dtype == torch.bfloat16
    assert torch.equal(v, torch.topk(x, 16).values)  # values bit for bit
    rv, ri = ref_topk_rows(x.reshape(6, -1).float().numpy(), 16, True)  # ties: ascending index
    assert np.array_equal(i.reshape(6, 16).numpy(), ri)


def test_other_forms_pass_through():
    x = torch.randn(3, 40000)
    before = sampling.stats().get("passed", 0)
    with sampling.topk_mode(_C):
        outs = [torch.topk(x, 8, largest=False), torch.topk(x, 8, sorted=False), torch.topk(x, 2, dim=0),
                torch.topk(x, 8, out=(torch.empty(3, 8), torch.empty(3, 8, dtype=torch.long)))]
    assert _C.calls == 0 and sampling.stats()["passed"] == before + len(outs)
    assert torch.equal(outs[0].values, torch.topk(x, 8, largest=False).values)


def test_rejected_arguments_run_torch_without_switching_the_piece_off():
    before = sampling.stats()
    with sampling.topk_mode(_C):
        a = torch.topk(torch.randn(2, 32), 4)  # rows too short
        b = torch.topk(torch.randn(17, 1000), 4)  # 17 rows
        c = torch.topk(torch.randn(2, 1000), 65)  # k > 64
    after = sampling.stats()
    assert _C.calls == 0 and not guard.off(sampling.PIECE)
    assert after["rejected"] == before.get("rejected", 0) + 3
    assert any(key.startswith("rejected: ") and "(got" not in key for key in after)
    assert a.values.shape == (2, 4) and b.values.shape == (17, 4) and c.values.shape == (2, 65)


def test_a_failing_topk_rows_switches_the_piece_off():
    class Bad:
        @staticmethod
        def topk_rows(x, k, index_order=False):
            raise RuntimeError("launch failed")

    x = torch.randn(2, 40000)
    with sampling.topk_mode(Bad):
        v, _ = torch.topk(x, 4)
    assert torch.equal(v, torch.topk(x, 4).values) and guard.off(sampling.PIECE)
    assert isinstance(sampling.topk_mode(_C), type(sampling.topk_mode(None)))  # a null context from now on


def test_sort_and_the_rest_of_the_filter_are_torch_own():
    x = torch.randn(3, 40000).round()  # many ties
    with sampling.topk_mode(_C):
        v, _ = torch.topk(x, 32)
        s, j = torch.sort(v, descending=True)
        p = torch.softmax(v, dim=-1)
    rs, rj = torch.sort(v, descending=True)
    assert torch.equal(s, rs) and torch.equal(j, rj) and torch.equal(p, torch.softmax(v, dim=-1))


def test_check_mode_returns_torch_and_counts():
    lg0 = torch.randn(2, 40000, generator=torch.Generator().manual_seed(5))  # fp32 normals: no ties
    before = sampling.stats()
    sampling.MODE = "check"
    ctx, rows = sampling.verify_rows(_C, lg0)
    with ctx:
        v, i = torch.topk(rows, 10)
    after = sampling.stats()
    assert _C.calls == 1 and after["checked"] == before.get("checked", 0) + 1
    assert after.get("check_mismatch", 0) == before.get("check_mismatch", 0)
    assert torch.equal(v, torch.topk(lg0, 10).values)


def test_verify_rows_hands_out_fp32_rows(monkeypatch):
    lg0 = torch.randn(2, 40000).bfloat16()
    ctx, rows = sampling.verify_rows(_C, lg0)
    assert rows.dtype == torch.float32 and torch.equal(rows, lg0.float())
    f = lg0.float()
    assert sampling.verify_rows(_C, f)[1] is f
    monkeypatch.setattr(sampling, "MODE", "0")
    ctx, _ = sampling.verify_rows(_C, lg0)
    with ctx:
        torch.topk(f, 4)
    assert _C.calls == 0
