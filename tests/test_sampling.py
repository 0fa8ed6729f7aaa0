"""The verify sampling's top-k mode (mono_b200.sampling; the reference's sampling.py) on CPU tensors with a
stand-in topk_rows (the oracle): eligible torch.topk calls are served, the bf16 rows stand for their fp32 copy,
sorted top-k values skip the sort, ineligible calls and check mode fall through to torch."""
import numpy as np
import pytest
import torch

from mono_b200 import guard, sampling
from oracle.topk import topk_rows as ref_topk_rows


class _C:
    calls = 0

    @classmethod
    def topk_rows(cls, x, k):
        cls.calls += 1
        v, i = ref_topk_rows(x.float().numpy(), k)
        return torch.from_numpy(v), torch.from_numpy(i)


@pytest.fixture(autouse=True)
def _cpu(monkeypatch):
    monkeypatch.setattr(sampling, "DEVICES", ("cpu",))
    monkeypatch.setattr(sampling, "MODE", "1")
    guard.reset()
    _C.calls = 0
    yield
    guard.reset()


def test_topk_is_served_and_matches_torch():
    g = torch.Generator().manual_seed(3)
    x = torch.randn(4, 40000, generator=g)
    with sampling.topk_mode(_C):
        v, i = torch.topk(x, 50)
        s, j = torch.sort(v, descending=True)
    tv, ti = torch.topk(x, 50)
    assert _C.calls == 1 and torch.equal(v, tv) and torch.equal(i, ti)
    assert torch.equal(s, v) and torch.equal(j, torch.arange(50).expand(4, 50))
    assert sampling.stats()["sorted"] >= 1


def test_ineligible_calls_fall_through():
    x = torch.randn(4, 1000)  # rows too short
    with sampling.topk_mode(_C):
        v, i = torch.topk(x, 8)
        w, _ = torch.topk(torch.randn(2, 40000), 8, largest=False)
    assert _C.calls == 0 and torch.equal(v, torch.topk(x, 8).values)


def test_bf16_rows_stand_in_for_their_fp32_copy():
    g = torch.Generator().manual_seed(4)
    lg0 = torch.randn(3, 40000, generator=g).bfloat16()
    ctx, rows = sampling.verify_rows(_C, lg0)
    assert rows is lg0
    with ctx:
        assert rows.dtype == torch.float32 and rows.shape == (3, 40000)
        v, i = torch.topk(rows, 16)
        probs = torch.softmax(rows, dim=-1)  # any other op runs on the fp32 copy
    assert _C.calls == 1 and probs.dtype == torch.float32
    rv, ri = ref_topk_rows(lg0.float().numpy(), 16)  # bf16 rows hold ties: the torch-XPU tie order, not torch CPU's
    assert np.array_equal(v.numpy(), rv) and np.array_equal(i.numpy(), ri)
    assert torch.equal(v, torch.topk(lg0.float(), 16).values)
    assert torch.allclose(probs, torch.softmax(lg0.float(), dim=-1))


def test_off_and_check_modes(monkeypatch):
    lg0 = torch.randn(2, 40000).bfloat16()
    monkeypatch.setattr(sampling, "MODE", "0")
    ctx, rows = sampling.verify_rows(_C, lg0)
    assert rows.dtype == torch.float32 and rows is not lg0
    monkeypatch.setattr(sampling, "MODE", "check")
    before = sampling.stats()
    x = torch.randn(2, 40000, generator=torch.Generator().manual_seed(5))  # fp32: no ties
    with sampling.topk_mode(_C):
        v, i = torch.topk(x, 10)
    after = sampling.stats()
    assert _C.calls == 1 and after["checked"] == before["checked"] + 1
    assert after["check_mismatch"] == before["check_mismatch"] and torch.equal(v, torch.topk(x, 10).values)


def test_a_failing_topk_rows_disables_the_piece():
    class Bad:
        @staticmethod
        def topk_rows(x, k):
            raise RuntimeError("rejected")

    x = torch.randn(2, 40000)
    with sampling.topk_mode(Bad):
        v, _ = torch.topk(x, 4)
    assert torch.equal(v, torch.topk(x, 4).values) and guard.off("sample_topk")
