"""Host logic of the batched decode streams on CPU: the per-stream collection of committed tokens from the ring of
result rows (mtp_loop.generate_device_streams, the same rows mono_mtp_accept writes: [n, commit[8], ...]), and the
strided view of the verify rows' values that the batched attention reads in place."""
from types import SimpleNamespace

import torch

from mono_b200 import mtp_loop
from mono_b200.streams import Qwen35W4A8Streams


class _FakeBatch:
    """Three streams committing 1, 2 or 3 tokens a step in turn (token = 1000 b + 10 step + i)."""
    streams = 3

    def __init__(self):
        self.k = 0

    def step(self):
        r = torch.zeros(self.streams, 32, dtype=torch.int64)
        for b in range(self.streams):
            n = 1 + (self.k + b) % 3
            r[b, 0] = n
            r[b, 1:1 + n] = 1000 * b + 10 * self.k + torch.arange(n)
            r[b, 1 + n:9] = -1
        self.k += 1
        return r


def _expected(b, steps, limit):
    out = []
    for k in range(steps):
        n = 1 + (k + b) % 3
        out += [1000 * b + 10 * k + i for i in range(n)]
    return out[:limit]


def test_generate_device_streams_collects_every_stream():
    for limit, sync in ((10, 4), (7, 8), (1, 2)):
        fake = _FakeBatch()
        out = mtp_loop.generate_device_streams(fake, limit, sync_every=sync)
        assert len(out) == 3
        for b in range(3):
            assert out[b] == _expected(b, fake.k, limit), (limit, sync, b)
        assert fake.k % sync == 0  # whole rings of steps


def test_tree_value_rows_view():
    B, R, Hk, hd = 2, 8, 4, 256
    pre = torch.arange(B * R * (3 * Hk * hd), dtype=torch.float32).view(B * R, 3 * Hk * hd)
    v = pre[:, 2 * Hk * hd:].view(1, B * R, Hk, hd)  # the value columns of the projection rows
    view = Qwen35W4A8Streams._kv_rows(SimpleNamespace(streams=B), v)
    assert tuple(view.shape) == (B, Hk, R, hd) and view.stride(3) == 1
    ref = v[0].reshape(B, R, Hk, hd).permute(0, 2, 1, 3)
    assert torch.equal(view, ref)
    assert view.data_ptr() == v.data_ptr()  # a view: the kernel reads the rows in place
