"""The top-k oracle's rank keys against the reference's stated orders (csrc/fast_topk.sycl:4-9, :22-40)."""
import numpy as np
import torch

from oracle import topk as ot


def test_all_equal_row_follows_the_gather_order():
    bits = np.zeros((1, 65536), dtype=np.uint16)
    _, i = ot.topk(bits, 8)
    assert list(i[0]) == list(range(8))  # iteration 0, thread 0, load 0, lanes 0..7
    bits[0, :8] = 0x8000  # -0 ranks below +0
    _, i = ot.topk(bits, 8)
    assert list(i[0]) == [8192, 8193, 8194, 8195, 8196, 8197, 8198, 8199]  # thread 0, load 1
    assert ot.argmax(bits)[0] == 0  # argmax: -0 == +0, smallest index


def test_nan_on_top_and_values_agree_with_torch_on_distinct_rows():
    g = torch.Generator().manual_seed(1)
    x = torch.randn(2, 50000, generator=g).to(torch.bfloat16)
    x[0, 123] = float("nan")
    bits = x.view(torch.int16).numpy().view(np.uint16)
    _, i = ot.topk(bits, 4)
    assert i[0, 0] == 123 and ot.argmax(bits)[0] == 123
    ref = x[1].float().topk(4).values.numpy()
    assert np.array_equal(x[1].float().numpy()[i[1]], ref)


def test_topk_rows_oracle_matches_torch_on_distinct_values():
    """Without ties the order is the value order: the oracle equals torch.topk (fp32, CPU)."""
    import numpy as np
    import torch

    from oracle.topk import topk_rows
    g = torch.Generator().manual_seed(31)
    x = torch.randn(3, 5000, generator=g)
    v, i = topk_rows(x.numpy(), 40)
    tv, ti = torch.topk(x, 40, dim=-1)
    assert np.array_equal(v, tv.numpy()) and np.array_equal(i, ti.numpy())


def test_topk_rows_oracle_ties_follow_the_gather_order():
    """Equal values come out in the torch-XPU gather order (csrc/topk_rows.sycl:7-10): iteration i / 32768, then
    (i % 4096) / 4, then (i % 32768) / 4096, then i % 4; -0 ranks below +0."""
    import numpy as np

    from oracle.topk import topk_rows
    N = 70000
    x = np.zeros((1, N), dtype=np.float32)
    v, i = topk_rows(x, 12)
    key = lambda j: ((j >> 15) << 15) | (((j % 32768) % 4096) // 4 << 5) | ((j % 32768) // 4096 << 2) | (j % 4)  # noqa: E731
    expect = sorted(range(N), key=key)[:12]
    assert list(i[0]) == expect
    y = np.array([[-0.0] * 64 + [0.0] * 64 + [1.0]], dtype=np.float32)
    v, i = topk_rows(y, 65)
    assert i[0, 0] == 128 and all(64 <= j < 128 for j in i[0, 1:65])
