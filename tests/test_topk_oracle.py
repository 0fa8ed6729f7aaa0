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
