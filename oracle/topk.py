"""Exact top-k / argmax over bf16 logit rows on the CPU (test infrastructure only; see oracle/__init__.py).

Restates the reference's rank keys (csrc/fast_topk.sycl:22-40): a 64-bit rank, larger = better.
  top-k:  high 32 bits = the bf16 radix key (NaN on top, -0 below +0: bits ^ 0xFFFF for negatives,
          bits ^ 0x8000 otherwise), low 32 bits = ~gather key, where the gather key orders ties as the
          XPU topk gathers them: (i >> 15) << 15 | ((i & 8191) >> 3) << 5 | ((i & 32767) >> 13) << 3 | (i & 7)
  argmax: high 32 bits = the float order key (NaN largest, -0 == +0), low 32 bits = ~i (smallest index wins).
"""
from __future__ import annotations

import numpy as np


def rank_topk(bits: np.ndarray) -> np.ndarray:
    b = bits.astype(np.uint64)
    i = np.arange(b.shape[-1], dtype=np.uint64)
    mask = np.where(b & 0x8000, np.uint64(0xFFFF), np.uint64(0x8000))
    nan = (b & 0x7FFF) > 0x7F80
    conv = np.where(nan, np.uint64(0xFFFF), (b ^ mask) & 0xFFFF)
    it, off = i >> np.uint64(15), i & np.uint64(32767)
    g = (it << np.uint64(15)) | (((off & np.uint64(8191)) >> np.uint64(3)) << np.uint64(5)) | \
        ((off >> np.uint64(13)) << np.uint64(3)) | (off & np.uint64(7))
    return (conv << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - g)


def rank_argmax(bits: np.ndarray) -> np.ndarray:
    b = bits.astype(np.uint64)
    i = np.arange(b.shape[-1], dtype=np.uint64)
    nan = (b & 0x7FFF) > 0x7F80
    b0 = np.where((b & 0x7FFF) == 0, np.uint64(0), b)
    key = np.where(b0 & 0x8000, np.uint64(0x7FFF) - (b0 & 0x7FFF), np.uint64(0x8000) + b0)
    key = np.where(nan, np.uint64(0xFFFFFFFF), key)
    return (key << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - i)


def topk(bits: np.ndarray, k: int, argmax_order: bool = False):
    """bits [rows, V] uint16. Returns (values [rows, k] uint16, indices [rows, k] int64)."""
    r = rank_argmax(bits) if argmax_order else rank_topk(bits)
    idx = np.empty((bits.shape[0], k), dtype=np.int64)
    for row in range(bits.shape[0]):
        top = np.argpartition(r[row], -k)[-k:] if k < bits.shape[1] else np.arange(bits.shape[1])
        idx[row] = top[np.argsort(r[row][top])[::-1]][:k]  # ranks are distinct: an exact order
    return np.take_along_axis(bits, idx, axis=-1), idx


def argmax(bits: np.ndarray) -> np.ndarray:
    return np.argmax(rank_argmax(bits), axis=-1).astype(np.int64)


def topk_rows_rank(bits32, i, index_order=False):
    """The topk_rows rank of fp32 bit patterns at indices i: the radix key (sign-flipped bits) << 32 | ~g, g the
    torch-XPU gather key of index i (the reference's, csrc/topk_rows.sycl:34-42), or with index_order g = i (equal
    values by ascending index: torch's CUDA topk order for k >= 33 and k = 1, measured on B200)."""
    b = np.asarray(bits32, dtype=np.uint64)
    key = b ^ np.where(b & 0x80000000, np.uint64(0xFFFFFFFF), np.uint64(0x80000000))
    i = np.asarray(i, dtype=np.uint64)
    if index_order:
        g = i
    else:
        off = i & np.uint64(32767)
        g = ((i >> np.uint64(15)) << np.uint64(15)) | (((off & np.uint64(4095)) >> np.uint64(2)) << np.uint64(5)) | \
            ((off >> np.uint64(12)) << np.uint64(2)) | (off & np.uint64(3))
    return (key << np.uint64(32)) | (np.uint64(0xFFFFFFFF) - g)


def topk_rows(x_f32, k, index_order=False):
    """torch.topk(x, k) of fp32 rows [R, N] as the topk_rows kernel defines it: the k largest 64-bit ranks per row,
    descending (equal values in the torch-XPU gather order of the reference's csrc/topk_rows.sycl:7-10, or by
    ascending index with index_order). Returns (values fp32 [R, k], indices int64 [R, k])."""
    x = np.ascontiguousarray(x_f32, dtype=np.float32)
    R, N = x.shape
    bits = x.view(np.uint32)
    idx = np.arange(N, dtype=np.uint64)
    vals, inds = [], []
    for r in range(R):
        rank = topk_rows_rank(bits[r], idx, index_order)
        top = np.argsort(rank)[::-1][:k]
        inds.append(top.astype(np.int64))
        vals.append(x[r, top])
    return np.stack(vals), np.stack(inds)
