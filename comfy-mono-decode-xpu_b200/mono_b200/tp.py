"""2-way tensor parallelism of one decode stream (the reference has no distributed path).

Sharding of the Qwen3.5 decode step over `world` ranks (one process per GPU, torch.distributed over NCCL):

  column-sharded (each rank its heads / channels, no communication)
    attention q | k | v     query heads [r H/W, (r + 1) H/W) (q and gate rows of a head together), kv heads alike
    GDN qkv | z, a | b      key heads [r HK/W, ...) of q and k, value heads [r HV/W, ...) of v, z, a, b; the conv
                            channels, dt_bias, decay, recurrent state and saved inputs of those heads
    MLP gate | up           intermediate rows [r I/W, (r + 1) I/W)
    MTP q | k | v, gate|up  as above (the MTP block's fc and norms are replicated)
  row-sharded (K split), followed by an all-reduce (sum) of the bf16 [M, 4096] output
    o_proj / out_proj, MLP down, the MTP block's o and down
  vocabulary-sharded
    lm_head rows [r V/W, (r + 1) V/W): each rank picks among its rows; the candidates (value bits and global index
    of the argmax and of the top-k) are all-gathered and merged by the same rank keys as the one-GPU pick, so the
    merged pick equals the pick over the whole vocabulary exactly (merge_pick)
  replicated: the embedding, the norms, the accept walk and its bookkeeping (every rank walks the same tokens)

The all-reduce: on two GPUs a one-shot kernel over NVLink peer memory (mono_allreduce2_bf16: each rank stores its
partial into the peer's buffer, raises the peer's counter, waits for its own, sums; MONO_DECODE_XPU_TP_P2P = "0"
uses NCCL instead). Numerics of the row-sharded projections: rank 0 adds the residual, every rank rounds its
partial to bf16, the all-reduce sums the partials (fp32 sum of the two bf16 values, rounded once); the fused MLP quantizes h with the amax of its own I / W columns (a finer grid than
the one-GPU model's). Against the one-GPU model the sharded outputs agree within a stated tolerance
(tests/test_tp.py), not bit for bit; the vocabulary merge is exact.
"""
from __future__ import annotations

import os

import torch

ARGMAX_TIE_SHIFT = 32


# ---- shard maps (index ranges into the one-GPU weights) ------------------------------------------------------

def head_rows(n_heads: int, rows_per_head: int, rank: int, world: int) -> tuple:
    """The [start, stop) rows of rank `rank`'s heads in a matrix of n_heads x rows_per_head rows."""
    if n_heads % world:
        raise ValueError(f"{n_heads} heads do not split over {world} ranks")
    per = n_heads // world
    return rank * per * rows_per_head, (rank + 1) * per * rows_per_head


def gdn_channels(hk: int, hv: int, d: int, rank: int, world: int) -> torch.Tensor:
    """The conv / qkv channels of a rank: its key heads of q, of k, and its value heads of v (int64 indices into
    the C = 2 hk d + hv d channels)."""
    q0, q1 = head_rows(hk, d, rank, world)
    v0, v1 = head_rows(hv, d, rank, world)
    kd = hk * d
    return torch.cat([torch.arange(q0, q1), torch.arange(kd + q0, kd + q1), torch.arange(2 * kd + v0, 2 * kd + v1)])


def split_range(n: int, rank: int, world: int) -> tuple:
    if n % world:
        raise ValueError(f"{n} does not split over {world} ranks")
    per = n // world
    return rank * per, (rank + 1) * per


def gptq_cols(packed: torch.Tensor, scales: torch.Tensor, k0: int, k1: int) -> tuple:
    """Columns [k0, k1) of a GPTQ matrix (packed [N, K/2] nibble bytes, scales [N, K/128]); k0, k1 multiples of 128."""
    if k0 % 128 or k1 % 128:
        raise ValueError("K slices of a GPTQ matrix start and end on 128-column groups")
    return packed[:, k0 // 2:k1 // 2].contiguous(), scales[:, k0 // 128:k1 // 128].contiguous()


# ---- the vocabulary-sharded pick --------------------------------------------------------------------------------

def argmax_rank(bits: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """The argmax rank of bf16 values (int64): float order key (NaN largest, -0 == +0) << 32 | ~index — larger is
    better; among equal values the smallest index wins (csrc/ranks.cuh rank_argmax)."""
    b = bits.to(torch.int64) & 0xFFFF
    nan = (b & 0x7FFF) > 0x7F80
    b = torch.where((b & 0x7FFF) == 0, torch.zeros_like(b), b)
    key = torch.where((b & 0x8000) != 0, 0x7FFF - (b & 0x7FFF), 0x8000 + b)
    key = torch.where(nan, torch.full_like(b, 0x10000), key)  # above every number's key (0xFF80 at most); the kernel
    return (key << ARGMAX_TIE_SHIFT) | (0xFFFFFFFF - index)   # uses 0xFFFFFFFF, the same order


def topk_rank(bits: torch.Tensor, index: torch.Tensor) -> torch.Tensor:
    """The top-k rank of bf16 values (int64): radix key (NaN on top, -0 below +0) << 32 | ~g(index), g the
    reference's gather key (csrc/ranks.cuh rank_topk)."""
    b = bits.to(torch.int64) & 0xFFFF
    nan = (b & 0x7FFF) > 0x7F80
    conv = torch.where((b & 0x8000) != 0, b ^ 0xFFFF, b ^ 0x8000)
    conv = torch.where(nan, torch.full_like(b, 0xFFFF), conv)
    i = index
    off = i & 32767
    g = ((i >> 15) << 15) | (((off & 8191) >> 3) << 5) | ((off >> 13) << 3) | (off & 7)
    return (conv << 32) | (0xFFFFFFFF - g)


def merge_pick(values: torch.Tensor, indices: torch.Tensor, am_values: torch.Tensor, am_indices: torch.Tensor, k: int):
    """Merge the ranks' candidates: values / indices [W, M, k] (each rank's top-k, global indices), am_values /
    am_indices [W, M] (each rank's argmax). Returns (argmax [M], top-k [M, k]) over the whole vocabulary."""
    W, M = am_values.shape
    ar = argmax_rank(am_values, am_indices)                      # [W, M]
    best = ar.argmax(dim=0)                                      # ranks are distinct: no ties
    am = am_indices.gather(0, best.view(1, M)).view(M)
    if k == 0:
        return am, None
    tr = topk_rank(values, indices).permute(1, 0, 2).reshape(M, W * k)
    order = tr.argsort(dim=1, descending=True)[:, :k]
    top = indices.permute(1, 0, 2).reshape(M, W * k).gather(1, order)
    return am, top


# ---- the sharded decoder ------------------------------------------------------------------------------------------

def local_config(cfg, world: int):
    """The per-rank shapes of the 2-way (or W-way) shard: heads, key / value heads and the MLP's intermediate size
    divided by `world`; hidden size and vocabulary (the embedding) whole."""
    import dataclasses
    for name in ("heads", "kv_heads", "gdn_k_heads", "gdn_v_heads", "inter"):
        if getattr(cfg, name) % world:
            raise ValueError(f"{name} = {getattr(cfg, name)} does not split over {world} ranks")
    if cfg.vocab % (8 * world) or (cfg.inter // world) % 1024:
        raise ValueError("the vocabulary shard and the MLP shard must keep the kernels' tile sizes")
    return dataclasses.replace(cfg, heads=cfg.heads // world, kv_heads=cfg.kv_heads // world,
                               gdn_k_heads=cfg.gdn_k_heads // world, gdn_v_heads=cfg.gdn_v_heads // world,
                               inter=cfg.inter // world)


def make_decoder(cfg, device, group, prompt_len, gen_tokens=512, seed=0x5EED + 4, draft_gemv=True):
    """The synthetic decoder of mono_b200.decoder sharded over the ranks of `group` (one stream; every rank builds
    its shard with the same seed, so the replicated parts are equal on every rank)."""
    import torch.distributed as dist

    from .decoder import Qwen35W4A8

    class Qwen35W4A8TP(Qwen35W4A8):
        """One decode stream over the ranks of a process group: local heads / channels / MLP rows, row-sharded
        projections followed by an all-reduce, a vocabulary shard of the lm_head with the merged pick."""

        def __init__(self):
            self.tp_group = group
            self.tp_rank, self.tp_world = dist.get_rank(group), dist.get_world_size(group)
            self.full_cfg = cfg
            super().__init__(local_config(cfg, self.tp_world), device, prompt_len, gen_tokens, seed,
                             draft_gemv=draft_gemv)
            v0, v1 = split_range(cfg.vocab, self.tp_rank, self.tp_world)
            self.lm_head = self.lm_head[v0:v1].contiguous()
            self.vocab_base = v0
            # the residual sums: the one-shot peer kernel on two GPUs (MONO_DECODE_XPU_TP_P2P, "0": NCCL)
            self.peer_sum = None
            if self.tp_world == 2 and os.environ.get("MONO_DECODE_XPU_TP_P2P", "1") == "1":
                def exchange(h):
                    out = [None] * self.tp_world
                    dist.all_gather_object(out, h, group=self.tp_group)
                    return out
                self.peer_sum = _C().PeerSum(device, 8 * cfg.hidden, exchange, 1 - self.tp_rank)

        def close(self):
            if self.peer_sum is not None:
                self.peer_sum.close()
                self.peer_sum = None

        def tp_reduces_per_step(self):
            """All-reduces of a step: two per layer, two per draft's MTP block."""
            return 2 * self.cfg.layers + 2 * self.cfg.depth

        def _residual(self, r):
            if self.tp_rank == 0:
                return r
            return False if r is True else None

        def _reduce(self, t):
            if self.peer_sum is not None:
                return self.peer_sum(t)
            dist.all_reduce(t, group=self.tp_group)
            return t

        def _pick(self, xf, k, argmax_out=None, children=None, dst=None, node=0):
            import torch
            M = xf.shape[0]
            am, tk, lg = _C().lmhead_pick(xf, self.lm_head, k=k, logits=True, index_base=self.vocab_base)
            bits = lg.view(torch.int16).to(torch.int64) & 0xFFFF
            cols = [bits.gather(1, (am - self.vocab_base).view(M, 1)), am.view(M, 1)]
            if k:
                cols += [bits.gather(1, tk - self.vocab_base), tk]
            mine = torch.cat(cols, dim=1)                                   # [M, 2 + 2k]
            parts = [torch.empty_like(mine) for _ in range(self.tp_world)]
            dist.all_gather(parts, mine, group=self.tp_group)
            allc = torch.stack(parts)                                       # [W, M, 2 + 2k]
            am_g, top_g = merge_pick(allc[:, :, 2:2 + k], allc[:, :, 2 + k:], allc[:, :, 0], allc[:, :, 1], k)
            if argmax_out is not None:
                argmax_out.copy_(am_g)
            if dst is not None:
                kids = [c for c in self.tree["children"][node] if c >= 0]
                for j, c in enumerate(kids):
                    dst[c:c + 1].copy_(am_g[:1] if (j == 0 or j >= k) else top_g[0, j:j + 1])

    return Qwen35W4A8TP()


def _C():
    from . import _C as ops
    return ops
