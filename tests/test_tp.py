"""The 2-way tensor-parallel variant (mono_b200.tp) on CPU: the shard maps reassemble the one-GPU weights, the
vocabulary-sharded pick merges into exactly the one-GPU pick (ties across the shard boundary included), and two
gloo ranks running their shards of an MLP block and of a row-sharded o_proj through the oracle, with the
all-reduce of the bf16 partials, match the one-GPU oracle within the stated tolerance:

    |tp - one_gpu| <= 2^-6 |one_gpu| + 2^-6 max |one_gpu|

(the row-sharded sums are rounded per rank and the shards quantize h with their own amax: a finer grid; the
bound is a few bf16 ulps of the output's scale)."""
import os
import socket
import sys

import numpy as np
import pytest
import torch
import torch.multiprocessing as mp

from mono_b200 import tp
from oracle import layers as ol
from oracle import topk as otk
from oracle import w4a8 as ow
from oracle.numerics import bf16_bits_to_f32, f32_to_bf16_bits

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def test_shard_maps_reassemble_the_weights():
    W = 2
    q = torch.arange(16 * 512).view(16 * 512, 1)  # 16 gated heads of 2 x 256 rows
    parts = [q[slice(*tp.head_rows(16, 512, r, W))] for r in range(W)]
    assert torch.equal(torch.cat(parts), q)
    ch = [tp.gdn_channels(16, 32, 128, r, W) for r in range(W)]
    allc = torch.cat(ch)
    assert sorted(allc.tolist()) == list(range(2 * 16 * 128 + 32 * 128)) and len(ch[0]) == 2 * 8 * 128 + 16 * 128
    assert ch[1][0] == 8 * 128 and ch[1][1024] == 16 * 128 + 8 * 128 and ch[1][2048] == 2 * 16 * 128 + 16 * 128
    packed, scales = ow.gen_gptq(64, 2048, 3)
    pk, sc = torch.from_numpy(packed), torch.from_numpy(scales)
    cols = [tp.gptq_cols(pk, sc, *tp.split_range(2048, r, W)) for r in range(W)]
    assert torch.equal(torch.cat([c[0] for c in cols], 1), pk) and torch.equal(torch.cat([c[1] for c in cols], 1), sc)
    with pytest.raises(ValueError):
        tp.gptq_cols(pk, sc, 64, 1024)
    from mono_b200.decoder import Qwen35Config
    local = tp.local_config(Qwen35Config(), 2)
    assert (local.heads, local.kv_heads, local.gdn_k_heads, local.gdn_v_heads, local.inter) == (8, 2, 8, 16, 6144)
    assert local.hidden == 4096 and local.vocab == 151936


def _shard_candidates(bits, r, Vl, k):
    """A rank's candidates as the kernel forms them (mono_lmhead_pick with index_base = r Vl): ranks of the
    shard's values at their global indices."""
    sb = torch.from_numpy(bits[:, r * Vl:(r + 1) * Vl].astype(np.int64))
    gi = torch.arange(r * Vl, (r + 1) * Vl).expand_as(sb)
    am = gi.gather(1, tp.argmax_rank(sb, gi).argmax(1, keepdim=True))
    top = gi.gather(1, tp.topk_rank(sb, gi).argsort(1, descending=True)[:, :k])
    vals = lambda idx: torch.from_numpy(bits[np.arange(bits.shape[0])[:, None], idx.numpy()].astype(np.int64))  # noqa: E731
    return vals(am)[:, 0], am[:, 0], vals(top), top


@pytest.mark.parametrize("seed", range(6))
def test_vocabulary_merge_equals_the_one_gpu_pick(seed):
    g = torch.Generator().manual_seed(seed)
    M, V, k, W = 3, 6000, 8, 2  # shard offset 3000: not aligned to the gather key's 32768 blocks
    x = (torch.randn(M, V, generator=g) * 2).round().bfloat16()  # many equal values
    x[:, 2990:3010] = x[:, 2990:2991]  # equal values straddling the shard boundary
    if seed % 2:
        x[:, ::11] = -0.0
    bits = x.view(torch.int16).numpy().view(np.uint16)
    cand = [_shard_candidates(bits, r, V // W, k) for r in range(W)]
    am, top = tp.merge_pick(torch.stack([c[2] for c in cand]), torch.stack([c[3] for c in cand]),
                            torch.stack([c[0] for c in cand]), torch.stack([c[1] for c in cand]), k)
    assert np.array_equal(am.numpy(), otk.argmax(bits))
    assert np.array_equal(top.numpy(), otk.topk(bits, k)[1])


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def _bf16_sum(parts):
    """The all-reduce of bf16 partials: their fp32 sum rounded to bf16 (two ranks: one addition)."""
    tot = np.zeros(parts[0].shape, dtype=np.float32)
    for p in parts:
        tot = (tot + bf16_bits_to_f32(p)).astype(np.float32)
    return f32_to_bf16_bits(tot)


def _rank(rank, world, port, out):
    import torch.distributed as dist
    os.environ.update(MASTER_ADDR="127.0.0.1", MASTER_PORT=str(port))
    dist.init_process_group("gloo", rank=rank, world_size=world)
    sys.path[:0] = [ROOT, os.path.join(ROOT, "comfy-mono-decode-xpu_b200")]
    from mono_b200 import tp as tpm
    H, I, M = 1024, 2048, 5
    gate, up, down = ow.gen_gptq(I, H, 11), ow.gen_gptq(I, H, 12), ow.gen_gptq(H, I, 13)
    o = ow.gen_gptq(H, 2048, 14)
    g = torch.Generator().manual_seed(7)
    x = f32_to_bf16_bits((torch.randn(M, H, generator=g) * 0.5).numpy())
    y = f32_to_bf16_bits((torch.randn(M, 2048, generator=g) * 0.5).numpy())
    ln = f32_to_bf16_bits((1 + 0.1 * torch.randn(H, generator=g)).numpy())
    allbf = torch.arange(65536, dtype=torch.int32).to(torch.int16).view(torch.bfloat16)
    lut = torch.nn.functional.silu(allbf.float()).bfloat16().view(torch.int16).numpy().view(np.uint16)
    # this rank's shards: gate / up rows, down columns; o_proj columns (heads)
    r0, r1 = tpm.split_range(I, rank, world)
    sg = (gate[0][r0:r1], gate[1][r0:r1])
    su = (up[0][r0:r1], up[1][r0:r1])
    sd = tuple(t.numpy() for t in tpm.gptq_cols(torch.from_numpy(down[0]), torch.from_numpy(down[1]), r0, r1))
    k0, k1 = tpm.split_range(2048, rank, world)
    so = tuple(t.numpy() for t in tpm.gptq_cols(torch.from_numpy(o[0]), torch.from_numpy(o[1]), k0, k1))
    mlp_part = ol.mlp_gptq(x, ln, 1e-6, sg, su, sd, lut, residual=(rank == 0))
    q, s = ow.act_quant(y[:, k0:k1])
    o_part = ow.gptq_linear(q, s, *so, residual=x if rank == 0 else None)
    gathered = [None] * world
    dist.all_gather_object(gathered, (mlp_part, o_part))
    if rank == 0:
        out["mlp_tp"] = _bf16_sum([p[0] for p in gathered])
        out["o_tp"] = _bf16_sum([p[1] for p in gathered])
        out["mlp_one"] = ol.mlp_gptq(x, ln, 1e-6, gate, up, down, lut)
        qf, sf = ow.act_quant(y)
        out["o_one"] = ow.gptq_linear(qf, sf, *o, residual=x)
    dist.barrier()
    dist.destroy_process_group()


def test_two_gloo_ranks_match_the_one_gpu_oracle():
    ctx = mp.get_context("spawn")
    manager = ctx.Manager()
    out = manager.dict()
    port = _port()
    procs = [ctx.Process(target=_rank, args=(r, 2, port, out)) for r in range(2)]
    for p in procs:
        p.start()
    for p in procs:
        p.join(300)
        assert p.exitcode == 0
    for name in ("mlp", "o"):
        a = bf16_bits_to_f32(out[name + "_tp"]).astype(np.float64)
        b = bf16_bits_to_f32(out[name + "_one"]).astype(np.float64)
        err = np.abs(a - b)
        bound = 2.0 ** -6 * np.abs(b) + 2.0 ** -6 * np.abs(b).max()
        assert (err <= bound).all(), (name, float((err / bound).max()))
