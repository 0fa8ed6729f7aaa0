"""The tensor-parallel decoder (mono_b200.tp) on one GPU as a one-rank NCCL group: the sharded code path (the
all-reduce hooks, the vocabulary pick through the candidate merge, the host-side draft scatter) with a shard of
the whole model commits exactly the tokens of the plain decoder built with the same seed, step after step,
including the result rows, the next token and the hidden row. The two-rank run is bench.py --tp on 2 GPUs."""
import socket

import pytest
import torch

pytestmark = pytest.mark.gpu


def _port():
    s = socket.socket()
    s.bind(("127.0.0.1", 0))
    p = s.getsockname()[1]
    s.close()
    return p


def test_one_rank_tp_decoder_commits_the_plain_decoders_tokens(cuda):
    import torch.distributed as dist

    from mono_b200 import tp
    from mono_b200.decoder import Qwen35Config, Qwen35W4A8
    dist.init_process_group("nccl", init_method=f"tcp://127.0.0.1:{_port()}", rank=0, world_size=1,
                            device_id=torch.device("cuda", torch.cuda.current_device()))
    try:
        cfg = Qwen35Config(hidden=2048, inter=4096, vocab=32768, layers=4, heads=8, kv_heads=2, gdn_k_heads=8,
                           gdn_v_heads=16)
        plain = Qwen35W4A8(cfg, cuda, prompt_len=64, gen_tokens=64, seed=5)
        sharded = tp.make_decoder(cfg, cuda, dist.group.WORLD, 64, gen_tokens=64, seed=5)
        assert sharded.tp_world == 1 and sharded.tp_reduces_per_step() == 2 * 4 + 2 * cfg.depth
        for step in range(5):
            a = plain.step().clone()
            b = sharded.step().clone()
            torch.cuda.synchronize()
            assert torch.equal(a, b), (step, a[:12].tolist(), b[:12].tolist())
            assert torch.equal(plain.drafts, sharded.drafts) and torch.equal(plain.next_tok, sharded.next_tok)
            assert torch.equal(plain.hidden.view(torch.int16), sharded.hidden.view(torch.int16))
        # the graphed loop of the sharded decoder (collectives inside CUDA graphs)
        for _ in range(4):
            a = plain.step_graphed().clone()
            b = sharded.step_graphed().clone()
            torch.cuda.synchronize()
            assert torch.equal(a, b)
        plain.release_graphs()
        sharded.release_graphs()
    finally:
        dist.destroy_process_group()
