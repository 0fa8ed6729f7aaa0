"""Batched decode streams (mono_b200.streams) on the GPU: a batch of two streams built from two one-stream models
(the same weights; different KV caches, GDN states, lengths, next tokens and hidden rows) commits, step by step,
exactly the tokens the two models commit on their own, and leaves exactly their states (bit for bit: every kernel
of the batched step is row-wise or chunks a stream's context as it would alone). The steered case forces a
multi-token accept (GDN replay of several rows, KV slot moves)."""
import pytest
import torch

pytestmark = pytest.mark.gpu


def _cfg():
    from mono_b200.decoder import Qwen35Config
    return Qwen35Config(hidden=2048, inter=4096, vocab=32768, layers=4, heads=8, kv_heads=2, gdn_k_heads=8,
                        gdn_v_heads=16)


def _perturb(m, seed, shift):
    g = torch.Generator(device=m.dev).manual_seed(seed)

    def rnd(t, scale=1.0):
        t.copy_((torch.randn(t.shape, device=m.dev, generator=g) * scale).to(t.dtype))

    for L in m.layers:
        if "kc" in L:
            rnd(L["kc"])
            rnd(L["vc"])
        else:
            rnd(L["state"], 0.1)
            rnd(L["conv_state"])
    rnd(m.mtp["kc"])
    rnd(m.mtp["vc"])
    rnd(m.hidden)
    m.next_tok.copy_(torch.randint(0, m.cfg.vocab, m.next_tok.shape, device=m.dev, generator=g))
    m.st[0] -= shift  # a shorter committed prefix (and MTP KV) than stream 0's
    m.st[1] -= shift


@pytest.mark.parametrize("B,steered", [(2, False), (2, True), (4, True)])
def test_streams_equal_separate_models(cuda, B, steered):
    """B = 4: 32 verify rows (the W4A8 kernels' four-tile path, tiles in batches; two lm_head pick launches)."""
    from mono_b200.decoder import Qwen35W4A8
    from mono_b200.streams import Qwen35W4A8Streams
    cfg = _cfg()
    models = [Qwen35W4A8(cfg, cuda, prompt_len=96, gen_tokens=64) for _ in range(B)]
    for b in range(1, B):
        _perturb(models[b], 10 + b, 13 * b + 3)
    batch = Qwen35W4A8Streams.from_models(models)
    assert batch.streams == B
    for step in range(3):
        force = steered and step != 1
        rb = batch.step(steer=(lambda t: t[:, 0].copy_(batch.drafts[:, 1])) if force else None).clone()
        rs = []
        for m in models:
            rs.append(m.step(steer=(lambda t, m=m: t[0, 0].copy_(m.drafts[1])) if force else None).clone())
        torch.cuda.synchronize()
        for b in range(B):
            assert torch.equal(rb[b], rs[b]), (step, b, rb[b, :10].tolist(), rs[b][:10].tolist())
        if force:
            assert all(int(r[0]) >= 2 for r in rs)
    Hk = cfg.kv_heads
    for b, m in enumerate(models):
        assert torch.equal(batch.st[b], m.st) and torch.equal(batch.ctl[b], m.ctl)
        assert torch.equal(batch.next_tok[b], m.next_tok.view(-1))
        assert torch.equal(batch.hidden[b], m.hidden.view(1, -1))
        for L, Lm in zip(batch.layers, m.layers):
            if "kc" in L:
                assert torch.equal(L["kc"][:, b * Hk:(b + 1) * Hk], Lm["kc"])
                assert torch.equal(L["vc"][:, b * Hk:(b + 1) * Hk], Lm["vc"])
            else:
                assert torch.equal(L["state"][b], Lm["state"])
                assert torch.equal(L["conv_state"][b], Lm["conv_state"])
                for p in range(2):
                    for q in range(3):
                        assert torch.equal(L["saved"][p][q][b], Lm["saved"][p][q])
        assert torch.equal(batch.mtp["kc"][:, b * Hk:(b + 1) * Hk], m.mtp["kc"])
        assert torch.equal(batch.mtp["vc"][:, b * Hk:(b + 1) * Hk], m.mtp["vc"])


def test_batched_streams_replay_from_graphs(cuda):
    """The batch steps from its CUDA graphs as it does eagerly (the bench's and generate loop's path). The first
    step_graphed() call runs two eager steps before its first replay, so it is the eager batch's third step."""
    from mono_b200 import mtp_loop
    from mono_b200.streams import Qwen35W4A8Streams
    cfg = _cfg()
    a = Qwen35W4A8Streams(cfg, cuda, prompt_len=80, streams=2, gen_tokens=128)
    b = Qwen35W4A8Streams(cfg, cuda, prompt_len=80, streams=2, gen_tokens=128)
    eager = [a.step().clone() for _ in range(8)][2:]
    graphed = [b.step_graphed().clone() for _ in range(6)]
    torch.cuda.synchronize()
    for x, y in zip(eager, graphed):
        assert torch.equal(x, y)
    out = mtp_loop.generate_device_streams(b, 12)
    assert len(out) == 2 and all(len(o) == 12 for o in out)
    assert all(0 <= t < cfg.vocab for o in out for t in o)
    b.release_graphs()
