"""Independent decode streams batched on one GPU: every weight byte is read once per step for all of them.

B streams (B x 8 verify rows <= 32: B <= 4 with the 8-row tree) share one model's weights and run one step
together. Their state is stacked:

  attention KV caches [1, B * Hk, cap, 256]      stream b: kv heads [b Hk, (b + 1) Hk)
  MTP KV cache        [1, B * Hk, cap, 256]
  GDN conv / recurrent state [B, ...], replay buffers [B, 8, ...], ctl int32 [B, 26]
  loop counters st [B, 4], next token [B, 1], hidden row [B, 1, H], verify tokens [B, 8]

and every row-wise kernel takes the B x 8 verify rows (B draft rows) as one batch:

  W4A8 row linears and fused MLP    M = 8 B rows: one weight stream for all streams
  Q/K norm + RoPE + KV write        mono_qk_norm_rope_kv_streams (stream b's rows go to its caches)
  tree attention                    mono_tree_attention_streams (stream b's q heads over its kv heads, its length)
  GDN conv + delta                  mono_gdn_step_deferred_streams (grid y = stream)
  draft head projections            mono_gemv_bf16 at M = B
  lm_head picks                     mono_lmhead_pick at M = B (each draft, dst row per stream) and for the verify
                                    in launches of up to 16 rows (one lm_head read per 2 streams)
  GDN layer_pre + a | b projection  mono_rowlin_norm_ab_gptq at M = 8 B
  MTP draft / verify prep           mono_mtp_prep_draft_streams / mono_mtp_prep_verify_streams (one launch each)
  MTP accept                        one launch per stream (a few microseconds each)

Each stream's arithmetic is exactly its one-stream step's (row-wise kernels; attention chunks a stream's context as
it would alone), so a batch of B streams commits the same tokens and states as B separate Qwen35W4A8 models:
tests/test_streams_gpu.py checks this bit for bit.
"""
from __future__ import annotations

import torch

from . import _C
from .decoder import Qwen35W4A8, _bf

MAX_ROWS = 32  # verify rows of one batched step: the fused MLP's and the row linear's row limit
PICK_ROWS = 16  # rows of one lm_head pick launch


def _state_of(m):
    """A one-stream model's decode state (the tensors themselves, not copies)."""
    c = m.cfg
    attn = [L for i, L in enumerate(m.layers) if c.is_attn(i)]
    gdn = [L for i, L in enumerate(m.layers) if not c.is_attn(i)]
    return {"kc": [L["kc"] for L in attn], "vc": [L["vc"] for L in attn],
            "conv": [L["conv_state"] for L in gdn], "state": [L["state"] for L in gdn],
            "saved": [L["saved"] for L in gdn], "mkc": m.mtp["kc"], "mvc": m.mtp["vc"],
            "st": m.st.view(4), "ctl": m.ctl.view(26), "next_tok": m.next_tok.view(1), "hidden": m.hidden.view(-1)}


class Qwen35W4A8Streams(Qwen35W4A8):
    """B decode streams of one model on one device, stepped together (see the module docstring)."""

    def __init__(self, cfg, device, prompt_len: int, streams: int, gen_tokens: int = 512, seed: int = 0x5EED + 4,
                 draft_gemv: bool = True, state_seed: int | None = None):
        super().__init__(cfg, device, prompt_len, gen_tokens, seed, draft_gemv=draft_gemv)
        g = torch.Generator(device=self.dev).manual_seed(seed + 0x51 if state_seed is None else state_seed)
        states = [self._own_state()] + [self._fresh_state(g) for _ in range(streams - 1)]
        self._stack(states)

    @classmethod
    def from_models(cls, models):
        """A batch of the given one-stream models (built with the same weights): their current states are copied
        and stacked; the models themselves are left as they are."""
        base = models[0]
        obj = cls.__new__(cls)
        obj.__dict__.update(base.__dict__)
        obj.layers = [dict(L) for L in base.layers]  # own dicts: the stacked state must not replace base's
        obj.mtp = dict(base.mtp)
        obj._graphs = None
        obj._stack([_state_of(m) for m in models])
        return obj

    # ---- state --------------------------------------------------------------------------------------------
    def _own_state(self):
        return _state_of(self)

    def _fresh_state(self, g):
        """Another stream's state: the shapes of this model's, random caches and states, the same counters."""
        s = self._own_state()
        dev = self.dev

        def rnd(t, scale=1.0):
            return (torch.randn(t.shape, device=dev, generator=g) * scale).to(t.dtype)

        return {"kc": [rnd(t) for t in s["kc"]], "vc": [rnd(t) for t in s["vc"]],
                "conv": [rnd(t) for t in s["conv"]], "state": [rnd(t, 0.1) for t in s["state"]],
                "saved": [[tuple(torch.zeros_like(x) for x in p) for p in sv] for sv in s["saved"]],
                "mkc": rnd(s["mkc"]), "mvc": rnd(s["mvc"]), "st": s["st"].clone(), "ctl": torch.zeros_like(s["ctl"]),
                "next_tok": torch.randint(0, self.cfg.vocab, (1,), device=dev, generator=g),
                "hidden": _bf((self.cfg.hidden,), g, dev, 1.0)}

    def _stack(self, states):
        c, dev = self.cfg, self.dev
        B = len(states)
        R = self.tree["rows"]
        if B < 1 or B * R > MAX_ROWS:
            raise ValueError(f"{B} streams of {R} verify rows exceed {MAX_ROWS} rows a step")
        if B > 1 and R < 8:
            raise ValueError("batched drafts write 8-slot verify-token rows: the tree needs 8 rows")
        self.streams = B
        ja = jg = 0
        for i, L in enumerate(self.layers):
            if c.is_attn(i):
                L["kc"] = torch.cat([s["kc"][ja] for s in states], dim=1).contiguous()
                L["vc"] = torch.cat([s["vc"][ja] for s in states], dim=1).contiguous()
                ja += 1
            else:
                L["conv_state"] = torch.stack([s["conv"][jg] for s in states]).contiguous()
                L["state"] = torch.stack([s["state"][jg] for s in states]).contiguous()
                L["saved"] = [tuple(torch.stack([s["saved"][jg][p][q] for s in states]).contiguous() for q in range(3))
                              for p in range(2)]
                jg += 1
        self.mtp["kc"] = torch.cat([s["mkc"] for s in states], dim=1).contiguous()
        self.mtp["vc"] = torch.cat([s["mvc"] for s in states], dim=1).contiguous()
        self.st = torch.stack([s["st"] for s in states]).contiguous()
        self.ctl = torch.stack([s["ctl"] for s in states]).contiguous()
        self.next_tok = torch.stack([s["next_tok"] for s in states]).contiguous()          # [B, 1]
        self.hidden = torch.stack([s["hidden"] for s in states]).view(B, 1, -1).contiguous()
        i64, i32 = torch.int64, torch.int32
        self.result = torch.zeros(B, 32, dtype=i64, device=dev)
        self.apos = torch.empty(B, R, dtype=i64, device=dev)
        self.aseq = torch.empty(B, dtype=i32, device=dev)
        self.vpos = torch.empty(B, R, dtype=i64, device=dev)
        self.mpos = torch.empty(B, 1, dtype=i64, device=dev)
        self.mseq = torch.empty(B, dtype=i32, device=dev)
        self.mfreq = torch.empty(B, c.rotary_dim // 2, 2, 2, device=dev)
        self.drafts = torch.zeros(B, R, dtype=i64, device=dev)
        self.toks = torch.zeros(B, R, dtype=i64, device=dev)
        self.total = torch.zeros(1, dtype=i64, device=dev)
        # stream b's caches: kv heads [b Hk, (b + 1) Hk) of every stacked cache
        per = c.kv_heads * self.cap * c.head_dim * 2
        caches = [t for L in self.layers if "kc" in L for t in (L["kc"], L["vc"])]
        self.kv_ptrs = torch.tensor([[t.data_ptr() + b * per for t in caches] for b in range(B)], dtype=i64,
                                    device=dev)
        self.fused, self.programs = False, None

    # ---- layers --------------------------------------------------------------------------------------------
    def _kv_rows(self, v):
        """v rows [1, B R, Hk, 256] (stream-major, a view of the projection's rows) as the attention's tree values
        [B, Hk, R, 256]: a strided view, read in place by the kernel."""
        B = self.streams
        M, Hk, hd = v.shape[1], v.shape[2], v.shape[3]
        return v[0].view(B, M // B, Hk, hd).permute(0, 2, 1, 3)

    def _attention(self, L, x, freqs, i=-1):
        c, B = self.cfg, self.streams
        M = x.shape[0]
        hd = c.head_dim
        pre = _C.rowlin_gptq(x, _C.ROWLIN_NORM, [(L["q"], 2 * c.heads * hd), (L["k"], c.kv_heads * hd),
                                                 (L["v"], c.kv_heads * hd)], norm_w=L["ln1"], eps=c.eps)
        nq = 2 * c.heads * hd
        qg = pre[:, :nq].view(1, M, c.heads, 2 * hd)
        rawk = pre[:, nq:nq + c.kv_heads * hd].view(1, M, c.kv_heads, hd)
        v = pre[:, nq + c.kv_heads * hd:].view(1, M, c.kv_heads, hd)
        q, k = _C.qk_norm_rope_kv(qg[..., :hd], rawk, v, L["q_norm"], L["k_norm"], freqs, L["kc"], L["vc"],
                                  self.apos.view(-1), c.eps, c.eps, c.rotary_dim, streams=B)
        y = _C.attn_dpas(q, L["kc"], L["vc"], self.aseq, k, self._kv_rows(v), self.mask[:M // B], streams=B)
        x1 = _C.rowlin_gptq(y[0], _C.ROWLIN_GATE, [(L["o"], c.hidden)], gate=pre[:, hd:nq], gate_head_stride=2 * hd,
                            lut=self.sig_lut, residual=x)
        out = _C.mlp_gptq(x1, L["ln2"], c.eps, L["gate"], L["up"], L["down"], silu_lut=self.silu_lut, I=c.inter)
        self._t("attn", i, x=x, y=y, x1=x1, out=out)
        return out

    def _gdn(self, L, x, i=-1):
        c, B = self.cfg, self.streams
        HV, D = c.gdn_v_heads, c.gdn_dim
        Ck = 2 * c.gdn_k_heads * D + HV * D
        xn = torch.empty_like(x)
        ab = torch.empty((x.shape[0], L["wab"].shape[0]), dtype=torch.bfloat16, device=x.device)
        pre = _C.rowlin_gptq(x, _C.ROWLIN_NORM, [(L["qkv"], Ck), (L["z"], HV * D)], norm_w=L["ln1"], eps=c.eps,
                             xn_out=xn, ab=(L["wab"], ab))  # + the a | b projection of xn in the same launch
        prev, save = L["saved"][self.parity], L["saved"][1 - self.parity]
        core = _C.gdn_step_deferred(pre[:, :Ck], pre[:, Ck:], ab[:, :HV], ab[:, HV:], L["conv_w"], L["conv_state"],
                                    L["dt_bias"], L["g_decay"], L["state"], L["gnorm"], c.eps, D ** -0.5,
                                    c.gdn_k_heads, self.ctl, prev, save, streams=B)
        x1 = _C.rowlin_gptq(core, _C.ROWLIN_QUANT, [(L["out"], c.hidden)], residual=x)
        out = _C.mlp_gptq(x1, L["ln2"], c.eps, L["gate"], L["up"], L["down"], silu_lut=self.silu_lut, I=c.inter)
        self._t("gdn", i, x=x, core=core, out=out)
        return out

    # ---- the step ------------------------------------------------------------------------------------------
    def verify(self, tokens):
        """Every stream's tree rows ([B, R] tokens) through the body in one batch; returns (greedy tokens [B, R],
        final hidden rows [B R, H])."""
        c, B = self.cfg, self.streams
        _C.mtp_prep_verify_streams(self.st, self.apos, self.aseq, self.vpos, self.tree_pos, self.ctl, self.tree_ctl,
                                   self.parity, 0)  # every stream, one launch
        freqs = self.rope[self.vpos.view(-1).clamp(max=self.cap - 1)]
        x = self.embed[tokens.view(-1)]
        for i, L in enumerate(self.layers):
            x = self._attention(L, x, freqs, i) if c.is_attn(i) else self._gdn(L, x, i)
        xf = _C.rmsnorm_add(x, self.final_norm, c.eps)
        toks = self.toks.view(-1)
        for r0 in range(0, xf.shape[0], PICK_ROWS):
            self._pick(xf[r0:r0 + PICK_ROWS], 0, argmax_out=toks[r0:r0 + PICK_ROWS])
        self._t("verify", -1, tokens=tokens, x=x, xf=xf, toks=self.toks)
        return self.toks, x

    def draft_token(self, hidden, k):
        """Draft k of every stream (one row each): hidden [B, 1, H]; each stream's pick writes its node k's children
        in its verify-token row. Returns the MTP hidden rows [B, 1, H]."""
        c, m, B = self.cfg, self.mtp, self.streams
        hd, H = c.head_dim, c.hidden
        _C.mtp_prep_draft_streams(self.st, k, self.rope, self.mfreq, self.mpos, self.mseq)  # every stream, one launch
        cat = _C.draft_embed_norm_cat(self.embed, self.drafts, k, m["enorm"], hidden.view(B, -1), m["hnorm"], c.eps)
        x = self._linear(cat, m["fc"])
        qkv = self._linear(_C.rmsnorm_add(x, m["ln1"], c.eps), m["qkv"])
        nq = 2 * c.heads * hd
        qg = qkv[:, :nq].view(1, B, c.heads, 2 * hd)
        rawk = qkv[:, nq:nq + c.kv_heads * hd].view(1, B, c.kv_heads, hd)
        v = qkv[:, nq + c.kv_heads * hd:].view(1, B, c.kv_heads, hd)
        q, kk = _C.qk_norm_rope_kv(qg[..., :hd], rawk, v, m["q_norm"], m["k_norm"], self.mfreq, m["kc"], m["vc"],
                                   self.mpos.view(-1), c.eps, c.eps, c.rotary_dim, streams=B)
        y = _C.attn_dpas(q, m["kc"], m["vc"], self.mseq, kk, self._kv_rows(v), self.no_mask, streams=B)
        yg = _C.lut_mul(y[0], qkv[:, hd:nq], self.sig_lut, b_head_stride=2 * hd)
        xn, x = _C.rmsnorm_add(x, m["ln2"], c.eps, add=self._linear(yg, m["o"]))
        gu = self._linear(xn, m["gate_up"])
        h = _C.lut_mul(gu[:, c.inter:], gu[:, :c.inter], self.silu_lut)
        xf, x = _C.rmsnorm_add(x, m["norm"], c.eps, add=self._linear(h, m["down"]))
        self._pick(xf, c.tree[k], children=self.children[8 * k:8 * k + 8], dst=self.drafts, node=k)
        self._t("draft", k, xf=xf, drafts=self.drafts)
        return x.view(B, 1, -1)

    def step(self, steer=None):
        """One step of every stream, queued on the current stream. Returns the device result rows [B, 32] (each
        mono_mtp_accept's row). steer (tests): a callable given the verify tokens [B, R] before the accepts."""
        c, B = self.cfg, self.streams
        R = self.tree["rows"]
        self.drafts[:, 0] = self.next_tok.view(-1)
        h = self.hidden
        for k in range(c.depth):
            h = self.draft_token(h, k)
        toks, x = self.verify(self.drafts)
        if steer is not None:
            steer(toks)
        for b in range(B):
            _C.mtp_accept(self.st[b], toks[b:b + 1], self.drafts[b:b + 1], None, self.children, R, c.depth,
                          x[b * R:(b + 1) * R], self.next_tok[b:b + 1], self.hidden[b], self.ctl[b], self.kv_ptrs[b],
                          c.kv_heads, self.cap, c.head_dim, self.result[b])
        self.total += self.result[:, 0].sum()
        self.parity = 1 - self.parity
        return self.result

    def own_launches_per_step(self) -> int:
        c, B = self.cfg, self.streams
        n_attn = sum(1 for i in range(c.layers) if c.is_attn(i))
        n_gdn = c.layers - n_attn
        body = c.layers * 3 + n_gdn * 2 + n_attn * 2
        draft = c.depth * (1 + 1 + 1 + 1 + 2 + 3 + 1 + (5 if self.draft_gemv else 0))
        picks = -(-B * self.tree["rows"] // PICK_ROWS)
        return body + draft + 1 + 1 + picks + B  # prep_verify (all streams), final norm, lm_head picks, accepts

    def step_bytes(self) -> int:
        """Algorithmic HBM bytes of one batched step: the weights once, every stream's GDN states and KV prefix."""
        c, B = self.cfg, self.streams
        body = sum(t.numel() for L in self.layers for k, t in L.items()
                   if k in ("gate", "up", "down", "q", "k", "v", "o", "qkv", "z", "out"))
        small = sum(L[k].numel() * L[k].element_size() for L in self.layers for k in ("wab", "conv_w") if k in L)
        state = sum(L["state"].numel() * 4 * 2 for L in self.layers if "state" in L)  # all streams' states
        lm = self.lm_head.numel() * 2
        picks = -(-B * self.tree["rows"] // PICK_ROWS)  # verify lm_head reads
        mtp = sum(t.numel() * t.element_size() for k, t in self.mtp.items() if k not in ("kc", "vc"))
        kv = int(self.st[:, 0].sum().item()) * c.kv_heads * c.head_dim * 2 * 2 * sum(1 for L in self.layers
                                                                                      if "kc" in L)
        return body + small + state + lm * (picks + c.depth) + mtp * c.depth + kv
