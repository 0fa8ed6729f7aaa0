"""The MTP decode step of the synthetic Qwen3.5-9B-shaped W4A8 model as torch-CPU eager operations (test
infrastructure: the CPU baseline and the reference arm of bench.py; see oracle/__init__.py).

The reference's own chain runs on XPU torch / oneDNN and cannot run here; this is its arithmetic restated as the
host's eager ops, on the host cores, following the build's CPU plan: every W4A8 linear is a per-token int8
quantization (absmax / 127, round half to even) and, per 128-group, an int8 x int8 -> int32 matmul
(torch._int_mm), then fp32 epilogues (group scale, chunk sums, the activation scale); the bf16 projections (MTP head,
lm_head, a|b) are torch bf16 linears; norms, RoPE, attention, the Gated-DeltaNet recurrence and the accept walk are
fp32 / integer torch code. One step = the draft tree (4 drafts of the MTP head + lm_head pick, top-2 per node of
tree4s1m8), the verify of the 8 tree rows through all layers with the tree mask, the lm_head argmax, the greedy
accept walk, and the replay of the accepted rows into the GDN states and the KV caches. Random-init weights of the
model's shapes (the same distributions as the GPU model; not the same values)."""
from __future__ import annotations

import math

import torch
import torch.nn.functional as F

from .mtp import accept_walk


class _Pool:
    """Random bytes for the int4 weights, made fast: one 64 MB block of uniform random bytes, from which each matrix
    takes a window at a random offset, XORed with a random byte (every matrix gets its own bytes, uniform)."""

    def __init__(self, g):
        self.g = g
        self.block = torch.randint(0, 256, (1 << 26,), dtype=torch.uint8, generator=g)

    def int4(self, n):
        out = torch.empty(n, dtype=torch.uint8)
        o, key = int(torch.randint(0, 1 << 26, (1,), generator=self.g)), int(torch.randint(0, 256, (1,), generator=self.g))
        done = 0
        while done < n:
            take = min(n - done, (1 << 26) - o)
            torch.bitwise_xor(self.block[o:o + take], key, out=out[done:done + take])
            done += take
            o = 0
        return (out & 15).view(torch.int8) - 8


class _W4:
    """GPTQ W4 weight for the CPU: int8 values in [-8, 7] laid out [G][128][N] (per group, K-major), fp32 scales
    [G][N]."""

    def __init__(self, N, K, g, pool):
        G = K // 128
        self.q = pool.int4(G * 128 * N).view(G, 128, N)
        self.s = (torch.randn(G, N, generator=g).abs() * (0.02 / 7) + 1e-4).half().float()
        self.N, self.K = N, K

    def nbytes_int4(self):
        return self.N * self.K // 2 + self.N * (self.K // 128) * 2


def _bf(shape, g, std=0.02, mean=0.0):
    return (torch.randn(*shape, generator=g) * std + mean).to(torch.bfloat16)


class CpuDecoder:
    def __init__(self, hidden=4096, inter=12288, vocab=151936, layers=32, attn_every=4, heads=16, kv_heads=4,
                 head_dim=256, rotary_dim=64, rope_theta=1e7, gdn_k_heads=16, gdn_v_heads=32, gdn_dim=128, eps=1e-6,
                 tree=(2, 2, 2, 1), prompt_len=1024, gen_tokens=256, seed=0x5EED + 4):
        g = torch.Generator().manual_seed(seed)
        pool = _Pool(g)
        self.H, self.I, self.V, self.eps = hidden, inter, vocab, eps
        self.heads, self.kvh, self.hd, self.rd = heads, kv_heads, head_dim, rotary_dim
        self.HK, self.HV, self.D = gdn_k_heads, gdn_v_heads, gdn_dim
        self.C = 2 * gdn_k_heads * gdn_dim + gdn_v_heads * gdn_dim
        self.cap = prompt_len + gen_tokens + 64
        H, I, hd = hidden, inter, head_dim
        self.embed = _bf((vocab, H), g)
        self.lm_head = _bf((vocab, H), g)
        self.final_norm = _bf((H,), g, 0.02, 1.0)
        self.layers = []
        for i in range(layers):
            L = {"attn": (i + 1) % attn_every == 0, "ln1": _bf((H,), g, 0.02, 1.0), "ln2": _bf((H,), g, 0.02, 1.0),
                 "gate": _W4(I, H, g, pool), "up": _W4(I, H, g, pool), "down": _W4(H, I, g, pool)}
            if L["attn"]:
                L.update(q=_W4(2 * heads * hd, H, g, pool), k=_W4(kv_heads * hd, H, g, pool), v=_W4(kv_heads * hd, H, g, pool),
                         o=_W4(H, heads * hd, g, pool), q_norm=_bf((hd,), g, 0.3, 1.0), k_norm=_bf((hd,), g, 0.3, 1.0),
                         kc=torch.randn(kv_heads, self.cap, hd, generator=g).bfloat16(),
                         vc=torch.randn(kv_heads, self.cap, hd, generator=g).bfloat16())
            else:
                HV, Dg = gdn_v_heads, gdn_dim
                L.update(qkv=_W4(self.C, H, g, pool), z=_W4(HV * Dg, H, g, pool), out=_W4(H, HV * Dg, g, pool), wab=_bf((2 * HV, H), g),
                         conv_w=_bf((self.C, 4), g, 0.5), conv_state=_bf((self.C, 3), g, 1.0),
                         dt_bias=torch.zeros(HV), g_decay=-torch.ones(HV), gnorm=_bf((Dg,), g, 0.1, 1.0),
                         state=torch.randn(HV, Dg, Dg, generator=g) * 0.1, saved=None)
            self.layers.append(L)
        self.mtp = {"enorm": _bf((H,), g, 0.02, 1.0), "hnorm": _bf((H,), g, 0.02, 1.0), "fc": _bf((H, 2 * H), g),
                    "ln1": _bf((H,), g, 0.02, 1.0), "qkv": _bf((2 * heads * hd + 2 * kv_heads * hd, H), g),
                    "o": _bf((H, heads * hd), g), "q_norm": _bf((hd,), g, 0.3, 1.0), "k_norm": _bf((hd,), g, 0.3, 1.0),
                    "ln2": _bf((H,), g, 0.02, 1.0), "gate_up": _bf((2 * I, H), g), "down": _bf((H, I), g),
                    "norm": _bf((H,), g, 0.02, 1.0),
                    "kc": torch.randn(kv_heads, self.cap, hd, generator=g).bfloat16(),
                    "vc": torch.randn(kv_heads, self.cap, hd, generator=g).bfloat16()}
        half = rotary_dim // 2
        inv = 1.0 / (rope_theta ** (torch.arange(half, dtype=torch.float64) * 2 / rotary_dim))
        ang = torch.arange(self.cap, dtype=torch.float64)[:, None] * inv[None, :]
        self.cos, self.sin = torch.cos(ang).float(), torch.sin(ang).float()
        # the verify tree (tree4s1m8 for (2, 2, 2, 1)): chain node k has tree[k] children, the first continuing
        self.tree = tree
        spec = []
        for w in reversed(tree):
            spec = [spec] + [[] for _ in range(w - 1)]
        self.parents, self.depth_of = [], []

        def add(node, p):
            r = len(self.parents)
            self.parents.append(p)
            self.depth_of.append(0 if p < 0 else self.depth_of[p] + 1)
            for child in node:
                add(child, r)
        add(spec, -1)
        self.R = len(self.parents)
        self.children = [[] for _ in range(self.R)]
        for r in range(1, self.R):
            self.children[self.parents[r]].append(r)
        self.mask = []
        for r in range(self.R):
            self.mask.append((self.mask[self.parents[r]] if self.parents[r] >= 0 else 0) | (1 << r))
        self.pos, self.mpos = prompt_len, prompt_len
        self.next_tok = int(torch.randint(0, vocab, (1,), generator=g))
        self.hidden = _bf((H,), g, 1.0)

    # ---- pieces --------------------------------------------------------------------------------------------
    def rms(self, x, w):
        xf = x.float()
        return (xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + self.eps) * w.float()).bfloat16()

    def w4a8(self, x, W: _W4, residual=None):
        """Per-token int8 quant, per-group int8 matmuls (int32), fp32 epilogue in chunk order, bf16 out."""
        xf = x.float()
        s = xf.abs().amax(-1, keepdim=True) / 127.0
        q = torch.where(s > 0, torch.round(xf / torch.where(s > 0, s, torch.ones_like(s))), torch.zeros_like(xf))
        q = q.clamp(-127, 127).to(torch.int8)
        M, G = q.shape[0], W.q.shape[0]
        qg = q.view(M, G, 128).transpose(0, 1).contiguous()
        total = torch.zeros(M, W.N)
        for c in range(G // 8):
            Fc = torch.zeros(M, W.N)
            for gi in range(c * 8, c * 8 + 8):
                Fc += torch._int_mm(qg[gi], W.q[gi]).float() * W.s[gi]
            total += Fc
        out = (total * s).bfloat16()
        return out if residual is None else (residual.float() + out.float()).bfloat16()

    def mlp(self, x, L):
        q = self.rms(x, L["ln2"])
        g, u = self.w4a8(q, L["gate"]), self.w4a8(q, L["up"])
        h = (F.silu(g.float()).bfloat16().float() * u.float()).bfloat16()
        return self.w4a8(h, L["down"], residual=x)

    def head_norm(self, t, w):
        tf = t.float()
        return (tf * torch.rsqrt(tf.pow(2).mean(-1, keepdim=True) + self.eps) * w.float()).bfloat16()

    def rope(self, t, pos):
        """split-half rotation of the first rd dims at positions pos [S]; t [S, heads, hd] bf16."""
        half = self.rd // 2
        c, s = self.cos[pos][:, None, :], self.sin[pos][:, None, :]
        tf = t.float()
        lo, hi = tf[..., :half], tf[..., half:self.rd]
        out = tf.clone()
        out[..., :half] = lo * c - hi * s
        out[..., half:self.rd] = hi * c + lo * s
        return out.bfloat16()

    def attend(self, q, kc, vc, L, k, v, mask):
        """q [S, Hq, hd], caches [Hk, cap, hd], this step's k / v [S, Hk, hd]; prefix [0, L) + the masked rows."""
        S, Hq, hd = q.shape
        grp = Hq // self.kvh
        out = torch.zeros(S, Hq * hd)
        for s in range(S):
            rows = [t for t in range(S) if (mask[s] >> t) & 1] if mask is not None else []
            for kh in range(self.kvh):
                K = torch.cat([kc[kh, :L].float(), k[rows, kh].float()])
                Vv = torch.cat([vc[kh, :L].float(), v[rows, kh].float()])
                sc = q[s, kh * grp:(kh + 1) * grp].float() @ K.T / math.sqrt(hd)
                p = torch.softmax(sc, -1)
                out[s, kh * grp * hd:(kh + 1) * grp * hd] = (p.bfloat16().float() @ Vv).reshape(-1)
        return out.bfloat16()

    def attention_layer(self, x, L, pos_rows, mask):
        R, hd, Hq = x.shape[0], self.hd, self.heads
        nq, nkv = 2 * Hq * hd, self.kvh * hd
        xn = self.rms(x, L["ln1"])
        pre = torch.cat([self.w4a8(xn, L["q"]), self.w4a8(xn, L["k"]), self.w4a8(xn, L["v"])], -1)
        qg = pre[:, :nq].view(R, Hq, 2 * hd)
        q = self.rope(self.head_norm(qg[..., :hd], L["q_norm"]), pos_rows)
        k = self.rope(self.head_norm(pre[:, nq:nq + nkv].view(R, self.kvh, hd), L["k_norm"]), pos_rows)
        v = pre[:, nq + nkv:].view(R, self.kvh, hd)
        for s in range(R):  # the verify rows' cache slots: pos + s
            L["kc"][:, self.pos + s] = k[s]
            L["vc"][:, self.pos + s] = v[s]
        y = self.attend(q, L["kc"], L["vc"], self.pos, k, v, mask)
        yg = (y.float() * torch.sigmoid(qg[..., hd:].reshape(R, -1).float()).bfloat16().float()).bfloat16()
        x1 = self.w4a8(yg, L["o"], residual=x)
        return self.mlp(x1, L)

    def _gdn_conv_gates(self, L, raw_rows, ab, parents, hist):
        """conv outputs of rows along their ancestry (parents; -1 = the committed history hist [C, 3])."""
        w = L["conv_w"].float()
        out = []
        for t in range(raw_rows.shape[0]):
            taps, anc, miss = [raw_rows[t].float()], t, 0
            for d in range(1, 4):
                anc = parents[anc] if anc >= 0 else -1
                if anc >= 0:
                    taps.append(raw_rows[anc].float())
                else:
                    miss += 1
                    taps.append(hist[:, 3 - miss].float())
            y = sum(taps[d] * w[:, 3 - d] for d in range(4)).bfloat16().float()
            out.append((y / (1 + torch.exp(-y))).bfloat16().float())
        conv = torch.stack(out)
        HV = self.HV
        av = ab[:, :HV].float() + L["dt_bias"]
        decay = torch.exp(L["g_decay"] * F.softplus(av))
        beta = torch.sigmoid(ab[:, HV:].float()).bfloat16().float()
        return conv, decay, beta

    def _delta(self, S, conv, decay, beta, entries):
        """entries: list of (row, commit); returns raw [rows, HV, D] for the rows named and the new S."""
        KD, HV, D = self.HK * self.D, self.HV, self.D
        q = conv[:, :KD].view(-1, self.HK, D)
        k = conv[:, KD:2 * KD].view(-1, self.HK, D)
        v = conv[:, 2 * KD:].view(-1, HV, D)
        qn = q * D ** -0.5 / q.norm(dim=-1, keepdim=True).clamp(min=1e-12)
        kn = k / k.norm(dim=-1, keepdim=True).clamp(min=1e-12)
        rep = HV // self.HK
        raw = torch.zeros(conv.shape[0], HV, D)
        for t, commit in entries:
            kk, qq = kn[t].repeat_interleave(rep, 0), qn[t].repeat_interleave(rep, 0)  # [HV, D]
            St = S * decay[t][:, None, None]
            mem = torch.einsum("hkv,hk->hv", St, kk)
            dl = (v[t] - mem) * beta[t][:, None]
            St = St + kk[:, :, None] * dl[:, None, :]
            raw[t] = torch.einsum("hkv,hk->hv", St, qq)
            if commit:
                S = St
        return raw, S

    def gdn_layer(self, x, L):
        R, HV, D = x.shape[0], self.HV, self.D
        xn = self.rms(x, L["ln1"])
        qkv, z = self.w4a8(xn, L["qkv"]), self.w4a8(xn, L["z"])
        ab = F.linear(xn, L["wab"])
        L["saved"] = (qkv, ab)
        conv, decay, beta = self._gdn_conv_gates(L, qkv, ab, self.parents, L["conv_state"])
        entries, node = [], 0
        while True:  # the verify program: chain nodes commit, leaves follow their parent
            entries.append((node, True))
            kids = self.children[node]
            entries.extend((leaf, False) for leaf in kids[1:])
            if not kids:
                break
            node = kids[0]
        raw, _ = self._delta(L["state"], conv, decay, beta, entries)
        rawb = raw.bfloat16().float()
        normed = (rawb * L["gnorm"].float() * torch.rsqrt(rawb.pow(2).mean(-1, keepdim=True) + self.eps)).bfloat16()
        zf = z.float().view(R, HV, D)
        core = (normed.float() * (zf / (1 + torch.exp(-zf))).bfloat16().float()).bfloat16().view(R, HV * D)
        x1 = self.w4a8(core, L["out"], residual=x)
        return self.mlp(x1, L)

    def gdn_commit(self, L, path):
        """The accepted rows into the conv state and the recurrent state (the replay, as a chain)."""
        qkv, ab = L["saved"]
        rows = qkv[path]
        chain = [-1] + list(range(len(path) - 1))
        conv, decay, beta = self._gdn_conv_gates(L, rows, ab[path], chain, L["conv_state"])
        _, L["state"] = self._delta(L["state"], conv, decay, beta, [(t, True) for t in range(len(path))])
        seq = torch.cat([L["conv_state"], rows.T], 1)
        L["conv_state"] = seq[:, -3:].contiguous()

    def lm_pick(self, x, k):
        lg = F.linear(x, self.lm_head)  # bf16 logits
        am = lg.float().argmax(-1)
        top = lg.float().topk(k, -1).indices if k > 1 else am[:, None]
        return am, top

    def draft(self, tok, hidden):
        m, H, hd = self.mtp, self.H, self.hd
        cat = torch.cat([self.rms(self.embed[tok][None], m["enorm"]), self.rms(hidden[None], m["hnorm"])], -1)
        x = F.linear(cat, m["fc"])
        qkv = F.linear(self.rms(x, m["ln1"]), m["qkv"])
        nq, nkv = 2 * self.heads * hd, self.kvh * hd
        qg = qkv[:, :nq].view(1, self.heads, 2 * hd)
        pos = torch.tensor([self.mpos])
        q = self.rope(self.head_norm(qg[..., :hd], m["q_norm"]), pos)
        k = self.rope(self.head_norm(qkv[:, nq:nq + nkv].view(1, self.kvh, hd), m["k_norm"]), pos)
        v = qkv[:, nq + nkv:].view(1, self.kvh, hd)
        m["kc"][:, self.mpos] = k[0]
        m["vc"][:, self.mpos] = v[0]
        y = self.attend(q, m["kc"], m["vc"], self.mpos + 1, k, v, None)
        yg = (y.float() * torch.sigmoid(qg[..., hd:].reshape(1, -1).float()).bfloat16().float()).bfloat16()
        x = (x.float() + F.linear(yg, m["o"]).float()).bfloat16()
        gu = F.linear(self.rms(x, m["ln2"]), m["gate_up"])
        h = (F.silu(gu[:, :self.I].float()).bfloat16().float() * gu[:, self.I:].float()).bfloat16()
        x = (x.float() + F.linear(h, m["down"]).float()).bfloat16()
        return self.rms(x, m["norm"]), x[0]

    # ---- one step ------------------------------------------------------------------------------------------
    def step(self):
        """Draft tree, verify, accept, replay. Returns the committed tokens."""
        verify = [0] * self.R
        verify[0] = self.next_tok
        h = self.hidden
        for kd in range(len(self.tree)):
            xf, h = self.draft(verify[kd], h)
            self.mpos += 1
            am, top = self.lm_pick(xf, self.tree[kd])
            kids = self.children[kd]
            verify[kids[0]] = int(am[0])
            for j, c in enumerate(kids[1:], 1):
                verify[c] = int(top[0, j])
        self.mpos -= len(self.tree)
        x = self.embed[torch.tensor(verify)]
        pos_rows = torch.tensor([self.pos + d for d in self.depth_of])
        for L in self.layers:
            x = self.attention_layer(x, L, pos_rows, self.mask) if L["attn"] else self.gdn_layer(x, L)
        toks, _ = self.lm_pick(self.rms(x, self.final_norm), 1)
        toks = toks.tolist()
        path, commit, _, row, on_chain, kept = accept_walk(self.children, toks, verify, len(self.tree), None)
        for L in self.layers:
            if L["attn"] and not on_chain:
                for kk in range(1, len(path)):
                    if path[kk] != kk:
                        L["kc"][:, self.pos + kk] = L["kc"][:, self.pos + path[kk]]
                        L["vc"][:, self.pos + kk] = L["vc"][:, self.pos + path[kk]]
            elif not L["attn"]:
                self.gdn_commit(L, path)
        self.pos += len(path)
        self.mpos += kept
        self.next_tok, self.hidden = toks[row], x[row].clone()
        return commit

    def step_bytes(self):
        """The weight bytes one step reads (int4 body, bf16 lm_head x 5, bf16 MTP block x 4)."""
        body = sum(w.nbytes_int4() for L in self.layers for key, w in L.items() if isinstance(w, _W4))
        mtp = sum(t.numel() * 2 for key, t in self.mtp.items() if key not in ("kc", "vc"))
        return body + self.lm_head.numel() * 2 * (1 + len(self.tree)) + mtp * len(self.tree)
