"""Synthetic Qwen3.5-9B-shaped W4A8 decoder on the B200 kernels, with the device-side MTP loop.

Random-init weights of the model's architecture (no checkpoint is available): 32 layers in a 3:1 Gated-DeltaNet :
full-attention pattern, hidden 4096, MLP 12288, vocab 151936, bf16 embedding and lm_head ~ N(0, 0.02), every body
projection GPTQ W4A8 (int4 uniform in [-8, 7], fp16 group-128 scales |N(0,1)| * 0.02 / 7 + 1e-4), a 1-layer bf16 MTP
head. One decode step of one stream, queued without any host read-back (the reference's device MTP loop,
comfy_mono_decode_xpu/mtp_loop.py:270-341):

  draft    a depth-4 top-k tree of 8 nodes (the reference test's tree4s1m8 spec, tests/test_mtp_accept.py:46-47: the
           chain 0-1-2-3-4 and one sibling beside each of nodes 1, 2, 3): draft k (k = 0..3) runs the MTP head on
           chain node k's token and the previous draft's hidden row; its lm_head pick (the bf16 lm_head, fused with
           the argmax and top-2: mono_lmhead_pick) writes the argmax into the first child's verify token and the
           second-best into the second child's (the reference's draft pick, csrc/draft_lmhead.sycl:4-17)
  verify   the 8 tree rows through the 32 layers (layer_pre / attention or GDN / layer_post / MLP), with the tree
           attention mask, the GDN verify tree (parents and program in the ctl row), final norm, lm_head + argmax
  accept   mono_mtp_accept: the greedy accept walk over the tree, the counters, the GDN replay ctl, the KV slot moves
           of an off-chain path, next token and hidden row (all on the device)

Per layer: full attention = rowlin(norm -> q|k|v) -> qk_norm_rope_kv -> tree attention -> rowlin(gate -> o_proj +
residual) -> fused MLP; GDN = rowlin(norm -> qkv|z, xn, + the a|b projection of xn on the launch's last CTAs:
mono_rowlin_norm_ab_gptq) -> deferred GDN step -> rowlin(quant -> out_proj + residual) -> fused MLP. The MTP head's five bf16 projections run on this build's bf16
GEMV (mono_gemv_bf16; cuBLAS through torch's F.linear with draft_gemv=False); its norms and gates are the row kernels
(mono_rmsnorm_add, mono_lut_mul).
"""
from __future__ import annotations

import math
from dataclasses import dataclass

import torch
import torch.nn.functional as F

from . import _C
from ._C import ROWS_GATE, ROWS_GDN, ROWS_NORM


@dataclass
class Qwen35Config:
    hidden: int = 4096
    inter: int = 12288
    vocab: int = 151936
    layers: int = 32
    attn_every: int = 4          # layers 3, 7, ..., 31 are full attention (3:1 GDN : attention)
    heads: int = 16
    kv_heads: int = 4
    head_dim: int = 256
    rotary_dim: int = 64
    rope_theta: float = 1e7
    gdn_k_heads: int = 16
    gdn_v_heads: int = 32
    gdn_dim: int = 128
    eps: float = 1e-6
    tree: tuple = (2, 2, 2, 1)   # children per chain node (tree4s1m8: depth 4, 8 verify rows); (1, 1, 1, 1): chain

    @property
    def depth(self) -> int:      # MTP drafts per step = the tree's chain depth
        return len(self.tree)

    def is_attn(self, i: int) -> bool:
        return (i + 1) % self.attn_every == 0


def _w4(N, K, g, dev, keep=None, name=None):
    """A random GPTQ W4 matrix (BASELINE configs[0] distributions) in the TILED layout. keep (a dict): also keep
    the checkpoint-layout packed / scales under `name` (for tests)."""
    packed = torch.randint(0, 256, (N, K // 2), dtype=torch.uint8, device=dev, generator=g)
    scales = (torch.randn(N, K // 128, device=dev, generator=g).abs() * (0.02 / 7) + 1e-4).half()
    t = _C.w4_repack(0, packed, scales, N, K)
    if keep is not None:
        keep[name] = (packed, scales)
    return t


def _bf(shape, g, dev, std=0.02, mean=0.0):
    return (torch.randn(*shape, device=dev, generator=g) * std + mean).to(torch.bfloat16)


def _rms(x, w, eps):
    xf = x.float()
    return ((xf * torch.rsqrt(xf.pow(2).mean(-1, keepdim=True) + eps)) * w.float()).to(torch.bfloat16)


def rope_table(cfg: Qwen35Config, cap: int, dev):
    """[cap, rd/2, 2, 2] fp32 split-half rotation per position: [[cos, -sin], [sin, cos]] (theta 1e7)."""
    half = cfg.rotary_dim // 2
    inv = 1.0 / (cfg.rope_theta ** (torch.arange(half, dtype=torch.float64) * 2 / cfg.rotary_dim))
    ang = torch.arange(cap, dtype=torch.float64)[:, None] * inv[None, :]
    c, s = torch.cos(ang), torch.sin(ang)
    return torch.stack([torch.stack([c, -s], -1), torch.stack([s, c], -1)], -2).float().to(dev).contiguous()


def verify_tree(widths):
    """The verify tree of a draft: chain node k (k = 0 .. len(widths) - 1) has widths[k] children, the first one
    continuing the chain, the others leaves (the shape qwen35's tree_spec builds; (2, 2, 2, 1) is the reference
    test's tree4s1m8). Rows are numbered depth-first, first child first (tests/test_mtp_accept.py:15-35 _tree).
    Returns rows, parents, children [8][8] (-1 padded), depth, attention mask (mask[r] = mask[parent] | 1 << r),
    and the GDN verify program (chain nodes commit, leaves follow their parent)."""
    spec = []
    for w in reversed(widths):
        spec = [spec] + [[] for _ in range(w - 1)]
    parents, depth = [], []

    def add(node, p):
        r = len(parents)
        parents.append(p)
        depth.append(0 if p < 0 else depth[p] + 1)
        for child in node:
            add(child, r)
    add(spec, -1)
    rows = len(parents)
    if rows > 8:
        raise ValueError(f"tree of {rows} rows: at most 8 verify rows")
    children = [[-1] * 8 for _ in range(8)]
    for r in range(1, rows):
        ch = children[parents[r]]
        ch[ch.index(-1)] = r
    mask = []
    for r in range(rows):
        mask.append((mask[parents[r]] if parents[r] >= 0 else 0) | (1 << r))
    # the GDN program: walk the chain, each chain node committing and followed by its leaves
    program, node = [], 0
    while True:
        program.append(node | 32)
        kids = [c for c in children[node] if c >= 0]
        program.extend(kids[1:])
        if not kids:
            break
        node = kids[0]
    return {"rows": rows, "parents": parents + [-1] * (8 - rows), "children": children, "depth": depth,
            "mask": mask, "program": program + [-1] * (8 - len(program)), "chain": len(widths)}


class Qwen35W4A8:
    """Weights and decode state of one stream on one device."""

    def __init__(self, cfg: Qwen35Config, device, prompt_len: int, gen_tokens: int = 512, seed: int = 0x5EED + 4,
                 fused: bool = False, prefetch: int = 0, draft_gemv: bool = True, keep_sources: bool = False):
        self.cfg, self.dev = cfg, torch.device(device)
        c, dev = cfg, self.dev
        g = torch.Generator(device=dev).manual_seed(seed)
        # keep_sources: the checkpoint-layout W4 weights too (w4_src[(layer, name)] = (packed, scales)), for checks
        # against the CPU oracle; trace: a callable(name, layer, tensors) the layer code reports to (None: off)
        self.w4_src = {} if keep_sources else None
        self.trace = None
        H, I, hd = c.hidden, c.inter, c.head_dim
        self.cap = ((prompt_len + gen_tokens + 64) + 63) // 64 * 64
        self.embed = _bf((c.vocab, H), g, dev)
        self.lm_head = _bf((c.vocab, H), g, dev)  # shared by the verify and the drafts (configs[4]: bf16)
        self.final_norm = _bf((H,), g, dev, 0.02, 1.0)
        self.layers = []
        Ck = 2 * c.gdn_k_heads * c.gdn_dim + c.gdn_v_heads * c.gdn_dim
        for i in range(c.layers):
            kp = self.w4_src
            L = {"ln1": _bf((H,), g, dev, 0.02, 1.0), "ln2": _bf((H,), g, dev, 0.02, 1.0),
                 "gate": _w4(I, H, g, dev, kp, (i, "gate")), "up": _w4(I, H, g, dev, kp, (i, "up")),
                 "down": _w4(H, I, g, dev, kp, (i, "down"))}
            if c.is_attn(i):
                L.update(q=_w4(2 * c.heads * hd, H, g, dev, kp, (i, "q")), k=_w4(c.kv_heads * hd, H, g, dev, kp, (i, "k")),
                         v=_w4(c.kv_heads * hd, H, g, dev, kp, (i, "v")), o=_w4(H, c.heads * hd, g, dev, kp, (i, "o")),
                         q_norm=_bf((hd,), g, dev, 0.3, 1.0), k_norm=_bf((hd,), g, dev, 0.3, 1.0),
                         kc=torch.randn(1, c.kv_heads, self.cap, hd, device=dev, generator=g).to(torch.bfloat16),
                         vc=torch.randn(1, c.kv_heads, self.cap, hd, device=dev, generator=g).to(torch.bfloat16))
            else:
                HV = c.gdn_v_heads
                L.update(qkv=_w4(Ck, H, g, dev, kp, (i, "qkv")), z=_w4(HV * c.gdn_dim, H, g, dev, kp, (i, "z")),
                         out=_w4(H, HV * c.gdn_dim, g, dev, kp, (i, "out")),
                         wab=_bf((2 * HV, H), g, dev), conv_w=_bf((Ck, 4), g, dev, 0.5),
                         conv_state=_bf((Ck, 3), g, dev, 1.0), dt_bias=torch.zeros(HV, device=dev),
                         g_decay=-torch.ones(HV, device=dev), gnorm=_bf((c.gdn_dim,), g, dev, 0.1, 1.0),
                         state=(torch.randn(HV, c.gdn_dim, c.gdn_dim, device=dev, generator=g) * 0.1).contiguous(),
                         saved=[(torch.zeros(8, Ck, dtype=torch.bfloat16, device=dev),
                                 torch.zeros(8, HV, dtype=torch.bfloat16, device=dev),
                                 torch.zeros(8, HV, dtype=torch.bfloat16, device=dev)) for _ in range(2)])
            self.layers.append(L)
        # MTP head (bf16): fc 2H -> H, one full-attention layer with its own KV cache, MLP
        self.mtp = {"enorm": _bf((H,), g, dev, 0.02, 1.0), "hnorm": _bf((H,), g, dev, 0.02, 1.0),
                    "fc": _bf((H, 2 * H), g, dev), "ln1": _bf((H,), g, dev, 0.02, 1.0),
                    "qkv": _bf((2 * c.heads * hd + 2 * c.kv_heads * hd, H), g, dev),
                    "o": _bf((H, c.heads * hd), g, dev), "q_norm": _bf((hd,), g, dev, 0.3, 1.0),
                    "k_norm": _bf((hd,), g, dev, 0.3, 1.0), "ln2": _bf((H,), g, dev, 0.02, 1.0),
                    "gate_up": _bf((2 * I, H), g, dev), "down": _bf((H, I), g, dev), "norm": _bf((H,), g, dev, 0.02, 1.0),
                    "kc": torch.randn(1, c.kv_heads, self.cap, hd, device=dev, generator=g).to(torch.bfloat16),
                    "vc": torch.randn(1, c.kv_heads, self.cap, hd, device=dev, generator=g).to(torch.bfloat16)}
        self.rope = rope_table(c, self.cap, dev)
        self.silu_lut, self.sig_lut = _C.act_luts(dev)
        # device loop state: st = [committed length, MTP KV length, 0, 0]; ctl of the GDN replay
        self.st = torch.tensor([prompt_len, prompt_len, 0, 0], dtype=torch.int64, device=dev)
        self.ctl = torch.zeros(26, dtype=torch.int32, device=dev)
        self.next_tok = torch.randint(0, c.vocab, (1, 1), device=dev, generator=g)
        self.hidden = _bf((1, 1, H), g, dev, 1.0)
        self.parity = 0
        tree = verify_tree(c.tree)
        R = tree["rows"]
        self.tree = tree
        self.children = torch.tensor(tree["children"], dtype=torch.int32).reshape(-1).to(dev)
        self.mask = torch.tensor(tree["mask"], dtype=torch.int32, device=dev)
        self.tree_pos = torch.tensor(tree["depth"], dtype=torch.int64, device=dev)
        self.tree_ctl = torch.tensor(tree["parents"] + tree["program"], dtype=torch.int32, device=dev)
        self.result = torch.zeros(32, dtype=torch.int64, device=dev)
        self.apos = torch.empty(8, dtype=torch.int64, device=dev)
        self.aseq = torch.empty(1, dtype=torch.int32, device=dev)
        self.vpos = torch.empty(1, R, dtype=torch.int64, device=dev)
        self.mpos = torch.empty(8, dtype=torch.int64, device=dev)
        self.mseq = torch.empty(1, dtype=torch.int32, device=dev)
        self.mfreq = torch.empty(1, self.cfg.rotary_dim // 2, 2, 2, device=dev)
        self.kv_ptrs = torch.tensor([t.data_ptr() for L in self.layers if "kc" in L for t in (L["kc"], L["vc"])],
                                    dtype=torch.int64, device=dev)
        self.drafts = torch.zeros(R, dtype=torch.int64, device=dev)  # the verify tokens of the tree's rows
        self.toks = torch.zeros(1, R, dtype=torch.int64, device=dev)
        self.no_mask = torch.empty(0, dtype=torch.int32, device=dev)
        self.total = torch.zeros(1, dtype=torch.int64, device=dev)  # tokens committed, summed on the device
        self.fused, self.prefetch, self.draft_gemv = fused, prefetch, draft_gemv
        self.programs = self._build_programs() if fused else None

    # ---- hooks of the tensor-parallel variant (mono_b200.tp): identities on one GPU --------------------------
    def _residual(self, r):
        """The residual a row-sharded projection adds: every rank but 0 adds none (None / False)."""
        return r

    def _reduce(self, t):
        """The sum of a row-sharded projection's partial outputs over the ranks (in place)."""
        return t

    def _pick(self, xf, k, argmax_out=None, children=None, dst=None, node=0):
        """The lm_head pick of the normed rows xf: the verify's argmax (argmax_out), or a draft's pick into dst."""
        _C.lmhead_pick(xf, self.lm_head, k=k, argmax_out=argmax_out, children=children, dst=dst)

    def _t(self, name, layer, **tensors):
        if self.trace is not None:
            self.trace(name, layer, {k: v.clone() for k, v in tensors.items()})

    # ---- layers ------------------------------------------------------------------------------------------
    def _attention(self, L, x, freqs, i=-1):
        c = self.cfg
        M = x.shape[0]
        hd = c.head_dim
        pre = _C.rowlin_gptq(x, _C.ROWLIN_NORM, [(L["q"], 2 * c.heads * hd), (L["k"], c.kv_heads * hd),
                                                 (L["v"], c.kv_heads * hd)], norm_w=L["ln1"], eps=c.eps)
        nq = 2 * c.heads * hd
        qg = pre[:, :nq].view(1, M, c.heads, 2 * hd)
        rawk = pre[:, nq:nq + c.kv_heads * hd].view(1, M, c.kv_heads, hd)
        v = pre[:, nq + c.kv_heads * hd:].view(1, M, c.kv_heads, hd)
        q, k = _C.qk_norm_rope_kv(qg[..., :hd], rawk, v, L["q_norm"], L["k_norm"], freqs, L["kc"], L["vc"],
                                  self.apos, c.eps, c.eps, c.rotary_dim)
        y = _C.attn_dpas(q, L["kc"], L["vc"], self.aseq, k, v.transpose(1, 2), self.mask[:M])
        x1 = _C.rowlin_gptq(y[0], _C.ROWLIN_GATE, [(L["o"], c.hidden)], gate=pre[:, hd:nq], gate_head_stride=2 * hd,
                            lut=self.sig_lut, residual=self._residual(x))
        x1 = self._reduce(x1)
        out = self._reduce(_C.mlp_gptq(x1, L["ln2"], c.eps, L["gate"], L["up"], L["down"], silu_lut=self.silu_lut,
                                       I=c.inter, residual=self._residual(True)))
        self._t("attn", i, x=x, pre=pre, q=q, k=k, kc=L["kc"], vc=L["vc"], y=y, x1=x1, out=out, freqs=freqs,
                apos=self.apos, aseq=self.aseq)
        return out

    def _gdn(self, L, x, i=-1):
        c = self.cfg
        M = x.shape[0]
        HV, D = c.gdn_v_heads, c.gdn_dim
        Ck = 2 * c.gdn_k_heads * D + HV * D
        xn = torch.empty_like(x)
        ab = torch.empty((x.shape[0], L["wab"].shape[0]), dtype=torch.bfloat16, device=x.device)
        pre = _C.rowlin_gptq(x, _C.ROWLIN_NORM, [(L["qkv"], Ck), (L["z"], HV * D)], norm_w=L["ln1"], eps=c.eps,
                             xn_out=xn, ab=(L["wab"], ab))  # + the a | b projection of xn in the same launch
        prev, save = L["saved"][self.parity], L["saved"][1 - self.parity]
        core = _C.gdn_step_deferred(pre[:, :Ck], pre[:, Ck:], ab[:, :HV], ab[:, HV:], L["conv_w"], L["conv_state"],
                                    L["dt_bias"], L["g_decay"],
                                    L["state"], L["gnorm"], c.eps, D ** -0.5, c.gdn_k_heads, self.ctl, prev, save)
        x1 = self._reduce(_C.rowlin_gptq(core, _C.ROWLIN_QUANT, [(L["out"], c.hidden)], residual=self._residual(x)))
        out = self._reduce(_C.mlp_gptq(x1, L["ln2"], c.eps, L["gate"], L["up"], L["down"], silu_lut=self.silu_lut,
                                       I=c.inter, residual=self._residual(True)))
        self._t("gdn", i, x=x, pre=pre, xn=xn, ab=ab, core=core, x1=x1, out=out, state=L["state"],
                conv_state=L["conv_state"])
        return out

    # ---- layer programs: the verify body as 9 persistent launches (one per run of layers between two attention
    # cores), separated by the attention kernels ----------------------------------------------------------------
    def _build_programs(self):
        """Two program sets (the GDN replay buffers alternate with the step parity); each set is a list of
        programs, program j running [post of attention layer 4j - 1 (j > 0)], the GDN layers, [pre of the next
        attention layer]. All activations live in fixed scratch buffers."""
        c, dev = self.cfg, self.dev
        R, H, I, hd = self.tree["rows"], c.hidden, c.inter, c.head_dim
        HV, D, hk = c.gdn_v_heads, c.gdn_dim, c.gdn_k_heads
        Ck, Z = 2 * hk * D + HV * D, HV * D
        nq, nkv = 2 * c.heads * hd, c.kv_heads * hd
        bf, i8, f32 = torch.bfloat16, torch.int8, torch.float32
        e = lambda *shape, dtype=bf: torch.zeros(*shape, dtype=dtype, device=dev)  # noqa: E731
        B = dict(X=e(R, H), X1=e(R, H), XN=e(R, H), Q1=e(16, max(H, 4096), dtype=i8), S1=e(64, dtype=f32),
                 PROJ=e(R, Ck + Z), AB=e(R, 2 * HV), RAW=e(R, Z), QC=e(16, max(Z, c.heads * hd), dtype=i8),
                 SC=e(64, dtype=f32), HB=e(R, I), Q2=e(16, I, dtype=i8), S2=e(64, dtype=f32),
                 AMAX=e(64, dtype=torch.int32), PRE=e(R, nq + 2 * nkv), Y=e(1, R, c.heads * hd),
                 GWS=e(_C._lib.load().mono_gdn_step_workspace(R, Ck, HV), dtype=torch.uint8))
        self.buf = B

        def post(P, L, w_o, K):  # out / o projection + residual, then the MLP block (the reference's layer_post)
            P.gemv([(w_o, H)], K, B["QC"], B["SC"], B["X1"], H, residual=B["X"], residual_stride=H)
            P.rows(ROWS_NORM, B["X1"], H, B["Q1"], B["S1"], norm_w=L["ln2"], eps=c.eps, zero=B["AMAX"])
            P.gemv([(L["gate"], I), (L["up"], I)], H, B["Q1"], B["S1"], B["HB"], I, paired=True, silu_lut=self.silu_lut,
                   amax=B["AMAX"])
            P.quant(B["HB"], I, B["AMAX"], B["Q2"], B["S2"])
            P.gemv([(L["down"], H)], I, B["Q2"], B["S2"], B["X"], H, residual=B["X1"], residual_stride=H)

        def gdn(P, L, parity):
            prev, save = L["saved"][parity], L["saved"][1 - parity]
            P.rows(ROWS_NORM, B["X"], H, B["Q1"], B["S1"], norm_w=L["ln1"], eps=c.eps, xn_out=B["XN"])
            P.ab(B["XN"], H, H, L["wab"], B["AB"])
            P.gemv([(L["qkv"], Ck), (L["z"], Z)], H, B["Q1"], B["S1"], B["PROJ"], Ck + Z)
            proj, ab = B["PROJ"], B["AB"]
            for delta in (0, 1):
                P.gdn(delta, proj, proj[:, Ck:], ab, ab[:, HV:], L["conv_w"], L["conv_state"], L["dt_bias"],
                      L["g_decay"], L["state"], L["gnorm"], c.eps, D ** -0.5, R, hk, HV, B["RAW"], self.ctl, prev, save,
                      Ck + Z, Ck + Z, 2 * HV, B["GWS"])
            P.rows(ROWS_GDN, B["RAW"], Z, B["QC"], B["SC"], norm_w=L["gnorm"], eps=c.eps, gate=proj[:, Ck:],
                   gate_row_stride=Ck + Z)
            post(P, L, L["out"], Z)

        sets = []
        for parity in (0, 1):
            progs, P = [], _C.Program(dev)
            for i, L in enumerate(self.layers):
                if c.is_attn(i):
                    P.rows(ROWS_NORM, B["X"], H, B["Q1"], B["S1"], norm_w=L["ln1"], eps=c.eps)
                    P.gemv([(L["q"], nq), (L["k"], nkv), (L["v"], nkv)], H, B["Q1"], B["S1"], B["PRE"], nq + 2 * nkv,
                           barrier=False)
                    progs.append(P.plan(R))
                    P = _C.Program(dev)
                    P.rows(ROWS_GATE, B["Y"].view(R, -1), c.heads * hd, B["QC"], B["SC"], gate=B["PRE"][:, hd:],
                           gate_row_stride=nq + 2 * nkv, gate_head_stride=2 * hd, lut=self.sig_lut)
                    post(P, L, L["o"], c.heads * hd)
                else:
                    gdn(P, L, parity)
            progs.append(P.plan(R))
            sets.append(progs)
        return sets

    def _verify_programs(self, tokens, freqs):
        c, B = self.cfg, self.buf
        R, hd = tokens.numel(), c.head_dim
        nq, nkv = 2 * c.heads * hd, c.kv_heads * hd
        torch.index_select(self.embed, 0, tokens.view(-1), out=B["X"])
        progs = self.programs[self.parity]
        attn = [L for i, L in enumerate(self.layers) if c.is_attn(i)]
        for j, P in enumerate(progs):
            P.launch(self.prefetch)
            if j < len(attn):
                L = attn[j]
                pre = B["PRE"]
                qg = pre[:, :nq].view(1, R, c.heads, 2 * hd)
                rawk = pre[:, nq:nq + nkv].view(1, R, c.kv_heads, hd)
                v = pre[:, nq + nkv:].view(1, R, c.kv_heads, hd)
                q, k = _C.qk_norm_rope_kv(qg[..., :hd], rawk, v, L["q_norm"], L["k_norm"], freqs, L["kc"], L["vc"],
                                          self.apos, c.eps, c.eps, c.rotary_dim)
                _C.attn_dpas(q, L["kc"], L["vc"], self.aseq, k, v.transpose(1, 2), self.mask[:R], out=B["Y"])
        return B["X"]

    def verify(self, tokens):
        """The tree's rows through the body; returns (greedy tokens [1, R], final hidden rows [R, H])."""
        c = self.cfg
        R = tokens.numel()
        _C.mtp_prep_verify(self.st, self.apos, self.aseq, self.vpos, self.tree_pos, self.ctl, self.tree_ctl,
                           self.parity, 0)
        freqs = self.rope[self.vpos.view(-1).clamp(max=self.cap - 1)]
        if self.fused:
            x = self._verify_programs(tokens, freqs)
        else:
            x = self.embed[tokens.view(-1)]
            for i, L in enumerate(self.layers):
                x = self._attention(L, x, freqs, i) if c.is_attn(i) else self._gdn(L, x, i)
        # final norm, then the bf16 lm_head with the greedy argmax fused (no logits written)
        xf = _C.rmsnorm_add(x, self.final_norm, c.eps)
        self._pick(xf, 0, argmax_out=self.toks.view(-1))
        self._t("verify", -1, tokens=tokens, x=x, xf=xf, toks=self.toks)
        return self.toks, x

    def _linear(self, x, w):
        """A draft projection x [1, K] @ w [N, K]^T (the reference's F.linear, draft_head.py:198-210): this build's
        GEMV, or torch's cuBLAS linear when the model was built with draft_gemv=False."""
        return _C.gemv_bf16(x, w) if self.draft_gemv else F.linear(x, w)

    def draft_token(self, hidden, k):
        """Draft k: the MTP head on chain node k's verify token (self.drafts[k]) and the previous hidden row [1, 1, H];
        its lm_head pick writes node k's children's verify tokens (argmax to the first child, the second best to the
        second). Returns the MTP hidden row [1, 1, H] for the next draft."""
        c, m = self.cfg, self.mtp
        hd, H = c.head_dim, c.hidden
        _C.mtp_prep_draft(self.st, k, self.rope.view(1, 1, self.cap, -1, 2, 2), self.mfreq.view(1, 1, 1, -1, 2, 2),
                          self.mpos, self.mseq)
        # cat(RMSNorm(embedding of node k's token), RMSNorm(hidden)): gather and both norms in one launch
        cat = _C.draft_embed_norm_cat(self.embed, self.drafts, k, m["enorm"], hidden.view(1, -1), m["hnorm"], c.eps)
        x = self._linear(cat, m["fc"])
        qkv = self._linear(_C.rmsnorm_add(x, m["ln1"], c.eps), m["qkv"])
        nq = 2 * c.heads * hd
        qg = qkv[:, :nq].view(1, 1, c.heads, 2 * hd)
        rawk = qkv[:, nq:nq + c.kv_heads * hd].view(1, 1, c.kv_heads, hd)
        v = qkv[:, nq + c.kv_heads * hd:].view(1, 1, c.kv_heads, hd)
        q, kk = _C.qk_norm_rope_kv(qg[..., :hd], rawk, v, m["q_norm"], m["k_norm"], self.mfreq, m["kc"], m["vc"],
                                   self.mpos, c.eps, c.eps, c.rotary_dim)
        y = _C.attn_dpas(q, m["kc"], m["vc"], self.mseq, kk, v.transpose(1, 2), self.no_mask)
        yg = _C.lut_mul(y[0], qkv[:, hd:nq], self.sig_lut, b_head_stride=2 * hd)
        xn, x = _C.rmsnorm_add(x, m["ln2"], c.eps, add=self._reduce(self._linear(yg, m["o"])))
        gu = self._linear(xn, m["gate_up"])
        h = _C.lut_mul(gu[:, c.inter:], gu[:, :c.inter], self.silu_lut)
        xf, x = _C.rmsnorm_add(x, m["norm"], c.eps, add=self._reduce(self._linear(h, m["down"])))
        self._pick(xf, c.tree[k], children=self.children[8 * k:8 * k + 8], dst=self.drafts, node=k)
        self._t("draft", k, xf=xf, drafts=self.drafts)
        return x.view(1, 1, -1)

    def step(self, steer=None):
        """One decode step, queued on the current stream: the draft tree, the verify, the accept. Returns the device
        result row of mono_mtp_accept ([n, commit[8], row, on_chain, ...]). steer (tests): a callable given the
        verify tokens [1, R] (device) before the accept, which may change them to force an accepted path."""
        c = self.cfg
        self.drafts[0:1] = self.next_tok.view(-1)
        h = self.hidden
        for k in range(c.depth):
            h = self.draft_token(h, k)
        toks, x = self.verify(self.drafts)
        if steer is not None:
            steer(toks)
        if self.trace is not None:  # (the stacked caches are a 50 MB copy: only when a test traces the step)
            self._t("accept_in", -1, toks=toks, drafts=self.drafts, st=self.st, ctl=self.ctl,
                    kv=torch.stack([t for L in self.layers if "kc" in L for t in (L["kc"], L["vc"])]))
        _C.mtp_accept(self.st, toks, self.drafts.view(1, -1), None, self.children, self.tree["rows"], c.depth, x,
                      self.next_tok, self.hidden, self.ctl, self.kv_ptrs, c.kv_heads, self.cap, c.head_dim,
                      self.result)
        self.total += self.result[0]
        self.parity = 1 - self.parity
        return self.result

    def step_graphed(self):
        """step(), replayed from CUDA graphs: the first call runs two eager steps (workspaces, tables) and captures
        one graph per GDN-buffer parity; every call then replays the graph of the current parity (the result row is
        the same device tensor as step()'s)."""
        if getattr(self, "_graphs", None) is None:
            self.step()
            self.step()
            torch.cuda.current_stream(self.dev).synchronize()
            graphs = {}
            for _ in range(2):
                p = self.parity
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g):
                    self.step()  # (flips self.parity; nothing runs until a replay)
                graphs[p] = g
            self._graphs = graphs
        self._graphs[self.parity].replay()
        self.parity = 1 - self.parity
        return self.result

    def release_graphs(self):
        self._graphs = None

    def own_launches_per_step(self) -> int:
        """This build's kernel launches per step (the rest are a few torch gathers / copies)."""
        c = self.cfg
        n_attn = sum(1 for i in range(c.layers) if c.is_attn(i))
        n_gdn = c.layers - n_attn
        if self.fused:  # one layer program per run of layers between attention cores; rope + attention x2
            body = (n_attn + 1) + n_attn * 3
        else:  # rowlin x2 (the GDN layers' first with the a|b projection) + MLP; GDN conv + delta; rope + attention x2
            body = c.layers * 3 + n_gdn * 2 + n_attn * 3
        # per draft: prep, embedding + 2 norms, rope, attention x2, 2 luts, 3 norm(-add)s, lm_head pick (+ 5 projections)
        draft = c.depth * (1 + 1 + 1 + 2 + 2 + 3 + 1 + (5 if self.draft_gemv else 0))
        return body + draft + 1 + 1 + 1 + 1  # prep_verify, final norm, lm_head pick, accept

    def step_bytes(self) -> int:
        """Algorithmic HBM bytes of one step: every weight byte read (W4 body once for the verify rows, the
        bf16 lm_head by the verify and by each draft, the MTP block per draft), GDN states read and written,
        the attended KV prefix."""
        c = self.cfg
        body = sum(t.numel() for L in self.layers for k, t in L.items()
                   if k in ("gate", "up", "down", "q", "k", "v", "o", "qkv", "z", "out"))
        small = sum(L[k].numel() * L[k].element_size() for L in self.layers for k in ("wab", "conv_w")
                    if k in L)
        state = sum(L["state"].numel() * 4 * 2 for L in self.layers if "state" in L)
        lm = self.lm_head.numel() * 2
        mtp = sum(t.numel() * t.element_size() for k, t in self.mtp.items() if k not in ("kc", "vc"))
        kv = int(self.st[0].item()) * c.kv_heads * c.head_dim * 2 * 2 * sum(1 for L in self.layers if "kc" in L)
        return body + small + state + lm * (1 + c.depth) + mtp * c.depth + kv
