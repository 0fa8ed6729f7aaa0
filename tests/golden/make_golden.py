"""Generate the golden fixtures of tests/golden/ from the reference's own CPU known-answer functions.

The reference ships no golden vectors; its tests state the arithmetic of a few paths as CPU functions, which
this script runs on seeded inputs (it needs the reference checkout, which is read, never modified):

  rope_kv.npz       tests/test_rope_kv.py:9-23       _reference: partial split-half RoPE, products rounded
                                                    separately, one bf16 rounding of the sum
  attn_fp64.npz     tests/test_attn_dpas.py:11-29    _mask / _reference: fp64 tree decode attention
  accept_walk.npz   comfy_mono_decode_xpu/mtp_loop.py:117-136  _upstream_walk: the greedy accept walk

Usage: python tests/golden/make_golden.py [reference_root]   (default: the REFERENCE_ROOT environment
variable). The functions are taken out of the reference files by name (ast) and run as they are written.
"""
from __future__ import annotations

import ast
import os
import sys

import numpy as np
import torch

HERE = os.path.dirname(os.path.abspath(__file__))


def _functions(path: str, names: list[str], env: dict) -> dict:
    src = open(path).read()
    tree = ast.parse(src)
    def assigned(n):
        out = []
        for t in n.targets:
            out += [t] if isinstance(t, ast.Name) else list(getattr(t, "elts", []))
        return [t.id for t in out if isinstance(t, ast.Name)]

    keep = [n for n in tree.body if (isinstance(n, ast.FunctionDef) and n.name in names) or
            (isinstance(n, ast.Assign) and any(a in names for a in assigned(n)))]
    mod = ast.Module(body=keep, type_ignores=[])
    ns = dict(env)
    exec(compile(mod, path, "exec"), ns)
    return {k: ns[k] for k in names if k in ns}


def bits(t: torch.Tensor) -> np.ndarray:
    return t.contiguous().view(torch.int16).numpy().view(np.uint16)


def make_rope(ref_root: str):
    fns = _functions(os.path.join(ref_root, "tests", "test_rope_kv.py"), ["_reference"], {"torch": torch})
    ref = fns["_reference"]
    g = torch.Generator().manual_seed(0x5EED + 2)
    out = {}
    cases = [(1, 16, 64), (3, 4, 64), (8, 16, 64), (8, 4, 128), (2, 1, 256)]
    for i, (S, H, rd) in enumerate(cases):
        x = (torch.randn(S, H, 256, generator=g) * torch.exp(torch.randn(S, H, 256, generator=g) * 2)).to(torch.bfloat16)
        f = torch.randn(S, rd // 2, 2, 2, generator=g)
        y = ref(x, f, rd)
        out[f"x{i}"], out[f"f{i}"], out[f"y{i}"], out[f"rd{i}"] = bits(x), f.numpy(), bits(y), np.int64(rd)
    np.savez_compressed(os.path.join(HERE, "rope_kv.npz"), n=np.int64(len(cases)), **out)


def make_attn(ref_root: str):
    path = os.path.join(ref_root, "tests", "test_attn_dpas.py")
    fns = _functions(path, ["_mask", "_reference", "H", "HK", "D"], {"torch": torch})
    H, HK, D = fns["H"], fns["HK"], fns["D"]
    g = torch.Generator().manual_seed(0x5EED + 2)
    out = {}
    cases = [(0, 16, [-1, 0, 1]), (5, 24, [-1, 0, 1, 2, 3, 4, 5, 6]), (40, 48, [-1, 0, 0, 0, 0, 1, 1, 1]),
             (33, 40, None)]
    for i, (L, cap, parents) in enumerate(cases):
        S = 1 if parents is None else len(parents)
        q = (torch.randn(1, H, S, D, generator=g) * 2).to(torch.bfloat16)
        k = (torch.randn(1, HK, cap, D, generator=g) * 1.5).to(torch.bfloat16)
        v = torch.randn(1, HK, cap, D, generator=g).to(torch.bfloat16)
        xk = (torch.randn(1, HK, S, D, generator=g) * 1.5).to(torch.bfloat16)
        xv = torch.randn(1, HK, S, D, generator=g).to(torch.bfloat16)
        mask = None if parents is None else fns["_mask"](parents)
        ref = fns["_reference"](q, k, v, L, xk, xv, mask)
        out.update({f"q{i}": bits(q[0]), f"k{i}": bits(k[0]), f"v{i}": bits(v[0]), f"xk{i}": bits(xk[0]),
                    f"xv{i}": bits(xv[0]), f"L{i}": np.int64(L), f"ref{i}": ref[0].numpy(),
                    f"mask{i}": np.array(mask if mask is not None else [], dtype=np.int64)})
    np.savez_compressed(os.path.join(HERE, "attn_fp64.npz"), n=np.int64(len(cases)), **out)


def make_accept(ref_root: str):
    import random
    walk = _functions(os.path.join(ref_root, "comfy_mono_decode_xpu", "mtp_loop.py"), ["_upstream_walk"], {})
    tfn = _functions(os.path.join(ref_root, "tests", "test_mtp_accept.py"), ["_tree", "_spec", "SLOTS"], {})
    spec, tree, SLOTS = tfn["_spec"], tfn["_tree"], tfn["SLOTS"]
    specs = [spec(w) for w in ((4, 3), (7,), (1, 1, 1, 1, 1, 1, 1), (2, 2, 3), (3, 1, 1, 2))]
    specs += [[[[[[]], []], []], []], [[[[[]]]]]]  # tree4s1m8, chain 4 (the reference test's list)
    out, k = {}, 0
    for si, sp in enumerate(specs):
        rng = random.Random(0x5EED + 4 + si)
        parent, children, depth_of, chain = tree(sp, SLOTS)
        for trial in range(12):
            toks = [rng.randrange(50) for _ in range(SLOTS)]
            dr = [rng.randrange(50) for _ in range(SLOTS)]
            for r in range(SLOTS):
                if children[r] and rng.random() < 0.8:
                    dr[rng.choice(children[r])] = toks[r]
            cand = [rng.randrange(50) for _ in range(49)]
            for node in range(chain):
                if rng.random() < 0.7:
                    cand[7 * node + rng.randrange(7)] = toks[node]
            path, commit, ranks, row, on_chain, kept = walk["_upstream_walk"](children, toks, dr, chain, cand)
            ch = np.full((SLOTS, SLOTS), -1, dtype=np.int32)
            for r, cs in enumerate(children):
                ch[r, :len(cs)] = cs
            out.update({f"children{k}": ch, f"toks{k}": np.array(toks), f"dr{k}": np.array(dr),
                        f"cand{k}": np.array(cand), f"depth{k}": np.int64(chain), f"path{k}": np.array(path),
                        f"commit{k}": np.array(commit), f"ranks{k}": np.array(ranks, dtype=np.int64),
                        f"row{k}": np.int64(row), f"on_chain{k}": np.int64(on_chain), f"kept{k}": np.int64(kept)})
            k += 1
    np.savez_compressed(os.path.join(HERE, "accept_walk.npz"), n=np.int64(k), **out)


if __name__ == "__main__":
    root = sys.argv[1] if len(sys.argv) > 1 else os.environ.get("REFERENCE_ROOT")
    if not root or not os.path.isdir(root):
        raise SystemExit("usage: make_golden.py <reference checkout>")
    make_rope(root)
    make_attn(root)
    make_accept(root)
    print("wrote", sorted(f for f in os.listdir(HERE) if f.endswith(".npz")))
