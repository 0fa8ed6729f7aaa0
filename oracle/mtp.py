"""Device-side MTP loop bookkeeping on the CPU (test infrastructure only; see oracle/__init__.py).

accept_walk restates the reference's host accept walk (comfy_mono_decode_xpu/mtp_loop.py:117-136, upstream's
qwen35 _generate_mtp step); mtp_accept / prep_draft / prep_verify restate csrc/mtp_loop.sycl:29-196 on numpy
arrays (the result row, the counters st, the deferred-delta ctl, the next token and hidden row, and the attention
KV slot moves of an off-chain path, FixedKVState.commit_path)."""
from __future__ import annotations

import numpy as np

SLOTS, RANKS = 8, 7


def accept_walk(children, toks, dr, depth, cand):
    """children: per row the list of child rows; toks: the verify's token at each row; dr: the draft token of
    each row; cand: the draft's RANKS candidates per chain node (flat) or None. Returns
    (path, commit, ranks, row, on_chain, kept)."""
    path = [0]
    while True:
        nxt = None
        for c in children[path[-1]]:
            if dr[c] == toks[path[-1]]:
                nxt = c
                break
        if nxt is None:
            break
        path.append(nxt)
    ranks = []
    if cand is not None:
        for node in path:
            if node >= depth:
                break
            cs = list(cand[RANKS * node:RANKS * node + RANKS])
            ranks.append(cs.index(toks[node]) if toks[node] in cs else RANKS)
    commit = [dr[r] for r in path[1:]] + [toks[path[-1]]]
    row = path[-1]
    on_chain = row == len(path) - 1
    kept = min(len(path) if on_chain else len(path) - 1, depth)
    return path, commit, ranks, row, on_chain, kept


def mtp_accept(st, toks, dr, cand, children_table, rows, depth, x, ctl, kv_caches, kv_cap):
    """The device accept step on host copies. children_table [8, 8] int (-1 ends a row's list); x [rows, H];
    kv_caches: list of [heads, cap, D] arrays (updated in place); st [4] int64 and ctl [26] int32 updated in
    place. Returns (result [32] int64, next_token, hidden row)."""
    children = [[int(c) for c in children_table[r] if c >= 0] for r in range(SLOTS)]
    # the device walk stops after `rows` entries
    path, commit, ranks, row, on_chain, kept = accept_walk(children, toks, dr, depth, cand)
    path = path[:rows]
    pos = int(st[0])
    res = np.zeros(32, dtype=np.int64)
    n = len(path)
    res[0] = n
    res[1:1 + len(commit)] = commit
    res[n + 1:SLOTS + 1] = -1
    res[9], res[10] = row, int(on_chain)
    res[11] = len(ranks)
    res[12:12 + len(ranks)] = ranks
    res[19], res[20] = pos, kept
    st[0] = pos + n
    st[1] = st[1] + kept
    ctl[0] = n
    for i in range(SLOTS):
        ctl[2 + i] = path[i] if i < n else i
    if not on_chain:
        for cache in kv_caches:
            for k in range(1, n):
                src = path[k]
                if src != k:
                    cache[:, (pos + k) % kv_cap] = cache[:, (pos + src) % kv_cap]
    return res, int(toks[row]), x[row].copy()


def prep_draft(st, k, ftab, np_):
    """MTP KV positions / seqlen for draft k and the draft's rope row (csrc/mtp_loop.sycl:29-55).
    ftab [cap, n]. Returns (freqs [n], mpos [np_], mseq)."""
    p, m = int(st[0]) + k, int(st[1]) + k
    row = min(p, ftab.shape[0] - 1)
    return ftab[row].copy(), np.arange(m, m + np_, dtype=np.int64), m + 1


def prep_verify(st, np_, tree_pos, ctl, tree_ctl, parity, rope_offset):
    """Attention positions / seqlen, verify rope positions, ctl parity and tree program (:57-90)."""
    pos = int(st[0])
    ctl[1] = parity
    ctl[2 + SLOTS:2 + 3 * SLOTS] = tree_ctl
    return np.arange(pos, pos + np_, dtype=np.int64), pos, np.asarray(tree_pos, dtype=np.int64) + pos + rope_offset
