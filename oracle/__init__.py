"""CPU oracle for the W4A8 decode step: a restatement of the reference's arithmetic in numpy (int64 /
fp64 where exact, IEEE fp32 where the reference rounds in fp32).

TEST INFRASTRUCTURE ONLY. It is imported by tests/, by __graft_entry__.smoke() and by bench.py's
cpu_baseline / reference leg, and only as the checker or the timed CPU baseline. The product path
(comfy-mono-decode-xpu_b200/) never imports it and has no CPU fallback.

Each function names the reference file:line it follows (paths inside xiangyuT/comfy-mono-decode-xpu).
The reference ships no golden vectors; where its own tests state the arithmetic in CPU code
(tests/test_rope_kv.py:9-23, tests/test_attn_dpas.py:18-29, tests/test_mtp_accept.py,
comfy_mono_decode_xpu/mtp_loop.py:117-136, tests/test_draft_lmhead.py:12-30) the oracle is pinned
against fixtures generated from those functions (tests/golden/). The W4A8 linear, rot_quant, RMSNorm,
MLP and GDN formulas are pinned by the cited kernel source only (parity pinned by formula); the GPTQ
format of BASELINE.json has no reference implementation and its fp32 order is defined here and in
include/mono_b200.h.
"""
