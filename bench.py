"""Benchmark of the W4A8 decode step on B200 (driver contract: one JSON line from rank 0).

  python bench.py [--gpus N] [--steps K] [--warmup W] [--impl ours|reference] [--workload decode|gemv|mlp]

Workload `decode` (default; BASELINE.json configs[4], the headline "decode tok/s"): the synthetic
Qwen3.5-9B-shaped W4A8 model (random-init weights, mono_b200.decoder) decoding with the device-side MTP loop
(8-node tree4s1m8 draft tree of depth 4, bf16 MTP head and lm_head, 8 verify rows, greedy accept), one stream
per GPU, prompt 1024 (a shorter second run at prompt 4096 goes into config); value = committed tokens / device
time of K steps (two CUDA graphs replayed back to back, CUDA events, max over ranks); roofline of the step's
dominant kernel (the fused MLP) timed alone; e2e reads every step's result row back to the host.

Workload `gemv` (configs[0], the "W4A8 GEMV HBM GB/s" part): 64 verify-row linears per step (M = 8, bf16 x
[8, 4096] -> act quant -> GPTQ W4A8 GEMV 4096 -> 12288) over 8 weight copies (208 MB > L2). Workload `mlp`
(configs[1]): the fused MLP block over 4 weight copies (312 MB > L2).

Multi-GPU: every rank runs its own replica (independent decode streams, no collective): scaling "weak".
--impl reference: the reference's arithmetic on the host cores (the CPU restatement; the reference itself is SYCL
for Intel GPUs and cannot run here): for decode, the whole decode step of the same model as torch-CPU eager ops.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(ROOT, "comfy-mono-decode-xpu_b200")
for _p in (ROOT, PKG):
    if _p not in sys.path:
        sys.path.insert(0, _p)

METRIC = "decode tok/s (1 stream, 1 B200) + aggregate tok/s at 2/4/8; W4A8 GEMV HBM GB/s"
N_OUT, K_IN, M_ROWS = 12288, 4096, 8
COPIES, PER_STEP = 8, 64
L2_BYTES = 126 * 2 ** 20


def gemv_bytes(M, N, K, x_bf16=True):
    """Algorithmic HBM bytes of one W4A8 linear: int4 weights + fp16 scales + activation in + bf16 out."""
    return N * K // 2 + N * (K // 128) * 2 + M * K * (2 if x_bf16 else 1) + M * N * 2 + (0 if x_bf16 else M * 4)


def peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), "measured"
    except Exception:
        return 6650.0, "fallback"


def traffic_fields(name):
    """roofline.traffic and its provenance: the per-launch DRAM bytes (dram__bytes_read.sum +
    dram__bytes_write.sum) of the kernel's committed ncu capture profiles/<name>.md, not of this run."""
    return {"traffic": profile_traffic(name),
            "traffic_source": f"ncu capture in profiles/{name}.md (an earlier run of the same kernel and shape)"}


def profile_traffic(name):
    """Per-launch DRAM bytes of a kernel from its committed ncu summary (profiles/<name>.md line
    `traffic_bytes_per_launch: N`), or None."""
    path = os.path.join(ROOT, "profiles", name + ".md")
    try:
        for line in open(path):
            if line.strip().startswith("traffic_bytes_per_launch:"):
                return int(float(line.split(":", 1)[1].strip().split()[0]))
    except Exception:
        pass
    return None


class Clocks:
    """nvidia-smi sampling of SM clocks and throttle reasons during the timed region."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, index):
        self.index, self.proc, self.lines = index, None, []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(["nvidia-smi", f"--id={self.index}", f"--query-gpu={self.Q}",
                                          "--format=csv,noheader,nounits", "-lms", "100"],
                                         stdout=subprocess.PIPE, stderr=subprocess.DEVNULL, text=True)
        except Exception:
            self.proc = None
        return self

    def __exit__(self, *a):
        if self.proc is not None:
            self.proc.terminate()
            try:
                out, _ = self.proc.communicate(timeout=5)
            except Exception:
                self.proc.kill()
                out = ""
            self.lines = [l for l in out.splitlines() if l.strip()]

    def summary(self):
        sm, mx, reasons = [], None, set()
        for l in self.lines:
            f = [x.strip() for x in l.split(",")]
            try:
                sm.append(float(f[1]))
                mx = float(f[2])
            except Exception:
                continue
            for name, v in zip(("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"), f[5:9]):
                if v.lower().startswith("active"):
                    reasons.add(name)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx, "reasons": sorted(reasons),
                "samples": len(sm)}


def dist_setup(n):
    rank, world = int(os.environ.get("RANK", 0)), int(os.environ.get("WORLD_SIZE", 1))
    if world != n and n > 1 and "RANK" not in os.environ:
        raise SystemExit("bench.py --gpus N>1 must run under torch.distributed.run (one rank per GPU)")
    return rank, world, int(os.environ.get("LOCAL_RANK", 0))


# ---- our implementation ---------------------------------------------------------------------------------

def run_ours(args):
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    from mono_b200 import _C
    from oracle import w4a8 as ow  # seeded weight generator + the cpu_baseline leg (test infrastructure)

    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)

    # weights: 8 distinct copies (tile-major), seeded like BASELINE configs[0]
    packed, scales = ow.gen_gptq(N_OUT, K_IN, seed=0x5EED + 0)
    pk0, sc0 = torch.from_numpy(packed).to(dev), torch.from_numpy(scales).to(dev)
    ws = []
    for c in range(COPIES):
        # distinct bytes per copy (flip the low nibble of every byte of copy c when c is odd): same shapes
        pk = pk0 ^ c if c else pk0.clone()
        ws.append(_C.w4_repack(0, pk.contiguous(), sc0, N_OUT, K_IN))
    assert COPIES * ws[0].numel() > L2_BYTES
    g = torch.Generator().manual_seed(0x5EED + rank)
    xs_host = [torch.randn(M_ROWS, K_IN, generator=g).to(torch.bfloat16) for _ in range(COPIES)]
    xs_dev = [x.to(dev) for x in xs_host]
    outs = [torch.empty(M_ROWS, N_OUT, dtype=torch.bfloat16, device=dev) for _ in range(COPIES)]

    stream = torch.cuda.Stream(dev)

    def linear(i):
        # config 0's op as the reference's eager chain runs it: per-token act quant, then the W4A8 GEMV
        c = i % COPIES
        xq, s = _C.act_quant(xs_dev[c])
        return _C.w4a8_gptq_linear(xq, s.view(-1), ws[c], None, tiled=True, N=N_OUT, out=outs[c])

    def step():
        for i in range(PER_STEP):
            linear(i)

    def gemv_only(i, xq, s):
        c = i % COPIES
        return _C.w4a8_gptq_linear(xq, s, ws[c], None, tiled=True, N=N_OUT)

    # correctness gate on this box: one linear against the oracle
    with torch.cuda.stream(stream):
        out0 = linear(0)
    stream.synchronize()
    rq, rs = ow.act_quant(xs_host[0].view(torch.int16).numpy().view(np.uint16))
    ok = np.array_equal(out0.cpu().view(torch.int16).numpy().view(np.uint16), ow.gptq_linear(rq, rs, packed, scales))

    # capture K steps into one CUDA graph (warm-up replays first)
    with torch.cuda.stream(stream):
        for _ in range(3):
            step()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    for _ in range(max(args.warmup, 3)):
        graph.replay()
    torch.cuda.synchronize()

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()

    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
        stream.synchronize()
    barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    step_bytes = PER_STEP * gemv_bytes(M_ROWS, N_OUT, K_IN)
    value = world * args.steps * step_bytes / (ms * 1e-3) / 1e9

    # the dominant kernel alone: a graph of GEMV launches (same rotating weights), averaged per launch
    with torch.cuda.stream(stream):
        xq_s, s_s = _C.act_quant(xs_dev[0])
        s_s = s_s.view(-1)
        for i in range(3):
            gemv_only(i, xq_s, s_s)
    stream.synchronize()
    g2 = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g2, stream=stream):
        for i in range(PER_STEP):
            gemv_only(i, xq_s, s_s)
    for _ in range(3):
        g2.replay()
    torch.cuda.synchronize()
    reps = max(20, args.steps // 4)
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        k0.record(stream)
        for _ in range(reps):
            g2.replay()
        k1.record(stream)
    stream.synchronize()
    kern_us = k0.elapsed_time(k1) * 1e3 / (reps * PER_STEP)
    kbytes = gemv_bytes(M_ROWS, N_OUT, K_IN, x_bf16=False)
    hbm, src = peaks()
    achieved = kbytes / (kern_us * 1e-6) / 1e9

    # e2e through the public op calls with host buffers (pinned), per linear: H2D x, quant, GEMV, D2H out
    host_x = [x.pin_memory() for x in xs_host]
    host_o = torch.empty(M_ROWS, N_OUT, dtype=torch.bfloat16).pin_memory()
    e2e_linears = max(PER_STEP, args.steps * PER_STEP // 50)

    def e2e_once(i):
        c = i % COPIES
        xd = host_x[c].to(dev, non_blocking=True)
        xq, s = _C.act_quant(xd)
        o = _C.w4a8_gptq_linear(xq, s.view(-1), ws[c], None, tiled=True, N=N_OUT)
        host_o.copy_(o, non_blocking=True)

    with torch.cuda.stream(stream):
        for i in range(8):
            e2e_once(i)
    stream.synchronize()
    barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        f0.record(stream)
        for i in range(e2e_linears):
            e2e_once(i)
        f1.record(stream)
    stream.synchronize()
    e2e_ms = f0.elapsed_time(f1)
    if world > 1:
        t = torch.tensor([e2e_ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        e2e_ms = float(t.item())
    e2e_value = world * e2e_linears * gemv_bytes(M_ROWS, N_OUT, K_IN) / (e2e_ms * 1e-3) / 1e9

    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu:
        cpu = cpu_baseline(ow, packed, scales)

    if rank == 0:
        line = {
            "metric": METRIC,
            "value": round(value, 1),
            "unit": "GB/s",
            "n_gpus": world,
            "steps": args.steps,
            "warmup": args.warmup,
            "ms_per_step": round(ms / args.steps, 5),
            "higher_is_better": True,
            "scaling": "weak",
            "vs_baseline": None,
            "dtype": "int8",
            "data": "synthetic (seeded, BASELINE configs[0] distributions)",
            "config": {"workload": "W4A8 GPTQ verify linear 4096->12288, M=8 rows (configs[0])",
                       "linears_per_step": PER_STEP, "weight_copies": COPIES,
                       "l2": "inputs larger than L2 (8 weight copies = 208 MB cycled)", "parallelism": f"replicas x{world}",
                       "layout": "tile-major (mono_w4_repack)", "parity_gate": bool(ok)},
            "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(achieved / hbm, 4), "peak_source": src,
                         **traffic_fields("w4a8_gemv_gptq_m8_4096x12288"),
                         "kernel": "linear_kernel<GPTQ,TILED,MT=1>", "us_per_launch": round(kern_us, 3),
                         "algorithmic_bytes_per_launch": kbytes},
            "e2e": {"value": round(e2e_value, 1), "unit": "GB/s", "h2d_bytes_per_step": PER_STEP * M_ROWS * K_IN * 2,
                    "d2h_bytes_per_step": PER_STEP * M_ROWS * N_OUT * 2},
            "gpu_launches": args.steps * PER_STEP * 2,
            "clocks": clk.summary(),
        }
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def mlp_bytes(M, H, I):
    """Algorithmic bytes of the fused MLP block: three W4 matrices + scales, norm weight, x in, out."""
    w = lambda n, k: n * k // 2 + n * (k // 128) * 2
    return 2 * w(I, H) + w(H, I) + H * 2 + M * H * 2 * 2


MLP_PHASES = ("start", "dependency wait", "P1 rows + barrier + staging", "P2 gate/up consumed", "P2 epilogue",
              "P2 barrier", "P3 re-quantization + barrier + staging", "P4 down consumed", "P4 epilogue",
              "(P3) row maxima read", "(P3) pieces quantized", "(P3) barrier", "(P1) rows", "(P1) barrier")


def mlp_phase_trace(launch, dev):
    """One launch with the phase trace on (include/mono_b200.h mono_trace_enable): per phase boundary, the median
    and the last CTA's time in us after the first CTA started."""
    import numpy as np
    import torch

    from mono_b200 import _lib
    nbytes = _lib.load().mono_trace_bytes()
    buf = torch.zeros(nbytes, dtype=torch.uint8, device=dev)
    torch.cuda.synchronize(dev)
    _lib.call("mono_trace_enable", buf.data_ptr(), nbytes)
    try:
        launch()
        torch.cuda.synchronize(dev)
    finally:
        _lib.call("mono_trace_enable", None, 0)
    t = buf.view(torch.int64).view(1024, 16)[:, :len(MLP_PHASES)].cpu().numpy().astype(np.float64)
    t = t[t[:, 0] > 0]
    rel = (t - t[:, 0].min()) / 1000.0
    return {name: {"median": round(float(np.median(rel[:, p])), 2), "last": round(float(rel[:, p].max()), 2)}
            for p, name in enumerate(MLP_PHASES)}


def run_mlp(args):
    """Config 1: the fused MLP block (RMSNorm -> gate/up -> SiLU*up -> requant -> down -> residual), M rows,
    hidden 4096, intermediate 12288; 4 weight copies (312 MB) cycled so every block streams from HBM."""
    import datetime

    import numpy as np
    import torch
    import torch.distributed as dist

    from mono_b200 import _C
    from oracle import layers as ol
    from oracle import w4a8 as ow

    H, I, M, copies, per_step = 4096, 12288, args.rows, 4, 16
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120), device_id=dev)
    mats = [ow.gen_gptq(I, H, 0x5EED + 1), ow.gen_gptq(I, H, 0x5EED + 2), ow.gen_gptq(H, I, 0x5EED + 3)]
    base = [(torch.from_numpy(p).to(dev), torch.from_numpy(s).to(dev), n, k)
            for (p, s), (n, k) in zip(mats, [(I, H), (I, H), (H, I)])]
    ws = []
    for c in range(copies):
        ws.append([_C.w4_repack(0, (p ^ c).contiguous() if c else p, s, n, k) for p, s, n, k in base])
    g = torch.Generator().manual_seed(0x5EED + 1 + rank)
    x = torch.randn(M, H, generator=g).to(torch.bfloat16)
    nw = (1 + torch.randn(H, generator=g) * 0.02).to(torch.bfloat16)
    xd, nwd = x.to(dev), nw.to(dev)
    lut = _C.act_luts(dev)[0]
    outs = [torch.empty_like(xd) for _ in range(copies)]
    stream = torch.cuda.Stream(dev)

    def step():
        for i in range(per_step):
            c = i % copies
            _C.mlp_gptq(xd, nwd, 1e-6, *ws[c], silu_lut=lut, out=outs[c])

    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    lut_np = lut.cpu().view(torch.int16).numpy().view(np.uint16)
    xb = x.view(torch.int16).numpy().view(np.uint16)
    ok = np.array_equal(outs[0].cpu().view(torch.int16).numpy().view(np.uint16),
                        ol.mlp_gptq(xb, nw.view(torch.int16).numpy().view(np.uint16), 1e-6, *mats, lut_np))
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    if world > 1:
        dist.barrier()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
        stream.synchronize()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    b = mlp_bytes(M, H, I)
    us = ms * 1e3 / (args.steps * per_step)
    hbm, src = peaks()
    value = world * args.steps * per_step * b / (ms * 1e-3) / 1e9
    # e2e: host x in, host out back, per block through the public call
    hx = x.pin_memory()
    ho = torch.empty_like(hx).pin_memory()
    n_e2e = 64
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        f0.record(stream)
        for i in range(n_e2e):
            xi = hx.to(dev, non_blocking=True)
            o = _C.mlp_gptq(xi, nwd, 1e-6, *ws[i % copies], silu_lut=lut)
            ho.copy_(o, non_blocking=True)
        f1.record(stream)
    stream.synchronize()
    e2e = world * n_e2e * b / (f0.elapsed_time(f1) * 1e-3) / 1e9
    trace = mlp_phase_trace(lambda: _C.mlp_gptq(xd, nwd, 1e-6, *ws[0], silu_lut=lut, out=outs[0]), dev) \
        if args.trace else None
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(value, 1), "unit": "GB/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded, BASELINE configs[1] distributions)",
            "config": {"workload": f"fused W4A8 MLP block 4096->12288->4096, M={M} rows (configs[1])",
                       "blocks_per_step": per_step, "weight_copies": copies,
                       "l2": "inputs larger than L2 (4 weight copies = 312 MB cycled)", "parity_gate": bool(ok),
                       **({"phase_trace_us": trace} if trace else {})},
            "roofline": {"bound": "hbm", "achieved": round(b / (us * 1e-6) / 1e9, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(b / (us * 1e-6) / 1e9 / hbm, 4), "peak_source": src,
                         **traffic_fields("mlp_kernel_m8"), "kernel": "mlp_kernel<1,2>",
                         "us_per_launch": round(us, 3), "algorithmic_bytes_per_launch": b},
            "e2e": {"value": round(e2e, 1), "unit": "GB/s", "h2d_bytes_per_step": per_step * M * H * 2,
                    "d2h_bytes_per_step": per_step * M * H * 2},
            "gpu_launches": args.steps * per_step, "clocks": clk.summary()}), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_lmhead(args):
    """The bf16 lm_head pick alone (mono_lmhead_pick: the verify's greedy argmax at --rows rows, or a draft's top-2
    pick at one row): 151,936 x 4096 bf16 weights (1.24 GB > L2) read once per call; the pick is checked against
    the oracle on the kernel's own logits before timing."""
    import numpy as np
    import torch

    from mono_b200 import _C
    from oracle import lmhead as olh

    V, K, M, per_step = 151936, 4096, args.rows, 8
    k = 2 if M == 1 else 0
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    g = torch.Generator(device=dev).manual_seed(0x5EED + 9 + rank)
    w = (torch.randn(V, K, device=dev, generator=g) * 0.02).to(torch.bfloat16)
    x = torch.randn(M, K, device=dev, generator=g).to(torch.bfloat16)
    am, tk, lg = _C.lmhead_pick(x, w, k=k, logits=True)
    lg_bits = lg.cpu().view(torch.int16).numpy().view(np.uint16)
    am_ref, top_ref = olh.pick_logits(lg_bits, k)
    ok = bool(np.array_equal(am.cpu().numpy(), am_ref) and (k == 0 or np.array_equal(tk.cpu().numpy(), top_ref)))
    stream = torch.cuda.Stream(dev)

    def step():
        for _ in range(per_step):
            _C.lmhead_pick(x, w, k=k)

    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
        stream.synchronize()
    ms = e0.elapsed_time(e1)
    b = V * K * 2 + M * K * 2
    us = ms * 1e3 / (args.steps * per_step)
    hbm, src = peaks()
    # e2e: host rows in, the picked indices back, per call through the public op
    hx = x.cpu().pin_memory()
    ha = torch.empty(M, dtype=torch.int64).pin_memory()
    n_e2e = 8
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        f0.record(stream)
        for _ in range(n_e2e):
            a2 = _C.lmhead_pick(hx.to(dev, non_blocking=True), w, k=k)[0]
            ha.copy_(a2, non_blocking=True)
        f1.record(stream)
    stream.synchronize()
    e2e_us = f0.elapsed_time(f1) * 1e3 / n_e2e
    if rank == 0:
        gbs = round(b / (us * 1e-6) / 1e9, 1)
        print(json.dumps({
            "metric": "lm_head pick GB/s (bf16 151936 x 4096, fused argmax / top-k)", "value": gbs, "unit": "GB/s",
            "n_gpus": 1, "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "bf16 -> fp32 accumulate",
            "data": "synthetic (seeded N(0, 0.02) weights, N(0, 1) rows)",
            "config": {"workload": f"bf16 lm_head 151936 x 4096 + pick, M = {M} rows, k = {k}", "calls_per_step": per_step,
                       "l2": "inputs larger than L2 (1.24 GB of weights)", "parity_gate": ok},
            "roofline": {"bound": "hbm", "achieved": gbs, "peak": hbm, "unit": "GB/s", "frac": round(gbs / hbm, 4),
                         "peak_source": src, **traffic_fields("lmhead_pick_kernel_m8" if M > 1 else "lmhead_pick_kernel_m1"),
                         "kernel": "lmhead_pick_kernel", "us_per_launch": round(us, 3), "algorithmic_bytes_per_launch": b},
            "e2e": {"value": round(b / (e2e_us * 1e-6) / 1e9, 1), "unit": "GB/s", "h2d_bytes_per_step": per_step * M * K * 2,
                    "d2h_bytes_per_step": per_step * M * 8},
            "gpu_launches": args.steps * per_step, "clocks": clk.summary()}))


def run_topk_rows(args):
    """The verify sampling's top-k filter (the reference's topk_rows, csrc/topk_rows.sycl): exact top-64 of 8 fp32
    rows of 248,320 logits per call (the reference's "8 x 248k"); 32 input copies (254 MB) cycled so every call
    reads its rows from HBM. GB/s of row bytes read; parity checked against the oracle on the first call."""
    import numpy as np
    import torch

    from mono_b200 import _C
    from oracle.topk import topk_rows as ref_topk_rows

    R, N, k, copies, per_step = 8, 248320, 64, 32, 32
    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    g = torch.Generator().manual_seed(0x5EED + 8 + rank)
    host = torch.randn(R, N, generator=g) * 3
    xs = [(host + c * 1e-3).to(dev) if c else host.to(dev) for c in range(copies)]
    rv, ri = ref_topk_rows(host.numpy(), k)
    v, i = _C.topk_rows(xs[0], k)
    ok = bool(np.array_equal(i.cpu().numpy(), ri) and np.array_equal(v.cpu().numpy(), rv))
    stream = torch.cuda.Stream(dev)

    def step():
        for j in range(per_step):
            _C.topk_rows(xs[j % copies], k)

    with torch.cuda.stream(stream):
        step()
    stream.synchronize()
    graph = torch.cuda.CUDAGraph()
    with torch.cuda.graph(graph, stream=stream):
        step()
    for _ in range(args.warmup):
        graph.replay()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with Clocks(local) as clk:
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(args.steps):
                graph.replay()
            e1.record(stream)
        stream.synchronize()
    ms = e0.elapsed_time(e1)
    b = R * N * 4 + R * k * 12
    us = ms * 1e3 / (args.steps * per_step)
    hbm, src = peaks()
    # e2e: host rows in, values / indices back, per call through the public op
    hx = host.pin_memory()
    hv = torch.empty(R, k).pin_memory()
    hi = torch.empty(R, k, dtype=torch.int64).pin_memory()
    n_e2e = 16
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        f0.record(stream)
        for _ in range(n_e2e):
            vv, ii = _C.topk_rows(hx.to(dev, non_blocking=True), k)
            hv.copy_(vv, non_blocking=True)
            hi.copy_(ii, non_blocking=True)
        f1.record(stream)
    stream.synchronize()
    e2e_us = f0.elapsed_time(f1) * 1e3 / n_e2e
    if rank == 0:
        print(json.dumps({
            "metric": "topk_rows GB/s (verify sampling top-k, 8 x 248320 fp32, k = 64)",
            "value": round(b / (us * 1e-6) / 1e9, 1), "unit": "GB/s", "n_gpus": 1, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": round(ms / args.steps, 5), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int64 ranks (fp32 keys)",
            "data": "synthetic (seeded N(0, 3) logits)",
            "config": {"workload": "exact top-64 of 8 rows x 248320 fp32 (the reference's topk_rows)",
                       "calls_per_step": per_step, "copies": copies,
                       "l2": "inputs larger than L2 (32 copies = 254 MB cycled)", "parity_gate": ok},
            "roofline": {"bound": "hbm", "achieved": round(b / (us * 1e-6) / 1e9, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(b / (us * 1e-6) / 1e9 / hbm, 4), "peak_source": src, "traffic": None,
                         "kernel": "topk_rows_partial + topk_rows_final", "us_per_call": round(us, 3),
                         "algorithmic_bytes_per_call": b},
            "e2e": {"value": round(b / (e2e_us * 1e-6) / 1e9, 1), "unit": "GB/s", "h2d_bytes_per_step": R * N * 4,
                    "d2h_bytes_per_step": R * k * 12},
            "gpu_launches": args.steps * per_step * 2, "clocks": clk.summary()}), flush=True)


def reduce_time_and_count(ms, count, device, world):
    """Max of the device time and sum of the counted units over the ranks (every rank calls it, in the same
    order); identity on one rank."""
    if world <= 1:
        return ms, count
    import torch
    import torch.distributed as dist
    t = torch.tensor([ms], dtype=torch.float64, device=device)
    c = torch.tensor([count], dtype=torch.float64, device=device)
    dist.all_reduce(t, op=dist.ReduceOp.MAX)
    dist.all_reduce(c, op=dist.ReduceOp.SUM)
    return float(t.item()), int(c.item())


def _decode_measure(model, stream, steps, warmup, world, dev):
    """Steps of the decode loop, captured in two CUDA graphs (the GDN replay buffers alternate) and replayed back to
    back; returns (ms, committed tokens, graphs)."""
    import torch
    with torch.cuda.stream(stream):
        for _ in range(2):  # eager warm-up: workspaces
            model.step()
    stream.synchronize()
    graphs = []
    for _ in range(2):
        gph = torch.cuda.CUDAGraph()
        with torch.cuda.graph(gph, stream=stream):
            model.step()
        graphs.append(gph)
    for i in range(max(warmup, 3)):
        graphs[i % 2].replay()
    torch.cuda.synchronize()
    n0 = int(model.total.item())
    if world > 1:
        import torch.distributed as dist
        dist.barrier()
    torch.cuda.synchronize()
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        e0.record(stream)
        for i in range(steps):
            graphs[i % 2].replay()
        e1.record(stream)
    stream.synchronize()
    ms, toks = reduce_time_and_count(e0.elapsed_time(e1), int(model.total.item()) - n0, dev, world)
    return ms, toks, graphs


def run_decode_tp(args):
    """The decode step of ONE stream over `--gpus` ranks in tensor parallel (mono_b200.tp: column / row sharding,
    an all-reduce of the [8, 4096] bf16 residual after every row-sharded projection, the vocabulary-sharded
    lm_head with the merged pick). Reports the single stream's tok/s (strong scaling) and the measured latency of
    one all-reduce of that size (a CUDA graph of 64)."""
    import datetime

    import torch
    import torch.distributed as dist

    from mono_b200 import mtp_loop
    from mono_b200 import tp as tpm
    from mono_b200.decoder import Qwen35Config

    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg = Qwen35Config()
    model = tpm.make_decoder(cfg, dev, dist.group.WORLD, args.prompt, gen_tokens=max(512, args.steps * 8 + 64))
    stream = torch.cuda.Stream(dev)
    with Clocks(local) as clk:
        ms, toks, graphs = _decode_measure(model, stream, args.steps, args.warmup, world, dev)
    toks //= world  # one stream: every rank counts the same tokens
    del graphs
    model.release_graphs()
    # one all-reduce of the residual's size (the decoder's own, then NCCL's), 64 in a graph
    buf = torch.zeros(8, cfg.hidden, dtype=torch.bfloat16, device=dev)

    def per_call_us(fn):
        with torch.cuda.stream(stream):
            for _ in range(3):
                fn(buf)
        stream.synchronize()
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(64):
                fn(buf)
        g.replay()
        torch.cuda.synchronize()
        dist.barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(10):
                g.replay()
            e1.record(stream)
        stream.synchronize()
        del g
        return reduce_time_and_count(e0.elapsed_time(e1) * 1e3 / 640, 0, dev, world)[0]

    ar_us = per_call_us(model._reduce)
    nccl_us = per_call_us(lambda t: dist.all_reduce(t))
    # e2e: the plugin's greedy loop, every rank in step (the same committed tokens on every rank)
    mtp_loop.generate_device(model, 16)
    torch.cuda.synchronize()
    dist.barrier()
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    f0.record()
    committed = mtp_loop.generate_device(model, args.steps)
    f1.record()
    torch.cuda.synchronize()
    e2e_ms, _ = reduce_time_and_count(f0.elapsed_time(f1), 0, dev, world)
    model.release_graphs()
    step_bytes = model.step_bytes()
    hbm, src = peaks()
    step_ms = ms / args.steps
    ar_mode = "one-shot peer kernel (mono_allreduce2_bf16)" if model.peer_sum is not None else "NCCL"
    torch.cuda.synchronize()
    dist.barrier()
    model.close()
    if rank == 0:
        print(json.dumps({
            "metric": METRIC, "value": round(toks / (ms * 1e-3), 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (random-init Qwen3.5-9B-shaped W4A8 weights, random tokens, seeded)",
            "config": {"workload": "Qwen3.5-9B-shaped W4A8 MTP decode (configs[4]), ONE stream in tensor parallel",
                       "parallelism": f"tp{world}", "all_reduces_per_step": model.tp_reduces_per_step(),
                       "all_reduce": ar_mode,
                       "all_reduce_us": round(ar_us, 2), "nccl_all_reduce_us": round(nccl_us, 2),
                       "all_reduce_bytes": 8 * cfg.hidden * 2,
                       "tokens_per_step": round(toks / args.steps, 3),
                       "per_gpu_bytes_per_step": step_bytes},
            "step_roofline": {"achieved": round(step_bytes / (step_ms * 1e-3) / 1e9, 1), "peak": hbm, "unit": "GB/s",
                              "frac": round(step_bytes / (step_ms * 1e-3) / 1e9 / hbm, 4), "peak_source": src,
                              "what": "one rank's shard per step"},
            "e2e": {"value": round(len(committed) / (e2e_ms * 1e-3), 2), "unit": "tok/s",
                    "path": "mono_b200.mtp_loop.generate_device on the sharded decoder"},
            "gpu_launches": args.steps * model.own_launches_per_step(), "clocks": clk.summary()}), flush=True)
    dist.barrier()
    dist.destroy_process_group()


def run_decode(args):
    """Config 4: the synthetic Qwen3.5-9B-shaped W4A8 decoder with the device MTP loop (the 8-node tree4s1m8 draft
    tree of depth 4 from the bf16 MTP head and bf16 lm_head, 8 verify rows, greedy accept), one stream per GPU.
    Steps are captured in two CUDA graphs and replayed back to back; the committed tokens are summed on the device.
    A second, shorter measurement at prompt 4096 goes into config (configs[4] names prompts 1024 and 4096)."""
    import datetime

    import torch
    import torch.distributed as dist

    from mono_b200.decoder import Qwen35Config, Qwen35W4A8

    rank, world, local = dist_setup(args.gpus)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=300), device_id=dev)
    cfg = Qwen35Config()
    prompt = args.prompt
    B = args.streams

    def make_model(plen):
        if B > 1:  # batched streams: one weight stream a step for all of them (mono_b200.streams)
            from mono_b200.streams import Qwen35W4A8Streams
            return Qwen35W4A8Streams(cfg, dev, prompt_len=plen, streams=B, gen_tokens=max(512, args.steps * 8 + 64),
                                     seed=0x5EED + 4 + rank, draft_gemv=not args.cublas_draft)
        return Qwen35W4A8(cfg, dev, prompt_len=plen, gen_tokens=max(512, args.steps * 8 + 64), seed=0x5EED + 4 + rank,
                          fused=args.programs, prefetch=args.prefetch, draft_gemv=not args.cublas_draft)

    model = make_model(prompt)
    stream = torch.cuda.Stream(dev)
    if args.profile_step:
        # for ncu --profile-from-start off: warm steps, then one eager step between profiler start / stop
        for _ in range(max(args.warmup, 3)):
            model.step()
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.start()
        model.step()
        torch.cuda.synchronize(dev)
        torch.cuda.profiler.stop()
        if rank == 0:
            print(json.dumps({"profile_step": "one decode step profiled", "launches": model.own_launches_per_step()}))
        return
    with Clocks(local) as clk:
        ms, toks, graphs = _decode_measure(model, stream, args.steps, args.warmup, world, dev)
    step_ms = ms / args.steps
    step_bytes = model.step_bytes()
    launches = args.steps * model.own_launches_per_step()  # this build's kernels in the timed steps
    hbm, src = peaks()
    achieved = step_bytes / (step_ms * 1e-3) / 1e9
    del graphs
    # e2e through the plugin entry: mono_b200.mtp_loop.generate_device, what the _generate_mtp install point runs for
    # a greedy generate (steps replayed from CUDA graphs, every step's result row copied to a device ring, the ring
    # read back to the host every 8 steps to collect the committed tokens and check for stop tokens). Inside the
    # timed region: the prompt's token ids copied host -> device (pinned) and seeding the loop (the prefill itself is
    # left to stock, as in the reference), and the committed tokens read back.
    from mono_b200 import mtp_loop
    prompt_ids = torch.randint(0, cfg.vocab, (B, prompt), generator=torch.Generator().manual_seed(rank)).pin_memory()
    dev_ids = torch.empty(B, prompt, dtype=torch.int64, device=dev)
    gen = (lambda n: mtp_loop.generate_device(model, n)) if B == 1 else \
        (lambda n: mtp_loop.generate_device_streams(model, n))
    with torch.cuda.stream(stream):
        gen(16)  # captures the loop's graphs (outside the timing)
    stream.synchronize()
    n_new = max(64, args.steps)
    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(stream):
        f0.record(stream)
        dev_ids.copy_(prompt_ids, non_blocking=True)
        model.next_tok.view(-1).copy_(dev_ids[:, -1])
        committed = gen(n_new)
        f1.record(stream)
    stream.synchronize()
    n_committed = len(committed) if B == 1 else sum(len(c) for c in committed)
    e2e_steps = -(-n_new // 8) * 8  # whole rings of 8 steps (about one token per step and stream)
    e2e_ms, e2e_toks = reduce_time_and_count(f0.elapsed_time(f1), n_committed, dev, world)
    model.release_graphs()
    # the dominant kernel alone (the fused MLP block): a graph of its launches over the layers' weights at the
    # step's 8 verify rows, averaged per launch with CUDA events
    import mono_b200._C as C_
    R = model.tree["rows"] * B  # the verify rows of all streams
    xs = torch.randn(R, cfg.hidden, device=dev).to(torch.bfloat16)
    outs = torch.empty_like(xs)
    with torch.cuda.stream(stream):
        for L in model.layers[:4]:
            C_.mlp_gptq(xs, L["ln2"], cfg.eps, L["gate"], L["up"], L["down"], silu_lut=model.silu_lut, out=outs, I=cfg.inter)
    stream.synchronize()
    gm = torch.cuda.CUDAGraph()
    with torch.cuda.graph(gm, stream=stream):
        for L in model.layers:
            C_.mlp_gptq(xs, L["ln2"], cfg.eps, L["gate"], L["up"], L["down"], silu_lut=model.silu_lut, out=outs, I=cfg.inter)
    gm.replay()
    torch.cuda.synchronize()
    k0, k1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    reps = 10
    with torch.cuda.stream(stream):
        k0.record(stream)
        for _ in range(reps):
            gm.replay()
        k1.record(stream)
    stream.synchronize()
    mlp_us = k0.elapsed_time(k1) * 1e3 / (reps * cfg.layers)
    mlp_b = mlp_bytes(R, cfg.hidden, cfg.inter)
    del gm
    # prompt 4096: a second model, a shorter run
    p4096 = None
    if prompt != 4096 and not args.no_second_prompt:
        del model
        torch.cuda.empty_cache()
        m2 = make_model(4096)
        steps2 = max(10, args.steps // 2)
        ms2, toks2, g2 = _decode_measure(m2, stream, steps2, args.warmup, world, dev)
        del g2
        p4096 = {"tok_s": round(toks2 / (ms2 * 1e-3), 2), "ms_per_step": round(ms2 / steps2, 4), "steps": steps2,
                 "algorithmic_bytes_per_step": m2.step_bytes()}
        model = m2
    # 2 and 4 streams batched in one step on this GPU (mono_b200.streams: 16 / 32 verify rows, one weight read per
    # step for all of them)
    batched = {}
    if B == 1 and not args.no_batched:
        from mono_b200.streams import Qwen35W4A8Streams
        for nb in (2, 4):
            del model
            torch.cuda.empty_cache()
            m3 = Qwen35W4A8Streams(cfg, dev, prompt_len=prompt, streams=nb, gen_tokens=max(512, args.steps * 8 + 64),
                                   seed=0x5EED + 4 + rank, draft_gemv=not args.cublas_draft)
            steps3 = max(10, args.steps // 2)
            ms3, toks3, g3 = _decode_measure(m3, stream, steps3, args.warmup, world, dev)
            del g3
            batched[nb] = {"streams": nb, "tok_s": round(toks3 / (ms3 * 1e-3), 2),
                           "ms_per_step": round(ms3 / steps3, 4), "steps": steps3,
                           "tokens_per_step": round(toks3 / (steps3 * world), 3),
                           "what": f"aggregate committed tok/s of {nb} independent streams on this GPU, stepped "
                                   f"together (bench.py --streams {nb} for the full line)"}
            model = m3
    cpu = cpu_decode_baseline(args) if (rank == 0 and world == 1 and not args.no_cpu) else None
    if rank == 0:
        line = {
            "metric": METRIC, "value": round(toks / (ms * 1e-3), 2), "unit": "tok/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(step_ms, 4), "higher_is_better": True,
            "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (random-init Qwen3.5-9B-shaped W4A8 weights, random tokens, seeded)",
            "config": {"workload": f"Qwen3.5-9B-shaped W4A8 MTP decode (configs[4]): 8-node tree4s1m8 draft tree of "
                                   f"depth 4 (bf16 MTP head, bf16 lm_head), 8 verify rows, greedy accept, prompt {prompt}, "
                                   + ("1 stream per GPU" if B == 1 else
                                      f"{B} streams per GPU batched in one step ({R} verify rows)"),
                       "streams_per_gpu": B,
                       "layers": cfg.layers, "steps_per_s": round(args.steps / (ms * 1e-3), 2),
                       "tokens_per_step": round(toks / (args.steps * world), 3),
                       "tokens_per_step_note": "random-init weights: the drafts rarely match the verify (about one "
                                               "token per step, as expected; not tuned away)",
                       "l2": "inputs larger than L2 (11.9 GB of weights read per step)",
                       "body": (f"{len(model.programs[0])} layer programs per step (prefetch {args.prefetch})"
                                if args.programs else "one launch per fused op (rowlin / a|b / GDN / MLP / attention)"),
                       "draft_projections": "cuBLAS (F.linear)" if args.cublas_draft else "mono_gemv_bf16",
                       "lm_head": "mono_lmhead_pick (bf16 GEMV with the argmax / top-2 pick fused), verify and drafts",
                       "prompt_4096": p4096,
                       "streams_2": batched.get(2), "streams_4": batched.get(4),
                       "parallelism": f"independent streams x{world * B} ({B} per GPU)"},
            "roofline": {"bound": "hbm", "achieved": round(mlp_b / (mlp_us * 1e-6) / 1e9, 1), "peak": hbm, "unit": "GB/s",
                         "frac": round(mlp_b / (mlp_us * 1e-6) / 1e9 / hbm, 4), "peak_source": src,
                         **(traffic_fields("mlp_kernel_m8") if R == 8 else
                            {"traffic": None, "traffic_source": f"no ncu capture at M = {R} committed"}),
                         "kernel": f"mlp_kernel (fused MLP block, the step's dominant W4A8 kernel), M = {R} verify rows",
                         "us_per_launch": round(mlp_us, 3), "algorithmic_bytes_per_launch": mlp_b},
            "step_roofline": {"achieved": round(achieved, 1), "peak": hbm, "unit": "GB/s", "frac": round(achieved / hbm, 4),
                              "algorithmic_bytes_per_step": step_bytes,
                              "what": "whole step: W4 body + bf16 lm_head (verify and 4 drafts) + bf16 MTP block x 4 + "
                                      "GDN states + KV"},
            "e2e": {"value": round(e2e_toks / (e2e_ms * 1e-3), 2), "unit": "tok/s",
                    "h2d_bytes_per_step": round(B * prompt * 8 / e2e_steps, 1), "d2h_bytes_per_step": B * 32 * 8,
                    "path": ("mono_b200.mtp_loop.generate_device (the _generate_mtp install point's greedy loop)"
                             if B == 1 else "mono_b200.mtp_loop.generate_device_streams (every stream's greedy loop)"),
                    "copies": f"h2d: the {B} prompts' {prompt} token ids (pinned) once per generate; d2h: a "
                              f"{B * 256}-byte block of result rows per step, read in rings of 8"},
            "gpu_launches": launches, "clocks": clk.summary()}
        if cpu is not None:
            line["cpu_baseline"] = cpu
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def _cpu_decode_run(prompt, warmup, steps, budget_s=None):
    """The decode step of the same model (configs[4] shapes, tree4s1m8, greedy) as torch-CPU eager ops
    (oracle/cpu_decode.py: int8 _int_mm per 128-group with fp32 epilogues, bf16 linears) on all the host's cores.
    Runs `warmup` untimed steps, then up to `steps` timed ones (fewer when budget_s of timed work is spent).
    Returns (seconds per step: list, committed tokens, threads, build seconds)."""
    import torch

    from oracle.cpu_decode import CpuDecoder
    torch.set_num_threads(os.cpu_count() or 1)
    t0 = time.perf_counter()
    model = CpuDecoder(prompt_len=prompt, gen_tokens=64 + 8 * (warmup + steps))
    build = time.perf_counter() - t0
    for _ in range(warmup):
        model.step()
    times, toks = [], 0
    spent = 0.0
    for _ in range(steps):
        t0 = time.perf_counter()
        toks += len(model.step())
        times.append(time.perf_counter() - t0)
        spent += times[-1]
        if budget_s is not None and spent > budget_s and len(times) >= 5:
            break
    return times, toks, torch.get_num_threads(), build


def cpu_decode_baseline(args=None):
    """cpu_baseline of the decode line: the median of 5 actually-run steps of the same decode step on the host
    cores (_cpu_decode_run), in tok/s (committed tokens per step / the median step time)."""
    prompt = args.prompt if args is not None else 1024
    times, toks, threads, build = _cpu_decode_run(prompt, warmup=1, steps=5)
    med = statistics.median(times)
    per_step = toks / len(times)
    return {"value": round(per_step / med, 4), "unit": "tok/s", "cores": threads, "kind": "port",
            "sample": f"the whole decode step of the same model and tree (prompt {prompt}) as torch-CPU eager ops "
                      f"(oracle/cpu_decode.py: int8 x int8 -> int32 per 128-group, fp32 epilogues, bf16 linears); "
                      f"median of {len(times)} steps = {med:.3f} s, {per_step:.2f} tokens per step "
                      f"(model built in {build:.0f} s)"}


def cpu_baseline(ow, packed, scales, rows=None):
    """The oracle's eager chain (act quant + GPTQ linear) on the host cores, on a bounded sample."""
    import numpy as np
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    rows = rows or N_OUT // 4
    g = torch.Generator().manual_seed(7)
    x = torch.randn(M_ROWS, K_IN, generator=g).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)
    times = []
    for _ in range(3):
        t0 = time.perf_counter()
        q, s = ow.act_quant(x)
        ow.gptq_linear(q, s, packed[:rows], scales[:rows])
        times.append(time.perf_counter() - t0)
    t = statistics.median(times)
    return {"value": round(gemv_bytes(M_ROWS, rows, K_IN) / t / 1e9, 3), "unit": "GB/s", "cores": torch.get_num_threads(),
            "kind": "port", "sample": f"one act-quant + GPTQ linear, {rows} of {N_OUT} output rows, M=8, K=4096; "
                                      f"median of 3 ({t:.2f} s)"}


def run_reference_decode(args):
    """The reference arm of the decode workload, on the repo arm's config: the reference's eager chain for the
    whole decode step (drafts of the tree, the verify of its 8 rows through all 32 layers, lm_head, greedy accept,
    replay) restated as torch-CPU eager ops (oracle/cpu_decode.py; the reference's own chain is XPU torch / oneDNN
    and cannot run here), on all the host's cores. W untimed steps, then the timed steps actually run (at most
    --steps; fewer if 150 s of timed work is spent: `steps` reports the count timed). value = committed tokens /
    the time of the timed steps."""
    warm = min(args.warmup, 2)
    times, toks, threads, build = _cpu_decode_run(args.prompt, warmup=warm, steps=args.steps, budget_s=150.0)
    total = sum(times)
    value = toks / total
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 4), "unit": "tok/s", "n_gpus": 1,
            "steps": len(times), "steps_requested": args.steps, "warmup": warm,
            "ms_per_step": round(total / len(times) * 1e3, 2), "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "int8", "data": "synthetic (random-init Qwen3.5-9B-shaped W4A8 weights, seeded)",
            "config": {"workload": f"Qwen3.5-9B-shaped W4A8 MTP decode (configs[4]): 8-node tree4s1m8 draft tree of "
                                   f"depth 4 (bf16 MTP head, bf16 lm_head), 8 verify rows, greedy accept, prompt "
                                   f"{args.prompt}, 1 stream",
                       "layers": 32, "tokens_per_step": round(toks / len(times), 3),
                       "engine": "torch-CPU eager ops (oracle/cpu_decode.py)", "model_build_s": round(build, 1)},
            "cpu_baseline": {"value": round(value, 4), "unit": "tok/s", "cores": threads, "kind": "port",
                             "sample": f"{len(times)} whole decode steps of the same model and tree, all timed "
                                       f"({total:.1f} s)"},
            "e2e": {"value": round(value, 4), "unit": "tok/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def run_reference(args):
    rank, world, _ = dist_setup(args.gpus)
    if rank != 0:
        return
    if args.workload == "decode":
        return run_reference_decode(args)
    from oracle import w4a8 as ow
    packed, scales = ow.gen_gptq(N_OUT, K_IN, seed=0x5EED)
    rows = 1024
    import numpy as np
    import torch
    torch.set_num_threads(os.cpu_count() or 1)
    g = torch.Generator().manual_seed(7)
    x = torch.randn(M_ROWS, K_IN, generator=g).to(torch.bfloat16).view(torch.int16).numpy().view(np.uint16)

    def step():
        q, s = ow.act_quant(x)
        ow.gptq_linear(q, s, packed[:rows], scales[:rows])

    for _ in range(args.warmup):
        step()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        step()
    t = time.perf_counter() - t0
    value = args.steps * gemv_bytes(M_ROWS, rows, K_IN) / t / 1e9
    line = {"impl": "reference", "metric": METRIC, "value": round(value, 3), "unit": "GB/s", "n_gpus": world,
            "steps": args.steps, "warmup": args.warmup, "ms_per_step": round(t * 1e3 / args.steps, 3),
            "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "int8",
            "data": "synthetic (seeded, BASELINE configs[0] distributions)",
            "config": {"workload": "W4A8 GPTQ verify linear 4096->12288, M=8 rows (configs[0])"},
            "cpu_baseline": {"value": round(value, 3), "unit": "GB/s", "cores": torch.get_num_threads(), "kind": "port",
                             "sample": f"per step one act-quant + GPTQ linear over {rows} of {N_OUT} output rows"},
            "e2e": {"value": round(value, 3), "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0}}
    print(json.dumps(line), flush=True)


def main():
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=None, help="default: 200 (decode), 2000 (gemv, mlp)")
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", default="ours", choices=["ours", "reference"])
    ap.add_argument("--workload", default="decode", choices=["gemv", "mlp", "decode", "topk_rows", "lmhead"])
    ap.add_argument("--prompt", type=int, default=1024, help="decode: committed prompt length (KV prefix)")
    ap.add_argument("--rows", type=int, default=8, help="activation rows (tree-verify rows)")
    ap.add_argument("--no-batched", action="store_true", help="decode: skip the 2- and 4-stream batched measurements")
    ap.add_argument("--streams", type=int, default=1,
                    help="decode: independent streams per GPU batched in one step (up to 4: 32 verify rows)")
    ap.add_argument("--no-cpu", action="store_true", help="skip the cpu_baseline leg")
    ap.add_argument("--no-second-prompt", action="store_true", help="decode: skip the prompt-4096 measurement")
    ap.add_argument("--trace", action="store_true", help="mlp: add the fused kernel's phase trace to config")
    ap.add_argument("--tp", action="store_true",
                    help="decode: one stream in tensor parallel over the --gpus ranks (mono_b200.tp) instead of replicas")
    ap.add_argument("--profile-step", action="store_true",
                    help="decode: run one eager step between cudaProfilerStart / Stop (for ncu --profile-from-start off)")
    ap.add_argument("--programs", action="store_true",
                    help="decode: run the verify body as layer programs (one persistent launch per run of layers) "
                         "instead of one launch per fused op")
    ap.add_argument("--prefetch", type=int, default=0, help="decode: L2 look-ahead of the layer programs (items)")
    ap.add_argument("--cublas-draft", action="store_true",
                    help="decode: the MTP head's bf16 projections on cuBLAS (F.linear) instead of mono_gemv_bf16")
    args = ap.parse_args()
    if args.steps is None:
        args.steps = 200 if args.workload == "decode" else 2000
    if args.warmup < 3:
        args.warmup = 3
    if args.impl == "reference":
        run_reference(args)
    elif args.workload == "mlp":
        run_mlp(args)
    elif args.workload == "decode" and args.tp:
        run_decode_tp(args)
    elif args.workload == "decode":
        run_decode(args)
    elif args.workload == "topk_rows":
        run_topk_rows(args)
    elif args.workload == "lmhead":
        run_lmhead(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
