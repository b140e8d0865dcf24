#!/usr/bin/env python
"""Benchmark of the quantized-linear forward path (QuantizedLinear.forward) on B200.

Default workload (the configuration the multi-GPU
scaling claim is made on): the seven linears of a Llama-3-70B-shaped decoder
layer (q, o 8192->8192; k, v 8192->1024; gate, up 8192->28672; down
28672->8192) as 3-bit RVQ (E8P 2-bit + 1-bit residual), random codes / signs /
stage scales from seeds, bf16 activations N(0,1), decode batch 1.  A step
pushes one batch through the whole layer set in decoder order, each layer
taking the latest earlier output of its input width (q takes the layer input;
k, v and o take q's output in place of the attention input / output; gate and up
take o's output; down takes up's output in place of act(gate) * up).

One GPU runs the layers unsharded; layers that read one input (k, v, o here,
as q, k, v in a decoder; gate and up) run as one group (groups.LinearGroup:
qs_linear_fwd_group overlaps their kernels on forked streams; --groups off
runs each layer's forward in turn).  N GPUs (torchrun, one process per GPU) run
them column-sharded over output rows (TPQuantizedLinear: each rank decodes and
multiplies its rows, its matmul CTAs push the float32 row shard into every
rank's receive buffer over NVLink as self-validating words, and every rank
applies the full output transform to the gathered rows): strong scaling, the
same tokens per step at every N.
Each rank cycles over enough distinct weight copies that its weights exceed
twice the 126 MB L2 (every weight read is an HBM read).

value: tokens through the layer set per second, CUDA-graph replay of the
modules' forward, CUDA events on the launching stream, max over ranks.
e2e: the same through the public module called eagerly from Python (no graph),
with the pinned host input copied in and the output copied back every step.
roofline: the fused decode + matmul kernel of the set, timed alone.
At one GPU the line also carries `decode_c2` (3-bit RVQ
4096 -> 11008 at batch 1) and `prefill_c4` (Qwen2.5-7B MLP
at 2048 tokens) sub-records, and with --breakdown the per-step timings of the
layer set (transforms / matmuls / each layer's input and output step).  `--impl reference` times the CPU port of the
reference algorithm (oracle/, numpy, all host cores) on the same workload.
Prints one JSON line (rank 0).
"""
from __future__ import annotations

import argparse
import datetime
import json
import math
import os
import statistics
import subprocess
import sys
import threading
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, ROOT)

L2_BYTES = 126 * 1024 * 1024
DEFAULT_CONFIG = "c5_llama3_70b_rvq3"


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=10)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--config", default=DEFAULT_CONFIG)
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--passes", type=int, default=0,
                   help="layer-set passes per step (0: about 2k layer forwards per step at decode batches)")
    p.add_argument("--cpu-sample-s", type=float, default=20.0)
    p.add_argument("--no-extras", action="store_true", help="skip the decode_c2 / prefill_c4 sub-records")
    p.add_argument("--groups", default="on", choices=["on", "off"],
                   help="one GPU: run the layers that read one input as one group (groups.LinearGroup); "
                        "off: each layer's forward in turn")
    p.add_argument("--breakdown", action="store_true",
                   help="one GPU: add per-step timings of the layer set (input / matmul / output steps)")
    return p.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks():
    """(hbm GB/s, bf16 burst TFLOP/s, bf16 sustained TFLOP/s, source)."""
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), float(d.get("bf16_tflops_sustained", 1400.0)), "measured"
    except Exception:
        return 6650.0, 1590.0, 1400.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running.  Entry
    waits for the first reading and exit for one more, so even a timed region shorter
    than the sampling period is bracketed by readings."""

    FIELDS = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
              "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
              "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, gpu_index: int):
        self.gpu = gpu_index
        self.proc = None
        self.lines = []

    def __enter__(self):
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", f"--query-gpu={self.FIELDS}", "--format=csv,noheader,nounits",
                 "-lms", "200", "-i", str(self.gpu)], stdout=subprocess.PIPE, stderr=subprocess.DEVNULL,
                text=True)
            self.t = threading.Thread(target=self._read, daemon=True)
            self.t.start()
            t0 = time.time()
            while not self.lines and time.time() - t0 < 5.0 and self.proc.poll() is None:
                time.sleep(0.02)
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
            n0, t0 = len(self.lines), time.time()
            while len(self.lines) <= n0 and time.time() - t0 < 1.0 and self.proc.poll() is None:
                time.sleep(0.02)
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except Exception:
                self.proc.kill()

    def summary(self):
        sm, mx, reasons = [], None, set()
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        for ln in self.lines:
            parts = [p.strip() for p in ln.split(",")]
            if len(parts) < 9:
                continue
            try:
                sm.append(float(parts[1]))
                mx = float(parts[2])
            except ValueError:
                continue
            for nm, v in zip(names, parts[5:9]):
                if v.lower() == "active":
                    reasons.add(nm)
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": mx,
                "reasons": sorted(reasons), "samples": len(sm)}


def config_spec(name):
    """(layers [(name, m, n)], kinds, dtype) of a BASELINE configuration."""
    from quipsharp_b200 import synthetic as syn
    spec = syn.CONFIGS[name]
    return spec["layers"], spec["kinds"], spec["dtype"]


def layer_sources(layers):
    """Input of each layer of a set: the latest earlier layer output of matching
    width, else the set's input (-1).  In decoder order this gives q <- input;
    k, v, o <- q; gate, up <- o; down <- up."""
    src, latest = [], {}
    for li, (_, m, n) in enumerate(layers):
        src.append(latest.get(n, -1))
        latest[m] = li
    return src


def gemv_bytes(m, n, kinds, batch):
    """Bytes the fused decode+matmul kernel must move per launch: packed codes
    (= the paper bit rate), fp16 transformed activations, fp32 y1 updates."""
    bits = sum(2 if k == "e8p" else 1 for k in kinds)
    return m * n * bits // 8 + batch * n * 2 + batch * m * 4


def _two_pass_width(N):
    """The library's two-pass RFFT width rule (qs_xform2.cu two_pass_rfft)."""
    if N < 4096:
        return False
    P = 0
    for q in (43, 41, 37, 31, 29, 23, 19, 17, 13, 11, 7, 5, 3):
        if N % q == 0:
            if P:
                return False
            P = q
    if not P or (N // P) % P == 0:
        return False
    N1 = N // P
    return N1 >= 64 and N1 & (N1 - 1) == 0


def kernels_per_forward(m, n, batch, sms, shards=1):
    """This library's kernel launches for one forward of an (n -> m) layer (m the full
    output width): input transform (two kernels for a two-pass RFFT width), matmul
    (batches 9-32: one launch per 16 tokens), with shards > 1 at prefill batches
    the push of the row shard to every rank, output transform (two kernels for a two-pass width; the
    gathered output step of a sharded layer is one kernel)."""
    pow2 = lambda v: v & (v - 1) == 0
    matmul = 1 if batch >= 33 or batch <= 8 else math.ceil(batch / 16)
    push = 1 if shards > 1 and batch >= 33 else 0  # decode batches: the matmul pushes
    if pow2(m) and pow2(n):
        return 1 + matmul + push + 1
    inp = 2 if _two_pass_width(n // 2) and (batch >= 33 or 2 * batch <= sms) else 1
    out = 2 if shards == 1 and _two_pass_width(m // 2) else 1
    return inp + matmul + push + out


def load_traffic_table():
    """DRAM bytes per launch set of the fused decode+matmul, measured with ncu and
    recorded in profiles/gemv_dram_traffic.md (lines `traffic <config> <batch> <world>
    <bytes>`).  Returns {(config, batch, world): bytes}."""
    out = {}
    try:
        with open(os.path.join(ROOT, "profiles", "gemv_dram_traffic.md")) as f:
            for line in f:
                parts = line.strip().strip("`").split()
                if len(parts) == 5 and parts[0] == "traffic":
                    out[(parts[1], int(parts[2]), int(parts[3]))] = float(parts[4])
    except OSError:
        pass
    return out


# ---------------------------------------------------------------- CPU (reference port)
def cpu_oracle_forward(m, n, kinds, batch, dtype, seed=1):
    """A callable running the numpy port of the reference forward (oracle/) on one
    synthetic layer of the workload's shape, on this host's cores."""
    from oracle import quipsharp_oracle as O
    from quipsharp_b200 import synthetic as syn
    lay = syn.make_layer(m, n, kinds, seed=seed)
    x = syn.make_activations(batch, n, dtype=dtype, seed=2).float().numpy()
    t = lambda v: None if v is None else v.numpy()
    args = dict(su=t(lay.su), sv=t(lay.sv), phase_u=t(lay.phase_u), phase_v=t(lay.phase_v))
    ss = None if lay.num_stages == 1 else list(lay.stage_scales)
    codes = lay.codes.numpy()
    return lambda: O.linear_forward(x, codes, list(lay.kinds), ss, lay.layer_scale, lay.transform_kind, **args)


def cpu_set_time(layers, kinds, batch, dtype, budget_s):
    """Median time of whole passes over the layer set (numpy port), within budget_s
    after one warm-up pass (at least one timed pass)."""
    runs = [cpu_oracle_forward(m, n, kinds, batch, dtype, seed=1 + li) for li, (_, m, n) in enumerate(layers)]
    for r in runs:
        r()
    times, t_end = [], time.perf_counter() + budget_s
    while not times or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        for r in runs:
            r()
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times)


def run_reference(args):
    world, rank, local = dist_env()
    if rank != 0:
        return
    layers, kinds, dtype = config_spec(args.config)
    runs = [cpu_oracle_forward(m, n, kinds, args.batch, dtype, seed=1 + li) for li, (_, m, n) in enumerate(layers)]
    for _ in range(args.warmup):
        for run in runs:
            run()
    per_step = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for run in runs:
            run()
        per_step.append(time.perf_counter() - t0)
    total = sum(per_step)
    value = args.batch * len(per_step) / total
    cores = os.cpu_count()
    sample = (f"{len(per_step)} timed passes (after {args.warmup} warm-up) over the full {len(layers)}-layer set, "
              f"batch {args.batch}: numpy port of the reference algorithm (oracle/quipsharp_oracle.py), "
              f"BLAS threads = all {cores} host cores")
    line = {
        "impl": "reference", "metric": f"quantized-linear tokens/s ({args.config} layer set, batch {args.batch})",
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * total / len(per_step), "higher_is_better": True,
        "scaling": "strong" if args.gpus > 1 else "weak", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.config, "batch": args.batch, "layers": [list(l) for l in layers],
                   "kinds": list(kinds), "step": "one forward of every layer of the set on the host CPU"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port", "sample": sample},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------- GPU
def make_full_module(name, m, n, kinds, li, copy_id, dev, chained):
    """A QuantizedLinear filled from a seeded synthetic layer; copy_id varies the codes
    so distinct copies are distinct weights."""
    import torch
    from quipsharp_b200 import synthetic as syn
    from quipsharp_b200.checkpoint import QuantizedLinear
    from quipsharp_b200.codebooks import E8PCodebook, E8OneBitCodebook
    from quipsharp_b200.quantize import RVQCodebookAdapter
    from quipsharp_b200.rvq import RVQStage
    base = syn.make_layer(m, n, kinds, seed=1 + li, layer_scale=(1.0 / math.sqrt(1.2 * n)) if chained else None)
    mod = QuantizedLinear(n, m, 8, base.transform_kind, num_stages=len(kinds)).to(dev)
    with torch.no_grad():
        c = base.codes.to(dev)
        if copy_id:
            if c.dim() == 2:
                c ^= (copy_id * 0x9E37) & 0x7FFF
            else:
                c[0] ^= (copy_id * 0x9E37) & 0x7FFF
                c[1] ^= (copy_id * 37) & 0xFF if kinds[1] == "e8_1bit" else (copy_id * 0x9E37) & 0x7FFF
        mod.codes.copy_(c)
        mod.scale.fill_(base.layer_scale)
        if base.transform_kind == "rht":
            mod.su.copy_(base.su)
            mod.sv.copy_(base.sv)
        else:
            mod.phase_u.copy_(base.phase_u)
            mod.phase_v.copy_(base.phase_v)
    cb = lambda k: E8PCodebook() if k == "e8p" else E8OneBitCodebook()
    mod.codebook = cb(kinds[0]) if len(kinds) == 1 else RVQCodebookAdapter(
        [RVQStage(cb(k), sc) for k, sc in zip(kinds, base.stage_scales)])
    return mod


class LayerSet:
    """Copies of a config's layer set on this rank (sharded when world > 1)."""

    def __init__(self, config, batch, dev, world, rank, copies=None, groups=False):
        import torch
        from quipsharp_b200 import _native as N
        from quipsharp_b200.groups import LinearGroup
        from quipsharp_b200.tensor_parallel import TPQuantizedLinear
        self.layers, self.kinds, self.dtype = config_spec(config)
        self.config, self.B, self.dev, self.world = config, batch, dev, world
        self.prefill = batch >= 33
        self.src = layer_sources(self.layers)
        karr = N.int_array([N.QS_CB_E8P if k == "e8p" else N.QS_CB_E8_1BIT for k in self.kinds])
        self.rank_bytes = sum(N.lib().qs_packed_bytes(len(self.kinds), karr, m // world, n)
                              for _, m, n in self.layers)
        if copies is None:
            copies = 1 if self.prefill else max(1, math.ceil(2 * L2_BYTES / self.rank_bytes))
        self.L = copies
        chained = len(self.layers) > 1
        self.mods = []  # [copy][layer]
        for c in range(copies):
            row = []
            for li, (name, m, n) in enumerate(self.layers):
                full = make_full_module(name, m, n, self.kinds, li, c * 131 + rank * 7 + 1, dev, chained)
                if world > 1:
                    row.append(TPQuantizedLinear(full))
                    del full
                else:
                    full.kernel()  # pack once, outside every timed region
                    row.append(full)
            self.mods.append(row)
        # layers that read one input run as one group (one GPU only: the tensor-
        # parallel matmuls wait on a grid barrier and must not share the GPU)
        self.group_of = {}  # first member -> member indices
        if groups and world == 1:
            by_src = {}
            for li, s in enumerate(self.src):
                by_src.setdefault(s, []).append(li)
            self.group_of = {members[0]: members for members in by_src.values() if len(members) > 1}
        self.groups = [{first: LinearGroup([row[j] for j in members]) for first, members in self.group_of.items()}
                       for row in self.mods]
        torch.cuda.synchronize(dev)

    def group_names(self):
        return [[self.layers[j][0] for j in members] for members in self.group_of.values()]

    def forward(self, x, copy):
        outs = [None] * len(self.layers)
        for li, mod in enumerate(self.mods[copy]):
            if outs[li] is not None:  # computed with its group
                continue
            inp = x if self.src[li] < 0 else outs[self.src[li]]
            members = self.group_of.get(li)
            if members:
                for j, y in zip(members, self.groups[copy][li](inp)):
                    outs[j] = y
            else:
                outs[li] = mod(inp)
        return outs[-1]

    def kernels(self, li, copy):
        mod = self.mods[copy][li]
        return mod.local if self.world > 1 else mod.kernel()


def _timed(fn, steps, warmup, stream, dev, world):
    import torch
    import torch.distributed as dist
    for _ in range(warmup):
        fn()
    if world > 1:
        dist.barrier()
    torch.cuda.synchronize(dev)
    e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    e0.record(stream)
    for _ in range(steps):
        fn()
    e1.record(stream)
    torch.cuda.synchronize(dev)
    if world > 1:
        dist.barrier()
    ms = e0.elapsed_time(e1)
    if world > 1:
        t = torch.tensor([ms], device=dev)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        ms = float(t.item())
    return ms


def _capture(fn, stream, dev):
    import torch
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        fn()  # warm (kernel attributes, packing, communicators)
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(g, stream=stream):
            out = fn()
    torch.cuda.synchronize(dev)
    return g, out


def measure_set(ls, steps, warmup, stream, dev, world, passes, clocks=None):
    """value (graph replay of the modules), matmul-only timing, eager e2e and graph
    e2e for one LayerSet.  Returns a dict of raw timings."""
    import torch
    from quipsharp_b200 import _native as N
    from quipsharp_b200 import synthetic as syn
    B, L = ls.B, ls.L
    n_in = ls.layers[0][2]
    x_host = syn.make_activations(B, n_in, dtype=ls.dtype, seed=2).pin_memory()
    x_dev = torch.empty(B, n_in, dtype=ls.dtype, device=dev)
    x_dev.copy_(x_host)
    # fail fast on a broken pipeline (a bounded wait that ran out)
    with torch.no_grad():
        ls.forward(x_dev, 0)
    torch.cuda.synchronize(dev)
    N.check(N.lib().qs_device_status(torch.cuda.current_stream(dev).cuda_stream))

    def one_step():
        y = None
        for _ in range(passes):
            for c in range(L):
                y = ls.forward(x_dev, c)
        return y

    with torch.no_grad():
        g_step, y_graph = _capture(one_step, stream, dev)

        def replay():
            with torch.cuda.stream(stream):
                g_step.replay()
        if clocks is not None:
            with clocks:
                ms_value = _timed(replay, steps, warmup, stream, dev, world)
        else:
            ms_value = _timed(replay, steps, warmup, stream, dev, world)

        # matmul-only: every layer's fused decode + matmul on this rank's rows
        ws, y1 = {}, {}
        for li, (_, m, n) in enumerate(ls.layers):
            k = ls.kernels(li, 0)
            if n not in ws:
                x = torch.randn(B, n, device=dev).to(ls.dtype)
                ws[n] = k.input(x, None)
            y1[li] = torch.empty(B, k.m, dtype=torch.float32, device=dev)

        def mm_step():
            for _ in range(passes):
                for c in range(L):
                    for li, (_, m, n) in enumerate(ls.layers):
                        ls.kernels(li, c).matmul(ws[n], B, y1[li])
        g_mm, _ = _capture(mm_step, stream, dev)

        def replay_mm():
            with torch.cuda.stream(stream):
                g_mm.replay()
        mm_steps = max(3, steps // 2)
        ms_mm = _timed(replay_mm, mm_steps, 2, stream, dev, world)

        # e2e: the public module called eagerly, host input in and output out per step
        y_host = torch.empty(B, ls.layers[-1][1], dtype=ls.dtype).pin_memory()

        def eager():
            with torch.cuda.stream(stream):
                x_dev.copy_(x_host, non_blocking=True)
                y = one_step()
                y_host.copy_(y, non_blocking=True)
        ms_e2e = _timed(eager, steps, max(2, warmup), stream, dev, world)

        def graph_e2e():
            with torch.cuda.stream(stream):
                x_dev.copy_(x_host, non_blocking=True)
                g_step.replay()
                y_host.copy_(y_graph, non_blocking=True)
        ms_e2e_graph = _timed(graph_e2e, steps, warmup, stream, dev, world)
    del g_step, g_mm
    return dict(ms_value=ms_value, ms_mm=ms_mm, mm_steps=mm_steps, ms_e2e=ms_e2e, ms_e2e_graph=ms_e2e_graph,
                h2d=x_host.numel() * x_host.element_size(), d2h=y_host.numel() * y_host.element_size())


def breakdown(ls, dev):
    """Where a decode step's time goes (one GPU): CUDA-graph replays of the whole
    layer set, of its transform steps alone (input + output step of every layer),
    of its matmuls alone (weights streamed from HBM: every copy of the set), and of
    each layer's input and output step repeated.  Microseconds per layer set / step."""
    import torch
    from quipsharp_b200 import _native as N
    B = ls.B
    stream = torch.cuda.Stream(dev)

    def timed(fn, R=20, reps=5):
        with torch.cuda.stream(stream):
            fn()
            torch.cuda.synchronize(dev)
            g = torch.cuda.CUDAGraph()
            with torch.cuda.graph(g, stream=stream):
                for _ in range(R):
                    fn()
            for _ in range(3):
                g.replay()
            torch.cuda.synchronize(dev)
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(reps):
                g.replay()
            e1.record(stream)
            torch.cuda.synchronize(dev)
        del g
        return e0.elapsed_time(e1) * 1e3 / (reps * R)

    xs = {n: torch.randn(B, n, device=dev).to(ls.dtype) for _, _, n in ls.layers}
    y1s, wss, ys = {}, {}, {}
    for li, (_, m, n) in enumerate(ls.layers):
        y1s[li] = torch.zeros(B, m, device=dev)
        wss[li] = ls.kernels(li, 0).input(xs[n], y1s[li])
        ys[li] = torch.empty(B, m, dtype=ls.dtype, device=dev)
    io = N.IO_DTYPES[ls.dtype]

    def in_step(li, c):
        k, n = ls.kernels(li, c), ls.layers[li][2]
        N.check(N.lib().qs_linear_input(N.ptr(xs[n]), io, B, n, k.transform, N.ptr(k.sv), N.ptr(k.phase_v),
                                        N.ptr(wss[li]), wss[li].numel(), N.ptr(y1s[li]), k.m, N.stream_of(xs[n])))

    def out_step(li, c):
        k = ls.kernels(li, c)
        N.check(N.lib().qs_linear_output(N.ptr(y1s[li]), k.m, 1, B, k.m, k.transform, N.ptr(k.su), N.ptr(k.phase_u),
                                         N.ptr(k.bias), N.ptr(ys[li]), io, N.stream_of(ys[li])))

    L, nl = ls.L, len(ls.layers)
    x0 = torch.randn(B, ls.layers[0][2], device=dev).to(ls.dtype)
    out = {"us_layer_set": timed(lambda: [ls.forward(x0, c) for c in range(L)]) / L,
           "us_transforms_only": timed(lambda: [(in_step(li, c), out_step(li, c))
                                                for c in range(L) for li in range(nl)]) / L,
           "us_matmuls_only": timed(lambda: [ls.kernels(li, c).matmul(wss[li], B, y1s[li])
                                             for c in range(L) for li in range(nl)]) / L}
    for li, (name, m, n) in enumerate(ls.layers):
        out[f"us_input_{name}"] = timed(lambda: in_step(li, 0), R=50)
        out[f"us_output_{name}"] = timed(lambda: out_step(li, 0), R=50)
    return {k: round(v, 2) for k, v in out.items()}


def default_passes(ls):
    if ls.prefill:
        return 1
    per_pass = ls.L * len(ls.layers)
    return max(1, math.ceil(2048 / per_pass))


def sub_record_decode(dev, stream):
    """BASELINE configs[1] (3-bit RVQ 4096 -> 11008, fp16, batch 1): per-layer token
    throughput and the fused decode + matmul against HBM bandwidth."""
    hbm, _, _, src = measured_peaks()
    ls = LayerSet("c2_rvq3_4096to11008", 1, dev, 1, 0)
    passes = max(1, math.ceil(4096 / ls.L))
    r = measure_set(ls, 5, 3, stream, dev, 1, passes)
    m, n = ls.layers[0][1], ls.layers[0][2]
    forwards = passes * ls.L
    us_mm = 1e3 * r["ms_mm"] / (r["mm_steps"] * forwards)
    gb = gemv_bytes(m, n, ls.kinds, 1)
    out = {"workload": "c2_rvq3_4096to11008", "batch": 1, "unit": "tokens/s",
           "value": forwards * 5 / (r["ms_value"] / 1e3), "us_per_forward": 1e3 * r["ms_value"] / (5 * forwards),
           "kernel_us": us_mm, "kernel_gbs": gb / us_mm / 1e3, "kernel_frac_hbm": gb / us_mm / 1e3 / hbm,
           "distinct_copies": ls.L, "peak_source": src}
    del ls
    return out


def sub_record_prefill(dev, stream):
    """BASELINE configs[3] (Qwen2.5-7B MLP gate, up, down as E8P 2-bit, bf16, 2048
    tokens): tokens/s, and TFLOP/s of the tcgen05 GEMM and of the whole layer set."""
    _, burst, sust, src = measured_peaks()
    ls = LayerSet("c4_qwen25_7b_prefill", 2048, dev, 1, 0)
    r = measure_set(ls, 5, 3, stream, dev, 1, 1)
    flops = sum(2.0 * 2048 * m * n for _, m, n in ls.layers)
    gemm_tf = flops * r["mm_steps"] / (r["ms_mm"] / 1e3) / 1e12
    set_tf = flops * 5 / (r["ms_value"] / 1e3) / 1e12
    out = {"workload": "c4_qwen25_7b_prefill", "batch": 2048, "unit": "tokens/s",
           "value": 2048 * 5 / (r["ms_value"] / 1e3), "ms_per_layer_set": r["ms_value"] / 5,
           "gemm_tflops": gemm_tf, "gemm_frac_burst": gemm_tf / burst, "gemm_frac_sustained": gemm_tf / sust,
           "set_tflops": set_tf, "set_frac_burst": set_tf / burst, "peak_source": src}
    del ls
    return out


def run_ours(args):
    import torch
    import torch.distributed as dist

    world, rank, local = dist_env()
    torch.cuda.set_device(local)  # before the process group: no context on another rank's GPU
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120),
                                device_id=torch.device("cuda", local))
    dev = torch.device("cuda", local)
    stream = torch.cuda.Stream(dev)
    hbm, burst, sust, peak_src = measured_peaks()

    ls = LayerSet(args.config, args.batch, dev, world, rank, groups=args.groups == "on")
    group_names = ls.group_names()
    passes = args.passes or default_passes(ls)
    clk = ClockSampler(local)
    r = measure_set(ls, args.steps, args.warmup, stream, dev, world, passes, clocks=clk)
    B = args.batch
    sets = passes * ls.L  # layer sets per step: each pass runs every weight copy once
    tokens = B * sets * args.steps
    value = tokens / (r["ms_value"] / 1e3)
    ms_step = r["ms_value"] / args.steps
    flops_set = sum(2.0 * B * m * n for _, m, n in ls.layers)
    launches_mm = r["mm_steps"] * passes * ls.L * len(ls.layers)
    us_per_mm = 1e3 * r["ms_mm"] / launches_mm
    if ls.prefill:
        achieved = flops_set / world * r["mm_steps"] * passes * ls.L / (r["ms_mm"] / 1e3) / 1e12
        roofline = {"bound": "tensor", "achieved": achieved, "peak": sust, "unit": "TFLOP/s",
                    "frac": achieved / sust, "traffic": None,
                    "kernel": "qs::gemm_tc_kernel (fused decode + tcgen05 GEMM, 128x256 tiles)",
                    "algorithmic_flops_per_layer_set_per_rank": flops_set / world, "us_per_launch": us_per_mm,
                    "peak_source": f"{peak_src} (MEASURED_PEAKS.json bf16_tflops_sustained; burst {burst})"}
    else:
        gb = sum(gemv_bytes(m // world, n, ls.kinds, B) for _, m, n in ls.layers)
        achieved = gb * r["mm_steps"] * passes * ls.L / (r["ms_mm"] / 1e3) / 1e9
        table = load_traffic_table()
        traffic, basis = table.get((args.config, B, world)), "measured at this rank count"
        if traffic is None and (args.config, B, 1) in table:  # a rank streams its m/N rows
            full = sum(gemv_bytes(m, n, ls.kinds, B) for _, m, n in ls.layers)
            traffic, basis = table[(args.config, B, 1)] * gb / full, "one-GPU capture scaled to this rank's rows"
        roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm, "unit": "GB/s", "frac": achieved / hbm,
                    "traffic": traffic,
                    "traffic_basis": "ncu dram__bytes_read.sum + dram__bytes_write.sum summed over one launch of "
                                     f"each layer of the set on one rank, {basis} (profiles/gemv_dram_traffic.md)",
                    "kernel": "qs::gemv_kernel (fused decode + mma.sync matmul)",
                    "algorithmic_bytes_per_layer_set_per_rank": gb, "us_per_launch": us_per_mm,
                    "peak_source": f"{peak_src} (MEASURED_PEAKS.json hbm_gbs)"}

    cpu = None
    if rank == 0 and world == 1 and args.cpu_sample_s > 0:
        t_set, cnt = cpu_set_time(ls.layers, ls.kinds, B, ls.dtype, args.cpu_sample_s)
        cpu = {"value": B / t_set, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{cnt} timed full passes (after one warm-up) over the {len(ls.layers)}-layer set at batch "
                         f"{B}: numpy port of the reference algorithm (oracle/quipsharp_oracle.py) on all host "
                         f"cores; median pass {t_set:.2f} s"}
    sms = torch.cuda.get_device_properties(dev).multi_processor_count
    launches = args.steps * passes * ls.L * sum(kernels_per_forward(m, n, B, sms, world) for _, m, n in ls.layers)
    copies = ls.L
    extras = {}
    if world == 1 and args.breakdown and not ls.prefill:
        extras["breakdown"] = breakdown(ls, dev)
    del ls
    if world == 1 and not args.no_extras:
        extras["decode_c2"] = sub_record_decode(dev, stream)
        extras["prefill_c4"] = sub_record_prefill(dev, stream)

    if rank == 0:
        c = clk.summary()
        layers, kinds, dtype = config_spec(args.config)
        line = {
            "metric": f"quantized-linear tokens/s ({args.config} layer set, batch {B})",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "strong" if world > 1 else "weak",
            "vs_baseline": None, "dtype": "bf16" if dtype == torch.bfloat16 else "f16", "data": "synthetic",
            "config": {"workload": args.config, "batch": B, "layers": [list(l) for l in layers], "kinds": list(kinds),
                       "parallelism": f"tp{world} (column-sharded output rows)" if world > 1 else "single GPU",
                       "layer_sets_per_step": sets,
                       "linear_groups": group_names or None,
                       "distinct_copies_per_rank": copies,
                       "l2": "inputs larger than L2: distinct weight copies cycled so each rank streams more than "
                             "2 x 126 MB per pass" if B < 33 else
                             "inputs larger than L2: activations / y1 of the batch exceed 126 MB",
                       "bits_per_weight": sum(2 if k == "e8p" else 1 for k in kinds)},
            "us_per_layer_set": 1e3 * ms_step / sets,
            "tflops": flops_set * sets * args.steps / (r["ms_value"] / 1e3) / 1e12,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": tokens / (r["ms_e2e"] / 1e3), "unit": "tokens/s", "h2d_bytes_per_step": r["h2d"],
                    "d2h_bytes_per_step": r["d2h"],
                    "path": "QuantizedLinear.forward (TPQuantizedLinear.forward at N > 1; LinearGroup.forward "
                            "for the layers of a linear group) called eagerly from Python over the layer set x "
                            "passes per step; pinned host input copied in and the last layer's output copied out "
                            "each step"},
            "e2e_graph": {"value": tokens / (r["ms_e2e_graph"] / 1e3), "unit": "tokens/s",
                          "path": "the same step captured once as a CUDA graph and replayed"},
            "gpu_launches": launches,
            "clocks": {"sm_mhz": c["sm_mhz"], "sm_max_mhz": c["sm_max_mhz"], "reasons": c["reasons"]},
        }
        line.update(extras)
        print(json.dumps(line), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
