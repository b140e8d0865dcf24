#!/usr/bin/env python
"""Benchmark of the quantized-linear forward (QuantizedLinear.forward) on B200.

Default workload: 3-bit RVQ linear (E8P 2-bit stage +
1-bit E8 residual stage), in=4096 -> out=11008, RFFT incoherence on both sides
(2048-point FFT in, 5504-point IFFT out), fp16 activations N(0,1), batch 1.

A step pushes one batch of tokens through a stack of `--stack` quantized
linears of that shape (independent layers, same input), cycling over L distinct
weight copies whose total size (> 2x the 126 MB L2) keeps every weight read an
HBM read.  value = tokens x layers / s, i.e. the per-layer token throughput.

Prints one JSON line (rank 0).  `--impl reference` times the CPU port of the
reference algorithm (oracle/, numpy, all host cores) on the same workload.
"""
from __future__ import annotations

import argparse
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


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=20)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--config", default="c2_rvq3_4096to11008")
    p.add_argument("--batch", type=int, default=1)
    p.add_argument("--stack", type=int, default=8192, help="layers per step")
    p.add_argument("--cpu-sample-s", type=float, default=15.0)
    return p.parse_args()


def dist_env():
    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    return world, rank, local


def measured_peaks():
    path = os.path.join(ROOT, "MEASURED_PEAKS.json")
    try:
        with open(path) as f:
            d = json.load(f)
        return float(d["hbm_gbs"]), float(d["bf16_tflops"]), "measured"
    except Exception:
        return 6650.0, 1590.0, "fallback"


class ClockSampler:
    """nvidia-smi clocks / throttle reasons sampled every 200 ms while running."""

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
        except Exception:
            self.proc = None
        return self

    def _read(self):
        for line in self.proc.stdout:
            self.lines.append(line.strip())

    def __exit__(self, *exc):
        if self.proc is not None:
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
    from quipsharp_b200 import synthetic as syn
    spec = syn.CONFIGS[name]
    assert len(spec["layers"]) == 1, "bench workload is a single-layer-shape config"
    _, m, n = spec["layers"][0]
    return m, n, spec["kinds"], spec["dtype"]


def algorithmic_bytes(m, n, kinds, batch, elem=2):
    """Survey 8(d): codes at the paper bit rate (2 bits/weight per E8P stage,
    1 bit/weight per 1-bit stage) + activations in + outputs out + transform
    vectors (+ nothing for bias here)."""
    bits = sum(2 if k == "e8p" else 1 for k in kinds)
    return m * n * bits // 8 + batch * n * elem + batch * m * elem + (m + n) * 4


def gemv_bytes(m, n, kinds, batch):
    """Bytes the fused decode+matmul kernel must move per launch: packed codes
    (= the paper bit rate), fp16 transformed activations, fp32 y1 updates."""
    bits = sum(2 if k == "e8p" else 1 for k in kinds)
    return m * n * bits // 8 + batch * n * 2 + batch * m * 4


def cpu_oracle_forward(m, n, kinds, batch, dtype):
    """A callable running the numpy port of the reference forward (oracle/)
    on one synthetic layer of the workload's shape, on this host's cores."""
    from oracle import quipsharp_oracle as O
    from quipsharp_b200 import synthetic as syn
    lay = syn.make_layer(m, n, kinds, seed=1)
    x = syn.make_activations(batch, n, dtype=dtype, seed=2).float().numpy()
    t = lambda v: None if v is None else v.numpy()
    args = dict(su=t(lay.su), sv=t(lay.sv), phase_u=t(lay.phase_u), phase_v=t(lay.phase_v))
    ss = None if lay.num_stages == 1 else list(lay.stage_scales)
    codes = lay.codes.numpy()
    return lambda: O.linear_forward(x, codes, list(lay.kinds), ss, lay.layer_scale, lay.transform_kind, **args)


def cpu_oracle_forward_time(m, n, kinds, batch, dtype, budget_s, warmup=2):
    run = cpu_oracle_forward(m, n, kinds, batch, dtype)
    for _ in range(warmup):
        run()
    times = []
    t_end = time.perf_counter() + budget_s
    while not times or time.perf_counter() < t_end:
        t0 = time.perf_counter()
        run()
        times.append(time.perf_counter() - t0)
    return statistics.median(times), len(times)


def run_reference(args):
    world, rank, local = dist_env()
    if rank != 0:
        return
    m, n, kinds, dtype = config_spec(args.config)
    run = cpu_oracle_forward(m, n, kinds, args.batch, dtype)
    for _ in range(args.warmup):
        run()
    per_step = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        run()
        per_step.append(time.perf_counter() - t0)
    total = sum(per_step)
    value = args.batch * len(per_step) / total
    cores = os.cpu_count()
    line = {
        "impl": "reference", "metric": f"quantized-linear tokens/s ({args.config}, batch {args.batch})",
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * total / len(per_step), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.config, "batch": args.batch, "m": m, "n": n, "kinds": list(kinds),
                   "step": "one full forward of one layer on the host CPU"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{len(per_step)} full forwards (numpy port of the reference algorithm, "
                                   f"oracle/quipsharp_oracle.py), BLAS threads = all {cores} host cores"},
        "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


def run_ours(args):
    import torch
    import torch.distributed as dist
    from quipsharp_b200 import _native as N
    from quipsharp_b200 import synthetic as syn
    from quipsharp_b200.checkpoint import QuantizedLinear
    from quipsharp_b200.codebooks import E8PCodebook, E8OneBitCodebook
    from quipsharp_b200.quantize import RVQCodebookAdapter
    from quipsharp_b200.rvq import RVQStage

    world, rank, local = dist_env()
    if world > 1:
        import datetime
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    m, n, kinds, dtype = config_spec(args.config)
    B = args.batch

    # ---- L distinct layer copies whose packed weights exceed 2x L2
    base = syn.make_layer(m, n, kinds, seed=1)
    karr = N.int_array([N.QS_CB_E8P if k == "e8p" else N.QS_CB_E8_1BIT for k in kinds])
    packed_bytes = N.lib().qs_packed_bytes(len(kinds), karr, m, n)
    L = max(2, math.ceil(2 * L2_BYTES / packed_bytes))
    cb = lambda k: E8PCodebook() if k == "e8p" else E8OneBitCodebook()
    codebook = cb(kinds[0]) if len(kinds) == 1 else RVQCodebookAdapter(
        [RVQStage(cb(k), s) for k, s in zip(kinds, base.stage_scales)])
    codes0 = base.codes.to(dev)
    mods = []
    for l in range(L):
        mod = QuantizedLinear(n, m, 8, base.transform_kind, num_stages=len(kinds)).to(dev)
        with torch.no_grad():
            c = codes0.clone()
            if c.dim() == 2:
                c ^= (l * 0x9E37 + rank * 0x3B1) & 0x7FFF
            else:
                c[0] ^= (l * 0x9E37 + rank * 0x3B1) & 0x7FFF
                c[1] ^= (l * 37 + rank) & 0xFF if kinds[1] == "e8_1bit" else (l * 0x9E37) & 0x7FFF
            mod.codes.copy_(c)
            mod.scale.fill_(base.layer_scale)
            if base.transform_kind == "rht":
                mod.su.copy_(base.su)
                mod.sv.copy_(base.sv)
            else:
                mod.phase_u.copy_(base.phase_u)
                mod.phase_v.copy_(base.phase_v)
        mod.codebook = codebook
        mod.kernel()  # pack once, outside every timed region
        mods.append(mod)
    del codes0
    kern = [md.kernel() for md in mods]
    S = args.stack
    R = max(1, S // L)
    S = R * L
    stream = torch.cuda.Stream(dev)
    x_host = syn.make_activations(B, n, dtype=dtype, seed=2).pin_memory()
    x_dev = torch.empty(B, n, dtype=dtype, device=dev)
    x_dev.copy_(x_host)
    y_dev = torch.empty(L, B, m, dtype=dtype, device=dev)
    y_host = torch.empty(L, B, m, dtype=dtype).pin_memory()

    # ---- direct C-ABI pass (value): input -> matmul -> output per layer
    ws_in_b = N.lib().qs_linear_input_bytes(B, n)
    ws_in = torch.empty(ws_in_b, dtype=torch.uint8, device=dev)
    y1 = torch.empty(B, m, dtype=torch.float32, device=dev)
    kc = [(k, k._kinds_c, k._ss_c) for k in kern]
    io = N.IO_DTYPES[dtype]

    def one_pass(s, matmul_only=False):
        for k, kinds_c, ss_c in kc:
            if not matmul_only:
                N.check(N.lib().qs_linear_input(N.ptr(x_dev), io, B, n, k.transform, N.ptr(k.sv), N.ptr(k.phase_v),
                                                N.ptr(ws_in), ws_in_b, N.ptr(y1), m, s))
            N.check(N.lib().qs_linear_matmul(N.ptr(ws_in), B, n, m, N.ptr(k.packed), len(k.kinds), kinds_c, ss_c,
                                             N.ptr(k.scale), N.ptr(y1), s))
            if not matmul_only:
                N.check(N.lib().qs_linear_output(N.ptr(y1), m, 1, B, m, k.transform, N.ptr(k.su), N.ptr(k.phase_u),
                                                 N.ptr(k.bias), N.ptr(y_dev[0]), io, s))

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            fn(stream.cuda_stream)  # warm (sets kernel attributes)
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(g, stream=stream):
                fn(stream.cuda_stream)
        torch.cuda.synchronize(dev)
        return g

    g_pass = capture(lambda s: one_pass(s))
    g_mm = capture(lambda s: one_pass(s, matmul_only=True))

    def barrier():
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize(dev)

    def timed(fn, steps, warmup):
        for _ in range(warmup):
            fn()
        barrier()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        for _ in range(steps):
            fn()
        e1.record(stream)
        barrier()
        ms = e0.elapsed_time(e1)
        if world > 1:
            t = torch.tensor([ms], device=dev)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms = float(t.item())
        return ms

    def step_value():
        with torch.cuda.stream(stream):
            for _ in range(R):
                g_pass.replay()

    # ---- value: device-resident inputs, graph of L layers x R passes per step
    with ClockSampler(local) as clk:
        ms_total = timed(step_value, args.steps, args.warmup)
    ms_step = ms_total / args.steps
    tokens = B * S * args.steps * world
    value = tokens / (ms_total / 1e3)

    # ---- dominant kernel: fused decode+matmul, timed alone on the same stream
    def step_mm():
        with torch.cuda.stream(stream):
            for _ in range(R):
                g_mm.replay()
    mm_steps = max(3, args.steps // 2)
    ms_mm = timed(step_mm, mm_steps, 2)
    mm_launches = mm_steps * R * L * math.ceil(B / 8)
    us_per_mm = 1e3 * ms_mm / (mm_steps * R * L)
    hbm_peak, _, peak_kind = measured_peaks()
    gb = gemv_bytes(m, n, kinds, B)
    achieved = gb / (us_per_mm * 1e-6) / 1e9
    traffic = None
    tfile = os.path.join(ROOT, "profiles", f"traffic_{args.config}_b{B}.json")
    if os.path.exists(tfile):
        with open(tfile) as f:
            traffic = json.load(f).get("dram_bytes_per_launch")

    # ---- e2e: public module API, pinned host input in / all outputs back per step
    def fwd_all(s):
        for l, md in enumerate(mods):
            y_dev[l].copy_(md(x_dev))

    g_api = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        fwd_all(None)
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(g_api, stream=stream):
            fwd_all(None)
    torch.cuda.synchronize(dev)

    def step_e2e():
        with torch.cuda.stream(stream):
            x_dev.copy_(x_host, non_blocking=True)
            for _ in range(R):
                g_api.replay()
            y_host.copy_(y_dev, non_blocking=True)
    ms_e2e = timed(step_e2e, args.steps, args.warmup)
    e2e_value = tokens / (ms_e2e / 1e3)

    cpu = None
    if rank == 0 and world == 1:
        t, cnt = cpu_oracle_forward_time(m, n, kinds, B, dtype, budget_s=args.cpu_sample_s)
        cpu = {"value": B / t, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{cnt} full forwards of one {m}x{n} layer, batch {B} (numpy port of the reference "
                         f"algorithm, oracle/quipsharp_oracle.py), median time {t:.3f} s"}

    if rank == 0:
        c = clk.summary()
        bits = sum(2 if k == "e8p" else 1 for k in kinds)
        line = {
            "metric": f"quantized-linear tokens/s ({args.config}, batch {B})",
            "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
            "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak", "vs_baseline": None,
            "dtype": "f16", "data": "synthetic",
            "config": {"workload": args.config, "batch": B, "m": m, "n": n, "kinds": list(kinds),
                       "transform": base.transform_kind, "layers_per_step": S, "distinct_layer_copies": L,
                       "weight_bytes_cycled": L * packed_bytes,
                       "l2": f"inputs larger than L2: {L} distinct layer copies = {L * packed_bytes / 1e6:.0f} MB "
                             f"of packed weights cycled per pass (L2 126 MB)",
                       "bits_per_weight": bits},
            "hbm_gbs_per_layer_forward": algorithmic_bytes(m, n, kinds, B) * S * args.steps / (ms_total / 1e3) / 1e9,
            "us_per_layer_forward": 1e3 * ms_step / S,
            "roofline": {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                         "frac": achieved / hbm_peak, "traffic": traffic,
                         "kernel": "qs::gemv_kernel (fused decode + mma.sync matmul)",
                         "algorithmic_bytes_per_launch": gb, "us_per_launch": us_per_mm,
                         "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"},
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": B * n * 2,
                    "d2h_bytes_per_step": L * B * m * 2,
                    "path": "QuantizedLinear.forward (public module) x layers per step, replayed as a CUDA graph; "
                            "pinned host input copied in and all layer outputs copied out each step"},
            "gpu_launches": args.steps * R * L * (2 + math.ceil(B / 8)),
            "clocks": {"sm_mhz": c["sm_mhz"], "sm_max_mhz": c["sm_max_mhz"], "reasons": c["reasons"]},
        }
        print(json.dumps(line), flush=True)
    del g_pass, g_mm, g_api
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
