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

# dram__bytes_read.sum + dram__bytes_write.sum per launch of the fused decode+matmul
# kernel, from the ncu capture summarised in profiles/gemv_c2_b1.md
NCU_TRAFFIC = {("c2_rvq3_4096to11008", 1): 16.98688e6}


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
    p.add_argument("--tp", action="store_true",
                   help="tensor-parallel mode (not the default contract): the config's layer set "
                        "column-sharded over the ranks, strong scaling")
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


def _two_pass_width(N):
    """The library's two-pass RFFT width rule (qs_xform2.cu two_pass_rfft): N = P * 2^a
    >= 4096 with one odd prime P <= 43 (not squared) and 2^a >= 64."""
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


def kernels_per_forward(m, n, batch, sms):
    """This library's kernel launches for one forward of an (n -> m) layer: input
    transform (two kernels for a two-pass RFFT width: many rows always, few rows in
    decode), matmul (batches 9-32: one launch per 16 tokens), output transform (two
    kernels for a two-pass width)."""
    pow2 = lambda v: v & (v - 1) == 0
    matmul = 1 if batch >= 33 or batch <= 8 else math.ceil(batch / 16)
    if pow2(m) and pow2(n):  # RHT both sides
        return 1 + matmul + 1
    inp = 2 if _two_pass_width(n // 2) and (batch >= 33 or 2 * batch <= sms) else 1
    out = 2 if _two_pass_width(m // 2) else 1
    return inp + matmul + out


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
    layers, kinds, dtype = config_spec(args.config)
    runs = [cpu_oracle_forward(m, n, kinds, args.batch, dtype) for _, m, n in layers]
    for _ in range(args.warmup):
        for run in runs:
            run()
    per_step = []
    for _ in range(args.steps):
        t0 = time.perf_counter()
        for run in runs:
            run()
        per_step.append(time.perf_counter() - t0)
    m, n = layers[0][1], layers[0][2]
    total = sum(per_step)
    value = args.batch * len(per_step) / total
    cores = os.cpu_count()
    line = {
        "impl": "reference", "metric": f"quantized-linear tokens/s ({args.config}, batch {args.batch})",
        "value": value, "unit": "tokens/s", "n_gpus": args.gpus, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": 1000 * total / len(per_step), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f32", "data": "synthetic",
        "config": {"workload": args.config, "batch": args.batch, "layers": [list(l) for l in layers],
                   "kinds": list(kinds), "step": "one full forward of every layer of the set on the host CPU"},
        "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": "port",
                         "sample": f"{len(per_step)} passes over the layer set (numpy port of the reference "
                                   f"algorithm, oracle/quipsharp_oracle.py), BLAS threads = all {cores} host cores"},
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
    layers, kinds, dtype = config_spec(args.config)
    B = args.batch
    prefill = B >= 33  # kTcMinBatch: the tcgen05 GEMM
    chained = len(layers) > 1
    karr = N.int_array([N.QS_CB_E8P if k == "e8p" else N.QS_CB_E8_1BIT for k in kinds])
    set_bytes = sum(N.lib().qs_packed_bytes(len(kinds), karr, m, n) for _, m, n in layers)
    # decode regime: cycle distinct copies of the layer set so weights always come from HBM
    L = 1 if prefill else max(1, math.ceil(2 * L2_BYTES / set_bytes))
    cb = lambda k: E8PCodebook() if k == "e8p" else E8OneBitCodebook()

    mods = []  # [copy][layer]
    for l in range(L):
        row = []
        for li, (name, m, n) in enumerate(layers):
            base = syn.make_layer(m, n, kinds, seed=1 + li,
                                  layer_scale=(1.0 / math.sqrt(1.2 * n)) if chained else None)
            mod = QuantizedLinear(n, m, 8, base.transform_kind, num_stages=len(kinds)).to(dev)
            with torch.no_grad():
                c = base.codes.to(dev)
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
            mod.codebook = cb(kinds[0]) if len(kinds) == 1 else RVQCodebookAdapter(
                [RVQStage(cb(k), sc) for k, sc in zip(kinds, base.stage_scales)])
            mod.kernel()  # pack once, outside every timed region
            row.append(mod)
        mods.append(row)
    # layers per step: whole passes over the copies, at least --stack layer forwards
    R = max(1, math.ceil(args.stack / (L * len(layers)))) if not prefill else max(1, args.stack // 8192)
    passes = R * L
    n_in = layers[0][2]
    stream = torch.cuda.Stream(dev)
    x_host = syn.make_activations(B, n_in, dtype=dtype, seed=2).pin_memory()
    x_dev = torch.empty(B, n_in, dtype=dtype, device=dev)
    x_dev.copy_(x_host)
    io = N.IO_DTYPES[dtype]

    # ---- buffers of the direct C-ABI pass (value): chain each layer's input by dimension
    max_in = max(n for _, _, n in layers)
    max_out = max(m for _, m, _ in layers)
    ws_in_b = max(N.lib().qs_linear_input_bytes(B, n) for _, _, n in layers)
    ws_in = torch.empty(ws_in_b, dtype=torch.uint8, device=dev)
    y1 = torch.empty(B * max_out, dtype=torch.float32, device=dev)
    outs = {}
    plan = []  # (kernel, input tensor, output tensor)
    for li, (name, m, n) in enumerate(layers):
        src = x_dev if n == n_in and li == 0 else outs.get(n, x_dev if n == n_in else None)
        if src is None:
            src = syn.make_activations(B, n, dtype=dtype, seed=10 + li).to(dev)
        out = torch.empty(B, m, dtype=dtype, device=dev)
        outs[m] = out
        plan.append((li, src, out, m, n))
    result = plan[-1][2]

    def one_pass(copy, s, matmul_only=False):
        for li, src, out, m, n in plan:
            k = mods[copy][li].kernel()
            if not matmul_only:
                N.check(N.lib().qs_linear_input(N.ptr(src), io, B, n, k.transform, N.ptr(k.sv), N.ptr(k.phase_v),
                                                N.ptr(ws_in), ws_in_b, None if prefill else N.ptr(y1), m, s))
            N.check(N.lib().qs_linear_matmul(N.ptr(ws_in), B, n, m, N.ptr(k.packed), len(k.kinds), k._kinds_c,
                                             k._ss_c, N.ptr(k.scale), N.ptr(y1), s))
            if not matmul_only:
                N.check(N.lib().qs_linear_output(N.ptr(y1), m, 1, B, m, k.transform, N.ptr(k.su),
                                                 N.ptr(k.phase_u), N.ptr(k.bias), N.ptr(out), io, s))

    def capture(fn):
        g = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            fn(stream.cuda_stream)  # warm (sets kernel attributes)
            torch.cuda.synchronize(dev)
            with torch.cuda.graph(g, stream=stream):
                fn(stream.cuda_stream)
        torch.cuda.synchronize(dev)
        return g

    g_pass = capture(lambda s: [one_pass(c, s) for c in range(L)])
    g_mm = capture(lambda s: [one_pass(c, s, matmul_only=True) for c in range(L)])

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

    # ---- value: device-resident inputs
    with ClockSampler(local) as clk:
        ms_total = timed(step_value, args.steps, args.warmup)
    ms_step = ms_total / args.steps
    tokens = B * passes * args.steps * world
    value = tokens / (ms_total / 1e3)
    flops_set = sum(2.0 * B * m * n for _, m, n in layers)

    # ---- dominant kernel, timed alone on the same stream
    def step_mm():
        with torch.cuda.stream(stream):
            for _ in range(R):
                g_mm.replay()
    mm_steps = max(3, args.steps // 2)
    ms_mm = timed(step_mm, mm_steps, 2)
    launches_mm = mm_steps * R * L * len(layers)
    us_per_mm = 1e3 * ms_mm / launches_mm
    hbm_peak, tc_peak, peak_kind = measured_peaks()
    if prefill:
        achieved = flops_set * mm_steps * R * L / (ms_mm / 1e3) / 1e12
        try:
            with open(os.path.join(ROOT, "MEASURED_PEAKS.json")) as f:
                tc_sust = float(json.load(f)["bf16_tflops_sustained"])
        except Exception:
            tc_sust = 1400.0
        roofline = {"bound": "tensor", "achieved": achieved, "peak": tc_sust, "unit": "TFLOP/s",
                    "frac": achieved / tc_sust, "traffic": None,
                    "kernel": "qs::gemm_tc_kernel (fused decode + tcgen05 GEMM, 128x256 tiles)",
                    "algorithmic_flops_per_layer_set": flops_set, "us_per_launch": us_per_mm,
                    "peak_source": f"{peak_kind} (MEASURED_PEAKS.json bf16_tflops_sustained; burst {tc_peak})"}
    else:
        gb = sum(gemv_bytes(m, n, kinds, B) for _, m, n in layers)
        achieved = gb * mm_steps * R * L / (ms_mm / 1e3) / 1e9
        # DRAM bytes per launch of the dominant kernel from an ncu capture of this
        # workload (profiles/gemv_c2_b1.md); other workloads have none yet
        traffic = NCU_TRAFFIC.get((args.config, B))
        roofline = {"bound": "hbm", "achieved": achieved, "peak": hbm_peak, "unit": "GB/s",
                    "frac": achieved / hbm_peak, "traffic": traffic,
                    "kernel": "qs::gemv_kernel (fused decode + mma.sync matmul)",
                    "algorithmic_bytes_per_layer_set": gb, "us_per_launch": us_per_mm,
                    "peak_source": f"{peak_kind} (MEASURED_PEAKS.json hbm_gbs)"}

    # ---- e2e: public module API; pinned host input in, the chain's result out, every step
    def fwd_all(s):
        o = None
        for c in range(L):
            cur = {n_in: x_dev}
            for li, (name, m, n) in enumerate(layers):
                inp = cur.get(n)
                if inp is None:
                    inp = plan[li][1]
                cur[m] = mods[c][li](inp)
            o = cur[layers[-1][1]]
        return o

    g_api = torch.cuda.CUDAGraph()
    with torch.cuda.stream(stream):
        fwd_all(None)
        torch.cuda.synchronize(dev)
        with torch.cuda.graph(g_api, stream=stream):
            api_out = fwd_all(None)
    torch.cuda.synchronize(dev)
    y_host = torch.empty(api_out.shape, dtype=api_out.dtype).pin_memory()

    def step_e2e():
        with torch.cuda.stream(stream):
            x_dev.copy_(x_host, non_blocking=True)
            for _ in range(R):
                g_api.replay()
            y_host.copy_(api_out, non_blocking=True)
    ms_e2e = timed(step_e2e, args.steps, args.warmup)
    e2e_value = tokens / (ms_e2e / 1e3)

    cpu = None
    if rank == 0 and world == 1 and args.cpu_sample_s > 0:
        t_set, cnt = 0.0, 0
        budget = args.cpu_sample_s / len(layers)
        for _, m, n in layers:
            t, c_ = cpu_oracle_forward_time(m, n, kinds, B, dtype, budget_s=budget)
            t_set += t
            cnt += c_
        cpu = {"value": B / t_set, "unit": "tokens/s", "cores": os.cpu_count(), "kind": "port",
               "sample": f"{cnt} full layer forwards over the {len(layers)}-layer set, batch {B} (numpy port of the "
                         f"reference algorithm, oracle/quipsharp_oracle.py); median per layer summed = {t_set:.3f} s"}

    if rank == 0:
        c = clk.summary()
        bits = sum(2 if k == "e8p" else 1 for k in kinds)
        metric = (f"quantized-linear prefill tokens/s ({args.config}, batch {B})" if prefill
                  else f"quantized-linear tokens/s ({args.config}, batch {B})")
        line = {
            "metric": metric, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True, "scaling": "weak",
            "vs_baseline": None, "dtype": "f16" if dtype == torch.float16 else "bf16", "data": "synthetic",
            "config": {"workload": args.config, "batch": B, "layers": [list(l) for l in layers], "kinds": list(kinds),
                       "layer_set_passes_per_step": passes, "distinct_copies": L,
                       "weight_bytes_per_copy": set_bytes,
                       "l2": (f"inputs larger than L2: {L} distinct copies = {L * set_bytes / 1e6:.0f} MB of packed "
                              f"weights cycled per pass (L2 126 MB)") if not prefill else
                             "inputs larger than L2: per-layer y1 / activations of the batch exceed 126 MB",
                       "bits_per_weight": bits},
            "us_per_layer_set": 1e3 * ms_step / passes,
            "hbm_gbs_per_forward": sum(algorithmic_bytes(m, n, kinds, B) for _, m, n in layers) * passes * args.steps
                                   / (ms_total / 1e3) / 1e9,
            "tflops": flops_set * passes * args.steps / (ms_total / 1e3) / 1e12,
            "roofline": roofline,
            "cpu_baseline": cpu,
            "e2e": {"value": e2e_value, "unit": "tokens/s", "h2d_bytes_per_step": B * n_in * x_host.element_size(),
                    "d2h_bytes_per_step": y_host.numel() * y_host.element_size(),
                    "path": "QuantizedLinear.forward (public module) over the layer set x passes per step, replayed "
                            "as a CUDA graph; pinned host input copied in and the last layer's output copied out "
                            "each step"},
            "gpu_launches": args.steps * R * L * sum(
                kernels_per_forward(m, n, B, torch.cuda.get_device_properties(dev).multi_processor_count)
                for _, m, n in layers),
            "clocks": {"sm_mhz": c["sm_mhz"], "sm_max_mhz": c["sm_max_mhz"], "reasons": c["reasons"]},
        }
        print(json.dumps(line), flush=True)
    del g_pass, g_mm, g_api
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def run_tp(args):
    """Tensor-parallel mode: every layer of the config's set column-sharded over the
    ranks (TPQuantizedLinear: local fused matmul, NCCL all-gather of the float32 y1
    shards, full-width output transform on every rank).  Strong scaling: one batch
    through the whole set per step, replayed as a CUDA graph (collectives included)
    and timed with CUDA events (max over ranks); at one rank the unsharded module
    runs, as the baseline."""
    import datetime
    import torch
    import torch.distributed as dist
    from quipsharp_b200 import synthetic as syn
    from quipsharp_b200.checkpoint import QuantizedLinear
    from quipsharp_b200.codebooks import E8PCodebook, E8OneBitCodebook
    from quipsharp_b200.quantize import RVQCodebookAdapter
    from quipsharp_b200.rvq import RVQStage
    from quipsharp_b200.tensor_parallel import TPQuantizedLinear

    world, rank, local = dist_env()
    if world > 1:
        dist.init_process_group("nccl", timeout=datetime.timedelta(seconds=120))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    layers, kinds, dtype = config_spec(args.config)
    B = args.batch
    cb = lambda k: E8PCodebook() if k == "e8p" else E8OneBitCodebook()
    mods = []
    for li, (name, m, n) in enumerate(layers):
        base = syn.make_layer(m, n, kinds, seed=1 + li, layer_scale=1.0 / math.sqrt(1.2 * n))
        full = QuantizedLinear(n, m, 8, base.transform_kind, num_stages=len(kinds)).to(dev)
        with torch.no_grad():
            full.codes.copy_(base.codes.to(dev))
            full.scale.fill_(base.layer_scale)
            if base.transform_kind == "rht":
                full.su.copy_(base.su)
                full.sv.copy_(base.sv)
            else:
                full.phase_u.copy_(base.phase_u)
                full.phase_v.copy_(base.phase_v)
        full.codebook = cb(kinds[0]) if len(kinds) == 1 else RVQCodebookAdapter(
            [RVQStage(cb(k), sc) for k, sc in zip(kinds, base.stage_scales)])
        if world > 1:
            mods.append((n, m, TPQuantizedLinear(full)))
            del full
        else:
            full.kernel()
            mods.append((n, m, full))
    x0 = syn.make_activations(B, layers[0][2], dtype=dtype, seed=2).to(dev)

    def step():
        latest = {x0.shape[1]: x0}
        for n, m, mod in mods:
            latest[m] = mod(latest[n])

    stream = torch.cuda.Stream(dev)
    graph = None

    def timed(k):
        if world > 1:
            dist.barrier()
        torch.cuda.synchronize()
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for _ in range(k):
                if graph is not None:
                    graph.replay()
                else:
                    step()
            e1.record(stream)
        torch.cuda.synchronize()
        ms = torch.tensor([e0.elapsed_time(e1)], device=dev)
        if world > 1:
            dist.all_reduce(ms, op=dist.ReduceOp.MAX)
        return float(ms.item())

    with torch.no_grad():
        timed(max(args.warmup, 3))  # eager warm-up (packing, NCCL communicator set-up)
        # one step (kernels and the NCCL all-gathers) captured as a CUDA graph and replayed
        graph = torch.cuda.CUDAGraph()
        with torch.cuda.stream(stream):
            torch.cuda.synchronize()
            with torch.cuda.graph(graph, stream=stream):
                step()
        torch.cuda.synchronize()
        timed(max(args.warmup, 3))
        with ClockSampler(local) as clk:
            ms = timed(args.steps)
    graph = None  # release the graph (it holds NCCL work) before the process group goes
    if rank == 0:
        c = clk.summary()
        print(json.dumps({
            "metric": f"quantized-linear tokens/s ({args.config}, batch {B}, tensor-parallel)",
            "value": B * args.steps / (ms / 1000.0), "unit": "tokens/s", "n_gpus": world,
            "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": ms / args.steps,
            "higher_is_better": True, "scaling": "strong", "vs_baseline": None,
            "dtype": str(dtype).replace("torch.", "").replace("bfloat16", "bf16").replace("float16", "f16"),
            "data": "synthetic", "config": {"workload": args.config, "batch": B, "tp": world,
                                            "layers": [list(l) for l in layers], "timing": "CUDA graph replay, max over ranks"},
            "clocks": {"sm_mhz": c["sm_mhz"], "sm_max_mhz": c["sm_max_mhz"], "reasons": c["reasons"]},
        }), flush=True)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()


def main():
    args = parse()
    if args.impl == "reference":
        run_reference(args)
    elif args.tp:
        run_tp(args)
    else:
        run_ours(args)


if __name__ == "__main__":
    main()
