"""Benchmark of the IQ3_S x MXFP8 linear path on B200 (driver contract: one JSON line on rank 0).

Workload ("decode GEMV sweep"): Llama-3-8B projection
shapes -- QKV 4096->6144, O 4096->4096, gate 4096->14336, up 4096->14336,
down 14336->4096 -- at M in {1, 2, 4, 8}. Each M uses its own layer of
seeded random IQ3_S weights, so one step streams 4 x 93.7 MB = 375 MB of
weights (larger than the 126 MB L2: no flush needed). A step runs, for each
M, the layer's 5 linears through the fused path (bf16 activations ->
MXFP8 quantization -> IQ3_S x MXFP8 GEMV -> bf16 output), captured once in
a CUDA graph and replayed.

value  = algorithmic bytes per step (weights + bf16 activations in + bf16 out)
         / device time per step, GB/s, summed over ranks (weak scaling: every
         rank runs the full workload on its own weights; the path does not
         shard at this size, so N > 1 runs independent replicas).
e2e    = the same step through the public API with pinned host buffers:
         host->device copy of the step's activations, the linears, and a
         device->host copy of the outputs, all inside the timed region.
roofline = the GEMV kernel alone: algorithmic bytes per launch / mean CUDA-event
         duration of a launch, against MEASURED_PEAKS.json's HBM copy bandwidth.

``--impl reference`` times the reference's CPU path (the C restatement of its
IQ3_S decode + MXFP8 codec + float64 dot, oracle/iq3s_ref.c) on this host.
"""

from __future__ import annotations

import argparse
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time
from pathlib import Path

ROOT = Path(__file__).resolve().parent
sys.path.insert(0, str(ROOT))

PROJECTIONS = (  # name, N, K (Llama-3-8B)
    ("qkv", 6144, 4096),
    ("o", 4096, 4096),
    ("gate", 14336, 4096),
    ("up", 14336, 4096),
    ("down", 4096, 14336),
)
M_SWEEP = (1, 2, 4, 8)
METRIC = "IQ3_S x MXFP8 decode linear (Llama-3-8B shapes, M in {1,2,4,8}) algorithmic GB/s"
HBM_FALLBACK_GBS = 6650.0


def load_peaks() -> tuple[float, str]:
    p = ROOT / "MEASURED_PEAKS.json"
    if p.is_file():
        try:
            return float(json.loads(p.read_text())["hbm_gbs"]), "measured"
        except (KeyError, ValueError):
            pass
    return HBM_FALLBACK_GBS, "fallback"


def read_profiled_traffic(key: str = "dram_bytes_per_launch"):
    """DRAM bytes per GEMV launch from the committed ncu summary (a line '<key>: N')."""
    path = ROOT / "profiles" / "iq3s_gemv_tm_decode_llama3_8b.md"
    if not path.is_file():
        return None
    for line in path.read_text().splitlines():
        if line.strip().startswith(key + ":"):
            try:
                return float(line.split(":", 1)[1].split()[0])
            except (ValueError, IndexError):
                return None
    return None


def layer_bytes() -> int:
    return sum(n * (k // 256) * 110 for _, n, k in PROJECTIONS)


def step_bytes() -> tuple[int, int, int]:
    """(weight bytes, activation-in bytes, output bytes) per step."""
    w = layer_bytes() * len(M_SWEEP)
    xin = sum(m * k * 2 for m in M_SWEEP for _, _, k in PROJECTIONS)
    out = sum(m * n * 2 for m in M_SWEEP for _, n, _ in PROJECTIONS)
    return w, xin, out


# ---------------------------------------------------------------------------
# clocks
# ---------------------------------------------------------------------------
class ClockSampler:
    QUERY = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.active,"
             "clocks_event_reasons.hw_slowdown,clocks_event_reasons.hw_thermal_slowdown,"
             "clocks_event_reasons.sw_thermal_slowdown,clocks_event_reasons.sw_power_cap")

    def __init__(self, index: int):
        self.index = index
        self.proc = None
        self.path = None

    def __enter__(self):
        fd, self.path = tempfile.mkstemp(suffix=".csv")
        os.close(fd)
        try:
            self.proc = subprocess.Popen(
                ["nvidia-smi", "-i", str(self.index), f"--query-gpu={self.QUERY}", "--format=csv,noheader,nounits",
                 "-lms", "50"], stdout=open(self.path, "w"), stderr=subprocess.DEVNULL)
        except (FileNotFoundError, OSError):
            self.proc = None
        time.sleep(0.3)
        return self

    def __exit__(self, *exc):
        if self.proc is not None:
            self.proc.terminate()
            try:
                self.proc.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.proc.kill()

    def summary(self) -> dict:
        if self.proc is None or self.path is None:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["nvidia-smi unavailable"]}
        rows = []
        for line in Path(self.path).read_text().splitlines():
            parts = [p.strip() for p in line.split(",")]
            if len(parts) < 9:
                continue
            try:
                rows.append((float(parts[1]), float(parts[2]), float(parts[3]), parts[5:9]))
            except ValueError:
                continue
        os.unlink(self.path)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["no samples"]}
        names = ("hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap")
        reasons = sorted({names[i] for r in rows for i, v in enumerate(r[3]) if v.lower() == "active"})
        return {"sm_mhz": statistics.median(r[0] for r in rows), "sm_max_mhz": max(r[1] for r in rows),
                "power_w_max": max(r[2] for r in rows), "samples": len(rows), "reasons": reasons}


# ---------------------------------------------------------------------------
# CPU baseline (the reference's CPU path, restated in C)
# ---------------------------------------------------------------------------
def cpu_baseline(budget_s: float = 15.0) -> dict:
    import numpy as np

    from oracle import c_oracle
    from oracle import iq3s_oracle as O

    threads = os.cpu_count() or 1
    m, n, k = 8, 4096, 4096  # the O projection at M = 8
    x = np.random.default_rng(20261017).standard_normal((m, k)).astype(np.float32)

    def run(rows: int) -> float:
        raw = O.make_synthetic_iq3s(rows, k, seed=0x1A3)
        t0 = time.perf_counter()
        q, s = c_oracle.quantize_mxfp8(x)
        c_oracle.iq3s_linear_f64(q, s, raw, threads=threads)
        return time.perf_counter() - t0

    t_small = run(256)
    rows = int(min(n, max(256, 256 * budget_s / max(t_small, 1e-6))))
    rows = max(256, rows // 256 * 256)
    t = run(rows)
    weight_bytes = rows * (k // 256) * 110
    alg = weight_bytes + m * k * 2 + m * rows * 2
    return {"value": alg / t / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "sample": f"O projection rows 0..{rows} of {n} x K={k}, M={m}: C oracle (IQ3_S decode + MXFP8 quant + "
                      f"float64 dot), {threads} host threads, {t:.2f} s"}


def run_reference(args) -> None:
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    budget = max(0.5, 60.0 / max(1, args.steps + args.warmup))
    res = None
    for _ in range(args.warmup):
        cpu_baseline(budget)
    t0 = time.perf_counter()
    vals = [cpu_baseline(budget) for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    res = vals[-1]
    value = statistics.mean(v["value"] for v in vals)
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall * 1000 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f64",
        "data": "synthetic", "config": {"workload": "decode_gemv_sweep_llama3_8b (bounded CPU sample)",
                                        "sample": res["sample"]},
        "cpu_baseline": {**res, "value": value},
        "e2e": {"value": value, "unit": "GB/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
    }
    print(json.dumps(line), flush=True)


# ---------------------------------------------------------------------------
# GPU
# ---------------------------------------------------------------------------
def build_workload(torch, dev):
    from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

    layers = {}
    for li, m in enumerate(M_SWEEP):
        projs = {}
        for pi, (name, n, k) in enumerate(PROJECTIONS):
            seed = 0x1A3 + 7919 * li + pi
            gen = torch.Generator(device=dev).manual_seed(seed)
            raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=dev, generator=gen)
            d = (torch.rand((n, k // 256), device=dev, generator=gen) * 9e-3 + 1e-3).half()
            raw[..., :2] = d.view(torch.uint8).view(n, k // 256, 2)
            projs[name] = prepare_iq3_s_fields(raw)
            del raw
        layers[m] = projs
    gen = torch.Generator(device="cpu").manual_seed(20261017)
    inputs = {m: {name: torch.randn((m, k), generator=gen).to(torch.bfloat16) for name, _, k in PROJECTIONS}
              for m in M_SWEEP}
    return layers, inputs


def measure_fp8_peak(torch, dev) -> tuple[float | None, str]:
    """cuBLASLt FP8 (e4m3) GEMM 8192^3 through torch._scaled_mm: best of 5, TFLOP/s."""
    try:
        n = 8192
        a = torch.randn((n, n), device=dev).to(torch.float8_e4m3fn)
        b = torch.randn((n, n), device=dev).to(torch.float8_e4m3fn)
        one = torch.tensor(1.0, device=dev)
        run = lambda: torch._scaled_mm(a, b.t(), scale_a=one, scale_b=one, out_dtype=torch.bfloat16)  # noqa: E731
        for _ in range(3):
            run()
        best = None
        for _ in range(5):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            run()
            e1.record()
            torch.cuda.synchronize(dev)
            ms = e0.elapsed_time(e1)
            best = ms if best is None else min(best, ms)
        return 2 * n ** 3 / (best * 1e-3) / 1e12, "measured here: torch._scaled_mm e4m3 8192^3 (cuBLASLt), best of 5"
    except Exception as ex:  # noqa: BLE001
        p = ROOT / "MEASURED_PEAKS.json"
        if p.is_file():
            return 2 * float(json.loads(p.read_text())["bf16_tflops"]), f"2 x measured bf16 ({type(ex).__name__})"
        return None, f"unavailable ({type(ex).__name__})"


def prefill_probe(torch, dev, m: int = 2048) -> dict:
    """The tcgen05 GEMM at M=2048 on the Llama-3-8B shapes (bf16 N(0,1) activations with
    1% of K columns x50): device time per launch with L2 flushed before each, TFLOP/s against an FP8 peak."""
    from mambo_b200.kernels.iq3_s_fp8 import linear_into, select_config
    from mambo_b200.kernels.quantize_fp8 import launch_quantize_fp8
    from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

    shapes = (("qkv", 6144, 4096), ("o", 4096, 4096), ("gate_up", 14336, 4096), ("down", 4096, 14336))
    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)
    rows, tot_flop, tot_us = [], 0, 0.0
    for i, (name, n, k) in enumerate(shapes):
        gen = torch.Generator(device=dev).manual_seed(0x51A + i)
        raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=dev, generator=gen)
        d = (torch.rand((n, k // 256), device=dev, generator=gen) * 9e-3 + 1e-3).half()
        raw[..., :2] = d.view(torch.uint8).view(n, k // 256, 2)
        fields = prepare_iq3_s_fields(raw)
        del raw, d
        x = torch.randn((m, k), device=dev, generator=gen)
        x[:, torch.randperm(k, device=dev, generator=gen)[: round(0.01 * k)]] *= 50.0
        xq, xs = launch_quantize_fp8(x.to(torch.bfloat16))
        out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        cfg = select_config(m, n, k, dev)
        for _ in range(3):
            linear_into(xq, xs, fields, out, config=cfg)
        torch.cuda.synchronize(dev)
        us = []
        for _ in range(5):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            linear_into(xq, xs, fields, out, config=cfg)
            e1.record()
            torch.cuda.synchronize(dev)
            us.append(e0.elapsed_time(e1) * 1000)
        t = statistics.median(us)
        flop = 2 * m * n * k
        rows.append({"proj": name, "n": n, "k": k, "us": round(t, 1), "tflops": round(flop / t / 1e6, 1)})
        tot_flop += flop
        tot_us += t
        del fields, x, xq, xs, out
    peak, kind = measure_fp8_peak(torch, dev)
    tf = tot_flop / tot_us / 1e6
    return {"m": m, "tflops": tf, "unit": "TFLOP/s", "peak_tflops": peak, "peak_kind": kind,
            "frac": (tf / peak) if peak else None, "kernel": "iq3s_gemm_f16_kernel (+ iq3s_x16_kernel: MXFP8 activations to FP16)",
            "l2": "flushed (256 MB write) before each timed launch", "per_shape": rows}


def run_single(args) -> None:
    """Four linear launches of one shape (for ncu captures of a single kernel)."""
    import torch

    from mambo_b200.kernels.iq3_s_fp8 import fused_linear_into, linear_into, select_config
    from mambo_b200.kernels.quantize_fp8 import launch_quantize_fp8
    from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

    n, k, m = (int(v) for v in args.single.split(","))
    dev = torch.device("cuda", 0)
    gen = torch.Generator(device=dev).manual_seed(1)
    raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=dev, generator=gen)
    d = (torch.rand((n, k // 256), device=dev, generator=gen) * 9e-3 + 1e-3).half()
    raw[..., :2] = d.view(torch.uint8).view(n, k // 256, 2)
    fields = prepare_iq3_s_fields(raw)
    x = torch.randn((m, k), device=dev, generator=gen).to(torch.bfloat16)
    xq, xs = launch_quantize_fp8(x)
    out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
    cfg = dict(select_config(m, n, k, dev))
    if args.kernel is not None:
        cfg["kernel"] = args.kernel
    for _ in range(4):
        if args.prequantized:
            linear_into(xq, xs, fields, out, config=cfg)
        else:  # the bench's decode step: bf16 activations through the fused entry point
            fused_linear_into(x, fields, out, config=cfg)
    torch.cuda.synchronize()
    print(f"single N={n} K={k} M={m} config={cfg}: ok")


def run_group_profile() -> None:
    """Four grouped launches of the decode sweep (for ncu captures of the grouped kernel)."""
    import torch

    from mambo_b200.kernels.iq3_s_fp8 import group_linear_into

    dev = torch.device("cuda", 0)
    layers, inputs = build_workload(torch, dev)
    order = [(m, p, n) for m in M_SWEEP for p, n, _ in PROJECTIONS]
    xs = [inputs[m][p].to(dev) for m, p, _ in order]
    ws = [layers[m][p] for m, p, _ in order]
    outs = [torch.empty((m, n), dtype=torch.bfloat16, device=dev) for m, _, n in order]
    for _ in range(4):
        group_linear_into(xs, ws, outs)
    torch.cuda.synchronize()
    print(f"group profile: {len(order)} linears per launch: ok")


LLAMA3_8B_LAYERS = 32


def run_llama3_8b(args) -> None:
    """every linear of a 32-layer Llama-3-8B-shaped model (random IQ3_S
    weights): one 4096-token prefill, then 128 decode steps at batch 8; linear time only.

    A layer is QKV, O, gate, up, down. Decode keeps a model's dependency order:
    per layer QKV, then O, then gate and up together (one grouped launch: they
    read the same input), then down, each a launch in one CUDA graph per step.
    Prefill runs each linear through the fused entry point (MXFP8 quantization,
    then the FP16-operand GEMM). Activations are fixed random bf16 buffers of
    each linear's shape (no attention or MLP math in between).
    """
    import torch

    from mambo_b200.kernels.iq3_s_fp8 import fused_linear_into, group_linear_into
    from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    prefill_m, decode_m, decode_steps = 4096, 8, 128
    layers = []
    for li in range(LLAMA3_8B_LAYERS):
        projs = {}
        for pi, (name, n, k) in enumerate(PROJECTIONS):
            gen = torch.Generator(device=dev).manual_seed(0x1A3 + 7919 * li + pi)
            raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=dev, generator=gen)
            d = (torch.rand((n, k // 256), device=dev, generator=gen) * 9e-3 + 1e-3).half()
            raw[..., :2] = d.view(torch.uint8).view(n, k // 256, 2)
            projs[name] = prepare_iq3_s_fields(raw)
            del raw
        layers.append(projs)
    gen = torch.Generator(device=dev).manual_seed(20261017)
    shapes = {name: (n, k) for name, n, k in PROJECTIONS}

    def buffers(m):
        x = {name: torch.randn((m, k), device=dev, generator=gen).to(torch.bfloat16) for name, (n, k) in shapes.items()}
        y = {name: torch.empty((m, n), device=dev, dtype=torch.bfloat16) for name, (n, k) in shapes.items()}
        return x, y

    xp, yp = buffers(prefill_m)
    xd, yd = buffers(decode_m)
    stream = torch.cuda.Stream(dev)

    def prefill():
        for w in layers:
            for name in shapes:
                fused_linear_into(xp[name], w[name], yp[name])

    def decode_step():
        for w in layers:
            fused_linear_into(xd["qkv"], w["qkv"], yd["qkv"])
            fused_linear_into(xd["o"], w["o"], yd["o"])
            group_linear_into([xd["gate"], xd["up"]], [w["gate"], w["up"]], [yd["gate"], yd["up"]])
            fused_linear_into(xd["down"], w["down"], yd["down"])

    def capture(fn):
        with torch.cuda.stream(stream):
            fn()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            fn()
        torch.cuda.synchronize(dev)
        return g

    g_prefill, g_decode = capture(prefill), capture(decode_step)

    def timed(g, reps):
        with torch.cuda.stream(stream):
            for _ in range(args.warmup):
                g.replay()
        torch.cuda.synchronize(dev)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(reps):
                g.replay()
        e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) / reps

    with ClockSampler(0) as clocks:
        prefill_ms = timed(g_prefill, 3)
        decode_ms = timed(g_decode, decode_steps)
    w_bytes = layer_bytes() * LLAMA3_8B_LAYERS
    flops = 2.0 * prefill_m * sum(n * k for _, n, k in PROJECTIONS) * LLAMA3_8B_LAYERS
    dec_bytes = w_bytes + LLAMA3_8B_LAYERS * sum(decode_m * (k + n) * 2 for _, n, k in PROJECTIONS)
    peak, peak_kind = load_peaks()
    total_ms = prefill_ms + decode_steps * decode_ms
    print(json.dumps({
        "metric": "Llama-3-8B linear layers (32 layers): 4096-token prefill + 128 decode steps at batch 8, linear time",
        "value": total_ms, "unit": "ms", "n_gpus": 1, "higher_is_better": False, "dtype": "e4m3",
        "data": "synthetic (random IQ3_S weights, bf16 N(0,1) activations)",
        "config": {"workload": "llama3_8b_linears (BASELINE config 4)", "layers": LLAMA3_8B_LAYERS,
                   "prefill_tokens": prefill_m, "decode_batch": decode_m, "decode_steps": decode_steps,
                   "weights_bytes": w_bytes,
                   "decode_step": "per layer: QKV, O, grouped gate+up, down (4 launches), one CUDA graph per step",
                   "prefill": "per linear: fused MXFP8 quantization + FP16-operand GEMM, one CUDA graph"},
        "prefill": {"ms": prefill_ms, "tflops": flops / (prefill_ms * 1e-3) / 1e12},
        "decode": {"ms_per_step": decode_ms, "gbs": dec_bytes / (decode_ms * 1e-3) / 1e9,
                   "hbm_frac": dec_bytes / (decode_ms * 1e-3) / 1e9 / peak, "peak_gbs": peak, "peak_kind": peak_kind,
                   "launches_per_step": 4 * LLAMA3_8B_LAYERS},
        "clocks": clocks.summary(),
    }), flush=True)


TP70B_GROUPS = (("qkv",), ("o",), ("gate", "up"), ("down",))  # launches per layer, in a model's order
TP70B = (  # name, N, K, split (Llama-3-70B)
    ("qkv", 10240, 8192, "column"),
    ("o", 8192, 8192, "row"),
    ("gate", 28672, 8192, "column"),
    ("up", 28672, 8192, "column"),
    ("down", 8192, 28672, "row"),
)


def run_tp70b(args) -> None:
    """Llama-3-70B linears tensor-parallel over the launched ranks (NCCL), M in {1, 64, 4096}.

    Column split for QKV/gate/up (outputs all-gathered), row split for O/down (FP32 partials all-reduced).
    Per M: CUDA-event time of one layer's 5 linears (max over ranks) -- each rank's compute replayed from a
    CUDA graph, the collectives issued eagerly in between -- and, eagerly, of its collectives alone; weights
    of two layers per rank alternate between steps so that every step streams them from HBM.
    """
    import datetime

    import torch
    import torch.distributed as dist

    from mambo_b200.sharding import TensorParallelIQ3SLinear, local_group

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    layers = []
    for li in range(2):
        lin = {}
        for pi, (name, n, k, split) in enumerate(TP70B):
            gen = torch.Generator(device=dev).manual_seed(0x70B + 97 * li + pi)  # same weights on every rank
            raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=dev, generator=gen)
            d = (torch.rand((n, k // 256), device=dev, generator=gen) * 9e-3 + 1e-3).half()
            raw[..., :2] = d.view(torch.uint8).view(n, k // 256, 2)
            lin[name] = TensorParallelIQ3SLinear(raw, split, out_dtype=torch.bfloat16)
            del raw, d
            torch.cuda.empty_cache()
        layers.append(lin)
    results = []
    for m in (1, 64, 4096):
        gen = torch.Generator(device=dev).manual_seed(20261017 + m)
        xs = {k: torch.randn((m, k), device=dev, generator=gen).to(torch.bfloat16) for k in (8192, 28672)}

        def layer(li, timed_coll=False):
            coll = 0.0
            for name, n, k, split in TP70B:
                lin = layers[li][name]
                lin(xs[k], time_collective=timed_coll)
                coll += lin.times.collective_ms if timed_coll else 0.0
            return coll

        # Eager warm-up on the capture stream (allocates its workspace outside the capture).
        stream = torch.cuda.Stream(dev)
        with torch.cuda.stream(stream):
            for w in range(args.warmup):
                layer(w & 1)
        torch.cuda.synchronize(dev)
        # A layer in a model's order: QKV, O, gate and up together (one grouped
        # launch: they read the same input), down. Per group a CUDA graph of this
        # rank's compute; the NCCL collectives run eagerly between replays on the
        # same stream. With one GPU (no collectives) the layer is one graph.
        kdim = {name: k for name, n, k, split in TP70B}

        def group_local(li, grp):
            if len(grp) == 1:
                return [layers[li][grp[0]].local(xs[kdim[grp[0]]])]
            return local_group([layers[li][name] for name in grp], xs[kdim[grp[0]]])

        with torch.cuda.stream(stream):
            for li in range(2):
                for grp in TP70B_GROUPS:
                    group_local(li, grp)  # eager warm-up of the grouped path
        torch.cuda.synchronize(dev)
        graphs = {}
        for li in range(2):
            if world == 1:
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    for grp in TP70B_GROUPS:
                        group_local(li, grp)
                graphs[li] = g
            else:
                for grp in TP70B_GROUPS:
                    g = torch.cuda.CUDAGraph()
                    with torch.cuda.graph(g, stream=stream):
                        ys = group_local(li, grp)
                    graphs[(li, grp)] = (g, ys)
        torch.cuda.synchronize(dev)

        def layer_graphed(li):
            if world == 1:
                graphs[li].replay()
                return
            for grp in TP70B_GROUPS:
                g, ys = graphs[(li, grp)]
                g.replay()
                for name, y in zip(grp, ys):
                    layers[li][name].combine(y)

        with torch.cuda.stream(stream):
            for w in range(args.warmup):
                layer_graphed(w & 1)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        steps = max(2, args.steps // 5)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for st in range(steps):
                layer_graphed(st & 1)
            e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / steps
        del graphs
        coll = sum(layer(st & 1, timed_coll=True) for st in range(2)) / 2
        if world > 1:
            t = torch.tensor([ms, coll], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms, coll = float(t[0]), float(t[1])
        w_bytes = sum(n * (k // 256) * 110 for _, n, k, _ in TP70B)
        flops = sum(2 * m * n * k for _, n, k, _ in TP70B)
        results.append({"m": m, "ms_per_layer": round(ms, 4), "collective_ms": round(coll, 4),
                        "weight_gbs_total": round(w_bytes / (ms * 1e-3) / 1e9, 1),
                        "tflops_total": round(flops / (ms * 1e-3) / 1e12, 1)})
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        peak, kind = load_peaks()
        print(json.dumps({"workload": "tp70b (BASELINE config 5)", "n_gpus": world, "parallelism": f"tp{world}",
                          "data": "synthetic", "weights_per_layer_bytes": sum(n * (k // 256) * 110
                                                                               for _, n, k, _ in TP70B),
                          "hbm_peak_gbs_per_gpu": peak, "peak_kind": kind,
                          "note": "ms_per_layer: QKV, O, grouped gate+up, down; per group a CUDA-graph replay of "
                                  "the rank's compute (fused quantization + linear) and the NCCL collectives issued "
                                  "eagerly (one graph per layer on one GPU); collective_ms: device time of the "
                                  "layer's all-gathers/all-reduces measured alone in eager steps",
                          "results": results}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("mambo", "reference"), default="mambo")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the M=2048 prefill GEMM probe")
    ap.add_argument("--single", metavar="N,K,M",
                    help="profiling mode: run four linears of one shape (random IQ3_S weights) and exit")
    ap.add_argument("--kernel", type=int, default=None, help="with --single: MAMBO_KERNEL_* to use")
    ap.add_argument("--prequantized", action="store_true",
                    help="with --single: MXFP8 activations quantized beforehand (mambo_iq3s_linear)")
    ap.add_argument("--workload", choices=("decode", "tp70b", "llama3_8b"), default="decode",
                    help="tp70b: Llama-3-70B linears tensor-parallel over the launched ranks; llama3_8b: every "
                         "linear of a 32-layer Llama-3-8B, prefill + 128 decode steps (each its own JSON line)")
    ap.add_argument("--group-profile", action="store_true",
                    help="profiling mode: four grouped launches of the decode sweep, then exit")
    args = ap.parse_args()
    args.warmup = max(3, args.warmup)
    if args.single:
        run_single(args)
        return
    if args.group_profile:
        run_group_profile()
        return
    if args.workload == "tp70b" and args.impl == "mambo":
        run_tp70b(args)
        return
    if args.workload == "llama3_8b" and args.impl == "mambo":
        run_llama3_8b(args)
        return

    if args.impl == "reference":
        run_reference(args)
        return

    import torch
    import torch.distributed as dist

    from mambo_b200.kernels.iq3_s_fp8 import fused_linear_into, group_linear_into, select_config

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=__import__("datetime").timedelta(seconds=120))

    layers, inputs = build_workload(torch, dev)
    stream = torch.cuda.Stream(dev)

    # device buffers, in sweep order (M, projection)
    order = [(m, p, n, k) for m in M_SWEEP for p, n, k in PROJECTIONS]
    xs_dev = {(m, p): inputs[m][p].to(dev) for m, p, _, _ in order}
    out_buf = {(m, p): torch.empty((m, n), dtype=torch.bfloat16, device=dev) for m, p, n, _ in order}
    configs = {(m, p): select_config(m, n, k, dev) for m, p, n, k in order}
    g_x = [xs_dev[(m, p)] for m, p, _, _ in order]
    g_w = [layers[m][p] for m, p, _, _ in order]
    g_o = [out_buf[(m, p)] for m, p, _, _ in order]

    def group_step():
        # the whole sweep (20 independent linears) as one grouped GEMV launch
        group_linear_into(g_x, g_w, g_o)

    def per_linear_step():
        # one launch per linear: the decode GEMV quantizes its bf16 activations itself
        for m, p, _, _ in order:
            fused_linear_into(xs_dev[(m, p)], layers[m][p], out_buf[(m, p)], config=configs[(m, p)])

    def capture(fn, copies: int = 1):
        with torch.cuda.stream(stream):
            for _ in range(2):
                fn()  # eager warm-up (allocates the workspace)
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(copies):
                fn()
        torch.cuda.synchronize(dev)
        return g

    graph = capture(group_step)
    graph_sep = capture(per_linear_step)

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(v: float) -> float:
        if world == 1:
            return v
        t = torch.tensor([v], device=dev, dtype=torch.float64)
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    def time_replays(g, steps: int) -> float:
        """ms per replay of g over `steps` replays, CUDA events on the launching stream."""
        t0, t1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        t0.record(stream)
        with torch.cuda.stream(stream):
            for _ in range(steps):
                g.replay()
        t1.record(stream)
        torch.cuda.synchronize(dev)
        return t0.elapsed_time(t1) / steps

    # ---- timed region: K graph replays of the step (one grouped launch) ----
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph.replay()
    torch.cuda.synchronize(dev)
    barrier()

    def keep_busy(seconds: float) -> None:
        # Back-to-back replays around the timed region so that the clock samples
        # (every 50 ms) see the GPU under the same load; not timed.
        t_end = time.perf_counter() + seconds
        with torch.cuda.stream(stream):
            while time.perf_counter() < t_end:
                for _ in range(20):
                    graph.replay()
                torch.cuda.synchronize(dev)

    with ClockSampler(local) as clocks:
        keep_busy(0.5)
        barrier()
        step_ms = time_replays(graph, args.steps)
        keep_busy(0.5)
        barrier()
    ms_per_step = max_over_ranks(step_ms)
    clock = clocks.summary()
    w_bytes, in_bytes, out_bytes = step_bytes()
    alg = w_bytes + in_bytes + out_bytes
    value = alg * world / (ms_per_step * 1e-3) / 1e9

    # ---- the same sweep as 20 separate launches (one per linear) -----------
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            graph_sep.replay()
    torch.cuda.synchronize(dev)
    barrier()
    sep_ms = max_over_ranks(time_replays(graph_sep, args.steps))

    # ---- roofline: the grouped launch, and every linear launched alone ------
    # Kernels are timed as back-to-back launches inside one graph, the way
    # they run in the step: separately launched work (a stream launch, or a
    # graph of one kernel) starts on a ~2 us grid on this GPU, which would
    # round each launch up.
    launches = 10
    g10 = capture(group_step, copies=launches)
    with torch.cuda.stream(stream):
        for _ in range(3):
            g10.replay()
    group_us = time_replays(g10, 5) * 1000 / launches
    del g10
    per_launch = []
    for m, p, n, k in order:
        g = capture(lambda: fused_linear_into(xs_dev[(m, p)], layers[m][p], out_buf[(m, p)], config=configs[(m, p)]),
                    copies=launches)
        with torch.cuda.stream(stream):
            for _ in range(3):
                g.replay()
        us = time_replays(g, 10) * 1000 / launches
        b = n * (k // 256) * 110 + m * k * 2 + m * n * 2
        per_launch.append({"m": m, "proj": p, "us": round(us, 3), "bytes": b, "gbs": round(b / us / 1e3, 1)})
        del g
    peak, peak_kind = load_peaks()
    achieved = alg / group_us / 1e3
    sep_achieved = sum(r["bytes"] for r in per_launch) / sum(r["us"] for r in per_launch) / 1e3
    traffic = read_profiled_traffic("dram_bytes_per_group_launch")

    # ---- e2e: public API with pinned host buffers, H2D + D2H in the region --
    # One pinned buffer holds every input of a step and one holds every output:
    # one H2D copy in, one D2H copy out per step, and in between one public
    # call (group_linear_into) that writes each linear's output into its view
    # of the device output buffer.
    host_in_all = torch.cat([inputs[m][p].reshape(-1) for m, p, _, _ in order]).pin_memory()
    host_out_all = torch.empty(sum(m * n for m, _, n, _ in order), dtype=torch.bfloat16).pin_memory()
    dev_in_all = torch.empty_like(host_in_all, device=dev)
    dev_out_all = torch.empty_like(host_out_all, device=dev)
    dev_in, host_out, off_i, off_o = {}, {}, 0, 0
    for m, p, n, k in order:
        dev_in[(m, p)] = dev_in_all[off_i:off_i + m * k].view(m, k)
        host_out[(m, p)] = host_out_all[off_o:off_o + m * n].view(m, n)
        off_i += m * k
        off_o += m * n
    e2e_x = [dev_in[(m, p)] for m, p, _, _ in order]
    e2e_o, off_o = [], 0
    for m, _, n, _ in order:
        e2e_o.append(dev_out_all[off_o:off_o + m * n].view(m, n))
        off_o += m * n

    def e2e_step():
        dev_in_all.copy_(host_in_all, non_blocking=True)
        group_linear_into(e2e_x, g_w, e2e_o)
        host_out_all.copy_(dev_out_all, non_blocking=True)

    g_e2e = capture(e2e_step)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            g_e2e.replay()
    torch.cuda.synchronize(dev)
    barrier()
    e2e_serial_ms = max_over_ranks(time_replays(g_e2e, args.steps))

    # Pipelined, as a serving loop runs it: PIPE steps per graph, each with its
    # own H2D copy of the step's inputs and D2H read of its outputs, on a copy
    # stream that overlaps them with the neighbouring steps' linears (two
    # device buffer sets).
    PIPE = 8
    copy_stream = torch.cuda.Stream(dev)
    sets = [(dev_in_all, dev_out_all, e2e_x, e2e_o)]
    di2, do2 = torch.empty_like(dev_in_all), torch.empty_like(dev_out_all)
    xs2, os2, oi, oo = [], [], 0, 0
    for m, p, n, k in order:
        xs2.append(di2[oi:oi + m * k].view(m, k))
        os2.append(do2[oo:oo + m * n].view(m, n))
        oi += m * k
        oo += m * n
    sets.append((di2, do2, xs2, os2))

    def e2e_pipelined():
        ev_in = [torch.cuda.Event() for _ in range(PIPE)]
        ev_out = [torch.cuda.Event() for _ in range(PIPE)]
        ev_d2h = [torch.cuda.Event() for _ in range(PIPE)]
        cur = torch.cuda.current_stream()
        copy_stream.wait_stream(cur)
        with torch.cuda.stream(copy_stream):
            for st in range(min(2, PIPE)):
                sets[st % 2][0].copy_(host_in_all, non_blocking=True)
                ev_in[st].record(copy_stream)
        for st in range(PIPE):
            di, do, xs_b, os_b = sets[st % 2]
            cur.wait_event(ev_in[st])
            if st >= 2:
                cur.wait_event(ev_d2h[st - 2])  # this set's outputs of step st-2 have been read back
            group_linear_into(xs_b, g_w, os_b)
            ev_out[st].record(cur)
            with torch.cuda.stream(copy_stream):
                copy_stream.wait_event(ev_out[st])
                host_out_all.copy_(do, non_blocking=True)
                ev_d2h[st].record(copy_stream)
                if st + 2 < PIPE:
                    di.copy_(host_in_all, non_blocking=True)  # step st has consumed this set's inputs
                    ev_in[st + 2].record(copy_stream)
        cur.wait_stream(copy_stream)

    g_pipe = capture(e2e_pipelined)
    with torch.cuda.stream(stream):
        for _ in range(args.warmup):
            g_pipe.replay()
    torch.cuda.synchronize(dev)
    barrier()
    e2e_ms = max_over_ranks(time_replays(g_pipe, args.steps) / PIPE)
    # eager (no graph) for reference
    torch.cuda.synchronize(dev)
    t_e = time.perf_counter()
    with torch.cuda.stream(stream):
        for _ in range(max(3, args.steps // 5)):
            e2e_step()
    torch.cuda.synchronize(dev)
    eager_ms = (time.perf_counter() - t_e) * 1000 / max(3, args.steps // 5)
    # correctness spot check of the e2e output against the device path
    with torch.cuda.stream(stream):
        graph.replay()
    torch.cuda.synchronize(dev)
    ok = all(torch.equal(host_out[(m, p)], out_buf[(m, p)].cpu()) for m, p, _, _ in order)

    if world > 1:
        del graph, graph_sep, g_e2e, g_pipe
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    prefill = None if args.no_prefill else prefill_probe(torch, dev)
    cpu = None if args.no_cpu_baseline else cpu_baseline()
    line = {
        "metric": METRIC,
        "value": value,
        "unit": "GB/s",
        "n_gpus": world,
        "steps": args.steps,
        "warmup": args.warmup,
        "ms_per_step": ms_per_step,
        "higher_is_better": True,
        "scaling": "weak",
        "vs_baseline": None,
        "dtype": "e4m3",
        "data": "synthetic",
        "config": {"workload": "decode_gemv_sweep_llama3_8b (BASELINE config 2)", "m_sweep": list(M_SWEEP),
                   "projections": {p: [n, k] for p, n, k in PROJECTIONS},
                   "bytes_per_step": {"weights": w_bytes, "act_in_bf16": in_bytes, "out_bf16": out_bytes},
                   "l2": "inputs larger than L2 (375 MB of weights per step)",
                   "execution": "cuda graph replay; the step's 20 independent linears in one grouped GEMV launch "
                                "(mambo_iq3s_linear_group)",
                   "parallelism": f"replicas{world}"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": traffic, "peak_kind": peak_kind,
                     "kernel": "iq3s_gemv_tm_kernel<1,8,GemvGroup>: the 20 linears of a step in one launch, "
                               "MXFP8 quantization fused",
                     "launch_us": group_us,
                     "timing": "10 back-to-back launches in one CUDA graph, 5 replays, mean"},
        # Every linear launched on its own (the reference's one-linear-per-call shape).
        "per_linear": {"value": alg * world / (sep_ms * 1e-3) / 1e9, "unit": "GB/s", "ms_per_step": sep_ms,
                       "gpu_launches_per_step": len(order), "kernel_achieved": sep_achieved,
                       "kernel_frac": sep_achieved / peak,
                       "timing": "per linear: 10 back-to-back launches in one CUDA graph, 10 replays, mean",
                       "per_launch": per_launch},
        "e2e": {"value": alg * world / (e2e_ms * 1e-3) / 1e9, "unit": "GB/s",
                "h2d_bytes_per_step": in_bytes, "d2h_bytes_per_step": out_bytes,
                "ms_per_step": e2e_ms,
                "execution": "per step: one H2D copy of all the step's inputs, one public-API call "
                             "(group_linear_into, 20 linears into views of one output buffer), one D2H copy of "
                             f"all outputs; CUDA graphs of {PIPE} such steps pipelined over a copy stream and two "
                             "device buffer sets (copies overlap the neighbouring steps' linears)",
                "serial_ms_per_step": e2e_serial_ms,
                "serial_value": alg * world / (e2e_serial_ms * 1e-3) / 1e9,
                "eager_ms_per_step": eager_ms, "matches_device_path": ok},
        # one grouped GEMV launch per step
        "gpu_launches": args.steps,
        "clocks": clock,
        "cpu_baseline": cpu,
        # BASELINE config 3 (prefill GEMM) at M=2048, for the TFLOP/s half of the metric
        "prefill": prefill,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
