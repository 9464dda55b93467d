"""Benchmark of the IQ3_S x MXFP8 linear path on B200 (driver contract: one JSON line on rank 0).

Headline workload ("decode GEMV sweep"): Llama-3-8B
projection shapes -- QKV 4096->6144, O 4096->4096, gate 4096->14336, up
4096->14336, down 14336->4096 -- at M in {1, 2, 4, 8}. Each M uses its own
layer of seeded random IQ3_S weights, so one step streams 4 x 93.7 MB =
375 MB of weights (larger than the 126 MB L2: no flush needed). A step runs,
for each M, the layer's 5 linears through the fused path (bf16 activations ->
MXFP8 quantization -> IQ3_S x MXFP8 GEMV -> bf16 output), captured once in a
CUDA graph and replayed.

value  = algorithmic bytes per step (weights + bf16 activations in + bf16 out)
         / device time per step, GB/s, summed over ranks (weak scaling: every
         rank runs the full sweep on its own weights).
e2e    = the same step through the public API with pinned host buffers:
         host->device copy of the step's activations, the linears, and a
         device->host copy of the outputs, all inside the timed region.
roofline = the GEMV kernel alone: algorithmic bytes per launch / mean CUDA-event
         duration of a launch, against MEASURED_PEAKS.json's HBM copy bandwidth.

Further blocks of the same JSON line:
tp      = BASELINE config 5 at every N: one Llama-3-70B layer's linears
          tensor-parallel over the launched ranks (column split QKV/gate/up,
          row split O/down, NCCL all-reduce), M in {1, 64, 4096}, with the
          sharded outputs checked against the unsharded linear on rank 0.
prefill = BASELINE config 3 (N = 1): bf16 activations with 1 % outlier
          columns -> quantization -> GEMM -> bf16 output, all inside the timed
          region, M in {512, 2048, 8192}, TFLOP/s against an FP8 peak measured
          in the same run.
model   = BASELINE config 4 (N = 1): every linear of a 32-layer Llama-3-8B,
          one 4096-token prefill + 128 decode steps at batch 8.
cpu_baseline = the reference's CPU path on BASELINE config 1 (N = 1).

``--impl reference`` times the reference's CPU path on BASELINE config 1 (the
O projection shape at M = 16): gguf-py's IQ3_S dequantize, the reference test
oracle's MXFP8 codec (restated in oracle/iq3s_oracle.py) and an fp32 matmul.
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
# CPU baselines (the reference's CPU path)
# ---------------------------------------------------------------------------
CONFIG1 = (16, 4096, 4096)  # M, N, K (the O projection shape)


def cpu_model() -> str:
    try:
        for line in Path("/proc/cpuinfo").read_text().splitlines():
            if line.startswith("model name"):
                return line.split(":", 1)[1].strip()
    except OSError:
        pass
    return "unknown"


def cpu_stock_step(raw, x) -> dict:
    """One pass of the reference's CPU path on [M,K] activations and [N,K/256,110] IQ3_S blocks.

    gguf-py's ``dequantize`` (the installed gguf package: the decoder the
    reference's tests call, tests/python/utils/compute_reference_gguf.py:80-100),
    the reference test oracle's MXFP8 codec ``encode_mxfp8_reference`` /
    ``decode_mxfp8`` (tests/python/utils/fp8_reference.py:64-86, restated in
    oracle/iq3s_oracle.py: nearest value, ties to the smaller magnitude), and
    an fp32 torch.matmul of the decoded operands on all host threads
    (compute_reference_gguf.py:111-121 multiplies them).
    """
    import numpy as np
    import torch
    from gguf import GGMLQuantizationType
    from gguf.quants import dequantize

    from oracle import iq3s_oracle as O

    n = raw.shape[0]
    t0 = time.perf_counter()
    w = dequantize(raw.reshape(n, -1), GGMLQuantizationType.IQ3_S)
    t1 = time.perf_counter()
    q, sc = O.quantize_mxfp8(x, rounding="ties_down")
    xd = O.decode_mxfp8(q, sc)
    t2 = time.perf_counter()
    y = torch.from_numpy(np.ascontiguousarray(xd)) @ torch.from_numpy(np.ascontiguousarray(w, dtype=np.float32)).T
    t3 = time.perf_counter()
    assert y.shape == (x.shape[0], n)
    return {"dequant_s": t1 - t0, "quant_s": t2 - t1, "matmul_s": t3 - t2, "total_s": t3 - t0}


def config1_inputs():
    import numpy as np

    from oracle import iq3s_oracle as O

    m, n, k = CONFIG1
    raw = O.make_synthetic_iq3s(n, k, seed=0x1A3)
    x = np.random.default_rng(20261017).standard_normal((m, k)).astype(np.float32)
    return raw, x


def config1_bytes() -> int:
    m, n, k = CONFIG1
    return n * (k // 256) * 110 + m * k * 2 + m * n * 2


def cpu_baseline_stock(reps: int = 2) -> dict:
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    raw, x = config1_inputs()
    runs = [cpu_stock_step(raw, x) for _ in range(reps)]
    best = min(runs, key=lambda r: r["total_s"])
    m, n, k = CONFIG1
    return {"value": config1_bytes() / best["total_s"] / 1e9, "unit": "GB/s", "cores": threads, "kind": "port",
            "cpu_model": cpu_model(),
            "sample": f"BASELINE config 1 (M={m}, N={n}, K={k}) through the reference's CPU path: gguf-py "
                      f"dequantize (single thread), the reference test oracle's MXFP8 codec (restated), fp32 "
                      f"torch.matmul on {threads} threads; best of {reps}",
            "seconds": {k2: round(v, 4) for k2, v in best.items()}}


def cpu_baseline_c_port(budget_s: float = 15.0) -> dict:
    """The same path restated in C (oracle/iq3s_ref.c: decode + MXFP8 + float64 dot, all host threads)."""
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


def cpu_baseline() -> dict:
    stock = cpu_baseline_stock()
    stock["c_port"] = cpu_baseline_c_port()
    return stock


def run_reference(args) -> None:
    """The reference arm: its CPU path on BASELINE config 1, one pass per step (rank 0 only)."""
    rank = int(os.environ.get("RANK", "0"))
    if rank != 0:
        return
    import torch

    threads = os.cpu_count() or 1
    torch.set_num_threads(threads)
    raw, x = config1_inputs()
    for _ in range(args.warmup):
        cpu_stock_step(raw, x)
    t0 = time.perf_counter()
    runs = [cpu_stock_step(raw, x) for _ in range(args.steps)]
    wall = time.perf_counter() - t0
    value = config1_bytes() * args.steps / wall / 1e9
    m, n, k = CONFIG1
    sample = (f"BASELINE config 1 (M={m}, N={n}, K={k}: the O projection of the decode sweep) per step: gguf-py "
              f"dequantize, the reference test oracle's MXFP8 codec (restated), fp32 torch.matmul on {threads} "
              f"threads")
    line = {
        "impl": "reference", "metric": METRIC, "value": value, "unit": "GB/s", "n_gpus": args.gpus,
        "steps": args.steps, "warmup": args.warmup, "ms_per_step": wall * 1000 / args.steps,
        "higher_is_better": True, "scaling": "weak", "vs_baseline": None, "dtype": "f32",
        "data": "synthetic", "config": {"workload": "decode_gemv_sweep_llama3_8b (bounded CPU sample: BASELINE "
                                                    "config 1)", "sample": sample},
        "cpu_baseline": {"value": value, "unit": "GB/s", "cores": threads, "kind": "port", "sample": sample,
                         "cpu_model": cpu_model(),
                         "seconds_per_step": {key: round(statistics.mean(r[key] for r in runs), 4)
                                              for key in ("dequant_s", "quant_s", "matmul_s", "total_s")}},
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


PREFILL_SHAPES = (("qkv", 6144, 4096), ("o", 4096, 4096), ("gate_up", 14336, 4096), ("down", 4096, 14336))
PREFILL_MS = (512, 2048, 8192)


def prefill_block(torch, dev, ms=PREFILL_MS) -> dict:
    """the Llama-3-8B shapes at prefill M, bf16 N(0,1) activations with 1 % of K columns x50.

    Timed per launch with L2 flushed before each: the whole path from bf16
    activations to the bf16 output through the public call (fused_linear_into:
    activation quantization, then the tcgen05 GEMM), and the GEMM alone on
    activations quantized beforehand.
    """
    from mambo_b200 import _lib
    from mambo_b200.kernels.iq3_s_fp8 import fused_linear_into, linear_into, select_config
    from mambo_b200.kernels.quantize_fp8 import launch_quantize_fp8
    from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

    flush = torch.empty(256 * 1024 * 1024, dtype=torch.uint8, device=dev)

    def timed(fn, reps=5) -> float:
        for _ in range(2):
            fn()
        torch.cuda.synchronize(dev)
        us = []
        for _ in range(reps):
            flush.zero_()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            fn()
            e1.record()
            torch.cuda.synchronize(dev)
            us.append(e0.elapsed_time(e1) * 1000)
        return statistics.median(us)

    weights = []
    for i, (name, n, k) in enumerate(PREFILL_SHAPES):
        gen = torch.Generator(device=dev).manual_seed(0x51A + i)
        raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=dev, generator=gen)
        d = (torch.rand((n, k // 256), device=dev, generator=gen) * 9e-3 + 1e-3).half()
        raw[..., :2] = d.view(torch.uint8).view(n, k // 256, 2)
        weights.append(prepare_iq3_s_fields(raw))
        del raw, d
    per_m = []
    for m in ms:
        rows, flop_tot, us_tot, gemm_us_tot, fold_us_tot, wide_us_tot = [], 0, 0.0, 0.0, 0.0, 0.0
        for i, (name, n, k) in enumerate(PREFILL_SHAPES):
            gen = torch.Generator(device=dev).manual_seed(0x51A + 100 * i + m)
            x = torch.randn((m, k), device=dev, generator=gen)
            x[:, torch.randperm(k, device=dev, generator=gen)[: round(0.01 * k)]] *= 50.0
            xb = x.to(torch.bfloat16)
            del x
            out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
            fields = weights[i]
            us = timed(lambda: fused_linear_into(xb, fields, out))
            xq, xs = launch_quantize_fp8(xb)
            cfg = select_config(m, n, k, dev)
            gemm_us = timed(lambda: linear_into(xq, xs, fields, out, config=cfg))
            # The folded variant (d folded, rounded, into the FP16 weights; 1e-3 bound), default stages/split.
            fold_cfg = dict(cfg, kernel=_lib.MAMBO_KERNEL_GEMM_F16_FOLD) if cfg.get("kernel") != \
                _lib.MAMBO_KERNEL_GEMM_F16_PAIR else {"kernel": _lib.MAMBO_KERNEL_GEMM_F16_FOLD, "stages": 4}
            fold_us = timed(lambda: fused_linear_into(xb, fields, out, config=fold_cfg))
            # The wide variant (CTA pairs, 256 x 256-token tiles, d folded as above).
            wide_cfg = {"kernel": _lib.MAMBO_KERNEL_GEMM_F16_WIDE, "warps": 8, "stages": 4}
            wide_us = timed(lambda: fused_linear_into(xb, fields, out, config=wide_cfg))
            flop = 2 * m * n * k
            rows.append({"proj": name, "n": n, "k": k, "us": round(us, 1), "tflops": round(flop / us / 1e6, 1),
                         "gemm_us": round(gemm_us, 1), "gemm_tflops": round(flop / gemm_us / 1e6, 1),
                         "folded_us": round(fold_us, 1), "folded_tflops": round(flop / fold_us / 1e6, 1),
                         "wide_us": round(wide_us, 1), "wide_tflops": round(flop / wide_us / 1e6, 1)})
            flop_tot += flop
            us_tot += us
            gemm_us_tot += gemm_us
            fold_us_tot += fold_us
            wide_us_tot += wide_us
            del xb, xq, xs, out
        per_m.append({"m": m, "tflops": flop_tot / us_tot / 1e6, "gemm_tflops": flop_tot / gemm_us_tot / 1e6,
                      "folded_tflops": flop_tot / fold_us_tot / 1e6, "wide_tflops": flop_tot / wide_us_tot / 1e6,
                      "per_shape": rows})
    del weights, flush
    torch.cuda.empty_cache()
    peak, kind = measure_fp8_peak(torch, dev)
    for r in per_m:
        r["frac"] = r["tflops"] / peak if peak else None
        r["gemm_frac"] = r["gemm_tflops"] / peak if peak else None
        r["folded_frac"] = r["folded_tflops"] / peak if peak else None
        r["wide_frac"] = r["wide_tflops"] / peak if peak else None
    head = next(r for r in per_m if r["m"] == 2048) if 2048 in ms else per_m[0]
    return {"m": head["m"], "tflops": head["tflops"], "unit": "TFLOP/s", "peak_tflops": peak, "peak_kind": kind,
            "frac": head["frac"], "per_m": per_m,
            "timed": "tflops: bf16 activations -> MXFP8 quantization -> GEMM -> bf16 output, one public call "
                     "(fused_linear_into) per shape; gemm_tflops: the GEMM alone on prequantized activations; "
                     "folded_tflops / wide_tflops: the same call with MAMBO_KERNEL_GEMM_F16_FOLD / _WIDE (block "
                     "scale folded into the FP16 weights, within the 1e-3 bound; wide: CTA pairs, 256 x 256-token "
                     "tiles)",
            "kernel": "iq3s_gemm_f16_kernel (FP16 operands, group scale folded exactly into the weights)",
            "l2": "flushed (256 MB write) before each timed launch"}


def synthetic_q4k(torch, dev, n: int, k: int, seed: int):
    """Random Q4_K blocks uint8 [N, K/256, 144] on the device: uniform bytes, fp16 d and dmin in +-[1e-4, 1e-2)."""
    gen = torch.Generator(device=dev).manual_seed(seed)
    raw = torch.randint(0, 256, (n, k // 256, 144), dtype=torch.uint8, device=dev, generator=gen)
    for f in range(2):
        sign = torch.randint(0, 2, (n, k // 256), device=dev, generator=gen) * 2 - 1
        v = ((torch.rand((n, k // 256), device=dev, generator=gen) * 9.9e-3 + 1e-4) * sign).half()
        raw[..., 2 * f:2 * f + 2] = v.view(torch.uint8).view(n, k // 256, 2)
    return raw


def q4k_block(torch, dev) -> dict:
    """Q4_K x MXFP8 decode linears (GGUF type Q4_K, 144 bytes per 256 weights) on the tcgen05 GEMV.

    The Llama-3-8B projections of the decode sweep at M in {1, 2, 4, 8}, random
    Q4_K weights (fp16 d and dmin in +-[1e-4, 1e-2)), bf16 N(0,1) activations.
    Per linear, 10 back-to-back launches in one CUDA graph: the GEMV alone on
    activations quantized beforehand (with their group sums), and the public
    call from bf16 activations (the quantizer with sums, then the GEMV).
    Weights per step exceed the L2 (the sweep's 20 weights are 487 MB).
    """
    from mambo_b200.kernels.q4_k_fp8 import launch_q4_k_fp8_matmul, launch_quantize_fp8_sums, \
        prepare_q4_k_fields, q4_k_fp8_linear, q4_k_linear_group_into

    stream = torch.cuda.Stream(dev)
    launches = 10

    def graph_us(fn, replays=10) -> float:
        with torch.cuda.stream(stream):
            fn()
        torch.cuda.synchronize(dev)
        g = torch.cuda.CUDAGraph()
        with torch.cuda.graph(g, stream=stream):
            for _ in range(launches):
                fn()
        with torch.cuda.stream(stream):
            for _ in range(3):
                g.replay()
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record(stream)
            for _ in range(replays):
                g.replay()
            e1.record(stream)
        torch.cuda.synchronize(dev)
        return e0.elapsed_time(e1) * 1000 / (replays * launches)

    rows, w_tot, b_tot, fb_tot, us_tot, fused_us_tot = [], 0, 0, 0, 0.0, 0.0
    for pi, (name, n, k) in enumerate(PROJECTIONS):
        gen = torch.Generator(device=dev).manual_seed(0x4B80 + pi)
        w = prepare_q4_k_fields(synthetic_q4k(torch, dev, n, k, seed=0x4B00 + pi))
        for m in M_SWEEP:
            x = torch.randn((m, k), device=dev, generator=gen).to(torch.bfloat16)
            xq, xs, xsum = launch_quantize_fp8_sums(x)
            out = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
            us = graph_us(lambda: launch_q4_k_fp8_matmul(xq, xs, xsum, w, out=out, stream=stream))
            fused_us = graph_us(lambda: q4_k_fp8_linear(x, w, out=out, stream=stream))
            wb = n * (k // 256) * 144
            b = wb + m * k + m * (k // 32) * 5 + m * n * 2  # weights, E4M3 codes, scales + sums, bf16 out
            rows.append({"m": m, "proj": name, "us": round(us, 2), "gbs": round(b / us / 1e3, 1),
                         "fused_us": round(fused_us, 2)})
            w_tot += wb
            b_tot += b
            fb_tot += wb + m * k * 2 + m * n * 2  # from bf16 activations to the bf16 output
            us_tot += us
            fused_us_tot += fused_us
        del w
    torch.cuda.empty_cache()
    # The same sweep as one grouped call: 20 distinct weights (487 MB), bf16 activations; the
    # quantization pre-pass (codes and group sums of all 20 inputs) and one grouped GEMV launch.
    gws, gxs, gouts, g_bytes = [], [], [], 0
    for mi, m in enumerate(M_SWEEP):
        for pi, (name, n, k) in enumerate(PROJECTIONS):
            gws.append(prepare_q4_k_fields(synthetic_q4k(torch, dev, n, k, seed=0x4C00 + 16 * mi + pi)))
            gen = torch.Generator(device=dev).manual_seed(0x4C80 + 16 * mi + pi)
            gxs.append(torch.randn((m, k), device=dev, generator=gen).to(torch.bfloat16))
            gouts.append(torch.empty((m, n), dtype=torch.bfloat16, device=dev))
            g_bytes += n * (k // 256) * 144 + m * k * 2 + m * n * 2
    group_us = graph_us(lambda: q4_k_linear_group_into(gxs, gws, gouts, stream=stream))
    del gws, gxs, gouts
    torch.cuda.empty_cache()
    peak, kind = load_peaks()
    achieved = b_tot / us_tot / 1e3
    return {"value": achieved, "unit": "GB/s", "frac": achieved / peak, "peak": peak, "peak_kind": kind,
            "weights_bytes_per_sweep": w_tot, "bytes_per_sweep": b_tot, "gemv_us_per_sweep": us_tot,
            "fused_us_per_sweep": fused_us_tot,
            "fused_gbs": fb_tot / fused_us_tot / 1e3,
            "grouped": {"us_per_sweep": group_us, "gbs": g_bytes / group_us / 1e3,
                        "frac": g_bytes / group_us / 1e3 / peak,
                        "execution": "the 20 linears of the sweep (distinct weights) in one call from bf16 "
                                     "activations: group_xtiles_kernel with group sums, then "
                                     "iq3s_gemv_tm_kernel<1,8,GemvGroupPre,false,true>; 10 calls per CUDA graph"},
            "kernel": "iq3s_gemv_tm_kernel<NT,8,GemvNoGroup,false,true> (Q4_K decoders, stream-K)",
            "timing": "per linear: 10 back-to-back launches in one CUDA graph, 10 replays, mean",
            "per_launch": rows}


def run_single(args) -> None:
    """Four linear launches of one shape (for ncu captures of a single kernel)."""
    import torch

    from mambo_b200.kernels.iq3_s_fp8 import fused_linear_into, linear_into, select_config
    from mambo_b200.kernels.quantize_fp8 import launch_quantize_fp8
    from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

    n, k, m = (int(v) for v in args.single.split(","))
    dev = torch.device("cuda", 0)
    if args.q4k:
        # Four Q4_K launches (prequantized activations with their group sums), then the IQ3_S ones below.
        from mambo_b200.kernels.q4_k_fp8 import launch_q4_k_fp8_matmul, launch_quantize_fp8_sums, \
            prepare_q4_k_fields
        w4 = prepare_q4_k_fields(synthetic_q4k(torch, dev, n, k, seed=2))
        xq4, xs4, xsum4 = launch_quantize_fp8_sums(torch.randn((m, k), device=dev).to(torch.bfloat16))
        out4 = torch.empty((m, n), dtype=torch.bfloat16, device=dev)
        for _ in range(4):
            launch_q4_k_fp8_matmul(xq4, xs4, xsum4, w4, out=out4)
        torch.cuda.synchronize()
        del w4
        args.prequantized = True
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


def model_block(torch, dev, warmup: int = 3) -> dict:
    """every linear of a 32-layer Llama-3-8B-shaped model (random IQ3_S
    weights): one 4096-token prefill, then 128 decode steps at batch 8; linear time only.

    A layer is QKV, O, gate, up, down. Decode keeps a model's dependency order:
    per layer QKV, then O, then gate and up together (one grouped launch: they
    read the same input), then down, each a launch in one CUDA graph per step.
    Prefill runs each linear through the fused entry point (MXFP8 quantization,
    then the FP16-operand GEMM). Activations are fixed random bf16 buffers of
    each linear's shape (no attention or MLP math in between).
    """
    from mambo_b200.kernels.iq3_s_fp8 import fused_linear_into, group_linear_into
    from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

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
            for _ in range(warmup):
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

    with ClockSampler(dev.index or 0) as clocks:
        prefill_ms = timed(g_prefill, 3)
        decode_ms = timed(g_decode, decode_steps)
    del g_prefill, g_decode, layers
    torch.cuda.empty_cache()
    w_bytes = layer_bytes() * LLAMA3_8B_LAYERS
    flops = 2.0 * prefill_m * sum(n * k for _, n, k in PROJECTIONS) * LLAMA3_8B_LAYERS
    dec_bytes = w_bytes + LLAMA3_8B_LAYERS * sum(decode_m * (k + n) * 2 for _, n, k in PROJECTIONS)
    peak, peak_kind = load_peaks()
    total_ms = prefill_ms + decode_steps * decode_ms
    return {
        "workload": "llama3_8b_linears (BASELINE config 4)", "layers": LLAMA3_8B_LAYERS,
        "prefill_tokens": prefill_m, "decode_batch": decode_m, "decode_steps": decode_steps,
        "weights_bytes": w_bytes, "total_ms": total_ms,
        "decode_step": "per layer: QKV, O, grouped gate+up (its quantization pre-pass and the grouped GEMV), "
                       "down (5 launches), one CUDA graph per step",
        "prefill_exec": "per linear: fused MXFP8 quantization + FP16-operand GEMM, one CUDA graph",
        "prefill": {"ms": prefill_ms, "tflops": flops / (prefill_ms * 1e-3) / 1e12},
        "decode": {"ms_per_step": decode_ms, "gbs": dec_bytes / (decode_ms * 1e-3) / 1e9,
                   "hbm_frac": dec_bytes / (decode_ms * 1e-3) / 1e9 / peak, "peak_gbs": peak,
                   "peak_kind": peak_kind, "launches_per_step": 5 * LLAMA3_8B_LAYERS},
        "clocks": clocks.summary(),
    }


def run_llama3_8b(args) -> None:
    """--workload llama3_8b: the model block alone, as its own JSON line."""
    import torch

    dev = torch.device("cuda", 0)
    torch.cuda.set_device(dev)
    r = model_block(torch, dev, warmup=args.warmup)
    print(json.dumps({
        "metric": "Llama-3-8B linear layers (32 layers): 4096-token prefill + 128 decode steps at batch 8, linear time",
        "value": r["total_ms"], "unit": "ms", "n_gpus": 1, "higher_is_better": False, "dtype": "e4m3",
        "data": "synthetic (random IQ3_S weights, bf16 N(0,1) activations)", "config": {"workload": r["workload"]},
        **r}), flush=True)


TP70B = (  # name, N, K, split (Llama-3-70B)
    ("qkv", 10240, 8192, "column"),
    ("o", 8192, 8192, "row"),
    ("gate", 28672, 8192, "column"),
    ("up", 28672, 8192, "column"),
    ("down", 8192, 28672, "row"),
)
TP70B_MS = (1, 64, 4096)
TP_PARITY_TOL = 1e-5


def _tp_raw(torch, dev, li: int, pi: int, n: int, k: int):
    gen = torch.Generator(device=dev).manual_seed(0x70B + 97 * li + pi)  # the same weights on every rank
    raw = torch.randint(0, 256, (n, k // 256, 110), dtype=torch.uint8, device=dev, generator=gen)
    d = (torch.rand((n, k // 256), device=dev, generator=gen) * 9e-3 + 1e-3).half()
    raw[..., :2] = d.view(torch.uint8).view(n, k // 256, 2)
    return raw


def tp_block(torch, world: int, rank: int, dev, steps: int, warmup: int) -> dict | None:
    """one Llama-3-70B layer's linears tensor-parallel over the launched ranks.

    Every rank (and the process group, when world > 1) takes part; rank 0 returns the results.
    A layer, as a tensor-parallel transformer layer runs its linears: QKV
    (column split, output kept sharded by heads), O (row split, input the
    rank's K slice, FP32 partials all-reduced), gate and up (column split, one
    grouped launch, outputs kept sharded), down (row split, all-reduced). Per
    rank: two CUDA graphs of its compute (QKV + O, gate/up + down), each followed
    by the NCCL all-reduce and the bf16 cast, issued eagerly. One GPU: the
    unsharded layer (QKV, O, grouped gate+up, down) in one CUDA graph. Weights of
    two layers alternate between steps, so every step streams them from HBM.

    Parity (world > 1): for every projection of layer 0 and every M, the
    gathered (column) or all-reduced (row) FP32 output against the unsharded
    linear on rank 0, relative Frobenius error.
    """
    import torch.distributed as dist

    from mambo_b200.kernels.iq3_s_fp8 import fused_linear_into, group_linear_into, iq3_s_fp8_linear
    from mambo_b200.sharding import FusedAllReduce, TensorParallelIQ3SLinear, gather_columns_group, local_group
    from mambo_b200.utils.iq3_s_weight import prepare_iq3_s_fields

    kdim = {name: k for name, n, k, split in TP70B}
    layers, full = [], {}
    for li in range(2):
        lin = {}
        for pi, (name, n, k, split) in enumerate(TP70B):
            raw = _tp_raw(torch, dev, li, pi, n, k)
            if world == 1:
                lin[name] = prepare_iq3_s_fields(raw)
            else:
                lin[name] = TensorParallelIQ3SLinear(raw, split, gather_output=False,
                                                     input_is_sharded=split == "row", out_dtype=torch.bfloat16)
                if li == 0 and rank == 0:
                    full[name] = prepare_iq3_s_fields(raw)
            del raw
            torch.cuda.empty_cache()
        layers.append(lin)
    stream = torch.cuda.Stream(dev)
    results = []
    fused_comm = None  # the fused row-split all-reduce's exchange buffers (world > 1, decode sizes)
    for m in TP70B_MS:
        gen = torch.Generator(device=dev).manual_seed(20261017 + m)  # the same activations on every rank
        x_full = {k: torch.randn((m, k), device=dev, generator=gen).to(torch.bfloat16) for k in (8192, 28672)}
        rec = {"m": m}
        if world == 1:
            outs = {name: torch.empty((m, n), dtype=torch.bfloat16, device=dev) for name, n, _, _ in TP70B}

            def layer_1gpu(li, w=None):
                w = w or layers[li]
                fused_linear_into(x_full[kdim["qkv"]], w["qkv"], outs["qkv"])
                fused_linear_into(x_full[kdim["o"]], w["o"], outs["o"])
                group_linear_into([x_full[8192]] * 2, [w["gate"], w["up"]], [outs["gate"], outs["up"]])
                fused_linear_into(x_full[kdim["down"]], w["down"], outs["down"])

            with torch.cuda.stream(stream):
                for li in range(2):
                    layer_1gpu(li)  # eager warm-up (allocates the workspace outside the capture)
            torch.cuda.synchronize(dev)
            graphs = []
            for li in range(2):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    layer_1gpu(li)
                graphs.append(g)

            def step(i):
                graphs[i & 1].replay()
        else:
            l0 = layers[0]
            # This rank's K slices of the row splits' inputs (attention output, MLP activation).
            x_o = x_full[8192][:, l0["o"].k0:l0["o"].k0 + l0["o"].local_k].contiguous()
            x_dn = x_full[28672][:, l0["down"].k0:l0["down"].k0 + l0["down"].local_k].contiguous()
            # Parity: every projection's combined FP32 output against the unsharded linear.
            errs = {}
            for name, n, k, split in TP70B:
                lin = l0[name]
                if split == "column":
                    y = lin(x_full[k], gather=True, out_dtype=torch.float32)
                else:
                    y = lin(x_full[k][:, lin.k0:lin.k0 + lin.local_k], out_dtype=torch.float32)
                if rank == 0:
                    ref = iq3_s_fp8_linear(x_full[k], full[name], out_dtype=torch.float32)
                    errs[name] = (torch.linalg.norm((y - ref).double()) / torch.linalg.norm(ref.double())).item()
            # The grouped gate/up gather (one collective) against the unsharded pair as well.
            g, u = local_group([l0["gate"], l0["up"]], x_full[8192])
            g32, u32 = gather_columns_group([l0["gate"], l0["up"]], [g.float(), u.float()])
            if rank == 0:
                for name, y in (("gate", g32), ("up", u32)):
                    ref = iq3_s_fp8_linear(x_full[8192], full[name], out_dtype=torch.bfloat16).float()
                    errs[f"{name}_grouped_bf16"] = (torch.linalg.norm((y - ref).double()) /
                                                    torch.linalg.norm(ref.double())).item()
                rec["parity_rel_frobenius"] = {k2: float(f"{v:.3g}") for k2, v in errs.items()}
                # bf16 entries: both sides rounded to bf16 after FP32 sums in different orders
                rec["parity_ok"] = all(v <= (TP_PARITY_TOL if "bf16" not in k2 else 1e-3) for k2, v in errs.items())

            def compute_a(li):  # QKV (column, kept sharded) and O's local partial
                w = layers[li]
                w["qkv"].local(x_full[8192])
                return w["o"].local(x_o)

            def compute_b(li):  # gate + up (one grouped launch) and down's local partial
                w = layers[li]
                local_group([w["gate"], w["up"]], x_full[8192])
                return w["down"].local(x_dn)

            with torch.cuda.stream(stream):
                for li in range(2):
                    compute_a(li)
                    compute_b(li)
            torch.cuda.synchronize(dev)
            graphs = []
            for li in range(2):
                ga, gb = torch.cuda.CUDAGraph(), torch.cuda.CUDAGraph()
                with torch.cuda.graph(ga, stream=stream):
                    ya = compute_a(li)
                with torch.cuda.graph(gb, stream=stream):
                    yb = compute_b(li)
                graphs.append((ga, ya, gb, yb))

            def step(i):
                ga, ya, gb, yb = graphs[i & 1]
                w = layers[i & 1]
                ga.replay()
                w["o"].combine(ya)
                gb.replay()
                w["down"].combine(yb)
        torch.cuda.synchronize(dev)
        with torch.cuda.stream(stream):
            for i in range(max(3, warmup)):
                step(i)
        torch.cuda.synchronize(dev)
        if world > 1:
            dist.barrier()
        n_steps = max(4, steps // 2)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        with torch.cuda.stream(stream):
            e0.record(stream)
            for i in range(n_steps):
                step(i)
            e1.record(stream)
        torch.cuda.synchronize(dev)
        ms = e0.elapsed_time(e1) / n_steps
        coll = 0.0
        if world > 1:
            # The layer's two all-reduces alone (eager, device time), on this layer's partials.
            ga, ya, gb, yb = graphs[0]
            with torch.cuda.stream(stream):
                for _ in range(2):
                    dist.all_reduce(ya)
                    dist.all_reduce(yb)
                torch.cuda.synchronize(dev)
                c0, c1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                c0.record(stream)
                for _ in range(4):
                    dist.all_reduce(ya)
                    dist.all_reduce(yb)
                c1.record(stream)
            torch.cuda.synchronize(dev)
            coll = c0.elapsed_time(c1) / 4
            t = torch.tensor([ms, coll], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            ms, coll = float(t[0]), float(t[1])
        del graphs
        torch.cuda.synchronize(dev)
        if world > 1 and m < 32:
            # Decode sizes: the row splits' all-reduces fused into their GEMVs (peer stores over NVLink, no
            # NCCL call), so the rank's whole layer is one CUDA graph.
            if fused_comm is None:
                fused_comm = FusedAllReduce(8192)
            l0 = layers[0]
            f_errs = {}
            for name, x_in in (("o", x_o), ("down", x_dn)):
                y32 = l0[name].fused(x_in, fused_comm, out_dtype=torch.float32)
                torch.cuda.synchronize(dev)
                if rank == 0:
                    ref = iq3_s_fp8_linear(x_full[kdim[name]], full[name], out_dtype=torch.float32)
                    f_errs[name] = (torch.linalg.norm((y32 - ref).double()) / torch.linalg.norm(ref.double())).item()
            y_o = torch.empty((m, 8192), dtype=torch.bfloat16, device=dev)
            y_dn = torch.empty((m, 8192), dtype=torch.bfloat16, device=dev)

            def layer_fused(li):
                w = layers[li]
                w["qkv"].local(x_full[8192])
                w["o"].fused(x_o, fused_comm, out=y_o)
                local_group([w["gate"], w["up"]], x_full[8192])
                w["down"].fused(x_dn, fused_comm, out=y_dn)

            with torch.cuda.stream(stream):
                for li in range(2):
                    layer_fused(li)
            torch.cuda.synchronize(dev)
            fgraphs = []
            for li in range(2):
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    layer_fused(li)
                fgraphs.append(g)
            with torch.cuda.stream(stream):
                for i in range(max(3, warmup)):
                    fgraphs[i & 1].replay()
            torch.cuda.synchronize(dev)
            dist.barrier()
            with torch.cuda.stream(stream):
                e0.record(stream)
                for i in range(n_steps):
                    fgraphs[i & 1].replay()
                e1.record(stream)
            torch.cuda.synchronize(dev)
            t = torch.tensor([e0.elapsed_time(e1) / n_steps], device=dev, dtype=torch.float64)
            dist.all_reduce(t, op=dist.ReduceOp.MAX)
            rec["ms_per_layer_fused_allreduce"] = round(float(t[0]), 4)
            if rank == 0:
                rec["parity_fused_allreduce_rel_frobenius"] = {k2: float(f"{v:.3g}") for k2, v in f_errs.items()}
                rec["parity_ok"] = rec.get("parity_ok", True) and all(v <= TP_PARITY_TOL for v in f_errs.values())
            del fgraphs
            torch.cuda.synchronize(dev)
            dist.barrier()
        # The unsharded layer on rank 0 of this box (the N = 1 figure next to the sharded one).
        if world > 1:
            if rank == 0:
                outs = {name: torch.empty((m, n), dtype=torch.bfloat16, device=dev) for name, n, _, _ in TP70B}

                def layer_full():
                    fused_linear_into(x_full[kdim["qkv"]], full["qkv"], outs["qkv"])
                    fused_linear_into(x_full[kdim["o"]], full["o"], outs["o"])
                    group_linear_into([x_full[8192]] * 2, [full["gate"], full["up"]], [outs["gate"], outs["up"]])
                    fused_linear_into(x_full[kdim["down"]], full["down"], outs["down"])

                with torch.cuda.stream(stream):
                    layer_full()
                torch.cuda.synchronize(dev)
                g = torch.cuda.CUDAGraph()
                with torch.cuda.graph(g, stream=stream):
                    layer_full()
                with torch.cuda.stream(stream):
                    for _ in range(3):
                        g.replay()
                    torch.cuda.synchronize(dev)
                    f0, f1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                    f0.record(stream)
                    for _ in range(n_steps):
                        g.replay()
                    f1.record(stream)
                torch.cuda.synchronize(dev)
                rec["ms_per_layer_1gpu"] = round(f0.elapsed_time(f1) / n_steps, 4)
                rec["speedup_vs_1gpu"] = round(rec["ms_per_layer_1gpu"] / ms, 3)
                if "ms_per_layer_fused_allreduce" in rec:
                    rec["speedup_fused_allreduce_vs_1gpu"] = round(
                        rec["ms_per_layer_1gpu"] / rec["ms_per_layer_fused_allreduce"], 3)
                del g
            dist.barrier()
        w_bytes = sum(n * (k // 256) * 110 for _, n, k, _ in TP70B)
        flops = sum(2 * m * n * k for _, n, k, _ in TP70B)
        rec.update({"ms_per_layer": round(ms, 4), "collective_ms": round(coll, 4),
                    "weight_gbs_total": round(w_bytes / (ms * 1e-3) / 1e9, 1),
                    "tflops_total": round(flops / (ms * 1e-3) / 1e12, 1)})
        results.append(rec)
    if fused_comm is not None:
        torch.cuda.synchronize(dev)
        dist.barrier()  # every rank is done writing into the peers' buffers
        fused_comm.close()
    del layers, full
    torch.cuda.empty_cache()
    if rank != 0:
        return None
    peak, kind = load_peaks()
    return {"workload": "tp70b (BASELINE config 5)", "n_gpus": world, "parallelism": f"tp{world}",
            "scaling": "strong", "weights_per_layer_bytes": sum(n * (k // 256) * 110 for _, n, k, _ in TP70B),
            "hbm_peak_gbs_per_gpu": peak, "peak_kind": kind, "parity_tol": TP_PARITY_TOL,
            "layer": ("one GPU: QKV, O, grouped gate+up, down in one CUDA graph. N GPUs: per rank a CUDA graph "
                      "of QKV (column shard) + O (row shard, local K slice), the NCCL all-reduce of O's FP32 "
                      "partials + bf16 cast, a graph of gate+up (one grouped launch) + down (row shard), the "
                      "all-reduce of down's partials + cast; column outputs stay sharded (the next row split "
                      "consumes them)"),
            "collective_ms": "device time of the layer's two all-reduces alone (eager), max over ranks",
            "fused_allreduce": ("M < 32, N GPUs: O and down each one launch of mambo_iq3s_linear_fused_ar (the GEMV "
                                "writes each row tile's FP32 partial into every rank's exchange buffer over NVLink "
                                "and sums all ranks' partials in rank order), the rank's whole layer one CUDA graph "
                                "with no NCCL call; parity of O and down against the unsharded linear"),
            "results": results}


def run_tp70b(args) -> None:
    """--workload tp70b: the TP block alone, as its own JSON line."""
    import datetime

    import torch
    import torch.distributed as dist

    world = int(os.environ.get("WORLD_SIZE", "1"))
    rank = int(os.environ.get("RANK", "0"))
    local = int(os.environ.get("LOCAL_RANK", "0"))
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    if world > 1:
        dist.init_process_group("nccl", device_id=dev, timeout=datetime.timedelta(seconds=120))
    r = tp_block(torch, world, rank, dev, args.steps, args.warmup)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank == 0:
        print(json.dumps({"data": "synthetic", **r}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=50)
    ap.add_argument("--warmup", type=int, default=5)
    ap.add_argument("--impl", choices=("mambo", "reference"), default="mambo")
    ap.add_argument("--no-cpu-baseline", action="store_true")
    ap.add_argument("--no-prefill", action="store_true", help="skip the prefill block (BASELINE config 3)")
    ap.add_argument("--no-tp", action="store_true", help="skip the tensor-parallel block (BASELINE config 5)")
    ap.add_argument("--no-model", action="store_true", help="skip the whole-model block (BASELINE config 4)")
    ap.add_argument("--no-q4k", action="store_true", help="skip the Q4_K decode block")
    ap.add_argument("--single", metavar="N,K,M",
                    help="profiling mode: run four linears of one shape (random IQ3_S weights) and exit")
    ap.add_argument("--kernel", type=int, default=None, help="with --single: MAMBO_KERNEL_* to use")
    ap.add_argument("--q4k", action="store_true",
                    help="with --single: four Q4_K launches of the shape first, then the IQ3_S ones prequantized")
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

    del graph, graph_sep, g_e2e, g_pipe, layers
    torch.cuda.synchronize(dev)
    torch.cuda.empty_cache()
    # BASELINE config 5 on every rank (tensor parallel over the launched GPUs).
    tp = None if args.no_tp else tp_block(torch, world, rank, dev, args.steps, args.warmup)
    if world > 1:
        dist.barrier()
        dist.destroy_process_group()
    if rank != 0:
        return

    # Single-GPU blocks (4 and 1) at N = 1 only.
    prefill = None if (args.no_prefill or world > 1) else prefill_block(torch, dev)
    model = None if (args.no_model or world > 1) else model_block(torch, dev)
    q4k = None if (args.no_q4k or world > 1) else q4k_block(torch, dev)
    cpu = None if (args.no_cpu_baseline or world > 1) else cpu_baseline()
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
                                "(mambo_iq3s_linear_group), preceded by its activation-quantization pre-pass "
                                "(group_xtiles_kernel, one small launch)",
                   "parallelism": f"replicas{world}"},
        "roofline": {"bound": "hbm", "achieved": achieved, "peak": peak, "unit": "GB/s", "frac": achieved / peak,
                     "traffic": None, "peak_kind": peak_kind,
                     "kernel": "iq3s_gemv_tm_kernel<1,8,GemvGroupPre>: the 20 linears of a step in one launch, "
                               "activations quantized by its pre-pass",
                     "launch_us": group_us,
                     "timing": "10 back-to-back grouped calls (pre-pass + GEMV) in one CUDA graph, 5 replays, mean; "
                               "the pre-pass's time is counted against the GEMV"},
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
        # per step: the quantization pre-pass and one grouped GEMV launch
        "gpu_launches": 2 * args.steps,
        "clocks": clock,
        "cpu_baseline": cpu,
        # prefill from bf16 activations, TFLOP/s half of the metric
        "prefill": prefill,
        # Llama-3-70B layer, tensor parallel over the N GPUs of this run
        "tp": tp,
        # every linear of a 32-layer Llama-3-8B
        "model": model,
        # the decode sweep's linears with Q4_K weights (the next GGUF type)
        "q4k": q4k,
    }
    print(json.dumps(line), flush=True)


if __name__ == "__main__":
    main()
