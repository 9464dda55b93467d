"""Device-timed autotuning and GGUF benchmark command.

Mirror of src/python/mambo/utils/kernel_benchmark.py (Menooker/Mambo): the same
``BenchmarkCase`` fields, ``mini_benchmark`` flow (exhaustive search, then
re-timing the winner host-synced, batched and with CUDA events) and CLI. The
search is timed on the device with CUDA events instead of cuTile's tuner, and
the winner of each case is recorded per (M, N, K) so later launches of that
shape use it (``iq3_s_fp8.register_tuned_config``); ``save_path`` writes the
records as JSON for ``iq3_s_fp8.load_tuned_configs``.

Run ``python -m mambo_b200.utils.kernel_benchmark --help``.
"""

from __future__ import annotations

import argparse
import importlib
import json
import tempfile
from dataclasses import dataclass, field
from pathlib import Path
from time import perf_counter
from typing import Any, Callable, Sequence

import numpy as np
import torch

Config = dict[str, Any]


@dataclass(frozen=True)
class BenchmarkCase:
    name: str
    stream: Any
    kernel: Callable[..., None]  # kernel(*args_fn(config)) launches one instance on `stream`
    search_space: Sequence[Config]
    grid_fn: Callable[[Config], tuple[int, ...]]
    args_fn: Callable[[Config], tuple[Any, ...]]
    hints_fn: Callable[[Config], dict[str, Any]] | None = None
    summary_keys: tuple[str, ...] = ()
    # Per-invocation state reset, included in reported timings after tuning.
    before_launch_fn: Callable[[Config], None] | None = None
    shape: tuple[int, int, int] | None = field(default=None)  # (M, N, K) the winner is recorded for


# Launches captured per timed graph, at least: a case that rotates weight copies
# (make_benchmark_cases) then takes each copy once per replay.
MIN_GRAPH_LAUNCHES = 32


def _event_time_us(case: BenchmarkCase, config: Config, warmup: int, iters: int) -> float:
    """Mean device time of one launch: `iters` launches captured into one CUDA graph, replayed and timed
    with CUDA events on the case's stream (eager launches from Python cannot keep a microsecond-scale
    decode kernel fed; a graph runs them back to back, as a serving step does). Falls back to eager
    launches when the stream cannot be captured (e.g. the legacy default stream) or a per-launch reset
    is needed."""
    args = case.args_fn(config)

    def launch() -> None:
        if case.before_launch_fn is not None:
            case.before_launch_fn(config)
        case.kernel(*args)

    with torch.cuda.stream(case.stream):
        for _ in range(warmup):
            launch()  # eager: sizes the workspace outside any capture
    case.stream.synchronize()
    graph = None
    if case.before_launch_fn is None and case.stream != torch.cuda.default_stream(case.stream.device):
        try:
            graph = torch.cuda.CUDAGraph()
            glaunches = max(iters, MIN_GRAPH_LAUNCHES)
            with torch.cuda.graph(graph, stream=case.stream):
                for _ in range(glaunches):
                    launch()
        except RuntimeError:
            graph = None
    start, stop = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    with torch.cuda.stream(case.stream):
        if graph is not None:
            graph.replay()  # warm replay
            start.record(case.stream)
            reps = 3
            for _ in range(reps):
                graph.replay()
            stop.record(case.stream)
        else:
            reps = 1
            start.record(case.stream)
            for _ in range(iters):
                launch()
            stop.record(case.stream)
    stop.synchronize()
    return start.elapsed_time(stop) * 1000.0 / (glaunches * reps if graph is not None else iters)


def mini_benchmark(cases: Sequence[BenchmarkCase], *, warmup: int = 5, iters: int = 20, quiet: bool = False,
                   save_path: str | Path | None = None) -> list[dict]:
    """Tune each case, then time its winner with any required per-launch reset."""
    results = []
    records = []
    for case in cases:
        successes, failures = [], []
        for config in case.search_space:
            try:
                successes.append((_event_time_us(case, config, 2, max(3, iters // 4)), config))
            except (ValueError, RuntimeError) as exc:
                failures.append((config, str(exc)))
        if not successes:
            raise RuntimeError(f"{case.name}: no configuration ran ({failures[:1]})")
        tuner_us, best = min(successes, key=lambda r: r[0])
        args = case.args_fn(best)

        def launch_once() -> None:
            if case.before_launch_fn is not None:
                case.before_launch_fn(best)
            case.kernel(*args)

        def measure(*, batched: bool) -> float:
            with torch.cuda.stream(case.stream):
                for _ in range(warmup):
                    launch_once()
                    if not batched:
                        case.stream.synchronize()
                case.stream.synchronize()
                start = perf_counter()
                for _ in range(iters):
                    launch_once()
                    if not batched:
                        case.stream.synchronize()
                case.stream.synchronize()
            return (perf_counter() - start) * 1e6 / iters

        mean_us = measure(batched=False)
        batched_us = measure(batched=True)
        event_us = _event_time_us(case, best, warmup, iters)
        if not quiet:
            print(f"{case.name}: best_config={best}, mean_us={mean_us:.3f}, batched_us={batched_us:.3f}, "
                  f"event_us={event_us:.3f}, tuner_us={tuner_us:.3f} (warmup={warmup}, iterations={iters}), "
                  f"candidates={len(successes)} passed/{len(failures)} failed")
        by_group: dict[tuple, float] = {}
        if case.summary_keys:
            for t, cfg in successes:
                key = tuple(cfg.get(k) for k in case.summary_keys)
                by_group[key] = min(by_group.get(key, float("inf")), t)
            if not quiet:
                print(f"  best latency by {case.summary_keys} (us): {by_group}")
        if case.shape is not None:
            from ..kernels.iq3_s_fp8 import register_tuned_config

            m, n, k = case.shape
            register_tuned_config(m, n, k, best)
            records.append({"m": m, "n": n, "k": k, "config": best, "event_us": event_us})
        results.append({"name": case.name, "best": best, "mean_us": mean_us, "batched_us": batched_us,
                         "event_us": event_us, "tuner_us": tuner_us, "passed": len(successes),
                         "failed": len(failures), "by_group": {str(k): v for k, v in by_group.items()}})
    if save_path is not None:
        Path(save_path).write_text(json.dumps(records, indent=1))
    return results


def load_gguf_weight(model: Path, weight_name: str, expected_type: str) -> torch.Tensor:
    """Load a named 2D packed GGUF tensor as uint8 [N, K/block_elements, block_bytes] on the GPU.

    Mirrors kernel_benchmark.py:103-122, reading the file with the gguf package.
    """
    from gguf import GGUFReader

    reader = GGUFReader(str(model))
    tensor = next((t for t in reader.tensors if t.name == weight_name), None)
    if tensor is None:
        raise ValueError(f"GGUF has no tensor named {weight_name!r}")
    if tensor.tensor_type.name.lower() != expected_type.lower() or len(tensor.shape) != 2:
        raise ValueError(f"{weight_name} must be a 2D {expected_type} tensor")
    k, n_rows = (int(v) for v in tensor.shape)
    block_values, block_bytes = 256, 110
    raw = np.asarray(tensor.data, dtype=np.uint8).reshape(n_rows, k // block_values, block_bytes)
    return torch.from_numpy(np.ascontiguousarray(raw)).cuda()


# Add a kernel module and an entry here for each new benchmark.
_BENCHMARKS = {
    "iq3_s_fp8": ("iq3_s", "mambo_b200.kernels.iq3_s_fp8", "make_benchmark_cases"),
}


def _merge_records(path: Path, records: list[dict]) -> None:
    """Write ``records`` into the JSON list at ``path``, replacing entries of the same (m, n, k)."""
    old = json.loads(path.read_text()) if path.is_file() else []
    keep = {(r["m"], r["n"], r["k"]): r for r in old}
    keep.update({(r["m"], r["n"], r["k"]): r for r in records})
    path.write_text(json.dumps([keep[key] for key in sorted(keep)], indent=1) + "\n")


def benchmark_main(argv: Sequence[str] | None = None) -> None:
    parser = argparse.ArgumentParser(description="Autotune an sm_100a kernel on a GGUF weight (or synthetic ones)")
    parser.add_argument("kernel", choices=sorted(_BENCHMARKS))
    parser.add_argument("--model", type=Path, help="GGUF model path")
    parser.add_argument("--weight-name", help="tensor name in the GGUF model")
    parser.add_argument("--synthetic", metavar="N,K", nargs="+",
                        help="seeded random IQ3_S weights of these shapes instead")
    parser.add_argument("--m", type=int, nargs="*", default=[4, 128], help="token counts to tune")
    parser.add_argument("--save", type=Path, help="write the tuned configs as JSON (merged into an existing file)")
    args = parser.parse_args(argv)

    expected_type, kernel_module, factory = _BENCHMARKS[args.kernel]
    make_cases = getattr(importlib.import_module(kernel_module), factory)
    if args.synthetic:
        weights = []
        for shape in args.synthetic:
            n, k = (int(v) for v in shape.split(","))
            rng = np.random.default_rng(0x1A3)
            raw = rng.integers(0, 256, size=(n, k // 256, 110), dtype=np.uint8)
            raw[..., :2] = rng.uniform(1e-3, 1e-2, size=(n, k // 256)).astype("<f2").view(np.uint8).reshape(n, -1, 2)
            weights.append(torch.from_numpy(raw).cuda())
    else:
        if args.model is None or args.weight_name is None:
            parser.error("--model and --weight-name are required without --synthetic")
        weights = [load_gguf_weight(args.model, args.weight_name, expected_type)]
    records = []
    for weight in weights:
        with tempfile.TemporaryDirectory() as tmp_dir:
            tmp = Path(tmp_dir) / "tuned.json"
            mini_benchmark(make_cases(weight, ms=tuple(args.m)), save_path=tmp)
            records += json.loads(tmp.read_text())
        del weight
        torch.cuda.empty_cache()
    if args.save is not None:
        _merge_records(args.save, records)


if __name__ == "__main__":
    benchmark_main()
