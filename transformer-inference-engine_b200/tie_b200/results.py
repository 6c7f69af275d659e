"""Results records in the reference benchmark harness's file format.

The reference writes one JSON file per run into bench/results/, and its later
stages read those files directly (reference bench/microbench/bench_common.h:121-184,
BENCHMARK_PROTOCOL.md section 9): a provenance header (stage id, git commit,
timestamps, device, compilers and flags, the protocol's limits) and a list of
records, each with the benchmark name, the configuration, the derived figure
and its units, the warm-up and sample counts, every raw per-sample time in
milliseconds, the summary statistics with a VALID/INVALID verdict, counters and
annotations.  ``bench.py`` writes one such file beside its JSON line, so the
reference's tooling can ingest B200 runs without a converter.

The validity rules are the reference's: at least 5 warm-up iterations, at least
20 samples, and a standard deviation of at most 5% of the median; an invalid
run keeps its numbers and says why (bench_common.h:20-22, 45-53).
"""
from __future__ import annotations

import datetime as _dt
import json
import math
import os
import platform
import shutil
import statistics
import subprocess

MIN_WARMUP = 5
MIN_SAMPLES = 20
MAX_STDDEV_PCT = 5.0

PKG_ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REPO_ROOT = os.path.dirname(PKG_ROOT)


def stats(samples_ms: list[float], warmup: int) -> dict:
    """Every statistic, then the verdict (bench_common.h:45-53)."""
    n = len(samples_ms)
    if n == 0:
        return {"n": 0, "mean_ms": None, "median_ms": None, "min_ms": None, "max_ms": None,
                "stddev_ms": None, "stddev_pct_of_median": None, "valid": False,
                "invalid_reason": "no samples"}
    med = statistics.median(samples_ms)
    sd = statistics.pstdev(samples_ms) if n > 1 else 0.0
    pct = 100.0 * sd / med if med > 0 else math.inf
    reasons = []
    if warmup < MIN_WARMUP:
        reasons.append(f"{warmup} warm-up iterations < {MIN_WARMUP}")
    if n < MIN_SAMPLES:
        reasons.append(f"{n} samples < {MIN_SAMPLES}")
    if pct > MAX_STDDEV_PCT:
        reasons.append(f"stddev {pct:.2f}% of median > {MAX_STDDEV_PCT}%")
    return {"n": n, "mean_ms": statistics.fmean(samples_ms), "median_ms": med, "min_ms": min(samples_ms),
            "max_ms": max(samples_ms), "stddev_ms": sd, "stddev_pct_of_median": pct,
            "valid": not reasons, "invalid_reason": "; ".join(reasons) or None}


def record(benchmark: str, configuration: str, units: str, value: float, warmup: int, samples_ms: list[float],
           counters: dict | None = None, annotations: dict | None = None) -> dict:
    return {"benchmark": benchmark, "configuration": configuration, "units": units, "value": value,
            "warmup_iterations": warmup, "samples_requested": len(samples_ms),
            "raw_samples_ms": [float(x) for x in samples_ms], "statistics": stats(samples_ms, warmup),
            "counters": counters or {}, "annotations": annotations or {}}


def _git_commit() -> str:
    git = shutil.which("git")
    if git:
        try:
            p = subprocess.run([git, "-C", REPO_ROOT, "rev-parse", "HEAD"], capture_output=True, text=True,
                               timeout=10)
            if p.returncode == 0 and p.stdout.strip():
                return p.stdout.strip()
        except (OSError, subprocess.SubprocessError):
            pass
    return "unknown"


def _nvcc_version() -> str:
    nvcc = shutil.which("nvcc") or "/usr/local/cuda/bin/nvcc"
    try:
        p = subprocess.run([nvcc, "--version"], capture_output=True, text=True, timeout=20)
        last = [l for l in p.stdout.splitlines() if l.strip()]
        return f"{last[-2].strip() if len(last) > 1 else 'nvcc'} ({nvcc})"
    except (OSError, subprocess.SubprocessError, IndexError):
        return "unknown"


def header(stage: str, device: str) -> dict:
    from . import build as _b
    lib = _b.LIB_PATH
    built = (_dt.datetime.fromtimestamp(os.path.getmtime(lib), _dt.timezone.utc).strftime("%Y-%m-%dT%H:%M:%SZ")
             if os.path.exists(lib) else None)
    return {"stage": os.environ.get("BENCH_STAGE_ID", stage), "git_commit": _git_commit(),
            "run_timestamp_utc": _dt.datetime.now(_dt.timezone.utc).strftime("%Y-%m-%dT%H:%M:%SZ"),
            "build_timestamp": built, "device": device,
            "cpu_timer": "time.perf_counter (CLOCK_MONOTONIC)",
            "gpu_timer": "cudaEvent on the model's stream + synchronize",
            "cxx_compiler": f"{platform.python_implementation()} host driver; nvcc host pass (-Xcompiler -fPIC,-O3)",
            "cxx_flags": " ".join(_b.NVCC_FLAGS),
            "cuda_compiler": _nvcc_version(), "cuda_flags": " ".join(_b.NVCC_FLAGS),
            "protocol": {"min_warmup": MIN_WARMUP, "min_samples": MIN_SAMPLES,
                         "max_stddev_pct_of_median": MAX_STDDEV_PCT}}


def write(results_dir: str, file_stem: str, head: dict, records: list[dict]) -> str:
    """Writes <results_dir>/<file_stem>.json; returns its path."""
    os.makedirs(results_dir, exist_ok=True)
    path = os.path.join(results_dir, f"{file_stem}.json")
    with open(path, "w") as f:
        json.dump(dict(head, records=records), f, indent=1)
    return path
