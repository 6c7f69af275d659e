#!/usr/bin/env python
"""bench.py -- the GPT-2 token loop on B200: greedy-generation tokens/s, the
roofline of the dominant kernel and of the whole step, and the reference's CPU
path beside it.

One step = one pass of the hot path over one batch: a prefill of every prompt
and the greedy decode of every new token, for the sequences this rank holds.
The headline workload is the batch-sharded throughput configuration (GPT-2
small fp32, 256 sequences x (64-token prompt + 448 greedy tokens), split 256/N
per GPU with no collective on the data path). At one GPU the default run adds
a `workloads` block, timed in the same process: batch-1 decode (GPT-2 small,
prompt 128, 128 greedy), the prefill sweep (batch 1 and 8 x prompt 128, 512,
1024), GPT-2 medium fp32/bf16 (batch 8, prompt 512, 256 greedy) and GPT-2 XL
fp32/bf16/int8 (batch 1, prompt 896, 128 greedy). Weights are seeded
random-init N(0, 0.02) (LayerNorm 1/0), prompts seeded uniform ids: synthetic
data of each configuration's shapes.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME]
                    [--workloads auto|none|NAME,...] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU; rank 0 prints one JSON line and
writes a results record in the reference harness's format (tie_b200.results).
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics
import subprocess
import sys
import tempfile
import time

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "transformer-inference-engine_b200"))

import numpy as np  # noqa: E402

from tie_b200 import results, synth  # noqa: E402
from tie_b200.shard import dist_env, shard_range  # noqa: E402

METRIC = "GPT-2 prefill & decode tokens/s at 1/2/4/8 B200; % of HBM/tensor roofline"

WORKLOADS = {
    # GPT-2 small fp32 throughput run: 256 independent sequences x (64 prompt + 448 greedy)
    "throughput": dict(shape="small", n_seq=256, n_prompt=64, n_new=448, prompt_seed=105),
    # GPT-2 small fp32, batch 1, prompt 128, greedy 128
    "decode1": dict(shape="small", n_seq=1, n_prompt=128, n_new=128, prompt_seed=101),
    # GPT-2 small fp32 prefill, batch 8 x 1024 tokens (the first new token included)
    "prefill": dict(shape="small", n_seq=8, n_prompt=1024, n_new=1, prompt_seed=102),
    # GPT-2 medium fp32, batch 8, prompt 512, greedy 256
    "medium": dict(shape="medium", n_seq=8, n_prompt=512, n_new=256, prompt_seed=103),
    # GPT-2 medium with bf16 weights (fp32 accumulate)
    "medium_bf16": dict(shape="medium", n_seq=8, n_prompt=512, n_new=256, prompt_seed=103, fmt="bf16"),
    # GPT-2 XL fp32, batch 1, prompt 896, greedy 128
    "xl": dict(shape="xl", n_seq=1, n_prompt=896, n_new=128, prompt_seed=104),
    # GPT-2 XL with bf16 / int8 per-output-channel weights (fp32 accumulate)
    "xl_bf16": dict(shape="xl", n_seq=1, n_prompt=896, n_new=128, prompt_seed=104, fmt="bf16"),
    "xl_int8": dict(shape="xl", n_seq=1, n_prompt=896, n_new=128, prompt_seed=104, fmt="int8"),
    # a small case of the throughput shapes, for profiler captures
    "probe": dict(shape="small", n_seq=64, n_prompt=64, n_new=16, prompt_seed=105),
}
# the prefill sweep: batch 1 and 8 x prompt 128, 512, 1024, prefill only
for _b in (1, 8):
    for _t in (128, 512, 1024):
        WORKLOADS[f"prefill_b{_b}_t{_t}"] = dict(shape="small", n_seq=_b, n_prompt=_t, n_new=1, prompt_seed=102)

# what the default one-GPU run times beside the headline, grouped by model
SUITE = ["decode1"] + [f"prefill_b{b}_t{t}" for b in (1, 8) for t in (128, 512, 1024)] + \
        ["medium", "medium_bf16", "xl", "xl_bf16", "xl_int8"]
WEIGHT_SEED = 1234
FMT_CODE = {"bf16": 1, "int8": 2}   # TIE_WEIGHTS_BF16, TIE_WEIGHTS_INT8


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--workload", default="throughput", choices=sorted(WORKLOADS))
    p.add_argument("--workloads", default="auto",
                   help="extra workloads timed after the headline at one GPU: 'auto' (the full suite "
                        "when the headline is the default throughput run), 'none', or a comma list")
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true")
    p.add_argument("--results-dir", default=os.path.join(ROOT, "bench_results"))
    p.add_argument("--kernel", default=None,
                   help="time one kernel alone (model_time_kernel) instead of the workload; "
                        "used for profiler captures on a small case")
    p.add_argument("--rows", type=int, default=128)
    p.add_argument("--context", type=int, default=256)
    p.add_argument("--iters", type=int, default=3)
    p.add_argument("--shape", default="small", choices=["small", "medium", "xl"],
                   help="model of the --kernel mode")
    p.add_argument("--fmt", default="f32", choices=["f32", "bf16", "int8"], help="weight format of the --kernel mode")
    return p.parse_args()


# ------------------------------------------------------------ arithmetic --
def dims(shape):
    s = synth.SHAPES[shape]
    return s.n_embd, s.n_head, s.n_layer, s.vocab_size


def matrix_params(shape):
    """Every matrix the decode streams, the tied head included."""
    E, _, L, V = dims(shape)
    return 12 * E * E * L + V * E


def vector_params(shape):
    """LayerNorm gains/shifts and biases: 13 E per layer plus LN_f."""
    E, _, L, _ = dims(shape)
    return 13 * E * L + 2 * E


def weight_bytes(shape, fmt):
    E, _, L, V = dims(shape)
    w = {"f32": 4, "bf16": 2, "int8": 1}[fmt]
    scales = 4 * (9 * E * L + V) if fmt == "int8" else 0   # one fp32 scale per output row
    return w * matrix_params(shape) + scales


def decode_step_bytes(shape, fmt, rows, ctx):
    """Algorithmic bytes of one decode step of `rows` sequences at mean context
    `ctx`: every weight once, every sequence's cached K/V read once and its new
    K/V row written, the embedding rows read."""
    E, _, L, _ = dims(shape)
    return (weight_bytes(shape, fmt) + 4 * vector_params(shape)
            + rows * (L * 2 * E * 4 * ctx + L * 2 * E * 4 + 2 * E * 4))


def prefill_flops(shape, rows, T):
    """Algorithmic FLOPs of a prefill of `rows` prompts of T tokens with the
    head at the last position only (what a greedy generation computes);
    causal attention counts the T(T+1)/2 pairs."""
    E, _, L, V = dims(shape)
    return rows * (T * 2.0 * 12 * E * E * L + 2.0 * E * V + 4.0 * E * L * T * (T + 1) / 2)


def mean_context(wl):
    return wl["n_prompt"] + wl["n_new"] // 2


# ------------------------------------------------------------------ clocks --
class ClockSampler:
    """nvidia-smi sampled every 200 ms while the timed region runs."""
    Q = ("index,clocks.sm,clocks.max.sm,power.draw,clocks_event_reasons.hw_slowdown,"
         "clocks_event_reasons.hw_thermal_slowdown,clocks_event_reasons.sw_thermal_slowdown,"
         "clocks_event_reasons.sw_power_cap")

    def __init__(self, gpus):
        self.gpus = set(gpus)
        self.f = tempfile.NamedTemporaryFile("w+", suffix=".csv", delete=False)
        try:
            self.p = subprocess.Popen(["nvidia-smi", f"--query-gpu={self.Q}", "--format=csv,noheader,nounits",
                                       "-lms", "200"], stdout=self.f, stderr=subprocess.DEVNULL)
        except OSError:
            self.p = None

    def stop(self):
        if self.p:
            self.p.terminate()
            try:
                self.p.wait(timeout=5)
            except subprocess.TimeoutExpired:
                self.p.kill()
        self.f.flush()
        rows = []
        for line in open(self.f.name):
            parts = [x.strip() for x in line.split(",")]
            if len(parts) < 8 or not parts[0].isdigit() or int(parts[0]) not in self.gpus:
                continue
            rows.append(parts)
        os.unlink(self.f.name)
        if not rows:
            return {"sm_mhz": None, "sm_max_mhz": None, "reasons": ["unsampled"]}
        names = ["hw_slowdown", "hw_thermal_slowdown", "sw_thermal_slowdown", "sw_power_cap"]
        reasons = sorted({names[i] for r in rows for i in range(4) if r[4 + i] == "Active"})
        sm = [float(r[1]) for r in rows if r[1].replace(".", "").isdigit()]
        mx = [float(r[2]) for r in rows if r[2].replace(".", "").isdigit()]
        return {"sm_mhz": statistics.median(sm) if sm else None, "sm_max_mhz": max(mx) if mx else None,
                "reasons": reasons, "samples": len(rows)}


# ------------------------------------------------------------ CPU baseline --
def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def sample_contexts(wl):
    """Decode contexts the CPU is timed at: the first step, the mean and the last."""
    if wl["n_new"] < 2:
        return []
    first, last = wl["n_prompt"] + 1, wl["n_prompt"] + wl["n_new"] - 1
    return sorted({first, min(last, max(first, mean_context(wl))), last})


def cpu_sampled(w, inv, cfg, prompts, wl, cores, rounds):
    """The reference's own CPU engine (oracle/_ref/ref_gpt2, compiled from its
    sources; else the C restatement of it) on `cores` concurrent processes, one
    sequence each, pinned one per core. Each times the prefill of its whole
    prompt once, then `rounds` rounds of one cached decode step at each of
    sample_contexts(wl). Returns per-core dicts and the checker's kind."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # test/bench infrastructure only: the CPU baseline leg and the reference arm
    kind = "reference" if oracle.reference_available() else "port"
    if kind == "port":
        oracle.build()
    ctx = sample_contexts(wl)
    ctx_arg = ",".join(str(c) for c in ctx) if ctx else "none"
    T, n_new = wl["n_prompt"], wl["n_new"]
    out = []
    with tempfile.TemporaryDirectory() as td:
        ids_path = os.path.join(td, "ids.bin")
        np.ascontiguousarray(prompts[:cores], np.int32).tofile(ids_path)
        procs = []
        cpus = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else list(range(cores))
        for c in range(cores):
            if kind == "reference":
                cmd = [oracle.REF_BIN, w, inv, cfg, ids_path, "1", str(T), str(max(n_new, 2)),
                       os.path.join(td, f"o{c}.bin"), "--first-seq", str(c), "--time-contexts", ctx_arg,
                       "--rounds", str(rounds)]
            else:
                if not ctx:
                    ctx_arg = str(T + 1)
                cmd = [sys.executable, os.path.join(ROOT, "oracle", "port_driver.py"), w, cfg, ids_path,
                       str(c), str(T), str(max(n_new, 2)), ctx_arg, str(rounds)]
            cpu = cpus[c % len(cpus)]
            procs.append(subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                                          preexec_fn=lambda cpu=cpu: os.sched_setaffinity(0, {cpu})))
        for p in procs:
            o, err = p.communicate()
            if p.returncode != 0:
                raise RuntimeError(f"CPU baseline failed: {err.strip()}")
            d = json.loads(o.strip().splitlines()[-1])
            if not ctx:
                d["contexts"], d["rounds"] = [], [[] for _ in d["rounds"]]
            out.append(d)
    return out, kind


def seq_ms_from_samples(prefill_ms, contexts, step_ms, wl):
    """A whole generation's CPU time from measured costs: the measured prefill
    of the full prompt, plus every decode step's cost from a least-squares line
    through the measured (context, step ms) samples (a step's cost is a fixed
    part, the matmuls, plus a part proportional to the context, the attention)."""
    n_new, T = wl["n_new"], wl["n_prompt"]
    if n_new < 2:
        return prefill_ms
    x = np.asarray(contexts, np.float64)
    y = np.asarray(step_ms, np.float64)
    if len(x) > 1 and np.ptp(x) > 0:
        b, a = np.polyfit(x, y, 1)
    else:
        a, b = float(y.mean()), 0.0
    steps = np.arange(T + 1, T + n_new, dtype=np.float64)   # step g attends over T + g positions
    return prefill_ms + float(np.sum(a + b * steps))


def cpu_rate(per_core, wl, round_index):
    """Aggregate tokens/s of the cores, from one round of samples."""
    rate = 0.0
    for d in per_core:
        ms = seq_ms_from_samples(d["prefill_ms"], d["contexts"], d["rounds"][round_index], wl)
        tokens = wl["n_new"] if wl["n_new"] > 1 else wl["n_prompt"]
        rate += tokens / (ms / 1e3)
    return rate


def sample_text(wl, cores, kind):
    ctx = sample_contexts(wl)
    dec = (f"then one cached decode step at each context {ctx}; a generation's time is the prefill plus "
           f"all {wl['n_new'] - 1} decode steps from the least-squares line through those samples"
           if ctx else "(prefill only)")
    return (f"{cores} concurrent sequences, one per core ({'the reference C engine compiled from its sources' if kind == 'reference' else 'the C restatement'}): "
            f"the full {wl['n_prompt']}-token prompt prefilled and timed, {dec}")


def config_of(name, wl, world):
    size = shard_range(wl["n_seq"], 0, world)[1]
    E, _, _, _ = dims(wl["shape"])
    return {"workload": name, "model": f"gpt2-{wl['shape']}", "weights": wl.get("fmt", "f32"),
            "n_seq": wl["n_seq"], "n_prompt": wl["n_prompt"], "n_new": wl["n_new"], "seq_per_gpu": size,
            "weight_seed": WEIGHT_SEED, "prompt_seed": wl["prompt_seed"],
            "parallelism": f"batch-sharded x{world}, no collective",
            "l2": f"inputs larger than L2 (weights {weight_bytes(wl['shape'], wl.get('fmt', 'f32')) / 1e9:.2f} GB)",
            "step": ("one greedy generation over the batch: prefill + (n_new - 1) decode steps" if wl["n_new"] > 1
                     else "one prefill of every prompt, the first greedy token included")}


def unit_tokens(wl):
    """Tokens one step produces: the generated ones, or for a prefill-only
    workload (one new token) the prompt tokens it processes."""
    return wl["n_seq"] * (wl["n_new"] if wl["n_new"] > 1 else wl["n_prompt"])


def run_reference_arm(args, rank, world):
    if rank != 0:
        return 0
    wl = WORKLOADS[args.workload]
    w, inv, cfg = synth.ensure_model(wl["shape"], seed=WEIGHT_SEED)
    V = synth.SHAPES[wl["shape"]].vocab_size
    cores = max(1, min(host_cores(), wl["n_seq"], 64))
    prompts = synth.prompt_ids(V, max(cores, 1), wl["n_prompt"], wl["prompt_seed"])
    t0 = time.perf_counter()
    per_core, kind = cpu_sampled(w, inv, cfg, prompts, wl, cores, rounds=args.warmup + args.steps)
    wall = time.perf_counter() - t0
    vals = [cpu_rate(per_core, wl, r) for r in range(args.warmup, args.warmup + args.steps)]
    value = statistics.median(vals)
    ms_step = unit_tokens(wl) / value * 1e3
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": ms_step, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference", "config": config_of(args.workload, wl, world),
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind,
                             "sample": sample_text(wl, cores, kind),
                             "prefill_ms": statistics.mean(d["prefill_ms"] for d in per_core),
                             "contexts": per_core[0]["contexts"],
                             "step_ms_by_context": [statistics.mean(d["rounds"][r][i] for d in per_core
                                                                    for r in range(args.warmup, args.warmup + args.steps))
                                                    for i in range(len(per_core[0]["contexts"]))]},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": round(wall, 1)}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------- our arm --

# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of a
# roofline kernel, from one ncu capture of that kernel at exactly the shape the
# workload times it at: (shape, kernel, rows, context) -> bytes
NCU_TRAFFIC = {
    ("small", "decode_attention", 256, 288): 453_862_912 + 8_279_296,
    ("small", "decode_attention", 1, 192): 1_223_424 + 0,
}


def measure_tf32_peak():
    """Dense TF32 tensor throughput of this GPU: cuBLAS (torch.matmul) on
    8192^3 fp32 operands with TF32 allowed, best of 10, CUDA events -- the
    measurement the bf16 figure of MEASURED_PEAKS.json uses, in TF32."""
    import torch
    mm = torch.backends.cuda.matmul
    prev = mm.allow_tf32
    mm.allow_tf32 = True
    try:
        n = 8192
        g = torch.Generator(device="cuda").manual_seed(0)
        a = torch.randn(n, n, device="cuda", generator=g)
        b = torch.randn(n, n, device="cuda", generator=g)
        for _ in range(3):
            torch.matmul(a, b)
        best = float("inf")
        for _ in range(10):
            e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
            e0.record()
            torch.matmul(a, b)
            e1.record()
            torch.cuda.synchronize()
            best = min(best, e0.elapsed_time(e1))
        del a, b
        torch.cuda.empty_cache()
        return 2.0 * n ** 3 / (best * 1e-3) / 1e12
    finally:
        mm.allow_tf32 = prev


def load_peaks():
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    return peaks


def kernel_table(wl, rows, measured, peaks):
    """Per-kernel live timings (CUDA events, each kernel alone at the
    workload's shapes) with each one's roofline. The tensor-core matmuls compute
    fp32-accurate products as three TF32 MMAs (3xTF32), so their ceiling is the
    measured TF32 peak / 3; the decode matmuls also carry their HBM fraction on
    the fp32 weight bytes they must read."""
    E, _, L, V = dims(wl["shape"])
    fmt = wl.get("fmt", "f32")
    wbytes = {"f32": 4, "bf16": 2, "int8": 1}[fmt]
    ctx = mean_context(wl)
    steps = wl["n_new"] - 1
    hbm = peaks.get("hbm_gbs", 6650.0)
    tf32 = peaks.get("tf32_tflops")
    ceiling = tf32 / 3 if tf32 else peaks.get("bf16_tflops", 1590.0) / 6
    k = {}

    def add(name, ms, per_gen, kind, work, hbm_work=None):
        if ms is None:
            return
        e = {"ms": ms, "launches_per_gen": per_gen}
        if kind == "hbm":
            e.update(bound="hbm", achieved=work / (ms * 1e-3) / 1e9, unit="GB/s", peak=hbm,
                     peak_source="measured HBM copy")
        else:
            e.update(bound="tensor", achieved=work / (ms * 1e-3) / 1e12, unit="TFLOP/s", peak=ceiling,
                     peak_source=("measured TF32 (cuBLAS 8192^3) / 3 MMAs per fp32-accurate product" if tf32
                                  else "fallback: bf16 peak / 6"))
        e["frac"] = e["achieved"] / e["peak"]
        if hbm_work is not None:
            e["hbm_achieved"] = hbm_work / (ms * 1e-3) / 1e9
            e["hbm_frac"] = e["hbm_achieved"] / hbm
        e["share_ms"] = ms * per_gen
        e["work_per_launch"] = work
        k[name] = e

    if steps > 0 and "decode_step" in measured:
        add("decode_step", measured.get("decode_step"), steps, "hbm",
            decode_step_bytes(wl["shape"], fmt, rows, ctx))
    elif steps > 0:
        add("decode_attention", measured.get("decode_attention"), L * steps, "hbm",
            rows * ctx * 2 * E * 4 + rows * 2 * E * 4)
        for name, N, K in (("decode_qkv", 3 * E, E), ("decode_fc", 4 * E, E), ("decode_mlp_proj", E, 4 * E)):
            ms = measured.get(name)
            wb = N * K * wbytes + rows * (N + K) * 4
            if rows <= 8:   # the streaming GEMVs
                add(name, ms, L * steps, "hbm", wb)
            else:
                add(name, ms, L * steps, "tensor", 2.0 * rows * N * K, hbm_work=N * K * 4 + rows * (N + K) * 4)
        if rows <= 8:
            add("decode_head", measured.get("decode_head"), steps, "hbm", V * E * wbytes + rows * V * 4)
        else:
            add("decode_head", measured.get("decode_head"), steps, "tensor", 2.0 * rows * V * E,
                hbm_work=V * E * 4 + rows * V * 4)
    else:
        T = wl["n_prompt"]
        add("prefill_fc", measured.get("prefill_fc"), L, "tensor", 2.0 * rows * T * 4 * E * E)
        add("prefill_attention", measured.get("prefill_attention"), L, "tensor",
            4.0 * rows * E * T * (T + 1) / 2)
    return k


def dominant_roofline(wl, rows, k, peaks):
    dom = max(k, key=lambda n: k[n]["share_ms"])
    d = k[dom]
    ctx = mean_context(wl) if wl["n_new"] > 1 else wl["n_prompt"]
    return {"kernel": dom, "bound": d["bound"], "achieved": d["achieved"], "peak": d["peak"], "unit": d["unit"],
            "frac": d["frac"], "traffic": NCU_TRAFFIC.get((wl["shape"], dom, rows, ctx)),
            "peak_source": "measured" if peaks else "fallback", "work_per_launch": d["work_per_launch"]}


def timed_steps(step, steps, warmup, stream, barrier=lambda: None):
    """W untimed steps, then K steps bracketed by a barrier and a synchronize
    on both sides, with a CUDA event between steps on the model's stream.
    Returns (mean ms per step, per-step ms)."""
    import torch
    for _ in range(warmup):
        step()
    torch.cuda.synchronize()
    evs = [torch.cuda.Event(enable_timing=True) for _ in range(steps + 1)]
    barrier()
    torch.cuda.synchronize()
    evs[0].record(stream)
    for i in range(steps):
        step()
        evs[i + 1].record(stream)
    torch.cuda.synchronize()
    barrier()
    per = [evs[i].elapsed_time(evs[i + 1]) for i in range(steps)]
    return evs[0].elapsed_time(evs[-1]) / steps, per


class Generation:
    """One workload's batch on one model: prompts on the device and pinned on
    the host, and the two ways to run a step (device API, host API)."""

    def __init__(self, m, wl, prompts):
        import torch
        self.m, self.wl = m, wl
        self.S, self.T, self.n_new = prompts.shape[0], wl["n_prompt"], wl["n_new"]
        m.batch_reserve(self.S, self.T + self.n_new - 1)
        self.stream = torch.cuda.ExternalStream(m.stream)
        self.d_prompts = torch.from_numpy(prompts).to("cuda")
        self.d_out = torch.zeros((self.S, self.n_new), dtype=torch.int32, device="cuda")
        self.h_prompts = torch.from_numpy(prompts).pin_memory()
        self.h_out = torch.zeros((self.S, self.n_new), dtype=torch.int32).pin_memory()
        torch.cuda.synchronize()

    def device_step(self):
        self.m.generate_greedy_device(self.d_prompts.data_ptr(), self.S, self.T, self.n_new, self.d_out.data_ptr())

    def host_step(self):
        import tie_b200
        rc = tie_b200.library().model_generate_greedy(
            self.m.h, C.cast(self.h_prompts.data_ptr(), C.POINTER(C.c_int32)), self.S, self.T, self.n_new,
            C.cast(self.h_out.data_ptr(), C.POINTER(C.c_int32)))
        if rc != 0:
            raise tie_b200.ModelError(rc, "model_generate_greedy")

    def e2e_ms(self, steps, barrier=lambda: None, reduce=lambda x: x):
        """Wall time per step through the public host API: pinned prompts in,
        ids out, inside the timed region."""
        self.host_step()
        barrier()
        t0 = time.perf_counter()
        for _ in range(steps):
            self.host_step()
        ms = reduce((time.perf_counter() - t0) * 1e3 / steps)
        assert np.array_equal(self.h_out.numpy(), self.d_out.cpu().numpy()), "host and device paths disagree"
        return ms

    def prefill_ms(self, reps=3, reduce=lambda x: x):
        """The batch prefill alone (model_prefill_batch), device-timed."""
        import torch
        prompts = self.h_prompts.numpy()
        self.m.prefill_batch(prompts)
        e0, e1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        e0.record(self.stream)
        for _ in range(reps):
            self.m.prefill_batch(prompts)
        e1.record(self.stream)
        torch.cuda.synchronize()
        return reduce(e0.elapsed_time(e1) / reps)

    def kernels(self):
        ctx = mean_context(self.wl)
        if self.n_new > 1:
            names = ["decode_attention", "decode_qkv", "decode_fc", "decode_mlp_proj", "decode_head"]
        else:
            names = ["prefill_fc", "prefill_attention"]
        return {n: self.m.time_kernel(n, self.S, ctx if n.startswith("decode") else self.T, iters=20)
                for n in names}

    def close(self):
        del self.d_prompts, self.d_out, self.h_prompts, self.h_out


def phase_block(wl, ms, pre_ms):
    if pre_ms is None:
        return None
    S, T, n_new = wl["n_seq"], wl["n_prompt"], wl["n_new"]
    dec = ms - pre_ms
    return {"prefill_ms": pre_ms, "prefill_tokens_per_s": S * T / (pre_ms / 1e3), "decode_ms": dec,
            "decode_ms_per_step": dec / (n_new - 1), "decode_tokens_per_s": S * (n_new - 1) / (dec / 1e3)}


def step_roofline(wl, rows, ms, pre_ms, peaks):
    """The whole workload against its bound: decode steps against HBM on
    their algorithmic bytes, a prefill-only step against the 3xTF32 tensor
    ceiling on its algorithmic FLOPs."""
    fmt = wl.get("fmt", "f32")
    if wl["n_new"] > 1 and pre_ms is not None:
        per_step_ms = (ms - pre_ms) / (wl["n_new"] - 1)
        b = decode_step_bytes(wl["shape"], fmt, rows, mean_context(wl))
        hbm = peaks.get("hbm_gbs", 6650.0)
        ach = b / (per_step_ms * 1e-3) / 1e9
        return {"scope": "every kernel of one decode step (mean over the horizon)", "bound": "hbm",
                "achieved": ach, "peak": hbm, "unit": "GB/s", "frac": ach / hbm, "bytes_per_step": b,
                "ms_per_step": per_step_ms, "peak_source": "measured HBM copy" if peaks else "fallback"}
    if wl["n_new"] == 1:
        f = prefill_flops(wl["shape"], rows, wl["n_prompt"])
        tf32 = peaks.get("tf32_tflops")
        ceil = tf32 / 3 if tf32 else peaks.get("bf16_tflops", 1590.0) / 6
        ach = f / (ms * 1e-3) / 1e12
        return {"scope": "the whole prefill (matmuls, attention, LayerNorm, head at the last row)",
                "bound": "tensor", "achieved": ach, "peak": ceil, "unit": "TFLOP/s", "frac": ach / ceil,
                "flops_per_step": f,
                "peak_source": ("measured TF32 (cuBLAS 8192^3) / 3 MMAs per fp32-accurate product" if tf32
                                else "fallback: bf16 peak / 6")}
    return None


def run_suite(names, args, peaks, records):
    """Each named workload on one GPU, in this process; models are loaded once
    per shape and switched between weight formats."""
    import tie_b200
    out = {}
    by_shape = {}
    for n in names:
        by_shape.setdefault(WORKLOADS[n]["shape"], []).append(n)
    steps, warmup = max(1, min(args.steps, 5)), max(3, min(args.warmup, 3))
    for shape, group in by_shape.items():
        w, inv, cfg = synth.ensure_model(shape, seed=WEIGHT_SEED)
        V = synth.SHAPES[shape].vocab_size
        m = tie_b200.Model(w, inv, cfg, device=0)
        try:
            for name in group:
                wl = WORKLOADS[name]
                fmt = wl.get("fmt", "f32")
                m.set_weight_format(FMT_CODE.get(fmt, 0))
                prompts = synth.prompt_ids(V, wl["n_seq"], wl["n_prompt"], wl["prompt_seed"])
                g = Generation(m, wl, prompts)
                ms, per = timed_steps(g.device_step, steps, warmup, g.stream)
                e2e = g.e2e_ms(steps)
                pre = g.prefill_ms() if wl["n_new"] > 1 else None
                k = kernel_table(wl, g.S, g.kernels(), peaks)
                tok = unit_tokens(wl)
                entry = {"value": tok / (ms / 1e3), "unit": "tokens/s", "ms_per_step": ms, "steps": steps,
                         "warmup": warmup, "config": config_of(name, wl, 1),
                         "dtype": "f32" if fmt == "f32" else f"{fmt} weights, f32 accumulate",
                         "e2e": {"value": tok / (e2e / 1e3), "unit": "tokens/s", "ms_per_step": e2e,
                                 "h2d_bytes_per_step": int(prompts.nbytes),
                                 "d2h_bytes_per_step": int(g.S * g.n_new * 4)},
                         "roofline": step_roofline(wl, g.S, ms, pre, peaks),
                         "dominant_kernel": dominant_roofline(wl, g.S, k, peaks),
                         "kernels": k}
                ph = phase_block(wl, ms, pre)
                if ph:
                    entry["phases"] = ph
                out[name] = entry
                records.append(results.record(f"tie_b200_{name}", json.dumps(entry["config"]), "tokens/s",
                                              entry["value"], warmup, per,
                                              counters={"tokens_per_step": tok,
                                                        "roofline_frac": entry["roofline"]["frac"],
                                                        "e2e_tokens_per_s": entry["e2e"]["value"]}))
                g.close()
        finally:
            m.close()
    return out


def run_ours(args, rank, local_rank, world):
    import torch
    import torch.distributed as dist
    from datetime import timedelta

    import tie_b200

    wl = WORKLOADS[args.workload]
    torch.cuda.set_device(local_rank)
    if world > 1:
        dist.init_process_group("nccl", timeout=timedelta(seconds=600),
                                device_id=torch.device("cuda", local_rank))

    def barrier():
        if world > 1:
            dist.barrier()

    def max_over_ranks(x):
        if world == 1:
            return x
        t = torch.tensor([x], dtype=torch.float64, device="cuda")
        dist.all_reduce(t, op=dist.ReduceOp.MAX)
        return float(t.item())

    if rank == 0:
        synth.ensure_model(wl["shape"], seed=WEIGHT_SEED)
    barrier()
    w, inv, cfg = synth.ensure_model(wl["shape"], seed=WEIGHT_SEED)
    V = synth.SHAPES[wl["shape"]].vocab_size
    start, size = shard_range(wl["n_seq"], rank, world)
    all_prompts = synth.prompt_ids(V, wl["n_seq"], wl["n_prompt"], wl["prompt_seed"])
    prompts = np.ascontiguousarray(all_prompts[start:start + size])
    fmt = wl.get("fmt", "f32")

    m = tie_b200.Model(w, inv, cfg, device=local_rank)
    if fmt != "f32":
        m.set_weight_format(FMT_CODE[fmt])
    g = Generation(m, wl, prompts)

    sampler = ClockSampler(range(world)) if rank == 0 else None
    l0 = m.kernel_launches()
    ms, per = timed_steps(g.device_step, args.steps, args.warmup, g.stream, barrier)
    # every step launches the same kernels: the timed region's share of the count
    launches = (m.kernel_launches() - l0) // (args.steps + args.warmup) * args.steps
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(ms)
    tok = unit_tokens(wl)
    value = tok / (ms / 1e3)

    e2e_ms = g.e2e_ms(args.steps, barrier, max_over_ranks)
    pre_ms = g.prefill_ms(reduce=max_over_ranks) if wl["n_new"] > 1 else None
    measured = g.kernels()
    peaks = load_peaks()
    if rank == 0:
        try:
            peaks["tf32_tflops"] = measure_tf32_peak()
            peaks["tf32_how"] = "torch.matmul fp32 8192^3 with TF32 allowed (cuBLAS), best of 10, CUDA events"
        except RuntimeError as e:
            peaks["tf32_error"] = str(e)
    k = kernel_table(wl, size, measured, peaks)
    roof = dominant_roofline(wl, size, k, peaks)
    g.close()
    m.close()

    line = None
    records = []
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None,
                "dtype": "f32" if fmt == "f32" else f"{fmt} weights, f32 accumulate",
                "data": "synthetic (seeded random-init weights, seeded uniform token ids)",
                "config": config_of(args.workload, wl, world),
                "e2e": {"value": tok / (e2e_ms / 1e3), "unit": "tokens/s",
                        "h2d_bytes_per_step": int(prompts.nbytes), "d2h_bytes_per_step": int(size * wl["n_new"] * 4),
                        "ms_per_step": e2e_ms},
                "gpu_launches": int(launches),
                "clocks": clocks,
                "roofline": roof,
                "step_roofline": step_roofline(wl, size, ms, pre_ms, peaks),
                "peaks": {k2: peaks[k2] for k2 in ("hbm_gbs", "bf16_tflops", "bf16_tflops_sustained", "tf32_tflops",
                                                   "tf32_how") if k2 in peaks},
                "kernels": k}
        ph = phase_block(wl, ms, pre_ms)
        if ph:
            line["phases"] = ph
        records.append(results.record(f"tie_b200_{args.workload}", json.dumps(line["config"]), "tokens/s", value,
                                      args.warmup, per,
                                      counters={"tokens_per_step": tok, "n_gpus": world,
                                                "roofline_frac": roof["frac"],
                                                "e2e_tokens_per_s": line["e2e"]["value"]},
                                      annotations={"timer": "CUDA events between steps on the model's stream; "
                                                            "max over ranks for the mean"}))
    barrier()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0 and world == 1:
        suite = [] if args.workloads == "none" else (
            (SUITE if args.workload == "throughput" else []) if args.workloads == "auto"
            else [n for n in args.workloads.split(",") if n])
        for n in suite:
            if n not in WORKLOADS:
                raise SystemExit(f"unknown workload {n}")
        if suite:
            line["workloads"] = run_suite(suite, args, peaks, records)
        if not args.no_cpu_baseline:
            cores = max(1, min(host_cores(), wl["n_seq"], 32))
            per_core, kind = cpu_sampled(w, inv, cfg, all_prompts, wl, cores, rounds=1)
            line["cpu_baseline"] = {"value": cpu_rate(per_core, wl, 0), "unit": "tokens/s", "cores": cores,
                                    "kind": kind, "sample": sample_text(wl, cores, kind),
                                    "prefill_ms": statistics.mean(d["prefill_ms"] for d in per_core),
                                    "contexts": per_core[0]["contexts"],
                                    "step_ms_by_context": [statistics.mean(d["rounds"][0][i] for d in per_core)
                                                           for i in range(len(per_core[0]["contexts"]))]}
    if rank == 0:
        try:
            dev = torch.cuda.get_device_name(local_rank) + " sm_100a"
            path = results.write(args.results_dir, f"gpt2_{args.workload}_n{world}", results.header("b200", dev),
                                 records)
            line["results_record"] = os.path.relpath(path, ROOT)
        except OSError as e:
            line["results_record"] = f"not written: {e}"
        print(json.dumps(line), flush=True)
    return 0


def run_kernel(args):
    """One kernel of a GPT-2 forward pass, alone, at (rows, context)."""
    import tie_b200
    w, inv, cfg = synth.ensure_model(args.shape, seed=WEIGHT_SEED)
    m = tie_b200.Model(w, inv, cfg, device=0)
    if args.fmt != "f32":
        m.set_weight_format(FMT_CODE[args.fmt])
    m.batch_reserve(args.rows, args.context)
    ms = m.time_kernel(args.kernel, args.rows, args.context, iters=args.iters)
    print(json.dumps({"kernel": args.kernel, "shape": args.shape, "fmt": args.fmt, "rows": args.rows,
                      "context": args.context,
                      "iters": args.iters, "ms_per_launch": ms}), flush=True)
    m.close()
    return 0


def main():
    args = parse()
    rank, local_rank, world = dist_env()
    if args.kernel:
        return run_kernel(args)
    if args.impl == "reference":
        return run_reference_arm(args, rank, world)
    return run_ours(args, rank, local_rank, world)


if __name__ == "__main__":
    sys.exit(main())
