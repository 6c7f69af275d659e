#!/usr/bin/env python
"""bench.py -- the GPT-2 token loop on B200: greedy-generation tokens/s, the
roofline of the dominant kernel, and the reference's CPU path beside it.

One step = one pass of the hot path over one batch: a prefill of every prompt
and the greedy decode of every new token, for the sequences this rank holds.
The default workload is the batch-sharded throughput configuration (GPT-2 small
fp32, 256 sequences x (64-token prompt + 448 greedy tokens), split 256/N per GPU
with no collective on the data path); other configurations are selectable with
--workload.  Weights are seeded random-init N(0, 0.02) (LayerNorm 1/0), prompts
seeded uniform ids: synthetic data of the configuration's shapes.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--workload NAME] [--impl ours|reference]

N > 1 runs under torchrun, one rank per GPU; rank 0 prints one JSON line.
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

ROOT = os.path.dirname(os.path.abspath(__file__))
sys.path.insert(0, os.path.join(ROOT, "transformer-inference-engine_b200"))

import numpy as np  # noqa: E402

from tie_b200 import synth  # noqa: E402
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
WEIGHT_SEED = 1234


def parse():
    p = argparse.ArgumentParser()
    p.add_argument("--gpus", type=int, default=1)
    p.add_argument("--steps", type=int, default=5)
    p.add_argument("--warmup", type=int, default=3)
    p.add_argument("--workload", default="throughput", choices=sorted(WORKLOADS))
    p.add_argument("--impl", default="ours", choices=["ours", "reference"])
    p.add_argument("--no-cpu-baseline", action="store_true")
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
def cpu_sample(w, inv, cfg, prompts, cores, prefix=16, n_new=5):
    """The reference's own CPU engine (oracle/_ref/ref_gpt2, compiled from its
    sources; else the C restatement of it) on `cores` concurrent processes, one
    sequence each, pinned one per core.  Each measures a prefill of the first
    `prefix` prompt tokens and n_new - 1 cached decode steps; returns per-core
    (prefill ms, mean step ms) and the kind of checker used."""
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle  # test/bench infrastructure only: the CPU baseline leg
    kind = "reference" if oracle.reference_available() else "port"
    if kind == "port":
        oracle.build()
    results = []
    with tempfile.TemporaryDirectory() as td:
        ids_path = os.path.join(td, "ids.bin")
        np.ascontiguousarray(prompts[:cores, :prefix], np.int32).tofile(ids_path)
        procs = []
        cpus = sorted(os.sched_getaffinity(0)) if hasattr(os, "sched_getaffinity") else list(range(cores))
        for c in range(cores):
            out = os.path.join(td, f"o{c}.bin")
            if kind == "reference":
                cmd = [oracle.REF_BIN, w, inv, cfg, ids_path, "1", str(prefix), str(n_new), out,
                       "--first-seq", str(c)]
            else:
                cmd = [sys.executable, os.path.join(ROOT, "oracle", "port_driver.py"), w, cfg, ids_path,
                       str(c), str(prefix), str(n_new)]
            cpu = cpus[c % len(cpus)]
            procs.append(subprocess.Popen(cmd, stdout=subprocess.PIPE, stderr=subprocess.PIPE, text=True,
                                          preexec_fn=lambda cpu=cpu: os.sched_setaffinity(0, {cpu})))
        for p in procs:
            out, err = p.communicate()
            if p.returncode != 0:
                raise RuntimeError(f"CPU baseline failed: {err.strip()}")
            t = json.loads(out.strip().splitlines()[-1])["seqs"][0]
            results.append((t["prefill_ms"], t["decode_ms"] / max(1, t["decode_steps"])))
    return results, kind


def cpu_rate(results, wl, prefix):
    """Whole-sequence generation rate of the CPU, from its measured per-token
    costs: a prefill of n_prompt tokens costs (n_prompt / prefix) x the measured
    prefix prefill (matmul work is linear in tokens), and each of the n_new - 1
    decode steps the measured mean step (taken at a shorter context, which
    slightly flatters the CPU)."""
    rates = []
    for pre_ms, step_ms in results:
        seq_ms = pre_ms * wl["n_prompt"] / prefix + step_ms * (wl["n_new"] - 1)
        rates.append(wl["n_new"] / (seq_ms / 1e3))
    return sum(rates)


def host_cores():
    try:
        return len(os.sched_getaffinity(0))
    except AttributeError:
        return os.cpu_count() or 1


def run_reference_arm(args, rank, world):
    if rank != 0:
        return 0
    wl = WORKLOADS[args.workload]
    w, inv, cfg = synth.ensure_model(wl["shape"], seed=WEIGHT_SEED)
    V = synth.SHAPES[wl["shape"]].vocab_size
    cores = min(host_cores(), wl["n_seq"], 64)
    prompts = synth.prompt_ids(V, max(cores, 1), wl["n_prompt"], wl["prompt_seed"])
    prefix = min(16, wl["n_prompt"])
    for _ in range(args.warmup):
        cpu_sample(w, inv, cfg, prompts, cores, prefix=4, n_new=2)
    vals, kind = [], None
    t0 = time.perf_counter()
    for _ in range(args.steps):
        res, kind = cpu_sample(w, inv, cfg, prompts, cores, prefix=prefix)
        vals.append(cpu_rate(res, wl, prefix))
    wall = time.perf_counter() - t0
    value = statistics.median(vals)
    seq_s = wl["n_new"] / (value / cores)
    sample = (f"{cores} concurrent sequences (one per core) of the {args.workload} workload: prefill of "
              f"the first {prefix} prompt tokens and {4} cached decode steps, per step; the rate is "
              f"n_new / (prefill x {wl['n_prompt']}/{prefix} + (n_new-1) x mean step)")
    line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
            "warmup": args.warmup, "ms_per_step": seq_s * 1e3, "higher_is_better": True,
            "scaling": "strong", "vs_baseline": None, "dtype": "f32", "data": "synthetic",
            "impl": "reference",
            "config": {"workload": args.workload, **wl, "weights": f"seeded N(0,0.02) seed {WEIGHT_SEED}"},
            "cpu_baseline": {"value": value, "unit": "tokens/s", "cores": cores, "kind": kind, "sample": sample},
            "e2e": {"value": value, "unit": "tokens/s", "h2d_bytes_per_step": 0, "d2h_bytes_per_step": 0},
            "wall_s": round(wall, 1)}
    print(json.dumps(line), flush=True)
    return 0


# ------------------------------------------------------------- our arm --


# DRAM bytes (dram__bytes_read.sum + dram__bytes_write.sum) of one launch of a
# roofline kernel, from one ncu capture of that kernel at exactly the shape the
# workload times it at: (shape, kernel, rows, context) -> bytes
NCU_TRAFFIC = {
    ("small", "decode_attention", 256, 288): 453_929_216 + 9_000_448,
    ("small", "decode_attention", 1, 192): 1_223_424 + 0,
}


def weight_bytes_per_elem(wl):
    return {"f32": 4, "bf16": 2, "int8": 1}[wl.get("fmt", "f32")]


def roofline_of(m, wl, rows, measured, peaks):
    """Per-kernel live timings (CUDA events, each kernel alone at the workload's
    shapes) and the roofline of the dominant one."""
    E, H, L, V = m.n_embd, m.n_head, m.n_layer, m.vocab
    ctx = wl["n_prompt"] + wl["n_new"] // 2            # mean context over the decode horizon
    steps = wl["n_new"] - 1
    hbm = peaks.get("hbm_gbs", 6650.0)
    bf16 = peaks.get("bf16_tflops", 1590.0)
    k = {}

    def add(name, ms, per_step, kind, work):
        if ms is None:
            return
        k[name] = {"ms": ms, "launches_per_gen": per_step}
        if kind == "hbm":
            k[name].update(bound="hbm", achieved=work / (ms * 1e-3) / 1e9, unit="GB/s", peak=hbm)
        else:
            k[name].update(bound="tensor", achieved=work / (ms * 1e-3) / 1e12, unit="TFLOP/s", peak=bf16)
        k[name]["frac"] = k[name]["achieved"] / k[name]["peak"]
        k[name]["share_ms"] = ms * per_step
        k[name]["work_per_launch"] = work

    if steps > 0 and "decode_step" in measured:
        # the persistent step kernel: every weight matrix once, the KV cache of
        # every layer once, per step
        step_bytes = (12 * E * E * L + V * E) * 4 + L * rows * ctx * 2 * E * 4
        add("decode_step", measured.get("decode_step"), steps, "hbm", step_bytes)
    elif steps > 0:
        kv_bytes = rows * ctx * 2 * E * 4 + rows * 2 * E * 4
        add("decode_attention", measured.get("decode_attention"), L * steps, "hbm", kv_bytes)
        for name, N, K in (("decode_qkv", 3 * E, E), ("decode_fc", 4 * E, E), ("decode_mlp_proj", E, 4 * E)):
            ms = measured.get(name)
            if rows <= 8:   # the streaming GEMVs (model.cu kGemvRows)
                add(name, ms, L * steps, "hbm", N * K * weight_bytes_per_elem(wl) + rows * (N + K) * 4)
            else:
                add(name, ms, L * steps, "tensor", 2.0 * rows * N * K)
        if rows <= 8:
            add("decode_head", measured.get("decode_head"), steps, "hbm",
                V * E * weight_bytes_per_elem(wl) + rows * V * 4)
        else:
            add("decode_head", measured.get("decode_head"), steps, "tensor", 2.0 * rows * V * E)
    else:
        T = wl["n_prompt"]
        add("prefill_fc", measured.get("prefill_fc"), L, "tensor", 2.0 * rows * T * 4 * E * E)
        add("prefill_attention", measured.get("prefill_attention"), L, "tensor",
            4.0 * rows * E * T * (T + 1) / 2)
    dom = max(k, key=lambda n: k[n]["share_ms"])
    d = k[dom]
    traffic = NCU_TRAFFIC.get((wl["shape"], dom, rows, ctx if steps > 0 else wl["n_prompt"]))
    roof = {"kernel": dom, "bound": d["bound"], "achieved": d["achieved"], "peak": d["peak"],
            "unit": d["unit"], "frac": d["frac"], "traffic": traffic,
            "peak_source": "measured" if peaks else "fallback",
            "work_per_launch": d["work_per_launch"]}
    return roof, k


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
        paths = synth.ensure_model(wl["shape"], seed=WEIGHT_SEED)
    barrier()
    w, inv, cfg = synth.ensure_model(wl["shape"], seed=WEIGHT_SEED)
    V = synth.SHAPES[wl["shape"]].vocab_size
    start, size = shard_range(wl["n_seq"], rank, world)
    all_prompts = synth.prompt_ids(V, wl["n_seq"], wl["n_prompt"], wl["prompt_seed"])
    prompts = np.ascontiguousarray(all_prompts[start:start + size])
    T, n_new = wl["n_prompt"], wl["n_new"]

    m = tie_b200.Model(w, inv, cfg, device=local_rank)
    fmt = wl.get("fmt", "f32")
    if fmt != "f32":
        m.set_weight_format({"bf16": tie_b200.TIE_WEIGHTS_BF16, "int8": tie_b200.TIE_WEIGHTS_INT8}[fmt])
    m.batch_reserve(size, T + n_new - 1)
    stream = torch.cuda.ExternalStream(m.stream)
    d_prompts = torch.from_numpy(prompts).to("cuda")
    d_out = torch.zeros((size, n_new), dtype=torch.int32, device="cuda")
    torch.cuda.synchronize()

    def step():
        m.generate_greedy_device(d_prompts.data_ptr(), size, T, n_new, d_out.data_ptr())

    for _ in range(args.warmup):
        step()
    torch.cuda.synchronize()

    sampler = ClockSampler(range(world)) if rank == 0 else None
    ev0, ev1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    barrier()
    torch.cuda.synchronize()
    l0 = m.kernel_launches()
    ev0.record(stream)
    for _ in range(args.steps):
        step()
    ev1.record(stream)
    torch.cuda.synchronize()
    barrier()
    launches = (m.kernel_launches() - l0) // args.steps
    clocks = sampler.stop() if sampler else None
    ms = max_over_ranks(ev0.elapsed_time(ev1) / args.steps)
    # tokens a step produces: the generated ones, or for a prefill-only workload
    # (one new token) the prompt tokens it processes
    gen_tokens = wl["n_seq"] * (n_new if n_new > 1 else T)
    value = gen_tokens / (ms / 1e3)

    # the same generation through the public host API: pinned prompts in, ids out
    h_prompts = torch.from_numpy(prompts).pin_memory()
    h_out = torch.zeros((size, n_new), dtype=torch.int32).pin_memory()
    import ctypes as C
    L = tie_b200.library()

    def e2e_step():
        rc = L.model_generate_greedy(m.h, C.cast(h_prompts.data_ptr(), C.POINTER(C.c_int32)), size, T,
                                     n_new, C.cast(h_out.data_ptr(), C.POINTER(C.c_int32)))
        if rc != 0:
            raise tie_b200.ModelError(rc, "model_generate_greedy")

    e2e_step()
    barrier()
    t0 = time.perf_counter()
    for _ in range(args.steps):
        e2e_step()
    e2e_ms = max_over_ranks((time.perf_counter() - t0) * 1e3 / args.steps)
    assert np.array_equal(h_out.numpy(), d_out.cpu().numpy()), "host and device paths disagree"

    # prefill alone (batch prefill through the public API, device-timed)
    pre_ms = None
    if n_new > 1:
        evp0, evp1 = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        m.prefill_batch(prompts)
        evp0.record(stream)
        for _ in range(3):
            m.prefill_batch(prompts)
        evp1.record(stream)
        torch.cuda.synchronize()
        pre_ms = max_over_ranks(evp0.elapsed_time(evp1) / 3)

    # per-kernel live timings at this rank's shapes
    measured = {}
    ctx = T + n_new // 2
    if n_new > 1:
        names = ["decode_attention", "decode_qkv", "decode_fc", "decode_mlp_proj", "decode_head"]
    else:
        names = ["prefill_fc", "prefill_attention"]
    for name in names:
        measured[name] = m.time_kernel(name, size, ctx if name.startswith("decode") else T, iters=20)
    peaks = {}
    try:
        peaks = json.load(open(os.path.join(ROOT, "MEASURED_PEAKS.json")))
    except (OSError, ValueError):
        pass
    roof, kernels = roofline_of(m, wl, size, measured, peaks)

    line = None
    if rank == 0:
        line = {"metric": METRIC, "value": value, "unit": "tokens/s", "n_gpus": world, "steps": args.steps,
                "warmup": args.warmup, "ms_per_step": ms, "higher_is_better": True, "scaling": "strong",
                "vs_baseline": None,
                "dtype": "f32" if fmt == "f32" else f"{fmt} weights, f32 accumulate",
                "data": "synthetic (seeded random-init weights, seeded uniform token ids)",
                "config": {"workload": args.workload, "model": f"gpt2-{wl['shape']}", "n_seq": wl["n_seq"],
                           "n_prompt": T, "n_new": n_new, "seq_per_gpu": size,
                           "parallelism": f"batch-sharded x{world}, no collective",
                           "l2": "inputs larger than L2 (weights 0.5 GB, KV cache GBs)",
                           "step": "one greedy generation over the batch: prefill + (n_new - 1) decode steps"},
                "e2e": {"value": gen_tokens / (e2e_ms / 1e3), "unit": "tokens/s",
                        "h2d_bytes_per_step": int(prompts.nbytes), "d2h_bytes_per_step": int(size * n_new * 4),
                        "ms_per_step": e2e_ms},
                "gpu_launches": int(launches),
                "clocks": clocks,
                "roofline": roof,
                "kernels": kernels}
        if pre_ms is not None:
            line["phases"] = {"prefill_ms": pre_ms, "prefill_tokens_per_s": wl["n_seq"] * T / (pre_ms / 1e3),
                              "decode_ms": ms - pre_ms,
                              "decode_tokens_per_s": wl["n_seq"] * (n_new - 1) / ((ms - pre_ms) / 1e3)}
    barrier()
    m.close()
    if world > 1:
        dist.destroy_process_group()
    if rank == 0 and world == 1 and not args.no_cpu_baseline:
        cores = min(host_cores(), 32)
        prefix = min(16, T)
        res, kind = cpu_sample(w, inv, cfg, all_prompts, cores, prefix=prefix)
        line["cpu_baseline"] = {
            "value": cpu_rate(res, wl, prefix), "unit": "tokens/s", "cores": cores, "kind": kind,
            "sample": f"{cores} concurrent sequences, one per core: prefill of {prefix} prompt tokens and 4 "
                      f"cached decode steps each; rate = n_new / (prefill x {T}/{prefix} + "
                      f"(n_new-1) x mean step)",
            "prefill_ms_per_token": statistics.mean(r[0] for r in res) / prefix,
            "decode_ms_per_step": statistics.mean(r[1] for r in res)}
    if rank == 0:
        print(json.dumps(line), flush=True)
    return 0


def run_kernel(args):
    """One kernel of a GPT-2 forward pass, alone, at (rows, context)."""
    import tie_b200
    w, inv, cfg = synth.ensure_model(args.shape, seed=WEIGHT_SEED)
    m = tie_b200.Model(w, inv, cfg, device=0)
    if args.fmt != "f32":
        m.set_weight_format({"bf16": tie_b200.TIE_WEIGHTS_BF16, "int8": tie_b200.TIE_WEIGHTS_INT8}[args.fmt])
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
