"""Generates the golden fixtures under tests/golden/ from the REFERENCE itself.

Every fixture is produced by running the reference's own C engine, compiled
unmodified from its source tree (oracle/_ref/ref_gpt2, built by `make -C oracle
ref`), on seeded random-init weights (tie_b200.synth) and seeded token ids.  The
tiny fixture additionally records the reference's PyTorch oracle
(reference/reference_impl.py, imported read-only from the reference checkout)
as a second, independent opinion.

Only small arrays are committed: greedy ids, the top-k logits (ids and values)
of the row each token was chosen from, top-k at prefill positions, and a few
full logit rows.  Weights are not committed; they are regenerated bit-for-bit
from (shape, seed, LayerNorm init) by tie_b200.synth.ensure_model.

    python tests/golden/make_golden.py tiny mini small_c1 small_c2 medium_c3 xl_c4 small_c5
"""
from __future__ import annotations

import argparse
import json
import os
import sys
import time
from concurrent.futures import ThreadPoolExecutor

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, os.path.join(ROOT, "transformer-inference-engine_b200"))
sys.path.insert(0, os.path.join(ROOT, "oracle"))

from tie_b200 import synth  # noqa: E402
import oracle  # noqa: E402

# fixture name -> (shape, weight seed, LN init, prompt seed, n_seq, n_prompt, n_new, topk, extras)
FIXTURES = {
    "tiny":      ("tiny", 7, "random", 3, 2, 8, 16, 4, {"prefill_logits": "all", "step_logits": True}),
    "mini":      ("mini", 7, "random", 5, 4, 100, 64, 8, {"prefill_logits": "last", "prefill_topk": True}),
    "small_c1":  ("small", 1234, "unit", 101, 1, 128, 128, 16, {"prefill_logits": "last", "prefill_topk": True}),
    "small_c2":  ("small", 1234, "unit", 102, 8, 1024, 1, 8, {"prefill_topk": True}),
    "medium_c3": ("medium", 1234, "unit", 103, 8, 512, 256, 8, {}),
    "xl_c4":     ("xl", 1234, "unit", 104, 1, 896, 128, 8, {}),
    "small_c5":  ("small", 1234, "unit", 105, 256, 64, 448, 4, {}),
}


def spec(name: str) -> dict:
    shape, wseed, ln, pseed, n_seq, n_prompt, n_new, topk, extras = FIXTURES[name]
    return dict(shape=shape, weight_seed=wseed, ln_affine=ln, prompt_seed=pseed, n_seq=n_seq,
                n_prompt=n_prompt, n_new=n_new, topk=topk, **extras)


def prompts_for(name: str) -> np.ndarray:
    s = spec(name)
    V = synth.SHAPES[s["shape"]].vocab_size
    return synth.prompt_ids(V, s["n_seq"], s["n_prompt"], s["prompt_seed"])


def _save(name: str, s: dict, prompts: np.ndarray, results: list, t0: float, extra: dict) -> None:
    n_seq = len(results)
    out = {"prompts": prompts[:n_seq],
           "ids": np.stack([r[0]["ids"] for r in results]),
           "topk_ids": np.stack([r[0]["topk_ids"] for r in results]),
           "topk_vals": np.stack([r[0]["topk_vals"] for r in results])}
    for key in ("prefill_topk_ids", "prefill_topk_vals", "prefill_logits", "step_logits"):
        if key in results[0][0]:
            out[key] = np.stack([r[0][key] for r in results])
    out.update(extra)
    np.savez_compressed(os.path.join(HERE, f"{name}.npz"), **out)
    meta = dict(spec=s, n_seq_recorded=n_seq, seconds=round(time.time() - t0, 1),
                cpu_timing=[r[1] for r in results],
                producer="oracle/_ref/ref_gpt2 (reference src/model.c, kv_cache.c, gemm_naive.c, "
                         "safetensors.c compiled unmodified with -O3 -mavx2 -mfma -std=gnu11 "
                         "-ffp-contract=off)")
    with open(os.path.join(HERE, f"{name}.json"), "w") as f:
        json.dump(meta, f, indent=1)


def _load_existing(name: str):
    """The sequences an earlier run recorded, as (seq dict, timing) pairs."""
    npz, meta = os.path.join(HERE, f"{name}.npz"), os.path.join(HERE, f"{name}.json")
    if not (os.path.isfile(npz) and os.path.isfile(meta)):
        return []
    g = np.load(npz)
    with open(meta) as f:
        timing = json.load(f)["cpu_timing"]
    keys = [k for k in ("ids", "topk_ids", "topk_vals", "prefill_topk_ids", "prefill_topk_vals",
                        "prefill_logits", "step_logits") if k in g.files]
    return [({k: g[k][i] for k in keys}, timing[i]) for i in range(g["ids"].shape[0])]


def make(name: str, workers: int, n_seq_limit: int | None = None, resume: bool = False) -> None:
    """Runs the reference on every sequence of fixture `name`.  With `resume`,
    the sequences already in the fixture are kept and only the rest are run;
    the fixture is rewritten after every chunk of sequences, so an interrupted
    run loses at most one chunk."""
    s = spec(name)
    w, inv, cfg = synth.ensure_model(s["shape"], seed=s["weight_seed"], ln_affine=s["ln_affine"])
    prompts = prompts_for(name)
    n_seq = min(s["n_seq"], n_seq_limit or s["n_seq"])
    kw = dict(prefill_logits=s.get("prefill_logits", "none"), step_logits=s.get("step_logits", False),
              topk=s["topk"], prefill_topk=s.get("prefill_topk", False))
    t0 = time.time()

    def one(i):
        seqs, timing = oracle.run_reference(w, inv, cfg, prompts, s["n_new"], first_seq=i, n_seq=1, **kw)
        return seqs[0], timing["seqs"][0]

    results = _load_existing(name) if resume else []
    if resume and results:
        recorded = np.load(os.path.join(HERE, f"{name}.npz"))["prompts"]
        if not np.array_equal(recorded, prompts[:len(results)]):
            raise SystemExit(f"{name}: the recorded prompts differ from the fixture's seed; not resuming")
    extra = {}
    if name == "tiny":
        t_seqs, _ = oracle.run_reference(w, inv, cfg, prompts, s["n_new"], n_seq=1, first_seq=0,
                                         prefill_logits="all", cproj_transposed=True, topk=s["topk"])
        extra["transposed_prefill_logits"] = t_seqs[0]["prefill_logits"][None]
        extra["transposed_ids"] = t_seqs[0]["ids"][None]
        torch_logits = torch_oracle(w, inv, cfg, prompts[0])
        if torch_logits is not None:
            extra["torch_prefill_logits"] = torch_logits[None]
    chunk = max(1, workers) * 2
    with ThreadPoolExecutor(max_workers=workers) as ex:
        while len(results) < n_seq:
            lo = len(results)
            hi = min(n_seq, lo + chunk)
            results += list(ex.map(one, range(lo, hi)))
            _save(name, s, prompts, results, t0, extra)
            print(f"{name}: {len(results)}/{n_seq} sequences, {time.time() - t0:.1f} s", flush=True)
    if not results:
        return
    _save(name, s, prompts, results, t0, extra)
    print(f"{name}: {n_seq} sequences in {time.time() - t0:.1f} s", flush=True)


def torch_oracle(w, inv, cfg, ids):
    """The reference's PyTorch oracle on the same weights, if importable here."""
    ref_dir = os.environ.get("TIE_REFERENCE_ROOT")
    if not ref_dir:
        return None
    path = os.path.join(ref_dir, "reference")
    if not os.path.isfile(os.path.join(path, "reference_impl.py")):
        return None
    sys.path.insert(0, path)
    try:
        import reference_impl  # type: ignore
        m = reference_impl.ReferenceGPT2(weights=w, config=cfg, inventory=inv)
        return m.forward([int(i) for i in ids]).numpy().astype(np.float32)
    finally:
        sys.path.remove(path)


def main(argv=None):
    p = argparse.ArgumentParser()
    p.add_argument("names", nargs="+", choices=sorted(FIXTURES))
    p.add_argument("--workers", type=int, default=max(1, (os.cpu_count() or 2) - 2))
    p.add_argument("--n-seq", type=int, default=None, help="record only the first N sequences")
    p.add_argument("--resume", action="store_true",
                   help="keep the sequences already recorded and run only the rest")
    a = p.parse_args(argv)
    if not oracle.reference_available():
        oracle.build()
    for n in a.names:
        make(n, a.workers, a.n_seq, a.resume)


if __name__ == "__main__":
    main()
