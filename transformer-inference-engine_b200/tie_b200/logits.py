"""Logit dumps and the divergence report between two of them.

The dump is the reference engine's binary block (src/main.c:262-271,
written by `gpt2_tool --dump-logits`): the 8-byte magic "TIE2LOGI", int32
positions, int32 vocabulary size (little-endian), then positions x vocab
float32 logits in row order. A dump written here can be read by the
reference's harness (bench/correctness.py:264-275) and the other way round.

`divergence_statistics` describes how far one logit matrix is from another
with the statistic set of the reference's correctness report
(bench/correctness.py:287-364): absolute and relative differences (relative to
|reference| + 1e-6) with their maxima, mean, median, RMS and percentiles; top-1
and top-5-set agreement per position; and the reference's top-1/top-2 margin
per position, the divergence greedy decoding can absorb before a token flips.
It applies no threshold. `python -m tie_b200.logits` compares two dumps and
prints the report as JSON.
"""
from __future__ import annotations

import json
import struct
import sys

import numpy as np

MAGIC = b"TIE2LOGI"
REL_EPS = 1e-6   # floor added to |reference| in the relative difference


def write_logit_dump(path: str, logits) -> None:
    """Writes a [positions, vocab] float32 matrix as a TIE2LOGI dump."""
    a = np.ascontiguousarray(logits, dtype=np.float32)
    if a.ndim != 2:
        raise ValueError(f"expected [positions, vocab]; got shape {a.shape}")
    with open(path, "wb") as f:
        f.write(MAGIC)
        f.write(struct.pack("<ii", a.shape[0], a.shape[1]))
        f.write(a.astype("<f4", copy=False).tobytes())


def read_logit_dump(path: str) -> np.ndarray:
    """Reads a TIE2LOGI dump into a [positions, vocab] float32 array."""
    with open(path, "rb") as f:
        magic = f.read(8)
        if magic != MAGIC:
            raise ValueError(f"{path}: not a logit dump (magic {magic!r})")
        head = f.read(8)
        if len(head) != 8:
            raise ValueError(f"{path}: truncated header")
        npos, nvocab = struct.unpack("<ii", head)
        if npos < 0 or nvocab <= 0:
            raise ValueError(f"{path}: bad shape {npos} x {nvocab}")
        want = npos * nvocab * 4
        raw = f.read(want)
    if len(raw) != want:
        raise ValueError(f"{path}: {len(raw)} bytes of logits for {npos} x {nvocab}")
    return np.frombuffer(raw, dtype="<f4").reshape(npos, nvocab).astype(np.float32)


def _percentiles(a: np.ndarray) -> dict:
    p50, p90, p99, p999 = np.percentile(a, [50, 90, 99, 99.9])
    return {"p50": float(p50), "p90": float(p90), "p99": float(p99), "p99_9": float(p999),
            "max": float(a.max())}


def _top5(row: np.ndarray) -> set:
    return set(np.argpartition(-row, 5)[:5].tolist())


def divergence_statistics(engine, reference, token_ids=None, label: str = "") -> dict:
    """How far `engine` logits are from `reference` logits ([positions, vocab],
    compared in float32 at every position over the whole vocabulary)."""
    e = np.asarray(engine, dtype=np.float32)
    r = np.asarray(reference, dtype=np.float32)
    if e.shape != r.shape:
        raise ValueError(f"shape mismatch: {e.shape} vs {r.shape}")
    if e.ndim != 2 or e.shape[0] == 0:
        raise ValueError(f"expected a non-empty [positions, vocab]; got {e.shape}")
    diff = np.abs(e - r).astype(np.float64)
    rel = diff / (np.abs(r).astype(np.float64) + REL_EPS)
    worst = int(np.argmax(diff))
    worst_pos, worst_tok = divmod(worst, e.shape[1])

    top1_e, top1_r = np.argmax(e, axis=1), np.argmax(r, axis=1)
    top1_same = top1_e == top1_r
    top5_same = np.array([_top5(e[t]) == _top5(r[t]) for t in range(e.shape[0])])

    ranked = np.sort(r, axis=1)
    margin = (ranked[:, -1] - ranked[:, -2]).astype(np.float64)
    n = e.shape[0]
    out = {
        "label": label,
        "positions": n,
        "vocab_size": int(e.shape[1]),
        "max_abs_diff": float(diff.max()),
        "max_abs_diff_position": int(worst_pos),
        "max_abs_diff_token_id": int(worst_tok),
        "max_rel_diff": float(rel.max()),
        "rel_diff_denominator": f"|reference| + {REL_EPS:g}, elementwise",
        "elements_below_rel_floor": int(np.count_nonzero(np.abs(r) < REL_EPS)),
        "mean_abs_diff": float(diff.mean()),
        "median_abs_diff": float(np.median(diff)),
        "rms_abs_diff": float(np.sqrt(np.mean(diff * diff))),
        "abs_diff_percentiles": _percentiles(diff),
        "rel_diff_percentiles": _percentiles(rel),
        "top1_agreement_positions": int(np.count_nonzero(top1_same)),
        "top1_agreement_fraction": float(np.count_nonzero(top1_same)) / n,
        "top1_disagreeing_positions": [int(t) for t in np.flatnonzero(~top1_same)],
        "top5_set_agreement_positions": int(np.count_nonzero(top5_same)),
        "top5_set_agreement_fraction": float(np.count_nonzero(top5_same)) / n,
        "top5_disagreeing_positions": [int(t) for t in np.flatnonzero(~top5_same)],
        "reference_top1_top2_margin": {
            "min": float(margin.min()),
            "median": float(np.median(margin)),
            "max": float(margin.max()),
            "argmin_position": int(np.argmin(margin)),
            "per_position": [float(x) for x in margin],
        },
        "margin_min_over_max_abs_diff": float(margin.min() / diff.max()) if diff.max() > 0 else None,
    }
    if token_ids is not None:
        out["token_ids"] = [int(i) for i in token_ids]
    return out


def main(argv=None) -> int:
    argv = list(sys.argv[1:] if argv is None else argv)
    if len(argv) not in (2, 3):
        print("usage: python -m tie_b200.logits ENGINE_DUMP REFERENCE_DUMP [LABEL]", file=sys.stderr)
        return 2
    stats = divergence_statistics(read_logit_dump(argv[0]), read_logit_dump(argv[1]),
                                  label=argv[2] if len(argv) == 3 else "")
    print(json.dumps(stats))
    return 0


if __name__ == "__main__":
    sys.exit(main())
