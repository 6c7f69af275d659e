"""CLI around the C restatement (liboracle.so) with ref_gpt2's timing output.

TEST / BASELINE INFRASTRUCTURE ONLY: used by bench.py's CPU-baseline leg when
the reference binary (oracle/_ref/ref_gpt2) is not available.

    python port_driver.py WEIGHTS CONFIG IDS.bin SEQ N_PROMPT N_NEW [CONTEXTS ROUNDS]

Without CONTEXTS it times a greedy generation of N_NEW tokens; with CONTEXTS
(comma-separated) it times the prompt's prefill once and then, ROUNDS times
over, one cached decode step at each context, as ref_gpt2 --time-contexts does.
"""
import json
import os
import sys
import time

import numpy as np

sys.path.insert(0, os.path.dirname(os.path.abspath(__file__)))
import oracle  # noqa: E402


def main(argv):
    weights, config, ids_path, seq, n_prompt, n_new = argv[1], argv[2], argv[3], int(argv[4]), int(argv[5]), int(argv[6])
    prompts = np.fromfile(ids_path, dtype=np.int32).reshape(-1, n_prompt)
    o = oracle.Oracle(weights, config, kv_capacity=n_prompt + n_new)
    ids = list(prompts[seq])
    t0 = time.perf_counter()
    row = o.prefill(ids, write_cache=True)[-1]
    pre = (time.perf_counter() - t0) * 1e3
    if len(argv) > 7:
        contexts = [int(c) for c in argv[7].split(",")]
        rounds = int(argv[8]) if len(argv) > 8 else 1
        fill = int(np.argmax(row))
        full = ids + [fill] * (n_prompt + n_new - len(ids))
        out = []
        for _ in range(rounds):
            r = []
            for c in contexts:
                o.kv_set_length(c - 1)
                t0 = time.perf_counter()
                o.decode_cached(full[:c])
                r.append((time.perf_counter() - t0) * 1e3)
            out.append(r)
        print(json.dumps({"mode": "sampled", "n_prompt": n_prompt, "prefill_ms": pre, "contexts": contexts,
                          "rounds": out}))
        return 0
    dec = 0.0
    for _ in range(n_new - 1):
        ids.append(int(np.argmax(row)))
        t0 = time.perf_counter()
        row = o.decode_cached(ids)
        dec += (time.perf_counter() - t0) * 1e3
    print(json.dumps({"seqs": [{"prefill_ms": pre, "decode_ms": dec, "decode_steps": n_new - 1}]}))
    return 0


if __name__ == "__main__":
    sys.exit(main(sys.argv))
