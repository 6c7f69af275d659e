"""The CPU oracle (oracle/gpt2_oracle.c) pinned against the reference itself.

The golden vectors under tests/golden/ were produced by the reference's own C
engine compiled unmodified (tests/golden/make_golden.py); the restatement must
reproduce them BIT FOR BIT, because it performs the same float operations in the
same order.  Where the reference binary is present (oracle/_ref) it is also run
live against the restatement.
"""
import os
import struct

import numpy as np
import pytest

import oracle
from conftest import golden


def bits(a):
    return np.ascontiguousarray(a, dtype=np.float32).view(np.uint32)


# ---------------------------------------------------------------- tiny golden --

def test_tiny_prefill_logits_bit_exact(tiny_paths):
    g, meta = golden("tiny")
    w, inv, cfg = tiny_paths
    o = oracle.Oracle(w, cfg)
    for s in range(g["prompts"].shape[0]):
        got = o.prefill(g["prompts"][s])
        assert np.array_equal(bits(got), bits(g["prefill_logits"][s]))


def test_tiny_greedy_and_step_logits_bit_exact(tiny_paths):
    g, meta = golden("tiny")
    w, inv, cfg = tiny_paths
    n_new = meta["spec"]["n_new"]
    for s in range(g["prompts"].shape[0]):
        o = oracle.Oracle(w, cfg)
        ids, t1, t2 = o.greedy(g["prompts"][s], n_new)
        assert np.array_equal(ids, g["ids"][s])
        assert np.array_equal(bits(t1), bits(g["topk_vals"][s][:, 0]))
        assert np.array_equal(bits(t2), bits(g["topk_vals"][s][:, 1]))
        # the step logits through the cached path, one step at a time
        o2 = oracle.Oracle(w, cfg)
        seq = list(g["prompts"][s])
        o2.prefill(seq, write_cache=True)
        seq.append(int(g["ids"][s][0]))
        for k in range(n_new - 1):
            row = o2.decode_cached(seq)
            assert np.array_equal(bits(row), bits(g["step_logits"][s][k])), k
            seq.append(int(g["ids"][s][k + 1]))


def test_tiny_transposed_reading_bit_exact(tiny_paths):
    g, _ = golden("tiny")
    w, inv, cfg = tiny_paths
    o = oracle.Oracle(w, cfg, cproj_transposed=True)
    got = o.prefill(g["prompts"][0])
    assert np.array_equal(bits(got), bits(g["transposed_prefill_logits"][0]))
    assert not np.array_equal(got, g["prefill_logits"][0]), "the two c_proj readings must differ"


def test_tiny_torch_oracle_agrees(tiny_paths):
    g, _ = golden("tiny")
    if "torch_prefill_logits" not in g:
        pytest.skip("torch oracle not recorded")
    w, inv, cfg = tiny_paths
    got = oracle.Oracle(w, cfg).prefill(g["prompts"][0])
    # an independent implementation (torch, fused ops): agreement to float rounding
    assert np.abs(got - g["torch_prefill_logits"][0]).max() < 1e-5


# ---------------------------------------------------------------- mini golden --

def test_mini_bit_exact(mini_paths):
    g, meta = golden("mini")
    w, inv, cfg = mini_paths
    for s in range(g["prompts"].shape[0]):
        o = oracle.Oracle(w, cfg)
        ids, t1, t2 = o.greedy(g["prompts"][s], meta["spec"]["n_new"])
        assert np.array_equal(ids, g["ids"][s])
        assert np.array_equal(bits(t1), bits(g["topk_vals"][s][:, 0]))
        last = oracle.Oracle(w, cfg).prefill(g["prompts"][s])[-1]
        assert np.array_equal(bits(last), bits(g["prefill_logits"][s][0]))
        # top-k at every prefill position
        full = oracle.Oracle(w, cfg).prefill(g["prompts"][s])
        k = g["prefill_topk_ids"].shape[-1]
        for t in range(full.shape[0]):
            order = np.lexsort((np.arange(full.shape[1]), -full[t]))[:k]
            assert np.array_equal(order, g["prefill_topk_ids"][s][t])


# ------------------------------------------------------ GPT-2 small, config 1 --

def test_small_c1_prefix_bit_exact(small_paths):
    """GPT-2 small, the 128-token prompt: the prefill's last row and the first
    greedy steps reproduce the reference bit for bit (about 40 s of CPU)."""
    g, meta = golden("small_c1")
    w, inv, cfg = small_paths
    o = oracle.Oracle(w, cfg, kv_capacity=160)
    prompt = g["prompts"][0]
    seq = list(prompt)
    row = o.prefill(seq, write_cache=True)[-1]
    assert np.array_equal(bits(row), bits(g["prefill_logits"][0][0]))
    assert int(np.argmax(row)) == int(g["ids"][0][0])
    for k in range(1, 4):
        seq.append(int(g["ids"][0][k - 1]))
        row = o.decode_cached(seq)
        top = np.lexsort((np.arange(row.size), -row))[:16]
        assert np.array_equal(top, g["topk_ids"][0][k])
        assert np.array_equal(bits(row[top]), bits(g["topk_vals"][0][k]))


# ------------------------------------------------ live against the reference --

@pytest.mark.skipif(not oracle.reference_available(), reason="oracle/_ref not built")
@pytest.mark.parametrize("transposed", [False, True])
def test_restatement_equals_reference_binary(tiny_paths, transposed):
    from tie_b200 import synth
    w, inv, cfg = tiny_paths
    prompts = synth.prompt_ids(500, 3, 12, seed=11)
    seqs, _ = oracle.run_reference(w, inv, cfg, prompts, 10, prefill_logits="all",
                                   step_logits=True, cproj_transposed=transposed)
    for s, ref in enumerate(seqs):
        o = oracle.Oracle(w, cfg, cproj_transposed=transposed)
        assert np.array_equal(bits(o.prefill(prompts[s])), bits(ref["prefill_logits"]))
        ids, _, _ = oracle.Oracle(w, cfg, cproj_transposed=transposed).greedy(prompts[s], 10)
        assert np.array_equal(ids, ref["ids"])


@pytest.mark.skipif(not oracle.reference_available(), reason="oracle/_ref not built")
def test_nocache_path_equals_cached_in_reference(tiny_paths):
    """The reference's own bit-identity of its two decode paths (test_model.c:284-316),
    observed through the binary, and the restatement's no-cache step matching it."""
    from tie_b200 import synth
    w, inv, cfg = tiny_paths
    prompts = synth.prompt_ids(500, 1, 6, seed=12)
    a, _ = oracle.run_reference(w, inv, cfg, prompts, 8, step_logits=True)
    b, _ = oracle.run_reference(w, inv, cfg, prompts, 8, step_logits=True, nocache=True)
    assert np.array_equal(a[0]["ids"], b[0]["ids"])
    assert np.array_equal(bits(a[0]["step_logits"]), bits(b[0]["step_logits"]))
    o = oracle.Oracle(w, cfg)
    seq = list(prompts[0]) + [int(a[0]["ids"][0])]
    assert np.array_equal(bits(o.decode_nocache(seq)), bits(a[0]["step_logits"][0]))


# ------------------------------------------------------ the unit-level pieces --

def test_naive_gemm_hand_values():
    """reference tests/test_gemm_naive.c:71-93"""
    A = np.array([[1, 2, 3], [4, 5, 6]], np.float32)
    B = np.array([[7, 8], [9, 10], [11, 12]], np.float32)
    assert oracle.gemm_naive(A, B).tolist() == [[58, 64], [139, 154]]
    assert oracle.gemm_naive_bt(A, B.T.copy()).tolist() == [[58, 64], [139, 154]]


def test_naive_gemm_identity_and_empty_sum():
    rng = np.random.default_rng(0)
    A = rng.standard_normal((7, 7)).astype(np.float32)
    I = np.eye(7, dtype=np.float32)
    assert np.array_equal(oracle.gemm_naive(A, I), A)
    assert np.array_equal(oracle.gemm_naive(I, A), A)
    assert np.array_equal(oracle.gemm_naive(np.zeros((2, 0), np.float32), np.zeros((0, 3), np.float32)),
                          np.zeros((2, 3), np.float32))


def lcg_row(n=768, seed=11):
    """the input of reference tests/test_model.c:80-99"""
    s, out = seed, np.empty(n, np.float32)
    for i in range(n):
        s = (s * 1664525 + 1013904223) & 0xFFFFFFFF
        out[i] = np.float32((s >> 8) / 8388608.0 - 1.0) * np.float32(7.0) + np.float32(3.0)
    return out


def test_layernorm_normalize_moments():
    y = oracle.layernorm_normalize(lcg_row(), 1e-5).astype(np.float64)
    assert abs(y.mean()) < 1e-5
    assert abs(y.var() - 1.0) < 1e-4


def test_argmax_rules():
    assert oracle.argmax(np.array([1, 3, 3, 2], np.float32)) == 1
    assert oracle.argmax(np.array([np.nan, 3, 4], np.float32)) == 0
    assert oracle.argmax(np.array([1, np.nan, 4, 4], np.float32)) == 2
