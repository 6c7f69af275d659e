"""The reference's structural model checks (tests/test_model.c), re-targeted at the
B200 engine through its C ABI, at the same reduced token counts (7 tokens).

Checks that are bit-exact in the reference stay bit-exact here when both sides
run the same kernels (causality, decode vs prefill on the no-cache path,
restoration repeatability, causality through the cache). The cached step runs
the decode GEMV while prefill runs the tiled GEMM: the two sum in different
orders, so cached-vs-prefill and cached-vs-no-cache agree to a stated tolerance
(max-abs 1e-4, same argmax at every position) instead of bit for bit.
"""
import numpy as np
import pytest

import oracle
import tie_b200
from tie_b200 import lib as tl
from tie_b200 import synth

pytestmark = pytest.mark.gpu
T = 7
TOL = 1e-4


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


def S(name):
    return tl.MODEL_STATUS.index(name)


@pytest.fixture(scope="module")
def m(mini_paths):
    w, inv, cfg = mini_paths
    mod = tie_b200.Model(w, inv, cfg)
    yield mod
    mod.close()


@pytest.fixture(scope="module")
def ids(m):
    return synth.prompt_ids(m.vocab, 1, T, seed=77)[0]


def test_config_and_tie(m):
    assert m.n_embd == m.n_head * m.head_dim
    assert m.head_weight_ptr() == m.token_embedding_ptr() and m.head_weight_ptr()
    assert m.gemm_name() == "tie_b200_sm100a"
    assert m.decode_path() == tie_b200.MODEL_PATH_NOCACHE


def test_prefill_matches_oracle(m, ids, mini_paths):
    w, inv, cfg = mini_paths
    got = m.prefill(ids)
    ref = oracle.Oracle(w, cfg).prefill(ids)
    assert np.abs(got - ref).max() <= 1e-3
    assert np.array_equal(got.argmax(1), ref.argmax(1))


def test_attention_rows_sum_to_one(m, ids):
    m.collect_attn_stats(True)
    m.prefill(ids)
    lo, hi, rows = m.attn_rowsum_range()
    m.collect_attn_stats(False)
    assert rows == m.n_layer * m.n_head * T
    assert 1 - 1e-5 < lo <= hi < 1 + 1e-5


def test_causality_bit_exact(m, ids):
    a = m.prefill(ids)
    alt = ids.copy()
    alt[T - 1] = (alt[T - 1] + 1234) % m.vocab
    b = m.prefill(alt)
    assert np.array_equal(bits(a[:T - 1]), bits(b[:T - 1]))
    assert not np.array_equal(a[T - 1], b[T - 1])


def test_nocache_decode_reproduces_prefill_bit_exact(m, ids):
    full = m.prefill(ids)
    for t in range(3, T):
        one = m.decode_step(ids[:t + 1])
        assert np.array_equal(bits(one), bits(full[t])), t


def test_cache_lifecycle_and_paths(mini_paths, ids):
    w, inv, cfg = mini_paths
    with tie_b200.Model(w, inv, cfg) as m:
        assert m.kv_footprint() == 0 and not m.kv_cache()
        assert m.kv_reserve(T + 2) == 0
        assert m.kv_footprint() == m.n_layer * 2 * (T + 2) * m.n_embd * 4
        assert m.kv_capacity() == T + 2
        full = m.prefill(ids)

        # CHECK 3 + 10: one-token prefill then one cached step per position
        m.set_decode_path(tie_b200.MODEL_PATH_CACHE)
        m.collect_attn_stats(True)
        cached = np.empty_like(full)
        cached[0] = m.prefill(ids[:1])[0]
        assert m.kv_length() == 1
        for t in range(1, T):
            cached[t] = m.decode_step_cached(ids[:t + 1])
        assert m.kv_length() == T
        lo, hi, rows = m.attn_rowsum_range()
        m.collect_attn_stats(False)
        assert rows == m.n_layer * m.n_head * T
        assert 1 - 1e-5 < lo <= hi < 1 + 1e-5
        assert np.abs(cached - full).max() <= TOL
        assert np.array_equal(cached.argmax(1), full.argmax(1))
        # the one-token cache-mode prefill is the no-cache prefill's row 0, exactly
        assert np.array_equal(bits(cached[0]), bits(full[0]))

        # CHECK 4: cached step vs no-cache step at the same context
        for ctx in range(3, T + 1):
            m.set_decode_path(tie_b200.MODEL_PATH_NOCACHE)
            nc = m.decode_step(ids[:ctx])
            m.set_decode_path(tie_b200.MODEL_PATH_CACHE)
            assert m.kv_set_length(ctx - 1) == 0
            c = m.decode_step_cached(ids[:ctx])
            assert np.abs(c - nc).max() <= TOL and c.argmax() == nc.argmax()

        # CHECK 7: a step, a restoration and the same step again
        m.prefill(ids[:T - 1])
        snap = [(m.kv_layer_to_host(l, 0, T - 1), m.kv_layer_to_host(l, 1, T - 1))
                for l in range(m.n_layer)]
        a = m.decode_step_cached(ids)
        assert m.kv_set_length(T - 1) == 0
        b = m.decode_step_cached(ids)
        assert np.array_equal(bits(a), bits(b))
        for l in range(m.n_layer):
            assert np.array_equal(bits(snap[l][0]), bits(m.kv_layer_to_host(l, 0, T - 1)))
            assert np.array_equal(bits(snap[l][1]), bits(m.kv_layer_to_host(l, 1, T - 1)))
        # the greedy-only step returns the argmax of the same logits
        assert m.kv_set_length(T - 1) == 0
        assert m.decode_step_greedy(ids) == int(a.argmax())

        # CHECK 5: causality through the cached path
        alt = ids.copy()
        alt[T - 1] = (alt[T - 1] + 1234) % m.vocab

        def assemble(seq):
            out = np.empty((T, m.vocab), np.float32)
            out[0] = m.prefill(seq[:1])[0]
            for t in range(1, T):
                out[t] = m.decode_step_cached(seq[:t + 1])
            return out
        x, y = assemble(ids), assemble(alt)
        assert np.array_equal(bits(x[:T - 1]), bits(y[:T - 1]))
        assert not np.array_equal(x[T - 1], y[T - 1])


def test_capacity_refusals(mini_paths, ids):
    """reference tests/test_model.c:411-453 (CHECK 8)"""
    w, inv, cfg = mini_paths
    with tie_b200.Model(w, inv, cfg) as s:
        s.set_decode_path(tie_b200.MODEL_PATH_CACHE)
        s.reserve(8)
        assert s.decode_step_cached(ids[:2], check=False)[0] == S("MODEL_ERR_ARG")
        assert s.prefill(ids[:2], check=False)[0] == S("MODEL_ERR_ARG")
        assert s.kv_reserve(3) == 0 and s.kv_capacity() == 3
        assert s.decode_step_cached(ids[:5], check=False)[0] == S("MODEL_ERR_CAPACITY")
        assert s.prefill(ids[:5], check=False)[0] == S("MODEL_ERR_CAPACITY")
        assert s.kv_length() == 0
        assert s.kv_set_length(9) == S("MODEL_ERR_CAPACITY")
        s.kv_set_length(1)
        assert s.decode_step_cached(ids[:3], check=False)[0] == S("MODEL_ERR_ARG")
        # range and argument refusals before any arithmetic
        bad = ids.copy()
        bad[0] = s.vocab
        s.set_decode_path(tie_b200.MODEL_PATH_NOCACHE)
        assert s.prefill(bad[:3], check=False)[0] == S("MODEL_ERR_RANGE")
        assert s.prefill(np.zeros(s.n_ctx + 1, np.int32), check=False)[0] in (
            S("MODEL_ERR_RANGE"), S("MODEL_ERR_CAPACITY"))
        assert s.kv_reserve(0) == S("MODEL_ERR_ARG")
        assert s.kv_reserve(s.n_ctx + 1) == S("MODEL_ERR_RANGE")


def test_both_cproj_readings(mini_paths, ids):
    """reference tests/test_model.c:459-502"""
    w, inv, cfg = mini_paths
    with tie_b200.Model(w, inv, cfg) as a:
        rec = [r for r in a.records() if "attn.c_proj" in r["name"]][0]
        assert rec["transposed_at_load"] == 0
        la = a.prefill(ids)[-1]
    with tie_b200.Model(w, inv, cfg, cproj=tie_b200.MODEL_CPROJ_TRANSPOSED) as b:
        rec = [r for r in b.records() if "attn.c_proj" in r["name"]][0]
        assert rec["transposed_at_load"] == 1
        lb = b.prefill(ids)[-1]
        ref = oracle.Oracle(w, cfg, cproj_transposed=True).prefill(ids)[-1]
        assert np.abs(lb - ref).max() <= 1e-3
    assert not np.array_equal(la, lb)
