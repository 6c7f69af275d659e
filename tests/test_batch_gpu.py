"""Batches, the paged pool and sharding, on the GPU.

Every kernel's per-sequence arithmetic is independent of the batch it runs in,
so a sequence's logits and tokens are BIT-IDENTICAL whether it is decoded alone,
in a batch, or in whichever shard of a multi-GPU split it lands (the property
batch sharding across GPUs relies on)."""
import numpy as np
import pytest

import tie_b200
from tie_b200 import synth
from tie_b200.shard import shard_range

pytestmark = pytest.mark.gpu


def bits(a):
    return np.ascontiguousarray(a, np.float32).view(np.uint32)


@pytest.fixture(scope="module")
def m(mini_paths):
    w, inv, cfg = mini_paths
    mod = tie_b200.Model(w, inv, cfg)
    yield mod
    mod.close()


@pytest.mark.parametrize("B", [8, 40])  # the GEMV path (<= 8 rows) and the tiled path
def test_batch_invariance(m, B):
    prompts = synth.prompt_ids(m.vocab, B, 20, seed=31)
    n_new = 24
    m.batch_reserve(B, 20 + n_new)
    full = m.generate_greedy(prompts, n_new)
    # the same sequences again as two half batches, each still on the same path
    h = B // 2
    a = m.generate_greedy(prompts[:h], n_new)
    b = m.generate_greedy(prompts[h:], n_new)
    assert np.array_equal(np.concatenate([a, b]), full)


def test_small_batches_match_single_sequence_api(m):
    """The batch pool path and the single-sequence cache path run the same
    kernels: B=1 generation equals the reference-API greedy loop bit for bit."""
    prompt = synth.prompt_ids(m.vocab, 1, 17, seed=41)
    n_new = 12
    m.batch_reserve(4, 17 + n_new)
    gen = m.generate_greedy(prompt, n_new)[0]
    m.set_decode_path(tie_b200.MODEL_PATH_CACHE)
    m.kv_reserve(17 + n_new)
    seq = list(prompt[0])
    rows = [m.prefill(seq)[-1]]
    ids = [int(rows[0].argmax())]
    for k in range(1, n_new):
        seq.append(ids[-1])
        rows.append(m.decode_step_cached(seq))
        ids.append(int(rows[-1].argmax()))
    m.set_decode_path(tie_b200.MODEL_PATH_NOCACHE)
    assert np.array_equal(gen, np.array(ids, np.int32))
    # and decode_step_batch reproduces the same logits, one step at a time
    nxt, _ = m.prefill_batch(prompt)
    assert int(nxt[0]) == ids[0]
    for k in range(1, n_new):
        nxt, lg = m.decode_step_batch([ids[k - 1]], want_logits=True)
        assert np.array_equal(bits(lg[0]), bits(rows[k])), k
        assert int(nxt[0]) == ids[k]


@pytest.mark.parametrize("world", [2, 4, 8])
def test_shards_reproduce_the_full_batch(m, world):
    """What `bench.py --gpus N` does on N GPUs, replayed shard by shard on one:
    every shard's tokens equal the full batch's rows."""
    n = 160  # every shard keeps more than 16 sequences: the same matmul and attention path as the full batch
    prompts = synth.prompt_ids(m.vocab, n, 16, seed=51)
    m.batch_reserve(n, 16 + 10)
    full = m.generate_greedy(prompts, 10)
    for r in range(world):
        start, size = shard_range(n, r, world)
        part = m.generate_greedy(prompts[start:start + size], 10)
        assert np.array_equal(part, full[start:start + size])


def test_decode_step_batch_refusals(mini_paths):
    w, inv, cfg = mini_paths
    with tie_b200.Model(w, inv, cfg) as m:
        rc, _, _ = m.prefill_batch(np.zeros((1, 4), np.int32), check=False)
        assert rc == tie_b200.MODEL_STATUS.index("MODEL_ERR_ARG")  # no pool reserved yet
        m.batch_reserve(2, 8)
        prompts = synth.prompt_ids(m.vocab, 2, 8, seed=61)
        m.prefill_batch(prompts)
        rc, _, _ = m.decode_step_batch([1, 2], check=False)
        assert rc == tie_b200.MODEL_STATUS.index("MODEL_ERR_CAPACITY")  # pool is full
        rc, _, _ = m.prefill_batch(np.zeros((3, 4), np.int32), check=False)
        assert rc == tie_b200.MODEL_STATUS.index("MODEL_ERR_ARG")  # more sequences than reserved
        rc, _, _ = m.prefill_batch(np.full((2, 4), m.vocab, np.int32), check=False)
        assert rc == tie_b200.MODEL_STATUS.index("MODEL_ERR_RANGE")


def test_paged_pool_assigns_pages_as_contexts_grow(mini_paths):
    """A pool over exactly the pages a generation needs (6 sequences x 49
    positions = 4 pages each, against 7 each for the full capacity of 100)
    produces the same ids as a full reservation; released pages are reused by
    the next batch with results equal to a fresh pool's; a generation that
    outgrows the pages is refused with MODEL_ERR_CAPACITY."""
    w, inv, cfg = mini_paths
    S, T, n_new, cap = 6, 20, 30, 100
    with tie_b200.Model(w, inv, cfg) as full:
        prompts = synth.prompt_ids(full.vocab, S, T, seed=51)
        prompts_b = synth.prompt_ids(full.vocab, S, T, seed=52)
        full.batch_reserve(S, cap)
        ref = full.generate_greedy(prompts, n_new)
        ref_b = full.generate_greedy(prompts_b, n_new)
    need = S * ((T + n_new - 1 + 15) // 16)
    with tie_b200.Model(w, inv, cfg) as pm:
        pm.batch_reserve_pages(S, cap, need)
        assert pm.batch_free_pages() == need
        got = pm.generate_greedy(prompts, n_new)
        assert np.array_equal(got, ref)
        assert pm.batch_free_pages() == 0
        for s in range(S):
            pm.batch_release(s)
        assert pm.batch_free_pages() == need
        assert np.array_equal(pm.generate_greedy(prompts_b, n_new), ref_b)
        for s in range(S):
            pm.batch_release(s)
        with pytest.raises(tie_b200.ModelError) as e:
            pm.generate_greedy(prompts, 60)   # 79 positions: 5 pages each
        assert tie_b200.MODEL_STATUS[e.value.status] == "MODEL_ERR_CAPACITY"
        with pytest.raises(tie_b200.ModelError):
            pm.batch_reserve_pages(S, cap, S * 7 + 1)   # more pages than the sequences can hold


def test_prefill_rows_do_not_depend_on_the_batch(m):
    """A prefill of 8 x 128 = 1024 rows gives every sequence's logits bit for
    bit as its own 128-row prefill: LayerNorm, the tensor-core matmuls (a row's
    sums do not depend on the tile it lands in) and attention compute each row
    independently of the batch."""
    S, T = 8, 128
    prompts = synth.prompt_ids(m.vocab, S, T, seed=61)
    m.batch_reserve(S, T)
    _, full = m.prefill_batch(prompts, want_logits=True)
    for s in (0, 3, 7):
        _, one = m.prefill_batch(prompts[s:s + 1], want_logits=True)
        assert np.array_equal(bits(one[0]), bits(full[s])), s
