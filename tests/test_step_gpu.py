"""The persistent decode step (one kernel per step for <= 4 sequences) against
the chained per-layer kernels of the same step.

Both paths form every sum in the same order, so their logits must be
bit-identical, not merely close; the end-to-end parity against the reference
(test_parity_gpu.py) then covers the persistent path too, because batch-1
generation runs through it by default.
"""
import numpy as np
import pytest

import tie_b200
from tie_b200 import synth

pytestmark = pytest.mark.gpu


def _model(shape, seed=7, ln="random"):
    w, inv, cfg = synth.ensure_model(shape, seed=seed, ln_affine=ln)
    return tie_b200.Model(w, inv, cfg)


def _decode_trace(m, kind, prompts, n_steps):
    """Prefill, then n_steps decode steps feeding back the greedy tokens;
    returns the stacked logits and tokens."""
    m.set_step_kernel(kind)
    S, T = prompts.shape
    m.batch_reserve(S, T + n_steps)
    nxt, _ = m.prefill_batch(prompts)
    logits, toks = [], [nxt.copy()]
    for _ in range(n_steps):
        nxt, lg = m.decode_step_batch(nxt, want_logits=True)
        logits.append(lg)
        toks.append(nxt.copy())
    return np.stack(logits), np.stack(toks)


@pytest.mark.parametrize("shape", ["tiny", "mini", "small"])
@pytest.mark.parametrize("n_seq", [1, 2, 3, 4])
def test_step_bit_identical_to_chain(shape, n_seq):
    with _model(shape) as m:
        prompts = synth.prompt_ids(m.vocab, n_seq, 21, seed=50 + n_seq)
        n_steps = 40 if shape != "small" else 12   # crosses several 16-position chunks
        lp, tp = _decode_trace(m, tie_b200.TIE_STEP_PERSISTENT, prompts, n_steps)
        lc, tc = _decode_trace(m, tie_b200.TIE_STEP_CHAINED, prompts, n_steps)
        assert np.array_equal(tp, tc)
        bad = np.argwhere(lp.view(np.uint32) != lc.view(np.uint32))
        assert len(bad) == 0, f"{len(bad)} logits differ, first {bad[:3].tolist()}"


@pytest.mark.parametrize("n_seq", [1, 3])
def test_step_long_context_bit_identical(n_seq):
    """Contexts past 256 positions: a head's attention spans several CTAs
    whose chunk partials the first one gathers and merges."""
    with _model("small", seed=1234, ln="unit") as m:
        prompts = synth.prompt_ids(m.vocab, n_seq, 700, seed=90 + n_seq)
        lp, tp = _decode_trace(m, tie_b200.TIE_STEP_PERSISTENT, prompts, 4)
        lc, tc = _decode_trace(m, tie_b200.TIE_STEP_CHAINED, prompts, 4)
        assert np.array_equal(tp, tc)
        assert np.array_equal(lp.view(np.uint32), lc.view(np.uint32))


def test_step_launches_one_kernel_per_step():
    with _model("mini") as m:
        m.set_step_kernel(tie_b200.TIE_STEP_PERSISTENT)
        prompts = synth.prompt_ids(m.vocab, 2, 9, seed=3)
        m.batch_reserve(2, 9 + 8)
        nxt, _ = m.prefill_batch(prompts)
        before = m.kernel_launches()
        for _ in range(5):
            nxt, _ = m.decode_step_batch(nxt)
        assert m.kernel_launches() - before == 5


def test_step_generation_matches_chain_small():
    """GPT-2 small, batch 1, 48 + 64 greedy tokens through each path."""
    with _model("small", seed=1234, ln="unit") as m:
        prompts = synth.prompt_ids(m.vocab, 1, 48, seed=11)
        m.batch_reserve(1, 48 + 64)
        m.set_step_kernel(tie_b200.TIE_STEP_PERSISTENT)
        a = m.generate_greedy(prompts, 64)
        m.set_step_kernel(tie_b200.TIE_STEP_CHAINED)
        b = m.generate_greedy(prompts, 64)
        assert np.array_equal(a, b)


def test_step_kernel_timer():
    with _model("mini") as m:
        m.batch_reserve(1, 64)
        ms = m.time_kernel("decode_step", 1, 40, iters=5)
        assert 0.0 < ms < 50.0


def test_step_kind_validation():
    with _model("tiny") as m:
        with pytest.raises(tie_b200.ModelError):
            m.set_step_kernel(7)


def test_chained_is_the_default():
    """Batch-1 steps run the chained kernels unless the persistent one is asked for."""
    with _model("mini") as m:
        prompts = synth.prompt_ids(m.vocab, 1, 9, seed=4)
        m.batch_reserve(1, 9 + 4)
        nxt, _ = m.prefill_batch(prompts)
        before = m.kernel_launches()
        nxt, _ = m.decode_step_batch(nxt)
        assert m.kernel_launches() - before > 1


@pytest.mark.parametrize("shape", ["tiny", "mini", "small"])
@pytest.mark.parametrize("n_seq", [1, 2, 3, 5, 8])
def test_stream_chain_bit_identical_to_unfused(shape, n_seq):
    """The stream chain (weights streamed into shared memory, LayerNorm,
    embedding and the attention merge folded into the matmuls) against the
    default chain of separate kernels: identical logits and tokens."""
    with _model(shape) as m:
        prompts = synth.prompt_ids(m.vocab, n_seq, 19, seed=70 + n_seq)
        n_steps = 36 if shape != "small" else 12
        ls, ts = _decode_trace(m, tie_b200.TIE_STEP_STREAM, prompts, n_steps)
        lu, tu = _decode_trace(m, tie_b200.TIE_STEP_CHAINED, prompts, n_steps)
        assert np.array_equal(ts, tu)
        bad = np.argwhere(ls.view(np.uint32) != lu.view(np.uint32))
        assert len(bad) == 0, f"{len(bad)} logits differ, first {bad[:3].tolist()}"


@pytest.mark.parametrize("fmt", [tie_b200.TIE_WEIGHTS_BF16, tie_b200.TIE_WEIGHTS_INT8])
@pytest.mark.parametrize("n_seq", [1, 4])
def test_stream_chain_reduced_formats_bit_identical(fmt, n_seq):
    with _model("mini") as m:
        m.set_weight_format(fmt)
        prompts = synth.prompt_ids(m.vocab, n_seq, 23, seed=80 + n_seq)
        ls, ts = _decode_trace(m, tie_b200.TIE_STEP_STREAM, prompts, 20)
        lu, tu = _decode_trace(m, tie_b200.TIE_STEP_CHAINED, prompts, 20)
        assert np.array_equal(ts, tu)
        assert np.array_equal(ls.view(np.uint32), lu.view(np.uint32))


def test_stream_chain_long_context_bit_identical():
    """Past 256 positions the merge folds more than 16 chunk partials."""
    with _model("small", seed=1234, ln="unit") as m:
        prompts = synth.prompt_ids(m.vocab, 2, 700, seed=93)
        ls, ts = _decode_trace(m, tie_b200.TIE_STEP_STREAM, prompts, 4)
        lu, tu = _decode_trace(m, tie_b200.TIE_STEP_CHAINED, prompts, 4)
        assert np.array_equal(ts, tu)
        assert np.array_equal(ls.view(np.uint32), lu.view(np.uint32))
