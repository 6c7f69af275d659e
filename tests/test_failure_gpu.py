"""Failure detection on the GPU without a fault: a bounded wait that runs out.

model_debug_wait_drill makes the next decode step's first matmul (on the
TIE_STEP_STREAM path, whose kernels wait on shared-memory barriers for their
bulk copies) wait on a barrier that nothing completes. The wait gives up after the
given limit, the kernel records the expiry in the model's device error flag
and returns; the call must report MODEL_ERR_DEVICE, leave the cache length
where it was, and the next step must run normally -- bit-identical to a model
that never failed. (The reference's own rule for a refused call is that it
leaves the state untouched: src/model.c:878-883.)"""
import numpy as np
import pytest

import tie_b200
from tie_b200 import synth

pytestmark = pytest.mark.gpu


def _steps(m, prompts, n, drill_at=None):
    m.set_step_kernel(tie_b200.TIE_STEP_STREAM)
    S, T = prompts.shape
    m.batch_reserve(S, T + n + 2)
    nxt, _ = m.prefill_batch(prompts)
    out, rcs = [], []
    k = 0
    while len(out) < n:
        if k == drill_at:
            m.debug_wait_drill(2_000_000)   # 2 ms
            rc, _, _ = m.decode_step_batch(nxt, check=False)
            rcs.append(rc)
        k += 1
        nxt, lg = m.decode_step_batch(nxt, want_logits=True)
        out.append(lg)
    return np.stack(out), rcs


@pytest.mark.parametrize("n_seq", [1, 3])
def test_expired_wait_reports_device_error_and_recovers(mini_paths, n_seq):
    w, inv, cfg = mini_paths
    prompts = synth.prompt_ids(2003, n_seq, 12, seed=71)
    with tie_b200.Model(w, inv, cfg) as clean:
        want, _ = _steps(clean, prompts, 6)
    with tie_b200.Model(w, inv, cfg) as m:
        got, rcs = _steps(m, prompts, 6, drill_at=2)
        assert rcs == [tie_b200.MODEL_STATUS.index("MODEL_ERR_DEVICE")]
        assert b"bounded wait" in tie_b200.library().tie_last_device_error()
    assert np.array_equal(got.view(np.uint32), want.view(np.uint32))


def test_drill_refusals(mini_paths):
    w, inv, cfg = mini_paths
    L = tie_b200.library()
    assert L.model_debug_wait_drill(None, 1000) == tie_b200.MODEL_STATUS.index("MODEL_ERR_ARG")
    with tie_b200.Model(w, inv, cfg) as m:
        assert L.model_debug_wait_drill(m.h, 0) == tie_b200.MODEL_STATUS.index("MODEL_ERR_ARG")
