"""Prefill logits dumped in the reference's TIE2LOGI format and compared with
the oracle's through the divergence report."""
import os
import sys

import numpy as np
import pytest

import tie_b200
from tie_b200 import logits as L
from tie_b200 import synth

pytestmark = pytest.mark.gpu
ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


@pytest.mark.parametrize("shape", ["tiny", "mini"])
def test_prefill_dump_against_oracle(tmp_path, shape):
    sys.path.insert(0, os.path.join(ROOT, "oracle"))
    import oracle
    w, inv, cfg = synth.ensure_model(shape, seed=7, ln_affine="random")
    with tie_b200.Model(w, inv, cfg) as m:
        ids = synth.prompt_ids(m.vocab, 1, 24, seed=5)[0]
        L.write_logit_dump(str(tmp_path / "engine.bin"), m.prefill(ids))
    L.write_logit_dump(str(tmp_path / "oracle.bin"), oracle.Oracle(w, cfg).prefill(ids))
    s = L.divergence_statistics(L.read_logit_dump(str(tmp_path / "engine.bin")),
                                L.read_logit_dump(str(tmp_path / "oracle.bin")), token_ids=ids, label=shape)
    print(f"{shape}: max-abs {s['max_abs_diff']:.3g}, rms {s['rms_abs_diff']:.3g}, "
          f"top-1 {s['top1_agreement_fraction']:.3f}, margin/diff {s['margin_min_over_max_abs_diff']}")
    assert s["positions"] == 24
    assert s["max_abs_diff"] <= 1e-3
    assert s["top1_agreement_fraction"] == 1.0
