"""The logit dump (the reference's TIE2LOGI block) and the divergence report."""
import json
import struct

import numpy as np
import pytest

from tie_b200 import logits as L


def test_dump_round_trip_and_layout(tmp_path):
    a = np.arange(12, dtype=np.float32).reshape(3, 4) - 5.5
    p = tmp_path / "x.bin"
    L.write_logit_dump(str(p), a)
    raw = p.read_bytes()
    assert raw[:8] == b"TIE2LOGI"
    assert struct.unpack("<ii", raw[8:16]) == (3, 4)
    assert len(raw) == 16 + 12 * 4
    assert np.array_equal(np.frombuffer(raw[16:], dtype="<f4").reshape(3, 4), a)
    assert np.array_equal(L.read_logit_dump(str(p)), a)


@pytest.mark.parametrize("body", [b"NOTLOGIT" + struct.pack("<ii", 1, 2) + b"\0" * 8,
                                  b"TIE2LOGI" + struct.pack("<ii", 2, 2) + b"\0" * 8,
                                  b"TIE2LOG"])
def test_bad_dumps_refused(tmp_path, body):
    p = tmp_path / "bad.bin"
    p.write_bytes(body)
    with pytest.raises(ValueError):
        L.read_logit_dump(str(p))


def test_statistics_on_a_known_case():
    ref = np.array([[3.0, 1.0, 0.0, -1.0, -2.0, -3.0],
                    [0.0, 2.0, 1.5, -1.0, -2.0, -3.0]], dtype=np.float32)
    eng = ref.copy()
    eng[1, 2] += 0.75          # position 1: top-1 flips from 1 to 2
    eng[0, 5] -= 0.25
    s = L.divergence_statistics(eng, ref, token_ids=[7, 8], label="case")
    assert s["positions"] == 2 and s["vocab_size"] == 6
    assert s["max_abs_diff"] == pytest.approx(0.75)
    assert (s["max_abs_diff_position"], s["max_abs_diff_token_id"]) == (1, 2)
    assert s["top1_agreement_positions"] == 1 and s["top1_disagreeing_positions"] == [1]
    assert s["top1_agreement_fraction"] == 0.5
    assert s["reference_top1_top2_margin"]["per_position"] == [2.0, 0.5]
    assert s["reference_top1_top2_margin"]["min"] == 0.5
    assert s["margin_min_over_max_abs_diff"] == pytest.approx(0.5 / 0.75)
    assert s["max_rel_diff"] == pytest.approx(0.75 / (1.5 + 1e-6))
    assert s["rms_abs_diff"] == pytest.approx(np.sqrt((0.75 ** 2 + 0.25 ** 2) / 12))
    assert s["elements_below_rel_floor"] == 2     # the two exact zeros of the reference
    assert s["top5_set_agreement_positions"] == 2
    assert s["token_ids"] == [7, 8] and s["label"] == "case"


def test_identical_logits():
    r = np.random.default_rng(1).standard_normal((5, 50)).astype(np.float32)
    s = L.divergence_statistics(r, r)
    assert s["max_abs_diff"] == 0.0 and s["margin_min_over_max_abs_diff"] is None
    assert s["top1_agreement_fraction"] == 1.0 and s["top5_set_agreement_fraction"] == 1.0


def test_shape_checks():
    with pytest.raises(ValueError):
        L.divergence_statistics(np.zeros((2, 3)), np.zeros((3, 2)))
    with pytest.raises(ValueError):
        L.divergence_statistics(np.zeros(3), np.zeros(3))


def test_command_line(tmp_path, capsys):
    r = np.random.default_rng(2).standard_normal((4, 30)).astype(np.float32)
    e = r + np.float32(1e-4)
    L.write_logit_dump(str(tmp_path / "e.bin"), e)
    L.write_logit_dump(str(tmp_path / "r.bin"), r)
    assert L.main([str(tmp_path / "e.bin"), str(tmp_path / "r.bin"), "cli"]) == 0
    s = json.loads(capsys.readouterr().out)
    assert s["label"] == "cli" and s["max_abs_diff"] == pytest.approx(1e-4, rel=1e-2)
    assert L.main([]) == 2
