"""The bench's results record in the reference harness's file format
(reference bench/microbench/bench_common.h:104-184): the statistics, the
VALID/INVALID verdict and the file layout, on CPU."""
import json
import math
import os

import pytest

from tie_b200 import results


def test_stats_valid_run():
    samples = [10.0 + 0.01 * (i % 3) for i in range(25)]
    st = results.stats(samples, warmup=5)
    assert st["n"] == 25 and st["valid"] and st["invalid_reason"] is None
    assert st["min_ms"] == 10.0 and st["max_ms"] == pytest.approx(10.02)
    assert st["median_ms"] == pytest.approx(10.01)
    assert st["stddev_pct_of_median"] < 1.0


@pytest.mark.parametrize("warmup, n, spread, reason", [
    (4, 25, 0.0, "warm-up"),
    (5, 19, 0.0, "samples"),
    (5, 25, 5.0, "stddev"),
])
def test_stats_invalid_runs_keep_their_numbers(warmup, n, spread, reason):
    samples = [10.0 + (spread if i % 2 else -spread) for i in range(n)]
    st = results.stats(samples, warmup)
    assert not st["valid"] and reason in st["invalid_reason"]
    assert st["median_ms"] is not None and st["n"] == n


def test_stats_no_samples():
    st = results.stats([], warmup=5)
    assert st["n"] == 0 and not st["valid"] and st["invalid_reason"] == "no samples"


def test_record_and_file_layout(tmp_path):
    rec = results.record("throughput", "gpt2-small 256x(64+448)", "tokens/s", 1234.5, 5,
                         [1.0] * 20, counters={"gpu_launches": 7}, annotations={"dtype": "f32"})
    assert rec["raw_samples_ms"] == [1.0] * 20 and rec["samples_requested"] == 20
    assert rec["statistics"]["valid"] and rec["counters"]["gpu_launches"] == 7
    head = {"stage": "s", "git_commit": "abc", "protocol": {"min_warmup": results.MIN_WARMUP}}
    path = results.write(str(tmp_path / "out"), "run1", head, [rec])
    assert os.path.basename(path) == "run1.json"
    doc = json.load(open(path))
    assert doc["stage"] == "s" and doc["records"][0]["benchmark"] == "throughput"
    assert math.isclose(doc["records"][0]["value"], 1234.5)


def test_protocol_limits_are_the_reference_harness_limits():
    assert (results.MIN_WARMUP, results.MIN_SAMPLES, results.MAX_STDDEV_PCT) == (5, 20, 5.0)
