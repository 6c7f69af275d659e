"""The reference's own C callers against this engine (drop-in check).

oracle/Makefile `callers` compiles, unmodified, the reference's CLI (its
src/main.c + src/tokenizer.c, the tokenizer-driven greedy tool) and its
tests/test_kv_cache.c, tests/test_gemm_naive.c and tests/test_model.c against
this repository's include/ and links them with libtie_b200.so. Here, on the CPU:
they link with every symbol they use exported by the engine, and the CLI runs
its argument and artifact checks -- it refuses a missing tokenizer and an
unknown flag the reference's way (src/main.c:100-160) -- before any device
work. The test programs themselves run on the GPU (test_callers_gpu.py).
"""
import os
import shutil
import subprocess

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
ORACLE = os.path.join(ROOT, "oracle")
REF = os.path.join(ORACLE, "_ref")
CALLERS = ["gpt2_tool", "test_kv_cache", "test_gemm_naive", "test_model"]
LIB = os.path.join(ROOT, "transformer-inference-engine_b200", "lib", "libtie_b200.so")


@pytest.fixture(scope="module")
def callers():
    args = ["make", "-s", "-C", ORACLE, "callers-if-present"]
    if os.environ.get("TIE_REFERENCE_ROOT"):
        args.append("REF=" + os.environ["TIE_REFERENCE_ROOT"])
    subprocess.run(args, check=True)
    paths = {c: os.path.join(REF, c) for c in CALLERS}
    if not all(os.path.isfile(p) for p in paths.values()):
        pytest.skip("the reference's caller sources are not present here and no prebuilt callers exist")
    return paths


def _exported():
    out = subprocess.run(["nm", "-D", "--defined-only", LIB], capture_output=True, text=True, check=True).stdout
    return {l.split()[-1] for l in out.splitlines() if l.strip()}


@pytest.mark.skipif(shutil.which("nm") is None, reason="binutils absent")
def test_callers_link_against_the_engine(callers):
    exported = _exported()
    for name, path in callers.items():
        ldd = subprocess.run(["ldd", path], capture_output=True, text=True).stdout
        assert "libtie_b200.so" in ldd and "not found" not in ldd, (name, ldd)
        undef = subprocess.run(["nm", "-u", path], capture_output=True, text=True, check=True).stdout
        engine = [l.split()[-1] for l in undef.splitlines()
                  if l.split()[-1].startswith(("model_", "kv_", "gemm_", "st_"))]
        assert engine, name
        assert sorted(set(engine) - exported) == [], name


def test_cli_refuses_before_device_work(callers, tmp_path):
    tool = callers["gpt2_tool"]
    p = subprocess.run([tool, "--tokenizer", str(tmp_path / "missing.json")], capture_output=True, text=True,
                       timeout=60)
    assert p.returncode == 1 and p.stderr.startswith("tokenizer:"), (p.returncode, p.stderr)
    p = subprocess.run([tool, "--no-such-flag"], capture_output=True, text=True, timeout=60)
    assert p.returncode == 2 and "usage" in p.stderr
    p = subprocess.run([tool, "--kv-cache", "sideways"], capture_output=True, text=True, timeout=60)
    assert p.returncode == 2
