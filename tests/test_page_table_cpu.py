"""The paged KV pool's page allocator (csrc/page_table.h) on CPU: assignment by
prefix, refusal without partial effects, release and reuse, the device view's
scratch entries, and a randomised run against a model of the allocation.
The checks are C++ (tests/page_table_check.cpp) built with the host compiler."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(os.path.dirname(HERE), "transformer-inference-engine_b200", "csrc")


@pytest.mark.skipif(shutil.which("g++") is None, reason="no host C++ compiler")
def test_page_allocator(tmp_path):
    exe = str(tmp_path / "page_table_check")
    subprocess.run(["g++", "-std=c++17", "-O1", "-Wall", "-Werror", "-I", CSRC,
                    os.path.join(HERE, "page_table_check.cpp"), "-o", exe], check=True)
    p = subprocess.run([exe], capture_output=True, text=True, timeout=120)
    assert p.returncode == 0 and p.stdout.strip() == "ok", p.stdout + p.stderr
