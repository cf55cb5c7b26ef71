"""FastDiv, the division by run-time constants used in the kernels' index
arithmetic, agrees with integer division (host build of the same header)."""
import os
import shutil
import subprocess

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


@pytest.mark.skipif(shutil.which("g++") is None, reason="needs g++")
def test_fastdiv_matches_integer_division(tmp_path):
    exe = tmp_path / "fastdiv_check"
    subprocess.run(["g++", "-O2", "-std=c++17", "-I", os.path.join(ROOT, "include"),
                    "-I", os.path.join(ROOT, "dcnv2_b200", "csrc"),
                    os.path.join(HERE, "native", "fastdiv_check.cpp"), "-o", str(exe)], check=True)
    out = subprocess.run([str(exe)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stdout + out.stderr
    assert "bad 0" in out.stdout
