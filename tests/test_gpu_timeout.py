"""Failure detection without a GPU fault: every mbarrier wait in the kernels is
bounded, and a kernel whose wait runs out records DCN_DEVERR_TIMEOUT in the
workspace status word, aborts its CTA and returns, leaving the context usable.

The test builds a study variant of the library (DCN_STUDY, a 2 ms wait limit)
in a temporary directory and, in a child process, runs one forward whose weight
tiles are withheld (study switch DCN_DEBUG_SKIP bit 3: the pipeline stage never
fills, nothing faults or traps): the call must raise with error bit 0x1
(DCN_DEVERR_TIMEOUT).  A following normal call in the same process must then
succeed and match the float64 oracle."""
import os
import shutil
import subprocess
import sys

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))

_CHILD = r"""
import os, sys
sys.path.insert(0, sys.argv[2])
sys.path.insert(0, os.path.join(sys.argv[2], "tests"))
sys.path.insert(0, sys.argv[1])          # the study build first
import torch
import oracle
from dcn_cases import Case, make_inputs, rel_err
from dcnv2_b200 import _C, _lib
assert _lib.LIB_PATH.startswith(sys.argv[1]), _lib.LIB_PATH
c = Case("t", 2, 64, 16, 16, 128, 3, 3)
x, w, b, off, m, gy = [t.to(torch.bfloat16) for t in make_inputs(c)]
cu = [t.cuda() for t in (x, w, b, off, m)]
os.environ["DCN_DEBUG_SKIP"] = "8"
try:
    _C.dcn_v2_forward(cu[0], cu[1], cu[4], cu[3], cu[2], 1, 1, 1, 1)
    print("NO-ERROR")
except RuntimeError as e:
    print("ERROR", e)
os.environ["DCN_DEBUG_SKIP"] = "0"
y = _C.dcn_v2_forward(cu[0], cu[1], cu[4], cu[3], cu[2], 1, 1, 1, 1)
torch.cuda.synchronize()
f = lambda t: t.double().numpy()
ref = oracle.forward(f(x), f(w), f(b), f(off), f(m), 1, 1)
print("AFTER", rel_err(y.double().cpu().numpy(), ref))
"""


@pytest.mark.gpu
def test_wait_runs_out_reports_timeout_and_context_survives(tmp_path):
    pkg = tmp_path / "var"
    pkg.mkdir()
    shutil.copytree(os.path.join(ROOT, "dcnv2_b200"), pkg / "dcnv2_b200",
                    ignore=shutil.ignore_patterns("_build", "*.so", "__pycache__"))
    shutil.copytree(os.path.join(ROOT, "include"), pkg / "include")
    build = (f"import sys; sys.path.insert(0, {str(pkg / 'dcnv2_b200')!r}); import build; "
             "build.build(8, False, extra_flags=['-DDCN_STUDY', '-DDCN_WAIT_TIMEOUT_NS=2000000ull'])")
    subprocess.run([sys.executable, "-c", build], check=True, timeout=900)
    env = dict(os.environ, DCN_CHECK="1")
    r = subprocess.run([sys.executable, "-c", _CHILD, str(pkg), ROOT], env=env, capture_output=True,
                       text=True, timeout=300)
    out = r.stdout
    assert r.returncode == 0, r.stdout + r.stderr
    assert "ERROR" in out and "0x1" in out, out
    after = float(out.split("AFTER")[1].split()[0])
    assert after <= 1e-2, out
