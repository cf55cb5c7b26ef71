"""Pins the C oracle (test infrastructure) against golden vectors:

* ref_*.npz: produced by the reference's own CUDA kernels (com.cu compiled for
  sm_100, tests/golden/make_ref_golden.py).  The reference backward is float32
  (cuBLAS SGEMM + fp32 kernels): oracle within 1e-5.  The reference forward rounds
  its GEMM operands to fp16 (com.cu:83, 87): oracle within 1e-3.
* tv_*.npz: torchvision.ops.deform_conv2d in float64 for dilation > 1 and
  deformable groups > 1 (tests/golden/make_tv_golden.py): oracle within 1e-12
  (sample positions formed in double, as torchvision does).
"""
import glob
import os

import numpy as np
import pytest

import oracle
from dcn_cases import rel_err

HERE = os.path.dirname(os.path.abspath(__file__))
GOLDEN = sorted(glob.glob(os.path.join(HERE, "golden", "*.npz")))
GRADS = ["grad_input", "grad_offset", "grad_mask", "grad_weight", "grad_bias"]


def _tols(name):
    if os.path.basename(name).startswith("ref_"):
        return 1e-3, 1e-5
    return 1e-12, 1e-12


def test_golden_present():
    names = [os.path.basename(f) for f in GOLDEN]
    assert any(n.startswith("ref_") for n in names) and any(n.startswith("tv_") for n in names)


@pytest.mark.parametrize("path", GOLDEN, ids=lambda p: os.path.basename(p)[:-4])
def test_oracle_matches_golden(path):
    z = np.load(path)
    s, p, d, dg = (int(v) for v in z["params"])
    tol_fwd, tol_bwd = _tols(path)
    # torchvision's double kernels form sample positions in double, the
    # reference's in float32 (the oracle's default)
    coord = "f32" if os.path.basename(path).startswith("ref_") else "f64"
    y = oracle.forward(z["x"], z["w"], z["b"], z["offset"], z["mask"], s, p, d, dg, coord=coord)
    assert rel_err(y, z["y"]) <= tol_fwd
    grads = oracle.backward(z["x"], z["w"], z["offset"], z["mask"], z["grad_out"], s, p, d, dg,
                            coord=coord)
    for name, g in zip(GRADS, grads):
        assert rel_err(g, z[name]) <= tol_bwd, name


def test_oracle_f32_close_to_f64():
    from dcn_cases import Case, make_inputs
    c = Case("t", 1, 8, 9, 7, 12, 3, 3, dg=2, dil=2, pad=2)
    x, w, b, off, m, gy = [t.numpy() for t in make_inputs(c)]
    y64 = oracle.forward(x, w, b, off, m, 1, 2, 2, 2)
    y32 = oracle.forward(x, w, b, off, m, 1, 2, 2, 2, dtype=np.float32)
    assert rel_err(y32, y64) < 1e-5
    g64 = oracle.backward(x, w, off, m, gy, 1, 2, 2, 2)
    g32 = oracle.backward(x, w, off, m, gy, 1, 2, 2, 2, dtype=np.float32)
    for a, r in zip(g32, g64):
        assert rel_err(a, r) < 1e-5


def test_oracle_zero_offsets_unit_mask_is_plain_conv():
    """offset 0, mask 1: DCNv2 reduces to an ordinary convolution."""
    import torch
    rng = np.random.default_rng(0)
    x = rng.standard_normal((2, 5, 8, 9))
    w = rng.standard_normal((7, 5, 3, 3))
    b = rng.standard_normal(7)
    off = np.zeros((2, 18, 8, 9))
    m = np.ones((2, 9, 8, 9))
    y = oracle.forward(x, w, b, off, m, 1, 1)
    ref = torch.nn.functional.conv2d(torch.from_numpy(x), torch.from_numpy(w), torch.from_numpy(b),
                                     padding=1).numpy()
    assert rel_err(y, ref) < 1e-12
