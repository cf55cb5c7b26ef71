"""GPU parity: the CUDA operator (through its C ABI, via the Conv2d._C-compatible
shim) against the float64 C oracle, on seeded inputs.

Tolerances (max|a-b| / max|b| per tensor): 1e-4 for float32 tensors, 1e-2 for
float16 / bfloat16 tensors (the oracle then runs on the same rounded inputs).
"""
import numpy as np
import pytest
import torch

import oracle
from dcn_cases import SMALL, make_inputs, record, rel_err

TOL = {torch.float32: 1e-4, torch.float16: 1e-2, torch.bfloat16: 1e-2}
DTYPES = [torch.float32, torch.bfloat16, torch.float16]
NAMES = ["grad_input", "grad_offset", "grad_mask", "grad_weight", "grad_bias"]


def _run(case, dtype, seed=0):
    from dcnv2_b200 import _C
    x, w, b, off, m, gy = [None if t is None else t.to(dtype) for t in make_inputs(case, seed)]
    f64 = lambda t: None if t is None else t.double().numpy()  # noqa: E731
    y_ref = oracle.forward(f64(x), f64(w), f64(b), f64(off), f64(m), case.stride, case.pad,
                           case.dil, case.dg)
    g_ref = oracle.backward(f64(x), f64(w), f64(off), f64(m), f64(gy), case.stride, case.pad,
                            case.dil, case.dg)
    dev = torch.device("cuda:0")
    cu = lambda t: None if t is None else t.to(dev)  # noqa: E731
    y = _C.dcn_v2_forward(cu(x), cu(w), cu(m), cu(off), cu(b), case.stride, case.stride,
                          case.pad, case.pad, case.dil, case.dil, case.dg)
    grads = _C.dcn_v2_backward(cu(x), cu(w), cu(m), cu(off), cu(b), cu(gy), case.stride,
                               case.stride, case.pad, case.pad, case.dil, case.dil, case.dg)
    torch.cuda.synchronize()
    return y, y_ref, grads, g_ref


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", DTYPES, ids=lambda d: str(d).split(".")[-1])
@pytest.mark.parametrize("case", SMALL, ids=lambda c: c.name)
def test_forward_backward_vs_oracle(case, dtype):
    y, y_ref, grads, g_ref = _run(case, dtype)
    tol = TOL[dtype]
    errs = {"output": rel_err(y.float().cpu().numpy(), y_ref)}
    for name, g, r in zip(NAMES, grads, g_ref):
        if name == "grad_bias" and not case.bias:
            assert g is None
            continue
        errs[name] = rel_err(g.float().cpu().numpy(), r)
    record(f"{case.name}_{str(dtype).split('.')[-1]}", errs, tol)
    bad = {k: v for k, v in errs.items() if not v <= tol}
    assert not bad, f"{case.name} {dtype}: errors {errs} (tol {tol})"


@pytest.mark.gpu
def test_deterministic_forward():
    from dcnv2_b200 import _C
    case = SMALL[0]
    x, w, b, off, m, _ = [t.cuda() for t in make_inputs(case)]
    y1 = _C.dcn_v2_forward(x, w, m, off, b, 1, 1, 1, 1)
    y2 = _C.dcn_v2_forward(x, w, m, off, b, 1, 1, 1, 1)
    assert torch.equal(y1, y2)


@pytest.mark.gpu
def test_empty_batch():
    from dcnv2_b200 import _C
    case = SMALL[0]
    x, w, b, off, m, gy = [t.cuda() for t in make_inputs(case)]
    y = _C.dcn_v2_forward(x[:0], w, m[:0], off[:0], b, 1, 1, 1, 1)
    assert y.shape == (0, case.Co, 16, 16)
    gi, go, gm, gw, gb = _C.dcn_v2_backward(x[:0], w, m[:0], off[:0], b, gy[:0], 1, 1, 1, 1)
    assert gi.shape == x[:0].shape and gw.abs().max().item() == 0 and gb.abs().max().item() == 0


GOLDEN_DIR = __import__("os").path.join(__import__("os").path.dirname(__file__), "golden")


def _golden_files():
    import glob
    import os
    return sorted(glob.glob(os.path.join(GOLDEN_DIR, "*.npz")))


@pytest.mark.gpu
@pytest.mark.parametrize("path", _golden_files(), ids=lambda p: p.split("/")[-1][:-4])
def test_golden_vectors_fp32(path):
    """float32 operator on the golden inputs (with integer offsets for ref_*):
    output within 1e-4 of the float64 oracle and within 1e-3 of the reference's
    fp16-GEMM forward; gradients within 1e-4 of the golden gradients."""
    from dcnv2_b200 import _C
    z = np.load(path)
    s, p, d, dg = (int(v) for v in z["params"])
    cu = {k: torch.from_numpy(np.ascontiguousarray(z[k]).astype(np.float32)).cuda()
          for k in ("x", "w", "b", "offset", "mask", "grad_out")}
    y = _C.dcn_v2_forward(cu["x"], cu["w"], cu["mask"], cu["offset"], cu["b"], s, s, p, p, d, d, dg)
    grads = _C.dcn_v2_backward(cu["x"], cu["w"], cu["mask"], cu["offset"], cu["b"], cu["grad_out"],
                               s, s, p, p, d, d, dg)
    f32 = {k: np.ascontiguousarray(z[k]).astype(np.float32).astype(np.float64)
           for k in ("x", "w", "b", "offset", "mask", "grad_out")}
    y_or = oracle.forward(f32["x"], f32["w"], f32["b"], f32["offset"], f32["mask"], s, p, d, dg)
    assert rel_err(y.cpu().numpy(), y_or) <= 1e-4
    assert rel_err(y.cpu().numpy(), z["y"]) <= 1e-3
    for name, g in zip(NAMES, grads):
        assert rel_err(g.cpu().numpy(), z[name]) <= 1e-4, name


_CHUNKED_SCRIPT = r"""
import sys, numpy as np, torch
sys.path.insert(0, sys.argv[1])
from dcn_cases import Case, make_inputs
from dcnv2_b200 import _C
H, W = int(sys.argv[4]), int(sys.argv[5])
c = Case("chunked", 3, 40, H, W, 72, 3, 3, off_std=2.0)
dt = {"bf16": torch.bfloat16, "fp32": torch.float32}[sys.argv[3]]
x, w, b, off, m, gy = [t.to(dt).cuda() for t in make_inputs(c, seed=3)]
g = _C.dcn_v2_backward(x, w, m, off, b, gy, 1, 1, 1, 1)
torch.cuda.synchronize()
np.savez(sys.argv[2], *[t.float().cpu().numpy() for t in g])
"""


@pytest.mark.gpu
@pytest.mark.parametrize("dtype,hw", [("fp32", (37, 29)), ("bf16", (37, 29)), ("bf16", (32, 32))],
                         ids=["fp32", "bf16", "bf16_direct"])
def test_backward_in_pixel_chunks(tmp_path, dtype, hw):
    """A 1 MB chunk budget (DCN_GCOL_MB=1) splits the backward of a 3219-pixel
    problem into chunks of 384 (bf16) or 128 (fp32) pixels, the last one ragged
    (not a multiple of 64); at 32x32 (3072 pixels, bf16) the GEMMs read
    grad_output directly and chunks cross image boundaries:
    every gradient still matches the float64 oracle."""
    import os
    import subprocess
    import sys
    from dcn_cases import Case
    c = Case("chunked", 3, 40, hw[0], hw[1], 72, 3, 3, off_std=2.0)
    out = tmp_path / "g.npz"
    env = dict(os.environ, DCN_GCOL_MB="1")
    here = os.path.dirname(os.path.abspath(__file__))
    subprocess.run([sys.executable, "-c", _CHUNKED_SCRIPT, here, str(out), dtype, str(hw[0]),
                    str(hw[1])], env=env,
                   check=True, cwd=os.path.dirname(here), timeout=300)
    z = np.load(out)
    tdt = {"bf16": torch.bfloat16, "fp32": torch.float32}[dtype]
    x, w, b, off, m, gy = [t.to(tdt).double().numpy() for t in make_inputs(c, seed=3)]
    ref = oracle.backward(x, w, off, m, gy, 1, 1, 1, 1)
    tol = 1e-4 if dtype == "fp32" else 1e-2
    for i, name in enumerate(NAMES):
        assert rel_err(z[f"arr_{i}"], ref[i]) <= tol, name
