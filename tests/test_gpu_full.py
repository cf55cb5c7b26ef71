"""Parity at the benchmark configurations' real sizes ([1],
[2] and [4]), where the kernels take paths the small cases never reach:
several persistent tiles per CTA, many pixel chunks of the weight-gradient
split, full 32-bit index ranges.

* configs[0] (fp32, B=8, C=64, 128x128, Co=256) and the three fp16 ResNet-50
  layers of configs[1]: every output and gradient against the float64 C oracle
  on the whole batch.
* configs[4] (B=4, C=96, 97x131, Co=160, 5x5, s2 p4 d2 dg2, offsets N(0,8),
  masks sigmoid(N(0,3))), fp32 and bf16: against the float64 oracle, whole batch.
* configs[2] (bf16, B=32, C=512, 32x32, Co=512, dg=4): the per-sample tensors
  (output, grad_input, grad_offset, grad_mask) of samples 0 and 31 against the
  oracle run on those two samples; grad_weight and grad_bias (sums over the
  whole batch) against torchvision's deform_conv2d run on the GPU in float64
  (the same arithmetic; torchvision differs from the reference only in
  grad_offset at integer sample coordinates, which is not compared with it).
* The bf16 README layer against the float64 oracle on the same rounded inputs
  (max-norm 1e-2) and on the UNROUNDED float32 inputs: the north star's "bf16
  within 1e-2 of the fp32 result", as a relative Frobenius norm (the max-norm
  error is recorded beside the part that rounding the inputs alone causes;
  grad_offset away from the samples that the input rounding moves into another
  bilinear cell, where it is discontinuous).
* Sample positions are formed in float32 in the kernels, in the reference
  (com.cu:184, 479, 587, 688) and in the oracle; grad_offset jumps at integer
  positions, so a position formed in another precision would land in another
  cell for the few samples within one ulp of an integer.

Tolerances (max|a-b| / max|b| per tensor, as in the other parity tests): 1e-4
for float32, 1e-2 for float16 / bfloat16.  Every achieved error is printed in
the assertion message and, with DCN_PARITY_LOG set, appended to that file.
"""
import functools

import numpy as np
import pytest
import torch

import oracle
from dcn_cases import Case, make_inputs, record, rel_err

NAMES = ["output", "grad_input", "grad_offset", "grad_mask", "grad_weight", "grad_bias"]
TOL = {torch.float32: 1e-4, torch.float16: 1e-2, torch.bfloat16: 1e-2}

README = Case("c0_readme", 8, 64, 128, 128, 256, 3, 3, off_std=1.5)
RESNET = [Case("c1_s1", 16, 128, 64, 64, 128, 3, 3), Case("c1_s2", 16, 256, 32, 32, 256, 3, 3),
          Case("c1_s3", 16, 512, 16, 16, 512, 3, 3)]
EDGE = Case("c4_edge", 4, 96, 97, 131, 160, 5, 5, stride=2, pad=4, dil=2, dg=2, off_std=8.0, mask_std=3.0)
C512 = Case("c2_c512_dg4", 32, 512, 32, 32, 512, 3, 3, dg=4, off_std=2.0)


def _cuda_run(case, tensors):
    from dcnv2_b200 import _C
    x, w, b, off, m, gy = [None if t is None else t.cuda() for t in tensors]
    s, p, d, dg = case.stride, case.pad, case.dil, case.dg
    y = _C.dcn_v2_forward(x, w, m, off, b, s, s, p, p, d, d, dg)
    grads = _C.dcn_v2_backward(x, w, m, off, b, gy, s, s, p, p, d, d, dg)
    torch.cuda.synchronize()
    return [t.double().cpu().numpy() for t in (y, *grads)]


def _oracle_run(case, tensors):
    x, w, b, off, m, gy = [None if t is None else t.double().numpy() for t in tensors]
    s, p, d, dg = case.stride, case.pad, case.dil, case.dg
    y = oracle.forward(x, w, b, off, m, s, p, d, dg)
    return [y, *oracle.backward(x, w, off, m, gy, s, p, d, dg)]


@functools.lru_cache(maxsize=2)
def _oracle_fp32_inputs(case):
    """The float64 oracle on the float32 inputs (shared by the fp32 and the
    bf16-against-fp32 tests of the same case)."""
    return _oracle_run(case, make_inputs(case))


def _compare(label, got, ref, tol, names=NAMES):
    errs = {n: rel_err(a, r) for n, a, r in zip(names, got, ref)}
    record(label, errs, tol)
    bad = {k: v for k, v in errs.items() if not v <= tol}
    assert not bad, f"{label}: errors {errs} (tol {tol})"


@pytest.mark.gpu
def test_c0_readme_fp32_full():
    case = README
    _compare("c0_readme_fp32", _cuda_run(case, make_inputs(case)), _oracle_fp32_inputs(case), 1e-4)


def _cell_flips(case, off_a, off_b):
    """Samples (b, group, tap, pixel) whose float32 sample position falls in a
    different bilinear cell, or on the other side of the validity bound, under
    the two offset tensors.  grad_offset is discontinuous there (the one-sided
    coordinate weights of com.cu:388-429 switch cells), so rounding the inputs
    to bf16 may move it by O(1) at those samples whatever the kernel does."""
    ho_n, wo_n = case.out_hw()
    K2 = case.kh * case.kw
    oa = off_a.numpy().astype(np.float32).reshape(case.B, case.dg, K2, 2, ho_n, wo_n)
    ob = off_b.float().numpy().astype(np.float32).reshape(case.B, case.dg, K2, 2, ho_n, wo_n)
    t = np.arange(K2)
    bh = (np.arange(ho_n)[None, :] * case.stride - case.pad + (t // case.kw)[:, None] * case.dil)
    bw = (np.arange(wo_n)[None, :] * case.stride - case.pad + (t % case.kw)[:, None] * case.dil)
    bh = bh.astype(np.float32)[None, None, :, :, None]
    bw = bw.astype(np.float32)[None, None, :, None, :]
    flips = np.zeros(oa.shape[:3] + (ho_n, wo_n), dtype=bool)
    ha, wa = bh + oa[:, :, :, 0], bw + oa[:, :, :, 1]
    hb, wb = bh + ob[:, :, :, 0], bw + ob[:, :, :, 1]

    def valid(h, w):
        return (h > -1) & (w > -1) & (h < case.H) & (w < case.W)

    flips |= (np.floor(ha) != np.floor(hb)) | (np.floor(wa) != np.floor(wb))
    flips |= valid(ha, wa) != valid(hb, wb)
    return flips   # [B][dg][K2][Ho][Wo]


def _fro(a, r, keep=None):
    """||a - r||_2 / ||r||_2 over the kept elements (all when keep is None)."""
    d = a - r
    if keep is not None:
        d, r = d[keep], r[keep]
    den = float(np.sqrt((r.astype(np.float64) ** 2).sum()))
    return float(np.sqrt((d.astype(np.float64) ** 2).sum())) / den if den else 0.0


@pytest.mark.gpu
def test_c0_readme_bf16_full():
    """bf16 README layer, whole batch.

    (1) Against the float64 oracle on the same bf16-rounded inputs: max-norm
        error <= 1e-2 (what the kernels themselves add).
    (2) Against the float64 result of the UNROUNDED float32 inputs (the north
        star's "within 1e-2 of the fp32 result"): relative Frobenius-norm error
        <= 1e-2.  The max-norm error against that result is recorded but not
        bounded by 1e-2: rounding the inputs to bf16 alone, with no kernel
        involved (the oracle on rounded against unrounded inputs, also
        recorded), already moves the max-norm error of output and grad_mask to
        about 1e-2 (output 0.010, grad_mask 0.015 on one sample of this layer).
    grad_offset is compared away from the samples whose position the input
    rounding moves into another bilinear cell (see _cell_flips)."""
    case = README
    t32 = make_inputs(case)
    t16 = [t.to(torch.bfloat16) for t in t32]
    got = _cuda_run(case, t16)
    ref16 = _oracle_run(case, t16)
    _compare("c0_readme_bf16", got, ref16, 1e-2)
    ref32 = _oracle_fp32_inputs(case)
    flips = _cell_flips(case, t32[3], t16[3])
    keep = ~np.repeat(flips[:, :, :, None], 2, axis=3).reshape(got[2].shape)
    fro, mx, irr = {}, {}, {}
    for i, n in enumerate(NAMES):
        k = keep if n == "grad_offset" else None
        fro[n] = _fro(got[i], ref32[i], k)
        sel = (lambda v: v[keep]) if n == "grad_offset" else (lambda v: v)
        den = np.abs(ref32[i]).max()
        mx[n] = float(np.abs(sel(got[i]) - sel(ref32[i])).max() / den)
        irr[n] = float(np.abs(sel(ref16[i]) - sel(ref32[i])).max() / den)
    record("c0_readme_bf16_vs_fp32_fro", fro, 1e-2)
    record("c0_readme_bf16_vs_fp32_max (not bounded)", mx, 1e-2)
    record("c0_readme_input_rounding_only_max", {**irr, "flipped_samples": int(flips.sum()),
                                                  "samples": int(flips.size)}, 1e-2)
    bad = {k: v for k, v in fro.items() if not v <= 1e-2}
    assert not bad, f"bf16 vs fp32 result (Frobenius): {fro}; max-norm {mx}; input rounding alone {irr}"


@pytest.mark.gpu
@pytest.mark.parametrize("case", RESNET, ids=lambda c: c.name)
def test_c1_resnet_fp16_full(case):
    t = [v.to(torch.float16) for v in make_inputs(case)]
    _compare(f"{case.name}_fp16", _cuda_run(case, t), _oracle_run(case, t), 1e-2)


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
def test_c4_edge_full(dtype):
    case = EDGE
    t = [v.to(dtype) for v in make_inputs(case)]
    _compare(f"c4_edge_{str(dtype).split('.')[-1]}", _cuda_run(case, t), _oracle_run(case, t), TOL[dtype])


@pytest.mark.gpu
def test_c2_c512_dg4_bf16_full():
    from torchvision.ops import deform_conv2d
    case = C512
    t = [v.to(torch.bfloat16) for v in make_inputs(case)]
    got = _cuda_run(case, t)
    # per-sample tensors of the first and the last sample against the oracle
    idx = [0, case.B - 1]
    sub = [t[0][idx], t[1], t[2], t[3][idx], t[4][idx], t[5][idx]]
    ref = _oracle_run(case, sub)
    _compare("c2_c512_dg4_bf16_samples", [g[idx] for g in got[:4]], ref[:4], 1e-2, NAMES[:4])
    # batch sums against torchvision on the GPU in float64
    x, w, b, off, m, gy = [v.double().cuda() for v in t]
    x.requires_grad_(True)
    w.requires_grad_(True)
    b.requires_grad_(True)
    s, p, d = case.stride, case.pad, case.dil
    y = deform_conv2d(x, off, w, b, stride=(s, s), padding=(p, p), dilation=(d, d), mask=m)
    y.backward(gy)
    torch.cuda.synchronize()
    tv = [y.detach(), x.grad, w.grad, b.grad]
    f = lambda v: v.double().cpu().numpy()  # noqa: E731
    _compare("c2_c512_dg4_bf16_tv", [got[0], got[1], got[4], got[5]], [f(v) for v in tv], 1e-2,
             ["output", "grad_input", "grad_weight", "grad_bias"])
