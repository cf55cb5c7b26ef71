"""Randomised GPU parity sweep: seeded random shapes and options against the
float64 oracle, so that combinations no hand-picked case covers are exercised
(kernel size, stride, padding, dilation, deformable groups, channel counts that
are and are not multiples of 8 / 64, images above and below the tile scatter's
16 x 16 minimum, NCHW and channels-last, the backward reusing the forward's
packed input or packing it again, every dtype).

The shapes are drawn from a fixed seed, so a failure names a reproducible case.
Tolerances as in test_gpu_parity: 1e-4 for float32, 1e-2 for 16-bit tensors
(the oracle runs on the same rounded inputs).
"""
import random

import pytest
import torch

import oracle
from dcn_cases import Case, make_inputs, record, rel_err

TOL = {torch.float32: 1e-4, torch.float16: 1e-2, torch.bfloat16: 1e-2}
DTYPES = [torch.float32, torch.bfloat16, torch.float16]
NAMES = ["grad_input", "grad_offset", "grad_mask", "grad_weight", "grad_bias"]


def _draw(n=24, seed=2024):
    rng = random.Random(seed)
    out = []
    while len(out) < n:
        k = rng.choice([1, 3, 3, 3, 5])
        kh, kw = (k, k) if rng.random() < 0.8 else (k, rng.choice([1, 3]))
        s = rng.choice([1, 1, 1, 2])
        d = rng.choice([1, 1, 2])
        p = rng.choice([0, (max(kh, kw) // 2) * d, 1])
        dg = rng.choice([1, 1, 2, 4])
        C = dg * rng.choice([4, 8, 12, 16, 24, 32, 48, 64])
        H, W = rng.randint(5, 40), rng.randint(5, 40)
        Co = rng.choice([8, 16, 40, 64, 72, 96, 128, 136])
        B = rng.choice([1, 2])
        c = Case(f"r{len(out)}", B, C, H, W, Co, kh, kw, stride=s, pad=p, dil=d, dg=dg,
                 off_std=rng.choice([0.5, 1.5, 3.0]), bias=rng.random() < 0.8)
        ho, wo = c.out_hw()
        if ho < 1 or wo < 1:
            continue
        dtype = DTYPES[len(out) % 3]
        nhwc = (len(out) // 3) % 2 == 1
        reuse = (len(out) // 2) % 2 == 0
        out.append((c, dtype, nhwc, reuse))
    return out


CASES = _draw()


def _id(p):
    c, dt, nhwc, reuse = p
    return (f"{c.name}_{c.B}x{c.C}x{c.H}x{c.W}_co{c.Co}_k{c.kh}x{c.kw}_s{c.stride}p{c.pad}d{c.dil}"
            f"g{c.dg}_{str(dt).split('.')[-1]}{'_nhwc' if nhwc else ''}{'_reuse' if reuse else ''}")


@pytest.mark.gpu
@pytest.mark.parametrize("params", CASES, ids=_id)
def test_random_case_vs_oracle(params):
    from dcnv2_b200 import _C
    c, dtype, nhwc, reuse = params
    x, w, b, off, m, gy = [None if t is None else t.to(dtype) for t in make_inputs(c, seed=11)]
    f64 = lambda t: None if t is None else t.double().numpy()  # noqa: E731
    y_ref = oracle.forward(f64(x), f64(w), f64(b), f64(off), f64(m), c.stride, c.pad, c.dil, c.dg)
    g_ref = oracle.backward(f64(x), f64(w), f64(off), f64(m), f64(gy), c.stride, c.pad, c.dil, c.dg)
    dev = torch.device("cuda:0")
    fmt = torch.channels_last if nhwc else torch.contiguous_format
    cu = lambda t: None if t is None else t.to(dev)  # noqa: E731
    cl = lambda t: t.to(dev).contiguous(memory_format=fmt)  # noqa: E731
    X, M, OFF, GY = cl(x), cl(m), cl(off), cl(gy)
    s, p, d, dg = c.stride, c.pad, c.dil, c.dg
    ws = _C.backward_workspace(X, cu(w), s, s, p, p, d, d, dg) if reuse else None
    y = _C.dcn_v2_forward(X, cu(w), M, OFF, cu(b), s, s, p, p, d, d, dg, workspace=ws)
    grads = _C.dcn_v2_backward(X, cu(w), M, OFF, cu(b), GY, s, s, p, p, d, d, dg, workspace=ws,
                               input_packed=reuse)
    torch.cuda.synchronize()
    tol = TOL[dtype]
    errs = {"output": rel_err(y.float().cpu().numpy(), y_ref)}
    for name, g, r in zip(NAMES, grads, g_ref):
        if name == "grad_bias" and not c.bias:
            assert g is None
            continue
        errs[name] = rel_err(g.float().cpu().numpy(), r)
    record("random_" + _id(params), errs, tol)
    bad = {k: v for k, v in errs.items() if not v <= tol}
    assert not bad, f"{_id(params)}: errors {errs} (tol {tol})"
