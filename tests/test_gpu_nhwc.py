"""Channels-last activations (DCN_NHWC): the operator fed tensors in PyTorch's
channels_last memory format must give the same results as the float64 oracle
(and return channels-last outputs and gradients), through the separate-tensor
API, the fused predictor API and the DCN module.  Tolerances as the other parity
tests: 1e-4 for float32, 1e-2 for 16-bit types."""
import pytest
import torch

import oracle
from dcn_cases import SMALL, Case, make_inputs, record, rel_err

CL = torch.channels_last
TOL = {torch.float32: 1e-4, torch.float16: 1e-2, torch.bfloat16: 1e-2}
NAMES = ["output", "grad_input", "grad_offset", "grad_mask", "grad_weight", "grad_bias"]
CASES = [c for c in SMALL if c.name in ("readme_small", "c_odd", "stride2_pad0", "dg4_bf", "edge_c4",
                                        "k1_nopad", "nobias", "direct_co100", "co512_c512", "win_20x32")]
CASES.append(Case("k1_c256_co64", 2, 256, 12, 10, 64, 1, 1, pad=0))


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16, torch.float16],
                         ids=lambda d: str(d).split(".")[-1])
@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_nhwc_vs_oracle(case, dtype):
    from dcnv2_b200 import _C
    x, w, b, off, m, gy = [None if t is None else t.to(dtype) for t in make_inputs(case, seed=2)]
    s, p, d, dg = case.stride, case.pad, case.dil, case.dg
    f64 = lambda t: None if t is None else t.double().numpy()  # noqa: E731
    ref = [oracle.forward(f64(x), f64(w), f64(b), f64(off), f64(m), s, p, d, dg),
           *oracle.backward(f64(x), f64(w), f64(off), f64(m), f64(gy), s, p, d, dg)]
    cl = lambda t: None if t is None else t.cuda().contiguous(memory_format=CL)  # noqa: E731
    cu = lambda t: None if t is None else t.cuda()  # noqa: E731
    xc, offc, mc, gyc = cl(x), cl(off), cl(m), cl(gy)
    y = _C.dcn_v2_forward(xc, cu(w), mc, offc, cu(b), s, s, p, p, d, d, dg)
    grads = _C.dcn_v2_backward(xc, cu(w), mc, offc, cu(b), gyc, s, s, p, p, d, d, dg)
    torch.cuda.synchronize()
    if case.C > 1:
        assert y.is_contiguous(memory_format=CL) and grads[0].is_contiguous(memory_format=CL)
    errs = {}
    for n, a, r in zip(NAMES, [y, *grads], ref):
        if n == "grad_bias" and not case.bias:
            continue
        errs[n] = rel_err(a.double().cpu().numpy(), r)
    tol = TOL[dtype]
    record(f"nhwc_{case.name}_{str(dtype).split('.')[-1]}", errs, tol)
    bad = {k: v for k, v in errs.items() if not v <= tol}
    assert not bad, f"{case.name} {dtype}: {errs}"


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
def test_nhwc_om_matches_nchw(dtype):
    """The fused predictor path with a channels-last predictor output equals the
    NCHW fused path (itself checked against the oracle)."""
    from dcnv2_b200 import _C
    case = Case("om_cl", 2, 64, 14, 18, 96, 3, 3, dg=2)
    x, w, b, off, m, gy = make_inputs(case, seed=4)
    logits = torch.randn(m.shape, generator=torch.Generator().manual_seed(3))
    om = torch.cat([off, logits], 1)
    x, w, b, om, gy = [t.to(dtype).cuda() for t in (x, w, b, om, gy)]
    args = (1, 1, 1, 1, 1, 1, case.dg)
    y0 = _C.dcn_v2_forward_om(x, w, om, b, *args)
    g0 = _C.dcn_v2_backward_om(x, w, om, b, gy, *args)
    xc, omc, gyc = [t.contiguous(memory_format=CL) for t in (x, om, gy)]
    y1 = _C.dcn_v2_forward_om(xc, w, omc, b, *args)
    g1 = _C.dcn_v2_backward_om(xc, w, omc, b, gyc, *args)
    torch.cuda.synchronize()
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    assert g1[1].is_contiguous(memory_format=CL)
    for a, r in zip([y1, *g1], [y0, *g0]):
        assert rel_err(a.float().cpu().numpy(), r.float().cpu().numpy()) <= tol


@pytest.mark.gpu
def test_dcn_module_channels_last():
    """DCN modules on a channels_last activation (what a channels_last network
    feeds them): outputs stay channels_last and the outputs and every parameter
    gradient equal those of the same modules on NCHW input.  The predictors'
    weights are zero and their biases random, so both layouts see bit-identical
    offsets and masks: grad_offset is discontinuous at integer sample positions,
    and the last-bit differences between cuDNN's NCHW and channels-last
    convolutions would otherwise move a few samples across a cell boundary."""
    from dcnv2_b200 import DCN
    torch.manual_seed(1)
    dev = torch.device("cuda:0")
    layers = [DCN(64, 64, 3, stride=1, padding=1).to(dev) for _ in range(2)]
    with torch.no_grad():
        for lay in layers:
            lay.conv_offset_mask.weight.zero_()
            lay.conv_offset_mask.bias.normal_(0, 0.7)
    torch.backends.cudnn.allow_tf32 = False
    x = torch.randn(2, 64, 16, 20, device=dev)
    gy = torch.randn(2, 64, 16, 20, device=dev)

    def run(xin, gin):
        for lay in layers:
            lay.zero_grad(set_to_none=True)
        xin = xin.clone().requires_grad_(True)
        h = xin
        for i, lay in enumerate(layers):
            h = lay(h)
            if i == 0:
                h = torch.relu(h)
        h.backward(gin)
        return h, xin.grad, [p.grad.clone() for lay in layers for p in lay.parameters()]

    y0, gx0, gp0 = run(x, gy)
    y1, gx1, gp1 = run(x.contiguous(memory_format=CL), gy.contiguous(memory_format=CL))
    assert y1.is_contiguous(memory_format=CL)
    assert rel_err(y1.detach().cpu().numpy(), y0.detach().cpu().numpy()) <= 1e-5
    assert rel_err(gx1.cpu().numpy(), gx0.cpu().numpy()) <= 1e-4
    for a, r in zip(gp1, gp0):
        assert rel_err(a.cpu().numpy(), r.cpu().numpy()) <= 1e-4
