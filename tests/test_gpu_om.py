"""The fused predictor path (dcn_forward_om / dcn_backward_om): the raw output of
the offset/mask predictor conv goes to the operator, which applies the
reference module's chunk / cat / sigmoid (dcn_v2_mm.py:133-137) itself.  Checked
against the separate-tensor path (itself checked against the float64 oracle) on
the same inputs, against the float64 oracle fed the reference module's own
sequence, and through the DCN module's autograd."""
import numpy as np
import pytest
import torch

from dcn_cases import SMALL, Case, make_inputs, record, rel_err

CASES = [c for c in SMALL if c.name in ("readme_small", "dg4_bf", "edge_c4", "c_odd", "direct_co100")]
TOL = {torch.float32: 1e-5, torch.float16: 1e-2, torch.bfloat16: 1e-2}


def _om_inputs(case, dtype):
    x, w, b, off, m, gy = make_inputs(case, seed=7)
    K2 = case.kh * case.kw
    logits = torch.randn(m.shape, generator=torch.Generator().manual_seed(11)) * case.mask_std
    om = torch.cat([off, logits], dim=1)
    dev = torch.device("cuda:0")
    cvt = lambda t: None if t is None else t.to(dtype).to(dev)  # noqa: E731
    x, w, b, om, gy = map(cvt, (x, w, b, om, gy))
    n_off = 2 * case.dg * K2
    offset = om[:, :n_off].contiguous()
    mask = torch.sigmoid(om[:, n_off:].float()).to(dtype).contiguous()
    return x, w, b, om, offset, mask, gy, n_off


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_om_matches_separate_tensors(case, dtype):
    from dcnv2_b200 import _C
    x, w, b, om, offset, mask, gy, n_off = _om_inputs(case, dtype)
    s, p, d, dg = case.stride, case.pad, case.dil, case.dg
    y_om = _C.dcn_v2_forward_om(x, w, om, b, s, s, p, p, d, d, dg)
    y = _C.dcn_v2_forward(x, w, mask, offset, b, s, s, p, p, d, d, dg)
    gi_om, gom, gw_om, gb_om = _C.dcn_v2_backward_om(x, w, om, b, gy, s, s, p, p, d, d, dg)
    gi, goff, gm, gw, gb = _C.dcn_v2_backward(x, w, mask, offset, b, gy, s, s, p, p, d, d, dg)
    torch.cuda.synchronize()
    sig = torch.sigmoid(om[:, n_off:].float())
    tol = TOL[dtype]
    f = lambda t: t.float().cpu().numpy()  # noqa: E731
    errs = {
        "output": rel_err(f(y_om), f(y)),
        "grad_input": rel_err(f(gi_om), f(gi)),
        "grad_offset": rel_err(f(gom[:, :n_off]), f(goff)),
        "grad_logit": rel_err(f(gom[:, n_off:]), f(gm.float() * sig * (1 - sig))),
        "grad_weight": rel_err(f(gw_om), f(gw)),
    }
    if b is not None:
        errs["grad_bias"] = rel_err(f(gb_om), f(gb))
    bad = {k: v for k, v in errs.items() if not v <= tol}
    assert not bad, f"{case.name} {dtype}: {errs}"


@pytest.mark.gpu
def test_dcn_module_uses_fused_path_and_matches_unfused():
    """DCN.forward (fused) against the reference module's own sequence (predictor,
    chunk, cat, sigmoid, dcn_v2_conv) with the same parameters, fp32."""
    from dcnv2_b200 import DCN, dcn_v2_conv
    torch.manual_seed(3)
    dev = torch.device("cuda:0")
    mod = DCN(32, 48, 3, stride=1, padding=1, deformable_groups=2).to(dev)
    with torch.no_grad():
        mod.conv_offset_mask.weight.normal_(0, 0.05)
        mod.conv_offset_mask.bias.normal_(0, 0.5)
    x = torch.randn(2, 32, 13, 17, device=dev, requires_grad=True)
    y = mod(x)
    gy = torch.randn_like(y)
    y.backward(gy)
    g_fused = [t.grad.clone() for t in (x, mod.weight, mod.bias, mod.conv_offset_mask.weight,
                                        mod.conv_offset_mask.bias)]
    for t in (x, mod.weight, mod.bias, mod.conv_offset_mask.weight, mod.conv_offset_mask.bias):
        t.grad = None
    out = mod.conv_offset_mask(x)
    o1, o2, mask = torch.chunk(out, 3, dim=1)
    y2 = dcn_v2_conv(x, mod.weight, torch.sigmoid(mask), torch.cat((o1, o2), dim=1), mod.bias,
                     mod.stride, mod.padding, mod.dilation, mod.deformable_groups)
    y2.backward(gy)
    g_ref = [t.grad for t in (x, mod.weight, mod.bias, mod.conv_offset_mask.weight,
                              mod.conv_offset_mask.bias)]
    assert rel_err(y.detach().cpu().numpy(), y2.detach().cpu().numpy()) <= 1e-5
    for a, r in zip(g_fused, g_ref):
        assert rel_err(a.cpu().numpy(), r.cpu().numpy()) <= 1e-4


@pytest.mark.gpu
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
@pytest.mark.parametrize("case", CASES + [Case("readme_b2", 2, 64, 128, 128, 256, 3, 3)],
                         ids=lambda c: c.name)
def test_om_vs_oracle(case, dtype):
    """dcn_forward_om / dcn_backward_om against the float64 oracle fed the
    reference module's own sequence (dcn_v2_mm.py:133-137): offset = om[:, :2dgK2]
    (the reference's cat(o1, o2)), mask = sigmoid(om[:, 2dgK2:]), and the logit
    gradient by the chain rule g_logit = g_mask * s * (1 - s), all in float64 on
    the dtype-rounded predictor output."""
    import oracle
    from dcnv2_b200 import _C
    x, w, b, om, _, _, gy, n_off = _om_inputs(case, dtype)
    s, p, d, dg = case.stride, case.pad, case.dil, case.dg
    y = _C.dcn_v2_forward_om(x, w, om, b, s, s, p, p, d, d, dg)
    gi, gom, gw, gb = _C.dcn_v2_backward_om(x, w, om, b, gy, s, s, p, p, d, d, dg)
    torch.cuda.synchronize()
    f64 = lambda t: None if t is None else t.double().cpu().numpy()  # noqa: E731
    om64 = f64(om)
    off64 = np.ascontiguousarray(om64[:, :n_off])
    sig = 1.0 / (1.0 + np.exp(-om64[:, n_off:]))
    y_r = oracle.forward(f64(x), f64(w), f64(b), off64, sig, s, p, d, dg)
    gx_r, goff_r, gm_r, gw_r, gb_r = oracle.backward(f64(x), f64(w), off64, sig, f64(gy), s, p, d, dg)
    glog_r = gm_r * sig * (1.0 - sig)
    tol = 1e-4 if dtype == torch.float32 else 1e-2
    gom64 = f64(gom)
    errs = {
        "output": rel_err(f64(y), y_r),
        "grad_input": rel_err(f64(gi), gx_r),
        "grad_offset": rel_err(gom64[:, :n_off], goff_r),
        "grad_logit": rel_err(gom64[:, n_off:], glog_r),
        "grad_weight": rel_err(f64(gw), gw_r),
    }
    if b is not None:
        errs["grad_bias"] = rel_err(f64(gb), gb_r)
    record(f"om_{case.name}_{str(dtype).split('.')[-1]}", errs, tol)
    bad = {k: v for k, v in errs.items() if not v <= tol}
    assert not bad, f"{case.name} {dtype}: {errs}"
