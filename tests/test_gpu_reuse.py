"""Workspace reuse (DCN_FLAG_INPUT_PACKED, DCN_FLAG_WEIGHT_PACKED).

* A backward that reuses the input the forward packed into a shared workspace
  must return what a backward that packs it again returns: the same kernels
  see the same bytes.  grad_offset and grad_mask are sums in a fixed order and
  must be identical; grad_input, grad_weight and grad_bias are accumulated with
  fp32 atomics (L2 reductions) whose order varies from run to run, so they are
  compared at 1e-5 (fp32) / 1e-2 (16-bit, one output rounding) of their max.
  NCHW and channels-last, the 16-bit register-transpose pack and the generic
  one (f32, odd sizes), the fused predictor path.
* The DCN module's autograd (which reuses by default) against the same module
  with the reuse switched off.
* The inference weight cache: a repeated forward with the same weight returns
  the same output; after an in-place update of the weight (a new version) the
  cached pack is not used and the output follows the new weight.
"""
import pytest
import torch

from dcn_cases import SMALL, make_inputs, rel_err

CASES = [c for c in SMALL if c.name in ("readme_small", "c_odd", "edge_c4", "win_20x32", "nobias")]


def _inputs(case, dtype, nhwc):
    dev = torch.device("cuda:0")
    x, w, b, off, m, gy = make_inputs(case, seed=3)
    cvt = lambda t: None if t is None else t.to(dtype).to(dev)  # noqa: E731
    x, w, b, off, m, gy = map(cvt, (x, w, b, off, m, gy))
    if nhwc:
        cl = torch.channels_last
        x, off, m, gy = (t.contiguous(memory_format=cl) for t in (x, off, m, gy))
    return x, w, b, off, m, gy


def _compare(got, ref, dtype, what, exact=("grad_offset", "grad_mask")):
    names = ["grad_input", "grad_offset", "grad_mask", "grad_weight", "grad_bias"]
    tol = 1e-5 if dtype == torch.float32 else 1e-2
    for n, a, r in zip(names, got, ref):
        if r is None:
            assert a is None
            continue
        if n in exact:
            assert torch.equal(a, r), f"{what}: {n} differs"
        else:
            e = rel_err(a.float().cpu().numpy(), r.float().cpu().numpy())
            assert e <= tol, f"{what}: {n} rel err {e}"


@pytest.mark.gpu
@pytest.mark.parametrize("nhwc", [False, True], ids=["nchw", "nhwc"])
@pytest.mark.parametrize("dtype", [torch.float32, torch.bfloat16], ids=["fp32", "bf16"])
@pytest.mark.parametrize("case", CASES, ids=lambda c: c.name)
def test_backward_reusing_packed_input_is_identical(case, dtype, nhwc):
    from dcnv2_b200 import _C
    x, w, b, off, m, gy = _inputs(case, dtype, nhwc)
    s, p, d, dg = case.stride, case.pad, case.dil, case.dg
    ref = _C.dcn_v2_backward(x, w, m, off, b, gy, s, s, p, p, d, d, dg)
    ws = _C.backward_workspace(x, w, s, s, p, p, d, d, dg)
    # stale accumulator contents must not leak into the result: dirty the buffer
    ws.fill_(0x5a)
    y = _C.dcn_v2_forward(x, w, m, off, b, s, s, p, p, d, d, dg, workspace=ws)
    got = _C.dcn_v2_backward(x, w, m, off, b, gy, s, s, p, p, d, d, dg, workspace=ws, input_packed=True)
    y_ref = _C.dcn_v2_forward(x, w, m, off, b, s, s, p, p, d, d, dg)
    torch.cuda.synchronize()
    assert torch.equal(y, y_ref)
    _compare(got, ref, dtype, f"{case.name} {dtype} nhwc={nhwc}")
    assert _C.read_device_status(ws) == 0


@pytest.mark.gpu
def test_om_backward_reusing_packed_input_is_identical():
    from dcnv2_b200 import _C
    case = [c for c in SMALL if c.name == "readme_small"][0]
    x, w, b, off, m, gy = _inputs(case, torch.bfloat16, False)
    om = torch.cat([off, m], dim=1).contiguous()
    ref = _C.dcn_v2_backward_om(x, w, om, b, gy, 1, 1, 1, 1)
    ws = _C.backward_workspace(x, w, 1, 1, 1, 1)
    _C.dcn_v2_forward_om(x, w, om, b, 1, 1, 1, 1, workspace=ws)
    got = _C.dcn_v2_backward_om(x, w, om, b, gy, 1, 1, 1, 1, workspace=ws, input_packed=True)
    torch.cuda.synchronize()
    # [grad_input, grad_offset_mask, grad_weight, grad_bias]
    _compare([got[0], got[1], None, got[2], got[3]], [ref[0], ref[1], None, ref[2], ref[3]],
             torch.bfloat16, "om", exact=("grad_offset",))


@pytest.mark.gpu
@pytest.mark.parametrize("nhwc", [False, True], ids=["nchw", "nhwc"])
def test_module_grads_with_and_without_reuse(nhwc):
    from dcnv2_b200 import _C
    from dcnv2_b200.modules import DCN
    torch.manual_seed(0)
    dev = torch.device("cuda:0")
    layer = DCN(64, 96, 3, stride=1, padding=1).to(dev).to(torch.bfloat16)
    with torch.no_grad():
        layer.conv_offset_mask.bias.normal_(0, 0.5)
    x = torch.randn(2, 64, 20, 24, device=dev, dtype=torch.bfloat16)
    if nhwc:
        layer = layer.to(memory_format=torch.channels_last)
        x = x.contiguous(memory_format=torch.channels_last)
    gy = torch.randn(2, 96, 20, 24, device=dev, dtype=torch.bfloat16)

    def run():
        layer.zero_grad(set_to_none=True)
        xx = x.clone().requires_grad_(True)
        layer(xx).backward(gy)
        return [xx.grad] + [p.grad.clone() for p in layer.parameters()]

    old = _C.REUSE_PACKED_INPUT
    try:
        _C.REUSE_PACKED_INPUT = True
        a = run()
        _C.REUSE_PACKED_INPUT = False
        r = run()
    finally:
        _C.REUSE_PACKED_INPUT = old
    # input grad, weight, bias, predictor weight, predictor bias (the predictor's
    # gradients come from cuDNN and follow the atomically summed grad_input)
    for i, (u, v) in enumerate(zip(a, r)):
        e = rel_err(u.float().cpu().numpy(), v.float().cpu().numpy())
        assert e <= 1e-2, f"gradient {i}: rel err {e}"


@pytest.mark.gpu
def test_inference_weight_cache_follows_weight_versions():
    from dcnv2_b200 import _C
    from dcnv2_b200.modules import DCNv2
    case = [c for c in SMALL if c.name == "readme_small"][0]
    x, w, b, off, m, _ = _inputs(case, torch.bfloat16, False)
    dev = x.device
    layer = DCNv2(case.C, case.Co, 3, 1, 1).to(dev).to(torch.bfloat16)
    with torch.no_grad():
        layer.weight.copy_(w)
        layer.bias.copy_(b)
    _C.enable_weight_cache(True)
    try:
        with torch.no_grad():
            y0 = layer(x, off, m)
            y1 = layer(x, off, m)            # packed weight from the cache
            assert len(_C._WCACHE) == 1
            layer.weight.mul_(0.5)           # in-place update: new version
            y2 = layer(x, off, m)
            assert len(_C._WCACHE) == 2
        ref2 = _C.dcn_v2_forward(x, layer.weight.detach(), m, off, layer.bias.detach(), 1, 1, 1, 1)
        torch.cuda.synchronize()
        assert torch.equal(y0, y1)
        assert torch.equal(y2, ref2)
        assert not torch.equal(y2, y0)
    finally:
        _C.enable_weight_cache(False)
