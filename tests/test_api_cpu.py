"""Host-side behaviour of the Conv2d._C-compatible ops and the modules
(reference dcn_v2_mm.py / com.cu error paths), without a GPU."""
import pytest
import torch

from dcnv2_b200 import DCN, DCNv2, _C, dcn_v2_conv


def _cpu_inputs():
    x = torch.randn(1, 4, 5, 5)
    w = torch.randn(6, 4, 3, 3)
    b = torch.zeros(6)
    off = torch.zeros(1, 18, 5, 5)
    m = torch.ones(1, 9, 5, 5)
    return x, w, m, off, b


def test_cpu_tensor_rejected_like_reference():
    x, w, m, off, b = _cpu_inputs()
    with pytest.raises(RuntimeError, match="input must be a CUDA tensor"):
        _C.dcn_v2_forward(x, w, m, off, b, 1, 1, 1, 1)
    with pytest.raises(RuntimeError, match="must be a CUDA tensor"):
        _C.dcn_v2_backward(x, w, m, off, b, torch.zeros(1, 6, 5, 5), 1, 1, 1, 1)


def test_module_parameters_match_reference_layout():
    mod = DCN(16, 32, kernel_size=3, stride=1, padding=1, deformable_groups=2)
    sd = mod.state_dict()
    assert set(sd) == {"weight", "bias", "conv_offset_mask.weight", "conv_offset_mask.bias"}
    assert sd["weight"].shape == (32, 16, 3, 3)
    assert sd["bias"].shape == (32,)
    assert sd["conv_offset_mask.weight"].shape == (2 * 3 * 9, 16, 3, 3)
    assert float(sd["conv_offset_mask.weight"].abs().sum()) == 0.0
    assert float(sd["bias"].abs().sum()) == 0.0
    bound = 1.0 / (16 * 9) ** 0.5
    assert float(sd["weight"].abs().max()) <= bound


def test_dcnv2_asserts_offset_mask_channels():
    mod = DCNv2(4, 6, 3, 1, 1)
    x, w, m, off, b = _cpu_inputs()
    with pytest.raises(AssertionError):
        mod(x, off[:, :9], m)
    with pytest.raises(AssertionError):
        mod(x, off, m[:, :4])


def test_autograd_function_is_exposed():
    assert callable(dcn_v2_conv)
