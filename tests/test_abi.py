"""The C ABI library loads, exports every function include/dcn_b200.h declares,
and validates descriptors on the host (no GPU needed)."""
import ctypes
import os
import re

import pytest

from dcnv2_b200 import _lib

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))


def _declared():
    txt = open(os.path.join(ROOT, "include", "dcn_b200.h")).read()
    return re.findall(r"DCN_API\s+[\w\s\*]+?\b(dcn_\w+)\s*\(", txt)


def test_header_symbols_exported():
    names = _declared()
    assert len(names) >= 8
    assert set(names) == set(_lib.EXPORTS)
    for n in names:
        assert hasattr(_lib.lib, n), n


def _desc(**kw):
    d = dict(B=8, C=64, H=128, W=128, Co=256, kh=3, kw=3, sh=1, sw=1, ph=1, pw=1, dh=1, dw=1, dg=1,
             dtype=_lib.DCN_BF16, has_bias=1)
    d.update(kw)
    return _lib.DcnDesc(**d)


def test_output_size_and_workspace():
    d = _desc()
    ho, wo = ctypes.c_int32(), ctypes.c_int32()
    assert _lib.lib.dcn_output_size(ctypes.byref(d), ctypes.byref(ho), ctypes.byref(wo)) == 0
    assert (ho.value, wo.value) == (128, 128)
    d2 = _desc(H=97, W=131, kh=5, kw=5, sh=2, sw=2, ph=4, pw=4, dh=2, dw=2, dg=2, C=96, Co=160)
    assert _lib.lib.dcn_output_size(ctypes.byref(d2), ctypes.byref(ho), ctypes.byref(wo)) == 0
    assert (ho.value, wo.value) == ((97 + 8 - 9) // 2 + 1, (131 + 8 - 9) // 2 + 1)
    f = _lib.lib.dcn_forward_workspace_size(ctypes.byref(d))
    b = _lib.lib.dcn_backward_workspace_size(ctypes.byref(d))
    # packed NHWC bf16 input (16.8 MB) at least; backward adds fp32 grad_input accumulator
    assert f >= 8 * 128 * 128 * 64 * 2 and b >= f + 8 * 128 * 128 * 64 * 4


@pytest.mark.parametrize("bad", [dict(C=63, dg=2), dict(kh=0), dict(sh=0), dict(dh=0), dict(dg=0),
                                 dict(dtype=7), dict(H=1, W=1, ph=0, pw=0), dict(Co=0), dict(layout=2),
                                 dict(flags=4), dict(flags=-1)])
def test_invalid_descriptors(bad):
    d = _desc(**bad)
    ho, wo = ctypes.c_int32(), ctypes.c_int32()
    assert _lib.lib.dcn_output_size(ctypes.byref(d), ctypes.byref(ho), ctypes.byref(wo)) < 0
    assert _lib.lib.dcn_forward_workspace_size(ctypes.byref(d)) == 0
    rc = _lib.lib.dcn_forward(ctypes.byref(d), None, None, None, None, None, None, None, 0, None)
    assert rc == -1


def test_null_and_workspace_errors():
    d = _desc()
    rc = _lib.lib.dcn_forward(ctypes.byref(d), None, None, None, None, None, None, None, 0, None)
    assert rc == -2  # DCN_E_NULLPTR (no workspace)
    rc = _lib.lib.dcn_forward(ctypes.byref(d), None, None, None, None, None, None,
                              ctypes.c_void_p(256), 16, None)
    assert rc == -3  # DCN_E_WORKSPACE (too small)


def test_strerror_and_version():
    assert "workspace" in _lib.strerror(-3)
    assert _lib.strerror(12345) == "unknown error"
    assert "sm_100a" in _lib.version()


def test_trace_collect_empty():
    _lib.trace_reset()
    assert _lib.trace_collect() == {}


def test_descriptor_layout_field():
    """dcn_desc ends with the layout and flags fields (18 int32); NCHW and NHWC
    give the same output size and workspace."""
    assert ctypes.sizeof(_lib.DcnDesc) == 18 * 4
    a, b = _desc(layout=_lib.DCN_NCHW), _desc(layout=_lib.DCN_NHWC)
    assert _lib.lib.dcn_forward_workspace_size(ctypes.byref(a)) == _lib.lib.dcn_forward_workspace_size(ctypes.byref(b))
    assert _lib.lib.dcn_backward_workspace_size(ctypes.byref(a)) == _lib.lib.dcn_backward_workspace_size(ctypes.byref(b))
