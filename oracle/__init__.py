"""CPU oracle for DCNv2 -- TEST INFRASTRUCTURE, never on the product path.

Thin ctypes wrapper over ``oracle/dcn_oracle.c`` (a plain-C restatement of the
reference operator's arithmetic; the C file lists the reference lines it follows).
Only ``tests/``, ``__graft_entry__.smoke()`` (as the checker) and ``bench.py``'s CPU
baseline / reference arm may import this package.

Parity pinning: the restatement is checked against (i) golden vectors produced by
the reference's own CUDA kernels on a B200 (``tests/golden/make_ref_golden.py``)
and (ii) ``torchvision.ops.deform_conv2d`` in float64 (``tests/golden/make_tv_golden.py``),
the same math for dilation > 1 and deformable groups > 1, which the reference kernels
do not implement.
"""
from __future__ import annotations

import ctypes
import os
import subprocess

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
_LIB_PATH = os.path.join(_HERE, "libdcn_oracle.so")
_lib = None


def build() -> str:
    """Compile the C oracle in place (``make -C oracle``); returns the library path."""
    subprocess.run(["make", "-s", "-C", _HERE], check=True)
    return _LIB_PATH


def _load():
    global _lib
    if _lib is not None:
        return _lib
    if not os.path.exists(_LIB_PATH) or os.path.getmtime(_LIB_PATH) < os.path.getmtime(
        os.path.join(_HERE, "dcn_oracle.c")
    ):
        build()
    lib = ctypes.CDLL(_LIB_PATH)
    for sfx, ct in (("f64", ctypes.c_double), ("f32", ctypes.c_float)):
        p = ctypes.POINTER(ct)
        ip = ctypes.POINTER(ctypes.c_int)
        f = getattr(lib, f"dcn_oracle_forward_{sfx}")
        f.argtypes = [p, p, p, p, p, p, ip]
        f.restype = None
        g = getattr(lib, f"dcn_oracle_backward_{sfx}")
        g.argtypes = [p, p, p, p, p, p, p, p, p, p, ip]
        g.restype = None
    lib.dcn_oracle_num_threads.restype = ctypes.c_int
    lib.dcn_oracle_set_coord_f32.argtypes = [ctypes.c_int]
    lib.dcn_oracle_set_coord_f32.restype = None
    lib.dcn_oracle_set_threads.argtypes = [ctypes.c_int]
    lib.dcn_oracle_set_threads.restype = None
    _lib = lib
    return lib


def num_threads() -> int:
    return int(_load().dcn_oracle_num_threads())


def set_threads(n: int) -> None:
    """Threads of the float32 CPU port (OpenMP)."""
    _load().dcn_oracle_set_threads(int(n))


def out_size(n: int, k: int, s: int, p: int, d: int) -> int:
    return (n + 2 * p - (d * (k - 1) + 1)) // s + 1


def _pair(v):
    return (v, v) if isinstance(v, int) else tuple(v)


def _shape(x, w, stride, padding, dilation, dg):
    B, C, H, W = x.shape
    Co, Cw, kh, kw = w.shape
    assert Cw == C, "weight in-channels must equal input channels"
    sh, sw = _pair(stride)
    ph, pw = _pair(padding)
    dh, dw = _pair(dilation)
    return np.array([B, C, H, W, Co, kh, kw, sh, sw, ph, pw, dh, dw, dg], dtype=np.int32)


def _np(a, dt):
    return np.ascontiguousarray(np.asarray(a, dtype=dt))


def forward(x, weight, bias, offset, mask, stride=1, padding=0, dilation=1, deformable_groups=1,
            dtype=np.float64, coord="f32"):
    """y = DCNv2(x; offset, mask, weight, bias) in ``dtype`` (float64 or float32).
    ``coord="f32"`` forms sample positions in float32 as the reference does;
    ``"f64"`` in ``dtype`` (torchvision's double kernels)."""
    lib = _load()
    lib.dcn_oracle_set_coord_f32(1 if coord == "f32" else 0)
    sfx = "f64" if dtype == np.float64 else "f32"
    ct = ctypes.c_double if sfx == "f64" else ctypes.c_float
    x, weight, offset, mask = (_np(a, dtype) for a in (x, weight, offset, mask))
    bias = None if bias is None else _np(bias, dtype)
    shp = _shape(x, weight, stride, padding, dilation, deformable_groups)
    Ho = out_size(shp[2], shp[5], shp[7], shp[9], shp[11])
    Wo = out_size(shp[3], shp[6], shp[8], shp[10], shp[12])
    y = np.zeros((shp[0], shp[4], Ho, Wo), dtype=dtype)
    P = lambda a: None if a is None else a.ctypes.data_as(ctypes.POINTER(ct))  # noqa: E731
    getattr(lib, f"dcn_oracle_forward_{sfx}")(
        P(x), P(weight), P(bias), P(offset), P(mask), P(y),
        shp.ctypes.data_as(ctypes.POINTER(ctypes.c_int)))
    return y


def backward(x, weight, offset, mask, grad_out, stride=1, padding=0, dilation=1,
             deformable_groups=1, dtype=np.float64, coord="f32"):
    """Returns (grad_input, grad_offset, grad_mask, grad_weight, grad_bias), the
    order of the reference's ``dcn_v2_backward`` (com.cu:845-847).  ``coord`` as
    in ``forward``."""
    lib = _load()
    lib.dcn_oracle_set_coord_f32(1 if coord == "f32" else 0)
    sfx = "f64" if dtype == np.float64 else "f32"
    ct = ctypes.c_double if sfx == "f64" else ctypes.c_float
    x, weight, offset, mask, grad_out = (_np(a, dtype) for a in (x, weight, offset, mask, grad_out))
    shp = _shape(x, weight, stride, padding, dilation, deformable_groups)
    gx = np.zeros_like(x)
    goff = np.zeros_like(offset)
    gmask = np.zeros_like(mask)
    gw = np.zeros_like(weight)
    gb = np.zeros((weight.shape[0],), dtype=dtype)
    P = lambda a: a.ctypes.data_as(ctypes.POINTER(ct))  # noqa: E731
    getattr(lib, f"dcn_oracle_backward_{sfx}")(
        P(x), P(weight), P(offset), P(mask), P(grad_out), P(gx), P(goff), P(gmask), P(gw), P(gb),
        shp.ctypes.data_as(ctypes.POINTER(ctypes.c_int)))
    return gx, goff, gmask, gw, gb
