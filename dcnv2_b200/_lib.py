"""ctypes binding of ``libdcn_b200.so`` (the C ABI in ``include/dcn_b200.h``).

The library must exist: there is no fallback.  Importing this module on a machine
without the built library raises ``ImportError`` with the build command.
"""
from __future__ import annotations

import ctypes
import os

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "libdcn_b200.so")

DCN_F32, DCN_F16, DCN_BF16 = 0, 1, 2
DCN_NCHW, DCN_NHWC = 0, 1
# dcn_desc.flags bits
DCN_FLAG_INPUT_PACKED, DCN_FLAG_WEIGHT_PACKED = 1, 2
DCN_OK = 0
DCN_E_SCRATCH_LIMIT = -7
NOALLOC_SCRATCH_BYTES = 48 << 20
DCN_DEVERR_TIMEOUT = 1

# every exported symbol of include/dcn_b200.h
EXPORTS = (
    "dcn_output_size",
    "dcn_forward_workspace_size",
    "dcn_backward_workspace_size",
    "dcn_forward",
    "dcn_backward",
    "dcn_forward_om",
    "dcn_backward_om",
    "dcn_read_device_status",
    "dcn_strerror",
    "dcn_version",
    "dcn_trace_enable",
    "dcn_trace_collect",
    "dcn_trace_reset",
    "dcn_forward_noalloc",
)


class DcnDesc(ctypes.Structure):
    """Mirror of ``struct dcn_desc``."""

    _fields_ = [(n, ctypes.c_int32) for n in (
        "B", "C", "H", "W", "Co", "kh", "kw", "sh", "sw", "ph", "pw", "dh", "dw", "dg",
        "dtype", "has_bias", "layout", "flags")]


class TraceEntry(ctypes.Structure):
    """Mirror of ``struct dcn_trace_entry``."""

    _fields_ = [("name", ctypes.c_char_p), ("launches", ctypes.c_int64), ("total_ms", ctypes.c_double)]


def _load() -> ctypes.CDLL:
    if not os.path.exists(LIB_PATH):
        raise ImportError(
            f"{LIB_PATH} is missing: build it with `python dcnv2_b200/build.py` "
            "(the DCNv2 operator has no fallback implementation)")
    lib = ctypes.CDLL(LIB_PATH)
    vp, sz, i32p = ctypes.c_void_p, ctypes.c_size_t, ctypes.POINTER(ctypes.c_int32)
    dp = ctypes.POINTER(DcnDesc)
    lib.dcn_output_size.argtypes = [dp, i32p, i32p]
    lib.dcn_output_size.restype = ctypes.c_int
    lib.dcn_forward_workspace_size.argtypes = [dp]
    lib.dcn_forward_workspace_size.restype = sz
    lib.dcn_backward_workspace_size.argtypes = [dp]
    lib.dcn_backward_workspace_size.restype = sz
    lib.dcn_forward.argtypes = [dp, vp, vp, vp, vp, vp, vp, vp, sz, vp]
    lib.dcn_forward.restype = ctypes.c_int
    lib.dcn_backward.argtypes = [dp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, sz, vp]
    lib.dcn_backward.restype = ctypes.c_int
    lib.dcn_forward_om.argtypes = [dp, vp, vp, vp, vp, vp, vp, sz, vp]
    lib.dcn_forward_om.restype = ctypes.c_int
    lib.dcn_backward_om.argtypes = [dp, vp, vp, vp, vp, vp, vp, vp, vp, vp, vp, sz, vp]
    lib.dcn_backward_om.restype = ctypes.c_int
    lib.dcn_read_device_status.argtypes = [vp, vp]
    lib.dcn_read_device_status.restype = ctypes.c_int
    lib.dcn_strerror.argtypes = [ctypes.c_int]
    lib.dcn_strerror.restype = ctypes.c_char_p
    lib.dcn_trace_enable.argtypes = [ctypes.c_int]
    lib.dcn_trace_enable.restype = ctypes.c_int
    lib.dcn_trace_collect.argtypes = [ctypes.POINTER(TraceEntry), ctypes.c_int]
    lib.dcn_trace_collect.restype = ctypes.c_int
    lib.dcn_trace_reset.argtypes = []
    lib.dcn_trace_reset.restype = ctypes.c_int
    lib.dcn_forward_noalloc.argtypes = [dp, vp, vp, vp, vp, vp, vp, vp]
    lib.dcn_forward_noalloc.restype = ctypes.c_int
    lib.dcn_version.argtypes = []
    lib.dcn_version.restype = ctypes.c_char_p
    return lib


lib = _load()


def strerror(code: int) -> str:
    return lib.dcn_strerror(int(code)).decode()


def version() -> str:
    return lib.dcn_version().decode()


def trace_enable(on: bool) -> None:
    lib.dcn_trace_enable(1 if on else 0)


def trace_reset() -> None:
    lib.dcn_trace_reset()


def trace_collect() -> dict:
    """Synchronises the traced events; returns {kernel: (launches, total_ms)}."""
    buf = (TraceEntry * 32)()
    n = lib.dcn_trace_collect(buf, 32)
    if n < 0:
        raise RuntimeError(f"dcn_trace_collect: {strerror(n)}")
    return {buf[i].name.decode(): (int(buf[i].launches), float(buf[i].total_ms)) for i in range(n)}
