"""Drop-in for the reference's ``Conv2d._C`` extension module (ext.cpp:15-18).

``dcn_v2_forward`` and ``dcn_v2_backward`` keep the reference's positional
signatures (name.h:15-36) and add optional trailing ``dilation_h, dilation_w,
deformable_groups`` (default 1).  Tensors are handed to ``libdcn_b200.so``
through its C ABI; outputs and the workspace come from PyTorch's caching
allocator on the tensors' device, and the work is queued on the current CUDA
stream, as the reference does (com.cu:215, 748).

Channels-last activations: when ``input`` is in PyTorch's ``channels_last``
memory format, the operator runs in the library's DCN_NHWC layout: offset, mask
(or the predictor output) and grad_output are taken channels-last (converted if
they are not), and the output and the input / offset / mask gradients are
returned channels-last, so stacked layers pass activations on without layout
passes.  Otherwise everything is NCHW-contiguous, as in the reference.

Workspace reuse (no counterpart in the reference): the functions take an
optional keyword ``workspace`` (a uint8 CUDA tensor).  ``dcn_v2_backward(...,
workspace=ws, input_packed=True)`` reuses the packed input that the forward
left in ``ws`` (allocate it with ``backward_workspace``, pass it to the forward,
keep it until the backward); the autograd functions in ``modules`` do this when
``REUSE_PACKED_INPUT`` is true (the default), holding the backward workspace
from the forward to the backward.  For inference, ``enable_weight_cache(True)``
keeps the packed weight of each (weight, version, shape, stream) in a small
cache and skips its repacking; it keys on ``weight._version``, so in-place
changes made through ``weight.data`` (which do not bump the version) must be
followed by ``clear_weight_cache()``.

Errors follow the reference: a CPU tensor raises ``RuntimeError("<name> must be a
CUDA tensor")`` (com.cu:209-213), a channel mismatch raises ``RuntimeError``
(com.cu:760-761), and a failing library call raises ``RuntimeError`` with the
library's message (com.cu:266-270).
"""
from __future__ import annotations

import collections
import ctypes
import os
from typing import List, Optional

import torch

from . import _lib

# DCN_CHECK=1: synchronise after every call and raise on device-side error bits
_CHECK = os.environ.get("DCN_CHECK", "0") not in ("", "0")

_DTYPES = {torch.float32: _lib.DCN_F32, torch.float16: _lib.DCN_F16, torch.bfloat16: _lib.DCN_BF16}


def _check_cuda(**tensors):
    """Every tensor must be a CUDA tensor (com.cu:209-213), and all on one device:
    the kernels run on the first tensor's GPU and would otherwise dereference
    another GPU's memory."""
    dev = None
    for name, t in tensors.items():
        if t is None:
            continue
        if not t.is_cuda:
            raise RuntimeError(f"{name} must be a CUDA tensor")
        if dev is None:
            dev = t.device
        elif t.device != dev:
            raise RuntimeError(f"{name} is on {t.device}, expected {dev} (all tensors on one device)")


_CL = torch.channels_last


def _is_nhwc(t) -> bool:
    """True for a 4-D tensor in PyTorch's channels_last memory format (and not
    also plain contiguous, which happens when C == 1 or H == W == 1)."""
    return t.dim() == 4 and not t.is_contiguous() and t.is_contiguous(memory_format=_CL)


def _dense(t, nhwc):
    return t.contiguous(memory_format=_CL) if nhwc else t.contiguous()


def _desc(input, weight, stride_h, stride_w, pad_h, pad_w, dil_h, dil_w, dg, has_bias, nhwc=False, flags=0):
    if input.dim() != 4 or weight.dim() != 4:
        raise RuntimeError("input and weight must be 4-D (NCHW / [Co, C, kh, kw])")
    B, C, H, W = input.shape
    Co, Cw, kh, kw = weight.shape
    if C != Cw:
        raise RuntimeError(f"Input shape and kernel channels wont match: ({C} vs {Cw}).")
    if input.dtype not in _DTYPES:
        raise RuntimeError(f"unsupported dtype {input.dtype}")
    d = _lib.DcnDesc(B, C, H, W, Co, kh, kw, int(stride_h), int(stride_w), int(pad_h), int(pad_w),
                     int(dil_h), int(dil_w), int(dg), _DTYPES[input.dtype], 1 if has_bias else 0,
                     _lib.DCN_NHWC if nhwc else _lib.DCN_NCHW, int(flags))
    Ho, Wo = ctypes.c_int32(), ctypes.c_int32()
    rc = _lib.lib.dcn_output_size(ctypes.byref(d), ctypes.byref(Ho), ctypes.byref(Wo))
    if rc != _lib.DCN_OK:
        raise RuntimeError(f"dcn: {_lib.strerror(rc)}")
    return d, Ho.value, Wo.value


def _prep(t, dtype, name, shape=None, nhwc=False):
    if t.dtype != dtype:
        raise RuntimeError(f"{name} must have dtype {dtype}, got {t.dtype}")
    if shape is not None and tuple(t.shape) != tuple(shape):
        raise RuntimeError(f"{name} has shape {tuple(t.shape)}, expected {tuple(shape)}")
    return _dense(t, nhwc)


def _ptr(t):
    return ctypes.c_void_p(t.data_ptr() if t is not None and t.numel() > 0 else 0)


def _check_device(ws):
    st = read_device_status(ws)
    if st != 0:
        raise RuntimeError(f"dcn: kernel reported device error bits {st:#x} (pipeline wait timed out)")


def _check(rc):
    if rc != _lib.DCN_OK:
        raise RuntimeError(f"dcn: {_lib.strerror(rc)}")


# backward workspace allocated by the autograd forward and handed to the backward
REUSE_PACKED_INPUT = os.environ.get("DCN_REUSE_PACKED_INPUT", "1") not in ("", "0")


def _workspace(d, backward, device, given):
    nbytes = (_lib.lib.dcn_backward_workspace_size if backward else _lib.lib.dcn_forward_workspace_size)(
        ctypes.byref(d))
    if given is None:
        return torch.empty((max(nbytes, 256),), dtype=torch.uint8, device=device)
    if given.dtype != torch.uint8 or not given.is_cuda or given.device != device or not given.is_contiguous():
        raise RuntimeError(f"workspace must be a contiguous uint8 tensor on {device}")
    if given.numel() < nbytes:
        raise RuntimeError(f"workspace has {given.numel()} bytes, {nbytes} needed")
    return given


def backward_workspace(input: torch.Tensor, weight: torch.Tensor, stride_h: int, stride_w: int,
                       pad_h: int, pad_w: int, dilation_h: int = 1, dilation_w: int = 1,
                       deformable_groups: int = 1) -> torch.Tensor:
    """A workspace that serves both the forward and the backward of this problem
    (dcn_backward_workspace_size bytes): pass it to the forward and, with
    ``input_packed=True``, to the backward."""
    d, _, _ = _desc(input, weight, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
                    deformable_groups, True, _is_nhwc(input))
    with torch.cuda.device(input.device):
        return _workspace(d, True, input.device, None)


# packed-weight cache for inference (off unless enabled)
_WCACHE_ON = os.environ.get("DCN_WEIGHT_CACHE", "0") not in ("", "0")
_WCACHE: "collections.OrderedDict" = collections.OrderedDict()
_WCACHE_MAX = 16


def enable_weight_cache(on: bool = True) -> None:
    """Turns the inference packed-weight cache on or off (and empties it)."""
    global _WCACHE_ON
    _WCACHE_ON = bool(on)
    _WCACHE.clear()


def clear_weight_cache() -> None:
    _WCACHE.clear()


def _cached_forward_ws(d, weight, stream):
    """(workspace, weight already packed in it) for an inference forward."""
    key = (weight.device.index, stream, bytes(d), weight.data_ptr(), weight._version)
    ws = _WCACHE.get(key)
    if ws is not None:
        _WCACHE.move_to_end(key)
        return ws, True
    ws = _workspace(d, False, weight.device, None)
    _WCACHE[key] = ws
    while len(_WCACHE) > _WCACHE_MAX:
        _WCACHE.popitem(last=False)
    return ws, False


def _forward_ws(d, weight, stream, given, cache_weight):
    if given is not None:
        return _workspace(d, False, weight.device, given)
    if cache_weight and _WCACHE_ON:
        ws, packed = _cached_forward_ws(d, weight, stream)
        if packed:
            d.flags |= _lib.DCN_FLAG_WEIGHT_PACKED
        return ws
    return _workspace(d, False, weight.device, None)


def dcn_v2_forward(input: torch.Tensor, weight: torch.Tensor, mask: torch.Tensor,
                   offset: torch.Tensor, bias: Optional[torch.Tensor], stride_h: int, stride_w: int,
                   pad_h: int, pad_w: int, dilation_h: int = 1, dilation_w: int = 1,
                   deformable_groups: int = 1, *, workspace: Optional[torch.Tensor] = None,
                   cache_weight: bool = False) -> torch.Tensor:
    """Output [B, Co, Ho, Wo] of modulated deformable convolution (MyDCN_forward).
    ``workspace``: optional caller-owned workspace (see ``backward_workspace``);
    ``cache_weight``: use the inference packed-weight cache when it is enabled."""
    _check_cuda(input=input, weight=weight, bias=bias, offset=offset, mask=mask)
    nhwc = _is_nhwc(input)
    d, Ho, Wo = _desc(input, weight, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
                      deformable_groups, bias is not None, nhwc)
    B, dg, K2 = input.shape[0], deformable_groups, weight.shape[2] * weight.shape[3]
    dt = input.dtype
    input = _dense(input, nhwc)
    weight = _prep(weight, dt, "weight")
    offset = _prep(offset, dt, "offset", (B, 2 * dg * K2, Ho, Wo), nhwc)
    mask = _prep(mask, dt, "mask", (B, dg * K2, Ho, Wo), nhwc)
    if bias is not None:
        bias = _prep(bias, dt, "bias", (weight.shape[0],))
    with torch.cuda.device(input.device):
        out = torch.empty((B, weight.shape[0], Ho, Wo), dtype=dt, device=input.device,
                          memory_format=_CL if nhwc else torch.contiguous_format)
        stream = torch.cuda.current_stream(input.device).cuda_stream
        ws = _forward_ws(d, weight, stream, workspace, cache_weight)
        _check(_lib.lib.dcn_forward(ctypes.byref(d), _ptr(input), _ptr(weight), _ptr(mask),
                                    _ptr(offset), _ptr(bias), _ptr(out), _ptr(ws), ws.numel(),
                                    ctypes.c_void_p(stream)))
        if _CHECK:
            _check_device(ws)
    return out


def dcn_v2_backward(input: torch.Tensor, weight: torch.Tensor, mask: torch.Tensor,
                    offset: torch.Tensor, bias: Optional[torch.Tensor], grad_output: torch.Tensor,
                    stride_h: int, stride_w: int, pad_h: int, pad_w: int, dilation_h: int = 1,
                    dilation_w: int = 1, deformable_groups: int = 1, *,
                    workspace: Optional[torch.Tensor] = None, input_packed: bool = False) -> List[torch.Tensor]:
    """[grad_input, grad_offset, grad_mask, grad_weight, grad_bias] (MyDCN_backward order).
    ``input_packed``: ``workspace`` went through the forward of this input and
    still holds its packed copy (DCN_FLAG_INPUT_PACKED)."""
    _check_cuda(input=input, weight=weight, bias=bias, offset=offset, mask=mask,
                grad_output=grad_output)
    has_bias = bias is not None
    nhwc = _is_nhwc(input)
    d, Ho, Wo = _desc(input, weight, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
                      deformable_groups, True, nhwc,
                      _lib.DCN_FLAG_INPUT_PACKED if input_packed else 0)
    B, dg, K2 = input.shape[0], deformable_groups, weight.shape[2] * weight.shape[3]
    Co = weight.shape[0]
    dt = input.dtype
    input = _dense(input, nhwc)
    weight = _prep(weight, dt, "weight")
    offset = _prep(offset, dt, "offset", (B, 2 * dg * K2, Ho, Wo), nhwc)
    mask = _prep(mask, dt, "mask", (B, dg * K2, Ho, Wo), nhwc)
    grad_output = _prep(grad_output, dt, "grad_output", (B, Co, Ho, Wo), nhwc)
    with torch.cuda.device(input.device):
        gi = torch.empty_like(input)
        goff = torch.empty_like(offset)
        gm = torch.empty_like(mask)
        gw = torch.empty_like(weight)
        gb = torch.empty((Co,), dtype=dt, device=input.device)
        if input_packed and workspace is None:
            raise RuntimeError("input_packed=True needs the workspace the forward used")
        ws = _workspace(d, True, input.device, workspace)
        stream = torch.cuda.current_stream(input.device).cuda_stream
        _check(_lib.lib.dcn_backward(ctypes.byref(d), _ptr(input), _ptr(weight), _ptr(mask),
                                     _ptr(offset), _ptr(bias), _ptr(grad_output), _ptr(gi),
                                     _ptr(goff), _ptr(gm), _ptr(gw), _ptr(gb), _ptr(ws),
                                     ws.numel(), ctypes.c_void_p(stream)))
        if _CHECK:
            _check_device(ws)
    return [gi, goff, gm, gw, gb if has_bias else None]


def dcn_v2_forward_om(input: torch.Tensor, weight: torch.Tensor, offset_mask: torch.Tensor,
                      bias: Optional[torch.Tensor], stride_h: int, stride_w: int, pad_h: int, pad_w: int,
                      dilation_h: int = 1, dilation_w: int = 1, deformable_groups: int = 1, *,
                      workspace: Optional[torch.Tensor] = None, cache_weight: bool = False) -> torch.Tensor:
    """Forward fed by the raw predictor output [B, 3*dg*K2, Ho, Wo]: offsets in the
    first 2*dg*K2 channels, mask logits (sigmoid applied in the kernel) in the rest;
    the same result as ``dcn_v2_forward`` with the reference module's chunk / cat /
    sigmoid (dcn_v2_mm.py:133-137) done in the operator."""
    _check_cuda(input=input, weight=weight, bias=bias, offset_mask=offset_mask)
    nhwc = _is_nhwc(input)
    d, Ho, Wo = _desc(input, weight, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
                      deformable_groups, bias is not None, nhwc)
    B, dg, K2 = input.shape[0], deformable_groups, weight.shape[2] * weight.shape[3]
    dt = input.dtype
    input = _dense(input, nhwc)
    weight = _prep(weight, dt, "weight")
    offset_mask = _prep(offset_mask, dt, "offset_mask", (B, 3 * dg * K2, Ho, Wo), nhwc)
    if bias is not None:
        bias = _prep(bias, dt, "bias", (weight.shape[0],))
    with torch.cuda.device(input.device):
        out = torch.empty((B, weight.shape[0], Ho, Wo), dtype=dt, device=input.device,
                          memory_format=_CL if nhwc else torch.contiguous_format)
        stream = torch.cuda.current_stream(input.device).cuda_stream
        ws = _forward_ws(d, weight, stream, workspace, cache_weight)
        _check(_lib.lib.dcn_forward_om(ctypes.byref(d), _ptr(input), _ptr(weight), _ptr(offset_mask),
                                       _ptr(bias), _ptr(out), _ptr(ws), ws.numel(), ctypes.c_void_p(stream)))
        if _CHECK:
            _check_device(ws)
    return out


def dcn_v2_backward_om(input: torch.Tensor, weight: torch.Tensor, offset_mask: torch.Tensor,
                       bias: Optional[torch.Tensor], grad_output: torch.Tensor, stride_h: int,
                       stride_w: int, pad_h: int, pad_w: int, dilation_h: int = 1, dilation_w: int = 1,
                       deformable_groups: int = 1, *, workspace: Optional[torch.Tensor] = None,
                       input_packed: bool = False) -> List[torch.Tensor]:
    """[grad_input, grad_offset_mask, grad_weight, grad_bias] of ``dcn_v2_forward_om``;
    grad_offset_mask holds the offset gradients and the mask-logit gradients."""
    _check_cuda(input=input, weight=weight, bias=bias, offset_mask=offset_mask, grad_output=grad_output)
    has_bias = bias is not None
    nhwc = _is_nhwc(input)
    d, Ho, Wo = _desc(input, weight, stride_h, stride_w, pad_h, pad_w, dilation_h, dilation_w,
                      deformable_groups, True, nhwc,
                      _lib.DCN_FLAG_INPUT_PACKED if input_packed else 0)
    B, dg, K2 = input.shape[0], deformable_groups, weight.shape[2] * weight.shape[3]
    Co = weight.shape[0]
    dt = input.dtype
    input = _dense(input, nhwc)
    weight = _prep(weight, dt, "weight")
    offset_mask = _prep(offset_mask, dt, "offset_mask", (B, 3 * dg * K2, Ho, Wo), nhwc)
    grad_output = _prep(grad_output, dt, "grad_output", (B, Co, Ho, Wo), nhwc)
    with torch.cuda.device(input.device):
        gi = torch.empty_like(input)
        gom = torch.empty_like(offset_mask)
        gw = torch.empty_like(weight)
        gb = torch.empty((Co,), dtype=dt, device=input.device)
        if input_packed and workspace is None:
            raise RuntimeError("input_packed=True needs the workspace the forward used")
        ws = _workspace(d, True, input.device, workspace)
        stream = torch.cuda.current_stream(input.device).cuda_stream
        _check(_lib.lib.dcn_backward_om(ctypes.byref(d), _ptr(input), _ptr(weight), _ptr(offset_mask),
                                        _ptr(bias), _ptr(grad_output), _ptr(gi), _ptr(gom), _ptr(gw),
                                        _ptr(gb), _ptr(ws), ws.numel(), ctypes.c_void_p(stream)))
        if _CHECK:
            _check_device(ws)
    return [gi, gom, gw, gb if has_bias else None]


def read_device_status(workspace: torch.Tensor) -> int:
    """Synchronises the current stream and returns (and clears) the device error bits."""
    stream = torch.cuda.current_stream(workspace.device).cuda_stream
    return int(_lib.lib.dcn_read_device_status(_ptr(workspace), ctypes.c_void_p(stream)))
