"""User-facing DCNv2 modules, API-compatible with the reference's dcn_v2_mm.py.

``_DCNv2`` / ``dcn_v2_conv`` / ``DCNv2`` / ``DCN`` keep the reference's names,
constructor arguments, parameter names and shapes (dcn_v2_mm.py:15-146), so
reference checkpoints load unchanged.  Unlike the reference, ``dilation`` and
``deformable_groups`` are forwarded to the operator (the reference stores them
but never passes them on, dcn_v2_mm.py:76-77, 94-102).
"""
from __future__ import annotations

import math

import torch
from torch import nn
from torch.autograd import Function
from torch.autograd.function import once_differentiable
from torch.nn.modules.utils import _pair

from . import _C


def _forward_workspace(ctx, input, weight):
    """Workspace for an autograd forward: the backward's, allocated now and kept
    on ctx, so that the backward reuses the input the forward packed into it
    (DCN_FLAG_INPUT_PACKED); None (a fresh forward-only workspace per call) when
    the reuse is switched off."""
    if _C.REUSE_PACKED_INPUT:
        return _C.backward_workspace(input, weight, ctx.stride[0], ctx.stride[1], ctx.padding[0],
                                     ctx.padding[1], ctx.dilation[0], ctx.dilation[1],
                                     ctx.deformable_groups)
    return None


class _DCNv2(Function):
    """Autograd glue (dcn_v2_mm.py:15-53); argument order input, weight, mask, offset, bias."""

    @staticmethod
    def forward(ctx, input, weight, mask, offset, bias, stride, padding, dilation=1,
                deformable_groups=1):
        ctx.stride = _pair(stride)
        ctx.padding = _pair(padding)
        ctx.dilation = _pair(dilation)
        ctx.deformable_groups = int(deformable_groups)
        ws = _forward_workspace(ctx, input, weight)
        output = _C.dcn_v2_forward(input, weight, mask, offset, bias, ctx.stride[0], ctx.stride[1],
                                   ctx.padding[0], ctx.padding[1], ctx.dilation[0],
                                   ctx.dilation[1], ctx.deformable_groups, workspace=ws)
        ctx.ws = ws
        ctx.save_for_backward(input, weight, mask, offset, bias)
        return output

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        input, weight, mask, offset, bias = ctx.saved_tensors
        ws, ctx.ws = ctx.ws, None
        grad_input, grad_offset, grad_mask, grad_weight, grad_bias = _C.dcn_v2_backward(
            input, weight, mask, offset, bias, grad_output, ctx.stride[0], ctx.stride[1],
            ctx.padding[0], ctx.padding[1], ctx.dilation[0], ctx.dilation[1],
            ctx.deformable_groups, workspace=ws, input_packed=ws is not None)
        return (grad_input, grad_weight, grad_mask, grad_offset, grad_bias, None, None, None, None)


dcn_v2_conv = _DCNv2.apply


class _DCNv2OM(Function):
    """Autograd glue of the fused predictor path: input, weight, the predictor's raw
    output (offsets, then mask logits) and bias; the gradient of the raw output goes
    straight back into the predictor conv."""

    @staticmethod
    def forward(ctx, input, weight, offset_mask, bias, stride, padding, dilation=1,
                deformable_groups=1):
        ctx.stride = _pair(stride)
        ctx.padding = _pair(padding)
        ctx.dilation = _pair(dilation)
        ctx.deformable_groups = int(deformable_groups)
        ws = _forward_workspace(ctx, input, weight)
        output = _C.dcn_v2_forward_om(input, weight, offset_mask, bias, ctx.stride[0], ctx.stride[1],
                                      ctx.padding[0], ctx.padding[1], ctx.dilation[0], ctx.dilation[1],
                                      ctx.deformable_groups, workspace=ws)
        ctx.ws = ws
        ctx.save_for_backward(input, weight, offset_mask, bias)
        return output

    @staticmethod
    @once_differentiable
    def backward(ctx, grad_output):
        input, weight, offset_mask, bias = ctx.saved_tensors
        ws, ctx.ws = ctx.ws, None
        grad_input, grad_om, grad_weight, grad_bias = _C.dcn_v2_backward_om(
            input, weight, offset_mask, bias, grad_output, ctx.stride[0], ctx.stride[1],
            ctx.padding[0], ctx.padding[1], ctx.dilation[0], ctx.dilation[1], ctx.deformable_groups,
            workspace=ws, input_packed=ws is not None)
        return (grad_input, grad_weight, grad_om, grad_bias, None, None, None, None)


dcn_v2_conv_om = _DCNv2OM.apply


class DCNv2(nn.Module):
    """Modulated deformable conv taking external offset and mask (dcn_v2_mm.py:59-102)."""

    def __init__(self, in_channels, out_channels, kernel_size, stride, padding, dilation=1,
                 deformable_groups=1):
        super().__init__()
        self.in_channels = in_channels
        self.out_channels = out_channels
        self.kernel_size = _pair(kernel_size)
        self.stride = _pair(stride)
        self.padding = _pair(padding)
        self.dilation = _pair(dilation)
        self.deformable_groups = deformable_groups
        self.weight = nn.Parameter(torch.Tensor(out_channels, in_channels, *self.kernel_size))
        self.bias = nn.Parameter(torch.Tensor(out_channels))
        self.reset_parameters()

    def reset_parameters(self):
        n = self.in_channels
        for k in self.kernel_size:
            n *= k
        stdv = 1.0 / math.sqrt(n)
        self.weight.data.uniform_(-stdv, stdv)
        self.bias.data.zero_()

    def forward(self, input, offset, mask):
        k2 = self.kernel_size[0] * self.kernel_size[1]
        assert 2 * self.deformable_groups * k2 == offset.shape[1]
        assert self.deformable_groups * k2 == mask.shape[1]
        if not torch.is_grad_enabled():
            # inference: no autograd record, and the packed-weight cache when enabled
            return _C.dcn_v2_forward(input, self.weight, mask, offset, self.bias, self.stride[0],
                                     self.stride[1], self.padding[0], self.padding[1], self.dilation[0],
                                     self.dilation[1], self.deformable_groups, cache_weight=True)
        return dcn_v2_conv(input, self.weight, mask, offset, self.bias, self.stride, self.padding,
                           self.dilation, self.deformable_groups)


class DCN(DCNv2):
    """DCNv2 with its own offset/mask predictor conv (dcn_v2_mm.py:105-146)."""

    def __init__(self, in_channels, out_channels, kernel_size, stride=1, padding=0, dilation=1,
                 deformable_groups=1):
        super().__init__(in_channels, out_channels, kernel_size, stride, padding, dilation,
                         deformable_groups)
        channels_ = self.deformable_groups * 3 * self.kernel_size[0] * self.kernel_size[1]
        self.conv_offset_mask = nn.Conv2d(self.in_channels, channels_,
                                          kernel_size=self.kernel_size, stride=self.stride,
                                          padding=self.padding, dilation=self.dilation, bias=True)
        self.init_offset()

    def init_offset(self):
        self.conv_offset_mask.weight.data.zero_()
        self.conv_offset_mask.bias.data.zero_()

    def forward(self, input):
        # the predictor's output goes to the operator as it is: the reference's
        # chunk / cat / sigmoid (dcn_v2_mm.py:133-137) happen inside the kernels
        out = self.conv_offset_mask(input)
        if not torch.is_grad_enabled():
            return _C.dcn_v2_forward_om(input, self.weight, out, self.bias, self.stride[0], self.stride[1],
                                        self.padding[0], self.padding[1], self.dilation[0],
                                        self.dilation[1], self.deformable_groups, cache_weight=True)
        return dcn_v2_conv_om(input, self.weight, out, self.bias, self.stride, self.padding,
                              self.dilation, self.deformable_groups)
