"""PyTorch integration of the depthwise 3x3 kernels: custom ops with autograd,
and an ``nn.Conv2d(groups=C)`` stand-in for channels-last models.

* ``torch.ops.tdc.dwconv3x3(x_nhwc, w_rsc, pad)`` — forward (C % 8), with
  ``torch.ops.tdc.dwconv3x3_bwd_data`` / ``torch.ops.tdc.dwconv3x3_bwd_weight``
  registered as its autograd formula (data gradient: the same kernel with
  flipped taps; weight gradient: a deterministic reduction kernel).  All three
  have fake implementations, so they trace under ``torch.compile``.
* ``DepthwiseConv3x3`` — a module with ``nn.Conv2d(C, C, 3, padding=p,
  groups=C, bias=...)``'s parameters and NCHW interface.  A channels-last
  NCHW tensor is NHWC in memory, so it runs on the kernels without a copy.
* ``convert_depthwise_convs(model)`` — swaps every eligible ``nn.Conv2d``
  (3x3, stride 1, dilation 1, groups = in = out channels, symmetric integer
  padding, zeros padding mode) for a ``DepthwiseConv3x3`` sharing its
  parameters.

The reference (haowen-han/tma-depthwise-conv) has a forward-only Python API
(``tma_dwconv.py``); everything here is beyond that surface and is built on
the same kernels.
"""
from __future__ import annotations

import torch
from torch import nn

import _tma_dwconv_C as _C  # type: ignore


def _out_hw(h: int, w: int, pad: int) -> tuple[int, int]:
    return h + 2 * pad - 2, w + 2 * pad - 2


@torch.library.custom_op("tdc::dwconv3x3", mutates_args=())
def dwconv3x3_op(x: torch.Tensor, w: torch.Tensor, pad: int) -> torch.Tensor:
    """Depthwise 3x3 forward: x [N,H,W,C] fp16, w [3,3,C] fp16 -> [N,P,Q,C]."""
    return _C.dwconv3x3(x.contiguous(), w.contiguous(), None, None, pad, 0, 2)


@dwconv3x3_op.register_fake
def _(x, w, pad):
    p, q = _out_hw(x.shape[1], x.shape[2], pad)
    return x.new_empty((x.shape[0], p, q, x.shape[3]))


@torch.library.custom_op("tdc::dwconv3x3_bwd_data", mutates_args=())
def dwconv3x3_bwd_data_op(dy: torch.Tensor, w: torch.Tensor, pad: int) -> torch.Tensor:
    """dx [N,H,W,C] of the forward, from dy [N,P,Q,C]."""
    return _C.dwconv3x3_bwd_data(dy.contiguous(), w.contiguous(), pad, 2)


@dwconv3x3_bwd_data_op.register_fake
def _(dy, w, pad):
    return dy.new_empty((dy.shape[0], dy.shape[1] - 2 * pad + 2, dy.shape[2] - 2 * pad + 2,
                         dy.shape[3]))


@torch.library.custom_op("tdc::dwconv3x3_bwd_weight", mutates_args=())
def dwconv3x3_bwd_weight_op(x: torch.Tensor, dy: torch.Tensor, pad: int) -> torch.Tensor:
    """dw [3,3,C] (fp32) of the forward, from x [N,H,W,C] and dy [N,P,Q,C]."""
    return _C.dwconv3x3_bwd_weight(x.contiguous(), dy.contiguous(), pad, 2)


@dwconv3x3_bwd_weight_op.register_fake
def _(x, dy, pad):
    return x.new_empty((3, 3, x.shape[3]), dtype=torch.float32)


def _setup_context(ctx, inputs, output):
    x, w, pad = inputs
    ctx.save_for_backward(x, w)
    ctx.pad = pad


def _backward(ctx, dy):
    x, w = ctx.saved_tensors
    dx = dw = None
    if ctx.needs_input_grad[0]:
        dx = dwconv3x3_bwd_data_op(dy, w, ctx.pad)
    if ctx.needs_input_grad[1]:
        dw = dwconv3x3_bwd_weight_op(x, dy, ctx.pad).to(w.dtype)
    return dx, dw, None


dwconv3x3_op.register_autograd(_backward, setup_context=_setup_context)


def dwconv3x3(x_nhwc: torch.Tensor, w_rsc: torch.Tensor, pad: int = 1) -> torch.Tensor:
    """Differentiable depthwise 3x3 (stride 1) on NHWC fp16 tensors."""
    return dwconv3x3_op(x_nhwc, w_rsc, int(pad))


class DepthwiseConv3x3(nn.Module):
    """``nn.Conv2d(C, C, 3, stride=1, padding=pad, groups=C, bias=bias)`` for
    fp16 channels-last NCHW inputs (NHWC memory), on the sm_100a kernels.

    Parameters keep ``nn.Conv2d``'s layout (weight [C, 1, 3, 3], bias [C]), so
    state dicts load unchanged.  Inputs that are not fp16 CUDA tensors in
    channels-last layout are converted (one copy).
    """

    def __init__(self, channels: int, padding: int = 1, bias: bool = True,
                 device=None, dtype=torch.float16):
        super().__init__()
        self.channels = channels
        self.padding = int(padding)
        self.weight = nn.Parameter(torch.empty(channels, 1, 3, 3, device=device, dtype=dtype))
        self.bias = nn.Parameter(torch.empty(channels, device=device, dtype=dtype)) if bias else None
        nn.init.kaiming_uniform_(self.weight, a=5 ** 0.5)
        if self.bias is not None:
            nn.init.uniform_(self.bias, -1.0 / 3.0, 1.0 / 3.0)

    @classmethod
    def from_conv2d(cls, conv: nn.Conv2d) -> "DepthwiseConv3x3":
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        m.channels = conv.in_channels
        m.padding = int(conv.padding[0])
        m.weight = conv.weight
        m.bias = conv.bias
        return m

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        x = x.to(torch.float16).contiguous(memory_format=torch.channels_last)
        x_nhwc = x.permute(0, 2, 3, 1)                       # contiguous view, no copy
        w_rsc = self.weight.to(torch.float16)[:, 0].permute(1, 2, 0)  # [3,3,C]
        y = dwconv3x3(x_nhwc, w_rsc.contiguous(), self.padding)
        if self.bias is not None:
            y = y + self.bias.to(torch.float16)
        return y.permute(0, 3, 1, 2)                          # NCHW view, channels-last memory

    def extra_repr(self) -> str:
        return f"{self.channels}, padding={self.padding}, bias={self.bias is not None}"


def _eligible(m: nn.Module) -> bool:
    return (isinstance(m, nn.Conv2d) and m.kernel_size == (3, 3) and m.stride == (1, 1)
            and m.dilation == (1, 1) and m.groups == m.in_channels == m.out_channels
            and m.in_channels % 8 == 0 and m.padding_mode == "zeros"
            and isinstance(m.padding, tuple) and m.padding[0] == m.padding[1])


def convert_depthwise_convs(model: nn.Module) -> int:
    """Replace eligible depthwise 3x3 ``nn.Conv2d`` children in place; returns the count."""
    count = 0
    for name, child in list(model.named_children()):
        if _eligible(child):
            setattr(model, name, DepthwiseConv3x3.from_conv2d(child))
            count += 1
        else:
            count += convert_depthwise_convs(child)
    return count
