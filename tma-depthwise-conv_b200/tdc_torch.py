"""PyTorch integration of the depthwise kernels: custom ops with autograd, and
an ``nn.Conv2d(groups=C)`` stand-in for channels-last models.

* ``torch.ops.tdc.dwconv3x3(x_nhwc, w_rsc, pad)`` — 3x3 stride-1 forward
  (C % 8), with ``torch.ops.tdc.dwconv3x3_bwd_data`` /
  ``torch.ops.tdc.dwconv3x3_bwd_weight`` registered as its autograd formula
  (data gradient: the same kernel with flipped taps; weight gradient: a
  deterministic reduction kernel).
* ``torch.ops.tdc.dwconv(x_nhwc, w_rsc, bias, stride, pad)`` — K x K (3, 5,
  7), stride 1 or 2, with the bias added in the kernel's fp32 epilogue.  Its
  autograd formula covers every geometry: ``tdc::dwconv_bwd_data`` /
  ``tdc::dwconv_bwd_weight`` (at stride 2 the transposed-stencil data
  gradient and the strided weight-gradient kernel; the 3x3 ops above at 3x3
  stride 1), and the bias gradient as a sum of dy.
  All ops have fake implementations, so they trace under ``torch.compile``.
* ``DepthwiseConv2d`` — a module with ``nn.Conv2d(C, C, K, stride, padding,
  groups=C, bias=...)``'s parameters and NCHW interface.  A channels-last NCHW
  tensor is NHWC in memory, so it runs on the kernels without a copy.
  ``DepthwiseConv3x3`` is its 3x3 stride-1 form.  ``padding="same"`` is
  TensorFlow's rule at any stride (ceil(H / stride) outputs, the odd row and
  column at the bottom / right), run by the kernels' per-side padding in
  inference and as explicit zero padding when a gradient is needed.
* ``convert_depthwise_convs(model)`` — swaps every eligible ``nn.Conv2d``
  (depthwise, dilation 1 — any dilation with ``forward_only=True`` —, symmetric
  integer padding or ``padding='same'``, zeros padding mode,
  C % 8 == 0; 3x3 / 5x5 / 7x7 at stride 1 or 2) for a ``DepthwiseConv2d``
  sharing its parameters.
* ``fuse_depthwise_bn_act(model)`` — for inference: a depthwise convolution
  followed by ``BatchNorm2d`` (and ReLU / ReLU6 / SiLU / Hardswish) in an
  ``nn.Sequential`` (torchvision's ``Conv2dNormActivation``) becomes one
  ``DepthwiseConv2d`` with the normalisation folded into its weight and bias
  and the activation in the kernel's fused epilogue: one pass over the
  activations instead of three.

The reference (haowen-han/tma-depthwise-conv) has a forward-only Python API
(``tma_dwconv.py``); everything here is beyond that surface and is built on
the same kernels.
"""
from __future__ import annotations

from typing import Optional

import torch
from torch import nn
from torch.nn.utils import parametrize as _parametrize

import _tma_dwconv_C as _C  # type: ignore
import tma_dwconv as _T
from tma_dwconv import DWCONV_STAGES

#: (K, stride) pairs the kernels implement, forward and backward.
GEOMETRIES = tuple(DWCONV_STAGES)
TRAINABLE = GEOMETRIES

#: n_stage of the ring kernels' data / weight gradients per (K, stride) (the
#: custom ops pass 0 and let the library pick the kernel by shape), measured at
#: 64 x 224 x 336 x 256 (stride 1 data gradient: the forward's table; weight
#: gradient, 2 / 3 / 4 stages, us: 5x5 1618 / 1540 / 1479, 7x7 3218 / 2840 /
#: 2890; stride 2: 3x3 526 / 467 / 458, 5x5 792 / 806 / 633, 7x7 1184 / 1101 /
#: 1119).
BWD_STAGES = {(3, 1): (DWCONV_STAGES[(3, 1)], 2), (5, 1): (DWCONV_STAGES[(5, 1)], 4),
              (7, 1): (DWCONV_STAGES[(7, 1)], 3),
              (3, 2): (2, 4), (5, 2): (2, 4), (7, 2): (2, 3)}
assert set(BWD_STAGES) == set(GEOMETRIES)


def _out_hw(h: int, w: int, pad: int, k: int = 3, stride: int = 1) -> tuple[int, int]:
    return (h + 2 * pad - k) // stride + 1, (w + 2 * pad - k) // stride + 1


# ------------------------------ 3x3, stride 1 ---------------------------------

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


# ------------------------------ K x K, stride ---------------------------------

@torch.library.custom_op("tdc::dwconv_bwd_data", mutates_args=())
def dwconv_bwd_data_op(dy: torch.Tensor, w: torch.Tensor, pad: int, stride: int, input_h: int,
                       input_w: int) -> torch.Tensor:
    """dx [N,H,W,C] of the K x K forward, from dy [N,P,Q,C] and w [K,K,C]
    (H = input_h, W = input_w: at stride 2, dy does not determine them)."""
    return _C.dwconv_bwd_data(dy.contiguous(), w.contiguous(), pad, stride, 0, input_h, input_w)


@dwconv_bwd_data_op.register_fake
def _(dy, w, pad, stride, input_h, input_w):
    return dy.new_empty((dy.shape[0], input_h, input_w, dy.shape[3]))


@torch.library.custom_op("tdc::dwconv_bwd_weight", mutates_args=())
def dwconv_bwd_weight_op(x: torch.Tensor, dy: torch.Tensor, k: int, pad: int,
                         stride: int) -> torch.Tensor:
    """dw [K,K,C] (fp32) of the K x K forward, from x and dy."""
    return _C.dwconv_bwd_weight(x.contiguous(), dy.contiguous(), k, pad, stride, 0)


@dwconv_bwd_weight_op.register_fake
def _(x, dy, k, pad, stride):
    return x.new_empty((k, k, x.shape[3]), dtype=torch.float32)


@torch.library.custom_op("tdc::dwconv", mutates_args=())
def dwconv_op(x: torch.Tensor, w: torch.Tensor, bias: Optional[torch.Tensor], stride: int,
              pad: int) -> torch.Tensor:
    """Depthwise K x K forward with an optional fused bias: x [N,H,W,C] fp16,
    w [K,K,C] fp16, bias [C] fp16 or None -> [N,P,Q,C]."""
    b = None if bias is None else bias.contiguous()
    return _C.dwconv_k(x.contiguous(), w.contiguous(), b, None, stride, pad, 0, 0)


@dwconv_op.register_fake
def _(x, w, bias, stride, pad):
    p, q = _out_hw(x.shape[1], x.shape[2], pad, w.shape[0], stride)
    return x.new_empty((x.shape[0], p, q, x.shape[3]))


def _setup_context_k(ctx, inputs, output):
    x, w, bias, stride, pad = inputs
    ctx.save_for_backward(x, w)
    ctx.geometry = (int(w.shape[0]), int(stride))
    ctx.pad = pad
    ctx.bias_dtype = None if bias is None else bias.dtype


def _grads_k(needs, x, w, dy, k, s, pad, bias_dtype, bwd_data, bwd_weight):
    """dx, dw, db of the K x K forward.  Both gradients of every geometry go
    through the K x K entry points, whose kernels follow the shape (plain
    kernels for narrow layers, the ring kernels otherwise; the 3x3 fp16 paths
    take any pad)."""
    dx = dw = db = None
    dy = dy.to(x.dtype)
    if needs[0]:
        dx = bwd_data(dy, w, pad, s, x.shape[1], x.shape[2])
    if needs[1]:
        dw = bwd_weight(x, dy, k, pad, s).to(w.dtype)
    if bias_dtype is not None and needs[2]:
        db = dy.sum(dim=(0, 1, 2), dtype=torch.float32).to(bias_dtype)
    return dx, dw, db, None, None


def _backward_k(ctx, dy):
    x, w = ctx.saved_tensors
    return _grads_k(ctx.needs_input_grad, x, w, dy, *ctx.geometry, ctx.pad, ctx.bias_dtype,
                    dwconv_bwd_data_op, dwconv_bwd_weight_op)


dwconv_op.register_autograd(_backward_k, setup_context=_setup_context_k)


def _bwd_data_eager(dy, w, pad, stride, input_h, input_w):
    return _C.dwconv_bwd_data(dy.contiguous(), w.contiguous(), pad, stride, 0, input_h, input_w)


def _bwd_weight_eager(x, dy, k, pad, stride):
    return _C.dwconv_bwd_weight(x.contiguous(), dy.contiguous(), k, pad, stride, 0)


class _DwconvFunction(torch.autograd.Function):
    """``torch.ops.tdc.dwconv`` and its autograd formula for eager mode, calling
    the extension directly: a custom op's dispatch costs ~46 us of host time
    per forward with autograd and ~17 us per backward op (measured), against
    ~10 us for this Function, which matters for small layers in training.
    Under ``torch.compile`` the custom op is used (it has fake kernels)."""

    @staticmethod
    def forward(ctx, x, w, bias, stride, pad):
        b = None if bias is None else bias.contiguous()
        y = _C.dwconv_k(x.contiguous(), w.contiguous(), b, None, stride, pad, 0, 0)
        ctx.save_for_backward(x, w)
        ctx.geometry = (int(w.shape[0]), int(stride))
        ctx.pad = pad
        ctx.bias_dtype = None if bias is None else bias.dtype
        return y

    @staticmethod
    def backward(ctx, dy):
        x, w = ctx.saved_tensors
        return _grads_k(ctx.needs_input_grad, x, w, dy, *ctx.geometry, ctx.pad, ctx.bias_dtype,
                        _bwd_data_eager, _bwd_weight_eager)


class _DepthwiseConvFunction(torch.autograd.Function):
    """The autograd path of ``DepthwiseConv2d`` in eager mode: one node from
    the module's own tensors (x [N,C,H,W] channels-last in the compute dtype,
    weight [C,1,K,K] and bias [C] in any float dtype) to y [N,C,P,Q]
    channels-last.  The [K,K,C] re-layout of the weight and the dtype casts
    happen inside, and the weight gradient comes back in the parameter's
    layout and dtype in one copy, so a training step adds no autograd nodes
    (and their backward copies) for them."""

    @staticmethod
    def forward(ctx, x, weight, bias, stride, pad, dt):
        x_nhwc = x.permute(0, 2, 3, 1)                   # contiguous view, no copy
        w_rsc = weight.to(dt)[:, 0].permute(1, 2, 0).contiguous()
        b = None if bias is None else bias.to(dt).contiguous()
        y = _C.dwconv_k(x_nhwc, w_rsc, b, None, stride, pad, 0, 0)
        ctx.save_for_backward(x_nhwc, w_rsc)
        ctx.conf = (int(weight.shape[-1]), stride, pad, weight.dtype,
                    None if bias is None else bias.dtype)
        return y.permute(0, 3, 1, 2)

    @staticmethod
    def backward(ctx, gy):
        x_nhwc, w_rsc = ctx.saved_tensors
        k, stride, pad, w_dtype, b_dtype = ctx.conf
        dy = gy.permute(0, 2, 3, 1).to(x_nhwc.dtype).contiguous()
        gx = gw = gb = None
        if ctx.needs_input_grad[0]:
            gx = _C.dwconv_bwd_data(dy, w_rsc, pad, stride, 0, x_nhwc.shape[1],
                                    x_nhwc.shape[2]).permute(0, 3, 1, 2)
        if ctx.needs_input_grad[1]:
            dw = _C.dwconv_bwd_weight(x_nhwc, dy, k, pad, stride, 0)  # [K,K,C] fp32
            gw = torch.empty((dw.shape[2], 1, k, k), dtype=w_dtype, device=dw.device)
            gw[:, 0].copy_(dw.permute(2, 0, 1))                        # transpose + cast
        if b_dtype is not None and ctx.needs_input_grad[2]:
            gb = dy.sum(dim=(0, 1, 2), dtype=torch.float32).to(b_dtype)
        return gx, gw, gb, None, None, None


def _dwconv_autograd(x, w, bias, stride: int, pad: int) -> torch.Tensor:
    if torch.compiler.is_compiling():
        return dwconv_op(x, w, bias, stride, pad)
    return _DwconvFunction.apply(x, w, bias, stride, pad)


def dwconv(x_nhwc: torch.Tensor, w_rsc: torch.Tensor, bias: Optional[torch.Tensor] = None,
           stride: int = 1, pad: Optional[int] = None) -> torch.Tensor:
    """Depthwise K x K on NHWC fp16 / bf16 tensors (differentiable at stride 1
    and 2); the custom op under ``torch.compile``, a lighter autograd
    Function in eager mode (same kernels, same results)."""
    if pad is None:
        pad = int(w_rsc.shape[0]) // 2
    return _dwconv_autograd(x_nhwc, w_rsc, bias, int(stride), int(pad))


# ------------------------------ nn.Conv2d stand-in ---------------------------

#: Activations the fused epilogue implements, with their PyTorch equivalents
#: (used when a gradient is needed: the op's autograd formula covers conv + bias).
_TORCH_ACTS = {"none": None, "relu": torch.nn.functional.relu, "relu6": torch.nn.functional.relu6,
               "silu": torch.nn.functional.silu, "hardswish": torch.nn.functional.hardswish}


class DepthwiseConv2d(nn.Module):
    """``nn.Conv2d(C, C, K, stride, padding, groups=C, bias=bias)`` for fp16
    or bf16 channels-last NCHW inputs (NHWC memory), on the sm_100a kernels,
    K in {3, 5, 7}, stride 1 or 2 (forward and backward).  bf16 inputs run in
    bf16 (3x3 stride 1 with padding up to 2); anything else is converted to
    fp16.

    Parameters keep ``nn.Conv2d``'s layout (weight [C, 1, K, K], bias [C]), so
    state dicts load unchanged.  Inputs that are not fp16 or bf16 CUDA tensors in
    channels-last layout are converted (one copy).
    """

    def __init__(self, channels: int, kernel_size: int = 3, stride: int = 1,
                 padding=None, bias: bool = True, device=None,
                 dtype=torch.float16, activation: str = "none", dilation: int = 1):
        super().__init__()
        if (kernel_size, stride) not in GEOMETRIES:
            raise ValueError(f"kernel_size must be 3, 5 or 7 and stride 1 or 2, got "
                             f"{kernel_size}, {stride}")
        if activation not in _TORCH_ACTS:
            raise ValueError(f"activation must be one of {sorted(_TORCH_ACTS)}, got {activation!r}")
        if int(dilation) < 1:
            raise ValueError(f"dilation must be >= 1, got {dilation}")
        self.activation = activation
        self.dilation = int(dilation)  # > 1: inference only (no gradient kernels)
        self.channels = channels
        self.kernel_size = int(kernel_size)
        self.stride = int(stride)
        # an int (the same on every side), or "same": TensorFlow's / PyTorch's
        # "same" padding, ceil(H / stride) output rows, computed per input
        self.padding = (self.dilation * (kernel_size - 1) // 2 if padding is None else
                        "same" if padding == "same" else int(padding))
        self.weight = nn.Parameter(torch.empty(channels, 1, kernel_size, kernel_size,
                                               device=device, dtype=dtype))
        self.bias = nn.Parameter(torch.empty(channels, device=device, dtype=dtype)) if bias else None
        nn.init.kaiming_uniform_(self.weight, a=5 ** 0.5)
        if self.bias is not None:
            bound = 1.0 / kernel_size
            nn.init.uniform_(self.bias, -bound, bound)

    @classmethod
    def from_conv2d(cls, conv: nn.Conv2d) -> "DepthwiseConv2d":
        m = cls.__new__(cls)
        nn.Module.__init__(m)
        m.channels = conv.in_channels
        m.kernel_size = int(conv.kernel_size[0])
        m.stride = int(conv.stride[0])
        m.padding = _conv2d_pad(conv)
        m.dilation = int(conv.dilation[0])
        m.weight = conv.weight
        m.bias = conv.bias
        m.activation = "none"
        return m

    def forward(self, x: torch.Tensor) -> torch.Tensor:
        dt = torch.bfloat16 if x.dtype == torch.bfloat16 else torch.float16
        act = self.activation
        needs_grad = torch.is_grad_enabled() and (
            x.requires_grad or self.weight.requires_grad
            or (self.bias is not None and self.bias.requires_grad))
        dil = getattr(self, "dilation", 1)
        if dil > 1 and needs_grad:
            raise RuntimeError("DepthwiseConv2d: gradients of dilated depthwise convolutions are "
                               "not implemented; run it without gradients (inference), e.g. "
                               "under torch.no_grad()")
        pad, pads = self.padding, None
        if pad == "same":
            pads = _T.same_padding(x.shape[2], x.shape[3], dil * (self.kernel_size - 1) + 1,
                                   self.stride)
            if pads[0] == pads[1] == pads[2] == pads[3]:
                pad, pads = pads[0], None
            elif needs_grad:
                # training: explicit zero padding, then the symmetric kernels
                # (whose gradients cover pad 0)
                x = torch.nn.functional.pad(x, (pads[2], pads[3], pads[0], pads[1]))
                pad, pads = 0, None
        x = x.to(dt).contiguous(memory_format=torch.channels_last)
        if needs_grad and not torch.compiler.is_compiling():
            # training, eager: one autograd node for conv + bias (the
            # activation, if any, runs outside the kernel)
            y = _DepthwiseConvFunction.apply(x, self.weight, self.bias, self.stride, pad, dt)
            return y if act == "none" else _TORCH_ACTS[act](y)
        x_nhwc = x.permute(0, 2, 3, 1)                                  # contiguous view, no copy
        w_rsc = self.weight.to(dt)[:, 0].permute(1, 2, 0)              # [K,K,C]
        b = None if self.bias is None else self.bias.to(dt)
        if not needs_grad:
            # inference: straight to the extension (which checks its arguments),
            # without the custom op's dispatch; the activation runs in the
            # kernel's fused epilogue
            b = None if b is None else b.contiguous()
            if pads is not None or dil > 1:  # per-side padding or dilated taps
                pads = pads if pads is not None else (pad,) * 4
                y = _C.dwconv_k_pads(x_nhwc, w_rsc.contiguous(), b, None, self.stride, dil, *pads,
                                     _T.ACTIVATIONS[act], 0)
            else:
                y = _C.dwconv_k(x_nhwc, w_rsc.contiguous(), b, None, self.stride, pad,
                                _T.ACTIVATIONS[act], 0)
        else:  # under torch.compile (pads already explicit): the custom op, which has fake kernels
            y = dwconv_op(x_nhwc, w_rsc.contiguous(), b, self.stride, pad)
            if act != "none":  # the autograd formula covers conv + bias
                y = _TORCH_ACTS[act](y)
        return y.permute(0, 3, 1, 2)                                    # NCHW view, channels-last memory

    def extra_repr(self) -> str:
        act = "" if self.activation == "none" else f", activation={self.activation}"
        dil = getattr(self, "dilation", 1)
        dil = "" if dil == 1 else f", dilation={dil}"
        return (f"{self.channels}, kernel_size={self.kernel_size}, stride={self.stride}, "
                f"padding={self.padding}{dil}, bias={self.bias is not None}{act}")


class DepthwiseConv3x3(DepthwiseConv2d):
    """``DepthwiseConv2d`` with a 3x3 kernel and stride 1."""

    def __init__(self, channels: int, padding: int = 1, bias: bool = True, device=None,
                 dtype=torch.float16):
        super().__init__(channels, 3, 1, padding, bias, device, dtype)


def _conv2d_pad(conv: nn.Conv2d) -> int:
    """The symmetric padding of an eligible depthwise nn.Conv2d: its integer
    padding, or K // 2 for ``padding='same'`` (PyTorch allows it at stride 1
    only, where an odd K pads K // 2 on every side)."""
    if conv.padding == "same":
        return int(conv.dilation[0]) * (int(conv.kernel_size[0]) - 1) // 2
    return int(conv.padding[0])


def _plain_conv2d(m: nn.Module) -> bool:
    """An ``nn.Conv2d`` whose computation is ``nn.Conv2d``'s own.  Subclasses
    that override ``forward`` or ``_conv_forward`` (timm's ``Conv2dSame``
    pads in ``forward``; QAT convolutions fake-quantise the weight), convs
    with a parametrized weight (weight norm, spectral norm) and convs with
    forward hooks are left alone: swapping them would silently drop what
    they add."""
    if not isinstance(m, nn.Conv2d):
        return False
    cls = type(m)
    if cls.forward is not nn.Conv2d.forward or cls._conv_forward is not nn.Conv2d._conv_forward:
        return False
    if _parametrize.is_parametrized(m):
        return False
    return not (m._forward_hooks or m._forward_pre_hooks)


def _eligible(m: nn.Module, forward_only: bool) -> bool:
    if not (_plain_conv2d(m) and m.dilation[0] == m.dilation[1]
            and (m.dilation[0] == 1 or forward_only)  # dilated: no gradient kernels
            and m.groups == m.in_channels == m.out_channels and m.in_channels % 8 == 0
            and m.padding_mode == "zeros"
            and ((isinstance(m.padding, tuple) and m.padding[0] == m.padding[1])
                 or (m.padding == "same" and m.kernel_size[0] % 2 == 1))
            and m.kernel_size[0] == m.kernel_size[1] and m.stride[0] == m.stride[1]):
        return False
    geometry = (m.kernel_size[0], m.stride[0])
    return geometry in (GEOMETRIES if forward_only else TRAINABLE)


def convert_depthwise_convs(model: nn.Module, forward_only: bool = False) -> int:
    """Replace eligible depthwise ``nn.Conv2d`` children in place; returns the count.

    Every geometry the kernels implement (3x3 / 5x5 / 7x7, stride 1 or 2) has
    a backward.  ``forward_only=True`` also converts dilated depthwise convs
    (atrous layers, e.g. DeepLab backbones), which run in inference only:
    their modules raise if called with a gradient.
    """
    count = 0
    for name, child in list(model.named_children()):
        if _eligible(child, forward_only):
            cls = DepthwiseConv3x3 if (child.kernel_size[0], child.stride[0]) == (3, 1) \
                else DepthwiseConv2d
            setattr(model, name, cls.from_conv2d(child))
            count += 1
        else:
            count += convert_depthwise_convs(child, forward_only)
    return count


_FUSABLE_ACTS = {nn.ReLU: "relu", nn.ReLU6: "relu6", nn.SiLU: "silu", nn.Hardswish: "hardswish"}


def _fold_bn(conv: nn.Module, bn: nn.BatchNorm2d, activation: str) -> DepthwiseConv2d:
    """conv (a depthwise nn.Conv2d or a DepthwiseConv2d) followed by bn in
    inference: w' = w * g, b' = (b - mean) * g + beta, g = gamma / sqrt(var + eps),
    computed in float32 and stored in the convolution's dtype."""
    w = conv.weight.detach().float()
    c = w.shape[0]
    b = conv.bias.detach().float() if conv.bias is not None else torch.zeros(c, device=w.device)
    gamma = bn.weight.detach().float() if bn.weight is not None else torch.ones(c, device=w.device)
    beta = bn.bias.detach().float() if bn.bias is not None else torch.zeros(c, device=w.device)
    g = gamma / torch.sqrt(bn.running_var.detach().float() + bn.eps)
    k = conv.kernel_size[0] if isinstance(conv.kernel_size, tuple) else conv.kernel_size
    stride = conv.stride[0] if isinstance(conv.stride, tuple) else conv.stride
    pad = conv.padding if isinstance(conv, DepthwiseConv2d) else _conv2d_pad(conv)
    d = conv.dilation[0] if isinstance(conv.dilation, tuple) else getattr(conv, "dilation", 1)
    m = DepthwiseConv2d(c, int(k), int(stride), pad, bias=True, device=w.device,
                        dtype=conv.weight.dtype, activation=activation, dilation=int(d))
    with torch.no_grad():
        m.weight.copy_(w * g[:, None, None, None])
        m.bias.copy_((b - bn.running_mean.detach().float()) * g + beta)
    return m


def _fuse_in_sequential(seq: nn.Sequential) -> int:
    items = list(seq._modules.items())
    count, i = 0, 0
    while i + 1 < len(items):
        (k0, m0), (k1, m1) = items[i], items[i + 1]
        conv_ok = _eligible(m0, True) or (type(m0) in (DepthwiseConv2d, DepthwiseConv3x3)
                                          and m0.activation == "none")
        if (conv_ok and isinstance(m1, nn.BatchNorm2d) and m1.running_mean is not None
                and m1.num_features == m0.weight.shape[0]):
            if m1.training:
                raise ValueError("fuse_depthwise_bn_act folds running statistics: call model.eval() first")
            act, k2 = "none", None
            if i + 2 < len(items) and type(items[i + 2][1]) in _FUSABLE_ACTS:
                k2 = items[i + 2][0]
                act = _FUSABLE_ACTS[type(items[i + 2][1])]
            seq._modules[k0] = _fold_bn(m0, m1, act)
            seq._modules[k1] = nn.Identity()
            if k2 is not None:
                seq._modules[k2] = nn.Identity()
            count += 1
            i += 3 if k2 is not None else 2
        else:
            i += 1
    return count


def fuse_depthwise_bn_act(model: nn.Module) -> int:
    """Fuse, for inference, every depthwise convolution that an ``nn.Sequential``
    follows with ``BatchNorm2d`` (and optionally ReLU / ReLU6 / SiLU /
    Hardswish), e.g. torchvision's ``Conv2dNormActivation`` blocks of
    MobileNet / EfficientNet.  The convolution (an eligible ``nn.Conv2d`` or a
    ``DepthwiseConv2d``) becomes a ``DepthwiseConv2d`` holding the folded
    weight and bias (new tensors, the convolution's dtype) with the activation
    in the kernel's epilogue; the normalisation and activation modules become
    ``nn.Identity``.  The model must be in eval mode (running statistics are
    folded).  Returns the number of fused blocks.
    """
    count = _fuse_in_sequential(model) if isinstance(model, nn.Sequential) else 0
    for child in model.children():
        count += fuse_depthwise_bn_act(child)
    return count

