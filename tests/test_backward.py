"""Backward of the depthwise 3x3 (beyond the reference's forward-only surface).

* data gradient (`dwconv3x3_bwd_data`: the forward kernel with flipped taps
  and padding 2 - pad) — bit for bit with the CPU oracle's restatement, which
  itself matches float64 autograd within fp16 rounding;
* weight gradient (`dwconv3x3_bwd_weight`: streaming reduction, fp32
  accumulation in a fixed order) — within 5e-4 of sum |x*dy| of the float64
  oracle, and bit-reproducible from run to run;
* autograd through `torch.ops.tdc.dwconv3x3` and the `nn.Conv2d` stand-in,
  against float32 PyTorch autograd.
"""
import numpy as np
import pytest
import torch

import oracle
import tdc_torch
import tma_dwconv as T

pytestmark = pytest.mark.gpu

SHAPES = [  # N, H, W, C, pad
    (2, 16, 16, 64, 1),
    (3, 19, 45, 72, 1),
    (2, 9, 34, 136, 0),
    (1, 12, 12, 8, 2),
    (2, 7, 9, 64, 3),       # pad > 2: the data gradient runs with negative padding (a crop)
    (4, 56, 56, 256, 1),
    (1, 1, 1, 64, 1),
]


def _tensors(N, H, W, C, pad, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, H, W, C, generator=g).half()
    w = (torch.randn(3, 3, C, generator=g) / 3).half()
    dy = torch.randn(N, H + 2 * pad - 2, W + 2 * pad - 2, C, generator=g).half()
    return x, w, dy


@pytest.mark.parametrize("N,H,W,C,pad", SHAPES)
def test_data_gradient_matches_oracle(N, H, W, C, pad):
    x, w, dy = _tensors(N, H, W, C, pad)
    dx = T._C.dwconv3x3_bwd_data(dy.cuda(), w.cuda(), pad, 2).cpu().numpy()
    want = oracle.dwconv_bwd_data_f16(dy.numpy(), w.numpy(), pad)
    assert dx.shape == x.shape
    assert np.array_equal(dx.view(np.uint16), want.view(np.uint16))


@pytest.mark.parametrize("N,H,W,C,pad", SHAPES)
def test_weight_gradient_close_to_float64(N, H, W, C, pad):
    x, w, dy = _tensors(N, H, W, C, pad, seed=1)
    dw = T._C.dwconv3x3_bwd_weight(x.cuda(), dy.cuda(), pad, 2).cpu().numpy()
    ref = oracle.dwconv_bwd_weight_f64(x.numpy(), dy.numpy(), pad)
    scale = oracle.dwconv_bwd_weight_f64(np.abs(x.numpy()), np.abs(dy.numpy()), pad)
    assert dw.dtype == np.float32 and dw.shape == (3, 3, C)
    assert (np.abs(dw - ref) <= 5e-4 * scale + 1e-6).all(), np.abs(dw - ref).max()


@pytest.mark.parametrize("n_stage", [2, 3, 4])
def test_weight_gradient_is_deterministic(n_stage):
    # Same device, same launch configuration: the summation order is fixed, so
    # repeated runs agree bit for bit.  (Different n_stage values may use a
    # different grid, hence a different, equally accurate, order.)
    x, w, dy = _tensors(8, 56, 56, 256, 1, seed=2)
    xd, dyd = x.cuda(), dy.cuda()
    a = T._C.dwconv3x3_bwd_weight(xd, dyd, 1, n_stage)
    for _ in range(3):
        b = T._C.dwconv3x3_bwd_weight(xd, dyd, 1, n_stage)
        assert torch.equal(a.view(torch.int32), b.view(torch.int32))


def test_large_weight_gradient():
    g = torch.Generator(device="cuda").manual_seed(3)
    x = (torch.rand(8, 224, 336, 256, device="cuda", generator=g) * 2 - 1).half()
    dy = (torch.rand(8, 224, 336, 256, device="cuda", generator=g) * 2 - 1).half()
    dw = T._C.dwconv3x3_bwd_weight(x, dy, 1, 2).cpu().numpy()
    ref = oracle.dwconv_bwd_weight_f64(x.cpu().numpy(), dy.cpu().numpy(), 1)
    scale = oracle.dwconv_bwd_weight_f64(np.abs(x.cpu().numpy()), np.abs(dy.cpu().numpy()), 1)
    assert (np.abs(dw - ref) <= 5e-4 * scale + 1e-6).all()


def _fp32_reference(x, w, pad, dy):
    xt = x.float().permute(0, 3, 1, 2).requires_grad_()
    wt = w.float().permute(2, 0, 1).unsqueeze(1).detach().requires_grad_()
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        y = torch.nn.functional.conv2d(xt, wt, padding=pad, groups=x.shape[3])
        y.backward(dy.float().permute(0, 3, 1, 2))
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    return (y.detach().permute(0, 2, 3, 1), xt.grad.permute(0, 2, 3, 1),
            wt.grad[:, 0].permute(1, 2, 0))


@pytest.mark.parametrize("N,H,W,C,pad", [(2, 16, 16, 64, 1), (3, 19, 45, 72, 2)])
def test_autograd_custom_op(N, H, W, C, pad):
    x, w, dy = _tensors(N, H, W, C, pad, seed=4)
    x, w, dy = x.cuda().requires_grad_(), w.cuda().requires_grad_(), dy.cuda()
    y = torch.ops.tdc.dwconv3x3(x, w, pad)
    y.backward(dy)
    ry, rdx, rdw = _fp32_reference(x.detach(), w.detach(), pad, dy)
    tol = lambda r: torch.from_numpy(oracle.f16_ulp(r.cpu().numpy())).cuda() + 1e-3
    assert ((y.float() - ry).abs() <= tol(ry)).all()
    assert ((x.grad.float() - rdx).abs() <= tol(rdx)).all()
    assert w.grad.dtype == torch.float16
    torch.testing.assert_close(w.grad.float(), rdw, rtol=2e-3, atol=2e-3)


def test_module_stand_in_for_depthwise_conv2d():
    torch.manual_seed(0)
    conv = torch.nn.Conv2d(64, 64, 3, padding=1, groups=64, bias=True).cuda().half()
    model = torch.nn.Sequential(conv, torch.nn.ReLU())
    x = torch.randn(2, 64, 20, 30, device="cuda").half().to(memory_format=torch.channels_last)
    want = model(x)
    assert tdc_torch.convert_depthwise_convs(model) == 1
    assert isinstance(model[0], tdc_torch.DepthwiseConv3x3) and model[0].weight is conv.weight
    got = model(x)
    assert got.is_contiguous(memory_format=torch.channels_last)
    torch.testing.assert_close(got, want, rtol=1e-2, atol=1e-2)
    got.float().sum().backward()
    assert conv.weight.grad is not None and conv.weight.grad.shape == (64, 1, 3, 3)
    assert conv.bias.grad is not None
