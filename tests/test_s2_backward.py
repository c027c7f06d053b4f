"""Backward of the K x K stride-2 forward (beyond the reference's forward-only,
3x3 stride-1 surface).

* data gradient (`dwconv_bwd_data(..., stride=2)`: the transposed-stencil
  kernel) — bit for bit with the CPU oracle's restatement
  (oracle_dwconv_bwd_data_s2_f16), which matches float64 autograd within
  fp16 rounding (tests/test_oracle.py);
* weight gradient (`dwconv_bwd_weight(..., stride=2)`: the strided weight-
  gradient kernel, tap rows split over launches as at stride 1) — within
  5e-4 of sum |x*dy| of the float64 oracle, and bit-reproducible;
* autograd through `torch.ops.tdc.dwconv` (fused bias) and the module,
  against float32 PyTorch autograd.
"""
import numpy as np
import pytest
import torch

import oracle
import tdc_torch
import tma_dwconv as T

pytestmark = pytest.mark.gpu

SHAPES = [  # N, H, W, C, pad (None: K // 2)
    (2, 16, 16, 64, None),
    (3, 19, 45, 72, None),
    (2, 9, 34, 136, 0),
    (1, 12, 13, 8, 1),
    (4, 56, 56, 256, None),
    (1, 7, 7, 64, None),
    (2, 33, 70, 64, 2),
    (1, 1, 1, 8, None),     # one pixel: only the centre tap reaches it
    (2, 2, 3, 16, None),
]


def _tensors(N, H, W, C, K, pad, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, H, W, C, generator=g).half()
    w = (torch.randn(K, K, C, generator=g) / K).half()
    P, Q = (H + 2 * pad - K) // 2 + 1, (W + 2 * pad - K) // 2 + 1
    dy = torch.randn(N, P, Q, C, generator=g).half()
    return x, w, dy


def _bits(a):
    return np.asarray(a).view(np.uint16)


@pytest.mark.parametrize("K", [3, 5, 7])
@pytest.mark.parametrize("N,H,W,C,pad", SHAPES)
def test_data_gradient_matches_oracle(K, N, H, W, C, pad):
    pad = K // 2 if pad is None else pad
    x, w, dy = _tensors(N, H, W, C, K, pad)
    want = oracle.dwconv_bwd_data_s2_f16(dy.numpy(), w.numpy(), pad, H, W)
    for n_stage in (2, 3, 4):
        dx = T._C.dwconv_bwd_data(dy.cuda(), w.cuda(), pad, 2, n_stage, H, W).cpu().numpy()
        assert dx.shape == x.shape
        assert np.array_equal(_bits(dx), _bits(want)), n_stage


@pytest.mark.parametrize("K", [3, 5, 7])
def test_data_gradient_every_padding_and_both_input_sizes(K):
    # H and H + 1 give the same P when H + 2*pad - K is even: the last input
    # row (read by no output) gets a zero gradient.
    for pad in range(K + 2):
        for H, W in ((11, 37), (12, 38)):
            if H + 2 * pad < K:
                continue
            x, w, dy = _tensors(2, H, W, 64, K, pad, seed=pad)
            dx = T._C.dwconv_bwd_data(dy.cuda(), w.cuda(), pad, 2, 2, H, W).cpu().numpy()
            want = oracle.dwconv_bwd_data_s2_f16(dy.numpy(), w.numpy(), pad, H, W)
            assert np.array_equal(_bits(dx), _bits(want)), (pad, H, W)


def test_data_gradient_default_input_size_is_the_smaller_one():
    x, w, dy = _tensors(2, 20, 30, 64, 3, 1, seed=3)  # P = 10: H = 19 or 20
    dx = T._C.dwconv_bwd_data(dy.cuda(), w.cuda(), 1, 2)
    assert dx.shape == (2, 19, 29, 64)
    full = T._C.dwconv_bwd_data(dy.cuda(), w.cuda(), 1, 2, 2, 20, 30)
    assert torch.equal(dx, full[:, :19, :29])
    with pytest.raises(RuntimeError, match="is not the stride-2 output"):
        T._C.dwconv_bwd_data(dy.cuda(), w.cuda(), 1, 2, 2, 22, 30)


def test_data_gradient_64bit_offsets():
    # dx holds more than 2^31 elements; images are independent, so the last
    # one is checked against the oracle on that image alone.
    N, H, W, C, K, pad = 170, 224, 224, 256, 3, 1
    P, Q = (H + 2 * pad - K) // 2 + 1, (W + 2 * pad - K) // 2 + 1
    assert N * H * W * C > 2 ** 31
    g = torch.Generator(device="cuda").manual_seed(7)
    dy = torch.randn(N, P, Q, C, device="cuda", generator=g).half()
    w = (torch.randn(K, K, C, device="cuda", generator=g) / K).half()
    dx = T._C.dwconv_bwd_data(dy, w, pad, 2, 2, H, W)
    last = dx[-1:].cpu().numpy()
    del dx
    want = oracle.dwconv_bwd_data_s2_f16(dy[-1:].cpu().numpy(), w.cpu().numpy(), pad, H, W)
    assert np.array_equal(_bits(last), _bits(want))


@pytest.mark.parametrize("K", [3, 5, 7])
@pytest.mark.parametrize("N,H,W,C,pad", SHAPES)
def test_weight_gradient_close_to_float64(K, N, H, W, C, pad):
    pad = K // 2 if pad is None else pad
    x, w, dy = _tensors(N, H, W, C, K, pad, seed=1)
    ref = oracle.dwconv_bwd_weight_f64(x.numpy(), dy.numpy(), pad, K, stride=2)
    scale = oracle.dwconv_bwd_weight_f64(np.abs(x.numpy()), np.abs(dy.numpy()), pad, K, stride=2)
    for n_stage in (2, 3, 4):
        dw = T._C.dwconv_bwd_weight(x.cuda(), dy.cuda(), K, pad, 2, n_stage).cpu().numpy()
        assert dw.dtype == np.float32 and dw.shape == (K, K, C)
        assert (np.abs(dw - ref) <= 5e-4 * scale + 1e-6).all(), (n_stage, np.abs(dw - ref).max())


@pytest.mark.parametrize("K", [3, 5, 7])
def test_weight_gradient_every_padding(K):
    for pad in range(K + 2):
        x, w, dy = _tensors(2, 13, 40, 64, K, pad, seed=10 + pad)
        ref = oracle.dwconv_bwd_weight_f64(x.numpy(), dy.numpy(), pad, K, stride=2)
        scale = oracle.dwconv_bwd_weight_f64(np.abs(x.numpy()), np.abs(dy.numpy()), pad, K, stride=2)
        dw = T._C.dwconv_bwd_weight(x.cuda(), dy.cuda(), K, pad, 2, 3).cpu().numpy()
        assert (np.abs(dw - ref) <= 5e-4 * scale + 1e-6).all(), pad


@pytest.mark.parametrize("K", [3, 5, 7])
def test_weight_gradient_is_deterministic(K):
    x, w, dy = _tensors(8, 56, 56, 256, K, K // 2, seed=2)
    xd, dyd = x.cuda(), dy.cuda()
    for n_stage in (2, 4):
        a = T._C.dwconv_bwd_weight(xd, dyd, K, K // 2, 2, n_stage)
        for _ in range(2):
            b = T._C.dwconv_bwd_weight(xd, dyd, K, K // 2, 2, n_stage)
            assert torch.equal(a.view(torch.int32), b.view(torch.int32))


def test_large_weight_gradient_7x7():
    g = torch.Generator(device="cuda").manual_seed(3)
    x = (torch.rand(4, 224, 336, 256, device="cuda", generator=g) * 2 - 1).half()
    dy = (torch.rand(4, 112, 168, 256, device="cuda", generator=g) * 2 - 1).half()
    dw = T._C.dwconv_bwd_weight(x, dy, 7, 3, 2).cpu().numpy()
    xn, dyn = x.cpu().numpy(), dy.cpu().numpy()
    ref = oracle.dwconv_bwd_weight_f64(xn, dyn, 3, 7, stride=2)
    scale = oracle.dwconv_bwd_weight_f64(np.abs(xn), np.abs(dyn), 3, 7, stride=2)
    assert (np.abs(dw - ref) <= 5e-4 * scale + 1e-6).all()


def test_weight_gradient_shape_errors():
    x, w, dy = _tensors(1, 12, 12, 64, 5, 2)
    with pytest.raises(RuntimeError, match="dy must be"):
        T._C.dwconv_bwd_weight(x.cuda(), dy.cuda(), 5, 2, 1)  # a stride-1 dy is larger
    with pytest.raises(RuntimeError, match="stride must be 1 or 2"):
        T._C.dwconv_bwd_weight(x.cuda(), dy.cuda(), 5, 2, 3)


def _fp32_autograd(x, w, b, pad, dy):
    xt = x.float().permute(0, 3, 1, 2).requires_grad_()
    wt = w.float().permute(2, 0, 1).unsqueeze(1).detach().requires_grad_()
    bt = b.float().detach().requires_grad_()
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        y = torch.nn.functional.conv2d(xt, wt, bt, stride=2, padding=pad, groups=x.shape[3])
        y.backward(dy.float().permute(0, 3, 1, 2))
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    return (y.detach().permute(0, 2, 3, 1), xt.grad.permute(0, 2, 3, 1),
            wt.grad[:, 0].permute(1, 2, 0), bt.grad)


@pytest.mark.parametrize("K", [3, 5, 7])
def test_autograd_custom_op_with_bias(K):
    N, H, W, C, pad = 2, 21, 30, 64, K // 2
    x, w, dy = _tensors(N, H, W, C, K, pad, seed=4)
    b = torch.randn(C, generator=torch.Generator().manual_seed(6)).half()
    x, w, b, dy = (x.cuda().requires_grad_(), w.cuda().requires_grad_(), b.cuda().requires_grad_(),
                   dy.cuda())
    y = torch.ops.tdc.dwconv(x, w, b, 2, pad)
    y.backward(dy)
    ry, rdx, rdw, rdb = _fp32_autograd(x.detach(), w.detach(), b.detach(), pad, dy)
    tol = lambda r: torch.from_numpy(oracle.f16_ulp(r.cpu().numpy())).cuda() + 1e-3
    assert ((y.float() - ry).abs() <= tol(ry)).all()
    assert x.grad.shape == x.shape
    assert ((x.grad.float() - rdx).abs() <= tol(rdx)).all()
    assert w.grad.dtype == torch.float16 and b.grad.dtype == torch.float16
    torch.testing.assert_close(w.grad.float(), rdw, rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(b.grad.float(), rdb, rtol=2e-3, atol=2e-2)


def test_module_trains_stride_2():
    # Same upstream gradient for both models (a ReLU after the conv would let
    # one-ulp forward differences flip its mask and change dy).
    torch.manual_seed(0)
    conv = torch.nn.Conv2d(64, 64, 5, stride=2, padding=2, groups=64, bias=True).cuda().half()
    model = torch.nn.Sequential(conv)
    x = torch.randn(2, 64, 21, 30, device="cuda").half().to(memory_format=torch.channels_last)
    x.requires_grad_()
    want = model(x)
    gy = torch.randn(want.shape, device="cuda").half().to(memory_format=torch.channels_last)
    want.backward(gy)
    gx_want, gw_want, gb_want = x.grad.clone(), conv.weight.grad.clone(), conv.bias.grad.clone()
    x.grad = conv.weight.grad = conv.bias.grad = None
    assert tdc_torch.convert_depthwise_convs(model) == 1
    assert type(model[0]) is tdc_torch.DepthwiseConv2d and model[0].weight is conv.weight
    got = model(x)
    torch.testing.assert_close(got, want, rtol=1e-2, atol=1e-2)
    got.backward(gy)
    assert x.grad.shape == x.shape and conv.weight.grad.shape == (64, 1, 5, 5)
    torch.testing.assert_close(x.grad.float(), gx_want.float(), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(conv.weight.grad.float(), gw_want.float(), rtol=2e-2, atol=1e-1)
    torch.testing.assert_close(conv.bias.grad.float(), gb_want.float(), rtol=2e-2, atol=1e-1)
