"""Backward of the 5x5 and 7x7 stride-1 forward (beyond the reference's
forward-only, 3x3 surface).

* data gradient (`dwconv_bwd_data`: the K x K forward kernel with flipped
  taps and padding K - 1 - pad) — bit for bit with the CPU oracle's
  restatement (oracle_dwconv_bwd_data_f16), which matches float64 autograd
  within fp16 rounding;
* weight gradient (`dwconv_bwd_weight`: the tap rows split over one or two
  streaming launches, fp32 sums in a fixed order) — within 5e-4 of
  sum |x*dy| of the float64 oracle, and bit-reproducible from run to run;
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
    (1, 12, 12, 8, 1),
    (4, 56, 56, 256, None),
    (1, 7, 7, 64, None),
]


def _tensors(N, H, W, C, K, pad, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, H, W, C, generator=g).half()
    w = (torch.randn(K, K, C, generator=g) / K).half()
    dy = torch.randn(N, H + 2 * pad - K + 1, W + 2 * pad - K + 1, C, generator=g).half()
    return x, w, dy


@pytest.mark.parametrize("K", [5, 7])
@pytest.mark.parametrize("N,H,W,C,pad", SHAPES)
def test_data_gradient_matches_oracle(K, N, H, W, C, pad):
    pad = K // 2 if pad is None else pad
    x, w, dy = _tensors(N, H, W, C, K, pad)
    for n_stage in (2, 3, 4):
        dx = T._C.dwconv_bwd_data(dy.cuda(), w.cuda(), pad, 1, n_stage).cpu().numpy()
        want = oracle.dwconv_bwd_data_f16(dy.numpy(), w.numpy(), pad)
        assert dx.shape == x.shape
        assert np.array_equal(dx.view(np.uint16), want.view(np.uint16)), n_stage


@pytest.mark.parametrize("K", [5, 7])
def test_data_gradient_every_padding(K):
    for pad in range(K):
        x, w, dy = _tensors(2, 11, 37, 64, K, pad, seed=pad)
        dx = T._C.dwconv_bwd_data(dy.cuda(), w.cuda(), pad).cpu().numpy()
        want = oracle.dwconv_bwd_data_f16(dy.numpy(), w.numpy(), pad)
        assert np.array_equal(dx.view(np.uint16), want.view(np.uint16)), pad


@pytest.mark.parametrize("K", [5, 7])
@pytest.mark.parametrize("N,H,W,C,pad", SHAPES)
def test_weight_gradient_close_to_float64(K, N, H, W, C, pad):
    pad = K // 2 if pad is None else pad
    x, w, dy = _tensors(N, H, W, C, K, pad, seed=1)
    ref = oracle.dwconv_bwd_weight_f64(x.numpy(), dy.numpy(), pad, K)
    scale = oracle.dwconv_bwd_weight_f64(np.abs(x.numpy()), np.abs(dy.numpy()), pad, K)
    for n_stage in (2, 3, 4):
        dw = T._C.dwconv_bwd_weight(x.cuda(), dy.cuda(), K, pad, 1, n_stage).cpu().numpy()
        assert dw.dtype == np.float32 and dw.shape == (K, K, C)
        assert (np.abs(dw - ref) <= 5e-4 * scale + 1e-6).all(), (n_stage, np.abs(dw - ref).max())


@pytest.mark.parametrize("K", [5, 7])
def test_weight_gradient_is_deterministic(K):
    x, w, dy = _tensors(8, 56, 56, 256, K, K // 2, seed=2)
    xd, dyd = x.cuda(), dy.cuda()
    for n_stage in (2, 4):
        a = T._C.dwconv_bwd_weight(xd, dyd, K, K // 2, 1, n_stage)
        for _ in range(2):
            b = T._C.dwconv_bwd_weight(xd, dyd, K, K // 2, 1, n_stage)
            assert torch.equal(a.view(torch.int32), b.view(torch.int32))


def test_large_weight_gradient_7x7():
    g = torch.Generator(device="cuda").manual_seed(3)
    x = (torch.rand(4, 224, 336, 256, device="cuda", generator=g) * 2 - 1).half()
    dy = (torch.rand(4, 224, 336, 256, device="cuda", generator=g) * 2 - 1).half()
    dw = T._C.dwconv_bwd_weight(x, dy, 7, 3).cpu().numpy()
    xn, dyn = x.cpu().numpy(), dy.cpu().numpy()
    ref = oracle.dwconv_bwd_weight_f64(xn, dyn, 3, 7)
    scale = oracle.dwconv_bwd_weight_f64(np.abs(xn), np.abs(dyn), 3, 7)
    assert (np.abs(dw - ref) <= 5e-4 * scale + 1e-6).all()


def test_3x3_routes_to_the_3x3_kernels():
    x, w, dy = _tensors(2, 20, 30, 64, 3, 1, seed=5)
    xd, wd, dyd = x.cuda(), w.cuda(), dy.cuda()
    assert torch.equal(T._C.dwconv_bwd_data(dyd, wd, 1), T._C.dwconv3x3_bwd_data(dyd, wd, 1, 2))
    assert torch.equal(T._C.dwconv_bwd_weight(xd, dyd, 3, 1), T._C.dwconv3x3_bwd_weight(xd, dyd, 1, 2))


def test_argument_errors():
    x, w, dy = _tensors(1, 12, 12, 64, 7, 3)
    with pytest.raises(RuntimeError, match="stride must be 1 or 2"):
        T._C.dwconv_bwd_data(dy.cuda(), w.cuda(), 3, 3)
    with pytest.raises(RuntimeError, match="stride must be 1 or 2"):
        T._C.dwconv_bwd_weight(x.cuda(), dy.cuda(), 7, 3, 3)
    with pytest.raises(RuntimeError, match="is not the stride-2 output"):
        T._C.dwconv_bwd_data(dy.cuda(), w.cuda(), 3, 2, 2, 12, 12)  # a stride-1 dy
    with pytest.raises(RuntimeError, match="needs pad <= 6"):
        T._C.dwconv_bwd_data(dy.cuda(), w.cuda(), 7)
    with pytest.raises(RuntimeError, match="dy must be"):
        T._C.dwconv_bwd_weight(x.cuda(), dy.cuda(), 5, 3)


def _fp32_autograd(x, w, b, pad, dy):
    xt = x.float().permute(0, 3, 1, 2).requires_grad_()
    wt = w.float().permute(2, 0, 1).unsqueeze(1).detach().requires_grad_()
    bt = b.float().detach().requires_grad_()
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        y = torch.nn.functional.conv2d(xt, wt, bt, padding=pad, groups=x.shape[3])
        y.backward(dy.float().permute(0, 3, 1, 2))
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    return (y.detach().permute(0, 2, 3, 1), xt.grad.permute(0, 2, 3, 1),
            wt.grad[:, 0].permute(1, 2, 0), bt.grad)


@pytest.mark.parametrize("K", [5, 7])
def test_autograd_custom_op_with_bias(K):
    N, H, W, C, pad = 2, 21, 30, 64, K // 2
    x, w, dy = _tensors(N, H, W, C, K, pad, seed=4)
    b = torch.randn(C, generator=torch.Generator().manual_seed(6)).half()
    x, w, b, dy = (x.cuda().requires_grad_(), w.cuda().requires_grad_(), b.cuda().requires_grad_(),
                   dy.cuda())
    y = torch.ops.tdc.dwconv(x, w, b, 1, pad)
    y.backward(dy)
    ry, rdx, rdw, rdb = _fp32_autograd(x.detach(), w.detach(), b.detach(), pad, dy)
    tol = lambda r: torch.from_numpy(oracle.f16_ulp(r.cpu().numpy())).cuda() + 1e-3
    assert ((y.float() - ry).abs() <= tol(ry)).all()
    assert ((x.grad.float() - rdx).abs() <= tol(rdx)).all()
    assert w.grad.dtype == torch.float16 and b.grad.dtype == torch.float16
    torch.testing.assert_close(w.grad.float(), rdw, rtol=2e-3, atol=2e-3)
    torch.testing.assert_close(b.grad.float(), rdb, rtol=2e-3, atol=2e-2)


def test_module_trains_7x7():
    torch.manual_seed(0)
    conv = torch.nn.Conv2d(64, 64, 7, padding=3, groups=64, bias=True).cuda().half()
    model = torch.nn.Sequential(conv, torch.nn.ReLU())
    x = torch.randn(2, 64, 20, 30, device="cuda").half().to(memory_format=torch.channels_last)
    want = model(x)
    assert tdc_torch.convert_depthwise_convs(model) == 1
    assert type(model[0]) is tdc_torch.DepthwiseConv2d and model[0].weight is conv.weight
    got = model(x)
    torch.testing.assert_close(got, want, rtol=1e-2, atol=1e-2)
    got.float().sum().backward()
    assert conv.weight.grad is not None and conv.weight.grad.shape == (64, 1, 7, 7)
    assert conv.bias.grad is not None and torch.isfinite(conv.weight.grad).all()


@pytest.mark.parametrize("K,S", [(3, 1), (3, 2), (5, 1), (5, 2), (7, 1), (7, 2)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_eager_function_matches_custom_op(K, S, dtype):
    """tdc_torch.dwconv in eager mode (an autograd Function calling the
    extension directly) and torch.ops.tdc.dwconv (the custom op, used under
    torch.compile): the same y, dx, dw and db, bit for bit."""
    import tdc_torch
    g = torch.Generator().manual_seed(K * 3 + S)
    x0 = torch.randn(3, 14, 14, 72, generator=g).to(dtype).cuda()
    w0 = (torch.randn(K, K, 72, generator=g) / K).to(dtype).cuda()
    b0 = torch.randn(72, generator=g).to(dtype).cuda()
    outs = []
    for fn in (lambda x, w, b: tdc_torch.dwconv(x, w, b, S, K // 2),
               lambda x, w, b: torch.ops.tdc.dwconv(x, w, b, S, K // 2)):
        x, w, b = (t.clone().requires_grad_() for t in (x0, w0, b0))
        y = fn(x, w, b)
        dy = torch.randn(y.shape, generator=torch.Generator().manual_seed(9)).to(dtype).cuda()
        y.backward(dy)
        outs.append([t.detach().view(torch.int16) for t in (y, x.grad, w.grad, b.grad)])
    for a, b in zip(*outs):
        assert torch.equal(a, b)


@pytest.mark.parametrize("K,S", [(3, 1), (3, 2), (5, 1), (5, 2), (7, 1), (7, 2)])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_module_training_path_matches_custom_op(K, S, dtype):
    """DepthwiseConv2d in eager training (one autograd Function over the
    module's own weight layout) against torch.ops.tdc.dwconv on the re-laid-out
    weight: the same y, x.grad, weight.grad (cast to the parameter dtype) and
    bias.grad, bit for bit."""
    import tdc_torch
    torch.manual_seed(K + S)
    conv = torch.nn.Conv2d(72, 72, K, stride=S, padding=K // 2, groups=72).cuda().to(dtype)
    mod = tdc_torch.DepthwiseConv2d.from_conv2d(conv)
    x0 = torch.randn(3, 72, 14, 15, device="cuda").to(dtype).to(memory_format=torch.channels_last)
    x = x0.clone().requires_grad_()
    y = mod(x)
    gy = torch.randn(y.shape, device="cuda").to(dtype).to(memory_format=torch.channels_last)
    y.backward(gy)
    xr = x0.permute(0, 2, 3, 1).contiguous().requires_grad_()
    wr = conv.weight.detach()[:, 0].permute(1, 2, 0).contiguous().requires_grad_()
    br = conv.bias.detach().clone().requires_grad_()
    yr = torch.ops.tdc.dwconv(xr, wr, br, S, K // 2)
    yr.backward(gy.permute(0, 2, 3, 1).contiguous())
    bits = lambda t: t.detach().contiguous().view(torch.int16)
    assert torch.equal(bits(y.permute(0, 2, 3, 1)), bits(yr))
    assert torch.equal(bits(x.grad.permute(0, 2, 3, 1)), bits(xr.grad))
    assert torch.equal(bits(mod.weight.grad[:, 0].permute(1, 2, 0)), bits(wr.grad))
    assert torch.equal(bits(mod.bias.grad), bits(br.grad))
