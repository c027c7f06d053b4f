"""K x K taps (3, 5, 7) and stride 2 (`tma_dwconv.dwconv`), on the GPU.

The reference kernel is 3x3 stride 1, though its parameter block carries a
stride (csrc/common.cuh:38-40).  Parity bar, as for the 3x3 path: bit for bit
with the CPU oracle's K x K forward (oracle/dwconv_oracle.c,
oracle_dwconv_ex_f16: fp32 chain in (r, s) order from +0, then bias / act /
residual, one fp16 RNE) for every activation but "silu", which stays within
oracle.silu_tolerance (one fp16 ulp plus 2^-20 of the silu term's size)
with at least 99 % of outputs bit-identical.  Against fp32
torch conv2d the outputs are within one fp16 ulp + 1e-3.
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
import tma_dwconv as T

pytestmark = pytest.mark.gpu


def _inputs(N, H, W, C, K, seed):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, H, W, C, generator=g).half()
    w = (torch.randn(K, K, C, generator=g) / K).half()
    b = torch.randn(C, generator=g).half()
    return x, w, b


def _same_bits(got: torch.Tensor, want: np.ndarray):
    g = got.cpu().numpy()
    assert g.shape == want.shape
    diff = g.view(np.uint16) != want.view(np.uint16)
    assert not diff.any(), f"{diff.sum()} of {diff.size} outputs differ"


GEOMS = [(K, S) for K in (3, 5, 7) for S in (1, 2)]


@pytest.mark.parametrize("K,S", GEOMS)
@pytest.mark.parametrize("N,H,W,C,pad", [
    (2, 19, 45, 64, None),     # odd sizes, W past one 32-column strip
    (1, 33, 70, 72, 0),        # partial channel block, no padding
    (3, 12, 9, 8, None),       # one channel pair block, narrow image
    (1, 40, 100, 136, 1),      # pad below K // 2
])
def test_matches_oracle(K, S, N, H, W, C, pad):
    pad = K // 2 if pad is None else pad
    x, w, _ = _inputs(N, H, W, C, K, seed=K * 100 + S * 10 + C)
    y = T.dwconv(x.cuda(), w.cuda(), pad, stride=S)
    _same_bits(y, oracle.dwconv_k_f16(x.numpy(), w.numpy(), pad, S))


@pytest.mark.parametrize("K,S", GEOMS)
def test_pad_larger_than_half_the_taps(K, S):
    pad = K // 2 + 2
    x, w, _ = _inputs(2, 11, 23, 64, K, seed=5)
    y = T.dwconv(x.cuda(), w.cuda(), pad, stride=S)
    _same_bits(y, oracle.dwconv_k_f16(x.numpy(), w.numpy(), pad, S))


@pytest.mark.parametrize("K,S", GEOMS)
def test_single_output_row_and_column(K, S):
    # H + 2*pad == K: exactly one output row; W likewise one output column
    x, w, _ = _inputs(3, K, K, 64, K, seed=11)
    y = T.dwconv(x.cuda(), w.cuda(), 0, stride=S)
    assert y.shape == (3, 1, 1, 64)
    _same_bits(y, oracle.dwconv_k_f16(x.numpy(), w.numpy(), 0, S))


@pytest.mark.parametrize("K,S", [(5, 2), (7, 1), (7, 2), (3, 2)])
def test_many_segments(K, S):
    # enough strips that the persistent grid takes several waves plus a banded tail
    x, w, _ = _inputs(6, 96, 200, 256, K, seed=21)
    y = T.dwconv(x.cuda(), w.cuda(), K // 2, stride=S)
    _same_bits(y, oracle.dwconv_k_f16(x.numpy(), w.numpy(), K // 2, S))


@pytest.mark.parametrize("K,S", GEOMS)
@pytest.mark.parametrize("activation", ["none", "relu", "relu6", "silu"])
def test_epilogue(K, S, activation):
    N, H, W, C = 2, 21, 38, 72
    pad = K // 2
    x, w, b = _inputs(N, H, W, C, K, seed=3)
    P, Q = oracle.output_hw_k(H, W, K, S, pad)
    r = torch.randn(N, P, Q, C, generator=torch.Generator().manual_seed(4)).half()
    y = T.dwconv(x.cuda(), w.cuda(), pad, stride=S, bias=b.cuda(), residual=r.cuda(),
                 activation=activation)
    want = oracle.dwconv_k_f16(x.numpy(), w.numpy(), pad, S, b.numpy(), r.numpy(), activation)
    if activation == "silu":
        g = y.cpu().numpy()
        assert (g.view(np.uint16) == want.view(np.uint16)).mean() >= 0.99
        assert (np.abs(g.astype(np.float32) - want.astype(np.float32))
                <= oracle.silu_tolerance(want, r.numpy())).all()
    else:
        _same_bits(y, want)


@pytest.mark.parametrize("K,S", GEOMS)
def test_stages_agree_and_match_fp32_conv(K, S):
    x, w, _ = _inputs(2, 30, 50, 128, K, seed=8)
    xd, wd = x.cuda(), w.cuda()
    ys = [T.dwconv(xd, wd, K // 2, stride=S, n_stage=ns) for ns in (2, 3, 4)]
    for y in ys[1:]:
        assert torch.equal(y.view(torch.int16), ys[0].view(torch.int16))
    ref = F.conv2d(x.float().permute(0, 3, 1, 2), w.float().permute(2, 0, 1).unsqueeze(1),
                   stride=S, padding=K // 2, groups=128).permute(0, 2, 3, 1).numpy()
    got = ys[0].cpu().float().numpy()
    assert (np.abs(got - ref) <= oracle.f16_ulp(ref) + 1e-3).all()


def test_3x3_stride_1_is_dwconv3x3():
    x, w, b = _inputs(2, 40, 64, 64, 3, seed=1)
    xd, wd, bd = x.cuda(), w.cuda(), b.cuda()
    assert torch.equal(T.dwconv(xd, wd, 1, bias=bd, activation="relu").view(torch.int16),
                       T.dwconv3x3(xd, wd, 1, bias=bd, activation="relu").view(torch.int16))


def test_argument_errors():
    x, w, _ = _inputs(1, 16, 16, 64, 5, seed=0)
    xd, wd = x.cuda(), w.cuda()
    with pytest.raises(ValueError, match="stride must be 1 or 2"):
        T.dwconv(xd, wd, 2, stride=3)
    with pytest.raises(ValueError, match="K in"):
        T.dwconv(xd, wd[:4, :4].contiguous(), 2)
    with pytest.raises(ValueError, match="C % 8"):
        T.dwconv(xd[..., :12].contiguous(), wd[..., :12].contiguous(), 2)
    with pytest.raises(RuntimeError, match="residual must be"):
        T.dwconv(xd, wd, 2, stride=2, residual=xd)
    with pytest.raises(RuntimeError, match="input too small"):
        T.dwconv(xd[:, :2, :2].contiguous(), wd, 1)


@pytest.mark.parametrize("K,S", GEOMS)
def test_custom_op_with_bias(K, S):
    import tdc_torch
    x, w, b = _inputs(2, 17, 29, 64, K, seed=12)
    y = torch.ops.tdc.dwconv(x.cuda(), w.cuda(), b.cuda(), S, K // 2)
    want = oracle.dwconv_k_f16(x.numpy(), w.numpy(), K // 2, S, b.numpy())
    _same_bits(y, want)
    assert tdc_torch.dwconv(x.cuda(), w.cuda(), None, S).shape == want.shape


def test_custom_op_backward_3x3_with_bias():
    x, w, b = _inputs(2, 16, 24, 64, 3, seed=13)
    xd, wd, bd = x.cuda().requires_grad_(), w.cuda().requires_grad_(), b.cuda().requires_grad_()
    y = torch.ops.tdc.dwconv(xd, wd, bd, 1, 1)
    dy = torch.randn(y.shape, generator=torch.Generator().manual_seed(14)).half().cuda()
    y.backward(dy)
    assert torch.equal(xd.grad, torch.ops.tdc.dwconv3x3_bwd_data(dy, wd.detach(), 1))
    assert torch.equal(wd.grad, torch.ops.tdc.dwconv3x3_bwd_weight(xd.detach(), dy, 1).half())
    torch.testing.assert_close(bd.grad.float(), dy.float().sum((0, 1, 2)), rtol=1e-3, atol=1e-2)


def test_custom_op_backward_at_stride_2_uses_the_stride_2_kernels():
    x, w, _ = _inputs(1, 13, 12, 64, 5, seed=15)
    xd, wd = x.cuda().requires_grad_(), w.cuda().requires_grad_()
    y = torch.ops.tdc.dwconv(xd, wd, None, 2, 2)
    dy = torch.randn(y.shape, generator=torch.Generator().manual_seed(16)).half().cuda()
    y.backward(dy)
    assert xd.grad.shape == xd.shape and wd.grad.shape == wd.shape
    assert torch.equal(xd.grad, T._C.dwconv_bwd_data(dy, wd.detach(), 2, 2, 2, 13, 12))
    assert torch.equal(wd.grad, T._C.dwconv_bwd_weight(xd.detach(), dy, 5, 2, 2, 2).half())


def test_module_conversion_forward_only():
    import tdc_torch
    torch.manual_seed(0)
    model = torch.nn.Sequential(
        torch.nn.Conv2d(64, 64, 7, padding=3, groups=64),
        torch.nn.ReLU(),
        torch.nn.Conv2d(64, 64, 5, stride=2, padding=2, groups=64),
        torch.nn.Conv2d(64, 64, 3, stride=2, padding=1, groups=64, bias=False),
    ).cuda().half()
    x = torch.randn(2, 64, 33, 47, device="cuda").half().to(memory_format=torch.channels_last)
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        with torch.no_grad():
            want = model.float()(x.float())
            model.half()
            assert tdc_torch.convert_depthwise_convs(model, forward_only=True) == 3
            got = model(x)
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    assert got.is_contiguous(memory_format=torch.channels_last)
    torch.testing.assert_close(got.float(), want, rtol=1e-2, atol=1e-2)
