"""bfloat16 tensors through the K x K forward and the backward (beyond the
reference's fp16-only surface).

* forward, every geometry (3x3 / 5x5 / 7x7, stride 1 / 2) and the fused
  epilogue: bit for bit with the CPU oracle's bfloat16 restatement
  (oracle_dwconv_ex_bf16: the same fp32 chain, one bfloat16 rounding), and
  within one bfloat16 ulp of float32 PyTorch;
* data gradient, stride 1 and 2: bit for bit with oracle_dwconv_bwd_data_bf16 /
  oracle_dwconv_bwd_data_s2_bf16;
* weight gradient: within 5e-4 of sum |x*dy| of the float64 oracle (bfloat16
  values are exact in float64), bit-reproducible;
* autograd through torch.ops.tdc.dwconv and the module on bfloat16 inputs.
"""
import numpy as np
import pytest
import torch

import oracle
import tdc_torch
import tma_dwconv as T

pytestmark = pytest.mark.gpu

GEOMETRIES = [(3, 1), (3, 2), (5, 1), (5, 2), (7, 1), (7, 2)]
SHAPES = [(2, 16, 16, 64), (3, 19, 45, 72), (1, 12, 13, 8), (2, 33, 70, 128)]


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _tensors(N, H, W, C, K, seed=0, stride=1, pad=None):
    pad = K // 2 if pad is None else pad
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, H, W, C, generator=g).bfloat16()
    w = (torch.randn(K, K, C, generator=g) / K).bfloat16()
    P, Q = (H + 2 * pad - K) // stride + 1, (W + 2 * pad - K) // stride + 1
    dy = torch.randn(N, P, Q, C, generator=g).bfloat16()
    return x, w, dy


def _bf16_ulp(v: np.ndarray) -> np.ndarray:
    a = np.abs(np.asarray(v, dtype=np.float32))
    return np.exp2(np.floor(np.log2(np.maximum(a, 2.0 ** -126))) - 7).astype(np.float32)


@pytest.mark.parametrize("K,S", GEOMETRIES)
@pytest.mark.parametrize("N,H,W,C", SHAPES)
def test_forward_matches_oracle(K, S, N, H, W, C):
    x, w, _ = _tensors(N, H, W, C, K, seed=K * 10 + S + C)
    want = oracle.dwconv_k_bf16(_bits(x), _bits(w), K // 2, S)
    for n_stage in (2, 3, 4):
        y = T.dwconv(x.cuda(), w.cuda(), stride=S, n_stage=n_stage)
        assert y.dtype == torch.bfloat16
        assert np.array_equal(_bits(y), want), n_stage


@pytest.mark.parametrize("K,S", GEOMETRIES)
def test_forward_within_one_ulp_of_float32(K, S):
    x, w, _ = _tensors(4, 40, 56, 64, K, seed=7)
    y = T.dwconv(x.cuda(), w.cuda(), stride=S).float().cpu().numpy()
    ref = torch.nn.functional.conv2d(x.float().permute(0, 3, 1, 2), w.float().permute(2, 0, 1)
                                     .unsqueeze(1), stride=S, padding=K // 2, groups=64)
    ref = ref.permute(0, 2, 3, 1).numpy()
    assert (np.abs(y - ref) <= _bf16_ulp(ref) + 1e-6).all()


@pytest.mark.parametrize("K,S", GEOMETRIES)
@pytest.mark.parametrize("activation", ["none", "relu", "relu6"])
def test_fused_epilogue_matches_oracle(K, S, activation):
    x, w, _ = _tensors(2, 21, 30, 64, K, seed=3)
    g = torch.Generator().manual_seed(4)
    b = torch.randn(64, generator=g).bfloat16()
    P, Q = (21 + 2 * (K // 2) - K) // S + 1, (30 + 2 * (K // 2) - K) // S + 1
    r = torch.randn(2, P, Q, 64, generator=g).bfloat16()
    y = T.dwconv(x.cuda(), w.cuda(), stride=S, bias=b.cuda(), residual=r.cuda(),
                 activation=activation)
    want = oracle.dwconv_k_bf16(_bits(x), _bits(w), K // 2, S, bias=_bits(b), residual=_bits(r),
                                activation=activation)
    assert np.array_equal(_bits(y), want)


def test_fused_silu_within_one_ulp():
    x, w, _ = _tensors(2, 21, 30, 64, 3, seed=5)
    b = torch.randn(64, generator=torch.Generator().manual_seed(6)).bfloat16()
    y = T.dwconv(x.cuda(), w.cuda(), bias=b.cuda(), activation="silu")
    want = oracle.bf16_to_f32(oracle.dwconv_k_bf16(_bits(x), _bits(w), 1, 1, bias=_bits(b),
                                                   activation="silu"))
    got = oracle.bf16_to_f32(_bits(y))
    assert (np.abs(got - want) <= _bf16_ulp(want)).all()


@pytest.mark.parametrize("K", [3, 5, 7])
@pytest.mark.parametrize("S", [1, 2])
def test_data_gradient_matches_oracle(K, S):
    for (N, H, W, C) in ((2, 16, 16, 64), (3, 19, 45, 72), (1, 13, 12, 8)):
        for pad in ((K // 2, 0, K - 1) if S == 1 else (K // 2, 0, K)):
            x, w, dy = _tensors(N, H, W, C, K, seed=pad + K, stride=S, pad=pad)
            want = oracle.dwconv_bwd_data_bf16(_bits(dy), _bits(w), pad, S, H, W)
            for n_stage in (2, 4):
                dx = T._C.dwconv_bwd_data(dy.cuda(), w.cuda(), pad, S, n_stage, H, W)
                assert dx.dtype == torch.bfloat16 and tuple(dx.shape) == (N, H, W, C)
                assert np.array_equal(_bits(dx), want), (N, H, W, C, pad, n_stage)


@pytest.mark.parametrize("K", [3, 5, 7])
@pytest.mark.parametrize("S", [1, 2])
def test_weight_gradient_close_to_float64(K, S):
    x, w, dy = _tensors(3, 19, 45, 72, K, seed=11, stride=S)
    xf = x.float().numpy().astype(np.float64)
    dyf = dy.float().numpy().astype(np.float64)
    ref = oracle.dwconv_bwd_weight_f64(xf, dyf, K // 2, K, stride=S)
    scale = oracle.dwconv_bwd_weight_f64(np.abs(xf), np.abs(dyf), K // 2, K, stride=S)
    for n_stage in (2, 3, 4):
        dw = T._C.dwconv_bwd_weight(x.cuda(), dy.cuda(), K, K // 2, S, n_stage).cpu().numpy()
        assert dw.dtype == np.float32 and dw.shape == (K, K, 72)
        assert (np.abs(dw - ref) <= 5e-4 * scale + 1e-6).all(), n_stage
    a = T._C.dwconv_bwd_weight(x.cuda(), dy.cuda(), K, K // 2, S, 2)
    b = T._C.dwconv_bwd_weight(x.cuda(), dy.cuda(), K, K // 2, S, 2)
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))


def test_mixed_dtypes_are_rejected():
    x, w, dy = _tensors(1, 8, 8, 64, 3)
    with pytest.raises(ValueError, match="same dtype"):
        T.dwconv(x.cuda(), w.half().cuda())
    with pytest.raises(RuntimeError, match="both fp16 or both bf16"):
        T._C.dwconv_bwd_weight(x.cuda(), dy.half().cuda(), 3, 1, 1, 2)
    with pytest.raises(RuntimeError, match="x's dtype"):
        T.dwconv(x.cuda(), w.cuda(), bias=torch.zeros(64, device="cuda").half())


@pytest.mark.parametrize("K,S", GEOMETRIES)
def test_autograd_custom_op_with_bias(K, S):
    N, H, W, C, pad = 2, 21, 30, 64, K // 2
    x, w, _ = _tensors(N, H, W, C, K, seed=13)
    b = torch.randn(C, generator=torch.Generator().manual_seed(14)).bfloat16()
    x, w, b = x.cuda().requires_grad_(), w.cuda().requires_grad_(), b.cuda().requires_grad_()
    y = torch.ops.tdc.dwconv(x, w, b, S, pad)
    dy = torch.randn(y.shape, generator=torch.Generator().manual_seed(15)).bfloat16().cuda()
    y.backward(dy)
    xt = x.detach().float().permute(0, 3, 1, 2).requires_grad_()
    wt = w.detach().float().permute(2, 0, 1).unsqueeze(1).requires_grad_()
    bt = b.detach().float().requires_grad_()
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        ry = torch.nn.functional.conv2d(xt, wt, bt, stride=S, padding=pad, groups=C)
        ry.backward(dy.float().permute(0, 3, 1, 2))
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    ry = ry.detach().permute(0, 2, 3, 1)
    rdx = xt.grad.permute(0, 2, 3, 1)
    tol = lambda r: torch.from_numpy(_bf16_ulp(r.cpu().numpy())).cuda() + 1e-3
    assert y.dtype == x.grad.dtype == w.grad.dtype == b.grad.dtype == torch.bfloat16
    assert ((y.float() - ry).abs() <= tol(ry)).all()
    assert ((x.grad.float() - rdx).abs() <= tol(rdx)).all()
    torch.testing.assert_close(w.grad.float(), wt.grad[:, 0].permute(1, 2, 0), rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(b.grad.float(), bt.grad, rtol=1e-2, atol=5e-2)


def test_module_runs_and_trains_in_bf16():
    torch.manual_seed(0)
    conv = torch.nn.Conv2d(64, 64, 5, stride=2, padding=2, groups=64, bias=True).cuda().bfloat16()
    model = torch.nn.Sequential(conv)
    x = torch.randn(2, 64, 21, 30, device="cuda").bfloat16().to(memory_format=torch.channels_last)
    x.requires_grad_()
    want = model(x)
    gy = torch.randn(want.shape, device="cuda").bfloat16()
    want.backward(gy)
    gx_want, gw_want = x.grad.clone(), conv.weight.grad.clone()
    x.grad = conv.weight.grad = conv.bias.grad = None
    assert tdc_torch.convert_depthwise_convs(model) == 1
    got = model(x)
    assert got.dtype == torch.bfloat16
    torch.testing.assert_close(got.float(), want.float(), rtol=2e-2, atol=2e-2)
    got.backward(gy)
    torch.testing.assert_close(x.grad.float(), gx_want.float(), rtol=2e-2, atol=2e-2)
    torch.testing.assert_close(conv.weight.grad.float(), gw_want.float(), rtol=5e-2, atol=5e-1)
