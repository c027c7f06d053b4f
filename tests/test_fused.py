"""General forward (`dwconv3x3`): C % 8 and the fused epilogue, on the GPU.

Parity bar: bit for bit with the CPU oracle's general forward
(oracle/dwconv_oracle.c: t = conv + bias; t = act(t); t += residual; fp16
RNE) for "none", "relu" and "relu6"; for "silu" (an expf inside) within one
fp16 ulp of the oracle plus 2^-20 of the silu term's size
(oracle.silu_tolerance), with at least 99 % of outputs bit-identical.
"""
import numpy as np
import pytest
import torch

import oracle
import tma_dwconv as T

pytestmark = pytest.mark.gpu


def _inputs(N, H, W, C, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, H, W, C, generator=g).half()
    w = (torch.randn(3, 3, C, generator=g) / 3).half()
    b = torch.randn(C, generator=g).half()
    return x, w, b


def _check(got: torch.Tensor, want: np.ndarray, activation: str, residual=None):
    g = got.cpu().numpy()
    assert g.shape == want.shape
    same = g.view(np.uint16) == want.view(np.uint16)
    if activation == "silu":
        assert same.mean() >= 0.99
        gf, wf = g.astype(np.float32), want.astype(np.float32)
        assert (np.abs(gf - wf) <= oracle.silu_tolerance(wf, residual)).all()
    else:
        assert same.all(), f"{(~same).sum()} outputs differ"


@pytest.mark.parametrize("C", [8, 24, 72, 136, 200, 256])
@pytest.mark.parametrize("pad", [0, 1, 2])
def test_channels_multiple_of_8(C, pad):
    x, w, _ = _inputs(2, 19, 45, C, seed=C + pad)
    y = T.dwconv3x3(x.cuda(), w.cuda(), pad)
    _check(y, oracle.dwconv_f16(x.numpy(), w.numpy(), pad), "none")


@pytest.mark.parametrize("activation", ["none", "relu", "relu6", "silu"])
@pytest.mark.parametrize("with_bias,with_res", [(True, False), (False, True), (True, True)])
@pytest.mark.parametrize("C", [64, 72])
def test_epilogue(activation, with_bias, with_res, C):
    N, H, W, pad = 3, 23, 37, 1
    x, w, b = _inputs(N, H, W, C, seed=7)
    r = torch.randn(N, H, W, C, generator=torch.Generator().manual_seed(9)).half() if with_res else None
    y = T.dwconv3x3(x.cuda(), w.cuda(), pad, bias=b.cuda() if with_bias else None,
                    residual=None if r is None else r.cuda(), activation=activation)
    want = oracle.dwconv_ex_f16(x.numpy(), w.numpy(), pad, b.numpy() if with_bias else None,
                                None if r is None else r.numpy(), activation)
    _check(y, want, activation, None if r is None else r.numpy())


def test_plain_general_forward_equals_ws():
    x, w, _ = _inputs(4, 56, 72, 128, seed=3)
    xd, wd = x.cuda(), w.cuda()
    for n_stage in (2, 3, 4):
        assert torch.equal(T.dwconv3x3(xd, wd, 1, n_stage=n_stage).view(torch.int16),
                           T.dwconv_ws(xd, wd, 1, n_stage).view(torch.int16))


def test_headline_shape_with_epilogue():
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.rand(2, 224, 336, 256, device="cuda", generator=g) * 2 - 1).half()
    w = ((torch.rand(3, 3, 256, device="cuda", generator=g) * 2 - 1) / 3).half()
    b = (torch.rand(256, device="cuda", generator=g) - 0.5).half()
    r = (torch.rand(2, 224, 336, 256, device="cuda", generator=g) - 0.5).half()
    y = T.dwconv3x3(x, w, 1, bias=b, residual=r, activation="relu6")
    want = oracle.dwconv_ex_f16(x.cpu().numpy(), w.cpu().numpy(), 1, b.cpu().numpy(), r.cpu().numpy(),
                                "relu6")
    _check(y, want, "relu6")


def test_argument_errors():
    x, w, b = _inputs(1, 8, 8, 64)
    xd, wd = x.cuda(), w.cuda()
    with pytest.raises(ValueError, match="activation must be one of"):
        T.dwconv3x3(xd, wd, 1, activation="gelu")
    with pytest.raises(ValueError, match=r"C % 8"):
        T.dwconv3x3(xd[..., :12].contiguous(), wd[..., :12].contiguous(), 1)
    with pytest.raises(RuntimeError, match="bias must be"):
        T.dwconv3x3(xd, wd, 1, bias=b[:32].cuda())
    with pytest.raises(RuntimeError, match="residual must be"):
        T.dwconv3x3(xd, wd, 1, residual=xd[:, :4].contiguous())


@pytest.mark.parametrize("activation", ["none", "relu", "relu6", "silu", "hardswish"])
@pytest.mark.parametrize("n_stage", [2, 3, 4])
def test_every_activation_kernel_and_ring_depth(activation, n_stage):
    """The 3x3 stride-1 fp16 epilogue has one kernel per activation and ring
    depth: each against the oracle, with a bias and with a bias + residual."""
    N, H, W, C, pad = 2, 29, 41, 72, 1
    x, w, b = _inputs(N, H, W, C, seed=11 + n_stage)
    r = torch.randn(N, H, W, C, generator=torch.Generator().manual_seed(13)).half()
    for res in (None, r):
        y = T.dwconv3x3(x.cuda(), w.cuda(), pad, bias=b.cuda(),
                        residual=None if res is None else res.cuda(), activation=activation,
                        n_stage=n_stage)
        want = oracle.dwconv_ex_f16(x.numpy(), w.numpy(), pad, b.numpy(),
                                    None if res is None else res.numpy(), activation)
        _check(y, want, activation, None if res is None else res.numpy())
