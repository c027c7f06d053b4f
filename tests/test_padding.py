"""Per-side zero padding (tdc_dwconv_fwd_asym, `tma_dwconv.dwconv(pad=(top,
bottom, left, right))`), TensorFlow-style "same" padding
(`tma_dwconv.same_padding`, `DepthwiseConv2d(padding="same")`) and dilation
(tdc_dwconv_fwd_dilated, `dwconv(dilation=D)`), on the GPU.

Parity bar: bit for bit with the CPU oracle's K x K forward at pad 0 on the
input zero-padded by hand, and for dilation D on the K' = D*(K-1)+1 kernel
with zeros between the taps (padding and the inserted zeros only add exact
zero products to the fp32 chain, which never holds -0, so these are the same
arithmetic in the same order).
"""
import numpy as np
import pytest
import torch
import torch.nn.functional as F

import oracle
import tdc_torch
import tma_dwconv as T

pytestmark = pytest.mark.gpu

GEOMS = [(K, S) for K in (3, 5, 7) for S in (1, 2)]


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _inputs(N, H, W, C, K, seed, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, H, W, C, generator=g).to(dtype)
    w = (torch.randn(K, K, C, generator=g) / K).to(dtype)
    b = torch.randn(C, generator=g).to(dtype)
    return x, w, b


def _want(x, w, pads, S, **epi):
    t, b, l, r = pads
    xp = np.pad(x.numpy(), ((0, 0), (t, b), (l, r), (0, 0)))
    return oracle.dwconv_k_f16(xp, w.numpy(), 0, S, **epi).view(np.uint16)


@pytest.mark.parametrize("K,S", GEOMS)
@pytest.mark.parametrize("N,H,W,C", [(2, 20, 37, 64), (3, 14, 14, 200), (1, 9, 40, 16)])
def test_per_side_padding_matches_oracle(K, S, N, H, W, C):
    x, w, b = _inputs(N, H, W, C, K, seed=K * 10 + S + C)
    xc, wc, bc = x.cuda(), w.cuda(), b.cuda()
    for pads in [(0, 1, 0, 1), (1, 2, 1, 2), (K // 2, 0, 0, K // 2), (2, 0, 1, 3),
                 T.same_padding(H, W, K, S)]:
        want = _want(x, w, pads, S, bias=b.numpy(), activation="relu6")
        for n_stage in (None, T.DWCONV_STAGES[(K, S)]):
            y = T.dwconv(xc, wc, pads, stride=S, bias=bc, activation="relu6", n_stage=n_stage)
            assert np.array_equal(_bits(y), want), (pads, n_stage)
        y = T._C.dwconv_k_pads(xc, wc, bc, None, S, 1, *pads, T.ACTIVATIONS["relu6"], 0)
        assert np.array_equal(_bits(y), want), pads


@pytest.mark.parametrize("K,S", GEOMS)
def test_per_side_padding_bf16(K, S):
    x, w, _ = _inputs(2, 23, 30, 72, K, seed=5, dtype=torch.bfloat16)
    pads = T.same_padding(23, 30, K, S)
    xp = np.pad(_bits(x), ((0, 0), (pads[0], pads[1]), (pads[2], pads[3]), (0, 0)))
    want = oracle.dwconv_k_bf16(xp, _bits(w), 0, S)
    y = T.dwconv(x.cuda(), w.cuda(), pads, stride=S)
    assert y.dtype == torch.bfloat16 and np.array_equal(_bits(y), want)


@pytest.mark.parametrize("K,S", GEOMS)
@pytest.mark.parametrize("H,W", [(112, 112), (15, 22)])
def test_same_module_inference_and_training(K, S, H, W):
    """DepthwiseConv2d(padding="same"): inference runs the per-side kernels
    (bit for bit with explicit padding + pad 0); training pads explicitly and
    its gradients match the explicit-padding module's."""
    torch.manual_seed(K + S)
    m = tdc_torch.DepthwiseConv2d(32, K, S, padding="same").cuda()
    ref = tdc_torch.DepthwiseConv2d(32, K, S, padding=0).cuda()
    ref.weight.data.copy_(m.weight.data)
    ref.bias.data.copy_(m.bias.data)
    x = torch.randn(2, 32, H, W, device="cuda").half().to(memory_format=torch.channels_last)
    t, b, l, r = T.same_padding(H, W, K, S)
    xp = F.pad(x, (l, r, t, b))
    with torch.no_grad():
        y = m(x)
        assert tuple(y.shape[2:]) == (-(-H // S), -(-W // S))
        assert torch.equal(y.view(torch.int16), ref(xp).view(torch.int16))
    xa = x.clone().requires_grad_()
    ya = m(xa)
    gy = torch.randn_like(ya)
    ya.backward(gy)
    xb = x.clone().requires_grad_()
    ref(F.pad(xb, (l, r, t, b))).backward(gy)
    torch.testing.assert_close(m.weight.grad, ref.weight.grad)
    torch.testing.assert_close(xa.grad, xb.grad)


def test_converted_same_padding_conv():
    torch.manual_seed(0)
    conv = torch.nn.Conv2d(64, 64, 5, padding="same", groups=64).cuda().half()
    model = torch.nn.Sequential(conv)
    x = torch.randn(2, 64, 19, 26, device="cuda").half().to(memory_format=torch.channels_last)
    with torch.no_grad():
        want = model(x)
        assert tdc_torch.convert_depthwise_convs(model) == 1
        got = model(x)
    assert model[0].padding == 2
    torch.testing.assert_close(got.float(), want.float(), rtol=2e-3, atol=2e-3)


def _dilated(w, D):
    K, _, C = w.shape
    Ke = D * (K - 1) + 1
    wd = np.zeros((Ke, Ke, C), dtype=w.dtype)
    wd[::D, ::D] = w
    return wd


@pytest.mark.parametrize("K,S", GEOMS)
@pytest.mark.parametrize("D", [2, 3])
@pytest.mark.parametrize("N,H,W,C", [(2, 21, 30, 64), (3, 17, 17, 200), (1, 33, 12, 16)])
def test_dilated_matches_oracle(K, S, D, N, H, W, C):
    x, w, b = _inputs(N, H, W, C, K, seed=K + S + D + C)
    Ke = D * (K - 1) + 1
    for pads in [(Ke // 2,) * 4, (0, 1, 2, 0), T.same_padding(H, W, Ke, S)]:
        t, bo, l, r = pads
        if H + t + bo < Ke or W + l + r < Ke:
            continue
        xp = np.pad(x.numpy(), ((0, 0), (t, bo), (l, r), (0, 0)))
        want = oracle.dwconv_k_f16(xp, _dilated(w.numpy(), D), 0, S, bias=b.numpy(),
                                   activation="silu" if K == 3 else "relu").view(np.uint16)
        act = "silu" if K == 3 else "relu"
        y = T.dwconv(x.cuda(), w.cuda(), pads, stride=S, bias=b.cuda(), activation=act,
                     dilation=D)
        if act == "silu":  # the kernels' fast exp / divide: within the oracle's silu bound
            got = y.float().cpu().numpy()
            ref = want.view(np.float16).astype(np.float32)
            assert (np.abs(got - ref) <= oracle.silu_tolerance(ref)).all(), pads
        else:
            assert np.array_equal(_bits(y), want), pads


def test_dilated_bf16():
    x, w, _ = _inputs(2, 19, 26, 72, 5, seed=9, dtype=torch.bfloat16)
    xp = np.pad(_bits(x), ((0, 0), (4, 4), (4, 4), (0, 0)))
    want = oracle.dwconv_k_bf16(xp, _dilated(_bits(w), 2), 0, 1)
    y = T.dwconv(x.cuda(), w.cuda(), 4, dilation=2)
    assert y.dtype == torch.bfloat16 and np.array_equal(_bits(y), want)


def test_dilated_module_is_inference_only():
    m = tdc_torch.DepthwiseConv2d(64, 3, 1, dilation=2).cuda()
    x = torch.randn(1, 64, 9, 9, device="cuda").half().to(memory_format=torch.channels_last)
    with torch.no_grad():
        assert m(x).shape == (1, 64, 9, 9)
    with pytest.raises(RuntimeError, match="not implemented"):
        m(x.requires_grad_())


def test_deeplabv3_mobilenet_end_to_end():
    """torchvision's DeepLabV3-MobileNetV3-Large (dilated depthwise layers in
    the last stages) with every depthwise + BatchNorm + activation fused,
    against the unfused fp16 model."""
    seg = pytest.importorskip("torchvision.models.segmentation")
    torch.manual_seed(0)
    model = seg.deeplabv3_mobilenet_v3_large(weights=None, weights_backbone=None,
                                             num_classes=21, aux_loss=False)
    for mod in model.modules():
        if isinstance(mod, torch.nn.BatchNorm2d):
            mod.running_mean.uniform_(-0.2, 0.2)
            mod.running_var.uniform_(0.5, 1.5)
    model = model.eval().cuda().half().to(memory_format=torch.channels_last)
    dilated = sum(1 for mod in model.modules() if isinstance(mod, torch.nn.Conv2d)
                  and mod.groups == mod.in_channels > 1 and mod.dilation[0] > 1)
    x = torch.randn(2, 3, 224, 224, device="cuda").half().to(memory_format=torch.channels_last)
    with torch.no_grad():
        want = model(x)["out"].float()
        fused = tdc_torch.fuse_depthwise_bn_act(model)
        got = model(x)["out"].float()
    assert dilated > 0 and fused >= 15
    assert not any(isinstance(mod, torch.nn.Conv2d) and mod.groups == mod.in_channels > 1
                   for mod in model.modules())
    err = (got - want).abs().max().item()
    assert err <= 2e-2 * want.abs().max().item() + 1e-2, err
