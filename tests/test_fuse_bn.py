"""Inference fusion of depthwise convolution + BatchNorm + activation
(`tdc_torch.fuse_depthwise_bn_act`) and the hardswish epilogue it needs for
MobileNetV3.

* the hardswish epilogue: bit for bit with the CPU oracle (fp16 and bf16);
* a folded block (conv -> BatchNorm2d with random statistics -> activation)
  against the unfused PyTorch block, every activation and geometry;
* torchvision MobileNetV2 / V3 in eval mode: every depthwise block fused,
  logits close to the unfused model's (both fp16 on the GPU);
* gradients still flow through a fused module (the activation then runs
  outside the kernel).
"""
import numpy as np
import pytest
import torch
from torch import nn

import oracle
import tdc_torch
import tma_dwconv as T

pytestmark = pytest.mark.gpu


def _bits(t):
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


@pytest.mark.parametrize("K,S", [(3, 1), (3, 2), (5, 1), (5, 2), (7, 1), (7, 2)])
def test_hardswish_epilogue_matches_oracle(K, S):
    g = torch.Generator().manual_seed(K * 10 + S)
    x = (torch.randn(2, 21, 30, 64, generator=g) * 2).half()
    w = (torch.randn(K, K, 64, generator=g) / K).half()
    b = torch.randn(64, generator=g).half()
    y = T.dwconv(x.cuda(), w.cuda(), stride=S, bias=b.cuda(), activation="hardswish")
    want = oracle.dwconv_k_f16(x.numpy(), w.numpy(), K // 2, S, bias=b.numpy(),
                               activation="hardswish")
    assert np.array_equal(_bits(y), want.view(np.uint16))
    xb, wb, bb = x.bfloat16(), w.bfloat16(), b.bfloat16()
    yb = T.dwconv(xb.cuda(), wb.cuda(), stride=S, bias=bb.cuda(), activation="hardswish")
    wantb = oracle.dwconv_k_bf16(_bits(xb), _bits(wb), K // 2, S, bias=_bits(bb),
                                 activation="hardswish")
    assert np.array_equal(_bits(yb), wantb)


def test_hardswish_3x3_general_path_and_residual():
    g = torch.Generator().manual_seed(3)
    x = (torch.randn(2, 16, 40, 72, generator=g) * 3).half()
    w = (torch.randn(3, 3, 72, generator=g) / 3).half()
    r = torch.randn(2, 16, 40, 72, generator=g).half()
    y = T.dwconv3x3(x.cuda(), w.cuda(), 1, residual=r.cuda(), activation="hardswish")
    want = oracle.dwconv_ex_f16(x.numpy(), w.numpy(), 1, residual=r.numpy(), activation="hardswish")
    assert np.array_equal(_bits(y), want.view(np.uint16))


def _randomize_bn(model, seed):
    g = torch.Generator().manual_seed(seed)
    for m in model.modules():
        if isinstance(m, nn.BatchNorm2d):
            c = m.num_features
            m.running_mean.copy_(torch.randn(c, generator=g) * 0.2)
            m.running_var.copy_(torch.rand(c, generator=g) + 0.5)
            m.weight.data.copy_(torch.rand(c, generator=g) + 0.5)
            m.bias.data.copy_(torch.randn(c, generator=g) * 0.2)


@pytest.mark.parametrize("act", [nn.ReLU, nn.ReLU6, nn.SiLU, nn.Hardswish, None])
@pytest.mark.parametrize("K,S", [(3, 1), (5, 2), (7, 1)])
def test_folded_block_matches_pytorch(act, K, S):
    torch.manual_seed(0)
    layers = [nn.Conv2d(64, 64, K, stride=S, padding=K // 2, groups=64, bias=False),
              nn.BatchNorm2d(64)] + ([act()] if act else [])
    block = nn.Sequential(*layers)
    _randomize_bn(block, 1)
    block = block.eval().cuda().half()
    x = torch.randn(2, 64, 33, 47, device="cuda").half().to(memory_format=torch.channels_last)
    with torch.no_grad():
        want = block(x)
        assert tdc_torch.fuse_depthwise_bn_act(block) == 1
        assert type(block[0]) is tdc_torch.DepthwiseConv2d and isinstance(block[1], nn.Identity)
        got = block(x)
    torch.testing.assert_close(got.float(), want.float(), rtol=1e-2, atol=1e-2)


def test_fusion_needs_eval_mode():
    block = nn.Sequential(nn.Conv2d(64, 64, 3, padding=1, groups=64), nn.BatchNorm2d(64)).cuda()
    with pytest.raises(ValueError, match="eval"):
        tdc_torch.fuse_depthwise_bn_act(block)


@pytest.mark.parametrize("arch", ["mobilenet_v2", "mobilenet_v3_small"])
def test_torchvision_mobilenet_end_to_end(arch):
    tv = pytest.importorskip("torchvision")
    torch.manual_seed(0)
    model = getattr(tv.models, arch)(num_classes=100)
    _randomize_bn(model, 2)
    model = model.eval().cuda().half().to(memory_format=torch.channels_last)
    depthwise = sum(1 for m in model.modules() if isinstance(m, nn.Conv2d)
                    and m.groups == m.in_channels == m.out_channels and m.in_channels > 1)
    x = torch.randn(4, 3, 224, 224, device="cuda").half().to(memory_format=torch.channels_last)
    with torch.no_grad():
        want = model(x).float()
        fused = tdc_torch.fuse_depthwise_bn_act(model)
        got = model(x).float()
    assert fused > 0 and fused == depthwise - sum(
        1 for m in model.modules() if isinstance(m, nn.Conv2d) and m.groups == m.in_channels
        == m.out_channels and m.in_channels > 1)
    err = (got - want).abs().max().item()
    assert err <= 2e-2 * want.abs().max().item() + 1e-2, err


def test_fused_module_still_trains():
    torch.manual_seed(0)
    block = nn.Sequential(nn.Conv2d(64, 64, 3, padding=1, groups=64), nn.BatchNorm2d(64),
                          nn.Hardswish())
    _randomize_bn(block, 3)
    block = block.eval().cuda().half()
    tdc_torch.fuse_depthwise_bn_act(block)
    x = torch.randn(2, 64, 20, 30, device="cuda").half().to(memory_format=torch.channels_last)
    with torch.no_grad():
        fused_out = block(x)                       # epilogue in the kernel
    x.requires_grad_()
    y = block(x)                                   # conv + bias op, hardswish outside
    torch.testing.assert_close(y.float(), fused_out.float(), rtol=1e-2, atol=1e-2)
    y.float().sum().backward()
    assert x.grad is not None and block[0].weight.grad is not None
