"""Python API argument checks, on the host (no GPU needed).

The checks and ValueError messages must be those of the reference's
tma_dwconv.py:39-53, 74-77 and 106-109, in the same order, so callers that
match on them keep working.  Tensors that pass the CUDA check are stood in
for by a small object exposing the attributes the checks read.
"""
import pytest
import torch

import tma_dwconv as T


class FakeCuda:
    def __init__(self, shape, dtype=torch.float16, contiguous=True):
        self.shape = tuple(shape)
        self.dtype = dtype
        self.is_cuda = True
        self._c = contiguous

    def dim(self):
        return len(self.shape)

    def is_contiguous(self):
        return self._c


X = FakeCuda((2, 16, 16, 64))
W = FakeCuda((3, 3, 64))


@pytest.mark.parametrize("x,w,pad,msg", [
    (torch.zeros(2, 16, 16, 64, dtype=torch.float16), W, 1, "x and w must be CUDA tensors"),
    (FakeCuda((2, 16, 16, 64), torch.float32), W, 1, "x and w must be fp16"),
    (X, FakeCuda((3, 3, 64), torch.bfloat16), 1, "x and w must be fp16"),
    (FakeCuda((16, 16, 64)), W, 1, r"x must be \[N,H,W,C\], got shape \(16, 16, 64\)"),
    (X, FakeCuda((9, 64)), 1, r"w must be \[R,S,C\], got shape \(9, 64\)"),
    (X, FakeCuda((3, 3, 32)), 1, "x and w must agree on C"),
    (FakeCuda((2, 16, 16, 64), contiguous=False), W, 1, "x and w must be contiguous"),
    (X, W, -1, "pad must be non-negative"),
])
def test_check_messages(x, w, pad, msg):
    for fn in (T.dwconv_v0, T.dwconv_ws, T.dwconv_ws_probe):
        with pytest.raises(ValueError, match=msg):
            fn(x, w, pad)


def test_ws_specific_checks():
    x, w = FakeCuda((2, 16, 16, 96)), FakeCuda((3, 3, 96))
    with pytest.raises(ValueError, match=r"dwconv_ws requires C % 64 == 0"):
        T.dwconv_ws(x, w, 1)
    with pytest.raises(ValueError, match=r"dwconv_ws_probe requires C % 64 == 0"):
        T.dwconv_ws_probe(x, w, 1)
    for bad in (1, 5, 0):
        with pytest.raises(ValueError, match=r"n_stage must be one of \{2, 3, 4\}, got %d" % bad):
            T.dwconv_ws(X, W, 1, bad)


def test_ref_dwconv_on_cpu_matches_layout_contract():
    torch.manual_seed(0)
    x = torch.randn(2, 9, 11, 64)
    w = torch.randn(3, 3, 64)
    y = T.ref_dwconv(x, w, 1)
    assert y.shape == (2, 9, 11, 64) and y.is_contiguous()
    ref = torch.nn.functional.conv2d(x.permute(0, 3, 1, 2), w.permute(2, 0, 1).unsqueeze(1), padding=1,
                                     groups=64).permute(0, 2, 3, 1)
    torch.testing.assert_close(y, ref)
    with pytest.raises(ValueError, match="channel mismatch"):
        T.ref_dwconv(x, torch.randn(3, 3, 32), 1)
    with pytest.raises(ValueError, match=r"x must be \[N,H,W,C\] and w must be \[R,S,C\]"):
        T.ref_dwconv(x[0], w, 1)


def test_extension_surface():
    for name in ("dwconv_v0", "dwconv_ws", "dwconv_ws_probe", "dwconv_ws_out", "device_status",
                 "set_wait_timeout_ns", "consumer_warps", "dwconv_ws_withhold"):
        assert hasattr(T._C, name), name
    assert T.CONSUMER_WARPS == 4
    assert "libtdc_sm100" not in T._C.__file__ and T._C.__file__.startswith(T.__file__.rsplit("/", 1)[0])


def test_dwconv_kxk_checks():
    x, w5 = FakeCuda((2, 16, 16, 64)), FakeCuda((5, 5, 64))
    with pytest.raises(ValueError, match="stride must be 1 or 2, got 3"):
        T.dwconv(x, w5, 2, stride=3)
    with pytest.raises(ValueError, match=r"K in \{3, 5, 7\}"):
        T.dwconv(x, FakeCuda((4, 4, 64)), 2)
    with pytest.raises(ValueError, match=r"K in \{3, 5, 7\}"):
        T.dwconv(x, FakeCuda((5, 3, 64)), 2)
    with pytest.raises(ValueError, match=r"dwconv requires C % 8 == 0"):
        T.dwconv(FakeCuda((2, 16, 16, 12)), FakeCuda((5, 5, 12)), 2)
    with pytest.raises(ValueError, match="activation must be one of"):
        T.dwconv(x, w5, 2, activation="gelu")
    with pytest.raises(ValueError, match=r"n_stage must be one of \{2, 3, 4\}, got 5"):
        T.dwconv(x, w5, 2, n_stage=5)
    with pytest.raises(ValueError, match="pad must be non-negative"):
        T.dwconv(x, w5, -1)
    assert set(T.DWCONV_STAGES) == {(k, s) for k in (3, 5, 7) for s in (1, 2)}
    assert hasattr(T._C, "dwconv_k")


def test_convert_depthwise_convs_eligibility():
    import tdc_torch
    nn = torch.nn
    model = nn.Sequential(
        nn.Conv2d(64, 64, 3, padding=1, groups=64),             # converted
        nn.Conv2d(64, 64, 7, padding=3, groups=64),             # converted
        nn.Conv2d(64, 64, 5, stride=2, padding=2, groups=64),   # converted (stride 2)
        nn.Sequential(nn.Conv2d(64, 64, 3, stride=2, padding=1, groups=64)),  # nested: converted
        nn.Conv2d(64, 64, 3, padding=1, groups=64, dilation=2),  # dilated: forward_only
        nn.Conv2d(64, 64, 3, padding=1, groups=32),              # not depthwise: never
        nn.Conv2d(12, 12, 3, padding=1, groups=12),              # C % 8 != 0: never
        nn.Conv2d(64, 64, 9, padding=4, groups=64),              # 9x9: never
        nn.Conv2d(64, 64, (3, 5), padding=(1, 2), groups=64),    # non-square: never
    )
    assert tdc_torch.convert_depthwise_convs(model) == 4  # every geometry has a backward
    assert isinstance(model[0], tdc_torch.DepthwiseConv3x3)
    assert type(model[1]) is tdc_torch.DepthwiseConv2d and model[1].kernel_size == 7
    assert model[2].stride == 2 and model[2].padding == 2 and model[3][0].stride == 2
    assert tdc_torch.convert_depthwise_convs(model) == 0  # nothing left for training
    # inference only: the dilated conv too
    assert tdc_torch.convert_depthwise_convs(model, forward_only=True) == 1
    assert type(model[4]) is tdc_torch.DepthwiseConv3x3 and model[4].dilation == 2
    assert all(isinstance(m, nn.Conv2d) for m in list(model)[5:])
    with pytest.raises(ValueError, match="kernel_size must be 3, 5 or 7"):
        tdc_torch.DepthwiseConv2d(64, 9)


def test_convs_that_add_to_conv2d_are_not_converted():
    """A depthwise conv whose module does more than nn.Conv2d's computation
    keeps it: a subclass that pads in forward (like timm's Conv2dSame), a
    parametrized weight (weight norm) and a conv with a forward hook.  A
    subclass that only adds attributes is still converted."""
    import tdc_torch
    nn = torch.nn

    class PadInForward(nn.Conv2d):  # "same" padding done by hand, as in TF ports
        def forward(self, x):
            return super().forward(nn.functional.pad(x, (0, 1, 0, 1)))

    class Tagged(nn.Conv2d):  # computation unchanged
        tag = "dw"

    hooked = nn.Conv2d(64, 64, 3, padding=1, groups=64)
    hooked.register_forward_hook(lambda *a: None)
    normed = nn.utils.parametrizations.weight_norm(nn.Conv2d(64, 64, 3, padding=1, groups=64))
    model = nn.Sequential(PadInForward(64, 64, 3, stride=2, groups=64), normed, hooked,
                          Tagged(64, 64, 3, padding=1, groups=64))
    assert tdc_torch.convert_depthwise_convs(model) == 1
    assert type(model[0]) is PadInForward and type(model[2]) is nn.Conv2d
    assert isinstance(model[3], tdc_torch.DepthwiseConv2d)
    assert nn.utils.parametrize.is_parametrized(model[1])
    fuse = nn.Sequential(PadInForward(64, 64, 3, stride=2, groups=64), nn.BatchNorm2d(64)).eval()
    assert tdc_torch.fuse_depthwise_bn_act(fuse) == 0


def test_same_padding_rule():
    """TensorFlow's "same": ceil(n / stride) outputs, total padding
    max((out - 1) * stride + K - n, 0), the odd one at the bottom / right."""
    for n in range(1, 40):
        for K in (3, 5, 7):
            for S in (1, 2):
                t, b, l, r = T.same_padding(n, n + 1, K, S)
                assert (n + t + b - K) // S + 1 == -(-n // S)
                assert (n + 1 + l + r - K) // S + 1 == -(-(n + 1) // S)
                assert 0 <= t <= b <= t + 1 and 0 <= l <= r <= l + 1
    assert T.same_padding(112, 112, 3, 2) == (0, 1, 0, 1)
    assert T.same_padding(112, 112, 5, 2) == (1, 2, 1, 2)
    assert T.same_padding(14, 14, 5, 1) == (2, 2, 2, 2)
    with pytest.raises(ValueError, match="top, bottom, left, right"):
        T.dwconv(FakeCuda((1, 8, 8, 64)), FakeCuda((3, 3, 64)), (1, 1, 1))


def test_padding_same_convs_are_converted():
    import tdc_torch
    nn = torch.nn
    model = nn.Sequential(nn.Conv2d(64, 64, 5, padding="same", groups=64),
                          nn.Conv2d(64, 64, 3, padding="same", groups=64, bias=False))
    assert tdc_torch.convert_depthwise_convs(model) == 2
    assert model[0].padding == 2 and model[1].padding == 1
    m = tdc_torch.DepthwiseConv2d(64, 3, 2, padding="same", device="cpu")
    assert m.padding == "same" and "padding=same" in repr(m)
