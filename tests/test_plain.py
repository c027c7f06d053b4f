"""The plain K x K forward (`tma_dwconv.dwconv_plain`, tdc_dwconv_fwd_plain)
and the automatic kernel choice of `tma_dwconv.dwconv` (n_stage=None), on the
GPU.

The plain kernel (no TMA, no shared memory) serves the shapes the ws kernel's
32-column x 64-channel strips fit badly: few channels, narrow images.  Parity
bar: bit for bit with the CPU oracle's K x K forward (oracle_dwconv_ex_f16 /
oracle_dwconv_ex_bf16) for every geometry, channel count, band height and
padding below, and bit for bit with the ws kernel for every fused epilogue,
silu included (both evaluate the same fp32 epilogue).
"""
import numpy as np
import pytest
import torch

import oracle
import tma_dwconv as T

pytestmark = pytest.mark.gpu

GEOMS = [(K, S) for K in (3, 5, 7) for S in (1, 2)]


def _bits(t: torch.Tensor) -> np.ndarray:
    return t.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _inputs(N, H, W, C, K, seed, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, H, W, C, generator=g).to(dtype)
    w = (torch.randn(K, K, C, generator=g) / K).to(dtype)
    b = torch.randn(C, generator=g).to(dtype)
    return x, w, b


@pytest.mark.parametrize("K,S", GEOMS)
@pytest.mark.parametrize("N,H,W,C,pad", [
    (2, 19, 45, 64, None),    # odd sizes
    (3, 12, 9, 8, None),      # one chunk of four channel pairs
    (2, 23, 17, 16, 0),       # no padding
    (1, 33, 70, 72, 1),       # 36 pairs: 16-byte chunks
    (4, 7, 7, 136, None),     # the late-stage 7 x 7 images
    (2, 14, 14, 200, None),
    (1, 1, 40, 24, None),     # one input row
    (1, 30, 1, 32, None),     # one input column
    (2, 11, 13, 48, "big"),   # pad beyond K // 2
])
def test_matches_oracle(K, S, N, H, W, C, pad):
    pad = K // 2 + 2 if pad == "big" else (K // 2 if pad is None else pad)
    if H + 2 * pad < K or W + 2 * pad < K:
        pytest.skip("no output")
    x, w, _ = _inputs(N, H, W, C, K, seed=K * 100 + S * 10 + C)
    want = oracle.dwconv_k_f16(x.numpy(), w.numpy(), pad, S).view(np.uint16)
    for band_rows in (0, 1, 2, 3, 1000):
        y = T.dwconv_plain(x.cuda(), w.cuda(), pad, stride=S, band_rows=band_rows)
        assert np.array_equal(_bits(y), want), band_rows


@pytest.mark.parametrize("K,S", GEOMS)
def test_bf16_matches_oracle(K, S):
    x, w, b = _inputs(3, 21, 30, 72, K, seed=K + S, dtype=torch.bfloat16)
    want = oracle.dwconv_k_bf16(_bits(x), _bits(w), K // 2, S, bias=_bits(b), activation="relu")
    for band_rows in (0, 2, 5):
        y = T.dwconv_plain(x.cuda(), w.cuda(), stride=S, bias=b.cuda(), activation="relu",
                           band_rows=band_rows)
        assert y.dtype == torch.bfloat16
        assert np.array_equal(_bits(y), want), band_rows


@pytest.mark.parametrize("K,S", GEOMS)
@pytest.mark.parametrize("activation", ["none", "relu", "relu6", "silu", "hardswish"])
def test_epilogue_matches_ws_kernel(K, S, activation):
    N, H, W, C = 2, 21, 37, 80
    x, w, b = _inputs(N, H, W, C, K, seed=7)
    P, Q = (H + 2 * (K // 2) - K) // S + 1, (W + 2 * (K // 2) - K) // S + 1
    r = torch.randn(N, P, Q, C, generator=torch.Generator().manual_seed(8)).half()
    xc, wc, bc, rc = x.cuda(), w.cuda(), b.cuda(), r.cuda()
    ws = T.dwconv(xc, wc, stride=S, bias=bc, residual=rc, activation=activation,
                  n_stage=T.DWCONV_STAGES[(K, S)])
    plain = T.dwconv_plain(xc, wc, stride=S, bias=bc, residual=rc, activation=activation)
    assert np.array_equal(_bits(plain), _bits(ws))
    if activation != "silu":
        want = oracle.dwconv_k_f16(x.numpy(), w.numpy(), K // 2, S, bias=b.numpy(),
                                   residual=r.numpy(), activation=activation)
        assert np.array_equal(_bits(plain), want.view(np.uint16))


@pytest.mark.parametrize("N,H,W,C,K,S", [
    (64, 112, 112, 16, 3, 1),   # MobileNetV3's first depthwise layer
    (64, 14, 14, 576, 3, 2),
    (64, 7, 7, 960, 5, 1),
    (64, 7, 7, 1152, 3, 1),
])
def test_model_layer_shapes_match_oracle(N, H, W, C, K, S):
    x, w, b = _inputs(N, H, W, C, K, seed=N + C)
    y = T.dwconv(x.cuda(), w.cuda(), stride=S, bias=b.cuda(), activation="relu6")
    assert T.uses_plain(N, H, W, C, K, S)
    want = oracle.dwconv_k_f16(x.numpy(), w.numpy(), K // 2, S, bias=b.numpy(),
                               activation="relu6")
    assert np.array_equal(_bits(y), want.view(np.uint16))


@pytest.mark.parametrize("K,S", GEOMS)
@pytest.mark.parametrize("N,H,W,C", [(2, 20, 40, 64), (2, 14, 14, 72), (1, 9, 100, 256)])
def test_automatic_choice_is_bit_identical(K, S, N, H, W, C):
    x, w, _ = _inputs(N, H, W, C, K, seed=3)
    xc, wc = x.cuda(), w.cuda()
    auto = T.dwconv(xc, wc, stride=S)
    ws = T.dwconv(xc, wc, stride=S, n_stage=T.DWCONV_STAGES[(K, S)])
    plain = T.dwconv_plain(xc, wc, stride=S)
    assert np.array_equal(_bits(auto), _bits(ws))
    assert np.array_equal(_bits(plain), _bits(ws))


def test_argument_errors():
    x, w, _ = _inputs(1, 8, 8, 64, 3, seed=0)
    xc, wc = x.cuda(), w.cuda()
    with pytest.raises(ValueError, match="band_rows must be non-negative"):
        T.dwconv_plain(xc, wc, band_rows=-1)
    with pytest.raises(ValueError, match="stride must be 1 or 2"):
        T.dwconv_plain(xc, wc, stride=3)
    with pytest.raises(ValueError, match="C % 8"):
        T.dwconv_plain(xc[..., :12].contiguous(), wc[..., :12].contiguous())
    with pytest.raises(RuntimeError, match="band_rows must be non-negative"):
        T._C.dwconv_plain(xc, wc, None, None, 1, 1, 0, -1)
    with pytest.raises(RuntimeError, match="x's dtype"):
        T.dwconv_plain(xc, wc, bias=torch.zeros(64, device="cuda", dtype=torch.bfloat16))
    y = T.dwconv_plain(xc[:0], wc)  # empty batch: nothing launched
    assert tuple(y.shape) == (0, 8, 8, 64)


def test_graph_capture_and_streams():
    x, w, b = _inputs(4, 14, 14, 96, 3, seed=2)
    xc, wc, bc = x.cuda(), w.cuda(), b.cuda()
    want = _bits(T.dwconv_plain(xc, wc, bias=bc, activation="relu"))
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(s):
        for _ in range(2):
            T.dwconv_plain(xc, wc, bias=bc, activation="relu")
    torch.cuda.current_stream().wait_stream(s)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        y = T.dwconv_plain(xc, wc, bias=bc, activation="relu")
    y.zero_()
    g.replay()
    torch.cuda.synchronize()
    assert np.array_equal(_bits(y), want)


@pytest.mark.parametrize("K", [3, 5, 7])
@pytest.mark.parametrize("N,H,W,C", [(4, 14, 14, 200), (2, 7, 7, 96), (3, 23, 30, 16),
                                     (2, 19, 40, 64)])
def test_automatic_data_gradient_matches_oracle(K, N, H, W, C):
    """Stride-1 data gradient with n_stage 0: the plain kernel with flipped
    taps where the shape calls for it, bit for bit with the oracle and with
    the ring kernel."""
    for pad in sorted({0, K // 2, K - 1}):
        P, Q = H + 2 * pad - K + 1, W + 2 * pad - K + 1
        if P < 1 or Q < 1:
            continue
        g = torch.Generator().manual_seed(K * 7 + pad)
        dy = torch.randn(N, P, Q, C, generator=g).half()
        w = (torch.randn(K, K, C, generator=g) / K).half()
        want = oracle.dwconv_bwd_data_f16(dy.numpy(), w.numpy(), pad).view(np.uint16)
        auto = T._C.dwconv_bwd_data(dy.cuda(), w.cuda(), pad, 1, 0, H, W)
        ring = T._C.dwconv_bwd_data(dy.cuda(), w.cuda(), pad, 1, T.DWCONV_STAGES[(K, 1)], H, W)
        assert np.array_equal(_bits(auto), want), pad
        assert np.array_equal(_bits(ring), want), pad


def _wgrad_ref(x, dy, pad, K, S):
    xf = x.float().numpy().astype(np.float64)
    dyf = dy.float().numpy().astype(np.float64)
    ref = oracle.dwconv_bwd_weight_f64(xf, dyf, pad, K, stride=S)
    scale = oracle.dwconv_bwd_weight_f64(np.abs(xf), np.abs(dyf), pad, K, stride=S)
    return ref, scale


@pytest.mark.parametrize("K,S", GEOMS)
@pytest.mark.parametrize("N,H,W,C,pad", [
    (4, 14, 14, 200, None), (3, 7, 7, 96, None), (2, 23, 30, 16, 0), (2, 19, 40, 72, "big"),
    (1, 1, 20, 8, None), (5, 9, 3, 24, None),
])
@pytest.mark.parametrize("dtype", [torch.float16, torch.bfloat16])
def test_plain_weight_gradient_close_to_float64(K, S, N, H, W, C, pad, dtype):
    """The plain weight gradient: within 5e-4 of sum |x * dy| of the float64
    oracle (the bar of the ring kernels' weight gradients), bit-reproducible."""
    pad = K - 1 if pad == "big" else (K // 2 if pad is None else pad)
    if H + 2 * pad < K or W + 2 * pad < K:
        pytest.skip("no output")
    P, Q = (H + 2 * pad - K) // S + 1, (W + 2 * pad - K) // S + 1
    g = torch.Generator().manual_seed(K * 10 + S + C)
    x = torch.randn(N, H, W, C, generator=g).to(dtype)
    dy = torch.randn(N, P, Q, C, generator=g).to(dtype)
    ref, scale = _wgrad_ref(x, dy, pad, K, S)
    a = T._C.dwconv_bwd_weight_plain(x.cuda(), dy.cuda(), K, pad, S)
    b = T._C.dwconv_bwd_weight_plain(x.cuda(), dy.cuda(), K, pad, S)
    dw = a.cpu().numpy()
    assert dw.dtype == np.float32 and dw.shape == (K, K, C)
    assert (np.abs(dw - ref) <= 5e-4 * scale + 1e-6).all(), np.abs(dw - ref).max()
    assert torch.equal(a.view(torch.int32), b.view(torch.int32))


@pytest.mark.parametrize("K,S", GEOMS)
def test_automatic_weight_gradient(K, S):
    """n_stage 0: the plain kernel where the shape calls for it (the same bits
    as calling it directly), the ring kernel elsewhere; both within the bar."""
    for (N, H, W, C) in [(8, 14, 14, 480), (4, 40, 72, 64)]:
        pad = K // 2
        P, Q = (H + 2 * pad - K) // S + 1, (W + 2 * pad - K) // S + 1
        g = torch.Generator().manual_seed(K + S + C)
        x = torch.randn(N, H, W, C, generator=g).half()
        dy = torch.randn(N, P, Q, C, generator=g).half()
        ref, scale = _wgrad_ref(x, dy, pad, K, S)
        auto = T._C.dwconv_bwd_weight(x.cuda(), dy.cuda(), K, pad, S, 0)
        assert (np.abs(auto.cpu().numpy() - ref) <= 5e-4 * scale + 1e-6).all()
        if T._C.dwconv_bwd_weight_uses_plain(N, H, W, C, K, S, pad):
            plain = T._C.dwconv_bwd_weight_plain(x.cuda(), dy.cuda(), K, pad, S)
            assert torch.equal(auto.view(torch.int32), plain.view(torch.int32))


def test_plain_weight_gradient_empty_batch_is_zero():
    x = torch.empty(0, 9, 9, 64, device="cuda", dtype=torch.float16)
    dy = torch.empty(0, 9, 9, 64, device="cuda", dtype=torch.float16)
    dw = T._C.dwconv_bwd_weight_plain(x, dy, 3, 1, 1)
    assert dw.shape == (3, 3, 64) and not dw.any()
