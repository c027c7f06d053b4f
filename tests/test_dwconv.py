"""GPU parity of the plain (v0) and TMA warp-specialised (ws) kernels.

Port of the reference's tests/test_dwconv.py:8-46 (ten shapes x {v0, ws with
n_stage 2, 3, 4}, seed 0, x ~ randn, w ~ randn*0.1, checked against
``ref_dwconv`` with rtol=atol=1e-2), strengthened:

* every output is compared BIT FOR BIT with the CPU oracle (the reference's
  fp32 multiply-add chain restated in C) on the same inputs;
* against float32 ``conv2d(groups=C)`` the error is within one fp16 ulp of the
  reference value plus 1e-3 (TF32 disabled);
* edge shapes: pad 0..5, ragged strips (Q not a multiple of 32), one-column
  and one-row outputs, tiny images, C = 64..320, empty outputs, and canary
  bands around the output buffer.
"""
import numpy as np
import pytest
import torch

import oracle
import tma_dwconv as T

pytestmark = pytest.mark.gpu

REF_CASES = [
    (1, 8, 8, 64, 1),
    (2, 16, 16, 64, 1),
    (4, 32, 32, 128, 1),
    (8, 56, 56, 256, 1),
    (8, 56, 224, 128, 1),
    (16, 112, 224, 128, 1),
    (32, 224, 336, 256, 1),
    (64, 224, 336, 256, 1),
    (72, 224, 336, 256, 1),
    (80, 224, 336, 320, 1),
]

EDGE_CASES = [
    (2, 16, 16, 64, 0),
    (2, 16, 16, 64, 2),
    (2, 16, 16, 64, 3),
    (1, 3, 3, 64, 5),      # output entirely fed by padding rows/cols but the centre
    (3, 7, 45, 128, 1),    # odd H, Q = 45: one full strip + a 13-column strip
    (1, 5, 33, 64, 0),     # Q = 31
    (2, 9, 34, 192, 1),    # Q = 34: a 2-column tail strip
    (1, 1, 1, 64, 1),      # 1x1 image -> 1x1 output
    (1, 1, 200, 64, 1),    # a single row
    (5, 100, 1, 64, 1),    # a single column
    (1, 40, 40, 320, 4),
    (2, 66, 130, 64, 1),   # band boundaries not aligned with stages
]

WS_STAGES = [2, 3, 4]

_cache = {}


def _inputs(N, H, W, C, seed=0):
    torch.manual_seed(seed)
    x = torch.randn(N, H, W, C, device="cuda", dtype=torch.float16)
    w = torch.randn(3, 3, C, device="cuda", dtype=torch.float16) * 0.1
    return x, w


def _case(N, H, W, C, pad):
    """Inputs and oracle output of one case (only the latest case is kept)."""
    key = (N, H, W, C, pad)
    if key not in _cache:
        _cache.clear()
        x, w = _inputs(N, H, W, C)
        y_or = oracle.dwconv_f16(x.cpu().numpy(), w.cpu().numpy(), pad)
        _cache[key] = (x, w, y_or)
    return _cache[key]


def _assert_bits_equal(y: torch.Tensor, y_or: np.ndarray):
    got = y.cpu().numpy()
    assert got.shape == y_or.shape
    a, b = got.view(np.uint16), y_or.view(np.uint16)
    if not np.array_equal(a, b):
        bad = np.argwhere(a != b)
        i = tuple(bad[0])
        raise AssertionError(f"{len(bad)} of {a.size} outputs differ from the oracle; first at "
                             f"{i}: got {got[i]!r} oracle {y_or[i]!r}")


@pytest.mark.parametrize("N,H,W,C,pad", REF_CASES + EDGE_CASES)
def test_v0_matches_oracle(N, H, W, C, pad):
    x, w, y_or = _case(N, H, W, C, pad)
    y = T.dwconv_v0(x, w, pad=pad)
    _assert_bits_equal(y, y_or)


@pytest.mark.parametrize("n_stage", WS_STAGES)
@pytest.mark.parametrize("N,H,W,C,pad", REF_CASES + EDGE_CASES)
def test_ws_matches_oracle(N, H, W, C, pad, n_stage):
    x, w, y_or = _case(N, H, W, C, pad)
    y = T.dwconv_ws(x, w, pad=pad, n_stage=n_stage)
    _assert_bits_equal(y, y_or)


@pytest.mark.parametrize("N,H,W,C,pad", REF_CASES[:7])
def test_ws_matches_cudnn_reference(N, H, W, C, pad):
    """The reference's own acceptance check (tests/test_dwconv.py:40-46)."""
    x, w = _inputs(N, H, W, C)
    y_ref = T.ref_dwconv(x, w, pad=pad)
    for n_stage in WS_STAGES:
        torch.testing.assert_close(T.dwconv_ws(x, w, pad=pad, n_stage=n_stage), y_ref,
                                   rtol=1e-2, atol=1e-2)
    torch.testing.assert_close(T.dwconv_v0(x, w, pad=pad), y_ref, rtol=1e-2, atol=1e-2)


@pytest.mark.parametrize("N,H,W,C,pad", [(2, 16, 16, 64, 1), (8, 56, 56, 256, 1),
                                         (16, 112, 224, 128, 1), (4, 224, 336, 256, 1),
                                         (3, 7, 45, 128, 2)])
def test_ws_within_ulp_of_fp32_conv(N, H, W, C, pad):
    """|y - conv2d_fp32| <= ulp_fp16(conv2d_fp32) + 1e-3 (float32 torch reference)."""
    x, w = _inputs(N, H, W, C)
    prev = torch.backends.cudnn.allow_tf32
    torch.backends.cudnn.allow_tf32 = False
    try:
        ref = torch.nn.functional.conv2d(
            x.float().permute(0, 3, 1, 2), w.float().permute(2, 0, 1).unsqueeze(1),
            padding=pad, groups=C).permute(0, 2, 3, 1)
    finally:
        torch.backends.cudnn.allow_tf32 = prev
    y = T.dwconv_ws(x, w, pad=pad, n_stage=2).float()
    ref_np = ref.cpu().numpy()
    tol = oracle.f16_ulp(ref_np) + 1e-3
    err = np.abs(y.cpu().numpy() - ref_np)
    assert (err <= tol).all(), f"max excess {(err - tol).max()}"


def test_uniform_headline_distribution_small():
    """x ~ U(-1,1), w ~ U(-1/3,1/3) (the headline workload's distribution)."""
    g = torch.Generator(device="cuda")
    g.manual_seed(0)
    x = (torch.rand(4, 224, 336, 256, device="cuda", generator=g) * 2 - 1).half()
    w = ((torch.rand(3, 3, 256, device="cuda", generator=g) * 2 - 1) / 3).half()
    y_or = oracle.dwconv_f16(x.cpu().numpy(), w.cpu().numpy(), 1)
    for n_stage in WS_STAGES:
        _assert_bits_equal(T.dwconv_ws(x, w, 1, n_stage), y_or)


@pytest.mark.parametrize("C", [8, 24, 72])
def test_v0_small_channel_counts(C):
    x, w = _inputs(2, 13, 21, C)
    _assert_bits_equal(T.dwconv_v0(x, w, 1), oracle.dwconv_f16(x.cpu().numpy(), w.cpu().numpy(), 1))


def test_v0_image_beyond_32bit_offsets():
    # One image of 2^32 elements (8.6 GB): past the plain kernel's 32-bit
    # offsets within an image, dwconv_v0 runs the general ring kernel; it
    # must equal dwconv_ws (64-bit output offsets) bit for bit.
    N, H, W, C = 1, 4096, 4096, 256
    assert H * W * C // 2 > 2 ** 31 - 1
    g = torch.Generator(device="cuda").manual_seed(3)
    x = torch.empty(N, H, W, C, device="cuda", dtype=torch.float16).uniform_(-1, 1, generator=g)
    w = (torch.rand(3, 3, C, device="cuda", generator=g) * 2 / 3 - 1 / 3).half()
    a = T.dwconv_v0(x, w, 1)
    b = T.dwconv_ws(x, w, 1, 2)
    del x
    assert torch.equal(a.view(torch.int16), b.view(torch.int16))
    del a, b
    torch.cuda.empty_cache()


def test_empty_output_and_batch():
    x, w = _inputs(2, 2, 2, 64)
    assert T.dwconv_ws(x, w, pad=0).shape == (2, 0, 0, 64)
    assert T.dwconv_v0(x, w, pad=0).shape == (2, 0, 0, 64)
    x0 = torch.empty(0, 8, 8, 64, device="cuda", dtype=torch.float16)
    assert T.dwconv_ws(x0, w, pad=1).shape == (0, 8, 8, 64)


def test_canary_bands_untouched():
    """The kernels write exactly the [N,P,Q,C] output and nothing around it."""
    N, H, W, C, pad = 3, 19, 45, 128, 1
    x, w = _inputs(N, H, W, C)
    P, Q = H + 2 * pad - 2, W + 2 * pad - 2
    n = N * P * Q * C
    guard = 4096
    buf = torch.full((n + 2 * guard,), float("nan"), device="cuda", dtype=torch.float16)
    sentinel = buf.clone()
    y = buf[guard:guard + n].view(N, P, Q, C)
    for n_stage in WS_STAGES:
        T.dwconv_ws_out(x, w, y, pad, n_stage)
        torch.cuda.synchronize()
        assert torch.equal(buf[:guard].view(torch.int16), sentinel[:guard].view(torch.int16))
        assert torch.equal(buf[-guard:].view(torch.int16), sentinel[-guard:].view(torch.int16))
    _assert_bits_equal(y, oracle.dwconv_f16(x.cpu().numpy(), w.cpu().numpy(), pad))


def test_non_default_stream_and_second_device_index():
    x, w = _inputs(2, 30, 40, 64)
    s = torch.cuda.Stream()
    with torch.cuda.stream(s):
        y = T.dwconv_ws(x, w, 1, 3)
    s.synchronize()
    _assert_bits_equal(y, oracle.dwconv_f16(x.cpu().numpy(), w.cpu().numpy(), 1))


def test_errors_match_reference_messages():
    x, w = _inputs(1, 8, 8, 64)
    with pytest.raises(ValueError, match="n_stage must be one of"):
        T.dwconv_ws(x, w, 1, 5)
    with pytest.raises(ValueError, match=r"dwconv_ws requires C % 64 == 0"):
        T.dwconv_ws(x[..., :32].contiguous(), w[..., :32].contiguous(), 1)
    with pytest.raises(ValueError, match="contiguous"):
        T.dwconv_ws(x.permute(0, 2, 1, 3), w, 1)
    with pytest.raises(RuntimeError, match="only 3x3 kernel supported"):
        T._C.dwconv_ws(x, torch.zeros(5, 5, 64, device="cuda", dtype=torch.float16), 1, 2)
    with pytest.raises(RuntimeError, match="C must be a multiple of BlockC=64"):
        T._C.dwconv_ws(x[..., :32].contiguous(), w[..., :32].contiguous(), 1, 2)
    with pytest.raises(RuntimeError, match=r"n_stage must be one of \{2, 3, 4\}, got 7"):
        T._C.dwconv_ws(x, w, 1, 7)
