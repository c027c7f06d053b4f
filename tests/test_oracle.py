"""The CPU oracle, pinned before it is trusted (no GPU needed).

* its fp16 codec: decode exact for all 65536 bit patterns, encode equal to
  IEEE round-to-nearest-even (numpy) on dense samples around every boundary;
* the C restatement and the numpy restatement agree bit for bit;
* both reproduce the golden vectors recorded from the reference's own
  dwconv_ws and dwconv_v0 kernels on a B200 (tests/golden/ref_kernels.npz,
  made by tests/golden/make_golden.py) bit for bit;
* against float32 torch conv2d(groups=C) the error is within one fp16 ulp
  plus 1e-3.
"""
import os

import numpy as np
import pytest
import torch

import oracle

GOLDEN = os.path.join(os.path.dirname(os.path.abspath(__file__)), "golden", "ref_kernels.npz")


def test_decode_all_bit_patterns():
    lib = oracle.load()
    h = np.arange(65536, dtype=np.uint16)
    ref = h.view(np.float16).astype(np.float32)
    got = np.array([lib.oracle_f16_to_f32(int(v)) for v in h], dtype=np.float32)
    same = (got.view(np.uint32) == ref.view(np.uint32)) | (np.isnan(got) & np.isnan(ref))
    assert same.all()


def test_encode_round_to_nearest_even():
    lib = oracle.load()
    rng = np.random.default_rng(1)
    parts = [rng.standard_normal(4000).astype(np.float32) * s
             for s in (1e-9, 3e-8, 6e-8, 1e-7, 1e-6, 6e-5, 1e-3, 1.0, 300.0, 6e4)]
    # every fp16 value, the midpoints between neighbours and their fp32 neighbours
    f16 = np.arange(0, 0x7c00, dtype=np.uint16).view(np.float16).astype(np.float64)
    mids = ((f16[:-1] + f16[1:]) / 2).astype(np.float32)
    parts += [f16.astype(np.float32)[::3], mids[::5], np.nextafter(mids[::7], np.float32(np.inf)),
              np.nextafter(mids[::7], np.float32(0)),
              np.array([65504, 65519, 65519.996, 65520, 65536, 1e30, np.inf, -np.inf, 0.0, -0.0,
                        2.0 ** -25, 2.0 ** -24, 3 * 2.0 ** -26, 2.0 ** -14], np.float32)]
    f = np.concatenate(parts)
    f = np.concatenate([f, -f])
    got = np.array([lib.oracle_f32_to_f16(float(v)) for v in f], dtype=np.uint16)
    with np.errstate(over="ignore"):
        exp = f.astype(np.float16).view(np.uint16)
    assert np.array_equal(got, exp), f[got != exp][:10]


@pytest.mark.parametrize("shape,pad", [((2, 16, 16, 64), 1), ((1, 7, 45, 128), 0), ((3, 5, 33, 8), 2),
                                       ((1, 1, 1, 64), 1), ((2, 3, 3, 16), 5), ((1, 30, 2, 24), 3)])
def test_c_and_numpy_restatements_agree(shape, pad):
    rng = np.random.default_rng(sum(shape) + pad)
    x = rng.standard_normal(shape).astype(np.float16)
    w = (rng.standard_normal((3, 3, shape[3])) / 3).astype(np.float16)
    a = oracle.dwconv_f16(x, w, pad)
    b = oracle.dwconv_f16_numpy(x, w, pad)
    assert a.shape == (shape[0], shape[1] + 2 * pad - 2, shape[2] + 2 * pad - 2, shape[3])
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))
    assert np.array_equal(a.view(np.uint16), oracle.dwconv_f16(x, w, pad, threads=1).view(np.uint16))


def test_special_values_propagate():
    x = np.zeros((1, 4, 4, 8), np.float16)
    x[0, 1, 1, 0] = np.inf
    x[0, 2, 2, 1] = np.nan
    x[0, 0, 0, 2] = 60000
    x[0, 0, 1, 2] = 60000  # the fp32 sum overflows fp16 -> inf
    w = np.ones((3, 3, 8), np.float16)
    w[..., 3] = np.inf  # padding taps multiply 0 * inf = nan
    a, b = oracle.dwconv_f16(x, w, 1), oracle.dwconv_f16_numpy(x, w, 1)
    assert np.array_equal(np.isnan(a), np.isnan(b))
    m = ~np.isnan(a)
    assert np.array_equal(a[m].view(np.uint16), b[m].view(np.uint16))
    assert np.isinf(a[0, 0, 0, 0]) and np.isnan(a[0, 1, 1, 1]) and np.isinf(a[0, 0, 0, 2])
    assert np.isnan(a[..., 3]).all()


def test_empty_and_invalid():
    x = np.zeros((2, 2, 2, 64), np.float16)
    w = np.zeros((3, 3, 64), np.float16)
    assert oracle.dwconv_f16(x, w, 0).shape == (2, 0, 0, 64)
    with pytest.raises(ValueError):
        oracle.dwconv_f16(np.zeros((1, 1, 1, 8), np.float16), np.zeros((3, 3, 8), np.float16), 0)
    with pytest.raises(ValueError):
        oracle.dwconv_f16(x, np.zeros((3, 3, 32), np.float16), 1)


@pytest.mark.parametrize("shape,pad", [((2, 16, 16, 64), 1), ((1, 56, 56, 256), 1), ((2, 9, 37, 128), 2)])
def test_within_ulp_of_fp32_conv(shape, pad):
    torch.manual_seed(0)
    x = torch.randn(shape).half()
    w = (torch.randn(3, 3, shape[3]) / 3).half()
    ref = torch.nn.functional.conv2d(x.float().permute(0, 3, 1, 2), w.float().permute(2, 0, 1).unsqueeze(1),
                                     padding=pad, groups=shape[3]).permute(0, 2, 3, 1).numpy()
    y = oracle.dwconv_f16(x.numpy(), w.numpy(), pad).astype(np.float32)
    assert (np.abs(y - ref) <= oracle.f16_ulp(ref) + 1e-3).all()


def _golden_cases():
    if not os.path.exists(GOLDEN):
        return []
    z = np.load(GOLDEN)
    return sorted({k.split("_")[0] for k in z.files})


@pytest.mark.parametrize("case", _golden_cases() or ["missing"])
def test_matches_reference_golden_vectors(case):
    if case == "missing":
        pytest.fail(f"golden vectors missing: {GOLDEN}")
    z = np.load(GOLDEN)
    N, H, W, C, pad = (int(v) for v in z[f"{case}_shape"])
    x = z[f"{case}_x"].view(np.float16)
    w = z[f"{case}_w"].view(np.float16)
    assert x.shape == (N, H, W, C)
    got = oracle.dwconv_f16(x, w, pad).view(np.uint16)
    assert np.array_equal(got, z[f"{case}_ws"]), "oracle != reference dwconv_ws"
    assert np.array_equal(got, z[f"{case}_v0"]), "oracle != reference dwconv_v0"
    assert np.array_equal(oracle.dwconv_f16_numpy(x, w, pad).view(np.uint16), z[f"{case}_ws"])


@pytest.mark.parametrize("K,S", [(3, 1), (3, 2), (5, 1), (5, 2), (7, 1), (7, 2)])
@pytest.mark.parametrize("pad", [0, 1, 3])
def test_kxk_restatements_agree(K, S, pad):
    rng = np.random.default_rng(K * 10 + S + pad)
    x = rng.standard_normal((2, 13, 19, 24)).astype(np.float16)
    w = (rng.standard_normal((K, K, 24)) / K).astype(np.float16)
    if 13 + 2 * pad < K:
        with pytest.raises(ValueError):
            oracle.dwconv_k_f16(x, w, pad, S)
        return
    c = oracle.dwconv_k_f16(x, w, pad, S)
    n = oracle.dwconv_k_f16_numpy(x, w, pad, S)
    assert c.shape[1:3] == oracle.output_hw_k(13, 19, K, S, pad)
    assert np.array_equal(c.view(np.uint16), n.view(np.uint16))
    ref = torch.nn.functional.conv2d(torch.from_numpy(x).float().permute(0, 3, 1, 2),
                                     torch.from_numpy(w).float().permute(2, 0, 1).unsqueeze(1),
                                     stride=S, padding=pad, groups=24).permute(0, 2, 3, 1).numpy()
    assert (np.abs(c.astype(np.float32) - ref) <= oracle.f16_ulp(ref) + 1e-3).all()
    if (K, S) == (3, 1):
        assert np.array_equal(c.view(np.uint16), oracle.dwconv_f16(x, w, pad).view(np.uint16))


def test_kxk_epilogue_matches_3x3_epilogue():
    rng = np.random.default_rng(1)
    x = rng.standard_normal((2, 9, 11, 16)).astype(np.float16)
    w = (rng.standard_normal((3, 3, 16)) / 3).astype(np.float16)
    b = rng.standard_normal(16).astype(np.float16)
    r = rng.standard_normal((2, 9, 11, 16)).astype(np.float16)
    for act in oracle.ACTS:
        a = oracle.dwconv_k_f16(x, w, 1, 1, b, r, act)
        e = oracle.dwconv_ex_f16(x, w, 1, b, r, act)
        assert np.array_equal(a.view(np.uint16), e.view(np.uint16)), act


@pytest.mark.parametrize("K", [3, 5, 7])
@pytest.mark.parametrize("pad", [0, 1, 2, 3, 8])
@pytest.mark.parametrize("H,W", [(9, 13), (10, 12), (7, 7), (17, 6)])
def test_stride_2_data_gradient_restatements_agree(K, pad, H, W):
    """C and numpy restatements of the stride-2 data gradient agree bit for
    bit, and both are within fp16 rounding of float64 autograd."""
    if H + 2 * pad < K or W + 2 * pad < K:
        pytest.skip("input smaller than one padded window")
    rng = np.random.default_rng(K * 100 + pad * 10 + H)
    P, Q = (H + 2 * pad - K) // 2 + 1, (W + 2 * pad - K) // 2 + 1
    dy = rng.standard_normal((2, P, Q, 16)).astype(np.float16)
    w = (rng.standard_normal((K, K, 16)) / K).astype(np.float16)
    a = oracle.dwconv_bwd_data_s2_f16(dy, w, pad, H, W)
    b = oracle.dwconv_bwd_data_s2_numpy(dy, w, pad, H, W)
    assert np.array_equal(a.view(np.uint16), b.view(np.uint16))
    x = torch.zeros(2, 16, H, W, dtype=torch.float64, requires_grad=True)
    wt = torch.from_numpy(w.astype(np.float64)).permute(2, 0, 1).unsqueeze(1)
    y = torch.nn.functional.conv2d(x, wt, stride=2, padding=pad, groups=16)
    assert tuple(y.shape[2:]) == (P, Q)
    y.backward(torch.from_numpy(dy.astype(np.float64)).permute(0, 3, 1, 2))
    ref = x.grad.permute(0, 2, 3, 1).numpy()
    assert (np.abs(a.astype(np.float64) - ref) <= oracle.f16_ulp(ref) + 1e-3).all()


def test_stride_2_data_gradient_rejects_a_mismatched_input_size():
    dy = np.zeros((1, 5, 5, 8), np.float16)
    w = np.zeros((3, 3, 8), np.float16)
    oracle.dwconv_bwd_data_s2_f16(dy, w, 1, 10, 9)  # 9 and 10 both give 5
    with pytest.raises(ValueError):
        oracle.dwconv_bwd_data_s2_f16(dy, w, 1, 12, 10)


@pytest.mark.parametrize("K", [3, 5, 7])
@pytest.mark.parametrize("stride", [1, 2])
def test_weight_gradient_f64_matches_autograd(K, stride):
    rng = np.random.default_rng(K + stride)
    pad = K // 2
    x = rng.standard_normal((2, 11, 14, 8)).astype(np.float16)
    xt = torch.from_numpy(x.astype(np.float64)).permute(0, 3, 1, 2)
    wt = torch.zeros(8, 1, K, K, dtype=torch.float64, requires_grad=True)
    y = torch.nn.functional.conv2d(xt, wt, stride=stride, padding=pad, groups=8)
    dy = rng.standard_normal(tuple(y.permute(0, 2, 3, 1).shape)).astype(np.float16)
    y.backward(torch.from_numpy(dy.astype(np.float64)).permute(0, 3, 1, 2))
    dw = oracle.dwconv_bwd_weight_f64(x, dy, pad, K, stride=stride)
    np.testing.assert_allclose(dw, wt.grad[:, 0].permute(1, 2, 0).numpy(), atol=1e-9)


@pytest.mark.parametrize("K", [3, 5, 7])
@pytest.mark.parametrize("S", [1, 2])
@pytest.mark.parametrize("D", [1, 2, 3])
def test_dilation_and_side_pads_equal_the_inflated_kernel(K, S, D):
    """The GPU tests hold per-side padding and dilation to the C oracle run
    at pad 0 on the input padded by hand with the K x K taps spread over a
    D*(K-1)+1 kernel of zeros.  Here that construction is checked, bit for
    bit, against a direct restatement of the dilated, per-side-padded chain
    (oracle.dwconv_dilated_f16_numpy), so the zeros it adds are shown to
    change nothing."""
    rng = np.random.default_rng(K * 100 + S * 10 + D)
    Ke = D * (K - 1) + 1
    for (N, H, W, C) in [(2, 13, 17, 16), (1, 9, 22, 8)]:
        x = rng.standard_normal((N, H, W, C)).astype(np.float16)
        w = (rng.standard_normal((K, K, C)) / K).astype(np.float16)
        for pads in [(Ke // 2,) * 4, (0, 1, 0, 1), (2, 0, 1, 3)]:
            t, b, l, r = pads
            if H + t + b < Ke or W + l + r < Ke:
                continue
            direct = oracle.dwconv_dilated_f16_numpy(x, w, pads, S, D)
            wd = np.zeros((Ke, Ke, C), dtype=np.float16)
            wd[::D, ::D] = w
            xp = np.pad(x, ((0, 0), (t, b), (l, r), (0, 0)))
            inflated = oracle.dwconv_k_f16(xp, wd, 0, S)
            assert direct.shape == inflated.shape
            assert np.array_equal(direct.view(np.uint16), inflated.view(np.uint16)), pads
            if D == 1 and t == b == l == r:
                assert np.array_equal(direct.view(np.uint16),
                                      oracle.dwconv_k_f16_numpy(x, w, t, S).view(np.uint16))
