"""Dilated forward on the ring (TMA) kernel, through the C ABI
(tdc_dwconv_fwd_dilated_ex with an explicit kernel: 1 = the ring kernel,
-1 = the plain kernel, 0 = chosen by shape).

The ring kernel runs each of the D*D phases (p mod D, q mod D) as an
undilated problem on the D-strided sub-lattice of x, which its tensor map
loads with traversal stride D.  Parity bar: bit for bit with the CPU
oracle's K x K forward at pad 0 on the input zero-padded by hand with the
K' = D*(K-1)+1 kernel that has zeros between the taps (the zeros only add
exact zero products to the fp32 chain), and with the plain kernel; silu
within the oracle's silu bound.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle
import tma_dwconv as T

pytestmark = pytest.mark.gpu

GEOMS = [(K, S) for K in (3, 5, 7) for S in (1, 2)]
ACT = {"none": 0, "relu": 1, "relu6": 2, "silu": 3, "hardswish": 4}
TDC_ERR_UNSUPPORTED = -17
REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "tma-depthwise-conv_b200", "libtdc_sm100.so")
i64 = ctypes.c_int64
vp = ctypes.c_void_p


@pytest.fixture(scope="module")
def lib():
    return ctypes.CDLL(LIB)


def _bits(a):
    return a.detach().cpu().contiguous().view(torch.int16).numpy().view(np.uint16)


def _inflated(w, D):
    K, _, C = w.shape
    Ke = D * (K - 1) + 1
    wd = np.zeros((Ke, Ke, C), dtype=w.dtype)
    wd[::D, ::D] = w
    return wd


def _run(lib, x, w, pads, S, D, kernel, bias=None, residual=None, act="none"):
    N, H, W, C = x.shape
    K = w.shape[0]
    Ke = D * (K - 1) + 1
    t, b, l, r = pads
    P, Q = (H + t + b - Ke) // S + 1, (W + l + r - Ke) // S + 1
    y = torch.full((N, P, Q, C), float("nan"), dtype=x.dtype, device=x.device)
    rc = lib.tdc_dwconv_fwd_dilated_ex(
        vp(x.data_ptr()), vp(w.data_ptr()), vp(bias.data_ptr() if bias is not None else None),
        vp(residual.data_ptr() if residual is not None else None), vp(y.data_ptr()),
        i64(N), i64(H), i64(W), i64(C), i64(K), i64(S), i64(D), i64(t), i64(b), i64(l), i64(r),
        i64(ACT[act]), i64(kernel), i64(1 if x.dtype == torch.bfloat16 else 0),
        vp(torch.cuda.current_stream().cuda_stream))
    return rc, y


def _want(x, w, pads, S, D, **epi):
    t, b, l, r = pads
    xp = np.pad(x.numpy(), ((0, 0), (t, b), (l, r), (0, 0)))
    return oracle.dwconv_k_f16(xp, _inflated(w.numpy(), D), 0, S, **epi).view(np.uint16)


def _inputs(N, H, W, C, K, seed, dtype=torch.float16):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, H, W, C, generator=g).to(dtype)
    w = (torch.randn(K, K, C, generator=g) / K).to(dtype)
    b = torch.randn(C, generator=g).to(dtype)
    return x, w, b


@pytest.mark.parametrize("K,S", GEOMS)
@pytest.mark.parametrize("D", [2, 3])
@pytest.mark.parametrize("N,H,W,C", [(2, 41, 70, 64), (1, 29, 37, 200)])
def test_ring_matches_oracle_and_plain(lib, K, S, D, N, H, W, C):
    x, w, b = _inputs(N, H, W, C, K, seed=K * 100 + S * 10 + D + C)
    xc, wc, bc = x.cuda(), w.cuda(), b.cuda()
    Ke = D * (K - 1) + 1
    for pads in [(Ke // 2,) * 4, (0, 1, 2, 0), T.same_padding(H, W, Ke, S)]:
        t, bo, l, r = pads
        if H + t + bo < Ke or W + l + r < Ke:
            continue
        want = _want(x, w, pads, S, D, bias=b.numpy(), activation="relu")
        rc, plain = _run(lib, xc, wc, pads, S, D, -1, bias=bc, act="relu")
        assert rc == 0 and np.array_equal(_bits(plain), want), pads
        rc, y = _run(lib, xc, wc, pads, S, D, 1, bias=bc, act="relu")
        assert rc == 0, (pads, rc)
        assert np.array_equal(_bits(y), want), pads


@pytest.mark.parametrize("K,S,D", [(3, 1, 4), (3, 1, 7), (5, 1, 6), (7, 2, 3), (3, 2, 3)])
def test_ring_largest_steps(lib, K, S, D):
    """Dilations at the tensor map's limits: the box spans D x (input columns
    of a strip) <= 256 columns."""
    N, H, W, C = 1, 3 * D * K + 3, 4 * D * K + 1, 64
    x, w, _ = _inputs(N, H, W, C, K, seed=D * 7 + K)
    Ke = D * (K - 1) + 1
    pads = (Ke // 2,) * 4
    want = _want(x, w, pads, S, D)
    rc, y = _run(lib, x.cuda(), w.cuda(), pads, S, D, 1)
    assert rc == 0
    assert np.array_equal(_bits(y), want)


@pytest.mark.parametrize("K,S,D,H,W", [(3, 1, 3, 8, 9), (3, 1, 4, 9, 9), (5, 2, 2, 10, 13), (3, 2, 3, 8, 8)])
def test_ring_phases_without_outputs(lib, K, S, D, H, W):
    """Outputs fewer than D in a direction: some phases have no rows or no
    columns, and their segments are skipped by the producer and the
    consumers alike."""
    x, w, b = _inputs(3, H, W, 96, K, seed=H * W + D)
    pads = (0, 0, 0, 0)
    want = _want(x, w, pads, S, D, bias=b.numpy(), activation="relu6")
    rc, y = _run(lib, x.cuda(), w.cuda(), pads, S, D, 1, bias=b.cuda(), act="relu6")
    assert rc == 0 and y.shape[1] * y.shape[2] > 0
    assert np.array_equal(_bits(y), want)


def test_ring_rejects_steps_beyond_the_map(lib):
    x = torch.zeros(1, 40, 300, 64, dtype=torch.float16, device="cuda")
    w = torch.zeros(3, 3, 64, dtype=torch.float16, device="cuda")
    rc, _ = _run(lib, x, w, (8, 8, 8, 8), 1, 8, 1)  # 34 columns x 8 > 256
    assert rc == TDC_ERR_UNSUPPORTED
    rc, _ = _run(lib, x, w, (1, 1, 1, 1), 1, 1, 1)  # dilation 1: the undilated kernels' job
    assert rc == TDC_ERR_UNSUPPORTED
    rc, y = _run(lib, x, w, (8, 8, 8, 8), 1, 8, 0)  # chosen by shape: the plain kernel
    assert rc == 0 and torch.count_nonzero(y) == 0


def test_ring_epilogue_residual_and_silu(lib):
    K, S, D = 3, 1, 2
    x, w, b = _inputs(3, 48, 77, 192, K, seed=5)
    Ke = D * (K - 1) + 1
    pads = (D, D, D, D)
    P, Q = 48 + 2 * D - Ke + 1, 77 + 2 * D - Ke + 1
    g = torch.Generator().manual_seed(6)
    res = torch.randn(3, P, Q, 192, generator=g).half()
    want = _want(x, w, pads, S, D, bias=b.numpy(), residual=res.numpy(), activation="relu6")
    rc, y = _run(lib, x.cuda(), w.cuda(), pads, S, D, 1, bias=b.cuda(), residual=res.cuda(),
                 act="relu6")
    assert rc == 0 and np.array_equal(_bits(y), want)
    want = _want(x, w, pads, S, D, bias=b.numpy(), activation="silu")
    rc, y = _run(lib, x.cuda(), w.cuda(), pads, S, D, 1, bias=b.cuda(), act="silu")
    assert rc == 0
    ref = want.view(np.float16).astype(np.float32)
    assert (np.abs(y.float().cpu().numpy() - ref) <= oracle.silu_tolerance(ref)).all()


def test_ring_bf16(lib):
    K, S, D = 5, 1, 2
    x, w, _ = _inputs(2, 38, 66, 72, K, seed=11, dtype=torch.bfloat16)
    Ke = D * (K - 1) + 1
    xb = x.view(torch.int16).numpy().view(np.uint16)
    wb = w.view(torch.int16).numpy().view(np.uint16)
    xp = np.pad(xb, ((0, 0), (Ke // 2,) * 2, (Ke // 2,) * 2, (0, 0)))
    want = oracle.dwconv_k_bf16(xp, _inflated(wb, D), 0, S)
    rc, y = _run(lib, x.cuda(), w.cuda(), (Ke // 2,) * 4, S, D, 1)
    assert rc == 0 and y.dtype == torch.bfloat16 and np.array_equal(_bits(y), want)


def test_ring_large_batch_matches_plain(lib):
    """A shape with whole-strip waves and a chunked tail (several hundred
    strips): the ring and plain kernels agree bit for bit, and one image
    against the oracle."""
    N, H, W, C, K, S, D = 12, 96, 160, 256, 3, 1, 2
    g = torch.Generator(device="cuda").manual_seed(12)
    x = torch.empty(N, H, W, C, device="cuda", dtype=torch.float16).uniform_(-1, 1, generator=g)
    w = (torch.rand(K, K, C, device="cuda", generator=g) * 2 / 3 - 1 / 3).half()
    pads = (D, D, D, D)
    rc, ring = _run(lib, x, w, pads, S, D, 1)
    assert rc == 0
    rc, plain = _run(lib, x, w, pads, S, D, -1)
    assert rc == 0
    assert torch.equal(ring.view(torch.int16), plain.view(torch.int16))
    want = _want(x[-1:].cpu(), w.cpu(), pads, S, D)
    assert np.array_equal(_bits(ring[-1:]), want)


def test_automatic_choice_runs_the_ring_kernel_on_large_layers(lib):
    """tdc_dwconv_fwd_dilated (n_stage 0) and tma_dwconv.dwconv equal both
    kernels on a layer the choice gives the ring kernel."""
    N, H, W, C, K, S, D = 4, 64, 96, 256, 3, 1, 2
    pads = (D, D, D, D)
    assert lib.tdc_dwconv_fwd_dilated_uses_plain(i64(N), i64(H), i64(W), i64(C), i64(K), i64(S),
                                                 i64(D), *(i64(v) for v in pads)) == 0
    x, w, _ = _inputs(N, H, W, C, K, seed=13)
    xc, wc = x.cuda(), w.cuda()
    rc, auto = _run(lib, xc, wc, pads, S, D, 0)
    assert rc == 0
    rc, ring = _run(lib, xc, wc, pads, S, D, 1)
    assert rc == 0
    assert torch.equal(auto.view(torch.int16), ring.view(torch.int16))
    y = T.dwconv(xc, wc, pads, dilation=D)
    assert torch.equal(y.view(torch.int16), ring.view(torch.int16))
