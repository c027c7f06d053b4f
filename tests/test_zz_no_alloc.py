"""The weight-gradient entry point that allocates nothing.

`tdc_dwconv3x3_bwd_weight_noalloc` serves callers that may not allocate
device memory when they need a weight gradient (a runtime with a device
budget fixed at start-up, a plug-in whose host framework owns every
allocation, a path where cudaMalloc could synchronise or fail).  Its
workspace is a 16 MiB array inside the library.  This file checks, through
the C ABI, that two calls in a row match `tdc_dwconv3x3_bwd_weight` (given a
caller workspace) within the weight-gradient tolerance of the other tests
(5e-4 of sum |x*dy|), that the second call does not see the first call's
leftovers, that the calls leave the device's free memory unchanged, and that
an oversized C is rejected.  It is named to run last: run alone in a fresh
process, its first call also performs the library's one-time set-up.
"""
import ctypes
import os

import numpy as np
import pytest
import torch

import oracle

pytestmark = pytest.mark.gpu

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "tma-depthwise-conv_b200", "libtdc_sm100.so")
i64 = ctypes.c_int64
vp = ctypes.c_void_p
TDC_ERR_SCRATCH_LIMIT = -15


@pytest.fixture(scope="module")
def lib():
    return ctypes.CDLL(LIB)


def _stream():
    return vp(torch.cuda.current_stream().cuda_stream)


def _with_workspace(lib, x, dy, pad, n_stage):
    N, H, W, C = x.shape
    nbytes = i64()
    assert lib.tdc_dwconv3x3_bwd_weight_workspace(i64(N), i64(H), i64(W), i64(C), i64(pad),
                                                  i64(n_stage), ctypes.byref(nbytes)) == 0
    ws = torch.empty(nbytes.value // 4 + 1, dtype=torch.float32, device=x.device)
    dw = torch.empty(3, 3, C, dtype=torch.float32, device=x.device)
    rc = lib.tdc_dwconv3x3_bwd_weight(vp(x.data_ptr()), vp(dy.data_ptr()), vp(dw.data_ptr()), i64(N),
                                      i64(H), i64(W), i64(C), i64(pad), i64(n_stage), vp(ws.data_ptr()),
                                      i64(nbytes.value), _stream())
    assert rc == 0
    return dw


def _noalloc(lib, x, dy, dw, pad, n_stage):
    N, H, W, C = x.shape
    return lib.tdc_dwconv3x3_bwd_weight_noalloc(vp(x.data_ptr()), vp(dy.data_ptr()), vp(dw.data_ptr()),
                                                i64(N), i64(H), i64(W), i64(C), i64(pad),
                                                i64(n_stage), _stream())


# (8, 56, 56, 1024): 144 * C bytes per CTA leave the 16 MiB room for 113 CTAs,
# fewer than the plan wants, so the entry point re-plans on a smaller grid
# (another tail split and number of partial sums than the workspace entry).
@pytest.mark.parametrize("N,H,W,C,pad", [(4, 56, 56, 256, 1), (2, 19, 45, 72, 2), (1, 30, 33, 640, 1),
                                         (8, 56, 56, 1024, 1)])
def test_two_calls_match_the_workspace_entry_point(lib, N, H, W, C, pad):
    g = torch.Generator(device="cuda").manual_seed(N * 1000 + C)
    x = (torch.rand(N, H, W, C, device="cuda", generator=g) * 2 - 1).half()
    dy = (torch.rand(N, H + 2 * pad - 2, W + 2 * pad - 2, C, device="cuda", generator=g) * 2 - 1).half()
    want = _with_workspace(lib, x, dy, pad, 2).cpu().numpy()
    scale = oracle.dwconv_bwd_weight_f64(np.abs(x.cpu().numpy()), np.abs(dy.cpu().numpy()), pad)
    results = []
    for _ in range(2):
        dw = torch.full((3, 3, C), float("nan"), dtype=torch.float32, device="cuda")
        assert _noalloc(lib, x, dy, dw, pad, 2) == 0
        torch.cuda.synchronize()
        got = dw.cpu().numpy()
        assert np.isfinite(got).all()
        assert (np.abs(got - want) <= 5e-4 * scale + 1e-6).all(), np.abs(got - want).max()
        results.append(got)
    # the second call starts from a cleared scratch, not from the first call's sums
    assert np.array_equal(results[0].view(np.uint32), results[1].view(np.uint32))


def test_allocates_no_device_memory(lib):
    g = torch.Generator(device="cuda").manual_seed(7)
    x = (torch.rand(2, 40, 40, 128, device="cuda", generator=g) - 0.5).half()
    dy = (torch.rand(2, 40, 40, 128, device="cuda", generator=g) - 0.5).half()
    dw = torch.empty(3, 3, 128, dtype=torch.float32, device="cuda")
    assert _noalloc(lib, x, dy, dw, 1, 2) == 0  # set-up (if not done yet) and first launch
    torch.cuda.synchronize()

    def free_after_three_calls():
        before_dev, before_torch = torch.cuda.mem_get_info()[0], torch.cuda.memory_allocated()
        for _ in range(3):
            assert _noalloc(lib, x, dy, dw, 1, 2) == 0
        torch.cuda.synchronize()
        assert torch.cuda.memory_allocated() == before_torch
        return before_dev, torch.cuda.mem_get_info()[0]

    # The device-wide figure also moves with other processes on the GPU: one
    # differing reading is taken again before it counts.
    before, after = free_after_three_calls()
    if after != before:
        before, after = free_after_three_calls()
    assert after == before


def test_rejects_channels_beyond_the_scratch(lib):
    C = 116512  # 4 warps x 9 taps x C floats per CTA > 16 MiB
    x = torch.empty(16, dtype=torch.float16, device="cuda")
    dw = torch.empty(16, dtype=torch.float32, device="cuda")
    rc = lib.tdc_dwconv3x3_bwd_weight_noalloc(vp(x.data_ptr()), vp(x.data_ptr()), vp(dw.data_ptr()),
                                              i64(1), i64(3), i64(3), i64(C), i64(1), i64(2), _stream())
    assert rc == TDC_ERR_SCRATCH_LIMIT
    lib.tdc_strerror.restype = ctypes.c_char_p
    assert b"static scratch" in lib.tdc_strerror(rc)
