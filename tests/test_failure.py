"""Failure detection of the ws pipeline, on the GPU, without a GPU fault.

Every mbarrier wait in the ws kernel is bounded.  Here the producer withholds
one load, so the full barrier of that stage is never completed (a flag that
nothing sets): the consumers' wait runs out after a short limit, the kernel
records TDC_DEVICE_FULL_TIMEOUT in the per-device status word (and its copy
in mapped host memory), the producer drains the copies it did issue, and
every CTA returns.  The tests then check that later calls report the failure
until it is cleared, and that the CUDA context still runs a correct launch.
"""
import pytest
import torch

import oracle
import tma_dwconv as T

pytestmark = pytest.mark.gpu

FULL_TIMEOUT = 1


def _inputs():
    # 16 rows split over 2 CTAs: each streams 10 input rows, i.e. at least two
    # loads for every n_stage, so load number 1 exists in every CTA.
    torch.manual_seed(0)
    x = torch.randn(1, 16, 16, 64, device="cuda", dtype=torch.float16)
    w = torch.randn(3, 3, 64, device="cuda", dtype=torch.float16) * 0.1
    return x, w


@pytest.mark.parametrize("n_stage", [2, 4])
def test_withheld_load_times_out_and_context_survives(n_stage):
    x, w = _inputs()
    T.device_status(clear=True)
    T._C.dwconv_ws_withhold(x, w, 1, n_stage, 1, 50_000_000)  # 50 ms limit
    code, block, stage, load = T.device_status(clear=True)
    assert code == FULL_TIMEOUT, (code, block, stage, load)
    assert stage == 1 % n_stage
    # the context is intact: a normal launch completes and is exact
    y = T.dwconv_ws(x, w, 1, n_stage)
    assert T.device_status(clear=True)[0] == 0
    ref = oracle.dwconv_f16(x.cpu().numpy(), w.cpu().numpy(), 1)
    assert (y.cpu().numpy().view("u2") == ref.view("u2")).all()


@pytest.mark.parametrize("n_stage", [2, 3])
def test_next_call_reports_an_earlier_timeout(n_stage):
    # The failed launch's record reaches the host through mapped memory: once
    # that launch has finished, every later call fails before launching
    # anything (no synchronisation on the call path) until the record is
    # cleared; then calls run again, exactly.
    x, w = _inputs()
    T.device_status(clear=True)
    T._C.dwconv_ws_withhold(x, w, 1, n_stage, 1, 50_000_000)
    torch.cuda.synchronize()
    with pytest.raises(RuntimeError, match="gave up waiting"):
        T.dwconv_ws(x, w, 1, n_stage)
    with pytest.raises(RuntimeError, match="gave up waiting"):
        T.dwconv3x3(x, w, 1, n_stage=n_stage)
    with pytest.raises(RuntimeError, match="gave up waiting"):
        T.dwconv(x, w, 1, stride=2)
    code, block, stage, load = T.device_status(clear=True)
    assert code == FULL_TIMEOUT, (code, block, stage, load)
    y = T.dwconv_ws(x, w, 1, n_stage)
    assert T.device_status(clear=True)[0] == 0
    ref = oracle.dwconv_f16(x.cpu().numpy(), w.cpu().numpy(), 1)
    assert (y.cpu().numpy().view("u2") == ref.view("u2")).all()


def test_withhold_none_is_a_normal_launch():
    x, w = _inputs()
    T.device_status(clear=True)
    y = T._C.dwconv_ws_withhold(x, w, 1, 2, -1, 50_000_000)
    assert T.device_status(clear=True)[0] == 0
    ref = oracle.dwconv_f16(x.cpu().numpy(), w.cpu().numpy(), 1)
    assert (y.cpu().numpy().view("u2") == ref.view("u2")).all()
