"""The ws forward on host buffers (`tma_dwconv.dwconv_ws_host`,
`tdc_dwconv_ws_host`): host->device copies, kernels and device->host copies
pipelined over chunks of images must give exactly `dwconv_ws`'s output for
every chunk size, with pinned or pageable host memory, and leave the caller's
stream ordered after the copy back."""
import pytest
import torch

import tma_dwconv as T

pytestmark = pytest.mark.gpu


def _inputs(N, H, W, C, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, H, W, C, generator=g).half()
    w = (torch.randn(3, 3, C, generator=g) / 3).half()
    return x, w


@pytest.mark.parametrize("chunk", [0, 1, 3, 5, 64])
def test_matches_device_call_for_every_chunk_size(chunk):
    x, w = _inputs(5, 37, 45, 128, seed=chunk)
    want = T.dwconv_ws(x.cuda(), w.cuda(), 1, 2).cpu()
    got = T.dwconv_ws_host(x.pin_memory(), w.pin_memory(), 1, 2, chunk_images=chunk)
    assert got.is_pinned() and not got.is_cuda
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


@pytest.mark.parametrize("pad,n_stage", [(0, 3), (2, 4), (1, 2)])
def test_pageable_memory_and_paddings(pad, n_stage):
    x, w = _inputs(3, 20, 70, 64, seed=pad)
    want = T.dwconv_ws(x.cuda(), w.cuda(), pad, n_stage).cpu()
    out = torch.empty(want.shape, dtype=torch.float16)  # pageable output
    got = T.dwconv_ws_host(x, w, pad, n_stage, chunk_images=2, out=out)
    assert got is out
    assert torch.equal(got.view(torch.int16), want.view(torch.int16))


def test_asynchronous_call_orders_the_current_stream():
    x, w = _inputs(16, 56, 56, 256, seed=9)
    want = T.dwconv_ws(x.cuda(), w.cuda(), 1, 2).cpu()
    xh, wh = x.pin_memory(), w.pin_memory()
    out = torch.empty(want.shape, dtype=torch.float16, pin_memory=True)
    for _ in range(3):
        out.zero_()
        T.dwconv_ws_host(xh, wh, 1, 2, chunk_images=3, out=out, sync=False)
        torch.cuda.current_stream().synchronize()
        assert torch.equal(out.view(torch.int16), want.view(torch.int16))


def test_argument_errors():
    x, w = _inputs(1, 8, 8, 64)
    with pytest.raises(ValueError, match="CPU tensors"):
        T.dwconv_ws_host(x.cuda(), w)
    with pytest.raises(ValueError, match="C % 64"):
        T.dwconv_ws_host(x[..., :32].contiguous(), w[..., :32].contiguous())
    with pytest.raises(RuntimeError, match="same shapes"):
        T._C.dwconv_ws_host(x, w, torch.empty(1, 8, 8, 64).half(), x.cuda(), w.cuda(),
                            torch.empty(1, 6, 6, 64, device="cuda").half(), 1, 2, 0)


def test_calls_from_two_host_threads():
    # The library's per-device copy / kernel streams are shared; concurrent
    # callers are serialised while they enqueue, and each gets its own result.
    import threading
    inputs = [_inputs(4, 30, 64, 64, seed=20 + i) for i in range(2)]
    wants = [T.dwconv_ws(x.cuda(), w.cuda(), 1, 2).cpu() for x, w in inputs]
    outs, errors = [None, None], []

    def run(i):
        try:
            x, w = inputs[i]
            for _ in range(5):
                outs[i] = T.dwconv_ws_host(x.pin_memory(), w.pin_memory(), 1, 2, chunk_images=1)
        except Exception as e:  # reported below
            errors.append(e)

    threads = [threading.Thread(target=run, args=(i,)) for i in range(2)]
    for t in threads:
        t.start()
    for t in threads:
        t.join()
    assert not errors, errors
    for got, want in zip(outs, wants):
        assert torch.equal(got.view(torch.int16), want.view(torch.int16))
