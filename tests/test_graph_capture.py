"""Forward calls inside a CUDA graph.

The forward kernels launch with programmatic stream serialization (their
set-up may overlap the previous kernel on the stream; every thread waits for
that kernel before touching global memory).  Captured into a CUDA graph, those
launches become programmatic dependencies; replays must give exactly the
eager results, also when consecutive captured calls write and then read the
same buffer."""
import pytest
import torch

import tma_dwconv as T

pytestmark = pytest.mark.gpu


def _inputs(N, H, W, C, K=3, seed=0):
    g = torch.Generator().manual_seed(seed)
    x = torch.randn(N, H, W, C, generator=g).half().cuda()
    w = (torch.randn(K, K, C, generator=g) / K).half().cuda()
    return x, w


def test_replay_matches_eager_for_chained_calls():
    x, w = _inputs(4, 40, 70, 128)
    w5 = _inputs(1, 5, 5, 128, K=5, seed=1)[1]
    b = torch.randn(128, generator=torch.Generator().manual_seed(2)).half().cuda()
    want1 = T.dwconv_ws(x, w, 1, 2)
    want2 = T.dwconv3x3(want1, w, 1, bias=b, activation="relu")         # reads call 1's output
    want3 = T.dwconv(want2, w5, stride=2)                                # reads call 2's output
    y1 = torch.empty_like(want1)
    s = torch.cuda.Stream()
    s.wait_stream(torch.cuda.current_stream())
    g = torch.cuda.CUDAGraph()
    with torch.cuda.stream(s):
        T.dwconv_ws_out(x, w, y1, 1, 2)                                  # warm-up outside capture
        torch.cuda.synchronize()
        with torch.cuda.graph(g, stream=s):
            T.dwconv_ws_out(x, w, y1, 1, 2)
            y2 = T.dwconv3x3(y1, w, 1, bias=b, activation="relu")
            y3 = T.dwconv(y2, w5, stride=2)
    torch.cuda.current_stream().wait_stream(s)
    for _ in range(3):
        y1.zero_()
        y2.zero_()
        y3.zero_()
        g.replay()
        torch.cuda.synchronize()
        assert torch.equal(y1, want1) and torch.equal(y2, want2) and torch.equal(y3, want3)


def test_back_to_back_calls_into_one_buffer():
    # Consecutive launches with the same output: the later one may start its
    # set-up early but must not write before the earlier one finished.
    x1, w = _inputs(8, 56, 56, 256, seed=3)
    x2, _ = _inputs(8, 56, 56, 256, seed=4)
    y = torch.empty_like(T.dwconv_ws(x1, w, 1, 2))
    want = T.dwconv_ws(x2, w, 1, 2)
    for _ in range(50):
        T.dwconv_ws_out(x1, w, y, 1, 2)
        T.dwconv_ws_out(x2, w, y, 1, 2)
    torch.cuda.synchronize()
    assert torch.equal(y, want)
