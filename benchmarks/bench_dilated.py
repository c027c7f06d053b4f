"""Dilated depthwise forward: the plain kernel, the ring kernel and the
automatic choice, on one GPU.

    python benchmarks/bench_dilated.py                      # the table's layers
    python benchmarks/bench_dilated.py --only 8,224,336,256,3,1,2 --kernel 1 --calls 5

Each layer (N, H, W, C, K, stride, dilation; pad D*(K-1)/2 on every side) is
run through tdc_dwconv_fwd_dilated_ex with kernel -1 (plain), 1 (ring) and 0
(the choice); the ring and plain outputs are compared bit for bit, then each
is timed as a CUDA graph of 20 calls (5 on layers above 200 M elements), 10
alternating rounds, median microseconds per call, with x + y GB/s.  With
--kernel only that kernel runs, --calls times (no timing): the command a
profiler wraps.  A script, not a test.
"""
from __future__ import annotations

import argparse
import ctypes as C
import json
import os
import statistics as S

import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "tma-depthwise-conv_b200", "libtdc_sm100.so")
LAYERS = [(8, 32, 32, 672, 5, 1, 2), (8, 32, 32, 960, 5, 1, 2), (8, 64, 64, 256, 3, 1, 2),
          (8, 64, 64, 256, 3, 1, 4), (8, 128, 128, 128, 3, 1, 6), (4, 65, 67, 72, 7, 2, 3),
          (2, 33, 40, 64, 3, 2, 2), (32, 128, 128, 256, 3, 1, 2), (16, 112, 112, 384, 5, 1, 2),
          (16, 128, 128, 256, 3, 1, 4), (32, 64, 64, 512, 3, 2, 2), (64, 224, 336, 256, 3, 1, 2)]
i64, vp = C.c_int64, C.c_void_p


def graph_of(fn, iters):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        fn()
    torch.cuda.current_stream().wait_stream(side)
    torch.cuda.synchronize()
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(iters):
            fn()
    g.replay()
    torch.cuda.synchronize()
    return g


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--only", default="", help="one layer: N,H,W,C,K,stride,dilation")
    ap.add_argument("--kernel", type=int, default=None, choices=[-1, 0, 1])
    ap.add_argument("--calls", type=int, default=5)
    args = ap.parse_args()
    lib = C.CDLL(LIB)
    layers = [tuple(int(v) for v in args.only.split(","))] if args.only else LAYERS
    dev = torch.device("cuda", 0)
    for (N, H, W, Cc, K, Sd, D) in layers:
        pad = D * (K - 1) // 2
        Ke = D * (K - 1) + 1
        P, Q = (H + 2 * pad - Ke) // Sd + 1, (W + 2 * pad - Ke) // Sd + 1
        g = torch.Generator(device=dev).manual_seed(0)
        x = torch.empty(N, H, W, Cc, device=dev, dtype=torch.float16).uniform_(-1, 1, generator=g)
        w = (torch.rand(K, K, Cc, device=dev, generator=g) * 0.6 - 0.3).half()
        kernels = {"plain": -1, "ring": 1, "choice": 0}
        if args.kernel is not None:
            kernels = {k: v for k, v in kernels.items() if v == args.kernel}
        ys = {k: torch.empty(N, P, Q, Cc, device=dev, dtype=torch.float16) for k in kernels}

        def call(k):
            y = ys[k]
            return lambda: lib.tdc_dwconv_fwd_dilated_ex(
                vp(x.data_ptr()), vp(w.data_ptr()), None, None, vp(y.data_ptr()), i64(N), i64(H),
                i64(W), i64(Cc), i64(K), i64(Sd), i64(D), i64(pad), i64(pad), i64(pad), i64(pad),
                i64(0), i64(kernels[k]), i64(0), vp(torch.cuda.current_stream().cuda_stream))

        fns = {k: call(k) for k in kernels}
        if args.kernel is not None:
            for _ in range(args.calls):
                assert next(iter(fns.values()))() == 0
            torch.cuda.synchronize()
            print(json.dumps({"layer": [N, H, W, Cc, K, Sd, D], "kernel": args.kernel, "calls": args.calls}))
            continue
        for k, f in fns.items():
            assert f() == 0, k
        torch.cuda.synchronize()
        out = {"layer": [N, H, W, Cc, K, Sd, D],
               "ring_equals_plain": bool(torch.equal(ys["ring"].view(torch.int16), ys["plain"].view(torch.int16))),
               "choice_is_plain": lib.tdc_dwconv_fwd_dilated_uses_plain(
                   i64(N), i64(H), i64(W), i64(Cc), i64(K), i64(Sd), i64(D), i64(pad), i64(pad), i64(pad),
                   i64(pad)) == 1}
        iters = 5 if N * H * W * Cc > 200e6 else 20
        graphs = {k: graph_of(f, iters) for k, f in fns.items()}
        t = {k: [] for k in fns}
        for r in range(10):
            for k in (list(fns) if r % 2 == 0 else list(fns)[::-1]):
                s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
                s.record()
                graphs[k].replay()
                e.record()
                e.synchronize()
                t[k].append(s.elapsed_time(e) / iters * 1e3)
        nbytes = 2 * (N * H * W * Cc + N * P * Q * Cc)
        for k in fns:
            us = S.median(t[k])
            out[k + "_us"] = round(us, 2)
            out[k + "_GBps"] = round(nbytes / us / 1e3, 1)
        print(json.dumps(out), flush=True)
        del graphs, x, ys
        torch.cuda.empty_cache()


if __name__ == "__main__":
    main()
