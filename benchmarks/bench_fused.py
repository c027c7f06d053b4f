"""Fused epilogue vs the same work as separate passes, on one GPU.

    python benchmarks/bench_fused.py [--images 64]

Headline shape (N x 224 x 336 x 256, pad 1, n_stage 2).  Times per call
(CUDA events, 10 warm-up + 50 calls) of:
  conv                 dwconv_ws alone
  fused bias           dwconv3x3(bias)
  fused relu           dwconv3x3(activation="relu")
  fused bias+relu      dwconv3x3(bias, "relu")
  fused bias+relu6     dwconv3x3(bias, "relu6")
  fused bias+silu      dwconv3x3(bias, "silu")
  fused residual       dwconv3x3(residual=r)
  fused bias+silu+res  dwconv3x3(bias, "silu", residual)
  unfused              dwconv_ws, then y + bias, silu, + residual as torch ops
Prints one JSON line per variant: µs, algorithmic GB/s (x + y + residual +
w + bias bytes of the fused op), speed-up of the fused call over the unfused
sequence.  A script, not a test.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [os.path.join(REPO, "tma-depthwise-conv_b200")]

import torch  # noqa: E402

import tma_dwconv as T  # noqa: E402


def bench_us(fn, warmup=10, iters=50) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters * 1e3


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--images", type=int, default=64)
    args = ap.parse_args()
    N, H, W, C = args.images, 224, 336, 256
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.rand(N, H, W, C, device="cuda", generator=g) * 2 - 1).half()
    w = ((torch.rand(3, 3, C, device="cuda", generator=g) * 2 - 1) / 3).half()
    b = (torch.rand(C, device="cuda", generator=g) - 0.5).half()
    r = (torch.rand(N, H, W, C, device="cuda", generator=g) - 0.5).half()
    io = 2 * N * H * W * C  # bytes of one NHWC fp16 tensor of this shape

    def unfused():
        y = T.dwconv_ws(x, w, 1, 2)
        y = torch.nn.functional.silu(y + b)
        return y + r

    rows = [
        ("conv", lambda: T.dwconv_ws(x, w, 1, 2), 2 * io),
        ("fused bias", lambda: T.dwconv3x3(x, w, 1, bias=b), 2 * io),
        ("fused relu", lambda: T.dwconv3x3(x, w, 1, activation="relu"), 2 * io),
        ("fused bias+relu", lambda: T.dwconv3x3(x, w, 1, bias=b, activation="relu"), 2 * io),
        ("fused bias+relu6", lambda: T.dwconv3x3(x, w, 1, bias=b, activation="relu6"), 2 * io),
        ("fused bias+silu", lambda: T.dwconv3x3(x, w, 1, bias=b, activation="silu"), 2 * io),
        ("fused residual", lambda: T.dwconv3x3(x, w, 1, residual=r), 3 * io),
        ("fused bias+silu+res", lambda: T.dwconv3x3(x, w, 1, bias=b, residual=r, activation="silu"),
         3 * io),
        ("unfused bias+silu+res", unfused, 3 * io),
    ]
    out = {}
    for name, fn, nbytes in rows:
        us = bench_us(fn)
        out[name] = us
        print(json.dumps({"variant": name, "images": N, "us": round(us, 1),
                          "algorithmic_GBps": round(nbytes / (us * 1e-6) / 1e9, 1)}), flush=True)
    print(json.dumps({"fused_over_unfused_speedup":
                      round(out["unfused bias+silu+res"] / out["fused bias+silu+res"], 2)}))


if __name__ == "__main__":
    main()
