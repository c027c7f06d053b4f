"""Backward of the depthwise 3x3 vs cuDNN, on one GPU.

    python tests/bench_backward.py [--images 64]

Headline shape (N x 224 x 336 x 256 fp16, pad 1).  CUDA events, 5 warm-up +
20 calls each:
  dgrad      dwconv3x3_bwd_data   (reads dy, writes dx: 4 B per element)
  wgrad      dwconv3x3_bwd_weight (reads x and dy: 4 B per element)
  cudnn      aten.convolution_backward on channels-last tensors, grad input
             and grad weight together (what nn.Conv2d's backward runs)
Prints one JSON line per variant with µs and algorithmic GB/s.  A script,
not a test.
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


def bench_us(fn, warmup=5, iters=20) -> float:
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
    N, H, W, C, pad = args.images, 224, 336, 256, 1
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.rand(N, H, W, C, device="cuda", generator=g) * 2 - 1).half()
    dy = (torch.rand(N, H, W, C, device="cuda", generator=g) * 2 - 1).half()
    w = ((torch.rand(3, 3, C, device="cuda", generator=g) * 2 - 1) / 3).half()
    io = 2 * N * H * W * C
    rows = [
        ("dgrad", lambda: T._C.dwconv3x3_bwd_data(dy, w, pad, 2), 2 * io),
        ("wgrad", lambda: T._C.dwconv3x3_bwd_weight(x, dy, pad, 2), 2 * io),
    ]
    xc, dyc = x.permute(0, 3, 1, 2), dy.permute(0, 3, 1, 2)  # channels-last NCHW views
    wc = w.permute(2, 0, 1).unsqueeze(1).contiguous()

    def cudnn_bwd():
        return torch.ops.aten.convolution_backward(dyc, xc, wc, None, [1, 1], [pad, pad], [1, 1],
                                                   False, [0, 0], C, [True, True, False])

    rows.append(("cudnn dgrad+wgrad", cudnn_bwd, 3 * io))
    out = {}
    for name, fn, nbytes in rows:
        us = bench_us(fn)
        out[name] = us
        print(json.dumps({"variant": name, "images": N, "us": round(us, 1),
                          "algorithmic_GBps": round(nbytes / (us * 1e-6) / 1e9, 1)}), flush=True)
    print(json.dumps({"ours_dgrad_plus_wgrad_us": round(out["dgrad"] + out["wgrad"], 1),
                      "speedup_vs_cudnn": round(out["cudnn dgrad+wgrad"] / (out["dgrad"] + out["wgrad"]), 2)}))


if __name__ == "__main__":
    main()
