"""Backward of the depthwise K x K (stride 1 or 2) vs cuDNN, on one GPU.

    python benchmarks/bench_backward.py [--images 64] [--K 3] [--stride 1] [--n-stage 2]
                                   [--wgrad-n-stage S] [--dtype fp16|bf16]

Headline shape (N x 224 x 336 x 256 fp16 input, pad K // 2; dy is
N x P x Q x 256 with P = (224 + 2*pad - K) // stride + 1).  CUDA events, 5
warm-up + 20 calls each:
  dgrad      dwconv_bwd_data   (reads dy, writes dx)
  wgrad      dwconv_bwd_weight (reads x and dy, once per tap-row launch)
  cudnn      aten.convolution_backward on channels-last tensors, grad input
             and grad weight together (what nn.Conv2d's backward runs)
Prints one JSON line per variant with µs, algorithmic GB/s (x + dy bytes,
dx counted as x) and the FMA rate (2 * N*P*Q*C*K*K flop per gradient).  A
script, not a test.
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
    ap.add_argument("--K", type=int, default=3)
    ap.add_argument("--stride", type=int, default=1, choices=[1, 2])
    ap.add_argument("--n-stage", type=int, default=2)
    ap.add_argument("--wgrad-n-stage", type=int, default=0, help="default: --n-stage")
    ap.add_argument("--dtype", choices=["fp16", "bf16"], default="fp16")
    args = ap.parse_args()
    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    K, S, ns = args.K, args.stride, args.n_stage
    wns = args.wgrad_n_stage or ns
    N, H, W, C, pad = args.images, 224, 336, 256, K // 2
    P, Q = (H + 2 * pad - K) // S + 1, (W + 2 * pad - K) // S + 1
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.rand(N, H, W, C, device="cuda", generator=g) * 2 - 1).to(dt)
    dy = (torch.rand(N, P, Q, C, device="cuda", generator=g) * 2 - 1).to(dt)
    w = ((torch.rand(K, K, C, device="cuda", generator=g) * 2 - 1) / K).to(dt)
    xb, dyb = 2 * N * H * W * C, 2 * N * P * Q * C
    flops = 2 * N * P * Q * C * K * K
    rows = [
        ("dgrad", lambda: T._C.dwconv_bwd_data(dy, w, pad, S, ns, H, W), xb + dyb),
        ("wgrad", lambda: T._C.dwconv_bwd_weight(x, dy, K, pad, S, wns), xb + dyb),
    ]
    xc, dyc = x.permute(0, 3, 1, 2), dy.permute(0, 3, 1, 2)  # channels-last NCHW views
    wc = w.permute(2, 0, 1).unsqueeze(1).contiguous()

    def cudnn_bwd():
        return torch.ops.aten.convolution_backward(dyc, xc, wc, None, [S, S], [pad, pad], [1, 1],
                                                   False, [0, 0], C, [True, True, False])

    rows.append(("cudnn dgrad+wgrad", cudnn_bwd, 2 * xb + 2 * dyb))
    out = {}
    for name, fn, nbytes in rows:
        us = bench_us(fn)
        out[name] = us
        nf = 2 * flops if name.startswith("cudnn") else flops
        print(json.dumps({"variant": name, "K": K, "stride": S, "dtype": args.dtype,
                          "n_stage": wns if name == "wgrad" else ns, "images": N, "us": round(us, 1),
                          "algorithmic_GBps": round(nbytes / (us * 1e-6) / 1e9, 1),
                          "fma_TFLOPs": round(nf / (us * 1e-6) / 1e12, 2)}), flush=True)
    print(json.dumps({"ours_dgrad_plus_wgrad_us": round(out["dgrad"] + out["wgrad"], 1),
                      "speedup_vs_cudnn": round(out["cudnn dgrad+wgrad"] / (out["dgrad"] + out["wgrad"]), 2)}))


if __name__ == "__main__":
    main()
