"""K x K taps and stride 2 (`tma_dwconv.dwconv`) vs cuDNN, on one GPU.

    python benchmarks/bench_kxk.py [--images 64] [--n-stage N] [--only K,S] [--iters 20] [--no-cudnn]
                              [--dtype fp16|bf16]

Input of the headline shape (N x 224 x 336 x 256 fp16), pad K // 2, for K in
{3, 5, 7} and stride 1 and 2.  CUDA events, 5 warm-up + 20 calls each (x is
2.5 GB at N = 64, far above L2).  Per variant, one JSON line:
  us            our kernel, per call
  cudnn_us      torch conv2d (groups = C) on channels-last views of the same tensors
  GBps          algorithmic bytes (x read once + y written once) / time
  fma_TFLOPs    2 * N*P*Q*C*K*K / time
  bound         the roofline limit: HBM (bytes / measured copy bandwidth) or the
                FP32 FMA pipe (148 SMs x 128 lanes x 2 flop x 1.965 GHz = 74.4 TFLOP/s,
                nominal), whichever takes longer
  frac          roofline time / measured time
A script, not a test.
"""
from __future__ import annotations

import argparse
import json
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [os.path.join(REPO, "tma-depthwise-conv_b200")]

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

import tma_dwconv as T  # noqa: E402

FMA_PEAK_TFLOPS = 148 * 128 * 2 * 1.965e9 / 1e12


def hbm_peak_gbps() -> float:
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"])
    except (OSError, KeyError, ValueError):
        return 6650.0


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
    ap.add_argument("--n-stage", type=int, default=None)
    ap.add_argument("--no-cudnn", action="store_true")
    ap.add_argument("--only", default=None, help="one geometry, e.g. 7,1 (K,stride)")
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--dtype", choices=["fp16", "bf16"], default="fp16")
    args = ap.parse_args()
    dt = torch.bfloat16 if args.dtype == "bf16" else torch.float16
    N, H, W, C = args.images, 224, 336, 256
    hbm = hbm_peak_gbps()
    g = torch.Generator(device="cuda").manual_seed(0)
    x = (torch.rand(N, H, W, C, device="cuda", generator=g) * 2 - 1).to(dt)
    xc = x.permute(0, 3, 1, 2)  # channels-last NCHW view
    only = tuple(int(v) for v in args.only.split(",")) if args.only else None
    for K in (3, 5, 7):
        w = ((torch.rand(K, K, C, device="cuda", generator=g) * 2 - 1) / K).to(dt)
        wc = w.permute(2, 0, 1).unsqueeze(1).contiguous(memory_format=torch.channels_last)
        for S in (1, 2):
            if only is not None and (K, S) != only:
                continue
            pad = K // 2
            P, Q = (H + 2 * pad - K) // S + 1, (W + 2 * pad - K) // S + 1
            ns = args.n_stage or T.DWCONV_STAGES[(K, S)]
            us = bench_us(lambda: T.dwconv(x, w, pad, stride=S, n_stage=ns), iters=args.iters)
            nbytes = 2 * N * C * (H * W + P * Q)
            flops = 2 * N * P * Q * C * K * K
            t_hbm = nbytes / (hbm * 1e9) * 1e6
            t_fma = flops / (FMA_PEAK_TFLOPS * 1e12) * 1e6
            row = {"K": K, "stride": S, "dtype": args.dtype, "images": N, "n_stage": ns,
                   "us": round(us, 1),
                   "GBps": round(nbytes / (us * 1e-6) / 1e9, 1),
                   "fma_TFLOPs": round(flops / (us * 1e-6) / 1e12, 2),
                   "bound": "hbm" if t_hbm >= t_fma else "fp32_fma",
                   "frac": round(max(t_hbm, t_fma) / us, 3)}
            if not args.no_cudnn:
                row["cudnn_us"] = round(bench_us(
                    lambda: F.conv2d(xc, wc, None, S, pad, 1, C)), 1)
                row["speedup_vs_cudnn"] = round(row["cudnn_us"] / us, 2)
            print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
