"""Side-by-side latency of this repository's kernels, the reference's kernels
and cuDNN, on the reference benchmark's shapes (tests/bench.py:32-39 of
haowen-han/tma-depthwise-conv), on one GPU.

    python benchmarks/bench_compare.py [--out table.md]

Method as the reference's tests/bench.py:18-29 (CUDA events around 100
back-to-back calls after 10 warm-up calls), with seeded inputs
(x ~ randn, w ~ randn*0.1, pad 1).  cuDNN is timed on a pre-permuted NCHW copy
(the reference's method) and on the channels-last view of the NHWC input.
The reference's kernels come from baseline/_ref (built by oracle/build_ref.py);
if that build is absent their columns are left empty.  A script, not a test:
it is the comparison table the reference's benchmark produces, without the
plot.
"""
from __future__ import annotations

import argparse
import glob
import importlib.util
import json
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [os.path.join(REPO, "tma-depthwise-conv_b200")]

import torch  # noqa: E402
import torch.nn.functional as F  # noqa: E402

import tma_dwconv as T  # noqa: E402

SHAPES = [
    (8, 56, 224, 128),
    (16, 112, 224, 128),
    (32, 224, 336, 256),
    (64, 224, 336, 256),
    (72, 224, 336, 256),
    (80, 224, 336, 320),
]


def load_reference():
    paths = glob.glob(os.path.join(REPO, "baseline", "_ref", "_tma_dwconv_ref_C*.so"))
    if not paths:
        return None
    spec = importlib.util.spec_from_file_location("_tma_dwconv_ref_C", paths[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def bench_ms(fn, warmup: int = 10, iters: int = 100) -> float:
    for _ in range(warmup):
        fn()
    torch.cuda.synchronize()
    s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
    s.record()
    for _ in range(iters):
        fn()
    e.record()
    torch.cuda.synchronize()
    return s.elapsed_time(e) / iters


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--out", default=None)
    args = ap.parse_args()
    ref = load_reference()
    pad = 1
    rows = []
    for (N, H, W, C) in SHAPES:
        torch.manual_seed(0)
        x = torch.randn(N, H, W, C, device="cuda", dtype=torch.float16)
        w = torch.randn(3, 3, C, device="cuda", dtype=torch.float16) * 0.1
        nbytes = 2 * N * H * W * C * 2 + 18 * C
        r = {"shape": [N, H, W, C]}
        r["ours_ws2"] = bench_ms(lambda: T.dwconv_ws(x, w, pad, 2))
        r["ours_ws3"] = bench_ms(lambda: T.dwconv_ws(x, w, pad, 3))
        r["ours_ws4"] = bench_ms(lambda: T.dwconv_ws(x, w, pad, 4))
        r["ours_v0"] = bench_ms(lambda: T.dwconv_v0(x, w, pad))
        if ref is not None:
            r["ref_ws2"] = bench_ms(lambda: ref.dwconv_ws(x, w, pad, 2))
            r["ref_ws4"] = bench_ms(lambda: ref.dwconv_ws(x, w, pad, 4))
            r["ref_v0"] = bench_ms(lambda: ref.dwconv_v0(x, w, pad))
        wc = w.permute(2, 0, 1).unsqueeze(1).contiguous()
        xcl = x.permute(0, 3, 1, 2)
        r["cudnn_cl"] = bench_ms(lambda: F.conv2d(xcl, wc, padding=pad, groups=C))
        xn = x.permute(0, 3, 1, 2).contiguous()
        r["cudnn_nchw"] = bench_ms(lambda: F.conv2d(xn, wc, padding=pad, groups=C))
        del xn
        r["gbs_ours_ws2"] = nbytes / (r["ours_ws2"] * 1e-3) / 1e9
        rows.append(r)
        print(json.dumps(r), flush=True)
        torch.cuda.empty_cache()
    cols = ["ours_ws2", "ours_ws3", "ours_ws4", "ours_v0", "ref_ws2", "ref_ws4", "ref_v0",
            "cudnn_cl", "cudnn_nchw"]
    lines = ["| N,H,W,C | " + " | ".join(c + " ms" for c in cols) + " | ours ws2 GB/s | ref ws2 / ours ws2 |",
             "|---" * (len(cols) + 3) + "|"]
    for r in rows:
        cells = [f"{r[c]:.3f}" if c in r else "—" for c in cols]
        speed = f"{r['ref_ws2'] / r['ours_ws2']:.2f}x" if "ref_ws2" in r else "—"
        lines.append(f"| {','.join(map(str, r['shape']))} | " + " | ".join(cells) +
                     f" | {r['gbs_ours_ws2']:.0f} | {speed} |")
    table = "\n".join(lines)
    print(table)
    if args.out:
        with open(args.out, "w") as f:
            f.write(table + "\n")


if __name__ == "__main__":
    main()
