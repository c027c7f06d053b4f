"""Producer / consumer wait-cycle probe of the ws kernel.

Port of the reference's tests/test_ws_time.py:1-171: the same four shapes x
three stage counts, a sanity check of the probed output, two warm-up and five
measured launches whose stall tensors are summed, and a one-line summary per
case.  The per-warp divisor comes from the module (``CONSUMER_WARPS``) instead
of being hard-coded.  Besides the reference's ``totals > 0`` assertion, the
tensor shape, the per-row consistency of the counters and bit-exactness of
the probed output are checked.

Run as pytest (prints the summary) or as a script:  python tests/test_ws_time.py
"""
from __future__ import annotations

import os
import sys

import pytest
import torch

if __name__ == "__main__":  # script mode: same import paths as conftest.py
    _repo = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
    sys.path[:0] = [os.path.join(_repo, "tma-depthwise-conv_b200"), os.path.join(_repo, "oracle")]

import tma_dwconv as T  # noqa: E402

CONSUMER_WARPS = T.CONSUMER_WARPS

CASES = [
    (8, 56, 56, 256, 1),
    (16, 112, 224, 128, 1),
    (32, 224, 336, 256, 1),
    (64, 224, 336, 256, 1),
]
WS_STAGES = [2, 3, 4]
N_WARMUP = 2
N_MEASURE = 5


def _make_inputs(N, H, W, C, seed=0):
    torch.manual_seed(seed)
    x = torch.randn(N, H, W, C, device="cuda", dtype=torch.float16)
    w = torch.randn(3, 3, C, device="cuda", dtype=torch.float16) * 0.1
    return x, w


def _summarize(stall_cpu: torch.Tensor) -> dict:
    prod = stall_cpu[:, 0].double()
    cons_per_warp = stall_cpu[:, 1].double() / CONSUMER_WARPS
    prod_total = stall_cpu[:, 2].double()
    cons_total_life = stall_cpu[:, 3].double() / CONSUMER_WARPS
    return {
        "num_blocks": stall_cpu.shape[0],
        "prod_mean": prod.mean().item(),
        "prod_p95": torch.quantile(prod, 0.95).item(),
        "cons_mean": cons_per_warp.mean().item(),
        "cons_p95": torch.quantile(cons_per_warp, 0.95).item(),
        "prod_total_mean": prod_total.mean().item(),
        "cons_total_mean": cons_total_life.mean().item(),
        "prod_frac": (prod / prod_total.clamp(min=1)).mean().item(),
        "cons_frac": (cons_per_warp / cons_total_life.clamp(min=1)).mean().item(),
    }


def _format_row(case, n_stage, s):
    N, H, W, C, _ = case
    bottleneck = "consumer" if s["prod_mean"] > s["cons_mean"] else "producer"
    return (f"  N={N:>3} H={H:>3} W={W:>3} C={C:>4}  stage={n_stage}  blks={s['num_blocks']:>5}  "
            f"prod mean={s['prod_mean']:>10.0f} p95={s['prod_p95']:>10.0f}  "
            f"cons/warp mean={s['cons_mean']:>10.0f} p95={s['cons_p95']:>10.0f}  "
            f"prod_tot={s['prod_total_mean']:>11.0f}  cons_tot/warp={s['cons_total_mean']:>11.0f}  "
            f"prod/prod_tot={s['prod_frac'] * 100:>5.1f}%  cons/cons_tot={s['cons_frac'] * 100:>5.1f}%"
            f"  -> {bottleneck} waits less")


def _run_case(case, n_stage):
    N, H, W, C, pad = case
    x, w = _make_inputs(N, H, W, C)
    y, stall = T.dwconv_ws_probe(x, w, pad=pad, n_stage=n_stage)
    assert stall.dtype == torch.int64 and stall.dim() == 2 and stall.shape[1] == 4
    assert torch.equal(y.view(torch.int16), T.dwconv_ws(x, w, pad, n_stage).view(torch.int16))
    torch.testing.assert_close(y, T.ref_dwconv(x, w, pad=pad), rtol=1e-2, atol=1e-2)
    for _ in range(N_WARMUP):
        T.dwconv_ws_probe(x, w, pad, n_stage)
    torch.cuda.synchronize()
    accum = None
    for _ in range(N_MEASURE):
        _, stall = T.dwconv_ws_probe(x, w, pad, n_stage)
        accum = stall if accum is None else accum + stall
    torch.cuda.synchronize()
    s = accum.cpu()
    # a wait never exceeds the lifetime of the warps that waited
    assert (s[:, 0] <= s[:, 2]).all() and (s[:, 1] <= s[:, 3]).all()
    return _summarize(s)


@pytest.mark.gpu
@pytest.mark.parametrize("n_stage", WS_STAGES)
@pytest.mark.parametrize("N,H,W,C,pad", CASES)
def test_ws_stall_probe(N, H, W, C, pad, n_stage, capsys):
    case = (N, H, W, C, pad)
    summary = _run_case(case, n_stage)
    with capsys.disabled():
        print()
        print(_format_row(case, n_stage, summary))
    assert summary["prod_total_mean"] > 0 and summary["cons_total_mean"] > 0


def main():
    print(f"ws kernel stall probe: CONSUMER_WARPS = {CONSUMER_WARPS}, warmup = {N_WARMUP}, "
          f"measured launches summed = {N_MEASURE}")
    for case in CASES:
        for n_stage in WS_STAGES:
            print(_format_row(case, n_stage, _run_case(case, n_stage)))
        print()


if __name__ == "__main__":
    main()
