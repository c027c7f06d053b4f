"""Benchmark of the NHWC fp16 depthwise 3x3 conv2d forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tdc|reference]
                    [--workload NAME] [--n-stage S] [--strong]

One step = one call of ``tma_dwconv.dwconv_ws`` (the reference's public API,
``tma_dwconv.py:63-78``) over the workload's whole batch, inputs resident in
HBM.  The headline workload is x [64,224,336,256] fp16 ~ U(-1,1),
w [3,3,256] ~ U(-1/3,1/3), pad 1 (4.93 GB of algorithmic traffic per call,
far larger than the 126 MB L2, so no flush is needed between calls).

Metric: achieved HBM bandwidth in GB/s = (x bytes + y bytes + w bytes) / time
per call, summed over all ranks; ``ms_per_step`` is the time per call.

Multi-GPU (torchrun, one process per GPU): every rank convolves its own
64-image shard of a 64*N-image batch (weak scaling, no collective on the data
path); the timed region is bracketed by barriers and the max over ranks is
reported.  ``--strong`` splits one 64-image batch over the ranks instead.

``--impl reference`` times the CPU restatement of the reference's arithmetic
(the oracle in oracle/, all host threads) on a bounded sample of the same
workload: one step = one image of the batch.  Only rank 0 runs it.
"""
from __future__ import annotations

import argparse
import json
import os
import statistics
import sys
import threading
import time

REPO = os.path.dirname(os.path.abspath(__file__))
PKG = os.path.join(REPO, "tma-depthwise-conv_b200")
sys.path.insert(0, PKG)

import torch  # noqa: E402

import tdc_dist  # noqa: E402
from tdc_workloads import HEADLINE, WORKLOADS, make_inputs, shard_range  # noqa: E402

FALLBACK_HBM_GBS = 6650.0
METRIC = "achieved HBM GB/s of the depthwise 3x3 forward ((x + y + w bytes) / time per call)"


def _peaks() -> tuple[float, str]:
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def _traffic_per_call(workload: str, n: int) -> float | None:
    """DRAM bytes per launch from the committed ncu summary, scaled to n images."""
    # lines: <kernel> <workload> <images captured> <dram read+write bytes per launch>
    path = os.path.join(REPO, "profiles", "dram_traffic.txt")
    try:
        for line in open(path):
            parts = line.split()
            if (len(parts) >= 4 and not line.startswith("#") and parts[0] == "dwconv_ws_kernel"
                    and parts[1] == workload):
                return float(parts[3]) * n / int(parts[2])
    except OSError:
        pass
    return None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }

    def __init__(self, index: int, period_s: float = 0.005):
        self.samples: list[int] = []
        self.reasons = 0
        self.max_mhz = None
        self._stop = threading.Event()
        self._period = period_s
        self._h = None
        try:
            import pynvml
            pynvml.nvmlInit()
            self._nv = pynvml
            self._h = pynvml.nvmlDeviceGetHandleByIndex(index)
            self.max_mhz = pynvml.nvmlDeviceGetMaxClockInfo(self._h, pynvml.NVML_CLOCK_SM)
        except Exception:
            self._h = None
        self._t = threading.Thread(target=self._run, daemon=True)

    def _sample(self):
        nv = self._nv
        self.samples.append(nv.nvmlDeviceGetClockInfo(self._h, nv.NVML_CLOCK_SM))
        self.reasons |= int(nv.nvmlDeviceGetCurrentClocksEventReasons(self._h))

    def _run(self):
        while not self._stop.is_set():
            try:
                self._sample()
            except Exception:
                return
            self._stop.wait(self._period)

    def __enter__(self):
        if self._h is not None:
            self._t.start()
        return self

    def __exit__(self, *exc):
        if self._h is not None:
            self._stop.set()
            self._t.join()
            try:
                self._sample()
            except Exception:
                pass

    def summary(self) -> dict:
        names = [k for k, v in self.REASONS.items() if self.reasons & v and k != "gpu_idle"]
        return {"sm_mhz": statistics.median(self.samples) if self.samples else None,
                "sm_max_mhz": self.max_mhz, "samples": len(self.samples), "reasons": names}


def _cuda_time(fn, steps: int, stream) -> float:
    """ms over `steps` calls of fn, CUDA events on `stream`, synchronized both sides."""
    start = torch.cuda.Event(enable_timing=True)
    end = torch.cuda.Event(enable_timing=True)
    torch.cuda.synchronize()
    tdc_dist.barrier()
    torch.cuda.synchronize()
    start.record(stream)
    for _ in range(steps):
        fn()
    end.record(stream)
    torch.cuda.synchronize()
    tdc_dist.barrier()
    return start.elapsed_time(end)


def _host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def _cpu_oracle_rate(wl, x_cpu, w_cpu, images: int, repeats: int):
    """Oracle throughput on `images` images: (seconds per image, threads)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle  # checker/baseline only
    xs = x_cpu[:images].numpy()
    ws = w_cpu.numpy()
    threads = _host_threads()
    oracle.dwconv_f16(xs[:1], ws, wl.pad, threads=threads)  # warm-up (page in, OpenMP pool)
    best = float("inf")
    for _ in range(repeats):
        t0 = time.perf_counter()
        oracle.dwconv_f16(xs, ws, wl.pad, threads=threads)
        best = min(best, time.perf_counter() - t0)
    return best / images, threads


def _torch_cpu_rate(wl, x_cpu, w_cpu, images: int):
    """torch CPU conv2d(groups=C) in float32 on the channels_last view: s per image."""
    threads = _host_threads()
    torch.set_num_threads(threads)
    xf = x_cpu[:images].float().permute(0, 3, 1, 2)  # NCHW view of NHWC memory = channels_last
    wf = w_cpu.float().permute(2, 0, 1).unsqueeze(1).contiguous()
    torch.nn.functional.conv2d(xf[:1], wf, padding=wl.pad, groups=wl.C)
    t0 = time.perf_counter()
    torch.nn.functional.conv2d(xf, wf, padding=wl.pad, groups=wl.C)
    return (time.perf_counter() - t0) / images, threads


def run_reference(args, wl) -> None:
    """CPU arm: the oracle (restatement of the reference arithmetic) on the host cores."""
    rank, world, _ = tdc_dist.env_rank()
    if rank != 0:
        return
    x, w = make_inputs(wl, "cpu", seed=0, n=1)
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import oracle
    xs, ws = x.numpy(), w.numpy()
    # every core this process may run on (torchrun sets OMP_NUM_THREADS=1)
    threads = _host_threads()
    for _ in range(args.warmup):
        oracle.dwconv_f16(xs, ws, wl.pad, threads=threads)
    t0 = time.perf_counter()
    for _ in range(args.steps):
        oracle.dwconv_f16(xs, ws, wl.pad, threads=threads)
    dt = (time.perf_counter() - t0) / args.steps
    gbs = wl.bytes_per_call(1) / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True, "scaling": "weak",
        "vs_baseline": None, "dtype": "f16 in/out, f32 accumulate", "data": "synthetic (seeded)",
        "config": {"workload": wl.name, "N": wl.N, "H": wl.H, "W": wl.W, "C": wl.C,
                   "pad": wl.pad, "step": "1 image of the batch on the host CPU"},
        "us_per_call_extrapolated": round(dt * wl.N * 1e6, 1),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "port",
                         "sample": f"1 of {wl.N} images per step, {args.steps} steps; C oracle "
                                   f"(fp32 fma chain, OpenMP) on {threads} threads"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


def _e2e(args, wl, T, x, w, y, stream, dev, total_bytes) -> dict:
    """Same metric through the public API with host buffers: every step is one
    ``tma_dwconv.dwconv_ws_host`` call, which copies w and x host->device
    (pinned), runs the kernel and copies y device->host, pipelined over
    chunks of images so the two copy directions overlap."""
    steps = max(2, min(args.steps, args.e2e_steps))
    xh = x.cpu().pin_memory()
    wh = w.cpu().pin_memory()
    yh = torch.empty(y.shape, dtype=y.dtype).pin_memory()

    def e2e_step():
        T.dwconv_ws_host(xh, wh, wl.pad, args.n_stage, out=yh, device=dev, sync=False)

    e2e_step()
    torch.cuda.synchronize()
    # the host copy holds the real result (one host copy of y serves both checks)
    y_ref = y.cpu().view(torch.int16)
    assert torch.equal(yh.view(torch.int16), y_ref)
    yh.zero_()
    ms = tdc_dist.max_over_ranks(_cuda_time(e2e_step, steps, stream), dev) / steps
    torch.cuda.synchronize()
    assert torch.equal(yh.view(torch.int16), y_ref)
    del y_ref
    return {"value": round(total_bytes / (ms * 1e-3) / 1e9, 3), "unit": "GB/s",
            "ms_per_step": round(ms, 3), "h2d_bytes_per_step": x.numel() * 2 + w.numel() * 2,
            "d2h_bytes_per_step": y.numel() * 2, "steps": steps,
            "path": "tma_dwconv.dwconv_ws_host (tdc_dwconv_ws_host: H2D / kernel / D2H "
                    "pipelined over chunks of images)"}


def run_tdc(args, wl) -> None:
    rank, world, local = tdc_dist.init("nccl", timeout_s=120.0)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import tma_dwconv as T

    per_rank = args.images or wl.N
    if args.strong:
        n0, n1 = shard_range(per_rank, world, rank)
    else:
        n0, n1 = rank * per_rank, (rank + 1) * per_rank
    n = n1 - n0
    x, w = make_inputs(wl, dev, seed=0, n=n, n_offset=n0)
    stream = torch.cuda.current_stream(dev)

    def step():
        return T.dwconv_ws(x, w, wl.pad, args.n_stage)

    for _ in range(max(args.warmup, 3)):
        y = step()
    torch.cuda.synchronize()

    with ClockSampler(local) as clocks:
        ms = _cuda_time(step, args.steps, stream)
    ms_max = tdc_dist.max_over_ranks(ms, dev)
    per_call_ms = ms_max / args.steps
    my_bytes = wl.bytes_per_call(n)
    total_bytes = tdc_dist.sum_over_ranks(float(my_bytes), dev)
    gbs = total_bytes / (per_call_ms * 1e-3) / 1e9
    local_ms = ms / args.steps
    achieved = my_bytes / (local_ms * 1e-3) / 1e9
    peak, peak_kind = _peaks()

    # cuDNN on the same data (the reference benchmark's comparison, tests/bench.py:52-57)
    cudnn = {}
    if not args.no_cudnn and not args.kernel_only:
        xc = x.permute(0, 3, 1, 2)  # channels_last view, no copy
        wc = w.permute(2, 0, 1).unsqueeze(1).contiguous()
        f = lambda: torch.nn.functional.conv2d(xc, wc, padding=wl.pad, groups=wl.C)
        for _ in range(3):
            f()
        cl = _cuda_time(f, max(3, min(args.steps, 20)), stream) / max(3, min(args.steps, 20))
        cudnn["channels_last_us"] = round(cl * 1e3, 1)
        del xc
        if not args.strong and n * wl.H * wl.W * wl.C * 2 * 2 < 40e9:
            xn = x.permute(0, 3, 1, 2).contiguous()
            f2 = lambda: torch.nn.functional.conv2d(xn, wc, padding=wl.pad, groups=wl.C)
            for _ in range(3):
                f2()
            cn = _cuda_time(f2, max(3, min(args.steps, 20)), stream) / max(3, min(args.steps, 20))
            cudnn["nchw_us"] = round(cn * 1e3, 1)
            del xn
        torch.cuda.empty_cache()

    # End to end through the public API with host buffers: H2D of x (and w),
    # the call, D2H of y, every step.
    e2e = None
    if not args.kernel_only:
        e2e = _e2e(args, wl, T, x, w, y, stream, dev, total_bytes)
    cpu = None
    if rank == 0 and world == 1 and not args.no_cpu and not args.kernel_only:
        images = min(n, args.cpu_images)
        x_cpu = x[:images].cpu()
        w_cpu = w.cpu()
        s_img, threads = _cpu_oracle_rate(wl, x_cpu, w_cpu, images, repeats=2)
        cpu = {"value": round(wl.bytes_per_call(1) / s_img / 1e9, 3), "unit": "GB/s",
               "cores": threads, "kind": "port",
               "sample": f"{images} of {wl.N} images, best of 2; C oracle (fp32 fma chain, OpenMP); "
                         f"{s_img * wl.N * 1e3:.0f} ms per full call extrapolated"}
        try:
            t_img, tthreads = _torch_cpu_rate(wl, x_cpu, w_cpu, min(images, 2))
            cpu["torch_conv2d_fp32"] = {"value": round(wl.bytes_per_call(1) / t_img / 1e9, 3),
                                        "unit": "GB/s", "threads": tthreads,
                                        "ms_per_call_extrapolated": round(t_img * wl.N * 1e3, 1)}
        except Exception as e:  # reported only
            cpu["torch_conv2d_fp32"] = {"error": str(e)[:200]}

    traffic = _traffic_per_call(wl.name, n)
    line = {
        "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(per_call_ms, 5),
        "higher_is_better": True, "scaling": "strong" if args.strong else "weak",
        "vs_baseline": None, "dtype": "f16 in/out, f32 accumulate", "data": "synthetic (seeded)",
        "config": {"workload": wl.name, "N_per_rank": n, "global_batch": n if world == 1 else
                   int(tdc_dist.sum_over_ranks(float(n), dev)), "H": wl.H, "W": wl.W, "C": wl.C,
                   "pad": wl.pad, "n_stage": args.n_stage, "parallelism": f"dp{world} (batch shards)",
                   "l2": "inputs larger than L2 (no flush needed)"},
        "us_per_call": round(per_call_ms * 1e3, 2),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "traffic": None if traffic is None else round(traffic),
                     "algorithmic_bytes": my_bytes, "kernel": "dwconv_ws_kernel"},
        "cpu_baseline": cpu,
        "e2e": e2e,
        "cudnn": cudnn or None,
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }
    if rank == 0:
        print(json.dumps(line), flush=True)
    tdc_dist.finalize()


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["tdc", "reference"], default="tdc")
    ap.add_argument("--workload", default=HEADLINE, choices=sorted(WORKLOADS))
    ap.add_argument("--n-stage", type=int, default=2, choices=[2, 3, 4])
    ap.add_argument("--strong", action="store_true")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-images", type=int, default=8)
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-cudnn", action="store_true")
    ap.add_argument("--images", type=int, default=0, help="images per rank (default: the workload's N)")
    ap.add_argument("--kernel-only", action="store_true",
                    help="time the kernel only (no cuDNN, end-to-end or CPU legs)")
    args = ap.parse_args()
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_tdc(args, wl)


if __name__ == "__main__":
    main()
