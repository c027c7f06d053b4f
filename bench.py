"""Benchmark of the NHWC fp16 depthwise 3x3 conv2d forward on B200.

    python bench.py [--gpus N] [--steps K] [--warmup W] [--impl tdc|reference]
                    [--workload NAME] [--n-stage S] [--weak]

One step = one call of ``tma_dwconv.dwconv_ws`` (the reference's public API,
``tma_dwconv.py:63-78``) over the workload's batch, inputs resident in HBM.
The headline workload is x [64,224,336,256] fp16 ~ U(-1,1), w [3,3,256] ~
U(-1/3,1/3), pad 1 (4.93 GB of algorithmic traffic per call, far larger than
the 126 MB L2, so no flush is needed between calls).

Metric: achieved HBM bandwidth in GB/s = (x bytes + y bytes + w bytes) / time
per call, summed over all ranks; ``ms_per_step`` is the time per call.

Multi-GPU (torchrun, one process per GPU): the 64-image batch is split over
the ranks (64 -> 32 / 16 / 8 images per GPU; "scaling": "strong"), one
independent launch per GPU, no collective on the data path; the timed region
is bracketed by barriers and the max over ranks is reported.  ``weak`` (64
images on every rank) and the same split of the 16x112x224x128 and
32x224x336x256 workloads (``strong_split``) are reported beside it; ``--weak``
makes 64 images per rank the headline instead.

Beside the headline the line carries, from the same process and the same
inputs: the reference's own ws kernel (n_stage 2, built from the reference's
sources into baseline/_ref by oracle/build_ref.py) and cuDNN (channels-last and
the reference benchmark's NCHW copy); ``per_config`` (N = 1: the other
workloads, timed as the reference's tests/bench.py:18-29 does: 10 warm-up +
100 back-to-back calls); the end-to-end call with host buffers and the plain
pinned-copy ceiling beside it; the CPU baseline (the oracle on the host cores,
which is also the checker: every rank compares one full image of its shard
with it, bit for bit, outside the timed regions).

``--impl reference`` times the reference's own CPU path for the operator,
torch's ``conv2d(groups=C)`` behind ``ref_dwconv`` (``tma_dwconv.py:14-34``), on
the host cores: the fastest of ``ref_dwconv`` as written (NCHW copies in and
out) and conv2d on the channels-last view (no copies), in fp16 or on float32
copies, chosen on one image; one step = 8 images of the batch.  Only rank 0
runs it.
"""
from __future__ import annotations

import argparse
import glob
import importlib.util
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
# workloads whose batch is split over the GPUs beside the headline
SPLIT_WORKLOADS = ["dw3x3_n16_h112_w224_c128", "dw3x3_n32_h224_w336_c256"]
# single-GPU workloads reported in per_config (the reference benchmark's method)
PER_CONFIG = ["dw3x3_n8_h56_w56_c256", "dw3x3_n16_h112_w224_c128", "dw3x3_n32_h224_w336_c256"]


def _peaks() -> tuple[float, str]:
    try:
        with open(os.path.join(REPO, "MEASURED_PEAKS.json")) as f:
            return float(json.load(f)["hbm_gbs"]), "measured"
    except Exception:
        return FALLBACK_HBM_GBS, "fallback"


def _traffic_per_call(workload: str, n: int) -> tuple[float | None, str | None]:
    """DRAM bytes per launch from the committed ncu summary, scaled to n images
    of `workload`'s image size (lines: <kernel> <workload> <images captured>
    <dram read+write bytes per launch>)."""
    path = os.path.join(REPO, "profiles", "dram_traffic.txt")
    try:
        for line in open(path):
            parts = line.split()
            if (len(parts) >= 4 and not line.startswith("#") and parts[0] == "dwconv_ws_kernel"
                    and parts[1] == workload):
                return float(parts[3]) * n / int(parts[2]), f"ncu capture of {parts[2]} images, scaled"
    except OSError:
        pass
    return None, None


class ClockSampler:
    """Samples SM clock and throttle reasons through NVML while running."""

    REASONS = {
        "gpu_idle": 0x1, "applications_clocks_setting": 0x2, "sw_power_cap": 0x4,
        "hw_slowdown": 0x8, "sync_boost": 0x10, "sw_thermal_slowdown": 0x20,
        "hw_thermal_slowdown": 0x40, "hw_power_brake_slowdown": 0x80,
        "display_clock_setting": 0x100,
    }

    def __init__(self, index: int, period_s: float = 0.002):
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
    """ms over `steps` calls of fn, CUDA events on `stream`, synchronized and
    barriered on both sides (every rank calls it the same number of times)."""
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


def _live_copy_gbs(dev) -> float:
    """This GPU's copy bandwidth now, the method of the measured peak: torch
    copy_ of 1 Gi bf16 elements, read + write bytes, best of 10, CUDA events."""
    a = torch.empty(1 << 30, dtype=torch.bfloat16, device=dev)
    b = torch.empty_like(a)
    best = float("inf")
    for _ in range(11):
        s, e = torch.cuda.Event(enable_timing=True), torch.cuda.Event(enable_timing=True)
        s.record()
        b.copy_(a)
        e.record()
        e.synchronize()
        best = min(best, s.elapsed_time(e))
    del a, b
    torch.cuda.empty_cache()
    return 2 * (1 << 30) * 2 / (best * 1e-3) / 1e9


def _host_threads() -> int:
    try:
        return len(os.sched_getaffinity(0))
    except (AttributeError, OSError):
        return os.cpu_count() or 1


def _load_reference_ext():
    """The reference's own extension (its dwconv_ws / dwconv_v0 kernels), built
    from its sources into baseline/_ref; None when absent."""
    paths = sorted(glob.glob(os.path.join(REPO, "baseline", "_ref", "_tma_dwconv_ref_C*.so")))
    if not paths:
        return None
    spec = importlib.util.spec_from_file_location("_tma_dwconv_ref_C", paths[0])
    mod = importlib.util.module_from_spec(spec)
    spec.loader.exec_module(mod)
    return mod


def _ref_dwconv_cpu(x_nhwc: torch.Tensor, w_rsc: torch.Tensor, pad: int) -> torch.Tensor:
    """The reference's CPU path for the operator, ``ref_dwconv``
    (``tma_dwconv.py:14-34``): NHWC -> NCHW copy, ``F.conv2d(groups=C)``, back."""
    C = x_nhwc.shape[3]
    x = x_nhwc.permute(0, 3, 1, 2).contiguous()
    w = w_rsc.permute(2, 0, 1).unsqueeze(1).contiguous()
    y = torch.nn.functional.conv2d(x, w, bias=None, stride=1, padding=pad, groups=C)
    return y.permute(0, 2, 3, 1).contiguous()


# ----------------------------- CPU baseline leg -----------------------------

def _cpu_baseline_leg(wl, x_cpu, w_cpu, y_dev_images, timed: bool) -> tuple[dict | None, bool]:
    """The oracle (the C restatement of the reference arithmetic, all host
    threads) on the images of x_cpu: timed when `timed` (rank 0 at N = 1, the
    cpu_baseline object), and in every case the checker of the GPU result for
    the same images (`y_dev_images`, bit for bit).  Returns (baseline, equal)."""
    sys.path.insert(0, os.path.join(REPO, "oracle"))
    import numpy as np
    import oracle  # the checker / CPU baseline only
    threads = _host_threads()
    xs, ws = x_cpu.numpy(), w_cpu.numpy()
    got = y_dev_images.cpu().numpy()
    if not timed:
        ref = oracle.dwconv_f16(xs, ws, wl.pad, threads=threads)
        return None, bool(np.array_equal(got.view(np.uint16), ref.view(np.uint16)))
    oracle.dwconv_f16(xs[:1], ws, wl.pad, threads=threads)  # warm-up (page in, OpenMP pool)
    best, ref = float("inf"), None
    for _ in range(2):
        t0 = time.perf_counter()
        ref = oracle.dwconv_f16(xs, ws, wl.pad, threads=threads)
        best = min(best, time.perf_counter() - t0)
    images = xs.shape[0]
    s_img = best / images
    base = {"value": round(wl.bytes_per_call(1) / s_img / 1e9, 3), "unit": "GB/s",
            "cores": threads, "kind": "port",
            "sample": f"{images} of {wl.N} images, best of 2; C oracle (fp32 fma chain, OpenMP); "
                      f"{s_img * wl.N * 1e3:.0f} ms per full call extrapolated"}
    try:
        t_img, path = _ref_cpu_rate(wl, x_cpu[:2], w_cpu)
        base["torch_conv2d"] = {"value": round(wl.bytes_per_call(1) / t_img / 1e9, 3), "unit": "GB/s",
                                "threads": threads, "path": path,
                                "ms_per_call_extrapolated": round(t_img * wl.N * 1e3, 1)}
    except Exception as e:  # reported only
        base["torch_conv2d"] = {"error": str(e)[:200]}
    return base, bool(np.array_equal(got.view(np.uint16), ref.view(np.uint16)))


def _cpu_candidates(x_cpu, w_cpu, pad):
    """torch's CPU convolutions of the operator: the reference's ``ref_dwconv``
    as written (NCHW copies in and out) and ``conv2d(groups=C)`` on the
    channels-last view of the NHWC data (the same arithmetic without the
    copies), each on the fp16 data and on float32 copies."""
    C = x_cpu.shape[3]
    out = {}
    for dt, (xx, ww) in {"float32": (x_cpu.float(), w_cpu.float()), "float16": (x_cpu, w_cpu)}.items():
        out[f"ref_dwconv {dt}"] = lambda xs, xx=xx, ww=ww: _ref_dwconv_cpu(xx[xs], ww, pad)
        wc = ww.permute(2, 0, 1).unsqueeze(1).contiguous()
        out[f"conv2d channels-last {dt}"] = (
            lambda xs, xx=xx, wc=wc: torch.nn.functional.conv2d(xx[xs].permute(0, 3, 1, 2), wc,
                                                                padding=pad, groups=C))
    return out


def _ref_cpu_rate(wl, x_cpu, w_cpu, repeats: int = 1) -> tuple[float, str]:
    """Seconds per image of the fastest of torch's CPU paths (_cpu_candidates)
    on the host cores over x_cpu's images (the choice made on one image)."""
    torch.set_num_threads(_host_threads())
    cands = _cpu_candidates(x_cpu, w_cpu, wl.pad)
    one = {}
    for name, f in cands.items():
        f(slice(0, 1))
        t0 = time.perf_counter()
        f(slice(0, 1))
        one[name] = time.perf_counter() - t0
    name = min(one, key=one.get)
    best = float("inf")
    for _ in range(repeats):
        t0 = time.perf_counter()
        cands[name](slice(None))
        best = min(best, time.perf_counter() - t0)
    return best / x_cpu.shape[0], name


# ----------------------------- reference arm --------------------------------

def run_reference(args, wl) -> None:
    """CPU arm: the reference's own CPU path (``ref_dwconv``) on the host cores.
    One step = ``--ref-images`` images of the batch (the same seeded images the
    GPU arm convolves)."""
    rank, world, _ = tdc_dist.env_rank()
    if rank != 0:
        return
    images = min(args.ref_images, wl.N)
    x, w = make_inputs(wl, "cpu", seed=0, n=images)
    threads = _host_threads()
    torch.set_num_threads(threads)  # every core (torchrun sets OMP_NUM_THREADS=1)
    # the fastest of torch's CPU paths for the operator, chosen on one image
    _, path = _ref_cpu_rate(wl, x[:1], w)
    f = _cpu_candidates(x, w, wl.pad)[path]
    for _ in range(args.warmup):
        f(slice(None))
    t0 = time.perf_counter()
    for _ in range(args.steps):
        f(slice(None))
    dt = (time.perf_counter() - t0) / args.steps
    gbs = wl.bytes_per_call(images) / dt / 1e9
    line = {
        "impl": "reference", "metric": METRIC, "value": round(gbs, 3), "unit": "GB/s",
        "n_gpus": world, "steps": args.steps, "warmup": args.warmup,
        "ms_per_step": round(dt * 1e3, 4), "higher_is_better": True,
        "scaling": "strong" if world > 1 and not args.weak else "weak",
        "vs_baseline": None, "dtype": f"{path.split()[-1]} (fp16 data; the fastest of the paths below)",
        "data": "synthetic (seeded)",
        "config": {"workload": wl.name, "N": wl.N, "H": wl.H, "W": wl.W, "C": wl.C,
                   "pad": wl.pad, "step": f"{images} images of the batch on the host CPU",
                   "path": f"{path}: the fastest on this host of ref_dwconv (reference "
                           "tma_dwconv.py:14-34: NHWC->NCHW copy, torch.nn.functional.conv2d(groups=C), "
                           "back) and conv2d(groups=C) on the channels-last view (no copies), in fp16 "
                           "and float32"},
        "ms_per_call_extrapolated": round(dt * wl.N / images * 1e3, 1),
        "cpu_baseline": {"value": round(gbs, 3), "unit": "GB/s", "cores": threads, "kind": "reference",
                         "sample": f"{images} of {wl.N} images per step, {args.steps} steps; "
                                   f"torch {path} on {threads} threads"},
        "e2e": {"value": round(gbs, 3), "unit": "GB/s", "h2d_bytes_per_step": 0,
                "d2h_bytes_per_step": 0},
        "gpu_launches": 0,
    }
    print(json.dumps(line), flush=True)


# ----------------------------- GPU arm ---------------------------------------

def _e2e(args, wl, T, x, w, y, stream, dev, total_bytes) -> dict:
    """Same metric through the public API with host buffers: every step is one
    ``tma_dwconv.dwconv_ws_host`` call, which copies w and x host->device
    (pinned), runs the kernel and copies y device->host, pipelined over
    chunks of images so the two copy directions overlap.  Beside it, the
    ceiling: plain pinned copies of the same bytes, both directions at once
    (one cudaMemcpyAsync per direction on two streams), all ranks at once."""
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

    # copy ceiling: H2D of x and D2H of y at the same time
    s_h2d = torch.cuda.Stream(dev)
    s_d2h = torch.cuda.Stream(dev)
    xd = torch.empty_like(x)

    def copies():
        ev = torch.cuda.Event()
        ev.record(stream)
        s_h2d.wait_event(ev)
        s_d2h.wait_event(ev)
        with torch.cuda.stream(s_h2d):
            xd.copy_(xh, non_blocking=True)
        with torch.cuda.stream(s_d2h):
            yh.copy_(y, non_blocking=True)
        stream.wait_stream(s_h2d)
        stream.wait_stream(s_d2h)

    copies()
    cms = tdc_dist.max_over_ranks(_cuda_time(copies, steps, stream), dev) / steps
    del xd
    value = total_bytes / (ms * 1e-3) / 1e9
    ceiling = total_bytes / (cms * 1e-3) / 1e9
    return {"value": round(value, 3), "unit": "GB/s",
            "ms_per_step": round(ms, 3), "h2d_bytes_per_step": x.numel() * 2 + w.numel() * 2,
            "d2h_bytes_per_step": y.numel() * 2, "steps": steps,
            "copy_ceiling_gbs": round(ceiling, 3), "copy_ceiling_ms": round(cms, 3),
            "frac_of_copy_ceiling": round(value / ceiling, 4),
            "path": "tma_dwconv.dwconv_ws_host (tdc_dwconv_ws_host: H2D / kernel / D2H "
                    "pipelined over chunks of images)",
            "ceiling": "pinned x H2D and y D2H of the same bytes at once, every rank at once"}


def _comparisons(args, ref_ext, x, w, pad, C, stream, dev, iters: int) -> dict:
    """The reference's ws kernel (n_stage 2) and cuDNN on the same device
    inputs, max over ranks (every rank runs the same steps)."""
    out = {}
    if ref_ext is not None:
        f = lambda: ref_ext.dwconv_ws(x, w, pad, 2)
        for _ in range(3):
            f()
        out["reference_ws_us"] = tdc_dist.max_over_ranks(_cuda_time(f, iters, stream), dev) / iters * 1e3
        torch.cuda.empty_cache()
    if not args.no_cudnn:
        xc = x.permute(0, 3, 1, 2)  # channels_last view, no copy
        wc = w.permute(2, 0, 1).unsqueeze(1).contiguous()
        f = lambda: torch.nn.functional.conv2d(xc, wc, padding=pad, groups=C)
        for _ in range(3):
            f()
        out["cudnn_channels_last_us"] = tdc_dist.max_over_ranks(_cuda_time(f, iters, stream), dev) / iters * 1e3
        if x.numel() * 2 * 2 < 40e9:
            xn = x.permute(0, 3, 1, 2).contiguous()
            f2 = lambda: torch.nn.functional.conv2d(xn, wc, padding=pad, groups=C)
            for _ in range(3):
                f2()
            out["cudnn_nchw_us"] = tdc_dist.max_over_ranks(_cuda_time(f2, iters, stream), dev) / iters * 1e3
            del xn
        torch.cuda.empty_cache()
    return {k: round(v, 2) for k, v in out.items()}


def _graph_us(fn, iters: int, stream) -> float | None:
    """µs per call of `iters` calls of fn captured in one CUDA graph and
    replayed: the device time of back-to-back calls without the host's launch
    path (Python, binding, C ABI, launch), which small problems can fall below."""
    try:
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
        us = _cuda_time(g.replay, 5, stream) / 5 * 1e3 / iters
        del g
        return us
    except Exception:  # reported only
        return None


def _device_warmup(fn, seconds: float) -> int:
    """Calls fn for `seconds` (synchronising every 4 calls); returns the count.
    In a fresh process, or after a fifth of a second idle, the GPU runs the
    first ~0.1 s of calls 5-10 % slower than the calls after them."""
    t_end = time.perf_counter() + seconds
    calls = 0
    while time.perf_counter() < t_end:
        for _ in range(4):
            fn()
        calls += 4
        torch.cuda.synchronize()
    return calls


def _time_workload(T, wl, n0, n1, dev, stream, n_stage, iters, warmup, rotate: int = 1,
                   graph: bool = False, device_warmup: float = 0.0):
    """µs per call of dwconv_ws on images [n0, n1) of wl (max over ranks), the
    output of the last call, and the inputs.  `rotate` > 1 cycles through that
    many input/output copies (L2-cold inputs for workloads smaller than L2)."""
    n = n1 - n0
    x, w = make_inputs(wl, dev, seed=0, n=n, n_offset=n0)
    xs = [x] + [x.clone() for _ in range(rotate - 1)]
    ys = [torch.empty((n, wl.P, wl.Q, wl.C), dtype=torch.float16, device=dev) for _ in range(rotate)]
    k = [0]

    def f():
        i = k[0] % rotate
        T.dwconv_ws_out(xs[i], w, ys[i], wl.pad, n_stage)
        k[0] += 1

    _device_warmup(f, device_warmup)
    for _ in range(warmup):
        f()
    us = tdc_dist.max_over_ranks(_cuda_time(f, iters, stream), dev) / iters * 1e3
    y = ys[(k[0] - 1) % rotate]
    if graph:
        return us, x, w, y, _graph_us(f, iters, stream)
    return us, x, w, y


def run_tdc(args, wl) -> None:
    rank, world, local = tdc_dist.init("nccl", timeout_s=120.0)
    torch.cuda.set_device(local)
    dev = torch.device("cuda", local)
    import tma_dwconv as T

    weak_headline = args.weak or world == 1
    per_rank = args.images or wl.N
    if weak_headline:
        n0, n1 = rank * per_rank, (rank + 1) * per_rank
    else:
        n0, n1 = shard_range(per_rank, world, rank)
    n = n1 - n0
    x, w = make_inputs(wl, dev, seed=0, n=n, n_offset=n0)
    stream = torch.cuda.current_stream(dev)
    peak, peak_kind = _peaks()
    ref_ext = None if args.kernel_only else _load_reference_ext()

    def step():
        return T.dwconv_ws(x, w, wl.pad, args.n_stage)

    sampler = ClockSampler(local)  # NVML set-up now, not between the warm-up and the timed steps
    # Device warm-up before the W warm-up steps: in a fresh process, or after
    # a fifth of a second idle, the first ~100 calls of this workload run
    # 5-10 % slower than the calls after them (880 vs 790-820 µs per call,
    # measured call by call; the GPU's clocks ramp under sustained load), so
    # the timed steps follow `--device-warmup` seconds of the same calls.
    warm_calls = _device_warmup(step, args.device_warmup)
    for _ in range(max(args.warmup, 3)):
        y = step()
    torch.cuda.synchronize()

    with sampler as clocks:
        ms = _cuda_time(step, args.steps, stream)
    ms_max = tdc_dist.max_over_ranks(ms, dev)
    per_call_ms = ms_max / args.steps
    my_bytes = wl.bytes_per_call(n)
    total_bytes = tdc_dist.sum_over_ranks(float(my_bytes), dev)
    gbs = total_bytes / (per_call_ms * 1e-3) / 1e9
    local_ms = ms / args.steps
    achieved = my_bytes / (local_ms * 1e-3) / 1e9
    traffic, traffic_src = _traffic_per_call(wl.name, n)
    live = _live_copy_gbs(dev)  # after the timed region

    line = {
        "metric": METRIC, "value": round(gbs, 2), "unit": "GB/s", "n_gpus": world,
        "steps": args.steps, "warmup": max(args.warmup, 3), "ms_per_step": round(per_call_ms, 5),
        "higher_is_better": True, "scaling": "weak" if weak_headline else "strong",
        "vs_baseline": None, "dtype": "f16 in/out, f32 accumulate", "data": "synthetic (seeded)",
        "config": {"workload": wl.name, "N_per_rank": n,
                   "global_batch": int(tdc_dist.sum_over_ranks(float(n), dev)), "H": wl.H, "W": wl.W,
                   "C": wl.C, "pad": wl.pad, "n_stage": args.n_stage,
                   "parallelism": f"dp{world} (batch split over the GPUs, no collective)",
                   "l2": "inputs larger than L2 (no flush needed)",
                   "device_warmup": f"{warm_calls} calls ({args.device_warmup} s) before the "
                                    f"warm-up steps: the first ~100 calls of a fresh process run "
                                    f"5-10 % slower"},
        "us_per_call": round(per_call_ms * 1e3, 2),
        "roofline": {"bound": "hbm", "achieved": round(achieved, 1), "peak": peak, "unit": "GB/s",
                     "frac": round(achieved / peak, 4), "peak_source": peak_kind,
                     "traffic": None if traffic is None else round(traffic),
                     "traffic_source": traffic_src,
                     "algorithmic_bytes": my_bytes, "kernel": "dwconv_ws_kernel",
                     "live_copy_gbs": round(live, 1), "frac_of_live_copy": round(achieved / live, 4)},
        "gpu_launches": args.steps,
        "clocks": clocks.summary(),
    }
    if not args.kernel_only:
        # Same-run comparisons on the same inputs (outside the timed region).
        cmp_ = _comparisons(args, ref_ext, x, w, wl.pad, wl.C, stream, dev, iters=10)
        line.update({k: v for k, v in cmp_.items()})
        if "reference_ws_us" in cmp_:
            line["reference_ws_speedup"] = round(cmp_["reference_ws_us"] / (per_call_ms * 1e3), 3)
        elif ref_ext is None:
            line["reference_ws_us"] = None
            line["reference_ws"] = "unavailable: baseline/_ref holds no build of the reference extension"
        # End to end through the public API with host buffers.
        line["e2e"] = _e2e(args, wl, T, x, w, y, stream, dev, total_bytes)

    # CPU baseline leg, which is also the checker of every rank's shard: the
    # oracle on images of this rank's shard against the GPU output for them.
    images = min(n, args.cpu_images) if (rank == 0 and world == 1) else min(n, 1)
    check_ok = True
    cpu = None
    if images > 0 and not args.no_cpu:
        lo = n - images  # the last images of the shard
        cpu, check_ok = _cpu_baseline_leg(wl, x[lo:].cpu(), w.cpu(), y[lo:],
                                          timed=(rank == 0 and world == 1))
    line["cpu_baseline"] = cpu
    checked = [f"{wl.name}: image {n0 + n - images}..{n1 - 1} of rank {rank}"] if images else []
    del y
    torch.cuda.empty_cache()

    if world > 1 and not args.kernel_only:
        # the other figures at N > 1: 64 images per rank, and the split of the
        # other multi-GPU workloads
        if not weak_headline:
            us_w, xw, ww, yw = _time_workload(T, wl, rank * wl.N, (rank + 1) * wl.N, dev, stream,
                                              args.n_stage, iters=10, warmup=3,
                                              device_warmup=args.device_warmup)
            tot = tdc_dist.sum_over_ranks(float(wl.bytes_per_call(wl.N)), dev)
            line["weak"] = {"images_per_rank": wl.N, "us_per_call": round(us_w, 2),
                            "value": round(tot / (us_w * 1e-6) / 1e9, 2), "unit": "GB/s"}
            del xw, ww, yw
            torch.cuda.empty_cache()
        split = {}
        for name in SPLIT_WORKLOADS:
            swl = WORKLOADS[name]
            s0, s1 = shard_range(swl.N, world, rank)
            iters = 100 if swl.bytes_per_call() < 1e9 else 30
            us, xs, wsw, ys = _time_workload(T, swl, s0, s1, dev, stream, args.n_stage, iters, 10,
                                             device_warmup=args.device_warmup)
            ok = True
            if s1 > s0 and not args.no_cpu:
                _, ok = _cpu_baseline_leg(swl, xs[-1:].cpu(), wsw.cpu(), ys[-1:], timed=False)
                checked.append(f"{name}: image {s1 - 1} of rank {rank}")
            check_ok = check_ok and ok
            agg = swl.bytes_per_call() / (us * 1e-6) / 1e9
            cmp_ = _comparisons(args, ref_ext, xs, wsw, swl.pad, swl.C, stream, dev, iters=10)
            split[name] = {"images_per_rank": s1 - s0, "us_per_call": round(us, 2),
                           "value": round(agg, 2), "unit": "GB/s",
                           "frac_of_n_peaks": round(agg / (world * peak), 4), **cmp_}
            del xs, wsw, ys
            torch.cuda.empty_cache()
        line["strong_split"] = split

    if world == 1 and not args.kernel_only:
        per = {}
        for name in PER_CONFIG:
            pwl = WORKLOADS[name]
            small = pwl.bytes_per_call() < 1e9
            timed = _time_workload(T, pwl, 0, pwl.N, dev, stream, args.n_stage, 100, 10, graph=small,
                                   device_warmup=args.device_warmup)
            us, xp, wp, yp = timed[:4]
            nbytes = pwl.bytes_per_call()
            ent = {"us_per_call": round(us, 2), "value": round(nbytes / (us * 1e-6) / 1e9, 2),
                   "unit": "GB/s", "frac": round(nbytes / (us * 1e-6) / 1e9 / peak, 4),
                   "method": "10 warm-up + 100 back-to-back calls (reference tests/bench.py:18-29)"}
            if small and timed[4] is not None:
                ent["us_per_call_graph"] = round(timed[4], 2)
                ent["graph"] = "the same 100 calls captured in one CUDA graph and replayed (device time)"
            if nbytes * 2 < 126e6:
                ent["l2"] = "hot: the same buffers every call (inputs and outputs fit in L2)"
                us_r, _, _, _ = _time_workload(T, pwl, 0, pwl.N, dev, stream, args.n_stage, 100, 10,
                                               rotate=8, device_warmup=args.device_warmup)
                ent["us_per_call_l2_cold"] = round(us_r, 2)
                ent["l2_cold"] = "8 rotating input/output sets (205 MB > L2)"
            else:
                ent["l2"] = "inputs larger than L2"
            if not args.no_cpu:
                _, ok = _cpu_baseline_leg(pwl, xp[-1:].cpu(), wp.cpu(), yp[-1:], timed=False)
                checked.append(f"{name}: image {pwl.N - 1}")
                check_ok = check_ok and ok
            ent.update(_comparisons(args, ref_ext, xp, wp, pwl.pad, pwl.C, stream, dev, iters=20))
            if ent.get("reference_ws_us"):
                ent["reference_ws_speedup"] = round(ent["reference_ws_us"] / us, 3)
            per[name] = ent
            del xp, wp, yp
            torch.cuda.empty_cache()
        line["per_config"] = per

    all_ok = tdc_dist.max_over_ranks(0.0 if check_ok else 1.0, dev) == 0.0
    line["shards_checked"] = bool(all_ok) if not args.no_cpu else None
    line["shards_checked_what"] = ("every rank: the last image of its shard of each timed workload "
                                   "(and, at N = 1, the CPU-baseline sample), bit for bit against "
                                   "the oracle")
    if rank == 0:
        print(json.dumps(line), flush=True)
    tdc_dist.finalize()
    if not all_ok:
        sys.exit(3)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--gpus", type=int, default=1)
    ap.add_argument("--steps", type=int, default=200)
    ap.add_argument("--warmup", type=int, default=10)
    ap.add_argument("--impl", choices=["tdc", "reference"], default="tdc")
    ap.add_argument("--workload", default=HEADLINE, choices=sorted(WORKLOADS))
    ap.add_argument("--n-stage", type=int, default=2, choices=[2, 3, 4])
    ap.add_argument("--weak", action="store_true",
                    help="N > 1: every rank convolves the whole batch (default: the batch is split)")
    ap.add_argument("--device-warmup", type=float, default=0.3,
                    help="seconds of untimed calls before the warm-up steps (GPU clocks ramp up)")
    ap.add_argument("--e2e-steps", type=int, default=5)
    ap.add_argument("--cpu-images", type=int, default=8)
    ap.add_argument("--ref-images", type=int, default=8,
                    help="--impl reference: images per step")
    ap.add_argument("--no-cpu", action="store_true")
    ap.add_argument("--no-cudnn", action="store_true")
    ap.add_argument("--images", type=int, default=0, help="images of the batch (default: the workload's N)")
    ap.add_argument("--kernel-only", action="store_true",
                    help="time the kernel only (no comparisons, per-config, end-to-end or CPU legs)")
    args = ap.parse_args()
    wl = WORKLOADS[args.workload]
    if args.impl == "reference":
        run_reference(args, wl)
    else:
        run_tdc(args, wl)


if __name__ == "__main__":
    main()
