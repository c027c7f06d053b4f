"""Whole-model inference with the depthwise layers on these kernels, on one GPU.

    python benchmarks/bench_models.py [--batch 64] [--size 224] [--iters 20] [--graphs]
    python benchmarks/bench_models.py --layers [--batch 64]
    python benchmarks/bench_models.py --layers-bwd [--batch 64]
    python benchmarks/bench_models.py --train [--batch 64]
    python benchmarks/bench_models.py --seg [--batch 8] [--size 512]

torchvision MobileNetV2, MobileNetV3-Large and EfficientNet-B0 (random
weights, random BatchNorm statistics), fp16, channels-last, eval mode.  Per
model, ms per forward (CUDA events, 5 warm-up + `iters` calls) for:
  cudnn        the unmodified model (cuDNN depthwise + BatchNorm + activation)
  converted    tdc_torch.convert_depthwise_convs: depthwise convs on these kernels
  fused        tdc_torch.fuse_depthwise_bn_act: BatchNorm folded, activation in
               the depthwise kernel's epilogue
and the largest logit difference of each variant against the unmodified
model.  Eager calls include the host's per-layer launch cost; ``--graphs``
captures each variant's forward once in a CUDA graph and times replays (GPU
time only).  Prints one JSON line per model.

``--layers`` instead times every distinct depthwise layer of the three models
alone (input shape recorded by forward hooks): cuDNN's channels-last conv2d,
the ws kernel (``_C.dwconv_k`` at the default ring depth) and the plain kernel
(``_C.dwconv_plain``), each as 20 back-to-back calls replayed from a CUDA
graph, the kernel the automatic choice takes, and the algorithmic bytes (x
read + y written) per call.  ``--layers-bwd`` does the same for the
gradients: cuDNN's data and weight gradients (``aten.convolution_backward``)
against ``_C.dwconv_bwd_data`` and ``_C.dwconv_bwd_weight`` with the
automatic kernel choice (n_stage 0) and with the ws kernels at their default
depths, and the plain weight gradient.  ``--train`` times a training step
(forward, loss, backward; BatchNorm in training mode) of each model, stock
against ``convert_depthwise_convs``, eager (use a batch of 128 or more so the
GPU, not the host's launches, sets the time).  Both fp16 models' losses
and depthwise weight gradients are compared with an fp32 copy of the model
(relative L2 distance per layer: largest and median).  ``--seg`` times
torchvision's DeepLabV3-MobileNetV3-Large (dilated depthwise layers in its
last stages) stock against ``fuse_depthwise_bn_act`` (CUDA graphs), and each
of its dilated depthwise layers alone against cuDNN.
A script, not a test.
"""
from __future__ import annotations

import argparse
import copy
import json
import os
import sys

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
sys.path[:0] = [os.path.join(REPO, "tma-depthwise-conv_b200")]

import torch  # noqa: E402
import torchvision  # noqa: E402

import tdc_torch  # noqa: E402


def bench_ms(fn, warmup=5, iters=20) -> float:
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


def graphed(m, x):
    """Capture ``m(x)`` in a CUDA graph; returns the replay callable."""
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            m(x)
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        m(x)
    return g.replay


def randomize_bn(model: torch.nn.Module, seed: int) -> None:
    g = torch.Generator().manual_seed(seed)
    for m in model.modules():
        if isinstance(m, torch.nn.BatchNorm2d):
            c = m.num_features
            m.running_mean.copy_(torch.randn(c, generator=g) * 0.2)
            m.running_var.copy_(torch.rand(c, generator=g) + 0.5)
            m.weight.data.copy_(torch.rand(c, generator=g) + 0.5)
            m.bias.data.copy_(torch.randn(c, generator=g) * 0.2)


def depthwise_layers(batch: int, size: int):
    """Distinct (N, H, W, C, K, stride, pad) of the models' depthwise convs."""
    seen = []
    for arch in ("mobilenet_v2", "mobilenet_v3_large", "efficientnet_b0"):
        model = getattr(torchvision.models, arch)().eval()
        hooks = []
        for m in model.modules():
            if (isinstance(m, torch.nn.Conv2d) and m.groups == m.in_channels == m.out_channels
                    and m.in_channels > 1):
                def hook(mod, inp, _out, arch=arch):
                    n, c, h, w = inp[0].shape
                    key = (n, h, w, c, mod.kernel_size[0], mod.stride[0], mod.padding[0])
                    if key not in [k for k, _ in seen]:
                        seen.append((key, arch))
                hooks.append(m.register_forward_hook(hook))
        with torch.no_grad():
            model(torch.zeros(1, 3, size, size))
        for h in hooks:
            h.remove()
    return [((batch,) + key[1:], arch) for key, arch in seen]


def graph_of(fn, reps=20):
    side = torch.cuda.Stream()
    side.wait_stream(torch.cuda.current_stream())
    with torch.cuda.stream(side):
        for _ in range(3):
            fn()
    torch.cuda.current_stream().wait_stream(side)
    g = torch.cuda.CUDAGraph()
    with torch.cuda.graph(g):
        for _ in range(reps):
            fn()
    return g.replay


def bench_layers(batch: int, size: int, iters: int) -> None:
    import tma_dwconv as T
    reps = 20
    tot_c = tot_t = 0.0
    for (n, h, w, c, k, s, pad), arch in depthwise_layers(batch, size):
        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(n, h, w, c, device="cuda", generator=g).half()
        wt = (torch.randn(k, k, c, device="cuda", generator=g) / k).half()
        x_nchw = x.permute(0, 3, 1, 2)                        # channels-last view
        w_conv = wt.permute(2, 0, 1).unsqueeze(1).contiguous()
        cudnn = graph_of(lambda: torch.nn.functional.conv2d(x_nchw, w_conv, None, s, pad,
                                                            groups=c), reps)
        ws = graph_of(lambda: T._C.dwconv_k(x, wt, None, None, s, pad, 0,
                                            T.DWCONV_STAGES[(k, s)]), reps)
        plain = graph_of(lambda: T._C.dwconv_plain(x, wt, None, None, s, pad, 0, 0), reps)
        p, q = (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1
        nbytes = 2 * n * c * (h * w + p * q)
        t_c = bench_ms(cudnn, iters=iters) / reps * 1e3
        t_w = bench_ms(ws, iters=iters) / reps * 1e3
        t_p = bench_ms(plain, iters=iters) / reps * 1e3
        use_plain = T.uses_plain(n, h, w, c, k, s, pad)
        t_t = t_p if use_plain else t_w
        tot_c, tot_t = tot_c + t_c, tot_t + t_t
        print(json.dumps({"model": arch, "N": n, "H": h, "W": w, "C": c, "K": k, "stride": s,
                          "MB": round(nbytes / 1e6, 2), "cudnn_us": round(t_c, 2),
                          "ws_us": round(t_w, 2), "plain_us": round(t_p, 2),
                          "auto": "plain" if use_plain else "ws",
                          "auto_GBps": round(nbytes / t_t / 1e3, 1),
                          "speedup_auto": round(t_c / t_t, 3)}), flush=True)
    print(json.dumps({"layers_total_cudnn_us": round(tot_c, 1),
                      "layers_total_auto_us": round(tot_t, 1)}), flush=True)


def bench_layers_bwd(batch: int, size: int, iters: int) -> None:
    import tma_dwconv as T
    reps = 10
    names = ("cudnn_dx", "cudnn_dw", "dx_auto", "dx_ws", "dw_auto", "dw_ws", "dw_plain")
    tot = dict.fromkeys(names, 0.0)
    conv_bwd = torch.ops.aten.convolution_backward
    for (n, h, w, c, k, s, pad), arch in depthwise_layers(batch, size):
        g = torch.Generator(device="cuda").manual_seed(0)
        x = torch.randn(n, h, w, c, device="cuda", generator=g).half()
        wt = (torch.randn(k, k, c, device="cuda", generator=g) / k).half()
        p, q = (h + 2 * pad - k) // s + 1, (w + 2 * pad - k) // s + 1
        dy = torch.randn(n, p, q, c, device="cuda", generator=g).half()
        x_nchw, dy_nchw = x.permute(0, 3, 1, 2), dy.permute(0, 3, 1, 2)
        w_conv = wt.permute(2, 0, 1).unsqueeze(1).contiguous()

        def cudnn(mask):
            return lambda: conv_bwd(dy_nchw, x_nchw, w_conv, None, [s, s], [pad, pad], [1, 1],
                                    False, [0, 0], c, mask)
        dx_stage, dw_stage = tdc_torch.BWD_STAGES[(k, s)]
        fns = {
            "cudnn_dx": cudnn([True, False, False]),
            "cudnn_dw": cudnn([False, True, False]),
            "dx_auto": lambda: T._C.dwconv_bwd_data(dy, wt, pad, s, 0, h, w),
            "dx_ws": lambda: T._C.dwconv_bwd_data(dy, wt, pad, s, dx_stage, h, w),
            "dw_auto": lambda: T._C.dwconv_bwd_weight(x, dy, k, pad, s, 0),
            "dw_ws": lambda: T._C.dwconv_bwd_weight(x, dy, k, pad, s, dw_stage),
            "dw_plain": lambda: T._C.dwconv_bwd_weight_plain(x, dy, k, pad, s),
        }
        row = {"model": arch, "N": n, "H": h, "W": w, "C": c, "K": k, "stride": s,
               "dw_uses_plain": bool(T._C.dwconv_bwd_weight_uses_plain(n, h, w, c, k, s, pad))}
        for name, fn in fns.items():
            t = bench_ms(graph_of(fn, reps), iters=iters) / reps * 1e3
            row[name + "_us"] = round(t, 2)
            tot[name] += t
        print(json.dumps(row), flush=True)
    print(json.dumps({"totals_us": {k_: round(v, 1) for k_, v in tot.items()}}), flush=True)


def bench_train(batch: int, size: int, iters: int) -> None:
    x = torch.randn(batch, 3, size, size, device="cuda").half()
    x = x.to(memory_format=torch.channels_last)
    for arch in ("mobilenet_v2", "mobilenet_v3_large", "efficientnet_b0"):
        torch.manual_seed(0)
        base = getattr(torchvision.models, arch)().train().cuda().half()
        base = base.to(memory_format=torch.channels_last)
        converted = copy.deepcopy(base)
        n_conv = tdc_torch.convert_depthwise_convs(converted)
        ref32 = copy.deepcopy(base).float()
        row = {"model": arch, "batch": batch, "size": size, "depthwise_converted": n_conv}
        grads = {}
        for name, m in (("fp32", ref32), ("cudnn", base), ("converted", converted)):
            xin = x.float() if name == "fp32" else x

            def step(m=m, xin=xin):
                # a sum, not a mean: keeps the fp16 gradients of the first
                # layers above fp16's underflow (no loss scaling here)
                loss = m(xin).float().square().sum()
                loss.backward()
                return loss
            for p_ in m.parameters():
                p_.grad = None
            first = step()
            dws = [mod.weight.grad.float().clone() for mod in m.modules()
                   if isinstance(mod, tdc_torch.DepthwiseConv2d)
                   or (isinstance(mod, torch.nn.Conv2d) and mod.groups == mod.in_channels > 1)]
            grads[name] = (first.item(), dws)
            for p_ in m.parameters():
                p_.grad = None
            if name != "fp32":
                row[f"{name}_ms"] = round(bench_ms(step, iters=iters), 3)
        (lr, gr), (l0, g0), (l1, g1) = grads["fp32"], grads["cudnn"], grads["converted"]

        def rel(ga, gb):  # per depthwise layer, relative L2 distance of gb from ga
            return [((b - a).norm() / a.norm()).item() for a, b in zip(ga, gb)]
        for tag, (l_, g_) in (("cudnn", (l0, g0)), ("converted", (l1, g1))):
            d = rel(gr, g_)
            row[f"{tag}_vs_fp32"] = {"loss": abs(l_ - lr) / abs(lr),
                                     "dw_max": round(max(d), 4),
                                     "dw_median": round(sorted(d)[len(d) // 2], 4),
                                     "finite": all(bool(t.isfinite().all()) for t in g_)}
        row["speedup"] = round(row["cudnn_ms"] / row["converted_ms"], 3)
        print(json.dumps(row), flush=True)


def bench_seg(batch: int, size: int, iters: int) -> None:
    import tma_dwconv as T
    from torchvision.models import segmentation as seg
    torch.manual_seed(0)
    base = seg.deeplabv3_mobilenet_v3_large(weights=None, weights_backbone=None,
                                            num_classes=21, aux_loss=False)
    randomize_bn(base, 1)
    base = base.eval().cuda().half().to(memory_format=torch.channels_last)
    layers = []
    for m in base.modules():
        if isinstance(m, torch.nn.Conv2d) and m.groups == m.in_channels > 1 and m.dilation[0] > 1:
            m.register_forward_hook(lambda mod, inp, out: layers.append(
                (tuple(inp[0].shape), mod.kernel_size[0], mod.stride[0], mod.dilation[0],
                 mod.padding[0])))
    x = torch.randn(batch, 3, size, size, device="cuda").half()
    x = x.to(memory_format=torch.channels_last)
    with torch.no_grad():
        ref = base(x)["out"].float()
        for m in base.modules():
            m._forward_hooks.clear()
        fused = copy.deepcopy(base)
        n_fused = tdc_torch.fuse_depthwise_bn_act(fused)
        row = {"model": "deeplabv3_mobilenet_v3_large", "batch": batch, "size": size,
               "blocks_fused": n_fused,
               "max_logit_diff": round((fused(x)["out"].float() - ref).abs().max().item(), 4),
               "logit_scale": round(ref.abs().max().item(), 3)}
        for name, m in (("cudnn", base), ("fused", fused)):
            row[f"{name}_ms"] = round(bench_ms(graphed(lambda inp, m=m: m(inp)["out"], x),
                                               iters=iters), 3)
        row["speedup"] = round(row["cudnn_ms"] / row["fused_ms"], 3)
        print(json.dumps(row), flush=True)
        reps = 20
        for (n, c, h, w), k, s, d, pad in dict.fromkeys(layers):
            g = torch.Generator(device="cuda").manual_seed(0)
            xl = torch.randn(n, h, w, c, device="cuda", generator=g).half()
            wt = (torch.randn(k, k, c, device="cuda", generator=g) / k).half()
            w_conv = wt.permute(2, 0, 1).unsqueeze(1).contiguous()
            xn = xl.permute(0, 3, 1, 2)
            cud = graph_of(lambda: torch.nn.functional.conv2d(xn, w_conv, None, s, pad, d, c), reps)
            ours = graph_of(lambda: T.dwconv(xl, wt, pad, stride=s, dilation=d), reps)
            t_c = bench_ms(cud, iters=iters) / reps * 1e3
            t_o = bench_ms(ours, iters=iters) / reps * 1e3
            p = (h + 2 * pad - d * (k - 1) - 1) // s + 1
            q = (w + 2 * pad - d * (k - 1) - 1) // s + 1
            nbytes = 2 * n * c * (h * w + p * q)
            print(json.dumps({"N": n, "H": h, "W": w, "C": c, "K": k, "stride": s, "dilation": d,
                              "cudnn_us": round(t_c, 2), "ours_us": round(t_o, 2),
                              "ours_GBps": round(nbytes / t_o / 1e3, 1),
                              "speedup": round(t_c / t_o, 3)}), flush=True)


def main() -> None:
    ap = argparse.ArgumentParser()
    ap.add_argument("--batch", type=int, default=64)
    ap.add_argument("--size", type=int, default=224)
    ap.add_argument("--iters", type=int, default=20)
    ap.add_argument("--graphs", action="store_true", help="time CUDA-graph replays")
    ap.add_argument("--layers", action="store_true", help="time each depthwise layer alone")
    ap.add_argument("--layers-bwd", action="store_true", help="time each layer's gradients")
    ap.add_argument("--train", action="store_true", help="time a training step per model")
    ap.add_argument("--seg", action="store_true", help="DeepLabV3-MobileNetV3 (dilated layers)")
    args = ap.parse_args()
    if args.seg:
        bench_seg(8 if args.batch == 64 else args.batch, 512 if args.size == 224 else args.size,
                  args.iters)
        return
    if args.train:
        bench_train(args.batch, args.size, args.iters)
        return
    if args.layers_bwd:
        bench_layers_bwd(args.batch, args.size, args.iters)
        return
    if args.layers:
        bench_layers(args.batch, args.size, args.iters)
        return
    x = torch.randn(args.batch, 3, args.size, args.size, device="cuda").half()
    x = x.to(memory_format=torch.channels_last)
    for arch in ("mobilenet_v2", "mobilenet_v3_large", "efficientnet_b0"):
        torch.manual_seed(0)
        base = getattr(torchvision.models, arch)()
        randomize_bn(base, 1)
        base = base.eval().cuda().half().to(memory_format=torch.channels_last)
        converted = copy.deepcopy(base)
        n_conv = tdc_torch.convert_depthwise_convs(converted)
        fused = copy.deepcopy(base)
        n_fused = tdc_torch.fuse_depthwise_bn_act(fused)
        row = {"model": arch, "batch": args.batch, "size": args.size,
               "depthwise_converted": n_conv, "blocks_fused": n_fused,
               "mode": "cuda_graph" if args.graphs else "eager"}
        with torch.no_grad():
            ref = base(x).float()
            for name, m in (("cudnn", base), ("converted", converted), ("fused", fused)):
                fn = graphed(m, x) if args.graphs else (lambda: m(x))
                row[f"{name}_ms"] = round(bench_ms(fn, iters=args.iters), 3)
                if name != "cudnn":
                    row[f"{name}_max_logit_diff"] = round((m(x).float() - ref).abs().max().item(), 4)
            row["logit_scale"] = round(ref.abs().max().item(), 3)
        row["speedup_fused_vs_cudnn"] = round(row["cudnn_ms"] / row["fused_ms"], 3)
        print(json.dumps(row), flush=True)


if __name__ == "__main__":
    main()
