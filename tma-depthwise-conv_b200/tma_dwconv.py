"""NHWC fp16 depthwise 3x3 conv2d forward on B200 (sm_100a): Python API.

Drop-in for the reference module ``tma_dwconv`` (haowen-han/tma-depthwise-conv
``tma_dwconv.py:1-110``): the same four public functions with the same
signatures, argument checks and ``ValueError`` messages, backed by the
``_tma_dwconv_C`` extension, which calls the C ABI of ``libtdc_sm100.so``.
There is no CPU fallback: importing this module fails if the extension is not
built, and every call needs CUDA tensors.

Layouts: x ``[N, H, W, C]`` fp16, w ``[R, S, C]`` fp16 (R = S = 3), output
``[N, P, Q, C]`` fp16 with P = H + 2*pad - 2, Q = W + 2*pad - 2.  Arithmetic:
fp32 multiply-add chain over the taps in (r, s) order from +0, one
round-to-nearest-even to fp16.
"""
from __future__ import annotations

import torch
import torch.nn.functional as F

import _tma_dwconv_C as _C  # type: ignore

__all__ = ["dwconv_v0", "dwconv_ws", "dwconv_ws_probe", "ref_dwconv",
           "dwconv_ws_out", "dwconv_ws_host", "dwconv3x3", "dwconv", "DWCONV_STAGES", "device_status",
           "set_wait_timeout_ns",
           "CONSUMER_WARPS", "ACTIVATIONS"]

#: Activations the general forward fuses into its epilogue.
ACTIVATIONS = {"none": 0, "relu": 1, "relu6": 2, "silu": 3, "hardswish": 4}

#: Consumer warps per CTA of the ws kernel (divide stall columns 1 and 3 by it
#: for per-warp figures, as the reference's probe report does).
CONSUMER_WARPS: int = int(_C.consumer_warps())


# ------------------------------ reference ----------------------------------

def ref_dwconv(x_nhwc: torch.Tensor, w_rsc: torch.Tensor, pad: int) -> torch.Tensor:
    """Depthwise conv2d via ``torch.nn.functional.conv2d(groups=C)``.

    Same contract as the reference's ``ref_dwconv`` (``tma_dwconv.py:14-34``):
    x ``[N,H,W,C]``, w ``[R,S,C]``, symmetric padding; returns ``[N,P,Q,C]``
    in x's dtype, computed by cuDNN on CUDA tensors or ATen on CPU.
    """
    if x_nhwc.dim() != 4 or w_rsc.dim() != 3:
        raise ValueError("x must be [N,H,W,C] and w must be [R,S,C]")
    C = x_nhwc.shape[3]
    if C != w_rsc.shape[2]:
        raise ValueError("channel mismatch between x and w")
    x = x_nhwc.permute(0, 3, 1, 2).contiguous()
    w = w_rsc.permute(2, 0, 1).unsqueeze(1).contiguous()
    y = F.conv2d(x, w, bias=None, stride=1, padding=pad, groups=C)
    return y.permute(0, 2, 3, 1).contiguous()


# ------------------------------ validation ---------------------------------

def _check(x: torch.Tensor, w: torch.Tensor, pad: int, bf16_ok: bool = False) -> None:
    # Same checks and messages as the reference (tma_dwconv.py:39-53); the
    # K x K forward (``dwconv``) also takes bfloat16.
    if not (x.is_cuda and w.is_cuda):
        raise ValueError("x and w must be CUDA tensors")
    if bf16_ok and x.dtype == torch.bfloat16:
        if w.dtype != torch.bfloat16:
            raise ValueError("x and w must have the same dtype")
    elif x.dtype != torch.float16 or w.dtype != torch.float16:
        raise ValueError("x and w must be fp16" + (" or both bf16" if bf16_ok else ""))
    if x.dim() != 4:
        raise ValueError(f"x must be [N,H,W,C], got shape {tuple(x.shape)}")
    if w.dim() != 3:
        raise ValueError(f"w must be [R,S,C], got shape {tuple(w.shape)}")
    if x.shape[3] != w.shape[2]:
        raise ValueError("x and w must agree on C")
    if not (x.is_contiguous() and w.is_contiguous()):
        raise ValueError("x and w must be contiguous")
    if pad < 0:
        raise ValueError("pad must be non-negative")


def _check_ws(x: torch.Tensor, w: torch.Tensor, pad: int, n_stage: int, name: str) -> None:
    _check(x, w, pad)
    if x.shape[3] % 64 != 0:
        raise ValueError(f"{name} requires C % 64 == 0")
    if n_stage not in (2, 3, 4):
        raise ValueError(f"n_stage must be one of {{2, 3, 4}}, got {n_stage}")


# ------------------------------ public API ---------------------------------

def dwconv_v0(x: torch.Tensor, w: torch.Tensor, pad: int = 1) -> torch.Tensor:
    """Plain kernel: direct 16-byte global loads, 8 channels per thread (C % 8 == 0)."""
    _check(x, w, pad)
    return _C.dwconv_v0(x, w, int(pad))


def dwconv_ws(x: torch.Tensor, w: torch.Tensor,
              pad: int = 1, n_stage: int = 2) -> torch.Tensor:
    """TMA + warp-specialised depthwise conv2d.

    Args:
        x: [N, H, W, C] fp16, contiguous, C % 64 == 0.
        w: [R, S, C]    fp16, contiguous.
        pad: zero-padding on both H and W.
        n_stage: shared-memory ring depth (pipeline stages). Supported: 2, 3, 4.
    """
    _check_ws(x, w, pad, n_stage, "dwconv_ws")
    return _C.dwconv_ws(x, w, int(pad), int(n_stage))


def dwconv_ws_out(x: torch.Tensor, w: torch.Tensor, y: torch.Tensor,
                  pad: int = 1, n_stage: int = 2) -> torch.Tensor:
    """``dwconv_ws`` writing into a preallocated contiguous ``y [N,P,Q,C]``."""
    _check_ws(x, w, pad, n_stage, "dwconv_ws_out")
    return _C.dwconv_ws_out(x, w, y, int(pad), int(n_stage))


def dwconv_ws_host(x: torch.Tensor, w: torch.Tensor, pad: int = 1, n_stage: int = 2,
                   chunk_images: int = 0, out: torch.Tensor | None = None,
                   device: torch.device | int | None = None, sync: bool = True) -> torch.Tensor:
    """``dwconv_ws`` for tensors in host memory, end to end.

    Copies w and x to ``device`` (default: the current CUDA device), runs the
    ws kernel and copies y back into ``out`` (a new pinned CPU tensor when
    None), pipelined over chunks of ``chunk_images`` images (0: N/64 rounded
    up) so the two copy directions and the kernels overlap.  ``x`` and ``w``
    are contiguous fp16 CPU tensors; pin ``x`` (``x.pin_memory()``) for the
    copies to overlap.  With ``sync`` the call returns once ``out`` holds the
    result; otherwise ``out`` is ready when the device's current stream is.
    """
    if x.is_cuda or w.is_cuda:
        raise ValueError("dwconv_ws_host takes CPU tensors (use dwconv_ws for device tensors)")
    if x.dtype != torch.float16 or w.dtype != torch.float16:
        raise ValueError("x and w must be fp16")
    if x.dim() != 4 or w.dim() != 3 or x.shape[3] != w.shape[2]:
        raise ValueError("x must be [N,H,W,C] and w [R,S,C] with the same C")
    if x.shape[3] % 64 != 0:
        raise ValueError("dwconv_ws_host requires C % 64 == 0")
    if n_stage not in (2, 3, 4):
        raise ValueError(f"n_stage must be one of {{2, 3, 4}}, got {n_stage}")
    if pad < 0:
        raise ValueError("pad must be non-negative")
    dev = torch.device("cuda", torch.cuda.current_device() if device is None else
                       (device if isinstance(device, int) else device.index))
    N, H, W, C = x.shape
    P, Q = H + 2 * pad - 2, W + 2 * pad - 2
    if out is None:
        out = torch.empty((N, P, Q, C), dtype=torch.float16, pin_memory=True)
    x, w = x.contiguous(), w.contiguous()
    with torch.cuda.device(dev):
        xd = torch.empty(x.shape, dtype=torch.float16, device=dev)
        wd = torch.empty(w.shape, dtype=torch.float16, device=dev)
        yd = torch.empty(out.shape, dtype=torch.float16, device=dev)
        _C.dwconv_ws_host(x, w, out, xd, wd, yd, int(pad), int(n_stage), int(chunk_images))
        if sync:
            torch.cuda.current_stream(dev).synchronize()
    return out


def dwconv_ws_probe(x: torch.Tensor, w: torch.Tensor,
                    pad: int = 1, n_stage: int = 2):
    """Same as ``dwconv_ws`` but instruments producer/consumer stalls.

    Returns:
        (y, stall): ``y`` is the output tensor; ``stall`` is an int64 CUDA
        tensor of shape ``[num_blocks, 4]``, one row per CTA of the launch
        (the ws grid is persistent, so ``num_blocks`` is the number of CTAs
        resident across the GPU, at most the number of work units):

          * col 0 — producer cycles waiting on ``empty`` barriers
          * col 1 — consumer cycles waiting on ``full`` barriers, summed over
                    the ``CONSUMER_WARPS`` consumer warps
          * col 2 — producer lifetime (cycles)
          * col 3 — consumer lifetime, summed over consumer warps

        Compare ``mean(col 0)`` with ``mean(col 1)/CONSUMER_WARPS``:
          * col0 >> col1  -> consumers are slower; the producer waits for them.
          * col1 >> col0  -> loads are slower; consumers wait for data.
    """
    _check_ws(x, w, pad, n_stage, "dwconv_ws_probe")
    return _C.dwconv_ws_probe(x, w, int(pad), int(n_stage))


def dwconv3x3(x: torch.Tensor, w: torch.Tensor, pad: int = 1,
              bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
              activation: str = "none", n_stage: int = 2) -> torch.Tensor:
    """General forward beyond the reference surface (same kernel as ``dwconv_ws``).

    Any C % 8 == 0 (``dwconv_ws`` keeps the reference's C % 64), and an
    optional fused epilogue computed per output in fp32 with one rounding at
    the end: ``t = conv + bias[c]; t = activation(t); t = t + residual``.

    Args:
        x: [N, H, W, C] fp16 CUDA, contiguous.   w: [3, 3, C] fp16.
        bias: [C] fp16 or None.   residual: [N, P, Q, C] fp16 or None.
        activation: "none", "relu" (t < 0 ? 0 : t), "relu6", "silu" (t / (1 + exp(-t))),
            "hardswish" (t * clamp(t + 3, 0, 6) / 6).
    """
    _check(x, w, pad)
    if w.shape[0] != 3 or w.shape[1] != 3:
        raise ValueError("only 3x3 kernels are supported")
    if x.shape[3] % 8 != 0:
        raise ValueError("dwconv3x3 requires C % 8 == 0")
    if n_stage not in (2, 3, 4):
        raise ValueError(f"n_stage must be one of {{2, 3, 4}}, got {n_stage}")
    if activation not in ACTIVATIONS:
        raise ValueError(f"activation must be one of {sorted(ACTIVATIONS)}, got {activation!r}")
    return _C.dwconv3x3(x, w, bias, residual, int(pad), ACTIVATIONS[activation], int(n_stage))


#: Ring stages ``dwconv`` uses when ``n_stage`` is None, per (K, stride): the
#: fastest of {2, 3, 4} measured on a B200 at 64 x 224 x 336 x 256, pad K // 2.
DWCONV_STAGES = {(3, 1): 2, (3, 2): 4, (5, 1): 4, (5, 2): 2, (7, 1): 3, (7, 2): 4}


def same_padding(H: int, W: int, K: int, stride: int = 1) -> tuple[int, int, int, int]:
    """TensorFlow's "SAME" padding of an H x W input for a K x K kernel:
    (top, bottom, left, right) giving ceil(H / stride) x ceil(W / stride)
    outputs, the odd row / column at the bottom / right."""
    def split(n):
        out = -(-n // stride)
        total = max((out - 1) * stride + K - n, 0)
        return total // 2, total - total // 2
    top, bottom = split(int(H))
    left, right = split(int(W))
    return top, bottom, left, right


def dwconv(x: torch.Tensor, w: torch.Tensor, pad: int | tuple | None = None, stride: int = 1,
           bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
           activation: str = "none", n_stage: int | None = None,
           dilation: int = 1) -> torch.Tensor:
    """K x K depthwise forward, K in {3, 5, 7}, stride 1 or 2 (beyond the reference surface).

    ``y[n,p,q,c] = round(epilogue(sum_{r,s} x[n, stride*p+r-pad, stride*q+s-pad, c] * w[r,s,c]))``,
    fp32 sums in (r, s) order from zero, zero outside the image, one
    rounding to x's dtype (fp16 or bfloat16).  The epilogue is
    ``dwconv3x3``'s.  ``pad`` defaults to K // 2.  ``n_stage`` 2, 3 or 4 runs
    the TMA ring kernel with that depth (for fp16, 3x3 stride 1 is
    ``dwconv3x3``); None leaves the kernel to the library: ``dwconv_plain``
    where ``uses_plain`` says so (few channels, narrow images), else the ring
    kernel at ``DWCONV_STAGES[(K, stride)]``.  The result is the same bit for
    bit either way.

    ``pad`` may also be a tuple (top, bottom, left, right) of per-side zero
    padding (e.g. ``same_padding(H, W, K, stride)``, TensorFlow's "SAME"):
    the top / left sides shift the taps, P = (H + top + bottom - K) // stride
    + 1 and Q likewise.  ``dilation`` D > 1 spaces the taps D apart (tap (r,
    s) reads x[n, stride*p + D*r - top, stride*q + D*s - left, c]; K becomes
    D*(K-1) + 1 in the output size), on a kernel that computes each output's
    taps directly (``n_stage`` is then ignored); same chain and rounding.

    Args:
        x: [N, H, W, C] fp16 or bf16 CUDA, contiguous, C % 8 == 0.   w: [K, K, C], x's dtype.
        bias: [C] or None.   residual: [N, P, Q, C] or None (x's dtype), with
        P = (H + 2*pad - K) // stride + 1 and Q likewise.
    """
    if w.dim() == 3 and pad is None:
        pad = int(w.shape[0]) // 2
    pads = None
    if isinstance(pad, (tuple, list)):
        if len(pad) != 4:
            raise ValueError(f"pad must be an int or (top, bottom, left, right), got {pad!r}")
        pads = tuple(int(v) for v in pad)
        pad = min(pads)
    _check(x, w, pad, bf16_ok=True)
    K = int(w.shape[0])
    if K not in (3, 5, 7) or w.shape[1] != K:
        raise ValueError(f"w must be [K,K,C] with K in {{3, 5, 7}}, got shape {tuple(w.shape)}")
    if stride not in (1, 2):
        raise ValueError(f"stride must be 1 or 2, got {stride}")
    if x.shape[3] % 8 != 0:
        raise ValueError("dwconv requires C % 8 == 0")
    if n_stage is not None and n_stage not in (2, 3, 4):
        raise ValueError(f"n_stage must be one of {{2, 3, 4}}, got {n_stage}")
    if activation not in ACTIVATIONS:
        raise ValueError(f"activation must be one of {sorted(ACTIVATIONS)}, got {activation!r}")
    ns = 0 if n_stage is None else int(n_stage)
    if int(dilation) < 1:
        raise ValueError(f"dilation must be >= 1, got {dilation}")
    if int(dilation) > 1 or (pads is not None and not (pads[0] == pads[1] == pads[2] == pads[3])):
        pads = pads if pads is not None else (int(pad),) * 4
        return _C.dwconv_k_pads(x, w, bias, residual, int(stride), int(dilation), *pads,
                                ACTIVATIONS[activation], ns)
    return _C.dwconv_k(x, w, bias, residual, int(stride), int(pad), ACTIVATIONS[activation], ns)


def dwconv_plain(x: torch.Tensor, w: torch.Tensor, pad: int | None = None, stride: int = 1,
                 bias: torch.Tensor | None = None, residual: torch.Tensor | None = None,
                 activation: str = "none", band_rows: int = 0) -> torch.Tensor:
    """``dwconv`` on the plain kernel: global loads through L1, no TMA, no
    shared memory.  A thread owns one channel pair of one output column over
    ``band_rows`` output rows (0: chosen from the shape).  Same arguments
    (``band_rows`` for ``n_stage``) and the same result, bit for bit."""
    if w.dim() == 3 and pad is None:
        pad = int(w.shape[0]) // 2
    _check(x, w, pad, bf16_ok=True)
    K = int(w.shape[0])
    if K not in (3, 5, 7) or w.shape[1] != K:
        raise ValueError(f"w must be [K,K,C] with K in {{3, 5, 7}}, got shape {tuple(w.shape)}")
    if stride not in (1, 2):
        raise ValueError(f"stride must be 1 or 2, got {stride}")
    if x.shape[3] % 8 != 0:
        raise ValueError("dwconv_plain requires C % 8 == 0")
    if band_rows < 0:
        raise ValueError(f"band_rows must be non-negative, got {band_rows}")
    if activation not in ACTIVATIONS:
        raise ValueError(f"activation must be one of {sorted(ACTIVATIONS)}, got {activation!r}")
    return _C.dwconv_plain(x, w, bias, residual, int(stride), int(pad), ACTIVATIONS[activation],
                           int(band_rows))


def uses_plain(N: int, H: int, W: int, C: int, K: int = 3, stride: int = 1,
               pad: int | None = None) -> bool:
    """Whether ``dwconv`` with ``n_stage=None`` runs the plain kernel on this shape."""
    return bool(_C.dwconv_uses_plain(int(N), int(H), int(W), int(C), int(K), int(stride),
                                     int(K // 2 if pad is None else pad)))


def device_status(device: int | None = None, clear: bool = True):
    """First pipeline-wait failure recorded on ``device`` as (code, block, stage, load).

    code 0 means none; 1 = a consumer gave up waiting for a filled stage,
    2 = the producer gave up waiting for a free stage, 3 = an issued copy never
    completed.  Synchronises the device.
    """
    if device is None:
        device = torch.cuda.current_device()
    return _C.device_status(int(device), bool(clear))


def set_wait_timeout_ns(ns: int) -> None:
    """Limit of every pipeline wait in later ws launches (default 2 s)."""
    _C.set_wait_timeout_ns(int(ns))
