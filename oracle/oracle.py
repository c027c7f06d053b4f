"""CPU oracle for the NHWC fp16 depthwise 3x3 conv2d forward.

TEST INFRASTRUCTURE ONLY: the parity tests, ``__graft_entry__.smoke()`` and the
CPU-baseline leg of ``bench.py`` use this module as the checker.  The shipped
library never imports it, and the product path has no CPU fallback.

Two independent restatements of the reference arithmetic
(haowen-han/tma-depthwise-conv ``csrc/kernel_v0_naive_float4.cu:37-74`` and
``csrc/kernel_tma_ws.cuh:218-246``: fp32 multiply-add chain from +0 in
r-major, s-minor order over the 3x3 taps, zero outside the image, one
round-to-nearest-even to fp16):

* :func:`dwconv_f16` calls the C restatement in ``dwconv_oracle.c``
  (``liboracle_dwconv.so``, OpenMP) — the fast one, used at every size;
* :func:`dwconv_f16_numpy` is a numpy restatement for small cases.

The two must agree bit for bit; tests/test_oracle.py checks that, and checks
both against the golden vectors recorded from the reference's own kernels.
"""
from __future__ import annotations

import ctypes
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(_HERE, "liboracle_dwconv.so")
_lib = None


def load() -> ctypes.CDLL:
    """Load liboracle_dwconv.so (built by ``make -C oracle``); raise if absent."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise RuntimeError(f"oracle library missing: {LIB_PATH} (run `make -C oracle`)")
        lib = ctypes.CDLL(LIB_PATH)
        i64 = ctypes.c_int64
        lib.oracle_dwconv3x3_f16.argtypes = [ctypes.c_void_p] * 3 + [i64] * 5 + [ctypes.c_int]
        lib.oracle_dwconv3x3_f16.restype = ctypes.c_int
        lib.oracle_dwconv3x3_ex_f16.argtypes = ([ctypes.c_void_p] * 5 + [i64] * 5 +
                                                [ctypes.c_int, ctypes.c_int])
        lib.oracle_dwconv3x3_ex_f16.restype = ctypes.c_int
        lib.oracle_dwconv_ex_f16.argtypes = ([ctypes.c_void_p] * 5 + [i64] * 7 +
                                             [ctypes.c_int, ctypes.c_int])
        lib.oracle_dwconv_ex_f16.restype = ctypes.c_int
        lib.oracle_dwconv_bwd_data_f16.argtypes = [ctypes.c_void_p] * 3 + [i64] * 6 + [ctypes.c_int]
        lib.oracle_dwconv_bwd_data_f16.restype = ctypes.c_int
        lib.oracle_dwconv_bwd_data_s2_f16.argtypes = ([ctypes.c_void_p] * 3 + [i64] * 6 +
                                                     [ctypes.c_int])
        lib.oracle_dwconv_bwd_data_s2_f16.restype = ctypes.c_int
        for name in ("oracle_dwconv_bwd_data_bf16", "oracle_dwconv_bwd_data_s2_bf16"):
            getattr(lib, name).argtypes = [ctypes.c_void_p] * 3 + [i64] * 6 + [ctypes.c_int]
            getattr(lib, name).restype = ctypes.c_int
        lib.oracle_dwconv_ex_bf16.argtypes = ([ctypes.c_void_p] * 5 + [i64] * 7 +
                                              [ctypes.c_int, ctypes.c_int])
        lib.oracle_dwconv_ex_bf16.restype = ctypes.c_int
        lib.oracle_bf16_to_f32.argtypes = [ctypes.c_uint16]
        lib.oracle_bf16_to_f32.restype = ctypes.c_float
        lib.oracle_f32_to_bf16.argtypes = [ctypes.c_float]
        lib.oracle_f32_to_bf16.restype = ctypes.c_uint16
        lib.oracle_dwconv3x3_bwd_data_f16.argtypes = [ctypes.c_void_p] * 3 + [i64] * 5 + [ctypes.c_int]
        lib.oracle_dwconv3x3_bwd_data_f16.restype = ctypes.c_int
        lib.oracle_f16_to_f32.argtypes = [ctypes.c_uint16]
        lib.oracle_f16_to_f32.restype = ctypes.c_float
        lib.oracle_f32_to_f16.argtypes = [ctypes.c_float]
        lib.oracle_f32_to_f16.restype = ctypes.c_uint16
        lib.oracle_max_threads.restype = ctypes.c_int
        _lib = lib
    return _lib


def output_hw(H: int, W: int, pad: int) -> tuple[int, int]:
    """P, Q of a stride-1 3x3 conv (reference csrc/kernel_tma_ws.cu:384-385)."""
    return H + 2 * pad - 3 + 1, W + 2 * pad - 3 + 1


def max_threads() -> int:
    return int(load().oracle_max_threads())


def dwconv_f16(x: np.ndarray, w: np.ndarray, pad: int, threads: int = 0) -> np.ndarray:
    """C oracle.  x: [N,H,W,C] float16, w: [3,3,C] float16 -> [N,P,Q,C] float16."""
    lib = load()
    x = np.ascontiguousarray(x, dtype=np.float16)
    w = np.ascontiguousarray(w, dtype=np.float16)
    if x.ndim != 4 or w.shape != (3, 3, x.shape[3]):
        raise ValueError("x must be [N,H,W,C] and w [3,3,C]")
    N, H, W, C = x.shape
    P, Q = output_hw(H, W, pad)
    if P < 0 or Q < 0:
        raise ValueError("negative output size")
    y = np.empty((N, P, Q, C), dtype=np.float16)
    rc = lib.oracle_dwconv3x3_f16(x.ctypes.data, w.ctypes.data, y.ctypes.data,
                                  N, H, W, C, pad, int(threads))
    if rc != 0:
        raise RuntimeError("oracle_dwconv3x3_f16 failed")
    return y


ACTS = {"none": 0, "relu": 1, "relu6": 2, "silu": 3, "hardswish": 4}


def dwconv_ex_f16(x: np.ndarray, w: np.ndarray, pad: int, bias: np.ndarray | None = None,
                  residual: np.ndarray | None = None, activation: str = "none",
                  threads: int = 0) -> np.ndarray:
    """C oracle of the general forward with its fused epilogue (any C; see
    dwconv_oracle.c: t = acc + bias; t = act(t); t += residual; fp16 RNE)."""
    lib = load()
    x = np.ascontiguousarray(x, dtype=np.float16)
    w = np.ascontiguousarray(w, dtype=np.float16)
    N, H, W, C = x.shape
    P, Q = output_hw(H, W, pad)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float16)
    r = None if residual is None else np.ascontiguousarray(residual, dtype=np.float16)
    if b is not None and b.shape != (C,):
        raise ValueError("bias must be [C]")
    if r is not None and r.shape != (N, P, Q, C):
        raise ValueError("residual must be [N,P,Q,C]")
    y = np.empty((N, P, Q, C), dtype=np.float16)
    rc = lib.oracle_dwconv3x3_ex_f16(x.ctypes.data, w.ctypes.data,
                                     None if b is None else b.ctypes.data,
                                     None if r is None else r.ctypes.data, y.ctypes.data,
                                     N, H, W, C, pad, ACTS[activation], int(threads))
    if rc != 0:
        raise RuntimeError("oracle_dwconv3x3_ex_f16 failed")
    return y


def output_hw_k(H: int, W: int, K: int, stride: int, pad: int) -> tuple[int, int]:
    """P, Q of a K x K depthwise conv with a stride and symmetric padding."""
    return (H + 2 * pad - K) // stride + 1, (W + 2 * pad - K) // stride + 1


def dwconv_k_f16(x: np.ndarray, w: np.ndarray, pad: int, stride: int = 1,
                 bias: np.ndarray | None = None, residual: np.ndarray | None = None,
                 activation: str = "none", threads: int = 0) -> np.ndarray:
    """C oracle of the K x K, strided forward with the fused epilogue.
    x: [N,H,W,C] float16, w: [K,K,C] float16 -> [N,P,Q,C] float16."""
    lib = load()
    x = np.ascontiguousarray(x, dtype=np.float16)
    w = np.ascontiguousarray(w, dtype=np.float16)
    N, H, W, C = x.shape
    K = w.shape[0]
    if w.shape != (K, K, C):
        raise ValueError("w must be [K,K,C]")
    if H + 2 * pad < K or W + 2 * pad < K:
        raise ValueError("negative output size")
    P, Q = output_hw_k(H, W, K, stride, pad)
    b = None if bias is None else np.ascontiguousarray(bias, dtype=np.float16)
    r = None if residual is None else np.ascontiguousarray(residual, dtype=np.float16)
    if b is not None and b.shape != (C,):
        raise ValueError("bias must be [C]")
    if r is not None and r.shape != (N, P, Q, C):
        raise ValueError("residual must be [N,P,Q,C]")
    y = np.empty((N, P, Q, C), dtype=np.float16)
    rc = lib.oracle_dwconv_ex_f16(x.ctypes.data, w.ctypes.data,
                                  None if b is None else b.ctypes.data,
                                  None if r is None else r.ctypes.data, y.ctypes.data,
                                  N, H, W, C, K, stride, pad, ACTS[activation], int(threads))
    if rc != 0:
        raise RuntimeError("oracle_dwconv_ex_f16 failed")
    return y


def _bits(a: np.ndarray, shape=None) -> np.ndarray:
    a = np.ascontiguousarray(a)
    if a.dtype not in (np.uint16, np.int16):
        raise ValueError("bfloat16 data is passed as its 16-bit patterns (uint16 / int16)")
    a = a.view(np.uint16)
    if shape is not None and a.shape != shape:
        raise ValueError(f"expected shape {shape}, got {a.shape}")
    return a


def bf16_to_f32(bits: np.ndarray) -> np.ndarray:
    """bfloat16 bit patterns -> float32 values (exact)."""
    return (_bits(bits).astype(np.uint32) << 16).view(np.float32)


def dwconv_k_bf16(x: np.ndarray, w: np.ndarray, pad: int, stride: int = 1,
                  bias: np.ndarray | None = None, residual: np.ndarray | None = None,
                  activation: str = "none", threads: int = 0) -> np.ndarray:
    """C oracle of the K x K, strided forward with bfloat16 elements: the same
    fp32 chain and epilogue as :func:`dwconv_k_f16`, one round-to-nearest-even
    to bfloat16 (``oracle_dwconv_ex_bf16``).  x [N,H,W,C], w [K,K,C], bias
    [C], residual [N,P,Q,C] and the result are bfloat16 bit patterns
    (uint16)."""
    lib = load()
    x = _bits(x)
    N, H, W, C = x.shape
    w = _bits(w)
    K = w.shape[0]
    if w.shape != (K, K, C):
        raise ValueError("w must be [K,K,C]")
    if H + 2 * pad < K or W + 2 * pad < K:
        raise ValueError("negative output size")
    P, Q = output_hw_k(H, W, K, stride, pad)
    b = None if bias is None else _bits(bias, (C,))
    r = None if residual is None else _bits(residual, (N, P, Q, C))
    y = np.empty((N, P, Q, C), dtype=np.uint16)
    rc = lib.oracle_dwconv_ex_bf16(x.ctypes.data, w.ctypes.data,
                                   None if b is None else b.ctypes.data,
                                   None if r is None else r.ctypes.data, y.ctypes.data,
                                   N, H, W, C, K, stride, pad, ACTS[activation], int(threads))
    if rc != 0:
        raise RuntimeError("oracle_dwconv_ex_bf16 failed")
    return y


def dwconv_bwd_data_bf16(dy: np.ndarray, w: np.ndarray, pad: int, stride: int = 1,
                         H: int | None = None, W: int | None = None,
                         threads: int = 0) -> np.ndarray:
    """C oracle of the data gradient with bfloat16 elements (bit patterns in
    and out): stride 1 is the flipped-tap chain of :func:`dwconv_bwd_data_f16`,
    stride 2 the transposed stencil of :func:`dwconv_bwd_data_s2_f16` (H, W
    required there)."""
    lib = load()
    dy = _bits(dy)
    w = _bits(w)
    N, P, Q, C = dy.shape
    K = w.shape[0]
    if stride == 1:
        H, W = P - 2 * pad + K - 1, Q - 2 * pad + K - 1
        fn = lib.oracle_dwconv_bwd_data_bf16
    else:
        if H is None or W is None:
            raise ValueError("the stride-2 data gradient needs the input H and W")
        if ((H + 2 * pad - K) // 2 + 1, (W + 2 * pad - K) // 2 + 1) != (P, Q):
            raise ValueError("dy does not match a stride-2 forward of an H x W input")
        fn = lib.oracle_dwconv_bwd_data_s2_bf16
    dx = np.empty((N, H, W, C), dtype=np.uint16)
    if fn(dy.ctypes.data, w.ctypes.data, dx.ctypes.data, N, H, W, C, K, pad, int(threads)) != 0:
        raise RuntimeError("oracle bf16 data gradient failed")
    return dx


def dwconv_k_f16_numpy(x: np.ndarray, w: np.ndarray, pad: int, stride: int = 1) -> np.ndarray:
    """numpy restatement of the K x K, strided forward (small sizes): the same
    chain in (r, s) order from +0, products exact in float32, one RNE."""
    x = np.asarray(x, dtype=np.float16)
    w = np.asarray(w, dtype=np.float16)
    N, H, W, C = x.shape
    K = w.shape[0]
    P, Q = output_hw_k(H, W, K, stride, pad)
    xp = np.zeros((N, H + 2 * pad + stride, W + 2 * pad + stride, C), dtype=np.float32)
    xp[:, pad:pad + H, pad:pad + W, :] = x.astype(np.float32)
    wf = w.astype(np.float32)
    acc = np.zeros((N, P, Q, C), dtype=np.float32)
    for r in range(K):
        for s in range(K):
            acc = acc + xp[:, r:r + stride * P:stride, s:s + stride * Q:stride, :] * wf[r, s]
    return acc.astype(np.float16)


def dwconv_dilated_f16_numpy(x: np.ndarray, w: np.ndarray, pads, stride: int = 1,
                             dilation: int = 1) -> np.ndarray:
    """numpy restatement of the dilated forward with per-side padding (small
    sizes), written directly rather than through a zero-inflated kernel:
    y[n,p,q,c] = fp16_rne(chain_{r,s} x[n, S*p + D*r - top, S*q + D*s - left, c]
    * w[r,s,c]) from +0 in (r, s) order, products exact in float32, with
    pads = (top, bottom, left, right) and P = (H + top + bottom - D*(K-1) - 1)
    // S + 1 (the formula of tdc_dwconv_fwd_dilated)."""
    x = np.asarray(x, dtype=np.float16)
    w = np.asarray(w, dtype=np.float16)
    N, H, W, C = x.shape
    K = w.shape[0]
    top, bottom, left, right = (int(v) for v in pads)
    S, D = int(stride), int(dilation)
    Ke = D * (K - 1) + 1
    P = (H + top + bottom - Ke) // S + 1
    Q = (W + left + right - Ke) // S + 1
    xp = np.zeros((N, H + top + bottom + S, W + left + right + S, C), dtype=np.float32)
    xp[:, top:top + H, left:left + W, :] = x.astype(np.float32)
    wf = w.astype(np.float32)
    acc = np.zeros((N, P, Q, C), dtype=np.float32)
    for r in range(K):
        for s in range(K):
            acc = acc + xp[:, D * r:D * r + S * P:S, D * s:D * s + S * Q:S, :] * wf[r, s]
    return acc.astype(np.float16)


def dwconv_ex_f16_numpy(x, w, pad, bias=None, residual=None, activation="none"):
    """numpy restatement of the general forward (small sizes)."""
    N, H, W, C = x.shape
    P, Q = output_hw(H, W, pad)
    xp = np.zeros((N, H + 2 * pad, W + 2 * pad, C), dtype=np.float32)
    xp[:, pad:pad + H, pad:pad + W, :] = np.asarray(x, np.float16).astype(np.float32)
    wf = np.asarray(w, np.float16).astype(np.float32)
    t = np.zeros((N, P, Q, C), dtype=np.float32)
    for rr in range(3):
        for ss in range(3):
            t = t + xp[:, rr:rr + P, ss:ss + Q, :] * wf[rr, ss]
    if bias is not None:
        t = t + np.asarray(bias, np.float16).astype(np.float32)
    if activation == "relu":
        t = np.where(t < 0, np.float32(0), t)
    elif activation == "relu6":
        t = np.where(t < 0, np.float32(0), np.where(t > 6, np.float32(6), t))
    elif activation == "silu":
        with np.errstate(over="ignore"):
            t = (t / (np.float32(1) + np.exp(-t))).astype(np.float32)
    elif activation == "hardswish":
        h = np.clip(t + np.float32(3), np.float32(0), np.float32(6)).astype(np.float32)
        t = ((t * h).astype(np.float32) / np.float32(6)).astype(np.float32)
    if residual is not None:
        t = t + np.asarray(residual, np.float16).astype(np.float32)
    return t.astype(np.float16)


def dwconv_f16_numpy(x: np.ndarray, w: np.ndarray, pad: int) -> np.ndarray:
    """numpy restatement (small sizes).  Same chain, same order, same rounding.

    numpy float32 ``acc + xs * ws`` rounds the product first, but the product
    of two fp16 values is exact in float32, so each step equals fmaf.
    """
    x = np.asarray(x, dtype=np.float16)
    w = np.asarray(w, dtype=np.float16)
    N, H, W, C = x.shape
    P, Q = output_hw(H, W, pad)
    xp = np.zeros((N, H + 2 * pad, W + 2 * pad, C), dtype=np.float32)
    xp[:, pad:pad + H, pad:pad + W, :] = x.astype(np.float32)
    wf = w.astype(np.float32)
    acc = np.zeros((N, P, Q, C), dtype=np.float32)
    for r in range(3):
        for s in range(3):
            acc = acc + xp[:, r:r + P, s:s + Q, :] * wf[r, s]
    return acc.astype(np.float16)  # numpy float32 -> float16 is round-to-nearest-even


def dwconv_bwd_data_f16(dy: np.ndarray, w: np.ndarray, pad: int, threads: int = 0) -> np.ndarray:
    """C oracle of the data gradient of the stride-1 forward: dx [N,H,W,C] fp16
    from dy [N,P,Q,C] and w [K,K,C] (taps flipped, fp32 chain in the kernel's
    order, fp16 RNE).  K = 3 runs the 3x3 restatement, other K the K x K one."""
    lib = load()
    dy = np.ascontiguousarray(dy, dtype=np.float16)
    w = np.ascontiguousarray(w, dtype=np.float16)
    N, P, Q, C = dy.shape
    K = w.shape[0]
    H, W = P - 2 * pad + K - 1, Q - 2 * pad + K - 1
    dx = np.empty((N, H, W, C), dtype=np.float16)
    if K == 3:
        rc = lib.oracle_dwconv3x3_bwd_data_f16(dy.ctypes.data, w.ctypes.data, dx.ctypes.data,
                                               N, H, W, C, pad, int(threads))
    else:
        rc = lib.oracle_dwconv_bwd_data_f16(dy.ctypes.data, w.ctypes.data, dx.ctypes.data,
                                            N, H, W, C, K, pad, int(threads))
    if rc != 0:
        raise RuntimeError("oracle data gradient failed")
    return dx


def dwconv_bwd_data_s2_f16(dy: np.ndarray, w: np.ndarray, pad: int, H: int, W: int,
                           threads: int = 0) -> np.ndarray:
    """C oracle of the data gradient of the stride-2 forward: dx [N,H,W,C] fp16
    from dy [N,P,Q,C], P = (H + 2*pad - K)//2 + 1, and w [K,K,C]: per output,
    the fp32 chain over the taps with h + pad - r and v + pad - s even, r then
    s descending, one fp16 rounding (``oracle_dwconv_bwd_data_s2_f16``)."""
    lib = load()
    dy = np.ascontiguousarray(dy, dtype=np.float16)
    w = np.ascontiguousarray(w, dtype=np.float16)
    N, P, Q, C = dy.shape
    K = w.shape[0]
    if ((H + 2 * pad - K) // 2 + 1, (W + 2 * pad - K) // 2 + 1) != (P, Q):
        raise ValueError("dy does not match a stride-2 forward of an H x W input")
    dx = np.empty((N, H, W, C), dtype=np.float16)
    rc = lib.oracle_dwconv_bwd_data_s2_f16(dy.ctypes.data, w.ctypes.data, dx.ctypes.data,
                                           N, H, W, C, K, pad, int(threads))
    if rc != 0:
        raise RuntimeError("oracle stride-2 data gradient failed")
    return dx


def dwconv_bwd_data_s2_numpy(dy: np.ndarray, w: np.ndarray, pad: int, H: int,
                             W: int) -> np.ndarray:
    """Numpy restatement of :func:`dwconv_bwd_data_s2_f16` for small cases: a
    scatter of every tap's product into the zero-upsampled, padded dx grid,
    taps visited r then s descending so each output sees its chain in the
    same order (products of fp16 values are exact in float32)."""
    dy = np.asarray(dy, np.float16).astype(np.float32)
    wf = np.asarray(w, np.float16).astype(np.float32)
    N, P, Q, C = dy.shape
    K = wf.shape[0]
    # acc over the padded grid [H + 2*pad (+ slack)]; dx[h] = grid[h + pad]
    Hg = max(H + 2 * pad, 2 * (P - 1) + K) + 2
    Wg = max(W + 2 * pad, 2 * (Q - 1) + K) + 2
    acc = np.zeros((N, Hg, Wg, C), np.float32)
    for r in range(K - 1, -1, -1):
        for s in range(K - 1, -1, -1):
            acc[:, r:r + 2 * P:2, s:s + 2 * Q:2] += dy * wf[r, s]
    # Grid cells no tap reaches hold +0; every reached cell saw its taps in the
    # oracle's order, except that out-of-range dy (zero products) are not
    # added, which leaves finite sums unchanged.
    return acc[:, pad:pad + H, pad:pad + W].astype(np.float16)


def dwconv_bwd_weight_f64(x: np.ndarray, dy: np.ndarray, pad: int, K: int = 3,
                          stride: int = 1) -> np.ndarray:
    """Weight gradient of the K x K forward in float64 (the accuracy reference
    for the fp32 kernels):
    dw[r,s,c] = sum_{n,p,q} x[n, stride*p+r-pad, stride*q+s-pad, c] * dy[n,p,q,c]."""
    x = np.asarray(x, np.float16).astype(np.float64)
    dy = np.asarray(dy, np.float16).astype(np.float64)
    N, H, W, C = x.shape
    P, Q = dy.shape[1], dy.shape[2]
    S = stride
    xp = np.zeros((N, max(H + 2 * pad, S * (P - 1) + K), max(W + 2 * pad, S * (Q - 1) + K), C))
    xp[:, pad:pad + H, pad:pad + W] = x
    dw = np.empty((K, K, C))
    for r in range(K):
        for s in range(K):
            dw[r, s] = np.einsum("npqc,npqc->c",
                                 xp[:, r:r + S * (P - 1) + 1:S, s:s + S * (Q - 1) + 1:S], dy)
    return dw


def f16_ulp(v: np.ndarray) -> np.ndarray:
    """fp16 spacing at |v| (2^-24 in the subnormal range)."""
    a = np.abs(np.asarray(v, dtype=np.float32))
    e = np.floor(np.log2(np.maximum(a, 2.0 ** -14)))
    return np.exp2(e - 10).astype(np.float32)


def silu_tolerance(want: np.ndarray, residual: np.ndarray | None = None) -> np.ndarray:
    """Bound on |kernel - oracle| for the fused silu epilogue.

    The kernel's silu (fast exp and divide) is within a few fp32 ulp of the
    oracle's expf-based one: a relative error of at most 2^-20 of the silu
    term t, which can flip the final fp16 rounding by one ulp of the result.
    When a residual r is added, |t| <= |y| + |r| can be much larger than the
    result (cancellation), so the bound is one fp16 ulp of y plus
    2^-20 * (|y| + |r|).
    """
    y = np.abs(np.asarray(want, dtype=np.float32))
    r = 0.0 if residual is None else np.abs(np.asarray(residual, dtype=np.float32))
    return f16_ulp(y) + np.float32(2.0 ** -20) * (y + r)
