"""C ABI of libtdc_sm100.so, checked without a GPU.

* the library loads and exports every function include/tdc_dwconv.h declares;
* argument errors come back as the documented status codes before any CUDA
  call (the same conditions the reference's TORCH_CHECKs reject,
  csrc/kernel_tma_ws.cu:54-65 / csrc/kernel_v0_naive_float4.cu:84-94);
* the ws launch planner covers every output element exactly once.
"""
import ctypes as C
import os
import re

import numpy as np
import pytest
import torch

REPO = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
LIB = os.path.join(REPO, "tma-depthwise-conv_b200", "libtdc_sm100.so")
HDR = os.path.join(REPO, "include", "tdc_dwconv.h")

i64 = C.c_int64


def _codes():
    txt = open(HDR).read()
    return {m.group(1): int(m.group(2)) for m in re.finditer(r"#define (TDC_\w+)\s+(-?\d+)", txt)}


CODES = _codes()


@pytest.fixture(scope="module")
def lib():
    L = C.CDLL(LIB)
    L.tdc_strerror.restype = C.c_char_p
    return L


def test_exports_every_declared_symbol(lib):
    names = re.findall(r"TDC_API\s+[\w\s\*]+?\b(tdc_\w+)\s*\(", open(HDR).read())
    assert len(names) >= 12
    for n in names:
        assert hasattr(lib, n), f"{n} declared in tdc_dwconv.h but not exported"


def test_strerror_covers_all_codes(lib):
    for name, code in CODES.items():
        if name.startswith("TDC_ERR_") or name == "TDC_OK":
            s = lib.tdc_strerror(code)
            assert s and b"unknown" not in s, name
    assert b"unknown" in lib.tdc_strerror(-999)


def test_output_hw(lib):
    P, Q = i64(), i64()
    assert lib.tdc_output_hw(i64(224), i64(336), i64(3), i64(3), i64(1), C.byref(P), C.byref(Q)) == 0
    assert (P.value, Q.value) == (224, 336)
    assert lib.tdc_output_hw(i64(16), i64(16), i64(3), i64(3), i64(0), C.byref(P), C.byref(Q)) == 0
    assert (P.value, Q.value) == (14, 14)
    assert lib.tdc_output_hw(i64(16), i64(16), i64(3), i64(3), i64(-1), C.byref(P), C.byref(Q)) == CODES["TDC_ERR_PAD"]


def _ws(lib, x=16, w=16, y=16, N=2, H=16, W=16, Cc=64, R=3, S=3, pad=1, ns=2):
    p = lambda v: C.c_void_p(v) if v else None
    return lib.tdc_dwconv_ws(p(x), p(w), p(y), i64(N), i64(H), i64(W), i64(Cc), i64(R), i64(S),
                             i64(pad), i64(ns), None)


def _v0(lib, x=16, w=16, y=16, N=2, H=16, W=16, Cc=64, R=3, S=3, pad=1):
    p = lambda v: C.c_void_p(v) if v else None
    return lib.tdc_dwconv_v0(p(x), p(w), p(y), i64(N), i64(H), i64(W), i64(Cc), i64(R), i64(S),
                             i64(pad), None)


def test_ws_argument_errors(lib):
    assert _ws(lib, x=0) == CODES["TDC_ERR_NULL_POINTER"]
    assert _ws(lib, y=0) == CODES["TDC_ERR_NULL_POINTER"]
    assert _ws(lib, H=0) == CODES["TDC_ERR_BAD_SHAPE"]
    assert _ws(lib, N=-1) == CODES["TDC_ERR_BAD_SHAPE"]
    assert _ws(lib, R=5, S=5) == CODES["TDC_ERR_FILTER_SHAPE"]
    assert _ws(lib, Cc=32) == CODES["TDC_ERR_CHANNELS"]
    assert _ws(lib, pad=-1) == CODES["TDC_ERR_PAD"]
    assert _ws(lib, ns=5) == CODES["TDC_ERR_N_STAGE"]
    assert _ws(lib, ns=1) == CODES["TDC_ERR_N_STAGE"]
    assert _ws(lib, x=24) == CODES["TDC_ERR_ALIGNMENT"]
    assert _ws(lib, H=1, W=1, pad=0) == CODES["TDC_ERR_BAD_SHAPE"]      # P = -1
    assert _ws(lib, N=1, H=1 << 20, W=1 << 20, Cc=1 << 10) == CODES["TDC_ERR_TOO_LARGE"]
    # empty outputs are a successful no-op, before any device query
    assert _ws(lib, N=0) == 0
    assert _ws(lib, H=2, W=2, pad=0) == 0                               # P = Q = 0


def test_v0_argument_errors(lib):
    assert _v0(lib, w=0) == CODES["TDC_ERR_NULL_POINTER"]
    assert _v0(lib, Cc=12) == CODES["TDC_ERR_CHANNELS"]
    assert _v0(lib, R=1, S=1) == CODES["TDC_ERR_FILTER_SHAPE"]
    assert _v0(lib, y=8) == CODES["TDC_ERR_ALIGNMENT"]
    assert _v0(lib, N=0) == 0


@pytest.mark.skipif(torch.cuda.is_available(), reason="checks the no-device path")
def test_valid_call_without_device_reports_no_device(lib):
    assert _ws(lib) == CODES["TDC_ERR_NO_DEVICE"]
    assert _v0(lib) == CODES["TDC_ERR_NO_DEVICE"]
    nb = i64()
    assert lib.tdc_ws_probe_blocks(i64(2), i64(16), i64(16), i64(64), i64(1), i64(2), C.byref(nb)) == CODES["TDC_ERR_NO_DEVICE"]


def test_general_forward_argument_errors(lib):
    p = C.c_void_p
    def fwd(C_=72, act=0, bias=None, res=None, x=16, ns=2):
        return lib.tdc_dwconv3x3_fwd(p(x), p(16), bias, res, p(16), i64(2), i64(16), i64(16),
                                     i64(C_), i64(1), i64(act), i64(ns), None)
    assert fwd(act=5) == CODES["TDC_ERR_ACT"]
    assert fwd(act=-1) == CODES["TDC_ERR_ACT"]
    assert fwd(C_=12) == CODES["TDC_ERR_CHANNELS"]
    assert fwd(ns=5) == CODES["TDC_ERR_N_STAGE"]
    assert fwd(bias=p(20)) == CODES["TDC_ERR_ALIGNMENT"]
    assert fwd(res=p(24)) == CODES["TDC_ERR_ALIGNMENT"]
    if not torch.cuda.is_available():
        assert fwd() == CODES["TDC_ERR_NO_DEVICE"]


def test_kxk_forward_argument_errors(lib):
    p = C.c_void_p
    def fwd(K=5, stride=2, C_=72, pad=2, H=16, act=0, ns=2, N=2, x=16):
        return lib.tdc_dwconv_fwd(p(x), p(16), None, None, p(16), i64(N), i64(H), i64(16),
                                  i64(C_), i64(K), i64(stride), i64(pad), i64(act), i64(ns), None)
    assert fwd(K=4) == CODES["TDC_ERR_FILTER_SHAPE"]
    assert fwd(K=9) == CODES["TDC_ERR_FILTER_SHAPE"]
    assert fwd(stride=3) == CODES["TDC_ERR_STRIDE"]
    assert fwd(stride=0) == CODES["TDC_ERR_STRIDE"]
    assert fwd(C_=12) == CODES["TDC_ERR_CHANNELS"]
    assert fwd(pad=-1) == CODES["TDC_ERR_PAD"]
    assert fwd(ns=1) == CODES["TDC_ERR_N_STAGE"]
    assert fwd(act=7) == CODES["TDC_ERR_ACT"]
    assert fwd(K=7, H=2, pad=2) == CODES["TDC_ERR_BAD_SHAPE"]  # 2 + 4 < 7: no output row
    assert fwd(x=24) == CODES["TDC_ERR_ALIGNMENT"]
    assert fwd(N=0) == CODES["TDC_OK"]  # empty: nothing to launch
    if not torch.cuda.is_available():
        assert fwd() == CODES["TDC_ERR_NO_DEVICE"]
        assert fwd(K=3, stride=1, pad=1) == CODES["TDC_ERR_NO_DEVICE"]


def test_probe_and_status_argument_errors(lib):
    p = C.c_void_p(16)
    assert lib.tdc_dwconv_ws_probe(p, p, p, i64(2), i64(16), i64(16), i64(64), i64(3), i64(3),
                                   i64(1), i64(2), None, None) == CODES["TDC_ERR_NULL_POINTER"]
    assert lib.tdc_ws_probe_blocks(i64(2), i64(16), i64(16), i64(64), i64(1), i64(2), None) == CODES["TDC_ERR_NULL_POINTER"]
    assert lib.tdc_set_wait_timeout_ns(i64(0)) != 0
    assert lib.tdc_ws_consumer_warps() == 4


PLAN_KEYS = ["stage_rows", "qstrips", "cblocks", "strips", "full_units", "tail_band_rows", "grid", "smem",
             "tail_chunk_rows"]


def _plan(lib, N, H, W, Cc, pad, ns, sms=148, occ=4):
    out = (i64 * 9)()
    rc = lib.tdc_ws_plan(i64(N), i64(H), i64(W), i64(Cc), i64(pad), i64(ns), i64(sms), i64(occ), out)
    assert rc == 0
    return dict(zip(PLAN_KEYS, list(out)))


def segments(pl, P, g):
    """(strip, first row, end row) of every segment CTA g processes, restating
    the kernel's SegmentIter: whole strips round-robin, then the remaining
    strips in bands, band-major, round-robin; or, with tail_chunk_rows = L,
    channel block g % cblocks of rows [k*L, (k+1)*L) (k = g // cblocks) of
    the tail's pixel strips' rows taken one pixel strip after the other."""
    out = []
    tail = pl["strips"] - pl["full_units"]
    hb = pl["tail_band_rows"]
    bands = -(-P // hb)
    L = pl.get("tail_chunk_rows", 0)
    k = g
    while k < pl["full_units"]:
        out.append((k, 0, P))
        k += pl["grid"]
    if L > 0:
        cb = pl["cblocks"]
        assert pl["grid"] % cb == 0 and tail % cb == 0
        total = tail // cb * P
        row = min(g // cb * L, total)
        end = min(row + L, total)
        while row < end:
            ps, first = divmod(row, P)
            last = min(P, first + end - row)
            out.append((pl["full_units"] + ps * cb + g % cb, first, last))
            row += last - first
        return out
    while True:
        t = k - pl["full_units"]
        if t >= tail * bands:
            break
        band = t // tail
        out.append((pl["full_units"] + t % tail, band * hb, min(P, band * hb + hb)))
        k += pl["grid"]
    return out


SHAPES = [(64, 224, 336, 256, 1), (32, 224, 336, 256, 1), (16, 112, 224, 128, 1), (8, 56, 56, 256, 1),
          (2, 16, 16, 64, 1), (1, 1, 1, 64, 1), (1, 3, 3, 64, 5), (3, 7, 45, 128, 1), (5, 100, 1, 64, 1),
          (1, 1000, 40, 64, 0), (80, 224, 336, 320, 1), (8, 224, 336, 256, 1), (2, 19, 45, 72, 1),
          (3, 9, 9, 8, 0)]


@pytest.mark.parametrize("N,H,W,Cc,pad", SHAPES)
@pytest.mark.parametrize("ns", [2, 3, 4])
def test_plan_covers_every_output_once(lib, N, H, W, Cc, pad, ns):
    pl = _plan(lib, N, H, W, Cc, pad, ns)
    P, Q = H + 2 * pad - 2, W + 2 * pad - 2
    assert pl["stage_rows"] >= 1
    assert pl["cblocks"] == -(-Cc // 64) and pl["qstrips"] == -(-Q // 32)
    assert pl["strips"] == N * pl["qstrips"] * pl["cblocks"]
    assert pl["full_units"] % pl["grid"] == 0 and 0 <= pl["full_units"] < pl["strips"]
    assert pl["strips"] - pl["full_units"] <= pl["grid"]
    assert 1 <= pl["tail_band_rows"] <= P
    assert 1 <= pl["grid"] <= 148 * 4
    assert pl["smem"] == ns * pl["stage_rows"] * 34 * 128 + 128 <= 227 * 1024
    cols = [q for s in range(pl["qstrips"]) for q in range(s * 32, min(s * 32 + 32, Q))]
    assert cols == list(range(Q))
    seen = set()
    for g in range(pl["grid"]):
        for strip, a, b in segments(pl, P, g):
            assert 0 <= a < b <= P
            for r in range(a, b):
                assert (strip, r) not in seen
                seen.add((strip, r))
    assert len(seen) == pl["strips"] * P


def _fwd_plan(lib, N, H, W, Cc, K, S, pad, ns, sms=148, occ=3):
    out = (i64 * 9)()
    rc = lib.tdc_dwconv_fwd_plan(i64(N), i64(H), i64(W), i64(Cc), i64(K), i64(S), i64(pad), i64(ns),
                                 i64(sms), i64(occ), out)
    assert rc == 0
    return dict(zip(PLAN_KEYS, list(out)))


def direct_scheme(K, S):
    """Restates tdc::direct_scheme: taps + accumulator sets + one input row of
    registers above 100 -> one output row at a time from its K input rows."""
    nacc = -(-K // S)
    return K * K + nacc * 16 + (S * 7 + K) > 100


def direct_rows(K, S):
    """Restates direct_rows(K, S): output rows per pass of the direct scheme."""
    return 1 if S == 2 else (3 if K <= 5 else 2)


def max_stages_held(rows, K, S, sr, R=1):
    """Restates the direct scheme's consumer bookkeeping over one segment of
    `rows` output rows, R per pass: the most ring stages a warp holds at once."""
    rows_in = S * (rows - 1) + K
    nst = -(-rows_in // sr)
    acquired = released = 0
    worst = 0
    for o in range(0, rows, R):
        nout = min(R, rows - o)
        acquired = max(acquired, min(nst, (S * (o + nout - 1) + K - 1) // sr + 1))
        worst = max(worst, acquired - released)
        released = nst if o + R >= rows else min(nst, S * (o + R) // sr)
        assert released <= acquired
    assert acquired == released == nst
    return worst


@pytest.mark.parametrize("K,S", [(3, 2), (5, 1), (5, 2), (7, 1), (7, 2)])
@pytest.mark.parametrize("N,H,W,Cc,pad", [(64, 224, 336, 256, None), (2, 19, 45, 72, 0), (3, 7, 9, 8, None),
                                          (1, 300, 40, 64, 4), (6, 96, 200, 256, None)])
@pytest.mark.parametrize("ns", [2, 3, 4])
def test_kxk_plan_covers_every_output_once(lib, K, S, N, H, W, Cc, pad, ns):
    pad = K // 2 if pad is None else pad
    pl = _fwd_plan(lib, N, H, W, Cc, K, S, pad, ns)
    P, Q = (H + 2 * pad - K) // S + 1, (W + 2 * pad - K) // S + 1
    sr = pl["stage_rows"]
    assert 1 <= sr <= 256 and S * 31 + K <= 256  # TMA box extents
    assert pl["smem"] == ns * sr * (S * 31 + K) * 128 + 128 <= 200 * 1024
    assert pl["qstrips"] == -(-Q // 32) and pl["cblocks"] == -(-Cc // 64)
    if direct_scheme(K, S):
        assert (ns - 1) * sr >= S * (direct_rows(K, S) - 1) + K - 1
    seen = set()
    for g in range(pl["grid"]):
        for strip, a, b in segments(pl, P, g):
            assert 0 <= a < b <= P
            if direct_scheme(K, S):
                assert max_stages_held(b - a, K, S, sr, direct_rows(K, S)) <= ns
            for r in range(a, b):
                assert (strip, r) not in seen
                seen.add((strip, r))
    assert len(seen) == pl["strips"] * P


@pytest.mark.parametrize("K,S,D", [(3, 1, 2), (3, 1, 3), (5, 1, 2), (3, 2, 2), (7, 2, 3), (7, 1, 4)])
@pytest.mark.parametrize("N,P,Q,Cc", [(2, 41, 70, 64), (1, 29, 37, 200), (12, 96, 160, 256), (3, 7, 5, 8),
                                      (2, 2, 3, 64), (1, 1, 1, 8)])
def test_dilated_ring_segments_cover_every_output_once(lib, K, S, D, N, P, Q, Cc):
    """The ring kernel's dilated schedule: the plan of the N*D*D phase
    sub-problems of the largest phase's ceil(P/D) x ceil(Q/D) outputs; a
    segment of image n' is phase (a, b) = divmod(n' % D^2, D) of image
    n' // D^2, its rows clipped to that phase's ceil((P - a)/D), its columns
    to ceil((Q - b)/D); phase output (p', q') is y's (a + D*p', b + D*q').
    Every output of y, per channel block, is written exactly once."""
    Pp, Qp = -(-P // D), -(-Q // D)
    H, W = S * (Pp - 1) + K, S * (Qp - 1) + K  # at pad 0 the sub-problem has Pp x Qp outputs
    ns = 2 if (K, S) == (3, 1) else 4
    pl = _fwd_plan(lib, N * D * D, H, W, Cc, K, S, 0, ns)
    seen = np.zeros((N, P, Q, pl["cblocks"]), dtype=np.int32)
    for g in range(pl["grid"]):
        for strip, a, b in segments(pl, Pp, g):
            cb = strip % pl["cblocks"]
            qs = strip // pl["cblocks"] % pl["qstrips"]
            nn = strip // pl["cblocks"] // pl["qstrips"]
            n, ph = divmod(nn, D * D)
            pa, pb = divmod(ph, D)
            last = min(b, -(-(P - pa) // D))
            qn = -(-(Q - pb) // D)
            if last <= a:
                continue  # a segment of a smaller phase left empty: skipped
            for r in range(a, last):
                for q in range(qs * 32, min(qs * 32 + 32, qn)):
                    seen[n, pa + D * r, pb + D * q, cb] += 1
    assert (seen == 1).all()


def test_dilated_kernel_choice(lib):
    """tdc_dwconv_fwd_dilated_uses_plain: the ring kernel for phases of at
    least 32 x 32 outputs that the undilated choice gives it, while its map
    can step D; the plain kernel otherwise."""
    def plain(N, H, W, Cc, K, S, D):
        pad = D * (K - 1) // 2
        return lib.tdc_dwconv_fwd_dilated_uses_plain(i64(N), i64(H), i64(W), i64(Cc), i64(K), i64(S),
                                                     i64(D), i64(pad), i64(pad), i64(pad), i64(pad))
    assert plain(32, 128, 128, 256, 3, 1, 2) == 0
    assert plain(16, 128, 128, 256, 3, 1, 4) == 0
    assert plain(16, 112, 112, 384, 5, 1, 2) == 0
    assert plain(8, 64, 64, 256, 3, 1, 2) == 0
    assert plain(8, 64, 64, 256, 3, 1, 4) == 1     # 16 x 16 phases
    assert plain(8, 32, 32, 960, 5, 1, 2) == 1     # DeepLab's layer: 16 x 16 phases
    assert plain(8, 256, 256, 256, 3, 1, 8) == 1   # 34 columns x 8 > the map's 256
    assert plain(8, 256, 256, 16, 3, 1, 2) == 1    # 16 of a strip's 64 channels


def test_kxk_plan_of_3x3_stride_1_is_the_ws_plan(lib):
    for ns in (2, 3, 4):
        assert _fwd_plan(lib, 8, 56, 56, 256, 3, 1, 1, ns, occ=4) == _plan(lib, 8, 56, 56, 256, 1, ns)


def test_kxk_consumer_schemes():
    assert [direct_scheme(K, S) for K in (3, 5, 7) for S in (1, 2)] == [False, False, True, False, True, True]


def test_kxk_backward_argument_errors(lib):
    p = C.c_void_p
    def bd(K=7, S=1, pad=3, C_=64, ns=2):
        return lib.tdc_dwconv_bwd_data(p(16), p(16), p(16), i64(2), i64(16), i64(16), i64(C_), i64(K),
                                       i64(S), i64(pad), i64(ns), None)
    def ws(K=7, S=1, pad=3, C_=64, ns=2):
        b = i64()
        return lib.tdc_dwconv_bwd_weight_workspace(i64(2), i64(16), i64(16), i64(C_), i64(K), i64(S),
                                                   i64(pad), i64(ns), C.byref(b))
    def bw(K=7, S=1, pad=3, C_=64, ns=2):
        return lib.tdc_dwconv_bwd_weight(p(16), p(16), p(16), i64(2), i64(16), i64(16), i64(C_), i64(K),
                                         i64(S), i64(pad), i64(ns), p(16), i64(1 << 30), None)
    for f in (bd, ws, bw):
        assert f(K=4) == CODES["TDC_ERR_FILTER_SHAPE"]
        assert f(S=3) == CODES["TDC_ERR_STRIDE"]
        for S in (1, 2):
            assert f(S=S, C_=12) == CODES["TDC_ERR_CHANNELS"]
            assert f(S=S, ns=5) == CODES["TDC_ERR_N_STAGE"]
            assert f(S=S, pad=-1) == CODES["TDC_ERR_PAD"]
    assert bd(pad=7) == CODES["TDC_ERR_PAD"]  # stride 1: pad' = K - 1 - pad < 0
    # stride 2: any pad >= 0; the padded input must hold one K x K window
    assert lib.tdc_dwconv_bwd_data(p(16), p(16), p(16), i64(2), i64(2), i64(2), i64(64), i64(7), i64(2),
                                   i64(1), i64(2), None) == CODES["TDC_ERR_BAD_SHAPE"]  # 2 + 2 < 7
    assert lib.tdc_dwconv_bwd_data(None, p(16), p(16), i64(2), i64(16), i64(16), i64(64), i64(7),
                                   i64(2), i64(3), i64(2), None) == CODES["TDC_ERR_NULL_POINTER"]
    assert lib.tdc_dwconv_bwd_data(p(8), p(16), p(16), i64(2), i64(16), i64(16), i64(64), i64(7),
                                   i64(2), i64(3), i64(2), None) == CODES["TDC_ERR_ALIGNMENT"]
    # empty batch: a successful no-op before any CUDA call
    assert lib.tdc_dwconv_bwd_data(None, None, None, i64(0), i64(16), i64(16), i64(64), i64(5), i64(2),
                                   i64(2), i64(2), None) == 0
    assert lib.tdc_dwconv_bwd_weight_workspace(i64(2), i64(16), i64(16), i64(64), i64(7), i64(1), i64(3),
                                               i64(2), None) == CODES["TDC_ERR_NULL_POINTER"]
    if not torch.cuda.is_available():
        for S in (1, 2):
            assert bd(S=S) == CODES["TDC_ERR_NO_DEVICE"]
            assert ws(S=S) == CODES["TDC_ERR_NO_DEVICE"]
            assert bw(S=S) == CODES["TDC_ERR_NO_DEVICE"]


def _wgrad_plan(lib, N, H, W, Cc, K, pad, ns, sms=148, occ=3):
    out = (i64 * 11)()
    assert lib.tdc_dwconv_bwd_weight_plan(i64(N), i64(H), i64(W), i64(Cc), i64(K), i64(pad), i64(ns),
                                          i64(sms), i64(occ), out) == 0
    return dict(zip(["stage_rows", "qstrips", "cblocks", "strips", "full_units", "tail_band_rows", "grid",
                     "smem", "passes", "rows", "step"], list(out)))


@pytest.mark.parametrize("K", [5, 7])
@pytest.mark.parametrize("N,H,W,Cc,pad", [(64, 224, 336, 256, None), (2, 19, 45, 72, 0), (3, 7, 9, 8, None),
                                          (1, 300, 40, 64, 4)])
@pytest.mark.parametrize("ns", [2, 3, 4])
def test_kxk_wgrad_plan_covers_every_dy_row_once(lib, K, N, H, W, Cc, pad, ns):
    pad = K // 2 if pad is None else pad
    pl = _wgrad_plan(lib, N, H, W, Cc, K, pad, ns)
    P, Q = H + 2 * pad - K + 1, W + 2 * pad - K + 1
    sr, nr, dr = pl["stage_rows"], pl["rows"], pl["step"]
    assert pl["passes"] in (1, 2) and 1 <= nr <= K and pl["passes"] * nr >= K and 1 <= dr <= 4
    assert (ns - 1) * sr >= nr + dr - 2
    assert pl["smem"] == ns * sr * ((32 + K - 1) * 128 + 4096) + 128 <= 200 * 1024
    seen = set()
    for g in range(pl["grid"]):
        for strip, a, b in segments(pl, P, g):
            assert max_stages_held(b - a, nr, 1, sr, dr) <= ns
            for r in range(a, b):
                assert (strip, r) not in seen
                seen.add((strip, r))
    assert len(seen) == pl["strips"] * P


def _s2_plan(lib, which, N, H, W, Cc, K, pad, ns, sms=148, occ=3):
    out = (i64 * 11)()
    assert lib.tdc_dwconv_bwd_s2_plan(i64(N), i64(H), i64(W), i64(Cc), i64(K), i64(pad), i64(ns),
                                      i64(which), i64(sms), i64(occ), out) == 0
    return dict(zip(["stage_rows", "qstrips", "cblocks", "strips", "full_units", "tail_band_rows", "grid",
                     "smem", "passes", "rows", "step"], list(out)))


def dgrad_s2_segment(h0, rows, pad, K, sr, ns, pairs):
    """Restates the stride-2 data gradient's consumer over one segment of dx
    rows [h0, h0 + rows): pairs of dx rows (h, h+1) with h + pad even, `pairs`
    of them per pass, pass k reading window rows pairs*k .. pairs*k + half +
    pairs - 1.  Returns the dx rows stored, the dy rows each stored row reads
    (by the kernel's tap formula) and the most ring stages held at once."""
    half = (K - 1) // 2
    win = half + pairs
    e0 = h0 + pad
    e_first = e0 & ~1
    npairs = (rows + (e0 & 1) + 1) // 2
    passes = -(-npairs // pairs)
    dy_row0 = (e_first >> 1) - half
    dy_rows = passes * pairs + half
    nst = -(-dy_rows // sr)
    acquired = released = worst = 0
    stored, reads = [], {}
    for k in range(passes):
        last_row = pairs * k + win - 1
        assert last_row < dy_rows
        while acquired < nst and acquired * sr <= last_row:
            acquired += 1
        worst = max(worst, acquired - released)
        for i in range(pairs):
            h_even = e_first + 2 * (pairs * k + i) - pad
            for h, taps in ((h_even, [K - 1 - 2 * u for u in range(half + 1)]),
                            (h_even + 1, [K - 2 * u for u in range(1, half + 1)])):
                if h0 <= h < h0 + rows:
                    stored.append(h)
                    # window row pairs*k + i + u holds dy row dy_row0 + that
                    reads[h] = (taps, [dy_row0 + pairs * k + i + ((K - 1 - r) // 2 if (K - 1 - r) % 2 == 0
                                                                   else (K - r) // 2) for r in taps])
        next_first = 1 << 30 if k == passes - 1 else pairs * (k + 1)
        while released < nst and (released + 1) * sr <= next_first:
            released += 1
        assert released <= acquired
    assert acquired == released == nst
    return stored, reads, worst


@pytest.mark.parametrize("K", [3, 5, 7])
@pytest.mark.parametrize("N,H,W,Cc,pad", [(64, 224, 336, 256, None), (2, 19, 45, 72, 0), (3, 7, 9, 8, None),
                                          (1, 301, 40, 64, 4), (4, 33, 47, 136, 1), (2, 8, 8, 64, 7)])
@pytest.mark.parametrize("ns", [2, 3, 4])
def test_dgrad_s2_plan_covers_every_dx_row_once(lib, K, N, H, W, Cc, pad, ns):
    pad = K // 2 if pad is None else pad
    pl = _s2_plan(lib, 0, N, H, W, Cc, K, pad, ns)
    sr, half, pairs = pl["stage_rows"], (K - 1) // 2, pl["passes"]
    assert 1 <= pairs <= 4 and pl["rows"] == half + pairs and pl["step"] == 2 * pairs
    assert (ns - 1) * sr >= pl["rows"] - 1 and 1 <= sr <= 256
    assert pl["smem"] == ns * sr * (16 + half) * 128 + 128 <= 200 * 1024
    assert pl["qstrips"] == -(-W // 32) and pl["cblocks"] == -(-Cc // 64)
    # dy columns: dx column v of strip qs reads (v + pad - s)/2, which must lie
    # in the box [16*qs + ceil(pad/2) - half, + 16 + half) for every tap it uses
    for qs in range(2):
        q0 = 16 * qs + (pad + 1) // 2 - half
        for v in range(32 * qs, 32 * qs + 32):
            for s_ in range(K):
                if (v + pad - s_) % 2 == 0:
                    j = (v + pad - s_) // 2 - q0
                    m, cw = (v - 32 * qs) % 8, (v - 32 * qs) // 8
                    assert 0 <= j < 16 + half
                    # the kernel's register index for (m, s)
                    assert j == 4 * cw + (m + (pad & 1) - s_) // 2 - (pad & 1) + half
    seen = set()
    for g in range(pl["grid"]):
        for strip, a, b in segments(pl, H, g):
            stored, reads, worst = dgrad_s2_segment(a, b - a, pad, K, sr, ns, pairs)
            assert worst <= ns
            assert sorted(stored) == list(range(a, b))
            for h, (taps, rows_read) in reads.items():
                # the kernel's rows are the transposed stencil's: p = (h + pad - r) / 2
                assert rows_read == [(h + pad - r) // 2 for r in taps]
                assert all((h + pad - r) % 2 == 0 for r in taps)
                assert sorted(taps, reverse=True) == taps
                assert set(taps) == {r for r in range(K) if (h + pad - r) % 2 == 0}
            for r in stored:
                assert (strip, r) not in seen
                seen.add((strip, r))
    assert len(seen) == pl["strips"] * H


@pytest.mark.parametrize("K", [3, 5, 7])
@pytest.mark.parametrize("N,H,W,Cc,pad", [(64, 224, 336, 256, None), (2, 19, 45, 72, 0), (3, 7, 9, 8, None),
                                          (1, 300, 40, 64, 4)])
@pytest.mark.parametrize("ns", [2, 3, 4])
def test_wgrad_s2_plan_covers_every_dy_row_once(lib, K, N, H, W, Cc, pad, ns):
    pad = K // 2 if pad is None else pad
    pl = _s2_plan(lib, 1, N, H, W, Cc, K, pad, ns)
    P = (H + 2 * pad - K) // 2 + 1
    sr, nr, dr = pl["stage_rows"], pl["rows"], pl["step"]
    assert pl["passes"] == (2 if K == 7 else 1) and nr == (4 if K == 7 else K) and 1 <= dr <= 4
    assert (ns - 1) * 2 * sr >= 2 * (dr - 1) + nr - 1
    assert pl["smem"] == ns * sr * (2 * (62 + K) * 128 + 4096) + 128 <= 200 * 1024
    seen = set()
    for g in range(pl["grid"]):
        for strip, a, b in segments(pl, P, g):
            # x rows: a stage holds 2*sr of them; a step of dr dy rows from o
            # needs x rows 2o .. 2(o + dr - 1) + nr - 1
            assert max_stages_held(b - a, nr, 2, 2 * sr, dr) <= ns
            for r in range(a, b):
                assert (strip, r) not in seen
                seen.add((strip, r))
    assert len(seen) == pl["strips"] * P


def test_plan_balances_the_headline_shape(lib):
    # the busiest CTA streams at most 3% more rows (halo included) than a perfect split
    for occ in (3, 4):
        pl = _plan(lib, 64, 224, 336, 256, 1, 2, occ=occ)
        assert pl["grid"] == 148 * occ
        streamed = [sum(b - a + 2 for _, a, b in segments(pl, 224, g)) for g in range(pl["grid"])]
        assert max(streamed) <= 1.03 * (64 * 44 * 224 / pl["grid"])


def test_host_pipeline_argument_errors(lib):
    p = C.c_void_p
    def hp(xh=16, wh=16, yh=16, xd=16, wd=16, yd=16, N=2, H=16, W=16, Cc=64, pad=1, ns=2, chunk=0):
        q = lambda v: p(v) if v else None
        return lib.tdc_dwconv_ws_host(q(xh), q(wh), q(yh), i64(N), i64(H), i64(W), i64(Cc), i64(pad),
                                      i64(ns), q(xd), q(wd), q(yd), i64(chunk), None)
    assert hp(xh=0) == CODES["TDC_ERR_NULL_POINTER"]
    assert hp(yd=0) == CODES["TDC_ERR_NULL_POINTER"]
    assert hp(xd=8) == CODES["TDC_ERR_ALIGNMENT"]
    assert hp(Cc=32) == CODES["TDC_ERR_CHANNELS"]
    assert hp(ns=5) == CODES["TDC_ERR_N_STAGE"]
    assert hp(pad=-1) == CODES["TDC_ERR_PAD"]
    assert hp(chunk=-1) == CODES["TDC_ERR_BAD_SHAPE"]
    assert hp(N=0, xh=0, wh=0, yh=0, xd=0, wd=0, yd=0) == 0  # empty: no-op
    if not torch.cuda.is_available():
        assert hp() == CODES["TDC_ERR_NO_DEVICE"]


def test_bf16_entry_points_validate_like_fp16(lib):
    p = C.c_void_p
    def fw(fn, K=3, S=1, C_=64, pad=1, act=0, ns=2, x=16):
        return fn(p(x) if x else None, p(16), None, None, p(16), i64(2), i64(16), i64(16), i64(C_),
                  i64(K), i64(S), i64(pad), i64(act), i64(ns), None)
    def bd(fn, K=3, S=1, C_=64, pad=1, ns=2):
        return fn(p(16), p(16), p(16), i64(2), i64(16), i64(16), i64(C_), i64(K), i64(S), i64(pad),
                  i64(ns), None)
    def bw(fn, K=3, S=1, C_=64, pad=1, ns=2):
        return fn(p(16), p(16), p(16), i64(2), i64(16), i64(16), i64(C_), i64(K), i64(S), i64(pad),
                  i64(ns), p(16), i64(1 << 30), None)
    for f16, b16 in ((lib.tdc_dwconv_fwd, lib.tdc_dwconv_fwd_bf16),):
        for kw in ({"K": 4}, {"S": 3}, {"C_": 12}, {"pad": -1}, {"act": 9}, {"ns": 5}, {"x": 0}):
            assert fw(b16, **kw) == fw(f16, **kw) != 0, kw
    for f16, b16 in ((lib.tdc_dwconv_bwd_data, lib.tdc_dwconv_bwd_data_bf16),
                     (lib.tdc_dwconv_bwd_weight, lib.tdc_dwconv_bwd_weight_bf16)):
        for kw in ({"K": 4}, {"S": 3}, {"C_": 12}, {"pad": -1}, {"ns": 5}):
            fn = bd if f16 is lib.tdc_dwconv_bwd_data else bw
            assert fn(b16, **kw) == fn(f16, **kw) != 0, kw
    # the 3x3 stride-1 bf16 data gradient takes the K x K path: pad <= 2
    assert bd(lib.tdc_dwconv_bwd_data_bf16, pad=3) == CODES["TDC_ERR_PAD"]
    b = i64()
    assert lib.tdc_dwconv_bwd_weight_workspace_bf16(i64(2), i64(16), i64(16), i64(64), i64(3), i64(1),
                                                    i64(1), i64(2), None) == CODES["TDC_ERR_NULL_POINTER"]
    if not torch.cuda.is_available():
        assert fw(lib.tdc_dwconv_fwd_bf16) == CODES["TDC_ERR_NO_DEVICE"]
        assert bd(lib.tdc_dwconv_bwd_data_bf16) == CODES["TDC_ERR_NO_DEVICE"]
        assert lib.tdc_dwconv_bwd_weight_workspace_bf16(i64(2), i64(16), i64(16), i64(64), i64(3), i64(1),
                                                        i64(1), i64(2), C.byref(b)) == CODES["TDC_ERR_NO_DEVICE"]


def test_plain_forward_argument_errors(lib):
    p = C.c_void_p
    def fwd(K=5, stride=2, C_=72, pad=2, H=16, act=0, band=0, N=2, x=16, f=None):
        f = f or lib.tdc_dwconv_fwd_plain
        return f(p(x), p(16), None, None, p(16), i64(N), i64(H), i64(16), i64(C_), i64(K),
                 i64(stride), i64(pad), i64(act), i64(band), None)
    for f in (lib.tdc_dwconv_fwd_plain, lib.tdc_dwconv_fwd_plain_bf16):
        assert fwd(K=4, f=f) == CODES["TDC_ERR_FILTER_SHAPE"]
        assert fwd(stride=3, f=f) == CODES["TDC_ERR_STRIDE"]
        assert fwd(C_=12, f=f) == CODES["TDC_ERR_CHANNELS"]
        assert fwd(pad=-1, f=f) == CODES["TDC_ERR_PAD"]
        assert fwd(act=5, f=f) == CODES["TDC_ERR_ACT"]
        assert fwd(band=-1, f=f) == CODES["TDC_ERR_BAD_SHAPE"]
        assert fwd(K=7, H=2, pad=2, f=f) == CODES["TDC_ERR_BAD_SHAPE"]
        assert fwd(x=24, f=f) == CODES["TDC_ERR_ALIGNMENT"]
        assert fwd(x=0, f=f) == CODES["TDC_ERR_NULL_POINTER"]
        assert fwd(N=0, f=f) == CODES["TDC_OK"]
        if not torch.cuda.is_available():
            assert fwd(f=f) == CODES["TDC_ERR_NO_DEVICE"]
    # n_stage 0 = automatic: argument checks as before, no device here
    r = lib.tdc_dwconv_fwd(p(16), p(16), None, None, p(16), i64(2), i64(16), i64(16), i64(72),
                           i64(5), i64(2), i64(2), i64(0), i64(0), None)
    if not torch.cuda.is_available():
        assert r == CODES["TDC_ERR_NO_DEVICE"]


def uses_plain(N, H, W, Cc, K, S, pad):
    """Restates tdc_dwconv_fwd_uses_plain: the plain kernel when less than
    half of the ws strips' lanes x columns hold outputs, at stride 2 only
    for 7-column-like outputs (fill_q <= 1/4) or layers under 64 MB."""
    P, Q = (H + 2 * pad - K) // S + 1, (W + 2 * pad - K) // S + 1
    fill_c = Cc / (64 * -(-Cc // 64))
    fill_q = Q / (32 * -(-Q // 32))
    if fill_c * fill_q >= 0.5:
        return False
    nbytes = 2 * N * Cc * (H * W + P * Q)
    return S == 1 or fill_q <= 0.25 or nbytes < 64e6


@pytest.mark.parametrize("K,S", [(3, 1), (3, 2), (5, 1), (5, 2), (7, 1), (7, 2)])
def test_automatic_kernel_choice(lib, K, S):
    for (N, H, W, Cc) in [(64, 224, 336, 256), (64, 112, 112, 16), (64, 56, 56, 72),
                          (64, 14, 14, 576), (64, 7, 7, 960), (8, 56, 56, 256),
                          (64, 28, 28, 240), (256, 28, 28, 240), (2, 20, 40, 64),
                          (1, 9, 100, 256), (256, 56, 56, 72), (256, 112, 112, 96)]:
        pad = K // 2
        got = lib.tdc_dwconv_fwd_uses_plain(i64(N), i64(H), i64(W), i64(Cc), i64(K), i64(S),
                                            i64(pad))
        assert got == int(uses_plain(N, H, W, Cc, K, S, pad)), (N, H, W, Cc)
    # the headline shape stays on the ws kernel; a 16-channel layer does not;
    # a large stride-2 layer with 14-column outputs stays, its batch-64 form not
    assert lib.tdc_dwconv_fwd_uses_plain(i64(64), i64(224), i64(336), i64(256), i64(3), i64(1), i64(1)) == 0
    assert lib.tdc_dwconv_fwd_uses_plain(i64(64), i64(112), i64(112), i64(16), i64(3), i64(1), i64(1)) == 1
    assert lib.tdc_dwconv_fwd_uses_plain(i64(256), i64(28), i64(28), i64(192), i64(3), i64(2), i64(1)) == 0
    assert lib.tdc_dwconv_fwd_uses_plain(i64(64), i64(28), i64(28), i64(192), i64(3), i64(2), i64(1)) == 1
    assert lib.tdc_dwconv_fwd_uses_plain(i64(1), i64(16), i64(16), i64(12), i64(3), i64(1), i64(1)) == 0


def plain_cols(K):
    return {3: 8, 5: 4, 7: 2}[K]


def plain_threads(N, P, Q, Cc, K, band_rows):
    """Restates dwconv_plain_kernel's thread -> (n, band, chunk, column
    group, pair) decomposition; yields (n, p0, rows, q0, n_valid, cp)."""
    cpairs = Cc // 2
    clog = 3 if cpairs % 8 == 0 else 2
    chunks = cpairs >> clog
    QT = plain_cols(K)
    qgroups = -(-Q // QT)
    bands = -(-P // band_rows)
    total = N * bands * chunks * qgroups * (1 << clog)
    for t in range(total):
        r = t >> clog
        qg = r % qgroups; r //= qgroups
        chunk = r % chunks; r //= chunks
        band = r % bands
        n = r // bands
        cp = (chunk << clog) + (t & ((1 << clog) - 1))
        p0 = band * band_rows
        yield n, p0, min(band_rows, P - p0), qg * QT, min(QT, Q - qg * QT), cp


@pytest.mark.parametrize("K", [3, 5, 7])
@pytest.mark.parametrize("N,P,Q,Cc,band_rows", [(2, 7, 7, 72, 3), (1, 5, 9, 16, 5),
                                                (3, 4, 3, 40, 1), (1, 10, 2, 8, 4),
                                                (1, 3, 17, 24, 2)])
def test_plain_threads_cover_every_output_once(K, N, P, Q, Cc, band_rows):
    seen = {}
    for n, p0, rows, q0, n_valid, cp in plain_threads(N, P, Q, Cc, K, band_rows):
        assert 0 <= cp < Cc // 2 and rows >= 1 and 1 <= n_valid <= plain_cols(K)
        for o in range(rows):
            for m in range(n_valid):
                key = (n, p0 + o, q0 + m, cp)
                assert key not in seen
                seen[key] = 1
    assert len(seen) == N * P * Q * (Cc // 2)


def dilated_threads(N, P, Q, Cc, K, D, band_rows):
    """Restates dwconv_plain_kernel's thread decomposition with dilation D
    (PlainParams dil / phases): (pair, column group, chunk, band, phase,
    image); a thread of phase (pa, pb) owns output rows pa + D*(p0 + o) and
    columns pb + D*(q0 + m).  Yields (n, pa, pb, p0, rows, q0, n_valid, cp)
    for the threads that have work."""
    cpairs = Cc // 2
    clog = 3 if cpairs % 8 == 0 else 2
    chunks = cpairs >> clog
    QT = plain_cols(K)
    Pp, Qp = -(-P // D), -(-Q // D)
    qgroups = -(-Qp // QT)
    bands = -(-Pp // band_rows)
    total = N * D * D * bands * chunks * qgroups * (1 << clog)
    for t in range(total):
        r = t >> clog
        qg = r % qgroups; r //= qgroups
        chunk = r % chunks; r //= chunks
        band = r % bands; r //= bands
        ph, n = r % (D * D), r // (D * D)
        pa, pb = divmod(ph, D)
        cp = (chunk << clog) + (t & ((1 << clog) - 1))
        p0, q0 = band * band_rows, qg * QT
        rows = min(band_rows, -(-(P - pa) // D) - p0)
        n_valid = min(QT, -(-(Q - pb) // D) - q0)
        if rows <= 0 or n_valid <= 0:
            continue
        yield n, pa, pb, p0, rows, q0, n_valid, cp


@pytest.mark.parametrize("K,S", [(3, 1), (5, 1), (5, 2), (7, 2)])
@pytest.mark.parametrize("D", [1, 2, 3, 4])
@pytest.mark.parametrize("N,P,Q,Cc,band_rows", [(2, 7, 9, 16, 2), (1, 10, 5, 24, 3), (1, 3, 17, 8, 4)])
def test_dilated_threads_cover_every_output_once(K, S, D, N, P, Q, Cc, band_rows):
    pad = 2
    seen = set()
    for n, pa, pb, p0, rows, q0, n_valid, cp in dilated_threads(N, P, Q, Cc, K, D, band_rows):
        h0 = S * (pa + D * p0) - pad
        w0 = S * (pb + D * q0) - pad
        for o in range(rows):
            p_ = pa + D * (p0 + o)
            for r in range(K):  # window row S*o + r of the thread reads input row h0 + D*(S*o + r)
                assert h0 + D * (S * o + r) == S * p_ + D * r - pad
            for m in range(n_valid):
                q_ = pb + D * (q0 + m)
                for s_ in range(K):
                    assert w0 + D * (S * m + s_) == S * q_ + D * s_ - pad
                key = (n, p_, q_, cp)
                assert 0 <= p_ < P and 0 <= q_ < Q and key not in seen
                seen.add(key)
    assert len(seen) == N * P * Q * (Cc // 2)


@pytest.mark.parametrize("K,S", [(3, 1), (3, 2), (5, 1), (5, 2), (7, 1), (7, 2)])
def test_plain_row_loop_feeds_each_output_its_taps_in_order(K, S):
    """Replays the kernel's row loop (unrolled by L = S * ceil(K/S) rows) for
    band heights 1..12: every output row gets tap rows r = 0..K-1 in order,
    starts its accumulator set at r = 0, is stored at r = K-1, and no two
    outputs in flight share an accumulator set."""
    A = -(-K // S)
    L = S * A
    for rows in range(1, 13):
        n_in = S * (rows - 1) + K
        taps = {o: [] for o in range(rows)}
        owner = {}  # accumulator set -> output using it
        stored = []
        for i0 in range(0, n_in, L):
            for U in range(L):
                i = i0 + U
                if i >= n_in:
                    continue
                for r in range(K):
                    if (U - r) % S != 0:
                        continue
                    o = i0 // S + (U - r) // S
                    assert o == (i - r) // S and (i - r) % S == 0
                    if o < 0 or o >= rows:
                        continue
                    a = ((U - r) // S) % A
                    if r == 0:
                        assert a not in owner
                        owner[a] = o
                    assert owner.get(a) == o
                    taps[o].append(r)
                    if r == K - 1:
                        stored.append(o)
                        del owner[a]
        assert all(taps[o] == list(range(K)) for o in range(rows)), rows
        assert sorted(stored) == list(range(rows))


def test_plain_weight_gradient_argument_errors(lib):
    p = C.c_void_p
    b = i64()
    def ws(K=5, stride=1, C_=72, pad=2, H=16, N=2):
        return lib.tdc_dwconv_bwd_weight_plain_workspace(i64(N), i64(H), i64(16), i64(C_), i64(K),
                                                         i64(stride), i64(pad), C.byref(b))
    def wg(K=5, stride=1, C_=72, pad=2, H=16, N=2, x=16, dw=16, f=None):
        f = f or lib.tdc_dwconv_bwd_weight_plain
        return f(p(x), p(16), p(dw), i64(N), i64(H), i64(16), i64(C_), i64(K), i64(stride),
                 i64(pad), p(16), i64(1 << 20), None)
    assert ws(K=4) == CODES["TDC_ERR_FILTER_SHAPE"]
    assert ws(stride=3) == CODES["TDC_ERR_STRIDE"]
    assert ws(C_=12) == CODES["TDC_ERR_CHANNELS"]
    assert ws(pad=-1) == CODES["TDC_ERR_PAD"]
    assert ws(K=7, H=2, pad=2) == CODES["TDC_ERR_BAD_SHAPE"]
    assert lib.tdc_dwconv_bwd_weight_plain_workspace(i64(2), i64(16), i64(16), i64(64), i64(3),
                                                     i64(1), i64(1), None) == CODES["TDC_ERR_NULL_POINTER"]
    for f in (lib.tdc_dwconv_bwd_weight_plain, lib.tdc_dwconv_bwd_weight_plain_bf16):
        assert wg(K=4, f=f) == CODES["TDC_ERR_FILTER_SHAPE"]
        assert wg(stride=0, f=f) == CODES["TDC_ERR_STRIDE"]
        assert wg(C_=12, f=f) == CODES["TDC_ERR_CHANNELS"]
        assert wg(x=0, f=f) == CODES["TDC_ERR_NULL_POINTER"]
        assert wg(dw=0, f=f) == CODES["TDC_ERR_NULL_POINTER"]
        assert wg(x=24, f=f) == CODES["TDC_ERR_ALIGNMENT"]
        if not torch.cuda.is_available():
            assert wg(f=f) == CODES["TDC_ERR_NO_DEVICE"]
            assert ws() == CODES["TDC_ERR_NO_DEVICE"]


def wgrad_uses_plain(N, H, W, Cc, K, S, pad):
    """Restates tdc_dwconv_bwd_weight_uses_plain: output width <= 16 or at
    most 16 channels."""
    Q = (W + 2 * pad - K) // S + 1
    return Q <= 16 or Cc <= 16


@pytest.mark.parametrize("K,S", [(3, 1), (3, 2), (5, 1), (5, 2), (7, 1), (7, 2)])
def test_weight_gradient_choice(lib, K, S):
    for (N, H, W, Cc) in [(64, 224, 336, 256), (64, 112, 112, 16), (64, 14, 14, 576),
                          (64, 7, 7, 960), (256, 28, 28, 192), (2, 20, 40, 64),
                          (64, 112, 112, 32), (64, 56, 56, 72), (64, 33, 33, 64)]:
        args = [i64(v) for v in (N, H, W, Cc, K, S, K // 2)]
        assert lib.tdc_dwconv_bwd_weight_uses_plain(*args) == int(
            wgrad_uses_plain(N, H, W, Cc, K, S, K // 2)), (N, H, W, Cc)
    assert lib.tdc_dwconv_bwd_weight_uses_plain(i64(64), i64(7), i64(7), i64(960), i64(5), i64(1), i64(2)) == 1
    assert lib.tdc_dwconv_bwd_weight_uses_plain(i64(64), i64(56), i64(56), i64(72), i64(3), i64(1), i64(1)) == 0


def wgrad_plain_plan(N, P, Cc, K, sms=148):
    """Restates wgrad_plain_plan: bands of dy rows for about 1024 threads per
    SM counting the K tap rows; units (image, band) dealt 16 or 32 to a CTA."""
    cpairs = Cc // 2
    clog = 3 if cpairs % 8 == 0 else 2
    per_band = max(1, N * cpairs * K)
    bands = min(P, max(1, -(-1024 * sms // per_band)))
    band_rows = -(-P // bands)
    bands = -(-P // band_rows)
    units = N * bands
    upc = 128 >> clog
    return dict(band_rows=band_rows, bands=bands, units=units, upc=upc,
                ugroups=-(-units // upc), chunks=cpairs >> clog, cpc=1 << clog)


@pytest.mark.parametrize("N,P,Cc,K", [(64, 7, 960, 5), (64, 112, 16, 3), (3, 5, 72, 7),
                                      (1, 1, 8, 3), (256, 14, 184, 3)])
def test_plain_weight_gradient_units_cover_every_dy_row_once(N, P, Cc, K):
    pl = wgrad_plain_plan(N, P, Cc, K)
    seen = set()
    for ugroup in range(pl["ugroups"]):          # blockIdx.x / chunks
        for ul in range(pl["upc"]):              # threadIdx.x >> chunk_log2
            u = ugroup * pl["upc"] + ul
            if u >= pl["units"]:
                continue
            n, band = divmod(u, pl["bands"])
            for pr in range(band * pl["band_rows"], min(P, (band + 1) * pl["band_rows"])):
                assert (n, pr) not in seen
                seen.add((n, pr))
    assert len(seen) == N * P
    assert pl["chunks"] * pl["cpc"] == Cc // 2


def test_per_side_padding_argument_errors(lib):
    p = C.c_void_p
    def fwd(K=5, stride=2, C_=72, pads=(0, 1, 0, 1), H=16, act=0, ns=0, N=2, x=16, f=None):
        f = f or lib.tdc_dwconv_fwd_asym
        return f(p(x), p(16), None, None, p(16), i64(N), i64(H), i64(16), i64(C_), i64(K),
                 i64(stride), *[i64(v) for v in pads], i64(act), i64(ns), None)
    for f in (lib.tdc_dwconv_fwd_asym, lib.tdc_dwconv_fwd_asym_bf16):
        assert fwd(K=4, f=f) == CODES["TDC_ERR_FILTER_SHAPE"]
        assert fwd(stride=3, f=f) == CODES["TDC_ERR_STRIDE"]
        assert fwd(C_=12, f=f) == CODES["TDC_ERR_CHANNELS"]
        assert fwd(pads=(0, -1, 0, 0), f=f) == CODES["TDC_ERR_PAD"]
        assert fwd(pads=(0, 0, -1, 0), ns=2, f=f) == CODES["TDC_ERR_PAD"]
        assert fwd(act=5, f=f) == CODES["TDC_ERR_ACT"]
        assert fwd(ns=1, f=f) == CODES["TDC_ERR_N_STAGE"]
        assert fwd(K=7, H=4, pads=(1, 1, 3, 3), f=f) == CODES["TDC_ERR_BAD_SHAPE"]  # 4 + 2 < 7
        assert fwd(x=24, f=f) == CODES["TDC_ERR_ALIGNMENT"]
        assert fwd(N=0, f=f) == CODES["TDC_OK"]
        if not torch.cuda.is_available():
            assert fwd(f=f) == CODES["TDC_ERR_NO_DEVICE"]


def test_dilated_forward_argument_errors(lib):
    p = C.c_void_p
    def fwd(K=3, stride=1, D=2, C_=64, pads=(2, 2, 2, 2), H=16, act=0, N=2, x=16, f=None):
        f = f or lib.tdc_dwconv_fwd_dilated
        return f(p(x), p(16), None, None, p(16), i64(N), i64(H), i64(16), i64(C_), i64(K),
                 i64(stride), i64(D), *[i64(v) for v in pads], i64(act), None)
    for f in (lib.tdc_dwconv_fwd_dilated, lib.tdc_dwconv_fwd_dilated_bf16):
        assert fwd(K=4, f=f) == CODES["TDC_ERR_FILTER_SHAPE"]
        assert fwd(stride=3, f=f) == CODES["TDC_ERR_STRIDE"]
        assert fwd(D=0, f=f) == CODES["TDC_ERR_BAD_SHAPE"]
        assert fwd(C_=12, f=f) == CODES["TDC_ERR_CHANNELS"]
        assert fwd(pads=(-1, 2, 2, 2), f=f) == CODES["TDC_ERR_PAD"]
        assert fwd(act=5, f=f) == CODES["TDC_ERR_ACT"]
        assert fwd(K=7, D=3, H=4, pads=(0, 0, 9, 9), f=f) == CODES["TDC_ERR_BAD_SHAPE"]  # 4 < 19
        assert fwd(x=24, f=f) == CODES["TDC_ERR_ALIGNMENT"]
        assert fwd(x=0, f=f) == CODES["TDC_ERR_NULL_POINTER"]
        assert fwd(N=0, f=f) == CODES["TDC_OK"]
        if not torch.cuda.is_available():
            assert fwd(f=f) == CODES["TDC_ERR_NO_DEVICE"]
            assert fwd(D=1, f=f) == CODES["TDC_ERR_NO_DEVICE"]  # dilation 1: the asym path



def test_dilated_forward_named_kernel_argument_errors(lib):
    """tdc_dwconv_fwd_dilated_ex: the same checks, an unknown kernel
    (TDC_ERR_UNSUPPORTED), and without a device the ring and plain kernels
    both reach the device check."""
    p = C.c_void_p
    def ex(kernel=1, D=2, act=0, bf16=0, K=3, C_=64, x=16, N=2):
        return lib.tdc_dwconv_fwd_dilated_ex(p(x), p(16), None, None, p(16), i64(N), i64(16), i64(16),
                                             i64(C_), i64(K), i64(1), i64(D), *[i64(D)] * 4, i64(act),
                                             i64(kernel), i64(bf16), None)
    for bf16 in (0, 1):
        assert ex(kernel=2, bf16=bf16) == CODES["TDC_ERR_UNSUPPORTED"]
        assert ex(kernel=-2, bf16=bf16) == CODES["TDC_ERR_UNSUPPORTED"]
        assert ex(act=7, bf16=bf16) == CODES["TDC_ERR_ACT"]
        assert ex(K=9, bf16=bf16) == CODES["TDC_ERR_FILTER_SHAPE"]
        assert ex(C_=20, bf16=bf16) == CODES["TDC_ERR_CHANNELS"]
        assert ex(x=8, bf16=bf16) == CODES["TDC_ERR_ALIGNMENT"]
        assert ex(N=0, bf16=bf16) == CODES["TDC_OK"]
        if not torch.cuda.is_available():
            for kernel in (-1, 0, 1):
                assert ex(kernel=kernel, bf16=bf16) == CODES["TDC_ERR_NO_DEVICE"]
            assert ex(kernel=-1, D=1, bf16=bf16) == CODES["TDC_ERR_NO_DEVICE"]  # plain, undilated
