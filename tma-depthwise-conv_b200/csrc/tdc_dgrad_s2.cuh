// tdc_dgrad_s2.cuh — data gradient of the K x K (K = 3, 5, 7) stride-2
// depthwise forward, sm_100a.
//
// The forward reads x[n, 2p - pad + r, 2q - pad + s, c] for output (p, q), so
//   dx[n,h,v,c] = sum over taps (r, s) with h + pad - r and v + pad - s even of
//                 dy[n, (h+pad-r)/2, (v+pad-s)/2, c] * w[r,s,c]   (dy = 0 outside [0,P)x[0,Q))
// a transposed stencil: a dx pixel takes ceil(K/2) or floor(K/2) tap rows
// (by the parity of h + pad) times as many tap columns.  Per output the fp32
// chain runs over its taps with r descending, then s descending (the order
// of the stride-1 data gradient, which is the forward with flipped taps),
// from +0, with one fp16 rounding.  Taps whose dy position is outside dy stay
// in the chain as zero products, as in the stride-1 data gradient.
//
// Work decomposition: the forward's persistent walk over 32-column strips,
// here of dx ([N,H,W,C]): SegmentIter with P = H, Q = W.  A segment's dx rows
// are taken in pairs (h, h + 1) with h + pad even; both rows of a pair read
// the same kHalf + 1 dy rows (e/2 - kHalf .. e/2, e = h + pad): the even row
// with taps r = K-1-2t, the odd row with r = K-2t (t >= 1) for window row t.
// A pass covers RP consecutive pairs (2*RP dx rows) from kHalf + RP dy rows,
// each read from shared memory once and fed to every row of the pass it is a
// tap row of.  The producer streams dy rows (16 + kHalf columns of 64
// channels, the dy columns of the strip) into an NS-deep ring; consumer warp
// cw owns dx columns 8cw .. 8cw+7 of the strip, which read dy columns
// 4cw .. 4cw + 3 + kHalf of the box.  A lane owns one channel pair; the taps
// are held in registers as packed fp16 pairs and the FMA is fma.rn.f32.f16.
#pragma once

#include "tdc_kernels.cuh"

namespace tdc {

// Pairs of dx rows per pass, measured at 64 x 224 x 336 x 256 (more pairs
// amortise the per-pass bookkeeping and stores' addressing; 7x7 keeps one:
// its 49 taps leave no registers for a second pair's accumulators).
#ifndef TDC_DGS2_PAIRS3
#define TDC_DGS2_PAIRS3 2
#endif
#ifndef TDC_DGS2_PAIRS5
#define TDC_DGS2_PAIRS5 2
#endif
#ifndef TDC_DGS2_PAIRS7
#define TDC_DGS2_PAIRS7 1
#endif
__host__ __device__ constexpr int dgrad_s2_pairs(int K) {
  return K == 3 ? TDC_DGS2_PAIRS3 : (K == 5 ? TDC_DGS2_PAIRS5 : TDC_DGS2_PAIRS7);
}

// Resident CTAs per SM the kernel is compiled for (bounds its registers).
#ifndef TDC_DGS2_MINB3
#define TDC_DGS2_MINB3 3
#endif
__host__ __device__ constexpr int dgrad_s2_min_blocks(int K) { return K == 3 ? TDC_DGS2_MINB3 : 3; }

template <int K>
struct DgradS2Geom {
  static constexpr int kHalf = (K - 1) / 2;
  static constexpr int kDyCols = kStripQ / 2 + kHalf;        // dy columns of a strip (TMA box)
  static constexpr int kDyRowB = kDyCols * kBlockC * 2;      // bytes of one ring row
  static constexpr int kDyWarp = kColsPerWarp / 2 + kHalf;   // dy columns one warp reads
  static constexpr int kPairs = dgrad_s2_pairs(K);           // dx row pairs per pass
  static constexpr int kWin = kHalf + kPairs;                // dy rows of one pass
};

// Ring capacity in dy rows, split over the n_stage stages.
constexpr int kDgradS2RingRows = 16;

struct DgradS2Params {
  const __half* w;
  __half* dx;
  int32_t H, W, C, P, Q, pad;
  int32_t qstrips, cblocks, stage_rows;
  int32_t tail_bands, tail_band_rows;
  int64_t full_units, tail_strips;
  uint64_t timeout_ns;
  int* status_host;  // this device's failure slot in mapped host memory, or null
};

// The forward's segment enumeration over dx's [N,H,W,C] strips.
__device__ __forceinline__ WsParams dgrad_s2_as_ws(const DgradS2Params& g) {
  WsParams p{};
  p.C = g.C; p.P = g.H; p.Q = g.W; p.pad = g.pad;
  p.qstrips = g.qstrips; p.cblocks = g.cblocks; p.stage_rows = g.stage_rows;
  p.tail_bands = g.tail_bands; p.tail_band_rows = g.tail_band_rows;
  p.full_units = g.full_units; p.tail_strips = g.tail_strips;
  return p;
}

// Passes and dy rows of a segment of dx rows [h0, h0 + rows): the first pair
// starts at the even e = h + pad at or below h0 + pad (its even row is h0 - 1,
// outside the segment, when h0 + pad is odd); pass k holds pairs
// kPairs*k .. kPairs*k + kPairs - 1 and reads window rows kPairs*k ..
// kPairs*k + kWin - 1.  Rows of pairs past the segment are computed, not stored.
struct DgradS2Seg {
  int e_first;   // h + pad of the even row of pair 0
  int passes;
  int dy_row0;   // first dy row of the segment's window (may be negative)
  int dy_rows;   // dy rows the segment streams
};

template <int K>
__host__ __device__ __forceinline__ DgradS2Seg dgrad_s2_segment(int h0, int rows, int pad) {
  using G = DgradS2Geom<K>;
  DgradS2Seg s;
  const int e0 = h0 + pad;
  s.e_first = e0 & ~1;
  const int pairs = (rows + (e0 & 1) + 1) / 2;
  s.passes = (pairs + G::kPairs - 1) / G::kPairs;
  s.dy_row0 = (s.e_first >> 1) - G::kHalf;
  s.dy_rows = s.passes * G::kPairs + G::kHalf;
  return s;
}

// PODD = pad & 1: the parity of v + pad for the warp's first column, which
// fixes at compile time which taps (and which dy column of the lane's
// registers) each of the 8 columns uses.
template <int NS, int K, int PODD, class E = F16>
__global__ void __launch_bounds__(kWsThreads, (dgrad_s2_min_blocks(K)))
    dwconv_dgrad_s2_kernel(const __grid_constant__ CUtensorMap dymap,
                           const __grid_constant__ DgradS2Params g) {
  using G = DgradS2Geom<K>;
  __shared__ __align__(8) uint64_t full_bar[NS];
  __shared__ __align__(8) uint64_t empty_bar[NS];
  __shared__ volatile int abort_flag;
  extern __shared__ uint8_t dyn_smem[];
  const uint32_t ring = (smem_addr(dyn_smem) + 127u) & ~127u;
  const uint8_t* ring_ptr = dyn_smem + (ring - smem_addr(dyn_smem));
  const int sr = g.stage_rows;
  const int ring_rows = NS * sr;
  const uint32_t stage_bytes = uint32_t(sr) * G::kDyRowB;
  const WsParams p = dgrad_s2_as_ws(g);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      mbar_init(smem_addr(&empty_bar[s]), kConsumerWarps);
    }
    abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&dymap);
  }
  __syncthreads();

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane != 0) return;
    uint32_t stage = 0, phase = 0;
    uint32_t armed = 0, armed_parity = 0;
    int64_t load = 0;
    bool ok = true;
    SegmentIter it(blockIdx.x, gridDim.x);
    Segment sg;
    while (ok && it.next_segment(p, sg)) {
      const DgradS2Seg d = dgrad_s2_segment<K>(sg.p0, sg.rows, g.pad);
      const int nst = (d.dy_rows + sr - 1) / sr;
      const int32_t c0 = sg.cb * kBlockC;
      // dy column of the strip's first dx column's lowest tap, v0 = 32 * qs:
      // (v0 + pad - s) / 2 over the strip starts at v0/2 + ceil(pad/2) - kHalf.
      const int32_t q0 = sg.qs * (kStripQ / 2) + ((g.pad + 1) >> 1) - G::kHalf;
      for (int t = 0; t < nst; ++t) {
        if (!mbar_wait_bounded(smem_addr(&empty_bar[stage]), phase ^ 1u, &abort_flag, true,
                               g.timeout_ns)) {
          if (!abort_flag) {
            record_failure(TDC_DEVICE_EMPTY_TIMEOUT, blockIdx.x, stage, load, g.status_host);
            abort_flag = 1;
          }
          ok = false;
          break;
        }
        const uint32_t fb = smem_addr(&full_bar[stage]);
        mbar_arrive_expect_tx(fb, stage_bytes);
        tma_load_4d(ring + stage * stage_bytes, &dymap, fb, c0, q0, d.dy_row0 + t * sr, sg.n);
        armed |= 1u << stage;
        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        ++load;
        if (++stage == NS) { stage = 0; phase ^= 1u; }
      }
    }
    // Never leave the CTA while one of its copies may still write shared memory.
    for (int s = 0; s < NS; ++s) {
      if (!(armed & (1u << s))) continue;
      if (!mbar_wait_bounded(smem_addr(&full_bar[s]), (armed_parity >> s) & 1u, &abort_flag,
                             false, g.timeout_ns))
        record_failure(TDC_DEVICE_DRAIN_TIMEOUT, blockIdx.x, s, load, g.status_host);
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  const int cw = warp - 1;
  SegmentIter it(blockIdx.x, gridDim.x);
  Segment sg;
  int last_cb = -1;
  uint32_t wt[K * K];
  // Next ring stage to acquire / release, as slot and phase (no division).
  int acq_slot = 0, rel_slot = 0;
  uint32_t acq_phase = 0;
  int seg_slot = 0;  // slot of the current segment's first stage
  bool failed = false;
  const int64_t dx_col_stride = g.C;
  const int64_t dx_row_stride = int64_t(g.W) * g.C;
  while (!failed && it.next_segment(p, sg)) {
    const DgradS2Seg d = dgrad_s2_segment<K>(sg.p0, sg.rows, g.pad);
    const int nst = (d.dy_rows + sr - 1) / sr;
    const int c0 = sg.cb * kBlockC;
    const bool chan_ok = c0 + 2 * lane < g.C;
    if (sg.cb != last_cb) {
      const uint32_t* wp = reinterpret_cast<const uint32_t*>(g.w + c0) + lane;
#pragma unroll
      for (int k = 0; k < K * K; ++k) wt[k] = chan_ok ? __ldg(wp + int64_t(k) * (g.C / 2)) : 0u;
      last_cb = sg.cb;
    }
    const int v_first = sg.qs * kStripQ + cw * kColsPerWarp;
    const int n_valid = min(kColsPerWarp, g.W - v_first);  // <= 0: warp idle
    __half* dxcol = g.dx + (int64_t(sg.n) * g.H * g.W + v_first) * g.C + c0 + 2 * lane;
    const int h_end = sg.p0 + sg.rows;
    int acquired = 0, released = 0;
    int acq_end = 0;  // window rows covered by the acquired stages (acquired * sr)
    int rel_end = sr; // window rows up to the end of stage `released`
    int rr0 = seg_slot * sr;  // ring row of window row 0 of the current pass
    for (int k = 0; k < d.passes; ++k) {
      // Pass k reads window rows kPairs*k .. kPairs*k + kWin - 1.
      const int last_row = G::kPairs * k + G::kWin - 1;
      while (acquired < nst && acq_end <= last_row) {
        const bool got = mbar_wait_bounded(smem_addr(&full_bar[acq_slot]), acq_phase, &abort_flag,
                                           true, g.timeout_ns);
        if (__any_sync(0xffffffffu, !got)) {
          if (lane == 0 && !abort_flag) {
            record_failure(TDC_DEVICE_FULL_TIMEOUT, blockIdx.x, acq_slot, -1, g.status_host);
            abort_flag = 1;
          }
          failed = true;
          break;
        }
        ++acquired;
        acq_end += sr;
        if (++acq_slot == NS) { acq_slot = 0; acq_phase ^= 1u; }
      }
      if (failed) break;
      const int h_first = d.e_first + 2 * G::kPairs * k - g.pad;  // even row of the pass's pair 0
      if (n_valid > 0) {
        RowAcc ae[G::kPairs], ao[G::kPairs];  // pair i: rows h_first + 2i (even e), + 1 (odd e)
#pragma unroll
        for (int i = 0; i < G::kPairs; ++i)
#pragma unroll
          for (int v = 0; v < 2 * kColsPerWarp; ++v) { ae[i].v[v] = 0.f; ao[i].v[v] = 0.f; }
#pragma unroll
        for (int t = 0; t < G::kWin; ++t) {
          int rr = rr0 + t;
          if (rr >= ring_rows) rr -= ring_rows;
          const uint32_t* src = reinterpret_cast<const uint32_t*>(
              ring_ptr + rr * G::kDyRowB + (cw * (kColsPerWarp / 2)) * (kBlockC * 2)) + lane;
          uint32_t dr[G::kDyWarp];
#pragma unroll
          for (int j = 0; j < G::kDyWarp; ++j) dr[j] = src[j * (kBlockC / 2)];
#pragma unroll
          for (int i = 0; i < G::kPairs; ++i) {
            const int u = t - i;  // window row of pair i
            if (u < 0 || u > G::kHalf) continue;
#pragma unroll
            for (int m = 0; m < kColsPerWarp; ++m) {
#pragma unroll
              for (int s = K - 1; s >= 0; --s) {
                if (((m + PODD + s) & 1) != 0) continue;  // v + pad - s must be even
                // dy column of (m, s) relative to the warp's first one
                const int j = (m + PODD - s) / 2 - PODD + G::kHalf;
                fma2<E>(dr[j], wt[(K - 1 - 2 * u) * K + s], ae[i].v[2 * m], ae[i].v[2 * m + 1]);
                if (u >= 1)
                  fma2<E>(dr[j], wt[(K - 2 * u) * K + s], ao[i].v[2 * m], ao[i].v[2 * m + 1]);
              }
            }
          }
        }
        if (chan_ok) {
#pragma unroll
          for (int i = 0; i < 2 * G::kPairs; ++i) {
            const int h = h_first + i;  // rows h_first .. h_first + 2*kPairs - 1
            if (h < sg.p0 || h >= h_end) continue;
            const RowAcc& a = (i & 1) ? ao[i / 2] : ae[i / 2];
            __half* dst = dxcol + int64_t(h) * dx_row_stride;
            if (n_valid == kColsPerWarp) {
#pragma unroll
              for (int m = 0; m < kColsPerWarp; ++m)
                *reinterpret_cast<uint32_t*>(dst + m * dx_col_stride) =
                    pack2_rn<E>(a.v[2 * m], a.v[2 * m + 1]);
            } else {
#pragma unroll
              for (int m = 0; m < kColsPerWarp; ++m)
                if (m < n_valid)
                  *reinterpret_cast<uint32_t*>(dst + m * dx_col_stride) =
                      pack2_rn<E>(a.v[2 * m], a.v[2 * m + 1]);
            }
          }
        }
      }
      // Release the stages wholly below the next pass's first window row.
      const int next_first = k == d.passes - 1 ? (1 << 30) : G::kPairs * (k + 1);
      if (released < nst && rel_end <= next_first) {
        __syncwarp();
        while (released < nst && rel_end <= next_first) {
          if (lane == 0) mbar_arrive(smem_addr(&empty_bar[rel_slot]));
          ++released;
          rel_end += sr;
          if (++rel_slot == NS) rel_slot = 0;
        }
      }
      rr0 += G::kPairs;
      if (rr0 >= ring_rows) rr0 -= ring_rows;
    }
    seg_slot = acq_slot;  // the next segment starts at a fresh stage
  }
}

}  // namespace tdc
