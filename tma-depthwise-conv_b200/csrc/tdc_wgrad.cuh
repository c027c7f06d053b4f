// tdc_wgrad.cuh — weight gradient of the depthwise 3x3 forward (and of the
// K x K forward at stride 1 or 2, below), sm_100a.
//
//   dw[r,s,c] = sum_{n,p,q} x[n, p+r-pad, q+s-pad, c] * dy[n,p,q,c]     (x = 0 outside)
//
// Same streaming structure as the forward: the persistent grid walks the
// (image, 32-column strip, 64-channel block) strips of dy with the forward's
// SegmentIter; a producer thread TMA-loads, per stage, `stage_rows` rows of
// x (34 halo'd columns) and the same rows of dy (32 columns) into an
// mbarrier ring; four consumer warps (lane = channel pair, warp = 8 columns)
// keep the last three dy rows in registers and, for every x row, FMA
// x[i][m+s] * dy[i-r][m] into 18 fp32 accumulators (9 taps x 2 channels) per
// lane.  Both operands stay fp16 (fma.rn.f32.f16).
//
// Reduction without atomics or cross-warp barriers, deterministic: when a
// warp moves to another channel block or finishes, it adds its accumulators
// into its own slice of a workspace, partial[cta][warp][tap][c] (zeroed by
// the CTA at start); a second kernel sums the slices in (cta, warp) order
// into dw (fp32).  The workspace is grid * 4 * 9 * C floats.
#pragma once

#include "tdc_kernels.cuh"

namespace tdc {

constexpr int kDyRowBytes = kStripQ * kBlockC * 2;  // 4096 B: 32 columns x 64 channels

struct WgradParams {
  float* partial;        // [gridDim.x][4 consumer warps][9][C] workspace
  int32_t C, P, Q, pad;
  int32_t qstrips, cblocks, stage_rows;
  int32_t tail_bands, tail_band_rows;
  int64_t full_units, tail_strips;
  uint64_t timeout_ns;
  int* status_host;  // this device's failure slot in mapped host memory, or null
};

// The forward's segment enumeration over dy's [N,P,Q,C] strips.
__device__ __forceinline__ WsParams wgrad_as_ws(const WgradParams& g) {
  WsParams p{};
  p.C = g.C; p.P = g.P; p.Q = g.Q; p.pad = g.pad;
  p.qstrips = g.qstrips; p.cblocks = g.cblocks; p.stage_rows = g.stage_rows;
  p.tail_bands = g.tail_bands; p.tail_band_rows = g.tail_band_rows;
  p.full_units = g.full_units; p.tail_strips = g.tail_strips;
  return p;
}

template <int NS, class E = F16>
__global__ void __launch_bounds__(kWsThreads, 1) dwconv_wgrad_kernel(
    const __grid_constant__ CUtensorMap xmap, const __grid_constant__ CUtensorMap dymap,
    const __grid_constant__ WgradParams g) {
  __shared__ __align__(8) uint64_t full_bar[NS];
  __shared__ __align__(8) uint64_t empty_bar[NS];
  __shared__ volatile int abort_flag;
  extern __shared__ uint8_t dyn_smem[];
  const uint32_t ring = (smem_addr(dyn_smem) + 127u) & ~127u;
  const uint8_t* ring_ptr = dyn_smem + (ring - smem_addr(dyn_smem));
  const uint32_t x_bytes = uint32_t(g.stage_rows) * kRowBytes;
  const uint32_t stage_bytes = x_bytes + uint32_t(g.stage_rows) * kDyRowBytes;
  const WsParams p = wgrad_as_ws(g);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // This CTA's workspace slices (one per consumer warp) start at zero.
  float* cta_slice = g.partial + int64_t(blockIdx.x) * kConsumerWarps * 9 * g.C;
  for (int i = threadIdx.x; i < kConsumerWarps * 9 * g.C; i += blockDim.x) cta_slice[i] = 0.f;

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      mbar_init(smem_addr(&empty_bar[s]), kConsumerWarps);
    }
    abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&xmap);
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
      const int nst = (sg.rows + 2 + g.stage_rows - 1) / g.stage_rows;
      const int32_t c0 = sg.cb * kBlockC;
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
        const uint32_t dst = ring + stage * stage_bytes;
        const int32_t row = sg.p0 + t * g.stage_rows;
        mbar_arrive_expect_tx(fb, stage_bytes);
        // x rows [p0 - pad + t*sr, ...), 34 columns from q0 - pad
        tma_load_4d(dst, &xmap, fb, c0, sg.qs * kStripQ - g.pad, row - g.pad, sg.n);
        // dy rows [p0 + t*sr, ...), 32 columns from q0 (rows past the segment are ignored)
        tma_load_4d(dst + x_bytes, &dymap, fb, c0, sg.qs * kStripQ, row, sg.n);
        armed |= 1u << stage;
        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        ++load;
        if (++stage == NS) { stage = 0; phase ^= 1u; }
      }
    }
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
  uint32_t stage = 0, phase = 0;
  SegmentIter it(blockIdx.x, gridDim.x);
  Segment sg;
  float acc[18];
#pragma unroll
  for (int k = 0; k < 18; ++k) acc[k] = 0.f;
  int cur_cb = -1;
  bool failed = false;

  // Adds this warp's accumulators into its slice and clears them.
  float* slice = cta_slice + int64_t(cw) * 9 * g.C;
  auto flush = [&](int cb) {
    const int ch = cb * kBlockC + 2 * lane;
    if (ch < g.C) {
#pragma unroll
      for (int k = 0; k < 9; ++k) {
        float2* d = reinterpret_cast<float2*>(slice + int64_t(k) * g.C + ch);
        float2 v = *d;
        v.x += acc[2 * k];
        v.y += acc[2 * k + 1];
        *d = v;
      }
    }
#pragma unroll
    for (int k = 0; k < 18; ++k) acc[k] = 0.f;
  };

  while (!failed && it.next_segment(p, sg)) {
    if (sg.cb != cur_cb) {
      if (cur_cb >= 0) flush(cur_cb);
      cur_cb = sg.cb;
    }
    const int rows_in = sg.rows + 2;
    const int q_first = sg.qs * kStripQ + cw * kColsPerWarp;
    const bool active = q_first < g.Q;  // warp-uniform
    uint32_t dyw[3][kColsPerWarp];      // dy rows i, i-1, i-2 (rotating)
#pragma unroll
    for (int r = 0; r < 3; ++r)
#pragma unroll
      for (int m = 0; m < kColsPerWarp; ++m) dyw[r][m] = 0u;
    int lr = 0;
    const uint8_t* sbuf = ring_ptr;
    for (int i = 0; i < rows_in; ++i) {
      if (lr == 0) {
        const bool got = mbar_wait_bounded(smem_addr(&full_bar[stage]), phase, &abort_flag, true,
                                           g.timeout_ns);
        if (__any_sync(0xffffffffu, !got)) {
          if (lane == 0 && !abort_flag) {
            record_failure(TDC_DEVICE_FULL_TIMEOUT, blockIdx.x, stage, -1, g.status_host);
            abort_flag = 1;
          }
          failed = true;
          break;
        }
        sbuf = ring_ptr + stage * stage_bytes;
      }
      if (active) {
        // shift the dy window and bring in dy row i (zero past the segment)
#pragma unroll
        for (int m = 0; m < kColsPerWarp; ++m) {
          dyw[2][m] = dyw[1][m];
          dyw[1][m] = dyw[0][m];
        }
        const uint32_t* dsrc = reinterpret_cast<const uint32_t*>(
            sbuf + x_bytes + lr * kDyRowBytes + (cw * kColsPerWarp) * (kBlockC * 2)) + lane;
        const bool dy_ok = i < sg.rows;
#pragma unroll
        for (int m = 0; m < kColsPerWarp; ++m)
          dyw[0][m] = (dy_ok && q_first + m < g.Q) ? dsrc[m * (kBlockC / 2)] : 0u;
        const uint32_t* xsrc = reinterpret_cast<const uint32_t*>(
            sbuf + lr * kRowBytes + (cw * kColsPerWarp) * (kBlockC * 2)) + lane;
        uint32_t xr[kColsPerWarp + 2];
#pragma unroll
        for (int j = 0; j < kColsPerWarp + 2; ++j) xr[j] = xsrc[j * (kBlockC / 2)];
        // x row i is tap r of dy row i - r
#pragma unroll
        for (int r = 0; r < 3; ++r) {
#pragma unroll
          for (int m = 0; m < kColsPerWarp; ++m)
#pragma unroll
            for (int s = 0; s < 3; ++s)
              fma2<E>(xr[m + s], dyw[r][m], acc[2 * (r * 3 + s)], acc[2 * (r * 3 + s) + 1]);
        }
      }
      if (++lr == g.stage_rows || i == rows_in - 1) {
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&empty_bar[stage]));
        lr = 0;
        if (++stage == NS) { stage = 0; phase ^= 1u; }
      }
    }
  }
  if (cur_cb >= 0 && !failed) flush(cur_cb);
}

// ============================================================================
// Weight gradient of the K x K stride-S forward (K = 5, 7 at stride 1; K =
// 3, 5, 7 at stride 2):
//   dw[r,s,c] = sum_{n,p,q} x[n, S*p+r-pad, S*q+s-pad, c] * dy[n,p,q,c]
// computed for the tap rows r in [R0, R0 + NR) by one launch (the host runs
// one or two launches to cover all K rows, so a lane never holds more than
// NR*K*2 sums).  The same persistent walk over dy's strips and the same
// producer, with the ring split in two: NS*S*sr rows of x (S*31 + K columns
// each) followed by NS*sr rows of dy (32 columns); stage t of a segment
// fills x rows [S*(p0 + t*sr) - pad + R0, ...) (S*sr of them) and dy rows
// [p0 + t*sr, ...) (sr of them) in slot (seq + t) % NS, so segment x row i
// sits at x ring row (S*sr*(seq % NS) + i) mod (NS*S*sr) and dy row o at dy
// ring row (sr*(seq % NS) + o) mod (NS*sr).  Consumers take one dy row o at
// a time with its NR x rows S*o .. S*o + NR - 1 (the direct scheme of the
// forward: the warp holds the stages of that window, which the host keeps
// within the ring with (NS - 1) * S * sr >= NR - 1) and accumulate
// x[S*o+R0+r][S*m+s] * dy[o][m] into NR*K*2 fp32 sums per lane.  Workspace
// slices hold all K*K taps (partial[cta][warp][K*K][C]); a launch zeroes and
// fills only its rows' taps, and the reduction of the 3x3 kernel sums them.
// ============================================================================
// dy rows a consumer step takes (they share the x rows of their windows, so
// an x row is read from shared memory once per step instead of once per dy
// row).  Measured at 64 x 224 x 336 x 256, best n_stage each (us, 1 / 2 / 3
// rows): stride 1 5x5 1812 / 1559 / 1479, 7x7 3165 / 2938 / 2840; stride 2
// (windows two x rows taller per extra dy row) 3x3 458 / 502 / 551, 5x5
// 633 / 675 / 793, 7x7 1101 / 1278 / 1288.
#ifndef TDC_WGRAD_DY_ROWS_S1
#define TDC_WGRAD_DY_ROWS_S1 3
#endif
#ifndef TDC_WGRAD_DY_ROWS_S2
#define TDC_WGRAD_DY_ROWS_S2 1
#endif
__host__ __device__ constexpr int wgrad_dy_rows(int K, int S) {
  return K > 0 && S == 1 ? TDC_WGRAD_DY_ROWS_S1 : TDC_WGRAD_DY_ROWS_S2;
}

template <int K, int S = 1>
struct WgradGeom {
  static constexpr int kXCols = S * (kStripQ - 1) + K;        // x columns of a strip
  static constexpr int kXRowB = kXCols * kBlockC * 2;         // bytes of one x ring row
  static constexpr int kXWarp = S * (kColsPerWarp - 1) + K;   // x columns one warp reads
};

template <int NS, int K, int R0, int NR, int S = 1, class E = F16>
__global__ void __launch_bounds__(kWsThreads, 3)
    dwconv_wgrad_kxk_kernel(const __grid_constant__ CUtensorMap xmap,
                            const __grid_constant__ CUtensorMap dymap,
                            const __grid_constant__ WgradParams g) {
  static_assert(R0 >= 0 && NR >= 1 && R0 + NR <= K, "tap rows");
  static_assert(S == 1 || S == 2, "stride");
  static_assert(NR >= S, "every dy row's stage is also an x stage of the segment");
  using G = WgradGeom<K, S>;
  __shared__ __align__(8) uint64_t full_bar[NS];
  __shared__ __align__(8) uint64_t empty_bar[NS];
  __shared__ volatile int abort_flag;
  extern __shared__ uint8_t dyn_smem[];
  const uint32_t ring = (smem_addr(dyn_smem) + 127u) & ~127u;
  const uint8_t* ring_ptr = dyn_smem + (ring - smem_addr(dyn_smem));
  const int sr = g.stage_rows;               // dy rows per stage (S * sr x rows)
  const int ring_rows = NS * sr;              // dy rows of the ring
  const int x_ring_rows = S * ring_rows;      // x rows of the ring
  const uint32_t x_stage_bytes = uint32_t(S * sr) * G::kXRowB;
  const uint32_t dy_stage_bytes = uint32_t(sr) * kDyRowBytes;
  const uint32_t dy_ring = ring + uint32_t(x_ring_rows) * G::kXRowB;  // 128-B aligned
  const uint8_t* dy_ring_ptr = ring_ptr + int64_t(x_ring_rows) * G::kXRowB;
  const WsParams p = wgrad_as_ws(g);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  // Zero this launch's taps (rows R0 .. R0+NR-1) of the CTA's warp slices.
  float* cta_slice = g.partial + int64_t(blockIdx.x) * kConsumerWarps * (K * K) * g.C;
  for (int i = threadIdx.x; i < kConsumerWarps * NR * K * g.C; i += blockDim.x) {
    const int w4 = i / (NR * K * g.C);
    cta_slice[int64_t(w4) * K * K * g.C + R0 * K * g.C + (i - w4 * NR * K * g.C)] = 0.f;
  }

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      mbar_init(smem_addr(&empty_bar[s]), kConsumerWarps);
    }
    abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&xmap);
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
      const int nst = (S * (sg.rows - 1) + NR + S * sr - 1) / (S * sr);
      const int32_t c0 = sg.cb * kBlockC;
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
        const int32_t row = sg.p0 + t * sr;
        mbar_arrive_expect_tx(fb, x_stage_bytes + dy_stage_bytes);
        // x rows [S*(p0 + t*sr) - pad + R0, ...), S*31 + K columns from S*q0 - pad
        tma_load_4d(ring + stage * x_stage_bytes, &xmap, fb, c0, S * sg.qs * kStripQ - g.pad,
                    S * row - g.pad + R0, sg.n);
        // dy rows [p0 + t*sr, ...), 32 columns from q0 (rows past the segment are not read)
        tma_load_4d(dy_ring + stage * dy_stage_bytes, &dymap, fb, c0, sg.qs * kStripQ, row, sg.n);
        armed |= 1u << stage;
        armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        ++load;
        if (++stage == NS) { stage = 0; phase ^= 1u; }
      }
    }
    for (int s = 0; s < NS; ++s) {
      if (!(armed & (1u << s))) continue;
      if (!mbar_wait_bounded(smem_addr(&full_bar[s]), (armed_parity >> s) & 1u, &abort_flag,
                             false, g.timeout_ns))
        record_failure(TDC_DEVICE_DRAIN_TIMEOUT, blockIdx.x, s, load, g.status_host);
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  constexpr int DR = wgrad_dy_rows(K, S);
  constexpr int kWin = S * (DR - 1) + NR;  // x rows of one step
  const int cw = warp - 1;
  SegmentIter it(blockIdx.x, gridDim.x);
  Segment sg;
  float acc[2 * NR * K];
#pragma unroll
  for (int k = 0; k < 2 * NR * K; ++k) acc[k] = 0.f;
  int cur_cb = -1;
  bool failed = false;
  // Next ring stage to acquire / release, as slot and phase (no division).
  int acq_slot = 0, rel_slot = 0;
  uint32_t acq_phase = 0;
  int seg_slot = 0;  // slot of the current segment's first stage
  const int xs = S * sr;  // x rows per stage

  float* slice = cta_slice + int64_t(cw) * (K * K) * g.C + int64_t(R0) * K * g.C;
  auto flush = [&](int cb) {
    const int ch = cb * kBlockC + 2 * lane;
    if (ch < g.C) {
#pragma unroll
      for (int k = 0; k < NR * K; ++k) {
        float2* d = reinterpret_cast<float2*>(slice + int64_t(k) * g.C + ch);
        float2 v = *d;
        v.x += acc[2 * k];
        v.y += acc[2 * k + 1];
        *d = v;
      }
    }
#pragma unroll
    for (int k = 0; k < 2 * NR * K; ++k) acc[k] = 0.f;
  };

  while (!failed && it.next_segment(p, sg)) {
    if (sg.cb != cur_cb) {
      if (cur_cb >= 0) flush(cur_cb);
      cur_cb = sg.cb;
    }
    const int rows_in = S * (sg.rows - 1) + NR;  // x rows of the segment
    const int nst = (rows_in + xs - 1) / xs;
    const bool active = sg.qs * kStripQ + cw * kColsPerWarp < g.Q;  // warp-uniform
    int acquired = 0, released = 0;
    int acq_end = 0;   // x rows covered by the acquired stages
    int rel_end = xs;  // x rows up to the end of stage `released`
    int rr0 = seg_slot * xs;  // x ring row of step's first dy row's first x row
    int dr0 = seg_slot * sr;  // dy ring row of the step's first dy row
    for (int o = 0; o < sg.rows; o += DR) {
      const int nout = min(DR, sg.rows - o);  // dy rows of this step
      const int last_x = S * (o + nout - 1) + NR - 1;
      while (acquired < nst && acq_end <= last_x) {
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
        acq_end += xs;
        if (++acq_slot == NS) { acq_slot = 0; acq_phase ^= 1u; }
      }
      if (failed) break;
      if (active) {
        // dy columns past Q were zero-filled by the copy.
        uint32_t dyr[DR][kColsPerWarp];
#pragma unroll
        for (int t = 0; t < DR; ++t) {
          int dr = dr0 + t;
          if (dr >= ring_rows) dr -= ring_rows;
          const uint32_t* dsrc = reinterpret_cast<const uint32_t*>(
              dy_ring_ptr + dr * kDyRowBytes + (cw * kColsPerWarp) * (kBlockC * 2)) + lane;
#pragma unroll
          for (int m = 0; m < kColsPerWarp; ++m) dyr[t][m] = t < nout ? dsrc[m * (kBlockC / 2)] : 0u;
        }
        // x row i of the step is tap row r = i - S*t of its dy row t.
#pragma unroll
        for (int i = 0; i < kWin; ++i) {
          if (i > last_x - S * o) break;  // past the last valid dy row's window (warp-uniform)
          int rr = rr0 + i;
          if (rr >= x_ring_rows) rr -= x_ring_rows;
          const uint32_t* xsrc = reinterpret_cast<const uint32_t*>(
              ring_ptr + rr * G::kXRowB + (S * cw * kColsPerWarp) * (kBlockC * 2)) + lane;
          uint32_t xr[G::kXWarp];
#pragma unroll
          for (int j = 0; j < G::kXWarp; ++j) xr[j] = xsrc[j * (kBlockC / 2)];
#pragma unroll
          for (int t = 0; t < DR; ++t) {
            const int r = i - S * t;
            if (r < 0 || r >= NR) continue;
#pragma unroll
            for (int s2 = 0; s2 < K; ++s2)
#pragma unroll
              for (int m = 0; m < kColsPerWarp; ++m)
                fma2<E>(xr[S * m + s2], dyr[t][m], acc[2 * (r * K + s2)],
                            acc[2 * (r * K + s2) + 1]);
          }
        }
      }
      // Release the stages wholly below the next step's first x row.
      const int next_first = o + DR >= sg.rows ? (1 << 30) : S * (o + DR);
      if (released < nst && rel_end <= next_first) {
        __syncwarp();
        while (released < nst && rel_end <= next_first) {
          if (lane == 0) mbar_arrive(smem_addr(&empty_bar[rel_slot]));
          ++released;
          rel_end += xs;
          if (++rel_slot == NS) rel_slot = 0;
        }
      }
      rr0 += S * DR;
      if (rr0 >= x_ring_rows) rr0 -= x_ring_rows;
      dr0 += DR;
      if (dr0 >= ring_rows) dr0 -= ring_rows;
    }
    seg_slot = acq_slot;  // the next segment starts at a fresh stage
  }
  if (cur_cb >= 0 && !failed) flush(cur_cb);
}

// dw[i] = sum over the slices of partial[slice][i] (i = k*C + c), in a fixed
// order: block b owns outputs 32b .. 32b+31; warp g of the block sums slices
// g, g + 32, g + 64, ... in ascending order for its lane's output, and the 32
// warp sums are combined by a fixed binary tree in shared memory.  The order
// depends only on the slice count, so results are bit-reproducible, and each
// output's 1 + slices/32 dependent loads keep the kernel short (one thread
// per output would chain all slices).
constexpr int kReduceGroups = 32;

__global__ void __launch_bounds__(32 * kReduceGroups) dwconv_wgrad_reduce_kernel(
    const float* __restrict__ partial, float* __restrict__ dw, int32_t slices, int32_t n) {
  __shared__ float part[kReduceGroups][33];
  const int lane = threadIdx.x & 31, grp = threadIdx.x >> 5;
  const int i = blockIdx.x * 32 + lane;
  float s = 0.f;
  if (i < n) {
#pragma unroll 4
    for (int b = grp; b < slices; b += kReduceGroups) s += partial[int64_t(b) * n + i];
  }
  part[grp][lane] = s;
  __syncthreads();
#pragma unroll
  for (int h = kReduceGroups / 2; h >= 1; h >>= 1) {
    if (grp < h) part[grp][lane] += part[grp + h][lane];
    __syncthreads();
  }
  if (grp == 0 && i < n) dw[i] = part[0][lane];
}

// Launch of the reduction over `slices` workspace slices of n floats.
inline cudaError_t launch_wgrad_reduce(const float* partial, float* dw, int32_t slices, int32_t n,
                                       cudaStream_t st) {
  dwconv_wgrad_reduce_kernel<<<dim3(unsigned((n + 31) / 32)), dim3(32 * kReduceGroups), 0, st>>>(
      partial, dw, slices, n);
  return cudaGetLastError();
}

}  // namespace tdc
