// tdc_kernels.cuh — sm_100a kernels for the NHWC fp16 depthwise conv2d
// forward: 3x3 stride 1 (the reference's surface), and K x K (K = 3, 5, 7)
// with stride 1 or 2; symmetric zero padding, fp32 accumulation, fp16 out.
//
// Arithmetic contract (shared with the CPU oracle, bit for bit):
//   acc = +0; for r in 0..K-1: for s in 0..K-1: acc = fma(fp32(x), fp32(w), acc)
//   y   = fp16 round-to-nearest-even(acc)
// with x = 0 outside the image.  For K = 3, stride 1 this is the per-output
// computation of the reference kernels (csrc/kernel_v0_naive_float4.cu:37-74
// and csrc/kernel_tma_ws.cuh:218-246: r-major, s-minor fp32 chain from 0).
#pragma once

#include <type_traits>

#include "tdc_ptx.cuh"
#include "tdc_dwconv.h"

namespace tdc {

// Calls f(std::integral_constant<int, U>{}) for U = 0 .. N-1, in order.
template <int U, int N>
struct UnrollSteps {
  template <class F>
  __device__ __forceinline__ static void run(F&& f) {
    if constexpr (U < N) {
      f(std::integral_constant<int, U>{});
      UnrollSteps<U + 1, N>::run(f);
    }
  }
};
template <int N, class F>
__device__ __forceinline__ void unroll_steps(F&& f) {
  UnrollSteps<0, N>::run(f);
}

// ============================================================================
// TMA warp-specialised kernel (the `dwconv_ws` / `dwconv_ws_probe` calls).
//
// Work decomposition.  A strip is (image n, 32 output columns, 64-channel
// block cb) over all P output rows; strips are enumerated (n, column strip,
// cb) with cb fastest, so strips running at the same moment on different
// SMs are the channel blocks of one pixel column (the same DRAM pages) and
// horizontal neighbours (sharing their halo columns through L2).
// The grid is persistent.  CTA g first takes whole strips g, g + grid, ...
// below `full_units` = (ceil(strips/grid) - 1) * grid.  The last
// `tail_strips` strips are cut either into `tail_bands` bands of
// `tail_band_rows` rows, these tail units, ordered (band, strip), dealt
// round-robin the same way, or into chunks of consecutive rows
// (`tail_chunk_rows`, see SegmentIter), whichever leaves the busiest CTA
// fewer rows to stream; either way CTAs running at the same moment work on
// neighbouring strips at the same rows.
// Per segment the producer (warp 0, one thread) streams input rows
// [p0 - pad, p0 - pad + rows + 2) as TMA boxes of (64 ch, 34 cols,
// stage_rows rows, 1 image) into an NS-deep shared-memory ring; box
// coordinates outside the image are zero-filled by the TMA unit, which
// implements the padding.  Four consumer warps each own 8 output columns.
// At 3x3 stride 1 a lane owns one 16-byte vector of 8 channels of two
// adjacent columns (ws_consumers_vec3x3: 16-byte shared-memory reads and
// 16-byte global stores); in the other geometries a lane owns one channel
// pair of all 8 columns (ws_consumers_pairs).  Either way every
// shared-memory read is conflict-free and each input row is read from shared
// memory once per lane and FMA'd into the accumulators of every output row it
// is a tap row of: a sliding window down the segment, so the vertical halo is
// never re-read.  A finished output row is rounded and stored with full
// 128-byte lines.
// ============================================================================
constexpr int kBlockC = 64;                        // channels per strip (128 B)
constexpr int kColsPerWarp = 8;                    // output columns per consumer warp
constexpr int kConsumerWarps = 4;
constexpr int kStripQ = kColsPerWarp * kConsumerWarps;  // 32 output columns
constexpr int kInCols = kStripQ + 2;               // 34 input columns per row
constexpr int kRowBytes = kInCols * kBlockC * 2;   // 4352 B per ring row
constexpr int kWsThreads = 32 * (1 + kConsumerWarps);

struct WsParams {
  const __half* w;
  __half* y;
  unsigned long long* stall;  // probe only
  const __half* bias;         // kModeEpilogue only: [C] or null
  const __half* residual;     // kModeEpilogue only: [N,P,Q,C] or null
  int32_t act;                // kModeEpilogue only: TDC_ACT_*
  int32_t flip_taps;          // kModeGeneral / kModeEpilogue: use w[2-r][2-s] (data gradient)
  int32_t H, W, C, P, Q, pad;
  int32_t pad_w;  // column offset (the left padding); pad is the row offset (top)
  int32_t qstrips, cblocks, stage_rows;
  int32_t tail_bands, tail_band_rows;
  int64_t full_units;   // strips handed out whole (a multiple of gridDim.x)
  int64_t tail_strips;  // strips handed out as bands or chunks
  uint64_t timeout_ns;
  int* status_host;     // this device's failure slot in mapped host memory, or null
  int64_t withhold;     // load index the producer withholds (-1: none)
  // > 0: the tail is cut into chunks of this many rows instead of bands (see
  // SegmentIter); requires gridDim.x % cblocks == 0.
  int32_t tail_chunk_rows;
  // Dilation D (forward; read only by the kernels instantiated with DIL,
  // which the host launches with D > 1 only).  With
  // D > 1, tap (r, s) of output (p, q) reads input (S*p + D*r - pad,
  // S*q + D*s - pad_w).  The outputs split into the D*D phases (p mod D,
  // q mod D); on phase (a, b) the outputs D apart read inputs D apart, an
  // undilated problem on the D-strided sub-lattice of x, which the tensor
  // map loads with traversal stride D.  The kernel then runs the undilated
  // schedule over N*D*D "images" (image n, phase a*D + b) of P x Q = the
  // largest phase's ceil(yP/D) x ceil(yQ/D) outputs, yP x yQ being y's rows
  // and columns.
  int32_t dil;
  int32_t yP, yQ;
};

// Per-device failure record written by the bounded waits:
// {code, block, stage, load index}.  The first failure on the device (until
// the host clears it) is also written through to `host`, the device's slot
// in a page of mapped pinned host memory, code last: the library reads that
// slot at the start of every later call, without synchronising, and fails
// the call while a failure is recorded.  `host` is null when the page does
// not exist (the allocation-free entry point never creates it).
__device__ int g_tdc_status[4];

__device__ __forceinline__ void record_failure(int code, int block, int stage, int64_t load,
                                               int* host) {
  if (atomicCAS(&g_tdc_status[0], 0, code) == 0) {
    g_tdc_status[1] = block;
    g_tdc_status[2] = stage;
    g_tdc_status[3] = int(load);
    if (host != nullptr) {
      volatile int* h = host;
      h[1] = block;
      h[2] = stage;
      h[3] = int(load);
      __threadfence_system();
      h[0] = code;
    }
  }
}

// A run of output rows [p0, p0 + rows) of one strip; with dilation, of
// phase (pa, pb) of image n.
struct Segment {
  int n, qs, cb, p0, rows;
  int pa, pb;
};

// Enumerates the segments of one CTA; the producer and every consumer warp
// run their own copy and see the same sequence.
//
// Tail by chunks (tail_chunk_rows = L > 0).  The tail strips form
// tail_strips / cblocks pixel strips (the cblocks channel blocks of one
// image's column strip); their rows, pixel strip after pixel strip, make one
// sequence of (tail_strips / cblocks) * P rows.  CTA g of the grid takes
// channel block g % cblocks of rows [k*L, (k+1)*L) of that sequence, k =
// g / cblocks: one or a few segments (one per pixel strip the chunk
// touches).  The cblocks CTAs of a chunk stream the same rows of the same
// pixels at the same time, as the channel-block-fastest strip order does for
// whole strips, and every CTA streams at most L rows plus two halo rows per
// segment, however the tail's rows divide by the grid.
//
// Dilation (p.dil = D > 1): strips run over N*D*D images of the largest
// phase's size; a phase with fewer rows clips its segments, and segments
// left empty are skipped.
struct SegmentIter {
  int64_t next;  // next work item: whole strips first, then tail units
  int64_t grid;
  int row = -1;  // chunk tail: next row of this CTA's chunk (-1: not started)

  __device__ SegmentIter(int64_t g, int64_t grid_) : next(g), grid(grid_) {}

  // kDilated: the dilated instantiations (p.dil > 1).
  template <bool kDilated = false>
  __device__ bool next_segment(const WsParams& p, Segment& s) {
    for (;;) {
      if (!next_unit(p, s)) return false;
      if (!kDilated) {
        s.pa = 0;
        s.pb = 0;
        return true;
      }
      const int D = p.dil;
      const int ph = s.n % (D * D);
      s.n /= D * D;
      s.pa = ph / D;
      s.pb = ph - s.pa * D;
      s.rows = min(s.rows, (p.yP - s.pa + D - 1) / D - s.p0);
      if (s.rows > 0) return true;
    }
  }

  __device__ bool next_unit(const WsParams& p, Segment& s) {
    int64_t strip;
    int first, last;
    if (next < p.full_units) {
      strip = next;
      first = 0;
      last = p.P;
      next += grid;
    } else if (p.tail_chunk_rows > 0) {
      // next stays at full_units + blockIdx.x; the host keeps the tail's rows
      // below 2^31.
      const int g = int(next - p.full_units);
      const int chunk = g / p.cblocks;
      const int total = int((p.tail_strips / p.cblocks) * p.P);
      const int end = chunk < int(grid) / p.cblocks ? min((chunk + 1) * p.tail_chunk_rows, total) : 0;
      if (row < 0) row = min(chunk * p.tail_chunk_rows, end);
      if (row >= end) return false;
      const int ps = row / p.P;  // pixel strip of the tail
      first = row - ps * p.P;
      last = min(p.P, first + (end - row));
      row += last - first;
      strip = p.full_units + int64_t(ps) * p.cblocks + g % p.cblocks;
    } else {
      const int64_t t = next - p.full_units;
      if (t >= p.tail_strips * p.tail_bands) return false;
      const int band = int(t / p.tail_strips);
      strip = p.full_units + t % p.tail_strips;
      first = band * p.tail_band_rows;
      last = min(p.P, first + p.tail_band_rows);
      next += grid;
    }
    s.cb = int(strip % p.cblocks);
    const int64_t r = strip / p.cblocks;
    s.qs = int(r % p.qstrips);
    s.n = int(r / p.qstrips);
    s.p0 = first;
    s.rows = last - first;
    return true;
  }
};

// Accumulators of one output row for one lane: kColsPerWarp columns x 2 channels.
struct RowAcc {
  float v[kColsPerWarp * 2];
};

// Fused epilogue of the general forward, per output (fp32 throughout, one
// rounding to fp16 at the end):
//   t = acc; t += bias[c]; t = act(t); t += residual[n,p,q,c]
// relu: t < 0 ? +0 : t;  relu6: min(relu(t), 6) (both exact);
// silu: t / (1 + exp(-t)) with the fast exp and divide intrinsics (a few fp32
// ulp, far below the fp16 rounding of the result); hardswish:
// t * clamp(t + 3, 0, 6) / 6 with a rounded multiply and an IEEE division
// (exact restatement in the oracle).
__device__ __forceinline__ float apply_act(float t, int act) {
  if (act == TDC_ACT_RELU) return t < 0.f ? 0.f : t;
  if (act == TDC_ACT_RELU6) return t < 0.f ? 0.f : (t > 6.f ? 6.f : t);
  if (act == TDC_ACT_SILU) return __fdividef(t, 1.f + __expf(-t));
  if (act == TDC_ACT_HARDSWISH) {
    float h = t + 3.f;
    h = h < 0.f ? 0.f : (h > 6.f ? 6.f : h);
    return (t * h) / 6.f;  // IEEE division: the oracle's arithmetic, bit for bit
  }
  return t;
}

// Kernel variants.
constexpr int kModeWs = 0;        // the reference surface: C % 64, plain output
constexpr int kModeGeneral = 1;   // C % 8 (partial last channel block), optional flipped taps
constexpr int kModeEpilogue = 2;  // kModeGeneral + bias / activation / residual
// kModeEpilogueAct + TDC_ACT_*: kModeEpilogue with the activation fixed at
// compile time (the 3x3 stride-1 fp16 forward), so the per-row epilogue
// carries no dispatch on it.
constexpr int kModeEpilogueAct = 16;
__host__ __device__ constexpr bool epilogue_mode(int mode) {
  return mode == kModeEpilogue || mode >= kModeEpilogueAct;
}

__host__ __device__ constexpr int pmod(int a, int b) { return ((a % b) + b) % b; }

// Output rows per pass of the direct scheme, measured at 64 x 224 x 336 x 256
// (5x5: 1 / 3 / 4 rows = 1.96 / 1.61 / 1.57 ms; 7x7: 1 / 2 / 3 / 4 rows =
// 3.01 / 2.71 / 2.96 / 3.80 ms).  Stride 2 keeps one: two rows need a 9-row
// window for 7x7, whose ring then allows only one CTA per SM (1.0 -> 1.5 ms).
__host__ __device__ constexpr int direct_rows(int K, int S) {
  return S == 2 ? 1 : (K <= 5 ? 3 : 2);
}

// Geometry of a K x K, stride-S depthwise kernel over one 32-column strip.
// Output column q reads input columns S*q - pad + s (s < K); output row p
// reads input rows S*p - pad + r (r < K).
template <int K, int S>
struct Geom {
  static constexpr int kWarpIn = S * (kColsPerWarp - 1) + K;  // input columns one warp reads
  static constexpr int kStripIn = S * (kStripQ - 1) + K;      // input columns of a strip (TMA box)
  static constexpr int kRowB = kStripIn * kBlockC * 2;        // bytes of one ring row
  // Output rows an input row can touch; they cycle through kNacc accumulator
  // sets, and the row loop is unrolled by kPeriod = S * kNacc input rows so
  // every set index is a compile-time constant.
  static constexpr int kNacc = (K + S - 1) / S;
  static constexpr int kPeriod = S * kNacc;
  // Consumer scheme.  Sliding window: every input row is read from shared
  // memory once and fed into the kNacc output rows it belongs to; the K*K
  // packed tap pairs and kNacc accumulator sets live in registers.  When
  // they do not fit (5x5 stride 1, 7x7) the direct scheme is used instead:
  // one output row at a time from its K input rows (read K / S times each),
  // one accumulator set, taps in registers.
  static constexpr bool kDirect = K * K + kNacc * 2 * kColsPerWarp + kWarpIn > 100;
  // Direct scheme: output rows per pass, and the input rows a pass holds.
  // The ring's stage height sr must satisfy (NS - 1) * sr >= kWindow - 1
  // (checked by the host planner).
  static constexpr int kRows = direct_rows(K, S);
  static constexpr int kWindow = S * (kRows - 1) + K;
  static_assert(kStripIn <= 256, "TMA box dimension");
};
static_assert(Geom<3, 1>::kRowB == kRowBytes, "3x3 stride-1 ring row");

// Geom<K, S>::kDirect and kWindow for run-time K and S (host planner).
__host__ __device__ constexpr bool direct_scheme(int K, int S) {
  return K * K + ((K + S - 1) / S) * 2 * kColsPerWarp + (S * (kColsPerWarp - 1) + K) > 100;
}
__host__ __device__ constexpr int direct_window(int K, int S) {
  return S * (direct_rows(K, S) - 1) + K;
}
static_assert(!direct_scheme(3, 1) && !direct_scheme(3, 2) && !direct_scheme(5, 2) &&
                  direct_scheme(5, 1) && direct_scheme(7, 1) && direct_scheme(7, 2),
              "consumer scheme per geometry");
static_assert(direct_window(7, 1) == Geom<7, 1>::kWindow && direct_window(7, 2) == Geom<7, 2>::kWindow &&
                  direct_window(5, 1) == Geom<5, 1>::kWindow,
              "host and device windows agree");

// Feeds input row u (mod the unroll period) — kWarpIn packed fp16 pairs of
// this lane — into the accumulator sets of every output row it is a tap row
// r of: the set of output o = (row - r) / S.  A set is initialised from +0
// by the first tap (r = 0, s = 0) of each of its outputs.  Within a row,
// inputs are consumed left to right, so every output sees its taps in (r, s)
// lexicographic order.  The FMAs take the fp16 operands directly
// (fma.rn.f32.f16), issuing on both FMA pipes with no conversion instruction.
template <int K, int S, int U, class E>
__device__ __forceinline__ void feed_row(const uint32_t (&xr)[Geom<K, S>::kWarpIn],
                                         const uint32_t (&wt)[K * K],
                                         RowAcc (&acc)[Geom<K, S>::kNacc]) {
  using G = Geom<K, S>;
#pragma unroll
  for (int j = 0; j < G::kWarpIn; ++j) {
#pragma unroll
    for (int s = 0; s < K; ++s) {
      if ((j - s) < 0 || (j - s) % S != 0) continue;
      const int m = (j - s) / S;
      if (m >= kColsPerWarp) continue;
#pragma unroll
      for (int r = 0; r < K; ++r) {
        if (pmod(U - r, S) != 0) continue;
        const int set = pmod((U - r - pmod(U - r, S)) / S, G::kNacc);
        RowAcc& a = acc[set];
        if (r == 0 && s == 0) {
          a.v[2 * m] = 0.f;
          a.v[2 * m + 1] = 0.f;
        }
        fma2<E>(xr[j], wt[r * K + s], a.v[2 * m], a.v[2 * m + 1]);
      }
    }
  }
}

// 16 fp32 values of 8 channels c .. c+7 (a 16-byte vector of fp16 or bf16
// elements): acc[2k], acc[2k+1] += x.(word k) * w.(word k).
template <class E>
__device__ __forceinline__ void fma_vec8(const uint4& x, const uint4& w, float* a) {
  fma2<E>(x.x, w.x, a[0], a[1]);
  fma2<E>(x.y, w.y, a[2], a[3]);
  fma2<E>(x.z, w.z, a[4], a[5]);
  fma2<E>(x.w, w.w, a[6], a[7]);
}

template <class E>
__device__ __forceinline__ uint4 pack_vec8(const float* a) {
  return make_uint4(pack2_rn<E>(a[0], a[1]), pack2_rn<E>(a[2], a[3]), pack2_rn<E>(a[4], a[5]),
                    pack2_rn<E>(a[6], a[7]));
}

// Consumer warps of the 3x3 stride-1 kernel, with 16-byte lanes.
//
// Lane l of consumer warp cw owns the 8 channels c0 + 8*(l % 8) .. + 7 (one
// 16-byte vector) of two adjacent output columns, q_first + 2*(l / 8) and the
// next, q_first being the first of the warp's 8 columns.  Per input row the
// lane reads the four input columns those outputs need as 16-byte vectors (a
// warp instruction reads four 128-byte column blocks of the ring row:
// conflict-free) and FMAs them into the three output rows the input row is tap
// row r = 2, 1, 0 of: 3 rotating sets x 2 columns x 8 channels of fp32
// accumulators, a sliding window down the segment, so vertical halo rows are
// never re-read.  A finished output row is rounded and stored with one
// 16-byte store per column (a warp instruction writes four full 128-byte
// lines).  Each output's chain is (r, s) lexicographic from +0, the same as
// every other kernel here.
template <int NS, bool PROBE, int MODE, class E, bool DIL>
__device__ __forceinline__ void ws_consumers_vec3x3(const WsParams& p, const uint8_t* ring_ptr,
                                                    uint32_t stage_bytes, uint64_t* full_bar,
                                                    uint64_t* empty_bar, volatile int* abort_flag,
                                                    int cw, int lane, uint64_t t_start) {
  constexpr int kVecPerCol = kBlockC * 2 / 16;  // 16-byte vectors per column of a ring row
  const int vl = lane & 7;                      // this lane's vector of the channel block
  const int cp = lane >> 3;                     // this lane's column pair of the warp's 8
  uint64_t stall_cycles = 0;
  uint32_t stage = 0, phase = 0;
  SegmentIter it(blockIdx.x, gridDim.x);
  Segment sg;
  int last_cb = -1;
  uint4 wt[9];
  float acc[3][16];
#pragma unroll
  for (int a = 0; a < 3; ++a)
#pragma unroll
    for (int k = 0; k < 16; ++k) acc[a][k] = 0.f;
  bool failed = false;
  while (!failed && it.next_segment<DIL>(p, sg)) {
    const int rows_in = sg.rows + 2;
    const int c0 = sg.cb * kBlockC;
    const int cl = c0 + 8 * vl;  // this lane's first channel
    const int q_first = sg.qs * kStripQ + cw * kColsPerWarp;
    // Dilation D (DIL only): this phase has ceil((yQ - pb) / D) output
    // columns.
    const int D = DIL ? p.dil : 1;
    const int qn = DIL ? (p.yQ - sg.pb + D - 1) / D : p.Q;
    const int n_valid = min(kColsPerWarp, qn - q_first);  // <= 0: warp idle
    // This lane's 8 channels exist (always on the ws path, C % 64 == 0; else
    // C % 8 == 0, so a vector is wholly inside C or wholly outside).
    const bool chan_ok = MODE == kModeWs || cl < p.C;
    if (sg.cb != last_cb) {
#pragma unroll
      for (int k = 0; k < 9; ++k) {
        const int src = (MODE != kModeWs && p.flip_taps) ? 8 - k : k;
        wt[k] = chan_ok ? __ldg(reinterpret_cast<const uint4*>(p.w + int64_t(src) * p.C + cl))
                        : make_uint4(0u, 0u, 0u, 0u);
      }
      last_cb = sg.cb;
    }
    // Output (p0 + o, q) of the segment is y's row pa + D*(p0 + o), column
    // pb + D*q.  The column step D*C (< 2^31, checked by the host) is
    // recomputed from the parameters where it is used.
    const int64_t y_off =
        DIL ? ((int64_t(sg.n) * p.yP + sg.pa + int64_t(D) * sg.p0) * p.yQ + sg.pb +
               int64_t(D) * (q_first + 2 * cp)) * p.C + cl
            : ((int64_t(sg.n) * p.P + sg.p0) * p.Q + q_first + 2 * cp) * p.C + cl;
    const int64_t y_row_stride = DIL ? int64_t(D) * p.yQ * p.C : int64_t(p.Q) * p.C;
    auto y_col = [&]() { return DIL ? p.dil * p.C : p.C; };
    const bool st0 = chan_ok && 2 * cp < n_valid;
    const bool st1 = chan_ok && 2 * cp + 1 < n_valid;

    // Finishes output row o of the segment from the accumulators a[0..15]
    // (column 2*cp at a[0..7], the next at a[8..15]) and stores it.
    auto store_row = [&](int o, float* a) {
      if constexpr (epilogue_mode(MODE)) {
        if (p.bias != nullptr && chan_ok) {
          // Reloaded per row (an L1 hit) rather than held in 8 registers.
          // t += b as fma(b, 1, t) on the packed 16-bit values: b * 1 is
          // exact, so this is the fp32 add, with no conversion instruction.
          const uint4 bv = __ldg(reinterpret_cast<const uint4*>(p.bias + cl));
          const uint32_t b4[4] = {bv.x, bv.y, bv.z, bv.w};
#pragma unroll
          for (int k = 0; k < 4; ++k) {
            fma2<E>(b4[k], ones2<E>(), a[2 * k], a[2 * k + 1]);
            fma2<E>(b4[k], ones2<E>(), a[8 + 2 * k], a[8 + 2 * k + 1]);
          }
        }
        switch (MODE >= kModeEpilogueAct ? MODE - kModeEpilogueAct : p.act) {
          case TDC_ACT_RELU:
#pragma unroll
            for (int k = 0; k < 16; ++k) a[k] = apply_act(a[k], TDC_ACT_RELU);
            break;
          case TDC_ACT_RELU6:
#pragma unroll
            for (int k = 0; k < 16; ++k) a[k] = apply_act(a[k], TDC_ACT_RELU6);
            break;
          case TDC_ACT_SILU:
#pragma unroll
            for (int k = 0; k < 16; ++k) a[k] = apply_act(a[k], TDC_ACT_SILU);
            break;
          case TDC_ACT_HARDSWISH:
#pragma unroll
            for (int k = 0; k < 16; ++k) a[k] = apply_act(a[k], TDC_ACT_HARDSWISH);
            break;
          default:
            break;
        }
        if (p.residual != nullptr) {
          // Loaded here, after the FMAs, rather than held through them (the
          // preloaded version spilled at the register limit); added as
          // fma(r, 1, t), like the bias.
          const __half* rp = p.residual + y_off + int64_t(o) * y_row_stride;
          const uint4 res[2] = {
              st0 ? __ldg(reinterpret_cast<const uint4*>(rp)) : make_uint4(0u, 0u, 0u, 0u),
              st1 ? __ldg(reinterpret_cast<const uint4*>(rp + y_col())) : make_uint4(0u, 0u, 0u, 0u)};
#pragma unroll
          for (int m = 0; m < 2; ++m) {
            const uint32_t w4[4] = {res[m].x, res[m].y, res[m].z, res[m].w};
#pragma unroll
            for (int k = 0; k < 4; ++k) fma2<E>(w4[k], ones2<E>(), a[8 * m + 2 * k], a[8 * m + 2 * k + 1]);
          }
        }
      }
      __half* dst = p.y + y_off + int64_t(o) * y_row_stride;
      if (st0) *reinterpret_cast<uint4*>(dst) = pack_vec8<E>(a);
      if (st1) *reinterpret_cast<uint4*>(dst + y_col()) = pack_vec8<E>(a + 8);
    };

    int lr = 0;  // row within the current stage
    const uint8_t* sbuf = ring_ptr;

    // One input row i (= U mod 3): acquire its stage, feed it, store the
    // output row it completes (i - 2), release the stage after its last row.
    auto step = [&](int i, auto u_tag) {
      constexpr int U = decltype(u_tag)::value;
      if (lr == 0) {
        [[maybe_unused]] uint64_t t0 = 0;
        if constexpr (PROBE) t0 = clock64();
        const bool got = mbar_wait_bounded(smem_addr(&full_bar[stage]), phase, abort_flag, true,
                                           p.timeout_ns);
        // Keep the warp uniform: one lane giving up makes the whole warp give up.
        if (__any_sync(0xffffffffu, !got)) {
          if (lane == 0 && !*abort_flag) {
            record_failure(TDC_DEVICE_FULL_TIMEOUT, blockIdx.x, stage, -1, p.status_host);
            *abort_flag = 1;
          }
          failed = true;
          return;
        }
        if constexpr (PROBE) stall_cycles += clock64() - t0;
        sbuf = ring_ptr + stage * stage_bytes;
      }
      if (n_valid > 0) {
        const uint4* src = reinterpret_cast<const uint4*>(
                               sbuf + lr * kRowBytes + (cw * kColsPerWarp + 2 * cp) * (kBlockC * 2)) +
                           vl;
        uint4 xr[4];
#pragma unroll
        for (int j = 0; j < 4; ++j) xr[j] = src[j * kVecPerCol];
#pragma unroll
        for (int j = 0; j < 4; ++j)
#pragma unroll
          for (int s = 0; s < 3; ++s) {
            const int m = j - s;  // output column (of the lane's two) input column j is tap s of
            if (m < 0 || m > 1) continue;
#pragma unroll
            for (int r = 0; r < 3; ++r) {
              float* a = acc[(U - r + 3) % 3] + 8 * m;  // the output row i - r
              if (r == 0 && s == 0) {
#pragma unroll
                for (int k = 0; k < 8; ++k) a[k] = 0.f;
              }
              fma_vec8<E>(xr[j], wt[r * 3 + s], a);
            }
          }
        if (i >= 2) store_row(i - 2, acc[(U + 1) % 3]);
      }
      if (++lr == p.stage_rows || i == rows_in - 1) {
        __syncwarp();
        if (lane == 0) mbar_arrive(smem_addr(&empty_bar[stage]));
        lr = 0;
        if (++stage == NS) { stage = 0; phase ^= 1u; }
      }
    };

    for (int i0 = 0; i0 < rows_in; i0 += 3) {
      bool stop = false;
      unroll_steps<3>([&](auto u_tag) {
        constexpr int U = decltype(u_tag)::value;
        if (stop) return;
        const int i = i0 + U;
        if (i >= rows_in) { stop = true; return; }
        step(i, u_tag);
        if (failed) stop = true;
      });
      if (stop) break;
    }
  }
  if constexpr (PROBE) {
    if (lane == 0) {
      unsigned long long* row = p.stall + 4ull * blockIdx.x;
      atomicAdd(row + 1, (unsigned long long)stall_cycles);
      atomicAdd(row + 3, (unsigned long long)(clock64() - t_start));
    }
  } else {
    (void)t_start;
  }
}

// Registers per thread of the ws kernels: 128, so that 3 CTAs of 160 threads
// are resident per SM.  At 136 only 2 fit (ncu: occupancy limit by
// registers 2 blocks, 136 allocated per thread), which cost the 3x3 kernel
// with an epilogue a third of its rate; at 128 it spills a few words
// instead.
template <int K, int S>
__host__ __device__ constexpr int ws_max_regs() {
  return 128;
}

template <int NS, bool PROBE, int MODE, int K, int S, class E, bool DIL>
__device__ __forceinline__ void ws_consumers_pairs(const WsParams& p, const uint8_t* ring_ptr,
                                                   uint32_t stage_bytes, uint64_t* full_bar,
                                                   uint64_t* empty_bar, volatile int* abort_flag,
                                                   int cw, int lane, uint64_t t_start);

// MODE (kMode*): kModeGeneral lets the last 64-channel block be partial (TMA
// zero-fills the missing channels; their lanes neither read taps nor store)
// and can flip the taps (the data gradient); kModeEpilogue adds the fused
// epilogue.  kModeWs is the ws call of the reference surface (3x3, stride 1).
// E (F16 / BF16) is the element type; the ws surface is fp16 only.
template <int NS, bool PROBE, int MODE = kModeWs, int K = 3, int S = 1, class E = F16, bool DIL = false>
__global__ void __maxnreg__((ws_max_regs<K, S>()))
    dwconv_ws_kernel(const __grid_constant__ CUtensorMap tmap, const __grid_constant__ WsParams p) {
  using G = Geom<K, S>;
  static_assert(MODE != kModeWs || (K == 3 && S == 1), "the ws surface is 3x3, stride 1");
  static_assert(MODE != kModeWs || std::is_same_v<E, F16>, "the ws surface is fp16");
  static_assert(!DIL || (MODE != kModeWs && !PROBE), "dilation: general forward modes only");
  __shared__ __align__(8) uint64_t full_bar[NS];
  __shared__ __align__(8) uint64_t empty_bar[NS];
  __shared__ volatile int abort_flag;
  extern __shared__ uint8_t dyn_smem[];
  // TMA destinations: 128-byte aligned ring of NS stages.
  const uint32_t ring = (smem_addr(dyn_smem) + 127u) & ~127u;
  const uint8_t* ring_ptr = dyn_smem + (ring - smem_addr(dyn_smem));
  const uint32_t stage_bytes = uint32_t(p.stage_rows) * G::kRowB;

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;

  uint64_t t_start = 0;
  if constexpr (PROBE) t_start = clock64();

  if (threadIdx.x == 0) {
#pragma unroll
    for (int s = 0; s < NS; ++s) {
      mbar_init(smem_addr(&full_bar[s]), 1);
      mbar_init(smem_addr(&empty_bar[s]), kConsumerWarps);
    }
    abort_flag = 0;
    fence_mbar_init();
    prefetch_tensormap(&tmap);
  }
  __syncthreads();
  // Launched with programmatic stream serialization: the set-up above may
  // overlap the previous kernel on the stream; global memory waits for it.
  // The next launch is released implicitly as each CTA exits (releasing it
  // early, with griddepcontrol.launch_dependents here, slowed the
  // 64 x 224 x 336 x 256 call from ~815 to ~910 us).
  griddep_wait();

  if (warp == 0) {
    // ------------------------------ producer ------------------------------
    if (lane != 0) return;
    uint64_t stall_cycles = 0;
    uint32_t stage = 0, phase = 0;
    uint32_t armed = 0, armed_parity = 0;  // bit s: stage s has a copy in flight / landed
    int64_t load = 0;
    bool ok = true;
    SegmentIter it(blockIdx.x, gridDim.x);
    Segment sg;
    while (ok && it.next_segment<DIL>(p, sg)) {
      const int rows_in = S * (sg.rows - 1) + K;
      const int nst = (rows_in + p.stage_rows - 1) / p.stage_rows;
      const int32_t c0 = sg.cb * kBlockC;
      // First input column and row of the segment; a stage of the ring
      // holds stage_rows rows, D apart (D = 1 without dilation).
      const int32_t D = DIL ? p.dil : 1;
      const int32_t w0 = S * sg.pb - p.pad_w + D * S * sg.qs * kStripQ;
      const int32_t h0 = S * sg.pa - p.pad + D * S * sg.p0;
      for (int t = 0; t < nst; ++t) {
        const uint32_t eb = smem_addr(&empty_bar[stage]);
        [[maybe_unused]] uint64_t t0 = 0;
        if constexpr (PROBE) t0 = clock64();
        if (!mbar_wait_bounded(eb, phase ^ 1u, &abort_flag, true, p.timeout_ns)) {
          if (!abort_flag) {
            record_failure(TDC_DEVICE_EMPTY_TIMEOUT, blockIdx.x, stage, load, p.status_host);
            abort_flag = 1;
          }
          ok = false;
          break;
        }
        if constexpr (PROBE) stall_cycles += clock64() - t0;
        if (load != p.withhold) {
          const uint32_t fb = smem_addr(&full_bar[stage]);
          mbar_arrive_expect_tx(fb, stage_bytes);
          tma_load_4d(ring + stage * stage_bytes, &tmap, fb, c0, w0, h0 + D * t * p.stage_rows, sg.n);
          armed |= 1u << stage;
          armed_parity = (armed_parity & ~(1u << stage)) | (phase << stage);
        } else {
          armed &= ~(1u << stage);
        }
        ++load;
        if (++stage == NS) { stage = 0; phase ^= 1u; }
      }
    }
    // Never leave the CTA while one of its copies may still write shared memory.
    for (int s = 0; s < NS; ++s) {
      if (!(armed & (1u << s))) continue;
      if (!mbar_wait_bounded(smem_addr(&full_bar[s]), (armed_parity >> s) & 1u, &abort_flag,
                             false, p.timeout_ns)) {
        record_failure(TDC_DEVICE_DRAIN_TIMEOUT, blockIdx.x, s, load, p.status_host);
      }
    }
    if constexpr (PROBE) {
      unsigned long long* row = p.stall + 4ull * blockIdx.x;
      atomicAdd(row + 0, (unsigned long long)stall_cycles);
      atomicAdd(row + 2, (unsigned long long)(clock64() - t_start));
    }
    return;
  }

  // ------------------------------ consumers ------------------------------
  if constexpr (K == 3 && S == 1) {
    ws_consumers_vec3x3<NS, PROBE, MODE, E, DIL>(p, ring_ptr, stage_bytes, full_bar, empty_bar,
                                            &abort_flag, warp - 1, lane, t_start);
    return;
  } else {
    ws_consumers_pairs<NS, PROBE, MODE, K, S, E, DIL>(p, ring_ptr, stage_bytes, full_bar, empty_bar,
                                                 &abort_flag, warp - 1, lane, t_start);
  }
}

// Consumer warps of the other geometries (3x3 stride 2, 5x5, 7x7): lane =
// channel pair, warp = 8 output columns; sliding window or direct scheme per
// Geom<K, S>::kDirect.
template <int NS, bool PROBE, int MODE, int K, int S, class E, bool DIL>
__device__ __forceinline__ void ws_consumers_pairs(const WsParams& p, const uint8_t* ring_ptr,
                                                   uint32_t stage_bytes, uint64_t* full_bar,
                                                   uint64_t* empty_bar, volatile int* abort_flag,
                                                   int cw, int lane, uint64_t t_start) {
  using G = Geom<K, S>;
  uint64_t stall_cycles = 0;
  uint32_t stage = 0, phase = 0;
  SegmentIter it(blockIdx.x, gridDim.x);
  Segment sg;
  int last_cb = -1;
  uint32_t wt[K * K];
  // Direct scheme: next ring stage to acquire / release, as slot and phase
  // (running counters, no division per pass).
  int acq_slot = 0, rel_slot = 0, seg_slot = 0;
  uint32_t acq_phase = 0;
  while (it.next_segment<DIL>(p, sg)) {
    const int rows_in = S * (sg.rows - 1) + K;
    const int c0 = sg.cb * kBlockC;
    const int q_first = sg.qs * kStripQ + cw * kColsPerWarp;
    // Dilation D (DIL only): this phase has ceil((yQ - pb) / D) output
    // columns.
    const int D = DIL ? p.dil : 1;
    const int qn = DIL ? (p.yQ - sg.pb + D - 1) / D : p.Q;
    const int n_valid = min(kColsPerWarp, qn - q_first);  // <= 0: warp idle
    // This lane's channel pair exists (always on the ws path, C % 64 == 0).
    const bool chan_ok = MODE == kModeWs || c0 + 2 * lane < p.C;
    if (sg.cb != last_cb) {
      const uint32_t* wp = reinterpret_cast<const uint32_t*>(p.w + c0) + lane;
#pragma unroll
      for (int k = 0; k < K * K; ++k) {
        const int src = (MODE != kModeWs && p.flip_taps) ? K * K - 1 - k : k;
        wt[k] = chan_ok ? __ldg(wp + int64_t(src) * (p.C / 2)) : 0u;
      }
      last_cb = sg.cb;
    }
    float bias0 = 0.f, bias1 = 0.f;
    if constexpr (epilogue_mode(MODE)) {
      if (p.bias != nullptr && chan_ok) {
        unpack2<E>(*reinterpret_cast<const uint32_t*>(p.bias + c0 + 2 * lane), bias0, bias1);
      }
    }
    // Output (p0 + o, q) of the segment is y's row pa + D*(p0 + o), column
    // pb + D*q.  The column step D*C (< 2^31, checked by the host) is
    // recomputed from the parameters where it is used.
    __half* yrow =
        p.y + c0 + 2 * lane +
        (DIL ? ((int64_t(sg.n) * p.yP + sg.pa + int64_t(D) * sg.p0) * p.yQ + sg.pb + int64_t(D) * q_first) * p.C
             : ((int64_t(sg.n) * p.P + sg.p0) * p.Q + q_first) * p.C);
    const int64_t y_row_stride = DIL ? int64_t(D) * p.yQ * p.C : int64_t(p.Q) * p.C;
    auto y_col = [&]() { return DIL ? p.dil * p.C : p.C; };

    bool failed = false;

    // Residual of output row o of the segment (epilogue only), fetched
    // before the FMAs that finish the row so its latency overlaps them.
    // The branch depends on kernel parameters only (warp-uniform).
    auto load_res = [&](int o, uint32_t (&res)[kColsPerWarp]) {
      if constexpr (epilogue_mode(MODE)) {
        if (p.residual != nullptr && chan_ok) {
          const __half* rrow = p.residual + ((yrow - p.y) + int64_t(o) * y_row_stride);
#pragma unroll
          for (int m = 0; m < kColsPerWarp; ++m)
            res[m] = m < n_valid ? __ldg(reinterpret_cast<const uint32_t*>(rrow + int64_t(m) * y_col()))
                                 : 0u;
        }
      }
    };

    // Stores output row o of the segment from accumulator set `fin`.
    auto store_row = [&](int o, RowAcc& fin, const uint32_t (&res)[kColsPerWarp]) {
      if constexpr (epilogue_mode(MODE)) {
        if (!chan_ok) return;
        float* t = fin.v;  // dead after this store: the set restarts from +0
        if (p.bias != nullptr) {
#pragma unroll
          for (int m = 0; m < kColsPerWarp; ++m) { t[2 * m] += bias0; t[2 * m + 1] += bias1; }
        }
        switch (p.act) {
          case TDC_ACT_RELU:
#pragma unroll
            for (int k = 0; k < 2 * kColsPerWarp; ++k) t[k] = apply_act(t[k], TDC_ACT_RELU);
            break;
          case TDC_ACT_RELU6:
#pragma unroll
            for (int k = 0; k < 2 * kColsPerWarp; ++k) t[k] = apply_act(t[k], TDC_ACT_RELU6);
            break;
          case TDC_ACT_SILU:
#pragma unroll
            for (int k = 0; k < 2 * kColsPerWarp; ++k) t[k] = apply_act(t[k], TDC_ACT_SILU);
            break;
          case TDC_ACT_HARDSWISH:
#pragma unroll
            for (int k = 0; k < 2 * kColsPerWarp; ++k) t[k] = apply_act(t[k], TDC_ACT_HARDSWISH);
            break;
          default:
            break;
        }
        if (p.residual != nullptr) {
#pragma unroll
          for (int m = 0; m < kColsPerWarp; ++m) {
            float r0, r1;
            unpack2<E>(res[m], r0, r1);
            t[2 * m] += r0;
            t[2 * m + 1] += r1;
          }
        }
      } else {
        (void)res;
      }
      if (!chan_ok) return;
      __half* dst = yrow + int64_t(o) * y_row_stride;
#pragma unroll
      for (int m = 0; m < kColsPerWarp; ++m)
        if (m < n_valid)
          *reinterpret_cast<uint32_t*>(dst + int64_t(m) * y_col()) =
              pack2_rn<E>(fin.v[2 * m], fin.v[2 * m + 1]);
    };

    if constexpr (G::kDirect) {
      // ---- direct scheme: R output rows o .. o+R-1 per pass, from input
      // rows S*o .. S*o + kWindow - 1 (kWindow = S*(R-1) + K) ----
      // Each input row of the pass is read from shared memory once and fed
      // to every output of the pass it is a tap row of.  Stage k of the
      // segment holds input rows [k*sr, (k+1)*sr) in ring slot
      // (seg_slot + k) % NS, so input row i sits at ring row
      // (seg_slot * sr + i) mod (NS * sr).  The warp holds the stages from
      // the first to the last input row of the pass; the host picks sr with
      // (NS - 1) * sr >= kWindow - 1 so that window always fits the ring.
      constexpr int R = G::kRows;
      const int sr = p.stage_rows;
      const int ring_rows = NS * sr;
      const int nst = (rows_in + sr - 1) / sr;
      int acquired = 0, released = 0;
      int acq_end = 0;   // input rows covered by the acquired stages
      int rel_end = sr;  // input rows up to the end of stage `released`
      int rr0 = seg_slot * sr;  // ring row of input row S*o
      for (int o = 0; o < sg.rows; o += R) {
        const int nout = min(R, sg.rows - o);  // outputs of this pass
        const int last_in = S * (o + nout - 1) + K - 1;
        while (acquired < nst && acq_end <= last_in) {
          [[maybe_unused]] uint64_t t0 = 0;
          if constexpr (PROBE) t0 = clock64();
          const bool got = mbar_wait_bounded(smem_addr(&full_bar[acq_slot]), acq_phase,
                                             abort_flag, true, p.timeout_ns);
          if (__any_sync(0xffffffffu, !got)) {
            if (lane == 0 && !*abort_flag) {
              record_failure(TDC_DEVICE_FULL_TIMEOUT, blockIdx.x, acq_slot, -1, p.status_host);
              *abort_flag = 1;
            }
            failed = true;
            break;
          }
          if constexpr (PROBE) stall_cycles += clock64() - t0;
          ++acquired;
          acq_end += sr;
          if (++acq_slot == NS) { acq_slot = 0; acq_phase ^= 1u; }
        }
        if (failed) break;
        if (n_valid > 0) {
          RowAcc a[R];
#pragma unroll
          for (int i = 0; i < G::kWindow; ++i) {
            // Rows past the segment's input (a short last pass) feed only
            // outputs that are not stored; skip them (warp-uniform).
            if (i >= K && i >= S * (nout - 1) + K) break;
            int rr = rr0 + i;
            if (rr >= ring_rows) rr -= ring_rows;
            const uint32_t* src = reinterpret_cast<const uint32_t*>(
                ring_ptr + rr * G::kRowB + (S * cw * kColsPerWarp) * (kBlockC * 2)) + lane;
            uint32_t xr[G::kWarpIn];
#pragma unroll
            for (int j = 0; j < G::kWarpIn; ++j) xr[j] = src[j * (kBlockC / 2)];
#pragma unroll
            for (int t = 0; t < R; ++t) {
              const int r = i - S * t;  // tap row of input row i for output o + t
              if (r < 0 || r >= K) continue;
#pragma unroll
              for (int s2 = 0; s2 < K; ++s2)
#pragma unroll
                for (int m = 0; m < kColsPerWarp; ++m) {
                  if (r == 0 && s2 == 0) { a[t].v[2 * m] = 0.f; a[t].v[2 * m + 1] = 0.f; }
                  fma2<E>(xr[S * m + s2], wt[r * K + s2], a[t].v[2 * m], a[t].v[2 * m + 1]);
                }
            }
          }
#pragma unroll
          for (int t = 0; t < R; ++t) {
            if (t >= nout) break;
            uint32_t res[kColsPerWarp];
            load_res(o + t, res);
            store_row(o + t, a[t], res);
          }
        }
        // Release the stages wholly below the first input row of the next pass.
        const int next_first = o + R >= sg.rows ? (1 << 30) : S * (o + R);
        if (released < nst && rel_end <= next_first) {
          __syncwarp();
          while (released < nst && rel_end <= next_first) {
            if (lane == 0) mbar_arrive(smem_addr(&empty_bar[rel_slot]));
            ++released;
            rel_end += sr;
            if (++rel_slot == NS) rel_slot = 0;
          }
        }
        rr0 += S * R;
        if (rr0 >= ring_rows) rr0 -= ring_rows;
      }
      if (failed) break;
      seg_slot = acq_slot;  // the next segment starts at a fresh stage
    } else {
      RowAcc acc[G::kNacc];
#pragma unroll
      for (int a = 0; a < G::kNacc; ++a)
#pragma unroll
        for (int k = 0; k < kColsPerWarp * 2; ++k) acc[a].v[k] = 0.f;

      int lr = 0;  // row within the current stage
      const uint8_t* sbuf = ring_ptr;

      // One input row i (= U mod the unroll period): acquire its stage, feed
      // it, store the output row it completes, release the stage after its
      // last row.
      auto step = [&](int i, auto u_tag) {
        constexpr int U = decltype(u_tag)::value;
        if (lr == 0) {
          [[maybe_unused]] uint64_t t0 = 0;
          if constexpr (PROBE) t0 = clock64();
          const bool got = mbar_wait_bounded(smem_addr(&full_bar[stage]), phase, abort_flag,
                                             true, p.timeout_ns);
          // Keep the warp uniform: one lane giving up makes the whole warp give up.
          if (__any_sync(0xffffffffu, !got)) {
            if (lane == 0 && !*abort_flag) {
              record_failure(TDC_DEVICE_FULL_TIMEOUT, blockIdx.x, stage, -1, p.status_host);
              *abort_flag = 1;
            }
            failed = true;
            return;
          }
          if constexpr (PROBE) stall_cycles += clock64() - t0;
          sbuf = ring_ptr + stage * stage_bytes;
        }
        if (n_valid > 0) {
          const uint32_t* src = reinterpret_cast<const uint32_t*>(
              sbuf + lr * G::kRowB + (S * cw * kColsPerWarp) * (kBlockC * 2)) + lane;
          uint32_t xr[G::kWarpIn];
#pragma unroll
          for (int j = 0; j < G::kWarpIn; ++j) xr[j] = src[j * (kBlockC / 2)];
          // The output whose last tap row (r = K-1) this row is, if any.
          constexpr bool kCompletes = pmod(U - (K - 1), S) == 0;
          uint32_t res[kColsPerWarp];
          if constexpr (kCompletes) {
            if (i >= K - 1) load_res((i - (K - 1)) / S, res);
          }
          feed_row<K, S, U, E>(xr, wt, acc);
          if constexpr (kCompletes) {
            if (i >= K - 1) {
              constexpr int kFin = pmod((U - (K - 1) - pmod(U - (K - 1), S)) / S, G::kNacc);
              store_row((i - (K - 1)) / S, acc[kFin], res);
            }
          }
        }
        if (++lr == p.stage_rows || i == rows_in - 1) {
          __syncwarp();
          if (lane == 0) mbar_arrive(smem_addr(&empty_bar[stage]));
          lr = 0;
          if (++stage == NS) { stage = 0; phase ^= 1u; }
        }
      };

      // Rows cycle through the accumulator sets; the loop is unrolled by the
      // period so every set index is resolved at compile time.
      for (int i0 = 0; i0 < rows_in; i0 += G::kPeriod) {
        bool stop = false;
        unroll_steps<G::kPeriod>([&](auto u_tag) {
          constexpr int U = decltype(u_tag)::value;
          if (stop) return;
          const int i = i0 + U;
          if (i >= rows_in) { stop = true; return; }
          step(i, u_tag);
          if (failed) stop = true;
        });
        if (stop) break;
      }
      if (failed) break;
    }
  }
  if constexpr (PROBE) {
    if (lane == 0) {
      unsigned long long* row = p.stall + 4ull * blockIdx.x;
      atomicAdd(row + 1, (unsigned long long)stall_cycles);
      atomicAdd(row + 3, (unsigned long long)(clock64() - t_start));
    }
  }
}

}  // namespace tdc
