// tdc_plain.cuh — plain K x K depthwise forward (K = 3, 5, 7, stride 1 or 2):
// global loads through L1, no shared memory, no TMA, no pipeline.
//
// The ws kernels tile the output in strips of 32 columns x 64 channels, so a
// layer with few channels (C = 16, 32, 72) or a narrow image (7 x 7, 14 x 14:
// the late stages of MobileNet / EfficientNet) leaves most lanes or most
// consumer warps of a strip without work, and its whole run is shorter than
// the persistent ring's set-up.  This kernel's tile is small: a thread owns
// one channel pair of plain_cols(K) consecutive output columns (8 for 3x3, 4
// for 5x5, 2 for 7x7) over a band of output rows.  Threads are dealt (channel pair
// within a chunk, column group, chunk, band, image), the chunk's pairs
// fastest, so a warp's loads and stores are whole 16- or 32-byte sectors and
// the column groups that share halo columns run in the same CTA (L1 hits).
//
// Per thread: the K*K packed tap pairs in registers; it slides down the band's
// input rows S*p0 - pad .. S*(p0 + rows - 1) - pad + K - 1, loading each row's
// S*(plain_cols(K) - 1) + K pairs once (one row ahead of their use) and feeding them
// to the ceil(K/S) output rows the row is a tap row of, exactly as the ws
// kernel's sliding window does: per output an fp32 chain from +0 in (r, s)
// order, the fused epilogue t = acc (+ bias) -> act -> (+ residual), one
// rounding.  The result is therefore bit-identical to the ws kernels and the
// oracle.
//
// Dilation (PlainParams::dil = D > 1, the atrous layers of segmentation
// backbones) runs on the same kernel: output rows and columns are split into
// the D*D phases (p mod D, q mod D); within a phase the outputs D apart read
// inputs D apart, i.e. an undilated problem on the D-strided sub-lattice of
// x, so a thread owns outputs D apart and its window steps D rows and columns
// at a time.  Each input element is then loaded once per thread window, as at
// D = 1, instead of once per tap (K*K loads per output, the first dilated
// kernel's scheme).
#pragma once

#include "tdc_kernels.cuh"

namespace tdc {

constexpr int kPlainThreads = 128;

// Output columns per thread: the accumulators (ceil(K/S) rows x kCols x 2),
// the K*K taps and two rows of inputs stay in registers without spilling.
__host__ __device__ constexpr int plain_cols(int K) { return K == 3 ? 8 : (K == 5 ? 4 : 2); }

struct PlainParams {
  const uint32_t* x;         // [N, H, W, C] as channel pairs
  const uint32_t* w;         // [K, K, C]
  const uint32_t* bias;      // [C] or null (epilogue only)
  const uint32_t* residual;  // [N, P, Q, C] or null (epilogue only)
  uint32_t* y;               // [N, P, Q, C]
  uint32_t total;            // threads of work: N * bands * chunks * qgroups * chunk_pairs
  int32_t H, W, P, Q;
  int32_t qgroups;           // ceil(Q / plain_cols(K))
  int32_t cpairs;            // C / 2
  int32_t chunk_log2;        // log2 of the channel pairs per chunk (2 or 3)
  int32_t chunks;            // cpairs >> chunk_log2
  int32_t bands, band_rows;
  int32_t pad;               // row offset (top padding); may be negative (a crop) for the
                             // flipped data gradient
  int32_t pad_w;             // column offset (left padding), likewise
  int32_t act;
  int32_t flip_taps;         // taps w[K-1-r][K-1-s] (data gradient of the stride-1 forward)
  // Dilation D (>= 1; 0 reads as 1): tap (r, s) of output (p, q) reads input
  // (S*p + D*r - pad, S*q + D*s - pad_w).  The outputs split into D*D phases
  // (p mod D, q mod D); on each, the outputs D apart read inputs D apart, an
  // undilated K x K stride-S problem on the D-strided sub-lattice of x, so a
  // thread's outputs are D apart and its sliding window steps D rows and
  // columns at a time.  bands / qgroups count the largest phase's
  // ceil(P/D) rows and ceil(Q/D) columns; phases = D*D threads' worth of them.
  int32_t dil;
  int32_t phases;
};

template <int K, int S, class E, bool EPI>
__global__ void __launch_bounds__(kPlainThreads) dwconv_plain_kernel(PlainParams p) {
  constexpr int A = (K + S - 1) / S;      // output rows an input row can touch
  constexpr int L = S * A;                // row-loop unroll: accumulator set indices are constants
  constexpr int QT = plain_cols(K);       // output columns per thread
  constexpr int NI = S * (QT - 1) + K;    // input columns per row
  static_assert(NI <= 32, "column mask");
  griddep_wait();                         // programmatic launch: the previous kernel's output is ready
  const uint32_t t = blockIdx.x * uint32_t(kPlainThreads) + threadIdx.x;
  if (t >= p.total) return;
  const uint32_t cmask = (1u << p.chunk_log2) - 1u;
  uint32_t r_ = t >> p.chunk_log2;
  const int qg = int(r_ % uint32_t(p.qgroups));   r_ /= uint32_t(p.qgroups);
  const int chunk = int(r_ % uint32_t(p.chunks)); r_ /= uint32_t(p.chunks);
  const int band = int(r_ % uint32_t(p.bands));   r_ /= uint32_t(p.bands);
  const int D = p.dil > 1 ? p.dil : 1;
  const uint32_t phases = p.phases > 1 ? uint32_t(p.phases) : 1u;
  const int ph = int(r_ % phases);
  const int n = int(r_ / phases);
  const int pa = ph / D, pb = ph - pa * D;  // this thread's output row / column phase
  const int cp = (chunk << p.chunk_log2) + int(t & cmask);
  const int p0 = band * p.band_rows;      // in rows of the phase
  const int rows = min(p.band_rows, (p.P - pa + D - 1) / D - p0);
  const int q0 = qg * QT;                 // in columns of the phase
  const int n_valid = min(QT, (p.Q - pb + D - 1) / D - q0);  // output columns of this thread
  if (rows <= 0 || n_valid <= 0) return;  // a phase smaller than the largest (D > 1 only)
  const int n_in = S * (rows - 1) + K;
  const int h0 = S * (pa + D * p0) - p.pad;    // input row of band row 0
  const int w0 = S * (pb + D * q0) - p.pad_w;  // input column of input j = 0

  uint32_t wt[K * K];
#pragma unroll
  for (int k = 0; k < K * K; ++k)
    wt[k] = __ldg(p.w + int64_t(p.flip_taps ? K * K - 1 - k : k) * p.cpairs + cp);
  float b0 = 0.f, b1 = 0.f;
  if constexpr (EPI) {
    if (p.bias != nullptr) unpack2<E>(__ldg(p.bias + cp), b0, b1);
  }
  uint32_t col_ok = 0;  // bit j: input column w0 + D*j is inside the image
#pragma unroll
  for (int j = 0; j < NI; ++j) col_ok |= (unsigned(w0 + D * j) < unsigned(p.W) ? 1u : 0u) << j;

  // Offsets within one image are 32-bit (the host checks H * W * C / 2 < 2^31).
  const uint32_t* xn = p.x + int64_t(n) * p.H * p.W * p.cpairs + cp;
  const uint32_t x_col = uint32_t(D * p.cpairs);           // between this thread's input columns
  const int64_t y_col = int64_t(D) * p.cpairs;             // ... and output columns
  const int64_t y_row = int64_t(D) * p.Q * p.cpairs;       // ... and output rows
  const int64_t y_off = (int64_t(n) * p.P + pa + int64_t(D) * p0) * p.Q * p.cpairs +
                        (pb + int64_t(D) * q0) * p.cpairs + cp;

  // The NI pairs of band input row i (zero outside the image).  The row test
  // is the same for every thread of a band; a column's offset is the
  // previous one plus D * C / 2.
  auto load_row = [&](int i, uint32_t (&v)[NI]) {
    const int h = h0 + D * i;
    if (unsigned(h) < unsigned(p.H)) {
      uint32_t off = uint32_t((h * p.W + w0) * p.cpairs);  // wraps below 0; used only when inside
#pragma unroll
      for (int j = 0; j < NI; ++j) {
        v[j] = ((col_ok >> j) & 1u) ? __ldg(xn + off) : 0u;
        off += x_col;
      }
    } else {
#pragma unroll
      for (int j = 0; j < NI; ++j) v[j] = 0u;
    }
  };

  auto store = [&](int o, float (&a)[QT][2]) {
#pragma unroll
    for (int m = 0; m < QT; ++m) {
      if (m >= n_valid) continue;
      float a0 = a[m][0], a1 = a[m][1];
      const int64_t off = y_off + int64_t(o) * y_row + int64_t(m) * y_col;
      if constexpr (EPI) {
        if (p.bias != nullptr) { a0 += b0; a1 += b1; }
        a0 = apply_act(a0, p.act);
        a1 = apply_act(a1, p.act);
        if (p.residual != nullptr) {
          float r0, r1;
          unpack2<E>(__ldg(p.residual + off), r0, r1);
          a0 += r0;
          a1 += r1;
        }
      }
      p.y[off] = pack2_rn<E>(a0, a1);
    }
  };

  float acc[A][QT][2];
  uint32_t xv[NI], xnext[NI];
  load_row(0, xv);
  // Input row i = i0 + U (i0 a multiple of L) is tap row r of output row
  // o = (i - r) / S whenever S divides i - r; that output's accumulator set
  // is ((U - r) / S) mod A, a compile-time constant.  Output column m reads
  // input j = S*m + s for tap s.
  auto step = [&](int i0, auto u_tag) {
    constexpr int U = decltype(u_tag)::value;
    const int i = i0 + U;
    if (i + 1 < n_in) load_row(i + 1, xnext);
#pragma unroll
    for (int r = 0; r < K; ++r) {
      if (pmod(U - r, S) != 0) continue;
      const int o = i0 / S + (U - r) / S;
      if (o < 0 || o >= rows) continue;
      float (&a)[QT][2] = acc[pmod((U - r) / S, A)];
      if (r == 0) {
#pragma unroll
        for (int m = 0; m < QT; ++m) { a[m][0] = 0.f; a[m][1] = 0.f; }
      }
#pragma unroll
      for (int m = 0; m < QT; ++m) {
#pragma unroll
        for (int s = 0; s < K; ++s) fma2<E>(xv[S * m + s], wt[r * K + s], a[m][0], a[m][1]);
      }
      if (r == K - 1) store(o, a);
    }
#pragma unroll
    for (int j = 0; j < NI; ++j) xv[j] = xnext[j];
  };
  for (int i0 = 0; i0 < n_in; i0 += L) {
    unroll_steps<L>([&](auto u_tag) {
      if (i0 + decltype(u_tag)::value < n_in) step(i0, u_tag);
    });
  }
}

// ============================================================================
// Plain weight gradient (K = 3, 5, 7, stride 1 or 2) for the same small
// shapes:  dw[r,s,c] = sum_{n,p,q} x[n, S*p+r-pad, S*q+s-pad, c] * dy[n,p,q,c].
//
// The ws-family weight gradients give every CTA a workspace slice of all C
// channels per consumer warp, which is cheap against a 5 GB input but not
// against a 12 MB one (7 x 7 x 960 at batch 64, 5x5: ~170 MB of partial sums
// for 12 MB of x and dy).  Here a CTA owns one tap row r (blockIdx.y), one
// channel chunk and kPlainThreads / chunk_pairs units (image, band of dy
// rows); a thread keeps the K sums of row r for one channel pair of one unit.
// The CTA adds its units up in a fixed order (a butterfly over the units of a
// warp, then the warps in order) and writes row r's taps of one slice of its
// chunk's channels.  The workspace is ugroups x K*K x C floats (ugroups =
// CTAs per chunk and row), and dwconv_wgrad_reduce_kernel sums the slices in
// a fixed order: deterministic, like the ws kernels.  Per dy row and 8-column
// chunk a thread loads the chunk's dy pairs and the S*7 + K x pairs of input
// row S*p + r - pad under them; each tap's sum takes the chunk's 8 products
// in column order.
// ============================================================================
constexpr int kWgradPlainCols = 8;  // dy columns per chunk

struct WgradPlainParams {
  const uint32_t* x;   // [N, H, W, C] as channel pairs
  const uint32_t* dy;  // [N, P, Q, C] as channel pairs
  float* partial;      // [ugroups][K*K][C]
  int32_t H, W, P, Q;
  int32_t cpairs, chunk_log2, chunks;
  int32_t bands, band_rows;
  int32_t units;       // N * bands
  int32_t pad;
};

template <int K, int S, class E>
__global__ void __launch_bounds__(kPlainThreads) dwconv_wgrad_plain_kernel(WgradPlainParams p) {
  constexpr int QC = kWgradPlainCols;
  constexpr int NI = S * (QC - 1) + K;  // x columns under one dy chunk
  constexpr int kWarps = kPlainThreads / 32;
  static_assert(NI <= 32, "column mask");
  __shared__ float red[kWarps][K * 2][8];
  griddep_wait();
  const int r = int(blockIdx.y);                  // tap row of this CTA
  const int cpc = 1 << p.chunk_log2;              // channel pairs per chunk
  const int upc = kPlainThreads >> p.chunk_log2;  // units per CTA
  const int chunk = int(blockIdx.x % uint32_t(p.chunks));
  const int ugroup = int(blockIdx.x / uint32_t(p.chunks));
  const int cp_in = int(threadIdx.x) & (cpc - 1);
  const int cp = chunk * cpc + cp_in;
  const int u = ugroup * upc + (int(threadIdx.x) >> p.chunk_log2);

  float acc[K][2];
#pragma unroll
  for (int s = 0; s < K; ++s) { acc[s][0] = 0.f; acc[s][1] = 0.f; }
  if (u < p.units) {
    const int n = u / p.bands;
    const int band = u - n * p.bands;
    const int p0 = band * p.band_rows;
    const int p1 = min(p.P, p0 + p.band_rows);
    const uint32_t* xn = p.x + int64_t(n) * p.H * p.W * p.cpairs + cp;
    const uint32_t* dyn = p.dy + int64_t(n) * p.P * p.Q * p.cpairs + cp;
    for (int pr = p0; pr < p1; ++pr) {
      const int h = S * pr + r - p.pad;
      if (unsigned(h) >= unsigned(p.H)) continue;  // the whole row is padding
      for (int q0 = 0; q0 < p.Q; q0 += QC) {
        uint32_t d[QC];
        uint32_t off = uint32_t((pr * p.Q + q0) * p.cpairs);
#pragma unroll
        for (int m = 0; m < QC; ++m) {
          d[m] = q0 + m < p.Q ? __ldg(dyn + off) : 0u;
          off += uint32_t(p.cpairs);
        }
        const int w0 = S * q0 - p.pad;
        uint32_t xv[NI];
        off = uint32_t((h * p.W + w0) * p.cpairs);  // wraps below 0; used only inside
#pragma unroll
        for (int j = 0; j < NI; ++j) {
          xv[j] = unsigned(w0 + j) < unsigned(p.W) ? __ldg(xn + off) : 0u;
          off += uint32_t(p.cpairs);
        }
#pragma unroll
        for (int s = 0; s < K; ++s) {
#pragma unroll
          for (int m = 0; m < QC; ++m) fma2<E>(xv[S * m + s], d[m], acc[s][0], acc[s][1]);
        }
      }
    }
  }
  // Fixed-order sum over the CTA's units: a butterfly over the units of a
  // warp (lanes cp_in + i * cpc), then warps 0 .. kWarps-1 in order.
  const int lane = int(threadIdx.x) & 31, warp = int(threadIdx.x) >> 5;
#pragma unroll
  for (int s = 0; s < K; ++s) {
#pragma unroll
    for (int c2 = 0; c2 < 2; ++c2) {
      float v = acc[s][c2];
      for (int off = 16; off >= cpc; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
      if (lane < cpc) red[warp][2 * s + c2][lane] = v;
    }
  }
  __syncthreads();
  if (threadIdx.x < unsigned(cpc)) {
    float* slice = p.partial + (int64_t(ugroup) * K * K + r * K) * (2 * p.cpairs) + 2 * cp;
#pragma unroll
    for (int s = 0; s < K; ++s) {
      float s0 = red[0][2 * s][cp_in], s1 = red[0][2 * s + 1][cp_in];
#pragma unroll
      for (int wi = 1; wi < kWarps; ++wi) {
        s0 += red[wi][2 * s][cp_in];
        s1 += red[wi][2 * s + 1][cp_in];
      }
      *reinterpret_cast<float2*>(slice + int64_t(s) * (2 * p.cpairs)) = make_float2(s0, s1);
    }
  }
}

}  // namespace tdc
