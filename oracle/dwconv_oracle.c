/*
 * dwconv_oracle.c — CPU oracle for the NHWC fp16 depthwise 3x3 conv2d forward.
 *
 * TEST INFRASTRUCTURE ONLY.  This file is the checker the parity tests, the
 * smoke test and the CPU-baseline leg of the benchmark compare the CUDA path
 * against; nothing in the shipped library links or calls it.
 *
 * It restates, on the CPU, the per-output arithmetic of the reference
 * kernels of haowen-han/tma-depthwise-conv:
 *   csrc/kernel_v0_naive_float4.cu:37-74   (acc[v] = 0; for r: for s:
 *                                          acc[v] += half2float(x)*half2float(w);
 *                                          y = __float2half(acc))
 *   csrc/kernel_tma_ws.cuh:218-246         (same chain over the smem tile)
 *   csrc/kernel_tma_ws.cu:382-385          (P = H + 2*pad - 3 + 1, Q likewise)
 *   csrc/kernel_tma_ws.cuh:148-149         (taps outside the image read 0:
 *                                          TMA out-of-bounds zero fill)
 * i.e. an fp32 multiply-add chain from +0 in r-major, s-minor order, then one
 * round-to-nearest-even to fp16.  Because the product of two fp16 values is
 * exact in fp32, acc + x*w and fmaf(x, w, acc) give the same bits; the
 * reference compiles `acc += a*b` to FFMA (nvcc --fmad=true), and this file
 * uses fmaf.
 *
 * fp16 <-> fp32 conversions are written out bit by bit below (IEEE 754
 * binary16, round-to-nearest-even, subnormals kept, overflow to infinity).
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>
#include <string.h>
#ifdef _OPENMP
#include <omp.h>
#endif

static float bits_to_f32(uint32_t b) { float f; memcpy(&f, &b, 4); return f; }
static uint32_t f32_to_bits(float f) { uint32_t b; memcpy(&b, &f, 4); return b; }

/* binary16 -> binary32, exact for every input. */
float oracle_f16_to_f32(uint16_t h) {
  const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
  const uint32_t e = (h >> 10) & 0x1fu;
  const uint32_t m = h & 0x3ffu;
  if (e == 0) {
    /* zero or subnormal: m * 2^-24, exact in binary32 */
    const float v = (float)m * 5.9604644775390625e-08f;
    return bits_to_f32(sign | f32_to_bits(v));
  }
  if (e == 31) return bits_to_f32(sign | 0x7f800000u | (m << 13)); /* inf / nan */
  return bits_to_f32(sign | ((e + 112u) << 23) | (m << 13));
}

/* binary32 -> binary16, round to nearest, ties to even. */
uint16_t oracle_f32_to_f16(float f) {
  const uint32_t x = f32_to_bits(f);
  const uint16_t sign = (uint16_t)((x >> 16) & 0x8000u);
  const uint32_t ax = x & 0x7fffffffu;
  if (ax >= 0x7f800000u) /* inf, nan (quiet, top payload bits kept) */
    return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? (0x200u | ((ax >> 13) & 0x3ffu)) : 0u));
  if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u); /* >= 65520 rounds to inf */
  if (ax >= 0x38800000u) {                                   /* normal fp16 range */
    const uint32_t mant = ax & 0x7fffffu;
    uint32_t h = ((((ax >> 23) & 0xffu) - 112u) << 10) | (mant >> 13);
    const uint32_t rem = mant & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) ++h; /* carry into exponent is correct */
    return (uint16_t)(sign | h);
  }
  if (ax <= 0x33000000u) return sign; /* <= 2^-25: rounds to (signed) zero */
  {
    /* subnormal result: count units of 2^-24 */
    const uint32_t e = (ax >> 23) & 0xffu;          /* 102 .. 112 */
    const uint32_t mfull = (ax & 0x7fffffu) | 0x800000u;
    const uint32_t shift = 126u - e;                /* 14 .. 24 */
    uint32_t h = mfull >> shift;
    const uint32_t rem = mfull & ((1u << shift) - 1u);
    const uint32_t half = 1u << (shift - 1u);
    if (rem > half || (rem == half && (h & 1u))) ++h;
    return (uint16_t)(sign | h);
  }
}

/* bfloat16 -> binary32: the top 16 bits of a binary32, exact. */
float oracle_bf16_to_f32(uint16_t b) { return bits_to_f32((uint32_t)b << 16); }

/* binary32 -> bfloat16, round to nearest, ties to even (infinities kept, a NaN
 * stays a quiet NaN of the same sign). */
uint16_t oracle_f32_to_bf16(float f) {
  uint32_t x = f32_to_bits(f);
  if ((x & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((x >> 16) | 0x40u);
  x += 0x7fffu + ((x >> 16) & 1u);
  return (uint16_t)(x >> 16);
}

/* Element codecs of the activations and filters: fp16 (the reference's) or
 * bf16.  Arithmetic is fp32 either way; products of two elements are exact. */
enum { CODEC_F16 = 0, CODEC_BF16 = 1 };

static void codec_lut(int codec, float* lut) {
  for (uint32_t i = 0; i < 65536u; ++i)
    lut[i] = codec == CODEC_BF16 ? oracle_bf16_to_f32((uint16_t)i) : oracle_f16_to_f32((uint16_t)i);
}

static uint16_t codec_round(int codec, float f) {
  return codec == CODEC_BF16 ? oracle_f32_to_bf16(f) : oracle_f32_to_f16(f);
}

/* Output size of a stride-1 3x3 conv with symmetric padding
 * (csrc/kernel_tma_ws.cu:384-385). */
void oracle_output_hw(int64_t H, int64_t W, int64_t pad, int64_t* P, int64_t* Q) {
  *P = H + 2 * pad - 3 + 1;
  *Q = W + 2 * pad - 3 + 1;
}

/* Activation codes of the general forward's fused epilogue. */
enum { ORACLE_ACT_NONE = 0, ORACLE_ACT_RELU = 1, ORACLE_ACT_RELU6 = 2, ORACLE_ACT_SILU = 3,
       ORACLE_ACT_HARDSWISH = 4 };

static float oracle_act(float t, int act) {
  if (act == ORACLE_ACT_RELU) return t < 0.0f ? 0.0f : t;
  if (act == ORACLE_ACT_RELU6) return t < 0.0f ? 0.0f : (t > 6.0f ? 6.0f : t);
  if (act == ORACLE_ACT_SILU) return t / (1.0f + expf(-t));
  if (act == ORACLE_ACT_HARDSWISH) {
    /* t * clamp(t + 3, 0, 6) / 6: one rounded multiply, one division */
    float h = t + 3.0f;
    h = h < 0.0f ? 0.0f : (h > 6.0f ? 6.0f : h);
    return (t * h) / 6.0f;
  }
  return t;
}

/*
 * General forward with the fused epilogue (no counterpart in the reference):
 *   t = chain_{r,s} fmaf(x, w, acc)            (as below)
 *   t = t + bias[c]      if bias != NULL       (fp32)
 *   t = act(t)                                 (fp32; relu/relu6 exact, silu via expf)
 *   t = t + residual[n,p,q,c] if residual      (fp32)
 *   y = f16_rne(t)
 */
int oracle_dwconv3x3_ex_f16(const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                            const uint16_t* residual, uint16_t* y, int64_t N, int64_t H,
                            int64_t W, int64_t C, int64_t pad, int act, int threads);

/*
 * y[n,p,q,c] = f16_rne( chain_{r=0..2, s=0..2} fmaf(x[n,p+r-pad,q+s-pad,c], w[r,s,c], acc) )
 * x: [N,H,W,C] fp16 bits, w: [3,3,C] fp16 bits, y: [N,P,Q,C] fp16 bits.
 * threads <= 0: use the OpenMP default.  Returns 0, or -1 on bad arguments /
 * allocation failure.
 */
int oracle_dwconv3x3_f16(const uint16_t* x, const uint16_t* w, uint16_t* y, int64_t N,
                         int64_t H, int64_t W, int64_t C, int64_t pad, int threads) {
  return oracle_dwconv3x3_ex_f16(x, w, NULL, NULL, y, N, H, W, C, pad, ORACLE_ACT_NONE, threads);
}

int oracle_dwconv3x3_ex_f16(const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                            const uint16_t* residual, uint16_t* y, int64_t N, int64_t H,
                            int64_t W, int64_t C, int64_t pad, int act, int threads) {
  if (!x || !w || !y || N < 0 || H < 1 || W < 1 || C < 0 || pad < 0) return -1;
  int64_t P, Q;
  oracle_output_hw(H, W, pad, &P, &Q);
  if (P < 0 || Q < 0) return -1;
  if (N == 0 || C == 0 || P == 0 || Q == 0) return 0;

  float* wf = (float*)malloc(sizeof(float) * 9 * (size_t)C);
  if (!wf) return -1;
  for (int64_t i = 0; i < 9 * C; ++i) wf[i] = oracle_f16_to_f32(w[i]);

  /* decode table: every fp16 bit pattern -> fp32 */
  float* lut = (float*)malloc(sizeof(float) * 65536);
  if (!lut) { free(wf); return -1; }
  for (uint32_t i = 0; i < 65536u; ++i) lut[i] = oracle_f16_to_f32((uint16_t)i);

  const int64_t WP = W + 2 * pad; /* decoded row with zero columns either side */
  int err = 0;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads) reduction(| : err)
#endif
  {
    float* rows = (float*)calloc((size_t)(3 * WP * C + 1), sizeof(float));
    float* zero_row = (float*)calloc((size_t)(WP * C + 1), sizeof(float));
    float* acc = (float*)malloc(sizeof(float) * (size_t)(C + 1));
    if (!rows || !zero_row || !acc) {
      err = 1;
    } else {
      int64_t cached[3] = {-1, -1, -1}; /* global (n*H + h) index held in each slot */
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
      for (int64_t np = 0; np < N * P; ++np) {
        const int64_t n = np / P, p = np % P;
        const float* in[3];
        for (int r = 0; r < 3; ++r) {
          const int64_t h = p + r - pad;
          if (h < 0 || h >= H) { in[r] = zero_row; continue; }
          const int64_t key = n * H + h;
          int slot = -1;
          for (int k = 0; k < 3; ++k) if (cached[k] == key) slot = k;
          if (slot < 0) {
            /* evict a slot not used by the other taps of this output row */
            for (int k = 0; k < 3 && slot < 0; ++k) {
              int used = 0;
              for (int rr = 0; rr < 3; ++rr) {
                const int64_t hh = p + rr - pad;
                if (hh >= 0 && hh < H && cached[k] == n * H + hh) used = 1;
              }
              if (!used) slot = k;
            }
            float* dst = rows + (int64_t)slot * WP * C + pad * C;
            const uint16_t* src = x + key * W * C;
            for (int64_t i = 0; i < W * C; ++i) dst[i] = lut[src[i]];
            cached[slot] = key;
          }
          in[r] = rows + (int64_t)slot * WP * C;
        }
        uint16_t* out = y + np * Q * C;
        for (int64_t q = 0; q < Q; ++q) {
          for (int64_t c = 0; c < C; ++c) acc[c] = 0.0f;
          for (int r = 0; r < 3; ++r)
            for (int s = 0; s < 3; ++s) {
              const float* xr = in[r] + (q + s) * C;
              const float* wr = wf + (r * 3 + s) * C;
              for (int64_t c = 0; c < C; ++c) acc[c] = fmaf(xr[c], wr[c], acc[c]);
            }
          const uint16_t* res = residual ? residual + np * Q * C + q * C : NULL;
          for (int64_t c = 0; c < C; ++c) {
            float t = acc[c];
            if (bias) t = t + lut[bias[c]];
            t = oracle_act(t, act);
            if (res) t = t + lut[res[c]];
            out[q * C + c] = oracle_f32_to_f16(t);
          }
        }
      }
    }
    free(rows);
    free(zero_row);
    free(acc);
  }
  free(lut);
  free(wf);
  return err ? -1 : 0;
}

/*
 * K x K depthwise forward with stride and the fused epilogue (no counterpart
 * in the reference, which is 3x3 stride 1; its ConvParams carries a stride,
 * csrc/common.cuh:38-40):
 *   t = chain_{r<K, s<K} fmaf(x[n, S*p+r-pad, S*q+s-pad, c], w[r,s,c], acc), acc from +0
 *   then bias / act / residual as oracle_dwconv3x3_ex_f16, y = f16_rne(t)
 * w: [K,K,C]; P = (H+2*pad-K)/S + 1, Q likewise.
 */
static int dwconv_ex(int codec, const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                     const uint16_t* residual, uint16_t* y, int64_t N, int64_t H, int64_t W,
                     int64_t C, int64_t K, int64_t S, int64_t pad, int act, int threads) {
  if (!x || !w || !y || N < 0 || H < 1 || W < 1 || C < 0 || pad < 0 || K < 1 || S < 1) return -1;
  if (H + 2 * pad < K || W + 2 * pad < K) return -1;
  const int64_t P = (H + 2 * pad - K) / S + 1, Q = (W + 2 * pad - K) / S + 1;
  if (N == 0 || C == 0) return 0;

  float* wf = (float*)malloc(sizeof(float) * (size_t)(K * K * C));
  float* lut = (float*)malloc(sizeof(float) * 65536);
  if (!wf || !lut) { free(wf); free(lut); return -1; }
  codec_lut(codec, lut);
  for (int64_t i = 0; i < K * K * C; ++i) wf[i] = lut[w[i]];

  const int64_t WP = W + 2 * pad;
  int err = 0;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads) reduction(| : err)
#endif
  {
    /* K decoded input rows, each with pad zero columns either side */
    float* rows = (float*)calloc((size_t)(K * WP * C + 1), sizeof(float));
    float* acc = (float*)malloc(sizeof(float) * (size_t)(C + 1));
    if (!rows || !acc) {
      err = 1;
    } else {
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
      for (int64_t np = 0; np < N * P; ++np) {
        const int64_t n = np / P, p = np % P;
        for (int64_t r = 0; r < K; ++r) {
          float* dst = rows + r * WP * C + pad * C;
          const int64_t h = S * p + r - pad;
          if (h < 0 || h >= H) {
            for (int64_t i = 0; i < W * C; ++i) dst[i] = 0.0f;
          } else {
            const uint16_t* src = x + (n * H + h) * W * C;
            for (int64_t i = 0; i < W * C; ++i) dst[i] = lut[src[i]];
          }
        }
        uint16_t* out = y + np * Q * C;
        for (int64_t q = 0; q < Q; ++q) {
          for (int64_t c = 0; c < C; ++c) acc[c] = 0.0f;
          for (int64_t r = 0; r < K; ++r)
            for (int64_t s = 0; s < K; ++s) {
              const float* xr = rows + r * WP * C + (S * q + s) * C;
              const float* wr = wf + (r * K + s) * C;
              for (int64_t c = 0; c < C; ++c) acc[c] = fmaf(xr[c], wr[c], acc[c]);
            }
          const uint16_t* res = residual ? residual + np * Q * C + q * C : NULL;
          for (int64_t c = 0; c < C; ++c) {
            float t = acc[c];
            if (bias) t = t + lut[bias[c]];
            t = oracle_act(t, act);
            if (res) t = t + lut[res[c]];
            out[q * C + c] = codec_round(codec, t);
          }
        }
      }
    }
    free(rows);
    free(acc);
  }
  free(lut);
  free(wf);
  return err ? -1 : 0;
}

int oracle_dwconv_ex_f16(const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                         const uint16_t* residual, uint16_t* y, int64_t N, int64_t H, int64_t W,
                         int64_t C, int64_t K, int64_t S, int64_t pad, int act, int threads) {
  return dwconv_ex(CODEC_F16, x, w, bias, residual, y, N, H, W, C, K, S, pad, act, threads);
}

/* The same with bfloat16 elements (x, w, bias, residual, y as bf16 bits):
 * decoded exactly to fp32, y = bf16_rne(t).  No counterpart in the reference. */
int oracle_dwconv_ex_bf16(const uint16_t* x, const uint16_t* w, const uint16_t* bias,
                          const uint16_t* residual, uint16_t* y, int64_t N, int64_t H, int64_t W,
                          int64_t C, int64_t K, int64_t S, int64_t pad, int act, int threads) {
  return dwconv_ex(CODEC_BF16, x, w, bias, residual, y, N, H, W, C, K, S, pad, act, threads);
}

/*
 * Data gradient (no counterpart in the reference):
 *   dx[n,h,w,c] = chain over (r', s') = (0..2, 0..2) of
 *                 fmaf(dy[n, h+pad-(2-r'), w+pad-(2-s'), c], w[2-r', 2-s', c], acc)
 * i.e. the forward's chain with the taps flipped — the order in which the
 * kernel visits them — with dy = 0 outside [0,P) x [0,Q); then f16 RNE.
 * dy: [N,P,Q,C], P = H+2*pad-2, Q = W+2*pad-2; dx: [N,H,W,C].
 */
int oracle_dwconv3x3_bwd_data_f16(const uint16_t* dy, const uint16_t* w, uint16_t* dx, int64_t N,
                                  int64_t H, int64_t W, int64_t C, int64_t pad, int threads) {
  if (!dy || !w || !dx || N < 0 || H < 1 || W < 1 || C < 0 || pad < 0) return -1;
  const int64_t P = H + 2 * pad - 2, Q = W + 2 * pad - 2;
  if (P < 1 || Q < 1) return -1;
  if (N == 0 || C == 0) return 0;
  float* wf = (float*)malloc(sizeof(float) * 9 * (size_t)C);
  float* lut = (float*)malloc(sizeof(float) * 65536);
  if (!wf || !lut) { free(wf); free(lut); return -1; }
  for (int64_t i = 0; i < 9 * C; ++i) wf[i] = oracle_f16_to_f32(w[i]);
  for (uint32_t i = 0; i < 65536u; ++i) lut[i] = oracle_f16_to_f32((uint16_t)i);
  int err = 0;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads) reduction(| : err)
#endif
  {
    float* acc = (float*)malloc(sizeof(float) * (size_t)(C + 1));
    if (!acc) {
      err = 1;
    } else {
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
      for (int64_t nh = 0; nh < N * H; ++nh) {
        const int64_t n = nh / H, h = nh % H;
        for (int64_t x = 0; x < W; ++x) {
          for (int64_t c = 0; c < C; ++c) acc[c] = 0.0f;
          for (int rp = 0; rp < 3; ++rp) {
            const int64_t p = h + pad - (2 - rp);
            for (int sp = 0; sp < 3; ++sp) {
              const int64_t q = x + pad - (2 - sp);
              const float* wr = wf + ((2 - rp) * 3 + (2 - sp)) * C;
              if (p < 0 || p >= P || q < 0 || q >= Q) {
                for (int64_t c = 0; c < C; ++c) acc[c] = fmaf(0.0f, wr[c], acc[c]);
              } else {
                const uint16_t* src = dy + ((n * P + p) * Q + q) * C;
                for (int64_t c = 0; c < C; ++c) acc[c] = fmaf(lut[src[c]], wr[c], acc[c]);
              }
            }
          }
          uint16_t* out = dx + ((n * H + h) * W + x) * C;
          for (int64_t c = 0; c < C; ++c) out[c] = oracle_f32_to_f16(acc[c]);
        }
      }
    }
    free(acc);
  }
  free(lut);
  free(wf);
  return err ? -1 : 0;
}

/*
 * Data gradient of the K x K stride-1 forward (no counterpart in the
 * reference): the 3x3 chain above with K taps,
 *   dx[n,h,w,c] = chain over (r', s') in (0..K-1, 0..K-1) of
 *                 fmaf(dy[n, h+pad-(K-1-r'), w+pad-(K-1-s'), c], w[K-1-r', K-1-s', c], acc)
 * with dy = 0 outside [0,P) x [0,Q), P = H+2*pad-K+1; then f16 RNE.
 */
static int bwd_data_s1(int codec, const uint16_t* dy, const uint16_t* w, uint16_t* dx, int64_t N,
                       int64_t H, int64_t W, int64_t C, int64_t K, int64_t pad, int threads) {
  if (!dy || !w || !dx || N < 0 || H < 1 || W < 1 || C < 0 || pad < 0 || K < 1) return -1;
  const int64_t P = H + 2 * pad - K + 1, Q = W + 2 * pad - K + 1;
  if (P < 1 || Q < 1) return -1;
  if (N == 0 || C == 0) return 0;
  float* wf = (float*)malloc(sizeof(float) * (size_t)(K * K * C));
  float* lut = (float*)malloc(sizeof(float) * 65536);
  if (!wf || !lut) { free(wf); free(lut); return -1; }
  codec_lut(codec, lut);
  for (int64_t i = 0; i < K * K * C; ++i) wf[i] = lut[w[i]];
  int err = 0;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads) reduction(| : err)
#endif
  {
    float* acc = (float*)malloc(sizeof(float) * (size_t)(C + 1));
    if (!acc) {
      err = 1;
    } else {
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
      for (int64_t nh = 0; nh < N * H; ++nh) {
        const int64_t n = nh / H, h = nh % H;
        for (int64_t x = 0; x < W; ++x) {
          for (int64_t c = 0; c < C; ++c) acc[c] = 0.0f;
          for (int64_t rp = 0; rp < K; ++rp) {
            const int64_t p = h + pad - (K - 1 - rp);
            for (int64_t sp = 0; sp < K; ++sp) {
              const int64_t q = x + pad - (K - 1 - sp);
              const float* wr = wf + ((K - 1 - rp) * K + (K - 1 - sp)) * C;
              if (p < 0 || p >= P || q < 0 || q >= Q) {
                for (int64_t c = 0; c < C; ++c) acc[c] = fmaf(0.0f, wr[c], acc[c]);
              } else {
                const uint16_t* src = dy + ((n * P + p) * Q + q) * C;
                for (int64_t c = 0; c < C; ++c) acc[c] = fmaf(lut[src[c]], wr[c], acc[c]);
              }
            }
          }
          uint16_t* out = dx + ((n * H + h) * W + x) * C;
          for (int64_t c = 0; c < C; ++c) out[c] = codec_round(codec, acc[c]);
        }
      }
    }
    free(acc);
  }
  free(lut);
  free(wf);
  return err ? -1 : 0;
}

int oracle_dwconv_bwd_data_f16(const uint16_t* dy, const uint16_t* w, uint16_t* dx, int64_t N,
                               int64_t H, int64_t W, int64_t C, int64_t K, int64_t pad,
                               int threads) {
  return bwd_data_s1(CODEC_F16, dy, w, dx, N, H, W, C, K, pad, threads);
}

/* bfloat16 elements, otherwise as oracle_dwconv_bwd_data_f16. */
int oracle_dwconv_bwd_data_bf16(const uint16_t* dy, const uint16_t* w, uint16_t* dx, int64_t N,
                                int64_t H, int64_t W, int64_t C, int64_t K, int64_t pad,
                                int threads) {
  return bwd_data_s1(CODEC_BF16, dy, w, dx, N, H, W, C, K, pad, threads);
}

/*
 * Data gradient of the K x K stride-2 forward (no counterpart in the
 * reference, whose forward is 3x3 stride 1).  The forward reads
 * x[n, 2p+r-pad, 2q+s-pad, c], so
 *   dx[n,h,v,c] = chain over r = K-1 .. 0 with (h+pad-r) even, then over
 *                 s = K-1 .. 0 with (v+pad-s) even, of
 *                 fmaf(dy[n, (h+pad-r)/2, (v+pad-s)/2, c], w[r,s,c], acc)
 * from +0 with dy = 0 outside [0,P) x [0,Q), P = (H+2*pad-K)/2 + 1; then
 * f16 RNE.  r and s descending is the order of the stride-1 data gradient
 * (the forward with flipped taps) restricted to the taps a stride-2 output
 * reaches.
 */
static int bwd_data_s2(int codec, const uint16_t* dy, const uint16_t* w, uint16_t* dx, int64_t N,
                       int64_t H, int64_t W, int64_t C, int64_t K, int64_t pad, int threads) {
  if (!dy || !w || !dx || N < 0 || H < 1 || W < 1 || C < 0 || pad < 0 || K < 1) return -1;
  if (H + 2 * pad < K || W + 2 * pad < K) return -1;
  const int64_t P = (H + 2 * pad - K) / 2 + 1, Q = (W + 2 * pad - K) / 2 + 1;
  if (N == 0 || C == 0) return 0;
  float* wf = (float*)malloc(sizeof(float) * (size_t)(K * K * C));
  float* lut = (float*)malloc(sizeof(float) * 65536);
  if (!wf || !lut) { free(wf); free(lut); return -1; }
  codec_lut(codec, lut);
  for (int64_t i = 0; i < K * K * C; ++i) wf[i] = lut[w[i]];
  int err = 0;
#ifdef _OPENMP
  if (threads <= 0) threads = omp_get_max_threads();
#pragma omp parallel num_threads(threads) reduction(| : err)
#endif
  {
    float* acc = (float*)malloc(sizeof(float) * (size_t)(C + 1));
    if (!acc) {
      err = 1;
    } else {
#ifdef _OPENMP
#pragma omp for schedule(static)
#endif
      for (int64_t nh = 0; nh < N * H; ++nh) {
        const int64_t n = nh / H, h = nh % H;
        for (int64_t v = 0; v < W; ++v) {
          for (int64_t c = 0; c < C; ++c) acc[c] = 0.0f;
          for (int64_t r = K - 1; r >= 0; --r) {
            const int64_t hp = h + pad - r;
            if (hp % 2 != 0) continue;
            const int64_t p = hp / 2;
            for (int64_t s = K - 1; s >= 0; --s) {
              const int64_t vq = v + pad - s;
              if (vq % 2 != 0) continue;
              const int64_t q = vq / 2;
              const float* wr = wf + (r * K + s) * C;
              if (p < 0 || p >= P || q < 0 || q >= Q) {
                for (int64_t c = 0; c < C; ++c) acc[c] = fmaf(0.0f, wr[c], acc[c]);
              } else {
                const uint16_t* src = dy + ((n * P + p) * Q + q) * C;
                for (int64_t c = 0; c < C; ++c) acc[c] = fmaf(lut[src[c]], wr[c], acc[c]);
              }
            }
          }
          uint16_t* out = dx + ((n * H + h) * W + v) * C;
          for (int64_t c = 0; c < C; ++c) out[c] = codec_round(codec, acc[c]);
        }
      }
    }
    free(acc);
  }
  free(lut);
  free(wf);
  return err ? -1 : 0;
}

int oracle_dwconv_bwd_data_s2_f16(const uint16_t* dy, const uint16_t* w, uint16_t* dx, int64_t N,
                                  int64_t H, int64_t W, int64_t C, int64_t K, int64_t pad,
                                  int threads) {
  return bwd_data_s2(CODEC_F16, dy, w, dx, N, H, W, C, K, pad, threads);
}

/* bfloat16 elements, otherwise as oracle_dwconv_bwd_data_s2_f16. */
int oracle_dwconv_bwd_data_s2_bf16(const uint16_t* dy, const uint16_t* w, uint16_t* dx,
                                   int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                   int64_t pad, int threads) {
  return bwd_data_s2(CODEC_BF16, dy, w, dx, N, H, W, C, K, pad, threads);
}

/* Threads an OpenMP parallel region would use by default (1 without OpenMP). */
int oracle_max_threads(void) {
#ifdef _OPENMP
  return omp_get_max_threads();
#else
  return 1;
#endif
}
