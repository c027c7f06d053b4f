/*
 * tdc_dwconv.h — C ABI of the sm_100a NHWC fp16 depthwise 3x3 conv2d forward.
 *
 * This is the drop-in boundary between any host (the `_tma_dwconv_C` PyTorch
 * extension, ctypes, cgo, JNI …) and the hand-written Blackwell kernels in
 * libtdc_sm100.so.  Signatures use plain pointers and 64-bit sizes only: no
 * torch, no CUDA headers.  `stream` is a `cudaStream_t` passed as `void*`
 * (NULL = the legacy default stream of the current device).
 *
 * Tensor layouts (all row-major, contiguous, fp16 = IEEE binary16):
 *   x  [N, H, W, C]      input activations (NHWC)
 *   w  [R, S, C]         depthwise filter, one RxS kernel per channel (R=S=3)
 *   y  [N, P, Q, C]      output, P = H + 2*pad - 2, Q = W + 2*pad - 2
 *
 * Semantics (identical for every entry point):
 *   y[n,p,q,c] = fp16_rne( sum_{r=0..2} sum_{s=0..2} fp32(x[n,p+r-pad,q+s-pad,c]) * fp32(w[r,s,c]) )
 * accumulated in fp32 from +0 in r-major, s-minor order, with x = 0 outside the
 * image.  Stride 1, symmetric zero padding pad >= 0.
 *
 * Ownership / threading: the caller allocates x, w, y (and `stall`) on the
 * CUDA device that is current for the calling thread; the library never
 * takes ownership and never synchronises.  Every entry point is stream-ordered
 * and re-entrant; it may be called from any host thread.
 *
 * Return value: TDC_OK (0) or a negative TDC_ERR_* code.  Argument errors are
 * detected on the host before any CUDA call is made.  An empty output
 * (N, C, P or Q == 0) is a successful no-op and may come with NULL pointers.
 * TDC_ERR_DEVICE_TIMEOUT from a call that launches work reports an EARLIER
 * launch on the device that gave up on a pipeline wait (see "pipeline-wait
 * failure detection" below); nothing was launched.
 */
#ifndef TDC_DWCONV_H_
#define TDC_DWCONV_H_

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

#if defined(__GNUC__)
#define TDC_API __attribute__((visibility("default")))
#else
#define TDC_API
#endif

/* ---- status codes ------------------------------------------------------- */
#define TDC_OK                    0
#define TDC_ERR_NULL_POINTER     -1  /* x, w, y (or stall for the probe) is NULL          */
#define TDC_ERR_BAD_SHAPE        -2  /* N or C < 0, H or W < 1, or a negative output size  */
#define TDC_ERR_FILTER_SHAPE     -3  /* R != 3 or S != 3                                     */
#define TDC_ERR_CHANNELS         -4  /* C not a multiple of 8 (v0, fwd) / 64 (ws)            */
#define TDC_ERR_PAD              -5  /* pad < 0                                             */
#define TDC_ERR_N_STAGE          -6  /* n_stage not in {2, 3, 4}                             */
#define TDC_ERR_ALIGNMENT        -7  /* x, w or y not 16-byte aligned                        */
#define TDC_ERR_TOO_LARGE        -8  /* a dimension exceeds what the TMA descriptor encodes  */
#define TDC_ERR_CUDA             -9  /* a CUDA runtime call failed (see tdc_last_cuda_error) */
#define TDC_ERR_TMA_ENCODE      -10  /* cuTensorMapEncodeTiled rejected the descriptor       */
#define TDC_ERR_DEVICE_TIMEOUT  -11  /* an earlier launch gave up waiting on its pipeline  */
#define TDC_ERR_NO_DEVICE       -12  /* no usable sm_100 device is current                   */
#define TDC_ERR_ACT             -13  /* unknown activation code (tdc_dwconv3x3_fwd)          */
#define TDC_ERR_WORKSPACE       -14  /* workspace too small (tdc_dwconv3x3_bwd_weight)       */
#define TDC_ERR_SCRATCH_LIMIT   -15  /* C beyond the static scratch (..._bwd_weight_noalloc) */
#define TDC_ERR_STRIDE          -16  /* stride not 1 or 2 (tdc_dwconv_fwd)                  */
#define TDC_ERR_UNSUPPORTED     -17  /* no kernel for this request (e.g. an unknown plan kind) */

/* Human-readable text for a status code (static storage, never NULL). */
TDC_API const char* tdc_strerror(int code);

/* cudaError_t of the most recent failing CUDA call made by this thread
 * inside the library, or the CUresult of a failed cuTensorMapEncodeTiled
 * (0 if none). */
TDC_API int tdc_last_cuda_error(void);

/* Output spatial size for a stride-1 RxS conv with symmetric padding:
 * P = H + 2*pad - R + 1, Q = W + 2*pad - S + 1.
 * Replaces the P/Q computation of the reference host launchers
 * (csrc/kernel_tma_ws.cu:382-385, csrc/kernel_v0_naive_float4.cu:96-99). */
TDC_API int tdc_output_hw(int64_t H, int64_t W, int64_t R, int64_t S, int64_t pad,
                          int64_t* P, int64_t* Q);

/* Plain (non-TMA) kernel: global loads through L1, no shared memory; a
 * thread slides 8 output columns of one channel pair down a band of rows
 * (the kernel of tdc_dwconv_fwd_plain).  Requires C % 8 == 0.
 * Replaces tma_dwconv::dwconv_v0 (csrc/bindings.cpp:6,
 * csrc/kernel_v0_naive_float4.cu:78-118), with y supplied by the caller. */
TDC_API int tdc_dwconv_v0(const void* x, const void* w, void* y,
                          int64_t N, int64_t H, int64_t W, int64_t C,
                          int64_t R, int64_t S, int64_t pad, void* stream);

/* TMA + warp-specialised kernel: one producer warp streams halo'd row tiles
 * into an n_stage-deep shared-memory ring (mbarrier full/empty pairs); four
 * consumer warps keep a 3-row sliding window of fp32 accumulators in
 * registers.  Requires C % 64 == 0 and n_stage in {2, 3, 4}.
 * Replaces tma_dwconv::dwconv_ws (csrc/bindings.cpp:7-8,
 * csrc/kernel_tma_ws.cu:52-82), with y supplied by the caller. */
TDC_API int tdc_dwconv_ws(const void* x, const void* w, void* y,
                          int64_t N, int64_t H, int64_t W, int64_t C,
                          int64_t R, int64_t S, int64_t pad, int64_t n_stage,
                          void* stream);

/* tdc_dwconv_ws for inputs and outputs in HOST memory: copies w and x to the
 * device, runs the ws kernel and copies y back, pipelined over chunks of
 * `chunk_images` images (0 = N/64 rounded up) so that the host->device copy
 * of one chunk, the kernel of the previous one and the device->host copy of
 * the one before run at the same time (the two copy directions use separate
 * copy engines).  x_host [N,H,W,C], w_host [3,3,C] and y_host [N,P,Q,C]
 * should be page-locked (cudaHostAlloc / cudaHostRegister) for the copies to
 * be asynchronous; x_dev, w_dev and y_dev are caller-owned device buffers of
 * the same sizes.  The work is ordered after what is already queued on
 * `stream`, and `stream` waits for the last copy back, so y_host holds the
 * result once `stream` has completed.  The library runs the chunks on three
 * streams of its own per device, created on the first call.  Same
 * requirements and status codes as tdc_dwconv_ws (R = S = 3 implied).
 * Replaces the caller-side sequence H2D copy -> tma_dwconv::dwconv_ws ->
 * D2H copy around the reference's extension call (csrc/bindings.cpp:7-8). */
TDC_API int tdc_dwconv_ws_host(const void* x_host, const void* w_host, void* y_host,
                               int64_t N, int64_t H, int64_t W, int64_t C, int64_t pad,
                               int64_t n_stage, void* x_dev, void* w_dev, void* y_dev,
                               int64_t chunk_images, void* stream);

/* ---- general forward ---------------------------------------------------------
 * The ws kernel widened beyond the reference's surface: any C % 8 == 0 (the
 * reference's ws requires C % 64) and an optional fused epilogue, computed
 * per output in fp32 with one rounding to fp16 at the end:
 *   t = sum_{r,s} x*w  (as above);  t += bias[c];  t = act(t);  t += residual[n,p,q,c]
 *   y = fp16_rne(t)
 * act: TDC_ACT_NONE, TDC_ACT_RELU (t < 0 ? +0 : t), TDC_ACT_RELU6
 * (min(relu(t), 6)), TDC_ACT_SILU (t / (1 + expf(-t))), TDC_ACT_HARDSWISH
 * (t * min(max(t + 3, 0), 6) / 6, rounded in that order).
 * bias: fp16 [C] or NULL; residual: fp16 [N,P,Q,C] or NULL (may be y itself).
 * No counterpart in the reference; the epilogue is what a depthwise block
 * applies next (bias, activation, skip connection), saving a full pass over y. */
#define TDC_ACT_NONE  0
#define TDC_ACT_RELU  1
#define TDC_ACT_RELU6 2
#define TDC_ACT_SILU  3
#define TDC_ACT_HARDSWISH 4

TDC_API int tdc_dwconv3x3_fwd(const void* x, const void* w, const void* bias,
                              const void* residual, void* y,
                              int64_t N, int64_t H, int64_t W, int64_t C,
                              int64_t pad, int64_t act, int64_t n_stage, void* stream);

/* General K x K depthwise forward, K in {3, 5, 7}, stride 1 or 2, symmetric
 * padding, with the same optional epilogue as tdc_dwconv3x3_fwd:
 *   y[n,p,q,c] = fp16_rne(epilogue( chain_{r<K, s<K} x[n, S*p+r-pad, S*q+s-pad, c] * w[r,s,c] ))
 * fp32 chain from +0 in (r, s) lexicographic order.  w: [K, K, C] fp16;
 * P = (H + 2*pad - K) / S + 1, Q likewise; C % 8 == 0.  (K, stride) = (3, 1)
 * is tdc_dwconv3x3_fwd.  n_stage 2, 3 or 4 runs the ws kernel with that ring
 * depth; n_stage 0 leaves the choice to the library: the plain kernel
 * (tdc_dwconv_fwd_plain) where tdc_dwconv_fwd_uses_plain says so, else the
 * ws kernel at the geometry's default depth.  The result is the same bit
 * for bit either way.  No counterpart in the reference (3x3, stride 1 only). */
TDC_API int tdc_dwconv_fwd(const void* x, const void* w, const void* bias,
                           const void* residual, void* y,
                           int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                           int64_t stride, int64_t pad, int64_t act, int64_t n_stage,
                           void* stream);

/* tdc_dwconv_fwd for bfloat16 tensors: x, w, bias, residual and y hold
 * bfloat16 (1 sign, 8 exponent, 7 mantissa bits) instead of fp16.  Same
 * geometries, epilogue and fp32 chain; each element is widened to fp32
 * exactly and the result is rounded to nearest-even bfloat16 once.  3x3
 * stride 1 included.  No counterpart in the reference (fp16 only). */
TDC_API int tdc_dwconv_fwd_bf16(const void* x, const void* w, const void* bias,
                                const void* residual, void* y,
                                int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                int64_t stride, int64_t pad, int64_t act, int64_t n_stage,
                                void* stream);

/* tdc_dwconv_fwd (and _bf16) with each side's zero padding given separately:
 *   y[n,p,q,c] = epilogue(chain_{r,s} x[n, S*p+r-pad_top, S*q+s-pad_left, c] * w[r,s,c])
 * with P = (H + pad_top + pad_bottom - K)/S + 1 and Q likewise, e.g.
 * TensorFlow's "SAME" padding at stride 2, which puts the odd row and column
 * at the bottom / right (3x3 on 112 x 112: top 0, bottom 1).  Same kernels,
 * arithmetic and n_stage meaning (0 = chosen from the shape) as
 * tdc_dwconv_fwd; every pad >= 0.  No counterpart in the reference
 * (symmetric padding only). */
TDC_API int tdc_dwconv_fwd_asym(const void* x, const void* w, const void* bias,
                                const void* residual, void* y,
                                int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                int64_t stride, int64_t pad_top, int64_t pad_bottom,
                                int64_t pad_left, int64_t pad_right, int64_t act,
                                int64_t n_stage, void* stream);
TDC_API int tdc_dwconv_fwd_asym_bf16(const void* x, const void* w, const void* bias,
                                     const void* residual, void* y,
                                     int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                     int64_t stride, int64_t pad_top, int64_t pad_bottom,
                                     int64_t pad_left, int64_t pad_right, int64_t act,
                                     int64_t n_stage, void* stream);

/* Dilated K x K forward (K = 3, 5, 7, stride 1 or 2, dilation >= 1) with
 * per-side padding:
 *   y[n,p,q,c] = epilogue(chain_{r,s} x[n, S*p + D*r - pad_top, S*q + D*s - pad_left, c] * w[r,s,c])
 * P = (H + pad_top + pad_bottom - D*(K-1) - 1)/S + 1, Q likewise; the same
 * fp32 chain, epilogue and rounding as tdc_dwconv_fwd (atrous depthwise layers,
 * e.g. DeepLab backbones).  dilation 1 is tdc_dwconv_fwd_asym with n_stage 0.
 * Above 1 the outputs split into the D*D phases (p mod D, q mod D); on each,
 * outputs D apart read inputs D apart: an undilated K x K problem on the
 * D-strided sub-lattice of x.  The ring (TMA) kernel runs the phases as
 * extra images, its tensor map loading the sub-lattice with traversal
 * stride D (while D * (32*S + K - S) <= 256); the plain kernel slides its
 * window D rows and columns at a time.  The ring kernel runs when the phases
 * are at least 32 x 32 outputs and the undilated choice of tdc_dwconv_fwd
 * (n_stage 0) gives them to it (tdc_dwconv_fwd_dilated_uses_plain).  No
 * counterpart in the reference (no dilation). */
TDC_API int tdc_dwconv_fwd_dilated(const void* x, const void* w, const void* bias,
                                   const void* residual, void* y,
                                   int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                   int64_t stride, int64_t dilation, int64_t pad_top,
                                   int64_t pad_bottom, int64_t pad_left, int64_t pad_right,
                                   int64_t act, void* stream);
TDC_API int tdc_dwconv_fwd_dilated_bf16(const void* x, const void* w, const void* bias,
                                        const void* residual, void* y,
                                        int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                        int64_t stride, int64_t dilation, int64_t pad_top,
                                        int64_t pad_bottom, int64_t pad_left, int64_t pad_right,
                                        int64_t act, void* stream);

/* tdc_dwconv_fwd_dilated / _bf16 (bf16 != 0) with the kernel named:
 * kernel 1 = the ring kernel, at the geometry's default ring depth
 * (TDC_ERR_UNSUPPORTED for dilation 1 or when its tensor map cannot step
 * `dilation` rows and columns), -1 = the plain kernel, 0 = chosen by shape
 * (tdc_dwconv_fwd_dilated).  Every kernel gives the same result, bit for
 * bit.  No counterpart in the reference. */
TDC_API int tdc_dwconv_fwd_dilated_ex(const void* x, const void* w, const void* bias,
                                      const void* residual, void* y,
                                      int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                      int64_t stride, int64_t dilation, int64_t pad_top,
                                      int64_t pad_bottom, int64_t pad_left, int64_t pad_right,
                                      int64_t act, int64_t kernel, int64_t bf16, void* stream);

/* 1 if tdc_dwconv_fwd_dilated runs the plain kernel on this shape, else 0
 * (pure host arithmetic).  No counterpart in the reference. */
TDC_API int tdc_dwconv_fwd_dilated_uses_plain(int64_t N, int64_t H, int64_t W, int64_t C,
                                              int64_t K, int64_t stride, int64_t dilation,
                                              int64_t pad_top, int64_t pad_bottom,
                                              int64_t pad_left, int64_t pad_right);

/* Plain K x K forward: global loads through L1, no TMA, no shared memory, no
 * pipeline.  A thread owns one channel pair of one output column over a band
 * of band_rows output rows (0 = chosen from the shape: the full height unless
 * that leaves fewer than two waves of threads).  For shapes the ws kernel's
 * 32-column x 64-channel strips fit badly (few channels, narrow images).
 * Same arguments (band_rows in place of n_stage), arithmetic and result, bit
 * for bit, as tdc_dwconv_fwd.  No counterpart in the reference. */
TDC_API int tdc_dwconv_fwd_plain(const void* x, const void* w, const void* bias,
                                 const void* residual, void* y,
                                 int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                 int64_t stride, int64_t pad, int64_t act, int64_t band_rows,
                                 void* stream);

/* tdc_dwconv_fwd_plain for bfloat16 tensors (as tdc_dwconv_fwd_bf16). */
TDC_API int tdc_dwconv_fwd_plain_bf16(const void* x, const void* w, const void* bias,
                                      const void* residual, void* y,
                                      int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                      int64_t stride, int64_t pad, int64_t act,
                                      int64_t band_rows, void* stream);

/* 1 if tdc_dwconv_fwd with n_stage 0 runs the plain kernel on this shape,
 * else 0 (pure host arithmetic). */
TDC_API int tdc_dwconv_fwd_uses_plain(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                      int64_t stride, int64_t pad);

/* Plain weight gradient of the K x K forward (K = 3, 5, 7, stride 1 or 2):
 * dw [K,K,C] fp32 as tdc_dwconv_bwd_weight, for the same small shapes as
 * tdc_dwconv_fwd_plain.  A thread keeps one channel pair's K*K sums of one
 * (image, band of dy rows); a CTA adds its units up in a fixed order and
 * writes one slice of its channels, so the workspace
 * (tdc_dwconv_bwd_weight_plain_workspace) is about units / 16 x K*K x C
 * floats rather than the ws kernels' grid x 4 x K*K x C; a fixed-order
 * reduction sums the slices (deterministic).  N = 0 writes zeros.  No
 * counterpart in the reference. */
TDC_API int tdc_dwconv_bwd_weight_plain_workspace(int64_t N, int64_t H, int64_t W, int64_t C,
                                                  int64_t K, int64_t stride, int64_t pad,
                                                  int64_t* bytes);
TDC_API int tdc_dwconv_bwd_weight_plain(const void* x, const void* dy, float* dw,
                                        int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                        int64_t stride, int64_t pad, void* workspace,
                                        int64_t workspace_bytes, void* stream);
TDC_API int tdc_dwconv_bwd_weight_plain_bf16(const void* x, const void* dy, float* dw,
                                             int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                             int64_t stride, int64_t pad, void* workspace,
                                             int64_t workspace_bytes, void* stream);

/* 1 if tdc_dwconv_bwd_weight(_workspace) with n_stage 0 run the plain kernel
 * on this shape, else 0 (pure host arithmetic): output width Q <= 16 or
 * C <= 16 (a plain thread walks the whole width, so wide images with more
 * channels stay on the ws kernels). */
TDC_API int tdc_dwconv_bwd_weight_uses_plain(int64_t N, int64_t H, int64_t W, int64_t C,
                                             int64_t K, int64_t stride, int64_t pad);

/* Launch plan tdc_dwconv_fwd would use (same layout as tdc_ws_plan's
 * plan[0..8]; pure host arithmetic).  For K >= 5 at stride 1 and 7x7 at
 * stride 2 the kernel holds the K input rows of one output row at once, and
 * stage_rows satisfies (n_stage - 1) * stage_rows >= K - 1.  The strip is
 * stride*31 + K input columns wide.  No counterpart in the reference. */
TDC_API int tdc_dwconv_fwd_plan(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                int64_t stride, int64_t pad, int64_t n_stage, int64_t sms,
                                int64_t ctas_per_sm, int64_t* plan);

/* ---- backward ------------------------------------------------------------------
 * Data gradient of the 3x3 forward (stride 1, padding pad):
 *   dx[n,h,w,c] = sum_{r,s} dy[n, h+pad-r, w+pad-s, c] * w[r,s,c]   (dy = 0 outside)
 * computed by the forward kernel on dy with the taps flipped (w[2-r][2-s])
 * and padding 2 - pad (negative = a crop), fp32 chain in flipped-tap order,
 * fp16 RNE.  dy: [N,P,Q,C] with P = H+2*pad-2 >= 1, Q likewise; dx: [N,H,W,C];
 * C % 8 == 0.  No counterpart in the reference (forward only). */
TDC_API int tdc_dwconv3x3_bwd_data(const void* dy, const void* w, void* dx,
                                   int64_t N, int64_t H, int64_t W, int64_t C,
                                   int64_t pad, int64_t n_stage, void* stream);

/* Weight gradient of the 3x3 forward (stride 1, padding pad):
 *   dw[r,s,c] = sum_{n,p,q} x[n, p+r-pad, q+s-pad, c] * dy[n,p,q,c]   (x = 0 outside)
 * x: [N,H,W,C] fp16, dy: [N,P,Q,C] fp16, dw: [3,3,C] fp32 (written, not
 * accumulated).  fp16 x fp16 products accumulated in fp32: per CTA and warp
 * in a fixed order into `workspace`, then summed over the slices in a fixed
 * order, so the result is bit-reproducible run to run.  `workspace` is
 * caller-owned device memory of at least the size
 * tdc_dwconv3x3_bwd_weight_workspace reports (it depends on the device's SM
 * count); its contents need not be initialised.  C % 8 == 0.
 * Two launches on `stream`.  No counterpart in the reference (forward only). */
TDC_API int tdc_dwconv3x3_bwd_weight_workspace(int64_t N, int64_t H, int64_t W, int64_t C,
                                               int64_t pad, int64_t n_stage, int64_t* bytes);
TDC_API int tdc_dwconv3x3_bwd_weight(const void* x, const void* dy, float* dw,
                                     int64_t N, int64_t H, int64_t W, int64_t C,
                                     int64_t pad, int64_t n_stage,
                                     void* workspace, int64_t workspace_bytes, void* stream);

/* Weight gradient for callers that cannot allocate device memory.  No
 * counterpart in the reference.  Same result as tdc_dwconv3x3_bwd_weight (up
 * to the summation order when the grid differs), but the workspace is a
 * 16 MiB array inside the library instead of caller memory, so the call
 * allocates nothing: no cudaMalloc, no cudaFree, no allocating library call.
 * It is meant for runtimes that fix their device budget at start-up and
 * forbid later allocation, plug-ins whose host framework owns all device
 * memory, and paths where an allocation could synchronise or fail.
 *   - Every GPU that loads the library holds the 16 MiB until the process exits.
 *   - The first call on a device looks up the array's device address
 *     (cudaGetSymbolAddress); make that first call before any stream capture.
 *     A lookup that fails returns TDC_ERR_CUDA and is tried again by the
 *     next call; a successful one is kept for the process.
 *   - All calls on a device share the array and it keeps the last call's
 *     contents (each call clears the part it uses); calls that overlap on the
 *     GPU, e.g. on two streams, race and give wrong results.
 *   - Limit: each CTA needs 144*C bytes of it, so the launch uses at most
 *     16 MiB / (144*C) CTAs (fewer than the device could run once C > 256 on
 *     a 148-SM part, which is slower, not wrong); C > 116508 is rejected with
 *     TDC_ERR_SCRATCH_LIMIT. */
TDC_API int tdc_dwconv3x3_bwd_weight_noalloc(const void* x, const void* dy, float* dw,
                                             int64_t N, int64_t H, int64_t W, int64_t C,
                                             int64_t pad, int64_t n_stage, void* stream);

/* Backward of the K x K forward (K = 3, 5, 7) at stride 1 or 2.  No
 * counterpart in the reference (forward only).
 *   tdc_dwconv_bwd_data: dx [N,H,W,C] fp16 from dy [N,P,Q,C] and w [K,K,C].
 *     Stride 1: P = H + 2*pad - K + 1; the forward kernel with flipped taps
 *     and pad' = K - 1 - pad, so the chain per output is (r', s')
 *     lexicographic over w[K-1-r'][K-1-s'] from +0, one fp16 rounding.  For
 *     K > 3, pad <= K - 1.  K = 3 is tdc_dwconv3x3_bwd_data.
 *     Stride 2: P = (H + 2*pad - K)/2 + 1 (H is needed: two input heights
 *     give the same P); any pad >= 0.  A transposed-stencil kernel:
 *       dx[n,h,v,c] = chain over r = K-1 .. 0 with h + pad - r even, then
 *                     s = K-1 .. 0 with v + pad - s even, of
 *                     fma(dy[n, (h+pad-r)/2, (v+pad-s)/2, c], w[r,s,c], acc)
 *     from +0 (dy = 0 outside [0,P) x [0,Q)), one fp16 rounding.
 *     n_stage 0 leaves the kernel to the library: at stride 1 the plain
 *     kernel (tdc_dwconv_fwd_plain with flipped taps) where
 *     tdc_dwconv_fwd_uses_plain(N, P, Q, C, K, 1, K - 1 - pad) says so, else
 *     the default ring depth; the result is the same bit for bit.
 *   tdc_dwconv_bwd_weight: dw [K,K,C] fp32 (written), deterministic like
 *     tdc_dwconv3x3_bwd_weight, with a caller workspace of at least the size
 *     tdc_dwconv_bwd_weight_workspace reports (same stride and n_stage
 *     arguments; n_stage 0 picks tdc_dwconv_bwd_weight_plain where
 *     tdc_dwconv_bwd_weight_uses_plain says so, else the default depth).  At
 *     stride 1, K = 3 is tdc_dwconv3x3_bwd_weight.  At stride 2,
 *       dw[r,s,c] = sum_{n,p,q} x[n, 2p+r-pad, 2q+s-pad, c] * dy[n,p,q,c]
 *     with P = (H + 2*pad - K)/2 + 1 (x rows and columns that no output
 *     reads do not contribute).
 *   tdc_dwconv_bwd_weight_plan: the K = 5, 7 weight-gradient launch plan,
 *     pure host arithmetic, into plan[0..10]: plan[0..7] as tdc_ws_plan (the
 *     ring holds stage_rows rows of x and of dy per stage), plan[8] =
 *     launches (the tap rows are split over them to bound the sums a lane
 *     holds), plan[9] = tap rows of the tallest launch, plan[10] = dy rows a
 *     consumer step takes (they share x rows; the step holds
 *     plan[9] + plan[10] - 1 x rows, and the ring keeps
 *     (n_stage - 1) * stage_rows >= plan[9] + plan[10] - 2). */
TDC_API int tdc_dwconv_bwd_data(const void* dy, const void* w, void* dx,
                                int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                int64_t stride, int64_t pad, int64_t n_stage, void* stream);
TDC_API int tdc_dwconv_bwd_weight_workspace(int64_t N, int64_t H, int64_t W, int64_t C,
                                            int64_t K, int64_t stride, int64_t pad,
                                            int64_t n_stage, int64_t* bytes);
TDC_API int tdc_dwconv_bwd_weight(const void* x, const void* dy, float* dw,
                                  int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                  int64_t stride, int64_t pad, int64_t n_stage,
                                  void* workspace, int64_t workspace_bytes, void* stream);
TDC_API int tdc_dwconv_bwd_weight_plan(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                       int64_t pad, int64_t n_stage, int64_t sms,
                                       int64_t ctas_per_sm, int64_t* plan);

/* The backward for bfloat16 tensors (dy, w, x, dx bfloat16; dw fp32): the
 * same kernels and results' definitions as tdc_dwconv_bwd_data /
 * tdc_dwconv_bwd_weight(_workspace), with bfloat16 elements and bfloat16
 * rounding of dx.  At stride 1 the data gradient needs pad <= K - 1 (also
 * for K = 3).  The workspace size can differ from the fp16 call's: query it
 * with tdc_dwconv_bwd_weight_workspace_bf16.  No counterpart in the
 * reference. */
TDC_API int tdc_dwconv_bwd_data_bf16(const void* dy, const void* w, void* dx,
                                     int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                     int64_t stride, int64_t pad, int64_t n_stage, void* stream);
TDC_API int tdc_dwconv_bwd_weight_workspace_bf16(int64_t N, int64_t H, int64_t W, int64_t C,
                                                 int64_t K, int64_t stride, int64_t pad,
                                                 int64_t n_stage, int64_t* bytes);
TDC_API int tdc_dwconv_bwd_weight_bf16(const void* x, const void* dy, float* dw,
                                       int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                       int64_t stride, int64_t pad, int64_t n_stage,
                                       void* workspace, int64_t workspace_bytes, void* stream);

/* Launch plan of the stride-2 backward (pure host arithmetic) into
 * plan[0..10], which = 0 for the data gradient, 1 for the weight gradient;
 * plan[0..7] as tdc_ws_plan.
 * Data gradient: strips and bands over dx [N,H,W,C]; stage_rows counts dy
 * rows of 16 + (K-1)/2 columns; plan[8] = pairs of dx rows per pass (one
 * launch); plan[9] = (K-1)/2 + plan[8], the dy rows one pass holds (the ring
 * keeps (n_stage - 1) * stage_rows >= plan[9] - 1); plan[10] = dx rows per
 * pass.  Weight gradient: strips over dy [N,P,Q,C]; a stage holds
 * stage_rows dy rows and 2*stage_rows x rows of 62 + K columns; plan[8] =
 * launches, plan[9] = tap rows of the tallest launch, plan[10] = dy rows a
 * consumer step takes (the step holds 2*(plan[10] - 1) + plan[9] x rows, and
 * the ring keeps (n_stage - 1) * 2 * stage_rows >= that - 1).
 * No counterpart in the reference. */
TDC_API int tdc_dwconv_bwd_s2_plan(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                   int64_t pad, int64_t n_stage, int64_t which, int64_t sms,
                                   int64_t ctas_per_sm, int64_t* plan);

/* Number of rows of the stall tensor that tdc_dwconv_ws_probe writes for
 * this problem (= number of CTAs the launch uses). */
TDC_API int tdc_ws_probe_blocks(int64_t N, int64_t H, int64_t W, int64_t C,
                                int64_t pad, int64_t n_stage, int64_t* num_blocks);

/* Consumer warps per CTA of the ws kernel (the divisor for column 1 and 3 of
 * the stall tensor when a per-warp figure is wanted). */
TDC_API int tdc_ws_consumer_warps(void);

/* Resident CTAs per SM of a ws kernel instantiation on the current device
 * (kind 0 = ws, 1 = ws probe, 2 = general forward without epilogue / data
 * gradient, 3 = general forward with an epilogue) and the
 * device's SM count: the inputs tdc_ws_plan takes. */
TDC_API int tdc_ws_occupancy(int64_t n_stage, int64_t kind, int64_t* ctas_per_sm, int64_t* sms);

/* Launch plan the ws kernel would use on a device with `sms` SMs and
 * `ctas_per_sm` resident CTAs (pure host arithmetic, no CUDA call):
 * plan[0..8] = {stage_rows, qstrips, cblocks, strips, full_units,
 * tail_band_rows, grid, dynamic smem bytes, tail_chunk_rows}: strips below
 * full_units are dealt whole, round-robin.  With tail_chunk_rows = 0 the rest
 * are cut into bands of tail_band_rows rows (the last band may be shorter)
 * and dealt the same way, band-major.  With tail_chunk_rows = L > 0 the rest
 * form (strips - full_units) / cblocks pixel strips whose rows, one pixel
 * strip after the other, are cut into chunks of L rows: CTA g takes channel
 * block g % cblocks of chunk g / cblocks (grid is then a multiple of
 * cblocks).  `plan` holds 9 values.  No counterpart in the reference (whose
 * grid is fixed at (ceil(P/8), C/64, N), csrc/kernel_tma_ws.cu:25-31);
 * exposed so the planner can be checked without a GPU. */
TDC_API int tdc_ws_plan(int64_t N, int64_t H, int64_t W, int64_t C, int64_t pad,
                        int64_t n_stage, int64_t sms, int64_t ctas_per_sm, int64_t* plan);

/* Same computation as tdc_dwconv_ws, instrumented with clock64() around the
 * pipeline waits.  `stall` is a caller-owned, zero-initialised device array of
 * num_blocks*4 uint64 (num_blocks from tdc_ws_probe_blocks); cycles are
 * atomically ADDED, per CTA row b:
 *   stall[4b+0] producer cycles waiting on the empty barriers
 *   stall[4b+1] consumer cycles waiting on the full barriers, summed over warps
 *   stall[4b+2] producer lifetime (cycles)
 *   stall[4b+3] consumer lifetime, summed over consumer warps
 * Replaces tma_dwconv::dwconv_ws_probe (csrc/bindings.cpp:9-10,
 * csrc/kernel_tma_ws.cu:410-452), with y and stall supplied by the caller. */
TDC_API int tdc_dwconv_ws_probe(const void* x, const void* w, void* y,
                                int64_t N, int64_t H, int64_t W, int64_t C,
                                int64_t R, int64_t S, int64_t pad, int64_t n_stage,
                                unsigned long long* stall, void* stream);

/* ---- pipeline-wait failure detection ----------------------------------------
 * Every mbarrier wait in the ws kernels is bounded.  A wait that exceeds the
 * limit records a TDC_DEVICE_* code in a per-device status word, tells the
 * other warps of its CTA to stop, waits (bounded) for the CTA's own TMA copies
 * still in flight, and returns.  The CUDA context stays usable, but that
 * launch's output is incomplete.
 *
 * The first such failure on a device is also written through to pinned host
 * memory that the GPU maps (one page for the process, created by the first
 * call that launches a pipelined kernel; tdc_dwconv3x3_bwd_weight_noalloc
 * never creates it).  Every later entry point that launches work reads it
 * on entry, without synchronising, and returns TDC_ERR_DEVICE_TIMEOUT before
 * launching anything while a failure is recorded, until tdc_device_status
 * (clear != 0) resets it.  It sees the failures of launches that have
 * finished by the time of the call; a failure of a launch still running is
 * reported by the first call after it finishes.  (The reference spins on its
 * barriers without a bound, csrc/kernel_tma_ws.cuh:167,199.) */
#define TDC_DEVICE_OK               0
#define TDC_DEVICE_FULL_TIMEOUT     1  /* consumer waited too long for a filled stage */
#define TDC_DEVICE_EMPTY_TIMEOUT    2  /* producer waited too long for a free stage   */
#define TDC_DEVICE_DRAIN_TIMEOUT    3  /* an issued TMA copy never completed          */

/* Wait limit used by subsequent launches from this process (default 2 s). */
TDC_API int tdc_set_wait_timeout_ns(int64_t ns);

/* Reads (and if clear != 0, resets) the status word of the CURRENT device
 * and its host copy.  Synchronises the device.  info[0..3] (may be NULL)
 * receives {code, block, stage, load index} of the first failure recorded;
 * returns TDC_ERR_DEVICE_TIMEOUT when there is one (with clear != 0, later
 * calls run again). */
TDC_API int tdc_device_status(int clear, int64_t* info);

/* ws launch in which the producer withholds load number `withhold_load`
 * (counting from 0 in the order a CTA issues them; -1 = withhold none), so
 * the consumer's wait for that stage runs out after `timeout_ns`.  It exists
 * to test the bounded-wait path: the kernel reports
 * TDC_DEVICE_FULL_TIMEOUT through tdc_device_status and returns.  No GPU
 * fault, trap or unbounded wait is involved. */
TDC_API int tdc_dwconv_ws_withhold(const void* x, const void* w, void* y,
                                   int64_t N, int64_t H, int64_t W, int64_t C,
                                   int64_t pad, int64_t n_stage,
                                   int64_t withhold_load, int64_t timeout_ns,
                                   void* stream);

#ifdef __cplusplus
}  /* extern "C" */
#endif

#endif  /* TDC_DWCONV_H_ */
