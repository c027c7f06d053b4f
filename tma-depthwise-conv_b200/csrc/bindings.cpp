// bindings.cpp — the `_tma_dwconv_C` PyTorch extension.
//
// Same module surface as the reference's csrc/bindings.cpp:13-26 (functions
// dwconv_v0 / dwconv_ws / dwconv_ws_probe with keyword arguments
// x, w, pad[, n_stage]) and the same TORCH_CHECK messages as its host
// launchers (csrc/kernel_v0_naive_float4.cu:79-94, csrc/kernel_tma_ws.cu:54-65,
// 369-380).  Output tensors are allocated here with torch's caching allocator
// on x's device; the computation goes through the C ABI of libtdc_sm100.so
// (include/tdc_dwconv.h) on torch's current stream.
#include <torch/extension.h>
#include <ATen/cuda/CUDAContext.h>
#include <c10/cuda/CUDAGuard.h>

#include <optional>
#include <tuple>

#include "tdc_dwconv.h"

namespace tma_dwconv {
namespace {

void check_common(const torch::Tensor& x, const torch::Tensor& w) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda(), "tensors must live on CUDA");
  TORCH_CHECK(x.scalar_type() == torch::kHalf, "x must be fp16");
  TORCH_CHECK(w.scalar_type() == torch::kHalf, "w must be fp16");
  TORCH_CHECK(x.dim() == 4, "x must be [N,H,W,C]");
  TORCH_CHECK(w.dim() == 3, "w must be [R,S,C]");
  TORCH_CHECK(x.is_contiguous() && w.is_contiguous(), "x/w must be contiguous");
  TORCH_CHECK(x.device() == w.device(), "x and w must be on the same device");
}

// The K x K forward and the backward take fp16 or bfloat16 (x and w alike);
// returns true for bfloat16.
bool check_common_16(const torch::Tensor& x, const torch::Tensor& w, const char* xname) {
  TORCH_CHECK(x.is_cuda() && w.is_cuda(), "tensors must live on CUDA");
  TORCH_CHECK(x.scalar_type() == torch::kHalf || x.scalar_type() == torch::kBFloat16, xname,
              " must be fp16 or bf16");
  TORCH_CHECK(w.scalar_type() == x.scalar_type(), "w must have ", xname, "'s dtype");
  TORCH_CHECK(x.dim() == 4, xname, " must be 4-D NHWC");
  TORCH_CHECK(w.dim() == 3, "w must be [R,S,C]");
  TORCH_CHECK(x.is_contiguous() && w.is_contiguous(), xname, "/w must be contiguous");
  TORCH_CHECK(x.device() == w.device(), xname, " and w must be on the same device");
  return x.scalar_type() == torch::kBFloat16;
}

void check_status(int rc, const char* what) {
  if (rc == TDC_OK) return;
  if (rc == TDC_ERR_CUDA) {
    TORCH_CHECK(false, what, ": ", tdc_strerror(rc), ": ",
                cudaGetErrorString(static_cast<cudaError_t>(tdc_last_cuda_error())));
  }
  if (rc == TDC_ERR_TMA_ENCODE) {
    TORCH_CHECK(false, what, ": ", tdc_strerror(rc), " (CUresult ", tdc_last_cuda_error(), ")");
  }
  TORCH_CHECK(false, what, ": ", tdc_strerror(rc), " (status ", rc, ")");
}

void* stream_of(const torch::Tensor& x) {
  return static_cast<void*>(at::cuda::getCurrentCUDAStream(x.device().index()).stream());
}

void check_ws_args(const torch::Tensor& x, const torch::Tensor& w, int64_t pad) {
  check_common(x, w);
  TORCH_CHECK(w.size(0) == 3 && w.size(1) == 3, "only 3x3 kernel supported");
  TORCH_CHECK(w.size(2) == x.size(3), "channel mismatch");
  TORCH_CHECK(x.size(3) % 64 == 0, "C must be a multiple of BlockC=64");
  TORCH_CHECK(pad >= 0, "pad must be non-negative");
}

torch::Tensor alloc_out(const torch::Tensor& x, int64_t pad) {
  int64_t P = 0, Q = 0;
  check_status(tdc_output_hw(x.size(1), x.size(2), 3, 3, pad, &P, &Q), "output size");
  TORCH_CHECK(P >= 0 && Q >= 0, "input too small for a 3x3 kernel with pad ", pad);
  return torch::empty({x.size(0), P, Q, x.size(3)}, x.options());
}

}  // namespace

torch::Tensor dwconv_v0(torch::Tensor x, torch::Tensor w, int64_t pad) {
  check_common(x, w);
  TORCH_CHECK(w.size(0) == 3 && w.size(1) == 3, "Only 3x3 kernel supported in v0");
  TORCH_CHECK(x.size(3) == w.size(2), "channel mismatch between x and w");
  TORCH_CHECK(x.size(3) % 8 == 0, "C must be a multiple of VEC=8 (fp16 float4)");
  TORCH_CHECK(pad >= 0, "pad must be non-negative");
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = alloc_out(x, pad);
  check_status(tdc_dwconv_v0(x.data_ptr(), w.data_ptr(), y.data_ptr(), x.size(0), x.size(1),
                             x.size(2), x.size(3), w.size(0), w.size(1), pad, stream_of(x)),
               "dwconv_v0");
  return y;
}

torch::Tensor dwconv_ws(torch::Tensor x, torch::Tensor w, int64_t pad, int64_t n_stage) {
  check_ws_args(x, w, pad);
  TORCH_CHECK(n_stage >= 2 && n_stage <= 4, "n_stage must be one of {2, 3, 4}, got ", n_stage);
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = alloc_out(x, pad);
  check_status(tdc_dwconv_ws(x.data_ptr(), w.data_ptr(), y.data_ptr(), x.size(0), x.size(1),
                             x.size(2), x.size(3), 3, 3, pad, n_stage, stream_of(x)),
               "dwconv_ws");
  return y;
}

// Writes into a caller-provided y [N,P,Q,C] (no allocation on the call path).
torch::Tensor dwconv_ws_out(torch::Tensor x, torch::Tensor w, torch::Tensor y, int64_t pad,
                            int64_t n_stage) {
  check_ws_args(x, w, pad);
  TORCH_CHECK(n_stage >= 2 && n_stage <= 4, "n_stage must be one of {2, 3, 4}, got ", n_stage);
  int64_t P = 0, Q = 0;
  check_status(tdc_output_hw(x.size(1), x.size(2), 3, 3, pad, &P, &Q), "output size");
  TORCH_CHECK(y.is_cuda() && y.device() == x.device() && y.scalar_type() == torch::kHalf &&
                  y.is_contiguous() && y.dim() == 4 && y.size(0) == x.size(0) &&
                  y.size(1) == P && y.size(2) == Q && y.size(3) == x.size(3),
              "y must be a contiguous fp16 [N,P,Q,C] tensor on x's device");
  const c10::cuda::CUDAGuard guard(x.device());
  check_status(tdc_dwconv_ws(x.data_ptr(), w.data_ptr(), y.data_ptr(), x.size(0), x.size(1),
                             x.size(2), x.size(3), 3, 3, pad, n_stage, stream_of(x)),
               "dwconv_ws");
  return y;
}

std::tuple<torch::Tensor, torch::Tensor> dwconv_ws_probe(torch::Tensor x, torch::Tensor w,
                                                         int64_t pad, int64_t n_stage) {
  check_ws_args(x, w, pad);
  TORCH_CHECK(n_stage >= 2 && n_stage <= 4, "n_stage must be one of {2, 3, 4}, got ", n_stage);
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = alloc_out(x, pad);
  int64_t blocks = 0;
  check_status(tdc_ws_probe_blocks(x.size(0), x.size(1), x.size(2), x.size(3), pad, n_stage,
                                   &blocks),
               "dwconv_ws_probe");
  auto stall = torch::zeros({blocks, 4},
                            torch::TensorOptions().dtype(torch::kInt64).device(x.device()));
  check_status(
      tdc_dwconv_ws_probe(x.data_ptr(), w.data_ptr(), y.data_ptr(), x.size(0), x.size(1),
                          x.size(2), x.size(3), 3, 3, pad, n_stage,
                          reinterpret_cast<unsigned long long*>(stall.data_ptr<int64_t>()),
                          stream_of(x)),
      "dwconv_ws_probe");
  return {y, stall};
}

torch::Tensor dwconv_ws_withhold(torch::Tensor x, torch::Tensor w, int64_t pad, int64_t n_stage,
                                 int64_t withhold_load, int64_t timeout_ns) {
  check_ws_args(x, w, pad);
  TORCH_CHECK(n_stage >= 2 && n_stage <= 4, "n_stage must be one of {2, 3, 4}, got ", n_stage);
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = alloc_out(x, pad);
  check_status(tdc_dwconv_ws_withhold(x.data_ptr(), w.data_ptr(), y.data_ptr(), x.size(0),
                                      x.size(1), x.size(2), x.size(3), pad, n_stage,
                                      withhold_load, timeout_ns, stream_of(x)),
               "dwconv_ws_withhold");
  return y;
}

// General forward: C % 8, optional bias [C], activation, residual [N,P,Q,C]

torch::Tensor dwconv3x3(torch::Tensor x, torch::Tensor w, std::optional<torch::Tensor> bias,
                        std::optional<torch::Tensor> residual, int64_t pad, int64_t act,
                        int64_t n_stage) {
  check_common(x, w);
  TORCH_CHECK(w.size(0) == 3 && w.size(1) == 3, "only 3x3 kernel supported");
  TORCH_CHECK(w.size(2) == x.size(3), "channel mismatch");
  TORCH_CHECK(x.size(3) % 8 == 0, "C must be a multiple of 8");
  TORCH_CHECK(pad >= 0, "pad must be non-negative");
  TORCH_CHECK(n_stage >= 2 && n_stage <= 4, "n_stage must be one of {2, 3, 4}, got ", n_stage);
  const c10::cuda::CUDAGuard guard(x.device());
  auto y = alloc_out(x, pad);
  const void* bptr = nullptr;
  const void* rptr = nullptr;
  if (bias.has_value()) {
    const auto& b = *bias;
    TORCH_CHECK(b.is_cuda() && b.device() == x.device() && b.scalar_type() == torch::kHalf &&
                    b.is_contiguous() && b.dim() == 1 && b.size(0) == x.size(3),
                "bias must be a contiguous fp16 [C] tensor on x's device");
    bptr = b.data_ptr();
  }
  if (residual.has_value()) {
    const auto& r = *residual;
    TORCH_CHECK(r.is_cuda() && r.device() == x.device() && r.scalar_type() == torch::kHalf &&
                    r.is_contiguous() && r.sizes() == y.sizes(),
                "residual must be a contiguous fp16 [N,P,Q,C] tensor on x's device");
    rptr = r.data_ptr();
  }
  check_status(tdc_dwconv3x3_fwd(x.data_ptr(), w.data_ptr(), bptr, rptr, y.data_ptr(), x.size(0),
                                 x.size(1), x.size(2), x.size(3), pad, act, n_stage, stream_of(x)),
               "dwconv3x3");
  return y;
}

// K x K (K = 3, 5, 7), stride 1 or 2, with the same optional epilogue.
torch::Tensor dwconv_k(torch::Tensor x, torch::Tensor w, std::optional<torch::Tensor> bias,
                       std::optional<torch::Tensor> residual, int64_t stride, int64_t pad,
                       int64_t act, int64_t n_stage) {
  const bool bf16 = check_common_16(x, w, "x");
  const int64_t K = w.size(0);
  TORCH_CHECK(w.size(1) == K && (K == 3 || K == 5 || K == 7), "w must be [K,K,C] with K in {3, 5, 7}");
  TORCH_CHECK(w.size(2) == x.size(3), "channel mismatch");
  TORCH_CHECK(x.size(3) % 8 == 0, "C must be a multiple of 8");
  TORCH_CHECK(stride == 1 || stride == 2, "stride must be 1 or 2, got ", stride);
  TORCH_CHECK(pad >= 0, "pad must be non-negative");
  TORCH_CHECK(n_stage == 0 || (n_stage >= 2 && n_stage <= 4),
              "n_stage must be one of {2, 3, 4} (or 0: chosen from the shape), got ", n_stage);
  TORCH_CHECK(x.size(1) + 2 * pad >= K && x.size(2) + 2 * pad >= K, "input too small for a ", K,
              "x", K, " kernel with pad ", pad);
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t P = (x.size(1) + 2 * pad - K) / stride + 1;
  const int64_t Q = (x.size(2) + 2 * pad - K) / stride + 1;
  auto y = torch::empty({x.size(0), P, Q, x.size(3)}, x.options());
  const void* bptr = nullptr;
  const void* rptr = nullptr;
  if (bias.has_value()) {
    const auto& b = *bias;
    TORCH_CHECK(b.is_cuda() && b.device() == x.device() && b.scalar_type() == x.scalar_type() &&
                    b.is_contiguous() && b.dim() == 1 && b.size(0) == x.size(3),
                "bias must be a contiguous [C] tensor of x's dtype on x's device");
    bptr = b.data_ptr();
  }
  if (residual.has_value()) {
    const auto& r = *residual;
    TORCH_CHECK(r.is_cuda() && r.device() == x.device() && r.scalar_type() == x.scalar_type() &&
                    r.is_contiguous() && r.sizes() == y.sizes(),
                "residual must be a contiguous [N,P,Q,C] tensor of x's dtype on x's device");
    rptr = r.data_ptr();
  }
  auto* fwd = bf16 ? &tdc_dwconv_fwd_bf16 : &tdc_dwconv_fwd;
  check_status(fwd(x.data_ptr(), w.data_ptr(), bptr, rptr, y.data_ptr(), x.size(0), x.size(1),
                   x.size(2), x.size(3), K, stride, pad, act, n_stage, stream_of(x)),
               "dwconv");
  return y;
}

// dwconv_k with each side's padding given (top, bottom, left, right) and a
// dilation (1: the sliding-window kernels with n_stage; above 1: the dilated
// plain kernel, n_stage ignored).
torch::Tensor dwconv_k_pads(torch::Tensor x, torch::Tensor w, std::optional<torch::Tensor> bias,
                            std::optional<torch::Tensor> residual, int64_t stride,
                            int64_t dilation, int64_t pad_top, int64_t pad_bottom,
                            int64_t pad_left, int64_t pad_right, int64_t act, int64_t n_stage) {
  const bool bf16 = check_common_16(x, w, "x");
  const int64_t K = w.size(0);
  TORCH_CHECK(w.size(1) == K && (K == 3 || K == 5 || K == 7), "w must be [K,K,C] with K in {3, 5, 7}");
  TORCH_CHECK(w.size(2) == x.size(3), "channel mismatch");
  TORCH_CHECK(x.size(3) % 8 == 0, "C must be a multiple of 8");
  TORCH_CHECK(stride == 1 || stride == 2, "stride must be 1 or 2, got ", stride);
  TORCH_CHECK(pad_top >= 0 && pad_bottom >= 0 && pad_left >= 0 && pad_right >= 0,
              "pads must be non-negative");
  TORCH_CHECK(n_stage == 0 || (n_stage >= 2 && n_stage <= 4),
              "n_stage must be one of {2, 3, 4} (or 0: chosen from the shape), got ", n_stage);
  TORCH_CHECK(dilation >= 1, "dilation must be >= 1, got ", dilation);
  const int64_t Ke = dilation * (K - 1) + 1;
  TORCH_CHECK(x.size(1) + pad_top + pad_bottom >= Ke && x.size(2) + pad_left + pad_right >= Ke,
              "input too small for a ", K, "x", K, " kernel (dilation ", dilation,
              ") with these pads");
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t P = (x.size(1) + pad_top + pad_bottom - Ke) / stride + 1;
  const int64_t Q = (x.size(2) + pad_left + pad_right - Ke) / stride + 1;
  auto y = torch::empty({x.size(0), P, Q, x.size(3)}, x.options());
  const void* bptr = nullptr;
  const void* rptr = nullptr;
  if (bias.has_value()) {
    const auto& b = *bias;
    TORCH_CHECK(b.is_cuda() && b.device() == x.device() && b.scalar_type() == x.scalar_type() &&
                    b.is_contiguous() && b.dim() == 1 && b.size(0) == x.size(3),
                "bias must be a contiguous [C] tensor of x's dtype on x's device");
    bptr = b.data_ptr();
  }
  if (residual.has_value()) {
    const auto& r = *residual;
    TORCH_CHECK(r.is_cuda() && r.device() == x.device() && r.scalar_type() == x.scalar_type() &&
                    r.is_contiguous() && r.sizes() == y.sizes(),
                "residual must be a contiguous [N,P,Q,C] tensor of x's dtype on x's device");
    rptr = r.data_ptr();
  }
  if (dilation == 1) {
    auto* fwd = bf16 ? &tdc_dwconv_fwd_asym_bf16 : &tdc_dwconv_fwd_asym;
    check_status(fwd(x.data_ptr(), w.data_ptr(), bptr, rptr, y.data_ptr(), x.size(0), x.size(1),
                     x.size(2), x.size(3), K, stride, pad_top, pad_bottom, pad_left, pad_right,
                     act, n_stage, stream_of(x)),
                 "dwconv_k_pads");
  } else {
    auto* fwd = bf16 ? &tdc_dwconv_fwd_dilated_bf16 : &tdc_dwconv_fwd_dilated;
    check_status(fwd(x.data_ptr(), w.data_ptr(), bptr, rptr, y.data_ptr(), x.size(0), x.size(1),
                     x.size(2), x.size(3), K, stride, dilation, pad_top, pad_bottom, pad_left,
                     pad_right, act, stream_of(x)),
                 "dwconv_k_pads");
  }
  return y;
}

// The plain K x K forward (no TMA): same checks and epilogue as dwconv_k,
// band_rows (0 = from the shape) in place of n_stage.
torch::Tensor dwconv_plain(torch::Tensor x, torch::Tensor w, std::optional<torch::Tensor> bias,
                           std::optional<torch::Tensor> residual, int64_t stride, int64_t pad,
                           int64_t act, int64_t band_rows) {
  const bool bf16 = check_common_16(x, w, "x");
  const int64_t K = w.size(0);
  TORCH_CHECK(w.size(1) == K && (K == 3 || K == 5 || K == 7), "w must be [K,K,C] with K in {3, 5, 7}");
  TORCH_CHECK(w.size(2) == x.size(3), "channel mismatch");
  TORCH_CHECK(x.size(3) % 8 == 0, "C must be a multiple of 8");
  TORCH_CHECK(stride == 1 || stride == 2, "stride must be 1 or 2, got ", stride);
  TORCH_CHECK(pad >= 0, "pad must be non-negative");
  TORCH_CHECK(band_rows >= 0, "band_rows must be non-negative (0: chosen from the shape)");
  TORCH_CHECK(x.size(1) + 2 * pad >= K && x.size(2) + 2 * pad >= K, "input too small for a ", K,
              "x", K, " kernel with pad ", pad);
  const c10::cuda::CUDAGuard guard(x.device());
  const int64_t P = (x.size(1) + 2 * pad - K) / stride + 1;
  const int64_t Q = (x.size(2) + 2 * pad - K) / stride + 1;
  auto y = torch::empty({x.size(0), P, Q, x.size(3)}, x.options());
  const void* bptr = nullptr;
  const void* rptr = nullptr;
  if (bias.has_value()) {
    const auto& b = *bias;
    TORCH_CHECK(b.is_cuda() && b.device() == x.device() && b.scalar_type() == x.scalar_type() &&
                    b.is_contiguous() && b.dim() == 1 && b.size(0) == x.size(3),
                "bias must be a contiguous [C] tensor of x's dtype on x's device");
    bptr = b.data_ptr();
  }
  if (residual.has_value()) {
    const auto& r = *residual;
    TORCH_CHECK(r.is_cuda() && r.device() == x.device() && r.scalar_type() == x.scalar_type() &&
                    r.is_contiguous() && r.sizes() == y.sizes(),
                "residual must be a contiguous [N,P,Q,C] tensor of x's dtype on x's device");
    rptr = r.data_ptr();
  }
  auto* fwd = bf16 ? &tdc_dwconv_fwd_plain_bf16 : &tdc_dwconv_fwd_plain;
  check_status(fwd(x.data_ptr(), w.data_ptr(), bptr, rptr, y.data_ptr(), x.size(0), x.size(1),
                   x.size(2), x.size(3), K, stride, pad, act, band_rows, stream_of(x)),
               "dwconv_plain");
  return y;
}

// The plain weight gradient (no TMA; workspace per channel chunk).
torch::Tensor dwconv_bwd_weight_plain(torch::Tensor x, torch::Tensor dy, int64_t K, int64_t pad,
                                      int64_t stride) {
  TORCH_CHECK(x.is_cuda() && dy.is_cuda() && x.device() == dy.device(), "tensors must live on CUDA");
  TORCH_CHECK((x.scalar_type() == torch::kHalf || x.scalar_type() == torch::kBFloat16) &&
                  dy.scalar_type() == x.scalar_type(),
              "x and dy must be both fp16 or both bf16");
  const bool bf16 = x.scalar_type() == torch::kBFloat16;
  TORCH_CHECK(x.dim() == 4 && dy.dim() == 4 && x.is_contiguous() && dy.is_contiguous(),
              "x and dy must be contiguous [N,H,W,C] / [N,P,Q,C]");
  TORCH_CHECK(K == 3 || K == 5 || K == 7, "K must be 3, 5 or 7, got ", K);
  TORCH_CHECK(stride == 1 || stride == 2, "stride must be 1 or 2, got ", stride);
  TORCH_CHECK(x.size(3) % 8 == 0, "C must be a multiple of 8");
  TORCH_CHECK(pad >= 0, "pad must be non-negative");
  TORCH_CHECK(x.size(1) + 2 * pad >= K && x.size(2) + 2 * pad >= K,
              "x is smaller than a ", K, "x", K, " kernel with pad ", pad, " needs");
  TORCH_CHECK(dy.size(0) == x.size(0) && dy.size(3) == x.size(3) &&
                  dy.size(1) == (x.size(1) + 2 * pad - K) / stride + 1 &&
                  dy.size(2) == (x.size(2) + 2 * pad - K) / stride + 1,
              "dy must be [N, (H+2*pad-K)/stride+1, (W+2*pad-K)/stride+1, C]");
  const c10::cuda::CUDAGuard guard(x.device());
  auto dw = torch::empty({K, K, x.size(3)}, x.options().dtype(torch::kFloat32));
  if (x.size(3) == 0) return dw;
  int64_t bytes = 0;
  check_status(tdc_dwconv_bwd_weight_plain_workspace(x.size(0), x.size(1), x.size(2), x.size(3),
                                                     K, stride, pad, &bytes),
               "dwconv_bwd_weight_plain");
  auto ws = torch::empty({std::max<int64_t>(4, (bytes + 3) / 4)}, x.options().dtype(torch::kFloat32));
  auto* bwd = bf16 ? &tdc_dwconv_bwd_weight_plain_bf16 : &tdc_dwconv_bwd_weight_plain;
  check_status(bwd(x.data_ptr(), dy.data_ptr(), dw.data_ptr<float>(), x.size(0), x.size(1),
                   x.size(2), x.size(3), K, stride, pad, ws.data_ptr(), bytes, stream_of(x)),
               "dwconv_bwd_weight_plain");
  return dw;
}

// Data gradient: dy [N,P,Q,C] -> dx [N,H,W,C] with H = P - 2*pad + 2.
torch::Tensor dwconv3x3_bwd_data(torch::Tensor dy, torch::Tensor w, int64_t pad, int64_t n_stage) {
  check_common(dy, w);
  TORCH_CHECK(w.size(0) == 3 && w.size(1) == 3 && w.size(2) == dy.size(3), "w must be [3,3,C]");
  TORCH_CHECK(dy.size(3) % 8 == 0, "C must be a multiple of 8");
  TORCH_CHECK(pad >= 0, "pad must be non-negative");
  const int64_t H = dy.size(1) - 2 * pad + 2, W = dy.size(2) - 2 * pad + 2;
  TORCH_CHECK(H >= 1 && W >= 1, "dy is smaller than a 3x3 kernel with pad ", pad, " can produce");
  const c10::cuda::CUDAGuard guard(dy.device());
  auto dx = torch::empty({dy.size(0), H, W, dy.size(3)}, dy.options());
  if (dx.numel() == 0 || dy.numel() == 0) return dx.zero_();
  check_status(tdc_dwconv3x3_bwd_data(dy.data_ptr(), w.data_ptr(), dx.data_ptr(), dy.size(0), H, W,
                                      dy.size(3), pad, n_stage, stream_of(dy)),
               "dwconv3x3_bwd_data");
  return dx;
}

// Weight gradient: x [N,H,W,C], dy [N,P,Q,C] -> dw [3,3,C] fp32 (workspace from
// torch's caching allocator).
torch::Tensor dwconv3x3_bwd_weight(torch::Tensor x, torch::Tensor dy, int64_t pad, int64_t n_stage) {
  TORCH_CHECK(x.is_cuda() && dy.is_cuda() && x.device() == dy.device(), "tensors must live on CUDA");
  TORCH_CHECK(x.scalar_type() == torch::kHalf && dy.scalar_type() == torch::kHalf,
              "x and dy must be fp16");
  TORCH_CHECK(x.dim() == 4 && dy.dim() == 4 && x.is_contiguous() && dy.is_contiguous(),
              "x and dy must be contiguous [N,H,W,C] / [N,P,Q,C]");
  TORCH_CHECK(x.size(3) % 8 == 0, "C must be a multiple of 8");
  TORCH_CHECK(pad >= 0, "pad must be non-negative");
  TORCH_CHECK(dy.size(0) == x.size(0) && dy.size(3) == x.size(3) &&
                  dy.size(1) == x.size(1) + 2 * pad - 2 && dy.size(2) == x.size(2) + 2 * pad - 2,
              "dy must be [N, H+2*pad-2, W+2*pad-2, C]");
  const c10::cuda::CUDAGuard guard(x.device());
  auto dw = torch::zeros({3, 3, x.size(3)}, x.options().dtype(torch::kFloat32));
  if (x.numel() == 0 || dy.numel() == 0) return dw;
  int64_t bytes = 0;
  check_status(tdc_dwconv3x3_bwd_weight_workspace(x.size(0), x.size(1), x.size(2), x.size(3), pad,
                                                  n_stage, &bytes),
               "dwconv3x3_bwd_weight");
  auto ws = torch::empty({(bytes + 3) / 4}, x.options().dtype(torch::kFloat32));
  check_status(tdc_dwconv3x3_bwd_weight(x.data_ptr(), dy.data_ptr(), dw.data_ptr<float>(),
                                        x.size(0), x.size(1), x.size(2), x.size(3), pad, n_stage,
                                        ws.data_ptr(), bytes, stream_of(x)),
               "dwconv3x3_bwd_weight");
  return dw;
}

// Backward of the K x K forward (K = 3, 5, 7) at stride 1 or 2.  At stride 2
// the input height / width are not determined by dy (two sizes give the same
// output); input_h / input_w < 0 pick the smaller one.
torch::Tensor dwconv_bwd_data(torch::Tensor dy, torch::Tensor w, int64_t pad, int64_t stride,
                              int64_t n_stage, int64_t input_h, int64_t input_w) {
  const bool bf16 = check_common_16(dy, w, "dy");
  const int64_t K = w.size(0);
  TORCH_CHECK(w.size(1) == K && (K == 3 || K == 5 || K == 7) && w.size(2) == dy.size(3),
              "w must be [K,K,C] with K in {3, 5, 7}");
  TORCH_CHECK(stride == 1 || stride == 2, "stride must be 1 or 2, got ", stride);
  TORCH_CHECK(dy.size(3) % 8 == 0, "C must be a multiple of 8");
  TORCH_CHECK(pad >= 0, "pad must be non-negative");
  int64_t H, W;
  if (stride == 1) {
    TORCH_CHECK((K == 3 && !bf16) || pad <= K - 1, "the ", K, "x", K,
                " data gradient needs pad <= ", K - 1);
    H = dy.size(1) - 2 * pad + K - 1;
    W = dy.size(2) - 2 * pad + K - 1;
    TORCH_CHECK(input_h < 0 || input_h == H, "input_h ", input_h, " does not match dy");
    TORCH_CHECK(input_w < 0 || input_w == W, "input_w ", input_w, " does not match dy");
  } else {
    TORCH_CHECK(dy.size(1) >= 1 && dy.size(2) >= 1, "dy must have at least one row and column");
    H = input_h >= 0 ? input_h : 2 * (dy.size(1) - 1) + K - 2 * pad;
    W = input_w >= 0 ? input_w : 2 * (dy.size(2) - 1) + K - 2 * pad;
    TORCH_CHECK(H + 2 * pad >= K && W + 2 * pad >= K &&
                    (H + 2 * pad - K) / 2 + 1 == dy.size(1) &&
                    (W + 2 * pad - K) / 2 + 1 == dy.size(2),
                "dy [", dy.size(1), ", ", dy.size(2), "] is not the stride-2 output of a ", H,
                "x", W, " input with pad ", pad);
  }
  TORCH_CHECK(H >= 1 && W >= 1, "dy is smaller than a ", K, "x", K, " kernel with pad ", pad,
              " can produce");
  const c10::cuda::CUDAGuard guard(dy.device());
  auto dx = torch::empty({dy.size(0), H, W, dy.size(3)}, dy.options());
  if (dx.numel() == 0 || dy.numel() == 0) return dx.zero_();
  auto* bwd = bf16 ? &tdc_dwconv_bwd_data_bf16 : &tdc_dwconv_bwd_data;
  check_status(bwd(dy.data_ptr(), w.data_ptr(), dx.data_ptr(), dy.size(0), H, W, dy.size(3), K,
                   stride, pad, n_stage, stream_of(dy)),
               "dwconv_bwd_data");
  return dx;
}

torch::Tensor dwconv_bwd_weight(torch::Tensor x, torch::Tensor dy, int64_t K, int64_t pad,
                                int64_t stride, int64_t n_stage) {
  TORCH_CHECK(x.is_cuda() && dy.is_cuda() && x.device() == dy.device(), "tensors must live on CUDA");
  TORCH_CHECK((x.scalar_type() == torch::kHalf || x.scalar_type() == torch::kBFloat16) &&
                  dy.scalar_type() == x.scalar_type(),
              "x and dy must be both fp16 or both bf16");
  const bool bf16 = x.scalar_type() == torch::kBFloat16;
  TORCH_CHECK(x.dim() == 4 && dy.dim() == 4 && x.is_contiguous() && dy.is_contiguous(),
              "x and dy must be contiguous [N,H,W,C] / [N,P,Q,C]");
  TORCH_CHECK(K == 3 || K == 5 || K == 7, "K must be 3, 5 or 7, got ", K);
  TORCH_CHECK(stride == 1 || stride == 2, "stride must be 1 or 2, got ", stride);
  TORCH_CHECK(x.size(3) % 8 == 0, "C must be a multiple of 8");
  TORCH_CHECK(pad >= 0, "pad must be non-negative");
  TORCH_CHECK(x.size(1) + 2 * pad >= K && x.size(2) + 2 * pad >= K,
              "x is smaller than a ", K, "x", K, " kernel with pad ", pad, " needs");
  TORCH_CHECK(dy.size(0) == x.size(0) && dy.size(3) == x.size(3) &&
                  dy.size(1) == (x.size(1) + 2 * pad - K) / stride + 1 &&
                  dy.size(2) == (x.size(2) + 2 * pad - K) / stride + 1,
              "dy must be [N, (H+2*pad-K)/stride+1, (W+2*pad-K)/stride+1, C]");
  const c10::cuda::CUDAGuard guard(x.device());
  // Every kernel path writes all of dw; only an empty problem needs zeros.
  if (x.numel() == 0 || dy.numel() == 0)
    return torch::zeros({K, K, x.size(3)}, x.options().dtype(torch::kFloat32));
  auto dw = torch::empty({K, K, x.size(3)}, x.options().dtype(torch::kFloat32));
  int64_t bytes = 0;
  auto* wsq = bf16 ? &tdc_dwconv_bwd_weight_workspace_bf16 : &tdc_dwconv_bwd_weight_workspace;
  check_status(wsq(x.size(0), x.size(1), x.size(2), x.size(3), K, stride, pad, n_stage, &bytes),
               "dwconv_bwd_weight");
  auto ws = torch::empty({(bytes + 3) / 4}, x.options().dtype(torch::kFloat32));
  auto* bwd = bf16 ? &tdc_dwconv_bwd_weight_bf16 : &tdc_dwconv_bwd_weight;
  check_status(bwd(x.data_ptr(), dy.data_ptr(), dw.data_ptr<float>(), x.size(0), x.size(1),
                   x.size(2), x.size(3), K, stride, pad, n_stage, ws.data_ptr(), bytes,
                   stream_of(x)),
               "dwconv_bwd_weight");
  return dw;
}

// ws forward on host tensors, pipelined over chunks of images (see
// tdc_dwconv_ws_host): x_host / w_host / y_host are CPU tensors (pinned for
// overlap), x_dev / w_dev / y_dev device buffers of the same shapes on the
// current device; returns y_host.
torch::Tensor dwconv_ws_host(torch::Tensor x_host, torch::Tensor w_host, torch::Tensor y_host,
                             torch::Tensor x_dev, torch::Tensor w_dev, torch::Tensor y_dev,
                             int64_t pad, int64_t n_stage, int64_t chunk_images) {
  TORCH_CHECK(!x_host.is_cuda() && !w_host.is_cuda() && !y_host.is_cuda(),
              "x_host, w_host and y_host must be CPU tensors");
  TORCH_CHECK(x_dev.is_cuda() && w_dev.is_cuda() && y_dev.is_cuda() &&
                  x_dev.device() == w_dev.device() && x_dev.device() == y_dev.device(),
              "x_dev, w_dev and y_dev must live on one CUDA device");
  for (const auto* t : {&x_host, &w_host, &y_host, &x_dev, &w_dev, &y_dev})
    TORCH_CHECK(t->scalar_type() == torch::kHalf && t->is_contiguous(),
                "host and device tensors must be contiguous fp16");
  TORCH_CHECK(x_host.sizes() == x_dev.sizes() && w_host.sizes() == w_dev.sizes() &&
                  y_host.sizes() == y_dev.sizes(),
              "host and device tensors must have the same shapes");
  check_ws_args(x_dev, w_dev, pad);
  int64_t P = 0, Q = 0;
  check_status(tdc_output_hw(x_dev.size(1), x_dev.size(2), 3, 3, pad, &P, &Q), "output size");
  TORCH_CHECK(y_dev.dim() == 4 && y_dev.size(0) == x_dev.size(0) && y_dev.size(1) == P &&
                  y_dev.size(2) == Q && y_dev.size(3) == x_dev.size(3),
              "y must be [N, P, Q, C]");
  const c10::cuda::CUDAGuard guard(x_dev.device());
  check_status(tdc_dwconv_ws_host(x_host.data_ptr(), w_host.data_ptr(), y_host.data_ptr(),
                                  x_dev.size(0), x_dev.size(1), x_dev.size(2), x_dev.size(3), pad,
                                  n_stage, x_dev.data_ptr(), w_dev.data_ptr(), y_dev.data_ptr(),
                                  chunk_images, stream_of(x_dev)),
               "dwconv_ws_host");
  return y_host;
}

// (code, block, stage, load) of the first pipeline-wait failure recorded on
// `device` since the last clear; code 0 = none.  Synchronises the device.
std::tuple<int64_t, int64_t, int64_t, int64_t> device_status(int64_t device, bool clear) {
  const c10::cuda::CUDAGuard guard(static_cast<c10::DeviceIndex>(device));
  int64_t info[4] = {0, 0, 0, 0};
  const int rc = tdc_device_status(clear ? 1 : 0, info);
  if (rc != TDC_OK && rc != TDC_ERR_DEVICE_TIMEOUT) check_status(rc, "device_status");
  return {info[0], info[1], info[2], info[3]};
}

void set_wait_timeout_ns(int64_t ns) { check_status(tdc_set_wait_timeout_ns(ns), "set_wait_timeout_ns"); }

int64_t consumer_warps() { return tdc_ws_consumer_warps(); }

}  // namespace tma_dwconv

PYBIND11_MODULE(TORCH_EXTENSION_NAME, m) {
  m.def("dwconv_v0", &tma_dwconv::dwconv_v0,
        "Depthwise conv2d NHWC, plain direct-load kernel (v0 surface).", pybind11::arg("x"),
        pybind11::arg("w"), pybind11::arg("pad"));
  m.def("dwconv_ws", &tma_dwconv::dwconv_ws,
        "Depthwise conv2d NHWC, TMA + warp-specialised ring of n_stage stages.",
        pybind11::arg("x"), pybind11::arg("w"), pybind11::arg("pad"), pybind11::arg("n_stage"));
  m.def("dwconv_ws_probe", &tma_dwconv::dwconv_ws_probe,
        "Same as dwconv_ws, also returns a per-CTA stall-cycle tensor of shape "
        "[num_blocks, 4] (cols: producer empty-wait, consumer full-wait summed over "
        "consumer warps, producer lifetime, consumer lifetime summed over consumer warps).",
        pybind11::arg("x"), pybind11::arg("w"), pybind11::arg("pad"), pybind11::arg("n_stage"));
  m.def("dwconv_ws_out", &tma_dwconv::dwconv_ws_out,
        "dwconv_ws into a preallocated y [N,P,Q,C]; returns y.", pybind11::arg("x"),
        pybind11::arg("w"), pybind11::arg("y"), pybind11::arg("pad"), pybind11::arg("n_stage"));
  m.def("dwconv_ws_host", &tma_dwconv::dwconv_ws_host,
        "dwconv_ws on host tensors: H2D copies, kernels and D2H copies pipelined over chunks "
        "of images; returns y_host.",
        pybind11::arg("x_host"), pybind11::arg("w_host"), pybind11::arg("y_host"),
        pybind11::arg("x_dev"), pybind11::arg("w_dev"), pybind11::arg("y_dev"), pybind11::arg("pad"),
        pybind11::arg("n_stage"), pybind11::arg("chunk_images") = 0);
  m.def("dwconv_ws_withhold", &tma_dwconv::dwconv_ws_withhold,
        "dwconv_ws whose producer withholds one load so the consumer's bounded wait runs out "
        "(tests the failure path; see device_status).",
        pybind11::arg("x"), pybind11::arg("w"), pybind11::arg("pad"), pybind11::arg("n_stage"),
        pybind11::arg("withhold_load"), pybind11::arg("timeout_ns"));
  m.def("dwconv_k", &tma_dwconv::dwconv_k,
        "K x K (3, 5, 7) depthwise forward, stride 1 or 2, optional fused epilogue",
        py::arg("x"), py::arg("w"), py::arg("bias"), py::arg("residual"), py::arg("stride"),
        py::arg("pad"), py::arg("act"), py::arg("n_stage"));
  m.def("dwconv_k_pads", &tma_dwconv::dwconv_k_pads,
        "K x K depthwise forward with each side's padding (top, bottom, left, right) and a "
        "dilation",
        py::arg("x"), py::arg("w"), py::arg("bias"), py::arg("residual"), py::arg("stride"),
        py::arg("dilation"), py::arg("pad_top"), py::arg("pad_bottom"), py::arg("pad_left"),
        py::arg("pad_right"), py::arg("act"), py::arg("n_stage"));
  m.def("dwconv_plain", &tma_dwconv::dwconv_plain,
        "plain (no TMA) K x K depthwise forward, the same result as dwconv_k",
        py::arg("x"), py::arg("w"), py::arg("bias"), py::arg("residual"), py::arg("stride"),
        py::arg("pad"), py::arg("act"), py::arg("band_rows"));
  m.def("dwconv_bwd_weight_plain", &tma_dwconv::dwconv_bwd_weight_plain,
        "plain (no TMA) weight gradient dw [K,K,C] fp32, deterministic",
        py::arg("x"), py::arg("dy"), py::arg("K"), py::arg("pad"), py::arg("stride"));
  m.def("dwconv_bwd_weight_uses_plain",
        [](int64_t N, int64_t H, int64_t W, int64_t C, int64_t K, int64_t stride, int64_t pad) {
          return tdc_dwconv_bwd_weight_uses_plain(N, H, W, C, K, stride, pad) != 0;
        },
        "whether dwconv_bwd_weight with n_stage 0 runs the plain kernel on this shape");
  m.def("dwconv_uses_plain",
        [](int64_t N, int64_t H, int64_t W, int64_t C, int64_t K, int64_t stride, int64_t pad) {
          return tdc_dwconv_fwd_uses_plain(N, H, W, C, K, stride, pad) != 0;
        },
        "whether dwconv_k with n_stage 0 runs the plain kernel on this shape");
  m.def("dwconv3x3", &tma_dwconv::dwconv3x3,
        "General forward: C % 8, fused bias / activation / residual epilogue.",
        pybind11::arg("x"), pybind11::arg("w"), pybind11::arg("bias"), pybind11::arg("residual"),
        pybind11::arg("pad"), pybind11::arg("act"), pybind11::arg("n_stage"));
  m.def("dwconv3x3_bwd_data", &tma_dwconv::dwconv3x3_bwd_data,
        "Data gradient of the 3x3 forward: dx [N,H,W,C] from dy [N,P,Q,C].", pybind11::arg("dy"),
        pybind11::arg("w"), pybind11::arg("pad"), pybind11::arg("n_stage") = 2);
  m.def("dwconv3x3_bwd_weight", &tma_dwconv::dwconv3x3_bwd_weight,
        "Weight gradient of the 3x3 forward: dw [3,3,C] fp32 (deterministic).", pybind11::arg("x"),
        pybind11::arg("dy"), pybind11::arg("pad"), pybind11::arg("n_stage") = 2);
  m.def("dwconv_bwd_data", &tma_dwconv::dwconv_bwd_data,
        "Data gradient of the K x K forward (stride 1 or 2): dx [N,H,W,C] from dy [N,P,Q,C]; "
        "input_h / input_w give H, W at stride 2 (default: the smaller size that fits dy).",
        pybind11::arg("dy"), pybind11::arg("w"), pybind11::arg("pad"), pybind11::arg("stride") = 1,
        pybind11::arg("n_stage") = 2, pybind11::arg("input_h") = -1, pybind11::arg("input_w") = -1);
  m.def("dwconv_bwd_weight", &tma_dwconv::dwconv_bwd_weight,
        "Weight gradient of the K x K forward (stride 1 or 2): dw [K,K,C] fp32 (deterministic).",
        pybind11::arg("x"), pybind11::arg("dy"), pybind11::arg("K"), pybind11::arg("pad"),
        pybind11::arg("stride") = 1, pybind11::arg("n_stage") = 2);
  m.def("device_status", &tma_dwconv::device_status,
        "(code, block, stage, load) of the first recorded pipeline-wait failure on a device.",
        pybind11::arg("device"), pybind11::arg("clear") = true);
  m.def("set_wait_timeout_ns", &tma_dwconv::set_wait_timeout_ns,
        "Limit of every pipeline wait of later launches (default 2 s).", pybind11::arg("ns"));
  m.def("consumer_warps", &tma_dwconv::consumer_warps, "Consumer warps per CTA of the ws kernel.");
}
