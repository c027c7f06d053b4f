// tdc_ptx.cuh — thin inline-PTX wrappers for sm_100a: mbarrier, TMA tiled
// loads, the global timer and the fp16-in / fp32-accumulate FMA forms the
// depthwise kernels use.  No CuTe/CUTLASS: every instruction is spelled out.
#pragma once

#include <cuda.h>        // CUtensorMap (type only; no driver symbols are linked)
#include <cuda_fp16.h>
#include <cstdint>
#include <type_traits>

namespace tdc {

__device__ __forceinline__ uint32_t smem_addr(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// ---- mbarrier ---------------------------------------------------------------
__device__ __forceinline__ void mbar_init(uint32_t bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(bar), "r"(count) : "memory");
}

// Makes the mbarrier initialisation visible to the async (TMA) proxy and to
// the other threads of the CTA (followed by __syncthreads by the caller).
__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint32_t bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(bar), "r"(bytes)
               : "memory");
}

__device__ __forceinline__ void mbar_arrive(uint32_t bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(bar) : "memory");
}

// One bounded probe of the phase with the given parity.  The hardware may
// suspend the thread for up to `hint_ns` while the phase is incomplete.
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity, uint32_t hint_ns) {
  uint32_t ok;
  asm volatile(
      "{\n"
      " .reg .pred p;\n"
      " mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n"
      " selp.u32 %0, 1, 0, p;\n"
      "}\n"
      : "=r"(ok)
      : "r"(bar), "r"(parity), "r"(hint_ns)
      : "memory");
  return ok != 0;
}

__device__ __forceinline__ uint64_t global_timer_ns() {
  uint64_t t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

// Bounded wait for the phase `parity` of an mbarrier.
//  * returns true once the phase completed;
//  * returns false when *abort_flag becomes non-zero (another warp of the CTA
//    gave up) or after `timeout_ns` of global time, or after a hard cap on
//    probes, whichever comes first.
// `check_abort` = false is used by the producer's final drain, which must wait
// for its own copies whatever the other warps do.
__device__ __forceinline__ bool mbar_wait_bounded(uint32_t bar, uint32_t parity,
                                                  const volatile int* abort_flag,
                                                  bool check_abort, uint64_t timeout_ns) {
  if (mbar_try_wait(bar, parity, 1000000u)) return true;  // fast path
  const uint64_t t0 = global_timer_ns();
  // Each probe suspends for at most ~20 us; the probe cap is a second bound
  // (about 20 s) that holds even if the global timer were frozen.
  for (uint32_t it = 1; it < (1u << 20); ++it) {
    if (mbar_try_wait(bar, parity, 20000u)) return true;
    if ((it & 15u) == 0) {
      if (check_abort && *abort_flag) return false;
      if (global_timer_ns() - t0 > timeout_ns) return false;
    }
  }
  return false;
}

// ---- TMA --------------------------------------------------------------------
// 4-D tiled bulk tensor load global -> shared (this CTA), completion signalled
// as transaction bytes on `bar`.  Coordinates are in descriptor order
// (innermost first); they may be negative or past the end, where the box is
// zero-filled.  No multicast.
__device__ __forceinline__ void tma_load_4d(uint32_t dst, const CUtensorMap* map, uint32_t bar,
                                            int32_t c0, int32_t c1, int32_t c2, int32_t c3) {
  asm volatile(
      "cp.async.bulk.tensor.4d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
      " [%0], [%1, {%2, %3, %4, %5}], [%6];" ::"r"(dst),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(c0), "r"(c1), "r"(c2), "r"(c3), "r"(bar)
      : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- programmatic dependent launch -----------------------------------------------
// A kernel launched with programmatic stream serialization may start while the
// previous kernel on its stream is still finishing.  griddep_wait blocks until
// that kernel has completed and its memory is visible (a no-op for a kernel
// launched without the attribute); every thread calls it before its first
// global-memory access.
__device__ __forceinline__ void griddep_wait() {
  asm volatile("griddepcontrol.wait;" ::: "memory");
}

// ---- arithmetic -------------------------------------------------------------
// acc{0,1} = fp32(x.{lo,hi}) * fp32(w.{lo,hi}) + acc{0,1}, one rounding each.
// The product of two fp16 values is exact in fp32, so this equals
// fmaf((float)x, (float)w, acc) bit for bit.  x2, w2 hold two packed fp16.
__device__ __forceinline__ void fma2_f16f32(uint32_t x2, uint32_t w2, float& acc0, float& acc1) {
  asm("{\n"
      " .reg .b16 xl, xh, wl, wh;\n"
      " mov.b32 {xl, xh}, %2;\n"
      " mov.b32 {wl, wh}, %3;\n"
      " fma.rn.f32.f16 %0, xl, wl, %0;\n"
      " fma.rn.f32.f16 %1, xh, wh, %1;\n"
      "}\n"
      : "+f"(acc0), "+f"(acc1)
      : "r"(x2), "r"(w2));
}

__device__ __forceinline__ uint32_t pack_half2_rn(float lo, float hi) {
  __half2 h = __floats2half2_rn(lo, hi);
  return *reinterpret_cast<uint32_t*>(&h);
}

// ---- element types ------------------------------------------------------------
// Activations and filters are 16-bit: fp16 (F16, the reference's type) or
// bfloat16 (BF16).  The kernels move them as raw 16-bit pairs (one uint32 =
// two channels) and only these helpers interpret them.  Products of two
// elements are exact in fp32 for both types, so fma(x, w, acc) equals
// acc + x*w with one rounding, as the CPU's fmaf.
struct F16 {};
struct BF16 {};

// Two packed 16-bit ones (the w operand of fma2 that adds x to acc exactly).
template <class E>
__host__ __device__ constexpr uint32_t ones2();
template <>
__host__ __device__ constexpr uint32_t ones2<F16>() { return 0x3C003C00u; }
template <>
__host__ __device__ constexpr uint32_t ones2<BF16>() { return 0x3F803F80u; }

// acc{0,1} += x.{lo,hi} * w.{lo,hi}: fma.rn.f32.f16 / fma.rn.f32.bf16.
template <class E>
__device__ __forceinline__ void fma2(uint32_t x2, uint32_t w2, float& acc0, float& acc1);
template <>
__device__ __forceinline__ void fma2<F16>(uint32_t x2, uint32_t w2, float& acc0, float& acc1) {
  fma2_f16f32(x2, w2, acc0, acc1);
}
template <>
__device__ __forceinline__ void fma2<BF16>(uint32_t x2, uint32_t w2, float& acc0, float& acc1) {
  asm("{\n"
      " .reg .b16 xl, xh, wl, wh;\n"
      " mov.b32 {xl, xh}, %2;\n"
      " mov.b32 {wl, wh}, %3;\n"
      " fma.rn.f32.bf16 %0, xl, wl, %0;\n"
      " fma.rn.f32.bf16 %1, xh, wh, %1;\n"
      "}\n"
      : "+f"(acc0), "+f"(acc1)
      : "r"(x2), "r"(w2));
}

// Two fp32 values rounded to nearest-even and packed (lo in the low half).
template <class E>
__device__ __forceinline__ uint32_t pack2_rn(float lo, float hi) {
  if constexpr (std::is_same_v<E, BF16>) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
  } else {
    return pack_half2_rn(lo, hi);
  }
}

// A packed pair of elements as two fp32 values (exact).
template <class E>
__device__ __forceinline__ void unpack2(uint32_t v, float& lo, float& hi) {
  if constexpr (std::is_same_v<E, BF16>) {
    lo = __uint_as_float(v << 16);
    hi = __uint_as_float(v & 0xffff0000u);
  } else {
    const __half2 h = *reinterpret_cast<const __half2*>(&v);
    lo = __low2float(h);
    hi = __high2float(h);
  }
}

}  // namespace tdc
