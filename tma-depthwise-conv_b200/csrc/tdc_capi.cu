// tdc_capi.cu — host half of libtdc_sm100.so: argument validation, launch
// planning, TMA descriptor encoding and kernel launches behind the C ABI
// declared in include/tdc_dwconv.h.
//
// The reference binds three C++ functions taking torch tensors
// (csrc/bindings.cpp:5-11 → csrc/kernel_v0_naive_float4.cu:78-118,
// csrc/kernel_tma_ws.cu:52-137).  Here the same three operations take raw
// device pointers and sizes; tensor allocation stays with the caller.
//
// Differences from the reference launchers, by design:
//  * validation returns a status code before any CUDA call is made;
//  * the TMA descriptor is encoded with the driver's cuTensorMapEncodeTiled,
//    fetched once through cudaGetDriverEntryPoint (no -lcuda, no CuTe);
//  * the dynamic-smem attribute and occupancy are queried once per device and
//    kernel instantiation instead of on every call (kernel_tma_ws.cu:36-38);
//  * the grid is persistent (SMs x resident CTAs): whole 32-column strips
//    round-robin, then the last strips in bands, instead of one CTA per
//    8-row tile.
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstdlib>
#include <cstring>
#include <mutex>
#include <vector>

#include "tdc_dwconv.h"
#include "tdc_kernels.cuh"
#include "tdc_wgrad.cuh"
#include "tdc_dgrad_s2.cuh"
#include "tdc_plain.cuh"

namespace {

thread_local int t_last_cuda_error = 0;
std::atomic<int64_t> g_timeout_ns{2000000000ll};

int cuda_fail(cudaError_t e) {
  t_last_cuda_error = int(e);
  return TDC_ERR_CUDA;
}

constexpr int kMaxDevices = 64;

struct DeviceInfo {
  std::once_flag once;
  int status = TDC_ERR_NO_DEVICE;
  int sms = 0;
  int ws_occupancy[3][4] = {};  // [n_stage-2][ws, probe, general, epilogue]
  int wgrad_occupancy[2][3] = {};  // [element type][n_stage-2]
};
DeviceInfo g_dev[kMaxDevices];

constexpr int kMaxDynSmem = 200 * 1024;

// Element type of a call: 0 = fp16 (the reference's), 1 = bfloat16.
constexpr int kF16 = 0, kBF16 = 1;

int stage_rows_for(int64_t n_stage);

int wgrad_stage_rows(int64_t n_stage);

template <int NS, class E>
cudaError_t prepare_wgrad(int* occ) {
  auto* k = &tdc::dwconv_wgrad_kernel<NS, E>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
  if (e != cudaSuccess) return e;
  const size_t smem = size_t(NS) * wgrad_stage_rows(NS) * (tdc::kRowBytes + tdc::kDyRowBytes) + 128;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, k, tdc::kWsThreads, smem);
}

template <int NS, bool PROBE, int MODE = tdc::kModeWs>
cudaError_t prepare_ws(int* occ) {
  auto* k = &tdc::dwconv_ws_kernel<NS, PROBE, MODE>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
  if (e != cudaSuccess) return e;
  // Occupancy at the ring this instantiation uses.
  const size_t smem = size_t(NS) * stage_rows_for(NS) * tdc::kRowBytes + 128;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, k, tdc::kWsThreads, smem);
}

template <int NS>
cudaError_t prepare_ws_act() {
  int occ = 0;
  cudaError_t e = cudaSuccess;
  if (e == cudaSuccess) e = prepare_ws<NS, false, tdc::kModeEpilogueAct + TDC_ACT_NONE>(&occ);
  if (e == cudaSuccess) e = prepare_ws<NS, false, tdc::kModeEpilogueAct + TDC_ACT_RELU>(&occ);
  if (e == cudaSuccess) e = prepare_ws<NS, false, tdc::kModeEpilogueAct + TDC_ACT_RELU6>(&occ);
  if (e == cudaSuccess) e = prepare_ws<NS, false, tdc::kModeEpilogueAct + TDC_ACT_SILU>(&occ);
  if (e == cudaSuccess) e = prepare_ws<NS, false, tdc::kModeEpilogueAct + TDC_ACT_HARDSWISH>(&occ);
  return e;
}

// Failure records of the kernels' bounded waits, written through by the GPU
// to mapped pinned host memory: 4 ints per device (code, block, stage, load)
// in one page, allocated by the first call that launches a pipelined kernel
// (never by tdc_dwconv3x3_bwd_weight_noalloc, which allocates nothing).
// With unified addressing the host pointer is also the device address.
std::mutex g_status_page_mutex;
std::atomic<int*> g_status_page{nullptr};

// This device's slot of the page (creating the page when allow_alloc), or
// null.  The allocation may come during a stream capture of the calling
// thread: the thread's capture mode is relaxed around it, and a failure
// leaves the page to a later call.
int* status_slot(int dev, bool allow_alloc) {
  int* page = g_status_page.load(std::memory_order_acquire);
  if (page == nullptr && allow_alloc) {
    std::lock_guard<std::mutex> lock(g_status_page_mutex);
    page = g_status_page.load(std::memory_order_acquire);
    if (page == nullptr) {
      cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
      cudaThreadExchangeStreamCaptureMode(&mode);
      void* mem = nullptr;
      const cudaError_t e = cudaHostAlloc(&mem, sizeof(int) * 4 * kMaxDevices,
                                          cudaHostAllocMapped | cudaHostAllocPortable);
      cudaThreadExchangeStreamCaptureMode(&mode);
      if (e != cudaSuccess) {
        (void)cudaGetLastError();
        return nullptr;
      }
      std::memset(mem, 0, sizeof(int) * 4 * kMaxDevices);
      page = static_cast<int*>(mem);
      g_status_page.store(page, std::memory_order_release);
    }
  }
  return page == nullptr ? nullptr : page + 4 * dev;
}

// The slot of the calling thread's current device (see status_slot).
int* current_status_slot(bool allow_alloc) {
  int dev = -1;
  if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= kMaxDevices) return nullptr;
  return status_slot(dev, allow_alloc);
}

// Returns TDC_OK and fills *info for the current device, or an error.  With
// check_failures, a failure a kernel recorded on this device (an earlier
// launch that gave up waiting on its pipeline) fails the call with
// TDC_ERR_DEVICE_TIMEOUT until tdc_device_status clears it; the record is
// read from mapped host memory, without synchronising, so it covers the
// launches that have finished by the time of the call.
int current_device(DeviceInfo** info, int* dev_out, bool check_failures = true) {
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver
                                   ? TDC_ERR_NO_DEVICE
                                   : cuda_fail(e);
  if (dev < 0 || dev >= kMaxDevices) return TDC_ERR_NO_DEVICE;
  // Make the device's primary context current on this thread.  A thread that
  // has only selected the device (for example a framework's worker thread)
  // may have no current context yet; kernel launches would bind it lazily,
  // but the driver's tensor-map encoder needs it bound.
  thread_local int bound_device = -1;
  if (bound_device != dev) {
    e = cudaSetDevice(dev);
    if (e != cudaSuccess) return cuda_fail(e);
    bound_device = dev;
  }
  DeviceInfo& d = g_dev[dev];
  std::call_once(d.once, [&d, dev]() {
    int major = 0, minor = 0, sms = 0;
    if (cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, dev) != cudaSuccess ||
        cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) {
      d.status = TDC_ERR_NO_DEVICE;
      return;
    }
    if (major != 10 || minor != 0) {  // the cubin is sm_100a only
      d.status = TDC_ERR_NO_DEVICE;
      return;
    }
    d.sms = sms;
    cudaError_t e2 = cudaSuccess;
    if (e2 == cudaSuccess) e2 = prepare_ws<2, false>(&d.ws_occupancy[0][0]);
    if (e2 == cudaSuccess) e2 = prepare_ws<3, false>(&d.ws_occupancy[1][0]);
    if (e2 == cudaSuccess) e2 = prepare_ws<4, false>(&d.ws_occupancy[2][0]);
    if (e2 == cudaSuccess) e2 = prepare_ws<2, true>(&d.ws_occupancy[0][1]);
    if (e2 == cudaSuccess) e2 = prepare_ws<3, true>(&d.ws_occupancy[1][1]);
    if (e2 == cudaSuccess) e2 = prepare_ws<4, true>(&d.ws_occupancy[2][1]);
    if (e2 == cudaSuccess) e2 = prepare_ws<2, false, tdc::kModeGeneral>(&d.ws_occupancy[0][2]);
    if (e2 == cudaSuccess) e2 = prepare_ws<3, false, tdc::kModeGeneral>(&d.ws_occupancy[1][2]);
    if (e2 == cudaSuccess) e2 = prepare_ws<4, false, tdc::kModeGeneral>(&d.ws_occupancy[2][2]);
    if (e2 == cudaSuccess) e2 = prepare_ws<2, false, tdc::kModeEpilogue>(&d.ws_occupancy[0][3]);
    if (e2 == cudaSuccess) e2 = prepare_ws<3, false, tdc::kModeEpilogue>(&d.ws_occupancy[1][3]);
    if (e2 == cudaSuccess) e2 = prepare_ws<4, false, tdc::kModeEpilogue>(&d.ws_occupancy[2][3]);
    // The compile-time-activation epilogue kernels run at the plan of kind 3.
    if (e2 == cudaSuccess) e2 = prepare_ws_act<2>();
    if (e2 == cudaSuccess) e2 = prepare_ws_act<3>();
    if (e2 == cudaSuccess) e2 = prepare_ws_act<4>();
    if (e2 == cudaSuccess) e2 = prepare_wgrad<2, tdc::F16>(&d.wgrad_occupancy[kF16][0]);
    if (e2 == cudaSuccess) e2 = prepare_wgrad<3, tdc::F16>(&d.wgrad_occupancy[kF16][1]);
    if (e2 == cudaSuccess) e2 = prepare_wgrad<4, tdc::F16>(&d.wgrad_occupancy[kF16][2]);
    if (e2 == cudaSuccess) e2 = prepare_wgrad<2, tdc::BF16>(&d.wgrad_occupancy[kBF16][0]);
    if (e2 == cudaSuccess) e2 = prepare_wgrad<3, tdc::BF16>(&d.wgrad_occupancy[kBF16][1]);
    if (e2 == cudaSuccess) e2 = prepare_wgrad<4, tdc::BF16>(&d.wgrad_occupancy[kBF16][2]);
    if (e2 != cudaSuccess) {
      t_last_cuda_error = int(e2);
      d.status = TDC_ERR_CUDA;
      return;
    }
    d.status = TDC_OK;
  });
  if (d.status != TDC_OK) return d.status;
  *info = &d;
  if (dev_out) *dev_out = dev;
  if (check_failures) {
    const volatile int* slot = status_slot(dev, false);
    if (slot != nullptr && slot[0] != 0) return TDC_ERR_DEVICE_TIMEOUT;
  }
  return TDC_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Common validation of the reference launchers (kernel_tma_ws.cu:54-65,
// kernel_v0_naive_float4.cu:84-94), in the same order.
// An empty output (N, C, P or Q zero) is valid and needs no pointers: torch
// hands out null data pointers for zero-element tensors.
int validate(const void* x, const void* w, const void* y, int64_t N, int64_t H, int64_t W,
             int64_t C, int64_t R, int64_t S, int64_t pad, int64_t cmult, int64_t* P,
             int64_t* Q, bool* empty, bool allow_negative_pad = false) {
  if (N < 0 || H < 1 || W < 1 || C < 0) return TDC_ERR_BAD_SHAPE;
  if (R != 3 || S != 3) return TDC_ERR_FILTER_SHAPE;
  if (C % cmult != 0) return TDC_ERR_CHANNELS;
  if (pad < 0 && !allow_negative_pad) return TDC_ERR_PAD;
  if (pad > (1 << 28) || pad < -(1 << 28)) return TDC_ERR_TOO_LARGE;
  *P = H + 2 * pad - R + 1;
  *Q = W + 2 * pad - S + 1;
  if (*P < 0 || *Q < 0) return TDC_ERR_BAD_SHAPE;
  *empty = N == 0 || C == 0 || *P == 0 || *Q == 0;
  if (*empty) return TDC_OK;
  if (!x || !w || !y) return TDC_ERR_NULL_POINTER;
  if (!aligned16(x) || !aligned16(w) || !aligned16(y)) return TDC_ERR_ALIGNMENT;
  return TDC_OK;
}

// ---------------------------------------------------------------------------
// ws launch plan
// ---------------------------------------------------------------------------
struct WsPlan {
  int stage_rows, qstrips, cblocks, tail_bands, tail_band_rows;
  int64_t strips, full_units, tail_strips, grid;
  size_t smem;
  int tail_chunk_rows;  // > 0: the tail is cut into chunks (SegmentIter), else bands
};

// Ring capacity in input rows per CTA, split evenly over the n_stage stages:
// 12 rows (52 KB) of 3x3 stride-1 rows for the K x K geometries
// (geom_stage_rows), 10 rows (43.5 KB) for 3x3 stride 1 itself.  At 3x3
// stride 1 the 444 CTAs' stages in flight (up to 2 x 26 KB each with 6-row
// stages) oversubscribe the memory system when the SMs run at full clock:
// measured in alternating bursts on 64 x 224 x 336 x 256, 5-row stages take
// 0.945 of the time of 6-row stages at 1965 MHz and 0.997 under the power
// cap (1.6-1.8 GHz); 4-row stages 0.880 and 1.028.
constexpr int kRingRows = 12;
constexpr int kRingRows3x3 = 10;
// A CTA is not given fewer output rows than this (each segment streams two
// halo rows).
constexpr int64_t kMinRowsPerCta = 8;

int stage_rows_for(int64_t n_stage) { return std::max<int>(1, kRingRows3x3 / int(n_stage)); }

// The weight-gradient ring carries x and dy rows (8448 B per row): 8 rows.
constexpr int kWgradRingRows = 8;
int wgrad_stage_rows(int64_t n_stage) { return std::max<int>(1, kWgradRingRows / int(n_stage)); }

// Rows the busiest CTA streams (halo rows included) when the tail's
// (tail_strips / cblocks) * P pixel-strip rows are cut into chunks of L rows,
// one chunk per cblocks CTAs; 0 when no chunk fits the grid.
int64_t chunk_tail_cost(int64_t tail_strips, int64_t cblocks, int64_t P, int64_t grid, int64_t L) {
  const int64_t total = (tail_strips / cblocks) * P;
  const int64_t chunks = grid / cblocks;
  if (L < 1 || chunks < 1 || (total + L - 1) / L > chunks) return 0;
  int64_t worst = 0;
  for (int64_t a = 0; a < total; a += L) {
    const int64_t b = std::min(total, a + L);
    const int64_t segments = (b - 1) / P - a / P + 1;
    worst = std::max(worst, (b - a) + 2 * segments);
  }
  return worst;
}

// Persistent grid of SMs x resident CTAs.  Whole strips are dealt
// round-robin while every CTA can take one: full_units =
// (ceil(strips/grid) - 1) * grid.  The remaining tail_strips strips are cut
// into bands; the band count minimises the rows the busiest CTA streams in
// the last wave, (tail units per CTA) x (band rows + 2 halo rows).  With
// `chunk_tail` (forward kernels) the tail may instead be cut into chunks of
// consecutive rows (SegmentIter), when that lets the busiest CTA stream fewer
// rows: e.g. 16 x 112 x 224 x 128 on 444 CTAs, 224 strips of 112 rows: bands
// of 16 rows leave the busiest CTA 4 bands = 72 rows, chunks of 57 rows 61.
WsPlan compute_plan(int64_t N, int64_t P, int64_t Q, int64_t C, int64_t n_stage, int64_t sms,
                    int64_t ctas_per_sm, bool chunk_tail) {
  WsPlan pl{};
  pl.stage_rows = stage_rows_for(n_stage);
  pl.qstrips = int((Q + tdc::kStripQ - 1) / tdc::kStripQ);
  pl.cblocks = int((C + tdc::kBlockC - 1) / tdc::kBlockC);
  pl.strips = N * pl.qstrips * pl.cblocks;
  const int64_t g0 = std::max<int64_t>(1, sms * ctas_per_sm);
  const int64_t total_rows = pl.strips * P;
  pl.grid = std::max<int64_t>(1, std::min(g0, (total_rows + kMinRowsPerCta - 1) / kMinRowsPerCta));
  const int64_t waves = (pl.strips + pl.grid - 1) / pl.grid;
  pl.full_units = (waves - 1) * pl.grid;
  pl.tail_strips = pl.strips - pl.full_units;
  int64_t best_cost = -1, best_rows = P;
  for (int64_t b = 1; b <= std::min<int64_t>(P, 256); ++b) {
    const int64_t rows = (P + b - 1) / b;
    const int64_t bands = (P + rows - 1) / rows;
    if (bands != b) continue;  // same band height as a smaller band count
    const int64_t per_cta = (pl.tail_strips * bands + pl.grid - 1) / pl.grid;
    const int64_t cost = per_cta * (rows + 2);
    if (best_cost < 0 || cost < best_cost) {
      best_cost = cost;
      best_rows = rows;
    }
  }
  pl.tail_band_rows = int(best_rows);
  pl.tail_bands = int((P + best_rows - 1) / best_rows);
  pl.tail_chunk_rows = 0;
  if (chunk_tail && pl.grid % pl.cblocks == 0) {
    const int64_t total = (pl.tail_strips / pl.cblocks) * P;
    const int64_t chunks = pl.grid / pl.cblocks;
    const int64_t L = std::max<int64_t>(kMinRowsPerCta, (total + chunks - 1) / chunks);
    const int64_t cost = chunk_tail_cost(pl.tail_strips, pl.cblocks, P, pl.grid, L);
    // Chunks cost DRAM re-reads bands do not: the two halo columns a strip
    // shares with each column-strip neighbour are read from L2 by both while
    // both run the same rows at the same time; chunks run neighbours' rows
    // at different times, so those columns come from DRAM twice (+8 % reads
    // at 8 x 224 x 336 x 256, ncu).  So chunks are taken only when they leave
    // the busiest CTA at least 1/16 fewer rows.  (The kernel counts the
    // tail's rows in 32 bits.)
    if (cost > 0 && cost + cost / 16 < best_cost && total + L + pl.grid < (int64_t(1) << 31))
      pl.tail_chunk_rows = int(L);
  }
  pl.smem = size_t(n_stage) * pl.stage_rows * tdc::kRowBytes + 128;
  return pl;
}

// A few recent results of a pure host computation, per host thread: the
// launch plan (a few microseconds of integer work) and the TMA descriptor
// are the same for every call on the same shapes and pointers, and on small
// problems they would otherwise be a visible part of the call.  Keys hold
// every input, so an entry is never stale.
template <class Key, class Value, int kEntries>
struct RecentCache {
  Key keys[kEntries];
  Value values[kEntries];
  bool used[kEntries] = {};
  int next = 0;
  const Value* find(const Key& k) const {
    for (int i = 0; i < kEntries; ++i)
      if (used[i] && std::memcmp(&keys[i], &k, sizeof(Key)) == 0) return &values[i];
    return nullptr;
  }
  void put(const Key& k, const Value& v) {
    keys[next] = k;
    values[next] = v;
    used[next] = true;
    next = (next + 1) % kEntries;
  }
};

struct PlanKey {
  int64_t N, P, Q, C, n_stage, sms, ctas_per_sm, chunk_tail;
};

WsPlan make_plan(int64_t N, int64_t P, int64_t Q, int64_t C, int64_t n_stage, int64_t sms,
                 int64_t ctas_per_sm, bool chunk_tail = false) {
  thread_local RecentCache<PlanKey, WsPlan, 8> cache;
  PlanKey k;
  std::memset(&k, 0, sizeof(k));
  k = PlanKey{N, P, Q, C, n_stage, sms, ctas_per_sm, chunk_tail ? 1 : 0};
  if (const WsPlan* hit = cache.find(k)) return *hit;
  const WsPlan pl = compute_plan(N, P, Q, C, n_stage, sms, ctas_per_sm, chunk_tail);
  cache.put(k, pl);
  return pl;
}

PFN_cuTensorMapEncodeTiled_v12000 get_encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = []() -> PFN_cuTensorMapEncodeTiled_v12000 {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
        q != cudaDriverEntryPointSuccess)
      return nullptr;
    return reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  }();
  return fn;
}

// 4-D map over an NHWC fp16 tensor viewed as (C, W, H, N), innermost first;
// box (64 ch, box_cols columns, box_rows rows, 1 image); out-of-bounds
// elements read 0.  With dil = D > 1 the columns and rows of the box are D
// apart (traversal stride D: the map's box spans D * box_cols columns and
// D * box_rows rows, of which the copy takes every D-th), so shared memory
// receives the same dense box.  Stores the CUresult of a failed encode for
// tdc_last_cuda_error.
// Limits of a tiled tensor map: elements per box dimension and traversal
// stride.
constexpr int kMaxTmaBox = 256;
constexpr int kMaxTmaStride = 8;

struct MapKey {
  const void* t;
  int64_t N, H, W, C, box_cols, box_rows, dt, dil;
};
struct alignas(64) MapValue {
  CUtensorMap map;
};

int encode_nhwc_map_uncached(CUtensorMap* map, const void* t, int64_t N, int64_t H, int64_t W,
                             int64_t C, int box_cols, int box_rows, int dt, int dil);

int encode_nhwc_map(CUtensorMap* map, const void* t, int64_t N, int64_t H, int64_t W, int64_t C,
                    int box_cols, int box_rows, int dt = kF16, int dil = 1) {
  thread_local RecentCache<MapKey, MapValue, 8> cache;
  MapKey k;
  std::memset(&k, 0, sizeof(k));
  k = MapKey{t, N, H, W, C, box_cols, box_rows, dt, dil};
  if (const MapValue* hit = cache.find(k)) {
    *map = hit->map;
    return TDC_OK;
  }
  const int rc = encode_nhwc_map_uncached(map, t, N, H, W, C, box_cols, box_rows, dt, dil);
  if (rc == TDC_OK) {
    MapValue v;
    v.map = *map;
    cache.put(k, v);
  }
  return rc;
}

int encode_nhwc_map_uncached(CUtensorMap* map, const void* t, int64_t N, int64_t H, int64_t W,
                             int64_t C, int box_cols, int box_rows, int dt, int dil) {
  auto fn = get_encode_fn();
  if (!fn) return TDC_ERR_TMA_ENCODE;
  if (dil < 1 || dil > kMaxTmaStride || box_cols * dil > kMaxTmaBox || box_rows * dil > kMaxTmaBox)
    return TDC_ERR_UNSUPPORTED;
  const cuuint64_t dims[4] = {cuuint64_t(C), cuuint64_t(W), cuuint64_t(H), cuuint64_t(N)};
  const cuuint64_t strides[3] = {cuuint64_t(C) * 2, cuuint64_t(W) * C * 2, cuuint64_t(H) * W * C * 2};
  const cuuint32_t box[4] = {cuuint32_t(tdc::kBlockC), cuuint32_t(box_cols * dil),
                             cuuint32_t(box_rows * dil), 1u};
  const cuuint32_t estr[4] = {1u, cuuint32_t(dil), cuuint32_t(dil), 1u};
  CUresult r = fn(map, dt == kBF16 ? CU_TENSOR_MAP_DATA_TYPE_BFLOAT16 : CU_TENSOR_MAP_DATA_TYPE_FLOAT16,
                  4, const_cast<void*>(t), dims, strides,
                  box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                  CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) t_last_cuda_error = int(r);
  return r == CUDA_SUCCESS ? TDC_OK : TDC_ERR_TMA_ENCODE;
}

// x of the 3x3 stride-1 kernels: 34 columns (a 32-column strip and its halo).
int encode_x_map(CUtensorMap* map, const void* x, int64_t N, int64_t H, int64_t W, int64_t C,
                 int stage_rows) {
  return encode_nhwc_map(map, x, N, H, W, C, tdc::kInCols, stage_rows);
}

// dy [N,P,Q,C] of the weight gradients: 32 columns (one strip).
int encode_dy_map(CUtensorMap* map, const void* dy, int64_t N, int64_t P, int64_t Q, int64_t C,
                  int stage_rows, int dt = kF16) {
  return encode_nhwc_map(map, dy, N, P, Q, C, tdc::kStripQ, stage_rows, dt);
}

// Limits of the descriptor and of the 32-bit fields the kernel keeps.
int check_ws_limits(int64_t N, int64_t H, int64_t W, int64_t C, int64_t P, int64_t Q) {
  const int64_t i32 = 0x7fffffffll;
  if (N > i32 || H > i32 || W > i32 || C > i32 || P > i32 || Q > i32) return TDC_ERR_TOO_LARGE;
  if (H * W * C * 2 >= (int64_t(1) << 40)) return TDC_ERR_TOO_LARGE;  // TMA stride limit
  return TDC_OK;
}

// Launches a forward kernel with programmatic stream serialization: its CTAs
// may start (barrier set-up, descriptor prefetch) while the previous kernel on
// the stream drains; the kernel waits for that kernel (griddepcontrol.wait)
// before its first global-memory access.  Saves part of the launch latency
// of back-to-back calls on small problems (8 x 56 x 56 x 256: 10.25 -> 8.3-8.5
// us per call; 64 x 224 x 336 x 256 unchanged within noise).
template <class... Args>
cudaError_t launch_pdl_block(void (*kernel)(Args...), int64_t grid, unsigned block, size_t smem,
                             cudaStream_t st, Args... args) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid));
  cfg.blockDim = dim3(block);
  cfg.dynamicSmemBytes = smem;
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, kernel, args...);
}

template <class... Args>
cudaError_t launch_pdl(void (*kernel)(Args...), int64_t grid, size_t smem, cudaStream_t st,
                       Args... args) {
  return launch_pdl_block(kernel, grid, unsigned(tdc::kWsThreads), smem, st, args...);
}

template <int NS, bool PROBE, int MODE = tdc::kModeWs>
cudaError_t launch_ws_t(const CUtensorMap& map, const tdc::WsParams& prm, const WsPlan& pl,
                        cudaStream_t st) {
  return launch_pdl(&tdc::dwconv_ws_kernel<NS, PROBE, MODE>, pl.grid, pl.smem, st, map, prm);
}

// The epilogue kernel with prm.act fixed at compile time.
template <int NS>
cudaError_t launch_ws_epi(const CUtensorMap& map, const tdc::WsParams& prm, const WsPlan& pl,
                          cudaStream_t st) {
  switch (prm.act) {
    case TDC_ACT_RELU: return launch_ws_t<NS, false, tdc::kModeEpilogueAct + TDC_ACT_RELU>(map, prm, pl, st);
    case TDC_ACT_RELU6: return launch_ws_t<NS, false, tdc::kModeEpilogueAct + TDC_ACT_RELU6>(map, prm, pl, st);
    case TDC_ACT_SILU: return launch_ws_t<NS, false, tdc::kModeEpilogueAct + TDC_ACT_SILU>(map, prm, pl, st);
    case TDC_ACT_HARDSWISH:
      return launch_ws_t<NS, false, tdc::kModeEpilogueAct + TDC_ACT_HARDSWISH>(map, prm, pl, st);
    default: return launch_ws_t<NS, false, tdc::kModeEpilogueAct + TDC_ACT_NONE>(map, prm, pl, st);
  }
}

struct Epilogue {
  bool fused = false;
  const void* bias = nullptr;
  const void* residual = nullptr;
  int act = TDC_ACT_NONE;
  bool flip_taps = false;  // data gradient: taps w[2-r][2-s], pad may be negative
};

// Padding on each side of the image (forward entries with asymmetric
// padding); the kernels take the top and left sides as row / column offsets,
// and the bottom and right sides only set the output size (rows and columns
// past the image read as zero).
struct Pad4 {
  int64_t top, bottom, left, right;
};

int ws_common(const void* x, const void* w, void* y, int64_t N, int64_t H, int64_t W, int64_t C,
              int64_t R, int64_t S, int64_t pad, int64_t n_stage, unsigned long long* stall,
              bool probe, int64_t withhold, int64_t timeout_ns, void* stream,
              const Epilogue& epi = Epilogue()) {
  int64_t P = 0, Q = 0;
  bool empty = false;
  // The data gradient runs the forward with pad' = 2 - pad, which is negative
  // (a crop) when pad > 2; TMA coordinates take it as it is.
  int rc = validate(x, w, y, N, H, W, C, R, S, pad, epi.fused ? 8 : tdc::kBlockC, &P, &Q,
                    &empty, epi.flip_taps);
  if (rc != TDC_OK) return rc;
  if (epi.fused && !empty &&
      ((epi.bias && !aligned16(epi.bias)) || (epi.residual && !aligned16(epi.residual))))
    return TDC_ERR_ALIGNMENT;
  if (n_stage < 2 || n_stage > 4) return TDC_ERR_N_STAGE;
  rc = check_ws_limits(N, H, W, C, P, Q);
  if (rc != TDC_OK) return rc;
  if (empty) return TDC_OK;  // nothing to do
  if (probe && !stall) return TDC_ERR_NULL_POINTER;
  DeviceInfo* dev = nullptr;
  rc = current_device(&dev, nullptr);
  if (rc != TDC_OK) return rc;
  const bool with_epilogue =
      epi.fused && (epi.bias != nullptr || epi.residual != nullptr || epi.act != TDC_ACT_NONE);
  const int kind = !epi.fused ? (probe ? 1 : 0) : (with_epilogue ? 3 : 2);
  const int occ = std::max(1, dev->ws_occupancy[n_stage - 2][kind]);
  const WsPlan pl = make_plan(N, P, Q, C, n_stage, dev->sms, occ, true);
  alignas(64) CUtensorMap map;
  rc = encode_x_map(&map, x, N, H, W, C, pl.stage_rows);
  if (rc != TDC_OK) return rc;
  tdc::WsParams prm{};
  prm.status_host = current_status_slot(true);
  prm.w = static_cast<const __half*>(w);
  prm.y = static_cast<__half*>(y);
  prm.stall = stall;
  prm.H = int32_t(H); prm.W = int32_t(W); prm.C = int32_t(C);
  prm.P = int32_t(P); prm.Q = int32_t(Q); prm.pad = int32_t(pad); prm.pad_w = int32_t(pad);
  prm.qstrips = pl.qstrips; prm.cblocks = pl.cblocks; prm.stage_rows = pl.stage_rows;
  prm.tail_bands = pl.tail_bands; prm.tail_band_rows = pl.tail_band_rows;
  prm.full_units = pl.full_units; prm.tail_strips = pl.tail_strips;
  prm.tail_chunk_rows = pl.tail_chunk_rows;
  prm.timeout_ns = uint64_t(timeout_ns > 0 ? timeout_ns : g_timeout_ns.load());
  prm.withhold = withhold;
  prm.bias = static_cast<const __half*>(epi.bias);
  prm.residual = static_cast<const __half*>(epi.residual);
  prm.act = epi.act;
  prm.flip_taps = epi.flip_taps ? 1 : 0;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e;
  if (with_epilogue) {
    switch (n_stage) {
      case 2: e = launch_ws_epi<2>(map, prm, pl, st); break;
      case 3: e = launch_ws_epi<3>(map, prm, pl, st); break;
      default: e = launch_ws_epi<4>(map, prm, pl, st); break;
    }
    return e == cudaSuccess ? TDC_OK : cuda_fail(e);
  }
  if (epi.fused) {
    switch (n_stage) {
      case 2: e = launch_ws_t<2, false, tdc::kModeGeneral>(map, prm, pl, st); break;
      case 3: e = launch_ws_t<3, false, tdc::kModeGeneral>(map, prm, pl, st); break;
      default: e = launch_ws_t<4, false, tdc::kModeGeneral>(map, prm, pl, st); break;
    }
    return e == cudaSuccess ? TDC_OK : cuda_fail(e);
  }
  switch (n_stage) {
    case 2: e = probe ? launch_ws_t<2, true>(map, prm, pl, st) : launch_ws_t<2, false>(map, prm, pl, st); break;
    case 3: e = probe ? launch_ws_t<3, true>(map, prm, pl, st) : launch_ws_t<3, false>(map, prm, pl, st); break;
    default: e = probe ? launch_ws_t<4, true>(map, prm, pl, st) : launch_ws_t<4, false>(map, prm, pl, st); break;
  }
  return e == cudaSuccess ? TDC_OK : cuda_fail(e);
}

// ---------------------------------------------------------------------------
// General forward for K x K taps (K = 3, 5, 7) and stride 1 or 2: one kernel
// instantiation per (K, stride, mode, n_stage), looked up in a table.
// ---------------------------------------------------------------------------
using GeomLaunchFn = cudaError_t (*)(const CUtensorMap&, const tdc::WsParams&, int64_t, size_t,
                                     cudaStream_t);
using GeomOccFn = cudaError_t (*)(int*, size_t);

template <int NS, int MODE, int K, int S, class E>
cudaError_t geom_launch_t(const CUtensorMap& map, const tdc::WsParams& prm, int64_t grid,
                          size_t smem, cudaStream_t st) {
  return launch_pdl(&tdc::dwconv_ws_kernel<NS, false, MODE, K, S, E>, grid, smem, st, map, prm);
}

template <int NS, int MODE, int K, int S, class E>
cudaError_t geom_occ_t(int* occ, size_t smem) {
  auto* k = &tdc::dwconv_ws_kernel<NS, false, MODE, K, S, E>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, k, tdc::kWsThreads, smem);
}

#define TDC_GEOM_NS(FN, E, MODE, K, S) \
  {FN<2, MODE, K, S, E>, FN<3, MODE, K, S, E>, FN<4, MODE, K, S, E>}
#define TDC_GEOM_MODES(FN, E, K, S) \
  {TDC_GEOM_NS(FN, E, tdc::kModeGeneral, K, S), TDC_GEOM_NS(FN, E, tdc::kModeEpilogue, K, S)}
#define TDC_GEOM_TABLE(FN, E)                                                  \
  {{TDC_GEOM_MODES(FN, E, 3, 1), TDC_GEOM_MODES(FN, E, 3, 2)},                 \
   {TDC_GEOM_MODES(FN, E, 5, 1), TDC_GEOM_MODES(FN, E, 5, 2)},                 \
   {TDC_GEOM_MODES(FN, E, 7, 1), TDC_GEOM_MODES(FN, E, 7, 2)}}
// [element type][K index: 3, 5, 7][stride - 1][mode: general, epilogue][n_stage - 2]
const GeomLaunchFn kGeomLaunch[2][3][2][2][3] = {TDC_GEOM_TABLE(geom_launch_t, tdc::F16),
                                                 TDC_GEOM_TABLE(geom_launch_t, tdc::BF16)};
const GeomOccFn kGeomOcc[2][3][2][2][3] = {TDC_GEOM_TABLE(geom_occ_t, tdc::F16),
                                           TDC_GEOM_TABLE(geom_occ_t, tdc::BF16)};
#undef TDC_GEOM_TABLE
#undef TDC_GEOM_MODES
#undef TDC_GEOM_NS

// Ring depth of the forward per geometry when the caller leaves it to the
// library (n_stage = 0), measured at 64 x 224 x 336 x 256.
constexpr int kFwdStages[3][2] = {{2, 4}, {4, 2}, {3, 4}};  // [K: 3, 5, 7][stride - 1]
constexpr int fwd_stages_of(int K, int S) { return kFwdStages[K / 2 - 1][S - 1]; }

// The dilated instantiations of the general forward (DIL = true), at the
// geometry's default ring depth.
template <int MODE, int K, int S, class E>
cudaError_t dil_launch_t(const CUtensorMap& map, const tdc::WsParams& prm, int64_t grid,
                         size_t smem, cudaStream_t st) {
  return launch_pdl(&tdc::dwconv_ws_kernel<fwd_stages_of(K, S), false, MODE, K, S, E, true>, grid,
                    smem, st, map, prm);
}

template <int MODE, int K, int S, class E>
cudaError_t dil_occ_t(int* occ, size_t smem) {
  auto* k = &tdc::dwconv_ws_kernel<fwd_stages_of(K, S), false, MODE, K, S, E, true>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, k, tdc::kWsThreads, smem);
}

#define TDC_DIL_MODES(FN, E, K, S) {FN<tdc::kModeGeneral, K, S, E>, FN<tdc::kModeEpilogue, K, S, E>}
#define TDC_DIL_TABLE(FN, E)                                              \
  {{TDC_DIL_MODES(FN, E, 3, 1), TDC_DIL_MODES(FN, E, 3, 2)},               \
   {TDC_DIL_MODES(FN, E, 5, 1), TDC_DIL_MODES(FN, E, 5, 2)},               \
   {TDC_DIL_MODES(FN, E, 7, 1), TDC_DIL_MODES(FN, E, 7, 2)}}
// [element type][K index: 3, 5, 7][stride - 1][mode: general, epilogue]
const GeomLaunchFn kDilLaunch[2][3][2][2] = {TDC_DIL_TABLE(dil_launch_t, tdc::F16),
                                             TDC_DIL_TABLE(dil_launch_t, tdc::BF16)};
const GeomOccFn kDilOcc[2][3][2][2] = {TDC_DIL_TABLE(dil_occ_t, tdc::F16),
                                       TDC_DIL_TABLE(dil_occ_t, tdc::BF16)};
#undef TDC_DIL_TABLE
#undef TDC_DIL_MODES

std::mutex g_geom_mutex;
int g_geom_occ[kMaxDevices][2][3][2][2][3] = {};  // 0 = not queried yet
int g_dil_occ[kMaxDevices][2][3][2][2] = {};      // 0 = not queried yet

int strip_in_cols(int K, int S) { return S * (tdc::kStripQ - 1) + K; }

// Ring of about 52 KB (what 12 rows of the 3x3 stride-1 strip take) split
// over n_stage stages.  A pass of the direct scheme holds its window of
// input rows (direct_window: S*(R-1) + K for R output rows) at once, across
// at most ceil((window-1)/sr) + 1 stages, so it needs
// (n_stage - 1) * sr >= window - 1; with 3 or 4 stages one more row per
// stage leaves the producer room to run ahead (measured on the 7x7 and 5x5
// kernels at 64 x 224 x 336 x 256: 3-8 % faster than the minimum).
int geom_stage_rows(int K, int S, int64_t n_stage) {
  if (K == 3 && S == 1) return stage_rows_for(n_stage);  // the ws kernel's ring
  const int ns = int(n_stage);
  const int row_bytes = strip_in_cols(K, S) * tdc::kBlockC * 2;
  const int ring_rows = std::max<int>(ns, (kRingRows * tdc::kRowBytes) / row_bytes);
  int sr = std::max(1, ring_rows / ns);
  if (tdc::direct_scheme(K, S)) {
    // The extra row leaves the producer a stage to fill while the window is
    // held.  Dropping it to fit three 7x7 stride-2 CTAs per SM (n_stage 4 x 2
    // rows = 70.6 KB instead of 4 x 3 = 106 KB) was slower, 1109 vs 870 us:
    // the 7-row window then holds every stage and nothing is prefetched.
    const int win = tdc::direct_window(K, S);
    sr = std::max(sr, (win - 1 + ns - 2) / (ns - 1) + (ns >= 3 ? 1 : 0));
  }
  return sr;
}

WsPlan make_geom_plan(int64_t N, int64_t P, int64_t Q, int64_t C, int K, int S, int64_t n_stage,
                      int64_t sms, int64_t ctas_per_sm) {
  WsPlan pl = make_plan(N, P, Q, C, n_stage, sms, ctas_per_sm, true);
  pl.stage_rows = geom_stage_rows(K, S, n_stage);
  pl.smem = size_t(n_stage) * pl.stage_rows * strip_in_cols(K, S) * tdc::kBlockC * 2 + 128;
  return pl;
}

// Resident CTAs per SM of the general forward kernel (queried once per
// device and instantiation).
int geom_occupancy(int devi, int dt, int K, int S, bool with_epilogue, int64_t n_stage, int* occ) {
  const int ki = K / 2 - 1, si = S - 1, mi = with_epilogue ? 1 : 0, ni = int(n_stage - 2);
  const size_t smem = make_geom_plan(1, 1, 1, 8, K, S, n_stage, 1, 1).smem;
  std::lock_guard<std::mutex> lock(g_geom_mutex);
  int v = g_geom_occ[devi][dt][ki][si][mi][ni];
  if (v == 0) {
    const cudaError_t e = kGeomOcc[dt][ki][si][mi][ni](&v, smem);
    if (e != cudaSuccess) return cuda_fail(e);
    v = std::max(1, v);
    g_geom_occ[devi][dt][ki][si][mi][ni] = v;
  }
  *occ = v;
  return TDC_OK;
}

int fwd_geom(const void* x, const void* w, void* y, int64_t N, int64_t H, int64_t W, int64_t C,
             int64_t K, int64_t S, int64_t pad, int64_t n_stage, const Epilogue& epi,
             void* stream, int dt = kF16, const Pad4* p4 = nullptr) {
  const Pad4 pd = p4 ? *p4 : Pad4{pad, pad, pad, pad};
  if (K != 3 && K != 5 && K != 7) return TDC_ERR_FILTER_SHAPE;
  if (S != 1 && S != 2) return TDC_ERR_STRIDE;
  if (N < 0 || H < 1 || W < 1 || C < 0) return TDC_ERR_BAD_SHAPE;
  if (C % 8 != 0) return TDC_ERR_CHANNELS;
  if (pd.top < 0 || pd.bottom < 0 || pd.left < 0 || pd.right < 0) return TDC_ERR_PAD;
  if (std::max({pd.top, pd.bottom, pd.left, pd.right}) > (1 << 28)) return TDC_ERR_TOO_LARGE;
  if (n_stage < 2 || n_stage > 4) return TDC_ERR_N_STAGE;
  if (H + pd.top + pd.bottom < K || W + pd.left + pd.right < K) return TDC_ERR_BAD_SHAPE;
  const int64_t P = (H + pd.top + pd.bottom - K) / S + 1, Q = (W + pd.left + pd.right - K) / S + 1;
  if (N == 0 || C == 0) return TDC_OK;
  if (!x || !w || !y) return TDC_ERR_NULL_POINTER;
  if (!aligned16(x) || !aligned16(w) || !aligned16(y) || (epi.bias && !aligned16(epi.bias)) ||
      (epi.residual && !aligned16(epi.residual)))
    return TDC_ERR_ALIGNMENT;
  int rc = check_ws_limits(N, H, W, C, P, Q);
  if (rc != TDC_OK) return rc;
  DeviceInfo* dev = nullptr;
  int devi = -1;
  rc = current_device(&dev, &devi);
  if (rc != TDC_OK) return rc;
  const bool with_epilogue =
      epi.bias != nullptr || epi.residual != nullptr || epi.act != TDC_ACT_NONE;
  const int ki = int(K / 2 - 1), si = int(S - 1), mi = with_epilogue ? 1 : 0, ni = int(n_stage - 2);
  const int stage_rows = geom_stage_rows(int(K), int(S), n_stage);
  int occ = 0;
  rc = geom_occupancy(devi, dt, int(K), int(S), with_epilogue, n_stage, &occ);
  if (rc != TDC_OK) return rc;
  const WsPlan pl = make_geom_plan(N, P, Q, C, int(K), int(S), n_stage, dev->sms, occ);
  alignas(64) CUtensorMap map;
  rc = encode_nhwc_map(&map, x, N, H, W, C, strip_in_cols(int(K), int(S)), stage_rows, dt);
  if (rc != TDC_OK) return rc;
  tdc::WsParams prm{};
  prm.status_host = current_status_slot(true);
  prm.w = static_cast<const __half*>(w);
  prm.y = static_cast<__half*>(y);
  prm.H = int32_t(H); prm.W = int32_t(W); prm.C = int32_t(C);
  prm.P = int32_t(P); prm.Q = int32_t(Q); prm.pad = int32_t(pd.top); prm.pad_w = int32_t(pd.left);
  prm.qstrips = pl.qstrips; prm.cblocks = pl.cblocks; prm.stage_rows = pl.stage_rows;
  prm.tail_bands = pl.tail_bands; prm.tail_band_rows = pl.tail_band_rows;
  prm.full_units = pl.full_units; prm.tail_strips = pl.tail_strips;
  prm.tail_chunk_rows = pl.tail_chunk_rows;
  prm.timeout_ns = uint64_t(g_timeout_ns.load());
  prm.withhold = -1;
  prm.bias = static_cast<const __half*>(epi.bias);
  prm.residual = static_cast<const __half*>(epi.residual);
  prm.act = epi.act;
  prm.flip_taps = epi.flip_taps ? 1 : 0;
  const cudaError_t e =
      kGeomLaunch[dt][ki][si][mi][ni](map, prm, pl.grid, pl.smem, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TDC_OK : cuda_fail(e);
}

// ---------------------------------------------------------------------------
// Plain forward (tdc_plain.cuh) for the shapes the ws strips fit badly, and
// the choice between it and the ws kernel.
// ---------------------------------------------------------------------------
using PlainLaunchFn = cudaError_t (*)(const tdc::PlainParams&, int64_t, cudaStream_t);

template <int K, int S, class E, bool EPI>
cudaError_t plain_launch_t(const tdc::PlainParams& prm, int64_t grid, cudaStream_t st) {
  return launch_pdl_block(&tdc::dwconv_plain_kernel<K, S, E, EPI>, grid,
                          unsigned(tdc::kPlainThreads), 0, st, prm);
}

#define TDC_PLAIN_EPI(E, K, S) {plain_launch_t<K, S, E, false>, plain_launch_t<K, S, E, true>}
#define TDC_PLAIN_TABLE(E)                                                  \
  {{TDC_PLAIN_EPI(E, 3, 1), TDC_PLAIN_EPI(E, 3, 2)},                        \
   {TDC_PLAIN_EPI(E, 5, 1), TDC_PLAIN_EPI(E, 5, 2)},                        \
   {TDC_PLAIN_EPI(E, 7, 1), TDC_PLAIN_EPI(E, 7, 2)}}
// [element type][K index: 3, 5, 7][stride - 1][epilogue]
const PlainLaunchFn kPlainLaunch[2][3][2][2] = {TDC_PLAIN_TABLE(tdc::F16),
                                                TDC_PLAIN_TABLE(tdc::BF16)};
#undef TDC_PLAIN_TABLE
#undef TDC_PLAIN_EPI

// Output rows per thread of the plain kernel: the whole height unless that
// leaves fewer than 384 threads per SM (about one wave at the kernels' 120-160
// registers), in which case the height is cut into bands, each re-reading its
// K - S halo rows.  Measured on MobileNet / EfficientNet layers at batch 64
// (us, band rows 1 / 2 / 4 / 7 / 14): 112 x 112 x 16: 39 / 29 / 24 / 24 / 26;
// 14 x 14 x 576: 26 / 20 / 17 / 15 / 17; 7 x 7 x 960 5x5: 32 / 25 / 17 / 15.
int64_t plain_band_rows(int64_t N, int64_t P, int64_t Q, int64_t C, int64_t K, int64_t sms) {
  const int64_t qgroups = (Q + tdc::plain_cols(int(K)) - 1) / tdc::plain_cols(int(K));
  const int64_t per_band = std::max<int64_t>(1, N * qgroups * (C / 2));
  const int64_t want = 384 * std::max<int64_t>(1, sms);
  const int64_t bands = std::min<int64_t>(P, std::max<int64_t>(1, (want + per_band - 1) / per_band));
  return (P + bands - 1) / bands;
}

int fwd_plain(const void* x, const void* w, void* y, int64_t N, int64_t H, int64_t W, int64_t C,
              int64_t K, int64_t S, int64_t pad, int64_t band_rows, const Epilogue& epi,
              void* stream, int dt, const Pad4* p4 = nullptr) {
  const Pad4 pd = p4 ? *p4 : Pad4{pad, pad, pad, pad};
  if (K != 3 && K != 5 && K != 7) return TDC_ERR_FILTER_SHAPE;
  if (S != 1 && S != 2) return TDC_ERR_STRIDE;
  if (N < 0 || H < 1 || W < 1 || C < 0 || band_rows < 0) return TDC_ERR_BAD_SHAPE;
  if (C % 8 != 0) return TDC_ERR_CHANNELS;
  if (!epi.flip_taps && (pd.top < 0 || pd.bottom < 0 || pd.left < 0 || pd.right < 0))
    return TDC_ERR_PAD;
  for (int64_t v : {pd.top, pd.bottom, pd.left, pd.right})
    if (v > (1 << 28) || v < -(1 << 28)) return TDC_ERR_TOO_LARGE;
  if (H + pd.top + pd.bottom < K || W + pd.left + pd.right < K) return TDC_ERR_BAD_SHAPE;
  const int64_t P = (H + pd.top + pd.bottom - K) / S + 1, Q = (W + pd.left + pd.right - K) / S + 1;
  if (N == 0 || C == 0) return TDC_OK;
  if (!x || !w || !y) return TDC_ERR_NULL_POINTER;
  if (!aligned16(x) || !aligned16(w) || !aligned16(y) || (epi.bias && !aligned16(epi.bias)) ||
      (epi.residual && !aligned16(epi.residual)))
    return TDC_ERR_ALIGNMENT;
  // 32-bit row / column arithmetic in the kernel (S * p0 - pad, S * q - pad + s)
  // and a 32-bit thread index.
  const int64_t i32 = 0x7fffffffll;
  if (N > i32 || C > i32 || H + std::abs(pd.top) + std::abs(pd.bottom) > i32 ||
      W + std::abs(pd.left) + std::abs(pd.right) > i32)
    return TDC_ERR_TOO_LARGE;
  if (N * Q > i32 || N * Q * (C / 2) > i32) return TDC_ERR_TOO_LARGE;
  if (H * W > i32 || H * W * (C / 2) > i32) return TDC_ERR_TOO_LARGE;  // 32-bit image offsets
  DeviceInfo* dev = nullptr;
  int rc = current_device(&dev, nullptr);
  if (rc != TDC_OK) return rc;
  const int64_t cpairs = C / 2;
  const int chunk_log2 = cpairs % 8 == 0 ? 3 : 2;  // 32- or 16-byte chunks (C % 8 == 0)
  const int64_t qgroups = (Q + tdc::plain_cols(int(K)) - 1) / tdc::plain_cols(int(K));
  const int64_t rows =
      band_rows > 0 ? std::min(band_rows, P) : plain_band_rows(N, P, Q, C, K, dev->sms);
  const int64_t bands = (P + rows - 1) / rows;
  const int64_t total = N * qgroups * cpairs * bands;  // < 2^62: both factors < 2^31
  if (total > 0xffffffffll - tdc::kPlainThreads) return TDC_ERR_TOO_LARGE;
  tdc::PlainParams prm{};
  prm.x = static_cast<const uint32_t*>(x);
  prm.w = static_cast<const uint32_t*>(w);
  prm.bias = static_cast<const uint32_t*>(epi.bias);
  prm.residual = static_cast<const uint32_t*>(epi.residual);
  prm.y = static_cast<uint32_t*>(y);
  prm.total = uint32_t(total);
  prm.H = int32_t(H); prm.W = int32_t(W); prm.P = int32_t(P); prm.Q = int32_t(Q);
  prm.qgroups = int32_t(qgroups);
  prm.cpairs = int32_t(cpairs);
  prm.chunk_log2 = chunk_log2;
  prm.chunks = int32_t(cpairs >> chunk_log2);
  prm.bands = int32_t(bands);
  prm.band_rows = int32_t(rows);
  prm.pad = int32_t(pd.top);
  prm.pad_w = int32_t(pd.left);
  prm.act = epi.act;
  prm.flip_taps = epi.flip_taps ? 1 : 0;
  prm.dil = 1;
  prm.phases = 1;
  const bool with_epilogue =
      epi.bias != nullptr || epi.residual != nullptr || epi.act != TDC_ACT_NONE;
  const int64_t grid = (total + tdc::kPlainThreads - 1) / tdc::kPlainThreads;
  const cudaError_t e = kPlainLaunch[dt][K / 2 - 1][S - 1][with_epilogue ? 1 : 0](
      prm, grid, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TDC_OK : cuda_fail(e);
}

// Dilated forward: the plain kernel on the D*D phases of the output (see
// PlainParams::dil).
// Ring depth of the ws forward per geometry when the caller leaves it to the
// library (n_stage = 0), measured at 64 x 224 x 336 x 256.
int default_fwd_stages(int64_t K, int64_t S) {
  return (K == 3 || K == 5 || K == 7) && (S == 1 || S == 2) ? fwd_stages_of(int(K), int(S)) : 2;
}

// Whether the plain kernel beats the ws kernel on this shape.  The ws kernel
// works in strips of 32 output columns x 64 channels; fill_c and fill_q are
// the fractions of a strip's lanes and columns that hold real outputs.  From
// both kernels timed on the 28 depthwise layers of MobileNetV2 / V3-Large /
// EfficientNet-B0 at batch 64 and 256: with fill_c * fill_q >= 0.5 the ws
// kernel wins or ties everywhere; below it the plain kernel wins at stride 1
// (e.g. 14 x 14 x 576: 10.3 vs 12.8 us, 112 x 112 x 16: 18.2 vs 44.4 us) and
// at stride 2 on 7-column outputs or layers under 64 MB, while larger
// stride-2 layers with wider outputs stay on the ws kernel (28 x 28 x 192 at
// batch 256: 20.2 vs 26.1 us).
bool prefer_plain_pq(int64_t Q, int64_t C, int64_t S, double bytes) {
  const double fill_c = double(C) / double(64 * ((C + 63) / 64));
  const double fill_q = double(Q) / double(32 * ((Q + 31) / 32));
  if (fill_c * fill_q >= 0.5) return false;
  return S == 1 || fill_q <= 0.25 || bytes < 64e6;
}

bool prefer_plain_pads(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K, int64_t S,
                       const Pad4& pd) {
  if (K != 3 && K != 5 && K != 7) return false;
  if ((S != 1 && S != 2) || C <= 0 || C % 8 != 0 || N <= 0) return false;
  if (H + pd.top + pd.bottom < K || W + pd.left + pd.right < K) return false;
  const int64_t P = (H + pd.top + pd.bottom - K) / S + 1, Q = (W + pd.left + pd.right - K) / S + 1;
  const double bytes = 2.0 * double(N) * double(C) * (double(H) * double(W) + double(P) * double(Q));
  return prefer_plain_pq(Q, C, S, bytes);
}

bool prefer_plain(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K, int64_t S,
                  int64_t pad) {
  return prefer_plain_pads(N, H, W, C, K, S, Pad4{pad, pad, pad, pad});
}

// Whether the ring kernel's tensor map can step D rows and columns: the box
// spans D * (input columns of a strip) columns and D * stage_rows rows (the
// dilated ring runs at the geometry's default depth).
bool dilated_ring_fits(int64_t K, int64_t S, int64_t D) {
  return D >= 1 && D <= kMaxTmaStride && strip_in_cols(int(K), int(S)) * D <= kMaxTmaBox &&
         geom_stage_rows(int(K), int(S), default_fwd_stages(K, S)) * D <= kMaxTmaBox;
}

// Whether the dilated forward with n_stage = 0 runs the plain kernel.  The
// ring kernel takes the phase sub-problems (ceil(P/D) x ceil(Q/D) outputs
// each) where its map can step D, the undilated choice would give them the
// ring kernel, and both sides are at least 32: on smaller phases its
// strips are short and the plain kernel wins.  Measured on one B200 (us,
// plain / ring; CUDA graphs): 32 x 128 x 128 x 256 3x3 D2 154.6 / 102.1,
// 16 x 112 x 112 x 384 5x5 D2 160.2 / 120.3, 16 x 128 x 128 x 256 3x3 D4
// 81.2 / 55.4, 8 x 64 x 64 x 256 3x3 D2 11.5 / 10.3; phases under 32:
// 8 x 64 x 64 x 256 D4 11.4 / 18.4, 8 x 128 x 128 x 128 D6 21.3 / 22.5,
// 8 x 32 x 32 x 960 5x5 D2 20.7 / 23.7, 32 x 64 x 64 x 512 stride 2 D2
// 31.1 / 32.7.
bool dilated_prefers_plain(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K, int64_t S,
                           int64_t D, int64_t P, int64_t Q) {
  const int64_t Pp = (P + D - 1) / D, Qp = (Q + D - 1) / D;
  const double bytes = 2.0 * double(N) * double(C) * (double(H) * double(W) + double(P) * double(Q));
  return !dilated_ring_fits(K, S, D) || std::min(Pp, Qp) < 32 ||
         prefer_plain_pq(Qp, C, S, bytes);
}

// Dilated forward on the ring kernel: the N*D*D phase sub-problems (each
// an undilated K x K stride-S problem on the D-strided sub-lattice of x,
// loaded with traversal stride D) are scheduled as N*D*D images of the
// largest phase's ceil(P/D) x ceil(Q/D) outputs; the kernel maps a phase's
// output (p', q') to y's (pa + D*p', pb + D*q').  Arguments are checked by
// fwd_dilated.
int fwd_dilated_ring(const void* x, const void* w, void* y, int64_t N, int64_t H, int64_t W,
                     int64_t C, int64_t K, int64_t S, int64_t D, int64_t P, int64_t Q,
                     const Pad4& pd, const Epilogue& epi, void* stream, int dt) {
  if (D < 2 || !dilated_ring_fits(K, S, D)) return TDC_ERR_UNSUPPORTED;
  const int64_t n_stage = default_fwd_stages(K, S);
  const int64_t Pp = (P + D - 1) / D, Qp = (Q + D - 1) / D;
  const int stage_rows = geom_stage_rows(int(K), int(S), n_stage);
  const int in_cols = strip_in_cols(int(K), int(S));
  // 32-bit tensor-map coordinates (row S*pa - pad + D*S*p0 + D*t*stage_rows,
  // column S*pb - pad_w + D*S*32*qs, plus the box) and column step D*C.
  const int64_t i32 = 0x7fffffffll;
  if (N * D * D > i32 || D * C > i32 ||
      D * S * (2 * Pp + 2) + D * (K + 2 * stage_rows) + pd.top > i32 ||
      D * S * (Qp + tdc::kStripQ + 1) + D * in_cols + pd.left > i32)
    return TDC_ERR_TOO_LARGE;
  int rc = check_ws_limits(N, H, W, C, P, Q);
  if (rc != TDC_OK) return rc;
  DeviceInfo* dev = nullptr;
  int devi = -1;
  rc = current_device(&dev, &devi);
  if (rc != TDC_OK) return rc;
  const bool with_epilogue =
      epi.bias != nullptr || epi.residual != nullptr || epi.act != TDC_ACT_NONE;
  const int ki = int(K / 2 - 1), si = int(S - 1), mi = with_epilogue ? 1 : 0;
  const WsPlan pl1 = make_geom_plan(1, 1, 1, 8, int(K), int(S), n_stage, 1, 1);
  int occ;
  {
    std::lock_guard<std::mutex> lock(g_geom_mutex);
    occ = g_dil_occ[devi][dt][ki][si][mi];
    if (occ == 0) {
      const cudaError_t e = kDilOcc[dt][ki][si][mi](&occ, pl1.smem);
      if (e != cudaSuccess) return cuda_fail(e);
      occ = std::max(1, occ);
      g_dil_occ[devi][dt][ki][si][mi] = occ;
    }
  }
  const WsPlan pl = make_geom_plan(N * D * D, Pp, Qp, C, int(K), int(S), n_stage, dev->sms, occ);
  alignas(64) CUtensorMap map;
  rc = encode_nhwc_map(&map, x, N, H, W, C, in_cols, stage_rows, dt, int(D));
  if (rc != TDC_OK) return rc;
  tdc::WsParams prm{};
  prm.status_host = current_status_slot(true);
  prm.w = static_cast<const __half*>(w);
  prm.y = static_cast<__half*>(y);
  prm.H = int32_t(H); prm.W = int32_t(W); prm.C = int32_t(C);
  prm.P = int32_t(Pp); prm.Q = int32_t(Qp); prm.pad = int32_t(pd.top); prm.pad_w = int32_t(pd.left);
  prm.dil = int32_t(D); prm.yP = int32_t(P); prm.yQ = int32_t(Q);
  prm.qstrips = pl.qstrips; prm.cblocks = pl.cblocks; prm.stage_rows = pl.stage_rows;
  prm.tail_bands = pl.tail_bands; prm.tail_band_rows = pl.tail_band_rows;
  prm.full_units = pl.full_units; prm.tail_strips = pl.tail_strips;
  prm.tail_chunk_rows = pl.tail_chunk_rows;
  prm.timeout_ns = uint64_t(g_timeout_ns.load());
  prm.withhold = -1;
  prm.bias = static_cast<const __half*>(epi.bias);
  prm.residual = static_cast<const __half*>(epi.residual);
  prm.act = epi.act;
  const cudaError_t e =
      kDilLaunch[dt][ki][si][mi](map, prm, pl.grid, pl.smem, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TDC_OK : cuda_fail(e);
}

// Dilated forward.  kernel = 1: the ring kernel (TDC_ERR_UNSUPPORTED when
// its tensor map cannot step D, or D = 1); -1: the plain kernel; 0: chosen
// by shape (dilated_prefers_plain).
int fwd_dilated(const void* x, const void* w, void* y, int64_t N, int64_t H, int64_t W,
                int64_t C, int64_t K, int64_t S, int64_t D, const Pad4& pd, const Epilogue& epi,
                int64_t kernel, void* stream, int dt) {
  if (K != 3 && K != 5 && K != 7) return TDC_ERR_FILTER_SHAPE;
  if (S != 1 && S != 2) return TDC_ERR_STRIDE;
  if (D < 1) return TDC_ERR_BAD_SHAPE;
  if (N < 0 || H < 1 || W < 1 || C < 0) return TDC_ERR_BAD_SHAPE;
  if (C % 8 != 0) return TDC_ERR_CHANNELS;
  if (pd.top < 0 || pd.bottom < 0 || pd.left < 0 || pd.right < 0) return TDC_ERR_PAD;
  if (kernel < -1 || kernel > 1) return TDC_ERR_UNSUPPORTED;
  const int64_t i32 = 0x7fffffffll;
  if (D > (1 << 24) || std::max({pd.top, pd.bottom, pd.left, pd.right}) > (1 << 28) ||
      N > i32 || C > i32 || H > i32 || W > i32)
    return TDC_ERR_TOO_LARGE;
  const int64_t Ke = D * (K - 1) + 1;  // the dilated kernel's extent
  if (H + pd.top + pd.bottom < Ke || W + pd.left + pd.right < Ke) return TDC_ERR_BAD_SHAPE;
  const int64_t P = (H + pd.top + pd.bottom - Ke) / S + 1, Q = (W + pd.left + pd.right - Ke) / S + 1;
  if (N == 0 || C == 0) return TDC_OK;
  if (!x || !w || !y) return TDC_ERR_NULL_POINTER;
  if (!aligned16(x) || !aligned16(w) || !aligned16(y) || (epi.bias && !aligned16(epi.bias)) ||
      (epi.residual && !aligned16(epi.residual)))
    return TDC_ERR_ALIGNMENT;
  if (kernel == 0) kernel = dilated_prefers_plain(N, H, W, C, K, S, D, P, Q) ? -1 : 1;
  if (kernel == 1) return fwd_dilated_ring(x, w, y, N, H, W, C, K, S, D, P, Q, pd, epi, stream, dt);
  // 32-bit row / column arithmetic in the plain kernel: a thread's first input row
  // S * (phase + D * p0) - pad plus D * (its window rows), likewise columns
  // with S * plain_cols(K) - S + K window columns.
  if (S * P + D * (S + K) + pd.top > i32 ||
      S * Q + D * (S * tdc::plain_cols(int(K)) + K) + pd.left > i32)
    return TDC_ERR_TOO_LARGE;
  if (H * W > i32 || H * W * (C / 2) > i32) return TDC_ERR_TOO_LARGE;  // 32-bit image offsets
  DeviceInfo* dev = nullptr;
  int rc = current_device(&dev, nullptr);
  if (rc != TDC_OK) return rc;
  const int64_t cpairs = C / 2;
  const int chunk_log2 = cpairs % 8 == 0 ? 3 : 2;
  // The largest phase: ceil(P / D) rows, ceil(Q / D) columns; D*D phases
  // per image.
  const int64_t Pp = (P + D - 1) / D, Qp = (Q + D - 1) / D;
  const int64_t qgroups = (Qp + tdc::plain_cols(int(K)) - 1) / tdc::plain_cols(int(K));
  if (N * D * D > i32 || N * D * D * qgroups > i32 || N * D * D * qgroups * cpairs > i32)
    return TDC_ERR_TOO_LARGE;
  const int64_t rows = plain_band_rows(N * D * D, Pp, Qp, C, K, dev->sms);
  const int64_t bands = (Pp + rows - 1) / rows;
  const int64_t total = N * D * D * qgroups * cpairs * bands;
  if (total > 0xffffffffll - tdc::kPlainThreads) return TDC_ERR_TOO_LARGE;
  tdc::PlainParams prm{};
  prm.x = static_cast<const uint32_t*>(x);
  prm.w = static_cast<const uint32_t*>(w);
  prm.bias = static_cast<const uint32_t*>(epi.bias);
  prm.residual = static_cast<const uint32_t*>(epi.residual);
  prm.y = static_cast<uint32_t*>(y);
  prm.total = uint32_t(total);
  prm.H = int32_t(H); prm.W = int32_t(W); prm.P = int32_t(P); prm.Q = int32_t(Q);
  prm.qgroups = int32_t(qgroups);
  prm.cpairs = int32_t(cpairs);
  prm.chunk_log2 = chunk_log2;
  prm.chunks = int32_t(cpairs >> chunk_log2);
  prm.bands = int32_t(bands);
  prm.band_rows = int32_t(rows);
  prm.pad = int32_t(pd.top);
  prm.pad_w = int32_t(pd.left);
  prm.act = epi.act;
  prm.dil = int32_t(D);
  prm.phases = int32_t(D * D);
  const bool with_epilogue =
      epi.bias != nullptr || epi.residual != nullptr || epi.act != TDC_ACT_NONE;
  const cudaError_t e = kPlainLaunch[dt][K / 2 - 1][S - 1][with_epilogue ? 1 : 0](
      prm, (total + tdc::kPlainThreads - 1) / tdc::kPlainThreads, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TDC_OK : cuda_fail(e);
}

// Plain weight gradient (tdc_plain.cuh): bands of dy rows chosen for about
// 1024 threads per SM counting the K tap rows, the units of one channel
// chunk summed per CTA, one workspace slice per unit group.
struct WgradPlainPlan {
  int64_t band_rows = 1, bands = 1, units = 0, ugroups = 0, chunks = 0;
  int chunk_log2 = 3;
};

int wgrad_plain_plan(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K, int64_t S,
                     int64_t pad, int64_t sms, WgradPlainPlan* pl, int64_t* P, int64_t* Q) {
  if (K != 3 && K != 5 && K != 7) return TDC_ERR_FILTER_SHAPE;
  if (S != 1 && S != 2) return TDC_ERR_STRIDE;
  if (N < 0 || H < 1 || W < 1 || C < 0) return TDC_ERR_BAD_SHAPE;
  if (C % 8 != 0) return TDC_ERR_CHANNELS;
  if (pad < 0) return TDC_ERR_PAD;
  if (pad > (1 << 28)) return TDC_ERR_TOO_LARGE;
  if (H + 2 * pad < K || W + 2 * pad < K) return TDC_ERR_BAD_SHAPE;
  *P = (H + 2 * pad - K) / S + 1;
  *Q = (W + 2 * pad - K) / S + 1;
  const int64_t i32 = 0x7fffffffll;
  const int64_t cpairs = C / 2;
  if (N > i32 || C > i32 || H + 2 * pad > i32 || W + 2 * pad > i32) return TDC_ERR_TOO_LARGE;
  if (H * W > i32 || H * W * cpairs > i32 || *P * *Q > i32 || *P * *Q * cpairs > i32)
    return TDC_ERR_TOO_LARGE;  // 32-bit offsets within an image
  pl->chunk_log2 = cpairs % 8 == 0 ? 3 : 2;
  pl->chunks = cpairs >> pl->chunk_log2;
  const int64_t per_band = std::max<int64_t>(1, N * cpairs * K);
  const int64_t want = 1024 * std::max<int64_t>(1, sms);
  const int64_t bands = std::min<int64_t>(*P, std::max<int64_t>(1, (want + per_band - 1) / per_band));
  pl->band_rows = (*P + bands - 1) / bands;
  pl->bands = (*P + pl->band_rows - 1) / pl->band_rows;
  pl->units = N * pl->bands;
  const int64_t upc = tdc::kPlainThreads >> pl->chunk_log2;
  pl->ugroups = (pl->units + upc - 1) / upc;
  if (pl->units > i32 || pl->ugroups * std::max<int64_t>(1, pl->chunks) > i32)
    return TDC_ERR_TOO_LARGE;
  return TDC_OK;
}

using WgradPlainLaunchFn = cudaError_t (*)(const tdc::WgradPlainParams&, int64_t, cudaStream_t);

// One CTA row per tap row (grid.y = K).
template <int K, int S, class E>
cudaError_t wgrad_plain_launch_t(const tdc::WgradPlainParams& prm, int64_t grid, cudaStream_t st) {
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(unsigned(grid), unsigned(K));
  cfg.blockDim = dim3(unsigned(tdc::kPlainThreads));
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  return cudaLaunchKernelEx(&cfg, &tdc::dwconv_wgrad_plain_kernel<K, S, E>, prm);
}

#define TDC_WGP_S(E, K) {wgrad_plain_launch_t<K, 1, E>, wgrad_plain_launch_t<K, 2, E>}
#define TDC_WGP_TABLE(E) {TDC_WGP_S(E, 3), TDC_WGP_S(E, 5), TDC_WGP_S(E, 7)}
// [element type][K index: 3, 5, 7][stride - 1]
const WgradPlainLaunchFn kWgradPlainLaunch[2][3][2] = {TDC_WGP_TABLE(tdc::F16),
                                                       TDC_WGP_TABLE(tdc::BF16)};
#undef TDC_WGP_TABLE
#undef TDC_WGP_S

int wgrad_plain_workspace(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K, int64_t S,
                          int64_t pad, int64_t* bytes) {
  if (!bytes) return TDC_ERR_NULL_POINTER;
  int64_t P, Q;
  WgradPlainPlan pl;
  int rc = wgrad_plain_plan(N, H, W, C, K, S, pad, 1, &pl, &P, &Q);  // shape checks first
  if (rc != TDC_OK) return rc;
  DeviceInfo* dev = nullptr;
  rc = current_device(&dev, nullptr);
  if (rc != TDC_OK) return rc;
  rc = wgrad_plain_plan(N, H, W, C, K, S, pad, dev->sms, &pl, &P, &Q);
  if (rc != TDC_OK) return rc;
  *bytes = pl.ugroups * K * K * C * int64_t(sizeof(float));
  return TDC_OK;
}

int wgrad_plain(int dt, const void* x, const void* dy, float* dw, int64_t N, int64_t H, int64_t W,
                int64_t C, int64_t K, int64_t S, int64_t pad, void* workspace,
                int64_t workspace_bytes, void* stream) {
  int64_t P, Q;
  WgradPlainPlan pl;
  int rc = wgrad_plain_plan(N, H, W, C, K, S, pad, 1, &pl, &P, &Q);  // shape checks first
  if (rc != TDC_OK) return rc;
  if (C == 0) return TDC_OK;
  if (!dw) return TDC_ERR_NULL_POINTER;
  if (N > 0 && (!x || !dy || !workspace)) return TDC_ERR_NULL_POINTER;
  if (!aligned16(dw) || (N > 0 && (!aligned16(x) || !aligned16(dy) || !aligned16(workspace))))
    return TDC_ERR_ALIGNMENT;
  DeviceInfo* dev = nullptr;
  rc = current_device(&dev, nullptr);
  if (rc != TDC_OK) return rc;
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (N == 0) {  // no products: the gradient is zero
    const cudaError_t e = cudaMemsetAsync(dw, 0, size_t(K * K * C) * sizeof(float), st);
    return e == cudaSuccess ? TDC_OK : cuda_fail(e);
  }
  rc = wgrad_plain_plan(N, H, W, C, K, S, pad, dev->sms, &pl, &P, &Q);
  if (rc != TDC_OK) return rc;
  if (workspace_bytes < pl.ugroups * K * K * C * int64_t(sizeof(float))) return TDC_ERR_WORKSPACE;
  tdc::WgradPlainParams prm{};
  prm.x = static_cast<const uint32_t*>(x);
  prm.dy = static_cast<const uint32_t*>(dy);
  prm.partial = static_cast<float*>(workspace);
  prm.H = int32_t(H); prm.W = int32_t(W); prm.P = int32_t(P); prm.Q = int32_t(Q);
  prm.cpairs = int32_t(C / 2);
  prm.chunk_log2 = pl.chunk_log2;
  prm.chunks = int32_t(pl.chunks);
  prm.bands = int32_t(pl.bands);
  prm.band_rows = int32_t(pl.band_rows);
  prm.units = int32_t(pl.units);
  prm.pad = int32_t(pad);
  cudaError_t e = kWgradPlainLaunch[dt][K / 2 - 1][S - 1](prm, pl.chunks * pl.ugroups, st);
  if (e == cudaSuccess)
    e = tdc::launch_wgrad_reduce(static_cast<const float*>(workspace), dw, int32_t(pl.ugroups),
                                 int32_t(K * K * C), st);
  return e == cudaSuccess ? TDC_OK : cuda_fail(e);
}

// ---------------------------------------------------------------------------
// Weight gradient of the K x K (K = 5, 7) stride-1 forward.
// ---------------------------------------------------------------------------
using WgradLaunchFn = cudaError_t (*)(const CUtensorMap&, const CUtensorMap&,
                                      const tdc::WgradParams&, int64_t, size_t, cudaStream_t);

// Tap-row passes of the K x K weight gradient: launch i covers rows
// [R0_i, R0_i + NR_i).  A single 7x7 pass would hold 98 sums per lane and
// spill at 128 registers (or drop to 1-2 CTAs per SM); two passes (rows 0-3,
// then 4-6) read x and dy twice but ran 11 % faster than the best single
// pass (3.54 vs 3.97 ms at 64 x 224 x 336 x 256).  5x5 runs as one pass
// (2.04 ms; split in 3 + 2 rows: 2.20 ms).
template <int K>
struct WgradPasses;
template <>
struct WgradPasses<3> {  // stride 2 only (the stride-1 3x3 has its own kernel)
  static constexpr int kCount = 1;
  static constexpr int kR0[2] = {0, 0};
  static constexpr int kNR[2] = {3, 0};
};
template <>
struct WgradPasses<5> {
  static constexpr int kCount = 1;
  static constexpr int kR0[2] = {0, 0};
  static constexpr int kNR[2] = {5, 0};
};
template <>
struct WgradPasses<7> {
  static constexpr int kCount = 2;
  static constexpr int kR0[2] = {0, 4};
  static constexpr int kNR[2] = {4, 3};
};

template <int NS, int K, int PASS, class E>
cudaError_t wgrad_kxk_launch_t(const CUtensorMap& xmap, const CUtensorMap& dymap,
                               const tdc::WgradParams& g, int64_t grid, size_t smem,
                               cudaStream_t st) {
  using WP = WgradPasses<K>;
  if constexpr (PASS < WP::kCount) {
    tdc::dwconv_wgrad_kxk_kernel<NS, K, WP::kR0[PASS], WP::kNR[PASS], 1, E>
        <<<dim3(unsigned(grid)), dim3(tdc::kWsThreads), smem, st>>>(xmap, dymap, g);
    return cudaGetLastError();
  } else {
    return cudaSuccess;
  }
}

template <int NS, int K, int PASS, class E>
cudaError_t wgrad_kxk_occ_t(int* occ, size_t smem) {
  using WP = WgradPasses<K>;
  if constexpr (PASS < WP::kCount) {
    auto* k = &tdc::dwconv_wgrad_kxk_kernel<NS, K, WP::kR0[PASS], WP::kNR[PASS], 1, E>;
    cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, k, tdc::kWsThreads, smem);
  } else {
    *occ = 1 << 20;  // no such pass: does not limit the grid
    return cudaSuccess;
  }
}

#define TDC_WGRAD_NS(FN, E, K, PASS) {FN<2, K, PASS, E>, FN<3, K, PASS, E>, FN<4, K, PASS, E>}
#define TDC_WGRAD_TABLE(FN, E)                                      \
  {{TDC_WGRAD_NS(FN, E, 5, 0), TDC_WGRAD_NS(FN, E, 5, 1)},          \
   {TDC_WGRAD_NS(FN, E, 7, 0), TDC_WGRAD_NS(FN, E, 7, 1)}}
// [element type][K index: 5, 7][pass][n_stage - 2]
const WgradLaunchFn kWgradKxkLaunch[2][2][2][3] = {TDC_WGRAD_TABLE(wgrad_kxk_launch_t, tdc::F16),
                                                   TDC_WGRAD_TABLE(wgrad_kxk_launch_t, tdc::BF16)};
const GeomOccFn kWgradKxkOcc[2][2][2][3] = {TDC_WGRAD_TABLE(wgrad_kxk_occ_t, tdc::F16),
                                            TDC_WGRAD_TABLE(wgrad_kxk_occ_t, tdc::BF16)};
#undef TDC_WGRAD_TABLE
#undef TDC_WGRAD_NS
int g_wgrad_kxk_occ[kMaxDevices][2][2][3] = {};  // min over passes; guarded by g_geom_mutex

int wgrad_kxk_passes(int K) { return K == 5 ? WgradPasses<5>::kCount : WgradPasses<7>::kCount; }
int wgrad_kxk_max_rows(int K) {  // the tallest pass's x window
  return K == 5 ? WgradPasses<5>::kNR[0] : WgradPasses<7>::kNR[0];
}

int wgrad_kxk_row_bytes(int K) { return (tdc::kStripQ + K - 1) * tdc::kBlockC * 2 + tdc::kDyRowBytes; }

// x rows one consumer step of the tallest pass holds: the tap rows of its dy
// rows (tdc::wgrad_dy_rows of them, S x rows apart).
int wgrad_window(int K, int S, int nr) { return S * (tdc::wgrad_dy_rows(K, S) - 1) + nr; }

// Ring of about 72 KB (3 CTAs per SM); the tallest pass's step window must
// fit, as in the direct forward.
int wgrad_kxk_stage_rows(int K, int64_t n_stage) {
  const int ns = int(n_stage);
  const int win = wgrad_window(K, 1, wgrad_kxk_max_rows(K));
  const int ring_rows = std::max(ns, (72 * 1024) / wgrad_kxk_row_bytes(K));
  const int sr = std::max(1, ring_rows / ns);
  return std::max(sr, (win - 1 + ns - 2) / (ns - 1) + (ns >= 3 ? 1 : 0));
}

WsPlan make_wgrad_kxk_plan(int64_t N, int64_t P, int64_t Q, int64_t C, int K, int64_t n_stage,
                           int64_t sms, int64_t ctas_per_sm) {
  WsPlan pl = make_plan(N, P, Q, C, n_stage, sms, ctas_per_sm);
  pl.stage_rows = wgrad_kxk_stage_rows(K, n_stage);
  pl.smem = size_t(n_stage) * pl.stage_rows * wgrad_kxk_row_bytes(K) + 128;
  return pl;
}

// Validates a K x K stride-1 weight-gradient call and plans its launch on the
// current device (which it binds).
int wgrad_kxk_plan(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K, int64_t pad,
                   int64_t n_stage, WsPlan* pl, int64_t* P, int64_t* Q, int dt = kF16) {
  if (N < 1 || H < 1 || W < 1 || C < 8) return TDC_ERR_BAD_SHAPE;
  if (C % 8 != 0) return TDC_ERR_CHANNELS;
  if (pad < 0) return TDC_ERR_PAD;
  if (pad > (1 << 28)) return TDC_ERR_TOO_LARGE;
  if (n_stage < 2 || n_stage > 4) return TDC_ERR_N_STAGE;
  *P = H + 2 * pad - K + 1;
  *Q = W + 2 * pad - K + 1;
  if (*P < 1 || *Q < 1) return TDC_ERR_BAD_SHAPE;
  int rc = check_ws_limits(N, H, W, C, *P, *Q);
  if (rc != TDC_OK) return rc;
  DeviceInfo* dev = nullptr;
  int devi = -1;
  rc = current_device(&dev, &devi);
  if (rc != TDC_OK) return rc;
  const int ki = K == 5 ? 0 : 1, ni = int(n_stage - 2);
  const size_t smem = make_wgrad_kxk_plan(1, 1, 1, 8, int(K), n_stage, 1, 1).smem;
  int occ;
  {
    // Every pass runs on the same grid (they share the workspace slices), so
    // the grid follows the pass with the lowest occupancy.
    std::lock_guard<std::mutex> lock(g_geom_mutex);
    occ = g_wgrad_kxk_occ[devi][dt][ki][ni];
    if (occ == 0) {
      occ = 1 << 20;
      for (int pass = 0; pass < 2; ++pass) {
        int o = 0;
        const cudaError_t e = kWgradKxkOcc[dt][ki][pass][ni](&o, smem);
        if (e != cudaSuccess) return cuda_fail(e);
        occ = std::min(occ, std::max(1, o));
      }
      g_wgrad_kxk_occ[devi][dt][ki][ni] = occ;
    }
  }
  *pl = make_wgrad_kxk_plan(N, *P, *Q, C, int(K), n_stage, dev->sms, occ);
  return TDC_OK;
}

int64_t wgrad_kxk_workspace_bytes(const WsPlan& pl, int64_t C, int64_t K) {
  return pl.grid * tdc::kConsumerWarps * K * K * C * int64_t(sizeof(float));
}

// ---------------------------------------------------------------------------
// Backward of the K x K stride-2 forward.
//   data gradient: dwconv_dgrad_s2_kernel<NS, K, pad & 1> over dx's strips;
//   weight gradient: dwconv_wgrad_kxk_kernel<NS, K, R0, NR, 2> over dy's
//   strips (tap rows split as at stride 1) + the fixed-order reduction.
// ---------------------------------------------------------------------------
using DgradS2LaunchFn = cudaError_t (*)(const CUtensorMap&, const tdc::DgradS2Params&, int64_t,
                                        size_t, cudaStream_t);

template <int NS, int K, int PODD, class E>
cudaError_t dgrad_s2_launch_t(const CUtensorMap& map, const tdc::DgradS2Params& g, int64_t grid,
                              size_t smem, cudaStream_t st) {
  tdc::dwconv_dgrad_s2_kernel<NS, K, PODD, E>
      <<<dim3(unsigned(grid)), dim3(tdc::kWsThreads), smem, st>>>(map, g);
  return cudaGetLastError();
}

template <int NS, int K, int PODD, class E>
cudaError_t dgrad_s2_occ_t(int* occ, size_t smem) {
  auto* k = &tdc::dwconv_dgrad_s2_kernel<NS, K, PODD, E>;
  cudaError_t e = cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
  if (e != cudaSuccess) return e;
  return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, k, tdc::kWsThreads, smem);
}

#define TDC_DGS2_NS(FN, E, K, PODD) {FN<2, K, PODD, E>, FN<3, K, PODD, E>, FN<4, K, PODD, E>}
#define TDC_DGS2_TABLE(FN, E)                                       \
  {{TDC_DGS2_NS(FN, E, 3, 0), TDC_DGS2_NS(FN, E, 3, 1)},            \
   {TDC_DGS2_NS(FN, E, 5, 0), TDC_DGS2_NS(FN, E, 5, 1)},            \
   {TDC_DGS2_NS(FN, E, 7, 0), TDC_DGS2_NS(FN, E, 7, 1)}}
// [element type][K index: 3, 5, 7][pad & 1][n_stage - 2]
const DgradS2LaunchFn kDgradS2Launch[2][3][2][3] = {TDC_DGS2_TABLE(dgrad_s2_launch_t, tdc::F16),
                                                    TDC_DGS2_TABLE(dgrad_s2_launch_t, tdc::BF16)};
const GeomOccFn kDgradS2Occ[2][3][2][3] = {TDC_DGS2_TABLE(dgrad_s2_occ_t, tdc::F16),
                                           TDC_DGS2_TABLE(dgrad_s2_occ_t, tdc::BF16)};
#undef TDC_DGS2_TABLE
#undef TDC_DGS2_NS
int g_dgrad_s2_occ[kMaxDevices][2][3][2][3] = {};  // guarded by g_geom_mutex

// dy columns of one 32-column dx strip (the TMA box width) and ring row bytes.
constexpr int dgrad_s2_dy_cols(int K) { return tdc::kStripQ / 2 + (K - 1) / 2; }
static_assert(dgrad_s2_dy_cols(3) == tdc::DgradS2Geom<3>::kDyCols &&
                  dgrad_s2_dy_cols(5) == tdc::DgradS2Geom<5>::kDyCols &&
                  dgrad_s2_dy_cols(7) == tdc::DgradS2Geom<7>::kDyCols,
              "host and device box widths agree");
int dgrad_s2_row_bytes(int K) { return dgrad_s2_dy_cols(K) * tdc::kBlockC * 2; }

// dy rows one pass holds at once: kHalf + pairs of dx rows per pass.
int dgrad_s2_window(int K) { return (K - 1) / 2 + tdc::dgrad_s2_pairs(K); }
static_assert(tdc::DgradS2Geom<3>::kWin == (1 + tdc::dgrad_s2_pairs(3)) &&
                  tdc::DgradS2Geom<7>::kWin == (3 + tdc::dgrad_s2_pairs(7)),
              "host and device windows agree");

// 16 dy rows split over the stages; a pass holds its window of consecutive
// rows, which needs (n_stage - 1) * sr >= window - 1.
int dgrad_s2_stage_rows(int K, int64_t n_stage) {
  const int ns = int(n_stage);
  const int sr = std::max(1, tdc::kDgradS2RingRows / ns);
  return std::max(sr, (dgrad_s2_window(K) - 1 + ns - 2) / (ns - 1));
}

WsPlan make_dgrad_s2_plan(int64_t N, int64_t H, int64_t W, int64_t C, int K, int64_t n_stage,
                          int64_t sms, int64_t ctas_per_sm) {
  WsPlan pl = make_plan(N, H, W, C, n_stage, sms, ctas_per_sm);
  pl.stage_rows = dgrad_s2_stage_rows(K, n_stage);
  pl.smem = size_t(n_stage) * pl.stage_rows * dgrad_s2_row_bytes(K) + 128;
  return pl;
}

// Validation shared by the stride-2 backward calls: dy [N,P,Q,C] with
// P = (H + 2*pad - K) / 2 + 1 >= 1, Q likewise.
int bwd_s2_shape(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K, int64_t pad,
                 int64_t n_stage, int64_t* P, int64_t* Q) {
  if (K != 3 && K != 5 && K != 7) return TDC_ERR_FILTER_SHAPE;
  if (N < 0 || H < 1 || W < 1 || C < 0) return TDC_ERR_BAD_SHAPE;
  if (C % 8 != 0) return TDC_ERR_CHANNELS;
  if (pad < 0) return TDC_ERR_PAD;
  if (pad > (1 << 28)) return TDC_ERR_TOO_LARGE;
  if (n_stage < 2 || n_stage > 4) return TDC_ERR_N_STAGE;
  if (H + 2 * pad < K || W + 2 * pad < K) return TDC_ERR_BAD_SHAPE;
  *P = (H + 2 * pad - K) / 2 + 1;
  *Q = (W + 2 * pad - K) / 2 + 1;
  return check_ws_limits(N, H, W, C, *P, *Q);
}

int dgrad_s2(const void* dy, const void* w, void* dx, int64_t N, int64_t H, int64_t W, int64_t C,
             int64_t K, int64_t pad, int64_t n_stage, void* stream, int dt = kF16) {
  int64_t P, Q;
  int rc = bwd_s2_shape(N, H, W, C, K, pad, n_stage, &P, &Q);
  if (rc != TDC_OK) return rc;
  if (N == 0 || C == 0) return TDC_OK;
  if (!dy || !w || !dx) return TDC_ERR_NULL_POINTER;
  if (!aligned16(dy) || !aligned16(w) || !aligned16(dx)) return TDC_ERR_ALIGNMENT;
  DeviceInfo* dev = nullptr;
  int devi = -1;
  rc = current_device(&dev, &devi);
  if (rc != TDC_OK) return rc;
  const int ki = int(K / 2 - 1), pi = int(pad & 1), ni = int(n_stage - 2);
  const size_t smem = make_dgrad_s2_plan(1, 1, 1, 8, int(K), n_stage, 1, 1).smem;
  int occ;
  {
    std::lock_guard<std::mutex> lock(g_geom_mutex);
    occ = g_dgrad_s2_occ[devi][dt][ki][pi][ni];
    if (occ == 0) {
      const cudaError_t e = kDgradS2Occ[dt][ki][pi][ni](&occ, smem);
      if (e != cudaSuccess) return cuda_fail(e);
      occ = std::max(1, occ);
      g_dgrad_s2_occ[devi][dt][ki][pi][ni] = occ;
    }
  }
  const WsPlan pl = make_dgrad_s2_plan(N, H, W, C, int(K), n_stage, dev->sms, occ);
  alignas(64) CUtensorMap map;
  rc = encode_nhwc_map(&map, dy, N, P, Q, C, dgrad_s2_dy_cols(int(K)), pl.stage_rows, dt);
  if (rc != TDC_OK) return rc;
  tdc::DgradS2Params g{};
  g.status_host = current_status_slot(true);
  g.w = static_cast<const __half*>(w);
  g.dx = static_cast<__half*>(dx);
  g.H = int32_t(H); g.W = int32_t(W); g.C = int32_t(C);
  g.P = int32_t(P); g.Q = int32_t(Q); g.pad = int32_t(pad);
  g.qstrips = pl.qstrips; g.cblocks = pl.cblocks; g.stage_rows = pl.stage_rows;
  g.tail_bands = pl.tail_bands; g.tail_band_rows = pl.tail_band_rows;
  g.full_units = pl.full_units; g.tail_strips = pl.tail_strips;
  g.timeout_ns = uint64_t(g_timeout_ns.load());
  const cudaError_t e =
      kDgradS2Launch[dt][ki][pi][ni](map, g, pl.grid, pl.smem, static_cast<cudaStream_t>(stream));
  return e == cudaSuccess ? TDC_OK : cuda_fail(e);
}

template <int NS, int K, int PASS, class E>
cudaError_t wgrad_s2_launch_t(const CUtensorMap& xmap, const CUtensorMap& dymap,
                              const tdc::WgradParams& g, int64_t grid, size_t smem,
                              cudaStream_t st) {
  using WP = WgradPasses<K>;
  if constexpr (PASS < WP::kCount) {
    tdc::dwconv_wgrad_kxk_kernel<NS, K, WP::kR0[PASS], WP::kNR[PASS], 2, E>
        <<<dim3(unsigned(grid)), dim3(tdc::kWsThreads), smem, st>>>(xmap, dymap, g);
    return cudaGetLastError();
  } else {
    return cudaSuccess;
  }
}

template <int NS, int K, int PASS, class E>
cudaError_t wgrad_s2_occ_t(int* occ, size_t smem) {
  using WP = WgradPasses<K>;
  if constexpr (PASS < WP::kCount) {
    auto* k = &tdc::dwconv_wgrad_kxk_kernel<NS, K, WP::kR0[PASS], WP::kNR[PASS], 2, E>;
    cudaError_t e =
        cudaFuncSetAttribute(k, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxDynSmem);
    if (e != cudaSuccess) return e;
    return cudaOccupancyMaxActiveBlocksPerMultiprocessor(occ, k, tdc::kWsThreads, smem);
  } else {
    *occ = 1 << 20;  // no such pass: does not limit the grid
    return cudaSuccess;
  }
}

#define TDC_WGS2_NS(FN, E, K, PASS) {FN<2, K, PASS, E>, FN<3, K, PASS, E>, FN<4, K, PASS, E>}
#define TDC_WGS2_TABLE(FN, E)                                       \
  {{TDC_WGS2_NS(FN, E, 3, 0), TDC_WGS2_NS(FN, E, 3, 1)},            \
   {TDC_WGS2_NS(FN, E, 5, 0), TDC_WGS2_NS(FN, E, 5, 1)},            \
   {TDC_WGS2_NS(FN, E, 7, 0), TDC_WGS2_NS(FN, E, 7, 1)}}
// [element type][K index: 3, 5, 7][pass][n_stage - 2]
const WgradLaunchFn kWgradS2Launch[2][3][2][3] = {TDC_WGS2_TABLE(wgrad_s2_launch_t, tdc::F16),
                                                  TDC_WGS2_TABLE(wgrad_s2_launch_t, tdc::BF16)};
const GeomOccFn kWgradS2Occ[2][3][2][3] = {TDC_WGS2_TABLE(wgrad_s2_occ_t, tdc::F16),
                                           TDC_WGS2_TABLE(wgrad_s2_occ_t, tdc::BF16)};
#undef TDC_WGS2_TABLE
#undef TDC_WGS2_NS
int g_wgrad_s2_occ[kMaxDevices][2][3][3] = {};  // min over passes; guarded by g_geom_mutex

int wgrad_s2_passes(int K) {
  return K == 3 ? WgradPasses<3>::kCount : wgrad_kxk_passes(K);
}
int wgrad_s2_max_rows(int K) { return K == 3 ? WgradPasses<3>::kNR[0] : wgrad_kxk_max_rows(K); }

// One stage row = 2 x rows of S*31 + K = 62 + K columns and 1 dy row.
int wgrad_s2_row_bytes(int K) { return 2 * (62 + K) * tdc::kBlockC * 2 + tdc::kDyRowBytes; }

// Ring of about 72 KB; the tallest pass's step window of x rows must fit:
// (n_stage - 1) * 2 * sr >= window - 1.
int wgrad_s2_stage_rows(int K, int64_t n_stage) {
  const int ns = int(n_stage);
  const int win = wgrad_window(K, 2, wgrad_s2_max_rows(K));
  const int ring_rows = std::max(ns, (72 * 1024) / wgrad_s2_row_bytes(K));
  const int sr = std::max(1, ring_rows / ns);
  return std::max(sr, (win - 1 + 2 * (ns - 1) - 1) / (2 * (ns - 1)));
}

WsPlan make_wgrad_s2_plan(int64_t N, int64_t P, int64_t Q, int64_t C, int K, int64_t n_stage,
                          int64_t sms, int64_t ctas_per_sm) {
  WsPlan pl = make_plan(N, P, Q, C, n_stage, sms, ctas_per_sm);
  pl.stage_rows = wgrad_s2_stage_rows(K, n_stage);
  pl.smem = size_t(n_stage) * pl.stage_rows * wgrad_s2_row_bytes(K) + 128;
  return pl;
}

// Validates a stride-2 weight-gradient call and plans its launch on the
// current device.
int wgrad_s2_plan(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K, int64_t pad,
                  int64_t n_stage, WsPlan* pl, int64_t* P, int64_t* Q, int dt = kF16) {
  int rc = bwd_s2_shape(N, H, W, C, K, pad, n_stage, P, Q);
  if (rc != TDC_OK) return rc;
  if (N < 1 || C < 8) return TDC_ERR_BAD_SHAPE;
  DeviceInfo* dev = nullptr;
  int devi = -1;
  rc = current_device(&dev, &devi);
  if (rc != TDC_OK) return rc;
  const int ki = int(K / 2 - 1), ni = int(n_stage - 2);
  const size_t smem = make_wgrad_s2_plan(1, 1, 1, 8, int(K), n_stage, 1, 1).smem;
  int occ;
  {
    std::lock_guard<std::mutex> lock(g_geom_mutex);
    occ = g_wgrad_s2_occ[devi][dt][ki][ni];
    if (occ == 0) {
      occ = 1 << 20;
      for (int pass = 0; pass < 2; ++pass) {
        int o = 0;
        const cudaError_t e = kWgradS2Occ[dt][ki][pass][ni](&o, smem);
        if (e != cudaSuccess) return cuda_fail(e);
        occ = std::min(occ, std::max(1, o));
      }
      g_wgrad_s2_occ[devi][dt][ki][ni] = occ;
    }
  }
  *pl = make_wgrad_s2_plan(N, *P, *Q, C, int(K), n_stage, dev->sms, occ);
  return TDC_OK;
}

int wgrad_s2(const void* x, const void* dy, float* dw, int64_t N, int64_t H, int64_t W, int64_t C,
             int64_t K, int64_t pad, int64_t n_stage, void* workspace, int64_t workspace_bytes,
             void* stream, int dt = kF16) {
  if (!x || !dy || !dw || !workspace) return TDC_ERR_NULL_POINTER;
  if (!aligned16(x) || !aligned16(dy) || !aligned16(dw) || !aligned16(workspace))
    return TDC_ERR_ALIGNMENT;
  WsPlan pl;
  int64_t P, Q;
  int rc = wgrad_s2_plan(N, H, W, C, K, pad, n_stage, &pl, &P, &Q, dt);
  if (rc != TDC_OK) return rc;
  if (workspace_bytes < wgrad_kxk_workspace_bytes(pl, C, K)) return TDC_ERR_WORKSPACE;
  alignas(64) CUtensorMap xmap, dymap;
  rc = encode_nhwc_map(&xmap, x, N, H, W, C, 62 + int(K), 2 * pl.stage_rows, dt);
  if (rc != TDC_OK) return rc;
  rc = encode_dy_map(&dymap, dy, N, P, Q, C, pl.stage_rows, dt);
  if (rc != TDC_OK) return rc;
  tdc::WgradParams g{};
  g.status_host = current_status_slot(true);
  g.partial = static_cast<float*>(workspace);
  g.C = int32_t(C); g.P = int32_t(P); g.Q = int32_t(Q); g.pad = int32_t(pad);
  g.qstrips = pl.qstrips; g.cblocks = pl.cblocks; g.stage_rows = pl.stage_rows;
  g.tail_bands = pl.tail_bands; g.tail_band_rows = pl.tail_band_rows;
  g.full_units = pl.full_units; g.tail_strips = pl.tail_strips;
  g.timeout_ns = uint64_t(g_timeout_ns.load());
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int ki = int(K / 2 - 1);
  for (int pass = 0; pass < wgrad_s2_passes(int(K)); ++pass) {
    const cudaError_t e =
        kWgradS2Launch[dt][ki][pass][n_stage - 2](xmap, dymap, g, pl.grid, pl.smem, st);
    if (e != cudaSuccess) return cuda_fail(e);
  }
  const int n = int(K * K * C);
  const cudaError_t e = tdc::launch_wgrad_reduce(static_cast<const float*>(workspace), dw,
                                int32_t(pl.grid * tdc::kConsumerWarps), n, st);
  return e == cudaSuccess ? TDC_OK : cuda_fail(e);
}

// ---------------------------------------------------------------------------
// Pipelined call with host buffers (tdc_dwconv_ws_host): the batch goes in
// chunks of images over three library-owned streams per device, one for the
// host->device copies, one for the kernels and one for the device->host
// copies, chained by events, so the two copy directions and the kernels
// overlap.  The streams and events are created once per device and reused;
// the enqueue is serialised per device, so calls from several host threads
// do not share an event in flight.
// ---------------------------------------------------------------------------
struct HostPipe {
  std::mutex m;
  bool ready = false;
  cudaStream_t s[3] = {nullptr, nullptr, nullptr};  // h2d, kernels, d2h
  cudaEvent_t start = nullptr, end = nullptr;
  std::vector<cudaEvent_t> copied, computed;        // per chunk
};
HostPipe g_pipe[kMaxDevices];

cudaError_t pipe_events(std::vector<cudaEvent_t>& v, size_t n) {
  while (v.size() < n) {
    cudaEvent_t e;
    const cudaError_t r = cudaEventCreateWithFlags(&e, cudaEventDisableTiming);
    if (r != cudaSuccess) return r;
    v.push_back(e);
  }
  return cudaSuccess;
}

cudaError_t pipe_ready(HostPipe& hp) {
  if (hp.ready) return cudaSuccess;
  for (auto& st : hp.s) {
    if (st) continue;
    const cudaError_t r = cudaStreamCreateWithFlags(&st, cudaStreamNonBlocking);
    if (r != cudaSuccess) return r;
  }
  cudaError_t r = hp.start ? cudaSuccess : cudaEventCreateWithFlags(&hp.start, cudaEventDisableTiming);
  if (r == cudaSuccess && !hp.end) r = cudaEventCreateWithFlags(&hp.end, cudaEventDisableTiming);
  hp.ready = r == cudaSuccess;
  return r;
}

}  // namespace

extern "C" {

TDC_API const char* tdc_strerror(int code) {
  switch (code) {
    case TDC_OK: return "success";
    case TDC_ERR_NULL_POINTER: return "null pointer argument";
    case TDC_ERR_BAD_SHAPE: return "bad shape: N,H,W,C must be non-negative with H,W >= 1 and a non-negative output size";
    case TDC_ERR_FILTER_SHAPE: return "only 3x3 kernel supported (5x5 and 7x7 through tdc_dwconv_fwd)";
    case TDC_ERR_CHANNELS: return "C must be a multiple of 8 (v0, general forward) or 64 (ws)";
    case TDC_ERR_PAD: return "pad must be non-negative";
    case TDC_ERR_N_STAGE: return "n_stage must be one of {2, 3, 4}";
    case TDC_ERR_ALIGNMENT: return "x, w and y must be 16-byte aligned";
    case TDC_ERR_TOO_LARGE: return "problem exceeds the TMA descriptor / 32-bit field limits";
    case TDC_ERR_CUDA: return "a CUDA runtime call failed";
    case TDC_ERR_TMA_ENCODE: return "cuTensorMapEncodeTiled failed";
    case TDC_ERR_DEVICE_TIMEOUT: return "an earlier launch on this device gave up waiting on a pipeline barrier and left its output incomplete; tdc_device_status(1, info) (tma_dwconv.device_status) reports and clears the record";
    case TDC_ERR_NO_DEVICE: return "no sm_100 CUDA device is current";
    case TDC_ERR_WORKSPACE: return "workspace smaller than tdc_dwconv3x3_bwd_weight_workspace reports";
    case TDC_ERR_SCRATCH_LIMIT: return "C too large for the 16 MiB static scratch of tdc_dwconv3x3_bwd_weight_noalloc (C <= 116508)";
    case TDC_ERR_STRIDE: return "stride must be 1 or 2";
    case TDC_ERR_UNSUPPORTED: return "not implemented for this geometry";
    case TDC_ERR_ACT: return "activation code is not one of TDC_ACT_NONE, _RELU, _RELU6, _SILU";
    default: return "unknown tdc status code";
  }
}

TDC_API int tdc_last_cuda_error(void) { return t_last_cuda_error; }

TDC_API int tdc_output_hw(int64_t H, int64_t W, int64_t R, int64_t S, int64_t pad, int64_t* P,
                          int64_t* Q) {
  if (!P || !Q) return TDC_ERR_NULL_POINTER;
  if (pad < 0) return TDC_ERR_PAD;
  *P = H + 2 * pad - R + 1;
  *Q = W + 2 * pad - S + 1;
  return TDC_OK;
}

TDC_API int tdc_dwconv_v0(const void* x, const void* w, void* y, int64_t N, int64_t H, int64_t W,
                          int64_t C, int64_t R, int64_t S, int64_t pad, void* stream) {
  int64_t P = 0, Q = 0;
  bool empty = false;
  int rc = validate(x, w, y, N, H, W, C, R, S, pad, 8, &P, &Q, &empty);
  if (rc != TDC_OK) return rc;
  if (empty) return TDC_OK;
  // The plain kernel (no TMA, no shared memory, loads through L1): a thread
  // slides 8 output columns of one channel pair down its band of rows.
  // Measured against this call's first kernel (one 8-channel vector of one
  // column per thread, 16-byte loads, 16-row bands) on the same B200, same
  // bits: 64 x 224 x 336 x 256 1240 vs 1766 us, 32 x 224 x 336 x 256 693 vs
  // 880, 16 x 112 x 224 x 128 62.0 vs 86.0, 8 x 56 x 56 x 256 10.3 vs 14.4.
  rc = fwd_plain(x, w, y, N, H, W, C, 3, 1, pad, 0, Epilogue(), stream, kF16);
  if (rc != TDC_ERR_TOO_LARGE) return rc;
  // One image beyond the plain kernel's 32-bit offsets within an image
  // (H * W * C / 2 >= 2^31, 8.6 GB of fp16): the general ring kernel, whose
  // output offsets are 64-bit; the same arithmetic.
  Epilogue epi;
  epi.fused = true;
  return ws_common(x, w, y, N, H, W, C, R, S, pad, 2, nullptr, false, -1, 0, stream, epi);
}

TDC_API int tdc_dwconv_ws(const void* x, const void* w, void* y, int64_t N, int64_t H, int64_t W,
                          int64_t C, int64_t R, int64_t S, int64_t pad, int64_t n_stage,
                          void* stream) {
  return ws_common(x, w, y, N, H, W, C, R, S, pad, n_stage, nullptr, false, -1, 0, stream);
}

TDC_API int tdc_dwconv_ws_host(const void* x_host, const void* w_host, void* y_host,
                               int64_t N, int64_t H, int64_t W, int64_t C, int64_t pad,
                               int64_t n_stage, void* x_dev, void* w_dev, void* y_dev,
                               int64_t chunk_images, void* stream) {
  int64_t P = 0, Q = 0;
  bool empty = false;
  int rc = validate(x_dev, w_dev, y_dev, N, H, W, C, 3, 3, pad, tdc::kBlockC, &P, &Q, &empty);
  if (rc != TDC_OK) return rc;
  if (n_stage < 2 || n_stage > 4) return TDC_ERR_N_STAGE;
  if (chunk_images < 0) return TDC_ERR_BAD_SHAPE;
  if (empty) return TDC_OK;
  if (!x_host || !w_host || !y_host) return TDC_ERR_NULL_POINTER;
  rc = check_ws_limits(N, H, W, C, P, Q);
  if (rc != TDC_OK) return rc;
  DeviceInfo* dev = nullptr;
  int devi = -1;
  rc = current_device(&dev, &devi);
  if (rc != TDC_OK) return rc;
  // Default: N/64 images per chunk (one image at N <= 64: measured on
  // 64 x 224 x 336 x 256, 1 / 2 / 4 / 8 / 16 images per chunk took 52.0 /
  // 52.6 / 54.5 / 56.4 / 60.8 ms; the copies alone 44.4 ms H2D, 43.1 ms D2H).
  const int64_t chunk = chunk_images > 0 ? std::min(chunk_images, N)
                                         : std::max<int64_t>(1, (N + 63) / 64);
  const int64_t chunks = (N + chunk - 1) / chunk;
  const size_t x_img = size_t(H) * W * C * 2, y_img = size_t(P) * Q * C * 2;
  auto* xh = static_cast<const uint8_t*>(x_host);
  auto* xd = static_cast<uint8_t*>(x_dev);
  auto* yh = static_cast<uint8_t*>(y_host);
  auto* yd = static_cast<uint8_t*>(y_dev);
  cudaStream_t caller = static_cast<cudaStream_t>(stream);
  HostPipe& hp = g_pipe[devi];
  std::lock_guard<std::mutex> lock(hp.m);
  cudaError_t e = pipe_ready(hp);
  if (e == cudaSuccess) e = pipe_events(hp.copied, size_t(chunks));
  if (e == cudaSuccess) e = pipe_events(hp.computed, size_t(chunks));
  if (e != cudaSuccess) return cuda_fail(e);
  // Everything starts after the work already queued on the caller's stream.
  e = cudaEventRecord(hp.start, caller);
  for (int i = 0; i < 3 && e == cudaSuccess; ++i) e = cudaStreamWaitEvent(hp.s[i], hp.start, 0);
  if (e == cudaSuccess)
    e = cudaMemcpyAsync(w_dev, w_host, size_t(9) * C * 2, cudaMemcpyHostToDevice, hp.s[0]);
  for (int64_t i = 0; i < chunks && e == cudaSuccess; ++i) {
    const int64_t n0 = i * chunk, n = std::min(chunk, N - n0);
    e = cudaMemcpyAsync(xd + n0 * x_img, xh + n0 * x_img, n * x_img, cudaMemcpyHostToDevice,
                        hp.s[0]);
    if (e == cudaSuccess) e = cudaEventRecord(hp.copied[i], hp.s[0]);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(hp.s[1], hp.copied[i], 0);
    if (e != cudaSuccess) break;
    rc = ws_common(xd + n0 * x_img, w_dev, yd + n0 * y_img, n, H, W, C, 3, 3, pad, n_stage,
                   nullptr, false, -1, 0, hp.s[1]);
    if (rc != TDC_OK) return rc;
    e = cudaEventRecord(hp.computed[i], hp.s[1]);
    if (e == cudaSuccess) e = cudaStreamWaitEvent(hp.s[2], hp.computed[i], 0);
    if (e == cudaSuccess)
      e = cudaMemcpyAsync(yh + n0 * y_img, yd + n0 * y_img, n * y_img, cudaMemcpyDeviceToHost,
                          hp.s[2]);
  }
  // The caller's stream continues once the last result is back on the host
  // (the d2h stream waited for every chunk's kernel, which waited for its copy).
  if (e == cudaSuccess) e = cudaEventRecord(hp.end, hp.s[2]);
  if (e == cudaSuccess) e = cudaStreamWaitEvent(caller, hp.end, 0);
  return e == cudaSuccess ? TDC_OK : cuda_fail(e);
}

TDC_API int tdc_dwconv3x3_fwd(const void* x, const void* w, const void* bias,
                              const void* residual, void* y, int64_t N, int64_t H, int64_t W,
                              int64_t C, int64_t pad, int64_t act, int64_t n_stage, void* stream) {
  if (act < TDC_ACT_NONE || act > TDC_ACT_HARDSWISH) return TDC_ERR_ACT;
  Epilogue epi;
  epi.fused = true;
  epi.bias = bias;
  epi.residual = residual;
  epi.act = int(act);
  return ws_common(x, w, y, N, H, W, C, 3, 3, pad, n_stage, nullptr, false, -1, 0, stream, epi);
}

// Whether the weight gradient with n_stage = 0 runs the plain kernel: narrow
// outputs (Q <= 16, half a ws strip or less) or at most 16 channels.  A plain
// thread walks the whole output width, so wide images with more channels stay
// on the ws kernels.  Measured on the 28 depthwise layers of MobileNetV2 /
// V3-Large / EfficientNet-B0 at batch 64 (us, plain vs ws): 7 x 7 x 960 5x5
// 19.5 vs 159, 14 x 14 x 576 21.9 vs 27.5, 112 x 112 x 16 30.6 vs 48.3;
// 112 x 112 x 32 66.7 vs 49.0, 56 x 56 x 72 47.3 vs 34.5.
bool prefer_plain_wgrad(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K, int64_t S,
                        int64_t pad) {
  if (K != 3 && K != 5 && K != 7) return false;
  if ((S != 1 && S != 2) || C <= 0 || C % 8 != 0 || N <= 0 || pad < 0) return false;
  if (H + 2 * pad < K || W + 2 * pad < K) return false;
  const int64_t Q = (W + 2 * pad - K) / S + 1;
  return Q <= 16 || C <= 16;
}

// Ring depth of the ws weight gradients when the caller leaves it to the
// library (n_stage = 0), measured at 64 x 224 x 336 x 256.
int default_wgrad_stages(int64_t K, int64_t S) {
  static const int kStages[3][2] = {{2, 4}, {4, 4}, {3, 3}};  // [K: 3, 5, 7][stride - 1]
  return (K == 3 || K == 5 || K == 7) && (S == 1 || S == 2) ? kStages[K / 2 - 1][S - 1] : 2;
}

static int fwd_entry(int dt, const void* x, const void* w, const void* bias,
                     const void* residual, void* y, int64_t N, int64_t H, int64_t W, int64_t C,
                     int64_t K, int64_t stride, int64_t pad, int64_t act, int64_t n_stage,
                     void* stream) {
  if (act < TDC_ACT_NONE || act > TDC_ACT_HARDSWISH) return TDC_ERR_ACT;
  if (n_stage == 0) {  // automatic: the kernel and ring depth follow the shape
    if (prefer_plain(N, H, W, C, K, stride, pad)) {
      Epilogue epi;
      epi.fused = true;
      epi.bias = bias;
      epi.residual = residual;
      epi.act = int(act);
      return fwd_plain(x, w, y, N, H, W, C, K, stride, pad, 0, epi, stream, dt);
    }
    n_stage = default_fwd_stages(K, stride);
  }
  if (dt == kF16 && K == 3 && stride == 1)
    return tdc_dwconv3x3_fwd(x, w, bias, residual, y, N, H, W, C, pad, act, n_stage, stream);
  Epilogue epi;
  epi.fused = true;
  epi.bias = bias;
  epi.residual = residual;
  epi.act = int(act);
  return fwd_geom(x, w, y, N, H, W, C, K, stride, pad, n_stage, epi, stream, dt);
}

TDC_API int tdc_dwconv_fwd(const void* x, const void* w, const void* bias, const void* residual,
                           void* y, int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                           int64_t stride, int64_t pad, int64_t act, int64_t n_stage,
                           void* stream) {
  return fwd_entry(kF16, x, w, bias, residual, y, N, H, W, C, K, stride, pad, act, n_stage,
                   stream);
}

TDC_API int tdc_dwconv_fwd_bf16(const void* x, const void* w, const void* bias,
                                const void* residual, void* y, int64_t N, int64_t H, int64_t W,
                                int64_t C, int64_t K, int64_t stride, int64_t pad, int64_t act,
                                int64_t n_stage, void* stream) {
  return fwd_entry(kBF16, x, w, bias, residual, y, N, H, W, C, K, stride, pad, act, n_stage,
                   stream);
}

// Forward with each side's padding given: the top / left sides are the
// kernels' row / column offsets, the bottom / right sides set P and Q.  The
// 3x3 stride-1 fp16 case runs the K x K kernel family (the same arithmetic).
static int fwd_asym_entry(int dt, const void* x, const void* w, const void* bias,
                          const void* residual, void* y, int64_t N, int64_t H, int64_t W,
                          int64_t C, int64_t K, int64_t stride, int64_t pad_top,
                          int64_t pad_bottom, int64_t pad_left, int64_t pad_right, int64_t act,
                          int64_t n_stage, void* stream) {
  if (act < TDC_ACT_NONE || act > TDC_ACT_HARDSWISH) return TDC_ERR_ACT;
  const Pad4 pd{pad_top, pad_bottom, pad_left, pad_right};
  Epilogue epi;
  epi.fused = true;
  epi.bias = bias;
  epi.residual = residual;
  epi.act = int(act);
  if (n_stage == 0) {  // automatic: the kernel and ring depth follow the shape
    if (pad_top >= 0 && pad_bottom >= 0 && pad_left >= 0 && pad_right >= 0 &&
        prefer_plain_pads(N, H, W, C, K, stride, pd))
      return fwd_plain(x, w, y, N, H, W, C, K, stride, pad_top, 0, epi, stream, dt, &pd);
    n_stage = default_fwd_stages(K, stride);
  }
  return fwd_geom(x, w, y, N, H, W, C, K, stride, pad_top, n_stage, epi, stream, dt, &pd);
}

TDC_API int tdc_dwconv_fwd_asym(const void* x, const void* w, const void* bias,
                                const void* residual, void* y, int64_t N, int64_t H, int64_t W,
                                int64_t C, int64_t K, int64_t stride, int64_t pad_top,
                                int64_t pad_bottom, int64_t pad_left, int64_t pad_right,
                                int64_t act, int64_t n_stage, void* stream) {
  return fwd_asym_entry(kF16, x, w, bias, residual, y, N, H, W, C, K, stride, pad_top,
                        pad_bottom, pad_left, pad_right, act, n_stage, stream);
}

TDC_API int tdc_dwconv_fwd_asym_bf16(const void* x, const void* w, const void* bias,
                                     const void* residual, void* y, int64_t N, int64_t H,
                                     int64_t W, int64_t C, int64_t K, int64_t stride,
                                     int64_t pad_top, int64_t pad_bottom, int64_t pad_left,
                                     int64_t pad_right, int64_t act, int64_t n_stage,
                                     void* stream) {
  return fwd_asym_entry(kBF16, x, w, bias, residual, y, N, H, W, C, K, stride, pad_top,
                        pad_bottom, pad_left, pad_right, act, n_stage, stream);
}

static int fwd_dilated_entry(int dt, const void* x, const void* w, const void* bias,
                             const void* residual, void* y, int64_t N, int64_t H, int64_t W,
                             int64_t C, int64_t K, int64_t stride, int64_t dilation,
                             int64_t pad_top, int64_t pad_bottom, int64_t pad_left,
                             int64_t pad_right, int64_t act, int64_t kernel, void* stream) {
  if (act < TDC_ACT_NONE || act > TDC_ACT_HARDSWISH) return TDC_ERR_ACT;
  if (dilation == 1 && kernel == 0)  // the undilated forward, chosen by shape
    return fwd_asym_entry(dt, x, w, bias, residual, y, N, H, W, C, K, stride, pad_top,
                          pad_bottom, pad_left, pad_right, act, 0, stream);
  Epilogue epi;
  epi.fused = true;
  epi.bias = bias;
  epi.residual = residual;
  epi.act = int(act);
  return fwd_dilated(x, w, y, N, H, W, C, K, stride, dilation,
                     Pad4{pad_top, pad_bottom, pad_left, pad_right}, epi, kernel, stream, dt);
}

TDC_API int tdc_dwconv_fwd_dilated(const void* x, const void* w, const void* bias,
                                   const void* residual, void* y, int64_t N, int64_t H,
                                   int64_t W, int64_t C, int64_t K, int64_t stride,
                                   int64_t dilation, int64_t pad_top, int64_t pad_bottom,
                                   int64_t pad_left, int64_t pad_right, int64_t act,
                                   void* stream) {
  return fwd_dilated_entry(kF16, x, w, bias, residual, y, N, H, W, C, K, stride, dilation,
                           pad_top, pad_bottom, pad_left, pad_right, act, 0, stream);
}

TDC_API int tdc_dwconv_fwd_dilated_bf16(const void* x, const void* w, const void* bias,
                                        const void* residual, void* y, int64_t N, int64_t H,
                                        int64_t W, int64_t C, int64_t K, int64_t stride,
                                        int64_t dilation, int64_t pad_top, int64_t pad_bottom,
                                        int64_t pad_left, int64_t pad_right, int64_t act,
                                        void* stream) {
  return fwd_dilated_entry(kBF16, x, w, bias, residual, y, N, H, W, C, K, stride, dilation,
                           pad_top, pad_bottom, pad_left, pad_right, act, 0, stream);
}

TDC_API int tdc_dwconv_fwd_dilated_ex(const void* x, const void* w, const void* bias,
                                      const void* residual, void* y, int64_t N, int64_t H,
                                      int64_t W, int64_t C, int64_t K, int64_t stride,
                                      int64_t dilation, int64_t pad_top, int64_t pad_bottom,
                                      int64_t pad_left, int64_t pad_right, int64_t act,
                                      int64_t kernel, int64_t bf16, void* stream) {
  return fwd_dilated_entry(bf16 ? kBF16 : kF16, x, w, bias, residual, y, N, H, W, C, K, stride,
                           dilation, pad_top, pad_bottom, pad_left, pad_right, act, kernel,
                           stream);
}

TDC_API int tdc_dwconv_fwd_dilated_uses_plain(int64_t N, int64_t H, int64_t W, int64_t C,
                                              int64_t K, int64_t stride, int64_t dilation,
                                              int64_t pad_top, int64_t pad_bottom,
                                              int64_t pad_left, int64_t pad_right) {
  const Pad4 pd{pad_top, pad_bottom, pad_left, pad_right};
  if (dilation == 1) return prefer_plain_pads(N, H, W, C, K, stride, pd) ? 1 : 0;
  if (K != 3 && K != 5 && K != 7) return 0;
  if ((stride != 1 && stride != 2) || dilation < 1 || dilation > (1 << 24) || N <= 0 || C <= 0 ||
      C % 8 != 0)
    return 0;
  const int64_t Ke = dilation * (K - 1) + 1;
  if (H + pad_top + pad_bottom < Ke || W + pad_left + pad_right < Ke) return 0;
  const int64_t P = (H + pad_top + pad_bottom - Ke) / stride + 1;
  const int64_t Q = (W + pad_left + pad_right - Ke) / stride + 1;
  return dilated_prefers_plain(N, H, W, C, K, stride, dilation, P, Q) ? 1 : 0;
}

static int plain_entry(int dt, const void* x, const void* w, const void* bias,
                       const void* residual, void* y, int64_t N, int64_t H, int64_t W, int64_t C,
                       int64_t K, int64_t stride, int64_t pad, int64_t act, int64_t band_rows,
                       void* stream) {
  if (act < TDC_ACT_NONE || act > TDC_ACT_HARDSWISH) return TDC_ERR_ACT;
  Epilogue epi;
  epi.fused = true;
  epi.bias = bias;
  epi.residual = residual;
  epi.act = int(act);
  return fwd_plain(x, w, y, N, H, W, C, K, stride, pad, band_rows, epi, stream, dt);
}

TDC_API int tdc_dwconv_fwd_plain(const void* x, const void* w, const void* bias,
                                 const void* residual, void* y, int64_t N, int64_t H, int64_t W,
                                 int64_t C, int64_t K, int64_t stride, int64_t pad, int64_t act,
                                 int64_t band_rows, void* stream) {
  return plain_entry(kF16, x, w, bias, residual, y, N, H, W, C, K, stride, pad, act, band_rows,
                     stream);
}

TDC_API int tdc_dwconv_fwd_plain_bf16(const void* x, const void* w, const void* bias,
                                      const void* residual, void* y, int64_t N, int64_t H,
                                      int64_t W, int64_t C, int64_t K, int64_t stride,
                                      int64_t pad, int64_t act, int64_t band_rows, void* stream) {
  return plain_entry(kBF16, x, w, bias, residual, y, N, H, W, C, K, stride, pad, act, band_rows,
                     stream);
}

TDC_API int tdc_dwconv_fwd_uses_plain(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                      int64_t stride, int64_t pad) {
  return prefer_plain(N, H, W, C, K, stride, pad) ? 1 : 0;
}

TDC_API int tdc_dwconv_bwd_weight_plain_workspace(int64_t N, int64_t H, int64_t W, int64_t C,
                                                  int64_t K, int64_t stride, int64_t pad,
                                                  int64_t* bytes) {
  return wgrad_plain_workspace(N, H, W, C, K, stride, pad, bytes);
}

TDC_API int tdc_dwconv_bwd_weight_plain(const void* x, const void* dy, float* dw, int64_t N,
                                        int64_t H, int64_t W, int64_t C, int64_t K,
                                        int64_t stride, int64_t pad, void* workspace,
                                        int64_t workspace_bytes, void* stream) {
  return wgrad_plain(kF16, x, dy, dw, N, H, W, C, K, stride, pad, workspace, workspace_bytes,
                     stream);
}

TDC_API int tdc_dwconv_bwd_weight_plain_bf16(const void* x, const void* dy, float* dw, int64_t N,
                                             int64_t H, int64_t W, int64_t C, int64_t K,
                                             int64_t stride, int64_t pad, void* workspace,
                                             int64_t workspace_bytes, void* stream) {
  return wgrad_plain(kBF16, x, dy, dw, N, H, W, C, K, stride, pad, workspace, workspace_bytes,
                     stream);
}

TDC_API int tdc_dwconv_bwd_weight_uses_plain(int64_t N, int64_t H, int64_t W, int64_t C,
                                             int64_t K, int64_t stride, int64_t pad) {
  return prefer_plain_wgrad(N, H, W, C, K, stride, pad) ? 1 : 0;
}

TDC_API int tdc_dwconv3x3_bwd_data(const void* dy, const void* w, void* dx, int64_t N, int64_t H,
                                   int64_t W, int64_t C, int64_t pad, int64_t n_stage,
                                   void* stream) {
  if (pad < 0) return TDC_ERR_PAD;
  if (pad > (1 << 28)) return TDC_ERR_TOO_LARGE;
  // dy is [N, P, Q, C]; it must not be empty in P or Q (dx would be all zero).
  const int64_t P = H + 2 * pad - 2, Q = W + 2 * pad - 2;
  if (H < 1 || W < 1 || P < 1 || Q < 1) return TDC_ERR_BAD_SHAPE;
  Epilogue epi;
  epi.fused = true;
  epi.flip_taps = true;
  // dx[n,h,w,c] = sum_{r,s} dy[n, h+pad-r, w+pad-s, c] * w[r,s,c]
  //            = forward(dy, w[2-r][2-s], pad' = 2 - pad)
  return ws_common(dy, w, dx, N, P, Q, C, 3, 3, 2 - pad, n_stage, nullptr, false, -1, 0, stream,
                   epi);
}

static int bwd_data_entry(int dt, const void* dy, const void* w, void* dx, int64_t N, int64_t H,
                          int64_t W, int64_t C, int64_t K, int64_t stride, int64_t pad,
                          int64_t n_stage, void* stream) {
  if (K != 3 && K != 5 && K != 7) return TDC_ERR_FILTER_SHAPE;
  if (stride != 1 && stride != 2) return TDC_ERR_STRIDE;
  if (n_stage == 0) {  // automatic: the kernel and ring depth follow the shape
    if (stride == 1 && pad >= 0 && pad <= K - 1 && H >= 1 && W >= 1) {
      const int64_t P = H + 2 * pad - K + 1, Q = W + 2 * pad - K + 1;
      if (P >= 1 && Q >= 1 && prefer_plain(N, P, Q, C, K, 1, K - 1 - pad)) {
        Epilogue epi;
        epi.fused = true;
        epi.flip_taps = true;
        return fwd_plain(dy, w, dx, N, P, Q, C, K, 1, K - 1 - pad, 0, epi, stream, dt);
      }
    }
    n_stage = stride == 2 ? 2 : default_fwd_stages(K, 1);
  }
  if (stride == 2) return dgrad_s2(dy, w, dx, N, H, W, C, K, pad, n_stage, stream, dt);
  if (K == 3 && dt == kF16) return tdc_dwconv3x3_bwd_data(dy, w, dx, N, H, W, C, pad, n_stage, stream);
  // pad' = K - 1 - pad must not be negative (pad above K - 1 leaves dx rows
  // no output depends on; supported by the fp16 3x3 path only).
  if (pad < 0 || pad > K - 1) return TDC_ERR_PAD;
  const int64_t P = H + 2 * pad - K + 1, Q = W + 2 * pad - K + 1;
  if (H < 1 || W < 1 || P < 1 || Q < 1) return TDC_ERR_BAD_SHAPE;
  Epilogue epi;
  epi.fused = true;
  epi.flip_taps = true;
  // dx[n,h,w,c] = sum_{r,s} dy[n, h+pad-r, w+pad-s, c] * w[r,s,c]
  //            = forward(dy, w[K-1-r][K-1-s], pad' = K - 1 - pad)
  return fwd_geom(dy, w, dx, N, P, Q, C, K, 1, K - 1 - pad, n_stage, epi, stream, dt);
}

TDC_API int tdc_dwconv_bwd_data(const void* dy, const void* w, void* dx, int64_t N, int64_t H,
                                int64_t W, int64_t C, int64_t K, int64_t stride, int64_t pad,
                                int64_t n_stage, void* stream) {
  return bwd_data_entry(kF16, dy, w, dx, N, H, W, C, K, stride, pad, n_stage, stream);
}

TDC_API int tdc_dwconv_bwd_data_bf16(const void* dy, const void* w, void* dx, int64_t N,
                                     int64_t H, int64_t W, int64_t C, int64_t K, int64_t stride,
                                     int64_t pad, int64_t n_stage, void* stream) {
  return bwd_data_entry(kBF16, dy, w, dx, N, H, W, C, K, stride, pad, n_stage, stream);
}

static int wgrad3x3_workspace(int dt, int64_t N, int64_t H, int64_t W, int64_t C, int64_t pad,
                              int64_t n_stage, int64_t* bytes);
static int wgrad3x3(int dt, const void* x, const void* dy, float* dw, int64_t N, int64_t H,
                    int64_t W, int64_t C, int64_t pad, int64_t n_stage, void* workspace,
                    int64_t workspace_bytes, void* stream);

static int bwd_weight_workspace_entry(int dt, int64_t N, int64_t H, int64_t W, int64_t C,
                                      int64_t K, int64_t stride, int64_t pad, int64_t n_stage,
                                      int64_t* bytes) {
  if (!bytes) return TDC_ERR_NULL_POINTER;
  if (K != 3 && K != 5 && K != 7) return TDC_ERR_FILTER_SHAPE;
  if (stride != 1 && stride != 2) return TDC_ERR_STRIDE;
  if (n_stage == 0) {  // automatic: must agree with bwd_weight_entry
    if (prefer_plain_wgrad(N, H, W, C, K, stride, pad))
      return wgrad_plain_workspace(N, H, W, C, K, stride, pad, bytes);
    n_stage = default_wgrad_stages(K, stride);
  }
  if (K == 3 && stride == 1) return wgrad3x3_workspace(dt, N, H, W, C, pad, n_stage, bytes);
  WsPlan pl;
  int64_t P, Q;
  const int rc = stride == 2 ? wgrad_s2_plan(N, H, W, C, K, pad, n_stage, &pl, &P, &Q, dt)
                             : wgrad_kxk_plan(N, H, W, C, K, pad, n_stage, &pl, &P, &Q, dt);
  if (rc != TDC_OK) return rc;
  *bytes = wgrad_kxk_workspace_bytes(pl, C, K);
  return TDC_OK;
}

static int bwd_weight_entry(int dt, const void* x, const void* dy, float* dw, int64_t N,
                            int64_t H, int64_t W, int64_t C, int64_t K, int64_t stride,
                            int64_t pad, int64_t n_stage, void* workspace, int64_t workspace_bytes,
                            void* stream) {
  if (K != 3 && K != 5 && K != 7) return TDC_ERR_FILTER_SHAPE;
  if (stride != 1 && stride != 2) return TDC_ERR_STRIDE;
  if (n_stage == 0) {  // automatic: the kernel follows the shape
    if (prefer_plain_wgrad(N, H, W, C, K, stride, pad))
      return wgrad_plain(dt, x, dy, dw, N, H, W, C, K, stride, pad, workspace, workspace_bytes,
                         stream);
    n_stage = default_wgrad_stages(K, stride);
  }
  if (stride == 2)
    return wgrad_s2(x, dy, dw, N, H, W, C, K, pad, n_stage, workspace, workspace_bytes, stream,
                    dt);
  if (K == 3)
    return wgrad3x3(dt, x, dy, dw, N, H, W, C, pad, n_stage, workspace, workspace_bytes, stream);
  if (!x || !dy || !dw || !workspace) return TDC_ERR_NULL_POINTER;
  if (!aligned16(x) || !aligned16(dy) || !aligned16(dw) || !aligned16(workspace))
    return TDC_ERR_ALIGNMENT;
  WsPlan pl;
  int64_t P, Q;
  int rc = wgrad_kxk_plan(N, H, W, C, K, pad, n_stage, &pl, &P, &Q, dt);
  if (rc != TDC_OK) return rc;
  if (workspace_bytes < wgrad_kxk_workspace_bytes(pl, C, K)) return TDC_ERR_WORKSPACE;
  alignas(64) CUtensorMap xmap, dymap;
  rc = encode_nhwc_map(&xmap, x, N, H, W, C, tdc::kStripQ + int(K) - 1, pl.stage_rows, dt);
  if (rc != TDC_OK) return rc;
  rc = encode_dy_map(&dymap, dy, N, P, Q, C, pl.stage_rows, dt);
  if (rc != TDC_OK) return rc;
  tdc::WgradParams g{};
  g.status_host = current_status_slot(true);
  g.partial = static_cast<float*>(workspace);
  g.C = int32_t(C); g.P = int32_t(P); g.Q = int32_t(Q); g.pad = int32_t(pad);
  g.qstrips = pl.qstrips; g.cblocks = pl.cblocks; g.stage_rows = pl.stage_rows;
  g.tail_bands = pl.tail_bands; g.tail_band_rows = pl.tail_band_rows;
  g.full_units = pl.full_units; g.tail_strips = pl.tail_strips;
  g.timeout_ns = uint64_t(g_timeout_ns.load());
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  for (int pass = 0; pass < wgrad_kxk_passes(int(K)); ++pass) {
    const cudaError_t e = kWgradKxkLaunch[dt][K == 5 ? 0 : 1][pass][n_stage - 2](
        xmap, dymap, g, pl.grid, pl.smem, st);
    if (e != cudaSuccess) return cuda_fail(e);
  }
  cudaError_t e;
  const int n = int(K * K * C);
  e = tdc::launch_wgrad_reduce(static_cast<const float*>(workspace), dw,
                                int32_t(pl.grid * tdc::kConsumerWarps), n, st);
  return e == cudaSuccess ? TDC_OK : cuda_fail(e);
}

TDC_API int tdc_dwconv_bwd_weight_workspace(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                            int64_t stride, int64_t pad, int64_t n_stage,
                                            int64_t* bytes) {
  return bwd_weight_workspace_entry(kF16, N, H, W, C, K, stride, pad, n_stage, bytes);
}

TDC_API int tdc_dwconv_bwd_weight_workspace_bf16(int64_t N, int64_t H, int64_t W, int64_t C,
                                                 int64_t K, int64_t stride, int64_t pad,
                                                 int64_t n_stage, int64_t* bytes) {
  return bwd_weight_workspace_entry(kBF16, N, H, W, C, K, stride, pad, n_stage, bytes);
}

TDC_API int tdc_dwconv_bwd_weight(const void* x, const void* dy, float* dw, int64_t N, int64_t H,
                                  int64_t W, int64_t C, int64_t K, int64_t stride, int64_t pad,
                                  int64_t n_stage, void* workspace, int64_t workspace_bytes,
                                  void* stream) {
  return bwd_weight_entry(kF16, x, dy, dw, N, H, W, C, K, stride, pad, n_stage, workspace,
                          workspace_bytes, stream);
}

TDC_API int tdc_dwconv_bwd_weight_bf16(const void* x, const void* dy, float* dw, int64_t N,
                                       int64_t H, int64_t W, int64_t C, int64_t K, int64_t stride,
                                       int64_t pad, int64_t n_stage, void* workspace,
                                       int64_t workspace_bytes, void* stream) {
  return bwd_weight_entry(kBF16, x, dy, dw, N, H, W, C, K, stride, pad, n_stage, workspace,
                          workspace_bytes, stream);
}

TDC_API int tdc_dwconv_bwd_weight_plan(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                       int64_t pad, int64_t n_stage, int64_t sms,
                                       int64_t ctas_per_sm, int64_t* plan) {
  if (!plan) return TDC_ERR_NULL_POINTER;
  if (K != 5 && K != 7) return TDC_ERR_FILTER_SHAPE;
  if (N < 1 || H < 1 || W < 1 || C < 8) return TDC_ERR_BAD_SHAPE;
  if (C % 8 != 0) return TDC_ERR_CHANNELS;
  if (pad < 0) return TDC_ERR_PAD;
  if (n_stage < 2 || n_stage > 4) return TDC_ERR_N_STAGE;
  if (sms < 1 || ctas_per_sm < 1) return TDC_ERR_BAD_SHAPE;
  const int64_t P = H + 2 * pad - K + 1, Q = W + 2 * pad - K + 1;
  if (P < 1 || Q < 1) return TDC_ERR_BAD_SHAPE;
  const WsPlan pl = make_wgrad_kxk_plan(N, P, Q, C, int(K), n_stage, sms, ctas_per_sm);
  plan[0] = pl.stage_rows;
  plan[1] = pl.qstrips;
  plan[2] = pl.cblocks;
  plan[3] = pl.strips;
  plan[4] = pl.full_units;
  plan[5] = pl.tail_band_rows;
  plan[6] = pl.grid;
  plan[7] = int64_t(pl.smem);
  plan[8] = wgrad_kxk_passes(int(K));
  plan[9] = wgrad_kxk_max_rows(int(K));
  plan[10] = tdc::wgrad_dy_rows(int(K), 1);
  return TDC_OK;
}

TDC_API int tdc_dwconv_bwd_s2_plan(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                   int64_t pad, int64_t n_stage, int64_t which, int64_t sms,
                                   int64_t ctas_per_sm, int64_t* plan) {
  if (!plan) return TDC_ERR_NULL_POINTER;
  if (which != 0 && which != 1) return TDC_ERR_UNSUPPORTED;
  if (sms < 1 || ctas_per_sm < 1) return TDC_ERR_BAD_SHAPE;
  int64_t P, Q;
  const int rc = bwd_s2_shape(N, H, W, C, K, pad, n_stage, &P, &Q);
  if (rc != TDC_OK) return rc;
  if (N < 1 || C < 8) return TDC_ERR_BAD_SHAPE;
  const WsPlan pl = which == 0 ? make_dgrad_s2_plan(N, H, W, C, int(K), n_stage, sms, ctas_per_sm)
                               : make_wgrad_s2_plan(N, P, Q, C, int(K), n_stage, sms, ctas_per_sm);
  plan[0] = pl.stage_rows;
  plan[1] = pl.qstrips;
  plan[2] = pl.cblocks;
  plan[3] = pl.strips;
  plan[4] = pl.full_units;
  plan[5] = pl.tail_band_rows;
  plan[6] = pl.grid;
  plan[7] = int64_t(pl.smem);
  plan[8] = which == 0 ? tdc::dgrad_s2_pairs(int(K)) : wgrad_s2_passes(int(K));
  plan[9] = which == 0 ? dgrad_s2_window(int(K)) : wgrad_s2_max_rows(int(K));
  plan[10] = which == 0 ? 2 * tdc::dgrad_s2_pairs(int(K)) : tdc::wgrad_dy_rows(int(K), 2);
  return TDC_OK;
}

// Plan of the weight-gradient launch: the forward planner over dy's strips.
int wgrad_plan(int64_t N, int64_t H, int64_t W, int64_t C, int64_t pad, int64_t n_stage,
               WsPlan* pl, int64_t* P, int64_t* Q, int dt = kF16) {
  if (N < 1 || H < 1 || W < 1 || C < 8) return TDC_ERR_BAD_SHAPE;
  if (C % 8 != 0) return TDC_ERR_CHANNELS;
  if (pad < 0) return TDC_ERR_PAD;
  if (pad > (1 << 28)) return TDC_ERR_TOO_LARGE;
  if (n_stage < 2 || n_stage > 4) return TDC_ERR_N_STAGE;
  *P = H + 2 * pad - 2;
  *Q = W + 2 * pad - 2;
  if (*P < 1 || *Q < 1) return TDC_ERR_BAD_SHAPE;
  int rc = check_ws_limits(N, H, W, C, *P, *Q);
  if (rc != TDC_OK) return rc;
  DeviceInfo* dev = nullptr;
  rc = current_device(&dev, nullptr);
  if (rc != TDC_OK) return rc;
  *pl = make_plan(N, *P, *Q, C, n_stage, dev->sms,
                  std::max(1, dev->wgrad_occupancy[dt][n_stage - 2]));
  pl->stage_rows = wgrad_stage_rows(n_stage);
  pl->smem = size_t(n_stage) * pl->stage_rows * (tdc::kRowBytes + tdc::kDyRowBytes) + 128;
  return TDC_OK;
}

int64_t wgrad_workspace_bytes(const WsPlan& pl, int64_t C) {
  return pl.grid * tdc::kConsumerWarps * 9 * C * int64_t(sizeof(float));
}

static int wgrad3x3_workspace(int dt, int64_t N, int64_t H, int64_t W, int64_t C, int64_t pad,
                              int64_t n_stage, int64_t* bytes) {
  if (!bytes) return TDC_ERR_NULL_POINTER;
  WsPlan pl;
  int64_t P, Q;
  const int rc = wgrad_plan(N, H, W, C, pad, n_stage, &pl, &P, &Q, dt);
  if (rc != TDC_OK) return rc;
  *bytes = wgrad_workspace_bytes(pl, C);
  return TDC_OK;
}

extern "C++" template <class E>
cudaError_t launch_wgrad3x3(int64_t n_stage, const CUtensorMap& xmap, const CUtensorMap& dymap,
                            const tdc::WgradParams& g, const WsPlan& pl, cudaStream_t st) {
  const dim3 grid(unsigned(pl.grid)), block(tdc::kWsThreads);
  switch (n_stage) {
    case 2: tdc::dwconv_wgrad_kernel<2, E><<<grid, block, pl.smem, st>>>(xmap, dymap, g); break;
    case 3: tdc::dwconv_wgrad_kernel<3, E><<<grid, block, pl.smem, st>>>(xmap, dymap, g); break;
    default: tdc::dwconv_wgrad_kernel<4, E><<<grid, block, pl.smem, st>>>(xmap, dymap, g); break;
  }
  return cudaGetLastError();
}

static int wgrad3x3(int dt, const void* x, const void* dy, float* dw, int64_t N, int64_t H,
                    int64_t W, int64_t C, int64_t pad, int64_t n_stage, void* workspace,
                    int64_t workspace_bytes, void* stream) {
  if (!x || !dy || !dw || !workspace) return TDC_ERR_NULL_POINTER;
  if (!aligned16(x) || !aligned16(dy) || !aligned16(dw) || !aligned16(workspace))
    return TDC_ERR_ALIGNMENT;
  WsPlan pl;
  int64_t P, Q;
  int rc = wgrad_plan(N, H, W, C, pad, n_stage, &pl, &P, &Q, dt);
  if (rc != TDC_OK) return rc;
  if (workspace_bytes < wgrad_workspace_bytes(pl, C)) return TDC_ERR_WORKSPACE;
  alignas(64) CUtensorMap xmap, dymap;
  rc = encode_nhwc_map(&xmap, x, N, H, W, C, tdc::kInCols, pl.stage_rows, dt);
  if (rc != TDC_OK) return rc;
  rc = encode_dy_map(&dymap, dy, N, P, Q, C, pl.stage_rows, dt);
  if (rc != TDC_OK) return rc;
  tdc::WgradParams g{};
  g.status_host = current_status_slot(true);
  g.partial = static_cast<float*>(workspace);
  g.C = int32_t(C); g.P = int32_t(P); g.Q = int32_t(Q); g.pad = int32_t(pad);
  g.qstrips = pl.qstrips; g.cblocks = pl.cblocks; g.stage_rows = pl.stage_rows;
  g.tail_bands = pl.tail_bands; g.tail_band_rows = pl.tail_band_rows;
  g.full_units = pl.full_units; g.tail_strips = pl.tail_strips;
  g.timeout_ns = uint64_t(g_timeout_ns.load());
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  cudaError_t e = dt == kBF16 ? launch_wgrad3x3<tdc::BF16>(n_stage, xmap, dymap, g, pl, st)
                              : launch_wgrad3x3<tdc::F16>(n_stage, xmap, dymap, g, pl, st);
  if (e != cudaSuccess) return cuda_fail(e);
  const int n = int(9 * C);
  e = tdc::launch_wgrad_reduce(static_cast<const float*>(workspace), dw,
                                int32_t(pl.grid * tdc::kConsumerWarps), n, st);
  return e == cudaSuccess ? TDC_OK : cuda_fail(e);
}

TDC_API int tdc_dwconv3x3_bwd_weight_workspace(int64_t N, int64_t H, int64_t W, int64_t C,
                                               int64_t pad, int64_t n_stage, int64_t* bytes) {
  return wgrad3x3_workspace(kF16, N, H, W, C, pad, n_stage, bytes);
}

TDC_API int tdc_dwconv3x3_bwd_weight(const void* x, const void* dy, float* dw, int64_t N,
                                     int64_t H, int64_t W, int64_t C, int64_t pad,
                                     int64_t n_stage, void* workspace, int64_t workspace_bytes,
                                     void* stream) {
  return wgrad3x3(kF16, x, dy, dw, N, H, W, C, pad, n_stage, workspace, workspace_bytes, stream);
}

// ---------------------------------------------------------------------------
// Weight gradient without allocation.
//
// Some callers cannot allocate device memory at the time they need the
// weight gradient: runtimes that reserve a fixed device budget at start-up
// and forbid later allocation, plug-ins whose host framework owns all device
// memory without exposing its allocator, and latency-critical paths where
// cudaMalloc may synchronise the device or fail at an arbitrary moment.  For
// them the workspace of tdc_dwconv3x3_bwd_weight lives in a file-scope
// device array instead.  The array's name is only a host-side stand-in in
// host code; its device address is looked up once per device with
// cudaGetSymbolAddress and passed to the kernels.
// ---------------------------------------------------------------------------
constexpr int64_t kNoAllocScratchBytes = int64_t(16) << 20;  // per device, held until exit
static __device__ __align__(256) float g_tdc_noalloc_scratch[kNoAllocScratchBytes / sizeof(float)];

// The scratch's device address per device, looked up on the first call that
// succeeds in doing so (a failed lookup is not cached: the next call tries
// again).
struct NoAllocScratch {
  std::mutex m;
  std::atomic<float*> ptr{nullptr};
};
NoAllocScratch g_noalloc[kMaxDevices];

TDC_API int tdc_dwconv3x3_bwd_weight_noalloc(const void* x, const void* dy, float* dw, int64_t N,
                                             int64_t H, int64_t W, int64_t C, int64_t pad,
                                             int64_t n_stage, void* stream) {
  if (!x || !dy || !dw) return TDC_ERR_NULL_POINTER;
  if (!aligned16(x) || !aligned16(dy) || !aligned16(dw)) return TDC_ERR_ALIGNMENT;
  WsPlan pl;
  int64_t P, Q;
  int rc = wgrad_plan(N, H, W, C, pad, n_stage, &pl, &P, &Q);  // also makes the device current
  if (rc != TDC_OK) return rc;
  // Each CTA needs 4 warps x 9 taps x C floats of the scratch: fewer CTAs
  // than the occupancy allows when C is large; none at all beyond the limit.
  const int64_t per_cta = tdc::kConsumerWarps * 9 * C * int64_t(sizeof(float));
  const int64_t max_grid = kNoAllocScratchBytes / per_cta;
  if (max_grid < 1) return TDC_ERR_SCRATCH_LIMIT;
  if (pl.grid > max_grid) {
    const int stage_rows = pl.stage_rows;
    const size_t smem = pl.smem;
    pl = make_plan(N, P, Q, C, n_stage, max_grid, 1);
    pl.stage_rows = stage_rows;
    pl.smem = smem;
  }
  int dev = -1;
  cudaError_t e = cudaGetDevice(&dev);
  if (e != cudaSuccess) return cuda_fail(e);
  NoAllocScratch& sc = g_noalloc[dev];
  float* scratch = sc.ptr.load(std::memory_order_acquire);
  if (scratch == nullptr) {
    std::lock_guard<std::mutex> lock(sc.m);
    scratch = sc.ptr.load(std::memory_order_acquire);
    if (scratch == nullptr) {
      void* p = nullptr;
      const cudaError_t err = cudaGetSymbolAddress(&p, g_tdc_noalloc_scratch);
      if (err != cudaSuccess || p == nullptr) {
        t_last_cuda_error = int(err);
        return TDC_ERR_CUDA;
      }
      scratch = static_cast<float*>(p);
      sc.ptr.store(scratch, std::memory_order_release);
    }
  }

  alignas(64) CUtensorMap xmap, dymap;
  rc = encode_x_map(&xmap, x, N, H, W, C, pl.stage_rows);
  if (rc != TDC_OK) return rc;
  rc = encode_dy_map(&dymap, dy, N, P, Q, C, pl.stage_rows);
  if (rc != TDC_OK) return rc;
  tdc::WgradParams g{};
  g.status_host = current_status_slot(false);  // never allocates the page
  g.partial = scratch;  // every CTA zeroes its own part before accumulating
  g.C = int32_t(C); g.P = int32_t(P); g.Q = int32_t(Q); g.pad = int32_t(pad);
  g.qstrips = pl.qstrips; g.cblocks = pl.cblocks; g.stage_rows = pl.stage_rows;
  g.tail_bands = pl.tail_bands; g.tail_band_rows = pl.tail_band_rows;
  g.full_units = pl.full_units; g.tail_strips = pl.tail_strips;
  g.timeout_ns = uint64_t(g_timeout_ns.load());
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const dim3 grid(unsigned(pl.grid)), block(tdc::kWsThreads);
  switch (n_stage) {
    case 2: tdc::dwconv_wgrad_kernel<2><<<grid, block, pl.smem, st>>>(xmap, dymap, g); break;
    case 3: tdc::dwconv_wgrad_kernel<3><<<grid, block, pl.smem, st>>>(xmap, dymap, g); break;
    default: tdc::dwconv_wgrad_kernel<4><<<grid, block, pl.smem, st>>>(xmap, dymap, g); break;
  }
  e = cudaGetLastError();
  if (e != cudaSuccess) return cuda_fail(e);
  const int n = int(9 * C);
  e = tdc::launch_wgrad_reduce(scratch, dw, int32_t(pl.grid * tdc::kConsumerWarps), n, st);
  return e == cudaSuccess ? TDC_OK : cuda_fail(e);
}

TDC_API int tdc_ws_probe_blocks(int64_t N, int64_t H, int64_t W, int64_t C, int64_t pad,
                                int64_t n_stage, int64_t* num_blocks) {
  if (!num_blocks) return TDC_ERR_NULL_POINTER;
  if (N < 0 || H < 1 || W < 1 || C < 0) return TDC_ERR_BAD_SHAPE;
  if (C % tdc::kBlockC != 0) return TDC_ERR_CHANNELS;
  if (pad < 0) return TDC_ERR_PAD;
  if (n_stage < 2 || n_stage > 4) return TDC_ERR_N_STAGE;
  const int64_t P = H + 2 * pad - 2, Q = W + 2 * pad - 2;
  if (P < 0 || Q < 0) return TDC_ERR_BAD_SHAPE;
  if (N == 0 || C == 0 || P == 0 || Q == 0) {
    *num_blocks = 0;
    return TDC_OK;
  }
  DeviceInfo* dev = nullptr;
  int rc = current_device(&dev, nullptr);
  if (rc != TDC_OK) return rc;
  const int occ = std::max(1, dev->ws_occupancy[n_stage - 2][1]);
  *num_blocks = make_plan(N, P, Q, C, n_stage, dev->sms, occ).grid;
  return TDC_OK;
}

TDC_API int tdc_ws_consumer_warps(void) { return tdc::kConsumerWarps; }

TDC_API int tdc_ws_occupancy(int64_t n_stage, int64_t kind, int64_t* ctas_per_sm, int64_t* sms) {
  if (!ctas_per_sm || !sms) return TDC_ERR_NULL_POINTER;
  if (n_stage < 2 || n_stage > 4) return TDC_ERR_N_STAGE;
  if (kind < 0 || kind > 3) return TDC_ERR_BAD_SHAPE;
  DeviceInfo* dev = nullptr;
  const int rc = current_device(&dev, nullptr);
  if (rc != TDC_OK) return rc;
  *ctas_per_sm = dev->ws_occupancy[n_stage - 2][kind];
  *sms = dev->sms;
  return TDC_OK;
}

TDC_API int tdc_dwconv_ws_probe(const void* x, const void* w, void* y, int64_t N, int64_t H,
                                int64_t W, int64_t C, int64_t R, int64_t S, int64_t pad,
                                int64_t n_stage, unsigned long long* stall, void* stream) {
  return ws_common(x, w, y, N, H, W, C, R, S, pad, n_stage, stall, true, -1, 0, stream);
}

TDC_API int tdc_set_wait_timeout_ns(int64_t ns) {
  if (ns <= 0) return TDC_ERR_BAD_SHAPE;
  g_timeout_ns.store(ns);
  return TDC_OK;
}

TDC_API int tdc_device_status(int clear, int64_t* info) {
  DeviceInfo* dev = nullptr;
  int devi = -1;
  int rc = current_device(&dev, &devi, false);
  if (rc != TDC_OK) return rc;
  cudaError_t e = cudaDeviceSynchronize();
  if (e != cudaSuccess) return cuda_fail(e);
  int h[4] = {0, 0, 0, 0};
  e = cudaMemcpyFromSymbol(h, tdc::g_tdc_status, sizeof(h));
  if (e != cudaSuccess) return cuda_fail(e);
  if (clear) {
    const int z[4] = {0, 0, 0, 0};
    e = cudaMemcpyToSymbol(tdc::g_tdc_status, z, sizeof(z));
    if (e != cudaSuccess) return cuda_fail(e);
    volatile int* slot = status_slot(devi, false);
    if (slot != nullptr)
      for (int i = 0; i < 4; ++i) slot[i] = 0;
  }
  if (info)
    for (int i = 0; i < 4; ++i) info[i] = h[i];
  return h[0] == 0 ? TDC_OK : TDC_ERR_DEVICE_TIMEOUT;
}

TDC_API int tdc_dwconv_ws_withhold(const void* x, const void* w, void* y, int64_t N, int64_t H,
                                   int64_t W, int64_t C, int64_t pad, int64_t n_stage,
                                   int64_t withhold_load, int64_t timeout_ns, void* stream) {
  if (timeout_ns <= 0) return TDC_ERR_BAD_SHAPE;
  return ws_common(x, w, y, N, H, W, C, 3, 3, pad, n_stage, nullptr, false, withhold_load,
                   timeout_ns, stream);
}

TDC_API int tdc_ws_plan(int64_t N, int64_t H, int64_t W, int64_t C, int64_t pad, int64_t n_stage,
                        int64_t sms, int64_t ctas_per_sm, int64_t* plan) {
  if (!plan) return TDC_ERR_NULL_POINTER;
  if (N < 1 || H < 1 || W < 1 || C < 8) return TDC_ERR_BAD_SHAPE;
  if (C % 8 != 0) return TDC_ERR_CHANNELS;
  if (pad < 0) return TDC_ERR_PAD;
  if (n_stage < 2 || n_stage > 4) return TDC_ERR_N_STAGE;
  if (sms < 1 || ctas_per_sm < 1) return TDC_ERR_BAD_SHAPE;
  const int64_t P = H + 2 * pad - 2, Q = W + 2 * pad - 2;
  if (P < 1 || Q < 1) return TDC_ERR_BAD_SHAPE;
  const WsPlan pl = make_plan(N, P, Q, C, n_stage, sms, ctas_per_sm, true);
  plan[0] = pl.stage_rows;
  plan[1] = pl.qstrips;
  plan[2] = pl.cblocks;
  plan[3] = pl.strips;
  plan[4] = pl.full_units;
  plan[5] = pl.tail_band_rows;
  plan[6] = pl.grid;
  plan[7] = int64_t(pl.smem);
  plan[8] = pl.tail_chunk_rows;
  return TDC_OK;
}

TDC_API int tdc_dwconv_fwd_plan(int64_t N, int64_t H, int64_t W, int64_t C, int64_t K,
                                int64_t stride, int64_t pad, int64_t n_stage, int64_t sms,
                                int64_t ctas_per_sm, int64_t* plan) {
  if (!plan) return TDC_ERR_NULL_POINTER;
  if (K != 3 && K != 5 && K != 7) return TDC_ERR_FILTER_SHAPE;
  if (stride != 1 && stride != 2) return TDC_ERR_STRIDE;
  if (N < 1 || H < 1 || W < 1 || C < 8) return TDC_ERR_BAD_SHAPE;
  if (C % 8 != 0) return TDC_ERR_CHANNELS;
  if (pad < 0) return TDC_ERR_PAD;
  if (n_stage < 2 || n_stage > 4) return TDC_ERR_N_STAGE;
  if (sms < 1 || ctas_per_sm < 1) return TDC_ERR_BAD_SHAPE;
  if (H + 2 * pad < K || W + 2 * pad < K) return TDC_ERR_BAD_SHAPE;
  const int64_t P = (H + 2 * pad - K) / stride + 1, Q = (W + 2 * pad - K) / stride + 1;
  const WsPlan pl = (K == 3 && stride == 1)
                        ? make_plan(N, P, Q, C, n_stage, sms, ctas_per_sm, true)
                        : make_geom_plan(N, P, Q, C, int(K), int(stride), n_stage, sms, ctas_per_sm);
  plan[0] = pl.stage_rows;
  plan[1] = pl.qstrips;
  plan[2] = pl.cblocks;
  plan[3] = pl.strips;
  plan[4] = pl.full_units;
  plan[5] = pl.tail_band_rows;
  plan[6] = pl.grid;
  plan[7] = int64_t(pl.smem);
  plan[8] = pl.tail_chunk_rows;
  return TDC_OK;
}

}  // extern "C"
