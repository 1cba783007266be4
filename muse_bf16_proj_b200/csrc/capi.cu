// C ABI of libmuse_proj.so: argument checks, plans, TMA descriptors and kernel launches.
// The kernels live in the .cuh headers included below; this is the only translation unit with device
// code, so the device error word in ptx.cuh has one definition.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <atomic>
#include <mutex>

#include "../../include/muse_proj.h"
#include "errors.h"
#include "gemv.cuh"
#include "tc_tile.cuh"
#include "tc_streamk.cuh"
#include "tc_gemm.cuh"
#include "tc_gemm2.cuh"
#include "tc12.cuh"
#include "tc_skinny.cuh"
#include "router.cuh"
#include "gemv12t.cuh"
#include "enc12.cuh"
#include "stream_read.cuh"
#include "tc_rows.cuh"
#include "tc_wide.cuh"
#include "tc_pairk.cuh"
#include "tc_pairsk.cuh"
#include "gemv_tiles.cuh"

#define MUSE_VERSION_STRING "muse_proj_b200 0.1 (sm_100a)"

namespace {

using muse::fail;

constexpr int kMaxDevices = 16;
constexpr int kSmemLimit = 227 * 1024;

struct DeviceInfo {
  bool ready = false;
  int sms = 0;
  int smem_optin = 0;
};
DeviceInfo g_dev[kMaxDevices];
std::mutex g_mu;

int current_device(int* dev) {
  cudaError_t e = cudaGetDevice(dev);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaGetDevice: %s", cudaGetErrorString(e));
  if (*dev < 0 || *dev >= kMaxDevices) return fail(MUSE_ERR_CUDA, "device index %d out of range", *dev);
  return MUSE_OK;
}

int device_info(DeviceInfo** out) {
  int dev;
  if (int rc = current_device(&dev)) return rc;
  std::lock_guard<std::mutex> lock(g_mu);
  DeviceInfo& d = g_dev[dev];
  if (!d.ready) {
    cudaError_t e = cudaDeviceGetAttribute(&d.sms, cudaDevAttrMultiProcessorCount, dev);
    if (e == cudaSuccess) e = cudaDeviceGetAttribute(&d.smem_optin, cudaDevAttrMaxSharedMemoryPerBlockOptin, dev);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaDeviceGetAttribute: %s", cudaGetErrorString(e));
    int major = 0;
    cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, dev);
    if (major != 10) return fail(MUSE_ERR_CUDA, "device %d is sm_%d0, this library is built for sm_100a", dev, major);
    d.ready = true;
  }
  *out = &d;
  return MUSE_OK;
}

// cuTensorMapEncodeTiled through the runtime's driver entry point (no link against libcuda).
PFN_cuTensorMapEncodeTiled_v12000 encode_fn() {
  static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* p = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(p);
  });
  return fn;
}

// 2-D BF16 tensor map over a row-major [rows, cols] matrix; box = 64 columns x box_rows rows,
// 128-byte swizzle; rows and columns past the edge read as zero.
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows,
             CUtensorMapSwizzle swizzle = CU_TENSOR_MAP_SWIZZLE_128B) {
  auto fn = encode_fn();
  if (!fn) return fail(MUSE_ERR_CUDA, "cuTensorMapEncodeTiled entry point not found");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 2)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, swizzle, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MUSE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return MUSE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

// Optional per-CTA trace buffer for the next launches (muse_set_trace); off when null.
std::atomic<muse::TraceRec*> g_trace{nullptr};
std::atomic<int> g_trace_cap{0};

int launch_error(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return MUSE_OK;
}

// ---- GEMV ------------------------------------------------------------------------------------

template <bool kTwelve, int M, int NW>
int launch_gemv_t(const muse::GemvArgs& a, int grid, int smem, bool pdl, cudaStream_t st) {
  auto kern = muse::gemv_stream_kernel<kTwelve, M, NW>;
  static bool configured[kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(gemv): %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(32 * (NW + 1), 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "gemv launch: %s", cudaGetErrorString(e));
  return MUSE_OK;
}

template <bool kTwelve, int M>
int launch_gemv_m(const muse::GemvArgs& a, int warps, int grid, int smem, bool pdl, cudaStream_t st) {
  switch (warps) {
    case 4: return launch_gemv_t<kTwelve, M, 4>(a, grid, smem, pdl, st);
    case 8: return launch_gemv_t<kTwelve, M, 8>(a, grid, smem, pdl, st);
    case 16: return launch_gemv_t<kTwelve, M, 16>(a, grid, smem, pdl, st);
    default: return fail(MUSE_ERR_PLAN, "gemv: warps must be 4, 8 or 16 (got %d)", warps);
  }
}

template <bool kTwelve>
int launch_gemv(const muse::GemvArgs& a, int m, int warps, int grid, int smem, bool pdl, cudaStream_t st) {
  switch (m) {
    case 1: return launch_gemv_m<kTwelve, 1>(a, warps, grid, smem, pdl, st);
    case 2: return launch_gemv_m<kTwelve, 2>(a, warps, grid, smem, pdl, st);
    case 3: return launch_gemv_m<kTwelve, 3>(a, warps, grid, smem, pdl, st);
    case 4: return launch_gemv_m<kTwelve, 4>(a, warps, grid, smem, pdl, st);
    case 5: return launch_gemv_m<kTwelve, 5>(a, warps, grid, smem, pdl, st);
    case 6: return launch_gemv_m<kTwelve, 6>(a, warps, grid, smem, pdl, st);
    case 7: return launch_gemv_m<kTwelve, 7>(a, warps, grid, smem, pdl, st);
    case 8: return launch_gemv_m<kTwelve, 8>(a, warps, grid, smem, pdl, st);
    default: return fail(MUSE_ERR_SHAPE, "gemv: M must be 1..8 (got %d)", m);
  }
}

// Shapes the grid and shared memory of a GEMV launch from the plan; fills a.rows_per_cta,
// a.chunk_units, a.stages.
int plan_gemv(bool twelve, int64_t m, int64_t n, int64_t k, const MusePlan& p, muse::GemvArgs& a, int* grid,
              int* smem, int* warps) {
  DeviceInfo* d;
  if (int rc = device_info(&d)) return rc;
  const int unit_elems = twelve ? 512 : 256, unit_bytes = twelve ? 768 : 512;
  if (m < 1 || m > 8) return fail(MUSE_ERR_SHAPE, "gemv: M must be 1..8 (got %lld)", (long long)m);
  if (k % unit_elems) return fail(MUSE_ERR_SHAPE, "gemv: K must be a multiple of %d (got %lld)", unit_elems, (long long)k);
  if (n > (int64_t(1) << 30) || k > (int64_t(1) << 20)) return fail(MUSE_ERR_SHAPE, "gemv: shape too large");
  *warps = p.warps ? p.warps : 8;
  const int segs = static_cast<int>(k / unit_elems);
  int ctas = p.ctas > 0 ? p.ctas : d->sms;
  ctas = static_cast<int>(std::min<int64_t>(ctas, n));
  const int chunk = p.chunk > 0 ? p.chunk : std::max(1, (16 * 1024) / unit_bytes);
  const int chunk_bytes = chunk * unit_bytes;
  if (chunk_bytes > 64 * 1024) return fail(MUSE_ERR_PLAN, "gemv: chunk of %d bytes exceeds 64 KB", chunk_bytes);
  const int limit = std::min(kSmemLimit, d->smem_optin);
  // More CTAs (fewer rows each) until the per-row partials and two ring stages fit.
  for (;;) {
    const int64_t rows = (n + ctas - 1) / ctas;
    const int64_t red = rows * segs * m * 4;
    const int64_t fixed = red + 16;
    const int64_t per_stage = chunk_bytes + 16;
    const int64_t fit = (limit - fixed) / per_stage;
    if (fit >= 2) {
      int stages = p.stages > 0 ? p.stages : 8;
      stages = static_cast<int>(std::min<int64_t>(stages, fit));
      if (p.stages > 0 && stages < p.stages)
        return fail(MUSE_ERR_PLAN, "gemv: %d stages do not fit shared memory (max %lld)", p.stages, (long long)fit);
      a.rows_per_cta = static_cast<int>(rows);
      a.chunk_units = chunk;
      a.stages = stages;
      a.trace = g_trace.load();
      a.trace_cap = a.trace ? g_trace_cap.load() : 0;
      *grid = static_cast<int>((n + rows - 1) / rows);
      *smem = static_cast<int>(stages * chunk_bytes + 16 * stages + red);
      return MUSE_OK;
    }
    if (ctas >= n) return fail(MUSE_ERR_SHAPE, "gemv: partial sums do not fit shared memory");
    ctas = static_cast<int>(std::min<int64_t>(n, ctas * 2));
  }
}

// ---- tcgen05 tile kernel ---------------------------------------------------------------------

constexpr int64_t kCounterBytes = 64 * 1024;  // per-tile split-K counters at the front of scratch
constexpr int64_t kMaxCounters = kCounterBytes / 4;

struct TcShape {
  int bnt, split, stages, mode;
  int64_t tiles;          // output tiles (row tiles x token tiles)
  int64_t partial_bytes;  // global split: tiles * split * bnt * 128 * 4
};

int tc_shape(int64_t m, int64_t n, int64_t k, const MusePlan& p, TcShape* out) {
  DeviceInfo* d;
  if (int rc = device_info(&d)) return rc;
  int bnt = p.tile_n;
  if (bnt == 0) {
    bnt = 16;
    while (bnt < m && bnt < 256) bnt *= 2;
  }
  if (bnt != 16 && bnt != 32 && bnt != 64 && bnt != 128 && bnt != 256)
    return fail(MUSE_ERR_PLAN, "tc_tile: tile_n must be 16, 32, 64, 128 or 256 (got %d)", bnt);
  const int nkb = static_cast<int>((k + muse::kTcBK - 1) / muse::kTcBK);
  const int split = p.split > 0 ? p.split : 1;
  const bool global = (p.flags & MUSE_FLAG_GLOBAL_SPLIT) != 0;
  if (split > (global ? 64 : 16) || split > nkb)
    return fail(MUSE_ERR_PLAN, "tc_tile: split %d must be <= %d and <= K / 64 = %d", split, global ? 64 : 16, nkb);
  if (m > (int64_t(1) << 24) || n > (int64_t(1) << 24) || k > (int64_t(1) << 24))
    return fail(MUSE_ERR_SHAPE, "tc_tile: dimension too large");
  const int limit = std::min(kSmemLimit, d->smem_optin);
  const int per_stage = muse::kTcABytes + muse::tc_tile_bbytes(bnt);
  const int max_stages = (limit - 1024 - 64) / (per_stage + 16);
  const int stages = p.stages > 0 ? p.stages : max_stages;
  if (stages > max_stages || stages < 2)
    return fail(MUSE_ERR_PLAN, "tc_tile: %d stages do not fit (max %d)", stages, max_stages);
  if (split > 1 && !global && bnt * 128 * 4 > stages * per_stage)
    return fail(MUSE_ERR_PLAN, "tc_tile: ring of %d stages too small for the split-K partial", stages);
  out->bnt = bnt;
  out->split = split;
  out->stages = stages;
  out->mode = global && split > 1 ? muse::kTcModeGlobalSplit : 0;
  out->tiles = ((n + 127) / 128) * ((m + bnt - 1) / bnt);
  out->partial_bytes = (out->mode & muse::kTcModeGlobalSplit) ? out->tiles * split * bnt * 128 * 4 : 0;
  if ((out->mode & muse::kTcModeGlobalSplit) && out->tiles > kMaxCounters)
    return fail(MUSE_ERR_SHAPE, "tc_tile: %lld output tiles exceed the %lld split-K counters", (long long)out->tiles,
                (long long)kMaxCounters);
  return MUSE_OK;
}

int64_t tc_scratch_bytes(const TcShape& s) { return s.partial_bytes ? kCounterBytes + s.partial_bytes : 0; }

template <int BNT, bool kGather = false>
int launch_tc_t(const CUtensorMap& tmw, const CUtensorMap& tmx, const muse::TcArgs& a, int m, int n, bool pdl,
                cudaStream_t st) {
  auto kern = muse::tc_tile_kernel<BNT, kGather>;
  const int smem = muse::tc_tile_smem(BNT, a.stages);
  static bool configured[kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  cudaError_t e = cudaSuccess;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e == cudaSuccess) e = cudaFuncSetAttribute(kern, cudaFuncAttributeNonPortableClusterSizeAllowed, 1);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(tc_tile): %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  const bool cluster = a.split > 1 && !(a.mode & muse::kTcModeGlobalSplit);
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(((n + 127) / 128) * a.split), static_cast<unsigned>((m + BNT - 1) / BNT), 1);
  cfg.blockDim = dim3(muse::kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(cluster ? a.split : 1);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cluster) {
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess || clusters < 1)
      return fail(MUSE_ERR_PLAN, "tc_tile: clusters of %d CTAs with %d B shared memory cannot be scheduled (%s)",
                  a.split, smem, e == cudaSuccess ? "occupancy 0" : cudaGetErrorString(e));
  }
  e = cudaLaunchKernelEx(&cfg, kern, tmw, tmx, a);
  if (e != cudaSuccess)
    return fail(MUSE_ERR_CUDA, "tc_tile launch (split %d, tile %d): %s", a.split, BNT, cudaGetErrorString(e));
  return MUSE_OK;
}

// W is row-major (tiles == nullptr) or packed tiles (w == nullptr).
// y32 != nullptr: FP32 output; kx > 0: x has kx columns and W (tiles) 2 * kx (the router's hi | lo).
int run_tc_tile(const void* x, const void* w, const void* tiles, void* y, int64_t m, int64_t n, int64_t k,
                const MusePlan& p, void* scratch, int64_t scratch_bytes, cudaStream_t st, float* y32 = nullptr,
                int64_t kx = 0, const muse::GatherOut* g = nullptr) {
  TcShape sh;
  if (int rc = tc_shape(m, n, k, p, &sh)) return rc;
  const int64_t need = tc_scratch_bytes(sh);
  if (need > 0 && (!scratch || scratch_bytes < need))
    return fail(MUSE_ERR_CAPACITY, "tc_tile: global split-K needs %lld bytes of zeroed scratch (got %lld)",
                (long long)need, (long long)(scratch ? scratch_bytes : 0));
  if (need > 0 && (reinterpret_cast<uintptr_t>(scratch) & 255u))
    return fail(MUSE_ERR_ALIGN, "tc_tile: scratch must be 256-byte aligned");
  CUtensorMap tmw, tmx;
  std::memset(&tmw, 0, sizeof(tmw));
  if (!tiles) {
    if (int rc = make_map(&tmw, w, n, k, 128)) return rc;
  }
  if (int rc = make_map(&tmx, x, m, kx > 0 ? kx : k, sh.bnt)) return rc;
  muse::TcArgs a;
  a.wtiles = static_cast<const uint8_t*>(tiles);
  a.y = static_cast<uint16_t*>(y);
  a.y32 = y32;
  a.kxb = kx > 0 ? static_cast<int>(kx / muse::kTcBK) : 0;
  a.counters = need > 0 ? static_cast<int*>(scratch) : nullptr;
  a.partials = need > 0 ? reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + kCounterBytes) : nullptr;
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.K = static_cast<int>(k);
  a.split = sh.split;
  a.stages = sh.stages;
  a.mode = sh.mode | (tiles ? muse::kTcModeTiles : 0);
  a.trace = g_trace.load();
  a.trace_cap = a.trace ? g_trace_cap.load() : 0;
  std::memset(&a.g, 0, sizeof(a.g));
  if (g) a.g = *g;
  const int mi = static_cast<int>(m), ni = static_cast<int>(n);
  // Programmatic launch only for grids without clusters.
  const bool pdl = (p.flags & MUSE_FLAG_PDL) != 0 && !(sh.split > 1 && !(sh.mode & muse::kTcModeGlobalSplit));
  if (g) {
    switch (sh.bnt) {
      case 16: return launch_tc_t<16, true>(tmw, tmx, a, mi, ni, pdl, st);
      case 32: return launch_tc_t<32, true>(tmw, tmx, a, mi, ni, pdl, st);
      case 64: return launch_tc_t<64, true>(tmw, tmx, a, mi, ni, pdl, st);
      case 128: return launch_tc_t<128, true>(tmw, tmx, a, mi, ni, pdl, st);
      default: return launch_tc_t<256, true>(tmw, tmx, a, mi, ni, pdl, st);
    }
  }
  switch (sh.bnt) {
    case 16: return launch_tc_t<16>(tmw, tmx, a, mi, ni, pdl, st);
    case 32: return launch_tc_t<32>(tmw, tmx, a, mi, ni, pdl, st);
    case 64: return launch_tc_t<64>(tmw, tmx, a, mi, ni, pdl, st);
    case 128: return launch_tc_t<128>(tmw, tmx, a, mi, ni, pdl, st);
    default: return launch_tc_t<256>(tmw, tmx, a, mi, ni, pdl, st);
  }
}

// ---- stream-K tcgen05 kernel -----------------------------------------------------------------

struct SkShape {
  int bnt, stages, g, smax;
  int rtiles, nkb, ttiles;
  long long units, tiles;
  int64_t scratch;
};

int sk_shape(int64_t m, int64_t n, int64_t k, const MusePlan& p, SkShape* out) {
  DeviceInfo* d;
  int sms = 148, limit = kSmemLimit;
  if (device_info(&d) == MUSE_OK) {
    sms = d->sms;
    limit = std::min(kSmemLimit, d->smem_optin);
  }
  muse::clear_error();
  int bnt = p.tile_n;
  if (bnt == 0) {
    bnt = 16;
    while (bnt < m && bnt < 128) bnt *= 2;
  }
  if (bnt != 16 && bnt != 32 && bnt != 64 && bnt != 128 && bnt != 256)
    return fail(MUSE_ERR_PLAN, "tc_streamk: tile_n must be 16, 32, 64, 128 or 256 (got %d)", bnt);
  if (m > (int64_t(1) << 24) || n > (int64_t(1) << 24) || k > (int64_t(1) << 24))
    return fail(MUSE_ERR_SHAPE, "tc_streamk: dimension too large");
  const int per_stage = 16384 + muse::sk_bbytes(bnt);
  const int max_stages = (limit - 1024 - 96) / (per_stage + 16);
  const int stages = p.stages > 0 ? p.stages : std::min(6, max_stages);
  if (stages < 2 || stages > max_stages)
    return fail(MUSE_ERR_PLAN, "tc_streamk: %d stages do not fit (max %d)", stages, max_stages);
  SkShape sh;
  sh.bnt = bnt;
  sh.stages = stages;
  sh.rtiles = static_cast<int>((n + 127) / 128);
  sh.nkb = static_cast<int>((k + 63) / 64);
  sh.ttiles = static_cast<int>((m + bnt - 1) / bnt);
  sh.tiles = static_cast<long long>(sh.rtiles) * sh.ttiles;
  sh.units = sh.tiles * sh.nkb;
  if (sh.tiles > kMaxCounters)
    return fail(MUSE_ERR_SHAPE, "tc_streamk: %lld output tiles exceed the %lld counters", sh.tiles, (long long)kMaxCounters);
  long long g = p.ctas > 0 ? p.ctas : sms;
  g = std::min<long long>(g, sh.units);
  sh.g = static_cast<int>(g);
  int smax = 1;
  for (long long t = 0; t < sh.tiles; ++t) {
    const int a0 = muse::sk_owner(t * sh.nkb, sh.units, sh.g);
    const int a1 = muse::sk_owner((t + 1) * sh.nkb - 1, sh.units, sh.g);
    smax = std::max(smax, a1 - a0 + 1);
  }
  sh.smax = smax;
  sh.scratch = kCounterBytes + static_cast<int64_t>(sh.tiles) * smax * bnt * 128 * 4;
  *out = sh;
  return MUSE_OK;
}

template <int BNT>
int launch_sk_t(const CUtensorMap& tmx, const muse::SkArgs& a, int g, bool pdl, cudaStream_t st) {
  auto kern = muse::tc_streamk_kernel<BNT>;
  static bool configured[kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(tc_streamk): %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(g), 1, 1);
  cfg.blockDim = dim3(muse::kSkThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(muse::sk_smem(BNT, a.stages));
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tmx, a);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "tc_streamk launch (tile %d): %s", BNT, cudaGetErrorString(e));
  return MUSE_OK;
}

int run_streamk(const void* x, const void* tiles, void* y, int64_t m, int64_t n, int64_t k, const MusePlan& p,
                void* scratch, int64_t scratch_bytes, cudaStream_t st) {
  SkShape sh;
  if (int rc = sk_shape(m, n, k, p, &sh)) return rc;
  if (!scratch || scratch_bytes < sh.scratch)
    return fail(MUSE_ERR_CAPACITY, "tc_streamk: needs %lld bytes of zeroed scratch (got %lld)", (long long)sh.scratch,
                (long long)(scratch ? scratch_bytes : 0));
  if (reinterpret_cast<uintptr_t>(scratch) & 255u) return fail(MUSE_ERR_ALIGN, "tc_streamk: scratch must be 256-byte aligned");
  CUtensorMap tmx;
  if (int rc = make_map(&tmx, x, m, k, sh.bnt)) return rc;
  muse::SkArgs a;
  a.wtiles = static_cast<const uint8_t*>(tiles);
  a.y = static_cast<uint16_t*>(y);
  a.counters = static_cast<int*>(scratch);
  a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + kCounterBytes);
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.K = static_cast<int>(k);
  a.stages = sh.stages;
  a.rtiles = sh.rtiles;
  a.nkb = sh.nkb;
  a.ttiles = sh.ttiles;
  a.units = sh.units;
  a.smax = sh.smax;
  a.trace = g_trace.load();
  a.trace_cap = a.trace ? g_trace_cap.load() : 0;
  const bool pdl = (p.flags & MUSE_FLAG_PDL) != 0;
  switch (sh.bnt) {
    case 16: return launch_sk_t<16>(tmx, a, sh.g, pdl, st);
    case 32: return launch_sk_t<32>(tmx, a, sh.g, pdl, st);
    case 64: return launch_sk_t<64>(tmx, a, sh.g, pdl, st);
    case 128: return launch_sk_t<128>(tmx, a, sh.g, pdl, st);
    default: return launch_sk_t<256>(tmx, a, sh.g, pdl, st);
  }
}

// ---- row-window tcgen05 kernel (few tokens, no split-K fix-up) --------------------------------

struct RwShape {
  int bnt, split, groups, units16, rmax, stages;
};

int rw_shape(int64_t m, int64_t n, int64_t k, const MusePlan& p, RwShape* out) {
  DeviceInfo* d;
  int sms = 148, limit = kSmemLimit;
  if (device_info(&d) == MUSE_OK) {
    sms = d->sms;
    limit = std::min(kSmemLimit, d->smem_optin);
  }
  muse::clear_error();
  if (m > 128) return fail(MUSE_ERR_SHAPE, "tc_rows: at most 128 tokens (got %lld)", (long long)m);
  if (n > (int64_t(1) << 24) || k > (int64_t(1) << 24)) return fail(MUSE_ERR_SHAPE, "tc_rows: dimension too large");
  int bnt = p.tile_n;
  if (bnt == 0) {
    bnt = 16;
    while (bnt < m) bnt *= 2;
  }
  if ((bnt != 16 && bnt != 32 && bnt != 64 && bnt != 128) || bnt < m)
    return fail(MUSE_ERR_PLAN, "tc_rows: tile_n must be 16, 32, 64 or 128 and hold all %lld tokens (got %d)", (long long)m,
                bnt);
  const int nkb = static_cast<int>((k + 63) / 64);
  const int split = p.split > 0 ? p.split : 1;
  if ((split != 1 && split != 2 && split != 4) || split > nkb)
    return fail(MUSE_ERR_PLAN, "tc_rows: split must be 1, 2 or 4 and at most K / 64 (got %d)", split);
  const int units16 = static_cast<int>((n + 15) / 16);
  int groups = (p.ctas > 0 ? p.ctas : sms) / split;
  groups = std::max(1, std::min(groups, units16));
  const int rmax = 16 * ((units16 + groups - 1) / groups);
  if (rmax > muse::kRwMaxRows)
    return fail(MUSE_ERR_PLAN, "tc_rows: %d windows leave %d rows a window (max %d): use more CTAs", groups, rmax,
                muse::kRwMaxRows);
  const int per = muse::rw_stage_bytes(bnt, rmax);
  int stages = p.stages;
  if (stages <= 0) stages = std::min(16, (limit - 1024 - 64) / (per + 16));  // the deepest ring that fits
  if (stages < 2 || muse::rw_smem(bnt, rmax, stages) > limit)
    return fail(MUSE_ERR_PLAN, "tc_rows: %d stages of %d bytes do not fit shared memory", stages, per);
  if (split > 1 && static_cast<int64_t>(bnt) * rmax * 4 > static_cast<int64_t>(stages) * per)
    return fail(MUSE_ERR_PLAN, "tc_rows: the FP32 partial does not fit the drained ring");
  out->bnt = bnt;
  out->split = split;
  out->groups = groups;
  out->units16 = units16;
  out->rmax = rmax;
  out->stages = stages;
  return MUSE_OK;
}

template <int BNT>
int launch_rw_t(const CUtensorMap& tmx, const muse::RwArgs& a, bool pdl, cudaStream_t st) {
  auto kern = muse::tc_rows_kernel<BNT>;
  static bool configured[kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  cudaError_t e = cudaSuccess;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(tc_rows): %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  const bool cluster = a.split > 1;
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(a.groups * a.split), 1, 1);
  cfg.blockDim = dim3(muse::kRwThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(muse::rw_smem(BNT, a.rmax, a.stages));
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(a.split);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = (pdl && !cluster) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  if (cluster) {
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess || clusters < 1)
      return fail(MUSE_ERR_PLAN, "tc_rows: clusters of %d CTAs with %zu B shared memory cannot be scheduled (%s)", a.split,
                  cfg.dynamicSmemBytes, e == cudaSuccess ? "occupancy 0" : cudaGetErrorString(e));
  }
  e = cudaLaunchKernelEx(&cfg, kern, tmx, a);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "tc_rows launch (tile %d, split %d): %s", BNT, a.split, cudaGetErrorString(e));
  return MUSE_OK;
}

// W as packed tiles (wrows == nullptr) or as the window-major copy (tiles == nullptr).
int run_rows(const void* x, const void* tiles, const void* wrows, void* y, int64_t m, int64_t n, int64_t k,
             const MusePlan& p, cudaStream_t st) {
  RwShape sh;
  if (int rc = rw_shape(m, n, k, p, &sh)) return rc;
  CUtensorMap tmx;
  if (int rc = make_map(&tmx, x, m, k, sh.bnt)) return rc;
  muse::RwArgs a;
  a.wtiles = static_cast<const uint8_t*>(tiles);
  a.wrows = static_cast<const uint8_t*>(wrows);
  a.y = static_cast<uint16_t*>(y);
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.nkb = static_cast<int>((k + 63) / 64);
  a.stages = sh.stages;
  a.split = sh.split;
  a.groups = sh.groups;
  a.units16 = sh.units16;
  a.rmax = sh.rmax;
  a.y_vec = (n % 8 == 0 && aligned16(y)) ? 1 : 0;
  a.trace = g_trace.load();
  a.trace_cap = a.trace ? g_trace_cap.load() : 0;
  const bool pdl = (p.flags & MUSE_FLAG_PDL) != 0;
  switch (sh.bnt) {
    case 16: return launch_rw_t<16>(tmx, a, pdl, st);
    case 32: return launch_rw_t<32>(tmx, a, pdl, st);
    case 64: return launch_rw_t<64>(tmx, a, pdl, st);
    default: return launch_rw_t<128>(tmx, a, pdl, st);
  }
}

// ---- persistent prefill GEMM -------------------------------------------------------------------

int run_gemm(const void* x, const void* tiles, void* y, int64_t m, int64_t n, int64_t k, const MusePlan& p,
             cudaStream_t st) {
  DeviceInfo* d;
  if (int rc = device_info(&d)) return rc;
  if (m > (int64_t(1) << 24) || n > (int64_t(1) << 24) || k > (int64_t(1) << 24))
    return fail(MUSE_ERR_SHAPE, "tc_gemm: dimension too large");
  const int limit = std::min(kSmemLimit, d->smem_optin);
  const int max_stages = (limit - 1024 - 128) / (muse::kGmABytes + muse::kGmBBytes + 16);
  const int stages = p.stages > 0 ? p.stages : std::min(4, max_stages);
  if (stages < 2 || stages > max_stages) return fail(MUSE_ERR_PLAN, "tc_gemm: %d stages do not fit (max %d)", stages, max_stages);
  CUtensorMap tmx;
  if (int rc = make_map(&tmx, x, m, k, 128)) return rc;
  muse::GmArgs a;
  a.wtiles = static_cast<const uint8_t*>(tiles);
  a.y = static_cast<uint16_t*>(y);
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.K = static_cast<int>(k);
  a.stages = stages;
  a.mtiles = static_cast<int>((m + 127) / 128);
  a.ntiles = static_cast<int>((n + muse::kGmBN - 1) / muse::kGmBN);
  a.nkb = static_cast<int>((k + 63) / 64);
  a.rtiles = static_cast<int>((n + 127) / 128);
  a.trace = g_trace.load();
  a.trace_cap = a.trace ? g_trace_cap.load() : 0;
  const long long tiles_total = static_cast<long long>(a.mtiles) * a.ntiles;
  if (tiles_total > INT32_MAX) return fail(MUSE_ERR_SHAPE, "tc_gemm: too many tiles");
  const int grid = static_cast<int>(std::min<long long>(p.ctas > 0 ? p.ctas : d->sms, tiles_total));
  auto kern = muse::tc_gemm_kernel;
  static bool configured[kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(tc_gemm): %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(grid), 1, 1);
  cfg.blockDim = dim3(muse::kGmThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(muse::gm_smem(stages));
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = (p.flags & MUSE_FLAG_PDL) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  cudaError_t e = cudaLaunchKernelEx(&cfg, kern, tmx, a);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "tc_gemm launch: %s", cudaGetErrorString(e));
  return MUSE_OK;
}

// ---- persistent prefill GEMM over CTA pairs --------------------------------------------------

// Stream-K layout of the pair GEMM for `pairs` CTA pairs: the first stream-K tile (0: all; with
// `tail`, the tiles after the last whole wave of pairs: the whole waves run persistently), the most
// pairs sharing a stream-K tile, and the scratch: 64 KB of tickets, then the partials of the stream-K
// tiles ([tile][contributor][CTA] of 128 KB). Returns the bytes; *tile0 == tiles: nothing to share.
int64_t g2_sk_layout(int64_t m, int64_t n, int64_t k, int64_t pairs, bool tail, int64_t* tile0, int* smax_out) {
  const int64_t tiles = ((m + 255) / 256) * ((n + 255) / 256);
  const int64_t nkb = (k + 63) / 64;
  pairs = std::max<int64_t>(1, pairs);
  const int64_t t0 = tail ? tiles / pairs * pairs : 0;
  const int64_t sk_tiles = tiles - t0;
  const int64_t minrange = std::max<int64_t>(1, sk_tiles * nkb / pairs);
  const int smax = static_cast<int>((nkb + minrange - 1) / minrange + 1);
  if (tile0) *tile0 = t0;
  if (smax_out) *smax_out = smax;
  return sk_tiles ? kCounterBytes + sk_tiles * smax * 2 * 128 * 256 * 4 : 0;
}

// Scratch for a stream-K plan of the pair GEMM on a device of `sms` SMs: the most any pair count up to
// sms / 2 needs (more pairs share a tile more ways; with a tail, fewer pairs can leave a longer tail).
int64_t g2_sk_scratch(int64_t m, int64_t n, int64_t k, int sms, bool tail) {
  int64_t need = 0;
  const int64_t hi = std::max(1, sms / 2);
  for (int64_t p = tail ? 1 : hi; p <= hi; ++p) need = std::max(need, g2_sk_layout(m, n, k, p, tail, nullptr, nullptr));
  return need;
}

// g != nullptr: the all-gather epilogue (y unused; every value goes to each rank's y_full).
// MUSE_FLAG_STREAMK: stream-K schedule over scratch (zeroed once; the kernel leaves it zeroed).
int run_gemm2(const void* x, const void* tiles, void* y, int64_t m, int64_t n, int64_t k, const MusePlan& p,
              cudaStream_t st, const muse::GatherOut* g = nullptr, void* scratch = nullptr, int64_t scratch_bytes = 0) {
  DeviceInfo* d;
  if (int rc = device_info(&d)) return rc;
  if (m > (int64_t(1) << 24) || n > (int64_t(1) << 24) || k > (int64_t(1) << 24))
    return fail(MUSE_ERR_SHAPE, "tc_gemm2: dimension too large");
  const int limit = std::min(kSmemLimit, d->smem_optin);
  const int extra = g ? muse::g2_smem_gather(0) - muse::g2_smem(0) : 0;  // the gather epilogue's staging
  const int max_stages = (limit - 1024 - 128 - extra) / (muse::kG2Stage + 16);
  const int stages = p.stages > 0 ? p.stages : std::min(6, max_stages);
  if (stages < 2 || stages > max_stages) return fail(MUSE_ERR_PLAN, "tc_gemm2: %d stages do not fit (max %d)", stages, max_stages);
  muse::G2Args a;
  a.y = static_cast<uint16_t*>(y);
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.K = static_cast<int>(k);
  a.stages = stages;
  a.mtiles = static_cast<int>((m + 255) / 256);
  a.ntiles = static_cast<int>((n + 255) / 256);
  a.nkb = static_cast<int>((k + 63) / 64);
  a.rtiles = static_cast<int>((n + 127) / 128);
  // Token tiles a group walks together (plan->split, else as many as keep the group's x within
  // 32 MB, a quarter of the L2, so it stays resident while W streams past; measured on a B200 at
  // 8192 x 57344 x 8192: groups of 8 token tiles 6.17 ms, 16: 6.18-6.27 ms, all 32: 6.75 ms).
  if (p.split < 0) return fail(MUSE_ERR_PLAN, "tc_gemm2: split (token tiles a group) must be >= 0");
  a.group_m = p.split > 0 ? std::min(p.split, a.mtiles)
                          : static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(a.mtiles, (32ll << 20) / (512 * k))));
  a.trace = g_trace.load();
  a.trace_cap = a.trace ? g_trace_cap.load() : 0;
  const long long tiles_total = static_cast<long long>(a.mtiles) * a.ntiles;
  const long long tile_rows = static_cast<long long>(a.rtiles) * a.nkb * 128;
  if (tiles_total > INT32_MAX || tile_rows > INT32_MAX) return fail(MUSE_ERR_SHAPE, "tc_gemm2: too many tiles");
  std::memset(&a.g, 0, sizeof(a.g));
  if (g) a.g = *g;
  a.streamk = 0;
  a.smax = 0;
  a.sk_tile0 = 0;
  a.partials = nullptr;
  a.counters = nullptr;
  const bool sk_all = (p.flags & MUSE_FLAG_STREAMK) != 0, sk_tail = (p.flags & MUSE_FLAG_SK_TAIL) != 0;
  if ((sk_all || sk_tail) && g)
    return fail(MUSE_ERR_PLAN, "tc_gemm2: the fused all-gather runs the persistent (not stream-K) schedule");
  if (sk_all && sk_tail) return fail(MUSE_ERR_PLAN, "tc_gemm2: MUSE_FLAG_STREAMK and MUSE_FLAG_SK_TAIL exclude each other");
  CUtensorMap tmx, tmw;
  if (int rc = make_map(&tmx, x, m, k, 128)) return rc;
  // The packed tile array seen as [tiles * 128 rows, 64] BF16: a box is one 16 KB tile, copied as is.
  if (int rc = make_map(&tmw, tiles, tile_rows, 64, 128, CU_TENSOR_MAP_SWIZZLE_NONE)) return rc;
  auto kern = g ? muse::tc_gemm2_kernel<true> : muse::tc_gemm2_kernel<false>;
  static bool configured[2][kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  cudaError_t e = cudaSuccess;
  if (!configured[g ? 1 : 0][dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(tc_gemm2): %s", cudaGetErrorString(e));
    configured[g ? 1 : 0][dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(muse::kG2Threads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(g ? muse::g2_smem_gather(stages) : muse::g2_smem(stages));
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 0;  // no programmatic launch with clusters
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cfg.gridDim = dim3(2, 1, 1);
  int clusters = 0;
  e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
  if (e != cudaSuccess || clusters < 1)
    return fail(MUSE_ERR_PLAN, "tc_gemm2: CTA pairs cannot be scheduled (%s)", e == cudaSuccess ? "occupancy 0" : cudaGetErrorString(e));
  long long pairs = p.ctas > 0 ? p.ctas / 2 : clusters;
  // Persistent tiles: no more pairs than tiles. Stream-K: every resident pair (up to one k block each).
  const long long cap = sk_all ? tiles_total * a.nkb : tiles_total;
  pairs = std::max<long long>(1, std::min<long long>({pairs, static_cast<long long>(clusters), cap}));
  if (sk_all || sk_tail) {
    // The stream-K tiles' pairs wait for no one (the last contributor of a tile sums it), but the
    // scratch was sized for at most sms / 2 pairs.
    pairs = std::min<long long>(pairs, std::max(1, d->sms / 2));
    int64_t tile0 = 0;
    int smax = 0;
    const int64_t need = g2_sk_layout(m, n, k, pairs, sk_tail, &tile0, &smax);
    if (tile0 < tiles_total) {
      if (!scratch || scratch_bytes < need)
        return fail(MUSE_ERR_CAPACITY, "tc_gemm2: stream-K needs %lld bytes of zeroed scratch (got %lld)", (long long)need,
                    (long long)(scratch ? scratch_bytes : 0));
      if (reinterpret_cast<uintptr_t>(scratch) & 255u)
        return fail(MUSE_ERR_ALIGN, "tc_gemm2: scratch must be 256-byte aligned");
      if ((tiles_total - tile0) * 2 > kMaxCounters) return fail(MUSE_ERR_SHAPE, "tc_gemm2: too many tiles for stream-K");
      a.streamk = 1;
      a.smax = smax;
      a.sk_tile0 = static_cast<int>(tile0);
      a.counters = static_cast<int*>(scratch);
      a.partials = reinterpret_cast<float4*>(static_cast<uint8_t*>(scratch) + kCounterBytes);
    }
  }
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  e = cudaLaunchKernelEx(&cfg, kern, tmx, tmw, a);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "tc_gemm2 launch: %s", cudaGetErrorString(e));
  return MUSE_OK;
}

// ---- medium-M pair GEMM (256 W rows x T tokens a CTA pair, K split reduced by the split's pairs) ----

struct PkShape {
  int t = 0, s = 1, stages = 0, nkb = 0, rtiles = 0, ttiles = 0;
  int64_t tiles = 0, partial_bytes = 0, scratch = 0;
};

int pk_shape(int64_t m, int64_t n, int64_t k, const MusePlan& p, PkShape* out) {
  if (m > (int64_t(1) << 24) || n > (int64_t(1) << 24) || k > (int64_t(1) << 24))
    return fail(MUSE_ERR_SHAPE, "tc_pairk: dimension too large");
  PkShape sh;
  sh.t = p.tile_n > 0 ? p.tile_n : static_cast<int>(std::min<int64_t>(256, (m + 15) / 16 * 16));
  if (sh.t % 16 || sh.t < 16 || sh.t > 256) return fail(MUSE_ERR_PLAN, "tc_pairk: tile_n must be a multiple of 16 in 16..256");
  sh.nkb = static_cast<int>((k + 63) / 64);
  sh.s = p.split > 0 ? p.split : 1;
  if (sh.s > sh.nkb || sh.t % sh.s || sh.s > 64)
    return fail(MUSE_ERR_PLAN, "tc_pairk: split %d must divide tile_n (%d) and not exceed the k blocks (%d) or 64", sh.s,
                sh.t, sh.nkb);
  sh.rtiles = static_cast<int>((n + 127) / 128);
  sh.ttiles = static_cast<int>((m + sh.t - 1) / sh.t);
  sh.tiles = ((n + 255) / 256) * sh.ttiles;
  const int limit = kSmemLimit;
  const int max_stages = (limit - 1024 - 128) / muse::pk_stage_bytes(sh.t);
  const int per_split = (sh.nkb + sh.s - 1) / sh.s;
  sh.stages = p.stages > 0 ? p.stages : std::max(2, std::min(max_stages, per_split));
  if (sh.stages < 2 || muse::pk_smem(sh.t, sh.s, sh.stages) > limit)
    return fail(MUSE_ERR_PLAN, "tc_pairk: %d stages of tile_n %d do not fit in shared memory", sh.stages, sh.t);
  if (sh.tiles * sh.s * 2 > INT32_MAX || static_cast<int64_t>(sh.rtiles) * sh.nkb * 128 > INT32_MAX)
    return fail(MUSE_ERR_SHAPE, "tc_pairk: too many tiles");
  if (sh.s > 1) {
    if (sh.tiles * 4 > kMaxCounters) return fail(MUSE_ERR_SHAPE, "tc_pairk: too many tiles for a K split");
    sh.partial_bytes = sh.tiles * 2 * sh.s * sh.t * 128 * 4;
    sh.scratch = kCounterBytes + sh.partial_bytes;
  }
  *out = sh;
  return MUSE_OK;
}

int run_pairk(const void* x, const void* tiles, void* y, int64_t m, int64_t n, int64_t k, const MusePlan& p, void* scratch,
              int64_t scratch_bytes, cudaStream_t st) {
  DeviceInfo* d;
  if (int rc = device_info(&d)) return rc;
  PkShape sh;
  if (int rc = pk_shape(m, n, k, p, &sh)) return rc;
  if (sh.s > 1) {
    if (!scratch || scratch_bytes < sh.scratch)
      return fail(MUSE_ERR_CAPACITY, "tc_pairk: split %d needs %lld bytes of zeroed scratch (got %lld)", sh.s,
                  (long long)sh.scratch, (long long)(scratch ? scratch_bytes : 0));
    if (reinterpret_cast<uintptr_t>(scratch) & 255u) return fail(MUSE_ERR_ALIGN, "tc_pairk: scratch must be 256-byte aligned");
  }
  muse::PkArgs a;
  a.y = static_cast<uint16_t*>(y);
  a.partials = sh.s > 1 ? reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + kCounterBytes) : nullptr;
  a.counters = sh.s > 1 ? static_cast<int*>(scratch) : nullptr;
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.T = sh.t;
  a.split = sh.s;
  a.stages = sh.stages;
  a.nkb = sh.nkb;
  a.rtiles = sh.rtiles;
  a.ttiles = sh.ttiles;
  a.trace = g_trace.load();
  a.trace_cap = a.trace ? g_trace_cap.load() : 0;
  CUtensorMap tmx, tmw, tmy;
  if (int rc = make_map(&tmx, x, m, k, sh.t / 2)) return rc;
  // The packed tile array seen as [tiles * 128 rows, 64] BF16: a box is one 16 KB tile, copied as is.
  if (int rc = make_map(&tmw, tiles, static_cast<int64_t>(sh.rtiles) * sh.nkb * 128, 64, 128, CU_TENSOR_MAP_SWIZZLE_NONE))
    return rc;
  // y by TMA tensor stores where its rows are 16-byte multiples: boxes of 128 columns (a CTA's W rows)
  // x T / split tokens (a reducer's slice), no swizzle.
  a.tma_y = (n % 8 == 0 && aligned16(y)) ? 1 : 0;
  std::memset(&tmy, 0, sizeof(tmy));
  if (a.tma_y) {
    auto fn = encode_fn();
    if (!fn) return fail(MUSE_ERR_CUDA, "cuTensorMapEncodeTiled entry point not found");
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(m)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(n * 2)};
    cuuint32_t box[2] = {128u, static_cast<cuuint32_t>(sh.t / sh.s)};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = fn(&tmy, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MUSE_ERR_CUDA, "cuTensorMapEncodeTiled (y) failed (%d)", static_cast<int>(r));
  }
  auto kern = muse::tc_pairk_kernel;
  static bool configured[kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  cudaError_t e = cudaSuccess;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(tc_pairk): %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(muse::kPkThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(muse::pk_smem(sh.t, sh.s, sh.stages));
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = (p.flags & MUSE_FLAG_PDL) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  const long long pairs = sh.tiles * sh.s;
  if (sh.s > 1) {
    // The split's pairs wait for one another: the whole grid must be resident at once.
    cfg.gridDim = dim3(2, 1, 1);
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess || clusters < 1)
      return fail(MUSE_ERR_PLAN, "tc_pairk: CTA pairs cannot be scheduled (%s)", e == cudaSuccess ? "occupancy 0" : cudaGetErrorString(e));
    if (pairs > clusters)
      return fail(MUSE_ERR_PLAN, "tc_pairk: %lld tiles x split %d = %lld CTA pairs exceed the %d that can be resident at once",
                  (long long)sh.tiles, sh.s, pairs, clusters);
  }
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  e = cudaLaunchKernelEx(&cfg, kern, tmx, tmw, tmy, a);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "tc_pairk launch: %s", cudaGetErrorString(e));
  return MUSE_OK;
}

// Stream-K schedule of the medium-M pair GEMM (MUSE_FLAG_STREAMK on a TC_PAIRK plan).
struct PsShape {
  int t = 0, stages = 0, nkb = 0, rtiles = 0, ttiles = 0, cmax = 0;
  int64_t tiles = 0, units = 0, scratch = 0;
};

// `pairs`: the CTA pairs the grid will have, at most one a unit (the scratch is sized for the most a
// device can hold: more pairs make shorter runs and so more contributors a tile).
int ps_shape(int64_t m, int64_t n, int64_t k, const MusePlan& p, int pairs, PsShape* out) {
  if (m > (int64_t(1) << 24) || n > (int64_t(1) << 24) || k > (int64_t(1) << 24))
    return fail(MUSE_ERR_SHAPE, "tc_pairk stream-K: dimension too large");
  PsShape sh;
  sh.t = p.tile_n > 0 ? p.tile_n : static_cast<int>(std::min<int64_t>(256, (m + 15) / 16 * 16));
  if (sh.t % 16 || sh.t < 16 || sh.t > 256) return fail(MUSE_ERR_PLAN, "tc_pairk: tile_n must be a multiple of 16 in 16..256");
  sh.nkb = static_cast<int>((k + 63) / 64);
  sh.rtiles = static_cast<int>((n + 127) / 128);
  sh.ttiles = static_cast<int>((m + sh.t - 1) / sh.t);
  sh.tiles = ((n + 255) / 256) * sh.ttiles;
  sh.units = sh.tiles * sh.nkb;
  if (pairs < 1) return fail(MUSE_ERR_PLAN, "tc_pairk stream-K: no CTA pairs");
  if (pairs > sh.units) pairs = static_cast<int>(sh.units);
  if ((sh.units + pairs - 1) / pairs > sh.nkb)
    return fail(MUSE_ERR_PLAN, "tc_pairk stream-K: runs of %lld k blocks exceed a tile's %d (more tiles than pairs can share: "
                               "use the split or the prefill kernels)", (long long)((sh.units + pairs - 1) / pairs), sh.nkb);
  const int max_stages = (kSmemLimit - 1024 - 128) / muse::pk_stage_bytes(sh.t);
  sh.stages = p.stages > 0 ? p.stages : max_stages;
  if (sh.stages < 2 || muse::ps_smem(sh.t, sh.stages) > kSmemLimit)
    return fail(MUSE_ERR_PLAN, "tc_pairk stream-K: %d stages of tile_n %d do not fit in shared memory", sh.stages, sh.t);
  if (sh.tiles * 4 > kMaxCounters) return fail(MUSE_ERR_SHAPE, "tc_pairk stream-K: too many tiles");
  int cmax = 1;
  for (int64_t t = 0; t < sh.tiles; ++t) {
    const int first = muse::t12_owner(t * sh.nkb, sh.units, pairs), last = muse::t12_owner((t + 1) * sh.nkb - 1, sh.units, pairs);
    cmax = std::max(cmax, last - first + 1);
  }
  sh.cmax = cmax;
  sh.scratch = kCounterBytes + sh.tiles * 2 * cmax * sh.t * 128 * 4;
  *out = sh;
  return MUSE_OK;
}

int run_pairsk(const void* x, const void* tiles, void* y, int64_t m, int64_t n, int64_t k, const MusePlan& p, void* scratch,
               int64_t scratch_bytes, cudaStream_t st) {
  DeviceInfo* d;
  if (int rc = device_info(&d)) return rc;
  auto kern = muse::tc_pairsk_kernel;
  static bool configured[kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  cudaError_t e = cudaSuccess;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(tc_pairsk): %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  // The scratch bound: contributors a tile with every pair the device has.
  PsShape bound;
  if (int rc = ps_shape(m, n, k, p, std::max(1, d->sms / 2), &bound)) return rc;
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(muse::kPkThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(muse::ps_smem(bound.t, bound.stages));
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = (p.flags & MUSE_FLAG_PDL) ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cfg.gridDim = dim3(2, 1, 1);
  int clusters = 0;
  e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
  if (e != cudaSuccess || clusters < 1)
    return fail(MUSE_ERR_PLAN, "tc_pairk stream-K: CTA pairs cannot be scheduled (%s)",
                e == cudaSuccess ? "occupancy 0" : cudaGetErrorString(e));
  // Every pair waits for the others of its tiles: the whole grid must be resident at once.
  int pairs = p.ctas > 0 ? p.ctas / 2 : clusters;
  if (pairs > clusters || pairs > d->sms / 2)
    return fail(MUSE_ERR_PLAN, "tc_pairk stream-K: %d CTA pairs exceed the %d that can be resident at once", pairs,
                std::min(clusters, d->sms / 2));
  if (pairs > bound.units) pairs = static_cast<int>(bound.units);  // at most one a unit
  PsShape sh;
  if (int rc = ps_shape(m, n, k, p, pairs, &sh)) return rc;
  if (!scratch || scratch_bytes < bound.scratch)
    return fail(MUSE_ERR_CAPACITY, "tc_pairk stream-K needs %lld bytes of zeroed scratch (got %lld)", (long long)bound.scratch,
                (long long)(scratch ? scratch_bytes : 0));
  if (reinterpret_cast<uintptr_t>(scratch) & 255u) return fail(MUSE_ERR_ALIGN, "tc_pairk: scratch must be 256-byte aligned");
  muse::PsArgs a;
  a.y = static_cast<uint16_t*>(y);
  a.counters = static_cast<int*>(scratch);
  a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + kCounterBytes);
  a.units = sh.units;
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.T = sh.t;
  a.stages = sh.stages;
  a.nkb = sh.nkb;
  a.rtiles = sh.rtiles;
  a.ttiles = sh.ttiles;
  a.cmax = bound.cmax;  // slot stride: the scratch layout muse_scratch_bytes sized
  a.trace = g_trace.load();
  a.trace_cap = a.trace ? g_trace_cap.load() : 0;
  CUtensorMap tmx, tmw, tmy;
  if (int rc = make_map(&tmx, x, m, k, sh.t / 2)) return rc;
  if (int rc = make_map(&tmw, tiles, static_cast<int64_t>(sh.rtiles) * sh.nkb * 128, 64, 128, CU_TENSOR_MAP_SWIZZLE_NONE))
    return rc;
  // y by 16-row TMA tensor stores where its rows are 16-byte multiples: boxes of 128 columns x 16 tokens.
  a.tma_y = (n % 8 == 0 && aligned16(y)) ? 1 : 0;
  std::memset(&tmy, 0, sizeof(tmy));
  if (a.tma_y) {
    auto fn = encode_fn();
    if (!fn) return fail(MUSE_ERR_CUDA, "cuTensorMapEncodeTiled entry point not found");
    cuuint64_t dims[2] = {static_cast<cuuint64_t>(n), static_cast<cuuint64_t>(m)};
    cuuint64_t strides[1] = {static_cast<cuuint64_t>(n * 2)};
    cuuint32_t box[2] = {128u, 16u};
    cuuint32_t estr[2] = {1u, 1u};
    CUresult r = fn(&tmy, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, y, dims, strides, box, estr, CU_TENSOR_MAP_INTERLEAVE_NONE,
                    CU_TENSOR_MAP_SWIZZLE_NONE, CU_TENSOR_MAP_L2_PROMOTION_NONE, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (r != CUDA_SUCCESS) return fail(MUSE_ERR_CUDA, "cuTensorMapEncodeTiled (y) failed (%d)", static_cast<int>(r));
  }
  cfg.dynamicSmemBytes = static_cast<size_t>(muse::ps_smem(sh.t, sh.stages));
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  e = cudaLaunchKernelEx(&cfg, kern, tmx, tmw, tmy, a);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "tc_pairk stream-K launch: %s", cudaGetErrorString(e));
  return MUSE_OK;
}

// ---- wide-tile pair GEMM (256 tokens x 512 W rows a CTA pair) -------------------------------------

int run_wide(const void* x, const void* tiles, void* y, int64_t m, int64_t n, int64_t k, const MusePlan& p, cudaStream_t st) {
  DeviceInfo* d;
  if (int rc = device_info(&d)) return rc;
  if (m > (int64_t(1) << 24) || n > (int64_t(1) << 24) || k > (int64_t(1) << 24))
    return fail(MUSE_ERR_SHAPE, "tc_wide: dimension too large");
  const int limit = std::min(kSmemLimit, d->smem_optin);
  // y by TMA tensor stores from a 32 KB staging tile where its rows are 16-byte multiples.
  const bool tma_y = n % 8 == 0 && aligned16(y);
  const int max_stages = (limit - 1024 - 128 - (tma_y ? muse::kWdStg : 0)) / (muse::kWdStage + 16);
  const int stages = p.stages > 0 ? p.stages : max_stages;
  if (stages < 2 || stages > max_stages) return fail(MUSE_ERR_PLAN, "tc_wide: %d stages do not fit (max %d)", stages, max_stages);
  if (p.split < 0) return fail(MUSE_ERR_PLAN, "tc_wide: split (token tiles a group) must be >= 0");
  muse::WdArgs a;
  a.y = static_cast<uint16_t*>(y);
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.stages = stages;
  a.mtiles = static_cast<int>((m + 255) / 256);
  a.ntiles = static_cast<int>((n + 511) / 512);
  a.nkb = static_cast<int>((k + 63) / 64);
  a.rtiles = static_cast<int>((n + 127) / 128);
  // Token tiles a group walks together: plan->split, else as many as keep the group's x within 64 MB
  // (measured on a B200 at 8192 x 57344 x 8192, interleaved medians: groups of 16 token tiles
  // 6.01 ms, of 8: 6.44 ms).
  a.group_m = p.split > 0 ? std::min(p.split, a.mtiles)
                          : static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(a.mtiles, (64ll << 20) / (512 * k))));
  a.tma_y = tma_y ? 1 : 0;
  a.trace = g_trace.load();
  a.trace_cap = a.trace ? g_trace_cap.load() : 0;
  const long long tiles_total = static_cast<long long>(a.mtiles) * a.ntiles;
  const long long tile_rows = static_cast<long long>(a.rtiles) * a.nkb * 128;
  if (tiles_total > INT32_MAX || tile_rows > INT32_MAX) return fail(MUSE_ERR_SHAPE, "tc_wide: too many tiles");
  CUtensorMap tmx, tmw, tmy;
  std::memset(&tmy, 0, sizeof(tmy));
  // y seen as [M, N] BF16, boxes of 64 columns x 128 rows, 128-byte swizzle (the staging tile's order).
  if (tma_y) {
    if (int rc = make_map(&tmy, y, m, n, 128)) return rc;
  }
  if (int rc = make_map(&tmx, x, m, k, 128)) return rc;
  // The packed tile array seen as [tiles * 128 rows, 64] BF16: a box is one 16 KB tile, copied as is.
  if (int rc = make_map(&tmw, tiles, tile_rows, 64, 128, CU_TENSOR_MAP_SWIZZLE_NONE)) return rc;
  auto kern = muse::tc_wide_kernel;
  static bool configured[kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  cudaError_t e = cudaSuccess;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(tc_wide): %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.blockDim = dim3(muse::kWdThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(muse::wd_smem(stages, tma_y));
  cfg.stream = st;
  cudaLaunchAttribute attr[2];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = 2;
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[1].val.programmaticStreamSerializationAllowed = 0;  // no programmatic launch with clusters
  cfg.attrs = attr;
  cfg.numAttrs = 2;
  cfg.gridDim = dim3(2, 1, 1);
  int clusters = 0;
  e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
  if (e != cudaSuccess || clusters < 1)
    return fail(MUSE_ERR_PLAN, "tc_wide: CTA pairs cannot be scheduled (%s)", e == cudaSuccess ? "occupancy 0" : cudaGetErrorString(e));
  long long pairs = p.ctas > 0 ? p.ctas / 2 : clusters;
  pairs = std::max<long long>(1, std::min<long long>({pairs, static_cast<long long>(clusters), tiles_total}));
  cfg.gridDim = dim3(static_cast<unsigned>(2 * pairs), 1, 1);
  e = cudaLaunchKernelEx(&cfg, kern, tmx, tmw, tmy, a);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "tc_wide launch: %s", cudaGetErrorString(e));
  return MUSE_OK;
}

// ---- stream-K skinny kernel: W as the UMMA's B operand (BF16 tiles or 12-bit blocks) -----------

struct SnShape {
  int bnt, stages, g, smax;
  int rtiles, rpairs, nkb, ttiles;
  long long units, tiles;
  int64_t scratch;
};

int sn_shape(bool twelve, int64_t m, int64_t n, int64_t k, const MusePlan& p, SnShape* out) {
  DeviceInfo* d;
  int sms = 148, limit = kSmemLimit;
  if (device_info(&d) == MUSE_OK) {
    sms = d->sms;
    limit = std::min(kSmemLimit, d->smem_optin);
  }
  muse::clear_error();
  const char* name = twelve ? "tc_12b" : "tc_skinny";
  if (twelve && (k < 512 || k % 512 || k > 65536))
    return fail(MUSE_ERR_SHAPE, "%s: K must be a multiple of 512 and <= 65536", name);
  if (m > (int64_t(1) << 24) || n > (int64_t(1) << 24) || k > (int64_t(1) << 24))
    return fail(MUSE_ERR_SHAPE, "%s: dimension too large", name);
  int bnt = p.tile_n;
  if (bnt == 0) {
    bnt = 16;
    while (bnt < m && bnt < 128) bnt *= 2;
  }
  if (bnt != 16 && bnt != 32 && bnt != 64 && bnt != 128)
    return fail(MUSE_ERR_PLAN, "%s: tile_n must be 16, 32, 64 or 128 (got %d)", name, bnt);
  const int per_stage = muse::sn_smem(bnt, 1) - muse::sn_smem(bnt, 0);
  const int max_stages = (limit - muse::sn_smem(bnt, 0)) / per_stage;
  // 12-bit: the decoder groups take units in turn, and a stage's successive units must belong to
  // one group (which handles them in order), or a group could wait on a slot two phases ahead of
  // its mbarrier: stages is a multiple of the group count.
  const int groups = twelve ? muse::kSnDecGroups : 1;
  const int stages = p.stages > 0 ? p.stages : std::min(twelve ? 6 : 5, max_stages) / groups * groups;
  if (stages < 2 || stages > max_stages)
    return fail(MUSE_ERR_PLAN, "%s: %d stages do not fit (max %d)", name, stages, max_stages);
  if (stages % groups)
    return fail(MUSE_ERR_PLAN, "%s: stages (%d) must be a multiple of the %d decoder groups", name, stages, groups);
  SnShape sh;
  sh.bnt = bnt;
  sh.stages = stages;
  sh.rtiles = static_cast<int>((n + 127) / 128);
  sh.rpairs = (sh.rtiles + 1) / 2;
  sh.nkb = static_cast<int>((k + 63) / 64);
  sh.ttiles = static_cast<int>((m + bnt - 1) / bnt);
  sh.tiles = static_cast<long long>(sh.rpairs) * sh.ttiles;
  sh.units = sh.tiles * sh.nkb;
  if (sh.tiles > kMaxCounters)
    return fail(MUSE_ERR_SHAPE, "%s: %lld output tiles exceed the %lld counters", name, sh.tiles, (long long)kMaxCounters);
  long long g = p.ctas > 0 ? p.ctas : sms;
  sh.g = static_cast<int>(std::min<long long>(g, sh.units));
  int smax = 1;
  for (long long t = 0; t < sh.tiles; ++t) {
    const int a0 = muse::t12_owner(t * sh.nkb, sh.units, sh.g);
    const int a1 = muse::t12_owner((t + 1) * sh.nkb - 1, sh.units, sh.g);
    smax = std::max(smax, a1 - a0 + 1);
  }
  sh.smax = smax;
  sh.scratch = kCounterBytes + static_cast<int64_t>(sh.tiles) * smax * bnt * muse::kSnRows * 4;
  *out = sh;
  return MUSE_OK;
}

template <bool kTwelve, int BNT>
int launch_sn_t(const CUtensorMap& tmx, const muse::SnArgs& a, int g, bool pdl, cudaStream_t st) {
  auto kern = muse::tc_skinny_kernel<kTwelve, BNT>;
  // Every CTA holds all 512 TMEM columns: ask for more than half an SM's shared memory so that
  // no two CTAs (of this or the next launch) share an SM.
  const int smem = std::max(muse::sn_smem(BNT, a.stages), 116 * 1024);
  static bool configured[kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  cudaError_t e = cudaSuccess;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(tc_skinny): %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(g), 1, 1);
  cfg.blockDim = dim3(muse::sn_threads(kTwelve), 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, tmx, a);
  if (e != cudaSuccess)
    return fail(MUSE_ERR_CUDA, "%s launch (%d CTAs, tile %d): %s", kTwelve ? "tc_12b" : "tc_skinny", g, BNT,
                cudaGetErrorString(e));
  return MUSE_OK;
}

// W: packed BF16 tiles (twelve = false) or 12-bit blocks with enc's escape list (twelve = true).
// ---- 12-bit GEMV on the 12-bit blocks (register decode) --------------------------------------

struct G12Shape {
  int mt, stages, rtiles, nkb, ctas, ucap, smax;
  int64_t scratch;
  int smem;
};

// CTAs of gemv12t_kernel<mt> an SM's registers hold (queried once per device and token count).
int g12_reg_limit(int mt) {
  static int cache[kMaxDevices][3] = {};
  int dev = 0;
  if (current_device(&dev) != MUSE_OK) return 6;
  const int idx = mt == 1 ? 0 : (mt == 2 ? 1 : 2);
  if (cache[dev][idx] == 0) {
    cudaFuncAttributes fa;
    cudaError_t e = mt == 1 ? cudaFuncGetAttributes(&fa, muse::gemv12t_kernel<1>)
                    : mt == 2 ? cudaFuncGetAttributes(&fa, muse::gemv12t_kernel<2>)
                              : cudaFuncGetAttributes(&fa, muse::gemv12t_kernel<4>);
    int lim = 6;
    if (e == cudaSuccess && fa.numRegs > 0) {
      const int per_warp = ((fa.numRegs * 32 + 255) / 256) * 256;  // allocated in 256-register units
      lim = std::max(1, 65536 / (per_warp * (muse::kG12Threads / 32)));
    }
    cache[dev][idx] = lim;
  }
  return cache[dev][idx];
}

// Stream-K grid: as many CTAs as stay resident (up to six an SM; the kernel needs about four to
// hide its latencies), each taking units / ctas consecutive (row tile, k block) units.
int g12_shape(int64_t m, int64_t n, int64_t k, const MusePlan& p, G12Shape* out) {
  DeviceInfo* d;
  int sms = 148, limit = kSmemLimit;
  if (device_info(&d) == MUSE_OK) {
    sms = d->sms;
    limit = std::min(kSmemLimit, d->smem_optin);
  }
  muse::clear_error();
  if (m < 1 || m > 4) return fail(MUSE_ERR_SHAPE, "gemv_12t: M must be 1..4 (got %lld)", (long long)m);
  if (k % 128 != 0 || n > (int64_t(1) << 24) || k > (int64_t(1) << 24))
    return fail(MUSE_ERR_SHAPE, "gemv_12t: K must be a multiple of 128 and N, K < 2^24");
  G12Shape sh;
  sh.mt = m == 1 ? 1 : (m == 2 ? 2 : 4);
  sh.rtiles = static_cast<int>((n + 127) / 128);
  sh.nkb = static_cast<int>(k / 64);
  sh.stages = p.stages > 0 ? p.stages : 3;
  if (sh.stages < 2) return fail(MUSE_ERR_PLAN, "gemv_12t: at least 2 stages");
  const int64_t units = static_cast<int64_t>(sh.rtiles) * sh.nkb;
  if (sh.rtiles > kMaxCounters || units > (int64_t(1) << 30)) return fail(MUSE_ERR_SHAPE, "gemv_12t: too many row tiles");
  int64_t ctas = 0;
  if (p.ctas > 0) {
    ctas = std::min<int64_t>(p.ctas, units);
  } else {
    for (int per_sm = std::min(6, g12_reg_limit(sh.mt)); per_sm >= 1 && ctas == 0; --per_sm) {
      const int64_t g = std::min<int64_t>(units, static_cast<int64_t>(per_sm) * sms);
      const int ucap = static_cast<int>((units + g - 1) / g);
      const int smem = muse::g12_smem(sh.stages, ucap, sh.mt);
      if (smem <= limit && 233472 / (smem + 1024) >= per_sm) ctas = g;
    }
    if (ctas == 0) ctas = std::min<int64_t>(units, sms);
  }
  sh.ctas = static_cast<int>(ctas);
  sh.ucap = static_cast<int>((units + ctas - 1) / ctas);
  const int64_t minrange = std::max<int64_t>(1, units / ctas);
  sh.smax = static_cast<int>((sh.nkb + minrange - 1) / minrange + 1);
  sh.smem = muse::g12_smem(sh.stages, sh.ucap, sh.mt);
  if (sh.smem > limit)
    return fail(MUSE_ERR_PLAN, "gemv_12t: %d stages and x for %d units need %d bytes of shared memory (limit %d)",
                sh.stages, sh.ucap, sh.smem, limit);
  sh.scratch = kCounterBytes + static_cast<int64_t>(sh.rtiles) * sh.smax * sh.mt * 128 * 4;
  *out = sh;
  return MUSE_OK;
}

template <int MT>
int launch_g12_t(const muse::G12Args& a, int smem, unsigned grid, bool pdl, cudaStream_t st) {
  auto kern = muse::gemv12t_kernel<MT>;
  static bool configured[kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  cudaError_t e = cudaSuccess;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(gemv_12t): %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(grid, 1, 1);
  cfg.blockDim = dim3(muse::kG12Threads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "gemv_12t launch: %s", cudaGetErrorString(e));
  return MUSE_OK;
}

int run_gemv12t(const void* tiles12, const MuseEnc12* enc, const void* x, void* y, int64_t m, const MusePlan& p,
                void* scratch, int64_t scratch_bytes, cudaStream_t st) {
  G12Shape sh;
  if (int rc = g12_shape(m, enc->n, enc->k, p, &sh)) return rc;
  if (sh.scratch > 0 && (!scratch || scratch_bytes < sh.scratch))
    return fail(MUSE_ERR_CAPACITY, "gemv_12t: %d CTAs need %lld bytes of zeroed scratch (got %lld)", sh.ctas,
                (long long)sh.scratch, (long long)(scratch ? scratch_bytes : 0));
  if (sh.scratch > 0 && (reinterpret_cast<uintptr_t>(scratch) & 255u))
    return fail(MUSE_ERR_ALIGN, "gemv_12t: scratch must be 256-byte aligned");
  muse::G12Args a;
  a.blocks = static_cast<const uint8_t*>(tiles12);
  a.x = static_cast<const uint16_t*>(x);
  a.y = static_cast<uint16_t*>(y);
  a.esc_ptr = enc->esc_ptr;
  a.esc_val = enc->esc_val;
  a.counters = sh.scratch > 0 ? static_cast<int*>(scratch) : nullptr;
  a.partials = sh.scratch > 0 ? reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + kCounterBytes) : nullptr;
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(enc->n);
  a.K = static_cast<int>(enc->k);
  a.nkb = sh.nkb;
  a.rtiles = sh.rtiles;
  a.smax = sh.smax;
  a.ucap = sh.ucap;
  a.stages = sh.stages;
  a.trace = g_trace.load();
  a.trace_cap = a.trace ? g_trace_cap.load() : 0;
  const bool pdl = (p.flags & MUSE_FLAG_PDL) != 0;
  const unsigned grid = static_cast<unsigned>(sh.ctas);
  switch (sh.mt) {
    case 1: return launch_g12_t<1>(a, sh.smem, grid, pdl, st);
    case 2: return launch_g12_t<2>(a, sh.smem, grid, pdl, st);
    default: return launch_g12_t<4>(a, sh.smem, grid, pdl, st);
  }
}

struct GtShape {
  int mt, qw, nkb, quads, split, warps, groups, grid, smem;
};

// A warp takes qw adjacent quads (4 W rows each; plan->chunk: 1, 2, 4 or 8 (M <= 2), 0 = 2) over one of `split` K
// segments (0: as many as leave each warp at least two batches, a divisor of the CTA's warps);
// `warps` warps a CTA (0: 8).
int gt_shape(int64_t m, int64_t n, int64_t k, const MusePlan& p, GtShape* out) {
  DeviceInfo* d;
  int limit = kSmemLimit;
  if (device_info(&d) == MUSE_OK) limit = std::min(kSmemLimit, d->smem_optin);
  muse::clear_error();
  if (m < 1 || m > 4) return fail(MUSE_ERR_SHAPE, "gemv_tiles: M must be 1..4 (got %lld)", (long long)m);
  if (n > (int64_t(1) << 28) || k > (int64_t(1) << 24))
    return fail(MUSE_ERR_SHAPE, "gemv_tiles: N must be below 2^28 and K below 2^24");
  GtShape g;
  g.qw = p.chunk > 0 ? p.chunk : 2;
  if (g.qw != 1 && g.qw != 2 && g.qw != 4 && g.qw != 8)
    return fail(MUSE_ERR_PLAN, "gemv_tiles: quads a warp (chunk) must be 1, 2, 4 or 8 (got %d)", g.qw);
  if (g.qw == 8 && m > 2)
    return fail(MUSE_ERR_PLAN, "gemv_tiles: 8 quads a warp only for M <= 2 (its accumulators need the registers)");
  g.warps = p.warps > 0 ? p.warps : 8;
  if (g.warps > 16) return fail(MUSE_ERR_PLAN, "gemv_tiles: at most 16 warps a CTA (got %d)", g.warps);
  g.nkb = static_cast<int>((k + 63) / 64);
  g.split = p.split;
  const int batch_kb = muse::kGtBatch / g.qw;  // k blocks a batch
  if (g.split <= 0) {
    g.split = 1;
    while (g.warps % (2 * g.split) == 0 && g.nkb / (2 * g.split) >= 2 * batch_kb) g.split *= 2;
  }
  if (g.warps % g.split != 0)
    return fail(MUSE_ERR_PLAN, "gemv_tiles: split %d must divide the %d warps of a CTA", g.split, g.warps);
  if (g.split > g.nkb) return fail(MUSE_ERR_PLAN, "gemv_tiles: split %d exceeds the %d k blocks", g.split, g.nkb);
  g.mt = m == 1 ? 1 : (m == 2 ? 2 : 4);
  g.smem = muse::gt_smem(g.mt, g.qw, g.nkb, g.warps, g.split);
  if (g.smem > limit)
    return fail(MUSE_ERR_SHAPE, "gemv_tiles: x of %d tokens x %d k blocks needs %d bytes of shared memory (limit %d)",
                g.mt, g.nkb, g.smem, limit);
  g.quads = static_cast<int>((n + 127) / 128) * 32;
  g.groups = g.warps / g.split;
  const int per_cta = g.groups * g.qw;
  g.grid = (g.quads + per_cta - 1) / per_cta;
  *out = g;
  return MUSE_OK;
}

template <int MT, int QW>
int launch_gemv_tiles(const muse::GtArgs& a, const GtShape& g, bool pdl, cudaStream_t st) {
  auto kern = muse::gemv_tiles_kernel<MT, QW>;
  static bool configured[kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  cudaError_t e = cudaSuccess;
  if (!configured[dev]) {
    e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(gemv_tiles): %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(g.grid), 1, 1);
  cfg.blockDim = dim3(static_cast<unsigned>(g.warps * 32), 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(g.smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
  attr[0].val.programmaticStreamSerializationAllowed = pdl ? 1 : 0;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  e = cudaLaunchKernelEx(&cfg, kern, a);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "gemv_tiles launch: %s", cudaGetErrorString(e));
  return MUSE_OK;
}

template <int MT>
int launch_gemv_tiles_qw(const muse::GtArgs& a, const GtShape& g, bool pdl, cudaStream_t st) {
  switch (g.qw) {
    case 1: return launch_gemv_tiles<MT, 1>(a, g, pdl, st);
    case 2: return launch_gemv_tiles<MT, 2>(a, g, pdl, st);
    case 4: return launch_gemv_tiles<MT, 4>(a, g, pdl, st);
    default:
      if constexpr (MT <= 2) return launch_gemv_tiles<MT, 8>(a, g, pdl, st);
      return fail(MUSE_ERR_PLAN, "gemv_tiles: 8 quads a warp only for M <= 2");
  }
}

int run_gemv_tiles(const void* x, const void* tiles, void* y, int64_t m, int64_t n, int64_t k, const MusePlan& p,
                   cudaStream_t st) {
  GtShape g;
  if (int rc = gt_shape(m, n, k, p, &g)) return rc;
  muse::GtArgs a;
  a.tiles = static_cast<const uint8_t*>(tiles);
  a.x = static_cast<const uint16_t*>(x);
  a.y = static_cast<uint16_t*>(y);
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.K = static_cast<int>(k);
  a.nkb = g.nkb;
  a.quads = g.quads;
  a.split = g.split;
  a.groups = g.groups;
  a.trace = g_trace.load();
  a.trace_cap = a.trace ? g_trace_cap.load() : 0;
  const bool pdl = (p.flags & MUSE_FLAG_PDL) != 0;
  switch (g.mt) {
    case 1: return launch_gemv_tiles_qw<1>(a, g, pdl, st);
    case 2: return launch_gemv_tiles_qw<2>(a, g, pdl, st);
    default: return launch_gemv_tiles_qw<4>(a, g, pdl, st);
  }
}

int run_skinny(bool twelve, const void* w, const MuseEnc12* enc, const void* x, void* y, int64_t m, int64_t n,
               int64_t k, const MusePlan& p, void* scratch, int64_t scratch_bytes, cudaStream_t st) {
  SnShape sh;
  if (int rc = sn_shape(twelve, m, n, k, p, &sh)) return rc;
  const char* name = twelve ? "tc_12b" : "tc_skinny";
  if (!scratch || scratch_bytes < sh.scratch)
    return fail(MUSE_ERR_CAPACITY, "%s: needs %lld bytes of zeroed scratch (got %lld)", name, (long long)sh.scratch,
                (long long)(scratch ? scratch_bytes : 0));
  if (reinterpret_cast<uintptr_t>(scratch) & 255u) return fail(MUSE_ERR_ALIGN, "%s: scratch must be 256-byte aligned", name);
  CUtensorMap tmx;
  if (int rc = make_map(&tmx, x, m, k, sh.bnt)) return rc;
  muse::SnArgs a;
  a.w = static_cast<const uint8_t*>(w);
  a.esc_ptr = twelve ? enc->esc_ptr : nullptr;
  a.esc_val = twelve ? enc->esc_val : nullptr;
  a.y = static_cast<uint16_t*>(y);
  a.counters = static_cast<int*>(scratch);
  a.partials = reinterpret_cast<float*>(static_cast<uint8_t*>(scratch) + kCounterBytes);
  a.M = static_cast<int>(m);
  a.N = static_cast<int>(n);
  a.stages = sh.stages;
  a.rtiles = sh.rtiles;
  a.rpairs = sh.rpairs;
  a.nkb = sh.nkb;
  a.ttiles = sh.ttiles;
  a.units = sh.units;
  a.smax = sh.smax;
  a.y_vec = (n % 8 == 0 && aligned16(y)) ? 1 : 0;
  a.trace = g_trace.load();
  a.trace_cap = a.trace ? g_trace_cap.load() : 0;
  const bool pdl = (p.flags & MUSE_FLAG_PDL) != 0;
  if (twelve) {
    switch (sh.bnt) {
      case 16: return launch_sn_t<true, 16>(tmx, a, sh.g, pdl, st);
      case 32: return launch_sn_t<true, 32>(tmx, a, sh.g, pdl, st);
      case 64: return launch_sn_t<true, 64>(tmx, a, sh.g, pdl, st);
      default: return launch_sn_t<true, 128>(tmx, a, sh.g, pdl, st);
    }
  }
  switch (sh.bnt) {
    case 16: return launch_sn_t<false, 16>(tmx, a, sh.g, pdl, st);
    case 32: return launch_sn_t<false, 32>(tmx, a, sh.g, pdl, st);
    case 64: return launch_sn_t<false, 64>(tmx, a, sh.g, pdl, st);
    default: return launch_sn_t<false, 128>(tmx, a, sh.g, pdl, st);
  }
}

}  // namespace

extern "C" {

const char* muse_version(void) { return MUSE_VERSION_STRING; }

const char* muse_last_error(void) { return muse::error_state().msg; }

int muse_sm_count(int* out) {
  muse::clear_error();
  if (!out) return fail(MUSE_ERR_INVALID, "sm_count: null output");
  DeviceInfo* d;
  if (int rc = device_info(&d)) return rc;
  *out = d->sms;
  return MUSE_OK;
}

int muse_device_error(int* code, void* stream) {
  muse::clear_error();
  if (!code) return fail(MUSE_ERR_INVALID, "device_error: null output");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  unsigned int v = 0, zero = 0;
  cudaError_t e = cudaMemcpyFromSymbolAsync(&v, muse::g_dev_error, sizeof(v), 0, cudaMemcpyDeviceToHost, st);
  if (e == cudaSuccess) e = cudaMemcpyToSymbolAsync(muse::g_dev_error, &zero, sizeof(zero), 0, cudaMemcpyHostToDevice, st);
  if (e == cudaSuccess) e = cudaStreamSynchronize(st);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "device_error: %s", cudaGetErrorString(e));
  *code = static_cast<int>(v);
  if (v) return fail(MUSE_ERR_TIMEOUT, "device error word set (device code 0x%x: a bounded wait expired, or 0x501 an "
                                        "escape of the device encoder outside its buffer)", v);
  return MUSE_OK;
}

int muse_plan_default(int64_t m, int64_t n, int64_t k, int weights, MusePlan* out) {
  muse::clear_error();
  if (!out) return fail(MUSE_ERR_INVALID, "plan_default: null output");
  if (m < 1 || n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "plan_default: non-positive size");
  if (weights < MUSE_WEIGHTS_ROW_MAJOR || weights > MUSE_WEIGHTS_F32)
    return fail(MUSE_ERR_INVALID, "plan_default: weights must be one of MUSE_WEIGHTS_*");
  DeviceInfo* d;
  int sms = 148;
  if (device_info(&d) == MUSE_OK) sms = d->sms;
  muse::clear_error();
  std::memset(out, 0, sizeof(*out));
  if (weights == MUSE_WEIGHTS_12B) {
    out->kernel = MUSE_KERNEL_GEMV_12B;
    out->warps = 16;
    return m <= 8 ? MUSE_OK : fail(MUSE_ERR_SHAPE, "plan_default: 12-bit weights serve M <= 8");
  }
  if (weights == MUSE_WEIGHTS_F32) {
    // The router (measured on a B200): FP32 on CUDA cores up to 16 tokens (6-8.5 us against 11.4 us
    // for the tensor cores); above, the hi | lo tiles with 16-token tiles and K split so that the
    // grid is about 256 CTAs (at most 16 ways).
    if (m <= 16) {
      out->kernel = MUSE_KERNEL_F32_GEMV;
      return MUSE_OK;
    }
    out->kernel = MUSE_KERNEL_TC_TILE;
    out->tile_n = 16;
    out->stages = 6;
    const int64_t tiles = ((n + 127) / 128) * ((m + 15) / 16);
    const int64_t split = std::max<int64_t>(1, std::min<int64_t>({16, 256 / tiles, (2 * k) / 64}));
    out->split = static_cast<int>(split);
    if (split > 1) out->flags = MUSE_FLAG_GLOBAL_SPLIT;
    return MUSE_OK;
  }
  if (weights == MUSE_WEIGHTS_12B_TILES) {
    // Stream-K over the 12-bit blocks on the tensor cores: one CTA an SM with a deep ring.
    if (k % 512 || k > 65536) return fail(MUSE_ERR_SHAPE, "plan_default: 12-bit tiles need K %% 512 == 0, K <= 65536");
    if (m <= 4) {  // few tokens: CUDA cores decode in registers (gemv12t.cuh)
      out->kernel = MUSE_KERNEL_GEMV_12T;
      out->stages = 3;
      return MUSE_OK;
    }
    int bnt = 16;
    while (bnt < m && bnt < 128) bnt *= 2;
    out->kernel = MUSE_KERNEL_TC_12B;
    out->tile_n = bnt;
    out->ctas = sms;
    return MUSE_OK;
  }
  if (m > 256) {
    if (weights != MUSE_WEIGHTS_TILES) return fail(MUSE_ERR_SHAPE, "plan_default: M > 256 needs packed tiles");
    // The wide-tile pair GEMM (256 x 512) moves a quarter fewer operand bytes a FLOP than the
    // 256 x 256 one and measured about 7 % faster per tile under the power cap, but has half as many
    // tiles: take it unless its last wave of CTA pairs leaves more of the GPU idle than that gains
    // (measured at 8192 x {57344, 28672, 14336, 7168} x 8192 and 4096 x 10240 x 8192: the rule picks
    // the faster kernel at each).
    const int64_t pairs = std::max(1, sms / 2), mt = (m + 255) / 256;
    auto wave_eff = [&](int64_t tiles) {
      const int64_t waves = (tiles + pairs - 1) / pairs;
      return static_cast<double>(tiles) / static_cast<double>(waves * pairs);
    };
    const double eff2 = wave_eff(mt * ((n + 255) / 256)), effw = wave_eff(mt * ((n + 511) / 512));
    out->kernel = effw * 1.07 > eff2 ? MUSE_KERNEL_TC_WIDE : MUSE_KERNEL_TC_GEMM2;
    return MUSE_OK;
  }
  int bnt = 16;
  while (bnt < m && bnt < 256) bnt *= 2;
  if (weights == MUSE_WEIGHTS_TILES && m <= 2) {
    // One or two tokens: the register-streaming GEMV, 8 adjacent quads (4 KB) a warp, 4 warps a CTA
    // (measured on a B200 ahead of every tensor-core plan at M <= 2 on every swept shape), when x fits
    // its shared memory.
    out->kernel = MUSE_KERNEL_GEMV_TILES;
    out->warps = 4;
    out->chunk = 8;
    GtShape g;
    if (gt_shape(m, n, k, *out, &g) == MUSE_OK) return MUSE_OK;
    muse::clear_error();
    std::memset(out, 0, sizeof(*out));
  }
  if (weights == MUSE_WEIGHTS_TILES && m <= 128) {
    // Stream-K: every SM streams the same share of W in one wave.
    out->kernel = MUSE_KERNEL_TC_STREAMK;
    out->tile_n = bnt;
    out->stages = 4;
    out->ctas = bnt <= 64 ? 2 * sms : sms;
    return MUSE_OK;
  }
  if (weights == MUSE_WEIGHTS_ROW_MAJOR && m <= 4 && k % 256 == 0) {
    out->kernel = MUSE_KERNEL_GEMV_BF16;
    out->warps = 16;
    return MUSE_OK;
  }
  out->kernel = MUSE_KERNEL_TC_TILE;
  out->tile_n = bnt;
  const int64_t tiles = ((n + 127) / 128) * ((m + bnt - 1) / bnt);
  const int64_t nkb = (k + 63) / 64;
  int64_t split = tiles >= sms ? 1 : sms / tiles;
  split = std::max<int64_t>(1, std::min<int64_t>({split, 8, nkb}));
  out->split = static_cast<int>(split);
  if (split > 1 && weights == MUSE_WEIGHTS_TILES) out->flags = MUSE_FLAG_GLOBAL_SPLIT;
  return MUSE_OK;
}

int muse_set_trace(void* records, int64_t capacity) {
  muse::clear_error();
  if (records && capacity < 1) return fail(MUSE_ERR_INVALID, "set_trace: capacity must be positive");
  if (records && (reinterpret_cast<uintptr_t>(records) & 15u)) return fail(MUSE_ERR_ALIGN, "set_trace: 16-byte alignment");
  g_trace_cap.store(records ? static_cast<int>(std::min<int64_t>(capacity, 1 << 30)) : 0);
  g_trace.store(static_cast<muse::TraceRec*>(records));
  return MUSE_OK;
}

int muse_stream_read(const void* src, int64_t bytes, int64_t chunk, int stages, int ctas, unsigned int* count,
                     void* stream) {
  muse::clear_error();
  if (!src || !count) return fail(MUSE_ERR_INVALID, "stream_read: null pointer");
  if (bytes < 16 || chunk < 16 || bytes % 16 || chunk % 16 || chunk > (1 << 20))
    return fail(MUSE_ERR_SHAPE, "stream_read: bytes and chunk must be positive multiples of 16 (chunk <= 1 MiB)");
  if (!aligned16(src) || (reinterpret_cast<uintptr_t>(count) & 3u))
    return fail(MUSE_ERR_ALIGN, "stream_read: src 16-byte and count 4-byte aligned");
  DeviceInfo* d;
  if (int rc = device_info(&d)) return rc;
  if (stages < 1) return fail(MUSE_ERR_PLAN, "stream_read: stages must be positive");
  const int smem = muse::read_floor_smem(static_cast<int>(chunk), stages);
  if (smem > std::min(kSmemLimit, d->smem_optin))
    return fail(MUSE_ERR_PLAN, "stream_read: %d stages of %lld bytes do not fit shared memory", stages, (long long)chunk);
  const int64_t nch = (bytes + chunk - 1) / chunk;
  const int grid = static_cast<int>(std::min<int64_t>(nch, ctas > 0 ? ctas : d->sms));
  static bool configured[kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  if (!configured[dev]) {
    const cudaError_t e = cudaFuncSetAttribute(muse::stream_read_kernel, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                               kSmemLimit);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(stream_read): %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  muse::ReadArgs a;
  a.src = static_cast<const uint8_t*>(src);
  a.bytes = bytes;
  a.chunk = static_cast<int>(chunk);
  a.stages = stages;
  a.count = count;
  muse::stream_read_kernel<<<grid, 32, smem, static_cast<cudaStream_t>(stream)>>>(a);
  return launch_error("stream_read launch");
}

static int check_rows_groups(const char* what, int64_t n, int64_t k, int groups) {
  if (n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "%s: non-positive size", what);
  if (n > (int64_t(1) << 24) || k > (int64_t(1) << 24)) return fail(MUSE_ERR_SHAPE, "%s: dimension too large", what);
  const int64_t units16 = (n + 15) / 16;
  if (groups < 1 || groups > units16)
    return fail(MUSE_ERR_INVALID, "%s: windows must be 1 .. ceil(N / 16) = %lld (got %d)", what, (long long)units16, groups);
  if ((units16 + groups - 1) / groups * 16 > muse::kRwMaxRows)
    return fail(MUSE_ERR_PLAN, "%s: %d windows leave more than %d rows a window", what, groups, muse::kRwMaxRows);
  return MUSE_OK;
}

int muse_rows_groups(int64_t m, int64_t n, int64_t k, const MusePlan* plan, int* groups) {
  muse::clear_error();
  if (!plan || !groups) return fail(MUSE_ERR_INVALID, "rows_groups: null pointer");
  if (m < 1 || n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "rows_groups: non-positive size");
  if (plan->kernel != MUSE_KERNEL_TC_ROWS) return fail(MUSE_ERR_PLAN, "rows_groups: plan kernel must be TC_ROWS");
  RwShape sh;
  if (int rc = rw_shape(m, n, k, *plan, &sh)) return rc;
  *groups = sh.groups;
  return MUSE_OK;
}

int muse_rows_bytes(int64_t n, int64_t k, int groups, int64_t* bytes) {
  muse::clear_error();
  if (!bytes) return fail(MUSE_ERR_INVALID, "rows_bytes: null output");
  if (int rc = check_rows_groups("rows_bytes", n, k, groups)) return rc;
  *bytes = ((n + 15) / 16) * 16 * ((k + 63) / 64) * 128;
  return MUSE_OK;
}

int muse_pack_rows(const void* w, void* out, int64_t n, int64_t k, int groups, void* stream) {
  muse::clear_error();
  if (!w || !out) return fail(MUSE_ERR_INVALID, "pack_rows: null pointer");
  if (int rc = check_rows_groups("pack_rows", n, k, groups)) return rc;
  if (!aligned16(w) || !aligned16(out) || k % 8) return fail(MUSE_ERR_ALIGN, "pack_rows: 16-byte alignment and K %% 8 == 0 needed");
  const int64_t units16 = (n + 15) / 16, nkb = (k + 63) / 64;
  const long long chunks = static_cast<long long>(units16) * 16 * nkb * 8;
  const int threads = 256;
  const long long blocks = std::min<long long>((chunks + threads - 1) / threads, 148LL * 64);
  muse::pack_rows_kernel<<<static_cast<unsigned>(blocks), threads, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(w), static_cast<uint4*>(out), static_cast<int>(n), static_cast<int>(k),
      static_cast<int>(nkb), static_cast<int>(units16), groups, chunks);
  return launch_error("pack_rows launch");
}

int muse_proj_bf16_rows(const void* x, const void* wrows, void* y, int64_t m, int64_t n, int64_t k, const MusePlan* plan,
                        void* stream) {
  muse::clear_error();
  if (!x || !wrows || !y || !plan) return fail(MUSE_ERR_INVALID, "proj_bf16_rows: null pointer");
  if (m < 1 || n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "proj_bf16_rows: non-positive size");
  if (!aligned16(x) || !aligned16(wrows) || (reinterpret_cast<uintptr_t>(y) & 1u) || (k * 2) % 16)
    return fail(MUSE_ERR_ALIGN, "proj_bf16_rows: x and wrows 16-byte aligned, y 2-byte aligned, K %% 8 == 0");
  if (plan->kernel != MUSE_KERNEL_TC_ROWS) return fail(MUSE_ERR_PLAN, "proj_bf16_rows: plan kernel must be TC_ROWS");
  return run_rows(x, nullptr, wrows, y, m, n, k, *plan, static_cast<cudaStream_t>(stream));
}

int muse_tiles_bytes(int64_t n, int64_t k, int64_t* bytes) {
  muse::clear_error();
  if (!bytes) return fail(MUSE_ERR_INVALID, "tiles_bytes: null output");
  if (n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "tiles_bytes: non-positive size");
  *bytes = ((n + 127) / 128) * ((k + 63) / 64) * int64_t(muse::kTcABytes);
  return MUSE_OK;
}

int muse_pack_tiles(const void* w, void* tiles, int64_t n, int64_t k, void* stream) {
  muse::clear_error();
  if (!w || !tiles) return fail(MUSE_ERR_INVALID, "pack_tiles: null pointer");
  if (n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "pack_tiles: non-positive size");
  if (!aligned16(w) || !aligned16(tiles) || k % 8) return fail(MUSE_ERR_ALIGN, "pack_tiles: 16-byte alignment and K %% 8 == 0 needed");
  if (n > (int64_t(1) << 24) || k > (int64_t(1) << 24)) return fail(MUSE_ERR_SHAPE, "pack_tiles: dimension too large");
  const int nkb = static_cast<int>((k + 63) / 64);
  const long long chunks = ((n + 127) / 128) * static_cast<long long>(nkb) * 1024;
  const int blocks = static_cast<int>(std::min<long long>((chunks + 255) / 256, 148 * 32));
  muse::pack_tiles_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(w), static_cast<uint4*>(tiles), static_cast<int>(n), static_cast<int>(k), nkb, chunks);
  return launch_error("pack_tiles launch");
}

int muse_scratch_bytes(int64_t m, int64_t n, int64_t k, const MusePlan* plan, int64_t* bytes) {
  muse::clear_error();
  if (!plan || !bytes) return fail(MUSE_ERR_INVALID, "scratch_bytes: null pointer");
  if (m < 1 || n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "scratch_bytes: non-positive size");
  *bytes = 0;
  if (plan->kernel == MUSE_KERNEL_TC_STREAMK) {
    SkShape sk;
    if (int rc = sk_shape(m, n, k, *plan, &sk)) return rc;
    *bytes = sk.scratch;
    return MUSE_OK;
  }
  if (plan->kernel == MUSE_KERNEL_GEMV_12T) {
    G12Shape g;
    if (int rc = g12_shape(m, n, k, *plan, &g)) return rc;
    *bytes = g.scratch;
    return MUSE_OK;
  }
  if (plan->kernel == MUSE_KERNEL_TC_12B || plan->kernel == MUSE_KERNEL_TC_SKINNY) {
    SnShape sn;
    if (int rc = sn_shape(plan->kernel == MUSE_KERNEL_TC_12B, m, n, k, *plan, &sn)) return rc;
    *bytes = sn.scratch;
    return MUSE_OK;
  }
  if (plan->kernel == MUSE_KERNEL_TC_GEMM2) {
    if (plan->flags & (MUSE_FLAG_STREAMK | MUSE_FLAG_SK_TAIL)) {
      DeviceInfo* d;
      int sms = 148;
      if (device_info(&d) == MUSE_OK) sms = d->sms;
      muse::clear_error();
      *bytes = g2_sk_scratch(m, n, k, sms, (plan->flags & MUSE_FLAG_SK_TAIL) != 0);
    }
    return MUSE_OK;
  }
  if (plan->kernel == MUSE_KERNEL_TC_PAIRK) {
    if (plan->flags & MUSE_FLAG_STREAMK) {
      DeviceInfo* d;
      int sms = 148;
      if (device_info(&d) == MUSE_OK) sms = d->sms;
      muse::clear_error();
      PsShape ps;
      if (int rc = ps_shape(m, n, k, *plan, std::max(1, sms / 2), &ps)) return rc;
      *bytes = ps.scratch;
      return MUSE_OK;
    }
    PkShape pk;
    if (int rc = pk_shape(m, n, k, *plan, &pk)) return rc;
    *bytes = pk.scratch;
    return MUSE_OK;
  }
  if (plan->kernel == MUSE_KERNEL_TC_ROWS) {  // no scratch: checks the plan only
    RwShape rw;
    return rw_shape(m, n, k, *plan, &rw);
  }
  if (plan->kernel == MUSE_KERNEL_GEMV_TILES) {  // no scratch: checks the plan only
    GtShape g;
    return gt_shape(m, n, k, *plan, &g);
  }
  if (plan->kernel != MUSE_KERNEL_TC_TILE) return MUSE_OK;
  TcShape sh;
  if (int rc = tc_shape(m, n, k, *plan, &sh)) return rc;
  *bytes = tc_scratch_bytes(sh);
  return MUSE_OK;
}

int muse_proj_bf16_tiles(const void* x, const void* tiles, void* y, int64_t m, int64_t n, int64_t k,
                         const MusePlan* plan, void* scratch, int64_t scratch_bytes, void* stream) {
  muse::clear_error();
  if (!x || !tiles || !y || !plan) return fail(MUSE_ERR_INVALID, "proj_bf16_tiles: null pointer");
  if (m < 1 || n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "proj_bf16_tiles: non-positive size");
  if (!aligned16(x) || !aligned16(tiles) || (reinterpret_cast<uintptr_t>(y) & 1u) || (k * 2) % 16)
    return fail(MUSE_ERR_ALIGN, "proj_bf16_tiles: x and tiles 16-byte aligned, y 2-byte aligned, K %% 8 == 0");
  if (plan->kernel == MUSE_KERNEL_TC_STREAMK)
    return run_streamk(x, tiles, y, m, n, k, *plan, scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
  if (plan->kernel == MUSE_KERNEL_TC_SKINNY)
    return run_skinny(false, tiles, nullptr, x, y, m, n, k, *plan, scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
  if (plan->kernel == MUSE_KERNEL_TC_GEMM) return run_gemm(x, tiles, y, m, n, k, *plan, static_cast<cudaStream_t>(stream));
  if (plan->kernel == MUSE_KERNEL_TC_GEMM2)
    return run_gemm2(x, tiles, y, m, n, k, *plan, static_cast<cudaStream_t>(stream), nullptr, scratch, scratch_bytes);
  if (plan->kernel == MUSE_KERNEL_TC_ROWS)
    return run_rows(x, tiles, nullptr, y, m, n, k, *plan, static_cast<cudaStream_t>(stream));
  if (plan->kernel == MUSE_KERNEL_TC_WIDE) return run_wide(x, tiles, y, m, n, k, *plan, static_cast<cudaStream_t>(stream));
  if (plan->kernel == MUSE_KERNEL_GEMV_TILES) return run_gemv_tiles(x, tiles, y, m, n, k, *plan, static_cast<cudaStream_t>(stream));
  if (plan->kernel == MUSE_KERNEL_TC_PAIRK && (plan->flags & MUSE_FLAG_STREAMK))
    return run_pairsk(x, tiles, y, m, n, k, *plan, scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
  if (plan->kernel == MUSE_KERNEL_TC_PAIRK)
    return run_pairk(x, tiles, y, m, n, k, *plan, scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
  if (plan->kernel != MUSE_KERNEL_TC_TILE)
    return fail(MUSE_ERR_PLAN, "proj_bf16_tiles: plan kernel must be TC_TILE, TC_STREAMK, TC_SKINNY, TC_GEMM, TC_GEMM2, "
                               "TC_ROWS, TC_WIDE, TC_PAIRK or GEMV_TILES");
  return run_tc_tile(x, nullptr, tiles, y, m, n, k, *plan, scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
}

int muse_proj_bf16(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, const MusePlan* plan,
                   void* scratch, int64_t scratch_bytes, void* stream) {
  muse::clear_error();
  if (!x || !w || !y || !plan) return fail(MUSE_ERR_INVALID, "proj_bf16: null pointer");
  if (m < 1 || n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "proj_bf16: non-positive size");
  if (!aligned16(x) || !aligned16(w) || !aligned16(y) || (k * 2) % 16)
    return fail(MUSE_ERR_ALIGN, "proj_bf16: x, W, y must be 16-byte aligned and K a multiple of 8");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (plan->kernel == MUSE_KERNEL_GEMV_BF16) {
    muse::GemvArgs a = {};
    a.wstream = static_cast<const uint8_t*>(w);
    a.x = static_cast<const uint16_t*>(x);
    a.y = static_cast<uint16_t*>(y);
    a.n = static_cast<int>(n);
    a.k = static_cast<int>(k);
    int grid, smem, warps;
    if (int rc = plan_gemv(false, m, n, k, *plan, a, &grid, &smem, &warps)) return rc;
    return launch_gemv<false>(a, static_cast<int>(m), warps, grid, smem, (plan->flags & MUSE_FLAG_PDL) != 0, st);
  }
  if (plan->kernel == MUSE_KERNEL_TC_TILE) return run_tc_tile(x, w, nullptr, y, m, n, k, *plan, scratch, scratch_bytes, st);
  return fail(MUSE_ERR_PLAN, "proj_bf16: kernel %d does not take BF16 weights", plan->kernel);
}

int muse_proj_12b(const MuseEnc12* enc, const void* x, void* y, int64_t m, const MusePlan* plan, void* stream) {
  muse::clear_error();
  if (!enc || !x || !y || !plan || !enc->planes || !enc->bases || !enc->esc_ptr || (enc->n_esc > 0 && !enc->esc_val))
    return fail(MUSE_ERR_INVALID, "proj_12b: null pointer");
  if (m < 1 || enc->n < 1 || enc->k < 1) return fail(MUSE_ERR_INVALID, "proj_12b: non-positive size");
  if (!aligned16(x) || !aligned16(enc->planes)) return fail(MUSE_ERR_ALIGN, "proj_12b: x and planes must be 16-byte aligned");
  if ((reinterpret_cast<uintptr_t>(y) & 1u) != 0) return fail(MUSE_ERR_ALIGN, "proj_12b: y must be 2-byte aligned");
  if (plan->kernel != MUSE_KERNEL_GEMV_12B) return fail(MUSE_ERR_PLAN, "proj_12b: plan kernel must be GEMV_12B");
  muse::GemvArgs a = {};
  a.wstream = enc->planes;
  a.x = static_cast<const uint16_t*>(x);
  a.y = static_cast<uint16_t*>(y);
  a.bases = enc->bases;
  a.esc_ptr = enc->esc_ptr;
  a.esc_val = enc->esc_val;
  a.n = static_cast<int>(enc->n);
  a.k = static_cast<int>(enc->k);
  int grid, smem, warps;
  if (int rc = plan_gemv(true, m, enc->n, enc->k, *plan, a, &grid, &smem, &warps)) return rc;
  return launch_gemv<true>(a, static_cast<int>(m), warps, grid, smem, (plan->flags & MUSE_FLAG_PDL) != 0,
                           static_cast<cudaStream_t>(stream));
}

int muse_tiles12_bytes(int64_t n, int64_t k, int64_t* bytes) {
  muse::clear_error();
  if (!bytes) return fail(MUSE_ERR_INVALID, "tiles12_bytes: null output");
  if (n < 1 || k < 512) return fail(MUSE_ERR_INVALID, "tiles12_bytes: need N >= 1 and K >= 512");
  if (k % 512 || k > 65536) return fail(MUSE_ERR_SHAPE, "tiles12_bytes: need K %% 512 == 0 and K <= 65536");
  *bytes = ((n + 127) / 128) * (k / 64) * int64_t(muse::kT12Block);
  return MUSE_OK;
}

int muse_pack_tiles12(const MuseEnc12* enc, void* tiles12, void* stream) {
  muse::clear_error();
  if (!enc || !enc->planes || !enc->bases || !enc->esc_ptr || (enc->n_esc > 0 && !enc->esc_val) || !tiles12)
    return fail(MUSE_ERR_INVALID, "pack_tiles12: null pointer");
  if (enc->n < 1 || enc->k < 512) return fail(MUSE_ERR_INVALID, "pack_tiles12: need N >= 1 and K >= 512");
  if (enc->k % 512 || enc->k > 65536 || enc->n > (int64_t(1) << 24))
    return fail(MUSE_ERR_SHAPE, "pack_tiles12: need K %% 512 == 0, K <= 65536 and N <= 2^24");
  if (!aligned16(enc->planes) || !aligned16(tiles12)) return fail(MUSE_ERR_ALIGN, "pack_tiles12: 16-byte alignment needed");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const int nkb = static_cast<int>(enc->k / 64);
  const long long blocks12 = ((enc->n + 127) / 128) * static_cast<long long>(nkb);
  const long long chunks = blocks12 * (muse::kT12Raw / 16);
  const int grid = static_cast<int>(std::min<long long>((chunks + 255) / 256, 148 * 32));
  muse::pack_tiles12_kernel<<<grid, 256, 0, st>>>(enc->planes, static_cast<uint8_t*>(tiles12), static_cast<int>(enc->n),
                                                  static_cast<int>(enc->k), nkb, chunks);
  if (int rc = launch_error("pack_tiles12 launch")) return rc;
  if (blocks12 > 0x7FFFFFFFll) return fail(MUSE_ERR_SHAPE, "pack_tiles12: too many blocks");
  muse::pack_escapes12_kernel<<<static_cast<unsigned>(blocks12), 128, 0, st>>>(
      enc->bases, enc->esc_ptr, enc->esc_val, static_cast<uint8_t*>(tiles12), static_cast<int>(enc->n),
      static_cast<int>(enc->k), nkb);
  return launch_error("pack_escapes12 launch");
}

// Shape and pointer checks shared by the two steps of the device encoder.
static int check_encode12_device(const char* what, const void* w, int64_t n, int64_t k) {
  if (!w) return fail(MUSE_ERR_INVALID, "%s: null pointer", what);
  if (n < 1 || k < 512) return fail(MUSE_ERR_INVALID, "%s: need N >= 1 and K >= 512", what);
  if (k % 512 || k > 65536 || n * k >= (int64_t(1) << 31))
    return fail(MUSE_ERR_SHAPE, "%s: need K %% 512 == 0, K <= 65536 and N * K < 2^31", what);
  if (!aligned16(w)) return fail(MUSE_ERR_ALIGN, "%s: W must be 16-byte aligned", what);
  return MUSE_OK;
}

int muse_encode12_device(const void* w, int64_t n, int64_t k, uint8_t* planes, uint8_t* bases, int32_t* esc_ptr,
                         void* stream) {
  muse::clear_error();
  if (int rc = check_encode12_device("encode12_device", w, n, k)) return rc;
  if (!planes || !bases || !esc_ptr) return fail(MUSE_ERR_INVALID, "encode12_device: null pointer");
  if (reinterpret_cast<uintptr_t>(planes) & 7u) return fail(MUSE_ERR_ALIGN, "encode12_device: planes must be 8-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  const auto* wp = static_cast<const uint16_t*>(w);
  const int64_t tiles = (n + muse::kEnc12Tile - 1) / muse::kEnc12Tile;  // <= 2^31 / 512 / 128: fits grid.y
  muse::enc12_bases_kernel<<<dim3(static_cast<unsigned>(k / muse::kEnc12Tile), static_cast<unsigned>(tiles)), 128, 0,
                             st>>>(wp, n, k, bases);
  if (int rc = launch_error("encode12_device bases launch")) return rc;
  const unsigned rows = static_cast<unsigned>((n + muse::kEnc12RowsPerCta - 1) / muse::kEnc12RowsPerCta);
  muse::enc12_planes_kernel<<<rows, 32 * muse::kEnc12RowsPerCta, 0, st>>>(wp, n, k, bases, planes, esc_ptr);
  if (int rc = launch_error("encode12_device planes launch")) return rc;
  muse::enc12_scan_kernel<<<1, muse::kEnc12ScanThreads, 0, st>>>(esc_ptr, n);
  return launch_error("encode12_device scan launch");
}

int muse_encode12_device_escapes(const void* w, int64_t n, int64_t k, const uint8_t* bases, const int32_t* esc_ptr,
                                 uint32_t* esc_val, int64_t esc_cap, void* stream) {
  muse::clear_error();
  if (int rc = check_encode12_device("encode12_device_escapes", w, n, k)) return rc;
  if (!bases || !esc_ptr || (esc_cap > 0 && !esc_val) || esc_cap < 0)
    return fail(MUSE_ERR_INVALID, "encode12_device_escapes: null pointer or negative capacity");
  const unsigned rows = static_cast<unsigned>((n + muse::kEnc12RowsPerCta - 1) / muse::kEnc12RowsPerCta);
  muse::enc12_escapes_kernel<<<rows, 32 * muse::kEnc12RowsPerCta, 0, static_cast<cudaStream_t>(stream)>>>(
      static_cast<const uint16_t*>(w), n, k, bases, esc_ptr, esc_val, esc_cap);
  return launch_error("encode12_device_escapes launch");
}

int muse_proj_12b_tiles(const MuseEnc12* enc, const void* tiles12, const void* x, void* y, int64_t m,
                        const MusePlan* plan, void* scratch, int64_t scratch_bytes, void* stream) {
  muse::clear_error();
  if (!enc || !tiles12 || !x || !y || !plan || !enc->esc_ptr || (enc->n_esc > 0 && !enc->esc_val))
    return fail(MUSE_ERR_INVALID, "proj_12b_tiles: null pointer");
  if (m < 1 || enc->n < 1 || enc->k < 1) return fail(MUSE_ERR_INVALID, "proj_12b_tiles: non-positive size");
  if (!aligned16(x) || !aligned16(tiles12) || (reinterpret_cast<uintptr_t>(y) & 1u))
    return fail(MUSE_ERR_ALIGN, "proj_12b_tiles: x and tiles 16-byte aligned, y 2-byte aligned");
  if (plan->kernel == MUSE_KERNEL_GEMV_12T)
    return run_gemv12t(tiles12, enc, x, y, m, *plan, scratch, scratch_bytes, static_cast<cudaStream_t>(stream));
  if (plan->kernel != MUSE_KERNEL_TC_12B)
    return fail(MUSE_ERR_PLAN, "proj_12b_tiles: plan kernel must be TC_12B or GEMV_12T");
  return run_skinny(true, tiles12, enc, x, y, m, enc->n, enc->k, *plan, scratch, scratch_bytes,
                    static_cast<cudaStream_t>(stream));
}

int muse_proj_bf16_tiles_f32(const void* x, const void* tiles, float* y, int64_t m, int64_t n, int64_t k,
                             const MusePlan* plan, void* scratch, int64_t scratch_bytes, void* stream) {
  muse::clear_error();
  if (!x || !tiles || !y || !plan) return fail(MUSE_ERR_INVALID, "proj_bf16_tiles_f32: null pointer");
  if (m < 1 || n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "proj_bf16_tiles_f32: non-positive size");
  if (!aligned16(x) || !aligned16(tiles) || (reinterpret_cast<uintptr_t>(y) & 3u) || (k * 2) % 16)
    return fail(MUSE_ERR_ALIGN, "proj_bf16_tiles_f32: x and tiles 16-byte aligned, y 4-byte aligned, K %% 8 == 0");
  if (plan->kernel != MUSE_KERNEL_TC_TILE) return fail(MUSE_ERR_PLAN, "proj_bf16_tiles_f32: plan kernel must be TC_TILE");
  return run_tc_tile(x, nullptr, tiles, nullptr, m, n, k, *plan, scratch, scratch_bytes,
                     static_cast<cudaStream_t>(stream), y, 0);
}

int muse_router_tiles_bytes(int64_t n, int64_t k, int64_t* bytes) {
  muse::clear_error();
  if (!bytes) return fail(MUSE_ERR_INVALID, "router_tiles_bytes: null output");
  if (n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "router_tiles_bytes: non-positive size");
  if (k % 64) return fail(MUSE_ERR_SHAPE, "router_tiles_bytes: K must be a multiple of 64");
  *bytes = ((n + 127) / 128) * ((2 * k) / 64) * int64_t(muse::kTcABytes);
  return MUSE_OK;
}

int muse_pack_router(const float* w, void* tiles, int64_t n, int64_t k, void* stream) {
  muse::clear_error();
  if (!w || !tiles) return fail(MUSE_ERR_INVALID, "pack_router: null pointer");
  if (n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "pack_router: non-positive size");
  if (k % 64) return fail(MUSE_ERR_SHAPE, "pack_router: K must be a multiple of 64");
  if (!aligned16(w) || !aligned16(tiles)) return fail(MUSE_ERR_ALIGN, "pack_router: 16-byte alignment needed");
  if (n > (int64_t(1) << 24) || k > (int64_t(1) << 23)) return fail(MUSE_ERR_SHAPE, "pack_router: dimension too large");
  const int nkb = static_cast<int>((2 * k) / 64);
  const long long chunks = ((n + 127) / 128) * static_cast<long long>(nkb) * 1024;
  const int blocks = static_cast<int>(std::min<long long>((chunks + 255) / 256, 148 * 32));
  muse::pack_router_kernel<<<blocks, 256, 0, static_cast<cudaStream_t>(stream)>>>(
      w, static_cast<uint4*>(tiles), static_cast<int>(n), static_cast<int>(k), nkb, chunks);
  return launch_error("pack_router launch");
}

int muse_proj_f32(const void* x, const float* w, const void* tiles, float* y, int64_t m, int64_t n, int64_t k,
                  const MusePlan* plan, void* scratch, int64_t scratch_bytes, void* stream) {
  muse::clear_error();
  if (!x || !y || !plan) return fail(MUSE_ERR_INVALID, "proj_f32: null pointer");
  if (m < 1 || n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "proj_f32: non-positive size");
  if (k % 64) return fail(MUSE_ERR_SHAPE, "proj_f32: K must be a multiple of 64");
  if (!aligned16(x) || (reinterpret_cast<uintptr_t>(y) & 3u))
    return fail(MUSE_ERR_ALIGN, "proj_f32: x 16-byte aligned, y 4-byte aligned");
  cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (plan->kernel == MUSE_KERNEL_F32_GEMV) {
    if (!w) return fail(MUSE_ERR_INVALID, "proj_f32: the FP32 kernel reads W: null pointer");
    if (!aligned16(w)) return fail(MUSE_ERR_ALIGN, "proj_f32: W must be 16-byte aligned");
    if (m > 32) return fail(MUSE_ERR_SHAPE, "proj_f32: the FP32 kernel serves M <= 32 (got %lld)", (long long)m);
    if (n > 0x7FFFFFFF) return fail(MUSE_ERR_SHAPE, "proj_f32: N too large");
    const float* wf = w;
    const uint16_t* xb = static_cast<const uint16_t*>(x);
    const int mi = static_cast<int>(m), ni = static_cast<int>(n), ki = static_cast<int>(k);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>(n), 1, 1);
    cfg.blockDim = dim3(muse::kRouterThreads, 1, 1);
    cfg.stream = st;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = (plan->flags & MUSE_FLAG_PDL) ? 1 : 0;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    cudaError_t e;
    if (m <= 1) e = cudaLaunchKernelEx(&cfg, muse::router_f32_kernel<1>, wf, xb, y, mi, ni, ki);
    else if (m <= 2) e = cudaLaunchKernelEx(&cfg, muse::router_f32_kernel<2>, wf, xb, y, mi, ni, ki);
    else if (m <= 4) e = cudaLaunchKernelEx(&cfg, muse::router_f32_kernel<4>, wf, xb, y, mi, ni, ki);
    // 5..16 tokens share the 16-token instance: measured faster than an 8-token one even at M = 5.
    else if (m <= 16) e = cudaLaunchKernelEx(&cfg, muse::router_f32_kernel<16>, wf, xb, y, mi, ni, ki);
    else e = cudaLaunchKernelEx(&cfg, muse::router_f32_kernel<32>, wf, xb, y, mi, ni, ki);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "router_f32 launch: %s", cudaGetErrorString(e));
    return MUSE_OK;
  }
  if (plan->kernel != MUSE_KERNEL_TC_TILE)
    return fail(MUSE_ERR_PLAN, "proj_f32: plan kernel must be F32_GEMV or TC_TILE");
  if (!tiles) return fail(MUSE_ERR_INVALID, "proj_f32: the tensor-core path reads the hi | lo tiles: null pointer");
  if (!aligned16(tiles)) return fail(MUSE_ERR_ALIGN, "proj_f32: tiles must be 16-byte aligned");
  return run_tc_tile(x, nullptr, tiles, nullptr, m, n, 2 * k, *plan, scratch, scratch_bytes, st, y, k);
}

// ---- all-gather fused into the epilogue: peer buffers over CUDA IPC ------------------------------

int muse_peer_ctl_bytes(int64_t* bytes) {
  muse::clear_error();
  if (!bytes) return fail(MUSE_ERR_INVALID, "peer_ctl_bytes: null output");
  *bytes = static_cast<int64_t>(sizeof(muse::PeerCtl));
  return MUSE_OK;
}

int muse_ipc_export(const void* ptr, void* handle, int64_t* offset) {
  muse::clear_error();
  if (!ptr || !handle || !offset) return fail(MUSE_ERR_INVALID, "ipc_export: null argument");
  static PFN_cuMemGetAddressRange_v3020 range_fn = nullptr;
  static std::once_flag once;
  std::call_once(once, [] {
    void* f = nullptr;
    cudaDriverEntryPointQueryResult q;
    if (cudaGetDriverEntryPoint("cuMemGetAddressRange", &f, cudaEnableDefault, &q) == cudaSuccess &&
        q == cudaDriverEntryPointSuccess)
      range_fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(f);
  });
  if (!range_fn) return fail(MUSE_ERR_CUDA, "cuMemGetAddressRange entry point not found");
  CUdeviceptr base = 0;
  size_t size = 0;
  if (range_fn(&base, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS)
    return fail(MUSE_ERR_INVALID, "ipc_export: pointer is not device memory of this process");
  cudaIpcMemHandle_t h;
  cudaError_t e = cudaIpcGetMemHandle(&h, reinterpret_cast<void*>(base));
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaIpcGetMemHandle: %s", cudaGetErrorString(e));
  static_assert(sizeof(h) == MUSE_IPC_HANDLE_BYTES, "IPC handle size");
  std::memcpy(handle, &h, sizeof(h));
  *offset = static_cast<int64_t>(reinterpret_cast<CUdeviceptr>(ptr) - base);
  return MUSE_OK;
}

int muse_ipc_open(const void* handle, int64_t offset, void** ptr) {
  muse::clear_error();
  if (!handle || !ptr || offset < 0) return fail(MUSE_ERR_INVALID, "ipc_open: bad argument");
  cudaIpcMemHandle_t h;
  std::memcpy(&h, handle, sizeof(h));
  void* base = nullptr;
  cudaError_t e = cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaIpcOpenMemHandle: %s", cudaGetErrorString(e));
  *ptr = static_cast<uint8_t*>(base) + offset;
  return MUSE_OK;
}

int muse_ipc_close(void* ptr, int64_t offset) {
  muse::clear_error();
  if (!ptr || offset < 0) return fail(MUSE_ERR_INVALID, "ipc_close: bad argument");
  cudaError_t e = cudaIpcCloseMemHandle(static_cast<uint8_t*>(ptr) - offset);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaIpcCloseMemHandle: %s", cudaGetErrorString(e));
  return MUSE_OK;
}

int muse_proj_bf16_tiles_gather(const void* x, const void* tiles, int64_t m, int64_t n, int64_t k,
                                const MuseGather* g, const MusePlan* plan, void* scratch, int64_t scratch_bytes,
                                void* stream) {
  muse::clear_error();
  if (!x || !tiles || !g || !plan) return fail(MUSE_ERR_INVALID, "proj_gather: null argument");
  if (m <= 0 || n <= 0 || k <= 0) return fail(MUSE_ERR_SHAPE, "proj_gather: m, n, k must be positive");
  if (k % 8 != 0) return fail(MUSE_ERR_SHAPE, "proj_gather: k must be a multiple of 8");
  if (!aligned16(x) || !aligned16(tiles)) return fail(MUSE_ERR_ALIGN, "proj_gather: x and tiles must be 16-byte aligned");
  if (g->world < 1 || g->world > muse::kMaxPeers || g->rank < 0 || g->rank >= g->world)
    return fail(MUSE_ERR_INVALID, "proj_gather: world must be 1..%d and 0 <= rank < world (got %d, %d)", muse::kMaxPeers,
                g->world, g->rank);
  if (g->col0 < 0 || g->ldy < g->col0 + n || g->ldy > (int64_t(1) << 24))
    return fail(MUSE_ERR_SHAPE, "proj_gather: columns col0 .. col0 + n must lie inside ldy (col0 %lld, n %lld, ldy %lld)",
                (long long)g->col0, (long long)n, (long long)g->ldy);
  if (g->ldy % 8 != 0 || g->col0 % 8 != 0 || n % 8 != 0)
    return fail(MUSE_ERR_SHAPE, "proj_gather: ldy, col0 and n must be multiples of 8");
  muse::GatherOut go;
  std::memset(&go, 0, sizeof(go));
  for (int p = 0; p < g->world; ++p) {
    if (!g->y[p] || !g->ctl[p]) return fail(MUSE_ERR_INVALID, "proj_gather: rank %d's buffer or control block is null", p);
    if (!aligned16(g->y[p])) return fail(MUSE_ERR_ALIGN, "proj_gather: rank %d's y_full must be 16-byte aligned", p);
    if (reinterpret_cast<uintptr_t>(g->ctl[p]) & 127u)
      return fail(MUSE_ERR_ALIGN, "proj_gather: rank %d's control block must be 128-byte aligned", p);
    go.y[p] = static_cast<uint16_t*>(g->y[p]);
    go.ctl[p] = static_cast<muse::PeerCtl*>(g->ctl[p]);
  }
  go.P = g->world;
  go.rank = g->rank;
  go.ldy = static_cast<int>(g->ldy);
  go.col0 = static_cast<int>(g->col0);
  const cudaStream_t st = static_cast<cudaStream_t>(stream);
  if (plan->kernel == MUSE_KERNEL_TC_GEMM2) return run_gemm2(x, tiles, nullptr, m, n, k, *plan, st, &go);
  if (plan->kernel == MUSE_KERNEL_TC_TILE) {
    if (plan->split > 1 && !(plan->flags & MUSE_FLAG_GLOBAL_SPLIT))
      return fail(MUSE_ERR_PLAN, "proj_gather: a K split must go through scratch (MUSE_FLAG_GLOBAL_SPLIT), not a cluster");
    return run_tc_tile(x, nullptr, tiles, nullptr, m, n, k, *plan, scratch, scratch_bytes, st, nullptr, 0, &go);
  }
  return fail(MUSE_ERR_PLAN, "proj_gather: the fused all-gather runs on the tc_tile or tc_gemm2 kernel (plan kernel %d)",
              plan->kernel);
}

}  // extern "C"

// ---- no-allocation entry point ----------------------------------------------------------------
//
// For callers that cannot allocate device memory themselves (an inference engine's plugin that is
// handed only its input and output buffers from the engine's own pool, or an application whose
// device memory budget is fixed when it starts): the stream-K projection with its split-K scratch
// in a fixed-size array inside this library instead of a caller buffer. The array is a
// file-scope device variable, so every GPU that loads the library holds its
// MUSE_NOALLOC_SCRATCH_BYTES until the process exits; nothing is allocated per call.

namespace {

static __device__ __align__(256) unsigned char g_noalloc_scratch[MUSE_NOALLOC_SCRATCH_BYTES];

void* g_noalloc_addr[kMaxDevices] = {};
std::mutex g_noalloc_mu;

// The array's device address on the current device. In host code `g_noalloc_scratch` is only a
// host-side stand-in for the symbol, so the address is looked up once per device, with that
// device current, and cached.
int noalloc_scratch(void** out) {
  int dev;
  if (int rc = current_device(&dev)) return rc;
  std::lock_guard<std::mutex> lock(g_noalloc_mu);
  if (!g_noalloc_addr[dev]) {
    void* p = nullptr;
    const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
    if (e != cudaSuccess || p == nullptr)
      return fail(MUSE_ERR_CUDA, "proj_bf16_tiles_noalloc: cudaGetSymbolAddress: %s",
                  e != cudaSuccess ? cudaGetErrorString(e) : "null address");
    g_noalloc_addr[dev] = p;
  }
  *out = g_noalloc_addr[dev];
  return MUSE_OK;
}

}  // namespace

extern "C" int muse_proj_bf16_tiles_noalloc(const void* x, const void* tiles, void* y, int64_t m, int64_t n, int64_t k,
                                            const MusePlan* plan, void* stream) {
  muse::clear_error();
  if (!x || !tiles || !y || !plan) return fail(MUSE_ERR_INVALID, "proj_bf16_tiles_noalloc: null pointer");
  if (m < 1 || n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "proj_bf16_tiles_noalloc: non-positive size");
  if (!aligned16(x) || !aligned16(tiles) || (reinterpret_cast<uintptr_t>(y) & 1u) || (k * 2) % 16)
    return fail(MUSE_ERR_ALIGN, "proj_bf16_tiles_noalloc: x and tiles 16-byte aligned, y 2-byte aligned, K %% 8 == 0");
  if (plan->kernel != MUSE_KERNEL_TC_STREAMK)
    return fail(MUSE_ERR_PLAN, "proj_bf16_tiles_noalloc: plan kernel must be TC_STREAMK");
  SkShape sh;
  if (int rc = sk_shape(m, n, k, *plan, &sh)) return rc;
  if (sh.scratch > MUSE_NOALLOC_SCRATCH_BYTES)
    return fail(MUSE_ERR_CAPACITY,
                "proj_bf16_tiles_noalloc: this shape and plan need %lld bytes of split-K scratch, the built-in area "
                "holds %lld (use muse_proj_bf16_tiles with caller scratch, fewer CTAs or a smaller tile_n)",
                (long long)sh.scratch, (long long)MUSE_NOALLOC_SCRATCH_BYTES);
  void* scratch = nullptr;
  if (int rc = noalloc_scratch(&scratch)) return rc;
  // The array keeps the previous call's contents: the tile counters this call uses must start at 0.
  const cudaError_t e = cudaMemsetAsync(scratch, 0, static_cast<size_t>(sh.tiles) * sizeof(int),
                                        static_cast<cudaStream_t>(stream));
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "proj_bf16_tiles_noalloc: cudaMemsetAsync: %s", cudaGetErrorString(e));
  return run_streamk(x, tiles, y, m, n, k, *plan, scratch, MUSE_NOALLOC_SCRATCH_BYTES,
                     static_cast<cudaStream_t>(stream));
}
