// C ABI of libmuse_proj.so: argument checks, plans, TMA descriptors and kernel launches.
// The kernels live in gemv.cuh and tc_tile.cuh; this is the only translation unit with device
// code, so the device error word in ptx.cuh has one definition.
#include <cuda.h>
#include <cuda_runtime.h>
#include <cudaTypedefs.h>

#include <algorithm>
#include <cstdint>
#include <cstring>
#include <mutex>

#include "../../include/muse_proj.h"
#include "errors.h"
#include "gemv.cuh"
#include "tc_tile.cuh"

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
int make_map(CUtensorMap* map, const void* base, int64_t rows, int64_t cols, int box_rows) {
  auto fn = encode_fn();
  if (!fn) return fail(MUSE_ERR_CUDA, "cuTensorMapEncodeTiled entry point not found");
  cuuint64_t dims[2] = {static_cast<cuuint64_t>(cols), static_cast<cuuint64_t>(rows)};
  cuuint64_t strides[1] = {static_cast<cuuint64_t>(cols * 2)};
  cuuint32_t box[2] = {64u, static_cast<cuuint32_t>(box_rows)};
  cuuint32_t estr[2] = {1u, 1u};
  CUresult r = fn(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
                  CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
  if (r != CUDA_SUCCESS) return fail(MUSE_ERR_CUDA, "cuTensorMapEncodeTiled failed (%d)", static_cast<int>(r));
  return MUSE_OK;
}

bool aligned16(const void* p) { return (reinterpret_cast<uintptr_t>(p) & 15u) == 0; }

int launch_error(const char* what) {
  cudaError_t e = cudaGetLastError();
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "%s: %s", what, cudaGetErrorString(e));
  return MUSE_OK;
}

// ---- GEMV ------------------------------------------------------------------------------------

template <bool kTwelve, int M, int NW>
int launch_gemv_t(const muse::GemvArgs& a, int grid, int smem, cudaStream_t st) {
  auto kern = muse::gemv_stream_kernel<kTwelve, M, NW>;
  static bool configured[kMaxDevices] = {};
  int dev;
  if (int rc = current_device(&dev)) return rc;
  if (!configured[dev]) {
    cudaError_t e = cudaFuncSetAttribute(kern, cudaFuncAttributeMaxDynamicSharedMemorySize, kSmemLimit);
    if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "cudaFuncSetAttribute(gemv): %s", cudaGetErrorString(e));
    configured[dev] = true;
  }
  kern<<<grid, 32 * (NW + 1), smem, st>>>(a);
  return launch_error("gemv launch");
}

template <bool kTwelve, int M>
int launch_gemv_m(const muse::GemvArgs& a, int warps, int grid, int smem, cudaStream_t st) {
  switch (warps) {
    case 4: return launch_gemv_t<kTwelve, M, 4>(a, grid, smem, st);
    case 8: return launch_gemv_t<kTwelve, M, 8>(a, grid, smem, st);
    case 16: return launch_gemv_t<kTwelve, M, 16>(a, grid, smem, st);
    default: return fail(MUSE_ERR_PLAN, "gemv: warps must be 4, 8 or 16 (got %d)", warps);
  }
}

template <bool kTwelve>
int launch_gemv(const muse::GemvArgs& a, int m, int warps, int grid, int smem, cudaStream_t st) {
  switch (m) {
    case 1: return launch_gemv_m<kTwelve, 1>(a, warps, grid, smem, st);
    case 2: return launch_gemv_m<kTwelve, 2>(a, warps, grid, smem, st);
    case 3: return launch_gemv_m<kTwelve, 3>(a, warps, grid, smem, st);
    case 4: return launch_gemv_m<kTwelve, 4>(a, warps, grid, smem, st);
    case 5: return launch_gemv_m<kTwelve, 5>(a, warps, grid, smem, st);
    case 6: return launch_gemv_m<kTwelve, 6>(a, warps, grid, smem, st);
    case 7: return launch_gemv_m<kTwelve, 7>(a, warps, grid, smem, st);
    case 8: return launch_gemv_m<kTwelve, 8>(a, warps, grid, smem, st);
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
      *grid = static_cast<int>((n + rows - 1) / rows);
      *smem = static_cast<int>(stages * chunk_bytes + 16 * stages + red);
      return MUSE_OK;
    }
    if (ctas >= n) return fail(MUSE_ERR_SHAPE, "gemv: partial sums do not fit shared memory");
    ctas = static_cast<int>(std::min<int64_t>(n, ctas * 2));
  }
}

// ---- tcgen05 tile kernel ---------------------------------------------------------------------

template <int BNT>
int launch_tc_t(const CUtensorMap& tmw, const CUtensorMap& tmx, uint16_t* y, int m, int n, int k, int split,
                int stages, cudaStream_t st) {
  auto kern = muse::tc_tile_kernel<BNT>;
  const int smem = muse::tc_tile_smem(BNT, stages);
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
  cudaLaunchConfig_t cfg = {};
  cfg.gridDim = dim3(static_cast<unsigned>(((n + 127) / 128) * split), static_cast<unsigned>((m + BNT - 1) / BNT), 1);
  cfg.blockDim = dim3(muse::kTcThreads, 1, 1);
  cfg.dynamicSmemBytes = static_cast<size_t>(smem);
  cfg.stream = st;
  cudaLaunchAttribute attr[1];
  attr[0].id = cudaLaunchAttributeClusterDimension;
  attr[0].val.clusterDim.x = static_cast<unsigned>(split);
  attr[0].val.clusterDim.y = 1;
  attr[0].val.clusterDim.z = 1;
  cfg.attrs = attr;
  cfg.numAttrs = 1;
  if (split > 1) {
    int clusters = 0;
    e = cudaOccupancyMaxActiveClusters(&clusters, kern, &cfg);
    if (e != cudaSuccess || clusters < 1)
      return fail(MUSE_ERR_PLAN, "tc_tile: clusters of %d CTAs with %d B shared memory cannot be scheduled (%s)", split,
                  smem, e == cudaSuccess ? "occupancy 0" : cudaGetErrorString(e));
  }
  e = cudaLaunchKernelEx(&cfg, kern, tmw, tmx, y, m, n, k, split, stages);
  if (e != cudaSuccess) return fail(MUSE_ERR_CUDA, "tc_tile launch (split %d, tile %d): %s", split, BNT, cudaGetErrorString(e));
  return MUSE_OK;
}

int run_tc_tile(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, const MusePlan& p,
                cudaStream_t st) {
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
  if (split > 16 || split > nkb)
    return fail(MUSE_ERR_PLAN, "tc_tile: split %d must be <= 16 and <= K / 64 = %d", split, nkb);
  if (m > (int64_t(1) << 24) || n > (int64_t(1) << 24) || k > (int64_t(1) << 24))
    return fail(MUSE_ERR_SHAPE, "tc_tile: dimension too large");
  const int limit = std::min(kSmemLimit, d->smem_optin);
  const int per_stage = muse::kTcABytes + muse::tc_tile_bbytes(bnt);
  int max_stages = (limit - 1024 - 64) / (per_stage + 16);
  int stages = p.stages > 0 ? p.stages : max_stages;
  if (stages > max_stages || stages < 2) return fail(MUSE_ERR_PLAN, "tc_tile: %d stages do not fit (max %d)", stages, max_stages);
  // The FP32 partial [tile_n][128] reuses the ring; it must fit there.
  if (split > 1 && bnt * 128 * 4 > stages * per_stage)
    return fail(MUSE_ERR_PLAN, "tc_tile: ring of %d stages too small for the split-K partial", stages);
  CUtensorMap tmw, tmx;
  if (int rc = make_map(&tmw, w, n, k, 128)) return rc;
  if (int rc = make_map(&tmx, x, m, k, bnt)) return rc;
  auto yy = static_cast<uint16_t*>(y);
  const int mi = static_cast<int>(m), ni = static_cast<int>(n), ki = static_cast<int>(k);
  switch (bnt) {
    case 16: return launch_tc_t<16>(tmw, tmx, yy, mi, ni, ki, split, stages, st);
    case 32: return launch_tc_t<32>(tmw, tmx, yy, mi, ni, ki, split, stages, st);
    case 64: return launch_tc_t<64>(tmw, tmx, yy, mi, ni, ki, split, stages, st);
    case 128: return launch_tc_t<128>(tmw, tmx, yy, mi, ni, ki, split, stages, st);
    default: return launch_tc_t<256>(tmw, tmx, yy, mi, ni, ki, split, stages, st);
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
  if (v) return fail(MUSE_ERR_TIMEOUT, "a kernel's bounded wait expired (device code 0x%x)", v);
  return MUSE_OK;
}

int muse_plan_default(int64_t m, int64_t n, int64_t k, int weights_12b, MusePlan* out) {
  muse::clear_error();
  if (!out) return fail(MUSE_ERR_INVALID, "plan_default: null output");
  if (m < 1 || n < 1 || k < 1) return fail(MUSE_ERR_INVALID, "plan_default: non-positive size");
  DeviceInfo* d;
  int sms = 148;
  if (device_info(&d) == MUSE_OK) sms = d->sms;
  muse::clear_error();
  std::memset(out, 0, sizeof(*out));
  if (weights_12b) {
    out->kernel = MUSE_KERNEL_GEMV_12B;
    out->warps = 8;
    return m <= 8 ? MUSE_OK : fail(MUSE_ERR_SHAPE, "plan_default: 12-bit weights serve M <= 8");
  }
  if (m <= 4 && k % 256 == 0) {
    out->kernel = MUSE_KERNEL_GEMV_BF16;
    out->warps = 8;
    return MUSE_OK;
  }
  out->kernel = MUSE_KERNEL_TC_TILE;
  int bnt = 16;
  while (bnt < m && bnt < 256) bnt *= 2;
  out->tile_n = bnt;
  const int64_t tiles = ((n + 127) / 128) * ((m + bnt - 1) / bnt);
  const int64_t nkb = (k + 63) / 64;
  int64_t split = tiles >= sms ? 1 : sms / tiles;
  split = std::max<int64_t>(1, std::min<int64_t>({split, 8, nkb}));
  out->split = static_cast<int>(split);
  return MUSE_OK;
}

int muse_proj_bf16(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, const MusePlan* plan,
                   void* stream) {
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
    return launch_gemv<false>(a, static_cast<int>(m), warps, grid, smem, st);
  }
  if (plan->kernel == MUSE_KERNEL_TC_TILE) return run_tc_tile(x, w, y, m, n, k, *plan, st);
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
  return launch_gemv<true>(a, static_cast<int>(m), warps, grid, smem, static_cast<cudaStream_t>(stream));
}

}  // extern "C"
