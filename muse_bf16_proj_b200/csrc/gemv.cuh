// Streaming split-K GEMV for few tokens (M <= 8), BF16 or 12-bit weights, FP32 accumulation.
//
// Grid: one CTA per block of `rows_per_cta` consecutive output rows (sized by the host to about
// one CTA per SM). A CTA's weights are one contiguous byte range of the row-major stream (W rows
// are contiguous in both formats), so one producer lane moves it with 1-D bulk copies
// (cp.async.bulk, L2 evict-first) through a `stages`-deep shared-memory ring; NW consumer warps
// decode and multiply. A "unit" is the slice of one row that one warp consumes at once: 256
// BF16 weights (512 B, 16 B a lane) or 512 12-bit weights (768 B: 16 low bytes + 8 code bytes a
// lane). Each unit's dot products are reduced over the warp with shuffles and parked in shared
// memory per (row, K-segment); the final pass adds a row's segments in a fixed order, so the
// result is deterministic (the K split inside the CTA is the "split-K"). 12-bit weights then get
// their escape corrections, also in a fixed order.
#pragma once

#include "ptx.cuh"
#include "tc12.cuh"  // decode12_bf16x8

namespace muse {

struct GemvArgs {
  const uint8_t* wstream;   // BF16 W [N, K] row-major, or the 12-bit unit stream
  const uint16_t* x;        // [M, K] BF16
  uint16_t* y;              // [M, N] BF16
  const uint8_t* bases;     // 12-bit: per-128x128-tile window bases [ceil(N/128)][K/128]
  const int32_t* esc_ptr;   // 12-bit: per-row CSR [N + 1]
  const uint32_t* esc_val;  // 12-bit: k << 16 | true BF16 bits
  int n, k, rows_per_cta, chunk_units, stages;
  TraceRec* trace;   // optional per-CTA timestamps (nullptr: off)
  int trace_cap;
};

template <bool kTwelve>
struct GemvFormat;
template <>
struct GemvFormat<false> {
  static constexpr int kUnitElems = 256;
  static constexpr int kUnitBytes = 512;
};
template <>
struct GemvFormat<true> {
  static constexpr int kUnitElems = 512;
  static constexpr int kUnitBytes = 768;
};

template <int M>
__device__ __forceinline__ void warp_sum(float (&v)[M]) {
#pragma unroll
  for (int m = 0; m < M; ++m) {
    float s = v[m];
    s += __shfl_xor_sync(0xffffffffu, s, 16);
    s += __shfl_xor_sync(0xffffffffu, s, 8);
    s += __shfl_xor_sync(0xffffffffu, s, 4);
    s += __shfl_xor_sync(0xffffffffu, s, 2);
    s += __shfl_xor_sync(0xffffffffu, s, 1);
    v[m] = s;
  }
}

// One unit: this lane's 8 (BF16) or 16 (12-bit) weights times every token, summed over the warp.
template <bool kTwelve, int M>
__device__ __forceinline__ void gemv_unit(const uint8_t* ubuf, const GemvArgs& a, int row, int seg, int lane,
                                          float (&acc)[M]) {
  if constexpr (!kTwelve) {
    const uint4 wv = *reinterpret_cast<const uint4*>(ubuf + lane * 16);
    const float wf[8] = {bf16lo(wv.x), bf16hi(wv.x), bf16lo(wv.y), bf16hi(wv.y),
                         bf16lo(wv.z), bf16hi(wv.z), bf16lo(wv.w), bf16hi(wv.w)};
    const int k0 = seg * 256 + lane * 8;
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const uint4 xv = ldg_nc_v4(a.x + static_cast<size_t>(m) * a.k + k0);
      float s = 0.f;
      s = fmaf(wf[0], bf16lo(xv.x), s); s = fmaf(wf[1], bf16hi(xv.x), s);
      s = fmaf(wf[2], bf16lo(xv.y), s); s = fmaf(wf[3], bf16hi(xv.y), s);
      s = fmaf(wf[4], bf16lo(xv.z), s); s = fmaf(wf[5], bf16hi(xv.z), s);
      s = fmaf(wf[6], bf16lo(xv.w), s); s = fmaf(wf[7], bf16hi(xv.w), s);
      acc[m] = s;
    }
  } else {
    const uint4 lv = *reinterpret_cast<const uint4*>(ubuf + lane * 16);
    const uint2 cv = *reinterpret_cast<const uint2*>(ubuf + 512 + lane * 8);
    const int k0 = seg * 512 + lane * 16;
    const uint32_t base = a.bases[static_cast<size_t>(row >> 7) * (a.k >> 7) + (k0 >> 7)];
    const uint32_t base4 = base * 0x01010101u;
    // The window as a byte table (byte j of l03:l47 = base + j) for the table-lookup decode.
    const uint32_t l03 = base4 + 0x03020100u, l47 = base4 + 0x07060504u;
    const uint4 d0 = decode12_bf16x8(lv.x, lv.y, cv.x, l03, l47);
    const uint4 d1 = decode12_bf16x8(lv.z, lv.w, cv.y, l03, l47);
    const float wf[16] = {bf16lo(d0.x), bf16hi(d0.x), bf16lo(d0.y), bf16hi(d0.y), bf16lo(d0.z), bf16hi(d0.z),
                          bf16lo(d0.w), bf16hi(d0.w), bf16lo(d1.x), bf16hi(d1.x), bf16lo(d1.y), bf16hi(d1.y),
                          bf16lo(d1.z), bf16hi(d1.z), bf16lo(d1.w), bf16hi(d1.w)};
#pragma unroll
    for (int m = 0; m < M; ++m) {
      const uint16_t* xr = a.x + static_cast<size_t>(m) * a.k + k0;
      const uint4 x0 = ldg_nc_v4(xr);
      const uint4 x1 = ldg_nc_v4(xr + 8);
      float s = 0.f;
      s = fmaf(wf[0], bf16lo(x0.x), s); s = fmaf(wf[1], bf16hi(x0.x), s);
      s = fmaf(wf[2], bf16lo(x0.y), s); s = fmaf(wf[3], bf16hi(x0.y), s);
      s = fmaf(wf[4], bf16lo(x0.z), s); s = fmaf(wf[5], bf16hi(x0.z), s);
      s = fmaf(wf[6], bf16lo(x0.w), s); s = fmaf(wf[7], bf16hi(x0.w), s);
      s = fmaf(wf[8], bf16lo(x1.x), s); s = fmaf(wf[9], bf16hi(x1.x), s);
      s = fmaf(wf[10], bf16lo(x1.y), s); s = fmaf(wf[11], bf16hi(x1.y), s);
      s = fmaf(wf[12], bf16lo(x1.z), s); s = fmaf(wf[13], bf16hi(x1.z), s);
      s = fmaf(wf[14], bf16lo(x1.w), s); s = fmaf(wf[15], bf16hi(x1.w), s);
      acc[m] = s;
    }
  }
  warp_sum<M>(acc);
}

// Shared memory: ring [stages][chunk bytes] | full[stages] | empty[stages] | red[rows][segs][M].
template <bool kTwelve, int M, int NW>
__global__ void __launch_bounds__(32 * (NW + 1), 1) gemv_stream_kernel(const GemvArgs a) {
  using F = GemvFormat<kTwelve>;
  extern __shared__ __align__(128) uint8_t smem[];
  const bool tracing = a.trace != nullptr && static_cast<int>(blockIdx.x) < a.trace_cap && threadIdx.x == 0;
  unsigned long long t_start = tracing ? globaltimer() : 0ull, t_ready = 0ull, t_main = 0ull;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int r0 = blockIdx.x * a.rows_per_cta;
  const int rows = min(a.rows_per_cta, a.n - r0);
  const int segs = a.k / F::kUnitElems;
  const int total_units = rows * segs;
  const int chunk_bytes = a.chunk_units * F::kUnitBytes;
  const int nchunks = (total_units + a.chunk_units - 1) / a.chunk_units;

  uint8_t* ring = smem;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(a.stages) * chunk_bytes);
  uint64_t* empty = full + a.stages;
  float* red = reinterpret_cast<float*>(empty + a.stages);

  if (threadIdx.x == 0) {
    for (int s = 0; s < a.stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], NW);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (tracing) t_ready = globaltimer();

  if (warp == NW) {
    // Producer: one lane streams this CTA's contiguous byte range.
    if (lane == 0) {
      const uint64_t pol = policy_evict_first();
      const uint8_t* src = a.wstream + static_cast<size_t>(r0) * segs * F::kUnitBytes;
      int issued = 0;
      for (int c = 0; c < nchunks; ++c) {
        const int s = c % a.stages;
        if (!mbar_wait(&empty[s], ((c / a.stages) & 1) ^ 1, kErrGemvProducer)) break;
        const int units = min(a.chunk_units, total_units - c * a.chunk_units);
        const uint32_t bytes = static_cast<uint32_t>(units * F::kUnitBytes);
        mbar_expect_tx(&full[s], bytes);
        bulk_g2s(ring + static_cast<size_t>(s) * chunk_bytes, src + static_cast<size_t>(c) * chunk_bytes, bytes,
                 &full[s], pol);
        ++issued;
      }
      // Let every copy this lane issued land before the CTA can exit (a no-op when all were consumed).
      for (int c = max(0, issued - a.stages); c < issued; ++c)
        mbar_wait(&full[c % a.stages], (c / a.stages) & 1, kErrDrain, kWaitLimitNs / 10);
    }
  } else {
    // Consumers. x (and y, written at the end) may belong to the grid this one overlaps with.
    pdl_wait();
    for (int c = 0; c < nchunks; ++c) {
      const int s = c % a.stages;
      // Warp-uniform, so no lane leaves the loop while others still shuffle.
      if (!__all_sync(0xffffffffu, mbar_wait(&full[s], (c / a.stages) & 1, kErrGemvConsumer))) break;
      const int units = min(a.chunk_units, total_units - c * a.chunk_units);
      const uint8_t* buf = ring + static_cast<size_t>(s) * chunk_bytes;
#pragma unroll 2
      for (int j = warp; j < units; j += NW) {
        const int g = c * a.chunk_units + j;
        const int row = g / segs;
        const int seg = g - row * segs;
        float acc[M];
        gemv_unit<kTwelve, M>(buf + j * F::kUnitBytes, a, r0 + row, seg, lane, acc);
        if (lane == 0) {
#pragma unroll
          for (int m = 0; m < M; ++m) red[static_cast<size_t>(g) * M + m] = acc[m];
        }
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
    }
    if (tracing) t_main = globaltimer();
  }
  __syncthreads();
  pdl_launch_dependents();  // every thread: the weights are consumed, the next grid may start

  // Fixed-order sum of each row's segments (then 12-bit escape corrections) and the BF16 store;
  // consecutive threads take consecutive rows of one token.
  for (int i = threadIdx.x; i < rows * M; i += blockDim.x) {
    const int m = i / rows;
    const int row = i - m * rows;
    const float* rp = red + static_cast<size_t>(row) * segs * M + m;
    float sum = 0.f;
    for (int sg = 0; sg < segs; ++sg) sum += rp[static_cast<size_t>(sg) * M];
    if constexpr (kTwelve) {
      const int r = r0 + row;
      const uint16_t* xr = a.x + static_cast<size_t>(m) * a.k;
      const uint8_t* brow = a.bases + static_cast<size_t>(r >> 7) * (a.k >> 7);
      for (int e = a.esc_ptr[r]; e < a.esc_ptr[r + 1]; ++e) {
        const uint32_t v = a.esc_val[e];
        const int kk = static_cast<int>(v >> 16);
        const float xv = bf16f(xr[kk]);
        const float placeholder = bf16f(static_cast<uint16_t>(static_cast<uint32_t>(brow[kk >> 7]) << 8));
        sum = fmaf(bf16f(static_cast<uint16_t>(v & 0xFFFFu)), xv, sum);
        sum = fmaf(-placeholder, xv, sum);
      }
    }
    a.y[static_cast<size_t>(m) * a.n + r0 + row] = f32_to_bf16(sum);
  }
  if (tracing) a.trace[blockIdx.x] = TraceRec{t_start, t_ready, t_main, globaltimer(), smid(), blockIdx.x, 0u, 0u};
}

}  // namespace muse
