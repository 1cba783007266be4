// Lossless 12-bit encoding on the device, in exactly muse_encode12's host format (the rules are in
// enc12_core.h), so everything downstream (muse_pack_tiles12, the 12-bit readers, the on-disk
// cache) is unchanged. Replaces nf12_pack_cuda (submission.py:591-626), which encoded with torch ops.
// Byte and integer work over W: four short HBM-bound passes (W read three times, planes written
// once), no tensor cores and no waits:
//   1. enc12_bases_kernel: one CTA per 128 x 128 tile, E7 histogram in shared memory, the window base.
//   2. enc12_planes_kernel: one warp per row, a lane encodes 8 weights per step (one 16-byte load,
//      an 8-byte and a 4-byte store), the row's escape count into esc_ptr[r + 1].
//   3. enc12_scan_kernel: one CTA turns the counts into the CSR offsets (in place, esc_ptr[0] = 0).
//   4. enc12_escapes_kernel: one warp per row with escapes, entries in ascending k (warp prefix
//      sum of each step's counts); a write outside the row's range or the buffer is skipped and
//      recorded (kErrEncode).
#pragma once

#include "enc12_core.h"
#include "ptx.cuh"

namespace muse {

constexpr unsigned int kErrEncode = 0x501;
constexpr int kEnc12RowsPerCta = 8;  // warps (rows) per CTA of the planes and escapes passes
constexpr int kEnc12ScanThreads = 1024;

__device__ __forceinline__ void enc12_unpack(const uint4& v, uint16_t* out) {
  const uint32_t w[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
  for (int q = 0; q < 4; ++q) {
    out[2 * q] = static_cast<uint16_t>(w[q] & 0xFFFFu);
    out[2 * q + 1] = static_cast<uint16_t>(w[q] >> 16);
  }
}

// grid (K / 128, ceil(N / 128)), 128 threads. A warp reads two rows of the tile per step (lanes
// 0-15 one row's 128 weights, 16-31 the next), 32 rows in all; each warp counts into its own
// histogram.
__global__ void __launch_bounds__(128) enc12_bases_kernel(const uint16_t* __restrict__ w, int64_t n, int64_t k,
                                                          uint8_t* __restrict__ bases) {
  __shared__ int hist[4][128];
  __shared__ int tot[128];
  const int j = blockIdx.x, warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int64_t t = blockIdx.y;
  for (int i = threadIdx.x; i < 4 * 128; i += 128) (&hist[0][0])[i] = 0;
  __syncthreads();
  for (int rr = warp * 2 + (lane >> 4); rr < kEnc12Tile; rr += 8) {
    const int64_t r = t * kEnc12Tile + rr;
    if (r >= n) break;  // rr only grows
    const uint4 v = __ldg(reinterpret_cast<const uint4*>(w + r * k + static_cast<int64_t>(j) * kEnc12Tile +
                                                         (lane & 15) * kEnc12Vec));
    uint16_t vals[kEnc12Vec];
    enc12_unpack(v, vals);
#pragma unroll
    for (int q = 0; q < kEnc12Vec; ++q) atomicAdd(&hist[warp][enc12_e7(vals[q])], 1);
  }
  __syncthreads();
  tot[threadIdx.x] = hist[0][threadIdx.x] + hist[1][threadIdx.x] + hist[2][threadIdx.x] + hist[3][threadIdx.x];
  __syncthreads();
  if (threadIdx.x == 0) bases[t * (k / kEnc12Tile) + j] = static_cast<uint8_t>(enc12_pick_base(tot));
}

// grid ceil(N / 8), 256 threads: warp = row. Lane l takes weights c = 8l + 256i.
__global__ void __launch_bounds__(32 * kEnc12RowsPerCta) enc12_planes_kernel(
    const uint16_t* __restrict__ w, int64_t n, int64_t k, const uint8_t* __restrict__ bases,
    uint8_t* __restrict__ planes, int32_t* __restrict__ esc_ptr) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kEnc12RowsPerCta + (threadIdx.x >> 5);
  if (r >= n) return;  // warp-uniform
  const int lane = threadIdx.x & 31;
  const int64_t units = k / kEnc12Unit;
  const uint8_t* brow = bases + (r / kEnc12Tile) * (k / kEnc12Tile);
  const uint16_t* row = w + r * k;
  uint32_t cnt = 0;
  for (int64_t c = lane * kEnc12Vec; c < k; c += 32 * kEnc12Vec) {  // the same trip count on every lane
    uint16_t vals[kEnc12Vec];
    enc12_unpack(__ldg(reinterpret_cast<const uint4*>(row + c)), vals);
    uint32_t lo0, lo1, code;
    cnt += __popc(enc12_encode8(vals, brow[c / kEnc12Tile], &lo0, &lo1, &code));
    int64_t lo_off, code_off;
    enc12_offsets(r, c, units, &lo_off, &code_off);
    *reinterpret_cast<uint2*>(planes + lo_off) = make_uint2(lo0, lo1);
    *reinterpret_cast<uint32_t*>(planes + code_off) = code;
  }
  cnt = __reduce_add_sync(0xffffffffu, cnt);
  if (lane == 0) esc_ptr[r + 1] = static_cast<int32_t>(cnt);
}

// One CTA: esc_ptr[1..N] (per-row counts) -> inclusive prefix sums, esc_ptr[0] = 0. Each thread
// sums a contiguous run of rows, thread 0 scans the 1024 run totals, each thread rewrites its run.
// The host guarantees N * K < 2^31, so no sum overflows.
__global__ void __launch_bounds__(kEnc12ScanThreads) enc12_scan_kernel(int32_t* __restrict__ esc_ptr, int64_t n) {
  __shared__ int64_t part[kEnc12ScanThreads];
  const int64_t per = (n + kEnc12ScanThreads - 1) / kEnc12ScanThreads;
  const int64_t b = 1 + static_cast<int64_t>(threadIdx.x) * per;
  const int64_t e = b + per < n + 1 ? b + per : n + 1;
  int64_t s = 0;
  for (int64_t i = b; i < e; ++i) s += esc_ptr[i];
  part[threadIdx.x] = s;
  __syncthreads();
  if (threadIdx.x == 0) {
    int64_t acc = 0;
    for (int i = 0; i < kEnc12ScanThreads; ++i) {
      const int64_t v = part[i];
      part[i] = acc;
      acc += v;
    }
    esc_ptr[0] = 0;
  }
  __syncthreads();
  int64_t acc = part[threadIdx.x];
  for (int64_t i = b; i < e; ++i) {
    acc += esc_ptr[i];
    esc_ptr[i] = static_cast<int32_t>(acc);
  }
}

// grid ceil(N / 8), 256 threads: warp = row, as the planes pass; rows without escapes return.
__global__ void __launch_bounds__(32 * kEnc12RowsPerCta) enc12_escapes_kernel(
    const uint16_t* __restrict__ w, int64_t n, int64_t k, const uint8_t* __restrict__ bases,
    const int32_t* __restrict__ esc_ptr, uint32_t* __restrict__ esc_val, int64_t esc_cap) {
  const int64_t r = static_cast<int64_t>(blockIdx.x) * kEnc12RowsPerCta + (threadIdx.x >> 5);
  if (r >= n) return;  // warp-uniform
  const int64_t o0 = esc_ptr[r], o1 = esc_ptr[r + 1];
  if (o1 <= o0) return;  // warp-uniform
  const int lane = threadIdx.x & 31;
  const uint8_t* brow = bases + (r / kEnc12Tile) * (k / kEnc12Tile);
  const uint16_t* row = w + r * k;
  const int64_t beg = o0 > 0 ? o0 : 0, end = o1 < esc_cap ? o1 : esc_cap;  // writes stay in [beg, end)
  int64_t o = o0;  // the row's next entry, the same on every lane
  for (int64_t c = lane * kEnc12Vec; c < k; c += 32 * kEnc12Vec) {
    uint16_t vals[kEnc12Vec];
    enc12_unpack(__ldg(reinterpret_cast<const uint4*>(row + c)), vals);
    uint32_t lo0, lo1, code;
    const uint32_t mask = enc12_encode8(vals, brow[c / kEnc12Tile], &lo0, &lo1, &code);
    const int m = __popc(mask);
    int incl = m;  // inclusive prefix over the lanes (lanes hold ascending k)
#pragma unroll
    for (int d = 1; d < 32; d <<= 1) {
      const int y = __shfl_up_sync(0xffffffffu, incl, d);
      if (lane >= d) incl += y;
    }
    const int total = __shfl_sync(0xffffffffu, incl, 31);
    int64_t dst = o + incl - m;
#pragma unroll
    for (int q = 0; q < kEnc12Vec; ++q) {
      if (!((mask >> q) & 1u)) continue;
      if (dst >= beg && dst < end) esc_val[dst] = enc12_escape_entry(c + q, vals[q]);
      else report_error(kErrEncode);
      ++dst;
    }
    o += total;
  }
}

}  // namespace muse
