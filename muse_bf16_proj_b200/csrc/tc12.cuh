// The 12-bit lossless weight blocks the tensor-core projection reads (tc_skinny.cuh), their pack
// kernels and the decode helpers.
//
// Format (muse_pack_tiles12): one 12416-byte block per (128-row tile rt, 64-k block kb), blocks
// ordered [rt][kb]:
//   bytes     0 .. 12287  six 2 KB slabs of 128 16-byte chunks (row r at r * 16): slabs 0-3 the
//                         low bytes of weights 16j .. 16j + 15, slabs 4-5 the code bytes of
//                         weights 32j .. 32j + 31 (low nibble = even k), so a decoder thread's six
//                         loads fall on consecutive addresses across a warp (no bank conflicts);
//   bytes 12288 .. 12415  the block's escape area: word 0 = window base << 16 | escape count;
//                         words 1 .. 31 = the first 31 escapes, r << 22 | (k - 64 kb) << 16 | bits,
//                         sorted by row then k. A block with more escapes (rare: 0.4% of its
//                         weights) sends its decoders to the per-row escape list instead.
// A weight rebuilds as high byte = (code & 8) << 4 | (base + (code & 7)), low byte verbatim; an
// escape's true bits overwrite its placeholder, so the tensor cores see the original BF16 weights
// bit for bit while HBM moves 12 bits a weight (plus 1% for the escape areas).
#pragma once

#include "ptx.cuh"

namespace muse {

constexpr int kT12Raw = 12288;    // the 12-bit planes of one 128 x 64 block
constexpr int kT12Block = 12416;  // + the escape area
constexpr int kT12EscSlots = 31;
constexpr int kT12Dec = 16384;    // one decoded BF16 A tile

__host__ __device__ __forceinline__ long long t12_start(long long c, long long units, int g) { return c * units / g; }

__host__ __device__ __forceinline__ int t12_owner(long long u, long long units, int g) {
  long long c = u * g / units;
  while (c + 1 < g && t12_start(c + 1, units, g) <= u) ++c;
  while (c > 0 && t12_start(c, units, g) > u) --c;
  return static_cast<int>(c);
}

// Planes -> the slab part of each block; rows past N are zero. One thread per 16-byte chunk.
__global__ void pack_tiles12_kernel(const uint8_t* __restrict__ planes, uint8_t* __restrict__ out, int n, int k,
                                    int nkb, long long chunks) {
  const int units = k / 512;
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < chunks;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long blk = i / (kT12Raw / 16);
    const int within = static_cast<int>(i % (kT12Raw / 16));
    const int rt = static_cast<int>(blk / nkb), kb = static_cast<int>(blk % nkb);
    const int slab = within >> 7, r = within & 127;
    const bool code = slab >= 4;  // slabs 0-3: 16 low bytes; 4-5: 16 code bytes (32 weights)
    const int kk = kb * 64 + (code ? (slab - 4) * 32 : slab * 16);
    const int row = rt * 128 + r;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < n) {
      const uint8_t* unit = planes + (static_cast<size_t>(row) * units + kk / 512) * 768;
      const int j = kk % 512;
      v = *reinterpret_cast<const uint4*>(code ? unit + 512 + j / 2 : unit + j);
    }
    *reinterpret_cast<uint4*>(out + blk * kT12Block + static_cast<size_t>(within) * 16) = v;
  }
}

// First index in [lo, hi) of a row's escape list whose k is >= k0 (the list is sorted by k).
__device__ __forceinline__ int t12_lower_bound(const uint32_t* __restrict__ esc_val, int lo, int hi, uint32_t k0) {
  while (lo < hi) {
    const int mid = (lo + hi) >> 1;
    if ((__ldg(esc_val + mid) >> 16) < k0) lo = mid + 1; else hi = mid;
  }
  return lo;
}

// The escape area of each block: one CTA of 128 threads per block, thread r = row r.
__global__ void __launch_bounds__(128) pack_escapes12_kernel(const uint8_t* __restrict__ bases,
                                                              const int32_t* __restrict__ esc_ptr,
                                                              const uint32_t* __restrict__ esc_val,
                                                              uint8_t* __restrict__ out, int n, int k, int nkb) {
  __shared__ int warp_sum[4];
  const long long blk = blockIdx.x;
  const int rt = static_cast<int>(blk / nkb), kb = static_cast<int>(blk % nkb);
  const int r = threadIdx.x, lane = r & 31, w = r >> 5;
  const int row = rt * 128 + r;
  int e0 = 0, cnt = 0;
  if (row < n) {
    const int lo = esc_ptr[row], hi = esc_ptr[row + 1];
    e0 = t12_lower_bound(esc_val, lo, hi, static_cast<uint32_t>(kb * 64));
    cnt = t12_lower_bound(esc_val, e0, hi, static_cast<uint32_t>(kb * 64 + 64)) - e0;
  }
  int incl = cnt;  // inclusive scan over rows
#pragma unroll
  for (int o = 1; o < 32; o <<= 1) {
    const int v = __shfl_up_sync(0xffffffffu, incl, o);
    if (lane >= o) incl += v;
  }
  if (lane == 31) warp_sum[w] = incl;
  __syncthreads();
  int before = 0, total = 0;
  for (int i = 0; i < 4; ++i) {
    if (i < w) before += warp_sum[i];
    total += warp_sum[i];
  }
  uint32_t* area = reinterpret_cast<uint32_t*>(out + blk * kT12Block + kT12Raw);
  const int off = before + incl - cnt;
  for (int j = 0; j < cnt && off + j < kT12EscSlots; ++j) {
    const uint32_t v = __ldg(esc_val + e0 + j);
    area[1 + off + j] = (static_cast<uint32_t>(r) << 22) | (((v >> 16) - static_cast<uint32_t>(kb * 64)) << 16) |
                        (v & 0xFFFFu);
  }
  if (r >= total && r < kT12EscSlots) area[1 + r] = 0u;  // unused slots
  if (r == 0) area[0] = (static_cast<uint32_t>(bases[static_cast<size_t>(rt) * (k / 128) + kb / 2]) << 16) |
                        static_cast<uint32_t>(min(total, 0xFFFF));
}

__device__ __forceinline__ void fence_proxy_async_smem() {
  asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}

// 8 weights -> four u32 each holding two BF16 (weight 2i in the low half). lo03 / lo47: low
// bytes; codes: 8 codes, low nibble first; l03 / l47: the window as a byte table, byte j of
// l03:l47 = base + j. Each code's low 3 bits pick its high byte from the table (byte permute; the
// code bytes are already nibble-packed selectors) and its bit 3 becomes the high byte's sign bit:
// it sits at bit 7 of a byte of `codes` (odd weights) or of `codes << 4` (even weights).
__device__ __forceinline__ uint4 decode12_bf16x8(uint32_t lo03, uint32_t lo47, uint32_t codes, uint32_t l03,
                                                 uint32_t l47) {
  const uint32_t sel = codes & 0x77777777u;
  const uint32_t a03 = __byte_perm(l03, l47, sel);
  const uint32_t a47 = __byte_perm(l03, l47, sel >> 16);
  const uint32_t c4 = codes << 4;
  const uint32_t h03 = a03 | (__byte_perm(c4, codes, 0x5140) & 0x80808080u);
  const uint32_t h47 = a47 | (__byte_perm(c4, codes, 0x7362) & 0x80808080u);
  return make_uint4(__byte_perm(lo03, h03, 0x5140), __byte_perm(lo03, h03, 0x7362), __byte_perm(lo47, h47, 0x5140),
                    __byte_perm(lo47, h47, 0x7362));
}

__device__ __forceinline__ void t12_patch(uint8_t* drow, int sw, int kk, uint32_t bits) {
  *reinterpret_cast<uint16_t*>(drow + (((kk >> 3) ^ sw) << 4) + (kk & 7) * 2) = static_cast<uint16_t>(bits);
}

}  // namespace muse
