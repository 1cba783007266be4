// The FP32 router projection: y[m, n] = sum_k x[m, k] * W[n, k] with W FP32 and y FP32.
//
// Few tokens (M <= 32): router_f32_kernel on CUDA cores reads W in FP32 (as the reference's
// _router_fp32_kernel, submission.py:131-169): one CTA per W row, thread t takes k = 4t + 1024j,
// eight 16-byte loads of W issued together (before the programmatic-launch wait: W is a
// prepare-time constant) and 8-byte loads of x, FP32 fused multiply-adds, a warp shuffle and a
// shared-memory sum over the CTA's eight warps.
//
// More tokens: the tensor-core tile kernel on the BF16 pair hi = BF16(W), lo = BF16(W - hi)
// (submission.py:1120-1124, 172-207), stored as the packed tiles of [hi | lo] ([N, 2K]) so one
// K = 2K projection with FP32 accumulation computes x . hi^T + x . lo^T (x's K coordinate wraps
// at K) and writes FP32. pack_router_kernel builds those tiles on the device.
#pragma once

#include "ptx.cuh"
#include "tc_tile.cuh"

namespace muse {

constexpr int kRouterThreads = 256;

template <int MT>
__global__ void __launch_bounds__(kRouterThreads)
    router_f32_kernel(const float* __restrict__ w, const uint16_t* __restrict__ x, float* __restrict__ y, int m, int n,
                      int k) {
  constexpr int kU = 8;  // K steps of 1024 whose W loads are issued together
  __shared__ float red[kRouterThreads / 32][MT];
  const int row = blockIdx.x;
  const int t = threadIdx.x, lane = t & 31, warp = t >> 5;
  const float* wrow = w + static_cast<size_t>(row) * k;
  float acc[MT];
#pragma unroll
  for (int i = 0; i < MT; ++i) acc[i] = 0.f;
  bool waited = false;
  for (int k0 = 4 * t; k0 < k; k0 += 4 * kRouterThreads * kU) {
    // W first (it never comes from the previous grid), all kU loads in flight at once.
    float4 wv[kU];
#pragma unroll
    for (int u = 0; u < kU; ++u) {
      const int kk = k0 + u * 4 * kRouterThreads;
      wv[u] = kk < k ? __ldcs(reinterpret_cast<const float4*>(wrow + kk)) : make_float4(0.f, 0.f, 0.f, 0.f);
    }
    if (!waited) {
      pdl_wait();  // x may be the previous grid's output
      waited = true;
    }
#pragma unroll
    for (int i = 0; i < MT; ++i) {
      if (i < m) {
        uint2 xv[kU];
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          const int kk = k0 + u * 4 * kRouterThreads;
          xv[u] = kk < k ? __ldg(reinterpret_cast<const uint2*>(x + static_cast<size_t>(i) * k + kk)) : make_uint2(0u, 0u);
        }
#pragma unroll
        for (int u = 0; u < kU; ++u) {
          acc[i] = fmaf(__uint_as_float(xv[u].x << 16), wv[u].x, acc[i]);
          acc[i] = fmaf(__uint_as_float(xv[u].x & 0xFFFF0000u), wv[u].y, acc[i]);
          acc[i] = fmaf(__uint_as_float(xv[u].y << 16), wv[u].z, acc[i]);
          acc[i] = fmaf(__uint_as_float(xv[u].y & 0xFFFF0000u), wv[u].w, acc[i]);
        }
      }
    }
  }
  if (!waited) pdl_wait();
  pdl_launch_dependents();
#pragma unroll
  for (int i = 0; i < MT; ++i) {
    float v = acc[i];
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    if (lane == 0) red[warp][i] = v;
  }
  __syncthreads();
  if (t < MT && t < m) {
    float s = 0.f;
#pragma unroll
    for (int j = 0; j < kRouterThreads / 32; ++j) s += red[j][t];
    y[static_cast<size_t>(t) * n + row] = s;
  }
}

// The packed tiles of [hi | lo] for an FP32 W [n, k] (k % 8 == 0): tile (rt, kb) of the [n, 2k]
// BF16 matrix, in pack_tiles_kernel's layout; columns kb * 64 .. < k hold hi, k .. < 2k hold lo.
// Both halves are rounded to nearest even, lo from the FP32 difference W - hi.
__global__ void pack_router_kernel(const float* __restrict__ w, uint4* __restrict__ out, int n, int k, int nkb,
                                   long long chunks) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < chunks;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long tile = i >> 10;
    const int within = static_cast<int>(i & 1023);
    const int r = within >> 3;
    const int c = (within & 7) ^ (r & 7);
    const int rt = static_cast<int>(tile / nkb), kb = static_cast<int>(tile % nkb);
    const int row = rt * 128 + r, col = kb * kTcBK + c * 8;  // column of [hi | lo]
    uint32_t h[4] = {0u, 0u, 0u, 0u};
    if (row < n && col < 2 * k) {
      const bool lo = col >= k;
      const float* src = w + static_cast<size_t>(row) * k + (lo ? col - k : col);
      const float4 a = *reinterpret_cast<const float4*>(src);
      const float4 b = *reinterpret_cast<const float4*>(src + 4);
      const float v[8] = {a.x, a.y, a.z, a.w, b.x, b.y, b.z, b.w};
      uint16_t o[8];
#pragma unroll
      for (int j = 0; j < 8; ++j) {
        const uint16_t hi = f32_to_bf16(v[j]);
        o[j] = lo ? f32_to_bf16(v[j] - __uint_as_float(static_cast<uint32_t>(hi) << 16)) : hi;
      }
#pragma unroll
      for (int j = 0; j < 4; ++j) h[j] = static_cast<uint32_t>(o[2 * j]) | (static_cast<uint32_t>(o[2 * j + 1]) << 16);
    }
    out[i] = make_uint4(h[0], h[1], h[2], h[3]);
  }
}

}  // namespace muse
