// CUDA-core GEMV for one to four tokens over the packed W tiles, built for the latency of a single
// call: no shared-memory ring, no mbarriers, no tensor memory, no scratch, nothing to set up before
// the first weight load leaves the SM.
//
// y[m, n] = sum_k x[m, k] * W[n, k], FP32 accumulation, BF16 out, for M <= 4.
//
// Work: a "quad" is 4 consecutive W rows. In the packed tiles ([rt][kb][128][64] BF16, row r's 16-byte
// chunk c at position c ^ (r % 8)) a quad's 64-k block is one contiguous 512-byte range, so one
// 16-byte load a lane covers it: lane l reads row (l >> 3) of the quad, chunk position l & 7, i.e.
// the 8 weights k = 64 kb + 8 ((l & 7) ^ (row % 8)) .. +7. A warp owns QW adjacent quads (1, 2, 4 or 8:
// QW x 512 contiguous bytes a k block, which HBM streams better than scattered 512-byte pieces) over
// one of `split` equal K segments and keeps 16 loads a lane in flight (two batches of 8 16-byte loads,
// double-buffered in registers); its first two batches are issued before the programmatic-launch
// wait, since the weights are not written by the previous grid. x [MT][K] is staged once a CTA as
// BF16 in shared memory after that wait (zero beyond M and K) and read with one conflict-free
// 16-byte load a lane a k block (each quarter warp reads one row's 8 chunks, a permutation).
// Products go through mixed-precision FMAs (fma.rn.f32.bf16: exact BF16 x BF16 products, FP32 sums)
// into max(2, 8 / QW) accumulators a (quad, token), summed in a fixed order, then over the 8 lanes of a row by xor
// shuffles; with split > 1 the CTA's warps of one quad add their segments through shared memory in
// segment order. Every sum has a fixed order, so the result is deterministic.
//
// CTA: `warps` warps = (warps / split) groups of QW quads x split segments.
// Grid: ceil(quads / (QW warps / split)).
// Roofline: HBM (N K 2 bytes of W, read once).
#pragma once

#include "ptx.cuh"

namespace muse {

constexpr int kGtBatch = 8;  // 16-byte loads a lane a batch (two batches in flight)

struct GtArgs {
  const uint8_t* tiles;  // packed W tiles [rtiles][nkb][128][64] BF16
  const uint16_t* x;     // [M, K] BF16
  uint16_t* y;           // [M, N] BF16
  int M, N, K, nkb;
  int quads;   // rtiles * 32
  int split;   // K segments (warps sharing a warp's quads)
  int groups;  // quad groups a CTA (warps / split); a group is QW adjacent quads
  TraceRec* trace;
  int trace_cap;
};

// Shared memory: x [mt][nkb * 64] BF16 | segment sums [warps][qw][4 rows][mt] FP32 (split > 1).
__host__ __device__ constexpr int gt_smem(int mt, int qw, int nkb, int warps, int split) {
  return mt * nkb * 128 + (split > 1 ? warps * qw * 4 * mt * 4 : 0);
}

// FP32 accumulators a (quad, token): 8 / QW, at least an even and an odd one.
__host__ __device__ constexpr int gt_na(int qw) { return qw >= 4 ? 2 : 8 / qw; }

// One batch: KB = kGtBatch / QW k blocks of the warp's QW quads. Quad j of a QW-aligned group (QW > 1)
// has row parity j & 1, so its lanes read x at xe (even quads) or xo (odd); with QW == 1 only xe.
template <int MT, int QW>
__device__ __forceinline__ void gt_batch(const uint4 (&b)[kGtBatch], int first, int nb, uint32_t xe, uint32_t xo,
                                         uint32_t xrow_bytes, float (&acc)[QW][MT][gt_na(QW)]) {
  constexpr int KB = kGtBatch / QW, NA = gt_na(QW);
#pragma unroll
  for (int i = 0; i < KB; ++i) {
    if (first + i < nb) {
      const uint32_t off = static_cast<uint32_t>(first + i) * 128u;
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        const uint4 xv0 = ld_shared_v4u(xe + off + m * xrow_bytes);
        uint4 xv1 = xv0;
        if constexpr (QW > 1) xv1 = ld_shared_v4u(xo + off + m * xrow_bytes);
#pragma unroll
        for (int j = 0; j < QW; ++j) {
          const uint4 w = b[i * QW + j];
          const uint4 xv = (j & 1) ? xv1 : xv0;
          fma_bf16x2(w.x, xv.x, acc[j][m][0 % NA], acc[j][m][1 % NA]);
          fma_bf16x2(w.y, xv.y, acc[j][m][2 % NA], acc[j][m][3 % NA]);
          fma_bf16x2(w.z, xv.z, acc[j][m][4 % NA], acc[j][m][5 % NA]);
          fma_bf16x2(w.w, xv.w, acc[j][m][6 % NA], acc[j][m][7 % NA]);
        }
      }
    }
  }
}

// Loads of one batch: k block first + i of quad j is 512 bytes at wp + (first + i) 16 KB + j 512, so
// a warp's QW quads of one k block are QW x 512 contiguous bytes.
template <int QW>
__device__ __forceinline__ void gt_load(uint4 (&b)[kGtBatch], const uint8_t* wp, int first, int nb, uint64_t pol) {
  constexpr int KB = kGtBatch / QW;
#pragma unroll
  for (int i = 0; i < KB; ++i)
#pragma unroll
    for (int j = 0; j < QW; ++j)
      if (first + i < nb) b[i * QW + j] = ldg_stream_v4(wp + static_cast<size_t>(first + i) * 16384u + j * 512, pol);
}

template <int MT, int QW>
__global__ void __launch_bounds__(512) gemv_tiles_kernel(const GtArgs a) {
  constexpr int KB = kGtBatch / QW, NA = gt_na(QW);
  extern __shared__ __align__(16) uint8_t gt_buf[];
  const int warp = static_cast<int>(threadIdx.x >> 5), lane = static_cast<int>(threadIdx.x & 31);
  const int g = warp / a.split, seg = warp - g * a.split;
  const int q0 = (static_cast<int>(blockIdx.x) * a.groups + g) * QW;  // first quad (QW-aligned: one row tile)
  const bool live = q0 < a.quads;
  const int kb0 = seg * a.nkb / a.split;
  const int nb = (seg + 1) * a.nkb / a.split - kb0;
  const int r4 = lane >> 3, pos = lane & 7;
  const uint8_t* wp = a.tiles + (static_cast<size_t>(q0 >> 5) * a.nkb + kb0) * 16384u +
                      static_cast<size_t>(q0 & 31) * 512u + lane * 16;
  const bool tracing = a.trace != nullptr && static_cast<int>(blockIdx.x) < a.trace_cap && threadIdx.x == 0;
  const unsigned long long t_start = tracing ? globaltimer() : 0ull;

  const uint64_t pol = policy_evict_first();
  uint4 b0[kGtBatch], b1[kGtBatch];
  if (live) {
    gt_load<QW>(b0, wp, 0, nb, pol);
    gt_load<QW>(b1, wp, KB, nb, pol);
  }

  pdl_wait();  // x and y may belong to the previous grid
  const int kp = a.nkb * 64;
  const int cpr = kp / 8;  // 16-byte chunks a staged x row
  const uint32_t xs = smem_u32(gt_buf);
  for (int i = static_cast<int>(threadIdx.x); i < MT * cpr; i += static_cast<int>(blockDim.x)) {
    const int m = i / cpr;
    const int k = (i - m * cpr) * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (m < a.M && k < a.K) v = ldg_cg_v4(a.x + static_cast<size_t>(m) * a.K + k);
    st_shared_v4u(xs + static_cast<uint32_t>(i) * 16u, v.x, v.y, v.z, v.w);
  }
  __syncthreads();
  const unsigned long long t_ready = tracing ? globaltimer() : 0ull;

  float acc[QW][MT][NA];
#pragma unroll
  for (int j = 0; j < QW; ++j)
#pragma unroll
    for (int m = 0; m < MT; ++m)
#pragma unroll
      for (int c = 0; c < NA; ++c) acc[j][m][c] = 0.f;
  // Logical 16-byte chunk of this lane's row: position ^ (row % 8), row % 8 = (quad & 1) * 4 + r4.
  const int par0 = q0 & 1;
  const uint32_t xbase = xs + static_cast<uint32_t>(kb0) * 128u;
  const uint32_t xe = xbase + static_cast<uint32_t>(pos ^ ((par0 << 2) | r4)) * 16u;
  const uint32_t xo = xbase + static_cast<uint32_t>(pos ^ (((par0 ^ 1) << 2) | r4)) * 16u;
  const uint32_t xrow_bytes = static_cast<uint32_t>(kp) * 2u;
  if (live) {
    for (int first = 0; first < nb; first += 2 * KB) {
      gt_batch<MT, QW>(b0, first, nb, xe, xo, xrow_bytes, acc);
      if (first + 2 * KB < nb) gt_load<QW>(b0, wp, first + 2 * KB, nb, pol);
      gt_batch<MT, QW>(b1, first + KB, nb, xe, xo, xrow_bytes, acc);
      if (first + 3 * KB < nb) gt_load<QW>(b1, wp, first + 3 * KB, nb, pol);
    }
  }
  const unsigned long long t_main = tracing ? globaltimer() : 0ull;
  pdl_launch_dependents();  // this CTA's weights are in registers: the next grid may start

  float s[QW][MT];
#pragma unroll
  for (int j = 0; j < QW; ++j)
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      float v = acc[j][m][0];
#pragma unroll
      for (int c = 1; c < NA; ++c) v += acc[j][m][c];
      v += __shfl_xor_sync(0xffffffffu, v, 1);
      v += __shfl_xor_sync(0xffffffffu, v, 2);
      v += __shfl_xor_sync(0xffffffffu, v, 4);
      s[j][m] = v;
    }
  if (a.split == 1) {
    if (live && pos == 0) {
#pragma unroll
      for (int j = 0; j < QW; ++j) {
        const int row = (q0 + j) * 4 + r4;
#pragma unroll
        for (int m = 0; m < MT; ++m)
          if (m < a.M && row < a.N) a.y[static_cast<size_t>(m) * a.N + row] = f32_to_bf16(s[j][m]);
      }
    }
  } else {
    float* red = reinterpret_cast<float*>(gt_buf + static_cast<size_t>(MT) * xrow_bytes);  // [warps][QW][4][MT]
    if (pos == 0) {
#pragma unroll
      for (int j = 0; j < QW; ++j)
#pragma unroll
        for (int m = 0; m < MT; ++m) red[((warp * QW + j) * 4 + r4) * MT + m] = s[j][m];
    }
    __syncthreads();
    for (int t = static_cast<int>(threadIdx.x); t < a.groups * QW * 4 * MT; t += static_cast<int>(blockDim.x)) {
      const int m = t % MT;
      const int rest = t / MT;
      const int rr = rest & 3, j = (rest >> 2) % QW, gg = (rest >> 2) / QW;
      float sum = 0.f;
      for (int sg = 0; sg < a.split; ++sg) sum += red[(((gg * a.split + sg) * QW + j) * 4 + rr) * MT + m];
      const int quad = (static_cast<int>(blockIdx.x) * a.groups + gg) * QW + j;
      const int row = quad * 4 + rr;
      if (quad < a.quads && row < a.N && m < a.M) a.y[static_cast<size_t>(m) * a.N + row] = f32_to_bf16(sum);
    }
  }
  if (tracing)
    a.trace[blockIdx.x] = TraceRec{t_start, t_ready, t_main, globaltimer(), smid(), blockIdx.x};
}

}  // namespace muse
