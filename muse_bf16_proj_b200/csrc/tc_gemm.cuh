// Persistent tcgen05 GEMM for prefill shapes (many tokens): y[m, n] = sum_k x[m, k] * W[n, k].
//
// A = x (128 tokens a tile, K-major, 2-D TMA with the 128-byte swizzle), B = W from the packed
// tiles (256 rows a tile = two consecutive 128-row packed tiles, two 16 KB bulk copies a stage),
// D = 128 x 256 FP32 in TMEM. One CTA per SM walks the output tiles t = blockIdx.x,
// blockIdx.x + gridDim.x, ... with the token tile fastest, so the CTAs working at the same time
// share a few W column tiles and all x row tiles (the working set stays in the 126 MB L2 for the
// prefill shapes). Two TMEM accumulators (2 x 256 columns = all of TMEM) let a tile's epilogue
// (tcgen05.ld -> BF16 -> global) run while the next tile's UMMAs accumulate.
//
// Warp roles (192 threads): warp 0 = producer, warp 1 = TMEM owner + UMMA issuer (M = 128,
// N = 256, K = 16), warps 2..5 = epilogue (warp w owns TMEM lanes / tile rows 32 * (w % 4) ..).
#pragma once

#include "ptx.cuh"

namespace muse {

constexpr int kGmThreads = 192;
constexpr int kGmBN = 256;                     // W rows a tile
constexpr int kGmABytes = 128 * 64 * 2;        // 16 KB of x a stage
constexpr int kGmBBytes = kGmBN * 64 * 2;      // 32 KB of W a stage
constexpr uint32_t kGmCols = 512;              // two 256-column accumulators

__host__ __device__ constexpr int gm_smem(int stages) {
  return 1024 + stages * (kGmABytes + kGmBBytes) + (2 * stages + 4) * 8 + 16;
}

struct GmArgs {
  const uint8_t* wtiles;  // packed tiles [ceil(N/128)][ceil(K/64)][16 KB]
  uint16_t* y;            // [M, N]
  int M, N, K, stages;
  int mtiles, ntiles, nkb, rtiles;
  TraceRec* trace;
  int trace_cap;
};

__global__ void __launch_bounds__(kGmThreads, 1)
    tc_gemm_kernel(const __grid_constant__ CUtensorMap tmx, const GmArgs a) {
  constexpr uint32_t kIdesc = umma_idesc_bf16(128, kGmBN);
  extern __shared__ uint8_t smem_raw[];
  const bool tracing = a.trace != nullptr && static_cast<int>(blockIdx.x) < a.trace_cap && threadIdx.x == 64;
  const unsigned long long t_start = tracing ? globaltimer() : 0ull;
  unsigned long long t_ready = 0ull, t_main = 0ull;
  uint8_t* smem = smem_align<1024>(smem_raw);
  const int stages = a.stages;
  uint8_t* sa = smem;
  uint8_t* sb = smem + static_cast<size_t>(stages) * kGmABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + static_cast<size_t>(stages) * kGmBBytes);
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int tiles = a.mtiles * a.ntiles;
  const int nkb = a.nkb;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmx);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kGmCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tracing) t_ready = globaltimer();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_keep = policy_evict_last();  // both operands are re-read by other tiles
      pdl_wait();
      Ring ring;     // ring position of the next k block
      int issued = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x) {
        const int mt = t % a.mtiles, nt = t / a.mtiles;
        const int rt0 = nt * 2;
        const int rt1 = rt0 + 1 < a.rtiles ? rt0 + 1 : rt0;  // past N: reload a valid tile, rows are masked
        const uint8_t* w0 = a.wtiles + static_cast<size_t>(rt0) * nkb * 16384;
        const uint8_t* w1 = a.wtiles + static_cast<size_t>(rt1) * nkb * 16384;
        for (int kb = 0; kb < nkb; ++kb, ++issued, ring.next(stages)) {
          const int s = ring.slot;
          if (!mbar_wait(&empty[s], ring.phase ^ 1u, kErrTcProducer)) {
            ok = false;
            break;
          }
          mbar_expect_tx(&full[s], static_cast<uint32_t>(kGmABytes + kGmBBytes));
          tma_load_2d(sa + static_cast<size_t>(s) * kGmABytes, &tmx, &full[s], kb * 64, mt * 128, pol_keep);
          uint8_t* bdst = sb + static_cast<size_t>(s) * kGmBBytes;
          bulk_g2s(bdst, w0 + static_cast<size_t>(kb) * 16384, 16384, &full[s], pol_keep);
          bulk_g2s(bdst + 16384, w1 + static_cast<size_t>(kb) * 16384, 16384, &full[s], pol_keep);
        }
      }
      for (int i = (issued > stages ? issued - stages : 0); i < issued; ++i)
        mbar_wait(&full[i % stages], static_cast<uint32_t>((i / stages) & 1), kErrDrain, kWaitLimitNs / 10);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      Ring ring;
      int local = 0;
      bool ok = true;
      for (int t = blockIdx.x; t < tiles && ok; t += gridDim.x, ++local) {
        const int b = local & 1;
        ok = mbar_wait(&acc_empty[b], static_cast<uint32_t>((local >> 1) & 1) ^ 1u, kErrTcMma);
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * kGmBN);
        for (int kb = 0; kb < nkb && ok; ++kb, ring.next(stages)) {
          const int s = ring.slot;
          if (!mbar_wait(&full[s], ring.phase, kErrTcMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(smem_u32(sa + static_cast<size_t>(s) * kGmABytes));
          const uint64_t db = umma_desc_sw128(smem_u32(sb + static_cast<size_t>(s) * kGmBBytes));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_bf16(d, da + 2 * kk, db + 2 * kk, kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit(&empty[s]);
        }
        umma_commit(&acc_full[b]);
      }
    }
  } else {
    // Epilogue: thread row = TMEM lane = token within the tile.
    const int q = warp & 3;
    const int row = q * 32 + lane;
    bool waited = false;
    int local = 0;
    const bool vec_ok = (a.N % 8) == 0;
    for (int t = blockIdx.x; t < tiles; t += gridDim.x, ++local) {
      const int b = local & 1;
      const int mt = t % a.mtiles, nt = t / a.mtiles;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[b], static_cast<uint32_t>((local >> 1) & 1),
                                                        kErrTcEpilogue));
      tc_fence_after();
      if (!waited) {
        if (tracing) t_main = globaltimer();
        pdl_wait();
        waited = true;
      }
      if (!ok) break;
      const int m = mt * 128 + row;
      const int n0 = nt * kGmBN;
      uint16_t* yrow = a.y + static_cast<size_t>(m) * a.N;
#pragma unroll 1
      for (int c = 0; c < kGmBN; c += 16) {
        float v[16];
        tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * kGmBN + c), v);
        const int n = n0 + c;
        if (m < a.M && n < a.N) {
          if (vec_ok && n + 16 <= a.N) {
            uint4 p0, p1;
            p0.x = pack_bf16x2(v[0], v[1]);
            p0.y = pack_bf16x2(v[2], v[3]);
            p0.z = pack_bf16x2(v[4], v[5]);
            p0.w = pack_bf16x2(v[6], v[7]);
            p1.x = pack_bf16x2(v[8], v[9]);
            p1.y = pack_bf16x2(v[10], v[11]);
            p1.z = pack_bf16x2(v[12], v[13]);
            p1.w = pack_bf16x2(v[14], v[15]);
            uint4* dst = reinterpret_cast<uint4*>(yrow + n);
            dst[0] = p0;
            dst[1] = p1;
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j)
              if (n + j < a.N) yrow[n + j] = f32_to_bf16(v[j]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
    }
    if (!waited) pdl_wait();
  }
  pdl_launch_dependents();

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kGmCols);
  }
  if (tracing) a.trace[blockIdx.x] = TraceRec{t_start, t_ready, t_main, globaltimer(), smid(), blockIdx.x, 0u, 0u};
}

}  // namespace muse
