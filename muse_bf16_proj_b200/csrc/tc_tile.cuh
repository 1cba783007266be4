// tcgen05 tile GEMM with W as the UMMA A operand: y[m, n] = sum_k x[m, k] * W[n, k].
//
// One CTA computes a 128 (rows of W) x BNT (tokens) FP32 tile in TMEM over a K range. W and x
// both stay K-major in global memory and arrive by 2-D TMA (128-byte swizzle, no multicast) into
// a `stages`-deep shared-memory ring; one thread issues the UMMAs (M = 128, N = BNT, K = 16);
// four epilogue warps read the accumulator back with tcgen05.ld.
//
// Split-K: the `split` CTAs of a thread-block cluster take consecutive K ranges of the same tile.
// Each parks its FP32 partial in its own shared memory; after a cluster barrier, CTA r sums the
// tokens j = r, r + split, ... over all peers' partials through DSMEM in rank order 0..split-1 and
// stores BF16. One launch, no global scratch, deterministic.
//
// Warp roles (192 threads): warp 0 = TMA producer, warp 1 = TMEM owner + UMMA issuer,
// warps 2..5 = epilogue (warp w reads TMEM lanes 32 * (w % 4) .. + 31).
#pragma once

#include "ptx.cuh"

namespace muse {

constexpr int kTcThreads = 192;
constexpr int kTcBK = 64;                   // K elements per stage (128 bytes of BF16)
constexpr int kTcABytes = 128 * kTcBK * 2;  // 16 KB: 128 W rows

__host__ __device__ constexpr int tc_tile_bbytes(int bnt) { return bnt * kTcBK * 2; }
__host__ __device__ constexpr int tc_tile_tmem_cols(int bnt) { return bnt < 32 ? 32 : bnt; }

// Shared memory bytes the kernel needs (plus up to 1 KB of alignment slack).
__host__ __device__ constexpr int tc_tile_smem(int bnt, int stages) {
  return 1024 + stages * (kTcABytes + tc_tile_bbytes(bnt)) + (2 * stages + 1) * 8 + 16;
}

template <int BNT>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_tile_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
                   uint16_t* __restrict__ y, int M, int N, int K, int split, int stages) {
  constexpr int kBBytes = tc_tile_bbytes(BNT);
  constexpr uint32_t kCols = tc_tile_tmem_cols(BNT);
  constexpr uint32_t kIdesc = umma_idesc_bf16(128, BNT);
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
  uint8_t* sa = smem;
  uint8_t* sb = smem + static_cast<size_t>(stages) * kTcABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + static_cast<size_t>(stages) * kBBytes);
  uint64_t* empty = full + stages;
  uint64_t* accf = empty + stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  float* part = reinterpret_cast<float*>(smem);  // [BNT][128], reuses the ring after the main loop

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = split > 1 ? cluster_ctarank() : 0u;
  const int rt = blockIdx.x / split;
  const int tt = blockIdx.y;
  const int nkb = (K + kTcBK - 1) / kTcBK;
  const int kb0 = static_cast<int>(static_cast<long long>(rank) * nkb / split);
  const int kb1 = static_cast<int>(static_cast<long long>(rank + 1) * nkb / split);
  const int nk = kb1 - kb0;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmw);
    prefetch_tensormap(&tmx);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      int issued = 0;
      for (int i = 0; i < nk; ++i) {
        const int s = i % stages;
        if (!mbar_wait(&empty[s], ((i / stages) & 1) ^ 1, kErrTcProducer)) break;
        mbar_expect_tx(&full[s], static_cast<uint32_t>(kTcABytes + kBBytes));
        const int kc = (kb0 + i) * kTcBK;
        tma_load_2d(sa + static_cast<size_t>(s) * kTcABytes, &tmw, &full[s], kc, rt * 128, pol_w);
        tma_load_2d(sb + static_cast<size_t>(s) * kBBytes, &tmx, &full[s], kc, tt * BNT, pol_x);
        ++issued;
      }
      for (int i = max(0, issued - stages); i < issued; ++i)
        mbar_wait(&full[i % stages], (i / stages) & 1, kErrDrain, kWaitLimitNs / 10);
    }
  } else if (warp == 1) {
    if (lane == 0) {
      for (int i = 0; i < nk; ++i) {
        const int s = i % stages;
        if (!mbar_wait(&full[s], (i / stages) & 1, kErrTcMma)) break;
        tc_fence_after();
        const uint64_t da = umma_desc_sw128(smem_u32(sa + static_cast<size_t>(s) * kTcABytes));
        const uint64_t db = umma_desc_sw128(smem_u32(sb + static_cast<size_t>(s) * kBBytes));
#pragma unroll
        for (int kk = 0; kk < kTcBK / 16; ++kk)  // 16 elements = 32 bytes = 2 descriptor units
          umma_bf16(tmem, da + 2 * kk, db + 2 * kk, kIdesc, (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit(&empty[s]);  // frees the stage once these UMMAs have read it
      }
      umma_commit(accf);  // always: also fences any UMMA still in flight on the error path
    }
  } else {
    // Epilogue warps 2..5.
    const int q = warp & 3;
    const int rl = q * 32 + lane;  // this thread's TMEM lane = W row within the tile
    const int n = rt * 128 + rl;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(accf, 0, kErrTcEpilogue));  // tcgen05.ld is warp-wide
    tc_fence_after();
    if (ok) {
#pragma unroll 1
      for (int c = 0; c < BNT; c += 16) {
        float v[16];
        tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(c), v);
        if (split == 1) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = tt * BNT + c + j;
            if (m < M && n < N) y[static_cast<size_t>(m) * N + n] = f32_to_bf16(v[j]);
          }
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) part[(c + j) * 128 + rl] = v[j];
        }
      }
    }
  }

  if (split > 1) {
    cluster_sync();  // every peer's partial is in its shared memory
    if (warp >= 2) {
      const int rl = threadIdx.x - 64;
      const int n = rt * 128 + rl;
      const uint32_t mine = smem_u32(part);
      for (int j = static_cast<int>(rank); j < BNT; j += split) {
        const int m = tt * BNT + j;
        if (m >= M) break;
        const uint32_t off = static_cast<uint32_t>((j * 128 + rl) * 4);
        float sum = 0.f;
        for (int p = 0; p < split; ++p) sum += ld_dsmem_f32(map_peer(mine + off, static_cast<uint32_t>(p)));
        if (n < N) y[static_cast<size_t>(m) * N + n] = f32_to_bf16(sum);
      }
    }
    cluster_sync();  // no CTA leaves while a peer may still read its partial
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
}

}  // namespace muse
