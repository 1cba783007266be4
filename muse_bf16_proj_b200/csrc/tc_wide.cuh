// Persistent tcgen05 GEMM over CTA pairs with 256 (tokens) x 512 (W rows) tiles, for prefill
// shapes with many W rows: y[m, n] = sum_k x[m, k] * W[n, k].
//
// The pair computes its tile as two cta_group::2 UMMAs a k step (M = 256, N = 256, K = 16) into
// two 256-column TMEM accumulators, both reading the same x stage. CTA r of the pair holds tokens
// r * 128 .. + 127 of A and, of each 256-row half h of the tile's W rows, rows h * 256 + r * 128
// .. + 127 (one packed 128-row tile) of B. A stage is 48 KB a CTA (x 16 KB + two W halves), so x
// crosses from L2 into shared memory once per 512 W rows instead of once per 256 (the 256 x 256
// pair GEMM): a quarter fewer operand bytes a FLOP, the traffic that bounds the pair GEMM's clock
// under the power cap.
//
// The two accumulators fill all 512 TMEM columns, so a tile's epilogue cannot hide behind the
// next tile's UMMAs entirely: the epilogue warps drain accumulator 0 and release it before
// draining accumulator 1, and the UMMA issuer runs the next tile's first k blocks on accumulator 0
// while accumulator 1 drains (up to stages - 1 k blocks ahead), then catches accumulator 1 up.
//
// Tiles are walked in groups of token tiles (as the 256 x 256 pair GEMM does), the group's x kept
// in L2 while W streams past. W tiles past N are read in bounds and their rows never stored.
//
// Warp roles (192 threads a CTA): warp 0 producer (lane 0), warp 1 TMEM owner + UMMA issuer
// (lane 0 of the pair's even CTA), warps 2..5 epilogue (TMEM lane quarter = warp % 4).
#pragma once

#include "ptx.cuh"
#include "tc_gemm.cuh"  // pack_bf16x2

namespace muse {

constexpr int kWdThreads = 192;
constexpr int kWdHalf = 16384;        // 128 rows x 64 k of BF16
constexpr int kWdStage = 3 * kWdHalf;  // x, W half 0, W half 1 (per CTA)
constexpr uint32_t kWdCols = 512;
constexpr unsigned int kErrWdProducer = 0x801, kErrWdMma = 0x802, kErrWdEpilogue = 0x803;

constexpr int kWdStg = 32768;  // y staging for the tensor-store epilogue: 128 token rows x 128 W rows of BF16
__host__ __device__ constexpr int wd_smem(int stages, bool tma_y = false) {
  return 1024 + stages * kWdStage + (tma_y ? kWdStg : 0) + (2 * stages + 6) * 8 + 32;
}

struct WdArgs {
  uint16_t* y;  // [M, N]
  int M, N, stages;
  int mtiles, ntiles, nkb, rtiles;  // 256-token tiles, 512-row tiles, k blocks, 128-row packed tiles
  int group_m;                      // token tiles walked together
  int tma_y;                        // 1: y written by TMA tensor stores from a staging tile (N % 8 == 0)
  TraceRec* trace;
  int trace_cap;
};

__device__ __forceinline__ void wd_tile_coords(const WdArgs& a, int t, int& mt, int& nt) {
  const int per_group = a.group_m * a.ntiles;
  const int g = t / per_group, w = t - g * per_group;
  const int m0 = g * a.group_m;
  const int gm = min(a.group_m, a.mtiles - m0);
  mt = m0 + w % gm;
  nt = w / gm;
}

__global__ void __launch_bounds__(kWdThreads, 1)
    tc_wide_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                   const __grid_constant__ CUtensorMap tmy, const WdArgs a) {
  constexpr uint32_t kIdesc = umma_idesc_bf16(256, 256);
  extern __shared__ uint8_t smem_raw[];
  const bool tracing = a.trace != nullptr && static_cast<int>(blockIdx.x) < a.trace_cap && threadIdx.x == 64;
  const unsigned long long t_start = tracing ? globaltimer() : 0ull;
  unsigned long long t_ready = 0ull, t_main = 0ull;
  uint8_t* smem = smem_align<1024>(smem_raw);
  const int stages = a.stages;
  // Stage s: x at s * 48 KB, W half 0 at + 16 KB, W half 1 at + 32 KB; then (tma_y) the y staging tile:
  // two 16 KB sub-tiles of 128 token rows x 64 W rows in the 128-byte-swizzled order of the y map.
  uint8_t* ystg = smem + static_cast<size_t>(stages) * kWdStage;
  uint64_t* full = reinterpret_cast<uint64_t*>(ystg + (a.tma_y ? kWdStg : 0));
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;  // [1] both accumulators of a tile complete
  uint64_t* acc_empty = acc_full + 1;   // [2] accumulator h drained (even CTA: 4 local + 4 remote arrives)
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* epi_abort = reinterpret_cast<int*>(tmem_slot + 1);  // tma_y: an epilogue warp's accumulator wait failed

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  const int tiles = a.mtiles * a.ntiles;
  const int nkb = a.nkb;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmx);
    prefetch_tensormap(&tmw);
    if (a.tma_y) prefetch_tensormap(&tmy);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(&acc_empty[0], 8);
    mbar_init(&acc_empty[1], 8);
    *epi_abort = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, kWdCols);
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tracing) t_ready = globaltimer();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_x = policy_evict_last();  // re-read by every W tile of the group
      const uint64_t pol_w = a.mtiles > 1 ? policy_evict_normal() : policy_evict_first();
      pdl_wait();
      Ring ring;
      int issued = 0;
      bool ok = true;
      for (int t = pair; ok && t < tiles; t += npairs) {
        int mt, nt;
        wd_tile_coords(a, t, mt, nt);
        const int xrow = mt * 256 + static_cast<int>(rank) * 128;
        int rt0 = nt * 4 + static_cast<int>(rank), rt1 = rt0 + 2;
        if (rt0 >= a.rtiles) rt0 = a.rtiles - 1;  // past N: a valid tile; its rows are never stored
        if (rt1 >= a.rtiles) rt1 = a.rtiles - 1;
        for (int kb = 0; kb < nkb; ++kb, ++issued, ring.next(stages)) {
          const int s = ring.slot;
          if (!mbar_wait(&empty[s], ring.phase ^ 1u, kErrWdProducer)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(&full[s], static_cast<uint32_t>(2 * kWdStage));
          const uint32_t bar = map_peer(smem_u32(&full[s]), 0u);
          uint8_t* st = smem + static_cast<size_t>(s) * kWdStage;
          tma_load_2d_pair(st, &tmx, bar, kb * 64, xrow, pol_x);
          tma_load_2d_pair(st + kWdHalf, &tmw, bar, 0, (rt0 * nkb + kb) * 128, pol_w);
          tma_load_2d_pair(st + 2 * kWdHalf, &tmw, bar, 0, (rt1 * nkb + kb) * 128, pol_w);
        }
      }
      // Every load this CTA issued is consumed (and so has landed) once its stage is released.
      for (int i = (issued > stages ? issued - stages : 0); i < issued; ++i)
        mbar_wait(&empty[i % stages], static_cast<uint32_t>((i / stages) & 1), kErrDrain, kWaitLimitNs / 10);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      Ring ring;  // the next stage to consume
      bool ok = true;
      int local = 0;
      const int ahead_max = stages - 1 < nkb ? stages - 1 : nkb;
      for (int t = pair; ok && t < tiles; t += npairs, ++local) {
        const uint32_t par = static_cast<uint32_t>(local & 1) ^ 1u;  // the previous tile's drains
        // Accumulator 0 alone for the first `ahead` k blocks (their stages kept), while
        // accumulator 1 may still be draining; then accumulator 1 catches up on those stages.
        if (!mbar_wait(&acc_empty[0], par, kErrWdMma)) break;
        tc_fence_after();
        int ahead = 0;
        Ring r = ring;
        for (; ahead < ahead_max; ++ahead, r.next(stages)) {
          if (!mbar_wait(&full[r.slot], r.phase, kErrWdMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* st = smem + static_cast<size_t>(r.slot) * kWdStage;
          const uint64_t da = umma_desc_sw128(smem_u32(st)), db0 = umma_desc_sw128(smem_u32(st + kWdHalf));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16_pair(tmem, da + 2 * kk, db0 + 2 * kk, kIdesc, (ahead > 0 || kk > 0) ? 1u : 0u);
        }
        if (!ok || !mbar_wait(&acc_empty[1], par, kErrWdMma)) {
          umma_commit_pair_mc(acc_full, 0x3);
          break;
        }
        tc_fence_after();
        for (int kb = 0; kb < ahead; ++kb, ring.next(stages)) {
          const uint8_t* st = smem + static_cast<size_t>(ring.slot) * kWdStage;
          const uint64_t da = umma_desc_sw128(smem_u32(st)), db1 = umma_desc_sw128(smem_u32(st + 2 * kWdHalf));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16_pair(tmem + 256u, da + 2 * kk, db1 + 2 * kk, kIdesc, (kb > 0 || kk > 0) ? 1u : 0u);
          umma_commit_pair_mc(&empty[ring.slot], 0x3);
        }
        for (int kb = ahead; kb < nkb; ++kb, ring.next(stages)) {
          if (!mbar_wait(&full[ring.slot], ring.phase, kErrWdMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* st = smem + static_cast<size_t>(ring.slot) * kWdStage;
          const uint64_t da = umma_desc_sw128(smem_u32(st));
          const uint64_t db0 = umma_desc_sw128(smem_u32(st + kWdHalf)), db1 = umma_desc_sw128(smem_u32(st + 2 * kWdHalf));
          const uint32_t acc0 = kb > 0 ? 1u : 0u;
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) {
            umma_bf16_pair(tmem, da + 2 * kk, db0 + 2 * kk, kIdesc, (acc0 | kk) ? 1u : 0u);
            umma_bf16_pair(tmem + 256u, da + 2 * kk, db1 + 2 * kk, kIdesc, (acc0 | kk) ? 1u : 0u);
          }
          umma_commit_pair_mc(&empty[ring.slot], 0x3);
        }
        umma_commit_pair_mc(acc_full, 0x3);  // also on the error path, so the epilogues' waits end
      }
    }
  } else {
    // Epilogue warps 2..5: TMEM lane quarter q = token rows q * 32 .. + 31 of this CTA's 128.
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const bool vec_ok = (a.N % 8) == 0;
    bool waited = false;
    int local = 0;
    for (int t = pair; t < tiles; t += npairs, ++local) {
      int mt, nt;
      wd_tile_coords(a, t, mt, nt);
      bool ok = __all_sync(0xffffffffu, mbar_wait_idle(acc_full, static_cast<uint32_t>(local & 1), kErrWdEpilogue));
      if (a.tma_y) {  // the four warps share named barriers below: the same answer in all of them
        if (!ok && lane == 0) *epi_abort = 1;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        ok = *reinterpret_cast<volatile int*>(epi_abort) == 0;
      }
      tc_fence_after();
      if (!waited) {
        if (tracing) t_main = globaltimer();
        pdl_wait();
        waited = true;
      }
      if (!ok) break;
      const int m = mt * 256 + static_cast<int>(rank) * 128 + row;
      uint16_t* yrow = a.y + static_cast<size_t>(m) * a.N;
#pragma unroll 1
      for (int h = 0; h < 2; ++h) {
        const int n0 = nt * 512 + h * 256;
        if (a.tma_y) {
          // Two rounds of 128 W rows: TMEM -> BF16 -> the swizzled staging tile -> two tensor stores
          // (rows and columns past M and N clipped by the store). The staging is reused only after the
          // previous round's stores have read it.
          const uint32_t stg = smem_u32(ystg);
#pragma unroll 1
          for (int r = 0; r < 2; ++r) {
            if (threadIdx.x == 64) bulk_wait_read_all();
            asm volatile("bar.sync 1, 128;" ::: "memory");
#pragma unroll 1
            for (int cc = 0; cc < 4; ++cc) {  // 32 W rows each: sub-tile cc / 2, 16-byte chunks 4 (cc % 2) .. + 3
              float v[32];
              tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(h * 256 + r * 128 + cc * 32), v);
              const uint32_t sub = stg + static_cast<uint32_t>((cc >> 1) * 16384 + row * 128);
#pragma unroll
              for (int j = 0; j < 4; ++j) {
                const uint32_t chunk = static_cast<uint32_t>(((cc & 1) * 4 + j) ^ (row & 7));
                st_shared_v4u(sub + chunk * 16u, pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                              pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
              }
            }
            fence_proxy_async_shared();  // the staged rows before the tensor stores read them
            asm volatile("bar.sync 1, 128;" ::: "memory");
            if (threadIdx.x == 64) {
              const int row0 = mt * 256 + static_cast<int>(rank) * 128;
              const uint64_t pol_y = policy_evict_first();  // written once, never re-read here
              tma_store_2d_hint(&tmy, ystg, n0 + r * 128, row0, pol_y);
              tma_store_2d_hint(&tmy, ystg + 16384, n0 + r * 128 + 64, row0, pol_y);
              bulk_commit();
            }
          }
        } else {
#pragma unroll 1
        for (int c = 0; c < 256; c += 32) {
          float v[32];
          tmem_ld32(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(h * 256 + c), v);
          const int n = n0 + c;
          if (m < a.M && n < a.N) {
            if (vec_ok && n + 32 <= a.N) {
              uint4* dst = reinterpret_cast<uint4*>(yrow + n);
#pragma unroll
              for (int j = 0; j < 4; ++j)
                dst[j] = make_uint4(pack_bf16x2(v[8 * j], v[8 * j + 1]), pack_bf16x2(v[8 * j + 2], v[8 * j + 3]),
                                    pack_bf16x2(v[8 * j + 4], v[8 * j + 5]), pack_bf16x2(v[8 * j + 6], v[8 * j + 7]));
            } else {
#pragma unroll
              for (int j = 0; j < 32; ++j)
                if (n + j < a.N) yrow[n + j] = f32_to_bf16(v[j]);
            }
          }
        }
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_peer(smem_u32(&acc_empty[h]), 0u));
      }
    }
    if (!waited) pdl_wait();
    if (a.tma_y && threadIdx.x == 64) bulk_wait_all();  // every tensor store of y has completed
  }
  pdl_launch_dependents();

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the pair's UMMAs and both epilogues are done before either CTA frees TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kWdCols);
  }
  if (tracing) a.trace[blockIdx.x] = TraceRec{t_start, t_ready, t_main, globaltimer(), smid(), blockIdx.x, 0u, 0u};
}

}  // namespace muse
