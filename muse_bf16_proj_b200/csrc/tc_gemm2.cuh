// Persistent tcgen05 GEMM over CTA pairs for prefill shapes: y[m, n] = sum_k x[m, k] * W[n, k].
//
// A cluster of 2 CTAs computes one 256 (tokens) x 256 (W rows) FP32 tile with cta_group::2 UMMAs
// (M = 256, N = 256, K = 16): CTA r of the pair holds tokens r * 128 .. + 127 of A and W rows
// r * 128 .. + 127 of B in its own shared memory, and its TMEM receives its 128 tokens x 256
// columns of D. Per stage each CTA loads 16 KB of x (2-D TMA, 128-byte swizzle) and one 16 KB
// packed W tile (2-D TMA over the tile array with no swizzle: the tile is already in swizzled
// order, so the copy is one contiguous 16 KB read); both loads complete on the even CTA's
// mbarrier (cta_group::2 form, no multicast), which expects the pair's 64 KB. The even CTA alone
// issues the UMMAs and commits to both CTAs' barriers. Each CTA only stages half of B, so a
// stage is 32 KB and six fit: twice the bytes in flight of the single-CTA kernel for the same
// UMMA work, and half of its B traffic per FLOP.
//
// Pairs walk the 256 x 256 tiles persistently in groups of token tiles (g2_tile_coords). Two TMEM accumulators
// (2 x 256 columns) overlap a tile's epilogue with the next tile's UMMAs; the odd CTA's epilogue
// warps release an accumulator with remote arrives on the even CTA's barrier.
#pragma once

#include "gather.cuh"
#include "ptx.cuh"
#include "tc12.cuh"     // t12_start / t12_owner: stream-K ranges
#include "tc_gemm.cuh"  // pack_bf16x2

namespace muse {

constexpr int kG2Threads = 192;
constexpr int kG2Half = 16384;                 // 128 rows x 64 k of BF16
constexpr int kG2Stage = 2 * kG2Half;          // x half + W half, per CTA
constexpr uint32_t kG2Cols = 512;

__host__ __device__ constexpr int g2_smem(int stages) { return 1024 + stages * kG2Stage + (2 * stages + 4) * 8 + 32; }
// The all-gather variant adds a 4 KB staging tile per epilogue warp (32 rows x 64 columns of BF16),
// so its stores leave as 128-byte row segments instead of 16 bytes on 32 different rows.
constexpr int kG2GatherStage = 4 * 32 * 128;
__host__ __device__ constexpr int g2_smem_gather(int stages) { return g2_smem(stages) + 128 + kG2GatherStage; }

struct G2Args {
  uint16_t* y;  // [M, N]
  int M, N, K, stages;
  int mtiles, ntiles, nkb, rtiles;  // 256-token tiles, 256-row tiles, k blocks, 128-row packed tiles
  int group_m;  // token tiles walked together: a group's x stays in L2 while all of W streams past it
  TraceRec* trace;
  int trace_cap;
  GatherOut g;  // kGather: every value also goes to each rank's y_full (y is unused)
  // Stream-K (streamk != 0): the (tile, k block) units are cut into equal runs, one per pair; a tile
  // shared by several pairs leaves FP32 partials in `partials` ([tile][contributor][CTA][64][128]
  // float4: column quad c of row r at c * 128 + r) and its last contributor adds them in order.
  int streamk, smax;
  // Tiles below sk_tile0 are walked persistently (whole tiles, no partials); stream-K covers the
  // units of the tiles from sk_tile0 on (0: every tile). A tile's partials and counters are indexed
  // from sk_tile0.
  int sk_tile0;
  float4* partials;
  int* counters;  // [tiles - sk_tile0][2], zero between launches
};

// Tile t's coordinates in the grouped order: groups of `group_m` token tiles (the last one
// smaller), each group walking every W tile with its token tiles fastest. A wave of the pairs then
// covers a few W tiles times the group's token tiles, so the group's x (group_m x 256 rows) is
// read from HBM once and stays in L2 while W streams past it, and each W tile is read once a group
// (mtiles / group_m times in all) instead of x being re-read for every W tile.
__device__ __forceinline__ void g2_tile_coords(const G2Args& a, int t, int& mt, int& nt) {
  const int per_group = a.group_m * a.ntiles;
  const int g = t / per_group, w = t - g * per_group;
  const int m0 = g * a.group_m;
  const int gm = min(a.group_m, a.mtiles - m0);
  mt = m0 + w % gm;
  nt = w / gm;
}

// The segments one pair computes, in order: whole tiles pair, pair + npairs, ... below the stream-K
// start (all tiles without stream-K), then under stream-K the pair's run of the remaining
// (tile, k block) units cut at tile boundaries.
struct G2Segs {
  long long u, u1;
  int t, step, t_end, nkb;
  bool sk;
  __device__ G2Segs(const G2Args& a, int pair, int npairs) {
    const int tiles = a.mtiles * a.ntiles;
    nkb = a.nkb;
    sk = a.streamk != 0;
    t = pair;
    step = npairs;
    t_end = sk ? a.sk_tile0 : tiles;
    const long long base = static_cast<long long>(a.sk_tile0) * nkb;
    const long long units = static_cast<long long>(tiles) * nkb - base;
    u = sk ? base + t12_start(pair, units, npairs) : 0;
    u1 = sk ? base + t12_start(pair + 1, units, npairs) : 0;
  }
  __device__ bool next(int& tile, int& kb0, int& kb1) {
    if (t < t_end) {
      tile = t;
      kb0 = 0;
      kb1 = nkb;
      t += step;
      return true;
    }
    if (!sk || u >= u1) return false;
    tile = static_cast<int>(u / nkb);
    kb0 = static_cast<int>(u - static_cast<long long>(tile) * nkb);
    kb1 = static_cast<int>(min(static_cast<long long>(nkb), kb0 + (u1 - u)));
    u += kb1 - kb0;
    return true;
  }
};

// kGather: the all-gather epilogue of gather.cuh instead of stores into y.
template <bool kGather>
__global__ void __launch_bounds__(kG2Threads, 1)
    tc_gemm2_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw, const G2Args a) {
  constexpr uint32_t kIdesc = umma_idesc_bf16(256, 256);
  extern __shared__ uint8_t smem_raw[];
  const bool tracing = a.trace != nullptr && static_cast<int>(blockIdx.x) < a.trace_cap && threadIdx.x == 64;
  const unsigned long long t_start = tracing ? globaltimer() : 0ull;
  unsigned long long t_ready = 0ull, t_main = 0ull;
  uint8_t* smem = smem_align<1024>(smem_raw);
  const int stages = a.stages;
  uint8_t* sa = smem;
  uint8_t* sb = smem + static_cast<size_t>(stages) * kG2Half;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + static_cast<size_t>(stages) * kG2Half);
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;  // [2]
  uint64_t* acc_empty = acc_full + 2;   // [2], used in the even CTA: 4 local + 4 remote arrives
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* epi_flag = reinterpret_cast<int*>(tmem_slot + 1);  // stream-K: [0] abort, [1] last contributor
  uint4* gather_stage = reinterpret_cast<uint4*>(smem_align<128>(reinterpret_cast<uint8_t*>(epi_flag + 2)));

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int npairs = gridDim.x >> 1;
  const int tiles = a.mtiles * a.ntiles;
  const int nkb = a.nkb;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmx);
    prefetch_tensormap(&tmw);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 8);
    }
    epi_flag[0] = epi_flag[1] = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, kG2Cols);
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tracing) t_ready = globaltimer();

  if (warp == 0) {
    if (lane == 0) {
      // x is re-read by every pair working on its token tile: keep it. A W tile is read by the
      // group's pairs at about the same time and not again until the next group: normal priority
      // with several token tiles, evict-first with one (M <= 256: W streams through once).
      const uint64_t pol = policy_evict_last();
      const uint64_t pol_w = a.mtiles > 1 ? policy_evict_normal() : policy_evict_first();
      pdl_wait();
      if constexpr (kGather) gather_announce(a.g, gather_epoch(a.g));  // early, so peers rarely wait
      Ring ring;     // ring position of the next k block
      int issued = 0;
      bool ok = true;
      G2Segs segs(a, pair, npairs);
      int t, kb0, kb1;
      while (ok && segs.next(t, kb0, kb1)) {
        int mt, nt;
        g2_tile_coords(a, t, mt, nt);
        const int xrow = mt * 256 + static_cast<int>(rank) * 128;
        int rt = nt * 2 + static_cast<int>(rank);
        if (rt >= a.rtiles) rt = nt * 2;  // past N: a valid tile; its rows are never stored
        for (int kb = kb0; kb < kb1; ++kb, ++issued, ring.next(stages)) {
          const int s = ring.slot;
          if (!mbar_wait(&empty[s], ring.phase ^ 1u, kErrTcProducer)) {
            ok = false;
            break;
          }
          if (leader) mbar_expect_tx(&full[s], static_cast<uint32_t>(2 * kG2Stage));
          const uint32_t bar = map_peer(smem_u32(&full[s]), 0u);
          tma_load_2d_pair(sa + static_cast<size_t>(s) * kG2Half, &tmx, bar, kb * 64, xrow, pol);
          tma_load_2d_pair(sb + static_cast<size_t>(s) * kG2Half, &tmw, bar, 0, (rt * nkb + kb) * 128, pol_w);
        }
      }
      // Every load this CTA issued is consumed (and so has landed) once its stage is released.
      for (int i = (issued > stages ? issued - stages : 0); i < issued; ++i)
        mbar_wait(&empty[i % stages], static_cast<uint32_t>((i / stages) & 1), kErrDrain, kWaitLimitNs / 10);
    }
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      Ring ring;
      int local = 0;
      bool ok = true;
      G2Segs segs(a, pair, npairs);
      int t, kb0, kb1;
      for (; ok && segs.next(t, kb0, kb1); ++local) {
        const int b = local & 1;
        ok = mbar_wait(&acc_empty[b], static_cast<uint32_t>((local >> 1) & 1) ^ 1u, kErrTcMma);
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * 256);
        for (int kb = kb0; kb < kb1 && ok; ++kb, ring.next(stages)) {
          const int s = ring.slot;
          if (!mbar_wait(&full[s], ring.phase, kErrTcMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(smem_u32(sa + static_cast<size_t>(s) * kG2Half));
          const uint64_t db = umma_desc_sw128(smem_u32(sb + static_cast<size_t>(s) * kG2Half));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk)
            umma_bf16_pair(d, da + 2 * kk, db + 2 * kk, kIdesc, (kb > kb0 || kk > 0) ? 1u : 0u);
          umma_commit_pair_mc(&empty[s], 0x3);
        }
        umma_commit_pair_mc(&acc_full[b], 0x3);
      }
    }
  } else {
    const int q = warp & 3;
    const int row = q * 32 + lane;
    const bool vec_ok = (a.N % 8) == 0;
    bool waited = false, peers = false;
    unsigned int epoch = 0u;
    int local = 0;
    G2Segs segs(a, pair, npairs);
    int t, kb0, kb1;
    for (; segs.next(t, kb0, kb1); ++local) {
      const int b = local & 1;
      int mt, nt;
      g2_tile_coords(a, t, mt, nt);
      bool ok = __all_sync(0xffffffffu, mbar_wait_idle(&acc_full[b], static_cast<uint32_t>((local >> 1) & 1),
                                                  kErrTcEpilogue));
      tc_fence_after();
      if (a.streamk) {
        // The four epilogue warps take the same named barriers below: agree on one answer first.
        if (!ok && lane == 0) epi_flag[0] = 1;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        ok = *reinterpret_cast<volatile int*>(&epi_flag[0]) == 0;
      }
      if (!waited) {
        if (tracing) t_main = globaltimer();
        pdl_wait();
        waited = true;
        if constexpr (kGather) {
          epoch = gather_epoch(a.g);
          peers = gather_arrived(a.g, epoch);
        }
      }
      if (!ok) break;
      const int m = mt * 256 + static_cast<int>(rank) * 128 + row;
      const int n0 = nt * 256;
      if (a.streamk && !(kb0 == 0 && kb1 == nkb)) {
        // Part of a tile shared with other pairs: park this CTA's 128 x 256 FP32 partial, release
        // the accumulator, take the tile's ticket; the last contributor adds every partial in
        // contributor order and stores BF16.
        const long long base = static_cast<long long>(a.sk_tile0) * nkb;
        const long long units = static_cast<long long>(tiles) * nkb - base;
        const int first = t12_owner(static_cast<long long>(t) * nkb - base, units, npairs);
        const int nseg = t12_owner(static_cast<long long>(t + 1) * nkb - 1 - base, units, npairs) - first + 1;
        const int ts = t - a.sk_tile0;  // this tile among the stream-K ones
        float4* tp = a.partials + static_cast<size_t>(ts) * a.smax * 2 * 64 * 128;  // this tile's partials
        float4* mine = tp + (static_cast<size_t>(pair - first) * 2 + rank) * 64 * 128;
#pragma unroll 1
        for (int c = 0; c < 256; c += 16) {
          float v[16];
          tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * 256 + c), v);
#pragma unroll
          for (int j = 0; j < 4; ++j)
            __stcg(mine + (c / 4 + j) * 128 + row, make_float4(v[4 * j], v[4 * j + 1], v[4 * j + 2], v[4 * j + 3]));
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_peer(smem_u32(&acc_empty[b]), 0u));
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (row == 0) epi_flag[1] = (ticket_acq_rel(a.counters + ts * 2 + static_cast<int>(rank)) == nseg - 1) ? 1 : 0;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (epi_flag[1]) {
          const float4* part = tp + static_cast<size_t>(rank) * 64 * 128 + row;
          uint16_t* yrow = a.y + static_cast<size_t>(m) * a.N;
          // 16 column quads at a time with every contributor's 16 loads in flight together, added
          // in contributor order.
#pragma unroll 1
          for (int c0 = 0; c0 < 64; c0 += 16) {
            float4 sum[16];
#pragma unroll
            for (int j = 0; j < 16; ++j) sum[j] = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 1
            for (int p = 0; p < nseg; ++p) {
              float4 v[16];
#pragma unroll
              for (int j = 0; j < 16; ++j) v[j] = __ldcg(part + (static_cast<size_t>(p) * 2 * 64 + c0 + j) * 128);
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                sum[j].x += v[j].x;
                sum[j].y += v[j].y;
                sum[j].z += v[j].z;
                sum[j].w += v[j].w;
              }
            }
            if (m < a.M) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int n = n0 + (c0 + j) * 4;
                if (vec_ok && n + 4 <= a.N) {
                  *reinterpret_cast<uint2*>(yrow + n) =
                      make_uint2(pack_bf16x2(sum[j].x, sum[j].y), pack_bf16x2(sum[j].z, sum[j].w));
                } else {
                  const float sv[4] = {sum[j].x, sum[j].y, sum[j].z, sum[j].w};
                  for (int e = 0; e < 4; ++e)
                    if (n + e < a.N) yrow[n + e] = f32_to_bf16(sv[e]);
                }
              }
            }
          }
          if (row == 0) a.counters[ts * 2 + static_cast<int>(rank)] = 0;  // as the next launch expects it
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");  // epi_flag[1] is rewritten by the next segment
        continue;
      }
      if constexpr (kGather) {
        // 64 columns at a time: this lane's row into the warp's staging tile (16-byte chunk j of
        // row r at position j ^ (r % 8): conflict-free), then 8 lanes per row write 128-byte
        // segments of 4 rows per instruction to every rank.
        uint4* stg = gather_stage + q * 256;
        const int m0 = m - lane;
#pragma unroll 1
        for (int cc = 0; cc < 256; cc += 64) {
#pragma unroll
          for (int h = 0; h < 4; ++h) {
            float v[16];
            tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * 256 + cc + h * 16), v);
            uint4 p0, p1;
            p0 = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]), pack_bf16x2(v[4], v[5]),
                            pack_bf16x2(v[6], v[7]));
            p1 = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]), pack_bf16x2(v[12], v[13]),
                            pack_bf16x2(v[14], v[15]));
            stg[lane * 8 + ((2 * h) ^ (lane & 7))] = p0;
            stg[lane * 8 + ((2 * h + 1) ^ (lane & 7))] = p1;
          }
          __syncwarp();
#pragma unroll
          for (int i = 0; i < 8; ++i) {
            const int r = i * 4 + (lane >> 3), c = lane & 7;
            const uint4 val = stg[r * 8 + (c ^ (r & 7))];
            const int n = n0 + cc + c * 8;
            if (m0 + r < a.M && n < a.N) gather_store8(a.g, peers, m0 + r, n, val);
          }
          __syncwarp();
        }
        tc_fence_before();
        __syncwarp();
        if (lane == 0) mbar_arrive_cluster(map_peer(smem_u32(&acc_empty[b]), 0u));
        continue;
      }
      uint16_t* yrow = a.y + static_cast<size_t>(m) * a.N;
#pragma unroll 1
      for (int c = 0; c < 256; c += 16) {
        float v[16];
        tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * 256 + c), v);
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
      if (lane == 0) mbar_arrive_cluster(map_peer(smem_u32(&acc_empty[b]), 0u));
    }
    if (!waited) pdl_wait();
  }
  pdl_launch_dependents();

  tc_fence_before();
  __syncthreads();
  if constexpr (kGather) {
    if (threadIdx.x == 0) {
      pdl_wait();
      gather_finish(a.g, gather_epoch(a.g), gridDim.x);
    }
  }
  cluster_sync();  // the pair's UMMAs and both epilogues are done before either CTA frees TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, kG2Cols);
  }
  if (tracing) a.trace[blockIdx.x] = TraceRec{t_start, t_ready, t_main, globaltimer(), smid(), blockIdx.x, 0u, 0u};
}

}  // namespace muse
