// tcgen05 tile GEMM with W as the UMMA A operand: y[m, n] = sum_k x[m, k] * W[n, k].
//
// One CTA computes a 128 (rows of W) x BNT (tokens) FP32 tile in TMEM over a K range. x arrives
// by 2-D TMA (128-byte swizzle, no multicast) and W either
//   - from "tiles": W repacked once (muse_pack_tiles) into contiguous 16 KB blocks
//     [N/128][K/64][128 rows][64 k], each already in the 128-byte-swizzled order the UMMA
//     descriptor reads, so a stage is ONE 1-D bulk copy of 16 contiguous KB (the DRAM-friendly
//     way to stream W), or
//   - from the row-major W by 2-D TMA boxes of 128 rows x 128 bytes (no repacking needed).
// One thread issues the UMMAs (M = 128, N = BNT, K = 16); four epilogue warps read the
// accumulator back with tcgen05.ld.
//
// Split-K, two ways, both deterministic (partials summed in rank order 0..split-1):
//   - cluster: the `split` CTAs of a thread-block cluster take consecutive K ranges; each parks its
//     FP32 partial in its own shared memory and CTA r sums tokens r, r + split, ... over the peers
//     through DSMEM. No global scratch; needs the whole cluster co-resident.
//   - global: each CTA writes its partial to caller scratch and bumps a per-tile counter; the CTA
//     that arrives last sums all partials and resets the counter to 0 (counters start at 0 and
//     every launch leaves them at 0). No co-scheduling constraint.
//
// Warp roles (192 threads): warp 0 = producer, warp 1 = TMEM owner + UMMA issuer,
// warps 2..5 = epilogue (warp w reads TMEM lanes 32 * (w % 4) .. + 31).
#pragma once

#include "gather.cuh"
#include "ptx.cuh"

namespace muse {

constexpr int kTcThreads = 192;
constexpr int kTcBK = 64;                   // K elements per stage (128 bytes of BF16)
constexpr int kTcABytes = 128 * kTcBK * 2;  // 16 KB: 128 W rows

constexpr int kTcModeTiles = 1;        // W given as packed tiles
constexpr int kTcModeGlobalSplit = 2;  // K-split partials reduced through global scratch

__host__ __device__ constexpr int tc_tile_bbytes(int bnt) { return bnt * kTcBK * 2; }
__host__ __device__ constexpr int tc_tile_tmem_cols(int bnt) { return bnt < 32 ? 32 : bnt; }

// Shared memory bytes the kernel needs (plus up to 1 KB of alignment slack).
__host__ __device__ constexpr int tc_tile_smem(int bnt, int stages) {
  return 1024 + stages * (kTcABytes + tc_tile_bbytes(bnt)) + (2 * stages + 1) * 8 + 16;
}

struct TcArgs {
  const uint8_t* wtiles;  // packed tiles (mode & kTcModeTiles)
  uint16_t* y;            // [M, N] BF16, or
  float* y32;             // [M, N] FP32 when not null (the router)
  int kxb;                // x's K in 64-blocks when W's K is twice x's (router hi | lo), else 0
  float* partials;        // global split: [tiles][split][BNT][128]
  int* counters;          // global split: [tiles], zero between launches
  int M, N, K, split, stages, mode;
  TraceRec* trace;  // optional per-CTA timestamps (nullptr: off)
  int trace_cap;
  GatherOut g;  // kGather: every value goes to each rank's y_full (y and y32 unused)
};

// Packed-tile layout: tile (rt, kb) = 16 KB at ((rt * nkb) + kb) * 16384; row r of the tile at
// r * 128; the 16-byte chunk holding k = kb * 64 + c * 8 .. + 7 at chunk position c ^ (r % 8).
// Rows >= N and columns >= K are zero. One thread per 16-byte output chunk.
__global__ void pack_tiles_kernel(const uint16_t* __restrict__ w, uint4* __restrict__ out, int n, int k, int nkb,
                                  long long chunks) {
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < chunks;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    const long long tile = i >> 10;
    const int within = static_cast<int>(i & 1023);
    const int r = within >> 3;
    const int c = (within & 7) ^ (r & 7);
    const int rt = static_cast<int>(tile / nkb), kb = static_cast<int>(tile % nkb);
    const int row = rt * 128 + r, col = kb * kTcBK + c * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < n && col < k) v = *reinterpret_cast<const uint4*>(w + static_cast<size_t>(row) * k + col);
    out[i] = v;
  }
}

// kGather: the all-gather epilogue of gather.cuh instead of stores into y.
template <int BNT, bool kGather = false>
__global__ void __launch_bounds__(kTcThreads, 1)
    tc_tile_kernel(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx, const TcArgs a) {
  constexpr int kBBytes = tc_tile_bbytes(BNT);
  constexpr uint32_t kCols = tc_tile_tmem_cols(BNT);
  constexpr uint32_t kIdesc = umma_idesc_bf16(128, BNT);
  extern __shared__ uint8_t smem_raw[];
  const int cta = blockIdx.y * gridDim.x + blockIdx.x;
  const bool tracing = a.trace != nullptr && cta < a.trace_cap && threadIdx.x == 64;  // first epilogue thread
  const unsigned long long t_start = tracing ? globaltimer() : 0ull;
  unsigned long long t_ready = 0ull, t_main = 0ull;
  uint8_t* smem = smem_align<1024>(smem_raw);
  const int stages = a.stages, split = a.split;
  uint8_t* sa = smem;
  uint8_t* sb = smem + static_cast<size_t>(stages) * kTcABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + static_cast<size_t>(stages) * kBBytes);
  uint64_t* empty = full + stages;
  uint64_t* accf = empty + stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* epi_abort = last_flag + 1;  // kGather: an epilogue warp's accumulator wait failed
  float* part = reinterpret_cast<float*>(smem);  // [BNT][128], reuses the ring after the main loop

  const bool tiles_mode = (a.mode & kTcModeTiles) != 0;
  bool peers = false;       // kGather: every rank arrived, so peers' buffers may be written
  unsigned int epoch = 0u;  // kGather: this call's epoch (read after the programmatic-launch wait)
  auto store = [&](int m, int n, float v) {  // y[m, n] in the output's precision
    if constexpr (kGather) gather_store(a.g, peers, m, n, f32_to_bf16(v));
    else if (a.y32 != nullptr) a.y32[static_cast<size_t>(m) * a.N + n] = v;
    else a.y[static_cast<size_t>(m) * a.N + n] = f32_to_bf16(v);
  };
  const bool global_split = (a.mode & kTcModeGlobalSplit) != 0;
  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const uint32_t rank = split == 1 ? 0u : (global_split ? blockIdx.x % split : cluster_ctarank());
  const int rt = blockIdx.x / split;
  const int tt = blockIdx.y;
  const int nkb = (a.K + kTcBK - 1) / kTcBK;
  const int kb0 = static_cast<int>(static_cast<long long>(rank) * nkb / split);
  const int kb1 = static_cast<int>(static_cast<long long>(rank + 1) * nkb / split);
  const int nk = kb1 - kb0;

  // The TMEM allocation first: a second CTA on this SM starts only once this one has allocated
  // and relinquished its permit (measured: the second CTA an SM started ~1 us after the first when
  // the allocation came after the barrier set-up).
  if (warp == 1) tmem_alloc(tmem_slot, kCols);
  const uint8_t* wsrc = a.wtiles + (static_cast<size_t>(rt) * nkb + kb0) * kTcABytes;
  auto load_w = [&](int i, int s, uint64_t pol_w) {
    if (tiles_mode)
      bulk_g2s(sa + static_cast<size_t>(s) * kTcABytes, wsrc + static_cast<size_t>(i) * kTcABytes, kTcABytes, &full[s],
               pol_w);
    else
      tma_load_2d(sa + static_cast<size_t>(s) * kTcABytes, &tmw, &full[s], (kb0 + i) * kTcBK, rt * 128, pol_w);
  };
  const int pre = min(stages, nk);
  if (threadIdx.x == 0) {
    if (!tiles_mode) prefetch_tensormap(&tmw);
    prefetch_tensormap(&tmx);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    *epi_abort = 0;
    fence_mbar_init();
    // Weights never come from the grid this one may overlap with (programmatic launch), so the
    // first ring-full of W streams at once, before the block barrier and the dependency wait; x
    // only after the wait.
    const uint64_t pol_w = policy_evict_first();
    for (int i = 0; i < pre; ++i) {
      mbar_expect_tx(&full[i], static_cast<uint32_t>(kTcABytes + kBBytes));
      load_w(i, i, pol_w);
    }
  }
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tracing) t_ready = globaltimer();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      // x's K block for W's K block kb: the same, or kb - kxb past x's end (W = [hi | lo]).
      auto xcol = [&](int kb) { return (a.kxb > 0 && kb >= a.kxb ? kb - a.kxb : kb) * kTcBK; };
      pdl_wait();
      if constexpr (kGather) gather_announce(a.g, gather_epoch(a.g));  // early, so peers rarely wait
      for (int i = 0; i < pre; ++i)
        tma_load_2d(sb + static_cast<size_t>(i) * kBBytes, &tmx, &full[i], xcol(kb0 + i), tt * BNT, pol_x);
      int issued = pre;
      Ring ring;  // position of unit pre
      for (int i = 0; i < pre; ++i) ring.next(stages);
      for (int i = pre; i < nk; ++i, ring.next(stages)) {
        const int s = ring.slot;
        if (!mbar_wait(&empty[s], ring.phase ^ 1u, kErrTcProducer)) break;
        mbar_expect_tx(&full[s], static_cast<uint32_t>(kTcABytes + kBBytes));
        load_w(i, s, pol_w);
        tma_load_2d(sb + static_cast<size_t>(s) * kBBytes, &tmx, &full[s], xcol(kb0 + i), tt * BNT, pol_x);
        ++issued;
      }
      for (int i = max(0, issued - stages); i < issued; ++i)
        mbar_wait(&full[i % stages], (i / stages) & 1, kErrDrain, kWaitLimitNs / 10);
    }
    pdl_launch_dependents();
  } else if (warp == 1) {
    if (lane == 0) {
      Ring ring;
      for (int i = 0; i < nk; ++i, ring.next(stages)) {
        const int s = ring.slot;
        if (!mbar_wait(&full[s], ring.phase, kErrTcMma)) break;
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
    pdl_launch_dependents();
  } else {
    // Epilogue warps 2..5.
    const int q = warp & 3;
    const int rl = q * 32 + lane;  // this thread's TMEM lane = W row within the tile
    const int n = rt * 128 + rl;
    const bool ok = __all_sync(0xffffffffu, mbar_wait(accf, 0, kErrTcEpilogue));  // tcgen05.ld is warp-wide
    tc_fence_after();
    if (tracing) t_main = globaltimer();
    pdl_launch_dependents();  // with warps 0 and 1 below: this CTA's loads are done, the next grid may start
    pdl_wait();               // y and the split-K counters may still be in use by the previous grid
    bool ok_all = ok;  // kGather: the same answer in all four warps, which share named barriers below
    if constexpr (kGather) {
      epoch = gather_epoch(a.g);
      peers = gather_arrived(a.g, epoch);
      if (!ok && lane == 0) *epi_abort = 1;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      ok_all = *reinterpret_cast<volatile int*>(epi_abort) == 0;
    }
    // kGather: 16 tokens of this tile's 128 W rows through a [16 tokens][128 rows] BF16 staging
    // tile in the drained ring, then written out as 256-byte token rows (16 lanes a row) to every
    // rank, instead of 2-byte stores 32 rows apart.
    auto stage16 = [&](int c, const float (&v)[16]) {
      uint16_t* stg = reinterpret_cast<uint16_t*>(smem);
#pragma unroll
      for (int j = 0; j < 16; ++j) stg[j * 128 + rl] = f32_to_bf16(v[j]);
      asm volatile("bar.sync 1, 128;" ::: "memory");
      const int e = static_cast<int>(threadIdx.x) - 64;
#pragma unroll
      for (int i = 0; i < 2; ++i) {
        const int id = e + 128 * i, j = id >> 4, ch = id & 15;
        const int m = tt * BNT + c + j, nn = rt * 128 + ch * 8;
        if (m < a.M && nn < a.N)
          gather_store8(a.g, peers, m, nn, *reinterpret_cast<const uint4*>(stg + j * 128 + ch * 8));
      }
      asm volatile("bar.sync 1, 128;" ::: "memory");
    };
    const int tile_id = rt * gridDim.y + tt;
    float* gpart = global_split ? a.partials + (static_cast<size_t>(tile_id) * split + rank) * (BNT * 128) : nullptr;
    if (kGather ? ok_all : ok) {
#pragma unroll 1
      for (int c = 0; c < BNT; c += 16) {
        float v[16];
        tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(c), v);
        if (kGather && split == 1) {
          stage16(c, v);
        } else if (split == 1) {
#pragma unroll
          for (int j = 0; j < 16; ++j) {
            const int m = tt * BNT + c + j;
            if (m < a.M && n < a.N) store(m, n, v[j]);
          }
        } else if (global_split) {
#pragma unroll
          for (int j = 0; j < 16; ++j) __stcg(gpart + (c + j) * 128 + rl, v[j]);
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j) part[(c + j) * 128 + rl] = v[j];
        }
      }
    }
    if (global_split && split > 1) {
      // Publish this partial, take a ticket; the last of the tile's `split` CTAs reduces.
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (rl == 0) *last_flag = (ticket_acq_rel(a.counters + tile_id) == split - 1) ? 1 : 0;
      asm volatile("bar.sync 1, 128;" ::: "memory");
      if (*last_flag) {
        const float* base = a.partials + static_cast<size_t>(tile_id) * split * (BNT * 128) + rl;
        // 16 tokens at a time, up to 8 peers' partials in flight together, added in rank order.
        for (int c = 0; c < BNT && tt * BNT + c < a.M; c += 16) {
          float sum[16];
          sum_partials16(base + c * 128, split, BNT * 128, sum);
          if constexpr (kGather) {
            stage16(c, sum);
          } else if (n < a.N) {
#pragma unroll
            for (int j = 0; j < 16; ++j) {
              const int m = tt * BNT + c + j;
              if (m < a.M) store(m, n, sum[j]);
            }
          }
        }
        if (rl == 0) a.counters[tile_id] = 0;  // leave the counter as the next launch expects it
      }
    }
  }

  if (split > 1 && !global_split) {
    cluster_sync();  // every peer's partial is in its shared memory
    if (warp >= 2) {
      // Tokens rank, rank + split, ... of this tile. Thread = (token lane tq, row quad rq): rows
      // 4 rq .. 4 rq + 3 as one 16-byte DSMEM load per peer; two tokens per round with every peer's
      // loads in flight together (up to 8 peers at a time), peers summed in rank order; y stored as
      // 4 consecutive BF16 (8 bytes) per token.
      const int e = static_cast<int>(threadIdx.x) - 64;
      const int tq = e >> 5, rq = e & 31;
      const uint32_t base = smem_u32(part) + static_cast<uint32_t>(rq * 16);
      const int ntok = (BNT - static_cast<int>(rank) + split - 1) / split;
      const int n = rt * 128 + 4 * rq;
      for (int u0 = 2 * tq; u0 < ntok; u0 += 8) {
        float4 acc[2] = {make_float4(0.f, 0.f, 0.f, 0.f), make_float4(0.f, 0.f, 0.f, 0.f)};
        for (int p0 = 0; p0 < split; p0 += 8) {
          float4 v[8][2];
#pragma unroll
          for (int pp = 0; pp < 8; ++pp)
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              const int p = p0 + pp, j = static_cast<int>(rank) + split * (u0 + t);
              v[pp][t] = (p < split && u0 + t < ntok)
                             ? ld_dsmem_v4(map_peer(base + static_cast<uint32_t>(j * 512), static_cast<uint32_t>(p)))
                             : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll
          for (int pp = 0; pp < 8; ++pp)
#pragma unroll
            for (int t = 0; t < 2; ++t) {
              if (p0 + pp < split) {
                acc[t].x += v[pp][t].x;
                acc[t].y += v[pp][t].y;
                acc[t].z += v[pp][t].z;
                acc[t].w += v[pp][t].w;
              }
            }
        }
#pragma unroll
        for (int t = 0; t < 2; ++t) {
          const int j = static_cast<int>(rank) + split * (u0 + t);
          const int m = tt * BNT + j;
          if (u0 + t >= ntok || m >= a.M) continue;
          const float sv[4] = {acc[t].x, acc[t].y, acc[t].z, acc[t].w};
          if (!kGather && a.y32 == nullptr && (a.N & 3) == 0 && n + 4 <= a.N) {
            *reinterpret_cast<uint2*>(a.y + static_cast<size_t>(m) * a.N + n) =
                make_uint2(pack_bf16x2(sv[0], sv[1]), pack_bf16x2(sv[2], sv[3]));
          } else {
#pragma unroll
            for (int q = 0; q < 4; ++q)
              if (n + q < a.N) store(m, n + q, sv[q]);
          }
        }
      }
    }
    cluster_sync();  // no CTA leaves while a peer may still read its partial
  }

  tc_fence_before();
  __syncthreads();
  if constexpr (kGather) {
    if (threadIdx.x == 0) {
      pdl_wait();
      gather_finish(a.g, gather_epoch(a.g), gridDim.x * gridDim.y);
    }
  }
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
  if (tracing) a.trace[cta] = TraceRec{t_start, t_ready, t_main, globaltimer(), smid(), static_cast<unsigned>(cta), 0u, 0u};
}

}  // namespace muse
