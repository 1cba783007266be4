// Stream-K tcgen05 GEMM for skinny projections (few tokens): y[m, n] = sum_k x[m, k] * W[n, k].
//
// The work is a list of units u = (token tile tt, row tile rt, k block kb), one 128 x 64 block of
// packed W (a contiguous 16 KB tile) times a BNT x 64 block of x. Units are ordered tt, rt, kb
// and CTA c of G takes the contiguous run [c * U / G, (c + 1) * U / G): every CTA streams the
// same number of bytes (+-16 KB), all CTAs run in one wave, and a CTA's W bytes are one
// contiguous range of the packed tiles. A run crosses row tiles; each maximal piece of it inside
// one tile is a "segment". A segment that covers its whole tile stores BF16 directly. Otherwise
// the segment's FP32 partial goes to caller scratch slot (tile, index of the CTA among the
// tile's contributors), the CTA takes a ticket on the tile's counter, and the CTA that arrives
// last sums the tile's partials in contributor order (deterministic for a fixed grid), stores
// BF16 and resets the counter to 0.
//
// Per CTA: warp 0 = producer (one lane; bulk copies of W tiles + 2-D TMA of x through a
// `stages`-deep ring), warp 1 = TMEM owner + UMMA issuer (M = 128, N = BNT, K = 16; two TMEM
// accumulators so a segment's epilogue overlaps the next segment's MMAs), warps 2..5 = epilogue.
// With programmatic launch the producer streams its first ring-full of W before waiting for the
// previous grid; x, y and scratch are touched only after that wait.
#pragma once

#include "ptx.cuh"

namespace muse {

constexpr int kSkThreads = 192;

__host__ __device__ constexpr int sk_bbytes(int bnt) { return bnt * 64 * 2; }
__host__ __device__ constexpr int sk_tmem_cols(int bnt) {
  return 2 * bnt <= 32 ? 32 : (2 * bnt <= 64 ? 64 : (2 * bnt <= 128 ? 128 : (2 * bnt <= 256 ? 256 : 512)));
}
__host__ __device__ constexpr int sk_smem(int bnt, int stages) {
  return 1024 + stages * (16384 + sk_bbytes(bnt)) + (2 * stages + 4) * 8 + 16;
}

struct SkArgs {
  const uint8_t* wtiles;  // packed tiles [ceil(N/128)][ceil(K/64)][16 KB]
  uint16_t* y;            // [M, N]
  float* partials;        // [tiles][smax][BNT][128]
  int* counters;          // [tiles], zero between launches
  int M, N, K, stages;
  int rtiles, nkb, ttiles;  // row tiles, k blocks, token tiles
  long long units;          // ttiles * rtiles * nkb
  int smax;                 // partial slots per tile
  TraceRec* trace;
  int trace_cap;
};

__host__ __device__ __forceinline__ long long sk_start(long long c, long long units, int g) { return c * units / g; }

// The CTA whose run holds unit u.
__host__ __device__ __forceinline__ int sk_owner(long long u, long long units, int g) {
  long long c = u * g / units;
  while (c + 1 < g && sk_start(c + 1, units, g) <= u) ++c;
  while (c > 0 && sk_start(c, units, g) > u) --c;
  return static_cast<int>(c);
}

// Two CTAs per SM (of this grid, or of this and the next programmatic launch) must fit: at most
// 65536 / (2 * 192) registers a thread.
template <int BNT>
__global__ void __launch_bounds__(kSkThreads, 2)
    tc_streamk_kernel(const __grid_constant__ CUtensorMap tmx, const SkArgs a) {
  constexpr int kABytes = 16384;
  constexpr int kBBytes = sk_bbytes(BNT);
  constexpr uint32_t kCols = sk_tmem_cols(BNT);
  constexpr uint32_t kIdesc = umma_idesc_bf16(128, BNT);
  extern __shared__ uint8_t smem_raw[];
  const bool tracing = a.trace != nullptr && static_cast<int>(blockIdx.x) < a.trace_cap && threadIdx.x == 64;
  const unsigned long long t_start = tracing ? globaltimer() : 0ull;
  unsigned long long t_ready = 0ull, t_main = 0ull;
  uint8_t* smem = smem_align<1024>(smem_raw);
  const int stages = a.stages;
  uint8_t* sa = smem;
  uint8_t* sb = smem + static_cast<size_t>(stages) * kABytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(sb + static_cast<size_t>(stages) * kBBytes);
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;   // [2]
  uint64_t* acc_empty = acc_full + 2;    // [2]
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = gridDim.x;
  const int c = blockIdx.x;
  const long long u0 = sk_start(c, a.units, g), u1 = sk_start(c + 1, a.units, g);
  const int nkb = a.nkb;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmx);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);  // one arrive per epilogue warp
    }
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tracing) t_ready = globaltimer();

  // Unit coordinates of u0, advanced kb, then rt, then tt (no division in the loops).
  struct Pos {
    int kb, rt, tt;
  };
  auto step = [&](Pos& p) {
    if (++p.kb == nkb) {
      p.kb = 0;
      if (++p.rt == a.rtiles) {
        p.rt = 0;
        ++p.tt;
      }
    }
  };
  Pos p0;
  p0.kb = static_cast<int>(u0 % nkb);
  p0.rt = static_cast<int>((u0 / nkb) % a.rtiles);
  p0.tt = static_cast<int>(u0 / nkb / a.rtiles);
  const int n_units = static_cast<int>(u1 - u0);

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      auto w_src = [&](const Pos& p) {
        return a.wtiles + (static_cast<size_t>(p.rt) * nkb + static_cast<size_t>(p.kb)) * kABytes;
      };
      const int pre = n_units < stages ? n_units : stages;
      Pos q = p0;
      for (int i = 0; i < pre; ++i, step(q)) {
        mbar_expect_tx(&full[i], static_cast<uint32_t>(kABytes + kBBytes));
        bulk_g2s(sa + static_cast<size_t>(i) * kABytes, w_src(q), kABytes, &full[i], pol_w);
      }
      pdl_wait();  // x may be the previous grid's output
      Ring ring;
      Pos p = p0;
      int issued = 0;
      for (int i = 0; i < n_units; ++i, ring.next(stages), step(p)) {
        const int s = ring.slot;
        if (i >= pre) {
          if (!mbar_wait(&empty[s], ring.phase ^ 1u, kErrTcProducer)) break;
          mbar_expect_tx(&full[s], static_cast<uint32_t>(kABytes + kBBytes));
          bulk_g2s(sa + static_cast<size_t>(s) * kABytes, w_src(p), kABytes, &full[s], pol_w);
        }
        tma_load_2d(sb + static_cast<size_t>(s) * kBBytes, &tmx, &full[s], p.kb * 64, p.tt * BNT, pol_x);
        ++issued;
      }
      for (int i = (issued > stages ? issued - stages : 0); i < issued; ++i)
        mbar_wait(&full[i % stages], static_cast<uint32_t>((i / stages) & 1), kErrDrain, kWaitLimitNs / 10);
    }
    pdl_launch_dependents();
  } else if (warp == 1) {
    if (lane == 0) {
      int kb = p0.kb;
      int seg = 0;
      Ring ring;
      for (int i = 0; i < n_units;) {
        const int b = seg & 1;
        // The epilogue must have drained this accumulator (its use seg / 2 - 1).
        if (!mbar_wait(&acc_empty[b], static_cast<uint32_t>((seg >> 1) & 1) ^ 1u, kErrTcMma)) {
          umma_commit(&acc_full[b]);
          break;
        }
        tc_fence_after();
        const uint32_t d = tmem + static_cast<uint32_t>(b * BNT);
        bool ok = true, first = true;
        for (; i < n_units; ++i) {  // one segment: until this output tile's k blocks end
          const int s = ring.slot;
          if (!mbar_wait(&full[s], ring.phase, kErrTcMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(smem_u32(sa + static_cast<size_t>(s) * kABytes));
          const uint64_t db = umma_desc_sw128(smem_u32(sb + static_cast<size_t>(s) * kBBytes));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_bf16(d, da + 2 * kk, db + 2 * kk, kIdesc, (first && kk == 0) ? 0u : 1u);
          first = false;
          umma_commit(&empty[s]);
          ring.next(stages);
          if (++kb == nkb) {
            kb = 0;
            ++i;
            break;
          }
        }
        umma_commit(&acc_full[b]);  // also on the error path, so the epilogue's wait ends
        ++seg;
        if (!ok) break;
      }
    }
    pdl_launch_dependents();
  } else {
    // Epilogue warps 2..5: one pass per segment, in order.
    const int q = warp & 3;
    const int rl = q * 32 + lane;
    int seg = 0;
    bool waited = false;
    for (long long u = u0; u < u1; ++seg) {
      const long long tile = u / nkb;
      const long long seg_end = min(u1, (tile + 1) * nkb);
      const bool whole = (u == tile * nkb) && (seg_end == (tile + 1) * nkb);
      const int b = seg & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&acc_full[b], static_cast<uint32_t>((seg >> 1) & 1),
                                                        kErrTcEpilogue));
      tc_fence_after();
      if (tracing) t_main = globaltimer();  // the last segment's value remains: main loop done
      if (!waited) {
        pdl_launch_dependents();
        pdl_wait();  // y and the counters may still be in use by the previous grid
        waited = true;
      }
      const int tt = static_cast<int>(tile / a.rtiles);
      const int rt = static_cast<int>(tile % a.rtiles);
      const int n = rt * 128 + rl;
      int first_c = c, nseg = 1;
      float* slot = nullptr;
      if (!whole) {
        first_c = sk_owner(tile * nkb, a.units, g);
        nseg = sk_owner((tile + 1) * nkb - 1, a.units, g) - first_c + 1;
        slot = a.partials + (static_cast<size_t>(tile) * a.smax + (c - first_c)) * (BNT * 128) + rl;
      }
      // 16 tokens at a time: TMEM -> registers -> BF16 output (whole tile) or FP32 partial slot.
      if (ok) {
#pragma unroll 1
        for (int c16 = 0; c16 < BNT; c16 += 16) {
          float v[16];
          tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * BNT + c16), v);
          if (whole) {
            if (n < a.N) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int m = tt * BNT + c16 + j;
                if (m < a.M) a.y[static_cast<size_t>(m) * a.N + n] = f32_to_bf16(v[j]);
              }
            }
          } else {
#pragma unroll
            for (int j = 0; j < 16; ++j) __stcg(slot + (c16 + j) * 128, v[j]);
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);  // accumulator b may be overwritten now
      if (!whole) {
        asm volatile("bar.sync 1, 128;" ::: "memory");  // every partial store of this CTA precedes the ticket
        if (rl == 0) *last_flag = (ticket_acq_rel(a.counters + tile) == nseg - 1) ? 1 : 0;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (*last_flag) {
          const float* base = a.partials + static_cast<size_t>(tile) * a.smax * (BNT * 128) + rl;
#pragma unroll 1
          for (int c16 = 0; c16 < BNT && tt * BNT + c16 < a.M; c16 += 16) {
            float sum[16];
            sum_partials16(base + c16 * 128, nseg, BNT * 128, sum);  // contributor order: deterministic
            if (n < a.N) {
#pragma unroll
              for (int j = 0; j < 16; ++j) {
                const int m = tt * BNT + c16 + j;
                if (m < a.M) a.y[static_cast<size_t>(m) * a.N + n] = f32_to_bf16(sum[j]);
              }
            }
          }
          if (rl == 0) a.counters[tile] = 0;
        }
        asm volatile("bar.sync 1, 128;" ::: "memory");  // last_flag is reused by the next segment
      }
      u = seg_end;
    }
    if (!waited) {
      pdl_launch_dependents();
      pdl_wait();
    }
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, kCols);
  }
  if (tracing) a.trace[blockIdx.x] = TraceRec{t_start, t_ready, t_main, globaltimer(), smid(), blockIdx.x, 0u, 0u};
}

}  // namespace muse
