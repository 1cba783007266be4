// Medium-M tcgen05 GEMM on CTA pairs with W as the UMMA A operand and a K split that the split's
// own pairs reduce: y[m, n] = sum_k x[m, k] * W[n, k], for a few dozen to a few hundred tokens.
//
// A pair computes a 256 (W rows) x T (tokens) tile over one K range with cta_group::2 UMMAs
// (M = 256, N = T, K = 16). CTA r of the pair holds W rows r * 128 .. + 127 of the tile (one packed
// 16 KB tile a k block) and tokens r * T/2 .. + T/2 - 1 of x; its TMEM holds the FP32 accumulator of
// its 128 rows for all T tokens. So W is read once per token tile, and x crosses from L2 into shared
// memory once per 256 W rows: half the x bytes a FLOP of the 128-row tile kernel, whose x traffic
// (48 KB a k block at T = 256) is what bounds it at these shapes.
//
// K split s > 1 (s divides T). The s pairs of a tile run its s K ranges side by side, and the grid is
// one wave (the host refuses a split grid with more pairs than can be resident at once, so every pair
// of a split group is running while its peers wait for it). Each CTA drains its accumulator into shared
// memory as [T][128] FP32, writes that (but its own slice) to scratch with bulk copies, arrives on its
// half tile's counter and waits (bounded) until all s have arrived. The CTA of split p then reduces tokens
// [p T/s, (p+1) T/s) of its 128 rows: its own slice is already in place, and one bulk copy a peer brings
// the same token range of each other partial into the same position of the drained staging area; the
// slices are summed in split order 0 .. s-1 (deterministic). Each reducer reads (s-1) T/s x 512 bytes,
// less than one partial whatever s is, so the reduction does not grow with the split as a
// last-arriver sum does. A second counter lets the last CTA past the wait reset both to 0: every
// launch leaves the scratch as it found it. s = 1: no scratch, the staged accumulator is the sum.
//
// Output: BF16 rows of the slice staged in shared memory and written by one TMA tensor store (rows
// and tokens past the edges are clipped by the store), or with plain stores when N is not a multiple
// of 8.
//
// Warp roles (192 threads a CTA): warp 0 producer (lane 0), warp 1 TMEM owner + UMMA issuer (lane 0
// of the even CTA), warps 2..5 epilogue and reduction (TMEM lane quarter = warp % 4). With
// programmatic launch the producer streams its first ring of W before waiting for the previous grid;
// x, y and scratch are touched only after that wait.
#pragma once

#include "ptx.cuh"

namespace muse {

constexpr int kPkThreads = 192;
constexpr int kPkW = 16384;  // 128 W rows x 64 k of BF16 (one packed tile)
constexpr unsigned int kErrPkProducer = 0x901, kErrPkMma = 0x902, kErrPkEpilogue = 0x903, kErrPkArrive = 0x904,
                       kErrPkReduce = 0x905;

__host__ __device__ constexpr int pk_stage_bytes(int t) { return kPkW + t * 64; }  // + T/2 token rows of 128 B
__host__ __device__ constexpr int pk_tmem_cols(int t) { return t <= 32 ? 32 : (t <= 64 ? 64 : (t <= 128 ? 128 : 256)); }
// Bytes of the ring or of the epilogue's staging ([T][128] FP32, then [T/s][128] BF16 of output),
// whichever is larger (they share the space). s divides T.
__host__ __device__ constexpr int pk_body(int t, int s, int stages) {
  return stages * pk_stage_bytes(t) > t * 512 + (t / s) * 256 ? stages * pk_stage_bytes(t) : t * 512 + (t / s) * 256;
}
__host__ __device__ constexpr int pk_smem(int t, int s, int stages) { return 1024 + pk_body(t, s, stages) + (2 * stages + 2) * 8 + 16; }

struct PkArgs {
  uint16_t* y;      // [M, N]
  float* partials;  // s > 1: [tiles][2][s][T][128] FP32
  int* counters;    // s > 1: [tiles][2] x {arrive, done}, zero between launches
  int M, N, T, split, stages, nkb, rtiles, ttiles;
  int tma_y;  // 1: y written by TMA tensor stores (N % 8 == 0, y 16-byte aligned)
  TraceRec* trace;
  int trace_cap;
};

__device__ __forceinline__ int ld_acquire_gpu_s32(const int* p) {
  int v;
  asm volatile("ld.acquire.gpu.global.s32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

__device__ __forceinline__ void red_release_gpu_add(int* p, int v) {
  asm volatile("red.release.gpu.global.add.s32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

__device__ __forceinline__ void pk_bar_epi() { asm volatile("bar.sync 1, 128;" ::: "memory"); }

// Bounded wait until *p >= target. false: gave up (recorded as `where`) or another wait already had.
__device__ __noinline__ bool pk_wait_count(const int* p, int target, unsigned int where) {
  const unsigned long long t0 = globaltimer();
  unsigned long long next_poll = t0 + kErrPollNs;
  while (ld_acquire_gpu_s32(p) < target) {
    __nanosleep(64);
    const unsigned long long t = globaltimer();
    if (t >= next_poll) {
      if (error_raised()) return false;
      if (t - t0 > kWaitLimitNs) {
        report_error(where);
        return false;
      }
      next_poll = t + kErrPollNs;
    }
  }
  return true;
}

__global__ void __launch_bounds__(kPkThreads, 1)
    tc_pairk_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                    const __grid_constant__ CUtensorMap tmy, const PkArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const bool tracing = a.trace != nullptr && static_cast<int>(blockIdx.x) < a.trace_cap && threadIdx.x == 64;
  const unsigned long long t_start = tracing ? globaltimer() : 0ull;
  unsigned long long t_ready = 0ull, t_main = 0ull;
  // Traced marks (ns after the main loop): partial staged, arrival wait done, slices copied, stores done,
  // slices summed, partial written to scratch.
  unsigned int mk_written = 0u, mk_arrived = 0u, mk_copied = 0u, mk_stored = 0u, mk_summed = 0u, mk_flushed = 0u;
  uint8_t* smem = smem_align<1024>(smem_raw);
  const int stages = a.stages, T = a.T, s = a.split;
  const int stage_bytes = pk_stage_bytes(T);
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + pk_body(T, s, stages));
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;
  uint64_t* red_bar = acc_full + 1;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 1);
  int* red_flag = reinterpret_cast<int*>(tmem_slot + 1);
  float* stg = reinterpret_cast<float*>(smem);  // after the main loop: [T][128] FP32 (slice p at tokens p T/s)
  uint8_t* outs = smem + static_cast<size_t>(T) * 512;  // then [T/s][128] BF16 of output

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1;
  const int sp = pair % s, tile = pair / s;
  const int rp = tile / a.ttiles, tt = tile - rp * a.ttiles;
  const int kb0 = static_cast<int>(static_cast<long long>(sp) * a.nkb / s);
  const int kb1 = static_cast<int>(static_cast<long long>(sp + 1) * a.nkb / s);
  const int nk = kb1 - kb0;
  int rt = rp * 2 + static_cast<int>(rank);
  if (rt >= a.rtiles) rt = a.rtiles - 1;  // past N: a valid tile whose rows are never stored
  const int xrow = tt * T + static_cast<int>(rank) * (T / 2);
  const uint32_t cols = static_cast<uint32_t>(pk_tmem_cols(T));

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmx);
    prefetch_tensormap(&tmw);
    if (a.tma_y) prefetch_tensormap(&tmy);
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(acc_full, 1);
    mbar_init(red_bar, 1);
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc_pair(tmem_slot, cols);
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // both CTAs' barriers initialised and TMEM allocated before any cross-CTA use
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tracing) t_ready = globaltimer();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = a.ttiles > 1 ? policy_evict_normal() : policy_evict_first();
      const uint64_t pol_x = policy_evict_last();  // re-read by every row pair
      const uint32_t bar0 = map_peer(smem_u32(&full[0]), 0u);  // the leader's full barriers
      const int pre = min(stages, nk);
      // Weights never come from the grid this one may overlap with: the first ring of W streams
      // before the dependency wait, x after it.
      for (int i = 0; i < pre; ++i) {
        if (leader) mbar_expect_tx(&full[i], static_cast<uint32_t>(2 * stage_bytes));
        tma_load_2d_pair(smem + static_cast<size_t>(i) * stage_bytes, &tmw, bar0 + 8u * i, 0, (rt * a.nkb + kb0 + i) * 128,
                         pol_w);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i)
        tma_load_2d_pair(smem + static_cast<size_t>(i) * stage_bytes + kPkW, &tmx, bar0 + 8u * i, (kb0 + i) * 64, xrow, pol_x);
      Ring ring;
      for (int i = 0; i < pre; ++i) ring.next(stages);
      int issued = pre;
      for (int i = pre; i < nk; ++i, ring.next(stages)) {
        const int sl = ring.slot;
        if (!mbar_wait(&empty[sl], ring.phase ^ 1u, kErrPkProducer)) break;
        if (leader) mbar_expect_tx(&full[sl], static_cast<uint32_t>(2 * stage_bytes));
        uint8_t* st = smem + static_cast<size_t>(sl) * stage_bytes;
        tma_load_2d_pair(st, &tmw, bar0 + 8u * sl, 0, (rt * a.nkb + kb0 + i) * 128, pol_w);
        tma_load_2d_pair(st + kPkW, &tmx, bar0 + 8u * sl, (kb0 + i) * 64, xrow, pol_x);
        ++issued;
      }
      // Every load this CTA issued is consumed (and so has landed) once its stage is released.
      for (int i = (issued > stages ? issued - stages : 0); i < issued; ++i)
        mbar_wait(&empty[i % stages], static_cast<uint32_t>((i / stages) & 1), kErrDrain, kWaitLimitNs / 10);
    }
    pdl_launch_dependents();
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      const uint32_t idesc = umma_idesc_bf16(256, T);
      Ring ring;
      for (int i = 0; i < nk; ++i, ring.next(stages)) {
        if (!mbar_wait(&full[ring.slot], ring.phase, kErrPkMma)) break;
        tc_fence_after();
        const uint8_t* st = smem + static_cast<size_t>(ring.slot) * stage_bytes;
        const uint64_t da = umma_desc_sw128(smem_u32(st)), db = umma_desc_sw128(smem_u32(st + kPkW));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) umma_bf16_pair(tmem, da + 2 * kk, db + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
        umma_commit_pair_mc(&empty[ring.slot], 0x3);
      }
      umma_commit_pair_mc(acc_full, 0x3);  // also on the error path, so both epilogues' waits end
    }
    pdl_launch_dependents();
  } else {
    // Epilogue warps 2..5: this thread's TMEM lane = W row `row` of the CTA's 128.
    const int q = warp & 3, row = q * 32 + lane;
    const int e = static_cast<int>(threadIdx.x) - 64;  // 0..127
    const bool ok = __all_sync(0xffffffffu, mbar_wait_idle(acc_full, 0u, kErrPkEpilogue));
    tc_fence_after();
    if (tracing) t_main = globaltimer();
    pdl_launch_dependents();
    pdl_wait();  // y and the scratch may still be in use by the previous grid
    const int g = tile * 2 + static_cast<int>(rank);  // this half tile
    const int nj = T / s, j0 = sp * nj;                // the token slice this CTA reduces
    const uint32_t stg_s = smem_u32(stg);
    if (ok) {
      // Accumulator -> [T][128] FP32 in shared memory: 64 columns a TMEM load where they fit, 16 for
      // the rest (T is a multiple of 16); lanes write consecutive words.
      const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16);
      const uint32_t dst = stg_s + static_cast<uint32_t>(row * 4);
      int c = 0;
#pragma unroll 1
      for (; c + 64 <= T; c += 64) {
        float v[64];
        tmem_ld64(taddr + static_cast<uint32_t>(c), v);
#pragma unroll
        for (int j = 0; j < 64; ++j) st_shared_f32(dst + static_cast<uint32_t>((c + j) * 512), v[j]);
      }
#pragma unroll 1
      for (; c < T; c += 16) {
        float v[16];
        tmem_ld16(taddr + static_cast<uint32_t>(c), v);
#pragma unroll
        for (int j = 0; j < 16; ++j) st_shared_f32(dst + static_cast<uint32_t>((c + j) * 512), v[j]);
      }
    }
    fence_proxy_async_shared();  // the staged partial before the bulk copy reads it
    pk_bar_epi();
    if (tracing) mk_written = static_cast<unsigned int>(globaltimer() - t_main);
    bool red_ok = ok;
    if (s > 1) {
      int* arrive = a.counters + 2 * g;
      int* done = arrive + 1;
      if (e == 0) {
        int fl = ok ? 1 : 0;
        float* part0 = a.partials + static_cast<size_t>(g) * s * (static_cast<size_t>(T) * 128);
        // The partial but this CTA's own slice (only the peers read it, each its own slice).
        float* mine = part0 + static_cast<size_t>(sp) * T * 128;
        if (j0 > 0) bulk_s2g(mine, stg, static_cast<uint32_t>(j0 * 512));
        if (j0 + nj < T)
          bulk_s2g(mine + static_cast<size_t>(j0 + nj) * 128, stg + static_cast<size_t>(j0 + nj) * 128,
                   static_cast<uint32_t>((T - j0 - nj) * 512));
        bulk_commit();
        bulk_wait_all();  // the partial is written (and the staging read)
        if (tracing) mk_flushed = static_cast<unsigned int>(globaltimer() - t_main);
        fence_proxy_async_global();  // ... before the release below publishes it
        red_release_gpu_add(arrive, 1);
        if (!pk_wait_count(arrive, s, kErrPkArrive)) fl = 0;
        if (tracing) mk_arrived = static_cast<unsigned int>(globaltimer() - t_main);
        if (fl) {
          fence_proxy_async_global();  // the peers' partials, acquired above, before the bulk copies read them
          mbar_expect_tx(red_bar, static_cast<uint32_t>((s - 1) * nj * 512));
          const uint64_t pol = policy_evict_first();
          for (int p = 0; p < s; ++p)
            if (p != sp)
              bulk_g2s(stg + static_cast<size_t>(p) * nj * 128,
                       part0 + static_cast<size_t>(p) * T * 128 + static_cast<size_t>(j0) * 128,
                       static_cast<uint32_t>(nj * 512), red_bar, pol);
        }
        // Past the wait (or given up): the last CTA of the half tile leaves both counters at 0.
        if (atomicAdd(done, 1) == s - 1) {
          *reinterpret_cast<volatile int*>(arrive) = 0;
          *reinterpret_cast<volatile int*>(done) = 0;
        }
        *reinterpret_cast<volatile int*>(red_flag) = fl;
      }
      pk_bar_epi();
      red_ok = *reinterpret_cast<volatile int*>(red_flag) != 0;
      if (red_ok) red_ok = __all_sync(0xffffffffu, mbar_wait_idle(red_bar, 0u, kErrPkReduce));
      if (tracing) mk_copied = static_cast<unsigned int>(globaltimer() - t_main);
      pk_bar_epi();  // red_ok is the same in every epilogue warp
    }
    if (red_ok) {
      // Thread (token lane tq, row quad rq): rows 4 rq .. 4 rq + 3 of tokens j0 + tq, + 4, ..., four
      // tokens an iteration; the s slices summed in split order. Branch-free inner loop (indices
      // clamped into the slice, the stores guarded once a token), so the four epilogue warps, one a
      // scheduler, are not held up by branch resolution between dependent loads. 4 BF16 (8 bytes)
      // out a token, 256 contiguous bytes a warp.
      const int rq = e & 31, tq = e >> 5;
      const int n = rp * 256 + static_cast<int>(rank) * 128 + 4 * rq;
      const float4* src = reinterpret_cast<const float4*>(stg) + rq;  // + (p nj + j) * 32
      uint2* outw = reinterpret_cast<uint2*>(outs) + rq;             // + j * 32
      const int mlim = a.M - (tt * T + j0);  // tokens of the slice that exist
      const int nvalid = nj < mlim ? nj : mlim;
      const bool vec = (a.N & 3) == 0 && n + 4 <= a.N;
      const bool tma_y = a.tma_y != 0;
      uint16_t* ybase = a.y + static_cast<size_t>(tt * T + j0) * a.N + n;
      const int ldy = a.N;
#pragma unroll 1
      for (int jj = tq; jj < nvalid; jj += 16) {
        int jt[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) jt[u] = min(jj + 4 * u, nvalid - 1);
        float4 acc[4];
#pragma unroll
        for (int u = 0; u < 4; ++u) acc[u] = src[jt[u] * 32];
#pragma unroll 1
        for (int p = 1; p < s; ++p) {
          const float4* sp4 = src + p * nj * 32;
          float4 v[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) v[u] = sp4[jt[u] * 32];
#pragma unroll
          for (int u = 0; u < 4; ++u) {
            acc[u].x += v[u].x;
            acc[u].y += v[u].y;
            acc[u].z += v[u].z;
            acc[u].w += v[u].w;
          }
        }
#pragma unroll
        for (int u = 0; u < 4; ++u) {
          const int j = jj + 4 * u;
          if (j >= nvalid) break;
          const uint2 w = make_uint2(pack_bf16x2(acc[u].x, acc[u].y), pack_bf16x2(acc[u].z, acc[u].w));
          if (tma_y) {
            outw[j * 32] = w;
          } else if (vec) {
            *reinterpret_cast<uint2*>(ybase + static_cast<size_t>(j) * ldy) = w;
          } else {
            const float sv[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
#pragma unroll
            for (int i = 0; i < 4; ++i)
              if (n + i < a.N) ybase[static_cast<size_t>(j) * ldy + i] = f32_to_bf16(sv[i]);
          }
        }
      }
      if (tracing) mk_summed = static_cast<unsigned int>(globaltimer() - t_main);
      if (a.tma_y) {
        fence_proxy_async_shared();  // the staged rows before the tensor store reads them
        pk_bar_epi();
        if (e == 0) {
          tma_store_2d(&tmy, outs, rp * 256 + static_cast<int>(rank) * 128, tt * T + j0);
          bulk_commit();
          bulk_wait_all();
        }
      }
    }
  }

  if (tracing) mk_stored = static_cast<unsigned int>(globaltimer() - t_main);
  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the pair's UMMAs and both epilogues are done before either CTA frees TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, cols);
  }
  if (tracing)
    a.trace[blockIdx.x] = TraceRec{t_start, t_ready, t_main, globaltimer(), smid(), blockIdx.x, mk_written, mk_arrived,
                                   mk_copied, mk_stored, mk_summed, mk_flushed};
}

}  // namespace muse
