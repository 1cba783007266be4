// Stream-K schedule for the medium-M pair GEMM of tc_pairk.cuh (W as the UMMA A operand, 256 W rows x
// T tokens a pair tile, cta_group::2): y[m, n] = sum_k x[m, k] * W[n, k].
//
// The (tile, k block) units, tile-major, are cut into P equal runs, one a CTA pair, all P pairs
// resident in one wave (the host refuses more). Every pair then streams the same number of W bytes
// whatever the tile count, which the fixed K split cannot do when the row pairs do not divide the
// 74 CTA pairs (10240 W rows: 40 tiles; 6144: 24). A run is at most one tile long (the host refuses
// longer runs), so it covers the end of one tile and the start of the next at most: two segments,
// each accumulated in its own T-column TMEM accumulator, so segment 0 drains while segment 1's UMMAs
// run.
//
// Reduction, as the split kernel's but with a tile's contributors being the pairs whose runs overlap
// it (c of them, in run order): each CTA writes each segment's FP32 partial [T][128] to scratch slot
// (tile, half, contributor index) straight from TMEM (lanes write consecutive words) and arrives on
// the tile half's counter. Only after both segments have arrived does it wait for any tile (so no pair
// waits while holding back an arrival). Contributor i of c then reduces tokens [16 floor(i T/16 / c),
// 16 floor((i+1) T/16 / c)) of its 128 rows: bulk copies of that token range of all c partials into
// its drained ring (in chunks that fit), summed in contributor order (deterministic for a fixed grid),
// staged as BF16 and written by 16-row TMA tensor stores (or plain stores when N is not a multiple of
// 8). The last CTA past a tile half's wait resets its counters to 0.
//
// Warp roles as tc_pairk.cuh: warp 0 producer, warp 1 TMEM owner + UMMA issuer (even CTA), warps 2..5
// epilogue and reduction.
#pragma once

#include "tc12.cuh"  // t12_start / t12_owner: equal runs of units and their owners
#include "tc_pairk.cuh"

namespace muse {

constexpr unsigned int kErrPsProducer = 0x911, kErrPsMma = 0x912, kErrPsEpilogue = 0x913, kErrPsArrive = 0x914,
                       kErrPsReduce = 0x915;

__host__ __device__ constexpr int ps_smem(int t, int stages) { return 1024 + stages * pk_stage_bytes(t) + (2 * stages + 3) * 8 + 16; }
// TMEM columns for the two T-column accumulators (a power of two, at least 32).
__host__ __device__ constexpr int ps_tmem_cols(int t) { return 2 * t <= 32 ? 32 : (2 * t <= 64 ? 64 : (2 * t <= 128 ? 128 : (2 * t <= 256 ? 256 : 512))); }

struct PsArgs {
  uint16_t* y;      // [M, N]
  float* partials;  // [tiles][2][cmax][T][128] FP32
  int* counters;    // [tiles][2] x {arrive, done}, zero between launches
  long long units;  // tiles * nkb
  int M, N, T, stages, nkb, rtiles, ttiles, cmax;
  int tma_y;  // 1: y written by 16-row TMA tensor stores
  TraceRec* trace;
  int trace_cap;
};

struct PsSeg {
  int tile, kb0, nk;
};

// The run [u0, u1) as at most two segments (one a tile).
__device__ __forceinline__ int ps_segments(long long u0, long long u1, int nkb, PsSeg (&sg)[2]) {
  const int t0 = static_cast<int>(u0 / nkb);
  const long long end0 = u1 < static_cast<long long>(t0 + 1) * nkb ? u1 : static_cast<long long>(t0 + 1) * nkb;
  sg[0] = PsSeg{t0, static_cast<int>(u0 - static_cast<long long>(t0) * nkb), static_cast<int>(end0 - u0)};
  sg[1] = PsSeg{t0 + 1, 0, static_cast<int>(u1 - end0)};
  return end0 < u1 ? 2 : 1;
}

__global__ void __launch_bounds__(kPkThreads, 1)
    tc_pairsk_kernel(const __grid_constant__ CUtensorMap tmx, const __grid_constant__ CUtensorMap tmw,
                     const __grid_constant__ CUtensorMap tmy, const PsArgs a) {
  extern __shared__ uint8_t smem_raw[];
  const bool tracing = a.trace != nullptr && static_cast<int>(blockIdx.x) < a.trace_cap && threadIdx.x == 64;
  const unsigned long long t_start = tracing ? globaltimer() : 0ull;
  unsigned long long t_ready = 0ull, t_main = 0ull;
  unsigned int mk_arrived = 0u, mk_waited = 0u;  // traced: own arrivals done, last tile's wait done (ns after t_main)
  uint8_t* smem = smem_align<1024>(smem_raw);
  const int stages = a.stages, T = a.T;
  const int stage_bytes = pk_stage_bytes(T);
  const int ring_bytes = stages * stage_bytes;
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + ring_bytes);
  uint64_t* empty = full + stages;
  uint64_t* acc_full = empty + stages;  // [2] one a segment
  uint64_t* red_bar = acc_full + 2;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(red_bar + 1);
  int* red_flag = reinterpret_cast<int*>(tmem_slot + 1);

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const uint32_t rank = cluster_ctarank();
  const bool leader = rank == 0;
  const int pair = blockIdx.x >> 1, npairs = gridDim.x >> 1;
  PsSeg sg[2];
  const int nseg = ps_segments(t12_start(pair, a.units, npairs), t12_start(pair + 1, a.units, npairs), a.nkb, sg);
  const int nk = sg[0].nk + (nseg > 1 ? sg[1].nk : 0);
  const uint32_t cols = static_cast<uint32_t>(ps_tmem_cols(T));

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmx);
    prefetch_tensormap(&tmw);
    if (a.tma_y) prefetch_tensormap(&tmy);
    for (int i = 0; i < stages; ++i) {
      mbar_init(&full[i], 1);
      mbar_init(&empty[i], 1);
    }
    mbar_init(&acc_full[0], 1);
    mbar_init(&acc_full[1], 1);
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
      const uint64_t pol_x = policy_evict_last();
      const uint32_t bar0 = map_peer(smem_u32(&full[0]), 0u);  // the leader's full barriers
      // Load i of the run: (W row, x coordinates) of its segment's tile and k block.
      const int nkb = a.nkb, ttiles = a.ttiles, rtiles = a.rtiles;
      auto coords = [&sg, nkb, ttiles, rtiles, rank, T](int i, int& wrow, int& xk, int& xrow) {
        const PsSeg& g = i < sg[0].nk ? sg[0] : sg[1];
        const int kb = i < sg[0].nk ? g.kb0 + i : i - sg[0].nk;
        const int rp = g.tile / ttiles, tt = g.tile - rp * ttiles;
        int rt = rp * 2 + static_cast<int>(rank);
        if (rt >= rtiles) rt = rtiles - 1;  // past N: a valid tile whose rows are never stored
        wrow = (rt * nkb + kb) * 128;
        xk = kb * 64;
        xrow = tt * T + static_cast<int>(rank) * (T / 2);
      };
      const int pre = min(stages, nk);
      // Weights never come from the grid this one may overlap with: the first ring of W streams
      // before the dependency wait, x after it.
      for (int i = 0; i < pre; ++i) {
        int wrow, xk, xrow;
        coords(i, wrow, xk, xrow);
        if (leader) mbar_expect_tx(&full[i], static_cast<uint32_t>(2 * stage_bytes));
        tma_load_2d_pair(smem + static_cast<size_t>(i) * stage_bytes, &tmw, bar0 + 8u * i, 0, wrow, pol_w);
      }
      pdl_wait();
      for (int i = 0; i < pre; ++i) {
        int wrow, xk, xrow;
        coords(i, wrow, xk, xrow);
        tma_load_2d_pair(smem + static_cast<size_t>(i) * stage_bytes + kPkW, &tmx, bar0 + 8u * i, xk, xrow, pol_x);
      }
      Ring ring;
      for (int i = 0; i < pre; ++i) ring.next(stages);
      int issued = pre;
      for (int i = pre; i < nk; ++i, ring.next(stages)) {
        const int sl = ring.slot;
        if (!mbar_wait(&empty[sl], ring.phase ^ 1u, kErrPsProducer)) break;
        int wrow, xk, xrow;
        coords(i, wrow, xk, xrow);
        if (leader) mbar_expect_tx(&full[sl], static_cast<uint32_t>(2 * stage_bytes));
        uint8_t* st = smem + static_cast<size_t>(sl) * stage_bytes;
        tma_load_2d_pair(st, &tmw, bar0 + 8u * sl, 0, wrow, pol_w);
        tma_load_2d_pair(st + kPkW, &tmx, bar0 + 8u * sl, xk, xrow, pol_x);
        ++issued;
      }
      for (int i = (issued > stages ? issued - stages : 0); i < issued; ++i)
        mbar_wait(&empty[i % stages], static_cast<uint32_t>((i / stages) & 1), kErrDrain, kWaitLimitNs / 10);
    }
    pdl_launch_dependents();
  } else if (warp == 1) {
    if (lane == 0 && leader) {
      const uint32_t idesc = umma_idesc_bf16(256, T);
      Ring ring;
      bool ok = true;
      for (int g = 0; g < nseg; ++g) {
        const uint32_t acc = tmem + static_cast<uint32_t>(g * T);
        for (int i = 0; ok && i < sg[g].nk; ++i, ring.next(stages)) {
          if (!mbar_wait(&full[ring.slot], ring.phase, kErrPsMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint8_t* st = smem + static_cast<size_t>(ring.slot) * stage_bytes;
          const uint64_t da = umma_desc_sw128(smem_u32(st)), db = umma_desc_sw128(smem_u32(st + kPkW));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_bf16_pair(acc, da + 2 * kk, db + 2 * kk, idesc, (i > 0 || kk > 0) ? 1u : 0u);
          umma_commit_pair_mc(&empty[ring.slot], 0x3);
        }
        umma_commit_pair_mc(&acc_full[g], 0x3);  // also on the error path, so the epilogues' waits end
      }
    }
    pdl_launch_dependents();
  } else {
    // Epilogue warps 2..5: this thread's TMEM lane = W row `row` of the CTA's 128.
    const int q = warp & 3, row = q * 32 + lane;
    const int e = static_cast<int>(threadIdx.x) - 64;  // 0..127
    int cidx[2], cnt[2];
    for (int g = 0; g < nseg; ++g) {
      const int first = t12_owner(static_cast<long long>(sg[g].tile) * a.nkb, a.units, npairs);
      const int last = t12_owner(static_cast<long long>(sg[g].tile + 1) * a.nkb - 1, a.units, npairs);
      cidx[g] = pair - first;
      cnt[g] = last - first + 1;
    }
    bool ok_all = true;
    // 1. Each segment's partial, straight from TMEM to its scratch slot; then its arrival.
    for (int g = 0; g < nseg; ++g) {
      const bool ok = __all_sync(0xffffffffu, mbar_wait_idle(&acc_full[g], 0u, kErrPsEpilogue));
      tc_fence_after();
      if (g == 0) {
        if (tracing) t_main = globaltimer();
        pdl_wait();  // the scratch and y may still be in use by the previous grid
      }
      ok_all = ok_all && ok;
      const int hg = sg[g].tile * 2 + static_cast<int>(rank);  // this tile half
      float* slot = a.partials + (static_cast<size_t>(hg) * a.cmax + cidx[g]) * (static_cast<size_t>(T) * 128) + row;
      if (ok) {
        const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(g * T);
        int c = 0;
#pragma unroll 1
        for (; c + 64 <= T; c += 64) {
          float v[64];
          tmem_ld64(taddr + static_cast<uint32_t>(c), v);
#pragma unroll
          for (int j = 0; j < 64; ++j) __stcg(slot + (c + j) * 128, v[j]);
        }
#pragma unroll 1
        for (; c < T; c += 16) {
          float v[16];
          tmem_ld16(taddr + static_cast<uint32_t>(c), v);
#pragma unroll
          for (int j = 0; j < 16; ++j) __stcg(slot + (c + j) * 128, v[j]);
        }
      }
      pk_bar_epi();  // the four warps' stores of this partial, before one thread publishes them
      if (e == 0) red_release_gpu_add(a.counters + 2 * hg, 1);  // cumulative over the barrier
    }
    if (tracing) mk_arrived = static_cast<unsigned int>(globaltimer() - t_main);
    // 2. Each tile's slice: wait for all contributors, copy, sum in contributor order, store.
    const uint32_t ring_s = smem_u32(smem);
    uint32_t red_phase = 0u;
    const int rq = e & 31, tq = e >> 5;
    for (int g = 0; g < nseg; ++g) {
      const int tile = sg[g].tile, hg = tile * 2 + static_cast<int>(rank);
      const int rp = tile / a.ttiles, tt = tile - rp * a.ttiles;
      const int c = cnt[g], ch = T / 16;
      const int j0 = 16 * static_cast<int>(static_cast<long long>(cidx[g]) * ch / c);
      const int nj = 16 * static_cast<int>(static_cast<long long>(cidx[g] + 1) * ch / c) - j0;
      // Tokens a chunk: the most (a multiple of 16) whose c FP32 slices and BF16 output fit the ring.
      int chunk = 16 * (ring_bytes / (16 * (c * 512 + 256)));
      if (chunk > nj) chunk = nj;
      int* arrive = a.counters + 2 * hg;
      int* done = arrive + 1;
      if (e == 0) {
        int fl = ok_all ? 1 : 0;
        if (!pk_wait_count(arrive, c, kErrPsArrive)) fl = 0;
        if (atomicAdd(done, 1) == c - 1) {  // the last CTA past the wait leaves both counters at 0
          *reinterpret_cast<volatile int*>(arrive) = 0;
          *reinterpret_cast<volatile int*>(done) = 0;
        }
        if (fl) fence_proxy_async_global();  // the peers' partials, acquired above, before the bulk copies
        *reinterpret_cast<volatile int*>(red_flag) = fl && chunk > 0;
      }
      pk_bar_epi();
      const bool go = *reinterpret_cast<volatile int*>(red_flag) != 0;
      if (tracing) mk_waited = static_cast<unsigned int>(globaltimer() - t_main);
      if (!go) continue;
      const float* src0 = a.partials + static_cast<size_t>(hg) * a.cmax * (static_cast<size_t>(T) * 128);
      const int n = rp * 256 + static_cast<int>(rank) * 128 + 4 * rq;
      const bool vec = (a.N & 3) == 0 && n + 4 <= a.N;
      uint8_t* outs = smem + static_cast<size_t>(c) * chunk * 512;  // [chunk][128] BF16 after the slices
#pragma unroll 1
      for (int jc = 0; jc < nj; jc += chunk) {
        const int nt = nj - jc < chunk ? nj - jc : chunk;
        if (e == 0) {
          mbar_expect_tx(red_bar, static_cast<uint32_t>(c * nt * 512));
          for (int p = 0; p < c; ++p)
            bulk_g2s(smem + static_cast<size_t>(p) * nt * 512,
                     src0 + static_cast<size_t>(p) * T * 128 + static_cast<size_t>(j0 + jc) * 128,
                     static_cast<uint32_t>(nt * 512), red_bar, policy_evict_first());
        }
        const bool landed = __all_sync(0xffffffffu, mbar_wait_idle(red_bar, red_phase, kErrPsReduce));
        red_phase ^= 1u;
        const int mlim = a.M - (tt * T + j0 + jc);
        const int nvalid = landed ? (nt < mlim ? nt : mlim) : 0;
        const float4* src = reinterpret_cast<const float4*>(smem) + rq;
        uint2* outw = reinterpret_cast<uint2*>(outs) + rq;
        uint16_t* ybase = a.y + static_cast<size_t>(tt * T + j0 + jc) * a.N + n;
        // Four tokens an iteration, indices clamped into the chunk: no branch between the loads.
#pragma unroll 1
        for (int jj = tq; jj < nvalid; jj += 16) {
          int jt[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) jt[u] = min(jj + 4 * u, nvalid - 1);
          float4 acc[4];
#pragma unroll
          for (int u = 0; u < 4; ++u) acc[u] = src[jt[u] * 32];
#pragma unroll 1
          for (int p = 1; p < c; ++p) {
            const float4* sp4 = src + p * nt * 32;
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
            if (a.tma_y) {
              outw[j * 32] = w;
            } else if (vec) {
              *reinterpret_cast<uint2*>(ybase + static_cast<size_t>(j) * a.N) = w;
            } else {
              const float sv[4] = {acc[u].x, acc[u].y, acc[u].z, acc[u].w};
#pragma unroll
              for (int i = 0; i < 4; ++i)
                if (n + i < a.N) ybase[static_cast<size_t>(j) * a.N + i] = f32_to_bf16(sv[i]);
            }
          }
        }
        if (a.tma_y) fence_proxy_async_shared();  // the staged rows before the tensor stores read them
        pk_bar_epi();  // every thread is done with this chunk's slices and staged rows
        if (a.tma_y && e == 0 && nvalid > 0) {
          for (int r16 = 0; r16 < nt; r16 += 16)
            tma_store_2d(&tmy, outs + static_cast<size_t>(r16) * 256, rp * 256 + static_cast<int>(rank) * 128,
                         tt * T + j0 + jc + r16);
          bulk_commit();
          bulk_wait_all();  // the next chunk reuses the staging
        }
        pk_bar_epi();
      }
    }
  }

  tc_fence_before();
  __syncthreads();
  cluster_sync();  // the pair's UMMAs and both epilogues are done before either CTA frees TMEM
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc_pair(tmem, cols);
  }
  if (tracing)
    a.trace[blockIdx.x] = TraceRec{t_start, t_ready, t_main, globaltimer(), smid(), blockIdx.x, mk_arrived, mk_waited};
}

}  // namespace muse
