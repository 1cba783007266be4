// tcgen05 projection over row windows of W, for few tokens (M <= 128): y[m, n] = sum_k x[m, k] W[n, k].
//
// Each CTA owns a window of R rows of W (R a multiple of 16, at most 512) and streams those rows
// over its whole K range, so no CTA shares an output element with another one: there is no split-K
// partial, ticket or fix-up after the main loop, only the accumulator's read-back and the stores
// of y. The N rows are spread over the grid in 16-row units as evenly as the units allow
// (windows differ by at most 16 rows), so every SM streams nearly the same share of W.
//
// The tokens are the UMMA's A operand (M = 128 rows: the first BNT of a stage are tokens, the rest
// read the stage's own W and padding, and their accumulator rows are never read)
// and the window's rows the B operand (N = R, or 256 + (R - 256) as two instructions). One
// tcgen05.mma costs about 45 cycles for N <= 48, 48 for N = 64 and 128 for N = 256, so a window of
// 48 rows already moves about 34 bytes of W a cycle through the tensor core, above an SM's share
// of HBM bandwidth (about 23 bytes a cycle).
//
// W comes either
//   - from the window-major copy (muse_pack_rows for the same number of windows): window g's rows
//     for k block kb are one contiguous R x 128-byte block at 16 u0 nkb 128 + kb R 128, in the
//     128-byte-swizzle order the UMMA reads, so a CTA streams one sequential byte range, one bulk
//     copy a k block (the pattern HBM serves at full rate), or
//   - from the packed 16 KB tiles (muse_pack_tiles: [N/128][K/64][128 rows][64 k]): a window's rows of
//     a k block are a contiguous range inside each 128-row tile it touches (one to five copies a k
//     block). Three CTAs then read slices of the same tiles at different times; measured on a
//     B200, HBM serves that at about a third of the window-major rate (2.1 vs 6+ TB/s).
// A window starts on a 16-row boundary, so the swizzle phase (row % 8) is the same in shared
// memory as in either source.
//
// Optional K split over a thread-block cluster of `split` CTAs (2 or 4): cluster rank s takes the
// s-th K range of the same window; after the main loop every CTA parks its FP32 partial
// [BNT][R] in its own shared memory and CTA s sums the partials of tokens s, s + split, ... over
// the cluster through DSMEM, ranks in order 0 .. split - 1 (deterministic).
//
// Warp roles (192 threads): warp 0 = producer (lane 0), warp 1 = TMEM owner + UMMA issuer
// (lane 0), warps 2..5 = epilogue (warp w reads TMEM lanes 32 (w % 4) .. + 31 = tokens).
#pragma once

#include "ptx.cuh"

namespace muse {

constexpr int kRwThreads = 192;
constexpr int kRwAWindow = 16384;  // the 128-row A operand an MMA reads from an x stage
constexpr int kRwMaxRows = 512;
constexpr unsigned int kErrRwProducer = 0x701, kErrRwMma = 0x702, kErrRwEpilogue = 0x703;

__host__ __device__ constexpr int rw_xbytes(int bnt) { return bnt * 128; }

// A stage is [x: BNT x 64 BF16][W: R x 64 BF16], padded to at least the 16 KB the MMA's 128-row A
// window reads from the stage's start, so that window covers only bytes the stage's own barrier
// has seen land. (A window reaching into other stages, whose copies are still in flight, made every
// MMA wait on them: about 430 ns a k block whatever the window's height.)
__host__ __device__ constexpr int rw_stage_bytes(int bnt, int rmax) {
  return rw_xbytes(bnt) + rmax * 128 > kRwAWindow ? rw_xbytes(bnt) + rmax * 128 : kRwAWindow;
}
// Layout: the ring [stages][rw_stage_bytes] | barriers.
__host__ __device__ constexpr int rw_smem(int bnt, int rmax, int stages) {
  return 1024 + stages * rw_stage_bytes(bnt, rmax) + (2 * stages + 1) * 8 + 16;
}

struct RwArgs {
  const uint8_t* wtiles;  // packed tiles [ceil(N/128)][nkb][16 KB], or
  const uint8_t* wrows;   // the window-major copy (muse_pack_rows; not null: used instead of wtiles)
  uint16_t* y;            // [M, N] BF16
  int M, N, nkb, stages, split;
  int groups;   // row windows (CTAs / split)
  int units16;  // ceil(N / 16): the 16-row units spread over the windows
  int rmax;     // rows of the largest window: the W stage stride is rmax * 128 bytes
  int y_vec;    // y rows 16-byte aligned (N % 8 == 0, y aligned): 16-byte stores
  TraceRec* trace;
  int trace_cap;
};

// Window g of `groups`: rows [16 u0, 16 (u0 + len)).
__host__ __device__ __forceinline__ void rw_window(int g, int groups, int units16, int* u0, int* len) {
  const int base = units16 / groups, extra = units16 % groups;
  *u0 = g * base + (g < extra ? g : extra);
  *len = base + (g < extra ? 1 : 0);
}

// Window-major re-layout of row-major BF16 W [N, K] for `groups` windows (muse_pack_rows): window g
// (rows 16 u0 .. 16 (u0 + len)) at byte 16 u0 nkb 128, then k block kb at + kb R 128, row r of the
// window at + r 128 with its 16-byte chunk c (k = 64 kb + 8 c .. + 7) at position c ^ (r % 8).
// Rows >= N and columns >= K are zero. One thread per 16-byte output chunk.
__global__ void pack_rows_kernel(const uint16_t* __restrict__ w, uint4* __restrict__ out, int n, int k, int nkb,
                                 int units16, int groups, long long chunks) {
  const int base = units16 / groups, extra = units16 % groups;
  const long long big = static_cast<long long>(extra) * (base + 1);  // units in the taller windows
  for (long long i = blockIdx.x * static_cast<long long>(blockDim.x) + threadIdx.x; i < chunks;
       i += static_cast<long long>(gridDim.x) * blockDim.x) {
    // i enumerates (row, kb, c) input-side: row-major over rows, then k blocks, then chunks.
    const int c = static_cast<int>(i & 7);
    const long long rk = i >> 3;
    const int kb = static_cast<int>(rk % nkb);
    const int row = static_cast<int>(rk / nkb);
    const int u = row >> 4;
    int g, u0, len;
    if (u < big) {
      g = u / (base + 1);
    } else {
      g = extra + static_cast<int>((u - big) / base);
    }
    rw_window(g, groups, units16, &u0, &len);
    const int r = row - 16 * u0;
    const long long off = (static_cast<long long>(16 * u0) * nkb * 128 + static_cast<long long>(kb) * len * 16 * 128 +
                           static_cast<long long>(r) * 128) / 16 + (c ^ (r & 7));
    const int col = kb * 64 + c * 8;
    uint4 v = make_uint4(0u, 0u, 0u, 0u);
    if (row < n && col < k) v = *reinterpret_cast<const uint4*>(w + static_cast<size_t>(row) * k + col);
    out[off] = v;
  }
}

template <int BNT>
__global__ void __launch_bounds__(kRwThreads, 1)
    tc_rows_kernel(const __grid_constant__ CUtensorMap tmx, const RwArgs a) {
  constexpr int kX = rw_xbytes(BNT);
  extern __shared__ uint8_t smem_raw[];
  const bool tracing = a.trace != nullptr && static_cast<int>(blockIdx.x) < a.trace_cap && threadIdx.x == 64;
  const unsigned long long t_start = tracing ? globaltimer() : 0ull;
  unsigned long long t_ready = 0ull, t_main = 0ull;
  uint8_t* smem = smem_align<1024>(smem_raw);
  const int stages = a.stages, split = a.split;
  const int sst = rw_stage_bytes(BNT, a.rmax);  // stage stride
  uint8_t* sx = smem;       // x of stage s at s * sst
  uint8_t* sw = smem + kX;  // W of stage s at s * sst + kX
  uint64_t* full = reinterpret_cast<uint64_t*>(smem + static_cast<size_t>(stages) * sst);
  uint64_t* empty = full + stages;
  uint64_t* accf = empty + stages;
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(accf + 1);
  float* part = reinterpret_cast<float*>(smem);  // split > 1: [BNT][R] FP32 over the drained rings

  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
  const int rank = split > 1 ? static_cast<int>(cluster_ctarank()) : 0;
  const int grp = static_cast<int>(blockIdx.x) / split;
  int u0, len;
  rw_window(grp, a.groups, a.units16, &u0, &len);
  const int r0 = 16 * u0, R = 16 * len;
  const int kb0 = static_cast<int>(static_cast<long long>(rank) * a.nkb / split);
  const int nk = static_cast<int>(static_cast<long long>(rank + 1) * a.nkb / split) - kb0;
  const uint32_t wbytes = static_cast<uint32_t>(R) * 128u;
  // Windows start their K walk at staggered k blocks (in proportion to the window index) and wrap:
  // with every CTA on the same k block, the requests in flight all sit one row tile's stride
  // (K / 64 x 16 KB) apart, and HBM serves that pattern at a third of its rate.
  const int rot = nk > 1 ? static_cast<int>(static_cast<long long>(grp) * nk / a.groups) : 0;
  auto kb_at = [&](int i) {
    const int j = i + rot;
    return kb0 + (j >= nk ? j - nk : j);
  };

  // The window's rows of k block kb into W stage `slot`: one bulk copy of the window-major block,
  // or one per 128-row tile touched.
  const uint8_t* wwin = a.wrows != nullptr ? a.wrows + static_cast<size_t>(r0) * a.nkb * 128 : nullptr;
  auto load_w = [&](int kb, int slot, uint64_t pol) {
    uint8_t* dst = sw + static_cast<size_t>(slot) * sst;
    if (wwin != nullptr) {
      bulk_g2s(dst, wwin + static_cast<size_t>(kb) * wbytes, wbytes, &full[slot], pol);
      return;
    }
    for (int r = r0; r < r0 + R;) {
      const int rt = r >> 7;
      const int hi = min(r0 + R, (rt + 1) * 128);
      const uint8_t* src = a.wtiles + (static_cast<size_t>(rt) * a.nkb + kb) * 16384 + static_cast<size_t>(r & 127) * 128;
      bulk_g2s(dst + static_cast<size_t>(r - r0) * 128, src, static_cast<uint32_t>(hi - r) * 128u, &full[slot], pol);
      r = hi;
    }
  };
  const int pre = min(stages, nk);

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
    }
    mbar_init(accf, 1);
    fence_mbar_init();
    // The weights never come from the grid this one may overlap with (programmatic launch), so the
    // first ring-full streams at once, before the TMEM allocation and the block barrier.
    const uint64_t pol_w = policy_evict_first();
    for (int i = 0; i < pre; ++i) {
      mbar_expect_tx(&full[i], wbytes + static_cast<uint32_t>(kX));
      load_w(kb_at(i), i, pol_w);
    }
  }
  const uint32_t cols = a.rmax <= 32 ? 32u : a.rmax <= 64 ? 64u : a.rmax <= 128 ? 128u : a.rmax <= 256 ? 256u : 512u;
  if (warp == 1) tmem_alloc(tmem_slot, cols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tracing) t_ready = globaltimer();

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      pdl_wait();  // x may be the previous grid's output
      for (int i = 0; i < pre; ++i)
        tma_load_2d(sx + static_cast<size_t>(i) * sst, &tmx, &full[i], kb_at(i) * 64, 0, pol_x);
      Ring ring;
      for (int i = 0; i < pre; ++i) ring.next(stages);
      int issued = pre;
      for (int i = pre; i < nk; ++i, ring.next(stages)) {
        const int s = ring.slot;
        if (!mbar_wait(&empty[s], ring.phase ^ 1u, kErrRwProducer)) break;
        mbar_expect_tx(&full[s], wbytes + static_cast<uint32_t>(kX));
        const int kb = kb_at(i);
        load_w(kb, s, pol_w);
        tma_load_2d(sx + static_cast<size_t>(s) * sst, &tmx, &full[s], kb * 64, 0, pol_x);
        ++issued;
      }
      // Every copy has landed before the CTA's shared memory can be released (bounded).
      for (int i = max(0, issued - stages); i < issued; ++i)
        mbar_wait(&full[i % stages], static_cast<uint32_t>((i / stages) & 1), kErrDrain, kWaitLimitNs / 10);
    }
    pdl_launch_dependents();
  } else if (warp == 1) {
    if (lane == 0) {
      const int n0 = R < 256 ? R : 256;
      const uint32_t idesc0 = umma_idesc_bf16(128, n0);
      const uint32_t idesc1 = R > 256 ? umma_idesc_bf16(128, R - 256) : 0u;
      Ring ring;
      for (int i = 0; i < nk; ++i, ring.next(stages)) {
        const int s = ring.slot;
        if (!mbar_wait(&full[s], ring.phase, kErrRwMma)) break;
        tc_fence_after();
        const uint64_t da = umma_desc_sw128(smem_u32(sx + static_cast<size_t>(s) * sst));
        const uint64_t db = umma_desc_sw128(smem_u32(sw + static_cast<size_t>(s) * sst));
        const uint64_t db1 = umma_desc_sw128(smem_u32(sw + static_cast<size_t>(s) * sst + 256 * 128));
#pragma unroll
        for (int kk = 0; kk < 4; ++kk) {  // 16 elements = 32 bytes = 2 descriptor units
          const uint32_t acc = (i > 0 || kk > 0) ? 1u : 0u;
          umma_bf16(tmem, da + 2 * kk, db + 2 * kk, idesc0, acc);
          if (R > 256) umma_bf16(tmem + 256u, da + 2 * kk, db1 + 2 * kk, idesc1, acc);
        }
        umma_commit(&empty[s]);  // frees the stage once these UMMAs have read it
      }
      umma_commit(accf);  // always: also fences any UMMA still in flight on the error path
    }
    pdl_launch_dependents();
  } else {
    // Epilogue warps 2..5: TMEM lane = token, column = row of the window.
    const int q = warp & 3;
    const int m = q * 32 + lane;
    const bool ok = __all_sync(0xffffffffu, mbar_wait_idle(accf, 0, kErrRwEpilogue));  // tcgen05.ld is warp-wide
    tc_fence_after();
    if (tracing) t_main = globaltimer();
    pdl_launch_dependents();
    pdl_wait();  // y may still be in use by the previous grid
    const int mrows = min(BNT, a.M);
    if (ok && q * 32 < mrows) {  // warp-uniform: the lane quarters holding tokens
      const bool mine = m < mrows;
      uint16_t* yrow = a.y + static_cast<size_t>(m) * a.N + r0;
#pragma unroll 1
      for (int c = 0; c < R; c += 16) {
        float v[16];
        tmem_ld16(tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(c), v);
        if (!mine) continue;
        if (split > 1) {
#pragma unroll
          for (int j = 0; j < 16; j += 4)
            *reinterpret_cast<float4*>(part + static_cast<size_t>(m) * R + c + j) = make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]);
        } else if (a.y_vec && r0 + c + 16 <= a.N) {
          *reinterpret_cast<uint4*>(yrow + c) = make_uint4(pack_bf16x2(v[0], v[1]), pack_bf16x2(v[2], v[3]),
                                                           pack_bf16x2(v[4], v[5]), pack_bf16x2(v[6], v[7]));
          *reinterpret_cast<uint4*>(yrow + c + 8) = make_uint4(pack_bf16x2(v[8], v[9]), pack_bf16x2(v[10], v[11]),
                                                               pack_bf16x2(v[12], v[13]), pack_bf16x2(v[14], v[15]));
        } else {
#pragma unroll
          for (int j = 0; j < 16; ++j)
            if (r0 + c + j < a.N) yrow[c + j] = f32_to_bf16(v[j]);
        }
      }
    }
  }

  if (split > 1) {
    cluster_sync();  // every CTA's partial is in its shared memory
    if (warp >= 2) {
      // Tokens rank, rank + split, ...: thread e takes float4 groups e, e + 128, ... of those tokens'
      // rows, the peers' partials summed in rank order.
      const int e = static_cast<int>(threadIdx.x) - 64;
      const int mrows = min(BNT, a.M);
      const int ntok = mrows > rank ? (mrows - rank + split - 1) / split : 0;
      const int g4 = R / 4;
      const uint32_t pbase = smem_u32(part);
      for (int idx = e; idx < ntok * g4; idx += 128) {
        const int t = rank + split * (idx / g4), c = 4 * (idx % g4);
        const uint32_t off = pbase + static_cast<uint32_t>((t * R + c) * 4);
        float4 v[4];
#pragma unroll
        for (int p = 0; p < 4; ++p)
          if (p < split) v[p] = ld_dsmem_v4(map_peer(off, static_cast<uint32_t>(p)));
        float4 acc = v[0];
#pragma unroll
        for (int p = 1; p < 4; ++p) {
          if (p < split) {
            acc.x += v[p].x;
            acc.y += v[p].y;
            acc.z += v[p].z;
            acc.w += v[p].w;
          }
        }
        uint16_t* dst = a.y + static_cast<size_t>(t) * a.N + r0 + c;
        if (a.y_vec && r0 + c + 4 <= a.N) {
          *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(acc.x, acc.y), pack_bf16x2(acc.z, acc.w));
        } else {
          const float sv[4] = {acc.x, acc.y, acc.z, acc.w};
#pragma unroll
          for (int j = 0; j < 4; ++j)
            if (r0 + c + j < a.N) dst[j] = f32_to_bf16(sv[j]);
        }
      }
    }
    cluster_sync();  // no CTA leaves while a peer may still read its partial
  }

  tc_fence_before();
  __syncthreads();
  if (warp == 1) {
    tc_fence_after();
    tmem_dealloc(tmem, cols);
  }
  if (tracing)
    a.trace[blockIdx.x] = TraceRec{t_start, t_ready, t_main, globaltimer(), smid(), blockIdx.x, 0u, 0u};
}

}  // namespace muse
