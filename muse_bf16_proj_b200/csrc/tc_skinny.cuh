// Stream-K tcgen05 projection for few tokens with W as the UMMA's B operand: y[m, n] = sum_k x[m, k] W[n, k].
//
// One tcgen05.mma costs about the same issue time whatever its M (64 or 128) and N (16 .. 256), so
// the rows of W one instruction consumes set how fast a CTA can stream W through the tensor core.
// Here an instruction is M = 128 token rows (x, the A operand) x N = 256 rows of W (the B operand)
// x K = 16: 8 KB of W an instruction, twice what W as the A operand (128 rows) moves.
//
// Only the first BNT rows of the A tile are tokens; the MMA reads its other rows from whatever
// shared memory follows (in bounds: every A window ends inside this CTA's allocation), and their
// accumulator rows are never read.
//
// Work split: units u = (token tile tt, 256-row pair rp, k block kb), kb fastest; CTA c of G takes
// [c U / G, (c + 1) U / G), one wave. A segment (a run's piece inside one output tile) covering
// the whole tile stores BF16; otherwise it writes an FP32 partial of its valid token rows to
// caller scratch and the last contributor (ticket) sums them in contributor order.
//
// W sources: kTwelve = false: the packed BF16 tiles (two 16 KB tiles of 128 rows, copied to one
// 32 KB B tile); kTwelve = true: the 12-bit blocks of tc12.cuh (two 12416-byte blocks a unit),
// decoded in place by eight decoder warps (thread r = row r of the 256): every decoder reads its
// row and escapes into registers, a named barrier, then the stage is overwritten with the 32 KB
// BF16 B tile the UMMA reads. So a stage is 32 KB for both sources and no separate decoded ring
// is needed.
//
// Warps: 0 producer (lane 0), 1 TMEM owner + UMMA issuer (lane 0), 2..5 epilogue (TMEM lane
// quarter = warp % 4), 6..13 decoders (kTwelve only).
#pragma once

#include "ptx.cuh"
#include "tc12.cuh"

namespace muse {

constexpr int kSnRows = 256;     // W rows a unit (the UMMA's N)
constexpr int kSnBTile = 32768;  // 256 x 64 BF16, 128-byte swizzled
constexpr int kSnAWindow = 16384;  // the 128-row A window the MMA reads from an x stage

constexpr int kSnDecGroups = 3;  // 12-bit: decoder groups of four warps, each on every third unit
__host__ __device__ constexpr int sn_threads(bool twelve) { return twelve ? 192 + 128 * kSnDecGroups : 192; }
__host__ __device__ constexpr int sn_xbytes(int bnt) { return bnt * 128; }
// Layout: x ring | W ring (32 KB stages) | escape areas (12-bit: 2 x 128 B a stage) | barriers.
// The W ring follows the x ring and is at least 64 KB, so the last x stage's 16 KB A window stays
// inside the allocation.
__host__ __device__ constexpr int sn_smem(int bnt, int stages) {
  return 1024 + stages * (sn_xbytes(bnt) + kSnBTile + 256) + (3 * stages + 4) * 8 + 32;
}

struct SnArgs {
  const uint8_t* w;         // packed BF16 tiles [rtiles][nkb][16 KB] or 12-bit blocks [rtiles][nkb][12416]
  const int32_t* esc_ptr;   // 12-bit: per-row escape list (slow path)
  const uint32_t* esc_val;
  uint16_t* y;              // [M, N]
  float* partials;          // [tiles][smax][BNT][256]
  int* counters;            // [tiles], zero between launches
  int M, N, stages;
  int rtiles, rpairs, nkb, ttiles;
  long long units;
  int smax;
  int y_vec;                // y rows 16-byte aligned (N % 8 == 0 and y aligned): vector stores
  TraceRec* trace;
  int trace_cap;
};

template <bool kTwelve, int BNT>
__global__ void __launch_bounds__(sn_threads(kTwelve), 1)
    tc_skinny_kernel(const __grid_constant__ CUtensorMap tmx, const SnArgs a) {
  constexpr int kX = sn_xbytes(BNT);
  constexpr int kW = kSnBTile;
  constexpr int kBlk = kTwelve ? kT12Block : 16384;  // one 128-row block of a unit
  constexpr uint32_t kIdesc = umma_idesc_bf16(128, kSnRows);
  constexpr uint32_t kCols = 512;  // two 256-column accumulators
  constexpr int kDecWarps = kTwelve ? 4 * kSnDecGroups : 0;
  constexpr int kEpiCols = kTwelve ? 32 : 64;  // TMEM columns an epilogue load brings in
  extern __shared__ uint8_t smem_raw[];
  const bool tracing = a.trace != nullptr && static_cast<int>(blockIdx.x) < a.trace_cap && threadIdx.x == 64;
  const unsigned long long t_start = tracing ? globaltimer() : 0ull;
  unsigned long long t_ready = 0ull, t_main = 0ull;
  uint8_t* smem = smem_align<1024>(smem_raw);
  const int stages = a.stages;
  uint8_t* sx = smem;                                      // [stages][BNT x 64 BF16]
  uint8_t* sw = sx + static_cast<size_t>(stages) * kX;     // [stages][32 KB], 1024-aligned
  uint32_t* sesc = reinterpret_cast<uint32_t*>(sw + static_cast<size_t>(stages) * kW);  // [stages][2][32]
  uint64_t* full = reinterpret_cast<uint64_t*>(sesc + static_cast<size_t>(stages) * 64);
  uint64_t* empty = full + stages;                 // UMMA commit: the stage may be refilled
  uint64_t* decoded = empty + stages;              // 12-bit: the decoder warps have written the B tile
  uint64_t* acc_full = decoded + stages;           // [2]
  uint64_t* acc_empty = acc_full + 2;              // [2] epilogue warps
  uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(acc_empty + 2);
  int* last_flag = reinterpret_cast<int*>(tmem_slot + 1);
  int* dec_abort = last_flag + 1;  // [kSnDecGroups] 12-bit: a group's wait failed; the group stops together

  const int warp = threadIdx.x >> 5;
  const int lane = threadIdx.x & 31;
  const int g = gridDim.x;
  const int c = blockIdx.x;
  const long long u0 = t12_start(c, a.units, g), u1 = t12_start(c + 1, a.units, g);
  const int n_units = static_cast<int>(u1 - u0);
  const int nkb = a.nkb;

  if (threadIdx.x == 0) {
    prefetch_tensormap(&tmx);
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 1);
      mbar_init(&decoded[s], kTwelve ? 4 : 1);  // one decoder group (four warps) a unit
    }
    for (int b = 0; b < 2; ++b) {
      mbar_init(&acc_full[b], 1);
      mbar_init(&acc_empty[b], 4);
    }
    for (int g2 = 0; g2 < kSnDecGroups; ++g2) dec_abort[g2] = 0;
    fence_mbar_init();
  }
  if (warp == 1) tmem_alloc(tmem_slot, kCols);
  tc_fence_before();
  __syncthreads();
  tc_fence_after();
  const uint32_t tmem = *tmem_slot;
  if (tracing) t_ready = globaltimer();

  // Unit coordinates, advanced kb, then rp, then tt.
  struct Pos {
    int kb, rp, tt;
  };
  auto step = [&](Pos& p) {
    if (++p.kb == nkb) {
      p.kb = 0;
      if (++p.rp == a.rpairs) {
        p.rp = 0;
        ++p.tt;
      }
    }
  };
  Pos p0;
  p0.kb = static_cast<int>(u0 % nkb);
  p0.rp = static_cast<int>((u0 / nkb) % a.rpairs);
  p0.tt = static_cast<int>(u0 / nkb / a.rpairs);

  if (warp == 0) {
    if (lane == 0) {
      const uint64_t pol_w = policy_evict_first();
      const uint64_t pol_x = policy_evict_last();
      // The unit's W blocks: (2 rp, kb) and, when it exists, (2 rp + 1, kb).
      auto issue_w = [&](const Pos& p, int s) {
        const int rt = 2 * p.rp;
        const int nblk = rt + 1 < a.rtiles ? 2 : 1;
        mbar_expect_tx(&full[s], static_cast<uint32_t>(nblk * kBlk + kX));
        const uint8_t* src = a.w + (static_cast<size_t>(rt) * nkb + p.kb) * kBlk;
        uint8_t* dst = sw + static_cast<size_t>(s) * kW;
        bulk_g2s(dst, src, kBlk, &full[s], pol_w);
        if (nblk == 2) bulk_g2s(dst + kBlk, src + static_cast<size_t>(nkb) * kBlk, kBlk, &full[s], pol_w);
      };
      const int pre = n_units < stages ? n_units : stages;
      Pos q = p0;
      for (int i = 0; i < pre; ++i, step(q)) issue_w(q, i);  // weights first: never the previous grid's output
      pdl_wait();  // x may be the previous grid's output
      Ring ring;
      Pos p = p0;
      int issued = 0;
      for (int i = 0; i < n_units; ++i, ring.next(stages), step(p)) {
        const int s = ring.slot;
        if (i >= pre) {
          if (!mbar_wait(&empty[s], ring.phase ^ 1u, kErrTcProducer)) break;
          issue_w(p, s);
        }
        tma_load_2d(sx + static_cast<size_t>(s) * kX, &tmx, &full[s], p.kb * 64, p.tt * BNT, pol_x);
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
      Ring rs;
      for (int i = 0; i < n_units;) {
        const int b = seg & 1;
        if (!mbar_wait(&acc_empty[b], static_cast<uint32_t>((seg >> 1) & 1) ^ 1u, kErrTcMma)) {
          umma_commit(&acc_full[b]);
          break;
        }
        tc_fence_after();
        const uint32_t acc = tmem + static_cast<uint32_t>(b * kSnRows);
        bool ok = true, first = true;
        for (; i < n_units; ++i) {  // one segment: until this output tile's k blocks end
          if ((kTwelve && !mbar_wait(&decoded[rs.slot], rs.phase, kErrTcMma)) ||
              !mbar_wait(&full[rs.slot], rs.phase, kErrTcMma)) {
            ok = false;
            break;
          }
          tc_fence_after();
          const uint64_t da = umma_desc_sw128(smem_u32(sx + static_cast<size_t>(rs.slot) * kX));
          const uint64_t db = umma_desc_sw128(smem_u32(sw + static_cast<size_t>(rs.slot) * kW));
#pragma unroll
          for (int kk = 0; kk < 4; ++kk) umma_bf16(acc, da + 2 * kk, db + 2 * kk, kIdesc, (first && kk == 0) ? 0u : 1u);
          first = false;
          umma_commit(&empty[rs.slot]);
          rs.next(stages);
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
  } else if (kTwelve && warp >= 6) {
    // Decoders: kSnDecGroups groups of four warps take units in turn (group g: units i with
    // i % kSnDecGroups == g), so that many units' load / decode / store chains overlap. Thread t of
    // a group decodes row t of both blocks of its units (rows t and t + 128 of the B tile).
    const int grp = (warp - 6) >> 2;
    const int t = ((warp - 6) & 3) * 32 + lane;
    const int swz = t & 7;  // (t + 128) % 8 == t % 8
    int* abort_flag = dec_abort + grp;
    Ring rs;
    Pos p = p0;
    for (int j = 0; j < grp && j < n_units; ++j) {
      rs.next(stages);
      step(p);
    }
    // The group's named barrier (ids 2, 3, ...: 0 is __syncthreads, 1 the epilogue's).
    auto group_bar = [&]() {
      if (grp == 0) asm volatile("bar.sync 2, 128;" ::: "memory");  // warp-uniform branches
      else if (grp == 1) asm volatile("bar.sync 3, 128;" ::: "memory");
      else asm volatile("bar.sync 4, 128;" ::: "memory");
    };
    static_assert(kSnDecGroups <= 3, "group_bar names three barriers");
    for (int i = grp; i < n_units; i += kSnDecGroups) {
      const int s = rs.slot;
      // Every warp of the group passes the group's named barrier on every unit, also after a
      // failed wait: a warp whose wait failed raises the group's abort flag before the barrier
      // and the whole group leaves after it.
      const bool got = __all_sync(0xffffffffu, mbar_wait(&full[s], rs.phase, kErrTcEpilogue));
      if (!got && lane == 0) *reinterpret_cast<volatile int*>(abort_flag) = 1;
      uint8_t* stage = sw + static_cast<size_t>(s) * kW;
      uint32_t* areas = sesc + static_cast<size_t>(s) * 64;  // this stage's two escape areas
      const int rt0 = 2 * p.rp;
      const bool have1 = rt0 + 1 < a.rtiles;  // the unit's second block exists
      // 1. Read both rows' 64 weights into registers; warp 0 of the group saves the escape
      //    areas, which the decoded tile overwrites.
      uint4 w[2][6];
      uint32_t l03[2] = {0u, 0u}, l47[2] = {0u, 0u};
      if (got) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (h == 1 && !have1) break;
          const uint8_t* blk = stage + h * kT12Block;
#pragma unroll
          for (int j = 0; j < 6; ++j) w[h][j] = *reinterpret_cast<const uint4*>(blk + j * 2048 + t * 16);
          const uint32_t* area = reinterpret_cast<const uint32_t*>(blk + kT12Raw);
          const uint32_t base4 = (area[0] >> 16) * 0x01010101u;
          l03[h] = base4 + 0x03020100u;
          l47[h] = base4 + 0x07060504u;
          if (t < 32) areas[h * 32 + t] = area[t];
        }
      }
      // 2. The group has read its inputs: overwrite the stage with the BF16 B tile.
      group_bar();
      const bool abort = *reinterpret_cast<volatile int*>(abort_flag) != 0;
      if (got && !abort) {
#pragma unroll
        for (int h = 0; h < 2; ++h) {
          if (h == 1 && !have1) break;
          const int r = h * 128 + t;
          uint8_t* drow = stage + r * 128;
          const uint4 l0 = w[h][0], l1 = w[h][1], l2 = w[h][2], l3 = w[h][3], c0 = w[h][4], c1 = w[h][5];
          // Chunk j (weights 8j .. 8j + 7) goes to 16-byte position j ^ (r % 8) of the row (128-byte swizzle).
          *reinterpret_cast<uint4*>(drow + ((0 ^ swz) << 4)) = decode12_bf16x8(l0.x, l0.y, c0.x, l03[h], l47[h]);
          *reinterpret_cast<uint4*>(drow + ((1 ^ swz) << 4)) = decode12_bf16x8(l0.z, l0.w, c0.y, l03[h], l47[h]);
          *reinterpret_cast<uint4*>(drow + ((2 ^ swz) << 4)) = decode12_bf16x8(l1.x, l1.y, c0.z, l03[h], l47[h]);
          *reinterpret_cast<uint4*>(drow + ((3 ^ swz) << 4)) = decode12_bf16x8(l1.z, l1.w, c0.w, l03[h], l47[h]);
          *reinterpret_cast<uint4*>(drow + ((4 ^ swz) << 4)) = decode12_bf16x8(l2.x, l2.y, c1.x, l03[h], l47[h]);
          *reinterpret_cast<uint4*>(drow + ((5 ^ swz) << 4)) = decode12_bf16x8(l2.z, l2.w, c1.y, l03[h], l47[h]);
          *reinterpret_cast<uint4*>(drow + ((6 ^ swz) << 4)) = decode12_bf16x8(l3.x, l3.y, c1.z, l03[h], l47[h]);
          *reinterpret_cast<uint4*>(drow + ((7 ^ swz) << 4)) = decode12_bf16x8(l3.z, l3.w, c1.w, l03[h], l47[h]);
          const int n_esc = static_cast<int>(areas[h * 32] & 0xFFFFu);
          if (n_esc > kT12EscSlots) {
            const int row = (rt0 + h) * 128 + t;  // escape-dense block: each row owner walks its list
            if (row < a.N) {
              const int hi = __ldg(a.esc_ptr + row + 1);
              for (int e = t12_lower_bound(a.esc_val, __ldg(a.esc_ptr + row), hi, static_cast<uint32_t>(p.kb * 64));
                   e < hi; ++e) {
                const uint32_t v = __ldg(a.esc_val + e);
                const int kk = static_cast<int>(v >> 16) - p.kb * 64;
                if (kk >= 64) break;
                t12_patch(drow, swz, kk, v);
              }
            }
          }
        }
        // 3. Escapes listed in the areas: once every row is written (group barrier), thread j of the
        //    group writes entry j's exact bits. The escape counts are the same for the whole group.
        const int ne0 = static_cast<int>(areas[0] & 0xFFFFu);
        const int ne1 = have1 ? static_cast<int>(areas[32] & 0xFFFFu) : 0;
        const bool listed0 = ne0 > 0 && ne0 <= kT12EscSlots, listed1 = ne1 > 0 && ne1 <= kT12EscSlots;
        if (listed0 || listed1) {
          group_bar();
#pragma unroll
          for (int h = 0; h < 2; ++h) {
            const int ne = h == 0 ? (listed0 ? ne0 : 0) : (listed1 ? ne1 : 0);
            if (t < ne) {
              const uint32_t e = areas[h * 32 + 1 + t];
              const int row = h * 128 + static_cast<int>(e >> 22);
              t12_patch(stage + row * 128, row & 7, static_cast<int>((e >> 16) & 63u), e);
            }
          }
        }
        fence_proxy_async_smem();  // the tensor cores read this tile through the async proxy
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&decoded[s]);
      if (abort) break;
      for (int j = 0; j < kSnDecGroups; ++j) {
        rs.next(stages);
        step(p);
      }
    }
  } else if (warp >= 2 && warp <= 5) {
    // Epilogue: TMEM lane = token row of the tile, columns = the unit's 256 W rows.
    const int q = warp & 3;
    const int t = (warp - 2) * 32 + lane;  // 0..127: reduction / store index
    int seg = 0;
    bool waited = false;
    for (long long u = u0; u < u1; ++seg) {
      const long long tile = u / nkb;
      const long long seg_end = min(u1, (tile + 1) * nkb);
      const bool whole = (u == tile * nkb) && (seg_end == (tile + 1) * nkb);
      const int b = seg & 1;
      const bool ok = __all_sync(0xffffffffu, mbar_wait_idle(&acc_full[b], static_cast<uint32_t>((seg >> 1) & 1),
                                                             kErrTcEpilogue));
      tc_fence_after();
      if (tracing) t_main = globaltimer();  // the last segment's value remains: main loop done
      if (!waited) {
        pdl_launch_dependents();
        pdl_wait();  // y and the counters may still be in use by the previous grid
        waited = true;
      }
      const int tt = static_cast<int>(tile / a.rpairs);
      const int rp = static_cast<int>(tile % a.rpairs);
      const int n0 = rp * kSnRows;
      const int mvalid = min(BNT, a.M - tt * BNT);  // token rows of this tile
      const int ml = q * 32 + lane;                  // this thread's TMEM lane = token row
      int first_c = c, nseg = 1;
      float* slots = nullptr;
      if (!whole) {
        first_c = t12_owner(tile * nkb, a.units, g);
        nseg = t12_owner((tile + 1) * nkb - 1, a.units, g) - first_c + 1;
        slots = a.partials + static_cast<size_t>(tile) * a.smax * (BNT * kSnRows);
      }
      if (ok && q * 32 < mvalid) {  // warp-uniform: lane quarters holding token rows
        const int m = tt * BNT + ml;
        const bool mine = ml < mvalid;
        float* slot = whole ? nullptr : slots + (static_cast<size_t>(c - first_c) * BNT + ml) * kSnRows;
#pragma unroll 1
        for (int cc = 0; cc < kSnRows; cc += kEpiCols) {
          float v[kEpiCols];
          const uint32_t taddr = tmem + (static_cast<uint32_t>(q * 32) << 16) + static_cast<uint32_t>(b * kSnRows + cc);
          if constexpr (kEpiCols == 64) tmem_ld64(taddr, v);
          else tmem_ld32(taddr, v);
          if (!mine) continue;
          if (whole) {
            const int n = n0 + cc;
            uint16_t* dst = a.y + static_cast<size_t>(m) * a.N + n;
            if (a.y_vec && n + kEpiCols <= a.N) {
#pragma unroll
              for (int j = 0; j < kEpiCols; j += 8)
                *reinterpret_cast<uint4*>(dst + j) = make_uint4(pack_bf16x2(v[j], v[j + 1]), pack_bf16x2(v[j + 2], v[j + 3]),
                                                                pack_bf16x2(v[j + 4], v[j + 5]), pack_bf16x2(v[j + 6], v[j + 7]));
            } else {
#pragma unroll
              for (int j = 0; j < kEpiCols; ++j)
                if (n + j < a.N) dst[j] = f32_to_bf16(v[j]);
            }
          } else {
#pragma unroll
            for (int j = 0; j < kEpiCols; j += 4)
              __stcg(reinterpret_cast<float4*>(slot + cc + j), make_float4(v[j], v[j + 1], v[j + 2], v[j + 3]));
          }
        }
      }
      tc_fence_before();
      __syncwarp();
      if (lane == 0) mbar_arrive(&acc_empty[b]);
      if (!whole) {
        asm volatile("bar.sync 1, 128;" ::: "memory");  // every partial store of this CTA precedes the ticket
        if (t == 0) *last_flag = (ticket_acq_rel(a.counters + tile) == nseg - 1) ? 1 : 0;
        asm volatile("bar.sync 1, 128;" ::: "memory");
        if (*last_flag) {
          // Sum the contributors' partials in contributor order (deterministic). The tile's valid
          // rows are float4 groups g = row * 64 + col / 4; thread t takes groups t, t + 128, ...,
          // kB at a time with their loads issued together.
          constexpr int kB = kTwelve ? 4 : 8;  // 12-bit: fewer registers (more threads)
          const int groups = mvalid * (kSnRows / 4);
          const float4* part = reinterpret_cast<const float4*>(slots);
          const size_t cstride = static_cast<size_t>(BNT) * (kSnRows / 4);  // float4s between contributors
#pragma unroll 1
          for (int g0 = t; g0 < groups; g0 += 128 * kB) {
            float4 acc[kB];
#pragma unroll
            for (int j = 0; j < kB; ++j) {
              const int gi = g0 + j * 128;
              acc[j] = gi < groups ? __ldcg(part + gi) : make_float4(0.f, 0.f, 0.f, 0.f);
            }
#pragma unroll 1
            for (int k2 = 1; k2 < nseg; ++k2) {
              float4 v[kB];
#pragma unroll
              for (int j = 0; j < kB; ++j) {
                const int gi = g0 + j * 128;
                v[j] = gi < groups ? __ldcg(part + k2 * cstride + gi) : make_float4(0.f, 0.f, 0.f, 0.f);
              }
#pragma unroll
              for (int j = 0; j < kB; ++j) {
                acc[j].x += v[j].x;
                acc[j].y += v[j].y;
                acc[j].z += v[j].z;
                acc[j].w += v[j].w;
              }
            }
#pragma unroll
            for (int j = 0; j < kB; ++j) {
              const int gi = g0 + j * 128;
              if (gi >= groups) continue;
              const int n = n0 + (gi & 63) * 4;
              uint16_t* dst = a.y + static_cast<size_t>(tt * BNT + (gi >> 6)) * a.N + n;
              if (a.y_vec && n + 4 <= a.N) {
                *reinterpret_cast<uint2*>(dst) = make_uint2(pack_bf16x2(acc[j].x, acc[j].y), pack_bf16x2(acc[j].z, acc[j].w));
              } else {
                const float e[4] = {acc[j].x, acc[j].y, acc[j].z, acc[j].w};
                for (int i = 0; i < 4; ++i)
                  if (n + i < a.N) dst[i] = f32_to_bf16(e[i]);
              }
            }
          }
          if (t == 0) a.counters[tile] = 0;
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
