// 12-bit GEMV for few tokens (M <= 4) on the 12-bit blocks of tc12.cuh, decoded in registers.
//
// y[m, n] = sum_k x[m, k] * W[n, k], FP32 accumulation, BF16 out. HBM moves 12 bits a weight (plus
// the blocks' 128-byte escape areas): one 1-D bulk copy of 12416 bytes a (128-row tile, 64-k block)
// through a shared-memory ring, then each of 128 consumer threads takes one W row of the block:
// six conflict-free 16-byte loads (its low bytes and codes; rows are 16 bytes apart in every slab),
// eight byte-permute decodes of 8 weights (decode12_bf16x8) straight into mixed-precision FMAs
// (fma.rn.f32.bf16: BF16 weight x BF16 x into an FP32 sum, an even-k and an odd-k accumulator; no
// conversion instructions) against x, staged once per CTA as BF16 in shared memory and read by
// broadcast. Escaped weights decode to the tile's placeholder (the encoder stores them
// as code 0, low byte 0: BF16 base << 8); the thread then adds (true - placeholder) * x for each escape of its row, found with one warp ballot over the block's
// sorted escape area (the per-row list in global memory for the rare block with more than 31).
// No decoded weight is written anywhere: the decode happens where the multiply does.
//
// Stream-K: the (row tile, k block) units in [rt][kb] order are cut into G equal ranges, one per
// CTA, all resident in one wave; a CTA's range is one contiguous run of blocks in memory. A row
// tile whose k blocks span several CTAs gets FP32 partials [rt][contributor][MT][128] in scratch
// and a ticket; its last contributor adds them in CTA order (deterministic) and resets the ticket.
// Warp 0 = producer (one lane), warps 1..4 = consumers (thread 32 + r: row r of the tile).
#pragma once

#include "ptx.cuh"
#include "tc12.cuh"

namespace muse {

constexpr int kG12Threads = 160;
constexpr unsigned int kErrG12Producer = 0x501, kErrG12Consumer = 0x502;

struct G12Args {
  const uint8_t* blocks;    // [ceil(N / 128)][nkb] blocks of kT12Block bytes
  const uint16_t* x;        // [M, K] BF16
  uint16_t* y;              // [M, N] BF16
  const int32_t* esc_ptr;   // per-row escape list [N + 1] (escape-dense blocks)
  const uint32_t* esc_val;  // k << 16 | true BF16 bits
  float* partials;          // [rtiles][smax][MT][128]: segments of row tiles shared by several CTAs
  int* counters;            // [rtiles], zero between launches
  int M, N, K, nkb, rtiles, smax, ucap, stages;  // ucap: most units a CTA takes
  TraceRec* trace;
  int trace_cap;
};

// Shared memory: ring [stages][kT12Block] | x [MT][ucap * 64] BF16 | full[stages] | empty[stages].
__host__ __device__ constexpr int g12_smem(int stages, int ucap, int mt) {
  return 128 + stages * kT12Block + mt * ucap * 64 * 2 + 2 * stages * 8 + 16;
}

// One block: this thread's row r, 64 weights, against x[m * xstride + xk ..  + 63] (BF16, shared).
template <int MT>
__device__ __forceinline__ void g12_block(const uint8_t* blk, const uint16_t* xs, int xstride, int xk, int r, int M,
                                          float (&acc)[MT][2]) {
  const uint32_t w0 = *reinterpret_cast<const uint32_t*>(blk + kT12Raw);
  const uint32_t base4 = ((w0 >> 16) & 0xFFu) * 0x01010101u;
  const uint32_t l03 = base4 + 0x03020100u, l47 = base4 + 0x07060504u;
  uint4 lo[4], cd[2];
#pragma unroll
  for (int j = 0; j < 4; ++j) lo[j] = *reinterpret_cast<const uint4*>(blk + j * 2048 + r * 16);
#pragma unroll
  for (int j = 0; j < 2; ++j) cd[j] = *reinterpret_cast<const uint4*>(blk + (4 + j) * 2048 + r * 16);
#pragma unroll
  for (int g = 0; g < 8; ++g) {
    const uint4 l = lo[g >> 1];
    const uint32_t la = (g & 1) ? l.z : l.x, lb = (g & 1) ? l.w : l.y;
    const uint4 c = cd[g >> 2];
    const uint32_t cw = (g & 3) == 0 ? c.x : (g & 3) == 1 ? c.y : (g & 3) == 2 ? c.z : c.w;
    const uint4 p = decode12_bf16x8(la, lb, cw, l03, l47);
#pragma unroll
    for (int m = 0; m < MT; ++m) {
      if (m < M) {
        const uint4 xv = *reinterpret_cast<const uint4*>(xs + m * xstride + xk + g * 8);
        fma_bf16x2(p.x, xv.x, acc[m][0], acc[m][1]);
        fma_bf16x2(p.y, xv.y, acc[m][0], acc[m][1]);
        fma_bf16x2(p.z, xv.z, acc[m][0], acc[m][1]);
        fma_bf16x2(p.w, xv.w, acc[m][0], acc[m][1]);
      }
    }
  }
}

// corr += (true - placeholder) * x[kk] for one escape.
template <int MT>
__device__ __forceinline__ void g12_fix(float (&corr)[MT], const uint16_t* xs, int xstride, int xk, int kk, uint32_t bits,
                                        float d_ph, int M) {
  const float d_true = __uint_as_float(bits << 16);
#pragma unroll
  for (int m = 0; m < MT; ++m) {
    if (m < M) {
      const float xv = bf16f(xs[m * xstride + xk + kk]);
      corr[m] = fmaf(d_true, xv, corr[m]);
      corr[m] = fmaf(-d_ph, xv, corr[m]);
    }
  }
}

// Escape corrections in this block for the warp's 32 rows: (true - stored) * x for each escape.
// Lane e reads entry e of the area (at most 31, sorted by row); a ballot finds those in this
// warp's rows, and each is broadcast in entry order to the lane owning its row (deterministic).
// A block with more escapes than its area holds sends every lane to its row's list instead.
template <int MT>
__device__ __forceinline__ void g12_escapes(const uint8_t* blk, const G12Args& a, const uint16_t* xs, int xstride, int xk,
                                            int r, int row, int kb, int lane, float (&corr)[MT]) {
  const uint32_t* area = reinterpret_cast<const uint32_t*>(blk + kT12Raw);
  const uint32_t w0 = area[0];
  const int count = static_cast<int>(w0 & 0xFFFFu);
  if (count == 0) return;
  // The encoder stores an escape as code 0 and low byte 0, so it decoded to the tile's placeholder
  // BF16 base << 8 (high byte = base + 0, positive).
  const float d_ph = __uint_as_float(((w0 >> 16) & 0xFFu) << 24);
  if (count <= kT12EscSlots) {
    const uint32_t v = lane < count ? area[1 + lane] : 0xFFFFFFFFu;
    const uint32_t warp_rows = static_cast<uint32_t>(r - lane) >> 5;  // this warp's 32-row group
    unsigned mask = __ballot_sync(0xffffffffu, lane < count && (v >> 27) == warp_rows);
    while (mask) {
      const int e = __ffs(mask) - 1;
      mask &= mask - 1;
      const uint32_t ve = __shfl_sync(0xffffffffu, v, e);
      if (static_cast<int>((ve >> 22) & 31u) == lane)
        g12_fix<MT>(corr, xs, xstride, xk, static_cast<int>((ve >> 16) & 63u), ve & 0xFFFFu, d_ph, a.M);
    }
  } else if (row < a.N) {
    const uint32_t k0 = static_cast<uint32_t>(kb) * 64u;
    const int end = a.esc_ptr[row + 1];
    for (int e = t12_lower_bound(a.esc_val, a.esc_ptr[row], end, k0); e < end; ++e) {
      const uint32_t v = __ldg(a.esc_val + e);
      if ((v >> 16) >= k0 + 64u) break;
      g12_fix<MT>(corr, xs, xstride, xk, static_cast<int>((v >> 16) - k0), v & 0xFFFFu, d_ph, a.M);
    }
  }
}

template <int MT>
__global__ void __launch_bounds__(kG12Threads, 1) gemv12t_kernel(const G12Args a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* smem = smem_align<128>(smem_raw);
  const bool tracing = a.trace != nullptr && static_cast<int>(blockIdx.x) < a.trace_cap && threadIdx.x == 32;
  const unsigned long long t_start = tracing ? globaltimer() : 0ull;
  unsigned long long t_ready = 0ull, t_main = 0ull;
  const int stages = a.stages, G = static_cast<int>(gridDim.x);
  const long long units = static_cast<long long>(a.rtiles) * a.nkb;
  const long long u0 = t12_start(blockIdx.x, units, G), u1 = t12_start(blockIdx.x + 1, units, G);
  const int nu = static_cast<int>(u1 - u0);
  uint8_t* ring = smem;
  uint16_t* xs = reinterpret_cast<uint16_t*>(smem + static_cast<size_t>(stages) * kT12Block);  // [MT][ucap * 64]
  const int xstride = a.ucap * 64;
  uint64_t* full = reinterpret_cast<uint64_t*>(xs + MT * xstride);
  uint64_t* empty = full + stages;
  int* last_flag = reinterpret_cast<int*>(empty + stages);
  const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

  if (threadIdx.x == 0) {
    for (int s = 0; s < stages; ++s) {
      mbar_init(&full[s], 1);
      mbar_init(&empty[s], 4);
    }
    fence_mbar_init();
  }
  __syncthreads();
  if (tracing) t_ready = globaltimer();

  if (warp == 0) {
    if (lane == 0) {
      // This CTA's units are consecutive blocks of the [rt][kb] array: one contiguous stream.
      const uint64_t pol = policy_evict_first();
      const uint8_t* src = a.blocks + static_cast<size_t>(u0) * kT12Block;
      Ring ring_pos;
      int issued = 0;
      for (int i = 0; i < nu; ++i, ring_pos.next(stages)) {
        const int s = ring_pos.slot;
        // The first ring-full streams at once (weights are never the previous grid's output).
        if (i >= stages && !mbar_wait(&empty[s], ring_pos.phase ^ 1u, kErrG12Producer)) break;
        mbar_expect_tx(&full[s], static_cast<uint32_t>(kT12Block));
        bulk_g2s(ring + static_cast<size_t>(s) * kT12Block, src + static_cast<size_t>(i) * kT12Block, kT12Block,
                 &full[s], pol);
        ++issued;
      }
      for (int i = max(0, issued - stages); i < issued; ++i)
        mbar_wait(&full[i % stages], (i / stages) & 1, kErrDrain, kWaitLimitNs / 10);
    }
  } else {
    const int r = threadIdx.x - 32;
    pdl_wait();  // x and y (and the scratch) may belong to the previous grid
    // x columns of each of this CTA's units, in unit order (slot i = unit u0 + i's k block).
    for (int c = r; c < MT * nu * 8; c += 128) {  // 16-byte chunks
      const int m = c / (nu * 8), rest = c - m * nu * 8, i = rest >> 3, part = rest & 7;
      const int kb = static_cast<int>((u0 + i) % a.nkb);
      reinterpret_cast<uint4*>(xs + m * xstride + i * 64)[part] =
          m < a.M ? ldg_nc_v4(a.x + static_cast<size_t>(m) * a.K + kb * 64 + part * 8) : make_uint4(0u, 0u, 0u, 0u);
    }
    asm volatile("bar.sync 1, 128;" ::: "memory");
    float acc[MT][2], corr[MT];  // even-k and odd-k sums, escape corrections
    auto clear = [&]() {
#pragma unroll
      for (int m = 0; m < MT; ++m) {
        acc[m][0] = acc[m][1] = 0.f;
        corr[m] = 0.f;
      }
    };
    clear();
    int rt = static_cast<int>(u0 / a.nkb), kb = static_cast<int>(u0 % a.nkb);
    int seg_first = kb;  // first k block of the current row tile's segment
    Ring ring_pos;
    for (int i = 0; i < nu; ++i, ring_pos.next(stages)) {
      const int s = ring_pos.slot;
      // On a failed wait (recorded in the error word) the warp skips the math but keeps taking the
      // same named barriers as the other warps below, so none of them can be left waiting.
      const bool ok = __all_sync(0xffffffffu, mbar_wait(&full[s], ring_pos.phase, kErrG12Consumer));
      const uint8_t* blk = ring + static_cast<size_t>(s) * kT12Block;
      const int row = rt * 128 + r;
      if (ok) {
        g12_block<MT>(blk, xs, xstride, i * 64, r, a.M, acc);
        g12_escapes<MT>(blk, a, xs, xstride, i * 64, r, row, kb, lane, corr);
      }
      __syncwarp();
      if (lane == 0) mbar_arrive(&empty[s]);
      if (++kb == a.nkb || i == nu - 1) {
        // End of this CTA's segment of row tile rt: y directly when the segment is the whole
        // tile, else a partial for the tile's last contributor to add in CTA order.
        float tot[MT];
#pragma unroll
        for (int m = 0; m < MT; ++m) tot[m] = (acc[m][0] + acc[m][1]) + corr[m];
        if (seg_first == 0 && kb == a.nkb) {
#pragma unroll
          for (int m = 0; m < MT; ++m)
            if (m < a.M && row < a.N) a.y[static_cast<size_t>(m) * a.N + row] = f32_to_bf16(tot[m]);
        } else {
          const int first_c = t12_owner(static_cast<long long>(rt) * a.nkb, units, G);
          const int nseg = t12_owner(static_cast<long long>(rt + 1) * a.nkb - 1, units, G) - first_c + 1;
          float* mine = a.partials + (static_cast<size_t>(rt) * a.smax + (blockIdx.x - first_c)) * MT * 128;
#pragma unroll
          for (int m = 0; m < MT; ++m) __stcg(mine + m * 128 + r, tot[m]);
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (r == 0) *last_flag = (ticket_acq_rel(a.counters + rt) == nseg - 1) ? 1 : 0;
          asm volatile("bar.sync 1, 128;" ::: "memory");
          if (*last_flag) {
            const float* base = a.partials + static_cast<size_t>(rt) * a.smax * MT * 128 + r;
#pragma unroll
            for (int m = 0; m < MT; ++m) {
              if (m >= a.M) continue;
              float sum = 0.f;
              for (int p = 0; p < nseg; ++p) sum += __ldcg(base + (static_cast<size_t>(p) * MT + m) * 128);
              if (row < a.N) a.y[static_cast<size_t>(m) * a.N + row] = f32_to_bf16(sum);
            }
            if (r == 0) a.counters[rt] = 0;  // leave the ticket as the next launch expects it
          }
          asm volatile("bar.sync 1, 128;" ::: "memory");  // last_flag is reused by the next segment
        }
        clear();
        if (kb == a.nkb) {
          kb = 0;
          ++rt;
        }
        seg_first = kb;
      }
    }
    if (tracing) t_main = globaltimer();
    pdl_launch_dependents();
  }
  if (warp == 0) pdl_launch_dependents();
  if (tracing) a.trace[blockIdx.x] = TraceRec{t_start, t_ready, t_main, globaltimer(), smid(), blockIdx.x, 0u, 0u};
}

}  // namespace muse
