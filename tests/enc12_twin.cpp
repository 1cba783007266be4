// Host replay of the device 12-bit encoder's four kernels (muse_bf16_proj_b200/csrc/enc12.cuh):
// the same grids, the same per-lane steps and index arithmetic, and the same shared rules
// (enc12_core.h), run one CTA, warp and lane after another. Test infrastructure: the CPU suite
// builds it with g++ and compares its output bit for bit with the host encoder (muse_encode12), so
// the rules and layout the kernels apply are checked without a GPU.
#include <cstdint>
#include <cstring>

#include "../muse_bf16_proj_b200/csrc/enc12_core.h"

using namespace muse;

static int popc(uint32_t v) { return __builtin_popcount(v); }

// Returns the number of escape writes skipped (outside a row's range or esc_cap), as the device
// pass records kErrEncode for each.
extern "C" int64_t enc12_twin(const uint16_t* w, int64_t n, int64_t k, uint8_t* planes, uint8_t* bases,
                              int32_t* esc_ptr, uint32_t* esc_val, int64_t esc_cap) {
  const int64_t tk = k / kEnc12Tile, tr = (n + kEnc12Tile - 1) / kEnc12Tile, units = k / kEnc12Unit;
  const int rows_per_cta = 8, scan_threads = 1024;

  // 1. enc12_bases_kernel: CTA (j, t), 4 warps; warp w, lane l reads row rr = 2w + (l >> 4) + 8i.
  for (int64_t t = 0; t < tr; ++t) {
    for (int64_t j = 0; j < tk; ++j) {
      int hist[4][128] = {};
      int tot[128];
      for (int warp = 0; warp < 4; ++warp)
        for (int lane = 0; lane < 32; ++lane)
          for (int rr = warp * 2 + (lane >> 4); rr < kEnc12Tile; rr += 8) {
            const int64_t r = t * kEnc12Tile + rr;
            if (r >= n) break;
            const uint16_t* v = w + r * k + j * kEnc12Tile + (lane & 15) * kEnc12Vec;
            for (int q = 0; q < kEnc12Vec; ++q) hist[warp][enc12_e7(v[q])]++;
          }
      for (int i = 0; i < 128; ++i) tot[i] = hist[0][i] + hist[1][i] + hist[2][i] + hist[3][i];
      bases[t * tk + j] = static_cast<uint8_t>(enc12_pick_base(tot));
    }
  }

  // 2. enc12_planes_kernel: CTA b, warp = row b * 8 + warp, lane l takes c = 8l + 256i.
  for (int64_t b = 0; b < (n + rows_per_cta - 1) / rows_per_cta; ++b) {
    for (int warp = 0; warp < rows_per_cta; ++warp) {
      const int64_t r = b * rows_per_cta + warp;
      if (r >= n) continue;
      const uint8_t* brow = bases + (r / kEnc12Tile) * tk;
      uint32_t cnt = 0;
      for (int lane = 0; lane < 32; ++lane)
        for (int64_t c = lane * kEnc12Vec; c < k; c += 32 * kEnc12Vec) {
          uint32_t lo0, lo1, code;
          cnt += popc(enc12_encode8(w + r * k + c, brow[c / kEnc12Tile], &lo0, &lo1, &code));
          int64_t lo_off, code_off;
          enc12_offsets(r, c, units, &lo_off, &code_off);
          std::memcpy(planes + lo_off, &lo0, 4);
          std::memcpy(planes + lo_off + 4, &lo1, 4);
          std::memcpy(planes + code_off, &code, 4);
        }
      esc_ptr[r + 1] = static_cast<int32_t>(cnt);
    }
  }

  // 3. enc12_scan_kernel: 1024 runs of `per` rows, run totals scanned, runs rewritten.
  {
    const int64_t per = (n + scan_threads - 1) / scan_threads;
    static int64_t part[1024];
    for (int tid = 0; tid < scan_threads; ++tid) {
      const int64_t b = 1 + tid * per, e = b + per < n + 1 ? b + per : n + 1;
      int64_t s = 0;
      for (int64_t i = b; i < e; ++i) s += esc_ptr[i];
      part[tid] = s;
    }
    int64_t acc = 0;
    for (int i = 0; i < scan_threads; ++i) {
      const int64_t v = part[i];
      part[i] = acc;
      acc += v;
    }
    esc_ptr[0] = 0;
    for (int tid = 0; tid < scan_threads; ++tid) {
      const int64_t b = 1 + tid * per, e = b + per < n + 1 ? b + per : n + 1;
      int64_t a = part[tid];
      for (int64_t i = b; i < e; ++i) {
        a += esc_ptr[i];
        esc_ptr[i] = static_cast<int32_t>(a);
      }
    }
  }

  // 4. enc12_escapes_kernel: warp = row; per step, the lanes' counts prefix-summed in lane order.
  int64_t skipped = 0;
  for (int64_t r = 0; r < n; ++r) {
    const int64_t o0 = esc_ptr[r], o1 = esc_ptr[r + 1];
    if (o1 <= o0) continue;
    const uint8_t* brow = bases + (r / kEnc12Tile) * tk;
    const int64_t beg = o0 > 0 ? o0 : 0, end = o1 < esc_cap ? o1 : esc_cap;
    int64_t o = o0;
    for (int64_t c_base = 0; c_base < k; c_base += 32 * kEnc12Vec) {
      uint32_t masks[32];
      int incl[32], running = 0;
      for (int lane = 0; lane < 32; ++lane) {
        const int64_t c = c_base + lane * kEnc12Vec;
        uint32_t lo0, lo1, code;
        masks[lane] = enc12_encode8(w + r * k + c, brow[c / kEnc12Tile], &lo0, &lo1, &code);
        running += popc(masks[lane]);
        incl[lane] = running;
      }
      for (int lane = 0; lane < 32; ++lane) {
        const int64_t c = c_base + lane * kEnc12Vec;
        int64_t dst = o + incl[lane] - popc(masks[lane]);
        for (int q = 0; q < kEnc12Vec; ++q) {
          if (!((masks[lane] >> q) & 1u)) continue;
          if (dst >= beg && dst < end) esc_val[dst] = enc12_escape_entry(c + q, w[r * k + c + q]);
          else ++skipped;
          ++dst;
        }
      }
      o += incl[31];
    }
  }
  return skipped;
}
