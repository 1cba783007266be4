// The per-weight rules of the 12-bit encoder, shared by the device encoder (enc12.cuh) and any
// host program that replays its grid (plain C++: no CUDA types). The format is muse_encode12's:
// per 128 x 128 tile a window base c0, the first c in 0..120 maximising the count of weights whose
// E7 (high byte without the sign) lies in [c, c + 7]; a weight inside its tile's window keeps its
// low byte and the 4-bit code s << 3 | (E7 - c0), one outside is stored as zeros and listed as an
// escape (u32 k << 16 | bits). Rows are K / 512 units of 768 bytes: 512 low bytes, then 256 code
// bytes, byte j = code[2j] | code[2j+1] << 4.
#pragma once

#include <cstdint>

#if defined(__CUDACC__)
#define MUSE_HD __host__ __device__ __forceinline__
#else
#define MUSE_HD inline
#endif

namespace muse {

constexpr int kEnc12Unit = 512, kEnc12UnitBytes = 768, kEnc12Tile = 128;
// Weights a lane takes per step: one 16-byte load of W.
constexpr int kEnc12Vec = 8;

MUSE_HD int enc12_e7(uint32_t bits) { return static_cast<int>((bits >> 8) & 0x7Fu); }

// The window base of a tile from its E7 histogram h[128]: the first c in 0..120 whose window
// [c, c + 7] holds the most weights.
MUSE_HD int enc12_pick_base(const int* h) {
  int win = 0;
  for (int i = 0; i < 8; ++i) win += h[i];
  int best = win, best_c = 0;
  for (int c = 1; c <= 120; ++c) {
    win += h[c + 7] - h[c - 1];
    if (win > best) best = win, best_c = c;
  }
  return best_c;
}

// Eight consecutive weights v[0..7] of one tile window (base c0): their low bytes (lo0 = bytes
// 0-3, lo1 = bytes 4-7, little-endian) and their four code bytes. Returns the escape mask (bit q:
// v[q] is outside the window; its low byte and code are 0).
MUSE_HD uint32_t enc12_encode8(const uint16_t* v, int c0, uint32_t* lo0, uint32_t* lo1, uint32_t* code) {
  uint32_t mask = 0, a = 0, b = 0, cw = 0;
  for (int q = 0; q < kEnc12Vec; ++q) {
    const uint32_t bits = v[q];
    const int e7 = enc12_e7(bits);
    uint32_t lo = 0, cd = 0;
    if (e7 >= c0 && e7 < c0 + 8) {
      lo = bits & 0xFFu;
      cd = ((bits >> 15) << 3) | static_cast<uint32_t>(e7 - c0);
    } else {
      mask |= 1u << q;
    }
    if (q < 4) a |= lo << (8 * q);
    else b |= lo << (8 * (q - 4));
    cw |= cd << (4 * q);  // byte q/2: code of weight 2j in its low nibble, 2j + 1 in its high one
  }
  *lo0 = a;
  *lo1 = b;
  *code = cw;
  return mask;
}

// Byte offsets in the planes of weight (r, c)'s low byte and of its code byte; c a multiple of 8,
// so the eight low bytes are 8-byte aligned and the four code bytes 4-byte aligned.
MUSE_HD void enc12_offsets(int64_t r, int64_t c, int64_t units, int64_t* lo_off, int64_t* code_off) {
  const int64_t unit = (r * units + (c >> 9)) * kEnc12UnitBytes;
  const int64_t o = c & (kEnc12Unit - 1);
  *lo_off = unit + o;
  *code_off = unit + kEnc12Unit + (o >> 1);
}

// An escape entry.
MUSE_HD uint32_t enc12_escape_entry(int64_t c, uint16_t bits) {
  return (static_cast<uint32_t>(c) << 16) | bits;
}

}  // namespace muse
