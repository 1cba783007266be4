// Host-side 12-bit lossless BF16 weight codec (encode + decode), multithreaded over rows.
// Format: see muse_encode12 in include/muse_proj.h.
#include <algorithm>
#include <atomic>
#include <cstdint>
#include <cstring>
#include <thread>
#include <vector>

#include "../../include/muse_proj.h"
#include "errors.h"

namespace {

constexpr int kUnit = 512;
constexpr int kUnitBytes = 768;
constexpr int kTile = 128;

inline int e7_of(uint16_t b) { return (b >> 8) & 0x7F; }

int resolve_threads(int threads) {
  if (threads > 0) return threads;
  unsigned hc = std::thread::hardware_concurrency();
  return hc ? static_cast<int>(hc) : 1;
}

// Runs fn(begin, end) over [0, count) split into contiguous blocks, one per worker.
template <class Fn>
void parallel_blocks(int64_t count, int threads, Fn fn) {
  const int workers = static_cast<int>(std::min<int64_t>(std::max(1, threads), std::max<int64_t>(1, count)));
  if (workers <= 1) {
    fn(int64_t(0), count);
    return;
  }
  std::vector<std::thread> pool;
  pool.reserve(workers);
  for (int t = 0; t < workers; ++t) {
    const int64_t b = count * t / workers, e = count * (t + 1) / workers;
    pool.emplace_back([=] { fn(b, e); });
  }
  for (auto& th : pool) th.join();
}

bool check_shape(int64_t n, int64_t k) {
  if (n < 1 || k < kUnit) return muse::fail(MUSE_ERR_INVALID, "encode12: need N >= 1 and K >= 512"), false;
  if (k % kUnit || k > 65536) return muse::fail(MUSE_ERR_SHAPE, "encode12: need K %% 512 == 0 and K <= 65536"), false;
  return true;
}

}  // namespace

extern "C" int muse_encode12_sizes(int64_t n, int64_t k, int64_t* planes_bytes, int64_t* bases_bytes) {
  muse::clear_error();
  if (!planes_bytes || !bases_bytes) return muse::fail(MUSE_ERR_INVALID, "encode12_sizes: null output");
  if (!check_shape(n, k)) return muse::last_code();
  *planes_bytes = n * k * 3 / 2;
  *bases_bytes = ((n + kTile - 1) / kTile) * (k / kTile);
  return MUSE_OK;
}

extern "C" int muse_encode12(const uint16_t* w, int64_t n, int64_t k, uint8_t* planes, uint8_t* bases,
                             int32_t* esc_ptr, uint32_t* esc_val, int64_t esc_cap, int64_t* n_esc, int threads) {
  muse::clear_error();
  if (!w || !planes || !bases || !esc_ptr || !n_esc || (esc_cap > 0 && !esc_val))
    return muse::fail(MUSE_ERR_INVALID, "encode12: null pointer");
  if (!check_shape(n, k)) return muse::last_code();
  threads = resolve_threads(threads);
  const int64_t tr = (n + kTile - 1) / kTile, tk = k / kTile, units = k / kUnit;

  // 1. Per-tile window base: the first c in 0..120 whose window [c, c + 7] of E7 holds the most.
  parallel_blocks(tr, threads, [&](int64_t b, int64_t e) {
    std::vector<int64_t> counts(static_cast<size_t>(tk) * 128);
    for (int64_t t = b; t < e; ++t) {
      std::fill(counts.begin(), counts.end(), 0);
      const int64_t r1 = std::min(n, (t + 1) * kTile);
      for (int64_t r = t * kTile; r < r1; ++r) {
        const uint16_t* row = w + r * k;
        for (int64_t c = 0; c < k; ++c) counts[(c / kTile) * 128 + e7_of(row[c])]++;
      }
      for (int64_t j = 0; j < tk; ++j) {
        const int64_t* h = &counts[j * 128];
        int64_t win = 0;
        for (int i = 0; i < 8; ++i) win += h[i];
        int64_t best = win;
        int best_c = 0;
        for (int c = 1; c <= 120; ++c) {
          win += h[c + 7] - h[c - 1];
          if (win > best) best = win, best_c = c;
        }
        bases[t * tk + j] = static_cast<uint8_t>(best_c);
      }
    }
  });

  // 2. Planes and per-row escape counts.
  std::vector<int64_t> row_esc(static_cast<size_t>(n), 0);
  parallel_blocks(n, threads, [&](int64_t b, int64_t e) {
    for (int64_t r = b; r < e; ++r) {
      const uint16_t* row = w + r * k;
      const uint8_t* brow = bases + (r / kTile) * tk;
      int64_t cnt = 0;
      for (int64_t u = 0; u < units; ++u) {
        uint8_t* unit = planes + (r * units + u) * kUnitBytes;
        for (int j = 0; j < kUnit; j += 2) {
          uint8_t code2[2];
          for (int h = 0; h < 2; ++h) {
            const int64_t c = u * kUnit + j + h;
            const uint16_t bits = row[c];
            const int c0 = brow[c / kTile];
            const int e7 = e7_of(bits);
            if (e7 >= c0 && e7 < c0 + 8) {
              unit[j + h] = static_cast<uint8_t>(bits & 0xFF);
              code2[h] = static_cast<uint8_t>(((bits >> 15) << 3) | (e7 - c0));
            } else {
              unit[j + h] = 0;
              code2[h] = 0;
              ++cnt;
            }
          }
          unit[kUnit + j / 2] = static_cast<uint8_t>(code2[0] | (code2[1] << 4));
        }
      }
      row_esc[static_cast<size_t>(r)] = cnt;
    }
  });

  int64_t total = 0;
  esc_ptr[0] = 0;
  for (int64_t r = 0; r < n; ++r) {
    total += row_esc[static_cast<size_t>(r)];
    if (total > INT32_MAX) return muse::fail(MUSE_ERR_CAPACITY, "encode12: more than 2^31 escapes");
    esc_ptr[r + 1] = static_cast<int32_t>(total);
  }
  *n_esc = total;
  if (total > esc_cap)
    return muse::fail(MUSE_ERR_CAPACITY, "encode12: %lld escapes, capacity %lld", (long long)total,
                      (long long)esc_cap);

  // 3. Escape entries, row-major, k ascending.
  parallel_blocks(n, threads, [&](int64_t b, int64_t e) {
    for (int64_t r = b; r < e; ++r) {
      if (row_esc[static_cast<size_t>(r)] == 0) continue;
      const uint16_t* row = w + r * k;
      const uint8_t* brow = bases + (r / kTile) * tk;
      int64_t o = esc_ptr[r];
      for (int64_t c = 0; c < k; ++c) {
        const int c0 = brow[c / kTile];
        const int e7 = e7_of(row[c]);
        if (!(e7 >= c0 && e7 < c0 + 8)) esc_val[o++] = (static_cast<uint32_t>(c) << 16) | row[c];
      }
    }
  });
  return MUSE_OK;
}

extern "C" int muse_decode12(const uint8_t* planes, const uint8_t* bases, const int32_t* esc_ptr,
                             const uint32_t* esc_val, int64_t n, int64_t k, uint16_t* w_out, int threads) {
  muse::clear_error();
  if (!planes || !bases || !esc_ptr || !w_out) return muse::fail(MUSE_ERR_INVALID, "decode12: null pointer");
  if (!check_shape(n, k)) return muse::last_code();
  if (esc_ptr[n] > 0 && !esc_val) return muse::fail(MUSE_ERR_INVALID, "decode12: null escapes");
  threads = resolve_threads(threads);
  const int64_t tk = k / kTile, units = k / kUnit;
  parallel_blocks(n, threads, [&](int64_t b, int64_t e) {
    for (int64_t r = b; r < e; ++r) {
      uint16_t* row = w_out + r * k;
      const uint8_t* brow = bases + (r / kTile) * tk;
      for (int64_t u = 0; u < units; ++u) {
        const uint8_t* unit = planes + (r * units + u) * kUnitBytes;
        for (int j = 0; j < kUnit; ++j) {
          const int64_t c = u * kUnit + j;
          const int code = (unit[kUnit + j / 2] >> ((j & 1) * 4)) & 0xF;
          const int hi = ((code & 8) << 4) | (brow[c / kTile] + (code & 7));
          row[c] = static_cast<uint16_t>((hi << 8) | unit[j]);
        }
      }
      for (int32_t i = esc_ptr[r]; i < esc_ptr[r + 1]; ++i) {
        const uint32_t v = esc_val[i];
        row[v >> 16] = static_cast<uint16_t>(v & 0xFFFFu);
      }
    }
  });
  return MUSE_OK;
}
