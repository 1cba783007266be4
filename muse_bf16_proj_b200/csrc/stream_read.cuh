// Streaming-read floor: reads a contiguous device range into shared memory with 1-D bulk copies
// through a ring of mbarrier-tracked stages and does nothing else with it. It is the fastest way
// this library's projections move weights from HBM (the same copy instruction, chunk sizes and
// grid shapes), so its time for the bytes a projection streams is the floor that projection's
// time is held against.
//
// CTA c of G takes chunks [c * C / G, (c + 1) * C / G) of the range (C = ceil(bytes / chunk)),
// one lane issuing the copies: the first `stages` at once, then one more each time a stage lands.
// Every wait is bounded (kWaitLimitNs). Each CTA adds the chunks it saw land to *count, which the
// caller checks against C.
#pragma once

#include "ptx.cuh"

namespace muse {

constexpr unsigned int kErrReadFloor = 0x601;

struct ReadArgs {
  const uint8_t* src;
  long long bytes;  // multiple of 16
  int chunk;        // bytes a copy, multiple of 16
  int stages;
  unsigned int* count;
};

__host__ __device__ constexpr int read_floor_smem(int chunk, int stages) { return 128 + stages * (chunk + 8); }

__global__ void __launch_bounds__(32, 1) stream_read_kernel(const ReadArgs a) {
  extern __shared__ uint8_t smem_raw[];
  uint8_t* ring = smem_align<128>(smem_raw);
  uint64_t* full = reinterpret_cast<uint64_t*>(ring + static_cast<size_t>(a.stages) * a.chunk);
  if (threadIdx.x != 0) return;
  const long long nch = (a.bytes + a.chunk - 1) / a.chunk;
  const long long c0 = blockIdx.x * nch / gridDim.x, c1 = (blockIdx.x + 1) * nch / gridDim.x;
  const int n = static_cast<int>(c1 - c0);
  for (int s = 0; s < a.stages; ++s) mbar_init(&full[s], 1);
  fence_mbar_init();
  const uint64_t pol = policy_evict_first();
  auto issue = [&](int i, int s) {
    const long long off = (c0 + i) * static_cast<long long>(a.chunk);
    const uint32_t len = static_cast<uint32_t>(min(static_cast<long long>(a.chunk), a.bytes - off));
    mbar_expect_tx(&full[s], len);
    bulk_g2s(ring + static_cast<size_t>(s) * a.chunk, a.src + off, len, &full[s], pol);
  };
  const int pre = min(a.stages, n);
  for (int i = 0; i < pre; ++i) issue(i, i);
  Ring ring_pos;
  unsigned int landed = 0u;
  int issued = pre;
  for (int i = 0; i < n; ++i, ring_pos.next(a.stages)) {
    if (!mbar_wait(&full[ring_pos.slot], ring_pos.phase, kErrReadFloor)) break;
    ++landed;
    if (issued < n) {
      issue(issued, ring_pos.slot);  // the stage's previous copy has landed: its slot is free
      ++issued;
    }
  }
  // After a timeout, wait (bounded, whatever the error word says) for the copies still in flight
  // before the CTA's shared memory is released.
  const unsigned long long t0 = globaltimer();
  for (int i = static_cast<int>(landed); i < issued; ++i) {
    const uint32_t bar = smem_u32(&full[i % a.stages]);
    while (!mbar_test(bar, static_cast<uint32_t>((i / a.stages) & 1)) && globaltimer() - t0 < kWaitLimitNs / 10) {
    }
  }
  atomicAdd(a.count, landed);
}

}  // namespace muse
