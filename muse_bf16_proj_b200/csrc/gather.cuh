// All-gather fused into a projection's epilogue: rank r of P computes the column slice
// y[:, col0 .. col0 + N) of the full output and stores every finished value straight into each
// rank's copy of y_full[M, ldy] (its own by a local store, the others' by stores over NVLink to
// buffers opened with CUDA IPC). No separate all-gather and no staging buffer in global memory:
// the transfer of a tile overlaps the math of the next one.
//
// Ordering, with a flag protocol in a small control block beside each rank's buffer (all flags
// carry the call's epoch, a per-rank counter advanced by one every call, so nothing is reset):
//   1. arrive: after the programmatic-launch wait (the previous grid on this stream, which may be
//      the last reader of y_full, has finished), every CTA writes arrive[r] = e into every other
//      rank's block. Before its first store a warp waits until all other ranks have arrived at e,
//      so no rank overwrites a buffer its owner may still be reading from the previous call.
//   2. done: each CTA takes a ticket after its stores; the rank's last CTA fences at system scope,
//      writes done[r] = e into every other rank's block, waits until all ranks are done with e,
//      then advances the rank's epoch. When the grid completes, y_full holds every rank's slice.
// Every wait is bounded (kWaitLimitNs); past it the kernel records kErrPeerArrive / kErrPeerDone
// in the device error word, skips the peer stores it was about to make and finishes, so a rank
// that never launched ends its peers' kernels with an error instead of a hang.
// Plain st.global to peer memory only: no TMA or bulk copy touches a peer's buffer.
#pragma once

#include "ptx.cuh"

namespace muse {

constexpr int kMaxPeers = 8;
constexpr unsigned int kErrPeerArrive = 0x401, kErrPeerDone = 0x402;

// One per rank, 256-byte aligned, zero-filled once when allocated (and again on every rank after any
// call that ended with kErrPeerArrive or kErrPeerDone: a timed-out call leaves its flags behind).
struct PeerCtl {
  unsigned int epoch;   // calls this rank has completed
  unsigned int ticket;  // CTAs of the current call that finished their stores (back to 0 after)
  unsigned int pad0[30];
  unsigned int arrive[kMaxPeers];  // arrive[q]: the last call rank q has entered
  unsigned int pad1[24];
  unsigned int done[kMaxPeers];  // done[q]: the last call whose slice rank q has finished storing
  unsigned int pad2[24];
};
static_assert(sizeof(PeerCtl) == 384, "PeerCtl layout");

struct GatherOut {
  uint16_t* y[kMaxPeers];   // each rank's y_full [M, ldy] BF16 (y[rank] is this rank's own)
  PeerCtl* ctl[kMaxPeers];  // each rank's control block (ctl[rank] is this rank's own)
  int P, rank, ldy, col0;
};

__device__ __forceinline__ unsigned int ld_acquire_sys(const unsigned int* p) {
  unsigned int v;
  asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
  return v;
}

// Release / acquire fences (lighter than the sequentially consistent __threadfence forms).
__device__ __forceinline__ void fence_acq_rel_gpu() { asm volatile("fence.acq_rel.gpu;" ::: "memory"); }
__device__ __forceinline__ void fence_acq_rel_sys() { asm volatile("fence.acq_rel.sys;" ::: "memory"); }

__device__ __forceinline__ void st_relaxed_sys(unsigned int* p, unsigned int v) {
  asm volatile("st.relaxed.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Epoch of the call in progress. Read after the programmatic-launch wait: the previous call's
// last CTA advanced it before that grid completed.
__device__ __forceinline__ unsigned int gather_epoch(const GatherOut& g) {
  return *reinterpret_cast<volatile const unsigned int*>(&g.ctl[g.rank]->epoch) + 1u;
}

// Bounded wait until flags[q] >= e (wrap-safe) for every rank q but `skip`. false: timed out
// (recorded).
__device__ __noinline__ bool gather_wait_all(const unsigned int* flags, int P, int skip, unsigned int e,
                                             unsigned int where) {
  const unsigned long long t0 = globaltimer();
  for (int q = 0; q < P; ++q) {
    if (q == skip) continue;
    for (uint32_t i = 1; static_cast<int>(ld_acquire_sys(flags + q) - e) < 0; ++i) {
      if ((i & 15u) == 0u) {
        if (error_raised()) return false;  // another wait already gave up: do not add a second
        if (globaltimer() - t0 > kWaitLimitNs) {
          report_error(where);
          return false;
        }
      }
      __nanosleep(64);
    }
  }
  return true;
}

// Step 1a, by one thread of every CTA right after its programmatic-launch wait and before any
// wait of its own (the stores are idempotent; as every CTA announces before it waits, a rank's
// announcement never waits for another CTA of its grid to be scheduled). Relaxed stores: what
// they announce, that the previous grid on this stream has completed, holds once the wait returned.
__device__ __forceinline__ void gather_announce(const GatherOut& g, unsigned int e) {
  for (int p = 0; p < g.P; ++p)
    if (p != g.rank) st_relaxed_sys(&g.ctl[p]->arrive[g.rank], e);
}

// Step 1b, by every warp that stores, before its first store (lane 0 polls, the warp learns the
// answer by shuffle): waits for every other rank's arrival. true: peers may be written.
__device__ __forceinline__ bool gather_arrived(const GatherOut& g, unsigned int e) {
  int ok = 1;
  if ((threadIdx.x & 31) == 0) ok = gather_wait_all(g.ctl[g.rank]->arrive, g.P, g.rank, e, kErrPeerArrive) ? 1 : 0;
  return __shfl_sync(0xffffffffu, ok, 0) != 0;
}

// One BF16 value to every rank's y_full (row m, local column n). `peers`: false after a timed-out
// arrival, when only this rank's own copy is written.
__device__ __forceinline__ void gather_store(const GatherOut& g, bool peers, int m, int n, uint16_t v) {
  const size_t off = static_cast<size_t>(m) * g.ldy + g.col0 + n;
  if (!peers) {
    g.y[g.rank][off] = v;
    return;
  }
  for (int p = 0; p < g.P; ++p) g.y[p][off] = v;
}

// Eight consecutive BF16 values (one 16-byte word, 16-byte aligned at every rank) likewise.
__device__ __forceinline__ void gather_store8(const GatherOut& g, bool peers, int m, int n, uint4 v) {
  const size_t off = static_cast<size_t>(m) * g.ldy + g.col0 + n;
  const int p0 = peers ? 0 : g.rank, p1 = peers ? g.P : g.rank + 1;
  for (int p = p0; p < p1; ++p) *reinterpret_cast<uint4*>(g.y[p] + off) = v;
}

// Step 2, by one thread of each CTA once the whole CTA has passed a barrier after its stores.
// The CTA's stores are ordered before its ticket by a GPU-scope fence; the last CTA, having seen
// every ticket, makes one system-scope fence (cumulative: it covers every store ordered before the
// tickets it observed) before it raises this rank's done flag at each peer. One system fence a
// launch, not one a CTA. `ctas`: the grid's CTA count.
// A call in which a wait gave up (the device error word is set: this rank's arrival wait timed
// out, so its slice went to its own buffer only) publishes no done flag: a peer that arrives late
// and waits for this rank's slice then ends with kErrPeerDone instead of completing with a y_full
// that silently lacks this rank's columns.
__device__ __forceinline__ void gather_finish(const GatherOut& g, unsigned int e, unsigned int ctas) {
  fence_acq_rel_gpu();  // release: this CTA's stores before its ticket
  PeerCtl* mine = g.ctl[g.rank];
  if (atomicAdd(&mine->ticket, 1u) != ctas - 1u) return;
  fence_acq_rel_gpu();  // acquire: every CTA's stores before what follows
  mine->ticket = 0u;  // the next call starts from 0 (it reads it only after this grid completes)
  if (error_raised()) {
    *reinterpret_cast<volatile unsigned int*>(&mine->epoch) = e;
    return;
  }
  fence_acq_rel_sys();  // release at system scope, before the done flags
  for (int p = 0; p < g.P; ++p)
    if (p != g.rank) st_relaxed_sys(&g.ctl[p]->done[g.rank], e);
  gather_wait_all(mine->done, g.P, g.rank, e, kErrPeerDone);
  *reinterpret_cast<volatile unsigned int*>(&mine->epoch) = e;
}

}  // namespace muse
