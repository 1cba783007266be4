// Inline-PTX helpers for sm_100a: mbarriers, bulk / tensor copies, tcgen05 (TMEM + UMMA),
// cluster barriers and DSMEM loads. Every wait on an mbarrier is bounded: after kWaitLimitNs
// it records a code in the device error word and returns false, so no kernel can hang the GPU.
#pragma once

#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

namespace muse {

// First device-side error wins. 0 = none. Read and cleared by muse_device_error().
__device__ unsigned int g_dev_error = 0;

constexpr unsigned long long kWaitLimitNs = 1000000000ull;  // 1 s: no legitimate wait is near it

enum DevErr : unsigned int {
  kErrNone = 0,
  kErrGemvProducer = 0x101, kErrGemvConsumer = 0x102,
  kErrTcProducer = 0x201, kErrTcMma = 0x202, kErrTcEpilogue = 0x203,
  kErrDrain = 0x301,
};

__device__ __forceinline__ uint32_t smem_u32(const void* p) {
  return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

// `base` (a __shared__ array) rounded up to kAlign bytes by adding an offset to the array itself, so
// the compiler still sees a shared-memory pointer and emits ld/st.shared (rounding the address as an
// integer would turn every access through the result into a slower generic load or store).
template <int kAlign>
__device__ __forceinline__ uint8_t* smem_align(uint8_t* base) {
  const uint32_t a = smem_u32(base);
  return base + ((kAlign - (a & (kAlign - 1))) & (kAlign - 1));
}

__device__ __forceinline__ unsigned long long globaltimer() {
  unsigned long long t;
  asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
  return t;
}

__device__ __forceinline__ void report_error(unsigned int code) { atomicCAS(&g_dev_error, 0u, code); }

__device__ __forceinline__ bool error_raised() {
  return *reinterpret_cast<volatile unsigned int*>(&g_dev_error) != 0u;
}

// ---- per-CTA timestamp trace (off unless the host set a buffer) -----------------------------

// One record per CTA: globaltimer (ns) at entry, after the prologue, when its main loop's last
// data has been consumed, and at exit; plus the SM it ran on.
struct TraceRec {
  unsigned long long t_start, t_ready, t_mainloop, t_end;
  unsigned int smid, block;
  unsigned int x1 = 0u, x2 = 0u, x3 = 0u, x4 = 0u, x5 = 0u, x6 = 0u;  // kernel-specific marks: ns after t_mainloop
};
static_assert(sizeof(TraceRec) == 64, "TraceRec layout");

__device__ __forceinline__ unsigned int smid() {
  unsigned int r;
  asm volatile("mov.u32 %0, %%smid;" : "=r"(r));
  return r;
}

// ---- mbarrier ------------------------------------------------------------------------------

__device__ __forceinline__ void mbar_init(uint64_t* bar, uint32_t count) {
  asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}

__device__ __forceinline__ void fence_mbar_init() {
  asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t* bar) {
  asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}

__device__ __forceinline__ void mbar_expect_tx(uint64_t* bar, uint32_t bytes) {
  asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
               : "memory");
}

// Phase test. MUSE_WAIT_MODE 0: try_wait (may suspend up to the system time limit),
// 1: try_wait with a 200 ns suspend hint, 2: test_wait (never suspends).
#ifndef MUSE_WAIT_MODE
#define MUSE_WAIT_MODE 2
#endif
__device__ __forceinline__ bool mbar_test(uint32_t bar, uint32_t parity) {
  uint32_t ok;
#if MUSE_WAIT_MODE == 0
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
#elif MUSE_WAIT_MODE == 1
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, 200;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
#else
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.test_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
#endif
  return ok != 0;
}

// How often a waiting thread looks at the device error word (another thread's wait gave up): every
// kErrPollNs of waiting, on the clock. The word is one global address that every waiting warp of
// every SM would otherwise load in its polling loop; at one load per poll the L2 slice holding it
// saturates, and since every weight stream crosses every slice, the whole grid's streaming slowed to
// a third (measured on a B200: 430 ns a k block instead of ~150).
constexpr unsigned long long kErrPollNs = 20000ull;

// Bounded wait for the phase of parity `parity` to complete. Returns false (after recording
// `where`) when the limit passes, or once another thread has recorded an error (noticed within
// kErrPollNs).
__device__ __noinline__ bool mbar_wait_slow(uint32_t bar, uint32_t parity, uint32_t where,
                                            unsigned long long limit_ns) {
  const unsigned long long t0 = globaltimer();
  unsigned long long next_poll = t0 + kErrPollNs;
  for (uint32_t i = 1;; ++i) {
    if (mbar_test(bar, parity)) return true;
    if ((i & 31u) == 0u) {
      const unsigned long long t = globaltimer();
      if (t >= next_poll) {
        if (error_raised()) return false;
        if (t - t0 > limit_ns) {
          report_error(where);
          return false;
        }
        next_poll = t + kErrPollNs;
      }
    }
  }
}

__device__ __forceinline__ bool mbar_wait(uint64_t* bar, uint32_t parity, uint32_t where,
                                          unsigned long long limit_ns = kWaitLimitNs) {
  const uint32_t b = smem_u32(bar);
  if (mbar_test(b, parity)) return true;
  return mbar_wait_slow(b, parity, where, limit_ns);
}

// Bounded wait that lets the warp sleep: mbarrier.try_wait suspends the thread until the phase
// completes or a hardware time limit passes, so a waiting warp takes no issue slots from the warps
// that share its scheduler. For roles that wait long (an epilogue waiting for a whole main loop).
__device__ __forceinline__ bool mbar_try_wait(uint32_t bar, uint32_t parity) {
  uint32_t ok;
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
      "selp.u32 %0, 1, 0, p;\n\t}"
      : "=r"(ok)
      : "r"(bar), "r"(parity)
      : "memory");
  return ok != 0;
}

__device__ __noinline__ bool mbar_wait_idle_slow(uint32_t bar, uint32_t parity, uint32_t where,
                                                 unsigned long long limit_ns) {
  const unsigned long long t0 = globaltimer();
  unsigned long long next_poll = t0 + kErrPollNs;
  for (;;) {
    if (mbar_try_wait(bar, parity)) return true;
    const unsigned long long t = globaltimer();
    if (t >= next_poll) {
      if (error_raised()) return false;
      if (t - t0 > limit_ns) {
        report_error(where);
        return false;
      }
      next_poll = t + kErrPollNs;
    }
  }
}

__device__ __forceinline__ bool mbar_wait_idle(uint64_t* bar, uint32_t parity, uint32_t where,
                                               unsigned long long limit_ns = kWaitLimitNs) {
  const uint32_t b = smem_u32(bar);
  if (mbar_try_wait(b, parity)) return true;
  return mbar_wait_idle_slow(b, parity, where, limit_ns);
}

// A position in a `stages`-deep ring: the slot and the parity of its current phase, advanced by
// increments. Hot loops use this instead of i % stages and i / stages, which for 64-bit or
// runtime divisors cost tens of dependent instructions in the single issuing lane.
struct Ring {
  int slot = 0;
  uint32_t phase = 0;
  __device__ __forceinline__ void next(int stages) {
    if (++slot == stages) {
      slot = 0;
      phase ^= 1u;
    }
  }
};

// ---- programmatic dependent launch -------------------------------------------------------------

// Waits until the grids this one depends on (launched before it in the stream) have completed and
// their memory is visible. Returns at once when the launch was not programmatic.
__device__ __forceinline__ void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Lets the next programmatic launch in the stream start scheduling its CTAs.
__device__ __forceinline__ void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ---- split-K tickets ---------------------------------------------------------------------------

// Called by one thread after a barrier that follows every partial store of its group: publishes
// the group's partials and takes a ticket; returns the ticket value. The atomic's release half is
// cumulative: the group's stores happen before it through the barrier, so they are visible to
// whichever thread acquires the counter after it (no separate fence, which would cost a second
// round trip to L2 on the split-K tail); its acquire half lets the reducer see every earlier
// contributor's partial.
__device__ __forceinline__ int ticket_acq_rel(int* counter) {
  int old;
  asm volatile("atom.add.acq_rel.gpu.s32 %0, [%1], 1;" : "=r"(old) : "l"(counter) : "memory");
  return old;
}

// Sum of `n` FP32 partials of 16 values each, laid out `stride` floats apart with value j at
// +j * 128, added in index order; the loads of 6 partials at a time are in flight together.
__device__ __forceinline__ void sum_partials16(const float* base, int n, size_t stride, float (&sum)[16]) {
#pragma unroll
  for (int j = 0; j < 16; ++j) sum[j] = 0.f;
  for (int p0 = 0; p0 < n; p0 += 6) {
    float v[6][16];
#pragma unroll
    for (int p = 0; p < 6; ++p) {
      if (p0 + p < n) {
        const float* src = base + static_cast<size_t>(p0 + p) * stride;
#pragma unroll
        for (int j = 0; j < 16; ++j) v[p][j] = __ldcg(src + j * 128);
      }
    }
#pragma unroll
    for (int p = 0; p < 6; ++p) {
      if (p0 + p < n) {
#pragma unroll
        for (int j = 0; j < 16; ++j) sum[j] += v[p][j];
      }
    }
  }
}

// ---- L2 cache policies -----------------------------------------------------------------------

__device__ __forceinline__ uint64_t policy_evict_first() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_normal() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_normal.b64 %0, 1.0;" : "=l"(p));
  return p;
}

__device__ __forceinline__ uint64_t policy_evict_last() {
  uint64_t p;
  asm volatile("createpolicy.fractional.L2::evict_last.b64 %0, 1.0;" : "=l"(p));
  return p;
}

// ---- bulk copies (no multicast anywhere in this library) ------------------------------------

// Contiguous global -> this CTA's shared memory; completes `bytes` of transaction on `bar`.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar,
                                         uint64_t policy) {
  asm volatile(
      "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], %4;" ::"r"(
          smem_u32(dst)),
      "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(policy)
      : "memory");
}

// 2-D tiled tensor load into this CTA's shared memory. c0 = innermost coordinate (elements),
// which callers keep a multiple of 64 BF16 elements (128 bytes).
__device__ __forceinline__ void tma_load_2d(void* dst, const CUtensorMap* map, uint64_t* bar, int c0, int c1,
                                            uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(smem_u32(bar)), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// This CTA's shared memory -> global, contiguous, tracked by the issuing thread's bulk groups.
// dst, src 16-byte aligned; bytes a multiple of 16.
__device__ __forceinline__ void bulk_s2g(void* dst, const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.global.shared::cta.bulk_group [%0], [%1], %2;" ::"l"(dst), "r"(smem_u32(src)), "r"(bytes)
               : "memory");
}

// 2-D tiled tensor store from this CTA's shared memory (the map's box; the parts of the box past
// the tensor's edges are not written). Coordinates non-negative, c0 x element size a multiple of 16.
__device__ __forceinline__ void tma_store_2d(const CUtensorMap* map, const void* src, int c0, int c1) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group [%0, {%2, %3}], [%1];" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1)
               : "memory");
}

// The same with an L2 eviction policy for the written lines (y written once and never re-read here).
__device__ __forceinline__ void tma_store_2d_hint(const CUtensorMap* map, const void* src, int c0, int c1,
                                                  uint64_t policy) {
  asm volatile("cp.async.bulk.tensor.2d.global.shared::cta.bulk_group.L2::cache_hint [%0, {%2, %3}], [%1], %4;" ::"l"(
                   reinterpret_cast<uint64_t>(map)),
               "r"(smem_u32(src)), "r"(c0), "r"(c1), "l"(policy)
               : "memory");
}

__device__ __forceinline__ void bulk_commit() { asm volatile("cp.async.bulk.commit_group;" ::: "memory"); }
// Every bulk group this thread committed has completed (its writes performed).
__device__ __forceinline__ void bulk_wait_all() { asm volatile("cp.async.bulk.wait_group 0;" ::: "memory"); }
// Every bulk group this thread committed has finished reading its shared-memory source.
__device__ __forceinline__ void bulk_wait_read_all() { asm volatile("cp.async.bulk.wait_group.read 0;" ::: "memory"); }

// Generic-proxy writes to shared memory before a later async-proxy read of them (bulk copy, UMMA).
__device__ __forceinline__ void fence_proxy_async_shared() { asm volatile("fence.proxy.async.shared::cta;" ::: "memory"); }
// The same between the generic and the async proxy for global memory.
__device__ __forceinline__ void fence_proxy_async_global() { asm volatile("fence.proxy.async.global;" ::: "memory"); }

__device__ __forceinline__ void st_shared_f32(uint32_t addr, float v) {
  asm volatile("st.shared.f32 [%0], %1;" ::"r"(addr), "f"(v) : "memory");
}
__device__ __forceinline__ void st_shared_v4u(uint32_t addr, uint32_t a, uint32_t b, uint32_t c, uint32_t d) {
  asm volatile("st.shared.v4.u32 [%0], {%1, %2, %3, %4};" ::"r"(addr), "r"(a), "r"(b), "r"(c), "r"(d) : "memory");
}
__device__ __forceinline__ void st_shared_v2(uint32_t addr, uint32_t a, uint32_t b) {
  asm volatile("st.shared.v2.u32 [%0], {%1, %2};" ::"r"(addr), "r"(a), "r"(b) : "memory");
}
__device__ __forceinline__ float4 ld_shared_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr) : "memory");
  return v;
}

// Prefetch `bytes` (multiple of 16, 16-byte aligned) of global memory into L2, no completion signal.
__device__ __forceinline__ void bulk_prefetch_l2(const void* src, uint32_t bytes) {
  asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

__device__ __forceinline__ void prefetch_tensormap(const CUtensorMap* map) {
  asm volatile("prefetch.tensormap [%0];" ::"l"(reinterpret_cast<uint64_t>(map)) : "memory");
}

// ---- cluster -------------------------------------------------------------------------------

__device__ __forceinline__ uint32_t cluster_ctarank() {
  uint32_t r;
  asm volatile("mov.u32 %0, %%cluster_ctarank;" : "=r"(r));
  return r;
}

__device__ __forceinline__ void cluster_sync() {
  asm volatile("barrier.cluster.arrive.release;\n\tbarrier.cluster.wait.acquire;" ::: "memory");
}

__device__ __forceinline__ uint32_t map_peer(uint32_t local_smem, uint32_t rank) {
  uint32_t r;
  asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(r) : "r"(local_smem), "r"(rank));
  return r;
}

__device__ __forceinline__ float ld_dsmem_f32(uint32_t addr) {
  float v;
  asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(addr));
  return v;
}

__device__ __forceinline__ float4 ld_dsmem_v4(uint32_t addr) {
  float4 v;
  asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];" : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w) : "r"(addr));
  return v;
}

// ---- tcgen05: TMEM allocation, UMMA, TMEM loads ---------------------------------------------

// Warp-wide. Writes the allocated TMEM base address to *slot (shared memory).
__device__ __forceinline__ void tmem_alloc(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols) : "memory");
}

__device__ __forceinline__ void tc_fence_before() {
  asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory");
}

__device__ __forceinline__ void tc_fence_after() {
  asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory");
}

// UMMA shared-memory descriptor for a K-major operand tile stored with the 128-byte swizzle:
// rows of 128 bytes, 8-row (1024-byte) swizzle atoms stacked along M/N (stride 1024 bytes).
// Fields: start address >> 4 [0,14), leading byte offset >> 4 [16,30) (unused for swizzled
// K-major, set to 1), stride byte offset >> 4 [32,46), descriptor version 1 [46,48),
// layout 2 = SWIZZLE_128B [61,64).
__device__ __forceinline__ uint64_t umma_desc_sw128(uint32_t saddr) {
  return static_cast<uint64_t>((saddr & 0x3FFFFu) >> 4) | (static_cast<uint64_t>(1) << 16) |
         (static_cast<uint64_t>(1024 >> 4) << 32) | (static_cast<uint64_t>(1) << 46) |
         (static_cast<uint64_t>(2) << 61);
}

// Instruction descriptor, kind::f16: D FP32 [4,6)=1, A BF16 [7,10)=1, B BF16 [10,13)=1, both
// K-major (bits 15, 16 = 0), N >> 3 at [17,23), M >> 4 at [24,29).
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
  return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
         (static_cast<uint32_t>(m >> 4) << 24);
}

// D[tmem] (+)= A[smem desc] * B[smem desc]^T, one 16-deep K step. Issued by one thread.
__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                          uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive on `bar` once every tcgen05 operation this thread issued before has completed.
__device__ __forceinline__ void umma_commit(uint64_t* bar) {
  asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(
                   smem_u32(bar))
               : "memory");
}

// Warp-wide: lane i gets 16 consecutive FP32 columns of TMEM lane (base lane + i).
__device__ __forceinline__ void tmem_ld16(uint32_t taddr, float (&v)[16]) {
  uint32_t r[16];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15}, [%16];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}

// 32 consecutive FP32 columns of this warp's 32 TMEM lanes (one load, one wait).
__device__ __forceinline__ void tmem_ld32(uint32_t taddr, float (&v)[32]) {
  uint32_t r[32];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, %14, "
      "%15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31}, [%32];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

// 64 consecutive FP32 columns of this warp's 32 TMEM lanes (one load, one wait).
__device__ __forceinline__ void tmem_ld64(uint32_t taddr, float (&v)[64]) {
  uint32_t r[64];
  asm volatile(
      "tcgen05.ld.sync.aligned.32x32b.x64.b32 {%0, %1, %2, %3, %4, %5, %6, %7, %8, %9, %10, %11, %12, %13, "
      "%14, %15, %16, %17, %18, %19, %20, %21, %22, %23, %24, %25, %26, %27, %28, %29, %30, %31, %32, %33, "
      "%34, %35, %36, %37, %38, %39, %40, %41, %42, %43, %44, %45, %46, %47, %48, %49, %50, %51, %52, %53, "
      "%54, %55, %56, %57, %58, %59, %60, %61, %62, %63}, [%64];"
      : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
        "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
        "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]),
        "=r"(r[23]), "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]),
        "=r"(r[30]), "=r"(r[31]), "=r"(r[32]), "=r"(r[33]), "=r"(r[34]), "=r"(r[35]), "=r"(r[36]),
        "=r"(r[37]), "=r"(r[38]), "=r"(r[39]), "=r"(r[40]), "=r"(r[41]), "=r"(r[42]), "=r"(r[43]),
        "=r"(r[44]), "=r"(r[45]), "=r"(r[46]), "=r"(r[47]), "=r"(r[48]), "=r"(r[49]), "=r"(r[50]),
        "=r"(r[51]), "=r"(r[52]), "=r"(r[53]), "=r"(r[54]), "=r"(r[55]), "=r"(r[56]), "=r"(r[57]),
        "=r"(r[58]), "=r"(r[59]), "=r"(r[60]), "=r"(r[61]), "=r"(r[62]), "=r"(r[63])
      : "r"(taddr));
  asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
  for (int i = 0; i < 64; ++i) v[i] = __uint_as_float(r[i]);
}

// ---- tcgen05 across a CTA pair (cta_group::2) -------------------------------------------------

// Both CTAs of the pair, same warp, same shared-memory slot: the same TMEM columns in each.
__device__ __forceinline__ void tmem_alloc_pair(uint32_t* slot, uint32_t cols) {
  asm volatile("tcgen05.alloc.cta_group::2.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(smem_u32(slot)),
               "r"(cols)
               : "memory");
  asm volatile("tcgen05.relinquish_alloc_permit.cta_group::2.sync.aligned;" ::: "memory");
}

__device__ __forceinline__ void tmem_dealloc_pair(uint32_t base, uint32_t cols) {
  asm volatile("tcgen05.dealloc.cta_group::2.sync.aligned.b32 %0, %1;" ::"r"(base), "r"(cols) : "memory");
}

// D (both CTAs' TMEM) (+)= A * B^T with A's and B's halves in the two CTAs' shared memory at the
// descriptors' offsets. Issued by one thread of the pair's even CTA.
__device__ __forceinline__ void umma_bf16_pair(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc,
                                               uint32_t accumulate) {
  asm volatile(
      "{\n\t.reg .pred p;\n\t"
      "setp.ne.b32 p, %4, 0;\n\t"
      "tcgen05.mma.cta_group::2.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
      "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
      : "memory");
}

// Arrive (once) on the mbarrier at this shared-memory offset in every CTA of `cta_mask` when the
// pair's earlier tcgen05 operations issued by this thread have completed.
__device__ __forceinline__ void umma_commit_pair_mc(uint64_t* bar, uint16_t cta_mask) {
  asm volatile(
      "tcgen05.commit.cta_group::2.mbarrier::arrive::one.shared::cluster.multicast::cluster.b64 [%0], %1;" ::"r"(
          smem_u32(bar)),
      "h"(cta_mask)
      : "memory");
}

// 2-D tensor load into this CTA's shared memory whose transaction bytes complete on the mbarrier at
// the shared::cluster address `bar_cluster` (the pair's even CTA). No multicast.
__device__ __forceinline__ void tma_load_2d_pair(void* dst, const CUtensorMap* map, uint32_t bar_cluster, int c0,
                                                 int c1, uint64_t policy) {
  asm volatile(
      "cp.async.bulk.tensor.2d.cta_group::2.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint"
      " [%0], [%1, {%3, %4}], [%2], %5;" ::"r"(smem_u32(dst)),
      "l"(reinterpret_cast<uint64_t>(map)), "r"(bar_cluster), "r"(c0), "r"(c1), "l"(policy)
      : "memory");
}

// Arrive on an mbarrier in another CTA of the cluster (shared::cluster address), release at cluster scope.
__device__ __forceinline__ void mbar_arrive_cluster(uint32_t bar_cluster) {
  asm volatile("mbarrier.arrive.release.cluster.shared::cluster.b64 _, [%0];" ::"r"(bar_cluster) : "memory");
}

// ---- numeric helpers ------------------------------------------------------------------------

__device__ __forceinline__ float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
__device__ __forceinline__ float bf16hi(uint32_t w) { return __uint_as_float(w & 0xFFFF0000u); }
__device__ __forceinline__ float bf16f(uint16_t w) { return __uint_as_float(static_cast<uint32_t>(w) << 16); }

// FP32 -> BF16 bits, round to nearest even (NaN stays NaN).
__device__ __forceinline__ uint16_t f32_to_bf16(float f) {
  uint32_t u = __float_as_uint(f);
  if ((u & 0x7FFFFFFFu) > 0x7F800000u) return static_cast<uint16_t>((u >> 16) | 0x0040u);
  u += 0x7FFFu + ((u >> 16) & 1u);
  return static_cast<uint16_t>(u >> 16);
}

// Two FP32 values -> two BF16 (lo in the low half), round to nearest even: one cvt.rn.bf16x2.f32
// (the same bits as f32_to_bf16 for every finite value and infinity; a NaN stays a NaN) instead of
// about a dozen integer operations, in the epilogues that convert every output.
__device__ __forceinline__ uint32_t pack_bf16x2(float lo, float hi) {
  uint32_t r;
  asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
  return r;
}

// acc_even += w.lo * x.lo, acc_odd += w.hi * x.hi for two BF16 pairs, each product exact and each
// sum rounded once to FP32 (mixed-precision FMA: the same numbers as widening both to FP32 first).
__device__ __forceinline__ void fma_bf16x2(uint32_t w2, uint32_t x2, float& acc_even, float& acc_odd) {
  asm("{\n\t.reg .b16 wl, wh, xl, xh;\n\tmov.b32 {wl, wh}, %2;\n\tmov.b32 {xl, xh}, %3;\n\t"
      "fma.rn.f32.bf16 %0, wl, xl, %0;\n\tfma.rn.f32.bf16 %1, wh, xh, %1;\n\t}"
      : "+f"(acc_even), "+f"(acc_odd)
      : "r"(w2), "r"(x2));
}

__device__ __forceinline__ uint4 ldg_nc_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.nc.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p));
  return v;
}

// 16 bytes of streamed read-only data (weights): not kept in L1, L2 eviction by `policy`.
__device__ __forceinline__ uint4 ldg_stream_v4(const void* p, uint64_t policy) {
  uint4 v;
  asm volatile("ld.global.nc.L1::no_allocate.L2::cache_hint.v4.u32 {%0, %1, %2, %3}, [%4], %5;"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p), "l"(policy));
  return v;
}

// 16 bytes cached in L2 only: data the previous grid may have written (read after its wait).
__device__ __forceinline__ uint4 ldg_cg_v4(const void* p) {
  uint4 v;
  asm volatile("ld.global.cg.v4.u32 {%0, %1, %2, %3}, [%4];"
               : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
               : "l"(p)
               : "memory");
  return v;
}

__device__ __forceinline__ uint4 ld_shared_v4u(uint32_t addr) {
  uint4 v;
  asm volatile("ld.shared.v4.u32 {%0, %1, %2, %3}, [%4];" : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w) : "r"(addr));
  return v;
}

}  // namespace muse
