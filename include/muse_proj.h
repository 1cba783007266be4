/*
 * muse_proj.h — C ABI of the B200 (sm_100a) BF16 projection library, libmuse_proj.so.
 *
 * y[M, N] = x[M, K] . W[N, K]^T with BF16 inputs, FP32 accumulation and a round-to-nearest-even
 * BF16 output: the dense projection that the reference serves from kernel_fn
 * (submission.py:1156-1170). Plain pointers and sizes only; every function returns MUSE_OK (0)
 * or a negative MUSE_ERR_* code and never throws across the ABI; muse_last_error() gives the
 * calling thread's last message. No function allocates device memory. Launches go on the
 * stream given (a cudaStream_t passed as void*), so they can be captured in a CUDA graph.
 *
 * Pointers named x, w, y, planes, bases, esc_* in the muse_proj_* calls are DEVICE pointers;
 * the muse_encode12 / muse_decode12 buffers are HOST pointers, the muse_encode12_device* ones
 * DEVICE pointers.
 */
#ifndef MUSE_PROJ_H
#define MUSE_PROJ_H

#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Status codes. */
#define MUSE_OK 0
#define MUSE_ERR_INVALID (-1)   /* null pointer or non-positive size */
#define MUSE_ERR_ALIGN (-2)     /* pointer not 16-byte aligned, or K * 2 bytes not a multiple of 16 */
#define MUSE_ERR_SHAPE (-3)     /* shape outside what the chosen kernel supports */
#define MUSE_ERR_CAPACITY (-4)  /* a caller-provided buffer is too small (see the count written) */
#define MUSE_ERR_CUDA (-5)      /* a CUDA runtime / driver call failed (message has the name) */
#define MUSE_ERR_TIMEOUT (-6)   /* the device error word was set: a kernel's bounded wait expired, or the
                                 * device encoder skipped an escape outside its buffer (0x501) */
#define MUSE_ERR_PLAN (-7)      /* unknown kernel id or plan field out of range */

/* Kernels a plan can name. */
#define MUSE_KERNEL_GEMV_BF16 1 /* streaming CUDA-core GEMV, BF16 W, M <= 8 */
#define MUSE_KERNEL_GEMV_12B 2  /* streaming CUDA-core GEMV, 12-bit W, M <= 8 */
#define MUSE_KERNEL_TC_TILE 3   /* tcgen05 128 x tile_n tiles, K split across a cluster or through scratch */
#define MUSE_KERNEL_TC_STREAMK 4 /* tcgen05 stream-K over packed tiles: equal work per CTA, one wave */
#define MUSE_KERNEL_TC_GEMM 5    /* persistent tcgen05 GEMM, 128 tokens x 256 W rows a tile (prefill) */
#define MUSE_KERNEL_TC_GEMM2 6   /* persistent tcgen05 GEMM on CTA pairs (cta_group::2), 256 x 256 a tile */
#define MUSE_KERNEL_TC_12B 7     /* stream-K tcgen05 on 12-bit tiles: W decoded to BF16 in shared memory */
#define MUSE_KERNEL_TC_SKINNY 8  /* stream-K tcgen05 over packed tiles with W as the B operand (256 W rows an MMA) */
#define MUSE_KERNEL_F32_GEMV 9   /* FP32 W on CUDA cores (the router), M <= 32 */
#define MUSE_KERNEL_GEMV_12T 10  /* 12-bit tiles on CUDA cores, decoded in registers, M <= 4 */
/* tcgen05 over row windows of the packed tiles, M <= 128: each CTA streams its own rows of W over K (no
 * split-K fix-up), tokens as the A operand; optional K split over a cluster of 2 or 4 (DSMEM sum). */
#define MUSE_KERNEL_TC_ROWS 11
/* persistent tcgen05 GEMM on CTA pairs with 256 tokens x 512 W rows a tile (two N = 256 UMMAs sharing an x
 * stage: a quarter fewer operand bytes a FLOP than TC_GEMM2); prefill with many W rows */
#define MUSE_KERNEL_TC_WIDE 12
/* tcgen05 on CTA pairs with W as the A operand: 256 W rows x tile_n tokens a pair, K split `split` ways
 * across pairs that reduce the split together (each sums a slice of the tokens from every partial in
 * scratch, in split order); medium M (about 32 .. 512 tokens). With MUSE_FLAG_STREAMK the (tile, k block)
 * units are cut into equal runs over every resident pair instead. A split or stream-K grid must fit in one
 * wave (the host refuses a larger one) because its pairs wait for one another: a pair that cannot be
 * scheduled within 1 s (another kernel holding SMs indefinitely) ends the launch with device error
 * 0x904 / 0x914, never a hang. */
#define MUSE_KERNEL_TC_PAIRK 13
/* CUDA-core GEMV over the packed tiles for 1..4 tokens, built for one-call latency: each warp loads 1, 2, 4 or 8
 * adjacent 4-row quads of one K segment straight into registers (16 loads a lane in flight, the first
 * issued before the programmatic-launch wait), no ring, barriers, tensor memory or scratch; a CTA's warps
 * of one quad group add their K segments in segment order. */
#define MUSE_KERNEL_GEMV_TILES 14

/* Plan flags. */
#define MUSE_FLAG_GLOBAL_SPLIT 1 /* TC_TILE: reduce K-split partials through caller scratch instead of a cluster */
/* Programmatic dependent launch: the kernel may start while the previous kernel in the stream
 * finishes; it streams its first weights before waiting for that kernel, and touches x, y and
 * scratch only after. Only for weights that the preceding kernel in the stream does not write. */
#define MUSE_FLAG_PDL 2
/* TC_GEMM2 and TC_PAIRK: stream-K schedule. The (tile, k block) units are cut into equal runs, one per
 * CTA pair, so a grid of few tiles still keeps every pair busy; tiles shared by several pairs are summed
 * from FP32 partials in scratch (muse_scratch_bytes) in a fixed order. TC_PAIRK: every pair resident at
 * once and runs of at most one tile (the host refuses other grids); each contributor of a tile reduces
 * a 16-token-aligned slice of it. */
#define MUSE_FLAG_STREAMK 4
/* TC_GEMM2: the whole waves of 256 x 256 tiles run persistently and only the tiles left over after the
 * last whole wave of CTA pairs run stream-K (their units cut into equal runs over every pair, summed
 * from partials in scratch by each tile's last contributor in a fixed order), so the last wave leaves no
 * pair idle. Excludes MUSE_FLAG_STREAMK. */
#define MUSE_FLAG_SK_TAIL 8

/* How one projection runs. Zero fields take the kernel's default. */
typedef struct MusePlan {
  int32_t kernel; /* MUSE_KERNEL_* */
  int32_t split;  /* TC_TILE: CTAs splitting K (cluster: 1..16; global: 1..64); TC_ROWS: 1, 2 or 4 (cluster);
                   * TC_GEMM2, TC_WIDE: 256-token tiles walked together as a group (0 = as many as keep 32 MB of x);
                   * TC_PAIRK: CTA pairs splitting K (1..64, at most tile_n); GEMV_TILES: warps splitting each
                   * 4-row quad's K, a divisor of warps (0 = about 16 k blocks a warp) */
  int32_t tile_n; /* tensor-core kernels: tokens per tile, 16/32/64/128 (TC_TILE, TC_STREAMK also 256; TC_PAIRK any
                   * multiple of 16 up to 256) */
  int32_t stages; /* shared-memory ring depth (0 = kernel default) */
  int32_t ctas;   /* GEMV, TC_STREAMK, TC_SKINNY, TC_12B, TC_ROWS: CTAs in the grid (0 = one per SM); TC_GEMM2,
                   * TC_WIDE, TC_PAIRK with MUSE_FLAG_STREAMK: 2 x the CTA pairs (0 = every pair that fits) */
  int32_t warps;  /* GEMV: consumer warps per CTA: 4, 8 or 16 (0 = 8); GEMV_TILES: warps per CTA, 1..16 (0 = 8) */
  int32_t chunk;  /* GEMV: units per bulk copy (0 = about 16 KB); GEMV_TILES: adjacent 4-row quads a warp, 1, 2, 4 or 8
                   * (8: M <= 2; 0 = 2) */
  int32_t flags;  /* MUSE_FLAG_* */
} MusePlan;

/* A 12-bit encoded weight resident on the device (see muse_encode12 for the format). */
typedef struct MuseEnc12 {
  const uint8_t* planes;   /* N * K * 3 / 2 bytes */
  const uint8_t* bases;    /* ceil(N / 128) * (K / 128) bytes */
  const int32_t* esc_ptr;  /* N + 1 */
  const uint32_t* esc_val; /* n_esc entries */
  int64_t n, k, n_esc;
} MuseEnc12;

/*
 * Per-CTA timestamp trace for the launches that follow (debug / profiling aid; NULL turns it
 * off). `records` is a device buffer of `capacity` 64-byte records, one per CTA (CTAs past the
 * capacity are not traced): u64 globaltimer ns at kernel entry, after the prologue, after the
 * main loop, at exit; u32 SM id; u32 CTA index; six u32 kernel-specific marks (ns after the main
 * loop; 0 where a kernel sets none). Process-wide setting.
 * No counterpart in the reference (it profiled through its judge's kernel table).
 */
int muse_set_trace(void* records, int64_t capacity);

/*
 * Streaming-read floor: reads `bytes` of device memory at `src` into shared memory with 1-D bulk
 * copies of `chunk` bytes (a ring of `stages` per CTA, `ctas` CTAs, 0 = one per SM; CTA c takes the
 * c-th contiguous share) and nothing else, adding the number of chunks that landed to the device
 * counter *count (ceil(bytes / chunk) when all did). The same copy path and grid shapes the
 * projections stream their weights with, so its time for a projection's bytes is the floor that
 * projection is measured against. bytes and chunk multiples of 16, src 16-byte aligned.
 * No counterpart in the reference (it estimated W streaming with a loads-only kernel variant,
 * qkv_tma.py:21-39).
 */
int muse_stream_read(const void* src, int64_t bytes, int64_t chunk, int stages, int ctas, unsigned int* count,
                     void* stream);

/* Library version string. */
const char* muse_version(void);

/* The calling thread's last error message ("" if none). */
const char* muse_last_error(void);

/* Number of SMs of the current device. */
int muse_sm_count(int* out);

/*
 * Reads the device error word that bounded waits set on timeout (and the device encoder on an
 * escape outside its buffer, 0x501), writes it to *code (0 = none) and clears it. Synchronizes `stream`. Returns MUSE_ERR_TIMEOUT when it was set.
 * No counterpart in the reference (its kernels have no bounded waits).
 */
int muse_device_error(int* code, void* stream);

/* How W is held, for muse_plan_default. */
#define MUSE_WEIGHTS_ROW_MAJOR 0 /* BF16 [N, K] row-major (muse_proj_bf16) */
#define MUSE_WEIGHTS_12B 1       /* 12-bit planes (muse_proj_12b) */
#define MUSE_WEIGHTS_TILES 2     /* packed tiles (muse_proj_bf16_tiles; TC_GEMM2 and TC_STREAMK plans need scratch) */
#define MUSE_WEIGHTS_12B_TILES 3 /* 12-bit tiles (muse_proj_12b_tiles; needs scratch) */
#define MUSE_WEIGHTS_F32 4        /* FP32 W and its hi | lo tiles (muse_proj_f32, the router) */

/*
 * The library's default plan for a shape and weight format (MUSE_WEIGHTS_*). Replaces the
 * reference's per-shape tables' fallback rule (submission.py:76-127, 900-908): shapes no table
 * row names get this plan. Packed tiles: GEMV_TILES at M <= 2 (when x fits its shared memory),
 * stream-K up to 128 tokens, the pair GEMMs above 256.
 */
int muse_plan_default(int64_t m, int64_t n, int64_t k, int weights, MusePlan* out);

/*
 * Bytes of device scratch a plan needs (0 for most plans). Scratch holds the per-tile split-K
 * counters (first 64 KB) and FP32 partials of MUSE_FLAG_GLOBAL_SPLIT plans. The caller zeroes it
 * once; every launch leaves the counters at zero again (after a device error, zero it again).
 * Launches that share one scratch buffer must not overlap in time (use one per stream): they would
 * mix their tile counters and partials.
 * No counterpart in the reference beyond its split-K counters (submission.py:112, 1126).
 */
int muse_scratch_bytes(int64_t m, int64_t n, int64_t k, const MusePlan* plan, int64_t* bytes);

/*
 * y = x . W^T for BF16 W [N, K] (row-major, rows contiguous; W[:n] of a bigger matrix is the
 * same pointer). Replaces, by plan->kernel:
 *   MUSE_KERNEL_GEMV_BF16: the Triton split-K bf16_gemm (submission.py:1084-1107) at few tokens;
 *   MUSE_KERNEL_TC_TILE:   TmaGemm.__call__ / wa_gemm (submission.py:977-988, 799-890) and the
 *                          cuBLAS F.linear fallback (submission.py:1170; baseline.py:60).
 * Needs x, w, y 16-byte aligned and K % 8 == 0 (GEMV: K % 256 == 0, M <= 8). scratch may be NULL
 * when muse_scratch_bytes reports 0.
 */
int muse_proj_bf16(const void* x, const void* w, void* y, int64_t m, int64_t n, int64_t k, const MusePlan* plan,
                   void* scratch, int64_t scratch_bytes, void* stream);

/*
 * Bytes of the packed-tile copy of W [N, K] made by muse_pack_tiles:
 * ceil(N / 128) * ceil(K / 64) * 16384.
 */
int muse_tiles_bytes(int64_t n, int64_t k, int64_t* bytes);

/*
 * Repacks row-major BF16 W [N, K] (device) into contiguous 16 KB tiles of 128 rows x 64 k, each in
 * the 128-byte-swizzled order the tensor cores read, zero-padded at the edges (device kernel on
 * `stream`). Lossless. Replaces pack_w_tiles (submission.py:926-934), which packed 64 * wg-row
 * tiles for the Hopper kernel.
 */
int muse_pack_tiles(const void* w, void* tiles, int64_t n, int64_t k, void* stream);

/*
 * y = x . W^T with W given as packed tiles (muse_pack_tiles of the full W: the first
 * ceil(n / 128) row tiles serve W[:n]). plan->kernel: MUSE_KERNEL_TC_TILE,
 * MUSE_KERNEL_TC_STREAMK or MUSE_KERNEL_TC_SKINNY (both always need scratch, see
 * muse_scratch_bytes; TC_SKINNY reads two tiles a k block as one 256-row B operand) or
 * MUSE_KERNEL_TC_GEMM / MUSE_KERNEL_TC_GEMM2 (prefill; replace the cuBLAS F.linear that served
 * the reference's large shapes, submission.py:1170; also MUSE_KERNEL_TC_WIDE), MUSE_KERNEL_TC_PAIRK (medium M; scratch when
 * split > 1; replaces wa_gemm's cluster split-K, submission.py:855-889), MUSE_KERNEL_TC_ROWS (M <= 128, no scratch;
 * replaces nf12_gemv / wa_gemm at few tokens, submission.py:357-474, 799-890) or MUSE_KERNEL_GEMV_TILES
 * (M <= 4, no scratch; the BF16 counterpart of the reference's CUDA-core nf12_gemv, submission.py:357-474, for
 * decode shapes its Triton bf16_gemm served, submission.py:209-251, 1084-1107). Each pipeline
 * stage moves one contiguous 16 KB tile with a 1-D bulk copy. Replaces TmaGemm.__call__
 * (submission.py:977-988), which read its pre-swizzled W the same way, and the Triton split-K
 * bf16_gemm with its atomic tile tickets (submission.py:209-251, 1084-1107).
 */
int muse_proj_bf16_tiles(const void* x, const void* tiles, void* y, int64_t m, int64_t n, int64_t k,
                         const MusePlan* plan, void* scratch, int64_t scratch_bytes, void* stream);

/* ---- window-major weights for MUSE_KERNEL_TC_ROWS ------------------------------------------------ */

/* The number of row windows a TC_ROWS plan splits N into for this shape (plan->ctas, else the
 * SM count, divided by plan->split; at most ceil(N / 16)): the `groups` of muse_pack_rows. */
int muse_rows_groups(int64_t m, int64_t n, int64_t k, const MusePlan* plan, int* groups);

/* Device bytes of the window-major copy of W [N, K]: ceil(N / 16) * 16 * ceil(K / 64) * 128. */
int muse_rows_bytes(int64_t n, int64_t k, int groups, int64_t* bytes);

/*
 * Re-lays row-major BF16 W [N, K] (device) for `groups` row windows: the N rows are spread over the
 * windows in 16-row units (windows differ by at most 16 rows); window g's rows for each 64-wide k
 * block form one contiguous block, blocks in k order, in the 128-byte-swizzled order the tensor
 * cores read (row r's 16-byte chunk c at c ^ (r % 8)); rows past N and columns past K are zero.
 * Lossless. Device kernel on `stream`. No counterpart in the reference (its nf12 planes and wgmma
 * tiles were laid out per kernel too, submission.py:591-626, 926-934).
 */
int muse_pack_rows(const void* w, void* out, int64_t n, int64_t k, int groups, void* stream);

/*
 * y = x . W^T with W as the window-major copy (muse_pack_rows with groups = muse_rows_groups for this
 * plan and shape): each CTA streams its own rows of W over K as one sequential byte range, with no
 * split-K fix-up. plan->kernel must be MUSE_KERNEL_TC_ROWS; M <= 128; no scratch. Replaces
 * nf12_cuda_gemv / nf12_gemv and wa_gemm at few tokens (submission.py:660-673, 357-474, 799-890).
 * x 16-byte aligned, K % 8 == 0.
 */
int muse_proj_bf16_rows(const void* x, const void* wrows, void* y, int64_t m, int64_t n, int64_t k, const MusePlan* plan,
                        void* stream);

/* ---- all-gather fused into the projection's epilogue (column-parallel shards over NVLink) ---- */

#define MUSE_MAX_PEERS 8
#define MUSE_IPC_HANDLE_BYTES 64

/* Each rank's output and control block, as this process sees them (its own and peers' opened
 * with muse_ipc_open). y[p] is rank p's y_full [M, ldy] BF16; this rank writes its columns
 * col0 .. col0 + N into every rank's copy. ctl[p] is rank p's control block of
 * muse_peer_ctl_bytes bytes, 128-byte aligned, zero-filled once before first use. */
typedef struct MuseGather {
  void* y[MUSE_MAX_PEERS];
  void* ctl[MUSE_MAX_PEERS];
  int32_t world, rank;
  int64_t ldy, col0;
} MuseGather;

/* Bytes of one rank's control block (epoch, ticket, arrive and done flags). */
int muse_peer_ctl_bytes(int64_t* bytes);

/* CUDA IPC handle (MUSE_IPC_HANDLE_BYTES) of the allocation holding device pointer `ptr`, and
 * ptr's byte offset inside it, for another process on the same node to open. */
int muse_ipc_export(const void* ptr, void* handle, int64_t* offset);

/* Opens a peer's exported allocation in this process (peer access enabled lazily) and returns
 * the device pointer at `offset` inside it. Close with muse_ipc_close before the peer frees it. */
int muse_ipc_open(const void* handle, int64_t offset, void** ptr);
int muse_ipc_close(void* ptr, int64_t offset);

/*
 * The column-parallel projection with its all-gather fused into the epilogue: this rank computes
 * y[:, col0 .. col0 + N) = x . W_shard^T from its packed W shard (muse_pack_tiles) and stores
 * each finished value into every rank's y_full over NVLink (plain stores to peer memory; no
 * separate all-gather). A flag barrier in the control blocks orders calls: no rank writes a
 * peer's buffer before that peer has entered the same call (its earlier work on the stream,
 * such as reads of the previous output, is done), and the launch completes only once every
 * rank's slice is in this rank's y_full. Every wait is bounded (1 s); a rank that never joins
 * makes the others' kernels record MUSE_ERR_TIMEOUT (muse_device_error) instead of hanging.
 * All ranks must make the same sequence of calls. After a call that ended with a peer timeout
 * (device code 0x401 or 0x402), re-zero every rank's control block before the next call: a rank
 * whose arrival wait timed out writes only its own copy and publishes no done flag, so a late peer
 * also ends with an error rather than with a y_full missing that rank's columns. plan->kernel: MUSE_KERNEL_TC_TILE (decode,
 * small M; a K split only with MUSE_FLAG_GLOBAL_SPLIT, scratch as muse_scratch_bytes) or
 * MUSE_KERNEL_TC_GEMM2 (prefill). ldy, col0, N multiples of 8; y_full 16-byte aligned.
 * Replaces the reference's sharded serving pattern in which the unpooler slice and the MLP-up
 * shards are followed by a separate all-gather (baseline.py:1-11; SGLang's column-parallel
 * layers); the reference itself runs no collective.
 */
int muse_proj_bf16_tiles_gather(const void* x, const void* tiles, int64_t m, int64_t n, int64_t k,
                                const MuseGather* g, const MusePlan* plan, void* scratch, int64_t scratch_bytes,
                                void* stream);

/* Size of the library's built-in scratch area used by muse_proj_bf16_tiles_noalloc. */
#define MUSE_NOALLOC_SCRATCH_BYTES (8 * 1024 * 1024)

/*
 * No counterpart in the reference: an addition for callers that cannot allocate device memory,
 * such as an inference engine's plugin that is handed only its input and output buffers from the
 * engine's own pool, or an application whose device memory is budgeted once at start-up.
 *
 * Same result as muse_proj_bf16_tiles with a MUSE_KERNEL_TC_STREAMK plan, but the split-K scratch
 * is a fixed area of MUSE_NOALLOC_SCRATCH_BYTES inside the library (a device variable held by
 * every GPU that loads the library until the process exits) instead of a caller buffer; the call
 * itself allocates nothing. Shapes whose scratch need (muse_scratch_bytes) exceeds that size are
 * rejected with MUSE_ERR_CAPACITY. The first call on each device looks up the area's address
 * (once per device, with that device current); make that first call before any stream capture.
 * Every call shares the one area and clears the split-K counters it uses on `stream` before its
 * launch, so calls whose execution overlaps on the GPU (other streams, other threads) race and
 * must be serialized by the caller. That clearing is a memset node between launches, so with a
 * MUSE_FLAG_PDL plan this entry does not overlap its launch with the previous kernel's tail as
 * muse_proj_bf16_tiles does. The area's device address is looked up once per device and kept for
 * the process: after cudaDeviceReset (which unloads the library's device code) the kept address is
 * stale, so do not call this entry again in that process after a reset.
 */
int muse_proj_bf16_tiles_noalloc(const void* x, const void* tiles, void* y, int64_t m, int64_t n, int64_t k,
                                 const MusePlan* plan, void* stream);

/*
 * y = x . decode12(W)^T from the 12-bit planes. Replaces nf12_cuda_gemv / nf12_gemv
 * (submission.py:660-673, 357-474). plan->kernel must be MUSE_KERNEL_GEMV_12B; M <= 8.
 */
int muse_proj_12b(const MuseEnc12* enc, const void* x, void* y, int64_t m, const MusePlan* plan, void* stream);

/* Device bytes of the 12-bit tile copy muse_pack_tiles12 writes: ceil(N / 128) * (K / 64) * 12416. */
int muse_tiles12_bytes(int64_t n, int64_t k, int64_t* bytes);

/*
 * Re-lays enc's 12-bit weights (device) into blocks of 128 rows x 64 k, 12416 bytes each,
 * ordered [row tile][k block]; rows past N are zero (two device kernels on `stream`):
 *   bytes 0 .. 12287: six 2048-byte slabs of 128 16-byte chunks (row r at r * 16). Slab j < 4
 *     holds the low bytes of weights 16j .. 16j + 15; slab 4 + j the code bytes of weights
 *     32j .. 32j + 31 (byte i = codes of weights 2i and 2i + 1, low nibble first);
 *   bytes 12288 .. 12415: u32 word 0 = the tile's window base << 16 | the block's escape count;
 *     words 1 .. 31 = its first 31 escapes as r << 22 | (k - 64 * block) << 16 | BF16 bits,
 *     sorted by row then k (a block with more is served from enc's per-row list).
 * No counterpart in the reference (its nf12 planes are read row-major by CUDA cores,
 * submission.py:268-271).
 */
int muse_pack_tiles12(const MuseEnc12* enc, void* tiles12, void* stream);

/*
 * y = x . decode12(W)^T on the tensor cores from the 12-bit tiles (muse_pack_tiles12) and enc's
 * per-row escape list (enc->planes and enc->bases are not read). Every BF16 weight reaching the
 * UMMA equals the original bit for bit, so the result matches a BF16 GEMM on the original W with
 * the same K split. Replaces nf12_cuda_gemv / nf12_gemv (submission.py:660-673, 357-474), which
 * serve M <= 16 on CUDA cores; any M here. plan->kernel must be MUSE_KERNEL_TC_12B. Needs
 * muse_scratch_bytes of scratch, 256-byte aligned, zeroed before its first use (every launch
 * leaves it zeroed again).
 */
int muse_proj_12b_tiles(const MuseEnc12* enc, const void* tiles12, const void* x, void* y, int64_t m,
                        const MusePlan* plan, void* scratch, int64_t scratch_bytes, void* stream);

/*
 * y (FP32 [M, N]) = x . W^T from packed BF16 tiles, FP32 accumulation, no rounding to BF16: the
 * partial a rank of a row-parallel (K-sharded) projection contributes before the reduce-scatter
 * that sums the ranks (muse_bf16_proj_b200/sharded.py). plan->kernel must be MUSE_KERNEL_TC_TILE;
 * scratch as in muse_proj_bf16_tiles. No counterpart in the reference (its `o` projection is this
 * GPU's K slice with BF16 output, reference.py:17; the sum over the TP group happens outside).
 */
int muse_proj_bf16_tiles_f32(const void* x, const void* tiles, float* y, int64_t m, int64_t n, int64_t k,
                             const MusePlan* plan, void* scratch, int64_t scratch_bytes, void* stream);

/* Device bytes of the router tiles muse_pack_router writes for an FP32 W [N, K]: the packed tiles
 * (muse_pack_tiles layout) of the BF16 matrix [hi | lo] of N rows and 2K columns. */
int muse_router_tiles_bytes(int64_t n, int64_t k, int64_t* bytes);

/*
 * Packs an FP32 W [N, K] (device, K % 64 == 0) as the tiles of [hi | lo]: hi = BF16(W) and
 * lo = BF16(W - hi), both rounded to nearest even. Replaces the router_hi / router_lo split of the
 * reference's prepare (submission.py:1120-1124). Device kernel on `stream`.
 */
int muse_pack_router(const float* w, void* tiles, int64_t n, int64_t k, void* stream);

/*
 * y = x . W^T for an FP32 W [N, K] (the router): x BF16 [M, K], y FP32 [M, N]. plan->kernel:
 *   MUSE_KERNEL_F32_GEMV: W read in FP32 on CUDA cores, FP32 accumulation, M <= 32 (`tiles` unused);
 *     replaces router_fp32 / _router_fp32_kernel (submission.py:1027-1042, 131-169);
 *   MUSE_KERNEL_TC_TILE: x . hi^T + x . lo^T as one K = 2K tensor-core projection over the tiles of
 *     muse_pack_router, FP32 accumulation and output (`w` unused); split-K plans take scratch as in
 *     muse_proj_bf16_tiles (muse_scratch_bytes with the same M, N, K); replaces router_hilo /
 *     _router_hilo_tma_kernel (submission.py:1053-1075, 172-207), which added its K splits into a
 *     zeroed output with atomics: here the last split sums them in rank order (deterministic).
 * K % 64 == 0; x 16-byte aligned.
 */
int muse_proj_f32(const void* x, const float* w, const void* tiles, float* y, int64_t m, int64_t n, int64_t k,
                  const MusePlan* plan, void* scratch, int64_t scratch_bytes, void* stream);

/* Host buffer sizes for muse_encode12: planes and bases bytes. */
int muse_encode12_sizes(int64_t n, int64_t k, int64_t* planes_bytes, int64_t* bases_bytes);

/*
 * Lossless 12-bit encoding of BF16 W [N, K] on the host (K % 512 == 0, K <= 65536).
 * Replaces nf12_pack_cuda (submission.py:591-626), with the window base chosen per 128 x 128
 * tile instead of once per matrix. Per tile, c0 = the first c maximising the count of weights
 * whose high byte without sign (E7) lies in [c, c + 7]. A weight inside its tile's window keeps
 * its low byte and a 4-bit code s << 3 | (E7 - c0); one outside is stored as zeros and listed as
 * an escape. Layout: each row is K / 512 units of 768 bytes (512 low bytes, then 256 code bytes,
 * byte j = code[2j] | code[2j+1] << 4); bases u8 [ceil(N/128)][K/128]; escapes a per-row CSR
 * (esc_ptr[N + 1]) of u32 entries k << 16 | true BF16 bits. Writes the escape count to *n_esc;
 * returns MUSE_ERR_CAPACITY (with *n_esc set) when esc_cap is too small. threads <= 0: all cores.
 */
int muse_encode12(const uint16_t* w, int64_t n, int64_t k, uint8_t* planes, uint8_t* bases, int32_t* esc_ptr,
                  uint32_t* esc_val, int64_t esc_cap, int64_t* n_esc, int threads);

/*
 * The same encoding on the device, step 1 of 2: from BF16 W [N, K] in device memory, writes the
 * planes, the bases and esc_ptr (N + 1 int32: the per-row CSR offsets, esc_ptr[N] = the escape
 * count) in exactly muse_encode12's format, into device buffers of muse_encode12_sizes' sizes.
 * The caller reads esc_ptr[N], sizes esc_val and runs step 2. Replaces nf12_pack_cuda
 * (submission.py:591-626), which encoded with torch ops on the GPU. K % 512 == 0, K <= 65536,
 * N * K < 2^31; W 16-byte and planes 8-byte aligned. Launches on `stream`; no allocation.
 */
int muse_encode12_device(const void* w, int64_t n, int64_t k, uint8_t* planes, uint8_t* bases, int32_t* esc_ptr,
                         void* stream);

/*
 * Step 2: the escape entries (u32 k << 16 | bits, row-major, k ascending) into esc_val, from
 * step 1's bases and esc_ptr. An entry that would fall outside esc_val[0, esc_cap) or outside
 * its row's range is skipped and recorded in the device error word (muse_device_error: 0x501).
 */
int muse_encode12_device_escapes(const void* w, int64_t n, int64_t k, const uint8_t* bases, const int32_t* esc_ptr,
                                 uint32_t* esc_val, int64_t esc_cap, void* stream);

/*
 * Host decode of the 12-bit format back to BF16 bits [N, K] (the round-trip check the reference
 * runs as an assert in nf12_pack_cuda, submission.py:611-617).
 */
int muse_decode12(const uint8_t* planes, const uint8_t* bases, const int32_t* esc_ptr, const uint32_t* esc_val,
                  int64_t n, int64_t k, uint16_t* w_out, int threads);

#ifdef __cplusplus
}
#endif

#endif /* MUSE_PROJ_H */
