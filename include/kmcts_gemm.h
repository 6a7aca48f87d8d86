/*
 * kmcts_gemm.h — C ABI of libkmcts_gemm_sm100.so, the B200 (sm_100a) BF16 GEMM
 * behind the kernel_mcts evaluation contract.
 *
 * Tensors (all device pointers, caller-owned, BF16 = 16-bit bfloat16 bits):
 *   A: [M, K] row-major.
 *   B: [K, N] column-major (element (k, j) at B[j*K + k]) when
 *      b_layout == KMCTS_B_COL — the reference contract,
 *      src/kernel_mcts/benchmarks/bf16_gemm.py:24-28 — or row-major
 *      (B[k*N + j]) when b_layout == KMCTS_B_ROW.
 *   C: [M, N] row-major.
 * Arithmetic: C = A·B with FP32 accumulation, one round-to-nearest-even to BF16.
 *
 * No function here allocates device memory per call except where stated.
 */
#ifndef KMCTS_GEMM_H
#define KMCTS_GEMM_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* Return codes.  0..3 keep the meaning of the reference's cuBLAS reference
 * entry point (src/kernel_mcts/benchmarks/kernels/bf16_reference.cu:5-41):
 * 0 ok, 1 handle/setup failure, 2 GEMM launch failure, 3 synchronize failure. */
#define KMCTS_OK 0
#define KMCTS_EHANDLE 1
#define KMCTS_EGEMM 2
#define KMCTS_ESYNC 3
#define KMCTS_EINVAL 4   /* bad pointer, shape, layout or config */
#define KMCTS_ESMEM 5    /* config needs more shared memory than a CTA has */
#define KMCTS_ETIMEOUT 6 /* a device-side bounded wait gave up (see device_status) */
#define KMCTS_ENOTSUP 7  /* the requested kernel cannot run this shape */
#define KMCTS_ENOSCRATCH 8 /* the call needs more scratch than the static array holds */

#define KMCTS_B_COL 0 /* B column-major [K,N] == [N,K] row-major (K-major) */
#define KMCTS_B_ROW 1 /* B row-major [K,N] (N-major) */

#define KMCTS_KERNEL_AUTO 0    /* tcgen05 when the shape allows it, else SIMT */
#define KMCTS_KERNEL_TCGEN05 1 /* tcgen05/TMA/TMEM kernel only (ENOTSUP otherwise) */
#define KMCTS_KERNEL_SIMT 2    /* CUDA-core kernel, any shape */

/* Schedule flags.  A persistent CTA-pair launch of T = qW + R tiles (W =
 * co-resident pairs, 0 < R < W) would leave W - R pairs idle for its whole
 * last round.  By default, when 2R <= W and tile_n is 256, the last R tiles
 * run as 2R half-width units, bit-identical to whole tiles.
 * KMCTS_FLAG_TAIL_STREAM_K instead cuts the K blocks of the last W + R tiles
 * (q >= 1) into W equal contiguous ranges, one per pair (stream-K): a tile
 * cut by a range boundary runs as a K prefix and a K suffix on two pairs,
 * whose FP32 partials meet in a per-stream library workspace before the
 * single BF16 rounding.  Its results are deterministic, bit-exact on integer
 * inputs and within the parity bound otherwise, but an output of a cut tile
 * is the sum of two K-ordered chains; a stream-K launch on a stream that is
 * being captured into a CUDA graph before that stream's workspace exists
 * falls back to the N split.  KMCTS_FLAG_NO_TAIL_SPLIT keeps every tile
 * whole.  The fused all-gather always uses the N split. */
#define KMCTS_FLAG_NO_TAIL_SPLIT 1
#define KMCTS_FLAG_TAIL_SPLIT_N 2  /* the default; kept for explicit requests */
#define KMCTS_FLAG_TAIL_STREAM_K 4
/* CTA pairs, tile_n 256, 2R <= W: each of the last R tiles runs as its two K
 * halves on two pairs.  When both halves are done each pair sends the other
 * its FP32 values of the other's 128 columns (through the per-stream
 * workspace) and writes its own 128 columns of C: each output is the FP32 sum
 * of the two K halves, rounded once (the same bits whichever pair adds).
 * Deterministic; exact on integer inputs, within the parity bound otherwise.
 * Without a workspace (growth under graph capture) the N split runs. */
#define KMCTS_FLAG_TAIL_SPLIT_K 32
/* One-CTA schedules (tile_m 128, 64 or 32) and CTA pairs: B's loads carry an
 * L2 evict-first policy.  For shapes whose M fits one or two tile rows B is
 * read once or twice, and streaming it through L2 at normal priority would
 * push out everything else there (dirty lines cost a DRAM write-back on
 * eviction).
 * Results are unchanged; only the cache policy differs.  The fused
 * all-gather ignores it. */
#define KMCTS_FLAG_B_EVICT_FIRST 8
/* The same policy on A's loads, for shapes whose N fits one or two tile
 * columns (A read once or twice).  Results are unchanged. */
#define KMCTS_FLAG_A_EVICT_FIRST 128
/* tile_m 32 (M <= 32), tile_n 128, tile_k 64 with 10 stages or 128 with 5:
 * the operands swap roles, C^T = B^T * A^T, so B's 128-column tiles are the
 * MMA's 128 rows and A's M rows its N (16 or 32): no tensor work is padding.
 * Each tile runs as S units, S = min(8, SMs / tiles, K blocks / 4); unit s
 * takes K blocks s, s + S, s + 2S, ..., so a tile's units move down B's rows
 * together.  The unit that finishes a tile last adds the FP32 partials, kept
 * in a per-stream library workspace, in unit order (deterministic; exact on
 * integer inputs, within the parity bound otherwise).  B's loads are
 * evict-first; k_splits is ignored.  Without a workspace (growth under graph
 * capture) each CTA takes one whole tile. */
#define KMCTS_FLAG_SWAP_AB 16
/* One-CTA schedules with k_splits 2..8: the K splits of each tile run as one
 * thread-block cluster (one CTA per split).  The other splits store their
 * FP32 values into split 0's shared memory, which adds them in split order
 * and writes C: no partial goes through the workspace, and the sum order,
 * hence every output bit, is the workspace path's.  The values take
 * (k_splits - 1) x rows x tile_n x 4 bytes (rows = tile_m for tile_m 32 or
 * 64, else 128): split 0 receives them in extra shared memory when that stays within
 * 227 KB, else in its pipeline stages once its own MMAs are done (when they
 * are large enough).  Every unit runs in its own CTA (units no more than the
 * SMs when persistent); otherwise the workspace path runs. */
#define KMCTS_FLAG_SPLIT_CLUSTER 64
/* With KMCTS_FLAG_SPLIT_CLUSTER: the additions spread over the cluster
 * instead of meeting in split 0.  The tile's pieces of 32 rows x 64 columns
 * (rows = tile_m for tile_m 32 or 64, else 128) are numbered quarter *
 * (tile_n / 64) + chunk, and piece p belongs to split p % k_splits (splits
 * past the pieces own none): every split copies the FP32 values of the
 * pieces it does not own into their owners' shared memory (bulk
 * shared-memory copies, no multicast), then adds its own pieces in split
 * order (the same bits as the workspace path) and writes them.  A split
 * receives at most ceil(pieces / k_splits) x (k_splits - 1) x 8 KB: in extra
 * shared memory when that stays within 227 KB, else in its pipeline stages
 * once every split's MMAs are done (the stages also hold its outgoing
 * pieces).  Where neither fits, the splits add up in split 0 as without
 * this flag, or through the workspace. */
#define KMCTS_FLAG_SPLIT_SCATTER 256

#define KMCTS_TAIL_NONE 0     /* kmcts_gemm_plan.tail_split: every tile whole */
#define KMCTS_TAIL_SPLIT_N 1  /* last wave as half-width units */
#define KMCTS_TAIL_STREAM_K 2 /* last W + R tiles as stream-K ranges */
#define KMCTS_TAIL_SPLIT_K 3  /* last R tiles as two K halves exchanging FP32 halves */

/* Kernel schedule.  Zero-initialise and call kmcts_default_config() first. */
typedef struct kmcts_gemm_config {
    int32_t tile_m;       /* 128: one CTA per tile; 256: one CTA pair per tile;
                             32 or 64: one CTA per tile staging 32 or 64 rows of A
                             (M <= 32 or M <= 64) */
    int32_t tile_n;       /* tile columns: 64, 128, 192, 256 (one CTA); 128, 256 (pair) */
    int32_t tile_k;       /* K per pipeline stage: 64 or 128 */
    int32_t stages;       /* shared-memory pipeline depth: 2..6 (9 for some tile_m 32 schedules) */
    int32_t cluster_m;    /* 1 with tile_m 128, 64 or 32; 2 with tile_m 256 (tcgen05 cta_group::2) */
    int32_t cluster_n;    /* 1; or 2 with tile_m 256, tile_n 256, tile_k 128, 3 stages: two CTA
                             pairs per 4-CTA cluster share A over distributed shared memory
                             (no TMA multicast); bit-identical to cluster_n 1, and slower */
    int32_t persistent;   /* 1: one CTA per SM loops over tiles; 0: one CTA per tile */
    int32_t raster_group; /* M-tiles per raster group (L2 locality), >= 1 */
    int32_t kernel;       /* KMCTS_KERNEL_* */
    int32_t flags;        /* KMCTS_FLAG_* bits */
    int64_t wait_limit_ns; /* bound on each device-side wait; 0 = 2 s default */
    int32_t k_splits;     /* one-CTA schedules and CTA pairs (cluster 2x1): K ranges per tile
                             (0 or 1 = none); see below */
    int32_t reserved;     /* zero */
} kmcts_gemm_config;

/* Split K (tile_m 128, 64 or 32, and tile_m 256 pairs in clusters of two; it takes
 * precedence over the pairs' tail splits).  With k_splits = S > 1 each output tile runs as S
 * units over consecutive K ranges, so a shape with few tiles (skinny M or N)
 * still streams its operands through every SM.  Each unit stores its FP32
 * partial in a per-stream library workspace and counts itself on the tile's
 * epoch-tagged counter; the unit that arrives last adds the S partials in
 * split order (deterministic) and writes the BF16 tile.  Nothing waits: the
 * last arrival only reads partials already published.  S is capped at the
 * number of K blocks; launches on a stream under CUDA-graph capture before its
 * workspace is large enough run unsplit.  Workspaces are never freed, so a
 * graph that captured one stays valid; graphs captured on one stream share
 * that stream's workspace and must not replay concurrently.  Every direct
 * launch tags the counters with a new epoch, but a graph replays the epoch it
 * captured: after a replay that reported KMCTS_ETIMEOUT, capture the graph
 * again before replaying it (the failed launch may have left arrivals counted
 * under that epoch). */

/* Fills *cfg with the tuned default schedule for B200 (the CTA-pair 256 x 256
 * x 128, 3-stage schedule that is fastest at 4096^3). Returns KMCTS_OK. */
int kmcts_default_config(kmcts_gemm_config* cfg);

/* Fills *cfg with the schedule a NULL cfg selects for this shape: for M <= 32
 * or M <= 64, one CTA per tile staging 32 or 64 rows of A (tile_m 32 or 64),
 * 128 columns wide, and from K = 4096 its K splits as one cluster per tile
 * (KMCTS_FLAG_SPLIT_CLUSTER; KMCTS_FLAG_SPLIT_SCATTER except for two splits
 * of tile_m 32), as many as keep every cluster resident (at most 8); else the default when its
 * 256 x 256 pair tiles fill the co-resident CTA pairs (with 64-deep stages when
 * K <= 768), or in two (three) K splits when those fill three quarters of them
 * and K >= 8192 (two splits with more than two tile columns as one CTA per
 * 128 x 256 tile, scatter); else one CTA per
 * 128 x 256 tile while those fill them (the default again from K = 4096),
 * else one CTA per 128 x 128 tile.  Few tiles over a long K get split K: for
 * M > 64 as scatter clusters (KMCTS_FLAG_SPLIT_SCATTER) of as many splits as
 * keep every cluster resident (at most 8; two only from K = 4096), unless
 * the workspace path would take more than 8; one-CTA
 * schedules for M <= 128 and pair schedules for M <= 512 (one or two tile
 * rows) add KMCTS_FLAG_B_EVICT_FIRST, schedules whose tiles span N in one or
 * two columns KMCTS_FLAG_A_EVICT_FIRST; N <= 128 takes one CTA per tile.  Every
 * schedule gives results within the parity criterion and bit-exact ones on
 * integer inputs.  Returns KMCTS_OK or KMCTS_EINVAL. */
int kmcts_select_config(int M, int N, int K, int b_layout, kmcts_gemm_config* cfg);

/* Drop-in for the reference's ctypes entry point kernel_mcts_bf16_reference
 * (src/kernel_mcts/benchmarks/kernels/bf16_reference.cu:5-41, loaded as in
 * src/kernel_mcts/cute_baseline.py:595-616): same arguments, column-major B,
 * default stream, synchronises, same return codes (plus KMCTS_EINVAL,
 * KMCTS_ETIMEOUT). */
int kmcts_bf16_gemm(const void* A, const void* B, void* C, int M, int N, int K);

/* Asynchronous GEMM on `stream` (a cudaStream_t; NULL = default stream).
 * cfg may be NULL (the schedule kmcts_select_config picks for the shape).  device_status, if not NULL, is a device
 * int that the kernel sets non-zero when a bounded wait gives up; the caller
 * zeroes it and reads it after synchronising.  Replaces the fixed 16x16
 * launch_candidate of src/kernel_mcts/benchmarks/kernels/bf16_gemm_harness.cu:61-72
 * with a launcher that owns grid, cluster and shared-memory attributes. */
int kmcts_bf16_gemm_ex(const void* A, const void* B, void* C, int M, int N, int K, int b_layout,
                       const kmcts_gemm_config* cfg, void* stream, int* device_status);

/* Static legality of a schedule for a shape (no GPU work).  Returns KMCTS_OK,
 * KMCTS_EINVAL, KMCTS_ESMEM or KMCTS_ENOTSUP, with a reason in why[0..len).
 * Used to mark sweep points STATICALLY_REJECTED without charging a trial, as
 * validate_cute_schedule does (src/kernel_mcts/cute_schedule.py:41-78). */
int kmcts_config_legal(const kmcts_gemm_config* cfg, int M, int N, int K, int b_layout, char* why,
                       int len);

/* Shared-memory bytes a schedule needs per CTA (0 if the schedule is invalid). */
int64_t kmcts_config_smem_bytes(const kmcts_gemm_config* cfg, int b_layout);

/* How a schedule would launch on the current device. */
typedef struct kmcts_gemm_plan {
    int32_t kernel;       /* 1: one CTA per tile; 2: CTA pair; 3: SIMT */
    int32_t ctas;         /* grid size in CTAs */
    int32_t cluster_size; /* CTAs per cluster */
    int32_t workers;      /* clusters that can be resident at once */
    int32_t tiles;        /* output tiles */
    int32_t full_tiles;   /* tiles run whole; the rest (the last wave) split */
    int32_t units;        /* work units the grid walks */
    int32_t smem_bytes;   /* dynamic shared memory per CTA */
    int32_t tail_split;   /* KMCTS_TAIL_*: how the tiles after full_tiles split */
    int32_t tail_clusters; /* pairs that share the tiles after full_tiles */
    int32_t tail_segments; /* most units one tile runs as (2 when split) */
    int32_t k_splits;     /* split K: K ranges per tile (1 = none) */
    int32_t split_reduce; /* KMCTS_SPLIT_*: where a split tile's K ranges add up */
} kmcts_gemm_plan;

#define KMCTS_SPLIT_WORKSPACE 0 /* per-stream workspace, last unit adds (or no split) */
#define KMCTS_SPLIT_CLUSTER 1   /* one cluster per tile, split 0 adds */
#define KMCTS_SPLIT_SCATTER 2   /* one cluster per tile, each split adds its pieces */

/* Fills *out with the launch shape kmcts_bf16_gemm_ex would use for this
 * schedule and shape on the current device (queries occupancy; launches
 * nothing).  Returns KMCTS_OK or the error kmcts_bf16_gemm_ex would return. */
int kmcts_gemm_plan_query(const kmcts_gemm_config* cfg, int M, int N, int K, int b_layout, kmcts_gemm_plan* out);

/* ------------------------------------------------- N-sharded GEMM (multi-GPU)
 * No counterpart in the reference (it has no multi-GPU code).  G ranks, one
 * per GPU, each hold A [M,K] and their shard of B's columns; the fused call
 * computes this rank's C columns [rank*N/G, (rank+1)*N/G) and stores every
 * finished tile into all G ranks' full C [M, N] (row-major) — the GEMM and the
 * all-gather of C in one kernel, over NVLink peer memory. */
#define KMCTS_IPC_HANDLE_BYTES 72 /* cudaIpcMemHandle_t + 8-byte offset in the allocation */
#define KMCTS_MAX_RANKS 8

/* Writes a CUDA IPC handle for a device allocation (cudaIpcGetMemHandle). */
int kmcts_ipc_export(const void* device_ptr, uint8_t* handle_out);
/* Maps a peer's exported allocation into this process (cudaIpcOpenMemHandle). */
int kmcts_ipc_import(const uint8_t* handle, void** device_ptr_out);
/* Unmaps an imported allocation. */
int kmcts_ipc_close(void* device_ptr);

/* No counterpart in the reference.  Copies `height` rows of `width_bytes`
 * bytes between device buffers (row pitches in bytes) on `stream`, with
 * cudaMemcpy2DAsync: into an IPC-imported peer buffer the GPU's copy engines
 * move the rows over NVLink while the SMs keep computing.  The copy-engine
 * all-gather of the N-sharded GEMM uses it to send finished row blocks of a
 * rank's C columns to every peer's C.  Asynchronous; KMCTS_ESYNC if the copy
 * cannot be queued. */
int kmcts_copy_2d(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t width_bytes,
                  size_t height, void* stream);

/* C_ranks[r] is rank r's full C (this rank's own buffer at index `rank`,
 * IPC-imported peer buffers elsewhere).  B_shard is this rank's columns:
 * [N/G, K] row-major for KMCTS_B_COL, [K, N/G] row-major for KMCTS_B_ROW.
 * N_total/num_ranks must be a multiple of 256 and num_ranks <= 8.  The
 * schedule must be a CTA pair (tile_m 256).  Asynchronous on `stream`; the
 * caller synchronises its stream and then all ranks (a host barrier) before
 * anyone reads C. */
int kmcts_bf16_gemm_allgather(const void* A, const void* B_shard, void* const* C_ranks, int num_ranks, int rank,
                              int M, int N_total, int K, int b_layout, const kmcts_gemm_config* cfg, void* stream,
                              int* device_status);

/* Evaluation inputs (host memory, BF16 bits).  A (a_count values) then B
 * (b_count values) from one generator:
 *   KMCTS_INPUTS_UNIFORM  the repository contract's stream, std::mt19937(seed)
 *                         with std::uniform_real_distribution<float>(-0.25, 0.25),
 *                         as in src/kernel_mcts/benchmarks/kernels/bf16_gemm_harness.cu:92-95;
 *   KMCTS_INPUTS_RANDN    std::mt19937_64(seed), N(0, 1);
 *   KMCTS_INPUTS_INT      std::mt19937(seed), integers uniform in {-2..2}.
 * Every value is rounded to BF16 with round-to-nearest-even. */
#define KMCTS_INPUTS_UNIFORM 0
#define KMCTS_INPUTS_RANDN 1
#define KMCTS_INPUTS_INT 2
int kmcts_generate_inputs(int kind, uint32_t seed, size_t a_count, size_t b_count, uint16_t* a_out,
                          uint16_t* b_out);

/* Library version string. */
const char* kmcts_version(void);

/* Result of the device-side comparison of an output against a reference. */
typedef struct kmcts_compare_result {
    double maximum_error;  /* max |c - ref| over finite pairs (NaN/inf counted below) */
    double mean_error;     /* sum |c - ref| / count */
    int64_t count;
    int64_t n_tolerance_fail; /* elements failing |c-ref| <= atol + rtol*|ref| or non-finite */
    int64_t n_nonfinite;      /* non-finite elements of c */
    int64_t ulp_hist[4];      /* elements at 0, 1, 2 and >2 BF16 ulps from ref */
    int32_t max_ulp;          /* largest ulp distance (65535 for NaN) */
    int32_t success;          /* n_tolerance_fail == 0 */
} kmcts_compare_result;

/* Bytes of device workspace kmcts_bf16_compare needs. */
size_t kmcts_compare_workspace_bytes(void);

/* Device-side restatement of the reference harness's host error scan
 * (src/kernel_mcts/benchmarks/kernels/bf16_gemm_harness.cu:154-164) with added
 * ulp statistics.  `workspace` is caller-owned device memory of
 * kmcts_compare_workspace_bytes() bytes.  Runs on `stream`, synchronises it,
 * and writes *out on the host. */
int kmcts_bf16_compare(const void* C, const void* reference, int64_t count, double rtol,
                       double atol, void* workspace, void* stream, kmcts_compare_result* out);

/* No counterpart in the reference.  kmcts_bf16_compare without a workspace
 * argument, for callers that cannot allocate device memory when they check a
 * result: a worker whose device memory is all owned by another allocator (a
 * framework's caching allocator that must account for every byte, so a
 * cudaMalloc behind its back could push it out of memory), or a host
 * application that embeds this library and hands it only the tensors it
 * passes in, with no allocation rights of its own.  The scratch is
 * a file-scope device array of KMCTS_NOALLOC_SCRATCH_BYTES (256 bytes) that
 * every GPU loading this library keeps until the process exits; the
 * comparison needs that much for any `count`, and a call needing more would
 * return KMCTS_ENOSCRATCH.  The first call on each device looks up the
 * array's device address (cudaGetSymbolAddress; again after the device's
 * context is recreated, e.g. by cudaDeviceReset), so make that first call
 * before any stream capture.  Each call zeroes the accumulators it uses, but
 * all calls share the one array: calls that overlap on the GPU (different
 * streams or threads) race and corrupt each other's results.  Allocates no
 * device memory; synchronises `stream`; writes *out on the host. */
#define KMCTS_NOALLOC_SCRATCH_BYTES 256
int kmcts_bf16_compare_noalloc(const void* C, const void* reference, int64_t count, double rtol,
                               double atol, void* stream, kmcts_compare_result* out);

/* No counterpart in the reference.  Self-test of the bounded device-side wait
 * behind every GEMM barrier: one thread waits on an mbarrier; with arrive = 1
 * the phase is already complete, with arrive = 0 nothing ever arrives and the
 * wait must give up after limit_ns (0 < limit_ns <= 10 s), setting
 * *device_status to KMCTS_ETIMEOUT | role << 8.  *device_waited_ns receives the
 * time spent waiting.  Asynchronous on `stream`; touches no TMA or TMEM. */
int kmcts_selftest_bounded_wait(int64_t limit_ns, int arrive, void* stream, int* device_status,
                                unsigned long long* device_waited_ns);

/* Number of kernels this library has launched in this process (all entry
 * points).  Lets callers count GPU launches inside a timed region. */
int64_t kmcts_launch_count(void);

/* C = A·B with A, B and C in host memory (page-locked, or the copies do not
 * overlap), through device scratch buffers the caller owns, as large as A
 * [M,K], B (K x N) and C [M,N]; their contents afterwards are unspecified
 * (B and C blocks are kept as dense sub-matrices).  No counterpart in the
 * reference, whose harness copies inputs and results around the timed
 * region.  A goes over in `chunks` row blocks (<= 0: 4; whole 128-row tiles)
 * and B in `chunks` column blocks (whole 256-column tiles; one block when
 * N < 512), alternating; each C block is computed once its A and B blocks
 * have landed and goes back at once, so both copy directions and the GEMMs
 * overlap.  Every block runs one schedule: cfg, or for a NULL cfg the one
 * kmcts_select_config picks for the whole problem, so C is bit-identical to
 * kmcts_bf16_gemm_ex on the whole problem with that schedule (except with
 * KMCTS_FLAG_TAIL_STREAM_K, whose splits depend on the shape).  Internal
 * copy streams wait for the work already on `stream`, and `stream` waits for
 * the last copy back: asynchronous on `stream`, complete when it is. */
int kmcts_bf16_gemm_host(const void* A_host, const void* B_host, void* C_host, void* A_dev, void* B_dev,
                         void* C_dev, int M, int N, int K, int b_layout, const kmcts_gemm_config* cfg,
                         int chunks, void* stream, int* device_status);

/* Times kmcts_bf16_gemm_ex with the reference harness's benchmark protocol
 * (src/kernel_mcts/benchmarks/kernels/bf16_gemm_harness.cu:177-215):
 * `warmups` launches, one synchronise, then `measurements` x (event record,
 * launch, event record, event synchronise), writing each launch's time in
 * microseconds to timings_us[0..measurements).  If flush is not NULL,
 * flush_bytes of it are overwritten before every timed launch, outside the
 * events (an L2 flush).  Synchronous.  Returns KMCTS_OK, the launch's error,
 * KMCTS_ESYNC, or KMCTS_ETIMEOUT when device_status (required) reports a
 * bounded wait that gave up. */
int kmcts_time_gemm(const void* A, const void* B, void* C, int M, int N, int K, int b_layout,
                    const kmcts_gemm_config* cfg, void* stream, int* device_status, int warmups,
                    int measurements, void* flush, size_t flush_bytes, float* timings_us);

#ifdef __cplusplus
}
#endif

#endif /* KMCTS_GEMM_H */
