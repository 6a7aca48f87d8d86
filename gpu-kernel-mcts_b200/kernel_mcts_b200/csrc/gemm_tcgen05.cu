// Persistent, warp-specialised BF16 GEMM for sm_100a.
//
//   C[M,N] (bf16, row-major) = A[M,K] (bf16, row-major) · B  (FP32 accumulate)
//
// This is the B200 replacement for the candidate kernel the reference harness
// launches (src/kernel_mcts/benchmarks/kernels/bf16_gemm_harness.cu:61-72,
// root program bf16_gemm_root.cu:8-44): same arithmetic contract, new engine.
//
// Per CTA (one per SM when persistent), 192 threads in three roles:
//   warp 0      TMA producer: one lane streams A/B K-slices into a ring of
//               `STAGES` 128-byte-swizzled shared-memory stages (full/empty
//               mbarriers, transaction-byte completion).
//   warp 1      MMA issuer: owns the TMEM allocation; one lane issues
//               tcgen05.mma (M=128, N=BN, K=16) into one of two TMEM
//               accumulators and commits stage releases / accumulator-ready.
//   warps 2-5   epilogue: tcgen05.ld each 32-lane quarter of the accumulator,
//               round to BF16 (RNE), stage through swizzled shared memory and
//               TMA-store.  Two TMEM accumulators let the epilogue of tile i
//               overlap the main loop of tile i+1.
// Skinny shapes stage only 32 or 64 rows of A (AR), leaving shared memory for
// more of B.  Split K runs each tile as k_splits K ranges whose FP32 values
// meet either in a per-stream workspace (the last unit to arrive adds them)
// or, as one thread-block cluster per tile, in split 0's shared memory.
// Operands read once can stream through L2 at evict-first priority.
// Every wait is bounded (limit_ns); on timeout the kernel records
// KMCTS_ETIMEOUT in *status, drains its own copies and MMAs, frees TMEM and
// returns.  No TMA multicast is used.
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>
#include <tuple>

#include "gemm_common.cuh"
#include "kmcts_internal.h"

namespace kmcts {

__device__ int g_default_status;

int* default_status_ptr() {
    // Device code of other translation units cannot name this symbol (the
    // library is built without relocatable device code), so launches there
    // get its address from here; one address per device.
    static std::mutex mu;
    static int* cached[64] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) return nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (!cached[device]) {
        void* p = nullptr;
        if (cudaGetSymbolAddress(&p, g_default_status) != cudaSuccess) return nullptr;
        cached[device] = static_cast<int*>(p);
    }
    return cached[device];
}

namespace {

using namespace gemm;

constexpr int kBM = 128;
constexpr int kMaxDevices = 64;
constexpr int kMaxClusterSplits = 8;  // portable cluster size

// AR: rows of A staged per tile.  128 normally; 32 or 64 for skinny GEMMs
// (M <= AR): the MMA still computes 128 rows, but rows AR-127 read whatever
// follows A's AR rows in the stage and are never stored, and the freed shared
// memory holds more B stages in flight.
template <int BN, int BK, int STAGES, bool B_MN, int AR = kBM>
struct Layout {
    static constexpr int kAHalf = AR * 128;  // one 64-wide K half of A
    static constexpr int kABytes = AR * BK * 2;
    static constexpr int kBBytes = BN * BK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStagingOffset = STAGES * kStageBytes;
    // Only the warps of TMEM lanes below AR ever store C.
    static constexpr int kStagingWarps = AR / 32;
    static constexpr int kBarrierOffset = kStagingOffset + kStagingWarps * 2 * kStagingBytes;
    static constexpr int kSmemBytes = kBarrierOffset + kSmemReserve;
    static constexpr uint32_t kTmemCols = tmem_columns_for(2 * BN);
    static_assert(BN % 64 == 0 && BN >= 64 && BN <= 256, "BN must be 64..256, step 64");
    static_assert(BK == 64 || BK == 128, "BK must be 64 or 128");
    static_assert(kSmemBytes <= kMaxSmem, "shared memory budget exceeded");
    static_assert(AR == kBM || AR == 32 || AR == 64, "A is staged as 128, 64 or 32 rows");
    // The MMA reads 128 rows (16 KB) from each A half: that must stay inside the stage.
    static_assert(AR == kBM || (BK / 64 - 1) * kAHalf + kBM * 128 <= kStageBytes, "A over-read leaves the stage");
};

// Split K: unit u is K range s = u % splits of tile u / splits.  Partials are
// [tile][split][lane quarter][BN/64 chunks] blocks of 32 rows x 64 FP32, each
// stored as 16 float4 groups interleaved across the 32 lanes (coalesced).
//
// With `cluster` set, the splits of a tile are the CTAs of one cluster
// (rank = split) and no partial goes through global memory: ranks 1.. store
// their FP32 values into rank 0's shared memory (same block layout, one slot
// per sending rank) and arrive on its receive barrier; rank 0 adds them to
// its own accumulator in split order and writes C.  The sum order is the
// global path's, so both give the same bits.  Where rank 0 receives:
//   kClusterBuffer  a buffer past its barriers (the launch adds its size);
//   kClusterStages  its pipeline stages, free once its UMMAs are done: rank 0
//                   then signals each sender's go barrier, senders wait for
//                   it before storing, and the cluster syncs before exit.
// kClusterScatter spreads the additions over the cluster: the tile's pieces
// of 32 rows x 64 columns (lane quarter q < AR / 32, chunk c) are numbered
// q * (BN / 64) + c, and piece p belongs to rank p % splits (ranks past the
// pieces own none and only send).  Each
// rank writes the FP32 values of every piece it does not own into its own
// pipeline stages (free once its UMMAs are done; piece p at p x 8 KB), then
// one lane per warp copies each of them into its owner's shared memory with
// a bulk shared::cta -> shared::cluster copy that completes its bytes on the
// owner's receive barrier (armed at set-up with the bytes the rank will
// receive).  The owner waits once, adds its pieces' values in split order
// and writes them.  The copies land
//   with kClusterBuffer  in a buffer past the barriers: free from the start,
//                        so each rank copies as soon as its pieces are written;
//   with kClusterStages  in the stages past the pieces: the cluster meets
//                        first (every rank's UMMAs are then done).
// The cluster syncs before exit, so no CTA leaves while a copy reads its
// stages or writes its shared memory.
constexpr int kClusterBuffer = 1, kClusterStages = 2, kClusterScatter = 4;

struct SplitK {
    int splits;
    float* partials;
    unsigned long long* counters;  // [tile][lane quarter]: epoch << 32 | units arrived
    int epoch;
    int cluster;  // 0 (workspace), or kClusterBuffer or kClusterStages, with kClusterScatter
};

// Pieces (32 rows x 64 columns) of a tile staging `ar` rows of A.
__host__ __device__ constexpr int scatter_pieces_of(int bn, int ar) { return (ar / 32) * (bn / 64); }

template <int BN>
__device__ __forceinline__ float4* split_chunk(const SplitK& sk, int tile, int split, int quarter, int c) {
    const size_t block = ((static_cast<size_t>(tile) * sk.splits + split) * 4 + quarter) * (BN / 64) + c;
    return reinterpret_cast<float4*>(sk.partials + block * 32 * 64);
}

// Float4 offset of (sending rank's slot, lane quarter, chunk) in rank 0's
// receive buffer.  `rows` is the rows of A staged per tile (32, 64 or 128).
template <int BN>
__device__ __forceinline__ int recv_chunk(int slot, int quarter, int c, int rows) {
    return ((slot * (rows / 32) + quarter) * (BN / 64) + c) * 16 * 32;
}

// FEAT selects what an instantiation carries: bit 0 the cache-hinted loads,
// bit 1 the cluster split K, bit 2 its scatter form.  Code a
// schedule does not use is compiled out (a runtime branch in the producer's
// loop costs the common schedules 1-2 us per launch); the launcher picks the
// smallest instantiation that serves.
constexpr int kFeatHints = 1, kFeatCluster = 2, kFeatScatter = 4;

template <int BN, int BK, int STAGES, bool B_MN, int AR, int FEAT = 0>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tcgen05(const __grid_constant__ CUtensorMap map_a,
                      const __grid_constant__ CUtensorMap map_b,
                      const __grid_constant__ CUtensorMap map_c, int M, int N, int K, int group,
                      uint64_t limit_ns, int* status, const SplitK sk, int evict_first) {
    using L = Layout<BN, BK, STAGES, B_MN, AR>;
    constexpr bool kScatter = (FEAT & kFeatScatter) != 0;
    static_assert(!kScatter || (FEAT & kFeatCluster), "the scatter split is a cluster split K");
    const int cluster_mode = (FEAT & kFeatCluster) ? sk.cluster : 0;  // compile-time 0 otherwise
    const int recv_mode = cluster_mode & (kClusterBuffer | kClusterStages);
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarrierOffset);
    uint64_t* empty = full + STAGES;
    uint64_t* tmem_full = empty + STAGES;
    uint64_t* tmem_empty = tmem_full + 2;
    uint64_t* drain = tmem_empty + 2;
    uint64_t* recv_full = drain + 1;  // cluster split K: rank 0 receives the other ranks' values
    uint64_t* go_bar = recv_full + 1;  // kClusterStages: rank 0's stages are free to receive
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(go_bar + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* no_abort = abort + 1;
    // Cluster split K's receive buffer: past the barriers (which take well
    // under 1 KB of the reserve; the launch adds its size to the shared
    // memory), or the pipeline stages.
    float4* recv = reinterpret_cast<float4*>(recv_mode == kClusterStages ? smem : smem + L::kBarrierOffset + 1024);

    if (status == nullptr) status = &g_default_status;
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int num_m = (M + kBM - 1) / kBM;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int num_kb = (K + BK - 1) / BK;
    const int splits = sk.splits;
    const int num_units = num_tiles * splits;

    // Producer state, used by thread 0 (warp 0, lane 0) only.
    int stage_p = 0;
    uint32_t phase_p = 0;
    uint32_t issued = 0, issued_phase = 0;
    // Operands read once (one tile row for B, one tile column for A): their
    // lines go first when L2 needs room.  Bit 0: B, bit 1: A.
    const bool b_evict_first = (FEAT & kFeatHints) && (evict_first & 1) != 0;
    const bool a_evict_first = (FEAT & kFeatHints) && (evict_first & 2) != 0;
    const uint64_t b_policy = b_evict_first ? ptx::policy_evict_first() : 0ull;
    const uint64_t a_policy = a_evict_first ? ptx::policy_evict_first() : 0ull;
    // Waits for the next stage to be free, then TMA-loads K block kb of the
    // tile at (m0, n0) into it.  False when the wait gave up.
    auto load_stage = [&](int kb, int m0, int n0) -> bool {
        if (!ptx::mbar_wait(&empty[stage_p], phase_p ^ 1u, limit_ns, abort)) {
            record_failure(status, abort, kRoleProducer);
            return false;
        }
        uint8_t* sa = smem + stage_p * L::kStageBytes;
        uint8_t* sb = sa + L::kABytes;
        ptx::mbar_arrive_expect_tx(&full[stage_p], L::kStageBytes);
#pragma unroll
        for (int kh = 0; kh < BK / 64; ++kh) {
            const int k0 = kb * BK + kh * 64;
            if (a_evict_first)
                ptx::tma_load_2d_hint(sa + kh * L::kAHalf, &map_a, &full[stage_p], k0, m0, a_policy);
            else
                ptx::tma_load_2d(sa + kh * L::kAHalf, &map_a, &full[stage_p], k0, m0);
            if constexpr (B_MN) {
#pragma unroll
                for (int nb = 0; nb < BN / 64; ++nb) {
                    uint8_t* dst = sb + (kh * (BN / 64) + nb) * 8192;
                    if (b_evict_first)
                        ptx::tma_load_2d_hint(dst, &map_b, &full[stage_p], n0 + nb * 64, k0, b_policy);
                    else
                        ptx::tma_load_2d(dst, &map_b, &full[stage_p], n0 + nb * 64, k0);
                }
            } else {
                if (b_evict_first)
                    ptx::tma_load_2d_hint(sb + kh * (BN * 128), &map_b, &full[stage_p], k0, n0, b_policy);
                else
                    ptx::tma_load_2d(sb + kh * (BN * 128), &map_b, &full[stage_p], k0, n0);
            }
        }
        issued |= 1u << stage_p;
        issued_phase = (issued_phase & ~(1u << stage_p)) | (phase_p << stage_p);
        if (++stage_p == STAGES) {
            stage_p = 0;
            phase_p ^= 1u;
        }
        return true;
    };

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            ptx::mbar_init(&tmem_full[a], 1);
            ptx::mbar_init(&tmem_empty[a], kEpilogueWarps);
        }
        ptx::mbar_init(drain, 1);
        // Gather: every lane of every epilogue warp of each sending rank
        // arrives once.  Scatter: one arrival (below), then the copies' bytes.
        uint32_t recv_count = 1;
        if (cluster_mode && !kScatter) recv_count = static_cast<uint32_t>((splits - 1) * kEpilogueWarps * 32);
        ptx::mbar_init(recv_full, recv_count);
        ptx::mbar_init(go_bar, 1);
        if (kScatter && cluster_mode) {
            // The bytes the other ranks copy in: 8 KB per owned piece and sender.
            // (None for ranks past the pieces: they only send.)
            const int owned =
                (scatter_pieces_of(BN, AR) - static_cast<int>(blockIdx.x % splits) + splits - 1) / splits;
            ptx::fence_mbarrier_init();
            ptx::mbar_arrive_expect_tx(recv_full, static_cast<uint32_t>(owned * (splits - 1) * 8192));
        }
        *abort = 0;
        *no_abort = 0;
        ptx::fence_mbarrier_init();
        ptx::prefetch_tensormap(&map_a);
        ptx::prefetch_tensormap(&map_b);
        ptx::prefetch_tensormap(&map_c);
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, L::kTmemCols);
        ptx::tmem_relinquish();
    }
    __syncwarp();  // every warp meets the CTA barrier converged
    // Cluster split K: every thread arrives on the cluster barrier once rank
    // 0's receive barrier is initialised; a thread waits on it before its
    // first access to another CTA (or at the end), so no CTA idles here.
    if (cluster_mode) ptx::cluster_arrive();
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            bool ok = true;
            for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x) {
                const int t = u / splits, s = u % splits;
                const TileCoord tc = tile_coord(t, num_m, num_n, group);
                const int kb1 = (s + 1) * num_kb / splits;
                for (int kb = s * num_kb / splits; kb < kb1; ++kb) {
                    if (!load_stage(kb, tc.m_blk * kBM, tc.n_blk * BN)) {
                        ok = false;
                        break;
                    }
                }
            }
            // Drain: every load this thread issued lands before the CTA exits.
            for (int s = 0; s < STAGES; ++s) {
                if (issued & (1u << s)) {
                    if (!ptx::mbar_wait(&full[s], (issued_phase >> s) & 1u, drain_limit(limit_ns), no_abort)) {
                        record_failure(status, abort, kRoleDrain);
                    }
                }
            }
        }
        __syncwarp();  // lanes 1-31 wait for the producer lane before the closing barrier
    } else if (warp == 1) {
        // ----------------------------------------------------------------- MMA
        if (lane == 0) {
            constexpr uint32_t idesc = ptx::make_idesc_bf16(kBM, BN, B_MN);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < num_units && ok; u += gridDim.x, ++local) {
                const int s = u % splits;
                const int kb0 = s * num_kb / splits, kb1 = (s + 1) * num_kb / splits;
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!ptx::mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, limit_ns, abort)) {
                    record_failure(status, abort, kRoleMma);
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = kb0; kb < kb1; ++kb) {
                    if (!ptx::mbar_wait(&full[stage], phase, limit_ns, abort)) {
                        record_failure(status, abort, kRoleMma);
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const uint32_t sa = ptx::smem_addr(smem + stage * L::kStageBytes);
                    const uint32_t sb = sa + L::kABytes;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const int kh = kk / 4;  // which 64-wide K half of the stage
                        const int kq = kk % 4;  // 16-element step inside it
                        const uint64_t adesc = ptx::make_sw128_desc(sa + kh * L::kAHalf + kq * 32, 16, 1024);
                        uint64_t bdesc;
                        if constexpr (B_MN) {
                            bdesc = ptx::make_sw128_desc(sb + kh * (BN / 64) * 8192 + kq * 2048,
                                                         8192, 1024);
                        } else {
                            bdesc = ptx::make_sw128_desc(sb + kh * (BN * 128) + kq * 32, 16, 1024);
                        }
                        ptx::umma_bf16(d_tmem, adesc, bdesc, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
                    }
                    ptx::umma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (ok) ptx::umma_commit(&tmem_full[acc]);
            }
            // Drain: all MMAs issued by this thread complete before TMEM is freed.
            ptx::umma_commit(drain);
            if (!ptx::mbar_wait(drain, 0, drain_limit(limit_ns), no_abort)) {
                record_failure(status, abort, kRoleDrain);
            }
        }
        __syncwarp();  // lanes 1-31 wait for the MMA lane before the closing barrier
    } else {
        // ------------------------------------------------------------ epilogue
        const int quarter = warp % 4;  // TMEM lanes this warp may access
        const int e = warp - 2;
        // A warp whose lanes hold rows of C has a staging pair of its own
        // (warps of lanes at or past AR never store).
        uint8_t* staging =
            smem + L::kStagingOffset + (L::kStagingWarps == kEpilogueWarps ? e : quarter) * 2 * kStagingBytes;
        int local = 0;
        int chunk_count = 0;
        // Cluster split K: rank 0's receive buffer and barrier as this CTA
        // addresses them (the same offsets in every CTA of the launch).
        const uint32_t recv_remote = cluster_mode ? ptx::mapa_shared(ptx::smem_addr(recv), 0) : 0u;
        const uint32_t recv_full_remote = cluster_mode ? ptx::mapa_shared(ptx::smem_addr(recv_full), 0) : 0u;
        // Rank 0's receive barrier is initialised (every thread of the
        // cluster arrived after set-up) before any store or arrive reaches it.
        if (cluster_mode) ptx::cluster_wait();
        bool got_recv = false;  // rank 0: the other ranks' values are all here
        bool met = false;       // scatter: this warp passed the cluster barrier between write and read
        for (int u = blockIdx.x; u < num_units; u += gridDim.x, ++local) {
            const int t = u / splits, s = u % splits;
            const TileCoord tc = tile_coord(t, num_m, num_n, group);
            const int m0 = tc.m_blk * kBM;
            const int n0 = tc.n_blk * BN;
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            const bool sender = !kScatter && cluster_mode && s != 0;
            const bool receiver = !kScatter && cluster_mode && s == 0;
            bool ok = ptx::mbar_wait(&tmem_full[acc], acc_phase, limit_ns, abort);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0) record_failure(status, abort, kRoleEpilogue);
                break;
            }
            ptx::tc_fence_after();
            if (receiver && recv_mode == kClusterStages && e == 0 && lane == 0) {
                // Every UMMA of this CTA has completed, so no stage is read
                // any more (its one unit's loads were all consumed): the
                // other ranks may store into them.
                ptx::fence_proxy_async_smem();
                for (int r = 1; r < splits; ++r)
                    ptx::mbar_arrive_release_cluster(ptx::mapa_shared(ptx::smem_addr(go_bar), static_cast<uint32_t>(r)));
            }
            const uint32_t row_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                      static_cast<uint32_t>(acc * BN);
            if constexpr (kScatter) {
                // One unit per CTA.  Write the pieces of this warp's quarter
                // that other ranks own into this CTA's stages (free: every
                // UMMA has completed and the unit's loads were all consumed),
                // copy each into its owner's receive slots (in stages mode
                // after the cluster meets, when every rank's stages are free),
                // then add the own pieces' values in split order.
                constexpr int kChunks = BN / 64;
                float4* parts = reinterpret_cast<float4*>(smem);  // piece p at p * 512 float4
                // Received copies: past the pieces in the stages, or in the
                // buffer past the barriers (free from the start: no meeting).
                const bool in_stages = recv_mode == kClusterStages;
                float4* received = in_stages ? parts + scatter_pieces_of(BN, AR) * 512 : recv;
                // Only the lane quarters below AR hold rows of the tile.
                const int quarter_chunks = quarter < AR / 32 ? kChunks : 0;
                ptx::fence_proxy_async_smem();  // generic writes after the async proxy's use
#pragma unroll 1
                for (int c = 0; c < quarter_chunks; ++c) {
                    const int piece = quarter * kChunks + c;
                    if (piece % splits == s) continue;
                    uint32_t lo[32], hi[32];
                    ptx::tmem_ld_32x32b_x32(row_addr + c * 64, lo);
                    ptx::tmem_ld_32x32b_x32(row_addr + c * 64 + 32, hi);
                    ptx::tmem_wait_ld();
                    float4* dst = parts + piece * 512;
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        dst[q * 32 + lane] = make_float4(__uint_as_float(lo[4 * q]), __uint_as_float(lo[4 * q + 1]),
                                                         __uint_as_float(lo[4 * q + 2]), __uint_as_float(lo[4 * q + 3]));
                        dst[(8 + q) * 32 + lane] =
                            make_float4(__uint_as_float(hi[4 * q]), __uint_as_float(hi[4 * q + 1]),
                                        __uint_as_float(hi[4 * q + 2]), __uint_as_float(hi[4 * q + 3]));
                    }
                }
                ptx::fence_proxy_async_smem();  // the copies (async proxy) read what this thread wrote
                if (in_stages) {
                    // Every rank's stages are free and its pieces written.
                    ptx::cluster_arrive();
                    ptx::cluster_wait();
                    met = true;
                } else {
                    __syncwarp();  // lane 0 copies what the warp wrote
                }
                if (lane == 0) {
                    for (int c = 0; c < quarter_chunks; ++c) {
                        const int piece = quarter * kChunks + c;
                        const int owner = piece % splits;
                        if (owner == s) continue;
                        const int slot = (piece / splits) * (splits - 1) + (s < owner ? s : s - 1);
                        ptx::bulk_copy_to_cluster(
                            ptx::mapa_shared(ptx::smem_addr(received + slot * 512), static_cast<uint32_t>(owner)),
                            ptx::smem_addr(parts + piece * 512), 8192u,
                            ptx::mapa_shared(ptx::smem_addr(recv_full), static_cast<uint32_t>(owner)));
                    }
                }
                bool waited = false;
#pragma unroll 1
                for (int c = 0; c < quarter_chunks; ++c) {
                    const int piece = quarter * kChunks + c;
                    if (piece % splits != s) continue;
                    if (!waited) {
                        bool got = ptx::mbar_wait_cluster(recv_full, 0, limit_ns, abort);
                        got = __all_sync(0xffffffffu, got);
                        waited = true;
                        if (!got) {
                            if (lane == 0) record_failure(status, abort, kRoleEpilogue);
                            break;
                        }
                    }
                    const float4* slots = received + (piece / splits) * (splits - 1) * 512;
                    uint32_t lo[32], hi[32];
                    // Split order, as the workspace path adds: split 0 first.
                    if (s == 0) {
                        ptx::tmem_ld_32x32b_x32(row_addr + c * 64, lo);
                        ptx::tmem_ld_32x32b_x32(row_addr + c * 64 + 32, hi);
                        ptx::tmem_wait_ld();
                    } else {
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const float4 f = slots[q * 32 + lane];
                            const float4 g = slots[(8 + q) * 32 + lane];
                            lo[4 * q] = __float_as_uint(f.x);
                            lo[4 * q + 1] = __float_as_uint(f.y);
                            lo[4 * q + 2] = __float_as_uint(f.z);
                            lo[4 * q + 3] = __float_as_uint(f.w);
                            hi[4 * q] = __float_as_uint(g.x);
                            hi[4 * q + 1] = __float_as_uint(g.y);
                            hi[4 * q + 2] = __float_as_uint(g.z);
                            hi[4 * q + 3] = __float_as_uint(g.w);
                        }
                    }
#pragma unroll 1
                    for (int j = 1; j < splits; ++j) {
                        if (j == s) {
                            uint32_t own[32];
                            ptx::tmem_ld_32x32b_x32(row_addr + c * 64, own);
                            ptx::tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                lo[i] = __float_as_uint(__uint_as_float(lo[i]) + __uint_as_float(own[i]));
                            ptx::tmem_ld_32x32b_x32(row_addr + c * 64 + 32, own);
                            ptx::tmem_wait_ld();
#pragma unroll
                            for (int i = 0; i < 32; ++i)
                                hi[i] = __float_as_uint(__uint_as_float(hi[i]) + __uint_as_float(own[i]));
                            continue;
                        }
                        const float4* part = slots + (j < s ? j : j - 1) * 512;
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const float4 f = part[q * 32 + lane];
                            lo[4 * q] = __float_as_uint(__uint_as_float(lo[4 * q]) + f.x);
                            lo[4 * q + 1] = __float_as_uint(__uint_as_float(lo[4 * q + 1]) + f.y);
                            lo[4 * q + 2] = __float_as_uint(__uint_as_float(lo[4 * q + 2]) + f.z);
                            lo[4 * q + 3] = __float_as_uint(__uint_as_float(lo[4 * q + 3]) + f.w);
                        }
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const float4 f = part[(8 + q) * 32 + lane];
                            hi[4 * q] = __float_as_uint(__uint_as_float(hi[4 * q]) + f.x);
                            hi[4 * q + 1] = __float_as_uint(__uint_as_float(hi[4 * q + 1]) + f.y);
                            hi[4 * q + 2] = __float_as_uint(__uint_as_float(hi[4 * q + 2]) + f.z);
                            hi[4 * q + 3] = __float_as_uint(__uint_as_float(hi[4 * q + 3]) + f.w);
                        }
                    }
                    if (m0 + quarter * 32 < M)
                        store_chunk(&map_c, staging, chunk_count, lo, hi, lane, n0 + c * 64, m0 + quarter * 32);
                }
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(&tmem_empty[acc]);
                continue;
            }
            if (m0 + quarter * 32 >= M) {
                // None of this warp's rows exist: nothing to store.
                ptx::tc_fence_before();
                __syncwarp();
                if (lane == 0) ptx::mbar_arrive(&tmem_empty[acc]);
                if (sender) ptx::mbar_arrive_release_cluster(recv_full_remote);
                continue;
            }
            if (sender && recv_mode == kClusterStages) {
                bool go = ptx::mbar_wait_cluster(go_bar, 0, limit_ns, abort);
                go = __all_sync(0xffffffffu, go);
                if (!go) {
                    // Rank 0 never freed its stages: store nothing and do not
                    // arrive; its own bounded wait for the values gives up.
                    if (lane == 0) record_failure(status, abort, kRoleEpilogue);
                    ptx::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(&tmem_empty[acc]);
                    continue;
                }
            }
            bool received = false;
#pragma unroll 1
            for (int c = 0; c < BN / 64; ++c) {
                uint32_t lo[32], hi[32];
                ptx::tmem_ld_32x32b_x32(row_addr + c * 64, lo);
                ptx::tmem_ld_32x32b_x32(row_addr + c * 64 + 32, hi);
                ptx::tmem_wait_ld();
                if (c == BN / 64 - 1) {
                    ptx::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive(&tmem_empty[acc]);
                }
                if (sender) {
                    const uint32_t dst = recv_remote + static_cast<uint32_t>(recv_chunk<BN>(s - 1, quarter, c, AR) * 16);
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        ptx::st_cluster_v4(dst + (q * 32 + lane) * 16, __uint_as_float(lo[4 * q]),
                                           __uint_as_float(lo[4 * q + 1]), __uint_as_float(lo[4 * q + 2]),
                                           __uint_as_float(lo[4 * q + 3]));
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        ptx::st_cluster_v4(dst + ((8 + q) * 32 + lane) * 16, __uint_as_float(hi[4 * q]),
                                           __uint_as_float(hi[4 * q + 1]), __uint_as_float(hi[4 * q + 2]),
                                           __uint_as_float(hi[4 * q + 3]));
                    continue;
                }
                if (receiver) {
                    if (!received) {
                        bool got = ptx::mbar_wait_cluster(recv_full, 0, limit_ns, abort);
                        got = __all_sync(0xffffffffu, got);
                        if (!got) {
                            if (lane == 0) record_failure(status, abort, kRoleEpilogue);
                            break;
                        }
                        received = true;
                        got_recv = true;
                    }
                    // Split 0's values, then every other split's, in split order.
#pragma unroll 1
                    for (int j = 1; j < splits; ++j) {
                        const float4* part = recv + recv_chunk<BN>(j - 1, quarter, c, AR);
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const float4 f = part[q * 32 + lane];
                            lo[4 * q] = __float_as_uint(__uint_as_float(lo[4 * q]) + f.x);
                            lo[4 * q + 1] = __float_as_uint(__uint_as_float(lo[4 * q + 1]) + f.y);
                            lo[4 * q + 2] = __float_as_uint(__uint_as_float(lo[4 * q + 2]) + f.z);
                            lo[4 * q + 3] = __float_as_uint(__uint_as_float(lo[4 * q + 3]) + f.w);
                        }
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            const float4 f = part[(8 + q) * 32 + lane];
                            hi[4 * q] = __float_as_uint(__uint_as_float(hi[4 * q]) + f.x);
                            hi[4 * q + 1] = __float_as_uint(__uint_as_float(hi[4 * q + 1]) + f.y);
                            hi[4 * q + 2] = __float_as_uint(__uint_as_float(hi[4 * q + 2]) + f.z);
                            hi[4 * q + 3] = __float_as_uint(__uint_as_float(hi[4 * q + 3]) + f.w);
                        }
                    }
                    store_chunk(&map_c, staging, chunk_count, lo, hi, lane, n0 + c * 64, m0 + quarter * 32);
                    continue;
                }
                if (splits > 1) {
                    float4* part = split_chunk<BN>(sk, t, s, quarter, c);
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        __stcg(part + q * 32 + lane, make_float4(__uint_as_float(lo[4 * q]), __uint_as_float(lo[4 * q + 1]),
                                                                 __uint_as_float(lo[4 * q + 2]), __uint_as_float(lo[4 * q + 3])));
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        __stcg(part + (8 + q) * 32 + lane,
                               make_float4(__uint_as_float(hi[4 * q]), __uint_as_float(hi[4 * q + 1]),
                                           __uint_as_float(hi[4 * q + 2]), __uint_as_float(hi[4 * q + 3])));
                    continue;
                }
                store_chunk(&map_c, staging, chunk_count, lo, hi, lane, n0 + c * 64, m0 + quarter * 32);
            }
            if (sender) {
                // Each lane releases its own stores into rank 0's buffer.
                ptx::mbar_arrive_release_cluster(recv_full_remote);
                continue;
            }
            if (receiver) continue;
            if (splits > 1) {
                // Publish this warp's partial rows, then count the unit.  The
                // unit that arrives last sums every split's rows in split
                // order and writes C; the others are done.
                __threadfence();
                __syncwarp();
                unsigned long long* counter = sk.counters + static_cast<size_t>(t) * 4 + quarter;
                int order = 0;
                if (lane == 0) order = arrive_counted(counter, sk.epoch);
                if (__shfl_sync(0xffffffffu, order, 0) != splits - 1) continue;
                __threadfence();
#pragma unroll 1
                for (int c = 0; c < BN / 64; ++c) {
                    float sum[64];
#pragma unroll 1
                    for (int j = 0; j < splits; ++j) {
                        const float4* part = split_chunk<BN>(sk, t, j, quarter, c);
#pragma unroll
                        for (int q = 0; q < 16; ++q) {
                            const float4 f = __ldcg(part + q * 32 + lane);
                            if (j == 0) {
                                sum[4 * q] = f.x;
                                sum[4 * q + 1] = f.y;
                                sum[4 * q + 2] = f.z;
                                sum[4 * q + 3] = f.w;
                            } else {
                                sum[4 * q] += f.x;
                                sum[4 * q + 1] += f.y;
                                sum[4 * q + 2] += f.z;
                                sum[4 * q + 3] += f.w;
                            }
                        }
                    }
                    uint32_t lo[32], hi[32];
#pragma unroll
                    for (int e = 0; e < 32; ++e) {
                        lo[e] = __float_as_uint(sum[e]);
                        hi[e] = __float_as_uint(sum[32 + e]);
                    }
                    store_chunk(&map_c, staging, chunk_count, lo, hi, lane, n0 + c * 64, m0 + quarter * 32);
                }
                __syncwarp();
                if (lane == 0) *counter = 0ull;  // every unit of the tile has arrived: clear for replays
            }
        }
        if (lane == 0) ptx::bulk_wait_group_read<0>();  // shared memory must outlive the stores' reads
        __syncwarp();
        // Rank 0 leaves only after the other ranks' stores into its buffer
        // are released, also when one of its own waits gave up (a rank that
        // gave up itself never stores: this wait then ends at its bound).
        // (The scatter form syncs the cluster below instead.)
        if (!kScatter && cluster_mode && blockIdx.x % splits == 0 && !got_recv)
            ptx::mbar_wait_cluster(recv_full, 0, drain_limit(limit_ns), no_abort);
        // A scatter warp that gave up before the meeting (stages mode)
        // still takes its phase, so the other CTAs' barrier completes.
        if (kScatter && recv_mode == kClusterStages && !met) {
            ptx::cluster_arrive();
            ptx::cluster_wait();
        }
    }

    if (cluster_mode && warp < 2) {
        ptx::cluster_wait();  // pairs this thread's arrive after set-up
        if (kScatter && recv_mode == kClusterStages) {
            // The scatter form's meeting counts every thread.
            ptx::cluster_arrive();
            ptx::cluster_wait();
        }
    }
    ptx::tc_fence_before();
    __syncthreads();
    // Receiving in its stages, rank 0 signalled the other ranks' barriers and
    // they stored into its shared memory; under the scatter form every rank
    // receives: no CTA leaves before all are done.
    if (recv_mode == kClusterStages || (kScatter && cluster_mode)) ptx::cluster_sync();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, L::kTmemCols);
    }
}

// ------------------------------------------------------------------ host side

// Whether a scatter split of `splits` ranks runs: 128-row tiles, every rank
// owning a piece, and the stages holding every piece (8 KB of FP32 each)
// plus the busiest rank's received copies.
// Copies the busiest rank of a scatter split receives (8 KB each).
int scatter_received(int bn, int ar, int splits) {
    return (scatter_pieces_of(bn, ar) + splits - 1) / splits * (splits - 1);
}

// Shared memory a receiving rank of a cluster split K needs beyond the
// kernel's own: rank 0, one slot of FP32 values per other rank; scatter,
// its received copies.
int cluster_recv_bytes(int bn, int ar, int splits, bool scatter) {
    return scatter ? scatter_received(bn, ar, splits) * 8192 : (splits - 1) * ar * bn * 4;
}

// How a cluster split K of `s` splits adds up.  Scatter (asked for, the
// pieces in the stages): receiving in a buffer past the kernel's own shared
// memory when that stays within 227 KB, else past the pieces in the stages
// when they hold both.  Otherwise rank 0 receives: in such a buffer, else in
// its stages, else nowhere (0).
int cluster_receive_mode(int s, int64_t own_smem, int64_t stage_bytes, int bn, int ar, bool scatter) {
    const int pieces = scatter_pieces_of(bn, ar);
    if (scatter && static_cast<int64_t>(pieces) * 8192 <= stage_bytes) {
        if (own_smem + cluster_recv_bytes(bn, ar, s, true) <= kMaxSmem) return kClusterScatter | kClusterBuffer;
        if (static_cast<int64_t>(pieces + scatter_received(bn, ar, s)) * 8192 <= stage_bytes)
            return kClusterScatter | kClusterStages;
    }
    if (own_smem + cluster_recv_bytes(bn, ar, s, false) <= kMaxSmem) return kClusterBuffer;
    if (cluster_recv_bytes(bn, ar, s, false) <= stage_bytes) return kClusterStages;
    return 0;
}

// K splits of a cluster split K for this launch (and where ranks receive,
// in *mode), or 0 when the workspace path runs: flag off, fewer than 2 or
// more than 8 splits, nowhere to receive, or (persistent launches) more
// units than SMs.
int cluster_splits(int flags, int k_splits, int num_kb, int tiles, bool persistent, int64_t own_smem,
                   int64_t stage_bytes, int bn, int ar, int* mode) {
    *mode = 0;
    if (!(flags & KMCTS_FLAG_SPLIT_CLUSTER)) return 0;
    const int s = k_splits < num_kb ? k_splits : num_kb;
    if (s < 2 || s > kMaxClusterSplits) return 0;
    if (persistent && static_cast<int64_t>(tiles) * s > multiprocessor_count()) return 0;
    *mode = cluster_receive_mode(s, own_smem, stage_bytes, bn, ar, (flags & KMCTS_FLAG_SPLIT_SCATTER) != 0);
    return *mode ? s : 0;
}

// K splits a launch can use: at most one per K block; 1 when the stream's
// workspace cannot be had (out of memory, or growth under graph capture).
template <int BN, int BK>
int resolve_splits(int M, int N, int K, int requested, cudaStream_t stream, SplitK* sk) {
    *sk = SplitK{1, nullptr, nullptr, 0, 0};
    const int num_kb = (K + BK - 1) / BK;
    int splits = requested < num_kb ? requested : num_kb;
    if (splits <= 1) return 1;
    const size_t tiles = static_cast<size_t>((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
    const size_t partial_bytes = tiles * splits * 4 * (BN / 64) * 32 * 64 * sizeof(float);
    const size_t counter_bytes = tiles * 4 * sizeof(unsigned long long);
    void* base = nullptr;
    int epoch = 0;
    if (!stream_workspace(stream, kWorkspaceSplitK, counter_bytes + partial_bytes, &base, &epoch)) return 1;
    sk->splits = splits;
    sk->counters = static_cast<unsigned long long*>(base);
    sk->partials = reinterpret_cast<float*>(static_cast<char*>(base) + counter_bytes);
    sk->epoch = epoch;
    return splits;
}

// The four instantiations of a one-CTA schedule: plain, cache hints only,
// cluster split K (with hints), and its scatter form.
template <int BN, int BK, int STAGES, bool B_MN, int AR>
struct Kernels {
    static constexpr int kScatterFeat = kFeatHints | kFeatCluster | kFeatScatter;
    static constexpr auto plain = gemm_bf16_tcgen05<BN, BK, STAGES, B_MN, AR, 0>;
    static constexpr auto hint = gemm_bf16_tcgen05<BN, BK, STAGES, B_MN, AR, kFeatHints>;
    static constexpr auto cluster = gemm_bf16_tcgen05<BN, BK, STAGES, B_MN, AR, kFeatHints | kFeatCluster>;
    static constexpr auto scatter = gemm_bf16_tcgen05<BN, BK, STAGES, B_MN, AR, kScatterFeat>;

    // The shared-memory opt-in is per device; set it once on each, to the
    // most any launch of this variant asks for (a cluster split K's receive
    // buffer comes on top of the variant's own layout).
    static bool configure() {
        static std::mutex mu;
        static bool configured[kMaxDevices] = {};
        int device = 0;
        if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return false;
        std::lock_guard<std::mutex> lock(mu);
        if (!configured[device]) {
            for (auto fn : {plain, hint, cluster, scatter})
                if (cudaFuncSetAttribute(fn, cudaFuncAttributeMaxDynamicSharedMemorySize, kMaxSmem) != cudaSuccess)
                    return false;
            configured[device] = true;
        }
        return true;
    }
};

// Clusters of `splits` CTAs of this schedule's cluster split K (receive
// `mode`) that can be resident at once on the current device, as the
// occupancy calculator places them (GPC by GPC); 0 when it cannot say.
template <int BN, int BK, int STAGES, bool B_MN, int AR>
int variant_cluster_capacity(int splits, int mode) {
    using L = Layout<BN, BK, STAGES, B_MN, AR>;
    using KS = Kernels<BN, BK, STAGES, B_MN, AR>;
    if (!KS::configure()) return 0;
    const bool scatter = (mode & kClusterScatter) != 0;
    int smem = L::kSmemBytes;
    if (mode & kClusterBuffer) smem += cluster_recv_bytes(BN, AR, splits, scatter);
    cudaLaunchConfig_t lc = {};
    lc.gridDim = dim3(static_cast<unsigned>(splits));
    lc.blockDim = dim3(kThreads);
    lc.dynamicSmemBytes = static_cast<size_t>(smem);
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    lc.attrs = attr;
    lc.numAttrs = 1;
    int clusters = 0;
    const cudaError_t rc = scatter ? cudaOccupancyMaxActiveClusters(&clusters, KS::scatter, &lc)
                                   : cudaOccupancyMaxActiveClusters(&clusters, KS::cluster, &lc);
    if (rc != cudaSuccess) {
        (void)cudaGetLastError();
        return 0;
    }
    return clusters;
}

template <int BN, int BK, int STAGES, bool B_MN, int AR>
int launch_variant(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mc, int M,
                   int N, int K, int group, bool persistent, int k_splits, int flags,
                   uint64_t limit_ns, cudaStream_t stream, int* status) {
    using L = Layout<BN, BK, STAGES, B_MN, AR>;
    using KS = Kernels<BN, BK, STAGES, B_MN, AR>;
    if (!KS::configure()) return KMCTS_EGEMM;
    const int tiles = ((M + kBM - 1) / kBM) * ((N + BN - 1) / BN);
    const int sms = multiprocessor_count();
    SplitK sk = {1, nullptr, nullptr, 0, 0};
    int mode = 0;
    int splits = cluster_splits(flags, k_splits, (K + BK - 1) / BK, tiles, persistent, L::kSmemBytes,
                                static_cast<int64_t>(STAGES) * L::kStageBytes, BN, AR, &mode);
    int smem = L::kSmemBytes;
    if (splits > 0) {
        sk = SplitK{splits, nullptr, nullptr, 0, mode};
        if (mode & kClusterBuffer) smem += cluster_recv_bytes(BN, AR, splits, (mode & kClusterScatter) != 0);
    } else splits = resolve_splits<BN, BK>(M, N, K, k_splits, stream, &sk);
    const int units = tiles * splits;
    int grid = units;
    if (persistent && !sk.cluster) grid = units < sms ? units : sms;
    const int evict_first =
        ((flags & KMCTS_FLAG_B_EVICT_FIRST) ? 1 : 0) | ((flags & KMCTS_FLAG_A_EVICT_FIRST) ? 2 : 0);
    auto kernel = (sk.cluster & kClusterScatter) ? KS::scatter
                  : sk.cluster                      ? KS::cluster
                  : evict_first                     ? KS::hint
                                                    : KS::plain;
    if (sk.cluster) {
        cudaLaunchConfig_t lc = {};
        lc.gridDim = dim3(static_cast<unsigned>(grid));
        lc.blockDim = dim3(kThreads);
        lc.dynamicSmemBytes = static_cast<size_t>(smem);
        lc.stream = stream;
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = static_cast<unsigned>(splits);
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        lc.attrs = attr;
        lc.numAttrs = 1;
        if (cudaLaunchKernelEx(&lc, kernel, ma, mb, mc, M, N, K, group, limit_ns, status, sk, evict_first) !=
            cudaSuccess)
            return KMCTS_EGEMM;
    } else {
        kernel<<<grid, kThreads, smem, stream>>>(ma, mb, mc, M, N, K, group, limit_ns, status, sk, evict_first);
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError() == cudaSuccess ? KMCTS_OK : KMCTS_EGEMM;
}

using Launcher = int (*)(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, int, int,
                         int, int, bool, int, int, uint64_t, cudaStream_t, int*);

struct Variant {
    int bn, bk, stages, b_mn, ar;
    Launcher fn;
    int (*capacity)(int splits, int mode);  // resident clusters of a cluster split K
};

#define KMCTS_VARIANT_AR(BN, BK, ST, MN, AR) \
    {BN, BK, ST, MN, AR, &launch_variant<BN, BK, ST, MN, AR>, &variant_cluster_capacity<BN, BK, ST, MN, AR>}
#define KMCTS_VARIANT(BN, BK, ST, MN) KMCTS_VARIANT_AR(BN, BK, ST, MN, kBM)
#define KMCTS_SKINNY(BN, BK, ST, MN) KMCTS_VARIANT_AR(BN, BK, ST, MN, 32)
#define KMCTS_HALF(BN, BK, ST, MN) KMCTS_VARIANT_AR(BN, BK, ST, MN, 64)

// The compiled 1-CTA schedule space: every (tile_n, tile_k, stages) of the
// sweep grid that fits 227 KB (stages*(128+BN)*BK*2 + 32 KB staging + 2 KB),
// plus a few off-grid shapes.
const Variant kVariants[] = {
    KMCTS_VARIANT(256, 64, 3, false), KMCTS_VARIANT(256, 64, 4, false),
    KMCTS_VARIANT(256, 64, 3, true),  KMCTS_VARIANT(256, 64, 4, true),
    KMCTS_VARIANT(128, 64, 3, false), KMCTS_VARIANT(128, 64, 3, true),
    KMCTS_VARIANT(128, 64, 4, false), KMCTS_VARIANT(128, 64, 5, false),
    KMCTS_VARIANT(128, 64, 6, false), KMCTS_VARIANT(128, 64, 4, true),
    KMCTS_VARIANT(128, 64, 5, true),  KMCTS_VARIANT(128, 64, 6, true),
    KMCTS_VARIANT(128, 128, 3, false), KMCTS_VARIANT(128, 128, 3, true),
    KMCTS_VARIANT(256, 128, 2, false), KMCTS_VARIANT(256, 128, 2, true),
    KMCTS_VARIANT(192, 64, 4, false), KMCTS_VARIANT(192, 64, 4, true),
    KMCTS_VARIANT(64, 64, 6, false),  KMCTS_VARIANT(64, 64, 6, true),
    // tile_m 32 (M <= 32): A staged as 32 rows and one warp's epilogue
    // staging, so more B stages are in flight.
    KMCTS_SKINNY(256, 64, 5, false),  KMCTS_SKINNY(256, 64, 5, true),
    KMCTS_SKINNY(128, 64, 9, false),  KMCTS_SKINNY(128, 64, 9, true),
    KMCTS_SKINNY(128, 128, 4, false), KMCTS_SKINNY(128, 128, 4, true),
    KMCTS_SKINNY(64, 128, 8, false),  KMCTS_SKINNY(64, 128, 8, true),
    // tile_m 64 (M <= 64): A staged as 64 rows, two warps' epilogue staging.
    KMCTS_HALF(128, 128, 4, false),   KMCTS_HALF(128, 128, 4, true),
    KMCTS_HALF(128, 128, 3, false),   KMCTS_HALF(128, 128, 3, true),
    KMCTS_HALF(64, 128, 6, false),    KMCTS_HALF(64, 128, 6, true),
};

// Rows of A a one-CTA schedule stages per tile: 32 or 64 for skinny M, else 128.
int a_rows(const kmcts_gemm_config& cfg) { return cfg.tile_m == 32 || cfg.tile_m == 64 ? cfg.tile_m : kBM; }

const Variant* find_variant(const kmcts_gemm_config& cfg, int b_layout) {
    for (const Variant& v : kVariants) {
        if (v.bn == cfg.tile_n && v.bk == cfg.tile_k && v.stages == cfg.stages &&
            v.b_mn == (b_layout == KMCTS_B_ROW ? 1 : 0) && v.ar == a_rows(cfg)) {
            return &v;
        }
    }
    return nullptr;
}

void put_reason(char* why, int len, const char* text) {
    if (why && len > 0) {
        std::strncpy(why, text, static_cast<size_t>(len) - 1);
        why[len - 1] = '\0';
    }
}

bool is_pair(const kmcts_gemm_config& cfg) { return cfg.tile_m == 256; }
bool is_one_cta(const kmcts_gemm_config& cfg) { return cfg.tile_m == kBM || cfg.tile_m == 64 || cfg.tile_m == 32; }

}  // namespace

bool is_swapped(const kmcts_gemm_config& cfg) { return (cfg.flags & KMCTS_FLAG_SWAP_AB) != 0; }

int64_t tcgen05_smem_bytes(const kmcts_gemm_config& cfg, int b_layout) {
    (void)b_layout;
    if (cfg.tile_n <= 0 || cfg.tile_k <= 0 || cfg.stages <= 0) return 0;
    if (is_swapped(cfg)) return cfg.tile_m == 32 ? stream_smem_bytes(cfg.tile_k, cfg.stages) : 0;
    if (cfg.tile_m == 256) return pair_smem_bytes(cfg.tile_n, cfg.tile_k, cfg.stages);
    if (cfg.tile_m != kBM && cfg.tile_m != 64 && cfg.tile_m != 32) return 0;
    return static_cast<int64_t>(cfg.stages) * (cfg.tile_m + cfg.tile_n) * cfg.tile_k * 2 +
           (cfg.tile_m / 32) * 2 * kStagingBytes + kSmemReserve;
}

int cluster_split_cap(const kmcts_gemm_config& cfg, int b_layout) {
    if (!is_one_cta(cfg) || is_swapped(cfg) || cfg.tile_n <= 0) return 1;
    const int64_t own = tcgen05_smem_bytes(cfg, b_layout);
    const int ar = a_rows(cfg);
    const int64_t stage_bytes = static_cast<int64_t>(cfg.stages) * (ar + cfg.tile_n) * cfg.tile_k * 2;
    int cap = 1;
    const bool scatter = (cfg.flags & KMCTS_FLAG_SPLIT_SCATTER) != 0;
    while (cap < kMaxClusterSplits && cluster_receive_mode(cap + 1, own, stage_bytes, cfg.tile_n, ar, scatter)) ++cap;
    return cap;
}

bool cluster_split_fits(const kmcts_gemm_config& cfg, int b_layout, int splits) {
    if (!is_one_cta(cfg) || is_swapped(cfg) || cfg.tile_n <= 0 || splits < 2 || splits > kMaxClusterSplits) return false;
    const int ar = a_rows(cfg);
    const int64_t stage_bytes = static_cast<int64_t>(cfg.stages) * (ar + cfg.tile_n) * cfg.tile_k * 2;
    const int mode = cluster_receive_mode(splits, tcgen05_smem_bytes(cfg, b_layout), stage_bytes, cfg.tile_n, ar,
                                          (cfg.flags & KMCTS_FLAG_SPLIT_SCATTER) != 0);
    return mode != 0 && ((mode & kClusterScatter) != 0) == ((cfg.flags & KMCTS_FLAG_SPLIT_SCATTER) != 0);
}

int cluster_capacity(const kmcts_gemm_config& cfg, int b_layout, int splits) {
    if (!is_one_cta(cfg) || is_swapped(cfg) || splits < 2 || splits > kMaxClusterSplits) return 0;
    const Variant* v = find_variant(cfg, b_layout);
    if (v == nullptr) return 0;
    const int64_t own = tcgen05_smem_bytes(cfg, b_layout);
    const int ar = a_rows(cfg);
    const int64_t stage_bytes = static_cast<int64_t>(cfg.stages) * (ar + cfg.tile_n) * cfg.tile_k * 2;
    const int mode = cluster_receive_mode(splits, own, stage_bytes, cfg.tile_n, ar,
                                          (cfg.flags & KMCTS_FLAG_SPLIT_SCATTER) != 0);
    if (mode == 0) return 0;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) {
        (void)cudaGetLastError();
        return 0;
    }
    // The answer depends on the device, the instantiation and the launch
    // shape only: ask the occupancy calculator once for each.
    static std::mutex mu;
    static std::map<std::tuple<int, const Variant*, int, int>, int> cache;
    const auto key = std::make_tuple(device, v, splits, mode);
    {
        std::lock_guard<std::mutex> lock(mu);
        const auto it = cache.find(key);
        if (it != cache.end()) return it->second;
    }
    const int clusters = v->capacity(splits, mode);
    std::lock_guard<std::mutex> lock(mu);
    cache[key] = clusters;
    return clusters;
}

int tcgen05_legal(const kmcts_gemm_config& cfg, int M, int N, int K, int b_layout, char* why,
                  int len) {
    if (b_layout != KMCTS_B_COL && b_layout != KMCTS_B_ROW) {
        put_reason(why, len, "b_layout must be 0 (column-major) or 1 (row-major)");
        return KMCTS_EINVAL;
    }
    if (M < 0 || N < 0 || K < 0) {
        put_reason(why, len, "negative dimension");
        return KMCTS_EINVAL;
    }
    if (cfg.raster_group < 1) {
        put_reason(why, len, "raster_group must be >= 1");
        return KMCTS_EINVAL;
    }
    if (cfg.k_splits < 0) {
        put_reason(why, len, "k_splits must be >= 0");
        return KMCTS_EINVAL;
    }
    if (is_swapped(cfg)) {
        if (cfg.tile_m != 32 || cfg.cluster_m != 1 || cfg.cluster_n != 1 || cfg.tile_n != 128) {
            put_reason(why, len, "the swapped schedule takes tile_m 32, tile_n 128 and a 1x1 cluster");
            return KMCTS_ENOTSUP;
        }
        if (M > 32) {
            put_reason(why, len, "the swapped schedule puts A's rows in the MMA's N: it takes M <= 32");
            return KMCTS_ENOTSUP;
        }
        const int64_t smem = tcgen05_smem_bytes(cfg, b_layout);
        if (smem <= 0 || smem > kMaxSmem) {
            put_reason(why, len, "shared memory per CTA exceeds 227 KB");
            return KMCTS_ESMEM;
        }
        if (!stream_variant_exists(cfg, b_layout)) {
            put_reason(why, len, "the swapped schedule is compiled for tile_k 64 x 10 stages and 128 x 5");
            return KMCTS_ENOTSUP;
        }
        if (K % 8 != 0 || N % 8 != 0) {
            put_reason(why, len, "TMA needs K and N to be multiples of 8");
            return KMCTS_ENOTSUP;
        }
        put_reason(why, len, "ok");
        return KMCTS_OK;
    }
    if (cfg.k_splits > 1 && !is_one_cta(cfg) && !(is_pair(cfg) && cfg.cluster_n == 1)) {
        put_reason(why, len, "split K runs on one-CTA schedules (tile_m 128 or 32) and CTA pairs (cluster 2x1)");
        return KMCTS_ENOTSUP;
    }
    if (cfg.cluster_m < 1 || cfg.cluster_n < 1) {
        put_reason(why, len, "cluster dimensions must be positive");
        return KMCTS_EINVAL;
    }
    if (cfg.cluster_n != 1 && !(cfg.cluster_n == 2 && cfg.tile_m == 256)) {
        put_reason(why, len,
                   "cluster_n 2 takes tile_m 256 (two CTA pairs sharing A); one-CTA schedules and larger "
                   "clusters would need a TMA multicast, which this library never issues");
        return KMCTS_ENOTSUP;
    }
    if (cfg.cluster_n == 2 && (cfg.tile_n != 256 || cfg.tile_k != 128 || cfg.stages != 3)) {
        put_reason(why, len, "cluster_n 2 is compiled for tile_n 256, tile_k 128, 3 stages");
        return KMCTS_ENOTSUP;
    }
    if (is_one_cta(cfg)) {
        if (cfg.cluster_m != 1) {
            put_reason(why, len, "tile_m 128, 64 and 32 run one CTA per tile (cluster 1x1)");
            return KMCTS_ENOTSUP;
        }
        if (cfg.tile_m == 32 && M > 32) {
            put_reason(why, len, "tile_m 32 stages 32 rows of A: it takes M <= 32");
            return KMCTS_ENOTSUP;
        }
        if (cfg.tile_m == 64 && M > 64) {
            put_reason(why, len, "tile_m 64 stages 64 rows of A: it takes M <= 64");
            return KMCTS_ENOTSUP;
        }
    } else if (cfg.tile_m == 256) {
        if (cfg.cluster_m != 2) {
            put_reason(why, len, "tile_m 256 is one CTA pair (cluster 2x1, tcgen05 cta_group::2)");
            return KMCTS_ENOTSUP;
        }
        if (cfg.tile_n != 128 && cfg.tile_n != 256) {
            put_reason(why, len, "a CTA pair takes tile_n 128 or 256");
            return KMCTS_ENOTSUP;
        }
    } else {
        put_reason(why, len, "tile_m must be 128, 64 or 32 (one CTA) or 256 (CTA pair)");
        return KMCTS_ENOTSUP;
    }
    const int64_t smem = tcgen05_smem_bytes(cfg, b_layout);
    if (smem <= 0 || smem > kMaxSmem) {
        put_reason(why, len, "shared memory per CTA exceeds 227 KB");
        return KMCTS_ESMEM;
    }
    const bool compiled = is_pair(cfg) ? pair_variant_exists(cfg, b_layout)
                                       : find_variant(cfg, b_layout) != nullptr;
    if (!compiled) {
        put_reason(why, len, "schedule (tile_m, tile_n, tile_k, stages) is not compiled in");
        return KMCTS_ENOTSUP;
    }
    // TMA: every global row stride must be a multiple of 16 bytes.
    if (K % 8 != 0 || N % 8 != 0) {
        put_reason(why, len, "TMA needs K and N to be multiples of 8");
        return KMCTS_ENOTSUP;
    }
    put_reason(why, len, "ok");
    return KMCTS_OK;
}

int launch_tcgen05(const void* A, const void* B, void* C, int M, int N, int K, int b_layout,
                   const kmcts_gemm_config& cfg, cudaStream_t stream, int* device_status) {
    int rc = tcgen05_legal(cfg, M, N, K, b_layout, nullptr, 0);
    if (rc != KMCTS_OK) return rc;
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B) |
         reinterpret_cast<uintptr_t>(C)) &
        15u) {
        return KMCTS_ENOTSUP;
    }
    if (M == 0 || N == 0) return KMCTS_OK;
    if (K == 0) {
        g_launches.fetch_add(1, std::memory_order_relaxed);
        return cudaMemsetAsync(C, 0, static_cast<size_t>(M) * N * 2, stream) == cudaSuccess
                   ? KMCTS_OK
                   : KMCTS_EGEMM;
    }
    if (is_swapped(cfg)) {
        const uint64_t limit =
            cfg.wait_limit_ns > 0 ? static_cast<uint64_t>(cfg.wait_limit_ns) : kDefaultWaitNs;
        int* status = device_status ? device_status : default_status_ptr();
        if (status == nullptr) return KMCTS_EHANDLE;
        return launch_stream(A, B, C, M, N, K, b_layout, cfg, limit, stream, status);
    }
    const bool pair = is_pair(cfg);
    // Each CTA stages 128 rows of A, and BN (one CTA) or BN/2 (pair) of B.
    const uint32_t b_rows = pair ? cfg.tile_n / 2 : cfg.tile_n;
    CUtensorMap ma, mb, mb_half, mc;
    bool ok = encode_tensor_map_2d(&ma, A, K, M, static_cast<uint64_t>(K) * 2, 64,
                                   pair ? kBM : static_cast<uint32_t>(a_rows(cfg)));
    if (b_layout == KMCTS_B_COL) {
        ok = ok && encode_tensor_map_2d(&mb, B, K, N, static_cast<uint64_t>(K) * 2, 64, b_rows);
        // Half-width units of a pair stage b_rows / 2 columns of B.
        ok = ok && (!pair || encode_tensor_map_2d(&mb_half, B, K, N, static_cast<uint64_t>(K) * 2, 64,
                                                  b_rows / 2));
    } else {
        ok = ok && encode_tensor_map_2d(&mb, B, N, K, static_cast<uint64_t>(N) * 2, 64, 64);
        mb_half = mb;
    }
    ok = ok && encode_tensor_map_2d(&mc, C, N, M, static_cast<uint64_t>(N) * 2, 64, 32);
    if (!ok) return KMCTS_EINVAL;
    const uint64_t limit =
        cfg.wait_limit_ns > 0 ? static_cast<uint64_t>(cfg.wait_limit_ns) : kDefaultWaitNs;
    if (pair) return launch_pair(ma, mb, mb_half, mc, M, N, K, b_layout, cfg, limit, stream, device_status);
    const Variant* v = find_variant(cfg, b_layout);
    return v->fn(ma, mb, mc, M, N, K, cfg.raster_group, cfg.persistent != 0, cfg.k_splits, cfg.flags, limit,
                 stream, device_status);
}

int launch_allgather_tcgen05(const void* A, const void* B_shard, void* const* C_ranks, int num_ranks, int rank,
                             int M, int N_total, int K, int b_layout, const kmcts_gemm_config& cfg,
                             cudaStream_t stream, int* device_status) {
    if (num_ranks < 1 || num_ranks > KMCTS_MAX_RANKS || rank < 0 || rank >= num_ranks || !C_ranks || M < 0 ||
        N_total < 0 || K < 0 || N_total % num_ranks != 0)
        return KMCTS_EINVAL;
    const int n_shard = N_total / num_ranks;
    if (n_shard % 256 != 0 || !is_pair(cfg) || cfg.cluster_n != 1) return KMCTS_ENOTSUP;
    int rc = tcgen05_legal(cfg, M, n_shard, K, b_layout, nullptr, 0);
    if (rc != KMCTS_OK) return rc;
    void* own = C_ranks[rank];
    void* peers[KMCTS_MAX_RANKS - 1];
    int peer_count = 0;
    for (int r = 0; r < num_ranks; ++r) {
        if (!C_ranks[r]) return KMCTS_EINVAL;
        if (r != rank) peers[peer_count++] = C_ranks[r];
    }
    if ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B_shard) | reinterpret_cast<uintptr_t>(own)) &
        15u)
        return KMCTS_ENOTSUP;
    if (M == 0 || n_shard == 0 || K == 0) return K == 0 ? KMCTS_ENOTSUP : KMCTS_OK;
    const uint32_t b_rows = cfg.tile_n / 2;
    CUtensorMap ma, mb, mb_half, mc;
    bool ok = encode_tensor_map_2d(&ma, A, K, M, static_cast<uint64_t>(K) * 2, 64, kBM);
    if (b_layout == KMCTS_B_COL) {
        ok = ok && encode_tensor_map_2d(&mb, B_shard, K, n_shard, static_cast<uint64_t>(K) * 2, 64, b_rows);
        ok = ok && encode_tensor_map_2d(&mb_half, B_shard, K, n_shard, static_cast<uint64_t>(K) * 2, 64, b_rows / 2);
    } else {
        ok = ok && encode_tensor_map_2d(&mb, B_shard, n_shard, K, static_cast<uint64_t>(n_shard) * 2, 64, 64);
        mb_half = mb;
    }
    // This rank's C map covers the full [M, N_total] C; the kernel adds the
    // rank's column offset to every store.
    ok = ok && encode_tensor_map_2d(&mc, own, N_total, M, static_cast<uint64_t>(N_total) * 2, 64, 32);
    if (!ok) return KMCTS_EINVAL;
    const uint64_t limit = cfg.wait_limit_ns > 0 ? static_cast<uint64_t>(cfg.wait_limit_ns) : kDefaultWaitNs;
    return launch_pair_allgather(ma, mb, mb_half, mc, M, n_shard, K, b_layout, cfg, limit, stream, device_status,
                                 peers, peer_count, N_total, rank * n_shard);
}

int plan_tcgen05(const kmcts_gemm_config& cfg, int M, int N, int K, int b_layout, kmcts_gemm_plan* out) {
    const int rc = tcgen05_legal(cfg, M, N, K, b_layout, nullptr, 0);
    if (rc != KMCTS_OK) return rc;
    if (is_pair(cfg)) return plan_pair(cfg, M, N, K, b_layout, out);
    if (is_swapped(cfg)) return plan_stream(cfg, M, N, K, out);
    kmcts_gemm_plan plan = {};
    plan.kernel = 1;
    plan.cluster_size = 1;
    plan.workers = multiprocessor_count();
    plan.tiles = ((M + kBM - 1) / kBM) * ((N + cfg.tile_n - 1) / cfg.tile_n);
    plan.full_tiles = plan.tiles;
    const int num_kb = (K + cfg.tile_k - 1) / cfg.tile_k;
    plan.k_splits = cfg.k_splits > 1 ? (cfg.k_splits < num_kb ? cfg.k_splits : num_kb) : 1;
    if (plan.k_splits < 1) plan.k_splits = 1;
    plan.units = plan.tiles * plan.k_splits;
    plan.ctas = cfg.persistent ? (plan.units < plan.workers ? plan.units : plan.workers) : plan.units;
    plan.smem_bytes = static_cast<int32_t>(tcgen05_smem_bytes(cfg, b_layout));
    const int ar = a_rows(cfg);
    int mode = 0;
    const int cs = cluster_splits(cfg.flags, cfg.k_splits, num_kb, plan.tiles, cfg.persistent != 0, plan.smem_bytes,
                                  static_cast<int64_t>(cfg.stages) * (ar + cfg.tile_n) * cfg.tile_k * 2, cfg.tile_n,
                                  ar, &mode);
    if (cs > 0) {
        plan.cluster_size = cs;
        // Resident clusters as the occupancy calculator places them; at most
        // one CTA per SM in whole clusters where it cannot say.
        const int capacity = cluster_capacity(cfg, b_layout, cs);
        plan.workers = capacity > 0 ? capacity : plan.workers / cs;
        plan.ctas = plan.units;
        if (mode & kClusterBuffer)
            plan.smem_bytes += cluster_recv_bytes(cfg.tile_n, ar, cs, (mode & kClusterScatter) != 0);
        plan.split_reduce = (mode & kClusterScatter) ? KMCTS_SPLIT_SCATTER : KMCTS_SPLIT_CLUSTER;
    }
    *out = plan;
    return KMCTS_OK;
}

int take_default_status(cudaStream_t stream, int* value) {
    int zero = 0;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return KMCTS_ESYNC;
    if (cudaMemcpyFromSymbol(value, g_default_status, sizeof(int)) != cudaSuccess)
        return KMCTS_ESYNC;
    if (*value != 0 && cudaMemcpyToSymbol(g_default_status, &zero, sizeof(int)) != cudaSuccess)
        return KMCTS_ESYNC;
    return KMCTS_OK;
}

}  // namespace kmcts
