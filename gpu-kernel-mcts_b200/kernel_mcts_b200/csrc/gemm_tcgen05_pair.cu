// CTA-pair (2-SM) persistent BF16 GEMM for sm_100a: one tcgen05.mma.cta_group::2
// computes a 256 x BN tile across a cluster of two CTAs.
//
// Why pairs: with one CTA per 128 x 256 tile every SM streams all 256 columns
// of B through its own shared memory; in a pair each CTA stages only its half
// of B (and its own 128 rows of A) and the pair's UMMA reads both halves, so
// shared-memory operand traffic per SM drops by a third and each B byte is
// fetched from L2 once per 256 rows of C instead of once per 128.
//
// Roles per CTA (192 threads), as in the 1-CTA kernel:
//   warp 0     TMA producer in both CTAs.  Each CTA loads its own A rows and
//              B columns; both signal the leader's (rank 0) full barrier with
//              cp.async.bulk.tensor...cta_group::2 (no multicast).  The leader
//              alone posts the pair's expected byte count.
//   warp 1     allocates TMEM in both CTAs (cta_group::2).  Lane 0 of the
//              leader issues every UMMA and commits, multicast to both CTAs,
//              the stage-release and accumulator-ready barriers.
//   warps 2-5  epilogue in both CTAs: drain this CTA's 128 accumulator rows
//              from TMEM, round to BF16, TMA-store; then arrive (remotely for
//              the peer) on the leader's accumulator-empty barrier.
// The slot schedule (cluster_n 2, 256 threads) runs two such pairs in a 4-CTA
// cluster that share their rows of A: warps 6 and 7 exchange K halves of A
// between the pairs over distributed shared memory (see "A exchange" below).
// EF instantiations load A and B with an L2 cache policy (evict-first for an
// operand read by one or two rows or columns of pair tiles).
// Every wait is bounded; see gemm_tcgen05.cu for the failure protocol.
#include <cstring>
#include <mutex>

#include "gemm_common.cuh"
#include "kmcts_internal.h"

namespace kmcts {

namespace {

using namespace gemm;

template <int BN, int BK, int STAGES, bool B_MN>
struct PairLayout {
    static constexpr int kHalfN = BN / 2;  // B columns staged by each CTA
    static constexpr int kABytes = 128 * BK * 2;
    static constexpr int kBBytes = kHalfN * BK * 2;
    static constexpr int kStageBytes = kABytes + kBBytes;
    static constexpr int kStagingOffset = STAGES * kStageBytes;
    static constexpr int kBarrierOffset = kStagingOffset + kEpilogueWarps * 2 * kStagingBytes;
    static constexpr int kSmemBytes = kBarrierOffset + kSmemReserve;
    static constexpr uint32_t kTmemCols = tmem_columns_for(2 * BN);
    static_assert(BN == 128 || BN == 256, "pair tile N must be 128 or 256");
    static_assert(BK == 64 || BK == 128, "BK must be 64 or 128");
    static_assert(kSmemBytes <= kMaxSmem, "shared memory budget exceeded");
};

// Where a fused GEMM + all-gather also writes C: the other ranks' full C
// buffers (IPC-mapped peer memory), their row stride, and this rank's column
// offset inside the full C.  Unused (count 0, offset 0) by plain GEMMs.
struct PeerOutputs {
    CUtensorMap map[KMCTS_MAX_RANKS - 1];  // each peer's full C [M, N_total]
    int count;
    int col_offset;
};

// Work list.  Tiles [0, full_tiles) run whole, round-robin over the W
// co-resident clusters.  With T tiles = q W + rem (0 < rem, q >= 1), a plain
// round-robin leaves W - rem clusters idle for the whole last round; the
// tiles after full_tiles run instead as:
//   kTailStreamK  (opt-in) the last W + rem tiles' K blocks, cut into W
//                 equal contiguous ranges, one per cluster (stream-K);
//                 full_tiles = (q - 1) W.  A range is at least one tile long,
//                 so a tile is either inside one range (run whole) or split
//                 at one range boundary into a K prefix, the last unit of
//                 cluster c - 1, and a K suffix, the first unit of cluster c.
//                 Per (CTA, TMEM lane quarter) the segment that reaches its
//                 epilogue first stores its FP32 rows to the boundary's
//                 partial slot and raises a ready flag; the second waits
//                 (bounded) for the flag, adds the partial, rounds once to
//                 BF16 and clears the flags.  The second only ever waits on a
//                 segment that has already arrived, so no wait depends on
//                 scheduling; and as the suffix runs first in its range and
//                 the prefix last in its, the partial is normally long stored
//                 when the prefix arrives.  Each output of a split tile is the
//                 FP32 sum of two K-ordered chains (addition commutes, so the
//                 bits do not depend on which segment arrived first).
//   kTailSplitN   (default; 2 rem <= W, BN 256) each of the last rem tiles as two
//                 BN/2-wide halves on two clusters.  Every output stays one
//                 full-K UMMA chain, bit-identical to whole tiles; but
//                 half-width pair MMAs stage 1.5x the operand bytes per FLOP,
//                 so a half unit takes about 3/4 of a whole tile's time.
// Flags carry the launch's epoch (a per-workspace host counter), so values
// left by an earlier failed launch are never taken for this launch's.
//
// kSplitK (k_splits = S > 1, few tiles over a long K) is not a tail mode: every
// tile runs as S units over consecutive K ranges, dealt round-robin like whole
// tiles (full_tiles then counts units).  Each unit stores both CTAs' FP32 rows
// in the workspace and counts itself per (CTA rank, lane quarter) on the
// tile's epoch-tagged counter; the unit that arrives last adds the S partials
// in split order and writes C, as the one-CTA kernel's split K does.  Nothing
// waits.
//
// kTailSplitK   (opt-in; 2 rem <= W, BN 256) each of the last rem tiles as its
//               two K halves on two clusters (c and c ^ 1).  Each half-unit
//               stores its FP32 values of the other's BN/2 columns in the
//               tile's partial slot and raises its ready flag, then waits
//               (bounded) for the other's flag, adds the other's values to
//               its own for its BN/2 columns, rounds once and stores C.  Both
//               units raise their flag before waiting, and both are the last
//               units of co-resident clusters with the same number of whole
//               tiles before them, so each wait is for work already running.
constexpr int kTailWhole = 0, kTailSplitN = 1, kTailStreamK = 2, kSplitK = 3, kTailSplitK = 4;

struct TailSplit {
    float* partials;  // stream-K: [boundary][CTA rank][quarter][BN/64 chunks][16 float4][32 lanes];
                      // split K: [tile][split][CTA rank][quarter][BN/64 chunks][16 float4][32 lanes]
    int* ready;       // [boundary][CTA rank][quarter]
    int* arrivals;    // [boundary][CTA rank][quarter]
    unsigned long long* counters;  // split K: [tile][CTA rank][quarter], epoch << 32 | units arrived
    int splits;                    // split K: K ranges per tile
    int epoch;
    int mode;
    int evict_first;  // L2 evict-first loads for operands read once or twice: bit 0 B, bit 1 A
};

struct Unit {
    int m_blk, n0, width, kb0, kb1;
    int boundary;  // stream-K: the range boundary splitting this tile, else -1
    int tile, split;  // split K: the tile and its K range, else -1
};

// Stream-K ranges: cluster c owns K blocks [lo(c), lo(c + 1)) of the
// stream-K tiles (tile-major, K blocks within a tile in order).
__device__ __forceinline__ long long sk_lo(int c, long long total, int p) {
    return static_cast<long long>(c) * total / p;
}

// The cluster whose range holds K block g: the largest c with lo(c) <= g.
__device__ __forceinline__ int sk_owner(long long g, long long total, int p) {
    return static_cast<int>(((g + 1) * p + total - 1) / total - 1);
}

// One cluster's work list: its whole tiles, then its tail units.
struct Schedule {
    int num_m, num_n, group, num_kb, full_tiles, clusters, cluster;
    int n_full, n_tail;
    long long g0, g1;  // stream-K range
    long long total;   // stream-K K blocks

    __device__ int count() const { return n_full + n_tail; }
};

__device__ __forceinline__ Schedule make_schedule(int M, int N, int K, int BN, int BK, int group, int full_tiles,
                                                  int cluster, int clusters, const TailSplit& tail) {
    Schedule s;
    s.num_m = (M + 255) / 256;
    s.num_n = (N + BN - 1) / BN;
    s.group = group;
    s.num_kb = (K + BK - 1) / BK;
    s.full_tiles = full_tiles;
    s.clusters = clusters;
    s.cluster = cluster;
    s.n_full = cluster < full_tiles ? (full_tiles - 1 - cluster) / clusters + 1 : 0;
    s.n_tail = 0;
    s.g0 = s.g1 = 0;
    const int rest = s.num_m * s.num_n - full_tiles;
    s.total = static_cast<long long>(rest) * s.num_kb;
    if (rest > 0 && (tail.mode == kTailSplitN || tail.mode == kTailSplitK)) {
        s.n_tail = cluster < 2 * rest ? 1 : 0;
    } else if (rest > 0 && tail.mode == kTailStreamK) {
        s.g0 = sk_lo(cluster, s.total, clusters);
        s.g1 = sk_lo(cluster + 1, s.total, clusters);
        s.n_tail = s.g1 > s.g0 ? static_cast<int>((s.g1 - 1) / s.num_kb - s.g0 / s.num_kb + 1) : 0;
    }
    return s;
}

template <int BN, bool SPLITK>
__device__ __forceinline__ Unit schedule_unit(const Schedule& s, int i, const TailSplit& tail) {
    Unit out = {0, 0, BN, 0, s.num_kb, -1, -1, -1};
    int t, half_n = 0;
    if (SPLITK) {
        const int u = s.cluster + i * s.clusters;
        t = u / tail.splits;
        out.tile = t;
        out.split = u % tail.splits;
        out.kb0 = out.split * s.num_kb / tail.splits;
        out.kb1 = (out.split + 1) * s.num_kb / tail.splits;
    } else if (i < s.n_full) {
        t = s.cluster + i * s.clusters;
    } else if (tail.mode == kTailSplitN) {
        t = s.full_tiles + s.cluster / 2;
        half_n = s.cluster & 1;
        out.width = BN / 2;
    } else if (tail.mode == kTailSplitK) {
        // K half (cluster & 1) of tail tile cluster / 2.
        t = s.full_tiles + s.cluster / 2;
        out.tile = s.cluster / 2;
        out.split = s.cluster & 1;
        out.kb0 = out.split * (s.num_kb / 2);
        out.kb1 = out.split ? s.num_kb : s.num_kb / 2;
    } else {
        const long long tt = s.g0 / s.num_kb + (i - s.n_full);
        const long long first_g = tt * s.num_kb;
        out.kb0 = static_cast<int>((s.g0 > first_g ? s.g0 : first_g) - first_g);
        out.kb1 = static_cast<int>((s.g1 < first_g + s.num_kb ? s.g1 : first_g + s.num_kb) - first_g);
        const int last = sk_owner(first_g + s.num_kb - 1, s.total, s.clusters);
        if (sk_owner(first_g, s.total, s.clusters) != last) out.boundary = last;
        t = s.full_tiles + static_cast<int>(tt);
    }
    const TileCoord tc = tile_coord(t, s.num_m, s.num_n, s.group);
    out.m_blk = tc.m_blk;
    out.n0 = tc.n_blk * BN + half_n * (BN / 2);
    return out;
}

// Slot schedule (cluster_n 2).  The grid is cut into slots of four CTAs
// (blocks 4s .. 4s + 3); slot s walks super tiles of 256 rows x 2 BN columns
// round-robin, and pair p of the slot (blocks 4s + 2p, 4s + 2p + 1) computes
// the BN-wide half p.  A super tile whose second half lies past N runs as two
// BN/2-wide halves of its one tile.  The last partial wave splits like
// kTailSplitN: each of its super tiles becomes two units on two slots, unit h
// covering tile 2 n + h as two BN/2-wide halves; a unit with no tile is
// dropped.  Both pairs of a slot always run the same rows of A over the same
// K blocks, which is what lets a 4-CTA cluster share A.
__device__ __forceinline__ Schedule make_slot_schedule(int M, int N, int K, int BN, int BK, int group,
                                                       int full_tiles, int slot, int slots, const TailSplit& tail) {
    Schedule s = make_schedule(M, N, K, 2 * BN, BK, group, full_tiles, slot, slots, tail);
    if (s.n_tail > 0 && (slot & 1)) {
        const TileCoord tc = tile_coord(full_tiles + slot / 2, s.num_m, s.num_n, group);
        if (2 * tc.n_blk + 1 >= (N + BN - 1) / BN) s.n_tail = 0;
    }
    return s;
}

template <int BN>
__device__ __forceinline__ Unit slot_unit(const Schedule& s, int i, int pair, int N) {
    Unit out = {0, 0, BN, 0, s.num_kb, -1, -1, -1};
    const int tiles_n = (N + BN - 1) / BN;
    if (i < s.n_full) {
        const TileCoord tc = tile_coord(s.cluster + i * s.clusters, s.num_m, s.num_n, s.group);
        out.m_blk = tc.m_blk;
        if (2 * tc.n_blk + 1 < tiles_n) {
            out.n0 = (2 * tc.n_blk + pair) * BN;
        } else {
            out.width = BN / 2;
            out.n0 = 2 * tc.n_blk * BN + pair * (BN / 2);
        }
    } else {
        const TileCoord tc = tile_coord(s.full_tiles + s.cluster / 2, s.num_m, s.num_n, s.group);
        out.m_blk = tc.m_blk;
        out.width = BN / 2;
        out.n0 = (2 * tc.n_blk + (s.cluster & 1)) * BN + pair * (BN / 2);
    }
    return out;
}

// Chunk c (32 rows x 64 FP32) of the partial at a range boundary for (CTA
// rank, lane quarter), stored as 16 float4 groups interleaved across the 32
// lanes, so that every warp-wide store and load is coalesced.
template <int BN>
__device__ __forceinline__ float4* partial_chunk(const TailSplit& tail, int boundary, int rank, int quarter, int c) {
    const size_t chunk = ((static_cast<size_t>(boundary) * 2 + rank) * 4 + quarter) * (BN / 64) + c;
    return reinterpret_cast<float4*>(tail.partials + chunk * 32 * 64);
}

__device__ __forceinline__ size_t flag_index(int boundary, int rank, int quarter) {
    return (static_cast<size_t>(boundary) * 2 + rank) * 4 + quarter;
}

// Chunk c of split `split`'s partial of `tile` for (CTA rank, lane quarter),
// in the same interleaved layout as partial_chunk.
template <int BN>
__device__ __forceinline__ float4* split_partial_chunk(const TailSplit& tail, int tile, int split, int rank,
                                                       int quarter, int c) {
    const size_t chunk =
        (((static_cast<size_t>(tile) * tail.splits + split) * 2 + rank) * 4 + quarter) * (BN / 64) + c;
    return reinterpret_cast<float4*>(tail.partials + chunk * 32 * 64);
}

// Threads of a pair kernel: the slot schedule adds two warps that exchange A
// inside a 4-CTA cluster (warp 6 sends, warp 7 relays what arrived).
template <bool SLOTS>
constexpr int pair_threads() {
    return SLOTS ? kThreads + 64 : kThreads;
}

// SPLITK instantiations run the split-K schedule (tail.mode kSplitK) and
// nothing else; the others never see it, so their code is the same as
// without split K.
// EF instantiations issue every operand load with an L2 cache policy
// (evict-first for the operands tail.evict_first names, normal for the
// other); the others issue plain loads, so the choice costs the common
// schedule nothing.
template <int BN, int BK, int STAGES, bool B_MN, bool ALLGATHER, bool SLOTS, bool SPLITK, bool EF = false>
__global__ void __launch_bounds__(pair_threads<SLOTS>(), 1)
    gemm_bf16_tcgen05_pair(const __grid_constant__ CUtensorMap map_a,
                           const __grid_constant__ CUtensorMap map_b,
                           const __grid_constant__ CUtensorMap map_b_half,
                           const __grid_constant__ CUtensorMap map_c, int M, int N, int K, int group,
                           int full_tiles, uint64_t limit_ns, int* status,
                           const __grid_constant__ PeerOutputs peers, const TailSplit tail) {
    using L = PairLayout<BN, BK, STAGES, B_MN>;
    // The A exchange splits each stage's A into its two 64-deep K halves.
    static_assert(!SLOTS || (BK == 128 && !ALLGATHER), "the slot schedule is built for BK 128, plain GEMM");
    static_assert(!SPLITK || (!SLOTS && !ALLGATHER), "split K is built for the plain pair schedule");
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarrierOffset);
    uint64_t* empty = full + STAGES;
    uint64_t* tmem_full = empty + STAGES;
    uint64_t* tmem_empty = tmem_full + 2;
    uint64_t* drain = tmem_empty + 2;
    uint64_t* partial_full = drain + 1;  // one per epilogue warp: partial landed in shared memory
    uint64_t* landed = partial_full + kEpilogueWarps;  // 4-CTA cluster: this CTA's K half of A landed
    uint64_t* fwd_in = landed + STAGES;                // 4-CTA cluster: the partner's K half of A landed
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(fwd_in + STAGES);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* no_abort = abort + 1;

    // A warp's rows of a stream-K partial (BN/64 chunks of 32 x 64 FP32) are
    // staged in the pipeline buffers when those hold all four warps' rows.
    constexpr uint32_t kPartialWarpBytes = (BN / 64) * 32 * 64 * 4;
    constexpr bool kStagePartial = L::kStagingOffset >= kEpilogueWarps * static_cast<int>(kPartialWarpBytes);
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    // The pair is cluster ranks {2q, 2q + 1} (tcgen05 pairs CTAs whose ranks
    // differ in bit 0); rank 2q leads it.  A 4-CTA cluster (slot schedule)
    // holds two pairs, and CTA r shares its rows of A with CTA r ^ 2.
    const uint32_t cta_rank = ptx::cluster_ctarank();
    const uint32_t rank = cta_rank & 1u;
    const uint32_t pair_base = cta_rank & ~1u;
    const uint32_t partner = cta_rank ^ 2u;
    const bool leader = rank == 0;
    bool quad = false;
    if constexpr (SLOTS) quad = ptx::cluster_nctarank() == 4;
    const int pair_id = SLOTS ? static_cast<int>((blockIdx.x >> 1) & 1u) : 0;
    const uint16_t pair_mask = static_cast<uint16_t>(0x3u << pair_base);
    const uint16_t stage_mask = quad ? static_cast<uint16_t>(0xF) : pair_mask;
    const Schedule sched =
        SLOTS ? make_slot_schedule(M, N, K, BN, BK, group, full_tiles, blockIdx.x / 4, gridDim.x / 4, tail)
              : make_schedule(M, N, K, BN, BK, group, full_tiles, blockIdx.x / 2, gridDim.x / 2, tail);
    auto unit_at = [&](int u) {
        return SLOTS ? slot_unit<BN>(sched, u, pair_id, N) : schedule_unit<BN, SPLITK>(sched, u, tail);
    };
    // Slots assume clusters of consecutive blocks (4s .. 4s + 3, or 2t, 2t + 1
    // when the launch fell back to pairs); anything else computes nothing and
    // reports KMCTS_EGEMM.
    bool layout_ok = true;
    if constexpr (SLOTS) layout_ok = (blockIdx.x & (quad ? 3u : 1u)) == cta_rank;
    const int num_units = layout_ok ? sched.count() : 0;

    if (threadIdx.x == 0) {
        if (!layout_ok) atomicCAS(status, 0, KMCTS_EGEMM);
        // 4-CTA cluster: the leader's full barrier also takes its own A half
        // (warp 6) and the non-leader's relay (warp 7); every empty barrier
        // both pairs' UMMA commits.
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full[s], quad ? 3 : 1);
            ptx::mbar_init(&empty[s], quad ? 2 : 1);
            ptx::mbar_init(&landed[s], 1);
            ptx::mbar_init(&fwd_in[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            ptx::mbar_init(&tmem_full[a], 1);
            ptx::mbar_init(&tmem_empty[a], 2 * kEpilogueWarps);
        }
        ptx::mbar_init(drain, 1);
        for (int w = 0; w < kEpilogueWarps; ++w) ptx::mbar_init(&partial_full[w], 1);
        *abort = 0;
        *no_abort = 0;
        ptx::fence_mbarrier_init();
    }
    if (warp == 0 && lane == 0) {
        ptx::prefetch_tensormap(&map_a);
        ptx::prefetch_tensormap(&map_b);
        ptx::prefetch_tensormap(&map_b_half);
        ptx::prefetch_tensormap(&map_c);
    }
    if (warp == 1) {
        ptx::tmem_alloc_pair(tmem_slot, L::kTmemCols);
        ptx::tmem_relinquish_pair();
    }
    __syncwarp();  // every warp meets the CTA barrier converged
    ptx::tc_fence_before();
    __syncthreads();
    ptx::cluster_sync();  // the leader's barriers exist before the peer signals them
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0, issued_phase = 0;
            bool ok = true;
            uint64_t a_policy = 0, b_policy = 0;
            if constexpr (EF) {
                b_policy = (tail.evict_first & 1) ? ptx::policy_evict_first() : ptx::policy_evict_normal();
                a_policy = (tail.evict_first & 2) ? ptx::policy_evict_first() : ptx::policy_evict_normal();
            }
            for (int u = 0; u < num_units && ok; ++u) {
                const Unit w = unit_at(u);
                const int m0 = w.m_blk * 256 + static_cast<int>(rank) * 128;
                const int b_cols = w.width / 2;  // B columns this CTA stages
                const int nb0 = w.n0 + static_cast<int>(rank) * b_cols;
                // The leader posts the pair's bytes on its full barrier: both
                // CTAs' B; and both CTAs' A, or in a 4-CTA cluster the A half
                // its partner copies in.
                const uint32_t unit_bytes = 2u * b_cols * BK * 2 + (quad ? L::kABytes / 2 : 2u * L::kABytes);
                const CUtensorMap* mb = w.width == BN ? &map_b : &map_b_half;
                for (int kb = w.kb0; kb < w.kb1; ++kb) {
                    if (!ptx::mbar_wait(&empty[stage], phase ^ 1u, limit_ns, abort)) {
                        record_failure(status, abort, kRoleProducer);
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + stage * L::kStageBytes;
                    uint8_t* sb = sa + L::kABytes;
                    if (leader) ptx::mbar_arrive_expect_tx(&full[stage], unit_bytes);
                    const uint32_t bar = ptx::mapa_shared(ptx::smem_addr(&full[stage]), pair_base);
#pragma unroll
                    for (int kh = 0; kh < BK / 64; ++kh) {
                        const int k0 = kb * BK + kh * 64;
                        if (!quad) {
                            if constexpr (EF)
                                ptx::tma_load_2d_pair_hint(sa + kh * (128 * 128), &map_a, bar, k0, m0, a_policy);
                            else
                                ptx::tma_load_2d_pair(sa + kh * (128 * 128), &map_a, bar, k0, m0);
                        } else if (kh == pair_id) {
                            // This CTA's K half of its A rows; warp 6 copies
                            // it to the partner once it lands.
                            ptx::mbar_arrive_expect_tx(&landed[stage], 128 * 128);
                            ptx::tma_load_2d(sa + kh * (128 * 128), &map_a, &landed[stage], k0, m0);
                        }
                        if constexpr (B_MN) {
                            for (int nb = 0; nb < b_cols / 64; ++nb) {
                                uint8_t* dst = sb + (kh * (L::kHalfN / 64) + nb) * 8192;
                                if constexpr (EF)
                                    ptx::tma_load_2d_pair_hint(dst, &map_b, bar, nb0 + nb * 64, k0, b_policy);
                                else
                                    ptx::tma_load_2d_pair(dst, &map_b, bar, nb0 + nb * 64, k0);
                            }
                        } else {
                            if constexpr (EF)
                                ptx::tma_load_2d_pair_hint(sb + kh * (L::kHalfN * 128), mb, bar, k0, nb0, b_policy);
                            else
                                ptx::tma_load_2d_pair(sb + kh * (L::kHalfN * 128), mb, bar, k0, nb0);
                        }
                    }
                    issued |= 1u << stage;
                    issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // Drain (leader): its full barriers count both CTAs' bytes.  In
            // a 4-CTA cluster every CTA also waits for its own A loads.
            for (int s = 0; s < STAGES; ++s) {
                if (!(issued & (1u << s))) continue;
                const uint32_t par = (issued_phase >> s) & 1u;
                if (leader && !ptx::mbar_wait(&full[s], par, drain_limit(limit_ns), no_abort))
                    record_failure(status, abort, kRoleDrain);
                if (quad && !ptx::mbar_wait(&landed[s], par, drain_limit(limit_ns), no_abort))
                    record_failure(status, abort, kRoleDrain);
            }
        }
        __syncwarp();  // lanes 1-31 wait for the producer lane before the closing barrier
    } else if (warp == 1) {
        // ----------------------------------------------------------------- MMA
        if (lane == 0 && leader) {
            constexpr uint32_t idesc_full = ptx::make_idesc_bf16(256, BN, B_MN);
            constexpr uint32_t idesc_half = ptx::make_idesc_bf16(256, BN / 2, B_MN);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            bool ok = true;
            for (int u = 0; u < num_units && ok; ++u, ++local) {
                const Unit w = unit_at(u);
                const uint32_t idesc = w.width == BN ? idesc_full : idesc_half;
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!ptx::mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, limit_ns, abort)) {
                    record_failure(status, abort, kRoleMma);
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = w.kb0; kb < w.kb1; ++kb) {
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
                        const int kh = kk / 4;
                        const int kq = kk % 4;
                        const uint64_t adesc = ptx::make_sw128_desc(sa + kh * (128 * 128) + kq * 32, 16, 1024);
                        uint64_t bdesc;
                        if constexpr (B_MN) {
                            bdesc = ptx::make_sw128_desc(sb + kh * (L::kHalfN / 64) * 8192 + kq * 2048, 8192, 1024);
                        } else {
                            bdesc = ptx::make_sw128_desc(sb + kh * (L::kHalfN * 128) + kq * 32, 16, 1024);
                        }
                        ptx::umma_bf16_pair(d_tmem, adesc, bdesc, idesc, (kb != w.kb0 || kk != 0) ? 1u : 0u);
                    }
                    ptx::umma_commit_pair(&empty[stage], stage_mask);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (ok) ptx::umma_commit_pair(&tmem_full[acc], pair_mask);
            }
            ptx::umma_commit_pair(drain, pair_mask);
        }
        __syncwarp();
    } else if (warp >= 2 + kEpilogueWarps) {
        // ---------------------------------------- A exchange (4-CTA cluster)
        // CTA x and CTA x ^ 2 (same rank in the two pairs) stage the same 128
        // rows of A; each loads one 64-deep K half per stage and copies it
        // into the other's same stage.  Leaders receive into their full
        // barrier (the producer's expected bytes include it); non-leaders
        // receive into fwd_in, and warp 7 relays "both halves here" to the
        // leader.  A copy into the partner's stage is safe once this CTA's
        // producer has loaded that stage: it loaded only after both pairs'
        // UMMAs released it, here and (same UMMAs) in the partner.  This
        // CTA's source half is free again once both pairs' UMMAs release the
        // stage: the partner pair's UMMAs read the copy, so it has landed.
        if (quad && lane == 0 && warp == 2 + kEpilogueWarps) {
            // Outgoing: copy each landed half to the partner.
            constexpr uint32_t kHalfBytes = 128 * 128;
            int stage = 0;
            uint32_t phase = 0;
            bool ok = true;
            for (int u = 0; u < num_units && ok; ++u) {
                const Unit w = unit_at(u);
                for (int kb = w.kb0; kb < w.kb1; ++kb) {
                    uint8_t* half = smem + stage * L::kStageBytes + pair_id * kHalfBytes;
                    if (!ptx::mbar_wait(&landed[stage], phase, limit_ns, abort)) {
                        record_failure(status, abort, kRoleProducer);
                        ok = false;
                        break;
                    }
                    uint64_t* dst_bar = leader ? &full[stage] : &fwd_in[stage];
                    ptx::bulk_copy_to_cta(ptx::mapa_shared(ptx::smem_addr(half), partner), half, kHalfBytes,
                                          ptx::mapa_shared(ptx::smem_addr(dst_bar), partner));
                    if (leader) ptx::mbar_arrive(&full[stage]);  // the leader's own half is here
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
        } else if (quad && !leader && lane == 0) {
            // Incoming (non-leader): once the partner's half and this CTA's
            // own half have landed, one arrival on the leader's full barrier.
            constexpr uint32_t kHalfBytes = 128 * 128;
            int stage = 0;
            uint32_t phase = 0;
            uint32_t armed = 0, armed_phase = 0;  // incoming copies expected and not yet seen
            bool ok = true;
            for (int u = 0; u < num_units && ok; ++u) {
                const Unit w = unit_at(u);
                for (int kb = w.kb0; kb < w.kb1; ++kb) {
                    ptx::mbar_arrive_expect_tx(&fwd_in[stage], kHalfBytes);
                    armed |= 1u << stage;
                    armed_phase = (armed_phase & ~(1u << stage)) | (phase << stage);
                    if (!ptx::mbar_wait(&fwd_in[stage], phase, limit_ns, abort) ||
                        !ptx::mbar_wait(&landed[stage], phase, limit_ns, abort)) {
                        record_failure(status, abort, kRoleProducer);
                        ok = false;
                        break;
                    }
                    armed &= ~(1u << stage);
                    ptx::mbar_arrive_cluster_relaxed(ptx::mapa_shared(ptx::smem_addr(&full[stage]), pair_base));
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
            }
            // Drain: no copy into this CTA may still be in flight at exit.
            for (int s = 0; s < STAGES; ++s) {
                if ((armed & (1u << s)) &&
                    !ptx::mbar_wait(&fwd_in[s], (armed_phase >> s) & 1u, drain_limit(limit_ns), no_abort))
                    record_failure(status, abort, kRoleDrain);
            }
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue
        const int quarter = warp % 4;
        uint8_t* staging = smem + L::kStagingOffset + (warp - 2) * 2 * kStagingBytes;
        int local = 0;
        int chunk_count = 0;
        for (int u = 0; u < num_units; ++u, ++local) {
            const Unit w = unit_at(u);
            const int m0 = w.m_blk * 256 + static_cast<int>(rank) * 128;
            const int n0 = w.n0;
            const int chunks = w.width / 64;
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            const bool split = w.boundary >= 0;
            int* arrival = split ? tail.arrivals + flag_index(w.boundary, static_cast<int>(rank), quarter) : nullptr;
            int* ready = split ? tail.ready + flag_index(w.boundary, static_cast<int>(rank), quarter) : nullptr;
            // A partner that has already published its partial makes this
            // segment the second; looked up while the MMAs still run.
            int published = 0;
            if (split && lane == 0) published = ptx::ld_acquire_gpu(ready) == tail.epoch;
            bool ok = ptx::mbar_wait(&tmem_full[acc], acc_phase, limit_ns, abort);
            ok = __all_sync(0xffffffffu, ok);
            bool second = false;  // stream-K: the other segment arrived first; this one writes C
            bool staged = false;  // stream-K: the partial is read from shared memory
            if (ok && split) {
                int prev = tail.epoch;
                if (lane == 0 && !published) prev = atomicExch(arrival, tail.epoch);
                second = __shfl_sync(0xffffffffu, prev, 0) == tail.epoch;
                if (second) {
                    // Wait (bounded) for the first segment's rows of the partial.
                    const uint64_t start = ptx::global_timer_ns();
                    while (ptx::ld_acquire_gpu(ready) != tail.epoch) {
                        if (*abort || ptx::global_timer_ns() - start > limit_ns) {
                            ok = false;
                            break;
                        }
                    }
                    ok = __all_sync(0xffffffffu, ok);
                    // In the cluster's last unit every MMA is done and no TMA
                    // load is left, so the pipeline stages are free: one bulk
                    // load brings this warp's rows of the partial on chip.
                    if (ok && kStagePartial && u == num_units - 1) {
                        uint8_t* dst = smem + (warp - 2) * kPartialWarpBytes;
                        if (lane == 0) {
                            ptx::fence_proxy_async_global();
                            ptx::mbar_arrive_expect_tx(&partial_full[warp - 2], kPartialWarpBytes);
                            ptx::bulk_load(dst, partial_chunk<BN>(tail, w.boundary, static_cast<int>(rank), quarter, 0),
                                           kPartialWarpBytes, &partial_full[warp - 2]);
                        }
                        ok = __all_sync(0xffffffffu, ptx::mbar_wait(&partial_full[warp - 2], 0, limit_ns, abort));
                        staged = true;
                    }
                }
            }
            if (!ok) {
                if (lane == 0) record_failure(status, abort, kRoleEpilogue);
                break;
            }
            ptx::tc_fence_after();
            const uint32_t row_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                      static_cast<uint32_t>(acc * BN);
            if constexpr (!SPLITK && !ALLGATHER && !SLOTS) {
                if (tail.mode == kTailSplitK && w.split >= 0) {
                    // K-half exchange: give the partner this half's FP32 values
                    // of its chunks, then add the partner's to this half's
                    // chunks and store them.
                    const int h = w.split;
                    const int half_chunks = chunks / 2;
                    const int give0 = (1 - h) * half_chunks, keep0 = h * half_chunks;
                    int* my_ready = tail.ready + flag_index(2 * w.tile + h, static_cast<int>(rank), quarter);
                    int* peer_ready = tail.ready + flag_index(2 * w.tile + 1 - h, static_cast<int>(rank), quarter);
#pragma unroll 1
                    for (int c = give0; c < give0 + half_chunks; ++c) {
                        uint32_t lo[32], hi[32];
                        ptx::tmem_ld_32x32b_x32(row_addr + c * 64, lo);
                        ptx::tmem_ld_32x32b_x32(row_addr + c * 64 + 32, hi);
                        ptx::tmem_wait_ld();
                        float4* part = partial_chunk<BN>(tail, w.tile, static_cast<int>(rank), quarter, c);
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            __stcg(part + q * 32 + lane,
                                   make_float4(__uint_as_float(lo[4 * q]), __uint_as_float(lo[4 * q + 1]),
                                               __uint_as_float(lo[4 * q + 2]), __uint_as_float(lo[4 * q + 3])));
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            __stcg(part + (8 + q) * 32 + lane,
                                   make_float4(__uint_as_float(hi[4 * q]), __uint_as_float(hi[4 * q + 1]),
                                               __uint_as_float(hi[4 * q + 2]), __uint_as_float(hi[4 * q + 3])));
                    }
                    __threadfence();
                    __syncwarp();
                    if (lane == 0) ptx::st_release_gpu(my_ready, tail.epoch);
                    // Wait (bounded) for the partner's values of this half's chunks.
                    bool got = true;
                    const uint64_t start = ptx::global_timer_ns();
                    while (ptx::ld_acquire_gpu(peer_ready) != tail.epoch) {
                        if (*abort || ptx::global_timer_ns() - start > limit_ns) {
                            got = false;
                            break;
                        }
                    }
                    if (!__all_sync(0xffffffffu, got)) {
                        if (lane == 0) record_failure(status, abort, kRoleEpilogue);
                        break;
                    }
#pragma unroll 1
                    for (int c = keep0; c < keep0 + half_chunks; ++c) {
                        uint32_t lo[32], hi[32];
                        ptx::tmem_ld_32x32b_x32(row_addr + c * 64, lo);
                        ptx::tmem_ld_32x32b_x32(row_addr + c * 64 + 32, hi);
                        ptx::tmem_wait_ld();
                        if (c == keep0 + half_chunks - 1) {
                            ptx::tc_fence_before();
                            __syncwarp();
                            if (lane == 0)
                                ptx::mbar_arrive_cluster(ptx::mapa_shared(ptx::smem_addr(&tmem_empty[acc]), pair_base));
                        }
                        const float4* part = partial_chunk<BN>(tail, w.tile, static_cast<int>(rank), quarter, c);
                        float4 p[16];  // all of the chunk's loads in flight at once
#pragma unroll
                        for (int q = 0; q < 16; ++q) p[q] = __ldcg(part + q * 32 + lane);
#pragma unroll
                        for (int q = 0; q < 8; ++q) {
                            lo[4 * q] = __float_as_uint(__uint_as_float(lo[4 * q]) + p[q].x);
                            lo[4 * q + 1] = __float_as_uint(__uint_as_float(lo[4 * q + 1]) + p[q].y);
                            lo[4 * q + 2] = __float_as_uint(__uint_as_float(lo[4 * q + 2]) + p[q].z);
                            lo[4 * q + 3] = __float_as_uint(__uint_as_float(lo[4 * q + 3]) + p[q].w);
                            hi[4 * q] = __float_as_uint(__uint_as_float(hi[4 * q]) + p[8 + q].x);
                            hi[4 * q + 1] = __float_as_uint(__uint_as_float(hi[4 * q + 1]) + p[8 + q].y);
                            hi[4 * q + 2] = __float_as_uint(__uint_as_float(hi[4 * q + 2]) + p[8 + q].z);
                            hi[4 * q + 3] = __float_as_uint(__uint_as_float(hi[4 * q + 3]) + p[8 + q].w);
                        }
                        store_chunk(&map_c, staging, chunk_count, lo, hi, lane, n0 + c * 64, m0 + quarter * 32);
                    }
                    // The partner's values are consumed: clear its flag, so a
                    // replay of this very launch (same epoch) starts clean.
                    __syncwarp();
                    if (lane == 0) *peer_ready = 0;
                    continue;
                }
            }
#pragma unroll 1
            for (int c = 0; c < chunks; ++c) {
                uint32_t lo[32], hi[32];
                ptx::tmem_ld_32x32b_x32(row_addr + c * 64, lo);
                ptx::tmem_ld_32x32b_x32(row_addr + c * 64 + 32, hi);
                ptx::tmem_wait_ld();
                if (c == chunks - 1) {
                    ptx::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive_cluster(ptx::mapa_shared(ptx::smem_addr(&tmem_empty[acc]), pair_base));
                }
                if (SPLITK) {
                    // Split K: store this K range's FP32 rows; the tile's last
                    // unit to arrive writes C after the loop.
                    float4* part = split_partial_chunk<BN>(tail, w.tile, w.split, static_cast<int>(rank), quarter, c);
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        __stcg(part + q * 32 + lane,
                               make_float4(__uint_as_float(lo[4 * q]), __uint_as_float(lo[4 * q + 1]),
                                           __uint_as_float(lo[4 * q + 2]), __uint_as_float(lo[4 * q + 3])));
#pragma unroll
                    for (int q = 0; q < 8; ++q)
                        __stcg(part + (8 + q) * 32 + lane,
                               make_float4(__uint_as_float(hi[4 * q]), __uint_as_float(hi[4 * q + 1]),
                                           __uint_as_float(hi[4 * q + 2]), __uint_as_float(hi[4 * q + 3])));
                    continue;
                }
                if (split) {
                    float4* part = partial_chunk<BN>(tail, w.boundary, static_cast<int>(rank), quarter, c);
                    if (!second) {
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            __stcg(part + q * 32 + lane,
                                   make_float4(__uint_as_float(lo[4 * q]), __uint_as_float(lo[4 * q + 1]),
                                               __uint_as_float(lo[4 * q + 2]), __uint_as_float(lo[4 * q + 3])));
#pragma unroll
                        for (int q = 0; q < 8; ++q)
                            __stcg(part + (8 + q) * 32 + lane,
                                   make_float4(__uint_as_float(hi[4 * q]), __uint_as_float(hi[4 * q + 1]),
                                               __uint_as_float(hi[4 * q + 2]), __uint_as_float(hi[4 * q + 3])));
                        continue;  // the second segment writes C
                    }
                    float4 p[16];  // all of the chunk's loads in flight at once
                    if (staged) {
                        const float4* sp = reinterpret_cast<const float4*>(smem + (warp - 2) * kPartialWarpBytes) +
                                           c * 16 * 32;
#pragma unroll
                        for (int q = 0; q < 16; ++q) p[q] = sp[q * 32 + lane];
                    } else {
#pragma unroll
                        for (int q = 0; q < 16; ++q) p[q] = __ldcg(part + q * 32 + lane);
                    }
#pragma unroll
                    for (int q = 0; q < 8; ++q) {
                        lo[4 * q] = __float_as_uint(__uint_as_float(lo[4 * q]) + p[q].x);
                        lo[4 * q + 1] = __float_as_uint(__uint_as_float(lo[4 * q + 1]) + p[q].y);
                        lo[4 * q + 2] = __float_as_uint(__uint_as_float(lo[4 * q + 2]) + p[q].z);
                        lo[4 * q + 3] = __float_as_uint(__uint_as_float(lo[4 * q + 3]) + p[q].w);
                        hi[4 * q] = __float_as_uint(__uint_as_float(hi[4 * q]) + p[8 + q].x);
                        hi[4 * q + 1] = __float_as_uint(__uint_as_float(hi[4 * q + 1]) + p[8 + q].y);
                        hi[4 * q + 2] = __float_as_uint(__uint_as_float(hi[4 * q + 2]) + p[8 + q].z);
                        hi[4 * q + 3] = __float_as_uint(__uint_as_float(hi[4 * q + 3]) + p[8 + q].w);
                    }
                }
                // Own C by TMA store; in a fused all-gather the same staged
                // chunk also goes to every peer's C (TMA stores over NVLink).
                store_chunk(&map_c, staging, chunk_count, lo, hi, lane, peers.col_offset + n0 + c * 64,
                            m0 + quarter * 32, ALLGATHER ? peers.map : nullptr, ALLGATHER ? peers.count : 0);
            }
            if (SPLITK) {
                // Publish this warp's rows of the partial, then count the
                // unit; the tile's last unit sums every split in split order.
                __threadfence();
                __syncwarp();
                unsigned long long* counter =
                    tail.counters + (static_cast<size_t>(w.tile) * 2 + rank) * 4 + quarter;
                int order = 0;
                if (lane == 0) order = arrive_counted(counter, tail.epoch);
                if (__shfl_sync(0xffffffffu, order, 0) == tail.splits - 1) {
                    __threadfence();
                    // In the cluster's last unit the stages are free (every
                    // MMA done, no TMA load left): each chunk's partials of
                    // every split come on chip by bulk loads, the next chunk's
                    // in flight while this one is added, instead of one
                    // dependent L2 round trip per split and chunk.
                    constexpr int kWarpStageBytes = L::kStagingOffset / kEpilogueWarps;
                    const int set_bytes = tail.splits * 8192;  // one chunk of every split
                    const bool on_chip = u == num_units - 1 && 2 * set_bytes <= kWarpStageBytes;
                    uint8_t* wbuf = smem + (warp - 2) * kWarpStageBytes;
                    auto fetch = [&](int c) {
                        if (lane == 0) {
                            uint8_t* dst = wbuf + (c & 1) * set_bytes;
                            ptx::mbar_arrive_expect_tx(&partial_full[warp - 2], static_cast<uint32_t>(set_bytes));
                            for (int j = 0; j < tail.splits; ++j)
                                ptx::bulk_load(dst + j * 8192,
                                               split_partial_chunk<BN>(tail, w.tile, j, static_cast<int>(rank), quarter, c),
                                               8192u, &partial_full[warp - 2]);
                        }
                    };
                    if (on_chip) {
                        if (lane == 0) ptx::fence_proxy_async_global();  // the partials were written by generic stores
                        fetch(0);
                    }
                    uint32_t set_phase = 0;
                    bool fine = true;
#pragma unroll 1
                    for (int c = 0; c < chunks && fine; ++c) {
                        float sum[64];
                        const float4* set = nullptr;
                        if (on_chip) {
                            fine = __all_sync(0xffffffffu,
                                              ptx::mbar_wait(&partial_full[warp - 2], set_phase, limit_ns, abort));
                            set_phase ^= 1u;
                            if (!fine) {
                                if (lane == 0) record_failure(status, abort, kRoleEpilogue);
                                break;
                            }
                            if (c + 1 < chunks) {
                                // The other buffer was last read for chunk c - 1.
                                ptx::fence_proxy_async_smem();
                                __syncwarp();
                                fetch(c + 1);
                            }
                            set = reinterpret_cast<const float4*>(wbuf + (c & 1) * set_bytes);
                        }
#pragma unroll 1
                        for (int j = 0; j < tail.splits; ++j) {
                            const float4* part =
                                on_chip ? set + j * 512
                                        : split_partial_chunk<BN>(tail, w.tile, j, static_cast<int>(rank), quarter, c);
#pragma unroll
                            for (int q = 0; q < 16; ++q) {
                                const float4 f = on_chip ? part[q * 32 + lane] : __ldcg(part + q * 32 + lane);
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
                        store_chunk(&map_c, staging, chunk_count, lo, hi, lane, peers.col_offset + n0 + c * 64,
                                    m0 + quarter * 32, ALLGATHER ? peers.map : nullptr, ALLGATHER ? peers.count : 0);
                    }
                    __syncwarp();
                    if (fine && lane == 0) *counter = 0ull;  // every unit of the tile has arrived: clear for replays
                }
            }
            if (split) {
                __syncwarp();
                if (!second) {
                    // Publish this warp's rows: every lane's stores, then one
                    // release of the ready flag.
                    __threadfence();
                    __syncwarp();
                    if (lane == 0) ptx::st_release_gpu(ready, tail.epoch);
                } else if (lane == 0) {
                    // Both segments are done with these flags: clear them, so
                    // a replay of this very launch (same epoch) starts clean.
                    *arrival = 0;
                    *ready = 0;
                }
            }
        }
        if (lane == 0) {
            // Shared memory must outlive the stores' reads of it; a fused
            // all-gather also waits for its peer writes to complete.
            if constexpr (ALLGATHER) {
                ptx::bulk_wait_group<0>();
            } else {
                ptx::bulk_wait_group_read<0>();
            }
        }
        __syncwarp();
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        // Both CTAs: every UMMA that touches this CTA's TMEM and shared memory
        // has completed (the leader's final commit arrives here in both CTAs).
        // Waited only after this CTA's epilogue finished, so the wait is short.
        if (lane == 0 && !ptx::mbar_wait(drain, 0, drain_limit(limit_ns), no_abort)) record_failure(status, abort, kRoleDrain);
        __syncwarp();
    }
    ptx::cluster_sync();  // no CTA leaves while its peer may still signal it
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc_pair(tmem_base, L::kTmemCols);
    }
}

// ------------------------------------------------------------------ host side

constexpr int kMaxDevices = 64;

// Co-resident CTA pairs of a pair kernel on the current device (cached).
template <int BN, int BK, int STAGES, bool B_MN, bool ALLGATHER = false, bool SLOTS = false>
int pair_workers(int device) {
    using L = PairLayout<BN, BK, STAGES, B_MN>;
    auto kernel = gemm_bf16_tcgen05_pair<BN, BK, STAGES, B_MN, ALLGATHER, SLOTS, false>;
    static std::mutex mu;
    static int max_clusters[kMaxDevices] = {};
    std::lock_guard<std::mutex> lock(mu);
    if (max_clusters[device] == 0) {
        if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes) != cudaSuccess)
            return -1;
        cudaLaunchConfig_t config = {};
        cudaLaunchAttribute attr[1];
        attr[0].id = cudaLaunchAttributeClusterDimension;
        attr[0].val.clusterDim.x = 2;
        attr[0].val.clusterDim.y = 1;
        attr[0].val.clusterDim.z = 1;
        config.gridDim = dim3(2 * (multiprocessor_count() / 2), 1, 1);
        config.blockDim = dim3(pair_threads<SLOTS>(), 1, 1);
        config.dynamicSmemBytes = L::kSmemBytes;
        config.attrs = attr;
        config.numAttrs = 1;
        int clusters = 0;
        if (cudaOccupancyMaxActiveClusters(&clusters, kernel, &config) != cudaSuccess || clusters <= 0) {
            cudaGetLastError();
            clusters = multiprocessor_count() / 2;
        }
        max_clusters[device] = clusters;
    }
    return max_clusters[device];
}

// Which tail split a schedule asks for (the flags), before the shape decides
// whether the tail can split at all.
int requested_tail(int flags) {
    if (flags & KMCTS_FLAG_NO_TAIL_SPLIT) return KMCTS_TAIL_NONE;
    if (flags & KMCTS_FLAG_TAIL_STREAM_K) return KMCTS_TAIL_STREAM_K;
    if (flags & KMCTS_FLAG_TAIL_SPLIT_K) return KMCTS_TAIL_SPLIT_K;
    return KMCTS_TAIL_SPLIT_N;
}

// Work units of the stream-K tiles over p clusters (host copy of the
// kernel's range arithmetic).
int stream_k_units(long long total, int num_kb, int p) {
    int units = 0;
    for (int c = 0; c < p; ++c) {
        const long long g0 = static_cast<long long>(c) * total / p, g1 = static_cast<long long>(c + 1) * total / p;
        if (g1 > g0) units += static_cast<int>((g1 - 1) / num_kb - g0 / num_kb + 1);
    }
    return units;
}

// The launch shape: how many pairs run, which tiles run whole, and how the
// tiles of the last partial wave are shared.
template <int BN, int BK>
kmcts_gemm_plan make_pair_plan(int M, int N, int K, int workers, bool persistent, int tail, int k_splits,
                               int64_t smem) {
    kmcts_gemm_plan plan = {};
    plan.kernel = 2;
    plan.cluster_size = 2;
    plan.workers = workers;
    plan.tiles = ((M + 255) / 256) * ((N + BN - 1) / BN);
    plan.full_tiles = plan.tiles;
    plan.units = plan.tiles;
    plan.k_splits = 1;
    const int num_kb_all = (K + BK - 1) / BK;
    const int splits = k_splits < num_kb_all ? k_splits : num_kb_all;
    if (splits > 1) {
        // Split K: every tile as `splits` K ranges, dealt like whole tiles;
        // full_tiles counts the units.
        plan.k_splits = splits;
        plan.units = plan.tiles * splits;
        plan.full_tiles = plan.units;
        const int clusters = persistent && plan.units > workers ? workers : plan.units;
        plan.ctas = 2 * clusters;
        plan.smem_bytes = static_cast<int32_t>(smem);
        return plan;
    }
    int clusters = plan.tiles;
    if (persistent) {
        clusters = plan.tiles < workers ? plan.tiles : workers;
        const int rem = plan.tiles % workers;
        const int num_kb = (K + BK - 1) / BK;
        if (rem != 0 && tail == KMCTS_TAIL_STREAM_K && plan.tiles > workers) {
            // The last full wave and the partial one, shared by all W pairs.
            plan.tail_split = KMCTS_TAIL_STREAM_K;
            plan.full_tiles = (plan.tiles / workers - 1) * workers;
            plan.tail_clusters = workers;
            plan.tail_segments = 2;
            const long long total = static_cast<long long>(plan.tiles - plan.full_tiles) * num_kb;
            plan.units = plan.full_tiles + stream_k_units(total, num_kb, workers);
            clusters = workers;
        } else if (rem != 0 && tail == KMCTS_TAIL_SPLIT_K && BN == 256 && 2 * rem <= workers && num_kb >= 2) {
            // Each tail tile as its two K halves on two clusters.
            plan.tail_split = KMCTS_TAIL_SPLIT_K;
            plan.tail_clusters = 2 * rem;
            plan.tail_segments = 2;
            plan.full_tiles = plan.tiles - rem;
            plan.units = plan.full_tiles + 2 * rem;
            clusters = plan.units < workers ? plan.units : workers;
        } else if (rem != 0 && tail != KMCTS_TAIL_NONE && BN == 256 && 2 * rem <= workers) {
            // Half-width units: BN/2 must be whole 64-column TMA boxes per CTA.
            plan.tail_split = KMCTS_TAIL_SPLIT_N;
            plan.tail_clusters = 2 * rem;
            plan.tail_segments = 1;
            plan.full_tiles = plan.tiles - rem;
            plan.units = plan.full_tiles + 2 * rem;
            clusters = plan.units < workers ? plan.units : workers;
        }
    }
    plan.ctas = 2 * clusters;
    plan.smem_bytes = static_cast<int32_t>(smem);
    return plan;
}

// Slot schedule (cluster_n 2): `slots` groups of four CTAs, each walking
// super tiles of 256 x 2 BN; the last partial wave splits as in the pair
// plan (stream-K requests take the N split).  Host copy of the kernel's
// make_slot_schedule.
template <int BN, int BK>
kmcts_gemm_plan make_slot_plan(int M, int N, int K, int slots, bool persistent, int tail, int group, int64_t smem) {
    kmcts_gemm_plan plan = {};
    plan.kernel = 2;
    plan.cluster_size = 4;
    plan.workers = slots;
    const int num_m = (M + 255) / 256, num_sn = (N + 2 * BN - 1) / (2 * BN), tiles_n = (N + BN - 1) / BN;
    plan.tiles = num_m * num_sn;
    plan.full_tiles = plan.tiles;
    plan.units = plan.tiles;
    int used = plan.tiles;
    if (persistent) {
        used = plan.tiles < slots ? plan.tiles : slots;
        const int rem = plan.tiles % slots;
        if (rem != 0 && tail != KMCTS_TAIL_NONE && 2 * rem <= slots) {
            plan.tail_split = KMCTS_TAIL_SPLIT_N;
            plan.full_tiles = plan.tiles - rem;
            plan.tail_clusters = 2 * rem;
            plan.tail_segments = 1;
            // Two units per tail super tile, one when it holds a single tile.
            plan.units = plan.full_tiles;
            for (int t = plan.full_tiles; t < plan.tiles; ++t)
                plan.units += 2 * tile_coord(t, num_m, num_sn, group).n_blk + 1 < tiles_n ? 2 : 1;
            used = 2 * rem > used ? 2 * rem : used;
        }
    }
    plan.ctas = 4 * used;
    plan.smem_bytes = static_cast<int32_t>(smem);
    plan.k_splits = 1;
    return plan;
}

template <int BN, int BK, int STAGES, bool B_MN, bool ALLGATHER = false, bool SLOTS = false>
int plan_pair_variant(int M, int N, int K, bool persistent, int tail, int group, int k_splits, kmcts_gemm_plan* out) {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return KMCTS_EHANDLE;
    const int workers = pair_workers<BN, BK, STAGES, B_MN, ALLGATHER, SLOTS>(device);
    if (workers <= 0) return KMCTS_EGEMM;
    constexpr int64_t smem = PairLayout<BN, BK, STAGES, B_MN>::kSmemBytes;
    if constexpr (SLOTS) {
        if (workers < 2) return KMCTS_EGEMM;
        (void)k_splits;
        *out = make_slot_plan<BN, BK>(M, N, K, workers / 2, persistent, tail, group, smem);
    } else {
        (void)group;
        *out = make_pair_plan<BN, BK>(M, N, K, workers, persistent, tail, ALLGATHER ? 0 : k_splits, smem);
    }
    return KMCTS_OK;
}

// FP32 partials and flags of stream-K tiles: one partial slot per range
// boundary (W - 1 at most, sized for W = SMs / 2), then the ready and arrival
// flags, in the stream's workspace.
constexpr size_t kPartialSlotBytes = 2 * 4 * (256 / 64) * 32 * 64 * sizeof(float);  // one 256 x 256 FP32 tile

bool tail_workspace(cudaStream_t stream, int boundaries, TailSplit* out) {
    const size_t slots = static_cast<size_t>(multiprocessor_count() / 2 + 1);
    if (static_cast<size_t>(boundaries) > slots) return false;
    const size_t flag_ints = slots * 2 * 4;
    void* base = nullptr;
    int epoch = 0;
    if (!stream_workspace(stream, kWorkspaceStreamK, slots * kPartialSlotBytes + 2 * flag_ints * sizeof(int), &base,
                          &epoch))
        return false;
    out->partials = static_cast<float*>(base);
    out->ready = reinterpret_cast<int*>(static_cast<char*>(base) + slots * kPartialSlotBytes);
    out->arrivals = out->ready + flag_ints;
    out->epoch = epoch;
    return true;
}

// Split K: the FP32 partials of every (tile, split) and the tiles' counters,
// in the stream's split-K workspace.
template <int BN>
bool split_workspace(cudaStream_t stream, int tiles, int splits, TailSplit* out) {
    const size_t counter_bytes = static_cast<size_t>(tiles) * 2 * 4 * sizeof(unsigned long long);
    const size_t partial_bytes = static_cast<size_t>(tiles) * splits * 2 * 4 * (BN / 64) * 32 * 64 * sizeof(float);
    void* base = nullptr;
    int epoch = 0;
    if (!stream_workspace(stream, kWorkspaceSplitK, counter_bytes + partial_bytes, &base, &epoch)) return false;
    out->counters = static_cast<unsigned long long*>(base);
    out->partials = reinterpret_cast<float*>(static_cast<char*>(base) + counter_bytes);
    out->splits = splits;
    out->epoch = epoch;
    return true;
}

// The shared-memory opt-in of a split-K or cache-hinted instantiation (per
// device, once); its occupancy is the plain one's (same shared memory and
// block).
template <int BN, int BK, int STAGES, bool B_MN, bool SPLITK, bool EF>
bool plain_smem_configured() {
    static std::mutex mu;
    static bool done[kMaxDevices] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return false;
    std::lock_guard<std::mutex> lock(mu);
    if (!done[device]) {
        if (cudaFuncSetAttribute(gemm_bf16_tcgen05_pair<BN, BK, STAGES, B_MN, false, false, SPLITK, EF>,
                                 cudaFuncAttributeMaxDynamicSharedMemorySize,
                                 PairLayout<BN, BK, STAGES, B_MN>::kSmemBytes) != cudaSuccess)
            return false;
        done[device] = true;
    }
    return true;
}

template <int BN, int BK, int STAGES, bool B_MN, bool ALLGATHER = false, bool SLOTS = false>
int launch_pair_variant_peers(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb_half,
                              const CUtensorMap& mc, int M, int N, int K, int group, bool persistent, int tail_req,
                              int k_splits, int evict_first, uint64_t limit_ns, cudaStream_t stream, int* status,
                              const PeerOutputs& peers) {
    using L = PairLayout<BN, BK, STAGES, B_MN>;
    if (status == nullptr) status = default_status_ptr();
    if (status == nullptr) return KMCTS_EGEMM;
    kmcts_gemm_plan plan;
    int rc = plan_pair_variant<BN, BK, STAGES, B_MN, ALLGATHER, SLOTS>(M, N, K, persistent, tail_req, group, k_splits,
                                                                       &plan);
    if (rc != KMCTS_OK) return rc;
    TailSplit tail = {};
    if (plan.k_splits > 1 && !split_workspace<BN>(stream, plan.tiles, plan.k_splits, &tail)) {
        // No workspace (out of memory, or growth under graph capture): unsplit.
        rc = plan_pair_variant<BN, BK, STAGES, B_MN, ALLGATHER, SLOTS>(M, N, K, persistent, tail_req, group, 0, &plan);
        if (rc != KMCTS_OK) return rc;
    }
    if (plan.tail_split == KMCTS_TAIL_STREAM_K && !tail_workspace(stream, plan.tail_clusters, &tail)) {
        // No workspace: the bit-identical N split (or whole tiles) instead.
        rc = plan_pair_variant<BN, BK, STAGES, B_MN, ALLGATHER, SLOTS>(M, N, K, persistent, KMCTS_TAIL_SPLIT_N,
                                                                       group, 0, &plan);
        if (rc != KMCTS_OK) return rc;
    }
    if (plan.tail_split == KMCTS_TAIL_SPLIT_K && !tail_workspace(stream, plan.tail_clusters, &tail)) {
        // No workspace: the N split, bit-identical to whole tiles.
        rc = plan_pair_variant<BN, BK, STAGES, B_MN, ALLGATHER, SLOTS>(M, N, K, persistent, KMCTS_TAIL_SPLIT_N,
                                                                       group, 0, &plan);
        if (rc != KMCTS_OK) return rc;
    }
    tail.evict_first = evict_first;
    tail.mode = plan.k_splits > 1                           ? kSplitK
                : plan.tail_split == KMCTS_TAIL_STREAM_K ? kTailStreamK
                : plan.tail_split == KMCTS_TAIL_SPLIT_K  ? kTailSplitK
                : plan.tail_split == KMCTS_TAIL_SPLIT_N  ? kTailSplitN
                                                         : kTailWhole;
    cudaLaunchConfig_t config = {};
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    // Slots: 4-CTA clusters where the GPCs hold them, pairs on the SMs left
    // over (the kernel reads which it got from %cluster_nctarank).
    attr[1].id = cudaLaunchAttributePreferredClusterDimension;
    attr[1].val.preferredClusterDim.x = 4;
    attr[1].val.preferredClusterDim.y = 1;
    attr[1].val.preferredClusterDim.z = 1;
    config.gridDim = dim3(plan.ctas, 1, 1);
    config.blockDim = dim3(pair_threads<SLOTS>(), 1, 1);
    config.dynamicSmemBytes = L::kSmemBytes;
    config.stream = stream;
    config.attrs = attr;
    config.numAttrs = SLOTS ? 2 : 1;
    cudaError_t err;
    if constexpr (!SLOTS && !ALLGATHER) {
        // Split K, and cache-hinted loads, run their own instantiations.
        const bool split = tail.mode == kSplitK;
        if (split || evict_first) {
            bool configured = false;
            if (split && evict_first) {
                configured = plain_smem_configured<BN, BK, STAGES, B_MN, true, true>();
                if (configured)
                    err = cudaLaunchKernelEx(&config, gemm_bf16_tcgen05_pair<BN, BK, STAGES, B_MN, false, false, true, true>,
                                             ma, mb, mb_half, mc, M, N, K, group, plan.full_tiles, limit_ns, status,
                                             peers, tail);
            } else if (split) {
                configured = plain_smem_configured<BN, BK, STAGES, B_MN, true, false>();
                if (configured)
                    err = cudaLaunchKernelEx(&config, gemm_bf16_tcgen05_pair<BN, BK, STAGES, B_MN, false, false, true, false>,
                                             ma, mb, mb_half, mc, M, N, K, group, plan.full_tiles, limit_ns, status,
                                             peers, tail);
            } else {
                configured = plain_smem_configured<BN, BK, STAGES, B_MN, false, true>();
                if (configured)
                    err = cudaLaunchKernelEx(&config, gemm_bf16_tcgen05_pair<BN, BK, STAGES, B_MN, false, false, false, true>,
                                             ma, mb, mb_half, mc, M, N, K, group, plan.full_tiles, limit_ns, status,
                                             peers, tail);
            }
            if (!configured) return KMCTS_EGEMM;
            g_launches.fetch_add(1, std::memory_order_relaxed);
            return err == cudaSuccess ? KMCTS_OK : KMCTS_EGEMM;
        }
    }
    err = cudaLaunchKernelEx(&config, gemm_bf16_tcgen05_pair<BN, BK, STAGES, B_MN, ALLGATHER, SLOTS, false>, ma, mb,
                             mb_half, mc, M, N, K, group, plan.full_tiles, limit_ns, status, peers, tail);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return err == cudaSuccess ? KMCTS_OK : KMCTS_EGEMM;
}

template <int BN, int BK, int STAGES, bool B_MN, bool SLOTS>
int launch_pair_variant(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb_half,
                        const CUtensorMap& mc, int M, int N, int K, int group, bool persistent, int tail_req,
                        int k_splits, int evict_first, uint64_t limit_ns, cudaStream_t stream, int* status) {
    const PeerOutputs none = {};
    return launch_pair_variant_peers<BN, BK, STAGES, B_MN, false, SLOTS>(ma, mb, mb_half, mc, M, N, K, group,
                                                                         persistent, tail_req, k_splits, evict_first,
                                                                         limit_ns, stream, status, none);
}

template <int BN, int BK, int STAGES, bool B_MN, bool SLOTS>
int plan_variant(int M, int N, int K, bool persistent, int tail, int group, int k_splits, kmcts_gemm_plan* out) {
    return plan_pair_variant<BN, BK, STAGES, B_MN, false, SLOTS>(M, N, K, persistent, tail, group, k_splits, out);
}

using PairLauncher = int (*)(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, int,
                             int, int, int, bool, int, int, int, uint64_t, cudaStream_t, int*);

using PairPlanner = int (*)(int, int, int, bool, int, int, int, kmcts_gemm_plan*);

struct PairVariant {
    int bn, bk, stages, b_mn, slots;
    PairLauncher fn;
    PairPlanner plan;
};

#define KMCTS_PAIR(BN, BK, ST, MN) \
    {BN, BK, ST, MN, 0, &launch_pair_variant<BN, BK, ST, MN, false>, &plan_variant<BN, BK, ST, MN, false>}
#define KMCTS_SLOTS(BN, BK, ST, MN) \
    {BN, BK, ST, MN, 1, &launch_pair_variant<BN, BK, ST, MN, true>, &plan_variant<BN, BK, ST, MN, true>}

// Every pair schedule of the sweep grid that fits 227 KB:
// stages * (128 + BN/2) * BK * 2 + 32 KB staging + 2 KB.
const PairVariant kPairVariants[] = {
    KMCTS_PAIR(256, 64, 3, false),  KMCTS_PAIR(256, 64, 4, false),  KMCTS_PAIR(256, 64, 5, false),
    KMCTS_PAIR(256, 64, 6, false),  KMCTS_PAIR(256, 128, 3, false), KMCTS_PAIR(128, 64, 3, false),
    KMCTS_PAIR(128, 64, 4, false),  KMCTS_PAIR(128, 64, 5, false),  KMCTS_PAIR(128, 64, 6, false),
    KMCTS_PAIR(128, 128, 3, false), KMCTS_PAIR(128, 128, 4, false),
    KMCTS_PAIR(256, 64, 3, true),   KMCTS_PAIR(256, 64, 4, true),   KMCTS_PAIR(256, 64, 5, true),
    KMCTS_PAIR(256, 64, 6, true),   KMCTS_PAIR(256, 128, 3, true),  KMCTS_PAIR(128, 64, 3, true),
    KMCTS_PAIR(128, 64, 4, true),   KMCTS_PAIR(128, 64, 5, true),   KMCTS_PAIR(128, 64, 6, true),
    KMCTS_PAIR(128, 128, 3, true),  KMCTS_PAIR(128, 128, 4, true),
    // cluster_n 2: two pairs per slot sharing A (BK 128: one 64-deep K half each).
    KMCTS_SLOTS(256, 128, 3, false), KMCTS_SLOTS(256, 128, 3, true),
};

}  // namespace

namespace {

const PairVariant* find_pair_variant(const kmcts_gemm_config& cfg, int b_layout) {
    const int mn = b_layout == KMCTS_B_ROW ? 1 : 0;
    const int slots = cfg.cluster_n == 2 ? 1 : 0;
    for (const PairVariant& v : kPairVariants) {
        if (v.bn == cfg.tile_n && v.bk == cfg.tile_k && v.stages == cfg.stages && v.b_mn == mn && v.slots == slots)
            return &v;
    }
    return nullptr;
}

}  // namespace

bool pair_variant_exists(const kmcts_gemm_config& cfg, int b_layout) {
    return find_pair_variant(cfg, b_layout) != nullptr;
}

int64_t pair_smem_bytes(int bn, int bk, int stages) {
    return static_cast<int64_t>(stages) * (128 + bn / 2) * bk * 2 + kEpilogueWarps * 2 * kStagingBytes +
           kSmemReserve;
}

int plan_pair(const kmcts_gemm_config& cfg, int M, int N, int K, int b_layout, kmcts_gemm_plan* out) {
    const PairVariant* v = find_pair_variant(cfg, b_layout);
    if (!v) return KMCTS_ENOTSUP;
    return v->plan(M, N, K, cfg.persistent != 0, requested_tail(cfg.flags), cfg.raster_group, cfg.k_splits, out);
}

int launch_pair_allgather(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb_half,
                          const CUtensorMap& mc, int M, int N_shard, int K, int b_layout,
                          const kmcts_gemm_config& cfg, uint64_t limit_ns, cudaStream_t stream, int* status,
                          void* const* peer_c, int peer_count, int ld, int col_offset) {
    if (cfg.tile_n != 256 || cfg.tile_k != 128 || cfg.stages != 3 || peer_count < 0 ||
        peer_count > KMCTS_MAX_RANKS - 1)
        return KMCTS_ENOTSUP;
    PeerOutputs peers = {};
    for (int p = 0; p < peer_count; ++p) {
        if (!encode_tensor_map_2d(&peers.map[p], peer_c[p], ld, M, static_cast<uint64_t>(ld) * 2, 64, 32))
            return KMCTS_EINVAL;
    }
    peers.count = peer_count;
    peers.col_offset = col_offset;
    // Only the N split: every output stays one full-K chain, so each rank's
    // columns are bit-identical to the single-GPU kernel on the full problem.
    const int split = requested_tail(cfg.flags) == KMCTS_TAIL_NONE ? KMCTS_TAIL_NONE : KMCTS_TAIL_SPLIT_N;
    if (b_layout == KMCTS_B_ROW)
        return launch_pair_variant_peers<256, 128, 3, true, true>(ma, mb, mb_half, mc, M, N_shard, K,
                                                                  cfg.raster_group, cfg.persistent != 0, split, 0,
                                                                  0, limit_ns, stream, status, peers);
    return launch_pair_variant_peers<256, 128, 3, false, true>(ma, mb, mb_half, mc, M, N_shard, K, cfg.raster_group,
                                                               cfg.persistent != 0, split, 0, 0, limit_ns, stream,
                                                               status, peers);
}

int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb_half, const CUtensorMap& mc,
                int M, int N, int K, int b_layout, const kmcts_gemm_config& cfg, uint64_t limit_ns,
                cudaStream_t stream, int* status) {
    const PairVariant* v = find_pair_variant(cfg, b_layout);
    if (!v) return KMCTS_ENOTSUP;
    return v->fn(ma, mb, mb_half, mc, M, N, K, cfg.raster_group, cfg.persistent != 0, requested_tail(cfg.flags),
                 cfg.k_splits,
                 ((cfg.flags & KMCTS_FLAG_B_EVICT_FIRST) ? 1 : 0) | ((cfg.flags & KMCTS_FLAG_A_EVICT_FIRST) ? 2 : 0),
                 limit_ns, stream, status);
}

}  // namespace kmcts
