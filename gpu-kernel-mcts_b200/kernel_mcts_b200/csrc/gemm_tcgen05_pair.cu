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
// Every wait is bounded; see gemm_tcgen05.cu for the failure protocol.
#include <cstring>
#include <mutex>

#include "gemm_common.cuh"
#include "kmcts_internal.h"

namespace kmcts {

extern __device__ int g_default_status;

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

// Work units.  Tiles [0, full_tiles) (in raster order) run whole; each later
// tile runs as two BN/2-wide halves, so a last partial wave of R <= W/2 tiles
// costs half a tile of time instead of a whole one.  Every output element is
// still one full-K UMMA chain: splitting changes no result bit.
struct Unit {
    int m_blk, n0, width;
};

template <int BN>
__device__ __forceinline__ Unit pair_unit(int u, int full_tiles, int num_m, int num_n, int group) {
    int t = u, half = 0, width = BN;
    if (u >= full_tiles) {
        const int v = u - full_tiles;
        t = full_tiles + v / 2;
        half = v & 1;
        width = BN / 2;
    }
    const TileCoord tc = tile_coord(t, num_m, num_n, group);
    return {tc.m_blk, tc.n_blk * BN + half * (BN / 2), width};
}

template <int BN, int BK, int STAGES, bool B_MN, bool ALLGATHER>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tcgen05_pair(const __grid_constant__ CUtensorMap map_a,
                           const __grid_constant__ CUtensorMap map_b,
                           const __grid_constant__ CUtensorMap map_b_half,
                           const __grid_constant__ CUtensorMap map_c, int M, int N, int K, int group,
                           int full_tiles, uint64_t limit_ns, int* status,
                           const __grid_constant__ PeerOutputs peers) {
    using L = PairLayout<BN, BK, STAGES, B_MN>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) &
                                               ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarrierOffset);
    uint64_t* empty = full + STAGES;
    uint64_t* tmem_full = empty + STAGES;
    uint64_t* tmem_empty = tmem_full + 2;
    uint64_t* drain = tmem_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* no_abort = abort + 1;

    if (status == nullptr) status = &g_default_status;
    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const uint32_t rank = ptx::cluster_ctarank();
    const bool leader = rank == 0;
    const int cluster_id = blockIdx.x / 2;
    const int num_clusters = gridDim.x / 2;
    const int num_m = (M + 255) / 256;
    const int num_n = (N + BN - 1) / BN;
    const int num_tiles = num_m * num_n;
    const int num_units = full_tiles + 2 * (num_tiles - full_tiles);
    const int num_kb = (K + BK - 1) / BK;

    if (threadIdx.x == 0) {
        for (int s = 0; s < STAGES; ++s) {
            ptx::mbar_init(&full[s], 1);
            ptx::mbar_init(&empty[s], 1);
        }
        for (int a = 0; a < 2; ++a) {
            ptx::mbar_init(&tmem_full[a], 1);
            ptx::mbar_init(&tmem_empty[a], 2 * kEpilogueWarps);
        }
        ptx::mbar_init(drain, 1);
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
            for (int u = cluster_id; u < num_units && ok; u += num_clusters) {
                const Unit w = pair_unit<BN>(u, full_tiles, num_m, num_n, group);
                const int m0 = w.m_blk * 256 + static_cast<int>(rank) * 128;
                const int b_cols = w.width / 2;  // B columns this CTA stages
                const int nb0 = w.n0 + static_cast<int>(rank) * b_cols;
                const uint32_t unit_bytes = 2u * (L::kABytes + b_cols * BK * 2);
                const CUtensorMap* mb = w.width == BN ? &map_b : &map_b_half;
                for (int kb = 0; kb < num_kb; ++kb) {
                    if (!ptx::mbar_wait(&empty[stage], phase ^ 1u, limit_ns, abort)) {
                        record_failure(status, abort, kRoleProducer);
                        ok = false;
                        break;
                    }
                    uint8_t* sa = smem + stage * L::kStageBytes;
                    uint8_t* sb = sa + L::kABytes;
                    if (leader) ptx::mbar_arrive_expect_tx(&full[stage], unit_bytes);
                    const uint32_t bar = ptx::mapa_shared(ptx::smem_addr(&full[stage]), 0);
#pragma unroll
                    for (int kh = 0; kh < BK / 64; ++kh) {
                        const int k0 = kb * BK + kh * 64;
                        ptx::tma_load_2d_pair(sa + kh * (128 * 128), &map_a, bar, k0, m0);
                        if constexpr (B_MN) {
                            for (int nb = 0; nb < b_cols / 64; ++nb) {
                                ptx::tma_load_2d_pair(sb + (kh * (L::kHalfN / 64) + nb) * 8192, &map_b, bar,
                                                      nb0 + nb * 64, k0);
                            }
                        } else {
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
            // Drain (leader): its full barriers count both CTAs' bytes.
            if (leader) {
                for (int s = 0; s < STAGES; ++s) {
                    if ((issued & (1u << s)) &&
                        !ptx::mbar_wait(&full[s], (issued_phase >> s) & 1u, drain_limit(limit_ns), no_abort)) {
                        record_failure(status, abort, kRoleDrain);
                    }
                }
            }
        }
    } else if (warp == 1) {
        // ----------------------------------------------------------------- MMA
        if (lane == 0 && leader) {
            constexpr uint32_t idesc_full = ptx::make_idesc_bf16(256, BN, B_MN);
            constexpr uint32_t idesc_half = ptx::make_idesc_bf16(256, BN / 2, B_MN);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            bool ok = true;
            for (int u = cluster_id; u < num_units && ok; u += num_clusters, ++local) {
                const uint32_t idesc = u < full_tiles ? idesc_full : idesc_half;
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!ptx::mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, limit_ns, abort)) {
                    record_failure(status, abort, kRoleMma);
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * BN;
                for (int kb = 0; kb < num_kb; ++kb) {
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
                        ptx::umma_bf16_pair(d_tmem, adesc, bdesc, idesc, (kb | kk) != 0 ? 1u : 0u);
                    }
                    ptx::umma_commit_pair(&empty[stage], 0x3);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (ok) ptx::umma_commit_pair(&tmem_full[acc], 0x3);
            }
            ptx::umma_commit_pair(drain, 0x3);
        }
        __syncwarp();
    } else {
        // ------------------------------------------------------------ epilogue
        const int quarter = warp % 4;
        uint8_t* staging = smem + L::kStagingOffset + (warp - 2) * 2 * kStagingBytes;
        int local = 0;
        int chunk_count = 0;
        for (int u = cluster_id; u < num_units; u += num_clusters, ++local) {
            const Unit w = pair_unit<BN>(u, full_tiles, num_m, num_n, group);
            const int m0 = w.m_blk * 256 + static_cast<int>(rank) * 128;
            const int n0 = w.n0;
            const int chunks = w.width / 64;
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            bool ok = ptx::mbar_wait(&tmem_full[acc], acc_phase, limit_ns, abort);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0) record_failure(status, abort, kRoleEpilogue);
                break;
            }
            ptx::tc_fence_after();
            const uint32_t row_addr = tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) +
                                      static_cast<uint32_t>(acc * BN);
#pragma unroll 1
            for (int c = 0; c < chunks; ++c) {
                uint32_t lo[32], hi[32];
                ptx::tmem_ld_32x32b_x32(row_addr + c * 64, lo);
                ptx::tmem_ld_32x32b_x32(row_addr + c * 64 + 32, hi);
                ptx::tmem_wait_ld();
                if (c == chunks - 1) {
                    ptx::tc_fence_before();
                    __syncwarp();
                    if (lane == 0) ptx::mbar_arrive_cluster(ptx::mapa_shared(ptx::smem_addr(&tmem_empty[acc]), 0));
                }
                // Own C by TMA store; in a fused all-gather the same staged
                // chunk also goes to every peer's C (TMA stores over NVLink).
                store_chunk(&map_c, staging, chunk_count, lo, hi, lane, peers.col_offset + n0 + c * 64,
                            m0 + quarter * 32, ALLGATHER ? peers.map : nullptr, ALLGATHER ? peers.count : 0);
            }
        }
        if (lane == 0) ptx::bulk_wait_group<0>();  // own and peer stores complete before the grid ends
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
template <int BN, int BK, int STAGES, bool B_MN, bool ALLGATHER = false>
int pair_workers(int device) {
    using L = PairLayout<BN, BK, STAGES, B_MN>;
    auto kernel = gemm_bf16_tcgen05_pair<BN, BK, STAGES, B_MN, ALLGATHER>;
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
        config.blockDim = dim3(kThreads, 1, 1);
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

// The launch shape: how many pairs run, and which tiles run whole.
template <int BN>
kmcts_gemm_plan make_pair_plan(int M, int N, int workers, bool persistent, bool split_tail, int64_t smem) {
    kmcts_gemm_plan plan = {};
    plan.kernel = 2;
    plan.cluster_size = 2;
    plan.workers = workers;
    plan.tiles = ((M + 255) / 256) * ((N + BN - 1) / BN);
    plan.full_tiles = plan.tiles;
    plan.units = plan.tiles;
    int clusters = plan.tiles;
    if (persistent) {
        // Split the last partial wave into half-width units when it fits in
        // one round of half units (2R <= W); half tiles need BN/2 to be a
        // whole number of 64-column TMA boxes per CTA for row-major B.
        const int rem = plan.tiles % workers;
        const bool can_split = split_tail && BN == 256 && rem != 0 && 2 * rem <= workers;
        plan.full_tiles = can_split ? plan.tiles - rem : plan.tiles;
        plan.units = plan.full_tiles + 2 * (plan.tiles - plan.full_tiles);
        clusters = plan.units < workers ? plan.units : workers;
    }
    plan.ctas = 2 * clusters;
    plan.smem_bytes = static_cast<int32_t>(smem);
    return plan;
}

template <int BN, int BK, int STAGES, bool B_MN, bool ALLGATHER = false>
int plan_pair_variant(int M, int N, bool persistent, bool split_tail, kmcts_gemm_plan* out) {
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return KMCTS_EHANDLE;
    const int workers = pair_workers<BN, BK, STAGES, B_MN, ALLGATHER>(device);
    if (workers <= 0) return KMCTS_EGEMM;
    *out = make_pair_plan<BN>(M, N, workers, persistent, split_tail, PairLayout<BN, BK, STAGES, B_MN>::kSmemBytes);
    return KMCTS_OK;
}

template <int BN, int BK, int STAGES, bool B_MN, bool ALLGATHER = false>
int launch_pair_variant_peers(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb_half,
                              const CUtensorMap& mc, int M, int N, int K, int group, bool persistent,
                              bool split_tail, uint64_t limit_ns, cudaStream_t stream, int* status,
                              const PeerOutputs& peers) {
    using L = PairLayout<BN, BK, STAGES, B_MN>;
    kmcts_gemm_plan plan;
    const int rc = plan_pair_variant<BN, BK, STAGES, B_MN, ALLGATHER>(M, N, persistent, split_tail, &plan);
    if (rc != KMCTS_OK) return rc;
    cudaLaunchConfig_t config = {};
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = 2;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    config.gridDim = dim3(plan.ctas, 1, 1);
    config.blockDim = dim3(kThreads, 1, 1);
    config.dynamicSmemBytes = L::kSmemBytes;
    config.stream = stream;
    config.attrs = attr;
    config.numAttrs = 1;
    const cudaError_t err = cudaLaunchKernelEx(&config, gemm_bf16_tcgen05_pair<BN, BK, STAGES, B_MN, ALLGATHER>,
                                               ma, mb, mb_half, mc, M, N, K, group, plan.full_tiles, limit_ns,
                                               status, peers);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return err == cudaSuccess ? KMCTS_OK : KMCTS_EGEMM;
}

template <int BN, int BK, int STAGES, bool B_MN>
int launch_pair_variant(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb_half,
                        const CUtensorMap& mc, int M, int N, int K, int group, bool persistent, bool split_tail,
                        uint64_t limit_ns, cudaStream_t stream, int* status) {
    const PeerOutputs none = {};
    return launch_pair_variant_peers<BN, BK, STAGES, B_MN, false>(ma, mb, mb_half, mc, M, N, K, group, persistent,
                                                                  split_tail, limit_ns, stream, status, none);
}

using PairLauncher = int (*)(const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, const CUtensorMap&, int,
                             int, int, int, bool, bool, uint64_t, cudaStream_t, int*);

using PairPlanner = int (*)(int, int, bool, bool, kmcts_gemm_plan*);

struct PairVariant {
    int bn, bk, stages, b_mn;
    PairLauncher fn;
    PairPlanner plan;
};

#define KMCTS_PAIR(BN, BK, ST, MN) \
    {BN, BK, ST, MN, &launch_pair_variant<BN, BK, ST, MN>, &plan_pair_variant<BN, BK, ST, MN>}

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
};

}  // namespace

bool pair_variant_exists(int bn, int bk, int stages, int b_layout) {
    const int mn = b_layout == KMCTS_B_ROW ? 1 : 0;
    for (const PairVariant& v : kPairVariants) {
        if (v.bn == bn && v.bk == bk && v.stages == stages && v.b_mn == mn) return true;
    }
    return false;
}

int64_t pair_smem_bytes(int bn, int bk, int stages) {
    return static_cast<int64_t>(stages) * (128 + bn / 2) * bk * 2 + kEpilogueWarps * 2 * kStagingBytes +
           kSmemReserve;
}

int plan_pair(const kmcts_gemm_config& cfg, int M, int N, int b_layout, kmcts_gemm_plan* out) {
    const int mn = b_layout == KMCTS_B_ROW ? 1 : 0;
    for (const PairVariant& v : kPairVariants) {
        if (v.bn == cfg.tile_n && v.bk == cfg.tile_k && v.stages == cfg.stages && v.b_mn == mn) {
            return v.plan(M, N, cfg.persistent != 0, (cfg.flags & KMCTS_FLAG_NO_TAIL_SPLIT) == 0, out);
        }
    }
    return KMCTS_ENOTSUP;
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
    const bool split = (cfg.flags & KMCTS_FLAG_NO_TAIL_SPLIT) == 0;
    if (b_layout == KMCTS_B_ROW)
        return launch_pair_variant_peers<256, 128, 3, true, true>(ma, mb, mb_half, mc, M, N_shard, K,
                                                                  cfg.raster_group, cfg.persistent != 0, split,
                                                                  limit_ns, stream, status, peers);
    return launch_pair_variant_peers<256, 128, 3, false, true>(ma, mb, mb_half, mc, M, N_shard, K, cfg.raster_group,
                                                               cfg.persistent != 0, split, limit_ns, stream, status,
                                                               peers);
}

int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb_half, const CUtensorMap& mc,
                int M, int N, int K, int b_layout, const kmcts_gemm_config& cfg, uint64_t limit_ns,
                cudaStream_t stream, int* status) {
    const int mn = b_layout == KMCTS_B_ROW ? 1 : 0;
    for (const PairVariant& v : kPairVariants) {
        if (v.bn == cfg.tile_n && v.bk == cfg.tile_k && v.stages == cfg.stages && v.b_mn == mn) {
            return v.fn(ma, mb, mb_half, mc, M, N, K, cfg.raster_group, cfg.persistent != 0,
                        (cfg.flags & KMCTS_FLAG_NO_TAIL_SPLIT) == 0, limit_ns, stream, status);
        }
    }
    return KMCTS_ENOTSUP;
}

}  // namespace kmcts
