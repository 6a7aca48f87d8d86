// Skinny BF16 GEMMs (M <= 32) on sm_100a: C^T = B^T · A^T on the tensor
// cores, with B streamed once through every SM.
//
// For M <= 32 the work is reading B (K x N BF16, every byte once); the MMA is
// nearly free.  The 1-CTA kernel computes 128 MMA rows of which M are real and
// holds each pipeline stage for the whole padded MMA.  Here the operands swap
// roles: B's 128-column tile is the UMMA's 128-row operand (M = 128 over N)
// and A's rows are its N (16 or 32), so no tensor work is padding, the MMA
// releases each stage after a few dozen cycles, and shared memory holds ten
// 20 KB stages in flight.
//
// Work split: S units per 128-column tile (S = SMs / tiles, at most 8; 1 when
// the tiles alone fill the SMs), unit s taking the tile's K blocks s, s + S,
// s + 2S, ...  Every CTA thus reads the same band of B's rows at the same
// time (one front down K): the rows' DRAM pages are read whole while open,
// instead of piece by piece at different times.  Cutting K into contiguous
// ranges instead (one per SM, stream-K style) spread the CTAs over the whole
// matrix and measured 30% slower than this.  With S > 1 each unit stores an
// FP32 partial and the unit that arrives last on the tile's counter sums the
// S partials in unit order (deterministic) and writes C.  Nothing waits on
// another CTA: the last arrival only reads partials already published.
//
// Per CTA, 192 threads: warp 0 TMA producer (B tiles at L2 evict-first
// priority: they are read once), warp 1 MMA issuer (one lane), warps 2-5
// epilogue (tcgen05.ld of their 32 TMEM lanes = 32 columns of C).  Every wait
// is bounded; on timeout the kernel records KMCTS_ETIMEOUT in *status, drains
// its own copies and MMAs, frees TMEM and returns.  No TMA multicast.
#include <cuda_bf16.h>

#include <cstring>
#include <mutex>

#include "gemm_common.cuh"
#include "kmcts_internal.h"

namespace kmcts {
namespace {

using namespace gemm;

constexpr int kTileN = 128;  // columns of C (rows of B^T) per tile: the UMMA's M
constexpr int kARows = 32;   // rows of A staged per stage (M <= 32)
constexpr int kAccCols = 32; // TMEM columns per accumulator (the UMMA's N <= 32)
constexpr int kMaxDevices = 64;

template <int BK, int STAGES>
struct StreamLayout {
    static constexpr int kBBytes = kTileN * BK * 2;  // B^T tile
    static constexpr int kABytes = kARows * BK * 2;  // A tile
    static constexpr int kStageBytes = kBBytes + kABytes;
    static constexpr int kBarrierOffset = STAGES * kStageBytes;
    static constexpr int kSmemBytes = kBarrierOffset + kSmemReserve;
    static_assert(BK == 64 || BK == 128, "BK must be 64 or 128");
    static_assert(kStageBytes % 1024 == 0, "stages must keep 1024-byte alignment");
    static_assert(kSmemBytes <= kMaxSmem, "shared memory budget exceeded");
};

// The work split: `units` = tiles * splits; unit u is K-interleaved split
// u % splits of tile u / splits.
struct StreamSplit {
    int kbs;            // K blocks per tile
    int splits;         // units per tile (S)
    int units;          // tiles * splits
    float* partials;    // [tile][split][128 lanes][32 columns], FP32 (splits > 1)
    unsigned long long* counters;  // [tile][4 lane quarters]: epoch << 32 | units arrived
    int epoch;
};

template <int BK, int STAGES, bool B_MN, int NU>
__global__ void __launch_bounds__(kThreads, 1)
    gemm_bf16_tcgen05_stream(const __grid_constant__ CUtensorMap map_bt, const __grid_constant__ CUtensorMap map_a,
                             __nv_bfloat16* __restrict__ C, int M, int N, uint64_t limit_ns, int* status,
                             const StreamSplit sp) {
    using L = StreamLayout<BK, STAGES>;
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L::kBarrierOffset);
    uint64_t* empty = full + STAGES;
    uint64_t* tmem_full = empty + STAGES;
    uint64_t* tmem_empty = tmem_full + 2;
    uint64_t* drain = tmem_empty + 2;
    uint32_t* tmem_slot = reinterpret_cast<uint32_t*>(drain + 1);
    volatile int* abort = reinterpret_cast<volatile int*>(tmem_slot + 1);
    volatile int* no_abort = abort + 1;

    const int warp = threadIdx.x / 32;
    const int lane = threadIdx.x % 32;
    const int kbs = sp.kbs;
    const int splits = sp.splits;

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
        *abort = 0;
        *no_abort = 0;
        ptx::fence_mbarrier_init();
    }
    if (warp == 0 && lane == 0) {
        ptx::prefetch_tensormap(&map_bt);
        ptx::prefetch_tensormap(&map_a);
    }
    if (warp == 1) {
        ptx::tmem_alloc(tmem_slot, 2 * kAccCols);
        ptx::tmem_relinquish();
    }
    __syncwarp();  // every warp meets the CTA barrier converged
    ptx::tc_fence_before();
    __syncthreads();
    ptx::tc_fence_after();
    const uint32_t tmem_base = *tmem_slot;

    if (warp == 0) {
        // ------------------------------------------------------------ producer
        if (lane == 0) {
            const uint64_t b_policy = ptx::policy_evict_first();
            int stage = 0;
            uint32_t phase = 0;
            uint32_t issued = 0, issued_phase = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < sp.units && ok; u += gridDim.x)
            for (int kb = u % splits; kb < kbs; kb += splits) {
                const int n0 = (u / splits) * kTileN;
                if (!ptx::mbar_wait(&empty[stage], phase ^ 1u, limit_ns, abort)) {
                    record_failure(status, abort, kRoleProducer);
                    ok = false;
                    break;
                }
                uint8_t* sb = smem + stage * L::kStageBytes;
                uint8_t* sa = sb + L::kBBytes;
                ptx::mbar_arrive_expect_tx(&full[stage], L::kStageBytes);
#pragma unroll
                for (int kh = 0; kh < BK / 64; ++kh) {
                    const int k0 = kb * BK + kh * 64;
                    if constexpr (B_MN) {
                        // Row-major B: two 64-column boxes of 64 K rows each.
                        ptx::tma_load_2d_hint(sb + (kh * 2) * 8192, &map_bt, &full[stage], n0, k0, b_policy);
                        ptx::tma_load_2d_hint(sb + (kh * 2 + 1) * 8192, &map_bt, &full[stage], n0 + 64, k0, b_policy);
                    } else {
                        // Column-major B: 128 columns of 64 contiguous K each.
                        ptx::tma_load_2d_hint(sb + kh * (kTileN * 128), &map_bt, &full[stage], k0, n0, b_policy);
                    }
                    ptx::tma_load_2d(sa + kh * (kARows * 128), &map_a, &full[stage], k0, 0);
                }
                issued |= 1u << stage;
                issued_phase = (issued_phase & ~(1u << stage)) | (phase << stage);
                if (++stage == STAGES) {
                    stage = 0;
                    phase ^= 1u;
                }
            }
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
            // D^T[n, m] = B^T[n, k] · A^T[k, m]: A operand B^T (K-major for a
            // column-major B, MN-major for a row-major one), B operand A (K-major).
            constexpr uint32_t idesc = ptx::make_idesc_bf16_ab(kTileN, NU, B_MN, false);
            int stage = 0;
            uint32_t phase = 0;
            int local = 0;
            bool ok = true;
            for (int u = blockIdx.x; u < sp.units && ok; u += gridDim.x, ++local) {
                const int kb0 = u % splits;
                const int acc = local & 1;
                const uint32_t acc_phase = (local >> 1) & 1;
                if (!ptx::mbar_wait(&tmem_empty[acc], acc_phase ^ 1u, limit_ns, abort)) {
                    record_failure(status, abort, kRoleMma);
                    break;
                }
                ptx::tc_fence_after();
                const uint32_t d_tmem = tmem_base + acc * kAccCols;
                for (int kb = kb0; kb < kbs; kb += splits) {
                    if (!ptx::mbar_wait(&full[stage], phase, limit_ns, abort)) {
                        record_failure(status, abort, kRoleMma);
                        ok = false;
                        break;
                    }
                    ptx::tc_fence_after();
                    const uint32_t sb = ptx::smem_addr(smem + stage * L::kStageBytes);
                    const uint32_t sa = sb + L::kBBytes;
#pragma unroll
                    for (int kk = 0; kk < BK / 16; ++kk) {
                        const int kh = kk / 4;  // which 64-deep K half of the stage
                        const int kq = kk % 4;  // 16-deep step inside it
                        uint64_t bt_desc;
                        if constexpr (B_MN) {
                            bt_desc = ptx::make_sw128_desc(sb + kh * 2 * 8192 + kq * 2048, 8192, 1024);
                        } else {
                            bt_desc = ptx::make_sw128_desc(sb + kh * (kTileN * 128) + kq * 32, 16, 1024);
                        }
                        const uint64_t a_desc = ptx::make_sw128_desc(sa + kh * (kARows * 128) + kq * 32, 16, 1024);
                        ptx::umma_bf16(d_tmem, bt_desc, a_desc, idesc, (kb != kb0 || kk != 0) ? 1u : 0u);
                    }
                    ptx::umma_commit(&empty[stage]);
                    if (++stage == STAGES) {
                        stage = 0;
                        phase ^= 1u;
                    }
                }
                if (ok) ptx::umma_commit(&tmem_full[acc]);
            }
            ptx::umma_commit(drain);
            if (!ptx::mbar_wait(drain, 0, drain_limit(limit_ns), no_abort)) {
                record_failure(status, abort, kRoleDrain);
            }
        }
        __syncwarp();  // lanes 1-31 wait for the MMA lane before the closing barrier
    } else {
        // ------------------------------------------------------------ epilogue
        const int quarter = warp % 4;  // TMEM lanes (C columns) this warp may access
        int local = 0;
        for (int u = blockIdx.x; u < sp.units; u += gridDim.x, ++local) {
            const int t = u / splits, split = u % splits;
            const int acc = local & 1;
            const uint32_t acc_phase = (local >> 1) & 1;
            bool ok = ptx::mbar_wait(&tmem_full[acc], acc_phase, limit_ns, abort);
            ok = __all_sync(0xffffffffu, ok);
            if (!ok) {
                if (lane == 0) record_failure(status, abort, kRoleEpilogue);
                break;
            }
            ptx::tc_fence_after();
            uint32_t r[32];
            ptx::tmem_ld_32x32b_x32(tmem_base + (static_cast<uint32_t>(quarter * 32) << 16) + acc * kAccCols, r);
            ptx::tmem_wait_ld();
            ptx::tc_fence_before();
            __syncwarp();
            if (lane == 0) ptx::mbar_arrive(&tmem_empty[acc]);

            const int n = t * kTileN + quarter * 32 + lane;
            if (splits > 1) {
                // Publish this unit's partial (NU FP32 values of this lane's
                // C column), then count it; the unit that arrives last sums
                // the tile's partials in split order and writes C.
                float4* slot = reinterpret_cast<float4*>(
                    sp.partials + ((static_cast<size_t>(t) * splits + split) * kTileN + quarter * 32 + lane) * kAccCols);
#pragma unroll
                for (int q = 0; q < NU / 4; ++q)
                    __stcg(slot + q, make_float4(__uint_as_float(r[4 * q]), __uint_as_float(r[4 * q + 1]),
                                                 __uint_as_float(r[4 * q + 2]), __uint_as_float(r[4 * q + 3])));
                __threadfence();
                __syncwarp();
                unsigned long long* counter = sp.counters + static_cast<size_t>(t) * 4 + quarter;
                int order = 0;
                if (lane == 0) order = arrive_counted(counter, sp.epoch);
                if (__shfl_sync(0xffffffffu, order, 0) != splits - 1) continue;
                __threadfence();
                float sum[NU];
#pragma unroll 1
                for (int j = 0; j < splits; ++j) {
                    const float4* part = reinterpret_cast<const float4*>(
                        sp.partials + ((static_cast<size_t>(t) * splits + j) * kTileN + quarter * 32 + lane) * kAccCols);
#pragma unroll
                    for (int q = 0; q < NU / 4; ++q) {
                        const float4 f = __ldcg(part + q);
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
#pragma unroll
                for (int m = 0; m < NU; ++m) r[m] = __float_as_uint(sum[m]);
                __syncwarp();
                if (lane == 0) *counter = 0ull;  // every unit of the tile has arrived: clear for the next launch
            }
            if (n < N) {
#pragma unroll
                for (int m = 0; m < NU; ++m)
                    if (m < M) C[static_cast<size_t>(m) * N + n] = __float2bfloat16_rn(__uint_as_float(r[m]));
            }
        }
    }

    ptx::tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        ptx::tc_fence_after();
        ptx::tmem_dealloc(tmem_base, 2 * kAccCols);
    }
}

// ------------------------------------------------------------------ host side

// Units per tile: enough to give every SM one (at most 8, each at least
// four K blocks deep); 1 once the tiles alone fill the SMs.
int stream_splits(int tiles, int kbs, int sms) {
    int splits = tiles < sms ? sms / tiles : 1;
    if (splits > 8) splits = 8;
    if (splits > kbs / 4) splits = kbs / 4;
    return splits < 1 ? 1 : splits;
}

template <int BK, int STAGES, bool B_MN, int NU>
int launch_stream_variant(const CUtensorMap& mbt, const CUtensorMap& ma, void* C, int M, int N, int K,
                          uint64_t limit_ns, cudaStream_t stream, int* status) {
    using L = StreamLayout<BK, STAGES>;
    auto kernel = gemm_bf16_tcgen05_stream<BK, STAGES, B_MN, NU>;
    static std::mutex mu;
    static bool configured[kMaxDevices] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return KMCTS_EHANDLE;
    {
        std::lock_guard<std::mutex> lock(mu);
        if (!configured[device]) {
            if (cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, L::kSmemBytes) !=
                cudaSuccess)
                return KMCTS_EGEMM;
            configured[device] = true;
        }
    }
    const int tiles = (N + kTileN - 1) / kTileN;
    const int sms = multiprocessor_count();
    StreamSplit sp = {};
    sp.kbs = (K + BK - 1) / BK;
    sp.splits = stream_splits(tiles, sp.kbs, sms);
    if (sp.splits > 1) {
        const size_t counter_bytes = static_cast<size_t>(tiles) * 4 * sizeof(unsigned long long);
        const size_t partial_bytes = static_cast<size_t>(tiles) * sp.splits * kTileN * kAccCols * sizeof(float);
        void* base = nullptr;
        int epoch = 0;
        if (stream_workspace(stream, kWorkspaceSplitK, counter_bytes + partial_bytes, &base, &epoch)) {
            sp.counters = static_cast<unsigned long long*>(base);
            sp.partials = reinterpret_cast<float*>(static_cast<char*>(base) + counter_bytes);
            sp.epoch = epoch;
        } else {
            sp.splits = 1;  // no workspace (out of memory, or growth under graph capture): whole tiles
        }
    }
    sp.units = tiles * sp.splits;
    const int grid = sp.units < sms ? sp.units : sms;
    kernel<<<grid, kThreads, L::kSmemBytes, stream>>>(mbt, ma, static_cast<__nv_bfloat16*>(C), M, N, limit_ns,
                                                      status, sp);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError() == cudaSuccess ? KMCTS_OK : KMCTS_EGEMM;
}

using StreamLauncher = int (*)(const CUtensorMap&, const CUtensorMap&, void*, int, int, int, uint64_t, cudaStream_t,
                               int*);

struct StreamVariant {
    int bk, stages, b_mn, nu;
    StreamLauncher fn;
};

#define KMCTS_STREAM(BK, ST, MN, NU) {BK, ST, MN, NU, &launch_stream_variant<BK, ST, MN, NU>}

const StreamVariant kStreamVariants[] = {
    KMCTS_STREAM(64, 10, false, 16),  KMCTS_STREAM(64, 10, false, 32),  KMCTS_STREAM(64, 10, true, 16),
    KMCTS_STREAM(64, 10, true, 32),   KMCTS_STREAM(128, 5, false, 16),  KMCTS_STREAM(128, 5, false, 32),
    KMCTS_STREAM(128, 5, true, 16),   KMCTS_STREAM(128, 5, true, 32),
};

const StreamVariant* find_stream_variant(const kmcts_gemm_config& cfg, int M, int b_layout) {
    const int nu = M <= 16 ? 16 : 32;
    for (const StreamVariant& v : kStreamVariants) {
        if (v.bk == cfg.tile_k && v.stages == cfg.stages && v.b_mn == (b_layout == KMCTS_B_ROW ? 1 : 0) && v.nu == nu)
            return &v;
    }
    return nullptr;
}

}  // namespace

bool stream_variant_exists(const kmcts_gemm_config& cfg, int b_layout) {
    return find_stream_variant(cfg, 16, b_layout) != nullptr;
}

int64_t stream_smem_bytes(int bk, int stages) {
    return static_cast<int64_t>(stages) * (kTileN + kARows) * bk * 2 + kSmemReserve;
}

int plan_stream(const kmcts_gemm_config& cfg, int M, int N, int K, kmcts_gemm_plan* out) {
    kmcts_gemm_plan plan = {};
    plan.kernel = 3;
    plan.cluster_size = 1;
    plan.workers = multiprocessor_count();
    plan.tiles = (N + kTileN - 1) / kTileN;
    plan.k_splits = stream_splits(plan.tiles, (K + cfg.tile_k - 1) / cfg.tile_k, plan.workers);
    plan.units = plan.tiles * plan.k_splits;
    plan.full_tiles = plan.k_splits == 1 ? plan.tiles : 0;
    plan.ctas = plan.units < plan.workers ? plan.units : plan.workers;
    plan.smem_bytes = static_cast<int32_t>(stream_smem_bytes(cfg.tile_k, cfg.stages));
    (void)M;
    *out = plan;
    return KMCTS_OK;
}

int launch_stream(const void* A, const void* B, void* C, int M, int N, int K, int b_layout,
                  const kmcts_gemm_config& cfg, uint64_t limit_ns, cudaStream_t stream, int* device_status) {
    const StreamVariant* v = find_stream_variant(cfg, M, b_layout);
    if (v == nullptr) return KMCTS_ENOTSUP;
    CUtensorMap mbt, ma;
    bool ok;
    if (b_layout == KMCTS_B_COL) {
        ok = encode_tensor_map_2d(&mbt, B, K, N, static_cast<uint64_t>(K) * 2, 64, kTileN);
    } else {
        ok = encode_tensor_map_2d(&mbt, B, N, K, static_cast<uint64_t>(N) * 2, 64, 64);
    }
    ok = ok && encode_tensor_map_2d(&ma, A, K, M, static_cast<uint64_t>(K) * 2, 64, kARows);
    if (!ok) return KMCTS_EINVAL;
    return v->fn(mbt, ma, C, M, N, K, limit_ns, stream, device_status);
}

}  // namespace kmcts
