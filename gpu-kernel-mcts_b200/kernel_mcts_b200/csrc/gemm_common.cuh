// Pieces shared by the 1-CTA and CTA-pair tcgen05 GEMM kernels.
#pragma once

#include <cuda_bf16.h>

#include <cstdint>

#include "kmcts_gemm.h"
#include "ptx_sm100.cuh"

namespace kmcts {
namespace gemm {

constexpr int kThreads = 192;        // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int kEpilogueWarps = 4;
constexpr int kStagingBytes = 32 * 128;  // one warp's 32 rows x 64 BF16 columns
constexpr int kSmemReserve = 2048;       // barriers + 1024-byte alignment slack
constexpr int kMaxSmem = 232448;         // 227 KB opt-in per CTA
constexpr uint64_t kDefaultWaitNs = 2000000000ull;

// Drains (waiting for this CTA's own in-flight copies and MMAs before it
// frees TMEM and exits) never use a shorter bound than the default, whatever
// limit the caller set for the main-loop waits.
__device__ __forceinline__ uint64_t drain_limit(uint64_t limit_ns) {
    return limit_ns > kDefaultWaitNs ? limit_ns : kDefaultWaitNs;
}

// Status word: low byte KMCTS_ETIMEOUT, next byte the role that gave up.
constexpr int kRoleProducer = 1, kRoleMma = 2, kRoleEpilogue = 3, kRoleDrain = 4;

struct TileCoord {
    int m_blk, n_blk;
};

// Grouped rasterisation: tiles walk `group` M-blocks down a column strip
// before moving right, so concurrently running CTAs share A and B panels in L2.
__host__ __device__ __forceinline__ TileCoord tile_coord(int t, int num_m, int num_n, int group) {
    const int per_group = group * num_n;
    const int g = t / per_group;
    const int first_m = g * group;
    const int rows = num_m - first_m < group ? num_m - first_m : group;
    const int r = t - g * per_group;
    return {first_m + r % rows, r / rows};
}

__device__ __forceinline__ void record_failure(int* status, volatile int* abort, int role) {
    *abort = 1;
    atomicCAS(status, 0, KMCTS_ETIMEOUT | (role << 8));
}

// Two FP32 accumulator bit patterns -> packed BF16x2, round-to-nearest-even.
__device__ __forceinline__ uint32_t pack_bf16x2(uint32_t lo_bits, uint32_t hi_bits) {
    __nv_bfloat162 v = __floats2bfloat162_rn(__uint_as_float(lo_bits), __uint_as_float(hi_bits));
    return *reinterpret_cast<uint32_t*>(&v);
}

// One epilogue warp writes a 32-row x 64-column BF16 chunk (this lane's row,
// 64 FP32 values in lo[0..31], hi[0..31]) into a 128-byte-swizzled staging
// buffer and TMA-stores it at (col0, row0) of C, and of each of `extra_count`
// further tensors (the peers' C in a fused all-gather).  Two staging buffers
// per warp alternate; the wait keeps at most one group of stores reading each.
__device__ __forceinline__ void store_chunk(const CUtensorMap* map_c, uint8_t* staging, int& chunk_count,
                                            const uint32_t (&lo)[32], const uint32_t (&hi)[32], int lane,
                                            int col0, int row0, const CUtensorMap* extra_maps = nullptr,
                                            int extra_count = 0) {
    uint32_t packed[32];
#pragma unroll
    for (int i = 0; i < 16; ++i) packed[i] = pack_bf16x2(lo[2 * i], lo[2 * i + 1]);
#pragma unroll
    for (int i = 0; i < 16; ++i) packed[16 + i] = pack_bf16x2(hi[2 * i], hi[2 * i + 1]);
    uint8_t* buf = staging + (chunk_count & 1) * kStagingBytes;
    if (lane == 0) ptx::bulk_wait_group_read<1>();
    __syncwarp();
    uint8_t* row = buf + lane * 128;
#pragma unroll
    for (int j = 0; j < 8; ++j) {
        const int phys = j ^ (lane & 7);  // SW128: 16-byte chunk XOR row-in-8
        *reinterpret_cast<uint4*>(row + phys * 16) =
            make_uint4(packed[4 * j], packed[4 * j + 1], packed[4 * j + 2], packed[4 * j + 3]);
    }
    ptx::fence_proxy_async_smem();
    __syncwarp();
    if (lane == 0) {
        ptx::tma_store_2d(map_c, buf, col0, row0);
        for (int i = 0; i < extra_count; ++i) ptx::tma_store_2d(&extra_maps[i], buf, col0, row0);
        ptx::bulk_commit_group();
    }
    ++chunk_count;
}

// Split K: counts one arrival on an epoch-tagged counter (epoch << 32 |
// units arrived) and returns how many units arrived before this one in this
// launch.  A counter left by an earlier launch counts as zero.
__device__ __forceinline__ int arrive_counted(unsigned long long* counter, int epoch) {
    const unsigned long long tag = static_cast<unsigned long long>(static_cast<unsigned>(epoch)) << 32;
    unsigned long long old = *reinterpret_cast<volatile unsigned long long*>(counter);
    while (true) {
        const bool same = (old >> 32) == static_cast<unsigned>(epoch);
        const unsigned long long next = same ? old + 1 : (tag | 1ull);
        const unsigned long long seen = atomicCAS(counter, old, next);
        if (seen == old) return same ? static_cast<int>(old & 0xffffffffull) : 0;
        old = seen;  // another unit arrived in between: retry on its value
    }
}

constexpr uint32_t tmem_columns_for(int cols) {
    return cols <= 32 ? 32 : cols <= 64 ? 64 : cols <= 128 ? 128 : cols <= 256 ? 256 : 512;
}

}  // namespace gemm
}  // namespace kmcts
