// extern "C" entry points of libkmcts_gemm_sm100.so (declared in include/kmcts_gemm.h).
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>
#include <random>

#include "kmcts_internal.h"

namespace kmcts {

std::atomic<int64_t> g_launches{0};

namespace {

PFN_cuTensorMapEncodeTiled_v12000 tensor_map_encoder() {
    static std::once_flag once;
    static PFN_cuTensorMapEncodeTiled_v12000 fn = nullptr;
    std::call_once(once, [] {
        void* entry = nullptr;
        cudaDriverEntryPointQueryResult query;
        if (cudaGetDriverEntryPointByVersion("cuTensorMapEncodeTiled", &entry, 12000,
                                             cudaEnableDefault, &query) == cudaSuccess &&
            query == cudaDriverEntryPointSuccess) {
            fn = reinterpret_cast<PFN_cuTensorMapEncodeTiled_v12000>(entry);
        }
    });
    return fn;
}

cudaStream_t as_stream(void* stream) { return static_cast<cudaStream_t>(stream); }

}  // namespace

bool encode_tensor_map_2d(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                          uint64_t row_stride_bytes, uint32_t box0, uint32_t box1) {
    auto encode = tensor_map_encoder();
    if (!encode) return false;
    const cuuint64_t dims[2] = {dim0, dim1};
    const cuuint64_t strides[1] = {row_stride_bytes};
    const cuuint32_t box[2] = {box0, box1};
    const cuuint32_t element_strides[2] = {1, 1};
    return encode(map, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims,
                  strides, box, element_strides, CU_TENSOR_MAP_INTERLEAVE_NONE,
                  CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
                  CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

int multiprocessor_count() {
    static int cached[64] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return 148;
    if (device >= 0 && device < 64 && cached[device] > 0) return cached[device];
    int count = 0;
    if (cudaDeviceGetAttribute(&count, cudaDevAttrMultiProcessorCount, device) != cudaSuccess ||
        count <= 0)
        count = 148;
    if (device >= 0 && device < 64) cached[device] = count;
    return count;
}

}  // namespace kmcts

using namespace kmcts;

extern "C" {

int kmcts_default_config(kmcts_gemm_config* cfg) {
    if (!cfg) return KMCTS_EINVAL;
    std::memset(cfg, 0, sizeof(*cfg));
    // CTA pair, 256 x 256 tile, BK 128, 3 stages: the fastest schedule of the
    // sweep at 4096^3 on B200 (ties cuBLAS; see the profiles directory).
    cfg->tile_m = 256;
    cfg->tile_n = 256;
    cfg->tile_k = 128;
    cfg->stages = 3;
    cfg->cluster_m = 2;
    cfg->cluster_n = 1;
    cfg->persistent = 1;
    cfg->raster_group = 8;
    cfg->kernel = KMCTS_KERNEL_AUTO;
    cfg->wait_limit_ns = 0;
    return KMCTS_OK;
}

namespace {

// K splits for `tiles` one-CTA tiles over K: as many as keep every unit in
// one wave (SMs / tiles), at most 16 (the last unit to arrive reads every
// split's FP32 partial), and at least sixteen 128-deep K blocks per unit.
// Measured on B200 (L2 flushed): the best split count fills one wave and no
// more, e.g. 4096 x 512 x 16384 (128 tiles) 77 us unsplit against 89 with two
// splits and 148 with eight; 2048 x 256 x 8192 (32 tiles) 27.8 us with four
// against 40 unsplit and 39.9 with eight; 128 x 128 x 65536 (one tile) best at
// 16 (46 us; 52 at 8, 59 at 32); shorter units lose (512 x 512 x 8192: 24.8 us
// with four splits, 26.6 with eight).  0 = no split.
int choose_splits(long long tiles, int K, int sms) {
    const int num_kb = (K + 127) / 128;
    if (tiles <= 0 || tiles >= sms || num_kb < 32) return 0;
    long long splits = sms / tiles;
    if (splits > 16) splits = 16;
    if (splits > num_kb / 16) splits = num_kb / 16;
    return splits >= 2 ? static_cast<int>(splits) : 0;
}

// Resident clusters of `splits` one-CTA-per-SM CTAs as the occupancy
// calculator placed them on a 148-SM B200 (GPC by GPC), for when it cannot
// be asked (no device): 74, 45, 33, 26, 22, 15, 15 for 2..8.
int fallback_cluster_capacity(int splits, int sms) {
    static const int kB200[9] = {0, 148, 74, 45, 33, 26, 22, 15, 15};
    return splits >= 1 && splits <= 8 ? kB200[splits] * sms / 148 : 0;
}

// Few 128 x 128 tiles over a long K: each tile as S K ranges on one cluster
// whose CTAs add up one share of the tile each (KMCTS_FLAG_SPLIT_SCATTER).
// S is the most splits that keep every unit on its own SM, every cluster
// resident at once, and K ranges of at least 512 (at most 8); two splits
// only from K = 4096 (below, the exchange costs more than the second SM
// saves: 1024 x 1024 x 2048 18.5 us against 17.4 unsplit).  Ranges of at
// most 1024 take 64-deep x 4 stages (the copies received past them), longer
// ones 128-deep x 3.  Measured, L2 flushed (workspace split -> scatter,
// cuBLAS): 512 x 512 x 8192 25.3 -> 21.7 us (18.1), 384 x 384 x 8192 24.9 ->
// 20.3 (18.0), 256 x 512 x 16384 30.9 -> 23.6 (23.6), 1024 x 1024 x 8192
// 32.0 -> 29.9 (25.0), 2048 x 256 x 8192 26.7 -> 23.8 (21.3), 128 x 2048 x
// 8192 26.7 -> 22.6 (19.7), and unsplit before: 300 x 1000 x 2048 18.5 ->
// 16.3 (10.9), 200 x 600 x 3000 28.4 -> 16.5 (12.2).  Returns false when no
// split fits.
bool scatter_schedule(long long tiles, int K, int b_layout, int sms, kmcts_gemm_config* cfg) {
    if (tiles <= 0 || 2 * tiles > sms) return false;
    int s = static_cast<int>(sms / tiles);
    if (s > 8) s = 8;
    const int max_by_k = K / 512;
    if (s > max_by_k) s = max_by_k;
    for (; s >= 2; --s) {
        if (s == 2 && K < 4096) break;
        // Where eight clusters' worth do not fit (16-24 tiles), five splits
        // beat six (L2 flushed, means of 120: 512 x 512 x 8192 20.6 us
        // against 21.0, 256 x 1024 x 8192 21.0 against 22.1, 128 x 2048 x 8192
        // 21.9 against 22.9).
        if (s == 6 || s == 7) continue;
        kmcts_gemm_config c = *cfg;
        c.tile_m = 128;
        c.tile_n = 128;
        c.k_splits = s;
        c.flags |= KMCTS_FLAG_SPLIT_CLUSTER | KMCTS_FLAG_SPLIT_SCATTER;
        const bool shallow = K / s <= 1024;
        c.tile_k = shallow ? 64 : 128;
        c.stages = shallow ? 4 : 3;
        int capacity = cluster_capacity(c, b_layout, s);
        if (capacity <= 0) capacity = fallback_cluster_capacity(s, sms);
        if (tiles <= capacity && cluster_split_fits(c, b_layout, s)) {
            *cfg = c;
            return true;
        }
    }
    return false;
}

// M <= 64 (tiles staging 32 or 64 rows of A, 128 columns wide, one tile
// row), K >= 4096: the tile's K splits as one cluster, as many as keep every
// unit on its own SM, every cluster resident and K ranges of at least 512
// (at most 8), added up by the scatter form (two splits of 32-row tiles by
// split 0).  Measured, L2 flushed, means (previous selection: 64-column tiles
// for narrow N and at most six splits, added up in split 0 -> this, cuBLAS):
// 16 x 1024 x 32768 32.3 -> 27.8 us (36.0), 16 x 1024 x 16384 22.6 -> 20.5
// (23.6), 16 x 2048 x 16384 27.0 -> 24.7 (37.6), 16 x 2048 x 8192 20.2 ->
// 18.5 (18.6), 33 x 1024 x 16384 23.3 -> 22.2 (27.3), 48 x 4096 x 8192 26.5 ->
// 24.0 (22.9), 64 x 2048 x 8192 21.3 -> 20.2 (19.8), 64 x 1024 x 8192 19.1 ->
// 18.2 (17.7), 64 x 4096 x 4096 19.6 -> 18.8 (16.2).  False when none fits.
bool skinny_cluster_split(long long tiles, int K, int b_layout, int sms, kmcts_gemm_config* cfg) {
    if (tiles <= 0 || 2 * tiles > sms || K < 4096) return false;
    int s = static_cast<int>(sms / tiles);
    if (s > 8) s = 8;
    if (s > K / 512) s = K / 512;
    for (; s >= 2; --s) {
        kmcts_gemm_config c = *cfg;
        c.k_splits = s;
        c.flags |= KMCTS_FLAG_SPLIT_CLUSTER;
        if (!(c.tile_m == 32 && s == 2)) c.flags |= KMCTS_FLAG_SPLIT_SCATTER;
        int capacity = cluster_capacity(c, b_layout, s);
        if (capacity <= 0) capacity = fallback_cluster_capacity(s, sms);
        if (tiles <= capacity && cluster_split_fits(c, b_layout, s)) {
            *cfg = c;
            return true;
        }
    }
    return false;
}

}  // namespace

// The schedule for the shape; kmcts_select_config adds the A-side cache policy.
static int select_schedule(int M, int N, int K, int b_layout, kmcts_gemm_config* cfg) {
    kmcts_default_config(cfg);
    // Measured on B200 (CUDA-graph replays, warm L2):
    // * M <= 64: one CTA per tile staging 32 or 64 rows of A (more B in
    //   flight per SM; the problem is bound by reading B): for M <= 32,
    //   128 x 256 tiles when they fill the SMs' pairs count; else 128-column
    //   tiles with split K over one cluster per tile on long K; B's loads at
    //   L2 evict-first priority (it is read once);
    // * the CTA-pair 256 x 256 schedule once its tiles fill the co-resident
    //   pairs (with 64-deep stages when K <= 768), or, split in two along K,
    //   when two units per tile fill three quarters of them and K >= 8192;
    // * below that, one CTA per 128 x 256 tile while those fill the pairs'
    //   count and K is short (from K = 4096 the pair's faster mainloop wins
    //   back its idle SMs), else one CTA per 128 x 128 tile, split K on long K.
    const int sms = multiprocessor_count();
    // Co-resident CTA pairs of the default pair kernel, as its launch plans
    // them (occupancy-derived; SMs / 2 where no device can be queried).
    int workers = sms / 2;
    {
        kmcts_gemm_plan plan = {};
        if (M > 0 && N > 0 && K > 0 && plan_tcgen05(*cfg, M, N, K, b_layout, &plan) == KMCTS_OK && plan.workers > 0)
            workers = plan.workers;
    }
    kmcts_gemm_config small = *cfg;
    small.cluster_m = 1;
    if (M > 0 && M <= 32) {
        small.tile_m = 32;
        kmcts_gemm_config split = small;
        split.tile_n = 128;
        split.tile_k = 128;
        split.stages = 4;
        split.flags |= KMCTS_FLAG_B_EVICT_FIRST;  // one tile row: B is read once
        if ((N + 255) / 256 < workers && skinny_cluster_split((N + 127) / 128, K, b_layout, sms, &split) &&
            tcgen05_legal(split, M, N, K, b_layout, nullptr, 0) == KMCTS_OK) {
            *cfg = split;
            return KMCTS_OK;
        }
        if ((N + 255) / 256 >= workers) {
            small.tile_n = 256;
            small.tile_k = 64;
            small.stages = 5;
        } else if (4 * ((N + 63) / 64) <= sms) {
            // Narrow N: 64-column tiles put twice the CTAs on the stream
            // (16 x 2048 x 8192 19.7 us against 20.4 for 128-column tiles).
            small.tile_n = 64;
            small.tile_k = 128;
            small.stages = 8;
        } else {
            small.tile_n = 128;
            small.tile_k = 128;
            small.stages = 4;
        }
        small.k_splits = choose_splits((N + small.tile_n - 1) / small.tile_n, K, sms);
        small.flags |= KMCTS_FLAG_B_EVICT_FIRST;  // one tile row: B is read once
        // The splits of a tile add up in shared memory, as one cluster, up to
        // as many as split 0 can receive and at most six: sixteen clusters of
        // eight do not all fit at once (L2 flushed: 16 x 1024 x 16384 22.6 us
        // with six splits, 34.5 with eight, 32.4 with eight through the
        // workspace; 16 x 8192 x 8192 33.1 against 34.6 with two each).
        if (small.k_splits > 1) {
            int cap = cluster_split_cap(small, b_layout);
            if (cap > 6) cap = 6;
            if (cap > 1) {
                if (small.k_splits > cap) small.k_splits = cap;
                small.flags |= KMCTS_FLAG_SPLIT_CLUSTER;
            }
        }
        if (tcgen05_legal(small, M, N, K, b_layout, nullptr, 0) == KMCTS_OK) {
            *cfg = small;
            return KMCTS_OK;
        }
        small = *cfg;
        small.cluster_m = 1;
    }
    if (M > 32 && M <= 64) {
        // 64 rows of A per tile; 64-column tiles while two splits of them fit
        // the SMs, else 128-column tiles (three stages when split, leaving
        // split 0 room to receive; four unsplit).  Measured, L2 flushed
        // (against the 128-row schedule): 33 x 1024 x 16384 22.5 us against
        // 30.6, 64 x 2048 x 8192 20.6 against 23.7, 64 x 4096 x 4096 18.6
        // against 22.5, 64 x 8192 x 8192 33.9 against 35.1, 64 x 16384 x 4096
        // 30.8 against 31.5.
        small.tile_m = 64;
        kmcts_gemm_config split = small;
        split.tile_n = 128;
        split.tile_k = 128;
        split.stages = 3;
        split.flags |= KMCTS_FLAG_B_EVICT_FIRST;
        if (skinny_cluster_split((N + 127) / 128, K, b_layout, sms, &split) &&
            tcgen05_legal(split, M, N, K, b_layout, nullptr, 0) == KMCTS_OK) {
            *cfg = split;
            return KMCTS_OK;
        }
        small.tile_k = 128;
        if (2 * ((N + 63) / 64) <= sms) {
            small.tile_n = 64;
            small.stages = 6;
        } else {
            small.tile_n = 128;
        }
        small.k_splits = choose_splits((N + small.tile_n - 1) / small.tile_n, K, sms);
        if (small.tile_n == 128) small.stages = small.k_splits > 1 ? 3 : 4;
        small.flags |= KMCTS_FLAG_B_EVICT_FIRST;
        if (small.k_splits > 1) {
            int cap = cluster_split_cap(small, b_layout);
            if (cap > 6) cap = 6;
            if (cap > 1) {
                if (small.k_splits > cap) small.k_splits = cap;
                small.flags |= KMCTS_FLAG_SPLIT_CLUSTER;
            }
        }
        if (tcgen05_legal(small, M, N, K, b_layout, nullptr, 0) == KMCTS_OK) {
            *cfg = small;
            return KMCTS_OK;
        }
        small = *cfg;
        small.cluster_m = 1;
    }
    const long long pair_tiles = static_cast<long long>((M + 255) / 256) * ((N + 255) / 256);
    // N <= 128 leaves half of every 256-column pair tile empty: one CTA per
    // 128 x 128 tile instead (L2 flushed, A at evict-first priority:
    // 16384 x 128 x 4096 33.1 us against 36.7 for the pair, 16384 x 64 x 8192
    // 55.5 against 59.6).
    const bool pair_fits_n = N > 128;
    // One or two rows of pair tiles (M <= 512): each B column is read by one
    // or two pairs, close together in time, so B streams through L2 at
    // evict-first priority (measured, L2 flushed: 256 x 16384 x 4096 37.8 us
    // against 43.8, 200 x 16384 x 8192 62.6 against 70.8, 256 x 8192 x 8192
    // split in two 43.7 against 48.8, 512 x 8192 x 8192 56.0 against 61.5,
    // 512 x 16384 x 4096 57.5 against 62.0; bit-identical).  With more rows
    // the re-reads miss: 1024 x 16384 x 4096 95.7 against 96.4, 4096^3 96.1
    // against 95.3, 8192^3 811 against 783.
    const int pair_b_flags = M <= 512 ? KMCTS_FLAG_B_EVICT_FIRST : 0;
    if (pair_tiles >= workers && pair_fits_n) {
        cfg->flags |= pair_b_flags;
        // Short K (at most six 128-deep blocks per tile): 64-deep stages keep
        // the pipeline full through each tile's few K blocks; six of them,
        // five below K = 256 (measured, L2 flushed: 8192^2 x 768 78.9 us
        // against 81.2 for the default, 4096 x 8192 x 768 46.1 against 47.7).
        if (K <= 768) {
            cfg->tile_k = 64;
            cfg->stages = K <= 256 ? 5 : 6;
        }
        return KMCTS_OK;
    }
    // Two K splits of the pair tiles fill at least three quarters of the pairs
    // and K is long enough to carry the 256 KB FP32 partial of each unit
    // (measured: 4096 x 512 x 16384 68.2 us against 76.5 for one-CTA tiles,
    // 256 x 8192 x 8192 49.0 against 52.4; at K = 4096, or with four splits,
    // one-CTA tiles win).  Not for M <= 128, where a 256-row pair tile would
    // be mostly empty.
    // Three K splits when those fill at least three quarters of the pairs
    // and two do not (L2 flushed, means, against the one-CTA 128 x 128
    // schedule unsplit: 768 x 2048 x 8192 39.4 us against 43.3, 1024 x 1536 x
    // 8192 38.9 against 42.7, 640 x 2048 x 8192 38.7 against 42.8).
    if (M > 128 && pair_fits_n && 3 * pair_tiles <= workers && 4 * pair_tiles >= workers && K >= 8192) {
        kmcts_gemm_config split = *cfg;
        split.tile_k = 64;
        split.stages = 6;
        split.k_splits = 3;
        split.flags |= pair_b_flags;
        if (tcgen05_legal(split, M, N, K, b_layout, nullptr, 0) == KMCTS_OK) {
            *cfg = split;
            return KMCTS_OK;
        }
    }
    if (M > 128 && pair_fits_n && 2 * pair_tiles <= workers && 8 * pair_tiles >= 3 * workers && K >= 8192) {
        // With more than two tile columns, one CTA per 128 x 256 tile in two
        // K splits added up across a 2-CTA cluster does a little better
        // (L2 flushed, means: 512 x 4096 x 8192 41.3 us against 43.5 for the
        // pairs, 1024 x 2048 x 8192 41.8 against 42.8, 256 x 8192 x 8192 44.2
        // against 44.5; 4096 x 512 x 16384 66.0 against 65.0 keeps the pairs).
        if ((N + 255) / 256 > 2) {
            kmcts_gemm_config wide = *cfg;
            wide.tile_m = 128;
            wide.cluster_m = 1;
            wide.tile_n = 256;
            wide.tile_k = 64;
            wide.stages = 4;
            wide.k_splits = 2;
            wide.flags |= pair_b_flags | KMCTS_FLAG_SPLIT_CLUSTER | KMCTS_FLAG_SPLIT_SCATTER;
            const long long wide_units = 2LL * ((M + 127) / 128) * ((N + 255) / 256);
            int capacity = cluster_capacity(wide, b_layout, 2);
            if (capacity <= 0) capacity = fallback_cluster_capacity(2, sms);
            if (wide_units <= sms && wide_units / 2 <= capacity && cluster_split_fits(wide, b_layout, 2) &&
                tcgen05_legal(wide, M, N, K, b_layout, nullptr, 0) == KMCTS_OK) {
                *cfg = wide;
                return KMCTS_OK;
            }
        }
        kmcts_gemm_config split = *cfg;
        split.tile_k = 64;
        split.stages = 6;
        split.k_splits = 2;
        split.flags |= pair_b_flags;
        if (tcgen05_legal(split, M, N, K, b_layout, nullptr, 0) == KMCTS_OK) {
            *cfg = split;
            return KMCTS_OK;
        }
    }
    small.tile_m = 128;
    const long long wide_tiles = static_cast<long long>((M + 127) / 128) * ((N + 255) / 256);
    if (wide_tiles >= workers && pair_fits_n) {
        if (K >= 4096) {
            cfg->flags |= pair_b_flags;  // the pair schedule after all
            return KMCTS_OK;
        }
        small.tile_n = 256;
        small.tile_k = 64;
        small.stages = 4;
    } else {
        small.tile_n = 128;
        small.tile_k = 128;
        small.stages = 3;
        const long long tiles = static_cast<long long>((M + 127) / 128) * ((N + 127) / 128);
        // More than eight workspace splits (a tile or two over a very long
        // K) beat a cluster's eight: 128 x 128 x 65536 48.8 us against 53.4.
        small.k_splits = choose_splits(tiles, K, sms);
        if (M > 64 && small.k_splits <= 8) scatter_schedule(tiles, K, b_layout, sms, &small);
    }
    // M within one 128-row tile: every B byte is read by one CTA only, so its
    // loads stream through L2 at evict-first priority (measured, L2 flushed
    // by a 512 MiB write: 128 x 16384 x 4096 31.8 us against 37.8 without the
    // hint and 36.8 for cuBLAS; 16 x 8192 x 8192 34.4 against 38.6).
    if (M <= 128) small.flags |= KMCTS_FLAG_B_EVICT_FIRST;
    // M <= 64 (reached only when no 64-row schedule is legal): the K splits
    // add up in split 0's pipeline stages, one cluster per tile (L2 flushed:
    // 64 x 2048 x 8192 23.4 us against 26.4 through the workspace, 48 x 4096
    // x 8192 26.8 against 27.9; at M = 128 the workspace wins, 128 x 4096 x
    // 8192 29.0 against 29.1-30.2).
    if (M <= 64 && small.k_splits > 1) {
        int cap = cluster_split_cap(small, b_layout);
        if (cap > 6) cap = 6;
        if (cap > 1) {
            if (small.k_splits > cap) small.k_splits = cap;
            small.flags |= KMCTS_FLAG_SPLIT_CLUSTER;
        }
    }
    if (tcgen05_legal(small, M, N, K, b_layout, nullptr, 0) == KMCTS_OK) *cfg = small;
    return KMCTS_OK;
}

int kmcts_select_config(int M, int N, int K, int b_layout, kmcts_gemm_config* cfg) {
    if (!cfg || M < 0 || N < 0 || K < 0) return KMCTS_EINVAL;
    const int rc = select_schedule(M, N, K, b_layout, cfg);
    // N within one or two tile columns: every A byte is read by one or two
    // CTAs (pairs), close together in time, so A streams through L2 at
    // evict-first priority (measured, L2 flushed by a 512 MiB write:
    // 28672 x 256 x 4096 63.0 us against 70.4, 8192 x 512 x 4096 35.3
    // against 39.4, 2048 x 256 x 8192 26.8 against 28.4; bit-identical).
    if (rc == KMCTS_OK && cfg->tile_n > 0 && N > 0 && (N + cfg->tile_n - 1) / cfg->tile_n <= 2 &&
        tcgen05_legal(*cfg, M, N, K, b_layout, nullptr, 0) == KMCTS_OK)
        cfg->flags |= KMCTS_FLAG_A_EVICT_FIRST;
    return rc;
}

const char* kmcts_version(void) { return "kmcts_gemm_sm100 0.1.0 (sm_100a tcgen05)"; }

int64_t kmcts_launch_count(void) { return g_launches.load(std::memory_order_relaxed); }

int kmcts_time_gemm(const void* A, const void* B, void* C, int M, int N, int K, int b_layout,
                    const kmcts_gemm_config* cfg, void* stream, int* device_status, int warmups,
                    int measurements, void* flush, size_t flush_bytes, float* timings_us) {
    if (warmups < 0 || measurements < 1 || !timings_us || !device_status || (flush_bytes && !flush))
        return KMCTS_EINVAL;
    cudaStream_t s = as_stream(stream);
    for (int i = 0; i < warmups; ++i) {
        const int rc = kmcts_bf16_gemm_ex(A, B, C, M, N, K, b_layout, cfg, stream, device_status);
        if (rc != KMCTS_OK) return rc;
    }
    if (cudaStreamSynchronize(s) != cudaSuccess) return KMCTS_ESYNC;
    cudaEvent_t start = nullptr, stop = nullptr;
    if (cudaEventCreate(&start) != cudaSuccess || cudaEventCreate(&stop) != cudaSuccess) {
        if (start) cudaEventDestroy(start);
        return KMCTS_EHANDLE;
    }
    int rc = KMCTS_OK;
    for (int i = 0; i < measurements && rc == KMCTS_OK; ++i) {
        if (flush && cudaMemsetAsync(flush, i & 0xff, flush_bytes, s) != cudaSuccess) {
            rc = KMCTS_ESYNC;
            break;
        }
        if (cudaEventRecord(start, s) != cudaSuccess) {
            rc = KMCTS_ESYNC;
            break;
        }
        rc = kmcts_bf16_gemm_ex(A, B, C, M, N, K, b_layout, cfg, stream, device_status);
        if (rc != KMCTS_OK) break;
        float ms = 0.0f;
        if (cudaEventRecord(stop, s) != cudaSuccess || cudaEventSynchronize(stop) != cudaSuccess ||
            cudaEventElapsedTime(&ms, start, stop) != cudaSuccess) {
            rc = KMCTS_ESYNC;
            break;
        }
        timings_us[i] = ms * 1000.0f;
    }
    cudaEventDestroy(start);
    cudaEventDestroy(stop);
    if (rc != KMCTS_OK) return rc;
    int status = 0;
    if (cudaMemcpyAsync(&status, device_status, sizeof(int), cudaMemcpyDeviceToHost, s) != cudaSuccess ||
        cudaStreamSynchronize(s) != cudaSuccess)
        return KMCTS_ESYNC;
    return status == 0 ? KMCTS_OK : KMCTS_ETIMEOUT;
}

int64_t kmcts_config_smem_bytes(const kmcts_gemm_config* cfg, int b_layout) {
    if (!cfg) return 0;
    return tcgen05_smem_bytes(*cfg, b_layout);
}

int kmcts_config_legal(const kmcts_gemm_config* cfg, int M, int N, int K, int b_layout, char* why,
                       int len) {
    if (!cfg) return KMCTS_EINVAL;
    return tcgen05_legal(*cfg, M, N, K, b_layout, why, len);
}

int kmcts_bf16_gemm_ex(const void* A, const void* B, void* C, int M, int N, int K, int b_layout,
                       const kmcts_gemm_config* cfg, void* stream, int* device_status) {
    if (M < 0 || N < 0 || K < 0) return KMCTS_EINVAL;
    if (b_layout != KMCTS_B_COL && b_layout != KMCTS_B_ROW) return KMCTS_EINVAL;
    if ((M > 0 && N > 0) && (!C || (K > 0 && (!A || !B)))) return KMCTS_EINVAL;
    kmcts_gemm_config local;
    if (cfg) {
        local = *cfg;
    } else {
        kmcts_select_config(M, N, K, b_layout, &local);
    }
    cudaStream_t s = as_stream(stream);
    if (local.kernel == KMCTS_KERNEL_SIMT) return launch_simt(A, B, C, M, N, K, b_layout, s);
    const int rc = launch_tcgen05(A, B, C, M, N, K, b_layout, local, s, device_status);
    if (rc == KMCTS_ENOTSUP && local.kernel == KMCTS_KERNEL_AUTO) {
        return launch_simt(A, B, C, M, N, K, b_layout, s);
    }
    return rc;
}

int kmcts_bf16_gemm(const void* A, const void* B, void* C, int M, int N, int K) {
    const int rc = kmcts_bf16_gemm_ex(A, B, C, M, N, K, KMCTS_B_COL, nullptr, nullptr, nullptr);
    if (rc != KMCTS_OK) return rc;
    if (cudaDeviceSynchronize() != cudaSuccess) return KMCTS_ESYNC;
    int status = 0;
    if (take_default_status(nullptr, &status) != KMCTS_OK) return KMCTS_ESYNC;
    return status == 0 ? KMCTS_OK : KMCTS_ETIMEOUT;
}

int kmcts_gemm_plan_query(const kmcts_gemm_config* cfg, int M, int N, int K, int b_layout, kmcts_gemm_plan* out) {
    if (!out) return KMCTS_EINVAL;
    kmcts_gemm_config local;
    if (cfg) {
        local = *cfg;
    } else {
        kmcts_select_config(M, N, K, b_layout, &local);
    }
    if (local.kernel != KMCTS_KERNEL_SIMT) {
        const int rc = plan_tcgen05(local, M, N, K, b_layout, out);
        if (rc != KMCTS_ENOTSUP || local.kernel == KMCTS_KERNEL_TCGEN05) return rc;
    }
    kmcts_gemm_plan plan = {};
    plan.kernel = 3;
    plan.cluster_size = 1;
    plan.tiles = ((M + 63) / 64) * ((N + 63) / 64);
    plan.full_tiles = plan.units = plan.ctas = plan.tiles;
    plan.workers = multiprocessor_count();
    plan.k_splits = 1;
    *out = plan;
    return KMCTS_OK;
}

int kmcts_bf16_gemm_allgather(const void* A, const void* B_shard, void* const* C_ranks, int num_ranks, int rank,
                              int M, int N_total, int K, int b_layout, const kmcts_gemm_config* cfg, void* stream,
                              int* device_status) {
    kmcts_gemm_config local;
    if (cfg) {
        local = *cfg;
    } else {
        kmcts_default_config(&local);
    }
    if (b_layout != KMCTS_B_COL && b_layout != KMCTS_B_ROW) return KMCTS_EINVAL;
    return launch_allgather_tcgen05(A, B_shard, C_ranks, num_ranks, rank, M, N_total, K, b_layout, local,
                                    as_stream(stream), device_status);
}

int kmcts_generate_inputs(int kind, uint32_t seed, size_t a_count, size_t b_count, uint16_t* a_out,
                          uint16_t* b_out) {
    if ((a_count && !a_out) || (b_count && !b_out)) return KMCTS_EINVAL;
    auto store = [](uint16_t* dst, float v) {
        const __nv_bfloat16 h = __float2bfloat16(v);
        std::memcpy(dst, &h, sizeof(uint16_t));
    };
    if (kind == KMCTS_INPUTS_UNIFORM) {
        // The repository contract's stream: one mt19937(seed), A then B,
        // U(-0.25, 0.25), RNE to BF16 (bf16_gemm_harness.cu:92-95).
        std::mt19937 generator(seed);
        std::uniform_real_distribution<float> distribution(-0.25f, 0.25f);
        for (size_t i = 0; i < a_count; ++i) store(a_out + i, distribution(generator));
        for (size_t i = 0; i < b_count; ++i) store(b_out + i, distribution(generator));
    } else if (kind == KMCTS_INPUTS_RANDN) {
        std::mt19937_64 generator(seed);
        std::normal_distribution<float> distribution(0.0f, 1.0f);
        for (size_t i = 0; i < a_count; ++i) store(a_out + i, distribution(generator));
        for (size_t i = 0; i < b_count; ++i) store(b_out + i, distribution(generator));
    } else if (kind == KMCTS_INPUTS_INT) {
        std::mt19937 generator(seed);
        std::uniform_int_distribution<int> distribution(-2, 2);
        for (size_t i = 0; i < a_count; ++i) store(a_out + i, static_cast<float>(distribution(generator)));
        for (size_t i = 0; i < b_count; ++i) store(b_out + i, static_cast<float>(distribution(generator)));
    } else {
        return KMCTS_EINVAL;
    }
    return KMCTS_OK;
}

size_t kmcts_compare_workspace_bytes(void) { return compare_workspace_bytes(); }

int kmcts_bf16_compare(const void* C, const void* reference, int64_t count, double rtol,
                       double atol, void* workspace, void* stream, kmcts_compare_result* out) {
    return compare_bf16_device(C, reference, count, rtol, atol, workspace, as_stream(stream), out);
}

}  // extern "C"
