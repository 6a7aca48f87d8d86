// Internal declarations shared by the translation units of libkmcts_gemm_sm100.so.
#pragma once

#include <atomic>
#include <cstdint>
#include <cuda.h>
#include <cuda_runtime.h>

#include "kmcts_gemm.h"

namespace kmcts {

// Counts every kernel launch the library makes (kmcts_launch_count()).
extern std::atomic<int64_t> g_launches;

// Encodes a 2-D BF16 tensor map (dim0 innermost) with 128-byte swizzle.
// Returns false when the driver rejects it.
bool encode_tensor_map_2d(CUtensorMap* map, const void* base, uint64_t dim0, uint64_t dim1,
                          uint64_t row_stride_bytes, uint32_t box0, uint32_t box1);

// Launch shape of a legal tcgen05 schedule on the current device.
int plan_tcgen05(const kmcts_gemm_config& cfg, int M, int N, int K, int b_layout, kmcts_gemm_plan* out);

// tcgen05 path.  Returns KMCTS_OK or an error code; launches nothing on error.
int launch_tcgen05(const void* A, const void* B, void* C, int M, int N, int K, int b_layout,
                   const kmcts_gemm_config& cfg, cudaStream_t stream, int* device_status);

// Static checks for the tcgen05 path (shape, alignment-free parts, schedule).
int tcgen05_legal(const kmcts_gemm_config& cfg, int M, int N, int K, int b_layout, char* why,
                  int len);
int64_t tcgen05_smem_bytes(const kmcts_gemm_config& cfg, int b_layout);
// Most K splits a one-CTA schedule can add up as a cluster split K
// (KMCTS_FLAG_SPLIT_CLUSTER): the receive buffer must fit beside its own
// shared memory, and a cluster holds at most 8 CTAs.  1 when none fits.
int cluster_split_cap(const kmcts_gemm_config& cfg, int b_layout);
// Whether a cluster split K of `splits` CTAs runs for cfg's schedule in the
// form its flags ask for (the scatter form's fit is not monotonic in splits).
bool cluster_split_fits(const kmcts_gemm_config& cfg, int b_layout, int splits);
// Clusters of a cluster split K of `splits` CTAs (cfg's schedule and split
// flags) that can be resident at once on the current device, from the
// occupancy calculator; 0 where it cannot say (no device, or no such split).
int cluster_capacity(const kmcts_gemm_config& cfg, int b_layout, int splits);

// CUDA-core path for any shape and alignment.
int launch_simt(const void* A, const void* B, void* C, int M, int N, int K, int b_layout,
                cudaStream_t stream);

// Device address of the library's default status word (for kernels launched
// with no status pointer), or nullptr if it cannot be had.
int* default_status_ptr();

// Reads and clears the library's default device status word.
int take_default_status(cudaStream_t stream, int* value);

int multiprocessor_count();

// A zeroed device workspace of at least `bytes` for kernels launched on
// `stream` (one per device, stream and `user`), and the launch epoch to tag
// its flags with.  False when none can be had now (out of memory, or growth
// needed while the stream is being captured).  Returned buffers are never
// freed, so graphs that captured them stay valid.  workspace.cu.
constexpr int kWorkspaceStreamK = 0, kWorkspaceSplitK = 1;
bool stream_workspace(cudaStream_t stream, int user, size_t bytes, void** ptr, int* epoch);

// Streamed skinny kernel (C^T = B^T A^T, M <= 32), gemm_tcgen05_stream.cu.
bool stream_variant_exists(const kmcts_gemm_config& cfg, int b_layout);
int64_t stream_smem_bytes(int bk, int stages);
int plan_stream(const kmcts_gemm_config& cfg, int M, int N, int K, kmcts_gemm_plan* out);
int launch_stream(const void* A, const void* B, void* C, int M, int N, int K, int b_layout,
                  const kmcts_gemm_config& cfg, uint64_t limit_ns, cudaStream_t stream, int* device_status);

// CTA-pair (cta_group::2) kernels, gemm_tcgen05_pair.cu.
bool pair_variant_exists(const kmcts_gemm_config& cfg, int b_layout);
int64_t pair_smem_bytes(int bn, int bk, int stages);
int plan_pair(const kmcts_gemm_config& cfg, int M, int N, int K, int b_layout, kmcts_gemm_plan* out);
int launch_pair_allgather(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb_half,
                          const CUtensorMap& mc, int M, int N_shard, int K, int b_layout,
                          const kmcts_gemm_config& cfg, uint64_t limit_ns, cudaStream_t stream, int* status,
                          void* const* peer_c, int peer_count, int ld, int col_offset);
int launch_allgather_tcgen05(const void* A, const void* B_shard, void* const* C_ranks, int num_ranks, int rank,
                             int M, int N_total, int K, int b_layout, const kmcts_gemm_config& cfg,
                             cudaStream_t stream, int* device_status);
int launch_pair(const CUtensorMap& ma, const CUtensorMap& mb, const CUtensorMap& mb_half, const CUtensorMap& mc,
                int M, int N, int K, int b_layout, const kmcts_gemm_config& cfg, uint64_t limit_ns,
                cudaStream_t stream, int* status);

}  // namespace kmcts

namespace kmcts {
size_t compare_workspace_bytes();
int compare_bf16_device(const void* C, const void* reference, int64_t count, double rtol,
                        double atol, void* workspace, cudaStream_t stream,
                        kmcts_compare_result* out);
}  // namespace kmcts
