// Host launcher for the reference's own root kernel, used only to pin the CPU
// oracle (TEST INFRASTRUCTURE ONLY: built into oracle/_ref/, never shipped).
//
// The kernel itself is compiled from the reference source where it lies,
// src/kernel_mcts/benchmarks/kernels/bf16_gemm_root.cu, by oracle/Makefile.
// The launch geometry restates the reference harness's launch_candidate,
// src/kernel_mcts/benchmarks/kernels/bf16_gemm_harness.cu:61-72:
// block (16,16,1), grid (ceil(N/16), ceil(M/16), 1), default stream.
#include <cuda_bf16.h>
#include <cuda_runtime.h>

extern "C" __global__ void bf16_gemm_root(const __nv_bfloat16* A, const __nv_bfloat16* B,
                                          __nv_bfloat16* C, int M, int N, int K);

// Returns 0 on success, 1 if the launch was rejected, 2 if the kernel failed.
extern "C" int kmcts_ref_root_gemm(const void* A, const void* B, void* C, int M, int N, int K) {
    dim3 block(16, 16, 1);
    dim3 grid((N + 15) / 16, (M + 15) / 16, 1);
    bf16_gemm_root<<<grid, block>>>(static_cast<const __nv_bfloat16*>(A),
                                    static_cast<const __nv_bfloat16*>(B),
                                    static_cast<__nv_bfloat16*>(C), M, N, K);
    if (cudaGetLastError() != cudaSuccess) return 1;
    if (cudaDeviceSynchronize() != cudaSuccess) return 2;
    return 0;
}
