// CUDA-core BF16 GEMM for shapes the tcgen05 path cannot take (K or N not a
// multiple of 8, unaligned pointers).  Any M, N, K and either B layout.
//
// Each output keeps one FP32 accumulator updated by one FMA per k in
// increasing k order, then one RNE rounding — the accumulation order of the
// reference root program (src/kernel_mcts/benchmarks/kernels/bf16_gemm_root.cu:18-40),
// so this kernel reproduces it bit for bit.
#include <cuda_bf16.h>

#include "kmcts_internal.h"

namespace kmcts {
namespace {

constexpr int kTile = 64;    // 64x64 outputs per CTA
constexpr int kDepth = 16;   // K per shared-memory step
constexpr int kPerThread = 4;  // 4x4 outputs per thread, 256 threads

template <bool B_ROW>
__global__ void __launch_bounds__(256) gemm_bf16_simt(const __nv_bfloat16* __restrict__ A,
                                                      const __nv_bfloat16* __restrict__ B,
                                                      __nv_bfloat16* __restrict__ C, int M, int N,
                                                      int K) {
    __shared__ float as[kDepth][kTile + 1];
    __shared__ float bs[kDepth][kTile + 1];
    const int tx = threadIdx.x % 16;
    const int ty = threadIdx.x / 16;
    const int row0 = blockIdx.y * kTile;
    const int col0 = blockIdx.x * kTile;
    float acc[kPerThread][kPerThread] = {};
    for (int k0 = 0; k0 < K; k0 += kDepth) {
        for (int i = threadIdx.x; i < kDepth * kTile; i += blockDim.x) {
            const int kk = i % kDepth, r = i / kDepth;
            const int gr = row0 + r, gk = k0 + kk;
            as[kk][r] = (gr < M && gk < K) ? __bfloat162float(A[(size_t)gr * K + gk]) : 0.0f;
            const int gc = col0 + r;
            float bv = 0.0f;
            if (gc < N && gk < K) {
                bv = B_ROW ? __bfloat162float(B[(size_t)gk * N + gc])
                           : __bfloat162float(B[(size_t)gc * K + gk]);
            }
            bs[kk][r] = bv;
        }
        __syncthreads();
        const int depth = min(kDepth, K - k0);
        for (int kk = 0; kk < depth; ++kk) {
#pragma unroll
            for (int i = 0; i < kPerThread; ++i) {
                const float a = as[kk][ty + 16 * i];
#pragma unroll
                for (int j = 0; j < kPerThread; ++j) {
                    acc[i][j] = __fmaf_rn(a, bs[kk][tx + 16 * j], acc[i][j]);
                }
            }
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < kPerThread; ++i) {
        const int r = row0 + ty + 16 * i;
        if (r >= M) continue;
#pragma unroll
        for (int j = 0; j < kPerThread; ++j) {
            const int c = col0 + tx + 16 * j;
            if (c < N) C[(size_t)r * N + c] = __float2bfloat16_rn(acc[i][j]);
        }
    }
}

}  // namespace

int launch_simt(const void* A, const void* B, void* C, int M, int N, int K, int b_layout,
                cudaStream_t stream) {
    if (M == 0 || N == 0) return KMCTS_OK;
    dim3 grid((N + kTile - 1) / kTile, (M + kTile - 1) / kTile, 1);
    auto a = static_cast<const __nv_bfloat16*>(A);
    auto b = static_cast<const __nv_bfloat16*>(B);
    auto c = static_cast<__nv_bfloat16*>(C);
    if (b_layout == KMCTS_B_ROW) {
        gemm_bf16_simt<true><<<grid, 256, 0, stream>>>(a, b, c, M, N, K);
    } else {
        gemm_bf16_simt<false><<<grid, 256, 0, stream>>>(a, b, c, M, N, K);
    }
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError() == cudaSuccess ? KMCTS_OK : KMCTS_EGEMM;
}

}  // namespace kmcts
