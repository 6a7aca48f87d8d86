// CUTLASS column of the vendor baselines: the reference's fixed CUTLASS 2.x
// template (src/kernel_mcts/benchmarks/kernels/bf16_gemm_vendor_baselines.cu:15-28,
// 81-97) instantiated from the CUTLASS headers vendored in this image, built
// for sm_100a.  Library code, timed beside the sm_100a kernels under the same
// protocol; it is a baseline, not part of the product path.
#include <cuda_runtime.h>

#include <cutlass/bfloat16.h>
#include <cutlass/gemm/device/gemm.h>

namespace {

using Element = cutlass::bfloat16_t;
// A row-major, B column-major, C row-major, FP32 accumulate; the reference's
// tile shapes (CTA 128x128x32, warp 64x64x32, instruction 16x8x16).
using VendorGemm = cutlass::gemm::device::Gemm<
    Element, cutlass::layout::RowMajor, Element, cutlass::layout::ColumnMajor, Element,
    cutlass::layout::RowMajor, float, cutlass::arch::OpClassTensorOp, cutlass::arch::Sm80,
    cutlass::gemm::GemmShape<128, 128, 32>, cutlass::gemm::GemmShape<64, 64, 32>,
    cutlass::gemm::GemmShape<16, 8, 16>>;

}  // namespace

// Returns 0 on success, 1 if CUTLASS rejected the problem, 2 if the launch failed.
extern "C" int kmcts_vendor_cutlass_sm80_gemm(const void* A, const void* B, void* C, int M, int N, int K,
                                              cudaStream_t stream) {
    VendorGemm op;
    VendorGemm::Arguments args({M, N, K}, {static_cast<const Element*>(A), K},
                               {static_cast<const Element*>(B), K}, {static_cast<Element*>(C), N},
                               {static_cast<Element*>(C), N}, {1.0f, 0.0f});
    if (op.can_implement(args) != cutlass::Status::kSuccess) return 1;
    return op(args, nullptr, stream) == cutlass::Status::kSuccess ? 0 : 2;
}
