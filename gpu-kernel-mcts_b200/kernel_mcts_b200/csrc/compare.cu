// Device-side correctness check of a BF16 output against a BF16 reference.
//
// Restates the reference harness's host scan
// (src/kernel_mcts/benchmarks/kernels/bf16_gemm_harness.cu:154-164): per element
// error = |c - ref| in double; maximum_error ignores NaN errors (std::max
// semantics), mean_error = sum / count; an element fails if c is not finite or
// error > atol + rtol * |ref|.  Adds BF16 ulp statistics.  One pass over both
// arrays (HBM-bound: 4 bytes read per element) instead of a 16.8 M-element
// host loop after two device-to-host copies.
#include <cuda_bf16.h>
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "kmcts_internal.h"

namespace kmcts {
namespace {

struct CompareWorkspace {
    unsigned long long max_error_bits;  // non-negative doubles order like integers
    double error_sum;
    unsigned long long n_fail;
    unsigned long long n_nonfinite;
    unsigned long long hist[4];
    unsigned int max_ulp;
    unsigned int pad;
};
static_assert(sizeof(CompareWorkspace) <= 256, "workspace grew");

__device__ __forceinline__ int ordered_bf16(uint16_t v) {
    return (v & 0x8000u) ? -static_cast<int>(v & 0x7fffu) : static_cast<int>(v);
}

__device__ __forceinline__ bool is_nan_bf16(uint16_t v) {
    return (v & 0x7f80u) == 0x7f80u && (v & 0x7fu) != 0u;
}

__global__ void __launch_bounds__(256) compare_bf16(const uint16_t* __restrict__ c,
                                                    const uint16_t* __restrict__ ref, int64_t count,
                                                    double rtol, double atol,
                                                    CompareWorkspace* ws) {
    double max_err = 0.0, sum = 0.0;
    unsigned long long fails = 0, nonfinite = 0, hist[4] = {0, 0, 0, 0};
    unsigned int max_ulp = 0;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count;
         i += stride) {
        const uint16_t cv = c[i], rv = ref[i];
        const double actual = __bfloat162float(__ushort_as_bfloat16(cv));
        const double expected = __bfloat162float(__ushort_as_bfloat16(rv));
        const double err = fabs(actual - expected);
        if (err > max_err) max_err = err;  // false for NaN, as std::max keeps the old value
        sum += err;
        const bool finite = isfinite(actual);
        if (!finite) ++nonfinite;
        if (!finite || err > atol + rtol * fabs(expected)) ++fails;
        unsigned int d;
        if (is_nan_bf16(cv) || is_nan_bf16(rv)) {
            d = 65535u;
        } else {
            const int diff = ordered_bf16(cv) - ordered_bf16(rv);
            d = static_cast<unsigned int>(diff < 0 ? -diff : diff);
        }
        if (d > max_ulp) max_ulp = d;
        hist[d > 2 ? 3 : d] += 1;
    }
    // Warp reduction, then one atomic per warp.
    for (int off = 16; off > 0; off >>= 1) {
        max_err = fmax(max_err, __shfl_down_sync(0xffffffffu, max_err, off));
        sum += __shfl_down_sync(0xffffffffu, sum, off);
        fails += __shfl_down_sync(0xffffffffu, fails, off);
        nonfinite += __shfl_down_sync(0xffffffffu, nonfinite, off);
        for (int h = 0; h < 4; ++h) hist[h] += __shfl_down_sync(0xffffffffu, hist[h], off);
        max_ulp = max(max_ulp, __shfl_down_sync(0xffffffffu, max_ulp, off));
    }
    if ((threadIdx.x & 31) == 0) {
        atomicMax(&ws->max_error_bits, static_cast<unsigned long long>(__double_as_longlong(max_err)));
        atomicAdd(&ws->error_sum, sum);
        atomicAdd(&ws->n_fail, fails);
        atomicAdd(&ws->n_nonfinite, nonfinite);
        for (int h = 0; h < 4; ++h) atomicAdd(&ws->hist[h], hist[h]);
        atomicMax(&ws->max_ulp, max_ulp);
    }
}

}  // namespace

size_t compare_workspace_bytes() { return 256; }

int compare_bf16_device(const void* C, const void* reference, int64_t count, double rtol,
                        double atol, void* workspace, cudaStream_t stream,
                        kmcts_compare_result* out) {
    if (!C || !reference || !workspace || !out || count < 0) return KMCTS_EINVAL;
    auto* ws = static_cast<CompareWorkspace*>(workspace);
    if (cudaMemsetAsync(ws, 0, sizeof(CompareWorkspace), stream) != cudaSuccess) return KMCTS_EGEMM;
    if (count > 0) {
        const int64_t blocks64 = (count + 255) / 256;
        const int blocks = static_cast<int>(blocks64 < 148 * 16 ? blocks64 : 148 * 16);
        compare_bf16<<<blocks, 256, 0, stream>>>(static_cast<const uint16_t*>(C),
                                                 static_cast<const uint16_t*>(reference), count,
                                                 rtol, atol, ws);
        g_launches.fetch_add(1, std::memory_order_relaxed);
        if (cudaGetLastError() != cudaSuccess) return KMCTS_EGEMM;
    }
    CompareWorkspace host;
    if (cudaMemcpyAsync(&host, ws, sizeof(host), cudaMemcpyDeviceToHost, stream) != cudaSuccess)
        return KMCTS_ESYNC;
    if (cudaStreamSynchronize(stream) != cudaSuccess) return KMCTS_ESYNC;
    std::memcpy(&out->maximum_error, &host.max_error_bits, sizeof(double));
    out->mean_error = count ? host.error_sum / static_cast<double>(count) : 0.0;
    out->count = count;
    out->n_tolerance_fail = static_cast<int64_t>(host.n_fail);
    out->n_nonfinite = static_cast<int64_t>(host.n_nonfinite);
    for (int h = 0; h < 4; ++h) out->ulp_hist[h] = static_cast<int64_t>(host.hist[h]);
    out->max_ulp = static_cast<int32_t>(host.max_ulp);
    out->success = host.n_fail == 0 ? 1 : 0;
    return KMCTS_OK;
}

}  // namespace kmcts

// ---------------------------------------------------------------------------
// Allocation-free comparison.
//
// Some callers cannot call cudaMalloc at the moment they want a correctness
// check: a worker in the middle of an evaluation whose memory budget is fully
// owned by another allocator (a framework caching allocator that must see
// every device allocation, or it may run the device out of memory), or an
// embedding host whose only device memory is the inputs and outputs it
// already passes in.  For them the
// comparison's scratch (its reduction accumulators) lives in this file-scope
// device array instead of a caller-provided workspace.  Every GPU that loads
// the library holds these bytes until the process exits.
namespace kmcts {
namespace {

constexpr size_t kNoAllocScratchBytes = KMCTS_NOALLOC_SCRATCH_BYTES;
static __device__ __align__(256) unsigned char g_compare_scratch[kNoAllocScratchBytes];

PFN_cuCtxGetCurrent_v4000 current_context_fn() {
    static std::once_flag once;
    static PFN_cuCtxGetCurrent_v4000 fn = nullptr;
    std::call_once(once, [] {
        void* entry = nullptr;
        cudaDriverEntryPointQueryResult query;
        if (cudaGetDriverEntryPointByVersion("cuCtxGetCurrent", &entry, 4000, cudaEnableDefault, &query) ==
                cudaSuccess &&
            query == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuCtxGetCurrent_v4000>(entry);
    });
    return fn;
}

// Device address of g_compare_scratch, looked up once per device with that
// device current (host code cannot use the symbol itself as a pointer), and
// looked up again if the device's context has been recreated since (after a
// cudaDeviceReset the module reloads and the array may move).
void* noalloc_scratch_address(int* rc) {
    static std::mutex mu;
    static void* address[64] = {};
    static CUcontext context[64] = {};
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= 64) {
        *rc = KMCTS_EHANDLE;
        return nullptr;
    }
    auto get_current = current_context_fn();
    CUcontext current = nullptr;
    if (get_current == nullptr || get_current(&current) != CUDA_SUCCESS) current = nullptr;
    std::lock_guard<std::mutex> lock(mu);
    if (address[device] == nullptr || context[device] != current) {
        void* ptr = nullptr;
        if (cudaGetSymbolAddress(&ptr, g_compare_scratch) != cudaSuccess || ptr == nullptr) {
            cudaGetLastError();
            *rc = KMCTS_EHANDLE;
            return nullptr;
        }
        // The lookup made the device's primary context current: remember it.
        if (get_current == nullptr || get_current(&current) != CUDA_SUCCESS) current = nullptr;
        address[device] = ptr;
        context[device] = current;
    }
    *rc = KMCTS_OK;
    return address[device];
}

}  // namespace
}  // namespace kmcts

extern "C" int kmcts_bf16_compare_noalloc(const void* C, const void* reference, int64_t count, double rtol,
                                          double atol, void* stream, kmcts_compare_result* out) {
    using namespace kmcts;
    if (!C || !reference || !out || count < 0) return KMCTS_EINVAL;
    // The scratch this comparison needs does not grow with `count`; a call
    // whose need exceeded the static array would be refused here.
    if (compare_workspace_bytes() > kNoAllocScratchBytes) return KMCTS_ENOSCRATCH;
    int rc = KMCTS_OK;
    void* scratch = noalloc_scratch_address(&rc);
    if (rc != KMCTS_OK) return rc;
    // compare_bf16_device zeroes the accumulators on `stream` before it reduces.
    return compare_bf16_device(C, reference, count, rtol, atol, scratch, static_cast<cudaStream_t>(stream), out);
}
