// kmcts_bf16_eval — the evaluation harness for the BF16 GEMM contract on B200.
//
// Same command line and JSON as the reference harness
// (src/kernel_mcts/benchmarks/kernels/bf16_gemm_harness.cu:74-215):
//   --mode=correctness|benchmark --M --N --K --seed --warmups --measurements
//   --rtol --atol
// prints ONE JSON line and exits 0 (ok), 1 (launch_failure) or 2
// (infrastructure_failure), as the backend expects
// (src/kernel_mcts/cuda_backend.py:466-503).
//
// Additive flags: --b-layout=col|row, --inputs=uniform|randn|int,
// --kernel=auto|tcgen05|simt|candidate|cublas|cutlass_sm80, --k-splits, --tile-m
// --cluster-m --cluster-n --tile-n --tile-k --stages --persistent --raster-group --flags
// --wait-limit-ns, --flush-l2=0|1.  cublas and cutlass_sm80 are the vendor
// baseline columns (src/kernel_mcts/vendor_baselines.py), timed under the
// same protocol as the library kernel.
// Additive JSON keys: max_ulp, n_gt_1ulp, ulp_hist, n_nonfinite, kernel.
//
// Candidate programs: compiled together with this file and
//   -DKMCTS_CANDIDATE_ROOT      the reference ABI: extern "C" __global__
//                               bf16_gemm_root(A, B, C, M, N, K), fixed
//                               16x16 launch (bf16_gemm_harness.cu:61-72);
//   -DKMCTS_CANDIDATE_LAUNCHER  a host launcher that owns its launch:
//                               extern "C" int bf16_gemm_launch(A, B, C, M, N,
//                               K, cudaStream_t) returning 0 on success.
// Without either macro the harness evaluates the library kernel.
#include <cublas_v2.h>
#include <cuda_bf16.h>
#include <cuda_runtime.h>

#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <string>
#include <vector>

#include "kmcts_gemm.h"

#if KMCTS_HAVE_CUTLASS
extern "C" int kmcts_vendor_cutlass_sm80_gemm(const void* A, const void* B, void* C, int M, int N, int K,
                                              cudaStream_t stream);
#endif

#if defined(KMCTS_CANDIDATE_ROOT)
extern "C" __global__ void bf16_gemm_root(const __nv_bfloat16* A, const __nv_bfloat16* B,
                                          __nv_bfloat16* C, int M, int N, int K);
#elif defined(KMCTS_CANDIDATE_LAUNCHER)
extern "C" int bf16_gemm_launch(const void* A, const void* B, void* C, int M, int N, int K,
                                cudaStream_t stream);
#endif

namespace {

[[noreturn]] void infrastructure_failure(const char* operation) {
    std::printf("{\"status\":\"infrastructure_failure\",\"operation\":\"%s\"}\n", operation);
    std::fflush(stdout);
    std::exit(2);
}

[[noreturn]] void launch_failure(const char* reason) {
    std::printf("{\"status\":\"launch_failure\",\"reason\":\"%s\"}\n", reason);
    std::fflush(stdout);
    std::exit(1);
}

void require(cudaError_t status, const char* operation) {
    if (status != cudaSuccess) infrastructure_failure(operation);
}

const char* find_arg(int argc, char** argv, const char* name) {
    const size_t len = std::strlen(name);
    for (int i = 1; i < argc; ++i) {
        if (std::strncmp(argv[i], "--", 2) == 0 && std::strncmp(argv[i] + 2, name, len) == 0 &&
            argv[i][2 + len] == '=') {
            return argv[i] + 3 + len;
        }
    }
    return nullptr;
}

long long int_arg(int argc, char** argv, const char* name, long long fallback) {
    const char* v = find_arg(argc, argv, name);
    if (!v) return fallback;
    char* end = nullptr;
    long long out = std::strtoll(v, &end, 10);
    if (end == v || *end) infrastructure_failure("arguments");
    return out;
}

double float_arg(int argc, char** argv, const char* name, double fallback) {
    const char* v = find_arg(argc, argv, name);
    if (!v) return fallback;
    char* end = nullptr;
    double out = std::strtod(v, &end);
    if (end == v || *end) infrastructure_failure("arguments");
    return out;
}

std::string string_arg(int argc, char** argv, const char* name, const char* fallback) {
    const char* v = find_arg(argc, argv, name);
    return v ? std::string(v) : std::string(fallback);
}

// JSON number: finite values with %.9g, non-finite as the tokens Python's json
// module accepts.
void print_number(double v) {
    if (std::isnan(v)) {
        std::printf("NaN");
    } else if (std::isinf(v)) {
        std::printf(v > 0 ? "Infinity" : "-Infinity");
    } else {
        std::printf("%.9g", v);
    }
}

enum class Impl { kLibrary, kCublas, kCutlass };

struct Launch {
    int M, N, K, b_layout;
    kmcts_gemm_config cfg;
    cudaStream_t stream;
    int* status;
    Impl impl;
    cublasHandle_t cublas;
};

// cuBLAS exactly as the reference calls it (bf16_gemm_harness.cu:117-143):
// row-major C viewed as column-major C^T = B^T * A^T, FP32 compute.
bool cublas_gemm(const Launch& l, const void* A, const void* B, void* C) {
    const float alpha = 1.0f, beta = 0.0f;
    const cublasOperation_t op_b = l.b_layout == KMCTS_B_COL ? CUBLAS_OP_T : CUBLAS_OP_N;
    const int ldb = l.b_layout == KMCTS_B_COL ? l.K : l.N;
    return cublasGemmEx(l.cublas, op_b, CUBLAS_OP_N, l.N, l.M, l.K, &alpha, B, CUDA_R_16BF, ldb, A,
                        CUDA_R_16BF, l.K, &beta, C, CUDA_R_16BF, l.N, CUBLAS_COMPUTE_32F,
                        CUBLAS_GEMM_DEFAULT_TENSOR_OP) == CUBLAS_STATUS_SUCCESS;
}

// Returns 0 on success.
int launch_candidate(const Launch& l, const void* A, const void* B, void* C) {
#if defined(KMCTS_CANDIDATE_ROOT)
    dim3 block(16, 16, 1);
    dim3 grid((l.N + 15) / 16, (l.M + 15) / 16, 1);
    bf16_gemm_root<<<grid, block, 0, l.stream>>>(static_cast<const __nv_bfloat16*>(A),
                                                 static_cast<const __nv_bfloat16*>(B),
                                                 static_cast<__nv_bfloat16*>(C), l.M, l.N, l.K);
    return cudaGetLastError() == cudaSuccess ? 0 : 1;
#elif defined(KMCTS_CANDIDATE_LAUNCHER)
    return bf16_gemm_launch(A, B, C, l.M, l.N, l.K, l.stream) == 0 ? 0 : 1;
#else
    if (l.impl == Impl::kCublas) return cublas_gemm(l, A, B, C) ? 0 : 1;
#if KMCTS_HAVE_CUTLASS
    if (l.impl == Impl::kCutlass) return kmcts_vendor_cutlass_sm80_gemm(A, B, C, l.M, l.N, l.K, l.stream) == 0 ? 0 : 1;
#endif
    return kmcts_bf16_gemm_ex(A, B, C, l.M, l.N, l.K, l.b_layout, &l.cfg, l.stream, l.status);
#endif
}

const char* kernel_name(const Launch& l) {
#if defined(KMCTS_CANDIDATE_ROOT)
    (void)l;
    return "candidate:bf16_gemm_root";
#elif defined(KMCTS_CANDIDATE_LAUNCHER)
    (void)l;
    return "candidate:bf16_gemm_launch";
#else
    if (l.impl == Impl::kCublas) return "vendor:cublasGemmEx";
    if (l.impl == Impl::kCutlass) return "vendor:cutlass_sm80_128x128x32";
    return "library:kmcts_bf16_gemm_ex";
#endif
}

void check_device_status(const Launch& l) {
    int value = 0;
    require(cudaMemcpy(&value, l.status, sizeof(int), cudaMemcpyDeviceToHost), "read_status");
    if (value != 0) launch_failure("device_wait_timeout");
}

}  // namespace

int main(int argc, char** argv) {
    const std::string mode = string_arg(argc, argv, "mode", "");
    const long long M = int_arg(argc, argv, "M", 0);
    const long long N = int_arg(argc, argv, "N", 0);
    const long long K = int_arg(argc, argv, "K", 0);
    const int seed = static_cast<int>(int_arg(argc, argv, "seed", 0));
    const long long warmups = int_arg(argc, argv, "warmups", 10);
    const long long measurements = int_arg(argc, argv, "measurements", 30);
    const double rtol = float_arg(argc, argv, "rtol", 0.02);
    const double atol = float_arg(argc, argv, "atol", 0.02);
    const std::string layout = string_arg(argc, argv, "b-layout", "col");
    const std::string inputs = string_arg(argc, argv, "inputs", "uniform");
    const std::string kernel = string_arg(argc, argv, "kernel", "auto");
    const bool flush_l2 = int_arg(argc, argv, "flush-l2", 0) != 0;
    if ((mode != "correctness" && mode != "benchmark") || M <= 0 || N <= 0 || K <= 0 ||
        M > (1 << 30) || N > (1 << 30) || K > (1 << 30) || warmups < 0 || measurements <= 0 ||
        (layout != "col" && layout != "row") ||
        (inputs != "uniform" && inputs != "randn" && inputs != "int")) {
        infrastructure_failure("arguments");
    }

    Launch l{};
    l.M = static_cast<int>(M);
    l.N = static_cast<int>(N);
    l.K = static_cast<int>(K);
    l.b_layout = layout == "row" ? KMCTS_B_ROW : KMCTS_B_COL;
    kmcts_select_config(l.M, l.N, l.K, l.b_layout, &l.cfg);  // explicit schedule flags override it
    l.cfg.tile_m = static_cast<int>(int_arg(argc, argv, "tile-m", l.cfg.tile_m));
    l.cfg.cluster_m = static_cast<int>(int_arg(argc, argv, "cluster-m", l.cfg.cluster_m));
    l.cfg.cluster_n = static_cast<int>(int_arg(argc, argv, "cluster-n", l.cfg.cluster_n));
    l.cfg.flags = static_cast<int>(int_arg(argc, argv, "flags", l.cfg.flags));
    l.cfg.tile_n = static_cast<int>(int_arg(argc, argv, "tile-n", l.cfg.tile_n));
    l.cfg.tile_k = static_cast<int>(int_arg(argc, argv, "tile-k", l.cfg.tile_k));
    l.cfg.stages = static_cast<int>(int_arg(argc, argv, "stages", l.cfg.stages));
    l.cfg.persistent = static_cast<int>(int_arg(argc, argv, "persistent", l.cfg.persistent));
    l.cfg.raster_group = static_cast<int>(int_arg(argc, argv, "raster-group", l.cfg.raster_group));
    l.cfg.k_splits = static_cast<int>(int_arg(argc, argv, "k-splits", l.cfg.k_splits));
    l.cfg.wait_limit_ns = int_arg(argc, argv, "wait-limit-ns", 0);
    l.impl = Impl::kLibrary;
    if (kernel == "tcgen05") {
        l.cfg.kernel = KMCTS_KERNEL_TCGEN05;
    } else if (kernel == "simt") {
        l.cfg.kernel = KMCTS_KERNEL_SIMT;
    } else if (kernel == "cublas") {
        l.impl = Impl::kCublas;
    } else if (kernel == "cutlass_sm80") {
#if KMCTS_HAVE_CUTLASS
        if (layout != "col") infrastructure_failure("cutlass_layout");
        l.impl = Impl::kCutlass;
#else
        infrastructure_failure("cutlass_unavailable");
#endif
    } else if (kernel != "auto" && kernel != "candidate") {
        infrastructure_failure("arguments");
    }


    const size_t a_count = static_cast<size_t>(M) * K;
    const size_t b_count = static_cast<size_t>(K) * N;
    const size_t c_count = static_cast<size_t>(M) * N;
    // Inputs from the library's generator, so the in-process evaluator and
    // this executable see the same bits for the same (inputs, seed).
    std::vector<uint16_t> hA(a_count), hB(b_count);
    const int kind = inputs == "uniform" ? KMCTS_INPUTS_UNIFORM
                     : inputs == "randn" ? KMCTS_INPUTS_RANDN
                                         : KMCTS_INPUTS_INT;
    if (kmcts_generate_inputs(kind, static_cast<uint32_t>(seed), a_count, b_count, hA.data(), hB.data()) !=
        KMCTS_OK) {
        infrastructure_failure("inputs");
    }

    void *dA = nullptr, *dB = nullptr, *dC = nullptr, *dRef = nullptr, *dWork = nullptr,
         *dFlush = nullptr;
    require(cudaMalloc(&dA, a_count * 2), "cudaMalloc_A");
    require(cudaMalloc(&dB, b_count * 2), "cudaMalloc_B");
    require(cudaMalloc(&dC, c_count * 2), "cudaMalloc_C");
    require(cudaMalloc(reinterpret_cast<void**>(&l.status), sizeof(int)), "cudaMalloc_status");
    require(cudaMemset(l.status, 0, sizeof(int)), "memset_status");
    require(cudaMemcpy(dA, hA.data(), a_count * 2, cudaMemcpyHostToDevice), "copy_A");
    require(cudaMemcpy(dB, hB.data(), b_count * 2, cudaMemcpyHostToDevice), "copy_B");
    require(cudaStreamCreateWithFlags(&l.stream, cudaStreamNonBlocking), "stream");
    if (cublasCreate(&l.cublas) != CUBLAS_STATUS_SUCCESS) infrastructure_failure("cublasCreate");
    if (cublasSetStream(l.cublas, l.stream) != CUBLAS_STATUS_SUCCESS) infrastructure_failure("cublasSetStream");

    if (launch_candidate(l, dA, dB, dC) != 0) launch_failure("launch");
    if (cudaStreamSynchronize(l.stream) != cudaSuccess) launch_failure("synchronize");
    check_device_status(l);

    if (mode == "correctness") {
        require(cudaMalloc(&dRef, c_count * 2), "cudaMalloc_reference");
        if (!cublas_gemm(l, dA, dB, dRef)) infrastructure_failure("cublasGemmEx");
        require(cudaStreamSynchronize(l.stream), "reference_synchronize");
        require(cudaMalloc(&dWork, kmcts_compare_workspace_bytes()), "cudaMalloc_workspace");
        kmcts_compare_result r;
        if (kmcts_bf16_compare(dC, dRef, static_cast<int64_t>(c_count), rtol, atol, dWork, l.stream,
                               &r) != KMCTS_OK) {
            infrastructure_failure("compare");
        }
        std::printf("{\"status\":\"ok\",\"success\":%s,\"maximum_error\":", r.success ? "true" : "false");
        print_number(r.maximum_error);
        std::printf(",\"mean_error\":");
        print_number(r.mean_error);
        std::printf(",\"failed_test_id\":%s,", r.success ? "null" : "\"fixed_shape\"");
        std::printf("\"reference_metadata\":{\"implementation\":\"cuBLAS\","
                    "\"compute_type\":\"CUBLAS_COMPUTE_32F\",\"seed\":%d,\"inputs\":\"%s\","
                    "\"b_layout\":\"%s\"},",
                    seed, inputs.c_str(), layout.c_str());
        std::printf("\"max_ulp\":%d,\"n_gt_1ulp\":%lld,\"ulp_hist\":[%lld,%lld,%lld,%lld],"
                    "\"n_nonfinite\":%lld,\"kernel\":\"%s\"}\n",
                    r.max_ulp, static_cast<long long>(r.ulp_hist[2] + r.ulp_hist[3]),
                    static_cast<long long>(r.ulp_hist[0]), static_cast<long long>(r.ulp_hist[1]),
                    static_cast<long long>(r.ulp_hist[2]), static_cast<long long>(r.ulp_hist[3]),
                    static_cast<long long>(r.n_nonfinite), kernel_name(l));
    } else {
        // Reference protocol (bf16_gemm_harness.cu:177-212): warm-up launches,
        // one synchronize, then one event pair per measured launch.
        for (long long i = 0; i < warmups; ++i) {
            if (launch_candidate(l, dA, dB, dC) != 0) launch_failure("launch");
        }
        if (cudaStreamSynchronize(l.stream) != cudaSuccess) launch_failure("synchronize");
        const size_t flush_bytes = static_cast<size_t>(512) << 20;
        if (flush_l2) require(cudaMalloc(&dFlush, flush_bytes), "cudaMalloc_flush");
        cudaEvent_t start, stop;
        require(cudaEventCreate(&start), "event_start");
        require(cudaEventCreate(&stop), "event_stop");
        std::vector<float> timings(static_cast<size_t>(measurements));
        for (long long i = 0; i < measurements; ++i) {
            if (flush_l2)
                require(cudaMemsetAsync(dFlush, static_cast<int>(i & 0xff), flush_bytes, l.stream),
                        "flush_l2");
            require(cudaEventRecord(start, l.stream), "record_start");
            if (launch_candidate(l, dA, dB, dC) != 0) launch_failure("launch");
            require(cudaEventRecord(stop, l.stream), "record_stop");
            if (cudaEventSynchronize(stop) != cudaSuccess) launch_failure("synchronize");
            float ms = 0.0f;
            require(cudaEventElapsedTime(&ms, start, stop), "event_elapsed");
            timings[static_cast<size_t>(i)] = ms * 1000.0f;
        }
        check_device_status(l);
        std::printf("{\"status\":\"ok\",\"timings_us\":[");
        for (long long i = 0; i < measurements; ++i) {
            if (i) std::printf(",");
            std::printf("%.9g", timings[static_cast<size_t>(i)]);
        }
        std::printf("],\"kernel\":\"%s\"}\n", kernel_name(l));
        cudaEventDestroy(start);
        cudaEventDestroy(stop);
    }
    cudaFree(dA);
    cudaFree(dB);
    cudaFree(dC);
    cudaFree(dRef);
    cudaFree(dWork);
    cudaFree(dFlush);
    cudaFree(l.status);
    cublasDestroy(l.cublas);
    cudaStreamDestroy(l.stream);
    return 0;
}
