// C = A·B for operands in host memory: the copies over PCIe and the GEMM
// overlap.  A goes over in row blocks and B in column blocks, interleaved
// (A0, B0, A1, B1, ...); each C block (i, j) is computed as soon as A block i
// and B block j have landed, and goes back at once, so the device-to-host
// direction starts after two blocks instead of after all of B and the two
// directions of the link are busy together for most of the call.
// Host-to-device copies run on one internal stream, device-to-host copies on
// another, the GEMMs on the caller's stream, ordered by events; the caller's
// stream waits for the last copy back, so the call is asynchronous on
// `stream` like every other entry point.
//
// Device buffers are scratch: a B column block is kept as its own dense
// matrix ([K, cb] for row-major B; a row slice already for column-major B)
// and each C block as a dense [rb, cb] matrix, so every block GEMM is a
// plain dense call; the copies back scatter the C blocks into the host C.
// Every block uses one schedule, the one the call would use on the whole
// problem, so the host C is bit-identical to kmcts_bf16_gemm_ex on it (each
// output is the same K-ordered chain in either).
#include <mutex>

#include "kmcts_internal.h"

namespace kmcts {
namespace {

constexpr int kMaxDevices = 64;

struct CopyStreams {
    cudaStream_t in = nullptr, out = nullptr;
};

bool copy_streams(CopyStreams* out) {
    static std::mutex mu;
    static CopyStreams streams[kMaxDevices];
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess || device < 0 || device >= kMaxDevices) return false;
    std::lock_guard<std::mutex> lock(mu);
    CopyStreams& s = streams[device];
    if (!s.in) {
        if (cudaStreamCreateWithFlags(&s.in, cudaStreamNonBlocking) != cudaSuccess) return false;
        if (cudaStreamCreateWithFlags(&s.out, cudaStreamNonBlocking) != cudaSuccess) {
            cudaStreamDestroy(s.in);
            s.in = nullptr;
            return false;
        }
    }
    *out = s;
    return true;
}

}  // namespace
}  // namespace kmcts

using namespace kmcts;

namespace kmcts {
namespace {

// Block edges: `count` blocks of a multiple of `quantum` (the last one ragged).
int block_size(int extent, int count, int quantum) {
    const int per = (extent + count - 1) / count;
    return (per + quantum - 1) / quantum * quantum;
}

}  // namespace
}  // namespace kmcts

extern "C" int kmcts_bf16_gemm_host(const void* A_host, const void* B_host, void* C_host, void* A_dev, void* B_dev,
                                    void* C_dev, int M, int N, int K, int b_layout, const kmcts_gemm_config* cfg,
                                    int chunks, void* stream, int* device_status) {
    if (M < 0 || N < 0 || K < 0 || (b_layout != KMCTS_B_COL && b_layout != KMCTS_B_ROW)) return KMCTS_EINVAL;
    if (M == 0 || N == 0) return KMCTS_OK;
    if (!A_host || !B_host || !C_host || !A_dev || !B_dev || !C_dev) return KMCTS_EINVAL;
    // One schedule for every block: the caller's, or the one chosen for the whole problem.
    kmcts_gemm_config schedule;
    if (cfg) {
        schedule = *cfg;
    } else if (kmcts_select_config(M, N, K, b_layout, &schedule) != KMCTS_OK) {
        return KMCTS_EINVAL;
    }
    if (chunks <= 0) chunks = 4;  // blocks per dimension; 4 x 4 measured best at 4096^3
    const int rows = block_size(M, chunks, 128);  // whole 128-row tiles per row block
    const int cols = N >= 2 * 256 ? block_size(N, chunks, 256) : N;  // whole 256-column tiles
    const int row_blocks = (M + rows - 1) / rows, col_blocks = (N + cols - 1) / cols;
    CopyStreams cs;
    if (!copy_streams(&cs)) return KMCTS_EHANDLE;
    cudaStream_t s = static_cast<cudaStream_t>(stream);
    const size_t esize = 2;  // BF16
    const char* a_host = static_cast<const char*>(A_host);
    const char* b_host = static_cast<const char*>(B_host);
    char* c_host = static_cast<char*>(C_host);
    char* a_dev = static_cast<char*>(A_dev);
    char* b_dev = static_cast<char*>(B_dev);
    char* c_dev = static_cast<char*>(C_dev);
    int rc = KMCTS_OK;
    const unsigned flags = cudaEventDisableTiming;
    cudaEvent_t start = nullptr, done_out = nullptr;
    if (cudaEventCreateWithFlags(&start, flags) != cudaSuccess || cudaEventCreateWithFlags(&done_out, flags) != cudaSuccess)
        rc = KMCTS_EHANDLE;
    // The copies start after the work already queued on the caller's stream.
    if (rc == KMCTS_OK && (cudaEventRecord(start, s) != cudaSuccess || cudaStreamWaitEvent(cs.in, start, 0) != cudaSuccess ||
                           cudaStreamWaitEvent(cs.out, start, 0) != cudaSuccess))
        rc = KMCTS_ESYNC;
    int have_a = 0, have_b = 0;  // blocks landed (in order)
    for (int step = 0; rc == KMCTS_OK && (have_a < row_blocks || have_b < col_blocks); ++step) {
        // Next copy in: A and B blocks alternate while both have some left.
        const bool take_a = have_a < row_blocks && (have_b >= col_blocks || have_a <= have_b);
        if (take_a) {
            const size_t r0 = static_cast<size_t>(have_a) * rows;
            const int rb = M - static_cast<int>(r0) < rows ? M - static_cast<int>(r0) : rows;
            const size_t bytes = static_cast<size_t>(rb) * K * esize;
            if (bytes && cudaMemcpyAsync(a_dev + r0 * K * esize, a_host + r0 * K * esize, bytes, cudaMemcpyHostToDevice,
                                         cs.in) != cudaSuccess)
                rc = KMCTS_ESYNC;
        } else {
            const size_t c0 = static_cast<size_t>(have_b) * cols;
            const int cb = N - static_cast<int>(c0) < cols ? N - static_cast<int>(c0) : cols;
            if (K > 0) {
                cudaError_t err;
                if (b_layout == KMCTS_B_COL) {  // B [N, K]: the block is a row slice
                    err = cudaMemcpyAsync(b_dev + c0 * K * esize, b_host + c0 * K * esize,
                                          static_cast<size_t>(cb) * K * esize, cudaMemcpyHostToDevice, cs.in);
                } else {  // B [K, N]: gather the block's columns into a dense [K, cb]
                    err = cudaMemcpy2DAsync(b_dev + c0 * K * esize, static_cast<size_t>(cb) * esize, b_host + c0 * esize,
                                            static_cast<size_t>(N) * esize, static_cast<size_t>(cb) * esize, K,
                                            cudaMemcpyHostToDevice, cs.in);
                }
                if (err != cudaSuccess) rc = KMCTS_ESYNC;
            }
        }
        cudaEvent_t landed = nullptr;
        if (rc == KMCTS_OK && cudaEventCreateWithFlags(&landed, flags) != cudaSuccess) rc = KMCTS_EHANDLE;
        if (rc == KMCTS_OK && (cudaEventRecord(landed, cs.in) != cudaSuccess || cudaStreamWaitEvent(s, landed, 0) != cudaSuccess))
            rc = KMCTS_ESYNC;
        if (landed) cudaEventDestroy(landed);  // released once the recorded work completes
        const int prev_a = have_a, prev_b = have_b;
        if (take_a) ++have_a; else ++have_b;
        // Every C block that just became computable: the new A block with all
        // B blocks in, or the new B block with all A blocks in.
        for (int i = 0; rc == KMCTS_OK && i < have_a; ++i) {
            for (int j = 0; rc == KMCTS_OK && j < have_b; ++j) {
                if (i < prev_a && j < prev_b) continue;  // computed before
                const size_t r0 = static_cast<size_t>(i) * rows, c0 = static_cast<size_t>(j) * cols;
                const int rb = M - static_cast<int>(r0) < rows ? M - static_cast<int>(r0) : rows;
                const int cb = N - static_cast<int>(c0) < cols ? N - static_cast<int>(c0) : cols;
                char* c_block = c_dev + (r0 * N + static_cast<size_t>(rb) * c0) * esize;  // dense [rb, cb]
                rc = kmcts_bf16_gemm_ex(a_dev + r0 * K * esize, b_dev + c0 * K * esize, c_block, rb, cb, K, b_layout,
                                        &schedule, s, device_status);
                cudaEvent_t computed = nullptr;
                if (rc == KMCTS_OK && cudaEventCreateWithFlags(&computed, flags) != cudaSuccess) rc = KMCTS_EHANDLE;
                if (rc == KMCTS_OK &&
                    (cudaEventRecord(computed, s) != cudaSuccess || cudaStreamWaitEvent(cs.out, computed, 0) != cudaSuccess ||
                     cudaMemcpy2DAsync(c_host + (r0 * N + c0) * esize, static_cast<size_t>(N) * esize, c_block,
                                       static_cast<size_t>(cb) * esize, static_cast<size_t>(cb) * esize, rb,
                                       cudaMemcpyDeviceToHost, cs.out) != cudaSuccess))
                    rc = KMCTS_ESYNC;
                if (computed) cudaEventDestroy(computed);
            }
        }
    }
    // The caller's stream ends after the last copy in each direction (also on
    // an error part-way, when a copy in may have no GEMM after it), so nothing
    // outlives the call unordered.
    if (done_out) {
        if (cudaEventRecord(done_out, cs.out) != cudaSuccess || cudaStreamWaitEvent(s, done_out, 0) != cudaSuccess ||
            cudaEventRecord(done_out, cs.in) != cudaSuccess || cudaStreamWaitEvent(s, done_out, 0) != cudaSuccess)
            rc = rc == KMCTS_OK ? KMCTS_ESYNC : rc;
        cudaEventDestroy(done_out);
    }
    if (start) cudaEventDestroy(start);
    return rc;
}
