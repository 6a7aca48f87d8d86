// Self-test of the bounded device-side wait that every GEMM barrier uses.
//
// One thread initialises an mbarrier expecting one arrival.  With `arrive`
// set it arrives first (the phase completes; the wait returns at once);
// without it nothing ever arrives (a flag nothing sets), so the bounded wait
// must give up after `limit_ns` and report KMCTS_ETIMEOUT in the status word.
// No TMA, no TMEM, no other CTA is involved: the test exercises the timeout
// path with nothing in flight.
#include "gemm_common.cuh"
#include "kmcts_internal.h"

namespace kmcts {
namespace {

__global__ void bounded_wait_probe(uint64_t limit_ns, int arrive, int* status, unsigned long long* waited_ns) {
    __shared__ uint64_t bar;
    __shared__ int abort;
    if (threadIdx.x != 0) return;
    abort = 0;
    ptx::mbar_init(&bar, 1);
    ptx::fence_mbarrier_init();
    if (arrive) ptx::mbar_arrive(&bar);
    const uint64_t start = ptx::global_timer_ns();
    const bool ok = ptx::mbar_wait(&bar, 0, limit_ns, &abort);
    *waited_ns = ptx::global_timer_ns() - start;
    if (!ok) atomicCAS(status, 0, KMCTS_ETIMEOUT | (gemm::kRoleMma << 8));
}

}  // namespace
}  // namespace kmcts

extern "C" int kmcts_selftest_bounded_wait(int64_t limit_ns, int arrive, void* stream, int* device_status,
                                           unsigned long long* device_waited_ns) {
    using namespace kmcts;
    if (limit_ns <= 0 || limit_ns > 10000000000ll || !device_status || !device_waited_ns) return KMCTS_EINVAL;
    bounded_wait_probe<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<uint64_t>(limit_ns), arrive,
                                                                         device_status, device_waited_ns);
    g_launches.fetch_add(1, std::memory_order_relaxed);
    return cudaGetLastError() == cudaSuccess ? KMCTS_OK : KMCTS_EGEMM;
}
