// Device workspaces for kernels that exchange partial results through global
// memory (the split-K and stream-K schedules): one per (device, stream, user).
//
// Launches on one stream run in order, so they may share a workspace;
// launches on different streams may overlap, so they may not.  A workspace is
// allocated zeroed on first use and grown (at least doubled) when a launch
// needs more.  Outgrown buffers are never freed: a CUDA graph captured
// earlier holds their address and may still replay.  Every buffer lives for
// the process.  Each
// call also advances the workspace's launch epoch, which the kernels write
// into their flags so that values left by an earlier failed launch are never
// taken for the current one's.
#include <cstring>
#include <mutex>
#include <thread>

#include "kmcts_internal.h"

namespace kmcts {
namespace {

struct Workspace {
    int device;
    cudaStream_t stream;
    std::thread::id thread;  // distinguishes per-thread default streams
    int user;
    void* ptr;
    size_t bytes;
    int epoch;
};

constexpr int kMaxWorkspaces = 128;

}  // namespace

bool stream_workspace(cudaStream_t stream, int user, size_t bytes, void** ptr, int* epoch) {
    static std::mutex mu;
    static Workspace spaces[kMaxWorkspaces];
    static int count = 0;
    int device = 0;
    if (cudaGetDevice(&device) != cudaSuccess) return false;
    const std::thread::id thread = stream == cudaStreamPerThread ? std::this_thread::get_id() : std::thread::id();
    std::lock_guard<std::mutex> lock(mu);
    Workspace* ws = nullptr;
    for (int i = 0; i < count; ++i) {
        const Workspace& w = spaces[i];
        if (w.device == device && w.stream == stream && w.thread == thread && w.user == user) ws = &spaces[i];
    }
    if (ws == nullptr) {
        if (count == kMaxWorkspaces) return false;
        ws = &spaces[count++];
        *ws = {device, stream, thread, user, nullptr, 0, 0};
    }
    if (ws->bytes < bytes) {
        // Allocation may not run while the stream is being captured.
        cudaStreamCaptureStatus capture = cudaStreamCaptureStatusNone;
        if (cudaStreamIsCapturing(stream, &capture) != cudaSuccess || capture != cudaStreamCaptureStatusNone) {
            cudaGetLastError();
            return false;
        }
        const size_t grown = bytes > 2 * ws->bytes ? bytes : 2 * ws->bytes;
        void* p = nullptr;
        if (cudaMalloc(&p, grown) != cudaSuccess) {
            cudaGetLastError();
            return false;
        }
        if (cudaMemset(p, 0, grown) != cudaSuccess) {
            cudaGetLastError();
            cudaFree(p);
            return false;
        }
        // The outgrown buffer stays allocated (see above).
        ws->ptr = p;
        ws->bytes = grown;
    }
    ws->epoch = ws->epoch % 0x7fffffff + 1;  // never 0, the cleared state
    *ptr = ws->ptr;
    *epoch = ws->epoch;
    return true;
}

}  // namespace kmcts
