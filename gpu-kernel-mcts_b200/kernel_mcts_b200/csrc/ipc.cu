// CUDA IPC for the N-sharded GEMM: each rank exports the device buffer that
// holds its full C, imports its peers' buffers, and the fused kernel stores
// finished tiles straight into them over NVLink (plain peer stores; no
// multicast objects, no NVLS).
//
// A handle is KMCTS_IPC_HANDLE_BYTES: the cudaIpcMemHandle_t of the
// allocation that contains the pointer, then the pointer's byte offset from
// that allocation's base (caching allocators hand out sub-ranges).
#include <cudaTypedefs.h>

#include <cstring>
#include <mutex>

#include "kmcts_internal.h"

namespace {

PFN_cuMemGetAddressRange_v3020 address_range_fn() {
    static std::once_flag once;
    static PFN_cuMemGetAddressRange_v3020 fn = nullptr;
    std::call_once(once, [] {
        void* entry = nullptr;
        cudaDriverEntryPointQueryResult query;
        if (cudaGetDriverEntryPointByVersion("cuMemGetAddressRange", &entry, 12000, cudaEnableDefault, &query) ==
                cudaSuccess &&
            query == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<PFN_cuMemGetAddressRange_v3020>(entry);
    });
    return fn;
}

bool allocation_base(const void* ptr, uintptr_t* base) {
    auto fn = address_range_fn();
    if (!fn) return false;
    CUdeviceptr b = 0;
    size_t size = 0;
    if (fn(&b, &size, reinterpret_cast<CUdeviceptr>(ptr)) != CUDA_SUCCESS) return false;
    *base = static_cast<uintptr_t>(b);
    return true;
}

}  // namespace

extern "C" {

int kmcts_ipc_export(const void* device_ptr, uint8_t* handle_out) {
    if (!device_ptr || !handle_out) return KMCTS_EINVAL;
    static_assert(sizeof(cudaIpcMemHandle_t) + sizeof(uint64_t) <= KMCTS_IPC_HANDLE_BYTES, "IPC handle size");
    uintptr_t base = 0;
    if (!allocation_base(device_ptr, &base)) return KMCTS_EHANDLE;
    cudaIpcMemHandle_t handle;
    if (cudaIpcGetMemHandle(&handle, reinterpret_cast<void*>(base)) != cudaSuccess) {
        cudaGetLastError();
        return KMCTS_EHANDLE;
    }
    const uint64_t offset = reinterpret_cast<uintptr_t>(device_ptr) - base;
    std::memset(handle_out, 0, KMCTS_IPC_HANDLE_BYTES);
    std::memcpy(handle_out, &handle, sizeof(handle));
    std::memcpy(handle_out + sizeof(handle), &offset, sizeof(offset));
    return KMCTS_OK;
}

int kmcts_ipc_import(const uint8_t* handle, void** device_ptr_out) {
    if (!handle || !device_ptr_out) return KMCTS_EINVAL;
    cudaIpcMemHandle_t h;
    uint64_t offset = 0;
    std::memcpy(&h, handle, sizeof(h));
    std::memcpy(&offset, handle + sizeof(h), sizeof(offset));
    void* base = nullptr;
    if (cudaIpcOpenMemHandle(&base, h, cudaIpcMemLazyEnablePeerAccess) != cudaSuccess) {
        cudaGetLastError();
        return KMCTS_EHANDLE;
    }
    *device_ptr_out = static_cast<char*>(base) + offset;
    return KMCTS_OK;
}

int kmcts_ipc_close(void* device_ptr) {
    if (!device_ptr) return KMCTS_EINVAL;
    uintptr_t base = 0;
    if (!allocation_base(device_ptr, &base)) return KMCTS_EHANDLE;
    if (cudaIpcCloseMemHandle(reinterpret_cast<void*>(base)) != cudaSuccess) {
        cudaGetLastError();
        return KMCTS_EHANDLE;
    }
    return KMCTS_OK;
}

int kmcts_copy_2d(void* dst, size_t dst_pitch, const void* src, size_t src_pitch, size_t width_bytes,
                  size_t height, void* stream) {
    if (!dst || !src || width_bytes > dst_pitch || width_bytes > src_pitch) return KMCTS_EINVAL;
    if (width_bytes == 0 || height == 0) return KMCTS_OK;
    if (cudaMemcpy2DAsync(dst, dst_pitch, src, src_pitch, width_bytes, height, cudaMemcpyDeviceToDevice,
                          static_cast<cudaStream_t>(stream)) != cudaSuccess) {
        cudaGetLastError();
        return KMCTS_ESYNC;
    }
    return KMCTS_OK;
}

}  // extern "C"
