// CUDA IPC mapping of device allocations between the rank processes of one
// node: the expert-parallel layer (ep.cu) shares its mailbox this way, and
// its kernels then store into the peers' mailboxes with plain peer stores
// over NVLink / NVSwitch (no multicast object).
#include <cstring>

#include "common.cuh"

using namespace glmvx;

// 64-byte CUDA IPC handle of a cudaMalloc'd base pointer (for the peers to map).
GLMVX_EXPORT int32_t glmvx_ipc_handle(void *base, uint8_t *handle64) {
    if (!base || !handle64) return set_error("ipc_handle: null pointer"), kInvalid;
    cudaIpcMemHandle_t h;
    GLMVX_CUDA(cudaIpcGetMemHandle(&h, base));
    std::memcpy(handle64, &h, sizeof(h));
    return kOk;
}

// Maps another process's allocation from its 64-byte handle (peer access
// enabled on first use).
GLMVX_EXPORT int32_t glmvx_ipc_open(const uint8_t *handle64, void **ptr) {
    if (!handle64 || !ptr) return set_error("ipc_open: null pointer"), kInvalid;
    cudaIpcMemHandle_t h;
    std::memcpy(&h, handle64, sizeof(h));
    GLMVX_CUDA(cudaIpcOpenMemHandle(ptr, h, cudaIpcMemLazyEnablePeerAccess));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_ipc_close(void *ptr) {
    if (!ptr) return kOk;
    GLMVX_CUDA(cudaIpcCloseMemHandle(ptr));
    return kOk;
}
