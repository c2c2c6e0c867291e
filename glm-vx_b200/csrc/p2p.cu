// Peer-memory exchange between the GPUs of one node (NVLink / NVSwitch), the
// data movement of the expert-parallel layer step without a collective
// library: every rank exposes a mailbox (cudaMalloc'd, mapped by its peers
// through CUDA IPC handles); a sender's kernel stores its rows straight into
// each destination's mailbox, then publishes an epoch number in the
// destination's flag slot for this sender (release at system scope); a
// receiver's kernel waits (bounded) until every sender's flag reached the
// epoch (acquire at system scope).  Plain peer loads/stores only: no
// multicast, no NVLink SHARP objects.
#include <cstdint>
#include <cstring>

#include "common.cuh"

namespace glmvx {

namespace {

constexpr int kP2pMaxWorld = 8, kP2pThreads = 256;

// Row ranges of one scatter: rows [src_begin[d], src_begin[d + 1]) of the
// send buffer go to dst[d] starting at row dst_row[d] (row_bytes each).
struct P2pScatter {
    char *dst[kP2pMaxWorld];
    int64_t src_begin[kP2pMaxWorld + 1];  // prefix over destinations; src_begin[world] = total rows
    int64_t dst_row[kP2pMaxWorld];
    int world;
};

__global__ void __launch_bounds__(kP2pThreads) p2p_scatter_kernel(const char *__restrict__ src, int64_t row_bytes,
                                                                  P2pScatter sc) {
    const int64_t total = sc.src_begin[sc.world];
    const int64_t vec = row_bytes / 16;  // 16-byte units (row_bytes % 16 == 0)
    for (int64_t row = blockIdx.x; row < total; row += gridDim.x) {
        int d = 0;
        while (d + 1 < sc.world && row >= sc.src_begin[d + 1]) ++d;
        const int4 *s = reinterpret_cast<const int4 *>(src + row * row_bytes);
        int4 *t = reinterpret_cast<int4 *>(sc.dst[d] + (sc.dst_row[d] + row - sc.src_begin[d]) * row_bytes);
        for (int64_t i = threadIdx.x; i < vec; i += kP2pThreads) t[i] = s[i];
    }
    __threadfence_system();  // the rows are visible system-wide before this kernel ends
}

__global__ void p2p_signal_kernel(P2pScatter flags, uint32_t epoch) {
    // flags.dst[d]: this rank's flag slot in rank d's mailbox.
    const int d = threadIdx.x;
    if (d >= flags.world) return;
    __threadfence_system();
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(flags.dst[d]), "r"(epoch) : "memory");
}

// One thread per sender: wait until flags[s] reached epoch (wrap-safe), at
// most 2 s; then the device error word is set instead.
__global__ void p2p_wait_kernel(const uint32_t *flags, int world, uint32_t epoch, int *err) {
    const int s = threadIdx.x;
    if (s >= world) return;
    const uint64_t start = globaltimer_ns();
    for (;;) {
        uint32_t v;
        asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(flags + s) : "memory");
        if (static_cast<int32_t>(v - epoch) >= 0) return;
        if (globaltimer_ns() - start > 2000000000ull) {  // a peer is gone or stuck
            report_device_error(err, kDevErrFullWait);
            return;
        }
        __nanosleep(200);
    }
}

int32_t fill_scatter(P2pScatter &sc, void *const *dst, const int64_t *counts, const int64_t *dst_rows, int world) {
    if (world < 1 || world > kP2pMaxWorld || !dst || !counts)
        return set_error("p2p: world must be 1..%d and arrays set", kP2pMaxWorld), kInvalid;
    std::memset(&sc, 0, sizeof(sc));
    sc.world = world;
    for (int d = 0; d < world; ++d) {
        if (counts[d] < 0 || (counts[d] && !dst[d])) return set_error("p2p: bad count or null destination"), kInvalid;
        sc.dst[d] = static_cast<char *>(dst[d]);
        sc.dst_row[d] = dst_rows ? dst_rows[d] : 0;
        sc.src_begin[d + 1] = sc.src_begin[d] + counts[d];
    }
    return kOk;
}

}  // namespace

}  // namespace glmvx

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

// Rows of `src` grouped by destination (counts[d] rows for rank d, in rank
// order) stored into dst[d] from row dst_rows[d] (dst_rows NULL: row 0),
// row_bytes each (a multiple of 16; src and every dst 16-byte aligned).
// dst[d] may be this rank's own memory or a mapped peer allocation.
GLMVX_EXPORT int32_t glmvx_p2p_scatter(const void *src, int64_t row_bytes, void *const *dst, const int64_t *counts,
                                       const int64_t *dst_rows, int32_t world, void *stream) {
    P2pScatter sc;
    if (const int32_t rc = fill_scatter(sc, dst, counts, dst_rows, world)) return rc;
    if (row_bytes <= 0 || row_bytes % 16 || (reinterpret_cast<uintptr_t>(src) & 15)) {
        set_error("p2p_scatter: row_bytes a positive multiple of 16, src 16-byte aligned");
        return kInvalid;
    }
    for (int d = 0; d < world; ++d)
        if (counts[d] && (reinterpret_cast<uintptr_t>(dst[d]) & 15))
            return set_error("p2p_scatter: destinations 16-byte aligned"), kInvalid;
    const int64_t total = sc.src_begin[world];
    if (total == 0) return kOk;
    const int grid = static_cast<int>(total < 4 * 148 ? total : 4 * 148);
    p2p_scatter_kernel<<<grid, kP2pThreads, 0, static_cast<cudaStream_t>(stream)>>>(static_cast<const char *>(src),
                                                                                    row_bytes, sc);
    GLMVX_CUDA(cudaGetLastError());
    return kOk;
}

// Publishes `epoch` in every peer's flag slot for this rank (flag_slots[d]:
// device address, in rank d's mailbox, of this rank's flag) once this
// stream's earlier stores are visible system-wide.
GLMVX_EXPORT int32_t glmvx_p2p_signal(void *const *flag_slots, int32_t world, uint32_t epoch, void *stream) {
    if (world < 1 || world > kP2pMaxWorld) return set_error("p2p_signal: world must be 1..%d", kP2pMaxWorld), kInvalid;
    P2pScatter sc;
    int64_t ones[kP2pMaxWorld];
    for (int d = 0; d < world; ++d) ones[d] = 1;
    if (const int32_t rc = fill_scatter(sc, flag_slots, ones, nullptr, world)) return rc;
    p2p_signal_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(sc, epoch);
    GLMVX_CUDA(cudaGetLastError());
    return kOk;
}

// Waits on the device until flags[s] reached epoch for every sender s < world
// (this rank's mailbox); after 2 s the device error word is set instead.
GLMVX_EXPORT int32_t glmvx_p2p_wait(const uint32_t *flags, int32_t world, uint32_t epoch, void *stream) {
    if (!flags || world < 1 || world > kP2pMaxWorld) return set_error("p2p_wait: bad arguments"), kInvalid;
    p2p_wait_kernel<<<1, 32, 0, static_cast<cudaStream_t>(stream)>>>(flags, world, epoch, device_error_word());
    GLMVX_CUDA(cudaGetLastError());
    return kOk;
}
