// Device runtime exported over the C ABI: error reporting, devices, memory,
// streams, events and CUDA graphs.  This replaces the reference's ctypes
// CUDA Driver API runtime (gpu/runtime.py:76-663) with a thin native layer;
// the Python side (gpu/runtime.py in this package) only marshals pointers.
#include <algorithm>
#include <cstdarg>
#include <cstdio>
#include <map>
#include <mutex>
#include <utility>

#include "common.cuh"

namespace glmvx {

static thread_local char g_last_error[512] = "";

void set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_last_error, sizeof g_last_error, fmt, ap);
    va_end(ap);
}

int32_t cuda_fail(cudaError_t e, const char *what) {
    set_error("%s failed: %s (%s)", what, cudaGetErrorName(e), cudaGetErrorString(e));
    return kCudaError;
}

int32_t launch_status(const char *kernel) {
    cudaError_t e = cudaGetLastError();
    if (e != cudaSuccess) {
        set_error("launch of %s failed: %s (%s)", kernel, cudaGetErrorName(e), cudaGetErrorString(e));
        return kCudaError;
    }
    return kOk;
}

// One error word per device, in device global memory.
static __device__ int g_device_error;

int *device_error_word() {
    int *p = nullptr;
    if (cudaGetSymbolAddress(reinterpret_cast<void **>(&p), g_device_error) != cudaSuccess) return nullptr;
    return p;
}

int sm_count() {
    static std::mutex mu;
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 148;
    std::lock_guard<std::mutex> lock(mu);
    if (!cached[dev]) {
        int n = 0;
        cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;  // the first query may come during a capture
        cudaThreadExchangeStreamCaptureMode(&mode);
        cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev);
        cudaThreadExchangeStreamCaptureMode(&mode);
        cached[dev] = n > 0 ? n : 148;
    }
    return cached[dev];
}

int32_t allow_dynamic_smem(const void *kernel, size_t bytes, const char *name) {
    if (bytes <= 48 * 1024) return kOk;  // below the default limit nothing needs raising
    int dev = 0;
    GLMVX_CUDA(cudaGetDevice(&dev));
    static std::mutex mu;
    static std::map<std::pair<int, const void *>, size_t> raised;  // (device, kernel) -> bytes allowed
    std::lock_guard<std::mutex> lock(mu);
    size_t &have = raised[{dev, kernel}];
    if (have >= bytes) return kOk;
    // The first launch may happen while this thread captures a graph: let
    // this one non-stream call through (relaxed mode) without invalidating it.
    cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
    cudaThreadExchangeStreamCaptureMode(&mode);
    const cudaError_t e =
        cudaFuncSetAttribute(kernel, cudaFuncAttributeMaxDynamicSharedMemorySize, static_cast<int>(bytes));
    cudaThreadExchangeStreamCaptureMode(&mode);
    if (e != cudaSuccess) return cuda_fail(e, name);
    have = bytes;
    return kOk;
}

}  // namespace glmvx

using namespace glmvx;

GLMVX_EXPORT const char *glmvx_last_error(void) { return g_last_error; }

GLMVX_EXPORT int32_t glmvx_version(void) { return 1; }

GLMVX_EXPORT int32_t glmvx_device_count(int32_t *count) {
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e == cudaErrorNoDevice || e == cudaErrorInsufficientDriver) {
        *count = 0;
        cudaGetLastError();
        return kOk;
    }
    GLMVX_CUDA(e);
    *count = n;
    return kOk;
}

// Makes `device` current for this thread.  Callers activate their device
// before every step; a device that is already current (cudaGetDevice reads
// the runtime's thread state) is left alone.
GLMVX_EXPORT int32_t glmvx_set_device(int32_t device) {
    int current = -1;
    if (cudaGetDevice(&current) == cudaSuccess && current == device) return kOk;
    GLMVX_CUDA(cudaSetDevice(device));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_get_device(int32_t *device) {
    int d = 0;
    GLMVX_CUDA(cudaGetDevice(&d));
    *device = d;
    return kOk;
}

// name: caller buffer of name_len bytes.  cc = major*10+minor.
GLMVX_EXPORT int32_t glmvx_device_info(int32_t device, char *name, int32_t name_len, int32_t *cc,
                                       int32_t *sms, int64_t *l2_bytes, int64_t *total_mem,
                                       int32_t *smem_optin) {
    cudaDeviceProp p;
    GLMVX_CUDA(cudaGetDeviceProperties(&p, device));
    if (name && name_len > 0) snprintf(name, name_len, "%s", p.name);
    if (cc) *cc = p.major * 10 + p.minor;
    if (sms) *sms = p.multiProcessorCount;
    if (l2_bytes) *l2_bytes = p.l2CacheSize;
    if (total_mem) *total_mem = static_cast<int64_t>(p.totalGlobalMem);
    if (smem_optin) *smem_optin = static_cast<int32_t>(p.sharedMemPerBlockOptin);
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_malloc(void **ptr, uint64_t bytes) {
    *ptr = nullptr;
    if (bytes == 0) return kOk;
    GLMVX_CUDA(cudaMalloc(ptr, bytes));
    return kOk;
}

// Free and total bytes of device memory on the current device (cudaMemGetInfo).
GLMVX_EXPORT int32_t glmvx_mem_get_info(uint64_t *free_bytes, uint64_t *total_bytes) {
    size_t f = 0, t = 0;
    GLMVX_CUDA(cudaMemGetInfo(&f, &t));
    if (free_bytes) *free_bytes = f;
    if (total_bytes) *total_bytes = t;
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_free(void *ptr) {
    if (ptr) GLMVX_CUDA(cudaFree(ptr));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_host_alloc(void **ptr, uint64_t bytes) {
    *ptr = nullptr;
    if (bytes == 0) return kOk;
    GLMVX_CUDA(cudaMallocHost(ptr, bytes));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_host_free(void *ptr) {
    if (ptr) GLMVX_CUDA(cudaFreeHost(ptr));
    return kOk;
}

// Asynchronous copies on `stream` (nullptr = legacy default stream).  Copies
// from pageable host memory are staged by the driver and return once the
// source may be reused.
GLMVX_EXPORT int32_t glmvx_memcpy_htod(void *dst, const void *src, uint64_t bytes, void *stream) {
    if (bytes) GLMVX_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_memcpy_dtoh(void *dst, const void *src, uint64_t bytes, void *stream) {
    if (bytes) GLMVX_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_memcpy_dtod(void *dst, const void *src, uint64_t bytes, void *stream) {
    if (bytes) GLMVX_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_memset(void *dst, int32_t value, uint64_t bytes, void *stream) {
    if (bytes) GLMVX_CUDA(cudaMemsetAsync(dst, value, bytes, (cudaStream_t)stream));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_device_synchronize(void) {
    GLMVX_CUDA(cudaDeviceSynchronize());
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_stream_create(void **stream) {
    cudaStream_t s;
    GLMVX_CUDA(cudaStreamCreateWithFlags(&s, cudaStreamNonBlocking));
    *stream = s;
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_stream_destroy(void *stream) {
    if (stream) GLMVX_CUDA(cudaStreamDestroy((cudaStream_t)stream));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_stream_synchronize(void *stream) {
    GLMVX_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_event_create(void **event) {
    cudaEvent_t e;
    GLMVX_CUDA(cudaEventCreate(&e));
    *event = e;
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_event_destroy(void *event) {
    if (event) GLMVX_CUDA(cudaEventDestroy((cudaEvent_t)event));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_event_record(void *event, void *stream) {
    GLMVX_CUDA(cudaEventRecord((cudaEvent_t)event, (cudaStream_t)stream));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_event_synchronize(void *event) {
    GLMVX_CUDA(cudaEventSynchronize((cudaEvent_t)event));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_event_elapsed_ms(void *start, void *end, float *ms) {
    GLMVX_CUDA(cudaEventElapsedTime(ms, (cudaEvent_t)start, (cudaEvent_t)end));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_stream_wait_event(void *stream, void *event) {
    GLMVX_CUDA(cudaStreamWaitEvent((cudaStream_t)stream, (cudaEvent_t)event, 0));
    return kOk;
}

// Stream capture into a CUDA graph: begin, launch work on `stream`, end.
GLMVX_EXPORT int32_t glmvx_graph_begin(void *stream) {
    GLMVX_CUDA(cudaStreamBeginCapture((cudaStream_t)stream, cudaStreamCaptureModeThreadLocal));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_graph_end(void *stream, void **graph_exec) {
    cudaGraph_t g = nullptr;
    GLMVX_CUDA(cudaStreamEndCapture((cudaStream_t)stream, &g));
    cudaGraphExec_t exec = nullptr;
    cudaError_t e = cudaGraphInstantiate(&exec, g, 0);
    cudaGraphDestroy(g);
    GLMVX_CUDA(e);
    *graph_exec = exec;
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_graph_launch(void *graph_exec, void *stream) {
    GLMVX_CUDA(cudaGraphLaunch((cudaGraphExec_t)graph_exec, (cudaStream_t)stream));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_graph_destroy(void *graph_exec) {
    if (graph_exec) GLMVX_CUDA(cudaGraphExecDestroy((cudaGraphExec_t)graph_exec));
    return kOk;
}

// Reads and clears the current device's kernel error word.  *code is 0 when
// no kernel reported a timeout; otherwise the first DeviceError recorded.
// Device address of that word, so a caller can copy it back together with a
// step's outputs (one transfer, one synchronisation) and call
// glmvx_check_device_error only when it is nonzero.
GLMVX_EXPORT int32_t glmvx_device_error_address(void **ptr) {
    if (!ptr) {
        set_error("device_error_address: null output pointer");
        return kInvalid;
    }
    int *word = device_error_word();
    if (!word) return cuda_fail(cudaGetLastError(), "cudaGetSymbolAddress(g_device_error)");
    *ptr = word;
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_check_device_error(int32_t *code) {
    int *word = device_error_word();
    if (!word) return cuda_fail(cudaGetLastError(), "cudaGetSymbolAddress(g_device_error)");
    int host = 0;
    GLMVX_CUDA(cudaMemcpy(&host, word, sizeof host, cudaMemcpyDeviceToHost));
    if (host) {
        const int zero = 0;
        GLMVX_CUDA(cudaMemcpy(word, &zero, sizeof zero, cudaMemcpyHostToDevice));
    }
    *code = host;
    return kOk;
}
