// Shared definitions for libglmvx_cuda.so: status codes, the thread-local
// error message, and the sm_100a PTX helpers (mbarrier + 1-D bulk copy) the
// streaming kernels use.  Every exported entry point returns an int32 status
// and never throws across the C boundary.
#pragma once

#include <cuda_runtime.h>
#include <cuda_fp16.h>
#include <stdint.h>
#include <stddef.h>

#include "glmvx.h"

#define GLMVX_EXPORT extern "C" __attribute__((visibility("default")))

namespace glmvx {

// Status values returned by every exported function.  -1 matches the
// reference C ABI's "invalid dimensions" (kernels/kernels.h:13).
enum Status : int32_t {
    kOk = 0,
    kInvalid = -1,     // rejected arguments (shape, pointer alignment, size)
    kCudaError = -2,   // a CUDA runtime call failed; see glmvx_last_error()
    kDeviceError = -3, // a kernel reported a bounded-wait timeout
    kUnsupported = -4, // format or shape has no kernel
};

// Thread-local message for the last failure on the calling thread.
void set_error(const char *fmt, ...) __attribute__((format(printf, 1, 2)));

// Convert a CUDA error into kCudaError with a message naming `what`.
int32_t cuda_fail(cudaError_t e, const char *what);

#define GLMVX_CUDA(call)                                  \
    do {                                                  \
        cudaError_t glmvx_e_ = (call);                    \
        if (glmvx_e_ != cudaSuccess) return ::glmvx::cuda_fail(glmvx_e_, #call); \
    } while (0)

// Checks the launch status of the most recent kernel.
int32_t launch_status(const char *kernel);

// Device word the kernels set (atomically, first error wins) when a bounded
// wait gives up.  Read and cleared by glmvx_check_device_error().
int *device_error_word();

// SM count of the current device (cached per device).
int sm_count();

// Allows `kernel` (a __global__ function) `bytes` of dynamic shared memory on
// the CURRENT device.  The attribute belongs to the function in one device's
// context, so it is raised once per (device, kernel) and size, under a lock
// (several host threads and several devices may launch the same kernel).
int32_t allow_dynamic_smem(const void *kernel, size_t bytes, const char *name);
template <class K>
inline int32_t allow_dynamic_smem(K *kernel, size_t bytes, const char *name) {
    return allow_dynamic_smem(reinterpret_cast<const void *>(kernel), bytes, name);
}

// ---------------------------------------------------------------- device ---

// Error codes written into the device error word.
enum DeviceError : int { kDevErrNone = 0, kDevErrFullWait = 1, kDevErrEmptyWait = 2, kDevErrBadIndex = 3 };

__device__ __forceinline__ uint64_t globaltimer_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}

__device__ __forceinline__ uint32_t smem_addr(const void *p) {
    return static_cast<uint32_t>(__cvta_generic_to_shared(p));
}

__device__ __forceinline__ void mbar_init(uint64_t *bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_addr(bar)), "r"(count));
}

__device__ __forceinline__ void fence_mbar_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
}

__device__ __forceinline__ void mbar_arrive(uint64_t *bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_addr(bar)) : "memory");
}

__device__ __forceinline__ void mbar_arrive_expect_tx(uint64_t *bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_addr(bar)), "r"(bytes)
                 : "memory");
}

__device__ __forceinline__ bool mbar_try_wait(uint64_t *bar, uint32_t parity) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity)
        : "memory");
    return done != 0;
}

// try_wait with a suspend-time hint: the thread sleeps in the barrier until
// the phase completes or about `hint_ns` pass, instead of re-issuing the test
// (a spinning warp takes issue slots from the warps doing the work).
__device__ __forceinline__ bool mbar_try_wait_suspend(uint64_t *bar, uint32_t parity, uint32_t hint_ns) {
    uint32_t done;
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2, %3;\n\t"
        "selp.u32 %0, 1, 0, p;\n\t}"
        : "=r"(done)
        : "r"(smem_addr(bar)), "r"(parity), "r"(hint_ns)
        : "memory");
    return done != 0;
}

// Wait for the phase with the given parity to complete, giving up after
// `limit_ns` of wall time.  Returns false on timeout (the caller records the
// error and returns; it never traps).
__device__ __forceinline__ bool mbar_wait_bounded(uint64_t *bar, uint32_t parity,
                                                  uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer_ns();
    for (;;) {
        if (mbar_try_wait_suspend(bar, parity, 100000u)) return true;
        if (globaltimer_ns() - start > limit_ns) return false;
    }
}

// As mbar_wait_bounded, polling without the suspend hint: for hand-offs on
// the critical path of a pipeline whose every stage waits on the previous
// one (a suspended thread resumes later than a polling one notices).
__device__ __forceinline__ bool mbar_wait_spin_bounded(uint64_t *bar, uint32_t parity,
                                                       uint64_t limit_ns = 2000000000ull) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t start = globaltimer_ns();
    for (uint32_t i = 1;; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 63u) == 0 && globaltimer_ns() - start > limit_ns) return false;
    }
}

// 1-D bulk copy global -> shared (TMA engine), completing `bytes` of
// transaction count on `bar`.  dst/src 16-byte aligned, bytes % 16 == 0.
// No cluster multicast: this is a plain per-CTA load.
__device__ __forceinline__ void bulk_g2s(void *dst, const void *src, uint32_t bytes, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes [%0], [%1], %2, [%3];" ::"r"(
            smem_addr(dst)),
        "l"(src), "r"(bytes), "r"(smem_addr(bar))
        : "memory");
}

__device__ __forceinline__ void named_barrier_sync(int id, int threads) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(threads) : "memory");
}

__device__ __forceinline__ void report_device_error(int *err, int code) {
    if (err) atomicCAS(err, 0, code);
}

// Programmatic dependent launch: let the next kernel on the stream start its
// prologue / wait until the previous kernel's writes are visible.
__device__ __forceinline__ void grid_dependency_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
__device__ __forceinline__ void allow_dependent_launch() { asm volatile("griddepcontrol.launch_dependents;"); }

// The reference's branch-stable logistic (kernels/kernels.vx:8-15).
__device__ __forceinline__ float sigmoid_ref(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(0.0f - x));
    const float z = expf(x);
    return z / (1.0f + z);
}

// SwiGLU element x*sigmoid(x)*u with the reference's branch-stable sigmoid
// and rounding order (kernels/kernels.vx:8-15,56-60).
__device__ __forceinline__ float silu_mul(float g, float u) {
    const float sg = g >= 0.0f ? 1.0f / (1.0f + expf(0.0f - g)) : expf(g) / (1.0f + expf(g));
    return __fmul_rn(__fmul_rn(g, sg), u);
}

__device__ __forceinline__ float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}

}  // namespace glmvx
