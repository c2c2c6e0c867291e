// FP8 (E4M3FN) block-scaled projection on sm_100a.
//
// Replaces the reference's GPU entry glm_vx_gpu_fp8_matvec (gpu/fp8.vx:50-89,
// launched by GLMKernels.fp8_matvec, gpu/runtime.py:1031-1053) with the same
// contract: weight u8 [rows, cols] E4M3FN (bias 7, no infinity, exponent 15
// with mantissa 7 is NaN), scales f32 [ceil(rows/128), ceil(cols/128)], x f32
// [cols] -> out f32 [rows], out[r] = sum_c (decode(w[r,c]) * s[r/128, c/128])
// * x[c] (gpu/fp8.vx:20-38).
//
// One warp per row; per step a lane takes four consecutive weights from each
// of four 128-column scale tiles (each load instruction of the warp reads 128
// contiguous bytes), converts pairs with the hardware E4M3x2 -> f16x2
// conversion (exact: every E4M3 value, subnormals included, is an f16 value;
// NaN encodings become NaN), widens to f32 and multiplies by the activations
// held in shared memory; the tile scale multiplies each 4-weight partial sum.
// The row sum is a fixed shuffle tree (deterministic).
// HBM-bound: 1 byte per weight.
#include <cuda_fp8.h>

#include "common.cuh"

namespace glmvx {

constexpr int kFp8Threads = 256, kFp8MaxSmemCols = 12288;

__device__ __forceinline__ float2 e4m3x2_to_float2(uint32_t two) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two & 0xffffu), __NV_E4M3);
    return __half22float2(*reinterpret_cast<const __half2 *>(&h));
}

template <bool SmemX>
__global__ void __launch_bounds__(kFp8Threads)
    fp8_matvec_kernel(float *__restrict__ out, const uint8_t *__restrict__ w, const float *__restrict__ scales,
                      const float *__restrict__ x, int rows, int cols) {
    extern __shared__ __align__(16) float xs[];
    const float *xv = x;
    if constexpr (SmemX) {
        for (int c = threadIdx.x; c < cols; c += kFp8Threads) xs[c] = x[c];
        __syncthreads();
        xv = xs;
    }
    const int lane = threadIdx.x & 31;
    const int64_t row = static_cast<int64_t>(blockIdx.x) * (kFp8Threads / 32) + (threadIdx.x >> 5);
    if (row >= rows) return;
    const int64_t scale_cols = (static_cast<int64_t>(cols) + 127) / 128;
    const float *srow = scales + (row / 128) * scale_cols;
    const uint8_t *wr = w + row * static_cast<int64_t>(cols);
    float sum = 0.0f;
    const bool vec = (cols & 3) == 0 && (reinterpret_cast<uintptr_t>(w) & 3) == 0 &&
                     (SmemX || (reinterpret_cast<uintptr_t>(x) & 15) == 0);
    if (vec) {
        // Step of 512 columns = four 128-column scale tiles; lane l takes
        // columns 4l..4l+3 of each tile (coalesced weight words, conflict-free
        // float4 activation reads).
        for (int c0 = 0; c0 < cols; c0 += 512) {
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                const int c = c0 + 128 * i + 4 * lane;
                if (c < cols) {
                    const uint32_t q = __ldg(reinterpret_cast<const uint32_t *>(wr + c));
                    const float4 xq = *reinterpret_cast<const float4 *>(xv + c);
                    const float2 a = e4m3x2_to_float2(q), b = e4m3x2_to_float2(q >> 16);
                    float part = a.x * xq.x;
                    part = fmaf(a.y, xq.y, part);
                    part = fmaf(b.x, xq.z, part);
                    part = fmaf(b.y, xq.w, part);
                    sum = fmaf(__ldg(srow + c / 128), part, sum);
                }
            }
        }
    } else {  // any width / alignment: one byte per lane per step
        for (int c = lane; c < cols; c += 32) {
            const float v = e4m3x2_to_float2(wr[c]).x;
            sum = fmaf(v * __ldg(srow + c / 128), xv[c], sum);
        }
    }
    sum = warp_sum(sum);
    if (lane == 0) out[row] = sum;
}

}  // namespace glmvx

using namespace glmvx;

// out[rows] = fp8 weight [rows, cols] (block scales) . x[cols]; device pointers,
// asynchronous on `stream`.  rows >= 1, cols >= 0 (gpu/runtime.py:1047-1050).
GLMVX_EXPORT int32_t glmvx_fp8_matvec(float *out, const uint8_t *weight, const float *scales, const float *x,
                                      int32_t rows, int32_t cols, void *stream) {
    if (rows < 1 || cols < 0 || !out || !weight || !scales || (cols && !x)) {
        set_error("fp8 matvec: rows must be >= 1, cols >= 0 and pointers set");
        return kInvalid;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const dim3 grid(static_cast<unsigned>((rows + 7) / 8));
    if (cols <= kFp8MaxSmemCols) {
        const size_t smem = sizeof(float) * static_cast<size_t>(cols);
        static bool configured = false;
        if (!configured) {
            GLMVX_CUDA(cudaFuncSetAttribute(fp8_matvec_kernel<true>, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            static_cast<int>(sizeof(float) * kFp8MaxSmemCols)));
            configured = true;
        }
        fp8_matvec_kernel<true><<<grid, kFp8Threads, smem, st>>>(out, weight, scales, x, rows, cols);
    } else {
        fp8_matvec_kernel<false><<<grid, kFp8Threads, 0, st>>>(out, weight, scales, x, rows, cols);
    }
    return launch_status("fp8_matvec_kernel");
}
