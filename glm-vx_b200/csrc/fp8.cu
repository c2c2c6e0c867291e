// FP8 (E4M3FN) block-scaled projection on sm_100a.
//
// Replaces the reference's GPU entry glm_vx_gpu_fp8_matvec (gpu/fp8.vx:50-89,
// launched by GLMKernels.fp8_matvec, gpu/runtime.py:1031-1053) with the same
// contract: weight u8 [rows, cols] E4M3FN (bias 7, no infinity, exponent 15
// with mantissa 7 is NaN), scales f32 [ceil(rows/128), ceil(cols/128)], x f32
// [cols] -> out f32 [rows], out[r] = sum_c (decode(w[r,c]) * s[r/128, c/128])
// * x[c] (gpu/fp8.vx:20-38).
//
// A CTA of 8 warps owns 8 rows (one per warp; below 4096 rows, 2 rows of 4
// warps each); the activations are read through L1.  A warp walks its row in
// 512-column steps.  Widths that are a multiple of 512: lane l takes the
// 4-byte words at columns 4l + 128k (k = 0..3) of a step, one coalesced
// 128-byte load per k and warp, with B steps of loads issued before any is
// used (row_steps512).  Other widths: 16 consecutive bytes per lane and step.
// Pairs convert with the hardware E4M3x2 -> f16x2 conversion (exact: every
// E4M3 value, subnormals included, is an f16 value; NaN encodings become
// NaN), widen to f32 and multiply the activations; a lane's columns of one
// load lie in one 128-column scale tile, whose scale multiplies the partial
// sum.  The row sum is a fixed shuffle tree (deterministic).
// HBM-bound: 1 byte per weight.
#include <cuda_fp8.h>

#include <algorithm>
#include <mutex>

#include "common.cuh"
#include "mma_gemv.cuh"

namespace glmvx {

// One row per warp (measured against two rows per warp: 6144 x 6144 in 17
// vs 27 us with the 16-byte mapping).
constexpr int kFp8Threads = 256, kFp8RowsPerWarp = 1, kFp8Unroll = 8, kFp8SplitRows = 4096;
constexpr int kFp8RowsPerCta = kFp8Threads / 32 * kFp8RowsPerWarp;

__device__ __forceinline__ float2 e4m3x2_to_float2(uint32_t two) {
    const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(static_cast<__nv_fp8x2_storage_t>(two & 0xffffu), __NV_E4M3);
    return __half22float2(*reinterpret_cast<const __half2 *>(&h));
}

// 16 weights (one 16-byte word) against 16 activations of the same columns;
// the four float4 activation reads go in a lane-rotated order.
__device__ __forceinline__ float dot16(const uint4 q, const float *x16, int rot) {
    const uint32_t words[4] = {q.x, q.y, q.z, q.w};
    float part = 0.0f;
#pragma unroll
    for (int jj = 0; jj < 4; ++jj) {
        const int j = (jj + rot) & 3;
        const uint32_t wj = j == 0 ? words[0] : (j == 1 ? words[1] : (j == 2 ? words[2] : words[3]));
        const float4 xq = __ldg(reinterpret_cast<const float4 *>(x16 + 4 * j));
        const float2 a = e4m3x2_to_float2(wj), b = e4m3x2_to_float2(wj >> 16);
        part = fmaf(a.x, xq.x, part);
        part = fmaf(a.y, xq.y, part);
        part = fmaf(b.x, xq.z, part);
        part = fmaf(b.y, xq.w, part);
    }
    return part;
}

// Rows whose width is a multiple of 512: lane l takes columns 4l + 128k
// (k = 0..3) of each 512-column step, so a weight load is one coalesced
// 128-byte word per warp, an activation load one contiguous 512-byte float4
// row, and the four words of a step fall in the scale tiles 4 step + k
// (uniform across the warp: no per-lane selection, no divergence).  Loads
// go out B steps at a time without a bounds test between them (a guarded
// loop keeps one load per lane in flight).  Measured on 6144 x 6144: 16.9 ->
// 13.3 us; 16384 x 6144 with B = 4: 42.5 -> 26.9 us.

__device__ __forceinline__ float dot4(uint32_t word, float4 xq) {
    const float2 a = e4m3x2_to_float2(word), b = e4m3x2_to_float2(word >> 16);
    float part = a.x * xq.x;
    part = fmaf(a.y, xq.y, part);
    part = fmaf(b.x, xq.z, part);
    return fmaf(b.y, xq.w, part);
}

// sum over steps step0, step0 + stride, ... (n of them) of one row.
template <int B>
__device__ __forceinline__ float row_steps512(const uint8_t *__restrict__ wr, const float *__restrict__ sr,
                                              const float *__restrict__ x, int step0, int stride, int n, int lane,
                                              float sum) {
    int i = 0;
    for (; i + B <= n; i += B) {
        uint32_t q[B][4];
#pragma unroll
        for (int j = 0; j < B; ++j)
#pragma unroll
            for (int k = 0; k < 4; ++k)
                q[j][k] = __ldg(reinterpret_cast<const uint32_t *>(wr + 512 * (step0 + (i + j) * stride) + 128 * k + 4 * lane));
#pragma unroll
        for (int j = 0; j < B; ++j) {
            const int st = step0 + (i + j) * stride;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                const float4 xq = __ldg(reinterpret_cast<const float4 *>(x + 512 * st + 128 * k + 4 * lane));
                sum = fmaf(__ldg(sr + 4 * st + k), dot4(q[j][k], xq), sum);
            }
        }
    }
    for (; i < n; ++i) {
        const int st = step0 + i * stride;
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const uint32_t q = __ldg(reinterpret_cast<const uint32_t *>(wr + 512 * st + 128 * k + 4 * lane));
            const float4 xq = __ldg(reinterpret_cast<const float4 *>(x + 512 * st + 128 * k + 4 * lane));
            sum = fmaf(__ldg(sr + 4 * st + k), dot4(q, xq), sum);
        }
    }
    return sum;
}

template <int B>
__global__ void __launch_bounds__(kFp8Threads)
    fp8_matvec_kernel(float *__restrict__ out, const uint8_t *__restrict__ w, const float *__restrict__ scales,
                      const float *__restrict__ x, int rows, int cols) {
    const float *xv = x;
    const int lane = threadIdx.x & 31;
    const int64_t row0 = static_cast<int64_t>(blockIdx.x) * kFp8RowsPerCta + (threadIdx.x >> 5) * kFp8RowsPerWarp;
    if (row0 >= rows) return;
    const int64_t scale_cols = (static_cast<int64_t>(cols) + 127) / 128;
    const bool vec = (cols & 15) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    float sum[kFp8RowsPerWarp] = {};
    if (vec && cols % 512 == 0) {
        static_assert(kFp8RowsPerWarp == 1, "one row per warp");
        sum[0] = row_steps512<B>(w + row0 * cols, scales + (row0 / 128) * scale_cols, xv, 0, 1, cols / 512, lane, 0.0f);
    } else if (vec) {
        // A step covers 512 columns: lane l owns columns 16l..16l+15, inside
        // the 128-column scale tile l/8.
#pragma unroll kFp8Unroll
        for (int c = 16 * lane; c < cols; c += 512) {
#pragma unroll
            for (int r = 0; r < kFp8RowsPerWarp; ++r) {
                const int64_t row = row0 + r;
                if (row < rows) {
                    const uint4 q = __ldg(reinterpret_cast<const uint4 *>(w + row * cols + c));
                    const float s = __ldg(scales + (row / 128) * scale_cols + c / 128);
                    sum[r] = fmaf(s, dot16(q, xv + c, lane >> 1), sum[r]);
                }
            }
        }
    } else {  // any width / alignment: one byte per lane per step
        for (int r = 0; r < kFp8RowsPerWarp; ++r) {
            const int64_t row = row0 + r;
            if (row >= rows) break;
            for (int c = lane; c < cols; c += 32) {
                const float v = e4m3x2_to_float2(w[row * cols + c]).x;
                sum[r] = fmaf(v * __ldg(scales + (row / 128) * scale_cols + c / 128), xv[c], sum[r]);
            }
        }
    }
#pragma unroll
    for (int r = 0; r < kFp8RowsPerWarp; ++r) {
        const float v = warp_sum(sum[r]);
        if (lane == 0 && row0 + r < rows) out[row0 + r] = v;
    }
}

// Below 4096 rows: `split` warps share a row, warp part p taking the
// 512-column steps p, p + split, ...; their sums meet in shared memory and
// are added in part order (deterministic).  More warps per row put more
// loads in flight when there are few rows.
template <int split, int B>
__global__ void __launch_bounds__(kFp8Threads)
    fp8_matvec_split_kernel(float *__restrict__ out, const uint8_t *__restrict__ w, const float *__restrict__ scales,
                      const float *__restrict__ x, int rows, int cols) {
    __shared__ float part_sum[kFp8Threads / 32][kFp8RowsPerWarp];
    const float *xv = x;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, part = warp % split;
    const int64_t row0 = (static_cast<int64_t>(blockIdx.x) * (kFp8Threads / 32 / split) + warp / split) * kFp8RowsPerWarp;
    const int64_t scale_cols = (static_cast<int64_t>(cols) + 127) / 128;
    const bool vec = (cols & 15) == 0 && (reinterpret_cast<uintptr_t>(w) & 15) == 0 &&
                     (reinterpret_cast<uintptr_t>(x) & 15) == 0;
    float sum[kFp8RowsPerWarp] = {};
    if (row0 < rows) {
        if (vec && cols % 512 == 0) {  // part p takes steps p, p + split, ...
            const int steps = cols / 512, n = part < steps ? (steps - part + split - 1) / split : 0;
            sum[0] = row_steps512<B>(w + row0 * cols, scales + (row0 / 128) * scale_cols, xv, part, split, n, lane, 0.0f);
        } else if (vec) {
            // A step covers 512 columns: lane l owns columns 16l..16l+15, inside
            // the 128-column scale tile l/8.
#pragma unroll kFp8Unroll
            for (int c = 16 * lane + 512 * part; c < cols; c += 512 * split) {
#pragma unroll
                for (int r = 0; r < kFp8RowsPerWarp; ++r) {
                    const int64_t row = row0 + r;
                    if (row < rows) {
                        const uint4 q = __ldg(reinterpret_cast<const uint4 *>(w + row * cols + c));
                        const float s = __ldg(scales + (row / 128) * scale_cols + c / 128);
                        sum[r] = fmaf(s, dot16(q, xv + c, lane >> 1), sum[r]);
                    }
                }
            }
        } else {  // any width / alignment: one byte per lane per step
            for (int r = 0; r < kFp8RowsPerWarp; ++r) {
                const int64_t row = row0 + r;
                if (row >= rows) break;
                for (int c = lane + 32 * part; c < cols; c += 32 * split) {
                    const float v = e4m3x2_to_float2(w[row * cols + c]).x;
                    sum[r] = fmaf(v * __ldg(scales + (row / 128) * scale_cols + c / 128), xv[c], sum[r]);
                }
            }
        }
    }
#pragma unroll
    for (int r = 0; r < kFp8RowsPerWarp; ++r) {
        const float v = warp_sum(sum[r]);
        if (lane == 0) part_sum[warp][r] = v;
    }
    __syncthreads();
    if (part == 0 && lane < kFp8RowsPerWarp && row0 + lane < rows) {
        float total = 0.0f;
        for (int p = 0; p < split; ++p) total += part_sum[warp + p][lane];
        out[row0 + lane] = total;
    }
}


// Batched: out[t][r] for tokens t < batch, x[t][cols] row-major.  Columns a
// multiple of 256 and 2..64 tokens go to the tcgen05 GEMM (weights times
// their tile scale in f32, three bf16 limbs); otherwise one GEMV per token.
GLMVX_EXPORT int32_t glmvx_fp8_gemm(float *out, const uint8_t *weight, const float *scales, const float *x,
                                    int32_t rows, int32_t cols, int32_t batch, int32_t *path, void *stream) {
    if (rows < 1 || cols < 0 || batch < 0 || !out || !weight || !scales || (cols && batch && !x)) {
        set_error("fp8 gemm: rows must be >= 1, cols and batch >= 0 and pointers set");
        return kInvalid;
    }
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (batch >= 2 && fp8_gemm_tc_supported(cols, batch) &&
        ((reinterpret_cast<uintptr_t>(weight) | reinterpret_cast<uintptr_t>(x)) & 15) == 0) {
        if (path) *path = 9;
        keep_pool_memory();
        void *scratch = nullptr;
        GLMVX_CUDA(cudaMallocAsync(&scratch, fp8_gemm_tc_scratch_bytes(rows, cols, batch), st));
        const int32_t rc = fp8_gemm_tc_device(out, weight, scales, x, rows, cols, batch,
                                              static_cast<uint8_t *>(scratch), st);
        const cudaError_t fe = cudaFreeAsync(scratch, st);
        if (rc) return rc;
        return fe == cudaSuccess ? kOk : cuda_fail(fe, "cudaFreeAsync");
    }
    if (path) *path = 1;
    for (int t = 0; t < batch; ++t)
        if (const int32_t rc = glmvx_fp8_matvec(out + static_cast<int64_t>(t) * rows, weight, scales,
                                                x + static_cast<int64_t>(t) * cols, rows, cols, stream))
            return rc;
    return kOk;
}

}  // namespace glmvx

using namespace glmvx;

// CTAs of fp8_matvec_kernel<2> resident at once on the current device (one
// wave), cached per device.
static int fp8_resident_ctas() {
    static std::mutex mu;
    static int cached[64] = {0};
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= 64) return 0;
    std::lock_guard<std::mutex> lock(mu);
    if (!cached[dev]) {
        int per_sm = 0;
        if (cudaOccupancyMaxActiveBlocksPerMultiprocessor(&per_sm, fp8_matvec_kernel<2>, kFp8Threads, 0) != cudaSuccess)
            per_sm = 1;
        cached[dev] = std::max(1, per_sm) * sm_count();
    }
    return cached[dev];
}

// out[rows] = fp8 weight [rows, cols] (block scales) . x[cols]; device pointers,
// asynchronous on `stream`.  rows >= 1, cols >= 0 (gpu/runtime.py:1047-1050).
GLMVX_EXPORT int32_t glmvx_fp8_matvec(float *out, const uint8_t *weight, const float *scales, const float *x,
                                      int32_t rows, int32_t cols, void *stream) {
    if (rows < 1 || cols < 0 || !out || !weight || !scales || (cols && !x)) {
        set_error("fp8 matvec: rows must be >= 1, cols >= 0 and pointers set");
        return kInvalid;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (rows < kFp8SplitRows) {  // few rows: four warps per row put more loads in flight (2048 x 6144: 6.5 us)
        constexpr int kSplit = 4, kRowsPerCta = kFp8Threads / 32 / kSplit;
        fp8_matvec_split_kernel<kSplit, 1><<<(rows + kRowsPerCta - 1) / kRowsPerCta, kFp8Threads, 0, st>>>(
            out, weight, scales, x, rows, cols);
        return launch_status("fp8_matvec_split_kernel");
    }
    const int ctas = (rows + kFp8RowsPerCta - 1) / kFp8RowsPerCta;
    const dim3 grid(static_cast<unsigned>(ctas));
    // Activations are read through L1 (they fit, and every warp of an SM
    // reuses them); no shared-memory staging, so weight loads start at once.
    // Two steps of loads per lane while the grid fits one wave of resident
    // CTAs, four (more registers, fewer CTAs per SM) beyond.
    if (ctas > fp8_resident_ctas()) {
        fp8_matvec_kernel<4><<<grid, kFp8Threads, 0, st>>>(out, weight, scales, x, rows, cols);
    } else {
        fp8_matvec_kernel<2><<<grid, kFp8Threads, 0, st>>>(out, weight, scales, x, rows, cols);
    }
    return launch_status("fp8_matvec_kernel");
}
