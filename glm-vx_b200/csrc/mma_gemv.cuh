// Integer tensor-core path of the packed GEMV/GEMM (packed_mma.cu), shared
// with the MoE layer (moe.cu).
//
// The packed weights are multiplied in their integer form (Q8_0 bytes, Q4_K
// nibbles, IQ1_S codebook entries) by int8 `mma.sync` instructions.  The f32
// activations enter as exact integers: a "prepared row" holds, per 256-column
// chunk, a power-of-two exponent E and the rounded integer x*2^E (|x*2^E| <
// 2^30) split into four signed int8 limbs, so that
//     x*2^E = limb0*2^24 + limb1*2^16 + limb2*2^8 + limb3
// and every product sum inside the tensor core is exact int32 arithmetic.
// The block scales are applied in f32 afterwards.  Rounding x*2^E to an
// integer changes each activation by at most 2^-31 of the largest magnitude
// in its chunk; everything else is ordinary f32 accumulation.
#pragma once

#include "common.cuh"

namespace glmvx {

// Prepared activation row of K columns (K % 256 == 0):
//   [0, 4K)                 int8 limbs [4][K], limb 0 most significant
//   [4K, +4*K/256)          int32 E per 256-column chunk, in [-98, 156], or
//                           kPrepNonFinite when the chunk holds a non-finite value
//   [align16(..), +4*K/32)  f32 sum of each 32-column sub-block of the activations
// Rows are 256-byte aligned.
constexpr int32_t kPrepNonFinite = 0x7fffffff;
__host__ __device__ inline size_t prep_scale_offset(int K) { return 4ull * K; }
__host__ __device__ inline size_t prep_sums_offset(int K) {
    return (4ull * K + 4ull * (K / 256) + 15) & ~static_cast<size_t>(15);
}
__host__ __device__ inline size_t prep_stride(int K) {
    return (prep_sums_offset(K) + 4ull * (K / 32) + 255) & ~static_cast<size_t>(255);
}

// One weight matrix applied to up to four prepared activation rows (two
// with pairs = 1, the slots 0 and 1).
constexpr int kMmaSlots = 4;
struct MmaJob {
    const uint8_t *w;              // packed rows [rows_per_job][row_bytes], 16-byte aligned
    const uint8_t *xp[kMmaSlots];  // prepared rows; nullptr marks an unused slot
    float *out[kMmaSlots];         // out[s][r] for r < rows_per_job
};

// A column segment of a longer matrix (rows too long for one tensor-core
// plan run as equal column segments): the weights' global row pitch in
// bytes (0: the segment's own row length), the f32 activation row stride in
// floats (0: cols), and whether results add onto `out` (later segments, in
// segment order) instead of replacing it.
struct ColSegment {
    int64_t pitch = 0;
    int xstride = 0;
    bool accumulate = false;
};

// True when `kind` and the column count take the tensor-core path.
bool mma_supported(int kind, int cols);
// True when job lists of four tokens per job (pairs = 2) are built for it.
bool mma_quad_supported(int kind, int cols);

// Prepare `rows` activation rows x[r][0..cols) (x2 set: SwiGLU(x, x2) =
// x*sigmoid(x)*x2 per element) into prep + r*prep_stride(cols).  With
// rows_dev set, only the first min(*rows_dev, rows) rows (a count written on
// the device by an earlier kernel; `rows` is then the capacity).
int32_t prep_rows_device(uint8_t *prep, const float *x, const float *x2, int rows, int cols, cudaStream_t stream,
                         const int *rows_dev = nullptr, int xstride = 0);

// Tensor-core packed GEMV over a job list.
//  * jobs != nullptr: device-resident descriptors; the job count is
//    *njobs_dev when njobs_dev is set (read on the device after the previous
//    kernel completes, clamped to max_jobs), else max_jobs.
//  * pairs = 2 (job lists only, mma_quad_supported): each decoded weight
//    fragment is multiplied into two token pairs, the job's slots 0-1 and 2-3.
//  * jobs == nullptr: `batch` tokens against one matrix: job j applies job0.w
//    to prepared rows 2j and 2j+1 of job0.xp[0] (stride prep_stride(cols))
//    and writes rows of job0.out[0] (stride rows_per_job floats).  With
//    x_raw set instead (f32 rows [batch][cols], 16-byte aligned), each CTA
//    prepares the rows of the jobs it reaches in shared memory, so no
//    separate preparation or scratch is needed; returns kUnsupported when the
//    shape leaves no room for that (use the prepared-row form then).
//  * seg: single-matrix calls only (jobs == nullptr).
int32_t mma_gemv_device(int32_t kind, const MmaJob &job0, const MmaJob *jobs, const int *njobs_dev, int max_jobs,
                        int batch, int rows_per_job, int cols, cudaStream_t stream, const float *x_raw = nullptr,
                        int pairs = 1, const ColSegment &seg = {});

// f16 tensor-core GEMM for token batches (packed_gemm.cu): the weights are
// decoded once per fragment for every token.  Q4_K, and IQ1_S with cols %
// 2048 == 0; cols % 256 == 0; kGemmMinTokens..kGemmMaxTokens tokens; 16-byte
// aligned w, x and scratch (gemm_f16_scratch_bytes).  kUnsupported when no
// launch plan fits the shape.
constexpr int kGemmMinTokens = 8, kGemmMaxTokens = 64;
bool gemm_f16_supported(int kind, int cols, int batch);
size_t gemm_f16_scratch_bytes(int cols, int batch);
int32_t gemm_f16_device(int32_t kind, float *out, const uint8_t *w, const float *x, int rows, int cols, int batch,
                        uint8_t *scratch, cudaStream_t stream, const ColSegment &seg = {});

// tcgen05 packed GEMM for token batches (packed_gemm_tc.cu): weights decoded
// to f32 and split into two TF32 limbs in shared memory, activations split
// likewise by a preparation kernel into `scratch` (gemm_tc_scratch_bytes:
// the prepared limbs, plus the partial sums when a tile's columns are split),
// three kind::tf32 MMAs per K step accumulating each row in tensor memory.
// Any format, 1..64 tokens, cols a multiple of the format's raw chunk (256
// columns for Q8_0 / Q4_K, 2048 for IQ1_S); 16-byte aligned w, x, scratch.
bool gemm_tc_supported(int kind, int cols, int batch);
size_t gemm_tc_scratch_bytes(int32_t kind, int rows, int cols, int batch);
int32_t gemm_tc_device(int32_t kind, float *out, const uint8_t *w, const float *x, int rows, int cols, int batch,
                       uint8_t *scratch, cudaStream_t stream, const ColSegment &seg = {});

// The same kernel for FP8 E4M3FN weights with f32 scales per 128 x 128 tile
// (the gpu/fp8.vx contract): out[t][r] = sum_c (decode(w[r][c]) *
// s[r/128][c/128]) * x[t][c]; cols a multiple of 256, 1..64 tokens.
// Keep freed blocks of the device's default stream-ordered pool (the
// tensor-core paths' scratch) instead of releasing them at every
// synchronisation; once per device, safe inside a graph capture.
void keep_pool_memory();

bool fp8_gemm_tc_supported(int cols, int batch);
size_t fp8_gemm_tc_scratch_bytes(int rows, int cols, int batch);
int32_t fp8_gemm_tc_device(float *out, const uint8_t *w, const float *scales, const float *x, int rows, int cols,
                           int batch, uint8_t *scratch, cudaStream_t stream);

}  // namespace glmvx
