// Job-list interface of the streaming GEMV (packed_gemv.cu), shared with the
// MoE layer (moe.cu), which writes job descriptors on the device.
#pragma once

#include "common.cuh"

namespace glmvx {

// out[r] = W[r,:] . act for r in [0, rows_per_job), act = x, or
// act = x*sigmoid(x)*x2 when x2 is set (fused SwiGLU input).
struct GemvJob {
    const uint8_t *w;
    const float *x;
    const float *x2;
    float *out;
};

// Launch one streaming GEMV over `njobs` device-resident job descriptors.
// `w_base`/`x_base` are representative pointers used for alignment checks;
// every job's weights must be 16-byte aligned with 16-byte multiple rows.
int32_t gemv_jobs_device(int32_t kind, const GemvJob *jobs, int32_t njobs, int32_t rows_per_job, int32_t cols,
                         const uint8_t *w_base, const float *x_base, cudaStream_t stream);

}  // namespace glmvx
