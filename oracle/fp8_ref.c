/*
 * TEST INFRASTRUCTURE ONLY -- CPU oracle for the FP8 E4M3FN block-scaled
 * projection.  Restates the CPU reference prefix of gpu/fp8.vx:3-38:
 * finite-only E4M3 (bias 7, exponent 15/mantissa 7 is NaN, no infinity) and a
 * sequential f32 row dot with 128x128 f32 block scales.  Only tests/, smoke()
 * and bench.py's CPU-baseline leg may load this library.
 */
#include <math.h>
#include <stdint.h>

#define EXPORT __attribute__((visibility("default")))

/* gpu/fp8.vx:3-17 */
EXPORT float glm_vx_fp8_decode(uint8_t byte) {
    int32_t bits = byte, exponent = (bits >> 3) & 15, mantissa = bits & 7;
    float magnitude = (float)mantissa / 512.0f;
    if (exponent > 0) magnitude = (float)(8 + mantissa) * (float)(1 << (exponent - 1)) / 512.0f;
    if (exponent == 15 && mantissa == 7) magnitude = NAN;
    return magnitude * ((bits & 128) ? -1.0f : 1.0f);
}

/* gpu/fp8.vx:20-38: out[r] = sum_c (decode(w[r,c]) * scale[r/128, c/128]) * x[c] */
EXPORT int32_t glm_vx_fp8_matvec_reference(float *out, const uint8_t *weight, const float *scales,
                                           const float *x, int32_t rows, int32_t cols) {
    if (rows < 0 || cols < 0) return -1;
    const int64_t scale_cols = ((int64_t)cols + 127) / 128;
    for (int32_t row = 0; row < rows; ++row) {
        const int64_t row_base = (int64_t)row * cols, scale_base = ((int64_t)row / 128) * scale_cols;
        float sum = 0.0f;
        for (int64_t c = 0; c < cols; ++c)
            sum = sum + (glm_vx_fp8_decode(weight[row_base + c]) * scales[scale_base + c / 128]) * x[c];
        out[row] = sum;
    }
    return 0;
}
