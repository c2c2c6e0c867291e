/*
 * TEST INFRASTRUCTURE ONLY -- CPU oracle for the f32 model primitives.
 *
 * A plain-C restatement of the reference's Vx CPU kernels in
 * kernels/kernels.vx:1-441, exporting the same C ABI (kernels/kernels.h:12-28).
 * Arithmetic is scalar f32 in the reference's operation order; libm expf and
 * sqrtf are used exactly where the Vx source calls them (kernels/kernels.vx:3-6).
 * Build with -ffp-contract=off.  Only tests/, smoke() and bench.py's
 * CPU-baseline leg may load this library.
 */
#include <math.h>
#include <stdint.h>
#include <stdlib.h>

#if defined(_OPENMP)
#define ROWS_PARALLEL _Pragma("omp parallel for schedule(static)")
#else
#define ROWS_PARALLEL
#endif
#define EXPORT __attribute__((visibility("default")))

#if defined(_OPENMP)
#include <omp.h>
#endif

/* Thread control of the OpenMP build (no reference counterpart): the timed
 * CPU legs set the thread count through the library itself, so an OpenMP
 * runtime that another module initialised earlier (with OMP_NUM_THREADS=1,
 * as torchrun exports) cannot pin it to one thread.  The serial build reports
 * one thread and ignores the request. */
EXPORT int32_t glm_vx_ref_set_threads(int32_t n) {
#if defined(_OPENMP)
    if (n > 0) omp_set_num_threads(n);
    return omp_get_max_threads();
#else
    (void)n;
    return 1;
#endif
}

/* Sign-split logistic (kernels/kernels.vx:8-15). */
static float sigmoid_f32(float x) {
    if (x >= 0.0f) return 1.0f / (1.0f + expf(0.0f - x));
    float z = expf(x);
    return z / (1.0f + z);
}

/* kernels/kernels.vx:17-27 */
EXPORT int32_t glm_vx_rmsnorm(float *out, const float *x, const float *weight, int32_t n, float eps) {
    if (n <= 0 || eps <= 0.0f) return -1;
    float ss = 0.0f;
    for (int32_t i = 0; i < n; ++i) ss = ss + x[i] * x[i];
    float inv = 1.0f / sqrtf(ss / (float)n + eps);
    for (int32_t i = 0; i < n; ++i) out[i] = x[i] * inv * weight[i];
    return 0;
}

/* kernels/kernels.vx:29-42 */
EXPORT int32_t glm_vx_layernorm(float *out, const float *x, const float *weight, const float *bias,
                                int32_t n, float eps) {
    if (n <= 0 || eps <= 0.0f) return -1;
    float mean = 0.0f;
    for (int32_t i = 0; i < n; ++i) mean = mean + x[i];
    mean = mean / (float)n;
    float variance = 0.0f;
    for (int32_t i = 0; i < n; ++i) {
        float d = x[i] - mean;
        variance = variance + d * d;
    }
    float inv = 1.0f / sqrtf(variance / (float)n + eps);
    for (int32_t i = 0; i < n; ++i) out[i] = (x[i] - mean) * inv * weight[i] + bias[i];
    return 0;
}

/* kernels/kernels.vx:44-54 */
EXPORT int32_t glm_vx_softmax(float *out, const float *x, int32_t n) {
    if (n <= 0) return -1;
    float maximum = x[0];
    for (int32_t i = 1; i < n; ++i)
        if (x[i] > maximum) maximum = x[i];
    float sum = 0.0f;
    for (int32_t i = 0; i < n; ++i) {
        float v = expf(x[i] - maximum);
        out[i] = v;
        sum = sum + v;
    }
    for (int32_t i = 0; i < n; ++i) out[i] = out[i] / sum;
    return 0;
}

/* kernels/kernels.vx:56-60: gate*sigmoid(gate)*up */
EXPORT int32_t glm_vx_swiglu(float *out, const float *gate, const float *up, int32_t n) {
    if (n < 0) return -1;
    for (int32_t i = 0; i < n; ++i) out[i] = gate[i] * sigmoid_f32(gate[i]) * up[i];
    return 0;
}

/* kernels/kernels.vx:62-72 */
EXPORT int32_t glm_vx_add(float *out, const float *a, const float *b, int32_t n) {
    if (n < 0) return -1;
    for (int32_t i = 0; i < n; ++i) out[i] = a[i] + b[i];
    return 0;
}
EXPORT int32_t glm_vx_axpy(float *out, const float *x, float alpha, int32_t n) {
    if (n < 0) return -1;
    for (int32_t i = 0; i < n; ++i) out[i] = out[i] + alpha * x[i];
    return 0;
}

/* kernels/kernels.vx:76-131.  The reference tiles 8 rows for SIMD but every
 * row keeps one ordered accumulation, which is what this loop computes. */
EXPORT int32_t glm_vx_matvec(float *out, const float *weight, const float *x, int32_t rows, int32_t cols) {
    if (rows < 0 || cols < 0) return -1;
    ROWS_PARALLEL
    for (int32_t r = 0; r < rows; ++r) {
        float sum = 0.0f;
        const float *wr = weight + (size_t)r * cols;
        for (int32_t c = 0; c < cols; ++c) sum = sum + wr[c] * x[c];
        out[r] = sum;
    }
    return 0;
}

/* kernels/kernels.vx:135-218: out[m,n] = A[m,k] . B[n,k]^T, ordered per element. */
EXPORT int32_t glm_vx_matmul_nt(float *out, const float *a, const float *b, int32_t m, int32_t n, int32_t k) {
    if (m < 0 || n < 0 || k < 0) return -1;
    ROWS_PARALLEL
    for (int32_t r = 0; r < m; ++r)
        for (int32_t c = 0; c < n; ++c) {
            float sum = 0.0f;
            for (int32_t j = 0; j < k; ++j) sum = sum + a[(size_t)r * k + j] * b[(size_t)c * k + j];
            out[(size_t)r * n + c] = sum;
        }
    return 0;
}

/* kernels/kernels.vx:226-248 */
EXPORT int32_t glm_vx_rope_offset(float *out, const float *x, const float *cosine, const float *sine,
                                  int32_t heads, int32_t head_dim, int32_t rope_dim, int32_t offset) {
    if (heads < 0 || rope_dim < 0 || offset < 0 || head_dim < rope_dim ||
        offset > head_dim - rope_dim || rope_dim % 2 != 0)
        return -1;
    for (int32_t h = 0; h < heads; ++h) {
        int32_t base = h * head_dim;
        for (int32_t d = 0; d < offset; ++d) out[base + d] = x[base + d];
        for (int32_t d = offset + rope_dim; d < head_dim; ++d) out[base + d] = x[base + d];
        for (int32_t p = 0; p < rope_dim / 2; ++p) {
            int32_t i = base + offset + p * 2;
            float a = x[i], b = x[i + 1];
            out[i] = a * cosine[p] - b * sine[p];
            out[i + 1] = a * sine[p] + b * cosine[p];
        }
    }
    return 0;
}

/* kernels/kernels.vx:222-224 */
EXPORT int32_t glm_vx_rope(float *out, const float *x, const float *cosine, const float *sine,
                           int32_t heads, int32_t head_dim, int32_t rope_dim) {
    return glm_vx_rope_offset(out, x, cosine, sine, heads, head_dim, rope_dim, head_dim - rope_dim);
}

/* Sigmoid + correction-bias top-k; bias chooses, never weighs; ties keep the
 * lower expert id; weights = sigmoid/(sum+1e-20)*scale (kernels/kernels.vx:252-279). */
EXPORT int32_t glm_vx_router(int32_t *indices, float *weights, const float *logits, const float *bias,
                             int32_t experts, int32_t k, float scale) {
    if (k <= 0 || experts < k) return -1;
    float total = 0.0f;
    for (int32_t slot = 0; slot < k; ++slot) {
        int32_t best = -1;
        float best_score = 0.0f;
        for (int32_t e = 0; e < experts; ++e) {
            int used = 0;
            for (int32_t p = 0; p < slot; ++p)
                if (indices[p] == e) used = 1;
            if (used) continue;
            float score = sigmoid_f32(logits[e]) + bias[e];
            if (best < 0 || score > best_score) {
                best = e;
                best_score = score;
            }
        }
        indices[slot] = best;
        float prob = sigmoid_f32(logits[best]);
        weights[slot] = prob;
        total = total + prob;
    }
    total = total + 1e-20f;
    for (int32_t slot = 0; slot < k; ++slot) weights[slot] = weights[slot] / total * scale;
    return 0;
}

/* Exact stable top-k (kernels/kernels.vx:281-355): descending score, equal
 * scores ordered by smaller index, +0 == -0.  The order is a strict total
 * order, so any correct selection yields the reference's output; this one
 * sorts candidate indices with that comparator. */
static const float *topk_scores;
static int topk_cmp(const void *pa, const void *pb) {
    int32_t a = *(const int32_t *)pa, b = *(const int32_t *)pb;
    float sa = topk_scores[a], sb = topk_scores[b];
    if (sa > sb) return -1;
    if (sa < sb) return 1;
    return (a > b) - (a < b);
}
EXPORT int32_t glm_vx_topk(int32_t *indices, const float *scores, int32_t n, int32_t k) {
    if (n < 0 || k < 0 || n < k) return -1;
    if (k == 0) return 0;
    int32_t *all = (int32_t *)malloc(sizeof(int32_t) * (size_t)n);
    if (!all) return -1;
    for (int32_t i = 0; i < n; ++i) all[i] = i;
    topk_scores = scores;
    qsort(all, (size_t)n, sizeof(int32_t), topk_cmp);
    for (int32_t i = 0; i < k; ++i) indices[i] = all[i];
    free(all);
    return 0;
}

/* kernels/kernels.vx:358-376 */
EXPORT int32_t glm_vx_attention(float *out, float *scratch, const float *q, const float *keys,
                                const float *values, int32_t tokens, int32_t dim, int32_t value_dim,
                                float scale) {
    if (tokens <= 0 || dim <= 0 || value_dim <= 0) return -1;
    for (int32_t t = 0; t < tokens; ++t) {
        float score = 0.0f;
        for (int32_t d = 0; d < dim; ++d) score = score + q[d] * keys[(size_t)t * dim + d];
        scratch[t] = score * scale;
    }
    glm_vx_softmax(scratch, scratch, tokens);
    for (int32_t d = 0; d < value_dim; ++d) {
        float sum = 0.0f;
        for (int32_t t = 0; t < tokens; ++t) sum = sum + scratch[t] * values[(size_t)t * value_dim + d];
        out[d] = sum;
    }
    return 0;
}

/* kernels/kernels.vx:379-400 */
EXPORT int32_t glm_vx_sparse_attention(float *out, float *scratch, const float *q, const float *keys,
                                       const float *values, const int32_t *selected, int32_t count,
                                       int32_t tokens, int32_t dim, int32_t value_dim, float scale) {
    if (count <= 0 || tokens <= 0 || dim <= 0 || value_dim <= 0) return -1;
    for (int32_t j = 0; j < count; ++j)
        if (selected[j] < 0 || selected[j] >= tokens) return -1;
    for (int32_t j = 0; j < count; ++j) {
        int32_t t = selected[j];
        float score = 0.0f;
        for (int32_t d = 0; d < dim; ++d) score = score + q[d] * keys[(size_t)t * dim + d];
        scratch[j] = score * scale;
    }
    glm_vx_softmax(scratch, scratch, count);
    for (int32_t d = 0; d < value_dim; ++d) {
        float sum = 0.0f;
        for (int32_t j = 0; j < count; ++j)
            sum = sum + scratch[j] * values[(size_t)selected[j] * value_dim + d];
        out[d] = sum;
    }
    return 0;
}

/* DSA score per token: sum_h w_h * relu(q_h.k_t * s) (kernels/kernels.vx:404-421). */
EXPORT int32_t glm_vx_index_scores(float *out, const float *q, const float *keys, const float *weights,
                                   int32_t tokens, int32_t heads, int32_t dim, float qk_scale) {
    if (tokens < 0 || heads <= 0 || dim <= 0) return -1;
    ROWS_PARALLEL
    for (int32_t t = 0; t < tokens; ++t) {
        float total = 0.0f;
        for (int32_t h = 0; h < heads; ++h) {
            float dot = 0.0f;
            for (int32_t d = 0; d < dim; ++d) dot = dot + q[(size_t)h * dim + d] * keys[(size_t)t * dim + d];
            float score = dot * qk_scale;
            if (score > 0.0f) total = total + weights[h] * score;
        }
        out[t] = total;
    }
    return 0;
}

/* Interleaved input pairs -> [rotated even half | rotated odd half]
 * (kernels/kernels.vx:425-441). */
EXPORT int32_t glm_vx_rope_glm(float *out, const float *x, const float *cosine, const float *sine,
                               int32_t heads, int32_t dim) {
    if (heads < 0 || dim <= 0 || dim % 2 != 0) return -1;
    for (int32_t h = 0; h < heads; ++h) {
        int32_t base = h * dim;
        for (int32_t p = 0; p < dim / 2; ++p) {
            float a = x[base + 2 * p], b = x[base + 2 * p + 1];
            out[base + p] = a * cosine[p] - b * sine[p];
            out[base + dim / 2 + p] = b * cosine[p] + a * sine[p];
        }
    }
    return 0;
}
