// Batched DSA indexer launches (ops.cu) used by the fused decode in mla.cu.
#pragma once
#include <cstdint>

#include <cuda_runtime.h>

namespace glmvx {

// scores[b][t] = sum_h w[b][h] relu(qk_scale q[b][h] . keys[b][t]) for t < lens[b]
// (lens nullptr: `tokens` for every query); keys of query b at keys + b * key_stride.
int32_t launch_index_scores_batch(float *out, const float *q, const float *keys, const float *w, int tokens,
                                  int heads, int dim, float qk_scale, const int32_t *lens, int64_t key_stride,
                                  int64_t out_stride, int batch, cudaStream_t stream);

// The same scores on the tensor cores (dsa_index.cu); kUnsupported when the
// shape has no tensor-core kernel (more than 256 heads, or heads x columns
// beyond its shared-memory budget).
int32_t launch_index_scores_tc(float *out, const float *q, const float *keys, const float *w, int tokens, int heads,
                               int dim, float qk_scale, const int32_t *lens, int64_t key_stride, int64_t out_stride,
                               int batch, cudaStream_t stream);

// indices[b][0:min(k, lens[b])] = stable descending top-k of scores[b][0:lens[b]],
// the rest of indices[b][0:k] -1.  1 <= k <= 4096.
int32_t launch_topk_batch(int32_t *indices, const float *scores, int n, int k, const int32_t *lens,
                          int64_t score_stride, int out_stride, int batch, cudaStream_t stream);

// Absorbed-MLA split partials on the tensor cores (mla_tc.cu) for a selection
// shared by all heads: heads <= 64, rank <= 512, rope_dim <= 64, at most
// 64 x 128 selected rows.  Splits of at most 128 rows, at most 64 of them
// (mla_tc_splits); partial numerators
// [batch][splits][heads][rank] and (max, mass) [batch][splits][heads][2] for
// mla_merge_kernel.  kUnsupported for other shapes.
bool mla_tc_supported(int heads, int rank, int rope_dim, int count);
int mla_tc_splits(int count, int batch);
int32_t launch_mla_tc(float *numerator, float *stats, const float *q_latent, const float *q_rope, const float *latent,
                      const float *rope, const int32_t *selected, const int32_t *lens, int heads, int rank,
                      int rope_dim, int tokens, int count, int splits, float scale, int64_t latent_stride,
                      int64_t rope_stride, int64_t sel_stride, int batch, cudaStream_t stream);

}  // namespace glmvx
