/*
 * libglmvx_cuda.so -- B200 (sm_100a) packed-GGUF dequant GEMV/GEMM library.
 *
 * Two C ABIs, no C++ types, no exceptions across the boundary:
 *
 *  1. The reference's CPU kernel ABI, unchanged (kernels/kernels.h:12-53 of
 *     gakonst/glm-vx).  HOST pointers; each call stages its inputs on the
 *     GPU, runs the kernel and copies the result back.  Loading this library
 *     with GLM_VX_LIBRARY=.../libglmvx_cuda.so makes the reference's own
 *     kernels/packed.py and kernels/backend.py run on the B200.
 *     Status: 0 ok, -1 rejected arguments (as the reference), -2 CUDA error,
 *     -3 a kernel's bounded wait expired.  Message: glmvx_last_error().
 *
 *  2. A resident DEVICE-pointer ABI (glmvx_*), the one the GPU backend and the
 *     benchmarks use: weights live in HBM, calls are asynchronous on the given
 *     stream (NULL = legacy default stream).  It replaces the reference's
 *     ctypes CUDA Driver API runtime and PTX entry points (gpu/runtime.py,
 *     gpu/kernels.h, gpu/gemm.vx, gpu/fp8.vx).
 *
 * GGML kinds: 1 F16, 8 Q8_0, 10 Q2_K, 11 Q3_K, 12 Q4_K, 13 Q5_K, 14 Q6_K,
 * 16 IQ2_XXS, 18 IQ3_XXS, 19 IQ1_S, 23 IQ4_XS (kernels/packed.py:14-19).
 */
#ifndef GLMVX_H
#define GLMVX_H
#include <stdint.h>
#ifdef __cplusplus
extern "C" {
#endif

/* ====================================================================== *
 * 1. Reference CPU ABI served by the GPU (host pointers)                  *
 * ====================================================================== */

/* Packed weights.  Replaces kernels/kernels.h:193-207 (GLM_VX_PACKED_DECL),
 * bodies kernels/packed.vx:154-470 and the generated batch_v2 exports
 * (kernels/packed.vx:473ff).  half/table must be the reference's exact
 * lookup tables (kernels/packed.py:27-37); they are verified, not used. */
#define GLMVX_REFERENCE_PACKED_DECL(kind)                                                          \
    int32_t glm_vx_packed_##kind(float *out, const uint8_t *w, const float *x, const float *half,   \
                                 const uint8_t *table, int32_t rows, int32_t cols);                \
    int32_t glm_vx_packed_batch_v2_##kind(float *out, const uint8_t *w, const float *x,            \
                                          const float *half, const uint8_t *table, int32_t rows,  \
                                          int32_t cols, int32_t batch);                            \
    int32_t glm_vx_unpack_##kind(float *out, const uint8_t *w, const float *half,                   \
                                 const uint8_t *table, int32_t blocks);
GLMVX_REFERENCE_PACKED_DECL(f16)
GLMVX_REFERENCE_PACKED_DECL(q8_0)
GLMVX_REFERENCE_PACKED_DECL(q2_k)
GLMVX_REFERENCE_PACKED_DECL(q3_k)
GLMVX_REFERENCE_PACKED_DECL(q4_k)
GLMVX_REFERENCE_PACKED_DECL(q5_k)
GLMVX_REFERENCE_PACKED_DECL(q6_k)
GLMVX_REFERENCE_PACKED_DECL(iq2_xxs)
GLMVX_REFERENCE_PACKED_DECL(iq3_xxs)
GLMVX_REFERENCE_PACKED_DECL(iq1_s)
GLMVX_REFERENCE_PACKED_DECL(iq4_xs)
#undef GLMVX_REFERENCE_PACKED_DECL

/* f32 primitives.  Replace kernels/kernels.h:168-184 one for one
 * (bodies kernels/kernels.vx:17-441). */
int32_t glm_vx_rmsnorm(float *out, const float *x, const float *weight, int32_t n, float eps);
int32_t glm_vx_layernorm(float *out, const float *x, const float *weight, const float *bias, int32_t n, float eps);
int32_t glm_vx_softmax(float *out, const float *x, int32_t n);
int32_t glm_vx_swiglu(float *out, const float *gate, const float *up, int32_t n);
int32_t glm_vx_add(float *out, const float *a, const float *b, int32_t n);
int32_t glm_vx_axpy(float *out, const float *x, float alpha, int32_t n);
int32_t glm_vx_matvec(float *out, const float *weight, const float *x, int32_t rows, int32_t cols);
int32_t glm_vx_matmul_nt(float *out, const float *a, const float *b, int32_t m, int32_t n, int32_t k);
int32_t glm_vx_rope(float *out, const float *x, const float *cosine, const float *sine, int32_t heads,
                    int32_t head_dim, int32_t rope_dim);
int32_t glm_vx_router(int32_t *indices, float *weights, const float *logits, const float *bias, int32_t experts,
                      int32_t k, float scale);
int32_t glm_vx_topk(int32_t *indices, const float *scores, int32_t n, int32_t k);
int32_t glm_vx_attention(float *out, float *scratch, const float *q, const float *keys, const float *values,
                         int32_t tokens, int32_t dim, int32_t value_dim, float scale);
int32_t glm_vx_sparse_attention(float *out, float *scratch, const float *q, const float *keys, const float *values,
                                const int32_t *selected, int32_t count, int32_t tokens, int32_t dim,
                                int32_t value_dim, float scale);
int32_t glm_vx_rope_offset(float *out, const float *x, const float *cosine, const float *sine, int32_t heads,
                           int32_t head_dim, int32_t rope_dim, int32_t offset);
int32_t glm_vx_index_scores(float *out, const float *q, const float *keys, const float *weights, int32_t tokens,
                            int32_t heads, int32_t dim, float qk_scale);
int32_t glm_vx_rope_glm(float *out, const float *x, const float *cosine, const float *sine, int32_t heads,
                        int32_t dim);

/* ====================================================================== *
 * 2. Resident device-pointer ABI                                          *
 * ====================================================================== */

/* Last error message of the calling thread ("" when none). */
const char *glmvx_last_error(void);
int32_t glmvx_version(void);

/* Device, memory, streams, events, graphs.  Replace the ctypes Driver API
 * runtime: CUDAContext (gpu/runtime.py:150-292), DeviceBuffer (:330-380),
 * Stream (:564-600), Event (:611-663). */
int32_t glmvx_device_count(int32_t *count);
int32_t glmvx_set_device(int32_t device);
int32_t glmvx_get_device(int32_t *device);
int32_t glmvx_device_info(int32_t device, char *name, int32_t name_len, int32_t *cc, int32_t *sms,
                          int64_t *l2_bytes, int64_t *total_mem, int32_t *smem_optin);
int32_t glmvx_malloc(void **ptr, uint64_t bytes);
int32_t glmvx_free(void *ptr);
/* Free / total device memory of the current device (cudaMemGetInfo; the
 * reference runtime's CUDAContext has no counterpart, tests use it to show
 * that an entry point allocates nothing). */
int32_t glmvx_mem_get_info(uint64_t *free_bytes, uint64_t *total_bytes);
int32_t glmvx_host_alloc(void **ptr, uint64_t bytes); /* pinned host memory */
int32_t glmvx_host_free(void *ptr);
int32_t glmvx_memcpy_htod(void *dst, const void *src, uint64_t bytes, void *stream);
int32_t glmvx_memcpy_dtoh(void *dst, const void *src, uint64_t bytes, void *stream);
int32_t glmvx_memcpy_dtod(void *dst, const void *src, uint64_t bytes, void *stream);
int32_t glmvx_memset(void *dst, int32_t value, uint64_t bytes, void *stream);
int32_t glmvx_device_synchronize(void);
int32_t glmvx_stream_create(void **stream);
int32_t glmvx_stream_destroy(void *stream);
int32_t glmvx_stream_synchronize(void *stream);
int32_t glmvx_stream_wait_event(void *stream, void *event);
int32_t glmvx_event_create(void **event);
int32_t glmvx_event_destroy(void *event);
int32_t glmvx_event_record(void *event, void *stream);
int32_t glmvx_event_synchronize(void *event);
int32_t glmvx_event_elapsed_ms(void *start, void *end, float *ms);
int32_t glmvx_graph_begin(void *stream);
int32_t glmvx_graph_end(void *stream, void **graph_exec);
int32_t glmvx_graph_launch(void *graph_exec, void *stream);
int32_t glmvx_graph_destroy(void *graph_exec);
/* Reads and clears the device word kernels set when a bounded wait expires. */
int32_t glmvx_check_device_error(int32_t *code);
/* Device address of that word (4 bytes), for an asynchronous copy back with a
   step's outputs; nonzero means call glmvx_check_device_error. */
int32_t glmvx_device_error_address(void **ptr);

/* Fused packed dequant + matvec: out[rows] = W[rows,cols] . x[cols].
 * Replaces glm_vx_packed_<kind> (kernels/packed.vx:154-470) for resident
 * weights; the reference GPU backend had no packed entry (gpu/backend.py:56). */
int32_t glmvx_packed_gemv(int32_t kind, float *out, const uint8_t *w, const float *x, int32_t rows, int32_t cols,
                          void *stream);
/* Small-batch: out[batch,rows] = x[batch,cols] . W^T, x row-major, batch <= 64.
 * Replaces glm_vx_packed_batch_v2_<kind> (kernels/packed.vx:473ff). */
int32_t glmvx_packed_gemm(int32_t kind, float *out, const uint8_t *w, const float *x, int32_t rows, int32_t cols,
                          int32_t batch, void *stream);
/* The tcgen05 packed GEMM alone: weights and activations split exactly into
 * three bf16 limbs in shared memory, six products (those above 2^-24 of the
 * leading term) in three kind::f16 MMAs per K step accumulating in f32 tensor
 * memory; any format, batch 1..64, cols a multiple of the format's raw
 * chunk (256 columns for Q8_0/Q4_K, 2048 for IQ1_S), 16-byte aligned w and x. */
int32_t glmvx_packed_gemm_tc(int32_t kind, float *out, const uint8_t *w, const float *x, int32_t rows, int32_t cols,
                             int32_t batch, void *stream);
/* As glmvx_packed_gemm; *path reports the kernel taken
 * (1 stream GEMV, 2 generic, 3 F16 element path, 5 tensor-core int8 path,
 * 6 f16 tensor-core GEMM, 7 / 8 the int8 path / f16 GEMM over equal column
 * segments of rows too long for one plan, later segments adding in order,
 * 9 the tcgen05 GEMM of glmvx_packed_gemm_tc, taken where it measured faster:
 * 33..64 tokens on long rows or many tiles, 17..32 tokens on 16384+ columns or
 * 65536+ rows). */
int32_t glmvx_packed_gemm_path(int32_t kind, float *out, const uint8_t *w, const float *x, int32_t rows,
                               int32_t cols, int32_t batch, void *stream, int32_t *path);
/* Diagnostic decode of `blocks` reference blocks (F16: elements) to f32.
 * Replaces glm_vx_unpack_<kind> (kernels/packed.vx:175-181 and siblings). */
int32_t glmvx_unpack(int32_t kind, float *out, const uint8_t *w, int64_t blocks, void *stream);

/* f32 primitives on device pointers.  Replace the reference PTX entries in
 * gpu/kernels.h:7-115 (matvec, rmsnorm(_rows), softmax(_rows), swiglu,
 * rope_glm, router, index_scores) and the CPU ones in kernels/kernels.h. */
int32_t glmvx_matvec_f32(float *out, const float *w, const float *x, int32_t rows, int32_t cols, void *stream);
int32_t glmvx_matmul_nt(float *out, const float *a, const float *b, int32_t m, int32_t n, int32_t k, void *stream);
int32_t glmvx_rmsnorm(float *out, const float *x, const float *w, int32_t rows, int32_t n, float eps, void *stream);
int32_t glmvx_layernorm(float *out, const float *x, const float *w, const float *b, int32_t rows, int32_t n,
                        float eps, void *stream);
int32_t glmvx_softmax(float *out, const float *x, int32_t rows, int32_t n, void *stream);
int32_t glmvx_swiglu(float *out, const float *gate, const float *up, int64_t n, void *stream);
int32_t glmvx_add(float *out, const float *a, const float *b, int64_t n, void *stream);
/* Sets *flag = 1 if any of x[0..n) is NaN or infinite and leaves it as it
   was otherwise: the caller zeroes it first (device pointers; lets a caller
   that copies a step's outputs back check them with one word; no reference
   counterpart -- the reference checks on the host). */
int32_t glmvx_nonfinite_flag(const float *x, int64_t n, uint32_t *flag, void *stream);
int32_t glmvx_axpy(float *out, const float *x, float alpha, int64_t n, void *stream);
int32_t glmvx_rope_offset(float *out, const float *x, const float *cosine, const float *sine, int32_t heads,
                          int32_t head_dim, int32_t rope_dim, int32_t offset, void *stream);
int32_t glmvx_rope_glm(float *out, const float *x, const float *cosine, const float *sine, int32_t heads,
                       int32_t dim, void *stream);
/* tokens rows of expert logits -> ids/weights [tokens,k]
 * (kernels/kernels.vx:252-279, gpu/kernels.vx:452-490). */
int32_t glmvx_router(int32_t *ids, float *weights, const float *logits, const float *bias, int32_t tokens,
                     int32_t experts, int32_t k, float scale, void *stream);
int64_t glmvx_topk_scratch_bytes(int32_t n);
int32_t glmvx_topk(int32_t *indices, const float *scores, int32_t n, int32_t k, void *scratch, void *stream);
int32_t glmvx_index_scores(float *out, const float *q, const float *keys, const float *w, int32_t tokens,
                           int32_t heads, int32_t dim, float qk_scale, void *stream);
int32_t glmvx_attention(float *out, float *scratch, const float *q, const float *keys, const float *values,
                        const int32_t *selected, int32_t count, int32_t tokens, int32_t dim, int32_t value_dim,
                        float scale, int32_t *bad, void *stream);
/* Absorbed-MLA decode over selected compressed KV rows, all heads
   (GLMKernels.mla_decode, gpu/runtime.py:896-915; glm_vx/model.py:209-221):
   out[h] = softmax_j(scale*(q_latent[h].latent[t_j] + q_rope[h].rope[t_j]))
   . latent[t_j], t_j = selected[h*selection_stride + j] (ids outside
   [0, tokens) skipped; selected NULL: t_j = j).  rank <= 1024, rope_dim <=
   128; scratch of glmvx_mla_scratch_bytes(heads, rank, count) bytes. */
int64_t glmvx_mla_scratch_bytes(int32_t heads, int32_t rank, int32_t count);
int32_t glmvx_mla_decode(float *out, const float *q_latent, const float *q_rope, const float *cache_latent,
                         const float *cache_rope, const int32_t *selected, int32_t heads, int32_t rank,
                         int32_t rope_dim, int32_t tokens, int32_t count, int32_t selection_stride, float scale,
                         void *scratch, uint64_t scratch_bytes, void *stream);
/* Fused DSA decode for a batch of queries over device-resident compressed
   caches (glm_vx/model.py:136-176 `_index` + :205-221 the fused attention
   branch): per query b, indexer scores of its lens[b] cached keys
   (index_scores), their stable top-min(topk, lens[b]) (topk), then the
   absorbed MLA above over those rows.  Layouts [batch][...] as in
   glmvx_index_scores / glmvx_mla_decode; caches [batch][capacity][dim];
   lens on the device; selected_out optional [batch][topk] (-1 padded).
   rank <= 512, rope_dim <= 128, topk <= 4096. */
int64_t glmvx_dsa_scratch_bytes(int32_t batch, int32_t heads, int32_t rank, int32_t capacity, int32_t topk);
int32_t glmvx_dsa_decode(float *out, int32_t *selected_out, const float *q_latent, const float *q_rope,
                         const float *q_index, const float *head_weights, const float *latents,
                         const float *rope_keys, const float *index_keys, const int32_t *lens, int32_t batch,
                         int32_t heads, int32_t rank, int32_t rope_dim, int32_t index_heads, int32_t index_dim,
                         int32_t capacity, int32_t topk, float index_scale, float scale, void *scratch,
                         uint64_t scratch_bytes, void *stream);
/* glmvx_dsa_decode with the attention stage (the first reader of q_latent and
   q_rope) waiting for `attention_inputs_ready` (a cudaEvent_t recorded after
   those queries' copy, e.g. on a second stream), so the indexer and top-k
   overlap the copy.  No reference counterpart: the reference's backend call
   (gpu/backend.py:233-254) takes host arrays and copies them before any
   kernel runs. */
int32_t glmvx_dsa_decode_wait(float *out, int32_t *selected_out, const float *q_latent, const float *q_rope,
                              const float *q_index, const float *head_weights, const float *latents,
                              const float *rope_keys, const float *index_keys, const int32_t *lens, int32_t batch,
                              int32_t heads, int32_t rank, int32_t rope_dim, int32_t index_heads, int32_t index_dim,
                              int32_t capacity, int32_t topk, float index_scale, float scale, void *scratch,
                              uint64_t scratch_bytes, void *attention_inputs_ready, void *stream);
/* One decode step's new rows (model.py:176-181, 146-151: latent, rope key and
   index key appended before indexing) written at lens[b] of each query's
   caches, then lens[b] += 1; *full (device) set for a full cache. */
int32_t glmvx_dsa_append(float *latents, float *rope_keys, float *index_keys, int32_t *lens, const float *new_latent,
                         const float *new_rope, const float *new_index, int32_t batch, int32_t capacity, int32_t rank,
                         int32_t rope_dim, int32_t index_dim, int32_t *full, void *stream);

/* Dense GEMM C[M,N] = A[M,K] B[K,N], row-major f32, the reference's resident
   GEMM contract (GEMMKernels.gemm, gpu/gemm.py:51-97; gpu/gemm.vx):
   precision 0 "f32" (f32 multiply-adds), 1 "tf32_rna" (multiplicands rounded
   to TF32 nearest/ties-away, f32 accumulation on tcgen05 tensor cores with
   TMEM accumulators).  K = 0 writes zeros; any 4-byte alignment; C must not
   overlap A or B.  err: device int32 error word (NULL: the library's own). */
int32_t glmvx_gemm(float *C, const float *A, const float *B, int32_t M, int32_t N, int32_t K, int32_t precision,
                   int32_t *err, void *stream);

/* Routed + shared MoE feed-forward layer (decode / small batches), device
 * pointers.  Replaces the per-expert Python loop of glm_vx/model.py:289-324
 * (and its grouped prefill form, glm_vx/prefill.py:44-81) for resident
 * experts: router logits (F32), sigmoid+bias top-k (kernels/kernels.vx:252-279),
 * grouping by expert, gate/up GEMVs, SwiGLU fused into the down GEMV's
 * activation load, and the ascending-expert-id weighted combine with the
 * shared expert added last.  Expert weights are packed GGML `kind` arrays
 * [experts][inter][hidden] (gate, up) and [experts][hidden][inter] (down);
 * the shared expert (all three pointers, or all NULL) has one such matrix
 * each.  `workspace` is caller scratch of glmvx_moe_workspace_bytes(...)
 * bytes; ids_out/weights_out (NULL or [tokens,top_k] device arrays) receive
 * the routing.  tokens*top_k <= 4096. */
int64_t glmvx_moe_workspace_bytes(int32_t tokens, int32_t hidden, int32_t inter, int32_t experts, int32_t top_k,
                                  int32_t has_shared);
int32_t glmvx_moe_ffn(float *y, const float *x, int32_t tokens, int32_t hidden, int32_t inter, const float *router_w,
                      const float *router_bias, int32_t experts, int32_t top_k, float scale, int32_t kind,
                      const uint8_t *gate, const uint8_t *up, const uint8_t *down, const uint8_t *shared_gate,
                      const uint8_t *shared_up, const uint8_t *shared_down, void *workspace, uint64_t workspace_bytes,
                      int32_t *ids_out, float *weights_out, void *stream);
/* glmvx_moe_ffn that also records events[0..6] (cudaEvent_t) on the stream
 * around its six stages: router logits, routing, grouping, gate+up, down,
 * combine.  For profiling; no counterpart in the reference. */
int32_t glmvx_moe_ffn_profiled(float *y, const float *x, int32_t tokens, int32_t hidden, int32_t inter,
                               const float *router_w, const float *router_bias, int32_t experts, int32_t top_k,
                               float scale, int32_t kind, const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                               const uint8_t *shared_gate, const uint8_t *shared_up, const uint8_t *shared_down,
                               void *workspace, uint64_t workspace_bytes, void *const *events, void *stream);
/* The job counts the last glmvx_moe_ffn / glmvx_moe_experts call on
 * `workspace` built, copied to counts4 (host) after synchronising `stream`:
 * two-token gate+up, two-token down, four-token gate+up, four-token down.
 * Diagnostic (which job lists a layer call used); no reference counterpart. */
int32_t glmvx_moe_job_counts(int32_t tokens, int32_t hidden, int32_t inter, int32_t experts, int32_t top_k,
                             int32_t has_shared, const void *workspace, int32_t *counts4, void *stream);
/* Expert-parallel building blocks (the reference runs all experts in one
 * process; these split glm_vx/model.py:289-324 between the rank that routes a
 * token and the rank that owns its expert).  glmvx_moe_experts: routed experts
 * for rows whose expert ids are given, y[i] = down_e(SwiGLU(gate_e x_i,
 * up_e x_i)), workspace glmvx_moe_workspace_bytes(rows, hidden, inter,
 * experts, 1, 0).  glmvx_moe_combine: ascending-expert-id weighted sum of pair
 * outputs plus optional shared-expert rows (glm_vx/model.py:305-316).
 * glmvx_gather_rows: out[i] = x[idx[i]]. */
int32_t glmvx_moe_experts(float *y, const float *x, const int32_t *expert_ids, int32_t rows, int32_t hidden,
                          int32_t inter, int32_t experts, int32_t kind, const uint8_t *gate, const uint8_t *up,
                          const uint8_t *down, void *workspace, uint64_t workspace_bytes, void *stream);
int32_t glmvx_moe_combine(float *y, const float *pair_out, const int32_t *comb, const float *combw,
                          const float *shared_rows, int32_t tokens, int32_t top_k, int32_t hidden, void *stream);
int32_t glmvx_gather_rows(float *out, const float *x, const int32_t *idx, int32_t n, int32_t cols, void *stream);
/* CUDA IPC mapping of cudaMalloc'd allocations between the rank processes of
 * one node (the expert-parallel mailboxes below): glmvx_ipc_handle writes the
 * 64-byte handle of a base pointer, glmvx_ipc_open maps a peer's handle
 * (peer access enabled on first use), glmvx_ipc_close unmaps it.  The
 * reference's runtime has no multi-process mapping (gpu/runtime.py). */
int32_t glmvx_ipc_handle(void *base, uint8_t *handle64);
int32_t glmvx_ipc_open(const uint8_t *handle64, void **ptr);
int32_t glmvx_ipc_close(void *ptr);
/* Expert-parallel sparse layer, one rank per GPU of a node (replaces the
 * NCCL all-to-all dispatch/combine the survey proposed as glmvx_ep_init /
 * dispatch / combine; the reference runs all experts in one process,
 * glm_vx/model.py:289-324).  Routed expert e lives on rank
 * e / (experts / world); router and shared expert are replicated.  Each rank
 * owns a mailbox that the other ranks store into over NVLink: prepared token
 * rows go to the expert's owner, whose down GEMV stores each output row
 * straight back into the sender's mailbox; epoch flags (system-scope
 * release / acquire, waits bounded to 2 s, then the device error word) order
 * the steps.  No host round trip inside a step; a step is capturable.
 *   glmvx_ep_create   this rank's layer: `gate`/`up`/`down` hold its own
 *                     experts/world experts, router / bias / shared expert
 *                     the full arrays (device pointers, 16-byte aligned,
 *                     kept by the caller); allocates the mailbox + scratch.
 *                     world <= 8, world * max_tokens * top_k <= 4096,
 *                     formats and widths of the tensor-core path.
 *   glmvx_ep_mailbox  this rank's mailbox (cudaMalloc'd: share it with
 *                     glmvx_ipc_handle) and its size.
 *   glmvx_ep_connect  every rank's mailbox in rank order as this process
 *                     addresses it (own included).
 *   glmvx_ep_dispatch / _experts / _combine  the three phases of a step
 *                     (route + store rows to owners; owner's experts +
 *                     return; wait + ordered combine); glmvx_ep_step = all
 *                     three.  Every rank runs every step (tokens may be 0).
 *   glmvx_ep_destroy  after every rank's last step and after the peers
 *                     unmapped this mailbox. */
int32_t glmvx_ep_create(void **layer, int32_t rank, int32_t world, int32_t max_tokens, int32_t hidden, int32_t inter,
                        int32_t experts, int32_t top_k, float scale, int32_t kind, const float *router_w,
                        const float *router_bias, const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                        const uint8_t *shared_gate, const uint8_t *shared_up, const uint8_t *shared_down);
int32_t glmvx_ep_mailbox(void *layer, void **base, uint64_t *bytes);
int32_t glmvx_ep_connect(void *layer, void *const *mailboxes);
int32_t glmvx_ep_dispatch(void *layer, const float *x, int32_t tokens, int32_t *ids_out, float *weights_out,
                          void *stream);
int32_t glmvx_ep_experts(void *layer, int32_t tokens, void *stream);
int32_t glmvx_ep_combine(void *layer, float *y, int32_t tokens, void *stream);
int32_t glmvx_ep_step(void *layer, float *y, const float *x, int32_t tokens, int32_t *ids_out, float *weights_out,
                      void *stream);
int32_t glmvx_ep_destroy(void *layer);
/* Batched decode-step pieces of the GLM-MoE-DSA model (one token for each of
 * `tokens` sequences, device pointers; the reference runs them per token on
 * the host, glm_vx/model.py:96-237, 359-392).
 *   glmvx_embed_rows   x[b] = row ids[b] of an F32 (kind 0) or Q8_0 (8) table
 *   glmvx_rope_rows    the reference rope (kernels/kernels.vx:425-441, pairs
 *                      rotated, output half-split) of `d` elements of `heads`
 *                      strided rows per sequence at position pos[b], cos/sin
 *                      from [max_pos][d/2] tables, plus `tail` copied elements
 *   glmvx_rmsnorm_rows rmsnorm of strided rows (kernels/kernels.vx:17-27)
 *   glmvx_absorb_query q_latent[b,h] = kv_b[h,:nope]^T query[b,h,:nope],
 *                      kv_b [heads][nope+vdim][rank], serial f32 sums
 *   glmvx_absorb_value out[b,h*vdim+i] = sum_r kv_b[h][nope+i][r] att[b,h,r],
 *                      kv_b [heads][nope+vdim][rank], serial f32 sums
 *   glmvx_scale        out = x * s
 *   glmvx_argmax_rows  first index of each row's maximum (numpy argmax)
 *   glmvx_fill_random  seeded synthetic weights: f32 N(0,1)*scale (or ones),
 *                      or Q8_0 / Q4_K / IQ1_S blocks of random bytes with
 *                      |N(0,1)|*scale fp16 block scales
 *   glmvx_dsa_attend   glmvx_dsa_decode's attention stage alone over given
 *                      selections [batch][topk] (-1 padded), for DSA layers
 *                      that reuse the previous layer's top-k (model.py:197-204) */
int32_t glmvx_embed_rows(float *out, const void *table, int32_t kind, const int32_t *ids, int32_t rows, int32_t vocab,
                         int32_t hidden, void *stream);
int32_t glmvx_rope_rows(float *out, const float *x, const float *cos_tab, const float *sin_tab, const int32_t *pos,
                        int32_t tokens, int32_t heads, int32_t d, int32_t tail, int64_t x_tok, int32_t x_head,
                        int32_t x_off, int64_t out_tok, int32_t out_head, int32_t out_off, int32_t max_pos,
                        void *stream);
int32_t glmvx_rmsnorm_rows(float *out, const float *x, const float *w, int32_t rows, int32_t n, int64_t x_stride,
                           int64_t out_stride, float eps, void *stream);
int32_t glmvx_absorb_query(float *q_latent, const float *query, const float *kvb, int32_t tokens, int32_t heads,
                           int32_t nope, int32_t qk_head, int32_t rank, int32_t vdim, void *stream);
int32_t glmvx_absorb_value(float *out, const float *att, const float *kvb, int32_t tokens, int32_t heads,
                           int32_t nope, int32_t rank, int32_t vdim, void *stream);
int32_t glmvx_scale(float *out, const float *x, float s, int64_t n, void *stream);
int32_t glmvx_argmax_rows(int32_t *ids, const float *logits, int32_t rows, int32_t n, void *stream);
int32_t glmvx_fill_random(void *out, int32_t kind, int64_t count, uint64_t seed, float scale, int32_t ones,
                          void *stream);
int32_t glmvx_dsa_attend(float *out, const int32_t *selected, const float *q_latent, const float *q_rope,
                         const float *latents, const float *rope_keys, const int32_t *lens, int32_t batch,
                         int32_t heads, int32_t rank, int32_t rope_dim, int32_t capacity, int32_t topk, float scale,
                         void *scratch, uint64_t scratch_bytes, void *stream);
/* FP8 E4M3FN block-scaled projection, device pointers: out[rows] =
 * sum_c (decode(weight[r,c]) * scales[r/128, c/128]) * x[c], weight u8
 * [rows, cols], scales f32 [ceil(rows/128), ceil(cols/128)].  Replaces the
 * reference's glm_vx_gpu_fp8_matvec (gpu/fp8.vx:50-89) launched by
 * GLMKernels.fp8_matvec (gpu/runtime.py:1031-1053).  rows >= 1, cols >= 0. */
int32_t glmvx_fp8_matvec(float *out, const uint8_t *weight, const float *scales, const float *x, int32_t rows,
                         int32_t cols, void *stream);
/* The same projection for a batch of tokens: out[t][r], x[t][cols] row-major.
 * 2..64 tokens with cols a multiple of 256 and 16-byte aligned weight and x
 * run on the tcgen05 GEMM (*path = 9: each weight times its tile scale in f32,
 * split exactly into three bf16 limbs, six kind::f16 MMAs per K step);
 * otherwise one glmvx_fp8_matvec per token (*path = 1).  path may be NULL.
 * The reference multiplies one token at a time (GLMKernels.fp8_matvec,
 * gpu/runtime.py:1031-1053); results agree within the f32 dot-product bound. */
int32_t glmvx_fp8_gemm(float *out, const uint8_t *weight, const float *scales, const float *x, int32_t rows,
                       int32_t cols, int32_t batch, int32_t *path, void *stream);
/* glmvx_moe_ffn without a caller workspace, for callers that cannot allocate
 * device memory (an embedding runtime that owns the whole memory budget, a
 * decode loop with a fixed footprint).  No counterpart in the reference.
 * Scratch is one 16 MiB file-scope device array per device: layers needing
 * more (glmvx_moe_workspace_bytes) are rejected with -1.  The first call on a
 * device looks the array up; make it before any stream capture.  Calls that
 * overlap in time on one device race on the array: issue them on one stream. */
int32_t glmvx_moe_ffn_static(float *y, const float *x, int32_t tokens, int32_t hidden, int32_t inter,
                             const float *router_w, const float *router_bias, int32_t experts, int32_t top_k,
                             float scale, int32_t kind, const uint8_t *gate, const uint8_t *up, const uint8_t *down,
                             const uint8_t *shared_gate, const uint8_t *shared_up, const uint8_t *shared_down,
                             int32_t *ids_out, float *weights_out, void *stream);

#ifdef __cplusplus
}
#endif
#endif /* GLMVX_H */
