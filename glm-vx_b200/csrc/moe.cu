// Routed + shared MoE feed-forward layer on sm_100a (decode and small batches).
//
// Semantics follow the reference model exactly (glm_vx/model.py:289-324 and
// glm_vx/prefill.py:44-81):
//   logits  = router_w . x                          (F32 matvec)
//   ids, w  = top-k of sigmoid(logits)+bias, w = sigmoid/(sum+1e-20)*scale
//             (kernels/kernels.vx:252-279)
//   y       = sum over the token's experts in ascending expert id of
//             down_e(SwiGLU(gate_e x, up_e x)) * w, then + shared(x)
//
// Device pipeline, no host round trip:
//   1. router logits     f32 GEMV/GEMM                     (ops.cu)
//   2. top-k routing     one CTA per token                 (ops.cu)
//   3. grouping          one CTA: assignments sorted by (expert, token), the
//                        gate/up/down job descriptors and each token's
//                        ascending-id combine order        (this file)
//   4. gate+up           packed GEMV over the gate and up jobs
//   5. down              packed GEMV over the down jobs, input SwiGLU(g, u)
//   6. combine           weighted sum in reference order   (this file)
// P = tokens*top_k (+ tokens for the shared expert) (token, expert) pairs.
//
// Formats and widths the tensor-core path takes (mma_gemv.cuh) use it: the
// token rows are prepared once (limbs) before step 1, the SwiGLU of each
// pair's gate/up outputs is prepared after step 4, and each job applies one
// expert matrix to TWO tokens routed to it, so an expert's weights are
// decoded once per pair of its tokens; from 16 tokens per call, IQ1_S experts
// routed three or more tokens and the shared expert go to a second job list
// of FOUR tokens per job (its own launch of the same kernel with two token
// pairs per decoded fragment).  Other formats run one streaming GEMV
// job per pair (packed_gemv.cu) with SwiGLU fused into the activation load.
// Jobs are ordered by expert so tokens sharing an expert stream its rows
// close together in time (L2 reuse).
#include <climits>
#include <mutex>

#include "codecs.cuh"
#include "gemv_jobs.cuh"
#include "mma_gemv.cuh"
#include "moe_jobs.cuh"

namespace glmvx {

struct MoeWorkspace {
    float *logits;
    int32_t *ids;
    float *wts;
    GemvJob *gu_jobs, *dn_jobs;
    int32_t *comb;
    float *combw;
    float *g_out, *u_out, *pair_out;
    uint8_t *xprep, *hprep;      // prepared token rows / SwiGLU inputs (tensor-core path)
    MmaJob *gu_mjobs, *dn_mjobs;  // two tokens per job
    MmaJob *gu_qjobs, *dn_qjobs;  // four tokens per job (experts with three or more)
    int *counts;                  // [gate+up, down] jobs of each list, written by the grouping kernel
    size_t bytes;
};

static MoeWorkspace carve(char *base, int T, int hidden, int inter, int E, int k, bool shared) {
    MoeWorkspace w{};
    size_t off = 0;
    auto take = [&](size_t n) {
        char *p = base ? base + off : nullptr;
        off += (n + 255) & ~static_cast<size_t>(255);
        return p;
    };
    const size_t P = static_cast<size_t>(T) * k + (shared ? T : 0);
    w.logits = reinterpret_cast<float *>(take(4ull * T * E));
    w.ids = reinterpret_cast<int32_t *>(take(4ull * T * k));
    w.wts = reinterpret_cast<float *>(take(4ull * T * k));
    w.gu_jobs = reinterpret_cast<GemvJob *>(take(sizeof(GemvJob) * 2 * P));
    w.dn_jobs = reinterpret_cast<GemvJob *>(take(sizeof(GemvJob) * P));
    w.comb = reinterpret_cast<int32_t *>(take(4ull * T * k));
    w.combw = reinterpret_cast<float *>(take(4ull * T * k));
    w.g_out = reinterpret_cast<float *>(take(4ull * P * inter));
    w.u_out = reinterpret_cast<float *>(take(4ull * P * inter));
    w.pair_out = reinterpret_cast<float *>(take(4ull * P * hidden));
    w.xprep = reinterpret_cast<uint8_t *>(take(T * prep_stride(hidden)));
    w.hprep = reinterpret_cast<uint8_t *>(take(P * prep_stride(inter)));
    w.gu_mjobs = reinterpret_cast<MmaJob *>(take(sizeof(MmaJob) * 2 * P));
    w.dn_mjobs = reinterpret_cast<MmaJob *>(take(sizeof(MmaJob) * P));
    w.gu_qjobs = reinterpret_cast<MmaJob *>(take(sizeof(MmaJob) * 2 * P));
    w.dn_qjobs = reinterpret_cast<MmaJob *>(take(sizeof(MmaJob) * P));
    w.counts = reinterpret_cast<int *>(take(4 * sizeof(int)));
    w.bytes = off;
    return w;
}

#ifndef GLMVX_QUAD_MIN_TOKENS
#define GLMVX_QUAD_MIN_TOKENS 16
#endif
constexpr int kQuadMinTokens = GLMVX_QUAD_MIN_TOKENS;

// Addresses of the single-GPU layer's assignments for form_mma_jobs:
// assignment a is token a / k; every pair's down output is row r of pair_out.
struct LocalJobSrc {
    const uint8_t *gate, *up, *down, *sgate, *sup, *sdown, *xprep;
    size_t gu_stride, dn_stride, xstride;
    float *pair_out;
    int k, hidden;
    __device__ const uint8_t *wg(int e) const { return gate + e * gu_stride; }
    __device__ const uint8_t *wu(int e) const { return up + e * gu_stride; }
    __device__ const uint8_t *wd(int e) const { return down + e * dn_stride; }
    __device__ const uint8_t *sg() const { return sgate; }
    __device__ const uint8_t *su() const { return sup; }
    __device__ const uint8_t *sd() const { return sdown; }
    __device__ const uint8_t *xp(int a) const { return xprep + static_cast<size_t>(a / k) * xstride; }
    __device__ float *out(int, int r) const { return pair_out + static_cast<size_t>(r) * hidden; }
    __device__ const uint8_t *xp_shared(int t) const { return xprep + static_cast<size_t>(t) * xstride; }
    __device__ float *out_shared(int, int r) const { return pair_out + static_cast<size_t>(r) * hidden; }
};

// Small batches are routed inside the grouping kernel (one launch less on
// the latency-bound decode path), with router_kernel's rules exactly (ops.cu,
// kernels/kernels.vx:252-279): score = sigmoid(logit) + bias, a NaN score
// ranked -inf; the experts ranked 0..k-1 by (larger score, then lower id) are
// the k picks in selection order; weight = the pick's sigmoid over the picks'
// sigmoids summed in that order + 1e-20, times scale.  Every (token, expert)
// is ranked by one thread against the token's row of scores in shared
// memory, so the ids and weights are byte-identical to router_kernel's.
constexpr int kFusedRouteExperts = 256, kFusedRouteTokens = 2;

// Rank each (token, slot) assignment by (expert id, token): the rank is its
// pair index, so pairs of one expert are contiguous and ordered by token.
// With `logits` set the kernel first routes every token itself (small
// batches, see kFusedRouteTokens), writing ids / wts.
// With mjobs set (tensor-core path) the job lists come from form_mma_jobs
// (moe_jobs.cuh): two tokens per job, and with qjobs set too experts routed
// three or more pairs and the shared expert in a list of four tokens per job.
// Otherwise one streaming GEMV job per pair (GemvJob).
__global__ void __launch_bounds__(kGroupThreads)
    moe_group_kernel(int32_t *ids, float *wts, int T, int k, int E, int shared, const uint8_t *gate,
                     const uint8_t *up, const uint8_t *down, size_t gu_stride, size_t dn_stride, const uint8_t *sgate,
                     const uint8_t *sup, const uint8_t *sdown, const float *x, int hidden, int inter, float *g_out,
                     float *u_out, float *pair_out, GemvJob *gu_jobs, GemvJob *dn_jobs, int32_t *comb, float *combw,
                     int *bad, MmaJob *gu_m, MmaJob *dn_m, MmaJob *gu_q, MmaJob *dn_q, int *counts,
                     const uint8_t *xprep, size_t xstride, const uint8_t *hprep, size_t hstride, const float *logits,
                     const float *bias, float scale) {
    __shared__ GroupSmem g;
    __shared__ float route_score[kFusedRouteTokens * kFusedRouteExperts];
    const int n = T * k;
    const int P = n + (shared ? T : 0);
    const bool mma = gu_m != nullptr;
    if (logits) {  // T <= kFusedRouteTokens, E <= kFusedRouteExperts (host-checked)
        for (int i = threadIdx.x; i < T * E; i += blockDim.x) {
            const int e = i % E;
            const float v = sigmoid_ref(logits[i]) + bias[e];
            route_score[i] = isnan(v) ? -INFINITY : v;
        }
        __syncthreads();
        for (int i = threadIdx.x; i < T * E; i += blockDim.x) {
            const int t = i / E, e = i % E;
            const float *row = route_score + t * E;
            const float v = row[e];
            int rank = 0;
            for (int f = 0; f < E; ++f) {
                const float u = row[f];
                rank += (u > v) | ((u == v) & (f < e));
            }
            if (rank < k) {
                ids[t * k + rank] = e;
                wts[t * k + rank] = sigmoid_ref(logits[i]);
            }
        }
        __syncthreads();
        for (int t = threadIdx.x; t < T; t += blockDim.x) {
            float total = 0.0f;
            for (int s = 0; s < k; ++s) total = total + wts[t * k + s];
            total = total + 1e-20f;
            for (int s = 0; s < k; ++s) wts[t * k + s] = wts[t * k + s] / total * scale;
        }
        __syncthreads();  // the block's writes to ids / wts are visible to every thread
    }
    for (int a = threadIdx.x; a < n; a += blockDim.x) {
        const int e = ids[a];
        g.ids[a] = static_cast<int16_t>(min(max(e, 0), E - 1));
        if (e < 0 || e >= E) report_device_error(bad, kDevErrBadIndex);
    }
    __syncthreads();
    if (mma) {
        const LocalJobSrc src{gate, up, down, sgate, sup, sdown, xprep, gu_stride, dn_stride, xstride, pair_out, k,
                              hidden};
        form_mma_jobs(src, g, n, shared ? T : 0, gu_q != nullptr, g_out, u_out, hprep, hstride, inter, gu_m, dn_m,
                      gu_q, dn_q, counts);
    } else {
        for (int a = threadIdx.x; a < n; a += blockDim.x) {
            const int e = g.ids[a];
            int lt = 0, eq = 0;
            for (int b = 0; b < n; ++b) {
                const int eb = g.ids[b];
                lt += eb < e;
                eq += (eb == e) & (b < a);
            }
            const int rank = lt + eq;
            g.pair[a] = static_cast<int16_t>(rank);
            const int t = a / k;
            gu_jobs[rank] = GemvJob{gate + e * gu_stride, x + static_cast<size_t>(t) * hidden, nullptr,
                                    g_out + static_cast<size_t>(rank) * inter};
            gu_jobs[P + rank] = GemvJob{up + e * gu_stride, x + static_cast<size_t>(t) * hidden, nullptr,
                                        u_out + static_cast<size_t>(rank) * inter};
            dn_jobs[rank] = GemvJob{down + e * dn_stride, g_out + static_cast<size_t>(rank) * inter,
                                    u_out + static_cast<size_t>(rank) * inter,
                                    pair_out + static_cast<size_t>(rank) * hidden};
        }
        if (shared) {
            for (int t = threadIdx.x; t < T; t += blockDim.x) {
                const int p = n + t;
                gu_jobs[p] = GemvJob{sgate, x + static_cast<size_t>(t) * hidden, nullptr,
                                     g_out + static_cast<size_t>(p) * inter};
                gu_jobs[P + p] = GemvJob{sup, x + static_cast<size_t>(t) * hidden, nullptr,
                                         u_out + static_cast<size_t>(p) * inter};
                dn_jobs[p] = GemvJob{sdown, g_out + static_cast<size_t>(p) * inter,
                                     u_out + static_cast<size_t>(p) * inter, pair_out + static_cast<size_t>(p) * hidden};
            }
        }
        __syncthreads();
    }
    // Each token's slots in ascending expert id (glm_vx/model.py:305-316).
    for (int t = threadIdx.x; t < T; t += blockDim.x) {
        for (int i = 0; i < k; ++i) {
            const int a = t * k + i, e = g.ids[a];
            int pos = 0;
            for (int j = 0; j < k; ++j) pos += g.ids[t * k + j] < e;
            comb[t * k + pos] = g.pair[a];
            combw[t * k + pos] = wts[a];
        }
    }
}

// y[t] = ((0 + o_0*w_0) + o_1*w_1 + ...) + shared_t, each product and sum
// rounded separately as the reference's f32 array arithmetic does.
// shared_rows (nullable) holds the shared expert's output of each token.
__global__ void moe_combine_kernel(float *y, const float *pair_out, const int32_t *comb, const float *combw, int T,
                                   int k, int hidden, const float *shared_rows) {
    const int t = blockIdx.y;
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    if (h >= hidden) return;
    float r = 0.0f;
    for (int i = 0; i < k; ++i) {
        const int p = comb[t * k + i];
        r = __fadd_rn(r, __fmul_rn(pair_out[static_cast<size_t>(p) * hidden + h], combw[t * k + i]));
    }
    if (shared_rows) r = __fadd_rn(r, shared_rows[static_cast<size_t>(t) * hidden + h]);
    y[static_cast<size_t>(t) * hidden + h] = r;
}

__global__ void fill_kernel(float *p, float v, int n) {
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) p[i] = v;
}

}  // namespace glmvx

using namespace glmvx;

GLMVX_EXPORT int64_t glmvx_moe_workspace_bytes(int32_t tokens, int32_t hidden, int32_t inter, int32_t experts,
                                               int32_t top_k, int32_t has_shared) {
    if (tokens < 0 || hidden <= 0 || inter <= 0 || experts <= 0 || top_k <= 0) return -1;
    return static_cast<int64_t>(carve(nullptr, tokens, hidden, inter, experts, top_k, has_shared != 0).bytes + 256);
}

// Job counts the last glmvx_moe_ffn / glmvx_moe_experts call on `workspace`
// built (device -> host, synchronising `stream`): [0] gate+up and [1] down
// jobs of two tokens, [2] gate+up and [3] down jobs of four tokens.  Zero
// four-token jobs means that list was not used; the CUDA-core path (formats
// without the tensor-core kernel) builds none of these lists.
GLMVX_EXPORT int32_t glmvx_moe_job_counts(int32_t tokens, int32_t hidden, int32_t inter, int32_t experts,
                                          int32_t top_k, int32_t has_shared, const void *workspace,
                                          int32_t *counts4, void *stream) {
    if (tokens <= 0 || hidden <= 0 || inter <= 0 || experts <= 0 || top_k <= 0 || !workspace || !counts4) {
        set_error("moe job counts: invalid arguments");
        return kInvalid;
    }
    const char *base = static_cast<const char *>(workspace);
    base += (256 - (reinterpret_cast<uintptr_t>(base) & 255)) & 255;
    const MoeWorkspace w = carve(const_cast<char *>(base), tokens, hidden, inter, experts, top_k, has_shared != 0);
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    GLMVX_CUDA(cudaMemcpyAsync(counts4, w.counts, 4 * sizeof(int), cudaMemcpyDeviceToHost, st));
    GLMVX_CUDA(cudaStreamSynchronize(st));
    return kOk;
}

static int32_t moe_ffn(float *y, const float *x, int32_t tokens, int32_t hidden, int32_t inter, const float *router_w,
                       const float *router_bias, int32_t experts, int32_t top_k, float scale, int32_t kind,
                       const uint8_t *gate, const uint8_t *up, const uint8_t *down, const uint8_t *shared_gate,
                       const uint8_t *shared_up, const uint8_t *shared_down, void *workspace, uint64_t workspace_bytes,
                       int32_t *ids_out, float *weights_out, void *stream, void *const *events,
                       const int32_t *given_ids = nullptr) {
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (tokens < 0 || hidden <= 0 || inter <= 0 || experts <= 0 || top_k <= 0 || top_k > experts || experts > 32767) {
        set_error("moe: invalid dimensions");
        return kInvalid;
    }
    if (static_cast<int64_t>(tokens) * top_k > kMaxAssignments) {
        set_error("moe: at most %d token-expert assignments per call", kMaxAssignments);
        return kInvalid;
    }
    const bool shared = shared_gate && shared_up && shared_down;
    if (!shared && (shared_gate || shared_up || shared_down)) {
        set_error("moe: shared expert needs gate, up and down");
        return kInvalid;
    }
    if (tokens == 0) return kOk;
    int blk = 0, bytes = 0;
    if (!reference_layout(kind, blk, bytes) || hidden % blk || inter % blk) {
        set_error("moe: unsupported expert format or block-misaligned dims");
        return kUnsupported;
    }
    char *base = static_cast<char *>(workspace);
    const uintptr_t mis = (256 - (reinterpret_cast<uintptr_t>(base) & 255)) & 255;
    base += mis;
    MoeWorkspace w = carve(base, tokens, hidden, inter, experts, top_k, shared);
    if (!workspace || w.bytes + mis > workspace_bytes) {
        set_error("moe: workspace needs %zu bytes", static_cast<size_t>(w.bytes + mis));
        return kInvalid;
    }
    const size_t gu_stride = static_cast<size_t>(inter) * (hidden / blk) * bytes;
    const size_t dn_stride = static_cast<size_t>(hidden) * (inter / blk) * bytes;
    const int P = tokens * top_k + (shared ? tokens : 0);
    auto mark = [&](int i) -> int32_t {
        if (events) GLMVX_CUDA(cudaEventRecord(static_cast<cudaEvent_t>(events[i]), st));
        return kOk;
    };
    auto a16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    const bool mma = mma_supported(kind, hidden) && mma_supported(kind, inter) && a16(x) && a16(gate) && a16(up) &&
                     a16(down) && (!shared || (a16(shared_gate) && a16(shared_up) && a16(shared_down)));
    // Four-token jobs pay off from about 16 tokens (experts sharing three or
    // more tokens, the shared expert); below, their two extra launches cost
    // more than they save.
    const bool quad = mma && tokens >= kQuadMinTokens && mma_quad_supported(kind, hidden) &&
                      mma_quad_supported(kind, inter);
    // Up to 64 tokens over up to 256 experts: the grouping kernel routes the
    // tokens itself (a warp per token) instead of a separate router launch.
    const bool fused_route = !given_ids && experts <= kFusedRouteExperts && tokens <= kFusedRouteTokens;
    int32_t st_ = mark(0);
    if (st_) return st_;
    if (mma && (st_ = prep_rows_device(w.xprep, x, nullptr, tokens, hidden, st))) return st_;
    if (given_ids) {  // routing supplied by the caller: unit combine weights
        GLMVX_CUDA(cudaMemcpyAsync(w.ids, given_ids, 4ull * tokens * top_k, cudaMemcpyDeviceToDevice, st));
        fill_kernel<<<(tokens * top_k + 255) / 256, 256, 0, st>>>(w.wts, 1.0f, tokens * top_k);
        if ((st_ = launch_status("fill_kernel")) || (st_ = mark(1)) || (st_ = mark(2))) return st_;
    } else {
        st_ = glmvx_matmul_nt(w.logits, x, router_w, tokens, experts, hidden, st);
        if (st_ || (st_ = mark(1))) return st_;
        if (!fused_route) {
            st_ = glmvx_router(w.ids, w.wts, w.logits, router_bias, tokens, experts, top_k, scale, st);
            if (st_) return st_;
        }
        if ((st_ = mark(2))) return st_;
    }
    moe_group_kernel<<<1, kGroupThreads, 0, st>>>(
        w.ids, w.wts, tokens, top_k, experts, shared, gate, up, down, gu_stride, dn_stride, shared_gate, shared_up,
        shared_down, x, hidden, inter, w.g_out, w.u_out, w.pair_out, w.gu_jobs, w.dn_jobs, w.comb, w.combw,
        device_error_word(), mma ? w.gu_mjobs : nullptr, w.dn_mjobs, quad ? w.gu_qjobs : nullptr, w.dn_qjobs, w.counts,
        w.xprep, prep_stride(hidden), w.hprep, prep_stride(inter), fused_route ? w.logits : nullptr, router_bias, scale);
    if ((st_ = launch_status("moe_group_kernel")) || (st_ = mark(3))) return st_;
    if (mma) {
        const MmaJob none{};
        if ((st_ = mma_gemv_device(kind, none, w.gu_mjobs, w.counts, 2 * P, 0, inter, hidden, st)) ||
            (quad && (st_ = mma_gemv_device(kind, none, w.gu_qjobs, w.counts + 2, 2 * P, 0, inter, hidden, st,
                                             nullptr, 2))) ||
            (st_ = mark(4)))
            return st_;
        if ((st_ = prep_rows_device(w.hprep, w.g_out, w.u_out, P, inter, st)) ||
            (st_ = mma_gemv_device(kind, none, w.dn_mjobs, w.counts + 1, P, 0, hidden, inter, st)) ||
            (quad && (st_ = mma_gemv_device(kind, none, w.dn_qjobs, w.counts + 3, P, 0, hidden, inter, st, nullptr,
                                             2))) ||
            (st_ = mark(5)))
            return st_;
    } else {
        if ((st_ = gemv_jobs_device(kind, w.gu_jobs, 2 * P, inter, hidden, gate, x, st)) || (st_ = mark(4)))
            return st_;
        if ((st_ = gemv_jobs_device(kind, w.dn_jobs, P, hidden, inter, down, w.g_out, st)) || (st_ = mark(5)))
            return st_;
    }
    moe_combine_kernel<<<dim3((hidden + 255) / 256, tokens), 256, 0, st>>>(
        y, w.pair_out, w.comb, w.combw, tokens, top_k, hidden,
        shared ? w.pair_out + static_cast<size_t>(tokens) * top_k * hidden : nullptr);
    if ((st_ = launch_status("moe_combine_kernel")) || (st_ = mark(6))) return st_;
    if (ids_out) GLMVX_CUDA(cudaMemcpyAsync(ids_out, w.ids, 4ull * tokens * top_k, cudaMemcpyDeviceToDevice, st));
    if (weights_out)
        GLMVX_CUDA(cudaMemcpyAsync(weights_out, w.wts, 4ull * tokens * top_k, cudaMemcpyDeviceToDevice, st));
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_moe_ffn(float *y, const float *x, int32_t tokens, int32_t hidden, int32_t inter,
                                   const float *router_w, const float *router_bias, int32_t experts, int32_t top_k,
                                   float scale, int32_t kind, const uint8_t *gate, const uint8_t *up,
                                   const uint8_t *down, const uint8_t *shared_gate, const uint8_t *shared_up,
                                   const uint8_t *shared_down, void *workspace, uint64_t workspace_bytes,
                                   int32_t *ids_out, float *weights_out, void *stream) {
    return moe_ffn(y, x, tokens, hidden, inter, router_w, router_bias, experts, top_k, scale, kind, gate, up, down,
                   shared_gate, shared_up, shared_down, workspace, workspace_bytes, ids_out, weights_out, stream,
                   nullptr);
}

// As glmvx_moe_ffn, also recording events[0..6] on the stream around its six
// stages (router logits, routing, grouping, gate+up, down, combine).
GLMVX_EXPORT int32_t glmvx_moe_ffn_profiled(float *y, const float *x, int32_t tokens, int32_t hidden, int32_t inter,
                                            const float *router_w, const float *router_bias, int32_t experts,
                                            int32_t top_k, float scale, int32_t kind, const uint8_t *gate,
                                            const uint8_t *up, const uint8_t *down, const uint8_t *shared_gate,
                                            const uint8_t *shared_up, const uint8_t *shared_down, void *workspace,
                                            uint64_t workspace_bytes, void *const *events, void *stream) {
    return moe_ffn(y, x, tokens, hidden, inter, router_w, router_bias, experts, top_k, scale, kind, gate, up, down,
                   shared_gate, shared_up, shared_down, workspace, workspace_bytes, nullptr, nullptr, stream, events);
}

// Routed experts only, for rows whose experts are already chosen (the owner
// rank's half of expert parallelism): y[i] = down_e(SwiGLU(gate_e x_i,
// up_e x_i)) with e = expert_ids[i] in [0, experts).  The same grouping,
// tensor-core jobs and ordering as glmvx_moe_ffn with one slot per row and no
// router; workspace = glmvx_moe_workspace_bytes(rows, hidden, inter, experts,
// 1, 0).  Out-of-range ids set the device error word (kDevErrBadIndex).
GLMVX_EXPORT int32_t glmvx_moe_experts(float *y, const float *x, const int32_t *expert_ids, int32_t rows,
                                       int32_t hidden, int32_t inter, int32_t experts, int32_t kind,
                                       const uint8_t *gate, const uint8_t *up, const uint8_t *down, void *workspace,
                                       uint64_t workspace_bytes, void *stream) {
    if (rows > 0 && !expert_ids) {
        set_error("moe experts: expert ids required");
        return kInvalid;
    }
    return moe_ffn(y, x, rows, hidden, inter, nullptr, nullptr, experts, 1, 1.0f, kind, gate, up, down, nullptr,
                   nullptr, nullptr, workspace, workspace_bytes, nullptr, nullptr, stream, nullptr, expert_ids);
}

// y[t] = ((0 + pair_out[comb[t,0]]*combw[t,0]) + ...) + shared_rows[t]: the
// reference's ascending-expert-id combine (glm_vx/model.py:305-316) over pair
// outputs gathered from elsewhere; shared_rows may be NULL.
GLMVX_EXPORT int32_t glmvx_moe_combine(float *y, const float *pair_out, const int32_t *comb, const float *combw,
                                       const float *shared_rows, int32_t tokens, int32_t top_k, int32_t hidden,
                                       void *stream) {
    if (tokens < 0 || top_k <= 0 || hidden <= 0) {
        set_error("moe combine: invalid dimensions");
        return kInvalid;
    }
    if (!tokens) return kOk;
    moe_combine_kernel<<<dim3((hidden + 255) / 256, tokens), 256, 0, static_cast<cudaStream_t>(stream)>>>(
        y, pair_out, comb, combw, tokens, top_k, hidden, shared_rows);
    return launch_status("moe_combine_kernel");
}

// ---------------------------------------------------------------------------
// Scratch-free variant of glmvx_moe_ffn.
//
// Some callers cannot hand this layer a workspace: a host that embeds the
// layer inside another runtime whose allocator owns the device's whole memory
// budget (it has no way to carve out a buffer for us), or a decode loop that
// must run with a fixed memory footprint and may not allocate when a larger
// batch first appears.  This entry keeps its scratch in one file-scope device
// array instead, so it never calls cudaMalloc, cudaFree or any allocating
// library routine.
//
// Limits and rules:
//  * The array holds kStaticMoeScratchBytes (16 MiB) per device; a layer whose
//    workspace (glmvx_moe_workspace_bytes) is larger is rejected with
//    kInvalid before anything is launched.  BASELINE-sized layers (hidden
//    6144, intermediate 2048, top-8 plus a shared expert) fit up to 35 tokens.
//  * Every scratch byte is written by an earlier stage of the same call
//    before any stage reads it, so nothing has to start at zero and no
//    clearing is done.
//  * The first call on each device looks the array's address up with
//    cudaGetSymbolAddress (with that device current) and caches it; make that
//    first call before any stream capture on the device.
//  * There is ONE array per device: calls whose work overlaps in time (two
//    streams, or two host threads, on the same device) race on it.  Callers
//    serialise such calls, e.g. by issuing them on one stream.
constexpr size_t kStaticMoeScratchBytes = 16ull << 20;
constexpr int kStaticMoeMaxDevices = 64;
static __device__ __align__(256) unsigned char g_moe_scratch[kStaticMoeScratchBytes];

static int32_t static_moe_scratch(void **out) {
    static std::mutex mu;
    static void *cached[kStaticMoeMaxDevices] = {nullptr};
    int dev = 0;
    GLMVX_CUDA(cudaGetDevice(&dev));
    if (dev < 0 || dev >= kStaticMoeMaxDevices) {
        set_error("moe static: device %d is beyond the %d devices this entry supports", dev, kStaticMoeMaxDevices);
        return kInvalid;
    }
    std::lock_guard<std::mutex> lock(mu);
    if (!cached[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_moe_scratch);
        if (e != cudaSuccess) return cuda_fail(e, "cudaGetSymbolAddress(g_moe_scratch)");
        cached[dev] = p;
    }
    *out = cached[dev];
    return kOk;
}

GLMVX_EXPORT int32_t glmvx_moe_ffn_static(float *y, const float *x, int32_t tokens, int32_t hidden, int32_t inter,
                                          const float *router_w, const float *router_bias, int32_t experts,
                                          int32_t top_k, float scale, int32_t kind, const uint8_t *gate,
                                          const uint8_t *up, const uint8_t *down, const uint8_t *shared_gate,
                                          const uint8_t *shared_up, const uint8_t *shared_down, int32_t *ids_out,
                                          float *weights_out, void *stream) {
    if (tokens < 0 || hidden <= 0 || inter <= 0 || experts <= 0 || top_k <= 0) {
        set_error("moe: invalid dimensions");
        return kInvalid;
    }
    const bool shared = shared_gate && shared_up && shared_down;
    const size_t need = carve(nullptr, tokens, hidden, inter, experts, top_k, shared).bytes;
    if (need > kStaticMoeScratchBytes) {
        set_error("moe static: this layer needs %zu scratch bytes; the static scratch holds %zu", need,
                  kStaticMoeScratchBytes);
        return kInvalid;
    }
    void *scratch = nullptr;
    const int32_t st = static_moe_scratch(&scratch);
    if (st) return st;
    return moe_ffn(y, x, tokens, hidden, inter, router_w, router_bias, experts, top_k, scale, kind, gate, up, down,
                   shared_gate, shared_up, shared_down, scratch, kStaticMoeScratchBytes, ids_out, weights_out, stream,
                   nullptr);
}
