// f32 model primitives on sm_100a, one device kernel per entry of the
// reference's C ABI (kernels/kernels.h:12-28, Vx bodies in kernels/kernels.vx).
// Exported with device pointers as glmvx_<op>(..., stream).
//
// Numerics: element-wise ops use the reference's operation order with IEEE
// division and square root (no fast-math).  Reductions (dot products, norms,
// softmax sums) run as parallel trees in f32, so they agree with the
// reference's ordered sums to rounding, not bit for bit.  The router's
// selection and top-k's ordering are exact functions of their scores.
#include <algorithm>
#include <cfloat>

#include "common.cuh"
#include "dsa.cuh"

namespace glmvx {


// Block-wide sum for blockDim.x == 256 (8 warps); result broadcast to all.
__device__ __forceinline__ float block_sum_256(float v, float *scratch) {
    v = warp_sum(v);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = 0.0f;
#pragma unroll
    for (int i = 0; i < 8; ++i) t += scratch[i];
    return t;
}

__device__ __forceinline__ float block_max_256(float v, float *scratch) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    __syncthreads();
    if (lane == 0) scratch[warp] = v;
    __syncthreads();
    float t = scratch[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) t = fmaxf(t, scratch[i]);
    return t;
}

// ---- f32 matvec / matmul_nt: one warp per weight row, TB tokens per slice.
template <int TB>
__global__ void __launch_bounds__(256)
    f32_rows_kernel(float *__restrict__ out, const float *__restrict__ wt, const float *__restrict__ x, int rows,
                    int cols, int batch, int out_row_major_tokens) {
    const int row = blockIdx.x * 8 + (threadIdx.x >> 5), lane = threadIdx.x & 31;
    if (row >= rows) return;
    const int t0 = blockIdx.y * TB, nt = min(TB, batch - t0);
    const float *wr = wt + static_cast<size_t>(row) * cols;
    float acc[TB];
#pragma unroll
    for (int t = 0; t < TB; ++t) acc[t] = 0.0f;
    const bool vec = ((reinterpret_cast<uintptr_t>(wr) | reinterpret_cast<uintptr_t>(x)) & 15) == 0 && (cols & 3) == 0;
    if (vec) {
        for (int c = lane * 4; c < cols; c += 128) {
            const float4 wv = __ldg(reinterpret_cast<const float4 *>(wr + c));
#pragma unroll
            for (int t = 0; t < TB; ++t)
                if (t < nt) {
                    const float4 xv = __ldg(reinterpret_cast<const float4 *>(x + static_cast<size_t>(t0 + t) * cols + c));
                    acc[t] = fmaf(wv.x, xv.x, acc[t]);
                    acc[t] = fmaf(wv.y, xv.y, acc[t]);
                    acc[t] = fmaf(wv.z, xv.z, acc[t]);
                    acc[t] = fmaf(wv.w, xv.w, acc[t]);
                }
        }
    } else {
        for (int c = lane; c < cols; c += 32) {
            const float wv = __ldg(wr + c);
#pragma unroll
            for (int t = 0; t < TB; ++t)
                if (t < nt) acc[t] = fmaf(wv, __ldg(x + static_cast<size_t>(t0 + t) * cols + c), acc[t]);
        }
    }
#pragma unroll
    for (int t = 0; t < TB; ++t) {
        const float v = warp_sum(acc[t]);
        if (lane == 0 && t < nt) {
            if (out_row_major_tokens) out[static_cast<size_t>(t0 + t) * rows + row] = v;
            else out[static_cast<size_t>(row) * batch + t0 + t] = v;
        }
    }
}

// ---- f32 matvec / matmul_nt, aligned rows: a CTA owns EB weight rows x TB
// tokens; its 8 warps split the columns (float4 per lane, coalesced), every
// loaded weight quad serves TB tokens and every activation quad EB rows.  The
// 8 warp partials of an output are summed in fixed order (deterministic).
template <int EB, int TB>
__global__ void __launch_bounds__(256)
    f32_tile_kernel(float *__restrict__ out, const float *__restrict__ wt, const float *__restrict__ x, int rows,
                    int cols, int batch, int out_row_major_tokens) {
    __shared__ float red[8][EB][TB];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int r0 = blockIdx.x * EB, t0 = blockIdx.y * TB;
    const int nr = min(EB, rows - r0), nt = min(TB, batch - t0);
    float acc[EB][TB];
#pragma unroll
    for (int e = 0; e < EB; ++e)
#pragma unroll
        for (int t = 0; t < TB; ++t) acc[e][t] = 0.0f;
    const int quads = cols >> 2;
    // The thread's quads f0, f0 + 256, ... (n of them), U at a time: U
    // iterations' loads are issued before the first is used, with no bounds
    // test between them (a guarded loop cannot move a load above the test
    // that ends it, which leaves one iteration's loads in flight).
    constexpr int U = TB > 1 ? 2 : 4;
    const int f0 = lane + 32 * warp;
    const int n = f0 < quads ? (quads - f0 + 255) / 256 : 0;
    auto load_w = [&](int f, float4 (&wv)[EB]) {
#pragma unroll
        for (int e = 0; e < EB; ++e)
            wv[e] = e < nr ? __ldg(reinterpret_cast<const float4 *>(wt + static_cast<size_t>(r0 + e) * cols) + f)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    auto load_x = [&](int f, float4 (&xv)[TB]) {
#pragma unroll
        for (int t = 0; t < TB; ++t)
            xv[t] = t < nt ? __ldg(reinterpret_cast<const float4 *>(x + static_cast<size_t>(t0 + t) * cols) + f)
                           : make_float4(0.f, 0.f, 0.f, 0.f);
    };
    auto fma_tile = [&](const float4 (&wv)[EB], const float4 (&xv)[TB]) {
#pragma unroll
        for (int e = 0; e < EB; ++e)
#pragma unroll
            for (int t = 0; t < TB; ++t) {
                acc[e][t] = fmaf(wv[e].x, xv[t].x, acc[e][t]);
                acc[e][t] = fmaf(wv[e].y, xv[t].y, acc[e][t]);
                acc[e][t] = fmaf(wv[e].z, xv[t].z, acc[e][t]);
                acc[e][t] = fmaf(wv[e].w, xv[t].w, acc[e][t]);
            }
    };
    int i = 0;
    for (; i + U <= n; i += U) {
        float4 wv[U][EB], xv[U][TB];
#pragma unroll
        for (int u = 0; u < U; ++u) {
            load_w(f0 + 256 * (i + u), wv[u]);
            load_x(f0 + 256 * (i + u), xv[u]);
        }
#pragma unroll
        for (int u = 0; u < U; ++u) fma_tile(wv[u], xv[u]);
    }
    for (; i < n; ++i) {
        float4 wv[EB], xv[TB];
        load_w(f0 + 256 * i, wv);
        load_x(f0 + 256 * i, xv);
        fma_tile(wv, xv);
    }
#pragma unroll
    for (int e = 0; e < EB; ++e)
#pragma unroll
        for (int t = 0; t < TB; ++t) {
            const float v = warp_sum(acc[e][t]);
            if (lane == 0) red[warp][e][t] = v;
        }
    __syncthreads();
    for (int i = threadIdx.x; i < EB * TB; i += 256) {
        const int e = i / TB, t = i % TB;
        if (e >= nr || t >= nt) continue;
        float v = 0.0f;
#pragma unroll
        for (int w = 0; w < 8; ++w) v += red[w][e][t];
        if (out_row_major_tokens) out[static_cast<size_t>(t0 + t) * rows + r0 + e] = v;
        else out[static_cast<size_t>(r0 + e) * batch + t0 + t] = v;
    }
}

int32_t f32_rows(float *out, const float *w, const float *x, int rows, int cols, int batch, bool token_major,
                 cudaStream_t s) {
    if (rows == 0 || batch == 0) return kOk;
    const bool vec = ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x)) & 15) == 0 && (cols & 3) == 0;
    // Tiles of EB rows x TB tokens, sized so a 256-row router gives 128-512
    // CTAs (two rows per CTA measured ~3 us faster than four at 32 tokens).
    if (vec && batch <= 1) {  // one row per CTA: a 256-row router spreads over the SMs
        f32_tile_kernel<1, 1><<<dim3(rows, 1), 256, 0, s>>>(out, w, x, rows, cols, batch, token_major);
        return launch_status("f32_tile_kernel");
    }
    if (vec && batch <= 8) {
        f32_tile_kernel<2, 8><<<dim3((rows + 1) / 2, 1), 256, 0, s>>>(out, w, x, rows, cols, batch, token_major);
        return launch_status("f32_tile_kernel");
    }
#ifndef GLMVX_TILE_EB
#define GLMVX_TILE_EB 2
#endif
    if (vec) {
        constexpr int EB = GLMVX_TILE_EB;
        f32_tile_kernel<EB, 8><<<dim3((rows + EB - 1) / EB, (batch + 7) / 8), 256, 0, s>>>(out, w, x, rows, cols,
                                                                                          batch, token_major);
        return launch_status("f32_tile_kernel");
    }
    if (batch <= 1) {
        f32_rows_kernel<1><<<dim3((rows + 7) / 8, 1), 256, 0, s>>>(out, w, x, rows, cols, batch, token_major);
    } else {
        f32_rows_kernel<8><<<dim3((rows + 7) / 8, (batch + 7) / 8), 256, 0, s>>>(out, w, x, rows, cols, batch,
                                                                                token_major);
    }
    return launch_status("f32_rows_kernel");
}

// ---- row-wise norms and softmax: one 256-thread CTA per row.
__global__ void __launch_bounds__(256) rmsnorm_kernel(float *out, const float *x, const float *w, int n, float eps) {
    __shared__ float scratch[8];
    const float *xr = x + static_cast<size_t>(blockIdx.x) * n;
    float *orow = out + static_cast<size_t>(blockIdx.x) * n;
    float ss = 0.0f;
    for (int i = threadIdx.x; i < n; i += 256) ss = fmaf(xr[i], xr[i], ss);
    ss = block_sum_256(ss, scratch);
    const float inv = 1.0f / sqrtf(ss / static_cast<float>(n) + eps);
    for (int i = threadIdx.x; i < n; i += 256) orow[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

__global__ void __launch_bounds__(256)
    layernorm_kernel(float *out, const float *x, const float *w, const float *b, int n, float eps) {
    __shared__ float scratch[8];
    const float *xr = x + static_cast<size_t>(blockIdx.x) * n;
    float *orow = out + static_cast<size_t>(blockIdx.x) * n;
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += 256) s += xr[i];
    const float mean = block_sum_256(s, scratch) / static_cast<float>(n);
    float v = 0.0f;
    for (int i = threadIdx.x; i < n; i += 256) {
        const float d = xr[i] - mean;
        v = fmaf(d, d, v);
    }
    const float inv = 1.0f / sqrtf(block_sum_256(v, scratch) / static_cast<float>(n) + eps);
    for (int i = threadIdx.x; i < n; i += 256)
        orow[i] = __fadd_rn(__fmul_rn(__fmul_rn(__fsub_rn(xr[i], mean), inv), w[i]), b[i]);
}

__global__ void __launch_bounds__(256) softmax_kernel(float *out, const float *x, int n) {
    __shared__ float scratch[8];
    const float *xr = x + static_cast<size_t>(blockIdx.x) * n;
    float *orow = out + static_cast<size_t>(blockIdx.x) * n;
    float m = -INFINITY;
    for (int i = threadIdx.x; i < n; i += 256) m = fmaxf(m, xr[i]);
    m = block_max_256(m, scratch);
    float s = 0.0f;
    for (int i = threadIdx.x; i < n; i += 256) {
        const float e = expf(xr[i] - m);
        orow[i] = e;
        s += e;
    }
    s = block_sum_256(s, scratch);
    for (int i = threadIdx.x; i < n; i += 256) orow[i] = orow[i] / s;
}

// ---- element-wise
__global__ void swiglu_kernel(float *out, const float *g, const float *u, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const float gv = g[i];
        out[i] = __fmul_rn(__fmul_rn(gv, sigmoid_ref(gv)), u[i]);  // kernels/kernels.vx:58
    }
}

__global__ void add_kernel(float *out, const float *a, const float *b, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = __fadd_rn(a[i], b[i]);
}

__global__ void axpy_kernel(float *out, const float *x, float alpha, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = __fadd_rn(out[i], __fmul_rn(alpha, x[i]));
}

// kernels/kernels.vx:226-248: rotate adjacent pairs at [offset, offset+rope_dim).
// One thread owns a whole pair (reads both, then writes both), so out == x
// (in place, allowed by kernels/kernels.h:17) is race-free.
__global__ void rope_offset_kernel(float *out, const float *x, const float *cs, const float *sn, int heads,
                                   int head_dim, int rope_dim, int offset) {
    const int64_t total = static_cast<int64_t>(heads) * head_dim;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int d = static_cast<int>(i % head_dim);
        if (d < offset || d >= offset + rope_dim) {
            out[i] = x[i];
        } else if (((d - offset) & 1) == 0) {
            const int p = (d - offset) >> 1;
            const float a = x[i], b = x[i + 1];
            out[i] = __fsub_rn(__fmul_rn(a, cs[p]), __fmul_rn(b, sn[p]));
            out[i + 1] = __fadd_rn(__fmul_rn(a, sn[p]), __fmul_rn(b, cs[p]));
        }
    }
}

// kernels/kernels.vx:425-441: interleaved pairs -> [even half | odd half].
__global__ void rope_glm_kernel(float *out, const float *x, const float *cs, const float *sn, int heads, int dim) {
    const int half = dim / 2;
    const int64_t total = static_cast<int64_t>(heads) * half;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < total;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        const int64_t h = i / half;
        const int p = static_cast<int>(i % half);
        const float a = x[h * dim + 2 * p], b = x[h * dim + 2 * p + 1];
        out[h * dim + p] = __fsub_rn(__fmul_rn(a, cs[p]), __fmul_rn(b, sn[p]));
        out[h * dim + half + p] = __fadd_rn(__fmul_rn(b, cs[p]), __fmul_rn(a, sn[p]));
    }
}

// ---- router (kernels/kernels.vx:252-279): one 256-thread CTA per token.
// score = sigmoid(logit)+bias picks experts (ties -> lower id); weights are
// the picked sigmoids / (ordered sum + 1e-20) * scale.
constexpr int kMaxRouterExperts = 4096, kMaxRouterK = 64;

__global__ void __launch_bounds__(256)
    router_kernel(int32_t *ids, float *weights, const float *logits, const float *bias, int experts, int k,
                  float scale) {
    __shared__ float score[kMaxRouterExperts];
    __shared__ float wbest[8];
    __shared__ int ibest[8];
    __shared__ int chosen[kMaxRouterK];
    const float *lr = logits + static_cast<size_t>(blockIdx.x) * experts;
    // A NaN score (non-finite activations) ranks as -inf, so every slot still
    // names a distinct expert in range; the outputs are then non-finite.
    for (int e = threadIdx.x; e < experts; e += 256) {
        const float v = sigmoid_ref(lr[e]) + bias[e];
        score[e] = isnan(v) ? -INFINITY : v;
    }
    __syncthreads();
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int slot = 0; slot < k; ++slot) {
        float bv = -INFINITY;
        int bi = INT_MAX;
        for (int e = threadIdx.x; e < experts; e += 256) {
            const float v = score[e];
            if (v > bv || (v == bv && e < bi)) {  // strict >, lower id wins ties
                bv = v;
                bi = e;
            }
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1) {
            const float ov = __shfl_xor_sync(0xffffffffu, bv, o);
            const int oi = __shfl_xor_sync(0xffffffffu, bi, o);
            if (ov > bv || (ov == bv && oi < bi)) {
                bv = ov;
                bi = oi;
            }
        }
        if (lane == 0) {
            wbest[warp] = bv;
            ibest[warp] = bi;
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            float v = wbest[0];
            int i = ibest[0];
            for (int q = 1; q < 8; ++q)
                if (wbest[q] > v || (wbest[q] == v && ibest[q] < i)) {
                    v = wbest[q];
                    i = ibest[q];
                }
            chosen[slot] = i;
            score[i] = NAN;  // excluded from later slots (never > or == anything)
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        float probs[kMaxRouterK];
        float total = 0.0f;
        for (int slot = 0; slot < k; ++slot) {
            probs[slot] = sigmoid_ref(lr[chosen[slot]]);
            total = total + probs[slot];
        }
        total = total + 1e-20f;
        for (int slot = 0; slot < k; ++slot) {
            ids[static_cast<size_t>(blockIdx.x) * k + slot] = chosen[slot];
            weights[static_cast<size_t>(blockIdx.x) * k + slot] = probs[slot] / total * scale;
        }
    }
}

// ---- exact stable top-k (kernels/kernels.vx:281-355) by sorting composite
// keys: descending score (with -0 folded onto +0), then ascending index.
__device__ __forceinline__ uint64_t topk_key(float v, int32_t i) {
    uint32_t b = __float_as_uint(v == 0.0f ? 0.0f : v);
    b = (b & 0x80000000u) ? ~b : (b | 0x80000000u);  // ascending float order
    return (static_cast<uint64_t>(~b) << 32) | static_cast<uint32_t>(i);  // ascending key = descending score
}

// Single-CTA bitonic sort of n2 (power of two) keys in `keys` (shared or global).
__device__ void bitonic_sort(uint64_t *keys, int n2) {
    for (int size = 2; size <= n2; size <<= 1) {
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            for (int i = threadIdx.x; i < n2 / 2; i += blockDim.x) {
                const int lo = 2 * i - (i & (stride - 1));
                const int hi = lo + stride;
                const bool up = (lo & size) == 0;
                const uint64_t a = keys[lo], b = keys[hi];
                if ((a > b) == up) {
                    keys[lo] = b;
                    keys[hi] = a;
                }
            }
            __syncthreads();
        }
    }
}

constexpr int kTopkSmemKeys = 4096;  // 32 KB of static shared memory

__global__ void __launch_bounds__(1024)
    topk_kernel(int32_t *indices, const float *scores, int n, int k, uint64_t *global_keys, int n2) {
    __shared__ uint64_t skeys[kTopkSmemKeys];
    uint64_t *keys = n2 <= kTopkSmemKeys ? skeys : global_keys;
    for (int i = threadIdx.x; i < n2; i += blockDim.x) keys[i] = i < n ? topk_key(scores[i], i) : ~0ull;
    __syncthreads();
    bitonic_sort(keys, n2);
    for (int i = threadIdx.x; i < k; i += blockDim.x) indices[i] = static_cast<int32_t>(keys[i] & 0xffffffffu);
}

// ---- top-k of many scores by radix selection (same order as topk_kernel):
// the descending-score key of each score (topk_key's high word) is resolved
// 12, 12 and 8 bits at a time.  After a pass the keys whose resolved bits
// are below the boundary digit are all in the top k; those equal to it are
// candidates.  As soon as both groups fit in kTopkSelectMaxK and in no more
// than the power of two the final sort needs anyway, they are gathered as
// composite (key, index) words and sorted together, which also orders ties
// by index; otherwise the three passes yield the k-th key T and the keys
// below T plus the lowest-index keys equal to T are gathered and sorted.
// One CTA, k <= kTopkSelectMaxK.  With STAGED the n keys are computed once
// into shared memory (n <= kTopkStagedScores) and every pass reads them
// there; otherwise each pass re-reads the scores.
constexpr int kTopkSelectMaxK = 4096, kTopkSelectThreads = 1024, kTopkStagedScores = 36 * 1024;
constexpr int kTopkBins = 4096;  // 12-bit digits
// sel + the merge sort's second buffer + hist, before the staged keys
constexpr int kTopkSelectSmem = 2 * kTopkSelectMaxK * 8 + kTopkBins * 4;

__device__ __forceinline__ uint64_t shfl_xor_u64(uint64_t v, int m) {
    const uint32_t lo = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(v), m);
    const uint32_t hi = __shfl_xor_sync(0xffffffffu, static_cast<uint32_t>(v >> 32), m);
    return (static_cast<uint64_t>(hi) << 32) | lo;
}

// Ascending bitonic sort of the warp's 64 words, lane l holding positions
// 2l (a) and 2l+1 (b): compare-exchanges across lanes by shuffles.
__device__ __forceinline__ void warp_sort64(uint64_t &a, uint64_t &b) {
    const int lane = threadIdx.x & 31;
#pragma unroll
    for (int size = 2; size <= 64; size <<= 1) {
        const bool up = ((2 * lane) & size) == 0;
#pragma unroll
        for (int stride = size >> 1; stride > 0; stride >>= 1) {
            if (stride == 1) {
                if ((a > b) == up) {
                    const uint64_t t = a;
                    a = b;
                    b = t;
                }
            } else {
                const int ls = stride >> 1;
                const uint64_t pa = shfl_xor_u64(a, ls), pb = shfl_xor_u64(b, ls);
                const bool keep_min = ((lane & ls) == 0) == up;
                a = keep_min ? (a < pa ? a : pa) : (a > pa ? a : pa);
                b = keep_min ? (b < pb ? b : pb) : (b > pb ? b : pb);
            }
        }
    }
}

// Ascending sort of n2 (a power of two) words of buf by warp-sorted runs of
// 64 and log2(n2/64) merge levels: each word's place in the merged run is
// its place in its own run plus its rank in the partner run (lower bound
// from the left run, upper bound from the right, so equal words keep
// distinct places).  tmp: n2 more words.  Returns the buffer holding the
// result.  Every thread of the block calls it.
__device__ uint64_t *block_merge_sort(uint64_t *buf, uint64_t *tmp, int n2) {
    if (n2 < 64) {
        bitonic_sort(buf, n2);
        return buf;
    }
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5, warps = blockDim.x >> 5;
    for (int run = warp; run < n2 / 64; run += warps) {
        uint64_t a = buf[64 * run + 2 * lane], b = buf[64 * run + 2 * lane + 1];
        warp_sort64(a, b);
        buf[64 * run + 2 * lane] = a;
        buf[64 * run + 2 * lane + 1] = b;
    }
    __syncthreads();
    uint64_t *src = buf, *dst = tmp;
    for (int len = 64; len < n2; len <<= 1) {
        for (int i = threadIdx.x; i < n2; i += blockDim.x) {
            const uint64_t x = src[i];
            const int r = i / len, p = i - r * len;
            const uint64_t *other = src + (r ^ 1) * len;
            int lo = 0, hi = len;
            if ((r & 1) == 0) {
                while (lo < hi) {
                    const int mid = (lo + hi) >> 1;
                    if (other[mid] < x) lo = mid + 1;
                    else hi = mid;
                }
            } else {
                while (lo < hi) {
                    const int mid = (lo + hi) >> 1;
                    if (other[mid] <= x) lo = mid + 1;
                    else hi = mid;
                }
            }
            dst[(r & ~1) * len + p + lo] = x;
        }
        __syncthreads();
        uint64_t *t = src;
        src = dst;
        dst = t;
    }
    return src;
}

__device__ __forceinline__ uint32_t topk_desc(float v) { return static_cast<uint32_t>(topk_key(v, 0) >> 32); }

__host__ __device__ constexpr int topk_pow2(int m) {
    int p = 1;
    while (p < m) p <<= 1;
    return p;
}

// Inclusive block scan of one int per thread (1024 threads).
__device__ __forceinline__ int block_scan_incl(int v, int *s_warp) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, v, o);
        if (lane >= o) v += y;
    }
    if (lane == 31) s_warp[warp] = v;
    __syncthreads();
    if (warp == 0) {
        int t = s_warp[lane];
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const int y = __shfl_up_sync(0xffffffffu, t, o);
            if (lane >= o) t += y;
        }
        s_warp[lane] = t;
    }
    __syncthreads();
    const int before = warp ? s_warp[warp - 1] : 0;
    __syncthreads();  // s_warp reusable
    return v + before;
}

template <bool STAGED>
__global__ void __launch_bounds__(kTopkSelectThreads, 1)
    topk_select_kernel(int32_t *indices, const float *scores, int n, int k, const int32_t *lens, int64_t score_stride,
                       int out_stride) {
    extern __shared__ __align__(16) unsigned char topk_smem[];
    uint64_t *sel = reinterpret_cast<uint64_t *>(topk_smem);
    uint64_t *sort_tmp = sel + kTopkSelectMaxK;
    int *hist = reinterpret_cast<int *>(topk_smem + 2 * kTopkSelectMaxK * 8);
    uint32_t *staged = reinterpret_cast<uint32_t *>(topk_smem + kTopkSelectSmem);
    __shared__ int s_warp[kTopkSelectThreads / 32];
    __shared__ int s_digit, s_rank, s_bin, s_count, s_ties;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    // Query blockIdx.x of a batch: min(k, its length) positions, then -1.
    scores += blockIdx.x * score_stride;
    indices += static_cast<int64_t>(blockIdx.x) * out_stride;
    if (lens) n = min(n, max(0, lens[blockIdx.x]));
    for (int i = min(k, n) + tid; i < k; i += kTopkSelectThreads) indices[i] = -1;
    k = min(k, n);
    if (k == 0) return;
    const uint32_t lanes_below = (1u << lane) - 1u;
    auto key_at = [&](int i) -> uint32_t { return STAGED ? staged[i] : topk_desc(__ldg(scores + i)); };
    const int k2 = topk_pow2(k);
    uint32_t prefix = 0, mask = 0;
    int rank = k;  // 1-based position of the k-th key among those matching prefix
    int bin = n;   // keys matching prefix
    bool gathered = false;
    for (int pass = 0; pass < 3; ++pass) {
        const int bits = pass < 2 ? 12 : 8, shift = pass == 0 ? 20 : pass == 1 ? 8 : 0, nb = 1 << bits;
        for (int i = tid; i < nb; i += kTopkSelectThreads) hist[i] = 0;
        __syncthreads();
        if (STAGED && pass == 0) {  // the keys are staged while the first digit is counted (every key counts)
#pragma unroll 8
            for (int i = tid; i < n; i += kTopkSelectThreads) {
                const uint32_t key = topk_desc(__ldg(scores + i));
                staged[i] = key;
                atomicAdd(&hist[key >> shift], 1);
            }
        } else {
            for (int i = tid; i < n; i += kTopkSelectThreads) {
                const uint32_t key = key_at(i);
                if ((key & mask) == prefix) atomicAdd(&hist[(key >> shift) & (nb - 1)], 1);
            }
        }
        __syncthreads();
        // The digit holding the rank-th key: each thread sums nb / 1024 bins.
        const int per = nb / kTopkSelectThreads > 0 ? nb / kTopkSelectThreads : 1;
        const int b0 = tid * per;
        int local = 0;
        for (int j = 0; j < per; ++j)
            if (b0 + j < nb) local += hist[b0 + j];
        int excl = block_scan_incl(local, s_warp) - local;
        if (excl < rank && rank <= excl + local) {  // exactly one thread: rank >= 1 and the total covers rank
            for (int j = 0; j < per; ++j) {
                const int c = hist[b0 + j];
                if (rank <= excl + c) {
                    s_digit = b0 + j;
                    s_rank = rank - excl;
                    s_bin = c;
                    break;
                }
                excl += c;
            }
        }
        __syncthreads();
        prefix |= static_cast<uint32_t>(s_digit) << shift;
        mask |= static_cast<uint32_t>(nb - 1) << shift;
        rank = s_rank;
        bin = s_bin;
        const int m = k - rank + bin;  // keys below the boundary digit + candidates
        if (m <= kTopkSelectMaxK && (topk_pow2(m) == k2 || pass == 2)) {
            gathered = true;
            break;
        }
    }
    if (tid == 0) s_count = s_ties = 0;
    __syncthreads();
    int m = k;  // sorted words
    if (gathered) {  // every key with (key & mask) <= prefix, in index order
        m = k - rank + bin;
        // Warp w takes a contiguous chunk of the keys: it counts its keys by
        // ballots, the warps' counts give each warp its first slot, and it
        // writes them there (no shared counter to contend on).
        constexpr int kWarps = kTopkSelectThreads / 32;
        const int chunk = ((n + kWarps - 1) / kWarps + 31) & ~31;
        const int begin = warp * chunk, end = min(n, begin + chunk);
        int count = 0;
        for (int i0 = begin; i0 < end; i0 += 32) {
            const int i = i0 + lane;
            count += __popc(__ballot_sync(0xffffffffu, i < end && (key_at(i) & mask) <= prefix));
        }
        if (lane == 0) s_warp[warp] = count;
        __syncthreads();
        int base = 0;
        for (int w = 0; w < warp; ++w) base += s_warp[w];
        for (int i0 = begin; i0 < end; i0 += 32) {
            const int i = i0 + lane;
            const uint32_t key = i < end ? key_at(i) : ~0u;
            const uint32_t take = __ballot_sync(0xffffffffu, i < end && (key & mask) <= prefix);
            if (take >> lane & 1u)
                sel[base + __popc(take & lanes_below)] = (static_cast<uint64_t>(key) << 32) | static_cast<uint32_t>(i);
            base += __popc(take);
        }
    } else {
        // prefix = T, with more keys equal to T than fit: the k - rank keys
        // below T, then the lowest-index `rank` keys equal to T, chunks of the
        // block in index order.
        for (int i0 = tid - lane; i0 < n; i0 += kTopkSelectThreads) {
            const int i = i0 + lane;
            const uint32_t key = i < n ? key_at(i) : ~0u;
            const uint32_t below = __ballot_sync(0xffffffffu, i < n && key < prefix);
            if (below) {
                int base = 0;
                if (lane == 0) base = atomicAdd(&s_count, __popc(below));
                base = __shfl_sync(0xffffffffu, base, 0);
                if (below >> lane & 1u)
                    sel[base + __popc(below & lanes_below)] = (static_cast<uint64_t>(key) << 32) | static_cast<uint32_t>(i);
            }
        }
        const uint64_t tkey = static_cast<uint64_t>(prefix) << 32;
        int taken = 0;
        for (int c0 = 0; c0 < n && taken < rank; c0 += kTopkSelectThreads) {
            const int i = c0 + tid;
            const bool is_tie = i < n && key_at(i) == prefix;
            const int before = block_scan_incl(is_tie ? 1 : 0, s_warp) - (is_tie ? 1 : 0) + taken;
            if (is_tie && before < rank) sel[k - rank + before] = tkey | static_cast<uint32_t>(i);
            if (tid == kTopkSelectThreads - 1) s_ties = before + (is_tie ? 1 : 0);
            __syncthreads();
            taken = s_ties;
            __syncthreads();
        }
    }
    const int m2 = topk_pow2(m);
    for (int i = m + tid; i < m2; i += kTopkSelectThreads) sel[i] = ~0ull;
    __syncthreads();
    const uint64_t *sorted = block_merge_sort(sel, sort_tmp, m2);
    for (int i = tid; i < k; i += kTopkSelectThreads) indices[i] = static_cast<int32_t>(sorted[i] & 0xffffffffu);
}

// ---- DSA index scores (kernels/kernels.vx:404-421): score_t = sum_h w_h *
// relu(scale * q_h . k_t).  Four threads per token, each taking every
// fourth head of a 32-head block (kIndexSplit-way split keeps ~28 warps per SM in flight
// over the key stream): the block's queries, up to 128 columns at a time,
// sit in shared memory (read as broadcasts, four columns per load with VEC);
// each thread streams its token's key row in 16-column pieces (the four
// threads of a token share the lines through L1) and keeps 8 running dots
// in registers; the four partial totals meet by shuffles.  VEC: dim a
// multiple of 16 and keys 16-byte aligned.
constexpr int kIndexHeadBlock = 32, kIndexDimBlock = 128, kIndexThreads = 128, kIndexSplit = 4;
constexpr int kIndexHeadsPerThread = kIndexHeadBlock / kIndexSplit, kIndexTokensPerCta = kIndexThreads / kIndexSplit;
constexpr int kIndexStride = kIndexDimBlock + 4;  // padded query row (floats)

template <bool VEC>
__global__ void __launch_bounds__(kIndexThreads, 8)
    index_scores_kernel(float *out, const float *q, const float *keys, const float *w, int tokens, int heads,
                        int dim, float qk_scale, const int32_t *lens, int64_t key_stride, int64_t out_stride) {
    __shared__ __align__(16) float sq[kIndexHeadBlock * kIndexStride];
    const int b = blockIdx.y;  // query of a batch: its own keys, queries, weights and length
    if (lens) tokens = min(tokens, max(0, lens[b]));
    if (static_cast<int>(blockIdx.x) * kIndexTokensPerCta >= tokens) return;  // whole CTA past the keys
    q += static_cast<size_t>(b) * heads * dim;
    w += static_cast<size_t>(b) * heads;
    keys += b * key_stride;
    out += b * out_stride;
    const int part = threadIdx.x % kIndexSplit;
    const int t = blockIdx.x * kIndexTokensPerCta + threadIdx.x / kIndexSplit;
    const bool live = t < tokens;
    const float *kr = keys + static_cast<size_t>(live ? t : 0) * dim;
    float total = 0.0f;
    for (int h0 = 0; h0 < heads; h0 += kIndexHeadBlock) {
        const int nh = min(kIndexHeadBlock, heads - h0);
        // This thread's heads within the block: part, part + 4, ... (the four
        // threads of a token then read queries 16 bytes apart, no bank conflict).
        float dot[kIndexHeadsPerThread];
#pragma unroll
        for (int h = 0; h < kIndexHeadsPerThread; ++h) dot[h] = 0.0f;
        for (int c0 = 0; c0 < dim; c0 += kIndexDimBlock) {
            const int nc = min(kIndexDimBlock, dim - c0);
            __syncthreads();  // the previous block of q is no longer read
            for (int i = threadIdx.x; i < nh * nc; i += kIndexThreads) {
                const int h = i / nc, c = i - h * nc;
                sq[h * kIndexStride + c] = q[static_cast<size_t>(h0 + h) * dim + c0 + c];
            }
            __syncthreads();
            if (!live || part >= nh) continue;
            for (int d = 0; d < nc; d += 16) {
                float kv[16];
                if (VEC) {
#pragma unroll
                    for (int i = 0; i < 4; ++i) {
                        const float4 v = __ldg(reinterpret_cast<const float4 *>(kr + c0 + d) + i);
                        kv[4 * i] = v.x, kv[4 * i + 1] = v.y, kv[4 * i + 2] = v.z, kv[4 * i + 3] = v.w;
                    }
                } else {
#pragma unroll
                    for (int i = 0; i < 16; ++i) kv[i] = d + i < nc ? __ldg(kr + c0 + d + i) : 0.0f;
                }
#pragma unroll
                for (int h = 0; h < kIndexHeadsPerThread; ++h) {
                    if (part + kIndexSplit * h < nh) {
                        const float *qh = sq + (part + kIndexSplit * h) * kIndexStride + d;
                        float acc = dot[h];
                        if (VEC) {
#pragma unroll
                            for (int i = 0; i < 4; ++i) {
                                const float4 a = reinterpret_cast<const float4 *>(qh)[i];
                                acc = fmaf(a.x, kv[4 * i], acc);
                                acc = fmaf(a.y, kv[4 * i + 1], acc);
                                acc = fmaf(a.z, kv[4 * i + 2], acc);
                                acc = fmaf(a.w, kv[4 * i + 3], acc);
                            }
                        } else {
#pragma unroll
                            for (int i = 0; i < 16; ++i)
                                if (d + i < nc) acc = fmaf(qh[i], kv[i], acc);
                        }
                        dot[h] = acc;
                    }
                }
            }
        }
#pragma unroll
        for (int h = 0; h < kIndexHeadsPerThread; ++h) {
            if (part + kIndexSplit * h < nh) {
                const float s = dot[h] * qk_scale;
                if (s > 0.0f) total = fmaf(__ldg(w + h0 + part + kIndexSplit * h), s, total);
            }
        }
    }
    // The token's four partial totals, added in a fixed order.
    total += __shfl_xor_sync(0xffffffffu, total, 1);
    total += __shfl_xor_sync(0xffffffffu, total, 2);
    if (live && part == 0) out[t] = total;
}

// ---- single-query attention over all or selected tokens
// (kernels/kernels.vx:358-400): scores -> softmax -> weighted value sum, one
// CTA.  `scratch` holds one f32 per attended token.  A selected id outside
// [0, tokens) is never dereferenced: it sets *bad and the host rejects the
// call, as the reference does before touching memory (kernels/kernels.vx:385).
__global__ void __launch_bounds__(256)
    attention_kernel(float *out, float *scratch, const float *q, const float *keys, const float *values,
                     const int32_t *selected, int count, int tokens, int dim, int value_dim, float scale,
                     int32_t *bad) {
    __shared__ float red[8];
    __shared__ int any_bad;
    if (threadIdx.x == 0) any_bad = 0;
    __syncthreads();
    if (selected)
        for (int j = threadIdx.x; j < count; j += 256)
            if (selected[j] < 0 || selected[j] >= tokens) any_bad = 1;
    __syncthreads();
    if (any_bad) {
        if (threadIdx.x == 0 && bad) *bad = 1;
        return;
    }
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    for (int j = warp; j < count; j += 8) {
        const int t = selected ? selected[j] : j;
        const float *kr = keys + static_cast<size_t>(t) * dim;
        float dot = 0.0f;
        for (int d = lane; d < dim; d += 32) dot = fmaf(q[d], kr[d], dot);
        dot = warp_sum(dot);
        if (lane == 0) scratch[j] = dot * scale;
    }
    __syncthreads();
    float m = -INFINITY;
    for (int j = threadIdx.x; j < count; j += 256) m = fmaxf(m, scratch[j]);
    m = block_max_256(m, red);
    float s = 0.0f;
    for (int j = threadIdx.x; j < count; j += 256) {
        const float e = expf(scratch[j] - m);
        scratch[j] = e;
        s += e;
    }
    s = block_sum_256(s, red);
    for (int j = threadIdx.x; j < count; j += 256) scratch[j] = scratch[j] / s;
    __syncthreads();
    for (int d = threadIdx.x; d < value_dim; d += 256) {
        float acc = 0.0f;
        for (int j = 0; j < count; ++j) {
            const int t = selected ? selected[j] : j;
            acc = fmaf(scratch[j], values[static_cast<size_t>(t) * value_dim + d], acc);
        }
        out[d] = acc;
    }
}

static int ew_grid(int64_t n) { return static_cast<int>(std::max<int64_t>(1, std::min<int64_t>((n + 255) / 256, 4 * 148 * 8))); }

// Batched launches shared with the fused DSA decode (mla.cu); `batch`
// queries along the grid's y (index scores) or x (top-k) dimension.
int32_t launch_index_scores_batch(float *out, const float *q, const float *keys, const float *w, int tokens,
                                  int heads, int dim, float qk_scale, const int32_t *lens, int64_t key_stride,
                                  int64_t out_stride, int batch, cudaStream_t stream) {
    if (tokens <= 0 || batch <= 0) return kOk;
    const int32_t tc = launch_index_scores_tc(out, q, keys, w, tokens, heads, dim, qk_scale, lens, key_stride,
                                              out_stride, batch, stream);
    if (tc != kUnsupported) return tc;
    const bool vec = dim % 16 == 0 && (reinterpret_cast<uintptr_t>(keys) & 15) == 0 && key_stride % 4 == 0;
    const dim3 grid((tokens + kIndexTokensPerCta - 1) / kIndexTokensPerCta, batch);
    if (vec)
        index_scores_kernel<true><<<grid, kIndexThreads, 0, stream>>>(out, q, keys, w, tokens, heads, dim, qk_scale,
                                                                      lens, key_stride, out_stride);
    else
        index_scores_kernel<false><<<grid, kIndexThreads, 0, stream>>>(out, q, keys, w, tokens, heads, dim,
                                                                       qk_scale, lens, key_stride, out_stride);
    return launch_status("index_scores_kernel");
}

int32_t launch_topk_batch(int32_t *indices, const float *scores, int n, int k, const int32_t *lens,
                          int64_t score_stride, int out_stride, int batch, cudaStream_t stream) {
    if (k <= 0 || k > kTopkSelectMaxK) return set_error("topk: 1 <= k <= %d", kTopkSelectMaxK), kInvalid;
    if (batch <= 0) return kOk;
    const bool staged = n <= kTopkStagedScores;
    const int smem = kTopkSelectSmem + (staged ? n * 4 : 0);
    if (const int32_t rc = staged ? allow_dynamic_smem(topk_select_kernel<true>, smem, "topk_select smem")
                                  : allow_dynamic_smem(topk_select_kernel<false>, smem, "topk_select smem"))
        return rc;
    if (staged)
        topk_select_kernel<true><<<batch, kTopkSelectThreads, smem, stream>>>(indices, scores, n, k, lens,
                                                                             score_stride, out_stride);
    else
        topk_select_kernel<false><<<batch, kTopkSelectThreads, smem, stream>>>(indices, scores, n, k, lens,
                                                                              score_stride, out_stride);
    return launch_status("topk_select_kernel");
}

}  // namespace glmvx

using namespace glmvx;
#define S_ (cudaStream_t) stream

__global__ void gather_rows_kernel(float *out, const float *x, const int32_t *idx, int n, int cols) {
    const int r = blockIdx.y;
    const float *src = x + static_cast<size_t>(idx[r]) * cols;
    float *dst = out + static_cast<size_t>(r) * cols;
    for (int c = blockIdx.x * blockDim.x + threadIdx.x; c < cols; c += gridDim.x * blockDim.x) dst[c] = src[c];
}

// out[i, :] = x[idx[i], :] for i < n (device pointers; idx must be in range).
GLMVX_EXPORT int32_t glmvx_gather_rows(float *out, const float *x, const int32_t *idx, int32_t n, int32_t cols,
                                       void *stream) {
    if (n < 0 || cols < 0) return set_error("gather rows dims"), kInvalid;
    if (!n || !cols) return kOk;
    gather_rows_kernel<<<dim3((cols + 255) / 256, n), 256, 0, S_>>>(out, x, idx, n, cols);
    return launch_status("gather_rows_kernel");
}

GLMVX_EXPORT int32_t glmvx_matvec_f32(float *out, const float *w, const float *x, int32_t rows, int32_t cols,
                                      void *stream) {
    if (rows < 0 || cols < 0) return set_error("matvec dims"), kInvalid;
    if (cols == 0) {
        if (rows) GLMVX_CUDA(cudaMemsetAsync(out, 0, sizeof(float) * rows, S_));
        return kOk;
    }
    return f32_rows(out, w, x, rows, cols, 1, true, S_);
}

// out[m,n] = a[m,k] . b[n,k]^T (kernels/kernels.vx:135-218).
GLMVX_EXPORT int32_t glmvx_matmul_nt(float *out, const float *a, const float *b, int32_t m, int32_t n, int32_t k,
                                     void *stream) {
    if (m < 0 || n < 0 || k < 0) return set_error("matmul_nt dims"), kInvalid;
    if (k == 0) {
        if (m && n) GLMVX_CUDA(cudaMemsetAsync(out, 0, sizeof(float) * m * n, S_));
        return kOk;
    }
    return f32_rows(out, b, a, n, k, m, true, S_);
}

GLMVX_EXPORT int32_t glmvx_rmsnorm(float *out, const float *x, const float *w, int32_t rows, int32_t n, float eps,
                                   void *stream) {
    if (n <= 0 || eps <= 0.0f || rows < 0) return set_error("rmsnorm dims/eps"), kInvalid;
    if (rows) rmsnorm_kernel<<<rows, 256, 0, S_>>>(out, x, w, n, eps);
    return launch_status("rmsnorm_kernel");
}

GLMVX_EXPORT int32_t glmvx_layernorm(float *out, const float *x, const float *w, const float *b, int32_t rows,
                                     int32_t n, float eps, void *stream) {
    if (n <= 0 || eps <= 0.0f || rows < 0) return set_error("layernorm dims/eps"), kInvalid;
    if (rows) layernorm_kernel<<<rows, 256, 0, S_>>>(out, x, w, b, n, eps);
    return launch_status("layernorm_kernel");
}

GLMVX_EXPORT int32_t glmvx_softmax(float *out, const float *x, int32_t rows, int32_t n, void *stream) {
    if (n <= 0 || rows < 0) return set_error("softmax dims"), kInvalid;
    if (rows) softmax_kernel<<<rows, 256, 0, S_>>>(out, x, n);
    return launch_status("softmax_kernel");
}

GLMVX_EXPORT int32_t glmvx_swiglu(float *out, const float *gate, const float *up, int64_t n, void *stream) {
    if (n < 0) return set_error("swiglu n"), kInvalid;
    if (n) swiglu_kernel<<<ew_grid(n), 256, 0, S_>>>(out, gate, up, n);
    return launch_status("swiglu_kernel");
}

GLMVX_EXPORT int32_t glmvx_add(float *out, const float *a, const float *b, int64_t n, void *stream) {
    if (n < 0) return set_error("add n"), kInvalid;
    if (n) add_kernel<<<ew_grid(n), 256, 0, S_>>>(out, a, b, n);
    return launch_status("add_kernel");
}

constexpr int kFlagThreads = 256, kFlagVecPerThread = 4;

// Sets *flag when a block sees a NaN or infinity; blocks that see none write
// nothing, so the caller zeroes the flag (the write is the same 1 from every
// block that writes).
__global__ void __launch_bounds__(kFlagThreads) nonfinite_kernel(const float *__restrict__ x, int64_t n, uint32_t *flag) {
    bool bad = false;
    const int64_t stride = static_cast<int64_t>(gridDim.x) * kFlagThreads;
    const int64_t first = static_cast<int64_t>(blockIdx.x) * kFlagThreads + threadIdx.x;
    int64_t scalar_from = 0;
    if ((reinterpret_cast<uintptr_t>(x) & 15) == 0) {
        const int64_t n4 = n / 4;
        for (int64_t i = first; i < n4; i += stride) {
            const float4 v = __ldg(reinterpret_cast<const float4 *>(x) + i);
            bad |= !isfinite(v.x) || !isfinite(v.y) || !isfinite(v.z) || !isfinite(v.w);
        }
        scalar_from = 4 * n4;
    }
    for (int64_t i = scalar_from + first; i < n; i += stride) bad |= !isfinite(__ldg(x + i));
    if (__syncthreads_or(bad) && threadIdx.x == 0) *flag = 1u;
}

GLMVX_EXPORT int32_t glmvx_nonfinite_flag(const float *x, int64_t n, uint32_t *flag, void *stream) {
    if (n < 0 || !flag || (n && !x)) return set_error("nonfinite_flag: bad arguments"), kInvalid;
    if (n == 0) return kOk;
    const int64_t units = (reinterpret_cast<uintptr_t>(x) & 15) ? n : n / 4 + 3;
    const int64_t per_block = static_cast<int64_t>(kFlagThreads) * kFlagVecPerThread;
    const int blocks = static_cast<int>(std::min<int64_t>((units + per_block - 1) / per_block, 4 * 148));
    nonfinite_kernel<<<blocks, kFlagThreads, 0, S_>>>(x, n, flag);
    return launch_status("nonfinite_kernel");
}

GLMVX_EXPORT int32_t glmvx_axpy(float *out, const float *x, float alpha, int64_t n, void *stream) {
    if (n < 0) return set_error("axpy n"), kInvalid;
    if (n) axpy_kernel<<<ew_grid(n), 256, 0, S_>>>(out, x, alpha, n);
    return launch_status("axpy_kernel");
}

GLMVX_EXPORT int32_t glmvx_rope_offset(float *out, const float *x, const float *cs, const float *sn, int32_t heads,
                                       int32_t head_dim, int32_t rope_dim, int32_t offset, void *stream) {
    if (heads < 0 || rope_dim < 0 || offset < 0 || head_dim < rope_dim || offset > head_dim - rope_dim ||
        rope_dim % 2 != 0)
        return set_error("rope dims"), kInvalid;
    const int64_t n = static_cast<int64_t>(heads) * head_dim;
    if (n) rope_offset_kernel<<<ew_grid(n), 256, 0, S_>>>(out, x, cs, sn, heads, head_dim, rope_dim, offset);
    return launch_status("rope_offset_kernel");
}

GLMVX_EXPORT int32_t glmvx_rope_glm(float *out, const float *x, const float *cs, const float *sn, int32_t heads,
                                    int32_t dim, void *stream) {
    if (heads < 0 || dim <= 0 || dim % 2 != 0) return set_error("rope_glm dims"), kInvalid;
    const int64_t n = static_cast<int64_t>(heads) * (dim / 2);
    if (n) rope_glm_kernel<<<ew_grid(n), 256, 0, S_>>>(out, x, cs, sn, heads, dim);
    return launch_status("rope_glm_kernel");
}

// tokens x experts logits -> ids/weights [tokens, k].
GLMVX_EXPORT int32_t glmvx_router(int32_t *ids, float *weights, const float *logits, const float *bias,
                                  int32_t tokens, int32_t experts, int32_t k, float scale, void *stream) {
    if (k <= 0 || experts < k || tokens < 0) return set_error("router k/experts"), kInvalid;
    if (experts > kMaxRouterExperts || k > kMaxRouterK)
        return set_error("GPU router supports at most %d experts and k <= %d", kMaxRouterExperts, kMaxRouterK),
               kUnsupported;
    if (tokens) router_kernel<<<tokens, 256, 0, S_>>>(ids, weights, logits, bias, experts, k, scale);
    return launch_status("router_kernel");
}

// Scratch bytes glmvx_topk needs for n scores (0 when it sorts in shared memory).
GLMVX_EXPORT int64_t glmvx_topk_scratch_bytes(int32_t n) {
    if (n > (1 << 30)) return -1;
    int64_t n2 = 1;
    while (n2 < n) n2 <<= 1;
    return n2 <= kTopkSmemKeys ? 0 : n2 * 8;
}

GLMVX_EXPORT int32_t glmvx_topk(int32_t *indices, const float *scores, int32_t n, int32_t k, void *scratch,
                                void *stream) {
    if (n < 0 || k < 0 || n < k) return set_error("topk n/k"), kInvalid;
    if (n > (1 << 30)) return set_error("topk: at most 2^30 scores"), kInvalid;
    if (k == 0) return kOk;
    int64_t n2 = 1;
    while (n2 < n) n2 <<= 1;
    if (n2 > kTopkSmemKeys && k <= kTopkSelectMaxK) {  // many scores, bounded k: radix selection
        return launch_topk_batch(indices, scores, n, k, nullptr, 0, 0, 1, S_);
    }
    if (n2 > kTopkSmemKeys && !scratch) return set_error("topk needs scratch for n > %d", kTopkSmemKeys), kInvalid;
    topk_kernel<<<1, 1024, 0, S_>>>(indices, scores, n, k, static_cast<uint64_t *>(scratch), n2);
    return launch_status("topk_kernel");
}

GLMVX_EXPORT int32_t glmvx_index_scores(float *out, const float *q, const float *keys, const float *w,
                                        int32_t tokens, int32_t heads, int32_t dim, float qk_scale, void *stream) {
    if (tokens < 0 || heads <= 0 || dim <= 0) return set_error("index_scores dims"), kInvalid;
    return launch_index_scores_batch(out, q, keys, w, tokens, heads, dim, qk_scale, nullptr, 0, 0, 1, S_);
}

// selected == nullptr attends to the first `count` tokens.  `bad` (device
// int32, required when `selected` is given) is set to 1 when a selected id is
// out of range; the kernel then writes nothing and the host must reject.
GLMVX_EXPORT int32_t glmvx_attention(float *out, float *scratch, const float *q, const float *keys,
                                     const float *values, const int32_t *selected, int32_t count, int32_t tokens,
                                     int32_t dim, int32_t value_dim, float scale, int32_t *bad, void *stream) {
    if (count <= 0 || tokens <= 0 || dim <= 0 || value_dim <= 0) return set_error("attention dims"), kInvalid;
    if (!selected && count > tokens) return set_error("attention count > tokens"), kInvalid;
    if (selected && !bad) return set_error("attention with selected ids needs a status word"), kInvalid;
    attention_kernel<<<1, 256, 0, S_>>>(out, scratch, q, keys, values, selected, count, tokens, dim, value_dim,
                                        scale, bad);
    return launch_status("attention_kernel");
}
