// Absorbed-MLA decode attention over DSA-selected compressed KV rows.
//
// Contract of the reference's fused entry (GLMKernels.mla_decode,
// gpu/runtime.py:896-915, kernels glm_vx_gpu_mla_partial / _merge,
// gpu/kernels.vx:204-310; model use glm_vx/model.py:209-221): for each head h
//   s_j   = scale * (q_latent[h] . latent[t_j] + q_rope[h] . rope[t_j])
//   out[h] = sum_j softmax(s)_j * latent[t_j]
// over the selected token ids t_j = selected[h * selection_stride + j]
// (j < count; ids outside [0, tokens) are skipped), the latent serving as
// both key and value.  f32 throughout with an online (running max) softmax
// per partition and a stable merge of the partitions.
//
// Layout here: a CTA takes a contiguous range (a split) of the selected ids;
// the lanes of a warp hold interleaved columns of a head's query and running
// output (column lane + 32i).  With one selection for all heads (the DSA
// case: the indexer's top-k is per query token) mla_shared_kernel stages
// tiles of the selected [latent | rope] rows in shared memory with cp.async,
// three tiles in flight, and each of its 8 warps scores and accumulates two
// heads against every staged row: a row crosses L2 once per 16 heads and
// each shared-memory word read feeds two heads.  Per-head selections take
// mla_partial_kernel, a warp per head reading its rows directly.  The merge
// takes one warp per head and 128-column block, a float4 of columns per lane.
#include <algorithm>
#include <cmath>

#include "common.cuh"
#include "dsa.cuh"

namespace glmvx {

namespace {

constexpr int kMlaHeadsPerCta = 8, kMlaMaxSplits = 64, kMlaBatch = 4;
constexpr int kMlaTileRows = 8, kMlaStages = 3, kMlaMinRowsPerSplit = 16;
constexpr int kMlaTargetCtas = 148;
#ifndef GLMVX_MLA_TC
#define GLMVX_MLA_TC 1
#endif
// Shared selections of up to 64 heads take the tensor-core partials
// (mla_tc.cu) from kMlaTcMinRows selected rows per call (over all queries):
// below that its few CTAs, each a chain of ~34 dependent load + MMA steps,
// lose to the CUDA-core kernel's one CTA per SM (measured at 2048 rows per
// query: 1 and 2 queries faster on CUDA cores, 4 and more on tensor cores).
constexpr bool kMlaUseTensorCores = GLMVX_MLA_TC != 0;
constexpr int64_t kMlaTcMinRows = 3 * 2048;  // one wave: the shared kernel holds one CTA per SM
constexpr int kMergeCols = 128;  // columns per merge warp

__device__ __forceinline__ void cp_async16(void *dst, const void *src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async4(void *dst, const void *src) {
    asm volatile("cp.async.ca.shared.global [%0], [%1], 4;" ::"r"(smem_addr(dst)), "l"(src) : "memory");
}
__device__ __forceinline__ void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
template <int N>
__device__ __forceinline__ void cp_async_wait() {
    asm volatile("cp.async.wait_group %0;" ::"n"(N) : "memory");
}

// Sums each of v[0..N) (N = 8 or 16) over the warp by halving exchanges (N
// shuffles instead of 5N), then hands every lane all N totals.
template <int N>
__device__ __forceinline__ void warp_sum_n(float (&v)[N]) {
    static_assert(N == 8 || N == 16, "8 or 16 values");
    constexpr int kLow = N == 16 ? 2 : 4;  // lanes sharing one value after the halving
    const int lane = threadIdx.x & 31;
    constexpr int kSteps = N == 16 ? 4 : 3;
#pragma unroll
    for (int step = 0; step < kSteps; ++step) {
        const int half = N >> (step + 1), bit = 16 >> step;
        const bool up = lane & bit;
#pragma unroll
        for (int i = 0; i < half; ++i) {
            const float send = up ? v[i] : v[i + half], keep = up ? v[i + half] : v[i];
            v[i] = keep + __shfl_xor_sync(0xffffffffu, send, bit);
        }
    }
#pragma unroll
    for (int step = kSteps; step < 5; ++step) v[0] += __shfl_xor_sync(0xffffffffu, v[0], 16 >> step);
    const float total = v[0];  // lane L: total of value L / kLow
#pragma unroll
    for (int i = 0; i < N; ++i) v[i] = __shfl_sync(0xffffffffu, total, kLow * i);
}

__device__ __forceinline__ float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// Latent column of a lane's i-th value in mla_shared_kernel: four adjacent
// columns per lane in each 128-column group, so rows are read as float4.
__device__ __forceinline__ int latent_col(int i, int lane) { return 128 * (i >> 2) + 4 * lane + (i & 3); }

// Cache row of selection position j of a shared list, -1 when j is past the
// split or the id is outside [0, tokens).
__device__ __forceinline__ int mla_row(const int32_t *selected, int j, int j1, int tokens) {
    if (j >= j1) return -1;
    const int t = selected ? __ldg(selected + j) : j;
    return t >= 0 && t < tokens ? t : -1;
}

// One selection for all heads, rank <= 512.  RPL (a multiple of 4) latent
// and PPL (2 or 4) rope values per lane, laid out as latent_col and
// PPL * lane + i, read from the staged rows as float4 / float2; HPW heads per
// warp; VEC: rank and rope_dim multiples of 4 and both caches 16-byte
// aligned (16-byte copies).  One CTA per SM: the compiler batches the
// unrolled shared-memory loads, which needs more than 128 registers.
template <int RPL, int PPL, int HPW, bool VEC>
__global__ void __launch_bounds__(32 * kMlaHeadsPerCta, 1)
    mla_shared_kernel(float *__restrict__ numerator, float *__restrict__ stats, const float *__restrict__ q_latent,
                      const float *__restrict__ q_rope, const float *__restrict__ latent,
                      const float *__restrict__ rope, const int32_t *__restrict__ selected, int heads, int rank,
                      int rope_dim, int tokens, int count, int splits, float scale, const int32_t *__restrict__ lens,
                      int64_t latent_stride, int64_t rope_stride, int64_t sel_stride) {
    constexpr int W = 32 * (RPL + PPL), kRowsFloats = kMlaTileRows * W;  // staged row: latent | rope
    extern __shared__ __align__(16) float tile[];                       // [kMlaStages][kMlaTileRows][W]
    grid_dependency_wait();
    allow_dependent_launch();
    {  // query blockIdx.z of a batch: its own queries, cache rows, selection and length
        const int bq = blockIdx.z;
        if (lens) {
            tokens = min(tokens, max(0, lens[bq]));
            count = min(count, tokens);
        }
        q_latent += static_cast<size_t>(bq) * heads * rank;
        q_rope += static_cast<size_t>(bq) * heads * rope_dim;
        latent += bq * latent_stride;
        rope += bq * rope_stride;
        if (selected) selected += bq * sel_stride;
        numerator += static_cast<size_t>(bq) * splits * heads * rank;
        stats += static_cast<size_t>(bq) * splits * heads * 2;
    }
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    constexpr int NV = kMlaTileRows * HPW;
    int hs[HPW];
#pragma unroll
    for (int a = 0; a < HPW; ++a) hs[a] = static_cast<int>(blockIdx.y) * kMlaHeadsPerCta * HPW + kMlaHeadsPerCta * a + warp;
    // Padding columns stay zero for the whole kernel.
    for (int i = tid; i < kMlaStages * kRowsFloats; i += 32 * kMlaHeadsPerCta) tile[i] = 0.0f;
    float q[HPW][RPL], qr[HPW][PPL], acc[HPW][RPL];
#pragma unroll
    for (int a = 0; a < HPW; ++a) {
        const bool live = hs[a] < heads;
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
            const int d = latent_col(i, lane);
            q[a][i] = live && d < rank ? q_latent[static_cast<size_t>(hs[a]) * rank + d] : 0.0f;
            acc[a][i] = 0.0f;
        }
#pragma unroll
        for (int i = 0; i < PPL; ++i) {
            const int d = PPL * lane + i;
            qr[a][i] = live && d < rope_dim ? q_rope[static_cast<size_t>(hs[a]) * rope_dim + d] : 0.0f;
        }
    }
    const int per = (count + splits - 1) / splits;
    const int j0 = min(count, static_cast<int>(blockIdx.x) * per), j1 = min(count, j0 + per);
    const int ntiles = (j1 - j0 + kMlaTileRows - 1) / kMlaTileRows;
    __syncthreads();  // the zero fill lands before any copy into the tiles
    // Stage tile tt: selected rows by copy, skipped rows (past the split, or
    // ids out of range) as zeros so that stale values never meet a zero weight.
    auto issue = [&](int tt) {
        if (tt < ntiles) {
            float *dst = tile + (tt % kMlaStages) * kRowsFloats;
            const int jb = j0 + tt * kMlaTileRows;
            const int unit = VEC ? 4 : 1, rq = rank / unit, cpr = rq + rope_dim / unit;
            for (int c = tid; c < kMlaTileRows * cpr; c += 32 * kMlaHeadsPerCta) {
                const int r = c / cpr, x = c - r * cpr;
                const int t = mla_row(selected, jb + r, j1, tokens);
                float *d = dst + r * W + (x < rq ? unit * x : 32 * RPL + unit * (x - rq));
                const size_t row = static_cast<size_t>(max(t, 0));
                const float *src = x < rq ? latent + row * rank + unit * x : rope + row * rope_dim + unit * (x - rq);
                if (VEC) {
                    if (t >= 0) cp_async16(d, src);
                    else *reinterpret_cast<float4 *>(d) = make_float4(0.0f, 0.0f, 0.0f, 0.0f);
                } else {
                    if (t >= 0) cp_async4(d, src);
                    else *d = 0.0f;
                }
            }
        }
        cp_async_commit();
    };
#pragma unroll
    for (int tt = 0; tt < kMlaStages - 1; ++tt) issue(tt);
    float m[HPW], l[HPW];
#pragma unroll
    for (int a = 0; a < HPW; ++a) m[a] = -INFINITY, l[a] = 0.0f;
    for (int tt = 0; tt < ntiles; ++tt) {
        cp_async_wait<kMlaStages - 2>();
        __syncthreads();  // tile tt complete for all threads; tile tt-1 no longer read
        issue(tt + kMlaStages - 1);
        const float *rows = tile + (tt % kMlaStages) * kRowsFloats;
        const int jb = j0 + tt * kMlaTileRows;
        float v[NV];  // v[8a + r]: head a . row r
#pragma unroll
        for (int r = 0; r < kMlaTileRows; ++r) {
            float d[HPW];
#pragma unroll
            for (int a = 0; a < HPW; ++a) d[a] = 0.0f;
#pragma unroll
            for (int g = 0; g < RPL / 4; ++g) {
                const float4 x = *reinterpret_cast<const float4 *>(rows + r * W + 128 * g + 4 * lane);
#pragma unroll
                for (int a = 0; a < HPW; ++a) {
                    d[a] = fmaf(q[a][4 * g], x.x, d[a]);
                    d[a] = fmaf(q[a][4 * g + 1], x.y, d[a]);
                    d[a] = fmaf(q[a][4 * g + 2], x.z, d[a]);
                    d[a] = fmaf(q[a][4 * g + 3], x.w, d[a]);
                }
            }
            if constexpr (PPL == 2) {
                const float2 x = *reinterpret_cast<const float2 *>(rows + r * W + 32 * RPL + 2 * lane);
#pragma unroll
                for (int a = 0; a < HPW; ++a) d[a] = fmaf(qr[a][1], x.y, fmaf(qr[a][0], x.x, d[a]));
            } else {
                const float4 x = *reinterpret_cast<const float4 *>(rows + r * W + 32 * RPL + 4 * lane);
#pragma unroll
                for (int a = 0; a < HPW; ++a)
                    d[a] = fmaf(qr[a][3], x.w, fmaf(qr[a][2], x.z, fmaf(qr[a][1], x.y, fmaf(qr[a][0], x.x, d[a]))));
            }
#pragma unroll
            for (int a = 0; a < HPW; ++a) v[kMlaTileRows * a + r] = d[a];
        }
        warp_sum_n(v);
        bool ok[kMlaTileRows];
#pragma unroll
        for (int r = 0; r < kMlaTileRows; ++r) ok[r] = mla_row(selected, jb + r, j1, tokens) >= 0;
        float alpha[HPW], beta[HPW][kMlaTileRows];
#pragma unroll
        for (int a = 0; a < HPW; ++a) {
            float mb = m[a];
#pragma unroll
            for (int r = 0; r < kMlaTileRows; ++r)
                if (ok[r]) mb = fmaxf(mb, v[kMlaTileRows * a + r] * scale);
            if (mb == -INFINITY) {  // nothing valid yet: no change
                alpha[a] = 1.0f;
#pragma unroll
                for (int r = 0; r < kMlaTileRows; ++r) beta[a][r] = 0.0f;
                continue;
            }
            alpha[a] = l[a] > 0.0f ? expf(m[a] - mb) : 0.0f;
            float la = l[a] * alpha[a];
#pragma unroll
            for (int r = 0; r < kMlaTileRows; ++r) {
                beta[a][r] = ok[r] ? expf(v[kMlaTileRows * a + r] * scale - mb) : 0.0f;
                la += beta[a][r];
            }
            l[a] = la;
            m[a] = mb;
        }
#pragma unroll
        for (int g = 0; g < RPL / 4; ++g) {
            float4 x[kMlaTileRows];
#pragma unroll
            for (int r = 0; r < kMlaTileRows; ++r)
                x[r] = *reinterpret_cast<const float4 *>(rows + r * W + 128 * g + 4 * lane);
#pragma unroll
            for (int a = 0; a < HPW; ++a) {
                float y0 = acc[a][4 * g] * alpha[a], y1 = acc[a][4 * g + 1] * alpha[a];
                float y2 = acc[a][4 * g + 2] * alpha[a], y3 = acc[a][4 * g + 3] * alpha[a];
#pragma unroll
                for (int r = 0; r < kMlaTileRows; ++r) {
                    y0 = fmaf(beta[a][r], x[r].x, y0);
                    y1 = fmaf(beta[a][r], x[r].y, y1);
                    y2 = fmaf(beta[a][r], x[r].z, y2);
                    y3 = fmaf(beta[a][r], x[r].w, y3);
                }
                acc[a][4 * g] = y0, acc[a][4 * g + 1] = y1, acc[a][4 * g + 2] = y2, acc[a][4 * g + 3] = y3;
            }
        }
    }
    cp_async_wait<0>();
#pragma unroll
    for (int a = 0; a < HPW; ++a) {
        if (hs[a] >= heads) continue;
        const size_t task = static_cast<size_t>(blockIdx.x) * heads + hs[a];
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
            const int d = latent_col(i, lane);
            if (d < rank) numerator[task * rank + d] = acc[a][i];
        }
        if (lane == 0) {
            stats[task * 2] = m[a];
            stats[task * 2 + 1] = l[a];
        }
    }
}

// RPL = rank columns per lane (rank <= 32*RPL), PPL = rope columns per lane.
template <int RPL, int PPL>
__global__ void __launch_bounds__(32 * kMlaHeadsPerCta)
    mla_partial_kernel(float *__restrict__ numerator, float *__restrict__ stats, const float *__restrict__ q_latent,
                       const float *__restrict__ q_rope, const float *__restrict__ latent,
                       const float *__restrict__ rope, const int32_t *__restrict__ selected, int heads, int rank,
                       int rope_dim, int tokens, int count, int stride, int splits, float scale) {
    grid_dependency_wait();
    allow_dependent_launch();
    const int lane = threadIdx.x & 31;
    const int h = blockIdx.y * kMlaHeadsPerCta + (threadIdx.x >> 5);
    const int split = blockIdx.x;
    if (h >= heads) return;  // warp-uniform
    float q[RPL], qr[PPL], acc[RPL];
#pragma unroll
    for (int i = 0; i < RPL; ++i) {
        const int d = lane + 32 * i;
        q[i] = d < rank ? q_latent[static_cast<size_t>(h) * rank + d] : 0.0f;
        acc[i] = 0.0f;
    }
#pragma unroll
    for (int i = 0; i < PPL; ++i) {
        const int d = lane + 32 * i;
        qr[i] = d < rope_dim ? q_rope[static_cast<size_t>(h) * rope_dim + d] : 0.0f;
    }
    const int per = (count + splits - 1) / splits;
    const int j0 = split * per, j1 = min(count, j0 + per);
    float m = -INFINITY, l = 0.0f;
    for (int j = j0; j < j1; j += kMlaBatch) {
        float lat[kMlaBatch][RPL], s[kMlaBatch];
        bool ok[kMlaBatch];
#pragma unroll
        for (int b = 0; b < kMlaBatch; ++b) {
            const int jj = j + b;
            int t = -1;
            if (jj < j1) t = selected ? selected[static_cast<size_t>(h) * stride + jj] : jj;
            ok[b] = t >= 0 && t < tokens;  // uniform across the warp
            float dot = 0.0f;
#pragma unroll
            for (int i = 0; i < RPL; ++i) {
                const int d = lane + 32 * i;
                lat[b][i] = ok[b] && d < rank ? latent[static_cast<size_t>(t) * rank + d] : 0.0f;
                dot = fmaf(q[i], lat[b][i], dot);
            }
#pragma unroll
            for (int i = 0; i < PPL; ++i) {
                const int d = lane + 32 * i;
                if (ok[b] && d < rope_dim) dot = fmaf(qr[i], rope[static_cast<size_t>(t) * rope_dim + d], dot);
            }
            s[b] = dot;
        }
#pragma unroll
        for (int b = 0; b < kMlaBatch; ++b) s[b] = warp_sum(s[b]) * scale;
        float mb = m;
#pragma unroll
        for (int b = 0; b < kMlaBatch; ++b)
            if (ok[b]) mb = fmaxf(mb, s[b]);
        if (mb == -INFINITY) continue;  // nothing valid yet
        const float alpha = l > 0.0f ? expf(m - mb) : 0.0f;
        float beta[kMlaBatch];
#pragma unroll
        for (int b = 0; b < kMlaBatch; ++b) beta[b] = ok[b] ? expf(s[b] - mb) : 0.0f;
        l = l * alpha;
#pragma unroll
        for (int b = 0; b < kMlaBatch; ++b) l += beta[b];
#pragma unroll
        for (int i = 0; i < RPL; ++i) {
            float v = acc[i] * alpha;
#pragma unroll
            for (int b = 0; b < kMlaBatch; ++b) v = fmaf(beta[b], lat[b][i], v);
            acc[i] = v;
        }
        m = mb;
    }
    const size_t task = static_cast<size_t>(split) * heads + h;
#pragma unroll
    for (int i = 0; i < RPL; ++i) {
        const int d = lane + 32 * i;
        if (d < rank) numerator[task * rank + d] = acc[i];
    }
    if (lane == 0) {
        stats[task * 2] = m;
        stats[task * 2 + 1] = l;
    }
}

// Grid (heads, ceil(rank / 128), queries), one warp: the lanes turn the
// splits' (max, mass) into factors e^(m_s - max) (splits with mass) and the
// denominator; then each lane adds its float4 of the 128-column block over
// the splits in split order (loads of 8 splits in flight).
__global__ void __launch_bounds__(32)
    mla_merge_kernel(float *__restrict__ out, const float *__restrict__ numerator, const float *__restrict__ stats,
                     int heads, int rank, int splits) {
    __shared__ float f[kMlaMaxSplits];
    grid_dependency_wait();
    allow_dependent_launch();
    const int h = blockIdx.x, lane = threadIdx.x;
    out += static_cast<size_t>(blockIdx.z) * heads * rank;  // query of a batch
    numerator += static_cast<size_t>(blockIdx.z) * splits * heads * rank;
    stats += static_cast<size_t>(blockIdx.z) * splits * heads * 2;
    float mx = -INFINITY;
    for (int s = lane; s < splits; s += 32) {
        const size_t task = static_cast<size_t>(s) * heads + h;
        if (stats[task * 2 + 1] > 0.0f) mx = fmaxf(mx, stats[task * 2]);
    }
    mx = warp_max(mx);
    float den = 0.0f;
    for (int s = lane; s < splits; s += 32) {
        const size_t task = static_cast<size_t>(s) * heads + h;
        const float ls = stats[task * 2 + 1];
        const float e = ls > 0.0f ? expf(stats[task * 2] - mx) : -1.0f;  // -1: no mass
        f[s] = e;
        if (ls > 0.0f) den = fmaf(ls, e, den);
    }
    den = warp_sum(den);
    __syncwarp();
    const int c = 128 * blockIdx.y + 4 * lane;
    if (c >= rank) return;
    const bool vec = (rank & 3) == 0;
    float4 acc = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
    for (int s = 0; s < splits; ++s) {
        const float fs = f[s];
        if (fs >= 0.0f) {
            const float *row = numerator + (static_cast<size_t>(s) * heads + h) * rank + c;
            float4 v;
            if (vec) {
                v = *reinterpret_cast<const float4 *>(row);
            } else {
                v.x = row[0];
                v.y = c + 1 < rank ? row[1] : 0.0f;
                v.z = c + 2 < rank ? row[2] : 0.0f;
                v.w = c + 3 < rank ? row[3] : 0.0f;
            }
            acc.x = fmaf(v.x, fs, acc.x);
            acc.y = fmaf(v.y, fs, acc.y);
            acc.z = fmaf(v.z, fs, acc.z);
            acc.w = fmaf(v.w, fs, acc.w);
        }
    }
    float *o = out + static_cast<size_t>(h) * rank + c;
    o[0] = den > 0.0f ? acc.x / den : 0.0f;
    if (c + 1 < rank) o[1] = den > 0.0f ? acc.y / den : 0.0f;
    if (c + 2 < rank) o[2] = den > 0.0f ? acc.z / den : 0.0f;
    if (c + 3 < rank) o[3] = den > 0.0f ? acc.w / den : 0.0f;
}

// Heads per CTA: two per warp in the shared-selection kernel (rank <= 512),
// one per warp in mla_partial_kernel.
int mla_shared_heads(int rank) { return kMlaHeadsPerCta * (rank <= 512 ? 2 : 1); }

// Splits: as many as keep the head groups x queries x splits CTAs within
// one wave (one CTA per SM; a partial second wave would cost a whole split's
// time), at least kMlaMinRowsPerSplit rows each, at most kMlaMaxSplits.
int mla_splits(int heads, int rank, int count, int batch = 1) {
    const int per_cta = mla_shared_heads(rank);
    const int groups = (heads + per_cta - 1) / per_cta;
    const int want = std::max(1, kMlaTargetCtas / (groups * batch));
    const int most = std::max(1, (count + kMlaMinRowsPerSplit - 1) / kMlaMinRowsPerSplit);
    return std::max(1, std::min({kMlaMaxSplits, want, most}));
}

template <int RPL, int PPL, int HPW, bool VEC>
int32_t launch_shared(dim3 grid, cudaStream_t st, float *numerator, float *stats, const float *q_latent,
                      const float *q_rope, const float *latent, const float *rope, const int32_t *selected,
                      int heads, int rank, int rope_dim, int tokens, int count, int splits, float scale,
                      const int32_t *lens, int64_t latent_stride, int64_t rope_stride, int64_t sel_stride) {
    constexpr int bytes = kMlaStages * kMlaTileRows * 32 * (RPL + PPL) * 4;
    if (const int32_t rc = allow_dynamic_smem(mla_shared_kernel<RPL, PPL, HPW, VEC>, bytes, "mla_shared smem"))
        return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = dim3(32 * kMlaHeadsPerCta);
    cfg.dynamicSmemBytes = bytes;
    cfg.stream = st;
    cudaLaunchAttribute at[1];
    at[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    at[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = at;
    cfg.numAttrs = 1;
    GLMVX_CUDA(cudaLaunchKernelEx(&cfg, mla_shared_kernel<RPL, PPL, HPW, VEC>, numerator, stats, q_latent, q_rope, latent,
                                  rope, selected, heads, rank, rope_dim, tokens, count, splits, scale, lens,
                                  latent_stride, rope_stride, sel_stride));
    return kOk;
}

// One CTA per query: copy its new rows to position lens[b] of each cache,
// then lens[b] + 1.  A full cache (lens[b] == capacity) is left as it is
// and flagged in *full.
__global__ void __launch_bounds__(256)
    dsa_append_kernel(float *latents, float *rope_keys, float *index_keys, int32_t *lens, const float *new_latent,
                      const float *new_rope, const float *new_index, int capacity, int rank, int rope_dim,
                      int index_dim, int32_t *full) {
    const int b = blockIdx.x;
    const int at = lens[b];
    __syncthreads();  // every thread has read lens[b] before it moves
    if (at < 0 || at >= capacity) {
        if (threadIdx.x == 0) atomicExch(full, 1);
        return;
    }
    const size_t row = static_cast<size_t>(b) * capacity + at;
    for (int i = threadIdx.x; i < rank; i += blockDim.x) latents[row * rank + i] = new_latent[b * rank + i];
    for (int i = threadIdx.x; i < rope_dim; i += blockDim.x) rope_keys[row * rope_dim + i] = new_rope[b * rope_dim + i];
    for (int i = threadIdx.x; i < index_dim; i += blockDim.x)
        index_keys[row * index_dim + i] = new_index[b * index_dim + i];
    if (threadIdx.x == 0) lens[b] = at + 1;
}

// The merge kernel holds one factor per split in shared memory.
int32_t check_merge_splits(int splits) {
    if (splits < 1 || splits > kMlaMaxSplits) return set_error("mla merge: %d splits (1..%d)", splits, kMlaMaxSplits), kInvalid;
    return kOk;
}

template <class K>
int32_t launch_pdl(K kern, dim3 grid, dim3 block, cudaStream_t stream, auto... args) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    GLMVX_CUDA(cudaLaunchKernelEx(&cfg, kern, args...));
    return kOk;
}

}  // namespace

}  // namespace glmvx

using namespace glmvx;

// Scratch of glmvx_mla_decode: per (split, head) the partial output row and
// its (max, mass).
GLMVX_EXPORT int64_t glmvx_mla_scratch_bytes(int32_t heads, int32_t rank, int32_t count) {
    if (heads <= 0 || rank <= 0 || count < 0) return -1;
    const int64_t splits = std::max(mla_splits(heads, rank, count), mla_tc_splits(count, 1));
    return 4 * splits * heads * (static_cast<int64_t>(rank) + 2);
}

// out[heads][rank]; q_latent [heads][rank], q_rope [heads][rope_dim], cache
// rows latent [tokens][rank] and rope [tokens][rope_dim]; selected ids
// [heads][selection_stride] (stride 0: one list for all heads; nullptr: the
// first `count` tokens).  rank <= 1024, rope_dim <= 128.
GLMVX_EXPORT int32_t glmvx_mla_decode(float *out, const float *q_latent, const float *q_rope,
                                      const float *cache_latent, const float *cache_rope, const int32_t *selected,
                                      int32_t heads, int32_t rank, int32_t rope_dim, int32_t tokens, int32_t count,
                                      int32_t selection_stride, float scale, void *scratch, uint64_t scratch_bytes,
                                      void *stream) {
    if (heads <= 0 || rank <= 0 || rank > 1024 || rope_dim < 0 || rope_dim > 128 || tokens < 0 || count < 0 ||
        selection_stride < 0 || !(scale > 0.0f) || !std::isfinite(scale)) {
        set_error("mla_decode: invalid dimensions or scale");
        return kInvalid;
    }
    if (!selected && count > tokens) {
        set_error("mla_decode: count exceeds tokens without a selection");
        return kInvalid;
    }
    const bool shared_sel = selection_stride == 0 || !selected;
    const bool tc = kMlaUseTensorCores && shared_sel && mla_tc_supported(heads, rank, rope_dim, count) &&
                    count >= kMlaTcMinRows;
    const int splits = tc ? mla_tc_splits(count, 1) : mla_splits(heads, rank, count);
    const int64_t need = glmvx_mla_scratch_bytes(heads, rank, count);
    if (!scratch || static_cast<int64_t>(scratch_bytes) < need || (reinterpret_cast<uintptr_t>(scratch) & 15)) {
        set_error("mla_decode: scratch needs %lld bytes, 16-byte aligned", static_cast<long long>(need));
        return kInvalid;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    float *numerator = static_cast<float *>(scratch);
    float *stats = numerator + static_cast<size_t>(splits) * heads * rank;
    int32_t rc;
    const int ppl = (rope_dim + 31) / 32;
    if (tc) {
        rc = launch_mla_tc(numerator, stats, q_latent, q_rope, cache_latent, cache_rope, selected, nullptr, heads, rank,
                           rope_dim, tokens, count, splits, scale, 0, 0, 0, 1, st);
    } else if (shared_sel && rank <= 512) {  // one selection for every head
        const int per_cta = mla_shared_heads(rank);
        const dim3 grid(splits, (heads + per_cta - 1) / per_cta);
        const bool vec = rank % 4 == 0 && rope_dim % 4 == 0 && (reinterpret_cast<uintptr_t>(cache_latent) & 15) == 0 &&
                         (rope_dim == 0 || (reinterpret_cast<uintptr_t>(cache_rope) & 15) == 0);
#define GLMVX_MLA_SHARED(R, P, H)                                                                                   \
    (vec ? launch_shared<R, P, H, true>(grid, st, numerator, stats, q_latent, q_rope, cache_latent, cache_rope, selected, \
                                        heads, rank, rope_dim, tokens, count, splits, scale, nullptr, 0, 0, 0)       \
         : launch_shared<R, P, H, false>(grid, st, numerator, stats, q_latent, q_rope, cache_latent, cache_rope,     \
                                         selected, heads, rank, rope_dim, tokens, count, splits, scale, nullptr, 0, 0, \
                                         0))
        rc = ppl <= 2 ? GLMVX_MLA_SHARED(16, 2, 2) : GLMVX_MLA_SHARED(16, 4, 2);
#undef GLMVX_MLA_SHARED
    } else {
        const dim3 grid(splits, (heads + kMlaHeadsPerCta - 1) / kMlaHeadsPerCta), block(32 * kMlaHeadsPerCta);
        if (rank <= 512) {
            rc = ppl <= 2 ? launch_pdl(mla_partial_kernel<16, 2>, grid, block, st, numerator, stats, q_latent, q_rope,
                                       cache_latent, cache_rope, selected, heads, rank, rope_dim, tokens, count,
                                       selection_stride, splits, scale)
                          : launch_pdl(mla_partial_kernel<16, 4>, grid, block, st, numerator, stats, q_latent, q_rope,
                                       cache_latent, cache_rope, selected, heads, rank, rope_dim, tokens, count,
                                       selection_stride, splits, scale);
        } else {
            rc = launch_pdl(mla_partial_kernel<32, 4>, grid, block, st, numerator, stats, q_latent, q_rope,
                            cache_latent, cache_rope, selected, heads, rank, rope_dim, tokens, count, selection_stride,
                            splits, scale);
        }
    }
    if (rc) return rc;
    if (const int32_t bad = check_merge_splits(splits)) return bad;
    return launch_pdl(mla_merge_kernel, dim3(heads, (rank + kMergeCols - 1) / kMergeCols), dim3(32), st, out,
                      const_cast<const float *>(numerator), const_cast<const float *>(stats), heads, rank, splits);
}

// ---- Fused DSA decode for a batch of queries over device-resident
// compressed caches (model.py:136-236 of the reference: `_index` then the
// fused branch of `_attention`): per query b
//   scores = sum_h head_weights[b][h] relu(index_scale q_index[b][h] . index_keys[b][t]), t < lens[b]
//   sel    = stable descending top-min(topk, lens[b]) of scores
//   out[b] = softmax-weighted latents over sel (the absorbed MLA above)
// Three launches after one another on `stream` (index scores, top-k, MLA
// partial + merge); lens lives on the device, so one captured graph serves
// every step as the caches grow.

// Scratch: scores [batch][capacity], selections [batch][topk], then the MLA
// partials [batch][splits][heads][rank] and their (max, mass).
GLMVX_EXPORT int64_t glmvx_dsa_scratch_bytes(int32_t batch, int32_t heads, int32_t rank, int32_t capacity,
                                             int32_t topk) {
    if (batch <= 0 || heads <= 0 || rank <= 0 || capacity <= 0 || topk <= 0) return -1;
    const int64_t splits = std::max(mla_splits(heads, rank, topk, batch), mla_tc_splits(topk, batch));
    const auto up16 = [](int64_t b) { return (b + 15) / 16 * 16; };
    return up16(4LL * batch * capacity) + up16(4LL * batch * topk) + 4LL * batch * splits * heads * (rank + 2);
}

// q_latent [batch][heads][rank], q_rope [batch][heads][rope_dim], q_index
// [batch][index_heads][index_dim], head_weights [batch][index_heads];
// caches latents [batch][capacity][rank], rope_keys [batch][capacity][rope_dim],
// index_keys [batch][capacity][index_dim]; lens (device) [batch] valid rows
// of each cache; out [batch][heads][rank]; selected_out, when given,
// [batch][topk] (-1 past min(topk, lens[b])).  rank <= 512, rope_dim <= 128,
// topk <= 4096.
namespace {

int32_t dsa_mla_stage(float *out, const int32_t *sel, const float *q_latent, const float *q_rope, const float *latents,
                      const float *rope_keys, const int32_t *lens, int32_t batch, int32_t heads, int32_t rank,
                      int32_t rope_dim, int32_t capacity, int32_t topk, float scale, float *numerator, float *stats,
                      int splits, bool tc, cudaStream_t st);

int32_t dsa_decode(float *out, int32_t *selected_out, const float *q_latent, const float *q_rope, const float *q_index,
                   const float *head_weights, const float *latents, const float *rope_keys, const float *index_keys,
                   const int32_t *lens, int32_t batch, int32_t heads, int32_t rank, int32_t rope_dim,
                   int32_t index_heads, int32_t index_dim, int32_t capacity, int32_t topk, float index_scale,
                   float scale, void *scratch, uint64_t scratch_bytes, cudaEvent_t attention_inputs_ready,
                   void *stream) {
    if (batch <= 0 || heads <= 0 || rank <= 0 || rank > 512 || rope_dim < 0 || rope_dim > 128 || index_heads <= 0 ||
        index_dim <= 0 || capacity <= 0 || topk <= 0 || topk > 4096 || !(scale > 0.0f) || !std::isfinite(scale) ||
        !std::isfinite(index_scale)) {
        set_error("dsa_decode: invalid dimensions or scale");
        return kInvalid;
    }
    if (!out || !q_latent || !q_index || !head_weights || !latents || !index_keys || !lens ||
        (rope_dim && (!q_rope || !rope_keys))) {
        set_error("dsa_decode: null pointer");
        return kInvalid;
    }
    const int64_t need = glmvx_dsa_scratch_bytes(batch, heads, rank, capacity, topk);
    if (!scratch || static_cast<int64_t>(scratch_bytes) < need || (reinterpret_cast<uintptr_t>(scratch) & 15)) {
        set_error("dsa_decode: scratch needs %lld bytes, 16-byte aligned", static_cast<long long>(need));
        return kInvalid;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    const auto up16 = [](int64_t b) { return (b + 15) / 16 * 16; };
    char *base = static_cast<char *>(scratch);
    float *scores = reinterpret_cast<float *>(base);
    int32_t *sel = reinterpret_cast<int32_t *>(base + up16(4LL * batch * capacity));
    float *numerator = reinterpret_cast<float *>(base + up16(4LL * batch * capacity) + up16(4LL * batch * topk));
    const bool tc = kMlaUseTensorCores && mla_tc_supported(heads, rank, rope_dim, topk) &&
                    static_cast<int64_t>(batch) * topk >= kMlaTcMinRows;
    const int splits = tc ? mla_tc_splits(topk, batch) : mla_splits(heads, rank, topk, batch);
    float *stats = numerator + static_cast<size_t>(batch) * splits * heads * rank;
    if (selected_out) sel = selected_out;
    int32_t rc = launch_index_scores_batch(scores, q_index, index_keys, head_weights, capacity, index_heads, index_dim,
                                           index_scale, lens, static_cast<int64_t>(capacity) * index_dim, capacity,
                                           batch, st);
    if (rc) return rc;
    rc = launch_topk_batch(sel, scores, capacity, topk, lens, capacity, topk, batch, st);
    if (rc) return rc;
    if (attention_inputs_ready) GLMVX_CUDA(cudaStreamWaitEvent(st, attention_inputs_ready, 0));
    return dsa_mla_stage(out, sel, q_latent, q_rope, latents, rope_keys, lens, batch, heads, rank, rope_dim, capacity,
                         topk, scale, numerator, stats, splits, tc, st);
}

// The attention stage of the DSA decode: absorbed MLA of every query over its
// selection sel [batch][topk] (ids outside [0, lens[b]) skipped), split
// partials into numerator/stats, then the ordered merge into out.
int32_t dsa_mla_stage(float *out, const int32_t *sel, const float *q_latent, const float *q_rope, const float *latents,
                      const float *rope_keys, const int32_t *lens, int32_t batch, int32_t heads, int32_t rank,
                      int32_t rope_dim, int32_t capacity, int32_t topk, float scale, float *numerator, float *stats,
                      int splits, bool tc, cudaStream_t st) {
    int32_t rc = kOk;
    const int64_t lstride = static_cast<int64_t>(capacity) * rank, rstride = static_cast<int64_t>(capacity) * rope_dim;
    if (tc) {
        rc = launch_mla_tc(numerator, stats, q_latent, q_rope, latents, rope_keys, sel, lens, heads, rank, rope_dim,
                           capacity, topk, splits, scale, lstride, rstride, topk, batch, st);
        if (rc) return rc;
        if (const int32_t bad = check_merge_splits(splits)) return bad;
        return launch_pdl(mla_merge_kernel, dim3(heads, (rank + kMergeCols - 1) / kMergeCols, batch), dim3(32), st, out,
                          const_cast<const float *>(numerator), const_cast<const float *>(stats), heads, rank, splits);
    }
    const int per_cta = mla_shared_heads(rank);
    const dim3 grid(splits, (heads + per_cta - 1) / per_cta, batch);
    const bool vec = rank % 4 == 0 && rope_dim % 4 == 0 && (reinterpret_cast<uintptr_t>(latents) & 15) == 0 &&
                     (rope_dim == 0 || (reinterpret_cast<uintptr_t>(rope_keys) & 15) == 0);
    const int ppl = (rope_dim + 31) / 32;
#define GLMVX_DSA_SHARED(P)                                                                                       \
    (vec ? launch_shared<16, P, 2, true>(grid, st, numerator, stats, q_latent, q_rope, latents, rope_keys, sel, heads, \
                                         rank, rope_dim, capacity, topk, splits, scale, lens, lstride, rstride, topk) \
         : launch_shared<16, P, 2, false>(grid, st, numerator, stats, q_latent, q_rope, latents, rope_keys, sel,      \
                                          heads, rank, rope_dim, capacity, topk, splits, scale, lens, lstride, rstride, \
                                          topk))
    rc = ppl <= 2 ? GLMVX_DSA_SHARED(2) : GLMVX_DSA_SHARED(4);
#undef GLMVX_DSA_SHARED
    if (rc) return rc;
    if (const int32_t bad = check_merge_splits(splits)) return bad;
    return launch_pdl(mla_merge_kernel, dim3(heads, (rank + kMergeCols - 1) / kMergeCols, batch), dim3(32), st, out,
                      const_cast<const float *>(numerator), const_cast<const float *>(stats), heads, rank, splits);
}

}  // namespace

GLMVX_EXPORT int32_t glmvx_dsa_decode(float *out, int32_t *selected_out, const float *q_latent, const float *q_rope,
                                      const float *q_index, const float *head_weights, const float *latents,
                                      const float *rope_keys, const float *index_keys, const int32_t *lens,
                                      int32_t batch, int32_t heads, int32_t rank, int32_t rope_dim,
                                      int32_t index_heads, int32_t index_dim, int32_t capacity, int32_t topk,
                                      float index_scale, float scale, void *scratch, uint64_t scratch_bytes,
                                      void *stream) {
    return dsa_decode(out, selected_out, q_latent, q_rope, q_index, head_weights, latents, rope_keys, index_keys, lens,
                      batch, heads, rank, rope_dim, index_heads, index_dim, capacity, topk, index_scale, scale, scratch,
                      scratch_bytes, nullptr, stream);
}

// glmvx_dsa_decode whose attention stage (the first reader of q_latent and
// q_rope) waits for `attention_inputs_ready` (a cudaEvent_t recorded after
// the queries' copy, e.g. on a second stream): the indexer and top-k run
// while those copies are still in flight.  On every failure the stream still
// waits for the event before the status is returned, so a stream capture
// that forked the copy stays joined and ends with the original error.
GLMVX_EXPORT int32_t glmvx_dsa_decode_wait(float *out, int32_t *selected_out, const float *q_latent,
                                           const float *q_rope, const float *q_index, const float *head_weights,
                                           const float *latents, const float *rope_keys, const float *index_keys,
                                           const int32_t *lens, int32_t batch, int32_t heads, int32_t rank,
                                           int32_t rope_dim, int32_t index_heads, int32_t index_dim, int32_t capacity,
                                           int32_t topk, float index_scale, float scale, void *scratch,
                                           uint64_t scratch_bytes, void *attention_inputs_ready, void *stream) {
    const cudaEvent_t ready = static_cast<cudaEvent_t>(attention_inputs_ready);
    const int32_t rc = dsa_decode(out, selected_out, q_latent, q_rope, q_index, head_weights, latents, rope_keys,
                                  index_keys, lens, batch, heads, rank, rope_dim, index_heads, index_dim, capacity,
                                  topk, index_scale, scale, scratch, scratch_bytes, ready, stream);
    if (rc && ready) cudaStreamWaitEvent(static_cast<cudaStream_t>(stream), ready, 0);  // a second wait is harmless
    return rc;
}

// The attention stage of glmvx_dsa_decode alone, over selections given by
// the caller (a DSA layer that reuses the previous layer's top-k,
// glm_vx/model.py:197-204): selected [batch][topk], -1 padded; each query
// attends to its ids in [0, lens[b]).  Scratch as glmvx_dsa_scratch_bytes.
GLMVX_EXPORT int32_t glmvx_dsa_attend(float *out, const int32_t *selected, const float *q_latent, const float *q_rope,
                                      const float *latents, const float *rope_keys, const int32_t *lens, int32_t batch,
                                      int32_t heads, int32_t rank, int32_t rope_dim, int32_t capacity, int32_t topk,
                                      float scale, void *scratch, uint64_t scratch_bytes, void *stream) {
    if (batch <= 0 || heads <= 0 || rank <= 0 || rank > 512 || rope_dim < 0 || rope_dim > 128 || capacity <= 0 ||
        topk <= 0 || topk > 4096 || !(scale > 0.0f) || !std::isfinite(scale)) {
        set_error("dsa_attend: invalid dimensions or scale");
        return kInvalid;
    }
    if (!out || !selected || !q_latent || !latents || !lens || (rope_dim && (!q_rope || !rope_keys))) {
        set_error("dsa_attend: null pointer");
        return kInvalid;
    }
    const int64_t need = glmvx_dsa_scratch_bytes(batch, heads, rank, capacity, topk);
    if (!scratch || static_cast<int64_t>(scratch_bytes) < need || (reinterpret_cast<uintptr_t>(scratch) & 15)) {
        set_error("dsa_attend: scratch needs %lld bytes, 16-byte aligned", static_cast<long long>(need));
        return kInvalid;
    }
    const auto up16 = [](int64_t b) { return (b + 15) / 16 * 16; };
    float *numerator = reinterpret_cast<float *>(static_cast<char *>(scratch) + up16(4LL * batch * capacity) +
                                                 up16(4LL * batch * topk));
    const bool tc = kMlaUseTensorCores && mla_tc_supported(heads, rank, rope_dim, topk) &&
                    static_cast<int64_t>(batch) * topk >= kMlaTcMinRows;
    const int splits = tc ? mla_tc_splits(topk, batch) : mla_splits(heads, rank, topk, batch);
    float *stats = numerator + static_cast<size_t>(batch) * splits * heads * rank;
    return dsa_mla_stage(out, selected, q_latent, q_rope, latents, rope_keys, lens, batch, heads, rank, rope_dim,
                         capacity, topk, scale, numerator, stats, splits, tc, static_cast<cudaStream_t>(stream));
}

// Appends one row per query to the caches of glmvx_dsa_decode (device
// pointers; new rows [batch][dim]); *full (device int32) is set to 1 for a
// query whose cache already holds `capacity` rows, which is then unchanged.
GLMVX_EXPORT int32_t glmvx_dsa_append(float *latents, float *rope_keys, float *index_keys, int32_t *lens,
                                      const float *new_latent, const float *new_rope, const float *new_index,
                                      int32_t batch, int32_t capacity, int32_t rank, int32_t rope_dim,
                                      int32_t index_dim, int32_t *full, void *stream) {
    if (batch < 0 || capacity <= 0 || rank <= 0 || rope_dim < 0 || index_dim < 0 || !lens || !full ||
        (index_dim && (!index_keys || !new_index))) {
        set_error("dsa_append: invalid arguments");
        return kInvalid;
    }
    if (batch == 0) return kOk;
    dsa_append_kernel<<<batch, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        latents, rope_keys, index_keys, lens, new_latent, new_rope, new_index, capacity, rank, rope_dim, index_dim, full);
    GLMVX_CUDA(cudaGetLastError());
    return kOk;
}
