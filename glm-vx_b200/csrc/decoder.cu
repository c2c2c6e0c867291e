// Batched decode-step pieces of the GLM-MoE-DSA model that sit between the
// packed projections, the DSA attention and the MoE layer: one token per
// sequence, B sequences per launch (glm_vx/model.py:359-392 for one token,
// here for a batch at per-sequence positions, all on the device so a decode
// step is one replayable graph).
//
//   embed_rows      x[b] = row ids[b] of the embedding table (F32, or Q8_0
//                   decoded exactly: fp16 d times int8 q), model.py:96-104
//   rope_rows       the reference's rope (kernels/kernels.vx:425-441: pairs
//                   (x[2p], x[2p+1]) rotated, output half-split) on strided
//                   rows at each sequence's position, with the cos/sin taken
//                   from a host-built table (the reference's float32
//                   coefficients, kernels/backend.py:32-39), plus a copied tail
//   rmsnorm_rows    rmsnorm on strided rows (kernels/kernels.vx:17-27)
//   absorb_query    q_latent[b,h] = kv_b[h, :nope]^T . query[b,h,:nope]
//                   (model.py:210-213), a serial f32 sum over nope
//   absorb_value    out[b,h] = kv_b[h, nope:] . attended[b,h] (model.py:219),
//                   a serial f32 sum over rank
//   scale_rows      out = x * s (model.py:159, the indexer head weights)
//   argmax_rows     first index of the row maximum (generate.py:96)
// The serial sums use separate f32 products and adds in the reference's
// order, as its C matvec does.
#include <algorithm>

#include <cuda_fp16.h>

#include "codecs.cuh"

namespace glmvx {

namespace {

constexpr int kDecThreads = 256;
// Loads a thread issues before it consumes any of them: a strided row loop
// written plainly waits out one memory latency per element.
constexpr int kRowBatch = 8;

__global__ void embed_rows_kernel(float *out, const uint8_t *table, int kind, const int32_t *ids, int vocab,
                                  int hidden, int *err) {
    const int b = blockIdx.x;
    int id = ids[b];
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) report_device_error(err, kDevErrBadIndex);
        id = min(max(id, 0), vocab - 1);
    }
    float *o = out + static_cast<size_t>(b) * hidden;
    const int step = blockDim.x;
    if (kind == 0) {
        const float *row = reinterpret_cast<const float *>(table) + static_cast<size_t>(id) * hidden;
        int i = threadIdx.x;
        for (; i + (kRowBatch - 1) * step < hidden; i += kRowBatch * step) {
            float v[kRowBatch];
#pragma unroll
            for (int u = 0; u < kRowBatch; ++u) v[u] = row[i + u * step];
#pragma unroll
            for (int u = 0; u < kRowBatch; ++u) o[i + u * step] = v[u];
        }
        for (; i < hidden; i += step) o[i] = row[i];
        return;
    }
    const uint8_t *row = table + static_cast<size_t>(id) * (hidden / 32) * 34;  // Q8_0
    auto elem = [&](int i) {
        const uint8_t *blk = row + (i / 32) * 34;
        return h2f(u16(blk)) * static_cast<float>(static_cast<int8_t>(blk[2 + i % 32]));
    };
    int i = threadIdx.x;
    for (; i + (kRowBatch - 1) * step < hidden; i += kRowBatch * step) {
        float v[kRowBatch];
#pragma unroll
        for (int u = 0; u < kRowBatch; ++u) v[u] = elem(i + u * step);
#pragma unroll
        for (int u = 0; u < kRowBatch; ++u) o[i + u * step] = v[u];
    }
    for (; i < hidden; i += step) o[i] = elem(i);
}

struct RopeRows {
    const float *x;
    float *out;
    int64_t x_tok, out_tok;  // strides between sequences (floats)
    int x_head, out_head;    // strides between the rows of one sequence
    int x_off, out_off;      // first element of a row
    int heads, d, tail;      // rows per sequence, rotated width, copied tail
};

__global__ void rope_rows_kernel(RopeRows r, const float *cos_tab, const float *sin_tab, const int32_t *pos,
                                 int max_pos, int *err) {
    const int b = blockIdx.y;
    int p = pos[b];
    if (p < 0 || p >= max_pos) {
        if (threadIdx.x == 0 && blockIdx.x == 0) report_device_error(err, kDevErrBadIndex);
        p = min(max(p, 0), max_pos - 1);
    }
    const int half = r.d / 2, width = half + r.tail;
    const float *cs = cos_tab + static_cast<size_t>(p) * half, *sn = sin_tab + static_cast<size_t>(p) * half;
    const int total = r.heads * width;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < total; i += gridDim.x * blockDim.x) {
        const int h = i / width, k = i % width;
        const float *xi = r.x + b * r.x_tok + static_cast<int64_t>(h) * r.x_head + r.x_off;
        float *oi = r.out + b * r.out_tok + static_cast<int64_t>(h) * r.out_head + r.out_off;
        if (k < half) {
            const float a = xi[2 * k], c = xi[2 * k + 1];
            oi[k] = __fsub_rn(__fmul_rn(a, cs[k]), __fmul_rn(c, sn[k]));
            oi[half + k] = __fadd_rn(__fmul_rn(c, cs[k]), __fmul_rn(a, sn[k]));
        } else {
            const int j = r.d + (k - half);
            oi[j] = xi[j];
        }
    }
}

__global__ void rmsnorm_rows_kernel(float *out, const float *x, const float *w, int n, int64_t x_stride,
                                    int64_t out_stride, float eps) {
    __shared__ float partial[kDecThreads / 32];
    const float *xr = x + blockIdx.x * x_stride;
    float *orow = out + blockIdx.x * out_stride;
    const int step = blockDim.x;
    float ss = 0.0f;
    int i = threadIdx.x;
    for (; i + (kRowBatch - 1) * step < n; i += kRowBatch * step) {  // same order as one element at a time
        float v[kRowBatch];
#pragma unroll
        for (int u = 0; u < kRowBatch; ++u) v[u] = xr[i + u * step];
#pragma unroll
        for (int u = 0; u < kRowBatch; ++u) ss = fmaf(v[u], v[u], ss);
    }
    for (; i < n; i += step) ss = fmaf(xr[i], xr[i], ss);
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) partial[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.0f;
    for (int k = 0; k < kDecThreads / 32; ++k) tot += partial[k];
    const float inv = 1.0f / sqrtf(tot / static_cast<float>(n) + eps);
    i = threadIdx.x;
    for (; i + (kRowBatch - 1) * step < n; i += kRowBatch * step) {
        float v[kRowBatch], g[kRowBatch];
#pragma unroll
        for (int u = 0; u < kRowBatch; ++u) {
            v[u] = xr[i + u * step];
            g[u] = w[i + u * step];
        }
#pragma unroll
        for (int u = 0; u < kRowBatch; ++u) orow[i + u * step] = __fmul_rn(__fmul_rn(v[u], inv), g[u]);
    }
    for (; i < n; i += step) orow[i] = __fmul_rn(__fmul_rn(xr[i], inv), w[i]);
}

// q_latent[b][h][r] = sum_j kv_b[h][j][r] * query[b][h][j], j < nope, serial
// in j.  A thread owns one r of one head for KT sequences (the weight read
// once for all of them); it loads U weights of its column before it adds
// any, so the loads of a column overlap while the sum keeps its order.
// Grid: (rank / kAbsorbThreads, heads, sequence groups of KT).
constexpr int kAbsorbThreads = 128, kAbsorbTok = 8;

// v[u] = p[u * stride] for u < U, all U loads issued before any is used: the
// loads are volatile PTX in program order, and the empty statements that
// read and rewrite the values keep every use behind the last load.
template <int U>
__device__ __forceinline__ void load_column(float (&v)[U], const float *p, size_t stride) {
    static_assert(U % 8 == 0, "loads in groups of eight");
#pragma unroll
    for (int u = 0; u < U; ++u) asm volatile("ld.global.nc.f32 %0, [%1];" : "=f"(v[u]) : "l"(p + u * stride));
#pragma unroll
    for (int u = 0; u < U; u += 8)
        asm volatile("" : "+f"(v[u]), "+f"(v[u + 1]), "+f"(v[u + 2]), "+f"(v[u + 3]), "+f"(v[u + 4]), "+f"(v[u + 5]),
                     "+f"(v[u + 6]), "+f"(v[u + 7]));
}

template <int KT, int U>
__global__ void __launch_bounds__(kAbsorbThreads)
    absorb_query_kernel(float *q_latent, const float *query, const float *kvb, int tokens, int heads, int nope,
                        int qk_head, int rank, int vdim) {
    extern __shared__ float qs[];  // [KT][nope]
    const int h = blockIdx.y, b0 = blockIdx.z * KT;
    const int nb = min(KT, tokens - b0);
    for (int i = threadIdx.x; i < KT * nope; i += blockDim.x) {
        const int tb = i / nope, j = i % nope;
        qs[i] = tb < nb ? query[(static_cast<size_t>(b0 + tb) * heads + h) * qk_head + j] : 0.0f;
    }
    __syncthreads();
    const int r = blockIdx.x * blockDim.x + threadIdx.x;
    if (r >= rank) return;
    const float *w = kvb + static_cast<size_t>(h) * (nope + vdim) * rank + r;
    float acc[KT];
#pragma unroll
    for (int tb = 0; tb < KT; ++tb) acc[tb] = 0.0f;
    int j = 0;
    for (; j + U <= nope; j += U) {
        float wv[U];
        load_column(wv, w + static_cast<size_t>(j) * rank, rank);
#pragma unroll
        for (int u = 0; u < U; ++u)
#pragma unroll
            for (int tb = 0; tb < KT; ++tb) acc[tb] = __fadd_rn(acc[tb], __fmul_rn(wv[u], qs[tb * nope + j + u]));
    }
    for (; j < nope; ++j) {
        const float wv = __ldg(w + static_cast<size_t>(j) * rank);
#pragma unroll
        for (int tb = 0; tb < KT; ++tb) acc[tb] = __fadd_rn(acc[tb], __fmul_rn(wv, qs[tb * nope + j]));
    }
#pragma unroll
    for (int tb = 0; tb < KT; ++tb)
        if (tb < nb) q_latent[(static_cast<size_t>(b0 + tb) * heads + h) * rank + r] = acc[tb];
}

// out[b][h*vdim + i] = sum_r kv_b[h][nope + i][r] * att[b][h][r], serial in
// r.  A thread owns output column i of one head for KT sequences and reads
// its contiguous kv_b row as float4s, U4 of them (4*U4 weights) issued
// before any is added.  Grid: (vdim / kAbsorbThreads, heads, groups of KT).
template <int KT, int U4>
__global__ void __launch_bounds__(kAbsorbThreads)
    absorb_value_kernel(float *out, const float *att, const float *kvb, int tokens, int heads, int nope, int rank,
                        int vdim) {
    extern __shared__ float as[];  // [KT][rank]
    const int h = blockIdx.y, b0 = blockIdx.z * KT;
    const int nb = min(KT, tokens - b0);
    for (int i = threadIdx.x; i < KT * rank; i += blockDim.x) {
        const int tb = i / rank, r = i % rank;
        as[i] = tb < nb ? att[(static_cast<size_t>(b0 + tb) * heads + h) * rank + r] : 0.0f;
    }
    __syncthreads();
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i >= vdim) return;
    const float *w = kvb + (static_cast<size_t>(h) * (nope + vdim) + nope + i) * rank;
    float acc[KT];
#pragma unroll
    for (int tb = 0; tb < KT; ++tb) acc[tb] = 0.0f;
    auto add = [&](float wv, int r) {
#pragma unroll
        for (int tb = 0; tb < KT; ++tb) acc[tb] = __fadd_rn(acc[tb], __fmul_rn(wv, as[tb * rank + r]));
    };
    int r = 0;
    if ((rank & 3) == 0) {  // rows start 16-byte aligned
        const float4 *w4 = reinterpret_cast<const float4 *>(w);
        for (; r + 4 * U4 <= rank; r += 4 * U4) {
            float4 v[U4];
#pragma unroll
            for (int u = 0; u < U4; ++u) v[u] = __ldg(w4 + r / 4 + u);
#pragma unroll
            for (int u = 0; u < U4; ++u) {
                add(v[u].x, r + 4 * u);
                add(v[u].y, r + 4 * u + 1);
                add(v[u].z, r + 4 * u + 2);
                add(v[u].w, r + 4 * u + 3);
            }
        }
    }
    for (; r < rank; ++r) add(__ldg(w + r), r);
#pragma unroll
    for (int tb = 0; tb < KT; ++tb)
        if (tb < nb) out[static_cast<size_t>(b0 + tb) * heads * vdim + h * vdim + i] = acc[tb];
}

__global__ void scale_kernel(float *out, const float *x, float s, int64_t n) {
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x)
        out[i] = __fmul_rn(x[i], s);
}

// One CTA per row: the largest value, ties to the smallest index; a NaN
// anywhere makes its first index the answer (numpy argmax).  Each thread
// scans its indices in increasing order, kRowBatch loads at a time.
constexpr int kArgmaxThreads = 1024;

// (v, j) replaces (best, bi) under the rule above.
__device__ __forceinline__ bool argmax_takes(float v, int j, float best, int bi) {
    const bool vn = v != v, bn = best != best;
    return (vn && !bn) || (vn == bn && (vn ? j < bi : (v > best || (v == best && j < bi))));
}

__global__ void __launch_bounds__(kArgmaxThreads) argmax_rows_kernel(int32_t *ids, const float *logits, int n) {
    __shared__ float sv[kArgmaxThreads / 32];
    __shared__ int si[kArgmaxThreads / 32];
    const float *row = logits + static_cast<size_t>(blockIdx.x) * n;
    const int step = blockDim.x;
    float best = -INFINITY;
    int bi = n;
    auto scan = [&](float v, int i) {
        const bool nan = v != v, bnan = best != best;
        if ((nan && !bnan) || (!bnan && v > best)) {  // strictly better, or the first NaN
            best = v;
            bi = i;
        }
    };
    int i = threadIdx.x;
    for (; i + (kRowBatch - 1) * step < n; i += kRowBatch * step) {
        float v[kRowBatch];
#pragma unroll
        for (int u = 0; u < kRowBatch; ++u) v[u] = row[i + u * step];
#pragma unroll
        for (int u = 0; u < kRowBatch; ++u) scan(v[u], i + u * step);
    }
    for (; i < n; i += step) scan(row[i], i);
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) {
        const float v = __shfl_xor_sync(0xffffffffu, best, o);
        const int j = __shfl_xor_sync(0xffffffffu, bi, o);
        if (argmax_takes(v, j, best, bi)) {
            best = v;
            bi = j;
        }
    }
    if ((threadIdx.x & 31) == 0) {
        sv[threadIdx.x >> 5] = best;
        si[threadIdx.x >> 5] = bi;
    }
    __syncthreads();
    if (threadIdx.x == 0) {
        for (int w = 1; w < static_cast<int>(blockDim.x) / 32; ++w) {
            if (argmax_takes(sv[w], si[w], best, bi)) {
                best = sv[w];
                bi = si[w];
            }
        }
        ids[blockIdx.x] = bi < n ? bi : 0;
    }
}

// SplitMix64's finaliser over (seed, counter): a stateless random stream.
__device__ __forceinline__ uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ull;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebull;
    return z ^ (z >> 31);
}

// N(0,1) by Box-Muller from the 64-bit hash of (seed, i).
__device__ __forceinline__ float normal_at(uint64_t seed, uint64_t i) {
    const uint64_t h = mix64(seed * 0x9e3779b97f4a7c15ull + i + 1);
    const float u1 = (static_cast<float>(h >> 40) + 0.5f) * (1.0f / 16777216.0f);
    const float u2 = static_cast<float>((h >> 16) & 0xffffffu) * (1.0f / 16777216.0f);
    return sqrtf(-2.0f * logf(u1)) * cosf(6.2831853f * u2);
}

// kind 0: `count` floats, N(0,1)*scale (ones: 1.0).  Packed kinds: `count`
// GGML blocks of random bytes whose fp16 scale fields (Q8_0, IQ1_S: d; Q4_K:
// d and dmin) are |N(0,1)|*scale.
__global__ void fill_random_kernel(uint8_t *out, int kind, int block_bytes, int scale_bytes, int64_t count,
                                   uint64_t seed, float scale, int ones) {
    const int64_t stride = static_cast<int64_t>(gridDim.x) * blockDim.x;
    if (kind == 0) {
        float *o = reinterpret_cast<float *>(out);
        for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < count; i += stride)
            o[i] = ones ? 1.0f : normal_at(seed, i) * scale;
        return;
    }
    const int64_t bytes = count * block_bytes;
    for (int64_t i = blockIdx.x * static_cast<int64_t>(blockDim.x) + threadIdx.x; i < bytes; i += stride) {
        const int64_t blk = i / block_bytes;
        const int j = static_cast<int>(i - blk * block_bytes);
        uint8_t v;
        if (j < scale_bytes) {  // byte j of the block's fp16 scale field(s)
            const uint16_t hbits =
                __half_as_ushort(__float2half_rn(fabsf(normal_at(seed ^ 0x5851f42d4c957f2dull, 2 * blk + j / 2)) * scale));
            v = static_cast<uint8_t>((j & 1) ? hbits >> 8 : hbits & 0xff);
        } else {
            v = static_cast<uint8_t>(mix64(seed + 0x632be59bd9b4e019ull * (i + 1)) >> 24);
        }
        out[i] = v;
    }
}

int ew_blocks(int64_t n) { return static_cast<int>(std::min<int64_t>((n + kDecThreads - 1) / kDecThreads, 8 * 148)); }

}  // namespace

}  // namespace glmvx

using namespace glmvx;

// x[b] = embedding row ids[b] (device ids) of `table` (kind 0: f32
// [vocab][hidden]; kind 8: Q8_0 [vocab][hidden/32 blocks]); an id outside
// [0, vocab) sets the device error word (the row is clamped).
GLMVX_EXPORT int32_t glmvx_embed_rows(float *out, const void *table, int32_t kind, const int32_t *ids, int32_t rows,
                                      int32_t vocab, int32_t hidden, void *stream) {
    if (rows < 0 || vocab <= 0 || hidden <= 0 || (kind != 0 && kind != 8) || (kind == 8 && hidden % 32))
        return set_error("embed_rows: F32 or Q8_0 table, positive sizes"), kInvalid;
    if (!rows) return kOk;
    embed_rows_kernel<<<rows, kDecThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        out, static_cast<const uint8_t *>(table), kind, ids, vocab, hidden, device_error_word());
    return launch_status("embed_rows_kernel");
}

// Rotates `d` elements of `heads` rows per sequence (row h of sequence b at
// x + b*x_tok + h*x_head + x_off) into the same layout of `out`, at position
// pos[b] (device) of the tables cos/sin [max_pos][d/2], and copies the `tail`
// elements after them.  out must not overlap x.
GLMVX_EXPORT int32_t glmvx_rope_rows(float *out, const float *x, const float *cos_tab, const float *sin_tab,
                                     const int32_t *pos, int32_t tokens, int32_t heads, int32_t d, int32_t tail,
                                     int64_t x_tok, int32_t x_head, int32_t x_off, int64_t out_tok, int32_t out_head,
                                     int32_t out_off, int32_t max_pos, void *stream) {
    if (tokens < 0 || heads <= 0 || d <= 0 || d % 2 || tail < 0 || max_pos <= 0)
        return set_error("rope_rows: invalid dimensions"), kInvalid;
    if (!tokens) return kOk;
    const RopeRows r{x, out, x_tok, out_tok, x_head, out_head, x_off, out_off, heads, d, tail};
    const int work = heads * (d / 2 + tail);
    const dim3 grid(std::max(1, std::min((work + kDecThreads - 1) / kDecThreads, 64)), tokens);
    rope_rows_kernel<<<grid, kDecThreads, 0, static_cast<cudaStream_t>(stream)>>>(r, cos_tab, sin_tab, pos, max_pos,
                                                                                  device_error_word());
    return launch_status("rope_rows_kernel");
}

GLMVX_EXPORT int32_t glmvx_rmsnorm_rows(float *out, const float *x, const float *w, int32_t rows, int32_t n,
                                        int64_t x_stride, int64_t out_stride, float eps, void *stream) {
    if (rows < 0 || n <= 0 || x_stride < n || out_stride < n || !(eps > 0.0f))
        return set_error("rmsnorm_rows: invalid arguments"), kInvalid;
    if (!rows) return kOk;
    rmsnorm_rows_kernel<<<rows, kDecThreads, 0, static_cast<cudaStream_t>(stream)>>>(out, x, w, n, x_stride,
                                                                                     out_stride, eps);
    return launch_status("rmsnorm_rows_kernel");
}

// query [tokens][heads][qk_head] (the first `nope` of each head used), kvb
// [heads][nope + vdim][rank] -> q_latent [tokens][heads][rank].
GLMVX_EXPORT int32_t glmvx_absorb_query(float *q_latent, const float *query, const float *kvb, int32_t tokens,
                                        int32_t heads, int32_t nope, int32_t qk_head, int32_t rank, int32_t vdim,
                                        void *stream) {
    if (tokens < 0 || heads <= 0 || heads > 65535 || nope <= 0 || qk_head < nope || rank <= 0 || vdim < 0 ||
        nope * kAbsorbTok * 4 > 48 * 1024)
        return set_error("absorb_query: invalid dimensions"), kInvalid;
    if (!tokens) return kOk;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned cols = (rank + kAbsorbThreads - 1) / kAbsorbThreads;
    if (tokens == 1) {
        absorb_query_kernel<1, 64><<<dim3(cols, heads, 1), kAbsorbThreads, nope * 4, st>>>(q_latent, query, kvb,
                                                                                          tokens, heads, nope,
                                                                                          qk_head, rank, vdim);
    } else {
        const dim3 grid(cols, heads, (tokens + kAbsorbTok - 1) / kAbsorbTok);
        absorb_query_kernel<kAbsorbTok, 16><<<grid, kAbsorbThreads, kAbsorbTok * nope * 4, st>>>(
            q_latent, query, kvb, tokens, heads, nope, qk_head, rank, vdim);
    }
    return launch_status("absorb_query_kernel");
}

// att [tokens][heads][rank], kvb [heads][nope + vdim][rank] -> out [tokens][heads * vdim].
GLMVX_EXPORT int32_t glmvx_absorb_value(float *out, const float *att, const float *kvb, int32_t tokens, int32_t heads,
                                        int32_t nope, int32_t rank, int32_t vdim, void *stream) {
    if (tokens < 0 || heads <= 0 || heads > 65535 || nope < 0 || rank <= 0 || vdim <= 0 ||
        rank * kAbsorbTok * 4 > 48 * 1024)
        return set_error("absorb_value: invalid dimensions"), kInvalid;
    if (!tokens) return kOk;
    const cudaStream_t st = static_cast<cudaStream_t>(stream);
    const unsigned cols = (vdim + kAbsorbThreads - 1) / kAbsorbThreads;
    if (tokens == 1) {
        absorb_value_kernel<1, 8><<<dim3(cols, heads, 1), kAbsorbThreads, rank * 4, st>>>(out, att, kvb, tokens, heads,
                                                                                         nope, rank, vdim);
    } else {
        const dim3 grid(cols, heads, (tokens + kAbsorbTok - 1) / kAbsorbTok);
        absorb_value_kernel<kAbsorbTok, 4><<<grid, kAbsorbThreads, kAbsorbTok * rank * 4, st>>>(
            out, att, kvb, tokens, heads, nope, rank, vdim);
    }
    return launch_status("absorb_value_kernel");
}

GLMVX_EXPORT int32_t glmvx_scale(float *out, const float *x, float s, int64_t n, void *stream) {
    if (n < 0) return set_error("scale: negative size"), kInvalid;
    if (!n) return kOk;
    scale_kernel<<<ew_blocks(n), kDecThreads, 0, static_cast<cudaStream_t>(stream)>>>(out, x, s, n);
    return launch_status("scale_kernel");
}

// Synthetic weights on the device (no reference counterpart: the reference
// draws test weights with NumPy on the host, glm_vx/model.py:415-490).
// kind 0: `count` f32 values N(0,1)*scale (ones != 0: all 1.0); kind 8 / 12
// / 19: `count` Q8_0 / Q4_K / IQ1_S blocks of random bytes with fp16 block
// scales |N(0,1)|*scale (Q4_K: d and dmin).  Deterministic in `seed`.
GLMVX_EXPORT int32_t glmvx_fill_random(void *out, int32_t kind, int64_t count, uint64_t seed, float scale,
                                       int32_t ones, void *stream) {
    int bytes = 4, scale_bytes = 0;  // per element (kind 0) or per block
    if (kind == 8) bytes = 34, scale_bytes = 2;
    else if (kind == 12) bytes = 144, scale_bytes = 4;
    else if (kind == 19) bytes = 50, scale_bytes = 2;
    else if (kind != 0) return set_error("fill_random: kind 0, 8, 12 or 19"), kInvalid;
    if (count < 0) return set_error("fill_random: negative count"), kInvalid;
    if (!count) return kOk;
    fill_random_kernel<<<8 * sm_count(), kDecThreads, 0, static_cast<cudaStream_t>(stream)>>>(
        static_cast<uint8_t *>(out), kind, bytes, scale_bytes, count, seed, scale, ones);
    return launch_status("fill_random_kernel");
}

GLMVX_EXPORT int32_t glmvx_argmax_rows(int32_t *ids, const float *logits, int32_t rows, int32_t n, void *stream) {
    if (rows < 0 || n <= 0) return set_error("argmax_rows: invalid dimensions"), kInvalid;
    if (!rows) return kOk;
    argmax_rows_kernel<<<rows, kArgmaxThreads, 0, static_cast<cudaStream_t>(stream)>>>(ids, logits, n);
    return launch_status("argmax_rows_kernel");
}
