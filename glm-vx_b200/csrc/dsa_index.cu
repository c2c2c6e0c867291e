// DSA indexer scores on the 5th-generation tensor cores
// (kernels/kernels.vx:404-421, gpu/kernels.vx:169-204; model.py:159-165):
//   score_t = sum_h w_h * relu(qk_scale * q_h . k_t)
// as a GEMM: the 128 keys of a tile (MMA M, one tensor-memory lane each)
// against all heads (MMA N = heads rounded up to 16) over the key columns
// (MMA K, chunks of 32 = one 128-byte swizzle row).  f32 accuracy from TF32
// operands by the three-term split x = hi + lo (hi = tf32_rna(x), lo =
// tf32_rna(x - hi)): q.k ~ qh.kh + ql.kh + qh.kl, each product exact in f32,
// the dropped ql.kl below 2^-22 of |q||k|; accumulation in f32 in tensor
// memory.  A CTA keeps one query's hi/lo heads in shared memory and walks
// tiles of its keys (persistent over the tiles of one query): 128 threads
// hold a tile's column chunk in registers (a warp reads 4 full 128-byte row
// segments per load; the next chunk's loads are issued before this one's
// MMAs), split it and store both halves as swizzled K-major tiles through a
// two-stage ring; one thread issues the 3 x 4 MMAs of each chunk into one of
// two accumulator buffers, so the epilogue of a tile -- each key's head dots
// read by its thread (tcgen05.ld), relu * weight reduced in head order --
// runs while the next tile's MMAs do.
#include <algorithm>
#include <cstdint>

#include "common.cuh"
#include "dsa.cuh"
#include "tcgen05.cuh"

namespace glmvx {

namespace {

constexpr int kIdxTile = 128, kIdxChunk = 32, kIdxThreads = 128, kIdxStages = 2;
constexpr int kIdxKeyBytes = kIdxTile * kIdxChunk * 4;  // 16 KB: hi or lo of one column chunk
constexpr int kIdxStageBytes = 2 * kIdxKeyBytes;
constexpr int kIdxMaxQRowChunks = 256;  // heads (rounded to 16) x column chunks: 64 KB of hi + lo
constexpr int kIdxMaxHeads = 128;       // two accumulator buffers of <= 128 columns
constexpr int kIdxSmem = kIdxStages * kIdxStageBytes + 2 * kIdxMaxQRowChunks * 128 + 1024;

__device__ __forceinline__ void split_tf32(float x, uint32_t &hi, uint32_t &lo) {
    hi = tf32_rna(x);
    lo = tf32_rna(x - __uint_as_float(hi));
}

// One column chunk of a tile's keys in registers: key r = i >> 3, columns
// 32c + 4p .. + 3 (p = i & 7) for i = tid + 128 j.
template <bool VEC>
__device__ __forceinline__ void idx_load(float4 (&v)[kIdxTile * 8 / kIdxThreads], const float *keys, int tokens,
                                         int dim, int t0, int c, int tid) {
#pragma unroll
    for (int j = 0; j < kIdxTile * 8 / kIdxThreads; ++j) {
        const int i = tid + kIdxThreads * j, t = t0 + (i >> 3), d = kIdxChunk * c + 4 * (i & 7);
        const float *src = keys + static_cast<int64_t>(t) * dim + d;
        if (VEC) {
            v[j] = (t < tokens && d < dim) ? __ldg(reinterpret_cast<const float4 *>(src))
                                           : make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
            v[j].x = (t < tokens && d < dim) ? __ldg(src) : 0.0f;
            v[j].y = (t < tokens && d + 1 < dim) ? __ldg(src + 1) : 0.0f;
            v[j].z = (t < tokens && d + 2 < dim) ? __ldg(src + 2) : 0.0f;
            v[j].w = (t < tokens && d + 3 < dim) ? __ldg(src + 3) : 0.0f;
        }
    }
}

template <bool VEC>
__global__ void __launch_bounds__(kIdxThreads, 2)
    index_tc_kernel(float *__restrict__ out, const float *__restrict__ q, const float *__restrict__ keys,
                    const float *__restrict__ w, int tokens, int heads, int dim, float qk_scale,
                    const int32_t *__restrict__ lens, int64_t key_stride, int64_t out_stride, int n_pad,
                    uint32_t acc_cols, int *err) {
    extern __shared__ uint8_t idx_smem_raw[];
    __shared__ uint64_t mma_done[kIdxStages];
    __shared__ uint64_t tile_done[2];
    __shared__ uint32_t tmem_slot;
    __shared__ float s_w[kIdxMaxHeads];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int b = blockIdx.y;  // query of a batch
    if (lens) tokens = min(tokens, max(0, lens[b]));
    const int ntiles = (tokens + kIdxTile - 1) / kIdxTile;
    if (static_cast<int>(blockIdx.x) >= ntiles) return;  // uniform, before any allocation
    q += static_cast<size_t>(b) * heads * dim;
    w += static_cast<size_t>(b) * heads;
    keys += b * key_stride;
    out += b * out_stride;
    const uint32_t raw = smem_addr(idx_smem_raw);
    const uint32_t pad = ((raw + 1023u) & ~1023u) - raw;  // swizzled tiles on 1 KB boundaries
    uint8_t *base = idx_smem_raw + pad;
    const uint32_t base_s = raw + pad;
    const int nchunks = (dim + kIdxChunk - 1) / kIdxChunk;
    const int qtile = n_pad * 128;  // bytes of one column chunk of the hi (or lo) queries
    uint8_t *qh = base + kIdxStages * kIdxStageBytes, *ql = qh + nchunks * qtile;
    const uint32_t qh_s = base_s + kIdxStages * kIdxStageBytes, ql_s = qh_s + nchunks * qtile;

    // Two accumulator buffers of acc_cols columns: tile i uses buffer i % 2,
    // so a tile's epilogue overlaps the next tile's MMAs.
    if (warp == 0) tmem_alloc(&tmem_slot, 2 * acc_cols);
    if (tid == 0) {
        for (int s = 0; s < kIdxStages; ++s) mbar_init(&mma_done[s], 1);
        mbar_init(&tile_done[0], 1);
        mbar_init(&tile_done[1], 1);
        fence_mbar_init();
    }
    // Queries (rows >= heads zero), split once per CTA.
    for (int i = tid; i < n_pad * nchunks * 8; i += kIdxThreads) {
        const int h = i / (nchunks * 8), rem = i - h * nchunks * 8, c = rem >> 3, p = rem & 7;
        uint32_t hi[4], lo[4];
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int d = kIdxChunk * c + 4 * p + e;
            split_tf32(h < heads && d < dim ? q[static_cast<size_t>(h) * dim + d] : 0.0f, hi[e], lo[e]);
        }
        const uint32_t off = c * qtile + sw128_offset(h, p);
        *reinterpret_cast<uint4 *>(qh + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
        *reinterpret_cast<uint4 *>(ql + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
    }
    for (int i = tid; i < heads; i += kIdxThreads) s_w[i] = w[i];
    fence_proxy_async_smem();
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const uint32_t idesc = umma_idesc_tf32(kIdxTile, n_pad);

    // Epilogue of this CTA's k-th tile: thread = key (tensor-memory lane),
    // relu * weight over the heads in order.
    auto epilogue = [&](int k) -> bool {
        const bool waited = mbar_wait_bounded(&tile_done[k & 1], (k >> 1) & 1);
        if (!__syncthreads_and(waited)) return false;  // uniform: every thread leaves together
        tc_fence_after();
        const int t = (static_cast<int>(blockIdx.x) + k * static_cast<int>(gridDim.x)) * kIdxTile + 32 * warp + lane;
        const uint32_t acc = tmem + (static_cast<uint32_t>(32 * warp) << 16) + (k & 1) * acc_cols;
        float total = 0.0f;
        for (int h0 = 0; h0 < n_pad; h0 += 32) {
            uint32_t v[32];
            tmem_ld32(acc + h0, v);
#pragma unroll
            for (int j = 0; j < 32; ++j) {
                if (h0 + j < heads) {
                    const float sc = __uint_as_float(v[j]) * qk_scale;
                    if (sc > 0.0f) total = fmaf(s_w[h0 + j], sc, total);
                }
            }
        }
        if (t < tokens) out[t] = total;
        tc_fence_before();  // these accumulators are overwritten by the tile after next
        return true;
    };

    const int my_tiles = (ntiles - static_cast<int>(blockIdx.x) + static_cast<int>(gridDim.x) - 1) / gridDim.x;
    const int total = my_tiles * nchunks;  // (tile, chunk) steps of this CTA
    float4 v[kIdxTile * 8 / kIdxThreads];
    idx_load<VEC>(v, keys, tokens, dim, blockIdx.x * kIdxTile, 0, tid);
    bool ok = true;
    for (int seq = 0; seq < total; ++seq) {
        const int k = seq / nchunks, c = seq - k * nchunks, s = seq % kIdxStages;
        if (seq >= kIdxStages) ok = mbar_wait_bounded(&mma_done[s], ((seq - kIdxStages) / kIdxStages) & 1);
        if (!__syncthreads_and(ok)) {  // the stage is still read by MMAs that did not finish
            if (tid == 0) report_device_error(err, kDevErrFullWait);
            ok = false;
            break;
        }
        uint8_t *kh = base + s * kIdxStageBytes, *kl = kh + kIdxKeyBytes;
#pragma unroll
        for (int j = 0; j < kIdxTile * 8 / kIdxThreads; ++j) {
            const int i = tid + kIdxThreads * j;
            uint32_t hi[4], lo[4];
            split_tf32(v[j].x, hi[0], lo[0]);
            split_tf32(v[j].y, hi[1], lo[1]);
            split_tf32(v[j].z, hi[2], lo[2]);
            split_tf32(v[j].w, hi[3], lo[3]);
            const uint32_t off = sw128_offset(i >> 3, i & 7);
            *reinterpret_cast<uint4 *>(kh + off) = make_uint4(hi[0], hi[1], hi[2], hi[3]);
            *reinterpret_cast<uint4 *>(kl + off) = make_uint4(lo[0], lo[1], lo[2], lo[3]);
        }
        if (seq + 1 < total) {  // the next step's keys are in flight during the MMAs and the epilogue
            const int k1 = (seq + 1) / nchunks, c1 = seq + 1 - k1 * nchunks;
            idx_load<VEC>(v, keys, tokens, dim, (static_cast<int>(blockIdx.x) + k1 * static_cast<int>(gridDim.x)) * kIdxTile,
                          c1, tid);
        }
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t kh_s = base_s + s * kIdxStageBytes, kl_s = kh_s + kIdxKeyBytes;
            const uint32_t qhc = qh_s + c * qtile, qlc = ql_s + c * qtile, acc = tmem + (k & 1) * acc_cols;
#pragma unroll
            for (int kk = 0; kk < kIdxChunk / 8; ++kk) {
                const uint64_t ah = umma_desc_sw128(kh_s + 32 * kk), al = umma_desc_sw128(kl_s + 32 * kk);
                const uint64_t bh = umma_desc_sw128(qhc + 32 * kk), bl = umma_desc_sw128(qlc + 32 * kk);
                umma_tf32(acc, ah, bh, idesc, (c > 0 || kk > 0) ? 1u : 0u);
                umma_tf32(acc, ah, bl, idesc, 1u);
                umma_tf32(acc, al, bh, idesc, 1u);
            }
            umma_commit(&mma_done[s]);
            if (c == nchunks - 1) umma_commit(&tile_done[k & 1]);
        }
        // After the last chunk of tile k: the epilogue of tile k - 1 (its
        // MMAs finished long ago; tile k's run meanwhile).
        if (c == nchunks - 1 && k >= 1 && !epilogue(k - 1)) {
            ok = false;
            break;
        }
    }
    if (ok && !epilogue(my_tiles - 1)) ok = false;
    if (!ok && tid == 0) report_device_error(err, kDevErrFullWait);
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, 2 * acc_cols);
}

}  // namespace

// The tensor-core path when heads <= 128 and the hi + lo queries fit
// (heads rounded to 16 x column chunks of 32 <= 256); kUnsupported otherwise.
int32_t launch_index_scores_tc(float *out, const float *q, const float *keys, const float *w, int tokens, int heads,
                               int dim, float qk_scale, const int32_t *lens, int64_t key_stride, int64_t out_stride,
                               int batch, cudaStream_t stream) {
    const int n_pad = (heads + 15) / 16 * 16, nchunks = (dim + kIdxChunk - 1) / kIdxChunk;
    if (heads < 1 || heads > kIdxMaxHeads || dim < 1 || n_pad * nchunks > kIdxMaxQRowChunks) return kUnsupported;
    if (tokens <= 0 || batch <= 0) return kOk;
    uint32_t cols = 32;
    while (cols < static_cast<uint32_t>(n_pad)) cols <<= 1;
    if (const int32_t rc = allow_dynamic_smem(index_tc_kernel<true>, kIdxSmem, "index_tc smem")) return rc;
    if (const int32_t rc = allow_dynamic_smem(index_tc_kernel<false>, kIdxSmem, "index_tc smem")) return rc;
    const int smem = kIdxStages * kIdxStageBytes + 2 * nchunks * n_pad * 128 + 1024;
    const int tiles = (tokens + kIdxTile - 1) / kIdxTile;
    // Two CTAs per SM, all resident at once: per query the floor of the
    // slots over the queries (the ceiling put CTAs into a second wave, e.g.
    // 19 x 16 = 304 > 296 at 16 queries: 180 -> 120 us for the indexer).
    const int per_query = std::max(1, std::min(tiles, 2 * sm_count() / batch));
    const dim3 grid(per_query, batch);
    const bool vec = dim % 4 == 0 && key_stride % 4 == 0 && (reinterpret_cast<uintptr_t>(keys) & 15) == 0;
    if (vec)
        index_tc_kernel<true><<<grid, kIdxThreads, smem, stream>>>(out, q, keys, w, tokens, heads, dim, qk_scale, lens,
                                                                   key_stride, out_stride, n_pad, cols,
                                                                   device_error_word());
    else
        index_tc_kernel<false><<<grid, kIdxThreads, smem, stream>>>(out, q, keys, w, tokens, heads, dim, qk_scale,
                                                                    lens, key_stride, out_stride, n_pad, cols,
                                                                    device_error_word());
    GLMVX_CUDA(cudaGetLastError());
    return kOk;
}

}  // namespace glmvx
