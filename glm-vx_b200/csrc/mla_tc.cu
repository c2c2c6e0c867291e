// Absorbed-MLA split partials on the 5th-generation tensor cores (the
// contract of mla_partial, gpu/runtime.py:840-882: per split of the selected
// rows, the unnormalised softmax-weighted latents with their (max, mass)),
// for one selection shared by all heads (the DSA case) and up to 64 heads.
//
// One CTA per (split of up to 128 selected rows, query).  Three phases, all
// operands K-major 128-byte-swizzled tiles in shared memory, f32 accuracy
// from the three-term TF32 split x = hi + lo (hi.hi + hi.lo + lo.hi):
//   1. S^T [rows x heads] = K [rows x (rank+rope)] . Q^T: MMA M = 128 rows
//      (tensor-memory lanes), N = heads rounded to 16, K = 32-column chunks
//      of [latent | rope]; the rows are gathered by id while loading.
//   2. Softmax over the split per head: S^T read by its row's thread, moved
//      through shared memory so one thread per (head, half of the rows)
//      takes the max, exp(s - max), the mass, and writes P^T [heads x rows]
//      (split hi/lo) as the next B operand.  Rows past the split or with ids
//      outside [0, tokens) get probability 0.
//   3. O^T [rank x heads] = V^T [rank x rows] . P^T: M = 128 latent columns
//      per block (tensor-memory lanes), K = 32-row chunks; V^T is the same
//      latent rows, transposed on the way into shared memory.
// The epilogue writes O^T (thread = latent column) as the split's partial
// numerator rows [heads][rank] and (max, mass) per head; mla_merge_kernel
// combines the splits.  Loads of the next step are issued before the
// current step's MMAs (registers), two stages, every wait bounded.
#include <algorithm>
#include <cmath>
#include <cstdint>

#include "common.cuh"
#include "dsa.cuh"
#include "tcgen05.cuh"

namespace glmvx {

namespace {

constexpr int kMtRows = 128, kMtThreads = 256, kMtChunk = 32, kMtMaxHeads = 64, kMtMaxRank = 512;
constexpr int kMtMaxRope = 64, kMtMaxSplits = 64;  // splits per query: the merge kernel's limit
constexpr int kMtTile = kMtRows * kMtChunk * 4;        // 16 KB: one hi or lo operand tile of 128 rows
constexpr int kMtQTile = kMtMaxHeads * kMtChunk * 4;   // 8 KB: a 32-column chunk of <= 64 query heads
constexpr int kMtStage = 2 * kMtTile + 2 * kMtQTile;   // phase 1: K hi, K lo, Q hi, Q lo (phase 3 uses 2 tiles)
constexpr int kMtStages = 2;
constexpr int kMtPTile = kMtMaxHeads * kMtChunk * 4;   // one 32-row atom of P^T for <= 64 heads
constexpr int kMtPBytes = 2 * 4 * kMtPTile;            // hi + lo, four 32-row atoms
constexpr int kMtSmem = kMtStages * kMtStage + kMtPBytes + 1024;
constexpr int kMtSStride = kMtMaxHeads + 1;            // transposition buffer row (floats)
constexpr uint32_t kMtTmemCols = 512;                  // O^T blocks at 64 * block, S^T at 256
constexpr uint32_t kMtSCol = 256;

__device__ __forceinline__ void mt_split(float x, uint32_t &hi, uint32_t &lo) {
    hi = tf32_rna(x);
    lo = tf32_rna(x - __uint_as_float(hi));
}

__device__ __forceinline__ void mt_store_split(uint8_t *hi_tile, uint8_t *lo_tile, uint32_t off, float4 v) {
    uint32_t h[4], l[4];
    mt_split(v.x, h[0], l[0]);
    mt_split(v.y, h[1], l[1]);
    mt_split(v.z, h[2], l[2]);
    mt_split(v.w, h[3], l[3]);
    *reinterpret_cast<uint4 *>(hi_tile + off) = make_uint4(h[0], h[1], h[2], h[3]);
    *reinterpret_cast<uint4 *>(lo_tile + off) = make_uint4(l[0], l[1], l[2], l[3]);
}

// Four consecutive f32 at src (n valid of them), vector load when VEC.
template <bool VEC>
__device__ __forceinline__ float4 mt_ld4(const float *src, int n) {
    if (VEC) return n >= 4 ? __ldg(reinterpret_cast<const float4 *>(src)) : make_float4(0.f, 0.f, 0.f, 0.f);
    float4 v;
    v.x = n > 0 ? __ldg(src) : 0.0f;
    v.y = n > 1 ? __ldg(src + 1) : 0.0f;
    v.z = n > 2 ? __ldg(src + 2) : 0.0f;
    v.w = n > 3 ? __ldg(src + 3) : 0.0f;
    return v;
}

struct MtArgs {
    float *numerator, *stats;
    const float *q_latent, *q_rope, *latent, *rope;
    const int32_t *selected, *lens;
    int heads, rank, rope_dim, tokens, count, splits, rows_per_split, n_pad;
    float scale;
    int64_t latent_stride, rope_stride, sel_stride;
    int *err;
};

template <bool VEC>
__global__ void __launch_bounds__(kMtThreads, 1) mla_tc_kernel(MtArgs a) {
    extern __shared__ uint8_t mt_smem_raw[];
    __shared__ uint64_t mma_done[kMtStages];
    __shared__ uint64_t phase_done;
    __shared__ uint32_t tmem_slot;
    __shared__ int s_ids[kMtRows];
    __shared__ float s_red[4][kMtMaxHeads], s_mass[4][kMtMaxHeads];
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int split = blockIdx.x, bq = blockIdx.z;
    int tokens = a.tokens, count = a.count;
    if (a.lens) {
        tokens = min(tokens, max(0, a.lens[bq]));
        count = min(count, tokens);
    }
    const float *q_latent = a.q_latent + static_cast<size_t>(bq) * a.heads * a.rank;
    const float *q_rope = a.q_rope + static_cast<size_t>(bq) * a.heads * a.rope_dim;
    const float *latent = a.latent + bq * a.latent_stride, *rope = a.rope + bq * a.rope_stride;
    const int32_t *selected = a.selected ? a.selected + bq * a.sel_stride : nullptr;
    float *numerator = a.numerator + static_cast<size_t>(bq) * a.splits * a.heads * a.rank;
    float *stats = a.stats + static_cast<size_t>(bq) * a.splits * a.heads * 2;
    const int rank = a.rank, rope_dim = a.rope_dim, heads = a.heads, n_pad = a.n_pad;
    const int j0 = split * a.rows_per_split, j1 = min(count, j0 + a.rows_per_split);

    const uint32_t raw = smem_addr(mt_smem_raw);
    const uint32_t pad = ((raw + 1023u) & ~1023u) - raw;  // swizzled tiles on 1 KB boundaries
    uint8_t *base = mt_smem_raw + pad;
    const uint32_t base_s = raw + pad;
    uint8_t *ph = base + kMtStages * kMtStage, *pl = ph + 4 * kMtPTile;
    const uint32_t ph_s = base_s + kMtStages * kMtStage, pl_s = ph_s + 4 * kMtPTile;
    float *sbuf = reinterpret_cast<float *>(base);  // phase 2 only: [128][65] over the ring

    if (warp == 0) tmem_alloc(&tmem_slot, kMtTmemCols);
    if (tid == 0) {
        for (int s = 0; s < kMtStages; ++s) mbar_init(&mma_done[s], 1);
        mbar_init(&phase_done, 1);
        fence_mbar_init();
    }
    if (tid < kMtRows) {
        const int j = j0 + tid;
        int id = -1;
        if (j < j1) {
            id = selected ? __ldg(selected + j) : j;
            if (id < 0 || id >= tokens) id = -1;
        }
        s_ids[tid] = id;
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    const uint32_t idesc = umma_idesc_tf32(kMtRows, n_pad);
    const int cl = (rank + kMtChunk - 1) / kMtChunk, cr = (rope_dim + kMtChunk - 1) / kMtChunk, nch = cl + cr;
    const int nb = (rank + 127) / 128;  // O^T blocks of 128 latent columns
    const int steps = nch + 4 * nb;     // phase 1 chunks, then phase 3 (block, 32-row chunk) steps
    bool ok = true;
    int done_phase = 0;  // completions of phase_done waited for

    // Registers of one step: phase 1 K rows (4 float4) + Q heads (2 float4);
    // phase 3 V rows (4 float4: 4 columns x 4 rows per thread).  Two sets:
    // the loads of steps st+1 and st+2 are in flight during step st.
    float4 rk0[4], rq0[2], rk1[4], rq1[2];
    auto load_step = [&](int st, float4 (&rk)[4], float4 (&rq)[2]) {
        if (st < nch) {  // K chunk st: row r = i >> 3, columns 4p.. (p = i & 7)
            const bool lat = st < cl;
            const int c0 = lat ? kMtChunk * st : kMtChunk * (st - cl), width = lat ? rank : rope_dim;
            const float *src_base = lat ? latent : rope;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int i = tid + kMtThreads * jj, r = i >> 3, d = c0 + 4 * (i & 7), id = s_ids[r];
                rk[jj] = id >= 0 ? mt_ld4<VEC>(src_base + static_cast<int64_t>(id) * width + d, width - d)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            }
            const float *qb = lat ? q_latent : q_rope;
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                const int i = tid + kMtThreads * jj, h = i >> 3, d = c0 + 4 * (i & 7);
                rq[jj] = h < heads ? mt_ld4<VEC>(qb + static_cast<size_t>(h) * width + d, width - d)
                                   : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        } else {  // V^T block mb, rows 32kc + 4g .. + 3 (g = tid >> 5), columns 128mb + 4 lane ..
            const int k = st - nch, mb = k >> 2, kc = k & 3, g = tid >> 5, d = 128 * mb + 4 * lane;
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int id = s_ids[32 * kc + 4 * g + jj];
                rk[jj] = id >= 0 ? mt_ld4<VEC>(latent + static_cast<int64_t>(id) * rank + d, rank - d)
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
            }
        }
    };
    auto store_step = [&](int st, uint8_t *stage, const float4 (&rk)[4], const float4 (&rq)[2]) {
        uint8_t *t_hi = stage, *t_lo = stage + kMtTile;
        if (st < nch) {
#pragma unroll
            for (int jj = 0; jj < 4; ++jj) {
                const int i = tid + kMtThreads * jj;
                mt_store_split(t_hi, t_lo, sw128_offset(i >> 3, i & 7), rk[jj]);
            }
            uint8_t *q_hi = stage + 2 * kMtTile, *q_lo = q_hi + kMtQTile;
#pragma unroll
            for (int jj = 0; jj < 2; ++jj) {
                const int i = tid + kMtThreads * jj;
                if ((i >> 3) < n_pad) mt_store_split(q_hi, q_lo, sw128_offset(i >> 3, i & 7), rq[jj]);
            }
        } else {  // transpose: column 4*lane + e of the block is row e of V^T; rows 4g..4g+3 are chunk g
            const int g = tid >> 5;
            mt_store_split(t_hi, t_lo, sw128_offset(4 * lane, g), make_float4(rk[0].x, rk[1].x, rk[2].x, rk[3].x));
            mt_store_split(t_hi, t_lo, sw128_offset(4 * lane + 1, g), make_float4(rk[0].y, rk[1].y, rk[2].y, rk[3].y));
            mt_store_split(t_hi, t_lo, sw128_offset(4 * lane + 2, g), make_float4(rk[0].z, rk[1].z, rk[2].z, rk[3].z));
            mt_store_split(t_hi, t_lo, sw128_offset(4 * lane + 3, g), make_float4(rk[0].w, rk[1].w, rk[2].w, rk[3].w));
        }
    };
    auto issue_step = [&](int st, uint32_t stage_s) {
        const uint32_t t_hi = stage_s, t_lo = stage_s + kMtTile;
        if (st < nch) {
            const uint32_t q_hi = stage_s + 2 * kMtTile, q_lo = q_hi + kMtQTile;
#pragma unroll
            for (int kk = 0; kk < kMtChunk / 8; ++kk) {
                const uint64_t ah = umma_desc_sw128(t_hi + 32 * kk), al = umma_desc_sw128(t_lo + 32 * kk);
                const uint64_t bh = umma_desc_sw128(q_hi + 32 * kk), bl = umma_desc_sw128(q_lo + 32 * kk);
                umma_tf32(tmem + kMtSCol, ah, bh, idesc, (st > 0 || kk > 0) ? 1u : 0u);
                umma_tf32(tmem + kMtSCol, ah, bl, idesc, 1u);
                umma_tf32(tmem + kMtSCol, al, bh, idesc, 1u);
            }
        } else {
            const int k = st - nch, mb = k >> 2, kc = k & 3;
            const uint32_t bh_s = ph_s + kc * kMtPTile, bl_s = pl_s + kc * kMtPTile;
#pragma unroll
            for (int kk = 0; kk < kMtChunk / 8; ++kk) {
                const uint64_t ah = umma_desc_sw128(t_hi + 32 * kk), al = umma_desc_sw128(t_lo + 32 * kk);
                const uint64_t bh = umma_desc_sw128(bh_s + 32 * kk), bl = umma_desc_sw128(bl_s + 32 * kk);
                const uint32_t d = tmem + 64 * mb;
                umma_tf32(d, ah, bh, idesc, (kc > 0 || kk > 0) ? 1u : 0u);
                umma_tf32(d, ah, bl, idesc, 1u);
                umma_tf32(d, al, bh, idesc, 1u);
            }
        }
    };
    // Waits for every MMA issued so far (committed to phase_done).
    auto wait_phase = [&]() -> bool {
        const bool w = mbar_wait_bounded(&phase_done, done_phase & 1);
        ++done_phase;
        return __syncthreads_and(w);
    };

    // One step on register set (rk, rq): false when a bounded wait expired.
    auto step = [&](int st, float4 (&rk)[4], float4 (&rq)[2]) -> bool {
        const int s = st % kMtStages;
        bool w = true;
        if (st >= kMtStages) w = mbar_wait_bounded(&mma_done[s], ((st - kMtStages) / kMtStages) & 1);
        if (!__syncthreads_and(w)) return false;
        if (st == nch) {
            // ---- phase 2: softmax of the split from S^T (all S MMAs committed below) ----
            if (!wait_phase()) return false;
            tc_fence_after();
            {  // warp w: rows 32 (w % 4) + lane, head columns 32 (w / 4) ..
                const int r = 32 * (warp & 3) + lane, h0 = 32 * (warp >> 2);
                const bool valid = s_ids[r] >= 0;
                if (h0 < n_pad) {
                    uint32_t v[32];
                    tmem_ld32(tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + kMtSCol + h0, v);
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (h0 + j < n_pad)
                            sbuf[r * kMtSStride + h0 + j] = valid ? __uint_as_float(v[j]) * a.scale : -INFINITY;
                }
            }
            __syncthreads();
            const int h = tid & 63, qq = tid >> 6;  // head, quarter of the rows (32 rows = one P^T atom)
            float m = -INFINITY;
            if (h < n_pad)
                for (int rr = 32 * qq; rr < 32 * qq + 32; ++rr) m = fmaxf(m, sbuf[rr * kMtSStride + h]);
            s_red[qq][h] = m;
            __syncthreads();
            m = fmaxf(fmaxf(s_red[0][h], s_red[1][h]), fmaxf(s_red[2][h], s_red[3][h]));
            float mass = 0.0f;
            if (h < n_pad) {
                for (int c = 0; c < 8; ++c) {  // rows 32 qq + 4c .. + 3: chunk c of P^T row h in atom qq
                    const int r0 = 32 * qq + 4 * c;
                    float4 p;
                    float *pp = &p.x;
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        const float sv = sbuf[(r0 + e) * kMtSStride + h];
                        pp[e] = sv == -INFINITY ? 0.0f : expf(sv - m);
                        mass += pp[e];
                    }
                    mt_store_split(ph + qq * kMtPTile, pl + qq * kMtPTile, sw128_offset(h, c), p);
                }
            }
            s_mass[qq][h] = mass;
            fence_proxy_async_smem();
            tc_fence_before();
            __syncthreads();
            tc_fence_after();
            if (tid < heads) {
                const size_t task = static_cast<size_t>(split) * heads + tid;
                stats[task * 2] = fmaxf(fmaxf(s_red[0][tid], s_red[1][tid]), fmaxf(s_red[2][tid], s_red[3][tid]));
                stats[task * 2 + 1] = (s_mass[0][tid] + s_mass[1][tid]) + (s_mass[2][tid] + s_mass[3][tid]);
            }
            __syncthreads();  // the ring (sbuf) is free again
        }
        uint8_t *stage = base + s * kMtStage;
        store_step(st, stage, rk, rq);
        if (st + 2 < steps) load_step(st + 2, rk, rq);
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            issue_step(st, base_s + s * kMtStage);
            umma_commit(&mma_done[s]);
            if (st == nch - 1 || st == steps - 1) umma_commit(&phase_done);
        }
        return true;
    };
    load_step(0, rk0, rq0);
    if (steps > 1) load_step(1, rk1, rq1);
    for (int st = 0; st < steps && ok; st += 2) {
        ok = step(st, rk0, rq0);
        if (ok && st + 1 < steps) ok = step(st + 1, rk1, rq1);
    }
    if (ok) ok = wait_phase();  // every O^T MMA
    if (ok) {
        tc_fence_after();
        const int h0 = 32 * (warp >> 2);  // warp w: lanes 32 (w % 4) .. of each block, heads h0 ..
        if (h0 < n_pad) {
            for (int mb = 0; mb < nb; ++mb) {
                const int d = 128 * mb + 32 * (warp & 3) + lane;  // latent column = tensor-memory lane of block mb
                uint32_t v[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + 64 * mb + h0, v);
                if (d < rank) {
#pragma unroll
                    for (int j = 0; j < 32; ++j)
                        if (h0 + j < heads)
                            numerator[(static_cast<size_t>(split) * heads + h0 + j) * rank + d] = __uint_as_float(v[j]);
                }
            }
        }
    } else if (tid == 0) {
        report_device_error(a.err, kDevErrFullWait);
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0) tmem_dealloc(tmem, kMtTmemCols);
}

}  // namespace

bool mla_tc_supported(int heads, int rank, int rope_dim, int count) {
    return heads >= 1 && heads <= kMtMaxHeads && rank >= 1 && rank <= kMtMaxRank && rope_dim >= 0 &&
           rope_dim <= kMtMaxRope && count <= kMtMaxSplits * kMtRows;
}

int mla_tc_splits(int count, int batch) {
    // 128 rows per split, or 64 when that leaves the GPU under one CTA per SM
    // and stays within kMtMaxSplits splits (the merge's limit).
    const int rows = (batch * ((count + 127) / 128) < 148 && count <= kMtMaxSplits * 64) ? 64 : 128;
    return std::max(1, (count + rows - 1) / rows);
}

int32_t launch_mla_tc(float *numerator, float *stats, const float *q_latent, const float *q_rope, const float *latent,
                      const float *rope, const int32_t *selected, const int32_t *lens, int heads, int rank,
                      int rope_dim, int tokens, int count, int splits, float scale, int64_t latent_stride,
                      int64_t rope_stride, int64_t sel_stride, int batch, cudaStream_t stream) {
    if (!mla_tc_supported(heads, rank, rope_dim, count)) return kUnsupported;
    if (splits > kMtMaxSplits) return set_error("mla_tc: more than %d splits", kMtMaxSplits), kInvalid;
    if (batch <= 0 || splits <= 0) return kOk;
    if (const int32_t rc = allow_dynamic_smem(mla_tc_kernel<true>, kMtSmem, "mla_tc smem")) return rc;
    if (const int32_t rc = allow_dynamic_smem(mla_tc_kernel<false>, kMtSmem, "mla_tc smem")) return rc;
    MtArgs args{numerator, stats, q_latent, q_rope, latent, rope, selected, lens, heads, rank, rope_dim, tokens,
                count, splits, (count + splits - 1) / splits, (heads + 15) / 16 * 16, scale, latent_stride,
                rope_stride, sel_stride, device_error_word()};
    if (args.rows_per_split > kMtRows) return set_error("mla_tc: more than 128 rows per split"), kInvalid;
    const bool vec = rank % 4 == 0 && rope_dim % 4 == 0 && latent_stride % 4 == 0 && rope_stride % 4 == 0 &&
                     ((reinterpret_cast<uintptr_t>(latent) | reinterpret_cast<uintptr_t>(rope) |
                       reinterpret_cast<uintptr_t>(q_latent) | reinterpret_cast<uintptr_t>(q_rope)) & 15) == 0;
    const dim3 grid(splits, 1, batch);
    if (vec) mla_tc_kernel<true><<<grid, kMtThreads, kMtSmem, stream>>>(args);
    else mla_tc_kernel<false><<<grid, kMtThreads, kMtSmem, stream>>>(args);
    GLMVX_CUDA(cudaGetLastError());
    return kOk;
}

}  // namespace glmvx
