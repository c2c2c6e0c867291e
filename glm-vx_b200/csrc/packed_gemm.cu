// Packed-GGUF GEMM for token batches on the f16 tensor cores (mma.sync
// m16n8k16, f32 accumulation).
//
// Same contract as the reference's batched packed kernels (the batch_v2 entry
// points, kernels/packed.vx:473ff) and the GEMV path (packed_mma.cu):
// out[t][r] = sum_j w[r][j] * x[t][j] in f32 with the weights decoded per GGML
// block.  With a batch of tokens each weight fragment is decoded once and
// multiplied into every token, so the decoded values carry the block's
// integer scales and the tensor core accumulates a whole 256-column block:
//
//   Q4_K   w = d*sc*q - dmin*m        A = sc*q (integers <= 945, exact in
//                                     f16); per superblock D*d, minus
//                                     dmin * sum_j m_j * X_j with X_j the
//                                     token's 32-column sums
//   IQ1_S  w = d*(2s+1)*(g + delta)   A = (2s+1)*(8g +- 1) (integers <= 135,
//                                     exact in f16); per block D*d/8
//   Q8_0   w = d*q                    A = q (exact in f16); d per 32 columns
//
// The activations enter as two f16 limbs.  Per 256-column chunk of a token,
// x*2^E (largest magnitude in [2^14, 2^15)) = hi + lo with hi = f16(x*2^E),
// lo = f16(x*2^E - hi): 22 significant bits per element (a subnormal lo, for
// elements far below the chunk's largest, loses only bits below 2^-38 of
// it).  Products of f16 operands are exact in the f32 accumulator, so the
// remaining error is that of f32 accumulation.
//
// Fragment layout (m16n8k16, A row-major, B column-major): lane (g = lane/4,
// t = lane%4) holds A rows g, g+8 at logical k {2t, 2t+1, 2t+8, 2t+9} and B
// column g at the same k.  Those four logical k are the physical columns
// 4t..4t+3 of the 16-column step, for A and B alike, so a lane decodes four
// consecutive weights of each of its rows.  B column g of an 8-column tile is
// token 4q + g/2 (tile q), limb g%2; the accumulator columns 2t, 2t+1 of a lane
// are then both limbs of token 4q + t.
//
// Kernel structure (gemm_f16_kernel): a persistent grid, one CTA per SM, each
// CTA owning a balanced range of rows, in tiles of 16*RG rows.  A producer
// warp loads a tile's packed rows into shared memory once (one bulk copy per
// row, rows padded so the 8 rows of a fragment fall in distinct banks), then
// streams the prepared activation chunks (one bulk copy each) through a ring
// of 2*S stages.  RG*TG*S consumer warps each take 16 rows x 4*NTW tokens x
// every S-th chunk; the S partial sums of a row and token are added in fixed
// order at the end of the tile.  Waits on mbarriers are bounded (2 s) and
// report through the device error word.
#include <algorithm>
#include <cuda_fp16.h>

#include "codecs.cuh"
#include "mma_gemv.cuh"

namespace glmvx {

namespace {

// ------------------------------------------------------------- fragments ---

__device__ __forceinline__ void mma_f16(float (&d)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                        uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(d[0]), "+f"(d[1]), "+f"(d[2]), "+f"(d[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// PRMT in its default mode (all selector nibbles used here are 0..6).
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// Two 16-bit integers n < 1024, given as 0x6400 + n per half (the f16 bit
// patterns of 1024 + n), to f16 n: one exact half2 subtraction.
__device__ __forceinline__ uint32_t f16_from_biased(uint32_t biased) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(biased), "r"(0x64006400u));
    return r;
}

__device__ __forceinline__ uint32_t hfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("fma.rn.f16x2 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

__device__ __forceinline__ uint32_t lds32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }
__device__ __forceinline__ uint32_t lds32_const(uint32_t addr) {
    uint32_t v;
    asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}
__device__ __forceinline__ float pow2(int e) { return __int_as_float((127 + e) << 23); }

// (a & b) | c as one LOP3 with all three operands in registers.
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

}  // namespace

// ------------------------------------------------------ prepared records ---

// Per 256-column chunk, one record of T4 = 4*nt8 tokens (tokens >= T zero):
//   [0, 4096*nt8)            B fragments [16 steps][nt8 tiles][32 lanes] x 8 B
//   [+0, 16*nt8)             int32 E per token, or kPrepNonFinite
//   [+16*nt8, +128*nt8)      f32 sums of the token's eight 32-column sub-blocks
struct GemmRecord {
    int nt8;
    __host__ __device__ size_t frag_bytes() const { return 4096ull * nt8; }
    __host__ __device__ size_t exps_off() const { return frag_bytes(); }
    __host__ __device__ size_t sums_off() const { return frag_bytes() + 16ull * nt8; }
    __host__ __device__ size_t bytes() const { return 4240ull * nt8; }
};

// One warp per (token, chunk), 8 columns per lane.
__global__ void __launch_bounds__(256)
    prep_f16_kernel(uint8_t *__restrict__ rec, const float *__restrict__ x, int T, int T4, int cols, int nt8,
                    int xstride) {
    grid_dependency_wait();
    allow_dependent_launch();
    const int chunks = cols >> 8;
    const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= static_cast<int64_t>(T4) * chunks) return;  // warp-uniform
    const int tok = static_cast<int>(wid / chunks), chunk = static_cast<int>(wid % chunks);
    const GemmRecord R{nt8};
    uint8_t *out = rec + static_cast<size_t>(chunk) * R.bytes();
    float v[8] = {0, 0, 0, 0, 0, 0, 0, 0};
    if (tok < T) {
        const float4 *xr = reinterpret_cast<const float4 *>(x + static_cast<size_t>(tok) * xstride + chunk * 256 + lane * 8);
        const float4 lo = __ldg(xr), hi = __ldg(xr + 1);
        v[0] = lo.x, v[1] = lo.y, v[2] = lo.z, v[3] = lo.w, v[4] = hi.x, v[5] = hi.y, v[6] = hi.z, v[7] = hi.w;
    }
    float mx = 0.0f;
    bool finite = true;
#pragma unroll
    for (int i = 0; i < 8; ++i) {
        mx = fmaxf(mx, fabsf(v[i]));
        finite &= isfinite(v[i]);
    }
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o));
    finite = __all_sync(0xffffffffu, finite);
    // 2^E puts the largest magnitude in [2^14, 2^15) (E in [-113, 141]).
    const int ebits = (__float_as_int(mx) >> 23) & 0xff;
    const int E = mx == 0.0f ? 0 : 141 - ebits;
    const float up0 = pow2(E / 2), up1 = pow2(E - E / 2);
    // Column 8*lane + i of the chunk: step lane/2, physical column
    // w = 8*(lane%2) + i of the step -> fragment lane t = w/4 of each column
    // g of token tok (limb 0 at g = 2*(tok%4), limb 1 next), register (w%4)/2.
    const int st = lane >> 1, q = tok >> 2, g0 = 2 * (tok & 3);
    uint32_t *frag = reinterpret_cast<uint32_t *>(out);
#pragma unroll
    for (int i = 0; i < 8; i += 2) {
        const float s0 = finite ? (v[i] * up0) * up1 : 0.0f, s1 = finite ? (v[i + 1] * up0) * up1 : 0.0f;
        const __half h0 = __float2half_rn(s0), h1 = __float2half_rn(s1);
        const __half l0 = __float2half_rn(s0 - __half2float(h0)), l1 = __float2half_rn(s1 - __half2float(h1));
        const int w = 8 * (lane & 1) + i, t = w >> 2, reg = (w & 3) >> 1;
        const size_t base = (static_cast<size_t>(st) * nt8 + q) * 32;
        frag[(base + g0 * 4 + t) * 2 + reg] =
            static_cast<uint32_t>(__half_as_ushort(h0)) | (static_cast<uint32_t>(__half_as_ushort(h1)) << 16);
        frag[(base + (g0 + 1) * 4 + t) * 2 + reg] =
            static_cast<uint32_t>(__half_as_ushort(l0)) | (static_cast<uint32_t>(__half_as_ushort(l1)) << 16);
    }
    float sum = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if ((lane & 3) == 0) reinterpret_cast<float *>(out + R.sums_off())[tok * 8 + (lane >> 2)] = sum;
    if (lane == 0) reinterpret_cast<int *>(out + R.exps_off())[tok] = finite ? E : kPrepNonFinite;
}

// ----------------------------------------------------------- per format ---

// 2^(11-3k): (qh & 7 << 3k) * c_gemm_iq1s_mul[k] = 2048 * (grid bits of group k
// of the sub-block), the selector table offset of those bits.  From the
// constant bank so the compiler keeps a multiply-add.
__constant__ uint32_t c_gemm_iq1s_mul[4] = {2048u, 256u, 32u, 4u};

template <class F>
struct GemmFmt;

template <>
struct GemmFmt<FmtQ4_K> {
    static constexpr int kChunkBytes = 144, kTableBytes = 0;
    __device__ static void init_table(uint8_t *, int, int) {}
    __device__ __forceinline__ static int sel6(uint32_t lo, uint32_t hi, int j) {
        return static_cast<int>(((j < 4 ? lo : hi) >> (8 * (j & 3))) & 0xffu);
    }
    // One superblock (chunk) of rows g (r0) and g+8 (r1) against tiles
    // tq0..tq0+NTW-1 of the record.
    template <int NTW>
    __device__ __forceinline__ static void chunk(const uint8_t *r0, const uint8_t *r1, const uint8_t *rec, int nt8,
                                                 int tq0, int lane, uint32_t, float (&tot)[NTW][2]) {
        const int t = lane & 3;
        const uint4 h0 = *reinterpret_cast<const uint4 *>(r0), h1 = *reinterpret_cast<const uint4 *>(r1);
        // 6-bit scales of sub-blocks 0..3 (lo) and 4..7 (hi), kernels/packed.vx:107-120
        const uint32_t sl0 = h0.y & 0x3F3F3F3Fu, sh0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
        const uint32_t sl1 = h1.y & 0x3F3F3F3Fu, sh1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
        const uint2 *bf = reinterpret_cast<const uint2 *>(rec) + tq0 * 32 + lane;
        float acc[NTW][4];
#pragma unroll
        for (int q = 0; q < NTW; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.0f;
#pragma unroll
        for (int m = 0; m < 4; ++m)
#pragma unroll
        for (int hs = 0; hs < 2; ++hs) {
            // bytes 32m + 16hs + 4t..+3: low nibbles = sub-block 2m, high = 2m+1
            const uint32_t w0 = lds32(r0 + 16 + 32 * m + 16 * hs + 4 * t);
            const uint32_t w1 = lds32(r1 + 16 + 32 * m + 16 * hs + 4 * t);
#pragma unroll
            for (int h = 0; h < 2; ++h) {
                const int j = 2 * m + h, st = 2 * j + hs;
                const uint32_t n0 = (h ? w0 >> 4 : w0) & 0x0F0F0F0Fu, n1 = (h ? w1 >> 4 : w1) & 0x0F0F0F0Fu;
                const uint32_t s0 = static_cast<uint32_t>(sel6(sl0, sh0, j));
                const uint32_t s1 = static_cast<uint32_t>(sel6(sl1, sh1, j));
                // (q_i | q_{i+1} << 16) * sc + 0x64006400: f16 bits of 1024 + sc*q per half
                const uint32_t a0 = f16_from_biased(prmt(n0, 0, 0x4140) * s0 + 0x64006400u);
                const uint32_t a2 = f16_from_biased(prmt(n0, 0, 0x4342) * s0 + 0x64006400u);
                const uint32_t a1 = f16_from_biased(prmt(n1, 0, 0x4140) * s1 + 0x64006400u);
                const uint32_t a3 = f16_from_biased(prmt(n1, 0, 0x4342) * s1 + 0x64006400u);
#pragma unroll
                for (int q = 0; q < NTW; ++q) {
                    const uint2 b = bf[(st * nt8 + q) * 32];
                    mma_f16(acc[q], a0, a1, a2, a3, b.x, b.y);
                }
            }
        }
        const GemmRecord R{nt8};
        const int *ex = reinterpret_cast<const int *>(rec + R.exps_off());
        const float *sums = reinterpret_cast<const float *>(rec + R.sums_off());
        const float d0 = h2f(h0.x & 0xffffu), d1 = h2f(h1.x & 0xffffu);
        const float dm0 = h2f(h0.x >> 16), dm1 = h2f(h1.x >> 16);
        const uint32_t ml0 = h0.z & 0x3F3F3F3Fu, mh0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
        const uint32_t ml1 = h1.z & 0x3F3F3F3Fu, mh1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
#pragma unroll
        for (int q = 0; q < NTW; ++q) {
            const int tok = 4 * (tq0 + q) + t, E = ex[tok];
            const bool bad = E == kPrepNonFinite;
            const float f1 = bad ? __int_as_float(0x7fc00000) : pow2(-(E / 2)), f2 = bad ? 1.0f : pow2(-(E - E / 2));
            const float4 xa = *reinterpret_cast<const float4 *>(sums + tok * 8);
            const float4 xb = *reinterpret_cast<const float4 *>(sums + tok * 8 + 4);
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            float m0 = 0.0f, m1 = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                m0 = fmaf(static_cast<float>(sel6(ml0, mh0, j)), xv[j], m0);
                m1 = fmaf(static_cast<float>(sel6(ml1, mh1, j)), xv[j], m1);
            }
            tot[q][0] += ((acc[q][0] + acc[q][1]) * f1) * (f2 * d0) - dm0 * m0;
            tot[q][1] += ((acc[q][2] + acc[q][3]) * f1) * (f2 * d1) - dm1 * m1;
        }
    }
};

template <>
struct GemmFmt<FmtIQ1_S> {
    static constexpr int kChunkBytes = 50;
    // Selector table: entry i (the codebook row of index i), word hf (its
    // columns 4hf..4hf+3) at 8i + 4hf holds two 16-bit PRMT selectors, one
    // per column pair (c, c+1): n_c | 4 << 4 | n_{c+1} << 8 | 4 << 12 with
    // n = grid value + 1.  Against (byte table, 0x64646464) a selector yields
    // the f16 bit patterns 0x6400 | (8g +- 1 + 128) of both columns.
    static constexpr int kTableBytes = 2048 * 8;
    // Byte tables (8g +- 1) + 128 for n = g + 1 = 0, 1, 2: delta +1/8 and -1/8.
    static constexpr uint32_t kLutPlus = 0x00898179u, kLutMinus = 0x00877F77u;
    __device__ static void init_table(uint8_t *table, int tid, int nthreads) {
        const uint2 *grid = reinterpret_cast<const uint2 *>(g_codebooks + kTabIq1sGrid);
        for (int i = tid; i < 2048; i += nthreads) {
            const uint2 src = grid[i];
            uint32_t w[2];
#pragma unroll
            for (int hf = 0; hf < 2; ++hf) {
                const uint32_t word = hf ? src.y : src.x;
                uint32_t sel[2];
#pragma unroll
                for (int pp = 0; pp < 2; ++pp) {
                    const uint32_t na = static_cast<uint32_t>(s8(word >> (16 * pp)) + 1);
                    const uint32_t nb = static_cast<uint32_t>(s8(word >> (16 * pp + 8)) + 1);
                    sel[pp] = na | (4u << 4) | (nb << 8) | (4u << 12);
                }
                w[hf] = sel[0] | (sel[1] << 16);
            }
            *reinterpret_cast<uint2 *>(table + 8 * i) = make_uint2(w[0], w[1]);
        }
    }
    template <int NTW>
    __device__ __forceinline__ static void chunk(const uint8_t *r0, const uint8_t *r1, const uint8_t *rec, int nt8,
                                                 int tq0, int lane, uint32_t tab_s, float (&tot)[NTW][2]) {
        const int t = lane & 3;
        // groups (t/2) and 2 + (t/2) of each sub-block, half t%2 of the group
        const uint32_t gk0 = t >> 1, gk1 = 2 + (t >> 1);
        const uint32_t mask0 = 7u << (3 * gk0), mask1 = 7u << (3 * gk1);
        const uint32_t mul0 = c_gemm_iq1s_mul[gk0], mul1 = c_gemm_iq1s_mul[gk1];
        const uint32_t tabl = tab_s + 4u * (t & 1);
        const uint32_t k14 = 14u, k1 = 1u;
        const uint8_t *q0 = r0 + 2 + (t >> 1), *q1 = r1 + 2 + (t >> 1);
        const uint2 *bf = reinterpret_cast<const uint2 *>(rec) + tq0 * 32 + lane;
        float acc[NTW][4];
#pragma unroll
        for (int q = 0; q < NTW; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.0f;
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const uint32_t h0 = u16(r0 + 34 + 2 * s), h1 = u16(r1 + 34 + 2 * s);
            // delta sign (bit 15) picks the byte table
            const uint32_t l0 = kLutPlus + (h0 >> 15) * (kLutMinus - kLutPlus);
            const uint32_t l1 = kLutPlus + (h1 >> 15) * (kLutMinus - kLutPlus);
            // 2s+1 in both halves as f16, and -1152*(2s+1): the selected
            // patterns are 1152 + v, so fma(pattern, dl, -1152*dl) = dl*v exactly
            const uint32_t dl0 = f16_from_biased((and_or(h0 >> 11, k14, k1) | 0x6400u) * 0x10001u);
            const uint32_t dl1 = f16_from_biased((and_or(h1 >> 11, k14, k1) | 0x6400u) * 0x10001u);
            uint32_t nd0, nd1;
            asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(nd0) : "r"(dl0), "r"(0xE480E480u));  // -1152
            asm("mul.rn.f16x2 %0, %1, %2;" : "=r"(nd1) : "r"(dl1), "r"(0xE480E480u));
#pragma unroll
            for (int hs = 0; hs < 2; ++hs) {
                const int st = 2 * s + hs;
                const uint32_t mask = hs ? mask1 : mask0, mul = hs ? mul1 : mul0;
                const uint32_t e0 = lds32_const((h0 & mask) * mul + (q0[4 * s + 2 * hs] * 8u + tabl));
                const uint32_t e1 = lds32_const((h1 & mask) * mul + (q1[4 * s + 2 * hs] * 8u + tabl));
                const uint32_t a0 = hfma2(prmt(l0, 0x64646464u, e0), dl0, nd0);
                const uint32_t a2 = hfma2(prmt(l0, 0x64646464u, e0 >> 16), dl0, nd0);
                const uint32_t a1 = hfma2(prmt(l1, 0x64646464u, e1), dl1, nd1);
                const uint32_t a3 = hfma2(prmt(l1, 0x64646464u, e1 >> 16), dl1, nd1);
#pragma unroll
                for (int q = 0; q < NTW; ++q) {
                    const uint2 b = bf[(st * nt8 + q) * 32];
                    mma_f16(acc[q], a0, a1, a2, a3, b.x, b.y);
                }
            }
        }
        const GemmRecord R{nt8};
        const int *ex = reinterpret_cast<const int *>(rec + R.exps_off());
        const float d0 = h2f(u16(r0)) * 0.125f, d1 = h2f(u16(r1)) * 0.125f;
#pragma unroll
        for (int q = 0; q < NTW; ++q) {
            const int E = ex[4 * (tq0 + q) + t];
            const bool bad = E == kPrepNonFinite;
            const float f1 = bad ? __int_as_float(0x7fc00000) : pow2(-(E / 2)), f2 = bad ? 1.0f : pow2(-(E - E / 2));
            tot[q][0] += ((acc[q][0] + acc[q][1]) * f1) * (f2 * d0);
            tot[q][1] += ((acc[q][2] + acc[q][3]) * f1) * (f2 * d1);
        }
    }
};

// Signed int8 bytes of a word, pairs (0,1) and (2,3), to f16x2: the bytes
// biased by 128 go into the mantissa of 1024 (f16 0x64xx = 1024 + byte),
// one exact half2 subtraction of 1152 leaves q.
__device__ __forceinline__ uint32_t s8pair_to_f16x2(uint32_t biased_word, uint32_t sel) {
    uint32_t r;
    asm("sub.rn.f16x2 %0, %1, %2;" : "=r"(r) : "r"(prmt(biased_word, 0x64646464u, sel)), "r"(0x64806480u));
    return r;
}

template <>
struct GemmFmt<FmtQ8_0> {
    // Eight 34-byte blocks per 256 columns; A = q (int8, exact in f16), the
    // block scale d applied per 32 columns (two k16 steps) in f32.
    static constexpr int kChunkBytes = 8 * 34, kTableBytes = 0;
    __device__ static void init_table(uint8_t *, int, int) {}
    template <int NTW>
    __device__ __forceinline__ static void chunk(const uint8_t *r0, const uint8_t *r1, const uint8_t *rec, int nt8,
                                                 int tq0, int lane, uint32_t, float (&tot)[NTW][2]) {
        const int t = lane & 3;
        const uint2 *bf = reinterpret_cast<const uint2 *>(rec) + tq0 * 32 + lane;
        float ctot[NTW][2];
#pragma unroll
        for (int q = 0; q < NTW; ++q) ctot[q][0] = ctot[q][1] = 0.0f;
#pragma unroll
        for (int b = 0; b < 8; ++b) {
            float acc[NTW][4];
#pragma unroll
            for (int q = 0; q < NTW; ++q) acc[q][0] = acc[q][1] = acc[q][2] = acc[q][3] = 0.0f;
#pragma unroll
            for (int hs = 0; hs < 2; ++hs) {
                // bytes 4t..4t+3 of the block's 16-column half hs; a block at an
                // odd index starts 2 bytes past a 4-byte boundary, so its quant
                // bytes are aligned, an even one's straddle two words
                const int off = 34 * b + 2 + 16 * hs + 4 * t;
                uint32_t w0, w1;
                if (b & 1) {
                    w0 = lds32(r0 + off);
                    w1 = lds32(r1 + off);
                } else {
                    w0 = __funnelshift_r(lds32(r0 + off - 2), lds32(r0 + off + 2), 16);
                    w1 = __funnelshift_r(lds32(r1 + off - 2), lds32(r1 + off + 2), 16);
                }
                w0 ^= 0x80808080u;
                w1 ^= 0x80808080u;
                const uint32_t a0 = s8pair_to_f16x2(w0, 0x4140), a2 = s8pair_to_f16x2(w0, 0x4342);
                const uint32_t a1 = s8pair_to_f16x2(w1, 0x4140), a3 = s8pair_to_f16x2(w1, 0x4342);
                const int st = 2 * b + hs;
#pragma unroll
                for (int q = 0; q < NTW; ++q) {
                    const uint2 bb = bf[(st * nt8 + q) * 32];
                    mma_f16(acc[q], a0, a1, a2, a3, bb.x, bb.y);
                }
            }
            const float d0 = h2f(u16(r0 + 34 * b)), d1 = h2f(u16(r1 + 34 * b));
#pragma unroll
            for (int q = 0; q < NTW; ++q) {
                ctot[q][0] = fmaf(acc[q][0] + acc[q][1], d0, ctot[q][0]);
                ctot[q][1] = fmaf(acc[q][2] + acc[q][3], d1, ctot[q][1]);
            }
        }
        const GemmRecord R{nt8};
        const int *ex = reinterpret_cast<const int *>(rec + R.exps_off());
#pragma unroll
        for (int q = 0; q < NTW; ++q) {
            const int E = ex[4 * (tq0 + q) + t];
            const bool bad = E == kPrepNonFinite;
            const float f1 = bad ? __int_as_float(0x7fc00000) : pow2(-(E / 2)), f2 = bad ? 1.0f : pow2(-(E - E / 2));
            tot[q][0] += (ctot[q][0] * f1) * f2;
            tot[q][1] += (ctot[q][1] * f1) * f2;
        }
    }
};

// ----------------------------------------------------------------- kernel ---

template <class F, int NTW>
__global__ void __launch_bounds__(13 * 32, 1)
    gemm_f16_kernel(float *__restrict__ out, const uint8_t *__restrict__ w, const uint8_t *__restrict__ rec, int rows,
                    int cols, int T, int nt8, int row_bytes, int srow, int RG, int TG, int S, int nst,
                    int rec_stride, int a_bytes, int64_t pitch, int accumulate, int *err) {
    using GF = GemmFmt<F>;
    extern __shared__ __align__(128) uint8_t smem[];
    const int NW = RG * TG * S, R = 16 * RG, T4 = 4 * nt8;
    const int C = cols >> 8;
    const GemmRecord REC{nt8};
    uint8_t *atile = smem;
    uint8_t *ring = smem + a_bytes;
    uint8_t *table = ring + static_cast<size_t>(nst) * rec_stride;
    float *red = reinterpret_cast<float *>(table + GF::kTableBytes);  // [S][R][T4]
    uint64_t *full = reinterpret_cast<uint64_t *>(red + static_cast<size_t>(S) * R * T4);
    uint64_t *empty = full + nst;
    uint64_t *a_full = empty + nst, *a_empty = a_full + 1;
    volatile int *abort_flag = reinterpret_cast<volatile int *>(a_empty + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < nst; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], RG * TG);
        }
        mbar_init(a_full, 1);
        mbar_init(a_empty, NW);
        *abort_flag = 0;
        fence_mbar_init();
    }
    __syncthreads();
    allow_dependent_launch();
    const int r_begin = static_cast<int>(static_cast<int64_t>(rows) * blockIdx.x / gridDim.x);
    const int r_end = static_cast<int>(static_cast<int64_t>(rows) * (blockIdx.x + 1) / gridDim.x);

    if (warp == NW) {  // producer
        grid_dependency_wait();  // the prepared records come from the previous kernel
        int i = 0;
        for (int r0 = r_begin; r0 < r_end; r0 += R, ++i) {
            const int nr = min(R, r_end - r0);
            int ok = 1;
            if (lane == 0) ok = mbar_wait_bounded(a_empty, (i & 1) ^ 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) report_device_error(err, kDevErrEmptyWait);
                return;
            }
            if (lane == 0) mbar_arrive_expect_tx(a_full, static_cast<uint32_t>(nr) * row_bytes);
            __syncwarp();
            for (int r = lane; r < nr; r += 32)
                bulk_g2s(atile + static_cast<size_t>(r) * srow, w + static_cast<size_t>(r0 + r) * pitch, row_bytes,
                         a_full);
            for (int c = 0; c < C; ++c) {
                const int k = i * C + c, s = k % nst;
                if (lane == 0) {
                    if (!mbar_wait_bounded(&empty[s], ((k / nst) & 1) ^ 1)) {
                        report_device_error(err, kDevErrEmptyWait);
                        ok = 0;
                    } else {
                        mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(REC.bytes()));
                        bulk_g2s(ring + static_cast<size_t>(s) * rec_stride, rec + static_cast<size_t>(c) * REC.bytes(),
                                 static_cast<uint32_t>(REC.bytes()), &full[s]);
                    }
                }
                ok = __shfl_sync(0xffffffffu, ok, 0);
                if (!ok) return;
            }
        }
        return;
    }

    GF::init_table(table, threadIdx.x, NW * 32);
    named_barrier_sync(1, NW * 32);
    const uint32_t tab_s = smem_addr(table);
    const int sw = warp % S, tg = (warp / S) % TG, rg = warp / (S * TG);
    const int g = lane >> 2, t = lane & 3;
    const int tq0 = tg * NTW;
    int i = 0;
    for (int r0 = r_begin; r0 < r_end; r0 += R, ++i) {
        const int nr = min(R, r_end - r0);
        bool ok = mbar_wait_bounded(a_full, i & 1);
        float tot[NTW][2];
#pragma unroll
        for (int q = 0; q < NTW; ++q) tot[q][0] = tot[q][1] = 0.0f;
        const uint8_t *row0 = atile + static_cast<size_t>(16 * rg + g) * srow, *row1 = row0 + 8 * static_cast<size_t>(srow);
        for (int c = sw; c < C && ok; c += S) {
            const int k = i * C + c, s = k % nst;
            ok = mbar_wait_bounded(&full[s], (k / nst) & 1);
            if (!ok) break;
            GF::template chunk<NTW>(row0 + c * GF::kChunkBytes, row1 + c * GF::kChunkBytes,
                                    ring + static_cast<size_t>(s) * rec_stride, nt8, tq0, lane, tab_s, tot);
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        if (!ok) {
            if (lane == 0) report_device_error(err, kDevErrFullWait);
            *abort_flag = 1;
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(a_empty);
        // partial sums of this slice: red[sw][row][token]
#pragma unroll
        for (int q = 0; q < NTW; ++q) {
            const int tok = 4 * (tq0 + q) + t;
            red[(static_cast<size_t>(sw) * R + 16 * rg + g) * T4 + tok] = tot[q][0];
            red[(static_cast<size_t>(sw) * R + 16 * rg + g + 8) * T4 + tok] = tot[q][1];
        }
        named_barrier_sync(2, NW * 32);
        if (*abort_flag) break;
        for (int idx = threadIdx.x; idx < nr * T; idx += NW * 32) {  // token-major: coalesced rows
            const int tok = idx / nr, r = idx % nr;
            float v = 0.0f;
            for (int q = 0; q < S; ++q) v += red[(static_cast<size_t>(q) * R + r) * T4 + tok];
            float *d = out + static_cast<size_t>(tok) * rows + r0 + r;
            *d = accumulate ? *d + v : v;
        }
        named_barrier_sync(2, NW * 32);  // red is rewritten by the next tile
    }
}

// ------------------------------------------------------------------- host ---

namespace {

struct GemmPlan {
    int ntw = 0, nt8 = 0, TG = 0, RG = 0, S = 0, nst = 0, srow = 0, rec_stride = 0, a_bytes = 0, grid = 0;
    size_t smem = 0;
};

constexpr size_t kGemmSmemBudget = 226 * 1024;
constexpr int kGemmMaxWarps = 12;

// Plan for NTW 8-column tiles (4*NTW tokens) per warp; false if nothing fits.
template <class F>
bool plan_gemm_ntw(int ntw, int rows, int cols, int batch, int row_bytes, GemmPlan &p) {
    using GF = GemmFmt<F>;
    const int nt8 = (batch + 3) / 4;
    p.ntw = ntw;
    p.nt8 = (nt8 + ntw - 1) / ntw * ntw;
    p.TG = p.nt8 / ntw;
    if (p.TG > kGemmMaxWarps) return false;
    p.grid = std::max(1, std::min(sm_count(), (rows + 15) / 16));
    const int per_cta = (rows + p.grid - 1) / p.grid;
    p.srow = ((row_bytes >> 4) & 1) ? row_bytes : row_bytes + 16;
    p.RG = std::max(1, std::min((per_cta + 15) / 16, kGemmMaxWarps / p.TG));
    // Tiles of several row groups stay within 100 KB; a single 16-row tile
    // of long rows (Q8_0 at 6144 columns, Q4_K at 16384) may take more, as
    // long as the whole plan fits the budget (checked below).
    while (p.RG > 1 && static_cast<size_t>(16 * p.RG) * p.srow > 100 * 1024) --p.RG;
    const GemmRecord rec{p.nt8};
    p.rec_stride = static_cast<int>((rec.bytes() + 127) & ~size_t(127));
    p.a_bytes = static_cast<int>((static_cast<size_t>(16 * p.RG) * p.srow + 127) & ~size_t(127));
    const int C = cols / 256;
    for (int S = 8; S >= 1; S /= 2) {
        if (C % S || p.RG * p.TG * S > kGemmMaxWarps) continue;
        const size_t smem = static_cast<size_t>(p.a_bytes) + 2ull * S * p.rec_stride + GF::kTableBytes +
                            4ull * S * 16 * p.RG * 4 * p.nt8 + 8ull * (4 * S + 2) + 16;
        if (smem <= kGemmSmemBudget) {
            p.S = S;
            p.nst = 2 * S;
            p.smem = smem;
            return true;
        }
    }
    return false;
}

// The tile width that gives the most consumer warps (latency hiding for the
// dependent tensor-core steps), the wider one on a tie (fewer decodes).
template <class F>
bool plan_gemm(int rows, int cols, int batch, int row_bytes, GemmPlan &p) {
    const int nt8 = (batch + 3) / 4;
    bool found = false;
    for (int ntw = 8; ntw >= 2; ntw /= 2) {
        if (ntw > 2 && ntw / 2 >= nt8) continue;  // a narrower tile covers the batch
        GemmPlan c;
        if (!plan_gemm_ntw<F>(ntw, rows, cols, batch, row_bytes, c)) continue;
        if (!found || c.RG * c.TG * c.S > p.RG * p.TG * p.S) p = c;
        found = true;
    }
    return found;
}

template <class F, int NTW>
int32_t launch_gemm(const GemmPlan &p, float *out, const uint8_t *w, const uint8_t *rec, int rows, int cols, int batch,
                    int row_bytes, const ColSegment &seg, cudaStream_t stream) {
    auto kern = gemm_f16_kernel<F, NTW>;
    if (const int32_t rc = allow_dynamic_smem(kern, p.smem, "packed_gemm smem")) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3((p.RG * p.TG * p.S + 1) * 32);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    GLMVX_CUDA(cudaLaunchKernelEx(&cfg, kern, out, w, rec, rows, cols, batch, p.nt8, row_bytes, p.srow, p.RG, p.TG, p.S,
                                  p.nst, p.rec_stride, p.a_bytes, seg.pitch ? seg.pitch : row_bytes,
                                  static_cast<int>(seg.accumulate), device_error_word()));
    return kOk;
}

}  // namespace

bool gemm_f16_supported(int kind, int cols, int batch) {
    if (batch < kGemmMinTokens || batch > kGemmMaxTokens || cols <= 0 || cols % 256) return false;
    return kind == 12 || kind == 8 || (kind == 19 && cols % 2048 == 0);
}

int32_t gemm_f16_device(int32_t kind, float *out, const uint8_t *w, const float *x, int rows, int cols, int batch,
                        uint8_t *scratch, cudaStream_t stream, const ColSegment &seg) {
    if (!gemm_f16_supported(kind, cols, batch) || rows <= 0) {
        set_error("gemm: unsupported format or shape");
        return kUnsupported;
    }
    if ((reinterpret_cast<uintptr_t>(w) | reinterpret_cast<uintptr_t>(x) | reinterpret_cast<uintptr_t>(scratch)) & 15) {
        set_error("gemm: weights, activations and scratch must be 16-byte aligned");
        return kInvalid;
    }
    int blk = 0, bytes = 0;
    reference_layout(kind, blk, bytes);
    const int row_bytes = cols / blk * bytes;
    if ((seg.pitch && (seg.pitch < row_bytes || seg.pitch % 16)) || (seg.xstride && seg.xstride < cols)) {
        set_error("gemm: a column segment needs a 16-byte row pitch and strides >= its width");
        return kInvalid;
    }
    const int xstride = seg.xstride ? seg.xstride : cols;
    int32_t st = kUnsupported;
    dispatch_format(kind, [&]<class F>() {
        if constexpr (std::is_same_v<F, FmtQ4_K> || std::is_same_v<F, FmtIQ1_S> || std::is_same_v<F, FmtQ8_0>) {
            GemmPlan p;
            if (!plan_gemm<F>(rows, cols, batch, row_bytes, p)) {
                // Long rows with many tokens may not fit one CTA's shared
                // memory: run the batch as halves (the weights stream twice).
                if (batch >= 2 * kGemmMinTokens) {
                    const int h = (batch + 1) / 2;
                    st = gemm_f16_device(kind, out, w, x, rows, cols, h, scratch, stream, seg);
                    if (!st)
                        st = gemm_f16_device(kind, out + static_cast<size_t>(h) * rows, w,
                                             x + static_cast<size_t>(h) * xstride, rows, cols, batch - h, scratch,
                                             stream, seg);
                    return;
                }
                set_error("gemm: no launch plan for this shape");
                return;
            }
            const int T4 = 4 * p.nt8, chunks = cols / 256;
            const int64_t warps = static_cast<int64_t>(T4) * chunks;
            cudaLaunchConfig_t cfg = {};
            cfg.gridDim = dim3(static_cast<unsigned>((warps + 7) / 8));
            cfg.blockDim = dim3(256);
            cfg.stream = stream;
            cudaLaunchAttribute attr[1];
            attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
            attr[0].val.programmaticStreamSerializationAllowed = 1;
            cfg.attrs = attr;
            cfg.numAttrs = 1;
            const cudaError_t e = cudaLaunchKernelEx(&cfg, prep_f16_kernel, scratch, x, batch, T4, cols, p.nt8, xstride);
            if (e != cudaSuccess) {
                st = cuda_fail(e, "prep_f16_kernel");
                return;
            }
            switch (p.ntw) {
            case 2: st = launch_gemm<F, 2>(p, out, w, scratch, rows, cols, batch, row_bytes, seg, stream); break;
            case 4: st = launch_gemm<F, 4>(p, out, w, scratch, rows, cols, batch, row_bytes, seg, stream); break;
            default: st = launch_gemm<F, 8>(p, out, w, scratch, rows, cols, batch, row_bytes, seg, stream); break;
            }
        }
    });
    return st;
}

// Enough for any tile width the planner picks (tokens padded to 32).
size_t gemm_f16_scratch_bytes(int cols, int batch) {
    const GemmRecord rec{((batch + 3) / 4 + 7) / 8 * 8};
    return rec.bytes() * static_cast<size_t>(cols / 256);
}

}  // namespace glmvx
