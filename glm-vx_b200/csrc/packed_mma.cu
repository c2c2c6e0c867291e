// Packed-GGUF GEMV / small-batch GEMM on the sm_100a tensor cores (int8 mma).
//
// Same contract as the reference's fused dequantise+dot kernels
// (glm_vx_packed_<fmt>, kernels/packed.vx:154-470, and the batch_v2 forms,
// kernels/packed.vx:473ff): out[t][r] = sum_j w[r][j] * x[t][j] in f32 with
// the weights decoded per GGML block.  Here the decode stops at the block's
// integers and the multiply runs on the tensor cores:
//
//   Q8_0   w = d * q                      A = q (s8), per 32-column block
//   Q4_K   w = d*sc * q - dmin*m          A = q (u8, 0..15); the min term
//                                         dmin*m*sum(x) uses the prepared
//                                         sub-block sums of x
//   IQ1_S  w = d*(2s+1) * (grid + delta)  A = 8*grid +/- 1 (s8): a nibble
//                                         codebook in shared memory, expanded
//                                         with one byte permute (the sign of
//                                         delta picks the byte table); the
//                                         odd multiplier 2s+1 is applied to
//                                         the int32 result, d/8 in f32
//
// The activations come as prepared rows (mma_gemv.cuh): four int8 limbs of
// x*2^E.  One m16n8k32 instruction takes 16 weight rows x 32 columns against
// 8 columns = 2 tokens x 4 limbs, so each weight byte is decoded once for
// both tokens of a job and every product is exact; the four limb partial
// sums are recombined in f32 at the end of the tile.
//
// Thread/fragment layout (m16n8k32, A row-major, B column-major): lane
// (g = lane/4, t = lane%4) holds A rows g and g+8 and B column g, each for the
// logical k = 4t..4t+3 and 4t+16..4t+19.  Those eight logical k are mapped to
// the eight physical columns 8t..8t+7 of the 32-column sub-block, for A and B
// alike, so a lane's A bytes are the 8 consecutive weights its group holds in
// the GGML block and its B bytes are 8 consecutive limb bytes.
//
// Kernel structure (mma_rows_kernel): a persistent grid, one CTA per SM, each
// CTA owning a balanced range of the job list's rows.  A producer warp
// streams tiles of 16*RG rows into a ring of shared-memory stages with 1-D
// bulk copies (TMA): one per tile when the row length already spreads the 8
// row groups of a fragment over distinct banks, else one per row into padded
// rows; S*RG consumer warps each take
// 16 rows x 512 columns of a tile (S = cols/512 column slices, RG row
// groups; IQ1_S warps take two 16-row fragments for more independent work),
// keep the B fragments of their slice in registers, and reduce the S
// slice partials of a row in fixed order through shared memory after every
// tile.  Waits on mbarriers are bounded (2 s) and report through the device
// error word.
#include <algorithm>
#include <type_traits>

#include "codecs.cuh"
#include "mma_gemv.cuh"

namespace glmvx {

// ------------------------------------------------------------- fragments ---

__device__ __forceinline__ void mma_s8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.s8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

__device__ __forceinline__ void mma_u8s8(int (&c)[4], uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3, uint32_t b0,
                                         uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k32.row.col.s32.u8.s8.s32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%10,%10,%10,%10};"
        : "=r"(c[0]), "=r"(c[1]), "=r"(c[2]), "=r"(c[3])
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1), "r"(0));
}

// 2^e for e in [-126, 127], exactly.
__device__ __forceinline__ float pow2(int e) { return __int_as_float((127 + e) << 23); }

__device__ __forceinline__ uint32_t lds32(const uint8_t *p) { return *reinterpret_cast<const uint32_t *>(p); }
__device__ __forceinline__ uint2 lds64(const uint8_t *p) { return *reinterpret_cast<const uint2 *>(p); }

// Per-format work on one 256-column chunk (chunk C of the warp's column
// slice) of kFR 16-row fragments.  p[f][0]/p[f][1] point at rows g and g+8
// of fragment f at the slice start in shared memory, b[] are the slice's B
// fragments (NB sub-blocks), xs is the chunk's scale relative to the slice's
// largest-magnitude chunk (for this lane's accumulator token), sums the
// slice's sub-block activation sums, table this lane's view of the format's
// shared-memory table.  af[] are the f32 accumulators (rows g, g+8 x this
// lane's two limb columns), am[] the min-term accumulators of rows g, g+8.
template <class F>
struct MmaFmt;

// PRMT in its default mode.  CUDA's __byte_perm ignores bit 3 of each
// selector nibble, so for a selector only known at run time the compiler
// masks it first; the codebook nibbles here are 0..2 (bit 3 clear), where
// both agree, so the mask is not needed.
__device__ __forceinline__ uint32_t prmt(uint32_t a, uint32_t b, uint32_t sel) {
    uint32_t r;
    asm("prmt.b32 %0, %1, %2, %3;" : "=r"(r) : "r"(a), "r"(b), "r"(sel));
    return r;
}

// (a & b) | c as one LOP3 with all three operands in registers.
__device__ __forceinline__ uint32_t and_or(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t r;
    asm("lop3.b32 %0, %1, %2, %3, 0xEA;" : "=r"(r) : "r"(a), "r"(b), "r"(c));
    return r;
}

// 32-bit load from a shared-memory address held as a 32-bit integer (no
// generic-to-shared conversion per access).  Only for data that does not
// change while the kernel runs after its initial barrier (the codebook).
__device__ __forceinline__ uint32_t lds32_const(uint32_t addr) {
    uint32_t v;
    asm("ld.shared.u32 %0, [%1];" : "=r"(v) : "r"(addr));
    return v;
}

// 2^(12-3t): (qh & 7 << 3t) * c_iq1s_hi_mul[t] = 4096 * (grid bits of group
// t), the codebook offset of those bits, as one multiply-add.  Read from the
// constant bank so the compiler keeps the multiply-add instead of a shift.
__constant__ uint32_t c_iq1s_hi_mul[4] = {4096u, 512u, 64u, 8u};

template <>
struct MmaFmt<FmtIQ1_S> {
    // Codebook as 8 nibbles g+1 (0..2) per entry, four interleaved copies:
    // copy c of entry i at byte 16*i + 4*c.  Lane t of a quad reads copy t,
    // so the 32 lanes of a lookup fall in four disjoint groups of 8 banks.
    // (Eight copies, spreading also by row parity, measured no faster.)
    static constexpr int kTableBytes = 2048 * 16, kSubPerBlock = 8, kBlockBytes = 50;
    static constexpr bool kMins = false;
    // 16-row fragments per warp (independent work to hide latency); long job
    // lists take kFRLong (fewer, larger tiles), short ones kFR (balance).
    static constexpr int kFR = 2, kFRLong = 3;
    // Byte lookup words for PRMT: nibble n = g+1 selects 8*g+1 (delta = +1/8)
    // or 8*g-1 (delta = -1/8) as int8.
    static constexpr uint32_t kLutPlus = 0x000901F9u, kLutMinus = 0x0007FFF7u;
    __device__ static void init_table(uint8_t *table, int tid, int nthreads) {
        const uint2 *grid = reinterpret_cast<const uint2 *>(g_codebooks + kTabIq1sGrid);
        for (int i = tid; i < 2048; i += nthreads) {
            const uint2 src = grid[i];
            uint32_t v = 0;
#pragma unroll
            for (int k = 0; k < 4; ++k) {
                v |= (static_cast<uint32_t>(s8(src.x >> (8 * k)) + 1) & 0xfu) << (4 * k);
                v |= (static_cast<uint32_t>(s8(src.y >> (8 * k)) + 1) & 0xfu) << (4 * k + 16);
            }
            *reinterpret_cast<uint4 *>(table + 16 * i) = make_uint4(v, v, v, v);
        }
    }
    // This lane's copy of the codebook.
    __device__ static const uint8_t *table_for_lane(const uint8_t *table, int lane) { return table + 4 * (lane & 3); }
    template <int C, int NB, int FR>
    __device__ __forceinline__ static void chunk(const uint8_t *const (&p)[FR][2], int t, const uint32_t (&b)[NB][2],
                                                 float xs, const float *, const uint8_t *tab, float (&af)[FR][4],
                                                 float (&)[FR][2]) {
        const int sh = 3 * t;
        const uint32_t hmask = 7u << sh, hmul = c_iq1s_hi_mul[t];
        constexpr uint32_t step = kLutMinus - kLutPlus;
        const uint32_t k14 = 14u, k1 = 1u;
        const uint32_t tab_s = smem_addr(tab);
        const uint8_t *q[FR][2], *qt[FR][2];  // block C of rows g, g+8; its qs byte of group t
#pragma unroll
        for (int f = 0; f < FR; ++f)
#pragma unroll
            for (int r = 0; r < 2; ++r) {
                q[f][r] = p[f][r] + C * kBlockBytes;
                qt[f][r] = q[f][r] + 2 + t;
            }
        int ai[FR][4] = {};
#pragma unroll
        for (int s = 0; s < 8; ++s)
#pragma unroll
        for (int f = 0; f < FR; ++f) {
            const uint32_t h0 = u16(q[f][0] + 34 + 2 * s), h1 = u16(q[f][1] + 34 + 2 * s);
            // entry (grid bits 3t..3t+2 of h, qs) at 4096*bits + 16*qs: index
            // 256*bits + qs, the grid bits taken in place and scaled by a
            // multiply-add rather than shifted into position
            const uint32_t e0 = lds32_const((h0 & hmask) * hmul + (qt[f][0][4 * s] * 16u + tab_s));
            const uint32_t e1 = lds32_const((h1 & hmask) * hmul + (qt[f][1][4 * s] * 16u + tab_s));
            // delta sign (bit 15) picks the byte table: P + sign * (M - P).
            const uint32_t l0 = kLutPlus + (h0 >> 15) * step, l1 = kLutPlus + (h1 >> 15) * step;
            int c[4];
            // selector bits 16..31 are ignored: e for bytes 0..3, e >> 16 for 4..7
            mma_s8s8(c, prmt(l0, 0, e0), prmt(l1, 0, e1), prmt(l0, 0, __umulhi(e0, 65536u)),
                     prmt(l1, 0, __umulhi(e1, 65536u)), b[8 * C + s][0], b[8 * C + s][1]);
            // 2s+1 from bits 12..14: ((h >> 11) & 14) | 1, one LOP3 with
            // both constants in registers.
            const int dl0 = static_cast<int>(and_or(h0 >> 11, k14, k1));
            const int dl1 = static_cast<int>(and_or(h1 >> 11, k14, k1));
            ai[f][0] += dl0 * c[0];
            ai[f][1] += dl0 * c[1];
            ai[f][2] += dl1 * c[2];
            ai[f][3] += dl1 * c[3];
        }
#pragma unroll
        for (int f = 0; f < FR; ++f) {
            const float s0 = h2f(u16(p[f][0] + C * kBlockBytes)) * (0.125f * xs);
            const float s1 = h2f(u16(p[f][1] + C * kBlockBytes)) * (0.125f * xs);
            af[f][0] = fmaf(s0, static_cast<float>(ai[f][0]), af[f][0]);
            af[f][1] = fmaf(s0, static_cast<float>(ai[f][1]), af[f][1]);
            af[f][2] = fmaf(s1, static_cast<float>(ai[f][2]), af[f][2]);
            af[f][3] = fmaf(s1, static_cast<float>(ai[f][3]), af[f][3]);
        }
    }
    // Two token pairs per job, one 16-row fragment (rows g, g+8 of p[0]):
    // each decoded fragment feeds two MMAs.  Same arithmetic per pair as
    // chunk(), so a token's result does not depend on the job it lands in.
    template <int C, int NB>
    __device__ __forceinline__ static void chunk2(const uint8_t *const (&p)[1][2], int t,
                                                  const uint32_t (&b)[2][NB][2], float xs0, float xs1,
                                                  const uint8_t *tab, float (&af)[2][1][4]) {
        const int sh = 3 * t;
        const uint32_t hmask = 7u << sh, hmul = c_iq1s_hi_mul[t];
        constexpr uint32_t step = kLutMinus - kLutPlus;
        const uint32_t k14 = 14u, k1 = 1u;
        const uint32_t tab_s = smem_addr(tab);
        const uint8_t *q0 = p[0][0] + C * kBlockBytes, *q1 = p[0][1] + C * kBlockBytes;
        const uint8_t *qt0 = q0 + 2 + t, *qt1 = q1 + 2 + t;
        int ai[2][4] = {};
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const uint32_t h0 = u16(q0 + 34 + 2 * s), h1 = u16(q1 + 34 + 2 * s);
            const uint32_t e0 = lds32_const((h0 & hmask) * hmul + (qt0[4 * s] * 16u + tab_s));
            const uint32_t e1 = lds32_const((h1 & hmask) * hmul + (qt1[4 * s] * 16u + tab_s));
            const uint32_t l0 = kLutPlus + (h0 >> 15) * step, l1 = kLutPlus + (h1 >> 15) * step;
            const uint32_t a0 = prmt(l0, 0, e0), a1 = prmt(l1, 0, e1);
            const uint32_t a2 = prmt(l0, 0, __umulhi(e0, 65536u)), a3 = prmt(l1, 0, __umulhi(e1, 65536u));
            const int dl0 = static_cast<int>(and_or(h0 >> 11, k14, k1));
            const int dl1 = static_cast<int>(and_or(h1 >> 11, k14, k1));
#pragma unroll
            for (int q = 0; q < 2; ++q) {
                int c[4];
                mma_s8s8(c, a0, a1, a2, a3, b[q][8 * C + s][0], b[q][8 * C + s][1]);
                ai[q][0] += dl0 * c[0];
                ai[q][1] += dl0 * c[1];
                ai[q][2] += dl1 * c[2];
                ai[q][3] += dl1 * c[3];
            }
        }
        const float d0 = h2f(u16(q0)), d1 = h2f(u16(q1));
#pragma unroll
        for (int q = 0; q < 2; ++q) {
            const float xq = q ? xs1 : xs0;
            const float s0 = d0 * (0.125f * xq), s1 = d1 * (0.125f * xq);
            af[q][0][0] = fmaf(s0, static_cast<float>(ai[q][0]), af[q][0][0]);
            af[q][0][1] = fmaf(s0, static_cast<float>(ai[q][1]), af[q][0][1]);
            af[q][0][2] = fmaf(s1, static_cast<float>(ai[q][2]), af[q][0][2]);
            af[q][0][3] = fmaf(s1, static_cast<float>(ai[q][3]), af[q][0][3]);
        }
    }
};

template <>
struct MmaFmt<FmtQ8_0> {
    static constexpr int kTableBytes = 0, kSubPerBlock = 1, kBlockBytes = 34;
    static constexpr bool kMins = false;
    static constexpr int kFR = 1;
    __device__ static void init_table(uint8_t *, int, int) {}
    __device__ static const uint8_t *table_for_lane(const uint8_t *table, int) { return table; }
    // Eight 34-byte blocks.  A block at an even index within the slice starts
    // 4-byte aligned (its bytes follow a 2-byte scale), one at an odd index
    // 2 bytes past alignment, so its bytes are.
    template <int C, int NB, int FR>
    __device__ __forceinline__ static void chunk(const uint8_t *const (&p)[FR][2], int t, const uint32_t (&b)[NB][2],
                                                 float xs, const float *, const uint8_t *, float (&afr)[FR][4],
                                                 float (&)[FR][2]) {
        static_assert(FR == 1, "one 16-row fragment per warp");
        const uint8_t *p0 = p[0][0], *p1 = p[0][1];
        float(&af)[4] = afr[0];
#pragma unroll
        for (int s = 0; s < 8; ++s) {
            const int i = 8 * C + s;
            const uint8_t *q0 = p0 + i * kBlockBytes, *q1 = p1 + i * kBlockBytes;
            uint32_t a0, a1, a2, a3;
            if ((i & 1) == 0) {
                const uint32_t w0 = lds32(q0 + 8 * t), w1 = lds32(q0 + 8 * t + 4), w2 = lds32(q0 + 8 * t + 8);
                const uint32_t v0 = lds32(q1 + 8 * t), v1 = lds32(q1 + 8 * t + 4), v2 = lds32(q1 + 8 * t + 8);
                a0 = __funnelshift_r(w0, w1, 16);
                a2 = __funnelshift_r(w1, w2, 16);
                a1 = __funnelshift_r(v0, v1, 16);
                a3 = __funnelshift_r(v1, v2, 16);
            } else {
                a0 = lds32(q0 + 2 + 8 * t);
                a2 = lds32(q0 + 6 + 8 * t);
                a1 = lds32(q1 + 2 + 8 * t);
                a3 = lds32(q1 + 6 + 8 * t);
            }
            int c[4];
            mma_s8s8(c, a0, a1, a2, a3, b[i][0], b[i][1]);
            const float s0 = h2f(u16(q0)) * xs, s1 = h2f(u16(q1)) * xs;
            af[0] = fmaf(s0, static_cast<float>(c[0]), af[0]);
            af[1] = fmaf(s0, static_cast<float>(c[1]), af[1]);
            af[2] = fmaf(s1, static_cast<float>(c[2]), af[2]);
            af[3] = fmaf(s1, static_cast<float>(c[3]), af[3]);
        }
    }
};

template <>
struct MmaFmt<FmtQ4_K> {
    static constexpr int kTableBytes = 0, kSubPerBlock = 8, kBlockBytes = 144;
    static constexpr bool kMins = true;
    static constexpr int kFR = 1;
    __device__ static void init_table(uint8_t *, int, int) {}
    __device__ static const uint8_t *table_for_lane(const uint8_t *table, int) { return table; }
    // Byte j of the 6-bit scale (or min) words of a K-quant head, sub-blocks
    // 0..3 in `lo`, 4..7 in `hi` (kernels/packed.vx:107-120 on packed words).
    __device__ __forceinline__ static int sel6(uint32_t lo, uint32_t hi, int j) {
        return static_cast<int>(((j < 4 ? lo : hi) >> (8 * (j & 3))) & 0xffu);
    }
    template <int C, int NB, int FR>
    __device__ __forceinline__ static void chunk(const uint8_t *const (&p)[FR][2], int t, const uint32_t (&b)[NB][2],
                                                 float xs, const float *sums, const uint8_t *, float (&afr)[FR][4],
                                                 float (&amr)[FR][2]) {
        static_assert(FR == 1, "one 16-row fragment per warp");
        float(&af)[4] = afr[0];
        float(&am)[2] = amr[0];
        const uint8_t *q0 = p[0][0] + C * kBlockBytes, *q1 = p[0][1] + C * kBlockBytes;
        const uint4 h0 = *reinterpret_cast<const uint4 *>(q0), h1 = *reinterpret_cast<const uint4 *>(q1);
        const uint32_t sl0 = h0.y & 0x3F3F3F3Fu, sh0 = (h0.w & 0x0F0F0F0Fu) | ((h0.y >> 2) & 0x30303030u);
        const uint32_t sl1 = h1.y & 0x3F3F3F3Fu, sh1 = (h1.w & 0x0F0F0F0Fu) | ((h1.y >> 2) & 0x30303030u);
        int ai[4] = {0, 0, 0, 0};
#pragma unroll
        for (int m = 0; m < 4; ++m) {
            const uint2 w0 = lds64(q0 + 16 + 32 * m + 8 * t), w1 = lds64(q1 + 16 + 32 * m + 8 * t);
            int c[4];
            mma_u8s8(c, w0.x & 0x0F0F0F0Fu, w1.x & 0x0F0F0F0Fu, w0.y & 0x0F0F0F0Fu, w1.y & 0x0F0F0F0Fu,
                     b[8 * C + 2 * m][0], b[8 * C + 2 * m][1]);
            int sc0 = sel6(sl0, sh0, 2 * m), sc1 = sel6(sl1, sh1, 2 * m);
            ai[0] += sc0 * c[0];
            ai[1] += sc0 * c[1];
            ai[2] += sc1 * c[2];
            ai[3] += sc1 * c[3];
            mma_u8s8(c, (w0.x >> 4) & 0x0F0F0F0Fu, (w1.x >> 4) & 0x0F0F0F0Fu, (w0.y >> 4) & 0x0F0F0F0Fu,
                     (w1.y >> 4) & 0x0F0F0F0Fu, b[8 * C + 2 * m + 1][0], b[8 * C + 2 * m + 1][1]);
            sc0 = sel6(sl0, sh0, 2 * m + 1);
            sc1 = sel6(sl1, sh1, 2 * m + 1);
            ai[0] += sc0 * c[0];
            ai[1] += sc0 * c[1];
            ai[2] += sc1 * c[2];
            ai[3] += sc1 * c[3];
        }
        const float s0 = h2f(h0.x & 0xffffu) * xs, s1 = h2f(h1.x & 0xffffu) * xs;
        af[0] = fmaf(s0, static_cast<float>(ai[0]), af[0]);
        af[1] = fmaf(s0, static_cast<float>(ai[1]), af[1]);
        af[2] = fmaf(s1, static_cast<float>(ai[2]), af[2]);
        af[3] = fmaf(s1, static_cast<float>(ai[3]), af[3]);
        if (sums) {
            const uint32_t ml0 = h0.z & 0x3F3F3F3Fu, mh0 = ((h0.w >> 4) & 0x0F0F0F0Fu) | ((h0.z >> 2) & 0x30303030u);
            const uint32_t ml1 = h1.z & 0x3F3F3F3Fu, mh1 = ((h1.w >> 4) & 0x0F0F0F0Fu) | ((h1.z >> 2) & 0x30303030u);
            // generic loads: the sums live in global or (fused preparation) shared memory
            const float4 xa = *reinterpret_cast<const float4 *>(sums + 8 * C);
            const float4 xb = *(reinterpret_cast<const float4 *>(sums + 8 * C) + 1);
            const float xv[8] = {xa.x, xa.y, xa.z, xa.w, xb.x, xb.y, xb.z, xb.w};
            float m0 = 0.0f, m1 = 0.0f;
#pragma unroll
            for (int j = 0; j < 8; ++j) {
                m0 = fmaf(static_cast<float>(sel6(ml0, mh0, j)), xv[j], m0);
                m1 = fmaf(static_cast<float>(sel6(ml1, mh1, j)), xv[j], m1);
            }
            am[0] = fmaf(h2f(h0.x >> 16), m0, am[0]);
            am[1] = fmaf(h2f(h1.x >> 16), m1, am[1]);
        }
    }
};

// --------------------------------------------------------------- prepare ---

// One warp prepares one 256-column chunk of one activation row (8 columns
// per lane): x (or SwiGLU(x, x2)) -> four int8 limb planes, the chunk's
// exponent and its 32-column sums, into the prepared row at `out`.
__device__ __forceinline__ void prep_chunk(uint8_t *out, const float *x, const float *x2, int cols, int chunk,
                                           int lane) {
    const int c0 = chunk * 256 + lane * 8;
    const float4 *xr = reinterpret_cast<const float4 *>(x + c0);
    float4 lo = __ldg(xr), hi = __ldg(xr + 1);
    if (x2) {
        const float4 *ur = reinterpret_cast<const float4 *>(x2 + c0);
        const float4 ulo = __ldg(ur), uhi = __ldg(ur + 1);
        lo = make_float4(silu_mul(lo.x, ulo.x), silu_mul(lo.y, ulo.y), silu_mul(lo.z, ulo.z), silu_mul(lo.w, ulo.w));
        hi = make_float4(silu_mul(hi.x, uhi.x), silu_mul(hi.y, uhi.y), silu_mul(hi.z, uhi.z), silu_mul(hi.w, uhi.w));
    }
    const float v[8] = {lo.x, lo.y, lo.z, lo.w, hi.x, hi.y, hi.z, hi.w};
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
    // 2^E puts the chunk's largest magnitude in [2^29, 2^30) (below 2^30 for
    // subnormal maxima, E = 156); applied as two exact power-of-two factors.
    const int ebits = (__float_as_int(mx) >> 23) & 0xff;
    const int E = mx == 0.0f ? 0 : 156 - ebits;
    const float up0 = pow2(E / 2), up1 = pow2(E - E / 2);
    uint32_t qq[8];
#pragma unroll
    for (int i = 0; i < 8; ++i)
        qq[i] = static_cast<uint32_t>(__float2int_rn(finite ? (v[i] * up0) * up1 : 0.0f)) + 0x808080u;
    // Balanced base-256 digits: the low three bytes of q + 0x808080 are
    // digit + 128, the top byte is the (signed) top digit.
#pragma unroll
    for (int l = 0; l < 4; ++l) {
        const int p = 3 - l;  // byte position of limb l
        const uint32_t sel = static_cast<uint32_t>(p | ((p + 4) << 4));
        const uint32_t flip = l ? 0x80808080u : 0u;
        const uint32_t w0 = __byte_perm(__byte_perm(qq[0], qq[1], sel), __byte_perm(qq[2], qq[3], sel), 0x5410) ^ flip;
        const uint32_t w1 = __byte_perm(__byte_perm(qq[4], qq[5], sel), __byte_perm(qq[6], qq[7], sel), 0x5410) ^ flip;
        *reinterpret_cast<uint2 *>(out + static_cast<size_t>(l) * cols + c0) = make_uint2(w0, w1);
    }
    float sum = ((v[0] + v[1]) + (v[2] + v[3])) + ((v[4] + v[5]) + (v[6] + v[7]));
    sum += __shfl_xor_sync(0xffffffffu, sum, 1);
    sum += __shfl_xor_sync(0xffffffffu, sum, 2);
    if ((lane & 3) == 0) reinterpret_cast<float *>(out + prep_sums_offset(cols))[c0 / 32] = sum;
    if (lane == 0) reinterpret_cast<int *>(out + prep_scale_offset(cols))[chunk] = finite ? E : kPrepNonFinite;
}

// One warp per (row, 256-column chunk).
__global__ void __launch_bounds__(256)
    prep_rows_kernel(uint8_t *__restrict__ prep, const float *__restrict__ x, const float *__restrict__ x2, int rows,
                     int cols, const int *rows_dev, int xstride) {
    grid_dependency_wait();
    allow_dependent_launch();
    if (rows_dev) rows = min(max(*rows_dev, 0), rows);
    const int chunks = cols >> 8;
    const int64_t wid = (static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x) >> 5;
    const int lane = threadIdx.x & 31;
    if (wid >= static_cast<int64_t>(rows) * chunks) return;  // warp-uniform
    const int row = static_cast<int>(wid / chunks), chunk = static_cast<int>(wid % chunks);
    prep_chunk(prep + static_cast<size_t>(row) * prep_stride(cols), x + static_cast<size_t>(row) * xstride,
               x2 ? x2 + static_cast<size_t>(row) * xstride : nullptr, cols, chunk, lane);
}

// ----------------------------------------------------------------- kernel ---

// a[i] for a run-time i with constant-index reads (a dynamic index would
// place the whole array in local memory).
template <int N, class T>
__device__ __forceinline__ T pick(const T (&a)[N], int i) {
    T r = a[0];
#pragma unroll
    for (int c = 1; c < N; ++c)
        if (i == c) r = a[c];
    return r;
}

__device__ __forceinline__ MmaJob job_at(const MmaJob &job0, const MmaJob *jobs, int j, int batch, int rows_per_job,
                                         size_t pstride) {
    if (jobs) return jobs[j];
    MmaJob r{};
    r.w = job0.w;
#pragma unroll
    for (int s = 0; s < 2; ++s) {
        const int tok = 2 * j + s;
        const bool on = tok < batch;
        r.xp[s] = on ? job0.xp[0] + static_cast<size_t>(tok) * pstride : nullptr;
        r.out[s] = on ? job0.out[0] + static_cast<size_t>(tok) * rows_per_job : nullptr;
    }
    return r;
}

// W = 256-column chunks per warp column slice (1 or 2); NT = token pairs
// per job (2: each decoded fragment is multiplied into two pairs, one 16-row
// fragment per warp; job lists of IQ1_S only); FR = 16-row fragments per warp.
template <class F, int S, int RG, int W, int NT, int FR>
__global__ void __launch_bounds__((S * RG + 1) * 32, 1)
    mma_rows_kernel(MmaJob job0, const MmaJob *__restrict__ jobs, const int *njobs_dev, int max_jobs, int batch,
                    int rows_per_job, int cols, int row_bytes, int srow, int stages, int stage_stride,
                    const float *__restrict__ x_raw, int64_t pitch, int xstride, int accumulate, int *err) {
    using MF = MmaFmt<F>;
    constexpr int NS = 2 * NT;                      // token slots per job
    constexpr int NW = S * RG, R = 16 * FR * RG;  // a warp owns FR 16-row fragments of the tile
    extern __shared__ __align__(128) uint8_t smem[];
    const size_t pstride = prep_stride(cols);
    // x_raw set (single matrix, `batch` token rows of f32): the CTA prepares
    // the two rows of each job it reaches into `bsm` itself.
    uint8_t *bsm = smem + static_cast<size_t>(stages) * stage_stride;
    uint8_t *table = bsm + (x_raw ? 2 * pstride : 0);
    float *red = reinterpret_cast<float *>(table + MF::kTableBytes);  // [2][R][S][NS]
    uint64_t *full = reinterpret_cast<uint64_t *>(red + 2 * R * S * NS);
    uint64_t *empty = full + stages;
    uint64_t *jobbar = empty + stages;  // consumer warps meet here around a job's preparation
    volatile int *abort_flag = reinterpret_cast<volatile int *>(jobbar + 1);  // [RG]
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], NW);
        }
        mbar_init(jobbar, NW);
        for (int i = 0; i < RG; ++i) abort_flag[i] = 0;
        fence_mbar_init();
    }
    __syncthreads();
    allow_dependent_launch();

    // The job count and, for device-built lists, the descriptors come from
    // the previous kernel: read them only after the grid dependency.
    auto range = [&](int &r_begin, int &r_end) {
        int nj = max_jobs;
        if (njobs_dev) nj = min(max(*njobs_dev, 0), max_jobs);
        const int64_t rows = static_cast<int64_t>(rows_per_job) * nj;
        r_begin = static_cast<int>(rows * blockIdx.x / gridDim.x);
        r_end = static_cast<int>(rows * (blockIdx.x + 1) / gridDim.x);
    };
    auto tile_end = [&](int r0, int r_end) {
        return min(min(r0 + R, r_end), (r0 / rows_per_job + 1) * rows_per_job);
    };

    if (warp == NW) {  // producer: one bulk copy per row, issued by the 32 lanes
        if (jobs) grid_dependency_wait();
        int r_begin, r_end;
        range(r_begin, r_end);
        int k = 0;
        for (int r0 = r_begin; r0 < r_end; r0 = tile_end(r0, r_end), ++k) {
            const int s = k % stages;
            int ok = 1;
            if (lane == 0) ok = mbar_wait_bounded(&empty[s], ((k / stages) & 1) ^ 1);
            ok = __shfl_sync(0xffffffffu, ok, 0);
            if (!ok) {
                if (lane == 0) report_device_error(err, kDevErrEmptyWait);
                break;
            }
            const int nr = tile_end(r0, r_end) - r0;
            const MmaJob j = job_at(job0, jobs, r0 / rows_per_job, batch, rows_per_job, pstride);
            uint8_t *stage = smem + static_cast<size_t>(s) * stage_stride;
            const uint8_t *src = j.w + static_cast<size_t>(r0 % rows_per_job) * pitch;
            if (srow == row_bytes && pitch == row_bytes) {  // rows already bank-spread: one contiguous copy
                if (lane == 0) {
                    mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(nr) * row_bytes);
                    bulk_g2s(stage, src, static_cast<uint32_t>(nr) * row_bytes, &full[s]);
                }
            } else {
                if (lane == 0) mbar_arrive_expect_tx(&full[s], static_cast<uint32_t>(nr) * row_bytes);
                __syncwarp();
                for (int i = lane; i < nr; i += 32)
                    bulk_g2s(stage + static_cast<size_t>(i) * srow, src + static_cast<size_t>(i) * pitch, row_bytes,
                             &full[s]);
            }
        }
        return;
    }

    MF::init_table(table, threadIdx.x, NW * 32);
    grid_dependency_wait();  // prepared activations come from the previous kernel
    int r_begin, r_end;
    range(r_begin, r_end);
    if (MF::kTableBytes) named_barrier_sync(1, NW * 32);

    const int sw = warp % S, rg = warp / S;
    const int g = lane >> 2, t = lane & 3;
    const uint8_t *ltab = MF::table_for_lane(table, lane);
    constexpr int SUB = 8 * W;  // 32-column sub-blocks per slice
    const int u0 = sw * SUB;    // first sub-block of the slice
    const size_t slice_off = static_cast<size_t>(u0 / MF::kSubPerBlock) * MF::kBlockBytes;
    const size_t scale_off = prep_scale_offset(cols), sums_off = prep_sums_offset(cols);
    uint32_t b[NT][SUB][2];
    float xs[NT][W] = {}, down[NT][2] = {};
    const float *sums[NT] = {};
    MmaJob J{};
    int loaded = -1;
    uint32_t jb_phase = 0;
    // Every consumer warp arrives; false if the others did not arrive in time.
    auto job_sync = [&]() -> bool {
        __syncwarp();
        if (lane == 0) mbar_arrive(jobbar);
        const bool ok = mbar_wait_bounded(jobbar, jb_phase & 1);
        ++jb_phase;
        return __all_sync(0xffffffffu, ok);
    };
    int k = 0;
    for (int r0 = r_begin; r0 < r_end; r0 = tile_end(r0, r_end), ++k) {
        const int job = r0 / rows_per_job;
        if (job != loaded) {  // uniform across the CTA
            loaded = job;
            J = job_at(job0, jobs, job, batch, rows_per_job, pstride);
            if (x_raw) {
                // The previous job's rows are in use until every warp is here.
                if (!job_sync()) {
                    if (lane == 0) report_device_error(err, kDevErrFullWait);
                    break;
                }
                const int chunks = cols >> 8;
                for (int c = warp; c < 2 * chunks; c += NW) {
                    const int slot = c / chunks, tok = 2 * job + slot;
                    if (tok < batch)
                        prep_chunk(bsm + slot * pstride, x_raw + static_cast<size_t>(tok) * xstride, nullptr, cols,
                                   c % chunks, lane);
                }
                if (!job_sync()) {
                    if (lane == 0) report_device_error(err, kDevErrFullWait);
                    break;
                }
                J.xp[0] = bsm;
                J.xp[1] = 2 * job + 1 < batch ? bsm + pstride : nullptr;
            }
#pragma unroll
            for (int q = 0; q < NT; ++q) {
                // pair q: B column g is token slot 2q + g/4, limb g%4
                const uint8_t *xb = pick(J.xp, 2 * q + (g >> 2));
#pragma unroll
                for (int u = 0; u < SUB; ++u) {
                    uint2 v = make_uint2(0u, 0u);
                    if (xb)
                        v = *reinterpret_cast<const uint2 *>(xb + static_cast<size_t>(g & 3) * cols + 32 * (u0 + u) +
                                                             8 * t);
                    b[q][u][0] = v.x;
                    b[q][u][1] = v.y;
                }
                // accumulator columns 2t, 2t+1: token slot 2q + t/2
                const uint8_t *xa = pick(J.xp, 2 * q + (t >> 1));
                // Chunk c holds x*2^E_c.  Relative to Eref = min over the slice's
                // chunks (the one of largest magnitude) its scale is 2^(Eref - E_c)
                // <= 1; the absolute 2^-Eref is applied once per tile in two exact
                // steps.  A chunk more than 2^126 below another contributes nothing.
                int e[W];
                bool bad = false;
#pragma unroll
                for (int c = 0; c < W; ++c) {
                    e[c] = xa ? reinterpret_cast<const int *>(xa + scale_off)[u0 / 8 + c] : 0;
                    bad |= e[c] == kPrepNonFinite;
                }
                int eref = e[0];
#pragma unroll
                for (int c = 1; c < W; ++c) eref = min(eref, e[c]);
                if (bad) eref = 0;
#pragma unroll
                for (int c = 0; c < W; ++c)
                    xs[q][c] = (xa && !bad && eref - e[c] >= -126) ? pow2(eref - e[c]) : 0.0f;
                down[q][0] = bad ? __int_as_float(0x7fc00000) : pow2(-(eref / 2));
                down[q][1] = pow2(-(eref - eref / 2));
                sums[q] = (MF::kMins && xa) ? reinterpret_cast<const float *>(xa + sums_off) + u0 : nullptr;
            }
        }
        const int s = k % stages;
        const bool ok = mbar_wait_bounded(&full[s], (k / stages) & 1);
        if (!ok) {
            if (lane == 0) report_device_error(err, kDevErrFullWait);
            abort_flag[rg] = 1;
        }
        const int nr = tile_end(r0, r_end) - r0;
        float af[NT][FR][4] = {}, am[NT][FR][2] = {};
        const int rbase = 16 * FR * rg;  // first tile row of this warp's fragments
        if (ok) {
            const uint8_t *p[FR][2];
#pragma unroll
            for (int f = 0; f < FR; ++f) {
                p[f][0] = smem + static_cast<size_t>(s) * stage_stride + static_cast<size_t>(rbase + 16 * f + g) * srow +
                          slice_off;
                p[f][1] = p[f][0] + 8 * static_cast<size_t>(srow);
            }
            if constexpr (NT == 1) {
                MF::template chunk<0>(p, t, b[0], xs[0][0], sums[0], ltab, af[0], am[0]);
                if constexpr (W == 2) MF::template chunk<1>(p, t, b[0], xs[0][W - 1], sums[0], ltab, af[0], am[0]);
            } else {
                MF::template chunk2<0>(p, t, b, xs[0][0], xs[1][0], ltab, af);
                if constexpr (W == 2) MF::template chunk2<1>(p, t, b, xs[0][W - 1], xs[1][W - 1], ltab, af);
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&empty[s]);
        }
        // Recombine the limbs: lanes with even t hold limbs 0,1 (x 2^24, 2^16)
        // and subtract the min term, odd t limbs 2,3 (x 2^8, 1).
        const float whi = (t & 1) ? 256.0f : 16777216.0f, wlo = (t & 1) ? 1.0f : 65536.0f;
        float *rb = red + static_cast<size_t>(k & 1) * R * S * NS;
#pragma unroll
        for (int q = 0; q < NT; ++q)
#pragma unroll
        for (int f = 0; f < FR; ++f) {
            float v0 = fmaf(af[q][f][0], whi, af[q][f][1] * wlo) * down[q][0] * down[q][1];
            float v1 = fmaf(af[q][f][2], whi, af[q][f][3] * wlo) * down[q][0] * down[q][1];
            if (MF::kMins && !(t & 1)) {
                v0 -= am[q][f][0];
                v1 -= am[q][f][1];
            }
            v0 += __shfl_xor_sync(0xffffffffu, v0, 1);
            v1 += __shfl_xor_sync(0xffffffffu, v1, 1);
            if (!(t & 1)) {
                rb[((rbase + 16 * f + g) * S + sw) * NS + 2 * q + (t >> 1)] = v0;
                rb[((rbase + 16 * f + g + 8) * S + sw) * NS + 2 * q + (t >> 1)] = v1;
            }
        }
        named_barrier_sync(2 + rg, S * 32);
        if (abort_flag[rg]) break;
        if (sw == 0) {  // 16*FR rows x NS tokens: S partials each, in fixed order
#pragma unroll
            for (int o2 = lane; o2 < 16 * FR * NS; o2 += 32) {
                const int i = rbase + o2 / NS, slot = o2 % NS;
                float v = 0.0f;
#pragma unroll
                for (int q = 0; q < S; ++q) v += rb[(i * S + q) * NS + slot];
                float *o = pick(J.out, slot);
                if (i < nr && o) {
                    float *d = o + (r0 + i) % rows_per_job;
                    *d = accumulate ? *d + v : v;
                }
            }
        }
    }
}

// ------------------------------------------------------------------- host ---

struct MmaPlan {
    int S = 0, RG = 0, W = 0, FR = 0, srow = 0, stages = 0, stage_stride = 0, grid = 0;
    size_t smem = 0;
};

// Below the 227 KB opt-in limit of dynamic shared memory per block.
constexpr size_t kMmaSmemBudget = 226 * 1024;

// Row groups per CTA for S column slices of W chunks: about twelve consumer
// warps with 512-column slices, twenty-four with 256-column ones (half the
// B fragments per warp leave room for twice the warps).
constexpr int mma_row_groups(int S, int W) {
    return W == 2 ? (S >= 12 ? 1 : 12 / S) : (S >= 24 ? 1 : 24 / S);
}

constexpr bool mma_slices_ok(int S, int W) {
    if (W == 2) return S == 1 || S == 2 || S == 3 || S == 4 || S == 6 || S == 8 || S == 12 || S == 16;
    return S == 8 || S == 12 || S == 24;
}

// 256-column slices (W = 1) are built only with GLMVX_MMA_NARROW set (1:
// IQ1_S, 2: every format); measured slower than 512-column slices with half
// the warps for the IQ1_S decode on B200, so off by default.
#ifndef GLMVX_MMA_NARROW
#define GLMVX_MMA_NARROW 0
#endif
template <class F>
static int mma_slice_chunks(int cols) {
    const bool narrow = GLMVX_MMA_NARROW == 2 || (GLMVX_MMA_NARROW == 1 && std::is_same_v<F, FmtIQ1_S>);
    if (narrow && cols % 256 == 0 && mma_slices_ok(cols / 256, 1)) return 1;
    return 2;
}

// Fragments per warp: one with two token pairs per job; for IQ1_S job lists
// of at least kMmaLongRows rows the larger tiles of kFRLong (measured faster
// on the 32-token MoE layer, slower at one token).
constexpr int64_t kMmaLongRows = 150000;
template <class F>
static int mma_plan_fragments(int pairs, int64_t max_rows) {
    if (pairs == 2) return 1;
    if constexpr (std::is_same_v<F, FmtIQ1_S>)
        if (max_rows >= kMmaLongRows) return MmaFmt<F>::kFRLong;
    return MmaFmt<F>::kFR;
}

template <class F>
static bool plan_mma(int64_t max_rows, int64_t max_tiles_extra, int cols, int row_bytes, bool fused, int pairs,
                     MmaPlan &p) {
    using MF = MmaFmt<F>;
    if (cols % 256 || row_bytes % 16) return false;
    p.W = mma_slice_chunks<F>(cols);
    if (cols % (256 * p.W)) return false;
    p.S = cols / (256 * p.W);
    if (!mma_slices_ok(p.S, p.W)) return false;
    p.RG = mma_row_groups(p.S, p.W);
    p.FR = mma_plan_fragments<F>(pairs, max_rows);
    const int R = 16 * p.FR * p.RG;
    // Shared-memory rows span an odd number of 16-byte units, so rows g = 0..7
    // of a fragment start in 8 different 4-bank groups.  Rows that already do
    // (IQ1_S: 400 or 1200 bytes) keep the global stride and arrive with one
    // bulk copy per tile; others are padded by 16 bytes, one copy per row.
    // (The Q8_0 fragment loads read at most 2 bytes past a block, never past
    // a row: the last block of a row has an odd index.)
    p.srow = ((row_bytes >> 4) & 1) ? row_bytes : row_bytes + 16;
    p.stage_stride = (R * p.srow + 127) & ~127;
    const size_t fixed =
        (fused ? 2 * prep_stride(cols) : 0) + MF::kTableBytes + 2ull * R * p.S * 2 * pairs * 4 + 16 * 8 + 64;
    const int fit = static_cast<int>((kMmaSmemBudget - std::min(fixed, kMmaSmemBudget)) / p.stage_stride);
    if (fit < 1) return false;
    const int64_t tiles = (max_rows + R - 1) / R + max_tiles_extra;
    p.stages = static_cast<int>(std::min<int64_t>(std::min(fit, 8), std::max<int64_t>(1, tiles)));
    // In-kernel preparation trades stages for its rows; keep it only while
    // every CTA still overlaps loading with compute, or has one tile anyway.
    if (fused && p.stages < 2 && tiles > sm_count()) return false;
    p.grid = static_cast<int>(std::max<int64_t>(1, std::min<int64_t>(sm_count(), tiles)));
    p.smem = static_cast<size_t>(p.stages) * p.stage_stride + fixed;
    return true;
}

template <class F, int S, int W, int NT, int FR>
static int32_t launch_mma_fr(const MmaPlan &p, const MmaJob &job0, const MmaJob *jobs, const int *njobs_dev,
                             int max_jobs, int batch, int rows_per_job, int cols, int row_bytes, const float *x_raw,
                             const ColSegment &seg, cudaStream_t stream) {
    constexpr int RG = mma_row_groups(S, W);
    auto kern = mma_rows_kernel<F, S, RG, W, NT, FR>;
    if (const int32_t rc = allow_dynamic_smem(kern, p.smem, "packed_mma smem")) return rc;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(p.grid);
    cfg.blockDim = dim3((S * RG + 1) * 32);
    cfg.dynamicSmemBytes = p.smem;
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    const int64_t pitch = seg.pitch ? seg.pitch : row_bytes;
    const int xstride = seg.xstride ? seg.xstride : cols;
    GLMVX_CUDA(cudaLaunchKernelEx(&cfg, kern, job0, jobs, njobs_dev, max_jobs, batch, rows_per_job, cols, row_bytes,
                                  p.srow, p.stages, p.stage_stride, x_raw, pitch, xstride,
                                  static_cast<int>(seg.accumulate), device_error_word()));
    return kOk;
}

template <class F, int S, int W, int NT>
static int32_t launch_mma(const MmaPlan &p, const MmaJob &job0, const MmaJob *jobs, const int *njobs_dev,
                          int max_jobs, int batch, int rows_per_job, int cols, int row_bytes, const float *x_raw,
                          const ColSegment &seg, cudaStream_t stream) {
    if constexpr (NT == 2) {
        return launch_mma_fr<F, S, W, 2, 1>(p, job0, jobs, njobs_dev, max_jobs, batch, rows_per_job, cols, row_bytes,
                                            x_raw, seg, stream);
    } else {
        if constexpr (std::is_same_v<F, FmtIQ1_S>)
            if (p.FR == MmaFmt<F>::kFRLong)
                return launch_mma_fr<F, S, W, 1, MmaFmt<F>::kFRLong>(p, job0, jobs, njobs_dev, max_jobs, batch,
                                                                    rows_per_job, cols, row_bytes, x_raw, seg, stream);
        return launch_mma_fr<F, S, W, 1, MmaFmt<F>::kFR>(p, job0, jobs, njobs_dev, max_jobs, batch, rows_per_job,
                                                          cols, row_bytes, x_raw, seg, stream);
    }
}

template <class F, int NT>
static int32_t launch_mma_s(const MmaPlan &p, const MmaJob &job0, const MmaJob *jobs, const int *njobs_dev,
                            int max_jobs, int batch, int rows_per_job, int cols, int row_bytes, const float *x_raw,
                            const ColSegment &seg, cudaStream_t stream) {
#define GLMVX_MMA_CASE(s, w)                                                                                     \
    case 2 * (s) + (w) - 1:                                                                                     \
        return launch_mma<F, s, w, NT>(p, job0, jobs, njobs_dev, max_jobs, batch, rows_per_job, cols, row_bytes, \
                                       x_raw, seg, stream);
    switch (2 * p.S + p.W - 1) {
        GLMVX_MMA_CASE(1, 2)
        GLMVX_MMA_CASE(2, 2)
        GLMVX_MMA_CASE(3, 2)
        GLMVX_MMA_CASE(4, 2)
        GLMVX_MMA_CASE(6, 2)
        GLMVX_MMA_CASE(8, 2)
        GLMVX_MMA_CASE(12, 2)
        GLMVX_MMA_CASE(16, 2)
#if GLMVX_MMA_NARROW
        GLMVX_MMA_CASE(8, 1)
        GLMVX_MMA_CASE(12, 1)
        GLMVX_MMA_CASE(24, 1)
#endif
    default: set_error("mma: unsupported column count"); return kUnsupported;
    }
#undef GLMVX_MMA_CASE
}

// Rows must be whole 16-byte units for the per-row bulk copies: always for
// Q8_0 (cols % 256) and Q4_K, for IQ1_S when cols % 2048 == 0.
// (Up to 12 column slices: with 16 the register budget of 17 warps spills.)
bool mma_quad_supported(int kind, int cols) { return kind == 19 && mma_supported(kind, cols) && cols <= 6144; }

bool mma_supported(int kind, int cols) {
    if (cols <= 0 || cols % 512 || !mma_slices_ok(cols / 512, 2)) return false;
    return kind == 8 || kind == 12 || (kind == 19 && cols % 2048 == 0);
}

int32_t prep_rows_device(uint8_t *prep, const float *x, const float *x2, int rows, int cols, cudaStream_t stream,
                         const int *rows_dev, int xstride) {
    if (rows <= 0) return kOk;
    if (cols % 256 || (reinterpret_cast<uintptr_t>(prep) & 15) || (reinterpret_cast<uintptr_t>(x) & 15) ||
        (reinterpret_cast<uintptr_t>(x2) & 15)) {
        set_error("prep: columns must be a multiple of 256 and buffers 16-byte aligned");
        return kInvalid;
    }
    const int64_t warps = static_cast<int64_t>(rows) * (cols / 256);
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((warps + 7) / 8));
    cfg.blockDim = dim3(256);
    cfg.stream = stream;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    GLMVX_CUDA(cudaLaunchKernelEx(&cfg, prep_rows_kernel, prep, x, x2, rows, cols, rows_dev, xstride ? xstride : cols));
    return kOk;
}

int32_t mma_gemv_device(int32_t kind, const MmaJob &job0, const MmaJob *jobs, const int *njobs_dev, int max_jobs,
                        int batch, int rows_per_job, int cols, cudaStream_t stream, const float *x_raw, int pairs,
                        const ColSegment &seg) {
    if (pairs != 1 && !(pairs == 2 && jobs && !x_raw && mma_quad_supported(kind, cols))) {
        set_error("mma: two token pairs per job need a job list of a supported format");
        return kInvalid;
    }
    if (x_raw && (jobs || (reinterpret_cast<uintptr_t>(x_raw) & 15))) {
        set_error("mma: in-kernel preparation needs a single matrix and 16-byte aligned activations");
        return kInvalid;
    }
    if (!mma_supported(kind, cols) || rows_per_job <= 0 || max_jobs <= 0) {
        set_error("mma: unsupported format or shape");
        return kUnsupported;
    }
    if (!jobs && (reinterpret_cast<uintptr_t>(job0.w) & 15)) {
        set_error("mma: weights must be 16-byte aligned");
        return kInvalid;
    }
    int blk = 0, bytes = 0;
    reference_layout(kind, blk, bytes);
    const int row_bytes = cols / blk * bytes;
    if ((seg.pitch || seg.xstride || seg.accumulate) &&
        (jobs || (seg.pitch && (seg.pitch < row_bytes || seg.pitch % 16)) || (seg.xstride && seg.xstride < cols))) {
        set_error("mma: a column segment needs a single matrix, a 16-byte row pitch and strides >= its width");
        return kInvalid;
    }
    const int64_t max_rows = static_cast<int64_t>(rows_per_job) * max_jobs;
    int32_t st = kUnsupported;
    dispatch_format(kind, [&]<class F>() {
        if constexpr (std::is_same_v<F, FmtQ8_0> || std::is_same_v<F, FmtQ4_K> || std::is_same_v<F, FmtIQ1_S>) {
            MmaPlan p;
            if (!plan_mma<F>(max_rows, max_jobs, cols, row_bytes, x_raw != nullptr, pairs, p)) {
                set_error("mma: no launch plan for this shape");
                st = kUnsupported;
                return;
            }
            if (pairs == 1) {
                st = launch_mma_s<F, 1>(p, job0, jobs, njobs_dev, max_jobs, batch, rows_per_job, cols, row_bytes, x_raw,
                                        seg, stream);
            } else if constexpr (std::is_same_v<F, FmtIQ1_S>) {
                st = launch_mma_s<F, 2>(p, job0, jobs, njobs_dev, max_jobs, batch, rows_per_job, cols, row_bytes, x_raw,
                                        seg, stream);
            }
        }
    });
    return st;
}

}  // namespace glmvx
