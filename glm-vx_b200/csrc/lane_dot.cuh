// Per-lane dot products for the streaming GEMV: one lane, one row, two
// consecutive 32-weight units (sub-blocks / Q8_0 blocks) whose 64 activations
// the lane holds in registers.
//
// These trade the bit-exact decode (codecs.cuh, used by unpack) for fewer
// instructions per weight; results stay within the f32 tolerance because
// every quantised integer is still represented exactly:
//
//  * Q4_K / IQ1_S: a small integer v (a nibble, or grid value + 1) is placed
//    in the top mantissa byte of the float 1.0 with one byte permute, giving
//    exactly f = 1 + v/2^s (s = 7 or 4 for Q4_K low/high nibbles, 3 for
//    IQ1_S).  FMAs accumulate sum f*x, and sum v*x = 2^s*(sum f*x - sum x)
//    with sum x precomputed per unit.  The cancellation this introduces is
//    bounded by ~2^s f32 ulps of sum |x| (f lies in [1, 2)), far inside the
//    1e-5 tolerance.
//  * Q8_0: signed bytes become 2^23 + 128 + q by one byte permute and are
//    re-centred with one exact FADD, then one FFMA.
//  * Scales are applied once per unit: Q4_K d*sc and dmin*m
//    (kernels/packed.vx:121-130), IQ1_S d*(2s+1) and the +-1/8 delta
//    (kernels/packed.vx:32-44), Q8_0 d (kernels/packed.vx:28-31).
// Other formats use the exact octet decoders.  Products accumulate with the
// packed f32x2 FMA (__ffma2_rn), two weights per instruction; the lane's
// activations are held as float2 pairs.
#pragma once

#include "codecs.cuh"

namespace glmvx {

__device__ __forceinline__ float perm_float(uint32_t bytes, uint32_t hi_const, uint32_t selector) {
    return __uint_as_float(__byte_perm(bytes, hi_const, selector));
}

// Byte k of `bytes` into bits 16..23 under exponent byte 0x3F: 1 + b*2^-7.
template <int K>
__device__ __forceinline__ float biased_one(uint32_t bytes) {
    return perm_float(bytes, 0x3F000000u, 0x7044u | (K << 8));
}

// Generic path: exact octet decode, packed FMA per weight pair.
template <class F>
struct LaneDot {
    static constexpr int kRowsPerWarp = 2;
    static constexpr int kTableBytes = 0;
    __device__ __forceinline__ static void init_table(uint8_t *, int, int) {}
    __device__ __forceinline__ static float dot(const uint8_t *row, int unit0, int units, const float2 (&x)[2][16],
                                                const float (&)[2], const uint8_t *) {
        float2 acc = make_float2(0.f, 0.f);
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (unit0 + u < units) {
#pragma unroll
                for (int o = 0; o < 4; ++o) {
                    float wv[8];
                    row_octet<F>(row, 4 * (unit0 + u) + o, wv);
#pragma unroll
                    for (int e = 0; e < 4; ++e) acc = __ffma2_rn(make_float2(wv[2 * e], wv[2 * e + 1]), x[u][4 * o + e], acc);
                }
            }
        }
        return acc.x + acc.y;
    }
};

// Small non-negative integer -> exact float without the conversion pipe.
__device__ __forceinline__ float small_int_float(uint32_t v) {
    return __uint_as_float(0x4B000000u | v) - 8388608.0f;
}

// Two weights of one word as biased floats (bytes K, K+1).
template <int K>
__device__ __forceinline__ float2 biased_pair(uint32_t bytes) {
    return make_float2(biased_one<K>(bytes), biased_one<K + 1>(bytes));
}

// Q4_K: units 2m, 2m+1 of one superblock share the 32 nibble bytes at 16+32m
// (low nibbles = sub-block 2m, high nibbles = sub-block 2m+1).  The twelve
// scale bytes are unpacked for all eight sub-blocks at once, four per word
// (kernels/packed.vx:107-120 restated on packed bytes).
template <>
struct LaneDot<FmtQ4_K> {
    static constexpr int kRowsPerWarp = 4;
    static constexpr int kTableBytes = 0;
    __device__ __forceinline__ static void init_table(uint8_t *, int, int) {}
    __device__ __forceinline__ static float dot(const uint8_t *row, int unit0, int units, const float2 (&x)[2][16],
                                                const float (&xs)[2], const uint8_t *) {
        if (unit0 >= units) return 0.0f;
        const uint8_t *blk = row + (unit0 >> 3) * 144;
        const int m = (unit0 & 7) >> 1;
        const uint4 head = *reinterpret_cast<const uint4 *>(blk);  // d, dmin, 12 scale bytes
        const float d = h2f(head.x & 0xffffu), dmin = h2f(head.x >> 16);
        // sub-blocks 0..3: 6 low bits of bytes 0..3 / 4..7; 4..7: nibbles of 8..11 plus top bits.
        const uint32_t sc = m < 2 ? (head.y & 0x3F3F3F3Fu) : ((head.w & 0x0F0F0F0Fu) | ((head.y >> 2) & 0x30303030u));
        const uint32_t mn = m < 2 ? (head.z & 0x3F3F3F3Fu)
                                  : (((head.w >> 4) & 0x0F0F0F0Fu) | ((head.z >> 2) & 0x30303030u));
        const int sh = 16 * (m & 1);  // bytes 2m%4, 2m%4+1
        const float dl0 = d * small_int_float((sc >> sh) & 0xffu);
        const float dl1 = d * small_int_float((sc >> (sh + 8)) & 0xffu);
        const float ml0 = dmin * small_int_float((mn >> sh) & 0xffu);
        const float ml1 = dmin * small_int_float((mn >> (sh + 8)) & 0xffu);
        const uint4 *nib = reinterpret_cast<const uint4 *>(blk + 16 + 32 * m);
        const uint4 n0 = nib[0], n1 = nib[1];
        const uint32_t words[8] = {n0.x, n0.y, n0.z, n0.w, n1.x, n1.y, n1.z, n1.w};
        float2 a = make_float2(0.f, 0.f), b = make_float2(0.f, 0.f);
#pragma unroll
        for (int i = 0; i < 8; ++i) {
            const uint32_t lo = (words[i] & 0x0F0F0F0Fu) | 0x80808080u;           // low nibble q -> 1 + q/128
            const uint32_t hi = ((words[i] >> 1) & 0x78787878u) | 0x80808080u;  // high nibble q -> 1 + q/16
            a = __ffma2_rn(biased_pair<0>(lo), x[0][2 * i], a);
            a = __ffma2_rn(biased_pair<2>(lo), x[0][2 * i + 1], a);
            b = __ffma2_rn(biased_pair<0>(hi), x[1][2 * i], b);
            b = __ffma2_rn(biased_pair<2>(hi), x[1][2 * i + 1], b);
        }
        const float q0 = 128.0f * ((a.x + a.y) - xs[0]);  // sum q*x, low sub-block
        const float q1 = 16.0f * ((b.x + b.y) - xs[1]);
        float r = fmaf(dl0, q0, -ml0 * xs[0]);
        if (unit0 + 1 < units) r += fmaf(dl1, q1, -ml1 * xs[1]);
        return r;
    }
};

// Q8_0: two 34-byte blocks, d*q.
template <>
struct LaneDot<FmtQ8_0> {
    static constexpr int kRowsPerWarp = 4;
    static constexpr int kTableBytes = 0;
    __device__ __forceinline__ static void init_table(uint8_t *, int, int) {}
    __device__ __forceinline__ static float dot(const uint8_t *row, int unit0, int units, const float2 (&x)[2][16],
                                                const float (&)[2], const uint8_t *) {
        const float2 centre = make_float2(-8388736.0f, -8388736.0f);  // -(2^23 + 128)
        float r = 0.0f;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (unit0 + u >= units) break;
            const uint8_t *blk = row + (unit0 + u) * 34;
            const float d = h2f(u16(blk));
            // 32 quant bytes at blk+2 (2-byte aligned): aligned words + funnel shift.
            const uintptr_t addr = reinterpret_cast<uintptr_t>(blk + 2);
            const uint32_t *base = reinterpret_cast<const uint32_t *>(addr & ~static_cast<uintptr_t>(3));
            const uint32_t sh = static_cast<uint32_t>(addr & 3) * 8;
            uint32_t wds[9];
#pragma unroll
            for (int i = 0; i < 9; ++i) wds[i] = base[i];
            float2 a = make_float2(0.f, 0.f);
#pragma unroll
            for (int i = 0; i < 8; ++i) {
                const uint32_t q = __funnelshift_r(wds[i], wds[i + 1], sh) ^ 0x80808080u;
                // bytes become 2^23 + 128 + q; one packed add recentres two exactly
                const float2 v0 = __fadd2_rn(make_float2(perm_float(q, 0x4B000000u, 0x7440u),
                                                         perm_float(q, 0x4B000000u, 0x7441u)), centre);
                const float2 v1 = __fadd2_rn(make_float2(perm_float(q, 0x4B000000u, 0x7442u),
                                                         perm_float(q, 0x4B000000u, 0x7443u)), centre);
                a = __ffma2_rn(v0, x[u][2 * i], a);
                a = __ffma2_rn(v1, x[u][2 * i + 1], a);
            }
            r = fmaf(d, a.x + a.y, r);
        }
        return r;
    }
};

// IQ1_S: sub-blocks g, g+1 of one superblock.  The CTA keeps a transformed
// iq1s grid in shared memory whose bytes already read 0x80|(g+1)<<4, so a
// byte permute yields f = 1 + (g+1)/8 directly.
template <>
struct LaneDot<FmtIQ1_S> {
    static constexpr int kRowsPerWarp = 4;
    static constexpr int kTableBytes = 2048 * 8;
    __device__ __forceinline__ static void init_table(uint8_t *table, int tid, int nthreads) {
        const uint32_t *src = reinterpret_cast<const uint32_t *>(g_codebooks + kTabIq1sGrid);
        uint32_t *dst = reinterpret_cast<uint32_t *>(table);
        for (int i = tid; i < 4096; i += nthreads) {
            const uint32_t g1 = (src[i] ^ 0x80808080u) - 0x7f7f7f7fu;  // bytes g+1 in {0,1,2}
            dst[i] = (g1 << 4) | 0x80808080u;
        }
    }
    __device__ __forceinline__ static float dot(const uint8_t *row, int unit0, int units, const float2 (&x)[2][16],
                                                const float (&xs)[2], const uint8_t *table) {
        if (unit0 >= units) return 0.0f;
        const uint8_t *blk = row + (unit0 >> 3) * 50;
        const float d = h2f(u16(blk));
        const uint2 *grid = reinterpret_cast<const uint2 *>(table);
        float r = 0.0f;
#pragma unroll
        for (int u = 0; u < 2; ++u) {
            if (unit0 + u >= units) break;
            const int g = (unit0 + u) & 7;
            const uint32_t high = u16(blk + 34 + 2 * g);
            const uint32_t qs = u16(blk + 2 + 4 * g) | (u16(blk + 4 + 4 * g) << 16);
            float2 a = make_float2(0.f, 0.f);
#pragma unroll
            for (int l = 0; l < 4; ++l) {
                const uint32_t idx = ((qs >> (8 * l)) & 0xffu) | (((high >> (3 * l)) & 7u) << 8);
                const uint2 gr = grid[idx];
                a = __ffma2_rn(biased_pair<0>(gr.x), x[u][4 * l + 0], a);
                a = __ffma2_rn(biased_pair<2>(gr.x), x[u][4 * l + 1], a);
                a = __ffma2_rn(biased_pair<0>(gr.y), x[u][4 * l + 2], a);
                a = __ffma2_rn(biased_pair<2>(gr.y), x[u][4 * l + 3], a);
            }
            // sum (g+1)*x = 8*(sum f*x - sum x);  sum g*x = that - sum x.
            const float gx = 8.0f * ((a.x + a.y) - xs[u]) - xs[u];
            const float dl = d * static_cast<float>(2 * ((high >> 12) & 7) + 1);
            const float delta = (high & 0x8000u) ? -0.125f : 0.125f;
            r = fmaf(dl, fmaf(delta, xs[u], gx), r);
        }
        return r;
    }
};

}  // namespace glmvx
