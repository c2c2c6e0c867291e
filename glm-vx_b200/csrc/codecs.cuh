// Device decoders for the 11 packed GGUF formats the reference supports
// (kernels/packed.py:14-19).  Each format exposes
//
//   octet(blk, j0, w[8])  -- weights j0..j0+7 of the block starting at blk
//                            (j0 a multiple of 8), bit-exact with the
//                            reference's scalar decoder;
//   kBlk / kBytes         -- elements and bytes per block.
//
// Bit-exactness: every f32 operation of the reference decoder
// (kernels/packed.vx:24-152) is issued as an explicitly rounded intrinsic
// (__fmul_rn / __fadd_rn / __fsub_rn) in the reference's order, so the
// compiler cannot contract a multiply and a subtract into one FMA.  fp16
// scales are widened with __half2float, which is exact for every fp16 value.
//
// F16 is handled with pseudo-blocks of 8 halves (16 bytes) so it can share
// the octet kernels; rows whose length is not a multiple of 8 use the
// element path (f16_elem).
#pragma once

#include "common.cuh"

namespace glmvx {

// The 19,600-byte GGML codebook blob (layout in codebooks.py), generated at
// build time from gguf-py and SHA-256-pinned to the reference's table.
static __device__ __align__(16) const uint8_t g_codebooks[19600] = {
#include "ggml_tables.inc"
};
constexpr int kTabIq1sGrid = 0, kTabIq2xxsGrid = 16384, kTabIq3xxsGrid = 18432, kTabKsigns = 19456,
              kTabKvaluesIq4nl = 19584;

__device__ __forceinline__ float h2f(uint32_t bits) {
    return __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
}
__device__ __forceinline__ uint32_t u8(const uint8_t *p) { return *p; }
// u16 fields sit at even offsets of even-sized blocks; callers guarantee the
// row base is 2-byte aligned.
__device__ __forceinline__ uint32_t u16(const uint8_t *p) {
    return *reinterpret_cast<const uint16_t *>(p);
}
__device__ __forceinline__ int32_t s8(uint32_t v) { return static_cast<int32_t>(static_cast<int8_t>(v)); }
// 8 bytes from a 2-byte aligned address, as two little-endian words.
__device__ __forceinline__ void ld8_a2(const uint8_t *p, uint32_t &lo, uint32_t &hi) {
    const uint16_t *h = reinterpret_cast<const uint16_t *>(p);
    lo = static_cast<uint32_t>(h[0]) | (static_cast<uint32_t>(h[1]) << 16);
    hi = static_cast<uint32_t>(h[2]) | (static_cast<uint32_t>(h[3]) << 16);
}
__device__ __forceinline__ uint32_t byte_of(uint32_t lo, uint32_t hi, int k) {
    return ((k < 4 ? lo : hi) >> (8 * (k & 3))) & 0xffu;
}
__device__ __forceinline__ int32_t low28(const uint8_t *p) {
    return static_cast<int32_t>(u16(p) | (u16(p + 2) << 16)) & 0x0fffffff;
}

// K-quant 6-bit sub-block scale and min (kernels/packed.vx:107-120).
__device__ __forceinline__ int32_t k4_scale(const uint8_t *s, int g) {
    return g < 4 ? (s[g] & 63) : ((s[g + 4] & 15) | ((s[g - 4] >> 6) << 4));
}
__device__ __forceinline__ int32_t k4_min(const uint8_t *s, int g) {
    return g < 4 ? (s[g + 4] & 63) : ((s[g + 4] >> 4) | ((s[g] >> 6) << 4));
}

struct FmtF16 {  // kernels/packed.vx:24-27 (pseudo-block of 8 halves)
    static constexpr int kKind = 1, kBlk = 8, kBytes = 16;
    __device__ __forceinline__ static void octet(const uint8_t *blk, int, float w[8]) {
#pragma unroll
        for (int k = 0; k < 8; ++k) w[k] = h2f(u16(blk + 2 * k));
    }
};

struct FmtQ8_0 {  // kernels/packed.vx:28-31: d*q
    static constexpr int kKind = 8, kBlk = 32, kBytes = 34;
    __device__ __forceinline__ static void octet(const uint8_t *blk, int j0, float w[8]) {
        const float d = h2f(u16(blk));
        uint32_t lo, hi;
        ld8_a2(blk + 2 + j0, lo, hi);
#pragma unroll
        for (int k = 0; k < 8; ++k) w[k] = __fmul_rn(d, static_cast<float>(s8(byte_of(lo, hi, k))));
    }
};

struct FmtQ2_K {  // kernels/packed.vx:85-94: (d*sc)*q - (dmin*m)
    static constexpr int kKind = 10, kBlk = 256, kBytes = 84;
    __device__ __forceinline__ static void octet(const uint8_t *blk, int j0, float w[8]) {
        const uint32_t sc = u8(blk + j0 / 16);
        const float dl = __fmul_rn(h2f(u16(blk + 80)), static_cast<float>(sc & 15));
        const float ml = __fmul_rn(h2f(u16(blk + 82)), static_cast<float>(sc >> 4));
        uint32_t lo, hi;
        ld8_a2(blk + 16 + (j0 / 128) * 32 + j0 % 32, lo, hi);
        const int shift = 2 * ((j0 % 128) / 32);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float q = static_cast<float>((byte_of(lo, hi, k) >> shift) & 3);
            w[k] = __fsub_rn(__fmul_rn(dl, q), ml);
        }
    }
};

struct FmtQ3_K {  // kernels/packed.vx:95-106: (d*sc)*q, q -= 4 when the hmask bit is clear
    static constexpr int kKind = 11, kBlk = 256, kBytes = 110;
    __device__ __forceinline__ static void octet(const uint8_t *blk, int j0, float w[8]) {
        const int g = j0 / 16;
        const int32_t low = (u8(blk + 96 + g % 8) >> (4 * (g / 8))) & 15;
        const int32_t high = (u8(blk + 104 + g % 4) >> (2 * (g / 4))) & 3;
        const float dsc = __fmul_rn(h2f(u16(blk + 108)), static_cast<float>((low | (high << 4)) - 32));
        uint32_t lo, hi, mlo, mhi;
        ld8_a2(blk + 32 + (j0 / 128) * 32 + j0 % 32, lo, hi);
        ld8_a2(blk + j0 % 32, mlo, mhi);
        const int shift = 2 * ((j0 % 128) / 32), mbit = j0 / 32;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            int32_t q = (byte_of(lo, hi, k) >> shift) & 3;
            if (((byte_of(mlo, mhi, k) >> mbit) & 1) == 0) q -= 4;
            w[k] = __fmul_rn(dsc, static_cast<float>(q));
        }
    }
};

struct FmtQ4_K {  // kernels/packed.vx:121-130: (d*sc)*q - (dmin*m)
    static constexpr int kKind = 12, kBlk = 256, kBytes = 144;
    __device__ __forceinline__ static void octet(const uint8_t *blk, int j0, float w[8]) {
        const int g = j0 / 32;
        const float dl = __fmul_rn(h2f(u16(blk)), static_cast<float>(k4_scale(blk + 4, g)));
        const float ml = __fmul_rn(h2f(u16(blk + 2)), static_cast<float>(k4_min(blk + 4, g)));
        uint32_t lo, hi;
        ld8_a2(blk + 16 + (j0 / 64) * 32 + j0 % 32, lo, hi);
        const int shift = 4 * (g % 2);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float q = static_cast<float>((byte_of(lo, hi, k) >> shift) & 15);
            w[k] = __fsub_rn(__fmul_rn(dl, q), ml);
        }
    }
};

struct FmtQ5_K {  // kernels/packed.vx:131-141
    static constexpr int kKind = 13, kBlk = 256, kBytes = 176;
    __device__ __forceinline__ static void octet(const uint8_t *blk, int j0, float w[8]) {
        const int g = j0 / 32;
        const float dl = __fmul_rn(h2f(u16(blk)), static_cast<float>(k4_scale(blk + 4, g)));
        const float ml = __fmul_rn(h2f(u16(blk + 2)), static_cast<float>(k4_min(blk + 4, g)));
        uint32_t lo, hi, hlo, hhi;
        ld8_a2(blk + 48 + (j0 / 64) * 32 + j0 % 32, lo, hi);
        ld8_a2(blk + 16 + j0 % 32, hlo, hhi);
        const int shift = 4 * (g % 2);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int32_t q = ((byte_of(lo, hi, k) >> shift) & 15) | (((byte_of(hlo, hhi, k) >> g) & 1) << 4);
            w[k] = __fsub_rn(__fmul_rn(dl, static_cast<float>(q)), ml);
        }
    }
};

struct FmtQ6_K {  // kernels/packed.vx:142-152: (d*sc)*q
    static constexpr int kKind = 14, kBlk = 256, kBytes = 210;
    __device__ __forceinline__ static void octet(const uint8_t *blk, int j0, float w[8]) {
        const int g = (j0 % 128) / 32;
        const float dsc = __fmul_rn(h2f(u16(blk + 208)), static_cast<float>(s8(u8(blk + 192 + j0 / 16))));
        uint32_t lo, hi, hlo, hhi;
        ld8_a2(blk + (j0 / 128) * 64 + (g % 2) * 32 + j0 % 32, lo, hi);
        ld8_a2(blk + 128 + (j0 / 128) * 32 + j0 % 32, hlo, hhi);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const int32_t low = (byte_of(lo, hi, k) >> (4 * (g / 2))) & 15;
            const int32_t high = (byte_of(hlo, hhi, k) >> (2 * g)) & 3;
            w[k] = __fmul_rn(dsc, static_cast<float>((low | (high << 4)) - 32));
        }
    }
};

struct FmtIQ2_XXS {  // kernels/packed.vx:45-59
    static constexpr int kKind = 16, kBlk = 256, kBytes = 66;
    __device__ __forceinline__ static void octet(const uint8_t *blk, int j0, float w[8]) {
        const int g = j0 / 32, l = (j0 % 32) / 8;
        const uint8_t *p = blk + 2 + 8 * g;
        const int32_t bits = low28(p + 4);
        const float dl =
            __fmul_rn(__fmul_rn(h2f(u16(blk)), __fadd_rn(0.5f, static_cast<float>(u8(p + 7) >> 4))), 0.25f);
        const uint8_t *grid = g_codebooks + kTabIq2xxsGrid + u8(p + l) * 8;
        const uint32_t sign = g_codebooks[kTabKsigns + ((bits >> (7 * l)) & 127)];
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const float s = (sign & (1u << k)) ? -1.0f : 1.0f;
            w[k] = __fmul_rn(__fmul_rn(dl, static_cast<float>(grid[k])), s);
        }
    }
};

struct FmtIQ3_XXS {  // kernels/packed.vx:60-74
    static constexpr int kKind = 18, kBlk = 256, kBytes = 98;
    __device__ __forceinline__ static void octet(const uint8_t *blk, int j0, float w[8]) {
        const int g = j0 / 32, l = (j0 % 32) / 8;
        const uint8_t *p = blk + 66 + 4 * g;
        const int32_t bits = low28(p);
        const float dl =
            __fmul_rn(__fmul_rn(h2f(u16(blk)), __fadd_rn(0.5f, static_cast<float>(u8(p + 3) >> 4))), 0.5f);
        const uint32_t sign = g_codebooks[kTabKsigns + ((bits >> (7 * l)) & 127)];
        const uint8_t *qs = blk + 2 + 8 * g + 2 * l;
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t v = g_codebooks[kTabIq3xxsGrid + u8(qs + k / 4) * 4 + k % 4];
            const float s = (sign & (1u << k)) ? -1.0f : 1.0f;
            w[k] = __fmul_rn(__fmul_rn(dl, static_cast<float>(v)), s);
        }
    }
};

struct FmtIQ1_S {  // kernels/packed.vx:32-44: d*(2s+1) * (grid + delta)
    static constexpr int kKind = 19, kBlk = 256, kBytes = 50;
    __device__ __forceinline__ static void octet(const uint8_t *blk, int j0, float w[8]) {
        const int g = j0 / 32, l = (j0 % 32) / 8;
        const uint32_t high = u16(blk + 34 + 2 * g);
        const uint32_t index = u8(blk + 2 + 4 * g + l) | (((high >> (3 * l)) & 7) << 8);
        const float dl = __fmul_rn(h2f(u16(blk)), static_cast<float>(2 * ((high >> 12) & 7) + 1));
        const float delta = (high & 0x8000u) ? -0.125f : 0.125f;
        const uint2 row = __ldg(reinterpret_cast<const uint2 *>(g_codebooks + kTabIq1sGrid) + index);
#pragma unroll
        for (int k = 0; k < 8; ++k)
            w[k] = __fmul_rn(dl, __fadd_rn(static_cast<float>(s8(byte_of(row.x, row.y, k))), delta));
    }
};

struct FmtIQ4_XS {  // kernels/packed.vx:75-84
    static constexpr int kKind = 23, kBlk = 256, kBytes = 136;
    __device__ __forceinline__ static void octet(const uint8_t *blk, int j0, float w[8]) {
        const int g = j0 / 32;
        const int32_t sc = ((u8(blk + 4 + g / 2) >> (4 * (g % 2))) & 15) | (((u16(blk + 2) >> (2 * g)) & 3) << 4);
        const float dl = __fmul_rn(h2f(u16(blk)), static_cast<float>(sc - 32));
        uint32_t lo, hi;
        ld8_a2(blk + 8 + 16 * g + j0 % 16, lo, hi);
        const int shift = 4 * ((j0 % 32) / 16);
#pragma unroll
        for (int k = 0; k < 8; ++k) {
            const uint32_t q = (byte_of(lo, hi, k) >> shift) & 15;
            w[k] = __fmul_rn(dl, static_cast<float>(s8(g_codebooks[kTabKvaluesIq4nl + q])));
        }
    }
};

// Element decode of one fp16 weight (rows of any length).
__device__ __forceinline__ float f16_elem(const uint8_t *row, int j) { return h2f(u16(row + 2 * j)); }

// Octet o of a row: the block it falls in and its first element in that block.
template <class F>
__device__ __forceinline__ void row_octet(const uint8_t *row, int o, float w[8]) {
    constexpr int kOctPerBlk = F::kBlk / 8;
    const int b = o / kOctPerBlk;
    F::octet(row + static_cast<size_t>(b) * F::kBytes, (o - b * kOctPerBlk) * 8, w);
}

// Invoke `fn.template operator()<Fmt>()` for a GGML kind; returns false for
// an unsupported kind.
template <class Fn>
__host__ bool dispatch_format(int kind, Fn &&fn) {
    switch (kind) {
    case 1: fn.template operator()<FmtF16>(); return true;
    case 8: fn.template operator()<FmtQ8_0>(); return true;
    case 10: fn.template operator()<FmtQ2_K>(); return true;
    case 11: fn.template operator()<FmtQ3_K>(); return true;
    case 12: fn.template operator()<FmtQ4_K>(); return true;
    case 13: fn.template operator()<FmtQ5_K>(); return true;
    case 14: fn.template operator()<FmtQ6_K>(); return true;
    case 16: fn.template operator()<FmtIQ2_XXS>(); return true;
    case 18: fn.template operator()<FmtIQ3_XXS>(); return true;
    case 19: fn.template operator()<FmtIQ1_S>(); return true;
    case 23: fn.template operator()<FmtIQ4_XS>(); return true;
    default: return false;
    }
}

// Reference block geometry (elements, bytes) per GGML kind; F16 is (1, 2).
__host__ __device__ inline bool reference_layout(int kind, int &blk, int &bytes) {
    switch (kind) {
    case 1: blk = 1; bytes = 2; return true;
    case 8: blk = 32; bytes = 34; return true;
    case 10: blk = 256; bytes = 84; return true;
    case 11: blk = 256; bytes = 110; return true;
    case 12: blk = 256; bytes = 144; return true;
    case 13: blk = 256; bytes = 176; return true;
    case 14: blk = 256; bytes = 210; return true;
    case 16: blk = 256; bytes = 66; return true;
    case 18: blk = 256; bytes = 98; return true;
    case 19: blk = 256; bytes = 50; return true;
    case 23: blk = 256; bytes = 136; return true;
    default: return false;
    }
}

}  // namespace glmvx
