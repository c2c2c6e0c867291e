// Packed-GGUF GEMM for token batches on the 5th-generation tensor cores
// (tcgen05), the batch_v2 contract (kernels/packed.vx:473ff):
// out[t][r] = sum_j w[r][j] * x[t][j] in f32 with w decoded per GGML block.
//
// Numerics.  Every weight is decoded to the f32 value the reference computes
// (Q8_0 and Q4_K by their own 16-weight decoders, the other formats by their
// `octet`, codecs.cuh) and split exactly into three bf16 limbs (w = a1 + a2 +
// a3: the top 8 significant bits, the next 8, the rest); the activations are
// split the same way (b1 + b2 + b3) by prep_tc_kernel.  bf16 keeps f32's
// exponent range, so nothing is scaled, and every limb product is exact in
// f32.  Three kind::f16 (bf16) MMAs per K step of 16 columns, a1 x [b1 | b2 |
// b3], a2 x [b1 | b2] and a3 x b1, accumulate the whole row in f32 in tensor
// memory; the epilogue adds the b1, b2 and b3 columns.  The dropped a2*b3,
// a3*b2, a3*b3 are below 2^-23 |w x|.  A non-finite activation turns its own
// token's outputs NaN only (columns are tokens).
//
// Kernel (gemm_tc_kernel<F>): one CTA per 128-row tile, 18 warps.
//   warp 0   producer: per chunk of `chunk_cols` columns one 2-D tiled TMA
//            copy of the tile's raw packed bytes (128 rows x the chunk's
//            bytes, the tensor map's rows past the matrix read as zeros)
//            into a ring of one or two stages -- one multi-KB copy instead
//            of 128 row copies of 144-880 bytes, which measured ~1 us per
//            32 columns; per 32-column atom one 1-D bulk copy of the
//            prepared activation limbs (already in the operand layout);
//   warp 1   allocates tensor memory; lane 0 issues the MMAs of each atom
//            (2 K steps x 3, M = 128) and commits them to the atom slot's
//            mbarrier;
//   warps 2-17 decode in two groups of 8 taking alternate atoms: per atom
//            128 rows x 32 columns, a thread 16 weights of one row, into
//            the three K-major A limb tiles (8 x 16-byte core matrices, no
//            swizzle) of the atom's slot;
//   warps 2-5 (one per lane quarter) read the accumulators at the end
//            (tcgen05.ld) and store out[t][row].
// Every mbarrier wait is bounded (2 s): on expiry the kernel records the
// device error word and returns after freeing its tensor memory.
//
// Measured costs that shape it: a tcgen05.mma of M = 128 and N <= 64 takes
// ~25 ns back to back whatever N (K = 8 TF32 or K = 16 f16/bf16), so few,
// wide MMAs -- bf16 limbs give twice the K of TF32 per MMA and half the
// operand bytes; per-row bulk copies of a few hundred bytes cost ~1 us per 32
// columns, hence the 2-D tensor-map copy.
#include <algorithm>
#include <type_traits>

#include <cuda.h>
#include <cuda_fp8.h>

#include "codecs.cuh"
#include "mma_gemv.cuh"
#include "tcgen05.cuh"

namespace glmvx {

namespace {

constexpr int kTcRows = 128;                    // weight rows per CTA (UMMA M)
constexpr int kTcAtomCols = 32;                 // columns per atom (one A slot, 2 K steps)
constexpr int kTcLimbs = 3;                     // bf16 limbs per operand (8 + 8 + 8 bits)
constexpr int kTcRowBytes = kTcAtomCols * 2;    // one row of one limb of an atom: 64 bytes
constexpr int kTcATile = kTcRows * kTcRowBytes; // one limb of one atom: 8 KB
constexpr int kTcGroupWarps = 8;                // a decode group: 8 warps, one atom at a time
// Threads of a CTA with NG decode groups: producer + MMA warps + groups.
__host__ __device__ constexpr int tc_threads(int ng) { return (2 + ng * kTcGroupWarps) * 32; }
// Shared memory of a CTA that shares its SM with another (one decode group):
// half the opt-in maximum less the per-CTA reservation.
constexpr int kTcSmemHalf = 112 * 1024;
constexpr int kTcSmemBudget = 226 * 1024;
constexpr int kTcMaxTokens = 64;

constexpr uint32_t kHi16 = 0xFFFF0000u;

// Columns per raw stage: the smallest multiple of 256 (and of the block)
// whose packed bytes per row are a multiple of 16, at most 2048.
__host__ __device__ constexpr int tc_chunk_cols(int blk, int bytes) {
    for (int c = 256; c <= 2048; c += 256)
        if (c % blk == 0 && (c / blk * bytes) % 16 == 0) return c;
    return 0;
}

// f32 -> three bf16 limbs, exactly: l1 = v truncated to bf16, l2 = (v - l1)
// truncated, l3 = the rest (at most 8 significant bits, a bf16 value).  Each
// limb is returned as the f32 bit pattern whose low 16 bits are zero.
__device__ __forceinline__ void bf16_limbs(float v, uint32_t &l1, uint32_t &l2, uint32_t &l3) {
    l1 = __float_as_uint(v) & kHi16;
    const float r1 = v - __uint_as_float(l1);
    l2 = __float_as_uint(r1) & kHi16;
    l3 = __float_as_uint(r1 - __uint_as_float(l2));
}

// Two limb values (low 16 bits zero) as one bf16x2 word, element 0 low.
__device__ __forceinline__ uint32_t pack_bf16(uint32_t e0, uint32_t e1) { return __byte_perm(e0, e1, 0x7632); }

// Instruction descriptor, kind::f16 with BF16 A and B (bits 7-9, 10-12 = 1),
// f32 accumulation (bits 4-5 = 1), both K-major, N >> 3 at bit 17, M >> 4 at 24.
__host__ __device__ constexpr uint32_t umma_idesc_bf16(int m, int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | (static_cast<uint32_t>(n >> 3) << 17) |
           (static_cast<uint32_t>(m >> 4) << 24);
}

__device__ __forceinline__ void umma_bf16(uint32_t tmem_d, uint64_t adesc, uint64_t bdesc, uint32_t idesc,
                                          uint32_t accumulate) {
    asm volatile(
        "{\n\t.reg .pred p;\n\t"
        "setp.ne.b32 p, %4, 0;\n\t"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n\t}" ::"r"(tmem_d),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(accumulate)
        : "memory");
}

// K-major operand tiles without swizzle, as core matrices of 8 rows x 16
// bytes (128 contiguous bytes): 16-byte chunk c (bf16 k = 8c..8c+7) of row r
// of a `rows`-row atom sits in K step c/2 (one MMA, K = 16), core matrix c%2
// of 8-row group r/8.  Per K step the tile is rows*32 contiguous bytes, so an
// MMA reads exactly its operands.
__host__ __device__ __forceinline__ uint32_t kmajor_offset(int r, int c, int rows) {
    return static_cast<uint32_t>((c >> 1) * rows * 32 + (r >> 3) * 256 + (c & 1) * 128 + (r & 7) * 16);
}

// UMMA shared-memory descriptor of a K-major SWIZZLE_NONE tile: leading
// byte offset 128 (between the two core matrices of a K step), stride byte
// offset 256 (between 8-row groups), version 1, layout type 0.
__device__ __forceinline__ uint64_t umma_desc_kmajor(uint32_t addr) {
    return static_cast<uint64_t>((addr >> 4) & 0x3FFFu) | (8ull << 16) | (16ull << 32) | (1ull << 46);
}

// Byte k of u as the float 2^23 + byte: the byte permuted into the mantissa.
template <int K>
__device__ __forceinline__ float byte_biased(uint32_t u) {
    return __uint_as_float(__byte_perm(u, 0x4B000000u, 0x7650u | K));
}

// The 16 weights of tile row `rc` (its bytes in the raw stage) at chunk
// columns a*32 + 16h .. +15, as the reference computes them in f32.
// Generic: two octets of the format's decoder.
template <class F>
struct TcDecode {
    static constexpr bool kWords = false;
    __device__ __forceinline__ static void run(const uint8_t *rc, int a, int h, float (&w)[16]) {
#pragma unroll
        for (int o = 0; o < 2; ++o) {
            const int col = a * kTcAtomCols + 16 * h + 8 * o;
            F::octet(rc + (col / F::kBlk) * F::kBytes, col % F::kBlk, w + 8 * o);
        }
    }
};

// Q8_0 (kernels/packed.vx:28-31, w = d*q): atom a is block a of the chunk;
// its 16 bytes come in four 32-bit loads (odd a: 4-byte aligned) or five
// and funnel shifts (even a: 2 bytes past alignment); q + 128 enters the
// mantissa of 2^23 and one subtraction gives q exactly.
template <>
struct TcDecode<FmtQ8_0> {
    static constexpr bool kWords = true;
    // Words q and q + 4 (weights 4q..4q+3 and 16+4q..16+4q+3) of atom a of
    // row `rc`: the lanes of a warp, 8 rows x 4 quarters, read 32 different
    // banks (rows are 68 words apart).
    __device__ __forceinline__ static void words(const uint8_t *rc, int a, int q, float, float (&w)[8]) {
        const uint8_t *blk = rc + a * FmtQ8_0::kBytes;
        const float d = h2f(u16(blk));
        uint32_t x[2];
        if (a & 1) {  // the block's bytes start 4-byte aligned
            const uint32_t *p = reinterpret_cast<const uint32_t *>(blk + 2);
            x[0] = p[q];
            x[1] = p[q + 4];
        } else {  // 2 bytes past alignment: join aligned neighbours
            const uint32_t *p = reinterpret_cast<const uint32_t *>(blk);
            x[0] = __funnelshift_r(p[q], p[q + 1], 16);
            x[1] = __funnelshift_r(p[q + 4], p[q + 5], 16);
        }
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            const uint32_t u = x[i] ^ 0x80808080u;
            w[4 * i + 0] = __fmul_rn(d, byte_biased<0>(u) - 8388736.0f);
            w[4 * i + 1] = __fmul_rn(d, byte_biased<1>(u) - 8388736.0f);
            w[4 * i + 2] = __fmul_rn(d, byte_biased<2>(u) - 8388736.0f);
            w[4 * i + 3] = __fmul_rn(d, byte_biased<3>(u) - 8388736.0f);
        }
    }
    __device__ __forceinline__ static void run(const uint8_t *rc, int a, int h, float (&w)[16]) {
        const uint8_t *blk = rc + a * FmtQ8_0::kBytes;
        const float d = h2f(u16(blk));
        uint32_t v[4];
        if (a & 1) {
            const uint32_t *p = reinterpret_cast<const uint32_t *>(blk + 2 + 16 * h);
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = p[i];
        } else {
            const uint32_t *p = reinterpret_cast<const uint32_t *>(blk + 16 * h);
            uint32_t x[5];
#pragma unroll
            for (int i = 0; i < 5; ++i) x[i] = p[i];
#pragma unroll
            for (int i = 0; i < 4; ++i) v[i] = __funnelshift_r(x[i], x[i + 1], 16);
        }
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            const uint32_t u = v[i] ^ 0x80808080u;
            w[4 * i + 0] = __fmul_rn(d, byte_biased<0>(u) - 8388736.0f);
            w[4 * i + 1] = __fmul_rn(d, byte_biased<1>(u) - 8388736.0f);
            w[4 * i + 2] = __fmul_rn(d, byte_biased<2>(u) - 8388736.0f);
            w[4 * i + 3] = __fmul_rn(d, byte_biased<3>(u) - 8388736.0f);
        }
    }
};

// Q4_K (kernels/packed.vx:121-130, w = (d*sc)*q - dmin*m): the chunk is one
// superblock, atom a its sub-block a; the 16 nibble bytes in one 16-byte load.
template <>
struct TcDecode<FmtQ4_K> {
    static constexpr bool kWords = true;
    // As TcDecode<FmtQ8_0>::words (rows 36 words apart).
    __device__ __forceinline__ static void words(const uint8_t *rc, int a, int q, float, float (&w)[8]) {
        const float dl = __fmul_rn(h2f(u16(rc)), static_cast<float>(k4_scale(rc + 4, a)));
        const float ml = __fmul_rn(h2f(u16(rc + 2)), static_cast<float>(k4_min(rc + 4, a)));
        const uint32_t *p = reinterpret_cast<const uint32_t *>(rc + 16 + 32 * (a >> 1));
        const int shift = 4 * (a & 1);
        const uint32_t x[2] = {(p[q] >> shift) & 0x0F0F0F0Fu, (p[q + 4] >> shift) & 0x0F0F0F0Fu};
#pragma unroll
        for (int i = 0; i < 2; ++i) {
            w[4 * i + 0] = __fsub_rn(__fmul_rn(dl, byte_biased<0>(x[i]) - 8388608.0f), ml);
            w[4 * i + 1] = __fsub_rn(__fmul_rn(dl, byte_biased<1>(x[i]) - 8388608.0f), ml);
            w[4 * i + 2] = __fsub_rn(__fmul_rn(dl, byte_biased<2>(x[i]) - 8388608.0f), ml);
            w[4 * i + 3] = __fsub_rn(__fmul_rn(dl, byte_biased<3>(x[i]) - 8388608.0f), ml);
        }
    }
    __device__ __forceinline__ static void run(const uint8_t *rc, int a, int h, float (&w)[16]) {
        const float dl = __fmul_rn(h2f(u16(rc)), static_cast<float>(k4_scale(rc + 4, a)));
        const float ml = __fmul_rn(h2f(u16(rc + 2)), static_cast<float>(k4_min(rc + 4, a)));
        const uint4 q = *reinterpret_cast<const uint4 *>(rc + 16 + 32 * (a >> 1) + 16 * h);
        const int shift = 4 * (a & 1);
        const uint32_t v[4] = {(q.x >> shift) & 0x0F0F0F0Fu, (q.y >> shift) & 0x0F0F0F0Fu, (q.z >> shift) & 0x0F0F0F0Fu,
                               (q.w >> shift) & 0x0F0F0F0Fu};
#pragma unroll
        for (int i = 0; i < 4; ++i) {
            w[4 * i + 0] = __fsub_rn(__fmul_rn(dl, byte_biased<0>(v[i]) - 8388608.0f), ml);
            w[4 * i + 1] = __fsub_rn(__fmul_rn(dl, byte_biased<1>(v[i]) - 8388608.0f), ml);
            w[4 * i + 2] = __fsub_rn(__fmul_rn(dl, byte_biased<2>(v[i]) - 8388608.0f), ml);
            w[4 * i + 3] = __fsub_rn(__fmul_rn(dl, byte_biased<3>(v[i]) - 8388608.0f), ml);
        }
    }
};

// 2-D tiled TMA load (box of the tensor map at element (x, y)) into shared
// memory, completing its bytes on `bar`.  No multicast.
__device__ __forceinline__ void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], [%4];" ::
            "r"(smem_addr(dst)),
        "l"(reinterpret_cast<uint64_t>(map)), "r"(x), "r"(y), "r"(smem_addr(bar))
        : "memory");
}

// FP8 E4M3FN weights with f32 scales per 128 x 128 tile (gpu/fp8.vx:20-38):
// w = decode(byte) * scale, one byte per weight; only this kernel uses it.
struct FmtFP8 {
    static constexpr int kBlk = 1, kBytes = 1;
};

template <>
struct TcDecode<FmtFP8> {
    static constexpr bool kWords = true;
    // Bytes of words q and q + 4 of atom a (32 bytes) through the hardware
    // E4M3x2 -> f16x2 conversion (exact, NaN codes to NaN).  The values have
    // at most 4 significant bits, so one bf16 limb holds them exactly; the
    // tile's scale goes into the activation limbs.
    __device__ __forceinline__ static void words(const uint8_t *rc, int a, int q, float, float (&w)[8]) {
        const uint32_t *p = reinterpret_cast<const uint32_t *>(rc + a * kTcAtomCols);
        const uint32_t x[2] = {p[q], p[q + 4]};
#pragma unroll
        for (int i = 0; i < 2; ++i)
#pragma unroll
            for (int k = 0; k < 2; ++k) {
                const __half2_raw h = __nv_cvt_fp8x2_to_halfraw2(
                    static_cast<__nv_fp8x2_storage_t>((x[i] >> (16 * k)) & 0xffffu), __NV_E4M3);
                const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h));
                w[4 * i + 2 * k] = f.x;
                w[4 * i + 2 * k + 1] = f.y;
            }
    }
    __device__ __forceinline__ static void run(const uint8_t *, int, int, float (&)[16]) {}
};

// A bounded wait whose outcome is the same for every lane of the warp (the
// tensor-memory loads after it are warp-collective).
__device__ __forceinline__ bool warp_wait(uint64_t *bar, uint32_t parity) {
    const bool ok = mbar_wait_bounded(bar, parity);
    return __all_sync(0xffffffffu, ok);
}

// Shared-memory layout of a CTA (offsets from the 1 KB-aligned base).
struct TcLayout {
    int npad, chunk_cols, chunk_bytes, slots, raw_stages;
    // Weight limbs per slot (3; FP8 values are exact in one bf16).
    int a_limbs = kTcLimbs;
    // Raw stage row pitch: the chunk's bytes, plus 16 when they are a multiple
    // of 128 (otherwise every row of the box would start in the same bank);
    // the TMA box then reads 16 bytes of the next chunk (or zeros past the row).
    __host__ __device__ int raw_row() const { return chunk_bytes + ((chunk_bytes % 128) == 0 ? 16 : 0); }
    __host__ __device__ int b_tile() const { return npad * kTcRowBytes; }     // one limb of one atom
    __host__ __device__ int b_off() const { return a_limbs * kTcATile; }  // B tile within a slot
    __host__ __device__ int slot_bytes() const { return b_off() + kTcLimbs * b_tile(); }
    __host__ __device__ int raw_stage() const { return kTcRows * raw_row(); }
    __host__ __device__ int raw_off() const { return slots * slot_bytes(); }
    __host__ __device__ int bar_off() const { return (raw_off() + raw_stages * raw_stage() + 15) & ~15; }
    // raw_full[2], raw_empty[2], a_full[slots], b_full[slots], op_empty[slots], acc_full, tmem slot
    __host__ __device__ int bytes() const { return bar_off() + 8 * (4 + 3 * slots + 1) + 16; }
};

}  // namespace

// Prepared activation limbs for the tensor-core GEMM: per 32-column atom a one
// K-major core-matrix tile of 3*npad rows of 64 bytes (32 bf16), row
// l*npad + n the bf16 limb l of token n (zeros past `tokens`), at
// a * 3*npad*64.  One thread per (atom, token row, 16-byte chunk of 8 columns).
__global__ void __launch_bounds__(256)
    prep_tc_kernel(uint8_t *__restrict__ rec, const float *__restrict__ x, int tokens, int npad, int cols,
                   int xstride) {
    grid_dependency_wait();
    allow_dependent_launch();
    const int64_t id = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x;
    const int atoms = cols / kTcAtomCols;
    if (id >= static_cast<int64_t>(atoms) * npad * 4) return;
    const int c = static_cast<int>(id & 3), n = static_cast<int>((id >> 2) % npad);
    const int a = static_cast<int>((id >> 2) / npad);
    float v[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    if (n < tokens) {
        const float4 *src = reinterpret_cast<const float4 *>(x + static_cast<size_t>(n) * xstride + a * kTcAtomCols + 8 * c);
        const float4 lo4 = __ldg(src), hi4 = __ldg(src + 1);
        v[0] = lo4.x, v[1] = lo4.y, v[2] = lo4.z, v[3] = lo4.w, v[4] = hi4.x, v[5] = hi4.y, v[6] = hi4.z, v[7] = hi4.w;
    }
    uint32_t l[3][8];
#pragma unroll
    for (int e = 0; e < 8; ++e) bf16_limbs(v[e], l[0][e], l[1][e], l[2][e]);
    uint8_t *atom = rec + static_cast<size_t>(a) * kTcLimbs * npad * kTcRowBytes;
#pragma unroll
    for (int k = 0; k < kTcLimbs; ++k)
        *reinterpret_cast<uint4 *>(atom + kmajor_offset(k * npad + n, c, kTcLimbs * npad)) =
            make_uint4(pack_bf16(l[k][0], l[k][1]), pack_bf16(l[k][2], l[k][3]), pack_bf16(l[k][4], l[k][5]),
                       pack_bf16(l[k][6], l[k][7]));
}

namespace {

template <class F, int NG>
__global__ void __launch_bounds__(tc_threads(NG), NG == 1 ? 2 : 1)
    gemm_tc_kernel(const __grid_constant__ CUtensorMap wmap, float *__restrict__ out, const uint8_t *__restrict__ rec,
                   const float *__restrict__ x, int xstride,
                   int rows, int cols, int tokens, int npad, int chunk_cols, int chunk_bytes, int slots, int raw_stages,
                   int accumulate, float *__restrict__ partial, const float *__restrict__ scales, int scale_cols,
                   int *err) {
    extern __shared__ uint8_t tc_smem_raw[];
    const uint32_t raw_s = smem_addr(tc_smem_raw);
    const uint32_t pad = ((raw_s + 1023u) & ~1023u) - raw_s;  // swizzled tiles: 1 KB-aligned addresses
    uint8_t *base = tc_smem_raw + pad;
    const uint32_t base_s = raw_s + pad;
    // FP8: one weight limb; the decode warps split the activations, times
    // the tile's scale, into limbs themselves (x read from L2 one atom ahead).
    constexpr bool kFP8 = std::is_same_v<F, FmtFP8>;
    constexpr int kAL = kFP8 ? 1 : kTcLimbs;
    const TcLayout L{npad, chunk_cols, chunk_bytes, slots, raw_stages, kAL};
    uint64_t *bars = reinterpret_cast<uint64_t *>(base + L.bar_off());
    uint64_t *raw_full = bars, *raw_empty = bars + 2, *a_full = bars + 4;
    uint64_t *b_full = a_full + slots, *op_empty = b_full + slots, *acc_full = op_empty + slots;
    uint32_t *tmem_slot = reinterpret_cast<uint32_t *>(acc_full + 1);
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int row0 = blockIdx.x * kTcRows;
    const int nrows = min(kTcRows, rows - row0);
    const int chunks_all = cols / chunk_cols, apc = chunk_cols / kTcAtomCols;
    // K split (grid.y > 1): this CTA's chunks [c_begin, c_end) of the row;
    // its sums go to partial[split][token][row] for the reduction kernel.
    const int c_begin = static_cast<int>(static_cast<int64_t>(chunks_all) * blockIdx.y / gridDim.y);
    const int c_end = static_cast<int>(static_cast<int64_t>(chunks_all) * (blockIdx.y + 1) / gridDim.y);
    const int chunks = c_end - c_begin, atoms = chunks * apc;
    // 2 npad accumulator columns; the epilogue reads 32-column groups at 0 ..
    // npad and npad .. 2 npad, so at least npad + 32 columns are allocated.
    const int need = max(kTcLimbs * npad, 2 * npad + 32);
    const uint32_t tmem_cols = need <= 32 ? 32u : (need <= 64 ? 64u : (need <= 128 ? 128u : 256u));
    const uint32_t idesc1 = umma_idesc_bf16(kTcRows, npad), idesc2 = umma_idesc_bf16(kTcRows, 2 * npad),
                   idesc3 = umma_idesc_bf16(kTcRows, 3 * npad);

    if (threadIdx.x == 0) {
        for (int i = 0; i < 2; ++i) {
            mbar_init(&raw_full[i], 1);
            mbar_init(&raw_empty[i], NG * kTcGroupWarps);
        }
        for (int i = 0; i < slots; ++i) {
            mbar_init(&a_full[i], kTcGroupWarps);
            mbar_init(&b_full[i], 1);
            mbar_init(&op_empty[i], 1);
        }
        mbar_init(acc_full, 1);
        fence_mbar_init();
    }
    if (warp == 1) tmem_alloc(tmem_slot, tmem_cols);
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    allow_dependent_launch();
    const uint32_t tmem = *tmem_slot;

    if (warp == 0) {  // producer
        bool ok = true;
        int slot = 0;
        uint32_t ph = 0;  // slot and phase of atom g (counters: no division by `slots`)
        for (int c = 0; c < chunks && ok; ++c) {
            const int s = raw_stages == 1 ? 0 : (c & 1);
            const uint32_t rph = raw_stages == 1 ? (c & 1) : ((c >> 1) & 1);
            int good = 1;
            if (lane == 0) good = mbar_wait_bounded(&raw_empty[s], rph ^ 1);
            good = __shfl_sync(0xffffffffu, good, 0);
            if (!good) {
                if (lane == 0) report_device_error(err, kDevErrEmptyWait);
                break;
            }
            uint8_t *stage = base + L.raw_off() + s * L.raw_stage();
            if (lane == 0) {
                mbar_arrive_expect_tx(&raw_full[s], static_cast<uint32_t>(kTcRows * L.raw_row()));
                tma_load_2d(stage, &wmap, (c_begin + c) * (chunk_bytes / 4), row0, &raw_full[s]);
            }
            __syncwarp();
            if constexpr (kFP8) continue;  // no prepared activation records
            if (c == 0) grid_dependency_wait();  // the activation limbs come from the previous kernel
            for (int a = 0; a < apc; ++a) {
                const int g = c * apc + a;
                if (lane == 0) {
                    if (!mbar_wait_bounded(&op_empty[slot], ph ^ 1)) {
                        report_device_error(err, kDevErrEmptyWait);
                        good = 0;
                    } else {
                        uint8_t *b = base + slot * L.slot_bytes() + L.b_off();
                        mbar_arrive_expect_tx(&b_full[slot], static_cast<uint32_t>(kTcLimbs * L.b_tile()));
                        bulk_g2s(b, rec + static_cast<size_t>(c_begin * apc + g) * kTcLimbs * L.b_tile(),
                                 static_cast<uint32_t>(kTcLimbs * L.b_tile()),
                                 &b_full[slot]);
                    }
                }
                good = __shfl_sync(0xffffffffu, good, 0);
                if (!good) {
                    ok = false;
                    break;
                }
                if (++slot == slots) {
                    slot = 0;
                    ph ^= 1;
                }
            }
        }
    } else if (warp == 1) {  // MMA issue
        if (lane == 0) {
            bool ok = true;
            int slot = 0;
            uint32_t ph = 0;
            for (int g = 0; g < atoms; ++g) {
                // (FP8: the decode warps consumed b_full and built B before a_full)
                if (!mbar_wait_spin_bounded(&a_full[slot], ph) || (!kFP8 && !mbar_wait_spin_bounded(&b_full[slot], ph))) {
                    report_device_error(err, kDevErrFullWait);
                    ok = false;
                    break;
                }
                // (No tcgen05 fence here: the tiles were published through the
                // async proxy -- TMA, or fence.proxy.async before the arrive.)
                // Descriptors of the slot's tiles; a K step adds its offset >> 4
                // to the start-address field (no carry: shared addresses < 256 KB).
                // Per K step (16 columns): a1 x [b1 | b2 | b3], a2 x [b1 | b2],
                // a3 x b1 -- B rows 0 .. k*npad of the stacked limb tile -- into
                // accumulator columns 0 .. 3 npad.
                const uint64_t da = umma_desc_kmajor(base_s + slot * L.slot_bytes());
                const uint64_t db = da + (L.b_off() >> 4);
#pragma unroll
                for (int kk = 0; kk < kTcAtomCols / 16; ++kk) {  // K = 16 bf16 = 32 bytes per MMA
                    const uint64_t oa = (kk * kTcRows * 32) >> 4, ob = static_cast<uint64_t>(kk * kTcLimbs * npad * 2);
                    umma_bf16(tmem, da + oa, db + ob, idesc3, (g > 0 || kk > 0) ? 1u : 0u);
                    if constexpr (!kFP8) {
                        umma_bf16(tmem, da + (kTcATile >> 4) + oa, db + ob, idesc2, 1u);
                        umma_bf16(tmem, da + ((2 * kTcATile) >> 4) + oa, db + ob, idesc1, 1u);
                    }
                }
                umma_commit(&op_empty[slot]);
                if (++slot == slots) {
                    slot = 0;
                    ph ^= 1;
                }
            }
            if (ok) umma_commit(acc_full);
        }
        __syncwarp();
    } else {  // decode (two groups of 8 warps, alternate atoms), then (warps 2-5) the epilogue
        const int grp = (warp - 2) / kTcGroupWarps, gt = threadIdx.x - 64 - grp * kTcGroupWarps * 32;
        const int r = gt >> 1, h = gt & 1;  // a thread: 16 weights of one tile row
        bool ok = true;
        int slot = grp;  // slot and phase of this group's atom g = grp, grp + NG, ... (NG <= slots)
        uint32_t ph = 0;
        // FP8: activations (token xn, columns 8 xq .. 8 xq + 7 of the atom; zeros
        // past the tokens) and the atom's scale, fetched one atom ahead.  A
        // quarter-warp takes 8 consecutive tokens of one column quarter, so its
        // 16-byte limb stores fill one 128-byte core matrix (no bank conflict).
        const int xn = (gt & 7) | ((gt >> 5) << 3), xq = (gt >> 3) & 3;
        const bool xact = kFP8 && gt < npad * 4 && xn < tokens;
        float4 xr0 = make_float4(0.f, 0.f, 0.f, 0.f), xr1 = xr0;
        float scr = 0.0f;
        auto fetch = [&](int g) {
            if constexpr (kFP8) {
                if (g < atoms) {
                    const int col = (c_begin * apc + g) * kTcAtomCols;
                    scr = __ldg(scales + static_cast<size_t>(blockIdx.x) * scale_cols + col / 128);
                    if (xact) {
                        const float4 *src = reinterpret_cast<const float4 *>(x + static_cast<size_t>(xn) * xstride + col + 8 * xq);
                        xr0 = __ldg(src);
                        xr1 = __ldg(src + 1);
                    }
                }
            }
        };
        if constexpr (kFP8) {
            grid_dependency_wait();  // x comes from the previous kernel
            fetch(grp);
        }
        for (int c = 0; c < chunks && ok; ++c) {
            const int s = raw_stages == 1 ? 0 : (c & 1);
            if (!warp_wait(&raw_full[s], raw_stages == 1 ? (c & 1) : ((c >> 1) & 1))) {
                if (lane == 0) report_device_error(err, kDevErrFullWait);
                ok = false;
                break;
            }
            const int raw_row = L.raw_row();
            const uint8_t *rc = base + L.raw_off() + s * L.raw_stage() + r * raw_row;
            for (int a = grp; a < apc; a += NG) {
                const int g = c * apc + a;
                const float4 x0 = xr0, x1 = xr1;
                const float scale = scr;  // FP8: this tile's scale (rows 128*blockIdx.x.., the atom's columns)
                fetch(g + NG);
                if (!warp_wait(&op_empty[slot], ph ^ 1)) {
                    if (lane == 0) report_device_error(err, kDevErrEmptyWait);
                    ok = false;
                    break;
                }
                uint8_t *at = base + slot * L.slot_bytes();
                if constexpr (TcDecode<F>::kWords) {
                    // lane = (row j, quarter q) of 8 rows per warp, two passes of
                    // 64 rows: conflict-free 4-byte raw loads and 8-byte stores
                    // (a half-warp covers 8 rows x both word parities)
                    const int wj = lane & 7, wq = lane >> 3, wg = (warp - 2) % kTcGroupWarps;
                    const uint8_t *stage = rc - r * raw_row;
#pragma unroll
                    for (int pass = 0; pass < 2; ++pass) {
                        const int rr = pass * 64 + wg * 8 + wj;
                        float v[8];
                        if (rr < nrows) {
                            TcDecode<F>::words(stage + rr * raw_row, a, wq, scale, v);
                        } else {
#pragma unroll
                            for (int e = 0; e < 8; ++e) v[e] = 0.0f;
                        }
#pragma unroll
                        for (int hw = 0; hw < 2; ++hw) {  // word wq, then wq + 4
                            const int wd = wq + 4 * hw;   // K positions 4wd .. 4wd+3
                            uint32_t l[3][4];
#pragma unroll
                            for (int e = 0; e < 4; ++e) bf16_limbs(v[4 * hw + e], l[0][e], l[1][e], l[2][e]);
                            const uint32_t off = kmajor_offset(rr, wd >> 1, kTcRows) + 8 * (wd & 1);
#pragma unroll
                            for (int k = 0; k < kAL; ++k)
                                *reinterpret_cast<uint2 *>(at + k * kTcATile + off) =
                                    make_uint2(pack_bf16(l[k][0], l[k][1]), pack_bf16(l[k][2], l[k][3]));
                        }
                    }
                } else {
                    float v[16];
                    if (r < nrows) {
                        TcDecode<F>::run(rc, a, h, v);
                    } else {
#pragma unroll
                        for (int e = 0; e < 16; ++e) v[e] = 0.0f;
                    }
#pragma unroll
                    for (int i = 0; i < 2; ++i) {  // 8 weights -> one 16-byte chunk per limb
                        uint32_t l[3][8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) bf16_limbs(v[8 * i + e], l[0][e], l[1][e], l[2][e]);
                        const uint32_t off = kmajor_offset(r, 2 * h + i, kTcRows);
#pragma unroll
                        for (int k = 0; k < kAL; ++k)
                            *reinterpret_cast<uint4 *>(at + k * kTcATile + off) =
                                make_uint4(pack_bf16(l[k][0], l[k][1]), pack_bf16(l[k][2], l[k][3]),
                                           pack_bf16(l[k][4], l[k][5]), pack_bf16(l[k][6], l[k][7]));
                    }
                }
                if constexpr (kFP8) {
                    // B = (x * scale) in three bf16 limbs, stacked as the prepared
                    // records of prep_tc_kernel: one (token, 8 columns) per thread
                    // (npad * 4 <= 256 threads).
                    if (gt < npad * 4) {
                        const float xv[8] = {x0.x, x0.y, x0.z, x0.w, x1.x, x1.y, x1.z, x1.w};
                        uint32_t l[3][8];
#pragma unroll
                        for (int e = 0; e < 8; ++e) bf16_limbs(__fmul_rn(xv[e], scale), l[0][e], l[1][e], l[2][e]);
                        uint8_t *bt = at + L.b_off();
#pragma unroll
                        for (int k = 0; k < kTcLimbs; ++k)
                            *reinterpret_cast<uint4 *>(bt + kmajor_offset(k * npad + xn, xq, kTcLimbs * npad)) =
                                make_uint4(pack_bf16(l[k][0], l[k][1]), pack_bf16(l[k][2], l[k][3]),
                                           pack_bf16(l[k][4], l[k][5]), pack_bf16(l[k][6], l[k][7]));
                    }
                }
                fence_proxy_async_smem();  // generic-proxy stores -> the tensor cores' async proxy
                __syncwarp();
                if (lane == 0) mbar_arrive(&a_full[slot]);
                if ((slot += NG) >= slots) {
                    slot -= slots;
                    ph ^= 1;
                }
            }
            __syncwarp();
            if (lane == 0 && ok) mbar_arrive(&raw_empty[s]);
        }
        if (warp < 6) {  // one warp per tensor-memory lane quarter: rows 32*(warp%4) ..
            const bool got = ok && warp_wait(acc_full, 0);
            if (ok && !got && lane == 0) report_device_error(err, kDevErrFullWait);
            tc_fence_after();
            grid_dependency_wait();  // `out` may be read or written by the previous kernel
            const int q = warp & 3, r = 32 * q + lane;
            for (int c0 = 0; c0 < npad && got; c0 += 32) {
                // columns t (a1 b1 + a2 b1 + a3 b1), npad + t (a1 b2 + a2 b2), 2 npad + t (a1 b3)
                float v[32];
                uint32_t u[32];
                tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(c0), u);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] = __uint_as_float(u[j]);
                tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(npad + c0), u);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += __uint_as_float(u[j]);
                tmem_ld32(tmem + (static_cast<uint32_t>(32 * q) << 16) + static_cast<uint32_t>(2 * npad + c0), u);
#pragma unroll
                for (int j = 0; j < 32; ++j) v[j] += __uint_as_float(u[j]);
                if (r < nrows) {
                    if (gridDim.y > 1) {
                        float *o = partial + static_cast<size_t>(blockIdx.y) * tokens * rows + row0 + r;
#pragma unroll
                        for (int j = 0; j < 32; ++j)
                            if (c0 + j < tokens) o[static_cast<size_t>(c0 + j) * rows] = v[j];
                    } else {
                        float *o = out + row0 + r;
#pragma unroll
                        for (int j = 0; j < 32; ++j) {
                            const int t = c0 + j;
                            if (t < tokens) {
                                float *d = o + static_cast<size_t>(t) * rows;
                                const float val = v[j];
                                *d = accumulate ? *d + val : val;
                            }
                        }
                    }
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) tmem_dealloc(tmem, tmem_cols);
}

// out[t][r] (+)= sum over splits, in split order, of partial[split][t][r].
__global__ void __launch_bounds__(256)
    tc_split_reduce_kernel(float *__restrict__ out, const float *__restrict__ partial, int64_t n, int splits,
                           int accumulate) {
    grid_dependency_wait();
    allow_dependent_launch();
    for (int64_t i = static_cast<int64_t>(blockIdx.x) * blockDim.x + threadIdx.x; i < n;
         i += static_cast<int64_t>(gridDim.x) * blockDim.x) {
        float v = partial[i];
        for (int k = 1; k < splits; ++k) v += partial[static_cast<int64_t>(k) * n + i];
        out[i] = accumulate ? out[i] + v : v;
    }
}

}  // namespace

namespace {

// budget: kTcSmemBudget (one CTA per SM, two decode groups) or kTcSmemHalf
// (two CTAs per SM, one group each).
template <class F>
bool plan_tc(int cols, int batch, TcLayout &L, size_t &smem, int budget = kTcSmemBudget) {
    const int chunk = tc_chunk_cols(F::kBlk, F::kBytes);
    if (!chunk || cols <= 0 || cols % chunk || batch < 1 || batch > kTcMaxTokens) return false;
    L.npad = (batch + 15) / 16 * 16;
    L.a_limbs = std::is_same_v<F, FmtFP8> ? 1 : kTcLimbs;
    L.chunk_cols = chunk;
    L.chunk_bytes = chunk / F::kBlk * F::kBytes;
    // Two raw stages (loads overlap decoding) where they fit, else one.
    for (int rs = 2; rs >= 1; --rs)
        for (int sl = 4; sl >= 2; --sl) {
            L.slots = sl;
            L.raw_stages = rs;
            if (static_cast<size_t>(L.bytes()) + 1024 <= static_cast<size_t>(budget)) {
                smem = static_cast<size_t>(L.bytes()) + 1024;  // + alignment slack of the 1 KB base
                return true;
            }
        }
    return false;
}

using EncodeTiledFn = CUresult (*)(CUtensorMap *, CUtensorMapDataType, cuuint32_t, void *, const cuuint64_t *,
                                   const cuuint64_t *, const cuuint32_t *, const cuuint32_t *, CUtensorMapInterleave,
                                   CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

// The driver's cuTensorMapEncodeTiled through the runtime (the library links
// no libcuda); looked up once, in relaxed capture mode (safe during a graph
// capture).
EncodeTiledFn encode_tiled() {
    static const EncodeTiledFn fn = [] {
        cudaStreamCaptureMode mode = cudaStreamCaptureModeRelaxed;
        cudaThreadExchangeStreamCaptureMode(&mode);
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q = cudaDriverEntryPointSymbolNotFound;
        const cudaError_t e = cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q);
        cudaThreadExchangeStreamCaptureMode(&mode);
        return (e == cudaSuccess && q == cudaDriverEntryPointSuccess) ? reinterpret_cast<EncodeTiledFn>(p) : nullptr;
    }();
    return fn;
}

}  // namespace

bool gemm_tc_supported(int kind, int cols, int batch) {
    bool ok = false;
    dispatch_format(kind, [&]<class F>() {
        TcLayout L{};
        size_t smem = 0;
        ok = plan_tc<F>(cols, batch, L, smem);
    });
    return ok;
}

namespace {

// Launch shape: two CTAs per SM (one decode group) where shared memory
// allows, else one with two groups; when the 128-row tiles leave SMs idle,
// each tile's chunks are split over grid.y CTAs (whole chunks, at least 512
// columns each) whose partial sums a reduction adds in split order.
struct TcShape {
    TcLayout L{};
    size_t smem = 0;
    bool pair = false;
    int splits = 1;
    size_t rec_bytes = 0, scratch_bytes = 0;
};

template <class F>
bool shape_tc(int rows, int cols, int batch, TcShape &sh) {
    sh.pair = plan_tc<F>(cols, batch, sh.L, sh.smem, kTcSmemHalf);
    if (!sh.pair && !plan_tc<F>(cols, batch, sh.L, sh.smem)) return false;
    const int tiles = (rows + kTcRows - 1) / kTcRows, chunks = cols / sh.L.chunk_cols;
    const int slots = sm_count() * (sh.pair ? 2 : 1);
    // Whole chunks, at least 16 atoms (512 columns) per split; the split count
    // minimising waves x atoms per CTA (a CTA's time is its chain of atoms).
    // Only when the tiles leave CTA slots idle (the partial sums cost a
    // write and a read of splits x tokens x rows floats).
    const int by_atoms = tiles >= slots ? 1 : std::max(1, std::min(chunks, cols / kTcAtomCols / 16));
    int64_t best = -1;
    for (int sp = 1; sp <= by_atoms; ++sp) {
        const int64_t waves = (static_cast<int64_t>(tiles) * sp + slots - 1) / slots;
        const int64_t cost = waves * ((chunks + sp - 1) / sp);
        if (best < 0 || cost < best) {
            best = cost;
            sh.splits = sp;
        }
    }
    sh.rec_bytes = std::is_same_v<F, FmtFP8>
                       ? 0  // FP8 builds its activation limbs in the kernel
                       : (static_cast<size_t>(cols / kTcAtomCols) * kTcLimbs * sh.L.npad * kTcRowBytes + 255) & ~size_t(255);
    sh.scratch_bytes = sh.rec_bytes + (sh.splits > 1 ? static_cast<size_t>(sh.splits) * batch * rows * 4 : 0);
    return true;
}

}  // namespace

size_t gemm_tc_scratch_bytes(int32_t kind, int rows, int cols, int batch) {
    size_t bytes = 0;
    dispatch_format(kind, [&]<class F>() {
        TcShape sh;
        if (shape_tc<F>(rows, cols, batch, sh)) bytes = sh.scratch_bytes;
    });
    return bytes;
}

namespace {

// Prepare the activation limbs and launch the GEMM (plus the split
// reduction) for format F; `scales` / `scale_cols` for FmtFP8 only.
template <class F>
int32_t launch_tc(float *out, const uint8_t *w, const float *x, int rows, int cols, int batch, uint8_t *scratch,
                  cudaStream_t stream, int64_t row_bytes, int64_t pitch, int xstride, bool accumulate,
                  const float *scales, int scale_cols) {
    // Two CTAs per SM with one decode group each where their shared memory
    // fits half an SM (two MMA-issuing threads keep the tensor core busier
    // than one), else one CTA with two groups; K split over idle SMs.
    TcShape sh;
    if (!shape_tc<F>(rows, cols, batch, sh)) {
        set_error("gemm_tc: no launch plan for this shape");
        return kUnsupported;
    }
    const TcLayout &L = sh.L;
    // The weights as a 2-D tensor of 4-byte elements: rows x (row bytes / 4),
    // row pitch `pitch` bytes; one box = 128 rows x one raw stage row.
    const EncodeTiledFn encode = encode_tiled();
    if (!encode) {
        set_error("gemm_tc: cuTensorMapEncodeTiled is not available");
        return kUnsupported;
    }
    CUtensorMap wmap;
    const cuuint64_t dims[2] = {static_cast<cuuint64_t>(row_bytes / 4), static_cast<cuuint64_t>(rows)};
    const cuuint64_t strides[1] = {static_cast<cuuint64_t>(pitch)};
    const cuuint32_t box[2] = {static_cast<cuuint32_t>(L.raw_row() / 4), static_cast<cuuint32_t>(kTcRows)};
    const cuuint32_t estr[2] = {1, 1};
    const CUresult ce = encode(&wmap, CU_TENSOR_MAP_DATA_TYPE_UINT32, 2, const_cast<uint8_t *>(w), dims, strides, box,
                               estr, CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_NONE,
                               CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE);
    if (ce != CUDA_SUCCESS) {
        set_error("gemm_tc: cuTensorMapEncodeTiled failed (%d)", static_cast<int>(ce));
        return kInvalid;
    }
    constexpr bool kFP8 = std::is_same_v<F, FmtFP8>;
    auto kern = sh.pair ? gemm_tc_kernel<F, 1> : gemm_tc_kernel<F, 2>;
    if (const int32_t rc = allow_dynamic_smem(kern, sh.smem, "gemm_tc smem")) return rc;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    const int64_t threads = static_cast<int64_t>(cols / kTcAtomCols) * L.npad * 4;
    cudaLaunchConfig_t pc = {};
    pc.gridDim = dim3(static_cast<unsigned>((threads + 255) / 256));
    pc.blockDim = dim3(256);
    pc.stream = stream;
    pc.attrs = attr;
    pc.numAttrs = 1;
    if constexpr (!kFP8) GLMVX_CUDA(cudaLaunchKernelEx(&pc, prep_tc_kernel, scratch, x, batch, L.npad, cols, xstride));
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(static_cast<unsigned>((rows + kTcRows - 1) / kTcRows), static_cast<unsigned>(sh.splits));
    cfg.blockDim = dim3(tc_threads(sh.pair ? 1 : 2));
    cfg.dynamicSmemBytes = sh.smem;
    cfg.stream = stream;
    cfg.attrs = attr;
    cfg.numAttrs = 1;
    GLMVX_CUDA(cudaLaunchKernelEx(&cfg, kern, wmap, out, static_cast<const uint8_t *>(scratch), x, xstride, rows, cols,
                                  batch, L.npad,
                                  L.chunk_cols, L.chunk_bytes, L.slots, L.raw_stages, static_cast<int>(accumulate),
                                  reinterpret_cast<float *>(scratch + sh.rec_bytes), scales, scale_cols,
                                  device_error_word()));
    if (sh.splits > 1) {
        const int64_t n = static_cast<int64_t>(batch) * rows;
        cudaLaunchConfig_t rc = {};
        rc.gridDim = dim3(static_cast<unsigned>(std::min<int64_t>((n + 255) / 256, 4 * sm_count())));
        rc.blockDim = dim3(256);
        rc.stream = stream;
        rc.attrs = attr;
        rc.numAttrs = 1;
        GLMVX_CUDA(cudaLaunchKernelEx(&rc, tc_split_reduce_kernel, out,
                                      reinterpret_cast<const float *>(scratch + sh.rec_bytes), n, sh.splits,
                                      static_cast<int>(accumulate)));
    }
    return kOk;
}

bool aligned16(const void *a, const void *b, const void *c) {
    return ((reinterpret_cast<uintptr_t>(a) | reinterpret_cast<uintptr_t>(b) | reinterpret_cast<uintptr_t>(c)) & 15) == 0;
}

}  // namespace

int32_t gemm_tc_device(int32_t kind, float *out, const uint8_t *w, const float *x, int rows, int cols, int batch,
                       uint8_t *scratch, cudaStream_t stream, const ColSegment &seg) {
    int blk = 0, bytes = 0;
    if (!reference_layout(kind, blk, bytes) || rows <= 0 || cols <= 0 || cols % blk) {
        set_error("gemm_tc: unsupported format or shape");
        return kUnsupported;
    }
    const int64_t row_bytes = static_cast<int64_t>(cols / blk) * bytes;
    const int64_t pitch = seg.pitch ? seg.pitch : row_bytes;
    const int xstride = seg.xstride ? seg.xstride : cols;
    if (!aligned16(w, x, scratch) || pitch % 16 || pitch < row_bytes || xstride < cols || xstride % 4) {
        set_error("gemm_tc: weights, activations and scratch 16-byte aligned, row pitch a multiple of 16");
        return kInvalid;
    }
    int32_t st = kUnsupported;
    dispatch_format(kind, [&]<class F>() {
        st = launch_tc<F>(out, w, x, rows, cols, batch, scratch, stream, row_bytes, pitch, xstride, seg.accumulate,
                          nullptr, 0);
    });
    return st;
}

bool fp8_gemm_tc_supported(int cols, int batch) {
    TcShape sh;
    return cols % 256 == 0 && shape_tc<FmtFP8>(128, cols, batch, sh);
}

size_t fp8_gemm_tc_scratch_bytes(int rows, int cols, int batch) {
    TcShape sh;
    return shape_tc<FmtFP8>(rows, cols, batch, sh) ? sh.scratch_bytes : 0;
}

int32_t fp8_gemm_tc_device(float *out, const uint8_t *w, const float *scales, const float *x, int rows, int cols,
                           int batch, uint8_t *scratch, cudaStream_t stream) {
    if (rows <= 0 || cols <= 0 || cols % 256 || batch < 1 || batch > kTcMaxTokens) {
        set_error("fp8 gemm: rows >= 1, columns a multiple of 256, 1..64 tokens");
        return kUnsupported;
    }
    if (!aligned16(w, x, scratch) || (reinterpret_cast<uintptr_t>(scales) & 3)) {
        set_error("fp8 gemm: weights, activations and scratch 16-byte aligned");
        return kInvalid;
    }
    return launch_tc<FmtFP8>(out, w, x, rows, cols, batch, scratch, stream, cols, cols, cols, false, scales,
                             (cols + 127) / 128);
}

}  // namespace glmvx
