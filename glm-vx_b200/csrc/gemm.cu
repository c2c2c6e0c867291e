// Dense f32 GEMM C[M,N] = A[M,K] B[K,N], row-major, the contract of the
// reference's resident GEMM (GEMMKernels.gemm, gpu/gemm.py:51-97; kernels
// gpu/gemm.vx:14-73 tf32, :75ff f32):
//   precision "tf32_rna": every multiplicand rounded to TF32 (nearest, ties
//   away from zero), products accumulated in f32 on the tensor cores;
//   precision "f32": f32 multiply-adds.
// Any M, N, K >= 0 (K = 0 writes zeros), any 4-byte alignment.
//
// tf32_rna on the 5th-generation tensor cores: a CTA owns a 128 x 256 tile
// of C whose f32 accumulators live in tensor memory (128 lanes x 256
// columns).  Per 32-wide K block its 256 threads load A [128 x 32] and B
// [32 x 256] from global memory into registers (the next block's loads are
// in flight while the current one is stored), round them (cvt.rna.tf32) and
// store them in shared memory as K-major 128-byte-swizzled tiles (row r of a
// tile at (r/8)*1024 + (r%8)*128 bytes, 16-byte chunk c at position
// c ^ (r%8): the canonical SWIZZLE_128B K-major layout of the UMMA
// descriptors; B is transposed on the way); one thread then issues four
// tcgen05.mma kind::tf32 (M=128, N=256, K=8) and commits them to the stage's
// mbarrier.  Three stages.  The epilogue reads the accumulators with
// tcgen05.ld (warp w owns lanes 32*(w%4).. i.e. rows, and half the columns)
// and writes C.
#include <cstdint>

#include "common.cuh"
#include "tcgen05.cuh"

namespace glmvx {

namespace {

constexpr int kGemmBM = 128, kGemmBN = 256, kGemmBK = 32, kGemmStages = 3, kGemmThreads = 256;
constexpr int kGemmABytes = kGemmBM * kGemmBK * 4, kGemmBBytes = kGemmBN * kGemmBK * 4;  // 16 KB, 32 KB
constexpr int kGemmStageBytes = kGemmABytes + kGemmBBytes;
constexpr int kGemmSmem = kGemmStages * kGemmStageBytes + 1024;  // + alignment slack
constexpr uint32_t kGemmTmemCols = kGemmBN;

constexpr uint32_t kGemmIdesc = umma_idesc_tf32(kGemmBM, kGemmBN);

// One K block of a CTA's operands in registers: A chunks (row, 4 k) and B
// blocks (4 k x 4 n), loaded while the previous block is stored and multiplied.
// VEC: K and N multiples of 4 and A, B 16-byte aligned (float4 loads, whole
// chunks in or out of range); otherwise scalar loads with per-element bounds.
constexpr int kGemmAPer = kGemmBM * 8 / kGemmThreads, kGemmBPer = kGemmBN * 8 / (4 * kGemmThreads);

template <bool VEC>
__device__ __forceinline__ void gemm_load(float4 (&ra)[kGemmAPer], float4 (&rb)[kGemmBPer][4], const float *A,
                                          const float *B, int M, int N, int K, int m0, int n0, int k0, int tid) {
#pragma unroll
    for (int i = 0; i < kGemmAPer; ++i) {
        const int q = tid + kGemmThreads * i, r = q >> 3, c = q & 7, m = m0 + r, k = k0 + 4 * c;
        const float *src = A + static_cast<int64_t>(m) * K + k;
        if (VEC) {
            ra[i] = (m < M && k < K) ? __ldg(reinterpret_cast<const float4 *>(src)) : make_float4(0.f, 0.f, 0.f, 0.f);
        } else {
            ra[i].x = (m < M && k < K) ? __ldg(src) : 0.0f;
            ra[i].y = (m < M && k + 1 < K) ? __ldg(src + 1) : 0.0f;
            ra[i].z = (m < M && k + 2 < K) ? __ldg(src + 2) : 0.0f;
            ra[i].w = (m < M && k + 3 < K) ? __ldg(src + 3) : 0.0f;
        }
    }
#pragma unroll
    for (int i = 0; i < kGemmBPer; ++i) {
        // block (k quad kq, n quad nq): a warp covers 32 consecutive n quads of one k quad
        const int q = tid + kGemmThreads * i, nq = q % (kGemmBN / 4), kq = q / (kGemmBN / 4);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const int k = k0 + 4 * kq + e, n = n0 + 4 * nq;
            const float *src = B + static_cast<int64_t>(k) * N + n;
            if (VEC) {
                rb[i][e] = (k < K && n < N) ? __ldg(reinterpret_cast<const float4 *>(src))
                                            : make_float4(0.f, 0.f, 0.f, 0.f);
            } else {
                rb[i][e].x = (k < K && n < N) ? __ldg(src) : 0.0f;
                rb[i][e].y = (k < K && n + 1 < N) ? __ldg(src + 1) : 0.0f;
                rb[i][e].z = (k < K && n + 2 < N) ? __ldg(src + 2) : 0.0f;
                rb[i][e].w = (k < K && n + 3 < N) ? __ldg(src + 3) : 0.0f;
            }
        }
    }
}

// Rounded to TF32 and stored as the stage's swizzled K-major tiles (B as B^T).
__device__ __forceinline__ void gemm_store(uint8_t *as, uint8_t *bs, const float4 (&ra)[kGemmAPer],
                                           const float4 (&rb)[kGemmBPer][4], int tid) {
#pragma unroll
    for (int i = 0; i < kGemmAPer; ++i) {
        const int q = tid + kGemmThreads * i;
        *reinterpret_cast<uint4 *>(as + sw128_offset(q >> 3, q & 7)) =
            make_uint4(tf32_rna(ra[i].x), tf32_rna(ra[i].y), tf32_rna(ra[i].z), tf32_rna(ra[i].w));
    }
#pragma unroll
    for (int i = 0; i < kGemmBPer; ++i) {
        const int q = tid + kGemmThreads * i, nq = q % (kGemmBN / 4), kq = q / (kGemmBN / 4);
        // column j of the 4x4 block is row n = 4nq + j of B^T, K chunk kq
        *reinterpret_cast<uint4 *>(bs + sw128_offset(4 * nq, kq)) = make_uint4(
            tf32_rna(rb[i][0].x), tf32_rna(rb[i][1].x), tf32_rna(rb[i][2].x), tf32_rna(rb[i][3].x));
        *reinterpret_cast<uint4 *>(bs + sw128_offset(4 * nq + 1, kq)) = make_uint4(
            tf32_rna(rb[i][0].y), tf32_rna(rb[i][1].y), tf32_rna(rb[i][2].y), tf32_rna(rb[i][3].y));
        *reinterpret_cast<uint4 *>(bs + sw128_offset(4 * nq + 2, kq)) = make_uint4(
            tf32_rna(rb[i][0].z), tf32_rna(rb[i][1].z), tf32_rna(rb[i][2].z), tf32_rna(rb[i][3].z));
        *reinterpret_cast<uint4 *>(bs + sw128_offset(4 * nq + 3, kq)) = make_uint4(
            tf32_rna(rb[i][0].w), tf32_rna(rb[i][1].w), tf32_rna(rb[i][2].w), tf32_rna(rb[i][3].w));
    }
}

template <bool VEC>
__global__ void __launch_bounds__(kGemmThreads, 1)
    gemm_tf32_kernel(float *__restrict__ C, const float *__restrict__ A, const float *__restrict__ B, int M, int N,
                     int K, int *err) {
    extern __shared__ uint8_t gemm_smem_raw[];
    __shared__ uint64_t mma_done[kGemmStages];
    __shared__ uint32_t tmem_slot;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const uint32_t raw = smem_addr(gemm_smem_raw);
    const uint32_t pad = ((raw + 1023u) & ~1023u) - raw;  // the swizzle works on address bits: 1 KB-aligned tiles
    uint8_t *tiles = gemm_smem_raw + pad;
    const uint32_t tiles_s = raw + pad;
    const int m0 = blockIdx.y * kGemmBM, n0 = blockIdx.x * kGemmBN;

    if (warp == 0) {
        tmem_alloc(&tmem_slot, kGemmTmemCols);
    }
    if (tid == 0) {
        for (int s = 0; s < kGemmStages; ++s) mbar_init(&mma_done[s], 1);
        fence_mbar_init();
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;

    const int nk = (K + kGemmBK - 1) / kGemmBK;
    bool ok = true;
    float4 ra[kGemmAPer], rb[kGemmBPer][4];
    if (nk > 0) gemm_load<VEC>(ra, rb, A, B, M, N, K, m0, n0, 0, tid);
    for (int kb = 0; kb < nk; ++kb) {
        const int s = kb % kGemmStages;
        if (kb >= kGemmStages) ok = mbar_wait_bounded(&mma_done[s], ((kb - kGemmStages) / kGemmStages) & 1);
        if (!__syncthreads_and(ok)) {  // the stage is still read by MMAs that did not finish
            if (tid == 0) report_device_error(err, kDevErrFullWait);
            ok = false;
            break;
        }
        uint8_t *as = tiles + s * kGemmStageBytes;
        gemm_store(as, as + kGemmABytes, ra, rb, tid);
        if (kb + 1 < nk) gemm_load<VEC>(ra, rb, A, B, M, N, K, m0, n0, (kb + 1) * kGemmBK, tid);
        // Generic-proxy stores become visible to the tensor cores' async proxy.
        fence_proxy_async_smem();
        __syncthreads();
        if (tid == 0) {
            tc_fence_after();
            const uint32_t a_s = tiles_s + s * kGemmStageBytes, b_s = a_s + kGemmABytes;
#pragma unroll
            for (int kk = 0; kk < kGemmBK / 8; ++kk)  // K = 8 tf32 = 32 bytes per MMA
                umma_tf32(tmem, umma_desc_sw128(a_s + 32 * kk), umma_desc_sw128(b_s + 32 * kk), kGemmIdesc,
                          (kb > 0 || kk > 0) ? 1u : 0u);
            umma_commit(&mma_done[s]);
        }
    }
    if (ok && nk > 0) {
        const int last = nk - 1;
        ok = mbar_wait_bounded(&mma_done[last % kGemmStages], (last / kGemmStages) & 1);
        if (!ok && lane == 0) report_device_error(err, kDevErrFullWait);
    }
    ok = __syncthreads_and(ok);
    tc_fence_after();
    // Epilogue: warp w reads tensor-memory lanes 32*(w%4).. (rows) and the
    // column half w/4; zeros when K == 0.
    const int row = m0 + 32 * (warp & 3) + lane, cbase = 128 * (warp >> 2);
    const bool vec_out = VEC && (reinterpret_cast<uintptr_t>(C) & 15) == 0;
#pragma unroll 1
    for (int c0 = cbase; c0 < cbase + 128; c0 += 32) {
        uint32_t v[32];
        if (nk > 0 && ok) {
            tmem_ld32(tmem + (static_cast<uint32_t>(32 * (warp & 3)) << 16) + c0, v);
        } else {
#pragma unroll
            for (int j = 0; j < 32; ++j) v[j] = 0u;
        }
        if (row < M && ok) {
            float *crow = C + static_cast<int64_t>(row) * N + n0 + c0;
            if (vec_out && n0 + c0 + 32 <= N) {
#pragma unroll
                for (int j = 0; j < 32; j += 4)
                    *reinterpret_cast<float4 *>(crow + j) = make_float4(
                        __uint_as_float(v[j]), __uint_as_float(v[j + 1]), __uint_as_float(v[j + 2]),
                        __uint_as_float(v[j + 3]));
            } else {
#pragma unroll
                for (int j = 0; j < 32; ++j)
                    if (n0 + c0 + j < N) crow[j] = __uint_as_float(v[j]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 0)
        tmem_dealloc(tmem, kGemmTmemCols);
}

// precision "f32": 64 x 64 tile per CTA, 16 x 16 threads with 4 x 4
// outputs each, K in blocks of 16 through shared memory; each output an
// ordered chain of f32 fused multiply-adds over k.
constexpr int kSgemmTile = 64, kSgemmBK = 16;

__global__ void __launch_bounds__(256)
    gemm_f32_kernel(float *__restrict__ C, const float *__restrict__ A, const float *__restrict__ B, int M, int N,
                    int K) {
    __shared__ float as[kSgemmBK][kSgemmTile + 4], bs[kSgemmBK][kSgemmTile + 4];
    const int tx = threadIdx.x & 15, ty = threadIdx.x >> 4;
    const int m0 = blockIdx.y * kSgemmTile, n0 = blockIdx.x * kSgemmTile;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += kSgemmBK) {
        for (int i = threadIdx.x; i < kSgemmTile * kSgemmBK; i += 256) {
            const int r = i / kSgemmBK, k = i % kSgemmBK;  // A tile: row r, column k
            as[k][r] = (m0 + r < M && k0 + k < K) ? __ldg(A + static_cast<int64_t>(m0 + r) * K + k0 + k) : 0.0f;
            const int kb = i / kSgemmTile, n = i % kSgemmTile;  // B tile: row kb, column n
            bs[kb][n] = (k0 + kb < K && n0 + n < N) ? __ldg(B + static_cast<int64_t>(k0 + kb) * N + n0 + n) : 0.0f;
        }
        __syncthreads();
#pragma unroll
        for (int k = 0; k < kSgemmBK; ++k) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) {
                a[i] = as[k][ty + 16 * i];
                b[i] = bs[k][tx + 16 * i];
            }
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int m = m0 + ty + 16 * i, n = n0 + tx + 16 * j;
            if (m < M && n < N) C[static_cast<int64_t>(m) * N + n] = acc[i][j];
        }
}

}  // namespace

}  // namespace glmvx

using namespace glmvx;

// precision 0 = "f32", 1 = "tf32_rna" (gpu/gemm.py:24-47).  C must not
// overlap A or B.  *err (device int32; NULL: the library's device error
// word) records a tensor-core wait that timed out.
GLMVX_EXPORT int32_t glmvx_gemm(float *C, const float *A, const float *B, int32_t M, int32_t N, int32_t K,
                                int32_t precision, int32_t *err, void *stream) {
    if (M < 0 || N < 0 || K < 0) {
        set_error("gemm: dimensions must be >= 0");
        return kInvalid;
    }
    if (precision != 0 && precision != 1) {
        set_error("precision must be 'f32' or explicit 'tf32_rna'");
        return kInvalid;
    }
    if (M == 0 || N == 0) return kOk;
    if (!err) err = device_error_word();
    if (!C || (K > 0 && (!A || !B))) {
        set_error("gemm: null pointer");
        return kInvalid;
    }
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    if (precision == 0) {
        const dim3 grid((N + kSgemmTile - 1) / kSgemmTile, (M + kSgemmTile - 1) / kSgemmTile);
        gemm_f32_kernel<<<grid, 256, 0, st>>>(C, A, B, M, N, K);
    } else {
        if (const int32_t rc = allow_dynamic_smem(gemm_tf32_kernel<true>, kGemmSmem, "gemm smem")) return rc;
        if (const int32_t rc = allow_dynamic_smem(gemm_tf32_kernel<false>, kGemmSmem, "gemm smem")) return rc;
        const bool vec = K % 4 == 0 && N % 4 == 0 &&
                         ((reinterpret_cast<uintptr_t>(A) | reinterpret_cast<uintptr_t>(B)) & 15) == 0;
        const dim3 grid((N + kGemmBN - 1) / kGemmBN, (M + kGemmBM - 1) / kGemmBM);
        if (vec) gemm_tf32_kernel<true><<<grid, kGemmThreads, kGemmSmem, st>>>(C, A, B, M, N, K, err);
        else gemm_tf32_kernel<false><<<grid, kGemmThreads, kGemmSmem, st>>>(C, A, B, M, N, K, err);
    }
    GLMVX_CUDA(cudaGetLastError());
    return kOk;
}
