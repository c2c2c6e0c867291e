// The reference's CPU C ABI (kernels/kernels.h:12-53), served by the B200.
//
// Every glm_vx_* symbol the reference's Python boundary binds through ctypes
// (kernels/packed.py:80-83,96-98,148-150; kernels/backend.py:61-75) is
// exported here with the same signature and the same status convention
// (0 = ok, -1 = rejected arguments), taking HOST pointers.  Each call copies
// its host inputs to the device, runs the sm_100a kernel and copies the
// result back before returning, so a library loaded through GLM_VX_LIBRARY
// is a drop-in for libglm_vx.so.  Weight bytes are uploaded on every call:
// callers that keep weights resident use the device-pointer API
// (glmvx_packed_gemv / glmvx_packed_gemm) instead.
//
// `half` and `table` must be the reference's exact lookup tables
// (kernels/packed.py:27-37).  The kernels decode fp16 in hardware (exact for
// every fp16 value) and read their own copy of the codebooks, so the tables
// are verified once per distinct pointer pair and a mismatch is rejected.
#include <cmath>
#include <cstring>
#include <vector>

#include "codecs.cuh"

namespace glmvx {

int32_t packed_matmul_device(int32_t kind, float *out, const uint8_t *w, const float *x, int32_t rows,
                             int32_t cols, int32_t batch, cudaStream_t stream, int32_t *path_out);
int32_t unpack_device(int32_t kind, float *out, const uint8_t *w, int64_t blocks, cudaStream_t stream);

static const uint8_t kHostCodebooks[19600] = {
#include "ggml_tables.inc"
};

namespace {

// Per-thread device staging: one stream and a grow-only arena.
struct Stage {
    cudaStream_t stream = nullptr;
    char *arena = nullptr;
    size_t cap = 0;
    const float *ok_half = nullptr;
    const uint8_t *ok_table = nullptr;
};
thread_local Stage g_stage;

int32_t stage_reserve(size_t bytes) {
    Stage &s = g_stage;
    if (!s.stream) GLMVX_CUDA(cudaStreamCreateWithFlags(&s.stream, cudaStreamNonBlocking));
    if (bytes > s.cap) {
        if (s.arena) {
            GLMVX_CUDA(cudaStreamSynchronize(s.stream));
            GLMVX_CUDA(cudaFree(s.arena));
            s.arena = nullptr;
            s.cap = 0;
        }
        size_t cap = 1 << 20;
        while (cap < bytes) cap <<= 1;
        GLMVX_CUDA(cudaMalloc(&s.arena, cap));
        s.cap = cap;
    }
    return kOk;
}

// Carves 256-byte aligned slices out of the arena; sizes are summed first.
struct Carver {
    size_t off = 0;
    size_t take(size_t bytes) {
        const size_t at = off;
        off += (bytes + 255) & ~static_cast<size_t>(255);
        return at;
    }
};

template <class T>
T *at(size_t off) {
    return reinterpret_cast<T *>(g_stage.arena + off);
}

int32_t h2d(void *dst, const void *src, size_t bytes) {
    if (bytes) GLMVX_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, g_stage.stream));
    return kOk;
}

int32_t finish(void *host_out, const void *dev_out, size_t bytes) {
    if (bytes)
        GLMVX_CUDA(cudaMemcpyAsync(host_out, dev_out, bytes, cudaMemcpyDeviceToHost, g_stage.stream));
    GLMVX_CUDA(cudaStreamSynchronize(g_stage.stream));
    int *word = device_error_word();
    int code = 0;
    if (word) {
        GLMVX_CUDA(cudaMemcpy(&code, word, sizeof code, cudaMemcpyDeviceToHost));
        if (code) {
            const int zero = 0;
            cudaMemcpy(word, &zero, sizeof zero, cudaMemcpyHostToDevice);
            set_error("kernel reported device error %d (bounded wait expired)", code);
            return kDeviceError;
        }
    }
    return kOk;
}

bool tables_match(const float *half, const uint8_t *table) {
    Stage &s = g_stage;
    if (half == s.ok_half && table == s.ok_table) return true;
    if (!half || !table || std::memcmp(table, kHostCodebooks, sizeof kHostCodebooks) != 0) return false;
    for (uint32_t bits = 0; bits < 65536; ++bits) {
        const float want = __half2float(__ushort_as_half(static_cast<unsigned short>(bits)));
        if (std::isnan(want) ? !std::isnan(half[bits]) : std::memcmp(&want, &half[bits], 4) != 0) return false;
    }
    s.ok_half = half;
    s.ok_table = table;
    return true;
}

// batch_v2 activations arrive as consecutive transposed [cols, tile] tiles of
// 64/32/16/8/4/2/1 tokens (kernels/packed.py:139-146); rebuild [batch, cols].
void untile(const float *xt, float *x, int cols, int batch) {
    int token = 0;
    for (int tile = 64; tile >= 1; tile >>= 1) {
        while (batch - token >= tile) {
            const float *src = xt + static_cast<size_t>(token) * cols;
            for (int c = 0; c < cols; ++c)
                for (int i = 0; i < tile; ++i) x[static_cast<size_t>(token + i) * cols + c] = src[static_cast<size_t>(c) * tile + i];
            token += tile;
        }
    }
}

int32_t host_packed(int kind, float *out, const uint8_t *w, const float *x, const float *half,
                    const uint8_t *table, int32_t rows, int32_t cols, int32_t batch, bool tiled) {
    int blk = 0, bytes = 0;
    if (!reference_layout(kind, blk, bytes)) return kInvalid;
    if (rows < 0 || cols <= 0 || cols % blk != 0 || batch < 0 || batch > 64) return kInvalid;
    if (!tables_match(half, table)) {
        set_error("half/table are not the reference lookup tables");
        return kInvalid;
    }
    if (rows == 0 || batch == 0) return kOk;
    const size_t wbytes = static_cast<size_t>(rows) * (cols / blk) * bytes;
    const size_t xbytes = static_cast<size_t>(batch) * cols * sizeof(float);
    const size_t obytes = static_cast<size_t>(batch) * rows * sizeof(float);
    Carver c;
    const size_t ow = c.take(wbytes), ox = c.take(xbytes), oo = c.take(obytes);
    if (int32_t st = stage_reserve(c.off)) return st;
    std::vector<float> rowmajor;
    if (tiled && batch > 1) {
        rowmajor.resize(static_cast<size_t>(batch) * cols);
        untile(x, rowmajor.data(), cols, batch);
        x = rowmajor.data();
    }
    if (int32_t st = h2d(at<uint8_t>(ow), w, wbytes)) return st;
    if (int32_t st = h2d(at<float>(ox), x, xbytes)) return st;
    if (int32_t st = packed_matmul_device(kind, at<float>(oo), at<uint8_t>(ow), at<float>(ox), rows, cols, batch,
                                          g_stage.stream, nullptr))
        return st;
    return finish(out, at<float>(oo), obytes);
}

int32_t host_unpack(int kind, float *out, const uint8_t *w, const float *half, const uint8_t *table,
                    int32_t blocks) {
    int blk = 0, bytes = 0;
    if (!reference_layout(kind, blk, bytes) || blocks < 0) return kInvalid;
    if (!tables_match(half, table)) {
        set_error("half/table are not the reference lookup tables");
        return kInvalid;
    }
    if (blocks == 0) return kOk;
    const size_t wbytes = static_cast<size_t>(blocks) * bytes;
    const size_t obytes = static_cast<size_t>(blocks) * blk * sizeof(float);
    Carver c;
    const size_t ow = c.take(wbytes), oo = c.take(obytes);
    if (int32_t st = stage_reserve(c.off)) return st;
    if (int32_t st = h2d(at<uint8_t>(ow), w, wbytes)) return st;
    if (int32_t st = unpack_device(kind, at<float>(oo), at<uint8_t>(ow), blocks, g_stage.stream)) return st;
    return finish(out, at<float>(oo), obytes);
}

}  // namespace
}  // namespace glmvx

using namespace glmvx;

// ------------------------------------------------ packed (kernels/kernels.h:193-207)
#define GLMVX_PACKED_HOST(name, kind)                                                                    \
    GLMVX_EXPORT int32_t glm_vx_packed_##name(float *out, const uint8_t *w, const float *x, const float *half, \
                                              const uint8_t *table, int32_t rows, int32_t cols) {             \
        return host_packed(kind, out, w, x, half, table, rows, cols, 1, false);                             \
    }                                                                                                     \
    GLMVX_EXPORT int32_t glm_vx_packed_batch_v2_##name(float *out, const uint8_t *w, const float *x,         \
                                                       const float *half, const uint8_t *table, int32_t rows, \
                                                       int32_t cols, int32_t batch) {                       \
        return host_packed(kind, out, w, x, half, table, rows, cols, batch, true);                          \
    }                                                                                                     \
    GLMVX_EXPORT int32_t glm_vx_unpack_##name(float *out, const uint8_t *w, const float *half,               \
                                              const uint8_t *table, int32_t blocks) {                       \
        return host_unpack(kind, out, w, half, table, blocks);                                              \
    }

GLMVX_PACKED_HOST(f16, 1)
GLMVX_PACKED_HOST(q8_0, 8)
GLMVX_PACKED_HOST(q2_k, 10)
GLMVX_PACKED_HOST(q3_k, 11)
GLMVX_PACKED_HOST(q4_k, 12)
GLMVX_PACKED_HOST(q5_k, 13)
GLMVX_PACKED_HOST(q6_k, 14)
GLMVX_PACKED_HOST(iq2_xxs, 16)
GLMVX_PACKED_HOST(iq3_xxs, 18)
GLMVX_PACKED_HOST(iq1_s, 19)
GLMVX_PACKED_HOST(iq4_xs, 23)

// ------------------------------------------------ f32 primitives (kernels/kernels.h:168-184)
#define STAGE_OR_RETURN(total)                          \
    do {                                                \
        if (int32_t st_ = stage_reserve(total)) return st_; \
    } while (0)
#define CHECK(x)                        \
    do {                                \
        if (int32_t st_ = (x)) return st_; \
    } while (0)

GLMVX_EXPORT int32_t glm_vx_rmsnorm(float *out, const float *x, const float *weight, int32_t n, float eps) {
    if (n <= 0 || eps <= 0.0f) return kInvalid;
    Carver c;
    const size_t ox = c.take(4ull * n), ow = c.take(4ull * n), oo = c.take(4ull * n);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(ox), x, 4ull * n));
    CHECK(h2d(at<float>(ow), weight, 4ull * n));
    CHECK(glmvx_rmsnorm(at<float>(oo), at<float>(ox), at<float>(ow), 1, n, eps, g_stage.stream));
    return finish(out, at<float>(oo), 4ull * n);
}

GLMVX_EXPORT int32_t glm_vx_layernorm(float *out, const float *x, const float *weight, const float *bias, int32_t n,
                                      float eps) {
    if (n <= 0 || eps <= 0.0f) return kInvalid;
    Carver c;
    const size_t ox = c.take(4ull * n), ow = c.take(4ull * n), ob = c.take(4ull * n), oo = c.take(4ull * n);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(ox), x, 4ull * n));
    CHECK(h2d(at<float>(ow), weight, 4ull * n));
    CHECK(h2d(at<float>(ob), bias, 4ull * n));
    CHECK(glmvx_layernorm(at<float>(oo), at<float>(ox), at<float>(ow), at<float>(ob), 1, n, eps, g_stage.stream));
    return finish(out, at<float>(oo), 4ull * n);
}

GLMVX_EXPORT int32_t glm_vx_softmax(float *out, const float *x, int32_t n) {
    if (n <= 0) return kInvalid;
    Carver c;
    const size_t ox = c.take(4ull * n), oo = c.take(4ull * n);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(ox), x, 4ull * n));
    CHECK(glmvx_softmax(at<float>(oo), at<float>(ox), 1, n, g_stage.stream));
    return finish(out, at<float>(oo), 4ull * n);
}

GLMVX_EXPORT int32_t glm_vx_swiglu(float *out, const float *gate, const float *up, int32_t n) {
    if (n < 0) return kInvalid;
    if (n == 0) return kOk;
    Carver c;
    const size_t og = c.take(4ull * n), ou = c.take(4ull * n), oo = c.take(4ull * n);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(og), gate, 4ull * n));
    CHECK(h2d(at<float>(ou), up, 4ull * n));
    CHECK(glmvx_swiglu(at<float>(oo), at<float>(og), at<float>(ou), n, g_stage.stream));
    return finish(out, at<float>(oo), 4ull * n);
}

GLMVX_EXPORT int32_t glm_vx_add(float *out, const float *a, const float *b, int32_t n) {
    if (n < 0) return kInvalid;
    if (n == 0) return kOk;
    Carver c;
    const size_t oa = c.take(4ull * n), ob = c.take(4ull * n), oo = c.take(4ull * n);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(oa), a, 4ull * n));
    CHECK(h2d(at<float>(ob), b, 4ull * n));
    CHECK(glmvx_add(at<float>(oo), at<float>(oa), at<float>(ob), n, g_stage.stream));
    return finish(out, at<float>(oo), 4ull * n);
}

GLMVX_EXPORT int32_t glm_vx_axpy(float *out, const float *x, float alpha, int32_t n) {
    if (n < 0) return kInvalid;
    if (n == 0) return kOk;
    Carver c;
    const size_t oo = c.take(4ull * n), ox = c.take(4ull * n);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(oo), out, 4ull * n));
    CHECK(h2d(at<float>(ox), x, 4ull * n));
    CHECK(glmvx_axpy(at<float>(oo), at<float>(ox), alpha, n, g_stage.stream));
    return finish(out, at<float>(oo), 4ull * n);
}

GLMVX_EXPORT int32_t glm_vx_matvec(float *out, const float *weight, const float *x, int32_t rows, int32_t cols) {
    if (rows < 0 || cols < 0) return kInvalid;
    if (rows == 0) return kOk;
    const size_t wb = 4ull * rows * cols, xb = 4ull * cols, ob = 4ull * rows;
    Carver c;
    const size_t ow = c.take(wb), ox = c.take(xb), oo = c.take(ob);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(ow), weight, wb));
    CHECK(h2d(at<float>(ox), x, xb));
    CHECK(glmvx_matvec_f32(at<float>(oo), at<float>(ow), at<float>(ox), rows, cols, g_stage.stream));
    return finish(out, at<float>(oo), ob);
}

GLMVX_EXPORT int32_t glm_vx_matmul_nt(float *out, const float *a, const float *b, int32_t m, int32_t n, int32_t k) {
    if (m < 0 || n < 0 || k < 0) return kInvalid;
    if (m == 0 || n == 0) return kOk;
    const size_t ab = 4ull * m * k, bb = 4ull * n * k, ob = 4ull * m * n;
    Carver c;
    const size_t oa = c.take(ab), obb = c.take(bb), oo = c.take(ob);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(oa), a, ab));
    CHECK(h2d(at<float>(obb), b, bb));
    CHECK(glmvx_matmul_nt(at<float>(oo), at<float>(oa), at<float>(obb), m, n, k, g_stage.stream));
    return finish(out, at<float>(oo), ob);
}

GLMVX_EXPORT int32_t glm_vx_rope_offset(float *out, const float *x, const float *cosine, const float *sine,
                                        int32_t heads, int32_t head_dim, int32_t rope_dim, int32_t offset) {
    if (heads < 0 || rope_dim < 0 || offset < 0 || head_dim < rope_dim || offset > head_dim - rope_dim ||
        rope_dim % 2 != 0)
        return kInvalid;
    const size_t n = static_cast<size_t>(heads) * head_dim, half = rope_dim / 2;
    if (n == 0) return kOk;
    Carver c;
    const size_t ox = c.take(4 * n), oc = c.take(4 * half + 4), os = c.take(4 * half + 4), oo = c.take(4 * n);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(ox), x, 4 * n));
    CHECK(h2d(at<float>(oc), cosine, 4 * half));
    CHECK(h2d(at<float>(os), sine, 4 * half));
    CHECK(glmvx_rope_offset(at<float>(oo), at<float>(ox), at<float>(oc), at<float>(os), heads, head_dim, rope_dim,
                            offset, g_stage.stream));
    return finish(out, at<float>(oo), 4 * n);
}

GLMVX_EXPORT int32_t glm_vx_rope(float *out, const float *x, const float *cosine, const float *sine, int32_t heads,
                                 int32_t head_dim, int32_t rope_dim) {
    return glm_vx_rope_offset(out, x, cosine, sine, heads, head_dim, rope_dim, head_dim - rope_dim);
}

GLMVX_EXPORT int32_t glm_vx_rope_glm(float *out, const float *x, const float *cosine, const float *sine,
                                     int32_t heads, int32_t dim) {
    if (heads < 0 || dim <= 0 || dim % 2 != 0) return kInvalid;
    const size_t n = static_cast<size_t>(heads) * dim, half = dim / 2;
    if (n == 0) return kOk;
    Carver c;
    const size_t ox = c.take(4 * n), oc = c.take(4 * half), os = c.take(4 * half), oo = c.take(4 * n);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(ox), x, 4 * n));
    CHECK(h2d(at<float>(oc), cosine, 4 * half));
    CHECK(h2d(at<float>(os), sine, 4 * half));
    CHECK(glmvx_rope_glm(at<float>(oo), at<float>(ox), at<float>(oc), at<float>(os), heads, dim, g_stage.stream));
    return finish(out, at<float>(oo), 4 * n);
}

GLMVX_EXPORT int32_t glm_vx_router(int32_t *indices, float *weights, const float *logits, const float *bias,
                                   int32_t experts, int32_t k, float scale) {
    if (k <= 0 || experts < k) return kInvalid;
    Carver c;
    const size_t ol = c.take(4ull * experts), ob = c.take(4ull * experts), oi = c.take(4ull * k),
                 ow = c.take(4ull * k);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(ol), logits, 4ull * experts));
    CHECK(h2d(at<float>(ob), bias, 4ull * experts));
    CHECK(glmvx_router(at<int32_t>(oi), at<float>(ow), at<float>(ol), at<float>(ob), 1, experts, k, scale,
                       g_stage.stream));
    GLMVX_CUDA(cudaMemcpyAsync(indices, at<int32_t>(oi), 4ull * k, cudaMemcpyDeviceToHost, g_stage.stream));
    return finish(weights, at<float>(ow), 4ull * k);
}

GLMVX_EXPORT int32_t glm_vx_topk(int32_t *indices, const float *scores, int32_t n, int32_t k) {
    if (n < 0 || k < 0 || n < k) return kInvalid;
    if (k == 0) return kOk;
    const size_t scratch = static_cast<size_t>(glmvx_topk_scratch_bytes(n));
    Carver c;
    const size_t os = c.take(4ull * n), oi = c.take(4ull * k), ok = c.take(scratch);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(os), scores, 4ull * n));
    CHECK(glmvx_topk(at<int32_t>(oi), at<float>(os), n, k, scratch ? at<void>(ok) : nullptr, g_stage.stream));
    return finish(indices, at<int32_t>(oi), 4ull * k);
}

GLMVX_EXPORT int32_t glm_vx_index_scores(float *out, const float *q, const float *keys, const float *weights,
                                         int32_t tokens, int32_t heads, int32_t dim, float qk_scale) {
    if (tokens < 0 || heads <= 0 || dim <= 0) return kInvalid;
    if (tokens == 0) return kOk;
    const size_t qb = 4ull * heads * dim, kb = 4ull * tokens * dim;
    Carver c;
    const size_t oq = c.take(qb), ok = c.take(kb), ow = c.take(4ull * heads), oo = c.take(4ull * tokens);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(oq), q, qb));
    CHECK(h2d(at<float>(ok), keys, kb));
    CHECK(h2d(at<float>(ow), weights, 4ull * heads));
    CHECK(glmvx_index_scores(at<float>(oo), at<float>(oq), at<float>(ok), at<float>(ow), tokens, heads, dim,
                             qk_scale, g_stage.stream));
    return finish(out, at<float>(oo), 4ull * tokens);
}

static int32_t host_attention(float *out, float *scratch, const float *q, const float *keys, const float *values,
                              const int32_t *selected, int32_t count, int32_t tokens, int32_t dim,
                              int32_t value_dim, float scale) {
    const size_t qb = 4ull * dim, kb = 4ull * tokens * dim, vb = 4ull * tokens * value_dim;
    Carver c;
    const size_t oq = c.take(qb), ok = c.take(kb), ov = c.take(vb), osel = c.take(selected ? 4ull * count : 0),
                 osc = c.take(4ull * count), oo = c.take(4ull * value_dim), obad = c.take(4);
    STAGE_OR_RETURN(c.off);
    CHECK(h2d(at<float>(oq), q, qb));
    CHECK(h2d(at<float>(ok), keys, kb));
    CHECK(h2d(at<float>(ov), values, vb));
    if (selected) CHECK(h2d(at<int32_t>(osel), selected, 4ull * count));
    GLMVX_CUDA(cudaMemsetAsync(at<int32_t>(obad), 0, 4, g_stage.stream));
    CHECK(glmvx_attention(at<float>(oo), at<float>(osc), at<float>(oq), at<float>(ok), at<float>(ov),
                          selected ? at<int32_t>(osel) : nullptr, count, tokens, dim, value_dim, scale,
                          at<int32_t>(obad), g_stage.stream));
    GLMVX_CUDA(cudaMemcpyAsync(scratch, at<float>(osc), 4ull * count, cudaMemcpyDeviceToHost, g_stage.stream));
    return finish(out, at<float>(oo), 4ull * value_dim);
}

GLMVX_EXPORT int32_t glm_vx_attention(float *out, float *scratch, const float *q, const float *keys,
                                      const float *values, int32_t tokens, int32_t dim, int32_t value_dim,
                                      float scale) {
    if (tokens <= 0 || dim <= 0 || value_dim <= 0) return kInvalid;
    return host_attention(out, scratch, q, keys, values, nullptr, tokens, tokens, dim, value_dim, scale);
}

GLMVX_EXPORT int32_t glm_vx_sparse_attention(float *out, float *scratch, const float *q, const float *keys,
                                             const float *values, const int32_t *selected, int32_t count,
                                             int32_t tokens, int32_t dim, int32_t value_dim, float scale) {
    if (count <= 0 || tokens <= 0 || dim <= 0 || value_dim <= 0) return kInvalid;
    for (int32_t j = 0; j < count; ++j)  // kernels/kernels.vx:385: reject before any write
        if (selected[j] < 0 || selected[j] >= tokens) return kInvalid;
    return host_attention(out, scratch, q, keys, values, selected, count, tokens, dim, value_dim, scale);
}
