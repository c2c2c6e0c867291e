// Expert-parallel routed + shared MoE layer over peer memory (NVLink /
// NVSwitch), one process (rank) per GPU, no collective library and no host
// round trip inside a step.
//
// The reference runs every expert of a layer in one process
// (glm_vx/model.py:289-324).  Here routed expert e lives on rank
// e / (experts / world); the router and the shared expert are replicated.
// Every rank owns a MAILBOX (cudaMalloc'd, mapped by its peers through CUDA
// IPC handles or, for ranks emulated in one process, shared directly):
//
//   fwd_flag[8], ret_flag[8]   u32 epochs, slot s written by rank s
//   fwd_count[8]               pairs rank s sent here this step
//   fwd_meta[world][cap]       local expert id of each received pair
//   fwd_rows[world][cap]       the pair's token row, already prepared
//                              (int8 limbs + exponents + sub-block sums,
//                              prep_stride(hidden) bytes)
//   ret_rows[world][cap]       f32 [hidden] expert outputs of THIS rank's
//                              pairs, written by the owner d at [d][pos]
//
// cap = max_tokens * top_k.  One step, all on the rank's stream:
//   1. prepare the T token rows; router logits; sigmoid top-k routing;
//   2. dispatch (ep_dispatch_kernel): each (token, slot) pair goes to the
//      owner of its expert, in (token, slot) order per destination: the
//      prepared row is stored straight into the owner's fwd_rows over NVLink,
//      with the local expert id and the per-destination count; the last CTA
//      bumps the step epoch and publishes it in every owner's fwd_flag slot
//      for this rank (system-scope release after a system fence);
//   3. experts (ep_group_kernel + the tensor-core job GEMVs): the owner
//      waits (acquire, bounded to 2 s) for every sender's flag, groups the
//      received pairs by local expert into the same two-/four-token job lists
//      as the single-GPU layer (moe_jobs.cuh), adds the shared expert's jobs
//      for its own tokens, runs gate+up, SwiGLU-prepares, and runs down with
//      each routed pair's output row ADDRESSED IN THE SENDER'S ret_rows, so
//      the down GEMV's stores cross NVLink directly (no copy kernel); a
//      signal kernel then releases ret_flag[rank] in every sender's mailbox;
//   4. combine (ep_combine_kernel): wait for every owner's ret_flag, then
//      y[t] = sum over the token's slots in ascending expert id of
//      ret_row * weight, plus the shared expert's row -- the reference's
//      order (glm_vx/model.py:305-316).
// A token's arithmetic is the single-GPU layer's in every job list, so the
// output does not depend on the number of ranks (bit for bit).
//
// Reuse of the mailbox across steps is safe without extra flags: a rank
// starts step i+1 only after its combine of step i saw every owner's return,
// which each owner sends after its down GEMV, i.e. after its last read of
// that rank's fwd_rows.  Waits are bounded (2 s): on expiry the kernel sets
// the device error word and the step produces no outputs (host reports).
// Plain peer loads and stores only: no multicast object, no TMA multicast.
#include <algorithm>
#include <cstring>
#include <new>

#include "codecs.cuh"
#include "mma_gemv.cuh"
#include "moe_jobs.cuh"

namespace glmvx {

namespace {

constexpr int kEpMaxWorld = 8, kEpDispatchThreads = 256;
constexpr uint64_t kEpWaitNs = 2000000000ull;

struct EpMailbox {  // byte offsets inside every rank's mailbox
    size_t fwd_flag, ret_flag, fwd_count, fwd_meta, fwd_rows, ret_rows, total;
};

EpMailbox mailbox_layout(int world, int cap, size_t xstride, int hidden) {
    EpMailbox m{};
    size_t off = 0;
    auto take = [&](size_t n) {
        const size_t o = off;
        off += (n + 255) & ~static_cast<size_t>(255);
        return o;
    };
    m.fwd_flag = take(4 * kEpMaxWorld);
    m.ret_flag = take(4 * kEpMaxWorld);
    m.fwd_count = take(4 * kEpMaxWorld);
    m.fwd_meta = take(4ull * world * cap);
    m.fwd_rows = take(xstride * world * cap);
    m.ret_rows = take(4ull * hidden * world * cap);
    m.total = off;
    return m;
}

struct EpCtrl {  // this rank's device-side step state
    unsigned epoch;
    unsigned arrive;
};

struct EpPeers {
    char *base[kEpMaxWorld];  // mailbox of every rank (own included)
};

struct EpState {
    int device, rank, world, max_tokens, hidden, inter, experts, per_rank, top_k, kind, cap, pmax;
    float scale;
    bool shared;
    size_t xstride, hstride, gu_stride, dn_stride;
    const float *router_w, *router_bias;
    const uint8_t *gate, *up, *down, *sgate, *sup, *sdown;
    EpMailbox mb;
    char *mail = nullptr;
    EpPeers peers{};
    bool connected = false;
    char *scratch = nullptr;
    float *logits, *wts, *combw, *g_out, *u_out, *shared_out;
    int32_t *ids, *comb;
    uint8_t *xprep, *hprep;
    MmaJob *gu_m, *dn_m, *gu_q, *dn_q;
    int *counts;  // [0..3] job counts of the four lists, [4] prepared down-input rows
    EpCtrl *ctrl;
};

__device__ __forceinline__ unsigned ld_acquire_sys(const unsigned *p) {
    unsigned v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}

__device__ __forceinline__ void st_release_sys(unsigned *p, unsigned v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}

// Wait until *flag reached epoch (wrap-safe), at most kEpWaitNs.
__device__ bool wait_epoch(const unsigned *flag, unsigned epoch) {
    if (static_cast<int>(ld_acquire_sys(flag) - epoch) >= 0) return true;
    const uint64_t start = globaltimer_ns();
    for (;;) {
        __nanosleep(100);
        if (static_cast<int>(ld_acquire_sys(flag) - epoch) >= 0) return true;
        if (globaltimer_ns() - start > kEpWaitNs) return false;
    }
}

// Step 2.  Warp 0 plans: for pair a = t*k + j (in order) its destination
// rank and its position among the pairs to that rank (ballots per
// destination, so the order is (token, slot)).  The CTAs then copy one
// prepared row per pair into the owners' mailboxes.  CTA 0 also publishes
// the per-destination counts and builds this rank's combine table: per token
// its slots in ascending expert id, as (owner * cap + position) rows of its
// own ret_rows.  The last CTA to finish bumps the epoch and signals.
__global__ void __launch_bounds__(kEpDispatchThreads)
    ep_dispatch_kernel(EpPeers peers, EpMailbox mb, int rank, int world, int cap, int T, int k, int per_rank,
                       int experts, const int32_t *__restrict__ ids, const float *__restrict__ wts,
                       const uint8_t *__restrict__ xprep, size_t xstride, int32_t *comb, float *combw, EpCtrl *ctrl,
                       int *err) {
    __shared__ int16_t s_pos[kMaxAssignments];
    __shared__ int8_t s_dst[kMaxAssignments];
    __shared__ int16_t s_loc[kMaxAssignments];
    __shared__ int s_cnt[kEpMaxWorld];
    const int n = T * k;
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    if (warp == 0) {
        int run = 0;  // lane d < world: pairs planned to destination d so far
        for (int base = 0; base < n; base += 32) {
            const int a = base + lane;
            int e = a < n ? ids[a] : 0;
            if (a < n && (e < 0 || e >= experts)) report_device_error(err, kDevErrBadIndex);
            e = min(max(e, 0), experts - 1);
            const int d = a < n ? e / per_rank : -1;
            int pos = 0;
            for (int dd = 0; dd < world; ++dd) {
                const unsigned m = __ballot_sync(0xffffffffu, d == dd);
                const int before = __shfl_sync(0xffffffffu, run, dd);
                if (d == dd) pos = before + __popc(m & ((1u << lane) - 1u));
                if (lane == dd) run += __popc(m);
            }
            if (a < n) {
                s_dst[a] = static_cast<int8_t>(d);
                s_pos[a] = static_cast<int16_t>(pos);
                s_loc[a] = static_cast<int16_t>(e - d * per_rank);
            }
        }
        if (lane < world) s_cnt[lane] = run;
    }
    __syncthreads();
    const size_t vec = xstride / 16;
    for (int a = blockIdx.x; a < n; a += gridDim.x) {
        const int d = s_dst[a], pos = s_pos[a];
        const int4 *src = reinterpret_cast<const int4 *>(xprep + static_cast<size_t>(a / k) * xstride);
        char *box = peers.base[d];
        int4 *dst = reinterpret_cast<int4 *>(box + mb.fwd_rows + (static_cast<size_t>(rank) * cap + pos) * xstride);
        for (size_t i = threadIdx.x; i < vec; i += blockDim.x) dst[i] = src[i];
        if (threadIdx.x == 0)
            reinterpret_cast<int32_t *>(box + mb.fwd_meta)[static_cast<size_t>(rank) * cap + pos] = s_loc[a];
    }
    if (blockIdx.x == 0) {
        if (threadIdx.x < world) reinterpret_cast<int32_t *>(peers.base[threadIdx.x] + mb.fwd_count)[rank] = s_cnt[threadIdx.x];
        for (int t = threadIdx.x; t < T; t += blockDim.x) {
            for (int i = 0; i < k; ++i) {
                const int a = t * k + i;
                const int e = s_dst[a] * per_rank + s_loc[a];
                int order = 0;
                for (int j = 0; j < k; ++j) order += s_dst[t * k + j] * per_rank + s_loc[t * k + j] < e;
                comb[t * k + order] = s_dst[a] * cap + s_pos[a];
                combw[t * k + order] = wts[a];
            }
        }
    }
    __threadfence_system();  // this thread's stores are visible system-wide
    __syncthreads();
    if (threadIdx.x == 0) {
        const unsigned prev = atomicAdd(&ctrl->arrive, 1u);
        if (prev == gridDim.x - 1) {  // every CTA's stores are fenced
            ctrl->arrive = 0;
            const unsigned epoch = ctrl->epoch + 1u;
            ctrl->epoch = epoch;
            __threadfence_system();
            for (int d = 0; d < world; ++d)
                st_release_sys(reinterpret_cast<unsigned *>(peers.base[d] + mb.fwd_flag) + rank, epoch);
        }
    }
}

// Addresses of the received pairs for form_mma_jobs: assignment a is row
// (sender s, position p) of this rank's fwd_rows; its down output goes to row
// (this rank, p) of the SENDER's ret_rows.  Shared-expert pairs are this
// rank's own token rows, their outputs local.
struct EpJobSrc {
    const uint8_t *gate, *up, *down, *sgate, *sup, *sdown, *xprep, *rows;
    size_t gu_stride, dn_stride, xstride;
    const int16_t *row_of;  // a -> s * cap + p
    EpPeers peers;
    size_t ret_rows;
    float *shared_out;
    int rank, cap, hidden;
    __device__ const uint8_t *wg(int e) const { return gate + e * gu_stride; }
    __device__ const uint8_t *wu(int e) const { return up + e * gu_stride; }
    __device__ const uint8_t *wd(int e) const { return down + e * dn_stride; }
    __device__ const uint8_t *sg() const { return sgate; }
    __device__ const uint8_t *su() const { return sup; }
    __device__ const uint8_t *sd() const { return sdown; }
    __device__ const uint8_t *xp(int a) const { return rows + static_cast<size_t>(row_of[a]) * xstride; }
    __device__ float *out(int a, int) const {
        const int s = row_of[a] / cap, p = row_of[a] % cap;
        return reinterpret_cast<float *>(peers.base[s] + ret_rows) + (static_cast<size_t>(rank) * cap + p) * hidden;
    }
    __device__ const uint8_t *xp_shared(int t) const { return xprep + static_cast<size_t>(t) * xstride; }
    __device__ float *out_shared(int t, int) const { return shared_out + static_cast<size_t>(t) * hidden; }
};

struct EpGroupArgs {
    EpPeers peers;
    EpMailbox mb;
    int rank, world, cap, per_rank, T, shared, quad, inter;
    EpJobSrc src;
    float *g_out, *u_out;
    const uint8_t *hprep;
    size_t hstride;
    MmaJob *gu_m, *dn_m, *gu_q, *dn_q;
    int *counts;
    const EpCtrl *ctrl;
    int *err;
};

// Step 3, grouping: wait for every sender, read the counts and local expert
// ids of the received pairs, build the job lists (moe_jobs.cuh).
__global__ void __launch_bounds__(kGroupThreads) ep_group_kernel(EpGroupArgs g_) {
    __shared__ GroupSmem g;
    __shared__ int16_t s_row[kMaxAssignments];
    __shared__ int s_off[kEpMaxWorld + 1];
    __shared__ int s_ok;
    const EpGroupArgs &A = g_;
    char *mail = A.peers.base[A.rank];
    if (threadIdx.x == 0) s_ok = 1;
    __syncthreads();
    const unsigned epoch = *reinterpret_cast<const volatile unsigned *>(&A.ctrl->epoch);
    if (threadIdx.x < A.world &&
        !wait_epoch(reinterpret_cast<const unsigned *>(mail + A.mb.fwd_flag) + threadIdx.x, epoch)) {
        report_device_error(A.err, kDevErrFullWait);
        s_ok = 0;
    }
    __syncthreads();
    if (!s_ok) {
        if (threadIdx.x < 5) A.counts[threadIdx.x] = 0;
        return;
    }
    if (threadIdx.x == 0) {
        int off = 0;
        for (int s = 0; s < A.world; ++s) {
            s_off[s] = off;
            off += min(max(__ldcg(reinterpret_cast<const int *>(mail + A.mb.fwd_count) + s), 0), A.cap);
        }
        s_off[A.world] = off;
    }
    __syncthreads();
    const int n = s_off[A.world];
    const int *meta = reinterpret_cast<const int *>(mail + A.mb.fwd_meta);
    for (int a = threadIdx.x; a < n; a += blockDim.x) {
        int s = 0;
        while (s + 1 < A.world && a >= s_off[s + 1]) ++s;
        const int p = a - s_off[s];
        const int e = __ldcg(meta + s * A.cap + p);
        if (e < 0 || e >= A.per_rank) report_device_error(A.err, kDevErrBadIndex);
        g.ids[a] = static_cast<int16_t>(min(max(e, 0), A.per_rank - 1));
        s_row[a] = static_cast<int16_t>(s * A.cap + p);
    }
    __syncthreads();
    EpJobSrc src = A.src;
    src.row_of = s_row;
    form_mma_jobs(src, g, n, A.shared ? A.T : 0, A.quad != 0, A.g_out, A.u_out, A.hprep, A.hstride, A.inter, A.gu_m,
                  A.dn_m, A.gu_q, A.dn_q, A.counts);
    if (threadIdx.x == 0) A.counts[4] = n + (A.shared ? A.T : 0);
}

// Step 3, after the down GEMV: this rank's outputs are in every sender's
// ret_rows; publish the epoch in each sender's ret_flag slot for this rank.
__global__ void ep_return_kernel(EpPeers peers, EpMailbox mb, int rank, int world, const EpCtrl *ctrl) {
    const int s = threadIdx.x;
    __threadfence_system();
    if (s >= world) return;
    const unsigned epoch = *reinterpret_cast<const volatile unsigned *>(&ctrl->epoch);
    st_release_sys(reinterpret_cast<unsigned *>(peers.base[s] + mb.ret_flag) + rank, epoch);
}

// Step 4: wait for every owner's return, then the ordered weighted sum.
__global__ void ep_combine_kernel(float *y, const char *mail, EpMailbox mb, const int32_t *comb, const float *combw,
                                  const float *shared_rows, int T, int k, int hidden, int world, const EpCtrl *ctrl,
                                  int *err) {
    __shared__ int s_ok;
    if (threadIdx.x == 0) s_ok = 1;
    __syncthreads();
    const unsigned epoch = *reinterpret_cast<const volatile unsigned *>(&ctrl->epoch);
    if (threadIdx.x < world &&
        !wait_epoch(reinterpret_cast<const unsigned *>(mail + mb.ret_flag) + threadIdx.x, epoch)) {
        report_device_error(err, kDevErrFullWait);
        s_ok = 0;
    }
    __syncthreads();
    const int t = blockIdx.y;
    const int h = blockIdx.x * blockDim.x + threadIdx.x;
    if (!s_ok || t >= T || h >= hidden) return;
    const float *ret = reinterpret_cast<const float *>(mail + mb.ret_rows);
    float r = 0.0f;
    for (int i = 0; i < k; ++i) {
        const int p = comb[t * k + i];
        r = __fadd_rn(r, __fmul_rn(__ldcg(ret + static_cast<size_t>(p) * hidden + h), combw[t * k + i]));
    }
    if (shared_rows) r = __fadd_rn(r, shared_rows[static_cast<size_t>(t) * hidden + h]);
    y[static_cast<size_t>(t) * hidden + h] = r;
}

size_t carve_scratch(EpState &s, char *base) {
    size_t off = 0;
    auto take = [&](size_t n) {
        char *p = base ? base + off : nullptr;
        off += (n + 255) & ~static_cast<size_t>(255);
        return p;
    };
    const size_t T = s.max_tokens, k = s.top_k, P = s.pmax;
    s.logits = reinterpret_cast<float *>(take(4 * T * s.experts));
    s.ids = reinterpret_cast<int32_t *>(take(4 * T * k));
    s.wts = reinterpret_cast<float *>(take(4 * T * k));
    s.comb = reinterpret_cast<int32_t *>(take(4 * T * k));
    s.combw = reinterpret_cast<float *>(take(4 * T * k));
    s.xprep = reinterpret_cast<uint8_t *>(take(T * s.xstride));
    s.g_out = reinterpret_cast<float *>(take(4 * P * s.inter));
    s.u_out = reinterpret_cast<float *>(take(4 * P * s.inter));
    s.shared_out = reinterpret_cast<float *>(take(4 * T * s.hidden));
    s.hprep = reinterpret_cast<uint8_t *>(take(P * s.hstride));
    s.gu_m = reinterpret_cast<MmaJob *>(take(sizeof(MmaJob) * 2 * P));
    s.dn_m = reinterpret_cast<MmaJob *>(take(sizeof(MmaJob) * P));
    s.gu_q = reinterpret_cast<MmaJob *>(take(sizeof(MmaJob) * 2 * P));
    s.dn_q = reinterpret_cast<MmaJob *>(take(sizeof(MmaJob) * P));
    s.counts = reinterpret_cast<int *>(take(8 * sizeof(int)));
    s.ctrl = reinterpret_cast<EpCtrl *>(take(sizeof(EpCtrl)));
    return off;
}

int32_t check_state(const EpState *s, const char *what) {
    if (!s) return set_error("%s: null layer", what), kInvalid;
    if (!s->connected) return set_error("%s: layer not connected to its peers (glmvx_ep_connect)", what), kInvalid;
    int dev = -1;
    GLMVX_CUDA(cudaGetDevice(&dev));
    if (dev != s->device) return set_error("%s: layer belongs to device %d, current is %d", what, s->device, dev), kInvalid;
    return kOk;
}

}  // namespace

}  // namespace glmvx

using namespace glmvx;

GLMVX_EXPORT int32_t glmvx_ep_create(void **layer, int32_t rank, int32_t world, int32_t max_tokens, int32_t hidden,
                                     int32_t inter, int32_t experts, int32_t top_k, float scale, int32_t kind,
                                     const float *router_w, const float *router_bias, const uint8_t *gate,
                                     const uint8_t *up, const uint8_t *down, const uint8_t *shared_gate,
                                     const uint8_t *shared_up, const uint8_t *shared_down) {
    if (!layer) return set_error("ep_create: null handle"), kInvalid;
    *layer = nullptr;
    if (world < 1 || world > kEpMaxWorld || rank < 0 || rank >= world)
        return set_error("ep_create: world must be 1..%d and 0 <= rank < world", kEpMaxWorld), kInvalid;
    if (max_tokens < 1 || hidden <= 0 || inter <= 0 || experts <= 0 || top_k <= 0 || top_k > experts ||
        experts % world || experts / world > 32767)
        return set_error("ep_create: invalid dimensions (experts must split evenly over the ranks)"), kInvalid;
    if (static_cast<int64_t>(world) * max_tokens * top_k > kMaxAssignments)
        return set_error("ep_create: world * max_tokens * top_k must be at most %d", kMaxAssignments), kInvalid;
    if (!(scale == scale)) return set_error("ep_create: scale must be a number"), kInvalid;
    const bool shared = shared_gate && shared_up && shared_down;
    if (!shared && (shared_gate || shared_up || shared_down))
        return set_error("ep_create: shared expert needs gate, up and down"), kInvalid;
    auto a16 = [](const void *p) { return (reinterpret_cast<uintptr_t>(p) & 15) == 0; };
    if (!router_w || !router_bias || !gate || !up || !down || !a16(gate) || !a16(up) || !a16(down) ||
        (shared && (!a16(shared_gate) || !a16(shared_up) || !a16(shared_down))))
        return set_error("ep_create: weights must be set and 16-byte aligned"), kInvalid;
    if (!mma_supported(kind, hidden) || !mma_supported(kind, inter))
        return set_error("ep_create: format %d at hidden %d / intermediate %d has no tensor-core kernel", kind, hidden,
                         inter), kUnsupported;
    int blk = 0, bytes = 0;
    reference_layout(kind, blk, bytes);
    auto *s = new (std::nothrow) EpState();
    if (!s) return set_error("ep_create: out of host memory"), kInvalid;
    GLMVX_CUDA(cudaGetDevice(&s->device));
    s->rank = rank;
    s->world = world;
    s->max_tokens = max_tokens;
    s->hidden = hidden;
    s->inter = inter;
    s->experts = experts;
    s->per_rank = experts / world;
    s->top_k = top_k;
    s->kind = kind;
    s->scale = scale;
    s->shared = shared;
    s->cap = max_tokens * top_k;
    s->pmax = world * s->cap + (shared ? max_tokens : 0);
    s->xstride = prep_stride(hidden);
    s->hstride = prep_stride(inter);
    s->gu_stride = static_cast<size_t>(inter) * (hidden / blk) * bytes;
    s->dn_stride = static_cast<size_t>(hidden) * (inter / blk) * bytes;
    s->router_w = router_w;
    s->router_bias = router_bias;
    s->gate = gate;
    s->up = up;
    s->down = down;
    s->sgate = shared_gate;
    s->sup = shared_up;
    s->sdown = shared_down;
    s->mb = mailbox_layout(world, s->cap, s->xstride, hidden);
    const size_t scratch = carve_scratch(*s, nullptr);
    cudaError_t e = cudaMalloc(&s->mail, s->mb.total);
    if (e == cudaSuccess) e = cudaMalloc(&s->scratch, scratch);
    if (e == cudaSuccess) e = cudaMemset(s->mail, 0, s->mb.fwd_meta);  // flags and counts start at 0
    if (e == cudaSuccess) {
        carve_scratch(*s, s->scratch);
        e = cudaMemset(s->ctrl, 0, sizeof(EpCtrl));
    }
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e != cudaSuccess) {
        cudaFree(s->mail);
        cudaFree(s->scratch);
        delete s;
        return cuda_fail(e, "ep_create");
    }
    *layer = s;
    return kOk;
}

// This rank's mailbox (device pointer, cudaMalloc'd: share it with the other
// ranks through glmvx_ipc_handle / glmvx_ipc_open) and its size.
GLMVX_EXPORT int32_t glmvx_ep_mailbox(void *layer, void **base, uint64_t *bytes) {
    auto *s = static_cast<EpState *>(layer);
    if (!s || !base) return set_error("ep_mailbox: null argument"), kInvalid;
    *base = s->mail;
    if (bytes) *bytes = s->mb.total;
    return kOk;
}

// The mailbox of every rank, in rank order (this rank's own included), as
// this process addresses it: an IPC mapping of a peer's allocation, or the
// other layer's own pointer when the ranks share one process and device.
GLMVX_EXPORT int32_t glmvx_ep_connect(void *layer, void *const *mailboxes) {
    auto *s = static_cast<EpState *>(layer);
    if (!s || !mailboxes) return set_error("ep_connect: null argument"), kInvalid;
    for (int d = 0; d < s->world; ++d) {
        if (!mailboxes[d] || (reinterpret_cast<uintptr_t>(mailboxes[d]) & 255))
            return set_error("ep_connect: mailbox %d null or not 256-byte aligned", d), kInvalid;
        s->peers.base[d] = static_cast<char *>(mailboxes[d]);
    }
    if (s->peers.base[s->rank] != s->mail) return set_error("ep_connect: entry `rank` must be this layer's mailbox"), kInvalid;
    s->connected = true;
    return kOk;
}

// Step phase 1: prepare, route and dispatch `tokens` rows x [tokens, hidden]
// (device, f32, 16-byte aligned).  ids_out / weights_out (nullable, device
// [tokens, top_k]) receive the routing.
GLMVX_EXPORT int32_t glmvx_ep_dispatch(void *layer, const float *x, int32_t tokens, int32_t *ids_out,
                                       float *weights_out, void *stream) {
    auto *s = static_cast<EpState *>(layer);
    if (const int32_t rc = check_state(s, "ep_dispatch")) return rc;
    if (tokens < 0 || tokens > s->max_tokens) return set_error("ep_dispatch: tokens must be 0..%d", s->max_tokens), kInvalid;
    if (tokens && (!x || (reinterpret_cast<uintptr_t>(x) & 15))) return set_error("ep_dispatch: x null or unaligned"), kInvalid;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    int32_t rc = kOk;
    if (tokens) {
        if ((rc = prep_rows_device(s->xprep, x, nullptr, tokens, s->hidden, st))) return rc;
        if ((rc = glmvx_matmul_nt(s->logits, x, s->router_w, tokens, s->experts, s->hidden, st))) return rc;
        if ((rc = glmvx_router(s->ids, s->wts, s->logits, s->router_bias, tokens, s->experts, s->top_k, s->scale, st)))
            return rc;
    }
    const int n = tokens * s->top_k;
    const int grid = std::max(1, std::min(n, 2 * sm_count()));
    ep_dispatch_kernel<<<grid, kEpDispatchThreads, 0, st>>>(s->peers, s->mb, s->rank, s->world, s->cap, tokens,
                                                            s->top_k, s->per_rank, s->experts, s->ids, s->wts, s->xprep,
                                                            s->xstride, s->comb, s->combw, s->ctrl, device_error_word());
    if ((rc = launch_status("ep_dispatch_kernel"))) return rc;
    if (tokens && ids_out) GLMVX_CUDA(cudaMemcpyAsync(ids_out, s->ids, 4ull * n, cudaMemcpyDeviceToDevice, st));
    if (tokens && weights_out) GLMVX_CUDA(cudaMemcpyAsync(weights_out, s->wts, 4ull * n, cudaMemcpyDeviceToDevice, st));
    return kOk;
}

// Step phase 2: this rank's experts on the pairs every rank dispatched to it
// (waits for them on the device), outputs stored into the senders'
// mailboxes, then the return signal.  `tokens` = this rank's own token count
// of the step (its shared-expert rows).
GLMVX_EXPORT int32_t glmvx_ep_experts(void *layer, int32_t tokens, void *stream) {
    auto *s = static_cast<EpState *>(layer);
    if (const int32_t rc = check_state(s, "ep_experts")) return rc;
    if (tokens < 0 || tokens > s->max_tokens) return set_error("ep_experts: tokens must be 0..%d", s->max_tokens), kInvalid;
    cudaStream_t st = static_cast<cudaStream_t>(stream);
    // Four-token jobs pay off once experts can see several tokens per step.
    const bool quad = static_cast<int64_t>(tokens) * s->world >= 16 && mma_quad_supported(s->kind, s->hidden) &&
                      mma_quad_supported(s->kind, s->inter);
    EpGroupArgs a{};
    a.peers = s->peers;
    a.mb = s->mb;
    a.rank = s->rank;
    a.world = s->world;
    a.cap = s->cap;
    a.per_rank = s->per_rank;
    a.T = tokens;
    a.shared = s->shared;
    a.quad = quad;
    a.inter = s->inter;
    a.src = EpJobSrc{s->gate, s->up, s->down, s->sgate, s->sup, s->sdown, s->xprep,
                     reinterpret_cast<const uint8_t *>(s->mail + s->mb.fwd_rows), s->gu_stride, s->dn_stride,
                     s->xstride, nullptr, s->peers, s->mb.ret_rows, s->shared_out, s->rank, s->cap, s->hidden};
    a.g_out = s->g_out;
    a.u_out = s->u_out;
    a.hprep = s->hprep;
    a.hstride = s->hstride;
    a.gu_m = s->gu_m;
    a.dn_m = s->dn_m;
    a.gu_q = quad ? s->gu_q : nullptr;
    a.dn_q = s->dn_q;
    a.counts = s->counts;
    a.ctrl = s->ctrl;
    a.err = device_error_word();
    ep_group_kernel<<<1, kGroupThreads, 0, st>>>(a);
    int32_t rc = launch_status("ep_group_kernel");
    if (rc) return rc;
    const int P = s->pmax;
    const MmaJob none{};
    if ((rc = mma_gemv_device(s->kind, none, s->gu_m, s->counts, 2 * P, 0, s->inter, s->hidden, st)) ||
        (quad && (rc = mma_gemv_device(s->kind, none, s->gu_q, s->counts + 2, 2 * P, 0, s->inter, s->hidden, st,
                                       nullptr, 2))) ||
        (rc = prep_rows_device(s->hprep, s->g_out, s->u_out, P, s->inter, st, s->counts + 4)) ||
        (rc = mma_gemv_device(s->kind, none, s->dn_m, s->counts + 1, P, 0, s->hidden, s->inter, st)) ||
        (quad && (rc = mma_gemv_device(s->kind, none, s->dn_q, s->counts + 3, P, 0, s->hidden, s->inter, st, nullptr,
                                       2))))
        return rc;
    ep_return_kernel<<<1, 32, 0, st>>>(s->peers, s->mb, s->rank, s->world, s->ctrl);
    return launch_status("ep_return_kernel");
}

// Step phase 3: wait for every owner's outputs, then y [tokens, hidden]
// (device) = the ordered combine plus the shared expert.
GLMVX_EXPORT int32_t glmvx_ep_combine(void *layer, float *y, int32_t tokens, void *stream) {
    auto *s = static_cast<EpState *>(layer);
    if (const int32_t rc = check_state(s, "ep_combine")) return rc;
    if (tokens < 0 || tokens > s->max_tokens) return set_error("ep_combine: tokens must be 0..%d", s->max_tokens), kInvalid;
    if (tokens && !y) return set_error("ep_combine: null output"), kInvalid;
    const dim3 grid((s->hidden + 255) / 256, std::max(tokens, 1));  // with no tokens one row of CTAs still waits
    ep_combine_kernel<<<grid, 256, 0, static_cast<cudaStream_t>(stream)>>>(
        y, s->mail, s->mb, s->comb, s->combw, s->shared ? s->shared_out : nullptr, tokens, s->top_k, s->hidden, s->world,
        s->ctrl, device_error_word());
    return launch_status("ep_combine_kernel");
}

// One whole step on this rank (the three phases in order).
GLMVX_EXPORT int32_t glmvx_ep_step(void *layer, float *y, const float *x, int32_t tokens, int32_t *ids_out,
                                   float *weights_out, void *stream) {
    int32_t rc = glmvx_ep_dispatch(layer, x, tokens, ids_out, weights_out, stream);
    if (!rc) rc = glmvx_ep_experts(layer, tokens, stream);
    if (!rc) rc = glmvx_ep_combine(layer, y, tokens, stream);
    return rc;
}

// Frees the mailbox and scratch (after every rank's last step has finished
// and the peers have closed their mappings of this mailbox).
GLMVX_EXPORT int32_t glmvx_ep_destroy(void *layer) {
    auto *s = static_cast<EpState *>(layer);
    if (!s) return kOk;
    int prev = -1;
    cudaGetDevice(&prev);
    cudaSetDevice(s->device);
    cudaDeviceSynchronize();
    cudaFree(s->mail);
    cudaFree(s->scratch);
    if (prev >= 0) cudaSetDevice(prev);
    delete s;
    return kOk;
}
