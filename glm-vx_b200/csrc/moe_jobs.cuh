// Grouping of (token, expert) assignments into tensor-core job lists, shared
// by the single-GPU MoE layer (moe.cu) and the expert-parallel layer
// (ep.cu).  One CTA of kGroupThreads threads does the whole grouping.
//
// Assignment a (0 <= a < n) names a routed expert g.ids[a] and a prepared
// activation row; its rank r is its index in the order (expert, a), so the
// pairs of one expert are contiguous and ordered by a.  Consecutive pairs of
// one expert share a job of two token slots; with `quad`, experts holding
// three or more pairs (and the shared expert's pairs) go to a second list of
// four slots per job, so their weights are decoded once per four tokens.
// Per pair rank r the gate/up outputs are rows r of g_out/u_out and the down
// input is prepared row r of hprep; the shared expert's ns pairs take ranks
// n .. n+ns-1.  A token's arithmetic is the same in every job and slot, so
// results do not depend on how the pairs were grouped.
#pragma once

#include "mma_gemv.cuh"

namespace glmvx {

constexpr int kGroupThreads = 512, kMaxAssignments = 4096;

struct GroupSmem {
    int16_t ids[kMaxAssignments];   // expert of each assignment (< 32768)
    int16_t pair[kMaxAssignments];  // rank of each assignment
    int16_t job[kMaxAssignments];   // per rank: opens a two-token job (0/1), then the job id + 1
    int16_t jobq[kMaxAssignments];  // per rank: opens a four-token job, then the job id + 1
    int8_t list[kMaxAssignments];   // per rank: 1 = four-token list
    int32_t warp[kGroupThreads / 32];
};

// Inclusive prefix sum of v[0..n) in place (n <= kMaxAssignments), whole CTA.
__device__ inline void block_inclusive_scan(int16_t *v, int n, int32_t *s_warp) {
    const int per = (n + kGroupThreads - 1) / kGroupThreads;
    const int b0 = min(static_cast<int>(threadIdx.x) * per, n), b1 = min(b0 + per, n);
    int sum = 0;
    for (int i = b0; i < b1; ++i) sum += v[i];
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    int incl = sum;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const int y = __shfl_up_sync(0xffffffffu, incl, o);
        if (lane >= o) incl += y;
    }
    if (lane == 31) s_warp[warp] = incl;
    __syncthreads();
    int before = 0;
    for (int w = 0; w < warp; ++w) before += s_warp[w];
    int run = before + incl - sum;
    for (int i = b0; i < b1; ++i) {
        run += v[i];
        v[i] = static_cast<int16_t>(run);
    }
    __syncthreads();
}

// g.ids[0..n) must be filled and visible (after a __syncthreads).  Writes
// g.pair, the job lists and counts[0..3] = {two-token gate+up jobs (gate then
// up), two-token down jobs, four-token gate+up jobs, four-token down jobs}.
// Src supplies the addresses (device functions, called with a < n or t < ns):
//   wg(e), wu(e), wd(e)             routed expert matrices
//   sg(), su(), sd()                shared expert matrices
//   xp(a), out(a, r)                prepared input row / down output row of
//                                   routed assignment a of rank r
//   xp_shared(t), out_shared(t, r)  the same for shared-expert pair t
template <class Src>
__device__ void form_mma_jobs(const Src &src, GroupSmem &g, int n, int ns, bool quad, float *g_out, float *u_out,
                              const uint8_t *hprep, size_t hstride, int inter, MmaJob *gu_m, MmaJob *dn_m,
                              MmaJob *gu_q, MmaJob *dn_q, int *counts) {
    for (int a = threadIdx.x; a < n; a += blockDim.x) {
        const int e = g.ids[a];
        int lt = 0, eq = 0, cnt = 0;
        for (int b = 0; b < n; ++b) {
            const int eb = g.ids[b];
            lt += eb < e;
            eq += (eb == e) & (b < a);
            cnt += eb == e;
        }
        const int rank = lt + eq;
        g.pair[a] = static_cast<int16_t>(rank);
        const bool q4 = quad && cnt >= 3;
        g.list[rank] = q4;
        g.job[rank] = static_cast<int16_t>(!q4 && (eq & 1) == 0);
        g.jobq[rank] = static_cast<int16_t>(q4 && (eq & 3) == 0);
    }
    __syncthreads();
    block_inclusive_scan(g.job, n, g.warp);   // g.job[r] = 1 + id of the two-token job holding rank r
    block_inclusive_scan(g.jobq, n, g.warp);  // g.jobq[r] = 1 + id of the four-token job holding rank r
    const bool shared_q = quad;
    const int routed = n ? g.job[n - 1] : 0, routed_q = n ? g.jobq[n - 1] : 0;
    const int J = routed + (!shared_q ? (ns + 1) / 2 : 0);
    const int JQ = routed_q + (shared_q ? (ns + 3) / 4 : 0);
    // Pass 0 writes whole jobs from the pair in slot 0 (other slots empty),
    // pass 1 fills the other slots.
    for (int pass = 0; pass < 2; ++pass) {
        for (int a = threadIdx.x; a < n + ns; a += blockDim.x) {
            int r, j, slot;
            bool q4;
            const uint8_t *wg, *wu, *wd, *xp;
            float *po;
            if (a < n) {
                const int e = g.ids[a];
                r = g.pair[a];
                q4 = g.list[r];
                slot = 0;
                if (q4) {  // preceding ranks of the same four-token job
                    j = g.jobq[r] - 1;
                    for (int c = 1; c <= 3 && r - c >= 0 && g.list[r - c] && g.jobq[r - c] == g.jobq[r]; ++c)
                        slot = c;
                } else {
                    j = g.job[r] - 1;
                    slot = (r > 0 && !g.list[r - 1] && g.job[r - 1] == g.job[r]) ? 1 : 0;
                }
                if ((slot != 0) != (pass != 0)) continue;
                wg = src.wg(e);
                wu = src.wu(e);
                wd = src.wd(e);
                xp = src.xp(a);
                po = src.out(a, r);
            } else {
                const int t = a - n;
                r = n + t;
                q4 = shared_q;
                j = q4 ? routed_q + t / 4 : routed + t / 2;
                slot = q4 ? t & 3 : t & 1;
                if ((slot != 0) != (pass != 0)) continue;
                wg = src.sg();
                wu = src.su();
                wd = src.sd();
                xp = src.xp_shared(t);
                po = src.out_shared(t, r);
            }
            const uint8_t *hp = hprep + static_cast<size_t>(r) * hstride;
            float *go = g_out + static_cast<size_t>(r) * inter, *uo = u_out + static_cast<size_t>(r) * inter;
            MmaJob *gl = q4 ? gu_q : gu_m, *dl = q4 ? dn_q : dn_m;
            const int Jl = q4 ? JQ : J;
            if (slot == 0) {
                gl[j] = MmaJob{wg, {xp}, {go}};
                gl[Jl + j] = MmaJob{wu, {xp}, {uo}};
                dl[j] = MmaJob{wd, {hp}, {po}};
            } else {
                gl[j].xp[slot] = xp;
                gl[j].out[slot] = go;
                gl[Jl + j].xp[slot] = xp;
                gl[Jl + j].out[slot] = uo;
                dl[j].xp[slot] = hp;
                dl[j].out[slot] = po;
            }
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        counts[0] = 2 * J;
        counts[1] = J;
        counts[2] = 2 * JQ;
        counts[3] = JQ;
    }
}

}  // namespace glmvx
