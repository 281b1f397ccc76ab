// gmoe.cu — the GLM-5.3-Flash MoE sublayer on the B200 (c/gmoe.h semantics).
//
// Decode shape: R <= 8 token rows, E routed experts (288) + 1 shared expert,
// top-k (8).  Per layer call, with no host round-trip:
//   1. router GEMV: fp32 logits [R][E] = x . gate_w (c/gmoe.h:168-173);
//   2. k_moe_route (one CTA): sigmoid (numpy-stable), +bias for selection,
//      stable top-k with lower-index ties, weights from the unbiased scores
//      normalised with the numpy pairwise sum and scaled (c/gmoe.h:191-208);
//      builds the device work list: the union of selected experts in
//      ascending order plus the shared expert last;
//   3. grouped FP8 GEMV over the work list: gate|up rows [2*inter][dim] of
//      every active expert -> gu [P][R][2*inter];
//   4. grouped FP8 GEMV down [dim][inter] whose activation staging applies the
//      SwiGLU with the clamps (c/gmoe.h:216-224) -> yd [P][R][dim];
//   5. k_moe_combine: per row, ascending expert index, contrib =
//      bf16(bf16(expert) * w) and y = bf16(y + contrib), shared expert last
//      (c/gmoe.h:305-336).
// Expert weights live in HBM packed per layer: codes [E+1][2*inter][dim]
// (gate rows then up rows; expert E is the shared expert) and
// [E+1][dim][inter], F32 128x128 block scales packed the same way.
#include "common.cuh"
#include "gcuda.h"
#include "gmoe_dev.h"

namespace apus {

__device__ int g_apus_ep_err;   // 5: an expert-parallel barrier gave up waiting

// c/gmhc.h:165-185 for n <= 8 (the router weight sum, n = topk)
APUS_DEV float pw_sum_small(const float *a, int n) {
    if (n < 8) {
        float r = a[0];
        for (int i = 1; i < n; i++) r += a[i];
        return r;
    }
    return pw_sum_leaf(a, n);
}

// The selection of one row r by one warp (c/gmoe.h:168-208): sigmoid
// (numpy-stable), +bias for selection, stable top-k with lower-index ties,
// weights from the unbiased scores normalised with the numpy pairwise sum and
// scaled.  Writes row_expert / row_weight (ascending experts) and row_sel (top-k
// order) at row r; sc is the row's score scratch; flag[e] = 1 for each
// selection when flag is given.
APUS_DEV void route_row(const MoeDev &m, int r, const float *logits_row, const int32_t *forced_row, float *sc,
                        int *flag) {
    const int E = m.E, K = m.topk;
    const int lane = threadIdx.x & 31;
    constexpr int EPL = MOE_MAX_E / 32;       // experts per lane: e = lane + 32u
    {
        float lg[EPL], bs[EPL];
#pragma unroll
        for (int u = 0; u < EPL; u++) {       // every load first
            const int e = lane + 32 * u;
            lg[u] = e < E ? logits_row[e] : 0.f;
            bs[u] = e < E ? m.gate_bias[e] : 0.f;
        }
        // selection key of the biased score: larger value first, lower index
        // on ties (the strict-greater scan of c/gmoe.h:175-189)
        unsigned long long key[EPL];
#pragma unroll
        for (int u = 0; u < EPL; u++) {
            const int e = lane + 32 * u;
            const float s = sigmoid_np(lg[u]);
            if (e < E) sc[e] = s;
            key[u] = e < E ? argmax_key(s + bs[u], (uint32_t)e) : 0ull;
        }
        __syncwarp();
        int my_sel = -1;                      // lane j < K: the j-th selection
        for (int j = 0; j < K; j++) {
            unsigned long long best = 0ull;
#pragma unroll
            for (int u = 0; u < EPL; u++) best = key[u] > best ? key[u] : best;
#pragma unroll
            for (int off = 16; off; off >>= 1) {
                const unsigned long long o = __shfl_xor_sync(0xffffffffu, best, off);
                best = o > best ? o : best;
            }
            const int idx = (int)argmax_key_index(best);
#pragma unroll
            for (int u = 0; u < EPL; u++)     // the winner leaves the pool
                if (lane + 32 * u == idx) key[u] = 0ull;
            const int pick = forced_row ? forced_row[j] : idx;
            if (lane == j) my_sel = pick;
        }
        __syncwarp();
        // weights from the unbiased scores, normalised with the numpy
        // pairwise sum in selection order (c/gmoe.h:191-208)
        float w = lane < K ? sc[my_sel] : 0.f;
        float wa[MOE_MAX_TOPK];
#pragma unroll
        for (int j = 0; j < MOE_MAX_TOPK; j++) wa[j] = __shfl_sync(0xffffffffu, w, j);
        const float sum = K ? pw_sum_small(wa, K) : 0.f;
        w = w / (sum + 1e-20f) * m.route_scale;
        // ascending expert order for the combine: rank among the selections
        int rank = 0;
#pragma unroll
        for (int j = 0; j < MOE_MAX_TOPK; j++) {
            const int o = __shfl_sync(0xffffffffu, my_sel, j);
            if (j < K && lane < K && o < my_sel) rank++;
        }
        if (lane < K) {
            m.row_expert[r * K + rank] = my_sel;
            m.row_weight[r * K + rank] = w;
            // unsorted selection, for inspection (c/gmoe.h:112-117 router_idx)
            m.row_sel[r * K + lane] = my_sel;
            if (flag) flag[my_sel] = 1;
        }
    }
}

__global__ void __launch_bounds__(256) k_moe_route(MoeDev m, int R, const float *logits, const int32_t *forced) {
    pdl_launch_dependents();
    __shared__ float sc[MOE_MAX_R][MOE_MAX_E];
    __shared__ int flag[MOE_MAX_E + 1];
    __shared__ int slot_of[MOE_MAX_E + 1];
    const int E = m.E, K = m.topk;
    for (int e = threadIdx.x; e <= E; e += blockDim.x) flag[e] = 0;
    __syncthreads();
    const int warp = threadIdx.x >> 5;
    if (warp < R)        // one warp per row
        route_row(m, warp, logits + (size_t)warp * E, forced ? forced + warp * K : nullptr, sc[warp], flag);
    __syncthreads();
    // work list: the flagged experts in ascending order (slot_of[e] = flagged
    // experts before e), by a ballot + popc scan over blocks of blockDim experts
    __shared__ int wsum[32], run;
    if (threadIdx.x == 0) run = 0;
    __syncthreads();
    const int nw = blockDim.x >> 5;
    const int lo = m.e0, hi = m.e0 + m.eloc;  // this rank's routed experts
    for (int e0 = 0; e0 < E; e0 += blockDim.x) {
        const int e = e0 + threadIdx.x;
        const int f = (e >= lo && e < hi) ? flag[e] : 0;
        const unsigned bal = __ballot_sync(0xffffffffu, f);
        const int ln = threadIdx.x & 31, w = threadIdx.x >> 5;
        if (ln == 0) wsum[w] = __popc(bal);
        __syncthreads();
        int p = run + __popc(bal & ((1u << ln) - 1u));
        for (int k = 0; k < w; k++) p += wsum[k];
        if (e < E) {
            slot_of[e] = (e >= lo && e < hi) ? p : -1;   // -1: another rank's expert
            if (f) m.prob_expert[p] = e - lo;             // local weight slot
        }
        __syncthreads();
        if (threadIdx.x == 0) {
            int tot = 0;
            for (int k = 0; k < nw; k++) tot += wsum[k];
            run += tot;
        }
        __syncthreads();
    }
    if (threadIdx.x == 0) {
        const int p = run;
        slot_of[E] = p;
        m.prob_expert[p] = m.eloc;         // shared expert (local slot eloc), always last
        *m.prob_count = p + 1;
        if (m.stat_problems) atomicAdd(m.stat_problems, (unsigned long long)(p + 1));
    }
    __syncthreads();
    for (int i = threadIdx.x; i < R * K; i += blockDim.x)
        m.row_prob[i] = slot_of[m.row_expert[i]];
    if (threadIdx.x < R) m.row_prob_shared[threadIdx.x] = slot_of[E];
    if (m.prob_slot) {   // (problem, row) -> selection slot, for the scatter epilogue
        const int np = slot_of[E] + 1;
        for (int i = threadIdx.x; i < np * 8; i += blockDim.x) m.prob_slot[i] = -1;
        __syncthreads();
        for (int i = threadIdx.x; i < R * K; i += blockDim.x) {
            const int p = slot_of[m.row_expert[i]];
            if (p >= 0) m.prob_slot[p * 8 + i / K] = i % K;
        }
    }
}

// out[r][i] = bf16(y + shared), y = ascending bf16 accumulation of
// bf16(bf16(expert) * w) (c/gmoe.h:305-336).  A thread owns 8 consecutive
// columns of one row; every expert row's 16-byte load is issued first.
__global__ void k_moe_combine(MoeDev m, int R, uint16_t *out, long ldo) {
    pdl_launch_dependents();
    const int d = m.dim, K = m.topk, nc = d / 8;
    const size_t pstride = (size_t)m.max_r * d;
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * nc) return;
    const int r = (int)(i / nc), c = (int)(i % nc) * 8;
    uint4 ev[MOE_MAX_TOPK + 1];
    float wt[MOE_MAX_TOPK];
#pragma unroll
    for (int j = 0; j < MOE_MAX_TOPK; j++)
        if (j < K) {
            const int p = m.row_prob[r * K + j];
            ev[j] = *(const uint4 *)(m.yd + p * pstride + (size_t)r * d + c);
            wt[j] = m.row_weight[r * K + j];
        }
    ev[MOE_MAX_TOPK] = *(const uint4 *)(m.yd + m.row_prob_shared[r] * pstride + (size_t)r * d + c);
    const uint32_t sw[4] = {ev[MOE_MAX_TOPK].x, ev[MOE_MAX_TOPK].y, ev[MOE_MAX_TOPK].z, ev[MOE_MAX_TOPK].w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 8; e++) {
        float y = 0.f;
#pragma unroll
        for (int j = 0; j < MOE_MAX_TOPK; j++) {
            if (j >= K) break;
            const uint32_t wd = (e >> 1) == 0 ? ev[j].x : (e >> 1) == 1 ? ev[j].y : (e >> 1) == 2 ? ev[j].z : ev[j].w;
            const float ex = (e & 1) ? bf16hi(wd) : bf16lo(wd);
            y = bf16_round(y + bf16_round(ex * wt[j]));
        }
        const uint16_t shb = (uint16_t)((e & 1) ? sw[e >> 1] >> 16 : sw[e >> 1] & 0xffffu);
        // a dense MLP (no routed experts) passes its output through unchanged
        const uint16_t v = K ? bf16_bits(y + bf16_f32(shb)) : shb;
        if (e & 1) o[e >> 1] |= (uint32_t)v << 16;
        else o[e >> 1] = v;
    }
    *(uint4 *)(out + (size_t)r * ldo + c) = make_uint4(o[0], o[1], o[2], o[3]);
}

// ---- the prompt pass: many rows a call (one GPU) ---------------------------

__global__ void __launch_bounds__(256) k_moe_route_rows(MoeDev m, MoeRows w, int R, const float *logits) {
    __shared__ float sc[MOE_MAX_R][MOE_MAX_E];
    const int warp = threadIdx.x >> 5, r = blockIdx.x * MOE_MAX_R + warp;
    if (r >= R) return;        // whole warps; no block barrier follows
    m.row_expert = w.row_expert;
    m.row_weight = w.row_weight;
    m.row_sel = w.row_sel;
    route_row(m, r, logits + (size_t)r * m.E, nullptr, sc[warp], nullptr);
}

// Problem lists: expert e's rows in ascending row order, 8 a problem, experts
// ascending; then the shared expert (local slot shared_id) over every row, 8
// a problem.  Thread e scans the selections for its own expert.
__global__ void __launch_bounds__(1024) k_moe_lists(MoeRows w, int R, int K, int E, int e0, int eloc,
                                                    int shared_id) {
    extern __shared__ int rex[];             // [R*K]
    __shared__ int cnt[MOE_MAX_E], pbase[MOE_MAX_E + 1];
    const int n = R * K, tid = threadIdx.x;
    for (int i = tid; i < n; i += blockDim.x) rex[i] = w.row_expert[i];
    for (int e = tid; e < E; e += blockDim.x) cnt[e] = 0;
    __syncthreads();
    for (int i = tid; i < n; i += blockDim.x) atomicAdd(&cnt[rex[i]], 1);
    __syncthreads();
    if (tid == 0) {
        int p = 0;
        for (int e = 0; e < E; e++) {
            pbase[e] = p;
            if (e >= e0 && e < e0 + eloc) p += (cnt[e] + 7) / 8;     // this rank's experts only
        }
        pbase[E] = p;
    }
    __syncthreads();
    for (int e = tid; e < E; e += blockDim.x) {
        const bool mine = e >= e0 && e < e0 + eloc;
        const int pb = pbase[e], np = pbase[e + 1] - pb;
        for (int q = 0; q < np; q++) {
            w.prob_expert[pb + q] = e - e0;                        // local weight slot
            for (int s = 0; s < 8; s++) w.prob_rows[(pb + q) * 8 + s] = -1;
        }
        int c = 0;
        for (int i = 0; i < n; i++)
            if (rex[i] == e) {
                if (!mine) { w.pair_slot[i] = -1; continue; }       // another rank's output
                const int slot = pb * 8 + c++;
                w.prob_rows[slot] = i / K;
                w.pair_slot[i] = slot;
            }
    }
    const int p0 = pbase[E], ns = (R + 7) / 8;
    for (int q = tid; q < ns * 8; q += blockDim.x) {
        const int p = p0 + q / 8;
        if (q % 8 == 0) w.prob_expert[p] = shared_id;
        w.prob_rows[q + p0 * 8] = q < R ? q : -1;
        if (q < R) w.shared_slot[q] = p0 * 8 + q;
    }
    if (tid == 0) *w.prob_count = p0 + ns;
}

// xg[slot] = x[prob_rows[slot]] (zeros for padding), one CTA per problem row.
__global__ void k_moe_gather(const uint16_t *x, long ldx, MoeRows w, int d) {
    const int slot = blockIdx.x;
    if (slot / 8 >= *w.prob_count) return;
    const int t = w.prob_rows[slot];
    for (int c = threadIdx.x; c < d / 8; c += blockDim.x) {
        const uint4 v = t >= 0 ? *(const uint4 *)(x + (size_t)t * ldx + c * 8) : make_uint4(0, 0, 0, 0);
        *(uint4 *)(w.xg + (size_t)slot * d + c * 8) = v;
    }
}

// The ordered combine of k_moe_combine over the gathered outputs.
__global__ void k_moe_combine_rows(MoeRows w, int R, int K, int d, uint16_t *out, long ldo) {
    const int nc = d / 8;
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * nc) return;
    const int r = (int)(i / nc), c = (int)(i % nc) * 8;
    uint4 ev[MOE_MAX_TOPK + 1];
    float wt[MOE_MAX_TOPK];
#pragma unroll
    for (int j = 0; j < MOE_MAX_TOPK; j++)
        if (j < K) {
            ev[j] = *(const uint4 *)(w.yd + (size_t)w.pair_slot[r * K + j] * d + c);
            wt[j] = w.row_weight[r * K + j];
        }
    ev[MOE_MAX_TOPK] = *(const uint4 *)(w.yd + (size_t)w.shared_slot[r] * d + c);
    const uint32_t sw[4] = {ev[MOE_MAX_TOPK].x, ev[MOE_MAX_TOPK].y, ev[MOE_MAX_TOPK].z, ev[MOE_MAX_TOPK].w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 8; e++) {
        float y = 0.f;
#pragma unroll
        for (int j = 0; j < MOE_MAX_TOPK; j++) {
            if (j >= K) break;
            const uint32_t wd = (e >> 1) == 0 ? ev[j].x : (e >> 1) == 1 ? ev[j].y : (e >> 1) == 2 ? ev[j].z : ev[j].w;
            const float ex = (e & 1) ? bf16hi(wd) : bf16lo(wd);
            y = bf16_round(y + bf16_round(ex * wt[j]));
        }
        const uint16_t shb = (uint16_t)((e & 1) ? sw[e >> 1] >> 16 : sw[e >> 1] & 0xffffu);
        const uint16_t v = bf16_bits(y + bf16_f32(shb));
        if (e & 1) o[e >> 1] |= (uint32_t)v << 16;
        else o[e >> 1] = v;
    }
    *(uint4 *)(out + (size_t)r * ldo + c) = make_uint4(o[0], o[1], o[2], o[3]);
}

// Expert parallelism: this rank's weighted outputs bf16(bf16(y) * w) into its
// region's half (epoch+1)&1 at [row][slot j] (the slot order of the row's
// ascending expert list), one thread per (row, selection, 8 columns).
__global__ void k_moe_scatter_rows(MoeRows w, EpCtx ep, int R, int K, int d) {
    const int nc = d / 8;
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * K * nc) return;
    const int pr = (int)(i / nc), c = (int)(i % nc) * 8;
    const int slot = w.pair_slot[pr];
    if (slot < 0) return;
    const int r = pr / K, j = pr % K;
    const int half = (*(volatile int *)ep.epoch + 1) & 1;
    const float wt = w.row_weight[pr];
    const uint4 v = *(const uint4 *)(w.yd + (size_t)slot * d + c);
    const uint32_t in[4] = {v.x, v.y, v.z, v.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
        const uint16_t lo = bf16_bits(bf16_round(bf16lo(in[e]) * wt)), hi = bf16_bits(bf16_round(bf16hi(in[e]) * wt));
        o[e] = (uint32_t)lo | ((uint32_t)hi << 16);
    }
    uint16_t *dst = (uint16_t *)(ep.peer[ep.rank] + ep.off_wide) +
                    ((((size_t)half * ep.wide_rows + r) * ep.wide_k + j) * d + c);
    *(uint4 *)dst = make_uint4(o[0], o[1], o[2], o[3]);
}

APUS_DEV void ep_signal_wait(const EpCtx &ep, int e, bool signal);

// One thread: signal every peer, wait for every peer's signal of the same
// epoch (bounded), advance the epoch.  The combine that follows in the stream
// reads the peers' regions.
__global__ void k_ep_barrier(EpCtx ep) {
    const int e = *(volatile int *)ep.epoch + 1;
    ep_signal_wait(ep, e, true);
    ep.epoch[0] = e;
}

// The ordered combine across ranks: per row, the slots in ascending expert
// order from their owners' regions, y = bf16(y + contribution), then the
// local shared expert.
__global__ void k_moe_combine_ep_rows(MoeRows w, EpCtx ep, int R, int K, int d, int eloc, uint16_t *out, long ldo) {
    const int nc = d / 8;
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * nc) return;
    const int r = (int)(i / nc), c = (int)(i % nc) * 8;
    const int half = *(volatile int *)ep.epoch & 1;
    uint4 ev[MOE_MAX_TOPK];
#pragma unroll
    for (int j = 0; j < MOE_MAX_TOPK; j++)
        if (j < K) {
            const int owner = w.row_expert[r * K + j] / eloc;
            const uint16_t *src = (const uint16_t *)(ep.peer[owner] + ep.off_wide) +
                                  ((((size_t)half * ep.wide_rows + r) * ep.wide_k + j) * d + c);
            ev[j] = __ldcv((const uint4 *)src);
        }
    const uint4 sh = *(const uint4 *)(w.yd + (size_t)w.shared_slot[r] * d + c);
    const uint32_t sw[4] = {sh.x, sh.y, sh.z, sh.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 8; e++) {
        float y = 0.f;
#pragma unroll
        for (int j = 0; j < MOE_MAX_TOPK; j++) {
            if (j >= K) break;
            const uint32_t wd = (e >> 1) == 0 ? ev[j].x : (e >> 1) == 1 ? ev[j].y : (e >> 1) == 2 ? ev[j].z : ev[j].w;
            y = bf16_round(y + ((e & 1) ? bf16hi(wd) : bf16lo(wd)));
        }
        const uint16_t shb = (uint16_t)((e & 1) ? sw[e >> 1] >> 16 : sw[e >> 1] & 0xffffu);
        const uint16_t v = bf16_bits(y + bf16_f32(shb));
        if (e & 1) o[e >> 1] |= (uint32_t)v << 16;
        else o[e >> 1] = v;
    }
    *(uint4 *)(out + (size_t)r * ldo + c) = make_uint4(o[0], o[1], o[2], o[3]);
}

// ---- expert parallelism --------------------------------------------------
// Every rank's down GEMV scatters bf16(bf16(expert) * w) of its own experts
// into its exchange region (half (epoch+1)&1, [row][slot j][dim], the slot
// order of the row's ascending expert list).  One exchange kernel then
// signals every peer, waits for every peer's signal of the same epoch and
// sums the slots from their owners' regions in slot order, the same
// ascending-expert BF16 accumulation as k_moe_combine.

// Thread 0 of a CTA: signal (CTA 0 only) and wait for every rank's epoch-e
// signal.  Each wait is bounded (about a second of clock cycles) and records
// an error instead of hanging.
// The signal is the release pattern of the PTX memory model (one fence at
// system scope, then relaxed flag stores to every peer) and the wait its
// acquire pattern (relaxed polls, then one fence), so the fence cost is paid
// once per exchange rather than once per peer.
APUS_DEV void ep_signal_wait(const EpCtx &ep, int e, bool signal) {
    if (signal) {
        asm volatile("fence.acq_rel.sys;" ::: "memory");
        for (int p = 0; p < ep.world; p++) {
            int *pf = (int *)(ep.peer[p] + ep.off_flags) + ep.rank;
            asm volatile("st.relaxed.sys.global.s32 [%0], %1;" ::"l"(pf), "r"(e) : "memory");
        }
    }
    const int *mine = (const int *)(ep.peer[ep.rank] + ep.off_flags);
    const long long t0 = clock64();
    for (int p = 0; p < ep.world; p++) {
        int v = 0;
        while (true) {
            asm volatile("ld.relaxed.sys.global.s32 %0, [%1];" : "=r"(v) : "l"(mine + p) : "memory");
            if (v >= e) break;
            if (clock64() - t0 > (1ll << 31)) {
                atomicExch(&g_apus_ep_err, 5);
                return;
            }
        }
    }
    asm volatile("fence.acq_rel.sys;" ::: "memory");
}

// Every CTA reads the epoch before it arrives; the last CTA to arrive (all
// others have read it by then) advances it for the next exchange.
APUS_DEV void ep_arrive(const EpCtx &ep, int e) {
    if (atomicAdd(ep.epoch + 1, 1) == (int)gridDim.x - 1) {
        ep.epoch[1] = 0;
        ep.epoch[0] = e;
    }
}

__global__ void k_moe_exchange(MoeDev m, int R, uint16_t *out, long ldo) {
    __shared__ int e_sh;
    if (threadIdx.x == 0) {
        const int e = *(volatile int *)m.ep.epoch + 1;
        e_sh = e;
        ep_signal_wait(m.ep, e, blockIdx.x == 0);
        ep_arrive(m.ep, e);
    }
    __syncthreads();
    pdl_launch_dependents();
    const int d = m.dim, K = m.topk, nc = d / 8;
    const size_t pstride = (size_t)m.max_r * d;
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * nc) return;
    const int r = (int)(i / nc), c = (int)(i % nc) * 8;
    const int half = e_sh & 1;
    uint4 ev[MOE_MAX_TOPK];
#pragma unroll
    for (int j = 0; j < MOE_MAX_TOPK; j++)
        if (j < K) {
            const int owner = m.row_expert[r * K + j] / m.eloc;
            const uint16_t *src = (const uint16_t *)m.ep.peer[owner] +
                                  (((size_t)half * MOE_MAX_R + r) * MOE_MAX_TOPK + j) * d + c;
            ev[j] = __ldcv((const uint4 *)src);          // a peer's region: fetched afresh, never cached
        }
    const uint4 sh = *(const uint4 *)(m.yd + m.row_prob_shared[r] * pstride + (size_t)r * d + c);
    const uint32_t sw[4] = {sh.x, sh.y, sh.z, sh.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 8; e++) {
        float y = 0.f;
#pragma unroll
        for (int j = 0; j < MOE_MAX_TOPK; j++) {
            if (j >= K) break;
            const uint32_t wd = (e >> 1) == 0 ? ev[j].x : (e >> 1) == 1 ? ev[j].y : (e >> 1) == 2 ? ev[j].z : ev[j].w;
            y = bf16_round(y + ((e & 1) ? bf16hi(wd) : bf16lo(wd)));
        }
        const uint16_t shb = (uint16_t)((e & 1) ? sw[e >> 1] >> 16 : sw[e >> 1] & 0xffffu);
        const uint16_t v = bf16_bits(y + bf16_f32(shb));
        if (e & 1) o[e >> 1] |= (uint32_t)v << 16;
        else o[e >> 1] = v;
    }
    *(uint4 *)(out + (size_t)r * ldo + c) = make_uint4(o[0], o[1], o[2], o[3]);
}

// One warp: publish this rank's argmax keys, signal, wait, reduce over ranks.
__global__ void k_ep_picks(EpCtx ep, const unsigned long long *keys, int R, int *picks, int n0, int *picks2) {
    __shared__ int e_sh;
    const int lane = threadIdx.x;
    if (lane == 0) e_sh = *(volatile int *)ep.epoch + 1;
    __syncwarp();
    const int e = e_sh, half = e & 1;
    unsigned long long *kd = (unsigned long long *)(ep.peer[ep.rank] + ep.off_keys) + (size_t)half * MOE_MAX_R;
    if (lane < R) kd[lane] = keys[lane];
    __syncwarp();
    if (lane == 0) {
        ep_signal_wait(ep, e, true);
        ep.epoch[0] = e;                                // one CTA: nobody else reads it
    }
    __syncwarp();
    pdl_launch_dependents();
    if (lane >= R) return;
    unsigned long long best = 0ull;
    for (int p = 0; p < ep.world; p++) {
        const unsigned long long k =
            __ldcv((const unsigned long long *)(ep.peer[p] + ep.off_keys) + (size_t)half * MOE_MAX_R + lane);
        best = k > best ? k : best;
    }
    if (lane < n0) picks[lane] = (int)argmax_key_index(best);
    else picks2[lane - n0] = (int)argmax_key_index(best);
}

}  // namespace apus

using namespace apus;

static bool ep_connected(const EpCtx &ep);

int moe_forward_launch(const MoeDev &m, const uint16_t *x, long ldx, int R, uint16_t *out, long ldo,
                       const int32_t *forced, cudaStream_t st) {
    if (R < 1 || R > m.max_r || R > MOE_MAX_R) return -1;
    // 1. router logits (fp32, no rounding); a dense MLP has no router
    if (m.E > 0) {
        GemvDesc r{};
        r.W = m.gate_w; r.x = x; r.ldx = ldx; r.R = R; r.O = m.E; r.K = m.dim; r.fp8 = 0;
        r.yf = m.logits; r.ldyf = m.E;
        r.part = m.part; r.ticket = m.tick;
        r.pdl = m.pdl;
        if (gemv_launch(r, st)) return -1;
    }
    // 2. routing + work list
    k_moe_route<<<1, 256, 0, st>>>(m, R, m.logits, forced);
    if (cudaGetLastError() != cudaSuccess) return -1;
    if (m.E == 0) {
        // a dense MLP (the shared expert of a 0-expert layer): two single
        // GEMVs, the down one split over K when the width passes one range
        // (intermediate 12288 in the reference's first three layers)
        GemvDesc gs{};
        gs.W = m.gu_codes; gs.WS = m.gu_scales; gs.nkb = (m.dim + 127) / 128;
        gs.x = x; gs.ldx = ldx; gs.R = R; gs.O = 2L * m.inter; gs.K = m.dim; gs.fp8 = 1;
        gs.y = m.gu; gs.ldy = 2L * m.inter;
        gs.part = m.part; gs.ticket = m.tick;
        gs.pdl = m.pdl;
        if (gemv_launch(gs, st)) return -1;
        GemvDesc ds{};
        ds.W = m.d_codes; ds.WS = m.d_scales; ds.nkb = (m.inter + 127) / 128;
        ds.x = m.gu; ds.ldx = 2L * m.inter; ds.R = R; ds.O = m.dim; ds.K = m.inter; ds.fp8 = 1;
        ds.y = m.yd; ds.ldy = m.dim;
        ds.x_swiglu = 1;
        ds.swiglu_limit = m.limit;
        ds.part = m.part; ds.ticket = m.tick;
        ds.pdl = m.pdl;
        if (gemv_launch(ds, st)) return -1;
        if (!out) return cudaGetLastError() != cudaSuccess ? -1 : 0;
        if (m.dim % 8 || ((uintptr_t)out & 15) || (ldo % 8)) return -1;
        const long n = (long)R * (m.dim / 8);
        k_moe_combine<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(m, R, out, ldo);
        return cudaGetLastError() == cudaSuccess ? 0 : -1;
    }
    // 3. gate|up of every active expert
    GemvDesc gu{};
    gu.W = m.gu_codes; gu.WS = m.gu_scales; gu.nkb = (m.dim + 127) / 128;
    gu.x = x; gu.ldx = ldx; gu.R = R; gu.O = 2L * m.inter; gu.K = m.dim; gu.fp8 = 1;
    gu.y = m.gu; gu.ldy = 2L * m.inter;
    gu.gexpert = m.prob_expert; gu.gcount = m.prob_count; gu.gmax = R * m.topk + 1; gu.gnum = m.eloc + 1;
    gu.w_estride = 2L * m.inter * m.dim;
    gu.s_estride = (2L * m.inter / 128) * ((m.dim + 127) / 128);
    gu.x_pstride = 0;
    gu.y_pstride = (long)m.max_r * 2 * m.inter;
    gu.pdl = m.pdl;
    if (gemv_launch(gu, st)) return -1;
    // 4. down with the SwiGLU applied while staging
    GemvDesc dn{};
    dn.W = m.d_codes; dn.WS = m.d_scales; dn.nkb = (m.inter + 127) / 128;
    dn.x = m.gu; dn.ldx = 2L * m.inter; dn.R = R; dn.O = m.dim; dn.K = m.inter; dn.fp8 = 1;
    dn.y = m.yd; dn.ldy = m.dim;
    dn.gexpert = m.prob_expert; dn.gcount = m.prob_count; dn.gmax = R * m.topk + 1; dn.gnum = m.eloc + 1;
    dn.w_estride = (long)m.dim * m.inter;
    dn.s_estride = ((m.dim + 127) / 128) * ((m.inter + 127) / 128);
    dn.x_pstride = (long)m.max_r * 2 * m.inter;
    dn.y_pstride = (long)m.max_r * m.dim;
    dn.x_swiglu = 1;
    dn.swiglu_limit = m.limit;
    dn.pdl = m.pdl;
    const bool ep = m.ep.world > 1 && m.E > 0;
    if (ep) {
        if (!ep_connected(m.ep) || m.eloc * m.ep.world != m.E || !m.prob_slot) return -1;
        dn.scat = (uint16_t *)m.ep.peer[m.ep.rank];
        dn.scat_slot = m.prob_slot;
        dn.scat_w = m.row_weight;
        dn.scat_epoch = m.ep.epoch;
        dn.scat_k = m.topk;
        dn.scat_j = MOE_MAX_TOPK;
        dn.scat_ld = m.dim;
    }
    if (gemv_launch(dn, st)) return -1;
    // 5. ordered combine (across ranks when the experts are split); with
    // out == null the caller combines (one GPU only)
    if (!out) return (ep || cudaGetLastError() != cudaSuccess) ? -1 : 0;
    if (m.dim % 8 || ((uintptr_t)out & 15) || (ldo % 8)) return -1;
    const long n = (long)R * (m.dim / 8);
    if (ep) {
        k_moe_exchange<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(m, R, out, ldo);
    } else {
        k_moe_combine<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(m, R, out, ldo);
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

// Every rank's region must be mapped before any exchange is launched.
int moe_combine_launch(const MoeDev &m, int R, uint16_t *out, long ldo, cudaStream_t st) {
    if (m.dim % 8 || ((uintptr_t)out & 15) || (ldo % 8) || R < 1 || R > m.max_r) return -1;
    const long n = (long)R * (m.dim / 8);
    k_moe_combine<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(m, R, out, ldo);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

static bool ep_connected(const EpCtx &ep) {
    if (ep.world < 2 || ep.world > EP_MAX_RANKS || ep.rank < 0 || ep.rank >= ep.world || !ep.epoch) return false;
    for (int p = 0; p < ep.world; p++)
        if (!ep.peer[p]) return false;
    return true;
}

// Rank p's slice is the rows [p*per, min((p+1)*per, V)), per = ceil(V/world)
// (the lm_head split); 8 columns a thread.
__global__ void k_ep_logits_gather(EpCtx ep, int R, uint16_t *logits, long ldl) {
    const int V = ep.vocab, nc = (V + 7) / 8;
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * nc) return;
    const int r = (int)(i / nc), c0 = (int)(i % nc) * 8;
    const int per = (V + ep.world - 1) / ep.world;
    for (int c = c0; c < c0 + 8 && c < V; c++) {
        const int owner = c / per;
        const uint16_t *src = (const uint16_t *)(ep.peer[owner] + ep.off_logits) + (size_t)r * V + c;
        logits[(size_t)r * ldl + c] = *(const volatile uint16_t *)src;
    }
}

int ep_logits_gather_launch(const EpCtx &ep, int R, uint16_t *logits, long ldl, cudaStream_t st) {
    if (!ep_connected(ep) || R < 1 || R > MOE_MAX_R || ep.vocab < 1) return -1;
    const long n = (long)R * ((ep.vocab + 7) / 8);
    k_ep_logits_gather<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(ep, R, logits, ldl);
    k_ep_barrier<<<1, 1, 0, st>>>(ep);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int ep_picks_exchange_launch(const EpCtx &ep, const unsigned long long *keys, int R, int *picks,
                             cudaStream_t st, int n0, int *picks2) {
    if (n0 < 0 || n0 > R) n0 = R;
    if (!ep_connected(ep) || R < 1 || R > MOE_MAX_R || !keys || !picks || (n0 < R && !picks2)) return -1;
    k_ep_picks<<<1, 32, 0, st>>>(ep, keys, R, picks, n0, picks2);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int ep_error_read_and_clear(void) {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_apus_ep_err, sizeof v);
    cudaMemcpyToSymbol(g_apus_ep_err, &z, sizeof z);
    return v;
}

size_t ep_wide_bytes(int rows, int topk, int dim) { return (size_t)2 * rows * topk * dim * 2; }

size_t ep_region_bytes(int dim) {
    const size_t contrib = (size_t)2 * MOE_MAX_R * MOE_MAX_TOPK * dim * 2;
    return contrib + 2 * MOE_MAX_R * 8 + EP_MAX_RANKS * 4 + 256;
}

// The MoE sublayer over R prompt rows (one GPU): router logits of every row
// on the tensor cores, each row's selection (the decode path's route_row),
// the problem lists, the rows gathered, the grouped FP8 GEMVs of the decode
// path over 8-row problems (so a (row, expert) output is the decode path's
// bit for bit), the ordered combine.
int moe_rows_launch(const MoeDev &m, const MoeRows &w, const uint16_t *x, long ldx, int R, uint16_t *out, long ldo,
                    cudaStream_t st) {
    const bool ep = m.ep.world > 1;
    if (m.E < 1 || R < 1 || R > w.W || m.dim % 8 || ldx % 8 || ldo % 8 || m.topk > MOE_MAX_TOPK) return -1;
    if (ep && (!ep_connected(m.ep) || m.ep.wide_rows < R || m.ep.wide_k < m.topk || m.eloc * m.ep.world != m.E))
        return -1;
    const int d = m.dim, K = m.topk;
    if (gemm_tc_launch(x, ldx, m.gate_w, d, nullptr, 0, w.logits, m.E, R, m.E, d, st)) return -1;
    k_moe_route_rows<<<(R + MOE_MAX_R - 1) / MOE_MAX_R, 256, 0, st>>>(m, w, R, w.logits);
    k_moe_lists<<<1, 1024, (size_t)R * K * sizeof(int), st>>>(w, R, K, m.E, m.e0, m.eloc, m.eloc);
    k_moe_gather<<<w.pmax * 8, 128, 0, st>>>(x, ldx, w, d);
    if (cudaGetLastError() != cudaSuccess) return -1;
    GemvDesc gu{};
    gu.W = m.gu_codes; gu.WS = m.gu_scales; gu.nkb = (d + 127) / 128;
    gu.x = w.xg; gu.ldx = d; gu.R = 8; gu.O = 2L * m.inter; gu.K = d; gu.fp8 = 1;
    gu.y = w.gu; gu.ldy = 2L * m.inter;
    gu.gexpert = w.prob_expert; gu.gcount = w.prob_count; gu.gmax = w.pmax; gu.gnum = m.eloc + 1;
    gu.w_estride = 2L * m.inter * d;
    gu.s_estride = (2L * m.inter / 128) * ((d + 127) / 128);
    gu.x_pstride = 8L * d;
    gu.y_pstride = 8L * 2 * m.inter;
    if (gemv_launch(gu, st)) return -1;
    GemvDesc dn{};
    dn.W = m.d_codes; dn.WS = m.d_scales; dn.nkb = (m.inter + 127) / 128;
    dn.x = w.gu; dn.ldx = 2L * m.inter; dn.R = 8; dn.O = d; dn.K = m.inter; dn.fp8 = 1;
    dn.y = w.yd; dn.ldy = d;
    dn.gexpert = w.prob_expert; dn.gcount = w.prob_count; dn.gmax = w.pmax; dn.gnum = m.eloc + 1;
    dn.w_estride = (long)d * m.inter;
    dn.s_estride = ((d + 127) / 128) * ((m.inter + 127) / 128);
    dn.x_pstride = 8L * 2 * m.inter;
    dn.y_pstride = 8L * d;
    dn.x_swiglu = 1;
    dn.swiglu_limit = m.limit;
    if (gemv_launch(dn, st)) return -1;
    const long n = (long)R * (d / 8);
    if (ep) {
        const long ns = (long)R * K * (d / 8);
        k_moe_scatter_rows<<<(unsigned)((ns + 127) / 128), 128, 0, st>>>(w, m.ep, R, K, d);
        k_ep_barrier<<<1, 1, 0, st>>>(m.ep);
        k_moe_combine_ep_rows<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(w, m.ep, R, K, d, m.eloc, out, ldo);
        return cudaGetLastError() == cudaSuccess ? 0 : -1;
    }
    k_moe_combine_rows<<<(unsigned)((n + 127) / 128), 128, 0, st>>>(w, R, K, d, out, ldo);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
