// layers.cu — per-layer kernels of the glm5_next decode stack on the B200.
//
// Each kernel restates one reference function; rounding points and, where it
// is cheap, summation orders are kept (numpy pairwise sums for norms, strictly
// sequential accumulations where the reference is sequential).  Everything is
// per token row, so a batch of R rows gives every row bitwise the result it
// gets alone (the verify == sequential decode property); the KDA recurrence
// and the DSA caches are stepped in row order.
#include "common.cuh"
#include "gcuda.h"
#include "model_dev.h"
#include "pipe.cuh"
#include "linear.cuh"
#include <cooperative_groups.h>

namespace apus {

// ---------------------------------------------------------------- helpers

// numpy pairwise sum of a[0..n) held in shared memory by the whole block
// (thread 0 walks the recursion; fine for the short vectors used here).
APUS_DEV float pw_sum_shared(const float *a, int n) {
    // recursion with an explicit stack, leaves via pw_sum_leaf
    struct Fr { int off, len, state; float left; };
    Fr st[24];
    int sp = 0;
    st[sp++] = {0, n, 0, 0.f};
    float ret = 0.f;
    while (sp) {
        Fr &f = st[sp - 1];
        if (f.len <= 128) { ret = f.len ? pw_sum_leaf(a + f.off, f.len) : 0.f; sp--; continue; }
        const int n2 = (f.len / 2) & ~7;
        if (f.state == 0) { f.state = 1; st[sp++] = {f.off, n2, 0, 0.f}; continue; }
        if (f.state == 1) { f.left = ret; f.state = 2; st[sp++] = {f.off + n2, f.len - n2, 0, 0.f}; continue; }
        ret = f.left + ret;
        sp--;
    }
    return ret;
}

// Levels of the numpy recursion when it is a perfect binary tree (every
// halving of a length > 128 is a multiple of 8: 16384, 4096, 1536, 512, ...),
// else -1.  Then the leaves are the 2^k equal runs of n >> k elements.
APUS_DEV int pw_perfect_levels(int n) {
    int k = 0;
    while ((n >> k) > 128) {
        if ((n >> k) & 15) return -1;
        k++;
    }
    return k;
}

// Block-parallel numpy pairwise sum, bitwise equal to pw_sum_shared.  A
// perfect tree: leaves by separate threads, then the pairs of each level
// combined left + right in parallel.  Otherwise the leaf table and the
// combine walk run on thread 0.
APUS_DEV float block_pw(const float *a, int n, float *leaf_buf, float *out_sh) {
    const int lv = pw_perfect_levels(n);
    if (lv >= 0 && lv <= 8) {
        const int nl = 1 << lv, L = n >> lv;
        if (L % 8 == 0 && (blockDim.x & 31) == 0) {
            // 8 lanes per leaf: lane k runs the leaf's k-th accumulator
            // (a[k], a[8+k], ... in order), then the fixed combine
            // ((r0+r1)+(r2+r3))+((r4+r5)+(r6+r7)) by shuffles (fp32 addition
            // is commutative, so a lane pair adds to the same bits either way)
            const int k = threadIdx.x & 7;
            for (int g0 = 0; g0 < nl; g0 += blockDim.x / 8) {
                const int g = g0 + (int)threadIdx.x / 8;
                float r = 0.f;
                if (g < nl) {
                    const float *lf = a + (size_t)g * L;
                    r = lf[k];
                    for (int i = 8; i < L; i += 8) r += lf[i + k];
                }
                r += __shfl_xor_sync(0xffffffffu, r, 1);
                r += __shfl_xor_sync(0xffffffffu, r, 2);
                r += __shfl_xor_sync(0xffffffffu, r, 4);
                if (g < nl && k == 0) leaf_buf[g] = r;
            }
        } else {
            for (int i = threadIdx.x; i < nl; i += blockDim.x) leaf_buf[i] = pw_sum_leaf(a + (size_t)i * L, L);
        }
        __syncthreads();
        for (int s = 1; s < nl; s <<= 1) {
            for (int q = threadIdx.x; q < nl / (2 * s); q += blockDim.x) {
                const int i = 2 * s * q;
                leaf_buf[i] = leaf_buf[i] + leaf_buf[i + s];
            }
            __syncthreads();
        }
        const float r = leaf_buf[0];
        __syncthreads();
        return r;
    }
    // leaf k covers the k-th <=128 piece in left-to-right order of the recursion
    __shared__ int leaf_off[256], leaf_len[256], nleaf;
    if (threadIdx.x == 0) {
        int so[24], sl[24], sp = 0, nl = 0;
        so[sp] = 0; sl[sp] = n; sp++;
        while (sp) {
            sp--;
            const int off = so[sp], len = sl[sp];
            if (len <= 128) { leaf_off[nl] = off; leaf_len[nl] = len; nl++; continue; }
            const int n2 = (len / 2) & ~7;
            so[sp] = off + n2; sl[sp] = len - n2; sp++;
            so[sp] = off; sl[sp] = n2; sp++;
        }
        nleaf = nl;
    }
    __syncthreads();
    for (int i = threadIdx.x; i < nleaf; i += blockDim.x)
        leaf_buf[i] = leaf_len[i] ? pw_sum_leaf(a + leaf_off[i], leaf_len[i]) : 0.f;
    __syncthreads();
    if (threadIdx.x == 0) {
        struct Fr { int len, state; float left; };
        Fr st[24];
        int sp = 0, cur = 0;
        st[sp++] = {n, 0, 0.f};
        float ret = 0.f;
        while (sp) {
            Fr &f = st[sp - 1];
            if (f.len <= 128) { ret = leaf_buf[cur++]; sp--; continue; }
            const int n2 = (f.len / 2) & ~7;
            if (f.state == 0) { f.state = 1; st[sp++] = {n2, 0, 0.f}; continue; }
            if (f.state == 1) { f.left = ret; f.state = 2; st[sp++] = {f.len - n2, 0, 0.f}; continue; }
            ret = f.left + ret;
            sp--;
        }
        *out_sh = ret;
    }
    __syncthreads();
    const float r = *out_sh;
    __syncthreads();
    return r;
}

// Weighted RMSNorm of one row held as fp32 in smem (c/gdsa.h:258-274):
// var = pairwise mean of squares; t = bf16(x * (1/sqrt(var+eps))); y = bf16(w*t).
APUS_DEV bool al16(const void *p) { return ((uintptr_t)p & 15) == 0; }

// Row x[0..n) (BF16) -> fp32 in shared memory; 16-byte loads when aligned,
// every load of a thread issued before any is used.
APUS_DEV void load_row_f32(const uint16_t *x, int n, float *xs) {
    if (n % 8 == 0 && al16(x)) {
        for (int c0 = threadIdx.x; c0 < n / 8; c0 += 4 * blockDim.x) {
            uint4 v[4];
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int c = c0 + u * blockDim.x;
                v[u] = c < n / 8 ? *(const uint4 *)(x + c * 8) : make_uint4(0, 0, 0, 0);
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const int c = c0 + u * blockDim.x;
                if (c >= n / 8) break;
                const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
                for (int e = 0; e < 4; e++) {
                    xs[c * 8 + 2 * e] = bf16lo(w[e]);
                    xs[c * 8 + 2 * e + 1] = bf16hi(w[e]);
                }
            }
        }
    } else {
#pragma unroll 4
        for (int i = threadIdx.x; i < n; i += blockDim.x) xs[i] = bf16_f32(x[i]);
    }
}

APUS_DEV void rmsnorm_row_smem(float *xs, float *sq, int n, const uint16_t *w, float eps, uint16_t *y,
                               float *leaf, float *res) {
    for (int i = threadIdx.x; i < n; i += blockDim.x) sq[i] = xs[i] * xs[i];
    __syncthreads();
    const float var = block_pw(sq, n, leaf, res) / (float)n;
    const float inv = 1.0f / sqrtf(var + eps);
    if (n % 8 == 0 && al16(w) && al16(y)) {
        for (int c = threadIdx.x; c < n / 8; c += blockDim.x) {
            const uint4 wv = *(const uint4 *)(w + c * 8);
            const uint32_t ww[4] = {wv.x, wv.y, wv.z, wv.w};
            uint32_t o[4];
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const float t0 = bf16_round(xs[c * 8 + 2 * e] * inv), t1 = bf16_round(xs[c * 8 + 2 * e + 1] * inv);
                o[e] = (uint32_t)bf16_bits(bf16lo(ww[e]) * t0) | ((uint32_t)bf16_bits(bf16hi(ww[e]) * t1) << 16);
            }
            *(uint4 *)(y + c * 8) = make_uint4(o[0], o[1], o[2], o[3]);
        }
    } else {
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const float t = bf16_round(xs[i] * inv);
            y[i] = bf16_bits(bf16_f32(w[i]) * t);
        }
    }
}

// ------------------------------------------------------------------ embed

__global__ void k_embed(const uint16_t *embed, const int32_t *ids, int d, int hc, uint16_t *h4) {
    pdl_launch_dependents();
    const int r = blockIdx.y;
    const uint16_t *row = embed + (size_t)ids[r] * d;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < d; i += gridDim.x * blockDim.x) {
        const uint16_t v = row[i];
        for (int j = 0; j < hc; j++) h4[((size_t)r * hc + j) * d + i] = v;
    }
}

// --------------------------------------------------------------------- mHC

// Gates + Sinkhorn of one row from its mixes m[(2+hc)*hc] (c/gmhc.h:197-265):
// pre, post and comb into shared arrays and post/comb into the row's outputs.
// One warp when hc*hc <= 32 (lane (j,k) owns comb[j][k]), else thread 0.
APUS_DEV void hc_maps(const float *m, const float *scale, const float *base, int hc, int iters, float hc_eps,
                      int r, float *pre, float *post, float *comb, float *post_out, float *comb_out) {
    if (hc * hc <= 32 && threadIdx.x < 32) {
        // one warp: lane (j, k) = (lane / hc, lane % hc) owns comb[j][k]; every
        // sum runs in the reference's sequential order (hc < 8) via shuffles
        const int lane = threadIdx.x, j = lane / hc, k = lane % hc;
        const bool act = lane < hc * hc;
        if (lane < hc) {
            pre[lane] = sigmoid_np(m[lane] * scale[0] + base[lane]) + hc_eps;
            post[lane] = 2.0f * sigmoid_np(m[hc + lane] * scale[1] + base[hc + lane]);
        }
        float c = act ? m[2 * hc + lane] * scale[2] + base[2 * hc + lane] : 0.f;
        const int rb = act ? j * hc : 0, cb = act ? k : 0;
        float mx = __shfl_sync(0xffffffffu, c, rb);
        for (int q = 1; q < hc; q++) {
            const float v = __shfl_sync(0xffffffffu, c, rb + q);
            if (v > mx) mx = v;
        }
        c = expf(c - mx);
        float sum = __shfl_sync(0xffffffffu, c, rb);
        for (int q = 1; q < hc; q++) sum += __shfl_sync(0xffffffffu, c, rb + q);
        c = c / sum + hc_eps;
        for (int it = 0; it < iters; it++) {
            if (it) {
                float den = __shfl_sync(0xffffffffu, c, rb);
                for (int q = 1; q < hc; q++) den += __shfl_sync(0xffffffffu, c, rb + q);
                c /= den + hc_eps;
            }
            float cs = __shfl_sync(0xffffffffu, c, cb);
            for (int q = 1; q < hc; q++) cs += __shfl_sync(0xffffffffu, c, q * hc + cb);
            c /= cs + hc_eps;
        }
        if (act) {
            comb[lane] = c;
            comb_out[r * hc * hc + lane] = c;
        }
        __syncwarp();
        if (lane < hc) post_out[r * hc + lane] = post[lane];
    } else if (hc * hc > 32 && threadIdx.x == 0) {
        for (int j = 0; j < hc; j++) pre[j] = sigmoid_np(m[j] * scale[0] + base[j]) + hc_eps;
        for (int j = 0; j < hc; j++) post[j] = 2.0f * sigmoid_np(m[hc + j] * scale[1] + base[hc + j]);
        for (int j = 0; j < hc; j++)
            for (int k = 0; k < hc; k++) {
                const int idx = 2 * hc + j * hc + k;
                comb[j * hc + k] = m[idx] * scale[2] + base[idx];
            }
        for (int j = 0; j < hc; j++) {      // row softmax + eps
            float *rr = comb + j * hc, mx = rr[0];
            for (int k = 1; k < hc; k++) if (rr[k] > mx) mx = rr[k];
            for (int k = 0; k < hc; k++) rr[k] = expf(rr[k] - mx);
            const float sum = pw_sum_leaf(rr, hc);
            for (int k = 0; k < hc; k++) rr[k] = rr[k] / sum + hc_eps;
        }
        for (int it = 0; it < iters; it++) {
            if (it)
                for (int j = 0; j < hc; j++) {
                    float *rr = comb + j * hc;
                    const float den = pw_sum_leaf(rr, hc) + hc_eps;
                    for (int k = 0; k < hc; k++) rr[k] /= den;
                }
            for (int k = 0; k < hc; k++) {
                float sum = comb[k];
                for (int j = 1; j < hc; j++) sum += comb[j * hc + k];
                const float den = sum + hc_eps;
                for (int j = 0; j < hc; j++) comb[j * hc + k] /= den;
            }
        }
        for (int j = 0; j < hc; j++) post_out[r * hc + j] = post[j];
        for (int j = 0; j < hc * hc; j++) comb_out[r * hc * hc + j] = comb[j];
    }
}

// mHC (c/gmhc.h:187-294) in two launches per sublayer boundary:
//   k_hc_postmix  CTA per 64-column chunk, all rows: the expand of the
//                 sublayer just finished (its output combined on the fly when
//                 it is the MoE), then the next site's pre-mix partials over
//                 the chunk: sum_i fn[m][i] h[i] and sum_i h[i]^2, in a fixed
//                 order (lane-sequential, then a fixed warp tree);
//   k_hc_pre      CTAs 0..R-1: mixes = inverse RMS * (chunk-ordered sums),
//                 pre gates, the collapse bf16(sum_j pre_j h_j) and the layer
//                 RMSNorm; CTAs R..2R-1: the same mixes, then post gates and
//                 the Sinkhorn comb (needed only by the next expand), so the
//                 Sinkhorn runs beside the collapse instead of before it.
// The inverse RMS multiplies the summed dot products (the reference scales
// the streams first, c/gmhc.h:241-251): equal up to fp32 rounding.
#define HC_PM_CW 64
// A grid with gridDim.y > 1 covers more rows, MAXR per y (the sublayer
// output given as x rows): block y takes rows MAXR*y ...
__global__ void __launch_bounds__(256) k_hc_postmix(HcPostMix a) {
    pdl_launch_dependents();
    if (blockIdx.y) {
        const size_t r0 = (size_t)blockIdx.y * MAXR;
        if (a.x) a.x += r0 * a.d;
        a.h4 += r0 * a.hc * a.d;
        a.post += r0 * a.hc;
        a.comb += r0 * a.hc * a.hc;
        if (a.h4out) a.h4out += r0 * a.hc * a.d;
        a.part += r0 * a.nchunk * (a.nmix + 1);
        a.R -= (int)r0;
    }
    if (a.R > MAXR) a.R = MAXR;
    __shared__ float xs[MAXR][HC_PM_CW];
    __shared__ float hs[MAXR][8][HC_PM_CW];
    const int c = blockIdx.x, i0 = c * HC_PM_CW, d = a.d, hc = a.hc, R = a.R;
    const int cw = min(HC_PM_CW, d - i0);
    const bool expand = a.h4out != nullptr;
    if (expand) {
        for (int q = threadIdx.x; q < R * HC_PM_CW; q += blockDim.x) {
            const int r = q / HC_PM_CW, ii = q % HC_PM_CW;
            if (ii >= cw) continue;
            const int i = i0 + ii;
            float v;
            if (a.x) {
                v = bf16_f32(a.x[(size_t)r * d + i]);
            } else {   // MoE output (c/gmoe.h:226-236): ascending experts, shared expert last
                const MoeDev &m = a.moe;
                const int K = m.topk;
                const size_t ps = (size_t)m.max_r * d, off = (size_t)r * d + i;
                // every load issued before the ordered sum uses any of them
                int pj[MOE_MAX_TOPK];
                float wj[MOE_MAX_TOPK];
#pragma unroll
                for (int j = 0; j < MOE_MAX_TOPK; j++)
                    if (j < K) { pj[j] = m.row_prob[r * K + j]; wj[j] = m.row_weight[r * K + j]; }
                uint16_t ev[MOE_MAX_TOPK];
#pragma unroll
                for (int j = 0; j < MOE_MAX_TOPK; j++)
                    if (j < K) ev[j] = m.yd[(size_t)pj[j] * ps + off];
                const uint16_t shv = m.yd[(size_t)m.row_prob_shared[r] * ps + off];
                float y = 0.f;
#pragma unroll
                for (int j = 0; j < MOE_MAX_TOPK; j++)
                    if (j < K) y = bf16_round(y + bf16_round(bf16_f32(ev[j]) * wj[j]));
                v = K ? bf16_round(y + bf16_f32(shv)) : bf16_f32(shv);
            }
            xs[r][ii] = v;
        }
        __syncthreads();
    }
    // expand (c/gmhc.h:278-294): y[j][i] = bf16(bf16(bf16(post[j]) x[i]) +
    // bf16(sum_k bf16(comb[k][j]) h[k][i])), or the input streams as they
    // are; four elements per thread with all their loads issued first
    const int tot = R * hc * HC_PM_CW;
    for (int q0 = threadIdx.x; q0 < tot; q0 += 4 * blockDim.x) {
        uint16_t hk[4][8];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int q = q0 + u * blockDim.x;
            const int r = q / (hc * HC_PM_CW), j = (q / HC_PM_CW) % hc, ii = q % HC_PM_CW;
            if (q >= tot || ii >= cw) continue;
            const uint16_t *hr = a.h4 + (size_t)r * hc * d + i0 + ii;
            if (expand) {
#pragma unroll
                for (int k = 0; k < 8; k++)
                    if (k < hc) hk[u][k] = hr[(size_t)k * d];
            } else {
                hk[u][0] = hr[(size_t)j * d];
            }
        }
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int q = q0 + u * blockDim.x;
            const int r = q / (hc * HC_PM_CW), j = (q / HC_PM_CW) % hc, ii = q % HC_PM_CW;
            if (q >= tot || ii >= cw) continue;
            float o;
            if (expand) {
                const float pb = bf16_round(a.post[r * hc + j]);
                const float t1 = bf16_round(pb * xs[r][ii]);
                float acc = 0.f;
#pragma unroll
                for (int k = 0; k < 8; k++)
                    if (k < hc) acc += bf16_round(a.comb[(r * hc + k) * hc + j]) * bf16_f32(hk[u][k]);
                const uint16_t ob = bf16_bits(t1 + bf16_round(acc));
                a.h4out[((size_t)r * hc + j) * d + i0 + ii] = ob;
                o = bf16_f32(ob);
            } else {
                o = bf16_f32(hk[u][0]);
            }
            hs[r][j][ii] = o;
        }
    }
    if (!a.fn) return;
    __syncthreads();
    // partials: warp w takes m = w, w+8, w+16, w+24 (m == nmix: the sum of
    // squares; nmix <= 31); lane l covers elements 8l.. of every 256-element
    // group of the chunk, its weight loads issued first
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31, E = hc * cw;
    float accr[4][MAXR];
#pragma unroll
    for (int u = 0; u < 4; u++)
#pragma unroll
        for (int r = 0; r < MAXR; r++) accr[u][r] = 0.f;
    for (int e0 = lane * 8; e0 < E; e0 += 256) {
        const int j = e0 / cw, ii = e0 % cw;
        uint4 fv[4];
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int m = warp + 8 * u;
            if (m < a.nmix) fv[u] = __ldg((const uint4 *)(a.fn + (size_t)m * hc * d + (size_t)j * d + i0 + ii));
        }
        float hv[MAXR][8];
#pragma unroll
        for (int r = 0; r < MAXR; r++)
#pragma unroll
            for (int e = 0; e < 8; e++) hv[r][e] = r < R ? hs[r][j][ii + e] : 0.f;
#pragma unroll
        for (int u = 0; u < 4; u++) {
            const int m = warp + 8 * u;
            if (m > a.nmix) break;
            const uint32_t fw[4] = {fv[u].x, fv[u].y, fv[u].z, fv[u].w};
#pragma unroll
            for (int r = 0; r < MAXR; r++) {
                if (r >= R) break;
#pragma unroll
                for (int e = 0; e < 8; e++) {
                    const float f = m < a.nmix ? ((e & 1) ? bf16hi(fw[e >> 1]) : bf16lo(fw[e >> 1])) : hv[r][e];
                    accr[u][r] += f * hv[r][e];
                }
            }
        }
    }
#pragma unroll
    for (int u = 0; u < 4; u++) {
        const int m = warp + 8 * u;
        if (m > a.nmix) break;
#pragma unroll
        for (int r = 0; r < MAXR; r++) {
            if (r >= R) break;
            float v = accr[u][r];
#pragma unroll
            for (int off = 16; off; off >>= 1) v += __shfl_xor_sync(0xffffffffu, v, off);
            if (lane == 0) a.part[((size_t)r * a.nchunk + c) * (a.nmix + 1) + m] = v;
        }
    }
}

__global__ void __launch_bounds__(512) k_hc_pre(const uint16_t *h4, const float *part, int nchunk,
                                                const float *scale, const float *base, const uint16_t *norm_w, int d,
                                                int hc, int iters, float hc_eps, float eps, int R, float *post_out,
                                                float *comb_out, uint16_t *x_out) {
    pdl_launch_dependents();
    extern __shared__ float ys[];                     // [d] collapsed row + [d] squares
    float *sq = ys + d;
    __shared__ float mixs[81], pre[8], post[8], comb[64], leaf[256], res;
    const bool maps = (int)blockIdx.x >= R;
    const int r = maps ? blockIdx.x - R : blockIdx.x, nmix = (2 + hc) * hc;
    const uint16_t *x = h4 + (size_t)r * hc * d;
    if ((int)threadIdx.x <= nmix) {
        // chunk-ordered sums of the partials, loads issued 16 at a time
        const float *pp = part + (size_t)r * nchunk * (nmix + 1) + threadIdx.x;
        float v = 0.f;
        for (int c0 = 0; c0 < nchunk; c0 += 16) {
            float t[16];
#pragma unroll
            for (int u = 0; u < 16; u++) t[u] = c0 + u < nchunk ? pp[(size_t)(c0 + u) * (nmix + 1)] : 0.f;
#pragma unroll
            for (int u = 0; u < 16; u++)
                if (c0 + u < nchunk) v = (c0 + u == 0) ? t[u] : v + t[u];
        }
        mixs[threadIdx.x] = v;
    }
    __syncthreads();
    if ((int)threadIdx.x < nmix) {
        const float inv = 1.0f / sqrtf(mixs[nmix] / (float)(hc * d) + eps);
        mixs[threadIdx.x] *= inv;
    }
    __syncthreads();
    if (maps) {     // post gates + Sinkhorn comb for the next expand
        hc_maps(mixs, scale, base, hc, iters, hc_eps, r, pre, post, comb, post_out, comb_out);
        return;
    }
    if ((int)threadIdx.x < hc)
        pre[threadIdx.x] = sigmoid_np(mixs[threadIdx.x] * scale[0] + base[threadIdx.x]) + hc_eps;
    __syncthreads();
    // collapse (c/gmhc.h:267-276): 8 consecutive columns per thread, the hc
    // stream loads issued together
    for (int c = threadIdx.x; c < d / 8; c += blockDim.x) {
        uint4 v[8];
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (j < hc) v[j] = *(const uint4 *)(x + (size_t)j * d + c * 8);
#pragma unroll
        for (int e = 0; e < 8; e++) {
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (j >= hc) break;
                const uint32_t word = (e >> 1) == 0 ? v[j].x : (e >> 1) == 1 ? v[j].y : (e >> 1) == 2 ? v[j].z : v[j].w;
                const float xe = (e & 1) ? bf16hi(word) : bf16lo(word);
                acc = j == 0 ? pre[0] * xe : acc + pre[j] * xe;
            }
            ys[c * 8 + e] = bf16_round(acc);
        }
    }
    __syncthreads();
    rmsnorm_row_smem(ys, sq, d, norm_w, eps, x_out + (size_t)r * d, leaf, &res);
}

// HyperHead mean (c/gmhc.h:296-304) + final RMSNorm
__global__ void k_head_norm(const uint16_t *h4, const uint16_t *w, int d, int hc, float eps, uint16_t *yn,
                            unsigned long long *keys) {
    pdl_launch_dependents();
    if (keys && threadIdx.x == 0) keys[blockIdx.x] = 0ull;
    extern __shared__ float ys[];
    float *sq = ys + d;
    __shared__ float leaf[256], res;
    const int r = blockIdx.x;
    const uint16_t *x4 = h4 + (size_t)r * hc * d;
    for (int c = threadIdx.x; c < d / 8; c += blockDim.x) {
        uint4 v[8];
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (j < hc) v[j] = *(const uint4 *)(x4 + (size_t)j * d + c * 8);
#pragma unroll
        for (int e = 0; e < 8; e++) {
            float acc = 0.f;
#pragma unroll
            for (int j = 0; j < 8; j++) {
                if (j >= hc) break;
                const uint32_t word = (e >> 1) == 0 ? v[j].x : (e >> 1) == 1 ? v[j].y : (e >> 1) == 2 ? v[j].z : v[j].w;
                const float xe = (e & 1) ? bf16hi(word) : bf16lo(word);
                acc = j == 0 ? xe : acc + xe;
            }
            ys[c * 8 + e] = bf16_round(acc / (float)hc);
        }
    }
    __syncthreads();
    rmsnorm_row_smem(ys, sq, d, w, eps, yn + (size_t)r * d, leaf, &res);
}

__global__ void k_rmsnorm_rows(const uint16_t *x, long ldx, const uint16_t *w, int n, float eps, uint16_t *y,
                               long ldy) {
    pdl_launch_dependents();
    extern __shared__ float ys[];
    float *sq = ys + n;
    __shared__ float leaf[256], res;
    const int r = blockIdx.x;
    load_row_f32(x + (size_t)r * ldx, n, ys);
    __syncthreads();
    rmsnorm_row_smem(ys, sq, n, w, eps, y + (size_t)r * ldy, leaf, &res);
}

struct NormSegs { NormSeg s[2]; };

__global__ void k_norm_seg(NormSegs sg, float eps, unsigned long long *keys) {
    pdl_launch_dependents();
    extern __shared__ float ys[];
    __shared__ float leaf[256], res;
    const NormSeg &g = sg.s[blockIdx.y];
    const int r = blockIdx.x, n = g.n;
    float *sq = ys + n;
    if (keys && blockIdx.y == 0 && threadIdx.x == 0) keys[r] = 0ull;
    uint16_t *xr = (uint16_t *)g.x + (size_t)(g.gather ? g.gather[r] : r) * g.ldx;
    load_row_f32(xr, n, ys);
    if (g.sub) {
        load_row_f32(g.sub + (size_t)r * g.ldsub, n, sq);
        __syncthreads();
        for (int i = threadIdx.x; i < n; i += blockDim.x) {
            const float v = bf16_round(ys[i] + sq[i]);
            ys[i] = v;
            xr[i] = bf16_bits(v);
        }
    }
    __syncthreads();
    rmsnorm_row_smem(ys, sq, n, g.w, eps, g.y + (size_t)r * g.ldy, leaf, &res);
}

__global__ void k_residual_add(uint16_t *x, const uint16_t *sub, long n) {
    pdl_launch_dependents();
    for (long i = blockIdx.x * (long)blockDim.x + threadIdx.x; i < n; i += (long)gridDim.x * blockDim.x)
        x[i] = bf16_bits(bf16_f32(x[i]) + bf16_f32(sub[i]));
}

// --------------------------------------------------------------------- KDA

// depthwise causal conv k=K + SiLU over the q|k|v channels, tokens chained
// (c/gkda.h:227-257).  The conv state after token t goes to checkpoint slot
// (cur+1+t) % NSLOT; the committed slot is never written.
__global__ void k_kda_conv(const uint16_t *kp, long ldkp, const uint16_t *conv_w, uint16_t *conv_slots,
                           const Ctl *ctl, int R, int C, int K, uint16_t *out) {
    pdl_launch_dependents();
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    const int cur = ctl->kda_cur;
    const size_t slot = (size_t)C * (K - 1);
    // every load first: weights, the committed state and each row's input
    uint16_t st[8], wc[9], xs[MAXR];
#pragma unroll
    for (int j = 0; j < 9; j++)
        if (j < K) wc[j] = conv_w[(size_t)c * K + j];
#pragma unroll
    for (int j = 0; j < 8; j++)
        if (j < K - 1) st[j] = conv_slots[cur * slot + (size_t)c * (K - 1) + j];
#pragma unroll
    for (int t = 0; t < MAXR; t++)
        if (t < R) xs[t] = kp[(size_t)t * ldkp + c];
#pragma unroll
    for (int t = 0; t < MAXR; t++) {
        if (t >= R) break;
        const uint16_t xc = xs[t];
        float acc = 0.f;
#pragma unroll
        for (int i = 0; i < 8; i++)
            if (i < K - 1) acc += bf16_f32(wc[i]) * bf16_f32(st[i]);
        acc += bf16_f32(wc[K - 1]) * bf16_f32(xc);
        out[(size_t)t * C + c] = bf16_bits(acc * sigmoid_np(acc));
#pragma unroll
        for (int j = 0; j < 7; j++)
            if (j + 1 < K - 1) st[j] = st[j + 1];
        st[K - 2] = xc;
        const int s = (cur + 1 + t) % NSLOT;
#pragma unroll
        for (int j = 0; j < 8; j++)
            if (j < K - 1) conv_slots[s * slot + (size_t)c * (K - 1) + j] = st[j];
    }
}

// The delta-rule recurrence of one head over R chained tokens
// (c/gkda.h:279-346) fused with the forget gate (:629-643), beta (:644-647)
// and the gated o_norm (:543-569).  128 threads; thread j owns column j of the
// fp32 state S[i][j] (128 registers), so kv[j] = sum_i S[i][j] k[i] and
// o[j] = sum_i S[i][j] q[i] run in the reference's sequential i order.
template <int D>
__global__ void __launch_bounds__(D) k_kda_rec(const uint16_t *qkvc, const uint16_t *kp, long ldkp, int beta_off,
                                               const uint16_t *fgo, long fg_pstride, const float *A_log,
                                               const float *dt_bias, const uint16_t *o_norm, float *rec_slots,
                                               const Ctl *ctl, int R, int H, float lower_bound, float eps,
                                               float qscale, uint16_t *core_out) {
    pdl_launch_dependents();
    const int h = blockIdx.x, j = threadIdx.x, qkv = H * D;
    __shared__ float qf[D], kf[D], dec[D], sq[D], red[2], beta_sh[MAXR];
    // every row's inputs of this thread's element j ([row][j]: q, k, v, forget
    // and output gates), loaded before the token chain so that the chain
    // waits on one memory round trip rather than several per token
    __shared__ uint16_t in_sh[5][MAXR][D];
    {
        uint16_t r5[5][MAXR];
#pragma unroll
        for (int t = 0; t < MAXR; t++)
            if (t < R) {
                const uint16_t *q = qkvc + (size_t)t * 3 * qkv + (size_t)h * D;
                r5[0][t] = q[j];
                r5[1][t] = q[qkv + j];
                r5[2][t] = q[2 * qkv + j];
                r5[3][t] = fgo[(size_t)t * qkv + (size_t)h * D + j];
                r5[4][t] = fgo[fg_pstride + (size_t)t * qkv + (size_t)h * D + j];
            }
#pragma unroll
        for (int t = 0; t < MAXR; t++)
            if (t < R)
#pragma unroll
                for (int c = 0; c < 5; c++) in_sh[c][t][j] = r5[c][t];
    }
    if (j < R) beta_sh[j] = bf16_round(sigmoid_np(bf16_f32(kp[(size_t)j * ldkp + beta_off + h])));
    const float dtb = dt_bias[(size_t)h * D + j], onw = bf16_f32(o_norm[j]);
    float S[D];
    const int cur = ctl->kda_cur;
    const size_t hs = (size_t)D * D;
    const float *S0 = rec_slots + (size_t)cur * H * hs + (size_t)h * hs;
#pragma unroll
    for (int i = 0; i < D; i++) S[i] = S0[(size_t)i * D + j];
    const float a = expf(A_log[h]);
    for (int t = 0; t < R; t++) {
        // l2norm q, k (c/gkda.h:263-273), pairwise sums of squares
        const float qv = bf16_f32(in_sh[0][t][j]), kv_ = bf16_f32(in_sh[1][t][j]), vj = bf16_f32(in_sh[2][t][j]);
        const float fz = bf16_f32(in_sh[3][t][j]), gz = bf16_f32(in_sh[4][t][j]);
        sq[j] = qv * qv;
        __syncthreads();
        if (j == 0) red[0] = sqrtf(pw_sum_leaf(sq, D) + 1e-6f);
        __syncthreads();
        sq[j] = kv_ * kv_;
        __syncthreads();
        if (j == 0) red[1] = sqrtf(pw_sum_leaf(sq, D) + 1e-6f);
        __syncthreads();
        qf[j] = (qv / red[0]) * qscale;
        kf[j] = kv_ / red[1];
        // forget gate: g = lb * sigmoid(exp(A_log) * (fg + dt_bias)); decay exp(g)
        const float z = fz + dtb;
        dec[j] = expf(lower_bound * sigmoid_np(a * z));
        const float beta = beta_sh[t];
        __syncthreads();
#pragma unroll
        for (int i = 0; i < D; i++) S[i] = S[i] * dec[i];
        float kvm = 0.f;
#pragma unroll
        for (int i = 0; i < D; i++) kvm += S[i] * kf[i];
        const float dl = (vj - kvm) * beta;
#pragma unroll
        for (int i = 0; i < D; i++) S[i] = S[i] + kf[i] * dl;
        float o = 0.f;
#pragma unroll
        for (int i = 0; i < D; i++) o += S[i] * qf[i];
        const float core = bf16_round(o);
        // checkpoint the state after this token
        float *Sd = rec_slots + (size_t)((cur + 1 + t) % NSLOT) * H * hs + (size_t)h * hs;
#pragma unroll
        for (int i = 0; i < D; i++) Sd[(size_t)i * D + j] = S[i];
        // gated o_norm, eps = rms_norm_eps
        __syncthreads();
        sq[j] = core * core;
        __syncthreads();
        if (j == 0) red[0] = 1.0f / sqrtf(pw_sum_leaf(sq, D) / (float)D + eps);
        __syncthreads();
        float y = core * red[0];
        y = onw * y;
        y = y * sigmoid_np(gz);
        core_out[(size_t)t * qkv + (size_t)h * D + j] = bf16_bits(y);
        __syncthreads();
    }
}

// --------------------------------------------------------------------- DSA

// Append this call's rows to the caches at base+t (c/gdsa.h:612-626 for K/V,
// :329-334 for the indexer key LayerNorm and compress gate).  Grid (R, AH):
// block (t, h) copies head h's K and V rows with 16-byte moves; block (t, 0)
// also writes the indexer rows.
__global__ void k_dsa_append(const uint16_t *kvb, const uint16_t *ikgw, const uint16_t *knw, const uint16_t *knb,
                             const int *base_n, int AH, int qd, int vd, int ID, int IH, int cap, DsaState ds) {
    pdl_launch_dependents();
    const int t = blockIdx.x, h = blockIdx.y;
    const int pos = *base_n + t;
    if (pos >= cap) return;
    const uint16_t *row = kvb + (size_t)t * AH * (qd + vd) + (size_t)h * (qd + vd);
    uint16_t *kd = ds.k + ((size_t)h * cap + pos) * qd, *vdst = ds.v + ((size_t)h * cap + pos) * vd;
    for (int i = threadIdx.x; i < (qd + vd) / 8; i += blockDim.x) {
        const uint4 v = *(const uint4 *)(row + i * 8);
        if (i < qd / 8) *(uint4 *)(kd + i * 8) = v;
        else *(uint4 *)(vdst + (i * 8 - qd)) = v;
    }
    if (h != 0) return;
    // LayerNorm of the indexer key (c/gdsa.h:276-305, eps 1e-6)
    __shared__ float xs[256], d2[256], leaf[256], res;
    const uint16_t *ir = ikgw + (size_t)t * (2 * ID + IH);
    for (int i = threadIdx.x; i < ID; i += blockDim.x) xs[i] = bf16_f32(ir[i]);
    __syncthreads();
    const float mu = block_pw(xs, ID, leaf, &res) / (float)ID;
    for (int i = threadIdx.x; i < ID; i += blockDim.x) { const float dd = xs[i] - mu; d2[i] = dd * dd; }
    __syncthreads();
    const float var = block_pw(d2, ID, leaf, &res) / (float)ID;
    const float inv = 1.0f / sqrtf(var + 1e-6f);
    for (int i = threadIdx.x; i < ID; i += blockDim.x) {
        float v = (xs[i] - mu) * inv;
        v = v * bf16_f32(knw[i]) + bf16_f32(knb[i]);
        ds.ik[(size_t)pos * ID + i] = bf16_bits(v);
        ds.ig[(size_t)pos * ID + i] = ir[ID + i];
    }
}

// Pool keys of the pools completed by this call (c/gdsa.h:344-372): the
// softmax(gate + ape) over the kpool members, probs cast to BF16, weighted
// average rounded to BF16.  A completed pool never changes, so it is
// computed once when its last member is appended.
__global__ void k_dsa_pool(const uint16_t *ape, const int *base_n, int R, int ID, int kp, int cap, DsaState ds) {
    pdl_launch_dependents();
    const int base = *base_n;
    const int t = blockIdx.x, pos = base + t;
    if (pos >= cap || (pos % kp) != kp - 1) return;
    const int p = pos / kp;
    for (int dd = threadIdx.x; dd < ID; dd += blockDim.x) {
        float lg[16], e[16];
        for (int c = 0; c < kp; c++)
            lg[c] = bf16_f32(ds.ig[(size_t)(p * kp + c) * ID + dd]) + bf16_f32(ape[c * ID + dd]);
        float mx = lg[0];
        for (int c = 1; c < kp; c++) if (lg[c] > mx) mx = lg[c];
        float sum = 0.f;
        for (int c = 0; c < kp; c++) { e[c] = expf(lg[c] - mx); sum += e[c]; }
        float acc = 0.f;
        for (int c = 0; c < kp; c++) acc += bf16_round(e[c] / sum) * bf16_f32(ds.ik[(size_t)(p * kp + c) * ID + dd]);
        ds.pkey[(size_t)p * ID + dd] = bf16_bits(acc);
    }
}

// Indexer scores (c/gdsa.h:376-403) for every pool visible to row t:
// sc = sum_h w_h * relu((idx_q[h] . key[p]) * ID^-0.5), w_h = bf16(wproj x) * IH^-0.5.
// 256 threads = 8 pools x 32 heads: thread (pool, h) runs the reference's
// sequential ID-long dot, then one thread per pool sums the heads in order.
// Grid (ceil(maxpools / 8), R); blocks past the visible pools exit.
__global__ void __launch_bounds__(256) k_dsa_score(const uint16_t *iq, const uint16_t *ikgw, const int *base_n,
                                                   int IH, int ID, int kp, int maxpools, DsaState ds, float *score) {
    pdl_launch_dependents();
    const int t = blockIdx.y;
    const int qpos = *base_n + t;
    const int nvalid = min((qpos + 1) / kp, maxpools);
    const int p0 = blockIdx.x * 8;
    if (p0 >= nvalid) return;
    const float idx_scale = (float)(1.0 / sqrt((double)ID)), ih_scale = (float)(1.0 / sqrt((double)IH));
    __shared__ float qs[32 * 129];          // [h][ID] with a one-float pad per head
    __shared__ float wh[32], wsc[8][32];
    {   // stage the row's index queries: 16-byte loads, all issued first
        const uint16_t *src = iq + (size_t)t * IH * ID;
        const int nv = IH * ID / 8;                    // <= 512 = 2 per thread
        uint4 v[2];
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int c = threadIdx.x + u * blockDim.x;
            v[u] = c < nv ? *(const uint4 *)(src + c * 8) : make_uint4(0, 0, 0, 0);
        }
#pragma unroll
        for (int u = 0; u < 2; u++) {
            const int c = threadIdx.x + u * blockDim.x;
            if (c >= nv) break;
            const uint32_t w[4] = {v[u].x, v[u].y, v[u].z, v[u].w};
#pragma unroll
            for (int e = 0; e < 8; e++) {
                const int i = c * 8 + e;
                qs[(i / ID) * (ID + 1) + i % ID] = (e & 1) ? bf16hi(w[e >> 1]) : bf16lo(w[e >> 1]);
            }
        }
    }
    for (int h = threadIdx.x; h < IH; h += blockDim.x)
        wh[h] = bf16_f32(ikgw[(size_t)t * (2 * ID + IH) + 2 * ID + h]) * ih_scale;
    __syncthreads();
    const int pl = threadIdx.x >> 5, h = threadIdx.x & 31, p = p0 + pl;
    if (p < nvalid && h < IH) {
        const uint16_t *key = ds.pkey + (size_t)p * ID;
        const float *qh = qs + h * (ID + 1);
        float dot = 0.f;
        for (int i = 0; i < ID; i++) dot += qh[i] * bf16_f32(key[i]);
        const float v = dot * idx_scale;
        wsc[pl][h] = wh[h] * (v > 0.f ? v : 0.f);
    }
    __syncthreads();
    if (h == 0 && p < nvalid) {
        float acc = 0.f;
        for (int hh = 0; hh < IH; hh++) acc += wsc[pl][hh];
        score[(size_t)t * maxpools + p] = acc;
    }
}

// Order key of a pool score: larger score, larger key; -0 counts as +0
// (the reference's comparisons treat them as equal).
APUS_DEV uint32_t score_key(float v) { return f32_order_key(__float_as_uint(v) == 0x80000000u ? 0.0f : v); }

// top-(topk/kpool) pools per row, stable with lower-index ties
// (c/gdsa.h:404-429).  One CTA per row finds the key K-th from the top with
// a 4-pass radix select (8 bits a pass, block histogram in shared memory),
// then keeps every pool above it and, of the pools equal to it, the lowest
// indices until K are kept -- the set the reference's stable top-k picks, in
// O(pools) work per row instead of O(pools^2).
__global__ void __launch_bounds__(256) k_dsa_select(const float *score, const int *base_n, int kp, int ksel,
                                                    int maxpools, uint8_t *sel) {
    pdl_launch_dependents();
    __shared__ int hist[256];
    __shared__ uint32_t pre_sh;
    __shared__ int k_sh, wsum[8];
    const int t = blockIdx.x, tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    const int nvalid = min((*base_n + t + 1) / kp, maxpools);
    const float *s = score + (size_t)t * maxpools;
    uint8_t *o = sel + (size_t)t * maxpools;
    if (nvalid <= ksel) {
        for (int p = tid; p < nvalid; p += blockDim.x) o[p] = 1;
        return;
    }
    uint32_t prefix = 0, mask = 0;
    int k = ksel;                                  // rank (from the top) still to place
    for (int shift = 24; shift >= 0; shift -= 8) {
        hist[tid] = 0;
        __syncthreads();
        for (int p = tid; p < nvalid; p += blockDim.x) {
            const uint32_t u = score_key(s[p]);
            if ((u & mask) == prefix) atomicAdd(&hist[(u >> shift) & 255u], 1);
        }
        __syncthreads();
        if (warp == 0) {
            // lane l sums digits 255-8l .. 248-8l (descending); a scan over the
            // lanes finds the digit where the count from the top reaches k
            int c[8], tot = 0;
#pragma unroll
            for (int j = 0; j < 8; j++) { c[j] = hist[255 - 8 * lane - j]; tot += c[j]; }
            int incl = tot;
#pragma unroll
            for (int off = 1; off < 32; off <<= 1) {
                const int v = __shfl_up_sync(0xffffffffu, incl, off);
                if (lane >= off) incl += v;
            }
            const int excl = incl - tot;
            const unsigned own = __ballot_sync(0xffffffffu, excl < k && k <= incl);
            if (lane == __ffs(own) - 1) {
                int cum = excl;
#pragma unroll
                for (int j = 0; j < 8; j++) {
                    if (cum + c[j] >= k) {
                        pre_sh = prefix | ((uint32_t)(255 - 8 * lane - j) << shift);
                        k_sh = k - cum;
                        break;
                    }
                    cum += c[j];
                }
            }
        }
        __syncthreads();
        prefix = pre_sh;
        k = k_sh;
        mask |= 255u << shift;
    }
    // prefix: the K-th key; k: how many pools equal to it to keep (lowest
    // indices first).  Thread tid owns pools [tid*chunk, (tid+1)*chunk).
    const int chunk = (nvalid + blockDim.x - 1) / blockDim.x;
    const int p0 = min(tid * chunk, nvalid), p1 = min(p0 + chunk, nvalid);
    int eq = 0;
    for (int p = p0; p < p1; p++) eq += score_key(s[p]) == prefix;
    int incl = eq;
#pragma unroll
    for (int off = 1; off < 32; off <<= 1) {
        const int v = __shfl_up_sync(0xffffffffu, incl, off);
        if (lane >= off) incl += v;
    }
    if (lane == 31) wsum[warp] = incl;
    __syncthreads();
    int before = incl - eq;
    for (int w = 0; w < warp; w++) before += wsum[w];
    for (int p = p0; p < p1; p++) {
        const uint32_t u = score_key(s[p]);
        const bool keep = u > prefix || (u == prefix && before++ < k);
        o[p] = keep ? 1 : 0;
    }
}

// Attention over the selected positions (c/gdsa.h:451-517).
//   sc = bf16(bf16(q.k) * qd^-0.5); p = bf16(softmax(sc)); o = bf16(sum p v)
// Visibility of position j for row t: j <= base+t and (its pool is
// selected, or j is in the row's incomplete tail pool).  p_j = 0 for every
// other position, so row t's output depends only on its own row (the rows
// of one call do not interact).
//
// One cluster of ASPLIT CTAs per head; CTA z owns the ATJ-position tiles
// z, z + ASPLIT, ... (a fixed function of the position, so a row gets the
// same partial sums whatever rows share the call).  Both contractions run on the tensor cores (mma.sync
// m16n8k16, bf16 in, f32 accumulate): scores = K_tile[pos][qd] . Q^T (the 8
// query rows are the n dimension), out^T = V_tile^T . P^T.  K and V stream
// through shared memory (cp.async, double buffered, 16-byte chunks
// XOR-swizzled by row so ldmatrix is conflict-free).  The softmax's row max,
// row sum and the output partials cross the cluster through distributed
// shared memory and are combined in CTA order, so every CTA sees the same
// bits.  p is stored as BF16 (exact: it is BF16-rounded by definition).
#define ATJ 64
#define ASPLIT 4
__device__ __forceinline__ uint32_t swz(int row, int chunk, int rowbytes) {
    return (uint32_t)(row * rowbytes + ((chunk ^ (row & 7)) << 4));
}

__global__ void __cluster_dims__(1, ASPLIT, 1) __launch_bounds__(256)
k_dsa_attn(const uint16_t *q, const int *base_n, int R, int AH, int qd, int vd, int kp, int maxpools,
           const uint8_t *sel, DsaState ds, float *sbuf, uint16_t *pbuf, int sstride, uint16_t *out) {
    pdl_launch_dependents();
    namespace cg = cooperative_groups;
    cg::cluster_group cluster = cg::this_cluster();
    extern __shared__ __align__(128) uint8_t dsm[];
    const int h = blockIdx.x, z = (int)cluster.block_rank();
    const int base = *base_n;
    const int nmax = base + R;            // positions that exist after this call's append
    const int nt = (nmax + ATJ - 1) / ATJ;
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int g = lane >> 2, q4 = lane & 3;
    const int wmax = qd > vd ? qd : vd;
    const int TB = ATJ * wmax * 2;                     // bytes of one K/V tile buffer
    const int PROW = (ATJ + 8) * 2, QROW = (qd + 8) * 2;
    uint8_t *kv0 = dsm, *pt0 = dsm + 2 * TB, *qs = pt0 + 2 * MAXR * PROW;
    float *opart = (float *)(qs + MAXR * QROW);        // [MAXR][vd] this CTA's output partial
    const float scale = (float)(1.0 / sqrt((double)qd));
    float *sc = sbuf + (size_t)h * MAXR * sstride;     // [MAXR][sstride] scores, then e
    uint16_t *pb = pbuf + (size_t)h * MAXR * sstride;  // [MAXR][sstride] p (BF16)
    __shared__ int tail_s[MAXR];
    __shared__ float rmax_s[MAXR], rsum_s[MAXR], wmax_s[ATJ / 16][MAXR];
    for (int i = threadIdx.x; i < MAXR * (qd / 8); i += blockDim.x) {
        const int t = i / (qd / 8), c = i % (qd / 8);
        uint4 v = make_uint4(0, 0, 0, 0);
        if (t < R) v = *(const uint4 *)(q + (size_t)t * AH * qd + (size_t)h * qd + c * 8);
        *(uint4 *)(qs + t * QROW + c * 16) = v;
    }
    for (int i = threadIdx.x; i < 2 * MAXR * (PROW / 16); i += blockDim.x)
        *(uint4 *)(pt0 + i * 16) = make_uint4(0, 0, 0, 0);
    if (threadIdx.x < MAXR) {
        const int vis = base + threadIdx.x + 1;
        tail_s[threadIdx.x] = vis - vis % kp;
        rmax_s[threadIdx.x] = -3.4028234663852886e+38f;
        rsum_s[threadIdx.x] = 0.f;
    }
    auto visible = [&](int t, int j) -> bool {
        if (j > base + t) return false;
        if (j >= tail_s[t]) return true;
        const int p = j / kp;
        return p < maxpools && sel[(size_t)t * maxpools + p];
    };
    auto stage = [&](const uint16_t *cache, int w, int ti, int b, bool probs) {
        const int j0 = ti * ATJ, cpr = w / 8;
        uint8_t *dst = kv0 + b * TB;
        for (int i = threadIdx.x; i < ATJ * cpr; i += blockDim.x) {
            const int jj = i / cpr, c = i % cpr;
            const int j = min(j0 + jj, nmax - 1);
            cp_async16(dst + swz(jj, c, w * 2), cache + ((size_t)h * ds.cap + j) * w + c * 8);
        }
        if (probs)
            for (int i = threadIdx.x; i < R * (ATJ / 8); i += blockDim.x) {
                const int t = i / (ATJ / 8), c = i % (ATJ / 8);
                cp_async16(pt0 + b * MAXR * PROW + t * PROW + c * 16, pb + (size_t)t * sstride + j0 + c * 8);
            }
        cp_async_commit();
    };
    __syncthreads();
    // ---- scores over this CTA's tiles: warp w owns positions [16w, 16w+16)
    // of a tile when w < ATJ/16
    uint32_t qb[16][2];
    const int nks = qd / 16;
    float kmax[2] = {-INFINITY, -INFINITY};
#pragma unroll
    for (int ks = 0; ks < 16; ks++)
        if (ks < nks) ldsm_x2(qb[ks][0], qb[ks][1], qs + (lane & 7) * QROW + (ks * 16 + ((lane >> 3) & 1) * 8) * 2);
    if (z < nt) stage(ds.k, qd, z, 0, false);
    for (int ti = z, it = 0; ti < nt; ti += ASPLIT, it++) {
        if (ti + ASPLIT < nt) stage(ds.k, qd, ti + ASPLIT, (it + 1) & 1, false);
        else cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        if (warp < ATJ / 16) {
            const uint8_t *kt = kv0 + (it & 1) * TB;
            const int r0 = warp * 16;
            float c0 = 0.f, c1 = 0.f, c2 = 0.f, c3 = 0.f;
#pragma unroll
            for (int ks = 0; ks < 16; ks++) {
                if (ks >= nks) break;
                uint32_t a0, a1, a2, a3;
                ldsm_x4(a0, a1, a2, a3, kt + swz(r0 + (lane & 15), ks * 2 + (lane >> 4), qd * 2));
                mma_bf16_16816(c0, c1, c2, c3, a0, a1, a2, a3, qb[ks][0], qb[ks][1]);
            }
            // c0/c1: position r0+g, rows 2q4 / 2q4+1; c2/c3: position r0+g+8.
            // Positions a row cannot see are stored as -inf (p = 0 below);
            // the row maxima of this CTA's positions accumulate in kmax.
            const int pa = ti * ATJ + r0 + g, pbp = pa + 8, t0 = 2 * q4, t1 = t0 + 1;
            const float cv[4] = {c0, c1, c2, c3};
#pragma unroll
            for (int e = 0; e < 4; e++) {
                const int j = (e & 2) ? pbp : pa, t = t0 + (e & 1);
                if (j < nmax && t < R) {
                    const float v = visible(t, j) ? bf16_round(bf16_round(cv[e]) * scale) : -INFINITY;
                    sc[(size_t)t * sstride + j] = v;
                    kmax[e & 1] = fmaxf(kmax[e & 1], v);
                }
            }
        }
        __syncthreads();
    }
    // row max of this CTA: lanes (g, q4) hold rows 2q4, 2q4+1 -> reduce over g
    // and the score warps in warp order
#pragma unroll
    for (int u = 0; u < 2; u++)
#pragma unroll
        for (int off = 4; off < 32; off <<= 1) kmax[u] = fmaxf(kmax[u], __shfl_xor_sync(0xffffffffu, kmax[u], off));
    if (warp < ATJ / 16 && lane < 4) {
        wmax_s[warp][2 * lane] = kmax[0];
        wmax_s[warp][2 * lane + 1] = kmax[1];
    }
    __syncthreads();
    // ---- softmax (warp t owns row t over this CTA's positions), cluster-wide.
    // Position j of tile ti is lane-slot (ti, j % 32): every lane walks its
    // slots in tile order, the eight loads of a tile issued together.
    const int t = warp;
    const bool row = t < R;
    const int qpos = base + t;
    float *srow = sc + (size_t)(row ? t : 0) * sstride;
    if (row && lane == 0) {
        float m = wmax_s[0][t];
        for (int w = 1; w < ATJ / 16; w++) m = fmaxf(m, wmax_s[w][t]);
        rmax_s[t] = m;
    }
    cluster.sync();
    float mx = -INFINITY;
    if (row)
        for (int zz = 0; zz < ASPLIT; zz++) mx = fmaxf(mx, cluster.map_shared_rank(rmax_s, zz)[t]);
    constexpr int PL = ATJ / 32;                      // slots of a lane in one tile
    if (row) {
        float su = 0.f;
        for (int ti = z; ti < nt; ti += ASPLIT) {
            float v[PL];
#pragma unroll
            for (int u = 0; u < PL; u++) {
                const int j = ti * ATJ + u * 32 + lane;
                v[u] = j <= qpos ? srow[j] : -INFINITY;
            }
#pragma unroll
            for (int u = 0; u < PL; u++)
                if (v[u] != -INFINITY) su += expf(v[u] - mx);
        }
#pragma unroll
        for (int off = 16; off; off >>= 1) su += __shfl_xor_sync(0xffffffffu, su, off);
        if (lane == 0) rsum_s[t] = su;
    }
    cluster.sync();
    if (row) {
        float sum = cluster.map_shared_rank(rsum_s, 0)[t];
        for (int zz = 1; zz < ASPLIT; zz++) sum += cluster.map_shared_rank(rsum_s, zz)[t];
        uint16_t *prow = pb + (size_t)t * sstride;
        for (int ti = z; ti < nt; ti += ASPLIT) {
            float v[PL];
#pragma unroll
            for (int u = 0; u < PL; u++) {
                const int j = ti * ATJ + u * 32 + lane;
                v[u] = j <= qpos && j < nmax ? srow[j] : -INFINITY;
            }
#pragma unroll
            for (int u = 0; u < PL; u++)
                prow[ti * ATJ + u * 32 + lane] = v[u] != -INFINITY ? bf16_bits(expf(v[u] - mx) / sum) : (uint16_t)0;
        }
    }
    __syncthreads();
    // ---- output partial over this CTA's tiles: warp w owns dv tiles w, w+8
    const int nmt = vd / 16;
    float acc[2][4];
#pragma unroll
    for (int u = 0; u < 2; u++)
#pragma unroll
        for (int e = 0; e < 4; e++) acc[u][e] = 0.f;
    if (z < nt) stage(ds.v, vd, z, 0, true);
    for (int ti = z, it = 0; ti < nt; ti += ASPLIT, it++) {
        if (ti + ASPLIT < nt) stage(ds.v, vd, ti + ASPLIT, (it + 1) & 1, true);
        else cp_async_commit();
        cp_async_wait<1>();
        __syncthreads();
        const uint8_t *vt = kv0 + (it & 1) * TB, *pt = pt0 + (it & 1) * MAXR * PROW;
#pragma unroll
        for (int ks = 0; ks < ATJ / 16; ks++) {
            uint32_t b0, b1;
            ldsm_x2(b0, b1, pt + (lane & 7) * PROW + (ks * 16 + ((lane >> 3) & 1) * 8) * 2);
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int mt = warp + 8 * u;
                if (mt >= nmt) break;
                // matrices: (dv 0-7, j 0-7), (dv 8-15, j 0-7), (dv 0-7, j 8-15), (dv 8-15, j 8-15)
                const int mi = lane >> 3;
                const int jr = ks * 16 + (mi >> 1) * 8 + (lane & 7), ch = mt * 2 + (mi & 1);
                uint32_t a0, a1, a2, a3;
                ldsm_x4_t(a0, a1, a2, a3, vt + swz(jr, ch, vd * 2));
                mma_bf16_16816(acc[u][0], acc[u][1], acc[u][2], acc[u][3], a0, a1, a2, a3, b0, b1);
            }
        }
        __syncthreads();
    }
    // acc: (dv = 16mt+g, rows 2q4 / 2q4+1) and (dv + 8, ...) -> this CTA's partial
#pragma unroll
    for (int u = 0; u < 2; u++) {
        const int mt = warp + 8 * u;
        if (mt >= nmt) break;
        const int dv = mt * 16 + g, t0 = 2 * q4, t1 = t0 + 1;
        opart[t0 * vd + dv] = acc[u][0];
        opart[t0 * vd + dv + 8] = acc[u][2];
        opart[t1 * vd + dv] = acc[u][1];
        opart[t1 * vd + dv + 8] = acc[u][3];
    }
    cluster.sync();
    if (z == 0)        // sum the partials in CTA order
        for (int i = threadIdx.x; i < R * vd; i += blockDim.x) {
            float o = opart[i];
            for (int zz = 1; zz < ASPLIT; zz++) o += cluster.map_shared_rank(opart, zz)[i];
            out[(size_t)(i / vd) * AH * vd + (size_t)h * vd + i % vd] = bf16_bits(o);
        }
    cluster.sync();    // keep every CTA's shared memory alive until rank 0 has read it
}

}  // namespace apus

using namespace apus;

static int ok_launch() { return cudaGetLastError() == cudaSuccess ? 0 : -1; }

static size_t dsa_attn_smem(const Dims &D) {
    const int w = D.qd > D.vd ? D.qd : D.vd;
    return (size_t)2 * ATJ * w * 2 + (size_t)2 * MAXR * (ATJ + 8) * 2 + (size_t)MAXR * (D.qd + 8) * 2 +
           (size_t)MAXR * D.vd * 4;
}

// Leaves of the numpy pairwise recursion over n (what block_pw's 256-entry
// leaf table must hold).
static int pw_leaves(int n) {
    if (n <= 128) return 1;
    const int n2 = (n / 2) & ~7;
    return pw_leaves(n2) + pw_leaves(n - n2);
}

int layers_prepare(const Dims &D) {
    const int rows[] = {D.hc * D.d, D.d, D.ql, D.kl, D.ID, D.D};
    for (int n : rows)
        if (n > 0 && pw_leaves(n) > 256) return -1;
    if (D.K < 2 || D.K > 9 || D.kpool > 16 || D.qd > 256 || D.vd > 256 || D.qd % 64 || D.vd % 64 || D.ID % 8 ||
        D.IH * D.ID > 32 * 128)
        return -1;
    if (cudaFuncSetAttribute(k_dsa_attn, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)dsa_attn_smem(D)))
        return -1;
    // row kernels keep one or two fp32 copies of the row in dynamic smem
    const int maxrow = D.d > D.ql ? (D.d > D.kl ? D.d : D.kl) : (D.ql > D.kl ? D.ql : D.kl);
    const size_t need_rms = (size_t)D.hc * D.d * 4, need_row = (size_t)2 * maxrow * 4;
    if (need_rms > 200 * 1024 || need_row > 200 * 1024) return -1;
    // k_hc_postmix: one warp slot per mix and the sum of squares (<= 32)
    if (D.d % 8 || D.hc > 8 || (2 + D.hc) * D.hc + 1 > 32 || (size_t)D.hc * D.d * 4 > 200 * 1024) return -1;
    if (cudaFuncSetAttribute(k_hc_pre, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)need_row) ||
        cudaFuncSetAttribute(k_head_norm, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)need_row) ||
        cudaFuncSetAttribute(k_rmsnorm_rows, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)need_row) ||
        cudaFuncSetAttribute(k_norm_seg, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)need_row))
        return -1;
    return 0;
}

int k_embed_launch(const uint16_t *embed, const int32_t *ids, int R, int d, int hc, uint16_t *h4, cudaStream_t st) {
    k_embed<<<dim3((d + 255) / 256, R), 256, 0, st>>>(embed, ids, d, hc, h4);
    return ok_launch();
}

int hc_nchunk(const Dims &D) { return (D.d + HC_PM_CW - 1) / HC_PM_CW; }

int hc_pre_launch(const Dims &D, const LayerW &W, int site, const uint16_t *h4, int R, Scratch &S,
                  cudaStream_t st) {
    k_hc_pre<<<2 * R, 512, (size_t)2 * D.d * 4, st>>>(h4, S.mix, hc_nchunk(D), W.hc_scale[site], W.hc_base[site],
                                                      site ? W.post_norm : W.input_norm, D.d, D.hc,
                                                      D.sinkhorn_iters, D.hc_eps, D.eps, R, S.post, S.comb, S.x);
    return ok_launch();
}

int hc_postmix_launch(const Dims &D, const uint16_t *x, const MoeDev *moe, const uint16_t *h4, int R, Scratch &S,
                      uint16_t *h4out, const uint16_t *fn_next, cudaStream_t st) {
    if (R < 1 || R > MAXR || (h4out && !x && !moe)) return -1;
    HcPostMix a{};
    a.x = x;
    if (moe) a.moe = *moe;
    a.h4 = h4; a.post = S.post; a.comb = S.comb; a.h4out = h4out;
    a.fn = fn_next; a.part = S.mix;
    a.d = D.d; a.hc = D.hc; a.nmix = (2 + D.hc) * D.hc; a.R = R; a.nchunk = hc_nchunk(D);
    k_hc_postmix<<<a.nchunk, 256, 0, st>>>(a);
    return ok_launch();
}

int hc_postmix_rows_launch(const Dims &D, const uint16_t *x, const uint16_t *h4, int R, Scratch &S, uint16_t *h4out,
                           const uint16_t *fn_next, cudaStream_t st) {
    if (R < 1 || (h4out && !x)) return -1;
    HcPostMix a{};
    a.x = x;
    a.h4 = h4; a.post = S.post; a.comb = S.comb; a.h4out = h4out;
    a.fn = fn_next; a.part = S.mix;
    a.d = D.d; a.hc = D.hc; a.nmix = (2 + D.hc) * D.hc; a.R = R; a.nchunk = hc_nchunk(D);
    k_hc_postmix<<<dim3(a.nchunk, (R + MAXR - 1) / MAXR), 256, 0, st>>>(a);
    return ok_launch();
}

int head_norm_launch(const Dims &D, const uint16_t *h4, const uint16_t *norm_w, int R, uint16_t *yn,
                     unsigned long long *keys, cudaStream_t st) {
    k_head_norm<<<R, 512, 2 * D.d * sizeof(float), st>>>(h4, norm_w, D.d, D.hc, D.eps, yn, keys);
    return ok_launch();
}

int rmsnorm_rows_launch(const uint16_t *x, long ldx, const uint16_t *w, int n, int R, float eps, uint16_t *y,
                        long ldy, cudaStream_t st) {
    k_rmsnorm_rows<<<R, 512, 2 * n * sizeof(float), st>>>(x, ldx, w, n, eps, y, ldy);
    return ok_launch();
}

int norm_seg_launch(const NormSeg *seg, int nseg, int R, float eps, unsigned long long *keys, cudaStream_t st) {
    if (nseg < 1 || nseg > 2) return -1;
    NormSegs sg{};
    int n = 0;
    for (int i = 0; i < nseg; i++) {
        sg.s[i] = seg[i];
        n = seg[i].n > n ? seg[i].n : n;
    }
    k_norm_seg<<<dim3(R, nseg), 512, (size_t)2 * n * sizeof(float), st>>>(sg, eps, keys);
    return ok_launch();
}

int residual_add_launch(uint16_t *x, const uint16_t *sub, long n, cudaStream_t st) {
    k_residual_add<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(x, sub, n);
    return ok_launch();
}

int kda_launch(const Dims &D, const LayerW &W, KdaState &KS, const Ctl *ctl, int R, Scratch &S, float *part,
               int *tick, cudaStream_t st) {
    const int qkv = D.qkv, ldkp = kda_ldkp(D);
    const int *d_probs = S.two_problems, *d_cnt = S.two_problems + 2;
    // q|k|v|f_a|g_a|b share the normed input: one GEMV
    GemvDesc g{};
    g.W = W.kda.proj; g.x = S.x; g.ldx = D.d; g.R = R; g.O = kda_nproj(D); g.K = D.d; g.fp8 = 0;
    g.y = S.kp; g.ldy = ldkp; g.part = part; g.ticket = tick;
    g.pdl = 1;
    if (gemv_launch(g, st)) return -1;
    // conv + SiLU over q|k|v, tokens chained, checkpointed
    k_kda_conv<<<(3 * qkv + 127) / 128, 128, 0, st>>>(S.kp, ldkp, W.kda.conv, KS.conv, ctl, R, 3 * qkv, D.K, S.qkvc);
    if (ok_launch()) return -1;
    // f_b and g_b (low-rank up-projections) as two problems of one launch
    GemvDesc fg{};
    fg.W = W.kda.fg_b; fg.x = S.kp + 3 * qkv; fg.ldx = ldkp; fg.R = R; fg.O = qkv; fg.K = D.Dr; fg.fp8 = 0;
    fg.y = S.fgo; fg.ldy = qkv;
    fg.gexpert = d_probs; fg.gcount = d_cnt; fg.gmax = 2; fg.gnum = 2;
    fg.w_estride = (long)qkv * D.Dr * 2; fg.x_pstride = D.Dr; fg.y_pstride = (long)MAXR * qkv;
    fg.pdl = 1;
    if (gemv_launch(fg, st)) return -1;
    if (D.D != 128) return -1;
    k_kda_rec<128><<<D.H, 128, 0, st>>>(S.qkvc, S.kp, ldkp, 3 * qkv + 2 * D.Dr, S.fgo, (long)MAXR * qkv,
                                         W.kda.A_log, W.kda.dt_bias, W.kda.o_norm, KS.rec, ctl, R, D.H,
                                         D.lower_bound, D.eps, (float)pow((double)D.D, -0.5), S.core);
    if (ok_launch()) return -1;
    GemvDesc o{};
    o.W = W.kda.o_w; o.x = S.core; o.ldx = qkv; o.R = R; o.O = D.d; o.K = qkv; o.fp8 = 0;
    o.y = S.sub; o.ldy = D.d; o.part = part; o.ticket = tick;
    o.pdl = 1;
    return gemv_launch(o, st);
}

int dsa_launch(const Dims &D, const DsaW &W, DsaState &DS, const int *base_n, int R, Scratch &S, const uint16_t *x,
               uint16_t *out, float *part, int *tick, cudaStream_t st) {
    const int ql = D.ql, kl = D.kl;
    GemvDesc a{};
    a.W = W.qkva_c; a.WS = W.qkva_s; a.nkb = (D.d + 127) / 128; a.x = x; a.ldx = D.d; a.R = R;
    a.O = ql + kl; a.K = D.d; a.fp8 = 1; a.y = S.qkva; a.ldy = ql + kl; a.part = part; a.ticket = tick;
    a.pdl = 1;
    if (gemv_launch(a, st)) return -1;
    {   // q_a and kv_a norms (c/gdsa.h:555-590) in one launch
        NormSeg sg[2] = {{S.qkva, ql + kl, nullptr, nullptr, 0, W.q_a_norm, ql, S.qres, ql},
                         {S.qkva + ql, ql + kl, nullptr, nullptr, 0, W.kv_a_norm, kl, S.kpass, kl}};
        if (norm_seg_launch(sg, 2, R, D.eps, nullptr, st)) return -1;
    }
    GemvDesc b{};
    b.W = W.q_b_c; b.WS = W.q_b_s; b.nkb = (ql + 127) / 128; b.x = S.qres; b.ldx = ql; b.R = R;
    b.O = (long)D.AH * D.qd; b.K = ql; b.fp8 = 1; b.y = S.q; b.ldy = (long)D.AH * D.qd; b.part = part; b.ticket = tick;
    b.pdl = 1;
    if (gemv_launch(b, st)) return -1;
    GemvDesc c{};
    c.W = W.kv_b; c.x = S.kpass; c.ldx = kl; c.R = R; c.O = (long)D.AH * (D.qd + D.vd); c.K = kl; c.fp8 = 0;
    c.y = S.kvb; c.ldy = c.O; c.part = part; c.ticket = tick;
    c.pdl = 1;
    if (gemv_launch(c, st)) return -1;
    GemvDesc e{};
    e.W = W.idx_kgw; e.x = x; e.ldx = D.d; e.R = R; e.O = 2 * D.ID + D.IH; e.K = D.d; e.fp8 = 0;
    e.y = S.ikgw; e.ldy = e.O; e.part = part; e.ticket = tick;
    e.pdl = 1;
    if (gemv_launch(e, st)) return -1;
    GemvDesc f{};
    f.W = W.idx_wq_b; f.x = S.qres; f.ldx = ql; f.R = R; f.O = (long)D.IH * D.ID; f.K = ql; f.fp8 = 0;
    f.y = S.iq; f.ldy = f.O; f.part = part; f.ticket = tick;
    f.pdl = 1;
    if (gemv_launch(f, st)) return -1;
    k_dsa_append<<<dim3(R, D.AH), 128, 0, st>>>(S.kvb, S.ikgw, W.idx_knorm_w, W.idx_knorm_b, base_n, D.AH, D.qd,
                                                 D.vd, D.ID, D.IH, DS.cap, DS);
    k_dsa_pool<<<R, 128, 0, st>>>(W.idx_ape, base_n, R, D.ID, D.kpool, DS.cap, DS);
    k_dsa_score<<<dim3((S.maxpools + 7) / 8, R), 256, 0, st>>>(S.iq, S.ikgw, base_n, D.IH, D.ID, D.kpool,
                                                                 S.maxpools, DS, S.iscore);
    k_dsa_select<<<R, 256, 0, st>>>(S.iscore, base_n, D.kpool, D.topk / D.kpool, S.maxpools, S.isel);
    if (ok_launch()) return -1;
    k_dsa_attn<<<dim3(D.AH, ASPLIT), 256, dsa_attn_smem(D), st>>>(S.q, base_n, R, D.AH, D.qd, D.vd, D.kpool, S.maxpools,
                                                     S.isel, DS, (float *)S.attn_scores, S.attn_p,
                                                     S.attn_sstride, S.attn);
    if (ok_launch()) return -1;
    GemvDesc o{};
    o.W = W.o_c; o.WS = W.o_s; o.nkb = ((long)D.AH * D.vd + 127) / 128; o.x = S.attn; o.ldx = (long)D.AH * D.vd;
    o.R = R; o.O = D.d; o.K = (long)D.AH * D.vd; o.fp8 = 1; o.y = out; o.ldy = D.d; o.part = part; o.ticket = tick;
    o.pdl = 1;
    return gemv_launch(o, st);
}

int dsa_rows_launch(const Dims &D, const DsaW &W, DsaState &DS, const int *pos_iota, int p0, int R,
                    const DsaRows &X, Scratch &S, uint16_t *wbuf, const uint16_t *x, uint16_t *out, cudaStream_t st) {
    const int ql = D.ql, kl = D.kl, d = D.d;
    const long nq = (long)D.AH * D.qd, nkv = (long)D.AH * (D.qd + D.vd), nik = 2L * D.ID + D.IH;
    const long ni = (long)D.IH * D.ID, na = (long)D.AH * D.vd;
    const int *base = pos_iota + p0;
    // q_a | kv_a (FP8), then their norms
    if (fp8_dequant_launch(W.qkva_c, W.qkva_s, wbuf, ql + kl, d, st)) return -1;
    if (gemm_tc_launch(x, d, wbuf, d, X.qkva, ql + kl, nullptr, 0, R, ql + kl, d, st)) return -1;
    {
        NormSeg sg[2] = {{X.qkva, ql + kl, nullptr, nullptr, 0, W.q_a_norm, ql, X.qres, ql},
                         {X.qkva + ql, ql + kl, nullptr, nullptr, 0, W.kv_a_norm, kl, X.kpass, kl}};
        if (norm_seg_launch(sg, 2, R, D.eps, nullptr, st)) return -1;
    }
    if (fp8_dequant_launch(W.q_b_c, W.q_b_s, wbuf, nq, ql, st)) return -1;
    if (gemm_tc_launch(X.qres, ql, wbuf, ql, X.q, nq, nullptr, 0, R, nq, ql, st)) return -1;
    if (gemm_tc_launch(X.kpass, kl, W.kv_b, kl, X.kvb, nkv, nullptr, 0, R, nkv, kl, st)) return -1;
    if (gemm_tc_launch(x, d, W.idx_kgw, d, X.ikgw, nik, nullptr, 0, R, nik, d, st)) return -1;
    if (gemm_tc_launch(X.qres, ql, W.idx_wq_b, ql, X.iq, ni, nullptr, 0, R, ni, ql, st)) return -1;
    // the chunk's cache rows, the pools they complete, every row's pool scores
    // and selection (each row sees the pools complete at its own position)
    k_dsa_append<<<dim3(R, D.AH), 128, 0, st>>>(X.kvb, X.ikgw, W.idx_knorm_w, W.idx_knorm_b, base, D.AH, D.qd, D.vd,
                                                 D.ID, D.IH, DS.cap, DS);
    k_dsa_pool<<<R, 128, 0, st>>>(W.idx_ape, base, R, D.ID, D.kpool, DS.cap, DS);
    k_dsa_score<<<dim3((S.maxpools + 7) / 8, R), 256, 0, st>>>(X.iq, X.ikgw, base, D.IH, D.ID, D.kpool, S.maxpools, DS,
                                                                 X.iscore);
    k_dsa_select<<<R, 256, 0, st>>>(X.iscore, base, D.kpool, D.topk / D.kpool, S.maxpools, X.isel);
    if (ok_launch()) return -1;
    // attention, 8 rows a launch: rows r0.. see positions <= p0 + r0 + t
    for (int r0 = 0; r0 < R; r0 += MAXR) {
        const int r = R - r0 < MAXR ? R - r0 : MAXR;
        k_dsa_attn<<<dim3(D.AH, ASPLIT), 256, dsa_attn_smem(D), st>>>(
            X.q + (size_t)r0 * nq, base + r0, r, D.AH, D.qd, D.vd, D.kpool, S.maxpools, X.isel + (size_t)r0 * S.maxpools,
            DS, S.attn_scores, S.attn_p, S.attn_sstride, X.attn + (size_t)r0 * na);
        if (ok_launch()) return -1;
    }
    if (fp8_dequant_launch(W.o_c, W.o_s, wbuf, d, na, st)) return -1;
    return gemm_tc_launch(X.attn, na, wbuf, na, out, d, nullptr, 0, R, d, na, st);
}
