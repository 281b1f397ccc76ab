// prefill.cu — the row kernels of the prompt pass (c/gmodel.h:1658-1666
// apus_gmodel_prefill_h): a chunk of prompt rows goes through each layer
// together, its linears on the tensor-core GEMM, instead of 8-row decode
// batches.
//
// What changes against the decode path is only what the reference's prefill
// changes: the KDA core is the chunked delta rule (c/gkda.h:350-539) over the
// prompt's 64-row chunks, and the DSA appends the chunk's rows before its
// queries attend (c/gdsa.h:555-674 forward3 over the chunk; every row still
// sees only positions <= its own).  Conv, gates, o_norm and the SwiGLU keep
// the decode path's per-row arithmetic.
#include "common.cuh"
#include "gcuda.h"
#include "model_dev.h"

namespace apus {

// Depthwise causal conv + SiLU (c/gkda.h:227-257) over R rows, chained per
// channel from the committed window conv_slot [C][K-1]; the window after the
// last row is written back there.  The rows' inputs are loaded eight ahead.
__global__ void __launch_bounds__(128) k_conv_rows(const uint16_t *kp, long ldkp, const uint16_t *conv_w,
                                                   uint16_t *conv_slot, int R, int C, int K, uint16_t *out) {
    const int c = blockIdx.x * blockDim.x + threadIdx.x;
    if (c >= C) return;
    uint16_t st[8], wc[9];
#pragma unroll
    for (int j = 0; j < 9; j++)
        if (j < K) wc[j] = conv_w[(size_t)c * K + j];
#pragma unroll
    for (int j = 0; j < 8; j++)
        if (j < K - 1) st[j] = conv_slot[(size_t)c * (K - 1) + j];
    for (int t0 = 0; t0 < R; t0 += 8) {
        uint16_t xs[8];
#pragma unroll
        for (int u = 0; u < 8; u++) xs[u] = t0 + u < R ? kp[(size_t)(t0 + u) * ldkp + c] : 0;
#pragma unroll
        for (int u = 0; u < 8; u++) {
            if (t0 + u >= R) break;
            float acc = 0.f;
#pragma unroll
            for (int i = 0; i < 8; i++)
                if (i < K - 1) acc += bf16_f32(wc[i]) * bf16_f32(st[i]);
            acc += bf16_f32(wc[K - 1]) * bf16_f32(xs[u]);
            out[(size_t)(t0 + u) * C + c] = bf16_bits(acc * sigmoid_np(acc));
#pragma unroll
            for (int j = 0; j < 7; j++)
                if (j + 1 < K - 1) st[j] = st[j + 1];
            st[K - 2] = xs[u];
        }
    }
#pragma unroll
    for (int j = 0; j < 8; j++)
        if (j < K - 1) conv_slot[(size_t)c * (K - 1) + j] = st[j];
}

// Forget gate and beta of R rows (c/gkda.h:629-647):
//   g[t][i] = lb * sigmoid(exp(A_log[h]) * (fg[t][i] + dt_bias[i]))   (fp32)
//   beta[t][h] = bf16(sigmoid(b[t][h]))
__global__ void k_kda_gates_rows(const uint16_t *fg, const uint16_t *kp, long ldkp, int beta_off, const float *A_log,
                                 const float *dt_bias, int R, int H, int D, float lb, float *g, uint16_t *beta) {
    const int qkv = H * D;
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i < (long)R * qkv) {
        const int c = (int)(i % qkv), h = c / D;
        const float z = bf16_f32(fg[i]) + dt_bias[c];
        g[i] = lb * sigmoid_np(expf(A_log[h]) * z);
    }
    if (i < (long)R * H) {
        const int t = (int)(i / H), h = (int)(i % H);
        beta[i] = bf16_bits(sigmoid_np(bf16_f32(kp[(size_t)t * ldkp + beta_off + h])));
    }
}

// Gated o_norm (c/gkda.h:543-569) of one (row, head) per CTA of D threads:
// y = bf16(o_norm * (core / sqrt(mean(core^2) + eps)) * sigmoid(gate)).
__global__ void k_kda_onorm_rows(const uint16_t *core, const uint16_t *gate, const uint16_t *o_norm, int H, int D,
                                 float eps, uint16_t *out) {
    __shared__ float sq[128];
    __shared__ float inv;
    const int t = blockIdx.x / H, h = blockIdx.x % H, j = threadIdx.x;
    const size_t o = (size_t)t * H * D + (size_t)h * D + j;
    const float c = bf16_f32(core[o]);
    sq[j] = c * c;
    __syncthreads();
    if (j == 0) inv = 1.0f / sqrtf(pw_sum_leaf(sq, D) / (float)D + eps);
    __syncthreads();
    float y = c * inv;
    y = bf16_f32(o_norm[j]) * y;
    y = y * sigmoid_np(bf16_f32(gate[o]));
    out[o] = bf16_bits(y);
}

// h[t][i] = bf16(bf16(silu(min(g, lim))) * clamp(u, -lim, lim)) from the
// [gate | up] rows (c/gmoe.h:216-224), 8 columns a thread.
__global__ void k_swiglu_rows(const uint16_t *gu, int R, int inter, float lim, uint16_t *h) {
    const int nc = inter / 8;
    const long i = blockIdx.x * (long)blockDim.x + threadIdx.x;
    if (i >= (long)R * nc) return;
    const int t = (int)(i / nc), c = (int)(i % nc) * 8;
    const uint16_t *row = gu + (size_t)t * 2 * inter;
    const uint4 gv = *(const uint4 *)(row + c), uv = *(const uint4 *)(row + inter + c);
    const uint32_t gw[4] = {gv.x, gv.y, gv.z, gv.w}, uw[4] = {uv.x, uv.y, uv.z, uv.w};
    uint32_t o[4];
#pragma unroll
    for (int e = 0; e < 4; e++) {
        uint16_t hh[2];
#pragma unroll
        for (int hf = 0; hf < 2; hf++) {
            float gf = hf ? bf16hi(gw[e]) : bf16lo(gw[e]);
            float uf = hf ? bf16hi(uw[e]) : bf16lo(uw[e]);
            if (gf > lim) gf = lim;
            if (uf > lim) uf = lim;
            else if (uf < -lim) uf = -lim;
            const float hv = bf16_round(gf * sigmoid_np(gf));
            hh[hf] = bf16_bits(hv * uf);
        }
        o[e] = (uint32_t)hh[0] | ((uint32_t)hh[1] << 16);
    }
    *(uint4 *)(h + (size_t)t * inter + c) = make_uint4(o[0], o[1], o[2], o[3]);
}

__global__ void k_iota(int *a, int n) {
    const int i = blockIdx.x * blockDim.x + threadIdx.x;
    if (i < n) a[i] = i;
}

}  // namespace apus
using namespace apus;

static int ok_launch() { return cudaGetLastError() == cudaSuccess ? 0 : -1; }

// The GEMM of R rows; fewer than 64 rows still run on the tensor cores (the
// rows past R read zeros and are not stored), so every prompt row takes the
// same arithmetic whatever the chunk's size.
static int gemm_rows(const uint16_t *x, long ldx, const uint16_t *w, long ldw, uint16_t *y, long ldy, int R, long O,
                     long K, cudaStream_t st) {
    return gemm_tc_launch(x, ldx, w, ldw, y, ldy, nullptr, 0, R, O, K, st);
}

int iota_launch(int *a, int n, cudaStream_t st) {
    k_iota<<<(n + 255) / 256, 256, 0, st>>>(a, n);
    return ok_launch();
}

int kda_rows_launch(const Dims &D, const LayerW &W, uint16_t *conv_slot, float *rec_slot, int R, const KdaRows &X,
                    const uint16_t *x, uint16_t *out, cudaStream_t st) {
    const int qkv = D.qkv, ldkp = kda_ldkp(D), nproj = kda_nproj(D);
    if (D.D != 128 || R < 1 || R > X.W) return -1;
    // q | k | v | f_a | g_a | b from the normed rows
    if (gemm_rows(x, D.d, W.kda.proj, D.d, X.kp, ldkp, R, nproj, D.d, st)) return -1;
    k_conv_rows<<<(3 * qkv + 127) / 128, 128, 0, st>>>(X.kp, ldkp, W.kda.conv, conv_slot, R, 3 * qkv, D.K, X.qkvc);
    if (ok_launch()) return -1;
    // f_b, g_b low-rank up-projections
    uint16_t *fb = X.fgo, *gb = X.fgo + (size_t)X.W * qkv;
    if (gemm_rows(X.kp + 3 * qkv, ldkp, W.kda.fg_b, D.Dr, fb, qkv, R, qkv, D.Dr, st)) return -1;
    if (gemm_rows(X.kp + 3 * qkv + D.Dr, ldkp, W.kda.fg_b + (size_t)qkv * D.Dr, D.Dr, gb, qkv, R, qkv, D.Dr, st))
        return -1;
    {
        const long n = (long)R * qkv;
        k_kda_gates_rows<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(fb, X.kp, ldkp, 3 * qkv + 2 * D.Dr,
                                                                      W.kda.A_log, W.kda.dt_bias, R, D.H, D.D,
                                                                      D.lower_bound, X.g, X.beta);
        if (ok_launch()) return -1;
    }
    // the chunked core over the rows, the state carried in the committed slot
    if (kda_chunk_launch(X.qkvc, X.qkvc + qkv, X.qkvc + 2 * qkv, X.g, X.beta, rec_slot, X.core, R, D.H, D.D, st,
                         3L * qkv))
        return -1;
    k_kda_onorm_rows<<<R * D.H, D.D, 0, st>>>(X.core, gb, W.kda.o_norm, D.H, D.D, D.eps, X.onorm);
    if (ok_launch()) return -1;
    return gemm_rows(X.onorm, qkv, W.kda.o_w, qkv, out, D.d, R, D.d, qkv, st);
}

// A dense MLP (the shared slot of a 0-expert layer) over R rows: the FP8
// gate|up and down matrices dequantised into wbuf, each used by one GEMM.
int mlp_rows_launch(const MoeDev &md, int R, const MlpRows &X, uint16_t *wbuf, const uint16_t *x, uint16_t *out,
                    cudaStream_t st) {
    const int d = md.dim, inter = md.inter;
    if (md.E != 0 || R < 1 || inter % 8) return -1;
    const size_t slot = (size_t)md.eloc;    // the MLP's local slot
    const size_t nkd = (d + 127) / 128, nki = (inter + 127) / 128;
    if (fp8_dequant_launch(md.gu_codes + slot * 2 * inter * d, md.gu_scales + slot * (2 * inter / 128) * nkd, wbuf,
                           2L * inter, d, st))
        return -1;
    if (gemm_rows(x, d, wbuf, d, X.gu, 2L * inter, R, 2L * inter, d, st)) return -1;
    const long n = (long)R * (inter / 8);
    k_swiglu_rows<<<(unsigned)((n + 255) / 256), 256, 0, st>>>(X.gu, R, inter, md.limit, X.h);
    if (ok_launch()) return -1;
    if (fp8_dequant_launch(md.d_codes + slot * d * inter, md.d_scales + slot * nkd * nki, wbuf, d, inter, st))
        return -1;
    return gemm_rows(X.h, inter, wbuf, inter, out, d, R, d, inter, st);
}
