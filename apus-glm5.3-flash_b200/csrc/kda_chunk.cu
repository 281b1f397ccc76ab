// kda_chunk.cu — the chunked KDA (delta-rule) prefill core on the device
// (c/gkda.h:350-539 apus_gkda_chunk): a prompt of s tokens is processed in
// chunks of 64 rows per head, carrying the fp32 state S [D][D] from chunk to
// chunk, instead of stepping the recurrence token by token.
//
// Per head and chunk (rows past s are zero; the in-chunk cumulative gate
// carries the last real row's value into them, as the reference):
//   q, k l2-normalised (numpy pairwise sum of squares, sqrt, divide), q scaled
//   by D^-1/2; gc = in-chunk cumulative sum of g (ascending);
//   attn[i][j<i] = -sum_d (k_i beta_i)_d k_j,d e^(gc_i,d - gc_j,d); the UT
//   transform row by row, then + I;
//   value = attn (v beta); kcd = attn (k beta e^gc);
//   v_new = value - kcd S; inter = (q e^gc) S;
//   intra[i][j<=i] = sum_d q_i,d k_j,d e^(gc_i,d - gc_j,d);
//   out = bf16(inter + intra v_new);
//   S = S e^(gc_last) + sum_j (k_j e^(gc_last - gc_j)) v_new_j.
// Every sum runs in the reference's order (ascending, from +0) and every
// product keeps its operand order, so the only differences from the
// reference are expf's last bits (CUDA's against libm's).
//
// q, k and v rows may be strided (ldx elements apart: the engine's prompt
// pass reads them from its [q | k | v] conv output); g, beta and out are dense.
//
// Layout: CTA (h, p) owns value columns [32p, 32p + 32) of head h, for its
// slice of v, v_new, the outputs and S; the four CTAs of a head each compute
// the chunk's attn / intra / kcd (shared-memory-resident, rows padded by one
// float so a warp's lanes hit distinct banks).  No CTA waits on another.
#include "common.cuh"
#include "gcuda.h"
#include "model_dev.h"
#include "../../include/apus_gcuda.h"

namespace apus {

constexpr int KC_C = 64, KC_D = 128, KC_SPLIT = 4, KC_DV = KC_D / KC_SPLIT, KC_T = 256;
constexpr int KC_PD = KC_D + 1, KC_PV = KC_DV + 1, KC_PC = KC_C + 1;

struct KcSmem {
    float qp[KC_C * KC_PD];      // q normalised and scaled; later q e^gc (rows padded:
    float kp[KC_C * KC_PD];      // k normalised                             read down a column)
    float gc[KC_C * KC_PD];      // in-chunk cumulative gate
    float kx[KC_C * KC_D];       // k beta e^gc, later k e^(gc_last - gc)
    float kcd[KC_C * KC_PD];     // attn (k beta e^gc)
    float attn[KC_C * KC_PC];
    float intra[KC_C * KC_PC];
    float vp[KC_C * KC_PV];      // v beta (this CTA's columns)
    float val[KC_C * KC_PV];     // UT transform row scratch, then value, then v_new
    float S[KC_D * KC_PV];       // this CTA's columns of the state
    float beta[KC_C];
};
static_assert(sizeof(KcSmem) <= 232448, "shared memory");

__global__ void __launch_bounds__(KC_T) k_kda_chunk(const uint16_t *q, const uint16_t *k, const uint16_t *v,
                                                    const float *g, const uint16_t *beta, float *S,
                                                    uint16_t *out, int s, int H, float qscale, long ldx) {
    extern __shared__ __align__(16) unsigned char kc_dyn[];
    KcSmem &sm = *reinterpret_cast<KcSmem *>(kc_dyn);
    const int h = blockIdx.x / KC_SPLIT, c0 = (blockIdx.x % KC_SPLIT) * KC_DV;
    const int tid = threadIdx.x;
    const size_t hd = (size_t)H * KC_D;
    float *Sh = S + (size_t)h * KC_D * KC_D;
    for (int e = tid; e < KC_D * KC_DV; e += KC_T) {
        const int m = e / KC_DV, c = e % KC_DV;
        sm.S[m * KC_PV + c] = Sh[(size_t)m * KC_D + c0 + c];
    }
    const int nch = (s + KC_C - 1) / KC_C;
    for (int n = 0; n < nch; n++) {
        __syncthreads();
        // ---- rows of the chunk (zero past s)
        for (int e = tid; e < KC_C * KC_D; e += KC_T) {
            const int i = e / KC_D, d = e % KC_D, t = n * KC_C + i;
            const bool ok = t < s;
            const size_t off = (size_t)t * hd + (size_t)h * KC_D + d, xo = (size_t)t * ldx + (size_t)h * KC_D + d;
            sm.qp[i * KC_PD + d] = ok ? bf16_f32(q[xo]) : 0.0f;
            sm.kp[i * KC_PD + d] = ok ? bf16_f32(k[xo]) : 0.0f;
            sm.gc[i * KC_PD + d] = ok ? g[off] : 0.0f;
        }
        if (tid < KC_C) {
            const int t = n * KC_C + tid;
            sm.beta[tid] = t < s ? bf16_f32(beta[(size_t)t * H + h]) : 0.0f;
        }
        __syncthreads();
        for (int e = tid; e < KC_C * KC_DV; e += KC_T) {
            const int i = e / KC_DV, c = e % KC_DV, t = n * KC_C + i;
            const float vv = t < s ? bf16_f32(v[(size_t)t * ldx + (size_t)h * KC_D + c0 + c]) : 0.0f;
            sm.vp[i * KC_PV + c] = vv * sm.beta[i];
        }
        // l2 norms (c/gkda.h:263-273): thread r < 2C normalises one real row
        if (tid < 2 * KC_C) {
            const int i = tid % KC_C;
            float *row = (tid < KC_C ? sm.qp : sm.kp) + i * KC_PD;
            if (n * KC_C + i < s) {
                float sq[KC_D];
#pragma unroll 8
                for (int d = 0; d < KC_D; d++) sq[d] = row[d] * row[d];
                const float root = __fsqrt_rn(pw_sum_leaf(sq, KC_D) + 1e-6f);
                for (int d = 0; d < KC_D; d++) row[d] = __fdiv_rn(row[d], root);
                if (tid < KC_C)
                    for (int d = 0; d < KC_D; d++) row[d] = row[d] * qscale;
            }
        }
        // in-chunk cumulative gate, ascending
        if (tid < KC_D)
            for (int i = 1; i < KC_C; i++)
                sm.gc[i * KC_PD + tid] = sm.gc[(i - 1) * KC_PD + tid] + sm.gc[i * KC_PD + tid];
        __syncthreads();
        // ---- attn (strictly lower) and intra (lower with the diagonal), one
        // decay each, over the 2080 lower-triangle pairs; zeros above
        for (int e = tid; e < KC_C * KC_C; e += KC_T) {
            const int i = e / KC_C, j = e % KC_C;
            if (j > i) { sm.attn[i * KC_PC + j] = 0.0f; sm.intra[i * KC_PC + j] = 0.0f; }
        }
        for (int p = tid; p < KC_C * (KC_C + 1) / 2; p += KC_T) {
            int i = (int)((sqrtf(8.0f * (float)p + 1.0f) - 1.0f) * 0.5f);
            while (i * (i + 1) / 2 > p) i--;
            while ((i + 1) * (i + 2) / 2 <= p) i++;
            const int j = p - i * (i + 1) / 2;
            const float bi = sm.beta[i];
            const float *qi = sm.qp + i * KC_PD, *ki = sm.kp + i * KC_PD, *kj = sm.kp + j * KC_PD;
            const float *gi = sm.gc + i * KC_PD, *gj = sm.gc + j * KC_PD;
            float a = 0.0f, b = 0.0f;
            for (int d = 0; d < KC_D; d++) {
                const float dec = expf(gi[d] - gj[d]);
                a += ((ki[d] * bi) * kj[d]) * dec;
                b += (qi[d] * kj[d]) * dec;
            }
            sm.attn[i * KC_PC + j] = j < i ? -a : 0.0f;
            sm.intra[i * KC_PC + j] = b;
        }
        // k beta e^gc for kcd
        for (int e = tid; e < KC_C * KC_D; e += KC_T) {
            const int j = e / KC_D, d = e % KC_D;
            sm.kx[j * KC_D + d] = (sm.kp[j * KC_PD + d] * sm.beta[j]) * expf(sm.gc[j * KC_PD + d]);
        }
        __syncthreads();
        // ---- UT transform: row i += row i . attn[:i, :i], ascending i; the
        // terms m <= j are zero products, so the sum starts at m = j + 1
        for (int i = 1; i < KC_C; i++) {
            if (tid < i) {
                const int j = tid;
                float a = 0.0f;
                for (int m = j + 1; m < i; m++) a += sm.attn[i * KC_PC + m] * sm.attn[m * KC_PC + j];
                sm.val[j] = a;
            }
            __syncthreads();
            if (tid < i) sm.attn[i * KC_PC + tid] = sm.attn[i * KC_PC + tid] + sm.val[tid];
            __syncthreads();
        }
        if (tid < KC_C) sm.attn[tid * KC_PC + tid] = sm.attn[tid * KC_PC + tid] + 1.0f;
        __syncthreads();
        // ---- value = attn (v beta); kcd = attn (k beta e^gc).  Register
        // tiles (each output still sums j = 0, 1, ... in order): value 2 rows
        // x 4 columns a thread, kcd 4 rows x 8 columns (columns 16 apart)
        {
            const int i0 = (tid >> 3) * 2, cb = (tid & 7) * 4;
            float a[2][4] = {};
            for (int j = 0; j < KC_C; j++) {
                const float x0 = sm.attn[i0 * KC_PC + j], x1 = sm.attn[(i0 + 1) * KC_PC + j];
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    const float vv = sm.vp[j * KC_PV + cb + w];
                    a[0][w] += x0 * vv;
                    a[1][w] += x1 * vv;
                }
            }
#pragma unroll
            for (int w = 0; w < 4; w++) { sm.val[i0 * KC_PV + cb + w] = a[0][w]; sm.val[(i0 + 1) * KC_PV + cb + w] = a[1][w]; }
        }
        {
            const int i0 = (tid >> 4) * 4, db = tid & 15;
            float a[4][8] = {};
            for (int j = 0; j < KC_C; j++) {
                float x[4];
#pragma unroll
                for (int u = 0; u < 4; u++) x[u] = sm.attn[(i0 + u) * KC_PC + j];
#pragma unroll
                for (int w = 0; w < 8; w++) {
                    const float kv = sm.kx[j * KC_D + db + 16 * w];
#pragma unroll
                    for (int u = 0; u < 4; u++) a[u][w] += x[u] * kv;
                }
            }
#pragma unroll
            for (int u = 0; u < 4; u++)
#pragma unroll
                for (int w = 0; w < 8; w++) sm.kcd[(i0 + u) * KC_PD + db + 16 * w] = a[u][w];
        }
        __syncthreads();
        // q e^gc (in place) and k e^(gc_last - gc) (over kx)
        for (int e = tid; e < KC_C * KC_D; e += KC_T) {
            const int i = e / KC_D, d = e % KC_D;
            sm.qp[i * KC_PD + d] = sm.qp[i * KC_PD + d] * expf(sm.gc[i * KC_PD + d]);
            sm.kx[i * KC_D + d] = sm.kp[i * KC_PD + d] * expf(sm.gc[(KC_C - 1) * KC_PD + d] - sm.gc[i * KC_PD + d]);
        }
        __syncthreads();
        // ---- v_new = value - kcd S (2 x 4 register tiles, d in order)
        const int i0 = (tid >> 3) * 2, cb = (tid & 7) * 4;
        {
            float a[2][4] = {};
            for (int d = 0; d < KC_D; d++) {
                const float x0 = sm.kcd[i0 * KC_PD + d], x1 = sm.kcd[(i0 + 1) * KC_PD + d];
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    const float sv = sm.S[d * KC_PV + cb + w];
                    a[0][w] += x0 * sv;
                    a[1][w] += x1 * sv;
                }
            }
#pragma unroll
            for (int w = 0; w < 4; w++) {
                sm.val[i0 * KC_PV + cb + w] = sm.val[i0 * KC_PV + cb + w] - a[0][w];
                sm.val[(i0 + 1) * KC_PV + cb + w] = sm.val[(i0 + 1) * KC_PV + cb + w] - a[1][w];
            }
        }
        __syncthreads();
        // ---- out = bf16(inter + intra v_new) for the real rows, inter = (q e^gc) S
        {
            float b[2][4] = {}, a[2][4] = {};
            for (int d = 0; d < KC_D; d++) {
                const float x0 = sm.qp[i0 * KC_PD + d], x1 = sm.qp[(i0 + 1) * KC_PD + d];
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    const float sv = sm.S[d * KC_PV + cb + w];
                    b[0][w] += x0 * sv;
                    b[1][w] += x1 * sv;
                }
            }
            for (int j = 0; j < KC_C; j++) {
                const float x0 = sm.intra[i0 * KC_PC + j], x1 = sm.intra[(i0 + 1) * KC_PC + j];
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    const float vv = sm.val[j * KC_PV + cb + w];
                    a[0][w] += x0 * vv;
                    a[1][w] += x1 * vv;
                }
            }
#pragma unroll
            for (int u = 0; u < 2; u++) {
                const int t = n * KC_C + i0 + u;
                if (t < s)
#pragma unroll
                    for (int w = 0; w < 4; w++)
                        out[(size_t)t * hd + (size_t)h * KC_D + c0 + cb + w] = bf16_bits(b[u][w] + a[u][w]);
            }
        }
        __syncthreads();     // the state update below overwrites S
        // ---- S = S e^(gc_last) + sum_j (k_j e^(gc_last - gc_j)) v_new_j (4 x 4 tiles, j in order)
        {
            const int m0 = (tid >> 3) * 4;
            float a[4][4] = {};
            for (int j = 0; j < KC_C; j++) {
                float kv[4];
#pragma unroll
                for (int u = 0; u < 4; u++) kv[u] = sm.kx[j * KC_D + m0 + u];
#pragma unroll
                for (int w = 0; w < 4; w++) {
                    const float vv = sm.val[j * KC_PV + cb + w];
#pragma unroll
                    for (int u = 0; u < 4; u++) a[u][w] += kv[u] * vv;
                }
            }
#pragma unroll
            for (int u = 0; u < 4; u++) {
                const float egl = expf(sm.gc[(KC_C - 1) * KC_PD + m0 + u]);
#pragma unroll
                for (int w = 0; w < 4; w++)
                    sm.S[(m0 + u) * KC_PV + cb + w] = sm.S[(m0 + u) * KC_PV + cb + w] * egl + a[u][w];
            }
        }
    }
    __syncthreads();
    for (int e = tid; e < KC_D * KC_DV; e += KC_T) {
        const int m = e / KC_DV, c = e % KC_DV;
        Sh[(size_t)m * KC_D + c0 + c] = sm.S[m * KC_PV + c];
    }
}

}  // namespace apus
using namespace apus;

int kda_chunk_launch(const uint16_t *q, const uint16_t *k, const uint16_t *v, const float *g, const uint16_t *beta,
                     float *S, uint16_t *out, int s, int H, int D, cudaStream_t st, long ldx) {
    if (D != KC_D || H < 1 || s < 0) {
        gcuda_set_error("kda_chunk: head dim %d (only %d), %d heads", D, KC_D, H);
        return -1;
    }
    if (s == 0) return 0;
    if (gcuda_smem_limit_once((const void *)k_kda_chunk, (int)sizeof(KcSmem))) return -1;
    const float qscale = (float)pow((double)D, -0.5);
    if (ldx <= 0) ldx = (long)H * KC_D;
    k_kda_chunk<<<H * KC_SPLIT, KC_T, sizeof(KcSmem), st>>>(q, k, v, g, beta, S, out, s, H, qscale, ldx);
    return gcuda_check(cudaGetLastError(), "kda_chunk launch");
}

extern "C" int apus_gcuda_kda_chunk_dev(const uint16_t *q, const uint16_t *k, const uint16_t *v, const float *g,
                                        const uint16_t *beta, float *S, uint16_t *out, size_t s, size_t H,
                                        size_t D, void *stream) {
    if (s > (size_t)1 << 30 || H > 4096) { gcuda_set_error("kda_chunk: %zu rows, %zu heads", s, H); return -1; }
    return kda_chunk_launch(q, k, v, g, beta, S, out, (int)s, (int)H, (int)D, (cudaStream_t)stream, 0);
}
