// linear.cu — FP8 128x128-block dequant and the decode GEMV kernels.
#include "linear.cuh"
#include "gcuda.h"

namespace apus {

// ---------------------------------------------------------------------------
// Standalone dequant (bit-exact with c/fp8blk.h:115-136): one fp32 multiply
// per element, BF16 RNE with NaN pass-through.  Each thread converts 16
// consecutive codes of one row when the row is 16-byte aligned, else one.
__global__ void k_fp8_dequant(const uint8_t *__restrict__ w, const float *__restrict__ ws,
                              uint16_t *__restrict__ out, size_t O, size_t K, size_t nkb,
                              int vec) {
    if (vec) {
        const size_t per_row = K / 16;
        const size_t total = O * per_row;
        for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
             i += (size_t)gridDim.x * blockDim.x) {
            size_t o = i / per_row, k0 = (i % per_row) * 16;
            uint4 c = ld_stream16(w + o * K + k0);
            float s = __ldg(ws + (o / 128) * nkb + k0 / 128);
            uint32_t cw[4] = {c.x, c.y, c.z, c.w};
            uint32_t res[8];
#pragma unroll
            for (int j = 0; j < 4; j++) {
                uint16_t b[4];
#pragma unroll
                for (int q = 0; q < 4; q++)
                    b[q] = bf16_bits(__fmul_rn(e4m3_f32((cw[j] >> (8 * q)) & 0xffu), s));
                res[2 * j] = (uint32_t)b[0] | ((uint32_t)b[1] << 16);
                res[2 * j + 1] = (uint32_t)b[2] | ((uint32_t)b[3] << 16);
            }
            uint4 *dst = reinterpret_cast<uint4 *>(out + o * K + k0);
            dst[0] = make_uint4(res[0], res[1], res[2], res[3]);
            dst[1] = make_uint4(res[4], res[5], res[6], res[7]);
        }
    } else {
        const size_t total = O * K;
        for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total;
             i += (size_t)gridDim.x * blockDim.x) {
            size_t o = i / K, k = i % K;
            float s = __ldg(ws + (o / 128) * nkb + k / 128);
            out[i] = bf16_bits(__fmul_rn(e4m3_f32(w[i]), s));
        }
    }
}

// ---------------------------------------------------------------------------
// Fast GEMV: CTA = 8 warps = RG row groups x KS k-splits; 8*RG weight rows.
template <bool FP8, int RG>
__global__ void __launch_bounds__(256) k_gemv(GemvDesc d) {
    constexpr int KS = 8 / RG;
    __shared__ float part[KS][RG][8][8];
    __shared__ unsigned long long keys[RG * 64];
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int rg = warp % RG, ks = warp / RG;
    const int g = lane >> 2, t = lane & 3;
    const long row_base = (long)blockIdx.x * (8 * RG) + rg * 8;
    const long wrow = min(row_base + g, (long)d.O - 1);
    const int NS = d.K / (FP8 ? 64 : 32);
    const int s0 = (int)((long)NS * ks / KS), s1 = (int)((long)NS * (ks + 1) / KS);
    const size_t row_bytes = FP8 ? (size_t)d.K : (size_t)d.K * 2;
    const uint8_t *wp = (const uint8_t *)d.W + (size_t)wrow * row_bytes + 16 * t;
    const uint16_t *xp = (g < d.R) ? d.x + (size_t)g * d.ldx + (FP8 ? 16 : 8) * t : nullptr;
    const float *srow = FP8 ? d.WS + (size_t)(wrow >> 7) * d.nkb : nullptr;
    float c0, c1;
    warp_rows8<FP8>(wp, xp, srow, s0, s1, c0, c1);
    part[ks][rg][g][2 * t] = c0;
    part[ks][rg][g][2 * t + 1] = c1;
    __syncthreads();
    const int tid = threadIdx.x;
    if (tid < RG * 64) {
        const int rr = tid / 64, m = (tid / 8) % 8, o = tid % 8;
        float acc = part[0][rr][m][o];
#pragma unroll
        for (int q = 1; q < KS; q++) acc = acc + part[q][rr][m][o];
        const long row = (long)blockIdx.x * (8 * RG) + rr * 8 + o;
        const bool ok = (m < d.R) && (row < d.O);
        if (ok) {
            if (d.y) d.y[(size_t)m * d.ldy + row] = bf16_bits(acc);
            if (d.yf) d.yf[(size_t)m * d.ldyf + row] = acc;
        }
        if (d.amax) keys[tid] = ok ? argmax_key(bf16_round(acc), (uint32_t)row) : 0ull;
    }
    if (d.amax) {
        __syncthreads();
        if (tid < d.R) {
            unsigned long long best = 0ull;
            for (int rr = 0; rr < RG; rr++)
                for (int o = 0; o < 8; o++) {
                    unsigned long long k = keys[rr * 64 + tid * 8 + o];
                    best = k > best ? k : best;
                }
            atomicMax(d.amax + tid, best);
        }
    }
}

// Generic GEMV for shapes the fast path cannot stream (K not a multiple of
// the 64-byte step, unaligned rows): one warp per weight row, lanes stride
// k, fixed xor-butterfly reduction.  Same numerics contract.
template <bool FP8>
__global__ void k_gemv_generic(GemvDesc d) {
    const int lane = threadIdx.x & 31;
    const long o = (long)blockIdx.x * (blockDim.x >> 5) + (threadIdx.x >> 5);
    if (o >= d.O) return;
    float acc[8];
#pragma unroll
    for (int r = 0; r < 8; r++) acc[r] = 0.f;
    for (long k = lane; k < d.K; k += 32) {
        float w;
        if (FP8) {
            const uint8_t c = ((const uint8_t *)d.W)[(size_t)o * d.K + k];
            const float s = d.WS[(size_t)(o >> 7) * d.nkb + (k >> 7)];
            w = bf16_round(__fmul_rn(e4m3_f32(c), s));
        } else {
            w = bf16_f32(((const uint16_t *)d.W)[(size_t)o * d.K + k]);
        }
#pragma unroll
        for (int r = 0; r < 8; r++)
            if (r < d.R) acc[r] = acc[r] + w * bf16_f32(d.x[(size_t)r * d.ldx + k]);
    }
#pragma unroll
    for (int r = 0; r < 8; r++)
#pragma unroll
        for (int off = 16; off; off >>= 1) acc[r] = acc[r] + __shfl_xor_sync(0xffffffffu, acc[r], off);
    if (lane < d.R) {
        float v = acc[0];
#pragma unroll
        for (int r = 1; r < 8; r++) if (lane == r) v = acc[r];
        if (d.y) d.y[(size_t)lane * d.ldy + o] = bf16_bits(v);
        if (d.yf) d.yf[(size_t)lane * d.ldyf + o] = v;
        if (d.amax) atomicMax(d.amax + lane, argmax_key(bf16_round(v), (uint32_t)o));
    }
}

__global__ void k_argmax_reset(unsigned long long *keys, int n) {
    if ((int)threadIdx.x < n) keys[threadIdx.x] = 0ull;
}

__global__ void k_argmax_extract(const unsigned long long *keys, int32_t *ids, int n) {
    if ((int)threadIdx.x < n) ids[threadIdx.x] = (int32_t)argmax_key_index(keys[threadIdx.x]);
}

}  // namespace apus

using namespace apus;

bool gemv_fast_ok(const GemvDesc &d) {
    const int kstep = d.fp8 ? 64 : 32;
    if (d.K <= 0 || d.K % kstep) return false;
    if (((uintptr_t)d.W & 15) || ((uintptr_t)d.x & 15)) return false;
    if ((d.ldx * 2) % 16) return false;
    return true;
}

int gemv_launch(const GemvDesc &d, cudaStream_t st) {
    if (d.R < 1 || d.R > 8 || d.O <= 0 || d.K <= 0) return -1;
    if (gemv_fast_ok(d)) {
        constexpr int RG = 2;
        const unsigned grid = (unsigned)((d.O + 8 * RG - 1) / (8 * RG));
        if (d.fp8) k_gemv<true, RG><<<grid, 256, 0, st>>>(d);
        else k_gemv<false, RG><<<grid, 256, 0, st>>>(d);
    } else {
        const unsigned grid = (unsigned)((d.O + 7) / 8);
        if (d.fp8) k_gemv_generic<true><<<grid, 256, 0, st>>>(d);
        else k_gemv_generic<false><<<grid, 256, 0, st>>>(d);
    }
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int fp8_dequant_launch(const uint8_t *w, const float *ws, uint16_t *out, size_t O, size_t K,
                       cudaStream_t st) {
    if (!O || !K) return 0;
    const size_t nkb = (K + 127) / 128;
    const int vec = (K % 16 == 0) && !((uintptr_t)w & 15) && !((uintptr_t)out & 15);
    const size_t items = vec ? O * (K / 16) : O * K;
    size_t blocks = (items + 255) / 256;
    if (blocks > 148 * 32) blocks = 148 * 32;
    k_fp8_dequant<<<(unsigned)blocks, 256, 0, st>>>(w, ws, out, O, K, nkb, vec);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int argmax_reset_launch(unsigned long long *keys, int n, cudaStream_t st) {
    k_argmax_reset<<<1, 32, 0, st>>>(keys, n);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int argmax_extract_launch(const unsigned long long *keys, int32_t *ids, int n, cudaStream_t st) {
    k_argmax_extract<<<1, 32, 0, st>>>(keys, ids, n);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
