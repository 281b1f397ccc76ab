// linear.cuh — decode-shape linear layers (R <= 8 activation rows).
//
// Semantics restated from the apus C engine:
//   FP8 linear (c/gdsa.h:525-534 = c/fp8blk.h dequant + c/bf16.h GEMM):
//     w[o,k]   = bf16_rne(e4m3(W[o,k]) * ws[o/128][k/128])   (one fp32 mul)
//     y[m,o]   = bf16_rne( sum_k f32(x[m,k]) * f32(w[o,k]) )  (fp32 acc)
//   BF16 linear (c/bf16.h:15-60): the same with w = W.
// The dequantized weight keeps the reference's exact BF16 value; only the
// fp32 summation ORDER differs (the reference is strictly sequential in k,
// this kernel reduces 16-wide k groups on the tensor core and combines
// k-split partials in a fixed order).  The order depends on (O, K) only, so
// every activation row gets bitwise the same result at any row count R —
// the batch invariance the speculative verify relies on.
//
// Work decomposition.  A warp owns 8 weight rows and a contiguous range of
// 64-byte k-steps.  Lane (g = lane/4, t = lane%4) reads 16 bytes of weight
// row g per step (FP8: 16 codes, BF16: 8 values) from the shared-memory
// stage the bulk copies filled, converts them into the B fragment of
// mma.m16n8k16.bf16 (the weight rows are the n = 8 columns), and loads the
// matching activation k-values of row g as the A fragment (rows 8..15 of A
// are padding).  The k-permutation inside a step is the same for A and B,
// so the dot products are unchanged.  D[m][n] lands in lane (m, n/2).
#pragma once
#include "common.cuh"

namespace apus {

APUS_DEV uint4 ld_stream16(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.L1::no_allocate.L2::256B.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

APUS_DEV uint4 ld_nc16(const void *p) {
    uint4 r;
    asm volatile("ld.global.nc.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r.x), "=r"(r.y), "=r"(r.z), "=r"(r.w) : "l"(p));
    return r;
}

// Two E4M3 codes (low byte = lower k) -> f16x2, exact.
APUS_DEV uint32_t cvt_e4m3x2_f16x2(uint32_t two_codes) {
    uint32_t r;
    uint16_t in = (uint16_t)two_codes;
    asm("cvt.rn.f16x2.e4m3x2 %0, %1;" : "=r"(r) : "h"(in));
    return r;
}

// Two E4M3 codes -> bf16x2, exact: every E4M3 value (subnormals included)
// is an f16 and a bf16, so the f16 detour rounds nothing.
APUS_DEV uint32_t e4m3x2_bf16x2(uint32_t two_codes);

// (lo, hi) fp32 -> bf16x2 with RNE; lo goes to the low half.
APUS_DEV uint32_t pack_bf16x2(float lo, float hi) {
    uint32_t r;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(r) : "f"(hi), "f"(lo));
    return r;
}

APUS_DEV uint32_t e4m3x2_bf16x2(uint32_t two_codes) {
    const uint32_t h = cvt_e4m3x2_f16x2(two_codes);
    const float2 f = __half22float2(*reinterpret_cast<const __half2 *>(&h));
    return pack_bf16x2(f.x, f.y);
}

// Four E4M3 codes of one 32-bit word times the block scale, each rounded to
// BF16 exactly like c/fp8blk.h:115-136, packed as two bf16x2 words.
APUS_DEV void dequant4(uint32_t w, float s, uint32_t &b0, uint32_t &b1) {
    uint32_t h01 = cvt_e4m3x2_f16x2(w & 0xffffu);
    uint32_t h23 = cvt_e4m3x2_f16x2(w >> 16);
    __half2 v01 = *reinterpret_cast<__half2 *>(&h01);
    __half2 v23 = *reinterpret_cast<__half2 *>(&h23);
    float2 f01 = __half22float2(v01);
    float2 f23 = __half22float2(v23);
    b0 = pack_bf16x2(__fmul_rn(f01.x, s), __fmul_rn(f01.y, s));
    b1 = pack_bf16x2(__fmul_rn(f23.x, s), __fmul_rn(f23.y, s));
}

// Largest BF16 exponent field among 8 packed values.
APUS_DEV int bf16x8_max_exp(uint4 v) {
    const uint32_t w[4] = {v.x, v.y, v.z, v.w};
    int m = 0;
#pragma unroll
    for (int e = 0; e < 4; e++) {
        m = max(m, (int)((w[e] >> 7) & 0xffu));
        m = max(m, (int)((w[e] >> 23) & 0xffu));
    }
    return m;
}

// Staging shift k for a row whose largest BF16 exponent field is E: the
// largest magnitude times 2^k lies in [2^14, 2^15), inside f16's range
// (clamped so 2^k and 2^-k are normal floats).
APUS_DEV int stage_shift(int E) {
    const int k = 141 - E;
    return k > 126 ? 126 : (k < -126 ? -126 : k);
}

APUS_DEV void mma_bf16_16816(float &d0, float &d1, float &d2, float &d3,
                             uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                             uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d0), "+f"(d1), "+f"(d2), "+f"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

APUS_DEV void mma_f16_16816(float &d0, float &d1, float &d2, float &d3,
                            uint32_t a0, uint32_t a1, uint32_t a2, uint32_t a3,
                            uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.f16.f16.f32 "
        "{%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, {%0,%1,%2,%3};"
        : "+f"(d0), "+f"(d1), "+f"(d2), "+f"(d3)
        : "r"(a0), "r"(a1), "r"(a2), "r"(a3), "r"(b0), "r"(b1));
}

// One 64-byte k-step of the staged GEMV for lane (g, t): wv is the lane's
// 16 weight bytes of row g; xw the activation words of row g covering the
// same k range (FP8: 8 words = 16 values, BF16: 4 words = 8 values).
template <bool FP8>
APUS_DEV void gemv_step(const uint4 wv4, const uint32_t *xw, float sc, float &d0, float &d1,
                        float &d2, float &d3) {
    const uint32_t wv[4] = {wv4.x, wv4.y, wv4.z, wv4.w};
    if (FP8) {
#pragma unroll
        for (int j = 0; j < 4; j++) {
            uint32_t b0, b1;
            dequant4(wv[j], sc, b0, b1);
            mma_bf16_16816(d0, d1, d2, d3, xw[2 * j], 0u, xw[2 * j + 1], 0u, b0, b1);
        }
    } else {
#pragma unroll
        for (int j = 0; j < 2; j++)
            mma_bf16_16816(d0, d1, d2, d3, xw[2 * j], 0u, xw[2 * j + 1], 0u, wv[2 * j], wv[2 * j + 1]);
    }
}

}  // namespace apus
