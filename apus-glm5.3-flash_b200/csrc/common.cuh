// common.cuh — shared device numerics for the apus B200 engine (sm_100a).
//
// Every helper here restates a scalar rule of the apus C engine so the CUDA
// kernels keep the same rounding points:
//   * BF16 narrow: round-to-nearest-even through the 0x7FFF + lsb bias, NaN
//     passed through as its high 16 bits (c/num.h:143-160).
//   * BF16 widen: exact, bits << 16 (c/num.h:162-166).
//   * E4M3 decode: exact; the NaN codes 0x7F/0xFF decode as +-480 like a
//     normal e=15, m=7 (c/num.h:136-141).
//   * numpy-stable sigmoid: e = expf(-|x|); x >= 0 ? 1/(1+e) : e/(1+e)
//     (c/gmhc.h:157-160).
//   * numpy pairwise float32 summation order (c/gmhc.h:165-185).
// The library is compiled with -fmad=false, so a*b+c is two roundings like
// the reference's -ffp-contract=off build.
#pragma once

#include <cuda_runtime.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <stdint.h>

#define APUS_DEV __device__ __forceinline__

namespace apus {

APUS_DEV float bf16_f32(uint16_t b) { return __uint_as_float((uint32_t)b << 16); }

APUS_DEV uint16_t bf16_bits(float x) {
    uint32_t u = __float_as_uint(x);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)(u >> 16);
    u += 0x7FFFu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

APUS_DEV float bf16_round(float x) { return bf16_f32(bf16_bits(x)); }

// Exact E4M3 decode (normals: (8+m)*2^(e-10); subnormals: m*2^-9).
APUS_DEV float e4m3_f32(uint32_t c) {
    uint32_t e = (c >> 3) & 15u, m = c & 7u;
    float v;
    if (e) v = __uint_as_float(((e + 120u) << 23) | (m << 20));
    else   v = (float)m * 0.001953125f;  // 2^-9, exact
    return (c & 0x80u) ? -v : v;
}

APUS_DEV float sigmoid_np(float x) {
    float e = expf(-fabsf(x));
    return x >= 0.0f ? 1.0f / (1.0f + e) : e / (1.0f + e);
}

// Programmatic dependent launch: a kernel lets the next one in the stream
// start early (the next one waits with pdl_wait before it reads anything
// this kernel writes); a no-op when the next kernel was launched without the
// programmatic-serialization attribute.
APUS_DEV void pdl_launch_dependents() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }
APUS_DEV void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }

// Widen a packed bf16x2 word: low half is the lower k index.
APUS_DEV float bf16lo(uint32_t w) { return __uint_as_float(w << 16); }
APUS_DEV float bf16hi(uint32_t w) { return __uint_as_float(w & 0xffff0000u); }

// numpy pairwise sum of a contiguous float array held in shared memory, for
// n <= 128: 8 accumulators unrolled, tree combine, sequential remainder.
// Serial (one thread); used only on short rows.
APUS_DEV float pw_sum_leaf(const float *a, int n) {
    if (n < 8) {
        float r = a[0];
        for (int i = 1; i < n; i++) r += a[i];
        return r;
    }
    float r[8];
#pragma unroll
    for (int j = 0; j < 8; j++) r[j] = a[j];
    int i = 8;
    for (; i + 8 <= n; i += 8) {
#pragma unroll
        for (int j = 0; j < 8; j++) r[j] += a[i + j];
    }
    float res = ((r[0] + r[1]) + (r[2] + r[3])) + ((r[4] + r[5]) + (r[6] + r[7]));
    for (; i < n; i++) res += a[i];
    return res;
}

// Block-wide numpy pairwise sum of a shared-memory array a[0..n).
// The numpy recursion splits n into (n/2)&~7 and the rest until a piece is
// <= 128 long; leaves are summed by one thread each, the tree is combined
// in the recursion's order. `work` needs room for the leaf results (n/64+2
// floats). All threads of the block must call it; returns the sum to all.
// Leaf enumeration is an explicit stack walk done by thread 0 (the leaf
// count is small: <= 2*n/128 + 1).
struct PwLeaf { int off, len; };

APUS_DEV int pw_collect_leaves(int n, PwLeaf *leaves) {
    // iterative DFS producing leaves in left-to-right order
    int stk_off[32], stk_len[32], sp = 0, nl = 0;
    stk_off[sp] = 0; stk_len[sp] = n; sp++;
    while (sp) {
        sp--;
        int off = stk_off[sp], len = stk_len[sp];
        if (len <= 128) { leaves[nl].off = off; leaves[nl].len = len; nl++; continue; }
        int n2 = (len / 2) & ~7;
        // push right then left so left is processed first
        stk_off[sp] = off + n2; stk_len[sp] = len - n2; sp++;
        stk_off[sp] = off; stk_len[sp] = n2; sp++;
    }
    return nl;
}

// Combine leaf sums following the recursion tree (same split rule).
APUS_DEV float pw_combine(const float *leafsum, int n, int *cursor) {
    // recursive definition expressed with an explicit stack of frames
    struct Fr { int len; int state; float left; };
    Fr st[32];
    int sp = 0;
    st[sp++] = {n, 0, 0.0f};
    float ret = 0.0f;
    while (sp) {
        Fr &f = st[sp - 1];
        if (f.len <= 128) { ret = leafsum[(*cursor)++]; sp--; continue; }
        int n2 = (f.len / 2) & ~7;
        if (f.state == 0) { f.state = 1; st[sp++] = {n2, 0, 0.0f}; continue; }
        if (f.state == 1) { f.left = ret; f.state = 2; st[sp++] = {f.len - n2, 0, 0.0f}; continue; }
        ret = f.left + ret; sp--;
    }
    return ret;
}

// Pairwise sum over shared memory a[0..n) by the whole block. n <= 65536.
// scratch: >= 2*(n/128)+2 floats + same count of PwLeaf in smem.
APUS_DEV float block_pw_sum(const float *a, int n, float *leafsum, PwLeaf *leaves,
                            int *nleaves_sh, float *result_sh) {
    if (threadIdx.x == 0) *nleaves_sh = pw_collect_leaves(n, leaves);
    __syncthreads();
    int nl = *nleaves_sh;
    for (int i = threadIdx.x; i < nl; i += blockDim.x)
        leafsum[i] = pw_sum_leaf(a + leaves[i].off, leaves[i].len);
    __syncthreads();
    if (threadIdx.x == 0) { int cur = 0; *result_sh = pw_combine(leafsum, n, &cur); }
    __syncthreads();
    float r = *result_sh;
    __syncthreads();
    return r;
}

// Order-preserving 32-bit key of a float (larger float -> larger key).
APUS_DEV uint32_t f32_order_key(float v) {
    uint32_t u = __float_as_uint(v);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}

// argmax key: value major, LOWER index wins ties (c/sample.h:76-81).
// -0 and +0 compare equal in the reference's comparisons, so both take the
// key of +0 and the index decides.
APUS_DEV unsigned long long argmax_key(float v, uint32_t idx) {
    if (__float_as_uint(v) == 0x80000000u) v = 0.0f;
    return ((unsigned long long)f32_order_key(v) << 32) | (unsigned long long)(0xFFFFFFFFu - idx);
}
APUS_DEV uint32_t argmax_key_index(unsigned long long k) {
    return 0xFFFFFFFFu - (uint32_t)(k & 0xFFFFFFFFull);
}

}  // namespace apus
