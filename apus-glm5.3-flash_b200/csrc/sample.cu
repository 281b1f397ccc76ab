// sample.cu — temperature / top-p sampling of BF16 logits rows on the device
// (c/sample.h:91-177: apus_sample_logits_u, apus_sample_top_p_u, splitmix64).
//
// The reference widens a BF16 logits row, takes p_i = expf((l_i - mx)/temp),
// q_i = (float)(p_i / sum), sorts q descending (ties: lower index first),
// keeps the prefix whose cumulative mass before each token is <= top_p, and
// draws the first sorted token whose renormalised CDF exceeds u.
//
// One cluster of SMP_C CTAs handles one row.  Because the logits are BF16, q
// depends on the 16-bit code alone, so the row never has to be sorted:
//   * each CTA counts its slice of the row in a 65,536-bin histogram of
//     16-bit counters over the order-preserving key of each logit; CTA c
//     then owns keys [c*8192, (c+1)*8192) and sums the cluster's counts for
//     them through DSMEM;
//   * per occupied bin: p, then q, and the bin's mass count * q;
//   * the cumulative mass of the sorted order at any point is then a scan of
//     bins from the highest key down, and a crossing "the first sorted token
//     whose cumulative mass exceeds X" is found by a scan over the CTAs'
//     totals, a scan inside the crossing CTA, and, inside the tie group of
//     equal q, the t-th element in index order.
// Arithmetic (bitwise restated by the oracle's exact sampler):
//   z = (l - mx) / temp in fp32 (IEEE, like the reference);
//   p = (float)exp_cw(z) with exp_cw below, a Cody-Waite reduction by ln 2
//     and the degree-13 Taylor polynomial in double (within a few double
//     ulps of e^z, so p is the correctly rounded e^z but for ~1e-8 of
//     inputs; glibc's expf is within 0.502 ulp);
//   sum = the exact sum of count * p at 2^-100 resolution, rounded once to
//     double (the reference adds the p_i sequentially in double);
//   q = (float)((double)p / sum), as the reference;
//   every cumulative mass is exact in integers of 2^-62 (the reference adds
//     doubles in sorted order); keep while cum_before <= top_p; draw the first
//     token with cum > u * kept (the reference: cum/kept > u, summed per token).
// So the token equals the reference's unless u * kept or top_p falls within
// about 1e-7 of a boundary of the cumulative mass.
#include <cooperative_groups.h>

#include "common.cuh"
#include "gcuda.h"
#include "model_dev.h"
#include "../../include/apus_gcuda.h"

namespace cg = cooperative_groups;

namespace apus {

constexpr int SMP_C = 8;                 // CTAs per row (one cluster)
constexpr int SMP_T = 256;               // threads per CTA
constexpr int SMP_NB = 65536 / SMP_C;    // key bins owned by one CTA
constexpr int SMP_BPT = SMP_NB / SMP_T;  // bins per thread
constexpr int SMP_W = SMP_T / 32;

typedef unsigned __int128 u128;
typedef unsigned long long u64;

// ---- exact arithmetic shared with the oracle's restatement ------------------

// e^z for z in [-105, 0]: z = k ln2 + r with k = rint(z / ln2), ln2 split
// into a 32-bit head (k * head exact) and a tail; e^r by Horner on the
// Taylor coefficients 1/n!, n <= 13 (|r| <= 0.347: truncation < 2^-57).
// Every operation is one IEEE double rounding (no contraction), so the
// oracle's C restatement computes the same bits.
__device__ double exp_cw(double z) {
    const double inv_ln2 = 0x1.71547652b82fep+0, ln2_hi = 0x1.62e42fee00000p-1, ln2_lo = 0x1.a39ef35793c76p-33;
    const double k = rint(__dmul_rn(z, inv_ln2));
    const double r = __dsub_rn(__dsub_rn(z, __dmul_rn(k, ln2_hi)), __dmul_rn(k, ln2_lo));
    const double c[14] = {1.0, 1.0, 0x1.0p-1, 0x1.5555555555555p-3, 0x1.5555555555555p-5, 0x1.1111111111111p-7,
                          0x1.6c16c16c16c17p-10, 0x1.a01a01a01a01ap-13, 0x1.a01a01a01a01ap-16,
                          0x1.71de3a556c734p-19, 0x1.27e4fb7789f5cp-22, 0x1.ae64567f544e4p-26,
                          0x1.1eed8eff8d898p-29, 0x1.6124613a86d09p-33};
    double e = c[13];
#pragma unroll
    for (int n = 12; n >= 0; n--) e = __dadd_rn(__dmul_rn(e, r), c[n]);
    const long long kb = (long long)k + 1023;          // k in [-152, 0]: a normal double
    return __dmul_rn(e, __longlong_as_double(kb << 52));
}

// p = e^((l - mx) / temp) rounded to float (0 below e^-105 < 2^-150).
APUS_DEV float smp_p(float l, float mx, float temp) {
    const float z = __fdiv_rn(__fsub_rn(l, mx), temp);
    if (!(z >= -105.0f)) return 0.0f;
    return __double2float_rn(exp_cw((double)z));
}

// floor(v * 2^s) of a non-negative float (exact shifts of its integer mantissa).
APUS_DEV u64 fix62(float v) {
    const uint32_t b = __float_as_uint(v), e = b >> 23;
    u64 M = b & 0x7FFFFFu;
    int E = -149;
    if (e) { M |= 0x800000u; E = (int)e - 150; }
    const int s = E + 62;
    return s >= 0 ? M << s : (s > -64 ? M >> -s : 0ull);
}
APUS_DEV u128 fix100(float v) {
    const uint32_t b = __float_as_uint(v), e = b >> 23;
    u64 M = b & 0x7FFFFFu;
    int E = -149;
    if (e) { M |= 0x800000u; E = (int)e - 150; }
    const int s = E + 100;
    return s >= 0 ? (u128)M << s : (u128)(s > -64 ? M >> -s : 0ull);
}

// x * 2^-100 rounded to the nearest double (ties to even).
APUS_DEV double u128_scaled_rn(u128 x) {
    const u64 hi = (u64)(x >> 64), lo = (u64)x;
    if (!hi && lo < (1ull << 53)) return __dmul_rn((double)lo, 0x1.0p-100);
    const int nb = hi ? 128 - __clzll(hi) : 64 - __clzll(lo);
    const int sh = nb - 53;
    u128 mant = x >> sh;
    const u128 rem = x - (mant << sh), half = (u128)1 << (sh - 1);
    if (rem > half || (rem == half && (mant & 1))) mant += 1;
    // mant <= 2^53 and sh - 100 in [-47, 28]: one exact power-of-two scaling
    return __dmul_rn((double)(u64)mant, __longlong_as_double((long long)(sh - 100 + 1023) << 52));
}

// splitmix64 (c/sample.h:159-170): the n-th draw after state s (n >= 1) is
// mix(s + n * golden); a uniform is its top 53 bits.
APUS_DEV u64 smp_mix(u64 z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

APUS_DEV uint32_t bf16_okey(uint16_t b) {
    return (b & 0x8000u) ? (uint32_t)(~b & 0xFFFFu) : (uint32_t)(b | 0x8000u);
}
APUS_DEV uint16_t okey_bf16(uint32_t k) {
    return (k & 0x8000u) ? (uint16_t)(k & 0x7FFFu) : (uint16_t)(~k & 0xFFFFu);
}

// ---- block collectives ----------------------------------------------------------

APUS_DEV u64 warp_sum64(u64 v) {
#pragma unroll
    for (int o = 16; o; o >>= 1) v += __shfl_down_sync(0xffffffffu, v, o);
    return v;
}

// Every thread gets the block sum (wsh: SMP_W slots).
APUS_DEV u64 block_sum64(u64 v, u64 *wsh) {
    v = warp_sum64(v);
    __syncthreads();
    if ((threadIdx.x & 31) == 0) wsh[threadIdx.x >> 5] = v;
    __syncthreads();
    u64 s = 0;
#pragma unroll
    for (int w = 0; w < SMP_W; w++) s += wsh[w];
    return s;
}

APUS_DEV u128 block_sum128(u128 v, u128 *wsh) {
#pragma unroll
    for (int o = 16; o; o >>= 1) {
        const u64 lo = __shfl_down_sync(0xffffffffu, (u64)v, o);
        const u64 hi = __shfl_down_sync(0xffffffffu, (u64)(v >> 64), o);
        v += ((u128)hi << 64) | lo;
    }
    __syncthreads();
    if ((threadIdx.x & 31) == 0) wsh[threadIdx.x >> 5] = v;
    __syncthreads();
    u128 s = 0;
#pragma unroll
    for (int w = 0; w < SMP_W; w++) s += wsh[w];
    return s;
}

// Values one CTA publishes to the others of its cluster (read through
// DSMEM after the cluster barrier that follows the write).  Each field is
// written once per launch, so no write can race a read of an older value.
struct SmpPub {
    u128 sum;                 // exact sum of count * p over the owned bins (2^-100 units)
    u64 mass;                 // sum of count * q over the owned bins (2^-62 units)
    u64 above[2];             // per crossing: mass of the owned bins with q > q*
    uint32_t maxkey;          // largest key of the CTA's elements
    float qstar[2];           // per crossing: q of the crossing bin (written by its finder)
    uint32_t ties[2], klo[2], khi[2];
    uint32_t cnt;             // elements of the tie group in the CTA's slice
};

constexpr int SMP_SEG = SMP_NB / 32;     // 32-bin segments of the owned bins (one per thread)
static_assert(SMP_SEG == SMP_T && SMP_W >= SMP_C, "segment / gather layout");

struct SmpShared {
    SmpPub pub;
    u128 w128[SMP_W];
    u64 w64[SMP_W];
    u64 seg[SMP_SEG];         // mass of each segment (2^-62 units)
    u64 mass[SMP_C];          // every CTA's mass
    u64 gath[SMP_C];
    uint32_t gath32[3][SMP_C];
    u64 gA;
    uint32_t gties, gklo, gkhi, gcnt[SMP_C];
    uint32_t wcnt[SMP_W];
    double S;
    float mx;
    uint32_t maxkey;
};

// Elements per CTA: ceil(V / SMP_C) rounded up to 8, so every slice starts
// on a 16-byte boundary of the row.
__host__ __device__ inline int smp_slice(int V) { return (((V + SMP_C - 1) / SMP_C) + 7) & ~7; }

struct SampleArgs {
    const uint16_t *logits;   // [rows][ld] BF16 codes
    long ld;
    int V, rows;
    float temp, top_p;
    const u64 *rng_dev;       // stream state before the draws (device), or null: rng_val
    u64 rng_val;
    int *out;                 // [rows]
};

// Crossing search for X: the first token of the sorted order whose
// cumulative mass exceeds X.  Returns false (uniformly over the cluster)
// when the whole row's mass is <= X; otherwise leaves in sh the mass of
// every token above the crossing token's tie group (gA), the group's size
// (gties) and key range [gklo, gkhi], and returns its q's mass unit.
__device__ bool smp_cross(cg::cluster_group &cl, int cr, SmpShared &sh, const uint32_t *hist, const float *qb,
                          u64 X, int which, u64 *fstar) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    u64 above = 0;
    int cc = -1;
    for (int c = SMP_C - 1; c >= 0; c--) {
        if (above + sh.mass[c] > X) { cc = c; break; }
        above += sh.mass[c];
    }
    if (cc < 0) return false;
    if (cr == cc) {
        // thread t holds segment t; suffix sums give the mass above it
        const u64 m = sh.seg[tid];
        u64 s = m;
#pragma unroll
        for (int o = 1; o < 32; o <<= 1) {
            const u64 v = __shfl_down_sync(0xffffffffu, s, o);
            if (lane + o < 32) s += v;
        }
        __syncthreads();
        if (lane == 0) sh.w64[w] = s;
        __syncthreads();
        u64 pre = above + (s - m);
        for (int w2 = w + 1; w2 < SMP_W; w2++) pre += sh.w64[w2];
        if (pre <= X && X < pre + m) {
            for (int b = tid * 32 + 31; b >= tid * 32; b--) {
                const uint32_t n = hist[b];
                if (!n) continue;
                const u64 wgt = (u64)n * fix62(qb[b]);
                if (pre + wgt > X) {
                    const float q = qb[b];
                    for (int c = 0; c < SMP_C; c++) cl.map_shared_rank(&sh.pub, c)->qstar[which] = q;
                    break;
                }
                pre += wgt;
            }
        }
    }
    cl.sync();
    const float qs = sh.pub.qstar[which];
    // the tie group of q*: a contiguous key range (q is monotone in the key)
    u64 a = 0;
    uint32_t nt = 0, klo = 0xFFFFFFFFu, khi = 0;
    for (int b = tid; b < SMP_NB; b += SMP_T) {
        const uint32_t n = hist[b];
        if (!n) continue;
        const float q = qb[b];
        if (q > qs) a += (u64)n * fix62(q);
        else if (q == qs) {
            nt += n;
            const uint32_t k = (uint32_t)(cr * SMP_NB + b);
            klo = min(klo, k);
            khi = max(khi, k);
        }
    }
    a = block_sum64(a, sh.w64);
    nt = (uint32_t)block_sum64(nt, sh.w64);
    klo = __reduce_min_sync(0xffffffffu, klo);
    khi = __reduce_max_sync(0xffffffffu, khi);
    __syncthreads();
    if (lane == 0) { sh.wcnt[w] = klo; sh.w64[w] = khi; }
    __syncthreads();
    if (tid == 0) {
        for (int w2 = 0; w2 < SMP_W; w2++) { klo = min(klo, sh.wcnt[w2]); khi = max(khi, (uint32_t)sh.w64[w2]); }
        sh.pub.above[which] = a;
        sh.pub.ties[which] = nt;
        sh.pub.klo[which] = klo;
        sh.pub.khi[which] = khi;
    }
    cl.sync();
    if (tid < SMP_C) {
        const SmpPub *rp = cl.map_shared_rank(&sh.pub, tid);
        sh.gath[tid] = rp->above[which];
        sh.gath32[0][tid] = rp->ties[which];
        sh.gath32[1][tid] = rp->klo[which];
        sh.gath32[2][tid] = rp->khi[which];
    }
    __syncthreads();
    if (tid == 0) {
        u64 A = 0;
        uint32_t T = 0, lo = 0xFFFFFFFFu, hi = 0;
        for (int c = 0; c < SMP_C; c++) {
            A += sh.gath[c];
            T += sh.gath32[0][c];
            lo = min(lo, sh.gath32[1][c]);
            hi = max(hi, sh.gath32[2][c]);
        }
        sh.gA = A; sh.gties = T; sh.gklo = lo; sh.gkhi = hi;
    }
    __syncthreads();
    *fstar = fix62(qs);
    return true;
}

// The t-th element (index order) whose key lies in [klo, khi]; written to
// *out by the thread that finds it.
__device__ void smp_locate(cg::cluster_group &cl, int cr, SmpShared &sh, const uint16_t *keys, int n_loc, int lo,
                           uint32_t klo, uint32_t khi, uint32_t t, int *out) {
    const int tid = threadIdx.x, lane = tid & 31, w = tid >> 5;
    const int per = (n_loc + SMP_T - 1) / SMP_T;
    const int a = min(tid * per, n_loc), b = min(a + per, n_loc);
    uint32_t n = 0;
    for (int i = a; i < b; i++) {
        const uint32_t k = keys[i];
        n += (k >= klo && k <= khi);
    }
    uint32_t s = n;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint32_t v = __shfl_up_sync(0xffffffffu, s, o);
        if (lane >= o) s += v;
    }
    __syncthreads();
    if (lane == 31) sh.wcnt[w] = s;
    __syncthreads();
    uint32_t pre = s - n, tot = 0;
    for (int w2 = 0; w2 < SMP_W; w2++) {
        if (w2 < w) pre += sh.wcnt[w2];
        tot += sh.wcnt[w2];
    }
    if (tid == 0) sh.pub.cnt = tot;
    cl.sync();
    if (tid < SMP_C) sh.gcnt[tid] = cl.map_shared_rank(&sh.pub, tid)->cnt;
    __syncthreads();
    uint32_t base = 0;
    for (int c = 0; c < cr; c++) base += sh.gcnt[c];
    if (t >= base && t < base + tot && t - base >= pre && t - base < pre + n) {
        uint32_t j = t - base - pre;
        for (int i = a; i < b; i++) {
            const uint32_t k = keys[i];
            if (k >= klo && k <= khi) {
                if (j == 0) { *out = lo + i; break; }
                j--;
            }
        }
    }
}

constexpr int SMP_LH = 65536 / 2;        // words of the packed 16-bit local histogram

__global__ void __cluster_dims__(SMP_C, 1, 1) __launch_bounds__(SMP_T) k_sample(SampleArgs d) {
    cg::cluster_group cl = cg::this_cluster();
    const int cr = (int)cl.block_rank();
    const int row = blockIdx.x / SMP_C;
    const int tid = threadIdx.x, lane = tid & 31;
    extern __shared__ __align__(16) unsigned char smp_dyn[];
    uint32_t *lh = (uint32_t *)smp_dyn;                // [SMP_LH] 16-bit counts of every key over this CTA's slice
    float *qb = (float *)smp_dyn;                      // [SMP_NB] p, then q, of the owned keys (over lh once merged)
    uint32_t *hist = lh + SMP_LH;                      // [SMP_NB] counts of the owned keys over the row
    uint16_t *keys = (uint16_t *)(hist + SMP_NB);      // [n_loc] keys of this CTA's slice
    __shared__ SmpShared sh;
    const bool smp = d.temp > 0.0f;

    const int SL = smp_slice(d.V);
    const int lo = min(cr * SL, d.V), hi = min(lo + SL, d.V), n_loc = hi - lo;
    const uint16_t *lg = d.logits + (size_t)row * d.ld;
    const bool vec = ((((uintptr_t)lg) | ((uintptr_t)lo * 2)) & 15) == 0;

    if (smp)
        for (int i = tid; i < SMP_LH / 4; i += SMP_T) ((uint4 *)lh)[i] = make_uint4(0u, 0u, 0u, 0u);
    __syncthreads();

    // keys, the slice's histogram (a shared-memory atomic per element: the
    // hardware merges a warp's equal addresses faster than a match + popc
    // aggregation) and its largest key; 8 consecutive elements per thread
    // (one 16-byte load where aligned).  A slice holds < 65536 elements, so
    // the 16-bit counts cannot carry.
    uint32_t mk = 0;
    for (int i0 = 0; i0 < n_loc; i0 += SMP_T * 8) {
        const int i = i0 + tid * 8;
        uint32_t k[8];
        if (vec && i + 8 <= n_loc) {
            const uint4 v = *(const uint4 *)(lg + lo + i);
            const uint32_t wv[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
            for (int j = 0; j < 4; j++) {
                k[2 * j] = bf16_okey((uint16_t)(wv[j] & 0xFFFFu));
                k[2 * j + 1] = bf16_okey((uint16_t)(wv[j] >> 16));
            }
        } else {
#pragma unroll
            for (int j = 0; j < 8; j++) k[j] = i + j < n_loc ? bf16_okey(lg[lo + i + j]) : 0xFFFFFFFFu;
        }
#pragma unroll
        for (int j = 0; j < 8; j++) {
            const bool ok = i + j < n_loc;
            if (ok) { keys[i + j] = (uint16_t)k[j]; mk = max(mk, k[j]); }
            if (smp && ok) atomicAdd(lh + (k[j] >> 1), 1u << ((k[j] & 1u) * 16));
        }
    }
    mk = __reduce_max_sync(0xffffffffu, mk);
    if (lane == 0) sh.wcnt[tid >> 5] = mk;
    __syncthreads();
    if (tid == 0) {
        for (int w = 0; w < SMP_W; w++) mk = max(mk, sh.wcnt[w]);
        sh.pub.maxkey = mk;
    }
    cl.sync();
    if (tid < SMP_C) sh.gath32[0][tid] = cl.map_shared_rank(&sh.pub, tid)->maxkey;
    __syncthreads();
    if (tid == 0) {
        uint32_t g = 0;
        for (int c = 0; c < SMP_C; c++) g = max(g, sh.gath32[0][c]);
        sh.maxkey = g;
        sh.mx = bf16_f32(okey_bf16(g));
    }
    __syncthreads();

    if (!smp) {
        // greedy (c/sample.h:76-81, 134): the lowest index holding the max
        // value (-0 and +0, keys 0x7FFF and 0x8000, are one value)
        smp_locate(cl, cr, sh, keys, n_loc, lo, sh.maxkey == 0x8000u ? 0x7FFFu : sh.maxkey, sh.maxkey, 0,
                   d.out + row);
        cl.sync();
        return;
    }

    // the owned keys' counts over the whole row: the cluster's slice
    // histograms summed through DSMEM, 8 keys per 16-byte load
    for (int v = tid; v < SMP_NB / 8; v += SMP_T) {
        uint32_t c[8] = {0, 0, 0, 0, 0, 0, 0, 0};
#pragma unroll
        for (int s = 0; s < SMP_C; s++) {
            const uint4 wv = ((const uint4 *)cl.map_shared_rank(lh, s))[cr * (SMP_NB / 8) + v];
            c[0] += wv.x & 0xFFFFu; c[1] += wv.x >> 16;
            c[2] += wv.y & 0xFFFFu; c[3] += wv.y >> 16;
            c[4] += wv.z & 0xFFFFu; c[5] += wv.z >> 16;
            c[6] += wv.w & 0xFFFFu; c[7] += wv.w >> 16;
        }
        ((uint4 *)hist)[2 * v] = make_uint4(c[0], c[1], c[2], c[3]);
        ((uint4 *)hist)[2 * v + 1] = make_uint4(c[4], c[5], c[6], c[7]);
    }
    cl.sync();    // every slice histogram has been read: its space now holds qb

    // p per occupied bin and the exact sum of count * p
    const float mx = sh.mx, temp = d.temp;
    u128 acc = 0;
    for (int b = tid; b < SMP_NB; b += SMP_T) {
        const uint32_t n = hist[b];
        if (!n) continue;
        const float p = smp_p(bf16_f32(okey_bf16((uint32_t)(cr * SMP_NB + b))), mx, temp);
        qb[b] = p;
        acc += (u128)n * fix100(p);
    }
    acc = block_sum128(acc, sh.w128);
    if (tid == 0) sh.pub.sum = acc;
    cl.sync();
    if (tid < SMP_C) sh.w128[tid] = cl.map_shared_rank(&sh.pub, tid)->sum;
    __syncthreads();
    if (tid == 0) {
        u128 tot = 0;
        for (int c = 0; c < SMP_C; c++) tot += sh.w128[c];
        sh.S = u128_scaled_rn(tot);
    }
    __syncthreads();
    const double S = sh.S;
    for (int b = tid; b < SMP_NB; b += SMP_T) {
        const uint32_t n = hist[b];
        if (n) qb[b] = __double2float_rn(__ddiv_rn((double)qb[b], S));
    }
    __syncthreads();
    // segment masses: thread t sums segment t, starting at bin t mod 32 of
    // it so that a warp's lanes read 32 different banks
    {
        u64 m = 0;
        for (int j = 0; j < 32; j++) {
            const int b = tid * 32 + ((j + tid) & 31);
            const uint32_t n = hist[b];
            if (n) m += (u64)n * fix62(qb[b]);
        }
        sh.seg[tid] = m;
    }
    __syncthreads();
    const u64 ms = block_sum64(sh.seg[tid], sh.w64);
    if (tid == 0) sh.pub.mass = ms;
    cl.sync();
    if (tid < SMP_C) sh.mass[tid] = cl.map_shared_rank(&sh.pub, tid)->mass;
    __syncthreads();

    // nucleus (c/sample.h:114-127): kept = cumulative mass through the first
    // sorted token whose cumulative mass exceeds top_p (all when none does)
    const float tp = d.top_p;
    const u64 TP = !(tp >= 0.0f) ? 0ull : (tp >= 4.0f ? ~0ull : __double2ull_rz(__dmul_rn((double)tp, 0x1.0p62)));
    u64 kept = 0;
    for (int c = 0; c < SMP_C; c++) kept += sh.mass[c];
    u64 fs;
    if (smp_cross(cl, cr, sh, hist, qb, TP, 0, &fs)) {
        u64 t = (TP - sh.gA) / fs;
        if (t >= sh.gties) t = sh.gties - 1;
        kept = sh.gA + (t + 1) * fs;
    }

    // draw (c/sample.h:128-131): the first sorted token with cum > u * kept
    const u64 s0 = d.rng_dev ? *d.rng_dev : d.rng_val;
    const u64 m53 = smp_mix(s0 + (u64)(row + 1) * 0x9E3779B97F4A7C15ull) >> 11;
    const u128 prod = (u128)m53 * kept;
    const u64 X = (u64)(prod >> 53);
    if (smp_cross(cl, cr, sh, hist, qb, X, 1, &fs)) {
        u64 t = (X - sh.gA) / fs;
        if (t >= sh.gties) t = sh.gties - 1;
        smp_locate(cl, cr, sh, keys, n_loc, lo, sh.gklo, sh.gkhi, (uint32_t)t, d.out + row);
    } else {    // unreachable (X < kept <= the row's mass): the top token
        smp_locate(cl, cr, sh, keys, n_loc, lo, sh.maxkey == 0x8000u ? 0x7FFFu : sh.maxkey, sh.maxkey, 0,
                   d.out + row);
    }
    cl.sync();    // no CTA leaves while another may still read its shared memory
}

constexpr int SMP_VMAX = SMP_C * 32000;   // slice keys + 160 KiB of histograms fit 227 KiB

}  // namespace apus
using namespace apus;

// Dynamic shared memory of one CTA for a vocabulary of V.
static size_t sample_smem(int V) { return (size_t)(SMP_LH + SMP_NB) * 4 + (size_t)smp_slice(V) * 2; }

int sample_prepare(int V) {
    if (V < 1 || V > SMP_VMAX) {
        gcuda_set_error("sample: vocabulary %d outside [1, %d]", V, SMP_VMAX);
        return -1;
    }
    return gcuda_check(cudaFuncSetAttribute(k_sample, cudaFuncAttributeMaxDynamicSharedMemorySize,
                                            (int)sample_smem(SMP_VMAX)), "sample smem");
}

int sample_launch(const uint16_t *logits, long ld, int V, int rows, float temp, float top_p, const u64 *rng_dev,
                  u64 rng_val, int *out, cudaStream_t st) {
    if (rows <= 0) return 0;
    if (V < 1 || V > SMP_VMAX) {
        gcuda_set_error("sample: vocabulary %d outside [1, %d]", V, SMP_VMAX);
        return -1;
    }
    SampleArgs a{logits, ld, V, rows, temp, top_p, rng_dev, rng_val, out};
    k_sample<<<rows * SMP_C, SMP_T, sample_smem(V), st>>>(a);
    return gcuda_check(cudaGetLastError(), "sample launch");
}

extern "C" {

int apus_gcuda_sample_rows_dev(const uint16_t *logits, size_t rows, size_t ld, size_t n, float temp,
                               float top_p, uint64_t rng_state, int32_t *out, void *stream) {
    if (n < 1 || n > (size_t)apus::SMP_VMAX || ld < n || rows > 65535) {
        gcuda_set_error("sample_rows: rows %zu, n %zu, ld %zu", rows, n, ld);
        return -1;
    }
    if (temp != temp) { gcuda_set_error("sample_rows: temperature is NaN"); return -1; }
    if (sample_prepare((int)n)) return -1;
    return sample_launch(logits, (long)ld, (int)n, (int)rows, temp, top_p, nullptr, rng_state, out,
                               (cudaStream_t)stream);
}

}  // extern "C"
