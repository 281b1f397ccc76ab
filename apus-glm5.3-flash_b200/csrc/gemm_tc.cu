// gemm_tc.cu — dense BF16 GEMM on the fifth-generation tensor cores
// (tcgen05), for linear layers of 64 rows or more (prefill chunks), where the
// contraction is compute-shaped: y[m][o] = bf16(sum_k x[m][k] * W[o][k]) with
// fp32 accumulation (c/bf16.h:739-767 apus_bf16_gemm_mt's contraction; an FP8
// matrix is first dequantised to BF16 as c/fp8blk.h:109-317 does).
//
// Persistent CTAs, one per SM, each taking 128 x 256 output tiles (128 rows of
// x against 256 rows of W) in turn; 192 threads:
//   * warp 0 lane 0 streams 64-wide k-blocks of both operands with 2-D tensor
//     copies (128-byte swizzle, every CTA loading its own tiles) into a 4-stage ring (48 KB a
//     stage);
//   * warp 1 lane 0 issues tcgen05.mma.cta_group::1.kind::f16 (M 128, N 256,
//     K 16; four per k-block) into one of two 256-column TMEM accumulators
//     and commits each stage back to the producer and each finished tile to
//     the epilogue;
//   * warps 2-5 drain the other accumulator meanwhile (warp w reads TMEM
//     lanes 32 (w mod 4) .. +31, one tile row per lane), round to BF16 (or
//     keep fp32) and store.
// Every mbarrier wait is bounded (pipe.cuh): a lost copy or commit ends the
// kernel with an error word, TMEM freed, instead of a hang.
#include <cuda.h>
#include <cudaTypedefs.h>

#include "common.cuh"
#include "gcuda.h"
#include "pipe.cuh"

namespace apus {

__device__ int g_tc_err;   // first failed wait's code (21 stage free, 22 stage full, 23 accumulator)

namespace tc {
constexpr int BM = 128, BK = 64, NST = 4;
constexpr int THREADS = 192;               // warp 0 TMA, warp 1 MMA, warps 2-5 epilogue
constexpr int A_BYTES = BM * BK * 2;
template <int BN> struct Cfg {
    static constexpr int B_BYTES = BN * BK * 2, STAGE = A_BYTES + B_BYTES;
    static constexpr int SMEM = NST * STAGE + 1024;   // + slack to align the ring to the 1024-byte atom
    static constexpr int TMEM_COLS = 2 * BN;          // two fp32 accumulators: one drains, one fills
    // instruction descriptor: D f32 (bits 4-5 = 1), A and B BF16 (bits 7-9,
    // 10-12 = 1), both K-major (bits 15, 16 = 0), N >> 3 at bit 17, M >> 4 at bit 24
    static constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                                      ((uint32_t)(BM >> 4) << 24);
};
}  // namespace tc

struct TcDesc {
    uint16_t *y;      // [M][ldy] BF16, or null
    float *yf;        // [M][ldyf] fp32, or null
    long ldy, ldyf;
    int M, O, K;
    int ntm, ntn, ntiles;  // output tiles along M, along O, in total
    int mfast;        // tile t: m tile t % ntm, o tile t / ntm (else m t / ntn, o t % ntn)
};

// Shared-memory matrix descriptor of a K-major operand tile whose rows are
// 128 bytes (64 BF16) in the 128-byte swizzle: 8-row core groups 1024 bytes
// apart (stride offset), leading offset unused (1), descriptor version 1,
// layout type 2 (128-byte swizzle).  Advancing k by 16 inside the atom adds
// 32 bytes to the start address.
APUS_DEV uint64_t umma_desc_sw128(uint32_t saddr) {
    return (uint64_t)((saddr >> 4) & 0x3FFFu) | ((uint64_t)1 << 16) | ((uint64_t)(1024 >> 4) << 32) |
           ((uint64_t)1 << 46) | ((uint64_t)2 << 61);
}

APUS_DEV void tma_load_2d(void *dst, const CUtensorMap *map, int x, int y, uint64_t *bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes"
        " [%0], [%1, {%2, %3}], [%4];"
        ::"r"(smem_u32(dst)), "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

APUS_DEV void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }
APUS_DEV void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }

APUS_DEV void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t idesc, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(idesc), "r"(accumulate)
        : "memory");
}

// The completion of every tcgen05 operation issued so far by this thread
// arrives once on `bar`.
APUS_DEV void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

// 32 consecutive fp32 columns of this warp's 32 TMEM lanes (one row per lane).
APUS_DEV void tc_ld32(uint32_t taddr, uint32_t (&v)[32]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,"
        "%16,%17,%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15]),
          "=r"(v[16]), "=r"(v[17]), "=r"(v[18]), "=r"(v[19]), "=r"(v[20]), "=r"(v[21]), "=r"(v[22]), "=r"(v[23]),
          "=r"(v[24]), "=r"(v[25]), "=r"(v[26]), "=r"(v[27]), "=r"(v[28]), "=r"(v[29]), "=r"(v[30]), "=r"(v[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

// Persistent: CTA b takes output tiles b, b + grid, ... (tile t covers rows
// 128 * (t / ntn) and weight rows 256 * (t % ntn)).  The k-block ring and the
// two TMEM accumulators carry their phases across tiles, so the epilogue of
// one tile overlaps the mainloop of the next.
template <int BN>
__global__ void __launch_bounds__(tc::THREADS, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap, TcDesc d) {
    using C = tc::Cfg<BN>;
    extern __shared__ __align__(1024) uint8_t tc_dyn[];
    __shared__ __align__(8) uint64_t full[tc::NST], empty[tc::NST], tfull[2], tempty[2];
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int nkb = (d.K + tc::BK - 1) / tc::BK;
    uint8_t *ring = tc_dyn + ((1024 - (smem_u32(tc_dyn) & 1023)) & 1023);

    if (tid == 0) {
        for (int s = 0; s < tc::NST; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        for (int a = 0; a < 2; a++) { mbar_init(&tfull[a], 1); mbar_init(&tempty[a], 128); }
        abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&tmem_slot)), "r"(C::TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    volatile int *ab = &abort_flag;

    if (warp == 0) {
        if (lane == 0) {   // producer
            int g = 0;     // k-blocks issued by this CTA
            for (int t = blockIdx.x; t < d.ntiles && !*ab; t += gridDim.x) {
                const int m0 = (d.mfast ? t % d.ntm : t / d.ntn) * tc::BM;
                const int n0 = (d.mfast ? t / d.ntm : t % d.ntn) * BN;
                for (int kb = 0; kb < nkb; kb++, g++) {
                    const int s = g % tc::NST;
                    if (g >= tc::NST && !mbar_wait(&empty[s], ((g / tc::NST) - 1) & 1, ab, &g_tc_err, 21)) break;
                    uint8_t *sa = ring + s * C::STAGE;
                    mbar_arrive_expect_tx(&full[s], C::STAGE);
                    tma_load_2d(sa, &amap, kb * tc::BK, m0, &full[s]);
                    tma_load_2d(sa + tc::A_BYTES, &bmap, kb * tc::BK, n0, &full[s]);
                }
            }
        }
    } else if (warp == 1) {
        if (lane == 0) {   // MMA issuer
            int g = 0, i = 0;
            for (int t = blockIdx.x; t < d.ntiles && !*ab; t += gridDim.x, i++) {
                const int acc = i & 1;
                if (i >= 2 && !mbar_wait(&tempty[acc], ((i >> 1) - 1) & 1, ab, &g_tc_err, 24)) break;
                tc_fence_after();
                const uint32_t td = tmem + (uint32_t)(acc * BN);
                bool ok = true;
                for (int kb = 0; kb < nkb; kb++, g++) {
                    const int s = g % tc::NST;
                    if (!mbar_wait(&full[s], (g / tc::NST) & 1, ab, &g_tc_err, 22)) { ok = false; break; }
                    tc_fence_after();
                    const uint32_t sa = smem_u32(ring + s * C::STAGE), sb = sa + tc::A_BYTES;
#pragma unroll
                    for (int kk = 0; kk < tc::BK / 16; kk++)
                        tc_mma(td, umma_desc_sw128(sa + kk * 32), umma_desc_sw128(sb + kk * 32), C::IDESC,
                               (kb | kk) != 0);
                    tc_commit(&empty[s]);
                }
                if (!ok) break;
                tc_commit(&tfull[acc]);
            }
        }
    } else {
        // epilogue: warp w reads TMEM lanes 32 * (w % 4) .. + 31, one tile row per lane
        const int q = warp & 3;
        int i = 0;
        for (int t = blockIdx.x; t < d.ntiles; t += gridDim.x, i++) {
            const int acc = i & 1;
            const bool have = mbar_wait(&tfull[acc], (i >> 1) & 1, ab, &g_tc_err, 23);
            if (!__all_sync(0xffffffffu, have)) break;   // warp-uniform: the TMEM loads are collective
            tc_fence_after();
            const int row = (d.mfast ? t % d.ntm : t / d.ntn) * tc::BM + q * 32 + lane;
            const int nb = (d.mfast ? t / d.ntm : t % d.ntn) * BN;
            const bool rok = row < d.M;
            for (int c = 0; c < BN; c += 32) {
                uint32_t v[32];
                tc_ld32(tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(acc * BN + c), v);
                const int col = nb + c;
                if (!rok || col >= d.O) continue;
                if (d.y) {
                    uint16_t *yp = d.y + (size_t)row * d.ldy + col;
                    if (col + 32 <= d.O && !(((uintptr_t)yp) & 15)) {
#pragma unroll
                        for (int h = 0; h < 4; h++) {
                            uint32_t pk[4];
#pragma unroll
                            for (int j = 0; j < 4; j++)
                                pk[j] = (uint32_t)bf16_bits(__uint_as_float(v[8 * h + 2 * j])) |
                                        ((uint32_t)bf16_bits(__uint_as_float(v[8 * h + 2 * j + 1])) << 16);
                            ((uint4 *)yp)[h] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                        }
                    } else {
#pragma unroll
                        for (int j = 0; j < 32; j++)
                            if (col + j < d.O) yp[j] = bf16_bits(__uint_as_float(v[j]));
                    }
                }
                if (d.yf) {
                    float *fp = d.yf + (size_t)row * d.ldyf + col;
#pragma unroll
                    for (int j = 0; j < 32; j++)
                        if (col + j < d.O) fp[j] = __uint_as_float(v[j]);
                }
            }
            tc_fence_before();
            mbar_arrive(&tempty[acc]);
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(C::TMEM_COLS)
                     : "memory");
}

}  // namespace apus
using namespace apus;

// 2-D BF16 tensor map of a row-major [rows][ld] matrix viewed as K x rows,
// box 64 x box_rows with the 128-byte swizzle (zero fill past the edges).
static int tc_map(CUtensorMap *m, const void *base, long rows, long K, long ld, int box_rows) {
    static PFN_cuTensorMapEncodeTiled_v12000 enc = nullptr;
    if (!enc) {
        void *p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) != cudaSuccess ||
            q != cudaDriverEntryPointSuccess)
            return -1;
        enc = (PFN_cuTensorMapEncodeTiled_v12000)p;
    }
    const cuuint64_t dims[2] = {(cuuint64_t)K, (cuuint64_t)rows};
    const cuuint64_t strides[1] = {(cuuint64_t)ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)tc::BK, (cuuint32_t)box_rows};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS ? 0 : -1;
}

// Shapes and alignments the kernel takes (16-byte aligned operand bases and
// row strides, for the tensor maps).  Any M >= 1: the rows of the last m tile
// past M read zeros and are not stored.
static bool gemm_tc_shape_ok(const void *x, long ldx, const void *w, long ldw, long M, long O, long K) {
    return M >= 1 && O >= 1 && K >= 1 && M < (1l << 31) && O < (1l << 31) && K < (1l << 31) && ldx >= K &&
           ldw >= K && (ldx % 8) == 0 && (ldw % 8) == 0 && !((uintptr_t)x & 15) && !((uintptr_t)w & 15);
}

// The linear hooks' policy: 64 rows or more go to the tensor cores, fewer
// stay on the batch-invariant GEMV.
bool gemm_tc_ok(const void *x, long ldx, const void *w, long ldw, long M, long O, long K) {
    return M >= 64 && gemm_tc_shape_ok(x, ldx, w, ldw, M, O, K);
}

template <int BN>
static int tc_launch(const CUtensorMap &am, const uint16_t *w, long ldw, TcDesc d, int nsm, cudaStream_t st) {
    if (gcuda_smem_limit_once((const void *)k_gemm_tc<BN>, tc::Cfg<BN>::SMEM)) return -1;
    CUtensorMap bm;
    if (tc_map(&bm, w, d.O, d.K, ldw, BN)) return -1;
    d.ntn = (d.O + BN - 1) / BN;
    d.ntiles = d.ntm * d.ntn;
    // the smaller operand is the one re-read across tiles: walk the m tiles
    // first when x is the smaller, so each W tile is streamed once
    d.mfast = d.M <= d.O;
    const int grid = d.ntiles < nsm ? d.ntiles : nsm;
    k_gemm_tc<BN><<<grid, tc::THREADS, tc::Cfg<BN>::SMEM, st>>>(am, bm, d);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int gemm_tc_launch(const uint16_t *x, long ldx, const uint16_t *w, long ldw, uint16_t *y, long ldy, float *yf,
                   long ldyf, long M, long O, long K, cudaStream_t st) {
    if (!gemm_tc_shape_ok(x, ldx, w, ldw, M, O, K)) {
        gcuda_set_error("gemm_tc: unsupported shape %ldx%ldx%ld (ldx %ld, ldw %ld)", M, O, K, ldx, ldw);
        return -1;
    }
    const int nsm = gcuda_num_sms();
    if (nsm < 1) return -1;
    const long ntm = (M + tc::BM - 1) / tc::BM;
    if (ntm * ((O + 127) / 128) >= (1l << 31)) return -1;
    CUtensorMap am;
    if (tc_map(&am, x, M, K, ldx, tc::BM)) return -1;
    TcDesc d{y, yf, ldy, ldyf, (int)M, (int)O, (int)K, (int)ntm, 0, 0, 0};
    // 256-wide tiles unless 128-wide ones finish sooner over whole waves of
    // SMs: measured, a 128-wide tile takes about 0.75 of a 256-wide one's
    // time (half the work, but each SM's operand stream runs closer to its
    // latency and shared-memory limits)
    const long t256 = ntm * ((O + 255) / 256), t128 = ntm * ((O + 127) / 128);
    const double c256 = (double)((t256 + nsm - 1) / nsm), c128 = (double)((t128 + nsm - 1) / nsm) * 0.75;
    return c128 < c256 ? tc_launch<128>(am, w, ldw, d, nsm, st) : tc_launch<256>(am, w, ldw, d, nsm, st);
}

int tc_error_read_and_clear(void) {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_tc_err, sizeof v);
    cudaMemcpyToSymbol(g_tc_err, &z, sizeof z);
    return v;
}
