// gemm_tc.cu — dense BF16 GEMM on the fifth-generation tensor cores
// (tcgen05), for linear layers of 64 rows or more (prefill chunks), where the
// contraction is compute-shaped: y[m][o] = bf16(sum_k x[m][k] * W[o][k]) with
// fp32 accumulation (c/bf16.h:739-767 apus_bf16_gemm_mt's contraction; an FP8
// matrix is first dequantised to BF16 as c/fp8blk.h:109-317 does).
//
// One CTA computes a 128 x 128 output tile (128 rows of x against 128 rows of
// W), 128 threads:
//   * warp 0 lane 0 streams 64-wide k-blocks of both operands with 2-D tensor
//     copies (128-byte swizzle, no multicast) into a 4-stage ring;
//   * warp 1 lane 0 issues tcgen05.mma.cta_group::1.kind::f16 (M 128, N 128,
//     K 16; four per k-block), accumulating in 128 TMEM columns, and commits
//     each stage back to the producer;
//   * all four warps then read the accumulator (warp w owns TMEM lanes
//     32w..32w+31, i.e. tile rows), round to BF16 (or keep fp32) and store.
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
constexpr int BM = 128, BN = 128, BK = 64, NST = 4, THREADS = 128;
constexpr int A_BYTES = BM * BK * 2, B_BYTES = BN * BK * 2, STAGE = A_BYTES + B_BYTES;
constexpr int SMEM = NST * STAGE + 1024;   // + slack to align the ring to the 1024-byte swizzle atom
constexpr int TMEM_COLS = BN;              // fp32 accumulator columns
// instruction descriptor: D f32 (bits 4-5 = 1), A and B BF16 (bits 7-9, 10-12
// = 1), both K-major (bits 15, 16 = 0), N >> 3 at bit 17, M >> 4 at bit 24
constexpr uint32_t IDESC = (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(BN >> 3) << 17) |
                           ((uint32_t)(BM >> 4) << 24);
}  // namespace tc

struct TcDesc {
    uint16_t *y;      // [M][ldy] BF16, or null
    float *yf;        // [M][ldyf] fp32, or null
    long ldy, ldyf;
    int M, O, K;
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

APUS_DEV void tc_mma(uint32_t tmem_d, uint64_t da, uint64_t db, uint32_t accumulate) {
    asm volatile(
        "{\n .reg .pred p;\n setp.ne.b32 p, %4, 0;\n"
        " tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n}"
        ::"r"(tmem_d), "l"(da), "l"(db), "r"(tc::IDESC), "r"(accumulate)
        : "memory");
}

// The completion of every tcgen05 operation issued so far by this thread
// arrives once on `bar`.
APUS_DEV void tc_commit(uint64_t *bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];"
                 ::"r"(smem_u32(bar)) : "memory");
}

APUS_DEV void tc_ld16(uint32_t taddr, uint32_t (&v)[16]) {
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(v[0]), "=r"(v[1]), "=r"(v[2]), "=r"(v[3]), "=r"(v[4]), "=r"(v[5]), "=r"(v[6]), "=r"(v[7]),
          "=r"(v[8]), "=r"(v[9]), "=r"(v[10]), "=r"(v[11]), "=r"(v[12]), "=r"(v[13]), "=r"(v[14]), "=r"(v[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
}

__global__ void __launch_bounds__(tc::THREADS, 1)
k_gemm_tc(const __grid_constant__ CUtensorMap amap, const __grid_constant__ CUtensorMap bmap, TcDesc d) {
    extern __shared__ __align__(1024) uint8_t tc_dyn[];
    __shared__ __align__(8) uint64_t full[tc::NST], empty[tc::NST], accb;
    __shared__ uint32_t tmem_slot;
    __shared__ int abort_flag;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int n0 = blockIdx.x * tc::BN, m0 = blockIdx.y * tc::BM;
    const int nkb = (d.K + tc::BK - 1) / tc::BK;
    uint8_t *ring = tc_dyn + ((1024 - (smem_u32(tc_dyn) & 1023)) & 1023);

    if (tid == 0) {
        for (int s = 0; s < tc::NST; s++) { mbar_init(&full[s], 1); mbar_init(&empty[s], 1); }
        mbar_init(&accb, 1);
        abort_flag = 0;
        fence_barrier_init();
    }
    if (warp == 2) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;"
                     ::"r"(smem_u32(&tmem_slot)), "r"(tc::TMEM_COLS) : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = tmem_slot;
    volatile int *ab = &abort_flag;

    if (warp == 0 && lane == 0) {
        // producer
        for (int kb = 0; kb < nkb; kb++) {
            const int s = kb % tc::NST;
            if (kb >= tc::NST && !mbar_wait(&empty[s], ((kb / tc::NST) - 1) & 1, ab, &g_tc_err, 21))
                break;
            uint8_t *sa = ring + s * tc::STAGE;
            mbar_arrive_expect_tx(&full[s], tc::STAGE);
            tma_load_2d(sa, &amap, kb * tc::BK, m0, &full[s]);
            tma_load_2d(sa + tc::A_BYTES, &bmap, kb * tc::BK, n0, &full[s]);
        }
    } else if (warp == 1 && lane == 0) {
        // MMA issuer
        bool ok = true;
        for (int kb = 0; kb < nkb && ok; kb++) {
            const int s = kb % tc::NST;
            if (!mbar_wait(&full[s], (kb / tc::NST) & 1, ab, &g_tc_err, 22)) { ok = false; break; }
            tc_fence_after();
            const uint32_t sa = smem_u32(ring + s * tc::STAGE), sb = sa + tc::A_BYTES;
#pragma unroll
            for (int kk = 0; kk < tc::BK / 16; kk++)
                tc_mma(tmem, umma_desc_sw128(sa + kk * 32), umma_desc_sw128(sb + kk * 32), (kb | kk) != 0);
            tc_commit(&empty[s]);
        }
        if (ok) tc_commit(&accb);
    }
    __syncwarp();

    // epilogue: thread (warp w, lane l) owns tile row 32w + l
    const bool have = mbar_wait(&accb, 0, ab, &g_tc_err, 23);
    __syncwarp();     // the TMEM loads below are warp-collective
    tc_fence_after();
    if (have) {
        const int row = m0 + warp * 32 + lane;
        const bool rok = row < d.M;
        for (int c = 0; c < tc::BN; c += 16) {
            uint32_t v[16];
            tc_ld16(tmem + ((uint32_t)(warp * 32) << 16) + (uint32_t)c, v);
            const int col = n0 + c;
            if (!rok || col >= d.O) continue;
            if (d.y) {
                uint16_t *yp = d.y + (size_t)row * d.ldy + col;
                if (col + 16 <= d.O && !(((uintptr_t)yp) & 15)) {
                    uint32_t pk[8];
#pragma unroll
                    for (int j = 0; j < 8; j++)
                        pk[j] = (uint32_t)bf16_bits(__uint_as_float(v[2 * j])) |
                                ((uint32_t)bf16_bits(__uint_as_float(v[2 * j + 1])) << 16);
                    ((uint4 *)yp)[0] = make_uint4(pk[0], pk[1], pk[2], pk[3]);
                    ((uint4 *)yp)[1] = make_uint4(pk[4], pk[5], pk[6], pk[7]);
                } else {
                    for (int j = 0; j < 16 && col + j < d.O; j++) yp[j] = bf16_bits(__uint_as_float(v[j]));
                }
            }
            if (d.yf) {
                float *fp = d.yf + (size_t)row * d.ldyf + col;
                for (int j = 0; j < 16 && col + j < d.O; j++) fp[j] = __uint_as_float(v[j]);
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 2)
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(tc::TMEM_COLS)
                     : "memory");
}

}  // namespace apus
using namespace apus;

// 2-D BF16 tensor map of a row-major [rows][ld] matrix viewed as K x rows,
// box 64 x 128 with the 128-byte swizzle (zero fill past the edges).
static int tc_map(CUtensorMap *m, const void *base, long rows, long K, long ld) {
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
    const cuuint32_t box[2] = {(cuuint32_t)tc::BK, (cuuint32_t)tc::BM};
    const cuuint32_t es[2] = {1, 1};
    return enc(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void *>(base), dims, strides, box, es,
               CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
               CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS ? 0 : -1;
}

bool gemm_tc_ok(const void *x, long ldx, const void *w, long ldw, long M, long O, long K) {
    return M >= 64 && O >= 1 && K >= 1 && M < (1l << 31) && O < (1l << 31) && K < (1l << 31) && ldx >= K &&
           ldw >= K && (ldx % 8) == 0 && (ldw % 8) == 0 && !((uintptr_t)x & 15) && !((uintptr_t)w & 15);
}

int gemm_tc_launch(const uint16_t *x, long ldx, const uint16_t *w, long ldw, uint16_t *y, long ldy, float *yf,
                   long ldyf, long M, long O, long K, cudaStream_t st) {
    if (!gemm_tc_ok(x, ldx, w, ldw, M, O, K)) return -1;
    static bool attr = false;
    if (!attr) {
        if (cudaFuncSetAttribute(k_gemm_tc, cudaFuncAttributeMaxDynamicSharedMemorySize, tc::SMEM) != cudaSuccess)
            return -1;
        attr = true;
    }
    CUtensorMap am, bm;
    if (tc_map(&am, x, M, K, ldx) || tc_map(&bm, w, O, K, ldw)) return -1;
    TcDesc d{y, yf, ldy, ldyf, (int)M, (int)O, (int)K};
    const dim3 grid((unsigned)((O + tc::BN - 1) / tc::BN), (unsigned)((M + tc::BM - 1) / tc::BM));
    k_gemm_tc<<<grid, tc::THREADS, tc::SMEM, st>>>(am, bm, d);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}

int tc_error_read_and_clear(void) {
    int v = 0, z = 0;
    cudaMemcpyFromSymbol(&v, g_tc_err, sizeof v);
    cudaMemcpyToSymbol(g_tc_err, &z, sizeof z);
    return v;
}
