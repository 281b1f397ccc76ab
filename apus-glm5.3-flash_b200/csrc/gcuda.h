// gcuda.h — internal (C++) declarations shared by the CUDA translation units.
#pragma once
#include <cuda_runtime.h>
#include <stddef.h>
#include <stdint.h>

// One decode linear: y[m, o] for m < R (R <= 8) over weight rows o < O.
struct GemvDesc {
    const void *W;          // [O][K] row-major: E4M3 codes (fp8) or BF16 codes
    const float *WS;        // fp8 block scales [ceil(O/128)][nkb]
    long nkb;               // ceil(K/128)
    const uint16_t *x;      // [R][ldx] BF16 codes
    long ldx;
    int R;
    long O, K;
    int fp8;
    uint16_t *y;            // optional BF16 out [R][ldy]
    long ldy;
    float *yf;              // optional fp32 out [R][ldyf] (no rounding)
    long ldyf;
    unsigned long long *amax;  // optional argmax keys [R] (reset beforehand)
    float *part;            // split-K scratch [ceil(O/16)][ceil(K/4096)][128] (K > 4096 only)
    int *ticket;            // split-K tile counters [ceil(O/16)], zero between launches
    int pdl;                // launch as a programmatic dependent of the previous kernel
    int weights_after_wait; // weight pointers are produced by the previous kernel
    // Grouped mode (gexpert != null): problem p of *gcount (<= gmax) uses the
    // weights of expert gexpert[p] inside packed arrays (W + w_estride bytes per
    // expert, WS + s_estride floats per expert), activations x + p*x_pstride
    // and output y + p*y_pstride.  K must fit one k-range (K <= 4096).
    const int *gexpert;
    const int *gcount;
    int gmax;
    long w_estride, s_estride, x_pstride, y_pstride;
    int gnum;               // weight blocks in the packed arrays (grouped mode)
    // set by gemv_launch from (O, K, fp8, grouped) alone: the K range of one
    // work item and the weight tiles per work item
    long kx;
    int tpi;
    int box_ko;             // 128-byte k-slabs per tensor copy
    // FP8 inner loop (set by the launcher): 1 = codes widened to f16 against
    // activations rescaled by a power of two into f16 range (one cvt per two
    // weights, a scan and a conversion pass when staging); 0 = codes widened
    // to bf16 against the activations as they are (exact e4m3 -> f16 -> bf16)
    int x16;
    // argmax keys carry row + row_base (a vocabulary slice's global ids)
    long row_base;
    // plan the k-ranges as for a matrix of plan_o rows (0: O), so a slice of a
    // matrix sums each row in the same order as the whole matrix
    long plan_o;
    // x holds [R][2K] gate|up pairs; the staged activation is the SwiGLU
    // h = bf16(bf16(silu(min(g, lim))) * clip(u, +-lim)) (c/gmoe.h:216-224).
    int x_swiglu;
    float swiglu_limit;
    // Grouped mode, expert parallelism: row m of problem p whose selection
    // slot j = scat_slot[p*8 + m] is >= 0 also stores bf16(y * scat_w[m*scat_k
    // + j]) (y already rounded to BF16) at element
    // ((half*8 + m)*scat_j + j)*scat_ld + row of scat, half = (*scat_epoch+1)&1:
    // the weighted expert output other ranks read after the next exchange.
    uint16_t *scat;
    const int *scat_slot;
    const float *scat_w;
    const int *scat_epoch;
    int scat_k, scat_j;
    long scat_ld;
    int scat_r0;            // row offset of this launch's rows (row groups)
};

bool gemv_fast_ok(const GemvDesc &d);
// Split-K scratch the fast GEMV needs for (O, K): partial floats and ticket
// ints (0 when K fits one k-range).
void gemv_scratch_need(long O, long K, size_t *part_floats, size_t *tickets);
int gemv_launch(const GemvDesc &d, cudaStream_t st);
int fp8_dequant_launch(const uint8_t *w, const float *ws, uint16_t *out, size_t O, size_t K,
                       cudaStream_t st);
int kernel_error_read_and_clear(void);
// tcgen05 GEMM for >= 64 rows (gemm_tc.cu): y / yf [M][ld] = x [M][ldx] . W [O][ldw]^T,
// BF16 operands, fp32 accumulation; ld multiples of 8, 16-byte aligned bases.
bool gemm_tc_ok(const void *x, long ldx, const void *w, long ldw, long M, long O, long K);
int gemm_tc_launch(const uint16_t *x, long ldx, const uint16_t *w, long ldw, uint16_t *y, long ldy, float *yf,
                   long ldyf, long M, long O, long K, cudaStream_t st);
int tc_error_read_and_clear(void);
int ep_error_read_and_clear(void);      // the expert-parallel barrier's timeout word
int argmax_reset_launch(unsigned long long *keys, int n, cudaStream_t st);
int argmax_extract_launch(const unsigned long long *keys, int32_t *ids, int n, cudaStream_t st);

// error plumbing (capi.cu)
void gcuda_set_error(const char *fmt, ...);
int gcuda_check(cudaError_t e, const char *what);
// Per-device set-up shared by every launcher, thread-safe (capi.cu): raise a
// kernel's dynamic shared-memory limit to `bytes` on the current device the
// first time it is asked there (0 / -1), and the current device's SM count
// (0 on error).
int gcuda_smem_limit_once(const void *func, int bytes);
int gcuda_num_sms(void);

// seeded device-side weight fill (init.cu)
enum { FILL_BF16_NORMAL = 0, FILL_E4M3_NORMAL = 1, FILL_F32_LOGUNIFORM = 2, FILL_F32_NORMAL = 3,
       FILL_F32_CONST = 4, FILL_BF16_CONST = 5 };
int fill_launch(int kind, void *dst, size_t n, uint64_t seed, uint64_t stream_id, float a, float b,
                cudaStream_t st, size_t first = 0);
