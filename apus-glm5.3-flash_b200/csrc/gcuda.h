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
};

bool gemv_fast_ok(const GemvDesc &d);
// Split-K scratch the fast GEMV needs for (O, K): partial floats and ticket
// ints (0 when K fits one k-range).
void gemv_scratch_need(long O, long K, size_t *part_floats, size_t *tickets);
int gemv_launch(const GemvDesc &d, cudaStream_t st);
int fp8_dequant_launch(const uint8_t *w, const float *ws, uint16_t *out, size_t O, size_t K,
                       cudaStream_t st);
int kernel_error_read_and_clear(void);
int argmax_reset_launch(unsigned long long *keys, int n, cudaStream_t st);
int argmax_extract_launch(const unsigned long long *keys, int32_t *ids, int n, cudaStream_t st);

// error plumbing (capi.cu)
void gcuda_set_error(const char *fmt, ...);
int gcuda_check(cudaError_t e, const char *what);
