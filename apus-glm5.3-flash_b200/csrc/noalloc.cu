// noalloc.cu — the fused BF16 GEMV + greedy pick with its scratch in a fixed
// file-scope device array, for callers that must not allocate.
//
// apus_gcuda_bf16_gemm_argmax_dev takes its scratch (the per-row argmax keys
// and, when K spans more than one 4096-wide range, the split-K partials and
// tickets) from a grow-only pool that calls cudaMalloc/cudaFree when a larger
// shape arrives.  Some callers cannot accept that: a serving process that has
// handed all of its HBM to its own page pool up front has nothing left to
// grow into, and a decode loop running other streams cannot take the
// device-wide synchronisation that cudaMalloc/cudaFree imply.  This variant
// runs the same kernels on the same split, so its results are bitwise those
// of the pooled entry point, but every byte of scratch comes from one static
// array of APUS_NOALLOC_SCRATCH_BYTES per device.
//
// Set-up: the first call on a device (with that device current) looks up the
// array's address with cudaGetSymbolAddress and caches it; that first call
// should therefore come before any stream capture.  The array is shared by
// every call on the device: calls that overlap in time (two host threads, or
// two streams) race on it and must be serialised by the caller.
#include <cstdio>
#include <mutex>

#include "gcuda.h"

#define APUS_NOALLOC_SCRATCH_BYTES (4u << 20)
#define APUS_NOALLOC_MAX_ROWS 64
#define APUS_NOALLOC_MAX_DEVICES 64

// [keys: MAX_ROWS u64][tickets: int, 256-byte padded][split-K partials: f32]
static __device__ __align__(256) unsigned char g_noalloc_scratch[APUS_NOALLOC_SCRATCH_BYTES];

static std::mutex g_noalloc_mu;
static unsigned char *g_noalloc_ptr[APUS_NOALLOC_MAX_DEVICES];

static unsigned char *noalloc_base() {
    int dev = -1;
    if (cudaGetDevice(&dev) != cudaSuccess || dev < 0 || dev >= APUS_NOALLOC_MAX_DEVICES) {
        gcuda_set_error("bf16_gemm_argmax_static: no usable current device");
        return nullptr;
    }
    std::lock_guard<std::mutex> lk(g_noalloc_mu);
    if (!g_noalloc_ptr[dev]) {
        void *p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_noalloc_scratch);
        if (e != cudaSuccess || !p) {
            gcuda_set_error("bf16_gemm_argmax_static: cudaGetSymbolAddress failed on device %d: %s", dev,
                            cudaGetErrorString(e));
            return nullptr;
        }
        g_noalloc_ptr[dev] = (unsigned char *)p;
    }
    return g_noalloc_ptr[dev];
}

extern "C" int apus_gcuda_bf16_gemm_argmax_static_dev(const uint16_t *w, const uint16_t *x, uint16_t *y,
                                                      int32_t *ids, size_t M, size_t O, size_t K,
                                                      void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    if (M == 0 || O == 0 || K == 0) return 0;
    if (O > 0xFFFFFFFEull) {
        gcuda_set_error("bf16_gemm_argmax_static: O = %zu exceeds the 32-bit pick index", O);
        return -1;
    }
    if (M > APUS_NOALLOC_MAX_ROWS) {
        gcuda_set_error("bf16_gemm_argmax_static: M = %zu rows exceeds the static maximum of %d", M,
                        APUS_NOALLOC_MAX_ROWS);
        return -1;
    }
    size_t part_floats, tickets;
    gemv_scratch_need((long)O, (long)K, &part_floats, &tickets);
    const size_t keys_bytes = APUS_NOALLOC_MAX_ROWS * sizeof(unsigned long long);
    const size_t tick_bytes = (tickets * sizeof(int) + 255) & ~(size_t)255;
    const size_t need = keys_bytes + tick_bytes + part_floats * sizeof(float);
    if (need > APUS_NOALLOC_SCRATCH_BYTES) {
        gcuda_set_error("bf16_gemm_argmax_static: O = %zu, K = %zu needs %zu scratch bytes, the static maximum "
                        "is %u", O, K, need, APUS_NOALLOC_SCRATCH_BYTES);
        return -1;
    }
    unsigned char *base = noalloc_base();
    if (!base) return -1;
    unsigned long long *keys = (unsigned long long *)base;
    int *tick = tickets ? (int *)(base + keys_bytes) : nullptr;
    float *part = part_floats ? (float *)(base + keys_bytes + tick_bytes) : nullptr;
    // the split-K tickets must start at zero (each launch leaves them zeroed;
    // clearing here also covers a launch that ended early on an error)
    if (tick && gcuda_check(cudaMemsetAsync(tick, 0, tickets * sizeof(int), st), "static scratch clear"))
        return -1;
    for (size_t m0 = 0; m0 < M; m0 += 8) {
        const int R = (int)((M - m0) < 8 ? (M - m0) : 8);
        if (argmax_reset_launch(keys + m0, R, st)) { gcuda_set_error("argmax reset launch failed"); return -1; }
        GemvDesc d{};
        d.W = w; d.x = x + m0 * K; d.ldx = (long)K; d.R = R;
        d.O = (long)O; d.K = (long)K; d.fp8 = 0;
        if (y) { d.y = y + m0 * O; d.ldy = (long)O; }
        d.amax = keys + m0;
        d.part = part; d.ticket = tick;
        if (gemv_launch(d, st)) { gcuda_set_error("gemv launch failed"); return -1; }
        if (argmax_extract_launch(keys + m0, ids + m0, R, st)) {
            gcuda_set_error("argmax extract launch failed");
            return -1;
        }
    }
    return 0;
}
