// capi.cu — the C ABI of include/apus_gcuda.h: error plumbing, HBM
// residency registry, host-pointer drop-ins and device-pointer twins of the
// linear leaf.
#include <cstdarg>
#include <cstdio>
#include <cstring>
#include <map>
#include <mutex>

#include "gcuda.h"
#include "../../include/apus_gcuda.h"

static thread_local char g_err[512];

void gcuda_set_error(const char *fmt, ...) {
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(g_err, sizeof g_err, fmt, ap);
    va_end(ap);
}

int gcuda_check(cudaError_t e, const char *what) {
    if (e == cudaSuccess) return 0;
    gcuda_set_error("%s: %s", what, cudaGetErrorString(e));
    return -1;
}

namespace {
std::mutex g_once_mu;
std::map<std::pair<const void *, int>, int> g_smem_set;   // (kernel, device) -> limit set
std::map<int, int> g_sms;                                 // device -> SM count
}  // namespace

int gcuda_smem_limit_once(const void *func, int bytes) {
    int dev = 0;
    if (gcuda_check(cudaGetDevice(&dev), "current device")) return -1;
    std::lock_guard<std::mutex> lk(g_once_mu);
    int &have = g_smem_set[{func, dev}];
    if (have >= bytes) return 0;
    if (gcuda_check(cudaFuncSetAttribute(func, cudaFuncAttributeMaxDynamicSharedMemorySize, bytes),
                    "kernel shared-memory limit"))
        return -1;
    have = bytes;
    return 0;
}

int gcuda_num_sms(void) {
    int dev = 0;
    if (cudaGetDevice(&dev) != cudaSuccess) return 0;
    std::lock_guard<std::mutex> lk(g_once_mu);
    int &n = g_sms[dev];
    if (!n && cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, dev) != cudaSuccess) n = 0;
    return n;
}

namespace {

struct Region {
    const uint8_t *host;
    size_t len;
    uint8_t *dev;
};

std::mutex g_mu;
std::map<uintptr_t, Region> g_regions;  // keyed by host start
bool g_enabled = false;
uint64_t g_pinned = 0, g_dispatch = 0, g_off_bf16 = 0, g_off_fp8 = 0;

// Grow-only per-process device scratch for the host-pointer entry points.
struct Scratch {
    void *p = nullptr;
    size_t cap = 0;
    void *get(size_t n) {
        if (n <= cap) return p;
        if (p) cudaFree(p);
        p = nullptr;
        cap = 0;
        if (cudaMalloc(&p, n) != cudaSuccess) return nullptr;
        cap = n;
        return p;
    }
};
Scratch g_sw, g_ss, g_sx, g_sy, g_keys, g_part, g_tick;
Scratch g_deq;   // BF16 copy of an FP8 matrix for the tensor-core path

// Split-K scratch of the library's own GEMV launches (grow-only; the ticket
// array is zeroed on growth and every launch leaves it zeroed).
int splitk_scratch(long O, long K, float **part, int **tick) {
    size_t pf, nt;
    gemv_scratch_need(O, K, &pf, &nt);
    *part = nullptr;
    *tick = nullptr;
    if (!pf) return 0;
    size_t old = g_tick.cap;
    *part = (float *)g_part.get(pf * sizeof(float));
    *tick = (int *)g_tick.get(nt * sizeof(int));
    if (!*part || !*tick) { gcuda_set_error("split-K scratch allocation failed"); return -1; }
    if (g_tick.cap != old && cudaMemset(*tick, 0, g_tick.cap) != cudaSuccess) return -1;
    return 0;
}
cudaStream_t g_stream = nullptr;

// y / yf / argmax keys of M rows: 64 rows or more (without the fused argmax)
// run the tcgen05 GEMM, an FP8 matrix dequantised to BF16 first exactly as
// c/fp8blk.h does; fewer rows run 8-row GEMV launches, each row bitwise
// independent of the others.  Caller holds g_mu.
int rows_locked(const void *dw, const float *dws, int fp8, const uint16_t *dx, uint16_t *dy, float *dyf,
                unsigned long long *keys, size_t M, size_t O, size_t K, cudaStream_t st, int pdl) {
    // (an FP8 matrix is checked through dx's alignment: its BF16 copy is a fresh allocation)
    if (M >= 64 && !keys && gemm_tc_ok(dx, (long)K, fp8 ? (const void *)dx : dw, (long)K, (long)M, (long)O, (long)K)) {
        const uint16_t *wb = (const uint16_t *)dw;
        if (fp8) {
            uint16_t *deq = (uint16_t *)g_deq.get(O * K * 2);
            if (!deq) { gcuda_set_error("dequant scratch allocation failed"); return -1; }
            if (fp8_dequant_launch((const uint8_t *)dw, dws, deq, O, K, st))
                return gcuda_check(cudaGetLastError(), "dequant launch") ? -1 : -1;
            wb = deq;
        }
        if (gemm_tc_launch(dx, (long)K, wb, (long)K, dy, (long)O, dyf, (long)O, (long)M, (long)O, (long)K, st))
            return gcuda_check(cudaGetLastError(), "tensor-core GEMM launch") ? -1 : -1;
        g_dispatch++;
        return 0;
    }
    float *part;
    int *tick;
    if (splitk_scratch((long)O, (long)K, &part, &tick)) return -1;
    for (size_t m0 = 0; m0 < M; m0 += 8) {
        GemvDesc d{};
        d.W = dw; d.WS = dws; d.nkb = (long)((K + 127) / 128);
        d.x = dx + m0 * K; d.ldx = (long)K;
        d.R = (int)((M - m0) < 8 ? (M - m0) : 8);
        d.O = (long)O; d.K = (long)K; d.fp8 = fp8;
        if (dy) { d.y = dy + m0 * O; d.ldy = (long)O; }
        if (dyf) { d.yf = dyf + m0 * O; d.ldyf = (long)O; }
        if (keys) d.amax = keys + m0;
        d.part = part; d.ticket = tick;
        d.pdl = pdl;
        if (gemv_launch(d, st)) return gcuda_check(cudaGetLastError(), "gemv launch") ? -1 : -1;
        g_dispatch++;
    }
    return 0;
}

int ensure_enabled() {
    if (g_enabled) return 0;
    char err[256];
    if (apus_gcuda_enable(err, sizeof err)) return -1;
    return 0;
}

// device view of a host range inside a registered region, else nullptr
const uint8_t *lookup(const void *p, size_t len) {
    uintptr_t a = (uintptr_t)p;
    auto it = g_regions.upper_bound(a);
    if (it == g_regions.begin()) return nullptr;
    --it;
    const Region &r = it->second;
    if (a >= (uintptr_t)r.host && a + len <= (uintptr_t)r.host + r.len)
        return r.dev + (a - (uintptr_t)r.host);
    return nullptr;
}

// Resolve a weight operand: resident copy, or a per-call upload.
const void *weight_dev(const void *host, size_t len, Scratch &s) {
    const uint8_t *d = lookup(host, len);
    if (d) return d;
    void *buf = s.get(len);
    if (!buf) { gcuda_set_error("cudaMalloc(%zu) failed", len); return nullptr; }
    if (gcuda_check(cudaMemcpyAsync(buf, host, len, cudaMemcpyHostToDevice, g_stream), "upload"))
        return nullptr;
    return buf;
}

int linear_host(const void *w, size_t wbytes, const float *ws, size_t sbytes, int fp8,
                const uint16_t *x, uint16_t *y, size_t M, size_t O, size_t K) {
    if (ensure_enabled()) return -1;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!M || !O) return 0;
    const void *dw = weight_dev(w, wbytes, g_sw);
    if (!dw) return -1;
    const float *dws = nullptr;
    if (fp8) {
        dws = (const float *)weight_dev(ws, sbytes, g_ss);
        if (!dws) return -1;
    }
    uint16_t *dx = (uint16_t *)g_sx.get(M * K * 2 + 16);
    uint16_t *dy = (uint16_t *)g_sy.get(M * O * 2 + 16);
    if (!dx || !dy) { gcuda_set_error("scratch allocation failed"); return -1; }
    if (gcuda_check(cudaMemcpyAsync(dx, x, M * K * 2, cudaMemcpyHostToDevice, g_stream), "x upload"))
        return -1;
    if (rows_locked(dw, dws, fp8, dx, dy, nullptr, nullptr, M, O, K, g_stream, 0)) return -1;
    if (gcuda_check(cudaMemcpyAsync(y, dy, M * O * 2, cudaMemcpyDeviceToHost, g_stream), "y download"))
        return -1;
    if (gcuda_check(cudaStreamSynchronize(g_stream), "sync")) return -1;
    if (fp8) g_off_fp8++; else g_off_bf16++;
    return 0;
}

}  // namespace

extern "C" {

int apus_gcuda_enable(char *err, size_t errcap) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (g_enabled) return 0;
    int dev = 0;
    cudaDeviceProp prop;
    if (cudaGetDevice(&dev) != cudaSuccess || cudaGetDeviceProperties(&prop, dev) != cudaSuccess) {
        if (err && errcap) snprintf(err, errcap, "gcuda: no CUDA device");
        gcuda_set_error("gcuda: no CUDA device");
        return -1;
    }
    if (prop.major != 10) {
        if (err && errcap) snprintf(err, errcap, "gcuda: device sm_%d%d is not sm_100", prop.major, prop.minor);
        gcuda_set_error("gcuda: device sm_%d%d is not sm_100", prop.major, prop.minor);
        return -1;
    }
    if (cudaStreamCreateWithFlags(&g_stream, cudaStreamNonBlocking) != cudaSuccess) {
        if (err && errcap) snprintf(err, errcap, "gcuda: stream creation failed");
        return -1;
    }
    g_enabled = true;
    return 0;
}

void apus_gcuda_disable(void) {
    std::lock_guard<std::mutex> lk(g_mu);
    if (!g_enabled) return;
    cudaStreamSynchronize(g_stream);
    for (auto &kv : g_regions) cudaFree(kv.second.dev);
    g_regions.clear();
    g_pinned = 0;
    for (Scratch *s : {&g_sw, &g_ss, &g_sx, &g_sy, &g_keys, &g_part, &g_tick}) {
        if (s->p) cudaFree(s->p);
        s->p = nullptr;
        s->cap = 0;
    }
    cudaStreamDestroy(g_stream);
    g_stream = nullptr;
    g_enabled = false;
}

int apus_gcuda_is_enabled(void) { return g_enabled ? 1 : 0; }

const char *apus_gcuda_last_error(void) { return g_err; }
void apus_gcuda_clear_error(void) { g_err[0] = 0; }

int apus_gcuda_kernel_error(void) {
    cudaDeviceSynchronize();
    const int a = kernel_error_read_and_clear(), b = ep_error_read_and_clear(), c = tc_error_read_and_clear();
    return a ? a : (b ? b : c);
}

int apus_gcuda_register_region(const void *ptr, size_t len) {
    if (ensure_enabled()) return -1;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!ptr || !len) return -1;
    if (g_regions.count((uintptr_t)ptr)) return 0;
    void *dev = nullptr;
    if (gcuda_check(cudaMalloc(&dev, len), "register_region cudaMalloc")) return -1;
    if (gcuda_check(cudaMemcpy(dev, ptr, len, cudaMemcpyHostToDevice), "register_region upload")) {
        cudaFree(dev);
        return -1;
    }
    g_regions[(uintptr_t)ptr] = Region{(const uint8_t *)ptr, len, (uint8_t *)dev};
    g_pinned += len;
    return 0;
}

void apus_gcuda_unregister_region(const void *ptr) {
    std::lock_guard<std::mutex> lk(g_mu);
    auto it = g_regions.find((uintptr_t)ptr);
    if (it == g_regions.end()) return;
    cudaStreamSynchronize(g_stream);
    cudaFree(it->second.dev);
    g_pinned -= it->second.len;
    g_regions.erase(it);
}

uint64_t apus_gcuda_bytes_pinned(void) { return g_pinned; }
uint64_t apus_gcuda_dispatches(void) { return g_dispatch; }
uint64_t apus_gcuda_offload_bf16(void) { return g_off_bf16; }
uint64_t apus_gcuda_offload_fp8blk(void) { return g_off_fp8; }

int apus_gcuda_bf16_gemm(const uint16_t *w, const uint16_t *x, uint16_t *y,
                         size_t M, size_t O, size_t K) {
    return linear_host(w, O * K * 2, nullptr, 0, 0, x, y, M, O, K) ? 1 : 0;
}

int apus_gcuda_fp8blk_linear(const uint8_t *codes, const float *scales,
                             const uint16_t *x, uint16_t *y,
                             size_t M, size_t O, size_t K) {
    const size_t sb = ((O + 127) / 128) * ((K + 127) / 128) * sizeof(float);
    return linear_host(codes, O * K, scales, sb, 1, x, y, M, O, K) ? 1 : 0;
}

void apus_gcuda_fill_hooks(ApusGcudaHooks *out) {
    out->bf16_gemm = apus_gcuda_bf16_gemm;
    out->fp8blk_linear = apus_gcuda_fp8blk_linear;
}

size_t apus_fp8blk_nblocks(size_t n) { return (n + 127) / 128; }

static void dequant_host(const uint8_t *w, const float *ws, uint16_t *out, size_t O, size_t K) {
    if (ensure_enabled()) return;
    std::lock_guard<std::mutex> lk(g_mu);
    if (!O || !K) return;
    const size_t sb = apus_fp8blk_nblocks(O) * apus_fp8blk_nblocks(K) * sizeof(float);
    const uint8_t *dw = (const uint8_t *)weight_dev(w, O * K, g_sw);
    const float *dws = dw ? (const float *)weight_dev(ws, sb, g_ss) : nullptr;
    uint16_t *dout = (uint16_t *)g_sy.get(O * K * 2 + 16);
    if (!dw || !dws || !dout) return;
    if (fp8_dequant_launch(dw, dws, dout, O, K, g_stream)) {
        gcuda_check(cudaGetLastError(), "dequant launch");
        return;
    }
    g_dispatch++;
    if (gcuda_check(cudaMemcpyAsync(out, dout, O * K * 2, cudaMemcpyDeviceToHost, g_stream), "download"))
        return;
    gcuda_check(cudaStreamSynchronize(g_stream), "sync");
}

void apus_fp8blk_dequant(const uint8_t *w, const float *ws, uint16_t *out, size_t O, size_t K) {
    dequant_host(w, ws, out, O, K);
}

void apus_fp8blk_dequant_mt(const uint8_t *w, const float *ws, uint16_t *out, size_t O, size_t K) {
    dequant_host(w, ws, out, O, K);
}

void apus_bf16_gemv_mt(const uint16_t *w, const uint16_t *x, float *xf, uint16_t *y,
                       size_t O, size_t K) {
    (void)xf;
    linear_host(w, O * K * 2, nullptr, 0, 0, x, y, 1, O, K);
}

void apus_bf16_gemm_mt(const uint16_t *w, const uint16_t *x, float *xf, uint16_t *y,
                       size_t M, size_t O, size_t K) {
    (void)xf;
    linear_host(w, O * K * 2, nullptr, 0, 0, x, y, M, O, K);
}

int apus_fp8blk_dequant_dev(const uint8_t *w, const float *ws, uint16_t *out,
                            size_t O, size_t K, void *stream) {
    return fp8_dequant_launch(w, ws, out, O, K, (cudaStream_t)stream)
               ? gcuda_check(cudaGetLastError(), "dequant launch") : 0;
}

static int g_pdl = 0;

void apus_gcuda_set_pdl(int on) { g_pdl = on ? 1 : 0; }

static int linear_dev(const void *w, const float *ws, int fp8, const uint16_t *x, uint16_t *y,
                      float *yf, unsigned long long *keys, size_t M, size_t O, size_t K,
                      cudaStream_t st) {
    std::lock_guard<std::mutex> lk(g_mu);
    return rows_locked(w, ws, fp8, x, y, yf, keys, M, O, K, st, g_pdl);
}

int apus_gcuda_fp8blk_linear_dev(const uint8_t *codes, const float *scales,
                                 const uint16_t *x, uint16_t *y,
                                 size_t M, size_t O, size_t K, void *stream) {
    return linear_dev(codes, scales, 1, x, y, nullptr, nullptr, M, O, K, (cudaStream_t)stream);
}

int apus_gcuda_bf16_gemm_dev(const uint16_t *w, const uint16_t *x, uint16_t *y,
                             size_t M, size_t O, size_t K, void *stream) {
    return linear_dev(w, nullptr, 0, x, y, nullptr, nullptr, M, O, K, (cudaStream_t)stream);
}

int apus_gcuda_bf16_gemm_f32_dev(const uint16_t *w, const uint16_t *x, float *y,
                                 size_t M, size_t O, size_t K, void *stream) {
    return linear_dev(w, nullptr, 0, x, nullptr, y, nullptr, M, O, K, (cudaStream_t)stream);
}

int apus_gcuda_bf16_gemm_argmax_dev(const uint16_t *w, const uint16_t *x, uint16_t *y,
                                    int32_t *ids, size_t M, size_t O, size_t K, void *stream) {
    cudaStream_t st = (cudaStream_t)stream;
    unsigned long long *keys;
    {
        std::lock_guard<std::mutex> lk(g_mu);
        keys = (unsigned long long *)g_keys.get(((M + 7) / 8) * 8 * sizeof(unsigned long long));
    }
    if (!keys) { gcuda_set_error("argmax scratch allocation failed"); return -1; }
    for (size_t m0 = 0; m0 < M; m0 += 8) {
        const int R = (int)((M - m0) < 8 ? (M - m0) : 8);
        if (argmax_reset_launch(keys + m0, R, st)) { gcuda_set_error("argmax reset launch failed"); return -1; }
    }
    if (linear_dev(w, nullptr, 0, x, y, nullptr, keys, M, O, K, st)) return -1;
    for (size_t m0 = 0; m0 < M; m0 += 8) {
        const int R = (int)((M - m0) < 8 ? (M - m0) : 8);
        if (argmax_extract_launch(keys + m0, ids + m0, R, st)) {
            gcuda_set_error("argmax extract launch failed");
            return -1;
        }
    }
    return 0;
}

}  // extern "C"
