// init.cu — seeded synthetic weight generation on the device (BASELINE
// distributions), so multi-GB random-init models never cross PCIe.
// Every value is a pure function of (seed, stream id, element index): a
// splitmix64 hash feeds a Box-Muller normal or a uniform.
#include "common.cuh"
#include "gcuda.h"

namespace apus {

APUS_DEV uint64_t mix64(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

APUS_DEV float uni01(uint64_t h) { return ((float)(h >> 40) + 0.5f) * (1.0f / 16777216.0f); }

APUS_DEV float normal_at(uint64_t key, size_t i) {
    const uint64_t h1 = mix64(key ^ (2 * (uint64_t)i)), h2 = mix64(key ^ (2 * (uint64_t)i + 1));
    const float u1 = uni01(h1), u2 = uni01(h2);
    return sqrtf(-2.0f * logf(u1)) * cospif(2.0f * u2);
}

// Element i of dst is element first + i of the seeded stream, so any slice of
// a tensor (one rank's share) gets the values the whole tensor has.
__global__ void k_fill(int kind, void *dst, size_t n, uint64_t key, float a, float b, size_t first) {
    for (size_t j = blockIdx.x * (size_t)blockDim.x + threadIdx.x; j < n; j += (size_t)gridDim.x * blockDim.x) {
        const size_t i = first + j;
        switch (kind) {
        case FILL_BF16_NORMAL:      // mean b, std a
            ((uint16_t *)dst)[j] = bf16_bits(b + a * normal_at(key, i));
            break;
        case FILL_E4M3_NORMAL: {    // RNE E4M3 of N(0,1)*a, clamped to +-448, NaN codes excluded
            float v = a * normal_at(key, i);
            v = fminf(fmaxf(v, -448.f), 448.f);
            uint16_t two;
            asm("cvt.rn.satfinite.e4m3x2.f32 %0, %1, %2;" : "=h"(two) : "f"(0.f), "f"(v));
            ((uint8_t *)dst)[j] = (uint8_t)(two & 0xff);
            break;
        }
        case FILL_F32_LOGUNIFORM:   // exp(U(log a, log b))
            ((float *)dst)[j] = expf(logf(a) + (logf(b) - logf(a)) * uni01(mix64(key ^ i)));
            break;
        case FILL_F32_NORMAL:
            ((float *)dst)[j] = b + a * normal_at(key, i);
            break;
        case FILL_F32_CONST:
            ((float *)dst)[j] = a;
            break;
        case FILL_BF16_CONST:
            ((uint16_t *)dst)[j] = bf16_bits(a);
            break;
        }
    }
}

}  // namespace apus

int fill_launch(int kind, void *dst, size_t n, uint64_t seed, uint64_t stream_id, float a, float b,
                cudaStream_t st, size_t first) {
    if (!n) return 0;
    const uint64_t key = seed * 0x9E3779B97F4A7C15ull ^ (stream_id * 0xD1B54A32D192ED03ull);
    size_t blocks = (n + 255) / 256;
    if (blocks > 148 * 64) blocks = 148 * 64;
    apus::k_fill<<<(unsigned)blocks, 256, 0, st>>>(kind, dst, n, key, a, b, first);
    return cudaGetLastError() == cudaSuccess ? 0 : -1;
}
