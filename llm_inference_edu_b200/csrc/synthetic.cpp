// Documented counter-based generator for synthetic weights and prompts.
//
// Every value is a pure function of (seed, stream, index), so any thread
// split gives the same bits and both the device model and the CPU oracle can
// be fed from one host array.
//
//   mix(z)   = splitmix64 finalizer of z + 0x9E3779B97F4A7C15
//   base     = mix(seed * 0x100000001B3 ^ mix(stream))
//   pair k   : a = mix(base + 2k), b = mix(base + 2k + 1)
//              u1 = ((a >> 11) + 1) * 2^-53 in (0, 1], u2 = (b >> 11) * 2^-53
//              r = sqrt(-2 ln u1); z0 = r cos(2 pi u2); z1 = r sin(2 pi u2)
//   element 2k = z0 * stddev, element 2k+1 = z1 * stddev, rounded to FP32
//   (and then to BF16, nearest-even, for BF16 output)
//   token i  : mix(base + i) mod vocab
#include <math.h>
#include <stdint.h>
#include <string.h>

#include "../../include/qwen_b200.h"

namespace {

inline uint64_t mix(uint64_t z) {
    z += 0x9E3779B97F4A7C15ull;
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}

inline uint64_t stream_base(uint64_t seed, uint64_t stream) {
    return mix(seed * 0x100000001B3ull ^ mix(stream));
}

inline uint16_t f32_to_bf16(float x) {
    uint32_t u;
    memcpy(&u, &x, 4);
    if ((u & 0x7f800000u) == 0x7f800000u && (u & 0x007fffffu)) return (uint16_t)((u | 0x00400000u) >> 16);
    uint32_t lsb = (u >> 16) & 1u;
    return (uint16_t)((u + 0x7fffu + lsb) >> 16);
}

}  // namespace

extern "C" uint32_t qb_synthetic_normal(uint64_t seed, uint64_t stream, size_t n, double stddev,
                                        uint32_t out_dtype, void *out) {
    if (!out && n) return QB_INVALID_PARAMETERS;
    if (out_dtype != QB_HOST_F32 && out_dtype != QB_HOST_BF16) return QB_INVALID_PARAMETERS;
    const uint64_t base = stream_base(seed, stream);
    const long long pairs = (long long)((n + 1) / 2);
    const double two_pi = 6.283185307179586476925286766559;
#pragma omp parallel for schedule(static)
    for (long long k = 0; k < pairs; ++k) {
        uint64_t a = mix(base + 2 * (uint64_t)k), b = mix(base + 2 * (uint64_t)k + 1);
        double u1 = (double)((a >> 11) + 1) * (1.0 / 9007199254740992.0);
        double u2 = (double)(b >> 11) * (1.0 / 9007199254740992.0);
        double r = sqrt(-2.0 * log(u1));
        double z[2] = {r * cos(two_pi * u2), r * sin(two_pi * u2)};
        for (int e = 0; e < 2; ++e) {
            size_t i = 2 * (size_t)k + e;
            if (i >= n) break;
            float v = (float)(z[e] * stddev);
            if (out_dtype == QB_HOST_F32) ((float *)out)[i] = v;
            else ((uint16_t *)out)[i] = f32_to_bf16(v);
        }
    }
    return QB_OK;
}

extern "C" uint32_t qb_synthetic_tokens(uint64_t seed, uint64_t stream, size_t n, uint32_t vocab,
                                        uint32_t *out) {
    if (vocab == 0 || (!out && n)) return QB_INVALID_PARAMETERS;
    const uint64_t base = stream_base(seed, stream);
    for (size_t i = 0; i < n; ++i) out[i] = (uint32_t)(mix(base + i) % vocab);
    return QB_OK;
}
