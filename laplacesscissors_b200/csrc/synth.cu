// Seeded synthetic inputs for benchmarks and tests: checkpoints and hidden states
// in the reference's layouts (safetensors bf16, row-major).  The generator is
// counter based -- element i of (seed, stream) is a pure function of the triple --
// so any slice can be produced independently and in parallel.
//
//   mix(z)      = SplitMix64 finaliser
//   key         = mix(seed ^ mix(stream + 0x9E3779B97F4A7C15))
//   bits(i)     = mix(key + (i + 1) * 0x9E3779B97F4A7C15)
//   normal(i)   : Box-Muller on the pair p = i / 2 with
//                 u1 = ((bits(2p) >> 11) + 1) * 2^-53 in (0, 1],
//                 u2 = (bits(2p + 1) >> 11) * 2^-53 in [0, 1),
//                 r = sqrt(-2 ln u1), element 2p = r cos(2 pi u2), 2p + 1 = r sin(2 pi u2)
//   value       = std * normal(i) in f64, rounded to f32 (nearest even), then to bf16
//                 (nearest even) when bf16 is requested
//   uniform(i)  = (bits(i) >> 32) * bound >> 32
#include <math.h>
#include <string.h>

#include <cmath>

#include "lsx_internal.h"

namespace {

inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xBF58476D1CE4E5B9ull;
    z = (z ^ (z >> 27)) * 0x94D049BB133111EBull;
    return z ^ (z >> 31);
}
constexpr uint64_t kGolden = 0x9E3779B97F4A7C15ull;

inline uint64_t stream_key(uint64_t seed, uint64_t stream) { return mix64(seed ^ mix64(stream + kGolden)); }
inline uint64_t bits_at(uint64_t key, uint64_t i) { return mix64(key + (i + 1) * kGolden); }

inline double normal_at(uint64_t key, uint64_t i) {
    uint64_t p = i >> 1;
    double u1 = (double)((bits_at(key, 2 * p) >> 11) + 1) * 0x1.0p-53;
    double u2 = (double)(bits_at(key, 2 * p + 1) >> 11) * 0x1.0p-53;
    double r = sqrt(-2.0 * log(u1));
    double angle = 6.283185307179586476925286766559 * u2;
    return (i & 1) ? r * sin(angle) : r * cos(angle);
}

inline uint16_t f32_to_bf16(float f) {
    uint32_t u;
    memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return 0x7fc0;
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

}  // namespace

extern "C" {

int lsx_synth_normal(uint64_t seed, uint64_t stream, uint64_t offset, size_t count, double std, lsx_dtype kind,
                     void* out) {
    LSX_ENSURE(out || count == 0, "output is NULL");
    LSX_ENSURE(kind == LSX_BF16 || kind == LSX_F32, "synthetic values are BF16 or F32");
    LSX_ENSURE(std::isfinite(std) && std >= 0.0, "standard deviation must be finite and non-negative");
    const uint64_t key = stream_key(seed, stream);
    const long long n = (long long)count;
#pragma omp parallel for schedule(static) if (count > (1u << 16))
    for (long long j = 0; j < n; ++j) {
        float v = (float)(std * normal_at(key, offset + (uint64_t)j));
        if (kind == LSX_BF16) ((uint16_t*)out)[j] = f32_to_bf16(v);
        else ((float*)out)[j] = v;
    }
    return LSX_OK;
}

int lsx_synth_uniform_u32(uint64_t seed, uint64_t stream, uint64_t offset, size_t count, uint32_t bound,
                          uint32_t* out) {
    LSX_ENSURE(out || count == 0, "output is NULL");
    LSX_ENSURE(bound > 0, "bound must be positive");
    const uint64_t key = stream_key(seed, stream);
    for (size_t j = 0; j < count; ++j)
        out[j] = (uint32_t)(((bits_at(key, offset + j) >> 32) * (uint64_t)bound) >> 32);
    return LSX_OK;
}

}  // extern "C"
