// synth.cuh — the synthetic-weight generator (host and device).
//
// Element i of a tensor named `name` is a function of (seed, FNV-1a(name), i)
// only: x = mix64(key + (i+1) * golden), key = mix64(seed ^ FNV-1a(name));
// the four 16-bit fields of x are summed (Irwin–Hall, 4 terms), centred, and
// scaled by one fp32 multiply, std * sqrt(3) / 65536; bf16 by round-to-nearest-even.
// Integer arithmetic up to a single rounding makes host and device bit-identical.
#pragma once
#include <stdint.h>

#ifdef __CUDACC__
#define TI_HD __host__ __device__ __forceinline__
#else
#define TI_HD inline
#endif

namespace ti {

TI_HD uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

inline uint64_t fnv1a(const char* s) {
    uint64_t h = 0xcbf29ce484222325ULL;
    for (const unsigned char* p = (const unsigned char*)s; *p; ++p) {
        h ^= *p;
        h *= 0x100000001b3ULL;
    }
    return h;
}

inline float synth_scale(float std_) { return (float)((double)std_ * 1.7320508075688772 / 65536.0); }

TI_HD int32_t synth_centered(uint64_t key, uint64_t i) {
    uint64_t x = mix64(key + (i + 1) * 0x9E3779B97F4A7C15ULL);
    return (int32_t)(x & 0xffffu) + (int32_t)((x >> 16) & 0xffffu) + (int32_t)((x >> 32) & 0xffffu) +
           (int32_t)(x >> 48) - 131070;
}

}  // namespace ti
