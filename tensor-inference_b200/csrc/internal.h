// internal.h — host-side helpers shared by the C-ABI translation units.
#pragma once
#include <cuda_runtime.h>

#include <cstdarg>
#include <cstdio>
#include <random>
#include <string>

#include "../../include/ti_b200.h"

namespace ti {

void set_error(const char* fmt, ...);
void clear_error();

struct Fail {
    ti_status st;
};

// throw-free helpers: each returns the status and records the message
inline ti_status fail(ti_status st, const char* fmt, ...) {
    char buf[512];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    set_error("%s", buf);
    return st;
}

#define TI_CUDA(expr)                                                                          \
    do {                                                                                       \
        cudaError_t _e = (expr);                                                               \
        if (_e != cudaSuccess)                                                                 \
            return ::ti::fail(TI_ERR_CUDA, "%s: %s (%s:%d)", #expr, cudaGetErrorString(_e),    \
                              __FILE__, __LINE__);                                             \
    } while (0)

#define TI_CHECK(cond, st, ...)                                                                \
    do {                                                                                       \
        if (!(cond)) return ::ti::fail((st), __VA_ARGS__);                                     \
    } while (0)

// RAII device guard: restores the previous current device
struct DeviceGuard {
    int prev = -1;
    explicit DeviceGuard(int dev) {
        cudaGetDevice(&prev);
        if (prev != dev) cudaSetDevice(dev);
    }
    ~DeviceGuard() {
        int cur = -1;
        cudaGetDevice(&cur);
        if (prev >= 0 && cur != prev) cudaSetDevice(prev);
    }
};

// rope frequency table (ops.cu:235-278) computed on the host in float
void rope_freqs(int head_dim, float theta, const ti_rope_scaling* sc, float* out);
// free the device RoPE tables the ops cache (ops.cu)
void rope_tables_release();

// The uniform draws of one sequence's sampler, as the reference's engines
// produce them: std::uniform_real_distribution<float>(0, 1) over
// std::mt19937_64 (top_p.cpp:84-86).  Top-p keeps one engine, seeded at
// reset() and advanced per draw (the reference's is thread_local); top-k builds
// a fresh engine from the seed at every draw (top_p.cpp:124).  Unseeded
// samplers seed from std::random_device, as an unset seed does.
struct SamplerDraws {
    ti_sampling cfg{};  // kind TI_SAMPLE_GREEDY: no draws
    std::mt19937_64 rng;
    void reset(const ti_sampling& s);
    float next();
};
// TI_OK when `s` is a valid sampler (sample.cu)
ti_status sampler_check(const ti_sampling& s);

}  // namespace ti
