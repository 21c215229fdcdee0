// api.cpp — error state, device management and memory entry points of the C ABI.
#include <cmath>
#include <cstring>
#include <string>

#include "internal.h"

namespace ti {

static thread_local std::string g_last_error;

void set_error(const char* fmt, ...) {
    char buf[1024];
    va_list ap;
    va_start(ap, fmt);
    vsnprintf(buf, sizeof buf, fmt, ap);
    va_end(ap);
    g_last_error = buf;
}
void clear_error() { g_last_error.clear(); }

// ops.cu:235-278: base_freq = 1 / theta^(2i/d) in float, Llama-3 three-regime scaling.
void rope_freqs(int head_dim, float theta, const ti_rope_scaling* sc, float* out) {
    const int half = head_dim / 2;
    ti_rope_scaling d = {0, 1.0f, 1.0f, 1.0f, 8192};
    if (!sc) sc = &d;
    const float pi2 = 2.0f * (float)M_PI;
    const float low_wavelen = (float)sc->original_max_pos / sc->low_freq_factor;
    const float high_wavelen = (float)sc->original_max_pos / sc->high_freq_factor;
    for (int i = 0; i < half; ++i) {
        const float base = 1.0f / std::pow(theta, (2.0f * (float)i) / (float)head_dim);
        if (!sc->apply_scaling) {
            out[i] = base;
            continue;
        }
        const float wavelen = pi2 / base;
        float f;
        if (wavelen < high_wavelen) f = base;
        else if (wavelen > low_wavelen) f = base / sc->factor;
        else {
            const float smooth = ((float)sc->original_max_pos / wavelen - sc->low_freq_factor) /
                                 (sc->high_freq_factor - sc->low_freq_factor);
            f = (1.0f - smooth) * (base / sc->factor) + smooth * base;
        }
        out[i] = f;
    }
}

}  // namespace ti

using namespace ti;

extern "C" {

const char* ti_last_error(void) { return g_last_error.c_str(); }
int ti_version(void) { return 100; }

ti_status ti_init(int* n_devices) {
    clear_error();
    int n = 0;
    const cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess || n == 0) {
        cudaGetLastError();
        return fail(TI_ERR_UNSUPPORTED, "ti_init: no CUDA device (%s)",
                    e != cudaSuccess ? cudaGetErrorString(e) : "none visible");
    }
    for (int d = 0; d < n; ++d) {
        int major = 0, minor = 0;
        TI_CUDA(cudaDeviceGetAttribute(&major, cudaDevAttrComputeCapabilityMajor, d));
        TI_CUDA(cudaDeviceGetAttribute(&minor, cudaDevAttrComputeCapabilityMinor, d));
        TI_CHECK(major == 10 && minor == 0, TI_ERR_UNSUPPORTED,
                 "ti_init: device %d has compute capability %d.%d; this build runs on sm_100 (B200) only", d, major,
                 minor);
    }
    if (n_devices) *n_devices = n;
    return TI_OK;
}

ti_status ti_shutdown(void) {
    clear_error();
    rope_tables_release();
    int n = 0;
    if (cudaGetDeviceCount(&n) != cudaSuccess) {
        cudaGetLastError();
        return TI_OK;
    }
    for (int d = 0; d < n; ++d) {
        cudaMemPool_t pool;
        if (cudaDeviceGetDefaultMemPool(&pool, d) == cudaSuccess) cudaMemPoolTrimTo(pool, 0);
    }
    cudaGetLastError();
    return TI_OK;
}

ti_status ti_device_count(int* count) {
    TI_CHECK(count, TI_ERR_INVALID, "ti_device_count: null");
    int n = 0;
    cudaError_t e = cudaGetDeviceCount(&n);
    if (e != cudaSuccess) {
        cudaGetLastError();
        n = 0;
    }
    *count = n;
    return TI_OK;
}

ti_status ti_device_info(int device, char* name, size_t name_len, size_t* total_mem) {
    cudaDeviceProp p;
    TI_CUDA(cudaGetDeviceProperties(&p, device));
    if (name && name_len) {
        std::strncpy(name, p.name, name_len - 1);
        name[name_len - 1] = 0;
    }
    if (total_mem) *total_mem = p.totalGlobalMem;
    return TI_OK;
}

ti_status ti_set_device(int device) {
    TI_CUDA(cudaSetDevice(device));
    return TI_OK;
}

// Stream-ordered pool allocation (cudaMallocAsync on the device's default
// mempool with a high release threshold): per-op temporaries of the
// tensor::backend shim reuse pool blocks instead of cudaMalloc/cudaFree per
// op (tensor.cu:72-121 of the reference synchronises on every free).
ti_status ti_malloc(int device, size_t bytes, void** ptr) {
    TI_CHECK(ptr, TI_ERR_INVALID, "ti_malloc: null out pointer");
    DeviceGuard g(device);
    static bool configured[64] = {};
    if (device >= 0 && device < 64 && !configured[device]) {
        cudaMemPool_t pool;
        if (cudaDeviceGetDefaultMemPool(&pool, device) == cudaSuccess) {
            uint64_t thr = ~0ull;
            cudaMemPoolSetAttribute(pool, cudaMemPoolAttrReleaseThreshold, &thr);
        }
        configured[device] = true;
    }
    void* p = nullptr;
    cudaError_t e = cudaMallocAsync(&p, bytes ? bytes : 1, (cudaStream_t)0);
    if (e != cudaSuccess) {
        cudaGetLastError();
        return fail(TI_ERR_OOM, "ti_malloc(%zu): %s", bytes, cudaGetErrorString(e));
    }
    *ptr = p;
    return TI_OK;
}

ti_status ti_free(int device, void* ptr) {
    if (!ptr) return TI_OK;
    DeviceGuard g(device);
    TI_CUDA(cudaFreeAsync(ptr, (cudaStream_t)0));
    return TI_OK;
}

ti_status ti_memset(void* dst, int value, size_t bytes, void* stream) {
    TI_CUDA(cudaMemsetAsync(dst, value, bytes, (cudaStream_t)stream));
    return TI_OK;
}
ti_status ti_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream) {
    TI_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyHostToDevice, (cudaStream_t)stream));
    TI_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    return TI_OK;
}
ti_status ti_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream) {
    TI_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    TI_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    return TI_OK;
}
ti_status ti_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream) {
    TI_CUDA(cudaMemcpyAsync(dst, src, bytes, cudaMemcpyDeviceToDevice, (cudaStream_t)stream));
    return TI_OK;
}
ti_status ti_stream_sync(void* stream) {
    TI_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    return TI_OK;
}

}  // extern "C"
