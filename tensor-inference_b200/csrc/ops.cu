// ops.cu — one sm_100a kernel per tensor::backend::ops function (the ti_op_* C ABI).
//
// These back the drop-in tensor::backend shim: the reference's unchanged model
// code (llama_model.cpp etc.) calls ops::* one op at a time, and each call
// lands here.  Rounding points and formulas follow src/backend/cuda/ops.cu of
// the reference, cited per kernel.  bf16 matmuls with few rows (decode) run on
// the weight-streaming GEMV, larger ones on the tcgen05 tensor-core GEMM; fp32
// and unaligned shapes on a tiled fp32-accumulate SIMT GEMM.
#include <map>
#include <mutex>
#include <tuple>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"

namespace ti {

// ------------------------------------------------------------------ embedding (ops.cu:46-88)
__global__ void k_gather_rows(const uint16_t* __restrict__ w, const int32_t* __restrict__ ids, uint16_t* __restrict__ out,
                              int hidden, int vocab, int* bad) {
    const int t = blockIdx.x;
    int id = ids[t];
    if (id < 0 || id >= vocab) {
        if (threadIdx.x == 0) atomicOr(bad, 1);
        return;
    }
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) out[(size_t)t * hidden + i] = w[(size_t)id * hidden + i];
}

// ------------------------------------------------------------------ tiled GEMM, C = A B^T (ops.cu:94-148)
// 64x64 output tile per CTA, K in steps of 32, 256 threads x 4x4 outputs, fp32 accumulate.
template <typename T>
__device__ __forceinline__ float ld_f(const T* p);
template <>
__device__ __forceinline__ float ld_f<uint16_t>(const uint16_t* p) {
    return __uint_as_float((uint32_t)(*p) << 16);
}
template <>
__device__ __forceinline__ float ld_f<float>(const float* p) {
    return *p;
}
template <typename T>
__device__ __forceinline__ void st_f(T* p, float v);
template <>
__device__ __forceinline__ void st_f<uint16_t>(uint16_t* p, float v) {
    *p = __bfloat16_as_ushort(__float2bfloat16_rn(v));
}
template <>
__device__ __forceinline__ void st_f<float>(float* p, float v) {
    *p = v;
}

template <typename T>
__global__ void __launch_bounds__(256) k_gemm_nt(const T* __restrict__ A, const T* __restrict__ B, T* __restrict__ C,
                                                 int M, int N, int K) {
    __shared__ float As[32][65];
    __shared__ float Bs[32][65];
    const int m0 = blockIdx.y * 64, n0 = blockIdx.x * 64;
    const int tx = threadIdx.x % 16, ty = threadIdx.x / 16;
    float acc[4][4] = {};
    for (int k0 = 0; k0 < K; k0 += 32) {
        for (int i = threadIdx.x; i < 64 * 32; i += 256) {
            const int r = i / 32, k = i % 32;
            As[k][r] = (m0 + r < M && k0 + k < K) ? ld_f<T>(A + (size_t)(m0 + r) * K + k0 + k) : 0.f;
            Bs[k][r] = (n0 + r < N && k0 + k < K) ? ld_f<T>(B + (size_t)(n0 + r) * K + k0 + k) : 0.f;
        }
        __syncthreads();
#pragma unroll 8
        for (int k = 0; k < 32; ++k) {
            float a[4], b[4];
#pragma unroll
            for (int i = 0; i < 4; ++i) a[i] = As[k][ty * 4 + i];
#pragma unroll
            for (int j = 0; j < 4; ++j) b[j] = Bs[k][tx * 4 + j];
#pragma unroll
            for (int i = 0; i < 4; ++i)
#pragma unroll
                for (int j = 0; j < 4; ++j) acc[i][j] = fmaf(a[i], b[j], acc[i][j]);
        }
        __syncthreads();
    }
#pragma unroll
    for (int i = 0; i < 4; ++i)
#pragma unroll
        for (int j = 0; j < 4; ++j) {
            const int m = m0 + ty * 4 + i, n = n0 + tx * 4 + j;
            if (m < M && n < N) st_f<T>(C + (size_t)m * N + n, acc[i][j]);
        }
}

// ------------------------------------------------------------------ RMSNorm (ops.cu:154-204, 726-774)
__global__ void __launch_bounds__(256) k_rms_norm(const uint16_t* __restrict__ x, const uint16_t* __restrict__ w,
                                                  uint16_t* __restrict__ out, int hidden, float eps, float off) {
    const int row = blockIdx.x;
    const uint16_t* xr = x + (size_t)row * hidden;
    float ss = 0.f;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x) {
        const float v = ld_f(xr + i);
        ss = fmaf(v, v, ss);
    }
    __shared__ float red[8];
    ss = warp_sum(ss);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float scale = rsqrtf(tot / (float)hidden + eps);
    for (int i = threadIdx.x; i < hidden; i += blockDim.x)
        st_f(out + (size_t)row * hidden + i, ld_f(xr + i) * scale * (ld_f(w + i) + off));
}

// ------------------------------------------------------------------ RoPE (ops.cu:210-233)
__global__ void k_rope(const uint16_t* __restrict__ x, uint16_t* __restrict__ out, const float* __restrict__ freqs,
                       int heads, int hd, int offset) {
    const int p = blockIdx.x, h = blockIdx.y, half = hd / 2;
    for (int i = threadIdx.x; i < half; i += blockDim.x) {
        const size_t base = ((size_t)p * heads + h) * hd;
        const float ang = (float)(p + offset) * freqs[i];
        const float c = cosf(ang), s = sinf(ang);
        const float x0 = ld_f(x + base + i), x1 = ld_f(x + base + i + half);
        st_f(out + base + i, x0 * c - x1 * s);
        st_f(out + base + i + half, x0 * s + x1 * c);
    }
}

// ------------------------------------------------------------------ elementwise (ops.cu:318-381, 707-724, 776-788)
__global__ void k_elementwise(int kind, const uint16_t* __restrict__ a, const uint16_t* __restrict__ b, float scalar,
                              uint16_t* __restrict__ out, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = ld_f(a + i);
        float r;
        switch (kind) {
            case TI_EW_SILU: r = v / (1.0f + expf(-v)); break;
            case TI_EW_GELU: {
                const float c1 = 0.7978845608f, c2 = 0.044715f;
                r = 0.5f * v * (1.0f + tanhf(c1 * (v + c2 * v * v * v)));
                break;
            }
            case TI_EW_MUL: r = v * ld_f(b + i); break;
            case TI_EW_ADD: r = v + ld_f(b + i); break;
            default: r = v * scalar; break;
        }
        st_f(out + i, r);
    }
}

// ------------------------------------------------------------------ bias (ops.cu:671-701)
__global__ void k_add_bias(const uint16_t* __restrict__ x, const uint16_t* __restrict__ bias, uint16_t* __restrict__ out,
                           int hidden) {
    const size_t row = blockIdx.x;
    for (int i = threadIdx.x; i < hidden; i += blockDim.x)
        st_f(out + row * hidden + i, ld_f(x + row * hidden + i) + ld_f(bias + i));
}

// ------------------------------------------------------------------ softmax (ops.cu:387-438)
template <typename T>
__global__ void __launch_bounds__(256) k_softmax(const T* __restrict__ x, float* __restrict__ out, int cols) {
    const size_t row = blockIdx.x;
    const T* xr = x + row * cols;
    float* o = out + row * cols;
    __shared__ float red[8];
    float m = -1e38f;
    for (int i = threadIdx.x; i < cols; i += blockDim.x) m = fmaxf(m, ld_f<T>(xr + i));
    m = warp_max(m);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = m;
    __syncthreads();
    float gm = red[0];
#pragma unroll
    for (int i = 1; i < 8; ++i) gm = fmaxf(gm, red[i]);
    __syncthreads();
    float s = 0.f;
    for (int i = threadIdx.x; i < cols; i += blockDim.x) s += expf(ld_f<T>(xr + i) - gm);
    s = warp_sum(s);
    if ((threadIdx.x & 31) == 0) red[threadIdx.x >> 5] = s;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float inv = 1.0f / tot;
    for (int i = threadIdx.x; i < cols; i += blockDim.x) o[i] = expf(ld_f<T>(xr + i) - gm) * inv;
}

// ------------------------------------------------------------------ attention (ops.cu:444-544)
// One CTA per (query row, q head): online softmax over key tiles of 128,
// fp32 throughout, bf16 output.  Mask only when causal && seq > 1.
constexpr int kOpAttnThreads = 128;
__global__ void __launch_bounds__(kOpAttnThreads) k_attention(const uint16_t* __restrict__ q, const uint16_t* __restrict__ k,
                                                            const uint16_t* __restrict__ v, uint16_t* __restrict__ out,
                                                            int seq, int n_heads, int kv_len, int n_kv, int hd,
                                                            int causal, int window, float scale) {
    extern __shared__ float sm[];
    float* qs = sm;          // [hd]
    float* p = qs + hd;      // [128]
    float* acc = p + 128;    // [hd]
    __shared__ float red[4];
    __shared__ float s_m, s_l, s_alpha;
    const int i = blockIdx.x, h = blockIdx.y;
    const int kvh = h / (n_heads / n_kv);
    const int tid = threadIdx.x;
    for (int d = tid; d < hd; d += kOpAttnThreads) {
        qs[d] = ld_f(q + ((size_t)i * n_heads + h) * hd + d);
        acc[d] = 0.f;
    }
    if (tid == 0) {
        s_m = -INFINITY;
        s_l = 0.f;
    }
    int jmax = kv_len, jmin = 0;
    if (causal && seq > 1) {
        const int off = kv_len - seq;
        jmax = min(kv_len, off + i + 1);
        if (window > 0) jmin = max(0, off + i - window + 1);
    }
    __syncthreads();
    for (int j0 = jmin; j0 < jmax; j0 += kOpAttnThreads) {
        const int j = j0 + tid;
        float s = -INFINITY;
        if (j < jmax) {
            const uint16_t* kr = k + ((size_t)j * n_kv + kvh) * hd;
            float d = 0.f;
            for (int e = 0; e < hd; ++e) d = fmaf(qs[e], ld_f(kr + e), d);
            s = scale * d;
        }
        float m = warp_max(s);
        if ((tid & 31) == 0) red[tid >> 5] = m;
        __syncthreads();
        if (tid == 0) {
            float tm = fmaxf(fmaxf(red[0], red[1]), fmaxf(red[2], red[3]));
            const float nm = fmaxf(s_m, tm);
            s_alpha = expf(s_m - nm);
            s_m = nm;
        }
        __syncthreads();
        const float pe = j < jmax ? expf(s - s_m) : 0.f;
        p[tid] = pe;
        float ls = warp_sum(pe);
        __syncthreads();
        if ((tid & 31) == 0) red[tid >> 5] = ls;
        __syncthreads();
        if (tid == 0) s_l = s_l * s_alpha + red[0] + red[1] + red[2] + red[3];
        const int nt = min(kOpAttnThreads, jmax - j0);
        for (int d = tid; d < hd; d += kOpAttnThreads) {
            float a = acc[d] * s_alpha;
            for (int t = 0; t < nt; ++t) a = fmaf(p[t], ld_f(v + ((size_t)(j0 + t) * n_kv + kvh) * hd + d), a);
            acc[d] = a;
        }
        __syncthreads();
    }
    for (int d = tid; d < hd; d += kOpAttnThreads) st_f(out + ((size_t)i * n_heads + h) * hd + d, acc[d] / s_l);
}

// ------------------------------------------------------------------ cast / transpose (ops.cu:559-616)
__global__ void k_cast(int src_dt, int dst_dt, const void* __restrict__ x, void* __restrict__ out, size_t n) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x) {
        const float v = src_dt == TI_DTYPE_F32 ? reinterpret_cast<const float*>(x)[i]
                                               : ld_f(reinterpret_cast<const uint16_t*>(x) + i);
        if (dst_dt == TI_DTYPE_F32) reinterpret_cast<float*>(out)[i] = v;
        else st_f(reinterpret_cast<uint16_t*>(out) + i, v);
    }
}

template <typename T>
__global__ void k_transpose(const T* __restrict__ x, T* __restrict__ out, int rows, int cols) {
    __shared__ T tile[32][33];
    const int c0 = blockIdx.x * 32, r0 = blockIdx.y * 32;
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int r = r0 + i, c = c0 + threadIdx.x;
        if (r < rows && c < cols) tile[i][threadIdx.x] = x[(size_t)r * cols + c];
    }
    __syncthreads();
    for (int i = threadIdx.y; i < 32; i += blockDim.y) {
        const int c = c0 + i, r = r0 + threadIdx.x;
        if (r < rows && c < cols) out[(size_t)c * rows + r] = tile[threadIdx.x][i];
    }
}

// rope tables cached per (device, head_dim, theta, scaling)
namespace {
std::mutex g_rope_mu;
std::map<std::tuple<int, int, float, int, float, float, float, int>, float*> g_rope_cache;
}  // namespace

void rope_tables_release() {
    std::lock_guard<std::mutex> lk(g_rope_mu);
    for (auto& kv : g_rope_cache) {
        int prev = 0;
        cudaGetDevice(&prev);
        cudaSetDevice(std::get<0>(kv.first));
        cudaFree(kv.second);
        cudaSetDevice(prev);
    }
    g_rope_cache.clear();
}

const float* rope_table(int dev, int hd, float theta, const void* scv) {
    const ti_rope_scaling* sc = reinterpret_cast<const ti_rope_scaling*>(scv);
    auto& mu = g_rope_mu;
    auto& cache = g_rope_cache;
    ti_rope_scaling z = {0, 1.f, 1.f, 1.f, 8192};
    const ti_rope_scaling& s = sc ? *sc : z;
    auto key = std::make_tuple(dev, hd, theta, s.apply_scaling, s.factor, s.low_freq_factor, s.high_freq_factor,
                               s.original_max_pos);
    std::lock_guard<std::mutex> lk(mu);
    auto it = cache.find(key);
    if (it != cache.end()) return it->second;
    std::vector<float> f(hd / 2);
    rope_freqs(hd, theta, &s, f.data());
    float* d = nullptr;
    if (cudaMalloc(&d, f.size() * 4) != cudaSuccess) return nullptr;
    cudaMemcpy(d, f.data(), f.size() * 4, cudaMemcpyHostToDevice);
    cache[key] = d;
    return d;
}

static int grid_for(size_t n) { return (int)std::min<size_t>((n + 255) / 256, 148 * 16); }

// bf16 matmul_t for more than 8 rows of `a` on the tensor cores: chunks of up
// to 256 rows, each one tcgen05 GEMM launch; partial-tile scratch from the pool.
static ti_status matmul_t_tc(const uint16_t* a, const uint16_t* b, uint16_t* c, int M, int N, int K,
                             cudaStream_t s) {
    int dev = 0;
    TI_CUDA(cudaGetDevice(&dev));
    constexpr size_t kWsCap = 16u << 20;  // floats
    GemvArgs g;
    g.W = b;
    g.N = N;
    g.K = K;
    g.nb = std::min(M, 256);
    g.x = a;
    g.x_stride = K;
    g.out = c;
    g.out_stride = N;
    TcPlan plan;
    std::string why;
    TI_CHECK(tc_plan(g, kEpiStore, dev, kWsCap, &plan, &why), TI_ERR_UNSUPPORTED, "matmul_t: %s", why.c_str());
    float* ws = nullptr;
    TI_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&ws), plan.ws_floats * 4 + (size_t)plan.tiles * 4, s));
    unsigned int* ctr = reinterpret_cast<unsigned int*>(ws + plan.ws_floats);
    TI_CUDA(cudaMemsetAsync(ctr, 0, (size_t)plan.tiles * 4, s));
    cudaError_t err = cudaSuccess;
    for (int m0 = 0; m0 < M && err == cudaSuccess; m0 += 256) {
        GemvArgs gc = g;
        gc.nb = std::min(256, M - m0);
        gc.x = a + (size_t)m0 * K;
        gc.out = c + (size_t)m0 * N;
        TcPlan pc;
        if (!tc_plan(gc, kEpiStore, dev, plan.ws_floats, &pc, &why)) {
            err = cudaErrorInvalidValue;
            break;
        }
        err = tc_launch(gc, kEpiStore, pc, ws, ctr, s, false);
    }
    if (ws) cudaFreeAsync(ws, s);
    TI_CHECK(err == cudaSuccess, TI_ERR_CUDA, "matmul_t: %s", cudaGetErrorString(err));
    return TI_OK;
}

}  // namespace ti

using namespace ti;

extern "C" {

ti_status ti_op_embedding(const void* weight, int vocab, int hidden, const int32_t* ids_host, int n, void* out,
                          void* stream) {
    TI_CHECK(weight && out && (ids_host || n == 0), TI_ERR_INVALID, "embedding: null argument");
    TI_CHECK(vocab > 0 && hidden > 0 && n >= 0, TI_ERR_INVALID, "embedding: bad shape");
    if (n == 0) return TI_OK;
    for (int i = 0; i < n; ++i)
        TI_CHECK(ids_host[i] >= 0 && ids_host[i] < vocab, TI_ERR_INVALID, "embedding: id %d out of [0, %d)",
                 ids_host[i], vocab);
    cudaStream_t s = (cudaStream_t)stream;
    int32_t* d_ids = nullptr;
    TI_CUDA(cudaMallocAsync(&d_ids, (size_t)n * 4 + 4, s));
    TI_CUDA(cudaMemcpyAsync(d_ids, ids_host, (size_t)n * 4, cudaMemcpyHostToDevice, s));
    int* bad = reinterpret_cast<int*>(d_ids + n);
    TI_CUDA(cudaMemsetAsync(bad, 0, 4, s));
    k_gather_rows<<<n, std::min(hidden, 256), 0, s>>>((const uint16_t*)weight, d_ids, (uint16_t*)out, hidden, vocab,
                                                      bad);
    TI_CUDA(cudaGetLastError());
    TI_CUDA(cudaFreeAsync(d_ids, s));
    TI_CUDA(cudaStreamSynchronize(s));  // ids_host may be released by the caller on return
    return TI_OK;
}

ti_status ti_op_matmul_t(int dtype, const void* a, const void* b, void* c, int M, int N, int K, void* stream) {
    TI_CHECK(a && b && c, TI_ERR_INVALID, "matmul_t: null argument");
    TI_CHECK(M > 0 && N > 0 && K > 0, TI_ERR_INVALID, "matmul_t: bad shape [%d,%d]x[%d,%d]^T", M, K, N, K);
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == TI_DTYPE_BF16) {
        if (M <= 8 && K % 64 == 0 && ((uintptr_t)a % 16) == 0 && ((uintptr_t)b % 16) == 0) {
            GemvArgs g;
            g.W = (const uint16_t*)b;
            g.N = N;
            g.K = K;
            g.nb = M;
            g.x = (const uint16_t*)a;
            g.x_stride = K;
            g.out = (uint16_t*)c;
            g.out_stride = N;
            int dev = 0;
            cudaGetDevice(&dev);
            GemvPlan plan;
            std::string why;
            if (gemv_plan(g, kEpiStore, dev, &plan, &why)) {
                TI_CUDA(gemv_launch(g, kEpiStore, plan, s, false));
                return TI_OK;
            }
        }
        if (M > 8 && K % 64 == 0 && ((uintptr_t)a % 16) == 0 && ((uintptr_t)b % 16) == 0)
            return matmul_t_tc((const uint16_t*)a, (const uint16_t*)b, (uint16_t*)c, M, N, K, s);
        dim3 grid((N + 63) / 64, (M + 63) / 64);
        k_gemm_nt<uint16_t><<<grid, 256, 0, s>>>((const uint16_t*)a, (const uint16_t*)b, (uint16_t*)c, M, N, K);
    } else if (dtype == TI_DTYPE_F32) {
        dim3 grid((N + 63) / 64, (M + 63) / 64);
        k_gemm_nt<float><<<grid, 256, 0, s>>>((const float*)a, (const float*)b, (float*)c, M, N, K);
    } else {
        return fail(TI_ERR_INVALID, "matmul_t: unsupported dtype");  // ops.cu:144
    }
    TI_CUDA(cudaGetLastError());
    return TI_OK;
}

ti_status ti_op_rms_norm(const void* x, const void* w, void* out, int rows, int hidden, float eps, int offset,
                         void* stream) {
    TI_CHECK(x && w && out, TI_ERR_INVALID, "rms_norm: null argument");
    TI_CHECK(rows >= 0 && hidden > 0, TI_ERR_INVALID, "rms_norm: bad shape");
    if (rows == 0) return TI_OK;
    k_rms_norm<<<rows, 256, 0, (cudaStream_t)stream>>>((const uint16_t*)x, (const uint16_t*)w, (uint16_t*)out, hidden,
                                                        eps, offset ? 1.0f : 0.0f);
    TI_CUDA(cudaGetLastError());
    return TI_OK;
}

ti_status ti_op_rope(const void* x, void* out, int seq, int heads, int head_dim, int seq_offset, float theta,
                     const ti_rope_scaling* scaling, void* stream) {
    TI_CHECK(x && out, TI_ERR_INVALID, "rope: null argument");
    TI_CHECK(seq >= 0 && heads > 0 && head_dim > 0 && head_dim % 2 == 0, TI_ERR_INVALID, "rope: bad shape");
    if (seq == 0) return TI_OK;
    int dev = 0;
    cudaGetDevice(&dev);
    const float* f = rope_table(dev, head_dim, theta, scaling);
    TI_CHECK(f, TI_ERR_OOM, "rope: table allocation failed");
    k_rope<<<dim3(seq, heads), std::min(head_dim / 2, 256), 0, (cudaStream_t)stream>>>(
        (const uint16_t*)x, (uint16_t*)out, f, heads, head_dim, seq_offset);
    TI_CUDA(cudaGetLastError());
    return TI_OK;
}

ti_status ti_op_elementwise(int kind, const void* a, const void* b, float scalar, void* out, size_t n, void* stream) {
    TI_CHECK(a && out, TI_ERR_INVALID, "elementwise: null argument");
    TI_CHECK(kind >= TI_EW_SILU && kind <= TI_EW_MUL_SCALAR, TI_ERR_INVALID, "elementwise: unknown kind %d", kind);
    TI_CHECK(!(kind == TI_EW_MUL || kind == TI_EW_ADD) || b, TI_ERR_INVALID, "elementwise: null second operand");
    if (n == 0) return TI_OK;
    k_elementwise<<<grid_for(n), 256, 0, (cudaStream_t)stream>>>(kind, (const uint16_t*)a, (const uint16_t*)b, scalar,
                                                                 (uint16_t*)out, n);
    TI_CUDA(cudaGetLastError());
    return TI_OK;
}

ti_status ti_op_add_bias(const void* x, const void* bias, void* out, int rows, int hidden, void* stream) {
    TI_CHECK(x && bias && out, TI_ERR_INVALID, "add_bias: null argument");
    TI_CHECK(rows >= 0 && hidden > 0, TI_ERR_INVALID, "add_bias: bad shape");
    if (rows == 0) return TI_OK;
    k_add_bias<<<rows, std::min(hidden, 256), 0, (cudaStream_t)stream>>>((const uint16_t*)x, (const uint16_t*)bias,
                                                                          (uint16_t*)out, hidden);
    TI_CUDA(cudaGetLastError());
    return TI_OK;
}

ti_status ti_op_softmax(int dtype, const void* x, float* out, int rows, int cols, void* stream) {
    TI_CHECK(x && out, TI_ERR_INVALID, "softmax: null argument");
    TI_CHECK(rows >= 0 && cols > 0, TI_ERR_INVALID, "softmax: bad shape");
    if (rows == 0) return TI_OK;
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == TI_DTYPE_F32) k_softmax<float><<<rows, 256, 0, s>>>((const float*)x, out, cols);
    else if (dtype == TI_DTYPE_BF16) k_softmax<uint16_t><<<rows, 256, 0, s>>>((const uint16_t*)x, out, cols);
    else return fail(TI_ERR_INVALID, "softmax: unsupported dtype");
    TI_CUDA(cudaGetLastError());
    return TI_OK;
}

ti_status ti_op_attention(const void* q, const void* k, const void* v, void* out, int seq, int n_heads, int kv_len,
                          int n_kv, int head_dim, int causal, int sliding_window, void* stream) {
    TI_CHECK(q && k && v && out, TI_ERR_INVALID, "attention: null argument");
    TI_CHECK(seq > 0 && n_heads > 0 && kv_len > 0 && n_kv > 0 && head_dim > 0 && n_heads % n_kv == 0,
             TI_ERR_INVALID, "attention: bad shape");
    TI_CHECK(kv_len >= seq || !causal, TI_ERR_INVALID, "attention: kv_len < seq with causal mask");
    const size_t smem = ((size_t)2 * head_dim + 128) * 4;
    k_attention<<<dim3(seq, n_heads), kOpAttnThreads, smem, (cudaStream_t)stream>>>(
        (const uint16_t*)q, (const uint16_t*)k, (const uint16_t*)v, (uint16_t*)out, seq, n_heads, kv_len, n_kv,
        head_dim, causal, sliding_window, 1.0f / sqrtf((float)head_dim));
    TI_CUDA(cudaGetLastError());
    return TI_OK;
}

ti_status ti_op_cast(int src_dtype, int dst_dtype, const void* x, void* out, size_t n, void* stream) {
    TI_CHECK(x && out, TI_ERR_INVALID, "cast: null argument");
    const bool ok = (src_dtype == TI_DTYPE_F32 || src_dtype == TI_DTYPE_BF16) &&
                    (dst_dtype == TI_DTYPE_F32 || dst_dtype == TI_DTYPE_BF16);
    TI_CHECK(ok, TI_ERR_INVALID, "cast: unsupported dtype pair");  // ops.cu:613
    if (n == 0) return TI_OK;
    cudaStream_t s = (cudaStream_t)stream;
    if (src_dtype == dst_dtype) {
        TI_CUDA(cudaMemcpyAsync(out, x, n * (src_dtype == TI_DTYPE_F32 ? 4 : 2), cudaMemcpyDeviceToDevice, s));
        return TI_OK;
    }
    k_cast<<<grid_for(n), 256, 0, s>>>(src_dtype, dst_dtype, x, out, n);
    TI_CUDA(cudaGetLastError());
    return TI_OK;
}

ti_status ti_op_transpose2d(int dtype, const void* x, void* out, int rows, int cols, void* stream) {
    TI_CHECK(x && out, TI_ERR_INVALID, "transpose: null argument");
    TI_CHECK(rows > 0 && cols > 0, TI_ERR_INVALID, "transpose: bad shape");
    dim3 grid((cols + 31) / 32, (rows + 31) / 32), block(32, 8);
    cudaStream_t s = (cudaStream_t)stream;
    if (dtype == TI_DTYPE_F32) k_transpose<float><<<grid, block, 0, s>>>((const float*)x, (float*)out, rows, cols);
    else if (dtype == TI_DTYPE_BF16)
        k_transpose<uint16_t><<<grid, block, 0, s>>>((const uint16_t*)x, (uint16_t*)out, rows, cols);
    else return fail(TI_ERR_INVALID, "transpose: unsupported dtype");  // ops.cu:581
    TI_CUDA(cudaGetLastError());
    return TI_OK;
}

}  // extern "C"
