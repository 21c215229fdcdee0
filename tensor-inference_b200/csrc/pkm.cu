// pkm.cu — product-key (PKM) adapter router: two-codebook nearest-address search.
//
// The reference specifies the router only in prose (README.md:58-72,157-180; the
// PKM benchmark configuration): a residual-stream query [2*D] splits into two
// halves; half h takes argmin_k ||q_h - C_h[k]||^2 over its codebook; the address
// is i * n_codes + j; a registry maps addresses to adapter ids (the lowest id
// wins when several adapter centroids share an address), -1 when empty.
//
// Exactness: every distance is the canonical fp32 sequence d = q[t] - c[t],
// acc = fma(d, d, acc) for t = 0..D-1 (each step correctly rounded on both the
// CPU and the GPU), and the argmin takes the lowest index among equal minima, so
// addresses are bit-identical to the CPU restatement.
//
// Tiling: a CTA owns 32 queries of one half and streams the codebook through
// shared memory in tiles of 64 codes; operands are stored dimension-major so a
// thread reads 2 queries and 4 codes as vectors; each thread keeps the running
// (distance, index) minimum of its (query, code-column) pairs; a final
// shared-memory merge across code columns keeps the first minimum.
#include <cstring>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"

namespace ti {

constexpr int kPkmThreads = 256;
constexpr int kPkmQ = 32;  // queries per CTA
constexpr int kPkmC = 64;  // codes per tile
// 256 threads = 16 query pairs x 16 code quads

template <int D>
__global__ void __launch_bounds__(kPkmThreads) k_pkm_assign(const float* __restrict__ queries, int n,
                                                            const float* __restrict__ c1, const float* __restrict__ c2,
                                                            int n_codes, const int32_t* __restrict__ table,
                                                            int32_t* __restrict__ addr, int32_t* __restrict__ adapter) {
    extern __shared__ __align__(16) float sm[];
    float* qs = sm;               // [D][kPkmQ]
    float* cs = qs + D * kPkmQ;   // [D][kPkmC]
    __shared__ float best_d[kPkmQ][16];
    __shared__ int best_i[kPkmQ][16];
    __shared__ int half_idx[2][kPkmQ];
    const int tid = threadIdx.x;
    const int qp = tid / 16, cq = tid % 16;  // query pair, code quad
    const int q0 = blockIdx.x * kPkmQ;

    for (int half = 0; half < 2; ++half) {
        const float* C = half ? c2 : c1;
        __syncthreads();
        // queries of this half, dimension-major
        for (int i = tid; i < kPkmQ * D; i += kPkmThreads) {
            const int q = i / D, t = i % D;
            qs[t * kPkmQ + q] = (q0 + q < n) ? queries[(size_t)(q0 + q) * (2 * D) + half * D + t] : 0.f;
        }
        float bd[2] = {INFINITY, INFINITY};
        int bi[2] = {0x7fffffff, 0x7fffffff};
        for (int c0 = 0; c0 < n_codes; c0 += kPkmC) {
            __syncthreads();
            for (int i = tid; i < kPkmC * D; i += kPkmThreads) {
                const int c = i / D, t = i % D;
                cs[t * kPkmC + c] = (c0 + c < n_codes) ? C[(size_t)(c0 + c) * D + t] : 0.f;
            }
            __syncthreads();
            float acc[2][4] = {};
#pragma unroll 4
            for (int t = 0; t < D; ++t) {
                const float2 qv = *reinterpret_cast<const float2*>(&qs[t * kPkmQ + qp * 2]);
                const float4 cv = *reinterpret_cast<const float4*>(&cs[t * kPkmC + cq * 4]);
                const float qa[2] = {qv.x, qv.y};
                const float ca[4] = {cv.x, cv.y, cv.z, cv.w};
#pragma unroll
                for (int a = 0; a < 2; ++a)
#pragma unroll
                    for (int b = 0; b < 4; ++b) {
                        const float d = __fsub_rn(qa[a], ca[b]);
                        acc[a][b] = __fmaf_rn(d, d, acc[a][b]);
                    }
            }
#pragma unroll
            for (int a = 0; a < 2; ++a)
#pragma unroll
                for (int b = 0; b < 4; ++b) {
                    const int k = c0 + cq * 4 + b;  // ascending within the thread: strict < keeps the first
                    if (k < n_codes && acc[a][b] < bd[a]) {
                        bd[a] = acc[a][b];
                        bi[a] = k;
                    }
                }
        }
        // merge the 16 code columns of each query: smaller distance, then lower index
#pragma unroll
        for (int a = 0; a < 2; ++a) {
            best_d[qp * 2 + a][cq] = bd[a];
            best_i[qp * 2 + a][cq] = bi[a];
        }
        __syncthreads();
        if (tid < kPkmQ) {
            float d = best_d[tid][0];
            int k = best_i[tid][0];
            for (int j = 1; j < 16; ++j) {
                const float dj = best_d[tid][j];
                const int kj = best_i[tid][j];
                if (dj < d || (dj == d && kj < k)) {
                    d = dj;
                    k = kj;
                }
            }
            half_idx[half][tid] = k;
        }
    }
    __syncthreads();
    if (tid < kPkmQ && q0 + tid < n) {
        const int a = half_idx[0][tid] * n_codes + half_idx[1][tid];
        addr[q0 + tid] = a;
        if (adapter) adapter[q0 + tid] = table ? table[a] : -1;
    }
}

static size_t pkm_smem(int D) { return (size_t)D * (kPkmQ + kPkmC) * 4; }

cudaError_t pkm_assign_launch(const float* queries, int n, const float* c1, const float* c2, int n_codes, int D,
                              const int32_t* table, int32_t* addr, int32_t* adapter, cudaStream_t s) {
    const void* f = nullptr;
    switch (D) {
        case 32: f = reinterpret_cast<const void*>(&k_pkm_assign<32>); break;
        case 64: f = reinterpret_cast<const void*>(&k_pkm_assign<64>); break;
        case 128: f = reinterpret_cast<const void*>(&k_pkm_assign<128>); break;
        case 256: f = reinterpret_cast<const void*>(&k_pkm_assign<256>); break;
        case 512: f = reinterpret_cast<const void*>(&k_pkm_assign<512>); break;
        default: return cudaErrorInvalidValue;
    }
    const size_t smem = pkm_smem(D);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    void* args[] = {&queries, &n, &c1, &c2, &n_codes, &table, &addr, &adapter};
    return cudaLaunchKernel(f, dim3((n + kPkmQ - 1) / kPkmQ), dim3(kPkmThreads), args, smem, s);
}

}  // namespace ti

using namespace ti;

struct ti_pkm {
    int dev = 0, n_codes = 0, D = 0;
    float *c1 = nullptr, *c2 = nullptr;
    int32_t* table = nullptr;           // device [n_codes^2]
    std::vector<int32_t> h_table;
};

extern "C" {

ti_status ti_pkm_create(int device, int n_codes, int half_dim, const float* c1_host, const float* c2_host,
                        ti_pkm** out) {
    clear_error();
    TI_CHECK(out && c1_host && c2_host, TI_ERR_INVALID, "pkm: null argument");
    TI_CHECK(n_codes >= 1 && n_codes <= 46340, TI_ERR_INVALID, "pkm: n_codes %d out of range", n_codes);
    TI_CHECK(half_dim == 32 || half_dim == 64 || half_dim == 128 || half_dim == 256 || half_dim == 512,
             TI_ERR_UNSUPPORTED, "pkm: half_dim %d (32..512, powers of two)", half_dim);
    DeviceGuard g(device);
    auto* p = new ti_pkm();
    p->dev = device;
    p->n_codes = n_codes;
    p->D = half_dim;
    const size_t cb = (size_t)n_codes * half_dim * 4;
    const size_t tb = (size_t)n_codes * n_codes * 4;
    cudaError_t e = cudaMalloc(&p->c1, cb);
    if (e == cudaSuccess) e = cudaMalloc(&p->c2, cb);
    if (e == cudaSuccess) e = cudaMalloc(&p->table, tb);
    if (e == cudaSuccess) e = cudaMemcpy(p->c1, c1_host, cb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemcpy(p->c2, c2_host, cb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = cudaMemset(p->table, 0xff, tb);
    if (e != cudaSuccess) {
        cudaGetLastError();
        cudaFree(p->c1);
        cudaFree(p->c2);
        cudaFree(p->table);
        delete p;
        return fail(TI_ERR_OOM, "pkm: %s", cudaGetErrorString(e));
    }
    p->h_table.assign((size_t)n_codes * n_codes, -1);
    *out = p;
    return TI_OK;
}

ti_status ti_pkm_destroy(ti_pkm* p) {
    if (!p) return TI_OK;
    DeviceGuard g(p->dev);
    cudaFree(p->c1);
    cudaFree(p->c2);
    cudaFree(p->table);
    delete p;
    return TI_OK;
}

// centroid addresses come from the same kernel as queries; the registry keeps
// the lowest adapter id per address
ti_status ti_pkm_register(ti_pkm* p, const float* centroids_host, const int32_t* adapter_ids, int n) {
    clear_error();
    TI_CHECK(p && centroids_host && adapter_ids && n >= 0, TI_ERR_INVALID, "pkm_register: bad argument");
    if (n == 0) return TI_OK;
    DeviceGuard g(p->dev);
    float* dq = nullptr;
    int32_t* da = nullptr;
    const size_t qb = (size_t)n * 2 * p->D * 4;
    TI_CUDA(cudaMalloc(&dq, qb));
    cudaError_t e = cudaMalloc(&da, (size_t)n * 4);
    if (e == cudaSuccess) e = cudaMemcpy(dq, centroids_host, qb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = pkm_assign_launch(dq, n, p->c1, p->c2, p->n_codes, p->D, nullptr, da, nullptr, 0);
    std::vector<int32_t> addr((size_t)n);
    if (e == cudaSuccess) e = cudaMemcpy(addr.data(), da, (size_t)n * 4, cudaMemcpyDeviceToHost);
    cudaFree(dq);
    cudaFree(da);
    TI_CHECK(e == cudaSuccess, TI_ERR_CUDA, "pkm_register: %s", cudaGetErrorString(e));
    for (int i = 0; i < n; ++i) {
        TI_CHECK(adapter_ids[i] >= 0, TI_ERR_INVALID, "pkm_register: negative adapter id");
        int32_t& slot = p->h_table[addr[i]];
        if (slot < 0 || adapter_ids[i] < slot) slot = adapter_ids[i];
    }
    TI_CUDA(cudaMemcpy(p->table, p->h_table.data(), p->h_table.size() * 4, cudaMemcpyHostToDevice));
    return TI_OK;
}

ti_status ti_pkm_query(ti_pkm* p, const float* queries, int n, int32_t* addr, int32_t* adapter, void* stream) {
    TI_CHECK(p && queries && addr && n >= 0, TI_ERR_INVALID, "pkm_query: bad argument");
    if (n == 0) return TI_OK;
    TI_CUDA(pkm_assign_launch(queries, n, p->c1, p->c2, p->n_codes, p->D, p->table, addr, adapter,
                              (cudaStream_t)stream));
    return TI_OK;
}

ti_status ti_pkm_query_host(ti_pkm* p, const float* queries, int n, int32_t* addr, int32_t* adapter) {
    clear_error();
    TI_CHECK(p && queries && addr && n >= 0, TI_ERR_INVALID, "pkm_query_host: bad argument");
    if (n == 0) return TI_OK;
    DeviceGuard g(p->dev);
    float* dq = nullptr;
    int32_t* dout = nullptr;
    const size_t qb = (size_t)n * 2 * p->D * 4;
    TI_CUDA(cudaMalloc(&dq, qb));
    cudaError_t e = cudaMalloc(&dout, (size_t)n * 8);
    if (e == cudaSuccess) e = cudaMemcpy(dq, queries, qb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess)
        e = pkm_assign_launch(dq, n, p->c1, p->c2, p->n_codes, p->D, p->table, dout, dout + n, 0);
    if (e == cudaSuccess) e = cudaMemcpy(addr, dout, (size_t)n * 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && adapter) e = cudaMemcpy(adapter, dout + n, (size_t)n * 4, cudaMemcpyDeviceToHost);
    cudaFree(dq);
    cudaFree(dout);
    TI_CHECK(e == cudaSuccess, TI_ERR_CUDA, "pkm_query_host: %s", cudaGetErrorString(e));
    return TI_OK;
}

}  // extern "C"
