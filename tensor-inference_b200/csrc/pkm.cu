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
// Tiling: a CTA owns 64 queries and streams the codebook of each half in tiles
// of 128 codes and chunks of 32 dimensions (the accumulators of a code tile stay
// in registers across its chunks, so every distance keeps the canonical order).
// The codebooks are stored dimension-major (transposed once, at create time, and
// padded to whole 128-code tiles), so a code chunk is a straight cp.async copy;
// query chunks are read as float4 rows and written transposed, lanes across
// queries (no shared-memory bank conflicts).  Both are double-buffered.  Thread
// (qg, cg) keeps 4 queries x 8 codes (codes 4cg..4cg+3 and 64+4cg..64+4cg+3 of the
// tile, so each 8-lane phase of a code load is 128 contiguous bytes): per dimension
// one 16-byte load of its queries, two of its codes, and 16 packed f32x2 subtractions + 16 packed FMAs
// (each lane individually rounded: the same sequence as the scalar form).  Each
// thread keeps the running (distance, index) minimum of its queries over its
// codes, in ascending code order; the 16 threads of a query group merge by
// shuffles, lower index first among equal distances.
#include <cstring>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"

namespace ti {

constexpr int kPkmThreads = 256;
constexpr int kPkmQ = 64;    // queries per CTA
constexpr int kPkmC = 128;   // codes per tile
constexpr int kPkmDc = 32;   // dimensions per chunk
// 256 threads = 16 query groups (4 queries) x 16 code groups (8 codes)

TI_DEVICE_INLINE float2 sub2(float2 a, float2 b) {
    unsigned long long av = *reinterpret_cast<unsigned long long*>(&a);
    unsigned long long bv = *reinterpret_cast<unsigned long long*>(&b);
    unsigned long long r;
    asm("sub.rn.f32x2 %0, %1, %2;" : "=l"(r) : "l"(av), "l"(bv));
    return *reinterpret_cast<float2*>(&r);
}
TI_DEVICE_INLINE void cp_async16(void* dst, const void* src) {
    asm volatile("cp.async.cg.shared.global [%0], [%1], 16;" ::"r"(smem_u32(dst)), "l"(src) : "memory");
}
TI_DEVICE_INLINE void cp_async_commit() { asm volatile("cp.async.commit_group;" ::: "memory"); }
TI_DEVICE_INLINE void cp_async_wait_1() { asm volatile("cp.async.wait_group 1;" ::: "memory"); }

// ct1 / ct2: dimension-major codebooks [D][ncp] (ncp = n_codes padded to 128)
template <int D>
__global__ void __launch_bounds__(kPkmThreads) k_pkm_assign(const float* __restrict__ queries, int n,
                                                            const float* __restrict__ ct1, const float* __restrict__ ct2,
                                                            int n_codes, int ncp, const int32_t* __restrict__ table,
                                                            int32_t* __restrict__ addr, int32_t* __restrict__ adapter) {
    // dynamic: qs [2][kPkmDc][kPkmQ] then cs [2][kPkmDc][kPkmC] (48 KB)
    extern __shared__ __align__(16) float pkm_sm[];
    auto qs = reinterpret_cast<float(*)[kPkmDc][kPkmQ]>(pkm_sm);
    auto cs = reinterpret_cast<float(*)[kPkmDc][kPkmC]>(pkm_sm + 2 * kPkmDc * kPkmQ);
    __shared__ int half_idx[2][kPkmQ];
    const int tid = threadIdx.x;
    const int qg = tid >> 4, cg = tid & 15;
    const int q0 = blockIdx.x * kPkmQ;
    constexpr int NCH = D / kPkmDc;
    const int ntile = ncp / kPkmC;
    const int total = 2 * ntile * NCH;  // iterations: (half, code tile, chunk)

    // loads of iteration it into buffer b: the code chunk by cp.async, the query chunk into registers
    float4 qreg[2];
    auto issue = [&](int it, int b) {
        const int half = it / (ntile * NCH), rem = it % (ntile * NCH);
        const int tile = rem / NCH, ch = rem % NCH;
        const float* C = (half ? ct2 : ct1) + (size_t)(ch * kPkmDc) * ncp + tile * kPkmC;
#pragma unroll
        for (int r = 0; r < kPkmDc * kPkmC / 4 / kPkmThreads; ++r) {
            const int i = tid + r * kPkmThreads;  // 16-byte piece: row i / 32, column (i % 32) * 4
            cp_async16(&cs[b][i >> 5][(i & 31) * 4], C + (size_t)(i >> 5) * ncp + (i & 31) * 4);
        }
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int i = tid + r * kPkmThreads;  // query i % 64, dimensions 4 * (i / 64) ..
            const int q = i & (kPkmQ - 1), t4 = i >> 6;
            qreg[r] = q0 + q < n ? __ldg(reinterpret_cast<const float4*>(queries + (size_t)(q0 + q) * (2 * D) +
                                                                           half * D + ch * kPkmDc + t4 * 4))
                                 : make_float4(0.f, 0.f, 0.f, 0.f);
        }
    };
    auto store_q = [&](int b) {
#pragma unroll
        for (int r = 0; r < 2; ++r) {
            const int i = tid + r * kPkmThreads;
            const int q = i & (kPkmQ - 1), t4 = i >> 6;
            qs[b][t4 * 4 + 0][q] = qreg[r].x;
            qs[b][t4 * 4 + 1][q] = qreg[r].y;
            qs[b][t4 * 4 + 2][q] = qreg[r].z;
            qs[b][t4 * 4 + 3][q] = qreg[r].w;
        }
    };

    float2 acc[4][4];  // [query][code pair]
    float bd[4];
    int bi[4];
    issue(0, 0);
    store_q(0);
    cp_async_commit();
    for (int it = 0; it < total; ++it) {
        const int b = it & 1;
        const int half = it / (ntile * NCH), rem = it % (ntile * NCH);
        const int tile = rem / NCH, ch = rem % NCH;
        if (it + 1 < total) issue(it + 1, b ^ 1);  // buffer b^1 was read by iteration it - 1, before the barrier
        cp_async_commit();
        cp_async_wait_1();  // this iteration's code chunk has landed
        __syncthreads();
        if (rem == 0) {
#pragma unroll
            for (int j = 0; j < 4; ++j) bd[j] = INFINITY, bi[j] = 0x7fffffff;
        }
        if (ch == 0) {
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int p = 0; p < 4; ++p) acc[j][p] = make_float2(0.f, 0.f);
        }
#pragma unroll 4
        for (int t = 0; t < kPkmDc; ++t) {
            const float4 qv = *reinterpret_cast<const float4*>(&qs[b][t][qg * 4]);
            // codes 4 cg .. 4 cg + 3 and 64 + 4 cg .. 64 + 4 cg + 3: each 8-lane phase of a
            // 16-byte load reads 128 contiguous bytes (no bank conflict)
            const float4 ca = *reinterpret_cast<const float4*>(&cs[b][t][cg * 4]);
            const float4 cb = *reinterpret_cast<const float4*>(&cs[b][t][kPkmC / 2 + cg * 4]);
            const float qa[4] = {qv.x, qv.y, qv.z, qv.w};
            const float2 cp[4] = {make_float2(ca.x, ca.y), make_float2(ca.z, ca.w), make_float2(cb.x, cb.y),
                                  make_float2(cb.z, cb.w)};
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const float2 d = sub2(make_float2(qa[j], qa[j]), cp[p]);
                    acc[j][p] = ffma2(d, d, acc[j][p]);
                }
        }
        if (ch == NCH - 1) {
            // the tile's distances are complete: running minimum in ascending code order
#pragma unroll
            for (int j = 0; j < 4; ++j)
#pragma unroll
                for (int p = 0; p < 4; ++p) {
                    const int k = tile * kPkmC + (p < 2 ? cg * 4 + p * 2 : kPkmC / 2 + cg * 4 + (p - 2) * 2);
                    if (k < n_codes && acc[j][p].x < bd[j]) bd[j] = acc[j][p].x, bi[j] = k;
                    if (k + 1 < n_codes && acc[j][p].y < bd[j]) bd[j] = acc[j][p].y, bi[j] = k + 1;
                }
            if (tile == ntile - 1) {
                // merge the 16 code groups of each query: smaller distance, then lower index
#pragma unroll
                for (int j = 0; j < 4; ++j) {
#pragma unroll
                    for (int o = 1; o < 16; o <<= 1) {
                        const float od = __shfl_xor_sync(0xffffffffu, bd[j], o);
                        const int oi = __shfl_xor_sync(0xffffffffu, bi[j], o);
                        if (od < bd[j] || (od == bd[j] && oi < bi[j])) bd[j] = od, bi[j] = oi;
                    }
                    if (cg == 0) half_idx[half][qg * 4 + j] = bi[j];
                }
            }
        }
        __syncthreads();  // buffer b is refilled by the next iteration's issue
        if (it + 1 < total) store_q(b ^ 1);
    }
    __syncthreads();
    if (tid < kPkmQ && q0 + tid < n) {
        const int a = half_idx[0][tid] * n_codes + half_idx[1][tid];
        addr[q0 + tid] = a;
        if (adapter) adapter[q0 + tid] = table ? table[a] : -1;
    }
}

// dimension-major copy of a codebook: ct[t][k] = c[k][t] (codes k >= n_codes zero)
__global__ void k_pkm_transpose(const float* __restrict__ c, int n_codes, int D, int ncp, float* __restrict__ ct) {
    const size_t total = (size_t)D * ncp;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int t = (int)(i / ncp), k = (int)(i % ncp);
        ct[i] = k < n_codes ? c[(size_t)k * D + t] : 0.f;
    }
}

cudaError_t pkm_assign_launch(const float* queries, int n, const float* ct1, const float* ct2, int n_codes, int ncp,
                              int D, const int32_t* table, int32_t* addr, int32_t* adapter, cudaStream_t s) {
    const void* f = nullptr;
    switch (D) {
        case 32: f = reinterpret_cast<const void*>(&k_pkm_assign<32>); break;
        case 64: f = reinterpret_cast<const void*>(&k_pkm_assign<64>); break;
        case 128: f = reinterpret_cast<const void*>(&k_pkm_assign<128>); break;
        case 256: f = reinterpret_cast<const void*>(&k_pkm_assign<256>); break;
        case 512: f = reinterpret_cast<const void*>(&k_pkm_assign<512>); break;
        default: return cudaErrorInvalidValue;
    }
    if (ncp % kPkmC != 0 || ncp < n_codes) return cudaErrorInvalidValue;
    void* args[] = {&queries, &n, &ct1, &ct2, &n_codes, &ncp, &table, &addr, &adapter};
    const size_t smem = (size_t)2 * kPkmDc * (kPkmQ + kPkmC) * 4;  // 48 KB: above the default with the static part
    cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
    if (e != cudaSuccess) return e;
    return cudaLaunchKernel(f, dim3((n + kPkmQ - 1) / kPkmQ), dim3(kPkmThreads), args, smem, s);
}

cudaError_t pkm_transpose_launch(const float* c, int n_codes, int D, int ncp, float* ct, cudaStream_t s) {
    k_pkm_transpose<<<256, 256, 0, s>>>(c, n_codes, D, ncp, ct);
    return cudaGetLastError();
}

}  // namespace ti

using namespace ti;

struct ti_pkm {
    int dev = 0, n_codes = 0, D = 0, ncp = 0;
    float *c1 = nullptr, *c2 = nullptr;  // dimension-major [D][ncp] (ncp = n_codes padded to 128)
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
    p->ncp = (n_codes + 127) / 128 * 128;
    const size_t cb = (size_t)n_codes * half_dim * 4;
    const size_t ctb = (size_t)p->ncp * half_dim * 4;
    const size_t tb = (size_t)n_codes * n_codes * 4;
    float* stage = nullptr;  // row-major upload, transposed on the device
    cudaError_t e = cudaMalloc(&p->c1, ctb);
    if (e == cudaSuccess) e = cudaMalloc(&p->c2, ctb);
    if (e == cudaSuccess) e = cudaMalloc(&p->table, tb);
    if (e == cudaSuccess) e = cudaMalloc(&stage, cb);
    if (e == cudaSuccess) e = cudaMemcpy(stage, c1_host, cb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = pkm_transpose_launch(stage, n_codes, half_dim, p->ncp, p->c1, 0);
    if (e == cudaSuccess) e = cudaMemcpy(stage, c2_host, cb, cudaMemcpyHostToDevice);
    if (e == cudaSuccess) e = pkm_transpose_launch(stage, n_codes, half_dim, p->ncp, p->c2, 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    cudaFree(stage);
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
    if (e == cudaSuccess) e = pkm_assign_launch(dq, n, p->c1, p->c2, p->n_codes, p->ncp, p->D, nullptr, da, nullptr, 0);
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
    TI_CUDA(pkm_assign_launch(queries, n, p->c1, p->c2, p->n_codes, p->ncp, p->D, p->table, addr, adapter,
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
        e = pkm_assign_launch(dq, n, p->c1, p->c2, p->n_codes, p->ncp, p->D, p->table, dout, dout + n, 0);
    if (e == cudaSuccess) e = cudaMemcpy(addr, dout, (size_t)n * 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess && adapter) e = cudaMemcpy(adapter, dout + n, (size_t)n * 4, cudaMemcpyDeviceToHost);
    cudaFree(dq);
    cudaFree(dout);
    TI_CHECK(e == cudaSuccess, TI_ERR_CUDA, "pkm_query_host: %s", cudaGetErrorString(e));
    return TI_OK;
}

}  // extern "C"
