// lora.cu — LoRA "shrink" step: t[b, :] = bf16(x_b @ A^T) for each token's adapter.
//
// The reference's apply_lora (qwen_adapter_model.cpp:22-30) computes
// down = matmul_t(x, lora_A) (rounded to bf16), up = matmul_t(down, lora_B),
// delta = up * (alpha / rank), and add_if_present adds it to the base
// projection (:35-43).  Here `down` is this kernel's output; the weight-streaming
// GEMV that produces the base projection applies the expansion in its epilogue.
// Per-token adapters make it a segmented gather: token b reads the A rows of
// adapter[b] (no adapter: nothing is written and the GEMV skips the delta); the
// grid runs over (row tile, adapter), the adapter's tokens are the rows of
// tensor-core mma tiles, so an adapter's rows are read once for all its tokens.
// x is the projection's input: RMSNorm(hidden) for q|k|v and gate|up (the same
// normalised row the reference passes to both the base and the LoRA matmul),
// the attention output for o, the SwiGLU activation for down.
#include <algorithm>

#include "common.cuh"
#include "kernels.h"

namespace ti {

// ---- shared helpers
// Tokens b < nb with adapter[b] == ad, ascending, into list (warp 0; ballot
// compaction); returns their count to every thread.
__device__ __forceinline__ int adapter_tokens(const int32_t* adapter, int nb, int ad, int* list, int* s_n) {
    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    if (warp == 0) {
        int n = 0;
        for (int base = 0; base < nb; base += 32) {
            const int b = base + lane;
            const bool m = b < nb && adapter[b] == ad;
            const unsigned int bal = __ballot_sync(0xffffffffu, m);
            if (m) list[n + __popc(bal & ((1u << lane) - 1u))] = b;
            n += __popc(bal);
        }
        if (lane == 0) *s_n = n;
    }
    __syncthreads();
    return *s_n;
}
TI_DEVICE_INLINE void ldsm_x4_l(uint32_t addr, uint32_t* r) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3])
                 : "r"(addr));
}
// D(16x8 fp32) += A(16x16 bf16, row) * B(16x8 bf16, col)
TI_DEVICE_INLINE void mma_bf16_16816(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
TI_DEVICE_INLINE uint32_t ldg_u32(const uint16_t* p) { return *reinterpret_cast<const uint32_t*>(p); }

// ---- shrink on the tensor cores: t[b, r] = x_b . A[ad_b][r] for the adapter's
//      tokens (mma rows, 16 at a time).  Grid (32-row tile of A, adapter,
//      K slice); warp w of a CTA takes the k-steps (16 columns) w, w + 8, ... of
//      its slice, with x and A fragments loaded straight from global memory (x
//      rows are small and L2-resident; each A row is read once per adapter).
//      The 8 warps' sums are added in warp order, the slices' by the last CTA of
//      the tile in slice order.  RMSNorm of x (when the projection's input is
//      the unnormalised hidden state) is applied to the fragments, with the
//      per-token scale reduced in the base projection's order (ops.cu:179).
constexpr int kShrinkThreads = 256;
constexpr int kShrinkWarps = kShrinkThreads / 32;
constexpr int kShrinkRows = 32;  // 4 n-tiles of 8 A rows
constexpr int kShrinkUnroll = 4;  // k-steps per warp with their loads in flight together

TI_DEVICE_INLINE uint32_t norm_pair(uint32_t v, uint32_t w, float sc, float off) {
    return pack_bf2(bf_lo(v) * sc * (bf_lo(w) + off), bf_hi(v) * sc * (bf_hi(w) + off));
}

__global__ void __launch_bounds__(kShrinkThreads) k_lora_shrink(const LoraShrinkArgs a, int ksplit, int kr) {
    extern __shared__ __align__(16) uint8_t smem[];
    float* red = reinterpret_cast<float*>(smem);                                  // [warps][16][32]
    int* list = reinterpret_cast<int*>(red + kShrinkWarps * 16 * kShrinkRows);    // [nb]
    __shared__ float sred[16][kShrinkWarps];
    __shared__ float sscale[16];
    __shared__ int s_n, s_last;
    const int ad = blockIdx.y, rt = blockIdx.x, ksl = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, q = lane & 3;
    if (tid == 0) pdl_trigger();
    // the adapter ids come with the step descriptor, not from the previous kernel
    const int n = adapter_tokens(a.adapter, a.nb, ad, list, &s_n);
    if (n == 0 || ad >= a.n_adapters) return;
    pdl_wait();
    const int K = a.K;
    const uint16_t* A = a.A + (size_t)ad * a.A_adapter_stride;
    const int r0 = rt * kShrinkRows;
    const int ntv = min(4, (a.T - r0) / 8);  // n-tiles inside T (T % 16 == 0)
    const int kb = ksl * kr, ke = min(K, kb + kr);
    const float off = a.norm_offset ? 1.0f : 0.0f;
    const uint16_t* arow[4];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) arow[nt] = A + (size_t)(r0 + (nt < ntv ? nt : 0) * 8 + g) * K + 2 * q;

    for (int m0 = 0; m0 < n; m0 += 16) {
        const int mt = min(16, n - m0);
        if (a.norm_w) {
            // the tokens' RMSNorm scales: per-thread strided sums, warp butterfly,
            // warp-ordered total (the base projection's prologue)
            for (int j = 0; j < mt; ++j) {
                const uint16_t* x = a.x + (size_t)list[m0 + j] * a.x_stride;
                float ss = 0.f;
                for (int c = tid * 8; c < K; c += kShrinkThreads * 8) {
                    const uint4 v = *reinterpret_cast<const uint4*>(x + c);
                    const uint32_t* vp = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
                    for (int e = 0; e < 4; ++e) {
                        ss = fmaf(bf_lo(vp[e]), bf_lo(vp[e]), ss);
                        ss = fmaf(bf_hi(vp[e]), bf_hi(vp[e]), ss);
                    }
                }
                ss = warp_sum(ss);
                if (lane == 0) sred[j][warp] = ss;
            }
            __syncthreads();
            if (tid < mt) {
                float tot = 0.f;
#pragma unroll
                for (int w = 0; w < kShrinkWarps; ++w) tot += sred[tid][w];
                sscale[tid] = rsqrtf(tot / (float)K + a.eps);
            }
            __syncthreads();
        }
        // this lane's two token rows (g, g + 8); absent tokens read as zero
        const bool v0 = g < mt, v1 = g + 8 < mt;
        const uint16_t* x0 = a.x + (size_t)(v0 ? list[m0 + g] : list[m0]) * a.x_stride + 2 * q;
        const uint16_t* x1 = a.x + (size_t)(v1 ? list[m0 + g + 8] : list[m0]) * a.x_stride + 2 * q;
        const float sc0 = a.norm_w && v0 ? sscale[g] : 0.f, sc1 = a.norm_w && v1 ? sscale[g + 8] : 0.f;
        float acc[4][4];
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) acc[nt][0] = acc[nt][1] = acc[nt][2] = acc[nt][3] = 0.f;
        for (int k0 = kb + warp * 16; k0 < ke; k0 += kShrinkWarps * 16 * kShrinkUnroll) {
            uint32_t xf[kShrinkUnroll][4], bf[kShrinkUnroll][4][2];
#pragma unroll
            for (int u = 0; u < kShrinkUnroll; ++u) {
                const int k = k0 + u * kShrinkWarps * 16;
                const bool in = k < ke;
                xf[u][0] = in && v0 ? ldg_u32(x0 + k) : 0u;
                xf[u][1] = in && v1 ? ldg_u32(x1 + k) : 0u;
                xf[u][2] = in && v0 ? ldg_u32(x0 + k + 8) : 0u;
                xf[u][3] = in && v1 ? ldg_u32(x1 + k + 8) : 0u;
#pragma unroll
                for (int nt = 0; nt < 4; ++nt) {
                    bf[u][nt][0] = in && nt < ntv ? ldg_u32(arow[nt] + k) : 0u;
                    bf[u][nt][1] = in && nt < ntv ? ldg_u32(arow[nt] + k + 8) : 0u;
                }
            }
#pragma unroll
            for (int u = 0; u < kShrinkUnroll; ++u) {
                const int k = k0 + u * kShrinkWarps * 16;
                if (k >= ke) break;  // warp-uniform
                if (a.norm_w) {
                    const uint32_t w0 = ldg_u32(a.norm_w + k + 2 * q), w1 = ldg_u32(a.norm_w + k + 8 + 2 * q);
                    xf[u][0] = norm_pair(xf[u][0], w0, sc0, off);
                    xf[u][1] = norm_pair(xf[u][1], w0, sc1, off);
                    xf[u][2] = norm_pair(xf[u][2], w1, sc0, off);
                    xf[u][3] = norm_pair(xf[u][3], w1, sc1, off);
                }
#pragma unroll
                for (int nt = 0; nt < 4; ++nt)
                    if (nt < ntv) mma_bf16_16816(acc[nt], xf[u], bf[u][nt][0], bf[u][nt][1]);
            }
        }
        // the 8 warps' sums, added in warp order
        if (m0 > 0) __syncthreads();  // red of the previous m-tile consumed
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            float* rw = red + (size_t)warp * 16 * kShrinkRows + nt * 8 + 2 * q;
            rw[g * kShrinkRows] = acc[nt][0];
            rw[g * kShrinkRows + 1] = acc[nt][1];
            rw[(g + 8) * kShrinkRows] = acc[nt][2];
            rw[(g + 8) * kShrinkRows + 1] = acc[nt][3];
        }
        __syncthreads();
        for (int i = tid; i < mt * kShrinkRows; i += kShrinkThreads) {
            const int j = i / kShrinkRows, rr = i - j * kShrinkRows, r = r0 + rr;
            if (r >= a.T) continue;
            float v = 0.f;
#pragma unroll
            for (int w = 0; w < kShrinkWarps; ++w) v += red[((size_t)w * 16 + j) * kShrinkRows + rr];
            const int b = list[m0 + j];
            if (ksplit > 1) {
                a.ws[((size_t)ksl * a.nb + b) * a.t_stride + r] = v;
            } else if (a.tp) {
                // row-parallel under tensor parallelism: fp32 partial to every rank
                for (int qq = 0; qq < a.tp; ++qq) a.peer_t[qq][(size_t)b * a.t_stride + r] = v;
            } else {
                a.t[(size_t)b * a.t_stride + r] = round_bf(v);
            }
        }
    }
    if (ksplit > 1) {
        // the last CTA of this (tile, adapter) adds the slices in order
        __threadfence();
        __syncthreads();
        unsigned int* ctr = a.ctr + (size_t)ad * ((a.T + kShrinkRows - 1) / kShrinkRows) + rt;
        if (tid == 0) s_last = atomicAdd(ctr, 1u) == (unsigned)ksplit - 1;
        __syncthreads();
        if (!s_last) return;
        __threadfence();
        for (int i = tid; i < n * kShrinkRows; i += kShrinkThreads) {
            const int j = i / kShrinkRows, rr = i - j * kShrinkRows, r = r0 + rr;
            if (r >= a.T) continue;
            const int b = list[j];
            float v = 0.f;
            for (int s = 0; s < ksplit; ++s) v += __ldcg(&a.ws[((size_t)s * a.nb + b) * a.t_stride + r]);
            if (a.tp) {
                for (int qq = 0; qq < a.tp; ++qq) a.peer_t[qq][(size_t)b * a.t_stride + r] = v;
            } else {
                a.t[(size_t)b * a.t_stride + r] = round_bf(v);
            }
        }
        if (tid == 0) *ctr = 0u;
    }
    if (a.tp) __threadfence_system();
}

cudaError_t lora_shrink_launch(const LoraShrinkArgs& a, cudaStream_t s, bool pdl) {
    if (a.K % 16 != 0 || a.T <= 0 || a.T % 16 != 0 || a.nb < 1 || a.n_adapters < 1) return cudaErrorInvalidValue;
    const int tiles = (a.T + kShrinkRows - 1) / kShrinkRows;
    // K slices: about two CTAs per SM over the (tile, adapter) pairs, slices of
    // at least 1024 columns, a multiple of 16
    int sms = 148, dev = 0;
    if (cudaGetDevice(&dev) == cudaSuccess) cudaDeviceGetAttribute(&sms, cudaDevAttrMultiProcessorCount, dev);
    int ksplit = 1;
    if (a.ws && a.ctr) {
        const long pairs = (long)tiles * a.n_adapters;
        ksplit = (int)std::max<long>(1, (2L * sms + pairs - 1) / pairs);
        ksplit = std::min(ksplit, std::max(1, a.K / 1024));
        ksplit = std::min(ksplit, kLoraMaxSplit);
    }
    int kr = (a.K + ksplit - 1) / ksplit;
    kr = (kr + 15) / 16 * 16;
    ksplit = (a.K + kr - 1) / kr;
    LoraShrinkArgs args = a;
    void* params[] = {&args, &ksplit, &kr};
    const size_t smem = (size_t)kShrinkWarps * 16 * kShrinkRows * 4 + (size_t)a.nb * 4;
    const void* f = reinterpret_cast<const void*>(&k_lora_shrink);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(f, dim3(tiles, a.n_adapters, ksplit), dim3(kShrinkThreads), smem, s, params, pdl);
}


// ---- expansion ahead of the tensor-core GEMM, on the tensor cores:
//      dval[b, n] = bf16(bf16(sum_r t[b, r] B[ad][n, r]) * scale[ad]) for the
//      adapter's tokens, 16 at a time (mma rows).  CTA (128 output rows,
//      adapter), 4 warps of 4 n-tiles; t staged in shared memory as bf16 (its
//      values are bf16 already), B fragments read straight from global memory:
//      each B row is read once per adapter.
constexpr int kExpandThreads = 128;

template <int KS>  // rank / 16 mma k-steps
__global__ void __launch_bounds__(kExpandThreads)
    k_lora_expand(const GemvLora L, int nb, int n_rows, int glu_n, uint16_t* dval, int dval_stride) {
    extern __shared__ __align__(16) uint8_t smem[];
    const int tw = L.t_stride + 8;                                        // staged row width (bf16)
    uint16_t* ts = reinterpret_cast<uint16_t*>(smem);                    // [16][tw]
    int* list = reinterpret_cast<int*>(smem + (size_t)16 * tw * 2);      // [nb]
    __shared__ int s_n;
    constexpr int R = KS * 16;
    const int ad = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int g = lane >> 2, q = lane & 3;
    if (tid == 0) pdl_trigger();
    const int n = adapter_tokens(L.adapter, nb, ad, list, &s_n);  // tokens without an adapter: no CTA
    if (n == 0 || ad >= L.n_adapters) return;
    const uint16_t* Bad = L.B + (size_t)ad * L.B_adapter_stride;
    const float sc = L.scale[ad];
    const int row0 = blockIdx.x * 128 + warp * 32;
    const int nt_n = max(0, min(4, (n_rows - row0) / 8));  // this warp's n-tiles (n_rows % 8 == 0)
    // B fragments of the warp's n-tiles (adapter weights: not the previous kernel's output)
    uint32_t bf[4][KS][2];
#pragma unroll
    for (int nt = 0; nt < 4; ++nt) {
        const uint16_t* br = Bad + (size_t)(row0 + (nt < nt_n ? nt : 0) * 8 + g) * R + 2 * q;
#pragma unroll
        for (int k = 0; k < KS; ++k) {
            bf[nt][k][0] = nt < nt_n ? ldg_u32(br + k * 16) : 0u;
            bf[nt][k][1] = nt < nt_n ? ldg_u32(br + k * 16 + 8) : 0u;
        }
    }
    const uint32_t tbase = smem_u32(ts) + (uint32_t)(((lane & 7) + ((lane >> 3) & 1) * 8) * tw + (lane >> 4) * 8) * 2u;
    pdl_wait();  // t is the previous kernel's output
    for (int m0 = 0; m0 < n; m0 += 16) {
        const int mt = min(16, n - m0);
        if (m0 > 0) __syncthreads();
        for (int i = tid; i < 16 * L.t_stride; i += kExpandThreads) {
            const int j = i / L.t_stride, k = i - j * L.t_stride;
            const float v = j < mt ? L.t[(size_t)list[m0 + j] * L.t_stride + k] : 0.f;
            ts[(size_t)j * tw + k] = __bfloat16_as_ushort(f2bf(v));
        }
        __syncthreads();
#pragma unroll
        for (int nt = 0; nt < 4; ++nt) {
            if (nt >= nt_n) break;  // warp-uniform
            const int n0 = row0 + nt * 8;
            int sec = 0;
            if (glu_n > 0) sec = n0 >= glu_n;
            else sec = (n0 >= L.sec1) + (n0 >= L.sec2);
            float c[4] = {0.f, 0.f, 0.f, 0.f};
#pragma unroll
            for (int k = 0; k < KS; ++k) {
                uint32_t af[4];
                ldsm_x4_l(tbase + (uint32_t)(sec * R + k * 16) * 2u, af);
                mma_bf16_16816(c, af, bf[nt][k][0], bf[nt][k][1]);
            }
            // c[0..1]: token g, rows n0 + 2q, +1; c[2..3]: token g + 8
            if (g < mt)
                *reinterpret_cast<uint32_t*>(dval + (size_t)list[m0 + g] * dval_stride + n0 + 2 * q) =
                    pack_bf2(round_bf(c[0]) * sc, round_bf(c[1]) * sc);
            if (g + 8 < mt)
                *reinterpret_cast<uint32_t*>(dval + (size_t)list[m0 + g + 8] * dval_stride + n0 + 2 * q) =
                    pack_bf2(round_bf(c[2]) * sc, round_bf(c[3]) * sc);
        }
    }
}

// ranks above 128: one output row per thread, CTA (row tile, token); the same
// element order as the GEMV epilogue's expansion
__global__ void __launch_bounds__(kExpandThreads)
    k_lora_expand_rows(const GemvLora L, int nb, int n_rows, int glu_n, uint16_t* dval, int dval_stride) {
    if (threadIdx.x == 0) pdl_trigger();
    const int b = blockIdx.y;
    const int ad = L.adapter[b];
    pdl_wait();
    if (ad < 0 || ad >= L.n_adapters || b >= nb) return;  // the epilogue skips tokens without an adapter
    const int row = blockIdx.x * kExpandThreads + threadIdx.x;
    if (row >= n_rows) return;
    int sec = 0;
    if (glu_n > 0) sec = row >= glu_n;
    else sec = (row >= L.sec1) + (row >= L.sec2);
    const uint16_t* br = L.B + (size_t)ad * L.B_adapter_stride + (size_t)row * L.rank;
    const float* t = L.t + (size_t)b * L.t_stride + sec * L.rank;
    float s = 0.f;  // the same element order as the GEMV epilogue's expansion
    for (int i = 0; i < L.rank; i += 8) {
        const uint4 w = *reinterpret_cast<const uint4*>(br + i);
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            s = fmaf(bf_lo(wp[e]), t[i + 2 * e], s);
            s = fmaf(bf_hi(wp[e]), t[i + 2 * e + 1], s);
        }
    }
    dval[(size_t)b * dval_stride + row] = __bfloat16_as_ushort(f2bf(round_bf(s) * L.scale[ad]));
}

cudaError_t lora_expand_launch(const GemvLora& L, int nb, int n_rows, int glu_n, uint16_t* dval, int dval_stride,
                               cudaStream_t s, bool pdl) {
    if (!L.adapter || L.rank % 16 != 0 || nb < 1 || L.n_adapters < 1 || n_rows % 8 != 0 || dval_stride % 2 != 0 ||
        L.t_stride % 8 != 0)
        return cudaErrorInvalidValue;
    const void* f = nullptr;
    switch (L.rank / 16) {
        case 1: f = reinterpret_cast<const void*>(&k_lora_expand<1>); break;
        case 2: f = reinterpret_cast<const void*>(&k_lora_expand<2>); break;
        case 3: f = reinterpret_cast<const void*>(&k_lora_expand<3>); break;
        case 4: f = reinterpret_cast<const void*>(&k_lora_expand<4>); break;
        case 5: f = reinterpret_cast<const void*>(&k_lora_expand<5>); break;
        case 6: f = reinterpret_cast<const void*>(&k_lora_expand<6>); break;
        case 7: f = reinterpret_cast<const void*>(&k_lora_expand<7>); break;
        case 8: f = reinterpret_cast<const void*>(&k_lora_expand<8>); break;
        default: break;
    }
    GemvLora args = L;
    void* params[] = {&args, &nb, &n_rows, &glu_n, &dval, &dval_stride};
    if (!f)
        return launch_pdl(reinterpret_cast<const void*>(&k_lora_expand_rows),
                          dim3((n_rows + kExpandThreads - 1) / kExpandThreads, nb), dim3(kExpandThreads), 0, s, params,
                          pdl);
    const size_t smem = (size_t)16 * (L.t_stride + 8) * 2 + (size_t)nb * 4;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(f, dim3((n_rows + 127) / 128, L.n_adapters), dim3(kExpandThreads), smem, s, params, pdl);
}

}  // namespace ti
