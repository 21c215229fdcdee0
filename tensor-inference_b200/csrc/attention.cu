// attention.cu — decode attention over the paged KV cache.
//
// One kernel replaces, per layer and step, the reference's
//   ops::rope(q), ops::rope(k)              (ops.cu:210-312)
//   raw cudaMemcpy of K/V into the cache     (llama_model.cpp:155-171)
//   ops::slice(cache) x2                     (ops.cu:648-665, a prefix copy each)
//   ops::attention(q, k_ctx, v_ctx)          (ops.cu:444-544: casts, per-head SGEMM
//                                             loop, softmax)
// Grid (split, kv head, token): each CTA takes one kv head and all q heads of
// its GQA group (q head g reads kv head g / group, ops.cu:470), so a K/V row is
// read once per group; the context [lo, pos] is cut into n_splits ranges
// ("flash-decoding") whose partial (max, sum, unnormalised output) are merged
// by the last CTA to finish (atomic ticket), with no second launch.
// Arithmetic follows the reference: RoPE in fp32 rounded to bf16,
// score = scale * dot(q, k) in fp32, exp-normalised fp32 softmax, fp32 P.V,
// bf16 output.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>

namespace ti {

constexpr int kAttnThreads = 128;
constexpr int kAttnMaxGroup = 16;
constexpr int kPage = 16;

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(const AttnArgs a) {
    extern __shared__ __align__(16) float sm[];
    constexpr int HALF = HD / 2;
    constexpr int DPL = HD / 32;  // dims per lane in the score loop
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.nq / a.nkv;

    float* qs = sm;               // [G][HD]
    float* ks = qs + G * HD;      // [HD]
    float* vs = ks + HD;          // [HD]
    float* ml = vs + HD;          // [G][2]
    float* sc = ml + 2 * kAttnMaxGroup;  // [G][max_chunk]
    __shared__ int s_last;

    pdl_wait();
    const int pos = a.pos[b];
    const int* pt = a.page_table + (size_t)a.seq[b] * a.pt_stride;
    const int L = pos + 1;
    const int window = a.window ? *a.window : -1;
    const int lo = window > 0 ? max(0, pos - window + 1) : 0;
    const int span = L - lo;
    const int chunk = (span + a.n_splits - 1) / a.n_splits;
    const int t0 = lo + split * chunk;
    int t1 = min(L, t0 + chunk);
    if (t1 - t0 > a.max_chunk) {  // host sizes n_splits so this cannot happen; never overrun smem
        if (tid == 0 && a.err) atomicOr(a.err, kErrBadIndex);
        t1 = t0 + a.max_chunk;
    }
    const int n = max(0, t1 - t0);

    // ---- RoPE on the group's q heads and the new k (ops.cu:224-232); v as is
    const uint16_t* row = a.qkv + (size_t)b * a.qkv_stride;
    for (int task = tid; task < (G + 1) * HALF; task += kAttnThreads) {
        const int hh = task / HALF, i = task - hh * HALF;
        const uint16_t* src = hh < G ? row + (size_t)(h * G + hh) * HD : row + (size_t)(a.nq + h) * HD;
        const float x0 = __uint_as_float((uint32_t)src[i] << 16);
        const float x1 = __uint_as_float((uint32_t)src[i + HALF] << 16);
        const float ang = (float)pos * a.freqs[i];
        const float c = cosf(ang), s = sinf(ang);
        float* dst = hh < G ? qs + hh * HD : ks;
        dst[i] = round_bf(x0 * c - x1 * s);
        dst[i + HALF] = round_bf(x0 * s + x1 * c);
    }
    for (int d = tid; d < HD; d += kAttnThreads)
        vs[d] = __uint_as_float((uint32_t)row[(size_t)(a.nq + a.nkv + h) * HD + d] << 16);
    __syncthreads();

    // ---- the CTA whose range holds `pos` appends the new K/V row to its page
    if (pos >= t0 && pos < t1) {
        const int page = pt[pos / kPage];
        if (page < 0 || page >= a.n_pages) {  // unreserved page: report, never write out of the pool
            if (tid == 0 && a.err) atomicOr(a.err, kErrBadIndex);
            return;
        }
        const size_t off = (((size_t)page * a.nkv + h) * kPage + (pos % kPage)) * HD;
        for (int d = tid; d < HD; d += kAttnThreads) {
            reinterpret_cast<bf16*>(a.kc)[off + d] = f2bf(ks[d]);
            reinterpret_cast<bf16*>(a.vc)[off + d] = f2bf(vs[d]);
        }
    }

    // ---- scores: warp per token, lane per DPL dims
    for (int j = t0 + warp; j < t1; j += kAttnThreads / 32) {
        float kv[DPL];
        if (j == pos) {
#pragma unroll
            for (int e = 0; e < DPL; ++e) kv[e] = ks[lane * DPL + e];
        } else {
            const int page = pt[j / kPage];
            const uint16_t* kp = a.kc + (((size_t)page * a.nkv + h) * kPage + (j % kPage)) * HD + lane * DPL;
#pragma unroll
            for (int e = 0; e < DPL; ++e) kv[e] = __uint_as_float((uint32_t)kp[e] << 16);
        }
        for (int g = 0; g < G; ++g) {
            float d = 0.f;
#pragma unroll
            for (int e = 0; e < DPL; ++e) d = fmaf(qs[g * HD + lane * DPL + e], kv[e], d);
            d = warp_sum(d);
            if (lane == 0) sc[g * a.max_chunk + (j - t0)] = a.scale * d;
        }
    }
    __syncthreads();

    // ---- softmax statistics per q head (ops.cu:393-419)
    for (int g = warp; g < G; g += kAttnThreads / 32) {
        float m = -INFINITY;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[g * a.max_chunk + j]);
        m = warp_max(m);
        float l = 0.f;
        for (int j = lane; j < n; j += 32) {
            const float p = n > 0 ? expf(sc[g * a.max_chunk + j] - m) : 0.f;
            sc[g * a.max_chunk + j] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) {
            ml[2 * g] = m;
            ml[2 * g + 1] = l;
        }
    }
    __syncthreads();

    // ---- P.V (ops.cu:526-539): thread -> dims
    constexpr int TG = HD >= kAttnThreads ? 1 : kAttnThreads / HD;  // token groups
    constexpr int DPT = HD >= kAttnThreads ? HD / kAttnThreads : 1;  // dims per thread
    float acc[kAttnMaxGroup][DPT];
#pragma unroll
    for (int g = 0; g < kAttnMaxGroup; ++g)
#pragma unroll
        for (int e = 0; e < DPT; ++e) acc[g][e] = 0.f;
    const int dbase = HD >= kAttnThreads ? tid : tid % HD;
    const int tgrp = HD >= kAttnThreads ? 0 : tid / HD;
    for (int jj = tgrp; jj < n; jj += TG) {
        const int j = t0 + jj;
        float v[DPT];
        if (j == pos) {
#pragma unroll
            for (int e = 0; e < DPT; ++e) v[e] = vs[dbase + e * kAttnThreads];
        } else {
            const int page = pt[j / kPage];
            const uint16_t* vp = a.vc + (((size_t)page * a.nkv + h) * kPage + (j % kPage)) * HD;
#pragma unroll
            for (int e = 0; e < DPT; ++e) v[e] = __uint_as_float((uint32_t)vp[dbase + e * kAttnThreads] << 16);
        }
#pragma unroll
        for (int g = 0; g < kAttnMaxGroup; ++g) {
            if (g < G) {
                const float p = sc[g * a.max_chunk + jj];
#pragma unroll
                for (int e = 0; e < DPT; ++e) acc[g][e] = fmaf(p, v[e], acc[g][e]);
            }
        }
    }
    if (TG > 1) {
        // fold token groups into group 0 through shared memory (reuse the score area)
        __syncthreads();
        float* red = sc;
        if (tgrp > 0)
#pragma unroll
            for (int g = 0; g < kAttnMaxGroup; ++g)
                if (g < G) red[((tgrp - 1) * G + g) * HD + dbase] = acc[g][0];
        __syncthreads();
        if (tgrp == 0)
            for (int t = 1; t < TG; ++t)
#pragma unroll
                for (int g = 0; g < kAttnMaxGroup; ++g)
                    if (g < G) acc[g][0] += red[((t - 1) * G + g) * HD + dbase];
    }

    if (a.n_splits == 1) {
        if (tgrp == 0)
#pragma unroll
            for (int g = 0; g < kAttnMaxGroup; ++g)
                if (g < G) {
                    const float l = ml[2 * g + 1];
#pragma unroll
                    for (int e = 0; e < DPT; ++e)
                        reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + (size_t)(h * G + g) * HD + dbase +
                                                       e * kAttnThreads] = f2bf(acc[g][e] / l);
                }
        return;
    }

    // ---- partial results, merged by the last CTA of this (token, kv head)
    const size_t pbase = (((size_t)b * a.nkv + h) * a.n_splits + split) * G;
    if (tgrp == 0)
#pragma unroll
        for (int g = 0; g < kAttnMaxGroup; ++g)
            if (g < G)
#pragma unroll
                for (int e = 0; e < DPT; ++e) a.part_o[(pbase + g) * HD + dbase + e * kAttnThreads] = acc[g][e];
    if (tid < G) {
        a.part_ml[(pbase + tid) * 2] = ml[2 * tid];
        a.part_ml[(pbase + tid) * 2 + 1] = ml[2 * tid + 1];
    }
    __threadfence();
    __syncthreads();
    if (tid == 0) {
        const unsigned int t = atomicAdd(&a.counters[b * a.nkv + h], 1u);
        s_last = (t == (unsigned)a.n_splits - 1);
    }
    __syncthreads();
    if (!s_last) return;
    __threadfence();
    const size_t p0 = ((size_t)b * a.nkv + h) * a.n_splits * G;
    for (int idx = tid; idx < G * HD; idx += kAttnThreads) {
        const int g = idx / HD, d = idx - g * HD;
        float M = -INFINITY;
        for (int s = 0; s < a.n_splits; ++s) {
            const float l = __ldcg(&a.part_ml[(p0 + (size_t)s * G + g) * 2 + 1]);
            if (l > 0.f) M = fmaxf(M, __ldcg(&a.part_ml[(p0 + (size_t)s * G + g) * 2]));
        }
        float Ls = 0.f, O = 0.f;
        for (int s = 0; s < a.n_splits; ++s) {
            const size_t q = p0 + (size_t)s * G + g;
            const float l = __ldcg(&a.part_ml[q * 2 + 1]);
            if (l > 0.f) {
                const float w = expf(__ldcg(&a.part_ml[q * 2]) - M);
                Ls = fmaf(l, w, Ls);
                O = fmaf(__ldcg(&a.part_o[q * HD + d]), w, O);
            }
        }
        reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + (size_t)(h * G + g) * HD + d] = f2bf(O / Ls);
    }
    if (tid == 0) a.counters[b * a.nkv + h] = 0u;
}

int attn_splits(int nb, int nkv, int max_len, int sms, int* max_chunk) {
    const int work = std::max(1, nb * nkv);
    const int target = std::max(1, (2 * sms + work - 1) / work);
    const int min_splits = (max_len + 255) / 256;
    int n = std::max(std::min(target, std::max(1, max_len / 16)), min_splits);
    n = std::max(1, n);
    *max_chunk = (max_len + n - 1) / n;
    return n;
}

static size_t attn_smem(int G, int HD, int max_chunk) {
    size_t f = (size_t)G * HD + 2 * HD + 2 * kAttnMaxGroup + (size_t)G * max_chunk;
    const int TG = HD >= kAttnThreads ? 1 : kAttnThreads / HD;
    f = std::max(f, (size_t)G * HD + 2 * HD + 2 * kAttnMaxGroup + (size_t)(TG - 1) * G * HD);
    return f * 4;
}

cudaError_t attn_launch(const AttnArgs& a, cudaStream_t s, bool pdl) {
    if (a.nkv <= 0 || a.nq % a.nkv != 0 || a.nq / a.nkv > kAttnMaxGroup) return cudaErrorInvalidValue;
    const void* f = nullptr;
    switch (a.hd) {
        case 64: f = reinterpret_cast<const void*>(&k_attn_decode<64>); break;
        case 128: f = reinterpret_cast<const void*>(&k_attn_decode<128>); break;
        case 256: f = reinterpret_cast<const void*>(&k_attn_decode<256>); break;
        default: return cudaErrorInvalidValue;
    }
    const size_t smem = attn_smem(a.nq / a.nkv, a.hd, a.max_chunk);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    AttnArgs args = a;
    void* params[] = {&args};
    return launch_pdl(f, dim3(a.n_splits, a.nkv, a.nb), dim3(kAttnThreads), smem, s, params, pdl);
}

}  // namespace ti
