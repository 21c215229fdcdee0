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
//
// Latency structure: cached K/V rows (positions < pos) were written by earlier
// steps, so each CTA bulk-copies its page spans (16 tokens x head_dim bf16 are
// contiguous per kv head) into shared memory BEFORE griddepcontrol.wait; only
// the new token's q/k/v come from the previous kernel.
// Arithmetic follows the reference: RoPE in fp32 rounded to bf16,
// score = scale * dot(q, k) in fp32, exp-normalised fp32 softmax, fp32 P.V,
// bf16 output.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cstdlib>

namespace ti {

constexpr int kAttnThreads = 128;
constexpr int kAttnMaxGroup = 16;
constexpr int kPage = 16;
constexpr int kAttnChunkCap = 64;  // tokens per CTA (shared-memory K/V tiles)

struct AttnSmem {
    uint32_t q, k, v, ml, sc, kbuf, vbuf, bar, total;
};

// sc_floats: floats reserved for the score area (also reused by the token-group
// fold and by the split merge)
__host__ __device__ inline AttnSmem attn_layout(int G, int HD, int max_chunk, int sc_floats) {
    AttnSmem L;
    uint32_t o = 0;
    L.q = o;
    o += G * HD * 4;
    L.k = o;
    o += HD * 4;
    L.v = o;
    o += HD * 4;
    L.ml = o;
    o += 2 * kAttnMaxGroup * 4;
    L.sc = o;
    o += sc_floats * 4;
    o = (o + 127u) & ~127u;
    L.kbuf = o;
    o += max_chunk * HD * 2;
    L.vbuf = o;
    o += max_chunk * HD * 2;
    L.bar = o;
    o += 16;
    L.total = o;
    return L;
}

__host__ __device__ inline int attn_sc_floats(int G, int HD, int max_chunk, int n_splits) {
    const int TG = HD >= kAttnThreads ? 1 : kAttnThreads / HD;
    int f = G * max_chunk;
    if ((TG - 1) * G * HD > f) f = (TG - 1) * G * HD;
    if (n_splits * G > f) f = n_splits * G;
    return f;
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads) k_attn_decode(const AttnArgs a) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int HALF = HD / 2;
    constexpr int DPL = HD / 32;  // dims per lane in the score loop
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.nq / a.nkv;
    const AttnSmem L = attn_layout(G, HD, a.max_chunk, attn_sc_floats(G, HD, a.max_chunk, a.n_splits));
    float* qs = reinterpret_cast<float*>(smem + L.q);
    float* ks = reinterpret_cast<float*>(smem + L.k);
    float* vs = reinterpret_cast<float*>(smem + L.v);
    float* ml = reinterpret_cast<float*>(smem + L.ml);
    float* sc = reinterpret_cast<float*>(smem + L.sc);
    uint16_t* kbuf = reinterpret_cast<uint16_t*>(smem + L.kbuf);
    uint16_t* vbuf = reinterpret_cast<uint16_t*>(smem + L.vbuf);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);
    __shared__ int s_last;

    // ---- before the dependency wait: state of earlier steps only
    const int pos = a.pos[b];
    const int* pt = a.page_table + (size_t)a.seq[b] * a.pt_stride;
    const int L1 = pos + 1;
    const int window = a.window ? *a.window : a.window_const;
    const int lo = window > 0 ? max(0, pos - window + 1) : 0;
    const int span = L1 - lo;
    const int chunk = (span + a.n_splits - 1) / a.n_splits;
    const int t0 = lo + split * chunk;
    int t1 = min(L1, t0 + chunk);
    if (t1 - t0 > a.max_chunk) {  // host sizes n_splits so this cannot happen; never overrun smem
        if (tid == 0 && a.err) atomicOr(a.err, kErrBadIndex);
        t1 = t0 + a.max_chunk;
    }
    const int n = max(0, t1 - t0);
    const int old_end = min(t1, pos);  // cached tokens [t0, old_end)
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
        bool ok = true;
        uint32_t bytes = 0;
        for (int j = t0; j < old_end;) {
            const int p = j / kPage, j_end = min(old_end, (p + 1) * kPage);
            const int page = pt[p];
            if (page < 0 || page >= a.n_pages) {
                ok = false;
                break;
            }
            bytes += (uint32_t)(j_end - j) * HD * 2 * 2;
            j = j_end;
        }
        if (!ok && a.err) atomicOr(a.err, kErrBadIndex);
        mbar_arrive_expect_tx(bar, ok ? bytes : 0u);
        if (ok)
            for (int j = t0; j < old_end;) {
                const int p = j / kPage, j_end = min(old_end, (p + 1) * kPage);
                const size_t src = (((size_t)pt[p] * a.nkv + h) * kPage + (j % kPage)) * HD;
                const uint32_t nbytes = (uint32_t)(j_end - j) * HD * 2;
                bulk_g2s_plain(kbuf + (size_t)(j - t0) * HD, a.kc + src, nbytes, bar);
                bulk_g2s_plain(vbuf + (size_t)(j - t0) * HD, a.vc + src, nbytes, bar);
                j = j_end;
            }
        pdl_trigger();
    }

    pdl_wait();  // the new token's q/k/v are the previous kernel's output

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
        if (page >= 0 && page < a.n_pages) {
            const size_t off = (((size_t)page * a.nkv + h) * kPage + (pos % kPage)) * HD;
            for (int d = tid; d < HD; d += kAttnThreads) {
                reinterpret_cast<bf16*>(a.kc)[off + d] = f2bf(ks[d]);
                reinterpret_cast<bf16*>(a.vc)[off + d] = f2bf(vs[d]);
            }
        } else if (tid == 0 && a.err) {
            atomicOr(a.err, kErrBadIndex);
        }
    }
    mbar_wait(bar, 0, a.err, kErrTimeoutFull);

    // ---- scores: warp per token, lane per DPL dims, all group heads at once
    for (int j = t0 + warp; j < t1; j += kAttnThreads / 32) {
        float kv[DPL];
        if (j == pos) {
#pragma unroll
            for (int e = 0; e < DPL; ++e) kv[e] = ks[lane * DPL + e];
        } else {
            const uint16_t* kp = kbuf + (size_t)(j - t0) * HD + lane * DPL;
#pragma unroll
            for (int e = 0; e < DPL; ++e) kv[e] = __uint_as_float((uint32_t)kp[e] << 16);
        }
        float d[kAttnMaxGroup];
#pragma unroll
        for (int g = 0; g < kAttnMaxGroup; ++g) {
            d[g] = 0.f;
            if (g < G)
#pragma unroll
                for (int e = 0; e < DPL; ++e) d[g] = fmaf(qs[g * HD + lane * DPL + e], kv[e], d[g]);
        }
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int g = 0; g < kAttnMaxGroup; ++g)
                if (g < G) d[g] += __shfl_xor_sync(0xffffffffu, d[g], o);
        if (lane == 0)
#pragma unroll
            for (int g = 0; g < kAttnMaxGroup; ++g)
                if (g < G) sc[g * a.max_chunk + (j - t0)] = a.scale * d[g];
    }
    __syncthreads();

    // ---- softmax statistics per q head (ops.cu:393-419)
    for (int g = warp; g < G; g += kAttnThreads / 32) {
        float m = -INFINITY;
        for (int j = lane; j < n; j += 32) m = fmaxf(m, sc[g * a.max_chunk + j]);
        m = warp_max(m);
        float l = 0.f;
        for (int j = lane; j < n; j += 32) {
            const float p = expf(sc[g * a.max_chunk + j] - m);
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
#pragma unroll
        for (int e = 0; e < DPT; ++e)
            v[e] = j == pos ? vs[dbase + e * kAttnThreads]
                            : __uint_as_float((uint32_t)vbuf[(size_t)jj * HD + dbase + e * kAttnThreads] << 16);
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
    // split weights w[s][g] = exp(m_s - M_g) (0 for empty splits), kept in the score area
    float* wsg = sc;    // [n_splits][G] maxima, then weights
    float* lsg = qs;    // [n_splits][G] sums (q no longer needed)
    for (int idx = tid; idx < a.n_splits * G; idx += kAttnThreads) {
        wsg[idx] = __ldcg(&a.part_ml[(p0 + idx) * 2]);
        lsg[idx] = __ldcg(&a.part_ml[(p0 + idx) * 2 + 1]);
    }
    __syncthreads();
    if (tid < G) {
        float M = -INFINITY;
        for (int s = 0; s < a.n_splits; ++s)
            if (lsg[s * G + tid] > 0.f) M = fmaxf(M, wsg[s * G + tid]);
        float Ls = 0.f;
        for (int s = 0; s < a.n_splits; ++s) {
            const float l = lsg[s * G + tid];
            const float w = l > 0.f ? expf(wsg[s * G + tid] - M) : 0.f;
            wsg[s * G + tid] = w;
            Ls = fmaf(l, w, Ls);
        }
        ml[2 * tid + 1] = Ls;
    }
    __syncthreads();
    // 4 consecutive (g, d) outputs per thread; the per-split loads are independent
    // float4 reads, so they are all in flight together
    for (int e = tid * 4; e < G * HD; e += kAttnThreads * 4) {
        const int g = e / HD;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll 8
        for (int s = 0; s < a.n_splits; ++s) {
            const float4 v = __ldcg(reinterpret_cast<const float4*>(a.part_o + (p0 + (size_t)s * G) * HD + e));
            const float w = wsg[s * G + g];
            O.x = fmaf(v.x, w, O.x);
            O.y = fmaf(v.y, w, O.y);
            O.z = fmaf(v.z, w, O.z);
            O.w = fmaf(v.w, w, O.w);
        }
        const float inv = ml[2 * g + 1];
        bf16* dst = reinterpret_cast<bf16*>(a.out) + (size_t)b * a.out_stride + (size_t)h * G * HD + e;
        dst[0] = f2bf(O.x / inv);
        dst[1] = f2bf(O.y / inv);
        dst[2] = f2bf(O.z / inv);
        dst[3] = f2bf(O.w / inv);
    }
    if (tid == 0) a.counters[b * a.nkv + h] = 0u;
}

int attn_splits(int nb, int nkv, int max_len, int sms, int* max_chunk) {
    // tokens per CTA are capped by the shared-memory K/V tile (env TI_ATTN_CHUNK, <= 64)
    const char* env = std::getenv("TI_ATTN_CHUNK");
    const int cap = env && std::atoi(env) >= 16 ? std::min(std::atoi(env), kAttnChunkCap) : kAttnChunkCap;
    const int work = std::max(1, nb * nkv);
    const int target = std::max(1, (sms + work - 1) / work);                // about one CTA per SM
    const int by_len = std::max(1, (max_len + 31) / 32);                    // at least ~32 tokens per CTA
    const int min_splits = (max_len + cap - 1) / cap;                      // smem tile bound
    const int n = std::max(std::min(target, by_len), min_splits);
    *max_chunk = (max_len + n - 1) / n;
    return n;
}

size_t attn_scratch_floats(int nb, int nq, int nkv, int hd, int n_splits) {
    const size_t G = (size_t)(nq / nkv);
    return (size_t)nb * nkv * n_splits * G * (hd + 2);
}

cudaError_t attn_launch(const AttnArgs& a, cudaStream_t s, bool pdl) {
    if (a.nkv <= 0 || a.nq % a.nkv != 0 || a.nq / a.nkv > kAttnMaxGroup) return cudaErrorInvalidValue;
    if (a.max_chunk > kAttnChunkCap || a.max_chunk < 1) return cudaErrorInvalidValue;
    const void* f = nullptr;
    switch (a.hd) {
        case 64: f = reinterpret_cast<const void*>(&k_attn_decode<64>); break;
        case 128: f = reinterpret_cast<const void*>(&k_attn_decode<128>); break;
        case 256: f = reinterpret_cast<const void*>(&k_attn_decode<256>); break;
        default: return cudaErrorInvalidValue;
    }
    const int G = a.nq / a.nkv;
    // the merge also stages n_splits x G sums in the q area
    if (a.n_splits * G > G * a.hd) return cudaErrorInvalidValue;
    const size_t smem = attn_layout(G, a.hd, a.max_chunk, attn_sc_floats(G, a.hd, a.max_chunk, a.n_splits)).total;
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    AttnArgs args = a;
    void* params[] = {&args};
    return launch_pdl(f, dim3(a.n_splits, a.nkv, a.nb), dim3(kAttnThreads), smem, s, params, pdl);
}

}  // namespace ti
