// attn_fused.cuh — decode attention of one token, run by the consumer warps of
// the o-projection GEMV (gemv.cu, ATT instances) before the GEMV's prologue.
//
// Replaces, for one layer and one new token, the reference's ops::rope(q, k)
// (ops.cu:210-312), the cudaMemcpy of K/V into the cache (llama_model.cpp:155-171),
// ops::slice x2 and ops::attention (ops.cu:444-544).  While these warps work,
// the GEMV's producer warp has the CTA's o-projection weight rows prefetched
// HBM -> L2 (a path that does not delay the warps' own loads), so HBM does not
// idle during attention; the shared-memory fills from L2 start once the CTA's
// latency-bound loads are done (the `go` barrier).  The separate attention
// kernel and its launch are gone.
//
// Work split: CTA c serves kv head h = c % nkv (grid >= nkv), together with the
// other CTAs of that head; the attended pages [lo/16, pos/16] are dealt out
// page by page, CTA first then warp.  A warp scores one 16-token page at a time
// for all q heads of the group with an online softmax (running max and sum per
// head): lane (t, half) takes token t and half of the dims of every q head for
// q.k (fp32 FMAs over bf16 values; the halves meet in one shuffle), and dims
// [lane * hd/32, +hd/32) of every q head for P.V.  All K loads of a page are
// issued before its arithmetic and its V loads before the softmax; before the
// kernel's dependency wait the warps prefetch their cached pages into L2 (cached
// rows do not depend on the previous kernel).  The warps' partials are merged in
// warp order in shared memory, the CTAs' partials in CTA order by the last CTA
// of the kv head to arrive (atomic ticket), which writes that head group's bf16
// output.  One bounded grid-wide wait (every kv head merged) precedes the GEMV,
// which reads the output as its x.  All CTAs of the grid are resident together:
// one CTA per SM and grid <= SMs; the wait gives up after 2 s and sets
// kErrTimeoutGrid.
//
// Arithmetic follows the reference: RoPE in fp32 rounded to bf16 (the rotated
// k is what the cache stores); scores q.k of bf16 values accumulated in fp32,
// times 1/sqrt(hd); softmax exp-normalised in fp32, evaluated as
// 2^(s log2(e) - m) with ex2.approx; P.V in fp32; output rounded to bf16.
#pragma once
#include <type_traits>

#include "common.cuh"
#include "kernels.h"

namespace ti {

constexpr int kAttnPageTokens = 16;
constexpr float kAttnLog2e = 1.4426950408889634f;
constexpr int kAttnFusedMaxGroup = 8;  // q heads per kv head the phase supports

// Attended pages of the token: [p_lo, p_lo + npg), tokens [lo, pos]
struct AttnSpan {
    int pos, lo, p_lo, npg;
    const int* pt;
};
TI_DEVICE_INLINE AttnSpan attn_span(const GemvAttn& t) {
    AttnSpan a;
    a.pos = t.pos[0];
    a.pt = t.page_table + (size_t)t.seq[0] * t.pt_stride;
    const int window = t.window ? *t.window : t.window_const;
    a.lo = window > 0 ? max(0, a.pos - window + 1) : 0;
    a.p_lo = a.lo / kAttnPageTokens;
    a.npg = a.pos / kAttnPageTokens - a.p_lo + 1;
    return a;
}

// L2 prefetch of the K and V pages warp `warp` of CTA `cta` will score, issued
// before the dependency wait.  Only a hint: a page id outside the pool is skipped.
TI_DEVICE_INLINE void attn_fused_prefetch(const GemvAttn& t, int warp, int lane, int cta, int grid) {
    if (warp >= t.warps || lane != 0) return;
    const int nkv = t.nkv, h = cta % nkv, k = cta / nkv;
    const int nh = (grid - h + nkv - 1) / nkv;
    const AttnSpan sp = attn_span(t);
    const uint32_t bytes = (uint32_t)kAttnPageTokens * t.hd * 2;
    for (int i = k + nh * warp; i < sp.npg; i += nh * t.warps) {
        const int page = sp.pt[sp.p_lo + i];
        if (page < 0 || page >= t.n_pages) continue;
        const size_t base = ((size_t)page * nkv + h) * kAttnPageTokens * t.hd;
        prefetch_l2_bulk(t.kc + base, bytes);
        prefetch_l2_bulk(t.vc + base, bytes);
    }
}

// The phase, run by `nthr` consumer threads (tid in [0, nthr)) of CTA `cta` of
// `grid`; `sm` is gemv_attn_smem(G, HD, t.warps, nh) bytes of shared memory.
// GM: compile-time bound on the q heads per kv head (4 or 8).  `go` (one
// arrival) releases the producer's shared-memory fills once this CTA's
// latency-bound loads are done.  Named barrier 2 synchronises the consumer threads.
template <int HD, int GM>
TI_DEVICE_INLINE void attn_fused_phase(const GemvAttn& t, float* sm, int tid, int nthr, int cta, int grid,
                                       uint64_t* go, int* err) {
    constexpr int HALF = HD / 2;
    constexpr int DL = HD / 32;  // P.V dims per lane
    constexpr int NC = HD / 8;   // 8-element chunks of a row
    const int warp = tid >> 5, lane = tid & 31;
    const int nkv = t.nkv, G = t.nq / t.nkv;
    const int h = cta % nkv, k = cta / nkv;
    const int nh = (grid - h + nkv - 1) / nkv;  // CTAs serving kv head h
    const int aw = t.warps;
    float* qs = sm;          // [G][HD]
    float* kn = qs + G * HD;  // [HD]
    float* vn = kn + HD;      // [HD]
    float* slots = vn + HD;   // [aw][G][HD + 2]
    int* flag = reinterpret_cast<int*>(slots + (size_t)aw * G * (HD + 2));
    float* mw = reinterpret_cast<float*>(flag + 4);  // merging CTA: [nh][G] (max, then weight; sum)
    const AttnSpan sp = attn_span(t);
    const int pos = sp.pos, lo = sp.lo;

    // ---- RoPE (ops.cu:224-232) on the group's q heads and the token's k; v as is
    const uint16_t* row = t.qkv;
    for (int task = tid; task < (G + 1) * HALF; task += nthr) {
        const int hq = task / HALF, i = task - hq * HALF;
        const uint16_t* src = hq < G ? row + (size_t)(h * G + hq) * HD : row + (size_t)(t.nq + h) * HD;
        const float x0 = __uint_as_float((uint32_t)src[i] << 16);
        const float x1 = __uint_as_float((uint32_t)src[i + HALF] << 16);
        const float ang = (float)pos * t.freqs[i];
        const float c = cosf(ang), s = sinf(ang);
        float* dst = hq < G ? qs + hq * HD : kn;
        dst[i] = round_bf(x0 * c - x1 * s);
        dst[i + HALF] = round_bf(x0 * s + x1 * c);
    }
    for (int d = tid; d < HD; d += nthr)
        vn[d] = __uint_as_float((uint32_t)row[(size_t)(t.nq + nkv + h) * HD + d] << 16);
    named_bar(2, nthr);

    // ---- pages: warp `warp` of CTA k takes pages k + nh * (warp + aw * j)
    if (warp < aw) {
        const int tt = lane & 15, hh = lane >> 4;
        const float scale2 = t.scale * kAttnLog2e;
        float m[GM], l[GM], o[GM][DL];
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            m[g] = -INFINITY, l[g] = 0.f;
#pragma unroll
            for (int d = 0; d < DL; ++d) o[g][d] = 0.f;
        }
        for (int i = k + nh * warp; i < sp.npg; i += nh * aw) {
            const int pg = sp.p_lo + i;
            const int page = sp.pt[pg];
            if (page < 0 || page >= t.n_pages) {
                if (lane == 0 && err) atomicOr(err, kErrBadIndex);
                continue;
            }
            const int t0 = pg * kAttnPageTokens;
            const size_t base = ((size_t)page * nkv + h) * kAttnPageTokens * HD;
            const int rnew = pos - t0;  // the token's row in this page, if 0..15
            const int r0 = max(lo - t0, 0), r1 = min(pos - t0, kAttnPageTokens - 1);  // attended rows
            // the lane's half K row: all loads in flight at once
            const bool own = tt == rnew;
            uint4 kr[NC / 2];
            const uint4* ksrc = reinterpret_cast<const uint4*>(t.kc + base + (size_t)tt * HD) + hh * (NC / 2);
#pragma unroll
            for (int c = 0; c < NC / 2; ++c) kr[c] = own ? make_uint4(0, 0, 0, 0) : __ldg(ksrc + c);
            if (rnew >= 0 && rnew < kAttnPageTokens) {
                // the token's rotated k and its v into the cache (llama_model.cpp:159-170)
                for (int d = lane; d < HD; d += 32) {
                    t.kc[base + (size_t)rnew * HD + d] = __bfloat16_as_ushort(f2bf(kn[d]));
                    t.vc[base + (size_t)rnew * HD + d] = __bfloat16_as_ushort(f2bf(vn[d]));
                }
            }
            // ---- scores of token tt, every q head (this lane's half of the dims)
            float s[GM];
#pragma unroll
            for (int g = 0; g < GM; ++g) s[g] = 0.f;
#pragma unroll
            for (int c = 0; c < NC / 2; ++c) {
                const int e0 = (hh * (NC / 2) + c) * 8;
                float f[8];
                if (own) {
                    const float4 a = *reinterpret_cast<const float4*>(kn + e0);
                    const float4 b = *reinterpret_cast<const float4*>(kn + e0 + 4);
                    f[0] = a.x, f[1] = a.y, f[2] = a.z, f[3] = a.w, f[4] = b.x, f[5] = b.y, f[6] = b.z, f[7] = b.w;
                } else {
                    const uint4 v = kr[c];
                    f[0] = bf_lo(v.x), f[1] = bf_hi(v.x), f[2] = bf_lo(v.y), f[3] = bf_hi(v.y);
                    f[4] = bf_lo(v.z), f[5] = bf_hi(v.z), f[6] = bf_lo(v.w), f[7] = bf_hi(v.w);
                }
#pragma unroll
                for (int g = 0; g < GM; ++g) {
                    if (g < G) {
                        const float4 qa = *reinterpret_cast<const float4*>(qs + g * HD + e0);
                        const float4 qb = *reinterpret_cast<const float4*>(qs + g * HD + e0 + 4);
                        float a = s[g];
                        a = fmaf(qa.x, f[0], a);
                        a = fmaf(qa.y, f[1], a);
                        a = fmaf(qa.z, f[2], a);
                        a = fmaf(qa.w, f[3], a);
                        a = fmaf(qb.x, f[4], a);
                        a = fmaf(qb.y, f[5], a);
                        a = fmaf(qb.z, f[6], a);
                        a = fmaf(qb.w, f[7], a);
                        s[g] = a;
                    }
                }
            }
            // the lane's V slices of the attended rows, in flight during the softmax
            using VT = typename std::conditional<DL == 4, uint2, uint32_t>::type;
            VT vr[kAttnPageTokens];
            const VT* vsrc = reinterpret_cast<const VT*>(t.vc + base) + lane;
#pragma unroll
            for (int r = 0; r < kAttnPageTokens; ++r)
                vr[r] = (r >= r0 && r <= r1 && r != rnew) ? __ldg(vsrc + (size_t)r * (HD / DL)) : VT{};
            const int tok = t0 + tt;
            const bool valid = tok >= lo && tok <= pos;
            // ---- online softmax over the page's 16 tokens (ops.cu:393-419), base 2
            float p[GM];
#pragma unroll
            for (int g = 0; g < GM; ++g) {
                p[g] = 0.f;
                if (g >= G) continue;
                const float full = s[g] + __shfl_xor_sync(0xffffffffu, s[g], 16);
                const float sg = valid ? full * scale2 : -INFINITY;
                float mx = sg;
#pragma unroll
                for (int o2 = 1; o2 < 16; o2 <<= 1) mx = fmaxf(mx, __shfl_xor_sync(0xffffffffu, mx, o2));
                const float mn = fmaxf(m[g], mx);
                const float u = mn == -INFINITY ? 0.f : mn;
                const float al = ex2(m[g] - u);  // 0 while nothing was seen
                p[g] = ex2(sg - u);
                float sum = p[g];
#pragma unroll
                for (int o2 = 1; o2 < 16; o2 <<= 1) sum += __shfl_xor_sync(0xffffffffu, sum, o2);
                l[g] = fmaf(l[g], al, sum);
                m[g] = mn;
#pragma unroll
                for (int d = 0; d < DL; ++d) o[g][d] *= al;
            }
            // ---- P.V over the attended rows: the lane's dims of every q head
#pragma unroll
            for (int r = 0; r < kAttnPageTokens; ++r) {
                if (r < r0 || r > r1) continue;  // warp-uniform
                float vf[DL];
                if (r == rnew) {
#pragma unroll
                    for (int d = 0; d < DL; ++d) vf[d] = vn[lane * DL + d];
                } else if constexpr (DL == 4) {
                    vf[0] = bf_lo(vr[r].x), vf[1] = bf_hi(vr[r].x), vf[2] = bf_lo(vr[r].y), vf[3] = bf_hi(vr[r].y);
                } else {
                    vf[0] = bf_lo(vr[r]), vf[1] = bf_hi(vr[r]);
                }
#pragma unroll
                for (int g = 0; g < GM; ++g) {
                    if (g >= G) continue;
                    const float pp = __shfl_sync(0xffffffffu, p[g], r);
#pragma unroll
                    for (int d = 0; d < DL; ++d) o[g][d] = fmaf(pp, vf[d], o[g][d]);
                }
            }
        }
        // ---- this warp's partial: unnormalised output, running max and sum per q head
        float* ws = slots + (size_t)warp * G * (HD + 2);
#pragma unroll
        for (int g = 0; g < GM; ++g) {
            if (g >= G) continue;
#pragma unroll
            for (int d = 0; d < DL; ++d) ws[g * (HD + 2) + lane * DL + d] = o[g][d];
            if (lane == 0) {
                ws[g * (HD + 2) + HD] = m[g];
                ws[g * (HD + 2) + HD + 1] = l[g];
            }
        }
    }
    named_bar(2, nthr);

    // ---- the CTA's partial: warps merged in warp order
    float* part = t.part + (size_t)cta * G * (HD + 2);
    for (int idx = tid; idx < G * HD; idx += nthr) {
        const int g = idx / HD, d = idx - g * HD;
        float M = -INFINITY;
        for (int w = 0; w < aw; ++w) {
            const float* ws = slots + ((size_t)w * G + g) * (HD + 2);
            if (ws[HD + 1] > 0.f) M = fmaxf(M, ws[HD]);
        }
        float L = 0.f, O = 0.f;
        for (int w = 0; w < aw; ++w) {
            const float* ws = slots + ((size_t)w * G + g) * (HD + 2);
            const float lw = ws[HD + 1];
            if (lw > 0.f) {
                const float f = ex2(ws[HD] - M);
                L = fmaf(lw, f, L);
                O = fmaf(ws[d], f, O);
            }
        }
        part[g * (HD + 2) + d] = O;
        if (d == 0) {
            part[g * (HD + 2) + HD] = M;
            part[g * (HD + 2) + HD + 1] = L;
        }
    }
    __threadfence();
    named_bar(2, nthr);
    if (tid == 0) {
        *flag = atomicAdd(&t.ticket[h], 1u) == (unsigned int)(nh - 1);
        if (!*flag) mbar_arrive(go);  // nothing latency-bound left here but the wait
    }
    named_bar(2, nthr);

    // ---- the last CTA of kv head h merges the head's CTAs in CTA order
    if (*flag) {
        __threadfence();
        // every partial's (max, sum), all loads in flight together
        for (int idx = tid; idx < nh * G; idx += nthr) {
            const int j = idx / G, g = idx - j * G;
            const float* pj = t.part + ((size_t)(h + j * nkv) * G + g) * (HD + 2);
            mw[2 * idx] = __ldcg(pj + HD);
            mw[2 * idx + 1] = __ldcg(pj + HD + 1);
        }
        named_bar(2, nthr);
        // per q head: the overall max, each partial's weight 2^(m_j - M) (0 when
        // empty) in place of its max, and the total sum (in qs, free by now)
        if (tid < G) {
            float M = -INFINITY;
            for (int j = 0; j < nh; ++j)
                if (mw[2 * (j * G + tid) + 1] > 0.f) M = fmaxf(M, mw[2 * (j * G + tid)]);
            float L = 0.f;
            for (int j = 0; j < nh; ++j) {
                const float lj = mw[2 * (j * G + tid) + 1];
                const float w = lj > 0.f ? ex2(mw[2 * (j * G + tid)] - M) : 0.f;
                mw[2 * (j * G + tid)] = w;
                L = fmaf(lj, w, L);
            }
            qs[tid] = L;
        }
        named_bar(2, nthr);
        for (int idx = tid; idx < G * HD; idx += nthr) {
            const int g = idx / HD, d = idx - g * HD;
            float O = 0.f;
#pragma unroll 8
            for (int j = 0; j < nh; ++j)
                O = fmaf(__ldcg(t.part + ((size_t)(h + j * nkv) * G + g) * (HD + 2) + d), mw[2 * (j * G + g)], O);
            const float L = qs[g];
            t.out[(size_t)(h * G + g) * HD + d] = __bfloat16_as_ushort(f2bf(L > 0.f ? O / L : 0.f));
        }
        __threadfence();
        named_bar(2, nthr);
        if (tid == 0) {
            atomicExch(&t.ticket[h], 0u);
            atomicAdd(&t.sync[0], 1u);
            mbar_arrive(go);
        }
    }

    // ---- every kv head's output in place before the GEMV reads x (bounded wait)
    if (tid == 0) {
        bool ok = ld_acquire_gpu(&t.sync[0]) >= (unsigned int)nkv;
        if (!ok) {
            const uint64_t t0 = global_ns();
            for (uint32_t i = 0; i < kSpinLimit; ++i) {
                if (ld_acquire_gpu(&t.sync[0]) >= (unsigned int)nkv) {
                    ok = true;
                    break;
                }
                if ((i & 255u) == 255u && global_ns() - t0 > kWaitNs) break;
            }
        }
        if (!ok && err) atomicOr(err, kErrTimeoutGrid);
        // the last CTA past the wait re-arms the counters for the next launch
        if (atomicAdd(&t.sync[1], 1u) == (unsigned int)(grid - 1)) {
            atomicExch(&t.sync[0], 0u);
            atomicExch(&t.sync[1], 0u);
        }
    }
    named_bar(2, nthr);
}

}  // namespace ti
