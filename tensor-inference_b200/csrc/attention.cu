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
// read once per group; the context is cut into page-aligned ranges
// ("flash-decoding") whose partial (max, sum, unnormalised output) are merged
// by the last CTA to finish (atomic ticket), with no second launch.
//
// Data movement: a page holds 16 tokens x head_dim bf16 of one kv head,
// contiguous.  Each CTA loads its pages with 2-D TMA boxes (16 rows x 64 dims,
// 128-byte swizzle) BEFORE griddepcontrol.wait: cached rows were written by
// earlier steps, only the new token's q/k/v come from the previous kernel.
// The swizzle makes both the ldmatrix reads of K and the row reads of V free
// of shared-memory bank conflicts.
//
// Arithmetic follows the reference: RoPE in fp32 rounded to bf16; scores
// q.k with bf16 operands and fp32 accumulation (on the tensor cores: mma.sync
// m16n8k16, the group's q heads padded to 16 rows; bf16 x bf16 products are
// exact in fp32), times 1/sqrt(head_dim); exp-normalised fp32 softmax; fp32
// P.V on the CUDA cores; bf16 output.
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace ti {

constexpr int kAttnThreads = 128;
constexpr int kAttnMaxGroup = 16;
constexpr int kPage = 16;
constexpr int kAttnMaxPages = 8;  // pages per split (128 tokens) the shared-memory tiles hold

struct AttnSmem {
    uint32_t kt, vt, qf, kn, vn, ml, sc, mw, red, bar, total;
};

__host__ __device__ inline int attn_gp(int G) {
    int gp = 1;
    while (gp < G) gp <<= 1;
    return gp;
}
// P.V thread layout: DPT consecutive dims x all GP heads per thread, TG token groups
__host__ __device__ constexpr int attn_dpt(int GP) { return GP <= 8 ? 8 : 4; }
__host__ __device__ constexpr int attn_tg(int HD, int GP) { return 128 / (HD / attn_dpt(GP)); }

// C: tokens per split (pages x 16); offsets from a 1024-byte aligned base
__host__ __device__ inline AttnSmem attn_layout(int G, int HD, int C, int n_splits) {
    AttnSmem L;
    const int GP = attn_gp(G);
    uint32_t o = 0;
    L.kt = o;  // K tile [HD/64][C][64] bf16, rows 128-byte swizzled
    o += (uint32_t)C * HD * 2;
    L.vt = o;
    o += (uint32_t)C * HD * 2;
    L.qf = o;  // q heads after RoPE (bf16 values as fp32) [G][HD]
    o += (uint32_t)G * HD * 4;
    L.kn = o;  // new token's k after RoPE, and v
    o += HD * 4;
    L.vn = o;
    o += HD * 4;
    L.ml = o;
    o += 2 * kAttnMaxGroup * 4;
    L.sc = o;  // scores, then probabilities [C][GP] (heads >= G hold 0)
    o += (uint32_t)GP * C * 4;
    L.mw = o;  // split merge: weights and sums [2][n_splits][G]
    o += 2u * n_splits * G * 4;
    o = (o + 15u) & ~15u;
    // fold of the P.V token groups [TG-1][G][HD] fp32: over the K/V tiles (dead by
    // then) when they are large enough, else its own region
    const uint32_t red = (uint32_t)(attn_tg(HD, GP) - 1) * G * HD * 4;
    if (red <= 2u * C * HD * 2) {
        L.red = L.kt;
    } else {
        L.red = o;
        o += red;
    }
    L.bar = o;
    o += 16;
    L.total = o + 1024;
    return L;
}

TI_DEVICE_INLINE void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
// D(16x8 fp32) += A(16x16 bf16, row) * B(16x8 bf16, col)
TI_DEVICE_INLINE void mma_16816_bf16(float* c, const uint32_t* a, uint32_t b0, uint32_t b1) {
    asm volatile(
        "mma.sync.aligned.m16n8k16.row.col.f32.bf16.bf16.f32 {%0,%1,%2,%3}, {%4,%5,%6,%7}, {%8,%9}, "
        "{%0,%1,%2,%3};"
        : "+f"(c[0]), "+f"(c[1]), "+f"(c[2]), "+f"(c[3])
        : "r"(a[0]), "r"(a[1]), "r"(a[2]), "r"(a[3]), "r"(b0), "r"(b1));
}
// byte offset of element (row, d) in a [HD/64][C][64] bf16 tile with 128-byte swizzled rows
TI_DEVICE_INLINE uint32_t tile_off(int C, int row, int d) {
    const int hh = d >> 6, cc = (d & 63) >> 3;
    return (uint32_t)(hh * C + row) * 128u + (uint32_t)((cc ^ (row & 7)) << 4) + (uint32_t)((d & 7) << 1);
}

// GP: the GQA group size G rounded up to a power of two (loop bound; heads >= G idle)
template <int HD, int GP>
__global__ void __launch_bounds__(kAttnThreads)
    k_attn_decode(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, const AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int HALF = HD / 2;
    constexpr int NH = HD / 64;  // 64-dim boxes per row
    constexpr int KS = HD / 16;  // mma k-steps
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int G = a.nq / a.nkv;
    const int C = a.max_chunk;
    const AttnSmem L = attn_layout(G, HD, C, a.n_splits);
    uint8_t* kt = smem + L.kt;
    uint8_t* vt = smem + L.vt;
    float* qf = reinterpret_cast<float*>(smem + L.qf);
    float* kn = reinterpret_cast<float*>(smem + L.kn);
    float* vn = reinterpret_cast<float*>(smem + L.vn);
    float* ml = reinterpret_cast<float*>(smem + L.ml);
    float* sc = reinterpret_cast<float*>(smem + L.sc);
    float* mw = reinterpret_cast<float*>(smem + L.mw);
    float* red = reinterpret_cast<float*>(smem + L.red);
    uint64_t* bar = reinterpret_cast<uint64_t*>(smem + L.bar);
    __shared__ int s_last;

    // ---- this CTA's pages [pg0, pg1) of the attended range [lo, pos]
    const int pos = a.pos[b];
    const int* pt = a.page_table + (size_t)a.seq[b] * a.pt_stride;
    const int L1 = pos + 1;
    const int window = a.window ? *a.window : a.window_const;
    const int lo = window > 0 ? max(0, pos - window + 1) : 0;
    const int pps = C / kPage;
    const int pg0 = lo / kPage + split * pps;
    const int pg1 = min((L1 + kPage - 1) / kPage, pg0 + pps);
    const int t0 = pg0 * kPage;                    // token of tile row 0
    const int n_rows = max(0, pg1 - pg0) * kPage;  // tile rows loaded
    const int vlo = max(lo, t0) - t0, vhi = min(L1, t0 + n_rows) - t0;  // valid rows [vlo, vhi)

    // ---- before the dependency wait: cached pages (earlier steps' state only)
    if (tid == 0) {
        mbar_init(bar, 1);
        fence_barrier_init();
        bool ok = true;
        for (int p = pg0; p < pg1; ++p) {
            const int page = pt[p];
            if (page < 0 || page >= a.n_pages) ok = false;
        }
        if (!ok && a.err) atomicOr(a.err, kErrBadIndex);
        const int npg = ok ? max(0, pg1 - pg0) : 0;
        mbar_arrive_expect_tx(bar, (uint32_t)npg * 2u * NH * kPage * 128u);
        for (int p = 0; p < npg; ++p) {
            const int row = (pt[pg0 + p] * a.nkv + h) * kPage;
#pragma unroll
            for (int hh = 0; hh < NH; ++hh) {
                const uint32_t off = (uint32_t)(hh * C + p * kPage) * 128u;
                tma_load_2d(kt + off, &tk, hh * 64, row, bar);
                tma_load_2d(vt + off, &tv, hh * 64, row, bar);
            }
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
        float* dst = hh < G ? qf + hh * HD : kn;
        dst[i] = round_bf(x0 * c - x1 * s);
        dst[i + HALF] = round_bf(x0 * s + x1 * c);
    }
    for (int d = tid; d < HD; d += kAttnThreads)
        vn[d] = __uint_as_float((uint32_t)row[(size_t)(a.nq + a.nkv + h) * HD + d] << 16);
    __syncthreads();

    // ---- the tiles are in; the CTA holding `pos` puts the new K/V row into its
    //      tile and appends it to its page
    mbar_wait(bar, 0, a.err, kErrTimeoutFull);
    if (pos >= t0 && pos < t0 + n_rows) {
        const int r = pos - t0;
        for (int d = tid; d < HD; d += kAttnThreads) {
            const uint32_t off = tile_off(C, r, d);
            *reinterpret_cast<bf16*>(kt + off) = f2bf(kn[d]);
            *reinterpret_cast<bf16*>(vt + off) = f2bf(vn[d]);
        }
        const int page = pt[pos / kPage];
        if (page >= 0 && page < a.n_pages) {
            const size_t off = (((size_t)page * a.nkv + h) * kPage + (pos % kPage)) * HD;
            for (int d = tid; d < HD; d += kAttnThreads) {
                reinterpret_cast<bf16*>(a.kc)[off + d] = f2bf(kn[d]);
                reinterpret_cast<bf16*>(a.vc)[off + d] = f2bf(vn[d]);
            }
        } else if (tid == 0 && a.err) {
            atomicOr(a.err, kErrBadIndex);
        }
    }
    __syncthreads();

    // ---- scores S = q K^T on the tensor cores: A = q heads (16 rows, >= G zero),
    //      B = 8 tokens x 16 dims per mma; warp w takes token octets w, w+4, ...
    {
        uint32_t qa[KS][4];
        const int r = lane >> 2, c2 = (lane & 3) * 2;
#pragma unroll
        for (int ks = 0; ks < KS; ++ks) {
            const int k0 = ks * 16;
            auto qv = [&](int rr, int cc) { return rr < G ? qf[rr * HD + cc] : 0.f; };
            qa[ks][0] = pack_bf2(qv(r, k0 + c2), qv(r, k0 + c2 + 1));
            qa[ks][1] = pack_bf2(qv(r + 8, k0 + c2), qv(r + 8, k0 + c2 + 1));
            qa[ks][2] = pack_bf2(qv(r, k0 + 8 + c2), qv(r, k0 + 8 + c2 + 1));
            qa[ks][3] = pack_bf2(qv(r + 8, k0 + 8 + c2), qv(r + 8, k0 + 8 + c2 + 1));
        }
        const uint32_t kbase = smem_u32(kt);
        for (int nt = warp; nt < n_rows / 8; nt += kAttnThreads / 32) {
            const int r0 = nt * 8;
            float acc[4] = {0.f, 0.f, 0.f, 0.f};
            const int ri = r0 + (lane & 7), mi = lane >> 3;
#pragma unroll
            for (int ks = 0; ks < KS; ks += 2) {
                uint32_t m0, m1, m2, m3;
                ldsm_x4(kbase + tile_off(C, ri, ks * 16 + mi * 8), m0, m1, m2, m3);
                mma_16816_bf16(acc, qa[ks], m0, m1);
                mma_16816_bf16(acc, qa[ks + 1], m2, m3);
            }
            // acc[0..1]: head lane/4, rows r0 + 2*(lane%4) + {0,1}; acc[2..3]: head lane/4 + 8
#pragma unroll
            for (int e = 0; e < 2; ++e) {
                const int jj = r0 + c2 + e;
                const bool valid = jj >= vlo && jj < vhi;
                if (r < G) sc[jj * GP + r] = valid ? a.scale * acc[e] : -INFINITY;
                else if (r < GP) sc[jj * GP + r] = 0.f;  // padding heads: probability 0
                if (r + 8 < G) sc[jj * GP + r + 8] = valid ? a.scale * acc[2 + e] : -INFINITY;
                else if (r + 8 < GP) sc[jj * GP + r + 8] = 0.f;
            }
        }
    }
    __syncthreads();

    // ---- softmax statistics per q head (ops.cu:393-419)
    for (int g = warp; g < G; g += kAttnThreads / 32) {
        float m = -INFINITY;
        for (int j = lane; j < n_rows; j += 32) m = fmaxf(m, sc[j * GP + g]);
        m = warp_max(m);
        float l = 0.f;
        for (int j = lane; j < n_rows; j += 32) {
            const float p = m == -INFINITY ? 0.f : expf(sc[j * GP + g] - m);
            sc[j * GP + g] = p;
            l += p;
        }
        l = warp_sum(l);
        if (lane == 0) {
            ml[2 * g] = m;
            ml[2 * g + 1] = l;
        }
    }
    __syncthreads();

    // ---- P.V (ops.cu:526-539) in fp32: thread -> DPT consecutive dims of every
    //      head of the group, over the tokens of its token group (j = tg mod TG);
    //      packed f32x2 FMAs; the token groups are folded in order afterwards
    constexpr int DPT = attn_dpt(GP);
    constexpr int NDG = HD / DPT;
    constexpr int TG = kAttnThreads / NDG;
    const int dg = tid % NDG, tg = tid / NDG, d0 = dg * DPT;
    float2 acc[GP][DPT / 2];
#pragma unroll
    for (int g = 0; g < GP; ++g)
#pragma unroll
        for (int k = 0; k < DPT / 2; ++k) acc[g][k] = make_float2(0.f, 0.f);
    for (int j = max(vlo, 0) + tg; j < vhi; j += TG) {
        float2 vf[DPT / 2];
        if constexpr (DPT == 8) {
            const uint4 v = *reinterpret_cast<const uint4*>(vt + tile_off(C, j, d0));
            vf[0] = bf2_to_f2(v.x);
            vf[1] = bf2_to_f2(v.y);
            vf[2] = bf2_to_f2(v.z);
            vf[3] = bf2_to_f2(v.w);
        } else {
            const uint2 v = *reinterpret_cast<const uint2*>(vt + tile_off(C, j, d0));
            vf[0] = bf2_to_f2(v.x);
            vf[1] = bf2_to_f2(v.y);
        }
        float p[GP];
        if constexpr (GP >= 4) {
#pragma unroll
            for (int g = 0; g < GP; g += 4) {
                const float4 q4 = *reinterpret_cast<const float4*>(sc + j * GP + g);
                p[g] = q4.x;
                p[g + 1] = q4.y;
                p[g + 2] = q4.z;
                p[g + 3] = q4.w;
            }
        } else {
#pragma unroll
            for (int g = 0; g < GP; ++g) p[g] = sc[j * GP + g];
        }
#pragma unroll
        for (int g = 0; g < GP; ++g) {
            const float2 pp = make_float2(p[g], p[g]);
#pragma unroll
            for (int k = 0; k < DPT / 2; ++k) acc[g][k] = ffma2(pp, vf[k], acc[g][k]);
        }
    }
    if (TG > 1) {
        __syncthreads();  // the K/V tiles are dead: the fold area may overlay them
        if (tg > 0)
#pragma unroll
            for (int g = 0; g < GP; ++g)
                if (g < G)
#pragma unroll
                    for (int k = 0; k < DPT / 2; ++k)
                        *reinterpret_cast<float2*>(red + (((size_t)(tg - 1) * G + g) * HD + d0 + 2 * k)) = acc[g][k];
        __syncthreads();
        if (tg == 0)
            for (int t = 0; t < TG - 1; ++t)
#pragma unroll
                for (int g = 0; g < GP; ++g)
                    if (g < G)
#pragma unroll
                        for (int k = 0; k < DPT / 2; ++k) {
                            const float2 o =
                                *reinterpret_cast<const float2*>(red + (((size_t)t * G + g) * HD + d0 + 2 * k));
                            acc[g][k].x += o.x;
                            acc[g][k].y += o.y;
                        }
    }

    if (a.n_splits == 1) {
        if (tg == 0)
#pragma unroll
            for (int g = 0; g < GP; ++g)
                if (g < G) {
                    const float l = ml[2 * g + 1];
                    bf16* dst =
                        reinterpret_cast<bf16*>(a.out) + (size_t)b * a.out_stride + (size_t)(h * G + g) * HD + d0;
#pragma unroll
                    for (int k = 0; k < DPT / 2; ++k) {
                        dst[2 * k] = f2bf(acc[g][k].x / l);
                        dst[2 * k + 1] = f2bf(acc[g][k].y / l);
                    }
                }
        return;
    }

    // ---- partial results, merged by the last CTA of this (token, kv head)
    const size_t pbase = (((size_t)b * a.nkv + h) * a.n_splits + split) * G;
    if (tg == 0)
#pragma unroll
        for (int g = 0; g < GP; ++g)
            if (g < G)
#pragma unroll
                for (int k = 0; k < DPT / 2; ++k)
                    *reinterpret_cast<float2*>(a.part_o + (pbase + g) * HD + d0 + 2 * k) = acc[g][k];
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
    // split weights w[s][g] = exp(m_s - M_g) (0 for empty splits)
    float* wsg = mw;                        // [n_splits][G] maxima, then weights
    float* lsg = mw + a.n_splits * G;       // [n_splits][G] sums
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
            const float w = wsg[s * G + g];
            if (w == 0.f) continue;
            const float4 v = __ldcg(reinterpret_cast<const float4*>(a.part_o + (p0 + (size_t)s * G) * HD + e));
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
    // pages per split: about two CTAs per SM over the batch's (token, kv head)
    // pairs at the longest context, at most kAttnMaxPages (env TI_ATTN_PPS overrides)
    const int max_pages = std::max(1, (max_len + kPage - 1) / kPage);
    const char* env = std::getenv("TI_ATTN_PPS");
    int pps;
    if (env && std::atoi(env) >= 1) {
        pps = std::min(std::atoi(env), kAttnMaxPages);
    } else {
        const long work = (long)std::max(1, nb * nkv) * max_pages;
        pps = (int)std::min<long>(kAttnMaxPages, std::max<long>(1, (work + 2L * sms - 1) / (2L * sms)));
    }
    *max_chunk = pps * kPage;
    return (max_pages + pps - 1) / pps;
}

size_t attn_scratch_floats(int nb, int nq, int nkv, int hd, int n_splits) {
    const size_t G = (size_t)(nq / nkv);
    return (size_t)nb * nkv * n_splits * G * (hd + 2);
}

namespace {

template <int HD>
const void* attn_func(int gp) {
    switch (gp) {
        case 1: return reinterpret_cast<const void*>(&k_attn_decode<HD, 1>);
        case 2: return reinterpret_cast<const void*>(&k_attn_decode<HD, 2>);
        case 4: return reinterpret_cast<const void*>(&k_attn_decode<HD, 4>);
        case 8: return reinterpret_cast<const void*>(&k_attn_decode<HD, 8>);
        default: return reinterpret_cast<const void*>(&k_attn_decode<HD, 16>);
    }
}

}  // namespace

cudaError_t attn_launch(const AttnArgs& a, cudaStream_t s, bool pdl) {
    if (a.nkv <= 0 || a.nq % a.nkv != 0 || a.nq / a.nkv > kAttnMaxGroup) return cudaErrorInvalidValue;
    if (a.max_chunk < kPage || a.max_chunk > kAttnMaxPages * kPage || a.max_chunk % kPage != 0)
        return cudaErrorInvalidValue;
    const int G = a.nq / a.nkv;
    const int gp = attn_gp(G);
    const void* f = nullptr;
    switch (a.hd) {
        case 64: f = attn_func<64>(gp); break;
        case 128: f = attn_func<128>(gp); break;
        case 256: f = attn_func<256>(gp); break;
        default: return cudaErrorInvalidValue;
    }
    CUtensorMap tk, tv;
    const uint64_t rows = (uint64_t)a.n_pages * a.nkv * kPage;
    if (!make_tmap_bf16_sw128(&tk, a.kc, rows, a.hd, a.hd, kPage)) return cudaErrorInvalidValue;
    if (!make_tmap_bf16_sw128(&tv, a.vc, rows, a.hd, a.hd, kPage)) return cudaErrorInvalidValue;
    const size_t smem = attn_layout(G, a.hd, a.max_chunk, a.n_splits).total;
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    {
        static std::mutex mu;
        std::lock_guard<std::mutex> lk(mu);
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    AttnArgs args = a;
    void* params[] = {&tk, &tv, &args};
    return launch_pdl(f, dim3(a.n_splits, a.nkv, a.nb), dim3(kAttnThreads), smem, s, params, pdl);
}

}  // namespace ti
