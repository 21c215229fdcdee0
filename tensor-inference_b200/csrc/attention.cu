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
// contiguous.  A CTA streams its page range through a ring of three stages of
// 32 KB (K and V of 128, 64 or 32 tokens for head_dim 64, 128, 256), loaded
// with 2-D TMA boxes (16 rows x 64 dims, 128-byte swizzle): the next stages are
// in flight while the current one is scored, with an online softmax (running
// max and sum per q head, the P.V accumulators rescaled when the max grows).
// The first stages are requested BEFORE griddepcontrol.wait: cached rows were
// written by earlier steps, only the new token's q/k/v come from the previous
// kernel.  The swizzle makes both the ldmatrix reads of K and the row reads of
// V free of shared-memory bank conflicts.
//
// Work split: warp w owns 16-token blocks of every stage.  Scores S = q K^T come
// out of mma.sync m16n8k16 (the group's q heads padded to 16 rows) in exactly
// the register layout of the A operand of the next mma, so P never leaves the
// registers: each warp keeps its own running max and sum per q head (quad
// shuffles), P.V accumulates on the tensor cores with V fragments read by
// ldmatrix.trans from the swizzled tile, and the four warps are merged once at
// the end.  A stage is released through an "empty" mbarrier (one arrival per
// warp), not a block barrier.
//
// Arithmetic follows the reference: RoPE in fp32 rounded to bf16; scores
// q.k with bf16 operands and fp32 accumulation (bf16 x bf16 products are exact
// in fp32), times 1/sqrt(head_dim); exp-normalised fp32 softmax; bf16 output.
// The reference's P.V is fp32 x bf16-valued V: here each fp32 probability is
// split into two bf16 terms p = hi + lo (hi = bf16(p), lo = bf16(p - hi)), each
// multiplied exactly by V in the fp32 accumulator; what the split drops is at
// most 2^-18 of p, far below the half-ulp (2^-9) of the bf16 output.
#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "kernels.h"

namespace ti {

constexpr int kAttnThreads = 128;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnMaxGroup = 16;              // q heads per kv head: the 16 rows of the mma
constexpr int kPage = 16;
constexpr int kAttnStages = 3;                 // ring depth
constexpr uint32_t kAttnStageBytes = 32768;    // K + V of one stage
constexpr int kAttnMaxSplits = 512;            // the merge weights fit over the ring

// tokens per stage: 128 / 64 / 32 for head_dim 64 / 128 / 256
__host__ __device__ constexpr int attn_ct(int HD) { return (int)(kAttnStageBytes / (4u * HD)); }

struct AttnSmem {
    uint32_t ring, qf, kn, vn, wml, hml, bar, total;
};

// offsets from a 1024-byte aligned base
__host__ __device__ inline AttnSmem attn_layout(int G, int HD) {
    AttnSmem L;
    uint32_t o = 0;
    L.ring = o;  // [stages] x {K tile [HD/64][CT][64] bf16, V tile}, rows 128-byte swizzled;
    o += kAttnStages * kAttnStageBytes;  // afterwards the warp merge and the split merge weights
    L.qf = o;    // q heads after RoPE (bf16 values as fp32) [G][HD]
    o += (uint32_t)G * HD * 4;
    L.kn = o;    // new token's k after RoPE, and v
    o += HD * 4;
    L.vn = o;
    o += HD * 4;
    L.wml = o;   // per warp running (max, sum) per q head [warps][16][2]
    o += kAttnWarps * kAttnMaxGroup * 2 * 4;
    L.hml = o;   // merged (max, sum) per q head [16][2]
    o += kAttnMaxGroup * 2 * 4;
    L.bar = o;   // full[stages], empty[stages]
    o += 2 * kAttnStages * 8;
    L.total = o + 1024;
    return L;
}

TI_DEVICE_INLINE void ldsm_x4(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.shared.b16 {%0,%1,%2,%3}, [%4];"
                 : "=r"(r0), "=r"(r1), "=r"(r2), "=r"(r3)
                 : "r"(addr));
}
TI_DEVICE_INLINE void ldsm_x4_t(uint32_t addr, uint32_t& r0, uint32_t& r1, uint32_t& r2, uint32_t& r3) {
    asm volatile("ldmatrix.sync.aligned.m8n8.x4.trans.shared.b16 {%0,%1,%2,%3}, [%4];"
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
// two fp32 probabilities -> bf16 pair hi and the bf16 pair of what hi left out
TI_DEVICE_INLINE void split_bf2(float p0, float p1, uint32_t& hi, uint32_t& lo) {
    hi = pack_bf2(p0, p1);
    lo = pack_bf2(p0 - bf_lo(hi), p1 - bf_hi(hi));
}

template <int HD>
__global__ void __launch_bounds__(kAttnThreads, 2)
    k_attn_decode(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, const AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int HALF = HD / 2;
    constexpr int NH = HD / 64;  // 64-dim boxes per row
    constexpr int KS = HD / 16;  // mma k-steps of the scores
    constexpr int CT = attn_ct(HD);
    constexpr int CP = CT / kPage;                 // pages per stage
    constexpr int NS = kAttnStages;
    constexpr int NTB = CT / 16;                   // 16-token blocks per stage
    constexpr int DPARTS = NTB >= kAttnWarps ? 1 : kAttnWarps / NTB;  // warps sharing a block split the dims
    constexpr int WPD = kAttnWarps / DPARTS;       // warps per dim part
    constexpr int TBW = NTB / WPD;                 // blocks per warp per stage
    constexpr int DW = HD / DPARTS;                // dims of a warp's P.V
    constexpr int NT = DW / 8;                     // P.V n-tiles
    constexpr uint32_t VOFF = kAttnStageBytes / 2;  // V tile after the K tile of a stage
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, qq = lane & 3;      // mma fragment row / column pair
    const int dp = warp / WPD, wi = warp % WPD;
    const int G = a.nq / a.nkv;
    const AttnSmem L = attn_layout(G, HD);
    uint8_t* ring = smem + L.ring;
    float* qf = reinterpret_cast<float*>(smem + L.qf);
    float* kn = reinterpret_cast<float*>(smem + L.kn);
    float* vn = reinterpret_cast<float*>(smem + L.vn);
    float* wml = reinterpret_cast<float*>(smem + L.wml);
    float* hml = reinterpret_cast<float*>(smem + L.hml);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar);
    uint64_t* empty = full + NS;
    __shared__ int s_last;

    // ---- this CTA's pages [pg0, pg1) of the attended range [lo, pos]
    const int pos = a.pos[b];
    const int* pt = a.page_table + (size_t)a.seq[b] * a.pt_stride;
    const int L1 = pos + 1;
    const int window = a.window ? *a.window : a.window_const;
    const int lo = window > 0 ? max(0, pos - window + 1) : 0;
    const int pps = a.max_chunk / kPage;
    const int pg0 = lo / kPage + split * pps;
    const int pg1 = min((L1 + kPage - 1) / kPage, pg0 + pps);
    const int npg = max(0, pg1 - pg0);
    const int n_st = (npg + CP - 1) / CP;
    const int t0 = pg0 * kPage;                                     // token of split row 0
    const int vlo = max(lo, t0) - t0, vhi = min(L1, t0 + npg * kPage) - t0;  // valid rows [vlo, vhi)

    // stage st -> ring slot st % NS: its pages' K and V boxes on one barrier
    auto issue = [&](int st) {
        uint8_t* kt = ring + (uint32_t)(st % NS) * kAttnStageBytes;
        const int p0 = pg0 + st * CP, pn = min(CP, pg1 - p0);
        int nv = 0;
        for (int p = 0; p < pn; ++p) {
            const int page = pt[p0 + p];
            nv += page >= 0 && page < a.n_pages;
        }
        if (nv < pn && a.err) atomicOr(a.err, kErrBadIndex);
        mbar_arrive_expect_tx(&full[st % NS], (uint32_t)nv * 2u * NH * kPage * 128u);
        for (int p = 0; p < pn; ++p) {
            const int page = pt[p0 + p];
            if (page < 0 || page >= a.n_pages) continue;
            const int row = (page * a.nkv + h) * kPage;
#pragma unroll
            for (int hh = 0; hh < NH; ++hh) {
                const uint32_t off = (uint32_t)(hh * CT + p * kPage) * 128u;
                tma_load_2d(kt + off, &tk, hh * 64, row, &full[st % NS]);
                tma_load_2d(kt + VOFF + off, &tv, hh * 64, row, &full[st % NS]);
            }
        }
    };

    // ---- before the dependency wait: cached pages (earlier steps' state only)
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kAttnWarps);
        }
        fence_barrier_init();
        for (int st = 0; st < min(NS, n_st); ++st) issue(st);
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

    // q fragments of the score mma: A = q heads (16 rows, >= G zero) x head_dim
    uint32_t qa[KS][4];
#pragma unroll
    for (int ks = 0; ks < KS; ++ks) {
        const int k0 = ks * 16 + qq * 2;
        auto qv = [&](int rr, int cc) { return rr < G ? qf[rr * HD + cc] : 0.f; };
        qa[ks][0] = pack_bf2(qv(gq, k0), qv(gq, k0 + 1));
        qa[ks][1] = pack_bf2(qv(gq + 8, k0), qv(gq + 8, k0 + 1));
        qa[ks][2] = pack_bf2(qv(gq, k0 + 8), qv(gq, k0 + 9));
        qa[ks][3] = pack_bf2(qv(gq + 8, k0 + 8), qv(gq + 8, k0 + 9));
    }

    // this warp's state: P.V accumulators (heads gq, gq+8 x its dims), running max
    // and this lane's share of the running sum for heads gq and gq+8
    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;

    for (int st = 0; st < n_st; ++st) {
        uint8_t* kt = ring + (uint32_t)(st % NS) * kAttnStageBytes;
        uint8_t* vt = kt + VOFF;
        const int r0 = st * CT;  // split row of stage row 0
        const int rows = min(CP, npg - st * CP) * kPage;
        const int jlo = max(vlo - r0, 0), jhi = min(vhi - r0, rows);  // valid stage rows
        mbar_wait(&full[st % NS], (uint32_t)(st / NS) & 1u, a.err, kErrTimeoutFull);
        __syncwarp();  // lanes leave the poll apart; ldmatrix and mma need the whole warp

        // the stage holding `pos` takes the new K/V row into its tile and its page
        if (pos >= t0 + r0 && pos < t0 + r0 + rows) {
            const int r = pos - t0 - r0;
            for (int d = tid; d < HD; d += kAttnThreads) {
                const uint32_t off = tile_off(CT, r, d);
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
            // the slot is refilled by TMA later: order these generic writes before it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncthreads();
        }

#pragma unroll
        for (int tbi = 0; tbi < TBW; ++tbi) {
            const int j0 = (wi + tbi * WPD) * 16;  // block rows [j0, j0 + 16)
            if (j0 + 16 <= jlo || j0 >= jhi) continue;  // warp-uniform
            if (j0 < jlo || j0 + 16 > jhi) {
                // rows outside [jlo, jhi) get probability 0: make their V finite (zero)
                for (int t = lane; t < 16 * (DW / 8); t += 32) {
                    const int jr = j0 + t / (DW / 8), d = dp * DW + (t % (DW / 8)) * 8;
                    if (jr < jlo || jr >= jhi) *reinterpret_cast<uint4*>(vt + tile_off(CT, jr, d)) = make_uint4(0, 0, 0, 0);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
            }
            // ---- scores of 16 tokens: two n-tiles of 8
            float c[2][4];
            const uint32_t kbase = smem_u32(kt);
#pragma unroll
            for (int nt = 0; nt < 2; ++nt) {
                c[nt][0] = c[nt][1] = c[nt][2] = c[nt][3] = 0.f;
                const int ri = j0 + nt * 8 + (lane & 7), mi = lane >> 3;
#pragma unroll
                for (int ks = 0; ks < KS; ks += 2) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(kbase + tile_off(CT, ri, ks * 16 + mi * 8), b0, b1, b2, b3);
                    mma_16816_bf16(c[nt], qa[ks], b0, b1);
                    mma_16816_bf16(c[nt], qa[ks + 1], b2, b3);
                }
            }
            // c[nt][0..1]: head gq, rows j0 + 8 nt + 2 qq + {0,1}; c[nt][2..3]: head gq + 8
            float mx0 = -INFINITY, mx1 = -INFINITY;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    const int jj = j0 + nt * 8 + qq * 2 + e;
                    const bool valid = jj >= jlo && jj < jhi;
                    c[nt][e] = valid ? a.scale * c[nt][e] : -INFINITY;
                    c[nt][2 + e] = valid ? a.scale * c[nt][2 + e] : -INFINITY;
                    mx0 = fmaxf(mx0, c[nt][e]);
                    mx1 = fmaxf(mx1, c[nt][2 + e]);
                }
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
            mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
            // ---- online softmax (ops.cu:393-419 over the whole row)
            const float n0 = fmaxf(m0, mx0), n1 = fmaxf(m1, mx1);
            const float al0 = m0 == -INFINITY ? 0.f : expf(m0 - n0);
            const float al1 = m1 == -INFINITY ? 0.f : expf(m1 - n1);
            m0 = n0;
            m1 = n1;
            float s0 = 0.f, s1 = 0.f;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    c[nt][e] = n0 == -INFINITY ? 0.f : expf(c[nt][e] - n0);
                    c[nt][2 + e] = n1 == -INFINITY ? 0.f : expf(c[nt][2 + e] - n1);
                    s0 += c[nt][e];
                    s1 += c[nt][2 + e];
                }
            l0 = fmaf(l0, al0, s0);
            l1 = fmaf(l1, al1, s1);
            if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    o[n][0] *= al0;
                    o[n][1] *= al0;
                    o[n][2] *= al1;
                    o[n][3] *= al1;
                }
            }
            // ---- P.V: A = P (heads x 16 tokens) as hi + lo bf16 pairs, B = V via ldmatrix.trans
            uint32_t ph[4], pl[4];
            split_bf2(c[0][0], c[0][1], ph[0], pl[0]);
            split_bf2(c[0][2], c[0][3], ph[1], pl[1]);
            split_bf2(c[1][0], c[1][1], ph[2], pl[2]);
            split_bf2(c[1][2], c[1][3], ph[3], pl[3]);
            const uint32_t vbase = smem_u32(vt);
            const int vr = j0 + (lane & 7) + ((lane >> 3) & 1) * 8;
#pragma unroll
            for (int n = 0; n < NT; n += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vbase + tile_off(CT, vr, dp * DW + n * 8 + (lane >> 4) * 8), b0, b1, b2, b3);
                mma_16816_bf16(o[n], ph, b0, b1);
                mma_16816_bf16(o[n], pl, b0, b1);
                mma_16816_bf16(o[n + 1], ph, b2, b3);
                mma_16816_bf16(o[n + 1], pl, b2, b3);
            }
        }
        // release the slot: every warp arrives; warp 0 refills it once all have
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[st % NS]);
        if (tid == 0 && st + NS < n_st) {
            mbar_wait(&empty[st % NS], (uint32_t)(st / NS) & 1u, a.err, kErrTimeoutFull);
            issue(st + NS);
        }
        __syncwarp();
    }

    // ---- merge the warps: per head the max over the warps of a dim part, each
    //      warp's accumulators and sums rescaled to it, summed in warp order
    l0 += __shfl_xor_sync(0xffffffffu, l0, 1);
    l0 += __shfl_xor_sync(0xffffffffu, l0, 2);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 1);
    l1 += __shfl_xor_sync(0xffffffffu, l1, 2);
    if (qq == 0) {
        wml[(warp * 16 + gq) * 2] = m0;
        wml[(warp * 16 + gq) * 2 + 1] = l0;
        wml[(warp * 16 + gq + 8) * 2] = m1;
        wml[(warp * 16 + gq + 8) * 2 + 1] = l1;
    }
    __syncthreads();  // also: every stage consumed, no copy in flight into the ring
    if (tid < kAttnMaxGroup) {
        // warps of dim part 0 saw every token block (the other parts saw the same ones)
        float M = -INFINITY;
        for (int w = 0; w < WPD; ++w) M = fmaxf(M, wml[(w * 16 + tid) * 2]);
        float Ls = 0.f;
        for (int w = 0; w < WPD; ++w) {
            const float mw = wml[(w * 16 + tid) * 2];
            if (mw != -INFINITY) Ls = fmaf(wml[(w * 16 + tid) * 2 + 1], expf(mw - M), Ls);
        }
        hml[2 * tid] = M;
        hml[2 * tid + 1] = Ls;
    }
    __syncthreads();
    float* red = reinterpret_cast<float*>(ring);  // [warps][16][DW]
    {
        const float M0 = hml[2 * gq], M1 = hml[2 * (gq + 8)];
        const float f0 = m0 == -INFINITY ? 0.f : expf(m0 - M0);
        const float f1 = m1 == -INFINITY ? 0.f : expf(m1 - M1);
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const int d = n * 8 + qq * 2;
            *reinterpret_cast<float2*>(red + ((size_t)warp * 16 + gq) * DW + d) = make_float2(o[n][0] * f0, o[n][1] * f0);
            *reinterpret_cast<float2*>(red + ((size_t)warp * 16 + gq + 8) * DW + d) =
                make_float2(o[n][2] * f1, o[n][3] * f1);
        }
    }
    __syncthreads();

    // 4 consecutive (g, d) outputs per thread
    const size_t pbase = (((size_t)b * a.nkv + h) * a.n_splits + split) * G;
    for (int e = tid * 4; e < G * HD; e += kAttnThreads * 4) {
        const int g = e / HD, d = e - g * HD;
        const int part = d / DW, dl = d - part * DW;
        float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
        for (int w = 0; w < WPD; ++w) {
            const float4 v = *reinterpret_cast<const float4*>(red + ((size_t)(part * WPD + w) * 16 + g) * DW + dl);
            O.x += v.x;
            O.y += v.y;
            O.z += v.z;
            O.w += v.w;
        }
        if (a.n_splits == 1) {
            const float l = hml[2 * g + 1];
            bf16* dst = reinterpret_cast<bf16*>(a.out) + (size_t)b * a.out_stride + (size_t)h * G * HD + e;
            dst[0] = f2bf(O.x / l);
            dst[1] = f2bf(O.y / l);
            dst[2] = f2bf(O.z / l);
            dst[3] = f2bf(O.w / l);
        } else {
            *reinterpret_cast<float4*>(a.part_o + (pbase + g) * HD + d) = O;
        }
    }
    if (a.n_splits == 1) return;

    // ---- partial results, merged by the last CTA of this (token, kv head)
    if (tid < G) {
        a.part_ml[(pbase + tid) * 2] = hml[2 * tid];
        a.part_ml[(pbase + tid) * 2 + 1] = hml[2 * tid + 1];
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
    // split weights w[s][g] = exp(m_s - M_g) (0 for empty splits), over the ring
    float* wsg = reinterpret_cast<float*>(ring);  // [n_splits][G] maxima, then weights
    float* lsg = wsg + a.n_splits * G;            // [n_splits][G] sums
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
        hml[2 * tid + 1] = Ls;
    }
    __syncthreads();
    // the per-split loads are independent float4 reads, all in flight together
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
        const float inv = hml[2 * g + 1];
        bf16* dst = reinterpret_cast<bf16*>(a.out) + (size_t)b * a.out_stride + (size_t)h * G * HD + e;
        dst[0] = f2bf(O.x / inv);
        dst[1] = f2bf(O.y / inv);
        dst[2] = f2bf(O.z / inv);
        dst[3] = f2bf(O.w / inv);
    }
    if (tid == 0) a.counters[b * a.nkv + h] = 0u;
}

int attn_splits(int nb, int nkv, int hd, int max_len, int sms, int* max_chunk) {
    // stages per split: about kWaves waves of two CTAs per SM over the batch's
    // (token, kv head) pairs at the longest context (env TI_ATTN_SPP overrides);
    // splits of near-equal length, at most kAttnMaxSplits of them
    const int ct = attn_ct(hd);
    const int max_pages = std::max(1, (max_len + kPage - 1) / kPage);
    const int stages = (max_pages + ct / kPage - 1) / (ct / kPage);
    const char* env = std::getenv("TI_ATTN_SPP");
    int spp;
    if (env && std::atoi(env) >= 1) {
        spp = std::atoi(env);
    } else {
        const char* wv = std::getenv("TI_ATTN_WAVES");
        const long waves = wv && std::atoi(wv) >= 1 ? std::atoi(wv) : 4;
        const long target = waves * 2L * sms;
        const long work = (long)std::max(1, nb * nkv) * stages;
        spp = (int)std::max<long>(1, (work + target - 1) / target);
    }
    spp = std::max(spp, (stages + kAttnMaxSplits - 1) / kAttnMaxSplits);
    spp = std::min(spp, stages);
    int n = (stages + spp - 1) / spp;
    spp = (stages + n - 1) / n;  // even out the splits
    n = (stages + spp - 1) / spp;
    *max_chunk = spp * ct;
    return n;
}

size_t attn_scratch_floats(int nb, int nq, int nkv, int hd, int n_splits) {
    const size_t G = (size_t)(nq / nkv);
    return (size_t)nb * nkv * n_splits * G * (hd + 2);
}

cudaError_t attn_launch(const AttnArgs& a, cudaStream_t s, bool pdl) {
    if (a.nkv <= 0 || a.nq % a.nkv != 0 || a.nq / a.nkv > kAttnMaxGroup) return cudaErrorInvalidValue;
    if (a.hd != 64 && a.hd != 128 && a.hd != 256) return cudaErrorInvalidValue;
    const int ct = attn_ct(a.hd);
    const int G = a.nq / a.nkv;
    if (a.max_chunk < ct || a.max_chunk % ct != 0) return cudaErrorInvalidValue;
    // the merge weights [2][n_splits][G] are laid over the ring
    if (a.n_splits < 1 || (size_t)2 * a.n_splits * G * 4 > (size_t)kAttnStages * kAttnStageBytes)
        return cudaErrorInvalidValue;
    const void* f = nullptr;
    switch (a.hd) {
        case 64: f = reinterpret_cast<const void*>(&k_attn_decode<64>); break;
        case 128: f = reinterpret_cast<const void*>(&k_attn_decode<128>); break;
        default: f = reinterpret_cast<const void*>(&k_attn_decode<256>); break;
    }
    CUtensorMap tk, tv;
    const uint64_t rows = (uint64_t)a.n_pages * a.nkv * kPage;
    if (!make_tmap_bf16_sw128(&tk, a.kc, rows, a.hd, a.hd, kPage)) return cudaErrorInvalidValue;
    if (!make_tmap_bf16_sw128(&tv, a.vc, rows, a.hd, a.hd, kPage)) return cudaErrorInvalidValue;
    const size_t smem = attn_layout(G, a.hd).total;
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
