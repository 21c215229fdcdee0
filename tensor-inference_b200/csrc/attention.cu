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
// Work split: eight warps; warp w owns one 16-token block of every stage and one
// 64-dim box of its P.V (head_dim 128: two warps per block, 256: four).  Scores S = q K^T come
// out of mma.sync m16n8k16 (the group's q heads padded to 16 rows) in exactly
// the register layout of the A operand of the next mma, so P never leaves the
// registers: each warp keeps its own running max and sum per q head (quad
// shuffles), P.V accumulates on the tensor cores with V fragments read by
// ldmatrix.trans from the swizzled tile, and the warps are merged once at
// the end.  A stage is released through an "empty" mbarrier (one arrival per
// warp), not a block barrier.
//
// Arithmetic follows the reference: RoPE in fp32 rounded to bf16; scores
// q.k with bf16 operands and fp32 accumulation (bf16 x bf16 products are exact
// in fp32), times 1/sqrt(head_dim); exp-normalised fp32 softmax, evaluated as
// 2^(s log2(e) - m) with ex2.approx (relative error about 2^-22); bf16 output.
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

constexpr int kAttnThreads = 256;
constexpr int kAttnWarps = kAttnThreads / 32;
constexpr int kAttnMaxGroup = 16;              // q heads per kv head: the 16 rows of the mma
constexpr int kPage = 16;
constexpr int kAttnStages = 6;                 // ring depth
constexpr uint32_t kAttnStageBytes = 16384;    // K + V of one stage
constexpr int kAttnMaxSplits = 512;            // the merge weights fit over the ring
constexpr int kAttnMaxSplitPages = 1024;       // page ids of a split staged in shared memory
constexpr float kLog2e = 1.4426950408889634f;  // softmax in base 2: e^x = 2^(x log2 e)

// tokens per stage: 64 / 32 / 16 for head_dim 64 / 128 / 256 (4 / 2 / 1 pages)
__host__ __device__ constexpr int attn_ct(int HD) { return (int)(kAttnStageBytes / (4u * HD)); }

struct AttnSmem {
    uint32_t ring, qs, kn, vn, wml, hml, pgs, cnt, bar, total;
};

// offsets from a 1024-byte aligned base
__host__ __device__ inline AttnSmem attn_layout(int HD) {
    AttnSmem L;
    uint32_t o = 0;
    L.ring = o;  // [stages] x {K tile [HD/64][CT][64] bf16, V tile}, rows 128-byte swizzled;
    o += kAttnStages * kAttnStageBytes;  // afterwards the warp merge and the split merge weights
    L.qs = o;    // q heads after RoPE, bf16 [HD/64][16][64] swizzled (rows >= G zero)
    o += 16u * HD * 2;
    L.kn = o;    // new token's k after RoPE, and v (fp32)
    o += HD * 4;
    L.vn = o;
    o += HD * 4;
    L.wml = o;   // per warp running (max, sum) per q head [warps][16][2]
    o += kAttnWarps * kAttnMaxGroup * 2 * 4;
    L.hml = o;   // merged (max, sum) per q head [16][2]
    o += kAttnMaxGroup * 2 * 4;
    L.pgs = o;   // page ids of the split
    o += kAttnMaxSplitPages * 4;
    L.cnt = o;   // per slot: warp arrivals so far (WPS per stage)
    o += kAttnStages * 4;
    o = (o + 7u) & ~7u;
    L.bar = o;   // full[stages]
    o += kAttnStages * 8;
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
// the warps' merge area over the ring: [warps][16 q heads][kRedStride] fp32; the
// row stride of 128 + 8 floats puts the 64-bit stores of a half-warp (8 rows x 4
// column pairs) on 32 distinct banks and keeps rows 16-byte aligned
constexpr int kRedStride = 136;
// cluster merge: offsets in the ring (free after the warps' merge, whose area ends
// below 72 KB): partial output [G][hd] (<= 16 KB), (max, sum) per q head, split 0's
// weights [n_splits][G][2]
constexpr uint32_t kClusterPartOff = 72u * 1024u;
constexpr uint32_t kClusterMlOff = kClusterPartOff + 16u * 1024u;
constexpr uint32_t kClusterWOff = kClusterMlOff + 256u;
constexpr int kAttnMaxCluster = 8;  // portable cluster size
static_assert(kClusterWOff + kAttnMaxCluster * kAttnMaxGroup * 8 <= kAttnStages * kAttnStageBytes, "ring holds it");

// all threads of every CTA of the cluster (release / acquire: shared-memory writes
// before it are visible to the cluster's reads after it)
TI_DEVICE_INLINE void cluster_sync_all() {
    asm volatile("barrier.cluster.arrive.release.aligned;\n\tbarrier.cluster.wait.acquire.aligned;" ::: "memory");
}
// load from the same shared-memory offset in cluster CTA `rank`
TI_DEVICE_INLINE float ld_dsmem_f32(const float* p, int rank) {
    uint32_t ra;
    float v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(p)), "r"(rank));
    asm volatile("ld.shared::cluster.f32 %0, [%1];" : "=f"(v) : "r"(ra) : "memory");
    return v;
}
TI_DEVICE_INLINE float4 ld_dsmem_f32x4(const float* p, int rank) {
    uint32_t ra;
    float4 v;
    asm volatile("mapa.shared::cluster.u32 %0, %1, %2;" : "=r"(ra) : "r"(smem_u32(p)), "r"(rank));
    asm volatile("ld.shared::cluster.v4.f32 {%0, %1, %2, %3}, [%4];"
                 : "=f"(v.x), "=f"(v.y), "=f"(v.z), "=f"(v.w)
                 : "r"(ra)
                 : "memory");
    return v;
}

// byte offset of element (row, d) in a [HD/64][C][64] bf16 tile with 128-byte swizzled rows
TI_DEVICE_INLINE uint32_t tile_off(int C, int row, int d) {
    const int hh = d >> 6, cc = (d & 63) >> 3;
    return (uint32_t)(hh * C + row) * 128u + (uint32_t)((cc ^ (row & 7)) << 4) + (uint32_t)((d & 7) << 1);
}
// wait (bounded) until a shared counter reaches `need`
TI_DEVICE_INLINE bool wait_count(const unsigned int* p, unsigned int need, int* err, int err_bit) {
    const volatile unsigned int* v = p;
    if (*v >= need) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (*v >= need) return true;
        if ((i & 255u) == 255u && global_ns() - t0 > kWaitNs) break;
    }
    if (err) atomicOr(err, err_bit);
    return false;
}
// two fp32 probabilities -> bf16 pair hi and the bf16 pair of what hi left out
TI_DEVICE_INLINE void split_bf2(float p0, float p1, uint32_t& hi, uint32_t& lo) {
    hi = pack_bf2(p0, p1);
    lo = pack_bf2(p0 - bf_lo(hi), p1 - bf_hi(hi));
}

// G16: the group has more than 8 q heads (rows 8..15 of the mma are real heads)
template <int HD, bool G16>
__global__ void __launch_bounds__(kAttnThreads, 2)
    k_attn_decode(const __grid_constant__ CUtensorMap tk, const __grid_constant__ CUtensorMap tv, const AttnArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    constexpr int HALF = HD / 2;
    constexpr int NH = HD / 64;                    // 64-dim boxes per row
    constexpr int KS = HD / 16;                    // mma k-steps of the scores
    constexpr int CT = attn_ct(HD);                // tokens per stage
    constexpr int CP = CT / kPage;                 // pages (= 16-token blocks) per stage
    constexpr int NS = kAttnStages;
    constexpr int DW = HD < 128 ? HD : 128;        // dims of a warp's P.V
    constexpr int DPARTS = HD / DW;                // warps sharing a block split its dims
    constexpr int NT = DW / 8;                     // P.V n-tiles
    constexpr int WPS = CP * DPARTS;               // warps per stage
    constexpr int SG = kAttnWarps / WPS;           // stages in progress at once
    static_assert(SG * WPS == kAttnWarps, "warps cover whole stages");
    constexpr uint32_t VOFF = kAttnStageBytes / 2;  // V tile after the K tile of a stage
    const int split = blockIdx.x, h = blockIdx.y, b = blockIdx.z;
    const int tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    const int gq = lane >> 2, qq = lane & 3;      // mma fragment row / column pair
    const int so = warp / WPS, wi = warp % WPS;   // stage group, place in the stage
    const int blk = wi % CP, dp = wi / CP;        // block of the stage, dim part
    const int G = a.nq / a.nkv;
    const AttnSmem L = attn_layout(HD);
    uint8_t* ring = smem + L.ring;
    uint8_t* qs = smem + L.qs;
    float* kn = reinterpret_cast<float*>(smem + L.kn);
    float* vn = reinterpret_cast<float*>(smem + L.vn);
    float* wml = reinterpret_cast<float*>(smem + L.wml);
    float* hml = reinterpret_cast<float*>(smem + L.hml);
    int* pgs = reinterpret_cast<int*>(smem + L.pgs);
    unsigned int* cnt = reinterpret_cast<unsigned int*>(smem + L.cnt);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.bar);
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

    // stage st -> ring slot st % NS: its pages' K and V boxes on one barrier;
    // ids[i] is the page id of split page i (the page table, or its copy in pgs)
    auto issue = [&](int st, const int* ids) {
        uint8_t* kt = ring + (uint32_t)(st % NS) * kAttnStageBytes;
        const int i0 = st * CP, pn = min(CP, npg - i0);
        int nv = 0;
        for (int p = 0; p < pn; ++p) {
            const int page = ids[i0 + p];
            nv += page >= 0 && page < a.n_pages;
        }
        if (nv < pn && a.err) atomicOr(a.err, kErrBadIndex);
        mbar_arrive_expect_tx(&full[st % NS], (uint32_t)nv * 2u * NH * kPage * 128u);
        for (int p = 0; p < pn; ++p) {
            const int page = ids[i0 + p];
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

    // ---- before the dependency wait: stages of cached pages.  The page holding
    //      `pos` may have been allocated in this step (its page-table entry is
    //      written by the step's first kernel), so a stage holding it waits.
    const int n_pre = min(NS, n_st);
    const int last_page = pos / kPage - pg0;  // split page index of pos (may be out of range)
    // (prefill: pages written by this step's kv_append hold rows of earlier entries)
    auto early = [&](int st) { return !a.prefill && st * CP + min(CP, npg - st * CP) - 1 < last_page; };
    if (tid == 0) {
        for (int s = 0; s < NS; ++s) mbar_init(&full[s], 1);
        fence_barrier_init();
        for (int st = 0; st < n_pre; ++st)
            if (early(st)) issue(st, pt + pg0);
        pdl_trigger();
    }
    if (tid < NS) cnt[tid] = 0u;

    pdl_wait();  // the new token's q/k/v are the previous kernel's output
    for (int i = tid; i < npg; i += kAttnThreads) pgs[i] = pt[pg0 + i];
    if (tid == 0)
        for (int st = 0; st < n_pre; ++st)
            if (!early(st)) issue(st, pt + pg0);

    // ---- RoPE on the group's q heads and the new k (ops.cu:224-232); v as is
    // all of a thread's q/k/v loads are issued before any of them is used (one
    // round trip to L2, not one per task)
    const uint16_t* row = a.qkv + (size_t)b * a.qkv_stride;
    constexpr int kRopeMax = ((kAttnMaxGroup + 1) * HALF + kAttnThreads - 1) / kAttnThreads;
    const int n_task = (G + 1) * HALF;
    float rx0[kRopeMax], rx1[kRopeMax], rf[kRopeMax];
#pragma unroll
    for (int k = 0; k < kRopeMax; ++k) {
        const int task = tid + k * kAttnThreads;
        if (task < n_task) {
            const int hh = task / HALF, i = task - hh * HALF;
            const uint16_t* src = hh < G ? row + (size_t)(h * G + hh) * HD : row + (size_t)(a.nq + h) * HD;
            rx0[k] = __uint_as_float((uint32_t)src[i] << 16);
            rx1[k] = __uint_as_float((uint32_t)src[i + HALF] << 16);
            rf[k] = a.freqs[i];
        }
    }
    const float vval = tid < HD ? __uint_as_float((uint32_t)row[(size_t)(a.nq + a.nkv + h) * HD + tid] << 16) : 0.f;
#pragma unroll
    for (int k = 0; k < kRopeMax; ++k) {
        const int task = tid + k * kAttnThreads;
        if (task < n_task) {
            const int hh = task / HALF, i = task - hh * HALF;
            const float x0 = rx0[k], x1 = rx1[k];
            const float ang = (float)pos * rf[k];
            const float c = cosf(ang), s = sinf(ang);
            const float y0 = x0 * c - x1 * s, y1 = x0 * s + x1 * c;
            if (hh < G) {
                *reinterpret_cast<bf16*>(qs + tile_off(16, hh, i)) = f2bf(y0);
                *reinterpret_cast<bf16*>(qs + tile_off(16, hh, i + HALF)) = f2bf(y1);
            } else {
                kn[i] = round_bf(y0);
                kn[i + HALF] = round_bf(y1);
            }
        }
    }
    for (int task = tid; task < (16 - G) * HD; task += kAttnThreads) {  // padding heads
        const int hh = G + task / HD, d = task % HD;
        *reinterpret_cast<bf16*>(qs + tile_off(16, hh, d)) = f2bf(0.f);
    }
    static_assert(HD <= kAttnThreads, "one v element per thread");
    if (tid < HD) vn[tid] = vval;
    __syncthreads();

    // lane-constant parts of the swizzled ldmatrix addresses (the row's low 3 bits
    // are the lane's, so the chunk XOR only depends on the lane and a constant)
    const uint32_t x7 = (uint32_t)(lane & 7);
    const uint32_t q_lane = ((lane & 7) + ((lane >> 3) & 1) * 8) * 128u;               // q: rows
    const uint32_t q_y = ((uint32_t)(lane >> 4) ^ x7);                                  // q chunk
    const uint32_t k_lane = (blk * 16 + (lane & 7)) * 128u;                             // K rows
    const uint32_t k_y = ((uint32_t)(lane >> 3) ^ x7);                                  // K chunk
    const uint32_t v_lane = (blk * 16 + (lane & 7) + ((lane >> 3) & 1) * 8) * 128u;    // V rows
    const uint32_t v_y = ((uint32_t)(lane >> 4) ^ x7);                                  // V chunk
    const uint32_t qbase = smem_u32(qs);
    const float scale2 = a.scale * kLog2e;
    const int j0 = blk * 16;  // this warp's block: stage rows [j0, j0 + 16)

    float o[NT][4];
#pragma unroll
    for (int n = 0; n < NT; ++n) o[n][0] = o[n][1] = o[n][2] = o[n][3] = 0.f;
    float m0 = -INFINITY, m1 = -INFINITY, l0 = 0.f, l1 = 0.f;  // heads gq, gq + 8 (base-2 units)

    for (int st = so; st < n_st; st += SG) {
        uint8_t* kt = ring + (uint32_t)(st % NS) * kAttnStageBytes;
        uint8_t* vt = kt + VOFF;
        const int r0 = st * CT;  // split row of stage row 0
        const int rows = min(CP, npg - st * CP) * kPage;
        const int jlo = max(vlo - r0, 0), jhi = min(vhi - r0, rows);  // valid stage rows
        // stage groups run apart: the slot may still hold stage st - NS (another
        // group's), whose barrier phase a parity wait cannot tell from this one.
        // Its WPS arrivals per earlier stage show when it is done.
        if (st >= NS) wait_count(&cnt[st % NS], (unsigned)WPS * (unsigned)(st / NS), a.err, kErrTimeoutEmpty);
        mbar_wait(&full[st % NS], (uint32_t)(st / NS) & 1u, a.err, kErrTimeoutFull);
        __syncwarp();  // lanes leave the poll apart; ldmatrix and mma need the whole warp

        // the warp(s) of the block holding `pos` put the new K/V row into the tile
        // (each writes the whole row before reading it) and one of them into the page
        if (pos >= t0 + r0 + j0 && pos < t0 + r0 + j0 + kPage && j0 < rows) {
            const int r = pos - t0 - r0;
            for (int d = lane; d < HD; d += 32) {
                const uint32_t off = tile_off(CT, r, d);
                *reinterpret_cast<bf16*>(kt + off) = f2bf(kn[d]);
                *reinterpret_cast<bf16*>(vt + off) = f2bf(vn[d]);
            }
            if (dp == 0) {
                const int page = pgs[pos / kPage - pg0];
                if (page >= 0 && page < a.n_pages) {
                    const size_t off = (((size_t)page * a.nkv + h) * kPage + (pos % kPage)) * HD;
                    for (int d = lane; d < HD; d += 32) {
                        reinterpret_cast<bf16*>(a.kc)[off + d] = f2bf(kn[d]);
                        reinterpret_cast<bf16*>(a.vc)[off + d] = f2bf(vn[d]);
                    }
                } else if (lane == 0 && a.err) {
                    atomicOr(a.err, kErrBadIndex);
                }
            }
            // the slot is refilled by TMA later: order these generic writes before it
            asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            __syncwarp();
        }

        if (j0 + 16 > jlo && j0 < jhi) {  // warp-uniform
            const bool edge = j0 < jlo || j0 + 16 > jhi;
            if (edge) {
                // rows outside [jlo, jhi) get probability 0: make their V finite (zero)
                for (int t = lane; t < 16 * (DW / 8); t += 32) {
                    const int jr = j0 + t / (DW / 8), d = dp * DW + (t % (DW / 8)) * 8;
                    if (jr < jlo || jr >= jhi) *reinterpret_cast<uint4*>(vt + tile_off(CT, jr, d)) = make_uint4(0, 0, 0, 0);
                }
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
                __syncwarp();
            }
            // ---- scores of 16 tokens: two n-tiles of 8, two accumulator chains each
            float c[2][4], c2[2][4];
            const uint32_t kbase = smem_u32(kt) + k_lane;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) c[nt][e] = c2[nt][e] = 0.f;
#pragma unroll
            for (int ks = 0; ks < KS; ks += 2) {
                uint32_t qa0[4], qa1[4];
                const uint32_t qoff = (uint32_t)(ks >> 2) * 16u * 128u;
                ldsm_x4(qbase + qoff + q_lane + ((((uint32_t)(ks & 3) * 2u) ^ q_y) << 4), qa0[0], qa0[1], qa0[2],
                        qa0[3]);
                ldsm_x4(qbase + qoff + q_lane + ((((uint32_t)((ks + 1) & 3) * 2u) ^ q_y) << 4), qa1[0], qa1[1],
                        qa1[2], qa1[3]);
                const uint32_t koff = (uint32_t)(ks >> 2) * CT * 128u + ((((uint32_t)(ks & 2) * 2u) ^ k_y) << 4);
#pragma unroll
                for (int nt = 0; nt < 2; ++nt) {
                    uint32_t b0, b1, b2, b3;
                    ldsm_x4(kbase + koff + nt * 1024u, b0, b1, b2, b3);
                    mma_16816_bf16(c[nt], qa0, b0, b1);
                    mma_16816_bf16(c2[nt], qa1, b2, b3);
                }
            }
            // c[nt][0..1]: head gq, rows j0 + 8 nt + 2 qq + {0,1}; c[nt][2..3]: head gq + 8
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int e = 0; e < 4; ++e) c[nt][e] = (c[nt][e] + c2[nt][e]) * scale2;
            if (edge) {
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int e = 0; e < 2; ++e) {
                        const int jj = j0 + nt * 8 + qq * 2 + e;
                        if (jj < jlo || jj >= jhi) c[nt][e] = c[nt][2 + e] = -INFINITY;
                    }
            }
            // ---- online softmax (ops.cu:393-419 over the whole row), base 2
            float mx0 = fmaxf(fmaxf(c[0][0], c[0][1]), fmaxf(c[1][0], c[1][1]));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 1));
            mx0 = fmaxf(mx0, __shfl_xor_sync(0xffffffffu, mx0, 2));
            const float n0 = fmaxf(m0, mx0);
            const float u0 = n0 == -INFINITY ? 0.f : n0;
            const float al0 = ex2(m0 - u0);  // 0 while nothing was seen
            m0 = n0;
            float s0 = 0.f;
#pragma unroll
            for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                for (int e = 0; e < 2; ++e) {
                    c[nt][e] = ex2(c[nt][e] - u0);
                    s0 += c[nt][e];
                }
            l0 = fmaf(l0, al0, s0);
            float al1 = 1.f;
            if constexpr (G16) {
                float mx1 = fmaxf(fmaxf(c[0][2], c[0][3]), fmaxf(c[1][2], c[1][3]));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 1));
                mx1 = fmaxf(mx1, __shfl_xor_sync(0xffffffffu, mx1, 2));
                const float n1 = fmaxf(m1, mx1);
                const float u1 = n1 == -INFINITY ? 0.f : n1;
                al1 = ex2(m1 - u1);
                m1 = n1;
                float s1 = 0.f;
#pragma unroll
                for (int nt = 0; nt < 2; ++nt)
#pragma unroll
                    for (int e = 2; e < 4; ++e) {
                        c[nt][e] = ex2(c[nt][e] - u1);
                        s1 += c[nt][e];
                    }
                l1 = fmaf(l1, al1, s1);
            } else {
                c[0][2] = c[0][3] = c[1][2] = c[1][3] = 0.f;  // padding heads
            }
            if (__any_sync(0xffffffffu, al0 != 1.f || al1 != 1.f)) {
#pragma unroll
                for (int n = 0; n < NT; ++n) {
                    o[n][0] *= al0;
                    o[n][1] *= al0;
                    if constexpr (G16) {
                        o[n][2] *= al1;
                        o[n][3] *= al1;
                    }
                }
            }
            // ---- P.V: A = P (heads x 16 tokens) as hi + lo bf16 pairs, B = V via ldmatrix.trans
            uint32_t ph[4], pl[4];
            split_bf2(c[0][0], c[0][1], ph[0], pl[0]);
            split_bf2(c[1][0], c[1][1], ph[2], pl[2]);
            if constexpr (G16) {
                split_bf2(c[0][2], c[0][3], ph[1], pl[1]);
                split_bf2(c[1][2], c[1][3], ph[3], pl[3]);
            } else {
                ph[1] = pl[1] = ph[3] = pl[3] = 0u;
            }
            const uint32_t vbase = smem_u32(vt) + v_lane + (uint32_t)(dp * DW / 64) * CT * 128u;
#pragma unroll
            for (int n = 0; n < NT; n += 2) {
                uint32_t b0, b1, b2, b3;
                ldsm_x4_t(vbase + (uint32_t)(n / 8) * CT * 128u + ((((uint32_t)(n & 7)) ^ v_y) << 4), b0, b1, b2,
                          b3);
                mma_16816_bf16(o[n], ph, b0, b1);
                mma_16816_bf16(o[n + 1], ph, b2, b3);
                mma_16816_bf16(o[n], pl, b0, b1);
                mma_16816_bf16(o[n + 1], pl, b2, b3);
            }
        }
        // release the slot: the last of its warps to finish refills it
        __syncwarp();
        if (lane == 0) {
            __threadfence_block();
            // the count only grows: every WPS-th arrival on a slot ends a stage
            const unsigned int done = atomicAdd(&cnt[st % NS], 1u);
            if ((done + 1u) % (unsigned)WPS == 0u) {
                __threadfence_block();
                if (st + NS < n_st) issue(st + NS, pgs);
            }
        }
        __syncwarp();
    }

    // ---- merge the warps: per head the max over the warps of dim part 0 (they
    //      saw every block; the other parts saw the same ones), each warp's
    //      accumulators and sums rescaled to it, summed in warp order
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
    auto part_of = [&](int w) { return (w % WPS) / CP; };
    if (tid < kAttnMaxGroup) {
        float M = -INFINITY;
        for (int w = 0; w < kAttnWarps; ++w)
            if (part_of(w) == 0) M = fmaxf(M, wml[(w * 16 + tid) * 2]);
        float Ls = 0.f;
        for (int w = 0; w < kAttnWarps; ++w) {
            const float mw = wml[(w * 16 + tid) * 2];
            if (part_of(w) == 0 && mw != -INFINITY) Ls = fmaf(wml[(w * 16 + tid) * 2 + 1], ex2(mw - M), Ls);
        }
        hml[2 * tid] = M;
        hml[2 * tid + 1] = Ls;
    }
    __syncthreads();
    float* red = reinterpret_cast<float*>(ring);  // [warps][16][kRedStride]
    static_assert(kAttnWarps * 16 * kRedStride * 4 <= kClusterPartOff, "merge area below the cluster partials");
    {
        const float M0 = hml[2 * gq], M1 = hml[2 * (gq + 8)];
        const float f0 = m0 == -INFINITY ? 0.f : ex2(m0 - M0);
        const float f1 = m1 == -INFINITY ? 0.f : ex2(m1 - M1);
#pragma unroll
        for (int n = 0; n < NT; ++n) {
            const int d = n * 8 + qq * 2;
            *reinterpret_cast<float2*>(red + ((size_t)warp * 16 + gq) * kRedStride + d) =
                make_float2(o[n][0] * f0, o[n][1] * f0);
            *reinterpret_cast<float2*>(red + ((size_t)warp * 16 + gq + 8) * kRedStride + d) =
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
        for (int w = 0; w < kAttnWarps; ++w) {
            if (part_of(w) != part) continue;
            const float4 v = *reinterpret_cast<const float4*>(red + ((size_t)w * 16 + g) * kRedStride + dl);
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
        } else if (a.cluster) {
            *reinterpret_cast<float4*>(ring + kClusterPartOff + (size_t)e * 4) = O;
        } else {
            *reinterpret_cast<float4*>(a.part_o + (pbase + g) * HD + d) = O;
        }
    }
    if (a.n_splits == 1) return;

    if (a.cluster) {
        // ---- the splits of this (token, kv head) are one thread-block cluster: each
        //      leaves its partial in its own shared memory, split 0 reads them all
        //      through distributed shared memory and merges in split order.  Every
        //      thread of every CTA passes both cluster barriers (no early exit).
        float* cml = reinterpret_cast<float*>(ring + kClusterMlOff);
        if (tid < G) {
            cml[2 * tid] = hml[2 * tid];
            cml[2 * tid + 1] = hml[2 * tid + 1];
        }
        cluster_sync_all();
        if (split == 0) {
            float* wsg = reinterpret_cast<float*>(ring + kClusterWOff);  // [n_splits][G] (max, then weight; sum)
            for (int idx = tid; idx < a.n_splits * G; idx += kAttnThreads) {
                const int sp = idx / G, g = idx - sp * G;
                wsg[2 * idx] = ld_dsmem_f32(cml + 2 * g, sp);
                wsg[2 * idx + 1] = ld_dsmem_f32(cml + 2 * g + 1, sp);
            }
            __syncthreads();
            if (tid < G) {
                float M = -INFINITY;
                for (int sp = 0; sp < a.n_splits; ++sp)
                    if (wsg[2 * (sp * G + tid) + 1] > 0.f) M = fmaxf(M, wsg[2 * (sp * G + tid)]);
                float Ls = 0.f;
                for (int sp = 0; sp < a.n_splits; ++sp) {
                    const float l = wsg[2 * (sp * G + tid) + 1];
                    const float w = l > 0.f ? ex2(wsg[2 * (sp * G + tid)] - M) : 0.f;
                    wsg[2 * (sp * G + tid)] = w;
                    Ls = fmaf(l, w, Ls);
                }
                hml[2 * tid + 1] = Ls;
            }
            __syncthreads();
            const float* cpo = reinterpret_cast<const float*>(ring + kClusterPartOff);
            for (int e = tid * 4; e < G * HD; e += kAttnThreads * 4) {
                const int g = e / HD;
                float4 v[kAttnMaxCluster];  // every split's values in flight together
#pragma unroll
                for (int sp = 0; sp < kAttnMaxCluster; ++sp)
                    if (sp < a.n_splits) v[sp] = ld_dsmem_f32x4(cpo + e, sp);
                float4 O = make_float4(0.f, 0.f, 0.f, 0.f);
#pragma unroll
                for (int sp = 0; sp < kAttnMaxCluster; ++sp) {
                    if (sp >= a.n_splits) break;
                    const float w = wsg[2 * (sp * G + g)];
                    O.x = fmaf(v[sp].x, w, O.x);
                    O.y = fmaf(v[sp].y, w, O.y);
                    O.z = fmaf(v[sp].z, w, O.z);
                    O.w = fmaf(v[sp].w, w, O.w);
                }
                const float inv = hml[2 * g + 1];
                bf16* dst = reinterpret_cast<bf16*>(a.out) + (size_t)b * a.out_stride + (size_t)h * G * HD + e;
                dst[0] = f2bf(O.x / inv);
                dst[1] = f2bf(O.y / inv);
                dst[2] = f2bf(O.z / inv);
                dst[3] = f2bf(O.w / inv);
            }
        }
        cluster_sync_all();  // the other splits' shared memory stays until split 0 has read it
        return;
    }

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
    // split weights w[s][g] = 2^(m_s - M_g) (0 for empty splits), over the ring
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
            const float w = l > 0.f ? ex2(wsg[s * G + tid] - M) : 0.f;
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

// K (RoPE, ops.cu:224-232, the same arithmetic as the attention kernel's) and V
// rows of every entry into its page: one CTA per entry
__global__ void __launch_bounds__(128) k_kv_append(const AttnArgs a) {
    if (threadIdx.x == 0) pdl_trigger();
    pdl_wait();  // q/k/v are the previous kernel's output
    const int b = blockIdx.x, hd = a.hd, half = hd / 2;
    const int pos = a.pos[b];
    const int page = a.page_table[(size_t)a.seq[b] * a.pt_stride + pos / kPage];
    if (page < 0 || page >= a.n_pages) {
        if (threadIdx.x == 0 && a.err) atomicOr(a.err, kErrBadIndex);
        return;
    }
    const uint16_t* row = a.qkv + (size_t)b * a.qkv_stride;
    for (int task = threadIdx.x; task < a.nkv * half; task += blockDim.x) {
        const int h = task / half, i = task - h * half;
        const uint16_t* src = row + (size_t)(a.nq + h) * hd;
        const float x0 = __uint_as_float((uint32_t)src[i] << 16);
        const float x1 = __uint_as_float((uint32_t)src[i + half] << 16);
        const float ang = (float)pos * a.freqs[i];
        const float c = cosf(ang), sn = sinf(ang);
        const size_t off = (((size_t)page * a.nkv + h) * kPage + (pos % kPage)) * hd;
        reinterpret_cast<bf16*>(a.kc)[off + i] = f2bf(round_bf(x0 * c - x1 * sn));
        reinterpret_cast<bf16*>(a.kc)[off + i + half] = f2bf(round_bf(x0 * sn + x1 * c));
    }
    for (int task = threadIdx.x; task < a.nkv * hd; task += blockDim.x) {
        const int h = task / hd, d = task - h * hd;
        const size_t off = (((size_t)page * a.nkv + h) * kPage + (pos % kPage)) * hd;
        a.vc[off + d] = row[(size_t)(a.nq + a.nkv + h) * hd + d];
    }
}

cudaError_t kv_append_launch(const AttnArgs& a, cudaStream_t s, bool pdl) {
    if (a.nkv <= 0 || a.hd % 2 != 0 || a.nb < 1) return cudaErrorInvalidValue;
    AttnArgs args = a;
    void* params[] = {&args};
    return launch_pdl(reinterpret_cast<const void*>(&k_kv_append), dim3(a.nb), dim3(128), 0, s, params, pdl);
}

int attn_splits(int nb, int nkv, int hd, int max_len, int sms, int* max_chunk) {
    // Splits per (token, kv head) pair, chosen on a cost model of the grid: CTAs
    // run two per SM (S = 2 sms slots); while at least `sms` CTAs are active the
    // grid streams at the HBM rate, below that each CTA is limited by its own
    // loads in flight.  Cost = (full waves + the last wave's share, counted as at
    // least sms CTAs) x (stages per split + a fixed start-up cost).  Long splits
    // amortise the start (first loads, RoPE) and the merge; the model avoids a
    // last wave of a few long CTAs.  Env TI_ATTN_SPP forces the stages per split.
    const int ct = attn_ct(hd), cp = ct / kPage;
    const int max_pages = std::max(1, (max_len + kPage - 1) / kPage);
    const int stages = (max_pages + cp - 1) / cp;
    const int max_spp = std::max(1, std::min(stages, kAttnMaxSplitPages / cp));
    const int min_n = std::max((stages + max_spp - 1) / max_spp, 1);
    int spp = 0;
    const char* env = std::getenv("TI_ATTN_SPP");
    if (env && std::atoi(env) >= 1) {
        spp = std::min(std::atoi(env), max_spp);
        spp = std::max(spp, (stages + kAttnMaxSplits - 1) / kAttnMaxSplits);
    } else {
        constexpr double kStartStages = 3.0;
        const long pairs = std::max(1, nb * nkv);
        const long S = 2L * sms, Q = sms;
        double best = 0.0;
        for (int n = min_n; n <= std::min(stages, kAttnMaxSplits); ++n) {
            const int sp = (stages + n - 1) / n;
            if ((stages + sp - 1) / sp != n) continue;  // the same split as a smaller n
            const long C = pairs * n, full = (C - 1) / S, r = C - full * S;
            const double cost = ((double)full + (double)std::max(r, Q) / (double)S) * ((double)sp + kStartStages);
            if (spp == 0 || cost < best) {
                best = cost;
                spp = sp;
            }
        }
    }
    int n = (stages + spp - 1) / spp;
    // up to 8 splits merge inside a thread-block cluster, without the global
    // partials' round trips: take 8 when that leaves at most 4 stages per split
    if (!(env && std::atoi(env) >= 1) && n > kAttnMaxCluster &&
        (stages + kAttnMaxCluster - 1) / kAttnMaxCluster <= 4) {
        spp = (stages + kAttnMaxCluster - 1) / kAttnMaxCluster;
        n = (stages + spp - 1) / spp;
    }
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
    if (a.max_chunk < ct || a.max_chunk % ct != 0 || a.max_chunk / kPage > kAttnMaxSplitPages)
        return cudaErrorInvalidValue;
    // the merge weights [2][n_splits][G] are laid over the ring
    if (a.n_splits < 1 || (size_t)2 * a.n_splits * G * 4 > (size_t)kAttnStages * kAttnStageBytes)
        return cudaErrorInvalidValue;
    const void* f = nullptr;
    const bool g16 = G > 8;
    switch (a.hd) {
        case 64: f = g16 ? reinterpret_cast<const void*>(&k_attn_decode<64, true>)
                         : reinterpret_cast<const void*>(&k_attn_decode<64, false>); break;
        case 128: f = g16 ? reinterpret_cast<const void*>(&k_attn_decode<128, true>)
                          : reinterpret_cast<const void*>(&k_attn_decode<128, false>); break;
        default: f = g16 ? reinterpret_cast<const void*>(&k_attn_decode<256, true>)
                         : reinterpret_cast<const void*>(&k_attn_decode<256, false>); break;
    }
    CUtensorMap tk, tv;
    const uint64_t rows = (uint64_t)a.n_pages * a.nkv * kPage;
    if (!make_tmap_bf16_sw128(&tk, a.kc, rows, a.hd, a.hd, kPage)) return cudaErrorInvalidValue;
    if (!make_tmap_bf16_sw128(&tv, a.vc, rows, a.hd, a.hd, kPage)) return cudaErrorInvalidValue;
    const size_t smem = attn_layout(a.hd).total;
    if (smem > 227 * 1024) return cudaErrorInvalidValue;
    {
        static std::mutex mu;
        std::lock_guard<std::mutex> lk(mu);
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    AttnArgs args = a;
    void* params[] = {&tk, &tv, &args};
    if (a.n_splits < 2 || a.n_splits > kAttnMaxCluster)
        return launch_pdl(f, dim3(a.n_splits, a.nkv, a.nb), dim3(kAttnThreads), smem, s, params, pdl);
    // the splits of each (token, kv head) as one cluster (merge in distributed shared memory)
    args.cluster = 1;
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = dim3(a.n_splits, a.nkv, a.nb);
    cfg.blockDim = dim3(kAttnThreads);
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[2];
    attr[0].id = cudaLaunchAttributeClusterDimension;
    attr[0].val.clusterDim.x = (unsigned)a.n_splits;
    attr[0].val.clusterDim.y = 1;
    attr[0].val.clusterDim.z = 1;
    attr[1].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[1].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 2 : 1;
    return cudaLaunchKernelExC(&cfg, f, params);
}

}  // namespace ti
