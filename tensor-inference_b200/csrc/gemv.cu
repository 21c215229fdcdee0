// gemv.cu — weight-streaming GEMV for decode (few tokens; bf16, GGUF Q4_0 or Q8_0 weights).
//
// Replaces ops::matmul_t at M = tokens (src/backend/cuda/ops.cu:94-148, one
// cuBLAS GemmEx per projection) and fuses the ops around it in the model code
// (llama_model.cpp:115-203, qwen_model.cpp:80-128):
//   prologue  RMSNorm of the input row (ops.cu:154-204 / 726-774)
//   epilogue  bias (ops.cu:671-701), residual add (ops.cu:361-381),
//             SiLU/GELU * up (ops.cu:318-359, 707-724), LoRA delta
//             (qwen_adapter_model.cpp:22-43), LM-head greedy argmax
//             (greedy.cpp:11-36, done on fp32 logits on the device).
// The bf16 rounding points of the reference are kept: every op output the
// model code materialises as a bf16 Tensor is rounded to bf16 here too.
// Quantised weights are dequantised in registers as they are consumed: each
// element becomes the exact fp32 value d * (q - 8) (Q4_0) or d * q (Q8_0) that
// GGUF's block formats define, then enters the same fp32 FMAs as a bf16 weight.
//
// Structure (one CTA per SM, 16 consumer warps + 1 producer warp + 1 epilogue warp):
//   producer: streams the CTA's contiguous row range of W from HBM into a ring
//     of shared-memory stages with cp.async.bulk (TMA, 1-D, evict-first L2
//     policy), completion on mbarriers, and keeps an L2 prefetch window
//     (cp.async.bulk.prefetch.L2) `pf` stages ahead of the ring, so the bytes
//     in flight to HBM are not bounded by shared memory.  It starts before
//     griddepcontrol.wait: weights never depend on the previous kernel.
//   consumers: warp w owns columns [w*K/16, (w+1)*K/16) of every row; its slice
//     of the (normalised) activation stays in registers (one token) or shared
//     memory (several).  Per stage: fp32 FMAs in element order for all rows,
//     one batched butterfly reduction, and the per-warp partial sums go to a
//     ring of partial slots (mbarrier full/empty pairs) — consumer warps never
//     wait for one another.
//   epilogue warp: per stage, sums the 16 warp partials of each row in warp
//     order (deterministic) and applies the fused epilogue.
#include "attn_fused.cuh"
#include "common.cuh"
#include "kernels.h"
#include "lora_epi.cuh"

#include <algorithm>
#include <cstdio>
#include <cstdlib>

namespace ti {

constexpr int kConsumerWarps = 16;
constexpr int kProducerWarp = kConsumerWarps;
constexpr int kEpilogueWarp = kConsumerWarps + 1;
constexpr int kThreads = (kConsumerWarps + 2) * 32;
constexpr int kPartSlots = 8;  // stages of partial sums in flight to the epilogue warp
constexpr int kRowsMax = 12;  // rows per stage (per unit) upper bound, for one token

struct GemvSmem {
    uint32_t stage_bytes, stages_off, full_off, empty_off, pfull_off, pempty_off, go_off, part_off, red_off, xs_off,
        epi_off, att_off, total;
};

// rows_cap: most rows one CTA owns; the epilogue warp keeps their residual
// (nb rows) and bias values in shared memory
// att_bytes: the fused attention phase's region (0 without it)
__host__ __device__ inline GemvSmem gemv_smem_layout(int K, int wf, int units, int rows_per_stage, int stages,
                                                     int nb, bool x_in_smem, int rows_cap, uint32_t att_bytes = 0) {
    GemvSmem L;
    uint32_t sb = (uint32_t)(rows_per_stage * units * wrow_bytes(K, wf));
    sb = (sb + 127u) & ~127u;
    L.stage_bytes = sb;
    L.stages_off = 0;
    uint32_t o = sb * stages;
    L.full_off = o;
    o += 8 * stages;
    L.empty_off = o;
    o += 8 * stages;
    L.pfull_off = o;
    o += 8 * kPartSlots;
    L.pempty_off = o;
    o += 8 * kPartSlots;
    L.go_off = o;  // ATT: the consumers' go for the producer's shared-memory fills
    o += 8;
    L.part_off = o;
    o += kPartSlots * rows_per_stage * units * nb * kConsumerWarps * 4;
    L.red_off = o;
    o += kConsumerWarps * nb * 4;
    o = (o + 15u) & ~15u;
    L.xs_off = o;
    if (x_in_smem) o += (uint32_t)nb * K * 2;
    o = (o + 15u) & ~15u;
    L.epi_off = o;
    o += (uint32_t)(nb + 1) * rows_cap * 2;
    o = (o + 15u) & ~15u;
    L.att_off = o;
    o += att_bytes;
    o = (o + 15u) & ~15u;
    L.total = o;
    return L;
}

TI_DEVICE_INLINE float glu_act(float g, int act) {
    if (act == 0) return round_bf(g / (1.0f + expf(-g)));  // ops.cu:326
    const float c1 = 0.7978845608f, c2 = 0.044715f;        // ops.cu:712-714
    return round_bf(0.5f * g * (1.0f + tanhf(c1 * (g + c2 * g * g * g))));
}

TI_DEVICE_INLINE void normalise8(uint4& v, const uint4 wn, float scale, float off) {
    uint32_t* vp = reinterpret_cast<uint32_t*>(&v);
    const uint32_t* wp = reinterpret_cast<const uint32_t*>(&wn);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        const float lo = bf_lo(vp[e]) * scale * (bf_lo(wp[e]) + off);
        const float hi = bf_hi(vp[e]) * scale * (bf_hi(wp[e]) + off);
        vp[e] = pack_bf2(lo, hi);
    }
}

TI_DEVICE_INLINE float sumsq8(const uint4 v, float ss) {
    const uint32_t* vp = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
    for (int e = 0; e < 4; ++e) {
        ss = fmaf(bf_lo(vp[e]), bf_lo(vp[e]), ss);
        ss = fmaf(bf_hi(vp[e]), bf_hi(vp[e]), ss);
    }
    return ss;
}

// 8 consecutive weights [c, c+8) of one stage row as fp32 pairs (even, odd):
// the exact values of the stored format.
TI_DEVICE_INLINE float2 magic_pair(uint32_t lo, uint32_t hi, uint32_t sel, float bias) {
    // bytes of lo / hi placed under the exponent of 2^23: float = 2^23 + byte
    const float a = __uint_as_float(__byte_perm(lo, 0x4B000000u, sel));
    const float b = __uint_as_float(__byte_perm(hi, 0x4B000000u, sel));
    return make_float2(a - bias, b - bias);
}
template <int WF>
TI_DEVICE_INLINE void load_w8(const uint8_t* row, int K, int c, float2 w[4]) {
    if constexpr (WF == kWQ4) {
        const uint32_t q = *reinterpret_cast<const uint32_t*>(row + (c >> 1));
        const float d = __half2float(*reinterpret_cast<const __half*>(row + (K >> 1) + ((c >> 5) << 1)));
        const uint32_t lo = q & 0x0F0F0F0Fu, hi = (q >> 4) & 0x0F0F0F0Fu;  // even / odd elements
        const float2 dd = make_float2(d, d);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 v = magic_pair(lo, hi, 0x7440u | (uint32_t)k, 8388616.0f);  // 2^23 + 8
            w[k] = make_float2(v.x * dd.x, v.y * dd.y);
        }
    } else {
        const uint2 q = *reinterpret_cast<const uint2*>(row + c);
        const float d = __half2float(*reinterpret_cast<const __half*>(row + K + ((c >> 5) << 1)));
        // int8 -> biased uint8 (q + 128), element pairs (2k, 2k+1)
        const uint32_t u0 = q.x ^ 0x80808080u, u1 = q.y ^ 0x80808080u;
        const uint32_t ev = __byte_perm(u0, u1, 0x6420), od = __byte_perm(u0, u1, 0x7531);
#pragma unroll
        for (int k = 0; k < 4; ++k) {
            const float2 v = magic_pair(ev, od, 0x7440u | (uint32_t)k, 8388736.0f);  // 2^23 + 128
            w[k] = make_float2(v.x * d, v.y * d);
        }
    }
}
TI_DEVICE_INLINE float2 dot8_f2(const float2 w[4], const float2* x, float2 acc) {
#pragma unroll
    for (int k = 0; k < 4; ++k) acc = ffma2(w[k], x[k], acc);
    return acc;
}
TI_DEVICE_INLINE float dot8_f32w(const float2 w[4], const uint4 x, float acc) {
    acc = fmaf(w[0].x, bf_lo(x.x), acc);
    acc = fmaf(w[0].y, bf_hi(x.x), acc);
    acc = fmaf(w[1].x, bf_lo(x.y), acc);
    acc = fmaf(w[1].y, bf_hi(x.y), acc);
    acc = fmaf(w[2].x, bf_lo(x.z), acc);
    acc = fmaf(w[2].y, bf_hi(x.z), acc);
    acc = fmaf(w[3].x, bf_lo(x.w), acc);
    acc = fmaf(w[3].y, bf_hi(x.w), acc);
    return acc;
}

// x[b, col .. col + 8) from the tensor-parallel inboxes (GemvRecv): rank-ordered
// fp32 sum, rounded to bf16, plus the bf16 residual, rounded (small.cu,
// k_tp_recv_resid); `store`: also into x_out
TI_DEVICE_INLINE uint4 recv_x8(const GemvRecv& r, int b, int K, int col, bool store) {
    float s[8] = {0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f, 0.f};
    for (int rr = 0; rr < r.tp; ++rr) {  // rank order
        const float* p = r.inbox + (size_t)rr * r.src_stride + (size_t)b * K + col;
        const float4 u = __ldcv(reinterpret_cast<const float4*>(p));
        const float4 v = __ldcv(reinterpret_cast<const float4*>(p + 4));
        s[0] += u.x, s[1] += u.y, s[2] += u.z, s[3] += u.w, s[4] += v.x, s[5] += v.y, s[6] += v.z, s[7] += v.w;
    }
    const uint4 rv = *reinterpret_cast<const uint4*>(r.resid + (size_t)b * K + col);
    uint4 o;
    o.x = pack_bf2(bf_lo(rv.x) + round_bf(s[0]), bf_hi(rv.x) + round_bf(s[1]));
    o.y = pack_bf2(bf_lo(rv.y) + round_bf(s[2]), bf_hi(rv.y) + round_bf(s[3]));
    o.z = pack_bf2(bf_lo(rv.z) + round_bf(s[4]), bf_hi(rv.z) + round_bf(s[5]));
    o.w = pack_bf2(bf_lo(rv.w) + round_bf(s[6]), bf_hi(rv.w) + round_bf(s[7]));
    if (store) *reinterpret_cast<uint4*>(r.x_out + (size_t)b * K + col) = o;
    return o;
}

// XR > 0: NB == 1, the lane's XR sub-chunks of the activation slice in registers.
// XR == 0: NB tokens, activation slices in shared memory.
// RG: compile-time bound on rows per stage (per unit).
// WF: weight row format (kWBf16 / kWQ4 / kWQ8).
// ATT > 0: one token whose decode attention (attn_fused.cuh) the consumer warps
//   run first; it writes x (= a.att.out), which the prologue then reads from L2.
//   The instance fixes the head geometry: 1 / 2 head_dim 128 with <= 4 / <= 8
//   q heads per kv head, 3 / 4 head_dim 64 likewise.
template <int NB, int EPI, int XR, int RG, int WF, int ATT = 0>
__global__ void __launch_bounds__(kThreads, 1)
    k_gemv(const GemvArgs a, const int rows_per_stage, const int stages, const int pf) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int U = (EPI == kEpiGlu) ? 2 : 1;
    constexpr bool XS = (XR == 0);
    constexpr int XRR = XS ? 1 : XR;
    const int K = a.K;
    const int rows_cap = (a.N + (int)gridDim.x - 1) / (int)gridDim.x;
    const uint32_t att_bytes =
        ATT ? gemv_attn_smem(a.att.nq / a.att.nkv, a.att.hd, a.att.warps, ((int)gridDim.x + a.att.nkv - 1) / a.att.nkv)
            : 0u;
    const GemvSmem L = gemv_smem_layout(K, WF, U, rows_per_stage, stages, NB, XS, rows_cap, att_bytes);
    const size_t rb = wrow_bytes(K, WF);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full_off);
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.empty_off);
    uint64_t* pfull = reinterpret_cast<uint64_t*>(smem + L.pfull_off);
    uint64_t* pempty = reinterpret_cast<uint64_t*>(smem + L.pempty_off);
    uint64_t* go = reinterpret_cast<uint64_t*>(smem + L.go_off);
    float* part = reinterpret_cast<float*>(smem + L.part_off);
    float* red = reinterpret_cast<float*>(smem + L.red_off);
    const int slot_floats = rows_per_stage * U * NB * kConsumerWarps;

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x, G = gridDim.x;
    const int u0 = (int)((long long)cta * a.N / G), u1 = (int)((long long)(cta + 1) * a.N / G);
    const int n_groups = (u1 - u0 + rows_per_stage - 1) / rows_per_stage;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        for (int p = 0; p < kPartSlots; ++p) {
            mbar_init(&pfull[p], kConsumerWarps);
            mbar_init(&pempty[p], 1);
        }
        mbar_init(go, 1);
        fence_barrier_init();
    }
    __syncthreads();
    // the next kernel may start launching now: its weight stream does not
    // depend on us, and its pdl_wait orders everything else
    if (threadIdx.x == 0) pdl_trigger();

    // ------------------------------------------------------------ producer
    if (warp == kProducerWarp) {
        if (lane == 0 && n_groups > 0) {
            const uint64_t pol = l2_policy_evict_first();
            const uint8_t* W = reinterpret_cast<const uint8_t*>(a.W);
            const size_t row_bytes = rb;
            auto rows_of = [&](int g) { return min(rows_per_stage, u1 - (u0 + g * rows_per_stage)); };
            auto prefetch = [&](int g) {
                const int row0 = u0 + g * rows_per_stage;
                const uint32_t bytes = (uint32_t)(rows_of(g) * row_bytes);
                prefetch_l2_bulk(W + (size_t)row0 * row_bytes, bytes);
                if (U == 2) prefetch_l2_bulk(W + ((size_t)a.N + row0) * row_bytes, bytes);
            };
            if constexpr (ATT > 0) {
                // while the consumers attend, the CTA's rows go HBM -> L2 only; the
                // shared-memory fills (from L2) wait for the consumers' go, so the
                // attention's latency-bound loads do not queue behind them
                for (int g = 0; g < n_groups; ++g) prefetch(g);
                mbar_wait(go, 0, a.err, kErrTimeoutFull);
            }
            for (int g = stages; g < min(n_groups, stages + pf); ++g) prefetch(g);
            for (int g = 0; g < n_groups; ++g) {
                const int s = g % stages, use = g / stages;
                if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, a.err, kErrTimeoutEmpty)) break;
                const int row0 = u0 + g * rows_per_stage;
                const uint32_t bytes = (uint32_t)(rows_of(g) * row_bytes);
                uint8_t* dst = smem + L.stages_off + (size_t)s * L.stage_bytes;
                mbar_arrive_expect_tx(&full[s], bytes * U);
                bulk_g2s(dst, W + (size_t)row0 * row_bytes, bytes, &full[s], pol);
                if (U == 2)
                    bulk_g2s(dst + (size_t)rows_per_stage * row_bytes, W + ((size_t)a.N + row0) * row_bytes, bytes,
                             &full[s], pol);
                if (g + stages + pf < n_groups) prefetch(g + stages + pf);
            }
            if (a.next_w && a.next_bytes > 0) {
                const int G2 = min(G, a.next_N);
                if (cta < G2) {
                    const int r0 = (int)((long long)cta * a.next_N / G2);
                    const int r1 = (int)((long long)(cta + 1) * a.next_N / G2);
                    const size_t nrb = wrow_bytes(a.next_K, a.next_wfmt);
                    const int rows = min(r1 - r0, max(1, (int)(a.next_bytes / (nrb * a.next_U))));
                    const uint8_t* NW = reinterpret_cast<const uint8_t*>(a.next_w);
                    prefetch_l2_bulk(NW + (size_t)r0 * nrb, (uint32_t)(rows * nrb));
                    if (a.next_U == 2) prefetch_l2_bulk(NW + ((size_t)a.next_N + r0) * nrb, (uint32_t)(rows * nrb));
                    // the budget left over: the first rows of the GEMV after the next one
                    const long long left = (long long)a.next_bytes - (long long)rows * nrb * a.next_U;
                    const int G3 = min(G, a.next2_N);
                    if (a.next2_w && left > 0 && cta < G3) {
                        const int s0 = (int)((long long)cta * a.next2_N / G3);
                        const int s1 = (int)((long long)(cta + 1) * a.next2_N / G3);
                        const size_t nrb2 = wrow_bytes(a.next2_K, a.next2_wfmt);
                        const int rows2 = min(s1 - s0, (int)(left / (long long)(nrb2 * a.next2_U)));
                        if (rows2 > 0) {
                            const uint8_t* NW2 = reinterpret_cast<const uint8_t*>(a.next2_w);
                            prefetch_l2_bulk(NW2 + (size_t)s0 * nrb2, (uint32_t)(rows2 * nrb2));
                            if (a.next2_U == 2)
                                prefetch_l2_bulk(NW2 + ((size_t)a.next2_N + s0) * nrb2, (uint32_t)(rows2 * nrb2));
                        }
                    }
                }
            }
        }
        return;
    }

    // ------------------------------------------------------------ epilogue warp
    if (warp == kEpilogueWarp) {
        pdl_wait();  // the residual is the previous kernel's output
        // residual and bias values of this CTA's rows, staged once (independent loads)
        uint16_t* e_res = reinterpret_cast<uint16_t*>(smem + L.epi_off);  // [NB][rows_cap]
        uint16_t* e_bias = e_res + NB * rows_cap;                          // [rows_cap]
        for (int i = lane; i < u1 - u0; i += 32) {
            if (EPI == kEpiResid)
#pragma unroll
                for (int b = 0; b < NB; ++b)
                    if (b < a.nb) e_res[b * rows_cap + i] = a.resid[(size_t)b * a.resid_stride + u0 + i];
            if (EPI == kEpiStore && a.bias) e_bias[i] = a.bias[u0 + i];
        }
        __syncwarp();
        unsigned long long best[NB];
#pragma unroll
        for (int b = 0; b < NB; ++b) best[b] = 0ull;
        for (int g = 0; g < n_groups; ++g) {
            const int slot = g % kPartSlots, use = g / kPartSlots;
            const int row0 = u0 + g * rows_per_stage;
            const int nr = min(rows_per_stage, u1 - row0);
            if (!mbar_wait(&pfull[slot], use & 1, a.err, kErrTimeoutFull)) break;
            const float* pbuf = part + (size_t)slot * slot_floats;
            const int r = lane / NB, b = lane % NB;
            if (lane < rows_per_stage * NB && r < nr && b < a.nb) {
                const int n = row0 + r;
                const int ad = a.lora.adapter ? a.lora.adapter[b] : -1;
                float accu[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    const float* pv = pbuf + ((r * U + u) * NB + b) * kConsumerWarps;
                    float sum = 0.f;
#pragma unroll
                    for (int w = 0; w < kConsumerWarps; ++w) sum += pv[w];
                    accu[u] = sum;
                }
                if (EPI == kEpiStore && a.ps.tp) {
                    // tensor-parallel all-reduce: the fp32 sum into every rank's inbox (NVLink stores)
                    for (int r = 0; r < a.ps.tp; ++r) a.ps.inbox[r][(size_t)b * a.out_stride + n] = accu[0];
                } else if (EPI == kEpiStore && a.partial) {
                    a.partial[(size_t)b * a.out_stride + n] = accu[0];
                } else if (EPI == kEpiStore) {
                    float v = round_bf(accu[0]);
                    if (a.bias) v = round_bf(v + __uint_as_float((uint32_t)e_bias[n - u0] << 16));
                    if (ad >= 0) {
                        // sections of the fused q|k|v rows: t offset = section * rank
                        const int sec = (n >= a.lora.sec1) + (n >= a.lora.sec2);
                        v = lora_delta(a.lora, ad, b, n, sec * a.lora.rank, v);
                    }
                    reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + n] = f2bf(v);
                } else if (EPI == kEpiResid) {
                    float v = round_bf(accu[0]);
                    if (ad >= 0) v = lora_delta(a.lora, ad, b, n, 0, v);
                    const float rr = __uint_as_float((uint32_t)e_res[b * rows_cap + (n - u0)] << 16);
                    reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + n] = f2bf(rr + v);
                } else if (EPI == kEpiGlu) {
                    float gv = round_bf(accu[0]);
                    float uv = round_bf(accu[U - 1]);
                    if (ad >= 0) {
                        gv = lora_delta(a.lora, ad, b, n, 0, gv);
                        uv = lora_delta(a.lora, ad, b, a.N + n, a.lora.rank, uv);
                    }
                    const float hv = glu_act(gv, a.act);
                    reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + n] = f2bf(hv * uv);
                } else {  // kEpiLmHead
                    const float v = accu[0];
                    reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + n] = f2bf(v);
                    if (a.logits_f32) a.logits_f32[(size_t)b * a.out_stride + n] = v;
                    const unsigned long long key = argmax_key(v, (uint32_t)(n + a.key_offset));
#pragma unroll
                    for (int bb = 0; bb < NB; ++bb)
                        if (bb == b && key > best[bb]) best[bb] = key;
                }
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&pempty[slot]);
        }
        if (EPI == kEpiLmHead) {
            // CTA argmax over the warp, then grid argmax through one 64-bit
            // atomicMax per token; the last CTA publishes the ids and re-arms
            // the keys for the next step.
#pragma unroll
            for (int b = 0; b < NB; ++b)
#pragma unroll
                for (int o = 16; o > 0; o >>= 1) {
                    const unsigned long long other = __shfl_xor_sync(0xffffffffu, best[b], o);
                    best[b] = other > best[b] ? other : best[b];
                }
            if (lane == 0) {
                for (int b = 0; b < a.nb && b < NB; ++b)
                    if (best[b]) atomicMax(&a.amax[b], best[b]);
                __threadfence();
                const unsigned int ticket = atomicAdd(a.done, 1u);
                if (ticket == gridDim.x - 1 && !a.publish) {
                    atomicExch(a.done, 0u);  // keys stay for the cross-rank reduction
                } else if (ticket == gridDim.x - 1) {
                    __threadfence();
                    for (int b = 0; b < a.nb && b < NB; ++b) {
                        const unsigned long long key = atomicExch(&a.amax[b], 0ull);
                        const int32_t id = (int32_t)(~(uint32_t)(key & 0xffffffffull));
                        a.out_ids[b] = id;
                        if (a.chain_tokens) a.chain_tokens[b] = id;
                        if (a.chain_pos) a.chain_pos[b] += 1;
                    }
                    atomicExch(a.done, 0u);
                }
            }
        }
        if (EPI == kEpiStore && a.ps.tp) {
            // this CTA's peer stores are visible system-wide before it counts itself;
            // the last CTA publishes the phase to every rank
            __threadfence_system();
            __syncwarp();
            if (lane == 0) {
                const unsigned int t = atomicAdd(a.ps.ticket, 1u);
                if (t == gridDim.x - 1) {
                    __threadfence_system();
                    if (a.ps.signal) {
                        const unsigned int seq = peer_seq(*a.ps.epoch, a.ps.seq_mul, a.ps.seq_add);
                        for (int r = 0; r < a.ps.tp; ++r) st_release_sys(a.ps.flag[r], seq);
                    }
                    atomicExch(a.ps.ticket, 0u);
                }
            }
        }
        return;
    }

    // ------------------------------------------------------------ consumers: prologue
    if constexpr (ATT > 0) attn_fused_prefetch(a.att, warp, lane, cta, G);
    pdl_wait();  // x (or, with ATT, the token's q|k|v) is produced by the previous kernel
    if constexpr (ATT > 0) {
        constexpr int AHD = ATT <= 2 ? 128 : 64, AGM = ATT % 2 == 1 ? 4 : 8;
        attn_fused_phase<AHD, AGM>(a.att, reinterpret_cast<float*>(smem + L.att_off), threadIdx.x,
                                   kConsumerWarps * 32, cta, G, go, a.err);
    }
    const bool recv = a.recv.tp > 0;
    if (recv) {
        // every rank's partial sums of the row-parallel projection have landed (bounded wait)
        if (threadIdx.x == 0) {
            const unsigned int seq = peer_seq(*a.recv.epoch, a.recv.seq_mul, a.recv.seq_add);
            for (int r = 0; r < a.recv.tp; ++r)
                if (!wait_seq_sys(a.recv.flags + r, seq, a.err, kErrTimeoutPeer)) break;
        }
        named_bar(1, kConsumerWarps * 32);
    }
    const int cols_per_warp = K / kConsumerWarps;
    const int col0 = warp * cols_per_warp;
    const int n_sc = cols_per_warp / 8;  // 16-byte sub-chunks per warp row slice
    uint4 xr[XRR];
    uint8_t* xs = smem + L.xs_off;
    {
        const bool norm = a.norm_w != nullptr;
        const float off = a.norm_offset ? 1.0f : 0.0f;
        if constexpr (!XS) {
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < XRR; ++j) {
                const int sc = j * 32 + lane;
                // with ATT, x was written by other CTAs of this grid: read it from L2
                xr[j] = sc >= n_sc  ? make_uint4(0, 0, 0, 0)
                        : recv      ? recv_x8(a.recv, 0, K, col0 + sc * 8, cta == 0)
                        : ATT > 0   ? __ldcg(reinterpret_cast<const uint4*>(a.x + col0 + sc * 8))
                                    : *reinterpret_cast<const uint4*>(a.x + col0 + sc * 8);
                if (norm) ss = sumsq8(xr[j], ss);
            }
            if (norm) {
                ss = warp_sum(ss);
                if (lane == 0) red[warp] = ss;
                named_bar(1, kConsumerWarps * 32);
                float tot = 0.f;
#pragma unroll
                for (int w = 0; w < kConsumerWarps; ++w) tot += red[w];
                const float scale = rsqrtf(tot / (float)K + a.eps);  // ops.cu:179
#pragma unroll
                for (int j = 0; j < XRR; ++j) {
                    const int sc = j * 32 + lane;
                    if (sc < n_sc)
                        normalise8(xr[j], *reinterpret_cast<const uint4*>(a.norm_w + col0 + sc * 8), scale, off);
                }
            }
        } else {
            float ss[NB];
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                ss[b] = 0.f;
                for (int sc = lane; sc < n_sc; sc += 32) {
                    const int c = col0 + sc * 8;
                    uint4 v = make_uint4(0, 0, 0, 0);
                    if (b < a.nb)
                        v = recv ? recv_x8(a.recv, b, K, c, cta == 0)
                                 : *reinterpret_cast<const uint4*>(a.x + (size_t)b * a.x_stride + c);
                    if (norm) ss[b] = sumsq8(v, ss[b]);
                    *reinterpret_cast<uint4*>(xs + ((size_t)b * K + c) * 2) = v;
                }
            }
            if (norm) {
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    const float t = warp_sum(ss[b]);
                    if (lane == 0) red[warp * NB + b] = t;
                }
                named_bar(1, kConsumerWarps * 32);
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    float tot = 0.f;
#pragma unroll
                    for (int w = 0; w < kConsumerWarps; ++w) tot += red[w * NB + b];
                    const float scale = rsqrtf(tot / (float)K + a.eps);  // ops.cu:179
                    for (int sc = lane; sc < n_sc; sc += 32) {
                        const int c = col0 + sc * 8;
                        uint4* p = reinterpret_cast<uint4*>(xs + ((size_t)b * K + c) * 2);
                        uint4 v = *p;
                        normalise8(v, *reinterpret_cast<const uint4*>(a.norm_w + c), scale, off);
                        *p = v;
                    }
                }
            }
            __syncwarp();
        }
    }

    // the (normalised, bf16-exact) activation slice unpacked to fp32 pairs once
    constexpr bool XF = !XS && XR <= 4;  // fp32 pairs for small slices, packed bf16 otherwise
    float2 xf[XF ? XRR : 1][4];
#pragma unroll
    for (int j = 0; j < (XF ? XRR : 0); ++j) {
        xf[j][0] = bf2_to_f2(xr[j].x);
        xf[j][1] = bf2_to_f2(xr[j].y);
        xf[j][2] = bf2_to_f2(xr[j].z);
        xf[j][3] = bf2_to_f2(xr[j].w);
    }

    // ------------------------------------------------------------ consumers: main loop
    for (int g = 0; g < n_groups; ++g) {
        const int s = g % stages, use = g / stages;
        const int row0 = u0 + g * rows_per_stage;
        const int nr = min(rows_per_stage, u1 - row0);
        if (!mbar_wait(&full[s], use & 1, a.err, kErrTimeoutFull)) break;
        const uint8_t* stage = smem + L.stages_off + (size_t)s * L.stage_bytes;

        float acc[RG][U][NB];
#pragma unroll
        for (int r = 0; r < RG; ++r)
#pragma unroll
            for (int u = 0; u < U; ++u)
#pragma unroll
                for (int b = 0; b < NB; ++b) acc[r][u][b] = 0.f;
        if constexpr (!XS) {
            // packed FFMA2: even / odd elements in the two halves, summed at the end
            float2 acc2[RG][U];
#pragma unroll
            for (int r = 0; r < RG; ++r)
#pragma unroll
                for (int u = 0; u < U; ++u) acc2[r][u] = make_float2(0.f, 0.f);
#pragma unroll
            for (int j = 0; j < XRR; ++j) {
                const int sc = j * 32 + lane;
                if (sc < n_sc) {
#pragma unroll
                    for (int r = 0; r < RG; ++r)
                        if (r < nr)
#pragma unroll
                            for (int u = 0; u < U; ++u) {
                                const uint8_t* wrow = stage + ((size_t)u * rows_per_stage + r) * rb;
                                if constexpr (WF == kWBf16) {
                                    const uint4 w = lds128(wrow + (size_t)(col0 + sc * 8) * 2);
                                    if constexpr (XF) {
                                        acc2[r][u] = dot8_bf16_f2(w, xf[j], acc2[r][u]);
                                    } else {
                                        acc2[r][u].x = dot8_bf16(w, xr[j], acc2[r][u].x);
                                    }
                                } else {
                                    float2 wv[4];
                                    load_w8<WF>(wrow, K, col0 + sc * 8, wv);
                                    if constexpr (XF) {
                                        acc2[r][u] = dot8_f2(wv, xf[j], acc2[r][u]);
                                    } else {
                                        acc2[r][u].x = dot8_f32w(wv, xr[j], acc2[r][u].x);
                                    }
                                }
                            }
                }
            }
#pragma unroll
            for (int r = 0; r < RG; ++r)
#pragma unroll
                for (int u = 0; u < U; ++u) acc[r][u][0] = acc2[r][u].x + acc2[r][u].y;
        } else {
            for (int sc = lane; sc < n_sc; sc += 32) {
                const int c = col0 + sc * 8;
                uint4 xv[NB];
#pragma unroll
                for (int b = 0; b < NB; ++b) xv[b] = lds128(xs + ((size_t)b * K + c) * 2);
#pragma unroll
                for (int r = 0; r < RG; ++r)
                    if (r < nr)
#pragma unroll
                        for (int u = 0; u < U; ++u) {
                            const uint8_t* wrow = stage + ((size_t)u * rows_per_stage + r) * rb;
                            if constexpr (WF == kWBf16) {
                                // unpacked once, shared by the tokens
                                const uint4 w = lds128(wrow + (size_t)c * 2);
                                const float2 wv[4] = {bf2_to_f2(w.x), bf2_to_f2(w.y), bf2_to_f2(w.z), bf2_to_f2(w.w)};
#pragma unroll
                                for (int b = 0; b < NB; ++b) acc[r][u][b] = dot8_f32w(wv, xv[b], acc[r][u][b]);
                            } else {
                                float2 wv[4];
                                load_w8<WF>(wrow, K, c, wv);
#pragma unroll
                                for (int b = 0; b < NB; ++b) acc[r][u][b] = dot8_f32w(wv, xv[b], acc[r][u][b]);
                            }
                        }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);  // stage fully read: the producer may refill it
        // batched butterfly: every (row, unit, token) partial reduced across the warp
#pragma unroll
        for (int o = 16; o > 0; o >>= 1)
#pragma unroll
            for (int r = 0; r < RG; ++r)
#pragma unroll
                for (int u = 0; u < U; ++u)
#pragma unroll
                    for (int b = 0; b < NB; ++b) acc[r][u][b] += __shfl_xor_sync(0xffffffffu, acc[r][u][b], o);
        const int slot = g % kPartSlots, puse = g / kPartSlots;
        if (lane == 0) {
            if (puse > 0) mbar_wait(&pempty[slot], (puse - 1) & 1, a.err, kErrTimeoutEmpty);
            float* pbuf = part + (size_t)slot * slot_floats;
#pragma unroll
            for (int r = 0; r < RG; ++r)
                if (r < nr)
#pragma unroll
                    for (int u = 0; u < U; ++u)
#pragma unroll
                        for (int b = 0; b < NB; ++b) pbuf[((r * U + u) * NB + b) * kConsumerWarps + warp] = acc[r][u][b];
            mbar_arrive(&pfull[slot]);
        }
    }
}

// ------------------------------------------------------------------ host side
template <int NB, int EPI, int XR, int RG, int WF, int ATT = 0>
static const void* fn() {
    return reinterpret_cast<const void*>(&k_gemv<NB, EPI, XR, RG, WF, ATT>);
}

// fused attention + o projection: one token, the o projection's epilogues
// (residual, or the tensor-parallel store), activation slice in registers;
// geo = the ATT head-geometry index
template <int EPI, int WF, int XR>
static const void* pick_att_geo(int geo) {
    switch (geo) {
        case 1: return fn<1, EPI, XR, kRowsMax, WF, 1>();
        case 2: return fn<1, EPI, XR, kRowsMax, WF, 2>();
        case 3: return fn<1, EPI, XR, kRowsMax, WF, 3>();
        case 4: return fn<1, EPI, XR, kRowsMax, WF, 4>();
        default: return nullptr;
    }
}
template <int EPI, int WF>
static const void* pick_att(int xr, int geo) {
    switch (xr) {
        case 1: return pick_att_geo<EPI, WF, 1>(geo);
        case 2: return pick_att_geo<EPI, WF, 2>(geo);
        default: return nullptr;
    }
}

template <int EPI, int WF>
static const void* pick(int nb, int xr) {
    constexpr int U = EPI == kEpiGlu ? 2 : 1;
    if (nb == 1) {
        switch (xr) {
            case 1: return fn<1, EPI, 1, kRowsMax / U, WF>();
            case 2: return fn<1, EPI, 2, kRowsMax / U, WF>();
            case 4: return fn<1, EPI, 4, (4 / U > 0 ? 4 / U : 1), WF>();
            case 8: return fn<1, EPI, 8, (2 / U > 0 ? 2 / U : 1), WF>();
            default: return fn<1, EPI, 0, kRowsMax / U, WF>();
        }
    }
    if (nb == 2) return fn<2, EPI, 0, 8 / U, WF>();
    if (nb <= 4) return fn<4, EPI, 0, 4 / U, WF>();
    if (nb <= 8) return fn<8, EPI, 0, (2 / U > 0 ? 2 / U : 1), WF>();
    return nullptr;
}

static int nb_tmpl(int nb) { return nb == 1 ? 1 : nb == 2 ? 2 : nb <= 4 ? 4 : 8; }
static int rg_tmpl(int nbt, int U, int xr) {
    if (nbt == 1) {
        if (xr == 4) return std::max(1, 4 / U);
        if (xr == 8) return std::max(1, 2 / U);
        return kRowsMax / U;
    }
    if (nbt == 2) return std::max(1, 8 / U);
    if (nbt == 4) return std::max(1, 4 / U);
    return std::max(1, 2 / U);
}

// Geometry knobs (KB): stage size, shared-memory ring, L2 prefetch window per CTA.
// Defaults come from sweeps on B200; the environment may override them.
static int tune_kb(const char* name, int dflt) {
    const char* v = std::getenv(name);
    return v && std::atoi(v) >= 0 ? std::atoi(v) : dflt;
}

bool gemv_plan(const GemvArgs& a, int epi, int device, GemvPlan* plan, std::string* why) {
    if (a.K <= 0 || a.K % (8 * kConsumerWarps) != 0) {
        if (why) *why = "gemv: K must be a positive multiple of 128";
        return false;
    }
    if (a.N <= 0 || a.nb < 1 || a.nb > 8) {
        if (why) *why = "gemv: need N > 0 and 1 <= tokens <= 8";
        return false;
    }
    const int U = epi == kEpiGlu ? 2 : 1;
    const int nbt = nb_tmpl(a.nb);
    if (a.wfmt != kWBf16 && (a.K % 256 != 0 || epi == kEpiLmHead)) {
        if (why) *why = "gemv: quantised weights need K % 256 == 0 (and not the LM head)";
        return false;
    }
    const size_t row_bytes = wrow_bytes(a.K, a.wfmt) * U;
    // register slice: sub-chunks per lane = ceil(K / 128 / 32)
    const int need = (a.K / (8 * kConsumerWarps) + 31) / 32;
    int xr = 0;
    if (nbt == 1) {
        for (int c : {1, 2, 4, 8})
            if (need <= c) {
                xr = c;
                break;
            }
    }
    int rps = (int)std::max<size_t>(1, (size_t)tune_kb("TI_GEMV_STAGE_KB", 96) * 1024 / row_bytes);
    rps = std::min(rps, rg_tmpl(nbt, U, xr));
    const bool xs = xr == 0;
    const size_t stage_bytes = ((size_t)rps * row_bytes + 127) & ~size_t(127);
    int stages = (int)std::min<size_t>(8, std::max<size_t>(2, (size_t)tune_kb("TI_GEMV_RING_KB", 200) * 1024 / stage_bytes));
    const int grid = std::min(num_sms(device), a.N);
    const int rows_cap = (a.N + grid - 1) / grid;
    // fused attention: one token, the o projection's epilogues, a supported head geometry;
    // merge slots for as many page-scoring warps as ~20 KB of shared memory holds
    const bool att = a.att.nq > 0;
    int att_warps = 0, att_geo = 0;
    uint32_t att_bytes = 0;
    if (att) {
        const int G = a.att.nkv > 0 && a.att.nq % a.att.nkv == 0 ? a.att.nq / a.att.nkv : 0;
        if (a.nb != 1 || (epi != kEpiResid && epi != kEpiStore) || (xr != 1 && xr != 2) || G < 1 ||
            G > kAttnFusedMaxGroup || (a.att.hd != 64 && a.att.hd != 128) || grid < a.att.nkv ||
            a.K != a.att.nq * a.att.hd || !a.att.out || !a.att.part || !a.att.ticket || !a.att.sync) {
            if (why) *why = "gemv: fused attention needs one token, head_dim 64/128, <= 8 q heads per kv head";
            return false;
        }
        att_geo = (a.att.hd == 128 ? 1 : 3) + (G > 4 ? 1 : 0);
        const int fl = 20 * 1024 / 4 - (G + 2) * a.att.hd;
        att_warps = std::max(1, std::min(kConsumerWarps, fl / (G * (a.att.hd + 2))));
        // TI_ATT_WARPS caps them (a test makes warps take several pages at short contexts)
        if (const char* v = std::getenv("TI_ATT_WARPS"))
            if (std::atoi(v) >= 1) att_warps = std::min(att_warps, std::atoi(v));
        att_bytes = gemv_attn_smem(G, a.att.hd, att_warps, (grid + a.att.nkv - 1) / a.att.nkv);
    }
    int max_smem = 0;
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    GemvSmem L;
    for (;;) {
        L = gemv_smem_layout(a.K, a.wfmt, U, rps, stages, nbt, xs, rows_cap, att_bytes);
        if ((int)L.total <= max_smem) break;
        if (stages > 2) --stages;
        else if (rps > 1) --rps;
        else {
            if (why) *why = "gemv: row does not fit in shared memory";
            return false;
        }
    }
    const void* f = nullptr;
    if (att) {
        switch (a.wfmt * 4 + epi) {
            case kEpiStore: f = pick_att<kEpiStore, kWBf16>(xr, att_geo); break;
            case kEpiResid: f = pick_att<kEpiResid, kWBf16>(xr, att_geo); break;
            case 4 * kWQ4 + kEpiStore: f = pick_att<kEpiStore, kWQ4>(xr, att_geo); break;
            case 4 * kWQ4 + kEpiResid: f = pick_att<kEpiResid, kWQ4>(xr, att_geo); break;
            case 4 * kWQ8 + kEpiStore: f = pick_att<kEpiStore, kWQ8>(xr, att_geo); break;
            case 4 * kWQ8 + kEpiResid: f = pick_att<kEpiResid, kWQ8>(xr, att_geo); break;
            default: break;
        }
    } else switch (a.wfmt * 4 + epi) {
        case kEpiStore: f = pick<kEpiStore, kWBf16>(a.nb, xr); break;
        case kEpiResid: f = pick<kEpiResid, kWBf16>(a.nb, xr); break;
        case kEpiGlu: f = pick<kEpiGlu, kWBf16>(a.nb, xr); break;
        case kEpiLmHead: f = pick<kEpiLmHead, kWBf16>(a.nb, xr); break;
        case 4 * kWQ4 + kEpiStore: f = pick<kEpiStore, kWQ4>(a.nb, xr); break;
        case 4 * kWQ4 + kEpiResid: f = pick<kEpiResid, kWQ4>(a.nb, xr); break;
        case 4 * kWQ4 + kEpiGlu: f = pick<kEpiGlu, kWQ4>(a.nb, xr); break;
        case 4 * kWQ8 + kEpiStore: f = pick<kEpiStore, kWQ8>(a.nb, xr); break;
        case 4 * kWQ8 + kEpiResid: f = pick<kEpiResid, kWQ8>(a.nb, xr); break;
        case 4 * kWQ8 + kEpiGlu: f = pick<kEpiGlu, kWQ8>(a.nb, xr); break;
        default: break;
    }
    if (!f) {
        if (why) *why = "gemv: no kernel instance";
        return false;
    }
    cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)L.total);
    if (e != cudaSuccess) {
        if (why) *why = std::string("gemv: cudaFuncSetAttribute: ") + cudaGetErrorString(e);
        return false;
    }
    plan->rows_per_stage = rps;
    plan->stages = stages;
    plan->att_warps = att_warps;
    plan->grid = grid;
    plan->smem = L.total;
    plan->func = f;
    // L2 prefetch window: ~256 KB per CTA beyond the ring
    plan->prefetch = (int)((size_t)tune_kb("TI_GEMV_PF_KB", 0) * 1024 / stage_bytes);
    return true;
}

cudaError_t gemv_launch(const GemvArgs& a, int epi, const GemvPlan& plan, cudaStream_t s, bool pdl) {
    (void)epi;
    GemvArgs args = a;
    args.att.warps = plan.att_warps;
    int rps = plan.rows_per_stage, st = plan.stages, pf = plan.prefetch;
    void* params[] = {&args, &rps, &st, &pf};
    return launch_pdl(plan.func, dim3(plan.grid), dim3(kThreads), plan.smem, s, params, pdl);
}

}  // namespace ti
