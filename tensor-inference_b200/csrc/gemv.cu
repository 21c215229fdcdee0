// gemv.cu — weight-streaming GEMV for decode (few tokens, bf16 weights).
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
//
// Structure (one CTA per SM, 9 warps):
//   warp 8 (producer): streams the CTA's contiguous row range of W from HBM
//     into a ring of shared-memory stages with cp.async.bulk (TMA, 1-D,
//     evict-first L2 policy), completion tracked by mbarriers.  It starts
//     before griddepcontrol.wait: weights never depend on the previous kernel,
//     so under programmatic dependent launch the stream starts while the
//     previous kernel drains.
//   warps 0-7 (consumers): warp w owns columns [w*K/8, (w+1)*K/8) of every
//     row; its slice of the (normalised) activation stays in registers.
//     Per stage: fp32 FMAs in element order, butterfly lane reduction, and a
//     fixed-order sum over the 8 warps — results are deterministic.
#include "common.cuh"
#include "kernels.h"

#include <algorithm>
#include <cstdio>

namespace ti {

constexpr int kConsumerWarps = 8;
constexpr int kThreads = (kConsumerWarps + 1) * 32;

struct GemvSmem {
    // offsets in bytes from the dynamic smem base
    uint32_t stage_bytes, stages_off, full_off, empty_off, part_off, red_off, xs_off, amax_off, total;
};

__host__ __device__ inline GemvSmem gemv_smem_layout(int K, int units, int rows_per_stage, int stages, int nb,
                                                     bool x_in_smem) {
    GemvSmem L;
    uint32_t sb = (uint32_t)rows_per_stage * units * K * 2;
    sb = (sb + 127u) & ~127u;
    L.stage_bytes = sb;
    L.stages_off = 0;
    uint32_t o = sb * stages;
    L.full_off = o;
    o += 8 * stages;
    L.empty_off = o;
    o += 8 * stages;
    L.part_off = o;
    o += 2 * rows_per_stage * units * nb * kConsumerWarps * 4;
    L.red_off = o;
    o += kConsumerWarps * nb * 4;
    o = (o + 15u) & ~15u;
    L.xs_off = o;
    if (x_in_smem) o += (uint32_t)nb * K * 2;
    o = (o + 15u) & ~15u;
    L.amax_off = o;
    o += 8 * nb;
    L.total = o;
    return L;
}

template <int EPI>
TI_DEVICE_INLINE float glu_act(float g, int act) {
    if (act == 0) return round_bf(g / (1.0f + expf(-g)));  // ops.cu:326
    const float c1 = 0.7978845608f, c2 = 0.044715f;        // ops.cu:712-714
    return round_bf(0.5f * g * (1.0f + tanhf(c1 * (g + c2 * g * g * g))));
}

// LoRA expansion of one output element (qwen_adapter_model.cpp:27-29 + :42)
TI_DEVICE_INLINE float lora_delta(const GemvLora& L, int b, int row, int t_off, float base) {
    const uint16_t* B = L.B[b];
    if (B == nullptr) return base;
    const uint16_t* br = B + (size_t)row * L.rank;
    const float* t = L.t + (size_t)b * L.t_stride + t_off;
    float s = 0.f;
    for (int i = 0; i < L.rank; ++i) s = fmaf(__uint_as_float((uint32_t)br[i] << 16), t[i], s);
    float up = round_bf(s);
    float delta = round_bf(up * L.scale[b]);
    return round_bf(base + delta);
}

// XR > 0: one token, the warp's activation slice held in XR uint4 registers per lane.
// XR == 0: NB tokens, activation slices in shared memory.
template <int NB, int EPI, int XR>
__global__ void __launch_bounds__(kThreads, 1) k_gemv(const GemvArgs a, const int rows_per_stage, const int stages) {
    extern __shared__ __align__(128) uint8_t smem[];
    constexpr int U = (EPI == kEpiGlu) ? 2 : 1;
    constexpr bool XS = (XR == 0);
    const int K = a.K;
    const GemvSmem L = gemv_smem_layout(K, U, rows_per_stage, stages, NB, XS);
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full_off);
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.empty_off);
    float* part = reinterpret_cast<float*>(smem + L.part_off);
    float* red = reinterpret_cast<float*>(smem + L.red_off);
    unsigned long long* amax_s = reinterpret_cast<unsigned long long*>(smem + L.amax_off);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int cta = blockIdx.x, G = gridDim.x;
    const int u0 = (int)((long long)cta * a.N / G), u1 = (int)((long long)(cta + 1) * a.N / G);
    const int n_groups = (u1 - u0 + rows_per_stage - 1) / rows_per_stage;

    if (threadIdx.x == 0) {
        for (int s = 0; s < stages; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&empty[s], kConsumerWarps);
        }
        for (int b = 0; b < NB; ++b) amax_s[b] = 0ull;
        fence_barrier_init();
    }
    __syncthreads();

    // ------------------------------------------------------------ producer
    if (warp == kConsumerWarps) {
        if (lane == 0 && n_groups > 0) {
            const uint64_t pol = l2_policy_evict_first();
            const uint8_t* W = reinterpret_cast<const uint8_t*>(a.W);
            const size_t row_bytes = (size_t)K * 2;
            for (int g = 0; g < n_groups; ++g) {
                const int s = g % stages, use = g / stages;
                if (use > 0 && !mbar_wait(&empty[s], (use - 1) & 1, a.err, kErrTimeoutEmpty)) break;
                const int row0 = u0 + g * rows_per_stage;
                const int nr = min(rows_per_stage, u1 - row0);
                const uint32_t bytes = (uint32_t)(nr * row_bytes);
                uint8_t* dst = smem + L.stages_off + (size_t)s * L.stage_bytes;
                mbar_arrive_expect_tx(&full[s], bytes * U);
                bulk_g2s(dst, W + (size_t)row0 * row_bytes, bytes, &full[s], pol);
                if (U == 2)
                    bulk_g2s(dst + (size_t)rows_per_stage * row_bytes, W + ((size_t)a.N + row0) * row_bytes, bytes,
                             &full[s], pol);
            }
        }
        return;
    }

    // ------------------------------------------------------------ consumers: prologue
    pdl_wait();  // x / resid are produced by the previous kernel
    const int cols_per_warp = K / kConsumerWarps;
    const int col0 = warp * cols_per_warp;
    const int n_sc = cols_per_warp / 8;  // 16-byte sub-chunks per warp row slice
    constexpr int XRR = XS ? 1 : XR;
    uint4 xr[XRR];
    uint8_t* xs = smem + L.xs_off;

    {
        const bool norm = a.norm_w != nullptr;
        const float off = a.norm_offset ? 1.0f : 0.0f;
        if constexpr (!XS) {
            // one token; the lane's XR sub-chunks of the slice live in registers
            float ss = 0.f;
#pragma unroll
            for (int j = 0; j < XRR; ++j) {
                const int sc = j * 32 + lane;
                if (sc < n_sc) {
                    xr[j] = *reinterpret_cast<const uint4*>(a.x + col0 + sc * 8);
                    if (norm) {
                        const uint32_t* vp = reinterpret_cast<const uint32_t*>(&xr[j]);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            ss = fmaf(bf_lo(vp[e]), bf_lo(vp[e]), ss);
                            ss = fmaf(bf_hi(vp[e]), bf_hi(vp[e]), ss);
                        }
                    }
                } else {
                    xr[j] = make_uint4(0, 0, 0, 0);
                }
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
                    if (sc < n_sc) {
                        const uint4 wn = *reinterpret_cast<const uint4*>(a.norm_w + col0 + sc * 8);
                        uint32_t* vp = reinterpret_cast<uint32_t*>(&xr[j]);
                        const uint32_t* wp = reinterpret_cast<const uint32_t*>(&wn);
#pragma unroll
                        for (int e = 0; e < 4; ++e) {
                            const float lo = bf_lo(vp[e]) * scale * (bf_lo(wp[e]) + off);
                            const float hi = bf_hi(vp[e]) * scale * (bf_hi(wp[e]) + off);
                            vp[e] = pack_bf2(lo, hi);
                        }
                    }
                }
            }
        } else {
            // NB tokens; the warp's column slice of every token in shared memory
            float ss[NB];
#pragma unroll
            for (int b = 0; b < NB; ++b) {
                ss[b] = 0.f;
                if (b < a.nb) {
                    const uint16_t* xrow = a.x + (size_t)b * a.x_stride;
                    for (int sc = lane; sc < n_sc; sc += 32) {
                        const int c = col0 + sc * 8;
                        const uint4 v = *reinterpret_cast<const uint4*>(xrow + c);
                        if (norm) {
                            const uint32_t* vp = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                ss[b] = fmaf(bf_lo(vp[e]), bf_lo(vp[e]), ss[b]);
                                ss[b] = fmaf(bf_hi(vp[e]), bf_hi(vp[e]), ss[b]);
                            }
                        }
                        *reinterpret_cast<uint4*>(xs + ((size_t)b * K + c) * 2) = v;
                    }
                } else {
                    for (int sc = lane; sc < n_sc; sc += 32)
                        *reinterpret_cast<uint4*>(xs + ((size_t)b * K + col0 + sc * 8) * 2) = make_uint4(0, 0, 0, 0);
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
                    if (b < a.nb) {
                        float tot = 0.f;
#pragma unroll
                        for (int w = 0; w < kConsumerWarps; ++w) tot += red[w * NB + b];
                        const float scale = rsqrtf(tot / (float)K + a.eps);  // ops.cu:179
                        for (int sc = lane; sc < n_sc; sc += 32) {
                            const int c = col0 + sc * 8;
                            uint4 v = *reinterpret_cast<const uint4*>(xs + ((size_t)b * K + c) * 2);
                            const uint4 wn = *reinterpret_cast<const uint4*>(a.norm_w + c);
                            uint32_t* vp = reinterpret_cast<uint32_t*>(&v);
                            const uint32_t* wp = reinterpret_cast<const uint32_t*>(&wn);
#pragma unroll
                            for (int e = 0; e < 4; ++e) {
                                const float lo = bf_lo(vp[e]) * scale * (bf_lo(wp[e]) + off);
                                const float hi = bf_hi(vp[e]) * scale * (bf_hi(wp[e]) + off);
                                vp[e] = pack_bf2(lo, hi);
                            }
                            *reinterpret_cast<uint4*>(xs + ((size_t)b * K + c) * 2) = v;
                        }
                    }
                }
            }
            __syncwarp();
        }
    }
    if (threadIdx.x == 0) pdl_trigger();

    // ------------------------------------------------------------ consumers: main loop
    unsigned long long best[NB];
#pragma unroll
    for (int b = 0; b < NB; ++b) best[b] = 0ull;
    const int n_vals = rows_per_stage * NB;  // epilogue threads per stage (unit, token)

    for (int g = 0; g < n_groups; ++g) {
        const int s = g % stages, use = g / stages;
        const int row0 = u0 + g * rows_per_stage;
        const int nr = min(rows_per_stage, u1 - row0);
        if (!mbar_wait(&full[s], use & 1, a.err, kErrTimeoutFull)) break;
        const uint8_t* stage = smem + L.stages_off + (size_t)s * L.stage_bytes;
        float* pbuf = part + (size_t)(g & 1) * rows_per_stage * U * NB * kConsumerWarps;

        for (int r = 0; r < nr; ++r) {
#pragma unroll
            for (int u = 0; u < U; ++u) {
                const uint8_t* wrow = stage + ((size_t)u * rows_per_stage + r) * K * 2;
                float acc[NB];
#pragma unroll
                for (int b = 0; b < NB; ++b) acc[b] = 0.f;
                if (!XS) {
#pragma unroll
                    for (int j = 0; j < XRR; ++j) {
                        const int sc = j * 32 + lane;
                        if (sc < n_sc) {
                            uint4 w = lds128(wrow + (size_t)(col0 + sc * 8) * 2);
                            acc[0] = dot8_bf16(w, xr[j], acc[0]);
                        }
                    }
                } else {
                    for (int sc = lane; sc < n_sc; sc += 32) {
                        const int c = col0 + sc * 8;
                        uint4 w = lds128(wrow + (size_t)c * 2);
#pragma unroll
                        for (int b = 0; b < NB; ++b) {
                            uint4 xv = lds128(xs + ((size_t)b * K + c) * 2);
                            acc[b] = dot8_bf16(w, xv, acc[b]);
                        }
                    }
                }
#pragma unroll
                for (int b = 0; b < NB; ++b) {
                    float t = warp_sum(acc[b]);
                    if (lane == 0) pbuf[((r * U + u) * NB + b) * kConsumerWarps + warp] = t;
                }
            }
        }
        __syncwarp();
        if (lane == 0) mbar_arrive(&empty[s]);
        named_bar(1, kConsumerWarps * 32);

        // epilogue: thread t -> (row r, token b)
        const int t = threadIdx.x;
        if (t < n_vals) {
            const int r = t / NB, b = t % NB;
            if (r < nr && b < a.nb) {
                const int n = row0 + r;
                float accu[U];
#pragma unroll
                for (int u = 0; u < U; ++u) {
                    float sum = 0.f;
                    const float* pv = pbuf + ((r * U + u) * NB + b) * kConsumerWarps;
#pragma unroll
                    for (int w = 0; w < kConsumerWarps; ++w) sum += pv[w];
                    accu[u] = sum;
                }
                if (EPI == kEpiStore) {
                    float v = round_bf(accu[0]);
                    if (a.bias) v = round_bf(v + bf2f(reinterpret_cast<const bf16*>(a.bias)[n]));
                    if (a.lora.B) {
                        // sections of the fused q|k|v rows: t offset = section * rank
                        const int sec = (n >= a.lora.sec1) + (n >= a.lora.sec2);
                        v = lora_delta(a.lora, b, n, sec * a.lora.rank, v);
                    }
                    reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + n] = f2bf(v);
                } else if (EPI == kEpiResid) {
                    float v = round_bf(accu[0]);
                    if (a.lora.B) v = lora_delta(a.lora, b, n, 0, v);
                    const float rr = bf2f(reinterpret_cast<const bf16*>(a.resid)[(size_t)b * a.resid_stride + n]);
                    reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + n] = f2bf(rr + v);
                } else if (EPI == kEpiGlu) {
                    float gv = round_bf(accu[0]);
                    float uv = round_bf(accu[U - 1]);
                    if (a.lora.B) {
                        gv = lora_delta(a.lora, b, n, 0, gv);
                        uv = lora_delta(a.lora, b, a.N + n, a.lora.rank, uv);
                    }
                    const float h = glu_act<EPI>(gv, a.act);
                    reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + n] = f2bf(h * uv);
                } else {  // kEpiLmHead
                    const float v = accu[0];
                    reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + n] = f2bf(v);
                    if (a.logits_f32) a.logits_f32[(size_t)b * a.out_stride + n] = v;
                    const unsigned long long key = argmax_key(v, (uint32_t)n);
#pragma unroll
                    for (int bb = 0; bb < NB; ++bb)
                        if (bb == b && key > best[bb]) best[bb] = key;
                }
            }
        }
    }

    if (EPI == kEpiLmHead) {
        // CTA argmax, then grid argmax through one 64-bit atomicMax per token;
        // the last CTA publishes the ids and re-arms the keys for the next step.
#pragma unroll
        for (int b = 0; b < NB; ++b)
            if (best[b]) atomicMax(&amax_s[b], best[b]);
        named_bar(1, kConsumerWarps * 32);
        if (threadIdx.x == 0) {
            for (int b = 0; b < a.nb && b < NB; ++b)
                if (amax_s[b]) atomicMax(&a.amax[b], amax_s[b]);
            __threadfence();
            const unsigned int ticket = atomicAdd(a.done, 1u);
            if (ticket == gridDim.x - 1) {
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
}

// ------------------------------------------------------------------ host side
template <int NB, int EPI, int XR>
static const void* fn() {
    return reinterpret_cast<const void*>(&k_gemv<NB, EPI, XR>);
}

template <int EPI>
static const void* pick(int nb, int xr) {
    if (nb == 1) {
        switch (xr) {
            case 1: return fn<1, EPI, 1>();
            case 2: return fn<1, EPI, 2>();
            case 4: return fn<1, EPI, 4>();
            case 8: return fn<1, EPI, 8>();
            case 16: return fn<1, EPI, 16>();
            default: return fn<1, EPI, 0>();
        }
    }
    if (nb == 2) return fn<2, EPI, 0>();
    if (nb <= 4) return fn<4, EPI, 0>();
    if (nb <= 8) return fn<8, EPI, 0>();
    return nullptr;
}

static int nb_tmpl(int nb) { return nb == 1 ? 1 : nb == 2 ? 2 : nb <= 4 ? 4 : 8; }

bool gemv_plan(const GemvArgs& a, int epi, int device, GemvPlan* plan, std::string* why) {
    if (a.K <= 0 || a.K % 64 != 0) {
        if (why) *why = "gemv: K must be a positive multiple of 64";
        return false;
    }
    if (a.N <= 0 || a.nb < 1 || a.nb > 8) {
        if (why) *why = "gemv: need N > 0 and 1 <= tokens <= 8";
        return false;
    }
    const int U = epi == kEpiGlu ? 2 : 1;
    const size_t row_bytes = (size_t)a.K * 2 * U;
    int rps = (int)std::max<size_t>(1, 32768 / row_bytes);
    rps = std::min(rps, 16);
    const int nbt = nb_tmpl(a.nb);
    // register slice: sub-chunks per lane = ceil(K / 64 / 32)
    const int need = (a.K / 64 + 31) / 32;
    int xr = 0;
    if (nbt == 1) {
        for (int c : {1, 2, 4, 8, 16})
            if (need <= c) { xr = c; break; }
    }
    const bool xs = xr == 0;
    const size_t stage_bytes = ((size_t)rps * row_bytes + 127) & ~size_t(127);
    int stages = (int)std::min<size_t>(6, std::max<size_t>(2, (96 * 1024) / stage_bytes));
    GemvSmem L;
    int sms = num_sms(device);
    int max_smem = 0;
    cudaDeviceGetAttribute(&max_smem, cudaDevAttrMaxSharedMemoryPerBlockOptin, device);
    for (;;) {
        L = gemv_smem_layout(a.K, U, rps, stages, nbt, xs);
        if ((int)L.total <= max_smem) break;
        if (stages > 2) --stages;
        else if (rps > 1) --rps;
        else {
            if (why) *why = "gemv: row does not fit in shared memory";
            return false;
        }
    }
    const void* f = nullptr;
    switch (epi) {
        case kEpiStore: f = pick<kEpiStore>(a.nb, xr); break;
        case kEpiResid: f = pick<kEpiResid>(a.nb, xr); break;
        case kEpiGlu: f = pick<kEpiGlu>(a.nb, xr); break;
        case kEpiLmHead: f = pick<kEpiLmHead>(a.nb, xr); break;
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
    plan->grid = std::min(sms, a.N);
    plan->smem = L.total;
    plan->func = f;
    return true;
}

cudaError_t gemv_launch(const GemvArgs& a, int epi, const GemvPlan& plan, cudaStream_t s, bool pdl) {
    (void)epi;
    GemvArgs args = a;
    int rps = plan.rows_per_stage, st = plan.stages;
    void* params[] = {&args, &rps, &st};
    return launch_pdl(plan.func, dim3(plan.grid), dim3(kThreads), plan.smem, s, params, pdl);
}

}  // namespace ti
