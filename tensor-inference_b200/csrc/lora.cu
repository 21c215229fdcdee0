// lora.cu — LoRA "shrink" step: t[b, :] = bf16(x_b @ A^T) for each token's adapter.
//
// The reference's apply_lora (qwen_adapter_model.cpp:22-30) computes
// down = matmul_t(x, lora_A) (rounded to bf16), up = matmul_t(down, lora_B),
// delta = up * (alpha / rank), and add_if_present adds it to the base
// projection (:35-43).  Here `down` is this kernel's output; the weight-streaming
// GEMV that produces the base projection applies the expansion in its epilogue.
// Per-token adapters make it a segmented gather: token b reads the A rows of
// adapter[b] (no adapter: nothing is written and the GEMV skips the delta).
// x is the projection's input: RMSNorm(hidden) for q|k|v and gate|up (the same
// normalised row the reference passes to both the base and the LoRA matmul),
// the attention output for o, the SwiGLU activation for down.
#include "common.cuh"
#include "kernels.h"

namespace ti {

constexpr int kShrinkThreads = 256;
constexpr int kShrinkRowsPerCta = 16;

__global__ void __launch_bounds__(kShrinkThreads) k_lora_shrink(const LoraShrinkArgs a) {
    extern __shared__ __align__(16) uint8_t smem[];
    uint16_t* xs = reinterpret_cast<uint16_t*>(smem);  // [K] normalised bf16 row
    __shared__ float red[kShrinkThreads / 32];
    const int b = blockIdx.y, tid = threadIdx.x, warp = tid >> 5, lane = tid & 31;
    if (tid == 0) pdl_trigger();
    const int ad = a.adapter[b];
    pdl_wait();
    if (ad < 0 || ad >= a.n_adapters) return;
    const int K = a.K;
    const uint16_t* x = a.x + (size_t)b * a.x_stride;
    // load (and normalise) the row: 8 bf16 per thread-iteration
    float ss = 0.f;
    for (int c = tid * 8; c < K; c += kShrinkThreads * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(x + c);
        *reinterpret_cast<uint4*>(xs + c) = v;
        const uint32_t* vp = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            ss = fmaf(bf_lo(vp[e]), bf_lo(vp[e]), ss);
            ss = fmaf(bf_hi(vp[e]), bf_hi(vp[e]), ss);
        }
    }
    if (a.norm_w) {
        ss = warp_sum(ss);
        if (lane == 0) red[warp] = ss;
        __syncthreads();
        float tot = 0.f;
#pragma unroll
        for (int w = 0; w < kShrinkThreads / 32; ++w) tot += red[w];
        const float scale = rsqrtf(tot / (float)K + a.eps);  // ops.cu:179
        const float off = a.norm_offset ? 1.0f : 0.0f;
        for (int c = tid * 8; c < K; c += kShrinkThreads * 8) {
            uint4 v = *reinterpret_cast<const uint4*>(xs + c);
            const uint4 wn = *reinterpret_cast<const uint4*>(a.norm_w + c);
            uint32_t* vp = reinterpret_cast<uint32_t*>(&v);
            const uint32_t* wp = reinterpret_cast<const uint32_t*>(&wn);
#pragma unroll
            for (int e = 0; e < 4; ++e) {
                const float lo = bf_lo(vp[e]) * scale * (bf_lo(wp[e]) + off);
                const float hi = bf_hi(vp[e]) * scale * (bf_hi(wp[e]) + off);
                vp[e] = pack_bf2(lo, hi);
            }
            *reinterpret_cast<uint4*>(xs + c) = v;
        }
    }
    __syncthreads();
    // rows of this CTA: warp w takes rows r0 + w, r0 + w + 8
    const uint16_t* A = a.A + (size_t)ad * a.A_adapter_stride;
    const int r0 = blockIdx.x * kShrinkRowsPerCta;
    for (int r = r0 + warp; r < min(a.T, r0 + kShrinkRowsPerCta); r += kShrinkThreads / 32) {
        const uint16_t* ar = A + (size_t)r * K;
        float acc = 0.f;
        for (int c = lane * 8; c < K; c += 32 * 8) {
            const uint4 w = *reinterpret_cast<const uint4*>(ar + c);
            const uint4 xv = *reinterpret_cast<const uint4*>(xs + c);
            acc = dot8_bf16(w, xv, acc);
        }
        acc = warp_sum(acc);
        if (lane == 0) {
            if (a.tp) {
                // row-parallel under tensor parallelism: fp32 partial to every rank
                for (int q = 0; q < a.tp; ++q) a.peer_t[q][(size_t)b * a.t_stride + r] = acc;
            } else {
                a.t[(size_t)b * a.t_stride + r] = round_bf(acc);
            }
        }
    }
    if (a.tp) __threadfence_system();
}

cudaError_t lora_shrink_launch(const LoraShrinkArgs& a, cudaStream_t s, bool pdl) {
    if (a.K % 8 != 0 || a.T <= 0) return cudaErrorInvalidValue;
    LoraShrinkArgs args = a;
    void* params[] = {&args};
    const size_t smem = (size_t)a.K * 2;
    const void* f = reinterpret_cast<const void*>(&k_lora_shrink);
    if (smem > 48 * 1024) {
        cudaError_t e = cudaFuncSetAttribute(f, cudaFuncAttributeMaxDynamicSharedMemorySize, (int)smem);
        if (e != cudaSuccess) return e;
    }
    return launch_pdl(f, dim3((a.T + kShrinkRowsPerCta - 1) / kShrinkRowsPerCta, a.nb), dim3(kShrinkThreads), smem, s,
                      params, pdl);
}


// ---- expansion ahead of the tensor-core GEMM: CTA (row tile, token b), one output
//      row per thread, t read as warp-uniform broadcasts.  One CTA per token (rather
//      than per adapter, rereading nothing) measured faster: the rereads of a B row
//      by tokens sharing an adapter hit L2, and the extra CTAs hide latency.
constexpr int kExpandThreads = 128;

__global__ void __launch_bounds__(kExpandThreads)
    k_lora_expand(const GemvLora L, int nb, int n_rows, int glu_n, uint16_t* dval, int dval_stride) {
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
    if (!L.adapter || L.rank % 8 != 0 || nb < 1) return cudaErrorInvalidValue;
    GemvLora args = L;
    void* params[] = {&args, &nb, &n_rows, &glu_n, &dval, &dval_stride};
    return launch_pdl(reinterpret_cast<const void*>(&k_lora_expand),
                      dim3((n_rows + kExpandThreads - 1) / kExpandThreads, nb), dim3(kExpandThreads), 0, s, params,
                      pdl);
}

}  // namespace ti
