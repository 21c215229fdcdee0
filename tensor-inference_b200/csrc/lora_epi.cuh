// lora_epi.cuh — the LoRA expansion applied in the epilogue of a projection
// (shared by the weight-streaming GEMV and the tensor-core GEMM).
#pragma once
#include "common.cuh"
#include "kernels.h"

namespace ti {

// LoRA expansion of one output element (qwen_adapter_model.cpp:27-29 + :42)
TI_DEVICE_INLINE float lora_delta(const GemvLora& L, int ad, int b, int row, int t_off, float base) {
    if (ad < 0 || ad >= L.n_adapters) return base;
    const uint16_t* br = L.B + (size_t)ad * L.B_adapter_stride + (size_t)row * L.rank;
    const float* t = L.t + (size_t)b * L.t_stride + t_off;
    float s = 0.f;
    for (int i = 0; i < L.rank; i += 8) {
        const uint4 w = *reinterpret_cast<const uint4*>(br + i);
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(&w);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            s = fmaf(bf_lo(wp[e]), t[i + 2 * e], s);
            s = fmaf(bf_hi(wp[e]), t[i + 2 * e + 1], s);
        }
    }
    const float up = round_bf(s);
    const float delta = round_bf(up * L.scale[ad]);
    return round_bf(base + delta);
}

// token b, output row `row`: the expansion precomputed in L.dval when present,
// else computed here (qwen_adapter_model.cpp:27-29 + :42)
TI_DEVICE_INLINE float lora_add(const GemvLora& L, int b, int row, int t_off, float base) {
    const int ad = L.adapter[b];
    if (ad < 0 || ad >= L.n_adapters) return base;
    if (L.dval) return round_bf(base + __uint_as_float((uint32_t)L.dval[(size_t)b * L.dval_stride + row] << 16));
    return lora_delta(L, ad, b, row, t_off, base);
}

}  // namespace ti
