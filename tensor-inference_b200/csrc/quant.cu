// quant.cu — GGUF Q4_0 / Q8_0 weights on the device.
//
// The reference names these formats as the planned second weight-map variant
// (include/tensor/parser/weight_map.hpp:24, README.md:30,292) without code;
// the block definitions are GGUF's (ggml):
//   Q4_0: 32 weights = fp16 d + 16 bytes; byte j holds element j (low nibble)
//         and element j + 16 (high nibble); w = d * (q - 8);
//         d = (element of largest magnitude) / -8, q = min(15, trunc(x / d + 8.5))
//   Q8_0: 32 weights = fp16 d + 32 int8; w = d * q; d = max|x| / 127, q = round(x / d)
// (ggml's quantize_row_q4_0_ref / quantize_row_q8_0_ref, restated).
//
// The engine keeps each quantised weight row as [K codes][K/32 fp16 scales]:
// Q4_0 codes in element order (element c in byte c/2, low nibble for even c),
// Q8_0 codes as int8 in element order.  A GEMV lane's 8 consecutive elements
// are then one aligned 32-bit (Q4_0) or 64-bit (Q8_0) load, and every row
// stays contiguous for the 1-D bulk copies of the weight stream.
//
// Quantisation on the device reproduces the CPU definition bit for bit: the
// same IEEE single-precision division, multiply and add (no contraction into
// FMA), round-to-nearest fp16 scale, truncation (Q4_0) or round-half-away
// (Q8_0) to integers.
#include "common.cuh"
#include "internal.h"
#include "kernels.h"

namespace ti {

namespace {

// one thread per 32-element block of an [nr, K] bf16 source (row pitch src_ld)
__global__ void k_quantize_rows(const uint16_t* __restrict__ src, int nr, int K, size_t src_ld,
                                uint8_t* __restrict__ dst, size_t dst_rb, int wf) {
    const int nblk = K / 32;
    const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (i >= (size_t)nr * nblk) return;
    const int r = (int)(i / nblk), blk = (int)(i % nblk);
    const uint16_t* x = src + (size_t)r * src_ld + (size_t)blk * 32;
    uint8_t* row = dst + (size_t)r * dst_rb;
    float v[32];
#pragma unroll
    for (int j = 0; j < 32; ++j) v[j] = __uint_as_float((uint32_t)x[j] << 16);
    if (wf == kWQ4) {
        float amax = 0.f, mx = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j)
            if (fabsf(v[j]) > amax) {
                amax = fabsf(v[j]);
                mx = v[j];
            }
        const float d = __fdiv_rn(mx, -8.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        uint8_t* codes = row + (size_t)blk * 16;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            int q0 = __float2int_rz(__fadd_rn(__fmul_rn(v[2 * j], id), 8.5f));
            int q1 = __float2int_rz(__fadd_rn(__fmul_rn(v[2 * j + 1], id), 8.5f));
            q0 = (int)(int8_t)q0;
            q1 = (int)(int8_t)q1;
            q0 = min(15, q0);
            q1 = min(15, q1);
            codes[j] = (uint8_t)((q0 & 15) | ((q1 & 15) << 4));
        }
        *reinterpret_cast<__half*>(row + (size_t)K / 2 + (size_t)blk * 2) = __float2half_rn(d);
    } else {
        float amax = 0.f;
#pragma unroll
        for (int j = 0; j < 32; ++j) amax = fmaxf(amax, fabsf(v[j]));
        const float d = __fdiv_rn(amax, 127.0f);
        const float id = d != 0.0f ? __fdiv_rn(1.0f, d) : 0.0f;
        int8_t* codes = reinterpret_cast<int8_t*>(row + (size_t)blk * 32);
#pragma unroll
        for (int j = 0; j < 32; ++j) codes[j] = (int8_t)(int)roundf(__fmul_rn(v[j], id));
        *reinterpret_cast<__half*>(row + (size_t)K + (size_t)blk * 2) = __float2half_rn(d);
    }
}

// GGUF blocks [nr, K/32] -> engine rows
__global__ void k_repack_gguf(const uint8_t* __restrict__ blocks, int nr, int K, uint8_t* __restrict__ dst,
                              size_t dst_rb, int wf) {
    const int nblk = K / 32;
    const size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x;
    if (i >= (size_t)nr * nblk) return;
    const int r = (int)(i / nblk), blk = (int)(i % nblk);
    uint8_t* row = dst + (size_t)r * dst_rb;
    if (wf == kWQ4) {
        const uint8_t* b = blocks + i * 18;
        uint8_t* codes = row + (size_t)blk * 16;
#pragma unroll
        for (int j = 0; j < 16; ++j) {
            // element e: byte e % 16 of the block, low nibble for e < 16
            const int e0 = 2 * j, e1 = 2 * j + 1;
            const int q0 = e0 < 16 ? (b[2 + e0] & 15) : (b[2 + e0 - 16] >> 4);
            const int q1 = e1 < 16 ? (b[2 + e1] & 15) : (b[2 + e1 - 16] >> 4);
            codes[j] = (uint8_t)(q0 | (q1 << 4));
        }
        row[(size_t)K / 2 + (size_t)blk * 2] = b[0];
        row[(size_t)K / 2 + (size_t)blk * 2 + 1] = b[1];
    } else {
        const uint8_t* b = blocks + i * 34;
#pragma unroll
        for (int j = 0; j < 32; ++j) row[(size_t)blk * 32 + j] = b[2 + j];
        row[(size_t)K + (size_t)blk * 2] = b[0];
        row[(size_t)K + (size_t)blk * 2 + 1] = b[1];
    }
}

}  // namespace

cudaError_t quantize_rows_launch(const uint16_t* src, int nr, int K, size_t src_ld, uint8_t* dst, size_t dst_rb,
                                 int wf, cudaStream_t s) {
    if (K % 32 != 0 || nr < 0 || (wf != kWQ4 && wf != kWQ8)) return cudaErrorInvalidValue;
    const size_t n = (size_t)nr * (K / 32);
    if (n == 0) return cudaSuccess;
    k_quantize_rows<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(src, nr, K, src_ld, dst, dst_rb, wf);
    return cudaGetLastError();
}

cudaError_t repack_gguf_launch(const uint8_t* blocks, int nr, int K, uint8_t* dst, size_t dst_rb, int wf,
                               cudaStream_t s) {
    if (K % 32 != 0 || nr < 0 || (wf != kWQ4 && wf != kWQ8)) return cudaErrorInvalidValue;
    const size_t n = (size_t)nr * (K / 32);
    if (n == 0) return cudaSuccess;
    k_repack_gguf<<<(unsigned)((n + 127) / 128), 128, 0, s>>>(blocks, nr, K, dst, dst_rb, wf);
    return cudaGetLastError();
}

// engine rows (host copy) -> GGUF blocks, the inverse of k_repack_gguf
void gguf_from_rows(const uint8_t* rows, int nr, int K, size_t rb, int wf, uint8_t* blocks) {
    const int nblk = K / 32;
    for (int r = 0; r < nr; ++r)
        for (int blk = 0; blk < nblk; ++blk) {
            const uint8_t* row = rows + (size_t)r * rb;
            if (wf == kWQ4) {
                uint8_t* b = blocks + ((size_t)r * nblk + blk) * 18;
                const uint8_t* codes = row + (size_t)blk * 16;
                b[0] = row[(size_t)K / 2 + (size_t)blk * 2];
                b[1] = row[(size_t)K / 2 + (size_t)blk * 2 + 1];
                for (int j = 0; j < 16; ++j) {
                    auto q = [&](int e) { return (codes[e / 2] >> (4 * (e & 1))) & 15; };
                    b[2 + j] = (uint8_t)(q(j) | (q(j + 16) << 4));
                }
            } else {
                uint8_t* b = blocks + ((size_t)r * nblk + blk) * 34;
                b[0] = row[(size_t)K + (size_t)blk * 2];
                b[1] = row[(size_t)K + (size_t)blk * 2 + 1];
                for (int j = 0; j < 32; ++j) b[2 + j] = row[(size_t)blk * 32 + j];
            }
        }
}

}  // namespace ti
