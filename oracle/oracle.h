/*
 * oracle.h — CPU restatement of the reference decode path (TEST INFRASTRUCTURE).
 *
 * This library is the parity checker for the B200 engine.  It is loaded only by
 * tests/, __graft_entry__.smoke() and bench.py's cpu_baseline / --impl reference
 * leg.  Nothing in the product links or calls it.
 *
 * Every function restates one piece of carbon-os/tensor-inference's CUDA path
 * (paths below are relative to that project's root) on the host, with the same
 * bf16 rounding points, so the GPU engine can be compared on identical inputs:
 *
 *   orc_embedding        src/backend/cuda/ops.cu:46-88
 *   orc_matmul_t_*       src/backend/cuda/ops.cu:94-148
 *   orc_rms_norm         src/backend/cuda/ops.cu:154-204, 726-774 (offset form)
 *   orc_rope_freqs       src/backend/cuda/ops.cu:235-278
 *   orc_rope             src/backend/cuda/ops.cu:210-233, 280-312
 *   orc_silu/mul/add     src/backend/cuda/ops.cu:318-381
 *   orc_softmax_f32      src/backend/cuda/ops.cu:387-438
 *   orc_attention        src/backend/cuda/ops.cu:444-544
 *   orc_add_bias         src/backend/cuda/ops.cu:671-701
 *   orc_gelu             src/backend/cuda/ops.cu:707-724
 *   orc_mul_scalar       src/backend/cuda/ops.cu:776-788
 *   orc_model_forward    src/models/llama/llama_model.cpp:103-238,
 *                        src/models/qwen/qwen_model.cpp:73-146,
 *                        src/models/qwen/qwen_adapter_model.cpp:22-193,
 *                        src/models/gemma/gemma_model.cpp:57-129,
 *                        src/models/mistral/mistral_model.cpp:109-178
 *   orc_q4_0_* / q8_0    GGUF block formats (ggml quantize_row_q4_0_ref /
 *                        quantize_row_q8_0_ref, as published by ggml); the
 *                        reference names them only as planned work
 *                        (include/tensor/parser/weight_map.hpp:24)
 *   orc_pkm_*            PKM router spec (README.md:58-72,157-180 and the
 *                        PKM benchmark configuration); no code in the reference
 *   orc_sample_top_p/k   src/inference/sampling/top_p.cpp:56-134
 *   orc_sample_exact     the device sampler's exact form of the same samplers
 *
 * Parity pinning: the reference has no tests or golden vectors for this path.
 * The oracle is pinned against the reference's own CUDA implementation, built
 * from its sources into oracle/_ref/libref.so and run on a B200; the committed
 * fixtures in tests/golden/ hold those outputs.  The samplers are pinned on the
 * host against the reference's own sampler code in the same library.
 */
#pragma once
#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

/* ---------------------------------------------------------------- synthetic */
uint64_t orc_name_hash(const char* name);
/* bf16 values ~ N(0, std) (4-term Irwin-Hall in integer arithmetic, one fp32
 * multiply, RNE to bf16); element i depends only on (seed, name_hash, i). */
void orc_fill_bf16(uint16_t* out, size_t n, uint64_t seed, uint64_t name_hash, float std_);
void orc_fill_f32(float* out, size_t n, uint64_t seed, uint64_t name_hash, float std_);
void orc_fill_ids(int32_t* out, size_t n, uint64_t seed, uint64_t name_hash, int32_t vocab);

/* ---------------------------------------------------------------- scalars */
uint16_t orc_f32_to_bf16(float f);
float orc_bf16_to_f32(uint16_t b);
uint16_t orc_f32_to_f16(float f);
float orc_f16_to_f32(uint16_t h);
void orc_set_threads(int n);
int orc_get_threads(void);

/* ---------------------------------------------------------------- ops */
void orc_embedding(const uint16_t* w, int vocab, int hidden, const int32_t* ids, int n, uint16_t* out);
void orc_matmul_t_bf16(const uint16_t* a, const uint16_t* b, uint16_t* c, int M, int N, int K);
/* same product, fp32 accumulators exposed (before bf16 rounding) */
void orc_matmul_t_bf16_f32out(const uint16_t* a, const uint16_t* b, float* c, int M, int N, int K);
void orc_matmul_t_f32(const float* a, const float* b, float* c, int M, int N, int K);
void orc_rms_norm(const uint16_t* x, const uint16_t* w, uint16_t* out, int rows, int hidden, float eps, int offset);
typedef struct {
    int   apply_scaling;
    float factor;
    float low_freq_factor;
    float high_freq_factor;
    int   original_max_pos;
} orc_rope_scaling;
void orc_rope_freqs(int head_dim, float theta, const orc_rope_scaling* sc, float* freqs);
void orc_rope(const uint16_t* x, uint16_t* out, int seq, int heads, int head_dim, int seq_offset,
              const float* freqs);
void orc_silu(const uint16_t* x, uint16_t* out, size_t n);
void orc_gelu(const uint16_t* x, uint16_t* out, size_t n);
void orc_mul(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n);
void orc_add(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n);
void orc_mul_scalar(const uint16_t* x, float s, uint16_t* out, size_t n);
void orc_add_bias(const uint16_t* x, const uint16_t* bias, uint16_t* out, int rows, int hidden);
void orc_softmax_f32(float* x, int rows, int cols);
void orc_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out,
                   int seq, int n_heads, int kv_len, int n_kv, int head_dim, int causal, int sliding_window);

/* ---------------------------------------------------------------- GGUF blocks */
/* Q4_0: 32 weights per block, 18 bytes: fp16 d, 16 bytes of nibbles
 * (low nibble = element j, high nibble = element j+16). */
void orc_q4_0_quantize(const float* x, size_t n, uint8_t* blocks);
void orc_q4_0_dequantize(const uint8_t* blocks, size_t n, float* out);
/* Q8_0: 32 weights per block, 34 bytes: fp16 d, 32 int8. */
void orc_q8_0_quantize(const float* x, size_t n, uint8_t* blocks);
void orc_q8_0_dequantize(const uint8_t* blocks, size_t n, float* out);
/* y[m,n] = bf16(sum_k x[m,k] * dequant(W)[n,k]); W in GGUF blocks, row-major */
void orc_matmul_t_q(const uint16_t* x, const uint8_t* wq, int qtype, uint16_t* y, float* y32, int M, int N, int K);

/* ---------------------------------------------------------------- PKM */
/* canonical squared distance: d = q[t]-c[t] (rn), acc = fma(d, d, acc), t = 0..D-1 */
float orc_pkm_dist(const float* q, const float* c, int dim);
void orc_pkm_assign(const float* c1, const float* c2, int n_codes, int half_dim,
                    const float* queries, int n, int32_t* addr);
/* table[n_codes^2] = lowest adapter id whose centroid maps to that address, else -1 */
void orc_pkm_build_table(const int32_t* centroid_addr, int n_adapters, int32_t* table, int table_size);

/* ---------------------------------------------------------------- model */
enum { ORC_ARCH_LLAMA = 0, ORC_ARCH_QWEN2 = 1, ORC_ARCH_GEMMA = 2, ORC_ARCH_MISTRAL = 3 };
enum { ORC_W_BF16 = 0, ORC_W_Q4_0 = 1, ORC_W_Q8_0 = 2 };
typedef struct {
    int   arch;
    int   hidden, n_layers, n_heads, n_kv_heads, head_dim, intermediate, vocab;
    float rms_eps, rope_theta;
    orc_rope_scaling rope;
    int   qkv_bias;
    int   sliding_window;
    int   weight_format;   /* ORC_W_*: linear weights of the layers quantised to GGUF blocks */
} orc_model_desc;

typedef struct orc_model orc_model;
orc_model* orc_model_create(const orc_model_desc* d);
void orc_model_destroy(orc_model* m);
/* fill every tensor of the model with synthetic values (names as in the HF
 * checkpoint the reference loads: model.layers.{i}.self_attn.q_proj.weight ...) */
void orc_model_init_synthetic(orc_model* m, uint64_t seed, float std_);
/* restrict synthetic init / forward to layers [0, n) (timing samples) */
void orc_model_limit_layers(orc_model* m, int n);
int orc_model_set_weight(orc_model* m, const char* name, const uint16_t* data, size_t n);
int orc_model_get_weight(orc_model* m, const char* name, uint16_t* out, size_t n);
/* LoRA adapter slot `slot`: rank, alpha; weights via orc_model_set_lora or synthetic */
int orc_model_add_adapter(orc_model* m, int slot, int rank, float alpha, int proj_mask,
                          uint64_t seed, float std_a, float std_b);
int orc_model_set_lora(orc_model* m, int slot, const char* name, const uint16_t* data, size_t n);

typedef struct orc_seq orc_seq;
orc_seq* orc_seq_create(orc_model* m, int max_seq);
void orc_seq_destroy(orc_seq* s);
int orc_seq_len(const orc_seq* s);
/* A context of `len` cached tokens with seeded N(0, std) K/V rows in every layer
 * (no prefill), for timing decode steps at a given context length. */
int orc_seq_fill_synthetic(orc_seq* s, int len, uint64_t seed, float std_);
/* One forward call (prefill when n > 1, decode when n == 1), as the reference's
 * Model::forward.  Writes bf16 logits of the LAST row to logits_bf16 (vocab),
 * fp32 logits (pre-rounding) of the last row to logits_f32; either may be NULL.
 * adapter = slot or -1.  Returns 0 or an error code. */
int orc_model_forward(orc_model* m, orc_seq* s, const int32_t* ids, int n, int adapter,
                      uint16_t* logits_bf16, float* logits_f32);
/* final hidden state (after final norm) of the last row, bf16 */
int orc_seq_last_hidden(const orc_seq* s, uint16_t* out, int hidden);
/* read K/V rows of one layer: [len, n_kv, head_dim] bf16 */
int orc_seq_read_kv(const orc_seq* s, int layer, int which, uint16_t* out, int len);
/* argmax with lowest-index tie break */
int32_t orc_argmax_f32(const float* x, int n);

/* Stochastic sampling of one fp32 logits row, restating
 * src/inference/sampling/top_p.cpp: TopP::sample (:56-99) and TopK::sample
 * (:102-134).  u is the uniform draw in [0, 1) the reference takes from its
 * engine; stable = 0 orders equal values as the reference's std::sort /
 * std::partial_sort do, stable = 1 by ascending token id. */
int32_t orc_sample_top_p(const float* logits, int vocab, float temperature, float p, float u, int stable);
int32_t orc_sample_top_k(const float* logits, int vocab, float temperature, int k, float u, int stable);
/* The device sampler's exact form of TopP / TopK on bf16 logits: order by
 * logit descending, equal logits by ascending id; per-token weights
 * floor(fp32(exp(v - vmax)) * 2^63) with exp evaluated by a fixed sequence of
 * IEEE operations; cut and pick by exact 128-bit integer sums (oracle.cpp has
 * the full statement).  kind: ORC_SAMPLE_TOP_P or ORC_SAMPLE_TOP_K. */
enum { ORC_SAMPLE_TOP_P = 1, ORC_SAMPLE_TOP_K = 2 };
int32_t orc_sample_exact(const uint16_t* logits, int vocab, int kind, float temperature, float p, int k, float u);
/* the first n draws of std::uniform_real_distribution<float>(0, 1) over
 * std::mt19937_64(seed) (top_p.cpp:84-86) */
void orc_sample_draws(uint64_t seed, int n, float* u);

#ifdef __cplusplus
}
#endif
