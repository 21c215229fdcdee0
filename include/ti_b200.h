/*
 * ti_b200.h — C ABI of the B200-native decode path (libti_b200.so).
 *
 * carbon-os/tensor-inference (the reference) has no C ABI (its README.md:32
 * only announces one); its compute boundary is the C++ interface
 * tensor::backend::{Device, Tensor, ops} (include/tensor/backend/{device,tensor,ops}.hpp) and
 * the models::CausalLM concept (include/tensor/models/concepts.hpp:16-23).
 * Each entry point below names the reference interface it replaces.
 *
 * Conventions
 *  - Every entry returns ti_status (0 = TI_OK) and never throws; on error a
 *    thread-local message is available from ti_last_error().
 *  - "device pointer" arguments are CUDA global-memory addresses on the
 *    engine's / op's device; "host pointer" arguments are ordinary (optionally
 *    pinned) host memory.  bf16 values travel as uint16_t bit patterns.
 *  - `stream` is a cudaStream_t passed as void* (NULL = legacy default stream).
 *  - Shapes are validated on the host before any launch; invalid arguments
 *    return TI_ERR_INVALID and launch nothing.
 */
#ifndef TI_B200_H
#define TI_B200_H

#include <stddef.h>
#include <stdint.h>

#ifdef __cplusplus
extern "C" {
#endif

typedef int ti_status;
enum {
    TI_OK = 0,
    TI_ERR_INVALID = 1,     /* bad argument / shape (reference: std::invalid_argument, ops.cu:144,552,561) */
    TI_ERR_CUDA = 2,        /* CUDA runtime error (reference: std::runtime_error from cuda_check, ops.cu:19-22) */
    TI_ERR_OOM = 3,         /* device or page-pool allocation failed */
    TI_ERR_UNSUPPORTED = 4, /* valid request this build does not support (dtype, head_dim ...) */
    TI_ERR_STATE = 5,       /* wrong object state (unknown sequence, KV cache full, ...) */
    TI_ERR_TIMEOUT = 6,     /* a bounded device-side wait gave up (see ti_engine_check) */
    TI_ERR_NOT_FOUND = 7    /* unknown tensor name (reference: parser::TensorNotFound, errors.hpp) */
};

const char* ti_last_error(void);
int ti_version(void); /* major*10000 + minor*100 + patch */
/* Library start-up check: every visible CUDA device is an sm_100 part (B200),
 * the only code this build carries; *n_devices (may be NULL) = their count.
 * TI_ERR_UNSUPPORTED names the first device that is not, or reports that no
 * device is visible.  Other entries do not require it; a caller calls it
 * first to fail early on the wrong hardware.  (The reference initialises
 * lazily: Device::cuda / cuBLAS handles, device.cu:15-43, ops.cu:30-40.) */
ti_status ti_init(int* n_devices);
/* Release what the library holds outside engines, PKM routers and GGUF files:
 * the ops' cached RoPE tables and the unused blocks of every device's
 * stream-ordered pool.  Call with no op in flight; the library stays usable. */
ti_status ti_shutdown(void);
/* Health check of the bounded device waits that guard every wait on another
 * CTA, kernel or rank (no counterpart in the reference, which never waits on
 * the device): on `device`, a wait on a flag nothing writes and a wait on an
 * mbarrier nothing completes, each limited to limit_us (1 .. 10^7).  TI_OK when
 * both gave up and set their error bits; waited_us[0..1] (may be NULL) = how
 * long each waited.  TI_ERR_STATE when a wait did not report giving up. */
ti_status ti_selftest_waits(int device, int limit_us, double* waited_us);

/* ================================================================= device
 * replaces tensor::backend::Device (include/tensor/backend/device.hpp:10-42,
 * src/backend/cuda/device.cu:15-43) and the allocation inside Tensor
 * (src/backend/cuda/tensor.cu:72-121).  Allocations come from a
 * stream-ordered caching pool, so per-op temporaries cost no cudaMalloc. */
ti_status ti_device_count(int* count);
ti_status ti_device_info(int device, char* name, size_t name_len, size_t* total_mem);
ti_status ti_set_device(int device);
ti_status ti_malloc(int device, size_t bytes, void** ptr);
ti_status ti_free(int device, void* ptr);
ti_status ti_memset(void* dst, int value, size_t bytes, void* stream);
ti_status ti_memcpy_h2d(void* dst, const void* src, size_t bytes, void* stream);
ti_status ti_memcpy_d2h(void* dst, const void* src, size_t bytes, void* stream);
ti_status ti_memcpy_d2d(void* dst, const void* src, size_t bytes, void* stream);
ti_status ti_stream_sync(void* stream);

/* ================================================================= ops
 * One entry per tensor::backend::ops function (include/tensor/backend/ops.hpp:19-117).
 * All tensors are contiguous, row-major, device pointers; `out` never aliases
 * an input unless stated.  Arithmetic and rounding points follow the
 * reference kernel cited beside each entry. */
enum { TI_DTYPE_F32 = 0, TI_DTYPE_BF16 = 1, TI_DTYPE_F16 = 2, TI_DTYPE_I32 = 3,
       TI_DTYPE_Q4_0 = 16, TI_DTYPE_Q8_0 = 17 };

/* ops.hpp:27 / ops.cu:46-88. ids: HOST array of n token ids. */
ti_status ti_op_embedding(const void* weight, int vocab, int hidden, const int32_t* ids_host, int n,
                          void* out, void* stream);
/* ops.hpp:34 / ops.cu:94-148: c[M,N] = a[M,K] @ b[N,K]^T, fp32 accumulate; dtype BF16 or F32. */
ti_status ti_op_matmul_t(int dtype, const void* a, const void* b, void* c, int M, int N, int K, void* stream);
/* ops.hpp:40,114 / ops.cu:154-204,726-774: offset=1 adds 1 to the weight (Gemma). */
ti_status ti_op_rms_norm(const void* x, const void* w, void* out, int rows, int hidden, float eps, int offset,
                         void* stream);
typedef struct {
    int   apply_scaling;
    float factor;
    float low_freq_factor;
    float high_freq_factor;
    int   original_max_pos;
} ti_rope_scaling;
/* ops.hpp:46-62 / ops.cu:210-312. x: [seq, heads, head_dim]; scaling may be NULL (plain RoPE). */
ti_status ti_op_rope(const void* x, void* out, int seq, int heads, int head_dim, int seq_offset, float theta,
                     const ti_rope_scaling* scaling, void* stream);
/* ops.hpp:67-73,111,117 / ops.cu:318-381,707-724,776-788 (bf16 in/out, fp32 math). */
enum { TI_EW_SILU = 0, TI_EW_GELU = 1, TI_EW_MUL = 2, TI_EW_ADD = 3, TI_EW_MUL_SCALAR = 4 };
ti_status ti_op_elementwise(int kind, const void* a, const void* b, float scalar, void* out, size_t n, void* stream);
/* ops.hpp:106 / ops.cu:671-701: x [rows, hidden] + bias [hidden]. */
ti_status ti_op_add_bias(const void* x, const void* bias, void* out, int rows, int hidden, void* stream);
/* ops.hpp:78 / ops.cu:387-438: fp32 row softmax; x may be F32 or BF16, out is F32. */
ti_status ti_op_softmax(int dtype, const void* x, float* out, int rows, int cols, void* stream);
/* ops.hpp:87 / ops.cu:444-544: GQA attention, bf16 in/out, fp32 inside.
 * q [seq, n_heads, hd], k/v [kv_len, n_kv, hd]; mask only when causal && seq > 1. */
ti_status ti_op_attention(const void* q, const void* k, const void* v, void* out, int seq, int n_heads,
                          int kv_len, int n_kv, int head_dim, int causal, int sliding_window, void* stream);
/* Decode attention over a paged KV cache, one new token per sequence: the
 * work of ops::rope x2 + the cache cudaMemcpy + ops::slice x2 + ops::attention
 * for one layer (llama_model.cpp:147-182, ops.cu:210-312,444-544).
 * qkv [batch, (n_heads + 2*n_kv)*head_dim] bf16 holds each token's q|k|v before
 * RoPE; pos[b] = tokens already cached for sequence seq[b]; the rotated k and v
 * are appended at position pos[b] of the sequence's pages; the token attends
 * to positions [max(0, pos - sliding_window + 1) or 0, pos].
 * page_table [*, pt_stride] int32 page ids (16 tokens per page);
 * k_pages / v_pages [n_pages, n_kv, 16, head_dim] bf16; out [batch, n_heads*head_dim].
 * max_len bounds pos + 1 (it sizes the split-KV work).  Split partials live in
 * scratch taken from the device's stream-ordered memory pool. */
ti_status ti_op_paged_attention(const void* qkv, int batch, int n_heads, int n_kv, int head_dim,
                                const int32_t* pos, const int32_t* seq, const int32_t* page_table, int pt_stride,
                                void* k_pages, void* v_pages, int n_pages, int max_len, float theta,
                                const ti_rope_scaling* scaling, int sliding_window, void* out, void* stream);
/* Same computation and arguments as ti_op_paged_attention, for callers that
 * cannot allocate device memory where they run it (a plugin whose host
 * application owns the device-memory budget, or a process whose memory is
 * fully reserved by another framework's allocator).  No counterpart in the
 * reference.  Calls no allocator: the scratch is a fixed 8 MiB array that every
 * GPU loading this library holds until exit.  The first call on a device looks
 * up that array's device address with a synchronous runtime query; that address
 * belongs to the device's CUDA context, so do not call this entry on a
 * device after resetting it (cudaDeviceReset).  Sizes whose scratch exceeds
 * 8 MiB return TI_ERR_INVALID.  All calls share the array, so calls that
 * overlap on the GPU race; order them on one stream.  As with
 * ti_op_paged_attention, out-of-range page ids or positions found on the device
 * are skipped, not reported: validate page tables on the host. */
ti_status ti_op_paged_attention_noalloc(const void* qkv, int batch, int n_heads, int n_kv, int head_dim,
                                        const int32_t* pos, const int32_t* seq, const int32_t* page_table,
                                        int pt_stride, void* k_pages, void* v_pages, int n_pages, int max_len,
                                        float theta, const ti_rope_scaling* scaling, int sliding_window, void* out,
                                        void* stream);
/* ops.hpp:98 / ops.cu:586-616 (BF16<->F32; same dtype = copy). */
ti_status ti_op_cast(int src_dtype, int dst_dtype, const void* x, void* out, size_t n, void* stream);
/* ops.hpp:95 / ops.cu:559-584: 2-D transpose [rows, cols] -> [cols, rows], F32 or BF16. */
ti_status ti_op_transpose2d(int dtype, const void* x, void* out, int rows, int cols, void* stream);

/* ================================================================= engine
 * The fused decode engine.  Replaces the per-token call chain
 * Generator::generate -> Model::forward -> layer_forward -> ops::*
 * (src/inference/generator.cpp:24-84, src/models/llama/llama_model.cpp:103-238,
 * src/models/qwen/qwen_model.cpp:73-146, src/models/qwen/qwen_adapter_model.cpp:22-193,
 * src/models/gemma/gemma_model.cpp:57-129, src/models/mistral/mistral_model.cpp:109-178)
 * and the contiguous KVCache (include/tensor/models/kv_cache.hpp:24-59) with a
 * paged bf16 KV cache of 16-token pages. */
enum { TI_ARCH_LLAMA = 0, TI_ARCH_QWEN2 = 1, TI_ARCH_GEMMA = 2, TI_ARCH_MISTRAL = 3 };
enum { TI_WFMT_BF16 = 0, TI_WFMT_Q4_0 = 1, TI_WFMT_Q8_0 = 2 };
enum { TI_PROJ_Q = 1, TI_PROJ_K = 2, TI_PROJ_V = 4, TI_PROJ_O = 8, TI_PROJ_GATE = 16, TI_PROJ_UP = 32,
       TI_PROJ_DOWN = 64 };

typedef struct {
    int   arch;                 /* TI_ARCH_* */
    int   hidden, n_layers, n_heads, n_kv_heads, head_dim, intermediate, vocab;
    float rms_eps, rope_theta;
    ti_rope_scaling rope;
    int   qkv_bias;             /* Qwen2: q/k/v carry a bias */
    int   sliding_window;       /* Mistral; <= 0 = none */
    int   weight_format;        /* TI_WFMT_*: storage of the layers' linear weights */
} ti_model_desc;

typedef struct {
    int device;                 /* CUDA device index */
    int max_batch;              /* sequences per decode step */
    int max_seqs;               /* live sequences */
    int max_seq_len;            /* tokens per sequence (page-table width = ceil(/16)) */
    int kv_pages;               /* pages in the pool; 0 = max_seqs * ceil(max_seq_len/16) */
    int max_adapters;           /* LoRA adapter slots resident in HBM (0 = LoRA off) */
    int max_lora_rank;
    int lora_proj_mask;         /* TI_PROJ_* the adapter slots reserve room for */
    int tp_size, tp_rank;       /* tensor parallel group (1, 0 = single GPU) */
    const void* nccl_id;        /* 128-byte ncclUniqueId shared by the TP group (NULL when tp_size == 1) */
} ti_engine_opts;

typedef struct ti_engine ti_engine;

/* ---- tensor parallelism (no counterpart in the reference, which runs one GPU;
 * the split is the one the decode path's north star names: q/k/v by heads and
 * gate/up by rows (column-parallel), o and down by input columns (row-parallel,
 * NCCL all-reduce of fp32 partial sums), LM head by vocabulary rows (greedy id
 * by an all-reduce max); embeddings and norms replicated). */
typedef struct {
    int tp, rank;
    int nq, nkv, q0, kv0;   /* local q / kv heads and the first global index of each */
    int inter, i0;          /* local intermediate rows of gate/up (= input columns of down) */
    int vocab, v0;          /* local LM-head rows (vocabulary slice) */
} ti_tp_shard;
/* the shard of rank tp_rank of tp_size (host only; validates the split) */
ti_status ti_tp_plan(const ti_model_desc* desc, int tp_size, int tp_rank, ti_tp_shard* out);
/* a fresh 128-byte NCCL unique id (one rank creates it, all pass it in ti_engine_opts.nccl_id) */
ti_status ti_nccl_unique_id(void* out128);

ti_status ti_engine_create(const ti_model_desc* desc, const ti_engine_opts* opts, ti_engine** out);
ti_status ti_engine_destroy(ti_engine* e);
/* device bytes held by weights / KV pool / adapters / work buffers */
ti_status ti_engine_memory(const ti_engine* e, size_t* weights, size_t* kv, size_t* adapters, size_t* work);

/* Upload one checkpoint tensor by its reference name ("model.embed_tokens.weight",
 * "model.layers.{i}.self_attn.q_proj.weight", "...q_proj.bias", "lm_head.weight", ...),
 * the names LlamaModel::load / QwenModel::load read (llama_model.cpp:47-72,
 * qwen_model.cpp:28-52).  dtype TI_DTYPE_BF16 for every tensor; for the
 * linear weights of a TI_WFMT_Q4_0 / Q8_0 engine, TI_DTYPE_Q4_0 / Q8_0 GGUF
 * blocks (row-major, K/32 blocks per row) are accepted as well.  Under tensor
 * parallelism the full tensor is passed and the engine keeps its shard. */
ti_status ti_engine_load_tensor(ti_engine* e, const char* name, int dtype, const void* host_data, size_t bytes);
/* ---- GGUF model files: the second weight format the reference plans behind
 * parser::WeightMap (include/tensor/parser/weight_map.hpp:24, "GGUF support
 * comes next"; WeightMap::open auto-detects .gguf, :31-33).  ti_gguf_open maps a
 * GGUF v2/v3 file read-only; its handle lists the tensors (llama.cpp names,
 * ggml types, ne[0] innermost), typed metadata and the model description, and
 * ti_engine_load_gguf uploads every model tensor under the reference's name
 * (q/k rows of llama-architecture files put back in the reference's RoPE
 * order; gemma norm weights stored as 1 + w put back to w; tensors of the
 * engine's block type passed as blocks, all others converted to bf16: f32,
 * f16, bf16, Q4_0, Q4_1, Q5_0, Q5_1, Q8_0 and the k-quants Q2_K .. Q6_K). */
enum { TI_GGML_F32 = 0, TI_GGML_F16 = 1, TI_GGML_Q4_0 = 2, TI_GGML_Q4_1 = 3, TI_GGML_Q5_0 = 6, TI_GGML_Q5_1 = 7,
       TI_GGML_Q8_0 = 8, TI_GGML_Q2_K = 10, TI_GGML_Q3_K = 11, TI_GGML_Q4_K = 12, TI_GGML_Q5_K = 13,
       TI_GGML_Q6_K = 14, TI_GGML_BF16 = 30 };
typedef struct ti_gguf ti_gguf;
ti_status ti_gguf_open(const char* path, ti_gguf** out);
ti_status ti_gguf_close(ti_gguf* g);
ti_status ti_gguf_tensor_count(const ti_gguf* g, int* n);
/* tensor i: name, ggml type, dims (ne[0..3], unused = 1), data in the mapping
 * and its bytes (0 for ggml types this reader does not decode) */
ti_status ti_gguf_tensor_info(const ti_gguf* g, int i, const char** name, int* ggml_type, int* n_dims,
                              int64_t* dims, const void** data, size_t* bytes);
ti_status ti_gguf_find(const ti_gguf* g, const char* name, int* index);
/* metadata by key: integers and bools, numbers (integers widen), strings, array lengths */
ti_status ti_gguf_meta_int(const ti_gguf* g, const char* key, int64_t* v);
ti_status ti_gguf_meta_float(const ti_gguf* g, const char* key, double* v);
ti_status ti_gguf_meta_string(const ti_gguf* g, const char* key, const char** v);
ti_status ti_gguf_meta_array_len(const ti_gguf* g, const char* key, int64_t* n);
/* Element i of array metadata (tokenizer.ggml.tokens / scores / token_type and the
 * like): a string as bytes and length (not NUL-terminated; valid while the file
 * is open), an integer of any integer or bool element type, or a float of f32 /
 * f64 elements.  TI_ERR_INVALID for another element type or an index out of range. */
ti_status ti_gguf_meta_array_string(const ti_gguf* g, const char* key, int64_t i, const char** str, size_t* len);
ti_status ti_gguf_meta_array_int(const ti_gguf* g, const char* key, int64_t i, int64_t* value);
ti_status ti_gguf_meta_array_float(const ti_gguf* g, const char* key, int64_t i, double* value);
/* architecture llama / qwen2 / gemma from "{arch}.*" metadata (block_count,
 * embedding_length, feed_forward_length, attention.head_count[_kv],
 * attention.key_length, attention.layer_norm_rms_epsilon, rope.freq_base);
 * vocab from token_embd.weight; weight_format from blk.0.attn_q.weight */
ti_status ti_gguf_model_desc(const ti_gguf* g, ti_model_desc* desc);
/* the reference's name of tensor i ("model.layers.3.self_attn.q_proj.weight"),
 * TI_ERR_NOT_FOUND for tensors the models do not read */
ti_status ti_gguf_reference_name(const ti_gguf* g, int i, char* buf, size_t cap);
/* tensor i as the engine receives it (rows in the reference's order): dtype
 * TI_DTYPE_BF16 (any supported ggml type, converted) or TI_DTYPE_Q4_0 / Q8_0
 * (the tensor's own blocks) */
ti_status ti_gguf_read(const ti_gguf* g, int i, int dtype, void* out, size_t bytes);
/* upload every model tensor of the file (tied embeddings: token_embd also as
 * lm_head.weight); *n_loaded (may be NULL) counts the uploads */
ti_status ti_engine_load_gguf(ti_engine* e, const ti_gguf* g, int* n_loaded);
/* the RoPE inverse frequencies of the file: theta^(-2i/head_dim) from
 * "{arch}.rope.freq_base", divided by the per-dimension factors of
 * rope_freqs.weight when the file has them (ti_engine_load_gguf applies them) */
ti_status ti_gguf_rope_inv_freq(const ti_gguf* g, float* out, int n);
/* replace the engine's RoPE inverse-frequency table (head_dim / 2 values; the
 * reference computes it from rope_theta and llama3 scaling, ops.cu:235-278) */
ti_status ti_engine_set_rope_freqs(ti_engine* e, const float* inv_freq, int n);

/* Fill every weight on the device with the synthetic generator
 * (element i of tensor `name` = f(seed, FNV-1a(name), i) ~ N(0, std)). */
ti_status ti_engine_init_synthetic(ti_engine* e, uint64_t seed, float std_);
/* Read back one weight (bf16, full tensor for TP rank 0 layouts) — tests. */
ti_status ti_engine_read_tensor(ti_engine* e, const char* name, void* host_out, size_t bytes);

/* sequences: replaces KVCache construction / clear (kv_cache.cpp:5-21, kv_cache.hpp:46-47) */
ti_status ti_seq_create(ti_engine* e, int* seq_id);
ti_status ti_seq_free(ti_engine* e, int seq_id);
ti_status ti_seq_reset(ti_engine* e, int seq_id);
ti_status ti_seq_len(ti_engine* e, int seq_id, int* len);

/* Samplers: replaces GenerateOptions::sampler (include/tensor/inference/
 * generator.hpp:22-38) and the host samplers it visits (greedy.cpp:11-36,
 * top_p.cpp:56-134), run on the device where the LM head leaves the logits.
 * Greedy ids are the LM head's fused argmax; top-p / top-k rows are sampled
 * from the step's bf16 logits by an exact integer-weight form of the reference's
 * algorithm (tokens by logit descending, equal logits by ascending id).
 * Draws: std::uniform_real_distribution<float>(0, 1) over std::mt19937_64 as
 * the reference; a top-p sequence owns one engine seeded when its sampler is
 * set, advanced once per sampled id (the reference's engine is thread_local,
 * top_p.cpp:84); top-k builds a fresh engine from the seed at every draw
 * (top_p.cpp:124).  seeded = 0 seeds from std::random_device. */
enum { TI_SAMPLE_GREEDY = 0, TI_SAMPLE_TOP_P = 1, TI_SAMPLE_TOP_K = 2 };
typedef struct ti_sampling {
    int      kind;         /* TI_SAMPLE_* */
    float    temperature;  /* logits / temperature when != 1 and > 0 (TopP / TopK::temperature) */
    float    p;            /* top-p: nucleus mass, finite (TopP::p) */
    uint32_t k;            /* top-k: candidates, >= 1 (TopK::k) */
    int      seeded;       /* 1: `seed` (TopP / TopK::seed); 0: std::random_device */
    uint64_t seed;
} ti_sampling;
/* The sampler of the ids ti_engine_decode / ti_engine_prefill(_chunked) return
 * for this sequence from now on; NULL or TI_SAMPLE_GREEDY restores greedy.
 * Under tensor parallelism every rank sets the same seeded sampler (ranks then
 * draw identical ids).  A bound device chain (ti_engine_bind) samples too (under
 * tensor parallelism its graph all-gathers the logits before the sampler): bind
 * draws every step the sequence's reserved pages allow ahead, from a
 * copy of its engine, and ti_engine_unbind advances the engine past the steps
 * taken, so the ids equal those of step-by-step decoding.  ti_seq_create starts
 * greedy; ti_seq_reset keeps the sampler. */
ti_status ti_engine_seq_set_sampler(ti_engine* e, int seq_id, const ti_sampling* s);
/* The same device sampler on caller-owned rows: logits [rows, vocab] bf16 and
 * out [rows] int32 in device memory; params and draws (uniform in [0, 1)) are
 * host arrays of `rows` entries (seed fields unused).  Greedy rows take the
 * lowest id of the largest logit.  Synchronises `stream` before returning. */
ti_status ti_op_sample(const void* logits, int rows, int vocab, const ti_sampling* params, const float* draws,
                       int32_t* out, void* stream);
/* The first n uniform draws a sequence with sampler `s` uses (host only, no
 * device): what ti_engine_seq_set_sampler's per-sequence engine produces. */
ti_status ti_sampler_draws(const ti_sampling* s, int n, float* out);
/* pre-allocate pages so the sequence can grow to n_tokens without host work */
ti_status ti_seq_reserve(ti_engine* e, int seq_id, int n_tokens);
/* Give a sequence n_tokens of synthetic cached context (pages allocated, K/V
 * of every layer filled from the seeded generator, length set) without running
 * them through the model: benchmarks of long-context decode.  No counterpart in
 * the reference. */
ti_status ti_seq_fill_synthetic(ti_engine* e, int seq_id, int n_tokens, uint64_t seed, float std_);
/* copy K or V (which = 0/1) of one layer for positions [0, len) into host memory
 * as [len, n_kv_local, head_dim] bf16 (tests) */
ti_status ti_seq_read_kv(ti_engine* e, int seq_id, int layer, int which, void* host_out, int len);

enum { TI_LOGITS_NONE = 0, TI_LOGITS_BF16 = 1, TI_LOGITS_F32 = 2 };

/* Run the prompt `ids[0..n)` through sequence `seq_id` (Model::forward with
 * seq_len = n, llama_model.cpp:210).  Writes the greedy next id (argmax of the
 * fp32 logits of the last row, lowest index on ties) to *next_id (host) and,
 * if logits_out != NULL, the last row's logits (host, format logits_mode). */
ti_status ti_engine_prefill(ti_engine* e, int seq_id, const int32_t* ids, int n, int adapter_id,
                            int32_t* next_id, int logits_mode, void* logits_out);

/* Prefill in steps of up to `chunk` tokens (<= max_batch): each step decodes
 * tokens len .. len + m - 1 of the sequence together (the tcgen05 path for 8+
 * tokens; every K/V row of the step is written to its page before attention,
 * each token attends causally up to its own position).  next_id / logits: the
 * last prompt token's.  No counterpart in the reference, whose prefill is one
 * forward over the prompt with a host-built causal mask (ops.cu:500-520). */
ti_status ti_engine_prefill_chunked(ti_engine* e, int seq_id, const int32_t* ids, int n, int adapter_id, int chunk,
                                    int32_t* next_id, int logits_mode, void* logits_out);
/* One decode step for `batch` sequences (Model::forward with one token each,
 * generator.cpp:78; Greedy::sample, greedy.cpp:11-36, becomes a device argmax).
 * Host pointers: tokens[batch], seq_ids[batch], adapter_ids[batch] (NULL = no
 * adapter; -1 entries = none), next_ids[batch] out.  logits_out (host,
 * [batch, vocab] in logits_mode) may be NULL.  Synchronous on `stream`. */
ti_status ti_engine_decode(ti_engine* e, int batch, const int32_t* seq_ids, const int32_t* tokens,
                           const int32_t* adapter_ids, int32_t* next_ids, int logits_mode, void* logits_out,
                           void* stream);

/* Device-resident chained decode: bind `batch` sequences once, then every
 * ti_engine_decode_device call runs one step whose input tokens are the
 * previous step's ids (greedy, or drawn by the sequence's sampler), all on the
 * device (no host synchronisation).  Sequences must have pages reserved
 * (ti_seq_reserve) for the steps run.  `stream` is a stream of the engine's
 * device, whatever device is current for the caller (0: that device's default
 * stream, the one ti_engine_unbind with stream 0 reads the ids on). */
ti_status ti_engine_bind(ti_engine* e, int batch, const int32_t* seq_ids, const int32_t* first_tokens,
                         const int32_t* adapter_ids);
ti_status ti_engine_decode_device(ti_engine* e, void* stream);
/* after a chain of device steps: read the last greedy ids (host) and commit
 * the number of steps run to the sequences' lengths */
ti_status ti_engine_unbind(ti_engine* e, int steps_run, int32_t* last_ids, void* stream);
/* device pointer to the [batch, vocab] bf16 logits of the last step */
ti_status ti_engine_logits_device(ti_engine* e, void** ptr);
/* 0 if no bounded device wait has timed out since the last call, else TI_ERR_TIMEOUT */
ti_status ti_engine_check(ti_engine* e);
/* Diagnostic: launch ONE kernel of a decode step alone on `stream`, with the
 * buffers of the last step (kind: 0 embed, 1 qkv GEMV, 2 attention, 3 o GEMV,
 * 4 gate|up GEMV, 5 down GEMV, 6 LM head; layer ignored for 0 and 6).  Used to
 * time and profile single kernels; no reference counterpart. */
enum { TI_KERNEL_EMBED = 0, TI_KERNEL_QKV = 1, TI_KERNEL_ATTN = 2, TI_KERNEL_O = 3, TI_KERNEL_GATEUP = 4,
       TI_KERNEL_DOWN = 5, TI_KERNEL_LMHEAD = 6 };
ti_status ti_engine_launch_kernel(ti_engine* e, int kind, int layer, int batch, void* stream);
/* kernels launched per decode step at this batch size (for launch accounting) */
ti_status ti_engine_launches_per_step(ti_engine* e, int batch, int* launches);

/* ================================================================= LoRA adapters
 * replaces AdapterLoader / AdapterWeights (src/adapter/adapter_loader.cpp:132-236,
 * include/tensor/adapter/adapter_weights.hpp:22-88) and apply_lora
 * (qwen_adapter_model.cpp:22-43): delta = bf16(bf16(bf16(x A^T) B^T) * alpha/rank). */
ti_status ti_adapter_create(ti_engine* e, int rank, float alpha, int proj_mask, int* adapter_id);
/* names as the adapter checkpoint: "layers.{i}.self_attn.q_proj.lora_A" (A [rank, in]),
 * "...lora_B" (B [out, rank]); 1-D flat tensors are accepted (adapter_loader.cpp:67-95). */
ti_status ti_adapter_load_tensor(ti_engine* e, int adapter_id, const char* name, const void* host_bf16,
                                 size_t bytes);
ti_status ti_adapter_init_synthetic(ti_engine* e, int adapter_id, uint64_t seed, float std_a, float std_b);
/* Async pinned host -> HBM fetch on the engine's side stream: the adapter's
 * weights are staged in pinned host memory (ti_adapter_stage_host) and copied
 * into a resident slot; decode steps that use it wait on the copy's event. */
ti_status ti_adapter_stage_host(ti_engine* e, int adapter_id);
ti_status ti_adapter_evict(ti_engine* e, int adapter_id);
ti_status ti_adapter_prefetch_async(ti_engine* e, int adapter_id);
ti_status ti_adapter_is_resident(ti_engine* e, int adapter_id, int* resident);

/* ================================================================= PKM router
 * Spec only in the reference (README.md:58-72,157-180): two codebooks of
 * n_codes x half_dim fp32; a query [2*half_dim] is split in halves, each half
 * takes the argmin squared-L2 code (canonical fp32 order: d = q-c,
 * acc = fma(d, d, acc) over t = 0..half_dim-1; lowest index on ties);
 * address = i * n_codes + j; adapter = registry[address] or -1. */
typedef struct ti_pkm ti_pkm;
ti_status ti_pkm_create(int device, int n_codes, int half_dim, const float* c1_host, const float* c2_host,
                        ti_pkm** out);
ti_status ti_pkm_destroy(ti_pkm* p);
/* register adapters by centroid ([n, 2*half_dim] host fp32); collisions keep the lowest id */
ti_status ti_pkm_register(ti_pkm* p, const float* centroids_host, const int32_t* adapter_ids, int n);
/* device pointers: queries [n, 2*half_dim] fp32 -> addr[n], adapter[n] int32 */
ti_status ti_pkm_query(ti_pkm* p, const float* queries, int n, int32_t* addr, int32_t* adapter, void* stream);
/* same with host buffers (copies inside, synchronous) */
ti_status ti_pkm_query_host(ti_pkm* p, const float* queries, int n, int32_t* addr, int32_t* adapter);

/* ================================================================= router pool + scheduler
 * Spec only in the reference (README.md:170-180: router/pool keeps a VRAM budget
 * of resident adapters with LRU eviction and async prefetch of a candidate;
 * router/scheduler switches adapters only once a semantic shift is decisive).
 * Per sequence, ti_router_observe takes the adapter the PKM router names for its
 * latest token (ti_pkm_query; -1 = base model): a new candidate is prefetched
 * after leading prefetch_after consecutive tokens and becomes the sequence's
 * adapter after switch_after (its first observation is taken at once).
 * ti_router_prepare makes a step's adapters resident (async copies the step
 * waits on), evicting least recently used adapters outside the step past
 * max_resident (speculative prefetches never evict a live sequence's adapter).
 * Eviction stages a host copy first (once).  A NULL engine records decisions
 * only (ti_router_actions: (kind, adapter) pairs, 1 = prefetch, 2 = evict). */
typedef struct ti_router ti_router;
typedef struct {
    int max_resident;    /* adapters resident in HBM at once (>= 1) */
    int prefetch_after;  /* tokens a candidate leads before its async prefetch (>= 1) */
    int switch_after;    /* tokens before the sequence switches (>= prefetch_after) */
} ti_router_opts;
typedef struct {
    int64_t observations, switches, prefetches, evictions, hits;
} ti_router_stats;
ti_status ti_router_create(ti_engine* e, const ti_router_opts* opts, ti_router** out);
ti_status ti_router_destroy(ti_router* r);
ti_status ti_router_observe(ti_router* r, int seq, int candidate, int* use_adapter);
ti_status ti_router_prepare(ti_router* r, const int32_t* adapters, int n);
ti_status ti_router_forget(ti_router* r, int seq);
ti_status ti_router_stats_get(const ti_router* r, ti_router_stats* out);
/* decisions since the last call (removed from the log); *n pairs written */
ti_status ti_router_actions(ti_router* r, int32_t* out, int cap, int* n);
/* adapters the router holds resident, most recently used first; *n = their count */
ti_status ti_router_resident(const ti_router* r, int32_t* out, int cap, int* n);

#ifdef __cplusplus
}
#endif
#endif /* TI_B200_H */
