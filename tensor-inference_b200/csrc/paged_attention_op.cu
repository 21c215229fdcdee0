// paged_attention_op.cu — the paged decode-attention kernel as a stand-alone op.
//
// One call does, for one layer and `batch` new tokens, what the reference's
// model code does with ops::rope x2, a raw cudaMemcpy into the KV cache,
// ops::slice x2 and ops::attention (llama_model.cpp:147-182).  The split-KV
// merge needs scratch memory (per-split partial outputs and completion
// counters); this entry takes it from the device's stream-ordered pool.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"

using namespace ti;

namespace {

ti_status check_paged_args(const void* qkv, int batch, int n_heads, int n_kv, int head_dim, const int32_t* pos,
                           const int32_t* seq, const int32_t* page_table, int pt_stride, void* k_pages, void* v_pages,
                           int n_pages, int max_len, void* out) {
    TI_CHECK(qkv && pos && seq && page_table && k_pages && v_pages && out, TI_ERR_INVALID,
             "paged_attention: null argument");
    TI_CHECK(batch >= 1 && n_heads >= 1 && n_kv >= 1 && n_heads % n_kv == 0, TI_ERR_INVALID,
             "paged_attention: bad head counts");
    TI_CHECK(n_heads / n_kv <= 16, TI_ERR_UNSUPPORTED, "paged_attention: GQA group > 16");
    TI_CHECK(head_dim == 64 || head_dim == 128 || head_dim == 256, TI_ERR_UNSUPPORTED,
             "paged_attention: head_dim %d (64/128/256 supported)", head_dim);
    TI_CHECK(max_len >= 1 && pt_stride * 16 >= max_len && n_pages >= 1, TI_ERR_INVALID,
             "paged_attention: max_len %d exceeds the page table (%d pages per sequence)", max_len, pt_stride);
    return TI_OK;
}

AttnArgs make_args(const void* qkv, int batch, int n_heads, int n_kv, int head_dim, const int32_t* pos,
                   const int32_t* seq, const int32_t* page_table, int pt_stride, void* k_pages, void* v_pages,
                   int n_pages, int max_len, const float* freqs, int sliding_window, void* out, int sms) {
    AttnArgs a;
    a.qkv = reinterpret_cast<const uint16_t*>(qkv);
    a.qkv_stride = (n_heads + 2 * n_kv) * head_dim;
    a.nb = batch;
    a.nq = n_heads;
    a.nkv = n_kv;
    a.hd = head_dim;
    a.pos = pos;
    a.seq = seq;
    a.page_table = page_table;
    a.pt_stride = pt_stride;
    a.kc = reinterpret_cast<uint16_t*>(k_pages);
    a.vc = reinterpret_cast<uint16_t*>(v_pages);
    a.freqs = freqs;
    a.scale = 1.0f / sqrtf((float)head_dim);  // ops.cu:455
    a.window = nullptr;
    a.window_const = sliding_window;
    a.n_pages = n_pages;
    a.n_splits = attn_splits(batch, n_kv, max_len, sms, &a.max_chunk);
    a.out = reinterpret_cast<uint16_t*>(out);
    a.out_stride = n_heads * head_dim;
    return a;
}

}  // namespace

extern "C" ti_status ti_op_paged_attention(const void* qkv, int batch, int n_heads, int n_kv, int head_dim,
                                           const int32_t* pos, const int32_t* seq, const int32_t* page_table,
                                           int pt_stride, void* k_pages, void* v_pages, int n_pages, int max_len,
                                           float theta, const ti_rope_scaling* scaling, int sliding_window,
                                           void* out, void* stream) {
    if (ti_status st = check_paged_args(qkv, batch, n_heads, n_kv, head_dim, pos, seq, page_table, pt_stride, k_pages,
                                        v_pages, n_pages, max_len, out))
        return st;
    int dev = 0;
    TI_CUDA(cudaGetDevice(&dev));
    const float* freqs = rope_table(dev, head_dim, theta, scaling);
    TI_CHECK(freqs, TI_ERR_OOM, "paged_attention: rope table allocation failed");
    AttnArgs a = make_args(qkv, batch, n_heads, n_kv, head_dim, pos, seq, page_table, pt_stride, k_pages, v_pages,
                           n_pages, max_len, freqs, sliding_window, out, num_sms(dev));
    cudaStream_t s = (cudaStream_t)stream;
    const size_t nf = attn_scratch_floats(batch, n_heads, n_kv, head_dim, a.n_splits);
    const size_t nctr = (size_t)batch * n_kv;
    float* scratch = nullptr;
    TI_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&scratch), nf * 4 + nctr * 4 + 16, s));
    const size_t G = (size_t)(n_heads / n_kv);
    a.part_o = scratch;
    a.part_ml = scratch + (size_t)batch * n_kv * a.n_splits * G * head_dim;
    a.counters = reinterpret_cast<unsigned int*>(scratch + nf);
    a.err = nullptr;
    cudaError_t e = cudaMemsetAsync(a.counters, 0, nctr * 4, s);
    if (e == cudaSuccess) e = attn_launch(a, s, false);
    cudaError_t f = cudaFreeAsync(scratch, s);
    TI_CHECK(e == cudaSuccess, TI_ERR_CUDA, "paged_attention: %s", cudaGetErrorString(e));
    TI_CUDA(f);
    return TI_OK;
}
