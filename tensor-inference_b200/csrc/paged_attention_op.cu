// paged_attention_op.cu — the paged decode-attention kernel as a stand-alone op.
//
// One call does, for one layer and `batch` new tokens, what the reference's
// model code does with ops::rope x2, a raw cudaMemcpy into the KV cache,
// ops::slice x2 and ops::attention (llama_model.cpp:147-182).  The split-KV
// merge needs scratch memory (per-split partial outputs and completion
// counters); this entry takes it from the device's stream-ordered pool.
#include <algorithm>
#include <mutex>

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
    a.n_splits = attn_splits(batch, n_kv, head_dim, max_len, sms, &a.max_chunk);
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

// ----------------------------------------------------------------------------
// Allocation-free variant.
//
// Some callers cannot allocate device memory at the point where they run this
// op: a plugin whose host application owns the whole device-memory budget and
// forbids allocation inside its execute call, or a process whose memory is
// fully reserved up front by another framework's caching allocator, so any
// cudaMalloc (or pool growth) would fail or stall.  For them this entry takes
// its scratch (split partials, merge counters, the RoPE table) from the
// fixed-size array below instead of the memory pool.
//
// The array is a file-scope __device__ variable: every GPU that loads this
// library holds kNoAllocScratchBytes of it until the process exits.  Host code
// cannot use the symbol as a device address, so the address is looked up once
// per device with cudaGetSymbolAddress, with that device current, on the first
// call made on that device; make that first call before any stream capture.
// All calls share the one array and it keeps the last call's contents, so
// calls that overlap on the GPU (different streams, or different host threads
// without ordering) race on it; order them on one stream.  The cached address
// belongs to the device's current CUDA context: a caller that destroys that
// context (cudaDeviceReset) must not call this entry on that device afterwards.
constexpr size_t kNoAllocScratchBytes = 8u << 20;  // 8 MiB per device
static __device__ __align__(256) unsigned char g_paged_attn_scratch[kNoAllocScratchBytes];

namespace {

// The RoPE frequency table travels as a kernel argument (copied by value at
// launch), so no host buffer has to outlive the call.
struct FreqTable {
    float f[128];
};

__global__ void k_store_freqs(FreqTable t, float* dst, int n) {
    if ((int)threadIdx.x < n) dst[threadIdx.x] = t.f[threadIdx.x];
}

std::mutex g_scratch_mu;
void* g_scratch_addr[64] = {};

ti_status scratch_address(int dev, void** out) {
    TI_CHECK(dev >= 0 && dev < 64, TI_ERR_UNSUPPORTED, "paged_attention_noalloc: device index %d >= 64", dev);
    std::lock_guard<std::mutex> lk(g_scratch_mu);
    if (!g_scratch_addr[dev]) {
        void* p = nullptr;
        const cudaError_t e = cudaGetSymbolAddress(&p, g_paged_attn_scratch);
        TI_CHECK(e == cudaSuccess && p, TI_ERR_CUDA, "paged_attention_noalloc: cudaGetSymbolAddress: %s",
                 cudaGetErrorString(e));
        g_scratch_addr[dev] = p;
    }
    *out = g_scratch_addr[dev];
    return TI_OK;
}

}  // namespace

extern "C" ti_status ti_op_paged_attention_noalloc(const void* qkv, int batch, int n_heads, int n_kv, int head_dim,
                                                   const int32_t* pos, const int32_t* seq,
                                                   const int32_t* page_table, int pt_stride, void* k_pages,
                                                   void* v_pages, int n_pages, int max_len, float theta,
                                                   const ti_rope_scaling* scaling, int sliding_window, void* out,
                                                   void* stream) {
    if (ti_status st = check_paged_args(qkv, batch, n_heads, n_kv, head_dim, pos, seq, page_table, pt_stride, k_pages,
                                        v_pages, n_pages, max_len, out))
        return st;
    int dev = 0;
    TI_CUDA(cudaGetDevice(&dev));
    void* base = nullptr;
    if (ti_status st = scratch_address(dev, &base)) return st;

    AttnArgs a = make_args(qkv, batch, n_heads, n_kv, head_dim, pos, seq, page_table, pt_stride, k_pages, v_pages,
                           n_pages, max_len, nullptr, sliding_window, out, num_sms(dev));
    // scratch layout: [rope table][merge counters][split partials], 256-byte aligned parts
    const size_t freq_bytes = ((size_t)head_dim / 2 * 4 + 255) & ~size_t(255);
    const size_t nctr = (size_t)batch * n_kv;
    const size_t ctr_bytes = (nctr * 4 + 255) & ~size_t(255);
    const size_t part_bytes = attn_scratch_floats(batch, n_heads, n_kv, head_dim, a.n_splits) * 4;
    const size_t need = freq_bytes + ctr_bytes + part_bytes;
    TI_CHECK(need <= kNoAllocScratchBytes, TI_ERR_INVALID,
             "paged_attention_noalloc: needs %zu scratch bytes for batch %d, %d kv heads, max_len %d; the fixed "
             "scratch holds %zu (use ti_op_paged_attention)",
             need, batch, n_kv, max_len, kNoAllocScratchBytes);

    uint8_t* p = reinterpret_cast<uint8_t*>(base);
    float* freqs = reinterpret_cast<float*>(p);
    unsigned int* counters = reinterpret_cast<unsigned int*>(p + freq_bytes);
    float* parts = reinterpret_cast<float*>(p + freq_bytes + ctr_bytes);
    const size_t G = (size_t)(n_heads / n_kv);
    a.freqs = freqs;
    a.counters = counters;
    a.part_o = parts;
    a.part_ml = parts + (size_t)batch * n_kv * a.n_splits * G * head_dim;
    a.err = nullptr;

    cudaStream_t s = (cudaStream_t)stream;
    // the same host-computed table as the pool-backed entry (ops.cu:235-278),
    // written into the scratch by a one-warp-pair kernel that carries it by value
    FreqTable t;
    rope_freqs(head_dim, theta, scaling, t.f);
    k_store_freqs<<<1, 128, 0, s>>>(t, freqs, head_dim / 2);
    TI_CUDA(cudaGetLastError());
    // the merge counters must start at zero whatever the previous call left
    TI_CUDA(cudaMemsetAsync(counters, 0, nctr * 4, s));
    TI_CUDA(attn_launch(a, s, false));
    return TI_OK;
}
