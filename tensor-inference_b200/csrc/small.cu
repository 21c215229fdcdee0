// small.cu — launch helper, embedding gather, synthetic initialisers.
#include <algorithm>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"
#include "synth.cuh"

namespace ti {

cudaError_t launch_pdl(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args, bool pdl) {
    cudaLaunchConfig_t cfg = {};
    cfg.gridDim = grid;
    cfg.blockDim = block;
    cfg.dynamicSmemBytes = smem;
    cfg.stream = s;
    cudaLaunchAttribute attr[1];
    attr[0].id = cudaLaunchAttributeProgrammaticStreamSerialization;
    attr[0].val.programmaticStreamSerializationAllowed = 1;
    cfg.attrs = attr;
    cfg.numAttrs = pdl ? 1 : 0;
    return cudaLaunchKernelExC(&cfg, func, args);
}

int num_sms(int device) {
    int n = 0;
    cudaDeviceGetAttribute(&n, cudaDevAttrMultiProcessorCount, device);
    return n > 0 ? n : 1;
}

// ops.cu:46-88 (row gather) + gemma_model.cpp:117 (times sqrt(hidden), bf16);
// first kernel of a step: also applies the step's page-table updates.
__global__ void k_embed(const EmbedArgs a) {
    if (threadIdx.x == 0) pdl_trigger();
    pdl_wait();
    if (blockIdx.x == 0 && a.n_updates) {
        const int nu = *a.n_updates;
        for (int i = threadIdx.x; i < nu; i += blockDim.x) {
            const int seq = a.pt_updates[3 * i], idx = a.pt_updates[3 * i + 1], page = a.pt_updates[3 * i + 2];
            a.page_table[(size_t)seq * a.pt_stride + idx] = page;
        }
    }
    if (blockIdx.x == 0 && threadIdx.x == 0 && a.epoch) *a.epoch += 1;
    const int b = blockIdx.x;
    int tok = a.tokens[b];
    if (tok < 0 || tok >= a.vocab) {
        if (threadIdx.x == 0 && a.err) atomicOr(a.err, kErrBadIndex);
        tok = 0;
    }
    const uint4* src = reinterpret_cast<const uint4*>(a.table + (size_t)tok * a.hidden);
    uint4* dst = reinterpret_cast<uint4*>(a.out + (size_t)b * a.hidden);
    for (int i = threadIdx.x; i < a.hidden / 8; i += blockDim.x) {
        uint4 v = src[i];
        if (a.scale != 0.f) {
            uint32_t* p = reinterpret_cast<uint32_t*>(&v);
#pragma unroll
            for (int e = 0; e < 4; ++e) p[e] = pack_bf2(bf_lo(p[e]) * a.scale, bf_hi(p[e]) * a.scale);
        }
        dst[i] = v;
    }
}

cudaError_t embed_launch(const EmbedArgs& a, cudaStream_t s, bool pdl) {
    if (a.hidden % 8) return cudaErrorInvalidValue;
    EmbedArgs args = a;
    void* params[] = {&args};
    return launch_pdl(reinterpret_cast<const void*>(&k_embed), dim3(a.nb), dim3(256), 0, s, params, pdl);
}

__global__ void k_synth_bf16(uint16_t* dst, size_t rows, size_t cols, size_t dst_ld, size_t r0, size_t c0,
                             size_t full_ld, uint64_t key, float c) {
    const size_t total = rows * cols;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const size_t r = i / cols, col = i - r * cols;
        const size_t gi = (r0 + r) * full_ld + c0 + col;
        const float v = __fmul_rn((float)synth_centered(key, gi), c);
        dst[r * dst_ld + col] = __bfloat16_as_ushort(__float2bfloat16_rn(v));
    }
}

__global__ void k_synth_f32(float* dst, size_t n, uint64_t key, float c) {
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < n; i += (size_t)gridDim.x * blockDim.x)
        dst[i] = __fmul_rn((float)synth_centered(key, i), c);
}

cudaError_t synth_bf16_launch(uint16_t* dst, size_t rows, size_t cols, size_t dst_ld, size_t r0, size_t c0,
                              size_t full_ld, uint64_t seed, uint64_t name_hash, float scale_c, cudaStream_t s) {
    if (rows == 0 || cols == 0) return cudaSuccess;
    const uint64_t key = mix64(seed ^ name_hash);
    k_synth_bf16<<<4 * 148, 256, 0, s>>>(dst, rows, cols, dst_ld, r0, c0, full_ld, key, scale_c);
    return cudaGetLastError();
}

cudaError_t synth_f32_launch(float* dst, size_t n, uint64_t seed, uint64_t name_hash, float scale_c, cudaStream_t s) {
    if (n == 0) return cudaSuccess;
    const uint64_t key = mix64(seed ^ name_hash);
    k_synth_f32<<<4 * 148, 256, 0, s>>>(dst, n, key, scale_c);
    return cudaGetLastError();
}


// ---- tensor-parallel glue
__global__ void k_tp_resid(const float* __restrict__ sum, const uint16_t* __restrict__ resid,
                           uint16_t* __restrict__ out, int n) {
    if (blockIdx.x == 0 && threadIdx.x == 0) pdl_trigger();
    pdl_wait();
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        const float r = __uint_as_float((uint32_t)resid[i] << 16);
        out[i] = __bfloat16_as_ushort(f2bf(r + round_bf(sum[i])));  // ops.cu:361-381 on the bf16 projection
    }
}

cudaError_t tp_resid_launch(const float* sum, const uint16_t* resid, uint16_t* out, int nb, int H, cudaStream_t s,
                            bool pdl) {
    int n = nb * H;
    void* params[] = {&sum, &resid, &out, &n};
    const int grid = std::min((n + 255) / 256, 1024);
    return launch_pdl(reinterpret_cast<const void*>(&k_tp_resid), dim3(grid), dim3(256), 0, s, params, pdl);
}

__global__ void k_tp_ids(unsigned long long* amax, int nb, int32_t* out_ids, int32_t* chain_tokens,
                         int32_t* chain_pos) {
    if (threadIdx.x == 0) pdl_trigger();
    pdl_wait();
    for (int b = threadIdx.x; b < nb; b += blockDim.x) {
        const unsigned long long key = amax[b];
        amax[b] = 0ull;
        const int32_t id = (int32_t)(~(uint32_t)(key & 0xffffffffull));
        out_ids[b] = id;
        if (chain_tokens) chain_tokens[b] = id;
        if (chain_pos) chain_pos[b] += 1;
    }
}

cudaError_t tp_ids_launch(unsigned long long* amax, int nb, int32_t* out_ids, int32_t* chain_tokens,
                          int32_t* chain_pos, cudaStream_t s, bool pdl) {
    void* params[] = {&amax, &nb, &out_ids, &chain_tokens, &chain_pos};
    return launch_pdl(reinterpret_cast<const void*>(&k_tp_ids), dim3(1), dim3(256), 0, s, params, pdl);
}


// ---- tensor-parallel all-reduce through peer memory (receive side)
struct RecvLora {
    GemvLora L;                 // adapter ids, B rows [out][R] of adapter 0, strides, rank R, scales
    const float* t_inbox = nullptr;
    size_t t_src_stride = 0;    // floats between senders' blocks
};

__global__ void k_tp_recv_resid(const float* __restrict__ inbox, size_t src_stride, const unsigned int* flags, int tp,
                                const int* epoch, int seq_mul, int seq_add, const uint16_t* __restrict__ resid,
                                uint16_t* __restrict__ out, int n, int* err) {
    __shared__ int ok;
    if (blockIdx.x == 0 && threadIdx.x == 0) pdl_trigger();
    pdl_wait();
    if (threadIdx.x == 0) {
        const unsigned int seq = peer_seq(*epoch, seq_mul, seq_add);
        bool good = true;
        for (int r = 0; r < tp && good; ++r) good = wait_seq_sys(flags + r, seq, err, kErrTimeoutPeer);
        ok = good;
    }
    __syncthreads();
    if (!ok) return;
    for (int i = blockIdx.x * blockDim.x + threadIdx.x; i < n; i += gridDim.x * blockDim.x) {
        float sum = 0.f;
        for (int r = 0; r < tp; ++r) sum += __ldcv(inbox + (size_t)r * src_stride + i);  // rank order
        const float rr = __uint_as_float((uint32_t)resid[i] << 16);
        out[i] = __bfloat16_as_ushort(f2bf(rr + round_bf(sum)));
    }
}

// With LoRA on the row-parallel projection the expansion runs here, on the full
// x.A^T (the rank-ordered sum of every rank's partial): CTA (row tile, token b),
// eight lanes per output row, each reading 16 contiguous bytes of the B row, so a
// warp reads four whole B rows per load (coalesced) and the eight partial sums
// meet in a 3-step shuffle.
constexpr int kRecvLoraRows = 128;

__global__ void __launch_bounds__(256)
    k_tp_recv_resid_lora(const float* __restrict__ inbox, size_t src_stride, const unsigned int* flags, int tp,
                         const int* epoch, int seq_mul, int seq_add, const uint16_t* __restrict__ resid,
                         uint16_t* __restrict__ out, int H, const RecvLora rl, int* err) {
    __shared__ int ok;
    __shared__ __align__(16) float tfull[256];  // this token's x.A^T rounded to bf16 (rank <= 256)
    if (blockIdx.x == 0 && blockIdx.y == 0 && threadIdx.x == 0) pdl_trigger();
    const int b = blockIdx.y, tid = threadIdx.x;
    pdl_wait();
    if (tid == 0) {
        const unsigned int seq = peer_seq(*epoch, seq_mul, seq_add);
        bool good = true;
        for (int r = 0; r < tp && good; ++r) good = wait_seq_sys(flags + r, seq, err, kErrTimeoutPeer);
        ok = good;
    }
    const int R = rl.L.rank;
    const int ad = rl.L.adapter[b];
    const bool has = ad >= 0 && ad < rl.L.n_adapters;
    __syncthreads();
    if (!ok) return;
    if (has) {
        for (int j = tid; j < R; j += blockDim.x) {
            float t = 0.f;
            for (int r = 0; r < tp; ++r) t += __ldcv(rl.t_inbox + (size_t)r * rl.t_src_stride + (size_t)b * R + j);
            tfull[j] = round_bf(t);  // the shrink output x.A^T (qwen_adapter_model.cpp:27)
        }
        __syncthreads();
    }
    const int sub = tid & 7;
    const float scale = has ? rl.L.scale[ad] : 0.f;
    const uint16_t* B = has ? rl.L.B + (size_t)ad * rl.L.B_adapter_stride : nullptr;
    const int r_end = min(H, (int)(blockIdx.x + 1) * kRecvLoraRows);
    for (int r0 = blockIdx.x * kRecvLoraRows; r0 < r_end; r0 += 32) {  // uniform trip count: whole warps shuffle
        const int row = r0 + (tid >> 3);
        const bool live = row < r_end;
        float s = 0.f;
        if (has && live) {
            const uint16_t* br = B + (size_t)row * R;
            for (int k0 = sub * 8; k0 < R; k0 += 64) {
                const uint4 w = *reinterpret_cast<const uint4*>(br + k0);
                const uint32_t* wp = reinterpret_cast<const uint32_t*>(&w);
                const float4 t0 = *reinterpret_cast<const float4*>(tfull + k0);
                const float4 t1 = *reinterpret_cast<const float4*>(tfull + k0 + 4);
                s = fmaf(bf_lo(wp[0]), t0.x, s);
                s = fmaf(bf_hi(wp[0]), t0.y, s);
                s = fmaf(bf_lo(wp[1]), t0.z, s);
                s = fmaf(bf_hi(wp[1]), t0.w, s);
                s = fmaf(bf_lo(wp[2]), t1.x, s);
                s = fmaf(bf_hi(wp[2]), t1.y, s);
                s = fmaf(bf_lo(wp[3]), t1.z, s);
                s = fmaf(bf_hi(wp[3]), t1.w, s);
            }
        }
        s += __shfl_xor_sync(0xffffffffu, s, 4);
        s += __shfl_xor_sync(0xffffffffu, s, 2);
        s += __shfl_xor_sync(0xffffffffu, s, 1);
        if (sub == 0 && live) {
            const size_t i = (size_t)b * H + row;
            float sum = 0.f;
            for (int r = 0; r < tp; ++r) sum += __ldcv(inbox + (size_t)r * src_stride + i);  // rank order
            float v = round_bf(sum);
            if (has) v = round_bf(v + round_bf(round_bf(s) * scale));  // qwen_adapter_model.cpp:28-29, :42
            const float rr = __uint_as_float((uint32_t)resid[i] << 16);
            out[i] = __bfloat16_as_ushort(f2bf(rr + v));
        }
    }
}

cudaError_t tp_recv_resid_launch(const float* inbox, size_t src_stride, const unsigned int* flags, int tp,
                                 const int* epoch, int seq_mul, int seq_add, const uint16_t* resid, uint16_t* out,
                                 int nb, int H, const GemvLora* lora, const float* t_inbox, size_t t_src_stride,
                                 int* err, cudaStream_t s, bool pdl) {
    if (lora && lora->adapter) {
        if (lora->rank % 8 != 0 || lora->rank > 256) return cudaErrorInvalidValue;
        RecvLora rl;
        rl.L = *lora;
        rl.t_inbox = t_inbox;
        rl.t_src_stride = t_src_stride;
        void* params[] = {&inbox, &src_stride, &flags, &tp, &epoch, &seq_mul, &seq_add, &resid, &out, &H, &rl, &err};
        return launch_pdl(reinterpret_cast<const void*>(&k_tp_recv_resid_lora),
                          dim3((H + kRecvLoraRows - 1) / kRecvLoraRows, nb), dim3(256), 0, s, params, pdl);
    }
    int n = nb * H;
    void* params[] = {&inbox, &src_stride, &flags, &tp, &epoch, &seq_mul, &seq_add, &resid, &out, &n, &err};
    const int grid = std::min((n + 255) / 256, 148);
    return launch_pdl(reinterpret_cast<const void*>(&k_tp_recv_resid), dim3(grid), dim3(256), 0, s, params, pdl);
}

struct KeysArgs {
    unsigned long long* amax;
    int nb, tp, rank, max_nb;
    unsigned long long* peer_keys[kMaxTp];  // rank r's keys inbox [tp][max_nb]
    unsigned int* peer_flags[kMaxTp];       // rank r's flags [tp]
    const unsigned long long* keys_inbox;   // this rank's inbox
    const unsigned int* flags;              // this rank's flags
    const int* epoch;
    int32_t *out_ids, *chain_tokens, *chain_pos;
    int* err;
};

__global__ void k_tp_keys(const KeysArgs a) {
    __shared__ int ok;
    if (threadIdx.x == 0) pdl_trigger();
    pdl_wait();
    const unsigned int seq = (unsigned int)*a.epoch;
    for (int b = threadIdx.x; b < a.nb; b += blockDim.x) {
        const unsigned long long key = a.amax[b];
        a.amax[b] = 0ull;
        for (int r = 0; r < a.tp; ++r) a.peer_keys[r][(size_t)a.rank * a.max_nb + b] = key;
    }
    __threadfence_system();
    __syncthreads();
    if (threadIdx.x == 0) {
        __threadfence_system();
        for (int r = 0; r < a.tp; ++r) st_release_sys(a.peer_flags[r] + a.rank, seq);
        bool good = true;
        for (int r = 0; r < a.tp && good; ++r) good = wait_seq_sys(a.flags + r, seq, a.err, kErrTimeoutPeer);
        ok = good;
    }
    __syncthreads();
    if (!ok) return;
    for (int b = threadIdx.x; b < a.nb; b += blockDim.x) {
        unsigned long long best = 0ull;
        for (int r = 0; r < a.tp; ++r) {
            const unsigned long long k = __ldcv(a.keys_inbox + (size_t)r * a.max_nb + b);
            best = k > best ? k : best;
        }
        const int32_t id = (int32_t)(~(uint32_t)(best & 0xffffffffull));
        a.out_ids[b] = id;
        if (a.chain_tokens) a.chain_tokens[b] = id;
        if (a.chain_pos) a.chain_pos[b] += 1;
    }
}

cudaError_t tp_keys_launch(unsigned long long* amax, int nb, unsigned long long* const* peer_keys,
                           unsigned int* const* peer_flags, int tp, int rank, const unsigned long long* keys_inbox,
                           const unsigned int* flags, int max_nb, const int* epoch, int32_t* out_ids,
                           int32_t* chain_tokens, int32_t* chain_pos, int* err, cudaStream_t s, bool pdl) {
    if (tp < 1 || tp > kMaxTp) return cudaErrorInvalidValue;
    KeysArgs a{};
    a.amax = amax;
    a.nb = nb;
    a.tp = tp;
    a.rank = rank;
    a.max_nb = max_nb;
    for (int r = 0; r < tp; ++r) {
        a.peer_keys[r] = peer_keys[r];
        a.peer_flags[r] = peer_flags[r];
    }
    a.keys_inbox = keys_inbox;
    a.flags = flags;
    a.epoch = epoch;
    a.out_ids = out_ids;
    a.chain_tokens = chain_tokens;
    a.chain_pos = chain_pos;
    a.err = err;
    void* params[] = {&a};
    return launch_pdl(reinterpret_cast<const void*>(&k_tp_keys), dim3(1), dim3(256), 0, s, params, pdl);
}


// synthetic KV cache content: pages of one sequence, every layer, K and V;
// element (layer, global kv head, position, dim) gets the generator value of its
// index, so tensor-parallel shards hold the same values as a single-GPU cache
__global__ void k_fill_kv(uint16_t* kpool, uint16_t* vpool, size_t layer_elems, int n_layers, const int32_t* pages,
                          int n_tok, int nkv, int kv0, int nkv_g, int hd, uint64_t key_k, uint64_t key_v, float c) {
    const size_t per_layer = (size_t)n_tok * nkv * hd;
    const size_t total = per_layer * n_layers;
    for (size_t i = blockIdx.x * (size_t)blockDim.x + threadIdx.x; i < total; i += (size_t)gridDim.x * blockDim.x) {
        const int layer = (int)(i / per_layer);
        size_t r = i - (size_t)layer * per_layer;
        const int pos = (int)(r / ((size_t)nkv * hd));
        r -= (size_t)pos * nkv * hd;
        const int h = (int)(r / hd), d = (int)(r - (size_t)h * hd);
        const size_t dst = (size_t)layer * layer_elems + (((size_t)pages[pos / 16] * nkv + h) * 16 + pos % 16) * hd + d;
        const size_t gi = (((size_t)layer * nkv_g + kv0 + h) * 1048576u + pos) * hd + d;
        kpool[dst] = __bfloat16_as_ushort(__float2bfloat16_rn(__fmul_rn((float)synth_centered(key_k, gi), c)));
        vpool[dst] = __bfloat16_as_ushort(__float2bfloat16_rn(__fmul_rn((float)synth_centered(key_v, gi), c)));
    }
}

cudaError_t fill_kv_launch(uint16_t* kpool, uint16_t* vpool, size_t layer_elems, int n_layers, const int32_t* pages,
                           int n_tok, int nkv, int kv0, int nkv_g, int hd, uint64_t key_k, uint64_t key_v, float c,
                           cudaStream_t s) {
    const size_t total = (size_t)n_tok * nkv * hd * n_layers;
    if (total == 0) return cudaSuccess;
    const unsigned grid = (unsigned)std::min<size_t>((total + 255) / 256, 148 * 32);
    k_fill_kv<<<grid, 256, 0, s>>>(kpool, vpool, layer_elems, n_layers, pages, n_tok, nkv, kv0, nkv_g, hd, key_k,
                                   key_v, c);
    return cudaGetLastError();
}


// ------------------------------------------------------------------ wait self-test
// The bounded waits on a flag nobody writes and on an mbarrier nobody arrives
// at, each limited to limit_ns: both must give up, set their error bits and
// report how long they waited (ns) in elapsed[0] / elapsed[1].
__global__ void k_wait_selftest(const unsigned int* flag, uint64_t limit_ns, int* err, unsigned long long* elapsed) {
    __shared__ __align__(8) uint64_t bar;
    if (threadIdx.x != 0) return;
    uint64_t t0 = global_ns();
    wait_seq_sys_for(flag, 1u, err, kErrTimeoutPeer, limit_ns);
    elapsed[0] = global_ns() - t0;
    mbar_init(&bar, 1);
    fence_barrier_init();
    t0 = global_ns();
    mbar_wait_for(&bar, 0, err, kErrTimeoutFull, limit_ns);
    elapsed[1] = global_ns() - t0;
}

cudaError_t wait_selftest_launch(const unsigned int* flag, uint64_t limit_ns, int* err, unsigned long long* elapsed,
                                 cudaStream_t s) {
    void* args[] = {&flag, &limit_ns, &err, &elapsed};
    return cudaLaunchKernel(reinterpret_cast<const void*>(&k_wait_selftest), dim3(1), dim3(32), args, 0, s);
}

}  // namespace ti

using namespace ti;

extern "C" ti_status ti_selftest_waits(int device, int limit_us, double* waited_us) {
    clear_error();
    TI_CHECK(limit_us >= 1 && limit_us <= 10000000, TI_ERR_INVALID, "selftest_waits: limit %d us out of range",
             limit_us);
    DeviceGuard g(device);
    uint8_t* buf = nullptr;  // [flag u32][err i32][pad][elapsed u64 x 2]
    TI_CUDA(cudaMalloc(&buf, 64));
    cudaError_t e = cudaMemset(buf, 0, 64);
    int err = 0;
    unsigned long long el[2] = {0, 0};
    if (e == cudaSuccess)
        e = wait_selftest_launch(reinterpret_cast<const unsigned int*>(buf), (uint64_t)limit_us * 1000,
                                 reinterpret_cast<int*>(buf + 4), reinterpret_cast<unsigned long long*>(buf + 16), 0);
    if (e == cudaSuccess) e = cudaDeviceSynchronize();
    if (e == cudaSuccess) e = cudaMemcpy(&err, buf + 4, 4, cudaMemcpyDeviceToHost);
    if (e == cudaSuccess) e = cudaMemcpy(el, buf + 16, 16, cudaMemcpyDeviceToHost);
    cudaFree(buf);
    TI_CHECK(e == cudaSuccess, TI_ERR_CUDA, "selftest_waits: %s", cudaGetErrorString(e));
    if (waited_us) {
        waited_us[0] = el[0] / 1000.0;
        waited_us[1] = el[1] / 1000.0;
    }
    TI_CHECK((err & (kErrTimeoutPeer | kErrTimeoutFull)) == (kErrTimeoutPeer | kErrTimeoutFull), TI_ERR_STATE,
             "selftest_waits: the waits did not report giving up (error bits 0x%x)", err);
    return TI_OK;
}
