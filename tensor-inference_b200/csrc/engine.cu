// engine.cu — the fused decode engine behind the ti_engine_* / ti_seq_* C ABI.
//
// Replaces, per generated token, Generator::generate -> Model::forward ->
// layer_forward -> ops::* (generator.cpp:24-84, llama_model.cpp:103-238,
// qwen_model.cpp:73-146, qwen_adapter_model.cpp:66-193, gemma_model.cpp:57-129,
// mistral_model.cpp:109-178) with one CUDA graph per batch size:
//   embed -> L x [qkv GEMV (+RMSNorm, +bias, +LoRA), attention (+RoPE, +KV append),
//   o GEMV (+residual), gate|up GEMV (+RMSNorm, +SiLU*up), down GEMV (+residual)]
//   -> LM-head GEMV (+final RMSNorm, +greedy argmax)
// every launch chained by programmatic dependent launch.
//
// HBM layout (per engine):
//   weights    embed [V, H]; per layer norm1, norm2 [H], Wqkv [(nq+2nkv)hd, H]
//              (q rows, k rows, v rows of this rank), bqkv, Wo [H, nq*hd],
//              Wgu [2*I, H] (gate rows then up rows), Wdown [H, I]; final norm;
//              lm_head [V_local, H].
//   KV pool    K and V each [L][n_pages][nkv][16][hd] bf16 — a 16-token page of
//              one kv head is 16*hd*2 bytes contiguous; pages are shared by all
//              layers (one page id per 16 positions of a sequence).
//   page table [max_seqs][ceil(max_seq_len/16)] int32, -1 = unallocated.
#include <algorithm>
#include <cmath>
#include <cstdio>
#include <cstdlib>
#include <cstring>
#include <map>
#include <memory>
#include <random>
#include <string>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"
#include "tp.h"
#include "synth.cuh"

using namespace ti;

namespace {

constexpr int kPageTokens = 16;

struct Slot {
    // a checkpoint tensor [rows, cols] of which this rank holds the window
    // rows [r0, r0+nr) x cols [c0, c0+nc), stored at dst with row stride ld
    std::string name;
    size_t rows = 0, cols = 0;
    size_t r0 = 0, nr = 0, c0 = 0, nc = 0;
    uint16_t* dst = nullptr;
    size_t ld = 0;
    bool linear = false;
    // quantised linear weights (wf != kWBf16): rows of wrow_bytes(nc, wf) bytes
    // starting at qdst (the window's first row); column windows are whole blocks
    int wf = kWBf16;
    uint8_t* qdst = nullptr;
    size_t rb = 0;
};

struct LayerW {
    uint16_t *norm1 = nullptr, *norm2 = nullptr, *bqkv = nullptr;
    // linear weights in the engine's weight format (bf16 or quantised rows)
    uint8_t *wqkv = nullptr, *wo = nullptr, *wgu = nullptr, *wdown = nullptr;
};

struct SeqState {
    bool live = false;
    int len = 0;
    std::vector<int> pages;
    // the sampler of the ids this sequence returns (GenerateOptions::sampler,
    // include/tensor/inference/generator.hpp:33-38) and its draws; greedy by default
    SamplerDraws smp;
};

struct GraphEntry {
    cudaGraphExec_t exec = nullptr;
    int launches = 0;
};

}  // namespace

struct ti_engine {
    ti_model_desc d{};
    ti_engine_opts o{};
    int dev = 0, sms = 148;
    int H = 0, nq = 0, nkv = 0, hd = 0, I = 0, V = 0, Vl = 0, qkv_rows = 0;
    int wf = kWBf16;  // format of the layers' linear weights
    // tensor parallelism: this rank's shard (tp.tp == 1: single GPU), the NCCL
    // communicator, fp32 partial sums of o / down, gathered logits for the host
    ti_tp_shard tp{};
    ncclComm_t comm = nullptr;
    float* red = nullptr;
    uint16_t* lgather = nullptr;
    // all-reduce through peer memory (default; TI_TP_ALLREDUCE=nccl selects NCCL):
    // one region per rank, mapped into every peer by CUDA IPC, same offsets on all ranks
    bool peer_ar = false;
    uint8_t* par = nullptr;
    std::vector<uint8_t*> peer;  // [tp] region base as seen from this rank (own base at [rank])
    size_t off_in[2] = {}, off_keys = 0, off_flags[3] = {}, off_ticket = 0, off_tin[2] = {};
    int* epoch = nullptr;
    cudaStream_t cap = nullptr;  // capture stream

    // device memory
    std::vector<void*> allocs;
    size_t bytes_w = 0, bytes_kv = 0, bytes_ad = 0, bytes_work = 0;
    uint16_t *embed = nullptr, *final_norm = nullptr, *lm_head = nullptr;
    std::vector<LayerW> layers;
    float* freqs = nullptr;
    uint16_t *kpool = nullptr, *vpool = nullptr;
    size_t kv_layer_elems = 0;
    int n_pages = 0, pt_stride = 0;
    int32_t* page_table = nullptr;
    std::vector<int> free_pages;
    std::vector<SeqState> seqs;

    // step descriptor: [n_updates, window, 0, 0][tokens B][seq B][pos B][adapter B][updates 3B]
    int32_t *d_desc = nullptr, *h_desc = nullptr;
    int desc_ints = 0;
    uint16_t *hidden = nullptr, *res1 = nullptr, *qkv = nullptr, *attn = nullptr, *act = nullptr, *logits = nullptr;
    unsigned long long* amax = nullptr;
    unsigned int* done = nullptr;
    int32_t* out = nullptr;  // [ids B][err]
    int32_t* h_out = nullptr;
    // device sampling (allocated at the first sampled step): per-row parameters, value histograms
    SampleRow *d_srows = nullptr, *h_srows = nullptr;
    uint32_t* shist = nullptr;
    // device chains that sample: pre-generated draws [max_batch][draw_cap] and per-row counters
    float* d_draws = nullptr;
    int32_t* d_draw_ctr = nullptr;
    int draw_cap = 0;
    int* err = nullptr;
    float *part_o = nullptr, *part_ml = nullptr;
    unsigned int* counters = nullptr;
    // attention fused into the o projection (single-token steps): per-CTA partials,
    // per-kv-head tickets and the grid counters ([2]); fuse_ao: the step uses it
    float* att_part = nullptr;
    unsigned int *att_ticket = nullptr, *att_sync = nullptr;
    bool fuse_ao = false;
    // tensor parallelism while a step is enqueued (fold_recv): a row-parallel
    // projection's receive (no LoRA on it) is held here and run by the next GEMV's
    // prologue, or launched as its own kernel when the next kernel cannot take it
    bool fold_recv = false;
    struct PendingRecv {
        bool on = false;
        GemvRecv r;
        int B = 0, H = 0;
    } pend;
    int attn_splits_n = 1, attn_max_chunk = 0;
    // tensor-core path (batches of tc_min..256 tokens): RMSNorm'd rows, partial
    // tiles shared between CTAs and their tickets
    int tc_min = 8;
    uint16_t* xn = nullptr;
    float* tc_ws = nullptr;
    size_t tc_ws_floats = 0;
    unsigned int* tc_ctr = nullptr;

    std::vector<Slot> slots;
    std::map<std::string, size_t> slot_index;
    std::map<int, GraphEntry> graphs;

    int bound_batch = 0;
    bool bound_lora = false;
    bool bound_sample = false;
    std::vector<int> bound_seqs;

    // ---- LoRA adapter pool (padded rank R, S slots; padding rows/cols are zero)
    struct AdapterMeta {
        bool live = false;
        int rank = 0, mask = 0;
        float alpha = 0.f;
        bool resident = true;
        void* host = nullptr;        // pinned host copy (ti_adapter_stage_host)
        cudaEvent_t ready = nullptr;  // completion of the last async prefetch
        bool pending = false;
    };
    int R = 0, S = 0, lmask = 0;
    // per kind (0 qkv, 1 o, 2 gate|up, 3 down): A / B pools, elements per layer per adapter
    uint16_t* lA[4] = {};
    uint16_t* lB[4] = {};
    size_t lA_layer[4] = {}, lB_layer[4] = {};
    int lK[4] = {}, lT[4] = {}, lRows[4] = {};  // A row length, A rows (sections*R), B rows
    float* lscale = nullptr;
    float* lt[4] = {};  // shrink outputs [B][T]
    float* lws[4] = {};          // shrink split-K partials [kLoraMaxSplit][B][T]
    unsigned int* lctr[4] = {};  // shrink tile counters [S][ceil(T / 32)]
    uint16_t* ldval = nullptr;  // expansions ahead of the tensor-core GEMM [B][rows] bf16
    std::vector<AdapterMeta> adapters;
    cudaStream_t side = nullptr;
    cudaStream_t tp_sync = nullptr;  // host barrier of the ranks (tensor parallelism)

    int32_t* dd_tokens() const { return d_desc + 4; }
    int32_t* dd_seq() const { return d_desc + 4 + o.max_batch; }
    int32_t* dd_pos() const { return d_desc + 4 + 2 * o.max_batch; }
    int32_t* dd_adapter() const { return d_desc + 4 + 3 * o.max_batch; }
    int32_t* dd_updates() const { return d_desc + 4 + 4 * o.max_batch; }
};

namespace {

ti_status dalloc(ti_engine* e, void** p, size_t bytes, size_t* acct) {
    cudaError_t err = cudaMalloc(p, bytes ? bytes : 16);
    if (err != cudaSuccess) {
        cudaGetLastError();
        return fail(TI_ERR_OOM, "engine: cudaMalloc(%zu bytes) failed: %s", bytes, cudaGetErrorString(err));
    }
    e->allocs.push_back(*p);
    if (acct) *acct += bytes;
    return TI_OK;
}

// LoRA rank as stored: padded to whole mma k-steps (16); padding rows of A and
// columns of B are zero.  Every buffer sized by the rank uses this.
inline int lora_padded_rank(int max_rank) { return (max_rank + 15) / 16 * 16; }

template <class T>
ti_status dalloc_t(ti_engine* e, T** p, size_t count, size_t* acct) {
    return dalloc(e, reinterpret_cast<void**>(p), count * sizeof(T), acct);
}

void free_all(ti_engine* e) {
    for (auto& kv : e->graphs)
        if (kv.second.exec) cudaGraphExecDestroy(kv.second.exec);
    e->graphs.clear();
    for (size_t r = 0; r < e->peer.size(); ++r)
        if ((int)r != e->tp.rank && e->peer[r]) cudaIpcCloseMemHandle(e->peer[r]);
    e->peer.clear();
    // graphs holding NCCL calls are gone before the communicator
    if (e->comm) {
        if (const NcclApi* n = nccl_api()) n->CommDestroy(e->comm);
        e->comm = nullptr;
    }
    for (void* p : e->allocs) cudaFree(p);
    e->allocs.clear();
    if (e->h_desc) cudaFreeHost(e->h_desc);
    if (e->h_out) cudaFreeHost(e->h_out);
    if (e->h_srows) cudaFreeHost(e->h_srows);
    e->h_desc = nullptr;
    e->h_out = nullptr;
    e->h_srows = nullptr;
    for (auto& a : e->adapters) {
        if (a.host) cudaFreeHost(a.host);
        if (a.ready) cudaEventDestroy(a.ready);
        a.host = nullptr;
        a.ready = nullptr;
    }
    if (e->side) cudaStreamDestroy(e->side);
    e->side = nullptr;
    if (e->tp_sync) cudaStreamDestroy(e->tp_sync);
    e->tp_sync = nullptr;
    if (e->cap) cudaStreamDestroy(e->cap);
    e->cap = nullptr;
}

void add_slot(ti_engine* e, const std::string& name, size_t rows, size_t cols, size_t r0, size_t nr, size_t c0,
              size_t nc, uint16_t* dst, size_t ld, bool linear) {
    Slot s;
    s.name = name;
    s.rows = rows;
    s.cols = cols;
    s.r0 = r0;
    s.nr = nr;
    s.c0 = c0;
    s.nc = nc;
    s.dst = dst;
    s.ld = ld;
    s.linear = linear;
    e->slot_index[name] = e->slots.size();
    e->slots.push_back(s);
}

// a linear weight: window rows [r0, r0+nr) of a [rows, cols] tensor at row `row`
// of the layer buffer `base` (bf16 rows of cols elements, or quantised rows)
void add_linear(ti_engine* e, const std::string& name, size_t rows, size_t cols, size_t r0, size_t nr, size_t c0,
                size_t nc, uint8_t* base, size_t row) {
    const size_t rb = wrow_bytes((int)nc, e->wf);
    if (e->wf == kWBf16) {
        add_slot(e, name, rows, cols, r0, nr, c0, nc, reinterpret_cast<uint16_t*>(base + row * rb), nc, true);
        return;
    }
    add_slot(e, name, rows, cols, r0, nr, c0, nc, nullptr, nc, true);
    Slot& s = e->slots.back();
    s.wf = e->wf;
    s.qdst = base + row * rb;
    s.rb = rb;
}

ti_status validate_desc(const ti_model_desc* d, const ti_engine_opts* o) {
    TI_CHECK(d && o, TI_ERR_INVALID, "engine: null desc/opts");
    TI_CHECK(d->arch >= TI_ARCH_LLAMA && d->arch <= TI_ARCH_MISTRAL, TI_ERR_INVALID, "engine: unknown arch %d",
             d->arch);
    TI_CHECK(d->hidden > 0 && d->n_layers > 0 && d->n_heads > 0 && d->n_kv_heads > 0 && d->head_dim > 0 &&
                 d->intermediate > 0 && d->vocab > 0,
             TI_ERR_INVALID, "engine: non-positive dimension");
    TI_CHECK(d->n_heads % d->n_kv_heads == 0, TI_ERR_INVALID, "engine: n_heads %% n_kv_heads != 0");
    TI_CHECK(d->n_heads / d->n_kv_heads <= 16, TI_ERR_UNSUPPORTED, "engine: GQA group > 16");
    TI_CHECK(d->head_dim == 64 || d->head_dim == 128 || d->head_dim == 256, TI_ERR_UNSUPPORTED,
             "engine: head_dim %d (64/128/256 supported)", d->head_dim);
    TI_CHECK(d->hidden % 128 == 0 && d->intermediate % 128 == 0 && (d->n_heads * d->head_dim) % 128 == 0,
             TI_ERR_UNSUPPORTED, "engine: hidden, intermediate and n_heads*head_dim must be multiples of 128");
    TI_CHECK(d->weight_format == TI_WFMT_BF16 || d->weight_format == TI_WFMT_Q4_0 || d->weight_format == TI_WFMT_Q8_0,
             TI_ERR_UNSUPPORTED, "engine: unknown weight format %d", d->weight_format);
    if (d->weight_format != TI_WFMT_BF16)
        TI_CHECK(d->hidden % 256 == 0 && d->intermediate % 256 == 0 && (d->n_heads * d->head_dim) % 256 == 0,
                 TI_ERR_UNSUPPORTED, "engine: GGUF weights need hidden, intermediate and n_heads*head_dim % 256 == 0");
    TI_CHECK(o->max_batch >= 1 && o->max_batch <= 256, TI_ERR_INVALID, "engine: max_batch out of range");
    TI_CHECK(o->max_seqs >= 1, TI_ERR_INVALID, "engine: max_seqs < 1");
    TI_CHECK(o->max_seq_len >= 1, TI_ERR_INVALID, "engine: max_seq_len < 1");
    TI_CHECK(o->max_adapters >= 0 && o->max_adapters <= 4096, TI_ERR_INVALID, "engine: max_adapters out of range");
    if (o->max_adapters > 0) {
        TI_CHECK(o->max_lora_rank >= 1 && o->max_lora_rank <= 256, TI_ERR_INVALID, "engine: max_lora_rank 1..256");
        TI_CHECK((o->lora_proj_mask & 0x7f) != 0 && (o->lora_proj_mask & ~0x7f) == 0, TI_ERR_INVALID,
                 "engine: lora_proj_mask must name projections (TI_PROJ_*)");
    }
    const int tp = o->tp_size <= 0 ? 1 : o->tp_size;
    if (tp > 1) {
        ti_tp_shard sh;
        if (ti_status st = tp_plan_make(d, tp, o->tp_rank, &sh)) return st;
        TI_CHECK(o->nccl_id, TI_ERR_INVALID, "engine: tp_size %d needs opts.nccl_id", tp);
        const char* ar = std::getenv("TI_TP_ALLREDUCE");
        TI_CHECK(o->max_adapters == 0 || !(ar && std::string(ar) == "nccl"), TI_ERR_UNSUPPORTED,
                 "engine: LoRA with tensor parallelism uses the peer-memory all-reduce (TI_TP_ALLREDUCE=nccl)");
        TI_CHECK(nccl_api(), TI_ERR_UNSUPPORTED, "engine: tensor parallelism needs libnccl.so.2");
    }
    return TI_OK;
}

ti_status build(ti_engine* e) {
    const ti_model_desc& d = e->d;
    DeviceGuard g(e->dev);
    e->sms = num_sms(e->dev);
    e->H = d.hidden;
    if (ti_status st = tp_plan_make(&d, e->o.tp_size, e->o.tp_size > 1 ? e->o.tp_rank : 0, &e->tp)) return st;
    e->nq = e->tp.nq;
    e->nkv = e->tp.nkv;
    e->hd = d.head_dim;
    e->I = e->tp.inter;
    e->V = d.vocab;
    e->Vl = e->tp.vocab;
    e->qkv_rows = (e->nq + 2 * e->nkv) * e->hd;
    e->wf = d.weight_format == TI_WFMT_Q4_0 ? kWQ4 : d.weight_format == TI_WFMT_Q8_0 ? kWQ8 : kWBf16;
    const int H = e->H, I = e->I, hd = e->hd, nq = e->nq, nkv = e->nkv;
    const size_t QW = (size_t)nq * hd;

    TI_CUDA(cudaStreamCreateWithFlags(&e->cap, cudaStreamNonBlocking));

    // ---- weights
    TI_CHECK(dalloc_t(e, &e->embed, (size_t)e->V * H, &e->bytes_w) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    add_slot(e, "model.embed_tokens.weight", e->V, H, 0, e->V, 0, H, e->embed, H, false);
    TI_CHECK(dalloc_t(e, &e->final_norm, H, &e->bytes_w) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    add_slot(e, "model.norm.weight", 1, H, 0, 1, 0, H, e->final_norm, H, false);
    TI_CHECK(dalloc_t(e, &e->lm_head, (size_t)e->Vl * H, &e->bytes_w) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    add_slot(e, "lm_head.weight", e->V, H, e->tp.v0, e->Vl, 0, H, e->lm_head, H, false);
    e->layers.resize(d.n_layers);
    for (int i = 0; i < d.n_layers; ++i) {
        LayerW& l = e->layers[i];
        const std::string p = "model.layers." + std::to_string(i) + ".";
        TI_CHECK(dalloc_t(e, &l.norm1, H, &e->bytes_w) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
        TI_CHECK(dalloc_t(e, &l.norm2, H, &e->bytes_w) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
        const size_t rbH = wrow_bytes(H, e->wf), rbQ = wrow_bytes((int)QW, e->wf), rbI = wrow_bytes(I, e->wf);
        TI_CHECK(dalloc(e, reinterpret_cast<void**>(&l.wqkv), (size_t)e->qkv_rows * rbH, &e->bytes_w) == TI_OK,
                 TI_ERR_OOM, "%s", ti_last_error());
        TI_CHECK(dalloc(e, reinterpret_cast<void**>(&l.wo), (size_t)H * rbQ, &e->bytes_w) == TI_OK, TI_ERR_OOM,
                 "%s", ti_last_error());
        TI_CHECK(dalloc(e, reinterpret_cast<void**>(&l.wgu), (size_t)2 * I * rbH, &e->bytes_w) == TI_OK, TI_ERR_OOM,
                 "%s", ti_last_error());
        TI_CHECK(dalloc(e, reinterpret_cast<void**>(&l.wdown), (size_t)H * rbI, &e->bytes_w) == TI_OK, TI_ERR_OOM,
                 "%s", ti_last_error());
        add_slot(e, p + "input_layernorm.weight", 1, H, 0, 1, 0, H, l.norm1, H, false);
        add_slot(e, p + "post_attention_layernorm.weight", 1, H, 0, 1, 0, H, l.norm2, H, false);
        // local shard: q/k/v heads [q0, q0+nq) / [kv0, kv0+nkv), gate/up rows and
        // down columns [i0, i0+I), o columns = the local q heads' width
        const size_t KW = (size_t)nkv * hd;
        const size_t QWg = (size_t)d.n_heads * hd, KWg = (size_t)d.n_kv_heads * hd, Ig = (size_t)d.intermediate;
        const size_t q0 = (size_t)e->tp.q0 * hd, k0 = (size_t)e->tp.kv0 * hd, i0 = (size_t)e->tp.i0;
        add_linear(e, p + "self_attn.q_proj.weight", QWg, H, q0, QW, 0, H, l.wqkv, 0);
        add_linear(e, p + "self_attn.k_proj.weight", KWg, H, k0, KW, 0, H, l.wqkv, QW);
        add_linear(e, p + "self_attn.v_proj.weight", KWg, H, k0, KW, 0, H, l.wqkv, QW + KW);
        add_linear(e, p + "self_attn.o_proj.weight", H, QWg, 0, H, q0, QW, l.wo, 0);
        add_linear(e, p + "mlp.gate_proj.weight", Ig, H, i0, I, 0, H, l.wgu, 0);
        add_linear(e, p + "mlp.up_proj.weight", Ig, H, i0, I, 0, H, l.wgu, I);
        add_linear(e, p + "mlp.down_proj.weight", H, Ig, 0, H, i0, I, l.wdown, 0);
        if (d.qkv_bias) {
            TI_CHECK(dalloc_t(e, &l.bqkv, e->qkv_rows, &e->bytes_w) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
            add_slot(e, p + "self_attn.q_proj.bias", 1, QWg, 0, 1, q0, QW, l.bqkv, QW, false);
            add_slot(e, p + "self_attn.k_proj.bias", 1, KWg, 0, 1, k0, KW, l.bqkv + QW, KW, false);
            add_slot(e, p + "self_attn.v_proj.bias", 1, KWg, 0, 1, k0, KW, l.bqkv + QW + KW, KW, false);
        }
    }
    std::vector<float> fr(hd / 2);
    rope_freqs(hd, d.rope_theta, &d.rope, fr.data());
    TI_CHECK(dalloc_t(e, &e->freqs, hd / 2, &e->bytes_w) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    TI_CUDA(cudaMemcpy(e->freqs, fr.data(), fr.size() * 4, cudaMemcpyHostToDevice));

    // ---- KV pool and page table
    e->pt_stride = (e->o.max_seq_len + kPageTokens - 1) / kPageTokens;
    e->n_pages = e->o.kv_pages > 0 ? e->o.kv_pages : e->o.max_seqs * e->pt_stride;
    e->kv_layer_elems = (size_t)e->n_pages * nkv * kPageTokens * hd;
    TI_CHECK(dalloc_t(e, &e->kpool, e->kv_layer_elems * d.n_layers, &e->bytes_kv) == TI_OK, TI_ERR_OOM, "%s",
             ti_last_error());
    TI_CHECK(dalloc_t(e, &e->vpool, e->kv_layer_elems * d.n_layers, &e->bytes_kv) == TI_OK, TI_ERR_OOM, "%s",
             ti_last_error());
    TI_CHECK(dalloc_t(e, &e->page_table, (size_t)e->o.max_seqs * e->pt_stride, &e->bytes_kv) == TI_OK, TI_ERR_OOM,
             "%s", ti_last_error());
    TI_CUDA(cudaMemset(e->page_table, 0xff, (size_t)e->o.max_seqs * e->pt_stride * 4));
    e->free_pages.resize(e->n_pages);
    for (int i = 0; i < e->n_pages; ++i) e->free_pages[i] = e->n_pages - 1 - i;
    e->seqs.assign(e->o.max_seqs, SeqState{});

    // ---- step buffers
    const int B = e->o.max_batch;
    e->desc_ints = 4 + 7 * B;
    TI_CHECK(dalloc_t(e, &e->d_desc, e->desc_ints, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    TI_CUDA(cudaMemset(e->d_desc, 0, e->desc_ints * 4));
    TI_CUDA(cudaMallocHost(&e->h_desc, e->desc_ints * 4));
    TI_CUDA(cudaMallocHost(&e->h_out, (B + 1) * 4));
    TI_CHECK(dalloc_t(e, &e->hidden, (size_t)B * H, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    TI_CHECK(dalloc_t(e, &e->res1, (size_t)B * H, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    TI_CHECK(dalloc_t(e, &e->qkv, (size_t)B * e->qkv_rows, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s",
             ti_last_error());
    TI_CHECK(dalloc_t(e, &e->attn, (size_t)B * QW, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    TI_CHECK(dalloc_t(e, &e->act, (size_t)B * I, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    TI_CHECK(dalloc_t(e, &e->logits, (size_t)B * e->Vl, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s",
             ti_last_error());
    TI_CHECK(dalloc_t(e, &e->amax, B, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    TI_CUDA(cudaMemset(e->amax, 0, B * 8));
    TI_CHECK(dalloc_t(e, &e->done, 16, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    TI_CUDA(cudaMemset(e->done, 0, 64));
    TI_CHECK(dalloc_t(e, &e->out, B + 1, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    TI_CUDA(cudaMemset(e->out, 0, (B + 1) * 4));
    e->err = reinterpret_cast<int*>(e->out + B);
    if (e->tp.tp > 1) {
        TI_CHECK(dalloc_t(e, &e->red, (size_t)B * H, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
        TI_CHECK(dalloc_t(e, &e->lgather, (size_t)B * e->V, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s",
                 ti_last_error());
        const NcclApi* n = nccl_api();
        ncclUniqueId id;
        std::memcpy(&id, e->o.nccl_id, sizeof id);
        const ncclResult_t r = n->CommInitRank(&e->comm, e->tp.tp, id, e->tp.rank);
        TI_CHECK(r == ncclSuccess, TI_ERR_CUDA, "ncclCommInitRank (rank %d of %d): %s", e->tp.rank, e->tp.tp,
                 n->GetErrorString(r));
        TI_CUDA(cudaStreamCreateWithFlags(&e->tp_sync, cudaStreamNonBlocking));
        const char* ar = std::getenv("TI_TP_ALLREDUCE");
        e->peer_ar = !(ar && std::string(ar) == "nccl") && e->tp.tp <= kMaxTp;
        if (e->peer_ar) {
            // [inbox o | inbox down] fp32 [tp][B][H] each, keys u64 [tp][B], flags u32 [3][tp], tickets
            const int tpn = e->tp.tp;
            size_t o = 0;
            auto take = [&](size_t bytes) {
                const size_t at = o;
                o = (o + bytes + 255) & ~size_t(255);
                return at;
            };
            e->off_in[0] = take((size_t)tpn * B * H * 4);
            e->off_in[1] = take((size_t)tpn * B * H * 4);
            e->off_keys = take((size_t)tpn * B * 8);
            // row-parallel LoRA: every rank's partial x.A^T (o, down), [tp][B][R]
            const int Rp = e->o.max_adapters > 0 ? lora_padded_rank(e->o.max_lora_rank) : 0;
            e->off_tin[0] = take((size_t)tpn * B * Rp * 4);
            e->off_tin[1] = take((size_t)tpn * B * Rp * 4);
            for (int k = 0; k < 3; ++k) e->off_flags[k] = take((size_t)tpn * 4);
            e->off_ticket = take(16);
            TI_CHECK(dalloc(e, reinterpret_cast<void**>(&e->par), o, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s",
                     ti_last_error());
            TI_CUDA(cudaMemset(e->par, 0, o));
            TI_CHECK(dalloc_t(e, &e->epoch, 1, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
            TI_CUDA(cudaMemset(e->epoch, 0, 4));
            // exchange the regions' IPC handles over the communicator
            cudaIpcMemHandle_t mine;
            TI_CUDA(cudaIpcGetMemHandle(&mine, e->par));
            uint8_t* stage = nullptr;
            TI_CHECK(dalloc(e, reinterpret_cast<void**>(&stage), (size_t)(tpn + 1) * sizeof mine, &e->bytes_work) ==
                         TI_OK,
                     TI_ERR_OOM, "%s", ti_last_error());
            TI_CUDA(cudaMemcpy(stage + (size_t)tpn * sizeof mine, &mine, sizeof mine, cudaMemcpyHostToDevice));
            const ncclResult_t r2 =
                n->AllGather(stage + (size_t)tpn * sizeof mine, stage, sizeof mine, ncclUint8, e->comm, e->cap);
            TI_CHECK(r2 == ncclSuccess, TI_ERR_CUDA, "ncclAllGather (IPC handles): %s", n->GetErrorString(r2));
            TI_CUDA(cudaStreamSynchronize(e->cap));
            std::vector<cudaIpcMemHandle_t> all(tpn);
            TI_CUDA(cudaMemcpy(all.data(), stage, (size_t)tpn * sizeof mine, cudaMemcpyDeviceToHost));
            e->peer.assign(tpn, nullptr);
            for (int q = 0; q < tpn; ++q) {
                if (q == e->tp.rank) {
                    e->peer[q] = e->par;
                    continue;
                }
                void* pp = nullptr;
                TI_CUDA(cudaIpcOpenMemHandle(&pp, all[q], cudaIpcMemLazyEnablePeerAccess));
                e->peer[q] = reinterpret_cast<uint8_t*>(pp);
            }
        }
    }
    {
        const char* env = std::getenv("TI_TC_MIN_BATCH");
        e->tc_min = env ? std::atoi(env) : 8;
        if (B >= e->tc_min && e->tc_min > 0) {
            const int kmax = std::max(H, std::max((int)QW, I));
            TI_CHECK(dalloc_t(e, &e->xn, (size_t)std::min(B, 256) * kmax, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s",
                     ti_last_error());
            e->tc_ws_floats = (size_t)12 << 20;  // 48 MB: 2 partial tiles per CTA at 256 tokens
            TI_CHECK(dalloc(e, reinterpret_cast<void**>(&e->tc_ws), e->tc_ws_floats * 4, &e->bytes_work) == TI_OK,
                     TI_ERR_OOM, "%s", ti_last_error());
            const size_t ntiles = (size_t)std::max(e->Vl, std::max(2 * I, e->qkv_rows)) / 64 + 64;
            TI_CHECK(dalloc(e, reinterpret_cast<void**>(&e->tc_ctr), ntiles * 4, &e->bytes_work) == TI_OK,
                     TI_ERR_OOM, "%s", ti_last_error());
            TI_CUDA(cudaMemset(e->tc_ctr, 0, ntiles * 4));
        }
    }
    if (e->o.max_adapters > 0) {
        e->S = e->o.max_adapters;
        e->R = lora_padded_rank(e->o.max_lora_rank);
        e->lmask = e->o.lora_proj_mask;
        const int R = e->R;
        const bool on[4] = {(e->lmask & 7) != 0, (e->lmask & 8) != 0, (e->lmask & 48) != 0, (e->lmask & 64) != 0};
        const int K[4] = {H, (int)QW, H, I};
        const int T[4] = {3 * R, R, 2 * R, R};
        const int rows[4] = {e->qkv_rows, H, 2 * I, H};
        for (int k = 0; k < 4; ++k) {
            if (!on[k]) continue;
            e->lK[k] = K[k];
            e->lT[k] = T[k];
            e->lRows[k] = rows[k];
            e->lA_layer[k] = (size_t)T[k] * K[k];
            e->lB_layer[k] = (size_t)rows[k] * R;
            const size_t na = e->lA_layer[k] * d.n_layers * e->S, nbb = e->lB_layer[k] * d.n_layers * e->S;
            TI_CHECK(dalloc_t(e, &e->lA[k], na, &e->bytes_ad) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
            TI_CHECK(dalloc_t(e, &e->lB[k], nbb, &e->bytes_ad) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
            TI_CUDA(cudaMemset(e->lA[k], 0, na * 2));
            TI_CUDA(cudaMemset(e->lB[k], 0, nbb * 2));
            if (!e->ldval && e->xn) {
                const size_t rmax = std::max<size_t>(std::max<size_t>(e->qkv_rows, H), 2 * (size_t)I);
                TI_CHECK(dalloc_t(e, &e->ldval, (size_t)std::min(B, 256) * rmax, &e->bytes_work) == TI_OK, TI_ERR_OOM,
                         "%s", ti_last_error());
            }
            TI_CHECK(dalloc_t(e, &e->lt[k], (size_t)B * T[k], &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s",
                     ti_last_error());
            TI_CHECK(dalloc_t(e, &e->lws[k], (size_t)kLoraMaxSplit * B * T[k], &e->bytes_work) == TI_OK, TI_ERR_OOM,
                     "%s", ti_last_error());
            const size_t nctr = (size_t)e->S * ((T[k] + 31) / 32);
            TI_CHECK(dalloc_t(e, &e->lctr[k], nctr, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
            TI_CUDA(cudaMemset(e->lctr[k], 0, nctr * 4));
        }
        TI_CHECK(dalloc_t(e, &e->lscale, e->S, &e->bytes_ad) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
        TI_CUDA(cudaMemset(e->lscale, 0, (size_t)e->S * 4));
        e->adapters.assign(e->S, ti_engine::AdapterMeta{});
        TI_CUDA(cudaStreamCreateWithFlags(&e->side, cudaStreamNonBlocking));
    }
    e->attn_splits_n = attn_splits(B, nkv, hd, e->o.max_seq_len, e->sms, &e->attn_max_chunk);
    // partials sized for the largest batch; smaller batches use more splits per (token, head)
    int max_parts = 0;
    for (int b = 1; b <= B; ++b) {
        int mc = 0;
        int n = attn_splits(b, nkv, hd, e->o.max_seq_len, e->sms, &mc);
        max_parts = std::max(max_parts, b * n);
    }
    const int G = nq / nkv;
    TI_CHECK(dalloc_t(e, &e->part_o, (size_t)max_parts * nkv * G * hd, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s",
             ti_last_error());
    TI_CHECK(dalloc_t(e, &e->part_ml, (size_t)max_parts * nkv * G * 2, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s",
             ti_last_error());
    TI_CHECK(dalloc_t(e, &e->counters, (size_t)B * nkv, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    TI_CUDA(cudaMemset(e->counters, 0, (size_t)B * nkv * 4));
    {
        // TI_FUSED_ATTN=1: single-token steps run attention inside the o
        // projection's GEMV (attn_fused.cuh).  Off by default: on the 8B shape at
        // batch 1 the step measured 3.12 ms fused against 2.91 ms with the
        // separate attention kernel (one warp per 16-token page and the
        // cross-CTA merge are latency-bound).
        const char* env = std::getenv("TI_FUSED_ATTN");
        e->fuse_ao = env && std::atoi(env) == 1 && G <= 8 && (hd == 64 || hd == 128) && e->sms >= nkv &&
                     (nq * hd) % 128 == 0;
        if (e->fuse_ao) {
            TI_CHECK(dalloc_t(e, &e->att_part, (size_t)e->sms * G * (hd + 2), &e->bytes_work) == TI_OK, TI_ERR_OOM,
                     "%s", ti_last_error());
            TI_CHECK(dalloc_t(e, &e->att_ticket, (size_t)nkv + 2, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s",
                     ti_last_error());
            TI_CUDA(cudaMemset(e->att_ticket, 0, ((size_t)nkv + 2) * 4));
            e->att_sync = e->att_ticket + nkv;
        }
    }
    TI_CUDA(cudaDeviceSynchronize());
    return TI_OK;
}

// ------------------------------------------------------------------ the kernels of one step
enum KernelKind { kKEmbed = 0, kKQkv = 1, kKAttn = 2, kKO = 3, kKGateUp = 4, kKDown = 5, kKLmHead = 6 };

// Enqueue one kernel of a B-token step on `s` (graph capture or a plain launch).
ti_status enqueue_kernel(ti_engine* e, int B, int kind, int li, cudaStream_t s, int* launches, bool lora,
                         bool prefill = false) {
    const ti_model_desc& d = e->d;
    const int H = e->H, I = e->I, nq = e->nq, nkv = e->nkv, hd = e->hd;
    const int QW = nq * hd;
    const bool gemma = d.arch == TI_ARCH_GEMMA;
    std::string why;

    // SIMT GEMV: batch chunks of <= 8 tokens, fewer when the tokens' activation
    // rows (kept in shared memory) would crowd out a two-stage weight ring
    auto gemv_all = [&](GemvArgs a, int epi, int x_stride_elems, int out_stride, int resid_stride) -> ti_status {
        const size_t U = epi == kEpiGlu ? 2 : 1;
        int chunk = 8;
        while (chunk > 1 && (size_t)chunk * a.K * 2 + 2 * U * (size_t)a.K * 2 + 16 * 1024 > 220 * 1024) chunk /= 2;
        for (int b0 = 0; b0 < B; b0 += chunk) {
            GemvArgs c = a;
            c.nb = std::min(chunk, B - b0);
            c.x = a.x + (size_t)b0 * x_stride_elems;
            c.out = a.out + (size_t)b0 * out_stride;
            if (a.partial) c.partial = a.partial + (size_t)b0 * out_stride;
            if (a.ps.tp) {
                for (int r = 0; r < a.ps.tp; ++r) c.ps.inbox[r] = a.ps.inbox[r] + (size_t)b0 * out_stride;
                c.ps.signal = b0 + chunk >= B ? a.ps.signal : 0;  // the last chunk publishes
            }
            if (a.resid) c.resid = a.resid + (size_t)b0 * resid_stride;
            if (a.recv.tp) {
                c.recv.inbox = a.recv.inbox + (size_t)b0 * a.K;
                c.recv.resid = a.recv.resid + (size_t)b0 * a.K;
                c.recv.x_out = a.recv.x_out + (size_t)b0 * a.K;
            }
            if (a.lora.adapter) {
                c.lora.adapter = a.lora.adapter + b0;
                c.lora.t = a.lora.t + (size_t)b0 * a.lora.t_stride;
            }
            if (epi == kEpiLmHead) {
                c.amax = a.amax + b0;
                c.done = a.done + (b0 / chunk) % 16;  // one completion counter per launch
                c.out_ids = a.out_ids + b0;
                if (a.chain_tokens) c.chain_tokens = a.chain_tokens + b0;
                if (a.chain_pos) c.chain_pos = a.chain_pos + b0;
            }
            GemvPlan plan;
            if (!gemv_plan(c, epi, e->dev, &plan, &why)) return fail(TI_ERR_UNSUPPORTED, "%s", why.c_str());
            TI_CUDA(gemv_launch(c, epi, plan, s, true));
            if (launches) ++*launches;
        }
        return TI_OK;
    };

    // batches of tc_min..256 tokens: RMSNorm pass (when the GEMV would fuse it) +
    // tcgen05 GEMM (GGUF weights dequantised to bf16 operands in TMEM;
    // the LoRA expansion precomputed and added in its epilogue)
    auto gemm = [&](GemvArgs a, int epi, int x_stride_elems, int out_stride, int resid_stride) -> ti_status {
        if (!(e->xn && B >= e->tc_min && B <= 256))
            return gemv_all(a, epi, x_stride_elems, out_stride, resid_stride);
        a.nb = B;
        if (a.norm_w) {
            TI_CUDA(rms_rows_launch(a.x, a.x_stride, a.norm_w, a.eps, a.norm_offset, a.K, B, e->xn, a.K, s, true));
            if (launches) ++*launches;
            a.x = e->xn;
            a.x_stride = a.K;
            a.norm_w = nullptr;
        }
        if (a.lora.adapter && e->ldval) {
            // LoRA expansion of every (token, row) ahead of the GEMM; its epilogue adds it
            const int rows = epi == kEpiGlu ? 2 * a.N : a.N;
            TI_CUDA(lora_expand_launch(a.lora, B, rows, epi == kEpiGlu ? a.N : 0, e->ldval, rows, s, true));
            if (launches) ++*launches;
            a.lora.dval = e->ldval;
            a.lora.dval_stride = rows;
        }
        // GGUF weights: launches of at most 128 tokens (the dequantised operands share
        // TMEM with the accumulators); the last launch publishes a tensor-parallel send
        const int chunk = a.wfmt != kWBf16 ? 128 : B;
        for (int b0 = 0; b0 < B; b0 += chunk) {
            GemvArgs c = a;
            c.nb = std::min(chunk, B - b0);
            if (b0 > 0) {
                c.x = a.x + (size_t)b0 * a.x_stride;
                c.out = a.out + (size_t)b0 * a.out_stride;
                if (a.resid) c.resid = a.resid + (size_t)b0 * a.resid_stride;
                if (a.partial) c.partial = a.partial + (size_t)b0 * a.out_stride;
                for (int r = 0; r < a.ps.tp; ++r) c.ps.inbox[r] = a.ps.inbox[r] + (size_t)b0 * a.out_stride;
                if (a.lora.adapter) {
                    c.lora.adapter = a.lora.adapter + b0;
                    c.lora.t = a.lora.t + (size_t)b0 * a.lora.t_stride;
                    if (a.lora.dval) c.lora.dval = a.lora.dval + (size_t)b0 * a.lora.dval_stride;
                }
            }
            if (a.ps.tp) c.ps.signal = b0 + chunk >= B ? a.ps.signal : 0;
            TcPlan plan;
            if (!tc_plan(c, epi, e->dev, e->tc_ws_floats, &plan, &why))
                return fail(TI_ERR_UNSUPPORTED, "%s", why.c_str());
            TI_CUDA(tc_launch(c, epi, plan, e->tc_ws, e->tc_ctr, s, true));
            if (launches) ++*launches;
        }
        return TI_OK;
    };

    // the tcgen05 path takes normalised rows: one RMSNorm pass ahead of the GEMM
    // (and of the LoRA shrink, which then reads the same rows)
    auto prenorm = [&](GemvArgs& a) -> ti_status {
        if (!(e->xn && B >= e->tc_min && B <= 256) || !a.norm_w) return TI_OK;
        TI_CUDA(rms_rows_launch(a.x, a.x_stride, a.norm_w, a.eps, a.norm_offset, a.K, B, e->xn, a.K, s, true));
        if (launches) ++*launches;
        a.x = e->xn;
        a.x_stride = a.K;
        a.norm_w = nullptr;
        return TI_OK;
    };

    // tensor parallelism: a row-parallel projection stores fp32 partial sums,
    // NCCL sums them over the group, then out = bf16(resid + bf16(sum))
    auto nccl_check = [&](ncclResult_t r, const char* what) -> ti_status {
        if (r == ncclSuccess) return TI_OK;
        return fail(TI_ERR_CUDA, "%s: %s", what, nccl_api()->GetErrorString(r));
    };
    auto row_parallel = [&](GemvArgs a, int x_stride_elems, uint16_t* out, const uint16_t* resid,
                            const GemvLora* lora) -> ti_status {
        a.out = nullptr;
        a.out_stride = H;
        a.resid = nullptr;
        if (e->peer_ar) {
            // the projection's epilogue writes into every rank's inbox; the receive
            // (wait for all ranks, rank-ordered sum + residual) runs in the next GEMV's
            // prologue when it can, else as k_tp_recv_resid
            const int ph = kind == kKO ? 0 : 1;
            const int MB = e->o.max_batch;
            a.ps.tp = e->tp.tp;
            for (int r = 0; r < e->tp.tp; ++r) {
                a.ps.inbox[r] = reinterpret_cast<float*>(e->peer[r] + e->off_in[ph]) + (size_t)e->tp.rank * MB * H;
                a.ps.flag[r] = reinterpret_cast<unsigned int*>(e->peer[r] + e->off_flags[ph]) + e->tp.rank;
            }
            a.ps.epoch = e->epoch;
            a.ps.seq_mul = d.n_layers;
            a.ps.seq_add = li + 1;
            a.ps.ticket = reinterpret_cast<unsigned int*>(e->par + e->off_ticket) + ph;
            if (ti_status st = gemm(a, kEpiStore, x_stride_elems, H, 0)) return st;
            if (e->fold_recv && !lora) {
                GemvRecv& r = e->pend.r;
                r.inbox = reinterpret_cast<const float*>(e->par + e->off_in[ph]);
                r.src_stride = (size_t)MB * H;
                r.flags = reinterpret_cast<const unsigned int*>(e->par + e->off_flags[ph]);
                r.tp = e->tp.tp;
                r.epoch = e->epoch;
                r.seq_mul = d.n_layers;
                r.seq_add = li + 1;
                r.resid = resid;
                r.x_out = out;
                e->pend.B = B;
                e->pend.H = H;
                e->pend.on = true;
                return TI_OK;
            }
            TI_CUDA(tp_recv_resid_launch(reinterpret_cast<const float*>(e->par + e->off_in[ph]), (size_t)MB * H,
                                         reinterpret_cast<const unsigned int*>(e->par + e->off_flags[ph]), e->tp.tp,
                                         e->epoch, d.n_layers, li + 1, resid, out, B, H, lora,
                                         reinterpret_cast<const float*>(e->par + e->off_tin[ph]),
                                         (size_t)MB * (lora ? lora->rank : 0), e->err, s, true));
            if (launches) ++*launches;
            return TI_OK;
        }
        a.partial = e->red;
        if (ti_status st = gemm(a, kEpiStore, x_stride_elems, H, 0)) return st;
        if (ti_status st = nccl_check(nccl_api()->AllReduce(e->red, e->red, (size_t)B * H, ncclFloat32, ncclSum,
                                                            e->comm, s),
                                      "ncclAllReduce"))
            return st;
        TI_CUDA(tp_resid_launch(e->red, resid, out, B, H, s, true));
        if (launches) ++*launches;
        return TI_OK;
    };

    if (kind == kKEmbed) {
        EmbedArgs ea;
        ea.table = e->embed;
        ea.vocab = e->V;
        ea.hidden = H;
        ea.nb = B;
        ea.tokens = e->dd_tokens();
        ea.out = e->hidden;
        ea.scale = gemma ? std::sqrt((float)H) : 0.f;
        ea.pt_updates = e->dd_updates();
        ea.n_updates = e->d_desc;
        ea.page_table = e->page_table;
        ea.pt_stride = e->pt_stride;
        ea.epoch = e->peer_ar ? e->epoch : nullptr;
        ea.err = e->err;
        TI_CUDA(embed_launch(ea, s, true));
        if (launches) ++*launches;
        return TI_OK;
    }
    // L2 warm-up target: the next GEMV of the step (qkv -> o -> gate|up -> down ->
    // next layer's qkv or the LM head; the LM head warms layer 0 for the next step)
    const char* next_env = std::getenv("TI_GEMV_NEXT_KB");
    const int next_kb = next_env ? std::atoi(next_env) : 640;
    // TI_GEMV_NEXT2=1: the q+k+v GEMV spends what its budget leaves after the o
    // projection on gate|up, so HBM keeps streaming while attention runs
    const char* next2_env = std::getenv("TI_GEMV_NEXT2");
    const bool next2 = next2_env && std::atoi(next2_env) == 1;
    auto set_next = [&](GemvArgs& a, const void* w, int N, int K, int U) {
        a.next_w = w;
        a.next_wfmt = w == e->lm_head ? kWBf16 : e->wf;
        a.next_N = N;
        a.next_K = K;
        a.next_U = U;
        a.next_bytes = next_kb * 1024;
    };
    // a receive held by the previous row-parallel projection: into this GEMV's
    // prologue, or as its own kernel when this kernel cannot take it (tensor-core
    // batch, or a LoRA shrink that reads x first)
    auto take_recv = [&](GemvArgs& g, bool can_fuse) -> ti_status {
        if (!e->pend.on) return TI_OK;
        e->pend.on = false;
        if (can_fuse && !(e->xn && B >= e->tc_min && B <= 256)) {
            g.recv = e->pend.r;
            return TI_OK;
        }
        const GemvRecv& r = e->pend.r;
        TI_CUDA(tp_recv_resid_launch(r.inbox, r.src_stride, r.flags, r.tp, r.epoch, r.seq_mul, r.seq_add, r.resid,
                                     r.x_out, e->pend.B, e->pend.H, nullptr, nullptr, 0, e->err, s, true));
        if (launches) ++*launches;
        return TI_OK;
    };
    if (kind == kKLmHead) {
        GemvArgs lm;
        lm.W = e->lm_head;
        lm.N = e->Vl;
        lm.K = H;
        lm.x = e->hidden;
        lm.x_stride = H;
        lm.norm_w = e->final_norm;
        lm.eps = d.rms_eps;
        lm.norm_offset = gemma;
        lm.out = e->logits;
        lm.out_stride = e->Vl;
        lm.amax = e->amax;
        lm.done = e->done;
        lm.out_ids = e->out;
        lm.chain_tokens = e->dd_tokens();
        lm.chain_pos = e->dd_pos();
        lm.err = e->err;
        set_next(lm, e->layers[0].wqkv, e->qkv_rows, H, 1);
        if (ti_status st = take_recv(lm, true)) return st;
        if (e->tp.tp == 1) return gemm(lm, kEpiLmHead, H, e->Vl, 0);
        // vocabulary-parallel: local keys carry global indices; max over the group
        lm.key_offset = e->tp.v0;
        lm.publish = 0;
        if (ti_status st = gemm(lm, kEpiLmHead, H, e->Vl, 0)) return st;
        if (e->peer_ar) {
            std::vector<unsigned long long*> pk(e->tp.tp);
            std::vector<unsigned int*> pf(e->tp.tp);
            for (int r = 0; r < e->tp.tp; ++r) {
                pk[r] = reinterpret_cast<unsigned long long*>(e->peer[r] + e->off_keys);
                pf[r] = reinterpret_cast<unsigned int*>(e->peer[r] + e->off_flags[2]);
            }
            TI_CUDA(tp_keys_launch(e->amax, B, pk.data(), pf.data(), e->tp.tp, e->tp.rank,
                                   reinterpret_cast<const unsigned long long*>(e->par + e->off_keys),
                                   reinterpret_cast<const unsigned int*>(e->par + e->off_flags[2]), e->o.max_batch,
                                   e->epoch, e->out, e->dd_tokens(), e->dd_pos(), e->err, s, true));
            if (launches) ++*launches;
            return TI_OK;
        }
        if (ti_status st = nccl_check(
                nccl_api()->AllReduce(e->amax, e->amax, (size_t)B, ncclUint64, ncclMax, e->comm, s), "ncclAllReduce"))
            return st;
        TI_CUDA(tp_ids_launch(e->amax, B, e->out, e->dd_tokens(), e->dd_pos(), s, true));
        if (launches) ++*launches;
        return TI_OK;
    }
    TI_CHECK(li >= 0 && li < d.n_layers, TI_ERR_INVALID, "layer %d out of range", li);
    const LayerW& l = e->layers[li];
    // LoRA (qwen_adapter_model.cpp:22-43): shrink t = bf16(x A^T) for each token's
    // adapter right before the adapted GEMV, whose epilogue adds bf16(bf16(B t) * s)
    auto lora_on = [&](int k) { return lora && e->lA[k] != nullptr; };
    auto shrink = [&](int k, const uint16_t* x, int x_stride, const uint16_t* norm_w) -> ti_status {
        LoraShrinkArgs la;
        la.x = x;
        la.x_stride = x_stride;
        la.K = e->lK[k];
        la.nb = B;
        la.norm_w = norm_w;
        la.eps = d.rms_eps;
        la.norm_offset = gemma;
        la.A = e->lA[k] + (size_t)li * e->lA_layer[k];
        la.A_adapter_stride = e->lA_layer[k] * d.n_layers;
        la.T = e->lT[k];
        la.adapter = e->dd_adapter();
        la.n_adapters = e->S;
        la.t = e->lt[k];
        la.t_stride = e->lT[k];
        la.ws = e->lws[k];
        la.ctr = e->lctr[k];
        if (e->tp.tp > 1 && (k == 1 || k == 3)) {
            // row-parallel: partial sums over this rank's input columns to every rank
            const int ph = k == 1 ? 0 : 1;
            la.tp = e->tp.tp;
            for (int r = 0; r < e->tp.tp; ++r)
                la.peer_t[r] = reinterpret_cast<float*>(e->peer[r] + e->off_tin[ph]) +
                               (size_t)e->tp.rank * e->o.max_batch * e->lT[k];
        }
        TI_CUDA(lora_shrink_launch(la, s, true));
        if (launches) ++*launches;
        return TI_OK;
    };
    auto set_lora = [&](GemvArgs& g, int k) {
        g.lora.adapter = e->dd_adapter();
        g.lora.B = e->lB[k] + (size_t)li * e->lB_layer[k];
        g.lora.B_adapter_stride = e->lB_layer[k] * d.n_layers;
        g.lora.t = e->lt[k];
        g.lora.t_stride = e->lT[k];
        g.lora.rank = e->R;
        g.lora.scale = e->lscale;
        g.lora.n_adapters = e->S;
        if (k == 0) {
            g.lora.sec1 = QW;
            g.lora.sec2 = QW + nkv * hd;
        }
    };
    // a single-token decode step whose o projection has no LoRA runs attention
    // inside the o projection's GEMV (attn_fused.cuh): no attention launch
    const bool fused_ao = e->fuse_ao && B == 1 && !prefill && !lora_on(1) && !(e->xn && B >= e->tc_min);
    switch (kind) {
        case kKQkv: {
            GemvArgs q;
            q.W = l.wqkv;
            q.wfmt = e->wf;
            q.N = e->qkv_rows;
            q.K = H;
            q.x = e->hidden;
            q.x_stride = H;
            q.norm_w = l.norm1;
            q.eps = d.rms_eps;
            q.norm_offset = gemma;
            q.out = e->qkv;
            q.out_stride = e->qkv_rows;
            q.bias = l.bqkv;
            q.err = e->err;
            set_next(q, l.wo, H, QW, 1);
            if (ti_status st = take_recv(q, !lora_on(0))) return st;
            if (next2) {
                q.next2_w = l.wgu;
                q.next2_wfmt = e->wf;
                q.next2_N = I;
                q.next2_K = H;
                q.next2_U = 2;
            }
            if (lora_on(0)) {
                if (ti_status st = prenorm(q)) return st;
                if (ti_status st = shrink(0, q.x, q.x_stride, q.norm_w)) return st;
                set_lora(q, 0);
            }
            return gemm(q, kEpiStore, H, e->qkv_rows, 0);
        }
        case kKAttn: {
            if (fused_ao) return TI_OK;
            int mc = 0;
            const int splits = attn_splits(B, nkv, hd, e->o.max_seq_len, e->sms, &mc);
            AttnArgs at;
            at.qkv = e->qkv;
            at.qkv_stride = e->qkv_rows;
            at.nb = B;
            at.nq = nq;
            at.nkv = nkv;
            at.hd = hd;
            at.pos = e->dd_pos();
            at.seq = e->dd_seq();
            at.page_table = e->page_table;
            at.pt_stride = e->pt_stride;
            at.kc = e->kpool + (size_t)li * e->kv_layer_elems;
            at.vc = e->vpool + (size_t)li * e->kv_layer_elems;
            at.freqs = e->freqs;
            at.scale = 1.0f / sqrtf((float)hd);  // ops.cu:455
            at.window = d.arch == TI_ARCH_MISTRAL ? e->d_desc + 1 : nullptr;
            at.n_pages = e->n_pages;
            at.n_splits = splits;
            at.max_chunk = mc;
            at.part_o = e->part_o;
            at.part_ml = e->part_ml;
            at.counters = e->counters;
            at.out = e->attn;
            at.out_stride = QW;
            at.err = e->err;
            if (prefill) {
                // entries are one sequence at consecutive positions: every K/V row of
                // the step goes into its page first, attention then loads pages after
                // its dependency wait
                TI_CUDA(kv_append_launch(at, s, true));
                if (launches) ++*launches;
                at.prefill = 1;
            }
            TI_CUDA(attn_launch(at, s, true));
            if (launches) ++*launches;
            return TI_OK;
        }
        case kKO: {
            GemvArgs ov;
            ov.W = l.wo;
            ov.wfmt = e->wf;
            ov.N = H;
            ov.K = QW;
            ov.x = e->attn;
            ov.x_stride = QW;
            ov.out = e->res1;
            ov.out_stride = H;
            ov.resid = e->hidden;
            ov.resid_stride = H;
            ov.err = e->err;
            set_next(ov, l.wgu, I, H, 2);
            if (fused_ao) {
                GemvAttn& t = ov.att;
                t.qkv = e->qkv;
                t.nq = nq;
                t.nkv = nkv;
                t.hd = hd;
                t.pos = e->dd_pos();
                t.seq = e->dd_seq();
                t.page_table = e->page_table;
                t.pt_stride = e->pt_stride;
                t.kc = e->kpool + (size_t)li * e->kv_layer_elems;
                t.vc = e->vpool + (size_t)li * e->kv_layer_elems;
                t.n_pages = e->n_pages;
                t.freqs = e->freqs;
                t.scale = 1.0f / sqrtf((float)hd);  // ops.cu:455
                t.window = d.arch == TI_ARCH_MISTRAL ? e->d_desc + 1 : nullptr;
                t.out = e->attn;
                t.part = e->att_part;
                t.ticket = e->att_ticket;
                t.sync = e->att_sync;
            }
            if (lora_on(1)) {
                if (ti_status st = shrink(1, e->attn, QW, nullptr)) return st;
                set_lora(ov, 1);
            }
            if (e->tp.tp > 1) {
                // the expansion runs after the all-reduce, on the full x.A^T
                const GemvLora lo = ov.lora;
                ov.lora = GemvLora{};
                return row_parallel(ov, QW, e->res1, e->hidden, lo.adapter ? &lo : nullptr);
            }
            return gemm(ov, kEpiResid, QW, H, H);
        }
        case kKGateUp: {
            GemvArgs gu;
            gu.W = l.wgu;
            gu.wfmt = e->wf;
            gu.N = I;
            gu.K = H;
            gu.x = e->res1;
            gu.x_stride = H;
            gu.norm_w = l.norm2;
            gu.eps = d.rms_eps;
            gu.norm_offset = gemma;
            gu.out = e->act;
            gu.out_stride = I;
            gu.act = gemma ? 1 : 0;
            gu.err = e->err;
            if (ti_status st = take_recv(gu, !lora_on(2))) return st;
            set_next(gu, l.wdown, H, I, 1);
            if (lora_on(2)) {
                if (ti_status st = prenorm(gu)) return st;
                if (ti_status st = shrink(2, gu.x, gu.x_stride, gu.norm_w)) return st;
                set_lora(gu, 2);
            }
            return gemm(gu, kEpiGlu, H, I, 0);
        }
        case kKDown: {
            GemvArgs dn;
            dn.W = l.wdown;
            dn.wfmt = e->wf;
            dn.N = H;
            dn.K = I;
            dn.x = e->act;
            dn.x_stride = I;
            dn.out = e->hidden;
            dn.out_stride = H;
            dn.resid = e->res1;
            dn.resid_stride = H;
            dn.err = e->err;
            if (li + 1 < d.n_layers) set_next(dn, e->layers[li + 1].wqkv, e->qkv_rows, H, 1);
            else set_next(dn, e->lm_head, e->Vl, H, 1);
            if (lora_on(3)) {
                if (ti_status st = shrink(3, e->act, I, nullptr)) return st;
                set_lora(dn, 3);
            }
            if (e->tp.tp > 1) {
                const GemvLora lo = dn.lora;
                dn.lora = GemvLora{};
                return row_parallel(dn, I, e->hidden, e->res1, lo.adapter ? &lo : nullptr);
            }
            return gemm(dn, kEpiResid, I, H, H);
        }
        default: return fail(TI_ERR_INVALID, "unknown kernel kind %d", kind);
    }
}

// sample: a device chain with top-p / top-k rows; after the LM head (whose greedy
// argmax already advanced every row) the sampler replaces the sampled rows' ids
// in `out` and in the chain's next tokens, each with its row's next pre-generated draw
ti_status enqueue_step(ti_engine* e, int B, cudaStream_t s, int* launches, bool lora, bool prefill,
                       bool sample = false) {
    // row-parallel receives fold into the next GEMV within this step only
    struct FoldScope {
        ti_engine* e;
        explicit FoldScope(ti_engine* x) : e(x) {
            e->fold_recv = e->peer_ar;
            e->pend.on = false;
        }
        ~FoldScope() {
            e->fold_recv = false;
            e->pend.on = false;
        }
    } fold(e);
    if (ti_status st = enqueue_kernel(e, B, kKEmbed, 0, s, launches, lora)) return st;
    for (int li = 0; li < e->d.n_layers; ++li)
        for (int k : {kKQkv, kKAttn, kKO, kKGateUp, kKDown})
            if (ti_status st = enqueue_kernel(e, B, k, li, s, launches, lora, prefill)) return st;
    if (ti_status st = enqueue_kernel(e, B, kKLmHead, 0, s, launches, lora)) return st;
    TI_CHECK(!e->pend.on, TI_ERR_STATE, "a tensor-parallel receive was left without a consumer");
    if (!sample) return TI_OK;
    TI_CHECK(e->d_draws && e->d_srows, TI_ERR_STATE, "sampled device chain: buffers not set up");
    SampleArgs a;
    a.vocab = e->V;
    if (e->tp.tp == 1) {
        a.logits = e->logits;
        a.seg = e->V;
        a.row_stride = (size_t)e->V;
    } else {
        // every rank samples the same gathered rows ([rank][b][j]) with the same draws
        const ncclResult_t r = nccl_api()->AllGather(e->logits, e->lgather, (size_t)B * e->Vl, ncclBfloat16, e->comm,
                                                     s);
        TI_CHECK(r == ncclSuccess, TI_ERR_CUDA, "ncclAllGather (sampled chain): %s", nccl_api()->GetErrorString(r));
        a.logits = e->lgather;
        a.seg = e->Vl;
        a.seg_stride = (size_t)B * e->Vl;
        a.row_stride = (size_t)e->Vl;
    }
    a.rows = e->d_srows;
    a.hist = e->shist;
    a.out = e->out;
    a.err = e->err;
    a.draws = e->d_draws;
    a.draw_cap = e->draw_cap;
    a.draw_ctr = e->d_draw_ctr;
    a.chain_tokens = e->dd_tokens();
    TI_CUDA(sample_launch(a, B, s));
    if (launches) ++*launches;
    return TI_OK;
}

ti_status capture_step(ti_engine* e, int B, bool lora, bool prefill, bool sample, GraphEntry* out) {
    cudaStream_t s = e->cap;
    int launches = 0;
    TI_CUDA(cudaStreamBeginCapture(s, cudaStreamCaptureModeThreadLocal));
    ti_status st = enqueue_step(e, B, s, &launches, lora, prefill, sample);
    cudaGraph_t graph = nullptr;
    cudaError_t ce = cudaStreamEndCapture(s, &graph);
    if (st) {
        if (graph) cudaGraphDestroy(graph);
        cudaGetLastError();
        return st;
    }
    TI_CHECK(ce == cudaSuccess, TI_ERR_CUDA, "cudaStreamEndCapture: %s", cudaGetErrorString(ce));
    cudaGraphExec_t exec = nullptr;
    cudaError_t ie = cudaGraphInstantiate(&exec, graph, 0);
    cudaGraphDestroy(graph);
    TI_CHECK(ie == cudaSuccess, TI_ERR_CUDA, "cudaGraphInstantiate: %s", cudaGetErrorString(ie));
    out->exec = exec;
    out->launches = launches;
    return TI_OK;
}

// one graph per (batch size, LoRA on/off, prefill, sampled device chain)
ti_status get_graph(ti_engine* e, int B, bool lora, GraphEntry** g, bool prefill = false, bool sample = false) {
    lora = lora && e->S > 0;
    const int key = ((B * 2 + (lora ? 1 : 0)) * 2 + (prefill ? 1 : 0)) * 2 + (sample ? 1 : 0);
    auto it = e->graphs.find(key);
    if (it == e->graphs.end()) {
        GraphEntry ge;
        if (ti_status st = capture_step(e, B, lora, prefill, sample, &ge)) return st;
        it = e->graphs.emplace(key, ge).first;
        if (e->tp.tp > 1 && e->comm) {
            // Every rank builds a new graph at the same step; capture, instantiation
            // and first-launch module loading take seconds on large models, so the
            // ranks meet on the host before the graph's cross-rank waits begin.
            const NcclApi* n = nccl_api();
            // one element of the reduction scratch (rewritten before every use in a step);
            // a zero-element collective would not synchronise
            const ncclResult_t r = n->AllReduce(e->red, e->red, 1, ncclFloat32, ncclSum, e->comm, e->tp_sync);
            TI_CHECK(r == ncclSuccess, TI_ERR_CUDA, "ncclAllReduce (rank barrier): %s", n->GetErrorString(r));
            TI_CUDA(cudaStreamSynchronize(e->tp_sync));
        }
    }
    *g = &it->second;
    return TI_OK;
}

// adapters a step uses must exist and be resident; pending prefetches are
// ordered before the step on `stream`
ti_status adapters_ready(ti_engine* e, int B, const int32_t* adapters, cudaStream_t stream, bool* any) {
    *any = false;
    if (!adapters) return TI_OK;
    for (int b = 0; b < B; ++b) {
        const int a = adapters[b];
        if (a < 0) continue;
        TI_CHECK(a < e->S && e->adapters[a].live, TI_ERR_STATE, "unknown adapter %d", a);
        auto& m = e->adapters[a];
        TI_CHECK(m.resident, TI_ERR_STATE, "adapter %d is not resident (ti_adapter_prefetch_async)", a);
        if (m.pending) TI_CUDA(cudaStreamWaitEvent(stream, m.ready, 0));
        *any = true;
    }
    return TI_OK;
}

ti_status seq_check(ti_engine* e, int sid) {
    TI_CHECK(sid >= 0 && sid < (int)e->seqs.size() && e->seqs[sid].live, TI_ERR_STATE, "unknown sequence %d", sid);
    return TI_OK;
}

// ensure pages cover positions [0, upto); page ids appended to `updates` as (seq, idx, page)
ti_status ensure_pages(ti_engine* e, int sid, int upto, std::vector<int32_t>* updates) {
    SeqState& s = e->seqs[sid];
    const int need = (upto + kPageTokens - 1) / kPageTokens;
    TI_CHECK(need <= e->pt_stride, TI_ERR_STATE, "sequence %d: %d tokens exceed max_seq_len %d", sid, upto,
             e->o.max_seq_len);
    while ((int)s.pages.size() < need) {
        TI_CHECK(!e->free_pages.empty(), TI_ERR_OOM, "KV page pool exhausted (%d pages)", e->n_pages);
        const int p = e->free_pages.back();
        e->free_pages.pop_back();
        updates->push_back(sid);
        updates->push_back((int)s.pages.size());
        updates->push_back(p);
        s.pages.push_back(p);
    }
    return TI_OK;
}

ti_status read_err(ti_engine* e, int32_t word) {
    if (word) {
        int zero = 0;
        cudaMemcpy(e->err, &zero, 4, cudaMemcpyHostToDevice);
        return fail(word & (kErrTimeoutFull | kErrTimeoutEmpty | kErrTimeoutPeer | kErrTimeoutGrid) ? TI_ERR_TIMEOUT : TI_ERR_STATE,
                    "device reported error bits 0x%x", word);
    }
    return TI_OK;
}

// the sampler's row parameters and histograms (first sampled step or chain)
ti_status sample_buffers(ti_engine* e) {
    const int MB = e->o.max_batch;
    if (e->d_srows) return TI_OK;
    TI_CHECK(dalloc_t(e, &e->shist, sample_scratch_bytes(MB) / 4, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s",
             ti_last_error());
    TI_CUDA(cudaMallocHost(&e->h_srows, (size_t)MB * sizeof(SampleRow)));
    TI_CHECK(dalloc_t(e, &e->d_srows, (size_t)MB, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s", ti_last_error());
    return TI_OK;
}

// a sequence's sampler as the kernel's row parameters (draw filled by the caller)
SampleRow sample_row(const SeqState& s) {
    SampleRow r{};
    const ti_sampling& c = s.smp.cfg;
    if (c.kind == TI_SAMPLE_GREEDY) return r;
    r.kind = c.kind == TI_SAMPLE_TOP_P ? kSampleTopP : kSampleTopK;
    r.temperature = c.temperature;
    r.p = c.p;
    r.k = (int32_t)std::min<uint32_t>(c.k, 0x7fffffffu);
    return r;
}

// Replace the argmax of every sampled row (a sequence with a top-p / top-k
// sampler; in a prefill step only the last entry's id is returned) by the
// device sampler's pick.  `logits` holds the rows as sample_launch indexes them.
ti_status sample_rows(ti_engine* e, int B, const int32_t* seq_ids, bool prefill, const uint16_t* logits, int seg,
                      size_t seg_stride, size_t row_stride, cudaStream_t stream) {
    if (ti_status st = sample_buffers(e)) return st;
    for (int b = 0; b < B; ++b) {
        SeqState& s = e->seqs[seq_ids[b]];
        SampleRow r{};
        if ((!prefill || b == B - 1) && s.smp.cfg.kind != TI_SAMPLE_GREEDY) {
            r = sample_row(s);
            r.u = s.smp.next();
        }
        e->h_srows[b] = r;
    }
    TI_CUDA(cudaMemcpyAsync(e->d_srows, e->h_srows, (size_t)B * sizeof(SampleRow), cudaMemcpyHostToDevice, stream));
    SampleArgs a;
    a.logits = logits;
    a.vocab = e->V;
    a.seg = seg;
    a.seg_stride = seg_stride;
    a.row_stride = row_stride;
    a.rows = e->d_srows;
    a.hist = e->shist;
    a.out = e->out;
    a.err = e->err;
    TI_CUDA(sample_launch(a, B, stream));
    return TI_OK;
}

// One step for `B` sequences with host inputs; `window` is the sliding window
// applied (prefill semantics) or -1 (decode semantics, as the reference).
// prefill: the B entries are tokens len .. len + B - 1 of one sequence (seq_ids
// all equal), decoded in one step; otherwise B distinct sequences, one token each.
// sample: the returned ids are drawn by the sequences' samplers (greedy ones keep
// the LM head's argmax)
ti_status run_step(ti_engine* e, int B, const int32_t* seq_ids, const int32_t* tokens, const int32_t* adapters,
                   int window, int32_t* next_ids, int logits_mode, void* logits_out, cudaStream_t stream,
                   bool prefill = false, bool sample = false) {
    TI_CHECK(B >= 1 && B <= e->o.max_batch, TI_ERR_INVALID, "batch %d out of range [1, %d]", B, e->o.max_batch);
    TI_CHECK(seq_ids && tokens, TI_ERR_INVALID, "null seq_ids/tokens");
    TI_CHECK(e->bound_batch == 0, TI_ERR_STATE, "engine is bound to a device chain; unbind first");
    std::vector<int32_t> upd;
    for (int b = 0; b < B; ++b) {
        if (ti_status st = seq_check(e, seq_ids[b])) return st;
        if (prefill) {
            TI_CHECK(seq_ids[b] == seq_ids[0], TI_ERR_INVALID, "prefill step: entries of one sequence expected");
        } else {
            for (int c = 0; c < b; ++c)
                TI_CHECK(seq_ids[c] != seq_ids[b], TI_ERR_INVALID, "sequence %d appears twice in one step",
                         seq_ids[b]);
        }
        TI_CHECK(tokens[b] >= 0 && tokens[b] < e->V, TI_ERR_INVALID, "token %d out of range [0, %d)", tokens[b], e->V);
        const int len = e->seqs[seq_ids[b]].len;
        const int need = prefill ? len + B : len + 1;
        TI_CHECK(need <= e->o.max_seq_len, TI_ERR_STATE, "sequence %d is full (%d tokens)", seq_ids[b], len);
        if (!prefill || b == 0)
            if (ti_status st = ensure_pages(e, seq_ids[b], need, &upd)) return st;
    }
    const int MB = e->o.max_batch;
    int32_t* h = e->h_desc;
    h[0] = (int32_t)(upd.size() / 3);
    h[1] = window;
    h[2] = h[3] = 0;
    for (int b = 0; b < B; ++b) {
        h[4 + b] = tokens[b];
        h[4 + MB + b] = seq_ids[b];
        h[4 + 2 * MB + b] = e->seqs[seq_ids[b]].len + (prefill ? b : 0);
        h[4 + 3 * MB + b] = adapters ? adapters[b] : -1;
    }
    TI_CHECK((int)upd.size() <= 3 * MB, TI_ERR_STATE, "too many page updates in one step");
    std::memcpy(h + 4 + 4 * MB, upd.data(), upd.size() * 4);
    bool any_lora = false;
    if (ti_status st = adapters_ready(e, B, adapters, stream, &any_lora)) return st;
    GraphEntry* g = nullptr;
    if (ti_status st = get_graph(e, B, any_lora, &g, prefill)) return st;
    TI_CUDA(cudaMemcpyAsync(e->d_desc, h, (size_t)e->desc_ints * 4, cudaMemcpyHostToDevice, stream));
    TI_CUDA(cudaGraphLaunch(g->exec, stream));
    bool any_sample = false;
    if (sample)
        for (int b = 0; b < B; ++b)
            any_sample |= (!prefill || b == B - 1) && e->seqs[seq_ids[b]].smp.cfg.kind != TI_SAMPLE_GREEDY;
    const bool want_logits = logits_out && logits_mode != TI_LOGITS_NONE;
    // tensor parallelism: every rank's vocabulary slice, gathered [rank][b][j]
    if (e->tp.tp > 1 && (any_sample || want_logits)) {
        const ncclResult_t r = nccl_api()->AllGather(e->logits, e->lgather, (size_t)B * e->Vl, ncclBfloat16, e->comm,
                                                     stream);
        TI_CHECK(r == ncclSuccess, TI_ERR_CUDA, "ncclAllGather: %s", nccl_api()->GetErrorString(r));
    }
    if (any_sample) {
        ti_status st = e->tp.tp == 1
                           ? sample_rows(e, B, seq_ids, prefill, e->logits, e->V, 0, (size_t)e->V, stream)
                           : sample_rows(e, B, seq_ids, prefill, e->lgather, e->Vl, (size_t)B * e->Vl, (size_t)e->Vl,
                                         stream);
        if (st) return st;
    }
    TI_CUDA(cudaMemcpyAsync(e->h_out, e->out, (size_t)(MB + 1) * 4, cudaMemcpyDeviceToHost, stream));
    // host logits [B, V] bf16: the local rows, or every rank's vocabulary slice gathered
    std::vector<uint16_t> lg;
    if (want_logits) {
        lg.resize((size_t)B * e->V);
        if (e->tp.tp == 1) {
            TI_CUDA(cudaMemcpyAsync(lg.data(), e->logits, lg.size() * 2, cudaMemcpyDeviceToHost, stream));
        } else {
            std::vector<uint16_t> gat(lg.size());
            TI_CUDA(cudaMemcpyAsync(gat.data(), e->lgather, gat.size() * 2, cudaMemcpyDeviceToHost, stream));
            TI_CUDA(cudaStreamSynchronize(stream));
            // gathered [rank][b][j] -> [b][rank * Vl + j]
            for (int r2 = 0; r2 < e->tp.tp; ++r2)
                for (int b = 0; b < B; ++b)
                    std::memcpy(&lg[(size_t)b * e->V + (size_t)r2 * e->Vl], &gat[((size_t)r2 * B + b) * e->Vl],
                                (size_t)e->Vl * 2);
        }
    }
    TI_CUDA(cudaStreamSynchronize(stream));
    if (logits_out && logits_mode == TI_LOGITS_BF16) std::memcpy(logits_out, lg.data(), lg.size() * 2);
    if (logits_out && logits_mode == TI_LOGITS_F32) {
        float* f = reinterpret_cast<float*>(logits_out);
        for (size_t i = 0; i < lg.size(); ++i) {
            uint32_t u = (uint32_t)lg[i] << 16;
            std::memcpy(&f[i], &u, 4);
        }
    }
    if (ti_status st = read_err(e, e->h_out[MB])) return st;
    for (int b = 0; b < B; ++b) {
        if (!prefill || b == 0) e->seqs[seq_ids[b]].len += prefill ? B : 1;
        if (next_ids) next_ids[b] = e->h_out[b];
    }
    return TI_OK;
}

}  // namespace

// ==================================================================== C ABI
namespace ti {
// the destination of a reference-named tensor: storage format and full shape
ti_status engine_slot_info(ti_engine* e, const char* name, int* wfmt, size_t* rows, size_t* cols) {
    TI_CHECK(e && name && wfmt && rows && cols, TI_ERR_INVALID, "engine_slot_info: null argument");
    auto it = e->slot_index.find(name);
    TI_CHECK(it != e->slot_index.end(), TI_ERR_NOT_FOUND, "unknown tensor '%s'", name);
    const Slot& s = e->slots[it->second];
    *wfmt = s.wf == kWQ4 ? TI_WFMT_Q4_0 : s.wf == kWQ8 ? TI_WFMT_Q8_0 : TI_WFMT_BF16;
    *rows = s.rows;
    *cols = s.cols;
    return TI_OK;
}
}  // namespace ti

extern "C" {

ti_status ti_engine_create(const ti_model_desc* desc, const ti_engine_opts* opts, ti_engine** out) {
    clear_error();
    TI_CHECK(out, TI_ERR_INVALID, "ti_engine_create: null out");
    *out = nullptr;
    if (ti_status st = validate_desc(desc, opts)) return st;
    int ndev = 0;
    if (cudaGetDeviceCount(&ndev) != cudaSuccess || ndev == 0) {
        cudaGetLastError();
        return fail(TI_ERR_CUDA, "ti_engine_create: no CUDA device");
    }
    TI_CHECK(opts->device >= 0 && opts->device < ndev, TI_ERR_INVALID, "ti_engine_create: device %d of %d",
             opts->device, ndev);
    auto* e = new ti_engine();
    e->d = *desc;
    e->o = *opts;
    if (e->o.tp_size <= 0) e->o.tp_size = 1;
    e->dev = opts->device;
    ti_status st = build(e);
    if (st) {
        std::string msg = ti_last_error();
        free_all(e);
        delete e;
        return fail(st, "%s", msg.c_str());
    }
    *out = e;
    return TI_OK;
}

ti_status ti_engine_destroy(ti_engine* e) {
    if (!e) return TI_OK;
    DeviceGuard g(e->dev);
    cudaDeviceSynchronize();
    free_all(e);
    delete e;
    return TI_OK;
}

ti_status ti_engine_memory(const ti_engine* e, size_t* w, size_t* kv, size_t* ad, size_t* work) {
    TI_CHECK(e, TI_ERR_INVALID, "null engine");
    if (w) *w = e->bytes_w;
    if (kv) *kv = e->bytes_kv;
    if (ad) *ad = e->bytes_ad;
    if (work) *work = e->bytes_work;
    return TI_OK;
}

// GGUF block bytes of one quantised row of K weights
static size_t gguf_row_bytes(int K, int wf) { return (size_t)K / 32 * (wf == kWQ4 ? 18 : 34); }

// A linear weight of a Q4_0 / Q8_0 engine: bf16 rows are quantised on the
// device (the GGUF definition, bit for bit), GGUF blocks are repacked.
static ti_status load_quantized(const Slot& s, const char* name, int dtype, const void* host, size_t bytes) {
    const int K = (int)s.nc;  // local row length (a column window of whole blocks under TP)
    const int gguf = s.wf == kWQ4 ? TI_DTYPE_Q4_0 : TI_DTYPE_Q8_0;
    TI_CHECK(dtype == TI_DTYPE_BF16 || dtype == gguf, TI_ERR_UNSUPPORTED,
             "tensor '%s': dtype %d (bf16 or this engine's GGUF block type expected)", name, dtype);
    const bool bf = dtype == TI_DTYPE_BF16;
    const size_t in_row = bf ? s.cols * 2 : gguf_row_bytes((int)s.cols, s.wf);
    const size_t win = bf ? (size_t)K * 2 : gguf_row_bytes(K, s.wf);
    const size_t win0 = bf ? s.c0 * 2 : gguf_row_bytes((int)s.c0, s.wf);
    TI_CHECK(bytes == s.rows * in_row, TI_ERR_INVALID, "tensor '%s': %zu bytes, expected %zu", name, bytes,
             s.rows * in_row);
    void* tmp = nullptr;
    TI_CUDA(cudaMalloc(&tmp, s.nr * win + 16));
    cudaError_t err = cudaMemcpy2D(tmp, win, reinterpret_cast<const uint8_t*>(host) + s.r0 * in_row + win0, in_row,
                                   win, s.nr, cudaMemcpyHostToDevice);
    if (err == cudaSuccess)
        err = dtype == TI_DTYPE_BF16
                  ? quantize_rows_launch(reinterpret_cast<const uint16_t*>(tmp), (int)s.nr, K, K, s.qdst, s.rb, s.wf, 0)
                  : repack_gguf_launch(reinterpret_cast<const uint8_t*>(tmp), (int)s.nr, K, s.qdst, s.rb, s.wf, 0);
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    cudaFree(tmp);
    TI_CHECK(err == cudaSuccess, TI_ERR_CUDA, "tensor '%s': %s", name, cudaGetErrorString(err));
    return TI_OK;
}

ti_status ti_engine_load_tensor(ti_engine* e, const char* name, int dtype, const void* host, size_t bytes) {
    clear_error();
    TI_CHECK(e && name && host, TI_ERR_INVALID, "ti_engine_load_tensor: null argument");
    auto it = e->slot_index.find(name);
    TI_CHECK(it != e->slot_index.end(), TI_ERR_NOT_FOUND, "unknown tensor '%s'", name);
    const Slot& s = e->slots[it->second];
    if (s.wf != kWBf16) {
        DeviceGuard g(e->dev);
        return load_quantized(s, name, dtype, host, bytes);
    }
    TI_CHECK(dtype == TI_DTYPE_BF16, TI_ERR_UNSUPPORTED, "tensor '%s': dtype %d (bf16 expected)", name, dtype);
    TI_CHECK(bytes == s.rows * s.cols * 2, TI_ERR_INVALID, "tensor '%s': %zu bytes, expected %zu", name, bytes,
             s.rows * s.cols * 2);
    DeviceGuard g(e->dev);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(host) + (s.r0 * s.cols + s.c0) * 2;
    TI_CUDA(cudaMemcpy2D(s.dst, s.ld * 2, src, s.cols * 2, s.nc * 2, s.nr, cudaMemcpyHostToDevice));
    return TI_OK;
}

ti_status ti_engine_set_rope_freqs(ti_engine* e, const float* inv_freq, int n) {
    clear_error();
    TI_CHECK(e && inv_freq, TI_ERR_INVALID, "ti_engine_set_rope_freqs: null argument");
    TI_CHECK(n == e->hd / 2, TI_ERR_INVALID, "ti_engine_set_rope_freqs: %d values, head_dim / 2 = %d expected", n,
             e->hd / 2);
    DeviceGuard g(e->dev);
    TI_CUDA(cudaMemcpy(e->freqs, inv_freq, (size_t)n * 4, cudaMemcpyHostToDevice));
    return TI_OK;
}

ti_status ti_engine_read_tensor(ti_engine* e, const char* name, void* host, size_t bytes) {
    clear_error();
    TI_CHECK(e && name && host, TI_ERR_INVALID, "ti_engine_read_tensor: null argument");
    auto it = e->slot_index.find(name);
    TI_CHECK(it != e->slot_index.end(), TI_ERR_NOT_FOUND, "unknown tensor '%s'", name);
    const Slot& s = e->slots[it->second];
    if (s.wf != kWBf16) {
        // quantised linear weight: the window's rows as GGUF blocks
        const size_t gb = gguf_row_bytes((int)s.nc, s.wf);
        TI_CHECK(bytes == s.nr * gb, TI_ERR_INVALID, "tensor '%s': %zu bytes, local window is %zu GGUF bytes", name,
                 bytes, s.nr * gb);
        DeviceGuard g(e->dev);
        std::vector<uint8_t> rows(s.nr * s.rb);
        TI_CUDA(cudaMemcpy(rows.data(), s.qdst, rows.size(), cudaMemcpyDeviceToHost));
        gguf_from_rows(rows.data(), (int)s.nr, (int)s.nc, s.rb, s.wf, reinterpret_cast<uint8_t*>(host));
        return TI_OK;
    }
    TI_CHECK(bytes == s.nr * s.nc * 2, TI_ERR_INVALID, "tensor '%s': %zu bytes, local window is %zu", name, bytes,
             s.nr * s.nc * 2);
    DeviceGuard g(e->dev);
    TI_CUDA(cudaMemcpy2D(host, s.nc * 2, s.dst, s.ld * 2, s.nc * 2, s.nr, cudaMemcpyDeviceToHost));
    return TI_OK;
}

ti_status ti_engine_init_synthetic(ti_engine* e, uint64_t seed, float std_) {
    clear_error();
    TI_CHECK(e, TI_ERR_INVALID, "null engine");
    DeviceGuard g(e->dev);
    const float c = synth_scale(std_);
    // quantised slots: the bf16 values the other formats get, then quantised
    size_t tmp_elems = 0;
    for (const Slot& s : e->slots)
        if (s.wf != kWBf16) tmp_elems = std::max(tmp_elems, s.nr * s.nc);
    uint16_t* tmp = nullptr;
    if (tmp_elems) TI_CUDA(cudaMalloc(&tmp, tmp_elems * 2));
    cudaError_t err = cudaSuccess;
    for (const Slot& s : e->slots) {
        if (err != cudaSuccess) break;
        if (s.wf == kWBf16) {
            err = synth_bf16_launch(s.dst, s.nr, s.nc, s.ld, s.r0, s.c0, s.cols, seed, fnv1a(s.name.c_str()), c,
                                    (cudaStream_t)0);
        } else {
            err = synth_bf16_launch(tmp, s.nr, s.nc, s.nc, s.r0, s.c0, s.cols, seed, fnv1a(s.name.c_str()), c,
                                    (cudaStream_t)0);
            if (err == cudaSuccess)
                err = quantize_rows_launch(tmp, (int)s.nr, (int)s.nc, s.nc, s.qdst, s.rb, s.wf, (cudaStream_t)0);
        }
    }
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    if (tmp) cudaFree(tmp);
    TI_CHECK(err == cudaSuccess, TI_ERR_CUDA, "init_synthetic: %s", cudaGetErrorString(err));
    return TI_OK;
}

ti_status ti_seq_create(ti_engine* e, int* sid) {
    clear_error();
    TI_CHECK(e && sid, TI_ERR_INVALID, "null argument");
    for (int i = 0; i < (int)e->seqs.size(); ++i)
        if (!e->seqs[i].live) {
            e->seqs[i] = SeqState{};
            e->seqs[i].live = true;
            *sid = i;
            return TI_OK;
        }
    return fail(TI_ERR_OOM, "all %d sequence slots in use", (int)e->seqs.size());
}

static void release_pages(ti_engine* e, int sid) {
    SeqState& s = e->seqs[sid];
    for (int p : s.pages) e->free_pages.push_back(p);
    if (!s.pages.empty()) {
        DeviceGuard g(e->dev);
        std::vector<int32_t> neg(s.pages.size(), -1);
        cudaMemcpy(e->page_table + (size_t)sid * e->pt_stride, neg.data(), neg.size() * 4, cudaMemcpyHostToDevice);
    }
    s.pages.clear();
    s.len = 0;
}

ti_status ti_seq_free(ti_engine* e, int sid) {
    clear_error();
    TI_CHECK(e, TI_ERR_INVALID, "null engine");
    if (ti_status st = seq_check(e, sid)) return st;
    release_pages(e, sid);
    e->seqs[sid].live = false;
    return TI_OK;
}

ti_status ti_seq_reset(ti_engine* e, int sid) {
    clear_error();
    TI_CHECK(e, TI_ERR_INVALID, "null engine");
    if (ti_status st = seq_check(e, sid)) return st;
    release_pages(e, sid);
    return TI_OK;
}

ti_status ti_engine_seq_set_sampler(ti_engine* e, int sid, const ti_sampling* smp) {
    clear_error();
    TI_CHECK(e, TI_ERR_INVALID, "null engine");
    if (ti_status st = seq_check(e, sid)) return st;
    const ti_sampling greedy{};
    const ti_sampling& s = smp ? *smp : greedy;
    if (ti_status st = sampler_check(s)) return st;
    TI_CHECK(e->tp.tp == 1 || s.kind == TI_SAMPLE_GREEDY || s.seeded, TI_ERR_INVALID,
             "tensor-parallel ranks draw the same ids only from a seeded sampler");
    e->seqs[sid].smp.reset(s);
    return TI_OK;
}

ti_status ti_seq_len(ti_engine* e, int sid, int* len) {
    TI_CHECK(e && len, TI_ERR_INVALID, "null argument");
    if (ti_status st = seq_check(e, sid)) return st;
    *len = e->seqs[sid].len;
    return TI_OK;
}

ti_status ti_seq_reserve(ti_engine* e, int sid, int n_tokens) {
    clear_error();
    TI_CHECK(e, TI_ERR_INVALID, "null engine");
    if (ti_status st = seq_check(e, sid)) return st;
    std::vector<int32_t> upd;
    if (ti_status st = ensure_pages(e, sid, n_tokens, &upd)) return st;
    DeviceGuard g(e->dev);
    for (size_t i = 0; i < upd.size(); i += 3)
        TI_CUDA(cudaMemcpy(e->page_table + (size_t)upd[i] * e->pt_stride + upd[i + 1], &upd[i + 2], 4,
                           cudaMemcpyHostToDevice));
    return TI_OK;
}

ti_status ti_seq_fill_synthetic(ti_engine* e, int sid, int n_tokens, uint64_t seed, float std_) {
    clear_error();
    TI_CHECK(e, TI_ERR_INVALID, "null engine");
    if (ti_status st = seq_check(e, sid)) return st;
    TI_CHECK(n_tokens >= 0 && n_tokens < e->o.max_seq_len, TI_ERR_INVALID, "n_tokens %d out of [0, %d)", n_tokens,
             e->o.max_seq_len);
    std::vector<int32_t> upd;
    if (ti_status st = ensure_pages(e, sid, n_tokens, &upd)) return st;
    DeviceGuard g(e->dev);
    for (size_t i = 0; i < upd.size(); i += 3)
        TI_CUDA(cudaMemcpy(e->page_table + (size_t)upd[i] * e->pt_stride + upd[i + 1], &upd[i + 2], 4,
                           cudaMemcpyHostToDevice));
    const std::vector<int>& pages = e->seqs[sid].pages;
    int32_t* dpages = nullptr;
    TI_CUDA(cudaMalloc(&dpages, std::max<size_t>(1, pages.size()) * 4));
    cudaError_t err = cudaMemcpy(dpages, pages.data(), pages.size() * 4, cudaMemcpyHostToDevice);
    if (err == cudaSuccess)
        err = fill_kv_launch(e->kpool, e->vpool, e->kv_layer_elems, e->d.n_layers, dpages, n_tokens, e->nkv,
                             e->tp.kv0, e->d.n_kv_heads, e->hd, mix64(seed ^ fnv1a("kv.k")), mix64(seed ^ fnv1a("kv.v")),
                             synth_scale(std_), 0);
    if (err == cudaSuccess) err = cudaDeviceSynchronize();
    cudaFree(dpages);
    TI_CHECK(err == cudaSuccess, TI_ERR_CUDA, "seq_fill_synthetic: %s", cudaGetErrorString(err));
    e->seqs[sid].len = n_tokens;
    return TI_OK;
}

ti_status ti_seq_read_kv(ti_engine* e, int sid, int layer, int which, void* host, int len) {
    clear_error();
    TI_CHECK(e && host, TI_ERR_INVALID, "null argument");
    if (ti_status st = seq_check(e, sid)) return st;
    TI_CHECK(layer >= 0 && layer < e->d.n_layers, TI_ERR_INVALID, "layer %d out of range", layer);
    const SeqState& s = e->seqs[sid];
    TI_CHECK(len >= 0 && len <= s.len, TI_ERR_INVALID, "len %d > sequence length %d", len, s.len);
    DeviceGuard g(e->dev);
    const uint16_t* pool = (which ? e->vpool : e->kpool) + (size_t)layer * e->kv_layer_elems;
    uint16_t* out = reinterpret_cast<uint16_t*>(host);
    const int hd = e->hd, nkv = e->nkv;
    std::vector<uint16_t> page((size_t)nkv * kPageTokens * hd);
    for (int p = 0; p * kPageTokens < len; ++p) {
        TI_CUDA(cudaMemcpy(page.data(), pool + (size_t)s.pages[p] * nkv * kPageTokens * hd, page.size() * 2,
                           cudaMemcpyDeviceToHost));
        for (int t = 0; t < kPageTokens && p * kPageTokens + t < len; ++t)
            for (int h = 0; h < nkv; ++h)
                std::memcpy(out + ((size_t)(p * kPageTokens + t) * nkv + h) * hd,
                            page.data() + ((size_t)h * kPageTokens + t) * hd, (size_t)hd * 2);
    }
    return TI_OK;
}

ti_status ti_engine_prefill(ti_engine* e, int sid, const int32_t* ids, int n, int adapter_id, int32_t* next_id,
                            int logits_mode, void* logits_out) {
    clear_error();
    TI_CHECK(e && ids, TI_ERR_INVALID, "null argument");
    TI_CHECK(n >= 1, TI_ERR_INVALID, "prefill: empty prompt");  // llama_model.cpp:212
    DeviceGuard g(e->dev);
    const int window = e->d.arch == TI_ARCH_MISTRAL ? e->d.sliding_window : -1;
    int32_t ad = adapter_id;
    for (int i = 0; i < n; ++i) {
        const bool last = i == n - 1;
        ti_status st = run_step(e, 1, &sid, ids + i, adapter_id >= 0 ? &ad : nullptr, window, last ? next_id : nullptr,
                                last ? logits_mode : TI_LOGITS_NONE, last ? logits_out : nullptr, e->cap, false, last);
        if (st) return st;
    }
    return TI_OK;
}

ti_status ti_engine_prefill_chunked(ti_engine* e, int sid, const int32_t* ids, int n, int adapter_id, int chunk,
                                    int32_t* next_id, int logits_mode, void* logits_out) {
    clear_error();
    TI_CHECK(e && ids, TI_ERR_INVALID, "null argument");
    TI_CHECK(n >= 1, TI_ERR_INVALID, "prefill: empty prompt");  // llama_model.cpp:212
    TI_CHECK(chunk >= 1, TI_ERR_INVALID, "prefill: chunk must be >= 1");
    DeviceGuard g(e->dev);
    chunk = std::min(chunk, e->o.max_batch);
    const int window = e->d.arch == TI_ARCH_MISTRAL ? e->d.sliding_window : -1;
    const size_t row_bytes = (size_t)e->V * (logits_mode == TI_LOGITS_F32 ? 4 : 2);
    std::vector<int32_t> sids((size_t)chunk, sid), ads((size_t)chunk, adapter_id), nexts((size_t)chunk);
    std::vector<uint8_t> lg;
    for (int i0 = 0; i0 < n; i0 += chunk) {
        const int m = std::min(chunk, n - i0);
        const bool last = i0 + m == n;
        const bool want = last && logits_out && logits_mode != TI_LOGITS_NONE;
        if (want) lg.resize((size_t)m * row_bytes);
        ti_status st = run_step(e, m, sids.data(), ids + i0, adapter_id >= 0 ? ads.data() : nullptr, window,
                                nexts.data(), want ? logits_mode : TI_LOGITS_NONE, want ? lg.data() : nullptr, e->cap,
                                m > 1, last);
        if (st) return st;
        if (last) {
            if (next_id) *next_id = nexts[m - 1];
            if (want) std::memcpy(logits_out, lg.data() + (size_t)(m - 1) * row_bytes, row_bytes);
        }
    }
    return TI_OK;
}

ti_status ti_engine_decode(ti_engine* e, int batch, const int32_t* seq_ids, const int32_t* tokens,
                           const int32_t* adapter_ids, int32_t* next_ids, int logits_mode, void* logits_out,
                           void* stream) {
    clear_error();
    TI_CHECK(e, TI_ERR_INVALID, "null engine");
    DeviceGuard g(e->dev);
    return run_step(e, batch, seq_ids, tokens, adapter_ids, -1, next_ids, logits_mode, logits_out,
                    (cudaStream_t)stream, false, true);
}

ti_status ti_engine_bind(ti_engine* e, int B, const int32_t* seq_ids, const int32_t* first_tokens,
                         const int32_t* adapter_ids) {
    clear_error();
    TI_CHECK(e && seq_ids && first_tokens, TI_ERR_INVALID, "null argument");
    TI_CHECK(B >= 1 && B <= e->o.max_batch, TI_ERR_INVALID, "batch %d out of range", B);
    TI_CHECK(e->bound_batch == 0, TI_ERR_STATE, "engine already bound");
    DeviceGuard g(e->dev);
    const int MB = e->o.max_batch;
    int32_t* h = e->h_desc;
    std::memset(h, 0, (size_t)e->desc_ints * 4);
    h[1] = -1;
    for (int b = 0; b < B; ++b) {
        if (ti_status st = seq_check(e, seq_ids[b])) return st;
        TI_CHECK(first_tokens[b] >= 0 && first_tokens[b] < e->V, TI_ERR_INVALID, "token out of range");
        const SeqState& s = e->seqs[seq_ids[b]];
        TI_CHECK((int)s.pages.size() * kPageTokens > s.len, TI_ERR_STATE,
                 "sequence %d has no reserved page for its next token (ti_seq_reserve)", seq_ids[b]);
        h[4 + b] = first_tokens[b];
        h[4 + MB + b] = seq_ids[b];
        h[4 + 2 * MB + b] = s.len;
        h[4 + 3 * MB + b] = adapter_ids ? adapter_ids[b] : -1;
    }
    bool any_lora = false;
    if (ti_status st = adapters_ready(e, B, adapter_ids, (cudaStream_t)0, &any_lora)) return st;
    bool any_sample = false;
    for (int b = 0; b < B; ++b) any_sample |= e->seqs[seq_ids[b]].smp.cfg.kind != TI_SAMPLE_GREEDY;
    if (any_sample) {
        // every step the chain can take (up to the sequence's reserved pages) gets its
        // draw now, from a copy of the sequence's engine; unbind advances the engine itself
        if (ti_status st = sample_buffers(e)) return st;
        if (!e->d_draws) {
            e->draw_cap = e->o.max_seq_len;
            TI_CHECK(dalloc_t(e, &e->d_draws, (size_t)MB * e->draw_cap, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s",
                     ti_last_error());
            TI_CHECK(dalloc_t(e, &e->d_draw_ctr, (size_t)MB, &e->bytes_work) == TI_OK, TI_ERR_OOM, "%s",
                     ti_last_error());
        }
        std::vector<float> draws((size_t)B * e->draw_cap, 0.0f);
        for (int b = 0; b < B; ++b) {
            const SeqState& s = e->seqs[seq_ids[b]];
            e->h_srows[b] = sample_row(s);
            if (s.smp.cfg.kind == TI_SAMPLE_GREEDY) continue;
            SamplerDraws ahead = s.smp;
            const int n = std::min(e->draw_cap, (int)s.pages.size() * kPageTokens - s.len);
            for (int i = 0; i < n; ++i) draws[(size_t)b * e->draw_cap + i] = ahead.next();
        }
        TI_CUDA(cudaMemcpy(e->d_srows, e->h_srows, (size_t)B * sizeof(SampleRow), cudaMemcpyHostToDevice));
        TI_CUDA(cudaMemcpy(e->d_draws, draws.data(), draws.size() * 4, cudaMemcpyHostToDevice));
        TI_CUDA(cudaMemset(e->d_draw_ctr, 0, (size_t)MB * 4));
    }
    GraphEntry* gr = nullptr;
    if (ti_status st = get_graph(e, B, any_lora, &gr, false, any_sample)) return st;
    TI_CUDA(cudaMemcpy(e->d_desc, h, (size_t)e->desc_ints * 4, cudaMemcpyHostToDevice));
    e->bound_batch = B;
    e->bound_lora = any_lora;
    e->bound_sample = any_sample;
    e->bound_seqs.assign(seq_ids, seq_ids + B);
    return TI_OK;
}

ti_status ti_engine_decode_device(ti_engine* e, void* stream) {
    TI_CHECK(e && e->bound_batch > 0, TI_ERR_STATE, "engine not bound");
    // stream 0 is the engine device's default stream (unbind reads the ids there): without
    // the guard a caller whose current device is another one would launch the step on that
    // device's default stream, unordered with unbind's copy
    DeviceGuard dg(e->dev);
    GraphEntry* g = nullptr;
    if (ti_status st = get_graph(e, e->bound_batch, e->bound_lora, &g, false, e->bound_sample)) return st;
    TI_CUDA(cudaGraphLaunch(g->exec, (cudaStream_t)stream));
    return TI_OK;
}

ti_status ti_engine_unbind(ti_engine* e, int steps, int32_t* last_ids, void* stream) {
    clear_error();
    TI_CHECK(e && e->bound_batch > 0, TI_ERR_STATE, "engine not bound");
    DeviceGuard g(e->dev);
    const int MB = e->o.max_batch;
    TI_CUDA(cudaMemcpyAsync(e->h_out, e->out, (size_t)(MB + 1) * 4, cudaMemcpyDeviceToHost, (cudaStream_t)stream));
    TI_CUDA(cudaStreamSynchronize((cudaStream_t)stream));
    const int B = e->bound_batch;
    for (int b = 0; b < B; ++b) {
        SeqState& s = e->seqs[e->bound_seqs[b]];
        s.len = std::min(s.len + steps, e->o.max_seq_len);
        if (last_ids) last_ids[b] = e->h_out[b];
        // a top-p sequence's engine moves past the draws its chain consumed
        if (e->bound_sample && s.smp.cfg.kind == TI_SAMPLE_TOP_P)
            for (int i = 0; i < steps; ++i) s.smp.next();
    }
    e->bound_batch = 0;
    e->bound_sample = false;
    e->bound_seqs.clear();
    return read_err(e, e->h_out[MB]);
}

ti_status ti_engine_logits_device(ti_engine* e, void** ptr) {
    TI_CHECK(e && ptr, TI_ERR_INVALID, "null argument");
    *ptr = e->logits;
    return TI_OK;
}

ti_status ti_engine_check(ti_engine* e) {
    TI_CHECK(e, TI_ERR_INVALID, "null engine");
    DeviceGuard g(e->dev);
    int32_t w = 0;
    TI_CUDA(cudaMemcpy(&w, e->err, 4, cudaMemcpyDeviceToHost));
    return read_err(e, w);
}

ti_status ti_engine_launch_kernel(ti_engine* e, int kind, int layer, int batch, void* stream) {
    TI_CHECK(e, TI_ERR_INVALID, "null engine");
    TI_CHECK(batch >= 1 && batch <= e->o.max_batch, TI_ERR_INVALID, "batch %d out of range", batch);
    DeviceGuard g(e->dev);
    return enqueue_kernel(e, batch, kind, layer, (cudaStream_t)stream, nullptr, false);
}

ti_status ti_engine_launches_per_step(ti_engine* e, int batch, int* launches) {
    TI_CHECK(e && launches, TI_ERR_INVALID, "null argument");
    DeviceGuard g(e->dev);
    GraphEntry* gr = nullptr;
    if (ti_status st = get_graph(e, batch, false, &gr)) return st;
    *launches = gr->launches;
    return TI_OK;
}

}  // extern "C"

// ==================================================================== LoRA adapters
namespace {

const char* kLoraProj[7] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                            "mlp.gate_proj",    "mlp.up_proj",      "mlp.down_proj"};
const int kLoraKind[7] = {0, 0, 0, 1, 2, 2, 3};

// projection p's (out, in) and where its A section / B rows sit in the kind's pool
void lora_geometry(const ti_engine* e, int p, int* out, int* in, int* a_sec, int* b_row0) {
    const int QW = e->nq * e->hd, KW = e->nkv * e->hd;
    const int outs[7] = {QW, KW, KW, e->H, e->I, e->I, e->H};
    const int ins[7] = {e->H, e->H, e->H, QW, e->H, e->H, e->I};
    const int secs[7] = {0, 1, 2, 0, 0, 1, 0};
    const int rows0[7] = {0, QW, QW + KW, 0, 0, e->I, 0};
    *out = outs[p];
    *in = ins[p];
    *a_sec = secs[p];
    *b_row0 = rows0[p];
}

// Under tensor parallelism an adapter tensor is a window of the full one: B rows
// of the local output rows (q, k, v, gate, up) or A columns of the local input
// columns (o, down).  Full shapes, window origin.
void lora_window(const ti_engine* e, int p, int* out_full, int* in_full, int* b_r0, int* a_c0) {
    const int hd = e->hd, H = e->H;
    const int QWg = e->d.n_heads * hd, KWg = e->d.n_kv_heads * hd, Ig = e->d.intermediate;
    const int outs[7] = {QWg, KWg, KWg, H, Ig, Ig, H};
    const int ins[7] = {H, H, H, QWg, H, H, Ig};
    const int r0[7] = {e->tp.q0 * hd, e->tp.kv0 * hd, e->tp.kv0 * hd, 0, e->tp.i0, e->tp.i0, 0};
    const int c0[7] = {0, 0, 0, e->tp.q0 * hd, 0, 0, e->tp.i0};
    *out_full = outs[p];
    *in_full = ins[p];
    *b_r0 = r0[p];
    *a_c0 = c0[p];
}

uint16_t* lora_A(ti_engine* e, int ad, int layer, int p) {
    const int k = kLoraKind[p];
    int out, in, sec, row0;
    lora_geometry(e, p, &out, &in, &sec, &row0);
    return e->lA[k] + ((size_t)ad * e->d.n_layers + layer) * e->lA_layer[k] + (size_t)sec * e->R * e->lK[k];
}
uint16_t* lora_B(ti_engine* e, int ad, int layer, int p) {
    const int k = kLoraKind[p];
    int out, in, sec, row0;
    lora_geometry(e, p, &out, &in, &sec, &row0);
    return e->lB[k] + ((size_t)ad * e->d.n_layers + layer) * e->lB_layer[k] + (size_t)row0 * e->R;
}

ti_status adapter_check(ti_engine* e, int id) {
    TI_CHECK(e, TI_ERR_INVALID, "null engine");
    TI_CHECK(e->S > 0, TI_ERR_STATE, "engine created without adapter slots (max_adapters = 0)");
    TI_CHECK(id >= 0 && id < e->S && e->adapters[id].live, TI_ERR_STATE, "unknown adapter %d", id);
    return TI_OK;
}

// the adapter's device regions, kind by kind (A then B): (pointer, elements)
std::vector<std::pair<uint16_t*, size_t>> adapter_regions(ti_engine* e, int id) {
    std::vector<std::pair<uint16_t*, size_t>> r;
    for (int k = 0; k < 4; ++k) {
        if (!e->lA[k]) continue;
        const size_t na = e->lA_layer[k] * e->d.n_layers, nb = e->lB_layer[k] * e->d.n_layers;
        r.push_back({e->lA[k] + (size_t)id * na, na});
        r.push_back({e->lB[k] + (size_t)id * nb, nb});
    }
    return r;
}

}  // namespace

extern "C" {

ti_status ti_adapter_create(ti_engine* e, int rank, float alpha, int proj_mask, int* adapter_id) {
    clear_error();
    TI_CHECK(e && adapter_id, TI_ERR_INVALID, "null argument");
    TI_CHECK(e->S > 0, TI_ERR_STATE, "engine created without adapter slots (max_adapters = 0)");
    TI_CHECK(rank >= 1 && rank <= e->R, TI_ERR_INVALID, "adapter rank %d outside [1, %d]", rank, e->R);
    TI_CHECK(proj_mask != 0 && (proj_mask & ~e->lmask) == 0, TI_ERR_INVALID,
             "adapter projections 0x%x not within the engine's lora_proj_mask 0x%x", proj_mask, e->lmask);
    int id = -1;
    for (int i = 0; i < e->S; ++i)
        if (!e->adapters[i].live) {
            id = i;
            break;
        }
    TI_CHECK(id >= 0, TI_ERR_OOM, "all %d adapter slots in use", e->S);
    DeviceGuard g(e->dev);
    for (auto& reg : adapter_regions(e, id)) TI_CUDA(cudaMemset(reg.first, 0, reg.second * 2));
    const float scale = alpha / (float)rank;  // AdapterWeights::scale, adapter_weights.hpp:85
    TI_CUDA(cudaMemcpy(e->lscale + id, &scale, 4, cudaMemcpyHostToDevice));
    auto& m = e->adapters[id];
    m.live = true;
    m.rank = rank;
    m.alpha = alpha;
    m.mask = proj_mask;
    m.resident = true;
    m.pending = false;
    *adapter_id = id;
    return TI_OK;
}

ti_status ti_adapter_load_tensor(ti_engine* e, int id, const char* name, const void* host, size_t bytes) {
    clear_error();
    if (ti_status st = adapter_check(e, id)) return st;
    TI_CHECK(name && host, TI_ERR_INVALID, "null argument");
    // "layers.{i}.{proj}.lora_A|B" (adapter_loader.cpp:180-222)
    const std::string nm(name);
    int layer = -1, p = -1;
    char which = 0;
    if (nm.rfind("layers.", 0) == 0 && nm.size() > 14 && nm.compare(nm.size() - 7, 6, ".lora_") == 0) {
        which = nm.back();
        const size_t dot = nm.find('.', 7);
        if (dot != std::string::npos) {
            layer = std::atoi(nm.substr(7, dot - 7).c_str());
            const std::string pr = nm.substr(dot + 1, nm.size() - 7 - dot - 1);
            for (int i = 0; i < 7; ++i)
                if (pr == kLoraProj[i]) p = i;
        }
    }
    TI_CHECK(p >= 0 && (which == 'A' || which == 'B') && layer >= 0 && layer < e->d.n_layers, TI_ERR_NOT_FOUND,
             "unknown adapter tensor '%s'", name);
    const auto& m = e->adapters[id];
    TI_CHECK(m.mask & (1 << p), TI_ERR_INVALID, "adapter %d does not inject %s", id, kLoraProj[p]);
    int out, in, sec, row0, out_f, in_f, b_r0, a_c0;
    lora_geometry(e, p, &out, &in, &sec, &row0);
    lora_window(e, p, &out_f, &in_f, &b_r0, &a_c0);
    DeviceGuard g(e->dev);
    const uint8_t* src = reinterpret_cast<const uint8_t*>(host);
    if (which == 'A') {  // [rank, in], flat accepted (adapter_loader.cpp:67-81); local input columns
        TI_CHECK(bytes == (size_t)m.rank * in_f * 2, TI_ERR_INVALID, "%s: %zu bytes, expected %zu", name, bytes,
                 (size_t)m.rank * in_f * 2);
        TI_CUDA(cudaMemcpy2D(lora_A(e, id, layer, p), (size_t)in * 2, src + (size_t)a_c0 * 2, (size_t)in_f * 2,
                             (size_t)in * 2, m.rank, cudaMemcpyHostToDevice));
    } else {  // [out, rank] into rows of padded width R (adapter_loader.cpp:83-95); local output rows
        TI_CHECK(bytes == (size_t)out_f * m.rank * 2, TI_ERR_INVALID, "%s: %zu bytes, expected %zu", name, bytes,
                 (size_t)out_f * m.rank * 2);
        TI_CUDA(cudaMemcpy2D(lora_B(e, id, layer, p), (size_t)e->R * 2, src + (size_t)b_r0 * m.rank * 2,
                             (size_t)m.rank * 2, (size_t)m.rank * 2, out, cudaMemcpyHostToDevice));
    }
    return TI_OK;
}

ti_status ti_adapter_init_synthetic(ti_engine* e, int id, uint64_t seed, float std_a, float std_b) {
    clear_error();
    if (ti_status st = adapter_check(e, id)) return st;
    DeviceGuard g(e->dev);
    const auto& m = e->adapters[id];
    const float ca = synth_scale(std_a), cb = synth_scale(std_b);
    for (int layer = 0; layer < e->d.n_layers; ++layer)
        for (int p = 0; p < 7; ++p) {
            if (!(m.mask & (1 << p))) continue;
            int out, in, sec, row0, out_f, in_f, b_r0, a_c0;
            lora_geometry(e, p, &out, &in, &sec, &row0);
            lora_window(e, p, &out_f, &in_f, &b_r0, &a_c0);
            const std::string base = "layers." + std::to_string(layer) + "." + kLoraProj[p];
            // windows of the full tensors' synthetic values (identical to a single-GPU engine's)
            TI_CUDA(synth_bf16_launch(lora_A(e, id, layer, p), m.rank, in, in, 0, a_c0, in_f, seed,
                                      fnv1a((base + ".lora_A").c_str()), ca, (cudaStream_t)0));
            TI_CUDA(synth_bf16_launch(lora_B(e, id, layer, p), out, m.rank, e->R, b_r0, 0, m.rank, seed,
                                      fnv1a((base + ".lora_B").c_str()), cb, (cudaStream_t)0));
        }
    TI_CUDA(cudaDeviceSynchronize());
    return TI_OK;
}

ti_status ti_adapter_stage_host(ti_engine* e, int id) {
    clear_error();
    if (ti_status st = adapter_check(e, id)) return st;
    DeviceGuard g(e->dev);
    auto& m = e->adapters[id];
    TI_CHECK(m.resident, TI_ERR_STATE, "adapter %d is not resident", id);
    const auto regs = adapter_regions(e, id);
    size_t total = 0;
    for (auto& r : regs) total += r.second * 2;
    if (!m.host) TI_CUDA(cudaMallocHost(&m.host, total));
    size_t off = 0;
    for (auto& r : regs) {
        TI_CUDA(cudaMemcpy(static_cast<uint8_t*>(m.host) + off, r.first, r.second * 2, cudaMemcpyDeviceToHost));
        off += r.second * 2;
    }
    return TI_OK;
}

ti_status ti_adapter_evict(ti_engine* e, int id) {
    clear_error();
    if (ti_status st = adapter_check(e, id)) return st;
    auto& m = e->adapters[id];
    TI_CHECK(m.host, TI_ERR_STATE, "adapter %d has no host copy (ti_adapter_stage_host first)", id);
    DeviceGuard g(e->dev);
    if (m.pending) TI_CUDA(cudaEventSynchronize(m.ready));
    for (auto& r : adapter_regions(e, id)) TI_CUDA(cudaMemset(r.first, 0, r.second * 2));
    TI_CUDA(cudaDeviceSynchronize());
    m.resident = false;
    m.pending = false;
    return TI_OK;
}

// pinned host -> HBM on the engine's side stream; steps that use the adapter
// wait on the copy's event (adapters_ready) instead of the host
ti_status ti_adapter_prefetch_async(ti_engine* e, int id) {
    clear_error();
    if (ti_status st = adapter_check(e, id)) return st;
    auto& m = e->adapters[id];
    TI_CHECK(m.host, TI_ERR_STATE, "adapter %d has no host copy (ti_adapter_stage_host first)", id);
    if (m.resident && !m.pending) return TI_OK;
    DeviceGuard g(e->dev);
    size_t off = 0;
    for (auto& r : adapter_regions(e, id)) {
        TI_CUDA(cudaMemcpyAsync(r.first, static_cast<const uint8_t*>(m.host) + off, r.second * 2,
                                cudaMemcpyHostToDevice, e->side));
        off += r.second * 2;
    }
    if (!m.ready) TI_CUDA(cudaEventCreateWithFlags(&m.ready, cudaEventDisableTiming));
    TI_CUDA(cudaEventRecord(m.ready, e->side));
    m.resident = true;
    m.pending = true;
    return TI_OK;
}

ti_status ti_adapter_is_resident(ti_engine* e, int id, int* resident) {
    clear_error();
    if (ti_status st = adapter_check(e, id)) return st;
    TI_CHECK(resident, TI_ERR_INVALID, "null argument");
    auto& m = e->adapters[id];
    if (m.pending) {
        const cudaError_t q = cudaEventQuery(m.ready);
        if (q == cudaSuccess) m.pending = false;
        else if (q != cudaErrorNotReady) return fail(TI_ERR_CUDA, "adapter %d copy: %s", id, cudaGetErrorString(q));
        else cudaGetLastError();
    }
    *resident = (m.resident && !m.pending) ? 1 : 0;
    return TI_OK;
}

}  // extern "C"
