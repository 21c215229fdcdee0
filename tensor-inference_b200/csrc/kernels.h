// kernels.h — host-side launch interface of the sm_100a kernels (internal).
#pragma once
#include <cuda.h>
#include <cuda_runtime.h>
#include <stdint.h>

#include <string>

namespace ti {

// ----------------------------------------------------------------- launch helper
// Launch with the programmatic-stream-serialization attribute (PDL) so the
// kernel's weight prefetch overlaps the tail of the previous kernel.
cudaError_t launch_pdl(const void* func, dim3 grid, dim3 block, size_t smem, cudaStream_t s, void** args, bool pdl);

int num_sms(int device);

// ----------------------------------------------------------------- weight-streaming GEMV
enum GemvEpi : int {
    kEpiStore = 0,   // out = bf16(acc) [+ bias -> bf16]
    kEpiResid = 1,   // out = bf16(resid + bf16(acc))
    kEpiGlu = 2,     // units are (gate row n, up row n + N): out = bf16(bf16(act(bf16(g))) * bf16(u))
    kEpiLmHead = 3,  // logits = bf16(acc); greedy argmax over fp32 acc (lowest index on ties)
};

struct GemvLora {
    // per-token low-rank expansion added after the base projection (and bias):
    // out = bf16(out + bf16(bf16(sum_r B[n, r] * t[b, r]) * scale[adapter[b]]))
    const int32_t* adapter = nullptr;  // [nb] adapter id per token (device); < 0 = none; nullptr = LoRA off
    const uint16_t* B = nullptr;       // adapter 0's B rows for this layer: [rows, rank]
    size_t B_adapter_stride = 0;       // elements from one adapter's rows to the next's
    const float* t = nullptr;          // [nb, t_stride] bf16-exact fp32 values of x A^T
    int t_stride = 0;
    int rank = 0;                      // padded rank (padding rows of A / cols of B are zero)
    const float* scale = nullptr;      // [n_adapters] alpha / rank
    int n_adapters = 0;
    // fused q|k|v rows: rows [0,sec1) use t[0:rank), [sec1,sec2) t[rank:2rank), the rest t[2rank:3rank)
    int sec1 = 1 << 30, sec2 = 1 << 30;
    // when set: the expansion bf16(bf16(t.B^T) * scale) of every (token, row) was
    // computed ahead by lora_expand_launch ([nb, dval_stride] bf16, rows as the
    // GEMM's output rows); the epilogue only adds it
    const uint16_t* dval = nullptr;
    int dval_stride = 0;
};

// LoRA expansion ahead of a batched GEMM: dval[b, n] = bf16(bf16(sum_r B[ad_b][n, r] t[b, r']) * scale[ad_b])
// for rows [0, n_rows) (kEpiGlu: glu_n gate rows then glu_n up rows, t sections 0 / 1)
cudaError_t lora_expand_launch(const GemvLora& L, int nb, int n_rows, int glu_n, uint16_t* dval, int dval_stride,
                               cudaStream_t s, bool pdl);

// One-shot all-reduce over NVLink peer memory (tensor parallelism).  The
// producer (a row-parallel projection) stores its fp32 outputs straight into
// every rank's inbox slot for this sender; every CTA fences system-wide and the
// last one publishes the phase's sequence number to every rank's flag for this
// sender.  A receiver waits (bounded) for all flags, then sums the inboxes in
// rank order, so all ranks get bit-identical results.
constexpr int kMaxTp = 8;
struct PeerSend {
    float* inbox[kMaxTp] = {};        // rank r's inbox block for this sender ([nb, out_stride])
    unsigned int* flag[kMaxTp] = {};  // rank r's flag for this sender
    int tp = 0;                       // ranks; 0 = off
    int signal = 1;                   // 0: store only (an earlier launch of a chunked batch)
    const int* epoch = nullptr;       // device step counter (the step's first kernel increments it)
    int seq_mul = 1, seq_add = 0;     // sequence number = (*epoch - 1) * seq_mul + seq_add
    unsigned int* ticket = nullptr;   // local CTA completion counter (zero; the last CTA resets it)
};

// sequence number of a phase (wrap-safe comparisons with (int)(a - b) >= 0)
__host__ __device__ inline unsigned int peer_seq(int epoch, int mul, int add) {
    return (unsigned int)(epoch - 1) * (unsigned int)mul + (unsigned int)add;
}

// LoRA shrink: t[b, r] = bf16(x_b . A[adapter[b]][r]), optional RMSNorm of x first
struct LoraShrinkArgs {
    const uint16_t* x = nullptr;  // [nb, x_stride] bf16
    int x_stride = 0, K = 0, nb = 1;
    const uint16_t* norm_w = nullptr;
    float eps = 1e-5f;
    int norm_offset = 0;
    const uint16_t* A = nullptr;  // adapter 0's A rows for this layer: [T, K]
    size_t A_adapter_stride = 0;
    int T = 0;                    // rows: sections x padded rank
    const int32_t* adapter = nullptr;
    int n_adapters = 0;
    float* t = nullptr;           // [nb, t_stride]
    int t_stride = 0;
    // tensor parallelism, row-parallel projection: x and A hold this rank's input
    // columns; the unrounded fp32 partial sums go to every rank's inbox instead of t
    float* peer_t[kMaxTp] = {};
    int tp = 0;
    // split-K workspace: partial sums [kLoraMaxSplit][nb][t_stride] and per
    // (adapter, 32-row tile) arrival counters [n_adapters][ceil(T / 32)] (zero;
    // the last CTA of a tile resets its counter)
    float* ws = nullptr;
    unsigned int* ctr = nullptr;
};
constexpr int kLoraMaxSplit = 16;
cudaError_t lora_shrink_launch(const LoraShrinkArgs& a, cudaStream_t s, bool pdl);

// Weight row formats the GEMV streams (TI_WFMT_* values).  Quantised rows are
// [K codes][K/32 fp16 block scales]: Q4_0 codes are 4-bit, element c in byte
// c/2 (low nibble for even c), value d * (q - 8); Q8_0 codes are int8, value
// d * q (GGUF's block formats, rows repacked so a lane's 8 elements are one
// aligned word).
enum WeightFmt : int { kWBf16 = 0, kWQ4 = 1, kWQ8 = 2 };
__host__ __device__ inline size_t wrow_bytes(int K, int wf) {
    return wf == kWQ4 ? (size_t)K / 2 + (size_t)K / 16 : wf == kWQ8 ? (size_t)K + (size_t)K / 16 : (size_t)K * 2;
}

// Decode attention of one token run inside the o-projection GEMV, ahead of its
// prologue: the work of ops::rope x2, the K/V cache write, ops::slice x2 and
// ops::attention for one layer (llama_model.cpp:147-182).  The kernel's x is
// the attention output, written by the kernel itself.
struct GemvAttn {
    const uint16_t* qkv = nullptr;  // the token's q|k|v before RoPE, bf16 [(nq + 2 nkv) * hd]
    int nq = 0, nkv = 0, hd = 0;    // nq = 0: off
    const int32_t* pos = nullptr;   // [1] tokens already cached for the sequence (device)
    const int32_t* seq = nullptr;   // [1] the sequence's page-table row (device)
    const int32_t* page_table = nullptr;
    int pt_stride = 0;
    uint16_t* kc = nullptr;  // this layer's K pages [n_pages][nkv][16][hd] bf16
    uint16_t* vc = nullptr;  // V pages, same layout
    int n_pages = 0;
    const float* freqs = nullptr;  // [hd / 2] RoPE frequencies
    float scale = 0.f;             // 1 / sqrt(hd)
    const int* window = nullptr;   // device sliding window (Mistral), or window_const when null; <= 0 = none
    int window_const = -1;
    uint16_t* out = nullptr;  // attention output bf16 [nq * hd] (the GEMV's x)
    float* part = nullptr;    // [grid][nq / nkv][hd + 2] per-CTA partials
    unsigned int* ticket = nullptr;  // [nkv] arrivals per kv head (zero; the merging CTA resets)
    unsigned int* sync = nullptr;    // [2] heads merged, CTAs past the wait (zero; the last CTA resets)
    int warps = 0;                   // consumer warps that score pages (shared-memory merge slots)
};
// shared memory of the attention phase: rotated q [G][hd], the token's k and v
// [2][hd], merge slots [warps][G][hd + 2], one flag (16 bytes), the merging
// CTA's per-partial (max, sum) [nh][G][2] (fp32; nh = CTAs per kv head)
__host__ __device__ inline uint32_t gemv_attn_smem(int G, int hd, int warps, int nh) {
    return (uint32_t)(((size_t)G * hd + 2 * (size_t)hd + (size_t)warps * G * (hd + 2) + (size_t)nh * G * 2) * 4 + 16);
}

// The receive half of the tensor-parallel all-reduce, run in a GEMV's prologue
// instead of a kernel of its own: once every rank's flag for the phase has reached
// its sequence number (bounded wait), x[b, k] = bf16(resid[b, k] + bf16(sum over
// ranks r, in rank order, of inbox[r * src_stride + b * K + k])) — the arithmetic
// of k_tp_recv_resid — and CTA 0 also stores x to x_out for later kernels.
struct GemvRecv {
    const float* inbox = nullptr;         // this rank's inbox blocks, [tp][src_stride] fp32
    size_t src_stride = 0;
    const unsigned int* flags = nullptr;  // this rank's flags [tp]
    int tp = 0;                           // 0: off (x is read from GemvArgs::x)
    const int* epoch = nullptr;
    int seq_mul = 1, seq_add = 0;
    const uint16_t* resid = nullptr;  // [nb, K] bf16
    uint16_t* x_out = nullptr;        // [nb, K] bf16
};

struct GemvArgs {
    const void* W = nullptr;  // [rows, K] in format wfmt; kEpiGlu: gate rows [0,N) then up rows [N,2N)
    int wfmt = kWBf16;
    int N = 0;                    // output units
    int K = 0;
    int nb = 1;                   // tokens
    const uint16_t* x = nullptr;  // bf16 [nb, x_stride]
    int x_stride = 0;
    const uint16_t* norm_w = nullptr;  // RMSNorm prologue over x when set
    float eps = 1e-5f;
    int norm_offset = 0;
    uint16_t* out = nullptr;  // bf16 [nb, out_stride]
    int out_stride = 0;
    const uint16_t* bias = nullptr;   // [N]
    const uint16_t* resid = nullptr;  // [nb, resid_stride]
    int resid_stride = 0;
    int act = 0;  // kEpiGlu: 0 = SiLU, 1 = tanh-GELU
    // LM head
    unsigned long long* amax = nullptr;  // [nb] argmax keys (zero before the step)
    unsigned int* done = nullptr;        // CTA completion counter (zero before the step)
    int32_t* out_ids = nullptr;          // [nb] greedy ids
    int32_t* chain_tokens = nullptr;     // [nb] next-step input tokens (optional)
    int32_t* chain_pos = nullptr;        // [nb] positions incremented after the step (optional)
    float* logits_f32 = nullptr;         // [nb, out_stride] optional fp32 logits
    int key_offset = 0;                  // LM head: global index of row 0 (vocabulary-parallel shard)
    int publish = 1;                     // LM head: 0 = leave the keys in amax (reduced across ranks later)
    // kEpiStore: when set, the unrounded fp32 sums go here instead ([nb, out_stride]);
    // the row-parallel half of tensor parallelism all-reduces them
    float* partial = nullptr;
    PeerSend ps;  // kEpiStore: fp32 sums into the ranks' inboxes (tensor-parallel all-reduce)
    GemvLora lora;
    // L2 warm-up of the next GEMV of the step: once this CTA's producer has
    // issued its own copies it prefetches the first `next_bytes` of the rows the
    // next kernel's CTA with the same index will stream first
    const void* next_w = nullptr;
    int next_N = 0, next_K = 0, next_U = 1, next_bytes = 0, next_wfmt = kWBf16;
    // when set, what `next_bytes` leaves after the next GEMV's rows goes to the
    // first rows of the GEMV after it (the q+k+v GEMV's budget, beyond the small
    // o projection, warms gate|up while attention runs)
    const void* next2_w = nullptr;
    int next2_N = 0, next2_K = 0, next2_U = 1, next2_wfmt = kWBf16;
    GemvAttn att;  // one token: its decode attention runs first and produces x
    GemvRecv recv;  // tensor parallelism: x is the all-reduce's receive, computed here
    int* err = nullptr;
};

struct GemvPlan {
    int rows_per_stage = 1;
    int stages = 3;
    int att_warps = 0;  // fused attention: page-scoring warps (GemvAttn::warps)
    int prefetch = 0;  // L2 prefetch window, in stages beyond the smem ring
    int grid = 0;
    size_t smem = 0;
    const void* func = nullptr;
};

// Chooses stage geometry, grid and kernel instance; false if unsupported.
bool gemv_plan(const GemvArgs& a, int epi, int device, GemvPlan* plan, std::string* why);
cudaError_t gemv_launch(const GemvArgs& a, int epi, const GemvPlan& plan, cudaStream_t s, bool pdl);

// ----------------------------------------------------------------- GGUF Q4_0 / Q8_0 rows
// bf16 [nr, K] (row pitch src_ld) -> quantised engine rows (wrow_bytes(K, wf) apart)
cudaError_t quantize_rows_launch(const uint16_t* src, int nr, int K, size_t src_ld, uint8_t* dst, size_t dst_rb,
                                 int wf, cudaStream_t s);
// GGUF blocks [nr, K/32] (18 / 34 bytes each) -> engine rows
cudaError_t repack_gguf_launch(const uint8_t* blocks, int nr, int K, uint8_t* dst, size_t dst_rb, int wf,
                               cudaStream_t s);
// engine rows (host memory) -> GGUF blocks (host memory)
void gguf_from_rows(const uint8_t* rows, int nr, int K, size_t rb, int wf, uint8_t* blocks);

// ----------------------------------------------------------------- tensor-core GEMM (tcgen05)
// Same arguments and epilogues as the GEMV (no RMSNorm prologue, no LoRA: the
// caller normalises rows with rms_rows_launch first); batches of 1..256 tokens.
struct TcPlan {
    int np = 0;  // tokens padded to a multiple of 32 (MMA N)
    int tiles = 0, kbs = 1, kblocks = 0, kpc = 0, grid = 0, stages = 0;  // kpc: k-blocks per CTA (stream-K)
    int pf = 0;  // weight k-blocks prefetched HBM -> L2 ahead of the ring's loads
    uint32_t stage_bytes = 0, tmem_cols = 0;
    uint32_t w_off = 0, x_off = 0, s_off = 0;  // stage layout (weights / tokens / GGUF scales)
    int cb = 0, n_abuf = 0, threads = 0;       // GGUF: code bytes per atom row, dequantised buffers
    int a_tmem = 0;                            // GGUF: dequantised buffers in TMEM (else shared memory)
    uint32_t a_col = 0;                        // GGUF, a_tmem: TMEM column of dequantised buffer 0
    int n_iss = 1;                             // MMA-issuing warps (GGUF with TMEM operands: up to 3)
    int n_acc = 2;                             // accumulators per issuer (2: double-buffered across units)
    size_t smem = 0;
    size_t ws_floats = 0;  // partial-tile workspace this launch needs
    const void* func = nullptr;
};
bool tc_plan(const GemvArgs& a, int epi, int device, size_t ws_floats_cap, TcPlan* plan, std::string* why);
// ws: >= plan.ws_floats floats; tile_ctr: >= plan.tiles zeroed counters
cudaError_t tc_launch(const GemvArgs& a, int epi, const TcPlan& plan, float* ws, unsigned int* tile_ctr,
                      cudaStream_t s, bool pdl);
// 2-D TMA map of a bf16 row-major matrix: boxes of 64 columns x box_rows, 128-byte swizzle
bool make_tmap_bf16_sw128(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                          uint32_t box_rows);
// out[b, :K] = bf16 RMSNorm(x[b, :K]) * (w [+ 1])
cudaError_t rms_rows_launch(const uint16_t* x, int x_stride, const uint16_t* w, float eps, int offset, int K, int nb,
                            uint16_t* out, int out_stride, cudaStream_t s, bool pdl);

// ----------------------------------------------------------------- paged decode attention
struct AttnArgs {
    const uint16_t* qkv = nullptr;  // [nb, qkv_stride] (q heads, k heads, v heads), pre-RoPE
    int qkv_stride = 0;
    int nb = 1;
    int nq = 0, nkv = 0, hd = 0;    // local heads
    const int32_t* pos = nullptr;   // [nb] position of the new token (= tokens already cached)
    const int32_t* seq = nullptr;   // [nb] sequence slot -> page-table row
    const int32_t* page_table = nullptr;  // [max_seqs, pt_stride]
    int pt_stride = 0;
    uint16_t* kc = nullptr;  // this layer's K pages: [n_pages, nkv, 16, hd]
    uint16_t* vc = nullptr;
    const float* freqs = nullptr;  // [hd/2]
    float scale = 1.f;
    const int32_t* window = nullptr;  // device scalar: attend to j > pos - window when > 0
    int window_const = -1;            // used when `window` is null
    int n_pages = 0;                  // pool size, bounds-checks page ids
    int n_splits = 1;
    int max_chunk = 0;   // tokens per split the smem is sized for
    float* part_o = nullptr;   // [nb, nkv, n_splits, group, hd]
    float* part_ml = nullptr;  // [nb, nkv, n_splits, group, 2]
    unsigned int* counters = nullptr;  // [nb, nkv] (zero; reset by the last CTA)
    // set by attn_launch: the n_splits (<= 8) CTAs of a (token, kv head) run as one
    // thread-block cluster and merge through distributed shared memory (part_o,
    // part_ml and counters unused)
    int cluster = 0;
    uint16_t* out = nullptr;  // [nb, out_stride]
    int out_stride = 0;
    int* err = nullptr;
    // prefill: the step's entries may be one sequence at consecutive positions,
    // whose K/V rows kv_append_launch wrote first; every page is loaded after the
    // dependency wait
    int prefill = 0;
};
// K (after RoPE) and V rows of every entry of a step into its page (ahead of a
// prefill step's attention); uses qkv, pos, seq, page_table, kc, vc, freqs,
// n_pages, nq, nkv, hd, nb, err of `a`
cudaError_t kv_append_launch(const AttnArgs& a, cudaStream_t s, bool pdl);
int attn_splits(int nb, int nkv, int hd, int max_len, int sms, int* max_chunk);
// scratch floats / counters one launch needs: part_o + part_ml, and nb*nkv counters
size_t attn_scratch_floats(int nb, int nq, int nkv, int hd, int n_splits);
cudaError_t attn_launch(const AttnArgs& a, cudaStream_t s, bool pdl);

// ----------------------------------------------------------------- tensor-parallel glue
// out[b, n] = bf16(resid[b, n] + bf16(sum[b, n])) after the all-reduce of a row-parallel projection
cudaError_t tp_resid_launch(const float* sum, const uint16_t* resid, uint16_t* out, int nb, int H, cudaStream_t s,
                            bool pdl);
// receive side of the peer all-reduce: wait (bounded) until every sender's flag
// reaches this phase's sequence number, out = bf16(resid + bf16(sum of the inboxes in rank order))
// With `lora` set (lora->adapter != nullptr, row-parallel LoRA): t_inbox holds
// every rank's partial x.A^T ([tp][t_src_stride]); the rank-ordered sums rounded
// to bf16 feed the expansion bf16(bf16(t.B^T) * scale) added to the projection.
cudaError_t tp_recv_resid_launch(const float* inbox, size_t src_stride, const unsigned int* flags, int tp,
                                 const int* epoch, int seq_mul, int seq_add, const uint16_t* resid, uint16_t* out,
                                 int nb, int H, const GemvLora* lora, const float* t_inbox, size_t t_src_stride,
                                 int* err, cudaStream_t s, bool pdl);
// greedy ids over the ranks' vocabulary slices through peer memory: send this
// rank's keys to every rank, wait for all, take the max (one CTA)
cudaError_t tp_keys_launch(unsigned long long* amax, int nb, unsigned long long* const* peer_keys,
                           unsigned int* const* peer_flags, int tp, int rank, const unsigned long long* keys_inbox,
                           const unsigned int* flags, int max_nb, const int* epoch, int32_t* out_ids,
                           int32_t* chain_tokens, int32_t* chain_pos, int* err, cudaStream_t s, bool pdl);
// greedy ids from the all-reduced argmax keys; re-arms the keys (cf. the LM-head epilogue)
cudaError_t tp_ids_launch(unsigned long long* amax, int nb, int32_t* out_ids, int32_t* chain_tokens,
                          int32_t* chain_pos, cudaStream_t s, bool pdl);

// ----------------------------------------------------------------- small kernels
struct EmbedArgs {
    const uint16_t* table = nullptr;  // [vocab, hidden]
    int vocab = 0, hidden = 0, nb = 1;
    const int32_t* tokens = nullptr;  // [nb]
    uint16_t* out = nullptr;          // [nb, hidden]
    float scale = 0.f;                // Gemma: embeddings times sqrt(hidden) (0 = none)
    // page-table updates applied before the step: (seq, index, page) triples
    const int32_t* pt_updates = nullptr;  // device [3 * max]
    const int32_t* n_updates = nullptr;   // device scalar
    int32_t* page_table = nullptr;
    int pt_stride = 0;
    int* epoch = nullptr;  // step counter for tensor-parallel phase sequence numbers (incremented here)
    int* err = nullptr;
};
cudaError_t embed_launch(const EmbedArgs& a, cudaStream_t s, bool pdl);

// ----------------------------------------------------------------- sampling
// Top-p / top-k sampling of bf16 logits rows, one CTA per row (sample.cu has
// the exact definition); rows of kind kSampleGreedy keep out[b] unchanged.
enum : int32_t { kSampleGreedy = 0, kSampleTopP = 1, kSampleTopK = 2 };
struct SampleRow {  // per-row parameters in device memory, 32 bytes
    int32_t kind = kSampleGreedy;
    float temperature = 1.0f;
    float p = 1.0f;
    int32_t k = 1;
    float u = 0.0f;  // uniform draw in [0, 1)
    int32_t pad[3] = {};
};
struct SampleArgs {
    // token i of row b at logits[(i / seg) * seg_stride + b * row_stride + i % seg]:
    // seg = vocab for contiguous rows, the per-rank slice for gathered TP logits
    const uint16_t* logits = nullptr;
    int vocab = 0, seg = 0;
    size_t seg_stride = 0, row_stride = 0;
    const SampleRow* rows = nullptr;  // [nb]
    uint32_t* hist = nullptr;         // sample_scratch_bytes(nb)
    int32_t* out = nullptr;           // [nb] sampled ids
    int* err = nullptr;               // error bits
    // device-resident decode chains: row b's draw is draws[b * draw_cap + draw_ctr[b]]
    // (then draw_ctr[b] advances) instead of rows[b].u, and the id also goes to chain_tokens[b]
    const float* draws = nullptr;
    int draw_cap = 0;
    int32_t* draw_ctr = nullptr;
    int32_t* chain_tokens = nullptr;
};
// bounded-wait self-test (small.cu): a flag and an mbarrier that nothing completes
cudaError_t wait_selftest_launch(const unsigned int* flag, uint64_t limit_ns, int* err, unsigned long long* elapsed,
                                 cudaStream_t s);

size_t sample_scratch_bytes(int nb);
cudaError_t sample_launch(const SampleArgs& a, int nb, cudaStream_t s);

// synthetic K/V rows for positions [0, n_tok) of one sequence (its pages[]), all layers
cudaError_t fill_kv_launch(uint16_t* kpool, uint16_t* vpool, size_t layer_elems, int n_layers, const int32_t* pages,
                           int n_tok, int nkv, int kv0, int nkv_g, int hd, uint64_t key_k, uint64_t key_v, float c,
                           cudaStream_t s);
// synthetic init of a [rows, cols] window (row stride dst_ld) of a full tensor
// with row length full_ld: dst[r][c] = gen(index (r0 + r) * full_ld + c0 + c)
cudaError_t synth_bf16_launch(uint16_t* dst, size_t rows, size_t cols, size_t dst_ld, size_t r0, size_t c0,
                              size_t full_ld, uint64_t seed, uint64_t name_hash, float scale_c, cudaStream_t s);
cudaError_t synth_f32_launch(float* dst, size_t n, uint64_t seed, uint64_t name_hash, float scale_c,
                             cudaStream_t s);

// rope frequency table on the device, cached per (device, head_dim, theta, scaling)
const float* rope_table(int dev, int hd, float theta, const void* scaling /* const ti_rope_scaling* */);

}  // namespace ti
