// tc_gemm.cu — tensor-core (tcgen05) skinny GEMM for batched decode and prefill.
//
// Y[t, n] = sum_k X[t, k] * W[n, k] for up to 256 tokens t: the reference's
// ops::matmul_t (ops.cu:94-148, cuBLAS GemmEx, fp32 accumulate, bf16 output)
// for a batch of tokens, with the same fused epilogues as the weight-streaming
// GEMV (bias, residual add, SwiGLU/GeGLU, LM-head argmax).  Once a decode batch
// has 16+ tokens the FMA work of a SIMT GEMV outgrows the weight stream; here the
// 5th-generation tensor cores do it and the kernel stays HBM-bound.
//
// Orientation: the weights are the MMA's M side (128 rows per tile, so a tile
// is a dense 16 KB block per 64-element K step) and the tokens its N side
// (padded to a multiple of 32; rows past the batch are zero-filled by TMA).
// D = W_tile (128 x K) * X^T (K x np) accumulates in TMEM, fp32.
//
// Structure (one persistent CTA per SM; bf16 weights 224 threads, GGUF 512):
//   warp 0      TMA producer: 2-D tiled bulk-tensor loads (128-byte swizzle) of
//               the weight tile (L2 evict-first) and the token tile into a
//               ring of shared-memory stages.  Weight loads of the first ring
//               are issued before griddepcontrol.wait, overlapping the previous
//               kernel's tail (weights do not depend on it).
//   warp 1      allocates TMEM and, with the other issuer warps below, one lane
//               issues tcgen05.mma (kind::f16, bf16 x bf16 -> fp32, M=128,
//               N=np, K=16 per instruction, 16 per stage split over the issuers,
//               each into its own two accumulators of np columns); tcgen05.commit
//               frees each stage and signals a finished accumulator.
//   warps 2-5   epilogue: tcgen05.ld of the accumulator (warp w owns TMEM
//               lanes 32*(w%4)..+31 = 32 weight rows), fused epilogue, stores.
//               Double-buffered TMEM lets the epilogue of one tile overlap the
//               main loop of the next.
//   warps 6-13  GGUF Q4_0 / Q8_0 weights only (512 threads): the ring holds the
//               raw codes (128-byte swizzled boxes) and fp16 scales; each thread
//               dequantises one weight row's half stage to bf16 pairs.  Up to 128
//               tokens the pairs go to TMEM (tcgen05.st into 2-3 operand buffers
//               above the accumulators) and the MMA reads A from TMEM, so shared
//               memory carries only the 0.56 (Q4_0) or 1.06 (Q8_0) bytes per
//               weight that HBM delivers; past 128 tokens they go to swizzled
//               shared-memory atoms (the engine launches GGUF batches in 128-token
//               pieces, so that form serves direct callers only).
//   warps 14-15 GGUF with TMEM operands: two more MMA issuers (a small tcgen05.mma
//               blocks its issuing thread ~100 cycles, so issuers in separate
//               warps add up); bf16: warp 6 is the second issuer (224 threads).
// Work split (stream-K): the row tiles x k-blocks of the GEMM, tile-major, are
// cut into equal contiguous ranges, one per CTA, so every SM streams the same
// number of weight bytes whatever the tile count.  A tile inside one range is
// finished by its CTA; a tile cut between CTAs has each part's fp32 partial
// stored, and the last part to finish (atomic ticket) sums them in CTA order
// (deterministic) and runs the epilogue.
//
// Every mbarrier wait is bounded (2 s): a timeout sets an error bit, the roles
// stop, the producer waits (bounded) for its copies in flight and TMEM is freed.
#include <cuda.h>

#include <algorithm>
#include <cstdlib>
#include <mutex>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"

namespace ti {

namespace {

constexpr int kTcThreads = 224;    // bf16 weights: TMA, MMA, 4 epilogue warps, a second MMA issuer
// GGUF: dequantising warps (warps 6..13).  16 (one atom per thread per stage) measured
// slower: 24 warps leave 80 registers a thread and the epilogue spills.
constexpr int kTcDeqWarps = 8;
constexpr int kTcThreadsQ = 32 * (6 + kTcDeqWarps + 2);  // GGUF weights: + dequantising warps + 2 more MMA issuers
constexpr int kTcMaxIss = 3;       // MMA-issuing warps at most (warp 1, then warps 14, 15)
constexpr int kTcBM = 128;        // weight rows per tile (MMA M)
constexpr int kTcBK = 64;         // K elements per swizzle atom: one 128-byte row
constexpr uint32_t kTcABytes = kTcBM * kTcBK * 2;  // 16 KB weight atom (128 rows x 64 K)
constexpr int kTcMaxTokens = 256;  // MMA N limit
constexpr size_t kTcSmemBudget = 220 * 1024;
constexpr int kTcMaxAbuf = 4;      // GGUF: dequantised operand buffers at most
constexpr int kTcQbs = 4;          // GGUF: atoms per stage (a 16-byte scales box)
constexpr int kTcAtPerThr = kTcQbs * 4 / kTcDeqWarps;  // GGUF: atoms one dequantising thread takes per stage

// ------------------------------------------------------------------ tcgen05 / TMA wrappers
TI_DEVICE_INLINE void tma_load_2d_hint(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar,
                                       uint64_t pol) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1, "
        "{%2, %3}], [%4], %5;" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
// L2 prefetch of one tiled box (no shared-memory destination, no multicast)
TI_DEVICE_INLINE void tma_prefetch_2d(const CUtensorMap* map, int x, int y) {
    asm volatile("cp.async.bulk.prefetch.tensor.2d.L2.global.tile [%0, {%1, %2}];" ::"l"(map), "r"(x), "r"(y)
                 : "memory");
}
TI_DEVICE_INLINE void tmap_prefetch(const CUtensorMap* map) {
    asm volatile("prefetch.tensormap [%0];" ::"l"(map) : "memory");
}
TI_DEVICE_INLINE void tc_fence_before() { asm volatile("tcgen05.fence::before_thread_sync;" ::: "memory"); }
TI_DEVICE_INLINE void tc_fence_after() { asm volatile("tcgen05.fence::after_thread_sync;" ::: "memory"); }

// shared-memory matrix descriptor: K-major operand, 128-byte swizzle, rows of
// 128 bytes, 8-row groups 1024 bytes apart (SBO), sm_100 descriptor version 1
TI_DEVICE_INLINE uint64_t smem_desc_sw128(uint32_t addr) {
    return (uint64_t)((addr & 0x3FFFFu) >> 4) | (1ull << 16) | ((uint64_t)(1024 >> 4) << 32) | (1ull << 46) |
           (2ull << 61);
}
// instruction descriptor, kind::f16: D fp32, A and B bf16, both K-major, M=128, N=n
__host__ __device__ constexpr uint32_t idesc_bf16(int n) {
    return (1u << 4) | (1u << 7) | (1u << 10) | ((uint32_t)(n >> 3) << 17) | ((uint32_t)(kTcBM >> 4) << 24);
}
TI_DEVICE_INLINE void tc_mma(uint32_t d_tmem, uint64_t adesc, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], %1, %2, %3, p;\n"
        "}\n" ::"r"(d_tmem),
        "l"(adesc), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
// 32 lanes x 16 consecutive fp32 columns (thread i <- lane base+i)
TI_DEVICE_INLINE void tmem_ld16(uint32_t taddr, float* v) {
    uint32_t r[16];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x16.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15}, [%16];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 16; ++i) v[i] = __uint_as_float(r[i]);
}
// bf16x2 arithmetic, each lane rounded once to nearest even
TI_DEVICE_INLINE uint32_t bsub2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("sub.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
TI_DEVICE_INLINE uint32_t bmul2(uint32_t a, uint32_t b) {
    uint32_t d;
    asm("mul.rn.bf16x2 %0, %1, %2;" : "=r"(d) : "r"(a), "r"(b));
    return d;
}
TI_DEVICE_INLINE uint32_t bfma2(uint32_t a, uint32_t b, uint32_t c) {
    uint32_t d;
    asm("fma.rn.bf16x2 %0, %1, %2, %3;" : "=r"(d) : "r"(a), "r"(b), "r"(c));
    return d;
}
// (lo, hi) fp32 -> bf16x2, round to nearest even
TI_DEVICE_INLINE uint32_t cvt_bf2(float lo, float hi) {
    uint32_t d;
    asm("cvt.rn.bf16x2.f32 %0, %1, %2;" : "=r"(d) : "f"(hi), "f"(lo));
    return d;
}
// the same with A (M=128 rows x K=16, bf16 pairs along 8 columns) read from TMEM
TI_DEVICE_INLINE void tc_mma_ts(uint32_t d_tmem, uint32_t a_tmem, uint64_t bdesc, uint32_t idesc, uint32_t acc) {
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "setp.ne.b32 p, %4, 0;\n"
        "tcgen05.mma.cta_group::1.kind::f16 [%0], [%1], %2, %3, p;\n"
        "}\n" ::"r"(d_tmem),
        "r"(a_tmem), "l"(bdesc), "r"(idesc), "r"(acc)
        : "memory");
}
// 32 lanes x 32 consecutive 32-bit columns (thread i -> lane base+i).  No memory clobber:
// it writes TMEM only, and tcgen05.wait::st (volatile, after it) orders it for the MMA
TI_DEVICE_INLINE void tmem_st32(uint32_t taddr, const uint32_t* r) {
    asm volatile(
        "tcgen05.st.sync.aligned.32x32b.x32.b32 [%0], {%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,"
        "%18,%19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31,%32};" ::"r"(taddr),
        "r"(r[0]), "r"(r[1]), "r"(r[2]), "r"(r[3]), "r"(r[4]), "r"(r[5]), "r"(r[6]), "r"(r[7]), "r"(r[8]),
        "r"(r[9]), "r"(r[10]), "r"(r[11]), "r"(r[12]), "r"(r[13]), "r"(r[14]), "r"(r[15]), "r"(r[16]), "r"(r[17]),
        "r"(r[18]), "r"(r[19]), "r"(r[20]), "r"(r[21]), "r"(r[22]), "r"(r[23]), "r"(r[24]), "r"(r[25]), "r"(r[26]),
        "r"(r[27]), "r"(r[28]), "r"(r[29]), "r"(r[30]), "r"(r[31]));
}
TI_DEVICE_INLINE void tc_commit(uint64_t* bar) {
    asm volatile("tcgen05.commit.cta_group::1.mbarrier::arrive::one.shared::cluster.b64 [%0];" ::"r"(smem_u32(bar))
                 : "memory");
}
// 32 lanes x 32 consecutive fp32 columns (thread i <- lane base+i)
TI_DEVICE_INLINE void tmem_ld32(uint32_t taddr, float* v) {
    uint32_t r[32];
    asm volatile(
        "tcgen05.ld.sync.aligned.32x32b.x32.b32 {%0,%1,%2,%3,%4,%5,%6,%7,%8,%9,%10,%11,%12,%13,%14,%15,%16,%17,%18,%"
        "19,%20,%21,%22,%23,%24,%25,%26,%27,%28,%29,%30,%31}, [%32];"
        : "=r"(r[0]), "=r"(r[1]), "=r"(r[2]), "=r"(r[3]), "=r"(r[4]), "=r"(r[5]), "=r"(r[6]), "=r"(r[7]),
          "=r"(r[8]), "=r"(r[9]), "=r"(r[10]), "=r"(r[11]), "=r"(r[12]), "=r"(r[13]), "=r"(r[14]), "=r"(r[15]),
          "=r"(r[16]), "=r"(r[17]), "=r"(r[18]), "=r"(r[19]), "=r"(r[20]), "=r"(r[21]), "=r"(r[22]), "=r"(r[23]),
          "=r"(r[24]), "=r"(r[25]), "=r"(r[26]), "=r"(r[27]), "=r"(r[28]), "=r"(r[29]), "=r"(r[30]), "=r"(r[31])
        : "r"(taddr));
    asm volatile("tcgen05.wait::ld.sync.aligned;" ::: "memory");
#pragma unroll
    for (int i = 0; i < 32; ++i) v[i] = __uint_as_float(r[i]);
}

TI_DEVICE_INLINE float tc_act(float g, int act) {
    if (act == 0) return round_bf(g / (1.0f + expf(-g)));  // ops.cu:326
    const float c1 = 0.7978845608f, c2 = 0.044715f;        // ops.cu:712-714
    return round_bf(0.5f * g * (1.0f + tanhf(c1 * (g + c2 * g * g * g))));
}

}  // namespace

struct TcKernelArgs {
    int N, K, nb, np;
    int tiles, kblocks;  // row tiles; k-blocks per tile (a k-block = kbs atoms = kbs * 64 K elements)
    int kbs;
    int kpc;             // k-blocks per CTA: CTA c owns global k-blocks [c * kpc, (c + 1) * kpc)
    int stages;
    int pf;              // the producer prefetches weight k-block it + pf into L2 as it loads k-block it
    // stage layout: bf16: [kbs weight atoms][kbs token atoms]; GGUF: [kbs token atoms]
    // [codes: kbs*cb/128 column blocks of 128 rows x 128 bytes, 128-byte swizzle]
    // [scales: 128 rows x kbs*4 bytes], dequantised into n_abuf bf16 operand
    // buffers of kbs atoms (TMEM, or shared memory after the ring)
    uint32_t w_off, x_off, s_off;
    int cb, n_abuf;
    int a_tmem;      // dequantised operand buffers in TMEM columns [a_col + b * kbs * 32, ...) (else shared memory)
    uint32_t a_col;
    int n_acc;       // accumulators per issuer: 2 (the epilogue of one unit overlaps the next) or 1
    int n_iss;       // MMA-issuing warps: issuer i takes K steps i, i + n_iss, ... of each stage into its
                     // own accumulators, TMEM columns [(i * n_acc + buf) * np, +np); the epilogue sums them in order
    uint32_t stage_bytes, tmem_cols;
    uint16_t* out;
    int out_stride;
    const uint16_t* bias;
    const uint16_t* resid;
    int resid_stride;
    int act;
    unsigned long long* amax;
    unsigned int* done;
    int32_t* out_ids;
    int32_t* chain_tokens;
    int32_t* chain_pos;
    float* logits_f32;
    int key_offset, publish;
    float* partial;
    PeerSend ps;
    float* ws;               // [grid][2][np][128] fp32 partials of tiles shared between CTAs
    unsigned int* tile_ctr;  // [tiles], zero; reset by each shared tile's last unit
    GemvLora lora;           // per-token LoRA expansion (adapter == nullptr: off)
    int* err;
};

// Shared memory after the stage ring (offsets from the 1024-aligned base).
struct TcSmem {
    uint32_t abuf, full, empty, xfull, afull, aempty, tfull, tempty, drain, misc, xch, best, total;
};
__host__ __device__ inline TcSmem tc_smem_layout(int stages, uint32_t stage_bytes, int np, int n_abuf, int kbs) {
    TcSmem L;
    uint32_t o = (uint32_t)stages * stage_bytes;
    L.abuf = o;  // dequantised bf16 weight atoms (GGUF weights)
    o += (uint32_t)n_abuf * kbs * kTcABytes;
    L.full = o;
    o += 8u * stages;
    L.empty = o;
    o += 8u * stages;
    L.xfull = o;  // GGUF: the stage's token tile (full[] then covers its codes and scales only)
    o += 8u * stages;
    L.afull = o;
    o += 8 * kTcMaxAbuf;
    L.aempty = o;
    o += 8 * kTcMaxAbuf;
    L.tfull = o;
    o += 16;
    L.tempty = o;
    o += 16;
    L.drain = o;
    o += 8;
    L.misc = o;  // [0] tmem base, [1] abort flag, [2] split ticket, [3] epilogue stop
    o += 16;
    o = (o + 15u) & ~15u;
    L.xch = o;  // GLU exchange: [2 row groups][32 tokens][32 rows] fp32
    o += 2 * 32 * 32 * 4;
    L.best = o;  // LM head: per-token argmax keys of this CTA
    o += 8u * (uint32_t)np;
    L.total = o + 1024;  // + alignment slack of the dynamic smem base
    return L;
}

// WF: weight format (bf16 rows through 128-byte-swizzled TMA atoms, or GGUF rows:
// codes and scales through plain TMA boxes, dequantised to bf16 atoms in shared memory)
template <int EPI, int WF>
__global__ void __launch_bounds__(WF == kWBf16 ? kTcThreads : kTcThreadsQ, 1)
    k_tc_gemm(const __grid_constant__ CUtensorMap tmw, const __grid_constant__ CUtensorMap tmx,
              const __grid_constant__ CUtensorMap tms, const TcKernelArgs a) {
    extern __shared__ uint8_t smem_raw[];
    uint8_t* smem = reinterpret_cast<uint8_t*>((reinterpret_cast<uintptr_t>(smem_raw) + 1023) & ~uintptr_t(1023));
    const TcSmem L = tc_smem_layout(a.stages, a.stage_bytes, a.np, a.a_tmem ? 0 : a.n_abuf, a.kbs);
    uint64_t* afull = reinterpret_cast<uint64_t*>(smem + L.afull);
    uint64_t* aempty = reinterpret_cast<uint64_t*>(smem + L.aempty);
    constexpr bool kQ = WF != kWBf16;
    uint64_t* full = reinterpret_cast<uint64_t*>(smem + L.full);
    uint64_t* empty = reinterpret_cast<uint64_t*>(smem + L.empty);
    uint64_t* xfull = reinterpret_cast<uint64_t*>(smem + L.xfull);
    uint64_t* tfull = reinterpret_cast<uint64_t*>(smem + L.tfull);
    uint64_t* tempty = reinterpret_cast<uint64_t*>(smem + L.tempty);
    uint64_t* drain = reinterpret_cast<uint64_t*>(smem + L.drain);
    volatile uint32_t* misc = reinterpret_cast<volatile uint32_t*>(smem + L.misc);
    float* xch = reinterpret_cast<float*>(smem + L.xch);
    unsigned long long* best = reinterpret_cast<unsigned long long*>(smem + L.best);

    const int warp = threadIdx.x >> 5, lane = threadIdx.x & 31;
    const int S = a.stages;
    const int np = a.np;
    constexpr bool kGlu = EPI == kEpiGlu;

    if (threadIdx.x == 0) {
        pdl_trigger();
        for (int s = 0; s < S; ++s) {
            mbar_init(&full[s], 1);
            mbar_init(&xfull[s], 1);
            mbar_init(&empty[s], a.n_iss);  // one tcgen05.commit per issuer
        }
        for (int j = 0; j < 2; ++j) {
            mbar_init(&tfull[j], a.n_iss);
            mbar_init(&tempty[j], 4);
        }
        for (int j = 0; j < kTcMaxAbuf; ++j) {
            mbar_init(&afull[j], kTcDeqWarps);  // the dequantising warps
            mbar_init(&aempty[j], a.n_iss);  // tcgen05.commit
        }
        mbar_init(drain, a.n_iss);
        misc[1] = 0;
        fence_barrier_init();
    }
    if (EPI == kEpiLmHead)
        for (int i = threadIdx.x; i < np; i += blockDim.x) best[i] = 0ull;
    if (warp == 1) {
        asm volatile("tcgen05.alloc.cta_group::1.sync.aligned.shared::cta.b32 [%0], %1;" ::"r"(
                         smem_u32((const void*)&misc[0])),
                     "r"(a.tmem_cols)
                     : "memory");
        asm volatile("tcgen05.relinquish_alloc_permit.cta_group::1.sync.aligned;" ::: "memory");
    }
    tc_fence_before();
    __syncthreads();
    tc_fence_after();
    const uint32_t tmem = misc[0];

    // Stream-K: the tiles x kblocks k-blocks, tile-major, are cut into equal
    // contiguous ranges, one per CTA.  A unit is the part of one tile inside the
    // range: whole tiles are finished by their CTA, a tile cut between CTAs is
    // summed by the last of them to finish (ticket), in CTA order.
    const long total = (long)a.tiles * a.kblocks;
    const long g_begin = (long)blockIdx.x * a.kpc, g_end = min(total, g_begin + a.kpc);
    // f(tile, k0, k1, first_unit) for each unit of this CTA; false stops
    auto units = [&](auto&& f) {
        bool first = true;
        for (long g = g_begin; g < g_end;) {
            const int tile = (int)(g / a.kblocks), k0 = (int)(g % a.kblocks);
            const int k1 = (int)min((long)a.kblocks, k0 + (g_end - g));
            if (!f(tile, k0, k1, first)) return;
            first = false;
            g += k1 - k0;
        }
    };
    // (tile, k-block) iterations of this CTA in issue order; f returns false to stop
    auto walk = [&](auto&& f) -> int {
        int it = 0;
        bool go = true;
        units([&](int tile, int k0, int k1, bool) {
            for (int kb = k0; kb < k1; ++kb, ++it)
                if (!f(tile, kb, it)) {
                    go = false;
                    return false;
                }
            return true;
        });
        (void)go;
        return it;
    };

    if (warp == 0) {
        // ------------------------------------------------------------ TMA producer
        if (lane == 0) {
            tmap_prefetch(&tmw);
            tmap_prefetch(&tmx);
            if (kQ) tmap_prefetch(&tms);
            const uint64_t pol = l2_policy_evict_first();
            const int kbs = a.kbs;
            const uint32_t xatom = (uint32_t)np * kTcBK * 2;
            // GGUF: full[] counts the codes and scales and xfull[] the token tile, so the
            // dequantising warps can start on the first ring pass while the previous
            // kernel (which produces the tokens) is still finishing
            const uint32_t tx = kQ ? (uint32_t)kTcBM * kbs * (a.cb + 4) : (uint32_t)kbs * (kTcABytes + xatom);
            const uint32_t tx_x = (uint32_t)kbs * xatom;
            auto load_w = [&](int tile, int kb, int s) {
                uint8_t* st = smem + (size_t)s * a.stage_bytes;
                if constexpr (kQ) {
                    // the codes (128-byte column blocks) and fp16 scales of kbs*64 columns
                    // of 128 rows (two halves of 64 rows for GLU)
                    const int xc = kb * kbs * a.cb, xs = kb * kbs * 4;
                    for (int h = 0; h < kbs * a.cb / 128; ++h) {
                        uint8_t* cbk = st + a.w_off + (size_t)h * kTcBM * 128;
                        if (kGlu) {
                            tma_load_2d_hint(cbk, &tmw, xc + h * 128, tile * 64, &full[s], pol);
                            tma_load_2d_hint(cbk + 64 * 128, &tmw, xc + h * 128, a.N + tile * 64, &full[s], pol);
                        } else {
                            tma_load_2d_hint(cbk, &tmw, xc + h * 128, tile * kTcBM, &full[s], pol);
                        }
                    }
                    if (kGlu) {
                        const uint32_t half_s = 64u * kbs * 4;
                        tma_load_2d_hint(st + a.s_off, &tms, xs, tile * 64, &full[s], pol);
                        tma_load_2d_hint(st + a.s_off + half_s, &tms, xs, a.N + tile * 64, &full[s], pol);
                    } else {
                        tma_load_2d_hint(st + a.s_off, &tms, xs, tile * kTcBM, &full[s], pol);
                    }
                } else {
                    // kbs adjacent 64-column atoms of each weight row back to back, so
                    // DRAM sees kbs * 128 contiguous bytes per row
                    for (int j = 0; j < kbs; ++j) {
                        const int x = (kb * kbs + j) * kTcBK;
                        uint8_t* at = st + (size_t)j * kTcABytes;
                        if (kGlu) {
                            tma_load_2d_hint(at, &tmw, x, tile * 64, &full[s], pol);
                            tma_load_2d_hint(at + kTcABytes / 2, &tmw, x, a.N + tile * 64, &full[s], pol);
                        } else {
                            tma_load_2d_hint(at, &tmw, x, tile * kTcBM, &full[s], pol);
                        }
                    }
                }
            };
            // the same boxes as load_w, HBM -> L2 only: keeps pf more k-blocks of
            // weights in flight than the shared-memory ring holds
            auto prefetch_w = [&](int it) {
                const long g = g_begin + it;
                if (a.pf <= 0 || g >= g_end) return;
                const int tile = (int)(g / a.kblocks), kb = (int)(g % a.kblocks);
                if constexpr (kQ) {
                    const int xc = kb * kbs * a.cb, xs = kb * kbs * 4;
                    for (int h = 0; h < kbs * a.cb / 128; ++h) {
                        if (kGlu) {
                            tma_prefetch_2d(&tmw, xc + h * 128, tile * 64);
                            tma_prefetch_2d(&tmw, xc + h * 128, a.N + tile * 64);
                        } else {
                            tma_prefetch_2d(&tmw, xc + h * 128, tile * kTcBM);
                        }
                    }
                    if (kGlu) {
                        tma_prefetch_2d(&tms, xs, tile * 64);
                        tma_prefetch_2d(&tms, xs, a.N + tile * 64);
                    } else {
                        tma_prefetch_2d(&tms, xs, tile * kTcBM);
                    }
                } else {
                    for (int j = 0; j < kbs; ++j) {
                        const int x = (kb * kbs + j) * kTcBK;
                        if (kGlu) {
                            tma_prefetch_2d(&tmw, x, tile * 64);
                            tma_prefetch_2d(&tmw, x, a.N + tile * 64);
                        } else {
                            tma_prefetch_2d(&tmw, x, tile * kTcBM);
                        }
                    }
                }
            };
            auto load_x = [&](int kb, int s) {
                uint8_t* xt = smem + (size_t)s * a.stage_bytes + a.x_off;
                for (int j = 0; j < kbs; ++j)
                    tma_load_2d(xt + (size_t)j * xatom, &tmx, (kb * kbs + j) * kTcBK, 0, kQ ? &xfull[s] : &full[s]);
            };
            // 1. weights of the first pass of the ring: they do not depend on the
            //    previous kernel, so they stream while it finishes
            const int first = walk([&](int tile, int kb, int it) {
                if (it >= S) return false;
                mbar_arrive_expect_tx(&full[it], tx);
                load_w(tile, kb, it);
                return true;
            });
            for (int it = first; it < first + a.pf; ++it) prefetch_w(it);
            // 2. the token tiles of those stages, once the previous kernel is done
            pdl_wait();
            walk([&](int, int kb, int it) {
                if (it >= first) return false;
                if (kQ) mbar_arrive_expect_tx(&xfull[it], tx_x);
                load_x(kb, it);
                return true;
            });
            // 3. steady state
            int issued = first;
            walk([&](int tile, int kb, int it) {
                if (it < first) return true;
                const int s = it % S;
                if (misc[1] || !mbar_wait(&empty[s], ((it / S) & 1) ^ 1, a.err, kErrTimeoutEmpty)) {
                    misc[1] = 1;
                    return false;
                }
                mbar_arrive_expect_tx(&full[s], tx);
                if (kQ) mbar_arrive_expect_tx(&xfull[s], tx_x);
                load_w(tile, kb, s);
                load_x(kb, s);
                prefetch_w(it + a.pf);
                issued = it + 1;
                return true;
            });
            // copies still in flight land before the CTA exits
            for (int j = max(0, issued - S); j < issued; ++j) {
                if (!mbar_wait(&full[j % S], (j / S) & 1, a.err, kErrTimeoutFull)) break;
                if (kQ && !mbar_wait(&xfull[j % S], (j / S) & 1, a.err, kErrTimeoutFull)) break;
            }
        }
    } else if (warp == 1 || (kQ && warp >= 6 + kTcDeqWarps) || (!kQ && warp == 6)) {
        // ------------------------------------------------------------ MMA issuers
        // A small tcgen05.mma blocks its issuing thread for about a hundred cycles
        // whatever N is, so one thread issuing M=128, N=32, K=16 steps reaches about
        // a third of the rate dequantised GGUF weights arrive at; issuers in separate
        // warps, each into its own accumulators, add up (A from TMEM; from shared memory
        // two issuers still double the rate).  Issuers: warp 1, then the two after the
        // dequantising warps (GGUF) or warp 6 (bf16).
        const int iss = warp == 1 ? 0 : kQ ? warp - (5 + kTcDeqWarps) : 1;
        if (lane == 0 && iss < a.n_iss) {
            const uint32_t idesc = idesc_bf16(np);
            int it = 0, j = 0;
            bool issued = false;
            units([&](int, int kb0, int kb1, bool) {
                const int buf = j % a.n_acc;
                if (misc[1] || !mbar_wait(&tempty[buf], ((j / a.n_acc) & 1) ^ 1, a.err, kErrTimeoutEmpty)) {
                    misc[1] = 1;
                    return false;
                }
                tc_fence_after();
                const uint32_t d = tmem + (uint32_t)((iss * a.n_acc + buf) * np);
                for (int kb = kb0; kb < kb1; ++kb, ++it) {
                    const int s = it % S;
                    if (misc[1] || !mbar_wait(&full[s], (it / S) & 1, a.err, kErrTimeoutFull) ||
                        (kQ && !mbar_wait(&xfull[s], (it / S) & 1, a.err, kErrTimeoutFull))) {
                        misc[1] = 1;
                        return false;
                    }
                    const int ab = kQ ? it % a.n_abuf : 0;
                    if (kQ && (misc[1] || !mbar_wait(&afull[ab], (it / a.n_abuf) & 1, a.err, kErrTimeoutFull))) {
                        misc[1] = 1;
                        return false;
                    }
                    tc_fence_after();
                    const uint32_t st_addr = smem_u32(smem + (size_t)s * a.stage_bytes);
                    const uint32_t b_addr = st_addr + a.x_off;
                    if (kQ && a.a_tmem) {
                        // weights from TMEM: atom jj in 32 columns of bf16 pairs, 8 per K=16 step
                        // K step m = 4 * atom + k of the stage (16 columns of bf16 pairs = 8 TMEM columns)
                        const uint32_t a_t = tmem + a.a_col + (uint32_t)(ab * a.kbs * 32);
                        const uint64_t b_d = smem_desc_sw128(b_addr);
                        for (int m = iss; m < a.kbs * (kTcBK / 16); m += a.n_iss) {
                            const int jj = m >> 2, k = m & 3;
                            tc_mma_ts(d, a_t + (uint32_t)(m * 8),
                                      b_d + (uint64_t)((jj * (uint32_t)np * kTcBK * 2 + k * 32) >> 4), idesc,
                                      (kb > kb0 || m > iss) ? 1u : 0u);
                        }
                    } else {
                        const uint32_t a_addr =
                            kQ ? smem_u32(smem + L.abuf + (size_t)ab * a.kbs * kTcABytes) : st_addr + a.w_off;
                        if (a.n_iss == 1) {
                            for (int jj = 0; jj < a.kbs; ++jj)
#pragma unroll
                                for (int k = 0; k < kTcBK / 16; ++k)
                                    tc_mma(d, smem_desc_sw128(a_addr + jj * kTcABytes + k * 32),
                                           smem_desc_sw128(b_addr + jj * (uint32_t)np * kTcBK * 2 + k * 32), idesc,
                                           (kb > kb0 || jj > 0 || k > 0) ? 1u : 0u);
                        } else {
                            // K step m = 4 * atom + k; issuer iss takes m = iss, iss + n_iss, ...
                            const uint64_t a_d = smem_desc_sw128(a_addr), b_d = smem_desc_sw128(b_addr);
                            for (int m = iss; m < a.kbs * (kTcBK / 16); m += a.n_iss) {
                                const int jj = m >> 2, k = m & 3;
                                tc_mma(d, a_d + (uint64_t)((jj * kTcABytes + k * 32) >> 4),
                                       b_d + (uint64_t)((jj * (uint32_t)np * kTcBK * 2 + k * 32) >> 4), idesc,
                                       (kb > kb0 || m > iss) ? 1u : 0u);
                            }
                        }
                    }
                    tc_commit(&empty[s]);
                    if (kQ) tc_commit(&aempty[ab]);
                    issued = true;
                }
                tc_commit(&tfull[buf]);
                ++j;
                return true;
            });
            // all MMAs retired before TMEM is released (every issuer has MMAs when any has)
            if (issued) {
                tc_commit(drain);
                mbar_wait(drain, 0, a.err, kErrTimeoutFull);
            }
        }
    } else if (kQ && warp >= 6 && warp < 6 + kTcDeqWarps) {
        // ------------------------------------------------------------ dequantising warps
        // thread -> one weight row (lane of the TMEM quarter warp % 4 may address) and
        // kTcAtPerThr of the stage's 4 atoms (part p of the warps 6 + 4p .. 9 + 4p).
        // Each value is the exact d*(q-8) (Q4_0) or d*q (Q8_0) rounded once to bf16.
        // Codes are read through the 128-byte swizzle the TMA wrote them with, so
        // each 8-row phase of a 16-byte load hits 8 distinct bank groups.
        const int quarter = warp & 3;
        const int row = quarter * 32 + lane;
        const int part = (warp - 6) >> 2;
        walk([&](int, int, int it) {
            const int s = it % S, ab = it % a.n_abuf;
            if (misc[1] || !mbar_wait(&full[s], (it / S) & 1, a.err, kErrTimeoutFull)) {
                misc[1] = 1;
                return false;
            }
            const uint8_t* st = smem + (size_t)s * a.stage_bytes;
            const uint8_t* crow = st + a.w_off + (size_t)row * 128;
            const uint4 sc = *reinterpret_cast<const uint4*>(st + a.s_off + (size_t)row * kTcQbs * 4);
            // the scales of this thread's atoms (register selects, no local array)
            uint32_t scw[kTcAtPerThr];
#pragma unroll
            for (int jj = 0; jj < kTcAtPerThr; ++jj) {
                const int j = part * kTcAtPerThr + jj;
                scw[jj] = j == 0 ? sc.x : j == 1 ? sc.y : j == 2 ? sc.z : sc.w;
            }
            bool buf_free = false;  // the operand buffer is waited for after the first atom's math
            // both atoms' code words loaded up front (their latency overlaps the first atom's math)
            constexpr int kWords = WF == kWQ4 ? 8 : 16;  // code words of one atom row
            uint32_t qa[kTcAtPerThr][kWords];
#pragma unroll
            for (int jj = 0; jj < kTcAtPerThr; ++jj)
#pragma unroll
                for (int t = 0; t < kWords / 4; ++t) {
                    const int L = (part * kTcAtPerThr + jj) * (kWords / 4) + t;  // 16-byte chunk of the row
                    const uint4 v = *reinterpret_cast<const uint4*>(crow + (size_t)(L >> 3) * kTcBM * 128 +
                                                                    (((L & 7) ^ (row & 7)) << 4));
                    qa[jj][4 * t] = v.x;
                    qa[jj][4 * t + 1] = v.y;
                    qa[jj][4 * t + 2] = v.z;
                    qa[jj][4 * t + 3] = v.w;
                }
#pragma unroll
            for (int jj = 0; jj < kTcAtPerThr; ++jj) {
                const int j = part * kTcAtPerThr + jj;
                const uint32_t* q = qa[jj];
                const float d0 = __half2float(__ushort_as_half((unsigned short)(scw[jj] & 0xFFFFu)));
                const float d1 = __half2float(__ushort_as_half((unsigned short)(scw[jj] >> 16)));
                uint32_t w[32];
                if constexpr (WF == kWQ4) {
                    // All in bf16x2 (no per-element conversion).  Per block, d = dh + dl with
                    // dh = bf16(d) and dl = d - dh (at most 3 significant bits, exact in
                    // bf16).  Per pair, P = (128 + q_even, 128 + 8 q_odd) built from the
                    // code bits, a = P - (136, 192) = (q - 8, 8 (q - 8)) exactly, and
                    // fma(a, (dh, dh/8), a * (dl, dl/8)) is d (q - 8) rounded once: the
                    // addend a * dl has at most 7 significant bits, so it is exact.
                    uint32_t dh[2], dl[2];
                    const float df[2] = {d0, d1};
#pragma unroll
                    for (int b = 0; b < 2; ++b) {
                        dh[b] = cvt_bf2(df[b], df[b] * 0.125f);
                        const float dlf = df[b] - __uint_as_float(dh[b] << 16);
                        dl[b] = cvt_bf2(dlf, dlf * 0.125f);
                    }
#pragma unroll
                    for (int c = 0; c < 8; ++c) {  // 8-element chunk c of 32-element block c / 4
                        const uint32_t qw = q[c], qs = q[c] >> 1;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {  // byte e: element 2e (low nibble), 2e+1 (high)
                            const uint32_t t = __byte_perm(qw, qs, (uint32_t)e | ((uint32_t)(e + 4) << 8));
                            const uint32_t P = (t & 0x0078000Fu) | 0x43004300u;
                            const uint32_t av = bsub2(P, 0x43404308u);  // (136, 192)
                            w[c * 4 + e] = bfma2(av, dh[c >> 2], bmul2(av, dl[c >> 2]));
                        }
                    }
                } else {
                    // the int8 code byte u = q + 128 under the exponent of 2^15 (m = 2^15 + u)
                    // and fma(m, d, -(2^15 + 128) d) = d q exactly (constant and result fit
                    // 24 bits, for finite scales), rounded once to bf16
                    const float2 dd0 = make_float2(d0, d0), dd1 = make_float2(d1, d1);
                    const float2 cc0 = make_float2(-32896.0f * d0, -32896.0f * d0);
                    const float2 cc1 = make_float2(-32896.0f * d1, -32896.0f * d1);
#pragma unroll
                    for (int c = 0; c < 8; ++c) {
                        const float2 dd = c < 4 ? dd0 : dd1, cc = c < 4 ? cc0 : cc1;
#pragma unroll
                        for (int e = 0; e < 4; ++e) {  // elements 2e, 2e+1 of the chunk
                            const uint32_t u = q[2 * c + (e >> 1)] ^ 0x80808080u;
                            const uint32_t m0 = __byte_perm(u, 0x47000000u, 0x7404u | ((2 * (e & 1)) << 4));
                            const uint32_t m1 = __byte_perm(u, 0x47000000u, 0x7404u | ((2 * (e & 1) + 1) << 4));
                            const float2 v = ffma2(make_float2(__uint_as_float(m0), __uint_as_float(m1)), dd, cc);
                            w[c * 4 + e] = cvt_bf2(v.x, v.y);
                        }
                    }
                }
                if (!buf_free) {
                    if (misc[1] || !mbar_wait(&aempty[ab], ((it / a.n_abuf) & 1) ^ 1, a.err, kErrTimeoutEmpty)) {
                        misc[1] = 1;
                        return false;
                    }
                    if (a.a_tmem) tc_fence_after();
                    buf_free = true;
                }
                if (a.a_tmem) {
                    tmem_st32(tmem + ((uint32_t)(quarter * 32) << 16) + a.a_col + (uint32_t)((ab * kTcQbs + j) * 32), w);
                } else {
                    uint8_t* A = smem + L.abuf + (size_t)(ab * kTcQbs + j) * kTcABytes + (size_t)row * 128;
#pragma unroll
                    for (int c = 0; c < 8; ++c)
                        *reinterpret_cast<uint4*>(A + ((c ^ (row & 7)) << 4)) =
                            make_uint4(w[4 * c], w[4 * c + 1], w[4 * c + 2], w[4 * c + 3]);
                }
            }
            if (a.a_tmem) {
                asm volatile("tcgen05.wait::st.sync.aligned;" ::: "memory");
                tc_fence_before();
            } else {
                // generic-proxy writes -> the tensor cores' async-proxy reads
                asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
            }
            __syncwarp();
            if (lane == 0) mbar_arrive(&afull[ab]);
            return true;
        });
    } else if (warp >= 2 && warp < 6) {
        // ------------------------------------------------------------ epilogue
        const int q = warp & 3;                 // TMEM lane quarter of this warp
        const int et = threadIdx.x - 64;        // 0..127 among the epilogue threads
        const int rl = q * 32 + lane;           // row of the tile (TMEM lane)
        pdl_wait();  // residual rows are the previous kernel's output
        int j = 0;
        units([&](int tile, int, int, bool first) {
            const int buf = j % a.n_acc;
            // one leader waits for the accumulator and the named barrier hands the
            // outcome to all four warps, so they stop (or go on) together: a
            // barrier that some warps skip would never complete
            if (et == 0) {
                const bool ok = misc[1] == 0 && mbar_wait(&tfull[buf], (j / a.n_acc) & 1, a.err, kErrTimeoutFull);
                misc[3] = ok ? 0u : 1u;
                if (!ok) misc[1] = 1;
            }
            named_bar(1, 128);
            if (misc[3]) return false;
            tc_fence_after();
            const uint32_t tbase = tmem + ((uint32_t)(q * 32) << 16) + (uint32_t)(buf * np);
            // 32 token columns of this row: the issuers' accumulators summed in issuer order
            auto ld_acc = [&](int c, float* v) {
                tmem_ld32(tbase + (uint32_t)(c * 32), v);
                for (int i = 1; i < a.n_iss; ++i)
#pragma unroll
                    for (int h = 0; h < 2; ++h) {
                        float w[16];
                        tmem_ld16(tbase + (uint32_t)(i * a.n_acc * np + c * 32 + h * 16), w);
#pragma unroll
                        for (int k = 0; k < 16; ++k) v[h * 16 + k] += w[k];
                    }
            };
            // row handled by this thread: GLU tiles hold 64 gate rows then the 64 matching up rows
            const int n = kGlu ? tile * 64 + (rl & 63) : tile * kTcBM + rl;
            const bool row_ok = n < a.N;
            const int nchunks = np / 32;

            // the LoRA expansion precomputed by lora_expand_launch, added to a bf16
            // projection: per 32-token chunk one ballot of which tokens have an
            // adapter and this row's 32 values loaded together, ahead of the adds
            uint32_t lmask = 0;
            float dv[32];
            auto lora_load = [&](int c, int row) {
                const int bb = c * 32 + lane;
                const int ad = bb < a.nb ? a.lora.adapter[bb] : -1;
                lmask = __ballot_sync(0xffffffffu, ad >= 0 && ad < a.lora.n_adapters);
                const uint16_t* dp = a.lora.dval + (size_t)c * 32 * a.lora.dval_stride + row;
#pragma unroll
                for (int i = 0; i < 32; ++i)
                    dv[i] = ((lmask >> i) & 1u) && row_ok
                                ? __uint_as_float((uint32_t)dp[(size_t)i * a.lora.dval_stride] << 16)
                                : 0.f;
            };
            auto lora_dval = [&](int i, float base) {
                return ((lmask >> i) & 1u) ? round_bf(base + dv[i]) : base;
            };
            auto apply = [&](int c, const float* v) {
                // v[i] = accumulator of (row n, token c*32 + i)
                if (a.lora.adapter) lora_load(c, kGlu && q >= 2 ? a.N + n : n);
                if (kGlu) {
                    float* xq = xch + (size_t)(q & 1) * 32 * 32;
                    if (q >= 2) {
                        for (int i = 0; i < 32; ++i) {
                            const int b = c * 32 + i;
                            float uv = round_bf(v[i]);
                            if (a.lora.adapter && b < a.nb && row_ok) uv = lora_dval(i, uv);
                            xq[i * 32 + lane] = uv;
                        }
                    }
                    named_bar(1, 128);
                    if (q < 2 && row_ok) {
                        for (int i = 0; i < 32; ++i) {
                            const int b = c * 32 + i;
                            if (b >= a.nb) break;
                            float gv = round_bf(v[i]);
                            if (a.lora.adapter) gv = lora_dval(i, gv);
                            const float uv = xq[i * 32 + lane];
                            reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + n] = f2bf(tc_act(gv, a.act) * uv);
                        }
                    }
                    named_bar(1, 128);
                } else if (EPI == kEpiStore && a.ps.tp) {
                    // tensor-parallel all-reduce: the fp32 sums into every rank's inbox (NVLink stores)
                    if (row_ok)
                        for (int i = 0; i < 32; ++i) {
                            const int b = c * 32 + i;
                            if (b >= a.nb) break;
                            for (int r = 0; r < a.ps.tp; ++r) a.ps.inbox[r][(size_t)b * a.out_stride + n] = v[i];
                        }
                } else if (EPI == kEpiStore && a.partial) {
                    if (row_ok)
                        for (int i = 0; i < 32; ++i) {
                            const int b = c * 32 + i;
                            if (b >= a.nb) break;
                            a.partial[(size_t)b * a.out_stride + n] = v[i];
                        }
                } else if (EPI == kEpiStore) {
                    if (row_ok) {
                        const float bv = a.bias ? __uint_as_float((uint32_t)a.bias[n] << 16) : 0.f;
                        for (int i = 0; i < 32; ++i) {
                            const int b = c * 32 + i;
                            if (b >= a.nb) break;
                            float val = round_bf(v[i]);
                            if (a.bias) val = round_bf(val + bv);
                            if (a.lora.adapter) val = lora_dval(i, val);
                            reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + n] = f2bf(val);
                        }
                    }
                } else if (EPI == kEpiResid) {
                    if (row_ok) {
                        for (int i = 0; i < 32; ++i) {
                            const int b = c * 32 + i;
                            if (b >= a.nb) break;
                            float val = round_bf(v[i]);
                            if (a.lora.adapter) val = lora_dval(i, val);
                            const float rr = __uint_as_float((uint32_t)a.resid[(size_t)b * a.resid_stride + n] << 16);
                            reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + n] = f2bf(rr + val);
                        }
                    }
                } else {  // kEpiLmHead
                    for (int i = 0; i < 32; ++i) {
                        const int b = c * 32 + i;
                        if (b >= a.nb) break;
                        unsigned long long key = 0ull;
                        if (row_ok) {
                            reinterpret_cast<bf16*>(a.out)[(size_t)b * a.out_stride + n] = f2bf(v[i]);
                            if (a.logits_f32) a.logits_f32[(size_t)b * a.out_stride + n] = v[i];
                            key = argmax_key(v[i], (uint32_t)(n + a.key_offset));
                        }
#pragma unroll
                        for (int o = 16; o > 0; o >>= 1) {
                            const unsigned long long other = __shfl_xor_sync(0xffffffffu, key, o);
                            key = other > key ? other : key;
                        }
                        if (lane == 0 && key) atomicMax(&best[b], key);
                    }
                }
            };

            // CTAs whose k-block ranges meet this tile
            const long tg0 = (long)tile * a.kblocks;
            const int c_lo = (int)(tg0 / a.kpc), c_hi = (int)((tg0 + a.kblocks - 1) / a.kpc);
            if (c_lo == c_hi) {
                for (int c = 0; c < nchunks; ++c) {
                    float v[32];
                    ld_acc(c, v);
                    if (c == nchunks - 1) {
                        // accumulator fully read: hand it back to the MMA warp
                        tc_fence_before();
                        __syncwarp();
                        if (lane == 0) mbar_arrive(&tempty[buf]);
                    }
                    apply(c, v);
                }
            } else {
                // partial slot: 2 per CTA (its first and its last unit may be cut)
                float* wsp = a.ws + ((size_t)blockIdx.x * 2 + (first ? 0 : 1)) * (size_t)np * kTcBM;
                for (int c = 0; c < nchunks; ++c) {
                    float v[32];
                    ld_acc(c, v);
#pragma unroll
                    for (int i = 0; i < 32; ++i) __stcg(wsp + (size_t)(c * 32 + i) * kTcBM + rl, v[i]);
                }
                tc_fence_before();
                __syncwarp();
                if (lane == 0) mbar_arrive(&tempty[buf]);
                __threadfence();
                named_bar(1, 128);
                if (et == 0) misc[2] = atomicAdd(&a.tile_ctr[tile], 1u);
                named_bar(1, 128);
                const bool last = misc[2] == (uint32_t)(c_hi - c_lo);
                named_bar(1, 128);  // misc[2] is rewritten by the next unit
                if (last) {
                    __threadfence();
                    for (int c = 0; c < nchunks; ++c) {
                        float v[32];
#pragma unroll
                        for (int i = 0; i < 32; ++i) v[i] = 0.f;
                        for (int cc = c_lo; cc <= c_hi; ++cc) {
                            // this tile is CTA cc's first unit unless cc started in an earlier tile
                            const bool cc_first = (int)(((long)cc * a.kpc) / a.kblocks) == tile;
                            const float* p = a.ws + ((size_t)cc * 2 + (cc_first ? 0 : 1)) * (size_t)np * kTcBM;
#pragma unroll
                            for (int i = 0; i < 32; ++i) v[i] += __ldcg(p + (size_t)(c * 32 + i) * kTcBM + rl);
                        }
                        apply(c, v);
                    }
                    if (et == 0) a.tile_ctr[tile] = 0u;
                }
            }
            named_bar(1, 128);  // misc[3] is rewritten for the next unit
            ++j;
            return true;
        });
        if (EPI == kEpiStore && a.ps.tp) {
            // this CTA's peer stores are visible system-wide before it counts itself;
            // the last CTA publishes the phase to every rank
            __threadfence_system();
            named_bar(1, 128);
            if (et == 0) {
                const unsigned int t = atomicAdd(a.ps.ticket, 1u);
                if (t == gridDim.x - 1) {
                    __threadfence_system();
                    if (a.ps.signal) {
                        const unsigned int seq = peer_seq(*a.ps.epoch, a.ps.seq_mul, a.ps.seq_add);
                        for (int r = 0; r < a.ps.tp; ++r) st_release_sys(a.ps.flag[r], seq);
                    }
                    atomicExch(a.ps.ticket, 0u);
                }
            }
        }
        if (EPI == kEpiLmHead) {
            // grid argmax: one 64-bit atomicMax per token per CTA; the last CTA
            // publishes the ids and re-arms the keys for the next step
            named_bar(1, 128);
            for (int b = et; b < a.nb; b += 128)
                if (best[b]) atomicMax(&a.amax[b], best[b]);
            __threadfence();
            named_bar(1, 128);
            if (et == 0) {
                const unsigned int ticket = atomicAdd(a.done, 1u);
                if (ticket == gridDim.x - 1 && !a.publish) {
                    atomicExch(a.done, 0u);  // keys stay for the cross-rank reduction
                } else if (ticket == gridDim.x - 1) {
                    __threadfence();
                    for (int b = 0; b < a.nb; ++b) {
                        const unsigned long long key = atomicExch(&a.amax[b], 0ull);
                        const int32_t id = (int32_t)(~(uint32_t)(key & 0xffffffffull));
                        a.out_ids[b] = id;
                        if (a.chain_tokens) a.chain_tokens[b] = id;
                        if (a.chain_pos) a.chain_pos[b] += 1;
                    }
                    atomicExch(a.done, 0u);
                }
            }
        }
    }
    tc_fence_before();
    __syncthreads();
    if (warp == 1) {
        tc_fence_after();
        asm volatile("tcgen05.dealloc.cta_group::1.sync.aligned.b32 %0, %1;" ::"r"(tmem), "r"(a.tmem_cols)
                     : "memory");
    }
}

// RMSNorm of whole rows into a bf16 buffer (the tensor-core GEMM reads its
// operand through TMA, so the norm that the GEMV fuses runs as its own pass):
// out = bf16(x * rsqrtf(mean(x^2) + eps) * (w [+1])), ops.cu:154-204 / :765-788.
__global__ void __launch_bounds__(256) k_rms_rows(const uint16_t* x, int x_stride, const uint16_t* w, float eps,
                                                  int offset, int K, uint16_t* out, int out_stride) {
    __shared__ float red[8];
    if (threadIdx.x == 0) pdl_trigger();
    pdl_wait();
    const int b = blockIdx.x, tid = threadIdx.x;
    const uint16_t* xr = x + (size_t)b * x_stride;
    float ss = 0.f;
    for (int c = tid * 8; c < K; c += 256 * 8) {
        const uint4 v = *reinterpret_cast<const uint4*>(xr + c);
        const uint32_t* vp = reinterpret_cast<const uint32_t*>(&v);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            ss = fmaf(bf_lo(vp[e]), bf_lo(vp[e]), ss);
            ss = fmaf(bf_hi(vp[e]), bf_hi(vp[e]), ss);
        }
    }
    ss = warp_sum(ss);
    if ((tid & 31) == 0) red[tid >> 5] = ss;
    __syncthreads();
    float tot = 0.f;
#pragma unroll
    for (int i = 0; i < 8; ++i) tot += red[i];
    const float scale = rsqrtf(tot / (float)K + eps);
    const float off = offset ? 1.0f : 0.0f;
    for (int c = tid * 8; c < K; c += 256 * 8) {
        uint4 v = *reinterpret_cast<const uint4*>(xr + c);
        const uint4 wn = *reinterpret_cast<const uint4*>(w + c);
        uint32_t* vp = reinterpret_cast<uint32_t*>(&v);
        const uint32_t* wp = reinterpret_cast<const uint32_t*>(&wn);
#pragma unroll
        for (int e = 0; e < 4; ++e) {
            const float lo = bf_lo(vp[e]) * scale * (bf_lo(wp[e]) + off);
            const float hi = bf_hi(vp[e]) * scale * (bf_hi(wp[e]) + off);
            vp[e] = pack_bf2(lo, hi);
        }
        *reinterpret_cast<uint4*>(out + (size_t)b * out_stride + c) = v;
    }
}

cudaError_t rms_rows_launch(const uint16_t* x, int x_stride, const uint16_t* w, float eps, int offset, int K, int nb,
                            uint16_t* out, int out_stride, cudaStream_t s, bool pdl) {
    if (K % 8 != 0 || nb < 1) return cudaErrorInvalidValue;
    void* params[] = {&x, &x_stride, &w, &eps, &offset, &K, &out, &out_stride};
    return launch_pdl(reinterpret_cast<const void*>(&k_rms_rows), dim3(nb), dim3(256), 0, s, params, pdl);
}

// ------------------------------------------------------------------ host side
namespace {

typedef CUresult (*EncodeTiledFn)(CUtensorMap*, CUtensorMapDataType, cuuint32_t, void*, const cuuint64_t*,
                                  const cuuint64_t*, const cuuint32_t*, const cuuint32_t*, CUtensorMapInterleave,
                                  CUtensorMapSwizzle, CUtensorMapL2promotion, CUtensorMapFloatOOBfill);

EncodeTiledFn encode_fn() {
    static EncodeTiledFn fn = nullptr;
    static std::once_flag once;
    std::call_once(once, [] {
        void* p = nullptr;
        cudaDriverEntryPointQueryResult q;
        if (cudaGetDriverEntryPoint("cuTensorMapEncodeTiled", &p, cudaEnableDefault, &q) == cudaSuccess &&
            q == cudaDriverEntryPointSuccess)
            fn = reinterpret_cast<EncodeTiledFn>(p);
    });
    return fn;
}

}  // namespace

// bf16 [rows, cols] row-major with row pitch `ld` elements; box = 64 columns x
// box_rows, 128-byte swizzle (the K-major operand layout of tcgen05 and the
// conflict-free layout the attention kernel reads with ldmatrix)
bool make_tmap_bf16_sw128(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t ld,
                          uint32_t box_rows) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {ld * 2};
    const cuuint32_t box[2] = {(cuuint32_t)kTcBK, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_BFLOAT16, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, CU_TENSOR_MAP_SWIZZLE_128B, CU_TENSOR_MAP_L2_PROMOTION_L2_256B,
              CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

namespace {

const void* tc_func(int epi, int wf) {
    switch (wf * 4 + epi) {
        case kEpiStore: return reinterpret_cast<const void*>(&k_tc_gemm<kEpiStore, kWBf16>);
        case kEpiResid: return reinterpret_cast<const void*>(&k_tc_gemm<kEpiResid, kWBf16>);
        case kEpiGlu: return reinterpret_cast<const void*>(&k_tc_gemm<kEpiGlu, kWBf16>);
        case kEpiLmHead: return reinterpret_cast<const void*>(&k_tc_gemm<kEpiLmHead, kWBf16>);
        case 4 * kWQ4 + kEpiStore: return reinterpret_cast<const void*>(&k_tc_gemm<kEpiStore, kWQ4>);
        case 4 * kWQ4 + kEpiResid: return reinterpret_cast<const void*>(&k_tc_gemm<kEpiResid, kWQ4>);
        case 4 * kWQ4 + kEpiGlu: return reinterpret_cast<const void*>(&k_tc_gemm<kEpiGlu, kWQ4>);
        case 4 * kWQ8 + kEpiStore: return reinterpret_cast<const void*>(&k_tc_gemm<kEpiStore, kWQ8>);
        case 4 * kWQ8 + kEpiResid: return reinterpret_cast<const void*>(&k_tc_gemm<kEpiResid, kWQ8>);
        case 4 * kWQ8 + kEpiGlu: return reinterpret_cast<const void*>(&k_tc_gemm<kEpiGlu, kWQ8>);
        default: return nullptr;
    }
}

// uint8 [rows, cols] with row pitch `pitch` bytes; box = box_cols x box_rows, no swizzle
bool make_tmap_u8(CUtensorMap* m, const void* base, uint64_t rows, uint64_t cols, uint64_t pitch, uint32_t box_cols,
                  uint32_t box_rows, bool sw128) {
    EncodeTiledFn fn = encode_fn();
    if (!fn) return false;
    const cuuint64_t dims[2] = {cols, rows};
    const cuuint64_t strides[1] = {pitch};
    const cuuint32_t box[2] = {box_cols, box_rows};
    const cuuint32_t estr[2] = {1, 1};
    return fn(m, CU_TENSOR_MAP_DATA_TYPE_UINT8, 2, const_cast<void*>(base), dims, strides, box, estr,
              CU_TENSOR_MAP_INTERLEAVE_NONE, sw128 ? CU_TENSOR_MAP_SWIZZLE_128B : CU_TENSOR_MAP_SWIZZLE_NONE,
              CU_TENSOR_MAP_L2_PROMOTION_L2_256B, CU_TENSOR_MAP_FLOAT_OOB_FILL_NONE) == CUDA_SUCCESS;
}

}  // namespace

bool tc_plan(const GemvArgs& g, int epi, int device, size_t ws_floats_cap, TcPlan* p, std::string* why) {
    if (g.nb < 1 || g.nb > kTcMaxTokens) {
        if (why) *why = "tc_gemm: batch must be 1..256";
        return false;
    }
    if (g.K % kTcBK != 0 || g.K < kTcBK) {  // whole 64-element atoms
        if (why) *why = "tc_gemm: K must be a multiple of 64";
        return false;
    }
    if (epi == kEpiGlu && g.N % 64 != 0) {
        if (why) *why = "tc_gemm: GLU width must be a multiple of 64";
        return false;
    }
    if (g.norm_w) {
        if (why) *why = "tc_gemm: the RMSNorm prologue runs as its own pass (rms_rows_launch)";
        return false;
    }
    const bool q = g.wfmt != kWBf16;
    if (q && (g.K % 256 != 0 || epi == kEpiLmHead)) {
        if (why) *why = "tc_gemm: GGUF weights need K % 256 == 0 (and not the LM head)";
        return false;
    }
    if (g.lora.adapter && !g.lora.dval) {
        if (why) *why = "tc_gemm: the LoRA expansion must be precomputed (lora_expand_launch)";
        return false;
    }
    // tokens padded to whole 32-column TMEM loads
    const int np = (g.nb + 31) / 32 * 32;
    const int sms = num_sms(device);
    const int tiles = epi == kEpiGlu ? g.N / 64 : (g.N + kTcBM - 1) / kTcBM;
    const int atoms = g.K / kTcBK;
    // atoms per stage: the widest of 4/2/1 that divides K and leaves two stages
    const char* env = std::getenv("TI_TC_KBS");
    int kbs_max = env ? std::max(1, std::min(8, std::atoi(env))) : 4;
    const uint32_t xatom = (uint32_t)np * kTcBK * 2;
    const TcSmem L0 = tc_smem_layout(0, 0, np, 0, 0);
    if (q) kbs_max = 4;  // a 16-byte scales box = 4 atoms of 64 columns
    while (!q && kbs_max > 1 && 2 * ((size_t)kbs_max * (kTcABytes + xatom) + 16) > kTcSmemBudget - L0.total)
        kbs_max /= 2;
    const int kbs = kbs_max;
    (void)kbs;
    // stream-K: equal contiguous ranges of the tiles x k-blocks space, one per
    // CTA; the atoms per stage (4, 2 or 1) that give the shortest range, in
    // atoms, wins, with a small bonus for wider (DRAM-friendlier) stages
    int best_kbs = 0, best_kpc = 0;
    double best_cost = 0;
    for (int kb = kbs_max; kb >= (q ? 4 : 1); kb /= 2) {
        if (atoms % kb != 0) continue;
        const long total = (long)tiles * (atoms / kb);
        const int kpc = (int)((total + sms - 1) / sms);
        const double cost = (double)kpc * kb * (kb >= 4 ? 1.0 : kb == 2 ? 1.03 : 1.10);
        if (best_kbs == 0 || cost < best_cost) {
            best_cost = cost;
            best_kbs = kb;
            best_kpc = kpc;
        }
    }
    const int kblocks = atoms / best_kbs;
    const long total = (long)tiles * kblocks;
    p->np = np;
    p->tiles = tiles;
    p->kbs = best_kbs;
    p->kblocks = kblocks;
    p->kpc = best_kpc;
    p->grid = (int)((total + best_kpc - 1) / best_kpc);
    p->ws_floats = (size_t)p->grid * 2 * np * kTcBM;
    if (p->ws_floats > ws_floats_cap) {
        if (why) *why = "tc_gemm: split workspace too small for this batch";
        return false;
    }
    p->cb = g.wfmt == kWQ4 ? 32 : g.wfmt == kWQ8 ? 64 : 0;  // code bytes per 64-column atom row
    p->a_tmem = 0;
    p->a_col = 0;
    p->n_iss = 1;
    p->n_acc = 2;
    if (!q && 4 * np <= 512) {
        // bf16: two issuers (four np-column accumulators) while TMEM holds them
        const char* bi = std::getenv("TI_TC_ISS");
        p->n_iss = bi && std::atoi(bi) == 1 ? 1 : 2;
    }
    if (!q) {
        p->stage_bytes = (uint32_t)best_kbs * (kTcABytes + xatom);
        p->w_off = 0;
        p->x_off = (uint32_t)best_kbs * kTcABytes;
        p->s_off = 0;
        p->n_abuf = 0;
    } else {
        // [token atoms (1024-aligned for the swizzle)][codes][scales]
        p->x_off = 0;
        p->w_off = (uint32_t)best_kbs * xatom;
        p->s_off = p->w_off + (uint32_t)kTcBM * best_kbs * p->cb;
        const uint32_t raw = p->s_off + (uint32_t)kTcBM * best_kbs * 4;
        p->stage_bytes = (raw + 1023u) & ~1023u;
        // two dequantised operand buffers when two raw stages still fit, else one;
        // TI_TC_QBUF=1 asks for one (the freed 64 KB holds about two more raw stages:
        // more weight bytes in flight, dequantisation no longer overlapping the MMA)
        p->n_abuf = 2;
        const size_t abuf = (size_t)best_kbs * kTcABytes;
        const TcSmem Lq = tc_smem_layout(0, 0, np, 0, 0);
        if (2 * abuf + 2 * ((size_t)p->stage_bytes + 24) > kTcSmemBudget - Lq.total) p->n_abuf = 1;
        const char* qb = std::getenv("TI_TC_QBUF");
        if (qb && std::atoi(qb) == 1) p->n_abuf = 1;
        // up to 128 tokens the dequantised operands live in TMEM columns above the two
        // accumulators (the whole 512 columns: one CTA per SM, as the ring's shared
        // memory already forces), so shared memory carries only the raw codes
        const char* qt = std::getenv("TI_TC_QTMEM");
        if (np <= 128 && !(qt && std::atoi(qt) == 0)) {
            p->a_tmem = 1;
            // as many issuers (up to 3) as leave two operand buffers
            p->n_iss = kTcMaxIss;
            while (p->n_iss > 1 && 2 * p->n_iss * np > 256) --p->n_iss;
            const char* qi = std::getenv("TI_TC_QISS");
            if (qi && std::atoi(qi) >= 1) p->n_iss = std::min(p->n_iss, std::atoi(qi));
            const char* qa = std::getenv("TI_TC_QACC");
            if (qa && std::atoi(qa) == 1) p->n_acc = 1;
            p->a_col = (uint32_t)(p->n_acc * p->n_iss * np + 127) / 128 * 128;
            p->n_abuf = std::min(kTcMaxAbuf, (int)((512 - p->a_col) / (uint32_t)(best_kbs * 32)));
        }
    }
    const size_t abuf_bytes = p->a_tmem ? 0 : (size_t)p->n_abuf * best_kbs * kTcABytes;
    p->stages = (int)std::min<size_t>(12, (kTcSmemBudget - L0.total - abuf_bytes) / (p->stage_bytes + 24));  // + full, empty, xfull
    if (p->stages < 2) {
        if (why) *why = "tc_gemm: token tile too large for a two-stage ring";
        return false;
    }
    p->smem = tc_smem_layout(p->stages, p->stage_bytes, np, p->a_tmem ? 0 : p->n_abuf, best_kbs).total;
    if (p->a_tmem && 2 * p->smem <= 228 * 1024) {
        // a second CTA on the SM could hold TMEM columns this one waits for
        if (why) *why = "tc_gemm: TMEM operands need one CTA per SM";
        return false;
    }
    // L2 prefetch window in k-blocks beyond the ring (TI_TC_PF overrides)
    const char* pfe = std::getenv("TI_TC_PF");
    p->pf = pfe ? std::max(0, std::atoi(pfe)) : 0;
    uint32_t cols = 32;
    while (cols < (uint32_t)(p->n_acc * p->n_iss * np)) cols <<= 1;
    p->tmem_cols = p->a_tmem ? 512u : cols;
    p->func = tc_func(epi, g.wfmt);
    p->threads = q ? kTcThreadsQ : kTcThreads;
    if (!p->func) {
        if (why) *why = "tc_gemm: no kernel instance";
        return false;
    }
    return true;
}

cudaError_t tc_launch(const GemvArgs& g, int epi, const TcPlan& p, float* ws, unsigned int* tile_ctr, cudaStream_t s,
                      bool pdl) {
    CUtensorMap mw, mx, ms;
    const uint64_t wrows = epi == kEpiGlu ? 2ull * g.N : (uint64_t)g.N;
    const uint32_t box_rows = epi == kEpiGlu ? 64 : kTcBM;
    if (g.wfmt == kWBf16) {
        if (!make_tmap_bf16_sw128(&mw, g.W, wrows, g.K, g.K, box_rows)) return cudaErrorInvalidValue;
        ms = mw;
    } else {
        // rows of [codes][scales] (wrow_bytes apart): two uint8 maps over the same rows
        const uint64_t pitch = wrow_bytes(g.K, g.wfmt);
        const uint64_t code_bytes = (uint64_t)g.K * p.cb / 64;
        const uint8_t* base = reinterpret_cast<const uint8_t*>(g.W);
        // codes in boxes of 128 bytes x rows, 128-byte swizzle (the dequantising warps' bank pattern)
        if (!make_tmap_u8(&mw, base, wrows, code_bytes, pitch, 128, box_rows, true)) return cudaErrorInvalidValue;
        if (!make_tmap_u8(&ms, base + code_bytes, wrows, (uint64_t)g.K / 16, pitch, (uint32_t)p.kbs * 4, box_rows,
                          false))
            return cudaErrorInvalidValue;
    }
    if (!make_tmap_bf16_sw128(&mx, g.x, g.nb, g.K, g.x_stride, p.np)) return cudaErrorInvalidValue;
    if (!ws || !tile_ctr) return cudaErrorInvalidValue;
    TcKernelArgs a{};
    a.N = g.N;
    a.K = g.K;
    a.nb = g.nb;
    a.np = p.np;
    a.tiles = p.tiles;
    a.kblocks = p.kblocks;
    a.kbs = p.kbs;
    a.kpc = p.kpc;
    a.stages = p.stages;
    a.pf = p.pf;
    a.stage_bytes = p.stage_bytes;
    a.w_off = p.w_off;
    a.x_off = p.x_off;
    a.s_off = p.s_off;
    a.cb = p.cb;
    a.n_abuf = p.n_abuf;
    a.a_tmem = p.a_tmem;
    a.a_col = p.a_col;
    a.n_iss = p.n_iss;
    a.n_acc = p.n_acc;
    a.tmem_cols = p.tmem_cols;
    a.out = g.out;
    a.out_stride = g.out_stride;
    a.bias = g.bias;
    a.resid = g.resid;
    a.resid_stride = g.resid_stride;
    a.act = g.act;
    a.amax = g.amax;
    a.done = g.done;
    a.out_ids = g.out_ids;
    a.chain_tokens = g.chain_tokens;
    a.chain_pos = g.chain_pos;
    a.logits_f32 = g.logits_f32;
    a.key_offset = g.key_offset;
    a.publish = g.publish;
    a.partial = g.partial;
    a.ps = g.ps;
    a.ws = ws;
    a.tile_ctr = tile_ctr;
    a.lora = g.lora;
    a.err = g.err;
    static std::mutex mu;
    static bool attr_set[12] = {};
    {
        std::lock_guard<std::mutex> lk(mu);
        const int idx = (g.wfmt * 4 + epi) % 12;
        if (!attr_set[idx]) {
            cudaError_t e = cudaFuncSetAttribute(p.func, cudaFuncAttributeMaxDynamicSharedMemorySize, 227 * 1024);
            if (e != cudaSuccess) return e;
            attr_set[idx] = true;
        }
    }
    void* params[] = {&mw, &mx, &ms, &a};
    return launch_pdl(p.func, dim3(p.grid), dim3(p.threads), p.smem, s, params, pdl);
}

}  // namespace ti
