// common.cuh — device helpers shared by the sm_100a kernels of libti_b200.
#pragma once
#include <cuda.h>
#include <cuda_bf16.h>
#include <cuda_fp16.h>
#include <cuda_runtime.h>
#include <stdint.h>

#ifndef TI_DEVICE_INLINE
#define TI_DEVICE_INLINE __device__ __forceinline__
#endif

namespace ti {

typedef __nv_bfloat16 bf16;

// Error bits written by bounded device waits (engine error word).
enum : int { kErrTimeoutFull = 1, kErrTimeoutEmpty = 2, kErrTimeoutPeer = 4, kErrBadIndex = 8, kErrTimeoutGrid = 16 };
// Iteration bound for every spin on an mbarrier or flag.  try_wait suspends
// for a hardware-defined interval per call, so this is seconds of waiting.
constexpr uint32_t kSpinLimit = 1u << 24;

// ------------------------------------------------------------------ bf16
TI_DEVICE_INLINE float bf_lo(uint32_t u) { return __uint_as_float(u << 16); }
TI_DEVICE_INLINE float bf_hi(uint32_t u) { return __uint_as_float(u & 0xffff0000u); }
TI_DEVICE_INLINE float bf2f(bf16 v) { return __bfloat162float(v); }
TI_DEVICE_INLINE bf16 f2bf(float v) { return __float2bfloat16_rn(v); }
TI_DEVICE_INLINE float round_bf(float v) { return __bfloat162float(__float2bfloat16_rn(v)); }
TI_DEVICE_INLINE uint32_t pack_bf2(float lo, float hi) {
    return (uint32_t)__bfloat16_as_ushort(f2bf(lo)) | ((uint32_t)__bfloat16_as_ushort(f2bf(hi)) << 16);
}

// 2^x (ex2.approx, relative error about 2^-22; 2^-inf = +0)
TI_DEVICE_INLINE float ex2(float x) {
    float y;
    asm("ex2.approx.ftz.f32 %0, %1;" : "=f"(y) : "f"(x));
    return y;
}

// ------------------------------------------------------------------ PDL
// Programmatic dependent launch: a kernel launched with the programmatic
// stream-serialization attribute may start before its predecessor finishes;
// pdl_wait() blocks until the predecessor grid completed and its writes are
// visible, pdl_trigger() lets the successor grid start launching.
TI_DEVICE_INLINE void pdl_wait() { asm volatile("griddepcontrol.wait;" ::: "memory"); }
TI_DEVICE_INLINE void pdl_trigger() { asm volatile("griddepcontrol.launch_dependents;" ::: "memory"); }

// ------------------------------------------------------------------ smem / mbarrier
TI_DEVICE_INLINE uint32_t smem_u32(const void* p) { return (uint32_t)__cvta_generic_to_shared(p); }

TI_DEVICE_INLINE void mbar_init(uint64_t* bar, uint32_t count) {
    asm volatile("mbarrier.init.shared::cta.b64 [%0], %1;" ::"r"(smem_u32(bar)), "r"(count) : "memory");
}
TI_DEVICE_INLINE void fence_barrier_init() {
    asm volatile("fence.mbarrier_init.release.cluster;" ::: "memory");
    asm volatile("fence.proxy.async.shared::cta;" ::: "memory");
}
TI_DEVICE_INLINE void mbar_arrive_expect_tx(uint64_t* bar, uint32_t bytes) {
    asm volatile("mbarrier.arrive.expect_tx.shared::cta.b64 _, [%0], %1;" ::"r"(smem_u32(bar)), "r"(bytes)
                 : "memory");
}
TI_DEVICE_INLINE void mbar_arrive(uint64_t* bar) {
    asm volatile("mbarrier.arrive.shared::cta.b64 _, [%0];" ::"r"(smem_u32(bar)) : "memory");
}
TI_DEVICE_INLINE bool mbar_try_wait(uint64_t* bar, uint32_t parity) {
    uint32_t ok;
    asm volatile(
        "{\n"
        ".reg .pred p;\n"
        "mbarrier.try_wait.parity.shared::cta.b64 p, [%1], %2;\n"
        "selp.u32 %0, 1, 0, p;\n"
        "}\n"
        : "=r"(ok)
        : "r"(smem_u32(bar)), "r"(parity)
        : "memory");
    return ok != 0;
}
TI_DEVICE_INLINE uint64_t global_ns() {
    uint64_t t;
    asm volatile("mov.u64 %0, %%globaltimer;" : "=l"(t));
    return t;
}
// Bounded wait: returns false (and sets `err_bit` in *err) if the phase did not
// complete within kWaitNs of wall time (or kSpinLimit polls).
constexpr uint64_t kWaitNs = 2000000000ull;  // 2 s
TI_DEVICE_INLINE bool mbar_wait_for(uint64_t* bar, uint32_t parity, int* err, int err_bit, uint64_t limit_ns) {
    if (mbar_try_wait(bar, parity)) return true;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < kSpinLimit; ++i) {
        if (mbar_try_wait(bar, parity)) return true;
        if ((i & 255u) == 255u && global_ns() - t0 > limit_ns) break;
    }
    if (err) atomicOr(err, err_bit);
    return false;
}
TI_DEVICE_INLINE bool mbar_wait(uint64_t* bar, uint32_t parity, int* err, int err_bit) {
    return mbar_wait_for(bar, parity, err, err_bit, kWaitNs);
}

// ------------------------------------------------------------------ bulk copies (TMA, non-tensor)
// L2 policy for streamed-once weights: evict first, so activations, KV pages
// and the next kernel's prefetch keep their L2 lines.
TI_DEVICE_INLINE uint64_t l2_policy_evict_first() {
    uint64_t pol;
    asm volatile("createpolicy.fractional.L2::evict_first.b64 %0, 1.0;" : "=l"(pol));
    return pol;
}
// global -> shared bulk copy completing on `bar`; dst, src 16-byte aligned,
// bytes a multiple of 16.  No cluster multicast.
TI_DEVICE_INLINE void bulk_g2s(void* dst, const void* src, uint32_t bytes, uint64_t* bar, uint64_t pol) {
    asm volatile(
        "cp.async.bulk.shared::cluster.global.mbarrier::complete_tx::bytes.L2::cache_hint [%0], [%1], %2, [%3], "
        "%4;" ::"r"(smem_u32(dst)),
        "l"(src), "r"(bytes), "r"(smem_u32(bar)), "l"(pol)
        : "memory");
}
TI_DEVICE_INLINE void prefetch_l2_bulk(const void* src, uint32_t bytes) {
    asm volatile("cp.async.bulk.prefetch.L2.global [%0], %1;" ::"l"(src), "r"(bytes) : "memory");
}

// 2-D tiled bulk-tensor load (TMA) of one box into shared memory, completing on
// `bar`; x (innermost coordinate) must be a multiple of 16 bytes.  No multicast.
TI_DEVICE_INLINE void tma_load_2d(void* dst, const CUtensorMap* map, int x, int y, uint64_t* bar) {
    asm volatile(
        "cp.async.bulk.tensor.2d.shared::cluster.global.tile.mbarrier::complete_tx::bytes [%0], [%1, {%2, %3}], "
        "[%4];" ::"r"(smem_u32(dst)),
        "l"(map), "r"(x), "r"(y), "r"(smem_u32(bar))
        : "memory");
}

// ------------------------------------------------------------------ system-scope flags (peer memory)
TI_DEVICE_INLINE unsigned int ld_acquire_sys(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.sys.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
TI_DEVICE_INLINE unsigned int ld_acquire_gpu(const unsigned int* p) {
    unsigned int v;
    asm volatile("ld.acquire.gpu.global.u32 %0, [%1];" : "=r"(v) : "l"(p) : "memory");
    return v;
}
TI_DEVICE_INLINE void st_release_sys(unsigned int* p, unsigned int v) {
    asm volatile("st.release.sys.global.u32 [%0], %1;" ::"l"(p), "r"(v) : "memory");
}
// Bounded wait until *p has reached `seq` (wrap-safe); false and err_bit on timeout.
// Waits on another rank are bounded more loosely than waits inside a kernel:
// a peer may be seconds behind (building or loading a graph) without being dead.
constexpr uint64_t kPeerWaitNs = 30000000000ull;  // 30 s
constexpr uint32_t kPeerSpinLimit = 1u << 31;
TI_DEVICE_INLINE bool wait_seq_sys_for(const unsigned int* p, unsigned int seq, int* err, int err_bit,
                                       uint64_t limit_ns) {
    if ((int)(ld_acquire_sys(p) - seq) >= 0) return true;
    // an earlier wait of this step already gave up: do not wait again
    if (err && (*reinterpret_cast<volatile int*>(err) & err_bit)) return false;
    const uint64_t t0 = global_ns();
    for (uint32_t i = 0; i < kPeerSpinLimit; ++i) {
        if ((int)(ld_acquire_sys(p) - seq) >= 0) return true;
        if ((i & 63u) == 63u && global_ns() - t0 > limit_ns) break;
    }
    if (err) atomicOr(err, err_bit);
    return false;
}
TI_DEVICE_INLINE bool wait_seq_sys(const unsigned int* p, unsigned int seq, int* err, int err_bit) {
    return wait_seq_sys_for(p, seq, err, err_bit, kPeerWaitNs);
}

// ------------------------------------------------------------------ loads
TI_DEVICE_INLINE uint4 lds128(const void* p) {
    uint4 v;
    asm volatile("ld.shared.v4.u32 {%0,%1,%2,%3}, [%4];"
                 : "=r"(v.x), "=r"(v.y), "=r"(v.z), "=r"(v.w)
                 : "r"(smem_u32(p)));
    return v;
}

// named barrier among `count` threads (multiple of 32)
TI_DEVICE_INLINE void named_bar(int id, int count) {
    asm volatile("bar.sync %0, %1;" ::"r"(id), "r"(count) : "memory");
}

// dot of 8 bf16 weights (packed in uint4) with 8 bf16 activations, fp32 FMA in element order
TI_DEVICE_INLINE float dot8_bf16(const uint4 w, const uint4 x, float acc) {
    acc = fmaf(bf_lo(w.x), bf_lo(x.x), acc);
    acc = fmaf(bf_hi(w.x), bf_hi(x.x), acc);
    acc = fmaf(bf_lo(w.y), bf_lo(x.y), acc);
    acc = fmaf(bf_hi(w.y), bf_hi(x.y), acc);
    acc = fmaf(bf_lo(w.z), bf_lo(x.z), acc);
    acc = fmaf(bf_hi(w.z), bf_hi(x.z), acc);
    acc = fmaf(bf_lo(w.w), bf_lo(x.w), acc);
    acc = fmaf(bf_hi(w.w), bf_hi(x.w), acc);
    return acc;
}

// packed fp32 FMA (sm_100 FFMA2): two independent round-to-nearest FMAs
TI_DEVICE_INLINE float2 ffma2(float2 a, float2 b, float2 c) {
    unsigned long long av = *reinterpret_cast<unsigned long long*>(&a);
    unsigned long long bv = *reinterpret_cast<unsigned long long*>(&b);
    unsigned long long cv = *reinterpret_cast<unsigned long long*>(&c);
    asm("fma.rn.f32x2 %0, %1, %2, %0;" : "+l"(cv) : "l"(av), "l"(bv));
    return *reinterpret_cast<float2*>(&cv);
}
TI_DEVICE_INLINE float2 bf2_to_f2(uint32_t u) { return make_float2(bf_lo(u), bf_hi(u)); }
// 8 bf16 weights x 8 fp32 activations (pairs); even and odd elements accumulate
// in the two lanes of `acc`, each in element order
TI_DEVICE_INLINE float2 dot8_bf16_f2(const uint4 w, const float2* x, float2 acc) {
    acc = ffma2(bf2_to_f2(w.x), x[0], acc);
    acc = ffma2(bf2_to_f2(w.y), x[1], acc);
    acc = ffma2(bf2_to_f2(w.z), x[2], acc);
    acc = ffma2(bf2_to_f2(w.w), x[3], acc);
    return acc;
}

TI_DEVICE_INLINE float warp_sum(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v += __shfl_xor_sync(0xffffffffu, v, o);
    return v;
}
TI_DEVICE_INLINE float warp_max(float v) {
#pragma unroll
    for (int o = 16; o > 0; o >>= 1) v = fmaxf(v, __shfl_xor_sync(0xffffffffu, v, o));
    return v;
}

// float -> order-preserving uint32 (larger float => larger key)
TI_DEVICE_INLINE uint32_t f32_order_key(float f) {
    uint32_t u = __float_as_uint(f);
    return (u & 0x80000000u) ? ~u : (u | 0x80000000u);
}
// argmax key: value in the high word, ~index in the low word (lowest index wins ties)
TI_DEVICE_INLINE unsigned long long argmax_key(float v, uint32_t idx) {
    return ((unsigned long long)f32_order_key(v) << 32) | (unsigned long long)(~idx);
}

}  // namespace ti
