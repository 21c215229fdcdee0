// sample.cu — top-p / top-k sampling of bf16 logits rows on the device.
//
// The reference samples on the host after copying the last logits row back
// (src/inference/sampling/top_p.cpp:56-134: temperature, softmax, sort, the
// cumsum >= p nucleus or the k best, then r = u * mass and a walk).  Here one
// CTA samples one row where the LM head left it, with an exact definition that
// needs no sort:
//   * tokens are ordered by logit descending, equal logits by ascending id;
//   * all tokens of one bf16 logit value share one weight
//     w = floor(e * 2^63), e = fp32(exp(v - vmax)), v = logit / temperature
//     when the temperature is != 1 and > 0 (as top_p.cpp:62-64);
//   * cut and pick compare exact 128-bit integer sums of weights:
//       top-p: shortest prefix with weight >= ceil(p * S), S the total;
//       top-k: the first min(k, vocab) tokens;
//       pick:  first token whose running weight reaches max(1, ceil(u * W)),
//              W the cut's weight, u the caller's uniform draw in [0, 1).
// A histogram of the 65536 possible logit values gives every prefix sum, so
// the kernel reads the row twice (histogram, then the pick's id) and never
// sorts.  exp is evaluated by a fixed sequence of IEEE operations (Cody-Waite
// reduction, Taylor series, fused multiply-adds), so the host restatement of
// this definition reproduces every id bit for bit.
#include <cmath>
#include <vector>

#include "common.cuh"
#include "internal.h"
#include "kernels.h"

namespace ti {
namespace {

typedef unsigned __int128 u128;

constexpr int kSampleThreads = 1024;
constexpr int kSampleWarps = kSampleThreads / 32;
constexpr int kKeys = 65536;
constexpr int kKeysPerThread = kKeys / kSampleThreads;  // 64

TI_DEVICE_INLINE uint32_t bf16_key(uint16_t b) {
    if (b == 0x8000u) b = 0;  // -0 and +0 are one value
    return (b & 0x8000u) ? (uint32_t)(~b & 0xffffu) : (uint32_t)(b | 0x8000u);
}

TI_DEVICE_INLINE float key_value(uint32_t key, float temperature) {
    const uint16_t b = (key & 0x8000u) ? (uint16_t)(key & 0x7fffu) : (uint16_t)(~key & 0xffffu);
    const float l = __uint_as_float((uint32_t)b << 16);
    return (temperature != 1.0f && temperature > 0.0f) ? __fdiv_rn(l, temperature) : l;
}

// exp(d), d in [-45, 0]: d = n ln2 + r (ln2 as a 24-bit head plus a tail,
// |r| <= ln2 / 2), exp(r) = sum_{i <= 13} r^i / i! in Horner form, times 2^n.
TI_DEVICE_INLINE double exp_taylor(double d) {
    const double kInvLn2 = 1.4426950408889634;
    const double kLn2Hi = 0.6931471824645996;      // ln 2 rounded to fp32
    const double kLn2Lo = -1.904654299957768e-09;  // ln 2 - kLn2Hi
    const double c[14] = {1.0, 1.0, 0.5, 0.16666666666666666, 0.041666666666666664,
                          0.008333333333333333, 0.001388888888888889, 0.0001984126984126984,
                          2.48015873015873e-05, 2.7557319223985893e-06, 2.755731922398589e-07,
                          2.505210838544172e-08, 2.08767569878681e-09, 1.6059043836821613e-10};
    const double n = rint(__dmul_rn(d, kInvLn2));
    const double r = __fma_rn(-n, kLn2Lo, __fma_rn(-n, kLn2Hi, d));
    double p = c[13];
#pragma unroll
    for (int i = 12; i >= 0; --i) p = __fma_rn(p, r, c[i]);
    const double scale = __longlong_as_double((long long)(1023 + (long long)n) << 52);
    return __dmul_rn(p, scale);
}

TI_DEVICE_INLINE uint64_t key_weight(uint32_t key, float vmax, float temperature) {
    const float d = __fsub_rn(key_value(key, temperature), vmax);
    if (!(d >= -45.0f)) return 0;  // exp(-45) * 2^63 < 1
    const float e = __double2float_rn(exp_taylor((double)d));
    return __double2ull_rz(__dmul_rn((double)e, 9223372036854775808.0));  // * 2^63, exact
}

// ceil(f * x) for finite f and x < 2^100; f <= 0 gives 0, f >= 2^23 saturates
TI_DEVICE_INLINE u128 ceil_mul(float f, u128 x) {
    if (!(f > 0.0f)) return 0;
    const uint32_t b = __float_as_uint(f);
    const uint32_t E = (b >> 23) & 0xffu;
    const u128 m = E ? ((b & 0x7fffffu) | 0x800000u) : (b & 0x7fffffu);
    const int s = E ? 150 - (int)E : 149;  // f = m * 2^-s
    if (s <= 0) return ~(u128)0;
    const u128 prod = m * x;
    if (s >= 127) return prod ? 1 : 0;
    return (prod + (((u128)1 << s) - 1)) >> s;
}

// smallest j in [1, c] with base + j * w >= target (target <= base + c * w)
TI_DEVICE_INLINE uint32_t tie_count(u128 base, uint64_t w, uint32_t c, u128 target) {
    uint32_t lo = 1, hi = c;
    while (lo < hi) {
        const uint32_t mid = lo + (hi - lo) / 2;
        if (base + (u128)mid * w >= target) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

// a row segment read 8 ids per 16-byte load: aligned start and whole loads
TI_DEVICE_INLINE bool vec_ok(const uint16_t* row, int n) {
    return (reinterpret_cast<uintptr_t>(row) & 15) == 0 && (n & 7) == 0;
}

struct SampleShared {
    u128 warp_w[kSampleWarps];
    uint32_t warp_c[kSampleWarps];
    uint32_t warp_max[kSampleWarps];
    uint32_t tile_cnt[2][kSampleWarps];
    u128 wcut;
    uint32_t pick_key, pick_rank;
    int32_t pick_id;
};

// exclusive prefix over the block of (w, c) in thread order; totals to *tw, *tc
TI_DEVICE_INLINE void block_scan(SampleShared& sh, u128 w, uint32_t c, u128* pw, uint32_t* pc, u128* tw,
                                 uint32_t* tc) {
    const int lane = threadIdx.x & 31, warp = threadIdx.x >> 5;
    u128 iw = w;
    uint32_t ic = c;
#pragma unroll
    for (int o = 1; o < 32; o <<= 1) {
        const uint64_t lo = __shfl_up_sync(0xffffffffu, (uint64_t)iw, o);
        const uint64_t hi = __shfl_up_sync(0xffffffffu, (uint64_t)(iw >> 64), o);
        const uint32_t cc = __shfl_up_sync(0xffffffffu, ic, o);
        if (lane >= o) {
            iw += ((u128)hi << 64) | lo;
            ic += cc;
        }
    }
    if (lane == 31) {
        sh.warp_w[warp] = iw;
        sh.warp_c[warp] = ic;
    }
    __syncthreads();
    u128 before_w = 0, all_w = 0;
    uint32_t before_c = 0, all_c = 0;
    for (int i = 0; i < kSampleWarps; ++i) {
        if (i == warp) {
            before_w = all_w;
            before_c = all_c;
        }
        all_w += sh.warp_w[i];
        all_c += sh.warp_c[i];
    }
    *pw = before_w + iw - w;
    *pc = before_c + ic - c;
    *tw = all_w;
    *tc = all_c;
}

// one CTA per row; rows whose kind is greedy keep the LM head's argmax
__global__ void __launch_bounds__(kSampleThreads, 1) k_sample(SampleArgs a) {
    __shared__ SampleShared sh;
    const int b = blockIdx.x;
    const SampleRow prm = a.rows[b];
    if (prm.kind != kSampleTopP && prm.kind != kSampleTopK) return;
    const int tid = threadIdx.x, lane = tid & 31, warp = tid >> 5;
    uint32_t* hist = a.hist + (size_t)b * kKeys;
    const int nseg = (a.vocab + a.seg - 1) / a.seg;

    // 1. clear the histogram
    for (int i = tid; i < kKeys / 4; i += kSampleThreads) reinterpret_cast<uint4*>(hist)[i] = make_uint4(0, 0, 0, 0);
    __syncthreads();

    // 2. count every logit value (warp-aggregated atomics); the largest value.
    // Segments that are 16-byte aligned with a multiple of 8 ids are read 8 ids
    // (one 16-byte load) per thread and iteration, the rest one id at a time.
    uint32_t kmax = 0;
    auto count = [&](uint32_t key, bool valid) {
        const unsigned act = __ballot_sync(0xffffffffu, valid);
        if (valid) {
            kmax = max(kmax, key);
            const unsigned peers = __match_any_sync(act, key);
            if (lane == __ffs(peers) - 1) atomicAdd(&hist[key], (uint32_t)__popc(peers));
        }
    };
    for (int s = 0; s < nseg; ++s) {
        const uint16_t* row = a.logits + (size_t)s * a.seg_stride + (size_t)b * a.row_stride;
        const int n = min(a.seg, a.vocab - s * a.seg);
        if (vec_ok(row, n)) {
            for (int base = 0; base < n; base += 8 * kSampleThreads) {
                const int i = base + 8 * tid;
                const bool valid = i < n;
                uint4 v = make_uint4(0, 0, 0, 0);
                if (valid) v = *reinterpret_cast<const uint4*>(row + i);
                const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                for (int e = 0; e < 8; ++e) count(bf16_key((uint16_t)(w4[e >> 1] >> (16 * (e & 1)))), valid);
            }
        } else {
            for (int base = 0; base < n; base += kSampleThreads) {
                const int i = base + tid;
                count(i < n ? bf16_key(row[i]) : 0u, i < n);
            }
        }
    }
    kmax = __reduce_max_sync(0xffffffffu, kmax);
    if (lane == 0) sh.warp_max[warp] = kmax;
    __syncthreads();
    kmax = 0;
    for (int i = 0; i < kSampleWarps; ++i) kmax = max(kmax, sh.warp_max[i]);
    const float vmax = key_value(kmax, prm.temperature);

    // 3. weights: thread t owns keys kmax - 64t - j, j = 0..63 (descending)
    const int q0 = tid * kKeysPerThread;
    u128 w_t = 0;
    uint32_t c_t = 0;
    for (int j = 0; j < kKeysPerThread; ++j) {
        const int key = (int)kmax - q0 - j;
        if (key < 0) break;
        const uint32_t c = __ldcg(&hist[key]);
        if (c) {
            w_t += (u128)c * key_weight((uint32_t)key, vmax, prm.temperature);
            c_t += c;
        }
    }
    u128 pw, total;
    uint32_t pc, total_c;
    block_scan(sh, w_t, c_t, &pw, &pc, &total, &total_c);

    // the cut's weight, found by the one thread whose keys cross the target
    if (tid == 0) sh.wcut = total;
    __syncthreads();
    if (prm.kind == kSampleTopK) {
        const uint32_t keff = (uint32_t)min(max(prm.k, 1), a.vocab);
        if (pc < keff && keff <= pc + c_t) {
            u128 cum = pw;
            uint32_t n = pc;
            for (int j = 0; j < kKeysPerThread; ++j) {
                const int key = (int)kmax - q0 - j;
                if (key < 0) break;
                const uint32_t c = __ldcg(&hist[key]);
                if (!c) continue;
                const uint64_t w = key_weight((uint32_t)key, vmax, prm.temperature);
                if (n + c >= keff) {
                    sh.wcut = cum + (u128)(keff - n) * w;
                    break;
                }
                n += c;
                cum += (u128)c * w;
            }
        }
    } else {
        u128 target = ceil_mul(prm.p, total);
        if (target < 1) target = 1;
        if (pw < target && target <= pw + w_t) {
            u128 cum = pw;
            for (int j = 0; j < kKeysPerThread; ++j) {
                const int key = (int)kmax - q0 - j;
                if (key < 0) break;
                const uint32_t c = __ldcg(&hist[key]);
                if (!c) continue;
                const uint64_t w = key_weight((uint32_t)key, vmax, prm.temperature);
                if (cum + (u128)c * w >= target) {
                    sh.wcut = cum + (u128)tie_count(cum, w, c, target) * w;
                    break;
                }
                cum += (u128)c * w;
            }
        }
    }
    __syncthreads();

    // 4. the pick: a logit value and the rank of the token among its ids
    float u = prm.u;
    int ctr = 0;
    if (a.draws) {  // a device chain: the row's next pre-generated draw
        ctr = a.draw_ctr[b];
        u = a.draws[(size_t)b * a.draw_cap + min(max(ctr, 0), a.draw_cap - 1)];
    }
    u128 r = ceil_mul(u, sh.wcut);
    if (r < 1) r = 1;
    if (tid == 0) {
        sh.pick_key = kmax;
        sh.pick_rank = 1;
        sh.pick_id = -1;
    }
    __syncthreads();
    if (pw < r && r <= pw + w_t) {
        u128 cum = pw;
        for (int j = 0; j < kKeysPerThread; ++j) {
            const int key = (int)kmax - q0 - j;
            if (key < 0) break;
            const uint32_t c = __ldcg(&hist[key]);
            if (!c) continue;
            const uint64_t w = key_weight((uint32_t)key, vmax, prm.temperature);
            if (cum + (u128)c * w >= r) {
                sh.pick_key = (uint32_t)key;
                sh.pick_rank = tie_count(cum, w, c, r);
                break;
            }
            cum += (u128)c * w;
        }
    }
    __syncthreads();

    // 5. the pick_rank-th id (ascending) holding pick_key: ordered tile scan.
    // A tile gives each thread `per` consecutive ids (8 on the vector path, else 1),
    // so ids run in (warp, lane, element) order: a shuffle scan of the threads'
    // hit counts within the warp and a prefix over the warps' totals rank every hit.
    const uint32_t pkey = sh.pick_key, prank = sh.pick_rank;
    uint32_t seen = 0;
    int tile = 0;
    for (int s = 0; s < nseg && seen < prank; ++s) {
        const uint16_t* row = a.logits + (size_t)s * a.seg_stride + (size_t)b * a.row_stride;
        const int n = min(a.seg, a.vocab - s * a.seg);
        const bool vec = vec_ok(row, n);
        const int per = vec ? 8 : 1;
        for (int base = 0; base < n && seen < prank; base += per * kSampleThreads, ++tile) {
            const int i0 = base + per * tid;
            uint32_t hits = 0;  // bit e: id i0 + e holds pick_key
            if (vec) {
                if (i0 < n) {
                    const uint4 v = *reinterpret_cast<const uint4*>(row + i0);
                    const uint32_t w4[4] = {v.x, v.y, v.z, v.w};
#pragma unroll
                    for (int e = 0; e < 8; ++e)
                        if (bf16_key((uint16_t)(w4[e >> 1] >> (16 * (e & 1)))) == pkey) hits |= 1u << e;
                }
            } else if (i0 < n && bf16_key(row[i0]) == pkey) {
                hits = 1;
            }
            const uint32_t mine = (uint32_t)__popc(hits);
            uint32_t incl = mine;  // inclusive scan of the hit counts over the warp's lanes
#pragma unroll
            for (int o = 1; o < 32; o <<= 1) {
                const uint32_t t = __shfl_up_sync(0xffffffffu, incl, o);
                if (lane >= o) incl += t;
            }
            uint32_t* cnt = sh.tile_cnt[tile & 1];
            if (lane == 31) cnt[warp] = incl;
            __syncthreads();
            uint32_t before = 0, all = 0;
            for (int w2 = 0; w2 < kSampleWarps; ++w2) {
                if (w2 == warp) before = all;
                all += cnt[w2];
            }
            const uint32_t first = seen + before + incl - mine;  // hits before this thread's ids
            if (mine && first < prank && prank <= first + mine) {
                uint32_t need = prank - first, h = hits;
                while (--need) h &= h - 1;  // drop the need-1 lowest hits
                sh.pick_id = s * a.seg + i0 + (__ffs(h) - 1);
            }
            seen += all;  // block-uniform
        }
    }
    __syncthreads();
    if (tid == 0) {
        if (sh.pick_id >= 0) {
            a.out[b] = sh.pick_id;
            if (a.chain_tokens) a.chain_tokens[b] = sh.pick_id;
        } else {
            atomicOr(a.err, kErrBadIndex);  // not reached: the picked value holds >= rank ids
        }
        if (a.draws) {
            if (ctr < 0 || ctr >= a.draw_cap) atomicOr(a.err, kErrBadIndex);  // ran past its pre-drawn steps
            a.draw_ctr[b] = ctr + 1;
        }
    }
}

}  // namespace

size_t sample_scratch_bytes(int nb) { return (size_t)nb * kKeys * sizeof(uint32_t); }

cudaError_t sample_launch(const SampleArgs& a, int nb, cudaStream_t s) {
    if (nb <= 0) return cudaSuccess;
    if (a.vocab <= 0 || a.seg <= 0 || (a.draws && (a.draw_cap <= 0 || !a.draw_ctr))) return cudaErrorInvalidValue;
    SampleArgs args = a;
    void* p[] = {&args};
    return cudaLaunchKernel(reinterpret_cast<const void*>(&k_sample), dim3(nb), dim3(kSampleThreads), p, 0, s);
}

}  // namespace ti

namespace ti {

void SamplerDraws::reset(const ti_sampling& s) {
    cfg = s;
    if (s.kind == TI_SAMPLE_TOP_P) rng.seed(s.seeded ? s.seed : (uint64_t)std::random_device{}());
}

float SamplerDraws::next() {
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);  // top_p.cpp:85
    if (cfg.kind == TI_SAMPLE_TOP_K) {
        std::mt19937_64 fresh(cfg.seeded ? cfg.seed : (uint64_t)std::random_device{}());
        return dist(fresh);
    }
    return dist(rng);
}

ti_status sampler_check(const ti_sampling& s) {
    TI_CHECK(s.kind >= TI_SAMPLE_GREEDY && s.kind <= TI_SAMPLE_TOP_K, TI_ERR_INVALID, "unknown sampler kind %d",
             s.kind);
    if (s.kind == TI_SAMPLE_GREEDY) return TI_OK;
    TI_CHECK(std::isfinite(s.temperature), TI_ERR_INVALID, "sampler temperature must be finite");
    TI_CHECK(s.kind != TI_SAMPLE_TOP_P || std::isfinite(s.p), TI_ERR_INVALID, "top-p: p must be finite");
    TI_CHECK(s.kind != TI_SAMPLE_TOP_K || s.k >= 1, TI_ERR_INVALID, "top-k: k must be >= 1");
    return TI_OK;
}

}  // namespace ti

using namespace ti;

extern "C" ti_status ti_sampler_draws(const ti_sampling* s, int n, float* out) {
    clear_error();
    TI_CHECK(s && (out || n == 0) && n >= 0, TI_ERR_INVALID, "sampler_draws: bad argument");
    if (ti_status st = sampler_check(*s)) return st;
    TI_CHECK(s->kind != TI_SAMPLE_GREEDY, TI_ERR_INVALID, "sampler_draws: a greedy sampler draws nothing");
    SamplerDraws d;
    d.reset(*s);
    for (int i = 0; i < n; ++i) out[i] = d.next();
    return TI_OK;
}

// One sampling call on caller-owned device rows, without an engine: every row's
// sampler and uniform draw come from the host arrays.  Greedy rows take the
// first id of the largest logit (top-k with k = 1 in the exact form).
extern "C" ti_status ti_op_sample(const void* logits, int rows, int vocab, const ti_sampling* params,
                                  const float* draws, int32_t* out, void* stream) {
    clear_error();
    TI_CHECK(logits && params && draws && out, TI_ERR_INVALID, "sample: null argument");
    TI_CHECK(rows >= 0 && vocab >= 1, TI_ERR_INVALID, "sample: %d rows of %d ids", rows, vocab);
    if (rows == 0) return TI_OK;
    std::vector<SampleRow> h((size_t)rows);
    for (int b = 0; b < rows; ++b) {
        const ti_sampling& q = params[b];
        if (ti_status st = sampler_check(q)) return st;
        TI_CHECK(draws[b] >= 0.0f && draws[b] < 1.0f, TI_ERR_INVALID, "sample: row %d: draw outside [0, 1)", b);
        SampleRow& r = h[b];
        if (q.kind == TI_SAMPLE_GREEDY) {
            r.kind = kSampleTopK;
            r.k = 1;
            continue;
        }
        r.kind = q.kind == TI_SAMPLE_TOP_P ? kSampleTopP : kSampleTopK;
        r.temperature = q.temperature;
        r.p = q.p;
        r.k = (int32_t)(q.k > 0x7fffffffu ? 0x7fffffffu : q.k);
        r.u = draws[b];
    }
    cudaStream_t s = (cudaStream_t)stream;
    const size_t rows_bytes = (size_t)rows * sizeof(SampleRow);
    const size_t hist_off = (rows_bytes + 255) / 256 * 256;
    uint8_t* scratch = nullptr;
    TI_CUDA(cudaMallocAsync(reinterpret_cast<void**>(&scratch), hist_off + sample_scratch_bytes(rows) + 16, s));
    int* err = reinterpret_cast<int*>(scratch + hist_off + sample_scratch_bytes(rows));
    SampleArgs a;
    a.logits = reinterpret_cast<const uint16_t*>(logits);
    a.vocab = vocab;
    a.seg = vocab;
    a.row_stride = (size_t)vocab;
    a.rows = reinterpret_cast<const SampleRow*>(scratch);
    a.hist = reinterpret_cast<uint32_t*>(scratch + hist_off);
    a.out = out;
    a.err = err;
    cudaError_t e = cudaMemcpyAsync(scratch, h.data(), rows_bytes, cudaMemcpyHostToDevice, s);
    if (e == cudaSuccess) e = cudaMemsetAsync(err, 0, 4, s);
    if (e == cudaSuccess) e = sample_launch(a, rows, s);
    int herr = 0;
    if (e == cudaSuccess) e = cudaMemcpyAsync(&herr, err, 4, cudaMemcpyDeviceToHost, s);
    if (e == cudaSuccess) e = cudaStreamSynchronize(s);
    cudaError_t f = cudaFreeAsync(scratch, s);
    TI_CHECK(e == cudaSuccess, TI_ERR_CUDA, "sample: %s", cudaGetErrorString(e));
    TI_CUDA(f);
    TI_CHECK(herr == 0, TI_ERR_STATE, "sample: device reported error bits 0x%x", herr);
    return TI_OK;
}
