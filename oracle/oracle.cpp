// oracle.cpp — CPU restatement of the reference decode path.
//
// TEST INFRASTRUCTURE ONLY: used by tests/, __graft_entry__.smoke() and the
// CPU-baseline leg of bench.py as the checker.  The product never links it.
// Each function cites the reference (carbon-os/tensor-inference) file:line it
// restates; the declarations in oracle.h carry the full map.
#include "oracle.h"

#include <algorithm>
#include <atomic>
#include <cmath>
#include <cstdlib>
#include <cstring>
#include <functional>
#include <map>
#include <random>
#include <string>
#include <thread>
#include <vector>

// ============================================================ threading
static int g_threads = 0;

extern "C" void orc_set_threads(int n) { g_threads = n; }
extern "C" int orc_get_threads(void) {
    if (g_threads > 0) return g_threads;
    const char* e = std::getenv("ORACLE_THREADS");
    if (e && std::atoi(e) > 0) return std::atoi(e);
    unsigned h = std::thread::hardware_concurrency();
    return h ? (int)h : 1;
}

// Run f(begin, end) over [0, n) split into contiguous chunks, one per thread.
static void parallel_for(size_t n, const std::function<void(size_t, size_t)>& f, size_t min_chunk = 1) {
    int T = orc_get_threads();
    if (n == 0) return;
    size_t chunks = std::min<size_t>((size_t)T, (n + min_chunk - 1) / min_chunk);
    if (chunks <= 1) { f(0, n); return; }
    std::vector<std::thread> th;
    th.reserve(chunks - 1);
    size_t per = n / chunks, rem = n % chunks, b = 0;
    std::vector<std::pair<size_t, size_t>> ranges;
    for (size_t c = 0; c < chunks; ++c) {
        size_t e = b + per + (c < rem ? 1 : 0);
        ranges.emplace_back(b, e);
        b = e;
    }
    for (size_t c = 1; c < chunks; ++c) th.emplace_back(f, ranges[c].first, ranges[c].second);
    f(ranges[0].first, ranges[0].second);
    for (auto& t : th) t.join();
}

// ============================================================ scalar formats
extern "C" float orc_bf16_to_f32(uint16_t b) {
    uint32_t u = (uint32_t)b << 16;
    float f;
    std::memcpy(&f, &u, 4);
    return f;
}

// Round-to-nearest-even, as __float2bfloat16 (used at every rounding point of
// src/backend/cuda/ops.cu).
extern "C" uint16_t orc_f32_to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);  // quiet NaN
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

static inline float bf(uint16_t b) { return orc_bf16_to_f32(b); }
static inline uint16_t tobf(float f) { return orc_f32_to_bf16(f); }

// IEEE binary16 with round-to-nearest-even (GGUF block scales).
extern "C" uint16_t orc_f32_to_f16(float f) {
    uint32_t x;
    std::memcpy(&x, &f, 4);
    uint32_t sign = (x >> 16) & 0x8000u;
    uint32_t ax = x & 0x7fffffffu;
    if (ax >= 0x7f800000u) return (uint16_t)(sign | 0x7c00u | (ax > 0x7f800000u ? 0x200u : 0));
    if (ax >= 0x477ff000u) return (uint16_t)(sign | 0x7c00u);  // rounds to >= 65520 -> inf
    if (ax < 0x38800000u) {                                      // subnormal half
        if (ax < 0x33000000u) return (uint16_t)sign;             // < 2^-25 -> 0
        uint32_t m = (ax & 0x7fffffu) | 0x800000u;
        int e = (int)(ax >> 23);                                 // 102..112
        int shift = 126 - e;                                     // 14..24
        uint32_t half_m = m >> shift;
        uint32_t rem = m & ((1u << shift) - 1u);
        uint32_t halfway = 1u << (shift - 1);
        if (rem > halfway || (rem == halfway && (half_m & 1u))) half_m++;
        return (uint16_t)(sign | half_m);
    }
    uint32_t e = (ax >> 23) - 112u;
    uint32_t m = ax & 0x7fffffu;
    uint32_t h = (e << 10) | (m >> 13);
    uint32_t rem = m & 0x1fffu;
    if (rem > 0x1000u || (rem == 0x1000u && (h & 1u))) h++;
    return (uint16_t)(sign | h);
}

extern "C" float orc_f16_to_f32(uint16_t h) {
    uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    uint32_t e = (h >> 10) & 0x1fu, m = h & 0x3ffu;
    uint32_t x;
    if (e == 0) {
        if (m == 0) x = sign;
        else {
            int s = 0;
            while (!(m & 0x400u)) { m <<= 1; s++; }
            m &= 0x3ffu;
            x = sign | ((uint32_t)(113 - s) << 23) | (m << 13);
        }
    } else if (e == 31) x = sign | 0x7f800000u | (m << 13);
    else x = sign | ((e + 112u) << 23) | (m << 13);
    float f;
    std::memcpy(&f, &x, 4);
    return f;
}

// ============================================================ synthetic data
// Counter-based generator shared (as a specification) with the engine's
// device-side initialiser: element i of a tensor depends only on
// (seed, FNV-1a(name), i), so host and device produce identical bytes.
static inline uint64_t mix64(uint64_t z) {
    z = (z ^ (z >> 30)) * 0xbf58476d1ce4e5b9ULL;
    z = (z ^ (z >> 27)) * 0x94d049bb133111ebULL;
    return z ^ (z >> 31);
}

extern "C" uint64_t orc_name_hash(const char* name) {
    uint64_t h = 0xcbf29ce484222325ULL;
    for (const unsigned char* p = (const unsigned char*)name; *p; ++p) {
        h ^= *p;
        h *= 0x100000001b3ULL;
    }
    return h;
}

static inline float synth_unit(uint64_t key, uint64_t i, float c) {
    uint64_t x = mix64(key + (i + 1) * 0x9E3779B97F4A7C15ULL);
    int32_t s = (int32_t)(x & 0xffffu) + (int32_t)((x >> 16) & 0xffffu) + (int32_t)((x >> 32) & 0xffffu) +
                (int32_t)(x >> 48) - 131070;
    return (float)s * c;  // |s| < 2^18: exact in fp32; one rounding
}

static inline float synth_scale(float std_) { return (float)((double)std_ * 1.7320508075688772 / 65536.0); }

extern "C" void orc_fill_bf16(uint16_t* out, size_t n, uint64_t seed, uint64_t name_hash, float std_) {
    const uint64_t key = mix64(seed ^ name_hash);
    const float c = synth_scale(std_);
    parallel_for(n, [&](size_t b, size_t e) {
        for (size_t i = b; i < e; ++i) out[i] = tobf(synth_unit(key, i, c));
    }, 1 << 16);
}

extern "C" void orc_fill_f32(float* out, size_t n, uint64_t seed, uint64_t name_hash, float std_) {
    const uint64_t key = mix64(seed ^ name_hash);
    const float c = synth_scale(std_);
    parallel_for(n, [&](size_t b, size_t e) {
        for (size_t i = b; i < e; ++i) out[i] = synth_unit(key, i, c);
    }, 1 << 16);
}

extern "C" void orc_fill_ids(int32_t* out, size_t n, uint64_t seed, uint64_t name_hash, int32_t vocab) {
    const uint64_t key = mix64(seed ^ name_hash);
    for (size_t i = 0; i < n; ++i)
        out[i] = (int32_t)(mix64(key + (i + 1) * 0x9E3779B97F4A7C15ULL) % (uint64_t)vocab);
}

// ============================================================ ops
// ops.cu:46-88 — row gather.
extern "C" void orc_embedding(const uint16_t* w, int vocab, int hidden, const int32_t* ids, int n, uint16_t* out) {
    for (int t = 0; t < n; ++t) {
        int id = ids[t];
        if (id < 0 || id >= vocab) id = 0;
        std::memcpy(out + (size_t)t * hidden, w + (size_t)id * hidden, (size_t)hidden * 2);
    }
}

// fp32 dot product of two bf16 rows; 16 independent fp32 partial sums combined
// in double: a fixed order, independent of the thread count.
static inline float dot_bf16(const uint16_t* a, const uint16_t* b, int K) {
    float acc[16] = {0};
    int k = 0;
    for (; k + 16 <= K; k += 16)
        for (int j = 0; j < 16; ++j) acc[j] += bf(a[k + j]) * bf(b[k + j]);
    double s = 0;
    for (int j = 0; j < 16; ++j) s += acc[j];
    for (; k < K; ++k) s += (double)bf(a[k]) * bf(b[k]);
    return (float)s;
}

static inline float dot_bf16_f32(const uint16_t* a, const float* b, int K) {
    float acc[16] = {0};
    int k = 0;
    for (; k + 16 <= K; k += 16)
        for (int j = 0; j < 16; ++j) acc[j] += bf(a[k + j]) * b[k + j];
    double s = 0;
    for (int j = 0; j < 16; ++j) s += acc[j];
    for (; k < K; ++k) s += (double)bf(a[k]) * b[k];
    return (float)s;
}

// The same sum as dot_bf16 over operands already widened to fp32 (the widening
// is exact): 16 independent fp32 partial sums combined in double.
static inline float dot_f32_fixed(const float* a, const float* b, int K) {
    float acc[16] = {0};
    int k = 0;
    for (; k + 16 <= K; k += 16)
        for (int j = 0; j < 16; ++j) acc[j] += a[k + j] * b[k + j];
    double s = 0;
    for (int j = 0; j < 16; ++j) s += acc[j];
    for (; k < K; ++k) s += (double)a[k] * b[k];
    return (float)s;
}

// C[m, n] = store(dot(A[m], B[n])): A widened once, each B row once per thread
template <class F>
static void matmul_rows(const uint16_t* a, const uint16_t* b, int M, int N, int K, F store) {
    std::vector<float> af((size_t)M * K);
    parallel_for((size_t)M * K, [&](size_t i0, size_t i1) {
        for (size_t i = i0; i < i1; ++i) af[i] = bf(a[i]);
    }, 1 << 16);
    parallel_for((size_t)N, [&](size_t n0, size_t n1) {
        std::vector<float> row((size_t)K);
        for (size_t n = n0; n < n1; ++n) {
            const uint16_t* bn = b + n * (size_t)K;
            for (int k = 0; k < K; ++k) row[k] = bf(bn[k]);
            for (int m = 0; m < M; ++m) store((size_t)m * N + n, dot_f32_fixed(af.data() + (size_t)m * K, row.data(), K));
        }
    }, 16);
}

// ops.cu:94-148 — C[M,N] = A[M,K] @ B[N,K]^T, fp32 accumulate, bf16 output.
extern "C" void orc_matmul_t_bf16_f32out(const uint16_t* a, const uint16_t* b, float* c, int M, int N, int K) {
    matmul_rows(a, b, M, N, K, [&](size_t i, float v) { c[i] = v; });
}

extern "C" void orc_matmul_t_bf16(const uint16_t* a, const uint16_t* b, uint16_t* c, int M, int N, int K) {
    matmul_rows(a, b, M, N, K, [&](size_t i, float v) { c[i] = tobf(v); });
}

extern "C" void orc_matmul_t_f32(const float* a, const float* b, float* c, int M, int N, int K) {
    parallel_for((size_t)N, [&](size_t n0, size_t n1) {
        for (size_t n = n0; n < n1; ++n)
            for (int m = 0; m < M; ++m) {
                double s = 0;
                for (int k = 0; k < K; ++k) s += (double)a[(size_t)m * K + k] * b[n * K + k];
                c[(size_t)m * N + n] = (float)s;
            }
    }, 16);
}

// ops.cu:154-204 (offset = 0) and 726-774 (offset = 1, Gemma's w + 1).
// out = bf16((x * rsqrt(mean(x^2) + eps)) * w), fp32 sum of squares.
extern "C" void orc_rms_norm(const uint16_t* x, const uint16_t* w, uint16_t* out, int rows, int hidden, float eps,
                             int offset) {
    for (int r = 0; r < rows; ++r) {
        const uint16_t* xr = x + (size_t)r * hidden;
        double ss = 0;
        for (int i = 0; i < hidden; ++i) ss += (double)bf(xr[i]) * bf(xr[i]);
        float scale = 1.0f / std::sqrt((float)ss / (float)hidden + eps);
        for (int i = 0; i < hidden; ++i) {
            float wi = bf(w[i]);
            if (offset) wi = wi + 1.0f;
            out[(size_t)r * hidden + i] = tobf(bf(xr[i]) * scale * wi);
        }
    }
}

// ops.cu:235-278 — per-pair angular frequency, with Llama-3 three-regime scaling.
extern "C" void orc_rope_freqs(int head_dim, float theta, const orc_rope_scaling* sc, float* freqs) {
    const int half = head_dim / 2;
    const float pi2 = 2.0f * (float)M_PI;
    orc_rope_scaling d = {0, 1.0f, 1.0f, 1.0f, 8192};
    if (!sc) sc = &d;
    const float low_wavelen = (float)sc->original_max_pos / sc->low_freq_factor;
    const float high_wavelen = (float)sc->original_max_pos / sc->high_freq_factor;
    for (int i = 0; i < half; ++i) {
        float base = 1.0f / std::pow(theta, (2.0f * (float)i) / (float)head_dim);
        if (!sc->apply_scaling) { freqs[i] = base; continue; }
        float wavelen = pi2 / base;
        float f;
        if (wavelen < high_wavelen) f = base;
        else if (wavelen > low_wavelen) f = base / sc->factor;
        else {
            float smooth = ((float)sc->original_max_pos / wavelen - sc->low_freq_factor) /
                           (sc->high_freq_factor - sc->low_freq_factor);
            f = (1.0f - smooth) * (base / sc->factor) + smooth * base;
        }
        freqs[i] = f;
    }
}

// ops.cu:210-233 — rotate-half pairs (i, i + d/2), angle = float(pos) * freq_i.
extern "C" void orc_rope(const uint16_t* x, uint16_t* out, int seq, int heads, int head_dim, int seq_offset,
                         const float* freqs) {
    const int half = head_dim / 2;
    for (int p = 0; p < seq; ++p)
        for (int h = 0; h < heads; ++h) {
            size_t base = ((size_t)p * heads + h) * head_dim;
            for (int i = 0; i < half; ++i) {
                float ang = (float)(p + seq_offset) * freqs[i];
                float c = std::cos(ang), s = std::sin(ang);
                float x0 = bf(x[base + i]), x1 = bf(x[base + i + half]);
                out[base + i] = tobf(x0 * c - x1 * s);
                out[base + i + half] = tobf(x0 * s + x1 * c);
            }
        }
}

// ops.cu:318-381
extern "C" void orc_silu(const uint16_t* x, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) {
        float v = bf(x[i]);
        out[i] = tobf(v / (1.0f + std::exp(-v)));
    }
}
extern "C" void orc_mul(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = tobf(bf(a[i]) * bf(b[i]));
}
extern "C" void orc_add(const uint16_t* a, const uint16_t* b, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = tobf(bf(a[i]) + bf(b[i]));
}
// ops.cu:707-724 — tanh-form GELU.
extern "C" void orc_gelu(const uint16_t* x, uint16_t* out, size_t n) {
    const float c1 = 0.7978845608f, c2 = 0.044715f;
    for (size_t i = 0; i < n; ++i) {
        float v = bf(x[i]);
        float val = 0.5f * v * (1.0f + std::tanh(c1 * (v + c2 * v * v * v)));
        out[i] = tobf(val);
    }
}
// ops.cu:776-788
extern "C" void orc_mul_scalar(const uint16_t* x, float s, uint16_t* out, size_t n) {
    for (size_t i = 0; i < n; ++i) out[i] = tobf(bf(x[i]) * s);
}
// ops.cu:671-701
extern "C" void orc_add_bias(const uint16_t* x, const uint16_t* bias, uint16_t* out, int rows, int hidden) {
    for (int r = 0; r < rows; ++r)
        for (int i = 0; i < hidden; ++i)
            out[(size_t)r * hidden + i] = tobf(bf(x[(size_t)r * hidden + i]) + bf(bias[i]));
}

// ops.cu:387-438 — row softmax in fp32.
extern "C" void orc_softmax_f32(float* x, int rows, int cols) {
    for (int r = 0; r < rows; ++r) {
        float* p = x + (size_t)r * cols;
        float m = -1e38f;
        for (int i = 0; i < cols; ++i) m = std::max(m, p[i]);
        double s = 0;
        for (int i = 0; i < cols; ++i) s += std::exp(p[i] - m);
        float inv = 1.0f / (float)s;
        for (int i = 0; i < cols; ++i) p[i] = std::exp(p[i] - m) * inv;
    }
}

// ops.cu:444-544 — GQA attention in fp32, bf16 output.  q head h reads kv head
// h / (n_heads / n_kv).  The mask applies only when causal && seq > 1 (so a
// decode step ignores sliding_window, as the reference does).
extern "C" void orc_attention(const uint16_t* q, const uint16_t* k, const uint16_t* v, uint16_t* out, int seq,
                              int n_heads, int kv_len, int n_kv, int head_dim, int causal, int sliding_window) {
    const int group = n_heads / n_kv;
    const float scale = 1.0f / std::sqrt((float)head_dim);
    parallel_for((size_t)n_heads, [&](size_t h0, size_t h1) {
        std::vector<float> sc((size_t)kv_len);
        std::vector<double> acc((size_t)head_dim);
        for (size_t h = h0; h < h1; ++h) {
            const int kvh = (int)h / group;
            for (int i = 0; i < seq; ++i) {
                const uint16_t* qi = q + ((size_t)i * n_heads + h) * head_dim;
                for (int j = 0; j < kv_len; ++j) {
                    const uint16_t* kj = k + ((size_t)j * n_kv + kvh) * head_dim;
                    double s = 0;
                    for (int d = 0; d < head_dim; ++d) s += (double)bf(qi[d]) * bf(kj[d]);
                    sc[j] = scale * (float)s;
                }
                if (causal && seq > 1) {
                    const int off = kv_len - seq;
                    for (int j = 0; j < kv_len; ++j) {
                        bool mask = j > off + i;
                        if (sliding_window > 0 && j <= off + i - sliding_window) mask = true;
                        if (mask) sc[j] = -1e38f;
                    }
                }
                orc_softmax_f32(sc.data(), 1, kv_len);
                std::fill(acc.begin(), acc.end(), 0.0);
                for (int j = 0; j < kv_len; ++j) {
                    const uint16_t* vj = v + ((size_t)j * n_kv + kvh) * head_dim;
                    for (int d = 0; d < head_dim; ++d) acc[d] += (double)sc[j] * bf(vj[d]);
                }
                uint16_t* o = out + ((size_t)i * n_heads + h) * head_dim;
                for (int d = 0; d < head_dim; ++d) o[d] = tobf((float)acc[d]);
            }
        }
    });
}

// ============================================================ GGUF blocks
// Q4_0 (ggml quantize_row_q4_0_ref): per 32-block, `max` = the signed value of
// largest magnitude, d = max / -8, q = min(15, (int8)(x / d + 8.5)),
// byte j = q[j] | q[j+16] << 4.  Dequantised weight = (q - 8) * fp16(d).
extern "C" void orc_q4_0_quantize(const float* x, size_t n, uint8_t* blocks) {
    for (size_t b = 0; b < n / 32; ++b) {
        const float* xb = x + b * 32;
        float amax = 0, mx = 0;
        for (int j = 0; j < 32; ++j)
            if (std::fabs(xb[j]) > amax) { amax = std::fabs(xb[j]); mx = xb[j]; }
        const float d = mx / -8.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint8_t* out = blocks + b * 18;
        uint16_t dh = orc_f32_to_f16(d);
        std::memcpy(out, &dh, 2);
        for (int j = 0; j < 16; ++j) {
            int q0 = std::min(15, (int)(int8_t)(xb[j] * id + 8.5f));
            int q1 = std::min(15, (int)(int8_t)(xb[j + 16] * id + 8.5f));
            out[2 + j] = (uint8_t)(q0 | (q1 << 4));
        }
    }
}
extern "C" void orc_q4_0_dequantize(const uint8_t* blocks, size_t n, float* out) {
    for (size_t b = 0; b < n / 32; ++b) {
        const uint8_t* in = blocks + b * 18;
        uint16_t dh;
        std::memcpy(&dh, in, 2);
        const float d = orc_f16_to_f32(dh);
        for (int j = 0; j < 16; ++j) {
            out[b * 32 + j] = (float)((int)(in[2 + j] & 0xf) - 8) * d;
            out[b * 32 + j + 16] = (float)((int)(in[2 + j] >> 4) - 8) * d;
        }
    }
}
// Q8_0 (ggml quantize_row_q8_0_ref): d = amax / 127, q = round(x / d).
extern "C" void orc_q8_0_quantize(const float* x, size_t n, uint8_t* blocks) {
    for (size_t b = 0; b < n / 32; ++b) {
        const float* xb = x + b * 32;
        float amax = 0;
        for (int j = 0; j < 32; ++j) amax = std::max(amax, std::fabs(xb[j]));
        const float d = amax / 127.0f;
        const float id = d != 0.0f ? 1.0f / d : 0.0f;
        uint8_t* out = blocks + b * 34;
        uint16_t dh = orc_f32_to_f16(d);
        std::memcpy(out, &dh, 2);
        for (int j = 0; j < 32; ++j) out[2 + j] = (uint8_t)(int8_t)std::lround(xb[j] * id);
    }
}
extern "C" void orc_q8_0_dequantize(const uint8_t* blocks, size_t n, float* out) {
    for (size_t b = 0; b < n / 32; ++b) {
        const uint8_t* in = blocks + b * 34;
        uint16_t dh;
        std::memcpy(&dh, in, 2);
        const float d = orc_f16_to_f32(dh);
        for (int j = 0; j < 32; ++j) out[b * 32 + j] = (float)(int8_t)in[2 + j] * d;
    }
}

extern "C" void orc_matmul_t_q(const uint16_t* x, const uint8_t* wq, int qtype, uint16_t* y, float* y32, int M, int N,
                               int K) {
    const size_t bpr = (size_t)K / 32 * (qtype == ORC_W_Q4_0 ? 18 : 34);
    parallel_for((size_t)N, [&](size_t n0, size_t n1) {
        std::vector<float> row((size_t)K);
        for (size_t n = n0; n < n1; ++n) {
            if (qtype == ORC_W_Q4_0) orc_q4_0_dequantize(wq + n * bpr, (size_t)K, row.data());
            else orc_q8_0_dequantize(wq + n * bpr, (size_t)K, row.data());
            for (int m = 0; m < M; ++m) {
                float v = dot_bf16_f32(x + (size_t)m * K, row.data(), K);
                if (y) y[(size_t)m * N + n] = tobf(v);
                if (y32) y32[(size_t)m * N + n] = v;
            }
        }
    }, 16);
}

// ============================================================ PKM
extern "C" float orc_pkm_dist(const float* q, const float* c, int dim) {
    float acc = 0.0f;
    for (int t = 0; t < dim; ++t) {
        float d = q[t] - c[t];
        acc = std::fma(d, d, acc);
    }
    return acc;
}

static int pkm_argmin(const float* q, const float* C, int n_codes, int dim) {
    int best = 0;
    float bd = orc_pkm_dist(q, C, dim);
    for (int k = 1; k < n_codes; ++k) {
        float d = orc_pkm_dist(q, C + (size_t)k * dim, dim);
        if (d < bd) { bd = d; best = k; }
    }
    return best;
}

extern "C" void orc_pkm_assign(const float* c1, const float* c2, int n_codes, int half_dim, const float* queries,
                               int n, int32_t* addr) {
    parallel_for((size_t)n, [&](size_t b, size_t e) {
        for (size_t i = b; i < e; ++i) {
            const float* q = queries + i * (size_t)(2 * half_dim);
            int a = pkm_argmin(q, c1, n_codes, half_dim);
            int c = pkm_argmin(q + half_dim, c2, n_codes, half_dim);
            addr[i] = a * n_codes + c;
        }
    }, 64);
}

extern "C" void orc_pkm_build_table(const int32_t* centroid_addr, int n_adapters, int32_t* table, int table_size) {
    for (int i = 0; i < table_size; ++i) table[i] = -1;
    for (int id = 0; id < n_adapters; ++id) {
        int a = centroid_addr[id];
        if (a >= 0 && a < table_size && table[a] < 0) table[a] = id;
    }
}

extern "C" int32_t orc_argmax_f32(const float* x, int n) {
    int best = 0;
    for (int i = 1; i < n; ++i)
        if (x[i] > x[best]) best = i;
    return best;
}

// ============================================================ sampling
// The reference's stochastic samplers (src/inference/sampling/top_p.cpp), one
// logits row at a time.  The uniform draw u in [0, 1) is an argument: the
// reference takes it from std::uniform_real_distribution<float> over
// std::mt19937_64 (top_p.cpp:84-86, :124-126), which orc_sample_draws
// reproduces with the same standard-library types.
namespace {

// token ids ordered by v descending: all of them (first_n < 0, std::sort as
// top_p.cpp:71-73) or the first first_n (std::partial_sort as top_p.cpp:113-114,
// also when first_n covers every id: the two order equal values differently).
// stable == 0 keeps the library's order of equal values (the reference's);
// stable != 0 orders them by ascending id.
std::vector<int32_t> order_desc(const std::vector<float>& v, long first_n, int stable) {
    std::vector<int32_t> idx(v.size());
    for (size_t i = 0; i < idx.size(); ++i) idx[i] = (int32_t)i;
    auto gt = [&](int32_t a, int32_t b) { return v[a] > v[b]; };
    auto gt_stable = [&](int32_t a, int32_t b) { return v[a] > v[b] || (v[a] == v[b] && a < b); };
    if (first_n < 0) {
        if (stable) std::sort(idx.begin(), idx.end(), gt_stable);
        else std::sort(idx.begin(), idx.end(), gt);
    } else {
        if (stable) std::partial_sort(idx.begin(), idx.begin() + first_n, idx.end(), gt_stable);
        else std::partial_sort(idx.begin(), idx.begin() + first_n, idx.end(), gt);
    }
    return idx;
}

}  // namespace

// TopP::sample, top_p.cpp:56-99.
extern "C" int32_t orc_sample_top_p(const float* logits, int vocab, float temperature, float p, float u,
                                    int stable) {
    std::vector<float> v(logits, logits + vocab);
    if (temperature != 1.0f && temperature > 0.0f)
        for (float& x : v) x /= temperature;
    float mx = v[0];
    for (int i = 1; i < vocab; ++i) mx = std::max(mx, v[i]);
    float sum = 0.0f;
    for (float& x : v) {
        x = std::exp(x - mx);
        sum += x;
    }
    for (float& x : v) x /= sum;
    std::vector<int32_t> idx = order_desc(v, -1, stable);
    float cum = 0.0f;
    int cut = vocab;
    for (int i = 0; i < vocab; ++i) {
        cum += v[idx[i]];
        if (cum >= p) {
            cut = i + 1;
            break;
        }
    }
    const float r = u * cum;
    float acc = 0.0f;
    for (int i = 0; i < cut; ++i) {
        acc += v[idx[i]];
        if (r <= acc) return idx[i];
    }
    return idx[0];
}

// TopK::sample, top_p.cpp:102-134.
extern "C" int32_t orc_sample_top_k(const float* logits, int vocab, float temperature, int k, float u, int stable) {
    std::vector<float> v(logits, logits + vocab);
    const size_t keff = std::min((size_t)(uint32_t)k, (size_t)vocab);
    if (temperature != 1.0f && temperature > 0.0f)
        for (float& x : v) x /= temperature;
    std::vector<int32_t> idx = order_desc(v, (long)keff, stable);
    const float mx = v[idx[0]];
    std::vector<float> pr(keff);
    float sum = 0.0f;
    for (size_t i = 0; i < keff; ++i) {
        pr[i] = std::exp(v[idx[i]] - mx);
        sum += pr[i];
    }
    const float r = u * sum;
    float acc = 0.0f;
    for (size_t i = 0; i < keff; ++i) {
        acc += pr[i];
        if (r <= acc) return idx[i];
    }
    return idx[0];
}

// ---------------------------------------------------------------- exact form
// The device sampler's definition of the same two samplers, restated here so
// that its ids can be checked bit for bit.  Inputs are the bf16 logits the
// reference's samplers receive from the model (top_p.cpp:31-39 widens them).
// Tokens are ordered by logit descending, equal logits by ascending id; every
// token of one logit value has weight w = floor(e * 2^63), e = the fp32
// rounding of exp(v - vmax) (v = logit / temperature when the temperature is
// != 1 and > 0, as top_p.cpp:62-64), and all cumulative sums are exact
// 128-bit integers, so no decision depends on a summation order.
//   top-p: the cut is the shortest prefix whose weight reaches ceil(p * S),
//          S the total weight (the cumsum >= p test of top_p.cpp:76-81);
//   top-k: the first min(k, vocab) tokens (top_p.cpp:111-115);
//   pick:  the first token whose running weight reaches max(1, ceil(u * W)),
//          W the cut's weight (r = u * cumsum and the r <= acc walk,
//          top_p.cpp:88-93, :127-132).
namespace {

typedef unsigned __int128 u128;

// exp(d) for d in [-45, 0], double: Cody-Waite reduction d = n ln2 + r with ln2
// split into a 24-bit head and a tail (|r| <= ln2 / 2), exp(r) by its Taylor
// series to degree 13 in Horner form with fused multiply-adds, times 2^n built
// from its exponent bits.  Every step is a correctly rounded IEEE operation, so
// the CUDA sampler (csrc/sample.cu) computes the same bits.
double exp_taylor(double d) {
    const double kInvLn2 = 1.4426950408889634;
    const double kLn2Hi = 0.6931471824645996;     // ln 2 rounded to fp32
    const double kLn2Lo = -1.904654299957768e-09; // ln 2 - kLn2Hi
    static const double c[14] = {1.0, 1.0, 0.5, 0.16666666666666666, 0.041666666666666664,
                                 0.008333333333333333, 0.001388888888888889, 0.0001984126984126984,
                                 2.48015873015873e-05, 2.7557319223985893e-06, 2.755731922398589e-07,
                                 2.505210838544172e-08, 2.08767569878681e-09, 1.6059043836821613e-10};
    const double n = std::nearbyint(d * kInvLn2);
    const double r = std::fma(-n, kLn2Lo, std::fma(-n, kLn2Hi, d));
    double p = c[13];
    for (int i = 12; i >= 0; --i) p = std::fma(p, r, c[i]);
    const uint64_t bits = (uint64_t)(1023 + (int64_t)n) << 52;
    double scale;
    std::memcpy(&scale, &bits, 8);
    return p * scale;
}

// bf16 bits -> unsigned key, ordered as the values (-0 and +0 share one key)
inline uint32_t bf16_key(uint16_t b) {
    if (b == 0x8000u) b = 0;
    return (b & 0x8000u) ? (uint32_t)(~b & 0xffffu) : (uint32_t)(b | 0x8000u);
}

inline uint16_t key_bf16(uint32_t k) { return (k & 0x8000u) ? (uint16_t)(k & 0x7fffu) : (uint16_t)(~k & 0xffffu); }

inline float scaled(uint32_t key, float temperature) {
    const float l = bf(key_bf16(key));
    return (temperature != 1.0f && temperature > 0.0f) ? l / temperature : l;
}

// weight of one token of logit key `key`, vmax the largest scaled logit
uint64_t key_weight(uint32_t key, float vmax, float temperature) {
    const float d = scaled(key, temperature) - vmax;
    if (!(d >= -45.0f)) return 0;  // exp(-45) * 2^63 < 1
    const float e = (float)exp_taylor((double)d);
    return (uint64_t)std::ldexp((double)e, 63);
}

// ceil(f * x) for finite f and x < 2^100; f <= 0 gives 0, f >= 2^23 saturates
u128 ceil_mul(float f, u128 x) {
    if (!(f > 0.0f)) return 0;
    uint32_t b;
    std::memcpy(&b, &f, 4);
    const uint32_t E = (b >> 23) & 0xffu;
    const u128 m = E ? ((b & 0x7fffffu) | 0x800000u) : (b & 0x7fffffu);
    const int s = E ? 150 - (int)E : 149;  // f = m * 2^-s
    if (s <= 0) return ~(u128)0;
    const u128 prod = m * x;
    if (s >= 127) return prod ? 1 : 0;
    return (prod + (((u128)1 << s) - 1)) >> s;
}

// smallest j in [1, c] with base + j * w >= target (target <= base + c * w)
uint32_t tie_count(u128 base, uint64_t w, uint32_t c, u128 target) {
    uint32_t lo = 1, hi = c;
    while (lo < hi) {
        const uint32_t mid = lo + (hi - lo) / 2;
        if (base + (u128)mid * w >= target) hi = mid;
        else lo = mid + 1;
    }
    return lo;
}

}  // namespace

extern "C" int32_t orc_sample_exact(const uint16_t* logits, int vocab, int kind, float temperature, float p, int k,
                                    float u) {
    std::vector<uint32_t> hist(65536, 0);
    uint32_t kmax = 0;
    for (int i = 0; i < vocab; ++i) {
        const uint32_t key = bf16_key(logits[i]);
        hist[key]++;
        kmax = std::max(kmax, key);
    }
    const float vmax = scaled(kmax, temperature);
    u128 total = 0;
    for (int key = (int)kmax; key >= 0; --key)
        if (hist[key]) total += (u128)hist[key] * key_weight((uint32_t)key, vmax, temperature);
    // the cut: its weight
    u128 wcut = total;
    if (kind == ORC_SAMPLE_TOP_K) {
        const uint32_t keff = (uint32_t)std::min(std::max(k, 1), vocab);
        u128 cum = 0;
        uint32_t n = 0;
        for (int key = (int)kmax; key >= 0; --key) {
            const uint32_t c = hist[key];
            if (!c) continue;
            const uint64_t w = key_weight((uint32_t)key, vmax, temperature);
            if (n + c >= keff) {
                wcut = cum + (u128)(keff - n) * w;
                break;
            }
            n += c;
            cum += (u128)c * w;
        }
    } else {
        const u128 target = std::max(ceil_mul(p, total), (u128)1);
        u128 cum = 0;
        for (int key = (int)kmax; key >= 0; --key) {
            const uint32_t c = hist[key];
            if (!c) continue;
            const uint64_t w = key_weight((uint32_t)key, vmax, temperature);
            if (cum + (u128)c * w >= target) {
                wcut = cum + (u128)tie_count(cum, w, c, target) * w;
                break;
            }
            cum += (u128)c * w;
        }
    }
    // the pick: a logit value and the rank of the token among its ids
    const u128 r = std::max(ceil_mul(u, wcut), (u128)1);
    u128 cum = 0;
    uint32_t pick_key = kmax, pick_rank = 1;
    for (int key = (int)kmax; key >= 0; --key) {
        const uint32_t c = hist[key];
        if (!c) continue;
        const uint64_t w = key_weight((uint32_t)key, vmax, temperature);
        if (cum + (u128)c * w >= r) {
            pick_key = (uint32_t)key;
            pick_rank = tie_count(cum, w, c, r);
            break;
        }
        cum += (u128)c * w;
    }
    for (int i = 0; i < vocab; ++i)
        if (bf16_key(logits[i]) == pick_key && --pick_rank == 0) return i;
    return -1;  // unreachable: the picked value's count is >= its rank
}

// u[i] = the i-th draw of std::uniform_real_distribution<float>(0, 1) from
// std::mt19937_64(seed): the sequence a seeded TopP sees on one thread (its
// engine is thread_local, top_p.cpp:84); a seeded TopK builds a fresh engine
// per call (top_p.cpp:124), so every one of its calls sees u[0].
extern "C" void orc_sample_draws(uint64_t seed, int n, float* u) {
    std::mt19937_64 rng(seed);
    std::uniform_real_distribution<float> dist(0.0f, 1.0f);
    for (int i = 0; i < n; ++i) u[i] = dist(rng);
}

// ============================================================ model
namespace {

struct Lora {
    int rank = 0;
    float alpha = 0;
    int mask = 0;
    std::map<std::string, std::vector<uint16_t>> w;  // "layers.{i}.self_attn.q_proj.lora_A"
    float scale() const { return alpha / (float)rank; }
};

const char* kProj[7] = {"self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj",
                        "mlp.gate_proj",    "mlp.up_proj",      "mlp.down_proj"};

}  // namespace

struct orc_model {
    orc_model_desc d;
    int layers_used;
    std::map<std::string, std::vector<uint16_t>> w;   // bf16 tensors by checkpoint name
    std::map<std::string, std::vector<uint8_t>> wq;   // GGUF blocks of the linear weights
    std::map<int, Lora> adapters;
    std::vector<float> freqs;
};

struct orc_seq {
    orc_model* m;
    int max_seq;
    int len = 0;
    std::vector<std::vector<uint16_t>> k, v;  // per layer [max_seq, n_kv, hd]
    std::vector<uint16_t> last_hidden;
};

static size_t proj_out(const orc_model_desc& d, int p) {
    switch (p) {
        case 0: return (size_t)d.n_heads * d.head_dim;
        case 1: case 2: return (size_t)d.n_kv_heads * d.head_dim;
        case 3: return (size_t)d.hidden;
        case 4: case 5: return (size_t)d.intermediate;
        default: return (size_t)d.hidden;
    }
}
static size_t proj_in(const orc_model_desc& d, int p) {
    switch (p) {
        case 3: return (size_t)d.n_heads * d.head_dim;
        case 6: return (size_t)d.intermediate;
        default: return (size_t)d.hidden;
    }
}

static std::vector<std::pair<std::string, size_t>> tensor_list(const orc_model_desc& d, int layers) {
    std::vector<std::pair<std::string, size_t>> t;
    t.push_back({"model.embed_tokens.weight", (size_t)d.vocab * d.hidden});
    t.push_back({"model.norm.weight", (size_t)d.hidden});
    t.push_back({"lm_head.weight", (size_t)d.vocab * d.hidden});
    for (int i = 0; i < layers; ++i) {
        std::string p = "model.layers." + std::to_string(i) + ".";
        t.push_back({p + "input_layernorm.weight", (size_t)d.hidden});
        t.push_back({p + "post_attention_layernorm.weight", (size_t)d.hidden});
        for (int j = 0; j < 7; ++j) t.push_back({p + kProj[j] + ".weight", proj_out(d, j) * proj_in(d, j)});
        if (d.qkv_bias)
            for (int j = 0; j < 3; ++j) t.push_back({p + kProj[j] + ".bias", proj_out(d, j)});
    }
    return t;
}

extern "C" orc_model* orc_model_create(const orc_model_desc* d) {
    if (!d || d->hidden <= 0 || d->n_heads <= 0 || d->n_kv_heads <= 0 || d->n_heads % d->n_kv_heads) return nullptr;
    auto* m = new orc_model();
    m->d = *d;
    m->layers_used = d->n_layers;
    m->freqs.resize(d->head_dim / 2);
    orc_rope_freqs(d->head_dim, d->rope_theta, &d->rope, m->freqs.data());
    return m;
}
extern "C" void orc_model_destroy(orc_model* m) { delete m; }
extern "C" void orc_model_limit_layers(orc_model* m, int n) { m->layers_used = std::min(n, m->d.n_layers); }

static void quantize_linear(orc_model* m, const std::string& name) {
    if (m->d.weight_format == ORC_W_BF16) return;
    auto& src = m->w[name];
    std::vector<float> f(src.size());
    for (size_t i = 0; i < f.size(); ++i) f[i] = bf(src[i]);
    const size_t bs = m->d.weight_format == ORC_W_Q4_0 ? 18 : 34;
    std::vector<uint8_t> q(src.size() / 32 * bs);
    const size_t nb = src.size() / 32;
    parallel_for(nb, [&](size_t b0, size_t b1) {
        if (m->d.weight_format == ORC_W_Q4_0) orc_q4_0_quantize(f.data() + b0 * 32, (b1 - b0) * 32, q.data() + b0 * bs);
        else orc_q8_0_quantize(f.data() + b0 * 32, (b1 - b0) * 32, q.data() + b0 * bs);
    }, 1024);
    m->wq[name] = std::move(q);
}

static bool is_linear(const std::string& name) {
    return name.find("model.layers.") == 0 && name.size() > 7 && name.compare(name.size() - 7, 7, ".weight") == 0 &&
           name.find("layernorm") == std::string::npos;
}

extern "C" void orc_model_init_synthetic(orc_model* m, uint64_t seed, float std_) {
    for (auto& [name, n] : tensor_list(m->d, m->layers_used)) {
        auto& v = m->w[name];
        v.resize(n);
        orc_fill_bf16(v.data(), n, seed, orc_name_hash(name.c_str()), std_);
        if (is_linear(name)) quantize_linear(m, name);
    }
}

extern "C" int orc_model_set_weight(orc_model* m, const char* name, const uint16_t* data, size_t n) {
    auto& v = m->w[name];
    v.assign(data, data + n);
    if (is_linear(name)) quantize_linear(m, name);
    return 0;
}

extern "C" int orc_model_get_weight(orc_model* m, const char* name, uint16_t* out, size_t n) {
    auto it = m->w.find(name);
    if (it == m->w.end() || it->second.size() != n) return 1;
    std::memcpy(out, it->second.data(), n * 2);
    return 0;
}

extern "C" int orc_model_add_adapter(orc_model* m, int slot, int rank, float alpha, int proj_mask, uint64_t seed,
                                     float std_a, float std_b) {
    Lora& L = m->adapters[slot];
    L.rank = rank;
    L.alpha = alpha;
    L.mask = proj_mask;
    L.w.clear();
    if (seed == 0) return 0;
    for (int i = 0; i < m->d.n_layers; ++i)
        for (int p = 0; p < 7; ++p) {
            if (!(proj_mask & (1 << p))) continue;
            std::string base = "layers." + std::to_string(i) + "." + kProj[p];
            std::string a = base + ".lora_A", b = base + ".lora_B";
            auto& va = L.w[a];
            va.resize((size_t)rank * proj_in(m->d, p));
            orc_fill_bf16(va.data(), va.size(), seed, orc_name_hash(a.c_str()), std_a);
            auto& vb = L.w[b];
            vb.resize(proj_out(m->d, p) * (size_t)rank);
            orc_fill_bf16(vb.data(), vb.size(), seed, orc_name_hash(b.c_str()), std_b);
        }
    return 0;
}

extern "C" int orc_model_set_lora(orc_model* m, int slot, const char* name, const uint16_t* data, size_t n) {
    auto it = m->adapters.find(slot);
    if (it == m->adapters.end()) return 1;
    it->second.w[name].assign(data, data + n);
    return 0;
}

extern "C" orc_seq* orc_seq_create(orc_model* m, int max_seq) {
    auto* s = new orc_seq();
    s->m = m;
    s->max_seq = max_seq;
    size_t per = (size_t)max_seq * m->d.n_kv_heads * m->d.head_dim;
    s->k.assign(m->d.n_layers, std::vector<uint16_t>(per, 0));
    s->v.assign(m->d.n_layers, std::vector<uint16_t>(per, 0));
    return s;
}
extern "C" void orc_seq_destroy(orc_seq* s) { delete s; }
extern "C" int orc_seq_len(const orc_seq* s) { return s->len; }

// A context of `len` cached tokens with seeded N(0, std) K/V rows in every
// layer (no prefill), for timing decode steps at a given context length.
extern "C" int orc_seq_fill_synthetic(orc_seq* s, int len, uint64_t seed, float std_) {
    if (len < 0 || len > s->max_seq) return 1;
    const size_t n = (size_t)len * s->m->d.n_kv_heads * s->m->d.head_dim;
    for (size_t li = 0; li < s->k.size(); ++li) {
        orc_fill_bf16(s->k[li].data(), n, seed, 2 * li + 1, std_);
        orc_fill_bf16(s->v[li].data(), n, seed, 2 * li + 2, std_);
    }
    s->len = len;
    return 0;
}

extern "C" int orc_seq_last_hidden(const orc_seq* s, uint16_t* out, int hidden) {
    if ((int)s->last_hidden.size() != hidden) return 1;
    std::memcpy(out, s->last_hidden.data(), (size_t)hidden * 2);
    return 0;
}

extern "C" int orc_seq_read_kv(const orc_seq* s, int layer, int which, uint16_t* out, int len) {
    if (layer < 0 || layer >= (int)s->k.size() || len > s->max_seq) return 1;
    const auto& src = which ? s->v[layer] : s->k[layer];
    size_t n = (size_t)len * s->m->d.n_kv_heads * s->m->d.head_dim;
    std::memcpy(out, src.data(), n * 2);
    return 0;
}

// y = x @ W^T for a linear weight (bf16 or GGUF blocks), bf16 output.
static std::vector<uint16_t> linear(orc_model* m, const std::vector<uint16_t>& x, int M, const std::string& name,
                                    size_t N, size_t K) {
    std::vector<uint16_t> y(M * N);
    auto q = m->wq.find(name);
    if (q != m->wq.end()) orc_matmul_t_q(x.data(), q->second.data(), m->d.weight_format, y.data(), nullptr, M, (int)N, (int)K);
    else orc_matmul_t_bf16(x.data(), m->w.at(name).data(), y.data(), M, (int)N, (int)K);
    return y;
}

// qwen_adapter_model.cpp:22-43 — base + bf16(bf16(bf16(x A^T) B^T) * scale).
static void add_lora(orc_model* m, const Lora* L, int layer, int p, const std::vector<uint16_t>& x, int M,
                     std::vector<uint16_t>& y) {
    if (!L || !(L->mask & (1 << p))) return;
    std::string base = "layers." + std::to_string(layer) + "." + kProj[p];
    auto ia = L->w.find(base + ".lora_A"), ib = L->w.find(base + ".lora_B");
    if (ia == L->w.end() || ib == L->w.end()) return;
    const int r = L->rank;
    const size_t K = proj_in(m->d, p), N = proj_out(m->d, p);
    std::vector<uint16_t> down((size_t)M * r), up((size_t)M * N), delta((size_t)M * N);
    orc_matmul_t_bf16(x.data(), ia->second.data(), down.data(), M, r, (int)K);
    orc_matmul_t_bf16(down.data(), ib->second.data(), up.data(), M, (int)N, r);
    orc_mul_scalar(up.data(), L->scale(), delta.data(), up.size());
    orc_add(y.data(), delta.data(), y.data(), y.size());
}

// llama_model.cpp:103-204 (and the Qwen / Qwen-adapter / Gemma / Mistral
// variants): one decoder layer over `M` new tokens at positions [off, off+M).
static std::vector<uint16_t> layer_forward(orc_model* m, orc_seq* s, int li, const std::vector<uint16_t>& hidden,
                                           int M, int off, const Lora* L) {
    const auto& d = m->d;
    const int H = d.hidden, nq = d.n_heads, nkv = d.n_kv_heads, hd = d.head_dim;
    const bool gemma = d.arch == ORC_ARCH_GEMMA;
    const std::string p = "model.layers." + std::to_string(li) + ".";
    std::vector<uint16_t> normed((size_t)M * H);
    orc_rms_norm(hidden.data(), m->w.at(p + "input_layernorm.weight").data(), normed.data(), M, H, d.rms_eps, gemma);

    std::vector<uint16_t> qkv[3];
    for (int j = 0; j < 3; ++j) {
        qkv[j] = linear(m, normed, M, p + kProj[j] + ".weight", proj_out(d, j), H);
        if (d.qkv_bias) {
            const auto& b = m->w.at(p + kProj[j] + ".bias");
            orc_add_bias(qkv[j].data(), b.data(), qkv[j].data(), M, (int)proj_out(d, j));
        }
        add_lora(m, L, li, j, normed, M, qkv[j]);
    }
    std::vector<uint16_t> qr(qkv[0].size()), kr(qkv[1].size());
    orc_rope(qkv[0].data(), qr.data(), M, nq, hd, off, m->freqs.data());
    orc_rope(qkv[1].data(), kr.data(), M, nkv, hd, off, m->freqs.data());

    const size_t row = (size_t)nkv * hd;
    std::memcpy(s->k[li].data() + (size_t)off * row, kr.data(), kr.size() * 2);
    std::memcpy(s->v[li].data() + (size_t)off * row, qkv[2].data(), qkv[2].size() * 2);
    const int kv_len = off + M;
    std::vector<uint16_t> attn((size_t)M * nq * hd);
    const int window = d.arch == ORC_ARCH_MISTRAL ? d.sliding_window : -1;
    orc_attention(qr.data(), s->k[li].data(), s->v[li].data(), attn.data(), M, nq, kv_len, nkv, hd, M > 1, window);

    std::vector<uint16_t> o = linear(m, attn, M, p + "self_attn.o_proj.weight", H, (size_t)nq * hd);
    add_lora(m, L, li, 3, attn, M, o);
    std::vector<uint16_t> res1((size_t)M * H);
    orc_add(hidden.data(), o.data(), res1.data(), res1.size());

    std::vector<uint16_t> normed2((size_t)M * H);
    orc_rms_norm(res1.data(), m->w.at(p + "post_attention_layernorm.weight").data(), normed2.data(), M, H, d.rms_eps,
                 gemma);
    std::vector<uint16_t> gate = linear(m, normed2, M, p + "mlp.gate_proj.weight", d.intermediate, H);
    add_lora(m, L, li, 4, normed2, M, gate);
    std::vector<uint16_t> up = linear(m, normed2, M, p + "mlp.up_proj.weight", d.intermediate, H);
    add_lora(m, L, li, 5, normed2, M, up);
    std::vector<uint16_t> act(gate.size());
    if (gemma) orc_gelu(gate.data(), act.data(), act.size());
    else orc_silu(gate.data(), act.data(), act.size());
    orc_mul(act.data(), up.data(), act.data(), act.size());
    std::vector<uint16_t> down = linear(m, act, M, p + "mlp.down_proj.weight", H, d.intermediate);
    add_lora(m, L, li, 6, act, M, down);
    std::vector<uint16_t> out((size_t)M * H);
    orc_add(res1.data(), down.data(), out.data(), out.size());
    return out;
}

// llama_model.cpp:210-238 — embed, layers, final norm, LM head.
extern "C" int orc_model_forward(orc_model* m, orc_seq* s, const int32_t* ids, int n, int adapter,
                                 uint16_t* logits_bf16, float* logits_f32) {
    if (n <= 0) return 1;
    if (s->len + n > s->max_seq) return 2;
    const auto& d = m->d;
    const int H = d.hidden;
    const Lora* L = nullptr;
    if (adapter >= 0) {
        auto it = m->adapters.find(adapter);
        if (it == m->adapters.end()) return 3;
        L = &it->second;
    }
    for (int i = 0; i < n; ++i)
        if (ids[i] < 0 || ids[i] >= d.vocab) return 4;
    std::vector<uint16_t> hidden((size_t)n * H);
    orc_embedding(m->w.at("model.embed_tokens.weight").data(), d.vocab, H, ids, n, hidden.data());
    if (d.arch == ORC_ARCH_GEMMA)  // gemma_model.cpp:117 — embeddings times sqrt(hidden)
        orc_mul_scalar(hidden.data(), std::sqrt((float)H), hidden.data(), hidden.size());
    const int off = s->len;
    for (int li = 0; li < m->layers_used; ++li) hidden = layer_forward(m, s, li, hidden, n, off, L);
    // only the last row's logits are produced (the row Generator samples from)
    std::vector<uint16_t> last(hidden.end() - H, hidden.end()), normed(H);
    orc_rms_norm(last.data(), m->w.at("model.norm.weight").data(), normed.data(), 1, H, d.rms_eps,
                 d.arch == ORC_ARCH_GEMMA);
    s->last_hidden = normed;
    std::vector<float> lf((size_t)d.vocab);
    orc_matmul_t_bf16_f32out(normed.data(), m->w.at("lm_head.weight").data(), lf.data(), 1, d.vocab, H);
    if (logits_f32) std::memcpy(logits_f32, lf.data(), lf.size() * 4);
    if (logits_bf16)
        for (int i = 0; i < d.vocab; ++i) logits_bf16[i] = tobf(lf[i]);
    s->len += n;
    return 0;
}
