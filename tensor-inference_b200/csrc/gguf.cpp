// gguf.cpp — GGUF model files: container reader and the engine loader.
//
// The reference plans GGUF as the second format behind parser::WeightMap
// (include/tensor/parser/weight_map.hpp:24, "GGUF support comes next"; its
// README names Q4_0 GGUF weights for the decode GEMV).  This file reads the
// published GGUF v2/v3 container (little-endian):
//   "GGUF" u32 version u64 n_tensors u64 n_kv
//   n_kv x { string key, u32 type, value }        (arrays: u32 elem type, u64 n, elems)
//   n_tensors x { string name, u32 n_dims, u64 ne[n_dims], u32 ggml_type, u64 offset }
//   padding to general.alignment (default 32), then the tensor data
// (string = u64 length + bytes; ne[0] is the innermost, contiguous dimension,
// so a [out, in] weight has ne = {in, out} and the same row-major bytes).
//
// Loading maps llama.cpp's tensor names to the reference's
// ("blk.{i}.attn_q.weight" -> "model.layers.{i}.self_attn.q_proj.weight", the
// names LlamaModel::load / QwenModel::load read, llama_model.cpp:47-72) and
// undoes two conventions of llama.cpp's checkpoint converter:
//   * llama-architecture files store the q and k rows of each head permuted
//     for llama.cpp's interleaved-pair RoPE: HF row (t * hd/2 + j) of a head is
//     stored at row (2 j + t).  The reference (and this engine) rotate the pair
//     (j, j + hd/2) (ops.cu:224-232), so the rows are put back.
//   * gemma files store RMSNorm weights as (1 + w); this engine applies the
//     reference's (1 + w) itself (rms_norm_offset), so 1 is subtracted.
// Per-dimension RoPE factors (rope_freqs.weight) divide the base frequencies
// theta^(-2i/d) and replace the engine's RoPE table.
// Tensors of the engine's block type (Q4_0 / Q8_0 linear weights of a
// quantised engine) pass through as blocks; every other tensor is converted to
// bf16 on the host (f32, f16, bf16, and Q4_0 / Q8_0 dequantised to d * q).
#include <fcntl.h>
#include <sys/mman.h>
#include <sys/stat.h>
#include <unistd.h>

#include <cmath>
#include <cstring>
#include <map>
#include <string>
#include <vector>

#include "internal.h"

struct ti_gguf {
    int fd = -1;
    const uint8_t* base = nullptr;
    size_t size = 0;
    uint32_t version = 0;
    struct Meta {
        uint32_t type = 0;   // GGUF value type
        int64_t i = 0;       // integer / bool values
        double f = 0.0;      // float values
        std::string s;       // string values
        uint32_t elem = 0;   // array element type
        uint64_t n = 0;      // array length
        const uint8_t* data = nullptr;  // array elements in the mapping
        std::vector<uint64_t> str_at;   // string arrays: offset of element k's length field from `data`
    };
    std::map<std::string, Meta> meta;
    struct Tensor {
        std::string name;
        int type = 0;
        int n_dims = 0;
        int64_t ne[4] = {1, 1, 1, 1};
        uint64_t offset = 0;
        const uint8_t* data = nullptr;
        size_t bytes = 0;
    };
    std::vector<Tensor> tensors;
    std::map<std::string, int> by_name;
    std::string arch;
};

namespace ti {
// engine side (engine.cu): the destination of a reference-named tensor
ti_status engine_slot_info(ti_engine* e, const char* name, int* wfmt, size_t* rows, size_t* cols);
}

namespace {

using ti::fail;

enum : uint32_t {
    kU8 = 0, kI8 = 1, kU16 = 2, kI16 = 3, kU32 = 4, kI32 = 5, kF32 = 6, kBool = 7, kStr = 8, kArr = 9,
    kU64 = 10, kI64 = 11, kF64 = 12
};

size_t scalar_size(uint32_t t) {
    switch (t) {
        case kU8: case kI8: case kBool: return 1;
        case kU16: case kI16: return 2;
        case kU32: case kI32: case kF32: return 4;
        case kU64: case kI64: case kF64: return 8;
        default: return 0;
    }
}

// bytes of n elements of a ggml type; 0 = unsupported
size_t type_bytes(int type, int64_t n) {
    switch (type) {
        case TI_GGML_F32: return (size_t)n * 4;
        case TI_GGML_F16: case TI_GGML_BF16: return (size_t)n * 2;
        case TI_GGML_Q4_0: return n % 32 ? 0 : (size_t)n / 32 * 18;
        case TI_GGML_Q8_0: return n % 32 ? 0 : (size_t)n / 32 * 34;
        case TI_GGML_Q4_1: return n % 32 ? 0 : (size_t)n / 32 * 20;
        case TI_GGML_Q5_0: return n % 32 ? 0 : (size_t)n / 32 * 22;
        case TI_GGML_Q5_1: return n % 32 ? 0 : (size_t)n / 32 * 24;
        case TI_GGML_Q2_K: return n % 256 ? 0 : (size_t)n / 256 * 84;
        case TI_GGML_Q3_K: return n % 256 ? 0 : (size_t)n / 256 * 110;
        case TI_GGML_Q4_K: return n % 256 ? 0 : (size_t)n / 256 * 144;
        case TI_GGML_Q5_K: return n % 256 ? 0 : (size_t)n / 256 * 176;
        case TI_GGML_Q6_K: return n % 256 ? 0 : (size_t)n / 256 * 210;
        default: return 0;
    }
}

struct Reader {
    const uint8_t* p;
    const uint8_t* end;
    bool ok = true;
    template <class T>
    T get() {
        T v{};
        if ((size_t)(end - p) < sizeof(T)) {
            ok = false;
            return v;
        }
        std::memcpy(&v, p, sizeof(T));
        p += sizeof(T);
        return v;
    }
    std::string str() {
        const uint64_t n = get<uint64_t>();
        if (!ok || (uint64_t)(end - p) < n) {
            ok = false;
            return {};
        }
        std::string s(reinterpret_cast<const char*>(p), (size_t)n);
        p += n;
        return s;
    }
    void skip(uint64_t n) {
        if ((uint64_t)(end - p) < n) {
            ok = false;
            return;
        }
        p += n;
    }
};

// IEEE binary16 -> binary32
float half_to_float(uint16_t h) {
    const uint32_t sign = (uint32_t)(h & 0x8000u) << 16;
    const uint32_t exp = (h >> 10) & 0x1f, man = h & 0x3ffu;
    uint32_t bits;
    if (exp == 0) {
        if (man == 0) {
            bits = sign;
        } else {  // subnormal: normalise
            int e = -1;
            uint32_t m = man;
            do {
                ++e;
                m <<= 1;
            } while ((m & 0x400u) == 0);
            bits = sign | ((uint32_t)(127 - 15 - e) << 23) | ((m & 0x3ffu) << 13);
        }
    } else if (exp == 31) {
        bits = sign | 0x7f800000u | (man << 13);
    } else {
        bits = sign | ((exp + 127 - 15) << 23) | (man << 13);
    }
    float f;
    std::memcpy(&f, &bits, 4);
    return f;
}

// binary32 -> bf16, round to nearest even (NaN kept quiet)
uint16_t float_to_bf16(float f) {
    uint32_t u;
    std::memcpy(&u, &f, 4);
    if ((u & 0x7fffffffu) > 0x7f800000u) return (uint16_t)((u >> 16) | 0x40u);
    u += 0x7fffu + ((u >> 16) & 1u);
    return (uint16_t)(u >> 16);
}

inline float half_at(const uint8_t* p) {
    uint16_t h;
    std::memcpy(&h, p, 2);
    return half_to_float(h);
}

// 6-bit scale (and min) j of a Q4_K / Q5_K super-block's 12 packed bytes: sub-blocks
// 0-3 keep theirs in the low 6 bits of bytes j and j + 4; sub-blocks 4-7 take their
// low 4 bits from the nibbles of byte j + 4 and their top 2 bits from the top bits
// of bytes j - 4 (scale) and j (min)
inline void k4_scale_min(const uint8_t* s, int j, int* sc, int* mn) {
    if (j < 4) {
        *sc = s[j] & 63;
        *mn = s[j + 4] & 63;
    } else {
        *sc = (s[j + 4] & 0x0f) | ((s[j - 4] >> 6) << 4);
        *mn = (s[j + 4] >> 4) | ((s[j] >> 6) << 4);
    }
}

// 6-bit signed scale i (16 per Q3_K super-block, biased by 32): the low 4 bits are
// the nibbles of bytes 0-7 (i < 8: low, else high nibble of byte i - 8), the top 2
// bits come from bytes 8-11 (byte 8 + i % 4, bit pair i / 4)
inline int k3_scale(const uint8_t* s, int i) {
    const int lo = i < 8 ? (s[i] & 0x0f) : (s[i - 8] >> 4);
    const int hi = (s[8 + (i & 3)] >> (2 * (i >> 2))) & 3;
    return (lo | (hi << 4)) - 32;
}

// The block formats of the ggml quantisation types beyond Q4_0 / Q8_0 (GGUF's
// published layouts), decoded element by element: element e of a block, where
// its code bits sit, and the scale (and offset) of its group.
void block_to_float(int type, const uint8_t* b, float* y) {
    switch (type) {
        case TI_GGML_Q4_1: {  // 32: fp16 d, fp16 m, 16 bytes of nibbles; x = d q + m
            const float d = half_at(b), m = half_at(b + 2);
            for (int e = 0; e < 32; ++e) y[e] = d * (float)((b[4 + (e & 15)] >> (4 * (e >> 4))) & 15) + m;
            break;
        }
        case TI_GGML_Q5_0:    // 32: fp16 d, 32 fifth bits (u32), nibbles; x = d (q - 16)
        case TI_GGML_Q5_1: {  // 32: fp16 d, fp16 m, fifth bits, nibbles; x = d q + m
            const bool one = type == TI_GGML_Q5_1;
            const float d = half_at(b), m = one ? half_at(b + 2) : 0.0f;
            const uint8_t* qh = b + (one ? 4 : 2);
            const uint8_t* qs = qh + 4;
            uint32_t hb;
            std::memcpy(&hb, qh, 4);
            for (int e = 0; e < 32; ++e) {
                const int q = ((qs[e & 15] >> (4 * (e >> 4))) & 15) | (int)(((hb >> e) & 1u) << 4);
                y[e] = one ? d * (float)q + m : d * (float)(q - 16);
            }
            break;
        }
        case TI_GGML_Q2_K: {  // 256: 16 scale|min bytes, 64 bytes of 2-bit codes, fp16 d, dmin
            const uint8_t* sc = b;
            const uint8_t* qs = b + 16;
            const float d = half_at(b + 80), dmin = half_at(b + 82);
            for (int e = 0; e < 256; ++e) {
                const int h = e >> 7, r = e & 127, j = r >> 5, second = (r >> 4) & 1, l = r & 15;
                const int q = (qs[32 * h + 16 * second + l] >> (2 * j)) & 3;
                const uint8_t s = sc[8 * h + 2 * j + second];
                y[e] = d * (float)(s & 15) * (float)q - dmin * (float)(s >> 4);
            }
            break;
        }
        case TI_GGML_Q3_K: {  // 256: 32 bytes of high bits, 64 bytes of 2-bit codes, 12 scale bytes, fp16 d
            const uint8_t* hm = b;
            const uint8_t* qs = b + 32;
            const uint8_t* sc = b + 96;
            const float d = half_at(b + 108);
            for (int e = 0; e < 256; ++e) {
                const int h = e >> 7, r = e & 127, j = r >> 5, second = (r >> 4) & 1, l = r & 15;
                const int lo = (qs[32 * h + 16 * second + l] >> (2 * j)) & 3;
                const int high = (hm[16 * second + l] >> (4 * h + j)) & 1;
                y[e] = d * (float)k3_scale(sc, 8 * h + 2 * j + second) * (float)(lo - (high ? 0 : 4));
            }
            break;
        }
        case TI_GGML_Q4_K:    // 256: fp16 d, dmin, 12 scale bytes, 128 bytes of nibbles
        case TI_GGML_Q5_K: {  // 256: fp16 d, dmin, 12 scale bytes, 32 bytes of fifth bits, nibbles
            const bool five = type == TI_GGML_Q5_K;
            const float d = half_at(b), dmin = half_at(b + 2);
            const uint8_t* sc = b + 4;
            const uint8_t* qh = b + 16;
            const uint8_t* qs = b + (five ? 48 : 16);
            for (int e = 0; e < 256; ++e) {
                const int c = e >> 6, r = e & 63, upper = r >> 5, l = r & 31;
                int q = (qs[32 * c + l] >> (4 * upper)) & 15;
                if (five) q |= ((qh[l] >> (2 * c + upper)) & 1) << 4;
                int s = 0, mn = 0;
                k4_scale_min(sc, 2 * c + upper, &s, &mn);
                y[e] = d * (float)s * (float)q - dmin * (float)mn;
            }
            break;
        }
        case TI_GGML_Q6_K: {  // 256: 128 bytes of low nibbles, 64 bytes of high bit pairs, 16 int8 scales, fp16 d
            const uint8_t* ql = b;
            const uint8_t* qh = b + 128;
            const int8_t* sc = reinterpret_cast<const int8_t*>(b + 192);
            const float d = half_at(b + 208);
            for (int e = 0; e < 256; ++e) {
                const int h = e >> 7, r = e & 127, k = r >> 5, l = r & 31;
                const int lo = (ql[64 * h + l + 32 * (k & 1)] >> (4 * (k >> 1))) & 15;
                const int hi = (qh[32 * h + l] >> (2 * k)) & 3;
                y[e] = d * (float)sc[8 * h + (l >> 4) + 2 * k] * (float)((lo | (hi << 4)) - 32);
            }
            break;
        }
        default: break;
    }
}

// one row of n elements of a ggml type -> float
void row_to_float(int type, const uint8_t* src, int64_t n, float* out) {
    switch (type) {
        case TI_GGML_F32: std::memcpy(out, src, (size_t)n * 4); break;
        case TI_GGML_F16:
            for (int64_t i = 0; i < n; ++i) {
                uint16_t h;
                std::memcpy(&h, src + 2 * i, 2);
                out[i] = half_to_float(h);
            }
            break;
        case TI_GGML_BF16:
            for (int64_t i = 0; i < n; ++i) {
                uint16_t h;
                std::memcpy(&h, src + 2 * i, 2);
                const uint32_t u = (uint32_t)h << 16;
                std::memcpy(&out[i], &u, 4);
            }
            break;
        case TI_GGML_Q4_0:  // block: fp16 d, 16 bytes; element j = low nibble of byte j, j + 16 = high nibble
            for (int64_t b = 0; b < n / 32; ++b) {
                const uint8_t* blk = src + b * 18;
                uint16_t dh;
                std::memcpy(&dh, blk, 2);
                const float d = half_to_float(dh);
                for (int j = 0; j < 16; ++j) {
                    out[b * 32 + j] = d * (float)((int)(blk[2 + j] & 0x0f) - 8);
                    out[b * 32 + j + 16] = d * (float)((int)(blk[2 + j] >> 4) - 8);
                }
            }
            break;
        case TI_GGML_Q8_0:  // block: fp16 d, 32 int8
            for (int64_t b = 0; b < n / 32; ++b) {
                const uint8_t* blk = src + b * 34;
                uint16_t dh;
                std::memcpy(&dh, blk, 2);
                const float d = half_to_float(dh);
                for (int j = 0; j < 32; ++j) out[b * 32 + j] = d * (float)(int8_t)blk[2 + j];
            }
            break;
        default: {
            const int64_t per = type_bytes(type, 256) == 0 ? 0 : (type_bytes(type, 32) ? 32 : 256);
            if (!per) break;
            const size_t bb = type_bytes(type, per);
            for (int64_t b = 0; b < n / per; ++b) block_to_float(type, src + b * bb, out + b * per);
            break;
        }
    }
}

// llama.cpp name -> reference name ("" = not a model tensor this engine holds)
std::string reference_name(const std::string& g) {
    static const std::map<std::string, std::string> top = {
        {"token_embd.weight", "model.embed_tokens.weight"},
        {"output_norm.weight", "model.norm.weight"},
        {"output.weight", "lm_head.weight"},
    };
    auto t = top.find(g);
    if (t != top.end()) return t->second;
    if (g.rfind("blk.", 0) != 0) return "";
    const size_t dot = g.find('.', 4);
    if (dot == std::string::npos) return "";
    const std::string layer = g.substr(4, dot - 4);
    if (layer.empty() || layer.find_first_not_of("0123456789") != std::string::npos) return "";
    static const std::map<std::string, std::string> per = {
        {"attn_norm.weight", "input_layernorm.weight"},
        {"ffn_norm.weight", "post_attention_layernorm.weight"},
        {"attn_q.weight", "self_attn.q_proj.weight"},
        {"attn_k.weight", "self_attn.k_proj.weight"},
        {"attn_v.weight", "self_attn.v_proj.weight"},
        {"attn_output.weight", "self_attn.o_proj.weight"},
        {"attn_q.bias", "self_attn.q_proj.bias"},
        {"attn_k.bias", "self_attn.k_proj.bias"},
        {"attn_v.bias", "self_attn.v_proj.bias"},
        {"ffn_gate.weight", "mlp.gate_proj.weight"},
        {"ffn_up.weight", "mlp.up_proj.weight"},
        {"ffn_down.weight", "mlp.down_proj.weight"},
    };
    auto p = per.find(g.substr(dot + 1));
    if (p == per.end()) return "";
    return "model.layers." + layer + "." + p->second;
}

const ti_gguf::Meta* find_meta(const ti_gguf* g, const std::string& key) {
    auto it = g->meta.find(key);
    return it == g->meta.end() ? nullptr : &it->second;
}

bool meta_int(const ti_gguf* g, const std::string& key, int64_t* v) {
    const ti_gguf::Meta* m = find_meta(g, key);
    if (!m || m->type == kStr || m->type == kArr || m->type == kF32 || m->type == kF64) return false;
    *v = m->i;
    return true;
}

bool meta_float(const ti_gguf* g, const std::string& key, double* v) {
    const ti_gguf::Meta* m = find_meta(g, key);
    if (!m) return false;
    if (m->type == kF32 || m->type == kF64) {
        *v = m->f;
        return true;
    }
    if (m->type == kStr || m->type == kArr) return false;
    *v = (double)m->i;
    return true;
}

// head count of the q or k tensor for the row un-permutation (0 = none); the
// metadata value unchecked (the caller rejects counts that do not divide the rows)
int64_t permute_heads(const ti_gguf* g, const std::string& gname) {
    if (g->arch != "llama") return 0;
    const bool q = gname.size() > 14 && gname.compare(gname.size() - 14, 14, ".attn_q.weight") == 0;
    const bool k = gname.size() > 14 && gname.compare(gname.size() - 14, 14, ".attn_k.weight") == 0;
    if (!q && !k) return 0;
    int64_t nh = 0, nkv = 0;
    if (!meta_int(g, "llama.attention.head_count", &nh)) return 0;
    if (!meta_int(g, "llama.attention.head_count_kv", &nkv)) nkv = nh;
    return q ? nh : nkv;
}

// source row of reference row r: heads of hd rows, HF row t * hd/2 + j of a head
// was stored at row 2 j + t
int64_t source_row(int64_t r, int64_t hd) {
    const int64_t h = r / hd, w = r % hd, half = hd / 2;
    const int64_t t = w / half, j = w % half;
    return h * hd + 2 * j + t;
}

}  // namespace

extern "C" {

ti_status ti_gguf_open(const char* path, ti_gguf** out) {
    ti::clear_error();
    TI_CHECK(path && out, TI_ERR_INVALID, "ti_gguf_open: null argument");
    *out = nullptr;
    const int fd = ::open(path, O_RDONLY);
    TI_CHECK(fd >= 0, TI_ERR_NOT_FOUND, "ti_gguf_open: cannot open '%s'", path);
    struct stat st {};
    if (fstat(fd, &st) != 0 || st.st_size < 24) {
        ::close(fd);
        return fail(TI_ERR_INVALID, "ti_gguf_open: '%s' is not a GGUF file (too short)", path);
    }
    void* m = mmap(nullptr, (size_t)st.st_size, PROT_READ, MAP_PRIVATE, fd, 0);
    if (m == MAP_FAILED) {
        ::close(fd);
        return fail(TI_ERR_INVALID, "ti_gguf_open: cannot map '%s'", path);
    }
    ti_gguf* g = new ti_gguf;
    g->fd = fd;
    g->base = reinterpret_cast<const uint8_t*>(m);
    g->size = (size_t)st.st_size;
    auto bad = [&](const char* why) {
        ti_gguf_close(g);
        return fail(TI_ERR_INVALID, "ti_gguf_open: '%s': %s", path, why);
    };
    Reader r{g->base, g->base + g->size};
    if (std::memcmp(g->base, "GGUF", 4) != 0) return bad("bad magic (not GGUF)");
    r.skip(4);
    g->version = r.get<uint32_t>();
    if (g->version < 2 || g->version > 3) return bad("unsupported GGUF version (2 or 3 expected)");
    const uint64_t n_tensors = r.get<uint64_t>(), n_kv = r.get<uint64_t>();
    if (!r.ok || n_tensors > (1u << 24) || n_kv > (1u << 24)) return bad("implausible header counts");
    for (uint64_t i = 0; i < n_kv && r.ok; ++i) {
        std::string key = r.str();
        ti_gguf::Meta v;
        v.type = r.get<uint32_t>();
        if (v.type == kStr) {
            v.s = r.str();
        } else if (v.type == kArr) {
            v.elem = r.get<uint32_t>();
            v.n = r.get<uint64_t>();
            v.data = r.p;
            if (v.elem == kStr) {
                if (v.n > g->size / 8) return bad("metadata array longer than the file");
                v.str_at.reserve((size_t)v.n);
                for (uint64_t k = 0; k < v.n && r.ok; ++k) {
                    v.str_at.push_back((uint64_t)(r.p - v.data));
                    r.skip(r.get<uint64_t>());
                }
            } else if (v.elem == kArr || scalar_size(v.elem) == 0) {
                return bad("unsupported metadata array element type");
            } else {
                if (v.n > g->size) return bad("metadata array longer than the file");
                r.skip(v.n * scalar_size(v.elem));
            }
        } else {
            switch (v.type) {
                case kU8: v.i = r.get<uint8_t>(); break;
                case kI8: v.i = r.get<int8_t>(); break;
                case kU16: v.i = r.get<uint16_t>(); break;
                case kI16: v.i = r.get<int16_t>(); break;
                case kU32: v.i = r.get<uint32_t>(); break;
                case kI32: v.i = r.get<int32_t>(); break;
                case kBool: v.i = r.get<uint8_t>() != 0; break;
                case kU64: v.i = (int64_t)r.get<uint64_t>(); break;
                case kI64: v.i = r.get<int64_t>(); break;
                case kF32: v.f = r.get<float>(); break;
                case kF64: v.f = r.get<double>(); break;
                default: return bad("unknown metadata value type");
            }
        }
        g->meta[key] = v;
    }
    if (!r.ok) return bad("truncated metadata");
    for (uint64_t i = 0; i < n_tensors && r.ok; ++i) {
        ti_gguf::Tensor t;
        t.name = r.str();
        t.n_dims = (int)r.get<uint32_t>();
        if (t.n_dims < 1 || t.n_dims > 4) return bad("tensor with an unsupported number of dimensions");
        for (int d = 0; d < t.n_dims; ++d) t.ne[d] = (int64_t)r.get<uint64_t>();
        t.type = (int)r.get<uint32_t>();
        t.offset = r.get<uint64_t>();
        g->tensors.push_back(t);
    }
    if (!r.ok) return bad("truncated tensor table");
    int64_t align = 32;
    if (const ti_gguf::Meta* a = find_meta(g, "general.alignment")) align = a->i;
    if (align <= 0 || (align & (align - 1)) != 0) return bad("general.alignment is not a power of two");
    const size_t data0 = ((size_t)(r.p - g->base) + (size_t)align - 1) / (size_t)align * (size_t)align;
    if (data0 > g->size) return bad("tensor data section beyond the end of the file");
    const size_t data_bytes = g->size - data0;
    for (size_t i = 0; i < g->tensors.size(); ++i) {
        ti_gguf::Tensor& t = g->tensors[i];
        int64_t n = 1;
        for (int d = 0; d < t.n_dims; ++d) {
            if (t.ne[d] <= 0 || n > (int64_t(1) << 40) / t.ne[d]) return bad("tensor dimensions out of range");
            n *= t.ne[d];
        }
        t.bytes = type_bytes(t.type, n);  // 0 for block types this reader does not decode
        // offsets come from the file: compare without forming data0 + offset (no wrap)
        if (t.bytes && (t.offset > data_bytes || t.bytes > data_bytes - t.offset))
            return bad("tensor data beyond the end of the file");
        t.data = t.bytes ? g->base + data0 + t.offset : nullptr;
        g->by_name[t.name] = (int)i;
    }
    if (const ti_gguf::Meta* a = find_meta(g, "general.architecture")) g->arch = a->s;
    *out = g;
    return TI_OK;
}

ti_status ti_gguf_close(ti_gguf* g) {
    if (!g) return TI_OK;
    if (g->base) munmap(const_cast<uint8_t*>(g->base), g->size);
    if (g->fd >= 0) ::close(g->fd);
    delete g;
    return TI_OK;
}

ti_status ti_gguf_tensor_count(const ti_gguf* g, int* n) {
    ti::clear_error();
    TI_CHECK(g && n, TI_ERR_INVALID, "ti_gguf_tensor_count: null argument");
    *n = (int)g->tensors.size();
    return TI_OK;
}

ti_status ti_gguf_tensor_info(const ti_gguf* g, int i, const char** name, int* ggml_type, int* n_dims, int64_t* dims,
                              const void** data, size_t* bytes) {
    ti::clear_error();
    TI_CHECK(g, TI_ERR_INVALID, "ti_gguf_tensor_info: null handle");
    TI_CHECK(i >= 0 && i < (int)g->tensors.size(), TI_ERR_INVALID, "tensor index %d out of range", i);
    const ti_gguf::Tensor& t = g->tensors[i];
    if (name) *name = t.name.c_str();
    if (ggml_type) *ggml_type = t.type;
    if (n_dims) *n_dims = t.n_dims;
    if (dims)
        for (int d = 0; d < 4; ++d) dims[d] = t.ne[d];
    if (data) *data = t.data;
    if (bytes) *bytes = t.bytes;
    return TI_OK;
}

ti_status ti_gguf_find(const ti_gguf* g, const char* name, int* index) {
    ti::clear_error();
    TI_CHECK(g && name && index, TI_ERR_INVALID, "ti_gguf_find: null argument");
    auto it = g->by_name.find(name);
    TI_CHECK(it != g->by_name.end(), TI_ERR_NOT_FOUND, "no tensor '%s' in the GGUF file", name);
    *index = it->second;
    return TI_OK;
}

ti_status ti_gguf_meta_int(const ti_gguf* g, const char* key, int64_t* v) {
    ti::clear_error();
    TI_CHECK(g && key && v, TI_ERR_INVALID, "ti_gguf_meta_int: null argument");
    TI_CHECK(meta_int(g, key, v), TI_ERR_NOT_FOUND, "no integer metadata '%s'", key);
    return TI_OK;
}

ti_status ti_gguf_meta_float(const ti_gguf* g, const char* key, double* v) {
    ti::clear_error();
    TI_CHECK(g && key && v, TI_ERR_INVALID, "ti_gguf_meta_float: null argument");
    TI_CHECK(meta_float(g, key, v), TI_ERR_NOT_FOUND, "no numeric metadata '%s'", key);
    return TI_OK;
}

ti_status ti_gguf_meta_string(const ti_gguf* g, const char* key, const char** v) {
    ti::clear_error();
    TI_CHECK(g && key && v, TI_ERR_INVALID, "ti_gguf_meta_string: null argument");
    const ti_gguf::Meta* m = find_meta(g, key);
    TI_CHECK(m && m->type == kStr, TI_ERR_NOT_FOUND, "no string metadata '%s'", key);
    *v = m->s.c_str();
    return TI_OK;
}

ti_status ti_gguf_meta_array_len(const ti_gguf* g, const char* key, int64_t* n) {
    ti::clear_error();
    TI_CHECK(g && key && n, TI_ERR_INVALID, "ti_gguf_meta_array_len: null argument");
    const ti_gguf::Meta* m = find_meta(g, key);
    TI_CHECK(m && m->type == kArr, TI_ERR_NOT_FOUND, "no array metadata '%s'", key);
    *n = (int64_t)m->n;
    return TI_OK;
}

// element i of array metadata `key`, whose elements must be of a type `ok` accepts
static ti_status array_elem(const ti_gguf* g, const char* key, int64_t i, const ti_gguf::Meta** out,
                            bool (*ok)(uint32_t)) {
    TI_CHECK(g && key, TI_ERR_INVALID, "gguf array element: null argument");
    const ti_gguf::Meta* m = find_meta(g, key);
    TI_CHECK(m && m->type == kArr, TI_ERR_NOT_FOUND, "no array metadata '%s'", key);
    TI_CHECK(ok(m->elem), TI_ERR_INVALID, "array metadata '%s' holds element type %u", key, m->elem);
    TI_CHECK(i >= 0 && (uint64_t)i < m->n, TI_ERR_INVALID, "array metadata '%s': index %lld of %llu", key,
             (long long)i, (unsigned long long)m->n);
    *out = m;
    return TI_OK;
}

ti_status ti_gguf_meta_array_string(const ti_gguf* g, const char* key, int64_t i, const char** str, size_t* len) {
    ti::clear_error();
    TI_CHECK(str && len, TI_ERR_INVALID, "ti_gguf_meta_array_string: null argument");
    const ti_gguf::Meta* m = nullptr;
    if (ti_status st = array_elem(g, key, i, &m, [](uint32_t t) { return t == (uint32_t)kStr; })) return st;
    const uint8_t* at = m->data + m->str_at[(size_t)i];
    uint64_t n = 0;
    std::memcpy(&n, at, 8);
    *str = reinterpret_cast<const char*>(at + 8);
    *len = (size_t)n;
    return TI_OK;
}

ti_status ti_gguf_meta_array_int(const ti_gguf* g, const char* key, int64_t i, int64_t* v) {
    ti::clear_error();
    TI_CHECK(v, TI_ERR_INVALID, "ti_gguf_meta_array_int: null argument");
    const ti_gguf::Meta* m = nullptr;
    if (ti_status st = array_elem(g, key, i, &m, [](uint32_t t) {
            return t == kU8 || t == kI8 || t == kU16 || t == kI16 || t == kU32 || t == kI32 || t == kU64 ||
                   t == kI64 || t == kBool;
        }))
        return st;
    const uint8_t* at = m->data + (size_t)i * scalar_size(m->elem);
    switch (m->elem) {
        case kU8: *v = *at; break;
        case kI8: *v = (int8_t)*at; break;
        case kBool: *v = *at != 0; break;
        case kU16: { uint16_t x; std::memcpy(&x, at, 2); *v = x; break; }
        case kI16: { int16_t x; std::memcpy(&x, at, 2); *v = x; break; }
        case kU32: { uint32_t x; std::memcpy(&x, at, 4); *v = x; break; }
        case kI32: { int32_t x; std::memcpy(&x, at, 4); *v = x; break; }
        case kU64: { uint64_t x; std::memcpy(&x, at, 8); *v = (int64_t)x; break; }
        default: { int64_t x; std::memcpy(&x, at, 8); *v = x; break; }
    }
    return TI_OK;
}

ti_status ti_gguf_meta_array_float(const ti_gguf* g, const char* key, int64_t i, double* v) {
    ti::clear_error();
    TI_CHECK(v, TI_ERR_INVALID, "ti_gguf_meta_array_float: null argument");
    const ti_gguf::Meta* m = nullptr;
    if (ti_status st = array_elem(g, key, i, &m, [](uint32_t t) { return t == kF32 || t == kF64; })) return st;
    const uint8_t* at = m->data + (size_t)i * scalar_size(m->elem);
    if (m->elem == kF32) {
        float x;
        std::memcpy(&x, at, 4);
        *v = x;
    } else {
        std::memcpy(v, at, 8);
    }
    return TI_OK;
}

ti_status ti_gguf_model_desc(const ti_gguf* g, ti_model_desc* d) {
    ti::clear_error();
    TI_CHECK(g && d, TI_ERR_INVALID, "ti_gguf_model_desc: null argument");
    std::memset(d, 0, sizeof *d);
    const std::string& a = g->arch;
    if (a == "llama") d->arch = TI_ARCH_LLAMA;
    else if (a == "qwen2") d->arch = TI_ARCH_QWEN2;
    else if (a == "gemma") d->arch = TI_ARCH_GEMMA;
    else return fail(TI_ERR_UNSUPPORTED, "GGUF architecture '%s' (llama, qwen2 or gemma supported)", a.c_str());
    int64_t v = 0;
    // an integer of the description: present (or `dflt` when given), within [lo, INT_MAX]
    auto get = [&](const char* k, int* dst, int64_t lo, const int* dflt) -> ti_status {
        if (!meta_int(g, a + "." + k, &v)) {
            TI_CHECK(dflt, TI_ERR_INVALID, "GGUF metadata '%s.%s' missing", a.c_str(), k);
            *dst = *dflt;
            return TI_OK;
        }
        TI_CHECK(v >= lo && v <= 0x7fffffff, TI_ERR_INVALID, "GGUF metadata '%s.%s' = %lld out of range", a.c_str(),
                 k, (long long)v);
        *dst = (int)v;
        return TI_OK;
    };
    if (ti_status st = get("block_count", &d->n_layers, 1, nullptr)) return st;
    if (ti_status st = get("embedding_length", &d->hidden, 1, nullptr)) return st;
    if (ti_status st = get("feed_forward_length", &d->intermediate, 1, nullptr)) return st;
    if (ti_status st = get("attention.head_count", &d->n_heads, 1, nullptr)) return st;
    if (ti_status st = get("attention.head_count_kv", &d->n_kv_heads, 1, &d->n_heads)) return st;
    const int hd_default = d->hidden / d->n_heads;
    if (ti_status st = get("attention.key_length", &d->head_dim, 1, &hd_default)) return st;
    double f = 0;
    d->rms_eps = meta_float(g, a + ".attention.layer_norm_rms_epsilon", &f) ? (float)f : 1e-6f;
    d->rope_theta = meta_float(g, a + ".rope.freq_base", &f) ? (float)f : 10000.0f;
    const int no_window = 0;
    if (ti_status st = get("attention.sliding_window", &d->sliding_window, 0, &no_window)) return st;
    auto emb = g->by_name.find("token_embd.weight");
    TI_CHECK(emb != g->by_name.end(), TI_ERR_INVALID, "GGUF file has no token_embd.weight");
    const int64_t vocab = g->tensors[emb->second].ne[1];
    TI_CHECK(vocab >= 1 && vocab <= 0x7fffffff, TI_ERR_INVALID, "GGUF token_embd.weight: %lld rows",
             (long long)vocab);
    d->vocab = (int)vocab;
    d->qkv_bias = g->by_name.count("blk.0.attn_q.bias") ? 1 : 0;
    d->weight_format = TI_WFMT_BF16;
    auto q = g->by_name.find("blk.0.attn_q.weight");
    if (q != g->by_name.end()) {
        const int t = g->tensors[q->second].type;
        if (t == TI_GGML_Q4_0) d->weight_format = TI_WFMT_Q4_0;
        else if (t == TI_GGML_Q8_0) d->weight_format = TI_WFMT_Q8_0;
    }
    return TI_OK;
}

ti_status ti_gguf_rope_inv_freq(const ti_gguf* g, float* out, int n) {
    ti::clear_error();
    TI_CHECK(g && out && n > 0, TI_ERR_INVALID, "ti_gguf_rope_inv_freq: null argument");
    const std::string& a = g->arch;
    double theta = 10000.0;
    meta_float(g, a + ".rope.freq_base", &theta);
    ti::rope_freqs(2 * n, (float)theta, nullptr, out);
    auto it = g->by_name.find("rope_freqs.weight");
    if (it == g->by_name.end()) return TI_OK;
    // llama.cpp's per-dimension factors: angle = pos * base_i / factor_i
    const ti_gguf::Tensor& t = g->tensors[it->second];
    TI_CHECK(t.bytes > 0 && t.n_dims == 1 && t.ne[0] == n, TI_ERR_INVALID,
             "rope_freqs.weight has %lld values, head_dim / 2 = %d expected", (long long)t.ne[0], n);
    std::vector<float> f((size_t)n);
    row_to_float(t.type, t.data, n, f.data());
    for (int i = 0; i < n; ++i) {
        TI_CHECK(f[i] > 0.f, TI_ERR_INVALID, "rope_freqs.weight[%d] = %g (positive factors expected)", i, f[i]);
        out[i] /= f[i];
    }
    return TI_OK;
}

ti_status ti_gguf_reference_name(const ti_gguf* g, int i, char* buf, size_t cap) {
    ti::clear_error();
    TI_CHECK(g && buf && cap > 0, TI_ERR_INVALID, "ti_gguf_reference_name: null argument");
    TI_CHECK(i >= 0 && i < (int)g->tensors.size(), TI_ERR_INVALID, "tensor index %d out of range", i);
    const std::string r = reference_name(g->tensors[i].name);
    TI_CHECK(!r.empty(), TI_ERR_NOT_FOUND, "GGUF tensor '%s' has no reference counterpart",
             g->tensors[i].name.c_str());
    TI_CHECK(r.size() < cap, TI_ERR_INVALID, "name buffer of %zu bytes too small", cap);
    std::memcpy(buf, r.c_str(), r.size() + 1);
    return TI_OK;
}

ti_status ti_gguf_read(const ti_gguf* g, int i, int dtype, void* out, size_t bytes) {
    ti::clear_error();
    TI_CHECK(g && out, TI_ERR_INVALID, "ti_gguf_read: null argument");
    TI_CHECK(i >= 0 && i < (int)g->tensors.size(), TI_ERR_INVALID, "tensor index %d out of range", i);
    const ti_gguf::Tensor& t = g->tensors[i];
    TI_CHECK(t.bytes > 0, TI_ERR_UNSUPPORTED,
             "GGUF tensor '%s': ggml type %d not supported (f32, f16, bf16, q4_0, q4_1, q5_0, q5_1, q8_0, q2_k .. q6_k)",
             t.name.c_str(), t.type);
    const int64_t cols = t.ne[0], rows = t.n_dims >= 2 ? t.ne[1] * t.ne[2] * t.ne[3] : 1;
    const int64_t heads = permute_heads(g, t.name);
    const int64_t hd = heads > 0 ? rows / heads : 0;
    TI_CHECK(heads == 0 || (heads > 0 && rows % heads == 0 && hd >= 2 && hd % 2 == 0), TI_ERR_INVALID,
             "GGUF tensor '%s': %lld rows do not split into %lld heads of an even size", t.name.c_str(),
             (long long)rows, (long long)heads);
    const size_t src_row = type_bytes(t.type, cols);
    auto src_of = [&](int64_t r) { return t.data + (size_t)(heads ? source_row(r, hd) : r) * src_row; };
    if (dtype == TI_DTYPE_BF16) {
        TI_CHECK(bytes == (size_t)(rows * cols) * 2, TI_ERR_INVALID, "GGUF tensor '%s': %zu bytes, bf16 needs %zu",
                 t.name.c_str(), bytes, (size_t)(rows * cols) * 2);
        const bool norm = g->arch == "gemma" && t.name.size() > 12 &&
                          t.name.compare(t.name.size() - 12, 12, "_norm.weight") == 0;
        std::vector<float> row((size_t)cols);
        uint16_t* o = reinterpret_cast<uint16_t*>(out);
        for (int64_t r = 0; r < rows; ++r) {
            row_to_float(t.type, src_of(r), cols, row.data());
            for (int64_t c = 0; c < cols; ++c) o[r * cols + c] = float_to_bf16(norm ? row[c] - 1.0f : row[c]);
        }
        return TI_OK;
    }
    const int want = dtype == TI_DTYPE_Q4_0 ? TI_GGML_Q4_0 : dtype == TI_DTYPE_Q8_0 ? TI_GGML_Q8_0 : -1;
    TI_CHECK(want >= 0 && want == t.type, TI_ERR_UNSUPPORTED,
             "GGUF tensor '%s' (ggml type %d): blocks are read in their own type only", t.name.c_str(), t.type);
    TI_CHECK(bytes == t.bytes, TI_ERR_INVALID, "GGUF tensor '%s': %zu bytes, expected %zu", t.name.c_str(), bytes,
             t.bytes);
    for (int64_t r = 0; r < rows; ++r) std::memcpy(reinterpret_cast<uint8_t*>(out) + r * src_row, src_of(r), src_row);
    return TI_OK;
}

ti_status ti_engine_load_gguf(ti_engine* e, const ti_gguf* g, int* n_loaded) {
    ti::clear_error();
    TI_CHECK(e && g, TI_ERR_INVALID, "ti_engine_load_gguf: null argument");
    int loaded = 0;
    bool have_lm_head = false;
    std::vector<uint8_t> buf;
    auto load_as = [&](int i, const std::string& ref) -> ti_status {
        int wf = 0;
        size_t rows = 0, cols = 0;
        if (ti_status st = ti::engine_slot_info(e, ref.c_str(), &wf, &rows, &cols)) return st;
        const ti_gguf::Tensor& t = g->tensors[i];
        const int64_t n = t.ne[0] * t.ne[1] * t.ne[2] * t.ne[3];
        TI_CHECK((size_t)n == rows * cols && (size_t)t.ne[0] == cols, TI_ERR_INVALID,
                 "GGUF tensor '%s' has ne = [%lld, %lld], the engine's '%s' is [%zu, %zu]", t.name.c_str(),
                 (long long)t.ne[0], (long long)t.ne[1], ref.c_str(), rows, cols);
        const bool blocks = (wf == TI_WFMT_Q4_0 && t.type == TI_GGML_Q4_0) ||
                            (wf == TI_WFMT_Q8_0 && t.type == TI_GGML_Q8_0);
        const int dtype = !blocks ? TI_DTYPE_BF16 : wf == TI_WFMT_Q4_0 ? TI_DTYPE_Q4_0 : TI_DTYPE_Q8_0;
        const size_t bytes = blocks ? t.bytes : rows * cols * 2;
        buf.resize(bytes);
        if (ti_status st = ti_gguf_read(g, i, dtype, buf.data(), bytes)) return st;
        if (ti_status st = ti_engine_load_tensor(e, ref.c_str(), dtype, buf.data(), bytes)) return st;
        ++loaded;
        return TI_OK;
    };
    for (int i = 0; i < (int)g->tensors.size(); ++i) {
        const std::string ref = reference_name(g->tensors[i].name);
        if (ref.empty()) continue;  // tokenizer / rope tables / tensors the engine does not hold
        if (ref == "lm_head.weight") have_lm_head = true;
        if (ti_status st = load_as(i, ref)) return st;
    }
    if (!have_lm_head) {
        // tied embeddings: the LM head is the embedding table
        auto it = g->by_name.find("token_embd.weight");
        TI_CHECK(it != g->by_name.end(), TI_ERR_INVALID, "GGUF file has neither output.weight nor token_embd.weight");
        if (ti_status st = load_as(it->second, "lm_head.weight")) return st;
    }
    if (g->by_name.count("rope_freqs.weight")) {
        // per-dimension RoPE factors (llama 3.1 style files) replace the engine's table
        const auto it = g->by_name.find("rope_freqs.weight");
        const int n = (int)g->tensors[it->second].ne[0];
        std::vector<float> inv((size_t)n);
        if (ti_status st = ti_gguf_rope_inv_freq(g, inv.data(), n)) return st;
        if (ti_status st = ti_engine_set_rope_freqs(e, inv.data(), n)) return st;
    }
    if (n_loaded) *n_loaded = loaded;
    return TI_OK;
}

}  // extern "C"
