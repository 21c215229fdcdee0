"""ctypes wrapper of the CPU oracle (oracle/_build/liboracle.so).

TEST INFRASTRUCTURE: imported only by tests/, __graft_entry__.smoke() and
bench.py's CPU-baseline legs, as the checker.  The product never imports it.
The C sources (oracle.cpp) restate the reference's decode path; see oracle.h
for the file:line map.
"""
import ctypes as C
import os
import subprocess

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(HERE, "_build", "liboracle.so")

ARCH_LLAMA, ARCH_QWEN2, ARCH_GEMMA, ARCH_MISTRAL = 0, 1, 2, 3
W_BF16, W_Q4_0, W_Q8_0 = 0, 1, 2


class RopeScaling(C.Structure):
    _fields_ = [("apply_scaling", C.c_int), ("factor", C.c_float), ("low_freq_factor", C.c_float),
                ("high_freq_factor", C.c_float), ("original_max_pos", C.c_int)]


class ModelDesc(C.Structure):
    _fields_ = [("arch", C.c_int), ("hidden", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
                ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("intermediate", C.c_int), ("vocab", C.c_int),
                ("rms_eps", C.c_float), ("rope_theta", C.c_float), ("rope", RopeScaling), ("qkv_bias", C.c_int),
                ("sliding_window", C.c_int), ("weight_format", C.c_int)]


def build():
    subprocess.run(["make", "-s", "-C", HERE], check=True)
    return LIB_PATH


_lib = None
P = C.c_void_p
I = C.c_int
SZ = C.c_size_t
F = C.c_float
U64 = C.c_uint64

_SIGS = {
    "orc_name_hash": (U64, [C.c_char_p]),
    "orc_fill_bf16": (None, [P, SZ, U64, U64, F]),
    "orc_fill_f32": (None, [P, SZ, U64, U64, F]),
    "orc_fill_ids": (None, [P, SZ, U64, U64, C.c_int32]),
    "orc_f32_to_bf16": (C.c_uint16, [F]),
    "orc_bf16_to_f32": (F, [C.c_uint16]),
    "orc_f32_to_f16": (C.c_uint16, [F]),
    "orc_f16_to_f32": (F, [C.c_uint16]),
    "orc_set_threads": (None, [I]),
    "orc_get_threads": (I, []),
    "orc_embedding": (None, [P, I, I, P, I, P]),
    "orc_matmul_t_bf16": (None, [P, P, P, I, I, I]),
    "orc_matmul_t_bf16_f32out": (None, [P, P, P, I, I, I]),
    "orc_matmul_t_f32": (None, [P, P, P, I, I, I]),
    "orc_rms_norm": (None, [P, P, P, I, I, F, I]),
    "orc_rope_freqs": (None, [I, F, C.POINTER(RopeScaling), P]),
    "orc_rope": (None, [P, P, I, I, I, I, P]),
    "orc_silu": (None, [P, P, SZ]),
    "orc_gelu": (None, [P, P, SZ]),
    "orc_mul": (None, [P, P, P, SZ]),
    "orc_add": (None, [P, P, P, SZ]),
    "orc_mul_scalar": (None, [P, F, P, SZ]),
    "orc_add_bias": (None, [P, P, P, I, I]),
    "orc_softmax_f32": (None, [P, I, I]),
    "orc_attention": (None, [P, P, P, P, I, I, I, I, I, I, I]),
    "orc_q4_0_quantize": (None, [P, SZ, P]),
    "orc_q4_0_dequantize": (None, [P, SZ, P]),
    "orc_q8_0_quantize": (None, [P, SZ, P]),
    "orc_q8_0_dequantize": (None, [P, SZ, P]),
    "orc_matmul_t_q": (None, [P, P, I, P, P, I, I, I]),
    "orc_pkm_dist": (F, [P, P, I]),
    "orc_pkm_assign": (None, [P, P, I, I, P, I, P]),
    "orc_pkm_build_table": (None, [P, I, P, I]),
    "orc_model_create": (P, [C.POINTER(ModelDesc)]),
    "orc_model_destroy": (None, [P]),
    "orc_model_init_synthetic": (None, [P, U64, F]),
    "orc_model_limit_layers": (None, [P, I]),
    "orc_model_set_weight": (I, [P, C.c_char_p, P, SZ]),
    "orc_model_get_weight": (I, [P, C.c_char_p, P, SZ]),
    "orc_model_add_adapter": (I, [P, I, I, F, I, U64, F, F]),
    "orc_model_set_lora": (I, [P, I, C.c_char_p, P, SZ]),
    "orc_seq_create": (P, [P, I]),
    "orc_seq_destroy": (None, [P]),
    "orc_seq_len": (I, [P]),
    "orc_seq_fill_synthetic": (I, [P, I, U64, F]),
    "orc_model_forward": (I, [P, P, P, I, I, P, P]),
    "orc_seq_last_hidden": (I, [P, P, I]),
    "orc_seq_read_kv": (I, [P, I, I, P, I]),
    "orc_argmax_f32": (C.c_int32, [P, I]),
    "orc_sample_top_p": (C.c_int32, [P, I, F, F, F, I]),
    "orc_sample_top_k": (C.c_int32, [P, I, F, I, F, I]),
    "orc_sample_draws": (None, [U64, I, P]),
    "orc_sample_exact": (C.c_int32, [P, I, I, F, F, I, F]),
}


def lib():
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            build()
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def ptr(a):
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"], "array must be contiguous"
    return a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- numpy helpers
def bf16_to_f32(a):
    a = np.ascontiguousarray(a, np.uint16)
    return (a.astype(np.uint32) << 16).view(np.float32)


def f32_to_bf16(a):
    """round-to-nearest-even (as __float2bfloat16)"""
    a = np.ascontiguousarray(a, np.float32)
    u = a.view(np.uint32).astype(np.uint64)
    r = (u + 0x7FFF + ((u >> 16) & 1)) >> 16
    nan = np.isnan(a)
    out = r.astype(np.uint16)
    out[nan] = ((a[nan].view(np.uint32) >> 16) | 0x40).astype(np.uint16)
    return out


def name_hash(name):
    return lib().orc_name_hash(name.encode())


def fill_bf16(name, shape, seed, std=0.02):
    out = np.empty(shape, np.uint16)
    lib().orc_fill_bf16(ptr(out), out.size, seed, name_hash(name), std)
    return out


def fill_f32(name, shape, seed, std=1.0):
    out = np.empty(shape, np.float32)
    lib().orc_fill_f32(ptr(out), out.size, seed, name_hash(name), std)
    return out


def fill_ids(name, n, seed, vocab):
    out = np.empty(n, np.int32)
    lib().orc_fill_ids(ptr(out), n, seed, name_hash(name), vocab)
    return out


def model_desc(**kw):
    d = ModelDesc()
    d.arch = kw.get("arch", ARCH_LLAMA)
    d.hidden = kw["hidden"]
    d.n_layers = kw["n_layers"]
    d.n_heads = kw["n_heads"]
    d.n_kv_heads = kw.get("n_kv_heads", kw["n_heads"])
    d.head_dim = kw.get("head_dim", kw["hidden"] // kw["n_heads"])
    d.intermediate = kw["intermediate"]
    d.vocab = kw["vocab"]
    d.rms_eps = kw.get("rms_eps", 1e-5)
    d.rope_theta = kw.get("rope_theta", 10000.0)
    rs = kw.get("rope_scaling")
    d.rope.apply_scaling = 1 if rs else 0
    d.rope.factor = rs.get("factor", 1.0) if rs else 1.0
    d.rope.low_freq_factor = rs.get("low_freq_factor", 1.0) if rs else 1.0
    d.rope.high_freq_factor = rs.get("high_freq_factor", 4.0) if rs else 1.0
    d.rope.original_max_pos = rs.get("original_max_pos", 8192) if rs else 8192
    d.qkv_bias = kw.get("qkv_bias", 0)
    d.sliding_window = kw.get("sliding_window", -1)
    d.weight_format = kw.get("weight_format", W_BF16)
    return d


class Model:
    """CPU restatement of Model::forward over a per-sequence contiguous KV cache."""

    def __init__(self, **kw):
        self.kw = kw
        self.desc = model_desc(**kw)
        self.h = lib().orc_model_create(C.byref(self.desc))
        if not self.h:
            raise ValueError("oracle: invalid model description")

    def __del__(self):
        try:
            if self.h:
                lib().orc_model_destroy(self.h)
        except Exception:
            pass

    def init_synthetic(self, seed, std=0.02):
        lib().orc_model_init_synthetic(self.h, seed, std)

    def limit_layers(self, n):
        lib().orc_model_limit_layers(self.h, n)

    def set_weight(self, name, arr):
        arr = np.ascontiguousarray(arr, np.uint16)
        assert lib().orc_model_set_weight(self.h, name.encode(), ptr(arr), arr.size) == 0

    def get_weight(self, name, shape):
        out = np.empty(shape, np.uint16)
        assert lib().orc_model_get_weight(self.h, name.encode(), ptr(out), out.size) == 0
        return out

    def add_adapter(self, slot, rank, alpha, proj_mask, seed=0, std_a=0.02, std_b=0.001):
        assert lib().orc_model_add_adapter(self.h, slot, rank, alpha, proj_mask, seed, std_a, std_b) == 0

    def new_seq(self, max_seq):
        return Seq(self, max_seq)


class Seq:
    def __init__(self, model, max_seq):
        self.m = model
        self.h = lib().orc_seq_create(model.h, max_seq)

    def __del__(self):
        try:
            lib().orc_seq_destroy(self.h)
        except Exception:
            pass

    def __len__(self):
        return lib().orc_seq_len(self.h)

    def forward(self, ids, adapter=-1):
        """returns (bf16 logits of the last row as uint16, fp32 logits)"""
        ids = np.ascontiguousarray(ids, np.int32)
        V = self.m.desc.vocab
        lb = np.empty(V, np.uint16)
        lf = np.empty(V, np.float32)
        rc = lib().orc_model_forward(self.m.h, self.h, ptr(ids), len(ids), adapter, ptr(lb), ptr(lf))
        if rc != 0:
            raise ValueError(f"oracle forward failed ({rc})")
        return lb, lf

    def fill_synthetic(self, length, seed=0, std=1.0):
        """`length` cached tokens with seeded K/V rows in every layer (no prefill)"""
        assert lib().orc_seq_fill_synthetic(self.h, length, seed, std) == 0

    def read_kv(self, layer, which, length):
        d = self.m.desc
        out = np.empty((length, d.n_kv_heads, d.head_dim), np.uint16)
        assert lib().orc_seq_read_kv(self.h, layer, which, ptr(out), length) == 0
        return out


def argmax(x):
    x = np.ascontiguousarray(x, np.float32)
    return int(lib().orc_argmax_f32(ptr(x), x.size))


def sample_top_p(logits, temperature, p, u, stable=False):
    x = np.ascontiguousarray(logits, np.float32)
    return int(lib().orc_sample_top_p(ptr(x), x.size, temperature, p, u, int(stable)))


def sample_top_k(logits, temperature, k, u, stable=False):
    x = np.ascontiguousarray(logits, np.float32)
    return int(lib().orc_sample_top_k(ptr(x), x.size, temperature, k, u, int(stable)))


def sample_draws(seed, n):
    u = np.empty(n, np.float32)
    lib().orc_sample_draws(seed, n, ptr(u))
    return u


SAMPLE_TOP_P, SAMPLE_TOP_K = 1, 2


def sample_exact(logits_bf16, kind, temperature, p=1.0, k=1, u=0.0):
    x = np.ascontiguousarray(logits_bf16, np.uint16)
    return int(lib().orc_sample_exact(ptr(x), x.size, kind, temperature, p, k, u))
