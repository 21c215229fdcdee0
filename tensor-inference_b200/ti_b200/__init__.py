"""Python binding of libti_b200.so (the C ABI declared in include/ti_b200.h).

This is host plumbing for tests and the benchmark: every call goes straight to
the C ABI.  There is no fallback — if the shared library is missing or cannot
be loaded, importing the library raises.

Model presets and the config.json reader mirror the reference's
tensor::parser::ModelConfig accessors and defaults (src/parser/config.cpp:101-182)
and the per-architecture config structs (include/tensor/models/*/..._config.hpp).
"""
import ctypes as C
import os

import numpy as np

_HERE = os.path.dirname(os.path.abspath(__file__))
LIB_PATH = os.path.join(os.path.dirname(_HERE), "libti_b200.so")

TI_OK, TI_ERR_INVALID, TI_ERR_CUDA, TI_ERR_OOM, TI_ERR_UNSUPPORTED, TI_ERR_STATE, TI_ERR_TIMEOUT, TI_ERR_NOT_FOUND = range(8)
DTYPE_F32, DTYPE_BF16, DTYPE_F16, DTYPE_I32 = 0, 1, 2, 3
DTYPE_Q4_0, DTYPE_Q8_0 = 16, 17
ARCH_LLAMA, ARCH_QWEN2, ARCH_GEMMA, ARCH_MISTRAL = 0, 1, 2, 3
WFMT_BF16, WFMT_Q4_0, WFMT_Q8_0 = 0, 1, 2
GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_BF16 = 0, 1, 2, 8, 30
EW_SILU, EW_GELU, EW_MUL, EW_ADD, EW_MUL_SCALAR = range(5)
LOGITS_NONE, LOGITS_BF16, LOGITS_F32 = 0, 1, 2
SAMPLE_GREEDY, SAMPLE_TOP_P, SAMPLE_TOP_K = 0, 1, 2
PROJ_Q, PROJ_K, PROJ_V, PROJ_O, PROJ_GATE, PROJ_UP, PROJ_DOWN = 1, 2, 4, 8, 16, 32, 64
KERNEL_EMBED, KERNEL_QKV, KERNEL_ATTN, KERNEL_O, KERNEL_GATEUP, KERNEL_DOWN, KERNEL_LMHEAD = range(7)


class TiError(RuntimeError):
    def __init__(self, status, msg):
        super().__init__(f"[ti status {status}] {msg}")
        self.status = status


class RopeScaling(C.Structure):
    _fields_ = [("apply_scaling", C.c_int), ("factor", C.c_float), ("low_freq_factor", C.c_float),
                ("high_freq_factor", C.c_float), ("original_max_pos", C.c_int)]


class Sampling(C.Structure):
    """ti_sampling: the reference's Greedy / TopP / TopK options (sampling/top_p.hpp)."""
    _fields_ = [("kind", C.c_int), ("temperature", C.c_float), ("p", C.c_float), ("k", C.c_uint32),
                ("seeded", C.c_int), ("seed", C.c_uint64)]


def sampler_draws(kind, n, seed=None, temperature=1.0, p=0.95, k=40):
    """the first n uniform draws of a sequence sampler (ti_sampler_draws)"""
    smp = Sampling(kind, temperature, p, k, 0 if seed is None else 1, 0 if seed is None else seed)
    out = (C.c_float * n)()
    check(lib().ti_sampler_draws(C.byref(smp), n, out))
    return np.array(out[:], np.float32)


class ModelDesc(C.Structure):
    _fields_ = [("arch", C.c_int), ("hidden", C.c_int), ("n_layers", C.c_int), ("n_heads", C.c_int),
                ("n_kv_heads", C.c_int), ("head_dim", C.c_int), ("intermediate", C.c_int), ("vocab", C.c_int),
                ("rms_eps", C.c_float), ("rope_theta", C.c_float), ("rope", RopeScaling), ("qkv_bias", C.c_int),
                ("sliding_window", C.c_int), ("weight_format", C.c_int)]


class EngineOpts(C.Structure):
    _fields_ = [("device", C.c_int), ("max_batch", C.c_int), ("max_seqs", C.c_int), ("max_seq_len", C.c_int),
                ("kv_pages", C.c_int), ("max_adapters", C.c_int), ("max_lora_rank", C.c_int),
                ("lora_proj_mask", C.c_int), ("tp_size", C.c_int), ("tp_rank", C.c_int), ("nccl_id", C.c_void_p)]


_lib = None

class TpShard(C.Structure):
    _fields_ = [("tp", C.c_int), ("rank", C.c_int), ("nq", C.c_int), ("nkv", C.c_int), ("q0", C.c_int),
                ("kv0", C.c_int), ("inter", C.c_int), ("i0", C.c_int), ("vocab", C.c_int), ("v0", C.c_int)]


_SIGS = {
    "ti_seq_fill_synthetic": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_uint64, C.c_float]),
    "ti_nccl_unique_id": (C.c_int, [C.c_void_p]),
    "ti_tp_plan": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "ti_last_error": (C.c_char_p, []),
    "ti_version": (C.c_int, []),
    "ti_device_count": (C.c_int, [C.POINTER(C.c_int)]),
    "ti_device_info": (C.c_int, [C.c_int, C.c_char_p, C.c_size_t, C.POINTER(C.c_size_t)]),
    "ti_set_device": (C.c_int, [C.c_int]),
    "ti_malloc": (C.c_int, [C.c_int, C.c_size_t, C.POINTER(C.c_void_p)]),
    "ti_free": (C.c_int, [C.c_int, C.c_void_p]),
    "ti_memset": (C.c_int, [C.c_void_p, C.c_int, C.c_size_t, C.c_void_p]),
    "ti_memcpy_h2d": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ti_memcpy_d2h": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ti_memcpy_d2d": (C.c_int, [C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ti_stream_sync": (C.c_int, [C.c_void_p]),
    "ti_op_embedding": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "ti_op_matmul_t": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "ti_op_rms_norm": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float, C.c_int, C.c_void_p]),
    "ti_op_rope": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_float,
                             C.POINTER(RopeScaling), C.c_void_p]),
    "ti_op_elementwise": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_float, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ti_op_add_bias": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "ti_op_softmax": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "ti_op_attention": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int,
                                  C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "ti_op_paged_attention_noalloc": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p,
                                                C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int,
                                                C.c_int, C.c_float, C.POINTER(RopeScaling), C.c_int, C.c_void_p,
                                                C.c_void_p]),
    "ti_op_cast": (C.c_int, [C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.c_size_t, C.c_void_p]),
    "ti_op_paged_attention": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p,
                                        C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_float,
                                        C.POINTER(RopeScaling), C.c_int, C.c_void_p, C.c_void_p]),
    "ti_op_transpose2d": (C.c_int, [C.c_int, C.c_void_p, C.c_void_p, C.c_int, C.c_int, C.c_void_p]),
    "ti_engine_create": (C.c_int, [C.POINTER(ModelDesc), C.POINTER(EngineOpts), C.POINTER(C.c_void_p)]),
    "ti_engine_destroy": (C.c_int, [C.c_void_p]),
    "ti_engine_memory": (C.c_int, [C.c_void_p] + [C.POINTER(C.c_size_t)] * 4),
    "ti_engine_load_tensor": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int, C.c_void_p, C.c_size_t]),
    "ti_engine_init_synthetic": (C.c_int, [C.c_void_p, C.c_uint64, C.c_float]),
    "ti_engine_read_tensor": (C.c_int, [C.c_void_p, C.c_char_p, C.c_void_p, C.c_size_t]),
    "ti_seq_create": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "ti_seq_free": (C.c_int, [C.c_void_p, C.c_int]),
    "ti_seq_reset": (C.c_int, [C.c_void_p, C.c_int]),
    "ti_seq_len": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_int)]),
    "ti_init": (C.c_int, [C.POINTER(C.c_int)]),
    "ti_shutdown": (C.c_int, []),
    "ti_selftest_waits": (C.c_int, [C.c_int, C.c_int, C.POINTER(C.c_double)]),
    "ti_engine_seq_set_sampler": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(Sampling)]),
    "ti_op_sample": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(Sampling), C.POINTER(C.c_float),
                               C.c_void_p, C.c_void_p]),
    "ti_sampler_draws": (C.c_int, [C.POINTER(Sampling), C.c_int, C.POINTER(C.c_float)]),
    "ti_seq_reserve": (C.c_int, [C.c_void_p, C.c_int, C.c_int]),
    "ti_seq_read_kv": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_int]),
    "ti_engine_prefill_chunked": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.c_int,
                                            C.POINTER(C.c_int32), C.c_int, C.c_void_p]),
    "ti_engine_prefill": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int32), C.c_int,
                                    C.c_void_p]),
    "ti_engine_decode": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p, C.c_void_p, C.c_int,
                                   C.c_void_p, C.c_void_p]),
    "ti_engine_bind": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "ti_engine_decode_device": (C.c_int, [C.c_void_p, C.c_void_p]),
    "ti_engine_unbind": (C.c_int, [C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "ti_engine_logits_device": (C.c_int, [C.c_void_p, C.POINTER(C.c_void_p)]),
    "ti_engine_check": (C.c_int, [C.c_void_p]),
    "ti_engine_launches_per_step": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_int)]),
    "ti_engine_launch_kernel": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_void_p]),
    "ti_pkm_create": (C.c_int, [C.c_int, C.c_int, C.c_int, C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    "ti_pkm_destroy": (C.c_int, [C.c_void_p]),
    "ti_pkm_register": (C.c_int, [C.c_void_p, C.c_void_p, C.c_void_p, C.c_int]),
    "ti_pkm_query": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p, C.c_void_p]),
    "ti_pkm_query_host": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.c_void_p, C.c_void_p]),
    "ti_adapter_create": (C.c_int, [C.c_void_p, C.c_int, C.c_float, C.c_int, C.POINTER(C.c_int)]),
    "ti_adapter_load_tensor": (C.c_int, [C.c_void_p, C.c_int, C.c_char_p, C.c_void_p, C.c_size_t]),
    "ti_adapter_init_synthetic": (C.c_int, [C.c_void_p, C.c_int, C.c_uint64, C.c_float, C.c_float]),
    "ti_adapter_stage_host": (C.c_int, [C.c_void_p, C.c_int]),
    "ti_adapter_evict": (C.c_int, [C.c_void_p, C.c_int]),
    "ti_adapter_prefetch_async": (C.c_int, [C.c_void_p, C.c_int]),
    "ti_adapter_is_resident": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_int)]),
    "ti_gguf_open": (C.c_int, [C.c_char_p, C.POINTER(C.c_void_p)]),
    "ti_gguf_close": (C.c_int, [C.c_void_p]),
    "ti_gguf_tensor_count": (C.c_int, [C.c_void_p, C.POINTER(C.c_int)]),
    "ti_gguf_tensor_info": (C.c_int, [C.c_void_p, C.c_int, C.POINTER(C.c_char_p), C.POINTER(C.c_int),
                                      C.POINTER(C.c_int), C.POINTER(C.c_int64), C.POINTER(C.c_void_p),
                                      C.POINTER(C.c_size_t)]),
    "ti_gguf_find": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_int)]),
    "ti_gguf_meta_int": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_int64)]),
    "ti_gguf_meta_float": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_double)]),
    "ti_gguf_meta_string": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_char_p)]),
    "ti_gguf_meta_array_len": (C.c_int, [C.c_void_p, C.c_char_p, C.POINTER(C.c_int64)]),
    "ti_gguf_meta_array_string": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int64, C.POINTER(C.c_void_p),
                                            C.POINTER(C.c_size_t)]),
    "ti_gguf_meta_array_int": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int64, C.POINTER(C.c_int64)]),
    "ti_gguf_meta_array_float": (C.c_int, [C.c_void_p, C.c_char_p, C.c_int64, C.POINTER(C.c_double)]),
    "ti_gguf_model_desc": (C.c_int, [C.c_void_p, C.c_void_p]),
    "ti_gguf_reference_name": (C.c_int, [C.c_void_p, C.c_int, C.c_char_p, C.c_size_t]),
    "ti_gguf_read": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.c_void_p, C.c_size_t]),
    "ti_engine_load_gguf": (C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_int)]),
    "ti_gguf_rope_inv_freq": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "ti_engine_set_rope_freqs": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "ti_router_create": (C.c_int, [C.c_void_p, C.c_void_p, C.POINTER(C.c_void_p)]),
    "ti_router_destroy": (C.c_int, [C.c_void_p]),
    "ti_router_observe": (C.c_int, [C.c_void_p, C.c_int, C.c_int, C.POINTER(C.c_int)]),
    "ti_router_prepare": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int]),
    "ti_router_forget": (C.c_int, [C.c_void_p, C.c_int]),
    "ti_router_stats_get": (C.c_int, [C.c_void_p, C.c_void_p]),
    "ti_router_actions": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.POINTER(C.c_int)]),
    "ti_router_resident": (C.c_int, [C.c_void_p, C.c_void_p, C.c_int, C.POINTER(C.c_int)]),
}


def lib():
    """Load libti_b200.so (raises OSError when it is missing: no fallback)."""
    global _lib
    if _lib is None:
        if not os.path.exists(LIB_PATH):
            raise OSError(f"libti_b200.so not built ({LIB_PATH}); run tensor-inference_b200/build.py")
        L = C.CDLL(LIB_PATH)
        for name, (res, args) in _SIGS.items():
            f = getattr(L, name)
            f.restype = res
            f.argtypes = args
        _lib = L
    return _lib


def exported_symbols():
    return sorted(_SIGS)


def check(status):
    if status != TI_OK:
        raise TiError(status, lib().ti_last_error().decode(errors="replace"))


def device_count():
    n = C.c_int(0)
    check(lib().ti_device_count(C.byref(n)))
    return n.value


def _ptr(a):
    """host pointer of a contiguous numpy array (or None)"""
    if a is None:
        return None
    assert a.flags["C_CONTIGUOUS"]
    return a.ctypes.data_as(C.c_void_p)


# ---------------------------------------------------------------- model configs
PRESETS = {
    # the benchmark configurations (shapes only; weights are synthetic)
    "tinyllama": dict(arch=ARCH_LLAMA, hidden=2048, n_layers=22, n_heads=32, n_kv_heads=4, head_dim=64,
                      intermediate=5632, vocab=32000, rms_eps=1e-5, rope_theta=10000.0),
    "llama3_8b": dict(arch=ARCH_LLAMA, hidden=4096, n_layers=32, n_heads=32, n_kv_heads=8, head_dim=128,
                      intermediate=14336, vocab=128256, rms_eps=1e-5, rope_theta=500000.0),
    "qwen25_7b": dict(arch=ARCH_QWEN2, hidden=3584, n_layers=28, n_heads=28, n_kv_heads=4, head_dim=128,
                      intermediate=18944, vocab=152064, rms_eps=1e-6, rope_theta=1000000.0, qkv_bias=1),
    "llama3_70b": dict(arch=ARCH_LLAMA, hidden=8192, n_layers=80, n_heads=64, n_kv_heads=8, head_dim=128,
                       intermediate=28672, vocab=128256, rms_eps=1e-5, rope_theta=500000.0),
}


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
    if rs:
        d.rope.apply_scaling = 1
        d.rope.factor = rs.get("factor", 1.0)
        d.rope.low_freq_factor = rs.get("low_freq_factor", 1.0)
        d.rope.high_freq_factor = rs.get("high_freq_factor", 4.0)
        d.rope.original_max_pos = rs.get("original_max_pos", 8192)
    else:
        d.rope.apply_scaling = 0
        d.rope.factor = 1.0
        d.rope.low_freq_factor = 1.0
        d.rope.high_freq_factor = 1.0
        d.rope.original_max_pos = 8192
    d.qkv_bias = kw.get("qkv_bias", 0)
    d.sliding_window = kw.get("sliding_window", -1)
    d.weight_format = kw.get("weight_format", WFMT_BF16)
    return d


def desc_from_config_json(cfg):
    """ModelConfig accessors with the reference's defaults (config.cpp:101-182,
    llama_config.cpp:5-33, qwen/gemma/mistral config structs)."""
    arch_name = (cfg.get("architectures") or [cfg.get("model_type", "")])[0] if isinstance(
        cfg.get("architectures"), list) and cfg.get("architectures") else cfg.get("model_type", "")
    a = str(arch_name).lower()
    t = cfg.get("text_config", cfg) if "mistral" in a else cfg
    arch = ARCH_QWEN2 if "qwen" in a else ARCH_GEMMA if "gemma" in a else ARCH_MISTRAL if "mistral" in a else ARCH_LLAMA
    hidden = t.get("hidden_size", 4096)
    heads = t.get("num_attention_heads", 32)
    kw = dict(arch=arch, hidden=hidden, n_layers=t.get("num_hidden_layers", 32), n_heads=heads,
              n_kv_heads=t.get("num_key_value_heads", heads), intermediate=t.get("intermediate_size", 11008),
              vocab=t.get("vocab_size", 32000), rms_eps=t.get("rms_norm_eps", 1e-5),
              rope_theta=t.get("rope_theta", 10000.0))
    if arch == ARCH_MISTRAL:
        kw["head_dim"] = t.get("head_dim", hidden // heads)
        sw = t.get("sliding_window")
        kw["sliding_window"] = sw if isinstance(sw, int) else -1
    else:
        kw["head_dim"] = hidden // heads
    if arch == ARCH_QWEN2:
        kw["qkv_bias"] = 1
    rs = cfg.get("rope_scaling")
    if isinstance(rs, dict) and rs.get("rope_type") in ("llama3", "yarn"):
        kw["rope_scaling"] = dict(factor=rs.get("factor", 1.0), low_freq_factor=rs.get("low_freq_factor", 1.0),
                                  high_freq_factor=rs.get("high_freq_factor", 4.0),
                                  original_max_pos=rs.get("original_max_position_embeddings", 8192))
    return model_desc(**kw)


def tensor_names(desc, layers=None):
    """checkpoint tensor names and shapes the engine expects (llama_model.cpp:47-72, qwen_model.cpp:28-52)"""
    H, I, hd = desc.hidden, desc.intermediate, desc.head_dim
    QW, KW = desc.n_heads * hd, desc.n_kv_heads * hd
    out = [("model.embed_tokens.weight", (desc.vocab, H)), ("model.norm.weight", (H,)),
           ("lm_head.weight", (desc.vocab, H))]
    for i in range(desc.n_layers if layers is None else layers):
        p = f"model.layers.{i}."
        out += [(p + "input_layernorm.weight", (H,)), (p + "post_attention_layernorm.weight", (H,)),
                (p + "self_attn.q_proj.weight", (QW, H)), (p + "self_attn.k_proj.weight", (KW, H)),
                (p + "self_attn.v_proj.weight", (KW, H)), (p + "self_attn.o_proj.weight", (H, QW)),
                (p + "mlp.gate_proj.weight", (I, H)), (p + "mlp.up_proj.weight", (I, H)),
                (p + "mlp.down_proj.weight", (H, I))]
        if desc.qkv_bias:
            out += [(p + "self_attn.q_proj.bias", (QW,)), (p + "self_attn.k_proj.bias", (KW,)),
                    (p + "self_attn.v_proj.bias", (KW,))]
    return out


def algorithmic_bytes_per_step(desc, batch, ctx_total, lora_bytes=0):
    """weights read once + K/V rows read (ctx_total = sum over sequences of cached tokens)"""
    H, I, hd = desc.hidden, desc.intermediate, desc.head_dim
    QW, KW = desc.n_heads * hd, desc.n_kv_heads * hd
    per_layer = (QW + 2 * KW) * H + H * QW + 3 * H * I
    # linear weights per element: bf16 2 bytes; GGUF Q4_0 18 / 32, Q8_0 34 / 32
    bpe = {WFMT_BF16: 2.0, WFMT_Q4_0: 18 / 32, WFMT_Q8_0: 34 / 32}[desc.weight_format]
    wbytes = bpe * desc.n_layers * per_layer + 2 * desc.vocab * H
    kv = ctx_total * desc.n_layers * 2 * KW * 2
    return wbytes + kv + lora_bytes


def nccl_unique_id():
    """128-byte NCCL unique id for a tensor-parallel group (one rank makes it, all use it)"""
    buf = C.create_string_buffer(128)
    check(lib().ti_nccl_unique_id(buf))
    return buf.raw


def tp_plan(desc, tp, rank):
    """the shard of `rank` in a group of `tp` (host only)"""
    sh = TpShard()
    check(lib().ti_tp_plan(C.byref(desc), tp, rank, C.byref(sh)))
    return {k: getattr(sh, k) for k, _ in TpShard._fields_}


# ---------------------------------------------------------------- engine
class RouterOpts(C.Structure):
    _fields_ = [("max_resident", C.c_int), ("prefetch_after", C.c_int), ("switch_after", C.c_int)]


class RouterStats(C.Structure):
    _fields_ = [(n, C.c_int64) for n in ("observations", "switches", "prefetches", "evictions", "hits")]


class Router:
    """Adapter pool + swap scheduler (ti_router_*) over an Engine's adapters;
    engine=None records the decisions only."""
    PREFETCH, EVICT = 1, 2

    def __init__(self, engine=None, max_resident=4, prefetch_after=2, switch_after=4):
        o = RouterOpts(max_resident, prefetch_after, switch_after)
        h = C.c_void_p()
        check(lib().ti_router_create(engine.h if engine is not None else None, C.byref(o), C.byref(h)))
        self.h = h
        self.engine = engine

    def close(self):
        if self.h:
            lib().ti_router_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def observe(self, seq, candidate):
        u = C.c_int()
        check(lib().ti_router_observe(self.h, seq, int(candidate), C.byref(u)))
        return u.value

    def prepare(self, adapters):
        a = np.ascontiguousarray(adapters, np.int32)
        check(lib().ti_router_prepare(self.h, _ptr(a), a.size))

    def forget(self, seq):
        check(lib().ti_router_forget(self.h, seq))

    def stats(self):
        s = RouterStats()
        check(lib().ti_router_stats_get(self.h, C.byref(s)))
        return {n: getattr(s, n) for n, _ in RouterStats._fields_}

    def actions(self):
        out = np.empty(2 * 256, np.int32)
        n = C.c_int()
        res = []
        while True:
            check(lib().ti_router_actions(self.h, _ptr(out), 256, C.byref(n)))
            res += [(int(out[2 * i]), int(out[2 * i + 1])) for i in range(n.value)]
            if n.value < 256:
                return res

    def resident(self):
        n = C.c_int()
        check(lib().ti_router_resident(self.h, None, 0, C.byref(n)))
        out = np.empty(max(1, n.value), np.int32)
        check(lib().ti_router_resident(self.h, _ptr(out), out.size, C.byref(n)))
        return [int(x) for x in out[:n.value]]


class Gguf:
    """A GGUF model file mapped read-only (ti_gguf_*): tensors with llama.cpp
    names and ggml types, metadata, the model description, and each tensor
    as the engine receives it (reference row order, bf16 or its own blocks)."""

    def __init__(self, path):
        h = C.c_void_p()
        check(lib().ti_gguf_open(os.fsencode(path), C.byref(h)))
        self.h = h

    def close(self):
        if self.h:
            lib().ti_gguf_close(self.h)
            self.h = None

    def __enter__(self):
        return self

    def __exit__(self, *a):
        self.close()

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def __len__(self):
        n = C.c_int()
        check(lib().ti_gguf_tensor_count(self.h, C.byref(n)))
        return n.value

    def info(self, i):
        name, t, nd = C.c_char_p(), C.c_int(), C.c_int()
        dims = (C.c_int64 * 4)()
        data, nbytes = C.c_void_p(), C.c_size_t()
        check(lib().ti_gguf_tensor_info(self.h, i, C.byref(name), C.byref(t), C.byref(nd), dims, C.byref(data),
                                        C.byref(nbytes)))
        return dict(name=name.value.decode(errors="replace"), type=t.value, dims=tuple(dims[:nd.value]), bytes=nbytes.value)

    def find(self, name):
        i = C.c_int()
        check(lib().ti_gguf_find(self.h, name.encode(), C.byref(i)))
        return i.value

    def meta_int(self, key):
        v = C.c_int64()
        check(lib().ti_gguf_meta_int(self.h, key.encode(), C.byref(v)))
        return v.value

    def meta_float(self, key):
        v = C.c_double()
        check(lib().ti_gguf_meta_float(self.h, key.encode(), C.byref(v)))
        return v.value

    def meta_str(self, key):
        v = C.c_char_p()
        check(lib().ti_gguf_meta_string(self.h, key.encode(), C.byref(v)))
        return v.value.decode(errors="replace")

    def meta_array_len(self, key):
        v = C.c_int64()
        check(lib().ti_gguf_meta_array_len(self.h, key.encode(), C.byref(v)))
        return v.value

    def meta_array(self, key):
        """array metadata as a list: str (decoded as UTF-8), int or float elements"""
        n = self.meta_array_len(key)
        k = key.encode()
        if n == 0:
            return []
        p, ln = C.c_void_p(), C.c_size_t()
        if lib().ti_gguf_meta_array_string(self.h, k, 0, C.byref(p), C.byref(ln)) == TI_OK:
            out = []
            for i in range(n):
                check(lib().ti_gguf_meta_array_string(self.h, k, i, C.byref(p), C.byref(ln)))
                out.append(C.string_at(p, ln.value).decode(errors="replace"))
            return out
        iv = C.c_int64()
        if lib().ti_gguf_meta_array_int(self.h, k, 0, C.byref(iv)) == TI_OK:
            out = []
            for i in range(n):
                check(lib().ti_gguf_meta_array_int(self.h, k, i, C.byref(iv)))
                out.append(iv.value)
            return out
        fv = C.c_double()
        out = []
        for i in range(n):
            check(lib().ti_gguf_meta_array_float(self.h, k, i, C.byref(fv)))
            out.append(fv.value)
        return out

    def model_desc(self):
        d = ModelDesc()
        check(lib().ti_gguf_model_desc(self.h, C.byref(d)))
        return d

    def rope_inv_freq(self, n):
        out = np.empty(n, np.float32)
        check(lib().ti_gguf_rope_inv_freq(self.h, _ptr(out), n))
        return out

    def reference_name(self, i):
        buf = C.create_string_buffer(256)
        check(lib().ti_gguf_reference_name(self.h, i, buf, len(buf)))
        return buf.value.decode(errors="replace")

    def read(self, i, dtype=DTYPE_BF16):
        """tensor i in the reference's row order: bf16 bits [rows, cols] (uint16) or
        its own GGUF blocks (uint8, dtype DTYPE_Q4_0 / DTYPE_Q8_0)"""
        inf = self.info(i)
        dims = inf["dims"]
        cols = dims[0]
        rows = int(np.prod(dims[1:])) if len(dims) > 1 else 1
        if dtype == DTYPE_BF16:
            out = np.empty((rows, cols), np.uint16)
        else:
            out = np.empty(inf["bytes"], np.uint8)
        check(lib().ti_gguf_read(self.h, i, dtype, _ptr(out), out.nbytes))
        return out


class Engine:
    def __init__(self, desc, device=0, max_batch=1, max_seqs=None, max_seq_len=4096, kv_pages=0, max_adapters=0,
                 max_lora_rank=0, lora_proj_mask=0, tp_size=1, tp_rank=0, nccl_id=None):
        L = lib()
        self.desc = desc
        o = EngineOpts()
        o.device = device
        o.max_batch = max_batch
        o.max_seqs = max_seqs or max_batch
        o.max_seq_len = max_seq_len
        o.kv_pages = kv_pages
        o.max_adapters = max_adapters
        o.max_lora_rank = max_lora_rank
        o.lora_proj_mask = lora_proj_mask
        o.tp_size = tp_size
        o.tp_rank = tp_rank
        self._nccl_id = nccl_id
        o.nccl_id = C.cast(C.c_char_p(nccl_id), C.c_void_p) if nccl_id else None
        self.opts = o
        h = C.c_void_p()
        check(L.ti_engine_create(C.byref(desc), C.byref(o), C.byref(h)))
        self.h = h

    def close(self):
        if self.h:
            lib().ti_engine_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def init_synthetic(self, seed, std=0.02):
        check(lib().ti_engine_init_synthetic(self.h, seed, std))

    def load_tensor(self, name, arr, dtype=DTYPE_BF16):
        arr = np.ascontiguousarray(arr)
        check(lib().ti_engine_load_tensor(self.h, name.encode(), dtype, _ptr(arr), arr.nbytes))

    def read_tensor(self, name, shape):
        out = np.empty(shape, np.uint16)
        check(lib().ti_engine_read_tensor(self.h, name.encode(), _ptr(out), out.nbytes))
        return out

    def set_rope_freqs(self, inv_freq):
        a = np.ascontiguousarray(inv_freq, np.float32)
        check(lib().ti_engine_set_rope_freqs(self.h, _ptr(a), a.size))

    def load_gguf(self, g):
        """upload every model tensor of an open Gguf; returns the number of uploads"""
        n = C.c_int()
        check(lib().ti_engine_load_gguf(self.h, g.h, C.byref(n)))
        return n.value

    def memory(self):
        v = [C.c_size_t() for _ in range(4)]
        check(lib().ti_engine_memory(self.h, *[C.byref(x) for x in v]))
        return dict(zip(("weights", "kv", "adapters", "work"), (x.value for x in v)))

    def seq_create(self):
        s = C.c_int()
        check(lib().ti_seq_create(self.h, C.byref(s)))
        return s.value

    def seq_free(self, sid):
        check(lib().ti_seq_free(self.h, sid))

    def seq_reset(self, sid):
        check(lib().ti_seq_reset(self.h, sid))

    def seq_len(self, sid):
        n = C.c_int()
        check(lib().ti_seq_len(self.h, sid, C.byref(n)))
        return n.value

    def set_sampler(self, sid, kind=SAMPLE_GREEDY, temperature=1.0, p=0.95, k=40, seed=None):
        """The sampler of the ids this sequence's decode / prefill calls return
        (defaults as TopP / TopK in the reference); seed None = std::random_device."""
        smp = Sampling(kind, temperature, p, k, 0 if seed is None else 1, 0 if seed is None else seed)
        check(lib().ti_engine_seq_set_sampler(self.h, sid, C.byref(smp)))

    def seq_reserve(self, sid, n_tokens):
        check(lib().ti_seq_reserve(self.h, sid, n_tokens))

    def seq_fill_synthetic(self, sid, n_tokens, seed=0, std=1.0):
        """n_tokens of synthetic cached context for sequence sid (long-context benchmarks)"""
        check(lib().ti_seq_fill_synthetic(self.h, sid, n_tokens, seed, std))

    def seq_read_kv(self, sid, layer, which, length):
        out = np.empty((length, self.desc.n_kv_heads // max(1, self.opts.tp_size), self.desc.head_dim), np.uint16)
        check(lib().ti_seq_read_kv(self.h, sid, layer, which, _ptr(out), length))
        return out

    def prefill(self, sid, ids, adapter=-1, logits=LOGITS_NONE, chunk=None):
        """run a prompt through a sequence; chunk: tokens per step (batched
        prefill, ti_engine_prefill_chunked) instead of one step per token"""
        ids = np.ascontiguousarray(ids, np.int32)
        nxt = C.c_int32()
        out = None
        if logits == LOGITS_BF16:
            out = np.empty(self.desc.vocab, np.uint16)
        elif logits == LOGITS_F32:
            out = np.empty(self.desc.vocab, np.float32)
        if chunk:
            check(lib().ti_engine_prefill_chunked(self.h, sid, _ptr(ids), len(ids), adapter, chunk, C.byref(nxt),
                                                  logits, _ptr(out)))
        else:
            check(lib().ti_engine_prefill(self.h, sid, _ptr(ids), len(ids), adapter, C.byref(nxt), logits,
                                          _ptr(out)))
        return (nxt.value, out) if logits else nxt.value

    def decode(self, seq_ids, tokens, adapters=None, logits=LOGITS_NONE, stream=None):
        seq_ids = np.ascontiguousarray(seq_ids, np.int32)
        tokens = np.ascontiguousarray(tokens, np.int32)
        ad = None if adapters is None else np.ascontiguousarray(adapters, np.int32)
        B = len(seq_ids)
        nxt = np.empty(B, np.int32)
        out = None
        if logits == LOGITS_BF16:
            out = np.empty((B, self.desc.vocab), np.uint16)
        elif logits == LOGITS_F32:
            out = np.empty((B, self.desc.vocab), np.float32)
        check(lib().ti_engine_decode(self.h, B, _ptr(seq_ids), _ptr(tokens), _ptr(ad), _ptr(nxt), logits, _ptr(out),
                                     C.c_void_p(stream) if stream else None))
        return (nxt, out) if logits else nxt

    def bind(self, seq_ids, first_tokens, adapters=None):
        seq_ids = np.ascontiguousarray(seq_ids, np.int32)
        first_tokens = np.ascontiguousarray(first_tokens, np.int32)
        ad = None if adapters is None else np.ascontiguousarray(adapters, np.int32)
        self._bound = len(seq_ids)
        check(lib().ti_engine_bind(self.h, len(seq_ids), _ptr(seq_ids), _ptr(first_tokens), _ptr(ad)))

    def decode_device(self, stream=None):
        check(lib().ti_engine_decode_device(self.h, C.c_void_p(stream) if stream else None))

    def unbind(self, steps, stream=None):
        out = np.empty(self._bound, np.int32)
        check(lib().ti_engine_unbind(self.h, steps, _ptr(out), C.c_void_p(stream) if stream else None))
        return out

    def logits_device_ptr(self):
        p = C.c_void_p()
        check(lib().ti_engine_logits_device(self.h, C.byref(p)))
        return p.value

    def check(self):
        check(lib().ti_engine_check(self.h))

    def launch_kernel(self, kind, layer, batch, stream=None):
        check(lib().ti_engine_launch_kernel(self.h, kind, layer, batch, C.c_void_p(stream) if stream else None))

    # ---- LoRA adapters
    def adapter_create(self, rank, alpha, proj_mask):
        a = C.c_int()
        check(lib().ti_adapter_create(self.h, rank, alpha, proj_mask, C.byref(a)))
        return a.value

    def adapter_load_tensor(self, adapter, name, arr):
        arr = np.ascontiguousarray(arr, np.uint16)
        check(lib().ti_adapter_load_tensor(self.h, adapter, name.encode(), _ptr(arr), arr.nbytes))

    def adapter_init_synthetic(self, adapter, seed, std_a=0.02, std_b=0.001):
        check(lib().ti_adapter_init_synthetic(self.h, adapter, seed, std_a, std_b))

    def adapter_stage_host(self, adapter):
        check(lib().ti_adapter_stage_host(self.h, adapter))

    def adapter_evict(self, adapter):
        check(lib().ti_adapter_evict(self.h, adapter))

    def adapter_prefetch_async(self, adapter):
        check(lib().ti_adapter_prefetch_async(self.h, adapter))

    def adapter_is_resident(self, adapter):
        r = C.c_int()
        check(lib().ti_adapter_is_resident(self.h, adapter, C.byref(r)))
        return bool(r.value)

    def launches_per_step(self, batch):
        n = C.c_int()
        check(lib().ti_engine_launches_per_step(self.h, batch, C.byref(n)))
        return n.value


# ---------------------------------------------------------------- PKM router
class Pkm:
    """two-codebook product-key router (ti_pkm_*)"""

    def __init__(self, c1, c2, device=0):
        c1 = np.ascontiguousarray(c1, np.float32)
        c2 = np.ascontiguousarray(c2, np.float32)
        assert c1.shape == c2.shape and c1.ndim == 2
        self.n_codes, self.half_dim = c1.shape
        h = C.c_void_p()
        check(lib().ti_pkm_create(device, self.n_codes, self.half_dim, _ptr(c1), _ptr(c2), C.byref(h)))
        self.h = h

    def close(self):
        if self.h:
            lib().ti_pkm_destroy(self.h)
            self.h = None

    def __del__(self):
        try:
            self.close()
        except Exception:
            pass

    def register(self, centroids, adapter_ids):
        centroids = np.ascontiguousarray(centroids, np.float32)
        ids = np.ascontiguousarray(adapter_ids, np.int32)
        check(lib().ti_pkm_register(self.h, _ptr(centroids), _ptr(ids), len(ids)))

    def query_host(self, queries):
        q = np.ascontiguousarray(queries, np.float32)
        n = q.shape[0]
        addr = np.empty(n, np.int32)
        ad = np.empty(n, np.int32)
        check(lib().ti_pkm_query_host(self.h, _ptr(q), n, _ptr(addr), _ptr(ad)))
        return addr, ad

    def query(self, q_dev, n, addr_dev, adapter_dev, stream=None):
        check(lib().ti_pkm_query(self.h, C.c_void_p(q_dev), n, C.c_void_p(addr_dev), C.c_void_p(adapter_dev),
                                 C.c_void_p(stream) if stream else None))

