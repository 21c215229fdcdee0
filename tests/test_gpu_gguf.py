"""GGUF files into the engine (ti_engine_load_gguf): an engine's weights are
written out the way llama.cpp lays out a checkpoint (llama.cpp names, q/k rows
of llama files permuted, gemma norms as 1 + w, Q4_0 / Q8_0 linear weights as
blocks, tied embeddings without output.weight) and loaded into a second engine,
which must produce bit-identical logits and greedy ids."""
import ctypes as C

import numpy as np
import pytest

import oracle
import ti_b200 as ti
from gguf_writer import (ARR, F32, GGML_BF16, GGML_F32, GGML_Q4_0, GGML_Q8_0, STR, U32, gguf_name, permute_rows,
                         write)

pytestmark = pytest.mark.gpu

SMALL = dict(arch=ti.ARCH_LLAMA, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, intermediate=512,
             vocab=1000, rms_eps=1e-5, rope_theta=10000.0)
ARCH_NAME = {ti.ARCH_LLAMA: "llama", ti.ARCH_QWEN2: "qwen2", ti.ARCH_GEMMA: "gemma"}


def _shapes(kw):
    H, I, V = kw["hidden"], kw["intermediate"], kw["vocab"]
    hd = kw["head_dim"]
    QW, KW = kw["n_heads"] * hd, kw["n_kv_heads"] * hd
    out = {"model.embed_tokens.weight": (V, H), "model.norm.weight": (H,), "lm_head.weight": (V, H)}
    for i in range(kw["n_layers"]):
        p = f"model.layers.{i}."
        out.update({p + "input_layernorm.weight": (H,), p + "post_attention_layernorm.weight": (H,),
                    p + "self_attn.q_proj.weight": (QW, H), p + "self_attn.k_proj.weight": (KW, H),
                    p + "self_attn.v_proj.weight": (KW, H), p + "self_attn.o_proj.weight": (H, QW),
                    p + "mlp.gate_proj.weight": (I, H), p + "mlp.up_proj.weight": (I, H),
                    p + "mlp.down_proj.weight": (H, I)})
        if kw.get("qkv_bias"):
            out.update({p + "self_attn.q_proj.bias": (QW,), p + "self_attn.k_proj.bias": (KW,),
                        p + "self_attn.v_proj.bias": (KW,)})
    return out


def _is_linear(name):
    return name.startswith("model.layers.") and name.endswith("_proj.weight")


def _export(eng, kw, path, wfmt, tied, extra=()):
    arch = ARCH_NAME[kw["arch"]]
    tensors = []
    for name, shape in _shapes(kw).items():
        if tied and name == "lm_head.weight":
            continue
        rows = shape[0] if len(shape) == 2 else 1
        heads = {"self_attn.q_proj.weight": kw["n_heads"], "self_attn.k_proj.weight": kw["n_kv_heads"]}.get(
            name.split(".", 3)[-1]) if arch == "llama" and _is_linear(name) else None
        if _is_linear(name) and wfmt != ti.WFMT_BF16:
            rb = shape[1] // 32 * (18 if wfmt == ti.WFMT_Q4_0 else 34)
            blocks = np.empty((rows, rb), np.uint8)
            ti.check(ti.lib().ti_engine_read_tensor(eng.h, name.encode(), blocks.ctypes.data_as(C.c_void_p),
                                                    blocks.nbytes))
            if heads:
                blocks = permute_rows(blocks, heads)
            t, data = (GGML_Q4_0 if wfmt == ti.WFMT_Q4_0 else GGML_Q8_0), np.ascontiguousarray(blocks).tobytes()
        else:
            a = eng.read_tensor(name, shape).reshape(rows, -1)
            if heads:
                a = permute_rows(a, heads)
            if arch == "gemma" and name.endswith("layernorm.weight") or (arch == "gemma" and name == "model.norm.weight"):
                t, data = GGML_F32, (oracle.bf16_to_f32(a) + 1.0).astype(np.float32).tobytes()  # stored as 1 + w
            else:
                t, data = GGML_BF16, np.ascontiguousarray(a).tobytes()
        tensors.append((gguf_name(name), t, tuple(reversed(shape)), data))
    meta = [("general.architecture", STR, arch), (f"{arch}.block_count", U32, kw["n_layers"]),
            (f"{arch}.embedding_length", U32, kw["hidden"]), (f"{arch}.feed_forward_length", U32, kw["intermediate"]),
            (f"{arch}.attention.head_count", U32, kw["n_heads"]),
            (f"{arch}.attention.head_count_kv", U32, kw["n_kv_heads"]),
            (f"{arch}.attention.key_length", U32, kw["head_dim"]),
            (f"{arch}.attention.layer_norm_rms_epsilon", F32, kw["rms_eps"]),
            (f"{arch}.rope.freq_base", F32, kw["rope_theta"]),
            ("tokenizer.ggml.tokens", ARR, (STR, [f"t{i}" for i in range(4)]))]
    write(path, meta, tensors + list(extra))


@pytest.mark.parametrize("arch,wfmt,tied", [(ti.ARCH_LLAMA, ti.WFMT_BF16, False), (ti.ARCH_LLAMA, ti.WFMT_Q4_0, False),
                                            (ti.ARCH_QWEN2, ti.WFMT_Q8_0, False), (ti.ARCH_GEMMA, ti.WFMT_BF16, True)])
def test_gguf_roundtrip_bit_identical(tmp_path, arch, wfmt, tied):
    kw = dict(SMALL, arch=arch, weight_format=wfmt)
    if arch == ti.ARCH_QWEN2:
        kw["qkv_bias"] = 1
    if arch == ti.ARCH_GEMMA:
        kw["rms_eps"] = 1e-6
    a = ti.Engine(ti.model_desc(**kw), device=0, max_batch=2, max_seqs=2, max_seq_len=64)
    a.init_synthetic(11, 0.05)
    if tied:
        emb = a.read_tensor("model.embed_tokens.weight", (kw["vocab"], kw["hidden"]))
        a.load_tensor("lm_head.weight", emb)
    path = tmp_path / "model.gguf"
    _export(a, kw, path, wfmt, tied)
    with ti.Gguf(path) as g:
        d = g.model_desc()
        assert (d.arch, d.hidden, d.n_layers, d.n_heads, d.n_kv_heads, d.head_dim, d.intermediate, d.vocab,
                d.weight_format, d.qkv_bias) == (arch, kw["hidden"], kw["n_layers"], kw["n_heads"], kw["n_kv_heads"],
                                                 kw["head_dim"], kw["intermediate"], kw["vocab"], wfmt,
                                                 kw.get("qkv_bias", 0))
        b = ti.Engine(d, device=0, max_batch=2, max_seqs=2, max_seq_len=64)
        n = b.load_gguf(g)
        assert n == len(_shapes(kw))  # tied: token_embd loaded twice (embedding and LM head)
    prompt = oracle.fill_ids("gg", 7, 3, kw["vocab"])
    outs = []
    for eng in (a, b):
        s = eng.seq_create()
        nxt, lb = eng.prefill(s, prompt, logits=ti.LOGITS_BF16)
        ids = [int(nxt)]
        for _ in range(3):
            nxt, l2 = eng.decode([s], [ids[-1]], logits=ti.LOGITS_BF16)
            ids.append(int(nxt[0]))
        outs.append((ids, lb, l2))
        eng.check()
    assert outs[0][0] == outs[1][0]
    np.testing.assert_array_equal(outs[0][1], outs[1][1])
    np.testing.assert_array_equal(outs[0][2], outs[1][2])
    a.close()
    b.close()


def _rope_table(hd, theta, scaling=None):
    out = np.empty(hd // 2, np.float32)
    rs = None
    if scaling:
        rs = oracle.RopeScaling(1, scaling["factor"], scaling["low_freq_factor"], scaling["high_freq_factor"],
                                scaling["original_max_pos"])
    oracle.lib().orc_rope_freqs(hd, theta, ctypes_ref(rs), oracle.ptr(out))
    return out


def ctypes_ref(x):
    return C.byref(x) if x is not None else None


def test_gguf_rope_factors_reproduce_llama3_scaling(tmp_path):
    # llama 3.1 style files carry per-dimension RoPE factors instead of scaling metadata
    sc = dict(factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0, original_max_pos=64)
    kw = dict(SMALL, rope_theta=500000.0, rope_scaling=sc, weight_format=ti.WFMT_BF16)
    a = ti.Engine(ti.model_desc(**kw), device=0, max_batch=1, max_seqs=1, max_seq_len=64)
    a.init_synthetic(13, 0.05)
    hd = kw["head_dim"]
    factors = (_rope_table(hd, kw["rope_theta"]) / _rope_table(hd, kw["rope_theta"], sc)).astype(np.float32)
    assert factors.max() > 1.5  # the scaling reaches these dimensions
    path = tmp_path / "scaled.gguf"
    _export(a, kw, path, ti.WFMT_BF16, False, [("rope_freqs.weight", GGML_F32, (hd // 2,), factors.tobytes())])
    with ti.Gguf(path) as g:
        b = ti.Engine(g.model_desc(), device=0, max_batch=1, max_seqs=1, max_seq_len=64)
        b.load_gguf(g)
    prompt = oracle.fill_ids("rs", 9, 4, kw["vocab"])
    res = []
    for eng in (a, b):
        s = eng.seq_create()
        nxt, lb = eng.prefill(s, prompt, logits=ti.LOGITS_BF16)
        ids = [int(nxt)]
        for _ in range(3):
            nxt, l2 = eng.decode([s], [ids[-1]], logits=ti.LOGITS_BF16)
            ids.append(int(nxt[0]))
        res.append((ids, oracle.bf16_to_f32(lb), oracle.bf16_to_f32(l2[0])))
        eng.check()
    assert res[0][0] == res[1][0]
    for k in (1, 2):
        err = float(np.abs(res[0][k] - res[1][k]).max() / np.abs(res[0][k]).max())
        assert err <= 1e-2, err  # base / factor equals the scaled table to about one ulp
    a.close()
    b.close()
