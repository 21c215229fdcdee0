"""GGUF reader (ti_gguf_*): container parsing, metadata, model description,
name mapping, conversions and the q/k row order of llama-architecture files.
Host-only: no GPU needed (the files are written by tests/gguf_writer.py)."""
import os

import numpy as np
import pytest

import oracle
import ti_b200 as ti
from gguf_writer import (ARR, BOOL, F32, F64, GGML_BF16, GGML_F16, GGML_F32, GGML_Q4_0, GGML_Q8_0, I32, STR, U8,
                         U32, U64, gguf_name, permute_rows, write)


def _blocks(x, quant):
    x = np.ascontiguousarray(x, np.float32).reshape(-1)
    nb = x.size // 32 * (18 if quant == "q4" else 34)
    out = np.empty(nb, np.uint8)
    f = oracle.lib().orc_q4_0_quantize if quant == "q4" else oracle.lib().orc_q8_0_quantize
    f(oracle.ptr(x), x.size, oracle.ptr(out))
    return out


def _dequant(blocks, n, quant):
    out = np.empty(n, np.float32)
    f = oracle.lib().orc_q4_0_dequantize if quant == "q4" else oracle.lib().orc_q8_0_dequantize
    f(oracle.ptr(np.ascontiguousarray(blocks)), n, oracle.ptr(out))
    return out


def _llama_meta(arch="llama", hidden=64, layers=1, heads=4, kv=2, ffn=128, extra=()):
    return [("general.architecture", STR, arch), ("general.alignment", U32, 32),
            (f"{arch}.block_count", U32, layers), (f"{arch}.embedding_length", U32, hidden),
            (f"{arch}.feed_forward_length", U32, ffn), (f"{arch}.attention.head_count", U32, heads),
            (f"{arch}.attention.head_count_kv", U32, kv),
            (f"{arch}.attention.layer_norm_rms_epsilon", F32, 1e-5), (f"{arch}.rope.freq_base", F32, 500000.0),
            ("tokenizer.ggml.tokens", ARR, (STR, ["<s>", "</s>", "a"])), *extra]


def test_container_metadata_and_tensor_table(tmp_path):
    rng = np.random.default_rng(0)
    f32 = rng.standard_normal(64).astype(np.float32)
    f16 = rng.standard_normal((3, 32)).astype(np.float16)
    bf = oracle.f32_to_bf16(rng.standard_normal((2, 64)).astype(np.float32))
    q4 = _blocks(rng.standard_normal((4, 64)), "q4")
    q8 = _blocks(rng.standard_normal((2, 32)), "q8")
    meta = _llama_meta() + [("x.u8", U8, 7), ("x.bool", BOOL, 1), ("x.u64", U64, 1 << 40), ("x.f64", F64, 2.5),
                            ("x.i32", I32, -3), ("x.arr", ARR, (U32, [1, 2, 3, 4]))]
    tensors = [("output_norm.weight", GGML_F32, (64,), f32.tobytes()),
               ("blk.0.ffn_up.weight", GGML_F16, (32, 3), f16.tobytes()),
               ("token_embd.weight", GGML_BF16, (64, 2), bf.tobytes()),
               ("blk.0.attn_v.weight", GGML_Q4_0, (64, 4), q4.tobytes()),
               ("blk.0.ffn_down.weight", GGML_Q8_0, (32, 2), q8.tobytes()),
               ("blk.0.exotic.weight", 16, (256, 1), bytes(66))]  # IQ2_XXS: a type this reader does not decode
    p = tmp_path / "m.gguf"
    write(p, meta, tensors)
    with ti.Gguf(p) as g:
        assert len(g) == 6
        names = [g.info(i)["name"] for i in range(6)]
        assert names == [t[0] for t in tensors]
        assert g.info(3)["type"] == ti.GGML_Q4_0 and g.info(3)["dims"] == (64, 4)
        assert g.info(3)["bytes"] == q4.nbytes and g.info(4)["bytes"] == q8.nbytes
        assert g.info(5)["bytes"] == 0
        assert g.find("blk.0.attn_v.weight") == 3
        assert g.meta_str("general.architecture") == "llama"
        assert g.meta_int("llama.block_count") == 1 and g.meta_int("x.u8") == 7 and g.meta_int("x.bool") == 1
        assert g.meta_int("x.u64") == 1 << 40 and g.meta_int("x.i32") == -3
        assert g.meta_float("x.f64") == 2.5 and g.meta_float("llama.block_count") == 1.0
        assert abs(g.meta_float("llama.rope.freq_base") - 500000.0) < 1e-3
        assert g.meta_array_len("tokenizer.ggml.tokens") == 3 and g.meta_array_len("x.arr") == 4
        with pytest.raises(ti.TiError) as ei:
            g.meta_int("general.architecture")  # a string, not an integer
        assert ei.value.status == ti.TI_ERR_NOT_FOUND
        with pytest.raises(ti.TiError) as ei:
            g.find("nope")
        assert ei.value.status == ti.TI_ERR_NOT_FOUND
        # conversions to bf16 (rows as the engine receives them)
        np.testing.assert_array_equal(g.read(0)[0], oracle.f32_to_bf16(f32))
        np.testing.assert_array_equal(g.read(1), oracle.f32_to_bf16(f16.astype(np.float32)))
        np.testing.assert_array_equal(g.read(2), bf)
        np.testing.assert_array_equal(g.read(3), oracle.f32_to_bf16(_dequant(q4, 256, "q4").reshape(4, 64)))
        np.testing.assert_array_equal(g.read(4), oracle.f32_to_bf16(_dequant(q8, 64, "q8").reshape(2, 32)))
        # blocks pass through in their own type only
        np.testing.assert_array_equal(g.read(3, ti.DTYPE_Q4_0), q4)
        with pytest.raises(ti.TiError) as ei:
            g.read(3, ti.DTYPE_Q8_0)
        assert ei.value.status == ti.TI_ERR_UNSUPPORTED
        with pytest.raises(ti.TiError) as ei:
            g.read(5)
        assert ei.value.status == ti.TI_ERR_UNSUPPORTED


def test_reference_names():
    for ref in ["model.embed_tokens.weight", "model.norm.weight", "lm_head.weight",
                "model.layers.0.input_layernorm.weight", "model.layers.11.post_attention_layernorm.weight",
                "model.layers.3.self_attn.q_proj.weight", "model.layers.3.self_attn.k_proj.bias",
                "model.layers.7.self_attn.o_proj.weight", "model.layers.2.mlp.gate_proj.weight",
                "model.layers.2.mlp.up_proj.weight", "model.layers.2.mlp.down_proj.weight"]:
        assert gguf_name(ref)  # the writer's table covers every reference name


def test_name_mapping_and_model_desc(tmp_path):
    hidden, heads, kv, ffn, vocab = 64, 4, 2, 128, 10
    hd = hidden // heads
    tensors = []
    names = ["model.embed_tokens.weight", "model.norm.weight", "model.layers.0.input_layernorm.weight",
             "model.layers.0.self_attn.q_proj.weight", "model.layers.0.self_attn.k_proj.weight",
             "model.layers.0.self_attn.v_proj.weight", "model.layers.0.self_attn.o_proj.weight",
             "model.layers.0.post_attention_layernorm.weight", "model.layers.0.mlp.gate_proj.weight",
             "model.layers.0.mlp.up_proj.weight", "model.layers.0.mlp.down_proj.weight"]
    shapes = {"model.embed_tokens.weight": (vocab, hidden), "model.norm.weight": (hidden,),
              "model.layers.0.input_layernorm.weight": (hidden,),
              "model.layers.0.post_attention_layernorm.weight": (hidden,),
              "model.layers.0.self_attn.q_proj.weight": (heads * hd, hidden),
              "model.layers.0.self_attn.k_proj.weight": (kv * hd, hidden),
              "model.layers.0.self_attn.v_proj.weight": (kv * hd, hidden),
              "model.layers.0.self_attn.o_proj.weight": (hidden, heads * hd),
              "model.layers.0.mlp.gate_proj.weight": (ffn, hidden), "model.layers.0.mlp.up_proj.weight": (ffn, hidden),
              "model.layers.0.mlp.down_proj.weight": (hidden, ffn)}
    for n in names:
        a = oracle.fill_bf16(n, shapes[n], 3, 0.05)
        tensors.append((gguf_name(n), GGML_BF16, tuple(reversed(shapes[n])), a.tobytes()))
    tensors.append(("rope_factors_long.weight", GGML_F32, (8,), bytes(32)))  # not a model tensor
    p = tmp_path / "m.gguf"
    write(p, _llama_meta("qwen2", hidden, 1, heads, kv, ffn), tensors)
    with ti.Gguf(p) as g:
        for i, n in enumerate(names):
            assert g.reference_name(i) == n
        with pytest.raises(ti.TiError) as ei:
            g.reference_name(len(names))
        assert ei.value.status == ti.TI_ERR_NOT_FOUND
        d = g.model_desc()
        assert (d.arch, d.hidden, d.n_layers, d.n_heads, d.n_kv_heads, d.head_dim, d.intermediate, d.vocab) == \
            (ti.ARCH_QWEN2, hidden, 1, heads, kv, hd, ffn, vocab)
        assert abs(d.rms_eps - 1e-5) < 1e-9 and d.rope_theta == 500000.0 and d.weight_format == ti.WFMT_BF16
        assert d.qkv_bias == 0
        # qwen2 files keep the reference row order
        np.testing.assert_array_equal(g.read(3), oracle.fill_bf16(names[3], shapes[names[3]], 3, 0.05))


@pytest.mark.parametrize("fmt", ["bf16", "q4"])
def test_llama_q_k_rows_put_back(tmp_path, fmt):
    heads, kv, hidden = 4, 2, 64
    hd = hidden // heads
    wq = oracle.bf16_to_f32(oracle.fill_bf16("q", (heads * hd, hidden), 5, 0.05))
    wk = oracle.bf16_to_f32(oracle.fill_bf16("k", (kv * hd, hidden), 6, 0.05))
    if fmt == "bf16":
        data = [oracle.f32_to_bf16(permute_rows(w, n)).tobytes() for w, n in ((wq, heads), (wk, kv))]
        t = GGML_BF16
    else:
        data = [_blocks(permute_rows(w, n), "q4").tobytes() for w, n in ((wq, heads), (wk, kv))]
        t = GGML_Q4_0
    tensors = [("blk.0.attn_q.weight", t, (hidden, heads * hd), data[0]),
               ("blk.0.attn_k.weight", t, (hidden, kv * hd), data[1]),
               ("token_embd.weight", GGML_F32, (hidden, 4), bytes(4 * hidden * 4))]
    p = tmp_path / "m.gguf"
    write(p, _llama_meta("llama", hidden, 1, heads, kv), tensors)
    with ti.Gguf(p) as g:
        if fmt == "bf16":
            np.testing.assert_array_equal(g.read(0), oracle.f32_to_bf16(wq))
            np.testing.assert_array_equal(g.read(1), oracle.f32_to_bf16(wk))
        else:
            np.testing.assert_array_equal(g.read(0, ti.DTYPE_Q4_0), _blocks(wq, "q4"))
            np.testing.assert_array_equal(g.read(1, ti.DTYPE_Q4_0), _blocks(wk, "q4"))
            assert g.model_desc().weight_format == ti.WFMT_Q4_0


def test_gemma_norms_back_to_w(tmp_path):
    w = oracle.bf16_to_f32(oracle.fill_bf16("n", (64,), 7, 0.05))
    tensors = [("blk.0.attn_norm.weight", GGML_F32, (64,), (w + 1.0).astype(np.float32).tobytes()),
               ("blk.0.attn_v.weight", GGML_F32, (64, 1), (w + 1.0).astype(np.float32).tobytes()),
               ("token_embd.weight", GGML_F32, (64, 2), bytes(512))]
    p = tmp_path / "m.gguf"
    write(p, _llama_meta("gemma", 64, 1, 4, 4), tensors)
    with ti.Gguf(p) as g:
        np.testing.assert_array_equal(g.read(0)[0], oracle.f32_to_bf16(w))          # norm: (1 + w) - 1
        np.testing.assert_array_equal(g.read(1)[0], oracle.f32_to_bf16(w + 1.0))    # other tensors as stored
        assert g.model_desc().arch == ti.ARCH_GEMMA


def test_rejects_bad_files(tmp_path):
    with pytest.raises(ti.TiError) as ei:
        ti.Gguf(tmp_path / "missing.gguf")
    assert ei.value.status == ti.TI_ERR_NOT_FOUND
    p = tmp_path / "bad.gguf"
    write(p, _llama_meta(), [], magic=b"GGML")
    with pytest.raises(ti.TiError) as ei:
        ti.Gguf(p)
    assert ei.value.status == ti.TI_ERR_INVALID and "magic" in str(ei.value)
    write(p, _llama_meta(), [], version=1)
    with pytest.raises(ti.TiError) as ei:
        ti.Gguf(p)
    assert ei.value.status == ti.TI_ERR_INVALID
    write(p, _llama_meta(), [("token_embd.weight", GGML_F32, (64, 2), bytes(512))])
    blob = open(p, "rb").read()
    for cut in (30, len(blob) // 2, len(blob) - 8):  # header, metadata / tensor table, tensor data
        open(p, "wb").write(blob[:cut])
        with pytest.raises(ti.TiError) as ei:
            ti.Gguf(p)
        assert ei.value.status == ti.TI_ERR_INVALID
    # a tensor offset near 2^64 must not wrap past the bounds check
    write(p, _llama_meta(), [("token_embd.weight", GGML_F32, (64, 2), bytes(512))])
    blob = bytearray(open(p, "rb").read())
    name = b"token_embd.weight"
    at = blob.index(name) + len(name) + 4 + 16 + 4  # n_dims u32, ne u64 x 2, type u32 -> offset u64
    blob[at:at + 8] = (2**64 - 64).to_bytes(8, "little")
    open(p, "wb").write(bytes(blob))
    with pytest.raises(ti.TiError) as ei:
        ti.Gguf(p)
    assert ei.value.status == ti.TI_ERR_INVALID
    write(p, _llama_meta("falcon"), [("token_embd.weight", GGML_F32, (64, 2), bytes(512))])
    with ti.Gguf(p) as g:
        with pytest.raises(ti.TiError) as ei:
            g.model_desc()
        assert ei.value.status == ti.TI_ERR_UNSUPPORTED
    write(p, _llama_meta(), [("token_embd.weight", GGML_F32, (64, 2), bytes(512)),
                             ("rope_freqs.weight", GGML_F32, (8,), bytes(32))])  # zero factors
    with ti.Gguf(p) as g:
        with pytest.raises(ti.TiError) as ei:
            g.rope_inv_freq(8)
        assert ei.value.status == ti.TI_ERR_INVALID


def _rope_table(hd, theta):
    out = np.empty(hd // 2, np.float32)
    oracle.lib().orc_rope_freqs(hd, theta, None, oracle.ptr(out))
    return out


def test_rope_factors(tmp_path):
    hd = 16
    p = tmp_path / "m.gguf"
    write(p, _llama_meta(), [("token_embd.weight", GGML_F32, (64, 2), bytes(512))])
    with ti.Gguf(p) as g:
        np.testing.assert_array_equal(g.rope_inv_freq(hd // 2), _rope_table(hd, 500000.0))
    factors = np.linspace(1.0, 8.0, hd // 2).astype(np.float32)  # per-dimension, as llama 3.1 files carry
    write(p, _llama_meta(), [("token_embd.weight", GGML_F32, (64, 2), bytes(512)),
                             ("rope_freqs.weight", GGML_F32, (hd // 2,), factors.tobytes())])
    with ti.Gguf(p) as g:
        np.testing.assert_array_equal(g.rope_inv_freq(hd // 2), _rope_table(hd, 500000.0) / factors)
        with pytest.raises(ti.TiError) as ei:
            g.rope_inv_freq(hd)  # the factor table fixes head_dim
        assert ei.value.status == ti.TI_ERR_INVALID


# ggml type -> (elements per block, bytes per block, byte offsets of its fp16 scale fields)
_BLOCKS = {3: (32, 20, (0, 2)), 6: (32, 22, (0,)), 7: (32, 24, (0, 2)), 10: (256, 84, (80, 82)),
           11: (256, 110, (108,)), 12: (256, 144, (0, 2)), 13: (256, 176, (0, 2)), 14: (256, 210, (208,))}


@pytest.mark.parametrize("gtype", sorted(_BLOCKS))
def test_block_types_decode_as_the_gguf_package(tmp_path, gtype):
    """Q4_1, Q5_0, Q5_1 and the k-quants Q2_K .. Q6_K: random blocks (finite fp16
    scales) read back as bf16 equal the gguf package's dequantisation (the
    llama.cpp project's Python reader) rounded to bf16."""
    quants = pytest.importorskip("gguf.quants")
    per, nbytes, halves = _BLOCKS[gtype]
    rows, cols = 3, 512
    rng = np.random.default_rng(gtype)
    raw = rng.integers(0, 256, size=(rows, cols // per, nbytes), dtype=np.uint8)
    for off in halves:
        h = (rng.uniform(0.001, 0.05, size=(rows, cols // per)) * rng.choice([-1, 1], size=(rows, cols // per)))
        raw[:, :, off:off + 2] = h.astype(np.float16).view(np.uint8).reshape(rows, cols // per, 2)
    raw = raw.reshape(rows, -1)
    want = quants.dequantize(raw, gtype).astype(np.float32).reshape(rows, cols)
    p = tmp_path / "blocks.gguf"
    write(p, _llama_meta(), [("blk.0.ffn_up.weight", gtype, (cols, rows), raw.tobytes())])
    with ti.Gguf(p) as g:
        inf = g.info(0)
        assert inf["type"] == gtype and inf["bytes"] == raw.nbytes
        got = g.read(0)
    np.testing.assert_array_equal(got, oracle.f32_to_bf16(want))


def test_files_written_by_the_gguf_package(tmp_path):
    """Interoperability: a file written by the llama.cpp project's GGUFWriter
    (its own metadata encoding, alignment padding and tensor table) reads back
    with the same metadata, tensor table and values, and gives the model
    description its metadata states."""
    gg = pytest.importorskip("gguf")
    from gguf import GGMLQuantizationType as Q
    from gguf import quants

    rng = np.random.default_rng(5)
    H, I, heads, kv, V = 256, 512, 4, 2, 1000
    p = tmp_path / "official.gguf"
    w = gg.GGUFWriter(str(p), "llama")
    w.add_block_count(1)
    w.add_context_length(2048)
    w.add_embedding_length(H)
    w.add_feed_forward_length(I)
    w.add_head_count(heads)
    w.add_head_count_kv(kv)
    w.add_layer_norm_rms_eps(1e-5)
    w.add_rope_freq_base(500000.0)
    w.add_string("general.name", "interop")
    w.add_array("tokenizer.ggml.tokens", ["<s>", "</s>", "x"])
    emb = rng.standard_normal((V, H)).astype(np.float32)
    norm = rng.standard_normal(H).astype(np.float32)
    up = rng.standard_normal((I, H)).astype(np.float32)
    down = rng.standard_normal((H, I)).astype(np.float32)
    gate = rng.standard_normal((I, H)).astype(np.float16)
    q4 = quants.quantize(up, Q.Q4_0)
    q8 = quants.quantize(down, Q.Q8_0)
    w.add_tensor("token_embd.weight", emb)
    w.add_tensor("output_norm.weight", norm)
    w.add_tensor("blk.0.ffn_up.weight", q4, raw_dtype=Q.Q4_0)
    w.add_tensor("blk.0.ffn_down.weight", q8, raw_dtype=Q.Q8_0)
    w.add_tensor("blk.0.ffn_gate.weight", gate)
    w.write_header_to_file()
    w.write_kv_data_to_file()
    w.write_tensors_to_file()
    w.close()
    with ti.Gguf(p) as g:
        assert len(g) == 5
        assert g.meta_str("general.architecture") == "llama" and g.meta_str("general.name") == "interop"
        assert g.meta_int("llama.block_count") == 1 and g.meta_int("llama.embedding_length") == H
        assert g.meta_array_len("tokenizer.ggml.tokens") == 3
        assert abs(g.meta_float("llama.rope.freq_base") - 500000.0) < 1e-3
        d = g.model_desc()
        assert (d.hidden, d.intermediate, d.n_heads, d.n_kv_heads, d.head_dim, d.vocab, d.n_layers) == \
            (H, I, heads, kv, H // heads, V, 1)
        info = {g.info(i)["name"]: g.info(i) for i in range(len(g))}
        assert info["blk.0.ffn_up.weight"]["type"] == ti.GGML_Q4_0 and info["blk.0.ffn_up.weight"]["dims"] == (H, I)
        assert info["blk.0.ffn_down.weight"]["type"] == ti.GGML_Q8_0
        assert info["blk.0.ffn_gate.weight"]["type"] == ti.GGML_F16
        checks = [("token_embd.weight", emb), ("output_norm.weight", norm[None, :]),
                  ("blk.0.ffn_up.weight", quants.dequantize(q4, Q.Q4_0)),
                  ("blk.0.ffn_down.weight", quants.dequantize(q8, Q.Q8_0)),
                  ("blk.0.ffn_gate.weight", gate.astype(np.float32))]
        for name, ref in checks:
            got = g.read(g.find(name))
            np.testing.assert_array_equal(got, oracle.f32_to_bf16(np.asarray(ref, np.float32)).reshape(got.shape))
        np.testing.assert_array_equal(g.read(g.find("blk.0.ffn_up.weight"), ti.DTYPE_Q4_0).reshape(q4.shape), q4)
        assert g.meta_array("tokenizer.ggml.tokens") == ["<s>", "</s>", "x"]


def test_metadata_arrays(tmp_path):
    """Elements of array metadata: strings (the vocabulary), integers of every
    width, floats; wrong element types and indices are errors."""
    import ctypes as C

    toks = ["<s>", "</s>", "héllo", "", "▁the"]
    meta = [m for m in _llama_meta() if m[0] != "tokenizer.ggml.tokens"] + list((
                              ("tokenizer.ggml.tokens", ARR, (STR, toks)),
                              ("tokenizer.ggml.scores", ARR, (F32, [0.0, -1.5, 2.25, 3.0, -4.0])),
                              ("tokenizer.ggml.token_type", ARR, (I32, [1, 3, 1, -1, 6])),
                              ("x.u8s", ARR, (U8, [0, 255, 7])), ("x.u64s", ARR, (U64, [1 << 40, 5])),
                              ("x.f64s", ARR, (F64, [0.5, -2.0])), ("x.bools", ARR, (BOOL, [1, 0]))))
    p = tmp_path / "arrays.gguf"
    write(p, meta, [("token_embd.weight", GGML_F32, (64, 2), bytes(512))])
    with ti.Gguf(p) as g:
        assert g.meta_array("tokenizer.ggml.tokens") == toks
        assert g.meta_array("tokenizer.ggml.scores") == [0.0, -1.5, 2.25, 3.0, -4.0]
        assert g.meta_array("tokenizer.ggml.token_type") == [1, 3, 1, -1, 6]
        assert g.meta_array("x.u8s") == [0, 255, 7] and g.meta_array("x.u64s") == [1 << 40, 5]
        assert g.meta_array("x.f64s") == [0.5, -2.0] and g.meta_array("x.bools") == [1, 0]
        v = C.c_int64()
        assert ti.lib().ti_gguf_meta_array_int(g.h, b"x.u8s", 3, C.byref(v)) == ti.TI_ERR_INVALID
        assert ti.lib().ti_gguf_meta_array_int(g.h, b"x.u8s", -1, C.byref(v)) == ti.TI_ERR_INVALID
        assert ti.lib().ti_gguf_meta_array_int(g.h, b"tokenizer.ggml.tokens", 0, C.byref(v)) == ti.TI_ERR_INVALID
        assert ti.lib().ti_gguf_meta_array_int(g.h, b"llama.block_count", 0, C.byref(v)) == ti.TI_ERR_NOT_FOUND


@pytest.mark.parametrize("arch", ["llama", "qwen2", "gemma"])
def test_tensor_names_match_the_gguf_package(tmp_path, arch):
    """The reader's llama.cpp -> reference (Hugging Face) name mapping against the
    llama.cpp project's own map (gguf.get_tensor_name_map) in the other direction:
    every tensor of a 3-layer model comes back under its reference name."""
    gg = pytest.importorskip("gguf")
    arch_enum = {"llama": gg.MODEL_ARCH.LLAMA, "qwen2": gg.MODEL_ARCH.QWEN2, "gemma": gg.MODEL_ARCH.GEMMA}[arch]
    names = ["model.embed_tokens.weight", "model.norm.weight", "lm_head.weight"]
    for i in range(3):
        p = f"model.layers.{i}."
        names += [p + n for n in ("self_attn.q_proj.weight", "self_attn.k_proj.weight", "self_attn.v_proj.weight",
                                  "self_attn.o_proj.weight", "mlp.gate_proj.weight", "mlp.up_proj.weight",
                                  "mlp.down_proj.weight", "input_layernorm.weight",
                                  "post_attention_layernorm.weight")]
        if arch == "qwen2":
            names += [p + n for n in ("self_attn.q_proj.bias", "self_attn.k_proj.bias", "self_attn.v_proj.bias")]
    m = gg.get_tensor_name_map(arch_enum, 3)
    pairs = [(n, m.get_name(n, try_suffixes=(".weight", ".bias"))) for n in names]
    # gemma ties the LM head to the embeddings: its files carry no output matrix
    assert [n for n, gn in pairs if gn is None] == (["lm_head.weight"] if arch == "gemma" else [])
    names = [n for n, gn in pairs if gn is not None]
    gnames = [gn for _, gn in pairs if gn is not None]
    p = tmp_path / "names.gguf"
    meta = [("general.architecture", STR, arch)]
    write(p, meta, [(g, GGML_F32, (32,), bytes(128)) for g in gnames])
    with ti.Gguf(p) as g:
        assert [g.reference_name(i) for i in range(len(g))] == names
