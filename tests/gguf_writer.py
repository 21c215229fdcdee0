"""Minimal GGUF v3 writer for the tests (the published container layout):

    "GGUF" u32 version, u64 n_tensors, u64 n_kv
    n_kv x (string key, u32 value type, value)       arrays: u32 elem type, u64 n, elems
    n_tensors x (string name, u32 n_dims, u64 ne[n_dims], u32 ggml type, u64 offset)
    zero padding to `alignment`, tensor data (each tensor aligned)

strings are u64 length + UTF-8 bytes; ne[0] is the innermost dimension.
Also: the llama.cpp tensor names of the reference's, and the q/k row order
llama.cpp's converter writes for llama-architecture checkpoints.
"""
import struct

import numpy as np

U8, I8, U16, I16, U32, I32, F32, BOOL, STR, ARR, U64, I64, F64 = range(13)
_SCALAR = {U8: "<B", I8: "<b", U16: "<H", I16: "<h", U32: "<I", I32: "<i", F32: "<f", BOOL: "<B", U64: "<Q",
           I64: "<q", F64: "<d"}

GGML_F32, GGML_F16, GGML_Q4_0, GGML_Q8_0, GGML_BF16 = 0, 1, 2, 8, 30


def _str(x):
    b = x.encode()
    return struct.pack("<Q", len(b)) + b


def _value(t, v):
    if t == STR:
        return _str(v)
    if t == ARR:
        et, items = v
        out = struct.pack("<IQ", et, len(items))
        for it in items:
            out += _value(et, it)
        return out
    return struct.pack(_SCALAR[t], v)


def write(path, meta, tensors, alignment=32, version=3, magic=b"GGUF"):
    """meta: [(key, type, value)] (arrays: value = (elem_type, [items]));
    tensors: [(name, ggml_type, ne tuple, raw bytes)]"""
    head = magic + struct.pack("<IQQ", version, len(tensors), len(meta))
    for k, t, v in meta:
        head += _str(k) + struct.pack("<I", t) + _value(t, v)
    offs, off = [], 0
    for _, _, _, data in tensors:
        offs.append(off)
        off += len(data)
        off = (off + alignment - 1) // alignment * alignment
    for (name, t, ne, _), o in zip(tensors, offs):
        head += _str(name) + struct.pack("<I", len(ne)) + b"".join(struct.pack("<Q", n) for n in ne)
        head += struct.pack("<IQ", t, o)
    pad = (-len(head)) % alignment
    blob = bytearray(head + b"\0" * pad)
    for (_, _, _, data), o in zip(tensors, offs):
        blob += b"\0" * (len(head) + pad + o - len(blob))
        blob += data
    with open(path, "wb") as f:
        f.write(bytes(blob))


# llama.cpp tensor names <- the reference's (LlamaModel::load / QwenModel::load names)
_TOP = {"model.embed_tokens.weight": "token_embd.weight", "model.norm.weight": "output_norm.weight",
        "lm_head.weight": "output.weight"}
_LAYER = {"input_layernorm.weight": "attn_norm.weight", "post_attention_layernorm.weight": "ffn_norm.weight",
          "self_attn.q_proj.weight": "attn_q.weight", "self_attn.k_proj.weight": "attn_k.weight",
          "self_attn.v_proj.weight": "attn_v.weight", "self_attn.o_proj.weight": "attn_output.weight",
          "self_attn.q_proj.bias": "attn_q.bias", "self_attn.k_proj.bias": "attn_k.bias",
          "self_attn.v_proj.bias": "attn_v.bias", "mlp.gate_proj.weight": "ffn_gate.weight",
          "mlp.up_proj.weight": "ffn_up.weight", "mlp.down_proj.weight": "ffn_down.weight"}


def gguf_name(ref):
    if ref in _TOP:
        return _TOP[ref]
    parts = ref.split(".")
    assert parts[0] == "model" and parts[1] == "layers", ref
    return f"blk.{parts[2]}." + _LAYER[".".join(parts[3:])]


def permute_rows(rows, n_heads):
    """the q/k row order of llama-architecture GGUF files: row t*hd/2 + j of a
    head (reference / HF order) is stored at row 2j + t (rows: [n, ...] array)"""
    n = rows.shape[0]
    hd = n // n_heads
    return rows.reshape(n_heads, 2, hd // 2, *rows.shape[1:]).swapaxes(1, 2).reshape(rows.shape)
