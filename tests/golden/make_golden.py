"""Generate the golden logits that pin the CPU oracle to the reference.

Runs on a GPU box:  python tests/golden/make_golden.py [out_dir]

For each case below it writes a synthetic checkpoint (config.json +
model.safetensors, and for the adapter case adapter.json + adapter.safetensors)
with the seeded generator the oracle and the engine share, runs the reference's
own model code on it (oracle/_ref/libref.so: the reference's unchanged
backend/parser/models/adapter sources compiled for sm_100a, driven through
Model::forward: the prompt, then one fed token per step), and stores the
reference's last-row logits as fp32 in <case>.npz next to this file.  The same
npz records the oracle's error against them.  tests/test_golden.py re-derives
the same inputs on the CPU and checks the oracle against these vectors.
"""
import ctypes as C
import json
import os
import struct
import sys
import tempfile

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(HERE))
sys.path.insert(0, ROOT)
sys.path.insert(0, os.path.join(ROOT, "tensor-inference_b200"))

import oracle  # noqa: E402

BASE = dict(hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, intermediate=512, vocab=1000,
            rms_eps=1e-5, rope_theta=10000.0)
CASES = {
    "llama_small": dict(BASE, arch=0),
    "llama_rope_scaled": dict(BASE, arch=0, rope_theta=500000.0,
                              rope_scaling=dict(factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0,
                                                original_max_pos=64)),
    "qwen2_bias": dict(BASE, arch=1, qkv_bias=1, rms_eps=1e-6, rope_theta=1000000.0),
    "qwen2_bias_lora": dict(BASE, arch=1, qkv_bias=1, rms_eps=1e-6, rope_theta=1000000.0,
                            lora=dict(rank=8, alpha=16.0, mask=0x0F, std_a=0.05, std_b=0.05)),
    "gemma": dict(BASE, arch=2, rms_eps=1e-6),
    "mistral_window": dict(BASE, arch=3, n_heads=8, head_dim=64, sliding_window=8),
}
SEED, STD = 7, 0.05
N_PROMPT, N_STEPS, MAX_SEQ = 20, 6, 64
PROJ = ["self_attn.q_proj", "self_attn.k_proj", "self_attn.v_proj", "self_attn.o_proj", "mlp.gate_proj",
        "mlp.up_proj", "mlp.down_proj"]


def tensor_shapes(kw):
    H, I, hd, V = kw["hidden"], kw["intermediate"], kw["head_dim"], kw["vocab"]
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


def lora_shapes(kw, mask):
    H, I, hd = kw["hidden"], kw["intermediate"], kw["head_dim"]
    QW, KW = kw["n_heads"] * hd, kw["n_kv_heads"] * hd
    io = [(QW, H), (KW, H), (KW, H), (H, QW), (I, H), (I, H), (H, I)]
    out = {}
    for i in range(kw["n_layers"]):
        for p, (o, inn) in enumerate(io):
            if mask & (1 << p):
                out[f"layers.{i}.{PROJ[p]}.lora_A"] = ("A", inn)
                out[f"layers.{i}.{PROJ[p]}.lora_B"] = ("B", o)
    return out


def write_safetensors(path, tensors):
    """tensors: name -> uint16 array (bf16 bits)"""
    header, off = {}, 0
    for name, a in tensors.items():
        header[name] = {"dtype": "BF16", "shape": list(a.shape), "data_offsets": [off, off + a.nbytes]}
        off += a.nbytes
    hb = json.dumps(header).encode()
    hb += b" " * ((8 - len(hb) % 8) % 8)
    with open(path, "wb") as f:
        f.write(struct.pack("<Q", len(hb)))
        f.write(hb)
        for a in tensors.values():
            f.write(np.ascontiguousarray(a).tobytes())


def write_config(d, kw):
    arch = kw["arch"]
    names = {0: ("LlamaForCausalLM", "llama"), 1: ("Qwen2ForCausalLM", "qwen2"), 2: ("GemmaForCausalLM", "gemma"),
             3: ("MistralForCausalLM", "mistral")}[arch]
    cfg = {"architectures": [names[0]], "model_type": names[1], "hidden_size": kw["hidden"],
           "intermediate_size": kw["intermediate"], "num_hidden_layers": kw["n_layers"],
           "num_attention_heads": kw["n_heads"], "num_key_value_heads": kw["n_kv_heads"], "vocab_size": kw["vocab"],
           "rms_norm_eps": kw["rms_eps"], "rope_theta": kw["rope_theta"], "max_position_embeddings": 4096,
           "bos_token_id": 1, "eos_token_id": 2, "tie_word_embeddings": False, "torch_dtype": "bfloat16"}
    if arch == 3:
        cfg["head_dim"] = kw["head_dim"]
        cfg["sliding_window"] = kw["sliding_window"]
    rs = kw.get("rope_scaling")
    if rs:
        cfg["rope_scaling"] = {"rope_type": "llama3", "factor": rs["factor"], "low_freq_factor": rs["low_freq_factor"],
                               "high_freq_factor": rs["high_freq_factor"],
                               "original_max_position_embeddings": rs["original_max_pos"]}
    with open(os.path.join(d, "config.json"), "w") as f:
        json.dump(cfg, f)


def case_inputs(kw):
    prompt = oracle.fill_ids("golden_prompt", N_PROMPT, SEED, kw["vocab"])
    feed = oracle.fill_ids("golden_feed", N_STEPS, SEED, kw["vocab"])
    return prompt, feed


def oracle_logits(kw):
    """the oracle's fp32 last-row logits for the prompt and each fed token"""
    okw = {k: v for k, v in kw.items() if k != "lora"}
    m = oracle.Model(**okw)
    m.init_synthetic(SEED, STD)
    ad = -1
    if kw.get("lora"):
        L = kw["lora"]
        m.add_adapter(0, L["rank"], L["alpha"], L["mask"], SEED, L["std_a"], L["std_b"])
        ad = 0
    prompt, feed = case_inputs(kw)
    s = m.new_seq(MAX_SEQ)
    rows = [s.forward(prompt, adapter=ad)[1]]
    for t in feed:
        rows.append(s.forward([int(t)], adapter=ad)[1])
    return np.stack(rows)


def build_case(d, kw):
    tensors = {name: oracle.fill_bf16(name, shape, SEED, STD) for name, shape in tensor_shapes(kw).items()}
    write_safetensors(os.path.join(d, "model.safetensors"), tensors)
    write_config(d, kw)
    adir = None
    if kw.get("lora"):
        L = kw["lora"]
        adir = os.path.join(d, "adapter")
        os.makedirs(adir)
        at = {}
        for name, (which, dim) in lora_shapes(kw, L["mask"]).items():
            shape = (L["rank"], dim) if which == "A" else (dim, L["rank"])
            at[name] = oracle.fill_bf16(name, shape, SEED, L["std_a"] if which == "A" else L["std_b"])
        write_safetensors(os.path.join(adir, "adapter.safetensors"), at)
        meta = {"architecture": "qwen2", "rank": L["rank"], "alpha": L["alpha"], "target_begin": 0,
                "target_end": kw["n_layers"] - 1, "inject_q": bool(L["mask"] & 1), "inject_k": bool(L["mask"] & 2),
                "inject_v": bool(L["mask"] & 4), "inject_o": bool(L["mask"] & 8),
                "inject_up": bool(L["mask"] & 48), "inject_down": bool(L["mask"] & 64), "domain": "golden"}
        with open(os.path.join(adir, "adapter.json"), "w") as f:
            json.dump(meta, f)
    return adir


def main():
    out_dir = sys.argv[1] if len(sys.argv) > 1 else HERE
    ref = C.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref.so"))
    ref.ref_run.restype = C.c_int
    ref.ref_run.argtypes = [C.c_char_p, C.c_int, C.c_char_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int,
                            C.c_void_p, C.c_int, C.c_char_p, C.c_int]
    for name, kw in CASES.items():
        with tempfile.TemporaryDirectory() as d:
            adir = build_case(d, kw)
            prompt, feed = case_inputs(kw)
            V = kw["vocab"]
            logits = np.zeros((N_STEPS + 1, V), np.float32)
            err = C.create_string_buffer(512)
            rc = ref.ref_run(d.encode(), kw["arch"], adir.encode() if adir else None, prompt.ctypes.data, len(prompt),
                             feed.ctypes.data, len(feed), MAX_SEQ, logits.ctypes.data, V, err, 512)
            if rc != 0:
                raise RuntimeError(f"{name}: reference failed: {err.value.decode()}")
        orc = oracle_logits(kw)
        rel = [float(np.abs(orc[i] - logits[i]).max() / np.abs(logits[i]).max()) for i in range(len(logits))]
        np.savez_compressed(os.path.join(out_dir, f"{name}.npz"), kw=json.dumps(kw), seed=SEED, std=STD,
                            prompt=prompt, feed=feed, ref_logits=logits, oracle_rel_err=np.array(rel))
        print(f"{name}: oracle vs reference max rel err {max(rel):.3e}", flush=True)


if __name__ == "__main__":
    main()
