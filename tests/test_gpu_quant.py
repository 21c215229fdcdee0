"""GGUF Q4_0 / Q8_0 weights on the device against the CPU oracle.

The device quantiser must produce the oracle's GGUF blocks bit for bit (the
oracle restates ggml's quantize_row_q4_0_ref / q8_0_ref); GGUF blocks loaded
directly must round-trip; decode through the dequantising weight-streaming
GEMV (and, for batches of 8+ tokens, the tcgen05 GEMM with in-kernel
dequantisation) must match the oracle's dequantise-then-fp32-dot path within 5e-2
max-abs relative for Q4_0 (the tolerance the spec states for Q4_0) and 2e-2
for Q8_0, with greedy ids equal up to recorded near-ties."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle
import ti_b200 as ti
from gpu_util import rel_err

pytestmark = pytest.mark.gpu

SMALL = dict(arch=ti.ARCH_LLAMA, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, intermediate=512,
             vocab=1000, rms_eps=1e-5, rope_theta=10000.0)
TOL = {ti.WFMT_Q4_0: 5e-2, ti.WFMT_Q8_0: 2e-2}
BLOCK = {ti.WFMT_Q4_0: 18, ti.WFMT_Q8_0: 34}


def oracle_blocks(wf, name, shape, seed, std):
    x = oracle.bf16_to_f32(oracle.fill_bf16(name, shape, seed, std)).astype(np.float32)
    out = np.zeros(x.size // 32 * BLOCK[wf], np.uint8)
    fn = oracle.lib().orc_q4_0_quantize if wf == ti.WFMT_Q4_0 else oracle.lib().orc_q8_0_quantize
    fn(oracle.ptr(x), x.size, oracle.ptr(out))
    return out


def read_blocks(eng, name, rows, cols, wf):
    out = np.zeros(rows * cols // 32 * BLOCK[wf], np.uint8)
    ti.check(ti.lib().ti_engine_read_tensor(eng.h, name.encode(), out.ctypes.data_as(C.c_void_p), out.nbytes))
    return out


@pytest.mark.parametrize("wf", [ti.WFMT_Q4_0, ti.WFMT_Q8_0])
def test_device_quantiser_is_bit_exact(wf):
    kw = dict(SMALL, weight_format=wf)
    eng = ti.Engine(ti.model_desc(**kw), max_batch=1, max_seq_len=64)
    eng.init_synthetic(5, 0.02)
    H, I = kw["hidden"], kw["intermediate"]
    for name, shape in (("model.layers.0.mlp.up_proj.weight", (I, H)), ("model.layers.1.mlp.down_proj.weight", (H, I)),
                        ("model.layers.1.self_attn.k_proj.weight", (2 * 64, H))):
        got = read_blocks(eng, name, shape[0], shape[1], wf)
        ref = oracle_blocks(wf, name, shape, 5, 0.02)
        assert np.array_equal(got, ref), name
    eng.close()


@pytest.mark.parametrize("wf", [ti.WFMT_Q4_0, ti.WFMT_Q8_0])
def test_gguf_blocks_load_and_read_back(wf):
    kw = dict(SMALL, weight_format=wf)
    eng = ti.Engine(ti.model_desc(**kw), max_batch=1, max_seq_len=64)
    name, shape = "model.layers.0.self_attn.o_proj.weight", (256, 256)
    blocks = oracle_blocks(wf, "some other tensor", shape, 9, 0.5)
    dt = ti.DTYPE_Q4_0 if wf == ti.WFMT_Q4_0 else ti.DTYPE_Q8_0
    ti.check(ti.lib().ti_engine_load_tensor(eng.h, name.encode(), dt, blocks.ctypes.data_as(C.c_void_p), blocks.nbytes))
    assert np.array_equal(read_blocks(eng, name, shape[0], shape[1], wf), blocks)
    # wrong block type / size are rejected before any copy
    other = ti.DTYPE_Q8_0 if dt == ti.DTYPE_Q4_0 else ti.DTYPE_Q4_0
    assert ti.lib().ti_engine_load_tensor(eng.h, name.encode(), other, blocks.ctypes.data_as(C.c_void_p),
                                          blocks.nbytes) != 0
    assert ti.lib().ti_engine_load_tensor(eng.h, name.encode(), dt, blocks.ctypes.data_as(C.c_void_p),
                                          blocks.nbytes - 1) != 0
    eng.close()


def _parity(kw, prompt_lens, steps, seed=0, std=0.02):
    wf = kw["weight_format"]
    B = len(prompt_lens)
    eng = ti.Engine(ti.model_desc(**kw), max_batch=B, max_seqs=B, max_seq_len=128)
    eng.init_synthetic(seed, std)
    m = oracle.Model(**kw)
    m.init_synthetic(seed, std)
    V = kw["vocab"]
    sids, oseqs, feed = [], [], []
    for b, n in enumerate(prompt_lens):
        ids = oracle.fill_ids(f"qp{b}", n, seed + b, V)
        sid = eng.seq_create()
        nxt, lb = eng.prefill(sid, ids, logits=ti.LOGITS_BF16)
        os_ = m.new_seq(128)
        _, lf = os_.forward(ids)
        assert rel_err(oracle.bf16_to_f32(lb), lf) <= TOL[wf]
        sids.append(sid)
        oseqs.append(os_)
        feed.append(int(np.argmax(lf)))
    flips = 0
    for step in range(steps):
        nxt, lb = eng.decode(sids, feed, logits=ti.LOGITS_BF16)
        new_feed = []
        for b in range(B):
            _, lf = oseqs[b].forward([feed[b]])
            g = oracle.bf16_to_f32(lb[b])
            err = rel_err(g, lf)
            assert err <= TOL[wf], (step, b, err)
            if int(nxt[b]) != int(np.argmax(lf)):
                s = np.sort(lf)
                assert s[-1] - s[-2] <= TOL[wf] * np.abs(lf).max(), (step, b)  # a near-tie, not a wrong id
                flips += 1
            new_feed.append(int(np.argmax(lf)))
        feed = new_feed
    eng.check()
    assert flips <= max(1, steps * B // 10)
    eng.close()


@pytest.mark.parametrize("wf", [ti.WFMT_Q4_0, ti.WFMT_Q8_0])
def test_quantised_decode_b1(wf):
    _parity(dict(SMALL, weight_format=wf), [7], steps=6)


@pytest.mark.parametrize("wf", [ti.WFMT_Q4_0, ti.WFMT_Q8_0])
def test_quantised_decode_batched(wf):
    # 3 tokens (GEMV, shared-memory activations) and 19 tokens (the tcgen05 GEMM)
    _parity(dict(SMALL, weight_format=wf), [4, 9, 2], steps=3)
    _parity(dict(SMALL, weight_format=wf), [2 + b % 5 for b in range(19)], steps=2)


@pytest.mark.parametrize("wf", [ti.WFMT_Q4_0, ti.WFMT_Q8_0])
def test_quantised_gemv_eight_tokens_qwen7b_shapes(wf, monkeypatch):
    # TI_TC_MIN_BATCH=9 keeps a batch of 8 on the GEMV (its 8-token instance; the
    # 18944-column down projection in launches of 2 tokens): the alternative to the
    # tcgen05 path for a quantised batch of 8
    monkeypatch.setenv("TI_TC_MIN_BATCH", "9")
    kw = dict(ti.PRESETS["qwen25_7b"], n_layers=2, weight_format=wf)
    _parity(kw, [2 + b % 3 for b in range(8)], steps=2)


def test_q4_qwen7b_shapes_bias():
    # Qwen2.5-7B projection shapes (hidden 3584, intermediate 18944: the packed-activation path), 2 layers
    kw = dict(ti.PRESETS["qwen25_7b"], n_layers=2, weight_format=ti.WFMT_Q4_0)
    _parity(kw, [5], steps=2)


@pytest.mark.parametrize("wf", [ti.WFMT_Q4_0, ti.WFMT_Q8_0])
def test_quantised_tensor_core_batch_qwen7b_shapes(wf):
    # 12 tokens: every projection on the tcgen05 GEMM with in-kernel dequantisation
    # (the dequantised weight is rounded to bf16 for the bf16 x bf16 MMA: <= 2^-9 relative)
    kw = dict(ti.PRESETS["qwen25_7b"], n_layers=2, weight_format=wf)
    _parity(kw, [2 + b % 3 for b in range(12)], steps=2)


@pytest.mark.parametrize("wf", [ti.WFMT_Q4_0, ti.WFMT_Q8_0])
@pytest.mark.parametrize("B", [64, 100, 136])
def test_quantised_tensor_core_wide_batches(wf, B):
    # 64 / 100 tokens: the dequantised operands in TMEM (3 and 2 buffers above the
    # accumulators); 136 tokens: past TMEM's room, the shared-memory operand buffers
    _parity(dict(SMALL, weight_format=wf), [1 + b % 4 for b in range(B)], steps=1)
