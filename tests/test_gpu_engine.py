"""Parity of the fused decode engine (libti_b200 C ABI) against the CPU oracle.

Every test builds the same seeded synthetic model on both sides, runs the
prompt, then decodes teacher-forced (both sides receive the oracle's greedy
token each step) and checks, per step and sequence: bf16 logits within
2e-2 max-abs relative, greedy ids equal (or a recorded near-tie), and for some
layers the KV pages bit-for-bit against the oracle's contiguous cache.
"""
import numpy as np
import pytest

import oracle
import ti_b200 as ti
from gpu_util import LOGIT_TOL, check_step, rel_err

pytestmark = pytest.mark.gpu

SMALL = dict(arch=ti.ARCH_LLAMA, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, intermediate=512,
             vocab=1000, rms_eps=1e-5, rope_theta=10000.0)


def _pair(kw, seed=0, std=0.02, max_batch=1, max_seq_len=256, **eopts):
    eng = ti.Engine(ti.model_desc(**kw), max_batch=max_batch, max_seq_len=max_seq_len, **eopts)
    eng.init_synthetic(seed, std)
    orc_kw = {k: v for k, v in kw.items()}
    m = oracle.Model(**orc_kw)
    m.init_synthetic(seed, std)
    return eng, m


def _run_parity(kw, prompt_lens, steps, seed=0, std=0.02, check_kv=True, max_seq_len=256):
    B = len(prompt_lens)
    eng, m = _pair(kw, seed, std, max_batch=B, max_seq_len=max_seq_len)
    V = kw["vocab"]
    sids, oseqs, feed = [], [], []
    ties = 0
    for b, n in enumerate(prompt_lens):
        ids = oracle.fill_ids(f"prompt{b}", n, seed + b, V)
        sid = eng.seq_create()
        nxt, lb = eng.prefill(sid, ids, logits=ti.LOGITS_BF16)
        os_ = m.new_seq(max(512, max_seq_len))
        _, lf = os_.forward(ids)
        ties += not check_step(nxt, lb, lf, f"prefill b{b}")
        sids.append(sid)
        oseqs.append(os_)
        feed.append(int(np.argmax(lf)))
    for step in range(steps):
        nxt, lb = eng.decode(sids, feed, logits=ti.LOGITS_BF16)
        new_feed = []
        for b in range(B):
            _, lf = oseqs[b].forward([feed[b]])
            ties += not check_step(int(nxt[b]), lb[b], lf, f"step {step} b{b}")
            new_feed.append(int(np.argmax(lf)))
        feed = new_feed
    if check_kv:
        for b in range(B):
            L = eng.seq_len(sids[b])
            assert L == prompt_lens[b] + steps
            for layer in (0, kw["n_layers"] - 1):
                for which in (0, 1):
                    g = oracle.bf16_to_f32(eng.seq_read_kv(sids[b], layer, which, L))
                    r = oracle.bf16_to_f32(oseqs[b].read_kv(layer, which, L))
                    assert rel_err(g, r) < LOGIT_TOL, (b, layer, which)
    eng.check()
    assert ties <= max(1, (steps + 1) * B // 10), f"{ties} near-tie flips"
    eng.close()


def test_synthetic_weights_bit_exact():
    eng = ti.Engine(ti.model_desc(**SMALL), max_batch=1, max_seq_len=64)
    eng.init_synthetic(7, 0.02)
    for name, shape in ti.tensor_names(eng.desc)[:6]:
        np.testing.assert_array_equal(eng.read_tensor(name, shape), oracle.fill_bf16(name, shape, 7, 0.02))
    eng.close()


def test_load_tensor_roundtrip_and_errors():
    eng = ti.Engine(ti.model_desc(**SMALL), max_batch=1, max_seq_len=64)
    w = oracle.fill_bf16("x", (1000, 256), 3)
    eng.load_tensor("model.embed_tokens.weight", w)
    np.testing.assert_array_equal(eng.read_tensor("model.embed_tokens.weight", (1000, 256)), w)
    with pytest.raises(ti.TiError) as ei:
        eng.load_tensor("model.layers.9.self_attn.q_proj.weight", w)
    assert ei.value.status == ti.TI_ERR_NOT_FOUND
    with pytest.raises(ti.TiError) as ei:
        eng.load_tensor("model.embed_tokens.weight", w[:10])
    assert ei.value.status == ti.TI_ERR_INVALID
    eng.close()


def test_llama_small_b1():
    _run_parity(SMALL, [7], steps=10)


def test_llama_small_ragged_batch():
    _run_parity(SMALL, [5, 17, 33], steps=6)


def test_qwen_bias():
    kw = dict(SMALL, arch=ti.ARCH_QWEN2, qkv_bias=1, rms_eps=1e-6, rope_theta=1e6)
    _run_parity(kw, [9], steps=6)


def test_gemma_ops():
    kw = dict(SMALL, arch=ti.ARCH_GEMMA, rms_eps=1e-6)
    _run_parity(kw, [6], steps=5)


def test_mistral_head_dim_override_and_window():
    # n_heads * head_dim != hidden; prompt longer than the window (prefill masks, decode does not)
    kw = dict(SMALL, arch=ti.ARCH_MISTRAL, n_heads=8, n_kv_heads=2, head_dim=64, sliding_window=8)
    _run_parity(kw, [20], steps=4)


def test_llama3_rope_scaling():
    kw = dict(SMALL, rope_theta=500000.0,
              rope_scaling=dict(factor=8.0, low_freq_factor=1.0, high_freq_factor=4.0, original_max_pos=64))
    _run_parity(kw, [40], steps=4)


def test_page_boundaries_long_context():
    # crosses many 16-token pages and several attention splits
    _run_parity(SMALL, [150], steps=20, check_kv=True)


def test_8b_layer_shapes_two_layers():
    # real Llama-3-8B projection shapes (K = 4096 / 14336, vocab 128256), 2 layers
    kw = dict(ti.PRESETS["llama3_8b"], n_layers=2)
    _run_parity(kw, [12], steps=3, check_kv=False)


def test_device_chain_matches_host_steps():
    eng, _ = _pair(SMALL, seed=4, max_batch=2, max_seqs=4)
    V = SMALL["vocab"]
    a, b = eng.seq_create(), eng.seq_create()
    p0 = oracle.fill_ids("pa", 5, 1, V)
    p1 = oracle.fill_ids("pb", 9, 2, V)
    n0, n1 = eng.prefill(a, p0), eng.prefill(b, p1)
    # host path: 12 greedy steps
    host = []
    feed = [n0, n1]
    for _ in range(12):
        feed = list(eng.decode([a, b], feed))
        host.append(feed)
    # device chain from the same state
    c, d = eng.seq_create(), eng.seq_create()
    eng.prefill(c, p0)
    eng.prefill(d, p1)
    eng.seq_reserve(c, 5 + 13)
    eng.seq_reserve(d, 9 + 13)
    eng.bind([c, d], [n0, n1])
    for _ in range(12):
        eng.decode_device()
    last = eng.unbind(12)
    assert list(last) == list(host[-1])
    assert eng.seq_len(c) == 5 + 12 and eng.seq_len(d) == 9 + 12
    eng.close()


def test_deterministic_bits():
    outs = []
    for _ in range(2):
        eng, _ = _pair(SMALL, seed=5)
        s = eng.seq_create()
        eng.prefill(s, oracle.fill_ids("p", 11, 5, SMALL["vocab"]))
        _, lb = eng.decode([s], [3], logits=ti.LOGITS_BF16)
        outs.append(lb.copy())
        eng.close()
    np.testing.assert_array_equal(outs[0], outs[1])


def test_errors_are_reported_not_launched():
    eng, _ = _pair(SMALL, max_seq_len=20)
    s = eng.seq_create()
    with pytest.raises(ti.TiError) as ei:
        eng.decode([s], [SMALL["vocab"]])  # token out of range
    assert ei.value.status == ti.TI_ERR_INVALID
    with pytest.raises(ti.TiError) as ei:
        eng.decode([s + 1], [1])  # unknown sequence
    assert ei.value.status == ti.TI_ERR_STATE
    eng.prefill(s, np.arange(20) % SMALL["vocab"])
    with pytest.raises(ti.TiError) as ei:  # KV cache full (the reference overflows silently)
        eng.decode([s], [1])
    assert ei.value.status == ti.TI_ERR_STATE
    eng.check()
    eng.close()
