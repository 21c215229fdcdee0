"""LoRA on the engine (qwen_adapter_model.cpp:22-193 semantics:
delta = bf16(bf16(bf16(x A^T) B^T) * alpha/rank) added after the base
projection and bias) against the oracle, including several adapters in one
batch (per-sequence segmented gather), ranks below the engine's padded rank,
and the pinned-host -> HBM async fetch."""
import numpy as np
import pytest

import oracle
import ti_b200 as ti
from gpu_util import check_step

pytestmark = pytest.mark.gpu

QWEN = dict(arch=ti.ARCH_QWEN2, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, intermediate=512,
            vocab=1000, rms_eps=1e-6, rope_theta=1e6, qkv_bias=1)
ALL = 0x7F


def _setup(kw, adapters, max_batch, seed=3, max_rank=8, mask=ALL):
    """adapters: list of (rank, alpha, mask, seed, std_a, std_b)"""
    eng = ti.Engine(ti.model_desc(**kw), max_batch=max_batch, max_seqs=max_batch + 2, max_seq_len=128,
                    max_adapters=len(adapters) + 1, max_lora_rank=max_rank, lora_proj_mask=mask)
    eng.init_synthetic(seed, 0.03)
    m = oracle.Model(**kw)
    m.init_synthetic(seed, 0.03)
    ids = []
    for slot, (rank, alpha, amask, aseed, sa, sb) in enumerate(adapters):
        a = eng.adapter_create(rank, alpha, amask)
        eng.adapter_init_synthetic(a, aseed, sa, sb)
        m.add_adapter(a, rank, alpha, amask, aseed, sa, sb)
        ids.append(a)
    return eng, m, ids


def _parity(eng, m, prompts, ads, steps):
    sids, oseqs, feed = [], [], []
    flips = 0
    for b, p in enumerate(prompts):
        sid = eng.seq_create()
        nxt, lb = eng.prefill(sid, p, adapter=ads[b], logits=ti.LOGITS_BF16)
        s = m.new_seq(256)
        _, lf = s.forward(p, adapter=ads[b])
        flips += not check_step(nxt, lb, lf, f"prefill {b}")
        sids.append(sid)
        oseqs.append(s)
        feed.append(int(np.argmax(lf)))
    for step in range(steps):
        nxt, lb = eng.decode(sids, feed, adapters=ads, logits=ti.LOGITS_BF16)
        nf = []
        for b in range(len(sids)):
            _, lf = oseqs[b].forward([feed[b]], adapter=ads[b])
            flips += not check_step(int(nxt[b]), lb[b], lf, f"step {step} b{b}")
            nf.append(int(np.argmax(lf)))
        feed = nf
    assert flips <= 1
    eng.check()


def test_single_adapter_qkvo():
    eng, m, ids = _setup(QWEN, [(8, 16.0, 0x0F, 11, 0.05, 0.05)], 1)
    _parity(eng, m, [oracle.fill_ids("p", 9, 1, 1000)], [ids[0]], steps=5)
    eng.close()


def test_multi_adapter_batch_mixed_ranks():
    ads = [(8, 8.0, ALL, 21, 0.05, 0.05), (4, 16.0, ALL, 22, 0.05, 0.05)]
    eng, m, ids = _setup(QWEN, ads, 3)
    prompts = [oracle.fill_ids(f"p{b}", n, b, 1000) for b, n in enumerate((7, 12, 5))]
    _parity(eng, m, prompts, [ids[0], ids[1], -1], steps=5)
    eng.close()


def test_llama_8b_shapes_rank16():
    kw = dict(ti.PRESETS["llama3_8b"], n_layers=2)
    eng, m, ids = _setup(kw, [(16, 32.0, 0x0F, 5, 0.02, 0.001)], 1, max_rank=16, mask=0x0F)
    _parity(eng, m, [oracle.fill_ids("p", 6, 2, kw["vocab"])], [ids[0]], steps=2)
    eng.close()


def test_zero_b_is_base_bit_exact():
    eng, _, ids = _setup(QWEN, [(8, 16.0, ALL, 31, 0.05, 0.0)], 2)
    p = oracle.fill_ids("p", 8, 4, 1000)
    a, b = eng.seq_create(), eng.seq_create()
    eng.prefill(a, p, adapter=ids[0])
    eng.prefill(b, p)
    _, lb = eng.decode([a, b], [5, 5], adapters=[ids[0], -1], logits=ti.LOGITS_BF16)
    np.testing.assert_array_equal(lb[0], lb[1])
    eng.close()


def test_load_tensor_matches_synthetic_and_flat_layout():
    eng, _, ids = _setup(QWEN, [(8, 16.0, 0x0F, 41, 0.05, 0.05)], 1)
    b = eng.adapter_create(8, 16.0, 0x0F)
    for i in range(QWEN["n_layers"]):
        for p, out in (("q_proj", 256), ("k_proj", 128), ("v_proj", 128), ("o_proj", 256)):
            inn = 256
            na, nb = f"layers.{i}.self_attn.{p}.lora_A", f"layers.{i}.self_attn.{p}.lora_B"
            eng.adapter_load_tensor(b, na, oracle.fill_bf16(na, (8 * inn,), 41, 0.05))  # flat 1-D, as exported
            eng.adapter_load_tensor(b, nb, oracle.fill_bf16(nb, (out, 8), 41, 0.05))
    with pytest.raises(ti.TiError) as ei:
        eng.adapter_load_tensor(b, "layers.0.mlp.down_proj.lora_A", np.zeros(8 * 512, np.uint16))
    assert ei.value.status == ti.TI_ERR_INVALID  # not injected by this adapter
    p = oracle.fill_ids("p", 6, 5, 1000)
    s1, s2 = eng.seq_create(), eng.seq_create()
    eng.prefill(s1, p, adapter=ids[0])
    eng.prefill(s2, p, adapter=b)
    _, l1 = eng.decode([s1], [7], adapters=[ids[0]], logits=ti.LOGITS_BF16)
    _, l2 = eng.decode([s2], [7], adapters=[b], logits=ti.LOGITS_BF16)
    np.testing.assert_array_equal(l1, l2)
    eng.close()


def test_evict_and_async_prefetch_roundtrip():
    eng, _, ids = _setup(QWEN, [(8, 16.0, ALL, 51, 0.05, 0.05)], 1)
    a = ids[0]
    p = oracle.fill_ids("p", 6, 6, 1000)
    s = eng.seq_create()
    eng.prefill(s, p, adapter=a)
    _, before = eng.decode([s], [9], adapters=[a], logits=ti.LOGITS_BF16)
    eng.adapter_stage_host(a)
    eng.adapter_evict(a)
    assert not eng.adapter_is_resident(a)
    with pytest.raises(ti.TiError) as ei:
        eng.decode([s], [9], adapters=[a])
    assert ei.value.status == ti.TI_ERR_STATE
    eng.adapter_prefetch_async(a)  # pinned host -> HBM on the side stream
    s2 = eng.seq_create()
    eng.prefill(s2, p, adapter=a)  # the step waits on the copy's event
    _, after = eng.decode([s2], [9], adapters=[a], logits=ti.LOGITS_BF16)
    np.testing.assert_array_equal(before, after)
    assert eng.adapter_is_resident(a)
    eng.close()


def test_multi_adapter_tensor_core_batch():
    # 12 tokens: every projection on the tcgen05 GEMM, LoRA expansion in its epilogue
    # (bias store, residual, and both halves of the gate|up pair), adapters mixed per token
    ads = [(8, 8.0, ALL, 41, 0.05, 0.05), (4, 16.0, ALL, 42, 0.05, 0.05), (8, 16.0, 0x0F, 43, 0.05, 0.05)]
    eng, m, ids = _setup(QWEN, ads, 12)
    prompts = [oracle.fill_ids(f"tcp{b}", 3 + b % 5, b, 1000) for b in range(12)]
    per_tok = [ids[b % 3] if b % 4 != 3 else -1 for b in range(12)]
    _parity(eng, m, prompts, per_tok, steps=3)
    eng.close()
