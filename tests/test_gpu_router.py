"""The router's pool drives real adapter residency (ti_router_prepare ->
ti_adapter_stage_host / evict / prefetch_async): three sequences on three
adapters decode in turn under a budget of two resident adapters, so adapters
are evicted and fetched back from pinned host memory every few steps; the
logits must equal an engine that keeps every adapter resident."""
import numpy as np
import pytest

import oracle
import ti_b200 as ti

pytestmark = pytest.mark.gpu

QWEN = dict(arch=ti.ARCH_QWEN2, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, intermediate=512,
            vocab=1000, rms_eps=1e-6, rope_theta=1e6, qkv_bias=1)


def _engine():
    eng = ti.Engine(ti.model_desc(**QWEN), max_batch=2, max_seqs=4, max_seq_len=128, max_adapters=3,
                    max_lora_rank=8, lora_proj_mask=0x7F)
    eng.init_synthetic(5, 0.03)
    ids = []
    for i in range(3):
        a = eng.adapter_create(8, 16.0, 0x7F)
        eng.adapter_init_synthetic(a, 40 + i, 0.05, 0.05)
        ids.append(a)
    return eng, ids


def test_router_residency_is_transparent():
    plain, ids = _engine()
    routed, ids2 = _engine()
    assert ids == ids2
    r = ti.Router(routed, max_resident=2, prefetch_after=1, switch_after=1)
    prompts = [oracle.fill_ids(f"r{b}", 4 + b, b, QWEN["vocab"]) for b in range(3)]
    out = {}
    for name, eng in (("plain", plain), ("routed", routed)):
        sids, feed, logs = [], [], []
        for b, p in enumerate(prompts):
            if eng is routed:
                r.prepare([ids[b]])
            s = eng.seq_create()
            nxt, lb = eng.prefill(s, p, adapter=ids[b], logits=ti.LOGITS_BF16)
            sids.append(s)
            feed.append(int(nxt))
            logs.append(lb)
        for step in range(6):
            b = step % 3                          # one sequence (one adapter) per step
            if eng is routed:
                r.prepare([ids[b]])
            nxt, lb = eng.decode([sids[b]], [feed[b]], adapters=[ids[b]], logits=ti.LOGITS_BF16)
            feed[b] = int(nxt[0])
            logs.append(lb)
        eng.check()
        out[name] = logs
    for a, b in zip(out["plain"], out["routed"]):
        np.testing.assert_array_equal(a, b)
    s = r.stats()
    assert s["evictions"] >= 3 and s["prefetches"] >= 3
    assert len(r.resident()) <= 2
    r.close()
    plain.close()
    routed.close()
