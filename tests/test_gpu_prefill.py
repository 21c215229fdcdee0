"""Batched prefill (ti_engine_prefill_chunked): the prompt decoded `chunk` tokens
per step (GEMV path below 8 tokens, tcgen05 path from 8; every K/V row of a
step written to its page before attention, each token attending causally up to
its own position) against the oracle's prompt forward; the KV cache it leaves
and the decode steps after it are checked too."""
import numpy as np
import pytest

import oracle
import ti_b200 as ti
from gpu_util import LOGIT_TOL, check_step, rel_err

pytestmark = pytest.mark.gpu

SMALL = dict(arch=ti.ARCH_LLAMA, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, intermediate=512,
             vocab=1000, rms_eps=1e-5, rope_theta=10000.0)


@pytest.mark.parametrize("arch,n,chunk", [("llama", 5, 8), ("llama", 23, 8), ("llama", 40, 16), ("llama", 37, 32),
                                          ("llama", 3, 2), ("qwen", 29, 12), ("mistral", 27, 9)])
def test_chunked_prefill_parity(arch, n, chunk):
    kw = dict(SMALL)
    if arch == "qwen":
        kw.update(arch=ti.ARCH_QWEN2, qkv_bias=1, rms_eps=1e-6, rope_theta=1e6)
    if arch == "mistral":
        kw.update(arch=ti.ARCH_MISTRAL, sliding_window=8)
    eng = ti.Engine(ti.model_desc(**kw), max_batch=32, max_seqs=2, max_seq_len=256)
    eng.init_synthetic(0, 0.02)
    m = oracle.Model(**kw)
    m.init_synthetic(0, 0.02)
    ids = oracle.fill_ids(f"pf{n}", n, 7, kw["vocab"])
    sid = eng.seq_create()
    nxt, lb = eng.prefill(sid, ids, logits=ti.LOGITS_BF16, chunk=chunk)
    os_ = m.new_seq(512)
    _, lf = os_.forward(ids)
    ties = not check_step(nxt, lb, lf, "prefill")
    assert eng.seq_len(sid) == n
    for layer in (0, kw["n_layers"] - 1):
        for which in (0, 1):
            g = oracle.bf16_to_f32(eng.seq_read_kv(sid, layer, which, n))
            r = oracle.bf16_to_f32(os_.read_kv(layer, which, n))
            assert rel_err(g, r) < LOGIT_TOL, (layer, which)
    feed = int(np.argmax(lf))
    for step in range(3):
        got, lb = eng.decode([sid], [feed], logits=ti.LOGITS_BF16)
        _, lf = os_.forward([feed])
        ties += not check_step(int(got[0]), lb[0], lf, f"decode {step}")
        feed = int(np.argmax(lf))
    assert ties <= 1
    eng.check()
    eng.close()


def test_chunked_prefill_errors():
    eng = ti.Engine(ti.model_desc(**SMALL), max_batch=8, max_seqs=1, max_seq_len=16)
    eng.init_synthetic(0, 0.02)
    sid = eng.seq_create()
    with pytest.raises(ti.TiError) as ei:
        eng.prefill(sid, oracle.fill_ids("x", 20, 1, SMALL["vocab"]), chunk=8)  # beyond max_seq_len
    assert ei.value.status == ti.TI_ERR_STATE
    eng.close()
