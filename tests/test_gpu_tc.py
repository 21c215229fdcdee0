"""Parity of the tensor-core (tcgen05) GEMM path against the CPU oracle.

ti_op_matmul_t sends bf16 products with more than 8 rows to the tcgen05 kernel;
the engine sends every projection of a decode batch of 16..256 tokens there
(with an RMSNorm pass in front of the normed ones).  Shapes below cover token
padding (rows not a multiple of 32), several token chunks, row tails (N not a
multiple of 128), K splits with the last-unit reduction, and the four fused
epilogues (bias store, residual, SwiGLU/GeGLU, LM-head argmax)."""
import numpy as np
import pytest

import oracle
import ti_b200 as ti
from gpu_util import DevBuf, LOGIT_TOL, check_step, rel_err

pytestmark = pytest.mark.gpu


@pytest.mark.parametrize("M,N,K", [(9, 512, 256), (16, 1000, 256), (33, 4096, 4096), (64, 1024, 14336),
                                   (200, 6144, 4096), (300, 640, 1024), (520, 256, 512)])
def test_matmul_t_tensor_cores(M, N, K):
    a = oracle.fill_bf16("tc_a", (M, K), M, 1.0)
    b = oracle.fill_bf16("tc_b", (N, K), N, 0.05)
    ref = np.empty((M, N), np.uint16)
    oracle.lib().orc_matmul_t_bf16(oracle.ptr(a), oracle.ptr(b), oracle.ptr(ref), M, N, K)
    da, db, dc = DevBuf.from_array(a), DevBuf.from_array(b), DevBuf(M * N * 2)
    ti.check(ti.lib().ti_op_matmul_t(ti.DTYPE_BF16, da.ptr, db.ptr, dc.ptr, M, N, K, None))
    out = oracle.bf16_to_f32(dc.to_array((M, N), np.uint16))
    r = oracle.bf16_to_f32(ref)
    assert rel_err(out, r) < 1e-2
    # every row of the output, not only the largest entries, must match
    row_err = np.abs(out - r).max(axis=1) / np.abs(r).max(axis=1)
    assert row_err.max() < 2e-2, int(row_err.argmax())


SMALL = dict(arch=ti.ARCH_LLAMA, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, intermediate=512,
             vocab=1000, rms_eps=1e-5, rope_theta=10000.0)


def _batched_parity(kw, B, steps, seed=0, std=0.02, prompt=lambda b: 2 + b % 7):
    eng = ti.Engine(ti.model_desc(**kw), max_batch=B, max_seqs=B, max_seq_len=128)
    eng.init_synthetic(seed, std)
    m = oracle.Model(**kw)
    m.init_synthetic(seed, std)
    V = kw["vocab"]
    sids, oseqs, feed = [], [], []
    for b in range(B):
        ids = oracle.fill_ids(f"tcp{b}", prompt(b), seed + b, V)
        sid = eng.seq_create()
        eng.prefill(sid, ids)
        os_ = m.new_seq(128)
        _, lf = os_.forward(ids)
        sids.append(sid)
        oseqs.append(os_)
        feed.append(int(np.argmax(lf)))
    ties = 0
    for step in range(steps):
        nxt, lb = eng.decode(sids, feed, logits=ti.LOGITS_BF16)
        new_feed = []
        for b in range(B):
            _, lf = oseqs[b].forward([feed[b]])
            ties += not check_step(int(nxt[b]), lb[b], lf, f"step {step} b{b}")
            new_feed.append(int(np.argmax(lf)))
        feed = new_feed
    eng.check()
    assert ties <= max(1, steps * B // 10), f"{ties} near-tie flips"
    eng.close()


def test_tc_decode_llama_b20():
    _batched_parity(SMALL, 20, steps=4)


def test_tc_decode_qwen_bias_b16():
    kw = dict(SMALL, arch=ti.ARCH_QWEN2, qkv_bias=1, rms_eps=1e-6, rope_theta=1e6)
    _batched_parity(kw, 16, steps=3)


def test_tc_decode_gemma_geglu_b33():
    kw = dict(SMALL, arch=ti.ARCH_GEMMA, rms_eps=1e-6)
    _batched_parity(kw, 33, steps=2)


def test_tc_decode_8b_shapes_b32():
    # Llama-3-8B projection shapes (K = 4096 / 14336, vocab 128256), 2 layers, batch 32
    kw = dict(ti.PRESETS["llama3_8b"], n_layers=2)
    _batched_parity(kw, 32, steps=2, prompt=lambda b: 2)


def test_tc_matches_gemv_path_bits():
    """the same batch through the GEMV (TI_TC_MIN_BATCH above the batch) and the
    tensor-core path agree to bf16 rounding of the logits"""
    import os

    B = 16
    out = {}
    for label, env in (("tc", "16"), ("gemv", "1000")):
        os.environ["TI_TC_MIN_BATCH"] = env
        try:
            eng = ti.Engine(ti.model_desc(**SMALL), max_batch=B, max_seqs=B, max_seq_len=64)
        finally:
            os.environ.pop("TI_TC_MIN_BATCH", None)
        eng.init_synthetic(3, 0.02)
        sids = [eng.seq_create() for _ in range(B)]
        for b, sid in enumerate(sids):
            eng.prefill(sid, oracle.fill_ids(f"eq{b}", 3, b, SMALL["vocab"]))
        feed = [int(x) for x in oracle.fill_ids("eqfeed", B, 1, SMALL["vocab"])]
        _, lb = eng.decode(sids, feed, logits=ti.LOGITS_BF16)
        out[label] = oracle.bf16_to_f32(lb)
        eng.check()
        eng.close()
    assert rel_err(out["tc"], out["gemv"]) < LOGIT_TOL
