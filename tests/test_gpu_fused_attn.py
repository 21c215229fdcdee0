"""With TI_FUSED_ATTN=1, single-token decode steps run attention inside the o
projection's GEMV (csrc/attn_fused.cuh): RoPE of q and k, the K/V row into its page, paged GQA
attention and the o projection in one kernel, the GEMV's weight stream running
while the consumer warps attend.  These cases stress its work split against the
CPU oracle (restating llama_model.cpp:147-187 and ops.cu:210-312, 444-544):
contexts where one warp scores several pages (TI_ATT_WARPS caps the scoring
warps), sliding windows that start inside a page, head_dim 64 and 128, GQA
groups of 1 to 8; and the fused step against the separate attention kernel
(TI_FUSED_ATTN=0) on the Llama-3-8B layer shapes at a 3,000-token context."""
import numpy as np
import pytest

import oracle
import ti_b200 as ti
from gpu_util import LOGIT_TOL, rel_err
from test_gpu_engine import _run_parity

pytestmark = pytest.mark.gpu


@pytest.fixture(autouse=True)
def _fused(monkeypatch):
    monkeypatch.setenv("TI_FUSED_ATTN", "1")  # opt-in path


@pytest.mark.parametrize("warps", [None, "1", "3"])
def test_several_pages_per_warp(monkeypatch, warps):
    # hidden 128: a grid of 128 CTAs, 32 per kv head; one scoring warp per CTA
    # puts pages 32.. of a 600-token context on warps that already scored one
    if warps:
        monkeypatch.setenv("TI_ATT_WARPS", warps)
    kw = dict(arch=ti.ARCH_LLAMA, hidden=128, n_layers=2, n_heads=8, n_kv_heads=4, head_dim=64, intermediate=256,
              vocab=512, rms_eps=1e-5, rope_theta=10000.0)
    _run_parity(kw, [600], steps=6, check_kv=True, max_seq_len=640)


@pytest.mark.parametrize("n_heads,n_kv,hd", [(8, 1, 128), (16, 2, 128), (4, 4, 128), (14, 2, 64), (8, 2, 128)])
def test_group_sizes_and_head_dims(n_heads, n_kv, hd):
    kw = dict(arch=ti.ARCH_LLAMA, hidden=256, n_layers=2, n_heads=n_heads, n_kv_heads=n_kv, head_dim=hd,
              intermediate=512, vocab=1000, rms_eps=1e-5, rope_theta=500000.0)
    _run_parity(kw, [70], steps=5, check_kv=True)


@pytest.mark.parametrize("window", [37, 16, 1])
def test_sliding_window_inside_a_page(window):
    kw = dict(arch=ti.ARCH_MISTRAL, hidden=256, n_layers=2, n_heads=8, n_kv_heads=2, head_dim=64,
              intermediate=512, vocab=1000, rms_eps=1e-5, rope_theta=10000.0, sliding_window=window)
    _run_parity(kw, [90], steps=5, check_kv=True)


def _logits_at_context(monkeypatch, fused, ctx):
    monkeypatch.setenv("TI_FUSED_ATTN", "1" if fused else "0")
    kw = dict(ti.PRESETS["llama3_8b"], n_layers=2)
    eng = ti.Engine(ti.model_desc(**kw), max_batch=1, max_seq_len=ctx + 16)
    try:
        eng.init_synthetic(0, 0.02)
        sid = eng.seq_create()
        eng.seq_fill_synthetic(sid, ctx, seed=3)
        outs = []
        tok = 17
        for _ in range(3):
            nxt, lb = eng.decode([sid], [tok], logits=ti.LOGITS_BF16)
            outs.append((int(nxt[0]), oracle.bf16_to_f32(lb[0])))
            tok = int(nxt[0])
        kv = eng.seq_read_kv(sid, 1, 0, ctx + 3)
        eng.check()
    finally:
        eng.close()
    return outs, kv


def test_fused_step_matches_attention_kernel_8b_long_context(monkeypatch):
    fused, kf = _logits_at_context(monkeypatch, True, 3000)
    plain, kp = _logits_at_context(monkeypatch, False, 3000)
    for (i0, l0), (i1, l1) in zip(fused, plain):
        assert rel_err(l0, l1) < LOGIT_TOL
        assert i0 == i1
    # the new rows' K (RoPE, bf16) agree; cached rows are the same synthetic values
    assert rel_err(oracle.bf16_to_f32(kf), oracle.bf16_to_f32(kp)) < LOGIT_TOL
    np.testing.assert_array_equal(kf[:3000], kp[:3000])
