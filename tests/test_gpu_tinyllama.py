"""Benchmark configuration 1 at full depth: the TinyLlama-1.1B shape that the
reference's run_llama tool decodes (tools/run_llama.cpp:104-183): hidden 2048,
22 layers, 32 q / 4 kv heads, head_dim 64, SwiGLU 5632, vocab 32000, RMSNorm
eps 1e-5, RoPE theta 10000, seeded N(0, 0.02) bf16 weights, a 128-token prompt
of ids uniform in [0, 32000), then 128 greedy steps at batch 1.

The steps are teacher-forced: engine and CPU oracle both receive the oracle's
greedy id, so one near-tie flip cannot cascade.  Every step checks bf16 logits
within 2e-2 max-abs relative and the greedy id (equal, or a recorded near-tie
whose top-2 margin is below the logits' own error); the K/V cache of the first
and last layers is compared after the run."""
import numpy as np
import pytest

import oracle
import ti_b200 as ti
from gpu_util import LOGIT_TOL, check_step, rel_err

pytestmark = pytest.mark.gpu

PROMPT, STEPS = 128, 128


def test_tinyllama_full_depth_128_greedy_steps():
    kw = dict(ti.PRESETS["tinyllama"])
    eng = ti.Engine(ti.model_desc(**kw), max_batch=1, max_seq_len=PROMPT + STEPS + 16)
    try:
        eng.init_synthetic(0, 0.02)
        m = oracle.Model(**kw)
        m.init_synthetic(0, 0.02)
        ids = np.random.default_rng(0).integers(0, kw["vocab"], size=PROMPT, dtype=np.int32)
        sid = eng.seq_create()
        nxt, lb = eng.prefill(sid, ids, logits=ti.LOGITS_BF16)
        s = m.new_seq(PROMPT + STEPS + 16)
        _, lf = s.forward(ids)
        ties = int(not check_step(nxt, lb, lf, "prompt"))
        feed = int(np.argmax(lf))
        for step in range(STEPS):
            got, lb = eng.decode([sid], [feed], logits=ti.LOGITS_BF16)
            _, lf = s.forward([feed])
            ties += int(not check_step(int(got[0]), lb[0], lf, f"step {step}"))
            feed = int(np.argmax(lf))
        L = PROMPT + STEPS
        assert eng.seq_len(sid) == L
        for layer in (0, kw["n_layers"] - 1):
            for which in (0, 1):
                g = oracle.bf16_to_f32(eng.seq_read_kv(sid, layer, which, L))
                r = oracle.bf16_to_f32(s.read_kv(layer, which, L))
                assert rel_err(g, r) < LOGIT_TOL, (layer, which)
        eng.check()
        assert ties <= (STEPS + 1) // 10, f"{ties} near-tie flips"
    finally:
        eng.close()
