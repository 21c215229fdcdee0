"""Device sampling (ti_op_sample, ti_engine_seq_set_sampler) against the oracle.

The CUDA sampler implements an exact integer-weight form of the reference's
TopP / TopK (src/inference/sampling/top_p.cpp:56-134): tokens by bf16 logit
descending, equal logits by ascending id, per-value weights floor(e * 2^63) with
e from a fixed sequence of IEEE operations, cut and pick by exact 128-bit sums.
oracle.sample_exact restates that form on the host, so every id must match bit
for bit; tests/test_sampling.py shows on the CPU that the form picks the same
logit value as the reference's own sampler (pinned against its code).

Draws: the engine's per-sequence std::mt19937_64 gives the reference's
sequence, which oracle.sample_draws reproduces (top-p: u_0, u_1, ...; top-k:
u_0 at every step)."""
import ctypes as C
import os

import numpy as np
import pytest

import oracle
import ti_b200 as ti
from gpu_util import DevBuf

pytestmark = pytest.mark.gpu

P, K = oracle.SAMPLE_TOP_P, oracle.SAMPLE_TOP_K
SMALL = dict(arch=ti.ARCH_LLAMA, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, intermediate=512,
             vocab=1000, rms_eps=1e-5, rope_theta=10000.0)


def _rows():
    """bf16 logits rows: model-like (a few strong tokens over a broad tail) at
    TinyLlama / Llama-3 / Qwen2 vocabularies, flat, all negative, runs of ties,
    signed zeros, a single token."""
    rng = np.random.default_rng(5)
    out = []
    for vocab, scale in ((1000, 1.0), (32000, 2.5), (128256, 3.0), (152064, 2.0)):
        x = (rng.standard_normal(vocab) * scale).astype(np.float32)
        x[rng.integers(0, vocab, 4)] += 10.0
        out.append(oracle.f32_to_bf16(x))
    out.append(oracle.f32_to_bf16(np.full(4096, 0.25, np.float32)))
    out.append(oracle.f32_to_bf16(-np.abs(rng.standard_normal(3000)).astype(np.float32) - 40.0))
    out.append(oracle.f32_to_bf16(rng.integers(-3, 4, 20000).astype(np.float32)))
    out.append(oracle.f32_to_bf16(np.array([0.0, -0.0, 0.0, -0.0, -1.0], np.float32)))
    out.append(oracle.f32_to_bf16(np.array([7.0], np.float32)))
    return out


CASES = [(ti.SAMPLE_TOP_P, 1.0, 0.95, 0), (ti.SAMPLE_TOP_P, 0.7, 0.9, 0), (ti.SAMPLE_TOP_P, 1.5, 0.5, 0),
         (ti.SAMPLE_TOP_P, 0.0, 1.0, 0), (ti.SAMPLE_TOP_P, 1.0, 1e-6, 0), (ti.SAMPLE_TOP_K, 1.0, 0.0, 40),
         (ti.SAMPLE_TOP_K, 0.8, 0.0, 1), (ti.SAMPLE_TOP_K, 1.2, 0.0, 100000), (ti.SAMPLE_GREEDY, 1.0, 0.0, 0)]


def _op_sample(x, params, draws):
    rows = x.shape[0]
    d = DevBuf.from_array(x)
    o = DevBuf(rows * 4)
    prm = (ti.Sampling * rows)(*params)
    u = np.ascontiguousarray(draws, np.float32)
    ti.check(ti.lib().ti_op_sample(d.ptr, rows, x.shape[1], prm, u.ctypes.data_as(C.POINTER(C.c_float)), o.ptr,
                                   None))
    return o.to_array((rows,), np.int32)


def _expected(row, kind, temperature, p, k, u):
    if kind == ti.SAMPLE_GREEDY:
        return oracle.sample_exact(row, K, 1.0, 0.0, 1, 0.0)
    return oracle.sample_exact(row, kind, temperature, p, k, u)


@pytest.mark.parametrize("kind,temperature,p,k", CASES)
def test_op_sample_matches_exact_form(kind, temperature, p, k):
    for ri, row in enumerate(_rows()):
        n = 24
        x = np.tile(row, (n, 1))  # one row, many draws: one CTA per (row, draw)
        u = oracle.sample_draws(1000 + ri, n)
        u[0] = 0.0
        params = [ti.Sampling(kind, temperature, p, k, 0, 0)] * n
        got = _op_sample(x, params, u)
        want = [_expected(row, kind, temperature, p, k, float(v)) for v in u]
        assert got.tolist() == want, (ri, kind, temperature, p, k)


def test_op_sample_greedy_is_first_max():
    rows = _rows()[:4]
    for row in rows:
        got = _op_sample(row[None, :], [ti.Sampling(ti.SAMPLE_GREEDY, 1.0, 0.0, 0, 0, 0)], [0.5])
        assert int(got[0]) == int(np.argmax(oracle.bf16_to_f32(row)))


def test_op_sample_mixed_rows():
    rng = np.random.default_rng(9)
    V = 32000
    x = oracle.f32_to_bf16((rng.standard_normal((6, V)) * 2).astype(np.float32))
    specs = [(ti.SAMPLE_TOP_P, 0.9, 0.8, 0), (ti.SAMPLE_TOP_K, 1.0, 0.0, 50), (ti.SAMPLE_GREEDY, 1.0, 0.0, 0),
             (ti.SAMPLE_TOP_P, 1.0, 1.0, 0), (ti.SAMPLE_TOP_K, 0.5, 0.0, 3), (ti.SAMPLE_TOP_P, 2.0, 0.3, 0)]
    u = oracle.sample_draws(77, 6)
    got = _op_sample(x, [ti.Sampling(kd, t, p, k, 0, 0) for kd, t, p, k in specs], u)
    want = [_expected(x[i], *specs[i], float(u[i])) for i in range(6)]
    assert got.tolist() == want


def test_op_sample_rejects_bad_arguments():
    x = DevBuf.from_array(oracle.f32_to_bf16(np.zeros(10, np.float32)))
    o = DevBuf(4)
    u = (C.c_float * 1)(0.5)
    for prm, draw in ((ti.Sampling(ti.SAMPLE_TOP_K, 1.0, 0.0, 0, 0, 0), 0.5),
                      (ti.Sampling(7, 1.0, 0.9, 1, 0, 0), 0.5),
                      (ti.Sampling(ti.SAMPLE_TOP_P, 1.0, 0.9, 0, 0, 0), 1.0)):
        u[0] = draw
        assert ti.lib().ti_op_sample(x.ptr, 1, 10, C.byref(prm), u, o.ptr, None) == ti.TI_ERR_INVALID


def _engine(**kw):
    eng = ti.Engine(ti.model_desc(**dict(SMALL, **kw)), max_batch=8, max_seqs=4, max_seq_len=128)
    eng.init_synthetic(0, 0.5)  # wide logits: the nucleus is neither one token nor the vocabulary
    return eng


@pytest.mark.parametrize("kind,temperature,p,k", [(ti.SAMPLE_TOP_P, 0.8, 0.9, 0), (ti.SAMPLE_TOP_K, 1.0, 0.0, 20)])
@pytest.mark.parametrize("chunk", [None, 4])
def test_engine_samples_each_returned_id(kind, temperature, p, k, chunk):
    eng = _engine()
    sid = eng.seq_create()
    seed = 4242
    eng.set_sampler(sid, kind, temperature, p, k, seed)
    prompt = oracle.fill_ids("smp", 10, 1, SMALL["vocab"])  # chunk 4: steps of 4, 4 and 2 tokens
    steps = 6
    u = oracle.sample_draws(seed, steps + 1)
    if kind == ti.SAMPLE_TOP_K:
        u[:] = u[0]  # a fresh engine per draw
    nxt, lb = eng.prefill(sid, prompt, logits=ti.LOGITS_BF16, chunk=chunk)
    assert int(nxt) == oracle.sample_exact(lb, kind, temperature, p, k, float(u[0]))
    tok = int(nxt)
    for i in range(steps):
        got, lb = eng.decode([sid], [tok], logits=ti.LOGITS_BF16)
        assert int(got[0]) == oracle.sample_exact(lb[0], kind, temperature, p, k, float(u[i + 1])), i
        tok = int(got[0])
    eng.check()
    eng.close()


def test_engine_mixed_batch_keeps_greedy_rows():
    a, b = _engine(), _engine()
    prompts = [oracle.fill_ids("mx0", 5, 2, SMALL["vocab"]), oracle.fill_ids("mx1", 7, 3, SMALL["vocab"])]
    sa = [a.seq_create() for _ in prompts]
    sb = [b.seq_create() for _ in prompts]
    b.set_sampler(sb[1], ti.SAMPLE_TOP_P, 1.0, 0.95, 0, 99)
    u = oracle.sample_draws(99, 5)
    toks_a, toks_b = [], []
    for i, pr in enumerate(prompts):
        toks_a.append(int(a.prefill(sa[i], pr)))
        nb, lb = b.prefill(sb[i], pr, logits=ti.LOGITS_BF16)
        toks_b.append(int(nb))
        if i == 1:
            assert toks_b[1] == oracle.sample_exact(lb, P, 1.0, 0.95, 0, float(u[0]))
    assert toks_a[0] == toks_b[0]
    for step in range(4):
        ga = a.decode(sa, toks_a)
        gb, lb = b.decode(sb, toks_b, logits=ti.LOGITS_BF16)
        assert int(gb[0]) == int(ga[0]), step  # greedy row: the LM head's argmax, as without sampling
        assert int(gb[1]) == oracle.sample_exact(lb[1], P, 1.0, 0.95, 0, float(u[step + 1])), step
        toks_a = [int(ga[0]), int(ga[1])]
        toks_b = [int(gb[0]), int(gb[1])]
    a.close()
    b.close()


@pytest.mark.parametrize("kind,temperature,p,k", [(ti.SAMPLE_TOP_P, 0.9, 0.8, 0), (ti.SAMPLE_TOP_K, 1.0, 0.0, 30)])
def test_device_chain_samples_as_host_steps(kind, temperature, p, k):
    """A bound device chain (no host work per step) draws from pre-generated
    draws: the same ids, K/V and later host draws as step-by-step decoding."""
    steps, seed = 7, 555
    prompt = oracle.fill_ids("chain", 6, 4, SMALL["vocab"])
    a, b = _engine(), _engine()
    sa, sb = a.seq_create(), b.seq_create()
    a.set_sampler(sa, kind, temperature, p, k, seed)
    b.set_sampler(sb, kind, temperature, p, k, seed)
    first_a, first_b = a.prefill(sa, prompt), b.prefill(sb, prompt)
    assert first_a == first_b
    tok = first_a
    for _ in range(steps):
        tok = int(a.decode([sa], [tok])[0])
    b.seq_reserve(sb, len(prompt) + steps + 1)
    b.bind([sb], [first_b])
    for _ in range(steps):
        b.decode_device()
    last = b.unbind(steps)
    assert int(last[0]) == tok
    n = len(prompt) + steps
    assert a.seq_len(sa) == b.seq_len(sb) == n
    for which in (0, 1):
        np.testing.assert_array_equal(a.seq_read_kv(sa, 0, which, n), b.seq_read_kv(sb, 0, which, n))
    # after the chain, host steps continue the same draw sequence
    assert int(a.decode([sa], [tok])[0]) == int(b.decode([sb], [tok])[0])
    a.check()
    b.check()
    a.close()
    b.close()


def test_engine_sampler_errors():
    eng = _engine()
    sid = eng.seq_create()
    with pytest.raises(ti.TiError) as ei:
        eng.set_sampler(sid, ti.SAMPLE_TOP_K, 1.0, 0.0, 0, 1)
    assert ei.value.status == ti.TI_ERR_INVALID
    with pytest.raises(ti.TiError) as ei:
        eng.set_sampler(sid, ti.SAMPLE_TOP_P, float("nan"), 0.9, 0, 1)
    assert ei.value.status == ti.TI_ERR_INVALID
    eng.close()
