"""Known-answer tests of the CPU oracle (no GPU): scalar formats, each op on
hand-checkable inputs, GGUF blocks, PKM, the synthetic generator, and the model
step against an independent numpy restatement."""
import numpy as np
import pytest

from numpy_model import NumpyModel, rb


def test_bf16_rounding_matches_numpy(orc):
    x = np.array([1.0, 1.00390625, 1.0078125 + 2**-9, -3.14159, 65504.0, 1e-40, 0.0, -0.0], np.float32)
    got = np.array([orc.lib().orc_f32_to_bf16(float(v)) for v in x], np.uint16)
    np.testing.assert_array_equal(got, orc.f32_to_bf16(x))
    # ties to even: 1 + 2^-8 is halfway between 1 and 1 + 2^-7
    assert orc.lib().orc_f32_to_bf16(1.0 + 2**-8) == orc.f32_to_bf16(np.float32(1.0))[()]


def test_f16_roundtrip(orc):
    L = orc.lib()
    for v in [0.0, 1.0, -2.5, 65504.0, 6.1035156e-05, 5.9604645e-08, 0.3333333]:
        h = L.orc_f32_to_f16(v)
        assert h == np.float16(v).view(np.uint16)
        assert L.orc_f16_to_f32(h) == float(np.float16(v))


def test_synthetic_generator_moments_and_determinism(orc):
    a = orc.fill_bf16("model.layers.0.self_attn.q_proj.weight", (512, 512), seed=0, std=0.02)
    b = orc.fill_bf16("model.layers.0.self_attn.q_proj.weight", (512, 512), seed=0, std=0.02)
    c = orc.fill_bf16("model.layers.0.self_attn.k_proj.weight", (512, 512), seed=0, std=0.02)
    np.testing.assert_array_equal(a, b)
    assert not np.array_equal(a, c)
    f = orc.bf16_to_f32(a)
    assert abs(f.mean()) < 1e-3 and abs(f.std() - 0.02) < 5e-4
    ids = orc.fill_ids("prompt", 4096, 0, 32000)
    assert ids.min() >= 0 and ids.max() < 32000 and len(np.unique(ids)) > 3500


def test_rope_identity_at_position_zero(orc):
    x = orc.fill_bf16("x", (1, 4, 64), 1)
    out = np.empty_like(x)
    fr = np.empty(32, np.float32)
    orc.lib().orc_rope_freqs(64, 10000.0, None, orc.ptr(fr))
    orc.lib().orc_rope(orc.ptr(x), orc.ptr(out), 1, 4, 64, 0, orc.ptr(fr))
    np.testing.assert_array_equal(out, x)


def test_rope_freqs_llama3_scaling(orc):
    sc = orc.RopeScaling(1, 8.0, 1.0, 4.0, 8192)
    fr = np.empty(64, np.float32)
    orc.lib().orc_rope_freqs(128, 500000.0, sc, orc.ptr(fr))
    base = (1.0 / np.power(np.float32(500000.0), np.arange(64, dtype=np.float32) * 2 / 128)).astype(np.float32)
    wl = 2 * np.pi / base
    assert np.allclose(fr[wl < 8192 / 4], base[wl < 8192 / 4])
    assert np.allclose(fr[wl > 8192], base[wl > 8192] / 8.0, rtol=1e-6)


def test_rms_norm_constant_row(orc):
    H = 256
    x = orc.f32_to_bf16(np.full(H, 0.5, np.float32))
    w = orc.f32_to_bf16(np.full(H, 2.0, np.float32))
    out = np.empty(H, np.uint16)
    orc.lib().orc_rms_norm(orc.ptr(x), orc.ptr(w), orc.ptr(out), 1, H, 1e-5, 0)
    expect = 0.5 / np.sqrt(np.float32(0.25) + np.float32(1e-5)) * 2.0
    np.testing.assert_allclose(orc.bf16_to_f32(out), expect, rtol=4e-3)
    orc.lib().orc_rms_norm(orc.ptr(x), orc.ptr(w), orc.ptr(out), 1, H, 1e-5, 1)  # Gemma: w + 1
    np.testing.assert_allclose(orc.bf16_to_f32(out), expect * 1.5, rtol=4e-3)


def test_softmax_uniform(orc):
    x = np.full((3, 7), 1.25, np.float32)
    orc.lib().orc_softmax_f32(orc.ptr(x), 3, 7)
    np.testing.assert_allclose(x, 1.0 / 7, rtol=1e-6)


def test_attention_gqa_head_mapping(orc):
    # one cached token: softmax of a single score is 1, so out[h] = v[h // group]
    nq, nkv, hd = 8, 2, 16
    q = orc.fill_bf16("q", (1, nq, hd), 3)
    k = orc.fill_bf16("k", (1, nkv, hd), 3)
    v = orc.fill_bf16("v", (1, nkv, hd), 3)
    out = np.empty((1, nq, hd), np.uint16)
    orc.lib().orc_attention(orc.ptr(q), orc.ptr(k), orc.ptr(v), orc.ptr(out), 1, nq, 1, nkv, hd, 0, -1)
    for h in range(nq):
        np.testing.assert_array_equal(out[0, h], v[0, h // (nq // nkv)])


def test_attention_causal_and_window(orc):
    nq = nkv = 2
    hd, T = 8, 5
    q = orc.fill_bf16("q", (T, nq, hd), 4)
    k = orc.fill_bf16("k", (T, nkv, hd), 4)
    v = orc.fill_bf16("v", (T, nkv, hd), 4)
    out = np.empty((T, nq, hd), np.uint16)
    orc.lib().orc_attention(orc.ptr(q), orc.ptr(k), orc.ptr(v), orc.ptr(out), T, nq, T, nkv, hd, 1, -1)
    # first row attends to key 0 only
    np.testing.assert_array_equal(out[0], v[0])
    # window 1: every row attends to itself only
    orc.lib().orc_attention(orc.ptr(q), orc.ptr(k), orc.ptr(v), orc.ptr(out), T, nq, T, nkv, hd, 1, 1)
    np.testing.assert_array_equal(out, v)


def test_q4_0_known_block(orc):
    # d = max / -8 with max = -8 -> d = 1; x = q - 8 exactly representable
    q = np.arange(32) % 16
    x = (q - 8).astype(np.float32)
    x[np.argmin(x)] = -8.0
    blk = np.empty(18, np.uint8)
    orc.lib().orc_q4_0_quantize(orc.ptr(x), 32, orc.ptr(blk))
    assert blk[:2].view(np.uint16)[0] == np.float16(1.0).view(np.uint16)
    assert blk[2] == (q[0] | (q[16] << 4))
    back = np.empty(32, np.float32)
    orc.lib().orc_q4_0_dequantize(orc.ptr(blk), 32, orc.ptr(back))
    np.testing.assert_array_equal(back, x)


def test_q8_0_roundtrip_error(orc):
    x = orc.fill_f32("w", (64 * 32,), 5, 0.02)
    blk = np.empty(64 * 34, np.uint8)
    orc.lib().orc_q8_0_quantize(orc.ptr(x), x.size, orc.ptr(blk))
    back = np.empty_like(x)
    orc.lib().orc_q8_0_dequantize(orc.ptr(blk), x.size, orc.ptr(back))
    amax = np.abs(x.reshape(-1, 32)).max(1, keepdims=True)
    # half a step, plus the fp16 rounding of d scaled by |q| <= 127
    assert np.all(np.abs(back - x).reshape(-1, 32) <= amax / 127 * (0.5 + 127 * 2.0**-11) * 1.01)


def test_pkm_codeword_query(orc):
    n, D = 64, 32
    c1 = orc.fill_f32("c1", (n, D), 6)
    c2 = orc.fill_f32("c2", (n, D), 6)
    q = np.concatenate([c1[17], c2[42]])[None].copy()
    addr = np.empty(1, np.int32)
    orc.lib().orc_pkm_assign(orc.ptr(c1), orc.ptr(c2), n, D, orc.ptr(q), 1, orc.ptr(addr))
    assert addr[0] == 17 * n + 42
    # registry: collisions keep the lowest adapter id
    table = np.empty(n * n, np.int32)
    ca = np.array([5, 9, 5, 7], np.int32)
    orc.lib().orc_pkm_build_table(orc.ptr(ca), 4, orc.ptr(table), n * n)
    assert table[5] == 0 and table[9] == 1 and table[7] == 3 and table[0] == -1


TINY = dict(arch=0, hidden=128, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=32, intermediate=256, vocab=512,
            rms_eps=1e-5, rope_theta=10000.0)


def _weights(orc, m, kw):
    import ti_b200

    d = ti_b200.model_desc(**kw)
    return {n: m.get_weight(n, s) for n, s in ti_b200.tensor_names(d)}


@pytest.mark.parametrize("bias", [0, 1])
def test_oracle_model_matches_numpy_restatement(orc, bias):
    kw = dict(TINY, qkv_bias=bias, arch=1 if bias else 0)
    m = orc.Model(**kw)
    m.init_synthetic(seed=11, std=0.05)
    npm = NumpyModel(kw, _weights(orc, m, kw))
    s = m.new_seq(64)
    ids = orc.fill_ids("prompt", 6, 11, kw["vocab"])
    for t in ids:
        _, lf = s.forward([int(t)])
        ref = npm.step(int(t))
        err = np.abs(lf - ref).max() / np.abs(ref).max()
        assert err < 2e-2, err


def test_oracle_prefill_equals_stepwise(orc):
    m = orc.Model(**TINY)
    m.init_synthetic(seed=3)
    ids = orc.fill_ids("prompt", 9, 3, TINY["vocab"])
    s1, s2 = m.new_seq(32), m.new_seq(32)
    _, lf1 = s1.forward(ids)
    for t in ids:
        _, lf2 = s2.forward([int(t)])
    assert np.abs(lf1 - lf2).max() <= 2e-2 * np.abs(lf2).max()
    k1, k2 = s1.read_kv(1, 0, 9), s2.read_kv(1, 0, 9)
    assert np.abs(orc.bf16_to_f32(k1) - orc.bf16_to_f32(k2)).max() < 0.05 * np.abs(orc.bf16_to_f32(k2)).max()


def test_oracle_lora_zero_b_is_base(orc):
    m = orc.Model(**TINY)
    m.init_synthetic(seed=5)
    m.add_adapter(0, rank=4, alpha=8.0, proj_mask=0x7F, seed=9, std_a=0.02, std_b=0.0)
    ids = orc.fill_ids("prompt", 4, 5, TINY["vocab"])
    s1, s2 = m.new_seq(16), m.new_seq(16)
    l1, _ = s1.forward(ids, adapter=0)
    l2, _ = s2.forward(ids, adapter=-1)
    np.testing.assert_array_equal(l1, l2)


def test_oracle_lora_matches_numpy(orc):
    m = orc.Model(**TINY)
    m.init_synthetic(seed=8, std=0.05)
    m.add_adapter(0, rank=4, alpha=8.0, proj_mask=0x7F, seed=21, std_a=0.05, std_b=0.05)
    import ti_b200

    lw = {}
    d = ti_b200.model_desc(**TINY)
    shapes = {"self_attn.q_proj": (128, 128), "self_attn.k_proj": (64, 128), "self_attn.v_proj": (64, 128),
              "self_attn.o_proj": (128, 128), "mlp.gate_proj": (256, 128), "mlp.up_proj": (256, 128),
              "mlp.down_proj": (128, 256)}
    for i in range(d.n_layers):
        for p, (o, inn) in shapes.items():
            a = f"layers.{i}.{p}.lora_A"
            b = f"layers.{i}.{p}.lora_B"
            lw[a] = orc.fill_bf16(a, (4, inn), 21, 0.05)
            lw[b] = orc.fill_bf16(b, (o, 4), 21, 0.05)
    npm = NumpyModel(TINY, _weights(orc, m, TINY), lora=dict(rank=4, alpha=8.0, w=lw))
    s = m.new_seq(16)
    for t in orc.fill_ids("prompt", 3, 8, TINY["vocab"]):
        _, lf = s.forward([int(t)], adapter=0)
        ref = npm.step(int(t))
        assert np.abs(lf - ref).max() / np.abs(ref).max() < 2e-2


def test_rb_helper():
    assert rb(np.float32(1.0 + 2**-9)) == np.float32(1.0)


@pytest.mark.parametrize("qtype", ["q4_0", "q8_0"])
def test_gguf_quantisers_match_the_gguf_package(orc, qtype):
    """The oracle's Q4_0 / Q8_0 quantiser and dequantiser (restated from the
    format's published definition) produce the same block bytes and values as
    the llama.cpp project's own Python implementation (gguf.quants), on values
    with ties, zeros, a wide range and exact block maxima."""
    quants = pytest.importorskip("gguf.quants")
    from gguf import GGMLQuantizationType as Q

    rng = np.random.default_rng(11)
    rows = [rng.standard_normal(4096).astype(np.float32),
            (rng.standard_normal(4096) * 1e-3).astype(np.float32),
            rng.integers(-8, 8, 4096).astype(np.float32),
            np.zeros(4096, np.float32),
            (rng.standard_normal(4096) * 300).astype(np.float32)]
    L = orc.lib()
    t, nb, q_fn, d_fn = ((Q.Q4_0, 18, L.orc_q4_0_quantize, L.orc_q4_0_dequantize) if qtype == "q4_0" else
                         (Q.Q8_0, 34, L.orc_q8_0_quantize, L.orc_q8_0_dequantize))
    for x in rows:
        ref = quants.quantize(x[None, :], t).reshape(-1)
        got = np.empty(x.size // 32 * nb, np.uint8)
        q_fn(orc.ptr(x), x.size, orc.ptr(got))
        np.testing.assert_array_equal(got, ref)
        back = np.empty(x.size, np.float32)
        d_fn(orc.ptr(got), x.size, orc.ptr(back))
        np.testing.assert_array_equal(back, quants.dequantize(ref[None, :], t).reshape(-1))


def test_oracle_under_sanitizers(tmp_path):
    """The oracle (the parity anchor) built with AddressSanitizer + UBSan passes
    its known-answer and sampling tests in a child process."""
    import os
    import subprocess
    import sys

    import host_sanitize

    if not host_sanitize.runtime():
        pytest.skip("gcc sanitizer runtimes not available")
    here = os.path.dirname(os.path.abspath(__file__))
    root = os.path.dirname(here)
    lib = str(tmp_path / "liboracle_asan.so")
    r = subprocess.run(["g++", "-O1", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
                        "-fno-omit-frame-pointer", "-march=x86-64-v3", "-ffp-contract=off", "-fPIC", "-std=c++17",
                        "-pthread", "-shared", "-o", lib, os.path.join(root, "oracle", "oracle.cpp")],
                       capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
    code = (f"import sys; sys.path[:0] = [{root!r}, {here!r}, {os.path.join(root, 'tensor-inference_b200')!r}]; "
            f"import oracle; oracle.LIB_PATH = {lib!r}; import pytest; "
            "sys.exit(pytest.main(['-q', '-x', '-p', 'no:cacheprovider', "
            "'-k', 'not sanitizers and not agrees and not distribution', "  # the long statistical sweeps
            f"{os.path.join(here, 'test_oracle_kat.py')!r}, {os.path.join(here, 'test_sampling.py')!r}]))")
    r = subprocess.run([sys.executable, "-c", code], env=host_sanitize.env(), capture_output=True, text=True,
                       timeout=900, cwd=root)
    assert r.returncode == 0, (r.stdout[-2000:], r.stderr[-2000:])
