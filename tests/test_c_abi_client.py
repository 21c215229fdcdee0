"""The C ABI from plain C: tests/c_abi_client.c compiles as strict C99 (and the
header as C11 and C++17) with every warning an error, links against
libti_b200.so alone, and, without a B200, stops at ti_init with a clear error.
On a B200 its greedy
and top-p ids equal those of the same engine driven through ctypes."""
import os
import subprocess

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "tensor-inference_b200")
INC = os.path.join(ROOT, "include")


def _build(tmp_path):
    import ti_b200 as ti

    if not os.path.exists(ti.LIB_PATH):
        pytest.skip("libti_b200.so not built")
    exe = str(tmp_path / "c_abi_client")
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I" + INC,
                        os.path.join(HERE, "c_abi_client.c"), "-o", exe, "-L" + PKG, "-lti_b200",
                        "-Wl,-rpath," + PKG], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    return exe


@pytest.mark.parametrize("std,lang", [("c11", "c"), ("c++17", "c++")])
def test_header_is_strict_c_and_cxx(tmp_path, std, lang):
    src = tmp_path / "h.c"
    src.write_text('#include "ti_b200.h"\nint main(void) { return TI_OK; }\n')
    cc = "gcc" if lang == "c" else "g++"
    r = subprocess.run([cc, "-x", lang, f"-std={std}", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I" + INC,
                        "-fsyntax-only", str(src)], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr


def test_client_builds_and_reports_missing_hardware(tmp_path):
    import torch

    exe = _build(tmp_path)
    if torch.cuda.device_count() > 0:
        pytest.skip("a GPU is visible: the GPU test runs the client")
    r = subprocess.run([exe, "2"], capture_output=True, text=True, timeout=120)
    assert r.returncode == 2, (r.returncode, r.stderr)
    assert "no CUDA device" in r.stderr


@pytest.mark.gpu
@pytest.mark.parametrize("mode", ["greedy", "p"])
def test_client_ids_equal_the_ctypes_engine(tmp_path, mode):
    import ti_b200 as ti

    exe = _build(tmp_path)
    steps = 5
    r = subprocess.run([exe, str(steps)] + (["p"] if mode == "p" else []), capture_output=True, text=True,
                       timeout=300)
    assert r.returncode == 0, r.stderr
    got = [int(v) for v in r.stdout.split()]
    kw = dict(arch=ti.ARCH_LLAMA, hidden=256, n_layers=2, n_heads=4, n_kv_heads=2, head_dim=64, intermediate=512,
              vocab=1000, rms_eps=1e-5, rope_theta=10000.0)
    eng = ti.Engine(ti.model_desc(**kw), max_batch=1, max_seqs=1, max_seq_len=64)
    eng.init_synthetic(0, 0.02)
    sid = eng.seq_create()
    if mode == "p":
        eng.set_sampler(sid, ti.SAMPLE_TOP_P, 0.8, 0.9, 0, 7)
    want = [int(eng.prefill(sid, np.array([1, 17, 256, 42, 999, 3], np.int32)))]
    for _ in range(steps):
        want.append(int(eng.decode([sid], [want[-1]])[0]))
    eng.close()
    assert got == want


def test_gguf_client_from_plain_c(tmp_path):
    """The GGUF half of the ABI needs no GPU: tests/c_gguf_client.c (strict C99)
    reads a file's model description, vocabulary and tensors, and prints what
    the Python binding reads from the same file."""
    import ti_b200 as ti
    from gguf_writer import ARR, F32, GGML_F32, GGML_Q4_0, STR, U32, write

    if not os.path.exists(ti.LIB_PATH):
        pytest.skip("libti_b200.so not built")
    exe = str(tmp_path / "c_gguf_client")
    r = subprocess.run(["gcc", "-std=c99", "-Wall", "-Wextra", "-pedantic", "-Werror", "-I" + INC,
                        os.path.join(HERE, "c_gguf_client.c"), "-o", exe, "-L" + PKG, "-lti_b200",
                        "-Wl,-rpath," + PKG], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr
    rng = np.random.default_rng(2)
    toks = ["<s>", "</s>", "hello", "wor ld"]
    meta = [("general.architecture", STR, "llama"), ("llama.block_count", U32, 1),
            ("llama.embedding_length", U32, 64), ("llama.feed_forward_length", U32, 128),
            ("llama.attention.head_count", U32, 4), ("llama.attention.head_count_kv", U32, 2),
            ("llama.attention.layer_norm_rms_epsilon", F32, 1e-5), ("tokenizer.ggml.tokens", ARR, (STR, toks))]
    q4 = rng.integers(0, 256, size=(128, 2, 18), dtype=np.uint8)
    q4[:, :, 0:2] = np.full((128, 2), 0.01, np.float16).view(np.uint8).reshape(128, 2, 2)
    tensors = [("token_embd.weight", GGML_F32, (64, 4), rng.standard_normal(256).astype(np.float32).tobytes()),
               ("blk.0.ffn_up.weight", GGML_Q4_0, (64, 128), q4.tobytes()),
               ("blk.0.ffn_down.weight", 12, (256, 64), rng.integers(0, 256, 64 * 144, dtype=np.uint8).tobytes())]
    path = tmp_path / "c.gguf"
    write(path, meta, tensors)
    out = subprocess.run([exe, str(path)], capture_output=True, text=True, timeout=120)
    assert out.returncode == 0, out.stderr
    lines = out.stdout.splitlines()
    with ti.Gguf(path) as g:
        d = g.model_desc()
        assert lines[0] == (f"desc arch {d.arch} hidden {d.hidden} layers {d.n_layers} heads {d.n_heads} "
                            f"kv {d.n_kv_heads} head_dim {d.head_dim} inter {d.intermediate} vocab {d.vocab} "
                            f"wfmt {d.weight_format}")
        assert lines[1:1 + len(toks)] == [f"token {i} {t}" for i, t in enumerate(toks)]
        want = []
        for i in range(len(g)):
            inf = g.info(i)
            total = int(g.read(i).astype(np.uint64).sum())
            want.append(f"tensor {inf['name']} type {inf['type']} ref {g.reference_name(i)} bf16sum {total}")
        assert lines[1 + len(toks):] == want
