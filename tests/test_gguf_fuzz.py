"""GGUF reader robustness: the reader parses files from untrusted sources on
the host, so every corrupted file must come back as an error status (or as a
valid file), never as a crash or a read outside the mapping.

Seeded mutations of a valid file (truncation, byte flips, extreme values
written over length / count / offset fields, both at random) each go through
every reader entry: open, tensor table, names, metadata queries, the model
description, RoPE factors and tensor reads.  The cases run in a spawned child
so a crash fails this test instead of ending the test session; the child
records the case it is on, so the failing mutation is named.  A second sweep
writes extreme values (negative, zero, 2^31 - 1) into each integer of the model
description.  Host-only."""
import multiprocessing as mp
import os
import subprocess
import sys

import numpy as np
import pytest

from gguf_writer import (ARR, F32, GGML_BF16, GGML_F16, GGML_F32, GGML_Q4_0, GGML_Q8_0, I32, STR, U32, write)

HERE = os.path.dirname(os.path.abspath(__file__))
N_CASES = 3000
KEYS = ["general.architecture", "llama.block_count", "llama.embedding_length", "llama.attention.head_count",
        "llama.attention.layer_norm_rms_epsilon", "llama.rope.freq_base", "tokenizer.ggml.tokens", "missing.key"]


INT_KEYS = ["llama.block_count", "llama.embedding_length", "llama.feed_forward_length", "llama.attention.head_count",
            "llama.attention.head_count_kv", "llama.attention.key_length"]
EXTREMES = [-2**31, -4, -1, 0, 1, 3, 2**31 - 1]


def _valid_file(path, override=None):
    rng = np.random.default_rng(1)
    ints = {"llama.block_count": 1, "llama.embedding_length": 64, "llama.feed_forward_length": 128,
            "llama.attention.head_count": 4, "llama.attention.head_count_kv": 2}
    if override:
        ints[override[0]] = override[1]
    meta = [("general.architecture", STR, "llama"), ("general.alignment", U32, 32),
            *[(k, I32 if v < 0 or override and k == override[0] else U32, v) for k, v in ints.items()],
            ("llama.attention.layer_norm_rms_epsilon", F32, 1e-5),
            ("llama.rope.freq_base", F32, 10000.0), ("tokenizer.ggml.tokens", ARR, (STR, ["<s>", "</s>", "a", "b"])),
            ("x.arr", ARR, (U32, [1, 2, 3]))]
    q4 = np.zeros(4 * 2 * 18, np.uint8)
    q8 = np.zeros(2 * 2 * 34, np.uint8)
    tensors = [("token_embd.weight", GGML_BF16, (64, 8), rng.integers(0, 2**16, 512, dtype=np.uint16).tobytes()),
               ("output_norm.weight", GGML_F32, (64,), rng.standard_normal(64).astype(np.float32).tobytes()),
               ("blk.0.attn_q.weight", GGML_Q4_0, (64, 4), q4.tobytes()),
               ("blk.0.attn_k.weight", GGML_Q8_0, (64, 2), q8.tobytes()),
               ("blk.0.ffn_up.weight", GGML_F16, (64, 2), rng.standard_normal(128).astype(np.float16).tobytes()),
               ("rope_freqs.weight", GGML_F32, (8,), np.ones(8, np.float32).tobytes()),
               # k-quant and legacy block types decoded to bf16 (Q4_K, Q6_K, Q5_1)
               ("blk.0.ffn_down.weight", 12, (256, 2), rng.integers(0, 256, 2 * 144, dtype=np.uint8).tobytes()),
               ("blk.0.attn_v.weight", 14, (256, 2), rng.integers(0, 256, 2 * 210, dtype=np.uint8).tobytes()),
               ("blk.0.attn_output.weight", 7, (64, 2), rng.integers(0, 256, 2 * 2 * 24, dtype=np.uint8).tobytes())]
    write(path, meta, tensors)


def _exercise(ti, path):
    try:
        g = ti.Gguf(path)
    except ti.TiError:
        return
    with g:
        n = len(g)
        for i in range(-1, min(n, 64) + 1):
            try:
                inf = g.info(i)
            except ti.TiError:
                continue
            for f in (lambda: g.reference_name(i), lambda: g.find(inf["name"])):
                try:
                    f()
                except ti.TiError:
                    pass
            dims = inf["dims"]
            elems = int(np.prod([max(d, 0) for d in dims], dtype=np.float64)) if dims else 0
            if 0 < elems <= 1 << 20 and inf["bytes"] <= 1 << 22:
                for dt in (ti.DTYPE_BF16, ti.DTYPE_Q4_0, ti.DTYPE_Q8_0):
                    try:
                        g.read(i, dt)
                    except ti.TiError:
                        pass
        for key in KEYS + ["x.arr"]:
            for f in (g.meta_int, g.meta_float, g.meta_str, g.meta_array_len, g.meta_array):
                try:
                    f(key)
                except ti.TiError:
                    pass
        for f in (g.model_desc, lambda: g.rope_inv_freq(32), lambda: g.rope_inv_freq(0)):
            try:
                f()
            except ti.TiError:
                pass


def _mutate(rng, blob):
    b = bytearray(blob)
    kind = int(rng.integers(0, 4))
    if kind == 0:  # truncate
        return bytes(b[:int(rng.integers(0, len(b)))])
    if kind == 1:  # flip bytes
        for _ in range(int(rng.integers(1, 17))):
            b[int(rng.integers(0, len(b)))] ^= int(rng.integers(1, 256))
        return bytes(b)
    # an extreme 4- or 8-byte value over a field of the header, metadata or tensor table
    head = min(len(b) - 8, 900)
    at = int(rng.integers(0, head))
    width = 8 if kind == 2 else 4
    v = int(rng.choice([0, 1, 2**31 - 1, 2**31, 2**32 - 1, 2**63 - 1, 2**63, 2**64 - 1, 2**40,
                        int(rng.integers(0, 2**62))]))
    b[at:at + width] = (v % (1 << (8 * width))).to_bytes(width, "little")
    return bytes(b)


def _import_ti(lib_path=None):
    """ti_b200, its entry points bound to `lib_path` when given (the sanitizer build)"""
    sys.path.insert(0, os.path.join(os.path.dirname(HERE), "tensor-inference_b200"))
    sys.path.insert(0, HERE)
    import ti_b200 as ti

    if lib_path:
        import host_sanitize

        host_sanitize.bind(ti, lib_path)
    return ti


def _worker(tmp, progress, lib_path=None, n_cases=N_CASES, seed=2024):
    ti = _import_ti(lib_path)

    src = os.path.join(tmp, "valid.gguf")
    _valid_file(src)
    blob = open(src, "rb").read()
    _exercise(ti, src)
    rng = np.random.default_rng(seed)
    path = os.path.join(tmp, "case.gguf")
    for case in range(n_cases):
        data = _mutate(rng, blob)
        with open(path, "wb") as f:
            f.write(data)
        with open(progress, "w") as f:
            f.write(str(case))
        _exercise(ti, path)
    with open(progress, "w") as f:
        f.write("done")


def _worker_meta(tmp, progress, lib_path=None):
    ti = _import_ti(lib_path)

    path = os.path.join(tmp, "meta.gguf")
    for key in INT_KEYS:
        for v in EXTREMES:
            _valid_file(path, (key, v))
            with open(progress, "w") as f:
                f.write(f"{key}={v}")
            _exercise(ti, path)
    with open(progress, "w") as f:
        f.write("done")


def _run(worker, tmp_path):
    progress = str(tmp_path / "progress")
    ctx = mp.get_context("spawn")
    p = ctx.Process(target=worker, args=(str(tmp_path), progress))
    p.start()
    p.join(timeout=600)
    if p.is_alive():
        p.kill()
        p.join()
    last = open(progress).read() if os.path.exists(progress) else "none"
    assert p.exitcode == 0 and last == "done", f"reader crashed or hung (exit {p.exitcode}) at case {last}"


def test_extreme_metadata_values_fail_cleanly(tmp_path):
    # negative, zero and huge counts (a negative head count once reached an
    # integer division by zero in the q/k row un-permutation)
    _run(_worker_meta, tmp_path)


def test_corrupted_files_fail_cleanly(tmp_path):
    _run(_worker, tmp_path)


def test_sanitized_reader(tmp_path):
    """gguf.cpp built with AddressSanitizer + UBSan (out-of-bounds reads of the
    mapping, integer overflow, division by zero abort the child) over the
    metadata sweep and 5000 mutated files."""
    import host_sanitize

    if not host_sanitize.runtime():
        pytest.skip("gcc sanitizer runtimes not available")
    lib = str(tmp_path / "libhost_asan.so")
    ok, err = host_sanitize.build(lib)
    assert ok, err
    code = (f"import sys; sys.path.insert(0, {HERE!r}); import test_gguf_fuzz as T; "
            f"T._worker_meta({str(tmp_path)!r}, {str(tmp_path / 'p1')!r}, {lib!r}); "
            f"T._worker({str(tmp_path)!r}, {str(tmp_path / 'p2')!r}, {lib!r}, 5000, 7)")
    r = subprocess.run([sys.executable, "-c", code], env=host_sanitize.env(), capture_output=True, text=True,
                       timeout=900)
    last = [open(tmp_path / f).read() if (tmp_path / f).exists() else "none" for f in ("p1", "p2")]
    assert r.returncode == 0 and last == ["done", "done"], (last, r.stderr[-3000:])
