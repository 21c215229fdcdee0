"""Generate the sampled ids that pin the oracle's samplers to the reference.

Runs on the CPU (no GPU):  python tests/golden/sampling/make_sampling_golden.py

The reference's own Greedy / TopP / TopK (src/inference/sampling/greedy.cpp,
top_p.cpp, compiled from its unchanged sources into oracle/_ref/libref.so with
the ref_sample entry of oracle/ref/ref_shim.cpp) sample seeded fp32 logits
rows held in host tensors; reference_ids.npz next to this file records the rows, the
sampler settings, the seeds and the reference's ids (a seeded TopP: 12 calls
on one thread, so 12 successive draws; TopK and Greedy: one call).
tests/test_sampling.py checks the oracle against these ids where the reference
build is absent too.
"""
import ctypes as C
import os
import sys

import numpy as np

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(os.path.dirname(os.path.dirname(HERE)))
sys.path.insert(0, ROOT)

import oracle  # noqa: E402

GREEDY, TOP_P, TOP_K = 0, 1, 2
N_DRAWS = 12


def rows():
    """fp32 rows, several of them bf16-rounded (runs of equal logits)"""
    rng = np.random.default_rng(123)
    out = []
    for vocab, scale, bf in ((50, 1.0, False), (1000, 3.0, False), (1000, 1.0, True), (4096, 2.0, True),
                             (3000, 0.3, True)):
        x = (rng.standard_normal(vocab) * scale).astype(np.float32)
        x[rng.integers(0, vocab, 3)] += 4.0 * scale
        out.append(oracle.bf16_to_f32(oracle.f32_to_bf16(x)) if bf else x)
    return out


SETTINGS = [(TOP_P, 1.0, 0.95, 0), (TOP_P, 0.7, 0.9, 0), (TOP_P, 1.4, 0.5, 0), (TOP_P, 0.0, 1.0, 0),
            (TOP_K, 1.0, 0.0, 40), (TOP_K, 0.8, 0.0, 5), (TOP_K, 1.0, 0.0, 100000), (GREEDY, 1.0, 0.0, 0)]


def main():
    L = C.CDLL(os.path.join(ROOT, "oracle", "_ref", "libref.so"))
    L.ref_sample.restype = C.c_int
    L.ref_sample.argtypes = [C.c_void_p, C.c_int, C.c_int, C.c_int, C.c_float, C.c_float, C.c_uint32, C.c_int,
                             C.c_uint64, C.c_int, C.c_void_p, C.c_char_p, C.c_int]
    rs = rows()
    out = {"settings": np.array(SETTINGS, np.float64)}
    for ri, x in enumerate(rs):
        out[f"row{ri}"] = x
        for si, (kind, t, p, k) in enumerate(SETTINGS):
            seed = 1000 * ri + si
            n = N_DRAWS if kind == TOP_P else 1
            ids = np.empty(n, np.int32)
            err = C.create_string_buffer(256)
            rc = L.ref_sample(oracle.ptr(x), 1, x.size, kind, t, p, k, 1, seed, n, oracle.ptr(ids), err, 256)
            assert rc == 0, err.value
            out[f"ids_{ri}_{si}"] = ids
            out[f"seed_{ri}_{si}"] = np.array([seed], np.uint64)
    path = os.path.join(HERE, "reference_ids.npz")
    np.savez_compressed(path, **out)
    print("wrote", path)


if __name__ == "__main__":
    main()
