"""Drop-in check: the reference's UNCHANGED model code (parser, Llama/Qwen/
QwenAdapter/Gemma/Mistral models, adapter loader — compiled from its sources
against this repo's tensor::backend headers) runs on libti_b200 through the
tensor::backend shim (tensor-inference_b200/backend), and its logits match the
reference's own CUDA backend on the same checkpoints (tests/golden/*.npz):
2e-2 max-abs relative, the benchmark tolerance."""
import ctypes as C
import glob
import json
import os
import sys
import tempfile

import numpy as np
import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
sys.path.insert(0, os.path.join(HERE, "golden"))
LIB = os.path.join(ROOT, "tensor-inference_b200", "backend", "_build", "libref_models_on_b200.so")
FIXTURES = sorted(glob.glob(os.path.join(HERE, "golden", "*.npz")))
pytestmark = pytest.mark.gpu


@pytest.fixture(scope="module")
def ref_on_b200():
    if not os.path.exists(LIB):
        pytest.fail(f"{LIB} not built (tensor-inference_b200/backend/Makefile needs the reference sources)")
    lib = C.CDLL(LIB)
    lib.ref_run.restype = C.c_int
    lib.ref_run.argtypes = [C.c_char_p, C.c_int, C.c_char_p, C.c_void_p, C.c_int, C.c_void_p, C.c_int, C.c_int,
                            C.c_void_p, C.c_int, C.c_char_p, C.c_int]
    return lib


@pytest.mark.parametrize("path", FIXTURES, ids=[os.path.basename(p)[:-4] for p in FIXTURES])
def test_reference_models_on_b200_backend(ref_on_b200, path):
    import make_golden as mg

    z = np.load(path)
    kw = json.loads(str(z["kw"]))
    with tempfile.TemporaryDirectory() as d:
        adir = mg.build_case(d, kw)
        prompt, feed = z["prompt"], z["feed"]
        V = kw["vocab"]
        logits = np.zeros((len(feed) + 1, V), np.float32)
        err = C.create_string_buffer(512)
        rc = ref_on_b200.ref_run(d.encode(), kw["arch"], adir.encode() if adir else None,
                                 np.ascontiguousarray(prompt, np.int32).ctypes.data, len(prompt),
                                 np.ascontiguousarray(feed, np.int32).ctypes.data, len(feed), mg.MAX_SEQ,
                                 logits.ctypes.data, V, err, 512)
        assert rc == 0, err.value.decode()
    ref = z["ref_logits"]
    for i in range(len(ref)):
        e = np.abs(logits[i] - ref[i]).max() / np.abs(ref[i]).max()
        assert e <= 2e-2, (i, e)
