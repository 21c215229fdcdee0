"""The C ABI without a GPU: libti_b200.so loads, exports every function that
include/ti_b200.h declares, and answers the calls that need no device (version,
last-error, argument validation of ops).  The Tier A shim libraries, where they
were built, carry no private copy of the C++ runtime."""
import ctypes as C
import os
import re
import subprocess
import sys

import pytest

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)
PKG = os.path.join(ROOT, "tensor-inference_b200")
HEADER = os.path.join(ROOT, "include", "ti_b200.h")
SHIM = os.path.join(PKG, "backend", "_build")


def declared_functions():
    src = open(HEADER).read()
    src = re.sub(r"/\*.*?\*/", "", src, flags=re.S)
    src = re.sub(r"//[^\n]*", "", src)
    return sorted(set(re.findall(r"\b(ti_[a-z0-9_]+)\s*\(", src)) - {"ti_status"})


@pytest.fixture(scope="module")
def lib():
    sys.path.insert(0, PKG)
    import ti_b200

    if not os.path.exists(ti_b200.LIB_PATH):
        import build as _b  # tensor-inference_b200/build.py

        _b.build()
    return ti_b200.lib()


def test_header_declares_the_engine_surface():
    names = declared_functions()
    for must in ("ti_engine_create", "ti_engine_decode", "ti_op_matmul_t", "ti_op_paged_attention",
                 "ti_adapter_prefetch_async", "ti_pkm_query"):
        assert must in names


def test_library_exports_every_declared_function(lib):
    missing = [n for n in declared_functions() if not hasattr(lib, n)]
    assert not missing, missing


def test_version_and_error_without_gpu(lib):
    lib.ti_version.restype = C.c_int
    assert lib.ti_version() >= 100
    lib.ti_last_error.restype = C.c_char_p
    assert isinstance(lib.ti_last_error(), bytes)


def test_ops_reject_bad_arguments_before_touching_a_device(lib):
    # null operands fail validation with TI_ERR_INVALID (1) and leave a message
    lib.ti_op_paged_attention.restype = C.c_int
    rc = lib.ti_op_paged_attention(None, 1, 32, 8, 128, None, None, None, 1, None, None, 1, 16, C.c_float(1e4), None,
                                   0, None, None)
    assert rc == 1
    lib.ti_last_error.restype = C.c_char_p
    assert b"null" in lib.ti_last_error()


@pytest.mark.parametrize("name", ["libtensor_backend_b200.so", "libref_models_on_b200.so"])
def test_shim_has_no_private_cxx_runtime(name):
    path = os.path.join(SHIM, name)
    if not os.path.exists(path):
        pytest.skip("Tier A shim not built (needs the reference sources)")
    out = subprocess.run(["nm", "-D", "--defined-only", path], capture_output=True, text=True, check=True).stdout
    leaked = [l for l in out.splitlines() if re.search(r"_ZSt4cout|_ZNSo9_M_insert|codecvt", l)]
    assert not leaked, leaked[:5]


def test_init_reports_the_hardware(lib):
    # here: no CUDA device is visible, and ti_init says so instead of going on;
    # on a B200 box it succeeds (tests/test_gpu_ops.py)
    import torch

    n = C.c_int(-1)
    st = lib.ti_init(C.byref(n))
    if torch.cuda.device_count() == 0:
        assert st == 4  # TI_ERR_UNSUPPORTED
        assert b"no CUDA device" in lib.ti_last_error()
        assert n.value == -1
    else:
        assert st == 0 and n.value == torch.cuda.device_count()
    assert lib.ti_shutdown() == 0


def test_selftest_waits_validates_before_any_device_work(lib):
    out = (C.c_double * 2)()
    for bad in (0, -5, 10_000_001):
        assert lib.ti_selftest_waits(0, bad, out) == 1  # TI_ERR_INVALID


BUILT_LIBRARIES = [
    os.path.join(PKG, "libti_b200.so"),
    os.path.join(SHIM, "libtensor_backend_b200.so"),
    os.path.join(SHIM, "libref_models_on_b200.so"),
    os.path.join(ROOT, "oracle", "_build", "liboracle.so"),
    os.path.join(ROOT, "oracle", "_ref", "libref.so"),
]


@pytest.mark.parametrize("path", BUILT_LIBRARIES, ids=os.path.basename)
def test_every_built_library_resolves_all_symbols(path):
    """Open each library with RTLD_NOW in a fresh interpreter: an undefined symbol
    (a source file missing from a link) fails here, on the CPU, instead of at the
    first GPU test that loads the library."""
    if not os.path.exists(path):
        pytest.skip(f"{os.path.basename(path)} not built (its sources are not present here)")
    code = f"import ctypes, os; ctypes.CDLL({path!r}, mode=os.RTLD_NOW)"
    r = subprocess.run([sys.executable, "-c", code], capture_output=True, text=True)
    assert r.returncode == 0, r.stderr[-2000:]
