"""Sanitizer build of the host-side units (GGUF reader, router, error state):
gguf.cpp, router.cpp and api.cpp with AddressSanitizer + UBSan, engine entry
points stubbed (host_asan_stub.cpp), for tests that re-run their host checks
against it in a child process with the sanitizer runtimes preloaded."""
import os
import subprocess

HERE = os.path.dirname(os.path.abspath(__file__))
ROOT = os.path.dirname(HERE)


def runtime():
    """LD_PRELOAD value for gcc's ASan + UBSan runtimes, or None"""
    libs = []
    for name in ("libasan.so", "libubsan.so"):
        r = subprocess.run(["gcc", "-print-file-name=" + name], capture_output=True, text=True)
        path = r.stdout.strip()
        if r.returncode != 0 or not os.path.isabs(path) or not os.path.exists(path):
            return None
        libs.append(path)
    return ":".join(libs)


def build(out_path):
    """compile the sanitizer build to out_path; returns (ok, compiler output)"""
    csrc = os.path.join(ROOT, "tensor-inference_b200", "csrc")
    cmd = ["g++", "-std=c++17", "-O1", "-g", "-fsanitize=address,undefined", "-fno-sanitize-recover=all",
           "-fno-omit-frame-pointer", "-fPIC", "-shared", "-I/usr/local/cuda/include", "-I" + csrc,
           "-I" + os.path.join(ROOT, "include"), os.path.join(csrc, "gguf.cpp"), os.path.join(csrc, "router.cpp"),
           os.path.join(csrc, "api.cpp"), os.path.join(HERE, "host_asan_stub.cpp"), "-o", out_path,
           "-L/usr/local/cuda/lib64", "-lcudart"]
    r = subprocess.run(cmd, capture_output=True, text=True)
    return r.returncode == 0, r.stderr[-2000:]


def bind(ti, lib_path):
    """point the ti_b200 module's entry points at the sanitizer build (the
    entries it holds; the rest stay unbound)"""
    import ctypes as C

    L = C.CDLL(lib_path)
    for name, (res, args) in ti._SIGS.items():
        try:
            f = getattr(L, name)
        except AttributeError:
            continue
        f.restype = res
        f.argtypes = args
    ti._lib = L


def env():
    return dict(os.environ, LD_PRELOAD=runtime() or "", ASAN_OPTIONS="detect_leaks=0:halt_on_error=1",
                UBSAN_OPTIONS="halt_on_error=1:print_stacktrace=1")
