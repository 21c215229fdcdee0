"""Build libti_b200.so (sm_100a) in-tree.

    python tensor-inference_b200/build.py [--verbose] [--ptxas-info]

Compiles csrc/*.cu and csrc/*.cpp with nvcc for sm_100a only and links the
shared library next to this file.  Objects go to _build/ (git-ignored);
unchanged sources are not recompiled.
"""
import argparse
import concurrent.futures as cf
import os
import subprocess
import sys

HERE = os.path.dirname(os.path.abspath(__file__))
CSRC = os.path.join(HERE, "csrc")
BUILD = os.path.join(HERE, "_build")
LIB = os.path.join(HERE, "libti_b200.so")
NVCC = os.environ.get("NVCC", "/usr/local/cuda/bin/nvcc")

ARCH = ["-gencode", "arch=compute_100a,code=sm_100a"]
COMMON = ["-O3", "-std=c++17", "-lineinfo", "-Xcompiler", "-fPIC", "--expt-relaxed-constexpr",
          "-I" + os.path.join(HERE, "..", "include")]


def _sources():
    out = []
    for f in sorted(os.listdir(CSRC)):
        if f.endswith(".cu") or f.endswith(".cpp"):
            out.append(os.path.join(CSRC, f))
    return out


def _headers_mtime():
    m = 0.0
    for d in (CSRC, os.path.join(HERE, "..", "include")):
        for f in os.listdir(d):
            if f.endswith((".h", ".cuh", ".hpp")):
                m = max(m, os.path.getmtime(os.path.join(d, f)))
    return m


def _compile(src, ptxas_info, verbose):
    obj = os.path.join(BUILD, os.path.basename(src) + ".o")
    hm = _headers_mtime()
    if os.path.exists(obj) and os.path.getmtime(obj) >= max(os.path.getmtime(src), hm):
        return obj, None
    cmd = [NVCC] + ARCH + COMMON + ["-c", src, "-o", obj]
    if src.endswith(".cpp"):
        cmd = [NVCC] + COMMON + ["-x", "c++", "-c", src, "-o", obj]
    if ptxas_info and src.endswith(".cu"):
        cmd += ["-Xptxas", "-v"]
    if verbose:
        print(" ".join(cmd), flush=True)
    r = subprocess.run(cmd, capture_output=True, text=True)
    if r.returncode != 0:
        return None, f"{src}:\n{r.stdout}\n{r.stderr}"
    if ptxas_info:
        sys.stderr.write(r.stderr)
    return obj, None


def build(verbose=False, ptxas_info=False):
    os.makedirs(BUILD, exist_ok=True)
    srcs = _sources()
    with cf.ThreadPoolExecutor(max_workers=min(8, os.cpu_count() or 4)) as ex:
        results = list(ex.map(lambda s: _compile(s, ptxas_info, verbose), srcs))
    errs = [e for _, e in results if e]
    if errs:
        raise RuntimeError("nvcc failed:\n" + "\n".join(errs))
    objs = [o for o, _ in results]
    if not os.path.exists(LIB) or any(os.path.getmtime(o) > os.path.getmtime(LIB) for o in objs):
        cmd = [NVCC] + ARCH + ["-shared", "-Xlinker", "--no-undefined", "-o", LIB] + objs + ["-lcudart_static", "-ldl", "-lrt", "-lpthread"]
        if verbose:
            print(" ".join(cmd), flush=True)
        r = subprocess.run(cmd, capture_output=True, text=True)
        if r.returncode != 0:
            raise RuntimeError("link failed:\n" + r.stdout + r.stderr)
    return LIB


if __name__ == "__main__":
    ap = argparse.ArgumentParser()
    ap.add_argument("--verbose", action="store_true")
    ap.add_argument("--ptxas-info", action="store_true")
    a = ap.parse_args()
    print(build(a.verbose, a.ptxas_info))
