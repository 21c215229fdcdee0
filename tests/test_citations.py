"""Every reference citation in the repository's code (comments and docstrings)
names a file that exists in the reference and lines within it:
full paths (src/..., include/...) and bare file names (ops.cu:46-88), which
must resolve to exactly one reference file.  Needs the reference tree; skipped
where it is absent."""
import glob
import os
import re

import pytest

ROOT = os.path.dirname(os.path.dirname(os.path.abspath(__file__)))
REF = os.environ.get("TI_REFERENCE_DIR") or os.path.join(os.path.dirname(ROOT), "reference")
SKIP_DIRS = ("_work", "baseline", "oracle/_ref", "gpurun_out")
FULL = re.compile(r"((?:src|include|tools|docs)/[\w./-]+\.(?:cpp|hpp|cu|h|md|txt|json)):(\d+)(?:-(\d+))?")
BARE = re.compile(r"(?<![\w/])([A-Za-z_]\w*\.(?:cpp|hpp|cu|md|txt)):(\d+)(?:-(\d+))?")


def _sources():
    out = []
    for f in glob.glob(os.path.join(ROOT, "**", "*"), recursive=True):
        rel = os.path.relpath(f, ROOT)
        if rel.startswith(SKIP_DIRS) or not os.path.isfile(f):
            continue
        if rel.endswith((".cu", ".cuh", ".cpp", ".h", ".py", ".c")):
            out.append(rel)
    return out


def _lines(path):
    with open(path, errors="replace") as f:
        return sum(1 for _ in f)


def test_reference_citations_resolve():
    if not os.path.isdir(os.path.join(REF, "src")):
        pytest.skip("reference tree not present")
    by_base = {}
    for p in glob.glob(os.path.join(REF, "**", "*"), recursive=True):
        if os.path.isfile(p) and p.endswith((".cpp", ".hpp", ".cu", ".h", ".md", ".txt")):
            by_base.setdefault(os.path.basename(p), []).append(p)
    own = {os.path.basename(f) for f in glob.glob(os.path.join(ROOT, "**", "*"), recursive=True)}
    bad, checked = [], 0
    for rel in _sources():
        text = open(os.path.join(ROOT, rel), errors="replace").read()
        for m in FULL.finditer(text):
            a, b = int(m.group(2)), int(m.group(3) or m.group(2))
            full = os.path.join(REF, m.group(1))
            checked += 1
            if not os.path.exists(full) or not a <= b <= _lines(full):
                bad.append((rel, m.group(0)))
        for m in BARE.finditer(text):
            cands = by_base.get(m.group(1), [])
            if not cands and m.group(1) in own:
                continue  # a file of this repository
            a, b = int(m.group(2)), int(m.group(3) or m.group(2))
            checked += 1
            if len(cands) != 1 or not a <= b <= _lines(cands[0]):
                bad.append((rel, m.group(0)))
    assert checked > 100
    assert not bad, bad[:20]
